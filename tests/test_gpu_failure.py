"""Failure detection without a GPU fault.

The streaming kernel's pipeline waits are bounded: a wait that runs out sets
bit 0 of the device error word (``holysht_stream_error_word``), the CTA skips
the rest of its reduction and the kernel still finishes, leaving the CUDA
context usable.  The test makes one wait run out on purpose through the test
hook ``HOLYSHT_TEST_STALL_CHUNK`` (warp 0 of the first CTA never requests that
table stage: a flag that nothing sets), in a child process so the read-once
hook does not leak into other tests, and checks the status, then runs a normal
contraction in the same context.  Nothing traps, faults or hangs.
"""
import os
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]

CHILD = textwrap.dedent("""
    import numpy as np, torch
    from holysht_b200 import _lib, ops
    from oracle import sht_oracle as orc
    dev = "cuda"
    rng = np.random.default_rng(0)
    B, K, L, M = 2, 64, 48, 49
    w = rng.standard_normal((L, K, M)).astype(np.float32)
    w *= (np.arange(M)[None, None, :] <= np.arange(L)[:, None, None])
    x = (rng.standard_normal((B, K, M)) + 1j * rng.standard_normal((B, K, M))).astype(np.complex64)
    wt, xt = torch.from_numpy(w).to(dev), torch.from_numpy(x).to(dev)
    out = torch.empty((B, L, M), dtype=torch.complex64, device=dev)
    kw = dict(kind=_lib.KIND_SCALAR, direction=_lib.DIR_FORWARD, input=xt, output=out, batch=B, nlat=K, lmax=L,
              mmax=M, in_strides=(K * M, 0, M), out_strides=(L * M, 0, M), out_cols=M)
    ops.legendre_contract(w0=ops.group_table8(wt, _lib.DIR_FORWARD), grouped8=True, **kw)
    torch.cuda.synchronize()                  # returns: the wait gave up instead of hanging
    word = ops.stream_error_word()
    assert word & 1, word
    assert ops.stream_error_word() == 0       # read and cleared
    # the context is still usable: the 4-row kernel (no test hook) gives the right answer
    ops.legendre_contract(w0=ops.group_table(wt, _lib.DIR_FORWARD), grouped=True, **kw)
    ref = orc.legendre_forward(x.astype(np.complex128), w.astype(np.float64))
    got = out.cpu().numpy().astype(np.complex128)
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-6
    print("OK")
""")


def test_stream_wait_timeout_sets_the_error_word_and_returns():
    env = dict(os.environ, HOLYSHT_TEST_STALL_CHUNK="1", PYTHONPATH=str(ROOT))
    res = subprocess.run([sys.executable, "-c", CHILD], cwd=ROOT, env=env, capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0 and "OK" in res.stdout, res.stdout + res.stderr
