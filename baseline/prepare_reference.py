"""Stage the unmodified reference package and its CUDA extension in ``baseline/_ref``.

    python baseline/prepare_reference.py <reference checkout>

The reference (chrisvoncsefalvay/holysht) has no setup.py or pyproject.toml,
so ``pip install --target baseline/_ref`` refuses it.  This script does what
that install would have done, without changing any reference file:

* copies ``torch-ext/`` and ``cuda/`` of the checkout into ``baseline/_ref/``
  (the layout the reference's own JIT loader ``torch-ext/holysht/_jit_ops.py``
  expects: repository root two levels above the package);
* compiles the reference's CUDA extension (``torch-ext/torch_binding.cpp``,
  ``cuda/fused_legendre.cu``, ``cuda/fused_sht.cu``) for sm_100a with the
  flags of ``_jit_ops.py:_cuda_flags`` (``-O3 -lineinfo -Xptxas=-warn-spills
  --expt-relaxed-constexpr --use_fast_math``) through
  ``torch.utils.cpp_extension`` into ``baseline/_ref/build/``, cross-compiling
  without a GPU, so the GPU box does not spend minutes on a JIT build;
* writes ``baseline/_ref/torch-ext/holysht/_ops.py``, the module a packaged
  (kernel-builder) build provides and the reference imports first
  (``__init__.py:37-38``): it loads the prebuilt library and exposes
  ``torch.ops.holysht_ops_cuda``.

``baseline/_ref`` is git-ignored (it is the reference's code and a build
product, not this project's source) and travels to the GPU box with the
working tree.  ``baseline/reference_cuda.py`` times it there.
"""
from __future__ import annotations

import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF = HERE / "_ref"
EXT_NAME = "holysht_ops_cuda"

OPS_PY = '''"""Packaged-build ops module: loads the prebuilt CUDA extension.
Written by baseline/prepare_reference.py (not part of the reference checkout)."""
from pathlib import Path

import torch

_LIB = Path(__file__).resolve().parents[2] / "build" / "{name}.so"
torch.ops.load_library(str(_LIB))
ops = getattr(torch.ops, "{name}")
'''


def main(argv):
    if len(argv) != 2:
        raise SystemExit(__doc__)
    src = Path(argv[1]).resolve()
    if not (src / "torch-ext" / "holysht" / "__init__.py").exists():
        raise SystemExit(f"{src} is not a holysht checkout")
    if REF.exists():
        shutil.rmtree(REF)
    REF.mkdir(parents=True)
    for d in ("torch-ext", "cuda"):
        shutil.copytree(src / d, REF / d)
    build = REF / "build"
    build.mkdir()

    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    os.environ.setdefault("MAX_JOBS", "4")
    from torch.utils import cpp_extension

    flags = ["-O3", "-lineinfo", "-Xptxas=-warn-spills", "--expt-relaxed-constexpr", "--use_fast_math"]
    try:
        cpp_extension.load(
            name=EXT_NAME,
            sources=[str(REF / "torch-ext" / "torch_binding.cpp"), str(REF / "cuda" / "fused_legendre.cu"),
                     str(REF / "cuda" / "fused_sht.cu")],
            extra_include_paths=[str(REF / "torch-ext")],
            extra_cflags=["-O3", "-std=c++17"],
            extra_cuda_cflags=flags,
            extra_ldflags=["-L/usr/local/cuda/lib64/stubs", "-lcuda"],
            build_directory=str(build),
            verbose=False,
            with_cuda=True,
            is_python_module=False,
        )
    except OSError as exc:  # built, but this machine has no CUDA driver to load it
        print(f"built (not loadable here: {exc.__class__.__name__})")
    so = build / f"{EXT_NAME}.so"
    if not so.exists():
        raise SystemExit("the reference extension did not build")
    (REF / "torch-ext" / "holysht" / "_ops.py").write_text(OPS_PY.format(name=EXT_NAME))
    print(so)


if __name__ == "__main__":
    main(sys.argv)
