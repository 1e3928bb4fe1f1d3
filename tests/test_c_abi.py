"""The C ABI from plain C: ``include/holysht_b200.h`` compiles as C99 and C++17,
and a C program linked against libholysht_b200.so calls the host-only
entries (version, error reporting, the streaming kernel's launch plan) with
no GPU and no Python in between."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
LIB = ROOT / "holysht_b200" / "libholysht_b200.so"

C_PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "holysht_b200.h"

int main(void) {
  int ks = 0, clusters = 0, items = 0;
  if (holysht_version() <= 0) return 1;
  /* RealVectorSHT 512x1024 batch 4, forward, planned for 148 SMs */
  if (holysht_stream_launch_plan(HOLYSHT_KIND_VECTOR, HOLYSHT_DIR_FORWARD, 4, 512, 512, 513, 513, 0, 0, 148,
                                 &ks, &clusters, &items) != HOLYSHT_OK) return 2;
  printf("plan %d %d %d\n", ks, clusters, items);
  /* an invalid call reports through the status and the message */
  if (holysht_stream_launch_plan(HOLYSHT_KIND_REAL, HOLYSHT_DIR_FORWARD, 4, 512, 512, 513, 513, 0, 0, 148,
                                 &ks, &clusters, &items) != HOLYSHT_ERR_INVALID) return 3;
  if (strlen(holysht_last_error()) == 0) return 4;
  printf("error %s\n", holysht_last_error());
  return 0;
}
"""


@pytest.fixture(scope="module")
def library():
    if not LIB.exists():
        from holysht_b200 import build

        build.build()
    return LIB


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_c_program_links_and_calls_the_library(tmp_path, library):
    src = tmp_path / "abi.c"
    src.write_text(C_PROGRAM)
    exe = tmp_path / "abi"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", str(ROOT / "include"), str(src), "-o", str(exe),
                    "-L", str(library.parent), "-lholysht_b200", f"-Wl,-rpath,{library.parent}"],
                   check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    assert "plan 2 72 72" in out
    assert "error " in out and "SCALAR and VECTOR" in out


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ not available")
def test_header_compiles_as_cpp(tmp_path):
    src = tmp_path / "abi.cpp"
    src.write_text('#include "holysht_b200.h"\nint main() { return holysht_version() > 0 ? 0 : 1; }\n')
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Werror", "-fsyntax-only", "-I", str(ROOT / "include"), str(src)],
                   check=True, capture_output=True, text=True)
