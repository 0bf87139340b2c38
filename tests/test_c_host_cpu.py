"""The C ABI from a plain C host: a C99 program that includes
include/fdl_kvcache.h, links libfdl_b200.so and calls entry points whose
argument checks return before any device work (no GPU needed).  This is the
binding a non-Python host of the reference would use."""
import shutil
import subprocess
from pathlib import Path

import pytest

from fast_v2_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]

PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "fdl_kvcache.h"

int main(void) {
  const char* v = fdl_version();
  if (strncmp(v, "fdl_b200", 8) != 0) return 10;
  void* bufs[2] = {(void*)0x1000, (void*)0x2000};
  /* nothing kept: nothing to move, pointers not looked at */
  if (fdl_kv_compact(NULL, 2, 64, 64, 4, NULL, 0, NULL) != FDL_OK) return 11;
  /* more kept rows than slots */
  if (fdl_kv_compact(bufs, 2, 64, 64, 4, (const int64_t*)0x3000, 5, NULL) != FDL_E_SHAPE) return 12;
  /* a block of 33 tokens is not supported by the selection kernels */
  if (fdl_focus_select((void*)0x1000, 33, (const uint8_t*)0x1000, 33, NULL, 0, 2, 33, 4, FDL_BF16,
                       (int64_t*)0x1000, 33, (int32_t*)0x1000, NULL) != FDL_E_SHAPE) return 13;
  /* head dim 64 is not a supported attention configuration */
  if (fdl_block_attn((void*)0x1000, (void*)0x1000, (void*)0x1000, (const int32_t*)0x1000, 64, NULL, NULL, 0,
                     NULL, 0, (void*)0x1000, 1, 32, 28, 4, 64, 0.125f, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0,
                     0, NULL, 0, NULL) != FDL_E_UNSUPPORTED) return 14;
  printf("%s\n", v);
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not installed")
def test_plain_c_host_links_and_calls_the_abi(tmp_path):
    lib = _lib.LIB_ABI
    assert lib.exists(), "build the library first (python fast_v2_b200/build.py)"
    src = tmp_path / "host.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "host"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-pedantic", f"-I{ROOT / 'include'}", str(src),
                    str(lib), f"-Wl,-rpath,{lib.parent}", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, (out.returncode, out.stderr)
    assert out.stdout.startswith("fdl_b200")
