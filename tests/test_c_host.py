"""The C ABI from C: include/gqa_sm100.h compiles as C99 and a C program linked
against libgqa_sm100.so calls its host-only entry points (no GPU) — what an FFI
host (cgo, JNI, a C++ engine) would do."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "gqa_sm100.h"

int main(void) {
  int plan[5];
  if (gqa_version() <= 0) return 1;
  if (strlen(gqa_strerror(GQA_ERR_UNSUPPORTED)) == 0) return 2;
  /* config 4 on 148 SMs: 256 whole units, head-major order */
  if (gqa_prefill_plan(4, 32, 8, 512, 16384, 128, 1, 148, plan) != GQA_OK) return 3;
  if (plan[0] != 256 || plan[1] != 1 || plan[3] != 1 || plan[4] != 256) return 4;
  /* 64 units on 148 SMs: the key axis split two ways */
  if (gqa_prefill_plan(1, 32, 8, 512, 16384, 128, 1, 148, plan) != GQA_OK) return 5;
  if (plan[1] != 2 || plan[4] != 128) return 6;
  /* argument errors come back as status codes, before any CUDA call */
  if (gqa_prefill_plan(1, 32, 8, 512, 512, 96, 1, 148, plan) != GQA_ERR_UNSUPPORTED) return 7;
  if (gqa_prefill_plan(1, 30, 8, 512, 512, 128, 1, 148, plan) != GQA_ERR_INVALID_ARG) return 8;
  printf("ok\n");
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_c_program_links_and_calls_host_entry_points(lib_path, tmp_path):
    src = tmp_path / "abi.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "abi"
    libdir = os.path.dirname(lib_path)
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src),
                    "-L", libdir, "-l:" + os.path.basename(lib_path), "-Wl,-rpath," + libdir, "-o", str(exe)],
                   check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0 and out.stdout.strip() == "ok", (out.returncode, out.stdout, out.stderr)
