"""The C ABI as a C program sees it: include/fastmka_b200.h compiles as C99
with gcc (no C++ or torch types leak into it), a program links against
libfastmka_b200.so, reads the version string and gets argument errors back as
status codes with messages. Nothing is launched, so no GPU is needed."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_DIR = os.path.join(ROOT, "mka_b200")

SRC = r'''
#include <stdio.h>
#include <string.h>
#include "fastmka_b200.h"

int main(void) {
  const char* v = fmka_version();
  if (v == NULL || strstr(v, "sm_100a") == NULL) return 10;
  char msg[256];
  int rc = fmka_gemm_bf16(NULL, 0, NULL, 0, NULL, NULL, 0, 1, 1, 1, (fmka_stream_t)0);
  if (rc != FMKA_ERR_INVALID_ARGUMENT) return 11;
  if (fmka_get_last_error(msg, (int)sizeof msg) != FMKA_ERR_INVALID_ARGUMENT) return 12;
  if (strstr(msg, "null") == NULL) return 13;
  void* p = NULL;
  if (fmka_peer_alloc(0, &p) != FMKA_ERR_INVALID_ARGUMENT || p != NULL) return 14;
  if (FMKA_PEER_HANDLE_BYTES != 64) return 15;
  printf("ok %s\n", v);
  return 0;
}
'''


def test_header_compiles_as_c_and_links():
    lib = os.path.join(LIB_DIR, "libfastmka_b200.so")
    if not os.path.exists(lib):
        pytest.skip("library not built")
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not found")
    import tempfile

    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "abi.c")
        exe = os.path.join(d, "abi")
        with open(src, "w") as f:
            f.write(SRC)
        subprocess.check_call([gcc, "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), src,
                               "-L", LIB_DIR, "-lfastmka_b200", "-Wl,-rpath," + LIB_DIR, "-o", exe])
        out = subprocess.run([exe], capture_output=True, text=True, timeout=120)
        assert out.returncode == 0, (out.returncode, out.stdout, out.stderr)
        assert out.stdout.startswith("ok")
