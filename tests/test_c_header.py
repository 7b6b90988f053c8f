"""The boundary is plain C: include/orca_cuda.h compiles as strict C99 and as
C++17 with warnings as errors, and a C program linked against
liborca_cuda.so calls it the way a cgo / Rust / JNI binding would -- only
entry points that answer without a GPU (version, status strings, argument
checks that fail before any device call)."""
import os
import shutil
import subprocess

import pytest

from orcaml_b200 import _lib as L

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(REPO, "include")

PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "orca_cuda.h"

#define EXPECT(cond) do { if (!(cond)) { printf("FAILED: %s\n", #cond); return 1; } } while (0)

int main(void) {
  void* host = NULL;
  float loss = 0.0f;
  EXPECT(orca_version() >= 0x000100u);
  EXPECT(strcmp(orca_status_string(ORCA_OK), "ok") == 0);
  EXPECT(strcmp(orca_status_string(ORCA_TIMEOUT), "timeout") == 0);
  EXPECT(orca_ctx_set_timeout(NULL, 1.0) == ORCA_INVALID_ARGUMENT);
  EXPECT(orca_ctx_sync(NULL, 1.0) == ORCA_INVALID_ARGUMENT);
  EXPECT(strlen(orca_last_error()) > 0);
  EXPECT(orca_mlp_create(NULL, NULL, NULL) == ORCA_INVALID_ARGUMENT);
  EXPECT(orca_mlp_step(NULL, NULL, NULL, &loss) == ORCA_INVALID_ARGUMENT);
  EXPECT(orca_mlp_stage_batch(NULL, 0, NULL, NULL) == ORCA_INVALID_ARGUMENT);
  EXPECT(orca_mlp_step_staged(NULL, 0, &loss) == ORCA_INVALID_ARGUMENT);
  EXPECT(orca_host_alloc(0, &host) == ORCA_INVALID_ARGUMENT && host == NULL);
  EXPECT(orca_host_free(NULL) == ORCA_OK);
  EXPECT(orca_buf_release(NULL) == ORCA_OK);
  EXPECT(orca_buf_len(NULL) == 0);
  EXPECT(orca_buf_device_ptr(NULL) == NULL);
  EXPECT(orca_mlp_destroy(NULL) == ORCA_OK);
  EXPECT(ORCA_MLP_STAGE_SLOTS == 2 && ORCA_COMM_ID_BYTES == 128);
  printf("ok\n");
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None or shutil.which("g++") is None,
                    reason="needs gcc and g++")
def test_header_is_c99_and_cxx17_and_links(tmp_path):
    src = tmp_path / "use_abi.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "use_abi"
    libdir = os.path.dirname(L.LIB_PATH)
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", INCLUDE,
                    str(src), "-o", str(exe), "-L", libdir, "-l:liborca_cuda.so",
                    f"-Wl,-rpath,{libdir}"], check=True, capture_output=True)
    cxx = tmp_path / "header.cpp"
    cxx.write_text('#include "orca_cuda.h"\nint main() { return orca_version() == 0; }\n')
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", INCLUDE,
                    "-fsyntax-only", str(cxx)], check=True, capture_output=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert out.stdout.strip().endswith("ok")
