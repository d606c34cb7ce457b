"""include/bolt3.h from a C or C++ host: one program compiled as C99 (gcc) and as C++17 (g++)
against the header, pedantic with warnings as errors, and linked to libbolt3.so. The compiler's
struct layouts must equal the library's (bolt3_args_size), the ABI version must match the
header's, and the entry points must reject null arguments with BOLT3_ERR_ARG (no GPU needed: they
return before any CUDA call)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "vsa_lm_b200")

C_SOURCE = r"""
#include <stdio.h>
#include "bolt3.h"

int main(void) {
  const size_t mine[] = {sizeof(bolt3_prep_args), sizeof(bolt3_consolidate_args), sizeof(bolt3_attend_args),
                         sizeof(bolt3_prefill_args), sizeof(bolt3_anchor_args), sizeof(bolt3_rmsnorm_args),
                         sizeof(bolt3_silu_mul_args)};
  int bad = 0;
  for (int i = 0; i < (int)(sizeof(mine) / sizeof(mine[0])); ++i) {
    if (bolt3_args_size(i) != mine[i]) {
      printf("struct %d: %zu in C, %zu in the library\n", i, mine[i], bolt3_args_size(i));
      bad = 1;
    }
  }
  if (bolt3_abi_version() != BOLT3_ABI_VERSION) {
    printf("abi %d, header %d\n", bolt3_abi_version(), BOLT3_ABI_VERSION);
    bad = 1;
  }
  const int rc[] = {bolt3_prep(NULL, NULL), bolt3_consolidate(NULL, NULL), bolt3_attend(NULL, NULL),
                    bolt3_prefill_fwd(NULL, NULL), bolt3_prefill_fwd_noalloc(NULL, NULL),
                    bolt3_anchor_decode(NULL, NULL), bolt3_rmsnorm(NULL, NULL), bolt3_silu_mul(NULL, NULL)};
  for (int i = 0; i < (int)(sizeof(rc) / sizeof(rc[0])); ++i) {
    if (rc[i] != BOLT3_ERR_ARG) {
      printf("entry point %d returned %d for null arguments: %s\n", i, rc[i], bolt3_status_string(rc[i]));
      bad = 1;
    }
  }
  if (bolt3_prefill_workspace_size(64, 8192, 128) == 0 || bolt3_prefill_workspace_size(1, 128, 96) != 0) {
    printf("workspace size\n");
    bad = 1;
  }
  printf(bad ? "FAIL\n" : "OK\n");
  return bad;
}
"""


@pytest.mark.parametrize("compiler,std,suffix", [("gcc", "-std=c99", "c"), ("g++", "-std=c++17", "cpp")])
def test_header_compiles_and_matches_the_library(tmp_path, compiler, std, suffix):
    if shutil.which(compiler) is None:
        pytest.skip(f"{compiler} is not here")
    from vsa_lm_b200 import _lib

    _lib.load()                                   # builds the library if it is missing
    src = tmp_path / f"host.{suffix}"
    src.write_text(C_SOURCE)
    exe = tmp_path / "host"
    subprocess.check_call([compiler, std, "-Wall", "-Wextra", "-pedantic", "-Werror", "-I",
                           os.path.join(ROOT, "include"), str(src), "-L", LIBDIR, "-lbolt3",
                           f"-Wl,-rpath,{LIBDIR}", "-o", str(exe)])
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip().endswith("OK"), r.stdout + r.stderr
