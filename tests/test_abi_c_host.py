"""The C ABI from a C (and a C++) host: ``include/b200_optim.h`` compiles as strict C11 and C++17,
and a program linked against the library plans chunks and gets argument errors -- the calls an
FFI host makes before it owns any device memory, so no GPU is needed."""

from __future__ import annotations

import shutil
import subprocess

import pytest

from minigpt_train_infra_b200 import _build

PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "b200_optim.h"

int main(void) {
  if (b2o_abi_version() != B2O_ABI_VERSION) return 10;
  if (strcmp(b2o_status_string(B2O_OK), "ok") != 0) return 11;

  /* three tensors: 1000 elements, 0 elements, 17 elements; fake 16-byte-aligned addresses */
  b2o_tensor t[3];
  memset(t, 0, sizeof t);
  const int64_t n[3] = {1000, 0, 17};
  for (int i = 0; i < 3; ++i) {
    void* a = (void*)(uintptr_t)(0x100000 + 0x10000 * i);
    t[i].grad = a; t[i].param = a; t[i].master = (float*)a;
    t[i].exp_avg = (float*)a; t[i].exp_avg_sq = (float*)a;
    t[i].numel = n[i]; t[i].group = i % 2; t[i].slot = i;
  }
  int64_t count = 0;
  if (b2o_plan_chunks(t, 3, 2, 3, 256, B2O_BF16, NULL, 0, &count) != B2O_OK) return 12;
  if (count != 4 + 0 + 1) return 13;
  b2o_chunk c[5];
  if (b2o_plan_chunks(t, 3, 2, 3, 256, B2O_BF16, c, 5, &count) != B2O_OK) return 14;
  if (c[3].tensor != 0 || c[3].begin != 768 || c[3].end != 1000) return 15;
  if (c[4].tensor != 2 || c[4].end != 17) return 16;
  if (t[0].chunk_count != 4 || t[2].chunk_begin != 4 || !(t[0].flags & B2O_FLAG_VECTOR)) return 17;
  if (b2o_plan_chunks(t, 3, 2, 3, 256, B2O_BF16, c, 4, &count) != B2O_ERR_CAPACITY) return 18;
  if (b2o_workspace_bytes(5, 3) != 64 + 8 * 5 + 8 * 4) return 19;
  /* launching entry points check their arguments before touching CUDA */
  if (b2o_grad_stats(NULL, 0, NULL, 0, 0, 0, NULL, NULL, NULL, 0, NULL, NULL, NULL) != B2O_ERR_ARG)
    return 20;
  if (b2o_scaler_update(NULL, NULL, NULL, 2.0, 0.5, 2000, NULL) != B2O_ERR_ARG) return 21;
  printf("c host ok\n");
  return 0;
}
"""


@pytest.mark.parametrize("lang", ["c", "c++"])
def test_header_and_library_from_a_native_host(tmp_path, lang):
    cc = shutil.which("gcc" if lang == "c" else "g++")
    if cc is None:
        pytest.skip(f"no {lang} compiler")
    lib = _build.build()
    src = tmp_path / ("host.c" if lang == "c" else "host.cpp")
    src.write_text(PROGRAM)
    exe = tmp_path / "host"
    std = ["-std=c11"] if lang == "c" else ["-std=c++17"]
    cmd = [cc, *std, "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", str(_build.INCLUDE),
           str(src), "-o", str(exe), "-L", str(lib.parent), "-lb200_optim",
           f"-Wl,-rpath,{lib.parent}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, (run.returncode, run.stdout, run.stderr)
    assert "c host ok" in run.stdout
