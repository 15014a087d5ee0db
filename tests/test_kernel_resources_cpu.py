"""The streaming kernels keep four CTAs of 256 threads resident per SM.

Both passes of the step are sized for that occupancy: 4 x 256 threads x 64 registers fill an
SM's 65,536 registers, and each CTA's static shared memory must leave room for three more on the
228 KB of a B200 SM (1 KB of each CTA's share is reserved by the hardware).  The grid is taken
from the occupancy calculator at run time, so a kernel that grew past either limit would still
run, only with a smaller grid and fewer loads in flight -- a silent slowdown.  This test compiles
the two kernel sources for sm_100a with ``-Xptxas -v`` (no GPU needed) and checks every
statistics and update kernel against both limits.
"""

from __future__ import annotations

import re
import shutil
import subprocess
from pathlib import Path

import pytest

from minigpt_train_infra_b200 import _build

MAX_REGISTERS = 64
MAX_SMEM_BYTES = 228 * 1024 // 4 - 1024   # static shared memory per CTA at 4 CTAs per SM
KERNELS = ("grad_stats_kernel", "rs_stats_kernel", "adamw_kernel")

_ENTRY = re.compile(r"Compiling entry function '([^']+)'")
_USED = re.compile(r"Used (\d+) registers.*?(\d+) bytes smem")


_NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"


def _resources(source: str, tmp_path) -> dict:
    nvcc = _NVCC
    cmd = [nvcc, *_build.ARCH, *_build.NVCC_FLAGS, "-Xptxas", "-v", "-I", str(_build.INCLUDE),
           "-I", str(_build.CSRC), "-c", str(_build.CSRC / source), "-o", str(tmp_path / "k.o")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr[-2000:]
    found, entry = {}, None
    for line in res.stderr.splitlines():
        m = _ENTRY.search(line)
        if m:
            entry = m.group(1)
            continue
        m = _USED.search(line)
        if m and entry is not None:
            found[entry] = (int(m.group(1)), int(m.group(2)))
            entry = None
    return found


@pytest.mark.skipif(not Path(_NVCC).exists(), reason="needs nvcc")
@pytest.mark.parametrize("source", ["b2o_stats.cu", "b2o_adamw.cu"])
def test_streaming_kernels_fit_four_ctas_per_sm(source, tmp_path):
    found = _resources(source, tmp_path)
    streaming = {name: v for name, v in found.items() if any(k in name for k in KERNELS)}
    assert streaming, f"no streaming kernel found in the ptxas report of {source}"
    for name, (regs, smem) in streaming.items():
        assert regs <= MAX_REGISTERS, (name, regs)
        assert smem <= MAX_SMEM_BYTES, (name, smem)
