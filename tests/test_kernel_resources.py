"""Build-time guard: the conv kernels keep their accumulator tiles in registers.  A stack frame
or a spill in the FP32 conv mainloop (e.g. from indexing the accumulators with a runtime bound)
costs 30-40% of conv throughput, so it fails here, on the CPU, before any GPU run."""
import re
import shutil
import subprocess
import concurrent.futures as cf

import pytest

from conftest import ROOT

NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"


@pytest.mark.skipif(not shutil.which("nvcc") and not __import__("os").path.exists(NVCC), reason="no nvcc")
def test_conv_kernels_have_no_stack_frame_or_spills(tmp_path):
    srcs = sorted((ROOT / "tensorium_b200" / "csrc").glob("conv_tile_*.cu"))
    assert srcs

    def ptxas(src):
        r = subprocess.run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                            "--fmad=false", "-I", str(ROOT / "include"), "-Xptxas", "-v", "-c", str(src),
                            "-o", str(tmp_path / (src.stem + ".o"))], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
        return r.stderr

    with cf.ThreadPoolExecutor(len(srcs)) as ex:
        logs = list(ex.map(ptxas, srcs))
    checked = 0
    for log in logs:
        blocks = re.split(r"Compiling entry function", log)
        for b in blocks[1:]:
            if "conv_fp32_kernel" not in b.split("\n")[0]:
                continue
            checked += 1
            m = re.search(r"(\d+) bytes stack frame, (\d+) bytes spill stores, (\d+) bytes spill loads", b)
            assert m, b
            assert (int(m.group(1)), int(m.group(2)), int(m.group(3))) == (0, 0, 0), b.split("\n")[0]
    assert checked == 12
