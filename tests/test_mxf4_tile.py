"""Known-answer test of the block-scaled FP4 MMA form (tcgen05 kind::mxf4 with packed
E2M1 operands and E8M0 scales per 32 elements) on one tile, against a float64 CPU
product (tests/cuda/mxf4_tile.cu).  It pins the operand layout (64-byte swizzled
K-major rows, the layout the MXFP4 box planes already have) and the scale-factor
addressing an FP4 expert GEMM would use."""
import os
import re
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def tile_binary(tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("mxf4") / "mxf4_tile")
    subprocess.run(["/usr/local/cuda/bin/nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-o", exe,
                    os.path.join(HERE, "cuda", "mxf4_tile.cu"), "-lcuda"], check=True)
    return exe


@pytest.mark.gpu
@pytest.mark.parametrize("n", [8, 16])
def test_mxf4_tile_matches_cpu_product(cuda_device, tile_binary, n):
    out = subprocess.run([tile_binary, str(n), "0", "2"], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    m = re.search(r"err (\d+) max scaled err ([0-9.e+-]+)", out.stdout)
    assert m, out.stdout
    assert int(m.group(1)) == 0 and float(m.group(2)) < 1e-5, out.stdout
