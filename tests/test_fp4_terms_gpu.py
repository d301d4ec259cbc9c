"""The device quantizer of the FP4 expert GEMMs (airllm_b200/csrc/fp4_terms.cuh:
five block-scaled E2M1 terms per value) against its CPU definition,
oracle_e2m1_terms, byte for byte: codes and E8M0 scale bytes, with 1, 2, 4 and 16
lanes sharing a 32-element block (the layouts the kernels use).  Inputs cover many binades, exact ties on the E2M1 grid, negative
values that round to zero (code 0, never the negative zero 8), all-zero and
subnormal blocks and the scale threshold at 6 * 2^e.  A block holding a NaN or an
infinity gets the E8M0 NaN scale on its first term (tests/cuda/fp4_terms_check.cu)."""
import os
import subprocess

import numpy as np
import pytest

import oracle

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "airllm_b200", "csrc")
TERMS = 5
LANES = (1, 2, 4, 16)


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("fp4") / "fp4_terms_check")
    subprocess.run(["/usr/local/cuda/bin/nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-I", CSRC,
                    "-o", exe, os.path.join(HERE, "cuda", "fp4_terms_check.cu")], check=True)
    return exe


def _inputs():
    r = np.random.default_rng(5)
    blocks = [(r.standard_normal((4096, 32)) * np.exp(r.normal(0, 3, (4096, 1)))).astype(np.float32)]
    grid_ties = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0], np.float32)
    for k in (-20, -3, 0, 4, 17):
        b = np.zeros((4, 32), np.float32)
        b[:, :8] = grid_ties * np.float32(2.0 ** k)
        b[:, 8:16] = -grid_ties * np.float32(2.0 ** k)
        b[:, 16:24] = -np.float32(0.1 * 2.0 ** k)  # rounds to zero on the first term
        b[1] *= np.float32(1.0000001)
        b[2, 0] = np.float32(6.0000005 * 2.0 ** k)  # just above the 6 * 2^e threshold
        b[3, 0] = np.float32(1.5 * 2.0 ** k)
        blocks.append(b)
    z = np.zeros((3, 32), np.float32)
    z[1, 3] = np.float32(1e-39)  # subnormal block maximum
    z[2, :] = np.float32(-3e-41)
    blocks.append(z)
    blocks.append((r.standard_normal((2, 32)) * 1e37).astype(np.float32))
    return np.concatenate(blocks).ravel()


def _run(checker, tmp_path, x):
    src = tmp_path / "x.f32"
    x.astype(np.float32).tofile(src)
    outs = [tmp_path / f"l{lanes}.bin" for lanes in LANES]
    p = subprocess.run([checker, str(src), *map(str, outs)], capture_output=True, text=True, timeout=120)
    assert p.returncode == 0, p.stdout + p.stderr
    n = x.size
    res = []
    for o in outs:
        raw = np.fromfile(o, np.uint8)
        res.append((raw[:TERMS * n // 2].reshape(TERMS, n // 2), raw[TERMS * n // 2:].reshape(TERMS, n // 32)))
    return res


@pytest.mark.gpu
def test_device_terms_equal_the_cpu_definition_byte_for_byte(cuda_device, checker, tmp_path):
    x = _inputs()
    want_codes, want_scales = oracle.e2m1_terms(x, TERMS)
    for lanes, (codes, scales) in zip(LANES, _run(checker, tmp_path, x)):
        bad_c = np.nonzero((codes != want_codes).any(axis=0))[0]
        bad_s = np.nonzero((scales != want_scales).any(axis=0))[0]
        assert not len(bad_s), f"{lanes} lane(s): scale bytes differ in blocks {bad_s[:8]}"
        assert not len(bad_c), f"{lanes} lane(s): codes differ at bytes {bad_c[:8]}"
        assert not ((codes & 0x0F) == 8).any() and not ((codes >> 4) == 8).any()  # no negative zero


@pytest.mark.gpu
def test_nan_or_infinite_blocks_get_the_nan_scale(cuda_device, checker, tmp_path):
    x = np.ones((3, 32), np.float32)
    x[0, 5] = np.nan
    x[1, 31] = -np.inf
    want_codes, want_scales = oracle.e2m1_terms(x[2], TERMS)  # the clean block as the CPU definition has it
    for codes, scales in _run(checker, tmp_path, x.ravel()):
        assert scales[0, 0] == 0xFF and scales[0, 1] == 0xFF
        assert np.array_equal(scales[:, 2], want_scales[:, 0]) and np.array_equal(codes[:, 32:], want_codes)
