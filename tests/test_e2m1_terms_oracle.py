"""The bit-exact definition of block-scaled FP4 activation terms (oracle_e2m1_terms),
the operand a block-scaled FP4 (mxf4) expert GEMM would take: per 32 elements, term
j rounds the remainder of the previous terms to nearest (ties to the even mantissa)
on the E2M1 grid, saturated at +-6, at the smallest power-of-two scale that fits the
remainder's maximum.  A GPU quantizer is to match these bytes exactly."""
import numpy as np
import pytest

import oracle
from test_fp4_term_numerics import e2m1_terms as numpy_terms


def _block(vals):
    x = np.zeros(32, np.float32)
    x[:len(vals)] = vals
    return x


def test_round_to_nearest_even_on_the_grid_and_saturation():
    # amax 6 -> scale 2^0; ties go to the code with the even mantissa bit
    vals = [6, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5, -0.25, -0.75, 0.3, 2.9]
    codes, scales = oracle.e2m1_terms(_block(vals), 1)
    assert scales[0, 0] == 127
    nib = np.stack([codes[0] & 15, codes[0] >> 4], -1).ravel()
    want = [7, 0, 2, 2, 4, 4, 6, 6, 0, 8 | 2, 1, 5]
    assert list(nib[:len(want)]) == want
    assert not nib[len(want):].any()


@pytest.mark.parametrize("amax,scale_byte", [(6.0, 127), (7.0, 128), (3.0, 126), (6.5, 128), (0.75, 124),
                                              (1e-39, 0), (0.0, 127)])
def test_smallest_power_of_two_scale_that_fits(amax, scale_byte):
    codes, scales = oracle.e2m1_terms(_block([amax, -amax / 3]), 1)
    assert scales[0, 0] == scale_byte


def test_terms_shrink_the_error_and_match_the_numpy_scheme():
    r = np.random.default_rng(1)
    x = (r.standard_normal(32 * 64) * np.exp(r.normal(0, 2, 64)).repeat(32)).astype(np.float32)
    amax = np.abs(x.reshape(-1, 32)).max(1).repeat(32)
    prev = np.inf
    for n in (1, 3, 5, 6):
        codes, scales = oracle.e2m1_terms(x, n)
        recon = oracle.e2m1_reconstruct(codes, scales)
        err = float(np.max(np.abs(recon - x) / amax))
        assert err < prev
        prev = err
        # the numpy restatement behind the tolerance evidence keeps float64 remainders and
        # breaks ties toward the lower grid value; later terms round remainders that can sit
        # exactly on a tie, so the two agree to within one term's rounding, not bitwise
        ref = numpy_terms(x, n)
        err_np = float(np.max(np.abs(ref - x) / amax))
        assert err <= 2 * err_np and err_np <= 2 * err
        assert float(np.max(np.abs(recon - ref) / amax)) <= 2 * max(err, err_np)
    assert prev < 2e-4


def test_rejects_bad_arguments():
    with pytest.raises(oracle.OracleError):
        oracle.e2m1_terms(np.zeros(31, np.float32), 2)
    with pytest.raises(oracle.OracleError):
        oracle.e2m1_terms(_block([np.inf]), 2)
