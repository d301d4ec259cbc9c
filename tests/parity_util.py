"""Parity criteria between the CUDA path and the oracle.

  - top-k expert indices identical, except rows whose differing choice is a tie
    in the oracle's float32 logits to within 1e-6;
  - the token->expert permutation identical;
  - block outputs within max-abs 2e-2 and relative L2 1e-3.
"""
import numpy as np

MAX_ABS = 2e-2
REL_L2 = 1e-3
TIE = 1e-6


def routing_mismatches(gpu_idx, ref_idx, ref_logits):
    """Rows whose top-k differs.  Returns (tie_rows, bad_rows)."""
    gpu_idx, ref_idx = np.asarray(gpu_idx), np.asarray(ref_idx)
    rows = np.nonzero((gpu_idx != ref_idx).any(axis=1))[0]
    ties, bad = [], []
    for t in rows:
        a = np.sort(ref_logits[t][gpu_idx[t]].astype(np.float64))
        b = np.sort(ref_logits[t][ref_idx[t]].astype(np.float64))
        (ties if np.all(np.abs(a - b) < TIE) else bad).append(int(t))
    return ties, bad


def output_errors(gpu_out, ref_out):
    d = gpu_out.astype(np.float64) - ref_out.astype(np.float64)
    max_abs = float(np.max(np.abs(d))) if d.size else 0.0
    rel = float(np.linalg.norm(d) / max(np.linalg.norm(ref_out.astype(np.float64)), 1e-30))
    return max_abs, rel


def assert_block_parity(gpu_out, ref_out, rows=None):
    if rows is not None:
        gpu_out, ref_out = gpu_out[rows], ref_out[rows]
    assert np.isfinite(gpu_out).all(), "non-finite GPU output"
    max_abs, rel = output_errors(gpu_out, ref_out)
    assert max_abs <= MAX_ABS and rel <= REL_L2, f"max-abs {max_abs:.3e}, rel-L2 {rel:.3e}"
    return max_abs, rel
