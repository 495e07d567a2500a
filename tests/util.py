"""Helpers shared by the tests (tolerances are stated where they are used)."""
from __future__ import annotations

import numpy as np
import torch

requires_cuda = None  # set by conftest-like import below


def max_rel_err(out: np.ndarray, ref: np.ndarray) -> float:
    """max |out - ref| / max |ref|: the 16-bit tolerance metric (bar 2e-2).

    Normalised by the largest reference magnitude.  An element-wise ratio (even floored at
    1e-3 * max|ref|) is not usable for a 16-bit layer: one-ulp rounding flips of stored
    intermediates dominate near-zero outputs, and the reference's own bf16 torch path
    scores > 1 on it (tests/test_oracle_golden.py::test_reference_bf16_path_metric)."""
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    if ref.size == 0:
        return 0.0
    return float(np.abs(out - ref).max() / max(np.abs(ref).max(), 1e-30))


def elementwise_rel_err(out, ref, floor=1e-3) -> float:
    """max |out-ref| / max(|ref|, floor * max|ref|) (reported for information only)."""
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    if ref.size == 0:
        return 0.0
    den = np.maximum(np.abs(ref), floor * np.abs(ref).max() + 1e-30)
    return float((np.abs(out - ref) / den).max())


def max_abs_err(out, ref) -> float:
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(out - ref).max()) if ref.size else 0.0


def to_dev(a, dtype=torch.float32, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device=device, dtype=dtype)


def rounded(a: np.ndarray, dtype: torch.dtype) -> np.ndarray:
    """Round float32 values through ``dtype`` (the compute dtype) back to float32."""
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dtype).float().numpy()


def routing_matches_up_to_ties(idx, ref_idx, logits, rtol=1e-5):
    """Rows whose selected expert SETS differ must be near-ties in the oracle logits."""
    idx = np.asarray(idx)
    ref_idx = np.asarray(ref_idx)
    bad = []
    for r in np.where((np.sort(idx, 1) != np.sort(ref_idx, 1)).any(1))[0]:
        lg = logits[r]
        a = np.sort(lg[idx[r]])
        b = np.sort(lg[ref_idx[r]])
        scale = np.abs(lg).max() + 1e-30
        if np.abs(a - b).max() > rtol * scale:
            bad.append(int(r))
    return bad
