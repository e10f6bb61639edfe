"""Shared helpers for the parity tests (tolerances are the north-star contract)."""
import numpy as np
import torch

import oracle as O

# GEMM outputs vs the fp32 host oracle: relative Frobenius error and
# max|C - R| / max|R| (BASELINE north_star tolerance).
REL_FROB_TOL = 1e-2
NORM_MAX_ABS_TOL = 2e-2


def np_(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().numpy()


def f32(t: torch.Tensor) -> np.ndarray:
    return np_(t.float())


def bits16(t: torch.Tensor) -> np.ndarray:
    return np_(t.view(torch.uint16) if t.dtype in (torch.float16, torch.bfloat16) else t)


def assert_gemm_close(got: np.ndarray, ref: np.ndarray, rel=REL_FROB_TOL, nmax=NORM_MAX_ABS_TOL):
    rf = O.rel_frob(got, ref)
    denom = float(np.abs(ref).max()) or 1.0
    nm = float(np.abs(got.astype(np.float64) - ref).max()) / denom
    assert rf <= rel, f"rel_frob {rf:.3e} > {rel}"
    assert nm <= nmax, f"normalised max_abs {nm:.3e} > {nmax}"
    return rf, nm
