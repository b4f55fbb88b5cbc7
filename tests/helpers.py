"""Test helpers: seeded modules built from oracle streams, and their references."""

from __future__ import annotations

import numpy as np
import torch

import oracle
from mlx_iqk_b200 import IqkSwitchLinear
from mlx_iqk_b200.format import component_shapes


def stacked(member: str, streams: dict, experts: int, out_features: int, n: int) -> dict:
    shapes = component_shapes(member, experts, out_features, n)
    return {k: np.ascontiguousarray(v).reshape(shapes[k]) for k, v in streams.items()}


def make_module(member: str, n: int, seed: int, experts: int = 8, out_features: int = 32,
                scales: str = "serving", device="cuda", wire: np.ndarray | None = None):
    """Module loaded with seeded random wire, plus the float32 CPU reference weights."""
    rows = experts * out_features
    if wire is None:
        wire = oracle.random_wire(member, rows, n, seed=seed, scales=scales)
    streams = oracle.pack(member, wire, n)
    ref = oracle.decode(member, streams, n).reshape(experts, out_features, n)
    mod = IqkSwitchLinear(member, experts, out_features, n, device=device)
    mod.load_streams(stacked(member, streams, experts, out_features, n))
    return mod, ref, wire


def rel_err(got, want) -> float:
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-300))


def ref_projection(ref, x, indices, paired: bool) -> np.ndarray:
    """float64 y[t, k] = W[indices[t,k]] @ x[t, 0 or k]."""
    x = np.asarray(x, dtype=np.float64)
    tokens, top_k = indices.shape
    xs = x.reshape(tokens, -1, x.shape[-1])
    sel = indices.reshape(-1).astype(np.int32)
    if paired:
        tok = np.arange(tokens * top_k, dtype=np.int32)
        xr = xs.reshape(tokens * top_k, -1)
    else:
        tok = np.repeat(np.arange(tokens, dtype=np.int32), top_k)
        xr = xs[:, 0]
    y = oracle.gemv_f64(ref, xr, sel, tok)
    return y.reshape(tokens, top_k, -1)


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy() if t.dtype == torch.bfloat16 else t.detach().cpu().numpy()


PREFILL_TOL = 2e-2
"""Prefill (tensor-core grouped GEMM) bound: bf16-GEMM tolerance per output."""


def per_output_err(got, want) -> float:
    """max over outputs of |got - want| / max(|want|, rms(want's row)).

    The per-output form of the prefill bound: each element against its own
    magnitude, floored by its row's rms so that outputs near zero are judged
    on the row's scale rather than on a vanishing denominator. Rows are the
    last axis (one pair's output features)."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    want2 = want.reshape(-1, want.shape[-1])
    rms = np.sqrt(np.mean(want2 * want2, axis=1, keepdims=True))
    den = np.maximum(np.abs(want2), np.maximum(rms, 1e-300))
    return float(np.max(np.abs(got.reshape(want2.shape) - want2) / den))


def assert_prefill_close(got, want, what="") -> tuple[float, float]:
    """Both prefill figures: the normwise max relative error and the
    per-output one, each within the 2e-2 bound."""
    norm = rel_err(got, want)
    per = per_output_err(got, want)
    print(f"prefill {what}: normwise {norm:.3e}, per-output {per:.3e}")
    assert norm < PREFILL_TOL, (what, norm)
    assert per < PREFILL_TOL, (what, per)
    return norm, per
