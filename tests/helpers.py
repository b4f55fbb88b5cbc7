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
