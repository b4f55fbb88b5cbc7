"""The fused SwitchGLU step (IqkSwitchGLU) against a float64 SwitchGLU.

The reference's projections are the per-projection seam of a SwitchGLU
(src/mlx_iqk/nn.py:1-22; its mixed-member layer test is
tests/test_nn.py:306-334 of the reference). Here the whole step -- gate,
up, SiLU * up * router weight, down, the top-k sum -- is checked against a
float64 computation with the CPU-dequantized weights: within 1e-4 of the
output's scale on the decode route (float32 h between the projections) and
within the prefill bound on the grouped route (bf16 h).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_prefill_close, rel_err, stacked
from mlx_iqk_b200 import IqkSwitchGLU
from mlx_iqk_b200 import kernels as K

pytestmark = pytest.mark.gpu

H, I = 4096, 2048


def make_layer(members, E, cuda, seed=0):
    layer = IqkSwitchGLU(members, E, H, I, device=cuda)
    weights = []
    for j, mod in enumerate((layer.gate, layer.up, layer.down)):
        rows = E * mod.out_features
        wire = oracle.random_wire(mod.member, rows, mod.in_features,
                                  seed=oracle.seed_for("glu", seed, j), scales="serving")
        st = oracle.pack(mod.member, wire, mod.in_features)
        mod.load_streams(stacked(mod.member, st, E, mod.out_features, mod.in_features))
        weights.append(oracle.decode(mod.member, st, mod.in_features)
                       .reshape(E, mod.out_features, mod.in_features))
    return layer, weights


def reference(weights, x, idx, scores, h_round=None):
    """float64 SwitchGLU: sum_k s_k * Wd_e (silu(Wg_e x) * (Wu_e x))."""
    Wg, Wu, Wd = weights
    T, k = idx.shape
    out = np.zeros((T, k, Wd.shape[1]))
    for t in range(T):
        for j in range(k):
            e = int(idx[t, j])
            a = Wg[e].astype(np.float64) @ x[t]
            h = a / (1 + np.exp(-a)) * (Wu[e].astype(np.float64) @ x[t])
            h = h * (1.0 if scores is None else float(scores[t, j]))
            if h_round is not None:
                h = h_round(h)
            out[t, j] = Wd[e].astype(np.float64) @ h
    return out if scores is None else out.sum(1)


@pytest.mark.parametrize("member", oracle.MEMBERS)
def test_glu_launch_equals_the_two_projections(cuda, member):
    """h from one gate+up launch == silu(gate) * up * w from two separate
    decode GEMVs of the same prepared workspace (the same dot products)."""
    E, T, k = 8, 5, 3
    layer, _ = make_layer((member, member, member), E, cuda, seed=1)
    g = torch.Generator(device=cuda).manual_seed(2)
    x = torch.randn((T, H), generator=g, device=cuda).to(torch.bfloat16)
    sel = torch.randint(0, E, (T * k,), generator=g, device=cuda, dtype=torch.int32)
    w = torch.rand(T * k, generator=g, device=cuda)
    ws = torch.empty(K.gemv_workspace_bytes(member, H, T, T * k), dtype=torch.uint8, device=cuda)
    K.gemv_prepare(x, E, H, sel, None, ws)
    h = torch.empty((T * k, I), device=cuda)
    K.gemv_glu_run(member, layer.gate._streams(), layer.up._streams(), E, I, H, T, T * k, w, h, ws)
    yg, yu = torch.empty_like(h), torch.empty_like(h)
    K.gemv_run(member, layer.gate._streams(), E, I, H, T, T * k, yg, ws)
    K.gemv_run(member, layer.up._streams(), E, I, H, T, T * k, yu, ws)
    want = yg.double() / (1 + torch.exp(-yg.double())) * yu.double() * w.double()[:, None]
    err = float(((h.double() - want).abs() / want.abs().clamp_min(1e-30)).max())
    assert err < 1e-5, err
    assert K.read_error(ws, H, T, T * k) == 0


@pytest.mark.parametrize("members", [("iq2_ks", "iq2_ks", "iq2_ks"), ("iq2_k", "iq2_k", "iq2_k"),
                                     ("iq1_s_r4", "iq1_s_r4", "iq1_s_r4"),
                                     ("iq2_ks", "iq2_k", "iq1_s_r4")],
                         ids=["iq2_ks", "iq2_k", "iq1_s_r4", "mixed"])
@pytest.mark.parametrize("tokens", [1, 8])
def test_decode_step_matches_float64(cuda, members, tokens):
    E, k = 16, 6
    layer, weights = make_layer(members, E, cuda, seed=3)
    rng = np.random.default_rng(tokens)
    x = rng.standard_normal((tokens, H)).astype(np.float32)
    idx = np.stack([rng.choice(E, k, replace=False) for _ in range(tokens)])
    scores = rng.dirichlet(np.ones(k), size=tokens).astype(np.float32)
    xb = torch.from_numpy(x).to(torch.bfloat16)
    got = layer(xb.to(cuda), torch.from_numpy(idx).to(cuda), torch.from_numpy(scores).to(cuda))
    assert got.shape == (tokens, H) and got.dtype == torch.float32
    want = reference(weights, xb.double().numpy(), idx, scores)
    assert rel_err(got.cpu().numpy(), want) < 1e-4
    per = layer(xb.to(cuda), torch.from_numpy(idx).to(cuda))  # no scores: per-pair outputs
    want_per = reference(weights, xb.double().numpy(), idx, None)
    assert per.shape == (tokens, k, H)
    assert rel_err(per.cpu().numpy(), want_per) < 1e-4


def test_prefill_step_matches_float64(cuda):
    E, T, k = 8, 40, 4
    layer, weights = make_layer(("iq2_ks", "iq2_ks", "iq2_k"), E, cuda, seed=5)
    rng = np.random.default_rng(7)
    x = rng.standard_normal((T, H)).astype(np.float32)
    idx = np.stack([rng.choice(E, k, replace=False) for _ in range(T)])
    scores = rng.dirichlet(np.ones(k), size=T).astype(np.float32)
    xb = torch.from_numpy(x).to(torch.bfloat16)
    got = layer(xb.to(cuda), torch.from_numpy(idx).to(cuda), torch.from_numpy(scores).to(cuda))
    bf16 = lambda h: torch.from_numpy(h).to(torch.bfloat16).double().numpy()  # noqa: E731
    want = reference(weights, xb.double().numpy(), idx, scores, h_round=bf16)
    assert_prefill_close(got.cpu().numpy(), want, "SwitchGLU prefill")
    # the sorted flag takes the same grouped route
    got_s = layer(xb.to(cuda), torch.from_numpy(idx).to(cuda), torch.from_numpy(scores).to(cuda),
                  sorted_indices=True)
    assert torch.equal(got_s, got)


def test_full_geometry_decode_step(cuda):
    """256 experts, the benchmark geometry, 8 tokens: sampled tokens against
    float64 of the experts they select."""
    from mlx_iqk_b200.profile_cases import random_streams
    E, T, k = 256, 8, 6
    layer = IqkSwitchGLU(("iq2_ks", "iq2_ks", "iq2_ks"), E, H, I, device=cuda)
    gen = torch.Generator(device=cuda).manual_seed(77)
    for mod in (layer.gate, layer.up, layer.down):
        mod.load_streams(random_streams(mod.member, E, mod.out_features, mod.in_features, cuda,
                                        gen))
    rng = np.random.default_rng(78)
    idx = np.stack([rng.choice(E, k, replace=False) for _ in range(T)])
    scores = rng.dirichlet(np.ones(k), size=T).astype(np.float32)
    x = torch.randn((T, H), generator=gen, device=cuda).to(torch.bfloat16)
    got = layer(x, torch.from_numpy(idx).to(cuda), torch.from_numpy(scores).to(cuda)).cpu().numpy()
    xs = x.double().cpu().numpy()
    dec = {}

    def w_of(mod, e):
        key = (id(mod), e)
        if key not in dec:
            st = {nm: getattr(mod, nm)[e].cpu().numpy().reshape(mod.out_features, -1)
                  for nm in mod.stream_names()}
            dec[key] = oracle.decode(mod.member, st, mod.in_features).astype(np.float64)
        return dec[key]

    for t in (0, T - 1):
        want = np.zeros(H)
        for j in range(k):
            e = int(idx[t, j])
            a = w_of(layer.gate, e) @ xs[t]
            h = a / (1 + np.exp(-a)) * (w_of(layer.up, e) @ xs[t]) * float(scores[t, j])
            want += w_of(layer.down, e) @ h
        assert rel_err(got[t], want) < 1e-4, t


@pytest.mark.parametrize("tokens", [1, 8])
def test_graphed_step_equals_the_eager_call(cuda, tokens):
    """IqkSwitchGLU.graphed: the captured decode step over static inputs gives
    the eager call's output bit for bit, replay after replay with new inputs."""
    from mlx_iqk_b200 import GraphedSwitchGLU
    E, k = 16, 6
    layer, _ = make_layer(("iq2_ks", "iq2_ks", "iq2_ks"), E, cuda, seed=5)
    step = layer.graphed(tokens, k)
    assert isinstance(step, GraphedSwitchGLU)
    rng = np.random.default_rng(90 + tokens)
    for r in range(3):
        idx = torch.from_numpy(np.stack([rng.choice(E, k, replace=False) for _ in range(tokens)])
                               .astype(np.int32)).to(cuda)
        w = torch.from_numpy(rng.dirichlet(np.ones(k), size=tokens).astype(np.float32)).to(cuda)
        x = torch.randn((tokens, H), device=cuda).to(torch.bfloat16)
        step.x.copy_(x)
        step.indices.copy_(idx)
        step.scores.copy_(w)
        got = step.replay().clone()
        want = layer(x, idx, w)
        torch.cuda.synchronize()
        assert torch.equal(got, want), r
