"""The tensor-core grouped GEMM (prefill route) against the CPU oracle.

The reference pins its prefill route (dequantize + gather_mm) by tolerance
against float64 (tests/test_nn.py:120-151 of the reference, rel < 3e-3); the
bound stated for this path is bf16-GEMM tolerance, a max relative error of
2e-2 per output, against the float64 product of the CPU-dequantized weights.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_prefill_close, make_module, ref_projection, rel_err
from mlx_iqk_b200 import IqkSwitchLinear
from mlx_iqk_b200 import kernels as K

pytestmark = pytest.mark.gpu

GROUPED_TOL = 2e-2
WIDTHS = (2048, 4096)


def _grouped(mod, x, sel, tok=None, y_dtype=torch.float32):
    pairs = sel.numel()
    y = torch.full((pairs, mod.out_features), float("nan"), device=x.device, dtype=y_dtype)
    ws = torch.empty(K.grouped_workspace_bytes(mod.in_features, mod.num_experts, pairs),
                     dtype=torch.uint8, device=x.device)
    K.grouped(mod.member, x, mod._streams(), mod.num_experts, mod.out_features,
              mod.in_features, sel, tok, y, ws)
    return y, ws


@pytest.mark.parametrize("member", K.GROUPED_MEMBERS)
@pytest.mark.parametrize("n", WIDTHS)
def test_grouped_matches_float64(cuda, member, n):
    mod, ref, _ = make_module(member, n, seed=oracle.seed_for(member, n, "grouped"),
                              experts=8, out_features=256)
    rng = np.random.default_rng(21)
    tokens, top_k = 48, 3
    x = rng.standard_normal((tokens, 1, 1, n)).astype(np.float32)
    idx = np.stack([rng.choice(8, top_k, replace=False) for _ in range(tokens)])
    got = mod.grouped(torch.from_numpy(x).to(cuda).to(torch.bfloat16),
                      torch.from_numpy(idx).to(cuda))
    assert got.shape == (tokens, top_k, 1, 256) and got.dtype == torch.float32
    xb = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    want = ref_projection(ref, xb, idx, paired=False)
    assert_prefill_close(got.cpu().numpy().reshape(want.shape), want, f"{member} n={n}")


@pytest.mark.parametrize("member", K.GROUPED_MEMBERS)
def test_grouped_on_reference_quantized_rows(cuda, golden, member):
    n = 4096
    wire = np.concatenate([golden[f"quant/{member}/{n}/im/wire"]] * 16)  # 128 rows = 1 expert
    mod, ref, _ = make_module(member, n, seed=0, experts=1, out_features=128, wire=wire)
    rng = np.random.default_rng(6)
    x = rng.standard_normal((80, 1, 1, n)).astype(np.float32)
    idx = np.zeros((80, 1), dtype=np.int64)
    got = mod(torch.from_numpy(x).to(cuda), torch.from_numpy(idx).to(cuda))
    want = ref_projection(ref, x, idx, paired=False)
    assert_prefill_close(got.cpu().numpy().reshape(want.shape), want, f"{member} quantized")


@pytest.mark.parametrize("member", K.GROUPED_MEMBERS)
def test_grouped_expert_runs_longer_than_one_tile(cuda, member):
    """~150 pairs per expert: every expert spans two 128-token tiles."""
    n = 2048
    mod, ref, _ = make_module(member, n, seed=oracle.seed_for(member, "tiles"), experts=4,
                              out_features=128)
    rng = np.random.default_rng(3)
    tokens, top_k = 300, 2
    x = rng.standard_normal((tokens, 1, 1, n)).astype(np.float32)
    idx = np.stack([rng.choice(4, top_k, replace=False) for _ in range(tokens)])
    got = mod.grouped(torch.from_numpy(x).to(cuda), torch.from_numpy(idx).to(cuda))
    want = ref_projection(ref, x, idx, paired=False)
    assert_prefill_close(got.cpu().numpy().reshape(want.shape), want, f"{member} two tiles")


@pytest.mark.parametrize("member", K.GROUPED_MEMBERS)
def test_grouped_down_seam_and_ragged_rows(cuda, member):
    """One activation row per pair ([T, top_k, 1, in]); out = 144 leaves a
    partial 128-row block; expert loads from 0 to many pairs."""
    n = 2048
    mod, ref, _ = make_module(member, n, seed=oracle.seed_for(member, "down"), experts=6,
                              out_features=144)
    rng = np.random.default_rng(4)
    tokens, top_k = 40, 4
    x = rng.standard_normal((tokens, top_k, 1, n)).astype(np.float32)
    idx = rng.choice(6, size=(tokens, top_k), p=[0.5, 0.3, 0.1, 0.1, 0.0, 0.0])
    got = mod.grouped(torch.from_numpy(x).to(cuda), torch.from_numpy(idx).to(cuda))
    want = ref_projection(ref, x, idx, paired=True)
    assert_prefill_close(got.cpu().numpy().reshape(want.shape), want, f"{member} down seam")


@pytest.mark.parametrize("member", K.GROUPED_MEMBERS)
def test_grouped_is_independent_of_pair_order(cuda, member):
    n = 4096
    mod, _, _ = make_module(member, n, seed=oracle.seed_for(member, "gorder"), experts=8,
                            out_features=128)
    g = torch.Generator(device=cuda).manual_seed(5)
    tokens, top_k = 70, 6
    x = torch.randn((tokens, n), generator=g, device=cuda).to(torch.bfloat16)
    rng = np.random.default_rng(5)
    idx = np.stack([rng.choice(8, top_k, replace=False) for _ in range(tokens)]).reshape(-1)
    tok = np.repeat(np.arange(tokens), top_k)
    perm = rng.permutation(idx.size)
    sel0 = torch.from_numpy(idx.astype(np.int32)).to(cuda)
    y0, _ = _grouped(mod, x, sel0)
    sel1 = torch.from_numpy(idx[perm].astype(np.int32)).to(cuda)
    tok1 = torch.from_numpy(tok[perm].astype(np.int32)).to(cuda)
    y1, _ = _grouped(mod, x, sel1, tok1)
    inv = np.argsort(perm)
    assert torch.equal(y0, y1[torch.from_numpy(inv).to(cuda)])


def test_module_routes_prefill_calls(cuda):
    n = 2048
    mod, _, _ = make_module("iq2_ks", n, seed=11)
    rng = np.random.default_rng(11)
    x = torch.from_numpy(rng.standard_normal((20, 1, 1, n)).astype(np.float32)).to(cuda)
    idx = torch.from_numpy(rng.integers(0, 8, size=(20, 4))).to(cuda)  # 80 pairs > 63
    assert torch.equal(mod(x, idx), mod.grouped(x, idx))
    few = idx[:2]
    assert torch.equal(mod(x[:2], few, sorted_indices=True), mod.grouped(x[:2], few))
    assert torch.equal(mod(x[:2], few), mod.gemv(x[:2], few))
    iq1, _, _ = make_module("iq1_s_r4", n, seed=12)
    assert torch.equal(iq1(x, idx), iq1.grouped(x, idx))  # every member has the prefill route
    assert torch.equal(iq1(x[:2], few), iq1.gemv(x[:2], few))


def test_grouped_bad_index_and_nonfinite_row(cuda):
    n = 2048
    mod, ref, _ = make_module("iq2_k", n, seed=13, experts=4, out_features=128)
    x = torch.randn((6, n), device=cuda)
    x[4, 7] = float("inf")
    sel = torch.tensor([0, 1, 2, 3, 9, 1, -1, 2, 0, 3, 1, 2], dtype=torch.int32, device=cuda)
    y, ws = _grouped(mod, x, sel)
    flags = K.grouped_read_error(ws)
    assert flags & K.DEVERR_EXPERT and flags & K.DEVERR_NONFINITE
    bad = [4, 6]  # expert 9 and -1
    assert torch.all(y[bad] == 0)
    assert torch.all(torch.isnan(y[8]) | torch.isinf(y[8]))  # pair 8 reads row 4
    good = [p for p in range(12) if p not in bad and p not in (8, 9)]
    xs = x.double().cpu().numpy()
    sel_np = sel.cpu().numpy()
    for p in good:
        want = ref[sel_np[p]].astype(np.float64) @ xs[p // 2]
        assert rel_err(y[p].cpu().numpy(), want) < GROUPED_TOL, p


def test_grouped_full_geometry_sampled(cuda):
    """Config-5 projection geometry (E=256, gate 2048 x 4096, IQ2_KS), 512
    tokens x top-6, checked on a sample of the selected experts."""
    member, E, out, n = "iq2_ks", 256, 2048, 4096
    gen = torch.Generator(device=cuda).manual_seed(17)
    shapes = {"qs": (E, out, n // 16), "scl": (E, out, n // 64), "sch": (E, out, n // 256),
              "sex": (E, out, n // 256)}
    streams = {k: torch.randint(0, 256, (int(np.prod(s)) * (4 if k == "qs" else 1),),
                                generator=gen, device=cuda, dtype=torch.uint8).view(
                   torch.uint32 if k == "qs" else torch.uint8).reshape(s)
               for k, s in shapes.items()}
    mag = torch.rand((E, out), generator=gen, device=cuda) * 8e-4 + 2e-5
    sign = torch.where(torch.rand((E, out), generator=gen, device=cuda) < 0.5, -1.0, 1.0)
    streams["dv"] = (mag * sign).to(torch.float16)
    mod = IqkSwitchLinear(member, E, out, n, device=cuda)
    mod.load_streams(streams)
    rng = np.random.default_rng(18)
    T = 512
    idx = np.stack([rng.choice(E, 6, replace=False) for _ in range(T)])
    x = torch.randn(T, 1, 1, n, generator=gen, device=cuda).to(torch.bfloat16)
    got = mod(x, torch.from_numpy(idx).to(cuda), sorted_indices=True).cpu().numpy()
    got = got.reshape(T, 6, out)
    xs = x.float().cpu().numpy().reshape(T, n).astype(np.float64)
    gots, wants = [], []
    for t in (0, 101, 511):
        for k in (0, 3, 5):
            e = int(idx[t, k])
            st = {nm: getattr(mod, nm)[e].cpu().numpy().reshape(out, -1)
                  for nm in mod.stream_names()}
            w = oracle.decode(member, st, n)
            wants.append(w.astype(np.float64) @ xs[t])
            gots.append(got[t, k])
    assert_prefill_close(np.stack(gots), np.stack(wants), "config-5 gate sampled")


def test_grouped_repeated_calls_never_time_out(cuda):
    """Config-5 gate geometry, 40 calls in a row: the bounded waits inside the
    kernel must never expire (the device error word stays free of TIMEOUT)."""
    from mlx_iqk_b200.profile_cases import random_module
    gen = torch.Generator(device=cuda).manual_seed(23)
    E, out, n, T = 256, 2048, 4096, 2048
    mod = random_module("iq2_ks", E, out, n, cuda, gen)
    x = torch.randn((T, n), generator=gen, device=cuda).to(torch.bfloat16)
    logits = torch.randn((T, E), generator=gen, device=cuda)
    sel = torch.topk(logits, 6, dim=-1).indices.to(torch.int32).reshape(-1).contiguous()
    y = torch.empty((sel.numel(), out), device=cuda)
    ws = torch.empty(K.grouped_workspace_bytes(n, E, sel.numel()), dtype=torch.uint8, device=cuda)
    K.grouped_prepare(x, E, n, sel, None, ws)
    for _ in range(40):
        K.grouped_run("iq2_ks", mod._streams(), E, out, n, sel.numel(), y, ws)
    assert K.grouped_read_error(ws) & 8 == 0  # IQK_DEVERR_TIMEOUT


@pytest.mark.parametrize("member", K.GROUPED_MEMBERS)
@pytest.mark.parametrize("n", WIDTHS)
def test_sorted_matmul_range_concat_matches_the_sorted_call(cuda, member, n):
    """Range outputs concatenated along features equal the unsplit sorted
    call bit for bit (the reference's gate, tests/test_nn.py:337-360), with
    ranges that cut 128-row blocks and a range that ends at the last row."""
    mod, _, _ = make_module(member, n, seed=oracle.seed_for(member, n, "nsplit"), experts=8,
                            out_features=512)
    rng = np.random.default_rng(67)
    tokens, top_k = 24, 4
    x = torch.from_numpy(rng.standard_normal((tokens, 1, 1, n)).astype(np.float32)).to(cuda)
    idx = np.sort(rng.integers(0, 8, size=(tokens, top_k)), axis=None).reshape(tokens, top_k)
    idx = torch.from_numpy(idx).to(cuda)
    full = mod(x, idx, sorted_indices=True)
    for cuts in ((0, 256, 512), (0, 64, 128, 256, 512), (0, 32, 64, 128, 256, 384, 448, 480, 512)):
        parts = []
        for a, b in zip(cuts, cuts[1:]):
            part = mod.sorted_matmul_range(x, idx, a, b - a)
            assert part.shape == (tokens, top_k, 1, b - a)
            parts.append(part)
        got = torch.cat(parts, dim=-1)
        assert torch.equal(got.view(torch.int32), full.view(torch.int32)), cuts


def test_sorted_matmul_range_refuses_a_bad_range(cuda):
    mod, _, _ = make_module("iq2_ks", 2048, seed=61, experts=8, out_features=64)
    x = torch.randn((2, 1, 1, 2048), device=cuda)
    idx = torch.zeros((2, 2), dtype=torch.int64, device=cuda)
    for start, rows in ((0, 0), (0, 12), (0, -8), (-8, 8), (60, 8), (0, 128)):
        with pytest.raises(K.IqkRuntimeError):
            mod.sorted_matmul_range(x, idx, start, rows)


def test_sorted_matmul_range_at_full_geometry(cuda):
    """E=256, gate [2048, 4096]: a 256-row slice of a 2048-token sorted
    dispatch equals that slice of the unsplit call."""
    from mlx_iqk_b200.profile_cases import random_module
    gen = torch.Generator(device=cuda).manual_seed(99)
    mod = random_module("iq2_k", 256, 2048, 4096, cuda, gen)
    T = 512
    idx = torch.topk(torch.randn((T, 256), generator=gen, device=cuda), 6, dim=-1).indices
    x = torch.randn((T, 1, 1, 4096), generator=gen, device=cuda).to(torch.bfloat16)
    full = mod(x, idx, sorted_indices=True)
    part = mod.sorted_matmul_range(x, idx, 1024, 256)
    assert torch.equal(part, full[..., 1024:1280])
