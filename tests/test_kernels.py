"""GPU kernels against the CPU oracle: bit-exact dequant, GEMV within 1e-4.

The reference's kernel gates (tests/test_kernels.py:135-203 of the reference)
restated for the C-ABI kernels: the dequantization must not move a single
weight bit (float32 output equal to the CPU dequantizer; float16 equal to
numpy's astype; bfloat16 equal to round-to-nearest-even of the float32), and
the decode GEMV must agree with a float64 dot product of the CPU-dequantized
weights within a max relative error of 1e-4 (the bound stated for this path).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from helpers import make_module, ref_projection, rel_err, stacked, to_np
from mlx_iqk_b200 import IqkSwitchLinear
from mlx_iqk_b200 import kernels as K

pytestmark = pytest.mark.gpu

MEMBERS = oracle.MEMBERS
WIDTHS = (2048, 4096)
GEMV_TOL = 1e-4


def fp16_bits(a):
    return np.ascontiguousarray(a).astype(np.float16).view(np.uint16)


# -- dequantization is bit-exact --------------------------------------------


@pytest.mark.parametrize("member", MEMBERS)
@pytest.mark.parametrize("n", WIDTHS)
@pytest.mark.parametrize("scales", ("serving", "sweep"))
def test_dequant_float32_is_the_cpu_dequantizer(cuda, member, n, scales):
    mod, ref, _ = make_module(member, n, seed=oracle.seed_for(member, n, scales), scales=scales)
    got = mod.dequantized(torch.float32).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("member", MEMBERS)
@pytest.mark.parametrize("n", WIDTHS)
def test_dequant_float16_and_bfloat16_round_once(cuda, member, n):
    mod, ref, _ = make_module(member, n, seed=oracle.seed_for(member, n, "half"),
                              scales="sweep")
    got16 = mod.dequantized(torch.float16).cpu().numpy()
    assert np.array_equal(got16.view(np.uint16), fp16_bits(ref))
    gotbf = mod.dequantized(torch.bfloat16).cpu()
    want = torch.from_numpy(ref).to(torch.bfloat16)
    assert torch.equal(gotbf.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("member", MEMBERS)
@pytest.mark.parametrize("n", WIDTHS)
def test_dequant_converted_rows_from_the_reference_codec(cuda, golden, member, n):
    """Rows the reference's own quantizer produced (golden fixture)."""
    wire = golden[f"quant/{member}/{n}/im/wire"]  # 8 rows
    want = golden[f"quant/{member}/{n}/im/want"]
    mod, _, _ = make_module(member, n, seed=0, experts=1, out_features=16,
                            wire=np.concatenate([wire, wire]))
    got = mod.dequantized(torch.float32).cpu().numpy().reshape(16, n)
    assert np.array_equal(got[:8].view(np.uint32), want)
    assert np.array_equal(got[8:].view(np.uint32), want)


@pytest.mark.parametrize("member", MEMBERS)
def test_dequant_exhaustive_value_space(cuda, golden, member):
    """Every (scale, alphabet, code) / (grid index, slot, scale, shift) combination.

    The fixture rows are 256 wide; the kernels are sized for 2048, so eight
    fixture rows are laid side by side into one 2048-wide row (the decode is
    per 32-weight group, so the concatenation decodes to the concatenation).
    """
    wire = golden[f"exhaustive/{member}/wire"]
    rows8 = wire.shape[0] - wire.shape[0] % 64
    streams = {k: np.ascontiguousarray(v)[:rows8].reshape(rows8, -1)
               for k, v in oracle.pack(member, wire, 256).items()}
    # Tile each 256-wide row 8 times along k. Per-row streams (the row scale of
    # iq2_ks / iq1_s_r4) stay as they are; everything else repeats.
    merged = {k: v if (k == "dv" and member != "iq2_k") else np.tile(v, (1, 8))
              for k, v in streams.items()}
    n = 2048
    want = np.tile(oracle.decode(member, streams, 256), (1, 8))
    experts = rows8 // 64
    mod = IqkSwitchLinear(member, experts, 64, n, device=cuda)
    mod.load_streams(stacked(member, merged, experts, 64, n))
    got = mod.dequantized(torch.float32).cpu().numpy().reshape(rows8, n)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("member", MEMBERS)
def test_dequant_range_is_the_full_slice(cuda, member):
    mod, _, _ = make_module(member, 4096, seed=oracle.seed_for(member, "range"), out_features=64)
    full = mod.dequantized(torch.float16).view(torch.int16).cpu()
    for start, rows in ((0, 8), (8, 8), (16, 16), (0, 64), (56, 8)):
        got = mod.dequantized_range(start, rows).view(torch.int16).cpu()
        assert torch.equal(got, full[:, start:start + rows]), (start, rows)


# -- decode GEMV against float64 ---------------------------------------------


@pytest.mark.parametrize("member", MEMBERS)
@pytest.mark.parametrize("n", WIDTHS)
@pytest.mark.parametrize("xdtype", (torch.float32, torch.bfloat16, torch.float16))
def test_gemv_matches_float64(cuda, member, n, xdtype):
    mod, ref, _ = make_module(member, n, seed=oracle.seed_for(member, n, "gemv"))
    rng = np.random.default_rng(17)
    tokens, top_k = 8, 3
    x = torch.from_numpy(rng.standard_normal((tokens, 1, 1, n)).astype(np.float32)).to(xdtype)
    idx = rng.integers(0, 8, size=(tokens, top_k)).astype(np.int64)
    got = mod.gemv(x.to(cuda), torch.from_numpy(idx).to(cuda))
    assert got.shape == (tokens, top_k, 1, 32) and got.dtype == torch.float32
    want = ref_projection(ref, x.float().numpy(), idx, paired=False)
    assert rel_err(got.cpu().numpy().reshape(want.shape), want) < GEMV_TOL


@pytest.mark.parametrize("member", MEMBERS)
@pytest.mark.parametrize("n", WIDTHS)
def test_gemv_on_reference_quantized_rows(cuda, golden, member, n):
    wire = golden[f"quant/{member}/{n}/im/wire"]
    wire = np.concatenate([wire] * 4)  # 32 rows = one expert
    mod, ref, _ = make_module(member, n, seed=0, experts=1, out_features=32, wire=wire)
    rng = np.random.default_rng(5)
    x = rng.standard_normal((2, 1, 1, n)).astype(np.float32)
    idx = np.zeros((2, 1), dtype=np.int64)
    got = mod(torch.from_numpy(x).to(cuda), torch.from_numpy(idx).to(cuda))
    want = ref_projection(ref, x, idx, paired=False)
    assert rel_err(got.cpu().numpy().reshape(want.shape), want) < GEMV_TOL


@pytest.mark.parametrize("member", MEMBERS)
def test_gemv_reads_the_expert_the_index_names(cuda, member):
    n = 2048
    mod, ref, _ = make_module(member, n, seed=555)
    rng = np.random.default_rng(23)
    x = rng.standard_normal((1, 1, 1, n)).astype(np.float32)
    for e in range(8):
        idx = np.array([[e]])
        got = mod.gemv(torch.from_numpy(x).to(cuda), torch.from_numpy(idx).to(cuda))
        want = ref[e].astype(np.float64) @ x.reshape(-1).astype(np.float64)
        assert rel_err(got.cpu().numpy().reshape(-1), want) < GEMV_TOL, e


def test_config1_expert_gemv(cuda, golden):
    """Config 1 head rows: the reference-quantized expert, fp32 x."""
    wire = golden["config1/wire_head"]  # 64 rows of the 2048-row expert
    mod, ref, _ = make_module("iq2_ks", 4096, seed=0, experts=1, out_features=64, wire=wire)
    x = golden["config1/x"]
    got = mod.gemv(torch.from_numpy(x).to(cuda).reshape(1, 1, 1, -1),
                   torch.zeros((1, 1), dtype=torch.int64, device=cuda))
    want = golden["config1/y_head_f64"]
    assert rel_err(got.cpu().numpy().reshape(-1), want) < GEMV_TOL
    w16 = mod.dequantized(torch.float32).cpu().numpy().reshape(64, 4096)
    assert np.array_equal(w16.view(np.uint32), golden["config1/want_head"])


@pytest.mark.parametrize("member", MEMBERS)
def test_gemv_is_independent_of_pair_order(cuda, member):
    """Sorted and unioned calls are bit-identical to the per-pair call."""
    n = 4096
    mod, _, _ = make_module(member, n, seed=oracle.seed_for(member, "order"))
    rng = np.random.default_rng(71)
    tokens, top_k = 6, 6
    idx = rng.integers(0, 5, size=(tokens, top_k))
    x = torch.from_numpy(rng.standard_normal((tokens, 1, 1, n)).astype(np.float32)).to(cuda)
    pair = mod.gemv(x, torch.from_numpy(idx).to(cuda)).reshape(tokens * top_k, -1)
    flat = idx.reshape(-1)
    order = np.argsort(flat, kind="stable")
    toks = (order // top_k).astype(np.int64)
    y = torch.empty_like(pair)
    K.gemv(member, x.reshape(tokens, n), mod._streams(), 8, 32, n,
           torch.from_numpy(flat[order]).to(cuda, torch.int32),
           torch.from_numpy(toks).to(cuda, torch.int32), y)
    inv = np.argsort(order)
    assert torch.equal(y[torch.from_numpy(inv).to(cuda)].view(torch.int32), pair.view(torch.int32))


def test_gemv_out_of_range_index_sets_the_error_word(cuda):
    n = 2048
    mod, ref, _ = make_module("iq2_ks", n, seed=3)
    x = torch.randn(2, n, device=cuda)
    sel = torch.tensor([1, 99, 2, -1], dtype=torch.int32, device=cuda)
    y = torch.full((4, 32), 7.0, device=cuda)
    ws = torch.empty(K.gemv_workspace_bytes("iq2_ks", n, 2, 4), dtype=torch.uint8, device=cuda)
    K.gemv("iq2_ks", x, mod._streams(), 8, 32, n, sel, None, y, ws)
    assert K.read_error(ws, n, 2, 4) & K.DEVERR_EXPERT
    yc = y.cpu().numpy()
    assert np.all(yc[1] == 0) and np.all(yc[3] == 0)
    want0 = ref[1].astype(np.float64) @ x[0].cpu().double().numpy()
    assert rel_err(yc[0], want0) < GEMV_TOL


def test_gemv_nonfinite_activation_row_gives_nan(cuda):
    n = 2048
    mod, _, _ = make_module("iq2_k", n, seed=4)
    x = torch.randn(2, 1, 1, n, device=cuda)
    x[1, 0, 0, 5] = float("inf")
    got = mod.gemv(x, torch.tensor([[0, 1], [2, 3]], device=cuda)).cpu().numpy()
    assert np.all(np.isfinite(got[0])) and np.all(np.isnan(got[1]))
    ws = torch.empty(K.gemv_workspace_bytes("iq2_k", n, 2, 4), dtype=torch.uint8, device=cuda)
    K.gemv_prepare(x.reshape(2, n), 8, n, torch.tensor([0, 1, 2, 3], dtype=torch.int32,
                                                       device=cuda), None, ws)
    assert K.read_error(ws, n, 2, 4) == K.DEVERR_NONFINITE


@pytest.mark.parametrize("member", MEMBERS)
def test_prepare_once_run_twice(cuda, member):
    """One preparation serves two projections (gate and up) bit-identically."""
    n = 4096
    gate, _, _ = make_module(member, n, seed=31)
    up, _, _ = make_module(member, n, seed=32)
    x = torch.randn(3, n, device=cuda, dtype=torch.bfloat16)
    idx = torch.randint(0, 8, (3, 6), device=cuda)
    sel = idx.reshape(-1).to(torch.int32)
    ws = torch.empty(K.gemv_workspace_bytes(member, n, 3, 18), dtype=torch.uint8, device=cuda)
    K.gemv_prepare(x, 8, n, sel, None, ws)
    yg = torch.empty(18, 32, device=cuda)
    yu = torch.empty(18, 32, device=cuda)
    K.gemv_run(member, gate._streams(), 8, 32, n, 3, 18, yg, ws)
    K.gemv_run(member, up._streams(), 8, 32, n, 3, 18, yu, ws)
    assert torch.equal(yg.view(-1, 32), gate.gemv(x.reshape(3, 1, 1, n), idx).reshape(18, 32))
    assert torch.equal(yu.view(-1, 32), up.gemv(x.reshape(3, 1, 1, n), idx).reshape(18, 32))


@pytest.mark.parametrize("member", MEMBERS)
def test_gemv_handles_many_pairs_per_expert(cuda, member):
    """Prefill-shaped call: 64 tokens x top-4 over 8 experts (~32 pairs/expert)."""
    n = 2048
    mod, ref, _ = make_module(member, n, seed=oracle.seed_for(member, "many"))
    rng = np.random.default_rng(9)
    x = rng.standard_normal((64, 1, 1, n)).astype(np.float32)
    idx = rng.integers(0, 8, size=(64, 4))
    got = mod.gemv(torch.from_numpy(x).to(cuda), torch.from_numpy(idx).to(cuda))
    want = ref_projection(ref, x, idx, paired=False)
    assert rel_err(got.cpu().numpy().reshape(want.shape), want) < GEMV_TOL


@pytest.mark.parametrize("member", MEMBERS)
@pytest.mark.parametrize("geom", [(2048, 4096), (4096, 2048)])
@pytest.mark.parametrize("tokens", [1, 8])
def test_full_geometry_both_item_shapes(cuda, member, geom, tokens):
    """E=256 at the benchmark projection shapes. One token gives fewer 64-row
    items than resident CTAs, so the run kernel takes its narrow shape (16-row
    items, the four compute warps a quarter of k each); eight tokens take the
    wide shape. Checked against float64 of the CPU-decoded selected experts."""
    from mlx_iqk_b200.profile_cases import random_module
    E = 256
    out, n = geom
    gen = torch.Generator(device=cuda).manual_seed(31 + tokens)
    mod = random_module(member, E, out, n, cuda, gen)
    rng = np.random.default_rng(40 + tokens)
    idx = np.stack([rng.choice(E, 6, replace=False) for _ in range(tokens)])
    x = torch.randn(tokens, 1, 1, n, generator=gen, device=cuda).to(torch.bfloat16)
    got = mod.gemv(x, torch.from_numpy(idx).to(cuda)).cpu().numpy().reshape(tokens, 6, out)
    xs = x.float().cpu().numpy().reshape(tokens, n).astype(np.float64)
    for t in sorted({0, tokens - 1}):
        for k in (0, 5):
            e = int(idx[t, k])
            st = {nm: getattr(mod, nm)[e].cpu().numpy().reshape(out, -1)
                  for nm in mod.stream_names()}
            want = oracle.decode(member, st, n).astype(np.float64) @ xs[t]
            assert rel_err(got[t, k], want) < GEMV_TOL, (member, geom, tokens, t, k)


def test_full_geometry_decode_sampled(cuda):
    """Config 2 geometry (E=256, gate 2048x4096), B=8, checked on the
    experts actually selected (size-independent sampling)."""
    member, E, out, n = "iq2_ks", 256, 2048, 4096
    gen = torch.Generator(device=cuda).manual_seed(7)
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
    rng = np.random.default_rng(8)
    idx = np.stack([rng.choice(E, 6, replace=False) for _ in range(8)])
    x = torch.randn(8, 1, 1, n, generator=gen, device=cuda).to(torch.bfloat16)
    got = mod(x, torch.from_numpy(idx).to(cuda)).cpu().numpy().reshape(8, 6, out)
    xs = x.float().cpu().numpy().reshape(8, n).astype(np.float64)
    for t in range(8):
        for k in (0, 5):
            e = int(idx[t, k])
            st = {nm: getattr(mod, nm)[e].cpu().numpy().reshape(out, -1) for nm in mod.stream_names()}
            w = oracle.decode(member, st, n)
            want = w.astype(np.float64) @ xs[t]
            assert rel_err(got[t, k], want) < GEMV_TOL, (t, k)


def test_an_expired_bounded_wait_reports_and_the_context_survives(cuda):
    """A wait that nothing satisfies gives up after its limit with
    IQK_DEVERR_TIMEOUT (the same bounded-wait code the decode kernels use),
    and the next kernels in the same context run normally."""
    import time
    t0 = time.perf_counter()
    assert K.check_bounded_wait(5_000_000, cuda) == K.DEVERR_TIMEOUT  # 5 ms limit
    assert time.perf_counter() - t0 < 5.0
    n = 2048
    mod, ref, _ = make_module("iq2_ks", n, seed=8)
    x = torch.randn(1, 1, 1, n, device=cuda)
    y = mod.gemv(x, torch.tensor([[3]], device=cuda)).cpu().numpy().reshape(-1)
    want = ref[3].astype(np.float64) @ x.double().cpu().numpy().reshape(-1)
    assert rel_err(y, want) < GEMV_TOL
