"""Dense members on the GPU against the oracle, and the dense surface's guards.

Modelled on the reference's tests/test_dense_kernels.py:

1. The dense dequantization is bit-exact: the float32 chain of the serving
   decode, rounded once to fp16 (or kept in f32), compared for equality; the
   range form equals the same slice of the full form.
2. The decode GEMV matches a float64 matmul of the oracle-decoded weights at
   every sized width, for fp16 and bfloat16 activations, at 1..16 tokens and
   past them; each output row comes from the row it names.
3. The two routes of ``dense_linear`` agree numerically.

The oracle (oracle/dense_oracle.py) is itself pinned bit for bit to the
reference's golden vectors (tests/test_dense_oracle.py).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import dense_oracle as D
from mlx_iqk_b200 import dense as dn
from mlx_iqk_b200 import kernels as K
from mlx_iqk_b200.format import IqkFormatError, dense_component_shapes

MEMBERS = ("iq4_ks", "iq4_k", "iq5_k", "iq6_k")
WIDTHS = (1024, 2048, 4096, 8192)
OUT = 32

_TORCH = {np.dtype(np.uint8): torch.uint8, np.dtype(np.uint32): torch.uint32,
          np.dtype(np.float16): torch.float16, np.dtype(np.float32): torch.float32}


def _to_torch(streams, device):
    return {k: torch.from_numpy(np.ascontiguousarray(v)).to(device) for k, v in streams.items()}


def _case(member, rows, n, seed, device="cuda"):
    wire = D.random_wire(member, rows, n, seed)
    st = D.pack(member, wire, n)
    return _to_torch(st, device), D.decode(member, st, n)


def _fp16_ulp(got: np.ndarray, want: np.ndarray) -> np.ndarray:
    def order(a):
        i = a.astype(np.float16).view(np.int16).astype(np.int64)
        return np.where(i < 0, np.int64(-32768) - i, i)
    return np.abs(order(got) - order(want))


# ------------------------------------------------------------- CPU guards


@pytest.mark.parametrize("member", MEMBERS)
@pytest.mark.parametrize("bad", [512, 1536, 2560, 3072, 4352, 16384])
def test_gemv_refuses_unsized_widths(member, bad):
    with pytest.raises(K.IqkKernelError):
        dn.check_dense_gemv_geometry(bad, OUT)


@pytest.mark.parametrize("bad", [24, 40, 100])
def test_gemv_refuses_out_features_that_do_not_tile(bad):
    with pytest.raises(K.IqkKernelError):
        dn.check_dense_gemv_geometry(2048, bad)


def test_a_row_width_that_is_not_a_block_multiple_is_a_format_error():
    with pytest.raises(IqkFormatError):
        dn.check_dense_gemv_geometry(4000, OUT)
    with pytest.raises(IqkFormatError):
        dn.dense_value_table("iq2_ks", "cpu")


@pytest.mark.parametrize("member", MEMBERS)
def test_stream_checks_fail_closed(member):
    streams, _ = _case(member, OUT, 1024, seed=3, device="cpu")
    assert len(dn.check_dense_streams(member, streams, OUT, 1024)) == len(streams)
    broken = dict(streams)
    broken.pop("qs")
    with pytest.raises(dn.IqkDenseError):
        dn.check_dense_streams(member, broken, OUT, 1024)
    broken = dict(streams)
    broken["scl"] = broken["scl"][:, :-1].contiguous()
    with pytest.raises(dn.IqkDenseError):
        dn.check_dense_streams(member, broken, OUT, 1024)
    broken = dict(streams)
    broken["qs"] = broken["qs"].view(torch.int32)
    with pytest.raises(dn.IqkDenseError):
        dn.check_dense_streams(member, broken, OUT, 1024)


@pytest.mark.parametrize("member", MEMBERS)
def test_stream_order_is_the_reference_component_order(member):
    streams, _ = _case(member, OUT, 1024, seed=4, device="cpu")
    ordered = dn.check_dense_streams(member, streams, OUT, 1024)
    names = list(dense_component_shapes(member, OUT, 1024))
    assert [t.data_ptr() for t in ordered] == [streams[nm].data_ptr() for nm in names]


def test_value_tables_match_the_oracle():
    import dense_tables as T
    assert np.array_equal(dn.dense_value_table("iq4_ks", "cpu").numpy(), T.IQ4K_VALUES.astype(np.float16))
    assert np.array_equal(dn.dense_value_table("iq5_k", "cpu").numpy(), T.IQ5NL_VALUES.astype(np.float16))
    assert np.array_equal(dn.dense_value_table("iq6_k", "cpu").numpy().view(np.uint32), T.IQ6K_BITS)


# ----------------------------------------------------------- dequantization


@pytest.mark.gpu
@pytest.mark.parametrize("member", MEMBERS)
@pytest.mark.parametrize("n", WIDTHS)
def test_dequant_is_bit_identical(cuda, member, n):
    streams, ref = _case(member, OUT, n, seed=D.QK_K + n)
    got = dn.dense_dequantized(member, streams, OUT, n).cpu().numpy()
    want = ref.astype(np.float16)
    assert int(np.sum(got.view(np.uint16) != want.view(np.uint16))) == 0
    ordered = dn.check_dense_streams(member, streams, OUT, n)
    f32 = torch.empty((OUT, n), dtype=torch.float32, device=cuda)
    K.dense_dequant(member, ordered, OUT, n, 0, OUT, f32)
    assert np.array_equal(f32.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    bf = torch.empty((OUT, n), dtype=torch.bfloat16, device=cuda)
    K.dense_dequant(member, ordered, OUT, n, 0, OUT, bf)
    assert torch.equal(bf.cpu(), torch.from_numpy(ref).to(torch.bfloat16))


@pytest.mark.gpu
@pytest.mark.parametrize("member", MEMBERS)
def test_dequant_on_golden_converted_rows(cuda, member):
    """Rows the reference's codec quantized, decoded by the reference."""
    gd = np.load(str(__import__("pathlib").Path(__file__).parent / "golden" / "golden_dense.npz"))
    wire = gd[f"converted/{member}/2048/wire"]
    want = gd[f"converted/{member}/2048/want"].view(np.float32)
    streams = _to_torch(D.pack(member, wire, 2048), cuda)
    rows = wire.shape[0]
    f32 = torch.empty((rows, 2048), dtype=torch.float32, device=cuda)
    K.dense_dequant(member, dn.check_dense_streams(member, streams, rows, 2048), rows, 2048,
                    0, rows, f32)
    assert np.array_equal(f32.cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("member", MEMBERS)
@pytest.mark.parametrize("start,rows", [(0, 16), (16, 16), (8, 8), (24, 8)])
def test_dequant_range_equals_the_full_slice(cuda, member, start, rows):
    streams, _ = _case(member, OUT, 1024, seed=11)
    full = dn.dense_dequantized(member, streams, OUT, 1024)
    part = dn.dense_dequantized_range(member, streams, OUT, 1024, start, rows)
    assert torch.equal(part, full[start:start + rows])
    with pytest.raises(dn.IqkDenseError):
        dn.dense_dequantized_range(member, streams, OUT, 1024, 0, 12)
    with pytest.raises(dn.IqkDenseError):
        dn.dense_dequantized_range(member, streams, OUT, 1024, 24, 16)


@pytest.mark.gpu
@pytest.mark.parametrize("member", ("iq4_ks", "iq6_k"))
def test_dequant_range_covers_a_ragged_tail(cuda, member):
    """A height that tiles as 1024-row ranges plus a 256-row tail (the lm_head
    arithmetic at a testable height)."""
    out, n = 1024 + 256, 1024
    streams, ref = _case(member, out, n, seed=21)
    tail = dn.dense_dequantized_range(member, streams, out, n, 1024, 256).cpu().numpy()
    assert np.array_equal(tail.view(np.uint16), ref[1024:].astype(np.float16).view(np.uint16))


# ------------------------------------------------------------------- GEMV


def _gemv_check(got, x, ref, tol=1.5e-3, exact_frac=None):
    """rel < tol of the largest output (the fp16 store is one rounding); with
    ``exact_frac`` also that share of outputs equal to the rounded float64
    result (the reference asks 0.99 of its 5 x 32 float64 case)."""
    want = D.gemv_f64(ref, x)
    rel = np.max(np.abs(got.astype(np.float64) - want)) / np.max(np.abs(want))
    assert rel < tol, rel
    if exact_frac is not None:
        ulp = _fp16_ulp(got, want.astype(np.float16))
        assert float(np.mean(ulp == 0)) > exact_frac, (float(np.mean(ulp == 0)), int(ulp.max()))
        assert int(ulp.max()) <= 1


@pytest.mark.gpu
@pytest.mark.parametrize("member", MEMBERS)
@pytest.mark.parametrize("n", WIDTHS)
def test_gemv_matches_a_float64_reference(cuda, member, n):
    streams, ref = _case(member, OUT, n, seed=3 * n + 1)
    x = np.random.default_rng(17).standard_normal((5, n)).astype(np.float16)
    got = dn.dense_gemv(member, torch.from_numpy(x).to(cuda), streams, OUT, n)
    assert got.shape == (5, OUT) and got.dtype == torch.float16
    _gemv_check(got.cpu().numpy(), x, ref, exact_frac=0.99)


@pytest.mark.gpu
@pytest.mark.parametrize("member", MEMBERS)
@pytest.mark.parametrize("tokens", [1, 8, 9, 16, 17, 40])
def test_gemv_token_counts(cuda, member, tokens):
    n = 2048
    streams, ref = _case(member, 64, n, seed=100 + tokens)
    x = np.random.default_rng(tokens).standard_normal((tokens, n)).astype(np.float16)
    got = dn.dense_gemv(member, torch.from_numpy(x).to(cuda), streams, 64, n)
    _gemv_check(got.cpu().numpy(), x, ref)


@pytest.mark.gpu
@pytest.mark.parametrize("member", MEMBERS)
@pytest.mark.parametrize("dtype", (torch.float16, torch.bfloat16))
def test_gemv_serves_both_activation_dtypes(cuda, member, dtype):
    """Values representable in both types make the seam's cast the identity."""
    n = 2048
    streams, ref = _case(member, OUT, n, seed=29)
    x16 = np.random.default_rng(29).standard_normal((3, n)).astype(np.float16)
    x = torch.from_numpy(x16).to(cuda).to(torch.bfloat16).to(torch.float16)
    got = dn.dense_gemv(member, x.to(dtype), streams, OUT, n).cpu().numpy()
    _gemv_check(got, x.cpu().numpy(), ref)


@pytest.mark.gpu
@pytest.mark.parametrize("member", MEMBERS)
def test_gemv_reads_the_row_the_output_names(cuda, member):
    n = 1024
    streams, ref = _case(member, OUT, n, seed=555)
    x = np.random.default_rng(23).standard_normal((1, n)).astype(np.float16)
    got = dn.dense_gemv(member, torch.from_numpy(x).to(cuda), streams, OUT, n).cpu().numpy()[0]
    want = ref.astype(np.float64) @ x[0].astype(np.float64)
    scale = np.max(np.abs(want))
    for row in range(OUT):
        assert abs(float(got[row]) - want[row]) <= max(1.5e-3 * scale, 1e-6), row


@pytest.mark.gpu
@pytest.mark.parametrize("member", MEMBERS)
def test_linear_routes_agree(cuda, member):
    n = 1024
    streams, _ = _case(member, OUT, n, seed=31)
    x = torch.from_numpy(np.random.default_rng(31).standard_normal((4, n)).astype(np.float16)).to(cuda)
    via_gemv = dn.dense_linear(member, x, streams, OUT, n, token_limit=64).double()
    via_mm = dn.dense_linear(member, x, streams, OUT, n, token_limit=0).double()
    scale = max(float(via_mm.abs().max()), 1e-6)
    assert float((via_gemv - via_mm).abs().max()) / scale < 3e-3


@pytest.mark.gpu
@pytest.mark.parametrize("member", MEMBERS)
@pytest.mark.parametrize("n", (1024, 8192))
@pytest.mark.parametrize("tokens", (1, 9))
def test_gemv_over_several_waves_of_row_tiles(cuda, member, n, tokens):
    """Heights of two and a bit CTA waves (every CTA walks several row-tile
    groups, the last one partial), every output row checked: the reference is
    a float64 matmul of the f32 dequantization, itself bit-exact to the
    oracle (test_dequant_is_bit_identical)."""
    from mlx_iqk_b200.profile_cases import random_dense_streams
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    # rows one CTA iteration covers: IQ4 members 16 warps / (n / 1024) k parts
    # of 16-row tiles; IQ5_K / IQ6_K 8 warps / (4 or 2) k parts, two CTAs per SM
    if member in ("iq4_ks", "iq4_k"):
        rows_per_group, ctas = 16 * (16 // (n // 1024)), sms
    else:
        rows_per_group, ctas = 16 * (8 // (4 if n >= 2048 else 2)), 2 * sms
    out = rows_per_group * (2 * ctas + 1) + 48
    gen = torch.Generator(device=cuda).manual_seed(n + tokens)
    st = dn.check_dense_streams(member, random_dense_streams(member, out, n, cuda, gen), out, n)
    w = torch.empty((out, n), dtype=torch.float32, device=cuda)
    K.dense_dequant(member, st, out, n, 0, out, w)
    x = torch.randn((tokens, n), generator=gen, device=cuda).half()
    y = torch.empty((tokens, out), dtype=torch.float32, device=cuda)
    K.dense_gemv(member, x, st, out, n, y)
    want = x.double() @ w.double().t()
    rel = float((y.double() - want).abs().max()) / float(want.abs().max())
    assert rel < 1e-4, rel
    del w


@pytest.mark.gpu
@pytest.mark.parametrize("member", ("iq4_ks", "iq6_k"))
def test_gemv_at_the_lm_head_shape(cuda, member):
    """One token through a 129280 x 4096 head (random streams made on the
    device), 512 sampled rows checked against the oracle's decode of them."""
    out, n = 129280, 4096
    gen = torch.Generator(device=cuda).manual_seed(37)
    streams = {}
    for name, shape in dense_component_shapes(member, out, n).items():
        if name == "dv":
            mag = torch.rand(shape, generator=gen, device=cuda) * 8e-4 + 2e-5
            sign = torch.where(torch.rand(shape, generator=gen, device=cuda) < 0.5, -1.0, 1.0)
            streams[name] = (mag * sign).to(torch.float32 if member == "iq4_ks" else torch.float16)
            continue
        dt = torch.uint32 if name in ("qs", "qh") else torch.uint8
        count = int(np.prod(shape)) * (4 if dt == torch.uint32 else 1)
        streams[name] = torch.randint(0, 256, (count,), generator=gen, device=cuda,
                                      dtype=torch.uint8).view(dt).reshape(shape)
    x = np.random.default_rng(37).standard_normal((1, n)).astype(np.float16)
    got = dn.dense_gemv(member, torch.from_numpy(x).to(cuda), streams, out, n).cpu().numpy()[0]
    rows = np.sort(np.random.default_rng(38).choice(out, 512, replace=False))
    idx = torch.from_numpy(rows).to(cuda)
    sub = {}
    for k, v in streams.items():  # (uint32 tensors have no gather: index their int32 view)
        picked = (v.view(torch.int32) if v.dtype == torch.uint32 else v).index_select(0, idx)
        sub[k] = picked.cpu().numpy().view(np.uint32) if v.dtype == torch.uint32 else picked.cpu().numpy()
    weights = D.decode(member, sub, n)
    want = weights.astype(np.float64) @ x[0].astype(np.float64)
    rel = np.max(np.abs(got[rows].astype(np.float64) - want)) / np.max(np.abs(want))
    assert rel < 1.5e-3, rel
