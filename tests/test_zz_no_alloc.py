"""iqk_gemv_static: the GEMV entry point that allocates nothing.

Its scratch is a static device array inside the library, so a caller that
cannot allocate device memory at launch time still gets the fused
dequant + GEMV. Every result is compared with the workspace entry point
(iqk_gemv) on the same inputs, for two calls in a row. The file name keeps it
last in collection, so it runs both after the whole suite and alone.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import make_module
from mlx_iqk_b200 import kernels as K

SCRATCH_BYTES = 1 << 20


def test_static_scratch_limit_is_stated_and_enforced_on_the_host():
    lib = K.library()
    assert lib.iqk_gemv_static_max_bytes() == SCRATCH_BYTES
    # 80 rows at in_features 4096 need more than 1 MiB: refused before any
    # device call, so this needs no GPU.
    rows = 80
    assert K.gemv_workspace_min_bytes("iq2_ks", 4096, rows, rows) > SCRATCH_BYTES
    fake = (torch.zeros(1, dtype=torch.int64),) * 5
    status = lib.iqk_gemv_static(0, 16, 2, rows, K.ptr_array(fake), 8, 32, 4096, 16, None,
                                 rows, 16, 0, None)
    assert status == 6  # IQK_ERR_WORKSPACE
    assert K.gemv_workspace_min_bytes("iq2_ks", 4096, 64, 512) <= SCRATCH_BYTES


def _case(member, n, tokens, top_k, paired, seed, experts=16, out=64):
    mod, _, _ = make_module(member, n, seed=seed, experts=experts, out_features=out)
    g = torch.Generator(device="cuda").manual_seed(seed)
    x_rows = tokens * top_k if paired else tokens
    x = torch.randn((x_rows, n), generator=g, device="cuda").to(torch.bfloat16)
    rng = np.random.default_rng(seed)
    sel = np.stack([rng.choice(experts, top_k, replace=False) for _ in range(tokens)])
    sel = torch.from_numpy(sel.reshape(-1).astype(np.int32)).cuda()
    return mod, x, sel, out


@pytest.mark.gpu
@pytest.mark.parametrize("member", ["iq2_ks", "iq2_k", "iq1_s_r4"])
@pytest.mark.parametrize("n,tokens,paired", [(4096, 8, False), (2048, 8, True), (4096, 1, False)])
def test_static_gemv_matches_workspace_gemv_twice_in_a_row(cuda, member, n, tokens, paired):
    top_k = 6
    results = []
    for call in range(2):  # two calls in a row, different inputs, same static scratch
        mod, x, sel, out = _case(member, n, tokens, top_k, paired, seed=100 * call + tokens)
        pairs = sel.numel()
        y_ws = torch.empty((pairs, out), device="cuda")
        y_st = torch.full((pairs, out), float("nan"), device="cuda")
        K.gemv(member, x, mod._streams(), mod.num_experts, out, n, sel, None, y_ws)
        K.gemv_static(member, x, mod._streams(), mod.num_experts, out, n, sel, None, y_st)
        results.append((y_ws, y_st))
    torch.cuda.synchronize()
    for y_ws, y_st in results:
        assert torch.isfinite(y_st).all()
        # same kernels on the same inputs: identical, well inside the GEMV's
        # 1e-4 relative tolerance
        assert torch.equal(y_ws, y_st)


@pytest.mark.gpu
def test_static_gemv_with_explicit_rows_and_no_new_device_memory(cuda):
    member, n, top_k = "iq2_ks", 2048, 6
    mod, x, sel, out = _case(member, n, 4, top_k, True, seed=7)
    pairs = sel.numel()
    tok = torch.randperm(x.shape[0], device="cuda").to(torch.int32)
    y_ws = torch.empty((pairs, out), device="cuda")
    y_st = torch.empty((pairs, out), device="cuda")
    K.gemv_static(member, x, mod._streams(), mod.num_experts, out, n, sel, tok, y_st)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        K.gemv_static(member, x, mod._streams(), mod.num_experts, out, n, sel, tok, y_st)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    K.gemv(member, x, mod._streams(), mod.num_experts, out, n, sel, tok, y_ws)
    torch.cuda.synchronize()
    assert torch.equal(y_ws, y_st)


@pytest.mark.gpu
@pytest.mark.parametrize("n,x_rows,pairs", [(4096, 64, 512), (2048, 128, 768)])
def test_static_gemv_at_the_largest_geometry_that_fits(cuda, n, x_rows, pairs):
    """The documented limit: scratch use within a few percent of the array,
    explicit activation rows, equal to iqk_gemv bit for bit."""
    member, experts, out = "iq2_ks", 16, 64
    assert K.gemv_workspace_min_bytes(member, n, x_rows, pairs) > 0.85 * SCRATCH_BYTES
    assert K.gemv_workspace_min_bytes(member, n, x_rows, pairs) <= SCRATCH_BYTES
    mod, _, _ = make_module(member, n, seed=77 + n, experts=experts, out_features=out)
    g = torch.Generator(device="cuda").manual_seed(n)
    x = torch.randn((x_rows, n), generator=g, device="cuda").to(torch.bfloat16)
    sel = torch.randint(0, experts, (pairs,), generator=g, device="cuda", dtype=torch.int32)
    tok = torch.randint(0, x_rows, (pairs,), generator=g, device="cuda", dtype=torch.int32)
    y_ws = torch.empty((pairs, out), device="cuda")
    y_st = torch.full((pairs, out), float("nan"), device="cuda")
    for _ in range(2):
        K.gemv_static(member, x, mod._streams(), experts, out, n, sel, tok, y_st)
    K.gemv(member, x, mod._streams(), experts, out, n, sel, tok, y_ws)
    torch.cuda.synchronize()
    assert torch.equal(y_ws, y_st)
    assert K.gemv_static_read_error(n, x_rows, pairs) == 0


@pytest.mark.gpu
def test_static_gemv_reports_a_bad_expert_index(cuda):
    """An out-of-range expert index made on the host: zeros for that pair and
    IQK_DEVERR_EXPERT through iqk_gemv_static_read_error."""
    member, n, experts, out = "iq2_k", 2048, 8, 32
    mod, _, _ = make_module(member, n, seed=91, experts=experts, out_features=out)
    x = torch.randn((2, n), device="cuda")
    sel = torch.tensor([1, 99, 2, 3], dtype=torch.int32, device="cuda")
    y = torch.full((4, out), 7.0, device="cuda")
    K.gemv_static(member, x, mod._streams(), experts, out, n, sel, None, y)
    assert K.gemv_static_read_error(n, 2, 4) & K.DEVERR_EXPERT
    assert torch.all(y[1] == 0)
    ok = torch.tensor([1, 2, 3, 0], dtype=torch.int32, device="cuda")
    K.gemv_static(member, x, mod._streams(), experts, out, n, ok, None, y)
    assert K.gemv_static_read_error(n, 2, 4) == 0
