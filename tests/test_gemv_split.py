"""The decode GEMV's balanced work division: cut items give the same bits.

With a workspace of ``iqk_gemv_workspace_bytes`` a wide decode grid divides
its rounds evenly over the CTAs and may cut an item between two of them; the
two parts meet in a split slot, where the later one adds the other's exact
integer row sums. With ``iqk_gemv_workspace_min_bytes`` the same call
divides whole items. Both must produce the same output bit for bit, on
every run over the same workspace (the slot counters reset themselves), and
the floor variant must run under the same division.
"""

from __future__ import annotations

import pytest
import torch

from mlx_iqk_b200 import kernels as K
from mlx_iqk_b200.profile_cases import random_module

E, OUT, N = 256, 2048, 4096


def _case(member, B, seed):
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(seed)
    mod = random_module(member, E, OUT, N, dev, gen)
    x = torch.randn((B, N), generator=gen, device=dev).to(torch.bfloat16)
    sel = torch.stack([torch.randperm(E, generator=gen, device=dev)[:6] for _ in range(B)])
    return mod, x, sel.reshape(-1).to(torch.int32)


def _run(member, mod, x, sel, ws, floor=False):
    B, P = x.shape[0], sel.numel()
    y = torch.full((P, OUT), float("nan"), device=x.device)
    K.gemv_prepare(x, E, N, sel, None, ws)
    (K.gemv_floor_run if floor else K.gemv_run)(member, mod._streams(), E, OUT, N, B, P, y, ws)
    return y


@pytest.mark.gpu
@pytest.mark.parametrize("member", ["iq2_ks", "iq1_s_r4", "iq2_k"])
@pytest.mark.parametrize("B", [4, 8, 16])
def test_cut_items_equal_whole_items(cuda, member, B):
    mod, x, sel = _case(member, B, seed=900 + B)
    P = sel.numel()
    full = torch.empty(K.gemv_workspace_bytes(member, N, B, P), dtype=torch.uint8, device=cuda)
    small = torch.empty(K.gemv_workspace_min_bytes(member, N, B, P), dtype=torch.uint8,
                        device=cuda)
    assert small.numel() < full.numel()
    y_whole = _run(member, mod, x, sel, small)
    y_cut = _run(member, mod, x, sel, full)
    y_again = _run(member, mod, x, sel, full)
    # gate and up share one preparation: two runs after one prepare
    y_third = torch.full_like(y_cut, float("nan"))
    K.gemv_run(member, mod._streams(), E, OUT, N, B, P, y_third, full)
    torch.cuda.synchronize()
    assert not torch.isnan(y_whole).any()
    assert torch.equal(y_whole, y_cut)
    assert torch.equal(y_cut, y_again)
    assert torch.equal(y_cut, y_third)
    assert K.read_error(full, N, B, P) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("member", ["iq2_ks", "iq1_s_r4"])
def test_floor_runs_under_the_same_division(cuda, member):
    mod, x, sel = _case(member, 8, seed=77)
    P = sel.numel()
    full = torch.empty(K.gemv_workspace_bytes(member, N, 8, P), dtype=torch.uint8, device=cuda)
    small = torch.empty(K.gemv_workspace_min_bytes(member, N, 8, P), dtype=torch.uint8,
                        device=cuda)
    a = _run(member, mod, x, sel, small, floor=True)
    b = _run(member, mod, x, sel, full, floor=True)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_minimum_workspace_is_smaller_and_accepted_sizes_are_ordered():
    for member in ("iq2_ks", "iq2_k", "iq1_s_r4"):
        lo = K.gemv_workspace_min_bytes(member, N, 8, 48)
        hi = K.gemv_workspace_bytes(member, N, 8, 48)
        assert 0 < lo < hi
