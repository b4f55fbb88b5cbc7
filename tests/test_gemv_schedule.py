"""The decode GEMV's dynamic work distribution gives the same bits every run.

With more items than CTAs, a launch's CTAs claim items from a counter in the
workspace header; the last CTA done resets it, so the next run over the same
workspace starts from zero. Each item's rows come from one CTA with exact
integer sums, so the output cannot depend on which CTA claimed what: runs
repeated over one workspace, two runs after one preparation (a SwitchGLU's
gate and up), and a run over a fresh workspace must agree bit for bit, for
every member and for the floor variant.
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


def _ws(member, B, P, dev):
    return torch.empty(K.gemv_workspace_bytes(member, N, B, P), dtype=torch.uint8, device=dev)


def _run(member, mod, x, sel, ws, floor=False, prepare=True):
    B, P = x.shape[0], sel.numel()
    y = torch.full((P, OUT), float("nan"), device=x.device)
    if prepare:
        K.gemv_prepare(x, E, N, sel, None, ws)
    (K.gemv_floor_run if floor else K.gemv_run)(member, mod._streams(), E, OUT, N, B, P, y, ws)
    return y


@pytest.mark.gpu
@pytest.mark.parametrize("member", ["iq2_ks", "iq1_s_r4", "iq2_k"])
@pytest.mark.parametrize("B", [4, 8, 16])
def test_claimed_items_give_the_same_bits_every_run(cuda, member, B):
    mod, x, sel = _case(member, B, seed=900 + B)
    P = sel.numel()
    ws = _ws(member, B, P, cuda)
    first = _run(member, mod, x, sel, ws)
    again = _run(member, mod, x, sel, ws)                   # counter reset by the last CTA
    no_prep = _run(member, mod, x, sel, ws, prepare=False)  # gate, then up, on one prepare
    fresh = _run(member, mod, x, sel, _ws(member, B, P, cuda))
    torch.cuda.synchronize()
    assert not torch.isnan(first).any()
    assert torch.equal(first, again)
    assert torch.equal(first, no_prep)
    assert torch.equal(first, fresh)
    assert K.read_error(ws, N, B, P) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("member", ["iq2_ks", "iq1_s_r4"])
def test_floor_variant_claims_the_same_way(cuda, member):
    mod, x, sel = _case(member, 8, seed=77)
    P = sel.numel()
    ws = _ws(member, 8, P, cuda)
    a = _run(member, mod, x, sel, ws, floor=True)
    b = _run(member, mod, x, sel, ws, floor=True)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_minimum_workspace_is_the_workspace():
    for member in ("iq2_ks", "iq2_k", "iq1_s_r4"):
        lo = K.gemv_workspace_min_bytes(member, N, 8, 48)
        hi = K.gemv_workspace_bytes(member, N, 8, 48)
        assert 0 < lo == hi
