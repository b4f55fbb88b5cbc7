"""Expert-parallel layer: dispatch / combine on gloo ranks (CPU) and the
CUDA expert path on one GPU.

The CPU tests run the real dispatch and combine code on world-size-2 and -4 gloo
process groups; the expert GEMMs there are a host stand-in (dense float
matrices), injected through ``expert_fn`` by the test only.
"""

from __future__ import annotations

import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mlx_iqk_b200.ep import ExpertParallelMoE

E, H, I, K_TOP = 8, 32, 16, 3


def dense_experts(seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(E, I, H, generator=g) * 0.2, torch.randn(E, I, H, generator=g) * 0.2,
            torch.randn(E, H, I, generator=g) * 0.2)


def reference_layer(x, idx, w, experts):
    """float64 SwitchGLU with router-weighted sum (all experts local)."""
    Wg, Wu, Wd = (t.double() for t in experts)
    x = x.to(torch.bfloat16).double()
    out = torch.zeros(x.shape[0], H, dtype=torch.float64)
    for t in range(x.shape[0]):
        for j in range(idx.shape[1]):
            e = int(idx[t, j])
            h = torch.nn.functional.silu(Wg[e] @ x[t]) * (Wu[e] @ x[t])
            out[t] += float(w[t, j]) * (Wd[e] @ h)
    return out


def make_stand_in(experts, first, local):
    Wg, Wu, Wd = experts

    def fn(rows, pair_row, pair_expert, pair_weight):
        out = torch.zeros(rows.shape[0], H, dtype=torch.float32)
        xr = rows.float()
        for p in range(pair_row.numel()):
            e = first + int(pair_expert[p])
            assert 0 <= int(pair_expert[p]) < local
            r = int(pair_row[p])
            h = torch.nn.functional.silu(Wg[e] @ xr[r]) * (Wu[e] @ xr[r])
            out[r] += float(pair_weight[p]) * (Wd[e] @ h)
        return out
    return fn


def tokens_for(rank, T=10, seed=100):
    g = torch.Generator().manual_seed(seed + rank)
    x = torch.randn(T, H, generator=g)
    logits = torch.randn(T, E, generator=g)
    top = torch.topk(logits, K_TOP, dim=-1)
    return x, top.indices, torch.softmax(top.values, dim=-1)


def _worker(rank, world, port, errq):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world)
        experts = dense_experts()
        layer = ExpertParallelMoE(E, H, I, group=None, device="cpu",
                                  expert_fn=make_stand_in(experts, rank * (E // world),
                                                          E // world))
        x, idx, w = tokens_for(rank)
        got = layer(x, idx, w).double()
        want = reference_layer(x, idx, w, experts)
        err = float((got - want).abs().max() / want.abs().max())
        if err > 2e-2:
            raise AssertionError(f"rank {rank}: rel err {err}")
        # every rank exchanged one chunk of the largest count with every rank
        if layer.last_stats["rows_exchanged"] != world * 10:
            raise AssertionError(f"rank {rank}: {layer.last_stats}")
        # a second call reuses the group, with different token counts per rank
        # (one rank of four has none)
        T2 = (7, 4, 0, 6)[rank]
        x2, idx2, w2 = tokens_for(rank, T=T2, seed=200)
        got2 = layer(x2, idx2, w2).double()
        if T2 == 0:
            if got2.shape != (0, H):
                raise AssertionError(f"rank {rank}: empty call gave {tuple(got2.shape)}")
        else:
            want2 = reference_layer(x2, idx2, w2, experts)
            err2 = float((got2 - want2).abs().max() / want2.abs().max())
            if err2 > 2e-2:
                raise AssertionError(f"rank {rank}: second call rel err {err2}")
        dist.barrier()
        dist.destroy_process_group()
        errq.put((rank, None))
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        errq.put((rank, repr(exc)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_dispatch_combine_on_gloo_ranks(world):
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, errq)) for r in range(world)]
    for p in procs:
        p.start()
    results = [errq.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, err in results:
        assert err is None, f"rank {rank}: {err}"


def test_single_rank_path_without_collectives():
    experts = dense_experts(1)
    layer = ExpertParallelMoE(E, H, I, device="cpu", expert_fn=make_stand_in(experts, 0, E))
    x, idx, w = tokens_for(0, T=12, seed=5)
    got = layer(x, idx, w).double()
    want = reference_layer(x, idx, w, experts)
    assert float((got - want).abs().max() / want.abs().max()) < 2e-2
    assert layer.last_stats["rows_exchanged"] == 12


def test_bad_expert_index_is_refused_before_any_exchange():
    experts = dense_experts(2)
    layer = ExpertParallelMoE(E, H, I, device="cpu", expert_fn=make_stand_in(experts, 0, E))
    x, idx, w = tokens_for(0, T=4)
    idx = idx.clone()
    idx[1, 0] = E
    with pytest.raises(RuntimeError):
        layer(x, idx, w)


@pytest.mark.gpu
def test_cuda_expert_path_single_gpu(cuda):
    """All experts on one GPU: the layer's CUDA grouped-GEMM path against a
    float64 SwitchGLU of the CPU-decoded weights."""
    import oracle
    from helpers import stacked
    n_h, n_i, Ex = 2048, 2048, 8
    layer = ExpertParallelMoE(Ex, n_h, n_i, members=("iq2_ks", "iq2_ks", "iq2_k"), device=cuda)
    decoded = []
    for mod, seed in ((layer.gate, 1), (layer.up, 2), (layer.down, 3)):
        rows = Ex * mod.out_features
        wire = oracle.random_wire(mod.member, rows, mod.in_features, seed=seed, scales="serving")
        streams = oracle.pack(mod.member, wire, mod.in_features)
        mod.load_streams(stacked(mod.member, streams, Ex, mod.out_features, mod.in_features))
        decoded.append(oracle.decode(mod.member, streams, mod.in_features)
                       .reshape(Ex, mod.out_features, mod.in_features).astype(np.float64))
    g = torch.Generator().manual_seed(9)
    T = 40
    x = torch.randn(T, n_h, generator=g)
    logits = torch.randn(T, Ex, generator=g)
    top = torch.topk(logits, 3, dim=-1)
    w = torch.softmax(top.values, dim=-1)
    got = layer(x.to(cuda), top.indices.to(cuda), w.to(cuda)).cpu().double().numpy()
    xb = x.to(torch.bfloat16).double().numpy()
    Wg, Wu, Wd = decoded
    want = np.zeros((T, n_h))
    for t in range(T):
        for j in range(3):
            e = int(top.indices[t, j])
            a = Wg[e] @ xb[t]
            h = a / (1 + np.exp(-a)) * (Wu[e] @ xb[t])
            h = torch.from_numpy(h).to(torch.bfloat16).double().numpy()  # the layer's bf16 h
            want[t] += float(w[t, j]) * (Wd[e] @ h)
    err = np.abs(got - want).max() / np.abs(want).max()
    assert err < 2e-2, err


def _shard_setup(cuda, tokens=40, top_k=3, seed=31):
    """An 8-expert module playing rank 1 of 2 (global experts 8..15): the slots'
    local indices run over [-8, 8), the negative ones another rank's."""
    import oracle
    from helpers import make_module
    mod, _, _ = make_module("iq2_ks", 2048, seed=oracle.seed_for("iq2_ks", "shard"), experts=8,
                            out_features=256, device=cuda)
    rng = np.random.default_rng(seed)
    glob = np.stack([rng.choice(16, top_k, replace=False) for _ in range(tokens)])
    sel = torch.from_numpy((glob - 8).astype(np.int32).reshape(-1)).to(cuda)
    x = torch.randn((tokens, 2048), generator=torch.Generator().manual_seed(seed)).to(cuda)
    return mod, x.to(torch.bfloat16), sel, top_k


@pytest.mark.gpu
def test_shard_preparation_skips_other_ranks_pairs(cuda):
    """Local slots equal a plain grouped call over just those pairs, bit for
    bit; other ranks' rows keep their previous contents; no error bit."""
    from mlx_iqk_b200 import kernels as K
    mod, x, sel, k = _shard_setup(cuda)
    P = sel.numel()
    ws = torch.empty(K.grouped_workspace_bytes(2048, 8, P), dtype=torch.uint8, device=cuda)
    K.grouped_prepare(x, 8, 2048, sel, None, ws, shard=True)
    y = torch.full((P, 256), float("nan"), device=cuda)
    K.grouped_run(mod.member, mod._streams(), 8, 256, 2048, P, y, ws)
    assert K.grouped_read_error(ws) == 0
    local = (sel >= 0).nonzero().flatten()
    tok = (local // k).to(torch.int32)
    y_ref = torch.empty((local.numel(), 256), device=cuda)
    K.grouped(mod.member, x, mod._streams(), 8, 256, 2048, sel[local].contiguous(), tok, y_ref)
    assert torch.equal(y[local], y_ref)
    foreign = (sel < 0).nonzero().flatten()
    assert foreign.numel() > 0 and bool(torch.isnan(y[foreign]).all())


@pytest.mark.gpu
def test_pairs_swiglu_and_combine(cuda):
    """The two pair-list kernels against torch on the same slots: SiLU(g)*u*w
    in float32 then one bf16 rounding; the per-row sum over local slots."""
    from mlx_iqk_b200 import kernels as K
    mod, x, sel, k = _shard_setup(cuda, tokens=64, seed=7)
    P, inter = sel.numel(), 512
    ws = torch.empty(K.grouped_workspace_bytes(2048, 8, P), dtype=torch.uint8, device=cuda)
    K.grouped_prepare(x, 8, 2048, sel, None, ws, shard=True)
    g = torch.Generator(device=cuda).manual_seed(3)
    gate = torch.randn((P, inter), generator=g, device=cuda) * 3
    up = torch.randn((P, inter), generator=g, device=cuda)
    w = torch.rand(P, generator=g, device=cuda)
    h = torch.full((P, inter), float("nan"), dtype=torch.bfloat16, device=cuda)
    K.pairs_swiglu(gate, up, w, 2048, 8, ws, h)
    local = (sel >= 0).nonzero().flatten()
    foreign = (sel < 0).nonzero().flatten()
    want = (torch.nn.functional.silu(gate) * up * w.unsqueeze(1))[local]
    got = h[local].float()
    # one bf16 rounding of a float32 value (2^-8 relative), expf vs torch's exp
    assert float(((got - want).abs() / want.abs().clamp_min(1e-3)).max()) < 2 ** -7
    assert bool(torch.isnan(h[foreign].float()).all())

    hidden = 256
    y = torch.randn((P, hidden), generator=g, device=cuda)
    y[foreign] = float("nan")  # never read
    rows = P // k
    for dt in (torch.float32, torch.bfloat16):
        out = torch.empty((rows, hidden), dtype=dt, device=cuda)
        K.pairs_combine(y, sel, k, 8, out)
        mask = (sel >= 0).view(rows, k, 1)
        want = torch.where(mask, y.view(rows, k, hidden), torch.zeros((), device=cuda)).sum(1)
        tol = 1e-5 if dt == torch.float32 else 2 ** -7
        assert float(((out.float() - want).abs() / want.abs().clamp_min(1e-2)).max()) < tol
