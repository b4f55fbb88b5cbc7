"""Expert-parallel layer on gloo ranks (CPU): the fixed-capacity path, the
lazy index check, and failures made on the host.

Nothing here touches a GPU. Failures are made the way a serving job meets
them: a rank that never joins the group, a rank that leaves between steps,
a rank whose call breaks the agreed capacity. Every case must end with an
error on every rank within the process group's short timeout, never a hang.
"""

from __future__ import annotations

import time
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mlx_iqk_b200.ep import ExpertParallelMoE
from test_ep import E, H, I, _free_port, dense_experts, make_stand_in, reference_layer, tokens_for

TIMEOUT = timedelta(seconds=4)


def _init(rank, world, port):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=TIMEOUT)


def _layer(rank, world, cap):
    experts = dense_experts()
    return experts, ExpertParallelMoE(
        E, H, I, device="cpu", max_tokens=cap,
        expert_fn=make_stand_in(experts, rank * (E // world), E // world))


def _run(target, world, *extra, timeout=90):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q, *extra)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=timeout) for _ in procs)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


def _capacity_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        experts, layer = _layer(rank, world, cap=12)
        # ragged token counts under one capacity, no host read of the counts
        T = (12, 5, 0, 9)[rank]
        x, idx, w = tokens_for(rank, T=T, seed=300)
        got = layer(x, idx, w).double()
        layer.check()
        if T:
            want = reference_layer(x, idx, w, experts)
            err = float((got - want).abs().max() / want.abs().max())
            assert err < 2e-2, f"rel err {err}"
        assert got.shape == (T, H)
        assert layer.last_stats["rows_exchanged"] == world * 12
        # a bad index on rank 1 only: the call returns, the check raises everywhere
        x2, idx2, w2 = tokens_for(rank, T=6, seed=400)
        if rank == 1:
            idx2 = idx2.clone()
            idx2[2, 1] = E + 3
        good = layer(x2, idx2, w2).double()
        try:
            layer.check()
            raised = False
        except RuntimeError:
            raised = True
        assert raised, "check() did not raise"
        if rank != 1:  # the clean ranks' results are still right
            want2 = reference_layer(x2, idx2, w2, experts)
            assert float((good - want2).abs().max() / want2.abs().max()) < 2e-2
        # the flag clears: the next clean call checks clean
        layer(x2.clone(), tokens_for(rank, T=6, seed=400)[1], w2)
        layer.check()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, None))
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        q.put((rank, repr(exc)))


@pytest.mark.parametrize("world", [2, 4])
def test_fixed_capacity_path_and_lazy_check(world):
    for rank, err in _run(_capacity_worker, world).items():
        assert err is None, f"rank {rank}: {err}"


def _lonely_worker(rank, world, port, q):
    """Rank 0 of two; rank 1 never starts."""
    t0 = time.monotonic()
    try:
        _init(rank, world, port)
        q.put((rank, "joined a group whose other rank never started"))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, ("raised", type(exc).__name__, time.monotonic() - t0)))


def test_a_rank_that_never_joins_ends_in_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_worker, args=(0, 2, _free_port(), q))
    p.start()
    rank, res = q.get(timeout=90)
    p.join(timeout=30)
    assert isinstance(res, tuple) and res[0] == "raised", res
    assert res[2] < 60, res


def _leaver_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        experts, layer = _layer(rank, world, cap=8)
        x, idx, w = tokens_for(rank, T=8, seed=500)
        layer(x, idx, w)
        layer.check()
        if rank == 1:  # leaves between steps, nothing in flight
            q.put((rank, "left"))
            return
        t0 = time.monotonic()
        try:
            layer(x, idx, w)
            layer.check()
            q.put((rank, "second step completed without its peer"))
        except Exception as exc:  # noqa: BLE001
            q.put((rank, ("raised", type(exc).__name__, time.monotonic() - t0)))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, repr(exc)))


def test_a_rank_that_leaves_between_steps():
    out = _run(_leaver_worker, 2)
    assert out[1] == "left"
    res = out[0]
    assert isinstance(res, tuple) and res[0] == "raised", res
    assert res[2] < 60, res


def _overflow_worker(rank, world, port, q):
    """Rank 1's call carries more tokens than the agreed capacity: it is
    refused on that rank before any exchange; the other rank's collective
    then ends with an error at the group's timeout."""
    try:
        _init(rank, world, port)
        experts, layer = _layer(rank, world, cap=6)
        T = 6 if rank == 0 else 7
        x, idx, w = tokens_for(rank, T=T, seed=600)
        t0 = time.monotonic()
        try:
            layer(x, idx, w)
            layer.check()
            q.put((rank, "completed"))
        except Exception as exc:  # noqa: BLE001
            q.put((rank, ("raised", type(exc).__name__, time.monotonic() - t0)))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, repr(exc)))


def test_mismatched_capacity_ends_in_errors_on_every_rank():
    out = _run(_overflow_worker, 2)
    for rank in (0, 1):
        assert isinstance(out[rank], tuple) and out[rank][0] == "raised", (rank, out[rank])
        assert out[rank][2] < 60, out[rank]
    assert out[1][1] == "IqkRuntimeError"
