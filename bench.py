"""Routed-decode benchmark: IQ2_KS, 256 experts, top-6.

One step = one MoE layer's routed projections for one decode step at each
batch size of the configuration (B = 1, 4 and 8 tokens): gate and up
([2048, 4096] per expert) and down ([4096, 2048] per expert), each through
the fused dequant+GEMV kernels of libiqk_b200.so. The gate and up projections
share one preparation (iqk_gemv_prepare), the down projection gets its own
(one activation row per pair). Per-batch figures are reported under "sweep".

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batches 1,4,8] [--impl reference]

Metric: achieved GB/s of algorithmic bytes = the distinct (expert,
projection) weight rows each step must stream (the reference's byte model,
bench/price.py:146, duplicates counted once) plus activations and outputs,
divided by the device time of exactly K steps. Inputs: random IQ2_KS streams
(uniform code/scale bytes, fp16 row scales at serving magnitudes, the
reference's own pricing inputs, bench/price.py:124), x ~ N(0,1) bf16, six
distinct experts per token. Step selections rotate so no expert recurs within
a window whose weight bytes exceed twice the 126 MB L2: no step can be served
from L2. At N>1 every rank runs an independent replica (decode does not
shard; weak scaling).

``--impl reference`` times the reference's own CPU path for the same step
(vendored ik_llama dequantizer compiled from the reference's sources into
oracle/_ref, then a numpy matvec) on all host cores.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from collections import deque
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

E, TOP_K = 256, 6  # E can be lowered with --experts for small profiling captures
GATE_UP = (2048, 4096)   # out, in
DOWN = (4096, 2048)
MEMBER = "iq2_ks"
L2_BYTES = 126 * 2 ** 20
# dram__bytes_read.sum + dram__bytes_write.sum of one gate GEMV launch at B=8,
# measured by ncu on this kernel build (reported as roofline.traffic).
GATE_B8_DRAM_BYTES = 111.57e6


def row_bytes(member: str, n: int) -> int:
    return {"iq2_ks": 2 + 70 * (n // 256), "iq2_k": 76 * (n // 256),
            "iq1_s_r4": 2 + 6 * (n // 32)}[member]


def expert_bytes_per_step(batch: int) -> float:
    """Expected weight bytes of one step at uniform top-6 (planning only)."""
    distinct = E * (1 - ((E - TOP_K) / E) ** batch)
    return distinct * (2 * GATE_UP[0] * row_bytes(MEMBER, GATE_UP[1])
                       + DOWN[0] * row_bytes(MEMBER, DOWN[1]))


def make_selections(pool: int, batch: int, window: int, seed: int) -> np.ndarray:
    """[pool, batch, 6] expert ids: 6 distinct per token, uniform among experts
    not used in the `window` neighbouring steps (cyclically), so a replay of
    the pool in order never re-reads an expert L2 could still hold."""
    rng = np.random.default_rng(seed)
    sels = np.zeros((pool, batch, TOP_K), dtype=np.int64)
    used = [set() for _ in range(pool)]

    def draw(s: int) -> None:
        banned = set()
        for d in range(1, window + 1):
            banned |= used[(s - d) % pool] | used[(s + d) % pool]
        avail = np.array([e for e in range(E) if e not in banned])
        if avail.size < TOP_K:
            avail = np.arange(E)
        for t in range(batch):
            sels[s, t] = rng.choice(avail, TOP_K, replace=False)
        used[s] = set(sels[s].ravel().tolist())

    for s in range(pool):
        draw(s)
    for s in range(min(window, pool)):  # re-draw the head against the tail
        used[s] = set()
        draw(s)
    return sels


# --------------------------------------------------------------- clocks

class ClockSampler:
    """NVML SM clock / throttle-reason sampler running during a timed region."""

    SLOW = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
            "sw_power_cap": 0x4}

    def __init__(self, index: int, period: float = 0.002):
        self.samples: list[tuple[int, int]] = []
        self.period = period
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as exc:  # noqa: BLE001 - report, never fail the bench
            self.err = repr(exc)

    def _run(self):
        nv = self.nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((mhz, rs))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self.ok:
            self.t.join()

    def summary(self) -> dict:
        if not self.ok:
            return {"error": getattr(self, "err", "nvml unavailable")}
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = [m for m, _ in self.samples]
        reasons = sorted({name for _, r in self.samples for name, bit in self.SLOW.items()
                          if r & bit})
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(mhz)}


# ---------------------------------------------------------- CPU baseline

def cpu_path(batches, steps: int, seconds: float, seed: int) -> dict:
    """The reference's CPU path on sampled decode steps: ik's dequantizer on
    the selected experts' wire rows, then a float32 matvec, all host cores.
    One step = one decode step at each batch size in `batches`."""
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle
    kind = "reference" if oracle.ref_available() else "port"
    deq = oracle.ref_dequantize if kind == "reference" else oracle.dequant_wire
    cores = oracle.cpu_count()
    cache: dict[tuple[str, int], np.ndarray] = {}

    def wire_for(proj: str, e: int) -> np.ndarray:
        key = (proj, e)
        if key not in cache:
            out, n = GATE_UP if proj != "down" else DOWN
            cache[key] = oracle.random_wire(MEMBER, out, n, seed=oracle.seed_for(proj, e),
                                            scales="serving")
        return cache[key]

    sels_by_b = {b: make_selections(min(max(steps, 1), 64), b, 1, seed + b) for b in batches}
    rng = np.random.default_rng(seed + 1)
    pool = ThreadPoolExecutor(max_workers=cores)

    def one(args):
        proj, e, xs = args
        out, n = GATE_UP if proj != "down" else DOWN
        w = deq(MEMBER, wire_for(proj, e), n)
        return w @ xs.T

    done, total_bytes, t_all = 0, 0.0, 0.0
    for s in range(steps):
        for batch in batches:
            sels = sels_by_b[batch]
            sel_s = sels[s % sels.shape[0]]
            experts = sorted(set(sel_s.ravel().tolist()))
            for proj in ("gate", "up", "down"):
                for e in experts:
                    wire_for(proj, e)  # generation is input staging, not timed
            x = rng.standard_normal((batch, GATE_UP[1])).astype(np.float32)
            xd = rng.standard_normal((batch * TOP_K, DOWN[1])).astype(np.float32)
            jobs = [(p, e, x) for p in ("gate", "up") for e in experts] + \
                   [("down", e, xd[np.nonzero(sel_s.ravel() == e)[0]]) for e in experts]
            t0 = time.perf_counter()
            list(pool.map(one, jobs))
            t_all += time.perf_counter() - t0
            total_bytes += len(experts) * (2 * GATE_UP[0] * row_bytes(MEMBER, GATE_UP[1])
                                           + DOWN[0] * row_bytes(MEMBER, DOWN[1]))
        done += 1
        if t_all > seconds:
            break
    pool.shutdown()
    return {"value": total_bytes / t_all / 1e9, "unit": "GB/s", "cores": cores, "kind": kind,
            "sample": f"{done} decode steps at each B in {batches} (gate+up+down of the "
                      f"selected experts): ik dequantize + float32 numpy matvec, {cores} threads",
            "ms_per_step": 1e3 * t_all / max(done, 1)}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    batches = [int(b) for b in args.batches.split(",")]
    warm = cpu_path(batches, max(1, min(args.warmup, 2)), 1e9, seed=99)
    del warm
    res = cpu_path(batches, args.steps, args.cpu_seconds * 6, seed=1234)
    line = {
        "impl": "reference", "metric": metric_name(batches), "value": round(res["value"], 4),
        "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(res["ms_per_step"], 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 dequant, f32 matvec",
        "data": "synthetic", "config": config(args, batches),
        "cpu_baseline": {"value": round(res["value"], 4), "unit": "GB/s", "cores": res["cores"],
                         "kind": res["kind"], "sample": res["sample"]},
        "e2e": {"value": round(res["value"], 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- GPU

def metric_name(batches) -> str:
    bs = "/".join(str(b) for b in batches)
    return (f"routed decode GB/s (IQ2_KS, 256 experts top-6, gate+up+down, "
            f"one step at each B in {bs})")


def config(args, batches) -> dict:
    return {"workload": "BASELINE configs[1]: IQ2_KS routed decode, 256 experts top-6, "
                        "B = 1, 4, 8 tokens",
            "member": MEMBER, "experts": E, "top_k": TOP_K, "gate_up": list(GATE_UP),
            "down": list(DOWN), "batches": batches,
            "l2": "rotating selections: no expert recurs within a window of > 2x L2 bytes",
            "parallelism": f"replicas x{args.gpus}"}


def random_streams(torch, out: int, n: int, gen, dev, member: str = "iq2_ks",
                   experts: int | None = None):
    """Uniform random relayout streams on the device, serving scales."""
    E = experts or globals()["E"]
    def u8(count):
        return torch.randint(0, 256, (count,), generator=gen, device=dev, dtype=torch.uint8)

    def scales(shape):
        mag = torch.rand(shape, generator=gen, device=dev) * 8e-4 + 2e-5
        sign = torch.where(torch.rand(shape, generator=gen, device=dev) < 0.5, -1.0, 1.0)
        return (mag * sign).to(torch.float16)

    if member == "iq2_ks":
        return {"qs": u8(E * out * n // 4).view(torch.uint32).reshape(E, out, n // 16),
                "scl": u8(E * out * n // 64).reshape(E, out, n // 64),
                "sch": u8(E * out * n // 256).reshape(E, out, n // 256),
                "sex": u8(E * out * n // 256).reshape(E, out, n // 256),
                "dv": scales((E, out))}
    return {"qs": u8(E * out * n // 4).view(torch.uint32).reshape(E, out, n // 16),
            "scl": u8(E * out * n // 32).reshape(E, out, n // 32),
            "sex": u8(E * out * n // 128).reshape(E, out, n // 128),
            "dv": scales((E, out, n // 256))}


# ---------------------------------------------------------------- prefill

PREFILL_TOKENS = 2048


def prefill_flops(pairs: int) -> float:
    return 2.0 * pairs * (2 * GATE_UP[0] * GATE_UP[1] + DOWN[0] * DOWN[1])


def measure_ep_prefill(torch, dist, K, dev, world, rank, barrier, max_over_ranks, steps):
    """Config 5 through ExpertParallelMoE: ms per layer step, max over ranks."""
    from mlx_iqk_b200.ep import ExpertParallelMoE
    gen = torch.Generator(device=dev).manual_seed(2000 + rank)
    layer = ExpertParallelMoE(E, GATE_UP[1], GATE_UP[0], members=("iq2_ks", "iq2_ks", "iq2_k"),
                              device=dev)
    for mod in (layer.gate, layer.up, layer.down):
        mod.load_streams(random_streams(torch, mod.out_features, mod.in_features, gen, dev,
                                        mod.member, experts=layer.local_experts))
    T = PREFILL_TOKENS // world
    x = torch.randn((T, GATE_UP[1]), generator=gen, device=dev).to(torch.bfloat16)
    logits = torch.randn((T, E), generator=gen, device=dev)
    top = torch.topk(logits, TOP_K, dim=-1)
    w = torch.softmax(top.values, dim=-1)
    for _ in range(3):
        layer(x, top.indices, w)
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for _ in range(steps):
        layer(x, top.indices, w)
    e1.record(stream)
    e1.synchronize()
    barrier()
    return max_over_ranks(e0.elapsed_time(e1) / steps)


class PrefillLayer:
    """BASELINE config 5 on one GPU: one MoE layer, gate/up IQ2_KS and down
    IQ2_K over all 256 experts, T tokens routed top-6 by N(0,1) logits
    (mildly skewed load), sorted_indices=True, through the grouped GEMM.
    Step = prepare(x) + gate + up + SiLU(gate)*up*router weight (one pass
    over the routed pairs) + prepare(h) + down + each token's sum over its
    slots -- the kernels ExpertParallelMoE runs on every rank."""

    def __init__(self, torch, K, dev, gen, tokens: int = PREFILL_TOKENS):
        from mlx_iqk_b200 import IqkSwitchLinear
        self.torch, self.K, self.T = torch, K, tokens
        self.gate = IqkSwitchLinear("iq2_ks", E, *GATE_UP, device=dev)
        self.up = IqkSwitchLinear("iq2_ks", E, *GATE_UP, device=dev)
        self.down = IqkSwitchLinear("iq2_k", E, *DOWN, device=dev)
        for mod in (self.gate, self.up, self.down):
            mod.load_streams(random_streams(torch, mod.out_features, mod.in_features, gen, dev,
                                            mod.member))
        logits = torch.randn((tokens, E), generator=gen, device=dev)
        top = torch.topk(logits, TOP_K, dim=-1)
        self.weights = torch.softmax(top.values, dim=-1).reshape(-1).contiguous()
        self.sel = top.indices.to(torch.int32).reshape(-1).contiguous()
        self.pairs = self.sel.numel()
        self.x = torch.randn((tokens, GATE_UP[1]), generator=gen, device=dev).to(torch.bfloat16)
        self.ws_gu = torch.empty(K.grouped_workspace_bytes(GATE_UP[1], E, self.pairs),
                                 dtype=torch.uint8, device=dev)
        self.ws_d = torch.empty(K.grouped_workspace_bytes(DOWN[1], E, self.pairs),
                                dtype=torch.uint8, device=dev)
        self.yg = torch.empty((self.pairs, GATE_UP[0]), device=dev)
        self.yu = torch.empty((self.pairs, GATE_UP[0]), device=dev)
        self.h = torch.empty((self.pairs, DOWN[1]), device=dev, dtype=torch.bfloat16)
        self.yd = torch.empty((self.pairs, DOWN[0]), device=dev)
        self.out = torch.empty((tokens, DOWN[0]), device=dev)
        self.side = torch.cuda.Stream(dev)
        counts = torch.bincount(self.sel.long(), minlength=E).cpu()
        self.load = {"max_pairs_per_expert": int(counts.max()),
                     "min_pairs_per_expert": int(counts.min())}

    def gate_up(self):
        K, torch = self.K, self.torch
        K.grouped_prepare(self.x, E, GATE_UP[1], self.sel, None, self.ws_gu)
        # gate and up on two streams: the second fills the first's tail
        main = torch.cuda.current_stream()
        self.side.wait_stream(main)
        K.grouped_run("iq2_ks", self.gate._streams(), E, GATE_UP[0], GATE_UP[1], self.pairs,
                      self.yg, self.ws_gu)
        with torch.cuda.stream(self.side):
            K.grouped_run("iq2_ks", self.up._streams(), E, GATE_UP[0], GATE_UP[1], self.pairs,
                          self.yu, self.ws_gu)
        main.wait_stream(self.side)

    def down_proj(self):
        K = self.K
        K.grouped_prepare(self.h, E, DOWN[1], self.sel, None, self.ws_d)
        K.grouped_run("iq2_k", self.down._streams(), E, DOWN[0], DOWN[1], self.pairs, self.yd,
                      self.ws_d)

    def step(self):
        K = self.K
        self.gate_up()
        K.pairs_swiglu(self.yg, self.yu, self.weights, GATE_UP[1], E, self.ws_gu, self.h)
        self.down_proj()
        K.pairs_combine(self.yd, self.sel, TOP_K, E, self.out)


class DecodeCell:
    """One batch size of the decode workload: a pool of rotating selections and
    activations, preallocated workspaces and outputs, and the 5-launch step.
    Gate and up read the same prepared activations and nothing of each other,
    so they run on two streams: the second fills the SMs the first's last wave
    leaves idle. Down follows both, as SiLU(gate)*up would in a model."""

    def __init__(self, torch, K, mods, B: int, dev, gen, seed: int):
        self.torch, self.K, self.B = torch, K, B
        self.gate, self.up, self.down = mods
        window = max(1, math.ceil(2 * L2_BYTES / expert_bytes_per_step(B)))
        self.pool = 128
        self.sels_np = make_selections(self.pool, B, window, seed=seed)
        self.sels = torch.from_numpy(self.sels_np).to(dev, torch.int32)
        self.xs = torch.randn((self.pool, B, GATE_UP[1]), generator=gen, device=dev).to(torch.bfloat16)
        self.xds = torch.randn((self.pool, B * TOP_K, DOWN[1]), generator=gen, device=dev).to(torch.bfloat16)
        rb_gu, rb_d = row_bytes(MEMBER, GATE_UP[1]), row_bytes(MEMBER, DOWN[1])
        self.rb_gu = rb_gu
        act = (B * GATE_UP[1] * 2 + B * TOP_K * DOWN[1] * 2          # x, x_down (bf16)
               + B * TOP_K * (2 * GATE_UP[0] + DOWN[0]) * 4)          # y (f32)
        self.step_bytes = [len(set(self.sels_np[s].ravel().tolist()))
                           * (2 * GATE_UP[0] * rb_gu + DOWN[0] * rb_d) + act
                           for s in range(self.pool)]
        self.pairs = B * TOP_K
        self.ws_gu = torch.empty(K.gemv_workspace_bytes(MEMBER, GATE_UP[1], B, self.pairs),
                                 dtype=torch.uint8, device=dev)
        self.ws_d = torch.empty(K.gemv_workspace_bytes(MEMBER, DOWN[1], self.pairs, self.pairs),
                                dtype=torch.uint8, device=dev)
        self.yg = torch.empty((self.pairs, GATE_UP[0]), device=dev)
        self.yu = torch.empty((self.pairs, GATE_UP[0]), device=dev)
        self.yd = torch.empty((self.pairs, DOWN[0]), device=dev)
        self.sg, self.su, self.sd = self.gate._streams(), self.up._streams(), self.down._streams()
        self.side = torch.cuda.Stream(dev)

    launches = 5

    def step(self, s: int) -> None:
        K, p, B, P = self.K, s % self.pool, self.B, self.pairs
        torch = self.torch
        K.gemv_prepare(self.xs[p], E, GATE_UP[1], self.sels[p].reshape(-1), None, self.ws_gu)
        main = torch.cuda.current_stream()
        self.side.wait_stream(main)
        K.gemv_run(MEMBER, self.sg, E, GATE_UP[0], GATE_UP[1], B, P, self.yg, self.ws_gu)
        with torch.cuda.stream(self.side):
            K.gemv_run(MEMBER, self.su, E, GATE_UP[0], GATE_UP[1], B, P, self.yu, self.ws_gu)
        main.wait_stream(self.side)
        K.gemv_prepare(self.xds[p], E, DOWN[1], self.sels[p].reshape(-1), None, self.ws_d)
        K.gemv_run(MEMBER, self.sd, E, DOWN[0], DOWN[1], P, P, self.yd, self.ws_d)

    def bytes(self, s: int) -> int:
        return self.step_bytes[s % self.pool]


class _Eager:
    """Stand-in for a CUDA graph: replays the same launches one by one (profiling)."""

    def __init__(self, fn):
        self.fn = fn

    def replay(self):
        self.fn()


def run_b200(args) -> None:
    import torch
    import torch.distributed as dist

    from mlx_iqk_b200 import IqkSwitchLinear
    from mlx_iqk_b200 import kernels as K

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    gate = IqkSwitchLinear(MEMBER, E, *GATE_UP, device=dev)
    up = IqkSwitchLinear(MEMBER, E, *GATE_UP, device=dev)
    down = IqkSwitchLinear(MEMBER, E, *DOWN, device=dev)
    for mod in (gate, up, down):
        mod.load_streams(random_streams(torch, mod.out_features, mod.in_features, gen, dev))
    batches = [int(b) for b in args.batches.split(",")]
    cells = [DecodeCell(torch, K, (gate, up, down), B, dev, gen, seed=7 + 31 * rank + B)
             for B in batches]

    def step(s: int) -> None:  # one decode step at every batch size of the sweep
        for c in cells:
            c.step(s)

    def step_bytes(s: int) -> int:
        return sum(c.bytes(s) for c in cells)

    launches_per_step = sum(c.launches for c in cells)
    step(0)
    torch.cuda.synchronize()

    def graph(fn):
        if args.eager:
            return _Eager(fn)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        return g

    W, Kst = args.warmup, args.steps
    g_warm = graph(lambda: [step(s) for s in range(W)])
    g_time = graph(lambda: [step(s) for s in range(W, W + Kst)])
    g_warm.replay()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(ms: float) -> float:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    stream = torch.cuda.current_stream(dev)

    def timed(g) -> float:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        e0.record(stream)
        g.replay()
        e1.record(stream)
        e1.synchronize()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1))

    with ClockSampler(local) as clk:
        ms_max = timed(g_time)
    bytes_timed = sum(step_bytes(s) for s in range(W, W + Kst))
    value = world * bytes_timed / (ms_max * 1e-3) / 1e9

    # ---- per batch size (same launches, one cell at a time)
    sweep = {}
    for c in cells:
        ks = max(50, Kst // 2)
        gw = graph(lambda c=c: [c.step(s) for s in range(3)])
        gt = graph(lambda c=c, ks=ks: [c.step(s) for s in range(3, 3 + ks)])
        gw.replay()
        ms_c = timed(gt)
        by = sum(c.bytes(s) for s in range(3, 3 + ks))
        sweep[f"B={c.B}"] = {"GB/s": round(world * by / (ms_c * 1e-3) / 1e9, 2),
                             "us_per_step": round(1e3 * ms_c / ks, 3),
                             "MB_per_step": round(by / ks / 1e6, 2)}
        del gw, gt

    # ---- kernel-only roofline: the gate GEMV at the largest batch, run over
    # pre-prepared routings (rotating experts), CUDA events on its stream
    c = cells[-1]
    nr = min(c.pool, 64)
    wss = [torch.empty_like(c.ws_gu) for _ in range(nr)]
    for i in range(nr):
        K.gemv_prepare(c.xs[i], E, GATE_UP[1], c.sels[i].reshape(-1), None, wss[i])
    reps = max(2, Kst // nr)
    gk = graph(lambda: [K.gemv_run(MEMBER, c.sg, E, GATE_UP[0], GATE_UP[1], c.B, c.pairs, c.yg,
                                   wss[i]) for r in range(reps) for i in range(nr)])
    gk.replay()
    kms = timed(gk) / (reps * nr)
    gate_bytes = np.mean([len(set(c.sels_np[i].ravel().tolist())) * GATE_UP[0] * c.rb_gu
                          + c.B * GATE_UP[1] * 2 + c.pairs * GATE_UP[0] * 4 for i in range(nr)])
    peaks = {}
    try:
        peaks = json.loads((REPO / "MEASURED_PEAKS.json").read_text())
    except Exception:  # noqa: BLE001
        pass
    hbm = peaks.get("hbm_gbs")
    peak_src = "measured" if hbm else "fallback"
    hbm = hbm or 6650.0
    achieved = gate_bytes / (kms * 1e-3) / 1e9
    roofline = {"bound": "hbm", "kernel": f"gemv_kernel<IQ2_KS> (gate 2048x4096, B={c.B})",
                "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(achieved / hbm, 4), "peak_source": peak_src,
                "us_per_launch": round(kms * 1e3, 3), "bytes_per_launch": int(gate_bytes),
                "traffic": args.traffic}

    # ---- prefill (config 5): the expert-parallel layer over all ranks
    # (experts sharded E/N per rank, the 2048 tokens sharded N ways: strong
    # scaling), then at N=1 the grouped GEMMs timed alone.
    prefill = None
    if not args.no_prefill:
        ep_ms = measure_ep_prefill(torch, dist, K, dev, world, rank, barrier, max_over_ranks,
                                   steps=max(5, args.prefill_steps // 2))
    if not args.no_prefill and world > 1:
        prefill = {"metric": "prefill tokens/s (config 5 layer, expert-parallel)",
                   "value": round(PREFILL_TOKENS / (ep_ms * 1e-3), 1), "unit": "tokens/s",
                   "ms_per_step": round(ep_ms, 4), "tokens": PREFILL_TOKENS,
                   "scaling": "strong", "parallelism": f"ep{world}: {E // world} experts/rank, "
                   "NCCL all_gather dispatch, all_to_all combine"}
    if not args.no_prefill and world == 1:
        pl = PrefillLayer(torch, K, dev, gen)
        pl.step()
        torch.cuda.synchronize()
        ps = max(5, args.prefill_steps)
        gpw = graph(lambda: [pl.step() for _ in range(3)])
        gpt = graph(lambda: [pl.step() for _ in range(ps)])
        gpw.replay()
        pms = timed(gpt) / ps
        # kernel-level: each grouped GEMM alone, repeated (same routing)
        reps = 10
        gk_g = graph(lambda: [K.grouped_run("iq2_ks", pl.gate._streams(), E, GATE_UP[0],
                                            GATE_UP[1], pl.pairs, pl.yg, pl.ws_gu)
                              for _ in range(reps)])
        gk_d = graph(lambda: [K.grouped_run("iq2_k", pl.down._streams(), E, DOWN[0], DOWN[1],
                                            pl.pairs, pl.yd, pl.ws_d) for _ in range(reps)])
        pl.gate_up()
        pl.down_proj()
        gk_g.replay()
        gk_d.replay()
        g_ms = timed(gk_g) / reps
        d_ms = timed(gk_d) / reps
        tf_peak = peaks.get("bf16_tflops") or 1590.0
        g_fl = 2.0 * pl.pairs * GATE_UP[0] * GATE_UP[1]
        d_fl = 2.0 * pl.pairs * DOWN[0] * DOWN[1]
        layer_fl = prefill_flops(pl.pairs)
        prefill = {
            "metric": "prefill tokens/s (config 5 layer: gate/up IQ2_KS, down IQ2_K, "
                      "256 experts top-6, sorted_indices=True)",
            "value": round(world * pl.T / (pms * 1e-3), 1), "unit": "tokens/s",
            "tokens_per_gpu": pl.T, "ms_per_step": round(pms, 4),
            "ep_layer": {"value": round(PREFILL_TOKENS / (ep_ms * 1e-3), 1), "unit": "tokens/s",
                         "ms_per_step": round(ep_ms, 4),
                         "path": "ExpertParallelMoE.forward (dispatch, SwitchGLU, combine)"},
            "layer_tflops": round(layer_fl / (pms * 1e-3) / 1e12, 1),
            "load": pl.load,
            "gemm": {
                "gate_or_up_us": round(g_ms * 1e3, 2),
                "gate_or_up_tflops": round(g_fl / (g_ms * 1e-3) / 1e12, 1),
                "down_us": round(d_ms * 1e3, 2),
                "down_tflops": round(d_fl / (d_ms * 1e-3) / 1e12, 1),
                "bound": "tensor", "peak_tflops": tf_peak,
                "peak_source": "measured" if peaks.get("bf16_tflops") else "fallback",
                "frac_gate_or_up": round(g_fl / (g_ms * 1e-3) / 1e12 / tf_peak, 4),
                "frac_down": round(d_fl / (d_ms * 1e-3) / 1e12 / tf_peak, 4),
            },
            "parallelism": f"replicas x{world}",
        }
        del gpw, gpt, gk_g, gk_d, pl

    # ---- end to end through the public module API, host buffers. Every step
    # copies its inputs from pinned host memory and its results back; the
    # copies run on two side streams (double-buffered device inputs), so step
    # i+1's inputs upload and step i's results download while step i+1
    # computes -- the pipelining a server does. The timed region runs from
    # the first upload to the last download.
    ne = min(Kst, 100)
    host, dbuf = [], []
    for c in cells:
        B = c.B
        host.append({
            "x": torch.randn((ne, B, 1, 1, GATE_UP[1])).to(torch.bfloat16).pin_memory(),
            "xd": torch.randn((ne, B, TOP_K, 1, DOWN[1])).to(torch.bfloat16).pin_memory(),
            # int32 routing indices, as the reference's router emits 32-bit ids
            "idx": torch.from_numpy(c.sels_np[np.arange(ne) % c.pool].astype(np.int32)).pin_memory(),
            "yg": torch.empty((ne, B, TOP_K, 1, GATE_UP[0])).pin_memory(),
            "yu": torch.empty((ne, B, TOP_K, 1, GATE_UP[0])).pin_memory(),
            "yd": torch.empty((ne, B, TOP_K, 1, DOWN[0])).pin_memory()})
        dbuf.append([{"dx": torch.empty((B, 1, 1, GATE_UP[1]), device=dev, dtype=torch.bfloat16),
                      "dxd": torch.empty((B, TOP_K, 1, DOWN[1]), device=dev, dtype=torch.bfloat16),
                      "didx": torch.empty((B, TOP_K), device=dev, dtype=torch.int32)}
                     for _ in range(2)])
    up_s, down_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    in_ev = [torch.cuda.Event() for _ in range(2)]    # inputs of buffer set b landed
    free_ev = [torch.cuda.Event() for _ in range(2)]  # buffer set b's step computed
    out_ev = torch.cuda.Event()                        # the step's results written

    def upload(i: int):
        b = i & 1
        with torch.cuda.stream(up_s):
            if i >= 2:
                up_s.wait_event(free_ev[b])
            for h, d in zip(host, dbuf):
                d[b]["dx"].copy_(h["x"][i], non_blocking=True)
                d[b]["dxd"].copy_(h["xd"][i], non_blocking=True)
                d[b]["didx"].copy_(h["idx"][i], non_blocking=True)
            in_ev[b].record(up_s)

    def e2e_run(n: int):
        up_s.wait_stream(stream)  # the timed region's start event comes first
        upload(0)
        for i in range(n):
            b = i & 1
            if i + 1 < n:
                upload(i + 1)
            stream.wait_event(in_ev[b])
            outs = []
            for d in dbuf:
                outs.append((gate(d[b]["dx"], d[b]["didx"]), up(d[b]["dx"], d[b]["didx"]),
                             down(d[b]["dxd"], d[b]["didx"])))
            free_ev[b].record(stream)
            out_ev.record(stream)
            with torch.cuda.stream(down_s):
                down_s.wait_event(out_ev)
                for h, (yg, yu, yd) in zip(host, outs):
                    for t in (yg, yu, yd):
                        t.record_stream(down_s)
                    h["yg"][i].copy_(yg, non_blocking=True)
                    h["yu"][i].copy_(yu, non_blocking=True)
                    h["yd"][i].copy_(yd, non_blocking=True)
        stream.wait_stream(down_s)
        stream.wait_stream(up_s)

    e2e_run(3)
    torch.cuda.synchronize()
    ems = timed(_Eager(lambda: e2e_run(ne)))
    e_bytes = sum(c.bytes(i) for c in cells for i in range(ne))
    h2d = sum(c.B * GATE_UP[1] * 2 + c.B * TOP_K * DOWN[1] * 2 + c.B * TOP_K * 4 for c in cells)
    d2h = sum(c.B * TOP_K * (2 * GATE_UP[0] + DOWN[0]) * 4 for c in cells)
    e2e = {"value": round(world * e_bytes / (ems * 1e-3) / 1e9, 2), "unit": "GB/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
           "ms_per_step": round(ems / ne, 4), "steps": ne,
           "path": "IqkSwitchLinear.__call__ (gate, up, down) per batch size, pinned host "
                   "in/out; copies on two side streams overlapped with the next step"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        res = cpu_path(batches, 10 ** 6, args.cpu_seconds, seed=4321)
        cpu = {k: (round(v, 4) if isinstance(v, float) else v) for k, v in res.items()
               if k in ("value", "unit", "cores", "kind", "sample")}

    if rank == 0:
        line = {
            "metric": metric_name(batches), "value": round(value, 2), "unit": "GB/s",
            "n_gpus": world, "steps": Kst, "warmup": W,
            "ms_per_step": round(ms_max / Kst, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "s8 x s8 -> s32 MMA, f64 epilogue (bf16 activations)",
            "data": "synthetic: random IQ2_KS streams (serving scales), x~N(0,1) bf16",
            "config": config(args, batches),
            "sweep": sweep,
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": launches_per_step * Kst,
            "clocks": clk.summary(),
            "hbm_frac_of_step": round(value / world / hbm, 4),
            "prefill": prefill,
        }
        print(json.dumps(line), flush=True)
    del g_warm, g_time, gk
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--batches", default="1,4,8",
                    help="decode batch sizes; one step runs one decode step at each")
    ap.add_argument("--impl", default="b200", choices=("b200", "reference"))
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--experts", type=int, default=256,
                    help="experts per projection (256 = the benchmark; fewer for profiling)")
    ap.add_argument("--eager", action="store_true",
                    help="launch kernels one by one instead of replaying CUDA graphs (profiling)")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill (config 5) leg")
    ap.add_argument("--prefill-steps", type=int, default=20)
    ap.add_argument("--traffic", type=float, default=GATE_B8_DRAM_BYTES,
                    help="dram bytes per GEMV launch from an ncu capture (reported as is)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    global E
    E = args.experts
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
