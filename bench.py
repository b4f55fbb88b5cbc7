"""Routed-expert benchmark: the routed decode headline, the other configurations as legs.

Headline step = one MoE layer's routed projections for one decode step at each
batch size B = 1, 4, 8: IQ2_KS gate and up
([2048, 4096] per expert) and down ([4096, 2048] per expert), 256 experts,
top-6, through the fused dequant+GEMV kernels of libiqk_b200.so. Gate and up
run on two streams, each prepared into its own workspace (the decode kernels
claim items from a counter there); down follows with its own preparation.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Metric: achieved GB/s of algorithmic bytes = the distinct (expert,
projection) weight rows a step must stream (the reference's byte model,
bench/price.py:146, duplicates counted once) plus activations and outputs,
over the device time of exactly K steps (CUDA graph replay, CUDA events,
max over ranks). Inputs: random relayout streams at serving scales (the
reference's own pricing inputs, bench/price.py:124), x ~ N(0,1) bf16, six
distinct experts per token; selections rotate so that no expert recurs within
a window whose weight bytes exceed twice the 126 MB L2.

Legs on one GPU (each a line under its own key):
  roofline   the gate GEMV at B=8 alone, beside its address floor
             (iqk_gemv_floor_run: same copies, decode deleted -- the
             reference's "vs own floor" ratio, bench/floors.py)
  configs    config 1 (one IQ2_KS expert, fp32 x), config 3 (IQ2_K at
             B = 1/16/64, unsorted and sorted), config 4 (IQ1_S_R4 at
             B = 1..8), all through IqkSwitchLinear.__call__
  dequant    the bit-exact dequantization of each member beside its floor
  dense      the dense members (IQ4_KS, IQ4_K, IQ5_K, IQ6_K): the decode GEMV
             at the lm_head shape [129280, 4096] and the fp16 dequantization
  prefill    config 5 (one layer, gate/up IQ2_KS, down IQ2_K, 2048 tokens)
             on one GPU and through the expert-parallel layer at every N,
             with the expert-parallel output checked against the one-GPU
             computation of the same tokens
  e2e        the headline step through the public module API with pinned
             host inputs and outputs copied inside the timed region
At N>1 every rank runs an independent decode replica (weak scaling); the
prefill layer shards experts and tokens (strong scaling).

``--impl reference`` times the reference's own CPU path (the vendored
ik_llama dequantizer compiled from the reference's sources into oracle/_ref,
then a numpy matmul) on the host cores, one BLAS thread per worker.
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
# dram bytes of one gate GEMV launch at B=8 from the committed ncu capture
TRAFFIC_FILE = REPO / "profiles" / "gemv_iq2ks_gate_b8_traffic.json"


def row_bytes(member: str, n: int) -> int:
    return {"iq2_ks": 2 + 70 * (n // 256), "iq2_k": 76 * (n // 256),
            "iq1_s_r4": 2 + 6 * (n // 32)}[member]


def layer_row_bytes(member: str) -> int:
    """Weight bytes of one expert's gate + up + down."""
    return 2 * GATE_UP[0] * row_bytes(member, GATE_UP[1]) + DOWN[0] * row_bytes(member, DOWN[1])


def expert_bytes_per_step(batch: int, member: str = MEMBER) -> float:
    """Expected weight bytes of one step at uniform top-6 (planning only)."""
    distinct = E * (1 - ((E - TOP_K) / E) ** batch)
    return distinct * layer_row_bytes(member)


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


def l2_window(batch: int, member: str = MEMBER) -> int:
    return max(1, math.ceil(2 * L2_BYTES / expert_bytes_per_step(batch, member)))


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

def cpu_info() -> dict:
    model = "unknown"
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle
    return {"cpu_model": model, "host_cores": oracle.cpu_count()}


def _oracle():
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle
    kind = "reference" if oracle.ref_available() else "port"
    deq = oracle.ref_dequantize if kind == "reference" else oracle.dequant_wire
    return oracle, kind, deq


def cpu_decode(batches, steps: int, seconds: float, seed: int, workers: int) -> dict:
    """The reference's CPU decode path on sampled decode steps: ik's
    dequantizer on the selected experts' wire rows, then a float32 matmul.
    ``workers`` threads over (projection, expert) jobs, each job's BLAS on one
    thread (ik's dequantizer is single-threaded; the ctypes call and numpy
    release the GIL), so ``workers`` is the core count used."""
    from threadpoolctl import threadpool_limits
    oracle, kind, deq = _oracle()
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

    def one(args):
        proj, e, xs = args
        out, n = GATE_UP if proj != "down" else DOWN
        w = deq(MEMBER, wire_for(proj, e), n)
        return w @ xs.T

    done, total_bytes, t_all = 0, 0.0, 0.0
    with threadpool_limits(limits=1), ThreadPoolExecutor(max_workers=workers) as pool:
        for s in range(steps):
            for batch in batches:
                sel_s = sels_by_b[batch][s % sels_by_b[batch].shape[0]]
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
                total_bytes += len(experts) * layer_row_bytes(MEMBER)
            done += 1
            if t_all > seconds:
                break
    return {"value": total_bytes / t_all / 1e9, "unit": "GB/s", "cores": workers, "kind": kind,
            "sample": f"{done} decode steps at each B in {batches} (gate+up+down of the "
                      f"selected experts): ik dequantize + float32 numpy matmul, {workers} "
                      f"worker thread(s), one BLAS thread each",
            "ms_per_step": 1e3 * t_all / max(done, 1), "steps": done}


def cpu_prefill(seconds: float, workers: int, seed: int = 77) -> dict:
    """Config 5 on the CPU, the reference's prefill path: per expert, ik's
    dequantizer on gate, up (IQ2_KS) and down (IQ2_K), then the expert's
    token group through silu(x Wg^T) * (x Wu^T) and down, float32 numpy.
    A bounded sample of experts (48 tokens each, the config's mean load) is
    timed with ``workers`` threads; the layer time is the sample's
    per-expert throughput times 256 experts."""
    from threadpoolctl import threadpool_limits
    oracle, kind, deq = _oracle()
    pool_n = max(4, workers)
    wires = [(oracle.random_wire("iq2_ks", GATE_UP[0], GATE_UP[1], seed=seed + 3 * i,
                                 scales="serving"),
              oracle.random_wire("iq2_ks", GATE_UP[0], GATE_UP[1], seed=seed + 3 * i + 1,
                                 scales="serving"),
              oracle.random_wire("iq2_k", DOWN[0], DOWN[1], seed=seed + 3 * i + 2,
                                 scales="serving")) for i in range(pool_n)]
    rng = np.random.default_rng(seed)
    tok = 2048 * TOP_K // E
    xs = [rng.standard_normal((tok, GATE_UP[1])).astype(np.float32) for _ in range(pool_n)]

    def one(i):
        wg, wu, wd = wires[i % pool_n]
        x = xs[i % pool_n]
        g = x @ deq("iq2_ks", wg, GATE_UP[1]).T
        u = x @ deq("iq2_ks", wu, GATE_UP[1]).T
        h = g / (1.0 + np.exp(-g)) * u
        return h @ deq("iq2_k", wd, DOWN[1]).T

    done, t_all = 0, 0.0
    with threadpool_limits(limits=1), ThreadPoolExecutor(max_workers=workers) as pool:
        list(pool.map(one, range(workers)))  # warm
        while t_all < seconds or done == 0:
            t0 = time.perf_counter()
            list(pool.map(one, range(done, done + workers)))
            t_all += time.perf_counter() - t0
            done += workers
    layer_s = t_all / done * E
    return {"value": round(2048 / layer_s, 2), "unit": "tokens/s", "cores": workers,
            "kind": kind, "layer_ms": round(1e3 * layer_s, 1),
            "sample": f"{done} experts x (gate+up+down) with {tok} tokens each: ik dequantize "
                      f"+ float32 numpy, {workers} worker thread(s), one BLAS thread each; "
                      f"layer = 256 experts at the sample's per-expert throughput"}


def cpu_baselines(batches, seconds: float) -> dict:
    """All-core decode (the headline cpu_baseline), plus single-core decode and
    the prefill layer on all cores and on one, within about ``seconds``."""
    info = cpu_info()
    cores = info["host_cores"]
    allc = cpu_decode(batches, 10 ** 6, 0.4 * seconds, seed=4321, workers=cores)
    one = cpu_decode(batches, 10 ** 6, 0.2 * seconds, seed=4321, workers=1)
    pre_all = cpu_prefill(0.25 * seconds, cores)
    pre_one = cpu_prefill(0.15 * seconds, 1)
    out = {k: (round(v, 4) if isinstance(v, float) else v) for k, v in allc.items()
           if k in ("value", "unit", "cores", "kind", "sample")}
    out.update(info)
    out["single_core"] = {"value": round(one["value"], 4), "unit": "GB/s", "cores": 1,
                          "sample": one["sample"]}
    out["prefill"] = {"all_cores": pre_all, "single_core": pre_one}
    return out


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    batches = [int(b) for b in args.batches.split(",")]
    info = cpu_info()
    cores = info["host_cores"]
    cpu_decode(batches, max(1, min(args.warmup, 2)), 1e9, seed=99, workers=cores)  # warm
    res = cpu_decode(batches, args.steps, args.cpu_seconds * 6, seed=1234, workers=cores)
    one = cpu_decode(batches, 10 ** 6, args.cpu_seconds, seed=1234, workers=1)
    pre = cpu_prefill(args.cpu_seconds, cores)
    line = {
        "impl": "reference", "metric": metric_name(batches), "value": round(res["value"], 4),
        "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(res["ms_per_step"], 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 dequant, f32 matmul",
        "data": "synthetic", "config": config(args, batches),
        "cpu_baseline": {"value": round(res["value"], 4), "unit": "GB/s", "cores": res["cores"],
                         "kind": res["kind"], "sample": res["sample"], **info,
                         "single_core": {"value": round(one["value"], 4), "unit": "GB/s",
                                         "cores": 1, "sample": one["sample"]},
                         "prefill": pre},
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


def layer_modules(torch, member: str, dev, gen, experts: int | None = None):
    """gate, up ([2048, 4096]) and down ([4096, 2048]) of one member, random
    relayout streams at serving scales."""
    from mlx_iqk_b200 import IqkSwitchLinear
    from mlx_iqk_b200.profile_cases import random_streams
    ne = experts or E
    mods = []
    for out, n in (GATE_UP, GATE_UP, DOWN):
        m = IqkSwitchLinear(member, ne, out, n, device=dev)
        m.load_streams(random_streams(member, ne, out, n, dev, gen))
        mods.append(m)
    return mods


class DecodeCell:
    """One batch size of the headline decode step on the kernel entry points:
    a pool of rotating selections and activations, preallocated workspaces
    and outputs, and the 6-launch step: gate and up each prepared into its
    own workspace and run on its own stream (the run kernels claim their items
    from a counter in their workspace, so runs on one workspace are
    stream-ordered, and two concurrent runs take two workspaces); the second
    fills the SMs the first's tail leaves idle. Down follows both, as
    SiLU(gate)*up would feed it in a model."""

    launches = 6

    def __init__(self, torch, K, mods, B: int, dev, gen, seed: int, member: str = MEMBER):
        self.torch, self.K, self.B, self.member = torch, K, B, member
        self.gate, self.up, self.down = mods
        self.pool = 128
        self.sels_np = make_selections(self.pool, B, l2_window(B, member), seed=seed)
        self.sels = torch.from_numpy(self.sels_np).to(dev, torch.int32)
        self.xs = torch.randn((self.pool, B, GATE_UP[1]), generator=gen, device=dev).to(torch.bfloat16)
        self.xds = torch.randn((self.pool, B * TOP_K, DOWN[1]), generator=gen, device=dev).to(torch.bfloat16)
        self.rb_gu = row_bytes(member, GATE_UP[1])
        act = (B * GATE_UP[1] * 2 + B * TOP_K * DOWN[1] * 2          # x, x_down (bf16)
               + B * TOP_K * (2 * GATE_UP[0] + DOWN[0]) * 4)          # y (f32)
        self.step_bytes = [len(set(self.sels_np[s].ravel().tolist())) * layer_row_bytes(member)
                           + act for s in range(self.pool)]
        self.pairs = B * TOP_K
        self.ws_gu = torch.empty(K.gemv_workspace_bytes(member, GATE_UP[1], B, self.pairs),
                                 dtype=torch.uint8, device=dev)
        self.ws_up = torch.empty_like(self.ws_gu)
        self.ws_d = torch.empty(K.gemv_workspace_bytes(member, DOWN[1], self.pairs, self.pairs),
                                dtype=torch.uint8, device=dev)
        self.yg = torch.empty((self.pairs, GATE_UP[0]), device=dev)
        self.yu = torch.empty((self.pairs, GATE_UP[0]), device=dev)
        self.yd = torch.empty((self.pairs, DOWN[0]), device=dev)
        self.sg, self.su, self.sd = self.gate._streams(), self.up._streams(), self.down._streams()
        self.side = torch.cuda.Stream(dev)

    def step(self, s: int) -> None:
        K, p, B, P, M = self.K, s % self.pool, self.B, self.pairs, self.member
        torch = self.torch
        main = torch.cuda.current_stream()
        self.side.wait_stream(main)
        K.gemv_prepare(self.xs[p], E, GATE_UP[1], self.sels[p].reshape(-1), None, self.ws_gu)
        K.gemv_run(M, self.sg, E, GATE_UP[0], GATE_UP[1], B, P, self.yg, self.ws_gu)
        with torch.cuda.stream(self.side):
            K.gemv_prepare(self.xs[p], E, GATE_UP[1], self.sels[p].reshape(-1), None, self.ws_up)
            K.gemv_run(M, self.su, E, GATE_UP[0], GATE_UP[1], B, P, self.yu, self.ws_up)
        main.wait_stream(self.side)
        K.gemv_prepare(self.xds[p], E, DOWN[1], self.sels[p].reshape(-1), None, self.ws_d)
        K.gemv_run(M, self.sd, E, DOWN[0], DOWN[1], P, P, self.yd, self.ws_d)

    def bytes(self, s: int) -> int:
        return self.step_bytes[s % self.pool]


class ModuleCell:
    """One decode (or sorted) step of a member's layer through the public
    module API, ``IqkSwitchLinear.__call__`` -- the route the drop-in takes:
    gate(x), up(x) and down(x_down), each with the same routing. With
    ``sorted_flat`` the flattened expert ids arrive in order and the call says
    so (sorted_indices=True), as the reference's sorted dispatch does."""

    def __init__(self, torch, mods, B: int, dev, gen, seed: int, member: str,
                 sorted_flat: bool = False):
        self.torch, self.B, self.sorted = torch, B, sorted_flat
        self.gate, self.up, self.down = mods
        self.pool = 64
        sels = make_selections(self.pool, B, l2_window(B, member), seed=seed)
        if sorted_flat:
            sels = np.sort(sels.reshape(self.pool, -1), axis=1).reshape(sels.shape)
        self.sels_np = sels
        self.sels = torch.from_numpy(sels).to(dev, torch.int32)
        self.xs = torch.randn((self.pool, B, 1, 1, GATE_UP[1]), generator=gen,
                              device=dev).to(torch.bfloat16)
        self.xds = torch.randn((self.pool, B, TOP_K, 1, DOWN[1]), generator=gen,
                               device=dev).to(torch.bfloat16)
        act = (B * GATE_UP[1] * 2 + B * TOP_K * DOWN[1] * 2
               + B * TOP_K * (2 * GATE_UP[0] + DOWN[0]) * 4)
        self.step_bytes = [len(set(sels[s].ravel().tolist())) * layer_row_bytes(member) + act
                           for s in range(self.pool)]

    def step(self, s: int) -> None:
        p = s % self.pool
        idx = self.sels[p]
        self.gate(self.xs[p], idx, sorted_indices=self.sorted)
        self.up(self.xs[p], idx, sorted_indices=self.sorted)
        self.down(self.xds[p], idx, sorted_indices=self.sorted)

    def bytes(self, s: int) -> int:
        return self.step_bytes[s % self.pool]


class _Eager:
    """Stand-in for a CUDA graph: replays the same launches one by one (profiling)."""

    def __init__(self, fn):
        self.fn = fn

    def replay(self):
        self.fn()


# ---------------------------------------------------------------- prefill

PREFILL_TOKENS = 2048


def prefill_flops(pairs: int) -> float:
    return 2.0 * pairs * (2 * GATE_UP[0] * GATE_UP[1] + DOWN[0] * DOWN[1])


def prefill_inputs(torch, dev, seed: int = 2024):
    """Config 5 inputs, identical on every rank: x ~ N(0,1) bf16 [2048, 4096],
    top-6 of N(0,1) router logits (mildly skewed load), softmax weights."""
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn((PREFILL_TOKENS, GATE_UP[1]), generator=g, device=dev).to(torch.bfloat16)
    logits = torch.randn((PREFILL_TOKENS, E), generator=g, device=dev)
    top = torch.topk(logits, TOP_K, dim=-1)
    return x, top.indices.to(torch.int32), torch.softmax(top.values, dim=-1)


class PrefillLayer:
    """Config 5 (prefill) on one GPU: one MoE layer (gate/up IQ2_KS, down
    IQ2_K) over all of ``mods``' experts, tokens routed top-6,
    sorted_indices=True, through the grouped GEMM. Step = prepare(x) + gate +
    up + SiLU(gate)*up*router weight (one pass over the routed pairs) +
    prepare(h) + down + each token's sum over its slots."""

    def __init__(self, torch, K, dev, mods, x, sel, weights):
        self.torch, self.K = torch, K
        self.gate, self.up, self.down = mods
        self.E = self.gate.num_experts
        self.T = x.shape[0]
        self.x = x
        self.sel = sel.reshape(-1).contiguous()
        self.weights = weights.reshape(-1).contiguous().float()
        self.pairs = self.sel.numel()
        self.ws_gu = torch.empty(K.grouped_workspace_bytes(GATE_UP[1], self.E, self.pairs),
                                 dtype=torch.uint8, device=dev)
        self.ws_d = torch.empty(K.grouped_workspace_bytes(DOWN[1], self.E, self.pairs),
                                dtype=torch.uint8, device=dev)
        self.yg = torch.empty((self.pairs, GATE_UP[0]), device=dev)
        self.yu = torch.empty((self.pairs, GATE_UP[0]), device=dev)
        self.h = torch.empty((self.pairs, DOWN[1]), device=dev, dtype=torch.bfloat16)
        self.yd = torch.empty((self.pairs, DOWN[0]), device=dev)
        self.out = torch.empty((self.T, DOWN[0]), device=dev)
        self.side = torch.cuda.Stream(dev)
        counts = torch.bincount(self.sel.long(), minlength=self.E).cpu()
        self.load = {"max_pairs_per_expert": int(counts.max()),
                     "min_pairs_per_expert": int(counts.min())}

    def gate_up(self):
        K, torch = self.K, self.torch
        K.grouped_prepare(self.x, self.E, GATE_UP[1], self.sel, None, self.ws_gu)
        main = torch.cuda.current_stream()
        self.side.wait_stream(main)
        K.grouped_run(self.gate.member, self.gate._streams(), self.E, GATE_UP[0], GATE_UP[1],
                      self.pairs, self.yg, self.ws_gu)
        with torch.cuda.stream(self.side):
            K.grouped_run(self.up.member, self.up._streams(), self.E, GATE_UP[0], GATE_UP[1],
                          self.pairs, self.yu, self.ws_gu)
        main.wait_stream(self.side)

    def down_proj(self):
        K = self.K
        K.grouped_prepare(self.h, self.E, DOWN[1], self.sel, None, self.ws_d)
        K.grouped_run(self.down.member, self.down._streams(), self.E, DOWN[0], DOWN[1],
                      self.pairs, self.yd, self.ws_d)

    def step(self):
        K = self.K
        self.gate_up()
        K.pairs_swiglu(self.yg, self.yu, self.weights, GATE_UP[1], self.E, self.ws_gu, self.h)
        self.down_proj()
        K.pairs_combine(self.yd, self.sel, TOP_K, self.E, self.out)
        return self.out


def config5_modules(torch, dev):
    """The config-5 layer's full expert set, the same bytes on every rank
    (one seeded generator), so any rank can compute any token's reference."""
    from mlx_iqk_b200 import IqkSwitchLinear
    from mlx_iqk_b200.profile_cases import random_streams
    g = torch.Generator(device=dev).manual_seed(5005)
    mods = []
    for member, (out, n) in (("iq2_ks", GATE_UP), ("iq2_ks", GATE_UP), ("iq2_k", DOWN)):
        m = IqkSwitchLinear(member, E, out, n, device=dev)
        m.load_streams(random_streams(member, E, out, n, dev, g))
        mods.append(m)
    return mods


def measure_ep_prefill(torch, K, dev, world, rank, barrier, max_over_ranks, steps, full):
    """Config 5 through ExpertParallelMoE: ms per layer step (max over ranks),
    and this rank's output checked against the one-GPU computation of its
    tokens over the full expert set (max over ranks of the relative error)."""
    from mlx_iqk_b200.ep import ExpertParallelMoE
    T = PREFILL_TOKENS // world
    layer = ExpertParallelMoE(E, GATE_UP[1], GATE_UP[0], members=("iq2_ks", "iq2_ks", "iq2_k"),
                              device=dev, max_tokens=T)
    lo, hi = layer.first_expert, layer.first_expert + layer.local_experts
    for mine, whole in zip((layer.gate, layer.up, layer.down), full):
        mine.load_streams({nm: getattr(whole, nm)[lo:hi] for nm in whole.stream_names()})
    x_all, idx_all, w_all = prefill_inputs(torch, dev)
    x, idx, w = (t[rank * T:(rank + 1) * T].contiguous() for t in (x_all, idx_all, w_all))
    for _ in range(3):
        out = layer(x, idx, w)
    layer.check()
    torch.cuda.synchronize()
    # the check: the same tokens through the one-GPU layer over all experts
    ref = PrefillLayer(torch, K, dev, full, x, idx, w).step().double()
    got = out.double()
    err = float((got - ref).abs().max() / ref.abs().max().clamp_min(1e-30))
    rms = ref.pow(2).mean(dim=1, keepdim=True).sqrt()
    per = float(((got - ref).abs() / torch.maximum(ref.abs(), rms)).max())
    run = (lambda: layer(x, idx, w))
    graph, capture_error = None, None
    if layer.capturable and not os.environ.get("IQK_EP_EAGER"):
        # every rank captures (collectives included) or none does
        try:
            graph = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                run()
                torch.cuda.synchronize()
                with torch.cuda.graph(graph, stream=s):
                    for _ in range(steps):
                        run()
            torch.cuda.current_stream(dev).wait_stream(s)
        except Exception as exc:  # noqa: BLE001 - time eagerly instead
            graph, capture_error = None, repr(exc)[:200]
        ok = max_over_ranks(0.0 if graph is not None else 1.0) == 0.0
        if not ok:
            graph = None
        barrier()
        if graph is not None:
            graph.replay()
        torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    if graph is not None:
        graph.replay()
    else:
        for _ in range(steps):
            run()
    e1.record(stream)
    e1.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    layer.check()
    phases = layer.profile_phases(x, idx, w) if hasattr(layer, "profile_phases") else None
    graphed = graph is not None
    del graph  # a graph holding NCCL calls goes before the process group does
    check = {"max_rel_err": max_over_ranks(err), "per_output_err": max_over_ranks(per),
             "tokens_checked_per_rank": T, "against": "one-GPU grouped-GEMM layer over all "
             "256 experts on the same tokens (float32 out)"}
    layer.timing = {"graph": graphed, "capture_error": capture_error}
    return ms, check, phases, layer


# ------------------------------------------------------------------ legs

class Timer:
    """CUDA-graph capture and device timing shared by every leg."""

    def __init__(self, torch, dev, world, eager: bool):
        self.torch, self.dev, self.world, self.eager = torch, dev, world, eager
        import torch.distributed as dist
        self.dist = dist

    def graph(self, fn):
        if self.eager:
            return _Eager(fn)
        g = self.torch.cuda.CUDAGraph()
        with self.torch.cuda.graph(g):
            fn()
        return g

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def max_over_ranks(self, v: float) -> float:
        t = self.torch.tensor([v], device=self.dev, dtype=self.torch.float64)
        if self.world > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def timed(self, g) -> float:
        """ms of one replay of ``g``, CUDA events on the current stream, max over ranks."""
        torch = self.torch
        stream = torch.cuda.current_stream(self.dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        self.barrier()
        e0.record(stream)
        g.replay()
        e1.record(stream)
        e1.synchronize()
        self.barrier()
        return self.max_over_ranks(e0.elapsed_time(e1))

    def cell_rate(self, cell, steps: int, warm: int = 3) -> dict:
        gw = self.graph(lambda: [cell.step(s) for s in range(warm)])
        gt = self.graph(lambda: [cell.step(s) for s in range(warm, warm + steps)])
        gw.replay()
        ms = self.timed(gt)
        by = sum(cell.bytes(s) for s in range(warm, warm + steps))
        return {"GB/s": round(self.world * by / (ms * 1e-3) / 1e9, 2),
                "us_per_step": round(1e3 * ms / steps, 3), "MB_per_step": round(by / steps / 1e6, 2)}


def hbm_peak() -> tuple[float, str, dict]:
    try:
        peaks = json.loads((REPO / "MEASURED_PEAKS.json").read_text())
    except Exception:  # noqa: BLE001
        peaks = {}
    hbm = peaks.get("hbm_gbs")
    return (hbm or 6650.0), ("measured" if hbm else "fallback"), peaks


def committed_traffic() -> dict | None:
    """DRAM bytes per launch of the roofline kernel from the committed ncu
    summary (profiles/), with the command that produced them."""
    try:
        return json.loads(TRAFFIC_FILE.read_text())
    except (OSError, ValueError):
        return None


def gemv_floor_leg(tm, K, cell, proj: str, reps_target: int) -> dict:
    """One projection's GEMV at the cell's batch, over pre-prepared rotating
    routings, beside its address floor (same copies, decode deleted)."""
    torch = tm.torch
    n_in = GATE_UP[1] if proj != "down" else DOWN[1]
    out = GATE_UP[0] if proj != "down" else DOWN[0]
    x_rows = cell.B if proj != "down" else cell.pairs
    streams = cell.sg if proj == "gate" else cell.sd
    nr = min(cell.pool, 64)
    wss = []
    for i in range(nr):
        ws = torch.empty(K.gemv_workspace_bytes(cell.member, n_in, x_rows, cell.pairs),
                         dtype=torch.uint8, device=tm.dev)
        xin = cell.xs[i] if proj != "down" else cell.xds[i]
        K.gemv_prepare(xin, E, n_in, cell.sels[i].reshape(-1), None, ws)
        wss.append(ws)
    y = torch.empty((cell.pairs, out), device=tm.dev)
    reps = max(2, reps_target // nr)
    res = {}
    for arm, fn in (("kernel", K.gemv_run), ("floor", K.gemv_floor_run)):
        g = tm.graph(lambda fn=fn: [fn(cell.member, streams, E, out, n_in, x_rows, cell.pairs, y,
                                       wss[i]) for _ in range(reps) for i in range(nr)])
        g.replay()
        res[arm] = tm.timed(g) / (reps * nr)
        del g
    rb = row_bytes(cell.member, n_in)
    nbytes = float(np.mean([len(set(cell.sels_np[i].ravel().tolist())) * out * rb
                            + x_rows * n_in * 2 + cell.pairs * out * 4 for i in range(nr)]))
    return {"us": round(res["kernel"] * 1e3, 3), "floor_us": round(res["floor"] * 1e3, 3),
            "vs_own_floor": round(res["kernel"] / res["floor"], 3),
            "bytes_per_launch": int(nbytes),
            "GB/s": round(nbytes / (res["kernel"] * 1e-3) / 1e9, 1),
            "floor_GB/s": round(nbytes / (res["floor"] * 1e-3) / 1e9, 1)}


def dequant_leg(tm, K, mod, hbm: float, experts: int = 32, reps: int = 4) -> dict:
    """Stacked f16 dequantization of ``experts`` experts per call (rotating
    expert ranges, 537 MB written per call at the gate shape) beside its
    address floor."""
    torch = tm.torch
    out, n = mod.out_features, mod.in_features
    dst = torch.empty((experts, out, n), dtype=torch.float16, device=tm.dev)
    ranges = [(i * experts) % max(mod.num_experts - experts + 1, 1) for i in range(reps)]
    streams = [[t[e0:e0 + experts] for t in mod._streams()] for e0 in ranges]
    res = {}
    for arm, fn in (("kernel", K.dequant), ("floor", K.dequant_floor)):
        g = tm.graph(lambda fn=fn: [fn(mod.member, st, experts, out, n, 0, out, dst)
                                    for st in streams])
        g.replay()
        res[arm] = tm.timed(g) / reps
        del g
    nbytes = experts * out * (row_bytes(mod.member, n) + n * 2)
    gbs = nbytes / (res["kernel"] * 1e-3) / 1e9
    return {"GB/s": round(gbs, 1), "frac": round(gbs / hbm, 4),
            "floor_GB/s": round(nbytes / (res["floor"] * 1e-3) / 1e9, 1),
            "vs_own_floor": round(res["kernel"] / res["floor"], 3),
            "us": round(res["kernel"] * 1e3, 2), "bytes": nbytes,
            "shape": f"{experts} x [{out}, {n}] -> f16"}


def dense_leg(tm, K, dev, gen, hbm: float) -> dict:
    """The dense members: the decode GEMV at the
    lm_head shape [129280, 4096] (1 and 8 tokens; the matrix is 280-440 MB,
    larger than L2, so every call streams it from HBM) and the fp16
    dequantization of 16384 of its rows, per member."""
    torch = tm.torch
    from mlx_iqk_b200 import dense as dn
    from mlx_iqk_b200.format import DENSE_MEMBERS, ik_row_bytes
    from mlx_iqk_b200.profile_cases import random_dense_streams
    out, n, rows = 129280, 4096, 16384
    res = {}
    for member in DENSE_MEMBERS:
        st = dn.check_dense_streams(member, random_dense_streams(member, out, n, dev, gen), out, n)
        wbytes = out * ik_row_bytes(member, n)
        leg = {"weights_MB": round(wbytes / 1e6, 1)}
        for T in (1, 8):
            x = torch.randn((T, n), generator=gen, device=dev).half()
            y = torch.empty((T, out), dtype=torch.float16, device=dev)
            g = tm.graph(lambda: [K.dense_gemv(member, x, st, out, n, y) for _ in range(4)])
            g.replay()
            ms = tm.timed(g) / 4
            del g
            gbs = wbytes / (ms * 1e-3) / 1e9
            leg[f"gemv T={T}"] = {"us": round(ms * 1e3, 2), "GB/s": round(gbs, 1),
                                  "frac": round(gbs / hbm, 4)}
        dst = torch.empty((rows, n), dtype=torch.float16, device=dev)
        starts = [0, 40960, 81920, 112896]
        g = tm.graph(lambda: [K.dense_dequant(member, st, out, n, s0, rows, dst) for s0 in starts])
        g.replay()
        ms = tm.timed(g) / len(starts)
        del g
        nb = rows * (ik_row_bytes(member, n) + 2 * n)
        leg["dequant"] = {"us": round(ms * 1e3, 2), "GB/s": round(nb / (ms * 1e-3) / 1e9, 1),
                          "frac": round(nb / (ms * 1e-3) / 1e9 / hbm, 4),
                          "shape": f"[{rows}, {n}] -> f16"}
        res[member] = leg
        del st, dst
        torch.cuda.empty_cache()
    return res


def config1_leg(tm, dev, gen) -> dict:
    """Config 1's call (one IQ2_KS [2048, 4096] expert, fp32 x, one
    token) through the module; 128 copies of the expert rotate so that no
    call is served from L2."""
    torch = tm.torch
    from mlx_iqk_b200 import IqkSwitchLinear
    from mlx_iqk_b200.profile_cases import random_streams
    copies = 128
    mod = IqkSwitchLinear("iq2_ks", copies, *GATE_UP, device=dev)
    mod.load_streams(random_streams("iq2_ks", copies, *GATE_UP, dev, gen))
    x = torch.randn((copies, 1, 1, 1, GATE_UP[1]), generator=gen, device=dev)
    idx = torch.arange(copies, device=dev, dtype=torch.int32).reshape(copies, 1, 1)
    g = tm.graph(lambda: [mod(x[i], idx[i]) for i in range(copies)])
    g.replay()
    ms = tm.timed(g) / copies
    nbytes = GATE_UP[0] * row_bytes("iq2_ks", GATE_UP[1]) + GATE_UP[1] * 4 + GATE_UP[0] * 4
    del g
    return {"us_per_call": round(ms * 1e3, 3), "GB/s": round(nbytes / (ms * 1e-3) / 1e9, 1),
            "bytes": nbytes, "path": "IqkSwitchLinear.__call__ (decode GEMV), x float32"}


def run_b200(args) -> None:
    import torch
    import torch.distributed as dist

    from mlx_iqk_b200 import kernels as K

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    tm = Timer(torch, dev, world, args.eager)
    hbm, peak_src, peaks = hbm_peak()

    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    mods = layer_modules(torch, MEMBER, dev, gen)
    batches = [int(b) for b in args.batches.split(",")]
    cells = [DecodeCell(torch, K, mods, B, dev, gen, seed=7 + 31 * rank + B) for B in batches]

    def step(s: int) -> None:  # one decode step at every batch size of the sweep
        for c in cells:
            c.step(s)

    launches_per_step = sum(c.launches for c in cells)
    step(0)
    torch.cuda.synchronize()
    W, Kst = args.warmup, args.steps
    g_warm = tm.graph(lambda: [step(s) for s in range(W)])
    g_time = tm.graph(lambda: [step(s) for s in range(W, W + Kst)])
    g_warm.replay()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        ms_max = tm.timed(g_time)
    bytes_timed = sum(c.bytes(s) for c in cells for s in range(W, W + Kst))
    value = world * bytes_timed / (ms_max * 1e-3) / 1e9
    del g_warm, g_time

    sweep = {f"B={c.B}": tm.cell_rate(c, max(50, Kst // 2)) for c in cells}

    # ---- kernel-only roofline: the gate GEMV at the largest batch, beside
    # its address floor; down at the same batch as a second floor pair
    c8 = cells[-1]
    gate_leg = gemv_floor_leg(tm, K, c8, "gate", max(2 * Kst, 128))
    down_leg = gemv_floor_leg(tm, K, c8, "down", max(2 * Kst, 128))
    traffic = committed_traffic()
    achieved = gate_leg["GB/s"]
    roofline = {"bound": "hbm", "kernel": f"gemv_kernel<IQ2_KS> (gate 2048x4096, B={c8.B})",
                "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": round(achieved / hbm, 4), "peak_source": peak_src,
                "us_per_launch": gate_leg["us"], "bytes_per_launch": gate_leg["bytes_per_launch"],
                # the committed capture's DRAM bytes per algorithmic byte, on
                # this launch's algorithmic bytes (its draw has other experts)
                "traffic": (round(traffic["traffic_over_algorithmic"]
                                  * gate_leg["bytes_per_launch"]) if traffic else None),
                "traffic_capture": ({k: traffic[k] for k in ("dram_bytes_per_launch",
                                                              "algorithmic_bytes_same_launch",
                                                              "traffic_over_algorithmic",
                                                              "command")} if traffic else None),
                "floor_us": gate_leg["floor_us"], "vs_own_floor": gate_leg["vs_own_floor"]}
    floors = {f"gemv gate B={c8.B}": gate_leg, f"gemv down B={c8.B}": down_leg}

    configs, dequant, dense = None, None, None
    if world == 1 and not args.no_legs:
        configs = {"config1 (IQ2_KS one expert, fp32 x)": config1_leg(tm, dev, gen)}
        for member, bs, sorts in (("iq2_k", (1, 16, 64), (False, True)),
                                  ("iq1_s_r4", tuple(range(1, 9)), (False,))):
            mm = layer_modules(torch, member, dev, gen)
            leg = {}
            for B in bs:
                for srt in sorts:
                    cell = ModuleCell(torch, mm, B, dev, gen, seed=900 + B, member=member,
                                      sorted_flat=srt)
                    key = f"B={B}" + (" sorted" if srt else "")
                    leg[key] = tm.cell_rate(cell, 30)
            name = ("config3 (IQ2_K, unsorted then sorted)" if member == "iq2_k"
                    else "config4 (IQ1_S_R4)")
            configs[name] = leg
            if dequant is None:
                dequant = {}
            dequant[member] = dequant_leg(tm, K, mm[0], hbm)
            del mm
        dequant[MEMBER] = dequant_leg(tm, K, mods[0], hbm)
        torch.cuda.empty_cache()
        dense = dense_leg(tm, K, dev, gen, hbm)

    # the same decode steps through the fused layer module, device-timed
    layer = glu_layer(torch, dev, mods)
    gcells = [GluCell(torch, layer, c, gen, dev) for c in cells]
    switchglu = {f"B={g.B}": tm.cell_rate(g, max(50, Kst // 2)) for g in gcells}
    prefill = run_prefill(args, torch, K, dev, world, rank, tm, peaks)
    e2e = run_e2e(args, torch, dev, layer, cells, tm)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baselines(batches, args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": metric_name(batches), "value": round(value, 2), "unit": "GB/s",
            "n_gpus": world, "steps": Kst, "warmup": W,
            "ms_per_step": round(ms_max / Kst, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "s8 x s8 -> s32 MMA, f64 epilogue (bf16 activations)",
            "data": "synthetic: random IQ2_KS streams (serving scales), x~N(0,1) bf16",
            "config": config(args, batches),
            "sweep": sweep, "switchglu_sweep": switchglu, "roofline": roofline, "floors": floors,
            "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": launches_per_step * Kst,
            "clocks": clk.summary(),
            "hbm_frac_of_step": round(value / world / hbm, 4),
            "configs": configs, "dequant": dequant, "dense": dense, "prefill": prefill,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_prefill(args, torch, K, dev, world, rank, tm, peaks) -> dict | None:
    """Config 5: the expert-parallel layer at every N (experts E/N per rank,
    the 2048 tokens sharded N ways: strong scaling) with its output check,
    and at N=1 the direct one-GPU layer and each grouped GEMM alone (IQ2_KS at
    the gate shape, IQ2_K at the down shape, IQ1_S_R4 at the gate shape)."""
    if args.no_prefill:
        return None
    full = config5_modules(torch, dev)
    ep_ms, check, phases, layer = measure_ep_prefill(
        torch, K, dev, world, rank, tm.barrier, tm.max_over_ranks,
        max(5, args.prefill_steps // 2), full)
    ep = {"value": round(PREFILL_TOKENS / (ep_ms * 1e-3), 1), "unit": "tokens/s",
          "ms_per_step": round(ep_ms, 4), "ep_check": check, "phases": phases,
          "path": "ExpertParallelMoE.forward (all-to-all dispatch, SwitchGLU, combine)",
          **layer.timing}
    ep_timing = layer.timing
    del layer
    if world > 1:
        return {"metric": "prefill tokens/s (config 5 layer, expert-parallel)",
                "value": ep["value"], "unit": "tokens/s", "ms_per_step": ep["ms_per_step"],
                "tokens": PREFILL_TOKENS, "scaling": "strong", "ep_check": check,
                "phases": phases, **ep_timing, "parallelism": f"ep{world}: {E // world} "
                "experts/rank, NCCL all_to_all dispatch and combine"}
    x, idx, w = prefill_inputs(torch, dev)
    pl = PrefillLayer(torch, K, dev, full, x, idx, w)
    pl.step()
    torch.cuda.synchronize()
    ps = max(5, args.prefill_steps)
    gpw = tm.graph(lambda: [pl.step() for _ in range(3)])
    gpt = tm.graph(lambda: [pl.step() for _ in range(ps)])
    gpw.replay()
    pms = tm.timed(gpt) / ps
    reps = 10
    g, u, d = full
    gk_g = tm.graph(lambda: [K.grouped_run("iq2_ks", g._streams(), E, GATE_UP[0], GATE_UP[1],
                                           pl.pairs, pl.yg, pl.ws_gu) for _ in range(reps)])
    gk_d = tm.graph(lambda: [K.grouped_run("iq2_k", d._streams(), E, DOWN[0], DOWN[1],
                                           pl.pairs, pl.yd, pl.ws_d) for _ in range(reps)])
    pl.gate_up()
    pl.down_proj()
    gk_g.replay()
    gk_d.replay()
    g_ms = tm.timed(gk_g) / reps
    d_ms = tm.timed(gk_d) / reps
    # IQ1_S_R4 experts of the gate shape over the same routed pairs and the
    # same prepared activations (the grouped workspace is member-independent)
    from mlx_iqk_b200 import IqkSwitchLinear
    from mlx_iqk_b200.profile_cases import random_streams
    iq1 = IqkSwitchLinear("iq1_s_r4", E, *GATE_UP, device=dev)
    iq1.load_streams(random_streams("iq1_s_r4", E, *GATE_UP, dev,
                                    torch.Generator(device=dev).manual_seed(5006)))
    gk_1 = tm.graph(lambda: [K.grouped_run("iq1_s_r4", iq1._streams(), E, GATE_UP[0],
                                           GATE_UP[1], pl.pairs, pl.yg, pl.ws_gu)
                             for _ in range(reps)])
    pl.gate_up()
    gk_1.replay()
    i_ms = tm.timed(gk_1) / reps
    tf_peak = peaks.get("bf16_tflops") or 1590.0
    g_fl = 2.0 * pl.pairs * GATE_UP[0] * GATE_UP[1]
    d_fl = 2.0 * pl.pairs * DOWN[0] * DOWN[1]
    out = {
        "metric": "prefill tokens/s (config 5 layer: gate/up IQ2_KS, down IQ2_K, "
                  "256 experts top-6, sorted_indices=True)",
        "value": round(pl.T / (pms * 1e-3), 1), "unit": "tokens/s",
        "tokens_per_gpu": pl.T, "ms_per_step": round(pms, 4), "ep_layer": ep,
        "layer_tflops": round(prefill_flops(pl.pairs) / (pms * 1e-3) / 1e12, 1),
        "load": pl.load,
        "gemm": {"gate_or_up_us": round(g_ms * 1e3, 2),
                 "gate_or_up_tflops": round(g_fl / (g_ms * 1e-3) / 1e12, 1),
                 "down_us": round(d_ms * 1e3, 2),
                 "down_tflops": round(d_fl / (d_ms * 1e-3) / 1e12, 1),
                 "bound": "tensor", "peak_tflops": tf_peak,
                 "peak_source": "measured" if peaks.get("bf16_tflops") else "fallback",
                 "frac_gate_or_up": round(g_fl / (g_ms * 1e-3) / 1e12 / tf_peak, 4),
                 "frac_down": round(d_fl / (d_ms * 1e-3) / 1e12 / tf_peak, 4),
                 "iq1_s_r4_gate_shape_us": round(i_ms * 1e3, 2),
                 "iq1_s_r4_gate_shape_tflops": round(g_fl / (i_ms * 1e-3) / 1e12, 1),
                 "frac_iq1_s_r4": round(g_fl / (i_ms * 1e-3) / 1e12 / tf_peak, 4)},
        "parallelism": "one GPU",
    }
    del gpw, gpt, gk_g, gk_d, gk_1, iq1, pl, full
    torch.cuda.empty_cache()
    return out


def glu_layer(torch, dev, mods):
    """The headline layer's projections as one IqkSwitchGLU (shared streams)."""
    from mlx_iqk_b200 import IqkSwitchGLU
    layer = IqkSwitchGLU((MEMBER, MEMBER, MEMBER), E, GATE_UP[1], GATE_UP[0], device=dev)
    layer.gate, layer.up, layer.down = mods
    return layer


class GluCell:
    """One decode step of the whole SwitchGLU layer through the public module
    (IqkSwitchGLU: gate and up in one launch, SiLU * up * router weight, down,
    the router-weighted top-k sum), on a DecodeCell's rotating selections."""

    def __init__(self, torch, layer, cell, gen, dev):
        self.layer, self.cell, self.B = layer, cell, cell.B
        self.scores = torch.softmax(torch.randn((cell.pool, cell.B, TOP_K), generator=gen,
                                                device=dev), dim=-1)

    def step(self, s: int) -> None:
        p = s % self.cell.pool
        self.layer(self.cell.xs[p], self.cell.sels[p], self.scores[p])

    def bytes(self, s: int) -> int:
        return self.cell.bytes(s)


def run_e2e(args, torch, dev, layer, cells, tm) -> dict:
    """The headline step through the public API with host buffers: per batch
    size one replay of the layer's captured decode step
    (IqkSwitchGLU.graphed: gate, up, down and the router-weighted sum, the
    layer's launches in one CUDA graph over static input / output tensors).
    Every step copies its inputs (activations, routing ids, router weights)
    from pinned host memory into the step's inputs and its output back; the
    copies run on two side streams (two captured steps per batch size, used
    alternately), so step i+1's inputs upload and step i's output downloads
    while step i+1 computes -- the pipelining a server does. The timed
    region runs from the first upload to the last download."""
    stream = torch.cuda.current_stream(dev)
    ne = min(args.steps, 100)
    host, dbuf = [], []
    for c in cells:
        B = c.B
        host.append({
            "x": torch.randn((ne, B, GATE_UP[1])).to(torch.bfloat16).pin_memory(),
            # int32 routing indices, as the reference's router emits 32-bit ids
            "idx": torch.from_numpy(c.sels_np[np.arange(ne) % c.pool].astype(np.int32)).pin_memory(),
            "w": torch.softmax(torch.randn((ne, B, TOP_K)), dim=-1).pin_memory(),
            "y": torch.empty((ne, B, DOWN[0])).pin_memory()})
        steps = [layer.graphed(B, TOP_K) for _ in range(2)]
        dbuf.append([{"dx": st.x, "didx": st.indices, "dw": st.scores, "step": st}
                     for st in steps])
    up_s, down_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    in_ev = [torch.cuda.Event() for _ in range(2)]    # inputs of buffer set b landed
    free_ev = [torch.cuda.Event() for _ in range(2)]  # buffer set b's step computed
    out_ev = torch.cuda.Event()                        # the step's results written
    dl_ev = [torch.cuda.Event() for _ in range(2)]    # buffer set b's outputs read back

    def upload(i: int):
        b = i & 1
        with torch.cuda.stream(up_s):
            if i >= 2:
                up_s.wait_event(free_ev[b])
            for h, d in zip(host, dbuf):
                d[b]["dx"].copy_(h["x"][i], non_blocking=True)
                d[b]["didx"].copy_(h["idx"][i], non_blocking=True)
                d[b]["dw"].copy_(h["w"][i], non_blocking=True)
            in_ev[b].record(up_s)

    def e2e_run(n: int):
        up_s.wait_stream(stream)  # the timed region's start event comes first
        upload(0)
        for i in range(n):
            b = i & 1
            if i + 1 < n:
                upload(i + 1)
            stream.wait_event(in_ev[b])
            if i >= 2:  # the captured step's static outputs: read back from step i - 2
                stream.wait_event(dl_ev[b])
            outs = [d[b]["step"].replay() for d in dbuf]
            free_ev[b].record(stream)
            out_ev.record(stream)
            with torch.cuda.stream(down_s):
                down_s.wait_event(out_ev)
                for h, y in zip(host, outs):
                    h["y"][i].copy_(y, non_blocking=True)
                dl_ev[b].record(down_s)
        stream.wait_stream(down_s)
        stream.wait_stream(up_s)

    e2e_run(min(3, ne))  # warm-up over the first steps' buffers
    torch.cuda.synchronize()
    ems = tm.timed(_Eager(lambda: e2e_run(ne)))
    e_bytes = sum(c.bytes(i) for c in cells for i in range(ne))
    h2d = sum(c.B * GATE_UP[1] * 2 + c.B * TOP_K * 4 + c.B * TOP_K * 4 for c in cells)
    d2h = sum(c.B * DOWN[0] * 4 for c in cells)
    return {"value": round(tm.world * e_bytes / (ems * 1e-3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": round(ems / ne, 4), "steps": ne,
            "path": "IqkSwitchGLU.graphed(B, 6).replay() (the layer's decode step: gate+up "
                    "in one launch, SiLU*up*router weight, down, top-k sum, captured once) per "
                    "batch size, pinned host in/out; copies on two side streams overlapped "
                    "with the next step"}


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
    ap.add_argument("--no-legs", action="store_true",
                    help="skip the config-1/3/4 and dequantization legs")
    ap.add_argument("--experts", type=int, default=256,
                    help="experts per projection (256 = the benchmark; fewer for profiling)")
    ap.add_argument("--eager", action="store_true",
                    help="launch kernels one by one instead of replaying CUDA graphs (profiling)")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill (config 5) leg")
    ap.add_argument("--prefill-steps", type=int, default=20)
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
