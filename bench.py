"""Routed-decode benchmark: IQ2_KS, 256 experts, top-6.

One step = one MoE layer's routed projections for a batch of B decode
tokens: gate and up ([2048, 4096] per expert) and down ([4096, 2048] per
expert), each through the fused dequant+GEMV kernels of libiqk_b200.so. The
gate and up projections share one preparation (iqk_gemv_prepare), the down
projection gets its own (one activation row per pair).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl reference]

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

def cpu_path(batch: int, steps: int, seconds: float, seed: int) -> dict:
    """The reference's CPU path on sampled decode steps: ik's dequantizer on
    the selected experts' wire rows, then a float32 matvec, all host cores."""
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

    sels = make_selections(min(max(steps, 1), 256), batch, 1, seed)
    rng = np.random.default_rng(seed + 1)
    pool = ThreadPoolExecutor(max_workers=cores)

    def one(args):
        proj, e, xs = args
        out, n = GATE_UP if proj != "down" else DOWN
        w = deq(MEMBER, wire_for(proj, e), n)
        return w @ xs.T

    done, total_bytes, t_all = 0, 0.0, 0.0
    for s in range(steps):
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
            "sample": f"{done} decode steps (B={batch}, gate+up+down of the selected experts): "
                      f"ik dequantize + float32 numpy matvec, {cores} threads",
            "ms_per_step": 1e3 * t_all / max(done, 1)}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    warm = cpu_path(args.batch, max(1, min(args.warmup, 2)), 1e9, seed=99)
    del warm
    res = cpu_path(args.batch, args.steps, args.cpu_seconds * 6, seed=1234)
    line = {
        "impl": "reference", "metric": metric_name(args.batch), "value": round(res["value"], 4),
        "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(res["ms_per_step"], 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 dequant, f32 matvec",
        "data": "synthetic", "config": config(args),
        "cpu_baseline": {"value": round(res["value"], 4), "unit": "GB/s", "cores": res["cores"],
                         "kind": res["kind"], "sample": res["sample"]},
        "e2e": {"value": round(res["value"], 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- GPU

def metric_name(batch: int) -> str:
    return (f"routed decode GB/s (IQ2_KS, 256 experts top-6, gate+up+down, B={batch})")


def config(args) -> dict:
    return {"workload": "BASELINE configs[1]: IQ2_KS routed decode, 256 experts top-6",
            "member": MEMBER, "experts": E, "top_k": TOP_K, "gate_up": list(GATE_UP),
            "down": list(DOWN), "batch": args.batch,
            "l2": "rotating selections: no expert recurs within a window of > 2x L2 bytes",
            "parallelism": f"replicas x{args.gpus}"}


def random_streams(torch, out: int, n: int, gen, dev):
    """Uniform random IQ2_KS relayout streams on the device, serving scales."""
    def u8(count):
        return torch.randint(0, 256, (count,), generator=gen, device=dev, dtype=torch.uint8)
    s = {"qs": u8(E * out * n // 4).view(torch.uint32).reshape(E, out, n // 16),
         "scl": u8(E * out * n // 64).reshape(E, out, n // 64),
         "sch": u8(E * out * n // 256).reshape(E, out, n // 256),
         "sex": u8(E * out * n // 256).reshape(E, out, n // 256)}
    mag = torch.rand((E, out), generator=gen, device=dev) * 8e-4 + 2e-5
    sign = torch.where(torch.rand((E, out), generator=gen, device=dev) < 0.5, -1.0, 1.0)
    s["dv"] = (mag * sign).to(torch.float16)
    return s


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

    B = args.batch
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    gate = IqkSwitchLinear(MEMBER, E, *GATE_UP, device=dev)
    up = IqkSwitchLinear(MEMBER, E, *GATE_UP, device=dev)
    down = IqkSwitchLinear(MEMBER, E, *DOWN, device=dev)
    for mod in (gate, up, down):
        mod.load_streams(random_streams(torch, mod.out_features, mod.in_features, gen, dev))

    window = max(1, math.ceil(2 * L2_BYTES / expert_bytes_per_step(B)))
    pool = 128
    sels_np = make_selections(pool, B, window, seed=7 + rank)
    sels = torch.from_numpy(sels_np).to(dev, torch.int32)
    xs = torch.randn((pool, B, GATE_UP[1]), generator=gen, device=dev).to(torch.bfloat16)
    xds = torch.randn((pool, B * TOP_K, DOWN[1]), generator=gen, device=dev).to(torch.bfloat16)
    step_bytes = []
    rb_gu, rb_d = row_bytes(MEMBER, GATE_UP[1]), row_bytes(MEMBER, DOWN[1])
    act_bytes = (B * GATE_UP[1] * 2 + B * TOP_K * DOWN[1] * 2            # x, x_down (bf16)
                 + B * TOP_K * (2 * GATE_UP[0] + DOWN[0]) * 4)            # y (f32)
    for s in range(pool):
        d = len(set(sels_np[s].ravel().tolist()))
        step_bytes.append(d * (2 * GATE_UP[0] * rb_gu + DOWN[0] * rb_d) + act_bytes)
    pairs = B * TOP_K
    ws_gu = torch.empty(K.gemv_workspace_bytes(MEMBER, GATE_UP[1], B, pairs), dtype=torch.uint8,
                        device=dev)
    ws_d = torch.empty(K.gemv_workspace_bytes(MEMBER, DOWN[1], pairs, pairs), dtype=torch.uint8,
                       device=dev)
    yg = torch.empty((pairs, GATE_UP[0]), device=dev)
    yu = torch.empty((pairs, GATE_UP[0]), device=dev)
    yd = torch.empty((pairs, DOWN[0]), device=dev)
    sg, su, sd = gate._streams(), up._streams(), down._streams()

    def step(s: int) -> None:
        p = s % pool
        K.gemv_prepare(xs[p], E, GATE_UP[1], sels[p].reshape(-1), None, ws_gu)
        K.gemv_run(MEMBER, sg, E, GATE_UP[0], GATE_UP[1], B, pairs, yg, ws_gu)
        K.gemv_run(MEMBER, su, E, GATE_UP[0], GATE_UP[1], B, pairs, yu, ws_gu)
        K.gemv_prepare(xds[p], E, DOWN[1], sels[p].reshape(-1), None, ws_d)
        K.gemv_run(MEMBER, sd, E, DOWN[0], DOWN[1], pairs, pairs, yd, ws_d)

    launches_per_step = 5
    step(0)
    torch.cuda.synchronize()

    def capture(n_steps: int, first: int):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for s in range(first, first + n_steps):
                step(s)
        return g

    W, Kst = args.warmup, args.steps
    if args.eager:
        # no CUDA graphs (profiler runs): the same launches, issued one by one
        class _Eager:
            def __init__(self, fn):
                self.fn = fn

            def replay(self):
                self.fn()
        g_warm = _Eager(lambda: [step(s) for s in range(W)])
        g_time = _Eager(lambda: [step(s) for s in range(W, W + Kst)])
    else:
        g_warm = capture(W, 0)
        g_time = capture(Kst, W)
    g_warm.replay()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(local) as clk:
        e0.record(stream)
        g_time.replay()
        e1.record(stream)
        e1.synchronize()
    barrier()
    ms = e0.elapsed_time(e1)
    ms_t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    bytes_timed = sum(step_bytes[s % pool] for s in range(W, W + Kst))
    value = world * bytes_timed / (ms_max * 1e-3) / 1e9

    # ---- kernel-only roofline: the gate GEMV run over pre-prepared routings
    nr = min(pool, 64)
    wss = [torch.empty_like(ws_gu) for _ in range(nr)]
    for i in range(nr):
        K.gemv_prepare(xs[i], E, GATE_UP[1], sels[i].reshape(-1), None, wss[i])
    reps = max(2, Kst // nr)

    def kernel_loop():
        for r in range(reps):
            for i in range(nr):
                K.gemv_run(MEMBER, sg, E, GATE_UP[0], GATE_UP[1], B, pairs, yg, wss[i])
    if args.eager:
        gk = _Eager(kernel_loop)
    else:
        gk = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gk):
            kernel_loop()
    gk.replay()
    torch.cuda.synchronize()
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0.record(stream)
    gk.replay()
    k1.record(stream)
    k1.synchronize()
    kms = k0.elapsed_time(k1) / (reps * nr)
    gate_bytes = np.mean([len(set(sels_np[i].ravel().tolist())) * GATE_UP[0] * rb_gu
                          + B * GATE_UP[1] * 2 + pairs * GATE_UP[0] * 4 for i in range(nr)])
    peaks = {}
    try:
        peaks = json.loads((REPO / "MEASURED_PEAKS.json").read_text())
    except Exception:  # noqa: BLE001
        pass
    hbm = peaks.get("hbm_gbs")
    peak_src = "measured" if hbm else "fallback"
    hbm = hbm or 6650.0
    achieved = gate_bytes / (kms * 1e-3) / 1e9
    roofline = {"bound": "hbm", "kernel": "gemv_kernel<IQ2_KS> (gate, 2048x4096)",
                "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(achieved / hbm, 4), "peak_source": peak_src,
                "us_per_launch": round(kms * 1e3, 3),
                "bytes_per_launch": int(gate_bytes),
                "traffic": args.traffic}

    # ---- end to end through the public module API, host buffers
    ne = min(Kst, 200)
    hx = torch.randn((ne, B, 1, 1, GATE_UP[1])).to(torch.bfloat16).pin_memory()
    hxd = torch.randn((ne, B, TOP_K, 1, DOWN[1])).to(torch.bfloat16).pin_memory()
    hidx = torch.from_numpy(sels_np[np.arange(ne) % pool]).pin_memory()
    hyg = torch.empty((ne, B, TOP_K, 1, GATE_UP[0])).pin_memory()
    hyu = torch.empty((ne, B, TOP_K, 1, GATE_UP[0])).pin_memory()
    hyd = torch.empty((ne, B, TOP_K, 1, DOWN[0])).pin_memory()
    dx = torch.empty((B, 1, 1, GATE_UP[1]), device=dev, dtype=torch.bfloat16)
    dxd = torch.empty((B, TOP_K, 1, DOWN[1]), device=dev, dtype=torch.bfloat16)
    didx = torch.empty((B, TOP_K), device=dev, dtype=torch.int64)

    def e2e_step(i: int):
        dx.copy_(hx[i], non_blocking=True)
        dxd.copy_(hxd[i], non_blocking=True)
        didx.copy_(hidx[i], non_blocking=True)
        hyg[i].copy_(gate(dx, didx), non_blocking=True)
        hyu[i].copy_(up(dx, didx), non_blocking=True)
        hyd[i].copy_(down(dxd, didx), non_blocking=True)

    for i in range(3):
        e2e_step(i)
    barrier()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record(stream)
    for i in range(ne):
        e2e_step(i)
    x1.record(stream)
    x1.synchronize()
    ems_t = torch.tensor([x0.elapsed_time(x1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ems_t, op=dist.ReduceOp.MAX)
    ems = float(ems_t.item())
    e_bytes = sum(step_bytes[i % pool] for i in range(ne))
    h2d = B * GATE_UP[1] * 2 + B * TOP_K * DOWN[1] * 2 + B * TOP_K * 8
    d2h = B * TOP_K * (2 * GATE_UP[0] + DOWN[0]) * 4
    e2e = {"value": round(world * e_bytes / (ems * 1e-3) / 1e9, 2), "unit": "GB/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
           "ms_per_step": round(ems / ne, 4), "steps": ne,
           "path": "IqkSwitchLinear.__call__ x3 per step, pinned host in/out"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        res = cpu_path(B, 10 ** 6, args.cpu_seconds, seed=4321)
        cpu = {k: (round(v, 4) if isinstance(v, float) else v) for k, v in res.items()
               if k in ("value", "unit", "cores", "kind", "sample")}

    if rank == 0:
        line = {
            "metric": metric_name(B), "value": round(value, 2), "unit": "GB/s",
            "n_gpus": world, "steps": Kst, "warmup": W,
            "ms_per_step": round(ms_max / Kst, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "s8 x s8 -> s32 MMA, f64 epilogue (bf16 activations)",
            "data": "synthetic: random IQ2_KS streams (serving scales), x~N(0,1) bf16",
            "config": config(args),
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": launches_per_step * Kst,
            "clocks": clk.summary(),
            "hbm_frac_of_step": round(value / world / hbm, 4),
        }
        print(json.dumps(line), flush=True)
    del g_warm, g_time, gk
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", default="b200", choices=("b200", "reference"))
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--experts", type=int, default=256,
                    help="experts per projection (256 = the benchmark; fewer for profiling)")
    ap.add_argument("--eager", action="store_true",
                    help="launch kernels one by one instead of replaying CUDA graphs (profiling)")
    ap.add_argument("--traffic", type=float, default=None,
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
