"""Run one kernel case repeatedly on ``cuda:0``, for timing and for profilers.

    python -m mlx_iqk_b200.profile_cases gemv    --member iq2_ks --batch 8   [--reps 20] [--graph]
    python -m mlx_iqk_b200.profile_cases grouped --member iq2_ks --tokens 2048
    python -m mlx_iqk_b200.profile_cases dequant --member iq2_ks [--experts 64]
    python -m mlx_iqk_b200.profile_cases layer   --tokens 2048

``layer`` is one config-5 MoE layer through ``ExpertParallelMoE`` on one GPU
(gate/up IQ2_KS, down IQ2_K, top-6 of 256 experts): both preparations, the
three grouped GEMMs, the SwiGLU and combine kernels, eager (the layer reads
its index check on the host, so it is not captured in a graph).

Each case builds random relayout streams for 256 experts (the benchmark
geometry: [2048, 4096] for gate-shaped, [4096, 2048] for down-shaped
projections), runs two untimed calls, then ``--reps`` timed calls, and prints
one line with the mean time per call (CUDA events) and the case's
algorithmic bytes or flops. Inputs are larger than L2 unless a case says
otherwise. Nothing here is on the product path.
"""

from __future__ import annotations

import argparse
import json

import torch

from . import kernels as K
from .format import component_shapes
from .nn import IqkSwitchLinear

E_DEFAULT = 256
ROW_BYTES = {"iq2_ks": lambda n: 2 + 70 * (n // 256), "iq2_k": lambda n: 76 * (n // 256),
             "iq1_s_r4": lambda n: 2 + 6 * (n // 32)}


_STREAM_DTYPES = {"uint8": torch.uint8, "uint16": torch.uint16, "uint32": torch.uint32,
                  "float16": torch.float16}


def random_streams(member: str, experts: int, out: int, n: int, dev, gen) -> dict:
    """Uniform random relayout streams on the device (every code, scale and
    grid byte uniform), f16 scales at the magnitudes the codec produces."""
    from .format import component_dtypes
    dtypes = component_dtypes(member)
    streams = {}
    for name, shape in component_shapes(member, experts, out, n).items():
        if name == "dv":
            mag = torch.rand(shape, generator=gen, device=dev) * 8e-4 + 2e-5
            sign = torch.where(torch.rand(shape, generator=gen, device=dev) < 0.5, -1.0, 1.0)
            streams[name] = (mag * sign).to(torch.float16)
            continue
        dt = _STREAM_DTYPES[dtypes[name].name]
        count = 1
        for s in shape:
            count *= s
        raw = torch.randint(0, 256, (count * dt.itemsize,), generator=gen, device=dev,
                            dtype=torch.uint8)
        streams[name] = raw.view(dt).reshape(shape)
    return streams


def random_dense_streams(member: str, out: int, n: int, dev, gen) -> dict:
    """Uniform random dense-member streams on the device, block scales at
    serving magnitudes (float32 row scale for ``iq4_ks``)."""
    from .format import dense_component_shapes
    streams = {}
    for name, shape in dense_component_shapes(member, out, n).items():
        if name == "dv":
            mag = torch.rand(shape, generator=gen, device=dev) * 8e-4 + 2e-5
            sign = torch.where(torch.rand(shape, generator=gen, device=dev) < 0.5, -1.0, 1.0)
            streams[name] = (mag * sign).to(torch.float32 if member == "iq4_ks" else torch.float16)
            continue
        dt = torch.uint32 if name in ("qs", "qh") else torch.uint8
        count = 1
        for s_ in shape:
            count *= s_
        raw = torch.randint(0, 256, (count * dt.itemsize,), generator=gen, device=dev,
                            dtype=torch.uint8)
        streams[name] = raw.view(dt).reshape(shape)
    return streams


def random_module(member: str, experts: int, out: int, n: int, dev, gen) -> IqkSwitchLinear:
    mod = IqkSwitchLinear(member, experts, out, n, device=dev)
    mod.load_streams(random_streams(member, experts, out, n, dev, gen))
    return mod


def timed(fn, reps: int, graph: bool = False) -> float:
    """Mean ms per call. With ``graph`` the ``reps`` calls are captured in one
    CUDA graph first, so host launch cost does not hide short kernels."""
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    run = fn
    if graph:
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
            for _ in range(reps):
                fn()
        torch.cuda.current_stream().wait_stream(s)
        g.replay()
        torch.cuda.synchronize()
        run = g.replay
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    if graph:
        run()
    else:
        for _ in range(reps):
            run()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / reps


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=("gemv", "grouped", "dequant", "layer", "step", "dense"))
    ap.add_argument("--member", default="iq2_ks")
    ap.add_argument("--batch", type=int, default=8, help="gemv: tokens (top-6 each)")
    ap.add_argument("--tokens", type=int, default=2048, help="grouped: tokens (top-6 each)")
    ap.add_argument("--experts", type=int, default=E_DEFAULT)
    ap.add_argument("--width", type=int, default=4096, help="in_features (2048 or 4096)")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--graph", action="store_true",
                    help="time the calls replayed from one CUDA graph (no host launch cost)")
    ap.add_argument("--floor", action="store_true",
                    help="gemv / dequant: run the kernel's address floor instead")
    ap.add_argument("--rotate", type=int, default=1,
                    help="gemv: routings prepared up front and cycled, so that the weights "
                         "do not stay in L2 across calls")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(11)
    n = args.width
    out = 2048 if n == 4096 else 4096
    E = args.experts
    if args.case == "layer":
        from .ep import ExpertParallelMoE
        T = args.tokens
        layer = ExpertParallelMoE(E, 4096, 2048, members=("iq2_ks", "iq2_ks", "iq2_k"),
                                  device=dev)
        for name in ("gate", "up", "down"):
            m = getattr(layer, name)
            setattr(layer, name, random_module(m.member, E, m.out_features, m.in_features,
                                               dev, gen))
        x = torch.randn((T, 4096), generator=gen, device=dev).to(torch.bfloat16)
        top = torch.topk(torch.randn((T, E), generator=gen, device=dev), 6, dim=-1)
        w = torch.softmax(top.values, dim=-1)
        ms = timed(lambda: layer(x, top.indices, w), args.reps)
        P = T * 6
        flops = 2.0 * P * (2 * 2048 * 4096 + 4096 * 2048)
        print(json.dumps({"case": "layer", "experts": E, "tokens": T, "pairs": P,
                          "us": round(ms * 1e3, 2), "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
                          "tokens_per_s": round(T / (ms * 1e-3), 1)}))
        return
    if args.case == "dense":
        # the dense decode GEMV at the lm_head shape ([129280, 4096], --batch
        # tokens) for --member (a dense member)
        from . import dense as dn
        from .format import ik_row_bytes
        m, out_d, n_d = args.member, 129280, 4096
        st = dn.check_dense_streams(m, random_dense_streams(m, out_d, n_d, dev, gen), out_d, n_d)
        x = torch.randn((args.batch, n_d), generator=gen, device=dev).half()
        y = torch.empty((args.batch, out_d), dtype=torch.float16, device=dev)
        ms = timed(lambda: K.dense_gemv(m, x, st, out_d, n_d, y), args.reps, args.graph)
        nbytes = out_d * ik_row_bytes(m, n_d)
        print(json.dumps({"case": "dense", "member": m, "out": out_d, "in": n_d,
                          "tokens": args.batch, "us": round(ms * 1e3, 2), "bytes": nbytes,
                          "GBps": round(nbytes / (ms * 1e-3) / 1e9, 1)}))
        return
    if args.case == "step":
        # one SwitchGLU decode step (gate, up, SiLU * up * weight, down, top-k
        # sum) through IqkSwitchGLU, routings rotated so weights leave L2
        from .glu import IqkSwitchGLU
        B, m = args.batch, args.member
        layer = IqkSwitchGLU((m, m, m), E, 4096, 2048, device=dev)
        for mm in (layer.gate, layer.up, layer.down):
            mm.load_streams(random_streams(m, E, mm.out_features, mm.in_features, dev, gen))
        R = max(1, args.rotate)
        xs = torch.randn((R, B, 4096), generator=gen, device=dev).to(torch.bfloat16)
        sels = torch.stack([torch.stack([torch.randperm(E, generator=gen, device=dev)[:6]
                                         for _ in range(B)]) for _ in range(R)])
        ws_ = torch.softmax(torch.randn((R, B, 6), generator=gen, device=dev), dim=-1)
        calls = {"i": 0}

        def one():
            i = calls["i"] % R
            calls["i"] += 1
            layer(xs[i], sels[i], ws_[i])

        ms = timed(one, args.reps, args.graph)
        distinct = sum(len(set(sels[i].reshape(-1).tolist())) for i in range(R)) / R
        rbm = ROW_BYTES[m]
        nbytes = int(distinct * (2 * 2048 * rbm(4096) + 4096 * rbm(2048)))
        print(json.dumps({"case": "step", "member": m, "batch": B, "distinct_experts": distinct,
                          "us": round(ms * 1e3, 2), "bytes": nbytes,
                          "GBps": round(nbytes / (ms * 1e-3) / 1e9, 1)}))
        return
    mod = random_module(args.member, E, out, n, dev, gen)
    rb = ROW_BYTES[args.member](n)
    line = {"case": args.case, "member": args.member, "experts": E, "out": out, "in": n}
    if args.case == "gemv":
        B = args.batch
        run = K.gemv_floor_run if args.floor else K.gemv_run
        wss, distincts = [], []
        for _ in range(max(1, args.rotate)):
            x = torch.randn((B, n), generator=gen, device=dev).to(torch.bfloat16)
            sel = torch.stack([torch.randperm(E, generator=gen, device=dev)[:6]
                               for _ in range(B)])
            sel = sel.reshape(-1).to(torch.int32)
            ws = torch.empty(K.gemv_workspace_bytes(args.member, n, B, B * 6),
                             dtype=torch.uint8, device=dev)
            K.gemv_prepare(x, E, n, sel, None, ws)
            wss.append(ws)
            distincts.append(len(set(sel.tolist())))
        y = torch.empty((B * 6, out), device=dev)
        calls = {"i": 0}

        def one():
            ws = wss[calls["i"] % len(wss)]
            calls["i"] += 1
            run(args.member, mod._streams(), E, out, n, B, B * 6, y, ws)

        ms = timed(one, args.reps, args.graph)
        distinct = sum(distincts) / len(distincts)
        nbytes = int(distinct * out * rb + B * n * 2 + B * 6 * out * 4)
        line.update(batch=B, distinct_experts=distinct, floor=args.floor, rotate=args.rotate,
                    us=round(ms * 1e3, 2),
                    bytes=nbytes, GBps=round(nbytes / (ms * 1e-3) / 1e9, 1),
                    note="run kernel only (prepared once); weights are L2-hot across reps "
                         "when distinct experts x rows x row bytes < 126 MB")
    elif args.case == "grouped":
        T = args.tokens
        x = torch.randn((T, n), generator=gen, device=dev).to(torch.bfloat16)
        logits = torch.randn((T, E), generator=gen, device=dev)
        sel = torch.topk(logits, 6, dim=-1).indices.to(torch.int32).reshape(-1).contiguous()
        P = sel.numel()
        y = torch.empty((P, out), device=dev)
        ws = torch.empty(K.grouped_workspace_bytes(n, E, P), dtype=torch.uint8, device=dev)
        K.grouped_prepare(x, E, n, sel, None, ws)
        ms = timed(lambda: K.grouped_run(args.member, mod._streams(), E, out, n, P, y, ws),
                   args.reps, args.graph)
        flops = 2.0 * P * out * n
        line.update(tokens=T, pairs=P, us=round(ms * 1e3, 2),
                    tflops=round(flops / (ms * 1e-3) / 1e12, 1))
    else:
        y = torch.empty((E, out, n), dtype=torch.float16, device=dev)
        fn = K.dequant_floor if args.floor else K.dequant
        ms = timed(lambda: fn(args.member, mod._streams(), E, out, n, 0, out, y),
                   args.reps, args.graph)
        nbytes = E * out * rb + E * out * n * 2
        line.update(us=round(ms * 1e3, 2), bytes=nbytes,
                    GBps=round(nbytes / (ms * 1e-3) / 1e9, 1))
    print(json.dumps(line))


if __name__ == "__main__":
    main()
