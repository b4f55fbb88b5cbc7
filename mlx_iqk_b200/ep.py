"""Expert-parallel MoE layer: experts sharded over ranks, NCCL all-to-all.

The reference serves a whole layer on one device; its SwitchGLU seam
(``src/mlx_iqk/nn.py:1-22``: gate and up ``IqkSwitchLinear`` on the token,
SiLU(gate) * up, down, router-weighted sum over top-k) is what this module
shards. Rank ``r`` of ``G`` holds experts ``[r*E/G, (r+1)*E/G)`` as three
``IqkSwitchLinear`` (gate, up, down) of ``E/G`` experts each, and owns a
shard of the tokens. One forward, at a per-rank token capacity ``C``:

1. **plan** (device) -- for every token the ranks that hold any of its
   experts; its position in each such rank's send chunk (a running count);
   the rows are packed into ``[G, C]`` send chunks, one row per (token,
   destination rank) however many of the token's experts live there, with a
   metadata row of that rank's local expert ids and router weights (-1: no
   slot). Unused chunk rows carry no slot;
2. **dispatch** -- ``all_to_all_single`` of the row chunks and of the
   metadata (equal splits of ``C`` rows, so no count ever reaches the host);
3. **expert compute** on the received rows' local slots -- the grouped GEMMs
   with a shard preparation (a -1 slot is skipped), SiLU(gate) * up * router
   weight in one pass (``iqk_pairs_swiglu``; down is linear, so the weight
   goes in before it), the down GEMM, each row's sum over its slots
   (``iqk_pairs_combine``, bf16);
4. **combine** -- ``all_to_all_single`` returns each partial row to the rank
   and chunk position it came from; each token adds its destinations'
   partials in rank order in float32.

Expert indices are checked on the device: an out-of-range slot contributes
nothing and sets an error flag that :meth:`ExpertParallelMoE.check` reads
(all ranks together), so a forward issues no host read and a fixed capacity
makes it capturable in a CUDA graph, collectives included. Without a capacity
(``max_tokens=None``) the layer instead exchanges the token counts and reads
them on the host, and an out-of-range index raises on every rank before any
data moves.

No kernel reads another GPU's memory and nothing uses TMA multicast; the
collectives are the ones above, taken by every rank in the same order. The
expert computation is a parameter (``expert_fn``) only so that CPU tests can
check the plan, dispatch and combine on ``gloo`` ranks against a host
stand-in; the default -- and the only product path -- is the CUDA grouped
GEMM.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

from . import kernels as K
from .nn import IqkSwitchLinear

ExpertFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]

PHASES = ("plan", "dispatch", "experts", "combine", "sum")


class ExpertParallelMoE:
    """One SwitchGLU MoE layer with its experts sharded over a process group.

    ``members`` gives the member of (gate, up, down), e.g. the config-5 mix
    ``("iq2_ks", "iq2_ks", "iq2_k")``. ``hidden`` is the model width (the gate
    and up input, the down output) and ``inter`` the expert width.
    ``max_tokens`` is the per-rank token capacity of a forward (no host read,
    capturable); ``None`` sizes each forward from a host read of the counts.
    """

    def __init__(self, num_experts: int, hidden: int, inter: int,
                 members=("iq2_ks", "iq2_ks", "iq2_k"), group=None, device=None,
                 expert_fn: ExpertFn | None = None, max_tokens: int | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not shard over {self.world} ranks")
        if max_tokens is not None and max_tokens <= 0:
            raise ValueError(f"max_tokens {max_tokens} is not positive")
        self.num_experts = num_experts
        self.local_experts = num_experts // self.world
        self.first_expert = self.rank * self.local_experts
        self.hidden, self.inter = hidden, inter
        self.max_tokens = max_tokens
        self.device = torch.device(device) if device is not None else (
            torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available()
            else torch.device("cpu"))
        self.expert_fn = expert_fn
        if expert_fn is None:
            g, u, d = members
            self.gate = IqkSwitchLinear(g, self.local_experts, inter, hidden, device=self.device)
            self.up = IqkSwitchLinear(u, self.local_experts, inter, hidden, device=self.device)
            self.down = IqkSwitchLinear(d, self.local_experts, hidden, inter, device=self.device)
        self.last_stats: dict = {}
        self._side: dict = {}  # per device: the stream the up GEMM runs on
        self._err = torch.zeros((), dtype=torch.int32, device=self.device)

    @property
    def capturable(self) -> bool:
        """A forward issues no host read (fixed capacity, CUDA experts)."""
        return self.max_tokens is not None and self.expert_fn is None

    def check(self) -> None:
        """Raise ``IqkRuntimeError`` if any rank's forward since the last check
        met an expert index outside ``[0, num_experts)``. Collective: every
        rank calls it at the same point, and every rank raises together."""
        flag = self._err.clone().to(torch.int64)
        self._err.zero_()
        if self.world > 1:
            dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=self.group)
        if int(flag.item()):
            raise K.IqkRuntimeError("expert index outside [0, num_experts)")

    # -- expert compute --------------------------------------------------

    def local_experts_forward(self, rows: torch.Tensor, sel: torch.Tensor, w: torch.Tensor,
                              out_dtype=torch.float32) -> torch.Tensor:
        """Router-weighted SwitchGLU of ``rows [R, hidden]`` over their local slots.

        ``sel [R, k]`` int32 holds each slot's local expert (outside
        ``[0, E/G)``: no slot here, skipped) and ``w [R, k]`` its router
        weight. Returns ``[R, hidden]`` in ``out_dtype`` (rows without a local
        slot are zeros).
        """
        R, k = sel.shape
        El = self.local_experts
        if self.expert_fn is not None:
            mask = (sel >= 0) & (sel < El)
            pr, pj = mask.nonzero(as_tuple=True)
            return self.expert_fn(rows, pr, sel[pr, pj], w[pr, pj]).to(out_dtype)
        out = torch.empty((R, self.hidden), dtype=out_dtype, device=rows.device)
        P = R * k
        if P == 0:
            return out.zero_()
        s = sel.reshape(-1).contiguous()
        ws = torch.empty(K.grouped_workspace_bytes(self.hidden, El, P), dtype=torch.uint8,
                         device=rows.device)
        K.grouped_prepare(rows.contiguous(), El, self.hidden, s, None, ws, shard=True)
        g = torch.empty((P, self.inter), dtype=torch.float32, device=rows.device)
        u = torch.empty_like(g)
        # gate and up read only the prepared workspace: the up GEMM runs on a
        # side stream, so it fills the SMs the gate GEMM's last wave leaves idle
        main = torch.cuda.current_stream(rows.device)
        side = self._side_stream(rows.device)
        side.wait_stream(main)
        K.grouped_run(self.gate.member, self.gate._streams(), El, self.inter, self.hidden, P,
                      g, ws)
        with torch.cuda.stream(side):
            K.grouped_run(self.up.member, self.up._streams(), El, self.inter, self.hidden, P,
                          u, ws)
            u.record_stream(side)
            ws.record_stream(side)
        main.wait_stream(side)
        h = torch.empty((P, self.inter), dtype=torch.bfloat16, device=rows.device)
        K.pairs_swiglu(g, u, w.reshape(-1).contiguous(), self.hidden, El, ws, h)
        del g, u
        ws_d = torch.empty(K.grouped_workspace_bytes(self.inter, El, P), dtype=torch.uint8,
                           device=rows.device)
        K.grouped_prepare(h, El, self.inter, s, None, ws_d, shard=True)
        y = torch.empty((P, self.hidden), dtype=torch.float32, device=rows.device)
        K.grouped_run(self.down.member, self.down._streams(), El, self.hidden, self.inter, P,
                      y, ws_d)
        return K.pairs_combine(y, s, k, El, out)

    def _side_stream(self, dev) -> torch.cuda.Stream:
        s = self._side.get(dev)
        if s is None:
            s = self._side[dev] = torch.cuda.Stream(dev)
        return s

    # -- plan / dispatch / combine ----------------------------------------

    def forward(self, x: torch.Tensor, indices: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        """``x [T, hidden]`` (this rank's tokens), ``indices [T, k]`` global expert
        ids, ``weights [T, k]`` router weights -> ``[T, hidden]`` float32.

        Ranks may pass different token counts (at most ``max_tokens`` each
        when a capacity is set)."""
        return self._forward(x, indices, weights, None)

    __call__ = forward

    def _capacity(self, T: int, bad: torch.Tensor) -> int:
        """Without a fixed capacity: every rank's count and index flag, read on
        the host, so that every rank raises together before data moves."""
        if self.world == 1:
            if bool(bad.any()):
                raise K.IqkRuntimeError("expert index outside [0, num_experts)")
            return T
        dev = bad.device
        info = torch.stack([torch.full((), T, dtype=torch.int64, device=dev),
                            bad.any().long()])
        info_all = torch.empty(2 * self.world, dtype=torch.int64, device=dev)
        dist.all_gather_into_tensor(info_all, info, group=self.group)
        host = info_all.tolist()
        if any(host[2 * r + 1] for r in range(self.world)):
            raise K.IqkRuntimeError("expert index outside [0, num_experts)")
        return max(host[0::2])

    def _forward(self, x, indices, weights, mark) -> torch.Tensor:
        T, k = indices.shape
        G, El, E, H = self.world, self.local_experts, self.num_experts, self.hidden
        dev = x.device
        mark = mark or (lambda name: None)
        mark("plan")
        idx = indices.to(device=dev, dtype=torch.int32)
        w = weights.to(device=dev, dtype=torch.float32)
        bad = (idx < 0) | (idx >= E)
        if self.max_tokens is None:
            C = self._capacity(T, bad)
        else:
            C = self.max_tokens
            if T > C:
                raise K.IqkRuntimeError(f"{T} tokens exceed the layer's capacity {C}")
            self._err.bitwise_or_(bad.any().to(torch.int32))
        idx = torch.where(bad, torch.full_like(idx, -1), idx)
        self.last_stats = {"capacity": C, "rows_exchanged": G * C, "slots": G * C * k}
        if G == 1:
            mark("experts")
            return self.local_experts_forward(x.to(torch.bfloat16), idx, w.contiguous())
        if C == 0:
            return torch.zeros((T, H), dtype=torch.float32, device=dev)
        # this rank's rows and slots, padded to C (pad slots name no expert)
        xs = torch.zeros((C, H), dtype=torch.bfloat16, device=dev)
        xs[:T] = x
        idp = torch.full((C, k), -1, dtype=torch.int64, device=dev)
        idp[:T] = idx
        wp = torch.zeros((C, k), dtype=torch.float32, device=dev)
        wp[:T] = w
        # destination rank of each slot (G: none); one send row per (token, rank)
        dest = torch.where(idp >= 0, idp // El, torch.full_like(idp, G))
        need = torch.zeros((C, G + 1), dtype=torch.bool, device=dev)
        need.scatter_(1, dest, True)
        need = need[:, :G]
        pos = need.to(torch.int64).cumsum(0) - 1
        ranks = torch.arange(G, device=dev)
        trash = G * C  # one spare row past the chunks takes the unneeded pairs
        flat = torch.where(need, ranks * C + pos, torch.full_like(pos, trash))
        send_x = torch.empty((G * C + 1, H), dtype=torch.bfloat16, device=dev)
        send_x[flat] = xs[:, None, :]
        on = dest[:, None, :] == ranks[None, :, None]                        # [C, G, k]
        loc = torch.where(on, idp[:, None, :] - ranks[None, :, None] * El,
                          torch.full_like(idp[:, None, :], -1)).to(torch.int32)
        wb = torch.where(on, wp[:, None, :], torch.zeros_like(wp[:, None, :])).view(torch.int32)
        send_meta = torch.full((G * C + 1, 2 * k), -1, dtype=torch.int32, device=dev)
        send_meta[flat] = torch.cat([loc, wb], dim=-1)
        mark("dispatch")
        recv_x = torch.empty((G * C, H), dtype=torch.bfloat16, device=dev)
        recv_meta = torch.empty((G * C, 2 * k), dtype=torch.int32, device=dev)
        dist.all_to_all_single(recv_x, send_x[:G * C], group=self.group)
        dist.all_to_all_single(recv_meta, send_meta[:G * C], group=self.group)
        mark("experts")
        partial = self.local_experts_forward(recv_x, recv_meta[:, :k].contiguous(),
                                             recv_meta[:, k:].contiguous().view(torch.float32),
                                             torch.bfloat16)
        mark("combine")
        back = torch.empty((G * C + 1, H), dtype=torch.bfloat16, device=dev)
        back[trash].zero_()
        dist.all_to_all_single(back[:G * C], partial, group=self.group)
        mark("sum")
        return back[flat[:T]].float().sum(1)

    def profile_phases(self, x, indices, weights) -> dict | None:
        """One forward with CUDA events between its phases: ms per phase, the
        max over ranks (collective: every rank calls it)."""
        if self.device.type != "cuda":
            return None
        self._forward(x, indices, weights, None)  # warm: workspaces, first-call set-up
        torch.cuda.synchronize(self.device)
        marks = []

        def mark(name):
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            marks.append((name, ev))

        self._forward(x, indices, weights, mark)
        mark("end")
        torch.cuda.synchronize(self.device)
        names = [n for n, _ in marks[:-1]]
        ms = torch.tensor([a.elapsed_time(b) for (_, a), (_, b) in zip(marks, marks[1:])],
                          dtype=torch.float64, device=self.device)
        if self.world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX, group=self.group)
        return {n: round(float(v), 4) for n, v in zip(names, ms.tolist())}


__all__ = ["ExpertParallelMoE", "PHASES"]
