"""Expert-parallel MoE layer: experts sharded over ranks, NCCL collectives.

The reference serves a whole layer on one device; its SwitchGLU seam
(``src/mlx_iqk/nn.py:1-22``: gate and up ``IqkSwitchLinear`` on the token,
SiLU(gate) * up, down, router-weighted sum over top-k) is what this module
shards. Rank ``r`` of ``G`` holds experts ``[r*E/G, (r+1)*E/G)`` as three
``IqkSwitchLinear`` (gate, up, down) of ``E/G`` experts each, and owns a
shard of the tokens. One forward:

1. **check** -- one tiny ``all_gather`` of every rank's token count and
   out-of-range-index flag, read on the host (the call's only host read), so
   that every rank raises together, before any data moves, and all ranks pad
   to the same token count ``Tc``;
2. **dispatch** -- ``all_gather_into_tensor`` of the bf16 token rows and of
   the routing slots (global expert id and router weight bits per slot):
   fixed sizes, so nothing else waits for the host. Every rank sees every
   token; with top-6 of 256 experts a token needs a given one of 2 ranks with
   probability 0.98, so a per-rank deduplication would save little;
3. **expert compute** on the local slots only -- the grouped GEMMs run on
   all ``G*Tc*k`` slots with a shard preparation
   (``iqk_grouped_prepare_shard``: another rank's expert is skipped, not an
   error), SiLU(gate) * up * router weight in one pass over the routed pairs
   (``iqk_pairs_swiglu``; the down projection is linear, so the weight goes
   in before it), the down GEMM, and each row's sum over its local slots in
   a fixed order (``iqk_pairs_combine``, bf16 out);
4. **combine** -- ``all_to_all_single`` with equal splits sends each rank's
   partial rows of rank ``s``'s tokens to ``s``, which adds the ``G``
   partials in float32.

With a single rank there is no collective: the index check is the host read
and the same expert kernels run on the rank's own slots.

No kernel reads another GPU's memory; the collectives are the ones above,
taken by every rank in the same order. The expert computation is a parameter
(``expert_fn``) only so that CPU tests can check the dispatch and combine
logic on ``gloo`` ranks against a host stand-in; the default -- and the only
product path -- is the CUDA grouped GEMM.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

from . import kernels as K
from .nn import IqkSwitchLinear

ExpertFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]


class ExpertParallelMoE:
    """One SwitchGLU MoE layer with its experts sharded over a process group.

    ``members`` gives the member of (gate, up, down), e.g. the config-5 mix
    ``("iq2_ks", "iq2_ks", "iq2_k")``. ``hidden`` is the model width (the gate
    and up input, the down output) and ``inter`` the expert width.
    """

    def __init__(self, num_experts: int, hidden: int, inter: int,
                 members=("iq2_ks", "iq2_ks", "iq2_k"), group=None, device=None,
                 expert_fn: ExpertFn | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not shard over {self.world} ranks")
        self.num_experts = num_experts
        self.local_experts = num_experts // self.world
        self.first_expert = self.rank * self.local_experts
        self.hidden, self.inter = hidden, inter
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

    # -- expert compute --------------------------------------------------

    def local_experts_forward(self, rows: torch.Tensor, sel: torch.Tensor, w: torch.Tensor,
                              out_dtype=torch.float32) -> torch.Tensor:
        """Router-weighted SwitchGLU of ``rows [R, hidden]`` over their local slots.

        ``sel [R, k]`` int32 holds each slot's local expert (outside
        ``[0, E/G)``: another rank's, skipped) and ``w [R, k]`` its router
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

    # -- dispatch / combine ----------------------------------------------

    def forward(self, x: torch.Tensor, indices: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        """``x [T, hidden]`` (this rank's tokens), ``indices [T, k]`` global expert
        ids, ``weights [T, k]`` router weights -> ``[T, hidden]`` float32.

        Ranks may pass different token counts; an expert index outside
        ``[0, num_experts)`` on any rank raises ``IqkRuntimeError`` on every
        rank before any data is exchanged.
        """
        T, k = indices.shape
        G, El, E = self.world, self.local_experts, self.num_experts
        dev = x.device
        idx = indices.to(device=dev, dtype=torch.int32)
        w = weights.to(device=dev, dtype=torch.float32).contiguous()
        bad = ((idx < 0) | (idx >= E)).any()
        if G == 1:
            if bool(bad):
                raise K.IqkRuntimeError("expert index outside [0, num_experts)")
            self.last_stats = {"rows_gathered": T, "slots": T * k}
            return self.local_experts_forward(x.to(torch.bfloat16), idx, w)

        info = torch.stack([torch.full((), T, dtype=torch.int64, device=dev), bad.long()])
        info_all = torch.empty(2 * G, dtype=torch.int64, device=dev)
        dist.all_gather_into_tensor(info_all, info, group=self.group)
        host = info_all.tolist()                                         # the one host read
        if any(host[2 * r + 1] for r in range(G)):
            raise K.IqkRuntimeError("expert index outside [0, num_experts)")
        Tc = max(host[0::2])
        self.last_stats = {"rows_gathered": G * Tc, "slots": G * Tc * k}
        if Tc == 0:
            return torch.zeros((T, self.hidden), dtype=torch.float32, device=dev)
        # this rank's rows and slots, padded to Tc (pad slots name no expert)
        xs = torch.zeros((Tc, self.hidden), dtype=torch.bfloat16, device=dev)
        xs[:T] = x
        meta = torch.full((Tc, 2 * k), -1, dtype=torch.int32, device=dev)
        meta[:T, :k] = idx
        meta[:T, k:] = w.view(torch.int32)
        x_all = torch.empty((G * Tc, self.hidden), dtype=torch.bfloat16, device=dev)
        meta_all = torch.empty((G * Tc, 2 * k), dtype=torch.int32, device=dev)
        dist.all_gather_into_tensor(x_all, xs, group=self.group)
        dist.all_gather_into_tensor(meta_all, meta, group=self.group)
        sel = meta_all[:, :k] - self.first_expert                        # local expert or foreign
        w_all = meta_all[:, k:].contiguous().view(torch.float32)
        partial = self.local_experts_forward(x_all, sel, w_all, torch.bfloat16)
        back = torch.empty_like(partial)
        dist.all_to_all_single(back, partial, group=self.group)
        return back.view(G, Tc, self.hidden)[:, :T].float().sum(0)

    __call__ = forward


__all__ = ["ExpertParallelMoE"]
