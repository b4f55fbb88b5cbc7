"""Expert-parallel MoE layer: experts sharded over ranks, NCCL all-to-all.

The reference serves a whole layer on one device; its SwitchGLU seam
(``src/mlx_iqk/nn.py:1-22``: gate and up ``IqkSwitchLinear`` on the token,
SiLU(gate) * up, down, router-weighted sum over top-k) is what this module
shards. Rank ``r`` of ``G`` holds experts ``[r*E/G, (r+1)*E/G)`` as three
``IqkSwitchLinear`` (gate, up, down) of ``E/G`` experts each, and owns a
shard of the tokens. One forward:

1. **dispatch** -- every token row goes once to every rank that holds at
   least one of its experts (deduplicated per (token, rank)), with the list
   of (row, local expert, router weight) pairs that need it:
   ``all_to_all_single`` of the split counts, then of the rows (bf16) and of
   the pair records (one int64 record per pair, the weight as its f32 bits);
2. **expert compute** on the receiving rank -- grouped GEMM of gate and up
   over the received pairs (``iqk_grouped_gemm`` with explicit rows),
   SiLU(gate) * up scaled by the pair's router weight (the down projection
   is linear, so the weight can go in before it), grouped GEMM of down, and
   the sum of each row's pairs;
3. **combine** -- one row per (token, rank) travels back the reverse way and
   is added into the token's output.

All routing arithmetic runs on the device; the host reads the split counts
once per call (that read also carries the out-of-range index check). With a
single rank there is no exchange and no gather.

No kernel reads another GPU's memory; the only collectives are the four
``all_to_all_single`` exchanges (counts, rows, pair records, result rows),
and every rank takes them in the same order. The expert computation is a
parameter (``expert_fn``) only so that CPU tests can check the dispatch and
combine logic on ``gloo`` ranks against a host stand-in; the default -- and
the only product path -- is the CUDA grouped GEMM.
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
        self._tok_cache: dict = {}

    # -- expert compute --------------------------------------------------

    def local_experts_forward(self, rows: torch.Tensor, pair_row: torch.Tensor,
                              pair_expert: torch.Tensor, pair_weight: torch.Tensor) -> torch.Tensor:
        """Router-weighted SwitchGLU of the received rows: ``[R, hidden]`` float32.

        ``pair_row[p]`` is the row the pair reads, ``pair_expert[p]`` its local
        expert and ``pair_weight[p]`` its router weight.
        """
        if self.expert_fn is not None:
            return self.expert_fn(rows, pair_row, pair_expert, pair_weight)
        R, P = rows.shape[0], pair_row.numel()
        out = torch.zeros((R, self.hidden), dtype=torch.float32, device=rows.device)
        if P == 0:
            return out
        sel = pair_expert.to(torch.int32).contiguous()
        tok = pair_row.to(torch.int32).contiguous()
        x = rows.contiguous()
        g = torch.empty((P, self.inter), dtype=torch.float32, device=rows.device)
        u = torch.empty_like(g)
        ws = torch.empty(K.grouped_workspace_bytes(self.hidden, self.local_experts, P),
                         dtype=torch.uint8, device=rows.device)
        K.grouped_prepare(x, self.local_experts, self.hidden, sel, tok, ws)
        K.grouped_run(self.gate.member, self.gate._streams(), self.local_experts, self.inter,
                      self.hidden, P, g, ws)
        K.grouped_run(self.up.member, self.up._streams(), self.local_experts, self.inter,
                      self.hidden, P, u, ws)
        # SiLU(gate) * up, with the router weight folded in before the down
        # projection (it is linear: w * (Wd h) == Wd (w * h)), so its output
        # needs no weighted copy.
        torch.nn.functional.silu(g, inplace=True)
        g.mul_(u).mul_(pair_weight.to(device=g.device, dtype=torch.float32).unsqueeze(1))
        h = g.to(torch.bfloat16)
        del g, u
        y = torch.empty((P, self.hidden), dtype=torch.float32, device=rows.device)
        ws_d = torch.empty(K.grouped_workspace_bytes(self.inter, self.local_experts, P),
                           dtype=torch.uint8, device=rows.device)
        K.grouped(self.down.member, h, self.down._streams(), self.local_experts, self.hidden,
                  self.inter, sel, None, y, ws_d)
        out.index_add_(0, pair_row.long(), y)
        return out

    # -- dispatch / combine ----------------------------------------------

    def _exchange(self, send: torch.Tensor, send_counts: list[int], recv_counts: list[int]):
        recv = torch.empty((sum(recv_counts),) + tuple(send.shape[1:]), dtype=send.dtype,
                           device=send.device)
        dist.all_to_all_single(recv, send.contiguous(), recv_counts, send_counts,
                               group=self.group)
        return recv

    def _token_index(self, T: int, k: int, dev) -> torch.Tensor:
        """pair -> token for token-major [T, k] routing (cached per shape)."""
        key = (T, k, str(dev))
        t = self._tok_cache.get(key)
        if t is None:
            if len(self._tok_cache) >= 8:
                self._tok_cache.clear()
            t = torch.arange(T, device=dev).repeat_interleave(k)
            self._tok_cache[key] = t
        return t

    def forward(self, x: torch.Tensor, indices: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        """``x [T, hidden]`` (this rank's tokens), ``indices [T, k]`` global expert
        ids, ``weights [T, k]`` router weights -> ``[T, hidden]`` float32.

        All routing arithmetic stays on the device; the host reads the split
        counts (and whether any index was out of range) once per call.
        """
        T, k = indices.shape
        G, El, E = self.world, self.local_experts, self.num_experts
        dev = x.device
        idx_in = indices.to(device=dev, dtype=torch.int64).reshape(-1)   # [T*k], token-major
        idx = idx_in.clamp(0, E - 1)                                     # keeps every index in range
        w = weights.to(device=dev, dtype=torch.float32).reshape(-1)
        tok = self._token_index(T, k, dev)                               # pair -> token
        if G == 1:
            # every token's rows stay here: no dispatch gathers, no exchange
            if bool((idx != idx_in).any()):
                raise K.IqkRuntimeError("expert index outside [0, num_experts)")
            y = self.local_experts_forward(x.to(torch.bfloat16), tok, idx, w)
            self.last_stats = {"rows_sent": T, "pairs_sent": T * k, "rows_received": T,
                               "pairs_received": T * k}
            return y

        dest = torch.div(idx, El, rounding_mode="floor")                 # [T*k]
        # one row per (token, destination rank), destination-major
        need = torch.zeros(G * T, dtype=torch.int64, device=dev)
        need.index_fill_(0, dest * T + tok, 1)
        rank_in_dest = need.view(G, T).cumsum(dim=1)                     # inclusive
        # per destination: rows, pairs, and this rank's out-of-range flag
        counts = torch.zeros((G, 3), dtype=torch.int64, device=dev)
        counts[:, 0] = rank_in_dest[:, -1]
        counts[:, 1].index_add_(0, dest, torch.ones_like(dest))
        counts[:, 2] = (idx != idx_in).any()
        recv_c = torch.empty_like(counts)
        dist.all_to_all_single(recv_c, counts, group=self.group)
        host = torch.cat([counts, recv_c]).tolist()                      # the one host read
        if any(r[2] for r in host):
            raise K.IqkRuntimeError("expert index outside [0, num_experts)")
        s_rows, s_pairs = [r[0] for r in host[:G]], [r[1] for r in host[:G]]
        r_rows, r_pairs = [r[0] for r in host[G:]], [r[1] for r in host[G:]]

        # rows to send: slot of (g, t) = first slot of g's block + rank within
        # it; unmarked (g, t) write a spare slot past the end
        row_base = counts[:, 0].cumsum(0) - counts[:, 0]
        slots = torch.where(need.view(G, T).bool(), rank_in_dest + (row_base - 1).unsqueeze(1),
                            G * T)
        send_tok = torch.empty(G * T + 1, dtype=torch.int64, device=dev)
        send_tok.scatter_(0, slots.reshape(-1), self._token_index(T, 1, dev).repeat(G))
        send_tok = send_tok[:sum(s_rows)]
        send_rows = x.to(torch.bfloat16).index_select(0, send_tok)
        # pair records (row in its destination block, local expert, weight
        # bits), destination-major and stable in token, then slot
        order = torch.argsort(dest, stable=True)
        p_dest = dest[order]
        recs = torch.stack([rank_in_dest.view(-1)[p_dest * T + tok[order]] - 1,
                            idx[order] - p_dest * El,
                            w[order].view(torch.int32).to(torch.int64)], dim=1)

        rows = self._exchange(send_rows, s_rows, r_rows)
        recv_recs = self._exchange(recs, s_pairs, r_pairs)
        # pair rows are relative to the sender's block: add each block's offset
        recv_base = recv_c[:, 0].cumsum(0) - recv_c[:, 0]
        src = torch.repeat_interleave(recv_base, recv_c[:, 1], output_size=sum(r_pairs))
        pair_w = recv_recs[:, 2].to(torch.int32).view(torch.float32)
        y_rows = self.local_experts_forward(rows, recv_recs[:, 0] + src, recv_recs[:, 1], pair_w)

        back = self._exchange(y_rows.to(torch.bfloat16), r_rows, s_rows)
        out = torch.zeros((T, self.hidden), dtype=torch.float32, device=dev)
        out.index_add_(0, send_tok, back.to(torch.float32))
        self.last_stats = {"rows_sent": int(sum(s_rows)), "pairs_sent": int(sum(s_pairs)),
                           "rows_received": int(sum(r_rows)), "pairs_received": int(sum(r_pairs))}
        return out

    __call__ = forward


__all__ = ["ExpertParallelMoE"]
