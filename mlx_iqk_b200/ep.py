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
   ``all_to_all_single`` of the split counts, then of the rows (bf16) and the
   pair records;
2. **expert compute** on the receiving rank -- grouped GEMM of gate and up
   over the received pairs (``iqk_grouped_gemm`` with explicit rows),
   SiLU(gate) * up, grouped GEMM of down, and the router-weighted sum of each
   row's pairs;
3. **combine** -- one row per (token, rank) travels back the reverse way and
   is added into the token's output.

No kernel reads another GPU's memory; the only data-path collectives are the
three ``all_to_all_single`` exchanges, and every rank takes them in the same
order. The expert computation is a parameter (``expert_fn``) only so that
CPU tests can check the dispatch and combine logic on ``gloo`` ranks against
a host stand-in; the default -- and the only product path -- is the CUDA
grouped GEMM.
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
        h = (torch.nn.functional.silu(g) * u).to(torch.bfloat16)
        y = torch.empty((P, self.hidden), dtype=torch.float32, device=rows.device)
        ws_d = torch.empty(K.grouped_workspace_bytes(self.inter, self.local_experts, P),
                           dtype=torch.uint8, device=rows.device)
        K.grouped(self.down.member, h, self.down._streams(), self.local_experts, self.hidden,
                  self.inter, sel, None, y, ws_d)
        out.index_add_(0, pair_row.long(), y * pair_weight.to(torch.float32).unsqueeze(1))
        return out

    # -- dispatch / combine ----------------------------------------------

    def _exchange(self, send: torch.Tensor, send_counts: list[int], recv_counts: list[int]):
        if self.world == 1:
            return send
        recv = torch.empty((sum(recv_counts),) + tuple(send.shape[1:]), dtype=send.dtype,
                           device=send.device)
        dist.all_to_all_single(recv, send.contiguous(), recv_counts, send_counts,
                               group=self.group)
        return recv

    def forward(self, x: torch.Tensor, indices: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        """``x [T, hidden]`` (this rank's tokens), ``indices [T, k]`` global expert
        ids, ``weights [T, k]`` router weights -> ``[T, hidden]`` float32."""
        T, k = indices.shape
        G, El = self.world, self.local_experts
        dev = x.device
        idx = indices.to(device=dev, dtype=torch.int64)
        if idx.numel() and (int(idx.min()) < 0 or int(idx.max()) >= self.num_experts):
            raise K.IqkRuntimeError("expert index outside [0, num_experts)")
        dest = idx // El                                        # [T, k]
        # one row per (token, destination rank), destination-major
        need = torch.zeros((G, T), dtype=torch.bool, device=dev)
        need[dest.reshape(-1), torch.arange(T, device=dev).repeat_interleave(k)] = True
        row_counts = need.sum(dim=1)                            # [G]
        rank_in_dest = torch.cumsum(need.to(torch.int64), dim=1) - 1  # [G, T]
        send_tok = need.nonzero(as_tuple=False)                 # [S, 2] (dest, token), sorted
        send_rows = x.to(torch.bfloat16)[send_tok[:, 1]]
        # pair records, destination-major (stable in token, then slot)
        flat_dest = dest.reshape(-1)
        order = torch.argsort(flat_dest, stable=True)
        p_tok = torch.arange(T, device=dev).repeat_interleave(k)[order]
        p_dest = flat_dest[order]
        p_row = rank_in_dest[p_dest, p_tok]                     # row within its destination block
        p_exp = (idx.reshape(-1)[order] - p_dest * El)
        p_w = weights.to(device=dev, dtype=torch.float32).reshape(-1)[order]
        pair_counts = torch.bincount(p_dest, minlength=G)

        counts = torch.stack([row_counts, pair_counts]).to(torch.int64)   # [2, G]
        if G > 1:
            recv_c = torch.empty_like(counts.t().contiguous())
            dist.all_to_all_single(recv_c, counts.t().contiguous(), group=self.group)
            recv_c = recv_c.t()
        else:
            recv_c = counts
        s_rows, s_pairs = counts[0].tolist(), counts[1].tolist()
        r_rows, r_pairs = recv_c[0].tolist(), recv_c[1].tolist()

        rows = self._exchange(send_rows, s_rows, r_rows)
        recs = torch.stack([p_row.to(torch.int64), p_exp.to(torch.int64)], dim=1)
        recv_recs = self._exchange(recs, s_pairs, r_pairs)
        recv_w = self._exchange(p_w, s_pairs, r_pairs)
        # pair rows are relative to the sender's block: add each block's offset
        row_base = torch.cumsum(torch.tensor([0] + r_rows[:-1], device=dev), 0)
        src_of_pair = torch.repeat_interleave(torch.arange(G, device=dev),
                                              torch.tensor(r_pairs, device=dev))
        pair_row = recv_recs[:, 0] + row_base[src_of_pair]
        y_rows = self.local_experts_forward(rows, pair_row, recv_recs[:, 1], recv_w)

        back = self._exchange(y_rows.to(torch.bfloat16), r_rows, s_rows)
        out = torch.zeros((T, self.hidden), dtype=torch.float32, device=dev)
        out.index_add_(0, send_tok[:, 1], back.to(torch.float32))
        self.last_stats = {"rows_sent": int(sum(s_rows)), "pairs_sent": int(sum(s_pairs)),
                           "rows_received": int(sum(r_rows)), "pairs_received": int(sum(r_pairs))}
        return out

    __call__ = forward


__all__ = ["ExpertParallelMoE"]
