"""One SwitchGLU MoE step over three ``IqkSwitchLinear`` projections.

The reference's module is the per-projection seam (``src/mlx_iqk/nn.py:1-22``):
the consuming runtime calls gate and up on the token, applies SiLU(gate) * up,
calls down, and sums the top-k outputs weighted by the router. Each of those
is a separate dispatch there. ``IqkSwitchGLU`` keeps the three projections
(each with its own member, as the reference allows) and runs the step with
the layer's work fused where the hardware allows:

* decode (few pairs, unsorted): one activation preparation; gate and up in
  one launch whose items cover the same 32 rows of both projections, so
  ``h = silu(gate) * up * router weight`` is formed before anything leaves
  the SM (``iqk_gemv_glu_run``; a layer whose gate and up members differ
  runs the two projections and ``iqk_swiglu_rows``); the down projection
  over one row of ``h`` per pair; each token's sum over its pairs
  (``iqk_pairs_combine``). Five launches for the whole layer, against nine
  module calls plus the caller's elementwise work on the reference's seam.
* prefill (more pairs, or ``sorted_indices``): the tensor-core grouped GEMMs
  with the same SiLU * up * weight pass over the routed pairs
  (``iqk_pairs_swiglu``, bf16 h) and the same combine.

The router weight goes in before the down projection (which is linear), so
the combine is a plain fixed-order sum: the result does not depend on how
pairs are grouped. With ``scores=None`` the step returns the unweighted
per-pair outputs ``[..., top_k, hidden]`` instead of the sum.
"""

from __future__ import annotations

import math

import torch
from torch import nn

from . import kernels as K
from .nn import DECODE_MAT_LIMIT, IqkRuntimeError, IqkSwitchLinear


class IqkSwitchGLU(nn.Module):
    """gate / up ``[inter, hidden]`` and down ``[hidden, inter]`` per expert."""

    def __init__(self, members, num_experts: int, hidden: int, inter: int, device=None):
        super().__init__()
        g, u, d = members
        self.gate = IqkSwitchLinear(g, num_experts, inter, hidden, device=device)
        self.up = IqkSwitchLinear(u, num_experts, inter, hidden, device=device)
        self.down = IqkSwitchLinear(d, num_experts, hidden, inter, device=device)
        if inter % 32:
            raise IqkRuntimeError(f"inter {inter} is not a multiple of 32")
        self.num_experts, self.hidden, self.inter = num_experts, hidden, inter
        self._ws: dict = {}

    @property
    def device(self) -> torch.device:
        return self.gate.device

    def _scratch(self, tag: str, nbytes: int, dtype=torch.uint8, shape=None) -> torch.Tensor:
        """Scratch reused across calls on one stream (stream order keeps a
        call's kernels after the previous call's); fresh under graph capture."""
        dev = self.device
        shape = shape or (max(nbytes, 256),)
        count = math.prod(shape)
        if torch.cuda.is_current_stream_capturing():
            return torch.empty(shape, dtype=dtype, device=dev)
        key = (K.stream_handle(dev), tag)
        t = self._ws.get(key)
        if t is None or t.numel() < count or t.dtype != dtype:
            if len(self._ws) >= 32:
                self._ws.clear()
            t = torch.empty(count, dtype=dtype, device=dev)
            self._ws[key] = t
        return t[:count].view(shape)

    def __call__(self, x, indices, scores=None, sorted_indices=False):
        return self.forward(x, indices, scores, sorted_indices)

    def graphed(self, batch: int, top_k: int, dtype: torch.dtype = torch.bfloat16) -> "GraphedSwitchGLU":
        """This layer's decode step for ``batch`` tokens captured in a CUDA
        graph over static input / output tensors (see :class:`GraphedSwitchGLU`)."""
        return GraphedSwitchGLU(self, batch, top_k, dtype)

    def forward(self, x, indices, scores=None, sorted_indices=False) -> torch.Tensor:
        """``x [..., hidden]``, ``indices [..., top_k]``, ``scores [..., top_k]``
        -> ``[..., hidden]`` float32 (or ``[..., top_k, hidden]`` when
        ``scores`` is None)."""
        dev, E, H, I = self.device, self.num_experts, self.hidden, self.inter
        lead, k = tuple(indices.shape[:-1]), indices.shape[-1]
        xt = x.reshape(-1, H)
        if xt.device != dev:
            xt = xt.to(dev)
        if xt.dtype not in K.DTYPE_IDS:
            xt = xt.float()
        xt = xt.contiguous()
        T = xt.shape[0]
        sel = indices.reshape(-1).to(device=dev, dtype=torch.int32).contiguous()
        P = sel.numel()
        if P != T * k:
            raise IqkRuntimeError(
                f"{P} token-expert pairs do not tile {T} activation row(s); "
                f"the operand and the routing disagree")
        w = None
        if scores is not None:
            w = scores.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
            if w.numel() != P:
                raise IqkRuntimeError(f"{w.numel()} router weights for {P} pairs")
        if P == 0:
            shape = lead + ((H,) if scores is not None else (k, H))
            return torch.zeros(shape, dtype=torch.float32, device=dev)
        if P <= DECODE_MAT_LIMIT and not sorted_indices:
            yd = self._decode(xt, sel, w, T, P)
        else:
            yd = self._prefill(xt, sel, w, P)
        if scores is None:
            return yd.view(*lead, k, H)
        out = torch.empty((T, H), dtype=torch.float32, device=dev)
        K.pairs_combine(yd, sel, k, E, out)
        return out.view(*lead, H)

    def _decode(self, xt, sel, w, T, P) -> torch.Tensor:
        E, H, I = self.num_experts, self.hidden, self.inter
        g, u, d = self.gate, self.up, self.down
        ws = self._scratch("gu", K.gemv_workspace_bytes(g.member, H, T, P))
        K.gemv_prepare(xt, E, H, sel, None, ws)
        h = self._scratch("h", 0, torch.float32, (P, I))
        if g.member == u.member:
            K.gemv_glu_run(g.member, g._streams(), u._streams(), E, I, H, T, P, w, h, ws)
        else:
            yg = self._scratch("yg", 0, torch.float32, (P, I))
            yu = self._scratch("yu", 0, torch.float32, (P, I))
            K.gemv_run(g.member, g._streams(), E, I, H, T, P, yg, ws)
            K.gemv_run(u.member, u._streams(), E, I, H, T, P, yu, ws)
            K.swiglu_rows(yg, yu, w, h)
        ws_d = self._scratch("d", K.gemv_workspace_bytes(d.member, I, P, P))
        K.gemv_prepare(h, E, I, sel, None, ws_d)
        yd = torch.empty((P, H), dtype=torch.float32, device=self.device)
        K.gemv_run(d.member, d._streams(), E, H, I, P, P, yd, ws_d)
        return yd

    def _prefill(self, xt, sel, w, P) -> torch.Tensor:
        E, H, I = self.num_experts, self.hidden, self.inter
        g, u, d = self.gate, self.up, self.down
        dev = self.device
        if w is None:
            w = torch.ones(P, dtype=torch.float32, device=dev)
        ws = torch.empty(K.grouped_workspace_bytes(H, E, P), dtype=torch.uint8, device=dev)
        K.grouped_prepare(xt, E, H, sel, None, ws)
        yg = torch.empty((P, I), dtype=torch.float32, device=dev)
        yu = torch.empty((P, I), dtype=torch.float32, device=dev)
        K.grouped_run(g.member, g._streams(), E, I, H, P, yg, ws)
        K.grouped_run(u.member, u._streams(), E, I, H, P, yu, ws)
        hb = torch.empty((P, I), dtype=torch.bfloat16, device=dev)
        K.pairs_swiglu(yg, yu, w, H, E, ws, hb)
        ws_d = torch.empty(K.grouped_workspace_bytes(I, E, P), dtype=torch.uint8, device=dev)
        K.grouped_prepare(hb, E, I, sel, None, ws_d)
        yd = torch.empty((P, H), dtype=torch.float32, device=dev)
        K.grouped_run(d.member, d._streams(), E, H, I, P, yd, ws_d)
        return yd


class GraphedSwitchGLU:
    """One decode step of an ``IqkSwitchGLU`` for a fixed batch, captured in a
    CUDA graph: the static device tensors ``x [batch, hidden]``, ``indices
    [batch, top_k]`` (int32) and ``scores [batch, top_k]`` (float32) are the
    inputs, ``out [batch, hidden]`` (float32) the output. A server copies the
    step's inputs into them (from pinned host memory, on any stream it orders
    before the replay), calls :meth:`replay` on the current stream and reads
    ``out`` -- the layer's launches then cost one graph launch instead of
    their host-side set-up. Built by :meth:`IqkSwitchGLU.graphed`."""

    def __init__(self, layer: "IqkSwitchGLU", batch: int, top_k: int,
                 dtype: torch.dtype = torch.bfloat16):
        dev = layer.device
        self.layer, self.batch, self.top_k = layer, int(batch), int(top_k)
        self.x = torch.zeros((batch, layer.hidden), dtype=dtype, device=dev)
        # distinct valid experts per token for the capture's warm-up
        ids = torch.arange(batch * top_k, device=dev, dtype=torch.int32) % layer.num_experts
        self.indices = ids.reshape(batch, top_k).contiguous()
        self.scores = torch.full((batch, top_k), 1.0 / top_k, device=dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            layer(self.x, self.indices, self.scores)  # first-call set-up outside capture
            torch.cuda.synchronize(dev)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=side):
                self.out = layer(self.x, self.indices, self.scores)
        torch.cuda.current_stream(dev).wait_stream(side)

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.out


__all__ = ["GraphedSwitchGLU", "IqkSwitchGLU"]
