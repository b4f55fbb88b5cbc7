"""Stacked-expert IQ_K projection with the ``(x, indices)`` switch interface, on B200.

``IqkSwitchLinear`` keeps the reference's surface (``src/mlx_iqk/nn.py:105-333``):
the constructor ``(member, num_experts, out_features, in_features)``,
``load_streams`` fed by ``format.pack`` output, ``__call__(x, indices,
sorted_indices=False)`` with the gate/up operand ``[..., 1, 1, in]`` or the down
operand ``[..., top_k, 1, in]`` and a ``[..., top_k, 1, out]`` result, plus
``gemv``, ``gemv_sorted``, ``gemv_union``, ``dequantized``,
``dequantized_range`` and ``sorted_matmul_range``. Every compute call runs the
sm_100a kernels of ``libiqk_b200.so`` on the current CUDA stream.

Differences from the reference, each deliberate:

* activations are consumed in their own dtype (float32, float16 or bfloat16);
  the reference casts to float16 first (``nn.py:247``);
* projections return float32: the decode kernel's result is exact up to one
  final rounding, and a 16-bit store would not hold the 1e-4 decode bound;
* every route streams each selected expert's rows once for all pairs that
  picked it (the reference's union formulation, for all three members).
"""

from __future__ import annotations

import numpy as np
import torch
from torch import nn

from . import kernels as K
from .format import IQ2NL_VALUES, check_member, component_dtypes, component_shapes

DECODE_MAT_LIMIT = 63
"""Token-expert pairs at or below which ``__call__`` serves the decode GEMV
(``src/mlx_iqk/nn.py:49``)."""

IqkRuntimeError = K.IqkRuntimeError
IqkKernelError = K.IqkKernelError

_TORCH_DTYPES = {"uint8": torch.uint8, "uint16": torch.uint16, "uint32": torch.uint32,
                 "float16": torch.float16}

_VALUE_TABLES: dict[torch.device, torch.Tensor] = {}
_GRID_TABLES: dict[torch.device, torch.Tensor] = {}


def _default_device() -> torch.device:
    return torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() \
        else torch.device("cpu")


def value_table(device: torch.device | None = None) -> torch.Tensor:
    """The fp16 ``iq2nl_values`` table, one shared tensor per device.

    The kernels carry the alphabet as immediates; the tensor exists for API
    parity with the reference (``nn.py:60-71``) and for callers that want it.
    """
    dev = device or _default_device()
    if dev not in _VALUE_TABLES:
        _VALUE_TABLES[dev] = torch.tensor(IQ2NL_VALUES.astype(np.float16), device=dev)
    return _VALUE_TABLES[dev]


def grid_table(device: torch.device | None = None) -> torch.Tensor:
    """The IQ1_S grid as uint32 words (2048 entries x 8 int8 values), shared per device."""
    dev = device or _default_device()
    if dev not in _GRID_TABLES:
        from .tables import grid_values
        words = np.ascontiguousarray(grid_values()).view(np.uint32).reshape(-1)
        _GRID_TABLES[dev] = torch.from_numpy(words.copy()).to(dev)
    return _GRID_TABLES[dev]


def member_table(member: str, device: torch.device | None = None) -> torch.Tensor:
    check_member(member)
    return grid_table(device) if member == "iq1_s_r4" else value_table(device)


class IqkSwitchLinear(nn.Module):
    """Stacked IQ_K experts for one projection, ``(x, indices)`` interface."""

    mode = "iqk"

    def __init__(self, member: str, num_experts: int, out_features: int, in_features: int,
                 device: torch.device | str | None = None):
        super().__init__()
        self.member = check_member(member)
        K.check_gemv_geometry(in_features, out_features)
        K.check_dequant_geometry(in_features, out_features)
        self.num_experts = int(num_experts)
        self.out_features = int(out_features)
        self.in_features = int(in_features)
        if self.num_experts <= 0:
            raise IqkRuntimeError(f"num_experts {num_experts} is not positive")
        dev = torch.device(device) if device is not None else _default_device()
        shapes = component_shapes(member, num_experts, out_features, in_features)
        dtypes = component_dtypes(member)
        for name, shape in shapes.items():
            self.register_buffer(
                name, torch.zeros(shape, dtype=_TORCH_DTYPES[dtypes[name].name], device=dev))
        self._names = tuple(shapes)           # kernel input order
        self._ws_cache: dict[int, torch.Tensor] = {}  # decode scratch per CUDA stream

    # -- wire streams -------------------------------------------------------

    def stream_names(self) -> list[str]:
        """Relayout stream names of this member, in kernel input order."""
        return list(component_shapes(self.member, self.num_experts, self.out_features,
                                     self.in_features))

    def _streams(self) -> list[torch.Tensor]:
        buffers = self._buffers
        return [buffers[name] for name in self._names]

    def _workspace(self, need: int, dev: torch.device, stream: int) -> torch.Tensor:
        """Decode scratch reused across calls on one stream (stream order keeps a
        call's kernels after the previous call's); fresh under graph capture."""
        if torch.cuda.is_current_stream_capturing():
            return torch.empty(max(need, 256), dtype=torch.uint8, device=dev)
        ws = self._ws_cache.get(stream)
        if ws is None or ws.numel() < need or ws.device != dev:
            if len(self._ws_cache) >= 8:
                self._ws_cache.clear()
            ws = torch.empty(max(need, 256), dtype=torch.uint8, device=dev)
            self._ws_cache[stream] = ws
        return ws

    @property
    def device(self) -> torch.device:
        return self.qs.device

    def load_streams(self, streams: dict) -> None:
        """Install packed streams (numpy or torch), checking every shape.

        Values are reinterpreted (not converted) as the stream's dtype, so a
        same-width integer view of the packed bytes is accepted; a different
        element width is refused.
        """
        shapes = component_shapes(self.member, self.num_experts, self.out_features,
                                  self.in_features)
        if set(streams) != set(shapes):
            raise IqkRuntimeError(
                f"{self.member} needs streams {sorted(shapes)}, got {sorted(streams)}")
        for name, want in shapes.items():
            got = tuple(streams[name].shape)
            if got != want:
                raise IqkRuntimeError(
                    f"stream {name} must be {want} for "
                    f"{self.num_experts}x{self.out_features}x{self.in_features}, got {got}")
        dtypes = component_dtypes(self.member)
        staged = {}
        for name, value in streams.items():
            want_t = _TORCH_DTYPES[dtypes[name].name]
            if isinstance(value, np.ndarray):
                arr = np.ascontiguousarray(value)
                if arr.dtype.itemsize != dtypes[name].itemsize:
                    raise IqkRuntimeError(
                        f"stream {name} has {arr.dtype} elements, expected {dtypes[name]}")
                t = torch.from_numpy(arr.view(dtypes[name]))
            elif isinstance(value, torch.Tensor):
                t = value
                if t.element_size() != dtypes[name].itemsize:
                    raise IqkRuntimeError(
                        f"stream {name} has {t.dtype} elements, expected {dtypes[name]}")
                if t.dtype != want_t:
                    t = t.contiguous().view(want_t)
            else:
                raise IqkRuntimeError(f"stream {name} is a {type(value).__name__}")
            staged[name] = t.to(self.device, non_blocking=False).contiguous()
        for name, t in staged.items():
            setattr(self, name, t)

    def load_wire(self, wire) -> None:
        """Install ik wire rows (``[E * out, ggml row bytes]`` uint8, e.g. the
        tensor bytes of a GGUF file), relaid out on the device.

        The same streams as ``load_streams(format.pack(member, wire, in))``
        bit for bit; the relayout runs as one kernel (``iqk_pack``) where the
        reference runs ``format.pack`` on the host (``src/mlx_iqk/format.py:612-678``).
        """
        from .format import ik_row_bytes
        rb = ik_row_bytes(self.member, self.in_features)
        rows = self.num_experts * self.out_features
        if isinstance(wire, np.ndarray):
            wire = torch.from_numpy(np.ascontiguousarray(wire, dtype=np.uint8))
        if not isinstance(wire, torch.Tensor) or wire.element_size() != 1:
            raise IqkRuntimeError("wire must be a uint8 array or tensor")
        if wire.numel() != rows * rb:
            raise IqkRuntimeError(
                f"wire of {wire.numel()} bytes is not {rows} rows of {rb} bytes")
        w = wire.reshape(rows, rb).to(self.device).contiguous()
        K.pack(self.member, w.view(torch.uint8), self.in_features, self._streams())

    # -- dequantized route --------------------------------------------------

    def dequantized(self, dtype: torch.dtype = torch.float16) -> torch.Tensor:
        """Full dequantization ``[E, out, in]``, bit-identical to the CPU decode
        rounded once to ``dtype`` (float16 by default, as the reference)."""
        out = torch.empty((self.num_experts, self.out_features, self.in_features),
                          dtype=dtype, device=self.device)
        return K.dequant(self.member, self._streams(), self.num_experts, self.out_features,
                         self.in_features, 0, self.out_features, out)

    def dequantized_range(self, start: int, rows: int,
                          dtype: torch.dtype = torch.float16) -> torch.Tensor:
        """Dequantization of out rows ``[start, start + rows)`` of every expert,
        ``[E, rows, in]``; the same bits as that slice of :meth:`dequantized`.

        ``rows`` must be a positive power of two, as in the reference
        (``src/mlx_iqk/nn.py:171-201``), whose range kernel is sized that way.
        """
        start, rows = int(start), int(rows)
        if rows <= 0 or rows & (rows - 1):
            raise IqkRuntimeError(f"range rows {rows} is not a positive power of two")
        if start < 0 or start + rows > self.out_features:
            raise IqkRuntimeError(
                f"range [{start}, {start + rows}) is outside out_features {self.out_features}")
        out = torch.empty((self.num_experts, rows, self.in_features), dtype=dtype,
                          device=self.device)
        return K.dequant(self.member, self._streams(), self.num_experts, self.out_features,
                         self.in_features, start, rows, out)

    def sorted_matmul_range(self, x, indices, start: int, rows: int) -> torch.Tensor:
        """The sorted projection restricted to out rows ``[start, start + rows)``:
        ``[..., top_k, 1, rows]``.

        Only those rows of every selected expert are read and multiplied (the
        reference bounds its live memory the same way,
        ``src/mlx_iqk/nn.py:203-217``); each output element is the same dot
        product as in the unsplit sorted call, so concatenating range outputs
        along the feature axis reproduces it bit for bit. ``rows`` is a
        positive power of two, as in the reference.
        """
        start, rows = int(start), int(rows)
        if rows <= 0 or rows & (rows - 1) or start < 0 or start + rows > self.out_features:
            raise IqkRuntimeError(
                f"range [{start}, {start + rows}) is not a power-of-two slice of "
                f"out_features {self.out_features}")
        if self.member not in K.GROUPED_MEMBERS:
            full = self.gemv(x, indices)
            return full[..., start:start + rows].contiguous()
        xt = self._prep(x)
        idx_shape = tuple(indices.shape)
        sel = self._idx(indices, self.device)
        mats, xrows = sel.numel(), xt.shape[0]
        if xrows <= 0 or mats % xrows:
            raise IqkRuntimeError(
                f"{mats} token-expert pairs do not tile {xrows} activation "
                f"row(s); the operand and the routing disagree")
        ws = torch.empty(K.grouped_workspace_bytes(self.in_features, self.num_experts, mats),
                         dtype=torch.uint8, device=self.device)
        K.grouped_prepare(xt, self.num_experts, self.in_features, sel, None, ws)
        y = torch.empty((mats, rows), dtype=torch.float32, device=self.device)
        K.grouped_run_range(self.member, self._streams(), self.num_experts, self.out_features,
                            self.in_features, mats, start, rows, y, ws)
        return y.reshape(*idx_shape, rows).unsqueeze(-2)

    # -- call ---------------------------------------------------------------

    def __call__(self, x, indices, sorted_indices=False):
        return self.forward(x, indices, sorted_indices)

    def forward(self, x, indices, sorted_indices=False) -> torch.Tensor:
        """Project ``x`` through the experts named by ``indices``.

        ``x`` is ``[..., 1, 1, in]`` (one row per token, shared by its top_k
        experts) or ``[..., top_k, 1, in]`` (one row per pair); ``indices``
        is ``[..., top_k]``; the result is ``[..., top_k, 1, out]`` float32.
        Decode-sized calls (``<= DECODE_MAT_LIMIT`` pairs, unsorted) run the
        fused dequant + GEMV; prefill-sized or ``sorted_indices=True`` calls
        run the tensor-core grouped GEMM (``src/mlx_iqk/nn.py:221-238`` makes
        the same split, with dequantize + ``gather_mm`` on the prefill side).
        """
        pairs = indices.numel() if isinstance(indices, torch.Tensor) else \
            int(np.asarray(indices).size)
        if self.member in K.GROUPED_MEMBERS and (sorted_indices or pairs > DECODE_MAT_LIMIT):
            return self.grouped(x, indices)
        return self.gemv(x, indices)

    def _prep(self, x: torch.Tensor, dev: torch.device | None = None) -> torch.Tensor:
        dev = self.device if dev is None else dev
        if not isinstance(x, torch.Tensor):
            x = torch.as_tensor(np.asarray(x))
        if x.device != dev:
            x = x.to(dev)
        if x.dtype not in K.DTYPE_IDS:
            x = x.to(torch.float32)
        return x.reshape(-1, self.in_features).contiguous()

    @staticmethod
    def _idx(t, device) -> torch.Tensor:
        if not isinstance(t, torch.Tensor):
            t = torch.as_tensor(np.asarray(t).astype(np.int64))
        return t.reshape(-1).to(device=device, dtype=torch.int32).contiguous()

    def gemv(self, x, indices) -> torch.Tensor:
        """Fused dequant + GEMV over the selected experts; valid for any pair count."""
        dev = self.device
        xt = self._prep(x, dev)
        idx_shape = tuple(indices.shape)
        sel = self._idx(indices, dev)
        mats, rows = sel.numel(), xt.shape[0]
        if rows <= 0 or mats % rows:
            raise IqkRuntimeError(
                f"{mats} token-expert pairs do not tile {rows} activation "
                f"row(s); the operand and the routing disagree")
        y = torch.empty((mats, self.out_features), dtype=torch.float32, device=dev)
        stream = K.stream_handle(dev)
        ws = self._workspace(K.gemv_workspace_bytes(self.member, self.in_features, rows, mats),
                             dev, stream)
        K.gemv(self.member, xt, self._streams(), self.num_experts, self.out_features,
               self.in_features, sel, None, y, ws, stream=stream)
        return y.view(idx_shape + (1, self.out_features))

    def grouped(self, x, indices) -> torch.Tensor:
        """Tensor-core grouped GEMM over the selected experts (the prefill route);
        same operands and result shape as :meth:`gemv`."""
        if self.member not in K.GROUPED_MEMBERS:
            raise IqkKernelError(
                f"the grouped GEMM covers {K.GROUPED_MEMBERS}; {self.member!r} uses gemv")
        xt = self._prep(x)
        idx_shape = tuple(indices.shape)
        sel = self._idx(indices, self.device)
        mats, rows = sel.numel(), xt.shape[0]
        if rows <= 0 or mats % rows:
            raise IqkRuntimeError(
                f"{mats} token-expert pairs do not tile {rows} activation "
                f"row(s); the operand and the routing disagree")
        y = torch.empty((mats, self.out_features), dtype=torch.float32, device=self.device)
        K.grouped(self.member, xt, self._streams(), self.num_experts, self.out_features,
                  self.in_features, sel, None, y)
        return y.reshape(*idx_shape, self.out_features).unsqueeze(-2)

    def _gemv_toks(self, x, sorted_ids, toks) -> torch.Tensor:
        if self.member not in K.IQ2_MEMBERS:
            raise IqkKernelError(
                f"the sorted and union decode GEMVs are recorded formulations "
                f"for {K.IQ2_MEMBERS}; {self.member!r} has no such variant")
        xt = self._prep(x)
        sel = self._idx(sorted_ids, self.device)
        tok = self._idx(toks, self.device)
        if tok.numel() != sel.numel():
            raise IqkRuntimeError(f"toks carries {tok.numel()} rows for {sel.numel()} pairs")
        y = torch.empty((sel.numel(), self.out_features), dtype=torch.float32,
                        device=self.device)
        K.gemv(self.member, xt, self._streams(), self.num_experts, self.out_features,
               self.in_features, sel, tok, y)
        return y

    def gemv_sorted(self, x, sorted_ids, toks) -> torch.Tensor:
        """GEMV over expert-sorted pairs with explicit activation rows; ``[pairs, out]``.

        Bit-identical to :meth:`gemv` after un-permuting (``src/mlx_iqk/nn.py:273-299``).
        """
        return self._gemv_toks(x, sorted_ids, toks)

    def gemv_union(self, x, sorted_ids, toks) -> torch.Tensor:
        """GEMV reading each distinct expert once; ``[pairs, out]``, bit-identical to
        :meth:`gemv` after un-permuting (``src/mlx_iqk/nn.py:301-333``)."""
        return self._gemv_toks(x, sorted_ids, toks)


__all__ = ["DECODE_MAT_LIMIT", "IqkKernelError", "IqkRuntimeError", "IqkSwitchLinear",
           "grid_table", "member_table", "value_table"]
