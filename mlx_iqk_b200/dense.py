"""Serving entry points for the dense IQ_K members (IQ4_KS, IQ4_K, IQ5_K, IQ6_K).

The reference's dense seam is functional (src/mlx_iqk/dense.py:1-25): a dense
projection is one matrix with no routing state, so the caller holds the
streams and passes them per call. Same names, arguments, checks and error
classes here, over the CUDA library:

- :func:`dense_value_table`  the member's value table (fp16 for the integer
  alphabets, float32 for IQ6_K's reconstruction), one tensor per device;
- :func:`dense_gemv`         the decode route, ``[..., out]`` fp16
  (``iqk_dense_gemv``: f16 tensor-core tiles, each sub-block's scale applied
  to its own float32 partial sum, as the reference's kernel factors it);
- :func:`dense_dequantized` / :func:`dense_dequantized_range`  fp16 weights,
  bit-identical to the reference decode rounded to fp16 (``iqk_dense_dequant``);
- :func:`dense_linear`       the route chooser: the GEMV at or below
  ``token_limit`` activation rows, else dequantize and one matmul.

``x`` may be fp16 or bfloat16 (or float32); it meets the kernel at fp16, the
cast at the call seam as in the reference (src/mlx_iqk/dense.py:107-112).
"""

from __future__ import annotations

import torch

from . import kernels as K
from .format import (
    DENSE_MEMBERS,
    IqkFormatError,
    check_dense_member,
    check_row_width,
    dense_component_dtypes,
    dense_component_shapes,
)
from .kernels import IqkKernelError
from .tables import dense_values

DENSE_DECODE_TOKEN_LIMIT = 16
"""Activation rows at or below which :func:`dense_linear` takes the GEMV
(the reference's provisional default, src/mlx_iqk/dense.py:44-50)."""

DENSE_SUPPORTED_IN_FEATURES = (1024, 2048, 4096, 8192)
"""Input widths the dense kernels are sized for (src/mlx_iqk/dense_kernels.py:56)."""

ROWS_PER_TG = 16
"""Output rows one GEMV CTA owns; out_features must tile by it."""

DENSE_DEQUANT_THREADS = 256

_TORCH = {"uint8": torch.uint8, "uint32": torch.uint32, "float16": torch.float16,
          "float32": torch.float32}


class IqkDenseError(RuntimeError):
    pass


def check_dense_gemv_geometry(in_features: int, out_features: int) -> tuple[int, int]:
    """Reject any geometry the dense decode GEMV does not cover
    (src/mlx_iqk/dense_kernels.py:70-81)."""
    n = check_row_width(in_features, "iq4_k")
    if n not in DENSE_SUPPORTED_IN_FEATURES:
        raise IqkKernelError(
            f"the dense decode gemv is sized per input width and covers "
            f"{DENSE_SUPPORTED_IN_FEATURES}, got {in_features}")
    out = int(out_features)
    if out <= 0 or out % ROWS_PER_TG:
        raise IqkKernelError(
            f"out_features {out_features} is not a positive multiple of {ROWS_PER_TG}")
    return n, out


def check_dense_dequant_geometry(in_features: int, out_features: int) -> tuple[int, int]:
    """Reject any geometry the dense dequantization does not cover
    (src/mlx_iqk/dense_kernels.py:84-98)."""
    n = check_row_width(in_features, "iq4_k")
    if n not in DENSE_SUPPORTED_IN_FEATURES:
        raise IqkKernelError(
            f"the dense dequantization is sized per input width and covers "
            f"{DENSE_SUPPORTED_IN_FEATURES}, got {in_features}")
    out = int(out_features)
    if out <= 0:
        raise IqkKernelError(f"out_features {out_features} is not positive")
    if DENSE_DEQUANT_THREADS % (n // 32):
        raise IqkKernelError(
            f"in_features {in_features} does not tile {DENSE_DEQUANT_THREADS} threads")
    return n, out


_VALUE_TABLES: dict = {}


def dense_value_table(member: str, device=None) -> torch.Tensor:
    """The member's value table, both alphabets, one tensor per device: fp16
    for the integer alphabets (exact), float32 for ``iq6_k`` (the float32
    outputs of ik's cubic reconstruction). The kernels compile the same table
    in; this is for callers that read it."""
    check_dense_member(member)
    dev = torch.device(device) if device is not None else torch.device("cuda", 0)
    key = (member, dev)
    t = _VALUE_TABLES.get(key)
    if t is None:
        v = dense_values(member)
        t = torch.from_numpy(v.astype("float32" if member == "iq6_k" else "float16")).to(dev)
        _VALUE_TABLES[key] = t
    return t


def check_dense_streams(member: str, streams: dict, out_features: int,
                        in_features: int) -> list[torch.Tensor]:
    """Validate stream names, shapes, dtypes and device; return them in kernel
    input order (src/mlx_iqk/dense.py:88-108)."""
    shapes = dense_component_shapes(member, out_features, in_features)
    dtypes = dense_component_dtypes(member)
    if set(streams) != set(shapes):
        raise IqkDenseError(f"{member} needs streams {sorted(shapes)}, got {sorted(streams)}")
    ordered = []
    dev = None
    for name, shape in shapes.items():
        value = streams[name]
        if not isinstance(value, torch.Tensor):
            raise IqkDenseError(f"stream {name} must be a torch tensor on the GPU")
        if tuple(value.shape) != shape:
            raise IqkDenseError(
                f"stream {name} must be {shape} for {out_features}x{in_features}, "
                f"got {tuple(value.shape)}")
        want = _TORCH[dtypes[name].name]
        if value.dtype != want:
            raise IqkDenseError(f"stream {name} must be {dtypes[name].name}, got {value.dtype}")
        if not value.is_contiguous():
            raise IqkDenseError(f"stream {name} must be contiguous")
        if value.data_ptr() % 16:
            raise IqkDenseError(f"stream {name} must start on a 16-byte boundary")
        if dev is None:
            dev = value.device
        elif value.device != dev:
            raise IqkDenseError(f"stream {name} is on {value.device}, the others on {dev}")
        ordered.append(value)
    return ordered


def _tokens_view(x: torch.Tensor, in_features: int) -> torch.Tensor:
    xt = x.reshape(-1, in_features)
    if xt.dtype != torch.float16:
        xt = xt.to(torch.float16)
    xt = xt.contiguous()
    if xt.data_ptr() % 16:  # the C ABI takes 16-byte aligned activations
        xt = xt.clone()
    return xt


def dense_gemv(member: str, x: torch.Tensor, streams: dict, out_features: int,
               in_features: int) -> torch.Tensor:
    """Project ``[..., in]`` activations through the dense matrix, fused:
    ``[..., out]`` fp16. Valid for any token count; the decode shapes are
    where it is the intended route."""
    check_dense_member(member)
    n, out = check_dense_gemv_geometry(in_features, out_features)
    ordered = check_dense_streams(member, streams, out, n)
    dev = ordered[0].device
    xt = _tokens_view(x.to(dev), n)
    tokens = int(xt.shape[0])
    if tokens <= 0:
        raise IqkDenseError("no activation rows")
    y = torch.empty((tokens, out), dtype=torch.float16, device=dev)
    K.dense_gemv(member, xt, ordered, out, n, y)
    return y.reshape(list(x.shape[:-1]) + [out])


def dense_dequantized(member: str, streams: dict, out_features: int,
                      in_features: int) -> torch.Tensor:
    """Full fp16 dequantization ``[out, in]``, bit-identical to the reference
    decode rounded to fp16."""
    check_dense_member(member)
    n, out = check_dense_dequant_geometry(in_features, out_features)
    ordered = check_dense_streams(member, streams, out, n)
    dst = torch.empty((out, n), dtype=torch.float16, device=ordered[0].device)
    return K.dense_dequant(member, ordered, out, n, 0, out, dst)


def dense_dequantized_range(member: str, streams: dict, out_features: int,
                            in_features: int, start: int, rows: int) -> torch.Tensor:
    """fp16 dequantization of out rows ``[start, start + rows)``: ``[rows, in]``,
    bit-identical to the same slice of :func:`dense_dequantized`; ``rows`` a
    positive power of two (src/mlx_iqk/dense.py:165-189)."""
    check_dense_member(member)
    n, out = check_dense_dequant_geometry(in_features, out_features)
    ordered = check_dense_streams(member, streams, out, n)
    start, rows = int(start), int(rows)
    if rows <= 0 or rows & (rows - 1):
        raise IqkDenseError(f"range rows {rows} is not a positive power of two")
    if start < 0 or start + rows > out:
        raise IqkDenseError(f"range [{start}, {start + rows}) is outside out_features {out}")
    dst = torch.empty((rows, n), dtype=torch.float16, device=ordered[0].device)
    return K.dense_dequant(member, ordered, out, n, start, rows, dst)


def dense_linear(member: str, x: torch.Tensor, streams: dict, out_features: int,
                 in_features: int, token_limit: int = DENSE_DECODE_TOKEN_LIMIT) -> torch.Tensor:
    """Project ``x`` through the dense matrix, choosing the route by shape: the
    fused GEMV at or below ``token_limit`` activation rows, above it one fp16
    dequantization and a plain matmul (src/mlx_iqk/dense.py:192-210)."""
    check_dense_member(member)
    xt = x.reshape(-1, int(in_features))
    if int(xt.shape[0]) <= int(token_limit):
        return dense_gemv(member, x, streams, out_features, in_features)
    weights = dense_dequantized(member, streams, out_features, in_features)
    result = torch.matmul(_tokens_view(x.to(weights.device), int(in_features)), weights.t())
    return result.reshape(list(x.shape[:-1]) + [int(out_features)])


__all__ = [
    "DENSE_DECODE_TOKEN_LIMIT", "DENSE_MEMBERS", "DENSE_SUPPORTED_IN_FEATURES",
    "IqkDenseError", "IqkFormatError", "check_dense_dequant_geometry",
    "check_dense_gemv_geometry", "check_dense_streams", "dense_dequantized",
    "dense_dequantized_range", "dense_gemv", "dense_linear", "dense_value_table",
]
