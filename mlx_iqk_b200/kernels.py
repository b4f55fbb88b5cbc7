"""ctypes binding of ``libiqk_b200.so`` plus the reference's geometry guards.

The CUDA library is the product: this module loads it (failing loudly when it
is missing -- there is no CPU or eager fallback), declares the C ABI of
``include/iqk_b200.h``, and maps status codes onto the reference's exception
classes. The guard functions keep the reference's names and messages
(``src/mlx_iqk/kernels.py:100-128``).
"""

from __future__ import annotations

import ctypes
import functools
import os
from pathlib import Path

import torch

from .format import (DENSE_MEMBER_IDS, MEMBER_IDS, IqkFormatError, check_dense_member,
                     check_member, check_row_width)

ROWS_PER_TG = 16
"""Output rows one decode work unit (a warp) covers; out_features must tile it."""

SUPPORTED_IN_FEATURES = (2048, 4096)
"""Input widths the kernels are sized for: the down and gate/up widths."""

IQ2_MEMBERS = ("iq2_ks", "iq2_k")
"""Members the reference records sorted/union GEMV formulations for."""

LIB_PATH = Path(__file__).resolve().parent / "libiqk_b200.so"

IQK_OK = 0
_STATUS_NAMES = {
    1: "IQK_ERR_MEMBER", 2: "IQK_ERR_WIDTH", 3: "IQK_ERR_GEOMETRY", 4: "IQK_ERR_ARGUMENT",
    5: "IQK_ERR_ALIGNMENT", 6: "IQK_ERR_WORKSPACE", 7: "IQK_ERR_CUDA", 8: "IQK_ERR_DEVICE",
}
DEVERR_EXPERT, DEVERR_TOKEN, DEVERR_NONFINITE, DEVERR_TIMEOUT = 1, 2, 4, 8
DTYPE_IDS = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


class IqkKernelError(RuntimeError):
    """Geometry the kernels are not sized for (reference class name)."""


class IqkRuntimeError(RuntimeError):
    """Operand/stream contract violation or a failed launch (reference class name)."""


def check_gemv_geometry(in_features: int, out_features: int) -> tuple[int, int]:
    """Reject any geometry the decode GEMV does not cover, before launching."""
    n = check_row_width(in_features)
    if n not in SUPPORTED_IN_FEATURES:
        raise IqkKernelError(
            f"the decode gemv is sized per input width and covers "
            f"{SUPPORTED_IN_FEATURES}, got {in_features}")
    out = int(out_features)
    if out <= 0 or out % ROWS_PER_TG:
        raise IqkKernelError(
            f"out_features {out_features} is not a positive multiple of {ROWS_PER_TG}")
    return n, out


def check_dequant_geometry(in_features: int, out_features: int) -> tuple[int, int]:
    """Reject any geometry the stacked dequantization does not cover."""
    n = check_row_width(in_features)
    if n not in SUPPORTED_IN_FEATURES:
        raise IqkKernelError(
            f"the dequantization is sized per input width and covers "
            f"{SUPPORTED_IN_FEATURES}, got {in_features}")
    out = int(out_features)
    if out <= 0:
        raise IqkKernelError(f"out_features {out_features} is not positive")
    return n, out


# ------------------------------------------------------------------ loading

_LIB = None


def library() -> ctypes.CDLL:
    """The loaded CUDA library; raises if it was never built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = Path(os.environ.get("IQK_B200_LIB", LIB_PATH))
    if not path.exists():
        raise IqkRuntimeError(
            f"{path} is not built; run `python -c 'import __graft_entry__ as g; g.build()'` "
            "(the IQ_K kernels have no CPU fallback)")
    lib = ctypes.CDLL(str(path))
    vp, i64, i32, sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
    lib.iqk_status_string.argtypes = [i32]
    lib.iqk_status_string.restype = ctypes.c_char_p
    lib.iqk_abi_version.restype = i32
    lib.iqk_check_device.restype = i32
    lib.iqk_check_bounded_wait.argtypes = [i64, vp, vp]
    lib.iqk_check_bounded_wait.restype = i32
    lib.iqk_dequant.argtypes = [i32, vp, i64, i64, i64, i64, i64, i32, vp, vp]
    lib.iqk_dequant.restype = i32
    lib.iqk_dense_dequant.argtypes = [i32, vp, i64, i64, i64, i64, i32, vp, vp]
    lib.iqk_dense_dequant.restype = i32
    lib.iqk_dense_gemv.argtypes = [i32, vp, i64, vp, i64, i64, vp, i32, vp]
    lib.iqk_dense_gemv.restype = i32
    lib.iqk_pack.argtypes = [i32, vp, i64, i64, vp, vp]
    lib.iqk_pack.restype = i32
    lib.iqk_gemv_workspace_bytes.argtypes = [i32, i64, i64, i64]
    lib.iqk_gemv_workspace_bytes.restype = sz
    lib.iqk_gemv_workspace_min_bytes.argtypes = [i32, i64, i64, i64]
    lib.iqk_gemv_workspace_min_bytes.restype = sz
    lib.iqk_gemv.argtypes = [i32, vp, i32, i64, vp, i64, i64, i64, vp, vp, i64, vp, i32, vp,
                             sz, vp]
    lib.iqk_gemv.restype = i32
    lib.iqk_gemv_prepare.argtypes = [vp, i32, i64, i64, i64, vp, vp, i64, vp, sz, vp]
    lib.iqk_gemv_prepare.restype = i32
    lib.iqk_gemv_run.argtypes = [i32, vp, i64, i64, i64, i64, i64, vp, i32, vp, sz, vp]
    lib.iqk_gemv_run.restype = i32
    lib.iqk_gemv_floor_run.argtypes = [i32, vp, i64, i64, i64, i64, i64, vp, i32, vp, sz, vp]
    lib.iqk_gemv_floor_run.restype = i32
    lib.iqk_gemv_glu_run.argtypes = [i32, vp, vp, i64, i64, i64, i64, i64, vp, vp, vp, sz, vp]
    lib.iqk_gemv_glu_run.restype = i32
    lib.iqk_swiglu_rows.argtypes = [vp, vp, vp, i64, i64, vp, vp]
    lib.iqk_swiglu_rows.restype = i32
    lib.iqk_dequant_floor.argtypes = [i32, vp, i64, i64, i64, i64, i64, i32, vp, vp]
    lib.iqk_dequant_floor.restype = i32
    lib.iqk_read_error.argtypes = [vp, i64, i64, i64, ctypes.POINTER(ctypes.c_int32), vp]
    lib.iqk_read_error.restype = i32
    lib.iqk_grouped_workspace_bytes.argtypes = [i64, i64, i64]
    lib.iqk_grouped_workspace_bytes.restype = sz
    lib.iqk_grouped_gemm.argtypes = [i32, vp, i32, i64, vp, i64, i64, i64, vp, vp, i64, vp, i32,
                                     vp, sz, vp]
    lib.iqk_grouped_gemm.restype = i32
    lib.iqk_grouped_prepare.argtypes = [vp, i32, i64, i64, i64, vp, vp, i64, vp, sz, vp]
    lib.iqk_grouped_prepare.restype = i32
    lib.iqk_grouped_run.argtypes = [i32, vp, i64, i64, i64, i64, vp, i32, vp, sz, vp]
    lib.iqk_grouped_run.restype = i32
    lib.iqk_grouped_run_range.argtypes = [i32, vp, i64, i64, i64, i64, i64, i64, vp, i32, vp,
                                          sz, vp]
    lib.iqk_grouped_run_range.restype = i32
    lib.iqk_grouped_read_error.argtypes = [vp, ctypes.POINTER(ctypes.c_int32), vp]
    lib.iqk_grouped_read_error.restype = i32
    lib.iqk_gemv_static_max_bytes.restype = sz
    lib.iqk_gemv_static.argtypes = [i32, vp, i32, i64, vp, i64, i64, i64, vp, vp, i64, vp, i32,
                                    vp]
    lib.iqk_gemv_static.restype = i32
    lib.iqk_gemv_static_read_error.argtypes = [i64, i64, i64, ctypes.POINTER(ctypes.c_int32), vp]
    lib.iqk_gemv_static_read_error.restype = i32
    lib.iqk_grouped_prepare_shard.argtypes = [vp, i32, i64, i64, i64, vp, vp, i64, vp, sz, vp]
    lib.iqk_grouped_prepare_shard.restype = i32
    lib.iqk_pairs_swiglu.argtypes = [vp, vp, vp, i64, i64, i64, i64, vp, sz, vp, vp]
    lib.iqk_pairs_swiglu.restype = i32
    lib.iqk_pairs_combine.argtypes = [vp, vp, i64, i32, i64, i64, vp, i32, vp]
    lib.iqk_pairs_combine.restype = i32
    _LIB = lib
    return lib


def exported_symbols() -> list[str]:
    """C ABI entry points declared in include/iqk_b200.h."""
    return ["iqk_status_string", "iqk_abi_version", "iqk_check_device", "iqk_dequant",
            "iqk_gemv_workspace_bytes", "iqk_gemv_workspace_min_bytes", "iqk_gemv",
            "iqk_gemv_prepare", "iqk_gemv_run",
            "iqk_read_error", "iqk_grouped_workspace_bytes", "iqk_grouped_gemm",
            "iqk_grouped_prepare", "iqk_grouped_run", "iqk_grouped_read_error",
            "iqk_gemv_static_max_bytes", "iqk_gemv_static", "iqk_gemv_static_read_error",
            "iqk_grouped_prepare_shard",
            "iqk_pairs_swiglu", "iqk_pairs_combine", "iqk_gemv_floor_run",
            "iqk_dequant_floor", "iqk_grouped_run_range", "iqk_pack",
            "iqk_gemv_glu_run", "iqk_swiglu_rows", "iqk_check_bounded_wait",
            "iqk_dense_dequant", "iqk_dense_gemv"]


def check_bounded_wait(limit_ns: int, device: torch.device) -> int:
    """``iqk_check_bounded_wait``: the device error bits a wait that nothing
    satisfies leaves after ``limit_ns`` (IQK_DEVERR_TIMEOUT expected)."""
    flags = torch.zeros(1, dtype=torch.int32, device=device)
    raise_for_status(library().iqk_check_bounded_wait(limit_ns, flags.data_ptr(),
                                                      stream_handle(device)),
                     "iqk_check_bounded_wait")
    return int(flags.item())


def raise_for_status(status: int, what: str) -> None:
    if status == IQK_OK:
        return
    msg = f"{what}: {library().iqk_status_string(status).decode()} ({_STATUS_NAMES.get(status, status)})"
    if status == 1:
        raise IqkFormatError(msg)
    if status in (2, 3):
        raise IqkKernelError(msg)
    raise IqkRuntimeError(msg)


_DEVICE_OK: dict[int, bool] = {}


def check_device(device: torch.device) -> None:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _DEVICE_OK:
        with torch.cuda.device(idx):
            raise_for_status(library().iqk_check_device(), "device check")
        _DEVICE_OK[idx] = True


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_PTR_ARRAYS: dict[tuple, ctypes.Array] = {}


def ptr_array(tensors) -> ctypes.Array:
    """The streams' device pointers as a C array (cached per pointer tuple:
    a module's streams keep their storage between calls)."""
    key = tuple(t.data_ptr() for t in tensors)
    arr = _PTR_ARRAYS.get(key)
    if arr is None:
        if len(_PTR_ARRAYS) > 256:
            _PTR_ARRAYS.clear()
        arr = (ctypes.c_void_p * len(key))(*key)
        _PTR_ARRAYS[key] = arr
    return arr


def pack(member: str, wire: torch.Tensor, in_features: int, streams) -> None:
    """``iqk_pack``: ik wire rows [rows, ggml row bytes] (uint8, on the device)
    into ``streams`` (component order, each [rows, length] viewed flat)."""
    check_device(wire.device)
    status = library().iqk_pack(MEMBER_IDS[check_member(member)], wire.data_ptr(),
                                wire.shape[0], in_features, ptr_array(streams),
                                stream_handle(wire.device))
    raise_for_status(status, "iqk_pack")


def dequant(member: str, streams, num_experts: int, out_features: int, in_features: int,
            row_start: int, rows: int, out: torch.Tensor) -> torch.Tensor:
    """``iqk_dequant`` into ``out`` [E, rows, in] on the current stream."""
    lib = library()
    check_device(out.device)
    status = lib.iqk_dequant(MEMBER_IDS[check_member(member)], ptr_array(streams), num_experts,
                             out_features, in_features, row_start, rows,
                             DTYPE_IDS[out.dtype], out.data_ptr(), stream_handle(out.device))
    raise_for_status(status, "iqk_dequant")
    return out


def dense_dequant(member: str, streams, out_features: int, in_features: int, row_start: int,
                  rows: int, out: torch.Tensor) -> torch.Tensor:
    """``iqk_dense_dequant``: rows [row_start, row_start + rows) of a dense
    matrix into ``out`` [rows, in] (f32, f16 or bf16)."""
    check_device(out.device)
    status = library().iqk_dense_dequant(DENSE_MEMBER_IDS[check_dense_member(member)],
                                         ptr_array(streams), out_features, in_features,
                                         row_start, rows, DTYPE_IDS[out.dtype], out.data_ptr(),
                                         stream_handle(out.device))
    raise_for_status(status, "iqk_dense_dequant")
    return out


def dense_gemv(member: str, x: torch.Tensor, streams, out_features: int, in_features: int,
               y: torch.Tensor) -> torch.Tensor:
    """``iqk_dense_gemv``: ``y [T, out] = x [T, in] W^T`` for f16 ``x``; ``y``
    f16 or f32."""
    check_device(y.device)
    if x.dtype != torch.float16 or not x.is_contiguous():
        raise IqkRuntimeError("the dense gemv takes contiguous fp16 activations")
    status = library().iqk_dense_gemv(DENSE_MEMBER_IDS[check_dense_member(member)],
                                      x.data_ptr(), x.shape[0], ptr_array(streams),
                                      out_features, in_features, y.data_ptr(),
                                      DTYPE_IDS[y.dtype], stream_handle(y.device))
    raise_for_status(status, "iqk_dense_gemv")
    return y


@functools.lru_cache(maxsize=1024)
def gemv_workspace_bytes(member: str, in_features: int, x_rows: int, pairs: int) -> int:
    return int(library().iqk_gemv_workspace_bytes(MEMBER_IDS[member], in_features, x_rows, pairs))


def gemv_workspace_min_bytes(member: str, in_features: int, x_rows: int, pairs: int) -> int:
    """The smallest workspace the GEMV accepts (no split slots: whole items)."""
    return int(library().iqk_gemv_workspace_min_bytes(MEMBER_IDS[member], in_features, x_rows,
                                                      pairs))


def gemv(member: str, x: torch.Tensor, streams, num_experts: int, out_features: int,
         in_features: int, sel: torch.Tensor, tok: torch.Tensor | None, y: torch.Tensor,
         workspace: torch.Tensor | None = None, stream: int | None = None) -> torch.Tensor:
    """``iqk_gemv``: x [x_rows, in], sel/tok int32 [pairs], y [pairs, out]; on
    ``stream`` (a CUDA stream handle), else the device's current stream."""
    lib = library()
    check_device(y.device)
    pairs = sel.numel()
    x_rows = x.shape[0]
    need = gemv_workspace_bytes(member, in_features, x_rows, pairs)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=y.device)
    status = lib.iqk_gemv(
        MEMBER_IDS[member], x.data_ptr(), DTYPE_IDS[x.dtype], x_rows, ptr_array(streams),
        num_experts, out_features, in_features, sel.data_ptr(),
        None if tok is None else tok.data_ptr(), pairs, y.data_ptr(), DTYPE_IDS[y.dtype],
        workspace.data_ptr(), workspace.numel(),
        stream_handle(y.device) if stream is None else stream)
    raise_for_status(status, "iqk_gemv")
    return y


def gemv_prepare(x: torch.Tensor, num_experts: int, in_features: int, sel: torch.Tensor,
                 tok: torch.Tensor | None, workspace: torch.Tensor) -> torch.Tensor:
    """``iqk_gemv_prepare``: activation digit planes + routing into ``workspace``."""
    lib = library()
    check_device(workspace.device)
    status = lib.iqk_gemv_prepare(
        x.data_ptr(), DTYPE_IDS[x.dtype], x.shape[0], in_features, num_experts,
        sel.data_ptr(), None if tok is None else tok.data_ptr(), sel.numel(),
        workspace.data_ptr(), workspace.numel(), stream_handle(workspace.device))
    raise_for_status(status, "iqk_gemv_prepare")
    return workspace


def gemv_run(member: str, streams, num_experts: int, out_features: int, in_features: int,
             x_rows: int, pairs: int, y: torch.Tensor, workspace: torch.Tensor) -> torch.Tensor:
    """``iqk_gemv_run``: one projection over a prepared workspace into ``y``."""
    lib = library()
    status = lib.iqk_gemv_run(
        MEMBER_IDS[member], ptr_array(streams), num_experts, out_features, in_features, x_rows,
        pairs, y.data_ptr(), DTYPE_IDS[y.dtype], workspace.data_ptr(), workspace.numel(),
        stream_handle(y.device))
    raise_for_status(status, "iqk_gemv_run")
    return y


def gemv_glu_run(member: str, gate_streams, up_streams, num_experts: int, out_features: int,
                 in_features: int, x_rows: int, pairs: int, weight: torch.Tensor | None,
                 h: torch.Tensor, workspace: torch.Tensor) -> torch.Tensor:
    """``iqk_gemv_glu_run``: h [pairs, out] float32 = silu(gate) * up * weight."""
    status = library().iqk_gemv_glu_run(
        MEMBER_IDS[member], ptr_array(gate_streams), ptr_array(up_streams), num_experts,
        out_features, in_features, x_rows, pairs,
        None if weight is None else weight.data_ptr(), h.data_ptr(), workspace.data_ptr(),
        workspace.numel(), stream_handle(h.device))
    raise_for_status(status, "iqk_gemv_glu_run")
    return h


def swiglu_rows(g: torch.Tensor, u: torch.Tensor, weight: torch.Tensor | None,
                h: torch.Tensor) -> torch.Tensor:
    """``iqk_swiglu_rows``: h = silu(g) * u * weight[row], float32 [rows, cols]."""
    status = library().iqk_swiglu_rows(
        g.data_ptr(), u.data_ptr(), None if weight is None else weight.data_ptr(), g.shape[0],
        g.shape[1], h.data_ptr(), stream_handle(h.device))
    raise_for_status(status, "iqk_swiglu_rows")
    return h


def gemv_floor_run(member: str, streams, num_experts: int, out_features: int,
                   in_features: int, x_rows: int, pairs: int, y: torch.Tensor,
                   workspace: torch.Tensor) -> torch.Tensor:
    """``iqk_gemv_floor_run``: the GEMV's address floor (benchmark only)."""
    status = library().iqk_gemv_floor_run(
        MEMBER_IDS[member], ptr_array(streams), num_experts, out_features, in_features, x_rows,
        pairs, y.data_ptr(), DTYPE_IDS[y.dtype], workspace.data_ptr(), workspace.numel(),
        stream_handle(y.device))
    raise_for_status(status, "iqk_gemv_floor_run")
    return y


def dequant_floor(member: str, streams, num_experts: int, out_features: int, in_features: int,
                  row_start: int, rows: int, out: torch.Tensor) -> torch.Tensor:
    """``iqk_dequant_floor``: the dequantization's address floor (benchmark only)."""
    status = library().iqk_dequant_floor(MEMBER_IDS[check_member(member)], ptr_array(streams),
                                         num_experts, out_features, in_features, row_start,
                                         rows, DTYPE_IDS[out.dtype], out.data_ptr(),
                                         stream_handle(out.device))
    raise_for_status(status, "iqk_dequant_floor")
    return out


def gemv_static(member: str, x: torch.Tensor, streams, num_experts: int, out_features: int,
                in_features: int, sel: torch.Tensor, tok: torch.Tensor | None,
                y: torch.Tensor) -> torch.Tensor:
    """``iqk_gemv_static``: as :func:`gemv`, scratch in the library's static device array."""
    lib = library()
    check_device(y.device)
    status = lib.iqk_gemv_static(
        MEMBER_IDS[member], x.data_ptr(), DTYPE_IDS[x.dtype], x.shape[0], ptr_array(streams),
        num_experts, out_features, in_features, sel.data_ptr(),
        None if tok is None else tok.data_ptr(), sel.numel(), y.data_ptr(), DTYPE_IDS[y.dtype],
        stream_handle(y.device))
    raise_for_status(status, "iqk_gemv_static")
    return y


def gemv_static_read_error(in_features: int, x_rows: int, pairs: int,
                           device: torch.device | None = None) -> int:
    """``iqk_gemv_static_read_error``: the device error bits of the last
    ``iqk_gemv_static`` call of this geometry on the current device."""
    flags = ctypes.c_int32(0)
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    raise_for_status(library().iqk_gemv_static_read_error(in_features, x_rows, pairs,
                                                          ctypes.byref(flags),
                                                          stream_handle(dev)),
                     "iqk_gemv_static_read_error")
    return int(flags.value)


GROUPED_MEMBERS = ("iq2_ks", "iq2_k", "iq1_s_r4")
"""Members the tensor-core grouped GEMM (prefill route) covers."""


def grouped_workspace_bytes(in_features: int, num_experts: int, pairs: int) -> int:
    return int(library().iqk_grouped_workspace_bytes(in_features, num_experts, pairs))


def grouped(member: str, x: torch.Tensor, streams, num_experts: int, out_features: int,
            in_features: int, sel: torch.Tensor, tok: torch.Tensor | None, y: torch.Tensor,
            workspace: torch.Tensor | None = None) -> torch.Tensor:
    """``iqk_grouped_gemm``: x [x_rows, in], sel/tok int32 [pairs], y [pairs, out]."""
    lib = library()
    check_device(y.device)
    pairs = sel.numel()
    need = grouped_workspace_bytes(in_features, num_experts, pairs)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=y.device)
    status = lib.iqk_grouped_gemm(
        MEMBER_IDS[member], x.data_ptr(), DTYPE_IDS[x.dtype], x.shape[0], ptr_array(streams),
        num_experts, out_features, in_features, sel.data_ptr(),
        None if tok is None else tok.data_ptr(), pairs, y.data_ptr(), DTYPE_IDS[y.dtype],
        workspace.data_ptr(), workspace.numel(), stream_handle(y.device))
    raise_for_status(status, "iqk_grouped_gemm")
    return y


def grouped_prepare(x: torch.Tensor, num_experts: int, in_features: int, sel: torch.Tensor,
                    tok: torch.Tensor | None, workspace: torch.Tensor,
                    shard: bool = False) -> torch.Tensor:
    """``iqk_grouped_prepare``; with ``shard`` ``iqk_grouped_prepare_shard``
    (pairs whose expert lies outside [0, num_experts) are another rank's:
    skipped, no error, their output rows left untouched)."""
    lib = library()
    check_device(workspace.device)
    fn = lib.iqk_grouped_prepare_shard if shard else lib.iqk_grouped_prepare
    status = fn(
        x.data_ptr(), DTYPE_IDS[x.dtype], x.shape[0], in_features, num_experts,
        sel.data_ptr(), None if tok is None else tok.data_ptr(), sel.numel(),
        workspace.data_ptr(), workspace.numel(), stream_handle(workspace.device))
    raise_for_status(status, "iqk_grouped_prepare_shard" if shard else "iqk_grouped_prepare")
    return workspace


def grouped_run(member: str, streams, num_experts: int, out_features: int, in_features: int,
                pairs: int, y: torch.Tensor, workspace: torch.Tensor) -> torch.Tensor:
    lib = library()
    status = lib.iqk_grouped_run(
        MEMBER_IDS[member], ptr_array(streams), num_experts, out_features, in_features, pairs,
        y.data_ptr(), DTYPE_IDS[y.dtype], workspace.data_ptr(), workspace.numel(),
        stream_handle(y.device))
    raise_for_status(status, "iqk_grouped_run")
    return y


def grouped_run_range(member: str, streams, num_experts: int, out_features: int,
                      in_features: int, pairs: int, row_start: int, rows: int, y: torch.Tensor,
                      workspace: torch.Tensor) -> torch.Tensor:
    """``iqk_grouped_run_range``: output rows [row_start, row_start + rows) of
    every expert over a prepared workspace into ``y`` [pairs, rows]."""
    status = library().iqk_grouped_run_range(
        MEMBER_IDS[member], ptr_array(streams), num_experts, out_features, in_features, pairs,
        row_start, rows, y.data_ptr(), DTYPE_IDS[y.dtype], workspace.data_ptr(),
        workspace.numel(), stream_handle(y.device))
    raise_for_status(status, "iqk_grouped_run_range")
    return y


def pairs_swiglu(g: torch.Tensor, u: torch.Tensor, w: torch.Tensor, in_features: int,
                 num_experts: int, workspace: torch.Tensor, h: torch.Tensor) -> torch.Tensor:
    """``iqk_pairs_swiglu``: h[q] = bf16((silu(g[q]) * u[q]) * w[q]) for the pairs
    routed by ``workspace`` (prepared with ``in_features`` and ``num_experts``)."""
    pairs, inter = g.shape
    status = library().iqk_pairs_swiglu(
        g.data_ptr(), u.data_ptr(), w.data_ptr(), inter, in_features, num_experts, pairs,
        workspace.data_ptr(), workspace.numel(), h.data_ptr(), stream_handle(h.device))
    raise_for_status(status, "iqk_pairs_swiglu")
    return h


def pairs_combine(y: torch.Tensor, sel: torch.Tensor, top_k: int, num_experts: int,
                  out: torch.Tensor) -> torch.Tensor:
    """``iqk_pairs_combine``: out[r] = sum_j y[r*k + j] over the slots of row r
    whose sel lies in [0, num_experts)."""
    rows, hidden = out.shape
    status = library().iqk_pairs_combine(
        y.data_ptr(), sel.data_ptr(), rows, top_k, num_experts, hidden, out.data_ptr(),
        DTYPE_IDS[out.dtype], stream_handle(out.device))
    raise_for_status(status, "iqk_pairs_combine")
    return out


def grouped_read_error(workspace: torch.Tensor) -> int:
    flags = ctypes.c_int32(0)
    raise_for_status(library().iqk_grouped_read_error(workspace.data_ptr(), ctypes.byref(flags),
                                                      stream_handle(workspace.device)),
                     "iqk_grouped_read_error")
    return int(flags.value)


def read_error(workspace: torch.Tensor, in_features: int, x_rows: int, pairs: int) -> int:
    flags = ctypes.c_int32(0)
    raise_for_status(library().iqk_read_error(workspace.data_ptr(), in_features, x_rows, pairs,
                                              ctypes.byref(flags),
                                              stream_handle(workspace.device)),
                     "iqk_read_error")
    return int(flags.value)


__all__ = [
    "IQ2_MEMBERS", "ROWS_PER_TG", "SUPPORTED_IN_FEATURES", "IqkKernelError", "IqkRuntimeError",
    "check_dequant_geometry", "check_gemv_geometry", "dequant", "gemv", "library",
]
