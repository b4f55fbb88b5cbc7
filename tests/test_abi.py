"""The C ABI library: loads on a CPU-only host, exports every declared symbol,
and rejects bad geometry before touching the device (no GPU needed)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from mlx_iqk_b200 import IqkSwitchLinear
from mlx_iqk_b200 import format as fmt
from mlx_iqk_b200 import kernels as K

REPO = Path(__file__).resolve().parents[1]


def declared_symbols() -> list[str]:
    text = (REPO / "include" / "iqk_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(iqk_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = K.library()
    names = declared_symbols()
    assert names, "no declarations parsed"
    for name in names:
        assert hasattr(lib, name), name
    assert sorted(K.exported_symbols()) == names


def test_status_strings_and_version():
    lib = K.library()
    assert lib.iqk_abi_version() == 1
    for code in range(0, 9):
        assert lib.iqk_status_string(code)


@pytest.mark.parametrize("member", [0, 1, 2])
def test_workspace_size_is_positive_and_grows(member):
    lib = K.library()
    a = lib.iqk_gemv_workspace_bytes(member, 4096, 1, 6)
    b = lib.iqk_gemv_workspace_bytes(member, 4096, 8, 48)
    assert 0 < a < b
    assert lib.iqk_gemv_workspace_bytes(member, 1024, 1, 6) == 0


def test_host_side_rejections_need_no_device():
    lib = K.library()
    streams = (ctypes.c_void_p * 5)()
    # bad member, bad width, bad geometry: decided before any CUDA call
    assert lib.iqk_dequant(7, streams, 1, 32, 2048, 0, 32, 0, None, None) == 1
    assert lib.iqk_dequant(0, streams, 1, 32, 1024, 0, 32, 0, None, None) == 2
    assert lib.iqk_dequant(0, streams, 0, 32, 2048, 0, 32, 0, None, None) == 3
    assert lib.iqk_dequant(0, streams, 1, 32, 2048, 16, 32, 0, None, None) == 3
    assert lib.iqk_dequant(2, streams, 1, 30, 2048, 0, 30, 0, None, None) == 3
    assert lib.iqk_gemv(0, None, 2, 1, streams, 8, 24, 2048, None, None, 6, None, 0, None, 0,
                        None) == 3  # out_features % 16
    assert lib.iqk_gemv(0, None, 2, 4, streams, 8, 32, 2048, None, None, 6, None, 0, None, 0,
                        None) == 3  # pairs do not tile the rows
    assert lib.iqk_gemv_run(0, streams, 8, 32, 3072, 1, 6, None, 0, None, 0, None) == 2
    assert lib.iqk_gemv_prepare(None, 9, 1, 2048, 8, None, None, 6, None, 0, None) == 4



def test_dense_alignment_rejections_need_no_device():
    """Every dense stream and the GEMV's activations must start on a 16-byte
    boundary (the GEMV stages stream rows with 16-byte asynchronous copies and
    loads 8-byte activation fragments); the ABI refuses others before any
    CUDA call."""
    lib = K.library()
    ok = [0x10000 * (i + 1) for i in range(5)]  # aligned stand-ins, never dereferenced

    def gemv(x, streams, member=4):
        arr = (ctypes.c_void_p * 5)(*streams)
        return lib.iqk_dense_gemv(member, x, 1, arr, 16, 1024, 0x90000, 1, None)

    assert gemv(0x80008, ok) == 5  # x 8-byte aligned only
    for i in range(5):  # IQ4_K has five streams: qs, scl, sch, sex, dv
        bad = list(ok)
        bad[i] += 8
        assert gemv(0x80000, bad) == 5, i
        arr = (ctypes.c_void_p * 5)(*bad)
        assert lib.iqk_dense_dequant(4, arr, 16, 1024, 0, 16, 1, 0x90000, None) == 5, i


# -- Python layer: geometry guards and the stream contract (CPU tensors) -----


@pytest.mark.parametrize("member", fmt.MEMBERS)
@pytest.mark.parametrize("bad", [1024, 1536, 2560, 3072, 4352, 8192])
def test_module_refuses_unsized_input_widths(member, bad):
    with pytest.raises(K.IqkKernelError):
        IqkSwitchLinear(member, 4, 32, bad, device="cpu")


@pytest.mark.parametrize("bad", [24, 40, 100])
def test_module_refuses_out_features_that_do_not_tile(bad):
    with pytest.raises(K.IqkKernelError):
        IqkSwitchLinear("iq2_ks", 4, bad, 2048, device="cpu")


def test_row_width_that_is_not_a_block_multiple_is_a_format_error():
    with pytest.raises(fmt.IqkFormatError):
        IqkSwitchLinear("iq2_ks", 4, 32, 4000, device="cpu")
    with pytest.raises(fmt.IqkFormatError):
        IqkSwitchLinear("iq3_k", 4, 32, 2048, device="cpu")


def test_nonpositive_experts_are_refused():
    with pytest.raises(K.IqkRuntimeError):
        IqkSwitchLinear("iq2_k", 0, 32, 2048, device="cpu")


@pytest.mark.parametrize("member", fmt.MEMBERS)
def test_load_streams_checks_names_shapes_and_widths(member):
    mod = IqkSwitchLinear(member, 4, 32, 2048, device="cpu")
    shapes = fmt.component_shapes(member, 4, 32, 2048)
    dtypes = fmt.component_dtypes(member)
    good = {k: np.zeros(s, dtype=dtypes[k]) for k, s in shapes.items()}
    mod.load_streams(good)
    bad = dict(good)
    bad["qs"] = np.zeros((4, 32, 3), dtype=np.uint32)
    with pytest.raises(K.IqkRuntimeError):
        mod.load_streams(bad)
    missing = dict(good)
    missing.pop(list(shapes)[1])
    with pytest.raises(K.IqkRuntimeError):
        mod.load_streams(missing)
    wide = dict(good)
    wide["dv"] = np.zeros(shapes["dv"], dtype=np.float32)
    with pytest.raises(K.IqkRuntimeError):
        mod.load_streams(wide)
    # a same-width integer view of the bytes is accepted and reinterpreted
    same = dict(good)
    same["qs"] = np.zeros(shapes["qs"], dtype=np.int32)
    mod.load_streams(same)
    assert mod.qs.dtype == torch.uint32


def test_stream_names_follow_the_format_order():
    for member in fmt.MEMBERS:
        mod = IqkSwitchLinear(member, 2, 16, 2048, device="cpu")
        assert mod.stream_names() == list(fmt.component_shapes(member, 1, 1, 2048))
        assert mod.mode == "iqk"


def test_range_guard_matches_the_reference():
    mod = IqkSwitchLinear("iq2_ks", 2, 32, 2048, device="cpu")
    for start, rows in ((0, 0), (0, 12), (0, -8), (-8, 8), (28, 8), (0, 64)):
        with pytest.raises(K.IqkRuntimeError):
            mod.dequantized_range(start, rows)


def test_iq1_has_no_sorted_or_union_formulation():
    mod = IqkSwitchLinear("iq1_s_r4", 2, 32, 2048, device="cpu")
    x = torch.zeros(2, 1, 1, 2048)
    ids = torch.zeros(4, dtype=torch.int32)
    with pytest.raises(K.IqkKernelError):
        mod.gemv_sorted(x, ids, ids)
    with pytest.raises(K.IqkKernelError):
        mod.gemv_union(x, ids, ids)


def test_gemv_refuses_a_pair_count_that_does_not_tile_the_rows():
    mod = IqkSwitchLinear("iq2_k", 2, 32, 2048, device="cpu")
    with pytest.raises(K.IqkRuntimeError):
        mod.gemv(torch.zeros(3, 1, 1, 2048), torch.zeros(1, 4, dtype=torch.int64))
