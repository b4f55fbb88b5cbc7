"""Geometry of the IQ_K relayout streams the B200 kernels serve.

The relayout itself is the reference's (``src/mlx_iqk/format.py``): one
logical weight tensor ``[out_features, in_features]`` per expert, every
stream k-contiguous per output row. This module restates the geometry the
serving side needs -- member names, row widths, byte budgets, stream shapes
and dtypes -- with the reference's names, signatures and error class, so a
caller's shape checks behave the same. Byte layout per member:

``iq2_ks``   qs u32[n/16], scl u8[n/64], sch u8[n/256], sex u8[n/256], dv f16[1]
``iq2_k``    qs u32[n/16], scl u8[n/32], sex u8[n/128], dv f16[n/256]
``iq1_s_r4`` qs u32[n/32], qh u16[n/32], dv f16[1]

and of the dense members (one ``[out, in]`` matrix, no expert axis;
src/mlx_iqk/format.py:898-935):

``iq4_ks``   qs u32[n/8], scl u8[n/32], dv f32[1]
``iq4_k``    qs u32[n/8], scl u8[n/32], sch u8[n/64], sex u8[n/128], dv f16[n/256]
``iq5_k``    qs u32[n/8], qh u32[n/32], scl u8[n/32], sch u8[n/64], sex u8[n/128], dv f16[n/256]
``iq6_k``    qs u32[n/8], qh u32[n/16], scl u8[n/16], sex u8[n/128], dv f16[n/256]

Reconstruction (the CPU dequantizer's float32 chain, which the dequant
kernel reproduces bit for bit): ``d * float(idx) * values[4*alpha + code]``
for the 2-bit members, ``d * float(2*ls + 1) * (float(grid) + shift)`` for
``iq1_s_r4``.
"""

from __future__ import annotations

import numpy as np

QK_K = 256
"""Weights per ik super-block of the two 2-bit members."""

IQ2NL_VALUES = np.array([-31, -13, 1, 17, -26, -8, 6, 22], dtype=np.int8)
"""``iq2nl_values``: base alphabet 0..3, shifted alphabet 4..7
(src/mlx_iqk/format.py:110)."""

MEMBERS = ("iq2_ks", "iq2_k", "iq1_s_r4")
"""Routed-expert members this package serves (src/mlx_iqk/format.py:116)."""

MEMBER_IDS = {"iq2_ks": 0, "iq2_k": 1, "iq1_s_r4": 2}
"""Member codes of the C ABI (``IQK_IQ2_KS`` ... in include/iqk_b200.h)."""

DENSE_MEMBERS = ("iq4_ks", "iq4_k", "iq5_k", "iq6_k")
"""Dense-tensor members (src/mlx_iqk/format.py:120), served by ``mlx_iqk_b200.dense``."""

DENSE_MEMBER_IDS = {"iq4_ks": 3, "iq4_k": 4, "iq5_k": 5, "iq6_k": 6}
"""Their member codes in the C ABI (``IQK_IQ4_KS`` ... in include/iqk_b200.h)."""

SUB_WEIGHTS = {"iq2_ks": 32, "iq2_k": 16, "iq1_s_r4": 32,
               "iq4_ks": 32, "iq4_k": 16, "iq5_k": 16, "iq6_k": 16}
"""Weights sharing one scale index (src/mlx_iqk/format.py:122-126)."""

WIRE_GROUP_ROWS = {"iq2_ks": 1, "iq2_k": 1, "iq1_s_r4": 4,
                   "iq4_ks": 1, "iq4_k": 1, "iq5_k": 1, "iq6_k": 1}
"""Rows one addressable ik-wire unit covers (src/mlx_iqk/format.py:130-139)."""

BLOCK_WEIGHTS = {"iq2_ks": QK_K, "iq2_k": QK_K, "iq1_s_r4": 32,
                 "iq4_ks": QK_K, "iq4_k": QK_K, "iq5_k": QK_K, "iq6_k": QK_K}
"""Weights per wire block: each member's row-width granularity."""

ALPHABET_SIZES = {"iq4_ks": 16, "iq4_k": 16, "iq5_k": 32, "iq6_k": 64}
"""Entries per alphabet of each dense member (two alphabets each)."""

IQ2_KS_BLOCK_BYTES = 70
IQ2_K_BLOCK_BYTES = 76
IQ1_S_R4_BLOCK_BYTES = 24
IQ2_KS_ROW_META_BYTES = 2
IQ1_S_R4_ROW_META_BYTES = 2
IQ1S_DELTA = 0.125

IQ4_KS_BLOCK_BYTES = 136
IQ4_KS_ROW_META_BYTES = 4
IQ4_K_BLOCK_BYTES = 144
IQ5_K_BLOCK_BYTES = 176
IQ6_K_BLOCK_BYTES = 212

_BLOCK_BYTES = {"iq2_ks": 70, "iq2_k": 76, "iq1_s_r4": 24 // 4,
                "iq4_ks": 136, "iq4_k": 144, "iq5_k": 176, "iq6_k": 212}
_ROW_META_BYTES = {"iq2_ks": 2, "iq1_s_r4": 2, "iq4_ks": 4}


class IqkFormatError(ValueError):
    """Geometry or member the relayout does not define (reference class name)."""


def check_member(member: str) -> str:
    if member not in MEMBERS:
        raise IqkFormatError(f"iqk routed member {member!r} not in {MEMBERS}")
    return member


def check_dense_member(member: str) -> str:
    if member not in DENSE_MEMBERS:
        raise IqkFormatError(f"iqk dense member {member!r} not in {DENSE_MEMBERS}")
    return member


def check_any_member(member: str) -> str:
    if member not in MEMBERS and member not in DENSE_MEMBERS:
        raise IqkFormatError(f"iqk member {member!r} not in {MEMBERS + DENSE_MEMBERS}")
    return member


def check_row_width(in_features: int, member: str = "iq2_ks") -> int:
    """Row widths the relayout defines: multiples of the member's block."""
    n = int(in_features)
    block = BLOCK_WEIGHTS[check_any_member(member)]
    if n <= 0 or n % block:
        raise IqkFormatError(
            f"in_features {in_features} is not a positive multiple of {block}; ik "
            "silently substitutes a different type for such a row rather than "
            "failing, so the width is rejected here instead")
    return n


def check_wire_rows(member: str, rows: int) -> int:
    group = WIRE_GROUP_ROWS[check_any_member(member)]
    r = int(rows)
    if r <= 0 or r % group:
        raise IqkFormatError(
            f"{member} wire rows come in groups of {group}; {rows} rows do "
            "not split into whole groups")
    return r


def ik_row_bytes(member: str, in_features: int) -> int:
    """Bytes of one ik-layout row (ggml's row size)."""
    n = check_row_width(in_features, member)
    return _ROW_META_BYTES.get(member, 0) + _BLOCK_BYTES[member] * (n // BLOCK_WEIGHTS[member])


def component_shapes(member: str, num_experts: int, out_features: int,
                     in_features: int) -> dict[str, tuple[int, ...]]:
    """Stacked-expert shape of every relayout stream, in kernel input order."""
    check_member(member)
    n = check_row_width(in_features, member)
    e, o = int(num_experts), int(out_features)
    if member == "iq2_ks":
        return {"qs": (e, o, n // 16), "scl": (e, o, n // 64), "sch": (e, o, n // 256),
                "sex": (e, o, n // 256), "dv": (e, o)}
    if member == "iq1_s_r4":
        return {"qs": (e, o, n // 32), "qh": (e, o, n // 32), "dv": (e, o)}
    return {"qs": (e, o, n // 16), "scl": (e, o, n // 32), "sex": (e, o, n // 128),
            "dv": (e, o, n // 256)}


def component_dtypes(member: str) -> dict[str, np.dtype]:
    """NumPy dtype of every relayout stream."""
    check_member(member)
    if member == "iq1_s_r4":
        return {"qs": np.dtype(np.uint32), "qh": np.dtype(np.uint16),
                "dv": np.dtype(np.float16)}
    names = ("qs", "scl", "sch", "sex", "dv") if member == "iq2_ks" else ("qs", "scl", "sex", "dv")
    return {nm: (np.dtype(np.float16) if nm == "dv" else
                 np.dtype(np.uint32) if nm == "qs" else np.dtype(np.uint8)) for nm in names}


def dense_component_shapes(member: str, out_features: int,
                           in_features: int) -> dict[str, tuple[int, ...]]:
    """Dense-matrix shape of every stream, in kernel input order: the
    single-expert case of the relayout, the expert axis dropped."""
    check_dense_member(member)
    n = check_row_width(in_features, member)
    o = int(out_features)
    if o <= 0:
        raise IqkFormatError(f"out_features {out_features} is not positive")
    if member == "iq4_ks":
        return {"qs": (o, n // 8), "scl": (o, n // 32), "dv": (o,)}
    if member == "iq4_k":
        return {"qs": (o, n // 8), "scl": (o, n // 32), "sch": (o, n // 64),
                "sex": (o, n // 128), "dv": (o, n // 256)}
    if member == "iq5_k":
        return {"qs": (o, n // 8), "qh": (o, n // 32), "scl": (o, n // 32),
                "sch": (o, n // 64), "sex": (o, n // 128), "dv": (o, n // 256)}
    return {"qs": (o, n // 8), "qh": (o, n // 16), "scl": (o, n // 16),
            "sex": (o, n // 128), "dv": (o, n // 256)}


def dense_component_dtypes(member: str) -> dict[str, np.dtype]:
    """NumPy dtype of every dense stream: ``dv`` is float32 for ``iq4_ks``
    (its row scale is fp32 on the wire), fp16 otherwise; ``scl`` of
    ``iq6_k`` holds the signed scale as its byte."""
    names = tuple(dense_component_shapes(member, 1, QK_K))
    dv = np.dtype(np.float32) if member == "iq4_ks" else np.dtype(np.float16)
    return {nm: (dv if nm == "dv" else np.dtype(np.uint32) if nm in ("qs", "qh")
                 else np.dtype(np.uint8)) for nm in names}


def bits_per_weight(member: str, in_features: int) -> float:
    return 8.0 * ik_row_bytes(member, in_features) / check_row_width(in_features, member)


def relayout_row_bytes(member: str, in_features: int) -> int:
    """Bytes of one relayout row; equal to :func:`ik_row_bytes` by construction."""
    if member in DENSE_MEMBERS:
        shapes = dense_component_shapes(member, 1, in_features)
        dtypes = dense_component_dtypes(member)
        return sum(int(np.prod(shape[1:])) * dtypes[nm].itemsize for nm, shape in shapes.items())
    shapes = component_shapes(member, 1, 1, in_features)
    dtypes = component_dtypes(member)
    return sum(int(np.prod(shape)) * dtypes[nm].itemsize for nm, shape in shapes.items())


__all__ = [
    "ALPHABET_SIZES", "BLOCK_WEIGHTS", "DENSE_MEMBERS", "DENSE_MEMBER_IDS", "IQ2NL_VALUES",
    "MEMBERS", "MEMBER_IDS", "QK_K", "SUB_WEIGHTS", "WIRE_GROUP_ROWS", "IqkFormatError",
    "bits_per_weight", "check_any_member", "check_dense_member", "check_member",
    "check_row_width", "check_wire_rows", "component_dtypes", "component_shapes",
    "dense_component_dtypes", "dense_component_shapes", "ik_row_bytes", "relayout_row_bytes",
]
