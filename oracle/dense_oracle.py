"""CPU oracle for the dense IQ_K members: TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs
import this module, and only as the checker; the product package never
imports it and has no CPU fallback.

A dense matrix is one ``[out_features, in_features]`` tensor of
``IQ4_KS``, ``IQ4_K``, ``IQ5_K`` or ``IQ6_K`` rows. This module restates, in
numpy of its own:

* the wire geometry (``src/mlx_iqk/format.py:249-261, 340-349``),
* the relayout of ik wire rows into the k-contiguous streams the serving
  kernels read (``src/mlx_iqk/format.py:898-1100``: 4-bit code planes
  gathered into little-endian words, IQ5_K / IQ6_K high code bits into 1- and
  2-bit planes, scale planes concatenated unchanged),
* the serving decode (``src/mlx_iqk/format.py:1166-1240``): the CPU
  dequantizer's float32 chain ``dl = d * float(scale_index)`` then
  ``w = dl * value``, with IQ6_K's values read from the table of ik's cubic
  reconstruction (``IQ6K_TABLE``, format.py:188-213),
* a seeded wire generator (random code and scale bytes, serving-magnitude
  block scales), written from the block layouts.

Pinned to golden vectors the reference produced
(``tests/golden/make_golden_dense.py``); ``tests/test_dense.py`` checks it.
"""

from __future__ import annotations

import numpy as np

from dense_tables import IQ4K_VALUES, IQ5NL_VALUES, IQ6K_TABLE

QK_K = 256
DENSE_MEMBERS = ("iq4_ks", "iq4_k", "iq5_k", "iq6_k")
SUB_WEIGHTS = {"iq4_ks": 32, "iq4_k": 16, "iq5_k": 16, "iq6_k": 16}
BLOCK_BYTES = {"iq4_ks": 136, "iq4_k": 144, "iq5_k": 176, "iq6_k": 212}


def ik_row_bytes(member: str, n: int) -> int:
    """ggml row size: IQ4_KS carries a float32 row scale before its blocks."""
    return (4 if member == "iq4_ks" else 0) + BLOCK_BYTES[member] * (n // QK_K)


def stream_specs(member: str, n: int) -> dict[str, tuple[int, np.dtype]]:
    """Per-row length and dtype of each stream, in kernel input order."""
    u8, u32, f16 = np.dtype(np.uint8), np.dtype(np.uint32), np.dtype(np.float16)
    if member == "iq4_ks":
        return {"qs": (n // 8, u32), "scl": (n // 32, u8), "dv": (1, np.dtype(np.float32))}
    if member == "iq4_k":
        return {"qs": (n // 8, u32), "scl": (n // 32, u8), "sch": (n // 64, u8),
                "sex": (n // 128, u8), "dv": (n // 256, f16)}
    if member == "iq5_k":
        return {"qs": (n // 8, u32), "qh": (n // 32, u32), "scl": (n // 32, u8),
                "sch": (n // 64, u8), "sex": (n // 128, u8), "dv": (n // 256, f16)}
    return {"qs": (n // 8, u32), "qh": (n // 16, u32), "scl": (n // 16, u8),
            "sex": (n // 128, u8), "dv": (n // 256, f16)}


# ---------------------------------------------------------------- relayout


def _qs_place(member: str) -> tuple[np.ndarray, np.ndarray]:
    """Byte and shift of each super-block weight's 4-bit code in ik's qs."""
    w = np.arange(QK_K)
    if member in ("iq4_ks", "iq4_k"):
        return 16 * (w // 32) + w % 16, 4 * ((w % 32) // 16)
    return 32 * (w // 64) + w % 32, 4 * ((w % 64) // 32)


def _qh_place(member: str) -> tuple[np.ndarray, np.ndarray, int]:
    """Byte, shift and super-block qh bytes of the high code bits."""
    w = np.arange(QK_K)
    if member == "iq5_k":
        return w % 32, w // 32, 32
    return 32 * (w // 128) + w % 32, 2 * ((w // 32) % 4), 64


def _pack_fields(fields: np.ndarray, bits: int) -> np.ndarray:
    """k-ordered ``bits``-wide fields -> little-endian uint32 words."""
    rows, n = fields.shape
    per = 32 // bits
    f = fields.astype(np.uint32).reshape(rows, n // per, per)
    shifts = (bits * np.arange(per, dtype=np.uint32))[None, None, :]
    return np.bitwise_or.reduce(f << shifts, axis=2).astype(np.uint32)


def _unpack_fields(words: np.ndarray, bits: int, n: int) -> np.ndarray:
    rows = words.shape[0]
    per = 32 // bits
    shifts = (bits * np.arange(per, dtype=np.uint32))[None, None, :]
    f = (words.astype(np.uint32)[:, :, None] >> shifts) & np.uint32((1 << bits) - 1)
    return f.reshape(rows, -1)[:, :n]


def pack(member: str, wire: np.ndarray, n: int) -> dict[str, np.ndarray]:
    """ik wire rows ``[rows, ik_row_bytes]`` -> relayout streams."""
    wire = np.ascontiguousarray(wire, dtype=np.uint8)
    rows, nb = wire.shape[0], n // QK_K
    assert wire.shape[1] == ik_row_bytes(member, n), (member, wire.shape)
    out: dict[str, np.ndarray] = {}
    if member == "iq4_ks":
        body = wire[:, 4:].reshape(rows, nb, 136)
        scl, qsb = body[:, :, 0:8], body[:, :, 8:136]
        dv = wire[:, :4].copy().view(np.float32).reshape(rows)
    else:
        body = wire.reshape(rows, nb, BLOCK_BYTES[member])
        dv = body[:, :, 0:2].copy().reshape(rows, -1).view(np.float16)
        sex = body[:, :, 2:4].reshape(rows, nb * 2)
        if member == "iq6_k":
            scl, qsb = body[:, :, 4:20], body[:, :, 20:148]
            qhb = body[:, :, 148:212]
        else:
            sch, scl, qsb = body[:, :, 4:8], body[:, :, 8:16], body[:, :, 16:144]
            if member == "iq5_k":
                qhb = body[:, :, 144:176]
    byte, shift = _qs_place(member)
    codes = (qsb[:, :, byte] >> shift[None, None, :]) & 0xF           # [rows, nb, 256]
    out["qs"] = _pack_fields(codes.reshape(rows, n), 4)
    if member in ("iq5_k", "iq6_k"):
        hb, hs, _ = _qh_place(member)
        bits = 1 if member == "iq5_k" else 2
        high = (qhb[:, :, hb] >> hs[None, None, :]) & ((1 << bits) - 1)
        out["qh"] = _pack_fields(high.reshape(rows, n), bits)
    out["scl"] = np.ascontiguousarray(scl.reshape(rows, -1))
    if member in ("iq4_k", "iq5_k"):
        out["sch"] = np.ascontiguousarray(sch.reshape(rows, -1))
    if member != "iq4_ks":
        out["sex"] = np.ascontiguousarray(sex)
    out["dv"] = np.ascontiguousarray(dv)
    return out


# ------------------------------------------------------------------ decode


def decode(member: str, streams: dict[str, np.ndarray], n: int) -> np.ndarray:
    """Relayout streams -> float32 weights ``[rows, n]``, bit for bit the
    serving decode: ``dl = d * float(scale_index)`` then ``dl * value``, two
    separate float32 multiplies (numpy does not contract them)."""
    qs = streams["qs"]
    rows = qs.shape[0]
    sub = SUB_WEIGHTS[member]
    nsub = n // sub
    codes = _unpack_fields(qs, 4, n).astype(np.int64)
    if member == "iq5_k":
        codes |= _unpack_fields(streams["qh"], 1, n).astype(np.int64) << 4
    elif member == "iq6_k":
        codes |= _unpack_fields(streams["qh"], 2, n).astype(np.int64) << 4
    if member == "iq4_ks":
        scl = streams["scl"].astype(np.int64)
        index = (scl & 254) - 127
        alpha = scl & 1
        d = np.asarray(streams["dv"], dtype=np.float32).reshape(rows, 1)
    else:
        if member == "iq6_k":
            index = streams["scl"].view(np.int8).astype(np.int64)
        else:
            scl = streams["scl"].astype(np.int64)
            sch = streams["sch"].astype(np.int64)
            lo = np.stack([scl & 15, scl >> 4], axis=2).reshape(rows, nsub)
            hi = np.stack([(sch >> (2 * j)) & 3 for j in range(4)], axis=2).reshape(rows, nsub)
            index = (lo | (hi << 4)) - 32
        sex = streams["sex"].astype(np.int64)
        alpha = np.stack([(sex >> j) & 1 for j in range(8)], axis=2).reshape(rows, nsub)
        d = np.repeat(np.asarray(streams["dv"]).astype(np.float32), QK_K // sub, axis=1)
    dl = (d * index.astype(np.float32)).astype(np.float32)                # [rows, nsub]
    width = {"iq4_ks": 4, "iq4_k": 4, "iq5_k": 5, "iq6_k": 6}[member]
    tidx = np.repeat(alpha << width, sub, axis=1) + codes
    if member == "iq6_k":
        values = IQ6K_TABLE[tidx]
    else:
        table = IQ5NL_VALUES if member == "iq5_k" else IQ4K_VALUES
        values = table.astype(np.float32)[tidx]
    return (np.repeat(dl, sub, axis=1) * values).astype(np.float32)


def dequant_wire(member: str, wire: np.ndarray, n: int) -> np.ndarray:
    return decode(member, pack(member, wire, n), n)


def gemv_f64(weights: np.ndarray, x: np.ndarray) -> np.ndarray:
    """``x [tokens, n] @ W.T`` in float64."""
    return np.asarray(x, dtype=np.float64) @ np.asarray(weights, dtype=np.float64).T


# --------------------------------------------------------------- generator


def random_wire(member: str, rows: int, n: int, seed: int) -> np.ndarray:
    """Random wire rows: every code, scale and alphabet byte uniform (all of
    them are legal and the decode is branch-free over them); the fp16 (IQ4_KS:
    float32) block scales drawn at serving magnitudes, so the reconstructed
    weights have the spread real layers have."""
    rng = np.random.default_rng(seed)
    nb = n // QK_K
    out = rng.integers(0, 256, size=(rows, ik_row_bytes(member, n)), dtype=np.uint8)
    if member == "iq4_ks":
        mag = rng.uniform(2e-5, 8e-4, size=rows).astype(np.float32)
        d = np.where(rng.random(rows) < 0.5, -mag, mag).astype(np.float32)
        out[:, 0:4] = d.view(np.uint8).reshape(rows, 4)
        return out
    body = out.reshape(rows, nb, BLOCK_BYTES[member])
    mag = rng.uniform(2e-5, 8e-4, size=(rows, nb))
    d = np.where(rng.random((rows, nb)) < 0.5, -mag, mag).astype(np.float16)
    body[:, :, 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
    return out


def random_streams(member: str, rows: int, n: int, seed: int) -> dict[str, np.ndarray]:
    return pack(member, random_wire(member, rows, n, seed), n)
