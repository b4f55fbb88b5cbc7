"""CPU oracle for the IQ_K routed-expert hot path: TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg import this module, and only as the checker. The product package
(``mlx_iqk_b200``) never imports it and has no CPU fallback.

What lives here:

* a numpy restatement of the reference's wire relayout, ``pack`` / ``unpack``
  (``src/mlx_iqk/format.py:423-772``), so a test can turn ik wire bytes into
  the streams ``IqkSwitchLinear.load_streams`` consumes;
* seeded wire generators of this repo's own (random byte space, serving
  scales, exhaustive decode value space), written from the block layouts,
  not from the reference's ``tests/wirepack.py``;
* ctypes bindings to ``oracle/iqk_oracle.c`` (the C restatement of the
  decode; see that file's header) and, when it was built, to the reference's
  own vendored codec in ``oracle/_ref/`` (``codec.quantize`` /
  ``codec.dequantize``, ``src/mlx_iqk/codec.py:238-293``).

Pinned against golden vectors the reference produced
(``tests/golden/make_golden.py``); ``tests/test_oracle.py`` checks it.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import zlib
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
QK_K = 256
MEMBERS = ("iq2_ks", "iq2_k", "iq1_s_r4")
IQ2NL_VALUES = np.array([-31, -13, 1, 17, -26, -8, 6, 22], dtype=np.int8)


def seed_for(*parts) -> int:
    """Stable seed from a label (crc32), independent of Python's hash salt."""
    return zlib.crc32("|".join(str(p) for p in parts).encode()) % (2 ** 31)


# ---------------------------------------------------------------- geometry


def ik_row_bytes(member: str, n: int) -> int:
    """ggml row size of one wire row (``src/mlx_iqk/format.py:340-349``)."""
    if member == "iq2_ks":
        return 2 + 70 * (n // QK_K)
    if member == "iq2_k":
        return 76 * (n // QK_K)
    if member == "iq1_s_r4":
        return 2 + 6 * (n // 32)
    raise ValueError(member)


def stream_specs(member: str, n: int) -> dict[str, tuple[int, np.dtype]]:
    """Per-row length and dtype of each relayout stream, in kernel order."""
    if member == "iq2_ks":
        return {"qs": (n // 16, np.uint32), "scl": (n // 64, np.uint8),
                "sch": (n // 256, np.uint8), "sex": (n // 256, np.uint8),
                "dv": (1, np.float16)}
    if member == "iq2_k":
        return {"qs": (n // 16, np.uint32), "scl": (n // 32, np.uint8),
                "sex": (n // 128, np.uint8), "dv": (n // 256, np.float16)}
    if member == "iq1_s_r4":
        return {"qs": (n // 32, np.uint32), "qh": (n // 32, np.uint16),
                "dv": (1, np.float16)}
    raise ValueError(member)


# ------------------------------------------------------ wire <-> relayout


def _code_positions(member: str, n: int) -> tuple[np.ndarray, np.ndarray]:
    """(byte, shift) of every k-ordered weight's 2-bit code in the wire qs.

    IQ2_K  (vendor/ik_llama/iqk_iq2.cpp:512-524): weight w of a super-block,
    ib32 = w/32, half = (w%32)/16, j = w%16 -> byte 32*(ib32/4) + 16*half + j,
    shift 2*(ib32%4).
    IQ2_KS (iqk_iq2.cpp:545-558): ib64 = w/64, half = (w%64)/32, j = w%32 ->
    byte 32*(ib64/2) + j, shift 4*(ib64%2) + 2*half.
    """
    w = np.arange(QK_K)
    if member == "iq2_k":
        ib32 = w // 32
        byte = 32 * (ib32 // 4) + 16 * ((w % 32) // 16) + (w % 16)
        shift = 2 * (ib32 % 4)
    else:
        ib64 = w // 64
        byte = 32 * (ib64 // 2) + (w % 32)
        shift = 4 * (ib64 % 2) + 2 * ((w % 64) // 32)
    nb = n // QK_K
    blocks = np.arange(nb)[:, None] * 64
    return (blocks + byte[None, :]).reshape(-1), np.tile(shift, nb)


def _codes_to_words(codes: np.ndarray) -> np.ndarray:
    """k-ordered 2-bit codes [rows, n] -> little-endian uint32 words [rows, n/16]."""
    rows, n = codes.shape
    c = codes.astype(np.uint32).reshape(rows, n // 16, 16)
    return np.bitwise_or.reduce(c << (2 * np.arange(16, dtype=np.uint32)), axis=2)


def _words_to_codes(words: np.ndarray, n: int) -> np.ndarray:
    rows = words.shape[0]
    w = words.astype(np.uint32).reshape(rows, n // 16, 1)
    return ((w >> (2 * np.arange(16, dtype=np.uint32))) & 3).reshape(rows, n).astype(np.uint8)


def _bits_lsb(bytes_: np.ndarray, count: int) -> np.ndarray:
    return np.unpackbits(bytes_, axis=1, bitorder="little")[:, :count]


def pack(member: str, wire: np.ndarray, n: int) -> dict[str, np.ndarray]:
    """ik wire rows [rows, ik_row_bytes] -> relayout streams, each [rows, len].

    Restates ``format.pack`` (``src/mlx_iqk/format.py:664-678``): the same bits
    re-placed so every stream is k-contiguous per row.
    """
    wire = np.ascontiguousarray(wire, dtype=np.uint8)
    rows = wire.shape[0]
    assert wire.shape[1] == ik_row_bytes(member, n), (wire.shape, member, n)
    if member == "iq1_s_r4":
        assert rows % 4 == 0
        nblock = n // 32
        groups = wire.reshape(rows // 4, 4 * ik_row_bytes(member, n))
        dv = groups[:, :8].copy().view(np.float16).reshape(rows)
        body = groups[:, 8:].reshape(rows // 4, nblock, 24)
        # qs byte 4*i + k: sub-group i of row k; qh u16 k: row k's block word.
        qsb = body[:, :, :16].reshape(rows // 4, nblock, 4, 4)       # [g, b, i, k]
        qs = np.ascontiguousarray(qsb.transpose(0, 3, 1, 2)).reshape(rows, nblock * 4)
        qh = body[:, :, 16:].copy().view(np.uint16).reshape(rows // 4, nblock, 4)
        return {"qs": qs.view(np.uint32).reshape(rows, nblock),
                "qh": np.ascontiguousarray(qh.transpose(0, 2, 1)).reshape(rows, nblock),
                "dv": dv.reshape(rows, 1)}
    nb = n // QK_K
    if member == "iq2_ks":
        dv = wire[:, :2].copy().view(np.float16).reshape(rows, 1)
        body = wire[:, 2:].reshape(rows, nb, 70)
        extra_lo, extra_hi = body[:, :, 0], body[:, :, 1]
        scales = body[:, :, 2:6].reshape(rows, nb * 4)
        qsw = body[:, :, 6:].reshape(rows, nb * 64)
        byte, shift = _code_positions(member, n)
        codes = (qsw[:, byte] >> shift[None, :]) & 3
        return {"qs": _codes_to_words(codes), "scl": np.ascontiguousarray(scales),
                "sch": np.ascontiguousarray(extra_hi), "sex": np.ascontiguousarray(extra_lo),
                "dv": dv}
    body = wire.reshape(rows, nb, 76)
    dv = body[:, :, 0:2].copy().view(np.float16).reshape(rows, nb)
    sex = body[:, :, 2:4].reshape(rows, nb * 2)
    scales = body[:, :, 4:12].reshape(rows, nb * 8)
    qsw = body[:, :, 12:].reshape(rows, nb * 64)
    byte, shift = _code_positions(member, n)
    codes = (qsw[:, byte] >> shift[None, :]) & 3
    return {"qs": _codes_to_words(codes), "scl": np.ascontiguousarray(scales),
            "sex": np.ascontiguousarray(sex), "dv": dv}


def unpack(member: str, streams: dict[str, np.ndarray], n: int) -> np.ndarray:
    """Inverse of :func:`pack` (``src/mlx_iqk/format.py:744-772``)."""
    specs = stream_specs(member, n)
    s = {k: np.ascontiguousarray(v).reshape(-1, specs[k][0]) for k, v in streams.items()}
    rows = s["qs"].shape[0]
    rb = ik_row_bytes(member, n)
    if member == "iq1_s_r4":
        nblock = n // 32
        out = np.zeros((rows // 4, 4 * rb), dtype=np.uint8)
        out[:, :8] = s["dv"].astype(np.float16).reshape(rows // 4, 4).view(np.uint8)
        body = out[:, 8:].reshape(rows // 4, nblock, 24)
        qsb = s["qs"].astype(np.uint32).view(np.uint8).reshape(rows // 4, 4, nblock, 4)
        body[:, :, :16] = qsb.transpose(0, 2, 3, 1).reshape(rows // 4, nblock, 16)
        qh = s["qh"].astype(np.uint16).reshape(rows // 4, 4, nblock).transpose(0, 2, 1)
        body[:, :, 16:] = np.ascontiguousarray(qh).view(np.uint8).reshape(rows // 4, nblock, 8)
        return out.reshape(rows, rb)
    nb = n // QK_K
    codes = _words_to_codes(s["qs"], n)
    byte, shift = _code_positions(member, n)
    qsw = np.zeros((rows, nb * 64), dtype=np.uint8)
    for sh in np.unique(shift):
        m = shift == sh
        qsw[:, byte[m]] |= (codes[:, m] << sh).astype(np.uint8)
    out = np.zeros((rows, rb), dtype=np.uint8)
    if member == "iq2_ks":
        out[:, :2] = s["dv"].astype(np.float16).reshape(rows, 1).view(np.uint8)
        body = out[:, 2:].reshape(rows, nb, 70)
        body[:, :, 0] = s["sex"].reshape(rows, nb)
        body[:, :, 1] = s["sch"].reshape(rows, nb)
        body[:, :, 2:6] = s["scl"].reshape(rows, nb, 4)
        body[:, :, 6:] = qsw.reshape(rows, nb, 64)
        return out
    body = out.reshape(rows, nb, 76)
    body[:, :, 0:2] = s["dv"].astype(np.float16).reshape(rows, nb, 1).view(np.uint8)
    body[:, :, 2:4] = s["sex"].reshape(rows, nb, 2)
    body[:, :, 4:12] = s["scl"].reshape(rows, nb, 8)
    body[:, :, 12:] = qsw.reshape(rows, nb, 64)
    return out


def decode(member: str, streams: dict[str, np.ndarray], n: int) -> np.ndarray:
    """Relayout streams -> float32 weights [rows, n] through the C restatement."""
    lib = load_port()
    s = {k: np.ascontiguousarray(v) for k, v in streams.items()}
    rows = s["qs"].shape[0]
    out = np.empty((rows, n), dtype=np.float32)
    p = _ptr
    if member == "iq2_ks":
        lib.orc_decode_iq2_ks(p(s["qs"]), p(s["scl"]), p(s["sch"]), p(s["sex"]),
                              p(s["dv"]), rows, n, p(out))
    elif member == "iq2_k":
        lib.orc_decode_iq2_k(p(s["qs"]), p(s["scl"]), p(s["sex"]), p(s["dv"]),
                             rows, n, p(out))
    else:
        lib.orc_decode_iq1_s_r4(p(s["qs"]), p(s["qh"]), p(s["dv"]), rows, n, p(out))
    return out


def dequant_wire(member: str, wire: np.ndarray, n: int) -> np.ndarray:
    """ik wire rows -> float32 through the C restatement of ik's dequantizer."""
    lib = load_port()
    w = np.ascontiguousarray(wire, dtype=np.uint8)
    rows = w.shape[0]
    out = np.empty((rows, n), dtype=np.float32)
    getattr(lib, f"orc_dequant_{member}")(_ptr(w), rows, n, _ptr(out))
    return out


def gemv_f64(weights: np.ndarray, x: np.ndarray, sel: np.ndarray,
             tok: np.ndarray) -> np.ndarray:
    """Float64 y[p, r] = sum_k W[sel[p], r, k] x[tok[p], k]; W float32 [E, out, n]."""
    lib = load_port()
    w = np.ascontiguousarray(weights, dtype=np.float32)
    e, out_f, n = w.shape
    xs = np.ascontiguousarray(x, dtype=np.float64).reshape(-1, n)
    sel = np.ascontiguousarray(sel, dtype=np.int32).reshape(-1)
    tok = np.ascontiguousarray(tok, dtype=np.int32).reshape(-1)
    y = np.empty((sel.size, out_f), dtype=np.float64)
    lib.orc_gemv_f64(_ptr(w), _ptr(xs), _ptr(sel), _ptr(tok), sel.size, out_f, n, _ptr(y))
    return y


# ---------------------------------------------------------------- generators


def finite_half(rng: np.random.Generator, size) -> np.ndarray:
    """Random finite fp16 values over the whole sign/exponent space."""
    bits = rng.integers(0, 1 << 16, size=size, dtype=np.uint32).astype(np.uint16)
    bits = np.where((bits & 0x7C00) == 0x7C00, bits & 0xBFFF, bits).astype(np.uint16)
    return bits.view(np.float16)


def serving_half(rng: np.random.Generator, size) -> np.ndarray:
    """fp16 scales at converted-expert magnitudes, |d| in [2e-5, 8.2e-4]."""
    mag = 2e-5 + 8e-4 * rng.random(size)
    sign = np.where(rng.random(size) < 0.5, -1.0, 1.0)
    return (mag * sign).astype(np.float16)


def random_wire(member: str, rows: int, n: int, seed: int,
                scales: str = "sweep") -> np.ndarray:
    """Uniform random wire bytes with drawn fp16 scales (every field is dense)."""
    rng = np.random.default_rng(seed)
    draw = finite_half if scales == "sweep" else serving_half
    rb = ik_row_bytes(member, n)
    w = rng.integers(0, 256, size=(rows, rb), dtype=np.uint16).astype(np.uint8)
    if member == "iq1_s_r4":
        assert rows % 4 == 0
        g = w.reshape(rows // 4, 4 * rb)
        g[:, :8] = draw(rng, (rows // 4, 4)).view(np.uint8).reshape(rows // 4, 8)
    elif member == "iq2_ks":
        w[:, :2] = draw(rng, rows).view(np.uint8).reshape(rows, 2)
    else:
        b = w.reshape(rows, n // QK_K, 76)
        b[:, :, :2] = draw(rng, (rows, n // QK_K)).view(np.uint8).reshape(rows, -1, 2)
    return w


def random_streams(member: str, rows: int, n: int, seed: int,
                   scales: str = "serving") -> dict[str, np.ndarray]:
    """Random relayout streams (same distribution as ``pack(random_wire)``)."""
    return pack(member, random_wire(member, rows, n, seed, scales), n)


def exhaustive_streams(member: str, seed: int = 0) -> dict[str, np.ndarray]:
    """Relayout rows of width 256 covering the member's whole decode value space.

    2-bit members: every (scale index, alphabet, code) triple at every weight
    position (4 code rotations per (index, alphabet)). IQ1_S_R4: every grid
    index at every sub-group slot, for every block scale and shift sign.
    Built directly in stream form; the fp16 scales sweep the finite space.
    """
    rng = np.random.default_rng(seed)
    n = 256
    k = np.arange(n)
    if member in ("iq2_ks", "iq2_k"):
        nidx, sub = (32, 32) if member == "iq2_ks" else (16, 16)
        rows = []
        for idx in range(nidx):
            for alpha in range(2):
                for rot in range(4):
                    rows.append((idx, alpha, (k + rot) % 4))
        r = len(rows)
        codes = np.stack([c for _, _, c in rows]).astype(np.uint8)
        idx = np.array([i for i, _, _ in rows], dtype=np.uint8)
        alpha = np.array([a for _, a, _ in rows], dtype=np.uint8)
        ngrp = n // sub
        lo = np.repeat((idx & 15)[:, None], ngrp, axis=1)
        scl = (lo[:, 0::2] | (lo[:, 1::2] << 4)).astype(np.uint8)
        bits_alpha = np.packbits(np.repeat(alpha[:, None], ngrp, axis=1), axis=1,
                                 bitorder="little")
        out = {"qs": _codes_to_words(codes), "scl": scl}
        if member == "iq2_ks":
            hi = np.repeat((idx >> 4)[:, None], ngrp, axis=1)
            out["sch"] = np.packbits(hi, axis=1, bitorder="little")
            out["sex"] = bits_alpha
            out["dv"] = finite_half(rng, (r, 1))
        else:
            out["sex"] = bits_alpha
            out["dv"] = finite_half(rng, (r, 1))
        return out
    # iq1_s_r4: 2048 indices tile 64 rows x 32 sub-groups; 4 rotations move
    # each index through the 4 slots of a block; x 8 scales x 2 signs.
    base = np.arange(2048).reshape(64, 32)
    qs_rows, qh_rows = [], []
    for ls in range(8):
        for neg in range(2):
            for rot in range(4):
                ind = np.roll(base, rot, axis=1).reshape(64, 8, 4)
                low = (ind & 255).astype(np.uint32)
                qs = low[:, :, 0] | (low[:, :, 1] << 8) | (low[:, :, 2] << 16) | (low[:, :, 3] << 24)
                hi = (ind >> 8).astype(np.uint32)
                qh = hi[:, :, 0] | (hi[:, :, 1] << 3) | (hi[:, :, 2] << 6) | (hi[:, :, 3] << 9)
                qh = qh | (ls << 12) | (neg << 15)
                qs_rows.append(qs)
                qh_rows.append(qh.astype(np.uint16))
    qs = np.concatenate(qs_rows).astype(np.uint32)
    qh = np.concatenate(qh_rows).astype(np.uint16)
    return {"qs": qs, "qh": qh, "dv": finite_half(rng, (qs.shape[0], 1))}


# ------------------------------------------------------------- libraries

_PORT = None
_REF = {}


def _ptr(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def load_port():
    """The C restatement (``oracle/_build/libiqk_oracle.so``), built on demand."""
    global _PORT
    if _PORT is not None:
        return _PORT
    lib_path = HERE / "_build" / "libiqk_oracle.so"
    src = HERE / "iqk_oracle.c"
    if not lib_path.exists() or lib_path.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE), "port"], check=True)
    lib = ctypes.CDLL(str(lib_path))
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    for name in ("orc_decode_iq2_ks",):
        getattr(lib, name).argtypes = [vp] * 5 + [i64, i64, vp]
    lib.orc_decode_iq2_k.argtypes = [vp] * 4 + [i64, i64, vp]
    lib.orc_decode_iq1_s_r4.argtypes = [vp] * 3 + [i64, i64, vp]
    for m in MEMBERS:
        getattr(lib, f"orc_dequant_{m}").argtypes = [vp, i64, i64, vp]
    lib.orc_gemv_f64.argtypes = [vp] * 4 + [i64, i64, i64, vp]
    lib.orc_half_to_float.argtypes = [ctypes.c_uint16]
    lib.orc_half_to_float.restype = ctypes.c_float
    for fn in lib.orc_decode_iq2_ks, lib.orc_decode_iq2_k, lib.orc_decode_iq1_s_r4:
        fn.restype = None
    _PORT = lib
    return lib


def ref_available() -> bool:
    d = HERE / "_ref"
    return (d / "libiqk_iq2.so").exists() and (d / "libiqk_iq1sr4.so").exists()


def load_ref(member: str):
    """The reference's own vendored codec, compiled by ``oracle/Makefile``."""
    lib_name = "libiqk_iq1sr4.so" if member == "iq1_s_r4" else "libiqk_iq2.so"
    if lib_name in _REF:
        return _REF[lib_name]
    path = HERE / "_ref" / lib_name
    if not path.exists():
        raise FileNotFoundError(f"{path} not built (make -C oracle ref IQK_REF=<checkout>)")
    lib = ctypes.CDLL(str(path))
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    members = ("iq1_s_r4",) if member == "iq1_s_r4" else ("iq2_k", "iq2_ks")
    for m in members:
        q = getattr(lib, f"iqk_quantize_{m}")
        q.argtypes = [vp, vp, i64, i64, vp]
        q.restype = ctypes.c_size_t
        d = getattr(lib, f"iqk_dequantize_{m}")
        d.argtypes = [vp, vp, i64, i64]
        d.restype = ctypes.c_int
    _REF[lib_name] = lib
    return lib


def ref_quantize(member: str, weights: np.ndarray, imatrix: np.ndarray | None) -> np.ndarray:
    """``codec.quantize`` through the reference's own compiled quantizer."""
    lib = load_ref(member)
    w = np.ascontiguousarray(weights, dtype=np.float32)
    rows, n = w.shape
    out = np.zeros((rows, ik_row_bytes(member, n)), dtype=np.uint8)
    im = None if imatrix is None else np.ascontiguousarray(imatrix, dtype=np.float32)
    wrote = getattr(lib, f"iqk_quantize_{member}")(
        _ptr(w), _ptr(out), rows, n, None if im is None else _ptr(im))
    assert wrote == out.size, (wrote, out.size)
    return out


def ref_dequantize(member: str, wire: np.ndarray, n: int) -> np.ndarray:
    """``codec.dequantize`` through the reference's own compiled dequantizer."""
    lib = load_ref(member)
    w = np.ascontiguousarray(wire, dtype=np.uint8)
    out = np.zeros((w.shape[0], n), dtype=np.float32)
    rc = getattr(lib, f"iqk_dequantize_{member}")(_ptr(w), _ptr(out), w.shape[0], n)
    assert rc == 0
    return out


def cpu_count() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
