"""Generate the golden vectors the oracle is pinned against, from the reference.

Runs in the build container only (the reference checkout and its compiled
codec exist there; ``make -C oracle ref IQK_REF=<checkout>`` builds the codec). Writes
``tests/golden/golden.npz``; the tests read that file and never the reference.

Every expected output comes from the reference's own code on the same bytes:

* ``format.pack``       (src/mlx_iqk/format.py:664-678) for the relayout,
* ``codec.dequantize``  (src/mlx_iqk/codec.py:272-293 -> the vendored
  ik_llama CPU dequantizers) for the float32 weights,
* ``codec.quantize``    (src/mlx_iqk/codec.py:238-269) for converted rows,
* ``wirepack.random_wire`` / ``exhaustive_*`` (tests/wirepack.py:97-194,
  385-426) for the wire bytes, so the fixtures cover the same value space the
  reference's own gates cover (tests/test_format.py:168-217, 266-280).

Large outputs are stored as SHA-256 digests of their float32 bytes.

    python tests/golden/make_golden.py
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np

import refshim

HERE = Path(__file__).resolve().parent
MEMBERS = ("iq2_ks", "iq2_k", "iq1_s_r4")


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a, dtype=np.float32).tobytes()).hexdigest()


def main() -> None:
    iq1grid, fmt, codec, wirepack = refshim.load()
    out: dict[str, np.ndarray] = {
        "iq1s_grid_codes": np.asarray(iq1grid.grid_codes(), dtype=np.uint16),
        "iq1s_grid_values": np.asarray(iq1grid.grid_values(), dtype=np.int8),
        "iq2nl_values": np.asarray(fmt.IQ2NL_VALUES, dtype=np.int8),
    }
    meta = []
    for member in MEMBERS:
        for n in (256, 2048, 4096):
            out[f"row_bytes/{member}/{n}"] = np.array(fmt.ik_row_bytes(member, n))
            shapes = fmt.component_shapes(member, 3, 32, n)
            for name, shape in shapes.items():
                out[f"shape/{member}/{n}/{name}"] = np.array(shape)
            # Random byte space, full fp16 scale sweep (test_format.py:194-200).
            wire = wirepack.random_wire(member, 8, n, seed=wirepack.seed_for(member, n))
            key = f"random/{member}/{n}"
            out[key + "/wire"] = wire
            out[key + "/want"] = codec.dequantize(member, wire, n).view(np.uint32)
            for name, value in fmt.pack(member, wire, n).items():
                out[key + "/stream/" + name] = np.ascontiguousarray(value)
            meta.append(key)
        for n in (2048, 4096):
            # Converted rows, with and without an imatrix; includes a zero row
            # and a 1e-4-scaled row (test_format.py:203-217).
            rng = np.random.default_rng(wirepack.seed_for("golden-quant", member, n))
            rows = (rng.standard_normal((8, n)) * 0.02).astype(np.float32)
            rows[3] = 0.0
            rows[5] *= 1e-4
            imatrix = rng.uniform(0.1, 1.0, n).astype(np.float32)
            for tag, im in (("im", imatrix), ("noim", None)):
                wire = codec.quantize(member, rows, im)
                key = f"quant/{member}/{n}/{tag}"
                out[key + "/rows"] = rows
                if im is not None:
                    out[key + "/imatrix"] = im
                out[key + "/wire"] = wire
                out[key + "/want"] = codec.dequantize(member, wire, n).view(np.uint32)
                meta.append(key)
    # Whole decode value space (test_format.py:168-191, 266-280).
    for member, fn in (("iq2_k", wirepack.exhaustive_iq2_k),
                       ("iq2_ks", wirepack.exhaustive_iq2_ks),
                       ("iq1_s_r4", wirepack.exhaustive_iq1_s_r4)):
        wire = fn(seed={"iq2_k": 1, "iq2_ks": 2, "iq1_s_r4": 3}[member])
        want = codec.dequantize(member, wire, 256)
        out[f"exhaustive/{member}/wire"] = wire
        out[f"exhaustive/{member}/sha256"] = np.array(digest(want))
    # config 1: one IQ2_KS expert [2048, 4096], N(0, 0.02^2) rows,
    # U(0.1, 1) imatrix, codec-quantized. The first 64 rows are stored; the
    # whole tensor is pinned by digest (regenerated where the codec is built).
    rng = np.random.default_rng(wirepack.seed_for("config1", "iq2_ks"))
    rows = (rng.standard_normal((2048, 4096)) * 0.02).astype(np.float32)
    imatrix = rng.uniform(0.1, 1.0, 4096).astype(np.float32)
    x = rng.standard_normal(4096).astype(np.float32)
    wire = codec.quantize("iq2_ks", rows, imatrix)
    want = codec.dequantize("iq2_ks", wire, 4096)
    out["config1/wire_head"] = wire[:64]
    out["config1/want_head"] = want[:64].view(np.uint32)
    out["config1/x"] = x
    out["config1/wire_sha256"] = np.array(hashlib.sha256(wire.tobytes()).hexdigest())
    out["config1/want_sha256"] = np.array(digest(want))
    out["config1/y_head_f64"] = want[:64].astype(np.float64) @ x.astype(np.float64)
    out["index"] = np.array(meta)
    np.savez_compressed(HERE / "golden.npz", **out)


if __name__ == "__main__":
    main()
