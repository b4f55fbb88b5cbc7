"""Golden vectors for the dense members (IQ4_KS, IQ4_K, IQ5_K, IQ6_K), from the reference.

Runs in the build container only, like ``make_golden.py``: the reference
checkout and its compiled codec (``make -C oracle ref IQK_REF=<checkout>``)
exist there. Writes ``tests/golden/golden_dense.npz``; the tests read that file
and never the reference.

Every expected output comes from the reference's own code on the same bytes:

* ``format.pack``        (src/mlx_iqk/format.py:664-678, dense rows at
  1021-1084) for the relayout streams,
* ``format.decode_wire`` (src/mlx_iqk/format.py:880-882 -> the dense decode
  at 1166-1240) for the float32 weights the serving kernels must reproduce,
* ``codec.dequantize``   (src/mlx_iqk/codec.py:272-293 -> the vendored
  ik_llama ``iqk_dense.cpp``) for ik's own CPU output on this host,
* ``codec.quantize``     (src/mlx_iqk/codec.py:238-269) for converted rows,
* ``wirepack.random_wire`` / ``exhaustive_*`` (tests/wirepack.py:303-426)
  for the wire bytes (the value space the reference's own gates cover,
  tests/test_dense_format.py).

The format constants (``IQ4K_VALUES``, ``IQ5NL_VALUES``, ``IQ6NL_VALUES`` and
the bit patterns of ``IQ6K_TABLE``, src/mlx_iqk/format.py:155-213) are
stored too, so the repo's own copies are pinned to them.

    python tests/golden/make_golden_dense.py
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np

import refshim

HERE = Path(__file__).resolve().parent
MEMBERS = ("iq4_ks", "iq4_k", "iq5_k", "iq6_k")


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a, dtype=np.float32).tobytes()).hexdigest()


def main() -> None:
    _, fmt, codec, wirepack = refshim.load()
    out: dict[str, np.ndarray] = {
        "values/iq4k": np.asarray(fmt.IQ4K_VALUES, dtype=np.int8),
        "values/iq5nl": np.asarray(fmt.IQ5NL_VALUES, dtype=np.int8),
        "values/iq6nl": np.asarray(fmt.IQ6NL_VALUES, dtype=np.int8),
        "values/iq6k_bits": np.asarray(fmt.IQ6K_TABLE, dtype=np.float32).view(np.uint32),
    }
    digests = []
    for member in MEMBERS:
        for n in (256, 1024, 2048, 4096, 8192):
            out[f"row_bytes/{member}/{n}"] = np.array(fmt.ik_row_bytes(member, n))
        for name, shape in fmt.dense_component_shapes(member, 32, 2048).items():
            out[f"shape/{member}/2048/{name}"] = np.array(shape)
            out[f"dtype/{member}/{name}"] = np.array(str(fmt.dense_component_dtypes(member)[name]))
        # serving-magnitude scales, the kernels' test case (8 rows, n = 1024)
        wire = wirepack.random_wire(member, 8, 1024, seed=wirepack.seed_for("dense", member),
                                    scales="serving")
        key = f"random/{member}/1024"
        out[key + "/wire"] = wire
        out[key + "/want"] = fmt.decode_wire(member, wire, 1024).astype(np.float32).view(np.uint32)
        out[key + "/ik"] = codec.dequantize(member, wire, 1024).astype(np.float32).view(np.uint32)
        for name, value in fmt.pack(member, wire, 1024).items():
            out[key + "/stream/" + name] = np.ascontiguousarray(value)
        # the full fp16 scale sweep at one super-block per row
        wire = wirepack.random_wire(member, 16, 256, seed=wirepack.seed_for("sweep", member),
                                    scales="sweep")
        key = f"sweep/{member}/256"
        out[key + "/wire"] = wire
        out[key + "/want"] = fmt.decode_wire(member, wire, 256).astype(np.float32).view(np.uint32)
        # the reference's enumeration of every code, scale and alphabet value
        wire = getattr(wirepack, f"exhaustive_{member}")()
        key = f"exhaustive/{member}"
        out[key + "/wire"] = wire
        want = fmt.decode_wire(member, wire, 256)
        out[key + "/want_sha256"] = np.array(digest(want))
        digests.append(key)
        # converted rows: the reference codec quantizing Gaussian rows
        rng = np.random.default_rng(4242)
        rows = (rng.standard_normal((8, 2048)) * 0.05).astype(np.float32)
        imatrix = rng.random(2048).astype(np.float32)
        wire = codec.quantize(member, rows, imatrix)
        key = f"converted/{member}/2048"
        out[key + "/wire"] = wire
        out[key + "/want"] = fmt.decode_wire(member, wire, 2048).astype(np.float32).view(np.uint32)
    np.savez_compressed(HERE / "golden_dense.npz", **out)
    print(f"wrote {len(out)} arrays to {HERE / 'golden_dense.npz'}")


if __name__ == "__main__":
    main()
