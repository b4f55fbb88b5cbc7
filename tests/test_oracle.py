"""The CPU oracle is pinned to the reference's own outputs (golden vectors).

Every expected value in ``tests/golden/golden.npz`` was produced by the
reference itself (``tests/golden/make_golden.py``: ``format.pack`` and the
vendored ik_llama ``codec.dequantize`` / ``codec.quantize``). These tests
check the oracle -- numpy relayout + C decode in ``oracle/`` -- against those
vectors bit for bit, the same gates the reference runs on its own decode
(``tests/test_format.py:168-296`` of the reference).
"""

from __future__ import annotations

import hashlib
import re
from pathlib import Path

import numpy as np
import pytest

import oracle

REPO = Path(__file__).resolve().parents[1]
MEMBERS = oracle.MEMBERS


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def digest(a):
    return hashlib.sha256(np.ascontiguousarray(a, dtype=np.float32).tobytes()).hexdigest()


def header_codes(path: Path) -> np.ndarray:
    text = path.read_text()
    return np.array([int(v, 16) for v in re.findall(r"0x[0-9a-fA-F]{4}", text)], dtype=np.uint16)


def test_grid_tables_match_the_reference(golden):
    want = golden["iq1s_grid_codes"]
    assert np.array_equal(header_codes(REPO / "oracle" / "iq1s_grid.h"), want)
    assert np.array_equal(header_codes(REPO / "mlx_iqk_b200" / "csrc" / "iq1s_grid.h"), want)
    from mlx_iqk_b200.tables import grid_values
    assert np.array_equal(grid_values(), golden["iq1s_grid_values"])
    assert np.array_equal(oracle.IQ2NL_VALUES, golden["iq2nl_values"])


@pytest.mark.parametrize("member", MEMBERS)
@pytest.mark.parametrize("n", (256, 2048, 4096))
def test_random_wire_relayout_and_decode(golden, member, n):
    key = f"random/{member}/{n}"
    wire = golden[key + "/wire"]
    streams = oracle.pack(member, wire, n)
    for name, value in streams.items():
        want = golden[key + "/stream/" + name]
        assert np.array_equal(np.ascontiguousarray(value).view(np.uint8).ravel(),
                              np.ascontiguousarray(want).view(np.uint8).ravel()), name
    assert np.array_equal(bits(oracle.decode(member, streams, n)), golden[key + "/want"])
    assert np.array_equal(bits(oracle.dequant_wire(member, wire, n)), golden[key + "/want"])
    assert np.array_equal(oracle.unpack(member, streams, n), wire)


@pytest.mark.parametrize("member", MEMBERS)
@pytest.mark.parametrize("n", (2048, 4096))
@pytest.mark.parametrize("tag", ("im", "noim"))
def test_quantized_rows_decode_bit_identically(golden, member, n, tag):
    key = f"quant/{member}/{n}/{tag}"
    wire = golden[key + "/wire"]
    streams = oracle.pack(member, wire, n)
    assert np.array_equal(bits(oracle.decode(member, streams, n)), golden[key + "/want"])
    assert np.array_equal(oracle.unpack(member, streams, n), wire)


@pytest.mark.parametrize("member", MEMBERS)
def test_exhaustive_value_space_is_bit_identical(golden, member):
    wire = golden[f"exhaustive/{member}/wire"]
    got = oracle.decode(member, oracle.pack(member, wire, 256), 256)
    assert digest(got) == str(golden[f"exhaustive/{member}/sha256"])


@pytest.mark.parametrize("member", MEMBERS)
def test_own_exhaustive_generator_covers_the_value_space(member):
    """The oracle's own generator: stream decode == wire dequant of its unpack."""
    streams = oracle.exhaustive_streams(member, seed=5)
    wire = oracle.unpack(member, streams, 256)
    a = oracle.decode(member, streams, 256)
    b = oracle.dequant_wire(member, wire, 256)
    assert np.array_equal(bits(a), bits(b))
    assert np.array_equal(oracle.unpack(member, oracle.pack(member, wire, 256), 256), wire)


def test_config1_head_matches(golden):
    wire = golden["config1/wire_head"]
    streams = oracle.pack("iq2_ks", wire, 4096)
    w = oracle.decode("iq2_ks", streams, 4096)
    assert np.array_equal(bits(w), golden["config1/want_head"])
    x = golden["config1/x"]
    y = oracle.gemv_f64(w[None], x[None].astype(np.float64), np.zeros(1, np.int32),
                        np.zeros(1, np.int32))[0]
    assert np.allclose(y, golden["config1/y_head_f64"], rtol=1e-12, atol=0)


@pytest.mark.skipif(not oracle.ref_available(), reason="reference codec not built")
def test_config1_full_tensor_regenerates(golden):
    """The full config-1 expert (2048 rows) re-quantized by the reference's codec."""
    rng = np.random.default_rng(oracle.seed_for("config1", "iq2_ks"))
    rows = (rng.standard_normal((2048, 4096)) * 0.02).astype(np.float32)
    imatrix = rng.uniform(0.1, 1.0, 4096).astype(np.float32)
    wire = oracle.ref_quantize("iq2_ks", rows, imatrix)
    assert hashlib.sha256(wire.tobytes()).hexdigest() == str(golden["config1/wire_sha256"])
    got = oracle.decode("iq2_ks", oracle.pack("iq2_ks", wire, 4096), 4096)
    assert digest(got) == str(golden["config1/want_sha256"])


@pytest.mark.skipif(not oracle.ref_available(), reason="reference codec not built")
@pytest.mark.parametrize("member", MEMBERS)
def test_c_restatement_matches_the_reference_codec(member):
    rng = np.random.default_rng(11)
    rows = (rng.standard_normal((8, 2048)) * 0.03).astype(np.float32)
    wire = oracle.ref_quantize(member, rows, rng.uniform(0.1, 1, 2048).astype(np.float32))
    assert np.array_equal(bits(oracle.ref_dequantize(member, wire, 2048)),
                          bits(oracle.dequant_wire(member, wire, 2048)))
    rw = oracle.random_wire(member, 16, 4096, seed=3)
    assert np.array_equal(bits(oracle.ref_dequantize(member, rw, 4096)),
                          bits(oracle.decode(member, oracle.pack(member, rw, 4096), 4096)))


def test_a_planted_mistake_is_caught():
    """Flip one code bit in the oracle's input: the decode must change."""
    streams = oracle.random_streams("iq2_ks", 4, 2048, seed=1)
    a = oracle.decode("iq2_ks", streams, 2048)
    bad = {k: v.copy() for k, v in streams.items()}
    bad["qs"][2, 7] ^= np.uint32(1)
    b = oracle.decode("iq2_ks", bad, 2048)
    assert (bits(a) != bits(b)).sum() == 1
