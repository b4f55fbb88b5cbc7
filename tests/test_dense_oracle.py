"""The dense-member oracle (IQ4_KS, IQ4_K, IQ5_K, IQ6_K) against the reference.

Everything here runs on CPU. The golden file holds the reference's own
outputs on the same wire bytes (``tests/golden/make_golden_dense.py``):
``format.pack`` for the streams and ``format.decode_wire`` for the float32
weights, over a random serving-scale case, the full fp16 scale sweep, the
reference's exhaustive enumeration of every code / scale / alphabet value,
and rows its codec quantized. The oracle must reproduce all of it bit for
bit before it may judge a kernel.
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest

import dense_oracle as D
import dense_tables

GOLDEN = Path(__file__).resolve().parent / "golden" / "golden_dense.npz"


@pytest.fixture(scope="module")
def gd():
    data = np.load(GOLDEN)
    return {k: data[k] for k in data.files}


def test_tables_are_the_reference_constants(gd):
    assert np.array_equal(dense_tables.IQ4K_VALUES, gd["values/iq4k"])
    assert np.array_equal(dense_tables.IQ5NL_VALUES, gd["values/iq5nl"])
    assert np.array_equal(dense_tables.IQ6K_BITS, gd["values/iq6k_bits"])


@pytest.mark.parametrize("member", D.DENSE_MEMBERS)
def test_row_bytes(member, gd):
    for n in (256, 1024, 2048, 4096, 8192):
        assert D.ik_row_bytes(member, n) == int(gd[f"row_bytes/{member}/{n}"])


@pytest.mark.parametrize("member", D.DENSE_MEMBERS)
def test_stream_shapes_and_dtypes(member, gd):
    for name, (per_row, dt) in D.stream_specs(member, 2048).items():
        shape = tuple(int(v) for v in gd[f"shape/{member}/2048/{name}"])
        assert shape in ((32, per_row), (32,)), (name, shape)
        assert str(dt) == str(gd[f"dtype/{member}/{name}"]), name


@pytest.mark.parametrize("member", D.DENSE_MEMBERS)
def test_pack_equals_the_reference_relayout(member, gd):
    key = f"random/{member}/1024"
    got = D.pack(member, gd[key + "/wire"], 1024)
    names = sorted(k.rsplit("/", 1)[1] for k in gd if k.startswith(key + "/stream/"))
    assert sorted(got) == names
    for name in names:
        want = gd[f"{key}/stream/{name}"]
        assert got[name].dtype == want.dtype and got[name].shape == want.shape, name
        assert np.array_equal(got[name].view(np.uint8), want.view(np.uint8)), name


@pytest.mark.parametrize("member", D.DENSE_MEMBERS)
@pytest.mark.parametrize("case,n", [("random", 1024), ("sweep", 256), ("converted", 2048)])
def test_decode_is_bit_identical(member, case, n, gd):
    key = f"{case}/{member}/{n}"
    got = D.dequant_wire(member, gd[key + "/wire"], n).view(np.uint32)
    assert np.array_equal(got, gd[key + "/want"])


@pytest.mark.parametrize("member", D.DENSE_MEMBERS)
def test_decode_covers_the_exhaustive_enumeration(member, gd):
    got = D.dequant_wire(member, gd[f"exhaustive/{member}/wire"], 256)
    digest = hashlib.sha256(np.ascontiguousarray(got, dtype=np.float32).tobytes()).hexdigest()
    assert digest == str(gd[f"exhaustive/{member}/want_sha256"])


@pytest.mark.parametrize("member", ("iq4_ks", "iq4_k", "iq5_k"))
def test_integer_members_agree_with_ik_on_this_host(member, gd):
    """ik's own CPU dequantizer (compiled for x86 here) gives the same bits
    for the integer-alphabet members."""
    key = f"random/{member}/1024"
    assert np.array_equal(gd[key + "/want"], gd[key + "/ik"])


def test_iq6_k_serves_the_table_not_this_hosts_cubic(gd):
    """IQ6_K's serving decode reads the table of ik's cubic outputs; ik's
    x86 build evaluates the cubic differently (the reference records the
    same host dependence), so the golden want is the table decode."""
    key = "random/iq6_k/1024"
    assert not np.array_equal(gd[key + "/want"], gd[key + "/ik"])
    got = D.dequant_wire("iq6_k", gd[key + "/wire"], 1024).view(np.uint32)
    assert np.array_equal(got, gd[key + "/want"])


@pytest.mark.parametrize("member", D.DENSE_MEMBERS)
def test_own_generator_is_valid_wire(member):
    wire = D.random_wire(member, 4, 2048, seed=D.QK_K)
    w = D.dequant_wire(member, wire, 2048)
    assert w.shape == (4, 2048) and np.isfinite(w).all() and np.abs(w).max() > 0
