"""Stream geometry of the package against the reference's (golden fixture)
and the ggml row-size facts (the reference's tests/test_format.py:31-152)."""

from __future__ import annotations

import pytest

from mlx_iqk_b200 import format as fmt

ROW_SIZE_FACTS = {"iq2_ks": (2, 70, 256), "iq2_k": (0, 76, 256), "iq1_s_r4": (2, 6, 32)}


@pytest.mark.parametrize("member", fmt.MEMBERS)
@pytest.mark.parametrize("n", (256, 2048, 4096))
def test_geometry_matches_the_reference(golden, member, n):
    assert fmt.ik_row_bytes(member, n) == int(golden[f"row_bytes/{member}/{n}"])
    for name, shape in fmt.component_shapes(member, 3, 32, n).items():
        assert tuple(golden[f"shape/{member}/{n}/{name}"]) == shape


@pytest.mark.parametrize("member", fmt.MEMBERS)
@pytest.mark.parametrize("n", (256, 1024, 2048, 4096, 8192))
def test_row_bytes_from_independent_struct_facts(member, n):
    meta, block, weights = ROW_SIZE_FACTS[member]
    assert fmt.ik_row_bytes(member, n) == meta + block * (n // weights)
    assert fmt.relayout_row_bytes(member, n) == fmt.ik_row_bytes(member, n)


def test_bits_per_weight():
    assert fmt.bits_per_weight("iq2_k", 4096) == 2.375
    assert fmt.bits_per_weight("iq2_ks", 4096) == 2.1875 + 16 / 4096
    assert fmt.bits_per_weight("iq1_s_r4", 2048) == 1.5 + 16 / 2048


@pytest.mark.parametrize("bad", [0, -256, 255, 300, 4095])
def test_row_width_guard(bad):
    with pytest.raises(fmt.IqkFormatError):
        fmt.check_row_width(bad)


def test_iq1_width_and_group_rules():
    assert fmt.check_row_width(96, "iq1_s_r4") == 96
    for bad in (0, -32, 31, 100):
        with pytest.raises(fmt.IqkFormatError):
            fmt.check_row_width(bad, "iq1_s_r4")
    assert fmt.check_wire_rows("iq1_s_r4", 8) == 8
    for bad in (0, -4, 2, 6, 37):
        with pytest.raises(fmt.IqkFormatError):
            fmt.check_wire_rows("iq1_s_r4", bad)
    with pytest.raises(fmt.IqkFormatError):
        fmt.check_member("iq3_k")
