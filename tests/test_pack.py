"""On-device relayout (iqk_pack) against the reference's own format.pack.

The golden file holds format.pack outputs the reference produced for seeded
wire of every member and width (tests/golden/make_golden.py); the kernel
must reproduce them bit for bit, and a module loaded from wire on the device
must equal one loaded from the host relayout, for random byte space,
reference-quantized rows and the exhaustive decode value space.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from helpers import stacked
from mlx_iqk_b200 import IqkSwitchLinear

pytestmark = pytest.mark.gpu

MEMBERS = oracle.MEMBERS


def _bytes(t) -> np.ndarray:
    a = t.detach().cpu().contiguous() if isinstance(t, torch.Tensor) else np.ascontiguousarray(t)
    if isinstance(a, torch.Tensor):
        a = a.view(torch.uint8).numpy() if a.dtype != torch.uint16 else \
            a.view(torch.int16).numpy().view(np.uint8)
    return np.ascontiguousarray(a).view(np.uint8).ravel()


def _from_wire(member, wire, n, experts, out, cuda):
    mod = IqkSwitchLinear(member, experts, out, n, device=cuda)
    mod.load_wire(torch.from_numpy(np.ascontiguousarray(wire)).to(cuda))
    return mod


@pytest.mark.parametrize("member", MEMBERS)
@pytest.mark.parametrize("n", (2048, 4096))
def test_pack_matches_the_reference_relayout(cuda, golden, member, n):
    key = f"random/{member}/{n}"
    wire = np.concatenate([golden[key + "/wire"]] * 2)  # 8 rows the reference packed, twice
    mod = _from_wire(member, wire, n, 1, wire.shape[0], cuda)
    for name in mod.stream_names():
        want = np.ascontiguousarray(golden[key + "/stream/" + name])
        want = np.concatenate([want.reshape(8, -1)] * 2)
        assert np.array_equal(_bytes(getattr(mod, name)), _bytes(want)), (member, n, name)


@pytest.mark.parametrize("member", MEMBERS)
@pytest.mark.parametrize("n", (2048, 4096))
@pytest.mark.parametrize("scales", ("serving", "sweep"))
def test_device_pack_equals_host_pack(cuda, member, n, scales):
    experts, out = 4, 64
    wire = oracle.random_wire(member, experts * out, n, seed=oracle.seed_for(member, n, "pk"),
                              scales=scales)
    mod = _from_wire(member, wire, n, experts, out, cuda)
    host = stacked(member, oracle.pack(member, wire, n), experts, out, n)
    for name in mod.stream_names():
        assert np.array_equal(_bytes(getattr(mod, name)), _bytes(host[name])), name
    ref = IqkSwitchLinear(member, experts, out, n, device=cuda)
    ref.load_streams(host)
    a = mod.dequantized(torch.float32).view(torch.int32)
    assert torch.equal(a, ref.dequantized(torch.float32).view(torch.int32))


@pytest.mark.parametrize("member", MEMBERS)
def test_pack_of_quantized_and_exhaustive_rows(cuda, golden, member):
    wire = np.concatenate([golden[f"quant/{member}/4096/im/wire"]] * 4)  # 32 rows
    mod = _from_wire(member, wire, 4096, 1, 32, cuda)
    host = oracle.pack(member, wire, 4096)
    for name in mod.stream_names():
        assert np.array_equal(_bytes(getattr(mod, name)), _bytes(host[name])), name
    ex = golden[f"exhaustive/{member}/wire"]  # 256-wide rows: the whole value space
    rows = ex.shape[0] - ex.shape[0] % 16
    # the module is sized for 2048 / 4096: pack the exhaustive rows through the
    # entry point directly at width 256
    from mlx_iqk_b200 import kernels as K
    specs = oracle.stream_specs(member, 256)
    outs = [torch.empty(rows * specs[k][0], dtype={1: torch.uint8, 2: torch.int16,
                                                   4: torch.int32}[np.dtype(specs[k][1]).itemsize],
                        device=cuda) for k in specs]
    K.pack(member, torch.from_numpy(np.ascontiguousarray(ex[:rows])).to(cuda), 256, outs)
    host = oracle.pack(member, ex[:rows], 256)
    for t, k in zip(outs, specs):
        assert np.array_equal(_bytes(t), _bytes(host[k])), k


def test_pack_rejects_a_bad_wire(cuda):
    from mlx_iqk_b200.nn import IqkRuntimeError
    mod = IqkSwitchLinear("iq2_ks", 2, 32, 2048, device=cuda)
    with pytest.raises(IqkRuntimeError):
        mod.load_wire(torch.zeros(100, dtype=torch.uint8))
