"""Format-constant tables shared by the Python layer and the CUDA library.

The IQ1_S grid codes live in one place, ``csrc/iq1s_grid.h``, which the CUDA
sources compile in; this module parses the same header so the host-side
table (``nn.grid_table``) cannot drift from the device one.
"""

from __future__ import annotations

import re
from functools import lru_cache
from pathlib import Path

import numpy as np

_HEADER = Path(__file__).resolve().parent / "csrc" / "iq1s_grid.h"


@lru_cache(maxsize=1)
def grid_codes() -> np.ndarray:
    """The 2048 packed IQ1_S grid codes, ``uint16`` (8 positions x 2 bits)."""
    text = _HEADER.read_text()
    body = text.split("#define IQK_IQ1S_GRID_CODES", 1)[1]
    codes = np.array([int(v, 16) for v in re.findall(r"0x[0-9a-fA-F]{4}", body)],
                     dtype=np.uint16)
    if codes.shape != (2048,):
        raise RuntimeError(f"{_HEADER} holds {codes.shape[0]} grid codes, expected 2048")
    return codes


def grid_values() -> np.ndarray:
    """The grid as ``int8 [2048, 8]`` values in {-1, 0, +1}."""
    codes = grid_codes().astype(np.int64)[:, None]
    return (((codes >> (2 * np.arange(8))[None, :]) & 3) - 1).astype(np.int8)


_DENSE_HEADER = Path(__file__).resolve().parent / "csrc" / "iqk_dense_tables.h"


@lru_cache(maxsize=None)
def _dense_macro(macro: str) -> tuple[int, ...]:
    text = _DENSE_HEADER.read_text()
    body = text.split(f"#define {macro} ", 1)[1].split("\n\n", 1)[0]
    return tuple(int(v, 0) for v in re.findall(r"-?0x[0-9a-fA-F]+|-?\d+", body.replace("u,", ",").replace("u ", " ")))


def dense_values(member: str) -> np.ndarray:
    """A dense member's value table, both alphabets back to back, as the CUDA
    library compiles it in (``csrc/iqk_dense_tables.h``): int8 for the integer
    alphabets (IQ4_KS / IQ4_K share one; IQ5_K), float32 for IQ6_K (the
    outputs of ik's cubic reconstruction)."""
    if member in ("iq4_ks", "iq4_k"):
        v = np.array(_dense_macro("IQK_IQ4K_VALUES"), dtype=np.int8)
        assert v.shape == (32,)
        return v
    if member == "iq5_k":
        v = np.array(_dense_macro("IQK_IQ5NL_VALUES"), dtype=np.int8)
        assert v.shape == (64,)
        return v
    if member == "iq6_k":
        v = np.array(_dense_macro("IQK_IQ6K_BITS"), dtype=np.uint32).view(np.float32)
        assert v.shape == (128,)
        return v
    raise ValueError(member)
