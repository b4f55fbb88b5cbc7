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
