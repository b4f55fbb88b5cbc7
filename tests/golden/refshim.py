"""Import the reference's codec/format modules without its mlx-importing package.

Fixture generation only: this runs in the build container, where the
reference checkout exists. Nothing on the GPU box imports it.

The reference package ``mlx_iqk`` imports ``mlx`` from its ``__init__``
(src/mlx_iqk/__init__.py:22-38), so the three numpy-only modules this repo
pins against (``iq1grid``, ``format``, ``codec``) are loaded by file path
under an empty stand-in package. ``codec`` hard-codes ``.dylib`` library
names (src/mlx_iqk/codec.py:88-100); they are pointed at the ``.so`` files
that ``oracle/Makefile`` compiles from the reference's own vendored sources.
"""

from __future__ import annotations

import importlib.util
import os
import sys
import types
from pathlib import Path

REPO = Path(__file__).resolve().parents[2]


def _reference() -> Path:
    """``$IQK_REF``, else the ``reference_path`` recorded in ``BASELINE.json``."""
    import json
    cand = os.environ.get("IQK_REF") or json.loads(
        (REPO / "BASELINE.json").read_text()).get("reference_path")
    if not cand or not Path(cand).is_dir():
        raise RuntimeError("set IQK_REF to the reference checkout")
    return Path(cand)


REF = _reference()
REF_LIBS = REPO / "oracle" / "_ref"


def load():
    """Return ``(iq1grid, format, codec, wirepack)`` from the reference."""
    src = REF / "src" / "mlx_iqk"
    if "mlx_iqk" not in sys.modules:
        pkg = types.ModuleType("mlx_iqk")
        pkg.__path__ = [str(src)]
        sys.modules["mlx_iqk"] = pkg
    mods = []
    for name in ("iq1grid", "format", "codec"):
        full = f"mlx_iqk.{name}"
        if full not in sys.modules:
            spec = importlib.util.spec_from_file_location(full, src / f"{name}.py")
            mod = importlib.util.module_from_spec(spec)
            sys.modules[full] = mod
            spec.loader.exec_module(mod)
            setattr(sys.modules["mlx_iqk"], name, mod)
        mods.append(sys.modules[full])
    codec = mods[2]
    codec.library_path = lambda: REF_LIBS / "libiqk_iq2.so"
    codec.iq1sr4_library_path = lambda: REF_LIBS / "libiqk_iq1sr4.so"
    codec.dense_library_path = lambda: REF_LIBS / "libiqk_dense.so"
    if str(REF / "tests") not in sys.path:
        sys.path.insert(0, str(REF / "tests"))
    import wirepack  # the reference's independent block packers
    return mods[0], mods[1], codec, wirepack
