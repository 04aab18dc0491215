"""Loads the reference's own Triton block-attention module for side-by-side checks.

Test and benchmark infrastructure only. The reference is installed (unmodified)
into ``baseline/_ref`` by ``pip install --no-index --no-build-isolation
--find-links /opt/wheelhouse --target baseline/_ref <reference checkout>``,
which travels with the working tree. That install flattens the reference's
``src`` package, while its kernel module still imports ``src.block_table``
(reference src/kernels/block_attention.py:73); this repository's package is
also named ``src``. So the two reference modules are loaded under the private
name ``ouro_ref``, with ``src.block_table`` pointing at the reference's own
module only while its kernel module is imported.
"""

from __future__ import annotations

import importlib.util
import sys
import types
from pathlib import Path

REF_ROOT = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def _load(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load(root: Path = REF_ROOT):
    """Returns the reference's ``block_attention`` module (its Triton kernel and wrapper).

    Raises FileNotFoundError when the reference is not installed under ``root``.
    """
    if "ouro_ref.kernels.block_attention" in sys.modules:
        return sys.modules["ouro_ref.kernels.block_attention"]
    src = root / "kernels" / "block_attention.py"
    if not src.exists():
        raise FileNotFoundError(f"reference not installed: {src} is missing")
    pkg = types.ModuleType("ouro_ref")
    pkg.__path__ = [str(root)]
    sys.modules["ouro_ref"] = pkg
    kpkg = types.ModuleType("ouro_ref.kernels")
    kpkg.__path__ = [str(root / "kernels")]
    sys.modules["ouro_ref.kernels"] = kpkg
    bt = _load("ouro_ref.block_table", root / "block_table.py")
    saved = {k: sys.modules.get(k) for k in ("src", "src.block_table")}
    alias = types.ModuleType("src")
    alias.block_table = bt
    sys.modules["src"], sys.modules["src.block_table"] = alias, bt
    try:
        return _load("ouro_ref.kernels.block_attention", src)
    finally:
        for k, mod in saved.items():
            if mod is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = mod
