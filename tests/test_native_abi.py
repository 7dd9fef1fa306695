"""The C ABI library loads without a GPU and exports every entry point ``include/chroma_b200.h`` declares."""

from __future__ import annotations

import re
import subprocess

from chroma_b200._src import native as nat
from tests.conftest import ROOT


def declared() -> set[str]:
    text = (ROOT / "include" / "chroma_b200.h").read_text()
    return set(re.findall(r"\b(chroma_b200_[a-z0-9_]+)\s*\(", text))


def test_header_declarations_are_exported_and_bound() -> None:
    names = declared()
    assert len(names) >= 16
    lib = nat.lib()
    for name in names:
        assert hasattr(lib, name), name
    assert names == set(nat.SIGNATURES), "ctypes bindings and header disagree"
    symbols = subprocess.run(["nm", "-D", "--defined-only", str(nat.library_path())], capture_output=True, text=True).stdout
    for name in names:
        assert re.search(rf"\bT {name}\b", symbols), name


def test_library_is_built_for_sm_100a() -> None:
    from chroma_b200 import build

    assert "arch=compute_100a,code=sm_100a" in " ".join(build.command())
    assert nat.library_path().exists()
