"""Test infrastructure: import the reference Chroma package from its read-only source tree.

This file is part of the ORACLE (checker) only. Nothing in ``chroma_b200`` imports it. It runs in the
development container, where the reference sources exist, to build the reference's own CPU programs
(``oracle/build_ref.py``) and the golden fixtures (``tests/golden/make_golden.py``). Only the reference's
``chroma`` and ``scripts`` packages are redirected; this repository's own ``tests`` package is untouched.

The reference targets Python 3.14. On this interpreter (3.12) three mechanical source patches are needed,
applied *in memory* while importing (no file is copied or written):

1. ``except A, B:`` (PEP 758, 3.14 only) at chroma/_src/build.py:45 becomes ``except (A, B):``.
2. ``from __future__ import annotations`` is prepended to each module, because the reference relies on
   deferred annotations (PEP 649), e.g. ``View.base: Value | None`` before ``Value`` exists
   (chroma/_src/value.py:19-23).

Header files (``codegen/cpu/kernels.h`` and friends) are read by the reference's build step from where they
lie: ``build.py`` passes ``-I <its own directory>``, which is the reference tree.
"""

from __future__ import annotations

import importlib.abc
import importlib.machinery
import importlib.util
import os
import re
import sys
from pathlib import Path
from typing import Any

# The reference checkout: $CHROMA_REFERENCE, else a directory named ``reference`` beside this repository.
REFERENCE = Path(os.environ.get("CHROMA_REFERENCE") or Path(__file__).resolve().parents[2] / "reference")
# The patched copy of the reference's ``chroma`` package that oracle/build_ref.py stages for machines without the
# reference sources (git-ignored; travels with the other reference programs under oracle/_ref).
STAGED = Path(__file__).resolve().parent / "_ref" / "pkg"
_PACKAGES = ("chroma", "scripts")
_EXCEPT = re.compile(r"^(\s*)except ([A-Za-z_][\w.]*(?:\s*,\s*[A-Za-z_][\w.]*)+):", re.M)


def _patch(source: str) -> str:
    source = _EXCEPT.sub(lambda m: f"{m.group(1)}except ({m.group(2)}):", source)
    lines = source.splitlines(keepends=True)
    # A module docstring must stay first; insert the future import after it when present.
    insert_at = 0
    stripped = source.lstrip()
    if stripped.startswith(('"""', "'''")):
        quote = stripped[:3]
        end = source.find(quote, source.find(quote) + 3)
        insert_at = source[: end + 3].count("\n") + 1
    if "from __future__ import annotations" not in source:
        lines.insert(insert_at, "from __future__ import annotations\n")
    return "".join(lines)


class _Loader(importlib.abc.SourceLoader):
    def __init__(self, fullname: str, path: Path) -> None:
        self.fullname = fullname
        self.path = path

    def get_filename(self, fullname: str) -> str:
        return str(self.path)

    def get_data(self, path: str) -> bytes:
        text = Path(path).read_text()
        if path.endswith(".py"):
            text = _patch(text)
        return text.encode()

    def path_stats(self, path: str) -> dict:
        # No bytecode cache: the patched source must never be written anywhere.
        raise OSError


class _Finder(importlib.abc.MetaPathFinder):
    def find_spec(self, fullname, path=None, target=None):  # type: ignore[no-untyped-def]
        if fullname.split(".")[0] not in _PACKAGES:
            return None
        parts = fullname.split(".")
        base = REFERENCE.joinpath(*parts)
        if (base / "__init__.py").exists():
            file, package = base / "__init__.py", True
        elif base.with_suffix(".py").exists():
            file, package = base.with_suffix(".py"), False
        elif base.is_dir():
            file, package = None, True
        else:
            return None
        if file is None:
            spec = importlib.machinery.ModuleSpec(fullname, None, is_package=True)
            spec.submodule_search_locations = [str(base)]
            return spec
        loader = _Loader(fullname, file)
        spec = importlib.util.spec_from_file_location(
            fullname, file, loader=loader, submodule_search_locations=[str(base)] if package else None
        )
        return spec


def install() -> None:
    """Make ``import chroma`` and ``import scripts.export`` resolve to the patched reference."""
    if not REFERENCE.exists():
        raise RuntimeError(f"reference tree not found at {REFERENCE}")
    sys.dont_write_bytecode = True
    if not any(isinstance(f, _Finder) for f in sys.meta_path):
        sys.meta_path.insert(0, _Finder())


def runtime() -> Any:
    """The reference's ``chroma`` package for loading and running programs: from the source tree when it is here,
    else from the staged copy (oracle/build_ref.py ``stage_package``). Raises ModuleNotFoundError when neither
    exists."""
    import importlib

    if REFERENCE.exists():
        install()
    elif (STAGED / "chroma" / "__init__.py").exists():
        sys.dont_write_bytecode = True
        if str(STAGED) not in sys.path:
            sys.path.insert(0, str(STAGED))
    else:
        raise ModuleNotFoundError("neither the reference sources nor the staged copy of its chroma package is here")
    return importlib.import_module("chroma")
