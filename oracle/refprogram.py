"""Test infrastructure: load a reference CPU artefact built by ``oracle/build_ref.py`` and run it.

Restates the loading steps of the reference's ``Program._load`` (chroma/_src/program.py:83-101): read
``model.json``, import the ``_chroma_<uuid>`` extension from the artefact directory, check its ``signature``
against the manifest's tensors (program.py:62-63), and construct ``Model(weights_path)``. The native
``run(inputs, outputs)`` (chroma/_src/core/bindings.h:41-74) then executes the reference's generated C++
(single-threaded). Only NumPy and ml_dtypes are needed, so this works on a machine without the reference
sources, which is how ``bench.py --impl reference`` times the reference's own CPU program.
"""

from __future__ import annotations

import hashlib
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent / "_ref"


def _signature(inputs: list, outputs: list) -> str:
    return hashlib.sha256(json.dumps({"inputs": inputs, "outputs": outputs}, sort_keys=True).encode()).hexdigest()


class RefProgram:
    def __init__(self, name_or_dir: str | Path) -> None:
        directory = Path(name_or_dir)
        if not directory.is_absolute() and not directory.exists():
            directory = ROOT / str(name_or_dir)
        self.directory = directory.resolve()
        manifest = json.loads((self.directory / "model.json").read_text())
        name = manifest["library"].split(".")[0]
        module = sys.modules.get(name)
        if module is None:
            spec = importlib.util.spec_from_file_location(name, self.directory / manifest["library"])
            if spec is None or spec.loader is None:
                raise ImportError(f"cannot load {manifest['library']}")
            module = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(module)
            sys.modules[name] = module
        if module.signature != _signature(manifest["inputs"], manifest["outputs"]):
            raise ValueError("reference artefact metadata does not match its library")
        self.inputs = manifest["inputs"]
        self.outputs = manifest["outputs"]
        self.stats = manifest["stats"]
        weights = self.directory / manifest["weights"]
        shared = self.directory / "shared_weights.json"
        if not weights.exists() and shared.exists():
            weights = self.directory.parent / json.loads(shared.read_text())["directory"] / manifest["weights"]
        self.model = module.Model(str(weights))
        self.device = "CPU"

    def __call__(self, *inputs: np.ndarray, out: list[np.ndarray] | None = None):  # type: ignore[no-untyped-def]
        from ml_dtypes import bfloat16  # noqa: F401  (registers the dtype name)

        arrays = [np.require(a, requirements=["C", "A"]) for a in inputs]
        outs = list(out) if out is not None else [np.empty(s["shape"], dtype=s["dtype"]) for s in self.outputs]
        self.model.run(arrays, outs)
        return outs[0] if len(outs) == 1 else tuple(outs)

    def close(self) -> None:
        self.model = None

    def __enter__(self) -> "RefProgram":
        return self

    def __exit__(self, *exc: object) -> None:
        self.close()


def available(name: str) -> bool:
    return (ROOT / name / "model.json").exists()
