"""``Program``: load a compiled artefact directory and run it on NumPy arrays (no Torch needed).

Mirrors the reference's public runtime object (chroma/_src/program.py:73-153): the same manifest checks
(version 2, Python ABI, tensor-signature hash), the same call surface (``inputs``, ``outputs``, ``stats``,
``device``, ``__call__(*arrays, out=None)``, ``close()``, context manager), the same error messages, and calls
serialised by a lock. The artefact's library module provides ``signature`` and ``Model`` (the native object
protocol), so a reference ``chroma.Program`` can load a B200 artefact too.
"""

from __future__ import annotations

import hashlib
import importlib.util
import json
import sys
import sysconfig
import threading
from collections.abc import Sequence
from pathlib import Path
from types import TracebackType
from typing import Any

import numpy as np


def signature(inputs: list[dict[str, Any]], outputs: list[dict[str, Any]]) -> str:
    """sha256 of the tensor specs, the binding check of chroma/_src/program.py:62-63."""
    return hashlib.sha256(json.dumps({"inputs": inputs, "outputs": outputs}, sort_keys=True).encode()).hexdigest()


def _import_library(directory: Path, library: str) -> Any:
    name = library.split(".")[0]
    module = sys.modules.get(name)
    if module is None:
        spec = importlib.util.spec_from_file_location(name, directory / library)
        if spec is None or spec.loader is None:
            raise ImportError("Cannot load the native model extension")
        module = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(module)
        sys.modules[name] = module
    return module


class Program:
    def __init__(self, directory: str | Path) -> None:
        manifest, native = self._load(directory)
        self._lock = threading.Lock()
        self._model: Any = native
        self._inputs = manifest["inputs"]
        self._outputs = manifest["outputs"]
        self._stats = manifest["stats"]
        self._plan = manifest.get("b200")
        self._directory = Path(directory).resolve()
        self._device = native.device

    @classmethod
    def from_native(cls, native: Any, stats: dict[str, Any] | None = None) -> "Program":
        """A Program over an already created native program (e.g. one whose weights live in device memory)."""
        self = cls.__new__(cls)
        self._lock = threading.Lock()

        class _Model:
            def __init__(self, n: Any) -> None:
                self.native = n
                self.device = n.device

            def run(self, inputs: list[Any], outputs: list[Any]) -> None:
                self.native.run(inputs, outputs)

        self._model = _Model(native)
        self._inputs = native.inputs
        self._outputs = native.outputs
        self._stats = stats or {}
        self._plan = native.plan
        self._directory = None
        self._device = native.device
        return self

    @staticmethod
    def _load(directory: str | Path) -> tuple[dict[str, Any], Any]:
        directory = Path(directory).resolve()
        manifest = json.loads((directory / "model.json").read_text())
        if manifest.get("version") != 2 or manifest.get("python_abi") != sysconfig.get_config_var("SOABI"):
            raise ValueError("Incompatible Chroma artifact; recompile it with this Python interpreter")
        module = _import_library(directory, manifest["library"])
        if module.signature != signature(manifest["inputs"], manifest["outputs"]):
            raise ValueError("Artifact tensor metadata does not match its native library")
        return manifest, module.Model(str(directory / manifest["weights"]))

    @property
    def device(self) -> str:
        return self._device

    @property
    def inputs(self) -> list[dict[str, Any]]:
        return self._inputs

    @property
    def outputs(self) -> list[dict[str, Any]]:
        return self._outputs

    @property
    def stats(self) -> dict[str, Any]:
        return self._stats

    @property
    def native(self) -> Any:
        """The ``chroma_b200`` native program (device-resident APIs), or None for a foreign artefact."""
        model = self._model
        return getattr(model, "native", None) if model is not None else None

    @staticmethod
    def _array(value: Any) -> np.ndarray:
        if isinstance(value, np.ndarray):
            array = value
        else:
            tensor = value.detach()
            if str(tensor.dtype) == "torch.bfloat16":
                import torch
                from ml_dtypes import bfloat16

                array = tensor.view(torch.uint16).numpy().view(bfloat16)
            else:
                array = tensor.numpy()
        return np.require(array, requirements=["C", "A"])

    def __call__(self, *inputs: Any, out: np.ndarray | Sequence[np.ndarray] | None = None) -> Any:
        arrays = [self._array(value) for value in inputs]
        if out is None:
            from chroma_b200._src.native import dtype_of

            # Results of the native runtime go to page-locked blocks (one DMA per output, no staging copy).
            pool = getattr(getattr(self._model, "native", None), "pinned", None)
            res: list[np.ndarray] = [
                pool.array(tuple(spec["shape"]), dtype_of(spec["dtype"])) if pool is not None
                else np.empty(spec["shape"], dtype=dtype_of(spec["dtype"]))
                for spec in self._outputs
            ]
        else:
            res = [out] if isinstance(out, np.ndarray) else list(out)
        with self._lock:
            if self._model is None:
                raise RuntimeError("Model is closed")
            self._model.run(arrays, res)
        return res[0] if len(res) == 1 else tuple(res)

    def close(self) -> None:
        with self._lock:
            model, self._model = self._model, None
        native = getattr(model, "native", None)
        if native is not None:
            native.close()

    def __enter__(self) -> "Program":
        return self

    def __exit__(self, exc_type: type[BaseException] | None, exc: BaseException | None, tb: TracebackType | None) -> None:
        self.close()
