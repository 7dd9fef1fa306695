"""chroma_b200: a B200-native (sm_100a) CUDA backend for Chroma's compiled GPT-OSS-style programs.

Public surface, as in the reference (chroma/__init__.py:14-26): ``compile``, ``Program``, ``Decoder``; plus
``BatchDecoder`` for device-resident batched decoding. Loading and running artefacts needs NumPy only; ``compile``
imports Torch on first use.
"""

from __future__ import annotations

from pathlib import Path
from typing import Any

from chroma_b200._src.decoder import BatchDecoder, Decoder
from chroma_b200._src.experts import ExpertGroup
from chroma_b200._src.program import Program


def compile(input: Any, output: str | Path, *, blas: bool = True, backend: str = "cuda") -> Program:
    """Compile an ``ExportedProgram`` (or a saved ``.pt2`` path) into ``output`` and load it."""
    from chroma_b200._src.compiler import compile_for_backend

    return compile_for_backend(input, output, blas=blas, backend=backend)


def compile_model(model: Any, output: str | Path, *, steps: int, context: int | None = None, last: bool = False,
                  experts: ExpertGroup | None = None) -> Program:
    """Compile a ``chroma_b200.models.Transformer`` straight from its parameters (no ``torch.export``): a forward
    over ``steps`` tokens, or with ``context`` a KV-cached step of ``steps`` rows (the prefill/decode programs).
    With ``experts`` (an ``ExpertGroup``), this rank's share of the experts only, bound to the group."""
    from chroma_b200._src.compiler import compile_model as _compile_model

    return _compile_model(model, output, steps=steps, context=context, last=last, experts=experts)


__all__ = ["BatchDecoder", "Decoder", "ExpertGroup", "Program", "compile", "compile_model"]
