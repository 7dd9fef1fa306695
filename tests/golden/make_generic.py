"""Golden outputs of the generic-graph cases (tests/generic_cases.py) from the reference's own compiled CPU programs.

Run in the development container (where the reference sources exist): ``python -m tests.golden.make_generic``.
Each case is exported with torch.export, compiled by the reference (``chroma.compile(..., backend="cpu",
blas=False)``: the portable loops, single-threaded) and run on two input sets; inputs and outputs are stored in
``generic.npz`` (bf16 arrays as their uint16 bits, with the dtype names beside them).
"""

from __future__ import annotations

import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def raw(a: np.ndarray) -> tuple[np.ndarray, str]:
    a = np.asarray(a)
    name = str(a.dtype)
    return (a.view(np.uint16) if name == "bfloat16" else a), name


def main() -> None:
    import torch

    from oracle import refimport
    from tests.generic_cases import cases, to_numpy

    chroma = refimport.runtime()
    data: dict[str, np.ndarray] = {}
    with tempfile.TemporaryDirectory() as tmp:
        for case in cases():
            sets = case.input_sets()
            exported = torch.export.export(case.module(), sets[0])
            with chroma.compile(exported, Path(tmp) / case.name, backend="cpu", blas=False) as program:
                for s, inputs in enumerate(sets):
                    arrays = [to_numpy(t) for t in inputs]
                    result = program(*arrays)
                    outs = list(result) if isinstance(result, (tuple, list)) else [result]
                    for k, a in enumerate(arrays):
                        data[f"{case.name}/in{s}_{k}"], data[f"{case.name}/in{s}_{k}_dtype"] = map(np.asarray, raw(a))
                    for k, a in enumerate(outs):
                        data[f"{case.name}/out{s}_{k}"], data[f"{case.name}/out{s}_{k}_dtype"] = map(np.asarray, raw(a))
            print("golden", case.name, flush=True)
    np.savez_compressed(HERE / "generic.npz", **data)


if __name__ == "__main__":
    main()
