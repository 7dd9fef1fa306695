"""GPU parity of generic exported graphs (chroma_b200/_src/graph.py + csrc/graph.cu) against the reference's own
compiled CPU program (tests/golden/generic.npz, tests/golden/make_generic.py), through ``chroma_b200.compile(...,
backend="cuda")`` and ``Program``: the reference's acceptance contract for its CUDA backend (tests/test_cuda.py:281-306
of the reference) -- two input sets, results within the case's tolerance (int64 exactly), ``out=`` arrays written in
place and returned by identity, earlier results untouched by later calls, the artefact reloaded by ``Program(dir)``.
The share of float elements bit-identical to the reference's is recorded per case."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import chroma_b200
from tests import generic_cases as gc
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def golden() -> dict[str, np.ndarray]:
    with np.load(GOLDEN / "generic.npz") as data:
        return {k: data[k] for k in data.files}


@pytest.mark.parametrize("name", [c.name for c in gc.cases()])
def test_generic_graph_matches_reference(gpu: None, tmp_path: Path, golden: dict, name: str,  # type: ignore[type-arg]
                                         record_property) -> None:  # type: ignore[no-untyped-def]
    case = gc.by_name()[name]
    sets = case.input_sets()
    with chroma_b200.compile(torch.export.export(case.module(), sets[0]), tmp_path / name) as program:
        assert program.stats.get("generic_graph") and program.stats["backend"] == "cuda"
        shares = []
        for s in range(len(sets)):
            inputs = gc.golden_arrays(golden, name, "in", s)
            want = gc.golden_arrays(golden, name, "out", s)
            got = program(*inputs)
            got = list(got) if isinstance(got, (tuple, list)) else [got]
            shares.append(gc.compare(case, got, want, inputs))
            reused = program(*inputs, out=got if len(got) > 1 else got[0])
            for a, b in zip(reused if isinstance(reused, (tuple, list)) else [reused], got):
                assert a is b
        saved = [np.array(a, copy=True) for a in got]
        program(*gc.golden_arrays(golden, name, "in", 0))
        for a, b in zip(got, saved):  # bit for bit (NaN included)
            np.testing.assert_array_equal(np.asarray(a).reshape(-1).view(np.uint8), np.asarray(b).reshape(-1).view(np.uint8))
        record_property("bit_identical_share", f"{min(shares):.4f}")
    with chroma_b200.Program(tmp_path / name) as loaded:
        inputs = gc.golden_arrays(golden, name, "in", 0)
        got = loaded(*inputs)
        gc.compare(case, list(got) if isinstance(got, (tuple, list)) else [got], gc.golden_arrays(golden, name, "out", 0),
                   inputs)


def test_generic_gather_bounds_and_recovery(gpu: None, tmp_path: Path) -> None:
    """Out-of-range rows raise IndexError and leave the program usable (the reference's Runner::run contract)."""
    case = gc.by_name()["int64_gather_cat_triangle"]
    x = np.arange(20, dtype=np.int64).reshape(5, 4)
    with chroma_b200.compile(torch.export.export(case.module(), case.inputs()), tmp_path / "g") as program:
        good = program(x, np.array([4, -1, 0]))
        for bad in (5, -6, 2**40):
            with pytest.raises(IndexError):
                program(x, np.array([bad, 0, 1]))
            again = program(x, np.array([4, -1, 0]))
            for a, b in zip(again, good):
                np.testing.assert_array_equal(a, b)
        np.testing.assert_array_equal(good[0], x[[4, -1, 0]])
