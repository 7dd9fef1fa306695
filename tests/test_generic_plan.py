"""CPU checks of the generic-graph lowering (chroma_b200/_src/graph.py): every case of tests/generic_cases.py is
compiled by this backend's compiler and its plan is run by the NumPy plan interpreter (tests/graph_emulator.py),
step for step what csrc/graph.cu computes, against the reference's own compiled CPU program's outputs
(tests/golden/generic.npz). Also the plan's refusal of what the reference refuses."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from chroma_b200._src.compiler import lower, pack
from tests import generic_cases as gc
from tests.conftest import GOLDEN
from tests.graph_emulator import Emulator


@pytest.fixture(scope="module")
def golden() -> dict[str, np.ndarray]:
    with np.load(GOLDEN / "generic.npz") as data:
        return {k: data[k] for k in data.files}


@pytest.mark.parametrize("name", [c.name for c in gc.cases()])
def test_plan_matches_reference_program(golden: dict[str, np.ndarray], name: str) -> None:
    case = gc.by_name()[name]
    sets = case.input_sets()
    lowered = lower(torch.export.export(case.module(), sets[0]))
    assert lowered.stats.get("generic_graph")
    weights, _ = pack(lowered.tensors)
    emulator = Emulator(lowered.plan["graph"], weights)
    for s in range(len(sets)):
        inputs = gc.golden_arrays(golden, name, "in", s)
        want = gc.golden_arrays(golden, name, "out", s)
        outs = [np.empty(w.shape, w.dtype) for w in want]
        emulator.run([np.ascontiguousarray(a) for a in inputs], outs)
        gc.compare(case, outs, want, inputs)


def test_plan_refuses_what_the_reference_refuses() -> None:
    ids = torch.tensor([1, 0])
    with pytest.raises(NotImplementedError):  # elementwise arithmetic on int64 (lowering.py:185-186)
        lower(torch.export.export(gc.Fn(lambda x: x * 2), (ids,)))
    with pytest.raises(NotImplementedError):  # an operator outside the table
        lower(torch.export.export(gc.Fn(lambda x: torch.tanh(x)), (torch.ones(3),)))
    with pytest.raises(NotImplementedError):  # top-k along an axis longer than 4096 (lowering.py:291-292)
        lower(torch.export.export(gc.Fn(lambda x: x.topk(2)), (torch.ones(5000),)))


def test_gather_out_of_range_raises_index_error(golden: dict[str, np.ndarray]) -> None:
    case = gc.by_name()["int64_gather_cat_triangle"]
    lowered = lower(torch.export.export(case.module(), case.inputs()))
    emulator = Emulator(lowered.plan["graph"], pack(lowered.tensors)[0])
    x = np.arange(20, dtype=np.int64).reshape(5, 4)
    outs = [np.empty(o["shape"], np.int64) for o in lowered.outputs]
    for bad in (5, -6, 2**40):
        with pytest.raises(IndexError):
            emulator.run([x, np.array([bad, 0, 1])], outs)
    emulator.run([x, np.array([4, -1, 0])], outs)
    np.testing.assert_array_equal(outs[0], x[[4, -1, 0]])
