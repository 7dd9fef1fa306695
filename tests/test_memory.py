"""Arena planner: the reference's known answer (tests/test_runtime.py:287-302) and native == Python planning."""

from __future__ import annotations

import ctypes

import numpy as np

from chroma_b200._src import native as nat
from chroma_b200._src.memory import Allocation, gptoss_arena, plan_memory


def test_known_answer_inclusive_lifetimes_alignment_and_coalescing() -> None:
    allocations = {"a": Allocation(64, 0, 1), "b": Allocation(128, 1, 2), "c": Allocation(64, 2, 3), "d": Allocation(192, 4, 5)}
    assert plan_memory(allocations) == 192
    assert allocations["a"].offset == allocations["c"].offset
    assert allocations["d"].offset == 0
    for left in allocations.values():
        for right in allocations.values():
            if left is right or left.end < right.start or right.end < left.start:
                continue
            assert left.offset + left.size <= right.offset or right.offset + right.size <= left.offset


def native_plan(sizes: list[int], starts: list[int], ends: list[int]) -> tuple[int, list[int]]:
    n = len(sizes)
    offsets = (ctypes.c_int64 * n)()
    total = nat.lib().chroma_b200_plan_arena(
        n, (ctypes.c_int64 * n)(*sizes), (ctypes.c_int32 * n)(*starts), (ctypes.c_int32 * n)(*ends), offsets)
    return int(total), list(offsets)


def test_native_planner_matches_python_planner() -> None:
    rng = np.random.default_rng(0)
    for _ in range(200):
        n = int(rng.integers(1, 24))
        starts = rng.integers(0, 40, n)
        ends = starts + rng.integers(0, 12, n)
        sizes = (rng.integers(1, 16, n) * 64).tolist()
        allocations = {str(i): Allocation(int(s), int(a), int(b)) for i, (s, a, b) in enumerate(zip(sizes, starts, ends))}
        total = plan_memory(allocations)
        ntotal, offsets = native_plan(sizes, starts.tolist(), ends.tolist())
        assert ntotal == total
        assert offsets == [allocations[str(i)].offset for i in range(n)]


def test_gptoss_arena_reuses_memory() -> None:
    desc = {"layers": 12, "hidden": 128, "heads": 8, "head_dim": 16, "kv_heads": 1, "top_k": 4, "intermediate": 128,
            "tokens": 8, "storage": 0, "kind": 1}
    planned, unreused = gptoss_arena(desc)
    assert 0 < planned < unreused
