"""Host bookkeeping of the device-resident Decoder (no GPU), over a recording fake of the native decoder: a step's
rows are committed right before the next step (the reference's atomic commit, chroma/_src/decoder.py:130-137),
positions and ring slots advance only after a step succeeds, and a failed or interrupted step leaves the state as it
was."""

from __future__ import annotations

import numpy as np
import pytest

from chroma_b200._src import decoder as dec_mod

CTX, V, STEPS = 8, 11, 4


class FakeProgram:
    def __init__(self, steps: int) -> None:
        cache = {"shape": [2, CTX, 1, 4], "dtype": "float32"}
        self.inputs = [{"shape": [steps], "dtype": "int64"}, {"shape": [steps], "dtype": "float32"}, cache, cache,
                       {"shape": [steps, CTX + steps], "dtype": "float32"},
                       {"shape": [steps, CTX + steps], "dtype": "float32"}, {"shape": [1], "dtype": "int64"}]
        self.outputs = [{"shape": [1, V], "dtype": "float32"}, {"shape": [2, steps, 1, 4], "dtype": "float32"},
                        {"shape": [2, steps, 1, 4], "dtype": "float32"}]
        self.device = "fake"


class FakePool:
    def array_ptr(self, shape, dtype):  # type: ignore[no-untyped-def]
        a = np.zeros(shape, dtype)
        return a, a.ctypes.data


class FakeNative:
    def __init__(self, prefill, decode, window, batch) -> None:  # type: ignore[no-untyped-def]
        self.steps = (STEPS, 1)
        self.pinned = FakePool()
        self.calls: list[tuple] = []
        self.fail_on: int | None = None
        self.cache_dtype, self.cache_bytes, self.cache_shape = np.dtype(np.float32), 0, (2, CTX, 1, 4)

    def step_one(self, which, ids, position, ptr) -> None:  # type: ignore[no-untyped-def]
        ids = [int(t) for t in ids]
        if self.fail_on in ids:
            raise IndexError("token out of range")
        self.calls.append(("step", which, ids, int(position)))

    def commit_one(self, which, count, first) -> None:  # type: ignore[no-untyped-def]
        self.calls.append(("commit", which, int(count), int(first)))

    def close(self) -> None:
        pass


@pytest.fixture()
def decoder(monkeypatch: pytest.MonkeyPatch):  # type: ignore[no-untyped-def]
    monkeypatch.setattr(dec_mod, "_natives", lambda a, b: (a, b))
    monkeypatch.setattr(dec_mod, "NativeDecoder", FakeNative)
    return dec_mod.Decoder(FakeProgram(STEPS), FakeProgram(1))


def test_commit_precedes_the_next_step_and_chunks_split(decoder) -> None:  # type: ignore[no-untyped-def]
    nd = decoder._native
    decoder.append([1, 2, 3, 4, 5, 6])  # a 4-row chunk, then a 2-row chunk, both through the prefill program
    decoder.append([7])
    assert nd.calls == [("step", 0, [1, 2, 3, 4], 0), ("commit", 0, 4, 0), ("step", 0, [5, 6], 4),
                        ("commit", 0, 2, 4), ("step", 1, [7], 6)]
    assert decoder.position == 7
    assert decoder._state.staged == (1, 1, 6)
    np.testing.assert_array_equal(decoder._state.slots, [0, 1, 2, 3, 4, 5, 6, -1])


def test_ring_slots_wrap(decoder) -> None:  # type: ignore[no-untyped-def]
    for t in range(CTX + 3):
        decoder.append([t % V])
    np.testing.assert_array_equal(decoder._state.slots, [8, 9, 10, 3, 4, 5, 6, 7])
    assert decoder.position == CTX + 3


def test_failed_and_interrupted_steps_keep_the_state(decoder) -> None:  # type: ignore[no-untyped-def]
    nd = decoder._native
    decoder.append([1, 2, 3])
    before = decoder._state
    nd.fail_on = 9
    with pytest.raises(IndexError):
        decoder.append([9])
    # The previous step's rows were committed (its staged marker cleared); position and slots are untouched.
    assert decoder.position == before.position == 3
    np.testing.assert_array_equal(decoder._state.slots, before.slots)
    assert decoder._state.staged is None
    nd.fail_on = None
    state = decoder._state
    step = nd.step_one

    def interrupted(*args, **kwargs):  # type: ignore[no-untyped-def]
        step(*args, **kwargs)
        raise KeyboardInterrupt

    nd.step_one = interrupted
    with pytest.raises(KeyboardInterrupt):
        decoder.append([4])
    assert decoder._state is state and decoder.position == 3
    nd.step_one = step
    decoder.append([4])
    assert decoder.position == 4 and nd.calls[-1] == ("step", 1, [4], 3)
