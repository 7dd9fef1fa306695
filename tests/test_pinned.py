"""Host logic of the page-locked result pool (no GPU): blocks are recycled only after every array viewing them is
gone, sizes are kept apart, idle blocks beyond the cap are freed, and close() frees the idle ones while blocks
behind live arrays are freed when those arrays go. The native allocator is replaced by a recording fake."""

from __future__ import annotations

import ctypes
import gc

import numpy as np
import pytest

from chroma_b200._src import native


@pytest.fixture()
def fake_host_memory(monkeypatch: pytest.MonkeyPatch):  # type: ignore[no-untyped-def]
    blocks: dict[int, ctypes.Array] = {}
    freed: list[int] = []

    def fake_call(name: str, nbytes, out) -> None:  # type: ignore[no-untyped-def]
        assert name == "chroma_b200_host_alloc"
        buf = (ctypes.c_char * int(nbytes.value))()
        ptr = ctypes.addressof(buf)
        blocks[ptr] = buf
        out._obj.value = ptr

    class FakeLib:
        def chroma_b200_host_free(self, p) -> None:  # type: ignore[no-untyped-def]
            freed.append(int(p.value))

    monkeypatch.setattr(native, "call", fake_call)
    monkeypatch.setattr(native, "lib", lambda: FakeLib())
    return blocks, freed


def test_blocks_recycle_only_after_the_last_view(fake_host_memory) -> None:  # type: ignore[no-untyped-def]
    blocks, freed = fake_host_memory
    pool = native.PinnedPool(keep=2)
    a, pa = pool.array_ptr((2, 8), np.float32)
    assert a.flags.writeable and a.flags.c_contiguous and a.ctypes.data == pa
    a[:] = 1.0
    view = a[1]
    del a
    gc.collect()
    b, pb = pool.array_ptr((2, 8), np.float32)
    assert pb != pa  # the first block is still behind `view`
    np.testing.assert_array_equal(view, np.ones(8, np.float32))
    del view
    gc.collect()
    c, pc = pool.array_ptr((2, 8), np.float32)
    assert pc == pa  # recycled once its last view went
    d, pd = pool.array_ptr((3,), np.int64)
    assert pd not in (pa, pb)  # another size: another block
    assert len(blocks) == 3 and not freed
    del b, c, d


def test_cap_and_close(fake_host_memory) -> None:  # type: ignore[no-untyped-def]
    blocks, freed = fake_host_memory
    pool = native.PinnedPool(keep=1)
    arrays = [pool.array((4,), np.float32) for _ in range(3)]
    ptrs = [x.ctypes.data for x in arrays]
    del arrays
    gc.collect()
    assert len(freed) == 2 and set(freed) <= set(ptrs)  # one idle block kept, the others freed
    live = pool.array((4,), np.float32)
    pool.close()
    assert len(freed) == 2  # the kept block is behind `live`
    ptr = live.ctypes.data
    del live
    gc.collect()
    assert freed[-1] == ptr and len(freed) == 3  # freed when its array went, the pool being closed
