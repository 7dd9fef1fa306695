"""Activation-arena planning.

The same contract as the reference's planner (chroma/_src/memory.py:12-50): every temporary has a size and an
inclusive lifetime [start, end] in kernel indices; allocations are visited in order of start, a temporary whose end
precedes the current start returns its range to a coalesced free list, and each allocation takes the best-fitting
free range (smallest that is large enough, lowest offset on ties) or extends the arena. The native runtime carries
an identical planner (``chroma_b200_plan_arena``) to lay out its arena; ``tests/test_memory.py`` checks both against
the reference's known answer.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass
class Allocation:
    size: int
    start: int
    end: int
    offset: int = 0


def plan_memory(allocations: dict[str, Allocation]) -> int:
    """Assign offsets in place and return the arena size in bytes."""
    live: list[Allocation] = []
    free: list[tuple[int, int]] = []  # (offset, size)
    total = 0
    for allocation in sorted(allocations.values(), key=lambda a: a.start):
        still = []
        for old in live:
            if old.end < allocation.start:
                free.append((old.offset, old.size))
            else:
                still.append(old)
        live = still
        merged: list[tuple[int, int]] = []
        for offset, size in sorted(free):
            if merged and merged[-1][0] + merged[-1][1] == offset:
                merged[-1] = (merged[-1][0], merged[-1][1] + size)
            else:
                merged.append((offset, size))
        free = merged
        fits = [(size, i) for i, (_, size) in enumerate(free) if size >= allocation.size]
        if fits:
            _, index = min(fits)
            offset, size = free.pop(index)
            allocation.offset = offset
            if size > allocation.size:
                free.append((offset + allocation.size, size - allocation.size))
        else:
            allocation.offset = total
            total += allocation.size
        live.append(allocation)
    return total


def gptoss_buffers(desc: dict, batch: int = 1) -> list[tuple[str, int, int, int]]:
    """(name, bytes, start, end) of one GPT-OSS call's temporaries, in the order the native executor plans them.

    Kernel indices: 0 embedding; per layer l: 1+5l QKV, 2+5l attention, 3+5l out, 4+5l router + expert up,
    5+5l expert down; then 1+5L final norm and 2+5L vocab. Per-layer buffers are reused by every layer.
    """
    L, d, H, hd, KV, k, I = (desc[x] for x in ("layers", "hidden", "heads", "head_dim", "kv_heads", "top_k", "intermediate"))
    N = batch * desc["tokens"]
    es = 2 if desc["storage"] == 1 else 4
    last = 5 * (L - 1)
    key_chunk = 512 if hd <= 32 else 256
    chunks = -(-(desc.get("context", 0) + desc["tokens"]) // key_chunk)
    G = H // KV
    out = [
        ("x", N * d * 4, 0, 1 + 5 * L),
        ("q", N * H * hd * 4, 1, 2 + last),
        ("attn", N * H * hd * 4, 2, 3 + last),
        ("x2", N * d * 4, 3, 5 + last),
        ("ridx", N * k * 4, 4, 5 + last),
        ("rw", N * k * 4, 4, 5 + last),
        ("act", N * k * I * 4, 4, 5 + last),
        ("partial", N * KV * G * chunks * (hd + 2) * 4, 2, 2 + last),
        ("tf", N * d * 4, 1 + 5 * L, 2 + 5 * L),
    ]
    if desc["kind"] != 2:  # uncached programs keep the layer's new K/V rows in the arena
        out += [("scratch_k", N * KV * hd * es, 1, 2 + last), ("scratch_v", N * KV * hd * es, 1, 2 + last)]
    return out


def is_large(desc: dict) -> bool:
    """The large-width bf16 path (tensor-core GEMMs, flash attention): hidden >= 1024, head_dim 64."""
    return (desc["storage"] == 1 and desc["hidden"] >= 1024 and desc["hidden"] % 64 == 0 and desc["head_dim"] == 64
            and desc["intermediate"] % 64 == 0 and desc["experts"] <= 256)


def large_arena(desc: dict, batch: int = 1, selected_rows: bool = True) -> int:
    """Arena bytes of the large-width executor (every buffer lives for the whole call)."""
    d, H, hd, KV, k, I, E = (desc[x] for x in ("hidden", "heads", "head_dim", "kv_heads", "top_k", "intermediate", "experts"))
    N = batch * desc["tokens"]
    P = N * k
    rows = batch if selected_rows else N
    chunks = -(-(desc.get("context", 0) + desc["tokens"]) // 256)
    heads = (H + 2 * KV) * hd
    sizes = [N * d * 2, N * d * 2, N * heads * 2, N * H * hd * 2, N * H * hd * 2, N * E * 2, P * d * 2, P * I * 2,
             P * d * 2, rows * d * 2, N * KV * hd * 2, N * KV * hd * 2, P * 4, rows * d * 4,
             N * KV * (H // KV) * chunks * (hd + 2) * 4, P * 4, P * 4, E * 4, E * 4, (E + 1) * 4, (E + 1) * 4]
    return sum(-(-s // 1024) * 1024 for s in sizes)


def gptoss_arena(desc: dict, batch: int = 1) -> tuple[int, int]:
    """(planned arena bytes, bytes without reuse) for a GPT-OSS executor."""
    if is_large(desc):
        total = large_arena(desc, batch, desc["kind"] != 1)
        return total, total
    allocations = {
        name: Allocation((size + 255) // 256 * 256, start, end) for name, size, start, end in gptoss_buffers(desc, batch)
    }
    return plan_memory(allocations), sum(a.size for a in allocations.values())
