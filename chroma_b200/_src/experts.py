"""``ExpertGroup``: the experts of GPT-OSS-shaped programs split across the GPUs of one node (one process per GPU).

The reference runs every expert on one device (chroma/models/gpt_oss.py:243-265). Here rank ``r`` of ``world``
owns experts ``[r*E/world, (r+1)*E/world)``; the routed rows travel between GPUs by stores into each other's device
memory (the native kernels in ``csrc/ep.cuh``), so a MoE layer needs no host round trip and no library collective.
The host side only sets the group up: each rank exports a handle to its shared buffer, the handles are gathered in
rank order through a host channel (``torch.distributed`` by default), and every rank opens the others'.

Programs bound to a group (``Native(plan, ..., ep=group)``, ``compile_model(..., experts=group)``) hold the local
experts only. Every rank must call the same programs in the same order; a rank that does not arrive within the bounded
wait (10 s, or ``CHROMA_B200_EP_TIMEOUT_MS`` when the group is created) turns into a ``RuntimeError`` on the others,
after which the group must be recreated.
"""

from __future__ import annotations

import ctypes
from collections.abc import Callable, Sequence
from typing import Any

from chroma_b200._src import native as nat


def torch_exchange(handle: bytes) -> list[bytes]:
    """Gather every rank's handle in rank order over the default ``torch.distributed`` process group."""
    import torch.distributed as dist

    out: list[Any] = [None] * dist.get_world_size()
    dist.all_gather_object(out, handle)
    return [bytes(h) for h in out]


def local_experts(rank: int, world: int, experts: int) -> range:
    """The global expert indices rank ``rank`` owns."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a group of {world}")
    if experts % world:
        raise ValueError(f"{experts} experts do not split evenly over {world} ranks")
    per = experts // world
    return range(rank * per, (rank + 1) * per)


def vocab_shard(rank: int, world: int, vocab: int) -> range:
    """The unembedding rows rank ``rank`` holds when the vocab projection is sharded: ceil(V / world) per rank."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a group of {world}")
    per = -(-vocab // world)
    return range(min(vocab, rank * per), min(vocab, (rank + 1) * per))


class ExpertGroup:
    """One rank's membership in an expert-parallel group on the current CUDA device.

    ``max_pairs``: the most (token, expert) pairs one call of any program on this rank routes (rows x top_k); it
    sizes the receive buffer (``world * max_pairs`` rows of ``hidden`` bf16) and the return buffer.
    ``vocab_rows`` > 0 (with ``vocab`` = V) also shards the vocab projection by vocab rows: this rank's programs hold
    unembedding rows ``vocab_slice`` only, and each call's final rows are projected on every rank's shard (at most
    ``vocab_rows`` final rows per call on a rank).
    ``exchange``: gathers one ``bytes`` handle per rank, in rank order (default ``torch_exchange``).
    """

    def __init__(self, rank: int, world: int, *, max_pairs: int, hidden: int, experts: int, vocab_rows: int = 0,
                 vocab: int = 0, exchange: Callable[[bytes], Sequence[bytes]] | None = None) -> None:
        self.rank, self.world, self.experts, self.hidden, self.max_pairs = rank, world, experts, hidden, max_pairs
        self.local = local_experts(rank, world, experts)
        self.vocab_slice = vocab_shard(rank, world, vocab) if vocab_rows > 0 else None
        handle = ctypes.c_void_p()
        nat.call("chroma_b200_ep_create", rank, world, max_pairs, hidden, experts, vocab_rows, vocab,
                 ctypes.byref(handle))
        self.handle = handle
        try:
            mine = ctypes.create_string_buffer(nat.EP_HANDLE_BYTES)
            nat.call("chroma_b200_ep_handle", handle, mine)
            handles = list((exchange or torch_exchange)(mine.raw))
            if len(handles) != world or any(len(h) != nat.EP_HANDLE_BYTES for h in handles):
                raise ValueError("the handle exchange must return one handle per rank")
            if handles[rank] != mine.raw:
                raise ValueError("the handle exchange returned another rank's handle in this rank's place")
            table = ctypes.create_string_buffer(b"".join(handles), world * nat.EP_HANDLE_BYTES)
            nat.call("chroma_b200_ep_open", handle, table)
        except BaseException:
            nat.lib().chroma_b200_ep_destroy(handle)
            self.handle = None
            raise

    def close(self) -> None:
        if self.handle is not None:
            nat.lib().chroma_b200_ep_destroy(self.handle)
            self.handle = None

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass

    def __enter__(self) -> "ExpertGroup":
        return self

    def __exit__(self, *exc: object) -> None:
        self.close()
