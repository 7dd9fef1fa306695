"""Host-side logic of expert parallelism (no GPU): expert ownership, the sharded weight layout, the sliced weights
of a rank, and the handle exchange of ``ExpertGroup`` over a real 2-rank ``gloo`` process group with the native
calls replaced by a recording fake."""

from __future__ import annotations

import dataclasses
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from chroma_b200 import models
from chroma_b200._src import compiler
from chroma_b200._src.experts import local_experts

ROOT = Path(__file__).resolve().parents[1]


def tiny_config(experts: int = 4):  # type: ignore[no-untyped-def]
    return dataclasses.replace(models.dev, num_hidden_layers=2, hidden_size=64, intermediate_size=64, head_dim=16,
                               num_attention_heads=4, num_key_value_heads=2, num_experts=experts, experts_per_token=2,
                               vocab_size=256)


def test_local_experts_partition() -> None:
    owned = [list(local_experts(r, 4, 128)) for r in range(4)]
    assert owned[0] == list(range(32)) and owned[3] == list(range(96, 128))
    assert sorted(sum(owned, [])) == list(range(128))
    with pytest.raises(ValueError):
        local_experts(0, 3, 128)
    with pytest.raises(ValueError):
        local_experts(2, 2, 8)


def test_vocab_shard_partition() -> None:
    from chroma_b200._src.experts import vocab_shard

    parts = [vocab_shard(r, 8, 201088) for r in range(8)]
    assert all(len(p) == 25136 for p in parts) and parts[7].stop == 201088
    assert [p.start for p in parts] == [25136 * r for r in range(8)]
    odd = [vocab_shard(r, 3, 10) for r in range(3)]
    assert [list(p) for p in odd] == [[0, 1, 2, 3], [4, 5, 6, 7], [8, 9]]


def test_sharded_layout_keeps_router_and_splits_experts() -> None:
    cfg = tiny_config(8)
    full = dict((n, s) for n, s, _ in compiler.gptoss_layout(cfg))
    half = dict((n, s) for n, s, _ in compiler.gptoss_layout(cfg, 2))
    assert full.keys() == half.keys()
    for name in full:
        if name.endswith(("mlp1_weight", "mlp1_bias", "mlp2_weight", "mlp2_bias")):
            assert half[name] == (full[name][0] // 2, *full[name][1:])
        else:
            assert half[name] == full[name]
    vocab_half = dict((n, s) for n, s, _ in compiler.gptoss_layout(cfg, 2, 128))
    assert vocab_half["unembedding.weight"] == (128, cfg.hidden_size)
    assert vocab_half["embedding.weight"] == full["embedding.weight"]
    plan, _ = compiler.synthetic_gptoss(cfg, steps=4, ep_world=2)
    full_plan, _ = compiler.synthetic_gptoss(cfg, steps=4)
    assert plan["desc"]["experts"] == 8 and plan["desc"]["weight_bytes"] < full_plan["desc"]["weight_bytes"]


def test_lowered_shard_is_the_slice_of_the_full_model() -> None:
    cfg = tiny_config(4)
    model = models.random_transformer(cfg, seed=3, std=0.05, dtype=torch.bfloat16)
    full = compiler.lower_model(model, steps=4)
    names = [n for n, _, _ in compiler.gptoss_layout(cfg)]
    for rank in range(2):
        from chroma_b200._src.experts import vocab_shard

        vocab = vocab_shard(rank, 2, cfg.vocab_size)
        shard = compiler.lower_model(model, steps=4, experts=local_experts(rank, 2, 4), vocab_rows=vocab)
        assert len(shard.tensors) == len(full.tensors)
        for name, a, b in zip(names, shard.tensors, full.tensors):
            if name.endswith(("mlp1_weight", "mlp1_bias", "mlp2_weight", "mlp2_bias")):
                per = b.shape[0] // 2
                np.testing.assert_array_equal(a.view(np.uint8), b[rank * per : (rank + 1) * per].view(np.uint8))
            elif name == "unembedding.weight":
                np.testing.assert_array_equal(a.view(np.uint8), b[vocab.start : vocab.stop].view(np.uint8))
            else:
                np.testing.assert_array_equal(a.view(np.uint8), b.view(np.uint8))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


def _exchange_rank(rank: int, world: int, port: int, out_dir: str) -> None:
    """One gloo rank: ExpertGroup over a fake native library that records what it is asked to open."""
    sys.path.insert(0, str(ROOT))
    import ctypes

    import torch.distributed as dist

    from chroma_b200._src import experts, native

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    opened: list[bytes] = []

    def fake_call(name: str, *args):  # type: ignore[no-untyped-def]
        if name == "chroma_b200_ep_create":
            r, w, pairs, hidden, e, vrows, vocab, out = args
            assert (r, w, pairs, hidden, e, vrows, vocab) == (rank, world, 64, 2880, 32, 0, 0)
            out._obj.value = 1000 + rank
        elif name == "chroma_b200_ep_handle":
            ctypes.memmove(args[1], bytes([rank + 1]) * native.EP_HANDLE_BYTES, native.EP_HANDLE_BYTES)
        elif name == "chroma_b200_ep_open":
            opened.append(args[1].raw)
        else:
            raise AssertionError(name)

    class FakeLib:
        destroyed: list[int] = []

        def chroma_b200_ep_destroy(self, handle):  # type: ignore[no-untyped-def]
            self.destroyed.append(handle.value)

    native.call = fake_call  # type: ignore[assignment]
    native.lib = lambda: FakeLib()  # type: ignore[assignment]
    group = experts.ExpertGroup(rank, world, max_pairs=64, hidden=2880, experts=32)
    assert list(group.local) == list(range(rank * 16, rank * 16 + 16))
    group.close()
    group.close()
    # A broken exchange (wrong count) fails cleanly and releases the native group.
    try:
        experts.ExpertGroup(rank, world, max_pairs=64, hidden=2880, experts=32, exchange=lambda h: [h])
        raise AssertionError("expected ValueError")
    except ValueError:
        pass
    Path(out_dir, f"rank{rank}.bin").write_bytes(opened[0])
    Path(out_dir, f"destroyed{rank}.txt").write_text(",".join(map(str, FakeLib.destroyed)))
    dist.destroy_process_group()


def test_expert_group_handle_exchange_over_gloo(tmp_path: Path) -> None:
    world = 2
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    mp.start_processes(_exchange_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    want = b"".join(bytes([r + 1]) * 64 for r in range(world))
    for rank in range(world):
        assert (tmp_path / f"rank{rank}.bin").read_bytes() == want
        assert (tmp_path / f"destroyed{rank}.txt").read_text() == f"{1000 + rank},{1000 + rank}"
