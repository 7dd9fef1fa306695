"""GPU tests of expert parallelism (csrc/ep.cuh through the C ABI).

* One rank (world 1): the whole exchange path runs against this GPU's own buffers; logits, routes and a decode
  sequence must be bit-identical to the program with all experts local (each expert row's GEMM output does not
  depend on which rows share its tile, and the combine sums slots in the same order).
* Vocab column shard (1 and 2 ranks): greedy ids identical to the replicated vocab, logits within bf16 rounding.
* Two ranks (needs 2 GPUs, one process each): every rank's logits equal those of a single-GPU program with all
  experts on the same tokens, bit for bit; then one rank stays away (alive, between calls, nothing in flight) and
  the other rank's call ends in a RuntimeError after the bounded wait, with its GPU still usable.
"""

from __future__ import annotations

import dataclasses
import os
import socket
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch

import chroma_b200
from chroma_b200 import models
from tests import helpers

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def ep_config():  # type: ignore[no-untyped-def]
    return dataclasses.replace(models.gpt_oss_20b, num_hidden_layers=2, hidden_size=1024, intermediate_size=1024,
                               num_attention_heads=16, num_key_value_heads=2, num_experts=8, experts_per_token=2,
                               vocab_size=8192, sliding_window=128)


def ep_model():  # type: ignore[no-untyped-def]
    return models.random_transformer(ep_config(), seed=31, std=0.02, dtype=torch.bfloat16)


def test_single_rank_group_matches_all_local_experts(gpu: None, tmp_path: Path) -> None:
    model = ep_model()
    tokens = np.random.default_rng(32).integers(0, 8192, 64)
    group = chroma_b200.ExpertGroup(0, 1, max_pairs=64 * 2, hidden=1024, experts=8, exchange=lambda h: [h])
    with chroma_b200.compile_model(model, tmp_path / "full", steps=64) as full, \
            chroma_b200.compile_model(model, tmp_path / "ep", steps=64, experts=group) as ep:
        want, got = np.asarray(full(tokens)), np.asarray(ep(tokens))
        np.testing.assert_array_equal(got.view(np.uint16), want.view(np.uint16))
        np.testing.assert_array_equal(ep.native.routes(), full.native.routes())
        for _ in range(2):  # repeated calls advance the group's epochs in step
            np.testing.assert_array_equal(np.asarray(ep(tokens)).view(np.uint16), want.view(np.uint16))
    # A prefill + decode sequence through the device-resident decoder, both programs on the group.
    outs = []
    for experts in (None, group):
        pre = chroma_b200.compile_model(model, tmp_path / f"pre{experts is None}", steps=32, context=96, experts=experts)
        dec = chroma_b200.compile_model(model, tmp_path / f"dec{experts is None}", steps=1, context=96, experts=experts)
        with chroma_b200.Decoder(pre, dec, sliding_window=128) as d:
            outs.append([np.asarray(d.append(tokens[:40]))] + [np.asarray(d.append([int(t)])) for t in tokens[40:46]])
    for a, b in zip(*outs):
        np.testing.assert_array_equal(a.view(np.uint16), b.view(np.uint16))
    group.close()


def test_single_rank_vocab_shard_matches_replicated_vocab(gpu: None, tmp_path: Path) -> None:
    model = ep_model()
    tokens = np.random.default_rng(33).integers(0, 8192, 40)
    group = chroma_b200.ExpertGroup(0, 1, max_pairs=64 * 2, hidden=1024, experts=8, vocab_rows=8, vocab=8192,
                                    exchange=lambda h: [h])
    assert group.vocab_slice == range(0, 8192)
    outs = []
    for experts in (None, group):
        pre = chroma_b200.compile_model(model, tmp_path / f"vpre{experts is None}", steps=32, context=96, experts=experts)
        dec = chroma_b200.compile_model(model, tmp_path / f"vdec{experts is None}", steps=1, context=96, experts=experts)
        with chroma_b200.BatchDecoder(pre, dec, 2) as bd:
            seqs = np.stack([tokens[:32], tokens[8:40]])
            logits = np.asarray(bd.append(seqs))
            ids = bd.append(seqs[:, -1:], argmax=True)
            outs.append((logits, ids, bd.generate(ids, 4)))
    # Two rows take the SIMT vocab kernel when replicated and the tensor-core GEMM when sharded: the same sums in
    # another order, so logits agree to the bf16 rounding of the last bit; the greedy ids are identical.
    helpers.assert_bf16_logits(outs[1][0].astype(np.float32), outs[0][0].astype(np.float32), rel=1e-2)
    np.testing.assert_array_equal(outs[0][1], outs[1][1])
    np.testing.assert_array_equal(outs[0][2], outs[1][2])
    group.close()


def test_group_rejects_mismatched_programs(gpu: None, tmp_path: Path) -> None:
    group = chroma_b200.ExpertGroup(0, 1, max_pairs=8, hidden=1024, experts=8, exchange=lambda h: [h])
    with pytest.raises(ValueError, match="pairs"):
        chroma_b200.compile_model(ep_model(), tmp_path / "big", steps=64, experts=group)
    with pytest.raises(ValueError):
        chroma_b200.ExpertGroup(0, 3, max_pairs=8, hidden=1024, experts=8, exchange=lambda h: [h] * 3)
    group.close()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


def _two_rank_child(rank: int, world: int, port: int, out_dir: str) -> None:
    sys.path.insert(0, str(ROOT))
    os.environ["CHROMA_B200_EP_TIMEOUT_MS"] = "1500"
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    tmp = Path(tempfile.mkdtemp(prefix=f"ep{rank}-"))
    model = ep_model()
    tokens = np.random.default_rng(100 + rank).integers(0, 8192, 64)
    group = chroma_b200.ExpertGroup(rank, world, max_pairs=64 * 2, hidden=1024, experts=8)
    full = chroma_b200.compile_model(model, tmp / "full", steps=64)
    ep = chroma_b200.compile_model(model, tmp / "ep", steps=64, experts=group)
    want = np.asarray(full(tokens))
    dist.barrier()
    results = [np.asarray(ep(tokens)) for _ in range(3)]
    for got in results:
        np.testing.assert_array_equal(got.view(np.uint16), want.view(np.uint16))
    np.testing.assert_array_equal(ep.native.routes(), full.native.routes())
    # Vocab column shard as well: decode through a batched decoder, logits gathered from both ranks' shards.
    vgroup = chroma_b200.ExpertGroup(rank, world, max_pairs=64 * 2, hidden=1024, experts=8, vocab_rows=4, vocab=8192)
    assert len(vgroup.vocab_slice) == 4096
    outs = []
    for experts in (None, vgroup):
        pre = chroma_b200.compile_model(model, tmp / f"vpre{experts is None}", steps=32, context=96, experts=experts)
        dec = chroma_b200.compile_model(model, tmp / f"vdec{experts is None}", steps=1, context=96, experts=experts)
        with chroma_b200.BatchDecoder(pre, dec, 2) as bd:
            seqs = np.stack([tokens[:32], tokens[16:48]])
            if experts is not None:
                dist.barrier()
            logits = np.asarray(bd.append(seqs))
            ids = bd.append(seqs[:, -1:], argmax=True)
            outs.append((logits, ids, bd.generate(ids, 4)))
    helpers.assert_bf16_logits(outs[1][0].astype(np.float32), outs[0][0].astype(np.float32), rel=1e-2)
    np.testing.assert_array_equal(outs[0][1], outs[1][1])
    np.testing.assert_array_equal(outs[0][2], outs[1][2])
    vgroup.close()
    # Failure: rank 1 stays out of the next call (alive, idle at a host barrier); rank 0 must time out cleanly.
    dist.barrier()
    status = "ok"
    if rank == 0:
        try:
            ep(tokens)
            status = "no error"
        except RuntimeError as exc:
            status = "timeout" if "timed out" in str(exc) else f"other: {exc}"
        again = np.asarray(full(tokens))  # the context is still usable
        if not np.array_equal(again.view(np.uint16), want.view(np.uint16)):
            status += " (context damaged)"
    dist.barrier()
    Path(out_dir, f"rank{rank}.txt").write_text(status)
    dist.destroy_process_group()


def test_two_ranks_match_single_gpu_and_time_out_cleanly(gpu: None, tmp_path: Path) -> None:
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs (one process each)")
    import torch.multiprocessing as mp

    mp.start_processes(_two_rank_child, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    assert (tmp_path / "rank0.txt").read_text() == "timeout"
    assert (tmp_path / "rank1.txt").read_text() == "ok"
