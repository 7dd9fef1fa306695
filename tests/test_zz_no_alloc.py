"""The allocation-free vocab projection + greedy argmax entry point (``chroma_b200_vocab_argmax_static``).

Some callers cannot let a library call cudaMalloc: code recorded inside a stream capture that another framework
owns, or hosts that hand the library pre-sized device buffers and keep the allocator to themselves. For them the
entry point keeps its only scratch (one 64-bit argmax key per row) in a static device array of 256 rows. These tests
call it through the C ABI on caller-allocated device buffers and check its logits and argmax ids against the regular
program run (``chroma_b200_run``) on the same rows, twice in a row and on two streams (the scratch is shared and
every call must clear it), over row counts that take each vocab kernel (1, up to 8 rows: register fragments; 9 to
256 fp32 rows: the tiled kernel), for fp32 and bf16 programs, with and without a logits buffer. The file is named to
be collected last.
"""

from __future__ import annotations

import ctypes
import dataclasses
from pathlib import Path

import numpy as np
import pytest
import torch

import chroma_b200
from chroma_b200 import models
from chroma_b200._src import native as nat
from oracle import gpt_oss as og
from tests import helpers

pytestmark = pytest.mark.gpu
VOCAB = 50021


def _ids_ptr(ids: torch.Tensor):  # type: ignore[no-untyped-def]
    return ctypes.cast(ids.data_ptr(), ctypes.POINTER(ctypes.c_int64))


def _static(handle, x: torch.Tensor, rows: int, logits: torch.Tensor | None, ids: torch.Tensor,  # type: ignore[no-untyped-def]
            stream: torch.cuda.Stream | None) -> None:
    nat.call("chroma_b200_vocab_argmax_static", handle, nat._VP(x.data_ptr()), rows,
             None if logits is None else nat._VP(logits.data_ptr()), _ids_ptr(ids),
             nat._VP(0 if stream is None else stream.cuda_stream))


def _check_ids(ids: np.ndarray, want: np.ndarray, rel: float) -> None:
    """Greedy ids equal the program's argmax, except where the program's own top logits lie within ``rel`` of the
    row's largest |logit| (the static call projects the oracle's final rows, which can differ from the program's in
    the last bits)."""
    want = np.asarray(want, np.float64)
    for r, (i, row) in enumerate(zip(ids, want)):
        j = int(np.argmax(row))
        if int(i) != j:
            assert row[int(i)] >= row[j] - rel * np.max(np.abs(row)), f"row {r}: id {int(i)} vs program's {j}"


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("rows", [1, 8, 9, 64, 256])
def test_static_scratch_vocab_argmax_matches_program_run(gpu: None, tmp_path: Path, rows: int, dtype: str) -> None:
    config = dataclasses.replace(models.dev, num_hidden_layers=2, vocab_size=VOCAB)
    tdtype = torch.float32 if dtype == "float32" else torch.bfloat16
    model = models.random_transformer(config, seed=3, std=0.05, dtype=tdtype)
    tokens = np.random.default_rng(rows).integers(0, VOCAB, rows).astype(np.int64)
    with chroma_b200.compile_model(model, tmp_path / "fwd", steps=rows) as program:
        want = np.asarray(program(tokens)).astype(np.float32)  # the existing entry point
        x = torch.from_numpy(og.final_rows(og.Config.from_model_config(config), og.Params.from_module(model),
                                           tokens)).cuda()
        handle = program.native.handle
        side = torch.cuda.Stream()
        # Two calls in a row on the legacy stream, then one on another stream: each must clear the shared keys.
        for stream in (None, None, side):
            out = torch.full((rows, VOCAB), float("nan"), dtype=tdtype, device="cuda")
            ids = torch.full((rows,), -1, dtype=torch.int64, device="cuda")
            _static(handle, x, rows, out, ids, stream)
            torch.cuda.synchronize()
            got = out.float().cpu().numpy()
            if dtype == "float32":
                np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-5)
                _check_ids(ids.cpu().numpy(), want, 1e-5)
            else:
                helpers.assert_bf16_logits(got, want)
                _check_ids(ids.cpu().numpy(), want, 1e-2)
            # The ids are the argmax of the call's own logits (lowest index on ties).
            np.testing.assert_array_equal(ids.cpu().numpy(), np.argmax(got, axis=-1))
        # Without a logits buffer: ids only, the same as with one.
        ids2 = torch.full((rows,), -1, dtype=torch.int64, device="cuda")
        _static(handle, x, rows, None, ids2, side)
        side.synchronize()
        np.testing.assert_array_equal(ids2.cpu().numpy(), ids.cpu().numpy())


def test_static_scratch_rejects_oversized_and_sharded_calls(gpu: None, tmp_path: Path) -> None:
    config = dataclasses.replace(models.dev, num_hidden_layers=1, vocab_size=VOCAB)
    model = models.random_transformer(config, seed=3, std=0.05)
    x = torch.zeros(257, 128, device="cuda")
    ids = torch.zeros(257, dtype=torch.int64, device="cuda")
    with chroma_b200.compile_model(model, tmp_path / "fwd", steps=8) as program:
        with pytest.raises(ValueError, match="static argmax scratch"):
            _static(program.native.handle, x, 257, None, ids, None)
        with pytest.raises(ValueError, match="static argmax scratch"):
            _static(program.native.handle, x, 0, None, ids, None)
    # A vocab-sharded expert-parallel program holds only its rank's unembedding rows: refused before any launch.
    ep_config = dataclasses.replace(models.gpt_oss_20b, num_hidden_layers=1, hidden_size=1024, intermediate_size=1024,
                                    num_attention_heads=16, num_key_value_heads=2, num_experts=8, experts_per_token=2,
                                    vocab_size=8192)
    big = models.random_transformer(ep_config, seed=31, std=0.02, dtype=torch.bfloat16)
    group = chroma_b200.ExpertGroup(0, 1, max_pairs=16, hidden=1024, experts=8, vocab_rows=8, vocab=8192,
                                    exchange=lambda h: [h])
    xs = torch.zeros(8, 1024, device="cuda")
    with chroma_b200.compile_model(big, tmp_path / "ep", steps=8, experts=group) as program:
        with pytest.raises(ValueError, match="vocab-sharded"):
            _static(program.native.handle, xs, 8, None, ids, None)
    group.close()
