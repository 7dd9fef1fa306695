"""The allocation-free vocab projection + greedy argmax entry point (``chroma_b200_vocab_argmax_static``).

Some callers cannot let a library call cudaMalloc: code recorded inside a stream capture that another framework
owns, or hosts that hand the library pre-sized device buffers and keep the allocator to themselves. For them the
entry point keeps its only scratch (one 64-bit argmax key per row) in a static device array. This test calls it
through the C ABI on caller-allocated device buffers and checks its logits and argmax ids against the regular
program run (``chroma_b200_run``) on the same rows, twice in a row (the scratch is shared and must be cleared by
every call). The file is named to be collected last.
"""

from __future__ import annotations

import ctypes
import dataclasses
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch

import chroma_b200
from chroma_b200 import models
from chroma_b200._src import native as nat
from oracle import gpt_oss as og

pytestmark = pytest.mark.gpu


def test_static_scratch_vocab_argmax_matches_program_run(gpu: None) -> None:
    config = dataclasses.replace(models.dev, num_hidden_layers=2, vocab_size=50021)
    model = models.random_transformer(config, seed=3, std=0.05)
    tokens = np.array([5, 17, 50020, 0, 9, 1000, 3, 2], dtype=np.int64)
    with tempfile.TemporaryDirectory() as tmp, chroma_b200.compile_model(model, Path(tmp) / "fwd", steps=8) as program:
        logits = program(tokens)  # the existing entry point
        rows = og.final_rows(og.Config.from_model_config(config), og.Params.from_module(model), tokens)
        x = torch.from_numpy(rows).cuda()
        handle = program.native.handle
        for _ in range(2):
            out = torch.full((8, config.vocab_size), float("nan"), device="cuda")
            ids = torch.full((8,), -1, dtype=torch.int64, device="cuda")
            nat.call("chroma_b200_vocab_argmax_static", handle, nat._VP(x.data_ptr()), 8, nat._VP(out.data_ptr()),
                     ctypes.cast(ids.data_ptr(), ctypes.POINTER(ctypes.c_int64)), nat._VP(0))
            torch.cuda.synchronize()
            np.testing.assert_allclose(out.cpu().numpy(), logits, rtol=1e-4, atol=1e-5)
            np.testing.assert_array_equal(ids.cpu().numpy(), np.argmax(logits, axis=-1))
        with pytest.raises(ValueError, match="static argmax scratch"):
            nat.call("chroma_b200_vocab_argmax_static", handle, nat._VP(x.data_ptr()), 257, None,
                     ctypes.cast(ids.data_ptr(), ctypes.POINTER(ctypes.c_int64)), nat._VP(0))
