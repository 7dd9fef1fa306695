"""The algorithmic bytes bench.py's roofline lines divide by (no GPU): the dev decode step's layers and the whole
step against the workload table's per-step figure (about 115 MB at batch 1: the 102.96 MB vocab matrix plus twelve
layers of attention weights, four routed experts and the 256-row cache)."""

from __future__ import annotations

import bench
from chroma_b200 import models


def test_decode_layer_bytes_counts_every_weight_the_step_reads() -> None:
    cfg = models.dev
    per_layer_static = 4 * (128 + 8 + 160 * 128 + 160 + 128 * 128 + 128 + 128 + 12 * 128 + 12)
    per_layer_experts = 4 * 4 * (256 * 128 + 256 + 128 * 128 + 128)
    per_layer_cache = 4 * (2 * 256 * 16 + 2 * 16)
    want = 12 * (per_layer_static + per_layer_experts + per_layer_cache) + 4 * 3 * 128
    assert bench.decode_layer_bytes(cfg, 256) == want == 11_777_472


def test_whole_step_matches_the_workload_table() -> None:
    vocab = models.dev.vocab_size * models.dev.hidden_size * 4 + models.dev.vocab_size * 4 + models.dev.hidden_size * 4
    step = bench.decode_layer_bytes(models.dev, 256) + vocab
    assert 114e6 < step < 117e6
