"""Our workload definitions reproduce the reference's seeded weights bit for bit (digests recorded from the
reference's own constructors by tests/golden/make_golden.py)."""

from __future__ import annotations

import torch

from tests import helpers
from tests.conftest import golden
from tests.golden.make_golden import digest


def test_dev_model_weights_match_reference_digest() -> None:
    assert digest(helpers.dev_model()) == str(golden("c1_fwd8")["weights_digest"])


def test_small_model_weights_match_reference_digests() -> None:
    g = golden("small")
    assert digest(helpers.cuda_small_model(torch.float32)) == str(g["float32_digest"])
    assert digest(helpers.cuda_small_model(torch.bfloat16)) == str(g["bfloat16_digest"])
    for head_dim in (8, 64):
        assert digest(helpers.decoder_small_model(head_dim)) == str(g[f"dec{head_dim}_digest"])


def test_parameter_count_of_dev_model() -> None:
    assert sum(p.numel() for p in helpers.dev_model().parameters()) == 59_079_408
