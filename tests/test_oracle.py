"""Pin the NumPy oracle to the reference: golden vectors come from the reference's own compiled CPU programs.

Tolerances: fp32 logits rtol 2e-5 / atol 2e-6 (the reference's own CPU-vs-Torch bar, tests/test_runtime.py:32);
bf16 rtol 2e-2 / atol 1e-2. Argmax ids and routing indices must be identical.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import gpt_oss as og
from tests import helpers
from tests.conftest import golden


def test_c1_forward_logits_argmax_and_routing() -> None:
    g = golden("c1_fwd8")
    cfg, p = helpers.dev_oracle()
    for s, tokens in enumerate(g["tokens"]):
        trace = og.Trace()
        logits = og.forward(cfg, p, tokens, trace)
        np.testing.assert_array_equal(np.argmax(logits, -1), g["argmax"][s])
        np.testing.assert_array_equal(np.stack(trace.routes), g["routes"][s])
        np.testing.assert_allclose(logits[:, g["sample_cols"]], g["sample"][s], rtol=2e-5, atol=2e-6)
        np.testing.assert_allclose(logits.astype(np.float64).sum(-1), g["rowsum"][s], rtol=1e-4, atol=1e-3)


def test_c2_decoder_prefill_and_steps() -> None:
    g = golden("c2_decode")
    cfg, p = helpers.dev_oracle()
    dec = og.Decoder(cfg, p, context=256, prefill_steps=8)
    outs = [dec.append(g["prompt"])] + [dec.append([int(t)]) for t in g["forced"]]
    for i, out in enumerate(outs):
        assert int(np.argmax(out)) == int(g["step_argmax"][i][0])
        np.testing.assert_allclose(out[:, g["sample_cols"]], g["step_sample"][i], rtol=2e-5, atol=2e-6)


def test_c2_decoder_ring_wrap_argmax() -> None:
    g = golden("c2_decode")
    cfg, p = helpers.dev_oracle()
    dec = og.Decoder(cfg, p, context=256, prefill_steps=8)
    tokens = g["long_tokens"]
    ids = [int(np.argmax(dec.append(tokens[:8])))]
    last = None
    for t in tokens[8:]:
        last = dec.append([int(t)])
        ids.append(int(np.argmax(last)))
    np.testing.assert_array_equal(ids, g["long_argmax"])
    np.testing.assert_allclose(last[:, g["sample_cols"]], g["tail_sample"][-1], rtol=2e-5, atol=2e-6)


def test_c3_micrograph_bits() -> None:
    g = golden("c3_micro")
    x = og.from_bf16_bits(g["x16"])
    gen = torch.Generator().manual_seed(0)
    ins = [torch.randn(16, 4096, generator=gen).to(torch.bfloat16).view(torch.uint16).numpy() for _ in range(3)]
    np.testing.assert_array_equal(ins[0], g["x16"])
    out = og.micro(*(og.from_bf16_bits(b) for b in ins), g["w"])
    want = og.from_bf16_bits(g["out16"])
    exact = np.mean(og.bf16_bits(out) == g["out16"])
    assert exact > 0.999, exact
    np.testing.assert_allclose(out, want, rtol=2e-2, atol=1e-2)
    assert x.shape == (16, 4096)


def test_small_models_full_and_decoder() -> None:
    g = golden("small")
    for dtype, rtol, atol in ((torch.float32, 2e-5, 2e-6), (torch.bfloat16, 2e-2, 1e-2)):
        name = str(dtype).split(".")[1]
        model = helpers.cuda_small_model(dtype)
        cfg = og.Config.from_model_config(helpers.small_config("cuda_small"))
        p = og.Params.from_module(model)
        for tokens, want in zip(g[f"{name}_full4_tokens"], g[f"{name}_full4"]):
            np.testing.assert_allclose(og.forward(cfg, p, tokens), want, rtol=rtol, atol=atol)
        dec = og.Decoder(cfg, p, context=5, prefill_steps=5, sliding_window=3)
        tokens = (np.arange(14) * 7 + 3) % 17
        logs, pos = [], 0
        for size in (2, 1, 4, 5, 2):
            logs.append(dec.append(tokens[pos : pos + size]))
            pos += size
        dec = og.Decoder(cfg, p, context=5, prefill_steps=5, sliding_window=3)
        logs.append(dec.append(tokens))
        np.testing.assert_allclose(np.concatenate(logs), g[f"{name}_decoder"], rtol=rtol, atol=atol)
    for head_dim in (8, 64):
        model = helpers.decoder_small_model(head_dim)
        cfg = og.Config.from_model_config(helpers.small_config(f"decoder_small_{head_dim}"))
        p = og.Params.from_module(model)
        tokens = (np.arange(23) * 7 + 3) % 31
        logs, pos = [], 0
        dec = og.Decoder(cfg, p, context=7, prefill_steps=7, sliding_window=3)
        for size in (3, 1, 5, 7, 1, 6):
            logs.append(dec.append(tokens[pos : pos + size]))
            pos += size
        logs.append(og.Decoder(cfg, p, context=7, prefill_steps=7, sliding_window=3).append(tokens))
        logs.append(og.Decoder(cfg, p, context=7, prefill_steps=7, sliding_window=3).append(tokens[:3]))
        np.testing.assert_allclose(np.concatenate(logs), g[f"dec{head_dim}_decoder"], rtol=2e-5, atol=2e-6)


def test_bf16_rounding_known_answers() -> None:
    # Ties to even, NaN canonicalised, infinities kept (reference tests/runtime_core.cc:26-35 table's cases).
    x = np.array([1 + 2**-8, 1 + 3 * 2**-8, -1 - 2**-8, -1 - 3 * 2**-8, np.inf, -np.inf, 0.0, -0.0], np.float32)
    np.testing.assert_array_equal(og.bf16_round(x), np.array([1, 1 + 2**-6, -1, -1 - 2**-6, np.inf, -np.inf, 0, -0.0], np.float32))
    assert og.bf16_bits(np.array([np.nan], np.float32))[0] == 0x7FC0


def test_c4_slice_forward_logits_and_routing() -> None:
    """The oracle at GPT-OSS-20B widths (one layer, bf16) against the reference's compiled CPU program."""
    import dataclasses

    from chroma_b200 import models

    g = golden("c4_slice")
    config = dataclasses.replace(models.gpt_oss_20b, num_hidden_layers=1)
    model = models.random_transformer(config, seed=11, std=0.02, dtype=torch.bfloat16)
    from tests.golden.make_golden import digest

    assert digest(model) == str(g["weights_digest"])
    trace = og.Trace()
    logits = og.forward(og.Config.from_model_config(config), og.Params.from_module(model), g["tokens"], trace)
    ours = np.stack(trace.routes)
    ok = helpers.routes_match(ours, g["routes"], g["oracle_gates"], 4)
    assert ok.all(), np.argwhere(~ok)
    # Tokens routed identically must also agree on logits; a tie broken differently changes that token's expert.
    same = np.all(ours == g["routes"], axis=-1).all(axis=0)
    assert same.sum() >= 14
    np.testing.assert_array_equal(np.argmax(logits, -1)[same], g["argmax"][same])
    np.testing.assert_allclose(logits[same][:, g["sample_cols"]], g["sample"][same], rtol=2e-2, atol=2e-2)
