"""GPU parity of the large-width bf16 path (tensor-core GEMMs, grouped MoE, flash attention) at GPT-OSS-20B widths.

One layer at full widths (d=2880, 64/8 heads of 64, 32 experts top-4, I=2880) and the full 201,088-entry vocabulary,
against the reference's own compiled CPU program on the same seeded weights (tests/golden/c4_slice.npz) and the
oracle. bf16 bar (tests/helpers.assert_bf16_logits): |diff| <= 2e-2 x the row's largest |logit|, and >= 99 % of
elements within 2e-2 relative / absolute; routing identical except where bf16 gate logits tie exactly at the top-k
boundary (the reference leaves that order unspecified); token ids identical for identically routed tokens.
"""

from __future__ import annotations

import dataclasses
import functools
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch

import chroma_b200
from chroma_b200 import models
from oracle import gpt_oss as og
from tests import helpers
from tests.conftest import golden

pytestmark = pytest.mark.gpu
_TMP = Path(tempfile.mkdtemp(prefix="chroma-b200-large-"))


def c4_config():  # type: ignore[no-untyped-def]
    return dataclasses.replace(models.gpt_oss_20b, num_hidden_layers=1)


@functools.lru_cache(maxsize=None)
def c4_model():  # type: ignore[no-untyped-def]
    return models.random_transformer(c4_config(), seed=11, std=0.02, dtype=torch.bfloat16)


def test_c4_slice_forward_matches_reference(gpu: None) -> None:
    g = golden("c4_slice")
    with chroma_b200.compile_model(c4_model(), _TMP / "c4fwd", steps=16) as program:
        assert program.stats["tensor_core_path"]
        logits = np.asarray(program(g["tokens"]), np.float32)
        routes = program.native.routes()
    ok = helpers.routes_match(routes, g["routes"], g["oracle_gates"], 4)
    assert ok.all(), np.argwhere(~ok)
    same = np.all(routes == g["routes"], axis=-1).all(axis=0)
    assert same.sum() >= 14
    helpers.assert_bf16_logits(logits[same][:, g["sample_cols"]], g["sample"][same])
    np.testing.assert_array_equal(np.argmax(logits, -1)[same], g["argmax"][same])


def test_c4_slice_prefill_and_decode_match_oracle(gpu: None) -> None:
    model = c4_model()
    tokens = np.random.default_rng(12).integers(0, 201088, 19)
    prefill = chroma_b200.compile_model(model, _TMP / "c4pre", steps=16, context=32)
    decode = chroma_b200.compile_model(model, _TMP / "c4dec", steps=1, context=32)
    with chroma_b200.Decoder(prefill, decode) as dec:
        outs = [dec.append(tokens[:16])] + [dec.append([int(t)]) for t in tokens[16:]]
    cfg, p = og.Config.from_model_config(c4_config()), og.Params.from_module(model)
    ref = og.Decoder(cfg, p, context=32, prefill_steps=16)
    want = [ref.append(tokens[:16])] + [ref.append([int(t)]) for t in tokens[16:]]
    for got, exp in zip(outs, want):
        helpers.assert_bf16_logits(np.asarray(got, np.float32), exp)
        assert int(np.argmax(got)) == int(np.argmax(exp))


def test_flash_prefill_chunks_cache_and_window_match_oracle(gpu: None) -> None:
    """Long prefill chunks through the flash kernel (the tcgen05 one by default): several 256-row query blocks, own key
    tiles below the diagonal (mask-free), a second chunk that reads live ring-cache tiles, a windowed layer (layer 0, window 160), decode
    steps in between and the ring wrapping. Steps whose oracle routing has a near-tie at the top-k boundary in some
    layer for the row whose logits are returned (helpers.near_tie) are held to the greedy token only."""
    cfg = dataclasses.replace(models.gpt_oss_20b, num_hidden_layers=2, hidden_size=1024, intermediate_size=1024,
                              num_attention_heads=16, num_key_value_heads=2, num_experts=8, experts_per_token=2,
                              vocab_size=8192, sliding_window=160)
    model = models.random_transformer(cfg, seed=21, std=0.02, dtype=torch.bfloat16)
    tokens = np.random.default_rng(22).integers(0, cfg.vocab_size, 780)
    chunks = [700, 1, 1, 1, 1, 76]
    prefill = chroma_b200.compile_model(model, _TMP / "flpre", steps=384, context=640)
    decode = chroma_b200.compile_model(model, _TMP / "fldec", steps=1, context=640)
    assert prefill.stats["tensor_core_path"]
    ref = og.Decoder(og.Config.from_model_config(cfg), og.Params.from_module(model), context=640, prefill_steps=384,
                     sliding_window=160)
    strict = 0
    with chroma_b200.Decoder(prefill, decode, sliding_window=160) as dec:
        offset = 0
        for size in chunks:
            part = tokens[offset : offset + size]
            offset += size
            got = np.asarray(dec.append(part), np.float32)
            trace = og.Trace()
            want = ref.append(part, trace)
            helpers.assert_greedy_token(got, want)
            last = size - 1 - 384 * ((size - 1) // 384) if size > 1 else 0  # last real row of the final chunk
            if not any(helpers.near_tie(g[last], cfg.experts_per_token).any() for g in trace.gates[-2:]):
                helpers.assert_bf16_logits(got, want)
                strict += 1
    assert strict >= 4


def test_128_expert_routing_matches_oracle(gpu: None, record_property) -> None:  # type: ignore[no-untyped-def]
    """C5's routing shape (128 experts, top-4) at reduced widths, a 16-token forward against the oracle. The tensor
    cores sum the gate GEMM in another order than the reference's sequential fp32 loops, so bf16 gate logits within a
    few ulps of the top-4 boundary may rank the other way. Stated bound: every routing whose oracle margin between
    the 4th and 5th gate logit exceeds 1/64 relative (4 bf16 ulps) must match exactly, layer by layer for tokens
    routed identically so far (helpers.route_agreement); the mismatch count and margins are recorded. Tokens routed
    identically in every layer are held to the bf16 logits bar and the greedy token."""
    cfg = dataclasses.replace(models.gpt_oss_120b, num_hidden_layers=2, hidden_size=1024, intermediate_size=1024,
                              num_attention_heads=16, num_key_value_heads=2, vocab_size=8192)
    assert cfg.num_experts == 128 and cfg.experts_per_token == 4
    model = models.random_transformer(cfg, seed=41, std=0.02, dtype=torch.bfloat16)
    tokens = np.random.default_rng(42).integers(0, cfg.vocab_size, 16)
    with chroma_b200.compile_model(model, _TMP / "e128fwd", steps=16) as program:
        assert program.stats["tensor_core_path"]
        logits = np.asarray(program(tokens), np.float32)
        routes = program.native.routes()
    trace = og.Trace()
    want = og.forward(og.Config.from_model_config(cfg), og.Params.from_module(model), tokens, trace)
    ref_routes, gates = np.stack(trace.routes), np.stack(trace.gates)
    stats = helpers.route_agreement(routes, ref_routes, gates, 4)
    record_property("route_mismatches", f"{stats['mismatched']} of {stats['compared']} (layer, token) routings, "
                                        f"oracle margins {['%.2e' % m for m in stats['margins']]}")
    # A mismatch needs a near-tie at the boundary: no more of them than compared routings with such a margin.
    near = sum(int(helpers.near_tie(gates[layer], 4).sum()) for layer in range(gates.shape[0]))
    assert stats["mismatched"] <= near, (stats, near)
    exact = stats["identical_tokens"]
    assert exact.any()
    helpers.assert_bf16_logits(logits[exact], want[exact])
    np.testing.assert_array_equal(np.argmax(logits[exact], -1), np.argmax(want[exact], -1))


def test_mma_sync_flash_kernel_matches_oracle(gpu: None) -> None:
    """The mma.sync flash-attention kernel (CHROMA_B200_FLASH_TC=0; the tcgen05 kernel is the default) through the
    same long-chunk case, in a subprocess so the switch is read fresh."""
    import os
    import subprocess
    import sys

    code = "import tests.test_gpu_large as t; t.test_flash_prefill_chunks_cache_and_window_match_oracle(None)"
    env = dict(os.environ, CHROMA_B200_FLASH_TC="0")
    subprocess.run([sys.executable, "-c", code], check=True, env=env, cwd=str(Path(__file__).resolve().parents[1]))


def _rope_case(fwd: str, pre: str, dec: str, tokens_path: str, out: str) -> None:
    """Forward of 512 tokens (logits of every row, routes, launch count) and a 512-token prefill + 3 decode steps
    through the programs at the given paths; results saved to `out`."""
    tokens = np.load(tokens_path)
    with chroma_b200.Program(fwd) as p:
        logits = np.asarray(p(tokens[:512]), np.float32)
        routes = p.native.routes()
        launches = p.native.launches
    with chroma_b200.Decoder(chroma_b200.Program(pre), chroma_b200.Program(dec)) as d:
        steps = [np.asarray(d.append(tokens[:512]), np.float32)]
        steps += [np.asarray(d.append([int(t)]), np.float32) for t in tokens[512:]]
    np.savez(out, logits=logits, routes=routes, steps=np.concatenate(steps), launches=launches)


def test_rope_epilogue_matches_separate_kernel(gpu: None) -> None:
    """RoPE in the QKV GEMM's epilogue (the default where that GEMM has no split-K: here 512 tokens at C4's attention
    widths, 64 / 8 heads of 64, d = 2,880) against the separate k_rope_split kernel (CHROMA_B200_ROPE_EPILOGUE=0, in
    a subprocess so the switch is read fresh). The forward's logits of every row and its routes, and a cached prefill
    (q, new K and V rows into the cache) followed by decode steps that read those rows, are bit-identical; the
    forward launches one kernel less per layer after the first (one (cos, sin) table per forward)."""
    import os
    import subprocess
    import sys

    cfg = dataclasses.replace(models.gpt_oss_20b, num_hidden_layers=2, num_experts=8, intermediate_size=1024,
                              vocab_size=8192)
    model = models.random_transformer(cfg, seed=31, std=0.02, dtype=torch.bfloat16)
    tokens = np.random.default_rng(32).integers(0, cfg.vocab_size, 515)
    paths = [str(_TMP / name) for name in ("ropefwd", "ropepre", "ropedec")]
    for path, kw in zip(paths, ({"steps": 512}, {"steps": 512, "context": 520}, {"steps": 1, "context": 520})):
        with chroma_b200.compile_model(model, path, **kw) as p:
            assert p.stats["tensor_core_path"]
    np.save(_TMP / "rope_tokens.npy", tokens)
    root = str(Path(__file__).resolve().parents[1])
    results = {}
    for mode in ("1", "0"):
        out = str(_TMP / f"rope{mode}.npz")
        code = "import sys, tests.test_gpu_large as t; t._rope_case(*sys.argv[1:])"
        env = dict(os.environ, CHROMA_B200_ROPE_EPILOGUE=mode, PYTHONPATH=root)
        subprocess.run([sys.executable, "-c", code, *paths, str(_TMP / "rope_tokens.npy"), out], check=True, env=env,
                       cwd=root)
        results[mode] = np.load(out)
    fused, separate = results["1"], results["0"]
    for key in ("logits", "steps"):
        np.testing.assert_array_equal(fused[key].view(np.uint32), separate[key].view(np.uint32))
    np.testing.assert_array_equal(fused["routes"], separate["routes"])
    assert int(fused["launches"]) == int(separate["launches"]) - (cfg.num_hidden_layers - 1)
