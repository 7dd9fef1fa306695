"""Exact ties, NaN and infinities in the MoE router's top-k and in the fused greedy vocab argmax, on the GPU.

The ranking rule is the reference's (chroma/_src/codegen/gpu.py:300-337 for the CUDA top-k; the CPU top-k's
comparator at chroma/_src/codegen/cpu/kernels.h:153-185 ranks NaN the same way): NaN ranks above every number,
+inf above every finite value, and among equal values the lowest index wins; the k selected experts come out
sorted. The reference's CPU top-k leaves the order of exactly tied values unspecified (docs/runtime.md, "Tied
top-k values"); its GPU backend and this one pick the lowest index, as ``oracle.gpt_oss.topk`` does. The greedy id
of a logits row follows ``np.argmax``: the first NaN if any, else the first maximum.

Inputs are crafted so the tied values are bit-identical in every implementation: router rows with zero weights
and equal biases (the gate logit is exactly the bias), duplicated gate rows (identical dot products), and a final
norm whose scale keeps one coordinate, so each logit is one product ``W[v, c] * x[c]``.

Paths: the per-slot MoE kernels (8 tokens), the expert-grouped kernels (48 tokens), the one-launch cluster decode
(batch-1 decode steps), the large-width fused router (few tokens) and tensor-core gate GEMM + top-k (many tokens);
for the argmax the register-fragment vocab GEMV (1-4 rows), the tiled fp32 vocab kernel (16 rows), the bf16 GEMV
(under 16 rows) and the tensor-core GEMM's argmax epilogue (16+ rows).
"""

from __future__ import annotations

import dataclasses
from pathlib import Path

import numpy as np
import pytest
import torch

import chroma_b200
from chroma_b200 import models
from oracle import gpt_oss as og
from tests import helpers

pytestmark = pytest.mark.gpu
FP32 = {"rtol": 1e-4, "atol": 1e-5}
VOCAB = 4096


def dev_config():  # type: ignore[no-untyped-def]
    return dataclasses.replace(models.dev, num_hidden_layers=2, vocab_size=VOCAB)


def wide_config():  # type: ignore[no-untyped-def]
    return dataclasses.replace(models.gpt_oss_20b, num_hidden_layers=2, hidden_size=1024, intermediate_size=1024,
                               num_attention_heads=16, num_key_value_heads=2, num_experts=8, experts_per_token=2,
                               vocab_size=VOCAB, sliding_window=0)


def oracle(model):  # type: ignore[no-untyped-def]
    return og.Config.from_model_config(model.config), og.Params.from_module(model)


def set_router(model, layer: int, bias: list[float], zero_weights: bool = True) -> None:  # type: ignore[no-untyped-def]
    gate = model.block[layer].mlp.gate
    with torch.no_grad():
        if zero_weights:
            gate.weight.zero_()
        gate.bias.copy_(torch.tensor(bias, dtype=torch.float32).to(gate.bias.dtype))


def duplicate_gate_rows(model, layer: int, pairs: list[tuple[int, int]]) -> None:  # type: ignore[no-untyped-def]
    gate = model.block[layer].mlp.gate
    with torch.no_grad():
        for a, b in pairs:
            gate.weight[b].copy_(gate.weight[a])
            gate.bias[b].copy_(gate.bias[a])


def routes_of(model, tokens: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:  # type: ignore[no-untyped-def]
    trace = og.Trace()
    logits = og.forward(*oracle(model), tokens, trace)
    return np.stack(trace.routes), np.stack(trace.gates), logits


def assert_same_nans(got: np.ndarray, want: np.ndarray) -> None:
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    np.testing.assert_array_equal(np.isnan(got), np.isnan(want))


@pytest.mark.parametrize("tokens", [8, 48])
def test_dev_router_ties_nan_and_inf(gpu: None, tmp_path: Path, tokens: int) -> None:
    ids = np.random.default_rng(tokens).integers(0, VOCAB, tokens)
    # Layer 0: zero weights, biases tied at the top (2, 5, 7) and at the boundary (0, 1, 3, 4, 8): the route of
    # every token is [2, 5, 7, 0]. Layer 1: random rows with two duplicated pairs (ties wherever x puts them).
    model = models.random_transformer(dev_config(), seed=4, std=0.05)
    set_router(model, 0, [0.5, 0.5, 3, 0.5, 0.5, 3, 0, 3, 0.5, 0, 0, 0])
    duplicate_gate_rows(model, 1, [(1, 6), (4, 10)])
    want_routes, gates, want = routes_of(model, ids)
    assert np.all(want_routes[0] == [2, 5, 7, 0])
    with chroma_b200.compile_model(model, tmp_path / "ties", steps=tokens) as program:
        got = program(ids)
        np.testing.assert_array_equal(program.native.routes(), want_routes)
    np.testing.assert_allclose(got, want, **FP32)
    # Layer 1 (last): NaN at expert 9, +inf at 4, -inf at 2 (the largest finite otherwise): every token routes
    # [9, 4, ...] and its MoE output, hence every logit, is NaN (softmax over a NaN / an infinite value).
    bias = (np.arange(12, dtype=np.float32) * 0.25).tolist()
    bias[9], bias[4], bias[2], bias[11] = float("nan"), float("inf"), float("-inf"), 50.0
    set_router(model, 1, bias, zero_weights=False)
    want_routes, _, want = routes_of(model, ids)
    assert np.all(want_routes[1][:, :3] == [9, 4, 11])
    with chroma_b200.compile_model(model, tmp_path / "nan", steps=tokens) as program:
        got = program(ids)
        np.testing.assert_array_equal(program.native.routes(), want_routes)
    assert np.isnan(got).all() and np.isnan(want).all()


def test_wide_bf16_router_ties_nan_and_inf(gpu: None, tmp_path: Path) -> None:
    """The large-width path: the fused router for few tokens, the tensor-core gate GEMM + top-k for many."""
    for tokens in (8, 64):
        ids = np.random.default_rng(100 + tokens).integers(0, VOCAB, tokens)
        model = models.random_transformer(wide_config(), seed=6, std=0.02, dtype=torch.bfloat16)
        set_router(model, 0, [0.5, 3, 0.5, 3, 0.5, 0.5, 0.0, 0.5])  # route [1, 3] for every token
        want_routes, _, want = routes_of(model, ids)
        assert np.all(want_routes[0] == [1, 3])
        with chroma_b200.compile_model(model, tmp_path / f"w{tokens}", steps=tokens) as program:
            got = program(ids)
            np.testing.assert_array_equal(program.native.routes()[0], want_routes[0])
        helpers.assert_bf16_logits(np.asarray(got, np.float32), np.asarray(want, np.float32))
        set_router(model, 1, [0.5, float("inf"), 2.0, float("nan"), float("-inf"), 0.5, 0.5, 0.5], zero_weights=True)
        want_routes, _, want = routes_of(model, ids)
        assert np.all(want_routes[1] == [3, 1])
        with chroma_b200.compile_model(model, tmp_path / f"wn{tokens}", steps=tokens) as program:
            got = np.asarray(program(ids), np.float32)
            np.testing.assert_array_equal(program.native.routes(), want_routes)
        assert np.isnan(got).all() and np.isnan(np.asarray(want, np.float32)).all()


def test_cluster_decode_router_ties_nan_and_inf(gpu: None, tmp_path: Path) -> None:
    """Batch-1 fp32 decode steps run every layer in one cluster launch with its own router (orderable keys)."""
    model = models.random_transformer(dev_config(), seed=8, std=0.05)
    set_router(model, 0, [0.5, 0.5, 3, 0.5, 0.5, 3, 0, 3, 0.5, 0, 0, 0])
    duplicate_gate_rows(model, 1, [(1, 6), (4, 10)])
    prompt = np.random.default_rng(9).integers(0, VOCAB, 8)
    steps = np.random.default_rng(10).integers(0, VOCAB, 12)
    pre = chroma_b200.compile_model(model, tmp_path / "pre", steps=8, context=64)
    dec = chroma_b200.compile_model(model, tmp_path / "dec", steps=1, context=64)
    ref = og.Decoder(*oracle(model), 64, 8)
    with chroma_b200.Decoder(pre, dec) as d:
        np.testing.assert_allclose(d.append(prompt), ref.append(prompt), **FP32)
        for t in steps:
            np.testing.assert_allclose(d.append([int(t)]), ref.append([int(t)]), **FP32)
    bias = [0.0] * 12
    bias[9], bias[4] = float("nan"), float("inf")
    set_router(model, 1, bias, zero_weights=False)
    pre = chroma_b200.compile_model(model, tmp_path / "pre2", steps=8, context=64)
    dec = chroma_b200.compile_model(model, tmp_path / "dec2", steps=1, context=64)
    with chroma_b200.BatchDecoder(pre, dec, 1) as bd:
        first = bd.append(prompt[None, :], argmax=True)
        ids = bd.generate(first, 4)
    # Every logit is NaN, so every greedy id is 0 (the lowest-index NaN), as np.argmax picks.
    assert int(first[0]) == 0 and np.all(ids == 0)


# ---- fused greedy argmax --------------------------------------------------------------------------------------
TIE_POS, TIE_NEG = [7, 50, 700], [9, 60, 900]


def craft_vocab(model, kind: str, coord: int = 5) -> None:  # type: ignore[no-untyped-def]
    """Final norm keeps coordinate ``coord`` only; unembedding column ``coord``: uniform(-1, 1) with exact ties at
    +5 (rows TIE_POS) and -5 (rows TIE_NEG), plus +inf/-inf (rows 3000, 3001) and NaN (rows 1200, 2500) by kind."""
    with torch.no_grad():
        model.norm.scale.zero_()
        model.norm.scale[coord] = 1.0
        col = np.random.default_rng(77).uniform(-1, 1, VOCAB).astype(np.float32)
        col[TIE_POS], col[TIE_NEG] = 5.0, -5.0
        if kind in ("inf", "nan"):
            col[3000], col[3001] = np.inf, -np.inf
        if kind == "nan":
            col[[2500, 1200]] = np.nan
        w = model.unembedding.weight
        w[:, coord] = torch.from_numpy(col).to(w.dtype)


def oracle_ids(model, sequences: np.ndarray, steps: np.ndarray) -> np.ndarray:  # type: ignore[no-untyped-def]
    """Greedy ids of each sequence after its prompt and after each forced step: np.argmax of the oracle's logits."""
    out = []
    for seq, forced in zip(sequences, steps):
        dec = og.Decoder(*oracle(model), 64, 8)
        row = [int(np.argmax(dec.append(seq)))]
        row += [int(np.argmax(dec.append([int(t)]))) for t in forced]
        out.append(row)
    return np.array(out)


@pytest.mark.parametrize("kind", ["ties", "inf", "nan"])
@pytest.mark.parametrize("wide", [False, True])
def test_greedy_argmax_ties_nan_and_inf(gpu: None, tmp_path: Path, kind: str, wide: bool) -> None:
    if wide:
        model = models.random_transformer(wide_config(), seed=12, std=0.02, dtype=torch.bfloat16)
        batches = (4, 16)  # bf16 GEMV below 16 rows, the tensor-core GEMM's argmax epilogue from 16
    else:
        model = models.random_transformer(dev_config(), seed=12, std=0.05)
        batches = (1, 4, 16)  # register-fragment GEMV (1, 4 rows), the tiled fp32 kernel (16 rows)
    craft_vocab(model, kind)
    pre = chroma_b200.compile_model(model, tmp_path / "pre", steps=8, context=64)
    dec = chroma_b200.compile_model(model, tmp_path / "dec", steps=1, context=64)
    rng = np.random.default_rng(13)
    for batch in batches:
        prompts = rng.integers(0, VOCAB, (batch, 8))
        forced = rng.integers(0, VOCAB, (batch, 2))
        want = oracle_ids(model, prompts, forced)
        with chroma_b200.BatchDecoder(pre, dec, batch) as bd:
            got = [bd.append(prompts, argmax=True)]
            got += [bd.append(forced[:, i : i + 1], argmax=True) for i in range(forced.shape[1])]
        got = np.stack(got, axis=1)
        np.testing.assert_array_equal(got, want)
        if kind == "ties":
            assert set(np.unique(got)) <= {TIE_POS[0], TIE_NEG[0]}
        elif kind == "inf":
            assert set(np.unique(got)) <= {3000, 3001}
        else:
            assert np.all(got == 1200)
    if not wide:  # batch-1 device generation: the cluster decode + the vocab kernel's keys fed back
        with chroma_b200.BatchDecoder(pre, dec, 1) as bd:
            first = bd.append(prompts[:1], argmax=True)
            ids = bd.generate(first, 3)[0]
        ref = og.Decoder(*oracle(model), 64, 8)
        want = [int(np.argmax(ref.append(prompts[0])))]
        for _ in range(3):
            want.append(int(np.argmax(ref.append([want[-1]]))))
        assert [int(first[0])] + ids.tolist() == want
