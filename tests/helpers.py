"""Shared test helpers: seeded models, oracle parameters, comparison utilities."""

from __future__ import annotations

import dataclasses
import functools

import numpy as np

from oracle import gpt_oss as og


@functools.lru_cache(maxsize=None)
def dev_model():  # type: ignore[no-untyped-def]
    from chroma_b200.models import make_dev_model

    return make_dev_model(0)


@functools.lru_cache(maxsize=None)
def dev_oracle() -> tuple[og.Config, og.Params]:
    from chroma_b200.models import dev

    return og.Config.from_model_config(dev), og.Params.from_module(dev_model())


def small_config(kind: str):  # type: ignore[no-untyped-def]
    """The reference tests' small configurations (tests/test_cuda.py:29-43, tests/test_decoder.py:21-37)."""
    from chroma_b200.models import dev

    if kind == "cuda_small":
        return dataclasses.replace(dev, num_hidden_layers=1, num_experts=2, experts_per_token=2, vocab_size=17,
                                   hidden_size=8, intermediate_size=8, head_dim=4, num_attention_heads=2,
                                   num_key_value_heads=1, sliding_window=3)
    head_dim = int(kind.rsplit("_", 1)[1])
    return dataclasses.replace(dev, num_hidden_layers=2, hidden_size=16, intermediate_size=16, vocab_size=31,
                               num_experts=4, experts_per_token=2, num_attention_heads=4, num_key_value_heads=2,
                               head_dim=head_dim, sliding_window=3, initial_context_length=4096,
                               rope_scaling_factor=32.0 if head_dim == 64 else 1.0)


def cuda_small_model(dtype):  # type: ignore[no-untyped-def]
    """Seed 5, N(0, 0.1), cast before init (tests/test_cuda.py:29-43)."""
    import torch

    from chroma_b200.models import Transformer, init_weights

    with torch.random.fork_rng(devices=[]):
        torch.manual_seed(5)
        model = Transformer(small_config("cuda_small")).to(dtype).eval()
        return init_weights(model, std=0.1, zero_bias=False)


def decoder_small_model(head_dim: int):  # type: ignore[no-untyped-def]
    from chroma_b200.models import random_transformer

    return random_transformer(small_config(f"decoder_small_{head_dim}"), seed=5, std=0.03)


def assert_logits(actual: np.ndarray, expected: np.ndarray, *, rtol: float, atol: float) -> None:
    np.testing.assert_allclose(np.asarray(actual, np.float32), np.asarray(expected, np.float32), rtol=rtol, atol=atol)


def summary(logits: np.ndarray, cols: np.ndarray) -> dict[str, np.ndarray]:
    logits = np.asarray(logits, np.float32).reshape(-1, logits.shape[-1])
    return {"argmax": np.argmax(logits, -1), "sample": logits[:, cols], "rowsum": logits.astype(np.float64).sum(-1)}


def routes_match(ours: np.ndarray, ref: np.ndarray, gates: np.ndarray, k: int) -> np.ndarray:
    """Per (layer, token): True when the routing equals the reference's, or differs only among experts whose bf16
    gate logits tie exactly at the top-k boundary (the reference's tie order is unspecified there)."""
    ok = np.all(ours == ref, axis=-1)
    for idx in zip(*np.nonzero(~ok)):
        g = gates[idx]
        kth = np.sort(g)[::-1][k - 1]
        above = set(np.nonzero(g > kth)[0].tolist())
        tied = set(np.nonzero(g == kth)[0].tolist())
        a, b = set(ours[idx].tolist()), set(ref[idx].tolist())
        ok[idx] = above <= a and above <= b and (a - above) <= tied and (b - above) <= tied and len(tied) > k - len(above)
    return ok


def routes_match_near(ours: np.ndarray, ref: np.ndarray, gates: np.ndarray, k: int, rel: float = 1 / 64) -> np.ndarray:
    """Per (layer, token): True when the routing equals the reference's, or differs only among experts whose gate
    logits lie within ``rel`` (relative) of the k-th largest: near-ties that the accumulation order of earlier GEMMs
    decides (see ``near_tie``). Experts clearly above the boundary must be selected by both."""
    ok = np.all(ours == ref, axis=-1)
    for idx in zip(*np.nonzero(~ok)):
        g = np.asarray(gates[idx], np.float64)
        kth = np.sort(g)[::-1][k - 1]
        tol = rel * max(abs(kth), 1e-6)
        a, b = set(ours[idx].tolist()), set(ref[idx].tolist())
        clear = set(np.nonzero(g > kth + tol)[0].tolist())
        ok[idx] = clear <= a and clear <= b and all(abs(g[e] - kth) <= tol for e in a ^ b)
    return ok


def assert_bf16_logits(got: np.ndarray, want: np.ndarray, rel: float = 2e-2, elementwise_share: float = 0.99) -> None:
    """bf16 logits bar: every |got - want| <= rel * (largest |want| of its row), and at least `elementwise_share` of
    the elements also within rel relative / rel absolute. Elementwise relative error alone is ill-conditioned for
    logits near zero after thousands of bf16-rounded accumulations."""
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    scale = np.max(np.abs(want), axis=-1, keepdims=True)
    worst = float(np.max(np.abs(got - want) / scale))
    assert worst <= rel, f"max |diff| / row scale = {worst:.4g} > {rel}"
    close = np.abs(got - want) <= rel + rel * np.abs(want)
    assert close.mean() >= elementwise_share, f"only {close.mean():.4%} of elements within {rel} rel/abs"


def near_tie(gates: np.ndarray, k: int, rel: float = 1 / 64) -> np.ndarray:
    """Rows whose k-th and (k+1)-th largest gate logits are within ``rel`` (relative) of each other.

    Routing on such rows depends on the last bits of the gate logits, which follow the accumulation order of every
    GEMM before the router; an implementation that sums in another order than the reference's sequential fp32 loops
    (chroma/_src/codegen/cpu/kernels.h:63-74) may pick the other expert there. Comparisons skip or relax those rows.
    """
    g = np.sort(np.asarray(gates, np.float32).reshape(-1, np.asarray(gates).shape[-1]), axis=-1)[:, ::-1]
    if g.shape[-1] <= k:
        return np.zeros(g.shape[0], bool)
    gap = np.abs(g[:, k - 1] - g[:, k])
    return gap <= rel * np.maximum(np.abs(g[:, k - 1]), np.abs(g[:, k]))


def assert_greedy_token(got: np.ndarray, want: np.ndarray, rel: float = 1e-2) -> None:
    """The greedy token of each row equals the reference's, unless the reference's own top logits are within
    ``rel`` x the row's largest |logit| of each other (a bf16 near-tie that summation order decides); then the
    chosen token must be one of those near-top logits."""
    got, want = np.atleast_2d(np.asarray(got, np.float64)), np.atleast_2d(np.asarray(want, np.float64))
    for g, w in zip(got, want):
        a, b = int(np.argmax(g)), int(np.argmax(w))
        if a != b:
            assert w[a] >= w[b] - rel * np.max(np.abs(w)), f"greedy token {a} (ref {w[a]:.5g}) vs {b} (ref {w[b]:.5g})"


def assert_top_and_rowsum(got: np.ndarray, top_idx: np.ndarray, top_val: np.ndarray, rowsum: np.ndarray, *,
                          rtol: float = 1e-4, atol: float = 1e-5) -> None:
    """Full-row checks against a golden summary of the reference's logits (tests/golden/make_golden.py ``summary``):
    the reference's 16 largest logits (``top_idx`` / ``top_val``) within the fp32 bar; our 16 largest in the same
    order, except where two neighbours are within that bar of each other (a near-tie swap); and the float64 row sum
    of all V logits within the bar summed over the row (rtol * sum |logit| + atol * V)."""
    got = np.asarray(got, np.float32).reshape(-1, np.asarray(got).shape[-1])
    top_idx, top_val = np.asarray(top_idx).reshape(got.shape[0], -1), np.asarray(top_val).reshape(got.shape[0], -1)
    rowsum = np.asarray(rowsum).reshape(-1)
    for r, row in enumerate(got):
        np.testing.assert_allclose(row[top_idx[r]], top_val[r], rtol=rtol, atol=atol)
        mine = np.argsort(-row, kind="stable")[: top_idx.shape[1]]
        for j in np.nonzero(mine != top_idx[r])[0]:
            a, b = float(row[mine[j]]), float(row[top_idx[r][j]])
            assert abs(a - b) <= atol + rtol * abs(float(top_val[r][j])), (r, j, int(mine[j]), int(top_idx[r][j]))
        total = float(row.astype(np.float64).sum())
        bound = rtol * float(np.abs(row).astype(np.float64).sum()) + atol * row.size
        assert abs(total - float(rowsum[r])) <= bound, (r, total, float(rowsum[r]), bound)


def route_agreement(ours: np.ndarray, ref: np.ndarray, gates: np.ndarray, k: int, rel: float = 1 / 64) -> dict:
    """Layer-by-layer routing comparison of [layers, tokens, k] routes against the oracle's, with the oracle's gate
    logits [layers, tokens, E]. A token is compared in a layer only while every earlier layer routed it identically
    (after a different choice its hidden state legitimately differs from the oracle's). Every compared (layer,
    token) whose oracle margin between the k-th and (k+1)-th gate logit exceeds ``rel`` (relative) must be routed
    identically; the others may differ among the experts near the boundary. Returns the counts and the margins at
    the mismatches for reporting."""
    layers, tokens = ours.shape[0], ours.shape[1]
    alive = np.ones(tokens, bool)
    compared = mismatched = 0
    margins: list[float] = []
    for layer in range(layers):
        g = np.sort(np.asarray(gates[layer], np.float64), axis=-1)[:, ::-1]
        margin = (g[:, k - 1] - g[:, k]) / np.maximum(np.maximum(np.abs(g[:, k - 1]), np.abs(g[:, k])), 1e-6)
        same = np.array([set(a.tolist()) == set(b.tolist()) for a, b in zip(ours[layer], ref[layer])])
        for t in np.nonzero(alive)[0]:
            compared += 1
            if same[t]:
                # The same experts: any difference in their order must be between near-equal gate logits.
                gt = np.asarray(gates[layer][t], np.float64)
                for a, b in zip(ours[layer][t], ref[layer][t]):
                    assert abs(gt[a] - gt[b]) <= rel * max(abs(gt[a]), abs(gt[b]), 1e-6), (layer, t, a, b)
                continue
            mismatched += 1
            margins.append(float(margin[t]))
            assert margin[t] <= rel, f"layer {layer} token {t}: routes differ with oracle margin {margin[t]:.3g}"
            ok = routes_match_near(ours[layer][t : t + 1], ref[layer][t : t + 1], gates[layer][t : t + 1], k, rel)
            assert ok.all(), f"layer {layer} token {t}: routes differ away from the top-k boundary"
        alive &= same
    return {"compared": compared, "mismatched": mismatched, "margins": margins, "identical_tokens": alive}
