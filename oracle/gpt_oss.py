"""ORACLE (test infrastructure only): a NumPy restatement of the reference's CPU program for GPT-OSS graphs.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may use this module, and only as
the checker. The product (``chroma_b200``) never imports it.

It restates, op by op, what the reference's portable CPU backend computes for the exported GPT-OSS graphs
(chroma/models/gpt_oss.py:30-310 and chroma/models/cached.py:16-51, lowered by chroma/_src/lowering.py:112-284
onto chroma/_src/codegen/cpu/kernels.h and expressions.h):

* every op computes in fp32; a bf16 result is rounded to nearest-even after EVERY exported bf16 op
  (chroma/_src/core/bfloat16.h:7-17; chroma/_src/codegen/cpu/codegen.py:41-42 ``encode``), and scalar operands of
  bf16 add/sub/pow are rounded to bf16 first (chroma/_src/lowering.py:201-209);
* RMSNorm is the fused fp32 kernel ``x * (1/sqrt(sum(x^2)/n + eps)) * w`` (kernels.h:101-115), recognised only
  on all-fp32 chains (chroma/_src/graph.py:58-95);
* fp32 linear is ``X W^T`` then ``+ bias`` in a second pass (kernels.h:46-61); bf16 linear rounds once after
  ``sum + bias`` (kernels.h:63-74); expert contractions are per-(token, expert) GEMVs (kernels.h:76-99);
* softmax subtracts the max, exponentiates, sums, divides (kernels.h:125-151);
* top-k ranks NaN highest; ties go to the lowest index here (the reference CPU order for ties is
  unspecified, chroma/_src/codegen/cpu/kernels.h:153-185; the reference GPU generator picks the lowest index,
  chroma/_src/codegen/gpu.py:300-337).

Matrix products accumulate in float64 and round to fp32 once; the reference accumulates sequentially in fp32.
The difference is far below the parity tolerances (1e-4 relative for fp32, 2e-2 for bf16), and the oracle is
pinned against golden vectors produced by the reference's own compiled CPU programs (``tests/golden``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

F32 = np.float32


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even); NaN becomes 0x7fc0 (bfloat16.h:7-17)."""
    x = np.ascontiguousarray(x, dtype=F32)
    word = x.view(np.uint32).astype(np.uint64)
    rounded = ((word + 0x7FFF + ((word >> 16) & 1)) >> 16).astype(np.uint32)
    nan = (word & 0x7FFFFFFF) > 0x7F800000
    rounded = np.where(nan, np.uint32(0x7FC0), rounded)
    return (rounded << 16).astype(np.uint32).view(F32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(F32)


@dataclass
class Numerics:
    """fp32 or bf16 storage semantics: ``r`` rounds a fresh op result to the storage type."""

    bf16: bool

    def r(self, x: np.ndarray) -> np.ndarray:
        return bf16_round(x) if self.bf16 else np.asarray(x, dtype=F32)

    def scalar(self, value: float) -> F32:
        """Scalar operand of a bf16 add/sub/pow is itself rounded to bf16 (lowering.py:201-209)."""
        return F32(bf16_round(np.array([value], F32))[0]) if self.bf16 else F32(value)


def matmul_t(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """X[..., K] @ W[N, K]^T accumulated in float64, rounded to fp32."""
    return np.matmul(x.astype(np.float64), w.astype(np.float64).T).astype(F32)


def linear(num: Numerics, x: np.ndarray, w: np.ndarray, b: np.ndarray | None) -> np.ndarray:
    """nn.Linear as the reference CPU computes it (kernels.h:46-74)."""
    y = matmul_t(x, w)
    if b is None:
        return num.r(y)
    if num.bf16:
        return bf16_round(y + b.astype(F32))
    return (y + b.astype(F32)).astype(F32)


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """Fused fp32 RMSNorm (kernels.h:101-115): scale = 1/sqrt(sum(x^2)/n + eps); out = x*scale*w."""
    x = x.astype(F32)
    total = np.sum(x.astype(np.float64) * x.astype(np.float64), axis=-1, keepdims=True).astype(F32)
    scale = (F32(1.0) / np.sqrt(total / F32(x.shape[-1]) + F32(eps))).astype(F32)
    return (x * scale * w.astype(F32)).astype(F32)


def softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    """kernels.h:125-151 in fp32 (max-subtracted exp, sum, divide)."""
    x = x.astype(F32)
    with np.errstate(invalid="ignore", over="ignore"):
        m = np.max(x, axis=axis, keepdims=True)
        e = np.exp(x - m).astype(F32)
        s = np.sum(e.astype(np.float64), axis=axis, keepdims=True).astype(F32)
        return (e / s).astype(F32)


def topk(x: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """Largest-k along the last axis, sorted descending; NaN ranks highest (above +inf), ties keep the lowest index
    (the comparator of chroma/_src/codegen/cpu/kernels.h:158-164 with the GPU backend's lowest-index tie order,
    chroma/_src/codegen/gpu.py:300-311)."""
    nan = np.isnan(x)
    key = np.where(nan, 0.0, x).astype(np.float64)
    # lexsort sorts by the last key first: NaN before numbers, then descending value, then ascending index.
    idx = np.arange(x.shape[-1])
    order = np.empty(x.shape[:-1] + (k,), dtype=np.int64)
    flat_x = key.reshape(-1, x.shape[-1])
    flat_n = nan.reshape(-1, x.shape[-1])
    flat_o = order.reshape(-1, k)
    for row in range(flat_x.shape[0]):
        flat_o[row] = np.lexsort((idx, -flat_x[row], ~flat_n[row]))[:k]
    values = np.take_along_axis(x, order, axis=-1)
    return values, order


def sigmoid(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return (F32(1.0) / (F32(1.0) + np.exp(-x.astype(F32)))).astype(F32)


# ---------------------------------------------------------------------------------------------------------
# Model


@dataclass
class Config:
    layers: int
    experts: int
    top_k: int
    vocab: int
    hidden: int
    intermediate: int
    swiglu_limit: float
    head_dim: int
    heads: int
    kv_heads: int
    sliding_window: int
    initial_context_length: int
    rope_theta: float
    rope_scaling_factor: float
    rope_ntk_alpha: float
    rope_ntk_beta: float

    @classmethod
    def from_model_config(cls, c) -> "Config":  # type: ignore[no-untyped-def]
        return cls(
            c.num_hidden_layers, c.num_experts, c.experts_per_token, c.vocab_size, c.hidden_size,
            c.intermediate_size, c.swiglu_limit, c.head_dim, c.num_attention_heads, c.num_key_value_heads,
            c.sliding_window, c.initial_context_length, c.rope_theta, c.rope_scaling_factor, c.rope_ntk_alpha,
            c.rope_ntk_beta,
        )


def rope(cfg: Config) -> tuple[float, np.ndarray]:
    """(concentration, inv_freq) computed in fp32 like the exported graph (gpt_oss.py:85-111)."""
    half = cfg.head_dim // 2
    exponent = (np.arange(0, cfg.head_dim, 2, dtype=F32) / F32(cfg.head_dim)).astype(F32)
    freq = np.power(F32(cfg.rope_theta), exponent).astype(F32)
    if cfg.rope_scaling_factor <= 1.0:
        return 1.0, (F32(1.0) / freq).astype(F32)
    concentration = 0.1 * math.log(cfg.rope_scaling_factor) + 1.0
    ctx = cfg.initial_context_length
    low = half * math.log(ctx / (cfg.rope_ntk_beta * 2 * math.pi)) / math.log(cfg.rope_theta)
    high = half * math.log(ctx / (cfg.rope_ntk_alpha * 2 * math.pi)) / math.log(cfg.rope_theta)
    ramp = ((np.arange(half, dtype=F32) - F32(low)) / F32(high - low)).astype(F32)
    keep = (F32(1) - np.clip(ramp, 0, 1)).astype(F32)
    interp = (F32(1.0) / (F32(cfg.rope_scaling_factor) * freq)).astype(F32)
    extrap = (F32(1.0) / freq).astype(F32)
    return concentration, (interp * (F32(1) - keep) + extrap * keep).astype(F32)


@dataclass
class Params:
    """Parameters by the reference's fully qualified names, as float32 arrays (bf16 values stay exact)."""

    tensors: dict[str, np.ndarray]
    bf16: bool
    prefix: str = ""

    def __getitem__(self, name: str) -> np.ndarray:
        return self.tensors[self.prefix + name]

    @classmethod
    def from_module(cls, module, prefix: str = "") -> "Params":  # type: ignore[no-untyped-def]
        import torch

        tensors = {}
        bf16 = False
        for name, value in module.state_dict().items():
            value = value.detach()
            if value.dtype == torch.bfloat16:
                bf16 = True
                value = value.float()
            tensors[name] = value.numpy().astype(F32)
        return cls(tensors, bf16, prefix)


@dataclass
class Trace:
    """Optional intermediate record: routing indices and gate logits per layer."""

    routes: list[np.ndarray] = field(default_factory=list)
    gates: list[np.ndarray] = field(default_factory=list)


def _rotate(num: Numerics, x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    # x [n, heads, hd]; cos/sin [n, hd/2] already in storage precision.
    half = x.shape[-1] // 2
    lo, hi = x[..., :half], x[..., half:]
    c, s = cos[:, None, :], sin[:, None, :]
    o1 = num.r(num.r(lo * c) - num.r(hi * s))
    o2 = num.r(num.r(hi * c) + num.r(lo * s))
    return np.concatenate([o1, o2], axis=-1)


def _cos_sin(num: Numerics, cfg: Config, positions: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    concentration, inv_freq = rope(cfg)
    angles = (positions.astype(F32)[:, None] * inv_freq[None, :]).astype(F32)
    cos = (np.cos(angles.astype(np.float64)).astype(F32) * F32(concentration)).astype(F32)
    sin = (np.sin(angles.astype(np.float64)).astype(F32) * F32(concentration)).astype(F32)
    return num.r(cos), num.r(sin)


def _attention(num: Numerics, cfg: Config, p: Params, layer: int, q: np.ndarray, keys: np.ndarray,
               values: np.ndarray, bias: np.ndarray) -> np.ndarray:
    """Sink softmax attention. q [n, KV, G, hd]; keys/values [K, KV, hd]; bias [n, K] additive."""
    n = q.shape[0]
    scale = F32(1.0 / math.sqrt(cfg.head_dim))
    # scores[h, m, q, k] = sum_d q[q,h,m,d] k[k,h,d]
    scores = np.einsum("qhmd,khd->hmqk", q.astype(np.float64), keys.astype(np.float64)).astype(F32)
    scores = num.r(scores)
    scores = num.r(scores * scale)
    scores = num.r(scores + bias[None, None, :, :].astype(F32))
    groups = cfg.heads // cfg.kv_heads
    sinks = p[f"block.{layer}.attn.sinks"].reshape(cfg.kv_heads, groups, 1, 1)
    sinks = np.broadcast_to(sinks, scores.shape[:3] + (1,))
    probs = num.r(softmax(np.concatenate([scores, sinks], axis=-1), axis=-1))[..., :-1]
    out = np.einsum("hmqk,khd->qhmd", probs.astype(np.float64), values.astype(np.float64)).astype(F32)
    return num.r(out).reshape(n, -1)


def _project(num: Numerics, cfg: Config, p: Params, layer: int, x: np.ndarray, positions: np.ndarray):  # type: ignore[no-untyped-def]
    a = f"block.{layer}.attn."
    t = num.r(rmsnorm(x, p[a + "norm.scale"], 1e-5))
    qkv = linear(num, t, p[a + "qkv.weight"], p[a + "qkv.bias"])
    hq, hk = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    n = x.shape[0]
    q = qkv[:, :hq].reshape(n, cfg.heads, cfg.head_dim)
    k = qkv[:, hq : hq + hk].reshape(n, cfg.kv_heads, cfg.head_dim)
    v = qkv[:, hq + hk : hq + 2 * hk].reshape(n, cfg.kv_heads, cfg.head_dim)
    cos, sin = _cos_sin(num, cfg, positions)
    q = _rotate(num, q, cos, sin).reshape(n, cfg.kv_heads, cfg.heads // cfg.kv_heads, cfg.head_dim)
    k = _rotate(num, k, cos, sin)
    return q, k, v


def _mlp(num: Numerics, cfg: Config, p: Params, layer: int, x: np.ndarray, trace: Trace | None) -> np.ndarray:
    m = f"block.{layer}.mlp."
    t = num.r(rmsnorm(x, p[m + "norm.scale"], 1e-5))
    g = linear(num, t, p[m + "gate.weight"], p[m + "gate.bias"])
    values, chosen = topk(g, cfg.top_k)
    if trace is not None:
        trace.routes.append(chosen.copy())
        trace.gates.append(g.copy())
    weights = num.r(softmax(values, axis=1))
    w1, b1 = p[m + "mlp1_weight"], p[m + "mlp1_bias"]
    w2, b2 = p[m + "mlp2_weight"], p[m + "mlp2_bias"]
    n = x.shape[0]
    # Per-(token, expert) GEMVs (kernels.h:76-99), evaluated one expert at a time.
    h = np.empty((n, cfg.top_k, 2 * cfg.intermediate), F32)
    for e in np.unique(chosen):
        bs, ss = np.nonzero(chosen == e)
        h[bs, ss] = matmul_t(t[bs], w1[e])
    h = num.r(num.r(h) + b1[chosen])
    limit = F32(cfg.swiglu_limit)
    glu = np.minimum(h[..., ::2], limit)
    lin = np.clip(h[..., 1::2], -limit, limit)
    act = num.r(glu * num.r(sigmoid(num.r(glu * F32(1.702)))))
    act = num.r(act * num.r(lin + num.scalar(1.0)))
    y = np.empty((n, cfg.top_k, cfg.hidden), F32)
    for e in np.unique(chosen):
        bs, ss = np.nonzero(chosen == e)
        y[bs, ss] = matmul_t(act[bs, ss], w2[e])
    y = num.r(num.r(y) + b2[chosen])
    combined = num.r(np.einsum("bec,be->bc", y.astype(np.float64), weights.astype(np.float64)).astype(F32))
    return num.r(x + combined)


def embed(p: Params, tokens: np.ndarray, vocab: int) -> np.ndarray:
    tokens = np.asarray(tokens, dtype=np.int64)
    if np.any((tokens < 0) | (tokens >= vocab)):
        raise IndexError("Tensor index out of range")
    return p["embedding.weight"][tokens].astype(F32)


def forward(cfg: Config, p: Params, tokens: np.ndarray, trace: Trace | None = None) -> np.ndarray:
    """Transformer.forward (gpt_oss.py:304-310): logits [n, V] for a causal pass over ``tokens``."""
    num = Numerics(p.bf16)
    return linear(num, final_rows(cfg, p, tokens, trace), p["unembedding.weight"], None)


def final_rows(cfg: Config, p: Params, tokens: np.ndarray, trace: Trace | None = None) -> np.ndarray:
    """The final-normed hidden rows [n, d] that Transformer.forward projects onto the vocabulary."""
    num = Numerics(p.bf16)
    x = embed(p, tokens, cfg.vocab)
    n = x.shape[0]
    positions = np.arange(n, dtype=F32)
    for layer in range(cfg.layers):
        q, k, v = _project(num, cfg, p, layer, x, positions)
        i, j = np.arange(n)[:, None], np.arange(n)[None, :]
        visible = j <= i
        window = cfg.sliding_window if layer % 2 == 0 else 0
        if window > 0:
            visible &= (i - j) < window
        bias = np.where(visible, F32(0), F32(-np.inf)).astype(F32)
        attn = _attention(num, cfg, p, layer, q, k, v, bias)
        a = f"block.{layer}.attn."
        x = num.r(x + linear(num, attn, p[a + "out.weight"], p[a + "out.bias"]))
        x = _mlp(num, cfg, p, layer, x, trace)
    return num.r(rmsnorm(x, p["norm.scale"], 1e-5))


def cached_step(cfg: Config, p: Params, tokens, positions, keys, values, mask, window_mask, last,  # type: ignore[no-untyped-def]
                trace: Trace | None = None):
    """CachedTransformer.forward (cached.py:16-51) -> (logits [1, V], new_keys, new_values [L, n, KV, hd])."""
    num = Numerics(p.bf16)
    x = embed(p, tokens, cfg.vocab)
    n = x.shape[0]
    new_k = np.empty((cfg.layers, n, cfg.kv_heads, cfg.head_dim), F32)
    new_v = np.empty_like(new_k)
    for layer in range(cfg.layers):
        q, k, v = _project(num, cfg, p, layer, x, np.asarray(positions, F32))
        new_k[layer], new_v[layer] = k, v
        all_k = np.concatenate([np.asarray(keys[layer], F32), k], axis=0)
        all_v = np.concatenate([np.asarray(values[layer], F32), v], axis=0)
        window = cfg.sliding_window if layer % 2 == 0 else 0
        bias = np.asarray(window_mask if window else mask, F32)
        attn = _attention(num, cfg, p, layer, q, all_k, all_v, bias)
        a = f"block.{layer}.attn."
        x = num.r(x + linear(num, attn, p[a + "out.weight"], p[a + "out.bias"]))
        x = _mlp(num, cfg, p, layer, x, trace)
    row = int(np.asarray(last).reshape(-1)[0])
    if row < -n or row >= n:
        raise IndexError("Tensor index out of range")
    t = num.r(rmsnorm(x, p["norm.scale"], 1e-5))[row]
    return linear(num, t[None, :], p["unembedding.weight"], None), new_k, new_v


def micro(x: np.ndarray, g: np.ndarray, u: np.ndarray, w: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """The C3 micrograph, bf16 in/out (fp32 values): y = bf16(RMSNorm(x)*w); z = y*g; out = z*sigmoid(z)*u + x."""
    y = bf16_round(rmsnorm(x, w, eps))
    z = bf16_round(y * g)
    s = bf16_round(sigmoid(z))
    out = bf16_round(bf16_round(bf16_round(z * s) * u) + x)
    return out


class Decoder:
    """Host-side rolling-cache decoder over ``cached_step`` (chroma/_src/decoder.py:44-152 semantics)."""

    def __init__(self, cfg: Config, p: Params, context: int, prefill_steps: int, sliding_window: int = 0) -> None:
        self.cfg, self.p = cfg, p
        self.context, self.steps = context, prefill_steps
        self.window = min(sliding_window or context, context)
        shape = (cfg.layers, context, cfg.kv_heads, cfg.head_dim)
        self.keys = np.zeros(shape, F32)
        self.values = np.zeros(shape, F32)
        self.slots = np.full(context, -1, np.int64)
        self.position = 0

    def append(self, tokens, trace: Trace | None = None) -> np.ndarray:  # type: ignore[no-untyped-def]
        ids = np.asarray(tokens, dtype=np.int64)
        offset = 0
        logits = None
        while offset < len(ids):
            remaining = len(ids) - offset
            steps = 1 if remaining == 1 else self.steps
            count = min(steps, remaining)
            times = self.position + np.arange(steps, dtype=np.int64)
            key_times = np.concatenate((self.slots, times))
            valid = np.concatenate((self.slots >= 0, np.ones(steps, dtype=bool)))
            causal = valid[None, :] & (key_times[None, :] <= times[:, None])
            masks = []
            for window in (self.context, self.window):
                mask = np.full((steps, self.context + steps), -np.inf, F32)
                mask[causal & (key_times[None, :] > times[:, None] - window)] = 0
                masks.append(mask)
            token_ids = np.zeros(steps, np.int64)
            token_ids[:count] = ids[offset : offset + count]
            logits, nk, nv = cached_step(self.cfg, self.p, token_ids, times.astype(F32), self.keys, self.values,
                                         masks[0], masks[1], np.array([count - 1]), trace)
            rows = times[:count] % self.context
            self.keys[:, rows] = nk[:, :count]
            self.values[:, rows] = nv[:, :count]
            self.slots[rows] = times[:count]
            self.position += count
            offset += count
        assert logits is not None
        return logits
