"""GPT-OSS-style workload definitions (PyTorch, export side only).

These modules define the programs the B200 backend executes. They follow the semantics of the reference's
model family (chroma/models/gpt_oss.py:10-310, chroma/models/cached.py:9-91, chroma/models/variants.py:3-20),
which itself follows the public gpt-oss architecture. Parameter names, shapes, dtypes and registration order
are kept identical to the reference so that

* state dicts are interchangeable (``compile`` reads parameters by their fully qualified names), and
* seeded initialisation draws the same random numbers: ``make_dev_model(seed)`` reproduces
  scripts/export.py:16-29 bit for bit (checked by ``tests/test_models.py`` against a digest recorded from the
  reference).

Importing this module needs Torch; loading and running compiled programs does not.
"""

from __future__ import annotations

import dataclasses
import math
from dataclasses import dataclass

import torch
from torch import Tensor, nn


@dataclass
class ModelConfig:
    num_hidden_layers: int
    num_experts: int
    experts_per_token: int
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    swiglu_limit: float
    head_dim: int
    num_attention_heads: int
    num_key_value_heads: int
    sliding_window: int
    initial_context_length: int
    rope_theta: float
    rope_scaling_factor: float
    rope_ntk_alpha: float
    rope_ntk_beta: float


# The dev configuration (chroma/models/variants.py:3-20): 59,079,408 parameters.
dev = ModelConfig(
    num_hidden_layers=12, num_experts=12, experts_per_token=4, vocab_size=201088, hidden_size=128,
    intermediate_size=128, swiglu_limit=7.0, head_dim=16, num_attention_heads=8, num_key_value_heads=1,
    sliding_window=0, initial_context_length=128, rope_theta=150000.0, rope_scaling_factor=1.0,
    rope_ntk_alpha=1.0, rope_ntk_beta=32.0,
)

# GPT-OSS-20B-shaped and -120B-shaped benchmark configurations. Fields the benchmark does not name keep
# the dev values.
gpt_oss_20b = dataclasses.replace(
    dev, num_hidden_layers=24, hidden_size=2880, intermediate_size=2880, num_attention_heads=64,
    num_key_value_heads=8, head_dim=64, num_experts=32, experts_per_token=4,
)
gpt_oss_120b = dataclasses.replace(gpt_oss_20b, num_hidden_layers=36, num_experts=128)


def rope_tables(config: ModelConfig) -> tuple[float, Tensor]:
    """(concentration, inv_freq[head_dim/2]) of the YaRN-capable rotary embedding (gpt_oss.py:85-111)."""
    half = config.head_dim // 2
    freq = config.rope_theta ** (torch.arange(0, config.head_dim, 2, dtype=torch.float32) / config.head_dim)
    if config.rope_scaling_factor <= 1.0:
        return 1.0, 1.0 / freq
    concentration = 0.1 * math.log(config.rope_scaling_factor) + 1.0
    ctx = config.initial_context_length
    low = half * math.log(ctx / (config.rope_ntk_beta * 2 * math.pi)) / math.log(config.rope_theta)
    high = half * math.log(ctx / (config.rope_ntk_alpha * 2 * math.pi)) / math.log(config.rope_theta)
    assert 0 < low < high < half - 1
    ramp = (torch.arange(half, dtype=torch.float32) - low) / (high - low)
    keep = 1 - ramp.clamp(0, 1)
    return concentration, (1.0 / (config.rope_scaling_factor * freq)) * (1 - keep) + (1.0 / freq) * keep


class RMSNorm(nn.Module):
    def __init__(self, num_features: int, eps: float = 1e-05) -> None:
        super().__init__()
        self.num_features = num_features
        self.eps = eps
        self.scale = nn.Parameter(torch.ones(num_features, dtype=torch.float32))

    def forward(self, x: Tensor) -> Tensor:
        dtype = x.dtype
        t = x.float()
        t = t * torch.rsqrt(torch.mean(t**2, dim=-1, keepdim=True) + self.eps)
        return (t * self.scale).to(dtype)


class Rotary(nn.Module):
    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.config = config
        self.head_dim = config.head_dim

    def cos_sin(self, count: int, positions: Tensor | None) -> tuple[Tensor, Tensor]:
        concentration, inv_freq = rope_tables(self.config)
        t = torch.arange(count, dtype=torch.float32) if positions is None else positions
        angles = torch.einsum("i,j->ij", t, inv_freq)
        return angles.cos() * concentration, angles.sin() * concentration

    @staticmethod
    def rotate(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
        cos = cos.unsqueeze(-2).to(x.dtype)
        sin = sin.unsqueeze(-2).to(x.dtype)
        lo, hi = torch.chunk(x, 2, dim=-1)
        return torch.cat((lo * cos - hi * sin, hi * cos + lo * sin), dim=-1)

    def forward(self, q: Tensor, k: Tensor, positions: Tensor | None = None) -> tuple[Tensor, Tensor]:
        n = q.shape[0]
        cos, sin = self.cos_sin(n, positions)
        q_shape, k_shape = q.shape, k.shape
        q = self.rotate(q.view(n, -1, self.head_dim), cos, sin).reshape(q_shape)
        k = self.rotate(k.view(n, -1, self.head_dim), cos, sin).reshape(k_shape)
        return q, k


class AttentionBlock(nn.Module):
    def __init__(self, config: ModelConfig, layer_idx: int = 0) -> None:
        super().__init__()
        self.head_dim = config.head_dim
        self.num_attention_heads = config.num_attention_heads
        self.num_key_value_heads = config.num_key_value_heads
        # The window applies to even layers only (gpt_oss.py:166).
        self.sliding_window = config.sliding_window if layer_idx % 2 == 0 else 0
        self.sinks = nn.Parameter(torch.empty(config.num_attention_heads, dtype=torch.bfloat16))
        self.norm = RMSNorm(config.hidden_size)
        qkv_dim = config.head_dim * (config.num_attention_heads + 2 * config.num_key_value_heads)
        self.qkv = nn.Linear(config.hidden_size, qkv_dim, dtype=torch.bfloat16)
        self.out = nn.Linear(config.head_dim * config.num_attention_heads, config.hidden_size, dtype=torch.bfloat16)
        self.sm_scale = 1 / math.sqrt(config.head_dim)
        self.rope = Rotary(config)

    def project(self, x: Tensor, positions: Tensor | None = None) -> tuple[Tensor, Tensor, Tensor]:
        qkv = self.qkv(self.norm(x))
        hq = self.num_attention_heads * self.head_dim
        hk = self.num_key_value_heads * self.head_dim
        q = qkv[:, :hq].contiguous()
        k = qkv[:, hq : hq + hk].contiguous()
        v = qkv[:, hq + hk : hq + 2 * hk].contiguous()
        groups = self.num_attention_heads // self.num_key_value_heads
        q = q.view(-1, self.num_key_value_heads, groups, self.head_dim)
        k = k.view(-1, self.num_key_value_heads, self.head_dim)
        v = v.view(-1, self.num_key_value_heads, self.head_dim)
        q, k = self.rope(q, k, positions)
        return q, k, v

    def attend(self, q: Tensor, k: Tensor, v: Tensor, bias: Tensor) -> Tensor:
        """Sink-augmented softmax attention; ``bias`` is the additive [queries, keys] mask."""
        n, heads, groups, _ = q.shape
        k = k[:, :, None, :].expand(-1, -1, groups, -1)
        v = v[:, :, None, :].expand(-1, -1, groups, -1)
        scores = torch.einsum("qhmd,khmd->hmqk", q, k) * self.sm_scale + bias[None, None, :, :]
        sinks = self.sinks.reshape(heads, groups, 1, 1).expand(-1, -1, n, -1)
        weights = torch.cat((scores, sinks), dim=-1).softmax(-1)[..., :-1]
        return torch.einsum("hmqk,khmd->qhmd", weights, v).reshape(n, -1)

    def forward(self, x: Tensor) -> Tensor:
        q, k, v = self.project(x)
        n = q.shape[0]
        bias = torch.triu(q.new_full((n, n), -float("inf")), diagonal=1)
        if self.sliding_window > 0:
            bias += torch.tril(bias.new_full((n, n), -float("inf")), diagonal=-self.sliding_window)
        return x + self.out(self.attend(q, k, v, bias))


def swiglu(x: Tensor, alpha: float = 1.702, limit: float = 7.0) -> Tensor:
    """Interleaved SwiGLU: even columns gate, odd columns linear (+1), both clamped (gpt_oss.py:212-219)."""
    gate = x[..., ::2].clamp(min=None, max=limit)
    linear = x[..., 1::2].clamp(min=-limit, max=limit)
    return gate * torch.sigmoid(alpha * gate) * (linear + 1)


class MLPBlock(nn.Module):
    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.num_experts = config.num_experts
        self.experts_per_token = config.experts_per_token
        self.swiglu_limit = config.swiglu_limit
        # Own parameters come first in named_parameters(), before the submodules' (gpt_oss.py:228-241).
        self.norm = RMSNorm(config.hidden_size)
        self.gate = nn.Linear(config.hidden_size, config.num_experts, dtype=torch.bfloat16)
        e, d, i = config.num_experts, config.hidden_size, config.intermediate_size
        self.mlp1_weight = nn.Parameter(torch.empty(e, 2 * i, d, dtype=torch.bfloat16))
        self.mlp1_bias = nn.Parameter(torch.empty(e, 2 * i, dtype=torch.bfloat16))
        self.mlp2_weight = nn.Parameter(torch.empty(e, d, i, dtype=torch.bfloat16))
        self.mlp2_bias = nn.Parameter(torch.empty(e, d, dtype=torch.bfloat16))

    def forward(self, x: Tensor) -> Tensor:
        t = self.norm(x)
        top = torch.topk(self.gate(t), k=self.experts_per_token, dim=-1, sorted=True)
        weights = nn.functional.softmax(top.values, dim=1)
        chosen = top.indices
        h = torch.einsum("beck,bk->bec", self.mlp1_weight[chosen, ...], t) + self.mlp1_bias[chosen, ...]
        h = swiglu(h, limit=self.swiglu_limit)
        y = torch.einsum("beck,bek->bec", self.mlp2_weight[chosen, ...], h)
        y += self.mlp2_bias[chosen, ...]
        return x + torch.einsum("bec,be->bc", y, weights)


class TransformerBlock(nn.Module):
    def __init__(self, config: ModelConfig, layer_idx: int) -> None:
        super().__init__()
        self.layer_idx = layer_idx
        self.attn = AttentionBlock(config, layer_idx)
        self.mlp = MLPBlock(config)

    def forward(self, x: Tensor) -> Tensor:
        return self.mlp(self.attn(x))


class Transformer(nn.Module):
    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.config = config
        self.embedding = nn.Embedding(config.vocab_size, config.hidden_size, dtype=torch.bfloat16)
        self.block = nn.ModuleList([TransformerBlock(config, i) for i in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size)
        self.unembedding = nn.Linear(config.hidden_size, config.vocab_size, bias=False, dtype=torch.bfloat16)

    def forward(self, x: Tensor) -> Tensor:
        x = self.embedding(x)
        for block in self.block:
            x = block(x)
        return self.unembedding(self.norm(x))


class CachedTransformer(nn.Module):
    """One prefill chunk or decode step against explicit K/V cache inputs (cached.py:9-51).

    Inputs: tokens [n] int64, positions [n] f32, keys/values [L, ctx, KV, hd], mask and window_mask
    [n, ctx+n] additive, last [1] int64. Outputs: logits [1, V] of row ``last``, new keys/values [L, n, KV, hd].
    """

    def __init__(self, model: Transformer) -> None:
        super().__init__()
        self.model = model

    def forward(self, tokens, positions, keys, values, mask, window_mask, last):  # type: ignore[no-untyped-def]
        x = self.model.embedding(tokens)
        new_keys, new_values = [], []
        for layer, block in enumerate(self.model.block):
            attention = block.attn
            q, k, v = attention.project(x, positions)
            new_keys.append(k.unsqueeze(0))
            new_values.append(v.unsqueeze(0))
            past = (keys.shape[1], attention.num_key_value_heads, attention.head_dim)
            all_k = torch.cat((keys[layer : layer + 1].reshape(past), k), dim=0)
            all_v = torch.cat((values[layer : layer + 1].reshape(past), v), dim=0)
            bias = window_mask if attention.sliding_window else mask
            x = block.mlp(x + attention.out(attention.attend(q, all_k, all_v, bias)))
        logits = self.model.unembedding(self.model.norm(x)[last])
        return logits, torch.cat(new_keys, dim=0), torch.cat(new_values, dim=0)


def export_cached(model: Transformer, context: int, steps: int) -> torch.export.ExportedProgram:
    """Export one cached step: ``steps=context`` for prefill, ``steps=1`` for decode (cached.py:68-84)."""
    if context < 1 or not 1 <= steps <= context:
        raise ValueError(f"{steps} steps, context {context}")
    first = model.block[0].attn
    shape = (len(model.block), context, first.num_key_value_heads, first.head_dim)
    dtype = first.qkv.weight.dtype
    inputs = (
        torch.zeros(steps, dtype=torch.int64),
        torch.arange(steps, dtype=torch.float32),
        torch.zeros(shape, dtype=dtype),
        torch.zeros(shape, dtype=dtype),
        torch.zeros(steps, context + steps, dtype=dtype),
        torch.zeros(steps, context + steps, dtype=dtype),
        torch.tensor([steps - 1], dtype=torch.int64),
    )
    with torch.no_grad():
        return torch.export.export(CachedTransformer(model).eval(), inputs)


def init_weights(model: Transformer, *, std: float, zero_bias: bool) -> Transformer:
    """Unit norm scales; zero biases and sinks when ``zero_bias``; N(0, std) elsewhere, in named order."""
    with torch.no_grad():
        for name, parameter in model.named_parameters():
            if name.endswith(".scale"):
                parameter.fill_(1.0)
            elif zero_bias and name.endswith(("bias", ".sinks")):
                parameter.zero_()
            else:
                parameter.normal_(mean=0.0, std=std)
    return model.requires_grad_(False)


def make_dev_model(seed: int = 0) -> Transformer:
    """The seeded fp32 dev model of scripts/export.py:16-29 (same draws, same values)."""
    with torch.random.fork_rng(devices=[]):
        torch.manual_seed(seed)
        model = Transformer(dev).float().eval()
        return init_weights(model, std=0.02, zero_bias=True)


def random_transformer(config: ModelConfig, *, seed: int, std: float, dtype: torch.dtype = torch.float32) -> Transformer:
    """Unit norm scales, N(0, std) elsewhere drawn in fp32, then cast (tests/helpers.py:19-29)."""
    with torch.random.fork_rng(devices=[]):
        torch.manual_seed(seed)
        model = Transformer(config).float().eval()
        init_weights(model, std=std, zero_bias=False)
    return model.to(dtype)
