"""``compile(export, directory, backend="cuda")``: turn a ``torch.export`` program into a B200 artefact.

The reference compiles any exported graph into generated C++/CUDA source and builds it with nvcc per graph
(chroma/_src/compiler.py:51-164, chroma/_src/build.py:50-113). This backend instead ships precompiled sm_100a
kernels (``libchroma_b200.so``) and compiles a graph into a small *launch plan* plus a weights file:

1. ``prepare``: load, ``run_decompositions({})`` and validate the export with the reference's rules and messages
   (chroma/_src/graph.py:15-55): static non-empty shapes, fp32/bf16/int64 only, supported operators only, no
   mutation, tensor inputs and outputs only.
2. ``recognize``: identify the program family and read its hyper-parameters from the graph:
   * GPT-OSS-style transformers (chroma/models/gpt_oss.py, chroma/models/cached.py): ``Transformer.forward``,
     ``CachedTransformer`` prefill/decode steps and ``UncachedTransformer``; parameters are read by their fully
     qualified names, scalars (eps, top-k, attention scale, SwiGLU clamp and slope, RoPE frequencies and
     concentration, per-layer window) from the graph nodes that use them;
   * the fused RMSNorm + gated-SiLU + residual row program (the benchmark micrograph).
   Any other graph goes to the generic path (``chroma_b200/_src/graph.py``): a plan of steps over strided views for
   the precompiled generic kernels (``csrc/graph.cu``); operators outside the reference's table raise
   ``NotImplementedError`` at compile time, as the reference does.
3. ``write_artifact``: pack the weights in the kernels' layout and write the manifest-v2 directory: ``model.json``
   (version 2, Python ABI, library, weights, inputs, outputs, stats; build.py:91-100), ``weights-<sha>.bin`` and
   the library module ``_chroma_<uuid>.py`` exposing ``signature`` and ``Model`` (the native object protocol of
   chroma/_src/core/bindings.h:35-75), so both this package's ``Program`` and the reference's load it. Files are
   staged in a temporary directory and moved into place, and stale artefact files are removed (build.py:59-112).
"""

from __future__ import annotations

import hashlib
import json
import math
import operator
import os
import shutil
import sysconfig
import tempfile
import uuid
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import numpy as np

from chroma_b200._src import native as nat
from chroma_b200._src.memory import gptoss_arena, is_large
from chroma_b200._src.program import Program, signature

# ATen targets the reference accepts (chroma/_src/lowering.py:34-86); the same names, as an interface table.
OPERATIONS: dict[str, str] = {
    **{f"aten.{n}": "elementwise" for n in (
        "abs.default", "add.Tensor", "clamp.default", "cos.default", "div.Tensor", "exp.default", "mul.Tensor",
        "neg.default", "pow.Scalar", "pow.Tensor_Scalar", "reciprocal.default", "rsub.Scalar", "rsqrt.default",
        "sigmoid.default", "sin.default", "square.default", "sub.Tensor")},
    **{f"aten.{n}": "layout" for n in (
        "view.default", "reshape.default", "_unsafe_view.default", "unsqueeze.default", "expand.default",
        "slice.Tensor", "permute.default", "transpose.int", "t.default", "to.dtype", "_to_copy.default",
        "clone.default", "contiguous.default", "split.Tensor", "split_with_sizes.default")},
    "aten.linear.default": "linear",
    "aten.embedding.default": "gather",
    "aten.index.Tensor": "gather",
    "aten.einsum.default": "einsum",
    "aten.mean.dim": "reduction",
    "aten.mean.default": "reduction",
    "aten.sum.default": "reduction",
    "aten.sum.dim_IntList": "reduction",
    "aten.softmax.int": "softmax",
    "aten.topk.default": "topk",
    "aten.cat.default": "cat",
    "aten.arange.default": "constant",
    "aten.arange.start": "constant",
    "aten.arange.start_step": "constant",
    "aten.new_full.default": "constant",
    "aten.full.default": "constant",
    "aten.triu.default": "triangular",
    "aten.tril.default": "triangular",
    "aten._assert_tensor_metadata.default": "metadata",
}

_DTYPE_NAMES = {"torch.float32": "float32", "torch.bfloat16": "bfloat16", "torch.int64": "int64"}
ALIGN = 256


def validate_tensor(tensor: Any) -> None:
    """Static, non-empty, CPU, supported dtype (chroma/_src/graph.py:15-25)."""
    if any(type(d) is not int for d in tensor.shape):
        raise ValueError(f"Dynamic shape {tuple(tensor.shape)}")
    if any(d <= 0 for d in tensor.shape):
        raise ValueError(f"empty dim in {tuple(tensor.shape)}")
    if tensor.numel() * tensor.element_size() >= 2**63:
        raise ValueError(f"{tensor.numel()} elements do not fit")
    if tensor.device.type != "cpu":
        raise ValueError(f"export is on {tensor.device.type}")
    if str(tensor.dtype) not in _DTYPE_NAMES:
        raise ValueError(f"Unsupported dtype {tensor.dtype}")


def prepare(program: Any) -> Any:
    import torch
    from torch.export.graph_signature import InputKind, OutputKind, TensorArgument
    from torch.utils._pytree import tree_leaves

    if isinstance(program, (str, os.PathLike)):
        program = torch.export.load(program)
    program = program.run_decompositions({})
    signature_ = program.graph_signature
    for spec in signature_.input_specs:
        if spec.kind == InputKind.USER_INPUT and not isinstance(spec.arg, TensorArgument):
            raise TypeError(f"Only tensor inputs are supported, got {spec.arg}")
    for spec in signature_.output_specs:
        if spec.kind != OutputKind.USER_OUTPUT:
            raise ValueError(f"Export mutates {spec.target}; mutation of inputs and buffers is unsupported")
        if not isinstance(spec.arg, TensorArgument):
            raise TypeError(f"Only tensor outputs are supported, got {spec.arg}")
    for node in program.graph.nodes:
        if node.op == "call_function" and node.target != operator.getitem and str(node.target) not in OPERATIONS:
            raise NotImplementedError(f"{node.name}: unsupported operator {node.target}")
        for tensor in tree_leaves(node.meta.get("val")):
            if isinstance(tensor, torch.Tensor):
                validate_tensor(tensor)
        if node.op not in {"placeholder", "call_function", "output"}:
            raise NotImplementedError(f"{node.name}: unsupported node kind {node.op}")
    return program


# ---------------------------------------------------------------------------------------------------------
@dataclass
class Lowered:
    """A recognised program: the native plan, its weights and the manifest's tensor specs."""

    plan: dict[str, Any]
    tensors: list[np.ndarray]  # packed in this order; offsets filled by write_artifact
    inputs: list[dict[str, Any]]
    outputs: list[dict[str, Any]]
    stats: dict[str, Any] = field(default_factory=dict)


def _spec(name: str, tensor: Any) -> dict[str, Any]:
    return {"name": name, "shape": list(tensor.shape), "dtype": _DTYPE_NAMES[str(tensor.dtype)]}


def _target(node: Any) -> str:
    return str(getattr(node, "target", ""))


def _is(node: Any, name: str) -> bool:
    return getattr(node, "op", None) == "call_function" and _target(node) == f"aten.{name}"


class _Graph:
    def __init__(self, program: Any) -> None:
        import torch

        self.program = program
        self.nodes = list(program.graph.nodes)
        sig = program.graph_signature
        self.params: dict[str, Any] = {}
        self.param_of: dict[str, str] = {}
        self.user_inputs: list[Any] = []
        placeholders = [n for n in self.nodes if n.op == "placeholder"]
        for node, spec in zip(placeholders, sig.input_specs, strict=True):
            if spec.kind.name == "USER_INPUT":
                self.user_inputs.append(node)
            else:
                state = program.constants if spec.kind.name == "CONSTANT_TENSOR" else program.state_dict
                tensor = state[spec.target]
                self.params[spec.target] = tensor.detach() if isinstance(tensor, torch.Tensor) else tensor
                self.param_of[node.name] = spec.target
        self.output_nodes = list(next(n for n in self.nodes if n.op == "output").args[0])

    def fold(self, node: Any) -> Any:
        """Evaluate a subgraph built only from constants and parameters (the reference folds these too,
        chroma/_src/compiler.py:83-108)."""
        import torch

        if not hasattr(node, "op"):
            return node
        if node.op == "placeholder":
            if node.name in self.param_of:
                return self.params[self.param_of[node.name]]
            raise ValueError(f"{node.name} is not constant")
        if node.op != "call_function":
            raise ValueError(f"{node.name} is not constant")
        args = torch.fx.node.map_arg(node.args, self.fold)
        kwargs = torch.fx.node.map_arg(node.kwargs, self.fold)
        with torch.no_grad():
            return node.target(*args, **kwargs)


def _source(node: Any) -> Any:
    """Walk back through layout ops to the node that produced the data."""
    while getattr(node, "op", None) == "call_function" and OPERATIONS.get(_target(node)) == "layout":
        node = node.args[0]
    return node


def _torch_bytes(tensor: Any, dtype: str) -> np.ndarray:
    import torch

    t = tensor.detach().contiguous()
    if dtype == "float32":
        return t.to(torch.float32).numpy()
    return t.to(torch.bfloat16).view(torch.uint16).numpy()


def _lower_gptoss(g: _Graph) -> Lowered:
    names = list(g.params)
    emb_name = next(n for n in names if n.endswith("embedding.weight") and not n.endswith("unembedding.weight"))
    prefix = emb_name[: -len("embedding.weight")]
    P = {n[len(prefix):]: t for n, t in g.params.items() if n.startswith(prefix)}
    layers = 1 + max(int(n.split(".")[1]) for n in P if n.startswith("block."))
    emb = P["embedding.weight"]
    V, d = emb.shape
    H = P["block.0.attn.sinks"].shape[0]
    qkv_rows = P["block.0.attn.qkv.weight"].shape[0]
    hd = P["block.0.attn.out.weight"].shape[1] // H
    KV = (qkv_rows // hd - H) // 2
    E, two_i, _ = P["block.0.mlp.mlp1_weight"].shape
    I = two_i // 2
    storage = _DTYPE_NAMES[str(emb.dtype)]
    if storage not in ("float32", "bfloat16"):
        raise NotImplementedError(f"GPT-OSS storage dtype {storage}")

    # Scalars from the graph.
    def first(pred):  # type: ignore[no-untyped-def]
        return next((n for n in g.nodes if pred(n)), None)

    eps_node = first(lambda n: _is(n, "add.Tensor") and _is(n.args[0], "mean.dim") and isinstance(n.args[1], (int, float)))
    topk = first(lambda n: _is(n, "topk.default"))
    clamp_hi = first(lambda n: _is(n, "clamp.default") and len(n.args) > 2 and n.args[1] is None)
    if clamp_hi is None:
        clamp_hi = first(lambda n: _is(n, "clamp.default") and n.kwargs.get("min") is None)
    alpha_node = next(u for u in clamp_hi.users if _is(u, "mul.Tensor") and isinstance(u.args[1], (int, float)))
    qk = [n for n in g.nodes if _is(n, "einsum.default") and n.args[0].replace(" ", "") == "qhmd,khmd->hmqk"]
    rope = first(lambda n: _is(n, "einsum.default") and n.args[0].replace(" ", "") == "i,j->ij")
    if eps_node is None or topk is None or rope is None or len(qk) != layers:
        raise NotImplementedError("graph is not a GPT-OSS-style transformer this backend recognises")
    scale_nodes = [next(u for u in n.users if _is(u, "mul.Tensor")) for n in qk]
    sm_scale = float(scale_nodes[0].args[1])
    inv_freq = g.fold(rope.args[1][1]).float().numpy().astype(np.float32)
    cos = next(u for u in rope.users if _is(u, "cos.default"))
    conc_node = next((u for u in cos.users if _is(u, "mul.Tensor")), None)
    concentration = float(conc_node.args[1]) if conc_node is not None else 1.0
    limit = float(clamp_hi.args[2] if len(clamp_hi.args) > 2 else clamp_hi.kwargs["max"])
    k = int(topk.args[1])

    # Program kind from the user inputs.
    user = g.user_inputs
    metas = [n.meta["val"] for n in user]
    window = 0
    layer_window = [0] * layers
    if len(user) == 7:
        kind = nat.GPTOSS_CACHED
        n_tok = metas[0].shape[0]
        context = metas[2].shape[1]
        mask_inputs = {user[4]: 0, user[5]: 1}
        for layer, mul in enumerate(scale_nodes):
            add = next(u for u in mul.users if _is(u, "add.Tensor"))
            src = _source(add.args[1])
            if src not in mask_inputs:
                raise NotImplementedError("cached attention mask is not one of the mask inputs")
            layer_window[layer] = mask_inputs[src]
    elif len(user) in (1, 2):
        kind = nat.GPTOSS_FORWARD if len(user) == 1 else nat.GPTOSS_LAST
        n_tok = metas[0].shape[0]
        context = 0
        layer = -1
        for node in g.nodes:
            if _is(node, "triu.default"):
                layer += 1
            elif _is(node, "tril.default") and layer >= 0:
                diag = int(node.args[1]) if len(node.args) > 1 else int(node.kwargs.get("diagonal", 0))
                layer_window[layer] = 1
                window = -diag
        if layer != layers - 1:
            raise NotImplementedError("could not attribute attention masks to layers")
    else:
        raise NotImplementedError("GPT-OSS program with an unexpected input signature")

    dtype = storage

    def T(name: str) -> np.ndarray:
        return _torch_bytes(P[name], dtype)

    def F(name: str) -> np.ndarray:
        return _torch_bytes(P[name], "float32")

    tensors = [T("embedding.weight"), F("norm.scale"), T("unembedding.weight")]
    for layer in range(layers):
        b = f"block.{layer}."
        tensors += [
            F(b + "attn.norm.scale"), T(b + "attn.sinks"), T(b + "attn.qkv.weight"), T(b + "attn.qkv.bias"),
            T(b + "attn.out.weight"), T(b + "attn.out.bias"), F(b + "mlp.norm.scale"), T(b + "mlp.gate.weight"),
            T(b + "mlp.gate.bias"), T(b + "mlp.mlp1_weight"), T(b + "mlp.mlp1_bias"), T(b + "mlp.mlp2_weight"),
            T(b + "mlp.mlp2_bias"),
        ]
    desc = {
        "kind": kind, "storage": nat.BF16 if dtype == "bfloat16" else nat.FP32, "layers": layers, "hidden": d,
        "heads": H, "kv_heads": KV, "head_dim": hd, "experts": E, "top_k": k, "intermediate": I, "vocab": V,
        "tokens": n_tok, "context": context, "window": window, "eps": float(eps_node.args[1]),
        "sm_scale": sm_scale, "swiglu_alpha": float(alpha_node.args[1]), "swiglu_limit": limit,
        "rope_concentration": concentration, "rows": 0, "cols": 0,
    }
    inputs = [_spec(n.name, n.meta["val"]) for n in user]
    outputs = [_spec(n.name, n.meta["val"]) for n in g.output_nodes]
    plan = {"desc": desc, "inv_freq": inv_freq.tolist(), "layer_window": layer_window}
    return Lowered(plan, tensors, inputs, outputs, _gptoss_stats(desc))


def _gptoss_stats(desc: dict[str, Any]) -> dict[str, Any]:
    """Kernel count of one call and its activation arena (planned like the native executor does)."""
    L = desc["layers"]
    workspace, unreused = gptoss_arena(desc)
    kernels = 1 + 13 * L + 2 if is_large(desc) else 1 + 5 * L + 2
    return {"kernels": kernels, "workspace_bytes": workspace, "unreused_workspace_bytes": unreused,
            "expert_contractions": 2 * L, "matrix_contractions": 4 * L + 1, "tensor_core_path": is_large(desc)}


def _lower_micro(g: _Graph) -> Lowered:
    """Match out = (z * sigmoid(z)) * u + x with z = bf16(rmsnorm_fp32(x) * w) * g."""
    if len(g.user_inputs) != 3 or len(g.output_nodes) != 1 or len(g.params) != 1:
        raise NotImplementedError("not a fused row program")
    x, gg, u = g.user_inputs

    def operands(node: Any, name: str) -> list[Any]:
        if not _is(node, name):
            raise NotImplementedError("not a fused row program")
        return list(node.args)

    def pick(pair: list[Any], want: Any) -> Any:
        if pair[1] is want:
            return pair[0]
        if pair[0] is want:
            return pair[1]
        raise NotImplementedError("not a fused row program")

    out = g.output_nodes[0]
    m4 = pick(operands(out, "add.Tensor"), x)
    m3 = pick(operands(m4, "mul.Tensor"), u)
    a, b = operands(m3, "mul.Tensor")
    z, sig = (a, b) if _is(b, "sigmoid.default") else (b, a)
    if not _is(sig, "sigmoid.default") or sig.args[0] is not z:
        raise NotImplementedError("not a fused row program")
    y16 = pick(operands(z, "mul.Tensor"), gg)
    (m1,) = operands(y16, "_to_copy.default")[:1]
    w_node = next(n for n in m1.args if getattr(n, "name", None) in g.param_of)
    m0 = pick(operands(m1, "mul.Tensor"), w_node)
    xf, r = operands(m0, "mul.Tensor")
    if _is(xf, "rsqrt.default"):
        xf, r = r, xf
    (added,) = operands(r, "rsqrt.default")
    mean, eps = operands(added, "add.Tensor")
    (sq, dims, keep) = operands(mean, "mean.dim")
    if list(dims) != [-1] or not keep or operands(sq, "pow.Tensor_Scalar") != [xf, 2]:
        raise NotImplementedError("not a fused row program")
    if operands(xf, "_to_copy.default")[0] is not x:
        raise NotImplementedError("not a fused row program")
    metas = [n.meta["val"] for n in (x, gg, u)]
    if any(str(m.dtype) != "torch.bfloat16" or tuple(m.shape) != tuple(metas[0].shape) or m.dim() != 2 for m in metas):
        raise NotImplementedError("fused row program wants three bf16 [rows, cols] inputs")
    rows, cols = metas[0].shape
    weight = _torch_bytes(g.params[g.param_of[w_node.name]], "float32")
    desc = {"kind": nat.MICRO, "storage": nat.BF16, "rows": rows, "cols": cols, "eps": float(eps),
            "layers": 0, "hidden": 0, "heads": 0, "kv_heads": 0, "head_dim": 0, "experts": 0, "top_k": 0,
            "intermediate": 0, "vocab": 0, "tokens": 0, "context": 0, "window": 0, "sm_scale": 0.0,
            "swiglu_alpha": 0.0, "swiglu_limit": 0.0, "rope_concentration": 0.0}
    inputs = [_spec(n.name, n.meta["val"]) for n in (x, gg, u)]
    outputs = [_spec(out.name, out.meta["val"])]
    return Lowered({"desc": desc}, [weight], inputs, outputs, {"kernels": 1, "workspace_bytes": 0,
                                                               "unreused_workspace_bytes": 0})


def gptoss_layout(config: Any, ep_world: int = 1, vocab_rows: int | None = None) -> list[tuple[str, tuple[int, ...], bool]]:
    """(name, shape, is_fp32_norm) of every weight tensor in packing order (include/chroma_b200.h layout). With
    ``ep_world`` > 1 the expert tensors hold one rank's share (E / ep_world experts); the router keeps all E.
    ``vocab_rows``: the unembedding rows of a vocab shard (default: all V)."""
    d, V, L = config.hidden_size, config.vocab_size, config.num_hidden_layers
    H, KV, hd = config.num_attention_heads, config.num_key_value_heads, config.head_dim
    E, I = config.num_experts, config.intermediate_size
    El = E // ep_world
    Vu = V if vocab_rows is None else vocab_rows
    out = [("embedding.weight", (V, d), False), ("norm.scale", (d,), True), ("unembedding.weight", (Vu, d), False)]
    for layer in range(L):
        b = f"block.{layer}."
        out += [
            (b + "attn.norm.scale", (d,), True), (b + "attn.sinks", (H,), False),
            (b + "attn.qkv.weight", ((H + 2 * KV) * hd, d), False), (b + "attn.qkv.bias", ((H + 2 * KV) * hd,), False),
            (b + "attn.out.weight", (d, H * hd), False), (b + "attn.out.bias", (d,), False),
            (b + "mlp.norm.scale", (d,), True), (b + "mlp.gate.weight", (E, d), False), (b + "mlp.gate.bias", (E,), False),
            (b + "mlp.mlp1_weight", (El, 2 * I, d), False), (b + "mlp.mlp1_bias", (El, 2 * I), False),
            (b + "mlp.mlp2_weight", (El, d, I), False), (b + "mlp.mlp2_bias", (El, d), False),
        ]
    return out


def _gptoss_specs(config: Any, dtype: str, steps: int, context: int | None, last: bool) -> tuple[list, list]:
    V = config.vocab_size
    if context is not None:
        cache = [config.num_hidden_layers, context, config.num_key_value_heads, config.head_dim]
        rows = [config.num_hidden_layers, steps, config.num_key_value_heads, config.head_dim]
        inputs = [
            {"name": "tokens", "shape": [steps], "dtype": "int64"},
            {"name": "positions", "shape": [steps], "dtype": "float32"},
            {"name": "keys", "shape": cache, "dtype": dtype},
            {"name": "values", "shape": cache, "dtype": dtype},
            {"name": "mask", "shape": [steps, context + steps], "dtype": dtype},
            {"name": "window_mask", "shape": [steps, context + steps], "dtype": dtype},
            {"name": "last", "shape": [1], "dtype": "int64"},
        ]
        outputs = [{"name": "logits", "shape": [1, V], "dtype": dtype}, {"name": "new_keys", "shape": rows, "dtype": dtype},
                   {"name": "new_values", "shape": rows, "dtype": dtype}]
    else:
        inputs = [{"name": "tokens", "shape": [steps], "dtype": "int64"}]
        if last:
            inputs.append({"name": "position", "shape": [1], "dtype": "int64"})
        outputs = [{"name": "logits", "shape": [1 if last else steps, V], "dtype": dtype}]
    return inputs, outputs


def _gptoss_desc(config: Any, dtype: str, steps: int, context: int | None, last: bool) -> dict[str, Any]:
    import math as _math

    kind = nat.GPTOSS_CACHED if context is not None else (nat.GPTOSS_LAST if last else nat.GPTOSS_FORWARD)
    return {
        "kind": kind, "storage": nat.BF16 if dtype == "bfloat16" else nat.FP32, "layers": config.num_hidden_layers,
        "hidden": config.hidden_size, "heads": config.num_attention_heads, "kv_heads": config.num_key_value_heads,
        "head_dim": config.head_dim, "experts": config.num_experts, "top_k": config.experts_per_token,
        "intermediate": config.intermediate_size, "vocab": config.vocab_size, "tokens": steps,
        "context": context or 0, "window": config.sliding_window if context is None else 0, "eps": 1e-5,
        "sm_scale": 1.0 / _math.sqrt(config.head_dim), "swiglu_alpha": 1.702, "swiglu_limit": config.swiglu_limit,
        "rope_concentration": 0.0, "rows": 0, "cols": 0,
    }


def synthetic_gptoss(config: Any, *, steps: int, context: int | None = None, dtype: str = "bfloat16",
                     last: bool = False, ep_world: int = 1,
                     vocab_rows: int | None = None) -> tuple[dict[str, Any], list[tuple[str, int, int, bool]]]:
    """The plan of a GPT-OSS program whose weights will be written straight into device memory (no host copy): returns
    (plan, regions) with regions = (name, byte offset, element count, is_fp32_norm) in packing order. Use with
    ``Native(plan, device_weights=ptr)`` over a buffer of ``plan["desc"]["weight_bytes"]`` bytes."""
    from chroma_b200.models import rope_tables

    es = 2 if dtype == "bfloat16" else 4
    regions, total = [], 0
    for name, shape, is_norm in gptoss_layout(config, ep_world, vocab_rows):
        total = (total + ALIGN - 1) // ALIGN * ALIGN
        numel = math.prod(shape)
        regions.append((name, total, numel, is_norm))
        total += numel * (4 if is_norm else es)
    total = (total + ALIGN - 1) // ALIGN * ALIGN
    conc, inv_freq = rope_tables(config)
    desc = _gptoss_desc(config, dtype, steps, context, last)
    desc["rope_concentration"] = float(conc)
    desc["weight_bytes"] = total
    inputs, outputs = _gptoss_specs(config, dtype, steps, context, last)
    windowed = [1 if config.sliding_window > 0 and layer % 2 == 0 else 0 for layer in range(config.num_hidden_layers)]
    plan = {"desc": desc, "inv_freq": inv_freq.float().numpy().tolist(), "layer_window": windowed,
            "offsets": [r[1] for r in regions], "inputs": inputs, "outputs": outputs}
    return plan, regions


def lower_model(model: Any, *, steps: int, context: int | None = None, last: bool = False,
                experts: range | None = None, vocab_rows: range | None = None) -> Lowered:
    """A GPT-OSS program straight from a ``chroma_b200.models.Transformer`` (no export).

    ``context=None``: ``Transformer.forward`` over ``steps`` tokens (``last=True``: the UncachedTransformer variant
    returning one row); otherwise a CachedTransformer step of ``steps`` rows against a ``context``-row cache. The
    plan is the one ``lower`` recognises from the corresponding export. ``experts``: the global expert indices
    this rank of an expert-parallel group owns (``ExpertGroup.local``); the expert tensors are sliced to them.
    """
    import math as _math

    from chroma_b200.models import rope_tables

    config = model.config
    state = {k: v.detach() for k, v in model.state_dict().items()}
    if experts is not None:
        for k in list(state):
            if k.endswith(("mlp.mlp1_weight", "mlp.mlp1_bias", "mlp.mlp2_weight", "mlp.mlp2_bias")):
                state[k] = state[k][experts.start : experts.stop].contiguous()
    if vocab_rows is not None:  # a vocab shard: this rank's unembedding rows only
        state["unembedding.weight"] = state["unembedding.weight"][vocab_rows.start : vocab_rows.stop].contiguous()
    dtype = _DTYPE_NAMES[str(state["embedding.weight"].dtype)]
    conc, inv_freq = rope_tables(config)

    def T(name: str) -> np.ndarray:
        return _torch_bytes(state[name], dtype)

    def F(name: str) -> np.ndarray:
        return _torch_bytes(state[name], "float32")

    L = config.num_hidden_layers
    tensors = [T("embedding.weight"), F("norm.scale"), T("unembedding.weight")]
    for layer in range(L):
        b = f"block.{layer}."
        tensors += [F(b + "attn.norm.scale"), T(b + "attn.sinks"), T(b + "attn.qkv.weight"), T(b + "attn.qkv.bias"),
                    T(b + "attn.out.weight"), T(b + "attn.out.bias"), F(b + "mlp.norm.scale"), T(b + "mlp.gate.weight"),
                    T(b + "mlp.gate.bias"), T(b + "mlp.mlp1_weight"), T(b + "mlp.mlp1_bias"), T(b + "mlp.mlp2_weight"),
                    T(b + "mlp.mlp2_bias")]
    windowed = [1 if config.sliding_window > 0 and layer % 2 == 0 else 0 for layer in range(L)]
    kind = nat.GPTOSS_CACHED if context is not None else (nat.GPTOSS_LAST if last else nat.GPTOSS_FORWARD)
    desc = {
        "kind": kind, "storage": nat.BF16 if dtype == "bfloat16" else nat.FP32, "layers": L,
        "hidden": config.hidden_size, "heads": config.num_attention_heads, "kv_heads": config.num_key_value_heads,
        "head_dim": config.head_dim, "experts": config.num_experts, "top_k": config.experts_per_token,
        "intermediate": config.intermediate_size, "vocab": config.vocab_size, "tokens": steps,
        "context": context or 0, "window": config.sliding_window if context is None else 0, "eps": 1e-5,
        "sm_scale": 1.0 / _math.sqrt(config.head_dim), "swiglu_alpha": 1.702, "swiglu_limit": config.swiglu_limit,
        "rope_concentration": float(conc), "rows": 0, "cols": 0,
    }
    cache = [config.num_hidden_layers, context or 0, config.num_key_value_heads, config.head_dim]
    if context is not None:
        inputs = [
            {"name": "tokens", "shape": [steps], "dtype": "int64"},
            {"name": "positions", "shape": [steps], "dtype": "float32"},
            {"name": "keys", "shape": cache, "dtype": dtype},
            {"name": "values", "shape": cache, "dtype": dtype},
            {"name": "mask", "shape": [steps, context + steps], "dtype": dtype},
            {"name": "window_mask", "shape": [steps, context + steps], "dtype": dtype},
            {"name": "last", "shape": [1], "dtype": "int64"},
        ]
        rows = [config.num_hidden_layers, steps, config.num_key_value_heads, config.head_dim]
        outputs = [
            {"name": "logits", "shape": [1, config.vocab_size], "dtype": dtype},
            {"name": "new_keys", "shape": rows, "dtype": dtype},
            {"name": "new_values", "shape": rows, "dtype": dtype},
        ]
    else:
        inputs = [{"name": "tokens", "shape": [steps], "dtype": "int64"}]
        if last:
            inputs.append({"name": "position", "shape": [1], "dtype": "int64"})
        outputs = [{"name": "logits", "shape": [1 if last else steps, config.vocab_size], "dtype": dtype}]
    plan = {"desc": desc, "inv_freq": inv_freq.float().numpy().tolist(), "layer_window": windowed}
    return Lowered(plan, tensors, inputs, outputs, _gptoss_stats(desc))


def lower(program: Any) -> Lowered:
    """prepare + recognise: a GPT-OSS program, the fused row program, or else a generic graph plan."""
    prepared = prepare(program)
    g = _Graph(prepared)
    if any(n.endswith("unembedding.weight") for n in g.params):
        return _lower_gptoss(g)
    try:
        return _lower_micro(g)
    except Exception:  # noqa: BLE001 - not the fused row program: any other graph goes to the generic path
        pass
    from chroma_b200._src.graph import lower_graph

    return lower_graph(prepared)


# ---------------------------------------------------------------------------------------------------------
def pack(tensors: list[np.ndarray]) -> tuple[bytes, list[int]]:
    offsets: list[int] = []
    total = 0
    for t in tensors:
        total = (total + ALIGN - 1) // ALIGN * ALIGN
        offsets.append(total)
        total += t.nbytes
    total = (total + ALIGN - 1) // ALIGN * ALIGN
    buf = bytearray(total)
    for off, t in zip(offsets, tensors):
        buf[off : off + t.nbytes] = np.ascontiguousarray(t).tobytes()
    return bytes(buf), offsets


def _library_source(plan: dict[str, Any], sig: str) -> str:
    return (
        '"""Library module of one chroma_b200 artefact: the native object protocol over libchroma_b200.so."""\n'
        f"signature = {sig!r}\n"
        f"PLAN = {json.dumps(plan)!r}\n"
        "import json as _json\n"
        "from chroma_b200._src.native import model_class as _model_class\n"
        "Model = _model_class(_json.loads(PLAN))\n"
    )


def _artifact_files(directory: Path) -> set[str]:
    try:
        manifest = json.loads((directory / "model.json").read_text())
        names = {manifest["library"], manifest["weights"]}
    except (OSError, ValueError, KeyError, TypeError):
        return set()
    return {name for name in names if isinstance(name, str) and name == Path(name).name}


def write_artifact(lowered: Lowered, output: str | os.PathLike[str]) -> Path:
    """Write the artefact directory; returns its path (nothing is loaded)."""
    weights, offsets = pack(lowered.tensors)
    plan = dict(lowered.plan)
    plan["offsets"] = offsets
    plan["desc"] = dict(plan["desc"], weight_bytes=len(weights))
    plan["inputs"] = lowered.inputs
    plan["outputs"] = lowered.outputs
    sig = signature(lowered.inputs, lowered.outputs)
    module = f"_chroma_{uuid.uuid4().hex}"
    library = module + ".py"
    weights_name = f"weights-{hashlib.sha256(weights).hexdigest()[:20]}.bin"
    in_bytes = [math.prod(s["shape"]) * nat.dtype_of(s["dtype"]).itemsize for s in lowered.inputs]
    out_bytes = [math.prod(s["shape"]) * nat.dtype_of(s["dtype"]).itemsize for s in lowered.outputs]
    stats = {
        "kernels": 0, "expressions": 0, "folded_constants": 0, "matrix_contractions": 0, "workspace_bytes": 0,
        "unreused_workspace_bytes": 0, **lowered.stats, "weight_bytes": len(weights), "output_bytes": sum(out_bytes),
        "backend": "cuda", "input_bytes": sum(in_bytes), "target": "sm_100a",
    }
    stats["cuda_buffer_bytes"] = stats["weight_bytes"] + stats["workspace_bytes"] + sum(in_bytes) + sum(out_bytes) + 4
    output = Path(output).resolve()
    output.mkdir(parents=True, exist_ok=True)
    stale = _artifact_files(output)
    with tempfile.TemporaryDirectory(prefix=".compile-", dir=output) as temporary:
        stage = Path(temporary)
        (stage / library).write_text(_library_source(plan, sig))
        (stage / weights_name).write_bytes(weights)
        manifest = {
            "version": 2, "python_abi": sysconfig.get_config_var("SOABI"), "library": library, "weights": weights_name,
            "inputs": lowered.inputs, "outputs": lowered.outputs, "stats": stats, "b200": plan,
        }
        (stage / "model.json").write_text(json.dumps(manifest, indent=2) + "\n")
        for name in (library, weights_name, "model.json"):
            os.replace(stage / name, output / name)
    for name in stale - {library, weights_name}:
        (output / name).unlink(missing_ok=True)
    shutil.rmtree(output / "__pycache__", ignore_errors=True)
    return output


def lower_micro(weight: np.ndarray, rows: int, cols: int, eps: float = 1e-5) -> Lowered:
    """The fused RMSNorm + gated-SiLU + residual row program for bf16 [rows, cols] inputs x, g, u (no export)."""
    desc = {"kind": nat.MICRO, "storage": nat.BF16, "rows": rows, "cols": cols, "eps": float(eps),
            "layers": 0, "hidden": 0, "heads": 0, "kv_heads": 0, "head_dim": 0, "experts": 0, "top_k": 0,
            "intermediate": 0, "vocab": 0, "tokens": 0, "context": 0, "window": 0, "sm_scale": 0.0,
            "swiglu_alpha": 0.0, "swiglu_limit": 0.0, "rope_concentration": 0.0}
    spec = {"shape": [rows, cols], "dtype": "bfloat16"}
    inputs = [{"name": n, **spec} for n in ("x", "g", "u")]
    outputs = [{"name": "out", **spec}]
    return Lowered({"desc": desc}, [np.asarray(weight, np.float32)], inputs, outputs,
                   {"kernels": 1, "workspace_bytes": 0, "unreused_workspace_bytes": 0})


def compile_model(model: Any, output: str | os.PathLike[str], *, steps: int, context: int | None = None,
                  last: bool = False, experts: Any = None) -> Program:
    """Write and load the artefact of a GPT-OSS model without exporting it (see ``lower_model``).

    ``experts``: an ``ExpertGroup``; the artefact then holds this rank's experts only, its manifest records the
    group's rank and size, and the returned program is bound to the group (``Program(dir)`` refuses such an
    artefact: it cannot run without its group)."""
    if experts is None:
        return Program(write_artifact(lower_model(model, steps=steps, context=context, last=last), output))
    lowered = lower_model(model, steps=steps, context=context, last=last, experts=experts.local,
                          vocab_rows=experts.vocab_slice)
    lowered.plan["expert_parallel"] = {"rank": experts.rank, "world": experts.world}
    directory = write_artifact(lowered, output)
    manifest = json.loads((directory / "model.json").read_text())
    native = nat.Native(manifest["b200"], str(directory / manifest["weights"]), ep=experts)
    return Program.from_native(native, manifest["stats"])


def compile_for_backend(program: Any, output: str | os.PathLike[str], *, blas: bool = True, backend: str = "cuda") -> Program:
    """``chroma.compile`` for ``backend="cuda"`` (``blas`` is accepted for compatibility; no BLAS is used)."""
    if backend != "cuda":
        raise ValueError(f"chroma_b200 implements backend='cuda' only, got {backend!r}")
    return Program(write_artifact(lower(program), output))
