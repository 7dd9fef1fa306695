"""Generic exported graphs: lower any graph over the reference's operator table to a plan for csrc/graph.cu.

The reference turns every exported graph into generated C++/CUDA (chroma/_src/compiler.py:51-164 driving
chroma/_src/lowering.py:113-330 and a code generator) and builds it with nvcc. This backend keeps precompiled
kernels and compiles a graph into *steps over strided views*:

* **views** instead of copies for the layout operators (view / reshape of contiguous data, unsqueeze, expand, slice,
  permute, transpose, t, split, clone, contiguous, same-type casts), as the reference's ``layout_view`` does
  (lowering.py:97-110, 125-180);
* **fused elementwise expressions** evaluated per output element by a register bytecode (``kGElementwise``), with
  the reference's per-operator semantics (chroma/_src/codegen/cpu/codegen.py:12-180): bf16 results rounded after
  every operator, bf16 scalar operands of add/sub/rsub/pow and ``alpha`` rounded first (lowering.py:196-209), clamp
  as ``min(max(x, low), high)`` keeping NaN and a NaN bound turning into a multiply by NaN (lowering.py:189-194);
  a value is materialised when more than one operator reads it, when it is a graph output, when a non-elementwise
  operator reads it, or when its expression reaches 24 operators (gpu.py:135's depth bound);
* one step per reduction, softmax, top-k, gather, concatenation part, triangle and contraction (linear, einsum), with
  the reference's CPU kernels' summation orders (kernels.h:24-151).

Constants (arange, full, new_full) are folded into the weights file with the graph's parameters and buffers.
"""

from __future__ import annotations

import math
import operator
import struct
from dataclasses import dataclass
from typing import Any

import numpy as np

F32, BF16, I64 = 0, 1, 2
_DTYPE = {"torch.float32": F32, "torch.bfloat16": BF16, "torch.int64": I64}
_ES = {F32: 4, BF16: 2, I64: 8}
_NAME = {F32: "float32", BF16: "bfloat16", I64: "int64"}
IN, OUT, ARENA, WEIGHT = 0, 1, 2, 3
MAX_RANK = 8
MAX_DEPTH = 24
ALIGN = 256

# Step kinds and opcodes of csrc/graph.cu.
K_EW, K_MOVE, K_REDUCE, K_CONTRACT, K_SOFTMAX, K_TOPK, K_GATHER = range(1, 8)
OPS = {name: i for i, name in enumerate(
    ["load", "const", "add", "sub", "mul", "div", "neg", "abs", "exp", "sin", "cos", "recip", "rsqrt", "sigmoid",
     "square", "pow", "maxc", "minc", "round"], start=1)}
_UNARY = {"aten.reciprocal.default": "recip", "aten.rsqrt.default": "rsqrt", "aten.sigmoid.default": "sigmoid",
          "aten.neg.default": "neg", "aten.sin.default": "sin", "aten.cos.default": "cos", "aten.exp.default": "exp",
          "aten.abs.default": "abs", "aten.square.default": "square"}
_BINARY = {"aten.add.Tensor": "add", "aten.sub.Tensor": "sub", "aten.mul.Tensor": "mul", "aten.div.Tensor": "div"}


def _contiguous(shape: tuple[int, ...]) -> tuple[int, ...]:
    out, acc = [], 1
    for d in reversed(shape):
        out.append(acc)
        acc *= d
    return tuple(reversed(out))


def _f32(value: float) -> float:
    return float(np.float32(value))


def _bf16(value: float) -> float:
    from ml_dtypes import bfloat16

    return float(np.float32(bfloat16(np.float32(value))))


@dataclass(frozen=True)
class View:
    """A strided view of one of the program's buffers (strides and offset in elements)."""

    kind: int
    index: int  # input / output number, or the byte offset of the arena region / weight tensor
    dtype: int
    shape: tuple[int, ...]
    strides: tuple[int, ...]
    offset: int = 0
    extra: int = 0  # elements a step reads beyond the view's own extent (along reduced axes)

    def span(self) -> int:
        return 1 + sum((s - 1) * abs(t) for s, t in zip(self.shape, self.strides)) + self.extra

    def broadcast(self, shape: tuple[int, ...]) -> "View":
        pad = len(shape) - len(self.shape)
        old = (1,) * pad + self.shape
        strides = (0,) * pad + self.strides
        return View(self.kind, self.index, self.dtype, shape,
                    tuple(0 if a == 1 and b != 1 else t for a, b, t in zip(old, shape, strides)), self.offset)

    def contiguous(self) -> bool:
        return all(s == 1 or t == c for s, t, c in zip(self.shape, self.strides, _contiguous(self.shape)))


@dataclass(frozen=True)
class Expr:
    """An unmaterialised elementwise value: op over args (Expr, View or float), result dtype and shape."""

    op: str
    args: tuple[Any, ...]
    dtype: int
    shape: tuple[int, ...]
    imm: float = 0.0
    depth: int = 1


def _depth(x: Any) -> int:
    return x.depth if isinstance(x, Expr) else 0


class Lowering:
    def __init__(self) -> None:
        self.tensors: list[np.ndarray] = []
        self.weight_bytes = 0
        self.arena_bytes = 0
        self.views: list[View] = []
        self.ops: list[tuple[int, int, int, int, float]] = []
        self.steps: list[dict[str, Any]] = []
        self.constants = 0
        self.contractions = 0

    # -- buffers ---------------------------------------------------------------------------------------------------
    def weight(self, array: np.ndarray, dtype: int) -> View:
        offset = (self.weight_bytes + ALIGN - 1) // ALIGN * ALIGN
        self.tensors.append(np.ascontiguousarray(array))
        self.weight_bytes = offset + array.nbytes
        shape = tuple(array.shape)
        return View(WEIGHT, offset, dtype, shape, _contiguous(shape))

    def arena(self, dtype: int, shape: tuple[int, ...]) -> View:
        offset = (self.arena_bytes + ALIGN - 1) // ALIGN * ALIGN
        self.arena_bytes = offset + max(1, math.prod(shape)) * _ES[dtype]
        return View(ARENA, offset, dtype, shape, _contiguous(shape))

    def view_id(self, v: View) -> int:
        if len(v.shape) > MAX_RANK:
            raise NotImplementedError(f"rank {len(v.shape)} > {MAX_RANK}")
        self.views.append(v)
        return len(self.views) - 1

    def step(self, kind: int, shape: tuple[int, ...], out: View, **kw: Any) -> None:
        if len(shape) > MAX_RANK:
            raise NotImplementedError(f"rank {len(shape)} > {MAX_RANK}")
        st = {"kind": kind, "rank": len(shape), "n": kw.pop("n", max(1, math.prod(shape))), "oshape": shape,
              "out": self.view_id(out), "out2": -1, "in": -1, "in2": -1, "bias": -1, "first_operand": 0,
              "n_operands": 0, "first_op": 0, "n_ops": 0, "rshape": (), "rstride_a": (), "rstride_b": (),
              "axis": 0, "width": 0, "k": 0, "largest": 0, "tri": 0, "diag": 0, "negative": 0, "divisor": 1.0}
        for key in ("out2", "in", "in2", "bias"):
            if key in kw:
                value = kw.pop(key)
                st[key] = self.view_id(value) if value is not None else -1
        st.update(kw)
        self.steps.append(st)

    # -- materialisation -------------------------------------------------------------------------------------------
    def materialize(self, value: Any, into: View | None = None) -> View:
        """A View holding `value` (an Expr is evaluated; a View is copied only when `into` is given)."""
        if isinstance(value, View) and into is None:
            return value
        if isinstance(value, View):
            if value.dtype != into.dtype:
                value = Expr("round" if into.dtype == BF16 else "cast", (value,), into.dtype, value.shape)
            else:
                self.step(K_MOVE, into.shape, into, **{"in": value.broadcast(into.shape)})
                return into
        out = into if into is not None else self.arena(value.dtype, value.shape)
        self.emit_expr(value, out)
        return out

    def emit_expr(self, expr: Expr, out: View) -> None:
        operands: list[View] = []
        code: list[tuple[int, int, int, int, float]] = []
        free: list[int] = []
        top = [0]

        def reg() -> int:
            if free:
                return free.pop()
            top[0] += 1
            if top[0] > 32:
                raise NotImplementedError("elementwise expression needs more than 32 registers")
            return top[0] - 1

        def walk(x: Any) -> int:
            if isinstance(x, View):
                v = x.broadcast(out.shape)
                if v.dtype == I64:
                    raise NotImplementedError("elementwise arithmetic on int64")
                if v not in operands:
                    operands.append(v)
                r = reg()
                code.append((OPS["load"], r, operands.index(v), 0, 0.0))
                return r
            if isinstance(x, float):
                r = reg()
                code.append((OPS["const"], r, 0, 0, x))
                return r
            if x.op == "cast":  # to fp32: the value itself
                return walk(x.args[0])
            srcs = [walk(a) for a in x.args]
            for s in srcs:
                free.append(s)
            r = reg()
            code.append((OPS[x.op], r, srcs[0], srcs[1] if len(srcs) > 1 else 0, x.imm))
            return r

        walk(expr)
        first_operand = len(self.views)
        for v in operands:
            self.view_id(v)
        first_op = len(self.ops)
        self.ops.extend(code)
        self.step(K_EW, out.shape, out, first_operand=first_operand, n_operands=len(operands), first_op=first_op,
                  n_ops=len(code))

    # -- plan words ------------------------------------------------------------------------------------------------
    def words(self, in_bytes: list[int], out_bytes: list[int]) -> list[int]:
        weight_bytes = (self.weight_bytes + ALIGN - 1) // ALIGN * ALIGN  # the packed file's size (compiler.pack)
        w: list[int] = [0x31474243, weight_bytes, self.arena_bytes, len(in_bytes), len(out_bytes), *in_bytes,
                        *out_bytes, len(self.views)]
        for v in self.views:
            w += [v.kind, v.index, v.span(), v.dtype, len(v.shape), v.offset]
            for d in range(MAX_RANK):
                w += [v.shape[d], v.strides[d]] if d < len(v.shape) else [1, 0]
        w.append(len(self.ops))
        for op, dst, a, b, imm in self.ops:
            w += [op | dst << 8 | a << 16 | b << 24, struct.unpack("<I", struct.pack("<f", imm))[0]]
        w.append(len(self.steps))
        for st in self.steps:
            w += [st["kind"], st["rank"], st["n"]]
            w += [st["oshape"][d] if d < st["rank"] else 1 for d in range(MAX_RANK)]
            w += [st[k] for k in ("out", "out2", "in", "in2", "bias", "first_operand", "n_operands", "first_op",
                                  "n_ops")]
            w.append(len(st["rshape"]))
            for d in range(MAX_RANK):
                if d < len(st["rshape"]):
                    w += [st["rshape"][d], st["rstride_a"][d], st["rstride_b"][d] if st["rstride_b"] else 0]
                else:
                    w += [1, 0, 0]
            w += [st["axis"], st["width"], st["k"], st["largest"], st["tri"], st["diag"], st["negative"],
                  struct.unpack("<I", struct.pack("<f", st["divisor"]))[0]]
        return w


def _axis(dim: int, rank: int) -> int:
    return dim + rank if dim < 0 else dim


def _arg(args: tuple[Any, ...], kwargs: dict[str, Any], index: int, name: str, default: Any = None) -> Any:
    return args[index] if len(args) > index else kwargs.get(name, default)


def lower_graph(program: Any) -> Any:
    """A prepared export (chroma_b200._src.compiler.prepare) -> ``Lowered`` with the graph plan."""
    import torch
    from torch.export.graph_signature import InputKind

    from chroma_b200._src.compiler import Lowered, _DTYPE_NAMES, _target

    low = Lowering()
    sig = program.graph_signature
    state = program.state_dict
    constants = getattr(program, "constants", {})
    spec_of = {spec.arg.name: spec for spec in sig.input_specs if hasattr(spec.arg, "name")}
    env: dict[str, Any] = {}
    users = {node.name: len(node.users) for node in program.graph.nodes}
    inputs: list[dict[str, Any]] = []
    outputs: list[dict[str, Any]] = []

    def dtype_of(t: Any) -> int:
        return _DTYPE[str(t.dtype)]

    def host(t: Any) -> np.ndarray:
        t = t.detach().contiguous()
        if t.dtype == torch.bfloat16:
            return t.view(torch.uint16).numpy().copy()
        return t.numpy().copy()

    def view_of(value: Any) -> View:
        return low.materialize(value)

    def finish(node: Any, value: Any) -> Any:
        # Materialise shared or deep expressions (the reference's rule: more than one reader, or depth >= 24).
        if isinstance(value, Expr) and (users[node.name] > 1 or value.depth >= MAX_DEPTH):
            return low.materialize(value)
        return value

    def elementwise(name: str, meta: Any, args: tuple[Any, ...], kwargs: dict[str, Any]) -> Any:
        dt = dtype_of(meta)
        if dt == I64:
            raise NotImplementedError(name)
        shape = tuple(meta.shape)
        bf = dt == BF16

        def rnd(e: Any) -> Any:
            return Expr("round", (e,), dt, shape, depth=_depth(e) + 1) if bf else e

        def mk(op: str, *xs: Any, imm: float = 0.0) -> Any:
            return rnd(Expr(op, tuple(xs), dt, shape, imm, 1 + max([_depth(x) for x in xs] + [0])))

        def scalar(v: Any, rounded: bool) -> Any:
            if isinstance(v, (View, Expr)):
                return v
            return _bf16(v) if rounded and bf else _f32(v)

        if name == "aten.clamp.default":
            low_, high = _arg(args, kwargs, 1, "min"), _arg(args, kwargs, 2, "max")
            x = args[0]
            if any(b is not None and math.isnan(b) for b in (low_, high)):
                return mk("mul", x, float("nan"))
            e: Any = x
            if low_ is not None:
                e = Expr("maxc", (e,), dt, shape, _f32(low_), _depth(e) + 1)
            if high is not None:
                e = Expr("minc", (e,), dt, shape, _f32(high), _depth(e) + 1)
            return rnd(e)
        if name in _UNARY:
            return mk(_UNARY[name], args[0])
        if name in _BINARY:
            alpha = kwargs.get("alpha", 1)
            rounded = name in ("aten.add.Tensor", "aten.sub.Tensor")
            a, b = scalar(args[0], rounded), scalar(args[1], rounded)
            if alpha != 1:
                b = mk("mul", b, _bf16(alpha) if bf else _f32(alpha))
            return mk(_BINARY[name], a, b)
        if name == "aten.rsub.Scalar":
            alpha = _arg(args, kwargs, 2, "alpha", 1)
            x, other = args[0], scalar(args[1], True)
            product = mk("mul", x, _bf16(alpha) if bf else _f32(alpha))
            return mk("sub", other, product)
        if name in ("aten.pow.Tensor_Scalar", "aten.pow.Scalar"):
            return mk("pow", scalar(args[0], True), scalar(args[1], True))
        raise NotImplementedError(name)

    def layout(name: str, node: Any, meta: Any, args: tuple[Any, ...], kwargs: dict[str, Any]) -> Any:
        x = args[0]
        if name in ("aten.to.dtype", "aten._to_copy.default"):
            dt = dtype_of(meta)
            xd = x.dtype
            if xd == dt:
                return x
            if I64 in (xd, dt):
                raise NotImplementedError(f"{_NAME[xd]} -> {_NAME[dt]}")
            shape = tuple(meta.shape)
            return Expr("round" if dt == BF16 else "cast", (x,), dt, shape, depth=_depth(x) + 1)
        if name in ("aten.clone.default", "aten.contiguous.default"):
            return x
        v = view_of(x)
        shape = tuple(meta.shape) if not isinstance(meta, (list, tuple)) else None
        if name in ("aten.view.default", "aten.reshape.default", "aten._unsafe_view.default"):
            if not v.contiguous():
                v = low.materialize(v, low.arena(v.dtype, v.shape))
            return View(v.kind, v.index, v.dtype, shape, _contiguous(shape), v.offset)
        strides = list(v.strides)
        if name in ("aten.split.Tensor", "aten.split_with_sizes.default"):
            dim = _axis(_arg(args, kwargs, 2, "dim", 0), len(v.shape))
            parts, offset = [], v.offset
            for part in meta:
                pshape = tuple(part.shape)
                parts.append(View(v.kind, v.index, v.dtype, pshape, tuple(strides), offset))
                offset += pshape[dim] * strides[dim]
            return tuple(parts)
        offset = v.offset
        if name == "aten.unsqueeze.default":
            strides.insert(_axis(args[1], len(shape)), 0)
        elif name == "aten.expand.default":
            return v.broadcast(shape)
        elif name == "aten.slice.Tensor":
            dim = _axis(_arg(args, kwargs, 1, "dim", 0), len(v.shape))
            start, _, step = slice(_arg(args, kwargs, 2, "start"), _arg(args, kwargs, 3, "end"),
                                   _arg(args, kwargs, 4, "step", 1)).indices(v.shape[dim])
            if step <= 0:
                raise NotImplementedError(f"slice step {step}")
            offset += start * strides[dim]
            strides[dim] *= step
        else:
            order = list(range(len(v.shape)))
            if name == "aten.permute.default":
                order = [_axis(d, len(v.shape)) for d in args[1]]
            elif len(order) > 1:
                a, b = (0, 1) if name == "aten.t.default" else (_axis(args[1], len(order)), _axis(args[2], len(order)))
                order[a], order[b] = order[b], order[a]
            strides = [strides[d] for d in order]
        return View(v.kind, v.index, v.dtype, shape, tuple(strides), offset)

    def constant(name: str, meta: Any, args: tuple[Any, ...], kwargs: dict[str, Any]) -> View:
        kw = {k: v for k, v in kwargs.items() if k in ("dtype",)}
        if name.startswith("aten.arange"):
            t = torch.arange(*args, **kw)
        elif name == "aten.full.default":
            t = torch.full(args[0], args[1], **kw)
        else:  # new_full(x, size, fill)
            t = torch.full(args[1], args[2], dtype=kw.get("dtype", meta.dtype))
        t = t.to(meta.dtype).reshape(meta.shape)
        low.constants += 1
        return low.weight(host(t), dtype_of(meta))

    def contract(meta: Any, a: View, b: View | None, out_idx_a: list[int], out_idx_b: list[int],
                 red_a: list[int], red_b: list[int], rshape: list[int], bias: View | None) -> View:
        shape = tuple(meta.shape)
        out = low.arena(dtype_of(meta), shape)
        extra_a = sum((n - 1) * abs(t) for n, t in zip(rshape, red_a))
        av = View(a.kind, a.index, a.dtype, shape, tuple(out_idx_a), a.offset, extra_a)
        if b is None:
            low.step(K_REDUCE, shape, out, **{"in": av}, rshape=tuple(rshape), rstride_a=tuple(red_a), rstride_b=(),
                     divisor=1.0)
            return out
        extra_b = sum((n - 1) * abs(t) for n, t in zip(rshape, red_b))
        bv = View(b.kind, b.index, b.dtype, shape, tuple(out_idx_b), b.offset, extra_b)
        low.step(K_CONTRACT, shape, out, **{"in": av, "in2": bv, "bias": bias}, rshape=tuple(rshape),
                 rstride_a=tuple(red_a), rstride_b=tuple(red_b))
        low.contractions += 1
        return out

    def linear(meta: Any, args: tuple[Any, ...], kwargs: dict[str, Any]) -> View:
        x, w = view_of(args[0]), view_of(args[1])
        bias = _arg(args, kwargs, 2, "bias")
        if any(v.dtype == I64 for v in (x, w)) or dtype_of(meta) == I64:
            raise NotImplementedError("linear on int64")
        shape = tuple(meta.shape)
        lead = len(shape) - 1
        a_out = list(x.strides[:-1]) + [0]
        b_out = [0] * lead + [w.strides[0]]
        bv = view_of(bias).broadcast(shape) if bias is not None else None
        return contract(meta, x, w, a_out, b_out, [x.strides[-1]], [w.strides[1]], [x.shape[-1]], bv)

    def einsum(meta: Any, equation: str, operands: list[Any]) -> View:
        eq = equation.replace(" ", "")
        if "->" not in eq or "." in eq or len(operands) not in (1, 2):
            raise NotImplementedError(f"einsum {equation}")
        lhs, out_labels = eq.split("->")
        labels = lhs.split(",")
        views = [view_of(v) for v in operands]
        reduction: list[str] = []
        for lab in labels:
            for c in lab:
                if c not in out_labels and c not in reduction:
                    reduction.append(c)
        sizes: dict[str, int] = {}
        for lab, v in zip(labels, views):
            for c, s in zip(lab, v.shape):
                if s != 1:
                    sizes[c] = s
        for c in out_labels + "".join(reduction):
            sizes.setdefault(c, 1)

        def strides_for(lab: str, v: View, which: str) -> list[int]:
            out = []
            for c in which:
                st = 0
                for pos, cc in enumerate(lab):
                    if cc == c and v.shape[pos] != 1:
                        st += v.strides[pos]
                out.append(st)
            return out

        red = "".join(reduction)
        a_out, a_red = strides_for(labels[0], views[0], out_labels), strides_for(labels[0], views[0], red)
        if len(views) == 1:
            return contract(meta, views[0], None, a_out, [], a_red, [], [sizes[c] for c in red], None)
        b_out, b_red = strides_for(labels[1], views[1], out_labels), strides_for(labels[1], views[1], red)
        return contract(meta, views[0], views[1], a_out, b_out, a_red, b_red, [sizes[c] for c in red], None)

    def reduction(name: str, meta: Any, args: tuple[Any, ...], kwargs: dict[str, Any]) -> View:
        x = args[0]
        dt = dtype_of(meta)
        if x.dtype == I64 or dt == I64:
            raise NotImplementedError(name)
        rank = len(x.shape)
        dims = _arg(args, kwargs, 1, "dim", []) or range(rank)
        axes = sorted({_axis(d, rank) for d in dims}) if rank else []
        keep = _arg(args, kwargs, 2, "keepdim", False)
        mean = name.startswith("aten.mean.")
        if not mean and x.dtype != dt:
            x = Expr("round" if dt == BF16 else "cast", (x,), dt, x.shape, depth=_depth(x) + 1)
        v = view_of(x)
        out_strides = []
        for d in range(rank):
            if d not in axes:
                out_strides.append(v.strides[d])
            elif keep:
                out_strides.append(0)
        shape = tuple(meta.shape)
        out = low.arena(dt, shape)
        rshape = [v.shape[d] for d in axes]
        count = math.prod(rshape) if mean else 1
        extra = sum((v.shape[d] - 1) * abs(v.strides[d]) for d in axes)
        low.step(K_REDUCE, shape, out, **{"in": View(v.kind, v.index, v.dtype, shape, tuple(out_strides), v.offset,
                                                     extra)},
                 rshape=tuple(rshape), rstride_a=tuple(v.strides[d] for d in axes), rstride_b=(),
                 divisor=float(count))
        return out

    def softmax(meta: Any, args: tuple[Any, ...]) -> View:
        x = args[0]
        dt = dtype_of(meta)
        if x.dtype != dt:
            x = Expr("round" if dt == BF16 else "cast", (x,), dt, x.shape, depth=_depth(x) + 1)
        v = view_of(x)
        shape = tuple(meta.shape)
        if not shape:
            v, shape1 = View(v.kind, v.index, v.dtype, (1,), (1,), v.offset), (1,)
        else:
            shape1 = shape
        dim = _axis(args[1], len(shape1)) if shape else 0
        out = low.arena(dt, shape)
        out1 = View(out.kind, out.index, out.dtype, shape1, _contiguous(shape1), out.offset)
        it = tuple(1 if d == dim else s for d, s in enumerate(shape1))
        low.step(K_SOFTMAX, it, out1, **{"in": v}, axis=dim, width=shape1[dim])
        return out

    def topk(meta: Any, args: tuple[Any, ...], kwargs: dict[str, Any]) -> tuple[View, View]:
        v = view_of(args[0])
        if v.dtype == I64:
            raise NotImplementedError("topk on int64")
        k = args[1]
        shape = tuple(meta[0].shape)
        if not shape:
            v, shape1 = View(v.kind, v.index, v.dtype, (1,), (1,), v.offset), (1,)
        else:
            shape1 = shape
        dim = _axis(_arg(args, kwargs, 2, "dim", -1), len(shape1)) if shape else 0
        width = v.shape[dim]
        if width > 4096:
            raise NotImplementedError(f"topk axis {width}")
        largest = _arg(args, kwargs, 3, "largest", True)
        values, indices = low.arena(v.dtype, shape), low.arena(I64, shape)
        vv = View(values.kind, values.index, values.dtype, shape1, _contiguous(shape1), values.offset)
        iv = View(indices.kind, indices.index, I64, shape1, _contiguous(shape1), indices.offset)
        it = tuple(1 if d == dim else s for d, s in enumerate(shape1))
        low.step(K_TOPK, it, vv, **{"in": v, "out2": iv}, axis=dim, width=width, k=k, largest=int(bool(largest)))
        return values, indices

    def gather(name: str, meta: Any, args: tuple[Any, ...]) -> View:
        negative = name == "aten.index.Tensor"
        if negative:
            idx = args[1]
            if len(idx) != 1 or idx[0] is None:
                raise NotImplementedError("index: one tensor, axis 0")
            table, ids = view_of(args[0]), view_of(idx[0])
        else:
            table, ids = view_of(args[0]), view_of(args[1])
        if ids.dtype != I64:
            raise NotImplementedError("index wants int64")
        shape = tuple(meta.shape)
        out = low.arena(table.dtype, shape)
        low.step(K_GATHER, shape, out, **{"in": table, "in2": ids}, negative=int(negative))
        return out

    def cat(meta: Any, args: tuple[Any, ...], kwargs: dict[str, Any]) -> View:
        shape = tuple(meta.shape)
        dim = _axis(_arg(args, kwargs, 1, "dim", 0), len(shape))
        out = low.arena(dtype_of(meta), shape)
        start = 0
        for part in args[0]:
            pshape = tuple(part.shape)
            dst = View(out.kind, out.index, out.dtype, pshape, out.strides, out.offset + start * out.strides[dim])
            low.materialize(part, dst)
            start += pshape[dim]
        return out

    def triangular(name: str, meta: Any, args: tuple[Any, ...], kwargs: dict[str, Any]) -> View:
        v = view_of(args[0])
        shape = tuple(meta.shape)
        out = low.arena(v.dtype, shape)
        low.step(K_MOVE, shape, out, **{"in": v}, tri=1 if name == "aten.triu.default" else 2,
                 diag=int(_arg(args, kwargs, 1, "diagonal", 0)))
        return out

    def resolve(a: Any) -> Any:
        if hasattr(a, "name") and hasattr(a, "op"):
            return env[a.name]
        if isinstance(a, (list, tuple)):
            return type(a)(resolve(x) for x in a)
        return a

    for node in program.graph.nodes:
        if node.op == "placeholder":
            spec = spec_of[node.name]
            meta = node.meta["val"]
            if spec.kind == InputKind.USER_INPUT:
                dt = dtype_of(meta)
                shape = tuple(meta.shape)
                env[node.name] = View(IN, len(inputs), dt, shape, _contiguous(shape))
                inputs.append({"name": node.name, "shape": list(shape), "dtype": _DTYPE_NAMES[str(meta.dtype)]})
            else:
                source = state if spec.target in state else constants
                t = source[spec.target]
                env[node.name] = low.weight(host(t), dtype_of(t))
            continue
        if node.op == "output":
            for k, arg in enumerate(node.args[0]):
                value = env[arg.name]
                meta = arg.meta["val"]
                shape = tuple(meta.shape)
                dt = dtype_of(meta)
                dst = View(OUT, k, dt, shape, _contiguous(shape))
                low.materialize(value, dst)
                outputs.append({"name": f"output_{k}", "shape": list(shape), "dtype": _DTYPE_NAMES[str(meta.dtype)]})
            continue
        name = _target(node)
        meta = node.meta.get("val")
        args, kwargs = resolve(tuple(node.args)), {k: resolve(v) for k, v in node.kwargs.items()}
        if node.target == operator.getitem:
            env[node.name] = args[0][args[1]]
            continue
        from chroma_b200._src.compiler import OPERATIONS

        kind = OPERATIONS.get(name)
        if kind == "metadata":
            env[node.name] = None
            continue
        if kind == "elementwise":
            value = elementwise(name, meta, args, kwargs)
        elif kind == "layout":
            value = layout(name, node, meta, args, kwargs)
        elif kind == "constant":
            value = constant(name, meta, args, kwargs)
        elif kind == "linear":
            value = linear(meta, args, kwargs)
        elif kind == "einsum":
            value = einsum(meta, args[0], list(args[1]))
        elif kind == "reduction":
            value = reduction(name, meta, args, kwargs)
        elif kind == "softmax":
            value = softmax(meta, args)
        elif kind == "topk":
            value = topk(meta, args, kwargs)
        elif kind == "gather":
            value = gather(name, meta, args)
        elif kind == "cat":
            value = cat(meta, args, kwargs)
        elif kind == "triangular":
            value = triangular(name, meta, args, kwargs)
        else:
            raise NotImplementedError(f"Unsupported runtime operation {node.target}")
        env[node.name] = finish(node, value)

    in_bytes = [max(1, math.prod(s["shape"])) * _ES[_DTYPE["torch." + s["dtype"]]] for s in inputs]
    out_bytes = [max(1, math.prod(s["shape"])) * _ES[_DTYPE["torch." + s["dtype"]]] for s in outputs]
    plan = {"desc": {"kind": 0, "weight_bytes": low.weight_bytes}, "graph": low.words(in_bytes, out_bytes)}
    stats = {"kernels": len(low.steps), "expressions": sum(1 for s in low.steps if s["kind"] == K_EW),
             "folded_constants": low.constants, "matrix_contractions": low.contractions,
             "workspace_bytes": low.arena_bytes, "unreused_workspace_bytes": low.arena_bytes, "generic_graph": True}
    return Lowered(plan, low.tensors, inputs, outputs, stats)


