"""Generic exported graphs (not GPT-OSS programs) exercising the reference's operator table the way its CUDA
acceptance tests do (tests/test_cuda.py:279-519 of the reference): fused elementwise chains over strided and
broadcast views, wide int64 values through views, linear on strided inputs, values shared across linear layers,
reductions, softmax, top-k with ties, NaN and infinities, gather with negative and out-of-range indices,
concatenation, triangles, einsum contractions, bf16 storage rounding with exact accumulation answers, non-finite
scalars, long chains, 0-d tensors and constant outputs.

Each case is (name, module factory, inputs factory, dtype tolerance). The goldens in tests/golden/generic.npz hold
the reference's own compiled CPU program's outputs for two input sets per case (tests/golden/make_generic.py).
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass
from typing import Any

import torch


class Fn(torch.nn.Module):
    def __init__(self, fn: Callable[..., Any]) -> None:
        super().__init__()
        self.fn = fn

    def forward(self, *args: torch.Tensor) -> Any:  # type: ignore[override]
        return self.fn(*args)


@dataclass
class Case:
    name: str
    module: Callable[[], torch.nn.Module]
    inputs: Callable[[], tuple[torch.Tensor, ...]]
    rtol: float = 2e-5
    atol: float = 5e-6
    unordered: bool = False  # top-k with sorted=False: the reference leaves the order of its k results open

    def input_sets(self) -> list[tuple[torch.Tensor, ...]]:
        """The inputs and a shifted copy (float inputs + 1), as the reference's check runs both."""
        first = self.inputs()
        second = tuple(x + 1 if x.is_floating_point() else x for x in first)
        return [first, second]


def _views_int64(x: torch.Tensor, y: torch.Tensor, ids: torch.Tensor) -> tuple[torch.Tensor, ...]:
    z = (x.cos() - y).clamp(-0.5, 0.75)
    return z, z, z.t().reshape(5, 8)[:, ::3], x, ids.t(), ids[:, 1:]


def _linear_strided(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> tuple[torch.Tensor, ...]:
    y = torch.nn.functional.linear(x[:, ::2], w.t(), b)
    return y.sigmoid(), y, torch.nn.functional.linear(x[:, 1::2] * 2, w.t())


def _shared(x: torch.Tensor, w: torch.Tensor) -> tuple[torch.Tensor, ...]:
    first = torch.nn.functional.linear(x, w)
    s = first.cos()
    second = torch.nn.functional.linear(s - 1, w)
    third = torch.nn.functional.linear(second * s, w)
    return third, first[:, 2:], s


def _reductions(x: torch.Tensor, y: torch.Tensor, ids: torch.Tensor) -> tuple[torch.Tensor, ...]:
    sel = x[ids]
    values, indices = sel.topk(3, dim=0, largest=False)
    return (sel.sum(0), sel.mean(1, keepdim=True), sel.softmax(1), values, indices, torch.cat((sel, y), dim=0),
            torch.triu(sel, 1), torch.tril(sel, -1), torch.einsum("ij,kj->ik", sel, y))


def _int64_ops(x: torch.Tensor, ids: torch.Tensor) -> tuple[torch.Tensor, ...]:
    sel = x[ids]
    return sel, torch.cat((sel, x[:2]), dim=0), torch.triu(x, 1), torch.tril(x, -1)


def _strided_nonfinite(x: torch.Tensor) -> tuple[torch.Tensor, ...]:
    y = x.t()[::2]
    values, indices = y.topk(2, dim=1, largest=False)
    return y, y.sum(1), y.mean(0), y.softmax(1), values, indices, torch.triu(y, -1)


def _warp(x: torch.Tensor) -> tuple[torch.Tensor, ...]:
    return x.sum((0, 2)), x.mean(-1, keepdim=True), x.softmax(1), (x * x).sum(-1)


def _contractions(a, b, c, d, e, f, g, h):  # type: ignore[no-untyped-def]
    return (torch.einsum("ij,j->i", a, b), torch.einsum("bik,bkj->bij", c, d), torch.einsum("km,kn->mn", e, f),
            torch.einsum("ij,ik->ijk", g, h))


def _bf16_rounding(x: torch.Tensor, y: torch.Tensor, one: torch.Tensor) -> tuple[torch.Tensor, ...]:
    r = y.bfloat16()
    return x.cos() + x, r, r.float(), (one + 2**-8) + 2**-8, (one * 0.333984375) - 0.333


def _bf16_linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> tuple[torch.Tensor, ...]:
    return torch.nn.functional.linear(x, w, b), torch.einsum("mk,nk->mn", x, w), w.sum(dim=1)


def _chain(x: torch.Tensor) -> tuple[torch.Tensor, ...]:
    z = x.clamp(-1.5, 1.5)
    for _ in range(60):
        z = z.clamp(-1.5, 1.5)
    return z, torch.add(x, x, alpha=0.75), torch.rsub(x, 2, alpha=0.25), 3.0**x, x.clamp(min=float("nan"))


def _rmsnorm(dtype: torch.dtype) -> torch.nn.Module:
    from chroma_b200.models import RMSNorm

    return RMSNorm(33).to(dtype).eval()


def _linspace(n: int, shape: tuple[int, ...], lo: float = -1.0, hi: float = 1.0) -> torch.Tensor:
    return torch.linspace(lo, hi, n).reshape(shape)


def _seeded(seed: int, *shapes: tuple[int, ...], dtype: torch.dtype = torch.float32) -> tuple[torch.Tensor, ...]:
    g = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(s, generator=g).to(dtype) for s in shapes)


def _nonfinite_matrix() -> tuple[torch.Tensor]:
    (x,) = _seeded(17, (13, 6))
    x[3, 1] = float("nan")
    x[6, 4] = float("inf")
    x[10, 0] = -float("inf")
    return (x,)


_TIED = [[3.0, 1.0, 0.0], [3.0, 1.0, 0.0], [1.0, 3.0, 0.0], [1.0, 3.0, 2.0], [0.0, 2.0, 2.0], [0.0, 2.0, 2.0]]


def cases() -> list[Case]:
    big = torch.tensor([[2**61 + 5, -(2**61) - 9, 2**41], [-13, 2**62 - 3, 7]], dtype=torch.int64)
    out: list[Case] = [
        Case("views_int64", lambda: Fn(_views_int64),
             lambda: (_linspace(40, (8, 5), -3, 3), torch.full((5,), 0.5), big.clone())),
        Case("linear_strided", lambda: Fn(_linear_strided), lambda: _seeded(42, (12, 20), (10, 6), (6,))),
        Case("linear_vector", lambda: _module(41, torch.nn.Linear(11, 5)), lambda: _seeded(43, (11,))),
        Case("linear_batched_nobias", lambda: _module(44, torch.nn.Linear(11, 5, bias=False)),
             lambda: _seeded(45, (2, 4, 11))),
        Case("shared_values", lambda: Fn(_shared), lambda: (_seeded(46, (4, 9))[0], torch.eye(9) * 0.5)),
        Case("int64_gather_cat_triangle", lambda: Fn(_int64_ops),
             lambda: (torch.arange(20, dtype=torch.int64).reshape(5, 4), torch.tensor([4, -1, 0]))),
        Case("strided_nonfinite", lambda: Fn(_strided_nonfinite), _nonfinite_matrix, 2e-4, 2e-5),
        Case("contractions", lambda: Fn(_contractions), lambda: (
            _linspace(4 * 257, (4, 257)), _linspace(257, (257,), 0.5, 1.5), _linspace(2 * 3 * 13, (2, 3, 13)),
            _linspace(13 * 5, (1, 13, 5), 1, -1), _linspace(13 * 3, (13, 3), -0.5, 0.5),
            _linspace(13 * 5, (13, 5), 0.75, -0.75), _linspace(6, (2, 3)), _linspace(8, (2, 4), 1, -1)), 5e-4, 2e-4),
        Case("bf16_rounding", lambda: Fn(_bf16_rounding), lambda: (
            torch.linspace(-1, 1, 16).bfloat16(),
            torch.tensor([1 + 2**-8, 1 + 3 * 2**-8, -1 - 2**-8, -1 - 3 * 2**-8, float("inf"), float("nan")]),
            torch.ones(1, dtype=torch.bfloat16)), 0.0, 0.0),
        Case("bf16_linear_exact", lambda: Fn(_bf16_linear), _bf16_linear_inputs, 0.0, 0.0),
        Case("nonfinite_chain", lambda: Fn(_chain),
             lambda: (torch.tensor([-float("inf"), -2.5, 0.25, float("inf"), float("nan")]),)),
        Case("scalar_0d", lambda: Fn(lambda x: x.cos() * 2 + 1), lambda: (torch.tensor(0.25),)),
        Case("constant_outputs", lambda: Fn(lambda x: (torch.arange(5), torch.full((2, 2), 1.5) + x)),
             lambda: (torch.ones(1),)),
        Case("identity", lambda: torch.nn.Identity(), lambda: (torch.arange(8, dtype=torch.float32),)),
    ]
    for dtype, rtol, atol in ((torch.float32, 2e-4, 2e-5), (torch.bfloat16, 0.03, 0.01)):
        tag = "f32" if dtype == torch.float32 else "bf16"
        out += [
            Case(f"reductions_{tag}", lambda: Fn(_reductions), lambda dtype=dtype: (
                torch.arange(-14, 14, dtype=torch.float32).reshape(7, 4).to(dtype),
                _seeded(9, (2, 4), dtype=dtype)[0], torch.tensor([5, -3, 0, 3])), rtol, atol),
            Case(f"warp_{tag}", lambda: Fn(_warp),
                 lambda dtype=dtype: (_linspace(3 * 33 * 19, (3, 33, 19), -3, 3).to(dtype),), rtol, atol),
            Case(f"rmsnorm_{tag}", lambda dtype=dtype: _rmsnorm(dtype),
                 lambda dtype=dtype: _seeded(47, (4, 33), dtype=dtype), rtol, atol),
        ]
    for largest in (True, False):
        out.append(Case(f"topk_ties_{'largest' if largest else 'smallest'}",
                        lambda largest=largest: Fn(lambda x: torch.topk(x, 4, dim=0, largest=largest, sorted=False)),
                        lambda: (torch.tensor(_TIED),), 0.0, 0.0, unordered=True))
    return out


def _module(seed: int, module: torch.nn.Module) -> torch.nn.Module:
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for p in module.parameters():
            p.copy_(torch.randn(p.shape, generator=g))
    return module.eval()


def _bf16_linear_inputs() -> tuple[torch.Tensor, ...]:
    x = torch.ones(2, 17, dtype=torch.bfloat16)
    w = torch.full((5, 17), 2**-8, dtype=torch.bfloat16)
    w[:, 0] = 1
    b = torch.full((5,), 2**-5, dtype=torch.bfloat16)
    return x, w, b


def by_name() -> dict[str, Case]:
    return {c.name: c for c in cases()}


def to_numpy(t: torch.Tensor) -> Any:
    """Host array in the manifest's representation (bf16 as ml_dtypes.bfloat16)."""
    from ml_dtypes import bfloat16

    t = t.detach().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.uint16).numpy().view(bfloat16)
    return t.numpy()


def golden_arrays(data: Any, name: str, which: str, index: int) -> list[Any]:
    """Arrays ``in``/``out`` of input set ``index`` of case ``name`` from tests/golden/generic.npz."""
    from ml_dtypes import bfloat16

    out, k = [], 0
    while f"{name}/{which}{index}_{k}" in data:
        a = data[f"{name}/{which}{index}_{k}"]
        out.append(a.view(bfloat16) if str(data[f"{name}/{which}{index}_{k}_dtype"]) == "bfloat16" else a)
        k += 1
    return out


def compare(case: Case, got: list[Any], want: list[Any], inputs: list[Any]) -> float:
    """Every output against the reference's: int64 exactly, floats within the case's tolerance (NaN where the
    reference has NaN). Unordered top-k results: the same values as a multiset, each value the input's at its index,
    distinct indices. Returns the share of float elements that are bit-identical to the reference's."""
    import numpy as np

    same = total = 0
    if case.unordered:
        (x,) = inputs
        values, indices = got
        np.testing.assert_array_equal(np.sort(values, axis=0), np.sort(want[0], axis=0))
        np.testing.assert_array_equal(values, np.take_along_axis(np.asarray(x), indices, axis=0))
        assert all(len(set(col.tolist())) == len(col) for col in indices.T)
        return 1.0
    assert len(got) == len(want)
    for g, w in zip(got, want):
        g, w = np.asarray(g), np.asarray(w)
        assert g.shape == w.shape and g.dtype == w.dtype, (g.shape, w.shape, g.dtype, w.dtype)
        if g.dtype == np.int64:
            np.testing.assert_array_equal(g, w)
            continue
        gf, wf = g.astype(np.float32), w.astype(np.float32)
        np.testing.assert_allclose(gf, wf, rtol=case.rtol, atol=case.atol, equal_nan=True)
        bits = g.view(np.uint16 if g.dtype.itemsize == 2 else np.uint32)
        wbits = w.view(bits.dtype)
        same += int(np.sum((bits == wbits) | (np.isnan(gf) & np.isnan(wf))))
        total += g.size
    return same / total if total else 1.0
