"""tcgen05 bf16 GEMM (``chroma_b200_gemm_bf16``) against a torch fp32 reference of the same op.

Tolerance: the kernel accumulates in fp32 and rounds once (per epilogue step) to bf16, like the reference's bf16
linear (chroma/_src/codegen/cpu/kernels.h:63-74); the torch reference rounds the fp32 product the same way, so
results agree to 1 bf16 ulp: rtol 1e-2, atol 1e-2 x the output scale.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import ctypes

import numpy as np
import pytest
import torch

from chroma_b200._src import native as nat

pytestmark = pytest.mark.gpu

STORE, RESIDUAL, SWIGLU, EXPERT = 0, 1, 2, 3


def gemm(a, b, bias=None, residual=None, epi=STORE, groups=1, offsets=None, n=None):  # type: ignore[no-untyped-def]
    m, k = a.shape
    n = n or b.shape[0] // groups
    cols = n // 2 if epi == SWIGLU else n
    c = torch.full((m, cols), float("nan"), dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    scratch = torch.zeros(groups + 1, dtype=torch.int32, device="cuda")
    ptr = lambda t: nat._VP(t.data_ptr()) if t is not None else None  # noqa: E731
    nat.call("chroma_b200_gemm_bf16", ptr(a), ptr(b), ptr(bias), ptr(residual), ptr(c), m, n, k, epi, 1.702, 7.0,
             groups, ptr(offsets), ptr(scratch), ptr(err), nat._VP(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert int(err.item()) == 0, f"GEMM error word {int(err.item())}"
    return c


def r16(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).float()


def reference(a, b, bias, residual, epi):  # type: ignore[no-untyped-def]
    acc = a.float() @ b.float().T
    if epi == STORE:
        return r16(acc + (bias.float() if bias is not None else 0))
    if epi == RESIDUAL:
        return r16(residual.float() + r16(acc + bias.float()))
    if epi == EXPERT:
        return r16(r16(acc) + bias.float())
    h = r16(r16(acc) + bias.float())
    glu, lin = h[:, ::2].clamp(max=7.0), h[:, 1::2].clamp(-7.0, 7.0)
    og = r16(glu * r16(torch.sigmoid(r16(glu * 1.702))))
    return r16(og * r16(lin + 1))


def check(got: torch.Tensor, want: torch.Tensor) -> None:
    scale = float(want.abs().max()) + 1e-6
    np.testing.assert_allclose(got.float().cpu().numpy(), want.cpu().numpy(), rtol=1e-2, atol=1e-2 * scale)


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (200, 300, 2880), (1000, 32, 2880), (4096, 5120, 2880), (77, 64, 4096)])
def test_dense_store(gpu: None, m: int, n: int, k: int) -> None:
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    b = (torch.randn(n, k, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    bias = torch.randn(n, generator=g, device="cuda").to(torch.bfloat16)
    check(gemm(a, b, bias), reference(a, b, bias, None, STORE))
    check(gemm(a, b, None), reference(a, b, None, None, STORE))


def test_dense_residual_and_repeat(gpu: None) -> None:
    g = torch.Generator(device="cuda").manual_seed(1)
    m, n, k = 300, 2880, 4096
    a = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    b = (torch.randn(n, k, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    bias = torch.randn(n, generator=g, device="cuda").to(torch.bfloat16)
    res = torch.randn(m, n, generator=g, device="cuda").to(torch.bfloat16)
    want = reference(a, b, bias, res, RESIDUAL)
    check(gemm(a, b, bias, res, RESIDUAL), want)
    check(gemm(a, b, bias, res, RESIDUAL), want)


def test_grouped_swiglu_and_expert(gpu: None) -> None:
    g = torch.Generator(device="cuda").manual_seed(2)
    E, k, i2 = 8, 2880, 5760
    counts = [0, 130, 1, 257, 0, 64, 500, 7]
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    m = int(offsets[-1])
    a = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    w1 = (torch.randn(E * i2, k, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    b1 = torch.randn(E, i2, generator=g, device="cuda").to(torch.bfloat16)
    off = torch.from_numpy(offsets).cuda()
    got = gemm(a, w1, b1, epi=SWIGLU, groups=E, offsets=off, n=i2)
    want = torch.empty(m, i2 // 2, device="cuda")
    for e in range(E):
        lo, hi = int(offsets[e]), int(offsets[e + 1])
        if hi > lo:
            want[lo:hi] = reference(a[lo:hi], w1[e * i2 : (e + 1) * i2], b1[e], None, SWIGLU)
    check(got, want)
    w2 = (torch.randn(E * k, i2 // 2, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    b2 = torch.randn(E, k, generator=g, device="cuda").to(torch.bfloat16)
    got2 = gemm(got, w2, b2, epi=EXPERT, groups=E, offsets=off, n=k)
    want2 = torch.empty(m, k, device="cuda")
    for e in range(E):
        lo, hi = int(offsets[e]), int(offsets[e + 1])
        if hi > lo:
            want2[lo:hi] = reference(got[lo:hi], w2[e * k : (e + 1) * k], b2[e], None, EXPERT)
    check(got2, want2)


def test_pair_kernel_dense_residual_ragged(gpu: None, monkeypatch: pytest.MonkeyPatch) -> None:
    """The CTA-pair kernel on dense problems (forced; by default it serves only the grouped SwiGLU GEMM): 256-row
    tiles that end mid-tile, N not a multiple of 256. Runs in a subprocess so the environment switch is read fresh."""
    import subprocess

    code = "import tests.test_gpu_gemm as t; t._pair_dense_body()"
    env = dict(os.environ, CHROMA_B200_PAIR_GEMM="1")
    subprocess.run([sys.executable, "-c", code], check=True, env=env, cwd=str(Path(__file__).resolve().parents[1]))


def _pair_dense_body() -> None:
    g = torch.Generator(device="cuda").manual_seed(5)
    m, n, k = 3000, 2880, 4096
    a = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    b = (torch.randn(n, k, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    bias = torch.randn(n, generator=g, device="cuda").to(torch.bfloat16)
    res = torch.randn(m, n, generator=g, device="cuda").to(torch.bfloat16)
    check(gemm(a, b, bias, res, RESIDUAL), reference(a, b, bias, res, RESIDUAL))
    check(gemm(a, b, bias), reference(a, b, bias, None, STORE))


def test_pair_kernel_grouped_ragged(gpu: None) -> None:
    """Grouped problems of >= 8192 rows take the CTA-pair kernel; groups end inside 256-row tiles, some are empty."""
    g = torch.Generator(device="cuda").manual_seed(6)
    E, k, i2 = 8, 2880, 5760
    counts = [0, 2050, 1, 3000, 0, 777, 2500, 7]
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    m = int(offsets[-1])
    a = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    w1 = (torch.randn(E * i2, k, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    b1 = torch.randn(E, i2, generator=g, device="cuda").to(torch.bfloat16)
    off = torch.from_numpy(offsets).cuda()
    got = gemm(a, w1, b1, epi=SWIGLU, groups=E, offsets=off, n=i2)
    want = torch.empty(m, i2 // 2, device="cuda")
    for e in range(E):
        lo, hi = int(offsets[e]), int(offsets[e + 1])
        if hi > lo:
            want[lo:hi] = reference(a[lo:hi], w1[e * i2 : (e + 1) * i2], b1[e], None, SWIGLU)
    check(got, want)
    w2 = (torch.randn(E * k, i2 // 2, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    b2 = torch.randn(E, k, generator=g, device="cuda").to(torch.bfloat16)
    got2 = gemm(got, w2, b2, epi=EXPERT, groups=E, offsets=off, n=k)
    want2 = torch.empty(m, k, device="cuda")
    for e in range(E):
        lo, hi = int(offsets[e]), int(offsets[e + 1])
        if hi > lo:
            want2[lo:hi] = reference(got[lo:hi], w2[e * k : (e + 1) * k], b2[e], None, EXPERT)
    check(got2, want2)


def test_narrow_tail_tiles_match_full_width(gpu: None, tmp_path: Path) -> None:
    """A last column tile of at most 128 columns runs as a narrow MMA scheduled after the full-width tiles. The same
    cases with that split (default) and without it (CHROMA_B200_GEMM_TAIL=0), each in a fresh process so the switch
    is read anew: N = 2,880 (a 64-column tail), N = 300 (44 columns, MMA width 48), the grouped SwiGLU GEMM with
    N = 5,760 (128) and the grouped expert GEMM with N = 2,880 over ragged groups. Both give the same bits, and the
    split run matches the torch reference."""
    import subprocess

    root = str(Path(__file__).resolve().parents[1])
    outs = {}
    for mode in ("1", "0"):
        path = tmp_path / f"tail{mode}.pt"
        code = f"import tests.test_gpu_gemm as t; t._tail_body({str(path)!r})"
        env = dict(os.environ, CHROMA_B200_GEMM_TAIL=mode)
        subprocess.run([sys.executable, "-c", code], check=True, env=env, cwd=root)
        outs[mode] = torch.load(path)
    for name, (got, want) in outs["1"].items():
        check(got.cuda(), want.cuda())
        assert torch.equal(got, outs["0"][name][0]), f"{name}: narrow tail tiles differ from full-width ones"


def _tail_body(path: str) -> None:
    g = torch.Generator(device="cuda").manual_seed(9)
    res: dict[str, tuple[torch.Tensor, torch.Tensor]] = {}
    for m, n, k in [(1200, 2880, 2880), (333, 300, 4096)]:
        a = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
        b = (torch.randn(n, k, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        bias = torch.randn(n, generator=g, device="cuda").to(torch.bfloat16)
        r = torch.randn(m, n, generator=g, device="cuda").to(torch.bfloat16)
        res[f"store{m}"] = (gemm(a, b, bias), reference(a, b, bias, None, STORE))
        res[f"residual{m}"] = (gemm(a, b, bias, r, RESIDUAL), reference(a, b, bias, r, RESIDUAL))
    E, k, i2 = 8, 2880, 5760
    counts = [0, 130, 1, 257, 0, 64, 500, 7]
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    m = int(offsets[-1])
    off = torch.from_numpy(offsets).cuda()
    a = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    w1 = (torch.randn(E * i2, k, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    b1 = torch.randn(E, i2, generator=g, device="cuda").to(torch.bfloat16)
    h = gemm(a, w1, b1, epi=SWIGLU, groups=E, offsets=off, n=i2)
    w2 = (torch.randn(E * k, i2 // 2, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    b2 = torch.randn(E, k, generator=g, device="cuda").to(torch.bfloat16)
    y = gemm(h, w2, b2, epi=EXPERT, groups=E, offsets=off, n=k)
    want_h = torch.empty(m, i2 // 2, device="cuda")
    want_y = torch.empty(m, k, device="cuda")
    for e in range(E):
        lo, hi = int(offsets[e]), int(offsets[e + 1])
        if hi > lo:
            want_h[lo:hi] = reference(a[lo:hi], w1[e * i2 : (e + 1) * i2], b1[e], None, SWIGLU)
            want_y[lo:hi] = reference(h[lo:hi], w2[e * k : (e + 1) * k], b2[e], None, EXPERT)
    res["swiglu"] = (h, want_h)
    res["expert"] = (y, want_y)
    torch.save({name: (got.cpu(), want.cpu()) for name, (got, want) in res.items()}, path)
