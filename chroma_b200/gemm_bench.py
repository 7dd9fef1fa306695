"""Microbenchmark of the tensor-core GEMM (``chroma_b200_gemm_bf16``): ``python -m chroma_b200.gemm_bench``.

Times C = A . B^T for GPT-OSS-20B-shaped problems with CUDA events (L2 flushed before each launch) and prints one
JSON line per shape with achieved TFLOP/s. Used as the small, self-contained case for kernel profiling.
"""

from __future__ import annotations

import argparse
import json
import statistics

import torch

from chroma_b200._src import native as nat

SHAPES = {
    "qkv": (8192, 5120, 2880, 0, 1),
    "out": (8192, 2880, 4096, 0, 1),
    "moe_up": (32768, 5760, 2880, 2, 32),
    "moe_down": (32768, 2880, 2880, 3, 32),
}


def run(m: int, n: int, k: int, epi: int, groups: int, reps: int, stream: torch.cuda.Stream) -> dict:
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    b = (torch.randn(groups * n, k, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    bias = torch.zeros(groups, n, dtype=torch.bfloat16, device="cuda")
    c = torch.empty(m, n // 2 if epi == 2 else n, dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    offsets = torch.arange(groups + 1, dtype=torch.int32, device="cuda") * (m // groups) if groups > 1 else None
    scratch = torch.zeros(groups + 1, dtype=torch.int32, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    ptr = lambda t: nat._VP(t.data_ptr()) if t is not None else None  # noqa: E731

    def call() -> None:
        nat.call("chroma_b200_gemm_bf16", ptr(a), ptr(b), ptr(bias), None, ptr(c), m, n, k, epi, 1.702, 7.0, groups,
                 ptr(offsets), ptr(scratch), ptr(err), nat._VP(stream.cuda_stream))

    times = []
    for i in range(reps + 2):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        call()
        e1.record(stream)
        if i >= 2:
            times.append((e0, e1))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ms = statistics.median(a_.elapsed_time(b_) for a_, b_ in times)
    flops = 2.0 * m * n * k
    return {"m": m, "n": n, "k": k, "groups": groups, "ms": ms, "tflops": flops / ms / 1e9}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", nargs="*", default=list(SHAPES))
    ap.add_argument("--reps", type=int, default=10)
    args = ap.parse_args()
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    for name in args.shapes:
        print(json.dumps({"shape": name, **run(*SHAPES[name], args.reps, stream)}), flush=True)


if __name__ == "__main__":
    main()
