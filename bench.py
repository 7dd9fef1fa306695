"""Benchmark: the dev model's KV-cached greedy decode step on B200 (config C2), plus the 8-token forward (C1).

Headline metric: decode tokens/s at batch 1 per GPU with a 256-token fp32 KV cache (the reference publishes a
3.27 ms cached decode step on an A100, docs/benchmarks.md:37, i.e. 305.8 tokens/s). One "step" = one decode step
of every sequence: embedding, 12 layers (norm, QKV, RoPE, sink attention over the cache, out-projection, router,
4 experts), final norm, the 201,088-way vocab projection, greedy argmax, KV commit and position advance.

* ``value``: device-resident greedy decoding (``BatchDecoder.advance_device``: no host transfer inside the timed
  region), CUDA events around each step on the launching stream, L2 flushed (256 MiB write) before every timed step.
* ``e2e``: the public ``Decoder.append([token])`` API from host arrays, logits [1, V] returned to the host, per
  step wall clock (the call synchronises), L2 flushed before every step.
* ``batch64`` and ``fwd8``: the same two measurements for 64 sequences and for ``Program(tokens[8])``.
* ``roofline``: the vocab-projection kernel (the dominant one) launched alone after an L2 flush, CUDA events.
* ``cpu_baseline``: the reference's own compiled CPU program for this decode step (``oracle/_ref``), 1 thread.

``--impl reference`` times the reference's CPU decode step instead (rank 0 only).
Multi-GPU (torchrun): one replica per GPU (the dev model does not shard); value = all ranks' tokens / max time.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

A100_DECODE_STEP_MS = 3.27  # reference, docs/benchmarks.md:37
# The reference's compiled CPU program (blas=False, 1 thread) for one C4-width layer over 16 tokens plus the vocab
# projection of those 16 rows (oracle/_ref/c4_slice_fwd16): 22.5 GFLOP in 10.59 s = 2.12 GFLOP/s, timed in the
# build container (the 3.9 GB program does not travel to the GPU hosts). C4/C5 CPU baselines extrapolate by FLOPs.
REF_CPU_GFLOPS = 22.5 / 10.59
A100_FWD8_MS = 4.25  # reference, docs/benchmarks.md:23
CONTEXT = 256
PREFILL = 8
DATA = "synthetic (seeded dev-model weights as scripts/export.py:16-29, seeded token ids)"
# DRAM bytes of one k_vocab launch of this workload, from an ncu capture (102.98 MB read + 3.87 MB written).
VOCAB_NCU_TRAFFIC = 106_851_584
CLUSTER_NCU_TRAFFIC = 30_900_789  # one k_decode_cluster launch of this workload, caches flushed (ncu)


def parse() -> argparse.Namespace:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--skip-c4", action="store_true", help="skip the GPT-OSS-20B-shaped prefill measurement")
    ap.add_argument("--c4-only", action="store_true", help="run only the GPT-OSS-20B-shaped prefill measurement")
    ap.add_argument("--c4-layers", type=int, default=0, help="layers of the C4 model (0: all 24; fewer for profiling)")
    ap.add_argument("--decode-only", action="store_true", help="only the headline decode measurement (profiling)")
    ap.add_argument("--fwd8-only", action="store_true", help="only the 8-token forward (C1) measurement (profiling)")
    ap.add_argument("--decode-batch", type=int, default=1, help="sequences of the --decode-only measurement")
    ap.add_argument("--skip-c5", action="store_true", help="skip the GPT-OSS-120B-shaped decode (multi-GPU runs)")
    ap.add_argument("--c5-only", action="store_true", help="run only the GPT-OSS-120B-shaped decode (needs >= 2 GPUs)")
    ap.add_argument("--c5-layers", type=int, default=0, help="layers of the C5 model (0: all 36)")
    ap.add_argument("--c5-sequences", type=int, default=256, help="sequences of the C5 decode over all GPUs")
    ap.add_argument("--skip-parity", action="store_true", help="skip the expert-parallel bit-identity check")
    ap.add_argument("--gemm", nargs="*", choices=sorted(GEMM_SHAPES), default=None,
                    help="only the tensor-core GEMM at GPT-OSS-20B shapes (all shapes when none is named): one JSON "
                         "line per shape, CUDA events, L2 flushed before each launch, median of --steps launches")
    return ap.parse_args()


# ---------------------------------------------------------------------------------------------------------
# The tensor-core GEMM (chroma_b200_gemm_bf16) alone at the C4 shapes: (M, N, K, epilogue, expert groups).
GEMM_SHAPES = {
    "qkv": (8192, 5120, 2880, 0, 1),
    "out": (8192, 2880, 4096, 0, 1),
    "moe_up": (32768, 5760, 2880, 2, 32),
    "moe_down": (32768, 2880, 2880, 3, 32),
}


def bench_gemm(name: str, reps: int, warmup: int) -> dict:
    import torch

    from chroma_b200._src import native as nat

    m, n, k, epi, groups = GEMM_SHAPES[name]
    stream = torch.cuda.current_stream()
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    b = (torch.randn(groups * n, k, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    bias = torch.zeros(groups, n, dtype=torch.bfloat16, device="cuda")
    c = torch.empty(m, n // 2 if epi == 2 else n, dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    offsets = torch.arange(groups + 1, dtype=torch.int32, device="cuda") * (m // groups) if groups > 1 else None
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    ptr = lambda t: nat._VP(t.data_ptr()) if t is not None else None  # noqa: E731
    times = []
    for i in range(warmup + reps):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        nat.call("chroma_b200_gemm_bf16", ptr(a), ptr(b), ptr(bias), None, ptr(c), m, n, k, epi, 1.702, 7.0, groups,
                 ptr(offsets), None, ptr(err), nat._VP(stream.cuda_stream))
        e1.record(stream)
        if i >= warmup:
            times.append((e0, e1))
    torch.cuda.synchronize()
    if int(err.item()):
        raise RuntimeError(f"GEMM error word {int(err.item())}")
    ms = statistics.median(x.elapsed_time(y) for x, y in times)
    return {"gemm": name, "m": m, "n": n, "k": k, "groups": groups, "ms": ms, "tflops": 2.0 * m * n * k / ms / 1e9}


# ---------------------------------------------------------------------------------------------------------
class Clocks:
    """nvidia-smi sampling of SM clock and throttle reasons during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int) -> None:
        self.index = index
        self.proc: subprocess.Popen | None = None

    def __enter__(self) -> "Clocks":
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc: object) -> None:
        time.sleep(0.2)
        self.samples: list[list[str]] = []
        if self.proc is not None:
            self.proc.terminate()
            out, _ = self.proc.communicate(timeout=10)
            self.samples = [[x.strip() for x in line.split(",")] for line in out.splitlines() if line.count(",") >= 7]

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for s in self.samples for n, v in zip(names, s[4:8]) if v.strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data["hbm_gbs"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


# ---------------------------------------------------------------------------------------------------------
def cpu_reference_decode(seconds: float, steps: int | None = None) -> dict:
    """The reference's compiled CPU decode step (oracle/_ref/c2_*) driven by the reference's own ``chroma.Decoder``
    and ``chroma.Program`` (the stock host path: per-step masks, full-cache inputs, cache copy on commit), from the
    patched copy of its package staged under oracle/_ref. Falls back to the NumPy oracle port if the reference
    programs or package were not built."""
    tokens = np.random.default_rng(7).integers(0, 201088, 4096)
    try:
        from oracle import refimport
        from oracle.refprogram import ROOT as REF_ROOT, available

        if not (available("c2_prefill8") and available("c2_decode")):
            raise FileNotFoundError("oracle/_ref/c2_* not built")
        chroma = refimport.runtime()
        dec = chroma.Decoder(chroma.Program(REF_ROOT / "c2_prefill8"), chroma.Program(REF_ROOT / "c2_decode"))
        kind = "reference"
        step = lambda t: dec.append([int(t)])  # noqa: E731
        dec.append(tokens[:PREFILL])
    except (FileNotFoundError, ModuleNotFoundError, ImportError, OSError) as exc:
        from oracle import gpt_oss as og
        from tests.helpers import dev_oracle

        cfg, p = dev_oracle()
        odec = og.Decoder(cfg, p, CONTEXT, PREFILL)
        odec.append(tokens[:PREFILL])
        kind = f"port ({exc})"
        step = lambda t: odec.append([int(t)])  # noqa: E731
    step(tokens[PREFILL])  # warm-up
    n, start = 0, time.perf_counter()
    while True:
        step(tokens[PREFILL + 1 + n % 2000])
        n += 1
        elapsed = time.perf_counter() - start
        if (steps is not None and n >= steps) or (steps is None and elapsed >= seconds and n >= 8):
            break
    return {"value": n / elapsed, "unit": "tokens/s", "cores": 1, "kind": kind.split(" ")[0],
            "ms_per_step": 1e3 * elapsed / n,
            "sample": f"{n} cached decode steps (batch 1, 256-token cache, after an 8-token prefill) through the "
                      f"reference's chroma.Decoder over its compiled single-threaded C++ programs (blas=False)"
                      + ("" if kind == "reference" else f"; {kind}")}


def c2_config(world: int) -> dict:
    """The headline workload's ``config``, printed identically by both arms."""
    return {"workload": "C2: dev GPT-OSS (12 layers, d=128, 59.1M params) KV-cached greedy decode step, 256-token "
                        "fp32 cache, 8-token prefill first, batch 1 per sequence",
            "model": "gpt-oss dev", "global_batch": world, "seq_len": CONTEXT,
            "parallelism": f"replicas x{world} (the dev model does not shard)",
            "l2": "flushed before every timed step (256 MiB write, then 256 MiB read)"}


def reference_arm(args: argparse.Namespace) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cpu_reference_decode(0, steps=max(1, args.warmup))
    res = cpu_reference_decode(0, steps=args.steps)
    line = {
        "impl": "reference", "metric": "dev decode tokens/s (KV cache 256, batch 1)", "value": res["value"],
        "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": res["ms_per_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": DATA,
        "config": c2_config(args.gpus),
        "execution": "rank 0 only: the reference's compiled CPU decode step on 1 host thread",
        "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": res["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------------------
def prefill_flops(cfg, batch: int, n: int) -> float:  # type: ignore[no-untyped-def]
    """Algorithmic FLOPs of one batched prefill chunk (GEMMs + causal attention + the last-row vocab projection)."""
    d, H, KV, hd, E, k, I = (cfg.hidden_size, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim,
                             cfg.num_experts, cfg.experts_per_token, cfg.intermediate_size)
    N = batch * n
    gemm = 2 * N * ((H + 2 * KV) * hd * d + d * H * hd + E * d + k * (2 * I * d + d * I))
    attention = batch * H * (n * (n + 1) / 2) * hd * 2 * 2
    return cfg.num_hidden_layers * (gemm + attention) + 2 * batch * cfg.vocab_size * d


def decode_layer_bytes(cfg, context: int) -> int:
    """Algorithmic bytes of the layers of one batch-1 fp32 decode step: every weight the step reads (norms, sinks,
    QKV, out-projection, router, the k routed experts' mlp1/mlp2 rows with biases), the K/V cache rows, the new
    K/V rows written, the embedding row and the final-norm row."""
    d, hd, H, KV, E, k, I = (cfg.hidden_size, cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads,
                             cfg.num_experts, cfg.experts_per_token, cfg.intermediate_size)
    qkv = (H + 2 * KV) * hd
    static = d + H + qkv * d + qkv + d * H * hd + d + d + E * d + E
    experts = k * (2 * I * d + 2 * I + d * I + d)
    cache = 2 * context * KV * hd + 2 * KV * hd
    return 4 * (cfg.num_hidden_layers * (static + experts + cache) + 3 * d)


def decode_flops_per_token(cfg, ctx: int) -> float:  # type: ignore[no-untyped-def]
    """Algorithmic FLOPs of one cached decode token (projections, router, top-k experts, attention over ctx, vocab)."""
    d, H, KV, hd, E, k, I = (cfg.hidden_size, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim,
                             cfg.num_experts, cfg.experts_per_token, cfg.intermediate_size)
    per_layer = 2 * ((H + 2 * KV) * hd * d + d * H * hd + E * d + k * (2 * I * d + d * I)) + 4 * H * ctx * hd
    return cfg.num_hidden_layers * per_layer + 2 * cfg.vocab_size * d


def bench_c4(args: argparse.Namespace, rng: np.random.Generator, max_over_ranks, barrier, rank: int = 0,
             world: int = 1) -> dict:  # type: ignore[no-untyped-def]
    """GPT-OSS-20B-shaped prefill of 2048-token sequences (config C4): bf16 weights N(0, 0.02) generated in device
    memory, the batched prefill program through BatchDecoder (tokens in from the host, greedy ids out).

    With several ranks (torchrun) the 32 experts are split over the GPUs (expert parallel, csrc/ep.cuh): each rank
    holds E / world experts plus the replicated attention, router and embeddings and exchanges routed rows with the
    other ranks every layer over NVLink peer memory. Two measurements: ``weak`` (4 x 2048 tokens per GPU) and, where
    4 sequences split evenly, ``strong`` (BASELINE's 4 x 2048 tokens in total, 4 / world sequences per GPU)."""
    import torch

    import chroma_b200
    from chroma_b200 import models
    from chroma_b200._src.compiler import synthetic_gptoss
    from chroma_b200._src.native import Native

    cfg = models.gpt_oss_20b
    if args.c4_layers:
        cfg = dataclasses.replace(cfg, num_hidden_layers=args.c4_layers)
    batch, n = 4, 2048
    plan_p, regions = synthetic_gptoss(cfg, steps=n, context=n, ep_world=world)
    plan_d, _ = synthetic_gptoss(cfg, steps=1, context=n, ep_world=world)
    wbuf = torch.empty(plan_p["desc"]["weight_bytes"], dtype=torch.uint8, device="cuda")
    _fill_synthetic(regions, wbuf, 20, 1000 + rank)  # replicated weights identical on every rank; own experts
    torch.cuda.synchronize()
    group = None
    if world > 1:
        group = chroma_b200.ExpertGroup(rank, world, max_pairs=batch * n * cfg.experts_per_token,
                                        hidden=cfg.hidden_size, experts=cfg.num_experts)
    pre = chroma_b200.Program.from_native(Native(plan_p, device_weights=wbuf.data_ptr(), ep=group))
    dec = chroma_b200.Program.from_native(Native(plan_d, device_weights=wbuf.data_ptr(), ep=group))
    peak = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops_sustained"] if (ROOT / "MEASURED_PEAKS.json").exists() else 1400.0

    def timed(seqs: int) -> tuple[float, int, np.ndarray]:
        bd = chroma_b200.BatchDecoder(pre, dec, seqs)
        tokens = rng.integers(0, cfg.vocab_size, (seqs, n))
        reps = max(2, min(5, args.steps // 40))
        for _ in range(max(1, min(3, args.warmup))):
            bd.reset()
            barrier()
            bd.append(tokens, argmax=True)
        times = []
        for _ in range(reps):
            bd.reset()
            barrier()
            t0 = time.perf_counter()
            ids = bd.append(tokens, argmax=True)
            times.append(time.perf_counter() - t0)
        bd.close()
        return max_over_ranks(statistics.median(times)), reps, ids

    t, reps, ids = timed(batch)
    flops = prefill_flops(cfg, batch, n) * world
    strong = None
    if world > 1 and batch % world == 0:
        ts, _, _ = timed(batch // world)
        sflops = prefill_flops(cfg, batch // world, n) * world
        strong = {"tokens_per_s": batch * n / ts, "ms": ts * 1e3, "sequences_per_gpu": batch // world,
                  "frac_of_bf16_sustained": sflops / ts / 1e12 / (peak * world)}
    barrier()
    del pre, dec
    if group is not None:
        group.close()
    del wbuf
    torch.cuda.empty_cache()
    return {
        "workload": f"C4: GPT-OSS-20B-shaped prefill ({cfg.num_hidden_layers} layers, d=2880, 64/8 heads, 32 experts "
                    f"top-4, bf16 N(0,0.02)), 4 x 2048 tokens per GPU, {world} GPU(s), "
                    + ("all experts local" if world == 1 else f"expert parallel ({cfg.num_experts // world} experts "
                                                               "per GPU, NVLink peer-memory dispatch/return)"),
        "tokens_per_s": world * batch * n / t, "ms": t * 1e3, "reps": reps, "n_gpus": world,
        "scaling": "weak",
        "strong": strong,
        "e2e": {"api": "BatchDecoder.append(tokens[4, 2048], argmax=True) on every rank",
                "h2d_bytes": batch * n * 8 + batch * 16, "d2h_bytes": batch * 8 + 4},
        "algorithmic_tflop": flops / 1e12, "achieved_tflops": flops / t / 1e12,
        "frac_of_bf16_sustained": flops / t / 1e12 / (peak * world),
        "peak_source": "MEASURED_PEAKS.json bf16_tflops_sustained (x GPUs)",
        "argmax_head": [int(v) for v in ids[:2]],
        "cpu_baseline": {"value": batch * n / (prefill_flops(cfg, batch, n) / 1e9 / REF_CPU_GFLOPS), "unit": "tokens/s",
                         "cores": 1, "kind": "reference (extrapolated)",
                         "sample": "reference compiled CPU program for one C4-width layer, 16 tokens (10.59 s in the "
                                   "build container, 2.12 GFLOP/s), extrapolated by FLOPs to this prefill"},
    }


def _fill_synthetic(regions, wbuf, shared_seed: int, expert_seed: int | None = None) -> None:  # type: ignore[no-untyped-def]
    """bf16 N(0, 0.02) weights (norm scales 1) written in device memory; the expert tensors from their own generator
    when ``expert_seed`` is given."""
    import torch

    shared_gen = torch.Generator(device="cuda").manual_seed(shared_seed)
    expert_gen = None if expert_seed is None else torch.Generator(device="cuda").manual_seed(expert_seed)
    for name, off, numel, is_norm in regions:
        if is_norm:
            wbuf[off : off + numel * 4].view(torch.float32).fill_(1.0)
        else:
            gen = expert_gen if (expert_gen is not None and ".mlp.mlp" in name) else shared_gen
            wbuf[off : off + numel * 2].view(torch.bfloat16).normal_(0.0, 0.02, generator=gen)


def _rank_slice(full_regions, rank_regions, full, out, rank: int, world: int, hidden: int,  # type: ignore[no-untyped-def]
                vocab: range | None) -> None:
    """Copy the all-local weights ``full`` into this rank's expert-parallel layout ``out``: replicated tensors whole,
    the expert tensors' rows of this rank's experts, and (vocab shard) this rank's unembedding rows."""
    src = {name: (off, numel) for name, off, numel, _ in full_regions}
    for name, off, numel, is_norm in rank_regions:
        soff, snumel = src[name]
        es = 4 if is_norm else 2
        start = 0
        if ".mlp.mlp" in name:
            start = rank * (snumel // world) * es
        elif name == "unembedding.weight" and vocab is not None:
            start = vocab.start * hidden * es
        out[off : off + numel * es].copy_(full[soff + start : soff + start + numel * es])


def ep_parity(rank: int, world: int, barrier) -> dict:  # type: ignore[no-untyped-def]
    """Bit-identity of the expert-parallel programs with the all-local program on the same tokens, on every rank,
    before any timing (the reference has no multi-GPU path, so the all-local program is the bar).

    * ``c4``: a 2-layer model at GPT-OSS-20B widths (32 experts, top-4), a 64-token forward per rank, experts split
      over the ranks: logits, routes and greedy ids bit for bit.
    * ``c5``: a 2-layer model at GPT-OSS-120B widths (128 experts) with the vocab projection column-sharded as well,
      16 sequences per rank through the batched decoder (16-token prefill, 3 greedy steps): greedy ids identical;
      prefill logits within the bf16 rounding of the last bit (the vocab GEMM over a shard tiles the sums
      differently from the whole-vocabulary GEMM).
    * ``artifacts``: a 2-layer model at reduced widths compiled per rank to its own artefact directory
      (``compile_model(..., experts=group)``: the rank's expert shard, the manifest recording rank and world): its
      32-token forward bit for bit against the all-local program.
    Semantics: chroma/models/gpt_oss.py:243-265 (MLPBlock.forward) on every rank's tokens."""
    import torch

    import chroma_b200
    from chroma_b200 import models
    from chroma_b200._src.compiler import synthetic_gptoss
    from chroma_b200._src.experts import vocab_shard
    from chroma_b200._src.native import Native

    out: dict = {"ranks": world}
    exchange = None if world > 1 else (lambda h: [h])
    # ---- C4 widths, forward
    cfg = dataclasses.replace(models.gpt_oss_20b, num_hidden_layers=2)
    n = 64
    fplan, fregions = synthetic_gptoss(cfg, steps=n)
    eplan, eregions = synthetic_gptoss(cfg, steps=n, ep_world=world)
    full = torch.empty(fplan["desc"]["weight_bytes"], dtype=torch.uint8, device="cuda")
    _fill_synthetic(fregions, full, 31)
    part = torch.empty(eplan["desc"]["weight_bytes"], dtype=torch.uint8, device="cuda")
    _rank_slice(fregions, eregions, full, part, rank, world, cfg.hidden_size, None)
    group = chroma_b200.ExpertGroup(rank, world, max_pairs=n * cfg.experts_per_token, hidden=cfg.hidden_size,
                                    experts=cfg.num_experts, exchange=exchange)
    tokens = np.random.default_rng(300 + rank).integers(0, cfg.vocab_size, n)
    local = chroma_b200.Program.from_native(Native(fplan, device_weights=full.data_ptr()))
    shared = chroma_b200.Program.from_native(Native(eplan, device_weights=part.data_ptr(), ep=group))
    want, want_routes = np.asarray(local(tokens)), local.native.routes()
    barrier()
    got = [np.asarray(shared(tokens)) for _ in range(2)]
    got_routes = shared.native.routes()
    out["c4"] = bool(all(np.array_equal(g.view(np.uint16), want.view(np.uint16)) for g in got)
                     and np.array_equal(got_routes, want_routes))
    barrier()
    local.close()
    shared.close()
    group.close()
    del full, part
    torch.cuda.empty_cache()
    # ---- per-rank artefacts: compile_model(..., experts=group) writes this rank's expert shard to its own
    # artefact directory (manifest records rank and world); its forward must equal the all-local program's bits.
    import tempfile as _tempfile

    small = dataclasses.replace(models.gpt_oss_20b, num_hidden_layers=2, hidden_size=1024, intermediate_size=1024,
                                num_attention_heads=16, num_key_value_heads=2, num_experts=8, experts_per_token=2,
                                vocab_size=8192)
    model = models.random_transformer(small, seed=61, std=0.02, dtype=torch.bfloat16)
    toks = np.random.default_rng(600 + rank).integers(0, small.vocab_size, 32)
    with _tempfile.TemporaryDirectory() as tmp:
        sgroup = chroma_b200.ExpertGroup(rank, world, max_pairs=32 * small.experts_per_token, hidden=1024, experts=8,
                                         exchange=exchange)
        local = chroma_b200.compile_model(model, Path(tmp) / "all", steps=32)
        shard = chroma_b200.compile_model(model, Path(tmp) / f"rank{rank}", steps=32, experts=sgroup)
        manifest = json.loads((Path(tmp) / f"rank{rank}" / "model.json").read_text())
        want = np.asarray(local(toks))
        barrier()
        got = np.asarray(shard(toks))
        out["artifacts"] = bool(manifest["b200"].get("expert_parallel") == {"rank": rank, "world": world}
                                and np.array_equal(got.view(np.uint16), want.view(np.uint16)))
        barrier()
        local.close()
        shard.close()
        sgroup.close()
    # ---- C5 widths, vocab shard, batched decode
    cfg = dataclasses.replace(models.gpt_oss_120b, num_hidden_layers=2)
    B, pre_n, ctx = 16, 16, 64
    vocab = vocab_shard(rank, world, cfg.vocab_size)
    plans = [synthetic_gptoss(cfg, steps=s, context=ctx) for s in (pre_n, 1)]
    eplans = [synthetic_gptoss(cfg, steps=s, context=ctx, ep_world=world, vocab_rows=len(vocab)) for s in (pre_n, 1)]
    full = torch.empty(plans[0][0]["desc"]["weight_bytes"], dtype=torch.uint8, device="cuda")
    _fill_synthetic(plans[0][1], full, 51)
    part = torch.empty(eplans[0][0]["desc"]["weight_bytes"], dtype=torch.uint8, device="cuda")
    _rank_slice(plans[0][1], eplans[0][1], full, part, rank, world, cfg.hidden_size, vocab)
    group = chroma_b200.ExpertGroup(rank, world, max_pairs=B * pre_n * cfg.experts_per_token, hidden=cfg.hidden_size,
                                    experts=cfg.num_experts, vocab_rows=B, vocab=cfg.vocab_size, exchange=exchange)
    rng = np.random.default_rng(500 + rank)
    prompts = rng.integers(0, cfg.vocab_size, (B, pre_n))
    results = []
    for weights, pl, grp in ((full, plans, None), (part, eplans, group)):
        pre = chroma_b200.Program.from_native(Native(pl[0][0], device_weights=weights.data_ptr(), ep=grp))
        dec = chroma_b200.Program.from_native(Native(pl[1][0], device_weights=weights.data_ptr(), ep=grp))
        with chroma_b200.BatchDecoder(pre, dec, B) as bd:
            if grp is not None:
                barrier()
            logits = np.asarray(bd.append(prompts)).astype(np.float32)
            ids = bd.append(prompts[:, -1:], argmax=True)
            results.append((logits, ids, bd.generate(ids, 3)))
    (la, ia, ga), (lb, ib, gb) = results
    scale = np.max(np.abs(la), axis=-1, keepdims=True)
    out["c5"] = bool(np.array_equal(ia, ib) and np.array_equal(ga, gb)
                     and float(np.max(np.abs(la - lb) / scale)) <= 1e-2)
    barrier()
    group.close()
    del full, part
    torch.cuda.empty_cache()
    return out


def bench_c5(args: argparse.Namespace, max_over_ranks, barrier, rank: int, world: int) -> dict:  # type: ignore[no-untyped-def]
    """GPT-OSS-120B-shaped greedy decode (config C5): 256 sequences over all ranks (256 / world each, data parallel
    attention), a 4,096-token bf16 cache per sequence filled with N(0, 1) values, current tokens at position 4,096;
    the 128 experts split over the ranks (expert parallel over NVLink peer memory). One step = one token for every
    sequence: 36 layers, vocab projection, argmax fed back, all on the device (``BatchDecoder.advance_device``)."""
    import torch

    import chroma_b200
    from chroma_b200 import models
    from chroma_b200._src.compiler import synthetic_gptoss
    from chroma_b200._src.native import Native

    cfg = models.gpt_oss_120b
    if args.c5_layers:
        cfg = dataclasses.replace(cfg, num_hidden_layers=args.c5_layers)
    total, ctx = args.c5_sequences, 4096
    if total % world or (world < 2 and not args.c5_layers):
        return {"unavailable": "C5 needs 2 or more GPUs dividing 256 sequences (233 GB of expert weights); "
                               "one GPU runs it only with fewer layers (--c5-layers)"}
    B, L, KV, hd = total // world, cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim
    from chroma_b200._src.experts import vocab_shard

    shard = vocab_shard(rank, world, cfg.vocab_size)  # vocab column shard: this rank's unembedding rows
    plan, regions = synthetic_gptoss(cfg, steps=1, context=ctx, ep_world=world, vocab_rows=len(shard))
    wbuf = torch.empty(plan["desc"]["weight_bytes"], dtype=torch.uint8, device="cuda")
    shared_gen = torch.Generator(device="cuda").manual_seed(50)
    expert_gen = torch.Generator(device="cuda").manual_seed(5000 + rank)
    for name, off, numel, is_norm in regions:
        if is_norm:
            wbuf[off : off + numel * 4].view(torch.float32).fill_(1.0)
        else:
            gen = expert_gen if (".mlp.mlp" in name or name == "unembedding.weight") else shared_gen
            wbuf[off : off + numel * 2].view(torch.bfloat16).normal_(0.0, 0.02, generator=gen)
    group = chroma_b200.ExpertGroup(rank, world, max_pairs=B * cfg.experts_per_token, hidden=cfg.hidden_size,
                                    experts=cfg.num_experts, vocab_rows=B, vocab=cfg.vocab_size,
                                    exchange=None if world > 1 else (lambda h: [h]))
    pre = chroma_b200.Program.from_native(Native(plan, device_weights=wbuf.data_ptr(), ep=group))
    dec = chroma_b200.Program.from_native(Native(plan, device_weights=wbuf.data_ptr(), ep=group))
    bd = chroma_b200.BatchDecoder(pre, dec, B)
    cache_gen = torch.Generator(device="cuda").manual_seed(700 + rank)
    for b in range(B):  # one sequence at a time keeps the staging small
        k = torch.randn((1, L, ctx, KV, hd), generator=cache_gen, device="cuda").to(torch.bfloat16)
        v = torch.randn((1, L, ctx, KV, hd), generator=cache_gen, device="cuda").to(torch.bfloat16)
        bd.load_cache(b, k, v, np.array([ctx]))
    del k, v
    torch.cuda.synchronize()
    tokens = np.random.default_rng(900 + rank).integers(0, cfg.vocab_size, B)
    barrier()
    bd.generate(tokens, 1)  # consumes the current tokens (position 4096) and leaves the argmax on the device
    stream = torch.cuda.current_stream()
    warm = max(3, args.warmup)
    barrier()
    bd.advance_device(warm, stream.cuda_stream)
    steps = max(10, min(50, args.steps))
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    bd.advance_device(steps, stream.cuda_stream)
    e1.record(stream)
    torch.cuda.synchronize()
    t = max_over_ranks(e0.elapsed_time(e1) / 1e3)
    ids = bd.generate(np.asarray(tokens), 1)[:, 0]
    # e2e: greedy steps through the public API, host token ids in and host greedy ids out every step.
    e2e_steps = max(5, min(20, args.steps))
    cur = np.asarray(bd.append(ids[:, None], argmax=True))  # warm-up
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        cur = np.asarray(bd.append(cur[:, None], argmax=True))
    e2e_t = max_over_ranks((time.perf_counter() - t0) / e2e_steps)
    barrier()
    d, I, E, k_ = cfg.hidden_size, cfg.intermediate_size, cfg.num_experts, cfg.experts_per_token
    expert_bytes = (2 * I * d + d * I + 2 * I + d) * 2
    attn_bytes = ((cfg.num_attention_heads + 2 * KV) * hd * d + d * cfg.num_attention_heads * hd) * 2
    per_rank = L * ((E // world) * expert_bytes + attn_bytes + E * d * 2 + B * ctx * KV * hd * 2 * 2)
    per_rank += len(shard) * d * 2
    bd.close()
    del pre, dec
    group.close()
    del wbuf
    torch.cuda.empty_cache()
    pk = peaks()["hbm_gbs"]
    return {
        "workload": f"C5: GPT-OSS-120B-shaped greedy decode ({L} layers, d=2880, 64/8 heads, 128 experts top-4, bf16 "
                    f"N(0,0.02)), {total} sequences ({B} per GPU) with a 4,096-token bf16 cache, {world} GPUs, "
                    f"{E // world} experts per GPU (NVLink peer-memory dispatch/return), vocab column shard of "
                    f"{len(shard)} rows per GPU",
        "tokens_per_s": total * steps / t, "ms_per_step": t * 1e3 / steps, "steps": steps, "n_gpus": world,
        "scaling": "strong (256 sequences in total)",
        "hbm_bytes_per_step_per_gpu": per_rank,
        "roofline_frac": per_rank / (t / steps) / 1e9 / pk,
        "roofline_note": "all experts of the rank assumed touched (B x top-4 routes over E / world experts); "
                         "measured copy peak of one GPU",
        "e2e": {"value": total / e2e_t, "unit": "tokens/s", "ms_per_step": e2e_t * 1e3,
                "h2d_bytes_per_step": B * 8, "d2h_bytes_per_step": B * 8,
                "api": f"BatchDecoder.append(ids[{B}, 1], argmax=True) on every rank, host ids fed back"},
        "argmax_head": [int(v) for v in ids[:2]],
        "cpu_baseline": {"value": 1.0 / (decode_flops_per_token(cfg, ctx) / 1e9 / REF_CPU_GFLOPS), "unit": "tokens/s",
                         "cores": 1, "kind": "reference (extrapolated)",
                         "sample": "the C4-layer CPU rate (2.12 GFLOP/s, reference compiled program, 1 thread) "
                                   "applied to one C5 decode token's FLOPs"},
    }


def measure_fwd8(fwd8, rng, V, args, flush, stream, reps, max_over_ranks):  # type: ignore[no-untyped-def]
    """C1: the 8-token forward `Program(tokens[8])`, device time of one run (CUDA events around the program's
    launch on `stream`, L2 flushed before each) and end to end through the public call; medians, ms."""
    import torch

    native = fwd8.native
    tokens8 = rng.integers(0, V, 8).astype(np.int64)
    torch.cuda.synchronize()
    fwd8(tokens8)
    f_ms = []
    for i in range(args.warmup + reps):
        flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        native.run_device(stream.cuda_stream)
        e1.record(stream)
        if i >= args.warmup:
            f_ms.append((e0, e1))
    native.check(stream.cuda_stream)
    f_ms = [a.elapsed_time(b) for a, b in f_ms]
    fe2e = []
    for i in range(args.warmup + reps):
        flush()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        fwd8(tokens8)  # the default call: the result array is the runtime's (page-locked) allocation
        if i >= args.warmup:
            fe2e.append(time.perf_counter() - t0)
    fwd_dev_ms = max_over_ranks(statistics.median(f_ms))
    fwd_e2e_ms = max_over_ranks(1e3 * statistics.median(fe2e))

    return fwd_dev_ms, fwd_e2e_ms


def main() -> None:
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    import torch

    import chroma_b200
    from chroma_b200 import models
    from chroma_b200._src.decoder import Decoder

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def barrier() -> None:
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # A dedicated stream: its handle is non-zero, so the native calls queue on it (0 would select the objects' own
    # streams) and the CUDA events below bracket exactly the queued work.
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    if args.gemm is not None:
        for name in args.gemm or sorted(GEMM_SHAPES):
            res = bench_gemm(name, max(1, args.steps), max(1, args.warmup))
            if rank == 0:
                print(json.dumps(res), flush=True)
        if dist is not None:
            dist.destroy_process_group()
        return
    if args.c5_only:
        c5 = bench_c5(args, max_over_ranks, barrier, rank, world)
        if rank == 0:
            print(json.dumps({"c5_decode": c5}), flush=True)
        if dist is not None:
            dist.destroy_process_group()
        return
    if args.c4_only:
        c4 = bench_c4(args, np.random.default_rng(rank), max_over_ranks, barrier, rank, world)
        if rank == 0:
            print(json.dumps({"c4_prefill": c4}), flush=True)
        if dist is not None:
            dist.destroy_process_group()
        return
    parity = None
    if not args.skip_parity:
        parity = ep_parity(rank, world, barrier)
        flags = torch.tensor([int(parity["c4"]), int(parity["c5"]), int(parity["artifacts"])], device="cuda",
                             dtype=torch.int32)
        if dist is not None:
            dist.all_reduce(flags, op=dist.ReduceOp.MIN)  # true only when every rank matched
        parity.update(c4=bool(flags[0].item()), c5=bool(flags[1].item()), artifacts=bool(flags[2].item()))
    flush_buf = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    flush_read = torch.ones(64 << 20, dtype=torch.float32, device="cuda")

    def flush() -> None:
        # Write 256 MiB (evicts everything), then read 256 MiB so the lines left in L2 are clean: the timed work
        # then pays neither hits from its previous run nor write-backs of the flush's dirty lines.
        flush_buf.fill_(1)
        flush_read.sum()

    model = models.make_dev_model(0)
    V = models.dev.vocab_size
    tmp = Path(tempfile.mkdtemp(prefix=f"chroma-b200-bench-{rank}-"))
    prefill = chroma_b200.compile_model(model, tmp / "prefill", steps=PREFILL, context=CONTEXT)
    decode = chroma_b200.compile_model(model, tmp / "decode", steps=1, context=CONTEXT)
    fwd8 = chroma_b200.compile_model(model, tmp / "fwd8", steps=8)
    rng = np.random.default_rng(1234 + rank)
    prompt = rng.integers(0, V, PREFILL)
    if args.fwd8_only:
        dev_ms, e2e_ms = measure_fwd8(fwd8, rng, V, args, flush, stream, max(3, min(50, args.steps)), max_over_ranks)
        if rank == 0:
            print(json.dumps({"fwd8_only": {"device_ms": dev_ms, "e2e_ms": e2e_ms}}), flush=True)
        if dist is not None:
            dist.destroy_process_group()
        return

    def timed_device(bd: "chroma_b200.BatchDecoder", steps: int) -> list[float]:
        times = []
        for _ in range(steps):
            flush()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            bd.advance_device(1, stream.cuda_stream)
            e1.record(stream)
            times.append((e0, e1))
        torch.cuda.synchronize()
        return [a.elapsed_time(b) for a, b in times]

    # ---- headline: batch-1 device-resident greedy decode
    nb = args.decode_batch if args.decode_only else 1
    bd1 = chroma_b200.BatchDecoder(prefill, decode, nb)
    first = bd1.append(prompt[None, :] if nb == 1 else rng.integers(0, V, (nb, PREFILL)), argmax=True)
    bd1.generate(first, 1)
    timed_device(bd1, args.warmup)
    barrier()
    with Clocks(local) as clocks:
        step_ms = timed_device(bd1, args.steps)
        barrier()
    launches_per_step = bd1._native.step_launches
    t_rank = sum(step_ms) / 1e3
    t_max = max_over_ranks(t_rank)
    value = world * args.steps / t_max
    if args.decode_only:
        if rank == 0:
            print(json.dumps({"decode_only": {"batch": nb, "value": value * nb, "ms_per_step": 1e3 * t_max / args.steps}}),
                  flush=True)
        bd1.close()
        if dist is not None:
            dist.destroy_process_group()
        return

    # ---- roofline: vocab kernel alone (L2 flushed before each launch)
    vocab_ms = []
    reps = max(3, min(50, args.steps))
    for i in range(args.warmup + reps):
        flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        bd1._native.launch_vocab(stream.cuda_stream)
        e1.record(stream)
        if i >= args.warmup:
            vocab_ms.append((e0, e1))
    torch.cuda.synchronize()
    vocab_ms = [a.elapsed_time(b) for a, b in vocab_ms]
    d = models.dev.hidden_size
    vocab_bytes = V * d * 4 + V * 4 + d * 4  # weights + one logits row + the normed row
    vocab_t = statistics.mean(vocab_ms) / 1e3
    pk = peaks()
    achieved = vocab_bytes / vocab_t / 1e9

    # ---- roofline of the dominant kernel: the layers (one cluster launch for batch-1 fp32), L2 flushed first
    layer_ms = []
    for i in range(args.warmup + reps):
        flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        bd1._native.launch_layers(stream.cuda_stream)
        e1.record(stream)
        if i >= args.warmup:
            layer_ms.append((e0, e1))
    torch.cuda.synchronize()
    layer_t = statistics.mean(a.elapsed_time(b) for a, b in layer_ms) / 1e3
    layer_bytes = decode_layer_bytes(models.dev, CONTEXT)
    layer_gbs = layer_bytes / layer_t / 1e9
    bd1.close()

    # ---- e2e batch 1 through the public Decoder API
    dec = Decoder(prefill, decode)
    forced = rng.integers(0, V, args.warmup + args.steps)
    dec.append(prompt)
    for t in forced[: args.warmup]:
        dec.append([int(t)])
    barrier()
    e2e_times = []
    for t in forced[args.warmup :]:
        flush()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        logits = dec.append([int(t)])
        e2e_times.append(time.perf_counter() - t0)
    e2e_max = max_over_ranks(sum(e2e_times))
    e2e_value = world * args.steps / e2e_max
    d2h = logits.nbytes + 4
    dec._native.close()
    dec._native = None

    # ---- batch 64: device value and e2e through BatchDecoder.append(argmax=True)
    B = 64
    bsteps = max(1, args.steps // 4)
    bd64 = chroma_b200.BatchDecoder(prefill, decode, B)
    bprompt = rng.integers(0, V, (B, PREFILL))
    firsts = bd64.append(bprompt, argmax=True)
    bd64.generate(firsts, 1)
    timed_device(bd64, args.warmup)
    b_ms = timed_device(bd64, bsteps)
    b_value = world * B * bsteps / max_over_ranks(sum(b_ms) / 1e3)
    bd64.reset()
    bforced = rng.integers(0, V, (B, args.warmup + bsteps))
    bd64.append(bprompt, argmax=True)
    for i in range(args.warmup):
        bd64.append(bforced[:, i : i + 1], argmax=True)
    be2e = []
    for i in range(args.warmup, args.warmup + bsteps):
        flush()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        bd64.append(bforced[:, i : i + 1], argmax=True)
        be2e.append(time.perf_counter() - t0)
    b_e2e = world * B * bsteps / max_over_ranks(sum(be2e))
    bd64.close()

    fwd_dev_ms, fwd_e2e_ms = measure_fwd8(fwd8, rng, V, args, flush, stream, reps, max_over_ranks)

    # ---- C3: the fused norm/SiLU micrograph, bf16 [16384, 4096] (HBM bound), device-resident inputs
    from chroma_b200._src.compiler import lower_micro, write_artifact

    mrows, mcols = 16384, 4096
    micro = chroma_b200.Program(write_artifact(lower_micro(np.ones(mcols, np.float32), mrows, mcols), tmp / "micro"))
    gen = np.random.default_rng(5)
    host = [gen.standard_normal((mrows, mcols), dtype=np.float32) for _ in range(3)]
    from ml_dtypes import bfloat16 as _bf16

    mout = micro(*[h.astype(_bf16) for h in host])  # uploads the inputs into the program's device buffers
    del host
    m_ms = []
    for i in range(args.warmup + reps):
        flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        micro.native.run_device(stream.cuda_stream)
        e1.record(stream)
        if i >= args.warmup:
            m_ms.append((e0, e1))
    micro.native.check(stream.cuda_stream)
    m_ms = [a.elapsed_time(b) for a, b in m_ms]
    micro_bytes = 4 * mrows * mcols * 2 + mcols * 4
    micro_t = statistics.mean(m_ms) / 1e3
    micro.close()
    del mout

    c4 = bench_c4(args, rng, max_over_ranks, barrier, rank, world) if not args.skip_c4 else None
    # C5 needs the experts of the 120B-shaped model spread over 2 or more GPUs.
    c5 = bench_c5(args, max_over_ranks, barrier, rank, world) if world > 1 and not args.skip_c5 else None

    cpu = None
    if rank == 0 and world == 1:
        cpu = cpu_reference_decode(args.cpu_seconds)
    barrier()
    if dist is not None:
        dist.destroy_process_group()
    if rank != 0:
        return
    ms_per_step = 1e3 * t_max / args.steps
    line = {
        "metric": "dev decode tokens/s (KV cache 256, batch 1)",
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": value / world / (1e3 / A100_DECODE_STEP_MS),
        "dtype": "f32",
        "data": DATA,
        "config": c2_config(world),
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": 16, "d2h_bytes_per_step": d2h,
                "api": "chroma_b200.Decoder.append([token]) -> logits [1, 201088] on the host"},
        "gpu_launches": launches_per_step * args.steps,
        "roofline": {
            "kernel": "k_decode_cluster (every layer of one decode step in a 16-CTA cluster; 60 dependent phases)",
            "bound": "hbm", "achieved": layer_gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": layer_gbs / pk["hbm_gbs"], "traffic": CLUSTER_NCU_TRAFFIC,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one k_decode_cluster launch of this "
                              "workload, caches flushed",
            "algorithmic_bytes": layer_bytes, "launch_us": layer_t * 1e6,
            "peak_source": f"{pk['source']} (MEASURED_PEAKS.json hbm_gbs, burst copy)",
            "timing": f"launched alone after an L2 flush, CUDA events, mean of {reps}",
            "note": "latency-bound: the weights touched per step are 12 MB; the kernel's time is its chain of "
                    "dependent phases, not bytes",
        },
        "roofline_step": {
            "what": "the whole decode step (layers + vocab GEMV): the per-step bytes of the workload table",
            "bound": "hbm", "algorithmic_bytes": layer_bytes + vocab_bytes,
            "achieved": (layer_bytes + vocab_bytes) / (ms_per_step / 1e3) / 1e9, "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": (layer_bytes + vocab_bytes) / (ms_per_step / 1e3) / 1e9 / pk["hbm_gbs"],
        },
        "roofline_vocab": {
            "kernel": "k_vocab_row (unembedding GEMV, 201088 x 128 fp32, 1 row)", "bound": "hbm", "achieved": achieved,
            "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"], "traffic": VOCAB_NCU_TRAFFIC,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one k_vocab<float, 1> launch of "
                              "this workload",
            "algorithmic_bytes": vocab_bytes, "launch_us": vocab_t * 1e6,
            "peak_source": f"{pk['source']} (MEASURED_PEAKS.json hbm_gbs, burst copy)",
            "timing": f"launched alone after an L2 flush, CUDA events, mean of {reps} (inside a step the vocab "
                      "matrix is prefetched into L2 beside the layers and this kernel reads it from L2)",
        },
        "cpu_baseline": None if cpu is None else {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "clocks": clocks.summary(),
        "batch64": {"value": b_value, "unit": "tokens/s", "ms_per_step": statistics.mean(b_ms),
                    "e2e": {"value": b_e2e, "unit": "tokens/s", "h2d_bytes_per_step": B * 16,
                            "d2h_bytes_per_step": B * 8 + 4, "api": "BatchDecoder.append(tokens[64,1], argmax=True)"}},
        "micro": {"workload": "C3 fused RMSNorm*w -> z=y*g -> z*sigmoid(z)*u + x, bf16 [16384, 4096]",
                  "device_us": micro_t * 1e6, "algorithmic_bytes": micro_bytes,
                  "achieved_gbs": micro_bytes / micro_t / 1e9, "frac": micro_bytes / micro_t / 1e9 / pk["hbm_gbs"]},
        "c4_prefill": c4,
        "c5_decode": c5,
        "fwd8": {"device_ms": fwd_dev_ms, "e2e_ms": fwd_e2e_ms, "vs_a100_e2e": A100_FWD8_MS / fwd_e2e_ms,
                 "h2d_bytes": 64, "d2h_bytes": 8 * V * 4, "api": "Program(tokens[8]) -> logits [8, 201088]"},
    }
    # Last and compact, so a reader that keeps only the end of the line still sees the multi-GPU results.
    line["multi_gpu"] = {
        "n": world,
        "ep_parity": parity,
        "c4_weak": None if not c4 else {"tok_s": round(c4["tokens_per_s"]), "ms": round(c4["ms"], 2),
                                        "frac_bf16": round(c4["frac_of_bf16_sustained"], 3)},
        "c4_strong": None if not c4 or not c4.get("strong") else {
            "tok_s": round(c4["strong"]["tokens_per_s"]), "ms": round(c4["strong"]["ms"], 2),
            "frac_bf16": round(c4["strong"]["frac_of_bf16_sustained"], 3)},
        "c5": None if not c5 or "unavailable" in c5 else {
            "tok_s": round(c5["tokens_per_s"]), "ms_step": round(c5["ms_per_step"], 3),
            "frac_hbm": round(c5["roofline_frac"], 3), "e2e_tok_s": round(c5["e2e"]["value"])},
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
