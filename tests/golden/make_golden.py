"""Generate the golden fixtures in this directory from the reference's own compiled CPU programs.

Run in the development container (where the reference sources exist): ``python -m tests.golden.make_golden``.
It builds (if needed) the reference CPU programs with ``oracle/build_ref.py`` and runs them through the reference's
own ``chroma.Program`` / ``chroma.Decoder`` on seeded inputs. Weights come from the reference's seeded constructors
(scripts/export.py:16-29 and the test helpers), which ``chroma_b200.models`` reproduces bit for bit (the digests
stored here are checked by ``tests/test_models.py``).

Fixtures are small: token ids, argmax ids, routing indices, top-16 (index, value) pairs, a fixed sample of 4096
logit columns, and per-row float64 sums; full outputs only where they are small.
"""

from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

V = 201088
SAMPLE = np.sort(np.random.default_rng(123).choice(V, 4096, replace=False)).astype(np.int64)


def digest(model) -> str:  # type: ignore[no-untyped-def]
    import torch

    h = hashlib.sha256()
    for k, v in model.state_dict().items():
        h.update(k.encode())
        t = v.detach().contiguous()
        h.update(t.view(torch.uint16).numpy().tobytes() if t.dtype == torch.bfloat16 else t.numpy().tobytes())
    return h.hexdigest()


def summary(logits: np.ndarray) -> dict[str, np.ndarray]:
    logits = np.asarray(logits, dtype=np.float32).reshape(-1, logits.shape[-1])
    top = np.argsort(-logits, axis=-1, kind="stable")[:, :16]
    return {
        "argmax": np.argmax(logits, axis=-1).astype(np.int64),
        "top_idx": top.astype(np.int64),
        "top_val": np.take_along_axis(logits, top, axis=-1),
        "sample": logits[:, SAMPLE] if logits.shape[-1] == V else logits,
        "rowsum": logits.astype(np.float64).sum(-1),
    }


def stack(items: list[dict[str, np.ndarray]], prefix: str) -> dict[str, np.ndarray]:
    return {f"{prefix}{k}": np.stack([it[k] for it in items]) for k in items[0]}


def c1_token_sets() -> np.ndarray:
    t = np.arange(8, dtype=np.int64)
    return np.stack([t, (t * 7919 + 17) % V, np.zeros(8, np.int64), t[::-1].copy(),
                     np.random.default_rng(0).integers(0, V, 8)])


def c4_slice() -> None:
    """One layer of the 20B-shaped model at full widths (d=2880, 64/8 heads, 32 experts, 201,088 vocab), bf16."""
    from oracle import build_ref, refimport

    refimport.install()

    build_ref.build("c4_slice_fwd16")
    model = build_ref.random_transformer(build_ref.small_config("c4_slice"), seed=11, std=0.02,
                                         dtype=__import__("torch").bfloat16)
    tokens = build_ref.c4_tokens().numpy()
    from oracle.refprogram import RefProgram

    # RefProgram follows the shared-weights record oracle/build_ref.py leaves after deduplicating weight files.
    logits = np.asarray(RefProgram("c4_slice_fwd16")(tokens), np.float32)
    build_ref.build("c4_slice_route16")
    _, routes = RefProgram("c4_slice_route16")(tokens)
    # The oracle's bf16 gate logits identify exact ties at the top-k boundary, where the reference's choice is
    # unspecified (nth_element, chroma/_src/codegen/cpu/kernels.h:153-185; docs/runtime.md "Tied top-k values").
    from oracle import gpt_oss as og

    trace = og.Trace()
    og.forward(og.Config.from_model_config(build_ref.small_config("c4_slice")), og.Params.from_module(model), tokens, trace)
    np.savez_compressed(HERE / "c4_slice.npz", tokens=tokens, sample_cols=SAMPLE, weights_digest=np.array(digest(model)),
                        routes=routes, oracle_gates=np.stack(trace.gates), **summary(logits))
    print("c4 slice done", flush=True)


def main() -> None:
    import sys as _sys

    if "--c4" in _sys.argv:
        c4_slice()
        return
    from oracle import build_ref, refimport

    refimport.install()
    import chroma
    import torch
    from scripts.export import make_dev_model

    for name in build_ref.names():
        build_ref.build(name)
    R = build_ref.ROOT

    dev_digest = digest(make_dev_model(0))

    # ---- C1: dev forward, 8 tokens, five token sets, with per-layer routing.
    sets = c1_token_sets()
    from oracle.refprogram import RefProgram

    fwd, route = RefProgram("c1_fwd8"), RefProgram("c1_route8")
    outs, routes = [], []
    for tokens in sets:
        outs.append(summary(fwd(tokens)))
        logits2, r = route(tokens)
        routes.append(r)
        assert np.array_equal(np.argmax(logits2, -1), outs[-1]["argmax"])
    np.savez_compressed(HERE / "c1_fwd8.npz", tokens=sets, routes=np.stack(routes), sample_cols=SAMPLE,
                        weights_digest=np.array(dev_digest), **stack(outs, ""))
    print("c1 done", flush=True)

    # ---- C2: dev decode through the reference Decoder (prefill chunk 8, context 256).
    def decoder():  # type: ignore[no-untyped-def]
        return chroma.Decoder(RefProgram("c2_prefill8"), RefProgram("c2_decode"))

    rng = np.random.default_rng(1)
    prompt = rng.integers(0, V, 8)
    forced = rng.integers(0, V, 24)
    steps = []
    with decoder() as dec:
        steps.append(summary(dec.append(prompt)))
        for t in forced:
            steps.append(summary(dec.append([int(t)])))
    # Long run through the ring wrap: 8-token prefill + 292 single steps (context 256).
    long_tokens = np.random.default_rng(2).integers(0, V, 300)
    long_argmax, long_tail = [], []
    with decoder() as dec:
        out = dec.append(long_tokens[:8])
        long_argmax.append(int(np.argmax(out)))
        for i, t in enumerate(long_tokens[8:]):
            out = dec.append([int(t)])
            long_argmax.append(int(np.argmax(out)))
            if i >= len(long_tokens) - 8 - 4:
                long_tail.append(summary(out))
    # Batch: 16 independent sequences of 8-token prefill + 4 forced steps.
    batch_tokens = np.random.default_rng(3).integers(0, V, (16, 12))
    batch = []
    for seq in batch_tokens:
        with decoder() as dec:
            per = [summary(dec.append(seq[:8]))]
            for t in seq[8:]:
                per.append(summary(dec.append([int(t)])))
        batch.append(stack(per, ""))
    np.savez_compressed(
        HERE / "c2_decode.npz", prompt=prompt, forced=forced, long_tokens=long_tokens,
        long_argmax=np.array(long_argmax, np.int64), batch_tokens=batch_tokens, sample_cols=SAMPLE,
        weights_digest=np.array(dev_digest), **stack(steps, "step_"), **stack(long_tail, "tail_"), **stack(batch, "batch_"),
    )
    print("c2 done", flush=True)

    # ---- C3: micrograph at 16 rows (full output) and at full size (checksums).
    from ml_dtypes import bfloat16

    def bits(t):  # type: ignore[no-untyped-def]
        return t.view(torch.uint16).numpy()

    inputs16 = build_ref.micro_inputs(16, 4096)
    w = build_ref.micro_module(16, 4096).norm.scale.detach().numpy().astype(np.float32)
    with chroma.Program(R / "c3_micro_16") as micro:
        out16 = micro(*[bits(t).view(bfloat16) for t in inputs16])
    inputs = build_ref.micro_inputs(16384, 4096)
    with chroma.Program(R / "c3_micro_full") as micro:
        full = micro(*[bits(t).view(bfloat16) for t in inputs])
    full_bits = full.view(np.uint16)
    np.savez_compressed(
        HERE / "c3_micro.npz", w=w, out16=out16.view(np.uint16), x16=bits(inputs16[0]),
        full_rowsum=full.astype(np.float32).astype(np.float64).sum(-1),
        full_sha256=np.array(hashlib.sha256(full_bits.tobytes()).hexdigest()),
        full_rows=full_bits[[0, 1, 8191, 16383]], full_input_row0=bits(inputs[0])[0],
    )
    print("c3 done", flush=True)

    # ---- Small models (reference tests' shapes): full logits.
    small: dict[str, np.ndarray] = {}
    for dtype_name in ("float32", "bfloat16"):
        model = build_ref.cuda_small_model(getattr(torch, dtype_name))
        small[f"{dtype_name}_digest"] = np.array(digest(model))
        sets4 = np.array([[0, 3, 6, 9], [1, 4, 2, 7], [0, 2, 9, 16]], np.int64)
        with chroma.Program(R / f"small_{dtype_name}_full4") as full4:
            small[f"{dtype_name}_full4_tokens"] = sets4
            small[f"{dtype_name}_full4"] = np.stack([np.asarray(full4(t), np.float32) for t in sets4])
        tokens = (np.arange(14) * 7 + 3) % 17
        logs = []
        with chroma.Decoder(chroma.Program(R / f"small_{dtype_name}_prefill5"),
                            chroma.Program(R / f"small_{dtype_name}_decode"), sliding_window=3) as dec:
            pos = 0
            for size in (2, 1, 4, 5, 2):
                logs.append(np.asarray(dec.append(tokens[pos : pos + size]), np.float32))
                pos += size
            dec.reset()
            logs.append(np.asarray(dec.append(tokens), np.float32))
        small[f"{dtype_name}_decoder"] = np.concatenate(logs)
    for head_dim in (8, 64):
        model = build_ref.random_transformer(build_ref.small_config(f"decoder_small_{head_dim}"), seed=5, std=0.03)
        small[f"dec{head_dim}_digest"] = np.array(digest(model))
        tokens = (np.arange(23) * 7 + 3) % 31
        logs = []
        with chroma.Decoder(chroma.Program(R / f"dec{head_dim}_prefill7"), chroma.Program(R / f"dec{head_dim}_decode"),
                            sliding_window=3) as dec:
            pos = 0
            for size in (3, 1, 5, 7, 1, 6):
                logs.append(np.asarray(dec.append(tokens[pos : pos + size]), np.float32))
                pos += size
            dec.reset()
            logs.append(np.asarray(dec.append(tokens), np.float32))
            dec.reset()
            logs.append(np.asarray(dec.append(tokens[:3]), np.float32))
        small[f"dec{head_dim}_decoder"] = np.concatenate(logs)
    np.savez_compressed(HERE / "small.npz", **small)
    print("small done", flush=True)


if __name__ == "__main__":
    main()
