"""GPU parity of the GPT-OSS kernels against the reference's golden vectors and the oracle.

Bars (from the backend's contract): argmax token ids and routing indices identical; fp32 logits within 1e-4
relative (atol 1e-5 for near-zero logits); bf16 logits within 2e-2 relative (atol 1e-2). Against the golden
summaries of the reference's full logits rows: a fixed sample of 4,096 columns, the 16 largest logits (index and
value) and the float64 row sum (helpers.assert_top_and_rowsum).
"""

from __future__ import annotations

import functools
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch

import chroma_b200
from chroma_b200 import models
from oracle import gpt_oss as og
from tests import helpers
from tests.conftest import ROOT, golden

pytestmark = pytest.mark.gpu
FP32 = {"rtol": 1e-4, "atol": 1e-5}
BF16 = {"rtol": 2e-2, "atol": 1e-2}
_TMP = Path(tempfile.mkdtemp(prefix="chroma-b200-tests-"))


@functools.lru_cache(maxsize=None)
def dev_forward() -> chroma_b200.Program:
    ep = torch.export.export(helpers.dev_model(), (torch.arange(8),))
    return chroma_b200.compile(ep, _TMP / "dev_fwd8")


@functools.lru_cache(maxsize=None)
def dev_pair() -> tuple[Path, Path]:
    model = helpers.dev_model()
    chroma_b200.compile(models.export_cached(model, 256, 8), _TMP / "dev_prefill8").close()
    chroma_b200.compile(models.export_cached(model, 256, 1), _TMP / "dev_decode").close()
    return _TMP / "dev_prefill8", _TMP / "dev_decode"


def dev_decoder() -> chroma_b200.Decoder:
    prefill, decode = dev_pair()
    return chroma_b200.Decoder(chroma_b200.Program(prefill), chroma_b200.Program(decode))


def test_c1_forward_matches_reference(gpu: None) -> None:
    g = golden("c1_fwd8")
    program = dev_forward()
    assert program.stats["backend"] == "cuda" and "B200" in program.device
    for s, tokens in enumerate(g["tokens"]):
        logits = program(tokens)
        np.testing.assert_array_equal(np.argmax(logits, -1), g["argmax"][s])
        np.testing.assert_allclose(logits[:, g["sample_cols"]], g["sample"][s], **FP32)
        helpers.assert_top_and_rowsum(logits, g["top_idx"][s], g["top_val"][s], g["rowsum"][s], **FP32)
        routes = program.native.routes()
        np.testing.assert_array_equal(routes, g["routes"][s])


def test_c1_routing_margins_are_reported(gpu: None) -> None:
    # Bit-exact routing is only meaningful when the 4th/5th gate logits are separated by more than the
    # accumulated rounding error; record the smallest margin the fixtures exercise.
    g = golden("c1_fwd8")
    cfg, p = helpers.dev_oracle()
    margins = []
    for tokens in g["tokens"]:
        trace = og.Trace()
        og.forward(cfg, p, tokens, trace)
        for gate in trace.gates:
            top = np.sort(gate, axis=-1)[:, ::-1]
            margins.append(float(np.min(top[:, 3] - top[:, 4])))
    assert min(margins) > 1e-5, min(margins)


def test_c1_repeated_calls_out_reuse_and_index_errors(gpu: None) -> None:
    program = dev_forward()
    tokens = np.arange(8, dtype=np.int64)
    first = program(tokens)
    kept = first.copy()
    program(tokens + 1)
    np.testing.assert_array_equal(first, kept)
    out = np.empty_like(first)
    assert program(tokens, out=out) is out
    np.testing.assert_array_equal(out, first)
    for bad in (models.dev.vocab_size, -1, 2**40):
        with pytest.raises(IndexError):
            program(np.full(8, bad, dtype=np.int64))
        np.testing.assert_array_equal(program(tokens), first)
    for invalid in (np.arange(8, dtype=np.int32), np.arange(7, dtype=np.int64)):
        with pytest.raises(ValueError):
            program(invalid)
    with pytest.raises(ValueError):
        program()
    readonly = np.empty_like(first)
    readonly.setflags(write=False)
    with pytest.raises(ValueError):
        program(tokens, out=readonly)
    noncontiguous = np.arange(16, dtype=np.int64)[::2]
    np.testing.assert_allclose(program(noncontiguous), og.forward(*helpers.dev_oracle(), noncontiguous), **FP32)


def test_c1_cluster_forward_matches_per_layer_kernels(gpu: None) -> None:
    """The one-launch cluster forward (up to 8 tokens, batch 1, fp32) against the per-layer kernel chain
    (CHROMA_B200_FWD_CLUSTER=0, in a subprocess) at 8 and 5 tokens: the same additions in the same order, so
    identical logits and routes, bit for bit; and the same index error for an out-of-range id."""
    rng = np.random.default_rng(81)
    cases = {}
    for n in (8, 5):
        path = _TMP / f"dev_fwd{n}_cluster"
        with chroma_b200.compile(torch.export.export(helpers.dev_model(), (torch.arange(n),)), path) as program:
            tokens = rng.integers(0, models.dev.vocab_size, (3, n))
            got, routes = [], []
            for t in tokens:
                got.append(np.asarray(program(t)))
                routes.append(program.native.routes())
            got, routes = np.stack(got), np.stack(routes)
            assert 0 < program.native.launches <= 3, program.native.launches  # prefetch, cluster, vocab
            with pytest.raises(IndexError):
                program(np.full(n, models.dev.vocab_size, dtype=np.int64))
            np.testing.assert_array_equal(np.asarray(program(tokens[0])), got[0])
        np.save(_TMP / f"fwd{n}_cluster_tokens.npy", tokens)
        cases[n] = (path, got, routes)
    code = (
        "import sys, numpy as np\n"
        "from chroma_b200 import Program\n"
        "with Program(sys.argv[1]) as p:\n"
        "    toks = np.load(sys.argv[2])\n"
        "    logits, routes = [], []\n"
        "    for t in toks:\n"
        "        logits.append(np.asarray(p(t)))\n"
        "        routes.append(p.native.routes())\n"
        "    np.savez(sys.argv[3], logits=np.stack(logits), routes=np.stack(routes), launches=p.native.launches)\n"
    )
    env = dict(os.environ, CHROMA_B200_FWD_CLUSTER="0", PYTHONPATH=str(ROOT))
    for n, (path, got, routes) in cases.items():
        out = _TMP / f"fwd{n}_per_layer.npz"
        subprocess.run([sys.executable, "-c", code, str(path), str(_TMP / f"fwd{n}_cluster_tokens.npy"), str(out)],
                       check=True, env=env)
        ref = np.load(out)
        assert int(ref["launches"]) > 8
        np.testing.assert_array_equal(got.view(np.uint32), ref["logits"].view(np.uint32))
        np.testing.assert_array_equal(routes, ref["routes"])


def test_c1_last_row_program_matches_forward_row(gpu: None) -> None:
    """The UncachedTransformer variant (tokens[8], position[1] -> logits[1, V]) against the full forward's row at
    that position, bit for bit (both on the cluster forward); negative positions wrap, out-of-range ones raise
    IndexError and leave the program usable."""
    model = models.make_dev_model(0)
    tokens = np.random.default_rng(17).integers(0, models.dev.vocab_size, 8)
    with chroma_b200.compile_model(model, _TMP / "last8", steps=8, last=True) as last, \
            chroma_b200.compile_model(model, _TMP / "fwd8_rows", steps=8) as fwd:
        full = np.asarray(fwd(tokens))
        for pos in (7, 0, 3, -1, -8):
            row = np.asarray(last(tokens, np.array([pos], np.int64)))
            assert row.shape == (1, models.dev.vocab_size)
            np.testing.assert_array_equal(row.view(np.uint32), full[pos % 8][None].view(np.uint32))
        for bad in (8, -9):
            with pytest.raises(IndexError):
                last(tokens, np.array([bad], np.int64))
        np.testing.assert_array_equal(np.asarray(last(tokens, np.array([2], np.int64))).view(np.uint32),
                                      full[2][None].view(np.uint32))


def test_c2_decoder_matches_reference(gpu: None) -> None:
    g = golden("c2_decode")
    with dev_decoder() as dec:
        outs = [dec.append(g["prompt"])] + [dec.append([int(t)]) for t in g["forced"]]
        assert dec.position == 8 + len(g["forced"])
    for i, out in enumerate(outs):
        assert out.shape == (1, models.dev.vocab_size)
        assert int(np.argmax(out)) == int(g["step_argmax"][i][0])
        np.testing.assert_allclose(out[:, g["sample_cols"]], g["step_sample"][i], **FP32)
        helpers.assert_top_and_rowsum(out, g["step_top_idx"][i], g["step_top_val"][i], g["step_rowsum"][i], **FP32)


def test_c2_decoder_ring_wrap(gpu: None) -> None:
    g = golden("c2_decode")
    tokens = g["long_tokens"]
    with dev_decoder() as dec:
        ids = [int(np.argmax(dec.append(tokens[:8])))]
        tail = []
        for i, t in enumerate(tokens[8:]):
            out = dec.append([int(t)])
            ids.append(int(np.argmax(out)))
            if i >= len(tokens) - 8 - 4:
                tail.append(out)
    np.testing.assert_array_equal(ids, g["long_argmax"])
    for i, (out, want) in enumerate(zip(tail, g["tail_sample"])):
        np.testing.assert_allclose(out[:, g["sample_cols"]], want, **FP32)
        helpers.assert_top_and_rowsum(out, g["tail_top_idx"][i], g["tail_top_val"][i], g["tail_rowsum"][i], **FP32)


def _decode_sequence(prefill: str, decode: str, tokens: np.ndarray) -> tuple[np.ndarray, int]:
    with chroma_b200.Decoder(chroma_b200.Program(prefill), chroma_b200.Program(decode)) as dec:
        outs = [dec.append(tokens[:8])] + [dec.append([int(t)]) for t in tokens[8:]]
        return np.concatenate(outs), dec._native.step_launches


def test_c2_cluster_decode_matches_per_layer_kernels(gpu: None) -> None:
    """The one-launch cluster decode of the batch-1 fp32 program against the per-layer kernel chain
    (CHROMA_B200_DECODE_CLUSTER=0, in a subprocess) through 292 decode steps and a ring wrap: greedy ids identical,
    logits within fp32 rounding (the two paths split the keys of the softmax differently)."""
    tokens = golden("c2_decode")["long_tokens"]
    prefill, decode = dev_pair()
    out = _TMP / "per_layer.npz"
    code = (
        "import sys, numpy as np\n"
        "import tests.test_gpu_gptoss as t\n"
        "logits, launches = t._decode_sequence(sys.argv[1], sys.argv[2], np.load(sys.argv[3])['long_tokens'])\n"
        "np.savez(sys.argv[4], logits=logits, launches=launches)\n"
    )
    env = dict(os.environ, CHROMA_B200_DECODE_CLUSTER="0", PYTHONPATH=str(ROOT))
    subprocess.run([sys.executable, "-c", code, str(prefill), str(decode), str(ROOT / "tests/golden/c2_decode.npz"),
                    str(out)], check=True, env=env, cwd=str(ROOT))
    ref = np.load(out)
    got, launches = _decode_sequence(str(prefill), str(decode), tokens)
    assert launches < 8 < int(ref["launches"]), (launches, int(ref["launches"]))
    np.testing.assert_array_equal(np.argmax(got, -1), np.argmax(ref["logits"], -1))
    np.testing.assert_allclose(got, ref["logits"], rtol=1e-5, atol=1e-6)


def test_decoder_logits_are_independent_page_locked_arrays(gpu: None) -> None:
    """Returned logits live in recycled page-locked blocks: a result the caller keeps is never overwritten by later
    steps, results are writable, and a block comes back to the pool only when its last view is gone."""
    with dev_decoder() as dec:
        a = dec.append([1, 2, 3])
        kept = a.copy()
        view = a[:, :16]
        b = dec.append([4])
        del a
        c = dec.append([5])
        np.testing.assert_array_equal(view, kept[:, :16])
        assert b.flags.writeable and c.flags.writeable and c.flags.c_contiguous
        assert not np.shares_memory(b, c)
        b[0, 0] = 0.0
        with dev_decoder() as ref:
            want = ref.append([1, 2, 3, 4, 5])
        np.testing.assert_allclose(c, want, **FP32)


def test_grouped_moe_matches_per_slot_kernels(gpu: None) -> None:
    """The expert-grouped MoE kernels (16+ tokens per launch) against the per-(token, slot) kernels
    (CHROMA_B200_PER_SLOT_MOE=1, in a subprocess): the same arithmetic in the same order, so identical bits; and the
    routing record of every layer."""
    path = _TMP / "dev_fwd48"
    tokens = np.random.default_rng(48).integers(0, models.dev.vocab_size, 48)
    with chroma_b200.compile(torch.export.export(helpers.dev_model(), (torch.arange(48),)), path) as program:
        got = np.asarray(program(tokens))
    np.save(_TMP / "fwd48_tokens.npy", tokens)
    code = (
        "import sys, numpy as np\n"
        "from chroma_b200 import Program\n"
        "with Program(sys.argv[1]) as p:\n"
        "    np.save(sys.argv[3], p(np.load(sys.argv[2])))\n"
    )
    env = dict(os.environ, CHROMA_B200_PER_SLOT_MOE="1", PYTHONPATH=str(ROOT))
    subprocess.run([sys.executable, "-c", code, str(path), str(_TMP / "fwd48_tokens.npy"), str(_TMP / "fwd48_ref.npy")],
                   check=True, env=env)
    want = np.load(_TMP / "fwd48_ref.npy")
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    np.testing.assert_allclose(got, og.forward(*helpers.dev_oracle(), tokens), **FP32)


def test_c2_device_generation_matches_host_steps(gpu: None) -> None:
    """Device-resident greedy generation of one sequence (the cluster kernel commits its rows in place and derives
    the position itself) against host steps through Decoder.append, across a ring wrap: the same token ids, and
    after it the same committed cache."""
    prefill, decode = dev_pair()
    prompt = golden("c2_decode")["prompt"]
    with chroma_b200.BatchDecoder(chroma_b200.Program(prefill), chroma_b200.Program(decode), 1) as bd:
        first = bd.append(prompt[None, :], argmax=True)
        ids = bd.generate(first, 260)[0]
        cache = bd._native.read()
    with dev_decoder() as dec:
        want = [int(np.argmax(dec.append(prompt)))]
        for _ in range(260):
            want.append(int(np.argmax(dec.append([want[-1]]))))
        dec._flush()  # commit the last host step's rows, as every device step does
        ref = dec._native.read()
    assert [int(first[0])] + ids.tolist() == want
    for got_part, ref_part in zip(cache, ref):
        np.testing.assert_array_equal(np.asarray(got_part).reshape(-1), np.asarray(ref_part).reshape(-1))


def test_c2_batch_decoder_matches_reference(gpu: None) -> None:
    g = golden("c2_decode")
    prefill, decode = dev_pair()
    toks = g["batch_tokens"]
    with chroma_b200.BatchDecoder(chroma_b200.Program(prefill), chroma_b200.Program(decode), len(toks)) as dec:
        outs = [dec.append(toks[:, :8])] + [dec.append(toks[:, 8 + i : 9 + i]) for i in range(4)]
        dec.reset()
        ids = [dec.append(toks[:, :8], argmax=True)] + [dec.append(toks[:, 8 + i : 9 + i], argmax=True) for i in range(4)]
    for step, (out, am) in enumerate(zip(outs, ids)):
        np.testing.assert_array_equal(np.argmax(out, -1), g["batch_argmax"][:, step, 0])
        np.testing.assert_array_equal(am, g["batch_argmax"][:, step, 0])
        np.testing.assert_allclose(out[:, g["sample_cols"]], g["batch_sample"][:, step, 0], **FP32)
        helpers.assert_top_and_rowsum(out, g["batch_top_idx"][:, step, 0], g["batch_top_val"][:, step, 0],
                                      g["batch_rowsum"][:, step, 0], **FP32)


def test_decoder_errors_keep_state_and_recover(gpu: None) -> None:
    # A failed append leaves the committed state as it was (decoder.py:130-137). A failing call may first apply
    # the previous step's staged rows, which replaces the state object but not its content.
    with dev_decoder() as dec:
        dec.append([1, 2, 3])
        before = dec._state
        for bad in ([-1], [models.dev.vocab_size], [2**40]):
            with pytest.raises(IndexError):
                dec.append(bad)
            assert dec.position == before.position == 3
            np.testing.assert_array_equal(dec._state.slots, before.slots)
        with pytest.raises(TypeError):
            dec.append([1.5])
        with pytest.raises(ValueError):
            dec.append([])
        # KeyboardInterrupt after the native call returns: nothing is committed (tests/test_decoder.py:122-131).
        state = dec._state
        step = dec._native.step_one

        def interrupted(*args, **kwargs):  # type: ignore[no-untyped-def]
            step(*args, **kwargs)
            raise KeyboardInterrupt

        dec._native.step_one = interrupted
        with pytest.raises(KeyboardInterrupt):
            dec.append([4])
        dec._native.step_one = step
        assert dec._state is state and dec.position == 3
        a = dec.append([4])
    with dev_decoder() as ref:
        b = ref.append([1, 2, 3, 4])
    np.testing.assert_allclose(a, b, **FP32)


def test_small_models_fp32_and_bf16(gpu: None) -> None:
    g = golden("small")
    for dtype, tol in ((torch.float32, FP32), (torch.bfloat16, BF16)):
        name = str(dtype).split(".")[1]
        model = helpers.cuda_small_model(dtype)
        tokens4 = g[f"{name}_full4_tokens"]
        with chroma_b200.compile(torch.export.export(model, (torch.tensor(tokens4[0]),)), _TMP / f"small_{name}") as prog:
            for tokens, want in zip(tokens4, g[f"{name}_full4"]):
                np.testing.assert_allclose(np.asarray(prog(tokens), np.float32), want, **tol)
            with pytest.raises(IndexError):
                prog(np.full(4, 17, dtype=np.int64))
        pre = chroma_b200.compile(models.export_cached(model, 5, 5), _TMP / f"small_{name}_pre")
        dec_p = chroma_b200.compile(models.export_cached(model, 5, 1), _TMP / f"small_{name}_dec")
        tokens = (np.arange(14) * 7 + 3) % 17
        with chroma_b200.Decoder(pre, dec_p, sliding_window=3) as dec:
            logs, pos = [], 0
            for size in (2, 1, 4, 5, 2):
                logs.append(np.asarray(dec.append(tokens[pos : pos + size]), np.float32))
                pos += size
            dec.reset()
            assert dec.position == 0
            logs.append(np.asarray(dec.append(tokens), np.float32))
        np.testing.assert_allclose(np.concatenate(logs), g[f"{name}_decoder"], **tol)


def test_small_decoders_window_yarn_wrap(gpu: None) -> None:
    g = golden("small")
    for head_dim in (8, 64):
        model = helpers.decoder_small_model(head_dim)
        pre = chroma_b200.compile(models.export_cached(model, 7, 7), _TMP / f"dec{head_dim}_pre")
        dec_p = chroma_b200.compile(models.export_cached(model, 7, 1), _TMP / f"dec{head_dim}_dec")
        tokens = (np.arange(23) * 7 + 3) % 31
        with chroma_b200.Decoder(pre, dec_p, sliding_window=3) as dec:
            logs, pos = [], 0
            for size in (3, 1, 5, 7, 1, 6):
                logs.append(dec.append(tokens[pos : pos + size]))
                pos += size
            dec.reset()
            logs.append(dec.append(tokens))
            dec.reset()
            logs.append(dec.append(tokens[:3]))
        np.testing.assert_allclose(np.concatenate(logs), g[f"dec{head_dim}_decoder"], **FP32)


def test_torch_free_reload(gpu: None) -> None:
    program = dev_forward()
    np.save(_TMP / "c1_expected.npy", program(np.arange(8, dtype=np.int64)))
    code = """
import sys
import numpy as np
from chroma_b200 import Program
assert 'torch' not in sys.modules
with Program(sys.argv[1]) as model:
    np.testing.assert_array_equal(model(np.arange(8, dtype=np.int64)), np.load(sys.argv[2]))
assert 'torch' not in sys.modules
"""
    env = dict(os.environ, PYTHONPATH=str(ROOT))
    subprocess.run([sys.executable, "-c", code, str(_TMP / "dev_fwd8"), str(_TMP / "c1_expected.npy")], check=True, env=env)
