"""The boundary, exercised by the reference's own runtime: an unmodified ``chroma.Program`` loads chroma_b200
artefacts and an unmodified ``chroma.Decoder`` drives a chroma_b200 prefill/decode pair.

The reference's loader (chroma/_src/program.py:83-101) checks the manifest version, the Python ABI and the library
module's ``signature``, then constructs ``Model(weights_path)`` and calls ``run(inputs, outputs)``; its Decoder
(chroma/_src/decoder.py:96-139) builds the masks and positions on the host and passes the whole cache as the
seven-input protocol every step. The reference package comes from its source tree when present, else from the
patched copy oracle/build_ref.py stages under oracle/_ref/pkg (test infrastructure).

* ``chroma.Program`` over a chroma_b200 artefact runs the same native program as ``chroma_b200.Program``: identical
  bits, the same errors.
* ``chroma.Decoder`` over a chroma_b200 pair runs the per-layer kernels on host-built inputs; ``chroma_b200.Decoder``
  keeps the cache on the device and runs batch-1 decode steps in the one-launch cluster kernel, whose attention
  splits the keys differently: greedy ids identical, logits within the fp32 bar, and both match the reference's
  golden outputs.
"""

from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

import chroma_b200
from tests import test_gpu_gptoss as tg
from tests.conftest import ROOT, golden

pytestmark = pytest.mark.gpu
FP32 = {"rtol": 1e-4, "atol": 1e-5}


def reference_chroma():  # type: ignore[no-untyped-def]
    from oracle import refimport

    try:
        return refimport.runtime()
    except ModuleNotFoundError as exc:
        pytest.skip(f"the reference's chroma package is not available here: {exc}")


def test_reference_program_loads_b200_artifact(gpu: None) -> None:
    chroma = reference_chroma()
    path = tg._TMP / "dev_fwd8"
    tg.dev_forward()  # writes the artefact
    g = golden("c1_fwd8")
    with chroma.Program(path) as ref_loaded, chroma_b200.Program(path) as ours:
        assert "B200" in ref_loaded.device
        assert ref_loaded.inputs == ours.inputs and ref_loaded.outputs == ours.outputs
        for s, tokens in enumerate(g["tokens"]):
            a, b = ref_loaded(tokens), ours(tokens)
            np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
            np.testing.assert_array_equal(np.argmax(a, -1), g["argmax"][s])
        out = np.empty_like(a)
        assert ref_loaded(g["tokens"][0], out=out) is out
        with pytest.raises(IndexError):
            ref_loaded(np.full(8, 201088, dtype=np.int64))
        np.testing.assert_array_equal(ref_loaded(g["tokens"][0]), out)


def test_reference_decoder_drives_b200_pair(gpu: None) -> None:
    chroma = reference_chroma()
    g = golden("c2_decode")
    prefill, decode = tg.dev_pair()
    tokens = [g["prompt"]] + [[int(t)] for t in g["forced"]]
    with chroma.Decoder(chroma.Program(prefill), chroma.Program(decode)) as ref_dec:
        ref_outs = [np.asarray(ref_dec.append(t)) for t in tokens]
    with chroma_b200.Decoder(chroma_b200.Program(prefill), chroma_b200.Program(decode)) as dec:
        outs = [np.asarray(dec.append(t)) for t in tokens]
    for i, (a, b) in enumerate(zip(ref_outs, outs)):
        assert int(np.argmax(a)) == int(np.argmax(b)) == int(g["step_argmax"][i][0])
        np.testing.assert_allclose(a, b, **FP32)
        np.testing.assert_allclose(a[:, g["sample_cols"]], g["step_sample"][i], **FP32)


def test_reference_program_is_torch_free(gpu: None) -> None:
    """Loading and running a chroma_b200 artefact through the reference's Program imports no Torch."""
    reference_chroma()
    tg.dev_forward()
    code = (
        "import sys, numpy as np\n"
        "from oracle import refimport\n"
        "chroma = refimport.runtime()\n"
        "with chroma.Program(sys.argv[1]) as p:\n"
        "    p(np.arange(8, dtype=np.int64))\n"
        "assert 'torch' not in sys.modules, 'torch imported'\n"
    )
    env = dict(os.environ, PYTHONPATH=str(ROOT))
    subprocess.run([sys.executable, "-c", code, str(tg._TMP / "dev_fwd8")], check=True, env=env, cwd=str(ROOT))


def test_reference_program_loads_generic_b200_artifact(gpu: None, tmp_path) -> None:  # type: ignore[no-untyped-def]
    """A generic graph compiled by this backend, loaded and run by the reference's unmodified Program."""
    import torch

    from tests import generic_cases as gc

    chroma = reference_chroma()
    case = gc.by_name()["reductions_f32"]
    inputs = case.inputs()
    chroma_b200.compile(torch.export.export(case.module(), inputs), tmp_path / "g").close()
    arrays = [gc.to_numpy(t) for t in inputs]
    with chroma.Program(tmp_path / "g") as ref_loaded, chroma_b200.Program(tmp_path / "g") as ours:
        for a, b in zip(ref_loaded(*arrays), ours(*arrays)):
            np.testing.assert_array_equal(a, b)
