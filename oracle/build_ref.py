"""Test infrastructure: build the reference's own CPU programs into ``oracle/_ref/<name>/``.

This is the recipe for the reference implementation used as (1) the source of the golden fixtures under
``tests/golden`` and (2) the timed CPU baseline (``bench.py --impl reference``). It runs only where the
reference tree exists (the development container). It imports the reference through ``oracle.refimport``
(in-memory Python 3.12 patches, nothing copied), exports each workload with the reference's own model code
(chroma/models/gpt_oss.py, chroma/models/cached.py, scripts/export.py:16-29) and compiles it with the
reference's own compiler, ``chroma.compile(..., backend="cpu", blas=False)`` (chroma/__init__.py:14-23).
``blas=False`` selects the portable loops (chroma/_src/codegen/cpu/codegen.py:404-409), since this machine
has no CBLAS; they also fix the summation order (chroma/_src/codegen/cpu/kernels.h:24-44).

Each output directory is a normal reference artefact: ``model.json``, ``_chroma_<uuid>.<abi>.so``,
``weights-<sha>.bin`` and ``model.cc``. The ``.so`` exposes the reference's native protocol
(``Model(weights).run(inputs, outputs)``, chroma/_src/core/bindings.h:35-75) and needs only NumPy to run,
so the directory can be loaded on a machine without the reference sources (``oracle/refprogram.py``).

Usage: ``python -m oracle.build_ref [name ...]`` (default: every program that is missing).
"""

from __future__ import annotations

import dataclasses
import json
import sys
import time
from collections.abc import Callable
from pathlib import Path

ROOT = Path(__file__).resolve().parent / "_ref"


def _reference():  # type: ignore[no-untyped-def]
    from oracle import refimport

    refimport.install()
    import chroma  # noqa: F401

    return chroma


def micro_module(rows: int, cols: int, seed: int = 0):  # type: ignore[no-untyped-def]
    """The C3 micrograph: y = RMSNorm(x)*w (fp32 math, bf16 result), z = y*g, out = z*sigmoid(z)*u + x.

    Uses the reference's RMSNorm module (chroma/models/gpt_oss.py:30-41). SiLU is spelled z*sigmoid(z)
    because aten.silu is not a supported operator (chroma/_src/lowering.py:34-86).
    """
    import torch

    from chroma.models.gpt_oss import RMSNorm

    class Micro(torch.nn.Module):
        def __init__(self) -> None:
            super().__init__()
            self.norm = RMSNorm(cols)
            g = torch.Generator().manual_seed(seed + 1)
            with torch.no_grad():
                self.norm.scale.copy_(torch.normal(1.0, 0.02, (cols,), generator=g))

        def forward(self, x, g, u):  # type: ignore[no-untyped-def]
            z = self.norm(x) * g
            return z * torch.sigmoid(z) * u + x

    return Micro().eval().requires_grad_(False)


def micro_inputs(rows: int, cols: int, seed: int = 0):  # type: ignore[no-untyped-def]
    import torch

    g = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(rows, cols, generator=g).to(torch.bfloat16) for _ in range(3))


def small_config(kind: str):  # type: ignore[no-untyped-def]
    """Small GPT-OSS configurations taken from the reference's tests."""
    from chroma.models.variants import dev

    if kind == "cuda_small":  # tests/test_cuda.py:29-43 and tests/test_bf16.py:42-55
        return dataclasses.replace(
            dev, num_hidden_layers=1, num_experts=2, experts_per_token=2, vocab_size=17, hidden_size=8,
            intermediate_size=8, head_dim=4, num_attention_heads=2, num_key_value_heads=1, sliding_window=3,
        )
    if kind.startswith("decoder_small"):  # tests/test_decoder.py:21-37
        head_dim = int(kind.rsplit("_", 1)[1])
        return dataclasses.replace(
            dev, num_hidden_layers=2, hidden_size=16, intermediate_size=16, vocab_size=31, num_experts=4,
            experts_per_token=2, num_attention_heads=4, num_key_value_heads=2, head_dim=head_dim, sliding_window=3,
            initial_context_length=4096, rope_scaling_factor=32.0 if head_dim == 64 else 1.0,
        )
    if kind == "c4_slice":  # one layer of the GPT-OSS-20B-shaped benchmark model (full widths and vocabulary)
        return dataclasses.replace(
            dev, num_hidden_layers=1, hidden_size=2880, intermediate_size=2880, num_attention_heads=64,
            num_key_value_heads=8, head_dim=64, num_experts=32, experts_per_token=4,
        )
    if kind == "yarn_small":  # tests/test_runtime.py:209-228
        return dataclasses.replace(
            dev, num_hidden_layers=2, hidden_size=16, head_dim=64, num_attention_heads=4, num_key_value_heads=2,
            vocab_size=257, sliding_window=3, initial_context_length=4096, rope_scaling_factor=32.0,
        )
    raise KeyError(kind)


def random_transformer(config, *, seed: int, std: float, dtype=None):  # type: ignore[no-untyped-def]
    """Unit norm scales, N(0, std) elsewhere, drawn in fp32 (the helper at tests/helpers.py:19-29)."""
    import torch

    from chroma.models.gpt_oss import Transformer

    with torch.random.fork_rng(devices=[]), torch.no_grad():
        torch.manual_seed(seed)
        model = Transformer(config, device=torch.device("cpu")).float().eval().requires_grad_(False)
        for name, parameter in model.named_parameters():
            if name.endswith(".scale"):
                parameter.fill_(1)
            else:
                parameter.normal_(std=std)
    return model.to(dtype or torch.float32)


def cuda_small_model(dtype):  # type: ignore[no-untyped-def]
    """tests/test_cuda.py:29-43: seed 5, std 0.1, cast after init."""
    import torch

    from chroma.models.gpt_oss import Transformer

    config = small_config("cuda_small")
    with torch.random.fork_rng(devices=[]), torch.no_grad():
        torch.manual_seed(5)
        model = Transformer(config, device=torch.device("cpu")).to(dtype).eval().requires_grad_(False)
        for name, parameter in model.named_parameters():
            if name.endswith(".scale"):
                parameter.fill_(1)
            else:
                parameter.normal_(std=0.1)
    return model


class RoutingProbe:
    """Wraps a reference Transformer so its compiled program also returns every layer's top-k routing.

    The probe calls the reference's own submodules in the order of TransformerBlock.forward
    (chroma/models/gpt_oss.py:277-283) and MLPBlock.forward (:243-265); the extra output is the
    ``torch.topk(..., sorted=True).indices`` each MLP block computes (:246).
    """

    @staticmethod
    def build(model):  # type: ignore[no-untyped-def]
        import torch

        class Probe(torch.nn.Module):
            def __init__(self) -> None:
                super().__init__()
                self.model = model

            def forward(self, tokens):  # type: ignore[no-untyped-def]
                x = self.model.embedding(tokens)
                routes = []
                for block in self.model.block:
                    x = block.attn(x)
                    t = block.mlp.norm(x)
                    g = block.mlp.gate(t)
                    routes.append(torch.topk(g, k=block.mlp.experts_per_token, dim=-1, sorted=True).indices)
                    x = block.mlp(x)
                # aten.stack is not a supported operator; cat of unsqueezed rows is.
                return self.model.unembedding(self.model.norm(x)), torch.cat([r.unsqueeze(0) for r in routes])

        return Probe().eval()


def c4_tokens():  # type: ignore[no-untyped-def]
    import torch

    return torch.from_numpy(__import__("numpy").random.default_rng(11).integers(0, 201088, 16))


def _programs() -> dict[str, Callable[[], object]]:
    """name -> thunk returning an ExportedProgram (built lazily; the reference must be importable)."""

    def dev_model():  # type: ignore[no-untyped-def]
        from scripts.export import make_dev_model

        return make_dev_model(0)

    def export(module, *inputs):  # type: ignore[no-untyped-def]
        import torch

        with torch.no_grad():
            return torch.export.export(module.eval(), inputs)

    def cached(model, context: int, steps: int):  # type: ignore[no-untyped-def]
        from chroma.models.cached import export_cached

        return export_cached(model, context, steps)

    import_torch = lambda: __import__("torch")  # noqa: E731

    programs: dict[str, Callable[[], object]] = {
        # C1: dev 8-token fp32 forward (scripts/export.py:72-76 traces arange(8)).
        "c1_fwd8": lambda: export(dev_model(), import_torch().arange(8)),
        # C1 with the per-layer routing as a second output.
        "c1_route8": lambda: export(RoutingProbe.build(dev_model()), import_torch().arange(8)),
        # C2: KV-cached decode pair, 256-token cache, 8-token prefill chunk and 1-token decode step.
        "c2_prefill8": lambda: cached(dev_model(), 256, 8),
        "c2_decode": lambda: cached(dev_model(), 256, 1),
        # C3: the micrograph at a fixture size and at the full benchmark size.
        "c3_micro_16": lambda: export(micro_module(16, 4096), *micro_inputs(16, 4096)),
        "c3_micro_full": lambda: export(micro_module(16384, 4096), *micro_inputs(16384, 4096)),
    }
    for dtype_name in ("float32", "bfloat16"):
        def small(dtype_name=dtype_name):  # type: ignore[no-untyped-def]
            return cuda_small_model(getattr(import_torch(), dtype_name))

        programs[f"small_{dtype_name}_full4"] = lambda small=small: export(small(), import_torch().arange(4) * 3 % 17)
        programs[f"small_{dtype_name}_prefill5"] = lambda small=small: cached(small(), 5, 5)
        programs[f"small_{dtype_name}_decode"] = lambda small=small: cached(small(), 5, 1)
    def c4_slice():  # type: ignore[no-untyped-def]
        return random_transformer(small_config("c4_slice"), seed=11, std=0.02, dtype=import_torch().bfloat16)

    programs["c4_slice_fwd16"] = lambda: export(c4_slice(), c4_tokens())
    programs["c4_slice_route16"] = lambda: export(RoutingProbe.build(c4_slice()), c4_tokens())
    for head_dim in (8, 64):
        def decoder_small(head_dim=head_dim):  # type: ignore[no-untyped-def]
            return random_transformer(small_config(f"decoder_small_{head_dim}"), seed=5, std=0.03)

        programs[f"dec{head_dim}_prefill7"] = lambda m=decoder_small: cached(m(), 7, 7)
        programs[f"dec{head_dim}_decode"] = lambda m=decoder_small: cached(m(), 7, 1)
    return programs


def build(name: str, *, force: bool = False) -> Path:
    """Compile reference program ``name`` into oracle/_ref/<name>/ unless it is already there."""
    target = ROOT / name
    if (target / "model.json").exists() and not force:
        return target
    chroma = _reference()
    thunk = _programs()[name]
    start = time.time()
    exported = thunk()
    program = chroma.compile(exported, target, backend="cpu", blas=False)
    program.close()
    (target / "build.json").write_text(json.dumps({"name": name, "seconds": time.time() - start}) + "\n")
    print(f"built {name} in {time.time() - start:.1f}s -> {target}", flush=True)
    dedupe()
    return target


def dedupe() -> None:
    """Keep one copy of identical weight files (the prefill/decode pair of one model share theirs).

    The reference names weight files by content hash (chroma/_src/build.py:61), so equal names mean equal bytes.
    A program whose file is a duplicate gets a relative symbolic link to the first copy in its place, so the
    reference's own ``Program`` (which reads ``weights`` from the artefact directory) loads it unchanged.
    """
    seen: dict[str, Path] = {}
    for directory in sorted(p for p in ROOT.iterdir() if (p / "model.json").exists()):
        weights = json.loads((directory / "model.json").read_text())["weights"]
        file = directory / weights
        if weights in seen:
            if file.is_symlink() and file.exists():
                continue
            if file.exists() or file.is_symlink():
                file.unlink()
            file.symlink_to(Path("..") / seen[weights].name / weights)
            (directory / "shared_weights.json").unlink(missing_ok=True)
        elif file.exists() and not file.is_symlink():
            seen[weights] = directory


def stage_package() -> Path:
    """A patched copy of the reference's Python package (``chroma``) under oracle/_ref/pkg, for machines without the
    reference sources (the GPU hosts): the same mechanical Python 3.12 patches ``oracle/refimport.py`` applies in
    memory, written out once. Only the ``.py`` modules are staged (enough for ``chroma.Program`` and
    ``chroma.Decoder``; compiling needs the source tree). Test infrastructure, never committed."""
    from oracle import refimport

    source = refimport.REFERENCE / "chroma"
    target = refimport.STAGED / "chroma"
    for path in sorted(source.rglob("*.py")):
        out = target / path.relative_to(source)
        out.parent.mkdir(parents=True, exist_ok=True)
        text = refimport._patch(path.read_text())
        if not out.exists() or out.read_text() != text:
            out.write_text(text)
    return refimport.STAGED


def names() -> list[str]:
    return list(_programs())


def main(argv: list[str]) -> None:
    wanted = argv or names()
    for name in wanted:
        build(name)


if __name__ == "__main__":
    main(sys.argv[1:])
