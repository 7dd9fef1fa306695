"""The fast sigmoid of bf16 inputs (csrc/common.cuh: __expf and rcp.approx, used by the C3 micrograph and the
tcgen05 GEMM's SwiGLU epilogue) against bf16(1 / (1 + expf(-z))) with the IEEE division, for every one of the
65,536 bf16 values: the kernels that use it rely on the two being identical after rounding to bf16."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def test_fast_sigmoid_matches_ieee_form_for_every_bf16_input(gpu: None, tmp_path: Path) -> None:
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).exists():
        pytest.skip("nvcc is not available")
    exe = tmp_path / "sigmoid_check"
    subprocess.run([nvcc, "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
                    "-I", str(ROOT / "chroma_b200" / "csrc"), str(ROOT / "tests" / "sigmoid_check.cu"), "-o", str(exe)],
                   check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()
    assert out[0] == "0", f"{out[0]} bf16 inputs differ: {out[1:]}"
