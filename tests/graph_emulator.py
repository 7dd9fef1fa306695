"""Test infrastructure: a NumPy interpreter of a generic-graph plan (chroma_b200/_src/graph.py), step for step what
csrc/graph.cu computes, for checking the lowering on machines without a GPU.

Arithmetic is fp32 with round-to-nearest after every operation (NumPy float32 scalars), bf16 rounding through
ml_dtypes; exp/sin/cos/pow use NumPy's float32 functions (the device uses CUDA's, so those differ in the last ulps).
Small graphs only: one Python loop iteration per element.
"""

from __future__ import annotations

import struct

import numpy as np
from ml_dtypes import bfloat16

F32, BF16, I64 = 0, 1, 2
_NP = {F32: np.float32, BF16: bfloat16, I64: np.int64}
_ES = {F32: 4, BF16: 2, I64: 8}
OPNAMES = ["load", "const", "add", "sub", "mul", "div", "neg", "abs", "exp", "sin", "cos", "recip", "rsqrt", "sigmoid",
           "square", "pow", "maxc", "minc", "round"]


def _f(bits: int) -> float:
    return struct.unpack("<f", struct.pack("<I", bits & 0xFFFFFFFF))[0]


class Emulator:
    def __init__(self, words: list[int], weights: bytes) -> None:
        it = iter(int(w) for w in words)
        assert next(it) == 0x31474243
        weight_bytes, arena_bytes, n_in, n_out = next(it), next(it), next(it), next(it)
        self.in_bytes = [next(it) for _ in range(n_in)]
        self.out_bytes = [next(it) for _ in range(n_out)]
        self.weights = bytearray(weights[:weight_bytes])
        self.arena = bytearray(arena_bytes)
        self.views = []
        for _ in range(next(it)):
            kind, index, _span, dtype, rank, offset = (next(it) for _ in range(6))
            shape, stride = [], []
            for _ in range(8):
                shape.append(next(it))
                stride.append(next(it))
            self.views.append((kind, index, dtype, rank, offset, shape[:rank], stride[:rank]))
        self.ops = []
        for _ in range(next(it)):
            a, imm = next(it), next(it)
            self.ops.append((a & 0xFF, (a >> 8) & 0xFF, (a >> 16) & 0xFF, (a >> 24) & 0xFF, np.float32(_f(imm))))
        self.steps = []
        for _ in range(next(it)):
            st = {"kind": next(it), "rank": next(it), "n": next(it)}
            st["oshape"] = [next(it) for _ in range(8)][: st["rank"]]
            for k in ("out", "out2", "in", "in2", "bias", "first_operand", "n_operands", "first_op", "n_ops"):
                st[k] = next(it)
            rrank = next(it)
            rs = [(next(it), next(it), next(it)) for _ in range(8)][:rrank]
            st["rshape"], st["ra"], st["rb"] = [r[0] for r in rs], [r[1] for r in rs], [r[2] for r in rs]
            for k in ("axis", "width", "k", "largest", "tri", "diag", "negative"):
                st[k] = next(it)
            st["divisor"] = np.float32(_f(next(it)))
            self.steps.append(st)
        assert next(it, None) is None

    # -- memory ------------------------------------------------------------------------------------------------------
    def _buf(self, kind: int, index: int) -> tuple[bytearray, int]:
        if kind == 0:
            return self.inputs[index], 0
        if kind == 1:
            return self.outputs[index], 0
        return (self.arena, index) if kind == 2 else (self.weights, index)

    def _addr(self, v: int, coords: list[int], extra: int = 0) -> tuple[bytearray, int, int]:
        kind, index, dtype, _rank, offset, _shape, stride = self.views[v]
        buf, base = self._buf(kind, index)
        e = offset + sum(c * s for c, s in zip(coords, stride)) + extra
        return buf, base + e * _ES[dtype], dtype

    def load(self, v: int, coords: list[int], extra: int = 0):  # type: ignore[no-untyped-def]
        buf, at, dtype = self._addr(v, coords, extra)
        value = np.frombuffer(bytes(buf[at : at + _ES[dtype]]), dtype=_NP[dtype])[0]
        return value if dtype == I64 else np.float32(value)

    def store(self, v: int, coords: list[int], value, extra: int = 0) -> None:  # type: ignore[no-untyped-def]
        buf, at, dtype = self._addr(v, coords, extra)
        buf[at : at + _ES[dtype]] = np.array([value]).astype(_NP[dtype]).tobytes()

    # -- execution ---------------------------------------------------------------------------------------------------
    def run(self, inputs: list[np.ndarray], outputs: list[np.ndarray]) -> None:
        self.inputs = [bytearray(np.ascontiguousarray(a).tobytes()) for a in inputs]
        self.outputs = [bytearray(n) for n in self.out_bytes]
        self.error = False
        for st in self.steps:
            getattr(self, f"_step{st['kind']}")(st)
        for buf, out in zip(self.outputs, outputs):
            out.reshape(-1).view(np.uint8)[:] = np.frombuffer(bytes(buf), dtype=np.uint8)
        if self.error:
            raise IndexError("Tensor idx out of range")

    @staticmethod
    def _coords(shape: list[int]):  # type: ignore[no-untyped-def]
        return [list(c) for c in np.ndindex(*shape)] if shape else [[]]

    def _step1(self, st: dict) -> None:  # elementwise
        f32 = np.float32
        with np.errstate(all="ignore"):
            for c in self._coords(st["oshape"]):
                r = [f32(0)] * 32
                last = 0
                for op, dst, a, b, imm in self.ops[st["first_op"] : st["first_op"] + st["n_ops"]]:
                    name = OPNAMES[op - 1]
                    x, y = r[a], r[b]
                    if name == "load":
                        v = self.load(st["first_operand"] + a, c)
                    elif name == "const":
                        v = imm
                    elif name in ("add", "sub", "mul", "div"):
                        v = {"add": x + y, "sub": x - y, "mul": x * y, "div": x / y}[name]
                    elif name == "neg":
                        v = -x
                    elif name == "abs":
                        v = abs(x)
                    elif name == "exp":
                        v = np.exp(x)
                    elif name == "sin":
                        v = np.sin(x)
                    elif name == "cos":
                        v = np.cos(x)
                    elif name == "recip":
                        v = f32(1) / x
                    elif name == "rsqrt":
                        v = f32(1) / np.sqrt(x)
                    elif name == "sigmoid":
                        v = f32(1) / (f32(1) + np.exp(-x))
                    elif name == "square":
                        v = x * x
                    elif name == "pow":
                        v = np.power(x, y)
                    elif name == "maxc":
                        v = imm if x < imm else x
                    elif name == "minc":
                        v = imm if imm < x else x
                    else:
                        v = f32(bfloat16(x))
                    r[dst] = f32(v)
                    last = dst
                self.store(st["out"], c, r[last])

    def _step2(self, st: dict) -> None:  # move / triangle
        for c in self._coords(st["oshape"]):
            keep = True
            if st["tri"]:
                diag = c[-1] - c[-2]
                keep = diag >= st["diag"] if st["tri"] == 1 else diag <= st["diag"]
            v = self.load(st["in"], c)
            self.store(st["out"], c, v if keep else type(v)(0))

    def _reduced(self, st: dict):  # type: ignore[no-untyped-def]
        return self._coords(st["rshape"])

    def _step3(self, st: dict) -> None:  # reduce
        for c in self._coords(st["oshape"]):
            s = np.float32(0)
            for rc in self._reduced(st):
                s = np.float32(s + self.load(st["in"], c, sum(i * t for i, t in zip(rc, st["ra"]))))
            self.store(st["out"], c, np.float32(s / st["divisor"]))

    def _step4(self, st: dict) -> None:  # contract
        for c in self._coords(st["oshape"]):
            s = np.float32(0)
            for rc in self._reduced(st):
                a = self.load(st["in"], c, sum(i * t for i, t in zip(rc, st["ra"])))
                b = self.load(st["in2"], c, sum(i * t for i, t in zip(rc, st["rb"])))
                s = np.float32(s + np.float32(a * b))
            if st["bias"] >= 0:
                s = np.float32(s + self.load(st["bias"], c))
            self.store(st["out"], c, s)

    def _axis_stride(self, v: int, axis: int) -> int:
        return self.views[v][6][axis]

    def _step5(self, st: dict) -> None:  # softmax
        si, so = self._axis_stride(st["in"], st["axis"]), self._axis_stride(st["out"], st["axis"])
        with np.errstate(all="ignore"):
            for c in self._coords(st["oshape"]):
                xs = [self.load(st["in"], c, k * si) for k in range(st["width"])]
                m = np.float32(-np.inf)
                for v in xs:
                    m = v if m < v else m
                total = np.float32(0)
                for v in xs:
                    total = np.float32(total + np.exp(np.float32(v - m)))
                for k, v in enumerate(xs):
                    self.store(st["out"], c, np.float32(np.exp(np.float32(v - m)) / total), k * so)

    def _step6(self, st: dict) -> None:  # top-k
        si = self._axis_stride(st["in"], st["axis"])
        sv, sx = self._axis_stride(st["out"], st["axis"]), self._axis_stride(st["out2"], st["axis"])
        for c in self._coords(st["oshape"]):
            xs = [self.load(st["in"], c, k * si) for k in range(st["width"])]

            def key(q: int):  # type: ignore[no-untyped-def]
                v = xs[q]
                if st["largest"]:
                    return (0 if np.isnan(v) else 1, 0.0 if np.isnan(v) else -float(v), q)
                return (1 if np.isnan(v) else 0, 0.0 if np.isnan(v) else float(v), q)

            for j, q in enumerate(sorted(range(st["width"]), key=key)[: st["k"]]):
                self.store(st["out"], c, xs[q], j * sv)
                self.store(st["out2"], c, np.int64(q), j * sx)

    def _step7(self, st: dict) -> None:  # gather
        ir = self.views[st["in2"]][3]
        rows = self.views[st["in"]][5][0]
        for c in self._coords(st["oshape"]):
            row = int(self.load(st["in2"], c[:ir]))
            if st["negative"] and row < 0:
                row += rows
            if row < 0 or row >= rows:
                self.error = True
                self.store(st["out"], c, 0)
                continue
            self.store(st["out"], c, self.load(st["in"], [row] + c[ir:]))
