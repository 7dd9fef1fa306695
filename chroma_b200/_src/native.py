"""ctypes binding of ``libchroma_b200.so`` (the C ABI declared in ``include/chroma_b200.h``).

Loading needs only NumPy: no Torch, no pybind11. ``Model`` implements the reference's native object protocol
(``Model(weights_path)`` with ``.device`` and ``.run(inputs, outputs)``, chroma/_src/program.py:66-70 and
chroma/_src/core/bindings.h:35-75), including its argument validation and error types:

* wrong array count, dtype/shape mismatch, non-contiguous, misaligned or read-only outputs, overlapping outputs
  -> ``ValueError``; a non-array -> ``TypeError`` (bindings.h:17-33, :58-62);
* an out-of-range index found on the device -> ``IndexError`` (runtime.h:160-162);
* a CUDA failure -> ``RuntimeError``.

ctypes releases the GIL for the duration of each native call, as ``py::gil_scoped_release`` does (bindings.h:66).
There is no CPU fallback: if the library is missing or no sm_100 GPU is present, construction fails loudly.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path
from typing import Any

import numpy as np

_LIB_NAME = "libchroma_b200.so"
_PACKAGE = Path(__file__).resolve().parents[1]

OK, INDEX, VALUE, RUNTIME = 0, 1, 2, 3
GPTOSS_FORWARD, GPTOSS_CACHED, MICRO, GPTOSS_LAST = 1, 2, 3, 4
FP32, BF16 = 0, 1


class Desc(ctypes.Structure):
    _fields_ = [
        ("kind", ctypes.c_int32),
        ("storage", ctypes.c_int32),
        ("layers", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("experts", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
        ("intermediate", ctypes.c_int32),
        ("vocab", ctypes.c_int32),
        ("tokens", ctypes.c_int32),
        ("context", ctypes.c_int32),
        ("window", ctypes.c_int32),
        ("eps", ctypes.c_float),
        ("sm_scale", ctypes.c_float),
        ("swiglu_alpha", ctypes.c_float),
        ("swiglu_limit", ctypes.c_float),
        ("rope_concentration", ctypes.c_float),
        ("rows", ctypes.c_int64),
        ("cols", ctypes.c_int64),
        ("inv_freq", ctypes.POINTER(ctypes.c_float)),
        ("layer_window", ctypes.POINTER(ctypes.c_int32)),
        ("offsets", ctypes.POINTER(ctypes.c_int64)),
        ("num_offsets", ctypes.c_int32),
        ("weight_bytes", ctypes.c_int64),
    ]


# Every exported symbol of include/chroma_b200.h with its ctypes signature.
_VP, _CP, _SZ, _I32, _I64P = ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_int32, ctypes.POINTER(ctypes.c_int64)
SIGNATURES: dict[str, tuple[Any, list[Any]]] = {
    "chroma_b200_create": (ctypes.c_int, [ctypes.POINTER(Desc), _CP, ctypes.POINTER(_VP), _CP, _SZ]),
    "chroma_b200_create_device": (ctypes.c_int, [ctypes.POINTER(Desc), _VP, ctypes.POINTER(_VP), _CP, _SZ]),
    "chroma_b200_run": (ctypes.c_int, [_VP, ctypes.POINTER(_VP), ctypes.POINTER(_VP), _CP, _SZ]),
    "chroma_b200_buffers": (ctypes.c_int, [_VP, ctypes.POINTER(_VP), ctypes.POINTER(_VP), _CP, _SZ]),
    "chroma_b200_run_device": (ctypes.c_int, [_VP, _VP, _CP, _SZ]),
    "chroma_b200_check": (ctypes.c_int, [_VP, _VP, _CP, _SZ]),
    "chroma_b200_device": (ctypes.c_char_p, [_VP]),
    "chroma_b200_launches": (ctypes.c_int32, [_VP]),
    "chroma_b200_destroy": (None, [_VP]),
    "chroma_b200_plan_arena": (ctypes.c_int64, [_I32, _I64P, ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32), _I64P]),
    "chroma_b200_workspace_bytes": (ctypes.c_int64, [_VP]),
    "chroma_b200_routes": (ctypes.c_int, [_VP, ctypes.POINTER(ctypes.c_int32), ctypes.c_int64, _CP, _SZ]),
    "chroma_b200_vocab_argmax_static": (ctypes.c_int, [_VP, _VP, _I32, _VP, _I64P, _VP, _CP, _SZ]),
    "chroma_b200_gemm_bf16": (ctypes.c_int, [_VP, _VP, _VP, _VP, _VP, _I32, _I32, _I32, _I32, ctypes.c_float,
                                             ctypes.c_float, _I32, _VP, _VP, _VP, _VP, _CP, _SZ]),
    "chroma_b200_decoder_create": (ctypes.c_int, [_VP, _VP, _I32, _I32, ctypes.POINTER(_VP), _CP, _SZ]),
    "chroma_b200_decoder_step": (ctypes.c_int, [_VP, _I32, _I64P, _I32, _I64P, _VP, _I64P, _CP, _SZ]),
    "chroma_b200_decoder_commit": (ctypes.c_int, [_VP, _I32, _I32, _I64P, _CP, _SZ]),
    "chroma_b200_decoder_reset": (ctypes.c_int, [_VP, _CP, _SZ]),
    "chroma_b200_decoder_read": (ctypes.c_int, [_VP, _VP, _VP, _I64P, _CP, _SZ]),
    "chroma_b200_decoder_destroy": (None, [_VP]),
    "chroma_b200_decoder_advance": (ctypes.c_int, [_VP, _I64P, _I64P, _I32, _VP, _I64P, _CP, _SZ]),
    "chroma_b200_decoder_step_launches": (ctypes.c_int32, [_VP]),
    "chroma_b200_decoder_launch_vocab": (ctypes.c_int, [_VP, _VP, _CP, _SZ]),
    "chroma_b200_decoder_launch_layers": (ctypes.c_int, [_VP, _VP, _CP, _SZ]),
    "chroma_b200_decoder_write": (ctypes.c_int, [_VP, _I32, _I32, _VP, _VP, _I64P, _CP, _SZ]),
    "chroma_b200_ep_create": (ctypes.c_int, [_I32, _I32, ctypes.c_int64, _I32, _I32, _I32, _I32, ctypes.POINTER(_VP),
                                             _CP, _SZ]),
    "chroma_b200_ep_handle": (ctypes.c_int, [_VP, _VP, _CP, _SZ]),
    "chroma_b200_ep_open": (ctypes.c_int, [_VP, _VP, _CP, _SZ]),
    "chroma_b200_ep_destroy": (None, [_VP]),
    "chroma_b200_create_ep": (ctypes.c_int, [ctypes.POINTER(Desc), _CP, _VP, _VP, ctypes.POINTER(_VP), _CP, _SZ]),
    "chroma_b200_host_alloc": (ctypes.c_int, [_SZ, ctypes.POINTER(_VP), _CP, _SZ]),
    "chroma_b200_host_free": (None, [_VP]),
    "chroma_b200_graph_create": (ctypes.c_int, [_I64P, _SZ, _CP, ctypes.POINTER(_VP), _CP, _SZ]),
    "chroma_b200_graph_run": (ctypes.c_int, [_VP, ctypes.POINTER(_VP), ctypes.POINTER(_VP), _CP, _SZ]),
    "chroma_b200_graph_device": (ctypes.c_char_p, [_VP]),
    "chroma_b200_graph_launches": (ctypes.c_int32, [_VP]),
    "chroma_b200_graph_destroy": (None, [_VP]),
}

EP_HANDLE_BYTES = 64  # CHROMA_B200_EP_HANDLE_BYTES

_lib: ctypes.CDLL | None = None
_lib_lock = threading.Lock()


def library_path() -> Path:
    return Path(os.environ.get("CHROMA_B200_LIBRARY", _PACKAGE / _LIB_NAME))


def lib() -> ctypes.CDLL:
    """Load the native library once. Raises if it has not been built: there is no fallback."""
    global _lib
    with _lib_lock:
        if _lib is None:
            path = library_path()
            if not path.exists():
                raise RuntimeError(
                    f"chroma_b200 native library not found at {path}; build it with "
                    "`python -c 'import __graft_entry__ as g; g.build()'` (nvcc, sm_100a)"
                )
            handle = ctypes.CDLL(str(path))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = handle
        return _lib


_ERRORS = {INDEX: IndexError, VALUE: ValueError, RUNTIME: RuntimeError}


def call(name: str, *args: Any) -> None:
    err = ctypes.create_string_buffer(1024)
    status = getattr(lib(), name)(*args, err, len(err))
    if status != OK:
        raise _ERRORS.get(status, RuntimeError)(err.value.decode(errors="replace") or name)


# ---------------------------------------------------------------------------------------------------------
# Page-locked result arrays.


class _PinnedBlock:
    """One page-locked host block exported as a buffer (PEP 688): numpy arrays made from it keep it alive, and it
    returns to its pool when the last of them is gone."""

    def __init__(self, pool: "PinnedPool", ptr: int, nbytes: int) -> None:
        self._pool, self._ptr, self._nbytes = pool, ptr, nbytes
        self._mem = (ctypes.c_char * nbytes).from_address(ptr)

    def __buffer__(self, flags: int) -> memoryview:
        return memoryview(self._mem)

    def __del__(self) -> None:
        try:
            self._pool.give_back(self._ptr, self._nbytes)
        except Exception:  # interpreter shutdown
            pass


class PinnedPool:
    """Recycles page-locked host blocks for the arrays a decoder returns every step, so the device-to-host copy of
    a step's logits is one DMA at link speed instead of a copy through the driver's staging buffer."""

    def __init__(self, keep: int = 4) -> None:
        self._free: dict[int, list[int]] = {}
        self._keep = keep
        self._lock = threading.Lock()

    def array(self, shape: tuple[int, ...], dtype: Any) -> np.ndarray:
        return self.array_ptr(shape, dtype)[0]

    def array_ptr(self, shape: tuple[int, ...], dtype: Any) -> tuple[np.ndarray, int]:
        """A page-locked array and its address."""
        dtype = np.dtype(dtype)
        count = 1
        for n in shape:
            count *= int(n)
        nbytes = max(1, count * dtype.itemsize)
        with self._lock:
            free = self._free.get(nbytes)
            ptr = free.pop() if free else None
        if ptr is None:
            out = _VP()
            call("chroma_b200_host_alloc", _SZ(nbytes), ctypes.byref(out))
            ptr = int(out.value)
        return np.frombuffer(_PinnedBlock(self, ptr, nbytes), dtype, count=count).reshape(shape), ptr

    def give_back(self, ptr: int, nbytes: int) -> None:
        with self._lock:
            free = self._free.setdefault(nbytes, [])
            if len(free) < self._keep:
                free.append(ptr)
                return
        lib().chroma_b200_host_free(_VP(ptr))

    def close(self) -> None:
        """Frees the idle blocks; blocks still behind live arrays are freed when those arrays go."""
        with self._lock:
            idle = [p for ptrs in self._free.values() for p in ptrs]
            self._free.clear()
            self._keep = 0
        for p in idle:
            lib().chroma_b200_host_free(_VP(p))


# ---------------------------------------------------------------------------------------------------------
# Array validation with the reference binding's semantics.


def checked(value: Any, shape: list[int], dtype: np.dtype, output: bool) -> np.ndarray:
    if not isinstance(value, np.ndarray):
        raise TypeError("not a numpy array")
    if value.dtype != dtype or list(value.shape) != list(shape):
        raise ValueError("shape or dtype")
    if (not value.flags.c_contiguous) or value.ctypes.data % dtype.alignment or (output and not value.flags.writeable):
        raise ValueError("want C-contiguous, aligned, writable outputs")
    return value


def dtype_of(name: str) -> np.dtype:
    if name == "bfloat16":
        from ml_dtypes import bfloat16

        return np.dtype(bfloat16)
    return np.dtype(name)


class Native:
    """Owns one ``chroma_b200_program``."""

    def __init__(self, plan: dict[str, Any], weights_path: str | None = None, *, device_weights: int | None = None,
                 ep: Any = None) -> None:
        self.plan = plan
        self._keep: list[Any] = []
        self.pinned = PinnedPool()  # results of calls without `out` live in page-locked memory
        desc = self._desc(plan)
        handle = _VP()
        if ep is not None:
            # An expert-parallel program: weights hold this rank's experts only; the group outlives the program.
            self._keep.append(ep)
            path = str(weights_path).encode() if device_weights is None else None
            call("chroma_b200_create_ep", ctypes.byref(desc), path, _VP(device_weights) if device_weights is not None
                 else None, ep.handle, ctypes.byref(handle))
        elif device_weights is not None:
            call("chroma_b200_create_device", ctypes.byref(desc), _VP(device_weights), ctypes.byref(handle))
        else:
            call("chroma_b200_create", ctypes.byref(desc), str(weights_path).encode(), ctypes.byref(handle))
        self.handle = handle
        self.inputs = plan["inputs"]
        self.outputs = plan["outputs"]
        self.in_types = [dtype_of(s["dtype"]) for s in self.inputs]
        self.out_types = [dtype_of(s["dtype"]) for s in self.outputs]

    def _desc(self, plan: dict[str, Any]) -> Desc:
        d = Desc()
        for key, value in plan["desc"].items():
            setattr(d, key, value)
        offsets = (ctypes.c_int64 * len(plan["offsets"]))(*plan["offsets"])
        d.offsets = offsets
        d.num_offsets = len(plan["offsets"])
        inv = plan.get("inv_freq") or [0.0]
        inv_freq = (ctypes.c_float * len(inv))(*inv)
        d.inv_freq = inv_freq
        lw = plan.get("layer_window") or [0]
        layer_window = (ctypes.c_int32 * len(lw))(*lw)
        d.layer_window = layer_window
        self._keep += [offsets, inv_freq, layer_window]
        return d

    @property
    def device(self) -> str:
        return lib().chroma_b200_device(self.handle).decode()

    @property
    def launches(self) -> int:
        return int(lib().chroma_b200_launches(self.handle))

    def run(self, inputs: list[Any], outputs: list[Any]) -> None:
        if not isinstance(inputs, list) or not isinstance(outputs, list):
            raise TypeError("inputs and outputs must be lists")
        if len(inputs) != len(self.inputs) or len(outputs) != len(self.outputs):
            raise ValueError("wrong number of arrays")
        regions: list[tuple[int, int]] = []
        in_ptrs = (_VP * len(inputs))()
        out_ptrs = (_VP * len(outputs))()
        for i, (value, spec, dtype) in enumerate(zip(inputs, self.inputs, self.in_types)):
            array = checked(value, spec["shape"], dtype, False)
            begin = array.ctypes.data
            in_ptrs[i] = begin
            regions.append((begin, begin + array.nbytes))
        for i, (value, spec, dtype) in enumerate(zip(outputs, self.outputs, self.out_types)):
            array = checked(value, spec["shape"], dtype, True)
            begin = array.ctypes.data
            end = begin + array.nbytes
            if any(begin < last and first < end for first, last in regions):
                raise ValueError("output overlap")
            out_ptrs[i] = begin
            regions.append((begin, end))
        call("chroma_b200_run", self.handle, in_ptrs, out_ptrs)

    def routes(self) -> np.ndarray:
        """Selected experts of the last run, [layers, tokens, top_k] (GPT-OSS programs)."""
        d = self.plan["desc"]
        shape = (d["layers"], d["tokens"], d["top_k"])
        out = np.empty(shape, np.int32)
        call("chroma_b200_routes", self.handle, out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), out.size)
        return out.astype(np.int64)

    @property
    def workspace_bytes(self) -> int:
        return int(lib().chroma_b200_workspace_bytes(self.handle))

    def buffers(self) -> tuple[list[int], list[int]]:
        ins = (_VP * len(self.inputs))()
        outs = (_VP * len(self.outputs))()
        call("chroma_b200_buffers", self.handle, ins, outs)
        return [int(p or 0) for p in ins], [int(p or 0) for p in outs]

    def run_device(self, stream: int = 0) -> None:
        call("chroma_b200_run_device", self.handle, _VP(stream))

    def check(self, stream: int = 0) -> None:
        call("chroma_b200_check", self.handle, _VP(stream))

    def close(self) -> None:
        handle, self.handle = getattr(self, "handle", None), None
        if handle:
            lib().chroma_b200_destroy(handle)
        pinned = getattr(self, "pinned", None)
        if pinned is not None:
            pinned.close()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass


class GraphNative:
    """Owns one ``chroma_b200_graph``: a generic exported graph run from its plan (chroma_b200/_src/graph.py)."""

    def __init__(self, plan: dict[str, Any], weights_path: str | None) -> None:
        self.plan = plan
        self.pinned = PinnedPool()
        words = np.asarray(plan["graph"], dtype=np.int64)
        self._words = words
        handle = _VP()
        path = str(weights_path).encode() if plan["desc"]["weight_bytes"] else None
        call("chroma_b200_graph_create", words.ctypes.data_as(_I64P), words.size, path, ctypes.byref(handle))
        self.handle = handle
        self.inputs = plan["inputs"]
        self.outputs = plan["outputs"]
        self.in_types = [dtype_of(s["dtype"]) for s in self.inputs]
        self.out_types = [dtype_of(s["dtype"]) for s in self.outputs]

    @property
    def device(self) -> str:
        return (lib().chroma_b200_graph_device(self.handle) or b"").decode()

    @property
    def launches(self) -> int:
        return int(lib().chroma_b200_graph_launches(self.handle))

    def run(self, inputs: list[Any], outputs: list[Any]) -> None:
        if not isinstance(inputs, list) or not isinstance(outputs, list):
            raise TypeError("inputs and outputs must be lists")
        if len(inputs) != len(self.inputs) or len(outputs) != len(self.outputs):
            raise ValueError("wrong number of arrays")
        regions: list[tuple[int, int]] = []
        in_ptrs = (_VP * max(1, len(inputs)))()
        out_ptrs = (_VP * len(outputs))()
        for i, (value, spec, dtype) in enumerate(zip(inputs, self.inputs, self.in_types)):
            array = checked(value, spec["shape"], dtype, False)
            in_ptrs[i] = array.ctypes.data
            regions.append((array.ctypes.data, array.ctypes.data + array.nbytes))
        for i, (value, spec, dtype) in enumerate(zip(outputs, self.outputs, self.out_types)):
            array = checked(value, spec["shape"], dtype, True)
            begin, end = array.ctypes.data, array.ctypes.data + array.nbytes
            if any(begin < last and first < end for first, last in regions):
                raise ValueError("output overlap")
            out_ptrs[i] = begin
            regions.append((begin, end))
        call("chroma_b200_graph_run", self.handle, in_ptrs, out_ptrs)

    def close(self) -> None:
        handle, self.handle = getattr(self, "handle", None), None
        if handle:
            lib().chroma_b200_graph_destroy(handle)
        pinned = getattr(self, "pinned", None)
        if pinned is not None:
            pinned.close()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass


def model_class(plan: dict[str, Any]) -> type:
    """The ``Model`` class a compiled artefact's library module exports (native object protocol)."""

    class Model:
        def __init__(self, weights_path: str) -> None:
            if plan.get("expert_parallel"):
                raise ValueError("This artefact holds one rank's experts of an expert-parallel group; load it with "
                                 "chroma_b200.compile_model(..., experts=group) on every rank")
            self._native = GraphNative(plan, weights_path) if "graph" in plan else Native(plan, weights_path)

        @property
        def device(self) -> str:
            return self._native.device

        def run(self, inputs: list[Any], outputs: list[Any]) -> None:
            self._native.run(inputs, outputs)

        @property
        def native(self) -> Any:
            return self._native

    return Model
