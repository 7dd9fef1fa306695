"""KV-cached generation over a prefill/decode program pair.

``Decoder`` keeps the reference's API and semantics (chroma/_src/decoder.py:44-152): ``append(tokens)`` consumes
new token ids and returns the ``[1, vocab]`` logits after the last one; a single token runs the decode program,
anything longer runs prefill in chunks; the cache is a ring of ``context`` rows whose positions keep advancing;
an ``append`` that fails or is interrupted leaves the committed state unchanged; ``reset()``/``close()``.

The cache lives in device memory inside a native ``chroma_b200_decoder``; masks are built on the device from
ring-slot positions; a step uploads only token ids and positions. New K/V rows are staged on the device and
written into the ring lazily: the committed ``CacheState`` records which staged rows are pending, and the next call
applies them first. The only commit point is the swap of ``self._state``, as in the reference (decoder.py:72-76).
Both programs must be chroma_b200 programs; the reference's own ``chroma.Decoder`` drives any other ``Program``
(and a chroma_b200 artefact too, through its seven-input protocol, decoder.py:96-139).

``BatchDecoder`` runs ``batch`` independent sequences through the same device path in one launch per step and can
return greedy argmax ids instead of logits (the ids are computed on the device).
"""

from __future__ import annotations

import ctypes

import threading
from collections.abc import Sequence
from dataclasses import dataclass
from types import TracebackType
from typing import Any

import numpy as np

from chroma_b200._src import native as nat


@dataclass(frozen=True)
class CacheState:
    keys: Any
    values: Any
    slots: np.ndarray  # absolute position held by each cache row, or -1
    position: int
    staged: tuple[int, int, int] | None = None  # (program index, count, first position) awaiting commit


def validate(prefill: Any, decode: Any) -> tuple[dict[str, Any], dict[str, Any]]:
    """The pairing checks of chroma/_src/decoder.py:27-41."""
    for name, model in (("prefill", prefill), ("decode", decode)):
        if len(model.inputs) != 7 or len(model.outputs) != 3:
            raise ValueError(f"Decoder {name} wants seven inputs and three outputs, not {len(model.inputs)} and {len(model.outputs)}")
    cache, logits = decode.inputs[2], decode.outputs[0]
    steps = prefill.inputs[0]["shape"][0]
    if (
        decode.inputs[0]["shape"] != [1]
        or prefill.inputs[2]["shape"] != cache["shape"]
        or prefill.outputs[0]["shape"] != logits["shape"]
        or not 1 <= steps <= cache["shape"][1]
    ):
        raise ValueError("Decoder prefill and decode were not exported as a pair")
    return cache, logits


class _DeviceCache:
    """Lazy host view of a native decoder's cache (read on first access)."""

    def __init__(self, decoder: "NativeDecoder", index: int) -> None:
        self._decoder, self._index = decoder, index

    def array(self) -> np.ndarray:
        return self._decoder.read()[self._index]

    @property
    def dtype(self) -> np.dtype:
        return self._decoder.cache_dtype

    @property
    def nbytes(self) -> int:
        return self._decoder.cache_bytes

    @property
    def shape(self) -> tuple[int, ...]:
        return self._decoder.cache_shape

    def __array__(self, dtype: Any = None, copy: Any = None) -> np.ndarray:
        a = self.array()
        return a.astype(dtype) if dtype is not None else a


class NativeDecoder:
    """Owns a ``chroma_b200_decoder`` (batch >= 1)."""

    def __init__(self, prefill: Any, decode: Any, sliding_window: int, batch: int) -> None:
        handle = nat._VP()
        nat.call("chroma_b200_decoder_create", prefill.handle, decode.handle, int(sliding_window), int(batch),
                 nat.ctypes.byref(handle))
        self.handle = handle
        self.batch = batch
        cache = decode.inputs[2]
        self.cache_shape = (batch, *cache["shape"]) if batch > 1 else tuple(cache["shape"])
        self.cache_dtype = nat.dtype_of(cache["dtype"])
        self.cache_bytes = int(np.prod(self.cache_shape)) * self.cache_dtype.itemsize
        self.context = cache["shape"][1]
        self.steps = (prefill.inputs[0]["shape"][0], 1)
        self.logit_dtype = nat.dtype_of(decode.outputs[0]["dtype"])
        self.vocab = decode.outputs[0]["shape"][1]
        self.pinned = nat.PinnedPool()  # returned logits live in page-locked memory
        # Argument buffers and entry points of the per-token calls, made once (ndarray.ctypes conversions and
        # symbol lookups cost more than a decode step's host work otherwise).
        self._tok = (nat.ctypes.c_int64 * (batch * max(self.steps)))()
        self._pos = (nat.ctypes.c_int64 * batch)()
        self._err = nat.ctypes.create_string_buffer(1024)
        lib = nat.lib()
        self._step_fn = lib.chroma_b200_decoder_step
        self._commit_fn = lib.chroma_b200_decoder_commit

    def step(self, which: int, tokens: np.ndarray, count: int, positions: np.ndarray,
             logits: np.ndarray | None, argmax: np.ndarray | None) -> None:
        tokens = np.ascontiguousarray(tokens, dtype=np.int64)
        positions = np.ascontiguousarray(positions, dtype=np.int64)
        i64 = nat.ctypes.POINTER(nat.ctypes.c_int64)
        nat.call(
            "chroma_b200_decoder_step", self.handle, int(which), tokens.ctypes.data_as(i64), int(count),
            positions.ctypes.data_as(i64), nat._VP(logits.ctypes.data if logits is not None else None),
            argmax.ctypes.data_as(i64) if argmax is not None else None,
        )

    def _check(self, status: int) -> None:
        if status != nat.OK:
            raise nat._ERRORS.get(status, RuntimeError)(self._err.value.decode(errors="replace") or "decoder step")

    def step_one(self, which: int, ids: np.ndarray, position: int, logits_ptr: int) -> None:
        """Batch-1 step of `ids` (at most the program's rows) from `position`, logits to `logits_ptr`."""
        steps = self.steps[which]
        count = len(ids)
        for i in range(steps):
            self._tok[i] = int(ids[i]) if i < count else 0
        self._pos[0] = position
        self._check(self._step_fn(self.handle, which, self._tok, count, self._pos, nat._VP(logits_ptr), None,
                                  self._err, len(self._err)))

    def commit_one(self, which: int, count: int, first: int) -> None:
        self._pos[0] = first
        self._check(self._commit_fn(self.handle, which, count, self._pos, self._err, len(self._err)))

    def advance(self, tokens: np.ndarray | None, positions: np.ndarray | None, steps: int, stream: int = 0,
                ids: np.ndarray | None = None) -> None:
        i64 = nat.ctypes.POINTER(nat.ctypes.c_int64)
        t = np.ascontiguousarray(tokens, np.int64) if tokens is not None else None
        p = np.ascontiguousarray(positions, np.int64) if positions is not None else None
        nat.call("chroma_b200_decoder_advance", self.handle, t.ctypes.data_as(i64) if t is not None else None,
                 p.ctypes.data_as(i64) if p is not None else None, int(steps), nat._VP(stream),
                 ids.ctypes.data_as(i64) if ids is not None else None)

    def launch_vocab(self, stream: int = 0) -> None:
        nat.call("chroma_b200_decoder_launch_vocab", self.handle, nat._VP(stream))

    def launch_layers(self, stream: int = 0) -> None:
        nat.call("chroma_b200_decoder_launch_layers", self.handle, nat._VP(stream))

    @property
    def step_launches(self) -> int:
        return int(nat.lib().chroma_b200_decoder_step_launches(self.handle))

    def commit(self, which: int, count: int, positions: np.ndarray) -> None:
        positions = np.ascontiguousarray(positions, dtype=np.int64)
        nat.call("chroma_b200_decoder_commit", self.handle, int(which), int(count),
                 positions.ctypes.data_as(nat.ctypes.POINTER(nat.ctypes.c_int64)))

    def reset(self) -> None:
        nat.call("chroma_b200_decoder_reset", self.handle)

    def read(self) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        keys = np.empty(self.cache_shape, self.cache_dtype)
        values = np.empty(self.cache_shape, self.cache_dtype)
        slots = np.empty((self.batch, self.context), np.int64)
        nat.call("chroma_b200_decoder_read", self.handle, nat._VP(keys.ctypes.data), nat._VP(values.ctypes.data),
                 slots.ctypes.data_as(nat.ctypes.POINTER(nat.ctypes.c_int64)))
        return keys, values, slots

    def close(self) -> None:
        handle, self.handle = getattr(self, "handle", None), None
        if handle:
            nat.lib().chroma_b200_decoder_destroy(handle)
        pinned = getattr(self, "pinned", None)
        if pinned is not None:
            pinned.close()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass


def _natives(prefill: Any, decode: Any) -> tuple[Any, Any] | None:
    a, b = getattr(prefill, "native", None), getattr(decode, "native", None)
    if isinstance(a, nat.Native) and isinstance(b, nat.Native):
        return a, b
    return None


class Decoder:
    def __init__(self, prefill: Any, decode: Any, *, sliding_window: int = 0) -> None:
        if sliding_window < 0:
            raise ValueError(f"sliding_window must be nonnegative, got {sliding_window}")
        cache, logits = validate(prefill, decode)
        self._models = (prefill, decode)
        self._shape = tuple(cache["shape"])
        self._cache_dtype = nat.dtype_of(cache["dtype"])
        self._logit_dtype = nat.dtype_of(logits["dtype"])
        self.context = self._shape[1]
        self.vocab_size = logits["shape"][1]
        self.device = decode.device
        self._window = min(sliding_window or self.context, self.context)
        self._lock = threading.Lock()
        self._closed = False
        natives = _natives(prefill, decode)
        if natives is None:
            # The cache lives in device memory next to the programs; programs of another backend are driven by the
            # reference's own host-side Decoder (chroma.Decoder), which takes any Program.
            raise TypeError("chroma_b200.Decoder drives chroma_b200 programs; use chroma.Decoder for other Programs")
        self._native: NativeDecoder | None = NativeDecoder(*natives, sliding_window, 1)
        self._commit(self._empty())

    # -- state ---------------------------------------------------------------------------------------------
    def _empty(self) -> CacheState:
        assert self._native is not None
        slots = np.full(self.context, -1, dtype=np.int64)
        return CacheState(_DeviceCache(self._native, 0), _DeviceCache(self._native, 1), slots, 0)

    def _commit(self, state: CacheState) -> None:
        # Swapping in a whole new state is the single commit point, so an interrupt cannot half-apply a step.
        self._state = state

    def _flush(self) -> CacheState:
        """Apply rows a previous successful step staged on the device (idempotent)."""
        state = self._state
        if state.staged is not None and self._native is not None:
            which, count, first = state.staged
            self._native.commit_one(which, count, first)
            state = CacheState(state.keys, state.values, state.slots, state.position)
            self._commit(state)
        return state

    @property
    def position(self) -> int:
        return self._state.position

    @property
    def stats(self) -> dict[str, Any]:
        return {
            "cache_bytes": self._state.keys.nbytes + self._state.values.nbytes,
            "prefill": self._models[0].stats,
            "decode": self._models[1].stats,
        }

    def reset(self) -> None:
        with self._lock:
            if self._closed:
                raise RuntimeError("Decoder is closed")
            if self._native is not None:
                self._native.reset()
            self._commit(self._empty())

    def cache(self) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        """Committed (keys, values, slots) as host arrays."""
        with self._lock:
            self._flush()
            if self._native is None:
                raise RuntimeError("Decoder is closed")
            keys, values, slots = self._native.read()
            return keys, values, slots[0]

    # -- stepping ------------------------------------------------------------------------------------------
    def append(self, tokens: Sequence[int] | np.ndarray) -> np.ndarray:
        """Consume new token IDs and return the logits after the last one."""
        ids = np.asarray(tokens)
        if ids.ndim != 1 or not len(ids):
            raise ValueError(f"append wants a nonempty 1-D sequence of token IDs, got shape {ids.shape}")
        if not np.issubdtype(ids.dtype, np.integer):
            raise TypeError(f"Token IDs must be integers, got {ids.dtype}")
        ids = ids.astype(np.int64)
        with self._lock:
            if self._closed or self._native is None:
                raise RuntimeError("Decoder is closed")
            return self._append_device(ids)

    def _append_device(self, ids: np.ndarray) -> np.ndarray:
        assert self._native is not None
        offset = 0
        logits = np.empty((1, self.vocab_size), dtype=self._logit_dtype)
        while offset < len(ids):
            remaining = len(ids) - offset
            index = 1 if remaining == 1 else 0
            steps = self._native.steps[index]
            count = min(steps, remaining)
            state = self._flush()
            logits, ptr = self._native.pinned.array_ptr((1, self.vocab_size), self._logit_dtype)
            pos = state.position
            self._native.step_one(index, ids[offset : offset + count], pos, ptr)
            slots = state.slots.copy()
            if count == 1:
                slots[pos % self.context] = pos
            else:
                slots[(pos + np.arange(count)) % self.context] = pos + np.arange(count)
            self._commit(CacheState(state.keys, state.values, slots, pos + count, (index, count, pos)))
            offset += count
        return logits

    def close(self) -> None:
        with self._lock:
            if self._native is not None:
                self._native.close()
            for model in self._models:
                model.close()
            self._closed = True

    def __enter__(self) -> "Decoder":
        return self

    def __exit__(self, exc_type: type[BaseException] | None, exc: BaseException | None, tb: TracebackType | None) -> None:
        self.close()


class BatchDecoder:
    """``batch`` independent sequences decoded in lockstep on the device (no reference counterpart: the reference
    Decoder is batch-1 and host-resident). Each ``append`` takes ``[batch, m]`` token ids (the same ``m`` for every
    sequence) and returns ``[batch, vocab]`` logits, or greedy ``[batch]`` argmax ids with ``argmax=True``."""

    def __init__(self, prefill: Any, decode: Any, batch: int, *, sliding_window: int = 0) -> None:
        if sliding_window < 0:
            raise ValueError(f"sliding_window must be nonnegative, got {sliding_window}")
        validate(prefill, decode)
        natives = _natives(prefill, decode)
        if natives is None:
            raise TypeError("BatchDecoder needs two chroma_b200 CUDA programs")
        self._models = (prefill, decode)
        self._native = NativeDecoder(*natives, sliding_window, batch)
        self.batch = batch
        self.context = self._native.context
        self.vocab_size = self._native.vocab
        self._lock = threading.Lock()
        self._position = np.zeros(batch, np.int64)
        self._staged: tuple[int, int, np.ndarray] | None = None

    @property
    def positions(self) -> np.ndarray:
        return self._position.copy()

    def reset(self) -> None:
        with self._lock:
            self._native.reset()
            self._position = np.zeros(self.batch, np.int64)
            self._staged = None

    def _flush(self) -> None:
        if self._staged is not None:
            which, count, first = self._staged
            self._native.commit(which, count, first)
            self._staged = None

    def append(self, tokens: np.ndarray, *, argmax: bool = False) -> np.ndarray:
        ids = np.asarray(tokens)
        if ids.ndim != 2 or ids.shape[0] != self.batch or not ids.shape[1]:
            raise ValueError(f"append wants [batch={self.batch}, m] token IDs, got shape {ids.shape}")
        if not np.issubdtype(ids.dtype, np.integer):
            raise TypeError(f"Token IDs must be integers, got {ids.dtype}")
        ids = ids.astype(np.int64)
        with self._lock:
            out: np.ndarray
            offset = 0
            while offset < ids.shape[1]:
                remaining = ids.shape[1] - offset
                index = 1 if remaining == 1 else 0
                steps = self._native.steps[index]
                count = min(steps, remaining)
                self._flush()
                chunk = np.zeros((self.batch, steps), dtype=np.int64)
                chunk[:, :count] = ids[:, offset : offset + count]
                first = self._position.copy()
                if argmax:
                    out = np.empty(self.batch, np.int64)
                    self._native.step(index, chunk, count, first, None, out)
                else:
                    out = self._native.pinned.array((self.batch, self.vocab_size), self._native.logit_dtype)
                    self._native.step(index, chunk, count, first, out, None)
                self._staged = (index, count, first)
                self._position = first + count
                offset += count
            return out

    def generate(self, tokens: np.ndarray, steps: int) -> np.ndarray:
        """Greedy decoding on the device: consume ``tokens`` [batch] (one per sequence), then feed each argmax back,
        ``steps`` times. Returns the generated ids [batch, steps]; ids[:, 0] follows ``tokens``."""
        tokens = np.asarray(tokens, np.int64).reshape(self.batch)
        with self._lock:
            self._flush()
            ids = np.empty((steps, self.batch), np.int64)
            self._native.advance(tokens, self._position, steps, 0, ids)
            self._position = self._position + steps
            return ids.T.copy()

    def load_cache(self, first: int, keys: Any, values: Any, positions: np.ndarray) -> None:
        """Install committed caches for sequences [first, first + len(positions)): ``keys``/``values`` shaped
        [count, layers, context, kv_heads, head_dim] in the cache dtype, as NumPy arrays or CUDA tensors (anything
        with ``data_ptr()``); ``positions`` [count] = tokens already in each sequence. The ring then holds each
        sequence's last ``context`` positions (slot = position % context), and its next token is at ``positions``."""
        pos = np.asarray(positions, np.int64).reshape(-1)
        count = len(pos)
        slots = np.full((count, self.context), -1, np.int64)
        for i, p in enumerate(pos):
            held = np.arange(max(0, int(p) - self.context), int(p), dtype=np.int64)
            slots[i, held % self.context] = held

        def ptr(a: Any) -> int:
            if hasattr(a, "data_ptr"):
                return int(a.data_ptr())
            a = np.ascontiguousarray(a)
            return int(a.ctypes.data)

        with self._lock:
            self._flush()
            nat.call("chroma_b200_decoder_write", self._native.handle, int(first), count, nat._VP(ptr(keys)),
                     nat._VP(ptr(values)), slots.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)))
            self._position[first : first + count] = pos

    def advance_device(self, steps: int, stream: int) -> None:
        """Continue greedy decoding from the device state left by ``generate`` without any host transfer; queued on
        ``stream`` (a cudaStream_t) and not synchronised. For benchmarks."""
        with self._lock:
            self._native.advance(None, None, steps, stream, None)
            self._position = self._position + steps

    def close(self) -> None:
        with self._lock:
            self._native.close()

    def __enter__(self) -> "BatchDecoder":
        return self

    def __exit__(self, exc_type: type[BaseException] | None, exc: BaseException | None, tb: TracebackType | None) -> None:
        self.close()
