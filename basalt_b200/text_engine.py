"""Python mirror of ``basalt.infer.TextEngine`` running on the CUDA engine.

Method names, argument meaning and failure behaviour follow the reference class
(src/main/java/basalt/infer/TextEngine.java): ``of``, ``vocabulary``, ``window``, ``scores``,
``scoresBatch``, ``generate``, ``stream``, ``streamSampled``, ``generateBatch``, ``sample``,
``seed``, ``save``, ``load``, ``close``. A rejected argument raises ``IllegalArgumentException``
where the reference throws one; every call crosses the C ABI of ``libbasalt_cuda.so`` once.

The reference binds an arbitrary Java ``Module``; here the module is described by a
:class:`ModelSpec` naming one of the supported architectures, and its weights are set by name
(``Module.loadStateDict``, torch/Module.java:68-76) or loaded from a TextEngine weight file.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Callable, Iterable, Optional, Sequence

import numpy as np

from . import _lib


class BasaltRuntimeException(RuntimeError):
    """Base of the reference's runtime exceptions (basalt/BasaltRuntimeException)."""

    def __init__(self, message: str, code: int = _lib.BST_PANIC):
        super().__init__(message)
        self.code = code


class IllegalArgumentException(BasaltRuntimeException, ValueError):
    pass


class IllegalStateException(BasaltRuntimeException):
    pass


class BasaltShapeException(IllegalArgumentException):
    pass


class BasaltMemoryException(BasaltRuntimeException, MemoryError):
    pass


class BasaltUnsupportedOperationException(BasaltRuntimeException):
    pass


# Status code -> exception class (native/src/error.rs:60-68; TextEngine's own IllegalState cases).
_EXCEPTIONS = {
    _lib.BST_INVALID: IllegalArgumentException,
    _lib.BST_SHAPE: BasaltShapeException,
    _lib.BST_UNKNOWN_HANDLE: IllegalStateException,
    _lib.BST_CONTEXT: IllegalStateException,
    _lib.BST_OOM: BasaltMemoryException,
    _lib.BST_UNSUPPORTED: BasaltUnsupportedOperationException,
}


def _raise(code: int, handle: int = 0):
    if code >= 0:
        return code
    message = _lib.last_error(handle if code != _lib.BST_UNKNOWN_HANDLE else 0)
    raise _EXCEPTIONS.get(code, BasaltRuntimeException)(f"{message} (code {code})", code)


FAMILIES = {
    "padded_decoder": _lib.FAMILY_PADDED_DECODER,
    "decoder": _lib.FAMILY_DECODER,
    "char_lm": _lib.FAMILY_CHAR_LM,
    "last_token": _lib.FAMILY_LAST_TOKEN,
}
DTYPES = {"f32": _lib.DTYPE_F32, "bf16": _lib.DTYPE_BF16}


@dataclass(frozen=True)
class ModelSpec:
    """The architecture a TextEngine serves.

    * ``padded_decoder`` — pre-norm causal decoder built from the reference's TransformerBlock
      (torch/TransformerBlock.java:37-43) with token and position embeddings, a final LayerNorm,
      the last-position slice and a Linear head. The id ``vocabulary`` is PAD: leading PADs are
      masked out as keys and positions count from the first real token, which makes an exact KV
      cache possible until the window fills.
    * ``decoder`` — the same blocks with the stock causal mask; positions are the window slots, so
      every step re-encodes the window, as the reference does.
    * ``char_lm`` — Zoo.charLm (zoo/Zoo.java:80-168): ``dimension`` is the embedding width and
      ``hidden`` the bottleneck.
    * ``last_token`` — TextEngineTest.LastTokenModel, the reference's decode-loop fixture.
    """

    family: str
    vocabulary: int
    window: int
    dimension: int = 0
    layers: int = 0
    heads: int = 1
    hidden: int = 0
    weight_dtype: str = "f32"
    kv_dtype: str = "f32"
    max_rows: int = 0

    def struct(self) -> _lib.ModelSpecStruct:
        if self.family not in FAMILIES:
            raise IllegalArgumentException(f"unknown model family {self.family!r}")
        s = _lib.ModelSpecStruct()
        s.family = FAMILIES[self.family]
        s.vocabulary = self.vocabulary
        s.window = self.window
        s.dimension = self.dimension
        s.layers = self.layers
        s.heads = self.heads
        s.hidden = self.hidden
        s.weight_dtype = DTYPES[self.weight_dtype]
        s.kv_dtype = DTYPES[self.kv_dtype]
        s.max_rows = self.max_rows
        return s


class Basalt:
    """The runtime a TextEngine lives in: one CUDA device (``Device.cuda(i)``, Device.java:46-51).

    Mirrors ``Basalt.create()`` for the decode path; the engine borrows it.
    """

    def __init__(self, device: int = 0):
        self.device = device

    @staticmethod
    def create(device: int = 0) -> "Basalt":
        return Basalt(device)

    @staticmethod
    def device_count() -> int:
        count = ctypes.c_int32(0)
        code = _lib.load().bst_device_count(ctypes.byref(count))
        return count.value if code == 0 else 0

    def close(self):
        pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def _as_i32_rows(contexts) -> np.ndarray:
    """Stacks contexts into [rows, length] int32, keeping only a common tail when lengths differ.

    The reference uses only each row's last ``window`` tokens, so rows of different lengths are
    trimmed to the shortest length first (the caller checks that it is at least the window).
    """
    if isinstance(contexts, np.ndarray) and contexts.ndim == 2:
        return np.ascontiguousarray(contexts, dtype=np.int32)
    rows = [np.asarray(c, dtype=np.int64).ravel() for c in contexts]
    shortest = min(len(r) for r in rows)
    return np.ascontiguousarray(np.stack([r[len(r) - shortest:] for r in rows]).astype(np.int32))


class TextEngine:
    """Decoding loop for a windowed language model, on the GPU (TextEngine.java:37-427)."""

    def __init__(self, runtime: Basalt, model: ModelSpec, handle: int):
        self._runtime = runtime
        self._model = model
        self._h = handle
        self._lib = _lib.load()

    # ---- construction (TextEngine.of, TextEngine.java:61-74) ----
    @staticmethod
    def of(runtime: Basalt, model: ModelSpec, vocabulary: int, window: int) -> "TextEngine":
        if runtime is None:
            raise IllegalArgumentException("runtime must not be null", _lib.BST_INVALID)
        if model is None:
            raise IllegalArgumentException("model must not be null", _lib.BST_INVALID)
        if vocabulary < 2:
            raise IllegalArgumentException(f"vocabulary must be at least 2, got {vocabulary}",
                                           _lib.BST_INVALID)
        if window < 1:
            raise IllegalArgumentException(f"window must be at least 1, got {window}",
                                           _lib.BST_INVALID)
        if model.vocabulary != vocabulary or model.window != window:
            raise IllegalArgumentException(
                f"model was built for vocabulary={model.vocabulary} window={model.window}",
                _lib.BST_INVALID)
        lib = _lib.load()
        spec = model.struct()
        handle = ctypes.c_uint64(0)
        _raise(lib.bst_engine_create(ctypes.byref(spec), runtime.device, ctypes.byref(handle)))
        return TextEngine(runtime, model, handle.value)

    @staticmethod
    def ofParameters(runtime: Basalt, named_parameters, vocabulary: int, window: int,
                     heads: int = 0, weight_dtype: str = "f32",
                     kv_dtype: str = "f32") -> "TextEngine":
        """TextEngine.of on a module given by its namedParameters: (name, array) pairs in the
        module's order, arrays in the reference's layout. Raises
        BasaltUnsupportedOperationException for a module the engine does not serve."""
        lib = _lib.load()
        args = _parameter_arrays(named_parameters)
        values = [np.ascontiguousarray(v, dtype=np.float32) for _, v in named_parameters]
        ptrs = (_lib._f32p * len(values))(*[v.ctypes.data_as(_lib._f32p) for v in values])
        handle = ctypes.c_uint64(0)
        _raise(lib.bst_engine_create_from_parameters(
            args[0], args[1], args[2], ptrs, len(values), vocabulary, window, heads,
            DTYPES[weight_dtype], DTYPES[kv_dtype], runtime.device, ctypes.byref(handle)))
        model = recognize_model(named_parameters, vocabulary, window, heads)
        from dataclasses import replace

        model = replace(model, weight_dtype=weight_dtype, kv_dtype=kv_dtype)
        return TextEngine(runtime, model, handle.value)

    def vocabulary(self) -> int:
        return self._model.vocabulary

    def window(self) -> int:
        return self._model.window

    def model(self) -> ModelSpec:
        return self._model

    @property
    def handle(self) -> int:
        return self._h

    def _call(self, code: int):
        return _raise(code, self._h)

    def _check_context(self, context):
        if context is None:
            raise IllegalArgumentException("context must not be null", _lib.BST_INVALID)

    # ---- scoring (TextEngine.java:96-148) ----
    def scores(self, context: Sequence[int]) -> np.ndarray:
        self._check_context(context)
        return self.scoresBatch([context])[0]

    def scoresBatch(self, contexts) -> np.ndarray:
        if contexts is None:
            raise IllegalArgumentException("contexts must not be null", _lib.BST_INVALID)
        if len(contexts) == 0:
            raise IllegalArgumentException("contexts must not be empty", _lib.BST_INVALID)
        for row, c in enumerate(contexts):
            if c is None or len(c) < self.window():
                got = "null" if c is None else len(c)
                raise IllegalArgumentException(
                    f"contexts[{row}] needs at least {self.window()} tokens, got {got}",
                    _lib.BST_INVALID)
        arr = _as_i32_rows(contexts)
        out = np.empty((arr.shape[0], self.vocabulary()), dtype=np.float64)
        self._call(self._lib.bst_scores(self._h, arr.ctypes.data_as(_lib._i32p), arr.shape[0],
                                        arr.shape[1], out.ctypes.data_as(_lib._f64p)))
        return out

    # ---- greedy (TextEngine.java:158-193, 232-254) ----
    def generate(self, context: Sequence[int], steps: int) -> np.ndarray:
        self._check_context(context)
        return self._generate([context], steps, None)[0]

    def stream(self, context: Sequence[int], steps: int,
               sink: Callable[[int], None]) -> np.ndarray:
        if sink is None:
            raise IllegalArgumentException("sink must not be null", _lib.BST_INVALID)
        self._check_context(context)
        return self._generate([context], steps, lambda row, step, token: sink(token))[0]

    def generateBatch(self, contexts, steps: int) -> np.ndarray:
        if contexts is None:
            raise IllegalArgumentException("contexts must not be null", _lib.BST_INVALID)
        if len(contexts) == 0:
            raise IllegalArgumentException("contexts must not be empty", _lib.BST_INVALID)
        return self._generate(contexts, steps, None)

    def streamBatch(self, contexts, steps: int,
                    sink: Callable[[int, int, int], None]) -> np.ndarray:
        """generateBatch with a per-token sink(row, step, token), in step order per row."""
        return self._generate(contexts, steps, sink)

    # ---- sampling (TextEngine.java:201-227, 267-290) ----
    def sample(self, context: Sequence[int], steps: int, temperature: float,
               topK: int) -> np.ndarray:
        self._check_context(context)
        return self._sample([context], steps, temperature, topK, None)[0]

    def streamSampled(self, context: Sequence[int], steps: int, temperature: float, topK: int,
                      sink: Callable[[int], None]) -> np.ndarray:
        if sink is None:
            raise IllegalArgumentException("sink must not be null", _lib.BST_INVALID)
        self._check_context(context)
        return self._sample([context], steps, temperature, topK,
                            lambda row, step, token: sink(token))[0]

    def sampleBatch(self, contexts, steps: int, temperature: float, topK: int,
                    sink: Optional[Callable[[int, int, int], None]] = None) -> np.ndarray:
        """Rows sampled together; the tokens equal ``len(contexts)`` successive ``sample`` calls
        on this engine, and the generator ends where those calls would leave it."""
        return self._sample(contexts, steps, temperature, topK, sink)

    def seed(self, seed: int):
        self._call(self._lib.bst_seed(self._h, int(seed)))

    @property
    def rng_state(self) -> int:
        v = ctypes.c_int64(0)
        self._call(self._lib.bst_get_rng_state(self._h, ctypes.byref(v)))
        return v.value

    @rng_state.setter
    def rng_state(self, state: int):
        """Sets the raw 48-bit java.util.Random state (see basalt_b200.sharding)."""
        self._call(self._lib.bst_set_rng_state(self._h, int(state)))

    # ---- weights (TextEngine.java:298-350, Module.java:59-76) ----
    def save(self, path):
        if path is None:
            raise IllegalArgumentException("path must not be null", _lib.BST_INVALID)
        self._call(self._lib.bst_save(self._h, str(path).encode()))

    def load(self, path):
        if path is None:
            raise IllegalArgumentException("path must not be null", _lib.BST_INVALID)
        self._call(self._lib.bst_load(self._h, str(path).encode()))

    def parameters(self) -> list[tuple[str, int]]:
        count = ctypes.c_int32(0)
        self._call(self._lib.bst_parameter_count(self._h, ctypes.byref(count)))
        out = []
        buf = ctypes.create_string_buffer(256)
        size = ctypes.c_int64(0)
        for i in range(count.value):
            self._call(self._lib.bst_parameter_info(self._h, i, buf, len(buf), ctypes.byref(size)))
            out.append((buf.value.decode(), size.value))
        return out

    def setParameter(self, name: str, values):
        v = np.ascontiguousarray(values, dtype=np.float32).ravel()
        self._call(self._lib.bst_set_parameter(self._h, name.encode(), v.ctypes.data_as(_lib._f32p),
                                               v.size))

    def loadStateDict(self, state: dict):
        for name, _ in self.parameters():
            if name not in state:
                raise IllegalArgumentException(f"missing state entry {name}", _lib.BST_INVALID)
            self.setParameter(name, state[name])

    def parameter(self, name: str) -> np.ndarray:
        size = dict(self.parameters())[name]
        v = np.empty(size, dtype=np.float32)
        self._call(self._lib.bst_get_parameter(self._h, name.encode(), v.ctypes.data_as(_lib._f32p),
                                               size))
        return v

    def stateDict(self) -> dict:
        return {name: self.parameter(name) for name, _ in self.parameters()}

    # ---- NativeContext-style scopes and stats ----
    def beginScope(self):
        self._call(self._lib.bst_begin_scope(self._h))

    def endScope(self) -> int:
        released = ctypes.c_int32(0)
        self._call(self._lib.bst_end_scope(self._h, ctypes.byref(released)))
        return released.value

    def scopeDepth(self) -> int:
        depth = ctypes.c_int32(0)
        self._call(self._lib.bst_scope_depth(self._h, ctypes.byref(depth)))
        return depth.value

    def stats(self) -> dict:
        out = (ctypes.c_int64 * 4)()
        self._call(self._lib.bst_engine_stats(self._h, out))
        return {"tensors": out[0], "bytes": out[1], "graph_nodes": out[2], "launches": out[3]}

    def cuda_stream(self) -> int:
        ptr = ctypes.c_void_p(0)
        self._call(self._lib.bst_engine_stream(self._h, ctypes.byref(ptr)))
        return ptr.value or 0

    def profile(self, enabled: bool = True):
        self._call(self._lib.bst_profile_enable(self._h, int(enabled)))

    def profile_reset(self):
        self._call(self._lib.bst_profile_reset(self._h))

    def profile_read(self) -> dict:
        out = {}
        buf = ctypes.create_string_buffer(64)
        n = ctypes.c_int64(0)
        ms, by, fl = ctypes.c_double(0), ctypes.c_double(0), ctypes.c_double(0)
        for cls in range(_lib.KERNEL_CLASSES):
            self._call(self._lib.bst_profile_read(self._h, cls, buf, len(buf), ctypes.byref(n),
                                                  ctypes.byref(ms), ctypes.byref(by),
                                                  ctypes.byref(fl)))
            if n.value:
                out[buf.value.decode()] = {"launches": n.value, "ms": ms.value,
                                           "bytes": by.value, "flops": fl.value}
        return out

    # ---- decode with per-step logits (parity checks) ----
    def generateWithLogits(self, contexts, steps: int):
        """Greedy decode of [rows] contexts; returns (tokens [rows, steps],
        logits [rows, steps, V]) — the logits each step's token was chosen from."""
        arr = self._prepare(contexts, steps)
        tokens = np.zeros((arr.shape[0], steps), dtype=np.int32)
        logits = np.zeros((arr.shape[0], steps, self.vocabulary()), dtype=np.float32)
        self._call(self._lib.bst_generate_logits(self._h, arr.ctypes.data_as(_lib._i32p),
                                                 arr.shape[0], arr.shape[1], steps,
                                                 tokens.ctypes.data_as(_lib._i32p),
                                                 logits.ctypes.data_as(_lib._f32p)))
        return tokens, logits

    def sampleWithLogits(self, contexts, steps: int, temperature: float, topK: int):
        arr = self._prepare(contexts, steps)
        tokens = np.zeros((arr.shape[0], steps), dtype=np.int32)
        logits = np.zeros((arr.shape[0], steps, self.vocabulary()), dtype=np.float32)
        self._call(self._lib.bst_sample_logits(self._h, arr.ctypes.data_as(_lib._i32p),
                                               arr.shape[0], arr.shape[1], steps,
                                               float(np.float32(temperature)), int(topK),
                                               tokens.ctypes.data_as(_lib._i32p),
                                               logits.ctypes.data_as(_lib._f32p)))
        return tokens, logits

    def generateWithLogitsOf(self, contexts, steps: int, rows: Sequence[int]):
        """generateWithLogits keeping only the logits of `rows`: (tokens [N, steps],
        logits [len(rows), steps, V])."""
        arr = self._prepare(contexts, steps)
        watch = np.ascontiguousarray(np.asarray(rows, dtype=np.int32))
        tokens = np.zeros((arr.shape[0], steps), dtype=np.int32)
        logits = np.zeros((watch.size, steps, self.vocabulary()), dtype=np.float32)
        self._call(self._lib.bst_generate_logits_rows(
            self._h, arr.ctypes.data_as(_lib._i32p), arr.shape[0], arr.shape[1], steps,
            tokens.ctypes.data_as(_lib._i32p), watch.size, watch.ctypes.data_as(_lib._i32p),
            logits.ctypes.data_as(_lib._f32p)))
        return tokens, logits

    def sampleWithLogitsOf(self, contexts, steps: int, temperature: float, topK: int,
                           rows: Sequence[int]):
        """sampleWithLogits keeping only the logits of `rows`."""
        arr = self._prepare(contexts, steps)
        watch = np.ascontiguousarray(np.asarray(rows, dtype=np.int32))
        tokens = np.zeros((arr.shape[0], steps), dtype=np.int32)
        logits = np.zeros((watch.size, steps, self.vocabulary()), dtype=np.float32)
        self._call(self._lib.bst_sample_logits_rows(
            self._h, arr.ctypes.data_as(_lib._i32p), arr.shape[0], arr.shape[1], steps,
            float(np.float32(temperature)), int(topK), tokens.ctypes.data_as(_lib._i32p),
            watch.size, watch.ctypes.data_as(_lib._i32p), logits.ctypes.data_as(_lib._f32p)))
        return tokens, logits

    # ---- device-buffer entry points (callers that keep contexts and tokens in HBM) ----
    def generate_device(self, contexts_ptr: int, rows: int, length: int, steps: int,
                        tokens_ptr: int):
        self._call(self._lib.bst_generate_device(self._h, contexts_ptr, rows, length, steps,
                                                 tokens_ptr))

    def sample_device(self, contexts_ptr: int, rows: int, length: int, steps: int,
                      temperature: float, topK: int, tokens_ptr: int):
        self._call(self._lib.bst_sample_device(self._h, contexts_ptr, rows, length, steps,
                                               temperature, topK, tokens_ptr))

    def close(self):
        if self._h:
            _raise(self._lib.bst_engine_destroy(self._h))
            self._h = 0

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            if self._h:
                self._lib.bst_engine_destroy(self._h)
                self._h = 0
        except Exception:
            pass

    # ---- shared plumbing ----
    def _prepare(self, contexts, steps):
        if steps < 1:
            raise IllegalArgumentException(f"steps must be at least 1, got {steps}",
                                           _lib.BST_INVALID)
        for row, c in enumerate(contexts):
            if c is None:
                raise IllegalArgumentException("context must not be null", _lib.BST_INVALID)
            if len(c) < self.window():
                raise IllegalArgumentException(
                    f"context needs at least {self.window()} tokens, got {len(c)}",
                    _lib.BST_INVALID)
        return _as_i32_rows(contexts)

    @staticmethod
    def _sink(sink):
        if sink is None:
            return _lib.TOKEN_SINK(0), []
        errors = []

        def trampoline(user, row, step, token):
            try:
                sink(row, step, token)
                return 0
            except BaseException as exc:  # surfaced after the call returns
                errors.append(exc)
                return 1

        return _lib.TOKEN_SINK(trampoline), errors

    def _generate(self, contexts, steps, sink):
        arr = self._prepare(contexts, steps)
        out = np.zeros((arr.shape[0], steps), dtype=np.int32)
        cb, errors = self._sink(sink)
        code = self._lib.bst_generate(self._h, arr.ctypes.data_as(_lib._i32p), arr.shape[0],
                                      arr.shape[1], steps, out.ctypes.data_as(_lib._i32p), cb,
                                      None)
        if errors:
            raise errors[0]
        self._call(code)
        return out

    def _sample(self, contexts, steps, temperature, topK, sink):
        if steps < 1:
            raise IllegalArgumentException(f"steps must be at least 1, got {steps}",
                                           _lib.BST_INVALID)
        t = np.float32(temperature)
        if not (t > 0) or not np.isfinite(t):
            raise IllegalArgumentException(
                f"temperature must be positive and finite, got {temperature}", _lib.BST_INVALID)
        if topK < 1:
            raise IllegalArgumentException(f"topK must be at least 1, got {topK}",
                                           _lib.BST_INVALID)
        arr = self._prepare(contexts, steps)
        out = np.zeros((arr.shape[0], steps), dtype=np.int32)
        cb, errors = self._sink(sink)
        code = self._lib.bst_sample(self._h, arr.ctypes.data_as(_lib._i32p), arr.shape[0],
                                    arr.shape[1], steps, float(t), int(topK),
                                    out.ctypes.data_as(_lib._i32p), cb, None)
        if errors:
            raise errors[0]
        self._call(code)
        return out


def _parameter_arrays(named_parameters):
    names = [n.encode() for n, _ in named_parameters]
    shapes = [np.shape(v) for _, v in named_parameters]
    c_names = (ctypes.c_char_p * len(names))(*names)
    ranks = (ctypes.c_int32 * len(shapes))(*[len(s) for s in shapes])
    flat = [int(x) for s in shapes for x in s]
    dims = (ctypes.c_int64 * max(1, len(flat)))(*flat)
    return c_names, ranks, dims


def recognize_model(named_parameters, vocabulary: int, window: int, heads: int = 0) -> ModelSpec:
    """The architecture the engine serves for a module with these namedParameters (name, array)
    pairs, or BasaltUnsupportedOperationException: the decision TextEngine's dispatch makes."""
    names, ranks, dims = _parameter_arrays(named_parameters)
    spec = _lib.ModelSpecStruct()
    _raise(_lib.load().bst_recognize_model(names, ranks, dims, len(named_parameters), vocabulary,
                                           window, heads, ctypes.byref(spec)))
    family = {v: k for k, v in FAMILIES.items()}[spec.family]
    return ModelSpec(family, spec.vocabulary, spec.window, spec.dimension, spec.layers, spec.heads,
                     spec.hidden)


def write_synthetic_weights(model: ModelSpec, path, seed: int, stddev: float = 0.02):
    """Writes a TextEngine weight file of N(0, stddev) parameters (LayerNorm gamma 1, beta 0)
    drawn with java.util.Random(seed).nextGaussian in namedParameters order; with bf16 weights
    the matrices are rounded to bf16-representable values so every reader sees the same model."""
    spec = model.struct()
    _raise(_lib.load().bst_write_synthetic_weights(ctypes.byref(spec), str(path).encode(),
                                                   int(seed), float(stddev)))


def synthetic_prompts(seed: int, rows: int, length: int, bound: int) -> np.ndarray:
    """``java.util.Random(seed).nextInt(bound)`` ids, one row after another."""
    out = np.empty((rows, length), dtype=np.int32)
    _raise(_lib.load().bst_synthetic_prompts(int(seed), rows, length, bound,
                                             out.ctypes.data_as(_lib._i32p)))
    return out


def left_pad(prompts: np.ndarray, window: int, pad: int) -> np.ndarray:
    """Left-pads [rows, P] prompts with PAD to the window, as the padded decoder expects."""
    rows, plen = prompts.shape
    if plen >= window:
        return np.ascontiguousarray(prompts[:, plen - window:], dtype=np.int32)
    out = np.full((rows, window), pad, dtype=np.int32)
    out[:, window - plen:] = prompts
    return out
