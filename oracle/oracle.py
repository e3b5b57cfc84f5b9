"""ctypes binding of the CPU oracle (liboracle.so) — TEST INFRASTRUCTURE ONLY.

The oracle restates the reference's TextEngine decode path on the CPU (see oracle.h for what is
restated from which reference file). Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` load this module; the CUDA product never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "liboracle.so"

FAMILY_PADDED_DECODER = 1
FAMILY_DECODER = 2
FAMILY_CHAR_LM = 3
FAMILY_LAST_TOKEN = 4


class OracleError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{message} (code {code})")
        self.code = code


class _Random(ctypes.Structure):
    _fields_ = [("seed", ctypes.c_uint64), ("have_next_gaussian", ctypes.c_int32),
                ("next_gaussian", ctypes.c_double)]


class _Spec(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in (
        "family", "vocabulary", "window", "dimension", "layers", "heads", "hidden", "fused_tiles")]


SINK = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32)


def build() -> Path:
    """Compiles liboracle.so with the committed Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIBRARY


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            build()
        L = ctypes.CDLL(str(LIBRARY))
        P = ctypes.POINTER
        f32p, f64p, i32p, i64p = (P(ctypes.c_float), P(ctypes.c_double), P(ctypes.c_int32),
                                  P(ctypes.c_int64))
        sig = {
            "orc_random_set_seed": (None, [P(_Random), ctypes.c_int64]),
            "orc_random_next": (ctypes.c_int32, [P(_Random), ctypes.c_int32]),
            "orc_random_next_int": (ctypes.c_int32, [P(_Random)]),
            "orc_random_next_int_bound": (ctypes.c_int32, [P(_Random), ctypes.c_int32]),
            "orc_random_next_float": (ctypes.c_float, [P(_Random)]),
            "orc_random_next_double": (ctypes.c_double, [P(_Random)]),
            "orc_random_next_gaussian": (ctypes.c_double, [P(_Random)]),
            "orc_matmul": (None, [f32p, f32p, f32p, ctypes.c_int64, ctypes.c_int64,
                                  ctypes.c_int64, ctypes.c_int32]),
            "orc_add": (ctypes.c_int32, [f32p, i64p, ctypes.c_int32, f32p, i64p, ctypes.c_int32,
                                         f32p]),
            "orc_mul": (ctypes.c_int32, [f32p, i64p, ctypes.c_int32, f32p, i64p, ctypes.c_int32,
                                         f32p]),
            "orc_relu": (None, [f32p, f32p, ctypes.c_int64]),
            "orc_gelu": (None, [f32p, f32p, ctypes.c_int64]),
            "orc_softmax": (ctypes.c_int32, [f32p, f32p, ctypes.c_int64, ctypes.c_int64]),
            "orc_layer_norm": (ctypes.c_int32, [f32p, f32p, f32p, f32p, ctypes.c_int64,
                                                ctypes.c_int64, ctypes.c_float]),
            "orc_engine_create": (ctypes.c_void_p, [P(_Spec)]),
            "orc_engine_destroy": (None, [ctypes.c_void_p]),
            "orc_engine_error": (ctypes.c_char_p, [ctypes.c_void_p]),
            "orc_param_count": (ctypes.c_int32, [ctypes.c_void_p]),
            "orc_param_name": (ctypes.c_char_p, [ctypes.c_void_p, ctypes.c_int32]),
            "orc_param_size": (ctypes.c_int64, [ctypes.c_void_p, ctypes.c_int32]),
            "orc_set_param": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_char_p, f32p,
                                               ctypes.c_int64]),
            "orc_get_param": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_char_p, f32p,
                                               ctypes.c_int64]),
            "orc_save": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_char_p]),
            "orc_load": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_char_p]),
            "orc_forward": (ctypes.c_int32, [ctypes.c_void_p, f32p, ctypes.c_int32, f32p]),
            "orc_scores_batch": (ctypes.c_int32, [ctypes.c_void_p, i32p, ctypes.c_int32,
                                                  ctypes.c_int32, f64p]),
            "orc_generate": (ctypes.c_int32, [ctypes.c_void_p, i32p, ctypes.c_int32,
                                              ctypes.c_int32, i32p, SINK, ctypes.c_void_p]),
            "orc_generate_batch": (ctypes.c_int32, [ctypes.c_void_p, i32p, ctypes.c_int32,
                                                    ctypes.c_int32, ctypes.c_int32, i32p]),
            "orc_generate_batch_cached": (ctypes.c_int32, [ctypes.c_void_p, i32p, ctypes.c_int32,
                                                    ctypes.c_int32, ctypes.c_int32, i32p]),
            "orc_sample": (ctypes.c_int32, [ctypes.c_void_p, i32p, ctypes.c_int32,
                                            ctypes.c_int32, ctypes.c_float, ctypes.c_int32, i32p,
                                            SINK, ctypes.c_void_p]),
            "orc_seed": (None, [ctypes.c_void_p, ctypes.c_int64]),
            "orc_rng_state": (ctypes.c_uint64, [ctypes.c_void_p]),
            "orc_set_rng_state": (None, [ctypes.c_void_p, ctypes.c_uint64]),
            "orc_forced_scores": (ctypes.c_int32, [ctypes.c_void_p, i32p, ctypes.c_int32,
                                                   ctypes.c_int32, i32p, f32p]),
            "orc_draw": (ctypes.c_int32, [ctypes.c_void_p, f64p, ctypes.c_int32, ctypes.c_float,
                                          ctypes.c_int32]),
            "orc_forced_scores_single_pass": (ctypes.c_int32, [ctypes.c_void_p, i32p,
                                                               ctypes.c_int32, ctypes.c_int32,
                                                               ctypes.c_int32, i32p, f32p]),
            "orc_fill_synthetic": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int64,
                                                    ctypes.c_double, ctypes.c_int32]),
            "orc_synthetic_prompts": (None, [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                             ctypes.c_int32, i32p]),
            "orc_threads": (ctypes.c_int32, []),
            "orc_set_threads": (None, [ctypes.c_int32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _ptr(array: np.ndarray, ctype):
    return array.ctypes.data_as(ctypes.POINTER(ctype))


class JavaRandom:
    """java.util.Random restated from the JDK specification."""

    def __init__(self, seed: int):
        self._state = _Random()
        lib().orc_random_set_seed(ctypes.byref(self._state), seed)

    @property
    def state(self) -> int:
        return int(self._state.seed)

    def next(self, bits: int) -> int:
        return lib().orc_random_next(ctypes.byref(self._state), bits)

    def next_int(self, bound: int | None = None) -> int:
        if bound is None:
            return lib().orc_random_next_int(ctypes.byref(self._state))
        return lib().orc_random_next_int_bound(ctypes.byref(self._state), bound)

    def next_float(self) -> float:
        return lib().orc_random_next_float(ctypes.byref(self._state))

    def next_double(self) -> float:
        return lib().orc_random_next_double(ctypes.byref(self._state))

    def next_gaussian(self) -> float:
        return lib().orc_random_next_gaussian(ctypes.byref(self._state))


def matmul(a: np.ndarray, b: np.ndarray, fused_tiles: bool = True) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    m, k = a.shape
    k2, n = b.shape
    assert k == k2
    c = np.empty((m, n), dtype=np.float32)
    lib().orc_matmul(_ptr(a, ctypes.c_float), _ptr(b, ctypes.c_float), _ptr(c, ctypes.c_float),
                     m, k, n, int(fused_tiles))
    return c


def _binary(fn, a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    out_shape = np.broadcast_shapes(a.shape, b.shape)
    out = np.empty(out_shape, dtype=np.float32)
    ash = np.array(a.shape, dtype=np.int64)
    bsh = np.array(b.shape, dtype=np.int64)
    status = fn(_ptr(a, ctypes.c_float), _ptr(ash, ctypes.c_int64), a.ndim,
                _ptr(b, ctypes.c_float), _ptr(bsh, ctypes.c_int64), b.ndim,
                _ptr(out, ctypes.c_float))
    if status:
        raise OracleError(status, "binary op shape mismatch")
    return out


def add(a, b):
    return _binary(lib().orc_add, a, b)


def mul(a, b):
    return _binary(lib().orc_mul, a, b)


def relu(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty_like(a)
    lib().orc_relu(_ptr(a, ctypes.c_float), _ptr(out, ctypes.c_float), a.size)
    return out


def gelu(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty_like(a)
    lib().orc_gelu(_ptr(a, ctypes.c_float), _ptr(out, ctypes.c_float), a.size)
    return out


def softmax(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty_like(a)
    status = lib().orc_softmax(_ptr(a, ctypes.c_float), _ptr(out, ctypes.c_float),
                               a.size // a.shape[-1], a.shape[-1])
    if status:
        raise OracleError(status, "softmax denominator is not finite")
    return out


def layer_norm(a, gamma, beta, eps=1e-5):
    a = np.ascontiguousarray(a, dtype=np.float32)
    gamma = np.ascontiguousarray(gamma, dtype=np.float32)
    beta = np.ascontiguousarray(beta, dtype=np.float32)
    out = np.empty_like(a)
    lib().orc_layer_norm(_ptr(a, ctypes.c_float), _ptr(gamma, ctypes.c_float),
                         _ptr(beta, ctypes.c_float), _ptr(out, ctypes.c_float),
                         a.size // a.shape[-1], a.shape[-1], eps)
    return out


class OracleEngine:
    """CPU restatement of ``TextEngine`` bound to one model (see oracle.h)."""

    def __init__(self, family: int, vocabulary: int, window: int, dimension: int = 0,
                 layers: int = 0, heads: int = 1, hidden: int = 0, fused_tiles: bool = True):
        spec = _Spec(family, vocabulary, window, dimension, layers, heads, hidden,
                     int(fused_tiles))
        self.vocabulary = vocabulary
        self.window = window
        self._h = lib().orc_engine_create(ctypes.byref(spec))
        if not self._h:
            raise OracleError(-1, "invalid model specification")

    @classmethod
    def from_spec(cls, spec) -> "OracleEngine":
        return cls(spec.family, spec.vocabulary, spec.window, spec.dimension, spec.layers,
                   spec.heads, spec.hidden)

    def close(self):
        if self._h:
            lib().orc_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, status: int):
        if status < 0:
            raise OracleError(status, lib().orc_engine_error(self._h).decode())
        return status

    def parameters(self):
        L = lib()
        return [(L.orc_param_name(self._h, i).decode(), L.orc_param_size(self._h, i))
                for i in range(L.orc_param_count(self._h))]

    def set(self, name: str, values: np.ndarray):
        v = np.ascontiguousarray(values, dtype=np.float32).ravel()
        self._check(lib().orc_set_param(self._h, name.encode(), _ptr(v, ctypes.c_float), v.size))

    def get(self, name: str) -> np.ndarray:
        size = dict(self.parameters())[name]
        v = np.empty(size, dtype=np.float32)
        self._check(lib().orc_get_param(self._h, name.encode(), _ptr(v, ctypes.c_float), size))
        return v

    def save(self, path):
        self._check(lib().orc_save(self._h, str(path).encode()))

    def load(self, path):
        self._check(lib().orc_load(self._h, str(path).encode()))

    def forward(self, ids: np.ndarray) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.float32)
        rows = ids.shape[0]
        out = np.empty((rows, self.vocabulary), dtype=np.float32)
        self._check(lib().orc_forward(self._h, _ptr(ids, ctypes.c_float), rows,
                                      _ptr(out, ctypes.c_float)))
        return out

    @staticmethod
    def _contexts(contexts):
        arr = np.ascontiguousarray(np.asarray(contexts, dtype=np.int32))
        if arr.ndim == 1:
            arr = arr[None, :]
        return arr

    def scores_batch(self, contexts) -> np.ndarray:
        arr = self._contexts(contexts)
        out = np.empty((arr.shape[0], self.vocabulary), dtype=np.float64)
        self._check(lib().orc_scores_batch(self._h, _ptr(arr, ctypes.c_int32), arr.shape[0],
                                           arr.shape[1], _ptr(out, ctypes.c_double)))
        return out

    def scores(self, context) -> np.ndarray:
        return self.scores_batch([context])[0]

    def _sink(self, sink):
        if sink is None:
            return SINK(0)
        return SINK(lambda user, row, step, token: sink(token))

    def generate(self, context, steps: int, sink=None) -> np.ndarray:
        arr = self._contexts(context)
        out = np.zeros(max(steps, 1), dtype=np.int32)
        cb = self._sink(sink)
        self._check(lib().orc_generate(self._h, _ptr(arr, ctypes.c_int32), arr.shape[1], steps,
                                       _ptr(out, ctypes.c_int32), cb, None))
        return out[:steps]

    def generate_batch(self, contexts, steps: int) -> np.ndarray:
        arr = self._contexts(contexts)
        out = np.zeros((arr.shape[0], max(steps, 1)), dtype=np.int32)
        self._check(lib().orc_generate_batch(self._h, _ptr(arr, ctypes.c_int32), arr.shape[0],
                                             arr.shape[1], steps, _ptr(out, ctypes.c_int32)))
        return out[:, :steps]

    def generate_batch_cached(self, contexts, steps: int) -> np.ndarray:
        """Greedy batch decode with a per-row KV cache (padded decoder; CPU timing baseline)."""
        arr = self._contexts(contexts)
        out = np.zeros((arr.shape[0], max(steps, 1)), dtype=np.int32)
        self._check(lib().orc_generate_batch_cached(self._h, _ptr(arr, ctypes.c_int32),
                                                    arr.shape[0], arr.shape[1], steps,
                                                    _ptr(out, ctypes.c_int32)))
        return out[:, :steps]

    def sample(self, context, steps: int, temperature: float, top_k: int,
               sink=None) -> np.ndarray:
        arr = self._contexts(context)
        out = np.zeros(max(steps, 1), dtype=np.int32)
        cb = self._sink(sink)
        self._check(lib().orc_sample(self._h, _ptr(arr, ctypes.c_int32), arr.shape[1], steps,
                                     temperature, top_k, _ptr(out, ctypes.c_int32), cb, None))
        return out[:steps]

    def seed(self, seed: int):
        lib().orc_seed(self._h, seed)

    @property
    def rng_state(self) -> int:
        return int(lib().orc_rng_state(self._h))

    @rng_state.setter
    def rng_state(self, state: int):
        lib().orc_set_rng_state(self._h, state)

    def forced_scores(self, context, forced) -> np.ndarray:
        arr = self._contexts(context)
        forced = np.ascontiguousarray(forced, dtype=np.int32)
        out = np.empty((forced.size, self.vocabulary), dtype=np.float32)
        self._check(lib().orc_forced_scores(self._h, _ptr(arr, ctypes.c_int32), arr.shape[1],
                                            forced.size, _ptr(forced, ctypes.c_int32),
                                            _ptr(out, ctypes.c_float)))
        return out

    def forced_scores_rows(self, contexts, forced) -> np.ndarray:
        """Teacher-forced logits [rows, steps, V] of several rows of the padded decoder.

        ``forced[r]`` are the tokens row r pushes after each step. Rows whose window still starts
        with PAD at every step take one causal pass each (``orc_forced_scores_single_pass``);
        otherwise every step recomputes the full window, as TextEngine does."""
        arr = self._contexts(contexts)
        forced = np.ascontiguousarray(np.asarray(forced, dtype=np.int32).reshape(arr.shape[0], -1))
        rows, steps = forced.shape
        out = np.empty((rows, steps, self.vocabulary), dtype=np.float32)
        status = lib().orc_forced_scores_single_pass(
            self._h, _ptr(arr, ctypes.c_int32), rows, arr.shape[1], steps,
            _ptr(forced, ctypes.c_int32), _ptr(out, ctypes.c_float))
        if status == -8:
            for r in range(rows):
                out[r] = self.forced_scores(arr[r], forced[r])
        else:
            self._check(status)
        return out

    def fill_synthetic(self, seed: int, stddev: float = 0.02, round_bf16: bool = False):
        """N(0, stddev) parameters from java.util.Random(seed).nextGaussian (LayerNorm 1 / 0)."""
        self._check(lib().orc_fill_synthetic(self._h, seed, stddev, int(round_bf16)))

    def draw(self, scores, temperature: float, top_k: int) -> int:
        s = np.ascontiguousarray(scores, dtype=np.float64)
        return self._check(lib().orc_draw(self._h, _ptr(s, ctypes.c_double), s.size,
                                          temperature, top_k))


def synthetic_prompts(seed: int, rows: int, length: int, bound: int) -> np.ndarray:
    """[rows, length] ids of java.util.Random(seed).nextInt(bound), row after row."""
    out = np.empty((rows, length), dtype=np.int32)
    lib().orc_synthetic_prompts(seed, rows, length, bound, _ptr(out, ctypes.c_int32))
    return out


def left_pad(prompts: np.ndarray, window: int, pad: int) -> np.ndarray:
    """Prompts left-padded with `pad` to at least `window` ids (TextEngine reads the tail)."""
    prompts = np.asarray(prompts, dtype=np.int32)
    if prompts.shape[1] >= window:
        return np.ascontiguousarray(prompts[:, prompts.shape[1] - window:])
    out = np.full((prompts.shape[0], window), pad, dtype=np.int32)
    out[:, window - prompts.shape[1]:] = prompts
    return out


def write_synthetic_weights(model, path, seed: int, stddev: float = 0.02) -> "OracleEngine":
    """Writes the TextEngine weight file of a synthetic model and returns the oracle bound to it.

    ``model`` is any object with the ModelSpec fields (family name, sizes, weight_dtype)."""
    family = {"padded_decoder": FAMILY_PADDED_DECODER, "decoder": FAMILY_DECODER,
              "char_lm": FAMILY_CHAR_LM, "last_token": FAMILY_LAST_TOKEN}[model.family]
    engine = OracleEngine(family, model.vocabulary, model.window, model.dimension, model.layers,
                          model.heads, model.hidden)
    engine.fill_synthetic(seed, stddev, model.weight_dtype == "bf16")
    engine.save(path)
    return engine


def lcg_advance(state: int, steps: int) -> int:
    """java.util.Random's generator state after `steps` steps, one step at a time."""
    for _ in range(steps):
        state = (state * 0x5DEECE66D + 0xB) & ((1 << 48) - 1)
    return state


def lcg_scramble(seed: int) -> int:
    return (seed ^ 0x5DEECE66D) & ((1 << 48) - 1)


def set_threads(threads: int):
    lib().orc_set_threads(threads)


def threads() -> int:
    return lib().orc_threads()


if os.environ.get("BASALT_ORACLE_THREADS"):
    set_threads(int(os.environ["BASALT_ORACLE_THREADS"]))
