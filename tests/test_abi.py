"""The C-ABI library without a GPU: it loads, exports every entry point the header declares,
and its host-only helpers (weight file format, seeded generators) agree with the oracle."""
import ctypes
import re
import struct

import numpy as np
import pytest

from basalt_b200 import _lib
from basalt_b200.text_engine import (Basalt, ModelSpec, synthetic_prompts,
                                     write_synthetic_weights)
from oracle import oracle as orc


def declared_symbols():
    text = _lib.HEADER.read_text()
    return sorted(set(re.findall(r"^\s*int32_t\s+(bst_\w+)\s*\(", text, flags=re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 25
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert lib.bst_abi_version() == 1


def test_header_status_codes_match_the_reference():
    # native/src/error.rs:9-17
    text = _lib.HEADER.read_text()
    codes = dict(re.findall(r"#define (BST_[A-Z_]+) \((-\d)\)", text))
    assert codes == {"BST_INVALID": "-1", "BST_SHAPE": "-2", "BST_UNKNOWN_HANDLE": "-3",
                     "BST_CONTEXT": "-4", "BST_GRAPH": "-5", "BST_PANIC": "-6", "BST_OOM": "-7",
                     "BST_UNSUPPORTED": "-8"}


def test_unknown_handles_are_rejected():
    lib = _lib.load()
    assert lib.bst_engine_destroy(12345678) == _lib.BST_UNKNOWN_HANDLE
    assert "not live" in _lib.last_error()
    depth = ctypes.c_int32(0)
    assert lib.bst_scope_depth(987654, ctypes.byref(depth)) == _lib.BST_UNKNOWN_HANDLE


def test_invalid_specs_fail_before_touching_a_device():
    lib = _lib.load()
    bad = [ModelSpec("padded_decoder", 1, 8, 32, 1, 1, 32),       # vocabulary < 2
           ModelSpec("padded_decoder", 10, 0, 32, 1, 1, 32),      # window < 1
           ModelSpec("padded_decoder", 10, 8, 30, 1, 4, 32)]      # d % heads != 0
    for spec in bad:
        s = spec.struct()
        h = ctypes.c_uint64(0)
        assert lib.bst_engine_create(ctypes.byref(s), 0, ctypes.byref(h)) == _lib.BST_INVALID
    s = ModelSpec("padded_decoder", 10, 8, 48, 1, 3, 32).struct()  # head dim 16
    h = ctypes.c_uint64(0)
    assert lib.bst_engine_create(ctypes.byref(s), 0, ctypes.byref(h)) == _lib.BST_UNSUPPORTED


@pytest.mark.skipif(Basalt.device_count() > 0, reason="checks the no-GPU failure path")
def test_engine_creation_fails_loudly_without_a_gpu():
    from basalt_b200 import BasaltUnsupportedOperationException, TextEngine

    spec = ModelSpec("last_token", 5, 3)
    with pytest.raises(BasaltUnsupportedOperationException):
        TextEngine.of(Basalt.create(), spec, 5, 3)


def test_synthetic_prompts_follow_java_random():
    prompts = synthetic_prompts(3, 4, 10, 4096)
    r = orc.JavaRandom(3)
    want = np.array([[r.next_int(4096) for _ in range(10)] for _ in range(4)], dtype=np.int32)
    np.testing.assert_array_equal(prompts, want)


def test_synthetic_weights_follow_java_random_and_the_file_format(tmp_path):
    spec = ModelSpec("padded_decoder", 7, 4, 32, 1, 1, 16)
    path = tmp_path / "w.bin"
    write_synthetic_weights(spec, path, seed=0, stddev=0.02)
    raw = path.read_bytes()
    # TextEngine.save layout (TextEngine.java:304-315): big-endian V, W, count, then entries.
    v, w, count = struct.unpack(">iii", raw[:12])
    assert (v, w) == (7, 4)
    e = orc.OracleEngine(orc.FAMILY_PADDED_DECODER, 7, 4, 32, 1, 1, 16)
    assert count == len(e.parameters())
    name_len = struct.unpack(">H", raw[12:14])[0]
    assert raw[14:14 + name_len] == b"embedding.weight"
    n = struct.unpack(">i", raw[14 + name_len:18 + name_len])[0]
    assert n == 8 * 32
    first = struct.unpack(">f", raw[18 + name_len:22 + name_len])[0]
    assert first == np.float32(orc.JavaRandom(0).next_gaussian() * 0.02)
    # The oracle reads the same file by name; LayerNorm gains are 1 and betas 0.
    e.load(path)
    np.testing.assert_array_equal(e.get("layer0.norm1.gamma"), np.ones(32, np.float32))
    np.testing.assert_array_equal(e.get("norm.beta"), np.zeros(32, np.float32))
    # Every random parameter is one nextGaussian per element, in file order.
    r = orc.JavaRandom(0)
    for name, size in e.parameters():
        values = e.get(name)
        if "norm" in name:
            continue
        want = np.array([np.float32(r.next_gaussian() * 0.02) for _ in range(size)], np.float32)
        np.testing.assert_array_equal(values, want, err_msg=name)


def test_bf16_synthetic_weights_are_bf16_representable(tmp_path):
    spec = ModelSpec("padded_decoder", 7, 4, 32, 1, 1, 16, weight_dtype="bf16")
    path = tmp_path / "w.bin"
    write_synthetic_weights(spec, path, seed=0)
    e = orc.OracleEngine(orc.FAMILY_PADDED_DECODER, 7, 4, 32, 1, 1, 16)
    e.load(path)
    for name, _ in e.parameters():
        bits = e.get(name).view(np.uint32)
        if name.endswith(".weight"):
            assert np.all(bits & 0xFFFF == 0), name
    assert np.any(e.get("layer0.attention.query.bias").view(np.uint32) & 0xFFFF)
