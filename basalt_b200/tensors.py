"""Python mirror of NativeContext, NativeTensorHandle, Device and CommandQueueBuilder for tensors on
``Device.cuda(i)``, over the C ABI of libbasalt_cuda.so.

The reference's classes (src/main/java/basalt/nativebridge/NativeContext.java,
NativeTensorHandle.java, CommandQueueBuilder.java; src/main/java/basalt/Device.java) keep their
method names and argument meaning here: a context creates tensors (``of``, ``zeros``), moves them
between the host and its GPU (``transferTensor`` with a device tag, cpu = 0, cuda:i = 1000 + i),
reads them back (``data``) and runs packed op queues (``CommandQueueBuilder(...).add(...)
.relu(...).mul(...).execute()``). Each command is the reference's 128-byte record, so a queue built
here is byte for byte what the Java builder writes.
"""
from __future__ import annotations

import ctypes
import struct
from typing import Sequence

import numpy as np

from . import _lib
from .text_engine import _raise

CPU_TAG = 0
CUDA_BASE_TAG = 1000

# Op codes (CommandQueueBuilder.java:31-68).
OP_MATMUL, OP_ADD, OP_RELU, OP_SUB, OP_MUL, OP_SIGMOID, OP_TANH = 1, 2, 3, 4, 5, 6, 7
OP_GELU, OP_EXP, OP_LOG, OP_SQRT, OP_ABS, OP_NEG, OP_DIV = 11, 23, 24, 25, 26, 27, 28


def cuda_tag(index: int) -> int:
    """Device.cuda(index).tag() (Device.java:46-51)."""
    if not 0 <= index < 1000:
        raise ValueError(f"cuda device index out of range: {index}")
    return CUDA_BASE_TAG + index


class TensorHandle:
    """NativeTensorHandle: a tensor owned by a context; ``close`` is idempotent."""

    def __init__(self, context: "CudaContext", handle: int):
        self.context = context
        self.handle = handle

    def shape(self) -> tuple:
        tag, rank = ctypes.c_int32(0), ctypes.c_int32(0)
        dims = (ctypes.c_int64 * 8)()
        _raise(self.context._lib.bst_tensor_info(self.context.handle, self.handle,
                                                 ctypes.byref(tag), ctypes.byref(rank), dims, 8))
        return tuple(dims[i] for i in range(rank.value))

    def device_tag(self) -> int:
        tag, rank = ctypes.c_int32(0), ctypes.c_int32(0)
        _raise(self.context._lib.bst_tensor_info(self.context.handle, self.handle,
                                                 ctypes.byref(tag), ctypes.byref(rank), None, 0))
        return tag.value

    def data(self) -> np.ndarray:
        out = np.empty(int(np.prod(self.shape(), dtype=np.int64)), dtype=np.float32)
        _raise(self.context._lib.bst_tensor_read(self.context.handle, self.handle,
                                                 out.ctypes.data_as(_lib._f32p), out.size))
        return out

    def setData(self, values):
        v = np.ascontiguousarray(values, dtype=np.float32).ravel()
        _raise(self.context._lib.bst_tensor_write(self.context.handle, self.handle,
                                                  v.ctypes.data_as(_lib._f32p), v.size))

    def close(self) -> bool:
        released = ctypes.c_int32(0)
        _raise(self.context._lib.bst_tensor_release(self.context.handle, self.handle,
                                                    ctypes.byref(released)))
        return bool(released.value)


class CudaContext:
    """NativeContext bound to CUDA device ``index`` (tensors on tag 1000 + index or the host)."""

    def __init__(self, index: int = 0):
        self._lib = _lib.load()
        self.device = index
        h = ctypes.c_uint64(0)
        _raise(self._lib.bst_context_create(cuda_tag(index), ctypes.byref(h)))
        self.handle = h.value

    def of(self, values, *shape: int, device_tag: int | None = None) -> TensorHandle:
        v = np.ascontiguousarray(values, dtype=np.float32).ravel()
        return self._create(shape, v, device_tag)

    def zeros(self, *shape: int, device_tag: int | None = None) -> TensorHandle:
        return self._create(shape, None, device_tag)

    def _create(self, shape: Sequence[int], values, device_tag) -> TensorHandle:
        dims = (ctypes.c_int64 * len(shape))(*shape)
        out = ctypes.c_uint64(0)
        tag = cuda_tag(self.device) if device_tag is None else device_tag
        ptr = values.ctypes.data_as(_lib._f32p) if values is not None else None
        _raise(self._lib.bst_tensor_create(self.handle, tag, dims, len(shape), ptr,
                                           ctypes.byref(out)))
        return TensorHandle(self, out.value)

    def transferTensor(self, tensor: TensorHandle, device_tag: int) -> TensorHandle:
        out = ctypes.c_uint64(0)
        _raise(self._lib.bst_tensor_transfer(self.handle, tensor.handle, device_tag,
                                             ctypes.byref(out)))
        return TensorHandle(self, out.value)

    def execute(self, records: bytes, count: int):
        buf = ctypes.create_string_buffer(records, len(records))
        _raise(self._lib.bst_execute_queue(self.handle, buf, count))

    def stats(self) -> dict:
        out = (ctypes.c_int64 * 4)()
        _raise(self._lib.bst_context_stats(self.handle, out))
        return {"tensors": out[0], "device_bytes": out[1], "graph_nodes": out[2],
                "launches": out[3]}

    def graphSize(self) -> int:
        return self.stats()["graph_nodes"]

    def clearGraph(self):
        _raise(self._lib.bst_context_clear_graph(self.handle))

    def close(self):
        if self.handle:
            _raise(self._lib.bst_context_destroy(self.handle))
            self.handle = 0

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def pack_command(op: int, inputs: Sequence[int], output: int, attrs: Sequence[int] = (),
                 flags: int = 0) -> bytes:
    """One 128-byte record of the wire format (CommandQueueBuilder.java:12-26)."""
    ins = list(inputs) + [0] * (5 - len(inputs))
    at = list(attrs) + [0] * (16 - len(attrs))
    return struct.pack("<BB6x5QQ16i8x", op, flags, *ins, output, *at)


class CommandQueueBuilder:
    """Packs ops into one buffer and runs them with a single call (CommandQueueBuilder.java)."""

    def __init__(self, context: CudaContext):
        self.context = context
        self.records = []

    def _push(self, op, inputs, output):
        self.records.append(pack_command(op, [t.handle for t in inputs], output.handle))
        return self

    def matMul(self, a, b, out):
        return self._push(OP_MATMUL, [a, b], out)

    def add(self, a, b, out):
        return self._push(OP_ADD, [a, b], out)

    def sub(self, a, b, out):
        return self._push(OP_SUB, [a, b], out)

    def mul(self, a, b, out):
        return self._push(OP_MUL, [a, b], out)

    def div(self, a, b, out):
        return self._push(OP_DIV, [a, b], out)

    def relu(self, a, out):
        return self._push(OP_RELU, [a], out)

    def sigmoid(self, a, out):
        return self._push(OP_SIGMOID, [a], out)

    def tanh(self, a, out):
        return self._push(OP_TANH, [a], out)

    def gelu(self, a, out):
        return self._push(OP_GELU, [a], out)

    def unary(self, op: int, a, out):
        return self._push(op, [a], out)

    def execute(self):
        self.context.execute(b"".join(self.records), len(self.records))
        self.records = []
