"""Device tensors and the op queue on Device.cuda(0), through the C ABI.

NativeTestSuite's queue and matmul cases (NativeTestSuite.java:60-111) with the tensors on the
GPU: the queued add/relu/mul of a [2, 3] tensor and a broadcast [3] bias must give
[110, 440, 990, 140, 500, 1080] and record three graph nodes, and matmul of the suite's shapes must
match the reference product within 2e-4. Transfers between the host (tag 0) and cuda:0 (tag 1000)
are real copies; every other op is checked against the oracle's restatement of ops.rs/nn_ops.rs.
"""
import numpy as np
import pytest

from basalt_b200 import BasaltShapeException, BasaltUnsupportedOperationException
from basalt_b200.tensors import (CPU_TAG, OP_ABS, OP_EXP, OP_LOG, OP_NEG, OP_SQRT,
                                 CommandQueueBuilder, CudaContext, cuda_tag, pack_command)
from basalt_b200.text_engine import IllegalStateException
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture()
def context(runtime):
    with CudaContext(runtime.device) as c:
        yield c


def test_queued_add_relu_mul_matches_the_native_suite(context):
    a = context.of([1, 2, 3, 4, 5, 6], 2, 3)
    bias = context.of([10, 20, 30], 3)
    total, activated, scaled = (context.zeros(2, 3) for _ in range(3))
    CommandQueueBuilder(context).add(a, bias, total).relu(total, activated) \
        .mul(activated, bias, scaled).execute()
    np.testing.assert_allclose(scaled.data(), [110, 440, 990, 140, 500, 1080], rtol=1e-4)
    assert context.graphSize() == 3
    assert scaled.device_tag() == cuda_tag(context.device)


def test_matmul_shapes_of_the_native_suite(context):
    rng = orc.JavaRandom(11)
    for m, k, n in [(1, 1, 1), (2, 3, 4), (7, 9, 11), (16, 17, 13), (33, 31, 9), (128, 96, 40)]:
        left = np.array([rng.next_float() * 2 - 1 for _ in range(m * k)], np.float32)
        right = np.array([rng.next_float() * 2 - 1 for _ in range(k * n)], np.float32)
        a, b, c = context.of(left, m, k), context.of(right, k, n), context.zeros(m, n)
        CommandQueueBuilder(context).matMul(a, b, c).execute()
        want = orc.matmul(left.reshape(m, k), right.reshape(k, n)).ravel()
        np.testing.assert_allclose(c.data(), want, rtol=2e-4, atol=2e-4 * np.abs(want).max())


def test_elementwise_ops_follow_the_oracle(context):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((4, 5, 6)).astype(np.float32)
    y = (rng.standard_normal((5, 6)) + 3.0).astype(np.float32)
    tx, ty = context.of(x, 4, 5, 6), context.of(y, 5, 6)
    outs = {name: context.zeros(4, 5, 6) for name in ("add", "sub", "mul", "div")}
    q = CommandQueueBuilder(context)
    q.add(tx, ty, outs["add"]).sub(tx, ty, outs["sub"]).mul(tx, ty, outs["mul"])
    q.div(tx, ty, outs["div"]).execute()
    np.testing.assert_array_equal(outs["add"].data(), orc.add(x, y).ravel())
    np.testing.assert_array_equal(outs["mul"].data(), orc.mul(x, y).ravel())
    np.testing.assert_array_equal(outs["sub"].data(), (x - y).ravel())
    np.testing.assert_array_equal(outs["div"].data(), (x / y).ravel())
    pos = np.abs(x) + 0.5
    tp = context.of(pos, 4, 5, 6)
    unary = {"relu": context.zeros(4, 5, 6), "gelu": context.zeros(4, 5, 6),
             "sigmoid": context.zeros(4, 5, 6), "tanh": context.zeros(4, 5, 6)}
    q = CommandQueueBuilder(context)
    q.relu(tx, unary["relu"]).gelu(tx, unary["gelu"]).sigmoid(tx, unary["sigmoid"])
    q.tanh(tx, unary["tanh"]).execute()
    np.testing.assert_array_equal(unary["relu"].data(), orc.relu(x).ravel())
    np.testing.assert_allclose(unary["gelu"].data(), orc.gelu(x).ravel(), rtol=2e-6, atol=1e-7)
    sig = np.where(x >= 0, 1 / (1 + np.exp(-x.astype(np.float64))),
                   np.exp(x.astype(np.float64)) / (1 + np.exp(x.astype(np.float64))))
    np.testing.assert_allclose(unary["sigmoid"].data(), sig.ravel(), rtol=2e-6)
    np.testing.assert_allclose(unary["tanh"].data(), np.tanh(x).ravel(), rtol=2e-6, atol=1e-7)
    for op, ref in [(OP_EXP, np.exp), (OP_LOG, np.log), (OP_SQRT, np.sqrt), (OP_ABS, np.abs),
                    (OP_NEG, np.negative)]:
        out = context.zeros(4, 5, 6)
        CommandQueueBuilder(context).unary(op, tp, out).execute()
        np.testing.assert_allclose(out.data(), ref(pos.astype(np.float64)).ravel(), rtol=2e-6)


def test_transfers_are_real_copies_between_host_and_device(context):
    values = np.arange(12, dtype=np.float32)
    host = context.of(values, 3, 4, device_tag=CPU_TAG)
    on_gpu = context.transferTensor(host, cuda_tag(context.device))
    assert on_gpu.device_tag() == cuda_tag(context.device) and on_gpu.shape() == (3, 4)
    host.setData(np.zeros(12))               # the copy does not alias its source
    np.testing.assert_array_equal(on_gpu.data(), values)
    doubled = context.zeros(3, 4)
    CommandQueueBuilder(context).add(on_gpu, on_gpu, doubled).execute()
    back = context.transferTensor(doubled, CPU_TAG)
    assert back.device_tag() == CPU_TAG
    np.testing.assert_array_equal(back.data(), 2 * values)
    # Ops do not run on host tensors, and a foreign CUDA device is not this context's.
    with pytest.raises(BasaltUnsupportedOperationException):
        CommandQueueBuilder(context).relu(back, context.zeros(3, 4)).execute()
    with pytest.raises(BasaltUnsupportedOperationException):
        context.transferTensor(on_gpu, cuda_tag(context.device + 1))


def test_handles_shapes_and_release(context):
    a, b = context.of([1, 2, 3, 4], 2, 2), context.zeros(3, 3)
    with pytest.raises(BasaltShapeException):
        CommandQueueBuilder(context).add(a, b, context.zeros(2, 2)).execute()
    with pytest.raises(BasaltShapeException):
        CommandQueueBuilder(context).matMul(a, b, context.zeros(2, 3)).execute()
    record = pack_command(2, [a.handle, 0], b.handle)   # a null input
    with pytest.raises(Exception, match="input 1 of the command is null"):
        context.execute(record, 1)
    before = context.stats()["tensors"]
    assert a.close() is True and a.close() is False     # idempotent, as NativeTensorHandle.close
    assert context.stats()["tensors"] == before - 1
    with pytest.raises(IllegalStateException):
        a.data()                                        # a released handle is not reused
    with pytest.raises(BasaltUnsupportedOperationException):
        CommandQueueBuilder(context).unary(15, b, b).execute()   # Conv2d has no kernel here


def test_engine_from_named_parameters_decodes_like_the_spec_engine(runtime, tmp_path):
    from basalt_b200 import ModelSpec, TextEngine, left_pad, synthetic_prompts
    from basalt_b200 import write_synthetic_weights

    spec = ModelSpec("padded_decoder", 96, 64, 128, 2, 4, 512)
    path = tmp_path / "w.bin"
    write_synthetic_weights(spec, path, 0, 0.05)
    oracle = orc.OracleEngine(orc.FAMILY_PADDED_DECODER, 96, 64, 128, 2, 4, 512)
    oracle.load(path)
    shapes = {"embedding.weight": (97, 128), "position.weight": (64, 128),
              "head.weight": (128, 96)}
    named = []
    for name, size in oracle.parameters():
        if name in shapes:
            shape = shapes[name]
        elif name.endswith("ffn1.weight"):
            shape = (128, 512)
        elif name.endswith("ffn2.weight"):
            shape = (512, 128)
        elif name.endswith(".weight"):
            shape = (128, 128)
        elif name.endswith(".bias"):
            shape = (1, size)
        else:
            shape = (size,)
        named.append((name, oracle.get(name).reshape(shape)))
    engine = TextEngine.ofParameters(runtime, named, 96, 64, heads=4)
    assert engine.model().family == "padded_decoder"
    ctx = left_pad(synthetic_prompts(1, 2, 16, 96), 64, 96)
    np.testing.assert_array_equal(engine.generateBatch(ctx, 24), oracle.generate_batch(ctx, 24))
