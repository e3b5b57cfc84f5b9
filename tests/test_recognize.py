"""Recognition of a module from its namedParameters (torch/Module.java:27-34) without a GPU: the
decision TextEngine's dispatch makes before it hands a module to the CUDA engine
(bst_recognize_model). Parameter shapes follow the reference's layout: Linear weight [in, out] and
bias [1, out], LayerNorm gamma/beta [d], Embedding [rows, d]."""
import numpy as np
import pytest

from basalt_b200 import BasaltShapeException, BasaltUnsupportedOperationException
from basalt_b200.text_engine import IllegalArgumentException, recognize_model
from oracle import oracle as orc


def decoder_parameters(V, W, d, L, F, padded=True):
    family = orc.FAMILY_PADDED_DECODER if padded else orc.FAMILY_DECODER
    o = orc.OracleEngine(family, V, W, d, L, 1, F)

    def shape(name, size):
        if name == "embedding.weight":
            return (V + 1 if padded else V, d)
        if name == "position.weight":
            return (W, d)
        if name == "head.weight":
            return (d, V)
        if name.endswith("ffn1.weight"):
            return (d, F)
        if name.endswith("ffn2.weight"):
            return (F, d)
        if name.endswith(".weight"):
            return (d, d)
        if name.endswith(".bias"):
            return (1, size)
        return (size,)

    return [(n, np.zeros(shape(n, s), np.float32)) for n, s in o.parameters()]


def char_lm_parameters(V, W, d, h):
    flat = W * d
    shapes = [(V, d), (flat, h), (1, h), (h, flat), (1, flat), (flat, V), (1, V)]
    return [(f"param{i}", np.zeros(s, np.float32)) for i, s in enumerate(shapes)]


def test_padded_and_stock_decoders_are_told_apart_by_the_embedding_rows():
    spec = recognize_model(decoder_parameters(96, 64, 128, 2, 512), 96, 64, heads=4)
    assert (spec.family, spec.dimension, spec.layers, spec.heads, spec.hidden) == \
        ("padded_decoder", 128, 2, 4, 512)
    spec = recognize_model(decoder_parameters(50, 24, 64, 3, 128, padded=False), 50, 24, heads=2)
    assert (spec.family, spec.layers, spec.heads) == ("decoder", 3, 2)


def test_char_lm_and_last_token_head():
    spec = recognize_model(char_lm_parameters(96, 8, 16, 64), 96, 8)
    assert (spec.family, spec.dimension, spec.hidden) == ("char_lm", 16, 64)
    spec = recognize_model([("param0", np.zeros((10, 10))), ("param1", np.zeros((1, 10)))], 10, 3)
    assert spec.family == "last_token"


def test_unrecognised_or_inconsistent_modules_are_rejected():
    with pytest.raises(BasaltUnsupportedOperationException):
        recognize_model([("fc.weight", np.zeros((4, 4)))], 4, 2)
    with pytest.raises(IllegalArgumentException, match="head count"):
        recognize_model(decoder_parameters(96, 64, 128, 2, 512), 96, 64, heads=0)
    # The window TextEngine.of is given must match the position table.
    with pytest.raises(BasaltShapeException, match="window"):
        recognize_model(decoder_parameters(96, 64, 128, 2, 512), 96, 32, heads=4)
    # A missing parameter (namedParameters out of order or incomplete).
    params = decoder_parameters(96, 64, 128, 2, 512)
    with pytest.raises(BasaltShapeException):
        recognize_model(params[:-1], 96, 64, heads=4)
    # A head dimension the kernels do not serve.
    with pytest.raises(BasaltUnsupportedOperationException, match="head dimension"):
        recognize_model(params, 96, 64, heads=8)
