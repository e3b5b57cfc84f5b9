"""basalt_b200 — B200 (sm_100a) decode engine behind Basalt's TextEngine.

The compute path is libbasalt_cuda.so (hand-written CUDA kernels, C ABI in
include/basalt_cuda.h); this package holds its build recipe and the Python mirror of
``basalt.infer.TextEngine``.
"""
from .text_engine import (  # noqa: F401
    Basalt,
    BasaltMemoryException,
    BasaltRuntimeException,
    BasaltShapeException,
    BasaltUnsupportedOperationException,
    IllegalArgumentException,
    IllegalStateException,
    ModelSpec,
    TextEngine,
    left_pad,
    synthetic_prompts,
    write_synthetic_weights,
)
from .configs import CONFIGS, config  # noqa: F401
