"""Named decode workloads: synthetic seeded models and prompts.

Every workload uses the padded decoder (see ``ModelSpec``) with parameters N(0, 0.02) drawn by
``java.util.Random(0).nextGaussian`` (LayerNorm gamma 1, beta 0) and prompts of
``java.util.Random(prompt_seed).nextInt(V)`` ids, left-padded with PAD = V to the window.
"""
from __future__ import annotations

from dataclasses import dataclass, replace

from .text_engine import ModelSpec


@dataclass(frozen=True)
class Workload:
    name: str
    model: ModelSpec
    rows: int
    prompt: int
    steps: int
    prompt_seed: int
    weight_seed: int = 0
    mode: str = "greedy"          # "greedy" or "sample"
    temperature: float = 1.0
    top_k: int = 0                # 0: the whole vocabulary
    sample_seed: int = 0

    @property
    def k(self) -> int:
        return self.top_k or self.model.vocabulary


def _decoder(V, d, L, H, F, W, wdt="f32", kvdt="f32", max_rows=0):
    return ModelSpec("padded_decoder", V, W, d, L, H, F, wdt, kvdt, max_rows)


_C1 = _decoder(96, 128, 2, 4, 512, 64)
_C2 = _decoder(96, 256, 4, 8, 1024, 128)
_C3 = _decoder(4096, 512, 6, 8, 2048, 512)
_C4 = _decoder(8192, 768, 12, 12, 3072, 1024, "bf16")

CONFIGS = {
    w.name: w
    for w in [
        Workload("v96-d128-l2-w64-b1-greedy", _C1, rows=1, prompt=16, steps=64, prompt_seed=1),
        Workload("v96-d256-l4-w128-b32-greedy", _C2, rows=32, prompt=32, steps=96, prompt_seed=2),
        Workload("v96-d256-l4-w128-b32-sampled", _C2, rows=32, prompt=32, steps=96, prompt_seed=2,
                 mode="sample", temperature=0.8, sample_seed=7),
        Workload("v4096-d512-l6-w512-b256-greedy", _C3, rows=256, prompt=256, steps=256,
                 prompt_seed=3),
        Workload("v4096-d512-l6-w512-b256-greedy-bf16w", replace(_C3, weight_dtype="bf16"),
                 rows=256, prompt=256, steps=256, prompt_seed=3),
        Workload("v8192-d768-l12-w1024-b1-greedy-bf16w", _C4, rows=1, prompt=512, steps=512,
                 prompt_seed=4),
        # 8192 sequences in waves of 2048 rows (~97 GB of fp32 cache at 640 slots): 10 % more
        # tokens/s than waves of 1024 on one B200, measured.
        Workload("v8192-d768-l12-w1024-n8192-sampled-bf16w", replace(_C4, max_rows=2048),
                 rows=8192, prompt=128, steps=512, prompt_seed=5, mode="sample",
                 temperature=1.0, sample_seed=9),
    ]
}


def config(name: str) -> Workload:
    return CONFIGS[name]
