"""The persistent decode-step kernel (greedy, up to 8 rows) against the oracle and against the
kernel-per-operation path on the same engine.

Greedy decode steps of at most 8 rows run as one cooperative kernel; BST_FUSED_DECODE=0 switches
an engine back to one kernel per operation. Both must reproduce the oracle's logits under teacher
forcing; their tokens agree except where the oracle's top-2 gap is a near tie.
"""
import os

import numpy as np
import pytest

from basalt_b200 import ModelSpec, TextEngine, left_pad, synthetic_prompts, write_synthetic_weights
from oracle import oracle as orc
from parity import ATOL, Report, check_greedy_row, compare_logits, top2_gap

pytestmark = pytest.mark.gpu


def make_pair(runtime, spec, path, seed=0, stddev=0.05):
    write_synthetic_weights(spec, path, seed, stddev)
    engine = TextEngine.of(runtime, spec, spec.vocabulary, spec.window)
    engine.load(path)
    family = {"padded_decoder": orc.FAMILY_PADDED_DECODER, "decoder": orc.FAMILY_DECODER}
    oracle = orc.OracleEngine(family[spec.family], spec.vocabulary, spec.window, spec.dimension,
                              spec.layers, spec.heads, spec.hidden)
    oracle.load(path)
    return engine, oracle


def perturb_norms(engine, oracle, seed=5):
    rng = np.random.default_rng(seed)
    for name, size in engine.parameters():
        if "norm" in name:
            base = 1.0 if name.endswith("gamma") else 0.0
            v = (base + 0.2 * rng.standard_normal(size)).astype(np.float32)
            engine.setParameter(name, v)
            oracle.set(name, v)


def run(engine, ctx, steps, fused: bool):
    old = os.environ.get("BST_FUSED_DECODE")
    os.environ["BST_FUSED_DECODE"] = "1" if fused else "0"
    try:
        engine.profile_reset()
        engine.profile(True)
        tokens, logits = engine.generateWithLogits(ctx, steps)
        prof = engine.profile_read()
        engine.profile(False)
    finally:
        if old is None:
            del os.environ["BST_FUSED_DECODE"]
        else:
            os.environ["BST_FUSED_DECODE"] = old
    return tokens, logits, prof


CASES = [
    # (vocabulary, window, dimension, layers, heads, hidden, weight dtype, kv dtype, rows)
    (96, 64, 128, 2, 4, 512, "f32", "f32", 1),        # head_dim 32
    (128, 48, 256, 2, 4, 1024, "f32", "f32", 3),      # head_dim 64
    (200, 40, 256, 2, 2, 768, "f32", "f32", 8),       # head_dim 128, 8 rows
    (512, 96, 256, 3, 4, 768, "bf16", "f32", 2),      # bf16 weights
    (512, 96, 256, 2, 4, 768, "f32", "bf16", 5),      # bf16 cache
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"v{c[0]}-d{c[2]}-h{c[4]}-{c[6]}w-{c[7]}kv-r{c[8]}")
def test_fused_step_matches_oracle_and_unfused_path(runtime, tmp_path, case):
    V, W, d, L, H, F, wdt, kvdt, rows = case
    spec = ModelSpec("padded_decoder", V, W, d, L, H, F,
                     weight_dtype="bf16" if wdt == "bf16" else "f32",
                     kv_dtype="bf16" if kvdt == "bf16" else "f32")
    engine, oracle = make_pair(runtime, spec, tmp_path / "w.bin")
    perturb_norms(engine, oracle)
    prompt = W // 3
    steps = W - prompt + 6  # the last steps see a saturated window (re-encoded, not fused)
    ctx = left_pad(synthetic_prompts(11, rows, prompt, V), W, V)
    tokens, logits, prof = run(engine, ctx, steps, fused=True)
    assert prof.get("decode_step", {}).get("launches", 0) > 0, prof
    assert "attn_decode" not in prof, prof
    ref_tokens, ref_logits, ref_prof = run(engine, ctx, steps, fused=False)
    assert "decode_step" not in ref_prof and ref_prof["attn_decode"]["launches"] > 0

    lossy = wdt == "bf16" or kvdt == "bf16"
    if not lossy:
        report = Report()
        for r in range(rows):
            check_greedy_row(oracle, ctx[r], tokens[r], logits[r], report, f"row{r}")
        assert not report.mismatches, report.mismatches[:3]
        assert len(report.near_ties) <= 1
    # Against the unfused path (same weights and dtypes): logits within the fp32 tolerance
    # wherever the tokens so far agree; any divergence starts at a near tie.
    for r in range(rows):
        diff = np.nonzero(tokens[r] != ref_tokens[r])[0]
        upto = int(diff[0]) if diff.size else steps
        compare_logits(logits[r, :upto + (1 if diff.size else 0)],
                       ref_logits[r, :upto + (1 if diff.size else 0)], where=f"row{r}")
        if diff.size:
            assert top2_gap(ref_logits[r, upto]) < ATOL, (r, upto)


def test_fused_step_batch1_long_context_many_chunks(runtime, tmp_path):
    # Window 600: up to 19 chunks of 32 keys per (row, head), merged through the tickets.
    spec = ModelSpec("padded_decoder", 300, 600, 128, 2, 4, 512)
    engine, oracle = make_pair(runtime, spec, tmp_path / "w.bin", seed=2)
    ctx = left_pad(synthetic_prompts(3, 1, 500, 300), 600, 300)
    tokens, logits, prof = run(engine, ctx, 60, fused=True)
    assert prof["decode_step"]["launches"] == 59
    ref = oracle.forced_scores(ctx[0], tokens[0])
    compare_logits(logits[0], ref, where="row0")
    for step in range(60):
        if int(np.argmax(ref[step])) != tokens[0, step]:
            assert top2_gap(ref[step]) < ATOL


def test_fused_step_repeats_exactly(runtime, tmp_path):
    # The fused step sums in a fixed order: two runs give identical logits bit for bit.
    spec = ModelSpec("padded_decoder", 128, 64, 256, 2, 4, 1024)
    engine, _ = make_pair(runtime, spec, tmp_path / "w.bin", seed=9)
    ctx = left_pad(synthetic_prompts(4, 4, 20, 128), 64, 128)
    a_tokens, a_logits, _ = run(engine, ctx, 30, fused=True)
    b_tokens, b_logits, _ = run(engine, ctx, 30, fused=True)
    np.testing.assert_array_equal(a_tokens, b_tokens)
    np.testing.assert_array_equal(a_logits, b_logits)


def test_stock_decoder_family_never_uses_the_cache_step(runtime, tmp_path):
    # The stock decoder re-encodes every window (no cache), so it has no decode steps to fuse.
    spec = ModelSpec("decoder", 64, 16, 64, 2, 2, 128)
    engine, oracle = make_pair(runtime, spec, tmp_path / "w.bin", seed=1)
    ctx = synthetic_prompts(2, 2, 16, 64)
    tokens, logits, prof = run(engine, ctx, 12, fused=True)
    assert "decode_step" not in prof
    report = Report()
    for r in range(2):
        check_greedy_row(oracle, ctx[r], tokens[r], logits[r], report, f"row{r}")
    assert not report.mismatches


@pytest.mark.parametrize("code,words", [(11, "grid barrier"), (12, "weight staging"),
                                        (3, "tensor-core GEMM")])
def test_a_recorded_pipeline_error_stops_the_run_before_the_sink(runtime, tmp_path, code, words):
    # Host-side injection: the run's status word starts out set, as a kernel that gave up on a
    # bounded wait leaves it (no kernel is made to fail). Every fused step of the run then returns
    # at entry, the call fails with BST_PANIC after the first step, the token sink never sees a
    # token, and the engine decodes normally afterwards.
    import time

    from basalt_b200 import BasaltRuntimeException

    spec = ModelSpec("padded_decoder", 96, 64, 128, 2, 4, 512)
    engine, oracle = make_pair(runtime, spec, tmp_path / "w.bin")
    ctx = left_pad(synthetic_prompts(1, 1, 16, 96), 64, 96)
    want = oracle.generate(ctx[0], 48)
    seen = []
    os.environ["BST_INJECT_PIPELINE_ERROR"] = str(code)
    try:
        start = time.perf_counter()
        with pytest.raises(BasaltRuntimeException) as info:
            engine.stream(ctx[0], 48, seen.append)
        elapsed = time.perf_counter() - start
    finally:
        del os.environ["BST_INJECT_PIPELINE_ERROR"]
    assert info.value.code == -6 and words in str(info.value)
    assert seen == []
    assert elapsed < 5.0
    np.testing.assert_array_equal(engine.generate(ctx[0], 48), want)
