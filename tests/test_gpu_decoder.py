"""Decoder parity on the GPU: the CUDA engine against the CPU oracle on seeded models.

The oracle recomputes every step's full window exactly as the reference does (no cache); the
engine decodes from its KV cache and re-encodes windows that slid past the PAD prefix. Logits are
compared step by step under teacher forcing (the oracle scores the windows the GPU produced).
"""
import numpy as np
import pytest

from basalt_b200 import (IllegalArgumentException, ModelSpec, TextEngine, config, left_pad,
                         synthetic_prompts, write_synthetic_weights)
from oracle import oracle as orc
from parity import Report, check_greedy_row, check_sampled_row, compare_logits

pytestmark = pytest.mark.gpu

FAMILY = {"padded_decoder": orc.FAMILY_PADDED_DECODER, "decoder": orc.FAMILY_DECODER}


def make_pair(runtime, spec: ModelSpec, path, seed=0, stddev=0.02):
    write_synthetic_weights(spec, path, seed, stddev)
    engine = TextEngine.of(runtime, spec, spec.vocabulary, spec.window)
    engine.load(path)
    oracle = orc.OracleEngine(FAMILY[spec.family], spec.vocabulary, spec.window, spec.dimension,
                              spec.layers, spec.heads, spec.hidden)
    oracle.load(path)
    return engine, oracle


def perturb_norms(engine, oracle, seed=1):
    """Random LayerNorm gains/biases so their handling is exercised (synthetic ones are 1/0)."""
    rng = np.random.default_rng(seed)
    for name, size in engine.parameters():
        if "norm" in name:
            base = 1.0 if name.endswith("gamma") else 0.0
            v = (base + 0.2 * rng.standard_normal(size)).astype(np.float32)
            engine.setParameter(name, v)
            oracle.set(name, v)


def assert_clean(report: Report, max_near=0):
    assert not report.mismatches, f"token mismatches: {report.mismatches[:5]}"
    assert len(report.near_ties) <= max_near, report.near_ties


def test_small_config_full_decode_with_window_saturation(runtime, tmp_path):
    # vocab 96, d 128, 2 layers, 4 heads, FFN 512, window 64: 16-token prompt, 64 greedy steps.
    # Steps 49..63 see a saturated window and are re-encoded from scratch.
    w = config("v96-d128-l2-w64-b1-greedy")
    engine, oracle = make_pair(runtime, w.model, tmp_path / "w.bin")
    prompts = synthetic_prompts(w.prompt_seed, w.rows, w.prompt, w.model.vocabulary)
    ctx = left_pad(prompts, w.model.window, w.model.vocabulary)
    tokens, logits = engine.generateWithLogits(ctx, w.steps)
    report = Report()
    check_greedy_row(oracle, ctx[0], tokens[0], logits[0], report, "row0")
    assert_clean(report)
    # Free-running oracle decode agrees token for token.
    np.testing.assert_array_equal(oracle.generate(ctx[0], w.steps), tokens[0])
    np.testing.assert_array_equal(engine.generate(ctx[0], w.steps), tokens[0])
    assert report.max_abs < 1e-4


def test_perturbed_norms_and_longer_prompt(runtime, tmp_path):
    spec = ModelSpec("padded_decoder", 96, 64, 128, 2, 4, 512)
    engine, oracle = make_pair(runtime, spec, tmp_path / "w.bin", seed=3, stddev=0.05)
    perturb_norms(engine, oracle)
    prompts = synthetic_prompts(11, 3, 40, 96)
    ctx = left_pad(prompts, 64, 96)
    tokens, logits = engine.generateWithLogits(ctx, 40)
    report = Report()
    for r in range(3):
        check_greedy_row(oracle, ctx[r], tokens[r], logits[r], report, f"row{r}")
    assert_clean(report, max_near=1)


def test_stock_decoder_recomputes_every_window(runtime, tmp_path):
    spec = ModelSpec("decoder", 50, 24, 64, 2, 2, 128)
    engine, oracle = make_pair(runtime, spec, tmp_path / "w.bin", seed=5, stddev=0.1)
    prompts = synthetic_prompts(12, 4, 30, 50)  # longer than the window: only the tail counts
    tokens, logits = engine.generateWithLogits(prompts, 20)
    report = Report()
    for r in range(4):
        check_greedy_row(oracle, prompts[r], tokens[r], logits[r], report, f"row{r}")
    assert_clean(report, max_near=1)


def test_ragged_prompts_mix_cached_and_reencoded_rows(runtime, tmp_path):
    # Rows with different PAD counts saturate at different steps, so steps mix prefill and decode
    # rows; one row starts saturated, one is all PAD (its first step scores the PAD token alone).
    spec = ModelSpec("padded_decoder", 40, 32, 64, 2, 2, 96)
    engine, oracle = make_pair(runtime, spec, tmp_path / "w.bin", seed=7, stddev=0.1)
    rng = np.random.default_rng(0)
    lengths = [1, 5, 17, 31, 32, 0, 12]
    ctx = np.full((len(lengths), 32), 40, dtype=np.int32)
    for r, n in enumerate(lengths):
        if n:
            ctx[r, 32 - n:] = rng.integers(0, 40, n)
    tokens, logits = engine.generateWithLogits(ctx, 24)
    report = Report()
    for r in range(len(lengths)):
        check_greedy_row(oracle, ctx[r], tokens[r], logits[r], report, f"row{r}")
    assert_clean(report, max_near=1)
    # Rows decoded together equal rows decoded alone.
    for r in (0, 3, 5):
        np.testing.assert_array_equal(engine.generate(ctx[r], 24), tokens[r])


def test_scores_match_the_oracle_on_batches(runtime, tmp_path):
    spec = ModelSpec("padded_decoder", 96, 64, 128, 2, 4, 512)
    engine, oracle = make_pair(runtime, spec, tmp_path / "w.bin")
    prompts = synthetic_prompts(5, 9, 64, 96)
    ctx = left_pad(prompts[:, :37], 64, 96)
    got = engine.scoresBatch(ctx)
    want = oracle.scores_batch(ctx)
    compare_logits(got, want, where="scoresBatch")
    # A context longer than the window: only the tail is used.
    longer = np.concatenate([np.zeros((9, 7), np.int32), ctx], axis=1)
    np.testing.assert_array_equal(engine.scoresBatch(longer), got)


def test_invalid_ids_are_rejected_like_the_embedding(runtime, tmp_path):
    spec = ModelSpec("padded_decoder", 20, 8, 32, 1, 1, 32)
    engine, _ = make_pair(runtime, spec, tmp_path / "w.bin")
    with pytest.raises(IllegalArgumentException, match="outside"):
        engine.generate([0, 1, 2, 3, 4, 5, 6, 21], 2)
    with pytest.raises(IllegalArgumentException, match="outside"):
        engine.generate([0, 1, 2, 3, 4, 5, 6, -1], 2)
    engine.generate([20] * 7 + [3], 2)  # PAD (= vocabulary) is a valid id


def test_bf16_weights_track_the_oracle_on_the_same_weights(runtime, tmp_path):
    # bf16-stored weights with fp32 activations and accumulation: the file holds bf16-representable
    # values, so the oracle computes on exactly the weights the GPU stores.
    spec = ModelSpec("padded_decoder", 512, 96, 256, 3, 4, 768, weight_dtype="bf16")
    engine, oracle = make_pair(runtime, spec, tmp_path / "w.bin")
    prompts = synthetic_prompts(3, 4, 48, 512)
    ctx = left_pad(prompts, 96, 512)
    tokens, logits = engine.generateWithLogits(ctx, 32)
    report = Report()
    for r in range(4):
        check_greedy_row(oracle, ctx[r], tokens[r], logits[r], report, f"row{r}")
    assert_clean(report, max_near=1)


def test_char96_batch32_greedy_subset(runtime, tmp_path):
    # vocab 96, d 256, 4 layers, 8 heads, FFN 1024, window 128; batch 32, 32-token prompts,
    # 96 greedy steps. All rows are decoded together; three rows are checked against the oracle.
    w = config("v96-d256-l4-w128-b32-greedy")
    engine, oracle = make_pair(runtime, w.model, tmp_path / "w.bin")
    prompts = synthetic_prompts(w.prompt_seed, w.rows, w.prompt, w.model.vocabulary)
    ctx = left_pad(prompts, w.model.window, w.model.vocabulary)
    tokens, logits = engine.generateWithLogits(ctx, w.steps)
    report = Report()
    for r in (0, 13, 31):
        check_greedy_row(oracle, ctx[r], tokens[r], logits[r], report, f"row{r}")
    assert_clean(report, max_near=1)
    single = engine.generate(ctx[13], w.steps)
    np.testing.assert_array_equal(single, tokens[13])


def test_char96_batch32_sampled_subset(runtime, tmp_path):
    # streamSampled at temperature 0.8, seed 7, over the same 32 prompts: the batch draws what 32
    # successive calls on one engine draw. Rows 0, 1 and 31 are replayed against the oracle.
    w = config("v96-d256-l4-w128-b32-sampled")
    engine, oracle = make_pair(runtime, w.model, tmp_path / "w.bin")
    prompts = synthetic_prompts(w.prompt_seed, w.rows, w.prompt, w.model.vocabulary)
    ctx = left_pad(prompts, w.model.window, w.model.vocabulary)
    engine.seed(w.sample_seed)
    tokens, logits = engine.sampleWithLogits(ctx, w.steps, w.temperature, w.k)
    start = orc.lcg_scramble(w.sample_seed)
    assert engine.rng_state == orc.lcg_advance(start, 2 * w.steps * w.rows)
    report = Report()
    for r in (0, 1, 31):
        state = orc.lcg_advance(start, 2 * w.steps * r)
        check_sampled_row(oracle, ctx[r], tokens[r], logits[r], w.temperature, w.k, state,
                          report, f"row{r}")
    assert_clean(report, max_near=1)
    # Free-running oracle (no teacher forcing) on row 0 reproduces the stream.
    oracle.rng_state = start
    seen = []
    np.testing.assert_array_equal(oracle.sample(ctx[0], w.steps, w.temperature, w.k,
                                                sink=seen.append), tokens[0])
    # streamSampled on the GPU delivers the same tokens in order.
    engine.seed(w.sample_seed)
    streamed = []
    out = engine.streamSampled(ctx[0], w.steps, w.temperature, w.k, streamed.append)
    np.testing.assert_array_equal(out, tokens[0])
    assert streamed == list(tokens[0])


@pytest.mark.parametrize("rows", [3, 40])
def test_greedy_selection_rules_on_crafted_head(runtime, tmp_path, rows):
    # TextEngine.argmax (TextEngine.java:392-400) on the batched path, whose head epilogue folds
    # each row's first maximum into a packed word (and on the fused step for <= 8 rows): with the
    # head weights zeroed the logits are the bias, so ties, signed zeros and NaN decide the token.
    spec = ModelSpec("padded_decoder", 50, 16, 64, 1, 2, 128)
    engine, oracle = make_pair(runtime, spec, tmp_path / "w.bin", seed=2, stddev=0.05)
    engine.setParameter("head.weight", np.zeros(64 * 50, np.float32))
    ctx = left_pad(synthetic_prompts(5, rows, 6, 50), 16, 50)
    cases = []
    tie = np.zeros(50, np.float32)
    tie[[7, 19, 33]] = 2.5                       # three equal maxima: the first wins
    cases.append((tie, 7))
    zeros = np.full(50, -1.0, np.float32)
    zeros[11] = -0.0
    zeros[4] = 0.0                               # +0 and -0 are equal: index 4 comes first
    cases.append((zeros, 4))
    nan0 = np.arange(50, dtype=np.float32)
    nan0[0] = np.nan                             # NaN at index 0 is never left
    cases.append((nan0, 0))
    nanmid = np.arange(50, dtype=np.float32)
    nanmid[49] = np.nan                          # a later NaN is never chosen
    cases.append((nanmid, 48))
    for bias, want in cases:
        engine.setParameter("head.bias", bias)
        tokens = engine.generateBatch(ctx, 2)
        assert (tokens == want).all(), (bias[:8], tokens[:, 0], want)
