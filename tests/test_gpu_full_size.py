"""Full-size workloads, checked through properties that do not need the oracle to replay every
step: at sampled (row, step) points the decode-path token equals the argmax of the reference's
full-window recompute of that step's window, the GPU's own full-window scores match the oracle's,
and a row decoded inside the batch equals the row decoded alone up to a near tie."""
import numpy as np
import pytest

from basalt_b200 import TextEngine, config, left_pad, synthetic_prompts, write_synthetic_weights
from oracle import oracle as orc
from parity import ATOL, compare_logits, top2_gap

pytestmark = pytest.mark.gpu


def pair(runtime, workload, path):
    m = workload.model
    write_synthetic_weights(m, path, workload.weight_seed)
    engine = TextEngine.of(runtime, m, m.vocabulary, m.window)
    engine.load(path)
    oracle = orc.OracleEngine(orc.FAMILY_PADDED_DECODER, m.vocabulary, m.window, m.dimension,
                              m.layers, m.heads, m.hidden)
    oracle.load(path)
    return engine, oracle


def window_at(ctx_row, tokens_row, step, window):
    full = np.concatenate([ctx_row, tokens_row[:step]])
    return full[-window:]


def check_points(engine, oracle, ctx, tokens, points, window):
    for r, g in points:
        win = window_at(ctx[r], tokens[r], g, window)
        ref = oracle.scores(win)
        compare_logits(engine.scores(win), ref, where=f"row {r} step {g}")
        if int(np.argmax(ref)) != int(tokens[r, g]):
            assert top2_gap(ref) < ATOL, f"row {r} step {g}: {tokens[r, g]} vs {np.argmax(ref)}"


def first_divergence_is_a_near_tie(oracle, ctx_row, a, b, window):
    diff = np.nonzero(a != b)[0]
    if diff.size == 0:
        return True
    g = int(diff[0])
    return top2_gap(oracle.scores(window_at(ctx_row, a, g, window))) < ATOL


def test_v4096_d512_l6_batch256_greedy(runtime, tmp_path):
    w = config("v4096-d512-l6-w512-b256-greedy")
    engine, oracle = pair(runtime, w, tmp_path / "w.bin")
    W, V = w.model.window, w.model.vocabulary
    ctx = left_pad(synthetic_prompts(w.prompt_seed, w.rows, w.prompt, V), W, V)
    tokens = engine.generateBatch(ctx, w.steps)
    assert tokens.shape == (256, 256) and tokens.min() >= 0 and tokens.max() < V
    check_points(engine, oracle, ctx, tokens, [(0, 0), (0, 255), (131, 128), (255, 255)], W)
    alone = engine.generate(ctx[77], w.steps)
    assert first_divergence_is_a_near_tie(oracle, ctx[77], tokens[77], alone, W)


def test_v4096_d512_l6_batch256_greedy_bf16_weights(runtime, tmp_path):
    w = config("v4096-d512-l6-w512-b256-greedy-bf16w")
    engine, oracle = pair(runtime, w, tmp_path / "w.bin")
    W, V = w.model.window, w.model.vocabulary
    ctx = left_pad(synthetic_prompts(w.prompt_seed, w.rows, w.prompt, V), W, V)
    tokens = engine.generateBatch(ctx, w.steps)
    check_points(engine, oracle, ctx, tokens, [(3, 0), (200, 200), (255, 255)], W)


def test_v8192_d768_l12_batch1_greedy_bf16_weights(runtime, tmp_path):
    w = config("v8192-d768-l12-w1024-b1-greedy-bf16w")
    engine, oracle = pair(runtime, w, tmp_path / "w.bin")
    W, V = w.model.window, w.model.vocabulary
    ctx = left_pad(synthetic_prompts(w.prompt_seed, 1, w.prompt, V), W, V)
    tokens = engine.generateBatch(ctx, w.steps)
    check_points(engine, oracle, ctx, tokens, [(0, 0), (0, 256), (0, 511)], W)


def test_v8192_d768_l12_sampled_rows_of_the_8192_sequence_run(runtime, tmp_path):
    # The 8192-sequence streamSampled workload (T = 1.0, seed 9): its first 64 rows, decoded in
    # waves of 32, draw what the first 64 successive calls of the full run draw. Draws are
    # replayed against the oracle at sampled steps from the skip-ahead generator state.
    from dataclasses import replace

    from parity import draw_margin

    w = config("v8192-d768-l12-w1024-n8192-sampled-bf16w")
    m = replace(w.model, max_rows=32)
    w = replace(w, model=m, rows=64, steps=48)
    engine, oracle = pair(runtime, w, tmp_path / "w.bin")
    W, V = m.window, m.vocabulary
    ctx = left_pad(synthetic_prompts(w.prompt_seed, 64, w.prompt, V), W, V)
    engine.seed(w.sample_seed)
    tokens = engine.sampleBatch(ctx, w.steps, w.temperature, w.k)
    start = orc.lcg_scramble(w.sample_seed)
    for r, g in [(0, 0), (0, 47), (31, 20), (32, 5), (63, 47)]:
        state = orc.lcg_advance(start, 2 * w.steps * r + 2 * g)
        ref = oracle.scores(window_at(ctx[r], tokens[r], g, W))
        want, margin, _ = draw_margin(ref, w.temperature, w.k, state)
        assert want == tokens[r, g] or margin < 1e-4, (r, g, tokens[r, g], want)


def test_v8192_d768_l12_512_rows_greedy_bf16_weights(runtime, tmp_path):
    # 512 rows (two lanes of 256) of the 8192-sequence run's architecture: its decode projections
    # have between one and two work units per SM (e.g. the QKV GEMM: 72 tiles x 3 splits), the
    # case served by the two-CTAs-per-SM ring of the one-tile GEMM.
    from dataclasses import replace

    w = config("v8192-d768-l12-w1024-n8192-sampled-bf16w")
    m = replace(w.model, max_rows=0)
    w = replace(w, model=m, rows=512, steps=4, mode="greedy")
    engine, oracle = pair(runtime, w, tmp_path / "w.bin")
    W, V = m.window, m.vocabulary
    ctx = left_pad(synthetic_prompts(w.prompt_seed, 512, w.prompt, V), W, V)
    tokens = engine.generateBatch(ctx, w.steps)
    assert tokens.shape == (512, 4) and tokens.min() >= 0 and tokens.max() < V
    check_points(engine, oracle, ctx, tokens, [(0, 0), (300, 3), (511, 3)], W)
