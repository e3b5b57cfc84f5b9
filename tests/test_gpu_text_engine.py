"""TextEngineTest's cases (src/test/java/basalt/tests/TextEngineTest.java) on the CUDA engine,
with the reference's LastTokenModel fixture, plus the argument and lifecycle rules of the API."""
import json

import numpy as np
import pytest

from basalt_b200 import (BasaltShapeException, IllegalArgumentException, IllegalStateException,
                         ModelSpec, TextEngine)
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def known(golden_dir):
    return json.loads((golden_dir / "reference_known_answers.json").read_text())["text_engine"]


@pytest.fixture()
def text(runtime, known):
    V, W = known["vocabulary"], known["window"]
    engine = TextEngine.of(runtime, ModelSpec("last_token", V, W), V, W)
    yield engine
    engine.close()


def test_batching_matches_single_row_scoring(text, known):
    batch = text.scoresBatch(known["batch_contexts"])
    assert batch.shape == (3, known["vocabulary"])
    for row, ctx in enumerate(known["batch_contexts"]):
        np.testing.assert_allclose(text.scores(ctx), batch[row], atol=known["batch_tolerance"])
    oracle = orc.OracleEngine(orc.FAMILY_LAST_TOKEN, known["vocabulary"], known["window"])
    np.testing.assert_array_equal(batch, oracle.scores_batch(known["batch_contexts"]))


def test_greedy_decoding_is_deterministic_and_uses_only_the_tail(text, known):
    first = text.generate(known["greedy_context"], known["greedy_steps"])
    second = text.generate(known["greedy_context"], known["greedy_steps"])
    np.testing.assert_array_equal(first, second)
    np.testing.assert_array_equal(first, known["greedy_expected"])
    np.testing.assert_array_equal(text.generate(known["tail_context"], 1), known["tail_expected"])


def test_batched_generation_agrees_with_sequential(text, known):
    contexts = known["batched_generation_contexts"]
    steps = known["batched_generation_steps"]
    batched = text.generateBatch(contexts, steps)
    for row, ctx in enumerate(contexts):
        np.testing.assert_array_equal(text.generate(ctx, steps), batched[row])


def test_sampling_is_seeded_and_honours_top_k(text, known):
    s = known["seeded_replay"]
    text.seed(s["seed"])
    first = text.sample(s["context"], s["steps"], s["temperature"], s["top_k"])
    text.seed(s["seed"])
    np.testing.assert_array_equal(first, text.sample(s["context"], s["steps"], s["temperature"],
                                                     s["top_k"]))
    g = known["top_k_one_is_greedy"]
    text.seed(g["seed"])
    np.testing.assert_array_equal(text.generate(g["context"], g["steps"]),
                                  text.sample(g["context"], g["steps"], 1.0, 1))


def test_sampling_matches_the_oracle_draw_for_draw(text, known):
    # The fixture's logits are exact (one-hot rows of the weight), so every draw must agree.
    V, W = known["vocabulary"], known["window"]
    oracle = orc.OracleEngine(orc.FAMILY_LAST_TOKEN, V, W)
    for seed, temperature, top_k in [(7, 1.0, 2), (42, 3.0, 5), (5, 0.25, 3), (9, 10.0, 100)]:
        text.seed(seed)
        oracle.seed(seed)
        got = text.sample([0, 0, 0], 64, temperature, top_k)
        want = oracle.sample([0, 0, 0], 64, temperature, top_k)
        np.testing.assert_array_equal(got, want, err_msg=f"seed {seed} T {temperature} k {top_k}")
        assert text.rng_state == oracle.rng_state


def test_batched_sampling_equals_successive_calls(text, known):
    V, W = known["vocabulary"], known["window"]
    contexts = [[0, 0, 0], [1, 2, 3], [4, 4, 4], [2, 2, 1], [3, 0, 1]]
    text.seed(21)
    batched = text.sampleBatch(contexts, 17, 2.0, 4)
    state_after = text.rng_state
    oracle = orc.OracleEngine(orc.FAMILY_LAST_TOKEN, V, W)
    oracle.seed(21)
    for row, ctx in enumerate(contexts):
        np.testing.assert_array_equal(batched[row], oracle.sample(ctx, 17, 2.0, 4))
    assert state_after == oracle.rng_state


def test_weights_round_trip_through_disk(runtime, text, known, tmp_path):
    V, W = known["vocabulary"], known["window"]
    ctx = known["round_trip_context"]
    before = text.scores(ctx)
    path = tmp_path / "text-engine.bin"
    text.save(path)
    restored = TextEngine.of(runtime, ModelSpec("last_token", V, W), V, W)
    restored.setParameter("param0", np.zeros(V * V, np.float32))
    restored.load(path)
    np.testing.assert_allclose(restored.scores(ctx), before, atol=known["round_trip_tolerance"])
    # The oracle reads the file the engine wrote.
    oracle = orc.OracleEngine(orc.FAMILY_LAST_TOKEN, V, W)
    oracle.load(path)
    np.testing.assert_array_equal(oracle.scores(ctx), before)
    restored.close()


def test_streaming_emits_the_same_tokens_in_order(text, known):
    s = known["streaming"]
    seen = []
    streamed = text.stream(s["context"], s["steps"], seen.append)
    np.testing.assert_array_equal(text.generate(s["context"], s["steps"]), streamed)
    assert seen == list(streamed)
    ss = known["streaming_sampled"]
    sampled_seen = []
    text.seed(ss["seed"])
    sampled = text.streamSampled(ss["context"], ss["steps"], ss["temperature"], ss["top_k"],
                                 sampled_seen.append)
    text.seed(ss["seed"])
    np.testing.assert_array_equal(
        text.sample(ss["context"], ss["steps"], ss["temperature"], ss["top_k"]), sampled)
    assert sampled_seen == list(sampled)


def test_rejects_shapes_it_cannot_serve(runtime, text):
    with pytest.raises(IllegalArgumentException):
        text.scores([0, 1])
    with pytest.raises(IllegalArgumentException):
        text.generate([0, 1, 2], 0)
    with pytest.raises(IllegalArgumentException):
        text.sample([0, 1, 2], 3, 0.0, 2)
    with pytest.raises(IllegalArgumentException):
        text.sample([0, 1, 2], 3, 1.0, 0)
    with pytest.raises(IllegalArgumentException):
        text.scoresBatch([[0, 1], [0, 1, 2]])
    with pytest.raises(IllegalArgumentException):
        TextEngine.of(runtime, ModelSpec("last_token", 1, 3), 1, 3)
    with pytest.raises(IllegalArgumentException):
        text.sample([0, 1, 2], 3, float("nan"), 2)


def test_sink_exceptions_stop_the_call(text):
    def sink(token):
        raise KeyError("stop")

    with pytest.raises(KeyError):
        text.stream([0, 0, 0], 5, sink)
    np.testing.assert_array_equal(text.generate([0, 0, 0], 2), [1, 2])  # engine still usable


def test_loading_a_mismatched_model_fails_by_name(runtime, text, tmp_path):
    path = tmp_path / "other.bin"
    other = TextEngine.of(runtime, ModelSpec("last_token", 6, 3), 6, 3)
    other.save(path)
    with pytest.raises(IllegalStateException):
        text.load(path)  # TextEngine.load: saved vocabulary/window differ
    other.close()
    with pytest.raises(BasaltShapeException):
        text.setParameter("param0", np.zeros(3, np.float32))
    with pytest.raises(IllegalArgumentException):
        text.setParameter("nope", np.zeros(3, np.float32))


def test_scopes_release_device_buffers(text):
    base = text.stats()
    assert base["graph_nodes"] == 0
    text.beginScope()
    assert text.scopeDepth() == 1
    text.generate([0, 0, 0], 8)
    inside = text.stats()
    assert inside["bytes"] > base["bytes"]
    released = text.endScope()
    assert released >= 1
    assert text.scopeDepth() == 0
    after = text.stats()
    assert after["bytes"] < inside["bytes"]
    assert after["launches"] > base["launches"]
    with pytest.raises(IllegalStateException):
        text.endScope()


def test_closed_engines_are_unknown_handles(runtime):
    from basalt_b200 import _lib

    engine = TextEngine.of(runtime, ModelSpec("last_token", 5, 3), 5, 3)
    handle = engine.handle
    engine.close()
    assert _lib.load().bst_engine_destroy(handle) == _lib.BST_UNKNOWN_HANDLE
    assert _lib.load().bst_seed(handle, 1) == _lib.BST_UNKNOWN_HANDLE
