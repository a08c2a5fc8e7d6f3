"""Teacher-forced replay on the device (itts_gpt_teacher_forced,
itts_gpt_alignment_attention) against the CPU checker: per-code log-probabilities within
the logits bound of the decoder (2e-2), alignment attention probabilities within 2e-3."""
import numpy as np
import pytest

import itts_gpt as ig
import oracle as orc
from itts_gpt.synth import ModelConfig, make_conds, make_text, make_weights

pytestmark = pytest.mark.gpu

CFG6 = ModelConfig(n_layers=6, d=768, ff=3072, text_vocab=500)
LP_TOL, MAP_TOL = 2e-2, 2e-3


@pytest.fixture(scope="module")
def m6():
    w = make_weights(CFG6, seed=5, ln_beta_std=0.02)
    g = ig.Gpt.from_weights(w, device=0)
    yield g, orc.OracleModel(w), w
    g.close()


@pytest.mark.parametrize("n_codes", [7, 40])
def test_teacher_forced_matches_checker(m6, n_codes):
    gpt, om, _ = m6
    rng = np.random.default_rng(n_codes)
    text = make_text(9, CFG6.text_vocab, seed=3)
    conds = make_conds(CFG6.d, 3, seed=4)
    codes = [int(c) for c in rng.integers(0, 8194, n_codes)]
    kv = ig.KvCache(gpt, max_seq=256, max_batch=2)
    tf = gpt.teacher_forced(text, conds, 1, codes, kv, slot=1)
    q0 = 3 + len(text) + 2
    lp, maps = om.replay(om.kv(256), text, conds, 1, codes[:-1], q0, 0, codes, True)
    assert tf.log_probs.shape == (n_codes,) and tf.attention.shape == (n_codes, len(text) + 2)
    np.testing.assert_allclose(tf.log_probs, lp, atol=LP_TOL)
    np.testing.assert_allclose(tf.attention, maps, atol=MAP_TOL)
    np.testing.assert_allclose(tf.attention.sum(1), maps.sum(1), atol=MAP_TOL)
    assert kv.valid_len(1) == 0  # scratch slot left reset
    np.testing.assert_array_equal(gpt.code_log_probs(text, conds, 1, codes, kv, slot=1), tf.log_probs)


def test_alignment_attention_matches_checker(m6):
    gpt, om, _ = m6
    text = make_text(14, CFG6.text_vocab, seed=8)
    conds = make_conds(CFG6.d, 32, seed=9)
    prior = [11, 2000, 7]
    codes = [5, 77, 8000, 3, 8191, 12, 40, 41, 42]
    kv = ig.KvCache(gpt, max_seq=256)
    got = gpt.alignment_attention(text, conds, 2, prior, codes, kv)
    q0 = 32 + len(text) + 2 + len(prior)
    _, maps = om.replay(om.kv(256), text, conds, 2, prior + codes[:-1], q0, 1, (), True)
    assert got.shape == (len(codes), len(text) + 2)
    np.testing.assert_allclose(got, maps, atol=MAP_TOL)


def test_replay_validation(m6, small_weights):
    gpt, _, _ = m6
    kv = ig.KvCache(gpt, max_seq=256)
    text, conds = make_text(5, CFG6.text_vocab, seed=1), make_conds(CFG6.d, 3, seed=2)
    with pytest.raises(ig.ValidationError, match="codes must not be empty"):
        gpt.teacher_forced(text, conds, 1, [], kv)
    with pytest.raises(ig.ValidationError, match="codes"):
        gpt.code_log_probs(text, conds, 1, [5, 9000], kv)
    # a model without the alignment heads still scores codes, but has no attention to give
    small = ig.Gpt.from_weights(small_weights, device=0)
    try:
        skv = ig.KvCache(small, max_seq=128)
        st, sc = make_text(6, 500, seed=3), make_conds(small.d, 3, seed=4)
        with pytest.raises(ig.ValidationError, match="alignment heads"):
            small.teacher_forced(st, sc, 1, [1, 2, 3], skv)
        lp = small.code_log_probs(st, sc, 1, [1, 2, 3], skv)
        ref, _ = orc.OracleModel(small_weights).replay(orc.OracleModel(small_weights).kv(128), st, sc, 1, [1, 2],
                                                      3 + 6 + 2, 0, [1, 2, 3], False)
        np.testing.assert_allclose(lp, ref, atol=LP_TOL)
    finally:
        small.close()
