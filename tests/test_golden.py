"""The committed golden fixtures (tests/golden/, made by make_golden.py) against the CPU
checker and, on a GPU, against the device decoder."""
import ctypes
import json
import sys
from pathlib import Path

import numpy as np
import pytest

import itts_gpt as ig
import oracle as orc

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import make_golden as mg  # noqa: E402


@pytest.fixture(scope="module")
def golden():
    z = np.load(GOLDEN / "decoder_small.npz")
    return {k: z[k] for k in z.files}


@pytest.fixture(scope="module")
def golden_weights(golden):
    w = mg.small_model()
    assert mg.weights_digest(w) == golden["weights_digest"].item().decode(), \
        "the seeded weight generator changed; regenerate the fixtures"
    return w


def test_prompt_generator_unchanged(golden):
    text, conds = mg.prompt()
    np.testing.assert_array_equal(np.asarray(text, np.int32), golden["text"])
    np.testing.assert_array_equal(conds.astype(np.float32), golden["conds"])


def test_checker_matches_golden_decoder(golden, golden_weights):
    om = orc.OracleModel(golden_weights)
    kv = om.kv(128)
    got = [om.prefill(kv, golden["text"], golden["conds"], int(golden["lang"]))]
    assert kv.valid_len() == int(golden["prefix_len"])
    for i, c in enumerate(golden["codes"]):
        got.append(om.step(kv, int(c), i + 2))
    for i, g in enumerate(got):
        np.testing.assert_allclose(g, golden["logits"][i], atol=2e-5, rtol=1e-4)


def _kat(name):
    return next(k for k in json.loads((GOLDEN / "sampler_kats.json").read_text()) if k["name"] == name)


def test_sampler_kats_penalty():
    k = _kat("repetition_penalty_on_seen_tokens")
    seen = ig.SeenTokenBitSet.new_with_initial_tokens()
    for t in k["insert"]:
        seen.insert(t)
    logits = np.zeros(k["n"], np.float32)
    for i, v in k["set"].items():
        logits[int(i)] = v
    w = np.array(seen.words, np.uint64)
    orc.lib().orc_apply_repetition_penalty(w.ctypes.data, logits.ctypes.data, k["n"], ctypes.c_float(k["penalty"]))
    for i, v in k["expected"].items():
        assert abs(logits[int(i)] - v) < k["atol"]


def test_sampler_kats_spike_seen_rng():
    k = _kat("spike_wins_with_default_params")
    logits = np.full(k["n"], k["fill"], np.float32)
    logits[k["spike_index"]] = k["spike_value"]
    seen = ig.SeenTokenBitSet.new_with_initial_tokens()
    tok, _ = orc.sample_next_token(logits, seen.words, orc.params_c(), orc.lib().orc_rng_new(k["rng_seed"]))
    assert tok == k["expected_token"]
    k = _kat("initial_seen_set")
    s = ig.SeenTokenBitSet.new_with_initial_tokens()
    assert all(s.contains(t) for t in k["expected_seen"])
    assert not any(s.contains(t) for t in k["expected_unseen"])
    k = _kat("rng_seed_mixing")
    assert orc.lib().orc_rng_new(k["seed"]) == k["expected_state"]
    assert ig.SamplerRng(k["seed"]).state == k["expected_state"]


@pytest.mark.gpu
def test_device_matches_golden_decoder(golden, golden_weights):
    """Prefill and five steps on the device against the golden logits, within the north_star
    bound (max-abs 2e-2, relative 1e-2)."""
    gpt = ig.Gpt.from_weights(golden_weights, device=0)
    try:
        kv = ig.KvCache(gpt, max_seq=128)
        got = [gpt.prefill(golden["text"], golden["conds"], int(golden["lang"]), kv)]
        for i, c in enumerate(golden["codes"]):
            got.append(gpt.step(kv, int(c), i + 2))
        for i, g in enumerate(got):
            ref = golden["logits"][i]
            err = np.abs(g - ref)
            assert err.max() <= 2e-2, (i, err.max())
            assert err.max() <= 1e-2 * np.abs(ref).max() + 2e-2
            assert int(np.argmax(g)) == int(np.argmax(ref)) or \
                ref.max() - ref[int(np.argmax(g))] <= 4e-2
    finally:
        gpt.close()


def test_reference_gpt_fixture_shapes():
    """The Stage-1 tensors extracted from the reference's golden fixture
    (crates/core/fixtures/golden_ref.safetensors) have the shapes its CP-10 / CP-11 tests
    use: conds [1, 3, 1280] (gpt.rs:549-553), 8,194 prefill logits, 32 greedy codes."""
    import numpy as np
    from pathlib import Path
    f = dict(np.load(Path(__file__).resolve().parent / "golden" / "reference_gpt_fixture.npz"))
    assert f["conds"].shape == (1, 3, 1280) and f["conds"].dtype == np.float32
    assert f["prefill_logits"].shape == (8194,) and np.isfinite(f["prefill_logits"]).all()
    assert f["greedy_codes"].shape == (32,) and ((0 <= f["greedy_codes"]) & (f["greedy_codes"] < 8193)).all()
    for i in range(6):
        t = f[f"token_ids_{i}"]
        assert t.dtype == np.int32 and 0 < t.size <= 600 and (t >= 0).all() and (t < 60510).all()
