"""On-device sampler (sample.cu) vs the CPU checker, bit for bit.

Given the same logits, seen set, parameters and SamplerRng state, the device must
return the same token, the same advanced RNG state (the draw happens exactly when
sampler.rs:274 draws) and the same penalized logits (sampler.rs:204 mutates the
slice in place)."""
import numpy as np
import pytest

import itts_gpt as ig
import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpt(small_weights):
    g = ig.Gpt.from_weights(small_weights, device=0)
    yield g
    g.close()


def _logits(rng, n, kind):
    if kind == 0:
        x = rng.normal(0, 2, n)
    elif kind == 1:
        x = rng.integers(-3, 4, n).astype(np.float64)  # heavy ties
    elif kind == 2:
        x = rng.normal(0, 0.3, n)
        x[rng.integers(0, n, 3)] = [9.0, 8.5, 8.9]
    elif kind == 3:
        x = rng.normal(0, 1, n)
        idx = rng.integers(0, n, 6)
        x[idx[0]], x[idx[1]], x[idx[2]], x[idx[3]], x[idx[4]] = np.nan, np.inf, -np.inf, -0.0, 0.0
    else:
        x = rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32).view(np.float32)
    return np.asarray(x, np.float32)


@pytest.mark.parametrize("seed", range(60))
def test_sampler_bit_exact(gpt, seed):
    rng = np.random.default_rng(1000 + seed)
    n = int(rng.choice([8194, 8194, 300, 1, 5000, 16384]))
    x = _logits(rng, n, seed % 5)
    seen = ig.SeenTokenBitSet.new_with_initial_tokens()
    for t in rng.integers(0, max(n, 1), 20):
        seen.insert(int(t))
    p = ig.SamplingParams(greedy=bool(seed % 7 == 0),
                          top_k=int(rng.choice([0, 1, 3, 30, 64, 500, 8194])),
                          top_p=float(rng.choice([0.01, 0.3, 0.8, 1.0])),
                          temperature=float(rng.choice([0.05, 0.8, 1.3, 2.0])),
                          repetition_penalty=float(rng.choice([1.0, 1.5, 10.0, 50.0])))
    state = int(rng.integers(0, 2**63))
    ref_logits = x.copy()
    ref_tok, ref_state = orc.sample_next_token(ref_logits, seen.words, orc.params_c(
        p.greedy, p.top_k, p.top_p, p.temperature, p.repetition_penalty), state)
    dev_logits = x.copy()
    r = ig.SamplerRng.from_state(state)
    tok = ig.sample_next_token(gpt, dev_logits, seen, p, r)
    assert tok == ref_tok
    assert r.state == ref_state
    # bitwise equal, except that NaN payloads may differ between host and device
    nan = np.isnan(ref_logits)
    assert np.array_equal(nan, np.isnan(dev_logits))
    assert np.array_equal(dev_logits[~nan].view(np.uint32), ref_logits[~nan].view(np.uint32))


def test_sampler_spike_kat(gpt):
    logits = np.full(8194, -10.0, np.float32)
    logits[42] = 25.0
    tok = ig.sample_next_token(gpt, logits, ig.SeenTokenBitSet.new_with_initial_tokens(),
                               ig.SamplingParams(), ig.SamplerRng(7))
    assert tok == 42  # sampler.rs:177-189


def test_sampler_sequence_of_draws(gpt):
    """A stream of 200 draws from one SamplerRng: every token and the final state match."""
    rng = np.random.default_rng(5)
    seen = ig.SeenTokenBitSet.new_with_initial_tokens()
    p = ig.SamplingParams(top_k=30, top_p=0.8, temperature=0.8, repetition_penalty=10.0)
    r = ig.SamplerRng(2024)
    st = r.state
    for _ in range(200):
        x = rng.normal(0, 1.5, 8194).astype(np.float32)
        a, b = x.copy(), x.copy()
        tok, st = orc.sample_next_token(a, seen.words, orc.params_c(False, 30, 0.8, 0.8, 10.0), st)
        assert ig.sample_next_token(gpt, b, seen, p, r) == tok
        assert r.state == st
        seen.insert(tok)


def test_sampler_validation(gpt):
    with pytest.raises(ig.ValidationError, match="logits"):
        ig.sample_next_token(gpt, np.zeros(0, np.float32), ig.SeenTokenBitSet(), ig.SamplingParams(),
                             ig.SamplerRng(0))
    with pytest.raises(ig.ValidationError, match="logits"):
        ig.sample_next_token(gpt, np.zeros(16385, np.float32), ig.SeenTokenBitSet(),
                             ig.SamplingParams(), ig.SamplerRng(0))
