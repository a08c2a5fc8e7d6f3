"""CPU checker (oracle/itts_oracle.c) vs the reference sampler's own known answers.

Known-answer tests carried over as behaviours from
crates/core/src/models/sampler.rs (tyrchen/index-tts-rs):
  :430-454  repetition penalty 2 -> 1, 4 -> 2, -3 -> -6, unseen unchanged
  :177-189  spike at 42 with default params and SamplerRng::new(7) -> 42
  :98-107   initial seen set {1, 8192}
  :33-38    SamplerRng::new(42).next_f32() in [0, 1)
  :456-485  property: any f32 logits (NaN/inf included), any params -> id in 0..8194
and a pure-Python restatement of sample_next_token (sampler.rs:191-284) as a
second, independent implementation on small cases.
"""
import ctypes
import math

import numpy as np
import pytest

import oracle as orc

STOP = 8193


def seen_initial():
    w = np.zeros(129, np.uint64)
    orc.lib().orc_seen_initial(w.ctypes.data)
    return w


def test_seen_initial_tokens():
    w = seen_initial()
    c = lambda t: bool(orc.lib().orc_seen_contains(w.ctypes.data, t))
    assert c(1) and c(8192) and not c(100)
    e = np.zeros(129, np.uint64)
    assert not orc.lib().orc_seen_contains(e.ctypes.data, 1)


def test_repetition_penalty_kat():
    w = seen_initial()
    orc.lib().orc_seen_insert(w.ctypes.data, 10)
    orc.lib().orc_seen_insert(w.ctypes.data, 20)
    logits = np.zeros(32, np.float32)
    logits[1], logits[10], logits[20], logits[25] = 2.0, 4.0, -3.0, 4.0
    orc.lib().orc_apply_repetition_penalty(w.ctypes.data, logits.ctypes.data, 32, 2.0)
    assert abs(logits[1] - 1.0) < 1e-6
    assert abs(logits[10] - 2.0) < 1e-6
    assert abs(logits[20] + 6.0) < 1e-6
    assert abs(logits[25] - 4.0) < 1e-6


def test_spike_kat_default_params():
    logits = np.full(8194, -10.0, np.float32)
    logits[42] = 25.0
    p = orc.params_c()  # SamplingParams::default(): top_k 3, top_p 0.8, T 0.8, rep 10
    tok, _ = orc.sample_next_token(logits, seen_initial(), p, orc.lib().orc_rng_new(7))
    assert tok == 42


def test_rng_range_and_sequence():
    st = ctypes.c_uint64(orc.lib().orc_rng_new(42))
    vals = [orc.lib().orc_rng_next_f32(ctypes.byref(st)) for _ in range(1000)]
    assert all(0.0 <= v < 1.0 for v in vals)
    # the same SplitMix64 variant restated in Python
    s = (42 ^ 0x9E3779B97F4A7C15) & (2**64 - 1)
    for v in vals[:50]:
        s = (s + 0x9E3779B97F4A7C15) & (2**64 - 1)
        z = s
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & (2**64 - 1)
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & (2**64 - 1)
        z ^= z >> 31
        assert np.float32(z >> 40) * np.float32(1.0 / 16777216) == np.float32(v)


# ---------------------------------------------------------------------------
# independent pure-Python restatement of sampler.rs:191-284 (small cases only)
# ---------------------------------------------------------------------------
f32 = np.float32


def py_sample(logits, seen_words, greedy, top_k, top_p, temp, pen, state):
    lg = [f32(v) for v in logits]
    n = len(lg)
    with np.errstate(all="ignore"):
        if abs(f32(pen) - f32(1.0)) > f32(1.1920929e-7):
            for i in range(min(n, 129 * 64)):
                if (int(seen_words[i // 64]) >> (i % 64)) & 1:
                    lg[i] = lg[i] * f32(pen) if lg[i] < 0 else lg[i] / f32(pen)
        if greedy:
            best, bv = 0, -math.inf
            for i, v in enumerate(lg):
                if math.isfinite(v) and v > bv:
                    best, bv = i, v
            return best, state
        inv = f32(1.0) / f32(temp)
        cands = [(i, f32(v * inv) if math.isfinite(v) else f32(-math.inf)) for i, v in enumerate(lg)]
        k = n if top_k == 0 else min(top_k, n)
        cands.sort(key=lambda c: (-float(c[1]), c[0]))
        cands = cands[:k]
        mx = cands[0][1] if math.isfinite(cands[0][1]) else f32(0.0)
        probs = [f32(math.exp(float(f32(v - mx)))) if math.isfinite(v) else f32(0.0) for _, v in cands]
        s = f32(0.0)
        for p in probs:
            s = f32(s + p)
        if s <= 0 or not math.isfinite(s):
            return cands[0][0], state
        cum, active = f32(0.0), len(cands)
        for i, p in enumerate(probs):
            norm = f32(p / s)
            if i > 0 and cum > f32(top_p):
                active = i
                break
            cum = f32(cum + norm)
        asum = f32(0.0)
        for p in probs[:active]:
            asum = f32(asum + p)
        if asum <= 0 or not math.isfinite(asum):
            return cands[0][0], state
        st = ctypes.c_uint64(state)
        u = orc.lib().orc_rng_next_f32(ctypes.byref(st))
        draw = f32(f32(u) * asum)
        acc = f32(0.0)
        for (i, _), p in zip(cands[:active], probs[:active]):
            acc = f32(acc + p)
            if draw <= acc:
                return i, st.value
        return cands[active - 1][0], st.value


def _case(rng, n):
    kind = rng.integers(0, 4)
    if kind == 0:
        x = rng.normal(0, 2, n).astype(np.float32)
    elif kind == 1:  # ties
        x = rng.integers(-3, 4, n).astype(np.float32)
    elif kind == 2:  # peaked
        x = rng.normal(0, 0.5, n).astype(np.float32)
        x[rng.integers(0, n)] = 12.0
    else:  # specials
        x = rng.normal(0, 1, n).astype(np.float32)
        idx = rng.integers(0, n, 6)
        x[idx[0]], x[idx[1]], x[idx[2]] = np.nan, np.inf, -np.inf
        x[idx[3]] = -0.0
        x[idx[4]] = 0.0
    return x


@pytest.mark.parametrize("seed", range(40))
def test_oracle_matches_python_restatement(seed):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(64, 400))
    logits = _case(rng, n)
    seen = np.zeros(129, np.uint64)
    for t in rng.integers(0, n, 8):
        orc.lib().orc_seen_insert(seen.ctypes.data, int(t))
    greedy = bool(rng.integers(0, 5) == 0)
    top_k = int(rng.choice([0, 1, 3, 30, n + 5]))
    top_p = float(rng.choice([0.01, 0.5, 0.8, 1.0]))
    temp = float(rng.choice([0.05, 0.8, 2.0]))
    pen = float(rng.choice([1.0, 2.0, 10.0]))
    state = int(rng.integers(0, 2**63))
    exp_tok, exp_state = py_sample(logits.copy(), seen, greedy, top_k, top_p, temp, pen, state)
    lg = logits.copy()
    tok, st = orc.sample_next_token(lg, seen, orc.params_c(greedy, top_k, top_p, temp, pen), state)
    assert (tok, st) == (exp_tok, exp_state)


def test_property_always_valid_token():
    rng = np.random.default_rng(123)
    for _ in range(200):
        raw = rng.integers(0, 2**32, 8194, dtype=np.uint64).astype(np.uint32).view(np.float32).copy()
        p = orc.params_c(bool(rng.integers(0, 2)), int(rng.integers(1, 501)),
                         float(rng.uniform(0.05, 1.0)), float(rng.uniform(0.05, 2.0)),
                         float(rng.uniform(1.0, 2.5)))
        tok, _ = orc.sample_next_token(raw, seen_initial(), p, int(rng.integers(0, 2**63)))
        assert 0 <= tok < 8194


def test_exp_choice_vs_glibc_expf():
    """The checker uses the correctly rounded exp; record how often glibc's expf
    (what Rust's f32::exp calls on Linux) differs on a sample of [-88, 0]."""
    libm = ctypes.CDLL("libm.so.6")
    libm.expf.restype = ctypes.c_float
    libm.expf.argtypes = [ctypes.c_float]
    xs = -np.random.default_rng(0).uniform(0, 88, 20000).astype(np.float32)
    diff = 0
    for x in xs:
        a = np.float32(libm.expf(ctypes.c_float(x)))
        b = np.float32(orc.lib().orc_expf(ctypes.c_float(x)))
        assert abs(int(a.view(np.int32)) - int(b.view(np.int32))) <= 1  # at most 1 ulp apart
        diff += a != b
    assert diff / xs.size < 0.01
