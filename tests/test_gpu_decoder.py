"""B200 decoder (through the C ABI) vs the CPU checker.

Tolerances are the ones the task states for this path: teacher-forced logits within
max-abs 2e-2 and relative 1e-2 (max |diff| / max |ref|) per step; greedy tokens agree
on at least 99% of steps; sampling bit-exact given the same logits and uniform draws
(test_gpu_sampler.py)."""
import numpy as np
import pytest

import itts_gpt as ig
import oracle as orc
from itts_gpt.synth import ModelConfig, make_conds, make_text, make_weights, save_safetensors

pytestmark = pytest.mark.gpu

ATOL = 2e-2
RTOL = 1e-2


def check_logits(got, ref, what=""):
    err = float(np.max(np.abs(got - ref)))
    rel = err / max(float(np.max(np.abs(ref))), 1e-12)
    assert err <= ATOL and rel <= RTOL, f"{what}: max abs {err:.3e}, rel {rel:.3e}"
    return err


@pytest.fixture(scope="module")
def small(small_weights):
    g = ig.Gpt.from_weights(small_weights, device=0)
    yield g, orc.OracleModel(small_weights)
    g.close()


def test_prefill_matches_checker(small, small_cfg):
    gpt, om = small
    for n_text, n_conds, lang, prior in ((1, 3, 0, []), (17, 3, 1, []), (64, 32, 5, [])
                                         , (40, 32, 1, [3, 900, 8191])):
        text = make_text(n_text, small_cfg.text_vocab, seed=n_text)
        conds = make_conds(small_cfg.d, n_conds, seed=n_conds)
        kv = ig.KvCache(gpt, max_seq=512)
        got = gpt.prefill_after(text, conds, lang, prior, kv)
        ref = om.prefill(om.kv(512), text, conds, lang, prior)
        check_logits(got, ref, f"prefill T={n_conds + n_text + 3 + len(prior)}")
        assert kv.valid_len() == n_conds + n_text + 3 + len(prior)


def _teacher_forced(gpt, om, cfg, n_text, n_conds, steps, seed, max_seq=1024):
    text = make_text(n_text, cfg.text_vocab, seed=seed)
    conds = make_conds(cfg.d, n_conds, seed=seed + 1)
    codes = np.random.default_rng(seed).integers(0, 8192, steps).tolist()
    kv = ig.KvCache(gpt, max_seq=max_seq)
    okv = om.kv(max_seq)
    g = [gpt.prefill(text, conds, 1, kv)]
    r = [om.prefill(okv, text, conds, 1)]
    for i, c in enumerate(codes):
        g.append(gpt.step(kv, c, i + 2))
        r.append(om.step(okv, c, i + 2))
    assert kv.valid_len() == okv.valid_len()
    return np.stack(g), np.stack(r)


# batch-1 decode kernels: the default clustered all-SM kernel and the persistent grid-wide
# kernel (ITTS_XK=0)
KERNELS = {"xk": ({}, "xk_decode_kernel"), "grid": ({"ITTS_XK": "0"}, "mk_decode_kernel")}


def _use_kernel(monkeypatch, gpt, name):
    env, want = KERNELS[name]
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    assert ig.KvCache(gpt, max_seq=64).decode_kernel(1) == want


def test_decode_kernel_selection(small, monkeypatch):
    gpt, _ = small
    kv4 = ig.KvCache(gpt, max_seq=256, max_batch=8)
    assert kv4.decode_kernel(1) == "xk_decode_kernel"
    assert kv4.decode_kernel(2) == "xk_decode_kernel"  # (one launch per column up to 4 columns)
    assert kv4.decode_kernel(4) == "xk_decode_kernel"
    assert kv4.decode_kernel(5) == "gemm path"
    for name in KERNELS:
        with monkeypatch.context() as mp:
            _use_kernel(mp, gpt, name)


@pytest.mark.parametrize("kernel", list(KERNELS))
@pytest.mark.parametrize("n_text,steps", [(52, 70), (140, 60)])
def test_teacher_forced_across_kv_tiles(small, small_cfg, monkeypatch, kernel, n_text, steps):
    """Decode steps whose KV length crosses 84-position K/V tiles (the tile of the cluster
    kernels; for 4 heads on many CTAs their attention ranges have idle CTAs between a
    head's), on every batch-1 decode kernel."""
    gpt, om = small
    _use_kernel(monkeypatch, gpt, kernel)
    g, r = _teacher_forced(gpt, om, small_cfg, n_text, 3, steps, seed=n_text)
    for i in range(len(g)):
        check_logits(g[i], r[i], f"step {i}")


def test_teacher_forced_steps_small(small, small_cfg):
    gpt, om = small
    g, r = _teacher_forced(gpt, om, small_cfg, 20, 3, 40, seed=3)
    for i in range(len(g)):
        check_logits(g[i], r[i], f"step {i}")
    agree = np.mean(np.argmax(g, 1) == np.argmax(r, 1))
    assert agree >= 0.99


def test_step_batch_equals_single_steps(small, small_cfg):
    gpt, _ = small
    kv = ig.KvCache(gpt, max_seq=256, max_batch=5)
    texts = [make_text(n, small_cfg.text_vocab, seed=n) for n in (3, 30, 9, 50, 12)]
    conds = make_conds(small_cfg.d, 3, seed=1)
    for s, t in enumerate(texts):
        gpt.prefill(t, conds, 1, kv, slot=s)
    slots = [4, 0, 2]
    out = gpt.step_batch(kv, slots, [7, 8, 9], [2, 2, 2])
    for j, s in enumerate(slots):
        kv1 = ig.KvCache(gpt, max_seq=256)
        gpt.prefill(texts[s], conds, 1, kv1)
        one = gpt.step(kv1, [7, 8, 9][j], 2)
        np.testing.assert_allclose(out[j], one, atol=1e-4, rtol=1e-4)
    assert [kv.valid_len(s) for s in range(5)] == [3 + t.size + 3 + (s in slots) for s, t in enumerate(texts)]


def test_generate_greedy_matches_checker(small, small_cfg):
    gpt, om = small
    text = make_text(25, small_cfg.text_vocab, seed=9)
    conds = make_conds(small_cfg.d, 32, seed=10)
    kv = ig.KvCache(gpt, max_seq=512)
    p = ig.SamplingParams(greedy=True, max_mel_tokens=64)
    codes = ig.generate_codes(gpt, text, conds, 1, kv, p, ig.SamplerRng(0))
    ref, _ = om.generate(om.kv(512), text, conds, 1, orc.params_c(greedy=True, max_mel_tokens=64), 0)
    n = min(len(codes), len(ref))
    agree = np.mean(np.array(codes[:n]) == np.array(ref[:n])) if n else 1.0
    assert agree >= 0.99 and len(codes) == len(ref)


def test_generate_sampled_matches_checker(small, small_cfg):
    """Sampled generation (T 0.8, top-k 30, top-p 0.8, rep 10).  The device logits differ from
    the checker's by ~1e-3 (fp16 activations), so a draw that lands within that margin of a
    cumulative-probability boundary may pick the neighbouring candidate; after that the two
    sequences legitimately diverge.  So the check is teacher-forced: along the device's code
    path, the checker's sampler (its own logits, the same SamplerRng stream) must choose the
    device's token on >= 95% of steps, and both must consume the same number of draws."""
    gpt, om = small
    text = make_text(30, small_cfg.text_vocab, seed=12)
    conds = make_conds(small_cfg.d, 3, seed=13)
    kv = ig.KvCache(gpt, max_seq=512)
    n = 48
    p = ig.SamplingParams(top_k=30, top_p=0.8, temperature=0.8, repetition_penalty=10.0,
                          max_mel_tokens=n)
    r = ig.SamplerRng(77)
    codes = ig.generate_codes_after(gpt, ig.CodePrompt(text, conds, 1, min_codes=n), kv, p, r)
    assert len(codes) == n
    agree, st, bad = _teacher_forced_agreement(om, ig.CodePrompt(text, conds, 1, min_codes=n),
                                               p, codes, ig.SamplerRng(77).state)
    assert not bad, bad  # every differing step is a near-tie within tolerance
    assert agree >= 0.95, agree
    assert r.state == st


# Largest logit difference the parity bound allows (north_star: max-abs 2e-2).
LOGIT_TOL = 2e-2


def _flip_margin(logits, seen_words, params, state, tok):
    """How far the checker's choice is from `tok` at this step, in the units the logit
    tolerance bounds.  Greedy: the logit gap between the best token and `tok`.  Sampled:
    the distance of this step's uniform draw from `tok`'s cumulative-probability interval
    (as a fraction of the active mass), or inf when `tok` is not a candidate.  Follows
    sampler.rs:204-283 in float64, which is precise enough for a margin."""
    lg = np.asarray(logits, np.float64).copy()
    pen = params.repetition_penalty
    if abs(pen - 1.0) > 1.1920929e-7:
        for i in range(min(lg.size, 129 * 64)):
            if (int(seen_words[i // 64]) >> (i % 64)) & 1:
                lg[i] = lg[i] * pen if lg[i] < 0 else lg[i] / pen
    fin = np.isfinite(lg)
    if params.greedy:
        return float(lg[fin].max() - lg[tok]) if fin[tok] else np.inf
    v = np.where(fin, lg / params.temperature, -np.inf)
    order = sorted(range(v.size), key=lambda i: (-v[i], i))
    k = v.size if params.top_k == 0 else min(params.top_k, v.size)
    order = order[:k]
    mx = v[order[0]] if np.isfinite(v[order[0]]) else 0.0
    probs = np.array([np.exp(v[i] - mx) if np.isfinite(v[i]) else 0.0 for i in order])
    norm = probs / probs.sum()
    active, cum = len(order), 0.0
    for i in range(len(order)):
        if i > 0 and cum > params.top_p:
            active = i
            break
        cum += norm[i]
    if tok not in order[:active]:
        if not np.isfinite(v[tok]):
            return np.inf
        if tok not in order:
            # outside the checker's top-k: allowed when a logit error within the bound could
            # swap it with the k-th candidate (returned in the units of a greedy gap)
            return ("logit", float((v[order[-1]] - v[tok]) * params.temperature))
        # inside the top-k but cut by top-p: allowed when the cumulative probability before
        # it is within the band of the top-p threshold
        j = order.index(tok)
        before = float(norm[:j].sum())
        return float(max(before - params.top_p, 0.0))
    j = order.index(tok)
    c = np.concatenate([[0.0], np.cumsum(probs[:active])]) / probs[:active].sum()
    u = ig.SamplerRng.from_state(state).next_f32()
    return float(max(c[j] - u, u - c[j + 1], 0.0))


def _flip_allowed(params, margin):
    """A different token is within tolerance when the margin is inside the band a logit
    error of LOGIT_TOL can move: 2*tol for a greedy gap (or a swap across the top-k
    boundary), exp(2*tol/T) - 1 for a sampled draw or the top-p cut."""
    if isinstance(margin, tuple):  # ("logit", gap)
        return margin[1] <= 2 * LOGIT_TOL
    band = 2 * LOGIT_TOL if params.greedy else np.expm1(2 * LOGIT_TOL / params.temperature)
    return margin <= band


def _teacher_forced_agreement(om, prompt, params, codes, rng_state):
    """Checker's sampler along the device's code path: fraction of steps where it picks
    the device's token, the SamplerRng state after the same draws, and the steps where
    the two differ by more than the logit tolerance can explain."""
    okv = om.kv(1024)
    logits = om.prefill(okv, prompt.text_tokens, prompt.conds, prompt.lang_id, prompt.prior_codes)
    seen = ig.SeenTokenBitSet.new_with_initial_tokens()
    pc = orc.params_c(params.greedy, params.top_k, params.top_p, params.temperature,
                      params.repetition_penalty)
    st, agree, bad = rng_state, 0, []
    for i, c in enumerate(codes):
        if i < prompt.min_codes:
            logits[8193] = -np.inf
        before, st0, words = logits.copy(), st, np.array(seen.words, np.uint64)
        tok, st = orc.sample_next_token(logits, seen.words, pc, st)
        agree += tok == c
        if tok != c:
            m = _flip_margin(before, words, params, st0, c)
            if not _flip_allowed(params, m):
                bad.append((i, tok, c, m))
        seen.insert(c)
        if i + 1 < len(codes):
            logits = om.step(okv, c, len(prompt.prior_codes) + i + 2)
    return agree / max(1, len(codes)), st, bad


@pytest.mark.parametrize("n_req", [3, 6, 20])
def test_generate_batch_matches_checker(small, small_cfg, n_req):
    """Ragged batched generation (3 requests: the persistent kernel; 6: the CUDA-core GEMM
    path; 20: the tensor-core GEMM path): every request's codes agree with the checker
    teacher-forced, with the same draws."""
    gpt, om = small
    lens = ([5, 40, 17, 60, 9, 33] * 4)[:n_req]
    prompts, params = [], []
    for i, n in enumerate(lens):
        steps = 12 + 5 * i
        prompts.append(ig.CodePrompt(make_text(n, small_cfg.text_vocab, seed=n),
                                     make_conds(small_cfg.d, 3 if i % 2 else 32, seed=i), 1 + i % 3,
                                     prior_codes=[1, 2, 3] if i == 2 else (), min_codes=steps))
        params.append(ig.SamplingParams(greedy=i % 2 == 0, top_k=30, max_mel_tokens=steps))
    kvb = ig.KvCache(gpt, max_seq=512, max_batch=n_req)
    rb = [ig.SamplerRng(100 + i) for i in range(n_req)]
    batch = ig.generate_batch(gpt, prompts, kvb, params, rb)
    for i in range(n_req):
        assert len(batch[i]) == params[i].max_mel_tokens
        agree, st, bad = _teacher_forced_agreement(om, prompts[i], params[i], batch[i],
                                                   ig.SamplerRng(100 + i).state)
        assert not bad, (i, bad)  # every differing step is a near-tie within tolerance
        assert agree >= 0.9, (i, agree)
        assert rb[i].state == st


def _batch_prompts(cfg, lens, seed0=0):
    return [ig.CodePrompt(make_text(n, cfg.text_vocab, seed=seed0 + n),
                          make_conds(cfg.d, 3 if i % 2 else 32, seed=seed0 + i), 1 + i % 3,
                          prior_codes=[7, 8190, 2, 511][: i % 4] if i % 3 == 2 else ())
            for i, n in enumerate(lens)]


def test_prefill_batch_matches_checker(small, small_cfg):
    """Packed prefill of ragged requests (tensor-core GEMMs over all positions, flash
    attention per request): every request's logits and KV cache equal a prefill of its
    own (the checker), and a decode step after it matches too."""
    gpt, om = small
    lens = [1, 29, 64, 7, 100, 33]
    prompts = _batch_prompts(small_cfg, lens)
    kv = ig.KvCache(gpt, max_seq=512, max_batch=len(lens))
    got = ig.prefill_batch(gpt, prompts, kv)
    for r, pr in enumerate(prompts):
        okv = om.kv(512)
        ref = om.prefill(okv, pr.text_tokens, pr.conds, pr.lang_id, list(pr.prior_codes))
        check_logits(got[r], ref, f"packed prefill request {r}")
        assert kv.valid_len(r) == okv.valid_len()
        step = gpt.step(kv, 4000 + r, len(pr.prior_codes) + 2, slot=r)
        check_logits(step, om.step(okv, 4000 + r, len(pr.prior_codes) + 2), f"step after request {r}")


def test_load_from_path_and_f32_scales(tmp_path, small_cfg, small_weights):
    path = tmp_path / "gpt_int8.safetensors"
    save_safetensors(str(path), small_weights)
    g1 = ig.Gpt.load_from_path(str(path))
    g2 = ig.Gpt.from_weights(small_weights)
    text = make_text(10, small_cfg.text_vocab, seed=1)
    conds = make_conds(small_cfg.d, 3, seed=2)
    a = g1.prefill(text, conds, 1, ig.KvCache(g1, 128))
    b = g2.prefill(text, conds, 1, ig.KvCache(g2, 128))
    assert np.array_equal(a, b)
    # the real checkpoint stores f32 scales/biases (loader.rs:875-931)
    cfg32 = ModelConfig(n_layers=2, d=256, ff=1024, text_vocab=500, sb_half=False)
    w32 = make_weights(cfg32, seed=3, ln_beta_std=0.02)
    g3 = ig.Gpt.from_weights(w32)
    assert not g3.scales_f16
    om = orc.OracleModel(w32)
    check_logits(g3.prefill(text, conds, 2, ig.KvCache(g3, 128)), om.prefill(om.kv(128), text, conds, 2))


def test_validation_errors(small, small_cfg):
    gpt, _ = small
    with pytest.raises(ig.ValidationError, match="max_seq"):
        ig.KvCache(gpt, max_seq=0)
    kv = ig.KvCache(gpt, max_seq=40)
    conds = make_conds(small_cfg.d, 3, seed=1)
    with pytest.raises(ig.ValidationError, match="text_tokens"):
        gpt.prefill([], conds, 1, kv)
    with pytest.raises(ig.ValidationError, match="text_tokens"):
        gpt.prefill([5] * 601, conds, 1, kv)
    with pytest.raises(ig.ValidationError, match="lang_id"):
        gpt.prefill([5], conds, 107, kv)
    with pytest.raises(ig.ValidationError, match="conds"):
        gpt.prefill([5], np.zeros((1, 3, 7), np.float32), 1, kv)
    with pytest.raises(ig.ValidationError, match="kv_cache"):
        gpt.prefill([5] * 40, conds, 1, kv)
    gpt.prefill([5] * 30, conds, 1, kv)
    with pytest.raises(ig.ValidationError, match="mel_token_id"):
        gpt.step(kv, 8194, 2)
    with pytest.raises(ig.ValidationError, match="pos_idx"):
        gpt.step(kv, 5, 1818)
    for i in range(4):
        gpt.step(kv, 5, 2 + i)
    with pytest.raises(ig.ValidationError, match="kv_cache"):
        gpt.step(kv, 5, 6)
    # generation that outgrows the cache fails like update_layer (gpt.rs:157-165)
    with pytest.raises(ig.ValidationError, match="kv_cache"):
        ig.generate_codes_after(gpt, ig.CodePrompt([5] * 30, conds, 1, min_codes=20), kv,
                                ig.SamplingParams(greedy=True, max_mel_tokens=20), ig.SamplerRng(0))
    with pytest.raises(ig.ValidationError, match="max_mel_tokens"):
        ig.generate_codes_after(gpt, ig.CodePrompt([5], conds, 1, prior_codes=[5] * 1815),
                                ig.KvCache(gpt, 4000), ig.SamplingParams(greedy=True), ig.SamplerRng(0))


# ---------------------------------------------------------------------------
# full-size decoder (24 layers, d=1280, 20 heads, ff=5120, fp16 scales)
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def full():
    cfg = ModelConfig()
    w = make_weights(cfg, seed=2024)
    g = ig.Gpt.from_weights(w, device=0)
    yield cfg, g, orc.OracleModel(w)
    g.close()


@pytest.mark.parametrize("kernel", list(KERNELS))
def test_full_size_teacher_forced(full, monkeypatch, kernel):
    cfg, gpt, om = full
    _use_kernel(monkeypatch, gpt, kernel)
    g, r = _teacher_forced(gpt, om, cfg, 64, 32, 24, seed=41, max_seq=512)
    errs = [check_logits(g[i], r[i], f"full step {i}") for i in range(len(g))]
    agree = np.mean(np.argmax(g, 1) == np.argmax(r, 1))
    assert agree >= 0.99, agree
    print(f"full-size teacher-forced: max |dlogit| {max(errs):.2e}, argmax agreement {agree:.3f}")


def test_full_size_prefill_batch(full):
    """Full-size packed prefill (prompts of 99, 163 and 226 positions: the 64-position
    attention tiles end inside and at the edge of a prompt) against the checker."""
    cfg, gpt, om = full
    prompts = [ig.CodePrompt(make_text(n, cfg.text_vocab, seed=n), make_conds(cfg.d, 32, seed=n + 1), 1)
               for n in (64, 128, 191)]
    kv = ig.KvCache(gpt, max_seq=512, max_batch=3)
    got = ig.prefill_batch(gpt, prompts, kv)
    for r, pr in enumerate(prompts):
        ref = om.prefill(om.kv(512), pr.text_tokens, pr.conds, pr.lang_id)
        err = check_logits(got[r], ref, f"full-size packed prefill {r}")
        assert np.argmax(got[r]) == np.argmax(ref)
        print(f"full-size packed prefill T={kv.valid_len(r)}: max |dlogit| {err:.2e}")


def test_full_size_greedy_generate(full):
    cfg, gpt, om = full
    text = make_text(64, cfg.text_vocab, seed=1)
    conds = make_conds(cfg.d, 32, seed=2)
    p = ig.SamplingParams(greedy=True, max_mel_tokens=32)
    codes = ig.generate_codes(gpt, text, conds, 1, ig.KvCache(gpt, 512), p, ig.SamplerRng(0))
    ref, _ = om.generate(om.kv(512), text, conds, 1, orc.params_c(greedy=True, max_mel_tokens=32), 0)
    n = min(len(codes), len(ref))
    assert n > 0 and np.mean(np.array(codes[:n]) == np.array(ref[:n])) >= 0.99


# ---------------------------------------------------------------------------
# non-finite and out-of-range values in the batch-1 cluster kernel's c_proj, whose
# per-head partials are summed as counted 64-bit fixed-point integers
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("name", ["gpt.h.1.attn.c_proj.scales", "gpt.h.1.mlp.c_proj.scales"])
def test_nonfinite_cproj_partial_propagates(small_weights, small_cfg, name):
    """A NaN scale in one row of the attention's or the MLP's c_proj makes that row's partial
    NaN.  The reference's fp32 sum carries it into h (or the next x), and the LayerNorm
    after it spreads it to every logit; the device step must give all-NaN logits too, not a
    finite value from a wrapped integer sum."""
    w = dict(small_weights)
    sc = w[name].copy()
    sc[5, 2] = np.float16(np.nan)
    w[name] = sc
    gpt = ig.Gpt.from_weights(w, device=0)
    try:
        om = orc.OracleModel(w)
        kv = ig.KvCache(gpt, max_seq=128)
        assert kv.decode_kernel(1) == "xk_decode_kernel"
        text = make_text(11, small_cfg.text_vocab, seed=4)
        conds = make_conds(small_cfg.d, 3, seed=5)
        okv = om.kv(128)
        gpt.prefill(text, conds, 1, kv)
        om.prefill(okv, text, conds, 1)
        got = gpt.step(kv, 77, 2)
        ref = om.step(okv, 77, 2)
        assert np.isnan(ref).all()
        assert np.isnan(got).all(), int(np.isfinite(got).sum())
    finally:
        gpt.close()


def test_cproj_partial_out_of_fixed_point_range_is_an_error():
    """A finite c_proj partial of 2^17 or more does not fit the counted 2^-28 fixed-point
    accumulator word: the step reports a device error instead of a wrapped value, and the
    next steps on a sound model in the same process are correct."""
    cfg32 = ModelConfig(n_layers=2, d=256, ff=1024, text_vocab=500, sb_half=False)
    w = make_weights(cfg32, seed=3, ln_beta_std=0.02)
    w["gpt.h.0.attn.c_proj.scales"] = w["gpt.h.0.attn.c_proj.scales"].copy()
    w["gpt.h.0.attn.c_proj.scales"][3, 1] = 1e12
    text = make_text(9, cfg32.text_vocab, seed=1)
    conds = make_conds(cfg32.d, 3, seed=2)
    bad = ig.Gpt.from_weights(w, device=0)
    try:
        kv = ig.KvCache(bad, max_seq=64)
        assert kv.decode_kernel(1) == "xk_decode_kernel"
        bad.prefill(text, conds, 1, kv)
        with pytest.raises(ig.DeviceError, match="fixed-point"):
            bad.step(kv, 5, 2)
    finally:
        bad.close()
    good_w = make_weights(cfg32, seed=3, ln_beta_std=0.02)
    good = ig.Gpt.from_weights(good_w, device=0)
    try:
        om = orc.OracleModel(good_w)
        kv, okv = ig.KvCache(good, max_seq=64), om.kv(64)
        check_logits(good.prefill(text, conds, 1, kv), om.prefill(okv, text, conds, 1), "prefill after the error")
        for i in range(3):
            check_logits(good.step(kv, 5 + i, 2 + i), om.step(okv, 5 + i, 2 + i), f"step {i} after the error")
    finally:
        good.close()


def test_generate_stops_early_and_skips_idle_steps(small_weights, small_cfg):
    """A request that stops at STOP (sampler.rs:378) leaves the rest of the replayed
    decode-step chunk idle: the batch-1 kernel returns at once for a slot that is no longer
    generating, so the decode time of a run that stops after 3 codes is far below that of
    a run of all its steps, and the codes match the checker."""
    w = dict(small_weights)
    w["mel_head.bias"] = w["mel_head.bias"].copy()
    w["mel_head.bias"][8193] = 40.0  # STOP wins every draw once it is no longer masked
    gpt = ig.Gpt.from_weights(w, device=0)
    try:
        om = orc.OracleModel(w)
        text = make_text(20, small_cfg.text_vocab, seed=6)
        conds = make_conds(small_cfg.d, 3, seed=7)
        kv = ig.KvCache(gpt, max_seq=512)
        assert kv.decode_kernel(1) == "xk_decode_kernel"
        p = ig.SamplingParams(greedy=True, max_mel_tokens=300)
        full = ig.generate_codes_after(gpt, ig.CodePrompt(text, conds, 1, min_codes=300), kv, p, ig.SamplerRng(0))
        assert len(full) == 300
        _, t_full, n_full = gpt.last_timing()
        early = ig.generate_codes_after(gpt, ig.CodePrompt(text, conds, 1, min_codes=3), kv, p, ig.SamplerRng(0))
        _, t_early, n_early = gpt.last_timing()
        ref, _ = om.generate(om.kv(512), text, conds, 1, orc.params_c(greedy=True, max_mel_tokens=300), 0,
                             min_codes=3)
        assert early == ref and len(early) == 3, (early, ref)
        # the first chunk replays 8 steps; all but 2 of them find the slot stopped
        assert n_early >= 8
        per_step_full = t_full / n_full
        assert t_early < 6 * per_step_full, (t_early, per_step_full)
        print(f"early stop: {n_early} replays in {t_early:.3f} ms; full run {per_step_full:.4f} ms per step")
    finally:
        gpt.close()


def test_device_wait_timeout_leaves_the_handle_usable(small, small_cfg):
    """A bounded device wait that runs out comes back as ITTS_E_TIMEOUT (the error convention
    of crates/core/src/error.rs extended by a timeout kind).  The batch-1 kernel's test hook
    (itts_test_stall) polls a word that nothing sets and gives up after 2,000 polls, before the
    step does anything else.  The slot is then as before the step, so the same step on the same
    handle gives the checker's logits; generate through the replayed graphs times out the same
    way, and after the hook is turned off a fresh request generates the checker's codes."""
    from itts_gpt import _lib as L
    lib = L.load_lib()
    gpt, om = small
    text = make_text(20, small_cfg.text_vocab, seed=7)
    conds = make_conds(small_cfg.d, 3, seed=8)
    kv, okv = ig.KvCache(gpt, max_seq=256), om.kv(256)
    assert kv.decode_kernel(1) == "xk_decode_kernel"
    check_logits(gpt.prefill(text, conds, 1, kv), om.prefill(okv, text, conds, 1), "prefill")
    n0 = kv.valid_len()
    assert lib.itts_test_stall(gpt._h, kv._h, 2000) == 0
    with pytest.raises(ig.TimeoutError_, match="timed out"):
        gpt.step(kv, 5, 2)
    assert kv.valid_len() == n0
    assert lib.itts_test_stall(gpt._h, kv._h, -1) == L.ITTS_E_VALIDATION
    assert lib.itts_test_stall(gpt._h, kv._h, 0) == 0
    for i in range(3):
        check_logits(gpt.step(kv, 5 + i, 2 + i), om.step(okv, 5 + i, 2 + i), f"step {i} after the timeout")

    p = ig.SamplingParams(greedy=True, max_mel_tokens=16)
    assert lib.itts_test_stall(gpt._h, kv._h, 2000) == 0
    with pytest.raises(ig.TimeoutError_, match="timed out"):
        ig.generate_codes(gpt, text, conds, 1, kv, p, ig.SamplerRng(0))
    assert lib.itts_test_stall(gpt._h, kv._h, 0) == 0
    codes = ig.generate_codes(gpt, text, conds, 1, kv, p, ig.SamplerRng(0))
    ref, _ = om.generate(om.kv(256), text, conds, 1, orc.params_c(greedy=True, max_mel_tokens=16), 0)
    assert codes == list(ref)
