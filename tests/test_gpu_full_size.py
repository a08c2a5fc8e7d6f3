"""Parity of the full-size decoder (24 layers, d 1280, 20 heads, ff 5120, fp16 scales) at
the shapes the benchmark runs, against the CPU checker.

* cfg2: the 635-position prompt, then teacher-forced decode steps up to
  2,135 cached positions on each batch-1 decode kernel and on the 2-column kernel;
  a 256-step generate with cfg2's sampling parameters.
* cfg4: the packed prefill of 32 prompts of 635 positions.
* cfg3: 64 ragged requests in one batched generate, some of them stopping
  early at STOP (reference loop: crates/core/src/models/sampler.rs:340-392).
* the teacher-forced replay (gpt.rs:766-915) on the 24-layer model.

Tolerances are the ones stated for this path: logits within max-abs 2e-2 and relative
1e-2 per step, argmax (greedy) agreement on at least 99% of steps, sampling bit-exact
given the same logits and uniforms (a different token only where the checker's logits
put the draw within the logit tolerance of a boundary)."""
import os

import numpy as np
import pytest

import itts_gpt as ig
import oracle as orc
from itts_gpt.synth import ModelConfig, make_conds, make_text, make_weights
from test_gpu_decoder import (KERNELS, _flip_allowed, _flip_margin, _use_kernel,
                              check_logits)

pytestmark = pytest.mark.gpu

CFG = ModelConfig()
N_CONDS, N_TEXT = 32, 600
PROMPT = N_CONDS + N_TEXT + 3           # 635 positions, as in cfg2 / cfg4
N_STEPS = 1500                          # cached positions grow 635 -> 2135
CHECK_EVERY = 50
SAMPLED = dict(top_k=30, top_p=0.8, temperature=0.8, repetition_penalty=10.0)


@pytest.fixture(scope="module")
def full():
    w = make_weights(CFG, seed=2024)
    g = ig.Gpt.from_weights(w, device=0)
    yield g, orc.OracleModel(w, n_threads=os.cpu_count() or 1)
    g.close()


@pytest.fixture(scope="module")
def cfg2_trajectory(full):
    """The checker's logits along a teacher-forced cfg2 decode: the prefill's and every
    CHECK_EVERY-th step's logits, and the argmax of every step."""
    _, om = full
    text = make_text(N_TEXT, CFG.text_vocab, seed=100)
    conds = make_conds(CFG.d, N_CONDS, seed=200)
    codes = np.random.default_rng(5).integers(0, 8192, N_STEPS).tolist()
    okv = om.kv(PROMPT + N_STEPS + 8)
    kept = {0: om.prefill(okv, text, conds, 1)}
    am = [int(np.argmax(kept[0]))]
    for i, c in enumerate(codes):
        lg = om.step(okv, c, i + 2)
        am.append(int(np.argmax(lg)))
        if (i + 1) % CHECK_EVERY == 0 or i + 1 == N_STEPS:
            kept[i + 1] = lg
    assert okv.valid_len() == PROMPT + N_STEPS
    return text, conds, codes, kept, np.array(am)


def _compare_trajectory(logits_of, traj, what):
    """logits_of(i): device logits after step i (0 = the prefill)."""
    _, _, codes, kept, am = traj
    errs = []
    for i, ref in kept.items():
        errs.append(check_logits(logits_of(i), ref, f"{what} after step {i} (KV {PROMPT + i})"))
    return max(errs)


@pytest.mark.parametrize("kernel", list(KERNELS))
def test_cfg2_kv_lengths_teacher_forced(full, cfg2_trajectory, monkeypatch, kernel):
    """Batch-1 decode steps over cfg2's whole KV range (635 -> 2,135 positions: 8 to 26 of
    the cluster kernel's 84-position K/V tiles per head) against the checker."""
    gpt, _ = full
    text, conds, codes, kept, am = cfg2_trajectory
    _use_kernel(monkeypatch, gpt, kernel)
    kv = ig.KvCache(gpt, max_seq=PROMPT + N_STEPS + 8)
    got = {0: gpt.prefill(text, conds, 1, kv)}
    gam = [int(np.argmax(got[0]))]
    for i, c in enumerate(codes):
        lg = gpt.step(kv, c, i + 2)
        gam.append(int(np.argmax(lg)))
        if i + 1 in kept:
            got[i + 1] = lg
    assert kv.valid_len() == PROMPT + N_STEPS
    err = _compare_trajectory(lambda i: got[i], cfg2_trajectory, kernel)
    agree = float(np.mean(np.array(gam) == am))
    assert agree >= 0.99, agree
    print(f"cfg2 KV 635-2135 on {kernel}: max |dlogit| {err:.2e}, argmax agreement {agree:.4f}")


def test_cfg2_kv_lengths_two_columns(full, cfg2_trajectory, monkeypatch):
    """The same trajectory in both columns of 2-column decode steps on the persistent
    grid-wide kernel (ITTS_XK=0: by default 2-column steps run the cluster kernel once per
    column, which the batch-1 tests cover): each column must match the checker."""
    gpt, _ = full
    text, conds, codes, kept, am = cfg2_trajectory
    monkeypatch.setenv("ITTS_XK", "0")
    kv = ig.KvCache(gpt, max_seq=PROMPT + N_STEPS + 8, max_batch=2)
    assert kv.decode_kernel(2) == "mk_decode_kernel"
    p0 = gpt.prefill(text, conds, 1, kv, slot=0)
    p1 = gpt.prefill(text, conds, 1, kv, slot=1)
    got = {0: (p0, p1)}
    gam = [[int(np.argmax(p0))], [int(np.argmax(p1))]]
    for i, c in enumerate(codes):
        lg = gpt.step_batch(kv, [1, 0], [c, c], [i + 2, i + 2])
        for col in range(2):
            gam[col].append(int(np.argmax(lg[col])))
        if i + 1 in kept:
            got[i + 1] = (lg[1], lg[0])  # (slot 0, slot 1)
    for col in range(2):
        err = _compare_trajectory(lambda i: got[i][col], cfg2_trajectory, f"slot {col} of 2")
        agree = float(np.mean(np.array(gam[col]) == am))
        assert agree >= 0.99, (col, agree)
        print(f"cfg2 KV 635-2135, 2 columns, slot {col}: max |dlogit| {err:.2e}, argmax agreement {agree:.4f}")


def _agreement(om, prompt, params, codes, rng_state, stopped, max_seq):
    """The checker's sampler along the device's code path: the fraction of steps where it
    picks the device's token, the steps where they differ beyond what the logit tolerance
    explains, and the SamplerRng state after the same draws (plus the STOP draw when the
    device stopped early, which the checker must also draw as STOP)."""
    okv = om.kv(max_seq)
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
        if tok != c and not _flip_allowed(params, _flip_margin(before, words, params, st0, c)):
            bad.append((i, tok, c))
        seen.insert(c)
        logits = om.step(okv, c, len(prompt.prior_codes) + i + 2)
    if stopped:
        if len(codes) < prompt.min_codes:
            logits[8193] = -np.inf
        tok, st = orc.sample_next_token(logits, seen.words, pc, st)
        if tok != 8193:
            bad.append((len(codes), tok, 8193))
    return agree / max(1, len(codes)), bad, st


def test_cfg2_sampled_generate(full):
    """256 tokens of cfg2's generate (T 0.8, top-k 30, top-p 0.8, repetition penalty 10)
    on the 635-position prompt.  Along the generated codes, (1) the device's teacher-forced
    logits match the checker's at every step, and (2) the reference sampler run on the
    device's own logits with the same SamplerRng stream picks exactly the generated code at
    every step and ends in the same RNG state: the graph-replayed loop is the reference loop
    (sampler.rs:340-392) on the device's logits, and those logits are the reference's within
    tolerance."""
    gpt, om = full
    text = make_text(N_TEXT, CFG.text_vocab, seed=101)
    conds = make_conds(CFG.d, N_CONDS, seed=201)
    n = 256
    prompt = ig.CodePrompt(text, conds, 1, min_codes=n)
    params = ig.SamplingParams(max_mel_tokens=n, **SAMPLED)
    r = ig.SamplerRng(2024)
    codes = ig.generate_codes_after(gpt, prompt, ig.KvCache(gpt, max_seq=PROMPT + n + 8), params, r)
    assert len(codes) == n
    kv, okv = ig.KvCache(gpt, max_seq=PROMPT + n + 8), om.kv(PROMPT + n + 8)
    glog = gpt.prefill(text, conds, 1, kv)
    olog = om.prefill(okv, text, conds, 1)
    seen = ig.SeenTokenBitSet.new_with_initial_tokens()
    pc = orc.params_c(False, **SAMPLED)
    st, errs = ig.SamplerRng(2024).state, []
    for i, c in enumerate(codes):
        errs.append(check_logits(glog, olog, f"teacher-forced logits at step {i}"))
        glog[8193] = -np.inf  # i < min_codes
        tok, st = orc.sample_next_token(glog, seen.words, pc, st)
        assert tok == c, (i, tok, c)
        seen.insert(c)
        if i + 1 < n:
            glog = gpt.step(kv, c, i + 2)
            olog = om.step(okv, c, i + 2)
    assert r.state == st
    print(f"cfg2 sampled generate, {n} steps: codes reproduced exactly; max |dlogit| {max(errs):.2e}")


def test_cfg4_packed_prefill(full):
    """configs[3]'s prefill: 32 prompts x 635 positions in one packed forward.  Three
    requests against the checker (with a decode step after one of them), all 32 against
    single-request prefills on the device."""
    gpt, om = full
    n = 32
    prompts = [ig.CodePrompt(make_text(N_TEXT, CFG.text_vocab, seed=100 + r),
                             make_conds(CFG.d, N_CONDS, seed=200 + r), 1) for r in range(n)]
    kv = ig.KvCache(gpt, max_seq=PROMPT + 8, max_batch=n)
    got = ig.prefill_batch(gpt, prompts, kv)
    assert np.isfinite(got).all()
    for r in (0, 13, 31):
        pr = prompts[r]
        okv = om.kv(PROMPT + 8)
        ref = om.prefill(okv, pr.text_tokens, pr.conds, pr.lang_id)
        err = check_logits(got[r], ref, f"cfg4 packed prefill request {r}")
        assert np.argmax(got[r]) == np.argmax(ref)
        print(f"cfg4 packed prefill request {r}: max |dlogit| {err:.2e}")
        if r == 13:
            step = gpt.step(kv, 4242, 2, slot=r)
            check_logits(step, om.step(okv, 4242, 2), "decode step after the packed prefill")
    kv1 = ig.KvCache(gpt, max_seq=PROMPT + 8)
    for r, pr in enumerate(prompts):
        one = gpt.prefill(pr.text_tokens, pr.conds, 1, kv1)
        check_logits(got[r], one, f"packed vs single prefill, request {r}")
        assert kv.valid_len(r) == PROMPT + (r == 13)  # request 13 took one decode step


@pytest.fixture(scope="module")
def full_stop_biased():
    """The full-size model with mel_head.bias[STOP] raised to 40: once STOP is no longer
    masked (n_codes >= min_codes, sampler.rs:372-376) it wins every draw, so a request
    stops exactly at its min_codes."""
    w = make_weights(CFG, seed=2025)
    w["mel_head.bias"] = w["mel_head.bias"].copy()
    w["mel_head.bias"][8193] = 40.0
    g = ig.Gpt.from_weights(w, device=0)
    yield g, orc.OracleModel(w, n_threads=os.cpu_count() or 1)
    g.close()


def test_cfg3_ragged_batch_with_early_stop(full_stop_biased):
    """configs[2]'s shape: 64 requests with text lengths uniform in [16, 600] and 32
    conditioning latents in one batched generate; every fourth request stops at STOP after
    its own number of codes, the others run to max_mel_tokens.  Every request's length is
    checked, and five of them (short and long prompts, stopped and not) against the checker."""
    gpt, om = full_stop_biased
    n_req, steps = 64, 48
    lens = np.random.default_rng(64).integers(16, 601, n_req)
    prompts, params, expect = [], [], []
    for r in range(n_req):
        stop_at = 3 + (r * 7) % 40 if r % 4 == 0 else steps
        prompts.append(ig.CodePrompt(make_text(int(lens[r]), CFG.text_vocab, seed=300 + r),
                                     make_conds(CFG.d, N_CONDS, seed=400 + r), 1, min_codes=stop_at))
        params.append(ig.SamplingParams(max_mel_tokens=steps, **SAMPLED))
        expect.append(stop_at)
    kv = ig.KvCache(gpt, max_seq=int(lens.max()) + N_CONDS + 3 + steps + 8, max_batch=n_req)
    rngs = [ig.SamplerRng(500 + r) for r in range(n_req)]
    out = ig.generate_batch(gpt, prompts, kv, params, rngs)
    for r in range(n_req):
        assert len(out[r]) == expect[r], (r, len(out[r]), expect[r])
        assert all(0 <= c < 8193 for c in out[r]), r
    stopped = [r for r in range(n_req) if expect[r] < steps]
    short = sorted(range(n_req), key=lambda r: lens[r])
    check = sorted({stopped[1], stopped[-1], short[0], short[1], int(np.argmax(lens))})
    n_agree = n_codes = 0
    for r in check:
        agree, bad, st = _agreement(om, prompts[r], params[r], out[r], ig.SamplerRng(500 + r).state,
                                    expect[r] < steps, int(lens[r]) + N_CONDS + 3 + steps + 8)
        assert not bad, (r, bad)  # every differing draw is a near-tie the logit bound allows
        assert rngs[r].state == st, r
        n_agree += round(agree * len(out[r]))
        n_codes += len(out[r])
        print(f"cfg3 request {r} (text {lens[r]}, {len(out[r])} codes): agreement {agree:.3f}")
    assert n_agree / n_codes >= 0.85, n_agree / n_codes


def test_teacher_forced_replay_full_size(full):
    """itts_gpt_teacher_forced / alignment_attention on the 24-layer model: per-code
    log-probabilities within the logit bound, alignment attention within 2e-3."""
    gpt, om = full
    text = make_text(100, CFG.text_vocab, seed=7)
    conds = make_conds(CFG.d, N_CONDS, seed=8)
    codes = [int(c) for c in np.random.default_rng(9).integers(0, 8194, 64)]
    kv = ig.KvCache(gpt, max_seq=512)
    tf = gpt.teacher_forced(text, conds, 1, codes, kv)
    q0 = N_CONDS + len(text) + 2
    lp, maps = om.replay(om.kv(512), text, conds, 1, codes[:-1], q0, 0, codes, True)
    np.testing.assert_allclose(tf.log_probs, lp, atol=2e-2)
    np.testing.assert_allclose(tf.attention, maps, atol=2e-3)
    prior = codes[:10]
    got = gpt.alignment_attention(text, conds, 1, prior, codes[10:], kv)
    _, maps2 = om.replay(om.kv(512), text, conds, 1, prior + codes[10:-1], q0 + len(prior), 1, (), True)
    np.testing.assert_allclose(got, maps2, atol=2e-3)


@pytest.mark.parametrize("n", [12, 40])
def test_wide_steps_on_int8_tiles(full, n):
    """Decode steps of 12 and 40 columns on the skinny int8 GEMMs (8 warps per CTA at 12
    columns, 16 at 40; the mlp projection sums its four K chunks in a second pass) against the
    checker, column by column, for 4 steps.  The 40-column case uses short prompts to keep the
    checker's prefills quick."""
    gpt, om = full
    if n <= 12:
        lens, n_conds = [10 + 7 * r for r in range(n)], [N_CONDS if r % 2 else 3 for r in range(n)]
    else:
        lens, n_conds = [8 + r % 24 for r in range(n)], [3] * n
    prompts = [ig.CodePrompt(make_text(lens[r], CFG.text_vocab, seed=600 + r),
                             make_conds(CFG.d, n_conds[r], seed=700 + r), 1) for r in range(n)]
    kv = ig.KvCache(gpt, max_seq=256, max_batch=n)
    assert kv.decode_kernel(n) == "gemm path"
    ig.prefill_batch(gpt, prompts, kv)
    okvs = [om.kv(256) for _ in range(n)]
    for r, pr in enumerate(prompts):
        om.prefill(okvs[r], pr.text_tokens, pr.conds, pr.lang_id)
    codes = np.random.default_rng(8).integers(0, 8192, (4, n))
    errs = []
    for s in range(4):
        got = gpt.step_batch(kv, list(range(n)), codes[s].tolist(), [2 + s] * n)
        for r in range(n):
            errs.append(check_logits(got[r], om.step(okvs[r], int(codes[s, r]), 2 + s), f"column {r} step {s}"))
    print(f"{n}-column steps on the int8 tiles: max |dlogit| {max(errs):.2e}")
