"""Continuous batching on the device (itts_batch_admit / _decode / _collect) and the
per-GPU dispatcher over it, against the CPU checker: every request's codes are what its
own generate_codes_after would give (sampler.rs:340-392), teacher-forced through the
checker with the same uniform stream, whatever requests shared its decode steps."""
import numpy as np
import pytest

import itts_gpt as ig
import oracle as orc
from itts_gpt.serve import Dispatcher, Request, RequestQueue, gpu_engine_factory
from itts_gpt.synth import make_conds, make_text
from test_gpu_full_size import _agreement

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def stop_biased(small_weights):
    """The small model with mel_head.bias[STOP] = 40: a request stops exactly at its
    min_codes (STOP is masked before, sampler.rs:372-376, and wins every draw after)."""
    w = dict(small_weights)
    w["mel_head.bias"] = w["mel_head.bias"].copy()
    w["mel_head.bias"][8193] = 40.0
    return w, orc.OracleModel(w)


def _requests(cfg, n, seed0=0, max_codes=40):
    rng = np.random.default_rng(seed0)
    out = []
    for i in range(n):
        stop_at = int(rng.integers(1, max_codes + 1))
        prompt = ig.CodePrompt(make_text(int(rng.integers(1, 90)), cfg.text_vocab, seed=seed0 + i),
                               make_conds(cfg.d, 3 if i % 2 else 32, seed=seed0 + 100 + i), 1 + i % 3,
                               prior_codes=[5, 6, 7][: i % 4] if i % 5 == 1 else (), min_codes=stop_at)
        params = ig.SamplingParams(greedy=i % 3 == 0, top_k=30, top_p=0.8, temperature=0.8,
                                   repetition_penalty=10.0, max_mel_tokens=max_codes)
        out.append(Request(i, prompt, params, seed=1000 + seed0 + i))
    return out


def _check(om, req, codes, state):
    stopped = len(codes) < req.params.max_mel_tokens
    assert len(codes) == min(req.prompt.min_codes, req.params.max_mel_tokens), (req.id, len(codes))
    agree, bad, st = _agreement(om, req.prompt, req.params, codes, ig.SamplerRng(req.seed).state, stopped, 512)
    assert not bad, (req.id, bad)
    assert st == state, req.id
    return agree


def test_batch_admit_decode_collect(stop_biased, small_cfg):
    w, om = stop_biased
    gpt = ig.Gpt.from_weights(w, device=0)
    try:
        kv = ig.KvCache(gpt, max_seq=256, max_batch=6)
        reqs = _requests(small_cfg, 5, seed0=7)
        ig.batch_admit(gpt, kv, [2, 0, 5], [r.prompt for r in reqs[:3]], [r.params for r in reqs[:3]],
                       [ig.SamplerRng(r.seed) for r in reqs[:3]])
        with pytest.raises(ig.ValidationError, match="not collected"):
            ig.batch_admit(gpt, kv, [0], [reqs[3].prompt], [reqs[3].params], [ig.SamplerRng(1)])
        with pytest.raises(ig.ValidationError, match="continuous batch"):
            gpt.step(kv, 5, 2, slot=2)
        with pytest.raises(ig.ValidationError, match="no finished request"):
            ig.batch_collect(gpt, kv, 5)
        where = {2: reqs[0], 0: reqs[1], 5: reqs[2]}
        done, admitted = {}, False
        while where:
            finished, n_live = ig.batch_decode(gpt, kv, 1 << 20, chunk=4)
            assert finished or n_live == 0
            for s in finished:
                codes, state, status = ig.batch_collect(gpt, kv, s)
                assert status == 0
                done[where.pop(s).id] = (codes, state)
                if not admitted:  # two more requests join while the others decode
                    ig.batch_admit(gpt, kv, [s, 1], [r.prompt for r in reqs[3:]], [r.params for r in reqs[3:]],
                                   [ig.SamplerRng(r.seed) for r in reqs[3:]])
                    where.update({s: reqs[3], 1: reqs[4]})
                    admitted = True
        assert sorted(done) == [0, 1, 2, 3, 4]
        for r in reqs:
            _check(om, r, *done[r.id])
        # reset cancels a live request and frees its slot
        ig.batch_admit(gpt, kv, [3], [reqs[0].prompt], [reqs[0].params], [ig.SamplerRng(reqs[0].seed)])
        kv.reset(3)
        assert ig.batch_decode(gpt, kv, 10) == ([], 0)
        pr = reqs[0].prompt  # the slot is free again for the other entry points
        gpt.prefill_after(pr.text_tokens, pr.conds, pr.lang_id, pr.prior_codes, kv, slot=3)
    finally:
        gpt.close()


@pytest.mark.parametrize("max_batch", [1, 3, 8])
def test_dispatcher_matches_checker(stop_biased, small_cfg, max_batch):
    """30 requests of different lengths through one GPU worker with max_batch slots (1: the
    batch-1 cluster kernel; 3: the grid-wide kernel with idle columns; 8: the GEMM path)."""
    w, om = stop_biased
    reqs = _requests(small_cfg, 30, seed0=max_batch)
    d = Dispatcher([gpu_engine_factory(w, 0, max_batch=max_batch, max_seq=256, chunk=4)])
    res = d.run(RequestQueue(reqs))
    assert d.workers[0].error is None, d.workers[0].error
    assert sorted(res) == list(range(30))
    agree = [_check(om, r, res[r.id].codes, res[r.id].rng_state) for r in reqs]
    assert np.mean(agree) >= 0.9, np.mean(agree)
