"""The reference's on-disk formats through the C ABI.

* A gpt_int8.safetensors file with the real checkpoint's dtypes (U32 packed weights, F32
  scales / biases / bias / LayerNorms / embeddings: loader.rs:875-931) read by
  itts_gpt_load.
* The reference's own Stage-1 golden tensors (crates/core/fixtures/golden_ref.safetensors,
  extracted by tests/golden/extract_reference_gpt_fixture.py): conds [1, 3, 1280] and the
  token ids of its six sentences, run through prefill and a 32-step greedy generate like
  CP-10 / CP-11 (gpt.rs:931-979, sampler.rs:488-536) on a synthetic model of the real
  shapes (d 1280, 60,510-row text table), against the CPU checker.
* CP-10 / CP-11 themselves against the fixture's logits and codes, which need the real
  checkpoint: like the reference's tests they do nothing without it (here: the
  environment variable ITTS_GPT_INT8 names the file)."""
import os
from pathlib import Path

import numpy as np
import pytest

import itts_gpt as ig
import oracle as orc
from itts_gpt.synth import ModelConfig, make_conds, make_text, make_weights, save_safetensors
from test_gpu_decoder import check_logits

pytestmark = pytest.mark.gpu

FIXTURE = Path(__file__).resolve().parent / "golden" / "reference_gpt_fixture.npz"
LANG_ZH = 1  # Language::Zh.token_id() (config.rs:366-373)


def test_f32_scale_checkpoint_file(tmp_path):
    cfg = ModelConfig(n_layers=2, d=256, ff=1024, text_vocab=500, sb_half=False)
    w = make_weights(cfg, seed=21, ln_beta_std=0.02)
    assert w["mel_head.scales"].dtype == np.float32 and w["gpt.h.0.mlp.c_fc.weight"].dtype == np.uint32
    path = tmp_path / "gpt_int8.safetensors"
    save_safetensors(str(path), w)
    g = ig.Gpt.load_from_path(str(path))
    ref = ig.Gpt.from_weights(w)
    try:
        assert not g.scales_f16
        om = orc.OracleModel(w)
        text, conds = make_text(30, cfg.text_vocab, seed=2), make_conds(cfg.d, 3, seed=3)
        kv, kv2, okv = ig.KvCache(g, 128), ig.KvCache(ref, 128), om.kv(128)
        a = g.prefill(text, conds, LANG_ZH, kv)
        np.testing.assert_array_equal(a, ref.prefill(text, conds, LANG_ZH, kv2))
        check_logits(a, om.prefill(okv, text, conds, LANG_ZH), "prefill from an F32-scale file")
        for i in range(8):
            check_logits(g.step(kv, 100 + i, 2 + i), om.step(okv, 100 + i, 2 + i), f"step {i}")
    finally:
        g.close()
        ref.close()


@pytest.fixture(scope="module")
def fixture():
    return dict(np.load(FIXTURE))


def test_reference_fixture_through_prefill_and_greedy(fixture):
    """The fixture's conds and token ids (real text-table ids up to 58,959) on a 2-layer
    model of the real widths: prefill logits of all six sentences, then CP-11's greedy
    32-code generate (repetition penalty 10, sampler.rs:204-208) for sentence 0."""
    cfg = ModelConfig(n_layers=2, text_vocab=60510)
    w = make_weights(cfg, seed=31)
    gpt = ig.Gpt.from_weights(w)
    try:
        om = orc.OracleModel(w)
        conds = fixture["conds"]
        assert conds.shape == (1, 3, 1280) and conds.dtype == np.float32
        for i in range(6):
            toks = fixture[f"token_ids_{i}"]
            kv = ig.KvCache(gpt)  # KvCache::new(DEFAULT_KV_MAX_SEQ)
            got = gpt.prefill(toks, conds, LANG_ZH, kv)
            assert kv.valid_len() == 3 + toks.size + 3
            check_logits(got, om.prefill(om.kv(2048), toks, conds[0], LANG_ZH), f"sentence {i} prefill")
        p = ig.SamplingParams(greedy=True, max_mel_tokens=32)
        codes = ig.generate_codes(gpt, fixture["token_ids_0"], conds, LANG_ZH, ig.KvCache(gpt), p, ig.SamplerRng(0))
        ref, _ = om.generate(om.kv(2048), fixture["token_ids_0"], conds[0], LANG_ZH,
                             orc.params_c(greedy=True, max_mel_tokens=32), ig.SamplerRng(0).state)
        assert len(codes) == len(ref) == 32
        assert np.mean(np.array(codes) == np.array(ref)) >= 0.99
    finally:
        gpt.close()


@pytest.mark.skipif(not os.environ.get("ITTS_GPT_INT8"), reason="needs the real gpt_int8.safetensors")
def test_cp10_cp11_with_real_checkpoint(fixture):
    gpt = ig.Gpt.load_from_path(os.environ["ITTS_GPT_INT8"])
    try:
        toks, conds = fixture["token_ids_0"], fixture["conds"]
        got = gpt.prefill(toks, conds, LANG_ZH, ig.KvCache(gpt))
        want = fixture["prefill_logits"]
        cos = float(np.dot(got, want) / (np.linalg.norm(got) * np.linalg.norm(want)))
        assert cos >= 0.9999, cos                                      # CP-10
        assert list(np.argsort(-got)[:10]) == list(np.argsort(-want)[:10])
        codes = ig.generate_codes(gpt, toks, conds, LANG_ZH, ig.KvCache(gpt),
                                  ig.SamplingParams(greedy=True, max_mel_tokens=32), ig.SamplerRng(0))
        assert codes == fixture["greedy_codes"].tolist()               # CP-11
    finally:
        gpt.close()
