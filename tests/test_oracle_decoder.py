"""CPU checker decoder vs an independent fp32 GPT-2 (HuggingFace transformers
GPT2Model with the dequantized weights), and the reference's validation behaviour.

Pins the restatement of crates/core/src/models/gpt.rs: sequence embedding
(:535-627), pre-LN block with tanh-GELU (:325-384), KV cache append + causal
attention at scale 0.125, the ln_f -> final_norm double LayerNorm and mel_head
(:673-692, :734-750).
"""
import numpy as np
import pytest
import torch

import oracle as orc
from itts_gpt.synth import dequantize, make_conds, make_text


def hf_reference_logits(w, cfg, text, conds, lang, codes):
    from transformers import GPT2Config, GPT2Model

    hc = GPT2Config(n_embd=cfg.d, n_layer=cfg.n_layers, n_head=cfg.n_heads, n_inner=cfg.ff,
                    activation_function="gelu_new", layer_norm_epsilon=1e-5, n_positions=4096,
                    vocab_size=16, resid_pdrop=0.0, embd_pdrop=0.0, attn_pdrop=0.0)
    m = GPT2Model(hc).eval()
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    with torch.no_grad():
        m.wpe.weight.zero_()
        for i in range(cfg.n_layers):
            p, b = f"gpt.h.{i}", m.h[i]
            b.ln_1.weight.copy_(T(w[p + ".ln_1.weight"])); b.ln_1.bias.copy_(T(w[p + ".ln_1.bias"]))
            b.ln_2.weight.copy_(T(w[p + ".ln_2.weight"])); b.ln_2.bias.copy_(T(w[p + ".ln_2.bias"]))
            for hf, ref in ((b.attn.c_attn, ".attn.c_attn"), (b.attn.c_proj, ".attn.c_proj"),
                            (b.mlp.c_fc, ".mlp.c_fc"), (b.mlp.c_proj, ".mlp.c_proj")):
                hf.weight.copy_(T(dequantize(w, p + ref).T))
                hf.bias.copy_(T(w[p + ref + ".bias"]))
        m.ln_f.weight.copy_(T(w["gpt.ln_f.weight"])); m.ln_f.bias.copy_(T(w["gpt.ln_f.bias"]))
        full = [0] + list(text) + [1]
        rows = [c for c in conds]
        for t, tok in enumerate(full):
            rows.append(w["text_embedding.weight"][tok] + w["lang_embedding.weight"][lang]
                        + w["text_pos_embedding.emb.weight"][t])
        rows.append(w["mel_embedding.weight"][8192] + w["mel_pos_embedding.emb.weight"][0])
        for c, tok in enumerate(codes):
            rows.append(w["mel_embedding.weight"][tok] + w["mel_pos_embedding.emb.weight"][c + 2])
        x = T(np.stack(rows).astype(np.float32))[None]
        h = m(inputs_embeds=x).last_hidden_state[0]
        h = torch.nn.functional.layer_norm(h, (cfg.d,), T(w["final_norm.weight"]),
                                           T(w["final_norm.bias"]), 1e-5)
        lg = h @ T(dequantize(w, "mel_head")).T + T(w["mel_head.bias"])
    return lg.numpy(), len(conds) + len(full) + 1


def test_oracle_prefill_and_steps_match_hf_gpt2(small_cfg, small_weights):
    text = make_text(11, small_cfg.text_vocab, seed=1)
    conds = make_conds(small_cfg.d, 3, seed=2)
    codes = [5, 77, 8000, 3, 8191]
    ref, P = hf_reference_logits(small_weights, small_cfg, text, conds, 1, codes)
    om = orc.OracleModel(small_weights)
    kv = om.kv(128)
    got = [om.prefill(kv, text, conds, 1)]
    assert kv.valid_len() == P
    for i, c in enumerate(codes):
        got.append(om.step(kv, c, i + 2))
    assert kv.valid_len() == P + len(codes)
    for i, g in enumerate(got):
        np.testing.assert_allclose(g, ref[P - 1 + i], atol=2e-5, rtol=1e-4)


def test_oracle_prefill_after_equals_stepping(small_cfg, small_weights):
    """prefill_after(prior) == prefill then step through the prior codes (gpt.rs:646-696)."""
    text = make_text(7, small_cfg.text_vocab, seed=5)
    conds = make_conds(small_cfg.d, 32, seed=6)
    prior = [11, 4000, 12]
    om = orc.OracleModel(small_weights)
    a = om.prefill(om.kv(128), text, conds, 3, prior)
    kv = om.kv(128)
    om.prefill(kv, text, conds, 3)
    for i, c in enumerate(prior):
        b = om.step(kv, c, i + 2)
    np.testing.assert_allclose(a, b, atol=2e-5, rtol=1e-4)


def test_oracle_validation(small_cfg, small_weights):
    om = orc.OracleModel(small_weights)
    with pytest.raises(orc.OracleError, match="max_seq"):
        om.kv(0)  # gpt.rs:103-108
    kv = om.kv(40)
    conds = make_conds(small_cfg.d, 3, seed=1)
    with pytest.raises(orc.OracleError, match="text_tokens"):
        om.prefill(kv, [], conds, 1)  # gpt.rs:536-541
    with pytest.raises(orc.OracleError, match="text"):
        om.prefill(kv, [5] * 601, conds, 1)  # gpt.rs:543-548
    with pytest.raises(orc.OracleError, match="lang_id"):
        om.prefill(kv, [5], conds, 107)  # gpt.rs:555-560
    with pytest.raises(orc.OracleError, match="kv_cache"):
        om.prefill(kv, [5] * 40, conds, 1)  # capacity (gpt.rs:157-165)
    om.prefill(kv, [5] * 30, conds, 1)  # 3 + 32 + 1 = 36 positions
    with pytest.raises(orc.OracleError, match="mel_token_id"):
        om.step(kv, 8194, 2)  # gpt.rs:707-712
    with pytest.raises(orc.OracleError, match="pos_idx"):
        om.step(kv, 5, 1818)  # gpt.rs:713-718
    for i in range(4):
        om.step(kv, 5, 2 + i)
    with pytest.raises(orc.OracleError, match="kv_cache"):
        om.step(kv, 5, 6)


def test_oracle_generate_loop_rules(small_cfg, small_weights):
    """generate_codes_after (sampler.rs:340-392): step cap, STOP masking by min_codes."""
    om = orc.OracleModel(small_weights)
    text = make_text(9, small_cfg.text_vocab, seed=8)
    conds = make_conds(small_cfg.d, 3, seed=9)
    codes, _ = om.generate(om.kv(256), text, conds, 1, orc.params_c(greedy=True, max_mel_tokens=20), 0)
    assert len(codes) <= 20 and all(0 <= c < 8193 for c in codes)
    # max_steps = min(max_mel_tokens, 1815 - prior): a 1815-code prior leaves nothing
    with pytest.raises(orc.OracleError, match="max_mel_tokens"):
        om.generate(om.kv(4000), text, conds, 1, orc.params_c(greedy=True), 0, prior=[5] * 1815)
    # with STOP made the argmax, greedy stops at once unless min_codes masks it
    w2 = dict(small_weights)
    b = w2["mel_head.bias"].copy()
    b[8193] = 100.0
    w2["mel_head.bias"] = b
    om2 = orc.OracleModel(w2)
    codes, _ = om2.generate(om2.kv(256), text, conds, 1, orc.params_c(greedy=True, max_mel_tokens=10), 0)
    assert codes == []
    codes, _ = om2.generate(om2.kv(256), text, conds, 1, orc.params_c(greedy=True, max_mel_tokens=10), 0,
                            min_codes=4)
    assert len(codes) == 4
