"""CPU checker of the teacher-forced replay (crates/core/src/models/gpt.rs:756-915)
against an independent fp32 GPT-2 (HuggingFace transformers, eager attention with the
attention probabilities returned): per-code log-probabilities (log_softmax of the logits
at rows <START_MEL>.., taken at the codes) and the text attention of heads (4, 10) and
(5, 10) averaged (crates/core/src/align/mod.rs:37-40)."""
import numpy as np
import pytest
import torch

import oracle as orc
from itts_gpt.synth import ModelConfig, dequantize, make_conds, make_text, make_weights

ALIGN = [(4, 10), (5, 10)]
CFG6 = ModelConfig(n_layers=6, d=768, ff=3072, text_vocab=500)


@pytest.fixture(scope="module")
def w6():
    return make_weights(CFG6, seed=5, ln_beta_std=0.02)


def hf_forward(w, cfg, text, conds, lang, fed):
    """logits of every row and the attention probabilities of every layer."""
    from transformers import GPT2Config, GPT2Model
    hc = GPT2Config(n_embd=cfg.d, n_layer=cfg.n_layers, n_head=cfg.n_heads, n_inner=cfg.ff,
                    activation_function="gelu_new", layer_norm_epsilon=1e-5, n_positions=4096,
                    vocab_size=16, resid_pdrop=0.0, embd_pdrop=0.0, attn_pdrop=0.0)
    hc._attn_implementation = "eager"
    m = GPT2Model(hc).eval()
    T_ = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    with torch.no_grad():
        m.wpe.weight.zero_()
        for i in range(cfg.n_layers):
            p, b = f"gpt.h.{i}", m.h[i]
            b.ln_1.weight.copy_(T_(w[p + ".ln_1.weight"])); b.ln_1.bias.copy_(T_(w[p + ".ln_1.bias"]))
            b.ln_2.weight.copy_(T_(w[p + ".ln_2.weight"])); b.ln_2.bias.copy_(T_(w[p + ".ln_2.bias"]))
            for hf, ref in ((b.attn.c_attn, ".attn.c_attn"), (b.attn.c_proj, ".attn.c_proj"),
                            (b.mlp.c_fc, ".mlp.c_fc"), (b.mlp.c_proj, ".mlp.c_proj")):
                hf.weight.copy_(T_(dequantize(w, p + ref).T))
                hf.bias.copy_(T_(w[p + ref + ".bias"]))
        m.ln_f.weight.copy_(T_(w["gpt.ln_f.weight"])); m.ln_f.bias.copy_(T_(w["gpt.ln_f.bias"]))
        full = [0] + list(text) + [1]
        rows = [c for c in conds]
        for t, tok in enumerate(full):
            rows.append(w["text_embedding.weight"][tok] + w["lang_embedding.weight"][lang]
                        + w["text_pos_embedding.emb.weight"][t])
        rows.append(w["mel_embedding.weight"][8192] + w["mel_pos_embedding.emb.weight"][0])
        for c, tok in enumerate(fed):
            rows.append(w["mel_embedding.weight"][tok] + w["mel_pos_embedding.emb.weight"][c + 2])
        x = T_(np.stack(rows).astype(np.float32))[None]
        out = m(inputs_embeds=x, output_attentions=True)
        h = torch.nn.functional.layer_norm(out.last_hidden_state[0], (cfg.d,), T_(w["final_norm.weight"]),
                                           T_(w["final_norm.bias"]), 1e-5)
        lg = h @ T_(dequantize(w, "mel_head")).T + T_(w["mel_head.bias"])
    return lg.numpy(), [a[0].numpy() for a in out.attentions]


def expected(w, cfg, text, conds, lang, prior, codes):
    fed = list(prior) + list(codes[:-1])
    lg, att = hf_forward(w, cfg, text, conds, lang, fed)
    klo, khi = len(conds), len(conds) + len(text) + 2
    q0 = khi + len(prior)
    lp = torch.log_softmax(torch.from_numpy(lg[q0:]), -1).numpy()
    logp = np.array([lp[i, c] for i, c in enumerate(codes)], np.float32)
    maps = np.mean([att[l][h][q0:, klo:khi] for l, h in ALIGN], axis=0)
    return logp, maps, q0


@pytest.mark.parametrize("prior", [(), (17, 900, 4)])
def test_oracle_replay_matches_hf_gpt2(w6, prior):
    text = make_text(9, CFG6.text_vocab, seed=3)
    conds = make_conds(CFG6.d, 3, seed=4)
    codes = [5, 77, 8000, 3, 8191, 12, 40]
    logp, maps, q0 = expected(w6, CFG6, text, conds, 1, prior, codes)
    om = orc.OracleModel(w6)
    kv = om.kv(128)
    fed = list(prior) + codes[:-1]
    got_lp, got_maps = om.replay(kv, text, conds, 1, fed, q0, 0, codes, True)
    np.testing.assert_allclose(got_lp, logp, atol=1e-4, rtol=1e-5)
    np.testing.assert_allclose(got_maps, maps, atol=1e-6)
    # alignment mode: the first six layers only, the same maps
    _, al = om.replay(kv, text, conds, 1, fed, q0, 1, (), True)
    np.testing.assert_allclose(al, maps, atol=1e-6)
    assert kv.valid_len() == 0  # the cache is scratch and left reset (gpt.rs:839, 912)
