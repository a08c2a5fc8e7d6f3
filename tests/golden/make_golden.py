"""Generates the golden fixtures in this folder.  Run from the repository root:

    python tests/golden/make_golden.py

decoder_small.npz: logits of an independent fp32 GPT-2 (HuggingFace transformers GPT2Model
loaded with the dequantized weights, plus the reference's sequence embedding, ln_f ->
final_norm double LayerNorm and mel_head; crates/core/src/models/gpt.rs:535-627, 673-692,
734-750) for the small seeded model, at the prompt's last position (prefill) and after each
of five teacher-forced codes (step).  The weights are regenerated from their seed by
itts_gpt.synth; `weights_digest` guards against a change of the generator.

sampler_kats.json: the known-answer behaviours of the reference's sampler tests
(crates/core/src/models/sampler.rs, test module), restated as input/expected pairs.
"""
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT / "index-tts-rs_b200"))

from itts_gpt.synth import SMALL, dequantize, make_conds, make_text, make_weights  # noqa: E402

SEED = 7
TEXT_SEED, COND_SEED, N_TEXT, N_CONDS, LANG = 1, 2, 11, 3, 1
CODES = [5, 77, 8000, 3, 8191]


def weights_digest(w) -> str:
    h = hashlib.sha256()
    for k in sorted(w):
        h.update(k.encode())
        h.update(np.ascontiguousarray(w[k]).tobytes())
    return h.hexdigest()


def small_model():
    return make_weights(SMALL, seed=SEED, ln_beta_std=0.02)


def prompt():
    return (make_text(N_TEXT, SMALL.text_vocab, seed=TEXT_SEED),
            make_conds(SMALL.d, N_CONDS, seed=COND_SEED))


def hf_logits(w, cfg, text, conds, lang, codes):
    import torch
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
    P = len(conds) + len(full) + 1
    return lg.numpy()[P - 1:], P


# sampler.rs test module, as behaviours: (name, logits, seen tokens beyond the initial set,
# params, rng seed, expected token or expected penalized logits)
SAMPLER_KATS = [
    {"name": "repetition_penalty_on_seen_tokens", "source": "sampler.rs:430-454",
     "n": 32, "set": {"1": 2.0, "10": 4.0, "20": -3.0, "25": 4.0}, "insert": [10, 20],
     "penalty": 2.0, "expected": {"1": 1.0, "10": 2.0, "20": -6.0, "25": 4.0}, "atol": 1e-6},
    {"name": "spike_wins_with_default_params", "source": "sampler.rs:177-189 (doc example)",
     "fill": -10.0,
     "n": 8194, "spike_index": 42, "spike_value": 25.0, "rng_seed": 7, "expected_token": 42},
    {"name": "initial_seen_set", "source": "sampler.rs:98-107 (doc example)",
     "expected_seen": [1, 8192], "expected_unseen": [100]},
    {"name": "rng_seed_mixing", "source": "sampler.rs:24-38 (SamplerRng::new)",
     "seed": 42, "expected_state": (42 ^ 0x9E3779B97F4A7C15) & (2**64 - 1)},
]


def main():
    w = small_model()
    text, conds = prompt()
    logits, P = hf_logits(w, SMALL, text, conds, LANG, CODES)
    np.savez_compressed(HERE / "decoder_small.npz", logits=logits.astype(np.float32),
                        text=np.asarray(text, np.int32), conds=conds.astype(np.float32),
                        codes=np.asarray(CODES, np.int32), lang=np.int32(LANG),
                        prefix_len=np.int32(P), weights_digest=np.bytes_(weights_digest(w)))
    (HERE / "sampler_kats.json").write_text(json.dumps(SAMPLER_KATS, indent=1) + "\n")
    print("wrote", HERE / "decoder_small.npz", logits.shape, "and sampler_kats.json")


if __name__ == "__main__":
    main()
