"""ctypes wrapper of the CPU restatement in itts_oracle.c.

TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg as the checker (and as the timed CPU stand-in for the reference,
which cannot be built here).  The shipped decoder never imports this module.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "libitts_oracle.so"
SYNTH_LIB = HERE / "libitts_oracle_synth.so"
BITSET_WORDS = 129
STOP_MEL = 8193

_lib = None


def build() -> None:
    r = subprocess.run(["make", "-s", "-C", str(HERE)], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")


class ParamsC(C.Structure):
    _fields_ = [("greedy", C.c_int32), ("top_k", C.c_uint32), ("top_p", C.c_float),
                ("temperature", C.c_float), ("repetition_penalty", C.c_float),
                ("max_mel_tokens", C.c_uint32)]


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = C.CDLL(str(LIB))
        P, I, F = C.c_void_p, C.c_int, C.c_float
        L.orc_last_error.restype = C.c_char_p
        L.orc_rng_new.restype = C.c_uint64
        L.orc_rng_new.argtypes = [C.c_uint64]
        L.orc_rng_next_u64.restype = C.c_uint64
        L.orc_rng_next_u64.argtypes = [C.POINTER(C.c_uint64)]
        L.orc_rng_next_f32.restype = F
        L.orc_rng_next_f32.argtypes = [C.POINTER(C.c_uint64)]
        L.orc_seen_initial.argtypes = [P]
        L.orc_seen_insert.argtypes = [P, C.c_int64]
        L.orc_seen_contains.argtypes = [P, C.c_int64]
        L.orc_apply_repetition_penalty.argtypes = [P, P, C.c_int64, F]
        L.orc_argmax_finite.argtypes = [P, C.c_int64]
        L.orc_expf.restype = F
        L.orc_expf.argtypes = [F]
        L.orc_sample_next_token.argtypes = [P, C.c_int64, P, C.POINTER(ParamsC),
                                            C.POINTER(C.c_uint64), C.POINTER(C.c_int32)]
        L.orc_model_new.restype = P
        L.orc_model_new.argtypes = [I] * 10
        L.orc_model_free.argtypes = [P]
        L.orc_model_set_linear.argtypes = [P, I, I, P, P, P, P]
        L.orc_model_set_layer_norms.argtypes = [P, I, P, P, P, P]
        L.orc_model_set_globals.argtypes = [P] * 10
        L.orc_kv_new.restype = P
        L.orc_kv_new.argtypes = [P, I]
        L.orc_kv_free.argtypes = [P]
        L.orc_kv_reset.argtypes = [P]
        L.orc_kv_valid_len.argtypes = [P]
        L.orc_kv_fill.argtypes = [P, I]
        L.orc_prefill.argtypes = [P, P, P, I, P, I, I, P, I, P]
        L.orc_replay.argtypes = [P, P, P, I, P, I, I, P, I, I, I, P, I, P, P]
        L.orc_step.argtypes = [P, P, I, I, P]
        L.orc_generate.argtypes = [P, P, P, I, P, I, I, P, I, I, C.POINTER(ParamsC),
                                   C.POINTER(C.c_uint64), P, I, C.POINTER(I)]
        L.orc_set_num_threads.argtypes = [I]
        _lib = L
    return _lib


def synth_lib_path() -> Path:
    """The seeded input generator built by this directory's Makefile (the same source as
    the package's generator, so both benchmark arms see identical weights and prompts)."""
    if not SYNTH_LIB.exists():
        build()
    return SYNTH_LIB


def error() -> str:
    return lib().orc_last_error().decode()


class OracleError(RuntimeError):
    pass


def _check(rc: int) -> None:
    if rc != 0:
        raise OracleError(error())


def params_c(greedy=False, top_k=3, top_p=0.8, temperature=0.8, repetition_penalty=10.0,
             max_mel_tokens=1500) -> ParamsC:
    return ParamsC(int(bool(greedy)), int(top_k), float(top_p), float(temperature),
                   float(repetition_penalty), int(max_mel_tokens))


def sample_next_token(logits: np.ndarray, seen_words: np.ndarray, params: ParamsC,
                      rng_state: int) -> tuple[int, int]:
    """(token, new rng state); `logits` (float32) receives the penalty in place."""
    assert logits.dtype == np.float32 and logits.flags["C_CONTIGUOUS"]
    st = C.c_uint64(rng_state)
    tok = C.c_int32()
    w = np.ascontiguousarray(seen_words, np.uint64)
    _check(lib().orc_sample_next_token(logits.ctypes.data, logits.size, w.ctypes.data,
                                       C.byref(params), C.byref(st), C.byref(tok)))
    return tok.value, st.value


class OracleModel:
    """The decoder restatement over host tensors (names as in gpt_int8.safetensors)."""

    def __init__(self, t: dict[str, np.ndarray], n_threads: int = 0):
        L = lib()
        if n_threads:
            L.orc_set_num_threads(n_threads)
        self.t = t
        mel = t["mel_embedding.weight"]
        self.d = mel.shape[1]
        self.mel_vocab = mel.shape[0]
        n_layers = 0
        while f"gpt.h.{n_layers}.ln_1.weight" in t:
            n_layers += 1
        self.n_layers = n_layers
        ff = t["gpt.h.0.mlp.c_fc.bias"].shape[0]
        sb_half = t["mel_head.scales"].dtype in (np.float16, np.uint16)
        self.h = L.orc_model_new(n_layers, self.d, self.d // 64, ff, self.mel_vocab,
                                 t["text_embedding.weight"].shape[0],
                                 t["lang_embedding.weight"].shape[0],
                                 t["mel_pos_embedding.emb.weight"].shape[0],
                                 t["text_pos_embedding.emb.weight"].shape[0], int(sb_half))
        p = lambda n: t[n].ctypes.data
        L.orc_model_set_globals(self.h, p("text_embedding.weight"), p("lang_embedding.weight"),
                                p("mel_embedding.weight"), p("mel_pos_embedding.emb.weight"),
                                p("text_pos_embedding.emb.weight"), p("gpt.ln_f.weight"),
                                p("gpt.ln_f.bias"), p("final_norm.weight"), p("final_norm.bias"))
        for i in range(n_layers):
            pre = f"gpt.h.{i}"
            L.orc_model_set_layer_norms(self.h, i, p(pre + ".ln_1.weight"), p(pre + ".ln_1.bias"),
                                        p(pre + ".ln_2.weight"), p(pre + ".ln_2.bias"))
            for which, name in enumerate(("attn.c_attn", "attn.c_proj", "mlp.c_fc", "mlp.c_proj")):
                q = f"{pre}.{name}"
                L.orc_model_set_linear(self.h, i, which, p(q + ".weight"), p(q + ".scales"),
                                       p(q + ".biases"), p(q + ".bias"))
        L.orc_model_set_linear(self.h, 0, 4, p("mel_head.weight"), p("mel_head.scales"),
                               p("mel_head.biases"), p("mel_head.bias"))

    def __del__(self):
        try:
            lib().orc_model_free(self.h)
        except Exception:
            pass

    def kv(self, max_seq: int) -> "OracleKv":
        return OracleKv(self, max_seq)

    def prefill(self, kv: "OracleKv", text, conds, lang: int, prior=()) -> np.ndarray:
        text = np.ascontiguousarray(np.asarray(text, np.int32))
        conds = np.ascontiguousarray(np.asarray(conds, np.float32).reshape(-1, self.d))
        prior = np.ascontiguousarray(np.asarray(prior, np.int32))
        out = np.empty(self.mel_vocab, np.float32)
        _check(lib().orc_prefill(self.h, kv.h, text.ctypes.data, text.size, conds.ctypes.data,
                                 conds.shape[0], lang, prior.ctypes.data if prior.size else None,
                                 prior.size, out.ctypes.data))
        return out

    def replay(self, kv: "OracleKv", text, conds, lang: int, fed, qs: int, mode: int = 0,
               targets=(), want_maps: bool = False):
        """Teacher-forced replay (gpt.rs:800-915): per-target log-probabilities of rows
        qs.. (mode 0) and the alignment attention of those rows (mode 1: the first six
        layers only).  Returns (log_probs or None, maps [rows, n_text + 2] or None)."""
        text = np.ascontiguousarray(np.asarray(text, np.int32))
        conds = np.ascontiguousarray(np.asarray(conds, np.float32).reshape(-1, self.d))
        fed = np.ascontiguousarray(np.asarray(fed, np.int32))
        targets = np.ascontiguousarray(np.asarray(targets, np.int32))
        T = conds.shape[0] + text.size + 3 + fed.size
        lp = np.empty(max(1, targets.size), np.float32) if targets.size else None
        maps = np.empty((T - qs, text.size + 2), np.float32) if want_maps else None
        _check(lib().orc_replay(self.h, kv.h, text.ctypes.data, text.size, conds.ctypes.data,
                                conds.shape[0], lang, fed.ctypes.data if fed.size else None,
                                fed.size, qs, mode, targets.ctypes.data if targets.size else None,
                                targets.size, lp.ctypes.data if lp is not None else None,
                                maps.ctypes.data if maps is not None else None))
        return (lp[:targets.size] if lp is not None else None), maps

    def step(self, kv: "OracleKv", tok: int, pos: int) -> np.ndarray:
        out = np.empty(self.mel_vocab, np.float32)
        _check(lib().orc_step(self.h, kv.h, int(tok), int(pos), out.ctypes.data))
        return out

    def generate(self, kv: "OracleKv", text, conds, lang: int, params: ParamsC, rng_state: int,
                 prior=(), min_codes: int = 0) -> tuple[list[int], int]:
        text = np.ascontiguousarray(np.asarray(text, np.int32))
        conds = np.ascontiguousarray(np.asarray(conds, np.float32).reshape(-1, self.d))
        prior = np.ascontiguousarray(np.asarray(prior, np.int32))
        codes = np.zeros(2048, np.int32)
        st = C.c_uint64(rng_state)
        n = C.c_int()
        _check(lib().orc_generate(self.h, kv.h, text.ctypes.data, text.size, conds.ctypes.data,
                                  conds.shape[0], lang, prior.ctypes.data if prior.size else None,
                                  prior.size, min_codes, C.byref(params), C.byref(st),
                                  codes.ctypes.data, codes.size, C.byref(n)))
        return codes[: n.value].tolist(), st.value


class OracleKv:
    def __init__(self, m: OracleModel, max_seq: int):
        self.h = lib().orc_kv_new(m.h, max_seq)
        if not self.h:
            raise OracleError(error())

    def valid_len(self) -> int:
        return lib().orc_kv_valid_len(self.h)

    def fill(self, n: int) -> None:
        """Timing aid: extends the cache to n positions (cyclic copies of the filled ones),
        so the next step costs what a step at KV length n costs."""
        _check(lib().orc_kv_fill(self.h, int(n)))

    def __del__(self):
        try:
            lib().orc_kv_free(self.h)
        except Exception:
            pass


class OracleCodec:
    """The SemanticCodec decode restatement (orc_codec_decode) over host tensors named as in
    raw/semantic_codec.safetensors."""

    def __init__(self, t: dict[str, np.ndarray]):
        L = lib()
        P, I = C.c_void_p, C.c_int
        L.orc_codec_new.restype = P
        L.orc_codec_new.argtypes = [I] * 9
        L.orc_codec_free.argtypes = [P]
        L.orc_codec_set_globals.argtypes = [P] * 14
        L.orc_codec_set_block.argtypes = [P, I] + [P] * 9
        L.orc_codec_decode.argtypes = [P, P, I, P]
        self.t = {k: np.ascontiguousarray(v, np.float32) for k, v in t.items()}
        t = self.t
        cb = t["quantizer.quantizers.0.codebook.weight"]
        emb = t["decoder.0.embed.weight"]
        pw1 = t["decoder.0.convnext.0.pwconv1.weight"]
        n_layers = 0
        while f"decoder.0.convnext.{n_layers}.gamma" in t:
            n_layers += 1
        self.hidden = emb.shape[2]
        self.h = L.orc_codec_new(n_layers, emb.shape[2], pw1.shape[1], pw1.shape[0], cb.shape[1], cb.shape[0],
                                 emb.shape[1], t["decoder.0.convnext.0.dwconv.weight"].shape[1],
                                 t["up.weight"].shape[1])
        p = lambda n: t[n].ctypes.data
        L.orc_codec_set_globals(self.h, p("quantizer.quantizers.0.codebook.weight"),
                                p("quantizer.quantizers.0.out_project.weight"),
                                p("quantizer.quantizers.0.out_project.bias"), p("decoder.0.embed.weight"),
                                p("decoder.0.embed.bias"), p("decoder.0.norm.weight"), p("decoder.0.norm.bias"),
                                p("decoder.0.final_layer_norm.weight"), p("decoder.0.final_layer_norm.bias"),
                                p("decoder.1.weight"), p("decoder.1.bias"), p("up.weight"), p("up.bias"))
        for l in range(n_layers):
            q = f"decoder.0.convnext.{l}."
            L.orc_codec_set_block(self.h, l, *[p(q + n) for n in (
                "dwconv.weight", "dwconv.bias", "norm.weight", "norm.bias", "pwconv1.weight", "pwconv1.bias",
                "pwconv2.weight", "pwconv2.bias", "gamma")])

    def decode(self, codes) -> np.ndarray:
        k = np.ascontiguousarray(np.asarray(codes, np.int32).reshape(-1))
        out = np.empty((2 * max(1, k.size), self.hidden), np.float32)
        _check(lib().orc_codec_decode(self.h, k.ctypes.data if k.size else None, k.size, out.ctypes.data))
        return out

    def __del__(self):
        try:
            lib().orc_codec_free(self.h)
        except Exception:
            pass
