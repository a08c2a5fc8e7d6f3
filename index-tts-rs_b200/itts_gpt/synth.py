"""Seeded synthetic decoder weights and inputs in the reference's on-disk layout.

The tensor names, shapes and dtypes are those ``Gpt::from_weights`` reads from
``gpt_int8.safetensors`` (crates/core/src/models/gpt.rs:229-250, 279-322,
477-515): quantized linears as ``weight`` u32 ``[out, in/4]``, ``scales`` and
``biases`` ``[out, in/64]`` and ``bias`` f32 ``[out]``; LayerNorms and embedding
tables f32.  Values follow the benchmark recipe: weights N(0, 0.02) quantized
affine int8 in groups of 64 (fp16 scales/biases by default), LN gamma
1 + N(0, 0.01), LN beta 0 (configurable), embeddings N(0, 0.02).

The numbers come from ``libitts_synth.so`` (csrc/synth.cpp): a pure function of
(seed, tensor name, element index), independent of thread count.
"""
from __future__ import annotations

import ctypes
import json
import os
import struct
from dataclasses import dataclass, field

import numpy as np

from ._lib import load_synth


@dataclass(frozen=True)
class ModelConfig:
    """Decoder geometry.  Defaults are the IndexTTS-2.5 GPT (gpt.rs:31-54) with
    the benchmark's 12000-row text table."""

    n_layers: int = 24
    d: int = 1280
    ff: int = 5120
    mel_vocab: int = 8194
    text_vocab: int = 12000
    lang_vocab: int = 107
    mel_pos_len: int = 1818
    text_pos_len: int = 602
    sb_half: bool = True  # fp16 scales/biases (benchmark); False = f32 (real checkpoint)

    @property
    def n_heads(self) -> int:
        return self.d // 64

    def weight_bytes(self) -> int:
        """Algorithmic bytes of one decode-step weight stream (int8 + s/b + bias + LN)."""
        sb = 2 if self.sb_half else 4

        def lin(o, i):
            return o * i + 2 * o * (i // 64) * sb + 4 * o

        per_layer = (lin(3 * self.d, self.d) + lin(self.d, self.d) + lin(self.ff, self.d)
                     + lin(self.d, self.ff) + 4 * self.d * 4)
        return self.n_layers * per_layer + lin(self.mel_vocab, self.d) + 4 * self.d * 4


SMALL = ModelConfig(n_layers=2, d=256, ff=1024, text_vocab=500)


def _linear_names(prefix: str):
    return [f"{prefix}.weight", f"{prefix}.scales", f"{prefix}.biases", f"{prefix}.bias"]


def linear_specs(cfg: ModelConfig):
    """(prefix, out, in) of every quantized linear, in load order."""
    out = []
    for i in range(cfg.n_layers):
        p = f"gpt.h.{i}"
        out += [(f"{p}.attn.c_attn", 3 * cfg.d, cfg.d), (f"{p}.attn.c_proj", cfg.d, cfg.d),
                (f"{p}.mlp.c_fc", cfg.ff, cfg.d), (f"{p}.mlp.c_proj", cfg.d, cfg.ff)]
    out.append(("mel_head", cfg.mel_vocab, cfg.d))
    return out


def make_weights(cfg: ModelConfig, seed: int = 1234, w_std: float = 0.02,
                 ln_beta_std: float = 0.0, bias_std: float = 0.02,
                 synth_path=None) -> dict[str, np.ndarray]:
    """All decoder tensors by reference name (`synth_path`: another build of the
    generator library, same values)."""
    lib = load_synth(synth_path)
    t: dict[str, np.ndarray] = {}

    def normal(name, shape, mean, std):
        a = np.empty(shape, np.float32)
        if std == 0.0:
            a.fill(mean)
        else:
            lib.itts_synth_normal_f32(seed, lib.itts_synth_tag(name.encode()), a.ctypes.data,
                                      a.size, mean, std)
        t[name] = a

    d = cfg.d
    normal("text_embedding.weight", (cfg.text_vocab, d), 0.0, 0.02)
    normal("lang_embedding.weight", (cfg.lang_vocab, d), 0.0, 0.02)
    normal("mel_embedding.weight", (cfg.mel_vocab, d), 0.0, 0.02)
    normal("mel_pos_embedding.emb.weight", (cfg.mel_pos_len, d), 0.0, 0.02)
    normal("text_pos_embedding.emb.weight", (cfg.text_pos_len, d), 0.0, 0.02)
    for i in range(cfg.n_layers):
        for ln in ("ln_1", "ln_2"):
            normal(f"gpt.h.{i}.{ln}.weight", (d,), 1.0, 0.01)
            normal(f"gpt.h.{i}.{ln}.bias", (d,), 0.0, ln_beta_std)
    for ln in ("gpt.ln_f", "final_norm"):
        normal(f"{ln}.weight", (d,), 1.0, 0.01)
        normal(f"{ln}.bias", (d,), 0.0, ln_beta_std)
    sb_dtype = np.uint16 if cfg.sb_half else np.float32
    for prefix, o, i in linear_specs(cfg):
        w = np.empty((o, i // 4), np.uint32)
        s = np.empty((o, i // 64), sb_dtype)
        b = np.empty((o, i // 64), sb_dtype)
        rc = lib.itts_synth_quant_linear(seed, lib.itts_synth_tag((prefix + ".weight").encode()),
                                         o, i, w_std, int(cfg.sb_half), w.ctypes.data,
                                         s.ctypes.data, b.ctypes.data)
        if rc != 0:
            raise ValueError(f"bad linear shape {prefix} {o}x{i}")
        t[prefix + ".weight"] = w
        t[prefix + ".scales"] = s.view(np.float16) if cfg.sb_half else s
        t[prefix + ".biases"] = b.view(np.float16) if cfg.sb_half else b
        normal(prefix + ".bias", (o,), 0.0, bias_std)
    return t


def make_conds(d: int, n_conds: int, seed: int, synth_path=None) -> np.ndarray:
    """``[n_conds, d]`` f32 conditioning latents drawn N(0,1) and rounded through fp16."""
    lib = load_synth(synth_path)
    a = np.empty((n_conds, d), np.float32)
    lib.itts_synth_normal_f16_as_f32(seed, lib.itts_synth_tag(b"conds"), a.ctypes.data, a.size,
                                     0.0, 1.0)
    return a


def make_text(n: int, text_vocab: int, seed: int) -> np.ndarray:
    """Uniform text token ids in [2, text_vocab)."""
    rng = np.random.default_rng(seed)
    return rng.integers(2, text_vocab, size=n, dtype=np.int64).astype(np.int32)


def dequantize(t: dict[str, np.ndarray], prefix: str) -> np.ndarray:
    """f32 ``[out, in]`` matrix of a quantized linear (W = s*q + b per group of 64)."""
    q = t[prefix + ".weight"].view(np.uint8).astype(np.float32)
    o, i = q.shape
    s = t[prefix + ".scales"].astype(np.float32)
    b = t[prefix + ".biases"].astype(np.float32)
    return (q.reshape(o, i // 64, 64) * s[:, :, None] + b[:, :, None]).reshape(o, i)


_ST_DTYPES = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16",
              np.dtype(np.uint32): "U32", np.dtype(np.int32): "I32"}


def save_safetensors(path: str, tensors: dict[str, np.ndarray]) -> None:
    """Writes a safetensors file (8-byte header length, JSON header, raw data)."""
    header, off, order = {}, 0, []
    for name in sorted(tensors):
        a = np.ascontiguousarray(tensors[name])
        n = a.nbytes
        header[name] = {"dtype": _ST_DTYPES[a.dtype], "shape": list(a.shape),
                        "data_offsets": [off, off + n]}
        order.append(a)
        off += n
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for a in order:
            f.write(a.tobytes())


def make_codec_weights(seed: int = 77, n_layers: int = 12, hidden: int = 1024, dim: int = 384,
                       inter: int = 2048, cdim: int = 8, n_codes: int = 8192, embed_k: int = 7,
                       dw_k: int = 7, up_k: int = 3, synth_path=None) -> dict[str, np.ndarray]:
    """Seeded SemanticCodec decoder tensors by the names of raw/semantic_codec.safetensors
    (crates/core/src/models/codec.rs:136-162, convnext.rs:40-60), F32, MLX conv layouts
    [C_out, K, C_in].  Weights N(0, 1/fan_in), biases N(0, 0.02), LayerNorm gamma
    1 + N(0, 0.01) and beta N(0, 0.01), layer scale N(0.1, 0.01), codebook N(0, 1)."""
    lib = load_synth(synth_path)
    t: dict[str, np.ndarray] = {}

    def normal(name, shape, mean, std):
        a = np.empty(shape, np.float32)
        lib.itts_synth_normal_f32(seed, lib.itts_synth_tag(name.encode()), a.ctypes.data, a.size, mean, std)
        t[name] = a

    q = "quantizer.quantizers.0."
    normal(q + "codebook.weight", (n_codes, cdim), 0.0, 1.0)
    normal(q + "out_project.weight", (hidden, 1, cdim), 0.0, cdim ** -0.5)
    normal(q + "out_project.bias", (hidden,), 0.0, 0.02)
    normal("decoder.0.embed.weight", (dim, embed_k, hidden), 0.0, (embed_k * hidden) ** -0.5)
    normal("decoder.0.embed.bias", (dim,), 0.0, 0.02)
    for ln in ("decoder.0.norm", "decoder.0.final_layer_norm"):
        normal(ln + ".weight", (dim,), 1.0, 0.01)
        normal(ln + ".bias", (dim,), 0.0, 0.01)
    for l in range(n_layers):
        p = f"decoder.0.convnext.{l}."
        normal(p + "dwconv.weight", (dim, dw_k, 1), 0.0, dw_k ** -0.5)
        normal(p + "dwconv.bias", (dim,), 0.0, 0.02)
        normal(p + "norm.weight", (dim,), 1.0, 0.01)
        normal(p + "norm.bias", (dim,), 0.0, 0.01)
        normal(p + "pwconv1.weight", (inter, dim), 0.0, dim ** -0.5)
        normal(p + "pwconv1.bias", (inter,), 0.0, 0.02)
        normal(p + "pwconv2.weight", (dim, inter), 0.0, inter ** -0.5)
        normal(p + "pwconv2.bias", (dim,), 0.0, 0.02)
        normal(p + "gamma", (dim,), 0.1, 0.01)
    normal("decoder.1.weight", (hidden, dim), 0.0, dim ** -0.5)
    normal("decoder.1.bias", (hidden,), 0.0, 0.02)
    normal("up.weight", (hidden, up_k, hidden), 0.0, (up_k * hidden) ** -0.5)
    normal("up.bias", (hidden,), 0.0, 0.02)
    return t
