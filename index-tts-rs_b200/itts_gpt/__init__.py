"""Python mirror of the index-tts-rs decoder / KV-cache / sampler interface over
the B200 C ABI (include/itts_gpt.h).

Names, argument meaning and error behaviour follow the Rust items in
crates/core/src/models/{gpt.rs,sampler.rs} and crates/core/src/config.rs:

  Gpt.load_from_path / Gpt.from_weights / Gpt.prefill / Gpt.prefill_after / Gpt.step
  KvCache(max_seq) .reset() .valid_len() .max_seq()
  SamplingParams, SamplerRng, SeenTokenBitSet, sample_next_token
  CodePrompt, generate_codes, generate_codes_after (+ generate_batch, ragged batches)

Errors raise IndexTtsError subclasses carrying the library's message
(Validation / Device / WeightLoad / Io), mirroring IndexTtsError in
crates/core/src/error.rs.  Every numeric step runs on the GPU; there is no
host fallback.
"""
from __future__ import annotations

import ctypes as C
import weakref
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np

from . import _lib
from ._lib import (BITSET_WORDS, CodePromptC, SamplingParamsC, Tensor, load_lib, last_error)

GPT_HEAD_DIM = 64
GPT_MEL_VOCAB = 8194
START_TEXT_TOKEN = 0
STOP_TEXT_TOKEN = 1
START_MEL_TOKEN = 8192
STOP_MEL_TOKEN = 8193
DEFAULT_KV_MAX_SEQ = 2048
GPT_MEL_POS_LEN = 1818


class IndexTtsError(Exception):
    code = -1

    def __init__(self, message: str):
        super().__init__(message)
        self.message = message


class ValidationError(IndexTtsError):
    code = _lib.ITTS_E_VALIDATION


class DeviceError(IndexTtsError):
    code = _lib.ITTS_E_CUDA


class WeightLoadError(IndexTtsError):
    code = _lib.ITTS_E_WEIGHTLOAD


class IoError(IndexTtsError):
    code = _lib.ITTS_E_IO


class TimeoutError_(IndexTtsError):
    code = _lib.ITTS_E_TIMEOUT


_ERR = {c.code: c for c in (ValidationError, DeviceError, WeightLoadError, IoError, TimeoutError_)}


def _check(rc: int) -> None:
    if rc != _lib.ITTS_OK:
        raise _ERR.get(rc, IndexTtsError)(last_error())


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


# ---------------------------------------------------------------------------
# config newtypes (config.rs:454-682, 1283-1320)
# ---------------------------------------------------------------------------
@dataclass
class SamplingParams:
    greedy: bool = False
    seed: int | None = None
    top_k: int = 3
    top_p: float = 0.8
    temperature: float = 0.8
    repetition_penalty: float = 10.0
    max_mel_tokens: int = 1500

    def to_c(self) -> SamplingParamsC:
        if not (0 <= int(self.top_k) <= 0xFFFFFFFF):
            raise ValidationError(f"validation error on `top_k`: must be <= 8194, got {self.top_k}")
        p = SamplingParamsC(int(bool(self.greedy)), int(self.top_k), float(self.top_p),
                            float(self.temperature), float(self.repetition_penalty),
                            max(0, min(int(self.max_mel_tokens), 0xFFFFFFFF)))
        _check(load_lib().itts_sampling_params_validate(C.byref(p)))
        return p


# ---------------------------------------------------------------------------
# SamplerRng / SeenTokenBitSet (sampler.rs:24-158)
# ---------------------------------------------------------------------------
_M64 = (1 << 64) - 1


class SamplerRng:
    """SplitMix64 variant of sampler.rs:24-62 (state = seed ^ 0x9E3779B97F4A7C15)."""

    def __init__(self, seed: int):
        self.state = (int(seed) ^ 0x9E3779B97F4A7C15) & _M64

    @classmethod
    def from_state(cls, state: int) -> "SamplerRng":
        r = cls(0)
        r.state = int(state) & _M64
        return r

    def next_u64(self) -> int:
        self.state = (self.state + 0x9E3779B97F4A7C15) & _M64
        z = self.state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
        return z ^ (z >> 31)

    def next_f32(self) -> float:
        return float(np.float32(self.next_u64() >> 40) * np.float32(1.0 / (1 << 24)))


class SeenTokenBitSet:
    def __init__(self, words: np.ndarray | None = None):
        self.words = np.zeros(BITSET_WORDS, np.uint64) if words is None else words.astype(np.uint64)

    @classmethod
    def empty(cls) -> "SeenTokenBitSet":
        return cls()

    @classmethod
    def new_with_initial_tokens(cls) -> "SeenTokenBitSet":
        s = cls()
        s.insert(STOP_TEXT_TOKEN)
        s.insert(START_MEL_TOKEN)
        return s

    def insert(self, token_id: int) -> None:
        w, b = divmod(int(token_id), 64)
        if 0 <= w < BITSET_WORDS and token_id >= 0:
            self.words[w] |= np.uint64(1 << b)

    def contains(self, token_id: int) -> bool:
        w, b = divmod(int(token_id), 64)
        return token_id >= 0 and w < BITSET_WORDS and bool((int(self.words[w]) >> b) & 1)


# ---------------------------------------------------------------------------
# Gpt / KvCache (gpt.rs:74-754)
# ---------------------------------------------------------------------------
_NP_DTYPE = {np.dtype(np.float32): _lib.DTYPE_F32, np.dtype(np.float16): _lib.DTYPE_F16,
             np.dtype(np.uint16): _lib.DTYPE_F16, np.dtype(np.uint32): _lib.DTYPE_U32,
             np.dtype(np.int32): _lib.DTYPE_I32}


class Gpt:
    """The Stage-1 decoder resident on one GPU (gpt.rs:436-450)."""

    def __init__(self, handle: int, device: int):
        self._h = C.c_void_p(handle)
        self.device = device
        self._caches: "weakref.WeakSet[KvCache]" = weakref.WeakSet()
        dims = np.zeros(10, np.int32)
        _check(load_lib().itts_gpt_dims(self._h, _ptr(dims)))
        (self.n_layers, self.d, self.n_heads, self.ff, self.mel_vocab, self.text_vocab,
         self.mel_pos_len, self.text_pos_len, self.lang_vocab, sb) = (int(x) for x in dims)
        self.scales_f16 = bool(sb)

    @classmethod
    def load_from_path(cls, path: str, device: int = 0) -> "Gpt":
        h = C.c_void_p()
        _check(load_lib().itts_gpt_load(str(path).encode(), device, C.byref(h)))
        return cls(h.value, device)

    @classmethod
    def from_weights(cls, tensors: dict[str, np.ndarray], device: int = 0) -> "Gpt":
        arr = (Tensor * len(tensors))()
        keep = []
        for i, (name, a) in enumerate(tensors.items()):
            a = np.ascontiguousarray(a)
            keep.append(a)
            nb = name.encode()
            keep.append(nb)
            arr[i].name = nb
            arr[i].dtype = _NP_DTYPE[a.dtype]
            arr[i].ndim = a.ndim
            for j, s in enumerate(a.shape):
                arr[i].shape[j] = s
            arr[i].data = a.ctypes.data
        h = C.c_void_p()
        _check(load_lib().itts_gpt_from_tensors(arr, len(tensors), device, C.byref(h)))
        return cls(h.value, device)

    def num_layers(self) -> int:
        return int(load_lib().itts_gpt_num_layers(self._h))

    def close(self) -> None:
        """Frees the device weights; caches made from this model are freed first (the C
        ABI requires every itts_kv of a model to be freed before the model)."""
        for kv in list(self._caches):
            kv.close()
        if self._h:
            load_lib().itts_gpt_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- forward ---------------------------------------------------------------
    def _conds(self, conds) -> np.ndarray:
        c = np.ascontiguousarray(np.asarray(conds, np.float32))
        if c.ndim == 3:
            if c.shape[0] != 1:
                raise ValidationError(f"validation error on `conds`: expected shape [1, n, {self.d}], got {list(c.shape)}")
            c = c[0]
        if c.ndim != 2 or c.shape[1] != self.d:
            raise ValidationError(f"validation error on `conds`: expected shape [1, n, {self.d}], got {list(c.shape)}")
        return np.ascontiguousarray(c)

    def prefill(self, text_tokens, conds, lang_id: int, cache: "KvCache", slot: int = 0) -> np.ndarray:
        return self.prefill_after(text_tokens, conds, lang_id, [], cache, slot)

    def prefill_after(self, text_tokens, conds, lang_id: int, prior_codes, cache: "KvCache",
                      slot: int = 0) -> np.ndarray:
        t = np.ascontiguousarray(np.asarray(text_tokens, np.int32).reshape(-1))
        p = np.ascontiguousarray(np.asarray(prior_codes, np.int32).reshape(-1))
        c = self._conds(conds)
        out = np.empty(self.mel_vocab, np.float32)
        _check(load_lib().itts_gpt_prefill(self._h, cache._h, slot, _ptr(t), t.size, _ptr(c),
                                           c.shape[0], int(lang_id), _ptr(p) if p.size else None,
                                           p.size, _ptr(out)))
        return out

    def step(self, cache: "KvCache", mel_token_id: int, pos_idx: int, slot: int = 0) -> np.ndarray:
        return self.step_batch(cache, [slot], [mel_token_id], [pos_idx])[0]

    def step_batch(self, cache: "KvCache", slots, toks, pos) -> np.ndarray:
        s = np.ascontiguousarray(np.asarray(slots, np.int32))
        t = np.ascontiguousarray(np.asarray(toks, np.int32))
        q = np.ascontiguousarray(np.asarray(pos, np.int32))
        out = np.empty((s.size, self.mel_vocab), np.float32)
        _check(load_lib().itts_gpt_step(self._h, cache._h, s.size, _ptr(s), _ptr(t), _ptr(q),
                                        _ptr(out)))
        return out

    def teacher_forced(self, text_tokens, conds, lang_id: int, codes, cache: "KvCache",
                       slot: int = 0) -> "TeacherForced":
        """Gpt::teacher_forced (gpt.rs:766-776): every code's log-probability and the text
        attention of the alignment heads, [len(codes), len(text) + 2]."""
        return self._replay(text_tokens, conds, lang_id, codes, cache, slot, True)

    def code_log_probs(self, text_tokens, conds, lang_id: int, codes, cache: "KvCache",
                       slot: int = 0) -> np.ndarray:
        """Gpt::code_log_probs (gpt.rs:785-797)."""
        return self._replay(text_tokens, conds, lang_id, codes, cache, slot, False).log_probs

    def _replay(self, text_tokens, conds, lang_id, codes, cache, slot, attention):
        t = np.ascontiguousarray(np.asarray(text_tokens, np.int32).reshape(-1))
        k = np.ascontiguousarray(np.asarray(codes, np.int32).reshape(-1))
        c = self._conds(conds)
        lp = np.empty(max(1, k.size), np.float32)
        att = np.empty((k.size, t.size + 2), np.float32) if attention else None
        _check(load_lib().itts_gpt_teacher_forced(
            self._h, cache._h, slot, _ptr(t), t.size, _ptr(c), c.shape[0], int(lang_id),
            _ptr(k) if k.size else None, k.size, _ptr(lp),
            _ptr(att) if att is not None and att.size else None))
        return TeacherForced(attention=att if att is not None else np.zeros((0,), np.float32),
                             log_probs=lp[:k.size])

    def alignment_attention(self, text_tokens, conds, lang_id: int, prior_codes, codes,
                            cache: "KvCache", slot: int = 0) -> np.ndarray:
        """Gpt::alignment_attention (gpt.rs:875-915): [len(codes), len(text) + 2]."""
        t = np.ascontiguousarray(np.asarray(text_tokens, np.int32).reshape(-1))
        p = np.ascontiguousarray(np.asarray(prior_codes, np.int32).reshape(-1))
        k = np.ascontiguousarray(np.asarray(codes, np.int32).reshape(-1))
        c = self._conds(conds)
        att = np.empty((max(1, k.size), t.size + 2), np.float32)
        _check(load_lib().itts_gpt_alignment_attention(
            self._h, cache._h, slot, _ptr(t), t.size, _ptr(c), c.shape[0], int(lang_id),
            _ptr(p) if p.size else None, p.size, _ptr(k) if k.size else None, k.size, _ptr(att)))
        return att[:k.size]

    def last_timing(self) -> tuple[float, float, int]:
        a, b, n = C.c_float(), C.c_float(), C.c_int32()
        _check(load_lib().itts_gpt_last_timing(self._h, C.byref(a), C.byref(b), C.byref(n)))
        return a.value, b.value, n.value


class KvCache:
    """KvCache::new(max_seq) (gpt.rs:102-128), with `max_batch` request slots."""

    def __init__(self, gpt: Gpt, max_seq: int = DEFAULT_KV_MAX_SEQ, max_batch: int = 1):
        self._h = C.c_void_p()
        self.gpt = gpt
        _check(load_lib().itts_kv_create(gpt._h, int(max_seq), int(max_batch), C.byref(self._h)))
        gpt._caches.add(self)

    def reset(self, slot: int = -1) -> None:
        _check(load_lib().itts_kv_reset(self._h, slot))

    def valid_len(self, slot: int = 0) -> int:
        v = C.c_int32()
        _check(load_lib().itts_kv_valid_len(self._h, slot, C.byref(v)))
        return v.value

    def max_seq(self) -> int:
        return int(load_lib().itts_kv_max_seq(self._h))

    def max_batch(self) -> int:
        return int(load_lib().itts_kv_max_batch(self._h))

    def decode_kernel(self, n_columns: int = 1) -> str:
        """Name of the decode-step kernel a step of `n_columns` columns runs."""
        k = int(load_lib().itts_kv_decode_kernel(self._h, int(n_columns)))
        return {2: "mk_decode_kernel", 3: "gemm path",
                4: "xk_decode_kernel"}.get(k, "none")

    def close(self) -> None:
        if self._h:
            load_lib().itts_kv_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# sampling and generation (sampler.rs:191-392)
# ---------------------------------------------------------------------------
def sample_next_token(gpt: Gpt, logits: np.ndarray, seen: SeenTokenBitSet,
                      params: SamplingParams, rng: SamplerRng) -> int:
    """sample_next_token on the device; `logits` (float32, contiguous) receives the
    repetition penalty in place and `rng` advances exactly when a draw happens."""
    if logits.dtype != np.float32 or not logits.flags["C_CONTIGUOUS"]:
        raise ValidationError("validation error on `logits`: expected a contiguous float32 array")
    p = params.to_c()
    st = C.c_uint64(rng.state)
    tok = C.c_int32()
    words = np.ascontiguousarray(seen.words, np.uint64)
    _check(load_lib().itts_sample_next_token(gpt._h, _ptr(logits), logits.size, _ptr(words),
                                             C.byref(p), C.byref(st), C.byref(tok)))
    rng.state = st.value
    return tok.value


@dataclass
class TeacherForced:
    """TeacherForced (gpt.rs:428-434): row-major attention [codes, text + 2] (empty when not
    requested) and the log-probability of every code."""

    attention: np.ndarray
    log_probs: np.ndarray


@dataclass
class CodePrompt:
    """CodePrompt (sampler.rs:287-301)."""

    text_tokens: Sequence[int]
    conds: np.ndarray
    lang_id: int
    prior_codes: Sequence[int] = ()
    min_codes: int = 0


def _prompt_c(gpt: Gpt, pr: CodePrompt, keep: list) -> CodePromptC:
    t = np.ascontiguousarray(np.asarray(pr.text_tokens, np.int32).reshape(-1))
    c = gpt._conds(pr.conds)
    p = np.ascontiguousarray(np.asarray(pr.prior_codes, np.int32).reshape(-1))
    keep += [t, c, p]
    return CodePromptC(t.ctypes.data if t.size else None, t.size, c.ctypes.data, c.shape[0],
                       int(pr.lang_id), p.ctypes.data if p.size else None, p.size,
                       int(pr.min_codes))


def prefill_batch(gpt: Gpt, prompts: Sequence[CodePrompt], cache: KvCache) -> np.ndarray:
    """Gpt::prefill_after for several requests in one packed forward: request r resets and
    fills slot r; returns the [n, mel_vocab] logits of each request's last position."""
    n = len(prompts)
    keep: list = []
    pcs = (CodePromptC * n)(*[_prompt_c(gpt, pr, keep) for pr in prompts])
    out = np.empty((n, gpt.mel_vocab), np.float32)
    _check(load_lib().itts_gpt_prefill_batch(gpt._h, cache._h, n, pcs, _ptr(out)))
    return out


def generate_codes(gpt: Gpt, text_tokens, conds, lang_id: int, cache: KvCache,
                   params: SamplingParams, rng: SamplerRng, slot: int = 0) -> list[int]:
    return generate_codes_after(gpt, CodePrompt(text_tokens, conds, lang_id), cache, params, rng,
                                slot)


def generate_codes_after(gpt: Gpt, prompt: CodePrompt, cache: KvCache, params: SamplingParams,
                         rng: SamplerRng, slot: int = 0) -> list[int]:
    keep: list = []
    pc = _prompt_c(gpt, prompt, keep)
    p = params.to_c()
    cap = max(1, gpt.mel_pos_len)
    codes = np.zeros(cap, np.int32)
    st = C.c_uint64(rng.state)
    n = C.c_int32()
    _check(load_lib().itts_generate_codes_after(gpt._h, cache._h, slot, C.byref(pc), C.byref(p),
                                                C.byref(st), _ptr(codes), cap, C.byref(n)))
    rng.state = st.value
    return codes[: n.value].tolist()


def generate_batch(gpt: Gpt, prompts: Sequence[CodePrompt], cache: KvCache,
                   params: SamplingParams | Sequence[SamplingParams],
                   rngs: Sequence[SamplerRng]) -> list[list[int]]:
    """Ragged batched generation: request r uses slot r; results equal independent
    generate_codes_after calls."""
    n = len(prompts)
    keep: list = []
    pcs = (CodePromptC * n)(*[_prompt_c(gpt, pr, keep) for pr in prompts])
    plist = list(params) if isinstance(params, (list, tuple)) else [params] * n
    ps = (SamplingParamsC * n)(*[p.to_c() for p in plist])
    states = np.array([r.state for r in rngs], np.uint64)
    cap = max(1, gpt.mel_pos_len)
    codes = np.zeros((n, cap), np.int32)
    counts = np.zeros(n, np.int32)
    _check(load_lib().itts_generate_batch(gpt._h, cache._h, n, pcs, ps, _ptr(states), _ptr(codes),
                                          cap, _ptr(counts)))
    for r, s in zip(rngs, states):
        r.state = int(s)
    return [codes[i, : counts[i]].tolist() for i in range(n)]


# ---------------------------------------------------------------------------
# continuous batching (include/itts_gpt.h itts_batch_*): requests enter free slots of a
# cache between decode chunks and leave at their own STOP
# ---------------------------------------------------------------------------
def batch_admit(gpt: Gpt, cache: KvCache, slots: Sequence[int], prompts: Sequence[CodePrompt],
                params: Sequence[SamplingParams], rngs: Sequence[SamplerRng]) -> None:
    """Starts requests r in slots[r] (free slots): packed prefill + first sample."""
    n = len(prompts)
    keep: list = []
    pcs = (CodePromptC * n)(*[_prompt_c(gpt, pr, keep) for pr in prompts])
    ps = (SamplingParamsC * n)(*[p.to_c() for p in params])
    sl = np.ascontiguousarray(np.asarray(slots, np.int32))
    states = np.array([r.state for r in rngs], np.uint64)
    _check(load_lib().itts_batch_admit(gpt._h, cache._h, n, _ptr(sl), pcs, ps, _ptr(states)))


def batch_decode(gpt: Gpt, cache: KvCache, max_steps: int, chunk: int = 8) -> tuple[list[int], int]:
    """Decode steps over all slots until a request finishes (or max_steps): returns the
    finished slots and the number of requests still generating."""
    out = np.zeros(max(1, cache.max_batch()), np.int32)
    nf, nl = C.c_int32(), C.c_int32()
    _check(load_lib().itts_batch_decode(gpt._h, cache._h, int(max_steps), int(chunk), _ptr(out),
                                        C.byref(nf), C.byref(nl)))
    return out[: nf.value].tolist(), nl.value


def batch_collect(gpt: Gpt, cache: KvCache, slot: int) -> tuple[list[int], int, int]:
    """Codes, final SamplerRng state and status (0, or the Validation code when the request
    outgrew the cache) of the finished request in `slot`; frees the slot."""
    cap = max(1, gpt.mel_pos_len)
    codes = np.zeros(cap, np.int32)
    n, st, status = C.c_int32(), C.c_uint64(), C.c_int32()
    _check(load_lib().itts_batch_collect(cache._h, int(slot), _ptr(codes), cap, C.byref(n), C.byref(st),
                                         C.byref(status)))
    return codes[: n.value].tolist(), st.value, status.value


# ---------------------------------------------------------------------------
# SemanticCodec decode (crates/core/src/models/codec.rs:104-239)
# ---------------------------------------------------------------------------
def _tensor_array(tensors: dict[str, np.ndarray]):
    arr = (Tensor * len(tensors))()
    keep = []
    for i, (name, a) in enumerate(tensors.items()):
        a = np.ascontiguousarray(a)
        nb = name.encode()
        keep += [a, nb]
        arr[i].name = nb
        arr[i].dtype = _NP_DTYPE[a.dtype]
        arr[i].ndim = a.ndim
        for j, sz in enumerate(a.shape):
            arr[i].shape[j] = sz
        arr[i].data = a.ctypes.data
    return arr, keep


class SemanticCodec:
    """Decoder half of the semantic codec on one GPU: mel codes -> [2T, 1024] features."""

    def __init__(self, handle: int, device: int):
        self._h = C.c_void_p(handle)
        self.device = device
        self.last_device_ms = 0.0
        dims = np.zeros(5, np.int32)
        _check(load_lib().itts_codec_dims(self._h, _ptr(dims)))
        self.n_layers, self.hidden, self.dim, self.inter, self.n_codes = (int(x) for x in dims)

    @classmethod
    def load_from_path(cls, path: str, device: int = 0) -> "SemanticCodec":
        h = C.c_void_p()
        _check(load_lib().itts_codec_load(str(path).encode(), device, C.byref(h)))
        return cls(h.value, device)

    @classmethod
    def from_weights(cls, tensors: dict[str, np.ndarray], device: int = 0) -> "SemanticCodec":
        arr, keep = _tensor_array(tensors)
        h = C.c_void_p()
        _check(load_lib().itts_codec_from_tensors(arr, len(tensors), device, C.byref(h)))
        return cls(h.value, device)

    def num_layers(self) -> int:
        return int(load_lib().itts_codec_num_layers(self._h))

    def decode(self, codes) -> np.ndarray:
        """SemanticCodec::decode for one sequence: [T] codes -> [2T, 1024] float32."""
        k = np.ascontiguousarray(np.asarray(codes, np.int32).reshape(-1))
        out = np.empty((2 * max(1, k.size), self.hidden), np.float32)
        ms = C.c_float()
        _check(load_lib().itts_codec_decode(self._h, _ptr(k) if k.size else None, k.size, _ptr(out),
                                            C.byref(ms)))
        self.last_device_ms = ms.value
        return out

    def close(self) -> None:
        if self._h:
            load_lib().itts_codec_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
