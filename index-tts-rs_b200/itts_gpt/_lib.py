"""ctypes binding of include/itts_gpt.h (the C ABI of libitts_gpt.so).

The library is built in-tree (``index-tts-rs_b200/build.py``).  There is no
fallback: if the shared library is missing, importing the decoder fails loudly.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent.parent
LIB_PATH = PKG_DIR / "libitts_gpt.so"
SYNTH_PATH = PKG_DIR / "libitts_synth.so"

ITTS_OK = 0
ITTS_E_VALIDATION = 1
ITTS_E_CUDA = 2
ITTS_E_WEIGHTLOAD = 3
ITTS_E_IO = 4
ITTS_E_TIMEOUT = 5

DTYPE_F32, DTYPE_F16, DTYPE_U32, DTYPE_I32 = 0, 1, 2, 3
BITSET_WORDS = 129
MAX_SAMPLE_LOGITS = 16384


class Tensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_int32), ("ndim", C.c_int32),
                ("shape", C.c_int64 * 4), ("data", C.c_void_p)]


class SamplingParamsC(C.Structure):
    _fields_ = [("greedy", C.c_int32), ("top_k", C.c_uint32), ("top_p", C.c_float),
                ("temperature", C.c_float), ("repetition_penalty", C.c_float),
                ("max_mel_tokens", C.c_uint32)]


class CodePromptC(C.Structure):
    _fields_ = [("text_tokens", C.c_void_p), ("n_text", C.c_int32), ("conds", C.c_void_p),
                ("n_conds", C.c_int32), ("lang_id", C.c_int32), ("prior_codes", C.c_void_p),
                ("n_prior", C.c_int32), ("min_codes", C.c_int32)]


# (name, restype, argtypes) of every exported entry point of include/itts_gpt.h
_P = C.c_void_p
_I32 = C.c_int32
SIGNATURES = [
    ("itts_last_error", C.c_size_t, [C.c_char_p, C.c_size_t]),
    ("itts_sampling_params_validate", C.c_int, [C.POINTER(SamplingParamsC)]),
    ("itts_rng_new", C.c_uint64, [C.c_uint64]),
    ("itts_rng_next_f32", C.c_float, [C.POINTER(C.c_uint64)]),
    ("itts_seen_initial", None, [_P]),
    ("itts_seen_insert", None, [_P, C.c_int64]),
    ("itts_gpt_load", C.c_int, [C.c_char_p, C.c_int, C.POINTER(_P)]),
    ("itts_gpt_from_tensors", C.c_int, [C.POINTER(Tensor), _I32, C.c_int, C.POINTER(_P)]),
    ("itts_gpt_free", None, [_P]),
    ("itts_gpt_num_layers", _I32, [_P]),
    ("itts_gpt_dims", C.c_int, [_P, _P]),
    ("itts_kv_create", C.c_int, [_P, _I32, _I32, C.POINTER(_P)]),
    ("itts_kv_free", None, [_P]),
    ("itts_kv_reset", C.c_int, [_P, _I32]),
    ("itts_kv_valid_len", C.c_int, [_P, _I32, C.POINTER(_I32)]),
    ("itts_kv_max_seq", _I32, [_P]),
    ("itts_kv_max_batch", _I32, [_P]),
    ("itts_kv_decode_kernel", _I32, [_P, _I32]),
    ("itts_gpt_prefill", C.c_int, [_P, _P, _I32, _P, _I32, _P, _I32, _I32, _P, _I32, _P]),
    ("itts_gpt_step", C.c_int, [_P, _P, _I32, _P, _P, _P, _P]),
    ("itts_gpt_teacher_forced", C.c_int,
     [_P, _P, _I32, _P, _I32, _P, _I32, _I32, _P, _I32, _P, _P]),
    ("itts_gpt_alignment_attention", C.c_int,
     [_P, _P, _I32, _P, _I32, _P, _I32, _I32, _P, _I32, _P, _I32, _P]),
    ("itts_sample_next_token", C.c_int,
     [_P, _P, _I32, _P, C.POINTER(SamplingParamsC), C.POINTER(C.c_uint64), C.POINTER(_I32)]),
    ("itts_sample_next_token_static", C.c_int,
     [_P, _I32, _P, C.POINTER(SamplingParamsC), C.POINTER(C.c_uint64), C.POINTER(_I32), _P]),
    ("itts_generate_codes_after", C.c_int,
     [_P, _P, _I32, C.POINTER(CodePromptC), C.POINTER(SamplingParamsC), C.POINTER(C.c_uint64),
      _P, _I32, C.POINTER(_I32)]),
    ("itts_gpt_prefill_batch", C.c_int, [_P, _P, _I32, C.POINTER(CodePromptC), _P]),
    ("itts_generate_batch", C.c_int,
     [_P, _P, _I32, C.POINTER(CodePromptC), C.POINTER(SamplingParamsC), _P, _P, _I32, _P]),
    ("itts_batch_admit", C.c_int,
     [_P, _P, _I32, _P, C.POINTER(CodePromptC), C.POINTER(SamplingParamsC), _P]),
    ("itts_batch_decode", C.c_int, [_P, _P, _I32, _I32, _P, C.POINTER(_I32), C.POINTER(_I32)]),
    ("itts_batch_collect", C.c_int,
     [_P, _I32, _P, _I32, C.POINTER(_I32), C.POINTER(C.c_uint64), C.POINTER(_I32)]),
    ("itts_codec_load", C.c_int, [C.c_char_p, C.c_int, C.POINTER(_P)]),
    ("itts_codec_from_tensors", C.c_int, [C.POINTER(Tensor), _I32, C.c_int, C.POINTER(_P)]),
    ("itts_codec_free", None, [_P]),
    ("itts_codec_num_layers", _I32, [_P]),
    ("itts_codec_dims", C.c_int, [_P, _P]),
    ("itts_codec_decode", C.c_int, [_P, _P, _I32, _P, C.POINTER(C.c_float)]),
    ("itts_gpt_last_timing", C.c_int,
     [_P, C.POINTER(C.c_float), C.POINTER(C.c_float), C.POINTER(_I32)]),
    ("itts_bench_decode_forward", C.c_int,
     [_P, _P, _I32, _I32, _I32, C.POINTER(C.c_float), C.POINTER(_I32)]),
    ("itts_bench_trace", C.c_int,
     [_P, _P, _I32, _I32, _P, _I32, C.POINTER(_I32), C.POINTER(_I32)]),
    ("itts_test_stall", C.c_int, [_P, _P, _I32]),
]

_lib = None
_synth: dict = {}


def load_lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python index-tts-rs_b200/build.py` "
                "(the decoder has no CPU fallback)")
        lib = C.CDLL(str(LIB_PATH))
        for name, res, args in SIGNATURES:
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
        _lib = lib
    return _lib


def load_synth(path=None) -> C.CDLL:
    """The seeded input generator; `path` picks another build of the same source."""
    global _synth
    key = str(path or SYNTH_PATH)
    if key not in _synth:
        if not Path(key).exists():
            raise RuntimeError(f"{key} is missing: run index-tts-rs_b200/build.py")
        s = C.CDLL(key)
        s.itts_synth_tag.restype = C.c_uint64
        s.itts_synth_tag.argtypes = [C.c_char_p]
        for fn in (s.itts_synth_normal_f32, s.itts_synth_normal_f16_as_f32):
            fn.restype = None
            fn.argtypes = [C.c_uint64, C.c_uint64, C.c_void_p, C.c_int64, C.c_float, C.c_float]
        s.itts_synth_quant_linear.restype = C.c_int
        s.itts_synth_quant_linear.argtypes = [C.c_uint64, C.c_uint64, C.c_int, C.c_int, C.c_float,
                                              C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
        _synth[key] = s
    return _synth[key]


def last_error() -> str:
    lib = load_lib()
    buf = C.create_string_buffer(1024)
    lib.itts_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")
