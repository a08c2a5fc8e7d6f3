"""The C ABI library loads on a CPU-only machine and exports every entry point that
include/itts_gpt.h declares; host-only entry points (parameter validation, the
SamplerRng / SeenTokenBitSet helpers, argument checks that fail before any device
work) behave like the reference.  No kernel runs here."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

import itts_gpt as ig
from itts_gpt import _lib

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "itts_gpt.h"


def header_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(itts_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    names = header_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    bound = {n for n, _, _ in _lib.SIGNATURES}
    assert set(names) == bound, set(names) ^ bound


def test_rng_and_seen_helpers_match_reference():
    lib = _lib.load_lib()
    st = ctypes.c_uint64(lib.itts_rng_new(7))
    py = ig.SamplerRng(7)
    assert st.value == py.state
    for _ in range(100):
        assert lib.itts_rng_next_f32(ctypes.byref(st)) == py.next_f32()
    w = np.zeros(129, np.uint64)
    lib.itts_seen_initial(w.ctypes.data)
    s = ig.SeenTokenBitSet.new_with_initial_tokens()
    assert np.array_equal(w, s.words)
    lib.itts_seen_insert(w.ctypes.data, 8256)  # out of range: ignored (sampler.rs:118-124)
    lib.itts_seen_insert(w.ctypes.data, -1)
    assert np.array_equal(w, s.words)


@pytest.mark.parametrize("field,kw", [
    ("temperature", dict(temperature=0.0)), ("temperature", dict(temperature=2.5)),
    ("temperature", dict(temperature=float("nan"))), ("top_p", dict(top_p=1.5)),
    ("top_p", dict(top_p=0.0)), ("top_k", dict(top_k=9000)),
    ("repetition_penalty", dict(repetition_penalty=0.5)),
    ("max_mel_tokens", dict(max_mel_tokens=0)), ("max_mel_tokens", dict(max_mel_tokens=1816)),
])
def test_sampling_params_validation(field, kw):
    with pytest.raises(ig.ValidationError, match=field):
        ig.SamplingParams(**kw).to_c()


def test_defaults_are_the_reference_defaults():
    p = ig.SamplingParams()
    assert (p.greedy, p.top_k, p.top_p, p.temperature, p.repetition_penalty, p.max_mel_tokens) == \
        (False, 3, 0.8, 0.8, 10.0, 1500)  # config.rs:614-620, 1309-1320
    p.to_c()


def test_load_errors_before_device_work(tmp_path):
    with pytest.raises(ig.IoError):
        ig.Gpt.load_from_path(str(tmp_path / "missing.safetensors"))
    bad = tmp_path / "bad.safetensors"
    bad.write_bytes(b"\x10\x00\x00\x00\x00\x00\x00\x00{not json}......")
    with pytest.raises(ig.WeightLoadError):
        ig.Gpt.load_from_path(str(bad))
    with pytest.raises(ig.WeightLoadError, match="mel_embedding"):
        ig.Gpt.from_weights({"x": np.zeros(4, np.float32)})


def test_null_handles_are_validation_errors():
    lib = _lib.load_lib()
    out = ctypes.c_void_p()
    assert lib.itts_kv_create(None, 16, 1, ctypes.byref(out)) == _lib.ITTS_E_VALIDATION
    assert "gpt" in _lib.last_error()
    assert lib.itts_gpt_prefill(None, None, 0, None, 0, None, 0, 0, None, 0, None) == _lib.ITTS_E_VALIDATION
