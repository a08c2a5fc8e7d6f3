"""itts_sample_next_token_static, the sampler entry point that allocates nothing, against
itts_sample_next_token on the same inputs.

The static variant keeps its device working set in one array per device that every call
shares, so the checks run two calls in a row with different slice lengths and
parameters: the second call must not see anything the first left behind.  The sampler
is bit-exact, so token, RNG state and penalized logits must be identical."""
import ctypes as C
import gc

import numpy as np
import pytest

import itts_gpt as ig
from itts_gpt import _lib

pytestmark = pytest.mark.gpu

MAX_LOGITS = 16384


def _static_sample(logits, seen, params, state, stream=None):
    """Calls the C entry point directly (host buffers; the default stream unless given)."""
    lib = _lib.load_lib()
    p = params.to_c()
    st = C.c_uint64(state)
    tok = C.c_int32(-7)
    words = np.ascontiguousarray(seen.words, np.uint64)
    rc = lib.itts_sample_next_token_static(logits.ctypes.data, int(logits.size), words.ctypes.data,
                                           C.byref(p), C.byref(st), C.byref(tok), stream)
    return rc, tok.value, st.value


def _cudart():
    """The CUDA runtime the library itself loaded (same soname), for memory queries and
    a stream of our own."""
    rt = C.CDLL("libcudart.so.12")
    rt.cudaMemGetInfo.argtypes = [C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]
    rt.cudaStreamCreate.argtypes = [C.POINTER(C.c_void_p)]
    rt.cudaStreamDestroy.argtypes = [C.c_void_p]
    return rt


def _free_bytes(rt):
    free, total = C.c_size_t(), C.c_size_t()
    assert rt.cudaMemGetInfo(C.byref(free), C.byref(total)) == 0
    return free.value


def _case(seed, n, params):
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 2, n).astype(np.float32)
    x[rng.integers(0, n, 4)] = [7.5, 7.25, 7.0, 6.5]
    seen = ig.SeenTokenBitSet.new_with_initial_tokens()
    for t in rng.integers(0, n, 25):
        seen.insert(int(t))
    return x, seen, params, int(rng.integers(0, 2**63))


# The first three select the top-k <= 64 kernel; the last three the full-sort kernel (top_k 0,
# i.e. every logit a candidate, or top_k above 64).
CASES = [
    (31, MAX_LOGITS, ig.SamplingParams(top_k=50, top_p=0.9, temperature=0.7, repetition_penalty=1.3)),
    (32, 8194, ig.SamplingParams()),
    (33, 8194, ig.SamplingParams(greedy=True, repetition_penalty=10.0)),
    (34, 8194, ig.SamplingParams(top_k=0, top_p=0.9, temperature=0.8)),
    (35, MAX_LOGITS, ig.SamplingParams(top_k=500, top_p=0.95, temperature=1.1, repetition_penalty=2.0)),
    (36, MAX_LOGITS, ig.SamplingParams(top_k=0, top_p=1.0, temperature=0.5)),
]


def test_static_sampler_matches_handle_sampler(small_weights):
    # The static entry point runs first, so that in a fresh process its first call (which
    # sets the device up) is also the first CUDA work of the process.
    got = []
    for seed, n, params in CASES:
        x, seen, p, state = _case(seed, n, params)
        xs = x.copy()
        rc, tok, st = _static_sample(xs, seen, p, state)
        assert rc == 0, _lib.last_error()
        got.append((tok, st, xs))
    gpt = ig.Gpt.from_weights(small_weights, device=0)
    try:
        for (seed, n, params), (tok, st, xs) in zip(CASES, got):
            x, seen, p, state = _case(seed, n, params)
            r = ig.SamplerRng.from_state(state)
            ref_tok = ig.sample_next_token(gpt, x, seen, p, r)
            assert tok == ref_tok, (seed, tok, ref_tok)
            assert st == r.state, seed
            np.testing.assert_array_equal(xs, x)  # penalized logits, bit for bit
            # and again with the handle open: two calls in a row on the shared array
            x2, seen2, p2, state2 = _case(seed, n, params)
            rc, tok2, st2 = _static_sample(x2, seen2, p2, state2)
            assert rc == 0, _lib.last_error()
            assert (tok2, st2) == (ref_tok, r.state)
            np.testing.assert_array_equal(x2, x)
    finally:
        gpt.close()


def test_static_sampler_rejects_oversize_slices():
    x, seen, p, state = _case(40, MAX_LOGITS + 1, ig.SamplingParams())
    before = x.copy()
    rc, tok, st = _static_sample(x, seen, p, state)
    assert rc == 1  # ITTS_E_VALIDATION
    msg = _lib.last_error()
    assert "16384" in msg and "static scratch" in msg, msg
    assert (tok, st) == (-7, state)
    np.testing.assert_array_equal(x, before)
    rc, _, _ = _static_sample(np.zeros(0, np.float32), seen, p, state)
    assert rc == 1
    # a valid call right after the rejections still matches the handle sampler's result
    x, seen, p, state = _case(41, 1000, ig.SamplingParams(top_k=0, top_p=1.0))
    rc, tok, st = _static_sample(x.copy(), seen, p, state)
    assert rc == 0 and 0 <= tok < 1000


def test_static_sampler_allocates_nothing_and_takes_a_stream():
    """After the first call (which sets the device up), further calls leave the device's
    free memory unchanged, and a call on a stream the caller created gives the same
    result as one on the default stream."""
    rt = _cudart()
    x, seen, p, state = _case(50, 8194, ig.SamplingParams(top_k=30, top_p=0.8))
    rc, tok0, st0 = _static_sample(x.copy(), seen, p, state)
    assert rc == 0, _lib.last_error()
    stream = C.c_void_p()
    assert rt.cudaStreamCreate(C.byref(stream)) == 0
    try:
        # one pass first: the CUDA runtime loads each kernel's code on its first launch
        # (lazy module loading), which takes device memory that is not the sampler's
        for seed, n, params in CASES:
            _static_sample(*_case(seed, n, params))
        _static_sample(x.copy(), seen, p, state, stream)
        gc.collect()  # handles of earlier tests freed now, not during the measurement
        before = _free_bytes(rt)
        for seed, n, params in CASES:
            xc, sc, pc, stc = _case(seed, n, params)
            assert _static_sample(xc, sc, pc, stc)[0] == 0, _lib.last_error()
        assert _free_bytes(rt) == before
        for _ in range(2):
            xs = x.copy()
            rc, tok, st = _static_sample(xs, seen, p, state, stream)
            assert rc == 0, _lib.last_error()
            assert (tok, st) == (tok0, st0)
        assert _free_bytes(rt) == before
    finally:
        rt.cudaStreamDestroy(stream)
