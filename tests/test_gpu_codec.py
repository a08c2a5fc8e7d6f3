"""SemanticCodec decode on the device (itts_codec_*) against the CPU checker, at the
checkpoint's geometry (12 ConvNeXt blocks, hidden 1024, backbone 384, intermediate 2048,
codebook 8192 x 8; crates/core/src/models/codec.rs:27-42).  Both sides compute in fp32; the
bound is max |diff| <= 2e-4 x max |reference| (summation order and erf rounding only)."""
import numpy as np
import pytest

import itts_gpt as ig
import oracle as orc
from itts_gpt.synth import make_codec_weights, save_safetensors

pytestmark = pytest.mark.gpu

REL = 2e-4


@pytest.fixture(scope="module")
def codec():
    w = make_codec_weights(seed=77)
    c = ig.SemanticCodec.from_weights(w, device=0)
    yield c, orc.OracleCodec(w), w
    c.close()


def _check(got, ref, what):
    err = float(np.max(np.abs(got - ref)))
    bound = REL * max(1.0, float(np.max(np.abs(ref))))
    assert err <= bound, f"{what}: max |diff| {err:.3e} > {bound:.3e}"
    return err


@pytest.mark.parametrize("T", [1, 2, 37, 300])
def test_codec_decode_matches_checker(codec, T):
    c, oc, _ = codec
    assert c.num_layers() == 12 and (c.hidden, c.dim, c.inter, c.n_codes) == (1024, 384, 2048, 8192)
    codes = np.random.default_rng(T).integers(0, 8192, T)
    got = c.decode(codes)
    assert got.shape == (2 * T, 1024) and np.isfinite(got).all()
    err = _check(got, oc.decode(codes), f"T={T}")
    print(f"codec decode T={T}: max |diff| {err:.2e}, device {c.last_device_ms:.3f} ms")


def test_codec_load_from_path_and_validation(codec, tmp_path):
    c, _, w = codec
    path = tmp_path / "semantic_codec.safetensors"
    save_safetensors(str(path), w)
    c2 = ig.SemanticCodec.load_from_path(str(path))
    try:
        codes = [5, 8191, 0, 4096, 77]
        np.testing.assert_array_equal(c2.decode(codes), c.decode(codes))
    finally:
        c2.close()
    with pytest.raises(ig.ValidationError, match="T must be >= 1"):
        c.decode([])
    with pytest.raises(ig.ValidationError, match="out of range"):
        c.decode([1, 8192])
    bad = dict(w)
    del bad["up.bias"]
    with pytest.raises(ig.WeightLoadError, match="up.bias"):
        ig.SemanticCodec.from_weights(bad)


def test_generated_codes_through_the_codec(small_weights, small_cfg, codec):
    """The step after the decoder (engine/actor.rs:597-615): greedy codes from the decoder,
    then their features."""
    c, oc, _ = codec
    from itts_gpt.synth import make_conds, make_text
    gpt = ig.Gpt.from_weights(small_weights)
    try:
        codes = ig.generate_codes(gpt, make_text(12, small_cfg.text_vocab, seed=1), make_conds(small_cfg.d, 3, seed=2),
                                  1, ig.KvCache(gpt, 256), ig.SamplingParams(greedy=True, max_mel_tokens=24),
                                  ig.SamplerRng(0))
    finally:
        gpt.close()
    assert codes and all(0 <= x < 8192 for x in codes)
    _check(c.decode(codes), oc.decode(codes), "generated codes")
