"""The SemanticCodec decode restatement (oracle/, orc_codec_decode) against an independent
implementation of the same model in torch (CPU): conv1d with the MLX channels-last weights
transposed to torch's [C_out, C_in, K], exact GELU, layer_norm (eps 1e-6), nearest x2
repeat (crates/core/src/models/codec.rs:202-239, convnext.rs:66-73)."""
import numpy as np
import torch
import torch.nn.functional as F

import oracle as orc
from itts_gpt.synth import make_codec_weights


def torch_decode(t, codes):
    g = {k: torch.from_numpy(v) for k, v in t.items()}
    conv = lambda x, w, b, pad: F.conv1d(x.T[None], w.permute(0, 2, 1), b, padding=pad)[0].T  # [T, C]
    z = g["quantizer.quantizers.0.codebook.weight"][torch.as_tensor(codes, dtype=torch.long)]
    x = conv(z, g["quantizer.quantizers.0.out_project.weight"], g["quantizer.quantizers.0.out_project.bias"], 0)
    ek = g["decoder.0.embed.weight"].shape[1]
    h = conv(x, g["decoder.0.embed.weight"], g["decoder.0.embed.bias"], (ek - 1) // 2)
    h = F.layer_norm(h, h.shape[-1:], g["decoder.0.norm.weight"], g["decoder.0.norm.bias"], 1e-6)
    l = 0
    while f"decoder.0.convnext.{l}.gamma" in g:
        p = f"decoder.0.convnext.{l}."
        w = g[p + "dwconv.weight"]  # [C, K, 1]
        y = F.conv1d(h.T[None], w.permute(0, 2, 1), g[p + "dwconv.bias"], padding=(w.shape[1] - 1) // 2,
                     groups=w.shape[0])[0].T
        y = F.layer_norm(y, y.shape[-1:], g[p + "norm.weight"], g[p + "norm.bias"], 1e-6)
        y = F.gelu(y @ g[p + "pwconv1.weight"].T + g[p + "pwconv1.bias"])
        y = y @ g[p + "pwconv2.weight"].T + g[p + "pwconv2.bias"]
        h = h + g[p + "gamma"] * y
        l += 1
    h = F.layer_norm(h, h.shape[-1:], g["decoder.0.final_layer_norm.weight"],
                     g["decoder.0.final_layer_norm.bias"], 1e-6)
    h = h @ g["decoder.1.weight"].T + g["decoder.1.bias"]
    h = torch.repeat_interleave(h, 2, dim=0)
    uk = g["up.weight"].shape[1]
    return conv(h, g["up.weight"], g["up.bias"], (uk - 1) // 2).numpy()


def test_oracle_codec_matches_torch():
    t = make_codec_weights(seed=5, n_layers=3, hidden=96, dim=32, inter=64, n_codes=200)
    oc = orc.OracleCodec(t)
    for T in (1, 2, 9, 40):
        codes = np.random.default_rng(T).integers(0, 200, T)
        got, ref = oc.decode(codes), torch_decode(t, codes)
        assert got.shape == (2 * T, 96)
        np.testing.assert_allclose(got, ref, atol=2e-5 * max(1.0, np.abs(ref).max()), rtol=0)


def test_oracle_codec_rejects_bad_codes():
    t = make_codec_weights(seed=6, n_layers=1, hidden=32, dim=32, inter=32, n_codes=16)
    oc = orc.OracleCodec(t)
    import pytest
    with pytest.raises(orc.OracleError):
        oc.decode([])
    with pytest.raises(orc.OracleError):
        oc.decode([3, 16])
