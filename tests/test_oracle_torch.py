"""Cross-checks the C++ oracle against a float64 PyTorch restatement of the
same forward (tests/torch_reference.py). PyTorch's stft/istft, conv,
group/layer norm and attention are the primitives the reference transcribes,
so agreement here pins the oracle's layer semantics end to end."""

import numpy as np
import pytest
import torch

import oracle
import synth
import torch_reference


@pytest.mark.parametrize("layer_scale", [1e-4, 1.0])
def test_oracle_matches_torch_float64(layer_scale):
    torch.set_num_threads(max(1, torch.get_num_threads()))
    w = synth.random_weights(11, layer_scale=layer_scale, norm_jitter=0.1)
    mix = synth.gaussian_audio(5, 1)
    tr_o, tr_t = {}, {}
    out_o = oracle.OracleModel(w).forward(mix, trace=tr_o)
    out_t = torch_reference.forward(w, mix, trace=tr_t)
    for name, ref in tr_t.items():
        got = tr_o[name]
        rms = np.sqrt(np.mean(ref.astype(np.float64) ** 2))
        rel = np.mean(np.abs(got.astype(np.float64) - ref)) / rms
        assert rel < 2e-5, f"{name}: mean-abs/rms {rel:.3e}"
    err = np.abs(out_o.astype(np.float64) - out_t)
    assert err.max() < 1e-5 * max(1.0, np.abs(out_t).max()), err.max()
