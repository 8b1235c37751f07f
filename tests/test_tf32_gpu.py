"""Tensor-core builds vs the CPU oracle (GPU): TF32 (tcgen05 kind::tf32),
TF32X3 (split operands) and BF16 (the transformer's linears on kind::f16 with
bf16 operands, the rest as TF32).

Gate from the north star: per-stem SNR >= 60 dB for the TF32/BF16 builds, on
the benchmark's random-init weights (LayerScale 1e-4). With LayerScale 1 the
transformer's residual branches carry their full weight, a stress case beyond
the benchmark's weights: TF32 still meets 60 dB there; bf16 operands carry
three fewer mantissa bits (about 18 dB less operand SNR), and the BF16 build
is held to 40 dB in that case.
SNR here is energy based, 10*log10(sum ref^2 / sum (ref - x)^2); the
reference's own mean-abs form (fixtures.rs:133-149) is reported beside it.
"""

import numpy as np
import pytest

import oracle
import synth

pytestmark = pytest.mark.gpu


def snr_db(ref, x):
    ref = ref.astype(np.float64)
    err = ref - x
    return 10 * np.log10(np.sum(ref ** 2) / max(np.sum(err ** 2), 1e-300))


def snr_meanabs_db(ref, x):
    ref = ref.astype(np.float64)
    return -20 * np.log10(np.mean(np.abs(ref - x)) / np.sqrt(np.mean(ref ** 2)))


@pytest.mark.parametrize("layer_scale", [1e-4, 1.0])
@pytest.mark.parametrize("precision", ["TF32", "TF32X3", "BF16"])
def test_tensor_core_forward(layer_scale, precision):
    import dmx
    w = synth.random_weights(3, layer_scale=layer_scale, norm_jitter=0.1)
    mix = synth.gaussian_audio(7, 1)
    tr_o, tr_g = {}, {}
    ref = oracle.OracleModel(w).forward(mix, trace=tr_o)
    h = dmx.Handle(synth.write_safetensors(w), device=0, precision=getattr(dmx, precision),
                   max_batch=2)
    h.set_trace(tr_g)
    got = h.forward(mix)
    for name, g in tr_g.items():
        print(f"{name:36s} snr {snr_db(tr_o[name], g):7.2f} dB")
    per_stem = [snr_db(ref[0, s], got[0, s]) for s in range(4)]
    print("per-stem SNR", per_stem, "mean-abs SNR", [snr_meanabs_db(ref[0, s], got[0, s]) for s in range(4)])
    assert np.isfinite(got).all()
    gate = 40.0 if precision == "BF16" and layer_scale == 1.0 else 60.0
    assert min(per_stem) >= gate, per_stem
    if precision == "TF32X3":
        # the split keeps fp32-class accuracy: the FP32 build's max-abs gate
        worst = np.abs(got.astype(np.float64) - ref).reshape(4, -1).max(axis=1)
        print("TF32X3 per-stem max-abs", worst)
        assert worst.max() <= 1e-4, worst


def test_bf16_wide_dconv_runs_on_the_tensor_cores_and_matches_the_oracle():
    """The BF16 build runs the C = 192 DConv layers on the fused tensor-core
    kernel: one launch per spectral row (encoder.2, decoder.1) and the three
    tiled launches over the waveform rows (tencoder.2, tdecoder.1, 5375 frames
    a row). With LayerScale 1 the branch carries its full weight, so the
    layers after it show its single-pass tf32 error undamped."""
    import dmx
    w = synth.random_weights(5, layer_scale=1.0, norm_jitter=0.1)
    mix = synth.gaussian_audio(11, 1)
    tr_o, tr_g = {}, {}
    oracle.OracleModel(w).forward(mix, trace=tr_o)
    h = dmx.Handle(synth.write_safetensors(w), device=0, precision=dmx.BF16, max_batch=1)
    h.set_trace(tr_g)
    got = h.forward(mix)
    assert np.isfinite(got).all()
    h.set_trace(None)
    h.set_stage_timing(True)
    again = h.forward(mix)
    tags = h.stage_times()
    assert np.array_equal(got, again)
    assert "dconv.tc192" in tags and "dconv.tctiled192" in tags, sorted(tags)
    assert not any(t in tags for t in ("dconv.row192", "dconv.tiled192")), sorted(tags)
    for name in ("encoder.2", "tencoder.2", "encoder.3", "tencoder.3"):
        s = snr_db(tr_o[name], tr_g[name])
        print(f"{name:12s} snr {s:7.2f} dB")
        assert s >= 50.0, (name, s)
