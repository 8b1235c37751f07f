"""CUDA forward vs the CPU oracle on seeded weights and audio (GPU).

The gate for the FP32 build is the north-star tolerance: max-abs <= 1e-4 per
stem against the reference CPU path (restated by the oracle), at the
benchmark's configuration 1 (one 343980-sample stereo segment, N(0, 0.1^2)
audio, random-init weights with LayerScale 1e-4) and with LayerScale 1 so the
residual branches carry weight.
"""

import numpy as np
import pytest

import oracle
import synth

pytestmark = pytest.mark.gpu


def _handle(weights, max_batch=4):
    import dmx
    return dmx.Handle(synth.write_safetensors(weights), device=0, max_batch=max_batch)


def _per_stem_maxabs(a, b):
    return np.abs(a.astype(np.float64) - b).reshape(a.shape[0], 4, -1).max(axis=-1)


@pytest.mark.parametrize("layer_scale", [1e-4, 1.0])
def test_forward_matches_oracle_fp32(layer_scale):
    w = synth.random_weights(3, layer_scale=layer_scale, norm_jitter=0.1)
    mix = synth.gaussian_audio(7, 1)
    ref = oracle.OracleModel(w).forward(mix)
    got = _handle(w).forward(mix)
    assert got.shape == ref.shape
    worst = _per_stem_maxabs(got, ref)
    assert np.isfinite(got).all()
    assert worst.max() <= 1e-4, worst


def test_stage_traces_match_oracle():
    w = synth.random_weights(4, layer_scale=1.0, norm_jitter=0.1)
    mix = synth.gaussian_audio(8, 1)
    tr_o, tr_g = {}, {}
    oracle.OracleModel(w).forward(mix, trace=tr_o)
    h = _handle(w)
    h.set_trace(tr_g)
    h.forward(mix)
    assert tr_g, "no traces recorded"
    for name, got in tr_g.items():
        ref = tr_o[name]
        assert got.shape == ref.shape, (name, got.shape, ref.shape)
        rms = np.sqrt(np.mean(ref.astype(np.float64) ** 2))
        rel = np.mean(np.abs(got.astype(np.float64) - ref)) / rms
        assert rel < 1e-4, f"{name}: mean-abs/rms {rel:.3e}"


@pytest.mark.parametrize("precision", ["FP32", "TF32", "TF32X3"])
def test_batch_independence_is_bitwise(precision):
    # demucs_alignment.rs:232-261 asks element 0 of a batch-2 run to match the single run
    # above 100 dB. Here every per-segment moment is reduced in an order fixed by the
    # position inside the segment, so a segment's output does not depend on its batch
    # neighbours or its place in the batch: the comparison is bit for bit, at batch
    # sizes whose tiles straddle segments (the 1344-token time stream is 10.5 row tiles)
    import dmx

    w = synth.random_weights(5)
    single = synth.lcg_audio(12345, (1, 2, synth.SEGMENT_SAMPLES), 0.1)
    others = synth.gaussian_audio(9, 4, std=0.05)
    h = dmx.Handle(synth.write_safetensors(w), device=0, max_batch=5,
                   precision=getattr(dmx, precision))
    one = h.forward(single)
    for at in (0, 1, 4):  # first, odd and last place in a batch of five
        batch = np.insert(others, at, single[0], axis=0)
        got = h.forward(batch)
        assert np.array_equal(got[at], one[0]), (precision, at)
    assert np.array_equal(h.forward(single), one)  # and run to run


@pytest.mark.parametrize("dtype", ["F16", "BF16"])
def test_half_precision_checkpoints_load_as_their_f32_upcast(dtype):
    # the published checkpoints store F16 (safetensors.rs:5-9, 110-135): a blob in F16 or
    # BF16 must load exactly as the F32 blob of the same (rounded) values
    import dmx

    w = synth.random_weights(4)
    rounded = synth.read_safetensors(synth.write_safetensors(w))  # f32 copies
    if dtype == "F16":
        rounded = {k: v.astype(np.float16).astype(np.float32) for k, v in rounded.items()}
    else:
        rounded = {k: (((v.view(np.uint32).astype(np.uint64) + 0x7FFF
                         + ((v.view(np.uint32) >> 16) & 1)) >> 16) << 16)
                   .astype(np.uint32).view(np.float32) for k, v in rounded.items()}
    mix = synth.gaussian_audio(8, 1)
    got = dmx.Handle(synth.write_safetensors(w, dtype=dtype), device=0, max_batch=1).forward(mix)
    ref = dmx.Handle(synth.write_safetensors(rounded), device=0, max_batch=1).forward(mix)
    assert np.array_equal(got, ref)


def test_torch_zip_checkpoint_loads_as_the_safetensors_blob():
    # a torch.save archive of the same state dict (the demucs .th package layout) gives
    # the same network: the forward is bit for bit the safetensors blob's
    import fractions
    import io
    from collections import OrderedDict

    import torch
    import dmx

    w = synth.random_weights(6)
    buf = io.BytesIO()
    torch.save({"klass": fractions.Fraction, "args": (),
                "kwargs": {"channels": 48, "segment": fractions.Fraction(39, 5)},
                "state": OrderedDict((k, torch.from_numpy(v.copy())) for k, v in w.items())}, buf)
    mix = synth.gaussian_audio(10, 1)
    got = dmx.Handle(buf.getvalue(), device=0, max_batch=1, precision=dmx.TF32).forward(mix)
    ref = dmx.Handle(synth.write_safetensors(w), device=0, max_batch=1, precision=dmx.TF32).forward(mix)
    assert np.array_equal(got, ref)
