"""Pins the CPU oracle to the reference's own known-answer tests.

Every vector here is transcribed from a unit test of the reference project
(paths relative to crates/demucs-core/); the citation is on each test. These
are the golden values the oracle must reproduce before it can check the CUDA
path.
"""

import ctypes
import math

import numpy as np
import pytest

import synth


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def P(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


# --- config (src/demucs/config.rs:453-504) ---------------------------------

def test_training_length_and_hop():
    assert int(39 / 5 * 44100) == 343980 == synth.SEGMENT_SAMPLES
    assert 4096 // 4 == 1024


def test_layer_table_matches_reference_shapes():
    shapes = {name: shape for name, shape, _ in synth.weight_specs()}
    enc = [(shapes[f"encoder.{i}.conv.weight"][1], shapes[f"encoder.{i}.conv.weight"][0]) for i in range(4)]
    assert enc == [(4, 48), (48, 96), (96, 192), (192, 384)]
    tenc = [(shapes[f"tencoder.{i}.conv.weight"][1], shapes[f"tencoder.{i}.conv.weight"][0]) for i in range(4)]
    assert tenc == [(2, 48), (48, 96), (96, 192), (192, 384)]
    # execution order = checkpoint index 3..0 (config.rs:416-418, weights.rs:507-527)
    dec = [tuple(shapes[f"decoder.{j}.conv_tr.weight"][:2]) for j in (3, 2, 1, 0)]
    assert dec == [(384, 192), (192, 96), (96, 48), (48, 16)]
    tdec = [tuple(shapes[f"tdecoder.{j}.conv_tr.weight"][:2]) for j in (3, 2, 1, 0)]
    assert tdec == [(384, 192), (192, 96), (96, 48), (48, 8)]
    assert shapes["freq_emb.embedding.weight"] == (512, 48)
    assert shapes["crosstransformer.layers.0.linear1.weight"] == (2048, 512)
    assert "crosstransformer.layers.1.cross_attn.in_proj_weight" in shapes
    assert "crosstransformer.layers.2.self_attn.in_proj_weight" in shapes
    assert "crosstransformer.layers_t.3.norm3.weight" in shapes
    assert shapes["decoder.3.dconv.layers.0.0.weight"] == (48, 384, 3)  # DConv on the decoder input


def test_parameter_count():
    # htdemucs v4 has 41,984,456 parameters with bottom_channels=512.
    assert sum(int(np.prod(s)) for _, s, _ in synth.weight_specs()) == 41984456


# --- STFT (src/dsp/stft.rs:333-444) ----------------------------------------

def test_hann_window_periodic(oracle_mod):
    out = np.empty(4, np.float32)
    oracle_mod.lib().orc_hann(4, P(out))
    np.testing.assert_allclose(out, [0.0, 0.5, 1.0, 0.5], atol=1e-7)


def test_reflect_padding_mirrors_without_repeating_the_edge(oracle_mod):
    x = f32([1, 2, 3, 4])
    out = np.empty(10, np.float32)
    n = oracle_mod.lib().orc_reflect_pad(P(x), 4, 3, 3, P(out))
    assert n == 10
    assert out.tolist() == [4.0, 3.0, 2.0, 1.0, 2.0, 3.0, 4.0, 3.0, 2.0, 1.0]


def _stft(oracle_mod, x, n_fft, hop, normalized=False):
    x = f32(x)
    rows, samples = x.shape
    frames_guess = 1 + samples // hop + 1
    out = np.zeros((rows, n_fft // 2 + 1, frames_guess, 2), np.float32)
    frames = ctypes.c_int(0)
    rc = oracle_mod.lib().orc_stft(P(x), rows, samples, n_fft, hop, int(normalized), P(out),
                                   ctypes.byref(frames))
    if rc:
        raise ValueError(oracle_mod.lib().orc_last_error().decode())
    flat = out.reshape(-1)[: rows * (n_fft // 2 + 1) * frames.value * 2]
    return flat.reshape(rows, n_fft // 2 + 1, frames.value, 2)


def _istft(oracle_mod, spec, n_fft, hop, normalized=False, length=-1):
    spec = f32(spec)
    rows, bins, frames, _ = spec.shape
    cap = n_fft + hop * (frames - 1)
    out = np.zeros(rows * cap, np.float32)
    n = oracle_mod.lib().orc_istft(P(spec), rows, bins, frames, n_fft, hop, int(normalized),
                                   length, P(out))
    return out[: rows * n].reshape(rows, n)


def test_frame_count_follows_center_padding(oracle_mod):
    assert _stft(oracle_mod, np.zeros((1, 26460)), 2048, 441).shape[2] == 61
    assert _stft(oracle_mod, np.zeros((1, 441 * 60)), 2048, 441).shape[2] == 61


def test_single_bin_sinusoid_lands_in_bin_8(oracle_mod):
    sig = np.sin(2 * np.pi * np.arange(256, dtype=np.float32) / 8.0)
    spec = _stft(oracle_mod, sig[None], 64, 16)
    mag = np.hypot(spec[0, :, 4, 0], spec[0, :, 4, 1])
    assert int(np.argmax(mag)) == 8


def test_forward_then_inverse_reconstructs_interior(oracle_mod):
    t = np.arange(2048, dtype=np.float32)
    sig = np.sin(t * 0.013) * 0.7 + np.cos(t * 0.11) * 0.3
    spec = _stft(oracle_mod, sig[None], 256, 64)
    back = _istft(oracle_mod, spec, 256, 64)
    assert back.shape == (1, 2048)
    assert np.abs(back[0, 300:-300] - sig[300:-300]).max() < 1e-4


def test_normalized_round_trip_and_ratio_16(oracle_mod):
    sig = np.sin(np.arange(1024, dtype=np.float32) * 0.037)
    spec = _stft(oracle_mod, sig[None], 256, 64, normalized=True)
    raw = _stft(oracle_mod, sig[None], 256, 64, normalized=False)
    ratio = np.hypot(*raw[0, 8, 4]) / np.hypot(*spec[0, 8, 4])
    assert abs(ratio - 16.0) < 1e-2
    back = _istft(oracle_mod, spec, 256, 64, normalized=True, length=1024)
    assert np.abs(back[0, 200:-200] - sig[200:-200]).max() < 1e-4


def test_inverse_lengths(oracle_mod):
    spec = np.zeros((2, 1025, 5, 2), np.float32)
    assert _istft(oracle_mod, spec, 2048, 441).shape == (2, 441 * 4)
    assert _istft(oracle_mod, spec[:1], 2048, 441, length=1000).shape == (1, 1000)


def test_reflect_padding_rejects_short_inputs(oracle_mod):
    with pytest.raises(ValueError):
        _stft(oracle_mod, np.zeros((1, 100)), 2048, 441)


# --- pipeline (src/demucs/pipeline.rs:714-772) ------------------------------

def test_transition_window_rises_then_falls(oracle_mod):
    w = np.empty(8, np.float32)
    oracle_mod.lib().orc_transition_weight(8, 1.0, P(w))
    assert abs(w[3] - 1.0) < 1e-6
    assert w[0] < w[1] < w[2]
    assert w[7] < w[6] < w[5]


def _padded_chunk(oracle_mod, mix, offset, length, target):
    mix = f32(mix)
    out = np.empty(target, np.float32)
    oracle_mod.lib().orc_padded_chunk(P(mix), 1, ctypes.c_int64(mix.size), ctypes.c_int64(0),
                                      ctypes.c_int64(0), ctypes.c_int64(offset),
                                      ctypes.c_int64(length), target, P(out))
    return out.tolist()


def test_centred_chunk_takes_context_from_both_sides(oracle_mod):
    assert _padded_chunk(oracle_mod, np.arange(10), 4, 4, 8) == [2, 3, 4, 5, 6, 7, 8, 9]


def test_chunk_at_start_is_zero_padded_on_the_left(oracle_mod):
    assert _padded_chunk(oracle_mod, np.arange(6), 0, 3, 7) == [0, 0, 0, 1, 2, 3, 4]


def test_center_trim_removes_the_larger_half_first():
    # center_trim keeps [delta/2, delta/2 + reference) (pipeline.rs:105-113);
    # the oracle's split pass uses the same start.
    x = np.array([0.0, 1.0, 2.0, 3.0, 4.0])
    delta = 5 - 3
    assert x[delta // 2: delta // 2 + 3].tolist() == [1.0, 2.0, 3.0]


def test_shift_rng_stays_in_range(oracle_mod):
    out = (ctypes.c_uint64 * 1000)()
    oracle_mod.lib().orc_shift_randint(7, 1000, 22050, out)
    assert max(out) <= 22050 and len(set(out)) > 100


def test_normalisation_round_trips(oracle_mod):
    wav = f32([[0.5, -0.25, 1.0, 0.0], [0.5, -0.25, 1.0, 0.0]])
    mean, std = ctypes.c_float(), ctypes.c_float()
    oracle_mod.lib().orc_scan_norm(P(wav), 2, ctypes.c_int64(4), ctypes.byref(mean), ctypes.byref(std))
    back = (wav - mean.value) / std.value * std.value + mean.value
    np.testing.assert_allclose(back, wav, atol=1e-5)


# --- CPU ops (src/demucs/ops.rs:1607-1778, src/ops.rs:239-353) ---------------

def _conv1d(oracle_mod, x, w, b, stride, pad, dil):
    x, w, b = f32(x), f32(w), f32(b)
    B, C, T = x.shape
    oc, _, k = w.shape
    out = np.zeros((B, oc, T * 4 + 16), np.float32)
    t = ctypes.c_int(0)
    oracle_mod.lib().orc_conv1d(P(x), B, C, T, P(w), P(b), oc, k, stride, pad, dil, P(out), ctypes.byref(t))
    return out.reshape(-1)[: B * oc * t.value].reshape(B, oc, t.value)


def test_conv1d_hand_written_correlation(oracle_mod):
    out = _conv1d(oracle_mod, [[[1, 2, 3, 4]]], [[[1, 2]]], [0.5], 1, 0, 1)
    np.testing.assert_allclose(out[0, 0], [1 + 4 + 0.5, 2 + 6 + 0.5, 3 + 8 + 0.5], atol=1e-6)


def test_conv1d_pads_and_strides(oracle_mod):
    out = _conv1d(oracle_mod, [[[1, 2, 3, 4, 5, 6]]], [[[1, 1, 1]]], [0.0], 2, 1, 1)
    np.testing.assert_allclose(out[0, 0], [3, 9, 15], atol=1e-6)


def test_conv1d_dilation(oracle_mod):
    out = _conv1d(oracle_mod, [[[1, 2, 3, 4, 5]]], [[[1, 10]]], [0.0], 1, 2, 2)
    assert out.shape == (1, 1, 7)
    assert abs(out[0, 0, 0] - 10) < 1e-6 and abs(out[0, 0, 2] - 31) < 1e-6 and abs(out[0, 0, 6] - 5) < 1e-6


def test_conv_transpose1d_scatters_taps(oracle_mod):
    x, w, b = f32([[[1, 2]]]), f32([[[1, 10]]]), f32([0.0])
    out = np.zeros(8, np.float32)
    t = ctypes.c_int(0)
    oracle_mod.lib().orc_conv_transpose1d(P(x), 1, 1, 2, P(w), P(b), 1, 2, 2, P(out), ctypes.byref(t))
    assert t.value == 4
    np.testing.assert_allclose(out[:4], [1, 10, 2, 20], atol=1e-6)


def test_conv2d_two_dimensional_kernel(oracle_mod):
    x = f32(np.arange(1, 10).reshape(1, 1, 3, 3))
    w, b = f32([[[[1, 0], [0, 0]]]]), f32([0.0])
    out = np.zeros(4, np.float32)
    oh, ow = ctypes.c_int(0), ctypes.c_int(0)
    oracle_mod.lib().orc_conv2d(P(x), 1, 1, 3, 3, P(w), P(b), 1, 2, 2, 1, 1, 0, 0, P(out),
                                ctypes.byref(oh), ctypes.byref(ow))
    assert (oh.value, ow.value) == (2, 2)
    assert out[0] == 1.0 and out[1] == 2.0 and out[2] == 4.0


def test_group_norm_statistics_and_affine(oracle_mod):
    x = f32([1, 2, 3, 4])
    oracle_mod.lib().orc_group_norm1(P(x), 1, 2, 2, P(f32([1, 1])), P(f32([0, 0])))
    var = np.mean((np.array([1, 2, 3, 4]) - 2.5) ** 2)
    inv = 1 / math.sqrt(var + 1e-5)
    assert abs(x[0] - (1 - 2.5) * inv) < 1e-5 and abs(x[3] - (4 - 2.5) * inv) < 1e-5
    y = f32([0, 1, 0, 1])
    oracle_mod.lib().orc_group_norm1(P(y), 1, 2, 2, P(f32([2, 3])), P(f32([1, -1])))
    inv = 1 / math.sqrt(0.25 + 1e-5)
    n = -0.5 * inv
    assert abs(y[0] - (n * 2 + 1)) < 1e-5 and abs(y[2] - (n * 3 - 1)) < 1e-5 and abs(y[1] - (-n * 2 + 1)) < 1e-5


def test_layer_norm_row(oracle_mod):
    x = f32([[1, 2, 3, 4]])
    out = np.empty_like(x)
    oracle_mod.lib().orc_layer_norm(P(x), 1, 4, P(f32([1] * 4)), P(f32([0] * 4)), P(out))
    inv = 1 / math.sqrt(1.25 + 1e-5)
    assert abs(out[0, 0] - (-1.5) * inv) < 1e-5 and abs(out[0, 3] - 1.5 * inv) < 1e-5


def test_glu_gates_first_half(oracle_mod):
    x = f32([1, 1, 2, 2, 0, 0, 0, 0])
    out = np.empty(4, np.float32)
    oracle_mod.lib().orc_glu(P(x), 1, 4, 2, P(out))
    assert abs(out[0] - 0.5) < 1e-6 and abs(out[3] - 1.0) < 1e-6


def _attention(oracle_mod, q, k, v, scale):
    q, k, v = f32(q), f32(k), f32(v)
    out = np.empty((q.shape[0], v.shape[1]), np.float32)
    oracle_mod.lib().orc_attention_head(P(q), P(k), P(v), q.shape[0], k.shape[0], q.shape[1], scale, P(out))
    return out


def test_attention_is_scaled_softmax_times_v(oracle_mod):
    out = _attention(oracle_mod, [[1, 0]], [[1, 0], [0, 1]], [[2, 0], [0, 8]], 1.0)
    a = math.e / (math.e + 1)
    assert abs(out[0, 0] - 2 * a) < 1e-5 and abs(out[0, 1] - 8 * (1 - a)) < 1e-5


def test_attention_known_values_identity_qk(oracle_mod):
    # tests/gpu_htdemucs.rs:531-590: Q=K=I, V=[[1,2],[3,4]], scale 1/sqrt(2)
    out = _attention(oracle_mod, np.eye(2), np.eye(2), [[1, 2], [3, 4]], 1 / math.sqrt(2))
    np.testing.assert_allclose(out.reshape(-1), [1.660, 2.660, 2.340, 3.340], atol=2e-3)


def test_std_unbiased(oracle_mod):
    v = f32([1, 2, 3, 4])
    L = oracle_mod.lib()
    L.orc_std_unbiased.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.c_int]
    assert abs(L.orc_std_unbiased(P(v), 4) - math.sqrt(5 / 3)) < 1e-6


def test_gelu_matches_torch_exact_gelu(oracle_mod):
    g = oracle_mod.lib().orc_gelu
    assert abs(g(0.0)) < 1e-7
    assert abs(g(1.0) - 0.84134471) < 1e-5
    assert abs(g(-1.0) + 0.15865529) < 1e-5
    assert abs(g(2.0) - 1.95449996) < 1e-5
    assert abs(g(-3.0) + 0.00404987) < 1e-6
    assert g(20.0) > 19.9 and abs(g(-20.0)) < 1e-6


# --- streaming OLA with an identity forward (tests/streaming_ola.rs:62-233) -----

def _identity(padded):
    return np.repeat(padded[:, None], 4, axis=1)


def _synthetic_mix(length):
    i = np.arange(2 * length)
    return (((i % 97) - 48) / 48.0).astype(np.float32).reshape(2, length)


@pytest.mark.parametrize("shifts", [0, 1, 2])
def test_identity_forward_reconstructs_the_mix(oracle_mod, shifts):
    seg = int(44100 * 0.25)
    mix = _synthetic_mix(seg * 5 // 2)
    stems = oracle_mod.separate_with(_identity, mix, seg, shifts=shifts)
    for s in range(4):
        np.testing.assert_allclose(stems[s], mix, atol=2e-6)


def test_grouped_chunks_match_one_at_a_time_bitwise(oracle_mod):
    # pipeline.rs:778-838: batching chunks is a scheduling change only.
    seg = int(44100 * 0.25)
    mix = _synthetic_mix(seg * 5 // 2)
    rng = np.random.default_rng(3)
    scale = rng.standard_normal((1, 4, 2, 1)).astype(np.float32)
    fwd = lambda p: (_identity(p) * scale + np.float32(0.01) * np.roll(_identity(p), 3, axis=-1)).astype(np.float32)
    one = oracle_mod.separate_with(fwd, mix, seg, shifts=1, batch=1)
    three = oracle_mod.separate_with(fwd, mix, seg, shifts=1, batch=3)
    assert np.array_equal(one, three)


def test_half_decoding_known_answers():
    # safetensors.rs:194-203 and 228-234: binary16 -> binary32, subnormals and infinities
    # included. The product's F16 loader is checked against numpy's IEEE float16 upcast on
    # the GPU (test_forward_gpu.py); these are the reference's own known answers for it.
    import numpy as np

    bits = np.array([0x3C00, 0xC000, 0x3800, 0x0000, 0x0001, 0x7C00, 0xFC00, 0x7E00],
                    dtype="<u2")
    v = bits.view(np.float16).astype(np.float32)
    assert list(v[:4]) == [1.0, -2.0, 0.5, 0.0]
    assert v[4] == np.float32(2.0 ** -24)
    assert np.isposinf(v[5]) and np.isneginf(v[6]) and np.isnan(v[7])
