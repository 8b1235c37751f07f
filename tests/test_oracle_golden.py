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


def test_center_trim_removes_the_larger_half_first(oracle_mod):
    # pipeline.rs:765-771: center_trim of [0, 1, 2, 3, 4] to 3 samples is [1, 2, 3]; the
    # oracle's split pass trims each chunk's output with the same function
    x = f32([[0.0, 1.0, 2.0, 3.0, 4.0]])
    out = np.full((1, 5), -1.0, np.float32)
    kept = oracle_mod.lib().orc_center_trim(P(x), 1, 5, 3, P(out))
    assert kept == 3 and out[0, :3].tolist() == [1.0, 2.0, 3.0]
    out = np.full((2, 4), -1.0, np.float32)  # an even excess: one sample off each end
    x2 = f32([[0, 1, 2, 3, 4, 5], [6, 7, 8, 9, 10, 11]])
    assert oracle_mod.lib().orc_center_trim(P(x2), 2, 6, 4, P(out)) == 4
    assert out.tolist() == [[1, 2, 3, 4], [7, 8, 9, 10]]


def test_shift_rng_stays_in_range(oracle_mod):
    # pipeline.rs:773-780
    out = (ctypes.c_uint64 * 1000)()
    oracle_mod.lib().orc_shift_randint(7, 1000, 22050, out)
    assert max(out) <= 22050 and len(set(out)) > 100


# ShiftRng (pipeline.rs:136-151): state0 = seed*A + 1; per draw state = state*A + C (mod
# 2^64), value = (state >> 33) % (max + 1), A = 6364136223846793005,
# C = 1442695040888963407. From seed 0x5eed_1234 (pipeline.rs:417) with max 22050 the first
# draws are, worked out by hand with exact integer arithmetic:
#   state0 = 0x5eed1234*A + 1 mod 2^64, state1 = state0*A + C mod 2^64, ...
SHIFT_DRAWS_5EED1234 = [11660, 18630, 3283, 15206]
SHIFT_DRAWS_SEED_7 = [17341, 18673, 12503]


def test_shift_rng_first_draws_are_pinned(oracle_mod):
    out = (ctypes.c_uint64 * 4)()
    oracle_mod.lib().orc_shift_randint(0x5EED1234, 4, 22050, out)
    assert list(out) == SHIFT_DRAWS_5EED1234
    out = (ctypes.c_uint64 * 3)()
    oracle_mod.lib().orc_shift_randint(7, 3, 22050, out)
    assert list(out) == SHIFT_DRAWS_SEED_7


def test_product_shift_offsets_are_the_pinned_draws():
    # the one generator the device drivers and the rank planner use (dmx_shift_offsets)
    import dmx
    import shard

    assert dmx.shift_offsets(4, 22050) == SHIFT_DRAWS_5EED1234
    assert shard.shift_offsets(2, 22050) == SHIFT_DRAWS_5EED1234[:2]
    assert shard.plan(10_584_000, 1, shifts=1).offset == SHIFT_DRAWS_5EED1234[0]


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


def _st_blob(header, data):
    # safetensors.rs:172-177: 8-byte little-endian header size, JSON header, data
    import json
    import struct

    text = json.dumps(header, separators=(",", ":")).encode()
    return struct.pack("<Q", len(text)) + text + data


def test_half_decoding_known_answers_through_the_product_loader():
    # safetensors.rs:194-203 and 228-234: binary16 -> binary32, subnormals and infinities
    # included, decoded by the library's own loader (dmx_read_tensor, the path dmx_create
    # takes for F16 checkpoints)
    import dmx

    bits = np.array([0x3C00, 0xC000, 0x3800, 0x0000, 0x0001, 0x7C00, 0xFC00, 0x7E00, 0x8000,
                     0x7BFF, 0x03FF], dtype="<u2")
    blob = _st_blob({"w": {"dtype": "F16", "shape": [len(bits)],
                           "data_offsets": [0, 2 * len(bits)]}}, bits.tobytes())
    v = dmx.read_tensor(blob, "w")
    assert v.dtype == np.float32 and v.shape == (len(bits),)
    assert list(v[:4]) == [1.0, -2.0, 0.5, 0.0]
    assert v[4] == np.float32(2.0 ** -24)                      # smallest subnormal
    assert np.isposinf(v[5]) and np.isneginf(v[6]) and np.isnan(v[7])
    assert v[8] == 0.0 and np.signbit(v[8])                    # negative zero
    assert v[9] == np.float32(65504.0)                         # largest finite
    assert v[10] == np.float32(1023 * 2.0 ** -24)              # largest subnormal


def test_safetensors_known_answers_through_the_product_loader():
    # safetensors.rs:179-225: an F32 tensor round trips with its shape, __metadata__ is
    # not a tensor, truncated data and a header longer than the file are rejected
    import struct

    import pytest

    import dmx

    data = np.array([1.0, 2.0, 3.0, 4.0], "<f4").tobytes()
    blob = _st_blob({"w": {"dtype": "F32", "shape": [2, 2], "data_offsets": [0, 16]}}, data)
    w = dmx.read_tensor(blob, "w")
    assert w.shape == (2, 2) and w[0, 1] == 2.0 and w[1, 1] == 4.0
    meta = _st_blob({"__metadata__": {"klass": "demucs.htdemucs.HTDemucs"},
                     "w": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]}},
                    np.array([0.5], "<f4").tobytes())
    assert dmx.read_tensor(meta, "w").tolist() == [0.5]
    with pytest.raises(dmx.DmxError, match="missing tensor __metadata__") as e:
        dmx.read_tensor(meta, "__metadata__")
    assert e.value.code == 2
    short = _st_blob({"w": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}, b"\0" * 8)
    with pytest.raises(dmx.DmxError, match="data_offsets") as e:
        dmx.read_tensor(short, "w")
    assert e.value.code == 2
    with pytest.raises(dmx.DmxError, match="header runs past the blob"):
        dmx.read_tensor(struct.pack("<Q", 4096), "w")
    # a header size near 2^64 must not wrap the bounds check
    with pytest.raises(dmx.DmxError, match="header runs past the blob"):
        dmx.read_tensor(struct.pack("<Q", (1 << 64) - 4) + b"{}", "w")
    # a shape whose element count overflows is rejected, not wrapped
    huge = _st_blob({"w": {"dtype": "F32", "shape": [1 << 40, 1 << 40], "data_offsets": [0, 0]}}, b"")
    with pytest.raises(dmx.DmxError, match="shape larger than the blob"):
        dmx.read_tensor(huge, "w")


def test_chunk_counts_are_the_reference_known_answers():
    # streaming.rs:856-861 through the product's dmx_num_chunks (stride from the overlap)
    import dmx

    assert dmx.num_chunks(100, 200, 0.25) == 1
    assert dmx.num_chunks(200, 200, 0.25) == 2
    assert dmx.num_chunks(343980 * 2, 343980, 0.25) == 3
