"""Seeded synthetic inputs for the HTDemucs v4 segment forward.

Everything the benchmarks and the parity tests feed the forward is made here,
from a seed, so the CUDA path and the CPU oracle read identical bytes:

* ``weight_specs`` lists every tensor the reference loads, by its PyTorch name
  and shape (crates/demucs-core/src/demucs/weights.rs:211-578; the layer table
  of crates/demucs-core/src/demucs/config.rs:325-445).
* ``random_weights`` fills them the way an untrained PyTorch module would:
  uniform(-1/sqrt(fan_in), 1/sqrt(fan_in)) for conv/linear weights and biases,
  norms at gamma=1 beta=0, LayerScale at ``layer_scale`` (1e-4 by default, the
  value the benchmark configuration names) and the frequency embedding drawn
  N(0, 1)/emb_scale so the loaded (x emb_scale) table is N(0, 1).
* ``write_safetensors`` / ``read_safetensors`` speak the plain safetensors
  container (8-byte little-endian header length, JSON header, raw f32 data),
  which is what ``dmx_create`` takes.
* ``gaussian_audio`` and ``pink_noise`` make the test and benchmark signals.
"""

from __future__ import annotations

import json
import struct
from collections import OrderedDict

import numpy as np

# Default HTDemucs v4 configuration (crates/demucs-core/src/demucs/config.rs:43-71).
SOURCES = ("drums", "bass", "other", "vocals")
AUDIO_CHANNELS = 2
SAMPLERATE = 44100
SEGMENT_SAMPLES = 343980  # int(39/5 * 44100), config.rs:222-224
CHANNELS = 48
DEPTH = 4
DCONV_COMPRESS = 8
DCONV_DEPTH = 2
BOTTOM = 512
T_LAYERS = 5
T_HIDDEN = 2048
EMB_SCALE = 10.0


def weight_specs():
    """(name, shape, kind) for every tensor, in a fixed order.

    ``kind`` says how ``random_weights`` fills it: ``w``/``b`` share a fan-in
    bound, ``g`` is a norm gain (1), ``z`` a norm bias (0), ``s`` a LayerScale,
    ``e`` the frequency embedding.
    """
    specs = []

    def conv(prefix, shape):
        fan_in = int(np.prod(shape[1:]))
        specs.append((f"{prefix}.weight", tuple(shape), ("w", fan_in)))
        specs.append((f"{prefix}.bias", (shape[0],), ("w", fan_in)))

    def conv_tr(prefix, shape):
        # nn.ConvTranspose: weight (in, out, k...); PyTorch's fan-in for the
        # uniform bound is computed from dim 1 (out) times the kernel.
        fan_in = int(shape[1] * np.prod(shape[2:]))
        specs.append((f"{prefix}.weight", tuple(shape), ("w", fan_in)))
        specs.append((f"{prefix}.bias", (shape[1],), ("w", fan_in)))

    def norm(prefix, c):
        specs.append((f"{prefix}.weight", (c,), ("g", 0)))
        specs.append((f"{prefix}.bias", (c,), ("z", 0)))

    def dconv(prefix, c, k):
        hidden = c // DCONV_COMPRESS
        for d in range(DCONV_DEPTH):
            at = f"{prefix}.dconv.layers.{d}"
            conv(f"{at}.0", (hidden, c, 3) if k == 1 else (hidden, c, 3))
            norm(f"{at}.1", hidden)
            conv(f"{at}.3", (2 * c, hidden, 1))
            norm(f"{at}.4", 2 * c)
            specs.append((f"{at}.6.scale", (c,), ("s", 0)))

    chin_z, chin, chout = AUDIO_CHANNELS * 2, AUDIO_CHANNELS, CHANNELS
    levels = []
    for i in range(DEPTH):
        levels.append((chin_z, chin, chout))
        conv(f"encoder.{i}.conv", (chout, chin_z, 8, 1))
        conv(f"encoder.{i}.rewrite", (2 * chout, chout, 1, 1))
        dconv(f"encoder.{i}", chout, 2)
        conv(f"tencoder.{i}.conv", (chout, chin, 8))
        conv(f"tencoder.{i}.rewrite", (2 * chout, chout, 1))
        dconv(f"tencoder.{i}", chout, 1)
        chin_z, chin = chout, chout
        chout *= 2
    # Decoders, construction index j: freq j maps 48*2^j -> (16 | 48*2^(j-1)),
    # time j maps 48*2^j -> (8 | 48*2^(j-1)) (config.rs:375-404).
    for j in range(DEPTH):
        cin = CHANNELS * (2 ** j)
        cout_f = AUDIO_CHANNELS * len(SOURCES) * 2 if j == 0 else CHANNELS * 2 ** (j - 1)
        cout_t = AUDIO_CHANNELS * len(SOURCES) if j == 0 else CHANNELS * 2 ** (j - 1)
        conv_tr(f"decoder.{j}.conv_tr", (cin, cout_f, 8, 1))
        conv(f"decoder.{j}.rewrite", (2 * cin, cin, 3, 3))
        dconv(f"decoder.{j}", cin, 2)
        conv_tr(f"tdecoder.{j}.conv_tr", (cin, cout_t, 8))
        conv(f"tdecoder.{j}.rewrite", (2 * cin, cin, 3))
        dconv(f"tdecoder.{j}", cin, 1)
    specs.append(("freq_emb.embedding.weight", (512, CHANNELS), ("e", 0)))
    pre = CHANNELS * 2 ** (DEPTH - 1)
    for name in ("channel_upsampler", "channel_upsampler_t"):
        conv(name, (BOTTOM, pre, 1))
    for name in ("channel_downsampler", "channel_downsampler_t"):
        conv(name, (pre, BOTTOM, 1))
    norm("crosstransformer.norm_in", BOTTOM)
    norm("crosstransformer.norm_in_t", BOTTOM)
    for stream in ("layers", "layers_t"):
        for l in range(T_LAYERS):
            cross = l % 2 == 1  # weights.rs:544
            at = f"crosstransformer.{stream}.{l}"
            attn = f"{at}.{'cross_attn' if cross else 'self_attn'}"
            specs.append((f"{attn}.in_proj_weight", (3 * BOTTOM, BOTTOM), ("w", BOTTOM)))
            specs.append((f"{attn}.in_proj_bias", (3 * BOTTOM,), ("w", BOTTOM)))
            specs.append((f"{attn}.out_proj.weight", (BOTTOM, BOTTOM), ("w", BOTTOM)))
            specs.append((f"{attn}.out_proj.bias", (BOTTOM,), ("w", BOTTOM)))
            specs.append((f"{at}.linear1.weight", (T_HIDDEN, BOTTOM), ("w", BOTTOM)))
            specs.append((f"{at}.linear1.bias", (T_HIDDEN,), ("w", BOTTOM)))
            specs.append((f"{at}.linear2.weight", (BOTTOM, T_HIDDEN), ("w", T_HIDDEN)))
            specs.append((f"{at}.linear2.bias", (BOTTOM,), ("w", T_HIDDEN)))
            norm(f"{at}.norm1", BOTTOM)
            norm(f"{at}.norm2", BOTTOM)
            if cross:
                norm(f"{at}.norm3", BOTTOM)
            norm(f"{at}.norm_out", BOTTOM)
            specs.append((f"{at}.gamma_1.scale", (BOTTOM,), ("s", 0)))
            specs.append((f"{at}.gamma_2.scale", (BOTTOM,), ("s", 0)))
    return specs


def random_weights(seed: int = 0, layer_scale: float = 1e-4, norm_jitter: float = 0.0):
    """Seeded random-init weights, ordered like ``weight_specs``.

    ``norm_jitter`` > 0 perturbs the norm gains/biases (gain 1 + j*N(0,1),
    bias j*N(0,1)) so kernel tests exercise the affine terms; the benchmark
    configuration keeps the PyTorch defaults (0).
    """
    rng = np.random.default_rng(seed)
    out = OrderedDict()
    for name, shape, (kind, fan_in) in weight_specs():
        if kind == "w":
            bound = 1.0 / np.sqrt(fan_in)
            value = rng.uniform(-bound, bound, size=shape)
        elif kind == "g":
            value = np.ones(shape) + (norm_jitter * rng.standard_normal(shape) if norm_jitter else 0)
        elif kind == "z":
            value = np.zeros(shape) + (norm_jitter * rng.standard_normal(shape) if norm_jitter else 0)
        elif kind == "s":
            value = np.full(shape, layer_scale)
        elif kind == "e":
            value = rng.standard_normal(shape) / EMB_SCALE
        else:  # pragma: no cover
            raise ValueError(kind)
        out[name] = np.ascontiguousarray(value, dtype=np.float32)
    return out


def _encode(value, dtype):
    """Raw little-endian bytes of an f32 array stored as ``dtype``."""
    if dtype == "F32":
        return np.ascontiguousarray(value, dtype="<f4").tobytes()
    if dtype == "F16":
        return np.ascontiguousarray(value, dtype="<f2").tobytes()
    if dtype == "BF16":  # round to nearest even on the upper 16 bits
        u = np.ascontiguousarray(value, dtype=np.float32).view(np.uint32).astype(np.uint64)
        u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
        return u.astype("<u2").tobytes()
    if dtype == "F64":
        return np.ascontiguousarray(value, dtype="<f8").tobytes()
    raise ValueError(dtype)


def write_safetensors(tensors, metadata=None, dtype: str = "F32") -> bytes:
    """Serialise ``{name: f32 array}`` as a safetensors blob, every tensor
    stored as ``dtype`` (F32, F16 — the published checkpoints' format — BF16
    or F64)."""
    header = OrderedDict()
    offset = 0
    chunks = []
    for name, value in tensors.items():
        value = np.ascontiguousarray(value, dtype=np.float32)
        raw = _encode(value, dtype)
        header[name] = {"dtype": dtype, "shape": list(value.shape),
                        "data_offsets": [offset, offset + len(raw)]}
        offset += len(raw)
        chunks.append(raw)
    if metadata:
        header["__metadata__"] = dict(metadata)
    text = json.dumps(header, separators=(",", ":")).encode()
    text += b" " * ((8 - len(text) % 8) % 8)
    return struct.pack("<Q", len(text)) + text + b"".join(chunks)


def read_safetensors(blob: bytes):
    """Parse a safetensors blob of F32 tensors into ``{name: array}``."""
    (n,) = struct.unpack("<Q", blob[:8])
    header = json.loads(blob[8:8 + n])
    base = 8 + n
    out = OrderedDict()
    for name, info in header.items():
        if name == "__metadata__":
            continue
        if info["dtype"] != "F32":
            raise ValueError(f"{name}: only F32 tensors are supported, got {info['dtype']}")
        a, b = info["data_offsets"]
        out[name] = np.frombuffer(blob[base + a:base + b], dtype=np.float32).reshape(info["shape"])
    return out


def gaussian_audio(seed: int, segments: int = 1, length: int = SEGMENT_SAMPLES, std: float = 0.1):
    """(segments, 2, length) i.i.d. N(0, std^2) audio (benchmark configuration 1)."""
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((segments, AUDIO_CHANNELS, length)) * std).astype(np.float32)


def pink_noise(seed: int, length: int, channels: int = AUDIO_CHANNELS, rms: float = 0.1):
    """(channels, length) 1/f noise: white Gaussian shaped by f^-1/2 in the
    FFT domain, DC removed, rescaled to ``rms`` per channel."""
    rng = np.random.default_rng(seed)
    out = np.empty((channels, length), dtype=np.float32)
    freqs = np.fft.rfftfreq(length)
    shape = np.zeros_like(freqs)
    shape[1:] = 1.0 / np.sqrt(freqs[1:])
    for c in range(channels):
        spectrum = np.fft.rfft(rng.standard_normal(length)) * shape
        signal = np.fft.irfft(spectrum, n=length)
        signal *= rms / np.sqrt(np.mean(signal ** 2))
        out[c] = signal.astype(np.float32)
    return out


def lcg_audio(seed: int, shape, scale: float = 0.1):
    """The reference's batch-independence test signal
    (crates/demucs-core/tests/demucs_alignment.rs:232-246):
    ``rng = rng*1664525 + 1013904223``, ``((rng>>8)/2^23 - 1) * scale``."""
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.float32)
    rng = seed & 0xFFFFFFFF
    for i in range(n):
        rng = (rng * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = np.float32(np.float32((rng >> 8) / 8388608.0) - np.float32(1.0)) * np.float32(scale)
    return out.reshape(shape)
