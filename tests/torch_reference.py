"""A PyTorch restatement of the reference host forward — TEST INFRASTRUCTURE.

It pins the C++ oracle to PyTorch's own primitives (torch.stft/istft,
F.conv*, F.group_norm, F.layer_norm, scaled-dot-product attention), which are
the semantics the reference transcribes (crates/demucs-core/src/demucs/host.rs
header: "a literal transcription of demucs/htdemucs.py"). It runs in float64
so it stands in for the exact value both the oracle and the CUDA path
approximate. Every step names the reference function it follows.
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

HOP, NFFT = 1024, 4096


def _w(weights, name, dtype):
    return torch.as_tensor(np.asarray(weights[name]), dtype=dtype)


def _dconv(weights, prefix, x, dtype):
    """host.rs:985-1059 on (rows, C, T)."""
    for d in range(2):
        at = f"{prefix}.dconv.layers.{d}"
        dil = 2 ** d
        y = F.conv1d(x, _w(weights, f"{at}.0.weight", dtype), _w(weights, f"{at}.0.bias", dtype),
                     padding=dil, dilation=dil)
        y = F.group_norm(y, 1, _w(weights, f"{at}.1.weight", dtype),
                         _w(weights, f"{at}.1.bias", dtype), eps=1e-5)
        y = F.gelu(y)
        y = F.conv1d(y, _w(weights, f"{at}.3.weight", dtype), _w(weights, f"{at}.3.bias", dtype))
        y = F.group_norm(y, 1, _w(weights, f"{at}.4.weight", dtype),
                         _w(weights, f"{at}.4.bias", dtype), eps=1e-5)
        y = F.glu(y, dim=1)
        x = x + _w(weights, f"{at}.6.scale", dtype)[:, None] * y
    return x


def _mha(weights, attn, q_in, k_in, dtype, heads=8):
    """host.rs:1199-1312: nn.MultiheadAttention(batch_first=True)."""
    w = _w(weights, f"{attn}.in_proj_weight", dtype)
    b = _w(weights, f"{attn}.in_proj_bias", dtype)
    dim = q_in.shape[-1]
    q = q_in @ w[:dim].T + b[:dim]
    k = k_in @ w[dim:2 * dim].T + b[dim:2 * dim]
    v = k_in @ w[2 * dim:].T + b[2 * dim:]
    B, nq, _ = q.shape
    nk = k.shape[1]
    dh = dim // heads
    q = q.view(B, nq, heads, dh).transpose(1, 2)
    k = k.view(B, nk, heads, dh).transpose(1, 2)
    v = v.view(B, nk, heads, dh).transpose(1, 2)
    att = torch.softmax((q @ k.transpose(-1, -2)) / math.sqrt(dh), dim=-1) @ v
    att = att.transpose(1, 2).reshape(B, nq, dim)
    return att @ _w(weights, f"{attn}.out_proj.weight", dtype).T + _w(weights, f"{attn}.out_proj.bias", dtype)


def _layer(weights, at, cross, x, other, dtype):
    """host.rs:1315-1429."""
    ln = lambda name, t: F.layer_norm(t, (t.shape[-1],), _w(weights, f"{at}.{name}.weight", dtype),
                                      _w(weights, f"{at}.{name}.bias", dtype), eps=1e-5)
    nq = ln("norm1", x)
    if cross:
        att = _mha(weights, f"{at}.cross_attn", nq, ln("norm2", other), dtype)
    else:
        att = _mha(weights, f"{at}.self_attn", nq, nq, dtype)
    out = x + att * _w(weights, f"{at}.gamma_1.scale", dtype)
    h = ln("norm3" if cross else "norm2", out)
    h = F.gelu(h @ _w(weights, f"{at}.linear1.weight", dtype).T + _w(weights, f"{at}.linear1.bias", dtype))
    h = h @ _w(weights, f"{at}.linear2.weight", dtype).T + _w(weights, f"{at}.linear2.bias", dtype)
    out = out + h * _w(weights, f"{at}.gamma_2.scale", dtype)
    out = F.group_norm(out.transpose(1, 2), 1, _w(weights, f"{at}.norm_out.weight", dtype),
                       _w(weights, f"{at}.norm_out.bias", dtype), eps=1e-5).transpose(1, 2)
    return out


def _pos2d(dim, height, width, max_period=10000.0):
    """host.rs:1078-1106, evaluated in f32 like the reference."""
    half, pairs = dim // 2, dim // 4
    log_period = np.float32(np.log(np.float32(max_period))) / np.float32(half)
    div = np.exp(-(2 * np.arange(pairs, dtype=np.float32)) * log_period).astype(np.float32)
    t = np.arange(width, dtype=np.float32)[:, None, None]
    f = np.arange(height, dtype=np.float32)[None, :, None]
    out = np.zeros((width, height, dim), dtype=np.float32)
    out[:, :, 0:half:2] = np.sin(t * div)
    out[:, :, 1:half:2] = np.cos(t * div)
    out[:, :, half::2] = np.sin(f * div)
    out[:, :, half + 1::2] = np.cos(f * div)
    return out.reshape(width * height, dim)


def _pos1d(length, dim, max_period=10000.0):
    """host.rs:1110-1122."""
    half = dim // 2
    exponent = (np.arange(half, dtype=np.float32) / np.float32(half - 1)).astype(np.float32)
    phase = (np.arange(length, dtype=np.float32)[:, None]
             / np.power(np.float32(max_period), exponent)).astype(np.float32)
    return np.concatenate([np.cos(phase), np.sin(phase)], axis=1).astype(np.float32)


def forward(weights, mix, dtype=torch.float64, trace=None):
    """Htdemucs::forward (host.rs:202-520) for mix (B, 2, L == segment)."""
    rec = (lambda k, v: trace.__setitem__(k, v.detach().to(torch.float32).numpy().copy())) if trace is not None else (lambda k, v: None)
    mix = torch.as_tensor(np.asarray(mix), dtype=dtype)
    B, C, L = mix.shape
    le = -(-L // HOP)
    pad = HOP // 2 * 3
    right = pad + le * HOP - L
    # _spec (spec.rs:62-113)
    padded = F.pad(mix, (pad, right), mode="reflect")
    window = torch.hann_window(NFFT, periodic=True, dtype=dtype)
    z = torch.stft(padded.reshape(B * C, -1), NFFT, HOP, NFFT, window, center=True,
                   pad_mode="reflect", normalized=True, return_complex=True)
    z = z[:, :-1, 2:2 + le].reshape(B, C, NFFT // 2, le)
    x = torch.view_as_real(z).permute(0, 1, 4, 2, 3).reshape(B, 2 * C, NFFT // 2, le)
    rec("_magnitude", x)
    mean = x.mean(dim=(1, 2, 3), keepdim=True)
    std = x.std(dim=(1, 2, 3), keepdim=True)
    x = (x - mean) / (1e-5 + std)
    mean_t = mix.mean(dim=(1, 2), keepdim=True)
    std_t = mix.std(dim=(1, 2), keepdim=True)
    xt = (mix - mean_t) / (1e-5 + std_t)
    rec("x_normalized", x)
    rec("xt_normalized", xt)
    saved, saved_t, lengths_t = [], [], []
    for i in range(4):
        # time_encoder_forward (host.rs:625-678)
        lengths_t.append(xt.shape[-1])
        if xt.shape[-1] % 4:
            xt = F.pad(xt, (0, 4 - xt.shape[-1] % 4))
        y = F.gelu(F.conv1d(xt, _w(weights, f"tencoder.{i}.conv.weight", dtype),
                            _w(weights, f"tencoder.{i}.conv.bias", dtype), stride=4, padding=2))
        y = _dconv(weights, f"tencoder.{i}", y, dtype)
        xt = F.glu(F.conv1d(y, _w(weights, f"tencoder.{i}.rewrite.weight", dtype),
                            _w(weights, f"tencoder.{i}.rewrite.bias", dtype)), dim=1)
        rec(f"tencoder.{i}", xt)
        saved_t.append(xt)
        # freq_encoder_forward (host.rs:577-622)
        y = F.gelu(F.conv2d(x, _w(weights, f"encoder.{i}.conv.weight", dtype),
                            _w(weights, f"encoder.{i}.conv.bias", dtype), stride=(4, 1), padding=(2, 0)))
        b_, c_, f_, t_ = y.shape
        y = y.permute(0, 2, 1, 3).reshape(b_ * f_, c_, t_)
        y = _dconv(weights, f"encoder.{i}", y, dtype)
        y = y.view(b_, f_, c_, t_).permute(0, 2, 1, 3)
        x = F.glu(F.conv2d(y, _w(weights, f"encoder.{i}.rewrite.weight", dtype),
                           _w(weights, f"encoder.{i}.rewrite.bias", dtype)), dim=1)
        rec(f"encoder.{i}", x)
        if i == 0:
            emb = _w(weights, "freq_emb.embedding.weight", dtype) * 10.0
            x = x + 0.2 * emb.t()[None, :, :, None]
            rec("encoder.0.post_emb", x)
        saved.append(x)
    b_, c_, f_, t_ = x.shape
    x = F.conv1d(x.reshape(b_, c_, f_ * t_), _w(weights, "channel_upsampler.weight", dtype),
                 _w(weights, "channel_upsampler.bias", dtype))
    xt = F.conv1d(xt, _w(weights, "channel_upsampler_t.weight", dtype),
                  _w(weights, "channel_upsampler_t.bias", dtype))
    rec("channel_upsampler", x)
    rec("channel_upsampler_t", xt)
    D = x.shape[1]
    spec = x.view(b_, D, f_, t_).permute(0, 3, 2, 1).reshape(b_, t_ * f_, D)
    time = xt.transpose(1, 2)
    spec = F.layer_norm(spec, (D,), _w(weights, "crosstransformer.norm_in.weight", dtype),
                        _w(weights, "crosstransformer.norm_in.bias", dtype), eps=1e-5)
    spec = spec + torch.as_tensor(_pos2d(D, f_, t_), dtype=dtype)
    time = F.layer_norm(time, (D,), _w(weights, "crosstransformer.norm_in_t.weight", dtype),
                        _w(weights, "crosstransformer.norm_in_t.bias", dtype), eps=1e-5)
    time = time + torch.as_tensor(_pos1d(time.shape[1], D), dtype=dtype)
    rec("crosstransformer.in#0", spec)
    rec("crosstransformer.in#1", time)
    for l in range(5):
        cross = l % 2 == 1
        a, at = f"crosstransformer.layers.{l}", f"crosstransformer.layers_t.{l}"
        old = spec
        spec = _layer(weights, a, cross, spec, time if cross else None, dtype)
        time = _layer(weights, at, cross, time, old if cross else None, dtype)
        rec(a, spec)
        rec(at, time)
    x = spec.view(b_, t_, f_, D).permute(0, 3, 2, 1).reshape(b_, D, f_ * t_)
    x = F.conv1d(x, _w(weights, "channel_downsampler.weight", dtype),
                 _w(weights, "channel_downsampler.bias", dtype))
    xt = F.conv1d(time.transpose(1, 2), _w(weights, "channel_downsampler_t.weight", dtype),
                  _w(weights, "channel_downsampler_t.bias", dtype))
    rec("channel_downsampler", x)
    rec("channel_downsampler_t", xt)
    x = x.view(b_, -1, f_, t_)
    for e in range(4):
        last = e == 3
        j = 3 - e
        # freq_decoder_forward (host.rs:682-759)
        x = x + saved.pop()
        y = F.glu(F.conv2d(x, _w(weights, f"decoder.{j}.rewrite.weight", dtype),
                           _w(weights, f"decoder.{j}.rewrite.bias", dtype), padding=1), dim=1)
        b_, c_, f_, t_ = y.shape
        y = y.permute(0, 2, 1, 3).reshape(b_ * f_, c_, t_)
        y = _dconv(weights, f"decoder.{j}", y, dtype)
        y = y.view(b_, f_, c_, t_).permute(0, 2, 1, 3)
        y = F.conv_transpose2d(y, _w(weights, f"decoder.{j}.conv_tr.weight", dtype),
                               _w(weights, f"decoder.{j}.conv_tr.bias", dtype), stride=(4, 1))
        x = y[:, :, 2:-2, :]
        if not last:
            x = F.gelu(x)
        rec(f"decoder.{j}", x)
        # time_decoder_forward (host.rs:763-827)
        xt = xt + saved_t.pop()
        length_t = lengths_t.pop()
        y = F.glu(F.conv1d(xt, _w(weights, f"tdecoder.{j}.rewrite.weight", dtype),
                           _w(weights, f"tdecoder.{j}.rewrite.bias", dtype), padding=1), dim=1)
        y = _dconv(weights, f"tdecoder.{j}", y, dtype)
        y = F.conv_transpose1d(y, _w(weights, f"tdecoder.{j}.conv_tr.weight", dtype),
                               _w(weights, f"tdecoder.{j}.conv_tr.bias", dtype), stride=4)
        xt = y[:, :, 2:2 + length_t]
        if not last:
            xt = F.gelu(xt)
        rec(f"tdecoder.{j}", xt)
    # _mask / _ispec (host.rs:466-497, spec.rs:115-175)
    x = x * std + mean
    Fq, T = x.shape[2], x.shape[3]
    zc = x.view(B, 4, 2, 2, Fq, T).permute(0, 1, 2, 4, 5, 3).contiguous()
    zc = torch.view_as_complex(zc)
    zc = F.pad(zc, (2, 2, 0, 1))
    ilen = HOP * le + 2 * pad
    wav = torch.istft(zc.reshape(B * 8, Fq + 1, T + 4), NFFT, HOP, NFFT, window,
                      center=True, normalized=True, length=ilen)
    wav = wav.view(B, 4, 2, -1)[..., pad:pad + L]
    time_out = xt.view(B, 4, 2, L) * std_t + mean_t
    return (time_out + wav).to(torch.float32).numpy()
