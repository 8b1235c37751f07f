"""Checkpoint containers through the library's own loader (no GPU needed).

* torch.save archives (`.th` / `.pth`, ckpt/mod.rs, ckpt/pickle.rs): every
  tensor of the state dict comes back exactly as torch holds it — views with
  offsets and strides onto shared storages, F16 / BF16 / F64 / integer
  storages upcast to f32 — whether the state dict is the top level or sits
  under `state` (the demucs package), `state_dict` or `model_state_dict`.
* The model kwargs (the demucs package's pickled dict, or a safetensors
  `__metadata__["kwargs"]` JSON string, config.rs:150-215) are checked against
  the htdemucs architecture the kernels implement.

Each archive is written here by torch.save itself, so the reader is checked
against PyTorch's own serialisation.
"""

import fractions
import io
import json
import struct
from collections import OrderedDict

import numpy as np
import pytest
import torch

import dmx
import synth

DEFAULT_KWARGS = {"sources": ["drums", "bass", "other", "vocals"], "audio_channels": 2,
                  "samplerate": 44100, "segment": fractions.Fraction(39, 5), "channels": 48,
                  "growth": 2, "nfft": 4096, "depth": 4, "cac": True, "t_layers": 5, "t_heads": 8}


def _save(obj):
    buf = io.BytesIO()
    torch.save(obj, buf)
    return buf.getvalue()


def test_a_demucs_package_reads_back_every_tensor_exactly():
    # the layout of the published .th files: {klass, args, kwargs, state}
    w = synth.random_weights(0)
    state = OrderedDict((k, torch.from_numpy(np.ascontiguousarray(v))) for k, v in w.items())
    blob = _save({"klass": fractions.Fraction, "args": (), "kwargs": DEFAULT_KWARGS, "state": state})
    assert blob[:4] == b"PK\x03\x04"
    for name in ("encoder.0.conv.weight", "crosstransformer.layers.1.cross_attn.in_proj_weight",
                 "tdecoder.3.conv_tr.bias", "freq_emb.embedding.weight"):
        got = dmx.read_tensor(blob, name)
        assert got.shape == w[name].shape and np.array_equal(got, w[name]), name


@pytest.mark.parametrize("wrapper", [None, "state_dict", "model_state_dict", "state"])
def test_views_dtypes_and_wrappers(wrapper):
    base = torch.arange(24, dtype=torch.float32).reshape(4, 6) / 7
    state = OrderedDict()
    state["slice"] = base[1:3, 2:5]          # a view with a storage offset and row stride
    state["transposed"] = base.t()           # the same storage, strides swapped
    state["half"] = (torch.randn(5, 3) * 3).to(torch.float16)
    state["bf16"] = torch.randn(7).to(torch.bfloat16)
    state["f64"] = torch.randn(2, 2, dtype=torch.float64)
    state["long"] = torch.arange(-3, 3, dtype=torch.int64)
    state["scalar"] = torch.tensor(2.5)
    obj = state if wrapper is None else {"epoch": 3, wrapper: state}
    blob = _save(obj)
    for name, t in state.items():
        got = dmx.read_tensor(blob, name)
        ref = t.to(torch.float32).numpy()
        assert got.shape == ref.shape, name
        assert np.array_equal(got, ref), name


def test_kwargs_of_another_architecture_are_rejected():
    state = OrderedDict(w=torch.ones(2))
    wider = dict(DEFAULT_KWARGS, channels=64)
    with pytest.raises(dmx.DmxError, match="channels = 64") as e:
        dmx.read_tensor(_save({"kwargs": wider, "state": state}), "w")
    assert e.value.code == 1
    other_segment = dict(DEFAULT_KWARGS, segment=fractions.Fraction(10, 1))
    with pytest.raises(dmx.DmxError, match="segment = 10"):
        dmx.read_tensor(_save({"kwargs": other_segment, "state": state}), "w")
    three = dict(DEFAULT_KWARGS, sources=["a", "b", "c"])
    with pytest.raises(dmx.DmxError, match="3 sources"):
        dmx.read_tensor(_save({"kwargs": three, "state": state}), "w")
    assert dmx.read_tensor(_save({"kwargs": DEFAULT_KWARGS, "state": state}), "w").tolist() == [1, 1]


def _st_blob(header, data):
    text = json.dumps(header, separators=(",", ":")).encode()
    return struct.pack("<Q", len(text)) + text + data


def test_safetensors_kwargs_metadata_is_checked():
    # the HuggingFace safetensors keep kwargs as a JSON string in __metadata__
    data = np.array([0.5], "<f4").tobytes()
    ok = {"__metadata__": {"kwargs": json.dumps({"channels": 48, "segment": {"numerator": 39, "denominator": 5},
                                                 "sources": ["drums", "bass", "other", "vocals"]})},
          "w": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]}}
    assert dmx.read_tensor(_st_blob(ok, data), "w").tolist() == [0.5]
    bad = json.loads(json.dumps(ok))
    bad["__metadata__"]["kwargs"] = json.dumps({"depth": 5})
    with pytest.raises(dmx.DmxError, match="depth = 5"):
        dmx.read_tensor(_st_blob(bad, data), "w")


def test_malformed_archives_are_rejected():
    state = OrderedDict(w=torch.ones(3))
    blob = bytearray(_save(state))
    with pytest.raises(dmx.DmxError):
        dmx.read_tensor(bytes(blob[: len(blob) // 2]), "w")   # truncated: no directory
    with pytest.raises(dmx.DmxError, match="missing tensor"):
        dmx.read_tensor(bytes(blob), "nope")
    with pytest.raises(dmx.DmxError, match="no tensor state dict"):
        dmx.read_tensor(_save({"config": {"a": 1}}), "w")
