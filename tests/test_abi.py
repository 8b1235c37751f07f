"""The C-ABI library loads and exports every function include/dmx.h declares
(no GPU needed: nothing is called)."""

import os
import re

import dmx

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    text = open(os.path.join(ROOT, "include", "dmx.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"\b(dmx_[a-z_]+)\s*\(", text)
    return sorted(set(names) - {"dmx_progress_fn", "dmx_trace_fn", "dmx_frames_fn", "dmx_read_fn"})


def test_library_exports_every_declared_function():
    lib = dmx.lib()
    declared = declared_functions()
    assert len(declared) >= 15
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, missing
    assert sorted(dmx.EXPORTS) == declared


def test_default_config_is_the_reference_default():
    c = dmx.default_config()
    assert (c.sources, c.audio_channels, c.samplerate, c.segment_samples) == (4, 2, 44100, 343980)


def test_chunk_plan_matches_the_reference_count():
    # streaming.rs:88-94: len(range(0, length, stride)), stride = int(0.75 * 343980)
    stride = int(0.75 * 343980)
    for length in (1, stride, stride + 1, 10_584_000, 10_584_000 + 22050):
        assert dmx.num_chunks(length) == -(-length // stride)
    assert dmx.num_chunks(0) == 0


def test_weight_blob_dtypes_are_checked_before_the_device_is_touched():
    # dmx_create parses and validates the safetensors blob (safetensors.rs:110-135 dtypes)
    # before any CUDA call, so malformed blobs fail with DMX_ERR_WEIGHTS on any host
    import json
    import struct

    import numpy as np
    import pytest
    import synth

    def blob(header, data):
        text = json.dumps(header).encode()
        return struct.pack("<Q", len(text)) + text + data

    bad_dtype = blob({"w": {"dtype": "F8_E4M3", "shape": [2], "data_offsets": [0, 2]}}, b"\0\0")
    short_f16 = blob({"w": {"dtype": "F16", "shape": [4], "data_offsets": [0, 6]}}, b"\0" * 6)
    for b, msg in ((bad_dtype, "unsupported safetensors dtype F8_E4M3"),
                   (short_f16, "data_offsets do not match the shape")):
        with pytest.raises(dmx.DmxError, match=msg) as e:
            dmx.Handle(b, device=0, max_batch=1)
        assert e.value.code == 2  # DMX_ERR_WEIGHTS
    # a well-formed F16 blob gets past parsing (on a host without a GPU the next step fails)
    w = {"x": np.array([1.0, -2.0, 0.5, 0.0], np.float32)}
    assert synth.write_safetensors(w, dtype="F16")[8:].startswith(b'{"x":{"dtype":"F16"')


def test_bag_arguments_map_stem_names_to_flags():
    # StemSelection (api.rs:895-906) as the C ABI's four `requested` flags
    import numpy as np
    import pytest

    w, req = dmx._bag_args(np.eye(4), ["vocals", "bass"])
    assert w.dtype == np.float32 and w.flags.c_contiguous and w.shape == (4, 4)
    assert list(req) == [0, 1, 0, 1]
    assert list(dmx._bag_args(np.eye(4), [0, 2])[1]) == [1, 0, 1, 0]
    assert dmx._bag_args(np.eye(4), None)[1] is None
    assert list(dmx._bag_args(np.eye(4), [])[1]) == [0, 0, 0, 0]
    with pytest.raises(ValueError):
        dmx._bag_args(np.ones((2, 3)), None)
