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
    return sorted(set(names) - {"dmx_progress_fn", "dmx_trace_fn"})


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
