"""The ``dmx`` command-line tool end to end on the GPU: ``dmx separate``
reads the WAV in windows and writes, block by block as
dmx_separate_track_windowed hands them over, exactly the stems
dmx_separate_track returns for the same samples (main.rs:313-602 of the
reference CLI: all four stems, ``--stem`` into one file, ``--two-stems`` with
the ``add`` and ``minus`` companions, mono input, ``--segment``,
``--dump-trace``); ``dmx bench`` and ``dmx profile`` run and report."""

import os
import struct
import subprocess

import numpy as np
import pytest

import dmx
import synth
from test_cli_cpu import build_wav, parse_float_wav

pytestmark = pytest.mark.gpu

SOURCES = ["drums", "bass", "other", "vocals"]


@pytest.fixture(scope="module")
def setup(tmp_path_factory):
    d = tmp_path_factory.mktemp("cli")
    blob = synth.write_safetensors(synth.random_weights(61))
    (d / "model.safetensors").write_bytes(blob)
    track = synth.pink_noise(62, int(44100 * 17.3))
    (d / "mix.wav").write_bytes(build_wav(3, 2, 44100, 32, track.T.astype("<f4").tobytes()))
    h = dmx.Handle(blob, device=0, max_batch=16, precision=dmx.TF32)
    return d, track, h


def run(*args):
    r = subprocess.run([dmx.cli_path(), *map(str, args)], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr
    return r.stdout


def stem_file(path):
    rate, ch, frames = parse_float_wav(open(path, "rb").read())
    assert (rate, ch) == (44100, 2)
    return frames.T


def test_separate_writes_the_driver_stems(setup):
    d, track, h = setup
    out = run("separate", d / "mix.wav", "-o", d / "all", "-m", d / "model.safetensors",
              "--precision", "tf32", "--timings")
    ref = h.separate_track(track[0], track[1], shifts=1, batch=16)
    for s, name in enumerate(SOURCES):
        assert np.array_equal(stem_file(d / "all" / f"{name}.wav"), ref[s]), name
    assert "separation " in out and "RTFx" in out and "per chunk:" in out
    assert f"peak {np.abs(ref[0]).max():.4f}" in out


def test_two_stems_companions(setup):
    d, track, h = setup
    ref = h.separate_track(track[0], track[1], shifts=1, batch=16)
    run("separate", d / "mix.wav", "-o", d / "add", "-m", d / "model.safetensors",
        "--two-stems", "vocals")
    assert sorted(os.listdir(d / "add")) == ["no_vocals.wav", "vocals.wav"]
    assert np.array_equal(stem_file(d / "add" / "vocals.wav"), ref[3])
    # the other stems summed in source order, in f32 (main.rs:515-527)
    acc = np.zeros_like(ref[0])
    for s in (0, 1, 2):
        acc = (acc + ref[s]).astype(np.float32)
    assert np.array_equal(stem_file(d / "add" / "no_vocals.wav"), acc)
    run("separate", d / "mix.wav", "-o", d / "minus", "-m", d / "model.safetensors",
        "--two-stems", "drums", "--other-method", "minus")
    assert np.array_equal(stem_file(d / "minus" / "minus_drums.wav"), track - ref[0])
    run("separate", d / "mix.wav", "-o", d / "none", "-m", d / "model.safetensors",
        "--two-stems", "bass", "--other-method", "none")
    assert os.listdir(d / "none") == ["bass.wav"]


def test_single_stem_file_segment_and_shifts(setup):
    d, track, h = setup
    run("separate", d / "mix.wav", "-o", d / "bass_only.wav", "-m", d / "model.safetensors",
        "--stem", "bass", "--segment", "5", "--shifts", "2", "--overlap", "0.3")
    ref = h.separate_track(track[0], track[1], shifts=2, batch=16, overlap=0.3, segment=5.0)
    assert np.array_equal(stem_file(d / "bass_only.wav"), ref[1])


def test_mono_input_is_separated_as_stereo(setup):
    d, track, h = setup
    mono = track[0, : 44100 * 9].copy()
    (d / "mono.wav").write_bytes(build_wav(1, 1, 44100, 16, (mono * 32767).astype("<i2").tobytes()))
    run("separate", d / "mono.wav", "-o", d / "mono", "-m", d / "model.safetensors")
    x = ((mono * 32767).astype(np.int16) / np.float32(32768)).astype(np.float32)
    ref = h.separate_track(x, x, shifts=1, batch=16)
    for s, name in enumerate(SOURCES):
        assert np.array_equal(stem_file(d / "mono" / f"{name}.wav"), ref[s]), name


def test_wrong_sample_rate_is_refused(setup):
    d, track, _ = setup
    (d / "48k.wav").write_bytes(build_wav(3, 2, 48000, 32, track[:, :4800].T.astype("<f4").tobytes()))
    r = subprocess.run([dmx.cli_path(), "separate", d / "48k.wav", "-o", d / "x", "-m",
                        d / "model.safetensors"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 1 and "44100" in r.stderr


def test_dump_trace_writes_the_first_forward(setup):
    d, track, _ = setup
    short = track[:, : 44100 * 3]
    (d / "short.wav").write_bytes(build_wav(3, 2, 44100, 32, short.T.astype("<f4").tobytes()))
    out = run("separate", d / "short.wav", "-o", d / "traced", "-m", d / "model.safetensors",
              "--dump-trace", d / "trace")
    names = sorted(os.listdir(d / "trace"))
    assert "crosstransformer_in_0.npy" in names, names
    assert any(n.startswith("decoder_") for n in names), names
    assert f"wrote {len(names)} traced activations" in out
    x = np.load(d / "trace" / "crosstransformer_in_0.npy")
    assert x.dtype == np.float32 and x.ndim == 3 and np.isfinite(x).all()


def test_bench_and_profile_report(setup):
    d, _, _ = setup
    out = run("bench", "-m", d / "model.safetensors", "--repeats", "2")
    assert "chunk forward" in out and "x raw" in out
    out = run("profile", d / "mix.wav", "-m", d / "model.safetensors", "--repeats", "2")
    lines = out.splitlines()
    assert lines[1].startswith("one segment:")
    assert lines[2].split() == ["stage", "total", "ms", "per", "call", "calls"]
    assert len(lines) > 10
