"""The ``dmx`` command-line tool's WAV reader and writer (no GPU: the
``wav-copy`` command decodes a WAV and writes it back as float32).

Known answers are those of the reference's audio tests (demucs-core
src/audio.rs:764-936): soundfile scaling of PCM 16 and 24, channel-major
deinterleaving, refusal of non-RIFF data and 8-bit PCM, mono duplicated for
the stereo model, and a float writer that interleaves frames on disk."""

import os
import struct
import subprocess

import numpy as np
import pytest

import dmx


def build_wav(tag, channels, rate, bits, payload, extra_chunks=b""):
    """A RIFF/WAVE file with one fmt chunk, optional chunks, then data."""
    fmt = struct.pack("<HHIIHH", tag, channels, rate, rate * channels * bits // 8,
                      channels * bits // 8, bits)
    body = b"WAVE" + b"fmt " + struct.pack("<I", len(fmt)) + fmt + extra_chunks
    body += b"data" + struct.pack("<I", len(payload)) + payload
    if len(payload) & 1:
        body += b"\0"
    return b"RIFF" + struct.pack("<I", len(body)) + body


def parse_float_wav(data):
    """(rate, channels, interleaved float32 frames) of a float WAV, read chunk by chunk."""
    assert data[:4] == b"RIFF" and data[8:12] == b"WAVE"
    assert struct.unpack("<I", data[4:8])[0] == len(data) - 8
    pos, fmt, payload = 12, None, None
    while pos + 8 <= len(data):
        cid, size = data[pos:pos + 4], struct.unpack("<I", data[pos + 4:pos + 8])[0]
        if cid == b"fmt ":
            fmt = struct.unpack("<HHIIHH", data[pos + 8:pos + 24])
        elif cid == b"data":
            payload = data[pos + 8:pos + 8 + size]
        pos += 8 + size + (size & 1)
    tag, channels, rate, byte_rate, align, bits = fmt
    assert (tag, bits, align, byte_rate) == (3, 32, 4 * channels, 4 * channels * rate)
    return rate, channels, np.frombuffer(payload, "<f4").reshape(-1, channels)


def copy(tmp_path, wav_bytes, *flags):
    src, dst = tmp_path / "in.wav", tmp_path / "out.wav"
    src.write_bytes(wav_bytes)
    r = subprocess.run([dmx.cli_path(), "wav-copy", str(src), str(dst), *flags],
                       capture_output=True, text=True, timeout=60)
    if r.returncode != 0:
        return None, r.stderr
    return parse_float_wav(dst.read_bytes()), r.stdout




@pytest.fixture(autouse=True)
def _cli():
    dmx.cli_path()


def test_reads_mono_float_wav(tmp_path):
    payload = np.array([0.5, -0.25, 0.125], "<f4").tobytes()
    (rate, ch, frames), out = copy(tmp_path, build_wav(3, 1, 44100, 32, payload))
    assert (rate, ch) == (44100, 1)
    assert frames[:, 0].tolist() == [0.5, -0.25, 0.125]
    assert "3 frames" in out


def test_deinterleaves_stereo_and_writes_interleaved(tmp_path):
    # frames (L=1, R=2), (L=3, R=4); the writer puts frame 0's L, R first on disk
    payload = np.array([1.0, 2.0, 3.0, 4.0], "<f4").tobytes()
    (rate, ch, frames), _ = copy(tmp_path, build_wav(3, 2, 44100, 32, payload))
    assert ch == 2
    assert frames[:, 0].tolist() == [1.0, 3.0]
    assert frames[:, 1].tolist() == [2.0, 4.0]


def test_pcm16_scaled_like_soundfile(tmp_path):
    payload = np.array([32767, -32768, 0], "<i2").tobytes()
    (_, _, frames), _ = copy(tmp_path, build_wav(1, 1, 44100, 16, payload))
    assert abs(frames[0, 0] - 0.9999695) < 1e-6
    assert frames[1, 0] == -1.0 and frames[2, 0] == 0.0


def test_pcm24_sign_extension(tmp_path):
    payload = bytes([0x00, 0x00, 0x80, 0xFF, 0xFF, 0x7F])
    (_, _, frames), _ = copy(tmp_path, build_wav(1, 1, 44100, 24, payload))
    assert frames[0, 0] == -1.0
    assert abs(frames[1, 0] - 0.99999988) < 1e-6


def test_pcm32_float64_and_extensible(tmp_path):
    ints = np.array([2**31 - 1, -2**31, 1 << 30], "<i4")
    (_, _, frames), _ = copy(tmp_path, build_wav(1, 1, 44100, 32, ints.tobytes()))
    np.testing.assert_array_equal(frames[:, 0], (ints / 2.0**31).astype(np.float32))
    doubles = np.array([0.1, -0.7, 1.5], "<f8")
    (_, _, frames), _ = copy(tmp_path, build_wav(3, 1, 44100, 64, doubles.tobytes()))
    np.testing.assert_array_equal(frames[:, 0], doubles.astype(np.float32))
    floats = np.array([0.25, -0.5], "<f4")
    (_, _, frames), _ = copy(tmp_path, build_wav(0xFFFE, 1, 48000, 32, floats.tobytes()))
    np.testing.assert_array_equal(frames[:, 0], floats)


def test_skips_chunks_between_fmt_and_data(tmp_path):
    # soundfile writes `fact` and `PEAK` chunks before `data` (audio.rs:838-874);
    # an odd-sized chunk carries one pad byte
    extra = b"fact" + struct.pack("<I", 4) + struct.pack("<I", 2)
    extra += b"PEAK" + struct.pack("<I", 5) + b"\1\2\3\4\5" + b"\0"
    payload = np.array([0.75, -0.125], "<f4").tobytes()
    (_, _, frames), _ = copy(tmp_path, build_wav(3, 1, 44100, 32, payload, extra))
    assert frames[:, 0].tolist() == [0.75, -0.125]


def test_mono_is_duplicated_for_stereo(tmp_path):
    payload = np.array([0.5, -0.5], "<f4").tobytes()
    (_, ch, frames), _ = copy(tmp_path, build_wav(3, 1, 44100, 32, payload), "--stereo")
    assert ch == 2
    assert frames.tolist() == [[0.5, 0.5], [-0.5, -0.5]]


def test_round_trip_keeps_rate_and_values(tmp_path):
    rng = np.random.default_rng(7)
    x = rng.standard_normal((1000, 2)).astype("<f4")
    (rate, ch, frames), _ = copy(tmp_path, build_wav(3, 2, 22050, 32, x.tobytes()))
    assert (rate, ch) == (22050, 2)
    np.testing.assert_array_equal(frames, x)
    # the copy reads back identically through the same reader
    src = (tmp_path / "out.wav").read_bytes()
    (_, _, again), _ = copy(tmp_path, src)
    np.testing.assert_array_equal(again, x)


@pytest.mark.parametrize("bad", [
    b"not a wav file at all",
    build_wav(1, 1, 44100, 8, bytes([1, 2, 3])),        # 8-bit PCM
    build_wav(3, 1, 44100, 16, bytes(4)),              # 16-bit float
    build_wav(1, 2, 44100, 16, bytes(6)),              # not whole frames
    build_wav(1, 0, 44100, 16, b""),                   # zero channels
    b"RIFF" + struct.pack("<I", 4) + b"WAVE",          # no chunks
])
def test_rejects_malformed_input(tmp_path, bad):
    result, err = copy(tmp_path, bad)
    assert result is None
    assert err.startswith("dmx: ")


def test_usage_errors():
    r = subprocess.run([dmx.cli_path(), "frobnicate"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "unknown command" in r.stderr
    r = subprocess.run([dmx.cli_path(), "separate", "x.wav", "-m", "m", "--stem", "drums",
                        "--two-stems", "bass", "-o", "out"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "exclude" in r.stderr


@pytest.mark.parametrize("window", [1, 7, 1000, 1 << 20])
@pytest.mark.parametrize("tag,bits,channels", [(1, 16, 2), (1, 24, 1), (3, 64, 2), (0xFFFE, 32, 1)])
def test_windowed_reads_match_the_whole_file(tmp_path, window, tag, bits, channels):
    # separate reads the input through the same source in windows of a forward's chunks
    rng = np.random.default_rng(bits + channels)
    n = 2501
    if tag == 1:
        raw = rng.integers(-(1 << (bits - 1)), 1 << (bits - 1), size=n * channels)
        payload = b"".join(int(v).to_bytes(bits // 8, "little", signed=True) for v in raw)
    else:
        payload = (rng.standard_normal(n * channels) * 0.3).astype("<f8" if bits == 64 else "<f4").tobytes()
    wav = build_wav(tag, channels, 44100, bits, payload)
    whole, _ = copy(tmp_path, wav, "--stereo")
    windowed, _ = copy(tmp_path, wav, "--stereo", "--window", str(window))
    assert windowed[1] == 2 and whole[1] == 2
    np.testing.assert_array_equal(windowed[2], whole[2])
