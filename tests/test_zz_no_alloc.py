"""The allocation-free track normalisation (dmx_normalize_track_noalloc).

It serves callers that may not allocate device memory where they need the
normalisation — real-time audio callbacks that must not block on the
driver's allocator, applications that pre-reserve their device budget — so
it keeps its scratch in a fixed device array instead. Checked through the
C ABI against the handle-based dmx_normalize_track_device on the same track,
on two calls in a row (the shared scratch must not leak state between calls).
This file is collected last on purpose.
"""

import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu


def test_noalloc_normalize_matches_handle_entry_point_twice():
    import torch
    import dmx

    n = 2_000_003  # not a multiple of the 65,536-sample partial blocks
    track = synth.pink_noise(41, n)
    lr = torch.from_numpy(track).cuda()
    h = dmx.Handle(synth.write_safetensors(synth.random_weights(0)), device=0, max_batch=1)
    ref = torch.empty_like(lr)
    ref_ms = torch.empty(2, dtype=torch.float32, device="cuda")
    h.normalize_track_device(lr.data_ptr(), n, ref.data_ptr(), ref_ms.data_ptr())
    h.synchronize()
    ref, ref_ms = ref.cpu().numpy(), ref_ms.cpu().numpy()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out = torch.full_like(lr, float("nan"))
        ms = torch.full((2,), float("nan"), dtype=torch.float32, device="cuda")
        dmx.normalize_track_noalloc(lr.data_ptr(), n, out.data_ptr(), ms.data_ptr(), stream)
        torch.cuda.synchronize()
        got_ms, got = ms.cpu().numpy(), out.cpu().numpy()
        # the partials are grouped differently (one per 65,536 samples vs a
        # fixed grid), so agreement is to f64-reduction rounding, not bitwise
        np.testing.assert_allclose(got_ms, ref_ms, rtol=1e-6, atol=0)
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6)
    h.close()


def test_noalloc_rejects_tracks_beyond_its_scratch():
    import dmx

    with pytest.raises(dmx.DmxError, match="allocation-free limit"):
        dmx.normalize_track_noalloc(16, 536_870_913, 16, 16)
