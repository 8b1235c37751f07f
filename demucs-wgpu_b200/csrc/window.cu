// Separation of a track that is never resident as a whole: the mix is read
// through a callback in windows (WindowedMix, mix.rs:61-330, over the
// MixSamples interface, mix.rs:18-60) and the overlap-add runs in a sliding
// device window (OlaRing, streaming.rs:96-261), so device memory holds one
// forward's chunks and one window of samples — O(batch x segment), whatever
// the track's length. The result equals dmx_separate_track's bit for bit:
// the moments are formed per thread in the whole-track pass's order, the
// normalisation, chunks, accumulation and finish are the same arithmetic on
// the same values, and only the buffers they live in are windows.
#include <algorithm>
#include <climits>
#include <string>

#include "runtime.cuh"

namespace dmx {

void ensure_emit(dmx_handle* h, int64_t cap) {
  if (cap <= h->emit_cap) return;
  for (int i = 0; i < 2; ++i) {
    cudaFreeHost(h->emit_pin[i]);
    h->emit_pin[i] = nullptr;
  }
  h->emit_cap = 0;
  for (int i = 0; i < 2; ++i) {
    CK(cudaMallocHost(&h->emit_pin[i], (size_t)8 * cap * sizeof(float)));
    if (!h->emit_ev[i]) CK(cudaEventCreateWithFlags(&h->emit_ev[i], cudaEventDisableTiming));
  }
  h->emit_cap = cap;
}

namespace {

// Mix samples [*lo, *hi) that chunks [c0, c1) of a shift view read: chunk c
// is centred in `chunk` samples around view [c * stride, + its length)
// (padded_chunk_shifted_mix, mix.rs:587-633; the gather kernel's indexing).
void group_mix_range(int64_t n, int64_t offset, int64_t max_shift, const PassGeom& pg,
                     int64_t vlen, int64_t c0, int64_t c1, int64_t* lo, int64_t* hi) {
  int64_t vmin = INT64_MAX, vmax = INT64_MIN;
  for (int64_t c = c0; c < c1; ++c) {
    const int64_t vstart = c * pg.stride;
    const int64_t len = std::min<int64_t>(pg.chunk, vlen - vstart);
    const int64_t start = vstart - (pg.chunk - len) / 2;
    vmin = std::min(vmin, std::max<int64_t>(start, 0));
    vmax = std::max(vmax, std::min<int64_t>(start + pg.chunk, vlen));
  }
  const int64_t shift = max_shift ? offset - max_shift : 0;
  *lo = std::min(n, std::max<int64_t>(0, vmin + shift));
  *hi = std::max(*lo, std::min<int64_t>(n, vmax + shift));
}

// Pinned read staging, two buffers of (2, cap): the host fills one while the
// copy from the other may still be in flight.
struct WindowReader {
  dmx_handle* h;
  dmx_read_fn fn;
  void* user;
  int64_t cap;
  int next = 0;
  bool used[2] = {false, false};

  // reads mix samples [t0, t0 + count) and queues their copy into d_win
  // (rows `cap` apart) on the handle's stream
  void load(int64_t t0, int64_t count, float* d_win) {
    if (count <= 0) return;
    const int slot = next;
    next ^= 1;
    if (used[slot]) CK(cudaEventSynchronize(h->win_ev[slot]));
    float* pin = h->win_pin[slot];
    if (fn(t0, count, pin, pin + cap, user) != 0)
      throw Error(DMX_ERR_INVALID, "the read callback failed for samples [" + std::to_string(t0) +
                                       ", " + std::to_string(t0 + count) + ")");
    CK(cudaMemcpy2DAsync(d_win, (size_t)cap * sizeof(float), pin, (size_t)cap * sizeof(float),
                         (size_t)count * sizeof(float), 2, cudaMemcpyHostToDevice, h->stream));
    CK(cudaEventRecord(h->win_ev[slot], h->stream));
    used[slot] = true;
  }
};

// Blocks of the several-shifts case: each pass's finished samples (acc / sw,
// mode 4) are summed on the host in pass order, as the reference sums its
// passes into an O(T) host array (pipeline.rs:451-500).
struct PassSum {
  std::vector<float> sum;  // (8, n)
  int64_t n;
};

void add_block(int64_t t0, int64_t count, const float* block, void* user) {
  PassSum& p = *static_cast<PassSum*>(user);
  for (int r = 0; r < 8; ++r) {
    float* dst = p.sum.data() + (size_t)r * p.n + t0;
    const float* src = block + (size_t)r * count;
    for (int64_t i = 0; i < count; ++i) dst[i] += src[i];
  }
}

}  // namespace

void separate_windowed_impl(dmx_handle* h, dmx_read_fn read, int64_t n,
                            const dmx_separate_opts* opts, dmx_frames_fn on_frames,
                            dmx_progress_fn progress, void* user) {
  const dmx_separate_opts o = separate_opts(opts);
  CK(cudaSetDevice(h->device));
  const PassGeom pg = pass_geom(h, chunk_samples(o), o.overlap, o.transition_power);
  const int64_t stride = pg.stride;
  const int64_t max_shift = o.shifts > 0 ? (int64_t)(0.5 * 44100.0) : 0;
  const int batch = std::max(1, o.batch > 0 ? std::min(o.batch, h->cfg.max_batch) : h->cfg.max_batch);
  // the accumulator and an output block span one group of chunks; the mix
  // window a group reads adds up to half a chunk on the left (a short last
  // chunk centred in its segment); a moments window is a multiple of the
  // moments grid
  const int64_t acap = (int64_t)(batch - 1) * stride + pg.chunk;
  const int64_t grid = moments_grid();
  const int64_t group_win = acap + pg.chunk / 2 + 1;
  const int64_t mwin = std::max<int64_t>(1, group_win / grid) * grid;
  const int64_t wcap = std::max(group_win, mwin);

  // pinned read staging, two (2, ld) buffers; the device window has the same rows
  if (wcap > h->win_pin_cap) {
    for (int i = 0; i < 2; ++i) {
      cudaFreeHost(h->win_pin[i]);
      h->win_pin[i] = nullptr;
    }
    h->win_pin_cap = 0;
    for (int i = 0; i < 2; ++i) CK(cudaMallocHost(&h->win_pin[i], (size_t)2 * wcap * sizeof(float)));
    h->win_pin_cap = wcap;
  }
  const int64_t ld = h->win_pin_cap;
  // device: moments state, (mean, std), mix window, two accumulators, two output blocks
  const size_t state_bytes = ((size_t)moments_state_doubles() * sizeof(double) + 255) / 256 * 256;
  const size_t need = state_bytes + 256 + (size_t)(2 * ld + 2 * 8 * acap + 2 * 8 * acap) * sizeof(float);
  if (need > h->win_cap) {
    cudaFree(h->win_ws);
    h->win_ws = nullptr;
    h->win_cap = 0;
    CK(cudaMalloc(&h->win_ws, need));
    h->win_cap = need;
  }
  double* d_state = reinterpret_cast<double*>(h->win_ws);
  float2* d_norm = reinterpret_cast<float2*>(h->win_ws + state_bytes);
  float* d_win = reinterpret_cast<float*>(h->win_ws + state_bytes + 256);
  float* d_acc[2] = {d_win + 2 * ld, d_win + 2 * ld + 8 * acap};
  float* d_out[2] = {d_acc[1] + 8 * acap, d_acc[1] + 16 * acap};
  for (int i = 0; i < 2; ++i) {
    if (!h->win_ev[i]) CK(cudaEventCreateWithFlags(&h->win_ev[i], cudaEventDisableTiming));
    if (!h->out_ev[i]) CK(cudaEventCreateWithFlags(&h->out_ev[i], cudaEventDisableTiming));
  }
  ensure_emit(h, acap);
  if (!h->copy_stream) {
    CK(cudaStreamCreateWithFlags(&h->copy_stream, cudaStreamNonBlocking));
    CK(cudaEventCreateWithFlags(&h->copy_ev, cudaEventDisableTiming));
  }
  ensure_io(h, batch);
  WindowReader reader{h, read, user, ld};
  h->launches = 0;

  // pass 1: the global moments (scan_norm, streaming.rs:52-78; scan_norm_file, mix.rs:61-120)
  h->mark("window.moments");
  CK(cudaMemsetAsync(d_state, 0, (size_t)moments_state_doubles() * sizeof(double), h->stream));
  for (int64_t t0 = 0; t0 < n; t0 += mwin) {
    const int64_t count = std::min<int64_t>(mwin, n - t0);
    reader.load(t0, count, d_win);
    launch_moments_window(d_win, d_win + ld, count, d_state, h->stream);
    ++h->launches;
  }
  launch_moments_final(d_state, n, d_norm, h->stream);
  h->launches += 2;
  CK(cudaGetLastError());

  // pass 2: the split passes (separate_forwarding_emit, pipeline.rs:380-515)
  const int passes = std::max(1, o.shifts);
  const float scale = o.shifts > 0 ? 1.0f / (float)o.shifts : 1.0f;
  const std::vector<int64_t> offsets =
      o.shifts > 0 ? shift_offsets(passes, max_shift) : std::vector<int64_t>(1, 0);
  size_t done = 0, total = 0;
  for (int pass = 0; pass < passes; ++pass) {
    const int64_t vlen = o.shifts > 0 ? n + max_shift - offsets[pass] : n;
    total += (size_t)((vlen + stride - 1) / stride);
  }
  PassSum psum;
  if (passes > 1) {
    psum.sum.assign((size_t)8 * n, 0.0f);
    psum.n = n;
  }
  HostSink sink;
  sink.emit = passes > 1 ? add_block : on_frames;
  sink.user = passes > 1 ? static_cast<void*>(&psum) : user;
  const int mode = o.shifts == 0 ? 0 : (o.shifts == 1 ? 1 : 4);
  bool out_used[2] = {false, false};
  int out_slot = 0;
  for (int pass = 0; pass < passes; ++pass) {
    const int64_t offset = offsets[pass];
    const int64_t vlen = o.shifts > 0 ? n + max_shift - offset : n;
    const int64_t chunks = (vlen + stride - 1) / stride;
    const int64_t trim = o.shifts > 0 ? max_shift - offset : 0;
    int cur = 0;
    int64_t acc_lo = 0, t_done = 0;
    CK(cudaMemsetAsync(d_acc[cur], 0, (size_t)8 * acap * sizeof(float), h->stream));
    for (int64_t c0 = 0; c0 < chunks; c0 += batch) {
      const int64_t c1 = std::min<int64_t>(chunks, c0 + batch);
      const int G = (int)(c1 - c0);
      int64_t m_lo, m_hi;
      group_mix_range(n, offset, max_shift, pg, vlen, c0, c1, &m_lo, &m_hi);
      if (m_hi - m_lo > wcap) throw Error(DMX_ERR_INVALID, "windowed driver: a mix window exceeds its buffer");
      h->mark("window.read");
      reader.load(m_lo, m_hi - m_lo, d_win);
      launch_normalize_window(d_win, ld, m_hi - m_lo, d_norm, h->stream);
      ++h->launches;
      DriverWindow w;
      w.mix_lo = m_lo;
      w.mix_ld = ld;
      w.mix_n = m_hi - m_lo;
      h->mark("track.gather");
      launch_gather_chunks(d_win, n, offset, max_shift, pg.chunk, stride, c0, G, h->io_in,
                           h->stream, kSegment, &w);
      ++h->launches;
      run_forward(h, h->io_in, G, h->io_out);
      h->mark("track.ola");
      launch_ola_accumulate(h->io_out, n, offset, max_shift, pg.chunk, stride, c0, G, pg.weight,
                            d_acc[cur], acc_lo, acc_lo + acap, h->stream, kSegment);
      ++h->launches;
      // view samples below chunk c1's start get no further contribution
      const int64_t t_hi =
          c1 == chunks ? n : std::min<int64_t>(n, std::max<int64_t>(0, c1 * stride - trim));
      if (t_hi > t_done) {
        const int slot = out_slot;
        out_slot ^= 1;
        // the block's previous contents have been copied out
        if (out_used[slot]) CK(cudaStreamWaitEvent(h->stream, h->out_ev[slot], 0));
        DriverWindow f;
        f.acc_lo = acc_lo;
        f.acc_ld = acap;
        f.out_lo = t_done;
        f.out_ld = acap;
        h->mark("track.finish");
        launch_ola_finish(d_acc[cur], n, offset, max_shift, pg.chunk, stride, pg.weight, d_norm,
                          scale, mode, nullptr, d_out[slot], h->stream, t_done, t_hi, &f);
        ++h->launches;
        CK(cudaEventRecord(h->copy_ev, h->stream));
        CK(cudaStreamWaitEvent(h->copy_stream, h->copy_ev, 0));
        sink.put(h, d_out[slot], acap, t_done, t_hi, t_done);
        CK(cudaEventRecord(h->out_ev[slot], h->copy_stream));
        out_used[slot] = true;
        t_done = t_hi;
      }
      // slide the accumulator to chunk c1's start; the samples it and the
      // chunks before it share carry over
      if (c1 < chunks) {
        const int64_t nlo = c1 * stride;
        const int64_t carry = std::max<int64_t>(0, (c1 - 1) * stride + pg.chunk - nlo);
        const int nxt = cur ^ 1;
        CK(cudaMemsetAsync(d_acc[nxt], 0, (size_t)8 * acap * sizeof(float), h->stream));
        if (carry > 0)
          CK(cudaMemcpy2DAsync(d_acc[nxt], (size_t)acap * sizeof(float), d_acc[cur] + (nlo - acc_lo),
                               (size_t)acap * sizeof(float), (size_t)carry * sizeof(float), 8,
                               cudaMemcpyDeviceToDevice, h->stream));
        cur = nxt;
        acc_lo = nlo;
      }
      CK(cudaGetLastError());
      done += (size_t)G;
      if (progress) {
        CK(cudaStreamSynchronize(h->stream));
        progress(done, total, user);
      }
    }
  }
  sink.flush(h);
  CK(cudaStreamSynchronize(h->copy_stream));
  CK(cudaStreamSynchronize(h->stream));
  check_device_flag(h);
  if (passes > 1) {
    // the scaled pass sum, denormalised (pipeline.rs:501-513 with
    // denormalize, pipeline.rs:60-67), in blocks through the emit staging:
    // each product and sum rounded on its own, as the device's finish does
    float2 nz;
    CK(cudaMemcpy(&nz, d_norm, sizeof(nz), cudaMemcpyDeviceToHost));
    float* block = h->emit_pin[0];
    for (int64_t t0 = 0; t0 < n; t0 += acap) {
      const int64_t count = std::min<int64_t>(acap, n - t0);
      for (int r = 0; r < 8; ++r) {
        const float* src = psum.sum.data() + (size_t)r * n + t0;
        float* dst = block + (size_t)r * count;
        for (int64_t i = 0; i < count; ++i) {
          volatile float scaled = src[i] * scale;
          volatile float spread = scaled * nz.y;
          dst[i] = spread + nz.x;
        }
      }
      on_frames(t0, count, block, user);
    }
  }
  h->mark("end");
}

}  // namespace dmx

extern "C" dmx_status dmx_separate_track_windowed(dmx_handle* h, dmx_read_fn read, int64_t n,
                                                  const dmx_separate_opts* opts,
                                                  dmx_frames_fn on_frames,
                                                  dmx_progress_fn progress, void* user) {
  using namespace dmx;
  try {
    if (!h || !read || !on_frames || n <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_separate_track_windowed: bad argument");
    try {
      separate_windowed_impl(h, read, n, opts, on_frames, progress, user);
    } catch (...) {
      // no copy into or out of the pinned staging outlives the call
      cudaStreamSynchronize(h->stream);
      if (h->copy_stream) cudaStreamSynchronize(h->copy_stream);
      throw;
    }
    finish_stage_times(h);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}
