// The C ABI of include/dmx.h: argument checks, the status codes and the
// thread-local error text around the runtime (loader.cu, forward.cu,
// track.cu). Nothing here throws across the boundary.
#include <chrono>
#include <cstdio>
#include <thread>

#include "runtime.cuh"

using namespace dmx;

namespace {
thread_local std::string g_error;
}  // namespace

namespace dmx {

int fail(const Error& e) {
  g_error = e.what();
  return e.code;
}
int fail_std(const std::exception& e) {
  g_error = e.what();
  return DMX_ERR_INVALID;
}

// Lets other translation units (noalloc.cu) report through dmx_last_error.
void set_last_error(const char* msg) { g_error = msg; }

}  // namespace dmx

extern "C" {

void dmx_default_config(dmx_config* c) {
  c->sources = 4;
  c->audio_channels = 2;
  c->samplerate = 44100;
  c->segment_samples = kSegment;
  c->precision = DMX_FP32;
  c->max_batch = 8;
}

const char* dmx_last_error(void) { return g_error.c_str(); }

dmx_status dmx_create(const dmx_config* cfg, const void* blob, size_t len, int device,
                      dmx_handle** out) {
  if (!cfg || !blob || !out) {
    g_error = "dmx_create: null argument";
    return DMX_ERR_INVALID;
  }
  std::unique_ptr<dmx_handle> h(new dmx_handle());
  try {
    if (cfg->sources != 4 || cfg->audio_channels != 2 || cfg->samplerate != 44100 ||
        cfg->segment_samples != kSegment)
      throw Error(DMX_ERR_INVALID,
                  "only the default htdemucs configuration is supported (4 sources, stereo, "
                  "44100 Hz, 343980-sample segments)");
    if (cfg->precision != DMX_FP32 && cfg->precision != DMX_TF32 &&
        cfg->precision != DMX_TF32X3 && cfg->precision != DMX_BF16)
      throw Error(DMX_ERR_INVALID, "precision must be DMX_FP32, DMX_TF32, DMX_BF16 or DMX_TF32X3");
    if (cfg->max_batch < 1 || cfg->max_batch > 256)
      throw Error(DMX_ERR_INVALID, "max_batch must be in [1, 256]");
    h->cfg = *cfg;
    h->device = device;
    const auto tensors = parse_checkpoint(blob, len);  // validated before any CUDA call
    CK(cudaSetDevice(device));
    CK(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));
    CK(cudaMalloc(&h->err, sizeof(int)));
    CK(cudaMemset(h->err, 0, sizeof(int)));
    load_model(h.get(), tensors);
    const char* st = getenv("DMX_STAGE_TIMING");
    h->stage_timing = st && st[0] == '1';
    *out = h.release();
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

void dmx_destroy(dmx_handle* h) {
  if (!h) return;
  cudaSetDevice(h->device);
  if (h->stream) cudaStreamSynchronize(h->stream);
  for (dmx_pending& p : h->pending) {
    if (p.done) cudaEventDestroy(p.done);
    cudaFree(p.in_dev);
    cudaFree(p.out_dev);
    cudaFreeHost(p.pin_in);
    cudaFreeHost(p.pin_out);
  }
  cudaFree(h->ola_w_custom);
  cudaFree(h->wdev);
  cudaFree(h->err);
  cudaFree(h->ws);
  cudaFree(h->io_in);
  cudaFree(h->io_out);
  cudaFree(h->track_ws);
  cudaFree(h->host_io);
  cudaFree(h->norm_scratch);
  cudaFree(h->bag_out);
  if (h->copy_stream) cudaStreamSynchronize(h->copy_stream);
  if (h->copy_ev) cudaEventDestroy(h->copy_ev);
  for (int i = 0; i < 2; ++i) {
    if (h->emit_ev[i]) cudaEventDestroy(h->emit_ev[i]);
    cudaFreeHost(h->emit_pin[i]);
  }
  if (h->copy_stream) cudaStreamDestroy(h->copy_stream);
  cudaFree(h->win_ws);
  for (int i = 0; i < 2; ++i) {
    cudaFreeHost(h->win_pin[i]);
    if (h->win_ev[i]) cudaEventDestroy(h->win_ev[i]);
    if (h->out_ev[i]) cudaEventDestroy(h->out_ev[i]);
  }
  cudaFree(h->batch_ws);
  cudaFree(h->tail_buf);
  if (h->shard_done) cudaEventDestroy(h->shard_done);
  cudaFree(h->batch_io);
  if (h->stream) cudaStreamDestroy(h->stream);
  delete h;
}

dmx_status dmx_set_trace(dmx_handle* h, dmx_trace_fn fn, void* user) {
  if (!h) return DMX_ERR_INVALID;
  h->trace = fn;
  h->trace_user = user;
  return DMX_OK;
}

dmx_status dmx_forward_device(dmx_handle* h, const float* mix_dev, int64_t n, float* out_dev,
                              void* stream) {
  try {
    CK(cudaSetDevice(h->device));
    h->launches = 0;
    cudaStream_t user = static_cast<cudaStream_t>(stream);
    if (user && user != h->stream) {
      cudaEvent_t e;
      CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
      CK(cudaEventRecord(e, user));
      CK(cudaStreamWaitEvent(h->stream, e, 0));
      run_forward(h, mix_dev, n, out_dev);
      CK(cudaEventRecord(e, h->stream));
      CK(cudaStreamWaitEvent(user, e, 0));
      CK(cudaEventDestroy(e));
    } else {
      run_forward(h, mix_dev, n, out_dev);
    }
    h->mark("end");
    finish_stage_times(h);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_forward_start(dmx_handle* h, const float* mix, int64_t n, dmx_pending** out) {
  try {
    if (!h || !mix || !out || n <= 0) throw Error(DMX_ERR_INVALID, "dmx_forward_start: bad argument");
    dmx_pending* p = nullptr;
    for (dmx_pending& q : h->pending)
      if (!q.busy) {
        p = &q;
        break;
      }
    if (!p)
      throw Error(DMX_ERR_INVALID, "dmx_forward_start: " + std::to_string(kPendingSlots) +
                                       " forwards are already in flight on this handle; collect "
                                       "one first");
    CK(cudaSetDevice(h->device));
    h->launches = 0;
    if (n > p->cap) {  // this slot's staging is free: nothing in flight uses it
      cudaFree(p->in_dev);
      cudaFree(p->out_dev);
      cudaFreeHost(p->pin_in);
      cudaFreeHost(p->pin_out);
      p->in_dev = p->out_dev = p->pin_in = p->pin_out = nullptr;
      p->cap = 0;
      CK(cudaMalloc(&p->in_dev, (size_t)n * 2 * kSegment * sizeof(float)));
      CK(cudaMalloc(&p->out_dev, (size_t)n * 8 * kSegment * sizeof(float)));
      CK(cudaMallocHost(&p->pin_in, (size_t)n * 2 * kSegment * sizeof(float)));
      CK(cudaMallocHost(&p->pin_out, (size_t)n * 8 * kSegment * sizeof(float)));
      p->cap = n;
    }
    if (!p->done) CK(cudaEventCreateWithFlags(&p->done, cudaEventDisableTiming));
    // the caller's array is copied before this returns: it may be freed or
    // reused at once (the reference drops its batch before collect)
    std::memcpy(p->pin_in, mix, (size_t)n * 2 * kSegment * sizeof(float));
    CK(cudaMemcpyAsync(p->in_dev, p->pin_in, (size_t)n * 2 * kSegment * sizeof(float),
                       cudaMemcpyHostToDevice, h->stream));
    run_forward(h, p->in_dev, n, p->out_dev);
    h->mark("end");
    CK(cudaMemcpyAsync(p->pin_out, p->out_dev, (size_t)n * 8 * kSegment * sizeof(float),
                       cudaMemcpyDeviceToHost, h->stream));
    CK(cudaEventRecord(p->done, h->stream));
    p->h = h;
    p->n = n;
    p->seq = ++h->pending_seq;
    p->busy = true;
    *out = p;
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_forward_collect(dmx_pending* p, float* out) {
  try {
    if (!p || !p->h || !p->busy || !out)
      throw Error(DMX_ERR_INVALID, "dmx_forward_collect: bad argument (not a queued forward)");
    dmx_handle* h = p->h;
    CK(cudaSetDevice(h->device));
    // bounded wait: poll the event with a deadline instead of blocking forever
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(600);
    while (true) {
      const cudaError_t e = cudaEventQuery(p->done);
      if (e == cudaSuccess) break;
      if (e != cudaErrorNotReady) {
        p->busy = false;
        CK(e);
      }
      if (std::chrono::steady_clock::now() > deadline) {
        p->busy = false;
        throw Error(DMX_ERR_TIMEOUT, "forward did not complete within the deadline");
      }
      std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    p->busy = false;
    check_device_flag(h);
    std::memcpy(out, p->pin_out, (size_t)p->n * 8 * kSegment * sizeof(float));
    bool others = false;  // stage times cover the forwards up to the last one collected
    for (const dmx_pending& q : h->pending) others = others || q.busy;
    if (!others) finish_stage_times(h);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_normalize_track_device(dmx_handle* h, const float* lr_dev, int64_t n,
                                      float* mix_norm_dev, float* mean_std_dev) {
  try {
    if (!h || !lr_dev || !mix_norm_dev || !mean_std_dev || n <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_normalize_track_device: bad argument");
    if ((reinterpret_cast<uintptr_t>(mean_std_dev) & 7) != 0)
      throw Error(DMX_ERR_INVALID, "mean_std_dev must be 8-byte aligned");
    CK(cudaSetDevice(h->device));
    const size_t need = (size_t)track_normalize_scratch_doubles() * sizeof(double);
    if (need > h->norm_cap) {
      cudaFree(h->norm_scratch);
      h->norm_scratch = nullptr;
      h->norm_cap = 0;
      CK(cudaMalloc(&h->norm_scratch, need));
      h->norm_cap = need;
    }
    launch_track_normalize(lr_dev, lr_dev + n, n, h->norm_scratch, mix_norm_dev,
                           reinterpret_cast<float2*>(mean_std_dev), h->stream);
    CK(cudaGetLastError());
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_track_finish(dmx_handle* h, const float* acc_dev, int64_t length,
                            int64_t shift_offset, int64_t max_shift, int segment, double overlap,
                            double transition_power, int shifts, const float* mean_std_dev,
                            float* stems_dev, int64_t t_lo, int64_t t_hi) {
  try {
    if (!h || !acc_dev || !mean_std_dev || !stems_dev || length <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_track_finish: bad argument");
    if (shifts < 0 || shifts > 1)
      throw Error(DMX_ERR_INVALID, "dmx_track_finish handles a single pass (shifts 0 or 1)");
    CK(cudaSetDevice(h->device));
    const PassGeom pg = pass_geom(h, segment, overlap, transition_power);
    h->mark("track.finish");
    launch_ola_finish(acc_dev, length, shift_offset, max_shift, pg.chunk, pg.stride, pg.weight,
                      reinterpret_cast<const float2*>(mean_std_dev), 1.0f, shifts, nullptr,
                      stems_dev, h->stream, t_lo, t_hi);
    CK(cudaGetLastError());
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_read_tensor(const void* blob, size_t len, const char* name, float* out,
                           int64_t cap, int64_t* shape, int* ndim) {
  try {
    if (!blob || !name || !out || !shape || !ndim || cap < 0)
      throw Error(DMX_ERR_INVALID, "dmx_read_tensor: bad argument");
    const auto tensors = parse_checkpoint(blob, len);
    auto it = tensors.find(name);
    if (it == tensors.end()) throw Error(DMX_ERR_WEIGHTS, std::string("missing tensor ") + name);
    const HostTensor& t = it->second;
    if (t.shape.size() > 8) throw Error(DMX_ERR_INVALID, "dmx_read_tensor: more than 8 dimensions");
    if ((int64_t)t.count() > cap)
      throw Error(DMX_ERR_INVALID, std::string(name) + ": " + std::to_string(t.count()) +
                                       " elements do not fit in " + std::to_string(cap));
    std::memcpy(out, t.data, t.count() * sizeof(float));
    for (size_t i = 0; i < t.shape.size(); ++i) shape[i] = t.shape[i];
    *ndim = (int)t.shape.size();
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_shift_offsets(int passes, int64_t max_shift, int64_t* out) {
  try {
    if (passes < 0 || max_shift < 0 || (passes > 0 && !out))
      throw Error(DMX_ERR_INVALID, "dmx_shift_offsets: bad argument");
    const std::vector<int64_t> v = shift_offsets(passes, max_shift);
    std::copy(v.begin(), v.end(), out);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

int64_t dmx_num_chunks(int64_t view_length, int segment, double overlap) {
  const int64_t stride = (int64_t)((1.0 - overlap) * (double)segment);
  if (view_length <= 0 || stride <= 0) return 0;
  return (view_length + stride - 1) / stride;
}

}  // extern "C"

extern "C" {

dmx_status dmx_separate_track_multi(dmx_handle* const* hs, int n_handles, const float* left,
                                    const float* right, int64_t n, const dmx_separate_opts* opts,
                                    float* stems_out) {
  std::vector<dmx_handle*> H;
  auto drain = [&] {  // no copy into the caller's memory outlives the call
    for (dmx_handle* h : H) {
      cudaSetDevice(h->device);
      cudaStreamSynchronize(h->stream);
    }
  };
  try {
    if (!hs || n_handles < 1 || n_handles > 64 || !left || !right || !stems_out || n <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_separate_track_multi: bad argument");
    for (int k = 0; k < n_handles; ++k) {
      if (!hs[k]) throw Error(DMX_ERR_INVALID, "handle " + std::to_string(k) + " is NULL");
      for (dmx_handle* o : H)
        if (o == hs[k]) throw Error(DMX_ERR_INVALID, "each rank needs its own handle");
      H.push_back(hs[k]);
    }
    separate_track_multi_impl(H, left, right, n, opts, stems_out);
    return DMX_OK;
  } catch (const Error& e) {
    drain();
    return fail(e);
  } catch (const std::exception& e) {
    drain();
    return fail_std(e);
  }
}

dmx_status dmx_separate_batch_device(dmx_handle* h, const float* const* lr_dev,
                                     const int64_t* lengths, int n_tracks,
                                     const dmx_separate_opts* opts, float* const* stems_dev,
                                     dmx_progress_fn progress, void* user) {
  try {
    if (!h) throw Error(DMX_ERR_INVALID, "dmx_separate_batch_device: bad argument");
    separate_batch_impl(h, lr_dev, lengths, n_tracks, opts, stems_dev, progress, user);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_separate_batch(dmx_handle* h, const float* const* left, const float* const* right,
                              const int64_t* lengths, int n_tracks, const dmx_separate_opts* opts,
                              float* const* stems_out, dmx_progress_fn progress, void* user) {
  try {
    if (!h || !left || !right || !lengths || !stems_out || n_tracks < 1)
      throw Error(DMX_ERR_INVALID, "dmx_separate_batch: bad argument");
    CK(cudaSetDevice(h->device));
    int64_t sum = 0;
    for (int i = 0; i < n_tracks; ++i) {
      if (lengths[i] <= 0 || !left[i] || !right[i] || !stems_out[i])
        throw Error(DMX_ERR_INVALID, "track " + std::to_string(i) + " is empty or has no buffer");
      sum += lengths[i];
    }
    // every track's input (2 n) and stems (8 n) stay on the device for the call
    const size_t need = (size_t)10 * sum * sizeof(float);
    if (need > h->batch_io_cap) {
      cudaFree(h->batch_io);
      h->batch_io = nullptr;
      h->batch_io_cap = 0;
      CK(cudaMalloc(&h->batch_io, need));
      h->batch_io_cap = need;
    }
    std::vector<const float*> d_lr(n_tracks);
    std::vector<float*> d_stems(n_tracks);
    float* at = h->batch_io;
    for (int i = 0; i < n_tracks; ++i) {
      const int64_t n = lengths[i];
      d_lr[i] = at;
      CK(cudaMemcpyAsync(at, left[i], n * sizeof(float), cudaMemcpyHostToDevice, h->stream));
      CK(cudaMemcpyAsync(at + n, right[i], n * sizeof(float), cudaMemcpyHostToDevice, h->stream));
      d_stems[i] = at + 2 * n;
      at += 10 * n;
    }
    separate_batch_impl(h, d_lr.data(), lengths, n_tracks, opts, d_stems.data(), progress, user);
    for (int i = 0; i < n_tracks; ++i)
      CK(cudaMemcpyAsync(stems_out[i], d_stems[i], 8 * lengths[i] * sizeof(float),
                         cudaMemcpyDeviceToHost, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    check_device_flag(h);
    finish_stage_times(h);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_track_shard(dmx_handle* h, const float* mix_norm_dev, int64_t length,
                           int64_t shift_offset, int64_t max_shift, int segment, double overlap,
                           double transition_power, int64_t chunk_lo, int64_t chunk_hi, int batch,
                           float* acc_dev, int64_t view_lo, int64_t view_hi) {
  try {
    if (!h || !mix_norm_dev || !acc_dev || length <= 0 || chunk_lo < 0 || chunk_hi < chunk_lo)
      throw Error(DMX_ERR_INVALID, "dmx_track_shard: bad argument");
    CK(cudaSetDevice(h->device));
    const PassGeom pg = pass_geom(h, segment, overlap, transition_power);
    const int cap = std::max(1, batch > 0 ? std::min(batch, h->cfg.max_batch) : h->cfg.max_batch);
    shard_chunks(h, nullptr, mix_norm_dev, length, shift_offset, max_shift, pg, chunk_lo, chunk_hi,
                 cap, acc_dev, view_lo, view_hi);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_separate_track_device(dmx_handle* h, const float* lr_dev, int64_t n,
                                     const dmx_separate_opts* opts, float* d_stems,
                                     dmx_progress_fn progress, void* user) {
  try {
    if (!h || !lr_dev || !d_stems || n <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_separate_track_device: bad argument");
    separate_track_impl(h, nullptr, lr_dev, n, opts, d_stems, progress, user);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_bag_combine_device(const float* const* outs_dev, int n_nets, const float* weights,
                                  const int* requested, int64_t n_segments, int64_t samples,
                                  float* combined_dev, void* stream) {
  try {
    if (!outs_dev || !combined_dev || n_segments <= 0 || samples <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_bag_combine_device: bad argument");
    std::vector<int> slot;
    BagTerms t = bag_terms(n_nets, weights, requested, &slot);
    for (int k = 0; k < n_nets; ++k) {
      if (slot[k] < 0) continue;
      if (!outs_dev[k])
        throw Error(DMX_ERR_INVALID, "bag output " + std::to_string(k) + " is NULL but weighted");
      t.out[slot[k]] = outs_dev[k];
    }
    launch_bag_combine(t, n_segments, samples, combined_dev, static_cast<cudaStream_t>(stream));
    CK(cudaGetLastError());
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_bag_forward_device(dmx_handle* const* nets, int n_nets, const float* weights,
                                  const int* requested, const float* mix_dev, int64_t n,
                                  float* out_dev) {
  try {
    if (!mix_dev || !out_dev || n <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_bag_forward_device: bad argument");
    BagPlan bag;
    make_bag(nets, n_nets, weights, requested, &bag);
    dmx_handle* lead = bag.nets[0];
    lead->launches = 0;
    int cap = lead->cfg.max_batch;
    for (dmx_handle* hk : bag.nets) cap = std::min(cap, hk->cfg.max_batch);
    cap = std::max(1, cap);
    for (int64_t s0 = 0; s0 < n; s0 += cap) {
      const int G = (int)std::min<int64_t>(cap, n - s0);
      bag_forward(lead, bag, mix_dev + s0 * 2 * kSegment, G, out_dev + s0 * 8 * kSegment);
    }
    lead->mark("end");
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_separate_track_bag_device(dmx_handle* const* nets, int n_nets, const float* weights,
                                         const int* requested, const float* lr_dev, int64_t n,
                                         const dmx_separate_opts* opts, float* stems_dev,
                                         dmx_progress_fn progress, void* user) {
  try {
    if (!lr_dev || !stems_dev || n <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_separate_track_bag_device: bad argument");
    BagPlan bag;
    make_bag(nets, n_nets, weights, requested, &bag);
    separate_track_impl(bag.nets[0], &bag, lr_dev, n, opts, stems_dev, progress, user);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_separate_track_bag(dmx_handle* const* nets, int n_nets, const float* weights,
                                  const int* requested, const float* left, const float* right,
                                  int64_t n, const dmx_separate_opts* opts, float* stems_out,
                                  dmx_progress_fn progress, void* user) {
  try {
    if (!left || !right || !stems_out || n <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_separate_track_bag: bad argument");
    BagPlan bag;
    make_bag(nets, n_nets, weights, requested, &bag);
    separate_track_host(bag.nets[0], &bag, left, right, n, opts, stems_out, progress, user);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_separate_track(dmx_handle* h, const float* left, const float* right, int64_t n,
                              const dmx_separate_opts* opts, float* stems_out,
                              dmx_progress_fn progress, void* user) {
  try {
    if (!h || !left || !right || !stems_out || n <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_separate_track: bad argument");
    separate_track_host(h, nullptr, left, right, n, opts, stems_out, progress, user);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_separate_track_emit(dmx_handle* h, const float* left, const float* right, int64_t n,
                                   const dmx_separate_opts* opts, dmx_frames_fn on_frames,
                                   dmx_progress_fn progress, void* user) {
  try {
    if (!h || !left || !right || !on_frames || n <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_separate_track_emit: bad argument");
    CK(cudaSetDevice(h->device));
    const dmx_separate_opts o = separate_opts(opts);
    const PassGeom pg = pass_geom(h, chunk_samples(o), o.overlap, o.transition_power);
    const int batch = std::max(1, o.batch > 0 ? std::min(o.batch, h->cfg.max_batch) : h->cfg.max_batch);
    // a block holds what one forward finishes: at most `batch` strides plus one segment
    ensure_emit(h, std::min<int64_t>(n, (int64_t)batch * pg.stride + pg.chunk));
    const size_t need = (size_t)10 * n * sizeof(float);
    if (need > h->host_io_cap) {
      cudaFree(h->host_io);
      h->host_io = nullptr;
      h->host_io_cap = 0;
      CK(cudaMalloc(&h->host_io, need));
      h->host_io_cap = need;
    }
    float* d_lr = h->host_io;
    float* d_stems = h->host_io + 2 * n;
    CK(cudaMemcpyAsync(d_lr, left, n * sizeof(float), cudaMemcpyHostToDevice, h->stream));
    CK(cudaMemcpyAsync(d_lr + n, right, n * sizeof(float), cudaMemcpyHostToDevice, h->stream));
    HostSink sink;
    sink.emit = on_frames;
    sink.user = user;
    try {
      separate_track_impl(h, nullptr, d_lr, n, &o, d_stems, progress, user, &sink);
    } catch (...) {
      cudaStreamSynchronize(h->copy_stream);  // no copy into the staging outlives the call
      throw;
    }
    CK(cudaStreamSynchronize(h->stream));
    check_device_flag(h);
    finish_stage_times(h);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_selftest_wait_timeout(dmx_handle* h, int wait_ms) {
  try {
    if (!h || wait_ms < 1 || wait_ms > 5000)
      throw Error(DMX_ERR_INVALID, "dmx_selftest_wait_timeout: wait_ms must be in [1, 5000]");
    CK(cudaSetDevice(h->device));
    launch_selftest_wait((uint64_t)wait_ms * 1000000ull, kSelftestCode, h->err, h->stream);
    CK(cudaGetLastError());
    CK(cudaStreamSynchronize(h->stream));  // ends: the kernel's wait is bounded
    check_device_flag(h);                  // turns the raised flag into DMX_ERR_TIMEOUT
    throw Error(DMX_ERR_INVALID, "dmx_selftest_wait_timeout: the wait did not report giving up");
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

int dmx_stage_times(dmx_handle* h, const char** names, float* ms, int* counts, double* flops,
                    double* bytes, int cap) {
  if (!h) return 0;
  const int n = std::min<int>(cap, (int)h->stage_names.size());
  for (int i = 0; i < n; ++i) {
    names[i] = h->stage_names[i].c_str();
    ms[i] = h->stage_ms[i];
    if (counts) counts[i] = h->stage_counts[i];
    if (flops) flops[i] = h->stage_flops[i];
    if (bytes) bytes[i] = h->stage_bytes[i];
  }
  return n;
}

dmx_status dmx_set_stage_timing(dmx_handle* h, int on) {
  if (!h) return DMX_ERR_INVALID;
  h->stage_timing = on != 0;
  return DMX_OK;
}

int64_t dmx_kernel_launches(dmx_handle* h) { return h ? h->launches : 0; }

void* dmx_stream(dmx_handle* h) { return h ? static_cast<void*>(h->stream) : nullptr; }

dmx_status dmx_synchronize(dmx_handle* h) {
  try {
    if (!h) throw Error(DMX_ERR_INVALID, "dmx_synchronize: null handle");
    CK(cudaSetDevice(h->device));
    // bounded wait on the handle's stream
    cudaEvent_t e;
    CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    CK(cudaEventRecord(e, h->stream));
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(600);
    while (true) {
      const cudaError_t q = cudaEventQuery(e);
      if (q == cudaSuccess) break;
      if (q != cudaErrorNotReady) {
        cudaEventDestroy(e);
        CK(q);
      }
      if (std::chrono::steady_clock::now() > deadline) {
        cudaEventDestroy(e);
        throw Error(DMX_ERR_TIMEOUT, "the handle's stream did not drain within the deadline");
      }
      std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    CK(cudaEventDestroy(e));
    check_device_flag(h);
    finish_stage_times(h);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  }
}

}  // extern "C"
