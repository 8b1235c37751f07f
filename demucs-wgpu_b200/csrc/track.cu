// The separation drivers on the device (Demucs::separate and its split
// passes: api.rs:438-545, 697-785; pipeline.rs:105-151, 380-515;
// streaming.rs:52-400; mix.rs:552-633): global normalisation, the ShiftRng
// shift views, centred chunks batched into forwards, the triangular
// overlap-add and its finish. Over one network, a bag of networks
// (BagCombineForward, api.rs:319-371), many pooled tracks, or one track's
// chunks spread over several GPUs.
#include <cmath>

#include "runtime.cuh"

namespace dmx {

// ShiftRng (pipeline.rs:136-151): state = seed * A + 1, then per draw
// state = state * A + C and randint(max) = (state >> 33) % (max + 1). Every
// separation seeds a fresh generator with 0x5eed_1234 (pipeline.rs:416-418).
std::vector<int64_t> shift_offsets(int passes, int64_t max_shift) {
  constexpr uint64_t kA = 6364136223846793005ULL, kC = 1442695040888963407ULL;
  uint64_t state = 0x5eed1234ULL * kA + 1ULL;
  std::vector<int64_t> out;
  for (int p = 0; p < passes; ++p) {
    state = state * kA + kC;
    out.push_back((int64_t)((state >> 33) % (uint64_t)(max_shift + 1)));
  }
  return out;
}

dmx_separate_opts separate_opts(const dmx_separate_opts* opts) {
  dmx_separate_opts o{1, 0.25, 1.0, 0, 0.0};
  if (opts) o = *opts;
  if (o.shifts < 0) throw Error(DMX_ERR_INVALID, "shifts must be >= 0");
  if (!(o.overlap >= 0.0 && o.overlap < 1.0))
    throw Error(DMX_ERR_INVALID, "overlap must be in [0, 1): it leaves a zero stride otherwise");
  if (!(o.transition_power > 0.0) || !std::isfinite(o.transition_power))
    throw Error(DMX_ERR_INVALID, "transition_power must be a positive finite number");
  if (o.segment < 0.0 || !std::isfinite(o.segment))
    throw Error(DMX_ERR_INVALID, "segment must be 0 (the model's) or a positive duration");
  return o;
}

// The chunk length is int(samplerate * segment) (streaming.rs:315-317); a
// chunk longer than the model's training length cannot be forwarded
// (host.rs:210-216). The transition weight (pipeline.rs:117-131) of the
// default geometry is built once at dmx_create; any other is built here on
// the host, in f32 as the reference does, and uploaded once per change.
int64_t chunk_samples(const dmx_separate_opts& o) {
  return o.segment > 0.0 ? (int64_t)(44100.0 * o.segment) : (int64_t)kSegment;
}

PassGeom pass_geom(dmx_handle* h, int64_t chunk, double overlap, double transition_power) {
  PassGeom g;
  if (chunk < 1) throw Error(DMX_ERR_INVALID, "segment is shorter than one sample");
  if (chunk > kSegment)
    throw Error(DMX_ERR_INVALID, "segment is " + std::to_string(chunk) +
                                     " samples but the model segment is 343980; chunks cannot "
                                     "be longer than the model's training length");
  if (!(transition_power > 0.0) || !std::isfinite(transition_power))
    throw Error(DMX_ERR_INVALID, "transition_power must be a positive finite number");
  g.chunk = (int)chunk;
  g.stride = (int64_t)((1.0 - overlap) * (double)chunk);
  if (g.stride <= 0) throw Error(DMX_ERR_INVALID, "overlap leaves a zero stride");
  if (g.chunk == kSegment && transition_power == 1.0) {
    g.weight = h->W(h->m.ola_w.off);
    return g;
  }
  if (h->ola_w_len != g.chunk || h->ola_w_power != transition_power) {
    const int half = g.chunk / 2;
    std::vector<float> w;
    w.reserve(g.chunk);
    for (int i = 1; i <= half; ++i) w.push_back((float)i);
    for (int i = g.chunk - half; i >= 1; --i) w.push_back((float)i);
    float mx = 0.f;
    for (float v : w) mx = std::max(mx, v);
    mx = std::max(mx, 1.0f);
    for (float& v : w) v = std::pow(v / mx, (float)transition_power);
    if (!h->ola_w_custom) CK(cudaMalloc(&h->ola_w_custom, (size_t)kSegment * sizeof(float)));
    h->ola_w_len = 0;
    // queued work may still read the previous table: the upload follows it on the stream
    CK(cudaMemcpyAsync(h->ola_w_custom, w.data(), (size_t)g.chunk * sizeof(float),
                       cudaMemcpyHostToDevice, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    h->ola_w_len = g.chunk;
    h->ola_w_power = transition_power;
  }
  g.weight = h->ola_w_custom;
  return g;
}

// Fills t.net / weight / count / total from `weights` (n_nets x sources, row
// per network) and `requested` (sources flags, NULL = all); `slot[k]` is the
// index network k gets in t.out (-1 = it does not run).
BagTerms bag_terms(int n_nets, const float* weights, const int* requested, std::vector<int>* slot) {
  if (n_nets < 1 || n_nets > kBagMaxNets)
    throw Error(DMX_ERR_INVALID, "a bag holds 1 to " + std::to_string(kBagMaxNets) + " networks");
  if (!weights) throw Error(DMX_ERR_INVALID, "bag weights are missing");
  constexpr int S = kBagMaxSources;
  auto req = [&](int s) { return requested == nullptr || requested[s] != 0; };
  BagTerms t{};
  t.sources = S;
  t.channels = 2;
  slot->assign(n_nets, -1);
  int used = 0;
  for (int k = 0; k < n_nets; ++k)
    for (int s = 0; s < S; ++s)
      if (weights[k * S + s] != 0.0f && req(s) && (*slot)[k] < 0) (*slot)[k] = used++;
  for (int s = 0; s < S; ++s) {
    if (!req(s)) continue;
    float total = 0.0f;
    int c = 0;
    for (int k = 0; k < n_nets; ++k) {
      const float w = weights[k * S + s];
      if (w == 0.0f) continue;
      t.net[s][c] = (*slot)[k];
      t.weight[s][c] = w;
      ++c;
      total += w;
    }
    if (total == 0.0f)  // api.rs:355-359
      throw Error(DMX_ERR_INVALID, "no network covers stem index " + std::to_string(s));
    t.count[s] = c;
    t.total[s] = total;
  }
  return t;
}

void make_bag(dmx_handle* const* nets, int n_nets, const float* weights, const int* requested,
              BagPlan* b) {
  if (!nets) throw Error(DMX_ERR_INVALID, "bag networks are missing");
  std::vector<int> slot;
  b->terms = bag_terms(n_nets, weights, requested, &slot);
  for (int k = 0; k < n_nets; ++k) {
    if (slot[k] < 0) continue;
    dmx_handle* hk = nets[k];
    if (!hk) throw Error(DMX_ERR_INVALID, "bag network " + std::to_string(k) + " is NULL");
    if (!b->nets.empty() && hk->device != b->nets[0]->device)
      throw Error(DMX_ERR_INVALID,
                  "the networks of a bag must share one device (for one network per GPU run "
                  "one process per GPU and combine with dmx_bag_combine_device)");
    for (dmx_handle* o : b->nets)
      if (o == hk) throw Error(DMX_ERR_INVALID, "each network of a bag needs its own handle");
    b->nets.push_back(hk);
  }
  if (b->nets.empty())
    throw Error(DMX_ERR_INVALID, "no stem is requested, so no network of the bag would run");
  CK(cudaSetDevice(b->nets[0]->device));
  CK(cudaEventCreateWithFlags(&b->ev, cudaEventDisableTiming));
}

static void ensure_bag_out(dmx_handle* h, int64_t G) {
  if (G <= h->bag_cap) return;
  cudaFree(h->bag_out);
  h->bag_out = nullptr;
  h->bag_cap = 0;
  CK(cudaMalloc(&h->bag_out, (size_t)G * 8 * kSegment * sizeof(float)));
  h->bag_cap = G;
}

// BagCombineForward::start (api.rs:326-361) on device: each running network
// forwards the same padded chunks (one after another, ordered by events on
// their streams), then the per-source weighted combination is written to
// `out` on the lead network's stream.
void bag_forward(dmx_handle* lead, BagPlan& b, const float* in, int G, float* out) {
  cudaStream_t prev = lead->stream;
  for (size_t i = 0; i < b.nets.size(); ++i) {
    dmx_handle* hk = b.nets[i];
    CK(cudaSetDevice(hk->device));
    ensure_bag_out(hk, G);
    if (hk->stream != prev) {
      CK(cudaEventRecord(b.ev, prev));
      CK(cudaStreamWaitEvent(hk->stream, b.ev, 0));
    }
    const int64_t before = hk->launches;
    run_forward(hk, in, G, hk->bag_out);
    if (hk != lead) lead->launches += hk->launches - before;
    b.terms.out[i] = hk->bag_out;
    prev = hk->stream;
  }
  if (prev != lead->stream) {
    CK(cudaEventRecord(b.ev, prev));
    CK(cudaStreamWaitEvent(lead->stream, b.ev, 0));
  }
  int64_t reads = 0;
  for (int s = 0; s < b.terms.sources; ++s) reads += b.terms.count[s];
  lead->mark("bag.combine", 0.0, (double)G * 2 * kSegment * 4.0 * (double)(reads + 4));
  launch_bag_combine(b.terms, G, kSegment, out, lead->stream);
  ++lead->launches;
  CK(cudaGetLastError());
}

// Chunks [chunk_lo, chunk_hi) of a shift view: gather, forward (one network,
// or the bag when `bag` is set), overlap-add into acc_dev.
void shard_chunks(dmx_handle* h, BagPlan* bag, const float* mix_norm_dev, int64_t length,
                  int64_t shift_offset, int64_t max_shift, const PassGeom& pg, int64_t chunk_lo,
                  int64_t chunk_hi, int cap, float* acc_dev, int64_t view_lo, int64_t view_hi) {
  ensure_io(h, cap);
  for (int64_t c0 = chunk_lo; c0 < chunk_hi; c0 += cap) {
    const int G = (int)std::min<int64_t>(cap, chunk_hi - c0);
    h->mark("track.gather");
    launch_gather_chunks(mix_norm_dev, length, shift_offset, max_shift, pg.chunk, pg.stride, c0, G,
                         h->io_in, h->stream, kSegment);
    ++h->launches;
    if (bag)
      bag_forward(h, *bag, h->io_in, G, h->io_out);
    else
      run_forward(h, h->io_in, G, h->io_out);
    h->mark("track.ola");
    launch_ola_accumulate(h->io_out, length, shift_offset, max_shift, pg.chunk, pg.stride, c0, G,
                          pg.weight, acc_dev, view_lo, view_hi, h->stream, kSegment);
    ++h->launches;
    CK(cudaGetLastError());
  }
}

// Pinned host stems that a single-pass separation fills while it runs: after
// each forward batch the output samples that no later chunk touches are
// finished and copied on the handle's copy stream, so the device-to-host
// copy overlaps the remaining forwards (the reference emits frames the same
// way as soon as they are final: streaming.rs:219-260).
void HostSink::flush(dmx_handle* h) {
  if (pending_count == 0) return;
  CK(cudaEventSynchronize(h->emit_ev[pending_slot]));
  emit(pending_t0, pending_count, h->emit_pin[pending_slot], user);
  pending_count = 0;
}

// Samples [t0, t1) of d_stems (8 rows `ld` apart, column 0 = sample col0)
// are final: copy them out as blocks.
void HostSink::put(dmx_handle* h, const float* d_stems, int64_t ld, int64_t t0, int64_t t1,
                   int64_t col0) {
  for (int64_t a = t0; a < t1; a += h->emit_cap) {
    const int64_t count = std::min<int64_t>(h->emit_cap, t1 - a);
    const int slot = next_slot;
    next_slot ^= 1;
    // the slot's previous block was handed over before the block after it was queued
    CK(cudaMemcpy2DAsync(h->emit_pin[slot], (size_t)count * sizeof(float), d_stems + (a - col0),
                         (size_t)ld * sizeof(float), (size_t)count * sizeof(float), 8,
                         cudaMemcpyDeviceToHost, h->copy_stream));
    CK(cudaEventRecord(h->emit_ev[slot], h->copy_stream));
    flush(h);
    pending_t0 = a;
    pending_count = count;
    pending_slot = slot;
  }
}

// Demucs::separate's device driver for one track (api.rs:438-545, 697-785;
// pipeline.rs:380-515; streaming.rs:52-400) over one network or, with `bag`,
// over the bag's lockstep combination; `h` is the network (the bag's lead)
// whose stream, track workspace and OLA weights the driver uses. With `sink`
// (single pass only) the stems are also copied to the host as they finish.
void separate_track_impl(dmx_handle* h, BagPlan* bag, const float* lr_dev, int64_t n,
                         const dmx_separate_opts* opts, float* d_stems, dmx_progress_fn progress,
                         void* user, HostSink* sink) {
  const dmx_separate_opts o = separate_opts(opts);
  CK(cudaSetDevice(h->device));
  const PassGeom pg = pass_geom(h, chunk_samples(o), o.overlap, o.transition_power);
  const int64_t stride = pg.stride;
  const int64_t max_shift = o.shifts > 0 ? (int64_t)(0.5 * 44100.0) : 0;
  const int64_t view_cap = n + max_shift;
  // track-sized scratch, kept on the handle between calls
  const size_t scratch_bytes = (size_t)track_normalize_scratch_doubles() * sizeof(double);
  const size_t need = (size_t)(2 * n + 8 * view_cap + (o.shifts > 1 ? 8 * n : 0)) * sizeof(float) +
                      scratch_bytes + 512;
  if (need > h->track_cap) {
    cudaFree(h->track_ws);
    h->track_ws = nullptr;
    h->track_cap = 0;
    CK(cudaMalloc(&h->track_ws, need));
    h->track_cap = need;
  }
  double* d_stats = reinterpret_cast<double*>(h->track_ws);
  float2* d_norm = reinterpret_cast<float2*>(h->track_ws + scratch_bytes);
  float* d_mix = reinterpret_cast<float*>(h->track_ws + scratch_bytes + 512);
  float* d_acc = d_mix + 2 * n;
  float* d_pass = o.shifts > 1 ? d_acc + 8 * view_cap : nullptr;
  h->launches = 0;
  if (d_pass) CK(cudaMemsetAsync(d_pass, 0, 8 * n * sizeof(float), h->stream));
  h->mark("track.normalize");
  launch_track_normalize(lr_dev, lr_dev + n, n, d_stats, d_mix, d_norm, h->stream);
  h->launches += 2;
  const int passes = std::max(1, o.shifts);
  const float scale = o.shifts > 0 ? 1.0f / (float)o.shifts : 1.0f;
  const std::vector<int64_t> offsets =
      o.shifts > 0 ? shift_offsets(passes, max_shift) : std::vector<int64_t>(1, 0);
  size_t done = 0, total = 0;
  for (int pass = 0; pass < passes; ++pass) {
    const int64_t vlen = o.shifts > 0 ? n + max_shift - offsets[pass] : n;
    total += (size_t)((vlen + stride - 1) / stride);
  }
  int max_batch = h->cfg.max_batch;
  if (bag)
    for (dmx_handle* hk : bag->nets) max_batch = std::min(max_batch, hk->cfg.max_batch);
  const int batch = std::max(1, o.batch > 0 ? std::min(o.batch, max_batch) : max_batch);
  // progress counts every running network's chunks (api.rs:764-776)
  const size_t active = bag ? bag->nets.size() : 1;
  const bool stream_out = sink && (sink->host || sink->emit) && passes == 1;
  if (sink && !h->copy_stream) {
    CK(cudaStreamCreateWithFlags(&h->copy_stream, cudaStreamNonBlocking));
    CK(cudaEventCreateWithFlags(&h->copy_ev, cudaEventDisableTiming));
  }
  for (int pass = 0; pass < passes; ++pass) {
    const int64_t offset = offsets[pass];
    const int64_t vlen = o.shifts > 0 ? n + max_shift - offset : n;
    const int64_t chunks = (vlen + stride - 1) / stride;
    const int mode = o.shifts == 0 ? 0 : (o.shifts == 1 ? 1 : 2);
    const int64_t trim = o.shifts > 0 ? max_shift - offset : 0;
    int64_t t_done = 0;  // output samples already finished (and copied) by the sink
    CK(cudaMemsetAsync(d_acc, 0, 8 * vlen * sizeof(float), h->stream));
    for (int64_t c0 = 0; c0 < chunks; c0 += batch) {
      const int64_t c1 = std::min<int64_t>(chunks, c0 + batch);
      shard_chunks(h, bag, d_mix, n, offset, max_shift, pg, c0, c1, batch, d_acc, 0, vlen);
      if (stream_out) {
        // view samples below chunk c1's start get no further contribution
        const int64_t t_hi = c1 == chunks ? n : std::min<int64_t>(n, std::max<int64_t>(0, c1 * stride - trim));
        if (t_hi > t_done) {
          h->mark("track.finish");
          ++h->launches;
          launch_ola_finish(d_acc, n, offset, max_shift, pg.chunk, stride, pg.weight, d_norm,
                            scale, mode, d_pass, d_stems, h->stream, t_done, t_hi);
          CK(cudaEventRecord(h->copy_ev, h->stream));
          CK(cudaStreamWaitEvent(h->copy_stream, h->copy_ev, 0));
          if (sink->host)
            CK(cudaMemcpy2DAsync(sink->host + t_done, (size_t)n * sizeof(float), d_stems + t_done,
                                 (size_t)n * sizeof(float), (size_t)(t_hi - t_done) * sizeof(float),
                                 8, cudaMemcpyDeviceToHost, h->copy_stream));
          else
            sink->put(h, d_stems, n, t_done, t_hi);
          t_done = t_hi;
        }
      }
      done += (size_t)(c1 - c0);
      if (progress) {
        CK(cudaStreamSynchronize(h->stream));
        progress(done * active, total * active, user);
      }
    }
    if (stream_out) continue;
    h->mark("track.finish");
    ++h->launches;
    launch_ola_finish(d_acc, n, offset, max_shift, pg.chunk, stride, pg.weight, d_norm, scale,
                      mode, d_pass, d_stems, h->stream);
  }
  if (o.shifts > 1) ++h->launches;
  if (o.shifts > 1)
    launch_ola_finish(d_acc, n, 0, max_shift, pg.chunk, stride, pg.weight, d_norm, scale, 3,
                      d_pass, d_stems, h->stream);
  if (sink && sink->emit) {
    if (!stream_out) {  // several shift passes: every sample is final only now
      CK(cudaEventRecord(h->copy_ev, h->stream));
      CK(cudaStreamWaitEvent(h->copy_stream, h->copy_ev, 0));
      sink->put(h, d_stems, n, 0, n);
    }
    sink->flush(h);
  }
  h->mark("end");
  CK(cudaGetLastError());
}

// Host arrays in, host stems out, through the handle's device staging.
void separate_track_host(dmx_handle* h, BagPlan* bag, const float* left, const float* right,
                         int64_t n, const dmx_separate_opts* opts, float* stems_out,
                         dmx_progress_fn progress, void* user) {
  CK(cudaSetDevice(h->device));
  // host-track staging kept on the handle between calls (grown on demand)
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
  // pinned stems are copied while the forwards run; pageable ones once at the end (a copy
  // to pageable memory would block this thread before the next forward is enqueued)
  cudaPointerAttributes attr{};
  const bool pinned = cudaPointerGetAttributes(&attr, stems_out) == cudaSuccess &&
                      attr.type == cudaMemoryTypeHost;
  cudaGetLastError();  // a pageable pointer may leave an error behind on some drivers
  const int shifts = opts ? opts->shifts : 1;
  HostSink sink;
  sink.host = stems_out;
  const bool streamed = pinned && shifts <= 1;
  try {
    separate_track_impl(h, bag, d_lr, n, opts, d_stems, progress, user, streamed ? &sink : nullptr);
  } catch (...) {
    if (h->copy_stream) cudaStreamSynchronize(h->copy_stream);  // no copy outlives the call
    throw;
  }
  if (streamed) {
    CK(cudaStreamSynchronize(h->copy_stream));
  } else {
    CK(cudaMemcpyAsync(stems_out, d_stems, 8 * n * sizeof(float), cudaMemcpyDeviceToHost,
                       h->stream));
  }
  CK(cudaStreamSynchronize(h->stream));
  check_device_flag(h);
  if (bag)
    for (dmx_handle* hk : bag->nets)
      if (hk != h) check_device_flag(hk);
  finish_stage_times(h);
}

// Many tracks through one network with their chunks pooled into full
// forwards (the many-track throughput configuration). The work units are (track,
// shift pass, chunk) in that order; consecutive units fill each forward of
// `batch` chunks regardless of which track or pass they belong to. Every
// track is driven exactly as separate_track_impl drives it — its own global
// normalisation, the same ShiftRng offsets (a fresh ShiftRng per track, as
// each Demucs::separate call seeds its own: pipeline.rs:416-418), its own
// overlap-add accumulator and finish — so each track's stems equal
// dmx_separate_track's on that track. A track holds one workspace slot
// (normalised mix, moments, pass sum, accumulator) from the forward that
// takes its first chunk to the one that takes its last.
void separate_batch_impl(dmx_handle* h, const float* const* lr_dev, const int64_t* lengths,
                         int n_tracks, const dmx_separate_opts* opts, float* const* stems_dev,
                         dmx_progress_fn progress, void* user) {
  if (!lr_dev || !lengths || !stems_dev || n_tracks < 1)
    throw Error(DMX_ERR_INVALID, "dmx_separate_batch: bad argument");
  const dmx_separate_opts o = separate_opts(opts);
  CK(cudaSetDevice(h->device));
  const PassGeom pg = pass_geom(h, chunk_samples(o), o.overlap, o.transition_power);
  const int64_t stride = pg.stride;
  const int64_t max_shift = o.shifts > 0 ? (int64_t)(0.5 * 44100.0) : 0;
  const int passes = std::max(1, o.shifts);
  const float scale = o.shifts > 0 ? 1.0f / (float)o.shifts : 1.0f;
  // the same ShiftRng offsets for every track (a fresh generator per track)
  const std::vector<int64_t> offsets =
      o.shifts > 0 ? shift_offsets(passes, max_shift) : std::vector<int64_t>(1, 0);
  auto view_len = [&](int64_t n, int pass) {
    return o.shifts > 0 ? n + max_shift - offsets[pass] : n;
  };
  std::vector<std::vector<int64_t>> chunks(n_tracks);  // per track, per pass
  std::vector<int64_t> first(n_tracks + 1, 0);         // first unit of each track
  int64_t n_max = 0;
  for (int i = 0; i < n_tracks; ++i) {
    if (lengths[i] <= 0 || !lr_dev[i] || !stems_dev[i])
      throw Error(DMX_ERR_INVALID, "track " + std::to_string(i) + " is empty or has no buffer");
    n_max = std::max(n_max, lengths[i]);
    int64_t units = 0;
    for (int pass = 0; pass < passes; ++pass) {
      chunks[i].push_back((view_len(lengths[i], pass) + stride - 1) / stride);
      units += chunks[i].back();
    }
    first[i + 1] = first[i] + units;
  }
  const int64_t total = first[n_tracks];
  const int batch = std::max(1, o.batch > 0 ? std::min(o.batch, h->cfg.max_batch) : h->cfg.max_batch);
  // slots: the most tracks any one forward touches
  int slots = 1;
  for (int64_t u0 = 0, i = 0; u0 < total; u0 += batch) {
    const int64_t u1 = std::min<int64_t>(total, u0 + batch);
    while (first[i + 1] <= u0) ++i;
    int64_t j = i;
    while (j + 1 < n_tracks && first[j + 1] < u1) ++j;
    slots = std::max(slots, (int)(j - i + 1));
  }
  const size_t scratch_bytes = (size_t)track_normalize_scratch_doubles() * sizeof(double);
  const size_t slot_floats = (size_t)(2 * n_max + (o.shifts > 1 ? 8 * n_max : 0) + 8 * (n_max + max_shift));
  const size_t slot_bytes = (scratch_bytes + 512 + slot_floats * sizeof(float) + 255) / 256 * 256;
  if ((size_t)slots * slot_bytes > h->batch_cap) {
    cudaFree(h->batch_ws);
    h->batch_ws = nullptr;
    h->batch_cap = 0;
    CK(cudaMalloc(&h->batch_ws, (size_t)slots * slot_bytes));
    h->batch_cap = (size_t)slots * slot_bytes;
  }
  struct Slot {
    double* stats;
    float2* norm;
    float* mix;
    float* pass;
    float* acc;
  };
  auto slot_at = [&](int k) {
    char* base = h->batch_ws + (size_t)k * slot_bytes;
    Slot sl;
    sl.stats = reinterpret_cast<double*>(base);
    sl.norm = reinterpret_cast<float2*>(base + scratch_bytes);
    sl.mix = reinterpret_cast<float*>(base + scratch_bytes + 512);
    sl.pass = o.shifts > 1 ? sl.mix + 2 * n_max : nullptr;
    sl.acc = sl.mix + 2 * n_max + (o.shifts > 1 ? 8 * n_max : 0);
    return sl;
  };
  std::vector<int> free_slots;
  for (int k = slots - 1; k >= 0; --k) free_slots.push_back(k);
  std::vector<int> slot_of(n_tracks, -1);
  ensure_io(h, batch);
  h->launches = 0;
  const float* w_ola = pg.weight;
  const int seg = kSegment;
  struct Run {
    int track, pass;
    int64_t c0, count, at;  // chunks [c0, c0 + count) of the pass, at forward row `at`
  };
  int ti = 0, tp = 0;
  int64_t tc = 0;  // cursor: next unit is chunk tc of pass tp of track ti
  for (int64_t u0 = 0; u0 < total; u0 += batch) {
    const int G = (int)std::min<int64_t>(batch, total - u0);
    std::vector<Run> runs;
    for (int64_t left = G, at = 0; left > 0;) {
      const int64_t take = std::min<int64_t>(left, chunks[ti][tp] - tc);
      runs.push_back({ti, tp, tc, take, at});
      at += take;
      left -= take;
      tc += take;
      if (tc == chunks[ti][tp]) {
        tc = 0;
        if (++tp == passes) {
          tp = 0;
          ++ti;
        }
      }
    }
    // tracks that start here: a slot, the global normalisation, a cleared pass sum
    for (const Run& r : runs) {
      if (r.pass != 0 || r.c0 != 0) continue;
      const int i = r.track;
      slot_of[i] = free_slots.back();
      free_slots.pop_back();
      const Slot sl = slot_at(slot_of[i]);
      h->mark("track.normalize");
      launch_track_normalize(lr_dev[i], lr_dev[i] + lengths[i], lengths[i], sl.stats, sl.mix,
                             sl.norm, h->stream);
      h->launches += 2;
      if (sl.pass) CK(cudaMemsetAsync(sl.pass, 0, 8 * lengths[i] * sizeof(float), h->stream));
    }
    for (const Run& r : runs) {
      const Slot sl = slot_at(slot_of[r.track]);
      h->mark("track.gather");
      launch_gather_chunks(sl.mix, lengths[r.track], offsets[r.pass], max_shift, pg.chunk, stride,
                           r.c0, (int)r.count, h->io_in + r.at * 2 * seg, h->stream, seg);
      ++h->launches;
    }
    run_forward(h, h->io_in, G, h->io_out);
    for (const Run& r : runs) {
      const int i = r.track;
      const Slot sl = slot_at(slot_of[i]);
      const int64_t n = lengths[i];
      const int64_t vlen = view_len(n, r.pass);
      if (r.c0 == 0) CK(cudaMemsetAsync(sl.acc, 0, 8 * vlen * sizeof(float), h->stream));
      h->mark("track.ola");
      launch_ola_accumulate(h->io_out + r.at * 8 * seg, n, offsets[r.pass], max_shift, pg.chunk,
                            stride, r.c0, (int)r.count, w_ola, sl.acc, 0, vlen, h->stream, seg);
      ++h->launches;
      if (r.c0 + r.count < chunks[i][r.pass]) continue;
      const int mode = o.shifts == 0 ? 0 : (o.shifts == 1 ? 1 : 2);
      h->mark("track.finish");
      launch_ola_finish(sl.acc, n, offsets[r.pass], max_shift, pg.chunk, stride, w_ola, sl.norm,
                        scale, mode, sl.pass, stems_dev[i], h->stream);
      ++h->launches;
      if (r.pass + 1 < passes) continue;
      if (o.shifts > 1) {
        launch_ola_finish(sl.acc, n, 0, max_shift, pg.chunk, stride, w_ola, sl.norm, scale, 3,
                          sl.pass, stems_dev[i], h->stream);
        ++h->launches;
      }
      free_slots.push_back(slot_of[i]);
      slot_of[i] = -1;
    }
    CK(cudaGetLastError());
    if (progress) {
      CK(cudaStreamSynchronize(h->stream));
      progress((size_t)(u0 + G), (size_t)total, user);
    }
  }
  h->mark("end");
}

// dmx_separate_track over several handles from one host thread (see
// include/dmx.h): contiguous chunk ranges, one per handle; every handle
// overlap-adds its own chunks, pulls its left neighbour's overlap tail by a
// peer copy and adds it, finishes the samples it owns and copies them to the
// host. With stride > chunk / 2 every sample gets at most two contributions
// and a rank's tail ends inside its right neighbour's own span, so the sums
// are those of one GPU.
void separate_track_multi_impl(const std::vector<dmx_handle*>& H, const float* left,
                               const float* right, int64_t n, const dmx_separate_opts* opts,
                               float* stems_out) {
  const int n_handles = (int)H.size();
  const dmx_separate_opts o = separate_opts(opts);
  if (o.shifts > 1)
    throw Error(DMX_ERR_INVALID,
                "dmx_separate_track_multi runs one pass (shifts 0 or 1); for more shift passes "
                "use dmx_separate_track or dmx_separate_batch per GPU");
  std::vector<PassGeom> pgs;
  for (dmx_handle* h : H) {
    CK(cudaSetDevice(h->device));
    pgs.push_back(pass_geom(h, chunk_samples(o), o.overlap, o.transition_power));
  }
  const int chunk_len = pgs[0].chunk;
  const int64_t stride = pgs[0].stride;
  if (2 * stride <= chunk_len)
    throw Error(DMX_ERR_INVALID,
                "dmx_separate_track_multi needs overlap < 0.5 (a stride longer than half a "
                "segment, so a rank's overlap tail ends inside its neighbour's own span); use "
                "dmx_separate_track for larger overlaps");
  // the single pass's view (ShiftRng's first draw, pipeline.rs:136-151, 416-418)
  const int64_t max_shift = o.shifts > 0 ? (int64_t)(0.5 * 44100.0) : 0;
  const int64_t offset = o.shifts > 0 ? shift_offsets(1, max_shift)[0] : 0;
  const int64_t vlen = o.shifts > 0 ? n + max_shift - offset : n;
  const int64_t trim = o.shifts > 0 ? max_shift - offset : 0;
  const int64_t chunks = (vlen + stride - 1) / stride;
  const int mode = o.shifts == 0 ? 0 : 1;
  // contiguous chunk ranges, the first `extra` ranks one chunk more
  struct Rank {
    int64_t lo, hi, own_hi, send_lo, send_hi, t_lo, t_hi;
    double* stats;
    float2* norm;
    float *lr, *mix, *acc, *stems;
  };
  std::vector<Rank> R(n_handles);
  const int64_t base = chunks / n_handles, extra = chunks % n_handles;
  int64_t c = 0;
  for (int k = 0; k < n_handles; ++k) {
    Rank& r = R[k];
    r.lo = c;
    r.hi = c + base + (k < extra ? 1 : 0);
    c = r.hi;
    const bool any = r.hi > r.lo;
    const int64_t span_hi = any ? std::min(vlen, (r.hi - 1) * stride + chunk_len) : 0;
    r.own_hi = !any ? 0 : (r.hi == chunks ? vlen : r.hi * stride);
    r.send_lo = r.own_hi;
    r.send_hi = any && r.hi < chunks ? span_hi : r.own_hi;
    const int64_t own_lo = r.lo * stride;
    r.t_lo = any ? std::max<int64_t>(0, own_lo - trim) : 0;
    r.t_hi = any ? std::max(r.t_lo, std::min(n, r.own_hi - trim)) : 0;
  }
  // per rank: the whole track, normalised (deterministic, so every rank agrees), and this
  // rank's chunks overlap-added into a view-sized accumulator
  const size_t scratch_bytes = (size_t)track_normalize_scratch_doubles() * sizeof(double);
  for (int k = 0; k < n_handles; ++k) {
    dmx_handle* h = H[k];
    Rank& r = R[k];
    CK(cudaSetDevice(h->device));
    grow(h->track_ws, h->track_cap,
         (size_t)(2 * n + 8 * (n + max_shift)) * sizeof(float) + scratch_bytes + 512);
    grow(h->host_io, h->host_io_cap, (size_t)10 * n * sizeof(float));
    if (!h->shard_done) CK(cudaEventCreateWithFlags(&h->shard_done, cudaEventDisableTiming));
    r.stats = reinterpret_cast<double*>(h->track_ws);
    r.norm = reinterpret_cast<float2*>(h->track_ws + scratch_bytes);
    r.mix = reinterpret_cast<float*>(h->track_ws + scratch_bytes + 512);
    r.acc = r.mix + 2 * n;
    r.lr = h->host_io;
    r.stems = h->host_io + 2 * n;
    h->launches = 0;
    CK(cudaMemcpyAsync(r.lr, left, n * sizeof(float), cudaMemcpyHostToDevice, h->stream));
    CK(cudaMemcpyAsync(r.lr + n, right, n * sizeof(float), cudaMemcpyHostToDevice, h->stream));
    h->mark("track.normalize");
    launch_track_normalize(r.lr, r.lr + n, n, r.stats, r.mix, r.norm, h->stream);
    h->launches += 2;
    CK(cudaMemsetAsync(r.acc, 0, 8 * vlen * sizeof(float), h->stream));
    if (r.hi > r.lo) {
      const int cap = std::max(1, o.batch > 0 ? std::min(o.batch, h->cfg.max_batch) : h->cfg.max_batch);
      shard_chunks(h, nullptr, r.mix, n, offset, max_shift, pgs[k], r.lo, r.hi, cap, r.acc, 0, vlen);
    }
    CK(cudaEventRecord(h->shard_done, h->stream));
  }
  // boundary: rank k + 1 copies rank k's tail (after rank k's chunks) and adds it
  for (int k = 0; k + 1 < n_handles; ++k) {
    const Rank& a = R[k];
    Rank& b = R[k + 1];
    const int64_t w = a.send_hi - a.send_lo;
    if (w <= 0 || b.hi <= b.lo) continue;
    dmx_handle* hb = H[k + 1];
    CK(cudaSetDevice(hb->device));
    grow(hb->tail_buf, hb->tail_cap, (size_t)8 * w * sizeof(float));
    CK(cudaStreamWaitEvent(hb->stream, H[k]->shard_done, 0));
    for (int row = 0; row < 8; ++row)
      CK(cudaMemcpyPeerAsync(hb->tail_buf + row * w, hb->device, a.acc + row * vlen + a.send_lo,
                             H[k]->device, (size_t)w * sizeof(float), hb->stream));
    hb->mark("track.merge");
    launch_tail_add(b.acc + a.send_lo, vlen, hb->tail_buf, w, 8, hb->stream);
    ++hb->launches;
    CK(cudaGetLastError());
  }
  // each rank finishes the samples it owns and copies them straight to the host stems
  for (int k = 0; k < n_handles; ++k) {
    dmx_handle* h = H[k];
    const Rank& r = R[k];
    if (r.t_hi <= r.t_lo) continue;
    CK(cudaSetDevice(h->device));
    h->mark("track.finish");
    launch_ola_finish(r.acc, n, offset, max_shift, chunk_len, stride, pgs[k].weight, r.norm, 1.0f,
                      mode, nullptr, r.stems, h->stream, r.t_lo, r.t_hi);
    ++h->launches;
    CK(cudaMemcpy2DAsync(stems_out + r.t_lo, (size_t)n * sizeof(float), r.stems + r.t_lo,
                         (size_t)n * sizeof(float), (size_t)(r.t_hi - r.t_lo) * sizeof(float), 8,
                         cudaMemcpyDeviceToHost, h->stream));
    h->mark("end");
  }
  for (dmx_handle* h : H) {
    CK(cudaSetDevice(h->device));
    CK(cudaStreamSynchronize(h->stream));
    check_device_flag(h);
    finish_stage_times(h);
  }
}

}  // namespace dmx
