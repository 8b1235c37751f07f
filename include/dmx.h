/*
 * dmx.h — C ABI of the B200 (sm_100a) HTDemucs v4 inference backend.
 *
 * This is the drop-in boundary a `Backend::Cuda` in the reference's library
 * binds to. Each entry point names the reference interface it replaces
 * (paths relative to the reference project, crates/demucs-core/src/...).
 *
 * Conventions: every function returns a dmx_status (0 = OK). On failure
 * dmx_last_error() returns a thread-local message. Host pointers are plain
 * float arrays, row-major; no CUDA or framework types cross the boundary.
 * A handle is used by one host thread at a time (the reference runner is
 * !Sync: gpu/htdemucs.rs:2344-2351).
 */
#ifndef DMX_H
#define DMX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int dmx_status;
enum {
  DMX_OK = 0,
  DMX_ERR_INVALID = 1,   /* bad argument, shape or configuration */
  DMX_ERR_WEIGHTS = 2,   /* weight blob missing a tensor or with a wrong shape */
  DMX_ERR_CUDA = 3,      /* a CUDA call failed */
  DMX_ERR_TIMEOUT = 4,   /* a bounded wait gave up */
  DMX_ERR_NOMEM = 5      /* device memory exhausted */
};

/* Arithmetic of the contractions (convolutions, linears).
 * FP32: SIMT fp32 FMA everywhere (the max-abs 1e-4 parity build).
 * TF32: tcgen05 kind::tf32 with both operands rounded to nearest tf32, fp32
 *       accumulate (the SNR >= 60 dB build).
 * TF32X3: tcgen05 kind::tf32 on split operands, hi*hi + hi*lo + lo*hi
 *       (fp32-class accuracy on the tensor cores).
 * BF16: the TF32 build with the transformer's linears (q/k/v, output
 *       projection, both FFN layers) on tcgen05 kind::f16 with bf16 operands
 *       (bf16 activations stored by their producers — LayerNorm, the FFN's
 *       GELU, attention — and bf16 weight copies) and fp32 accumulate;
 *       the DConv branches' contractions single-pass tf32 (TF32 and TF32X3
 *       split them); attention on kind::f16 with bf16 q, k, V^T and P;
 *       convolutions as in TF32. */
typedef enum { DMX_FP32 = 0, DMX_TF32 = 1, DMX_BF16 = 2, DMX_TF32X3 = 3 } dmx_precision;

typedef struct {
  int sources;         /* 4 (config.rs:46-49) */
  int audio_channels;  /* 2 */
  int samplerate;      /* 44100 */
  int segment_samples; /* 343980 = int(39/5 * 44100) (config.rs:222-224) */
  int precision;       /* dmx_precision */
  int max_batch;       /* segments per forward the workspace is sized for */
} dmx_config;

typedef struct dmx_handle dmx_handle;
typedef struct dmx_pending dmx_pending;

/* Fills the reference defaults (HtdemucsConfig::default, config.rs:43-71). */
void dmx_default_config(dmx_config* cfg);

/* Demucs::load / GpuHtdemucsRunner::with_selector + GpuWeights::load
 * (api.rs:394-420, gpu/htdemucs.rs:536-660, 2377-2388; weights.rs:28-80):
 * parse a checkpoint blob holding the PyTorch-named tensors (weights.rs:
 * 211-578), repack them and upload them once to `device`. The blob is either
 * a safetensors file — F32, or F16 (the published checkpoints), BF16, F64 and
 * integer types upcast to f32 as safetensors.rs:110-135 does — or a torch.save
 * zip (`.th` / `.pth`, recognised by its first bytes; ckpt/mod.rs,
 * ckpt/pickle.rs) whose state dict is the top level or sits under `state`,
 * `state_dict` or `model_state_dict`. The model kwargs (safetensors
 * __metadata__["kwargs"] JSON, or the .th package's pickled kwargs dict;
 * config.rs:150-215) must describe the htdemucs default architecture these
 * kernels implement; a checkpoint of another shape is DMX_ERR_INVALID naming
 * the field. The blob is validated (DMX_ERR_WEIGHTS) before any CUDA call. */
dmx_status dmx_create(const dmx_config* cfg, const void* safetensors_blob, size_t blob_len,
                      int device, dmx_handle** out);
void dmx_destroy(dmx_handle* h);
const char* dmx_last_error(void);

/* SegmentForward::start (demucs/pipeline.rs:178-190; DeviceForward::start,
 * gpu/htdemucs.rs:2824-2847): queue one forward of `mix`, a host
 * (n_segments, 2, segment_samples) array of already-normalised padded chunks,
 * and return with the work in flight. `mix` is copied into the pending
 * forward's own staging before this returns, so the caller may free or reuse
 * it at once (the reference drops its batch before collect, pipeline.rs:
 * 596-623). Up to two forwards may be in flight on one handle, each with its
 * own staging (PendingStems, gpu/htdemucs.rs:2744-2782), so the reference's
 * queue-one-ahead loop — start(group n), then collect(group n - 1) — works
 * as is; a third start before a collect fails with DMX_ERR_INVALID. The
 * forwards run in start order on the handle's stream. */
dmx_status dmx_forward_start(dmx_handle* h, const float* mix, int64_t n_segments,
                             dmx_pending** out);
/* SegmentForward::collect: wait (bounded) for that forward and write its
 * (n_segments, 4, 2, segment_samples) stems in normalised units to host
 * `out`. Each pending forward is collected once; pending forwards may be
 * collected in any order. */
dmx_status dmx_forward_collect(dmx_pending* p, float* out);

/* The same forward on device buffers of the handle's GPU (no host copies):
 * mix_dev (n, 2, segment_samples) -> out_dev (n, 4, 2, segment_samples),
 * enqueued on `stream` (a cudaStream_t, NULL = the handle's stream). */
dmx_status dmx_forward_device(dmx_handle* h, const float* mix_dev, int64_t n_segments,
                              float* out_dev, void* stream);

typedef struct {
  int shifts;              /* SeparateOptions::shifts (pipeline.rs:17-38) */
  double overlap;          /* 0.25; in [0, 1) */
  double transition_power; /* 1.0; the triangular window's exponent (pipeline.rs:117-131) */
  int batch;               /* chunks per forward (DEMUCS_BATCH); 0 = max_batch */
  double segment;          /* SeparateOptions::segment, seconds; 0 = the model's 7.8 s.
                              Chunks of int(44100 * segment) samples (at most the model's
                              343980) are zero padded to the model's length for the forward
                              and trimmed back, as Htdemucs::forward does (host.rs:210-229) */
} dmx_separate_opts;

typedef void (*dmx_progress_fn)(size_t done, size_t total, void* user);

/* Demucs::separate_with_options for one stereo track (api.rs:438-545 with the
 * driver of pipeline.rs:380-515 and streaming.rs:52-400): global
 * normalisation, shift passes (ShiftRng seed 0x5eed1234), chunking, batched
 * forwards, triangular overlap-add and denormalisation, all on the device.
 * `stems_out` is (4, 2, n) host memory. */
dmx_status dmx_separate_track(dmx_handle* h, const float* left, const float* right, int64_t n,
                              const dmx_separate_opts* opts, float* stems_out,
                              dmx_progress_fn progress, void* user);

/* A block of finished stems for dmx_separate_track_emit: output samples
 * [t0, t0 + count) of the track, `block` is (8, count) row-major — rows
 * drums L, drums R, bass L, bass R, other L, other R, vocals L, vocals R —
 * denormalised, valid only during the call. */
typedef void (*dmx_frames_fn)(int64_t t0, int64_t count, const float* block, void* user);

/* Demucs::separate_streaming (api.rs:600-650 over separate_forwarding_emit,
 * pipeline.rs:380-515, and the OLA ring's in-order emission, streaming.rs:
 * 96-261): the dmx_separate_track driver, but the stems are handed to
 * `on_frames` in ascending blocks as soon as no later chunk can change them
 * (after every forward of opts->batch chunks for shifts 0 or 1; after the
 * last pass for shifts > 1), so host memory holds two blocks of at most
 * opts->batch strides each instead of the whole (4, 2, n) result. Blocks are
 * copied on a side stream and handed over while the next forward runs.
 * `progress` and `on_frames` receive the same `user`. */
dmx_status dmx_separate_track_emit(dmx_handle* h, const float* left, const float* right, int64_t n,
                                   const dmx_separate_opts* opts, dmx_frames_fn on_frames,
                                   dmx_progress_fn progress, void* user);

/* Reads samples [t0, t0 + count) of the track's two channels into `left` and
 * `right` (pinned host buffers the library owns, valid during the call) and
 * returns 0, or nonzero to stop the separation with DMX_ERR_INVALID
 * (MixSamples::at over a WindowedMix, mix.rs:18-60, 265-360). */
typedef int (*dmx_read_fn)(int64_t t0, int64_t count, float* left, float* right, void* user);

/* Demucs::separate_streaming over a windowed source (the reference CLI's
 * separate: scan_norm_file, mix.rs:61-120, then separate_streaming_normalized_mix
 * over WindowedMix, api.rs:600-650, mix.rs:265-360, with the OLA ring of
 * streaming.rs:96-261): the track of `n` samples is never held whole. A first
 * pass reads it through `read` in windows for the global moments; the split
 * passes then read, for each forward of opts->batch chunks, only the samples
 * those chunks cover, and overlap-add in a device window that slides with
 * the chunks. Device memory is O(batch x segment) — about 0.3 GB at batch 16,
 * 50 MB at batch 1 — and independent of n; finished stems reach `on_frames`
 * in ascending blocks as dmx_separate_track_emit hands them over. With
 * shifts > 1 the passes are summed in host memory (8 n floats, as the
 * reference's O(T) pass sum, pipeline.rs:451-513) and emitted after the last
 * pass. The stems equal dmx_separate_track's bit for bit. `read`, `progress`
 * and `on_frames` receive the same `user`. */
dmx_status dmx_separate_track_windowed(dmx_handle* h, dmx_read_fn read, int64_t n,
                                       const dmx_separate_opts* opts, dmx_frames_fn on_frames,
                                       dmx_progress_fn progress, void* user);

/* dmx_separate_track over several GPUs from one host thread (the whole-track
 * multi-GPU entry of the drop-in plan; the reference runs one device:
 * api.rs:438-545, streaming.rs:296-400). hs[k] holds the same network on
 * rank k's GPU (handles may share a GPU). The single pass's chunks are split
 * into contiguous ranges, one per rank; every rank normalises the whole track
 * (a deterministic reduction, so all agree), overlap-adds its chunks, receives
 * its left neighbour's overlap tail by a peer copy and adds it (at most two
 * contributions per sample, so the sums equal one GPU's), finishes the
 * samples it owns and copies them straight into `stems_out` (4, 2, n), all
 * ranks at once. shifts must be 0 or 1 (one pass); for more shift passes use
 * dmx_separate_track or dmx_separate_batch per GPU. The overlap must be below
 * 0.5 (stride > segment / 2): a larger one would let a rank's tail reach past
 * its neighbour's own span, and is rejected with DMX_ERR_INVALID. */
dmx_status dmx_separate_track_multi(dmx_handle* const* hs, int n_handles, const float* left,
                                    const float* right, int64_t n, const dmx_separate_opts* opts,
                                    float* stems_out);

/* dmx_separate_track on device buffers of the handle's GPU: lr_dev holds the
 * raw (2, n) stereo track, stems_dev receives (4, 2, n). Enqueued on the
 * handle's stream; returns without waiting unless `progress` is set. */
dmx_status dmx_separate_track_device(dmx_handle* h, const float* lr_dev, int64_t n,
                                     const dmx_separate_opts* opts, float* stems_dev,
                                     dmx_progress_fn progress, void* user);

/* Many tracks in one call, with their chunks pooled (the `dmx_separate_batch`
 * of the drop-in plan; in the reference each track is one
 * Demucs::separate_with_options call, api.rs:438-545). The work units —
 * (track, shift pass, chunk), in that order — fill every forward of
 * opts->batch chunks (0 = max_batch) regardless of which track they belong to,
 * so short tracks and the tails of shift passes do not leave forwards
 * half-empty. Each track is otherwise driven exactly as dmx_separate_track
 * drives it (its own global normalisation, the ShiftRng offsets of a fresh
 * seed 0x5eed1234, its own overlap-add), so its stems match that call's.
 * left[i] / right[i] hold lengths[i] samples; stems_out[i] receives
 * (4, 2, lengths[i]). All tracks' inputs and stems stay in device memory for
 * the call (10 floats per sample), plus one workspace slot (about 18 floats
 * per sample of the longest track) per track that a single forward touches.
 * Progress counts units. */
dmx_status dmx_separate_batch(dmx_handle* h, const float* const* left, const float* const* right,
                              const int64_t* lengths, int n_tracks, const dmx_separate_opts* opts,
                              float* const* stems_out, dmx_progress_fn progress, void* user);

/* dmx_separate_batch on device buffers of the handle's GPU: lr_dev[i] is the
 * raw (2, lengths[i]) track i, stems_dev[i] receives (4, 2, lengths[i]).
 * Enqueued on the handle's stream; returns without waiting unless `progress`
 * is set. */
dmx_status dmx_separate_batch_device(dmx_handle* h, const float* const* lr_dev,
                                     const int64_t* lengths, int n_tracks,
                                     const dmx_separate_opts* opts, float* const* stems_dev,
                                     dmx_progress_fn progress, void* user);

/* Global normalisation of a raw stereo track on the device (Separator's
 * normalisation: streaming.rs:52-85 scan_norm + apply_norm_inplace): from
 * lr_dev (2, n) writes (x - mean) / std into mix_norm_dev (2, n) and
 * {mean, std} into mean_std_dev (2 floats, 8-byte aligned); mean and the
 * unbiased std of the channel-mean signal are reduced in f64 in a fixed
 * order, so every rank of a sharded run derives the same constants.
 * Enqueued on the handle's stream. */
dmx_status dmx_normalize_track_device(dmx_handle* h, const float* lr_dev, int64_t n,
                                      float* mix_norm_dev, float* mean_std_dev);

/* Allocation-free track normalisation. No counterpart in the reference: it
 * exists for callers that cannot allocate device memory when they need it —
 * real-time audio hosts whose processing callback must not block on the
 * driver's allocator, and applications that reserve their whole device budget
 * up front — and so cannot create a dmx_handle either. It computes what
 * dmx_normalize_track_device computes on the current device's buffers (lr_dev
 * (2, n) -> mix_norm_dev (2, n), mean_std_dev {mean, std}), equal to it up to
 * the rounding of the f64 reduction (its per-block partials group the samples
 * differently), enqueued on `stream` (a cudaStream_t, NULL = legacy default
 * stream), with no cudaMalloc/cudaFree: its scratch is a 128 KiB file-scope
 * device array (partials of one block per 65,536 samples), so n is limited to
 * 536,870,912 samples per channel and larger tracks are rejected with
 * DMX_ERR_INVALID. Every call resolves that array's device address
 * (cudaGetSymbolAddress) with the caller's device current, so a device reset
 * leaves nothing stale; the first call on a device may load the library's
 * module there and should come before any stream capture. All calls on a
 * device share the array: calls that overlap on the GPU (different streams,
 * no ordering between them) race and must be serialised by the caller. */
dmx_status dmx_normalize_track_noalloc(const float* lr_dev, int64_t n, float* mix_norm_dev,
                                       float* mean_std_dev, void* stream);

/* Bags of networks (htdemucs_ft). A bag is `n_nets` (1..8) loaded networks and
 * a weight matrix `weights` (n_nets x 4, one row per network, sources in the
 * config's order drums, bass, other, vocals; htdemucs_ft ships the identity),
 * plus `requested`, 4 flags for the stems the caller wants (NULL = all; the
 * reference's StemSelection, api.rs:895-906). A network runs only when it
 * carries a nonzero weight on a requested stem (api.rs:907-916); a requested
 * stem whose weights sum to zero is rejected with DMX_ERR_INVALID ("no network
 * covers stem", api.rs:954-960). Stems that are not requested come out as the
 * zero signal (the track mean after denormalisation).
 *
 * The combination step of BagCombineForward::start (api.rs:326-361) on device
 * buffers of the current device: for each stem s, combined = (sum over the
 * networks k, in bag order, of outs[k][s] * w[k][s]) / (sum of those w), with
 * the reference's f32 roundings (product, then sum, then quotient). outs_dev
 * holds n_nets device pointers, each (n_segments, 4, 2, samples) — entries
 * of networks that carry no requested weight may be NULL — and combined_dev
 * is the same shape. Enqueued on `stream` (a cudaStream_t, NULL = legacy
 * default stream); allocates nothing. Used per chunk batch by the lockstep
 * driver below, and on rank 0 to combine whole-track stems gathered from
 * one network per GPU. */
dmx_status dmx_bag_combine_device(const float* const* outs_dev, int n_nets, const float* weights,
                                  const int* requested, int64_t n_segments, int64_t samples,
                                  float* combined_dev, void* stream);

/* BagCombineForward as a SegmentForward (api.rs:319-371) on device buffers:
 * every running network forwards mix_dev (n, 2, segment_samples), one after
 * another on its own stream, and the combination is written to out_dev
 * (n, 4, 2, segment_samples) on the stream of the first running network
 * (the lead). All running networks must be handles on one device. */
dmx_status dmx_bag_forward_device(dmx_handle* const* nets, int n_nets, const float* weights,
                                  const int* requested, const float* mix_dev, int64_t n,
                                  float* out_dev);

/* Demucs::separate_with_options for an htdemucs_ft bag (api.rs:736-785:
 * run_mix -> separate_streaming_normalized_mix -> separate_forwarding_emit
 * over BagCombineForward): the dmx_separate_track driver with each chunk
 * batch forwarded through every running network and combined before the
 * overlap-add. The lead network's handle supplies the stream and the track
 * staging. Progress counts chunks times running networks (api.rs:764-776). */
dmx_status dmx_separate_track_bag(dmx_handle* const* nets, int n_nets, const float* weights,
                                  const int* requested, const float* left, const float* right,
                                  int64_t n, const dmx_separate_opts* opts, float* stems_out,
                                  dmx_progress_fn progress, void* user);

/* dmx_separate_track_bag on device buffers of the bag's device: lr_dev (2, n)
 * -> stems_dev (4, 2, n), enqueued on the lead's stream. */
dmx_status dmx_separate_track_bag_device(dmx_handle* const* nets, int n_nets, const float* weights,
                                         const int* requested, const float* lr_dev, int64_t n,
                                         const dmx_separate_opts* opts, float* stems_dev,
                                         dmx_progress_fn progress, void* user);

/* ShiftRng (pipeline.rs:136-151, 416-418): the offsets, each in
 * [0, max_shift], that the separation drivers draw for `passes` shift passes
 * (every separation seeds a fresh generator with 0x5eed_1234), written to
 * out[0 .. passes). For callers that spread the passes or chunks of a track
 * over processes themselves. */
dmx_status dmx_shift_offsets(int passes, int64_t max_shift, int64_t* out);

/* Peer memory for one process per GPU (the multi-process form of the track
 * sharding; the reference runs one device: streaming.rs:296-400). A rank
 * exports a device buffer of its GPU (`device`) as a 64-byte CUDA IPC handle
 * and the offset of dev_ptr inside its allocation; another process on the
 * same node maps it with dmx_ipc_open on its own GPU (peer access over
 * NVLink enabled lazily) and unmaps it with dmx_ipc_close (the same offset).
 * The exporting process must keep the buffer alive while it is mapped. */
dmx_status dmx_ipc_export(int device, const void* dev_ptr, unsigned char handle[64],
                          int64_t* offset);
dmx_status dmx_ipc_open(int device, const unsigned char handle[64], int64_t offset, void** ptr);
dmx_status dmx_ipc_close(int device, void* ptr, int64_t offset);

/* The multi-process boundary merge and stem gather (the overlap-add tail a
 * rank adds from its left neighbour, streaming.rs:219-260, and the gather of
 * the stems to one rank): dst (rows x width, row stride dst_ld floats) =
 * src (row stride src_ld), or dst += src for dmx_rows_add (each sum rounded on
 * its own, so a merged sample equals the one-GPU overlap-add's bit for bit),
 * on the handle's stream, with the SMs reading src — typically a peer GPU's
 * buffer mapped by dmx_ipc_open — over NVLink. The caller orders the reads
 * after the peer's writes (e.g. a collective on both streams) and the peer's
 * next writes after the reads. */
dmx_status dmx_rows_copy(dmx_handle* h, float* dst, int64_t dst_ld, const float* src,
                         int64_t src_ld, int rows, int64_t width);
dmx_status dmx_rows_add(dmx_handle* h, float* dst, int64_t dst_ld, const float* src,
                        int64_t src_ld, int rows, int64_t width);

/* Chunk plan of a split pass (streaming.rs:88-94, 296-330): number of chunks
 * of a view of `view_length` samples. */
int64_t dmx_num_chunks(int64_t view_length, int segment, double overlap);

/* One shard of a track for multi-GPU chunk sharding: forward chunks
 * [chunk_lo, chunk_hi) (chunks of `segment` samples, at most 343980) of the
 * shift view of the (device, normalised) mix and
 * overlap-add them, unnormalised by the window sum, into `acc_dev` over view
 * samples [view_lo, view_hi) — (8, view_hi - view_lo) floats — adding to what
 * is there. The window sums are analytic (dmx_ola_finish divides by them). */
dmx_status dmx_track_shard(dmx_handle* h, const float* mix_norm_dev, int64_t length,
                           int64_t shift_offset, int64_t max_shift, int segment, double overlap,
                           double transition_power, int64_t chunk_lo, int64_t chunk_hi,
                           int batch, float* acc_dev, int64_t view_lo, int64_t view_hi);

/* The end of one split pass over the samples a rank owns (the flush and
 * denormalisation of streaming.rs:219-260 and api.rs:713-724): for output
 * samples t in [t_lo, t_hi) (t_hi < 0: to the end), stems = acc / (sum of the
 * triangular weights covering view sample t + trim) * std + mean, read from
 * acc_dev (8, view_length) as dmx_track_shard filled it (over the whole view)
 * and mean_std_dev from dmx_normalize_track_device. stems_dev is (4, 2,
 * length). Single pass only: shifts 0 (no trim) or 1 (trim max_shift -
 * shift_offset); scale 1/shifts = 1. */
dmx_status dmx_track_finish(dmx_handle* h, const float* acc_dev, int64_t length,
                            int64_t shift_offset, int64_t max_shift, int segment, double overlap,
                            double transition_power, int shifts, const float* mean_std_dev,
                            float* stems_dev, int64_t t_lo, int64_t t_hi);

/* SafeTensors::parse + get (safetensors.rs:38-108, 110-160) and
 * Checkpoint::from_bytes + get (ckpt/mod.rs:44-130): tensor `name` of a
 * checkpoint blob (safetensors or torch.save zip, as dmx_create reads them) as
 * f32, decoded by the loader dmx_create uses (F32, F16, BF16, F64 and integer
 * types upcast as safetensors.rs:110-135 does; views gathered through their
 * strides). Writes
 * the element count's floats to `out` (DMX_ERR_INVALID if more than `cap`),
 * the shape to `shape` (up to 8 dimensions) and its rank to `*ndim`; a
 * missing tensor or a malformed blob is DMX_ERR_WEIGHTS. Makes no CUDA call. */
dmx_status dmx_read_tensor(const void* safetensors_blob, size_t blob_len, const char* name,
                           float* out, int64_t cap, int64_t* shape, int* ndim);

/* Optional activation tracing (mirrors TraceSink, demucs/host.rs:117-125):
 * named intermediates copied to host in the reference's own layouts. */
typedef void (*dmx_trace_fn)(const char* name, const float* data, const int64_t* shape, int ndim,
                             void* user);
dmx_status dmx_set_trace(dmx_handle* h, dmx_trace_fn fn, void* user);

/* Per-launch device timing (cudaEvents between consecutive launches on the
 * handle's stream), off by default; it serialises nothing but adds one event
 * per launch. dmx_stage_times then reports, for the last forward, each kernel
 * tag with its summed milliseconds, launch count, algorithmic FLOPs (2 per
 * multiply-add) and minimum HBM bytes (every operand read once, every result
 * written once); `counts`, `flops` and `bytes` may be NULL. Returns the count
 * of tags written (at most `cap`). No counterpart in the reference (its
 * per-stage timing is the TraceSink, host.rs:117-125). */
dmx_status dmx_set_stage_timing(dmx_handle* h, int on);
int dmx_stage_times(dmx_handle* h, const char** names, float* ms, int* counts, double* flops,
                    double* bytes, int cap);

/* Self-test of the bounded-wait error path; no counterpart in the reference
 * (its device path has no waits that can time out). Every wait in this
 * library's tensor-core kernels gives up after a fixed time, raises the
 * handle's device error flag and returns, so a stuck pipeline becomes
 * DMX_ERR_TIMEOUT on the host instead of a hung GPU. Those waits only run out
 * when something is broken; this entry point runs one that always does: one
 * warp on the handle's stream waits on a device flag that nothing sets, gives
 * up after `wait_ms` (1..5000), and raises the flag. Returns DMX_ERR_TIMEOUT
 * (with dmx_last_error() naming the self-test) and leaves the handle usable. */
dmx_status dmx_selftest_wait_timeout(dmx_handle* h, int wait_ms);

/* Number of kernels the last forward launched. */
int64_t dmx_kernel_launches(dmx_handle* h);

/* The handle's CUDA stream (a cudaStream_t), for callers that order their
 * own work or events around the device entry points. */
void* dmx_stream(dmx_handle* h);

/* Waits (bounded) until the handle's stream has drained. */
dmx_status dmx_synchronize(dmx_handle* h);

#ifdef __cplusplus
}
#endif

#endif /* DMX_H */
