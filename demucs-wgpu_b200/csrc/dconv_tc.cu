// DConv residual branch on the tensor cores (host.rs:985-1059; the fused
// GroupNorm + GLU + LayerScale tail of ops.rs:930-1094) for the narrow layers
// (C = 48, 96): the spectral branch's rows of T = 336 frames and the waveform
// branch's long rows:
//
//   y = conv1(x)                    k = 3, C -> C/8, padding = dilation
//   g = GELU(GroupNorm1(y))         one group over (C/8, T) per row
//   z = conv2(g)                    1x1, C/8 -> 2C
//   x += gamma * GLU(GroupNorm1(z)) one group over (2C, T) per row
//
// Persistent: one CTA per SM walks work items of 384 frames (a row of at most
// 380 frames, or one tile of a longer row; the kernel below says how tiles
// and their 2-frame halos are laid). Per item:
//  * conv1 as tcgen05 MMAs (M = 128 frames x 3 blocks, N = the three taps'
//    16-slot outputs side by side, K = C): warp 0 streams the x tiles with TMA
//    (frames outside the row are TMA's zero fill) against conv1 weights that
//    stay in shared memory; warps 2-3 write each tile's low part
//    (x - tf32(x)); warp 1 issues the MMAs.
//  * warps 4-15 read the conv1 accumulators out of TMEM (which frees them for
//    the next item's conv1; warp 4 + 4b + q takes TMEM lanes 32q.. of block
//    b), combine the taps through shared memory, reduce the moments of y, and
//    write g (and its low part) to shared memory as the A operand of conv2.
//  * the moments of z come from g alone. With w_c the conv2 weights of output
//    column c (its bias on a constant-1 input slot), sum_c z_c = v.g and
//    sum_c z_c^2 = g'Mg for v = sum_c w_c and M = sum_c w_c w_c', constants
//    computed on the host; so z leaves TMEM once, for the output.
//  * conv2 against the resident conv2 weights (N = 96 columns per MMA) is
//    issued between the next item's conv1 stages; warps 4-15 combine it with
//    the residual (staged by TMA) straight into x, a third of the columns each.
//
// K slots: hidden channel h < HID/2 sits at slot h, the others at slot
// 8 + h - HID/2; slot 15 is the constant 1 that carries conv2's bias. The
// host packs the tensor-core weight copies in this order.
//
// Precision: 3xTF32 (lo*hi + hi*lo + hi*hi). The high part of an fp32 operand
// is the operand itself (the tensor core reads it truncated to tf32); the low
// part is x - trunc_tf32(x), exact in fp32. The weights' high parts are
// rounded to nearest on the host and their residuals stored beside them. The
// result agrees with fp32 arithmetic to ~1e-6 relative; moments are summed in
// f64 as the reference's GroupNorm does. With SPLIT off (the BF16 build) the
// contractions are single-pass tf32: no low parts, one product per K step.
// No load uses cluster multicast.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace dmx {

namespace {

constexpr int kThreads = 512;  // w0 TMA, w1 MMA, w2-3 converter, w4-15 epilogue
constexpr int kEpiBase = 128;  // first epilogue thread
constexpr int kEpiThreads = 384;
constexpr int kEpiWarps = 12;

template <int C>
struct DcTc {
  static constexpr int HID = C / 8;
  static constexpr int JA = HID / 2;              // hidden channels below K slot 8
  static constexpr int ACT = HID + 1;             // conv2 K slots in use (hidden, bias)
  static constexpr int NQ = ACT * (ACT + 1) / 2;  // packed upper triangle of M
  static constexpr int YS = (HID + 3) / 4 * 4;    // floats per frame of the y buffer
  static constexpr int HP = 16;                   // K slots of conv2 (conv1 N per tap)
  static constexpr int N1 = 3 * HP;               // conv1 N: the three taps' outputs side by side
  static constexpr int BK = C % 32 == 0 ? 32 : 16;  // conv1 K (channels) per stage
  static constexpr int KB = C / BK;               // conv1 K blocks per 128-frame block
  static constexpr int NCH = 96;                  // conv2 columns per MMA (48 channels)
  static constexpr int NCHUNK = 2 * C / NCH;
  // C = 48: the three blocks' conv2 outputs (3 x 96 columns) fit in TMEM next
  // to conv1's, so conv2 runs once per item into them; otherwise in 96-column
  // chunks through two TMEM buffers
  static constexpr bool ALL = NCHUNK == 1;
  static constexpr int A_BYTES = 128 * BK * 4;
  static constexpr int STAGE = 2 * A_BYTES;  // x tile | its low part
  static constexpr int STAGES = C == 48 ? 4 : 3;
  static constexpr int W1_KB = N1 * BK * 4;        // conv1 weights of one K block (3 taps)
  static constexpr int W1_BYTES = KB * W1_KB;      // [kb][tap][16 slots][BK], hi or lo
  static constexpr int G_BYTES = 128 * HP * 4;     // one 128-frame block of g
  static constexpr int W2_BYTES = 2 * C * HP * 4;
  static constexpr int OFF_W1 = STAGES * STAGE;    // w1 hi | w1 lo
  // g hi [3] | g lo [3]; before g is formed the same 48 KB holds the tap-0
  // and tap-2 outputs of all 384 frames for the neighbour exchange
  static constexpr int OFF_G = OFF_W1 + 2 * W1_BYTES;
  static constexpr int OFF_W2 = OFF_G + 6 * G_BYTES;       // w2 hi | w2 lo
  static constexpr int OFF_CH = OFF_W2 + 2 * W2_BYTES;     // per-channel constants [C][8]
  static constexpr int OFF_AFF = OFF_CH + C * 32;          // per-item GN2 affine [C] float4
  // ALL: the item's x (the residual), 9 TMA boxes of 16 channels x 128
  // frames, [block][channel group][frame][16], 64-byte swizzle
  static constexpr int OFF_RES = (OFF_AFF + C * 16 + 1023) / 1024 * 1024;
  static constexpr int RES_BOX = 128 * 64;
  static constexpr int RES_BYTES = ALL ? 9 * RES_BOX : 0;
  static constexpr int SMEM = OFF_RES + RES_BYTES + 1024;
  static_assert(2 * C % NCH == 0 && HID % 2 == 0 && JA <= 7 && SMEM <= 227 * 1024, "shape");
  static_assert(!ALL || BK == 16, "the residual boxes reuse the x map");
  // K slot of the i-th input of conv2 (the hidden channels, then the bias)
  static constexpr int act_slot(int i) { return i < JA ? i : (i < HID ? 8 + i - JA : 15); }
  // 16-byte chunks (of a 16-slot row) that hold hidden channels
  static constexpr bool chunk_used(int c) { return (c % 2) * 4 < JA; }
};

// C = 192 (hidden 24), single-pass tf32 only (dconv_tc_wide_kernel): conv1's
// three taps come from three x tiles loaded at frame offsets -d, 0, +d into
// one accumulator of 32 columns (the hidden channels, zero-padded), so no
// tap exchange is needed; g lives in TMEM as conv2's A operand, 32 K slots
// (hidden channel h at slot h, the constant 1 that carries the bias at slot
// 31). Shared memory: the x ring, conv1's weights (3 taps x 6 K blocks of
// 32 x 32) and conv2's (384 x 32), all with 128-byte rows.
template <>
struct DcTc<192> {
  static constexpr int C = 192;
  static constexpr int HID = C / 8;
  static constexpr int ACT = HID + 1;
  static constexpr int NQ = ACT * (ACT + 1) / 2;
  static constexpr int YS = (HID + 3) / 4 * 4;
  static constexpr int KS = 32;        // conv1 N per block = conv2 K slots
  static constexpr int BIAS = KS - 1;  // the K slot of conv2's bias
  static constexpr int BK = 32;        // conv1 K (channels) per x tile
  static constexpr int KB = C / BK;
  static constexpr int NCH = 96;       // conv2 columns per MMA (48 channels)
  static constexpr int NCHUNK = 2 * C / NCH;
  static constexpr int NB2 = 3;        // conv2 accumulators in TMEM
  static constexpr int A_BYTES = 128 * BK * 4;
  static constexpr int STAGES = 5;
  static constexpr int W1_TILE = KS * BK * 4;        // one tap, one K block
  static constexpr int W1_BYTES = 3 * KB * W1_TILE;  // [tap][kb][32 rows][32]
  static constexpr int W2_BYTES = 2 * C * KS * 4;    // [2C rows][32 slots]
  static constexpr int OFF_W1 = STAGES * A_BYTES;
  static constexpr int OFF_W2 = OFF_W1 + W1_BYTES;
  static constexpr int OFF_CH = OFF_W2 + W2_BYTES;  // per-channel constants [C][8]
  static constexpr int OFF_AFF = OFF_CH + C * 32;   // per-item GN2 affine [C] float4
  static constexpr int SMEM = OFF_AFF + C * 16 + 1024;
  // TMEM columns: conv1 of block m at 32 m, g of block m at 96 + 32 m, the
  // conv2 accumulators at 192 + 96 j
  static constexpr uint32_t TM_D1 = 0, TM_G = 96, TM_D2 = 192;
  static_assert(TM_D2 + NB2 * NCH <= 512 && HID < BIAS && 2 * C % NCH == 0, "tmem");
  // dynamic shared memory plus the kernel's static barriers within 227 KB
  static_assert(SMEM <= 227 * 1024 - 1024, "smem");
};

// Per-layer constants, passed by value (they sit in the constant bank): the
// moments of z as functions of g (v and M above, over the active K slots in
// act_slot order) and GroupNorm1's per-channel terms with conv1's bias.
template <int C>
struct DcConst {
  float v[DcTc<C>::ACT];
  float m[DcTc<C>::NQ];  // upper triangle by rows, off-diagonal entries doubled
  float b1[DcTc<C>::HID], n1w[DcTc<C>::HID], n1b[DcTc<C>::HID];
};

__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

DMX_DEVICE float trunc_tf32(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

DMX_DEVICE void epi_bar() { asm volatile("bar.sync 1, 384;" ::: "memory"); }

DMX_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Sum of (s, q) over the epilogue threads, fixed order; all get the result.
DMX_DEVICE void epi_sum2(double& s, double& q, double* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    q += __shfl_xor_sync(0xffffffffu, q, o);
  }
  const int e = threadIdx.x / 32 - kEpiBase / 32;
  if ((threadIdx.x & 31) == 0) {
    red[2 * e] = s;
    red[2 * e + 1] = q;
  }
  epi_bar();
  s = 0.0;
  q = 0.0;
#pragma unroll
  for (int w = 0; w < kEpiWarps; ++w) {
    s += red[2 * w];
    q += red[2 * w + 1];
  }
  epi_bar();  // red may be rewritten by the next reduction
}

// GroupNorm statistics from the sums; inv_count = 1 / (elements in the group).
DMX_DEVICE void norm_of(double s, double q, double inv_count, float& mean, float& inv) {
  const double m = s * inv_count;
  const double var = fmax(q * inv_count - m * m, 0.0);
  mean = (float)m;
  inv = 1.0f / sqrtf((float)(var + 1e-5));
}

// Work item = (row, tile): local frame i of the item is frame ts + i of the
// row, ts = 380 tile - 2; the item owns local frames 2 .. 381 (those inside
// the row). Rows of at most 380 frames are one item (mode DC_ROW, all of the
// branch in one launch, row moments reduced inside the CTA). Longer rows run
// three launches: DC_STATS1 (conv1 from x: y into the y buffer and the
// moments of y per tile), DC_STATS2 (g from y with the row's moments summed
// over its tiles in a fixed order; the moments of z per tile — launched as
// dconv_tc_stats2_kernel, which runs the same arithmetic many blocks per SM)
// and DC_OUT
// (conv2 and the output). Only DC_STATS1 reads the halo frames, so the
// output written in place by one tile never reaches another tile's input.
enum DcMode : int { DC_ROW = 0, DC_STATS1 = 1, DC_STATS2 = 2, DC_OUT = 3 };
constexpr int kTileStride = 380;

template <int C, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
    dconv_tc_row_kernel(const __grid_constant__ CUtensorMap tmX,
                        const __grid_constant__ CUtensorMap tmW1,
                        const __grid_constant__ CUtensorMap tmW1lo,
                        const __grid_constant__ CUtensorMap tmW2,
                        const __grid_constant__ CUtensorMap tmW2lo, const DConvArgs a,
                        const __grid_constant__ DcConst<C> k, int mode) {
  using S = DcTc<C>;
  // x ring: 3xTF32 stages hold a tile and its low part; single-pass ones only
  // the tile, so the same bytes make twice the stages
  constexpr int NST = SPLIT ? S::STAGES : 2 * S::STAGES;
  constexpr int SST = SPLIT ? S::STAGE : S::A_BYTES;
  static_assert(NST * SST == S::STAGES * S::STAGE, "ring");
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ __align__(8) uint64_t full[NST], empty[NST], conv[NST];
  __shared__ __align__(8) uint64_t w1_full, w2_full, d1_full, d1_empty, g_ready, res_full;
  __shared__ __align__(8) uint64_t d2_full[2], d2_empty[2];
  __shared__ uint32_t tmem_slot;
  __shared__ double red[2 * kEpiWarps];

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (a.err && *reinterpret_cast<volatile int*>(a.err) != 0) return;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], 64);
    }
    mbar_init(&w1_full, 1);
    mbar_init(&w2_full, 1);
    mbar_init(&d1_full, 1);
    mbar_init(&d1_empty, kEpiThreads);
    mbar_init(&g_ready, kEpiThreads);
    mbar_init(&res_full, 1);
    for (int j = 0; j < 2; ++j) {
      mbar_init(&d2_full[j], 1);
      mbar_init(&d2_empty[j], kEpiThreads);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_slot;
  // D1 (conv1, block m): columns 64 m; D2 (conv2): 192 + 96 m (ALL) or the
  // two buffers 256 + 128 j
  const uint32_t tm_d1 = tmem, tm_d2 = tmem + 256;
  const int T = a.T;
  const int items = a.rows * a.tiles;
  const bool conv1 = mode == DC_ROW || mode == DC_STATS1;
  const bool conv2 = mode == DC_ROW || mode == DC_OUT;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      if (conv2) {
        mbar_expect_tx(&w2_full, (SPLIT ? 2 : 1) * S::W2_BYTES);
        tma_load_2d(smem + S::OFF_W2, &tmW2, &w2_full, 0, 0);
        if (SPLIT) tma_load_2d(smem + S::OFF_W2 + S::W2_BYTES, &tmW2lo, &w2_full, 0, 0);
      }
      if (conv1) {
        // conv1 weights, once: K block kb's taps side by side (B rows 16 tap ..)
        mbar_expect_tx(&w1_full, (SPLIT ? 2 : 1) * S::W1_BYTES);
        for (int kb = 0; kb < S::KB; ++kb)
          for (int tap = 0; tap < 3; ++tap) {
            unsigned char* b = smem + S::OFF_W1 + kb * S::W1_KB + tap * S::HP * S::BK * 4;
            tma_load_2d(b, &tmW1, &w1_full, tap * C + kb * S::BK, 0);
            if (SPLIT) tma_load_2d(b + S::W1_BYTES, &tmW1lo, &w1_full, tap * C + kb * S::BK, 0);
          }
        uint32_t it = 0;
        bool ok = true;
        for (int w = blockIdx.x; w < items && ok; w += gridDim.x) {
          const int row = w / a.tiles, ts = (w - row * a.tiles) * kTileStride - 2;
          for (int m = 0; m < 3 && ok; ++m) {
            for (int kb = 0; kb < S::KB; ++kb, ++it) {
              const int s = it % NST;
              if (!mbar_wait(&empty[s], ((it / NST) & 1) ^ 1, a.err, 31)) {
                ok = false;
                break;
              }
              mbar_expect_tx(&full[s], S::A_BYTES);
              // frames ts + 128 m .. +127 (zero outside the row), channels kb BK ..
              tma_load_3d(smem + s * SST, &tmX, &full[s], kb * S::BK, ts + m * 128, row);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc1 = idesc_tf32(128, S::N1);
      constexpr uint32_t idesc2 = idesc_tf32(128, S::NCH);
      bool ok = (!conv1 || mbar_wait(&w1_full, 0, a.err, 29)) &&
                (!conv2 || mbar_wait(&w2_full, 0, a.err, 32));
      uint32_t it = 0, u = 0;
      // conv2 of item `pend` (-1: none) is issued once its g is in shared
      // memory: `g_in` says that wait is over, `cur` counts its issued chunks
      int pend = -1, cur = 0;
      bool g_in = false;
      // conv2 of block m, 96 columns from w2 column 96 ch, into TMEM column d
      auto conv2_mma = [&](uint32_t d, int m, int ch) {
        const uint32_t g_hi = smem_u32(smem + S::OFF_G + m * S::G_BYTES);
        const uint32_t g_lo = g_hi + 3 * S::G_BYTES;
        const uint32_t w_hi = smem_u32(smem + S::OFF_W2 + ch * S::NCH * 64);
        const uint32_t w_lo = w_hi + S::W2_BYTES;
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const uint64_t gh = umma_desc_k(g_hi + kk * 32, 64);
          const uint64_t wh = umma_desc_k(w_hi + kk * 32, 64);
          if (SPLIT) {
            umma_tf32(d, umma_desc_k(g_lo + kk * 32, 64), wh, idesc2, kk != 0);
            umma_tf32(d, gh, umma_desc_k(w_lo + kk * 32, 64), idesc2, 1);
            umma_tf32(d, gh, wh, idesc2, 1);
          } else {
            umma_tf32(d, gh, wh, idesc2, kk != 0);
          }
        }
      };
      // Issues what it can of item pend's conv2; with `block`, all of it.
      auto conv2_progress = [&](bool block) {
        if (pend < 0 || !ok) return;
        if (!g_in) {
          if (block) {
            if (!mbar_wait(&g_ready, pend & 1, a.err, 34)) {
              ok = false;
              return;
            }
          } else if (!mbar_test(&g_ready, pend & 1)) {
            return;
          }
          g_in = true;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        }
        if constexpr (S::ALL) {
          // the previous item's outputs have been read out of TMEM
          const uint32_t par = (pend & 1) ^ 1;
          if (block) {
            if (!mbar_wait(&d2_empty[0], par, a.err, 35)) {
              ok = false;
              return;
            }
          } else if (!mbar_test(&d2_empty[0], par)) {
            return;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll 1
          for (int m = 0; m < 3; ++m) conv2_mma(tmem + 192 + 96 * m, m, 0);
          umma_commit(&d2_full[0]);
        } else {
          while (cur < 3 * S::NCHUNK) {
            const int j = u & 1;
            const uint32_t par = ((u >> 1) & 1) ^ 1;
            if (block) {
              if (!mbar_wait(&d2_empty[j], par, a.err, 35)) {
                ok = false;
                return;
              }
            } else if (!mbar_test(&d2_empty[j], par)) {
              return;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            conv2_mma(tm_d2 + 128 * j, cur / S::NCHUNK, cur % S::NCHUNK);
            umma_commit(&d2_full[j]);
            ++u;
            ++cur;
          }
        }
        pend = -1;
      };
      int ri = 0;
      if (conv1) {
        for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++ri) {
          // D1 is free once the epilogue has read the previous item's conv1
          if (!mbar_wait(&d1_empty, (ri & 1) ^ 1, a.err, 30)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          for (int m = 0; m < 3 && ok; ++m) {
            const uint32_t d = tm_d1 + 64 * m;
            for (int kb = 0; kb < S::KB; ++kb, ++it) {
              conv2_progress(false);
              const int s = it % NST;
              const uint32_t par = (it / NST) & 1;
              const uint32_t a_hi = smem_u32(smem + s * SST);
              const uint32_t a_lo = a_hi + S::A_BYTES;
              const uint32_t b_hi = smem_u32(smem + S::OFF_W1 + kb * S::W1_KB);
              const uint32_t b_lo = b_hi + S::W1_BYTES;
              // the x tile has landed: its high-part products
              if (!ok || !mbar_wait(&full[s], par, a.err, 33)) {
                ok = false;
                break;
              }
              asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
              for (int j = 0; j < S::BK / 8; ++j) {
                const uint64_t ah = umma_desc_k(a_hi + j * 32, S::BK * 4);
                umma_tf32(d, ah, umma_desc_k(b_hi + j * 32, S::BK * 4), idesc1, (kb | j) != 0);
                if (SPLIT) umma_tf32(d, ah, umma_desc_k(b_lo + j * 32, S::BK * 4), idesc1, 1);
              }
              if (SPLIT) {
                // its low part is written: the last product
                if (!mbar_wait(&conv[s], par, a.err, 28)) {
                  ok = false;
                  break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
                for (int j = 0; j < S::BK / 8; ++j)
                  umma_tf32(d, umma_desc_k(a_lo + j * 32, S::BK * 4),
                            umma_desc_k(b_hi + j * 32, S::BK * 4), idesc1, 1);
              }
              umma_commit(&empty[s]);
            }
          }
          if (!ok) break;
          umma_commit(&d1_full);
          conv2_progress(true);  // the rest of the previous item's conv2
          if (conv2) {
            pend = ri;
            cur = 0;
            g_in = false;
          }
        }
        conv2_progress(true);
      } else if (conv2) {
        // DC_OUT: conv2 alone, item by item
        for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++ri) {
          pend = ri;
          cur = 0;
          g_in = false;
          conv2_progress(true);
        }
      }
    }
  } else if (warp < 4) {
    // ---------------- converter: the low part of each x tile row ----------------
    if (conv1 && SPLIT) {
      const int c = threadIdx.x - 64;  // rows c and c + 64 (the same swizzle phase)
      const int swz = S::BK == 32 ? (c & 7) : ((c >> 1) & 3);
      uint32_t it = 0;
      bool live = true;
      for (int w = blockIdx.x; w < items; w += gridDim.x)
        for (int m = 0; m < 3; ++m)
          for (int kb = 0; kb < S::KB; ++kb, ++it) {
            const int s = it % NST;
            if (live && !mbar_wait(&full[s], (it / NST) & 1, a.err, 36)) live = false;
            if (live) {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int r = c + 64 * h;
                const float4* x4 = reinterpret_cast<const float4*>(smem + s * SST + r * S::BK * 4);
                float4* lo4 = reinterpret_cast<float4*>(smem + s * SST + S::A_BYTES + r * S::BK * 4);
#pragma unroll
                for (int qq = 0; qq < S::BK / 4; ++qq) {
                  const int q = qq ^ swz;
                  const float4 x = x4[q];
                  lo4[q] = make_float4(x.x - trunc_tf32(x.x), x.y - trunc_tf32(x.y),
                                       x.z - trunc_tf32(x.z), x.w - trunc_tf32(x.w));
                }
              }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(&conv[s]);
          }
    }
  } else {
    // ---------------- epilogue: warps 4-15 ----------------
    // TMEM lane quarter q = warp % 4 (frames 32q .. 32q+31 of a block); b:
    // the block of this warp's frames for conv1, its third of the columns of
    // each 96-column conv2 chunk for the output
    const int e = warp - 4, q = warp % 4, b = e / 4;
    const int r = q * 32 + lane;
    const int p = 128 * b + r;  // this thread's frame (conv1, g)
    const int et = threadIdx.x - kEpiBase;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    // per channel c: conv2 bias (value, gate), GN2 weight and bias (value,
    // gate), LayerScale
    float4* chan = reinterpret_cast<float4*>(smem + S::OFF_CH);
    for (int c = et; c < C; c += kEpiThreads) {
      chan[2 * c] = make_float4(a.b2[2 * c], a.b2[2 * c + 1], a.n2w[c], a.n2w[c + C]);
      chan[2 * c + 1] = make_float4(a.n2b[c], a.n2b[c + C], a.gamma[c], 0.f);
    }
    epi_bar();
    const double ic1 = 1.0 / ((double)S::HID * T), ic2 = 1.0 / (2.0 * C * T);
    // the row's moments from its tiles' partials, summed by one warp in a
    // fixed order; every epilogue thread gets them
    auto row_sum = [&](const double* part, int row, double& s, double& q2) {
      if (warp == kEpiBase / 32) {
        double ls = 0.0, lq = 0.0;
        for (int t = lane; t < a.tiles; t += 32) {
          ls += part[2 * ((int64_t)row * a.tiles + t)];
          lq += part[2 * ((int64_t)row * a.tiles + t) + 1];
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
          ls += __shfl_xor_sync(0xffffffffu, ls, o);
          lq += __shfl_xor_sync(0xffffffffu, lq, o);
        }
        if (lane == 0) {
          red[0] = ls;
          red[1] = lq;
        }
      }
      epi_bar();
      s = red[0];
      q2 = red[1];
      epi_bar();
    };
    uint32_t u = 0;
    int ri = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < items; w += gridDim.x, ++ri) {
      const int row = w / a.tiles, ts = (w - row * a.tiles) * kTileStride - 2;
      // local frame i = 128 m + r is frame ts + i; owned: 2 <= i < 382, inside the row
      auto owned = [&](int i) { return i >= 2 && i < 382 && ts + i < T; };
      const bool mine = owned(p);
      // the item's x for the residual, 9 boxes of 16 channels (ALL): issued
      // once every thread is past the previous item's output
      auto stage_residual = [&]() {
        if constexpr (S::ALL) {
          if (conv2 && threadIdx.x == kEpiBase) {
            mbar_expect_tx(&res_full, S::RES_BYTES);
            for (int m = 0; m < 3; ++m)
              for (int g = 0; g < 3; ++g)
                tma_load_3d(smem + S::OFF_RES + (3 * m + g) * S::RES_BOX, &tmX, &res_full, 16 * g,
                            ts + 128 * m, row);
          }
        }
      };
      float yh[S::HID];  // y of frame p by hidden channel
      double s, sq;
      if (conv1) {
        // ---- y = conv1 + bias ----
        // D1 holds Y_k = W_k x (k = tap) per frame; y[p] = Y_0[p-d] + Y_1[p] +
        // Y_2[p+d]. Y_0 and Y_2 go through shared memory to the neighbours
        // (frames 384 x 16 slots each, 64-byte rows with the 64-byte swizzle).
        if (ok && !mbar_wait(&d1_full, ri & 1, a.err, 37)) ok = false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        float* x0s = reinterpret_cast<float*>(smem + S::OFF_G);
        float* x2s = x0s + 384 * 16;
        float y1[16];
        {
          uint32_t d1[48];
          __syncwarp();
#pragma unroll
          for (int tap = 0; tap < 3; ++tap)
            tmem_ld16_nw(tm_d1 + lane_base + 64 * b + 16 * tap, d1 + 16 * tap);
          tmem_ld_wait<48>(d1);
          // D1 is read out: the next item's conv1 may overwrite it
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          mbar_arrive(&d1_empty);
#pragma unroll
          for (int j = 0; j < 16; ++j) y1[j] = __uint_as_float(d1[16 + j]);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            if (!S::chunk_used(c)) continue;
            const int off = p * 16 + ((c ^ ((p >> 1) & 3)) << 2);
            *reinterpret_cast<uint4*>(x0s + off) =
                make_uint4(d1[4 * c], d1[4 * c + 1], d1[4 * c + 2], d1[4 * c + 3]);
            *reinterpret_cast<uint4*>(x2s + off) =
                make_uint4(d1[32 + 4 * c], d1[32 + 4 * c + 1], d1[32 + 4 * c + 2], d1[32 + 4 * c + 3]);
          }
        }
        epi_bar();
        stage_residual();
        const int pl = p - a.dil, pr = p + a.dil;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (!S::chunk_used(c)) continue;
          float4 l = make_float4(0.f, 0.f, 0.f, 0.f), rg = l;
          if (pl >= 0)
            l = *reinterpret_cast<const float4*>(x0s + pl * 16 + ((c ^ ((pl >> 1) & 3)) << 2));
          if (pr < 384)
            rg = *reinterpret_cast<const float4*>(x2s + pr * 16 + ((c ^ ((pr >> 1) & 3)) << 2));
          y1[4 * c] += l.x + rg.x;
          y1[4 * c + 1] += l.y + rg.y;
          y1[4 * c + 2] += l.z + rg.z;
          y1[4 * c + 3] += l.w + rg.w;
        }
        float fs = 0.f, fq = 0.f;
#pragma unroll
        for (int h = 0; h < S::HID; ++h) {
          yh[h] = y1[S::act_slot(h)] + k.b1[h];
          fs += yh[h];
          fq = fmaf(yh[h], yh[h], fq);
        }
        s = mine ? fs : 0.f;
        sq = mine ? fq : 0.f;
        if (mode == DC_STATS1) {
          // y of the owned frames for the later launches
          if (mine) {
            float4* yp = reinterpret_cast<float4*>(a.y + ((int64_t)row * T + ts + p) * S::YS);
#pragma unroll
            for (int c = 0; c < S::YS / 4; ++c) {
              float t4[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) t4[i] = 4 * c + i < S::HID ? yh[4 * c + i] : 0.f;
              yp[c] = make_float4(t4[0], t4[1], t4[2], t4[3]);
            }
          }
          epi_sum2(s, sq, red);
          if (threadIdx.x == kEpiBase) {
            a.part1[2 * (int64_t)w] = s;
            a.part1[2 * (int64_t)w + 1] = sq;
          }
          continue;
        }
        epi_sum2(s, sq, red);
      } else {
        // DC_STATS2, DC_OUT: y of the owned frames from the buffer
        if (mine) {
          const float4* yp = reinterpret_cast<const float4*>(a.y + ((int64_t)row * T + ts + p) * S::YS);
#pragma unroll
          for (int c = 0; c < S::YS / 4; ++c) {
            const float4 v = yp[c];
            const float t4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
              if (4 * c + i < S::HID) yh[4 * c + i] = t4[i];
          }
        } else {
#pragma unroll
          for (int h = 0; h < S::HID; ++h) yh[h] = 0.f;
        }
        row_sum(a.part1, row, s, sq);
        stage_residual();
      }
      // ---- g = GELU(GN1(y)) of frame p; conv2's A operand ----
      float mean, inv;
      norm_of(s, sq, ic1, mean, inv);
      float ga[S::ACT];  // g by conv2 input (hidden channels, then the bias input 1)
#pragma unroll
      for (int h = 0; h < S::HID; ++h) {
        const float scale = inv * k.n1w[h];
        ga[h] = mine ? gelu_tc(yh[h] * scale + (k.n1b[h] - mean * scale)) : 0.f;
      }
      ga[S::HID] = 1.0f;
      if (conv2) {
        float gs[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) gs[j] = 0.f;
#pragma unroll
        for (int i = 0; i < S::ACT; ++i) gs[S::act_slot(i)] = ga[i];
        // row r of block b's 128 x 16 K-major tile, 64-byte swizzle: 16-byte
        // chunk c lives at chunk c ^ ((r / 2) % 4)
        unsigned char* hi = smem + S::OFF_G + b * S::G_BYTES + r * 64;
        unsigned char* lo = hi + 3 * S::G_BYTES;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int phys = (c ^ ((r >> 1) & 3)) << 4;
          const float4 v = make_float4(gs[4 * c], gs[4 * c + 1], gs[4 * c + 2], gs[4 * c + 3]);
          *reinterpret_cast<float4*>(hi + phys) = v;
          if (SPLIT)
            *reinterpret_cast<float4*>(lo + phys) =
                make_float4(v.x - trunc_tf32(v.x), v.y - trunc_tf32(v.y), v.z - trunc_tf32(v.z),
                            v.w - trunc_tf32(v.w));
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        mbar_arrive(&g_ready);
      }

      // ---- moments of z: the sums of v.g and g'Mg over the owned frames ----
      if (mode == DC_OUT) {
        row_sum(a.part2, row, s, sq);
      } else {
        float l = 0.f, qf = 0.f;
        if (mine) {
#pragma unroll
          for (int i = 0, idx = 0; i < S::ACT; ++i) {
            l = fmaf(k.v[i], ga[i], l);
            float t = 0.f;
#pragma unroll
            for (int j = i; j < S::ACT; ++j, ++idx) t = fmaf(k.m[idx], ga[j], t);
            qf = fmaf(ga[i], t, qf);
          }
        }
        s = l;
        sq = qf;
        epi_sum2(s, sq, red);
        if (mode == DC_STATS2) {
          if (threadIdx.x == kEpiBase) {
            a.part2[2 * (int64_t)w] = s;
            a.part2[2 * (int64_t)w + 1] = sq;
          }
          continue;
        }
      }
      float mean2, inv2;
      norm_of(s, sq, ic2, mean2, inv2);
      // GN2 with LayerScale folded in: gamma * value = z_v * a + b, gate = z_g * c + d
      float4* aff = reinterpret_cast<float4*>(smem + S::OFF_AFF);
      for (int c = et; c < C; c += kEpiThreads) {
        const float4 t0 = chan[2 * c], t1 = chan[2 * c + 1];
        const float vs = inv2 * t0.z, gs = inv2 * t0.w;
        aff[c] = make_float4(t1.z * vs, t1.z * (t1.x - mean2 * vs), gs, t1.y - mean2 * gs);
      }
      epi_bar();

      // ---- conv2, the output: x += gamma * GLU(GN2(z)) ----
      // TMEM column of conv2 block m (ALL), or of buffer j (chunked)
      auto d2_col = [&](int m, int j) -> uint32_t {
        return S::ALL ? 192u + 96u * m : 256u + 128u * j;
      };
      if (S::ALL) {
        if (ok && !mbar_wait(&d2_full[0], ri & 1, a.err, 38)) ok = false;
        if (ok && !mbar_wait(&res_full, ri & 1, a.err, 27)) ok = false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      }
      for (int m = 0; m < 3; ++m)
        for (int ch = 0; ch < S::NCHUNK; ++ch) {
          const int j = u & 1;
          const int pm = m * 128 + r;
          const bool own = owned(pm);
          const int c0 = ch * (S::NCH / 2) + 16 * b;  // this thread's 16 channels
          float* xp = a.x + ((int64_t)row * T + (own ? ts + pm : 0)) * C + c0;
          // the residual, then the output, of this thread's 16 channels (64
          // bytes at a 32-byte-aligned address: frames are 192 or 384 bytes)
          float o[16];
          if (!S::ALL) {
            // the residual from HBM, in flight while this chunk's conv2 completes
            if (ok && own) {
              ld_global8(xp, o);
              ld_global8(xp + 8, o + 8);
            }
            if (ok && !mbar_wait(&d2_full[j], (u >> 1) & 1, a.err, 39)) ok = false;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          }
          uint32_t zr[32];
          __syncwarp();
          tmem_ld16_nw(tmem + lane_base + d2_col(m, j) + 32 * b, zr);
          tmem_ld16_nw(tmem + lane_base + d2_col(m, j) + 32 * b + 16, zr + 16);
          if (S::ALL) {
            const unsigned char* rb = smem + S::OFF_RES + (3 * m + b) * S::RES_BOX + r * 64;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float4 t = *reinterpret_cast<const float4*>(rb + ((i ^ ((r >> 1) & 3)) << 4));
              o[4 * i] = t.x;
              o[4 * i + 1] = t.y;
              o[4 * i + 2] = t.z;
              o[4 * i + 3] = t.w;
            }
          }
          tmem_ld_wait<32>(zr);
          if (!S::ALL) {
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            mbar_arrive(&d2_empty[j]);
            ++u;
          }
          if (ok && own) {
#pragma unroll
            for (int kk = 0; kk < 16; ++kk) {
              const float4 f = aff[c0 + kk];
              // gamma * GN2(value), GN2(gate)
              const float value = fmaf(__uint_as_float(zr[2 * kk]), f.x, f.y);
              const float gate = fmaf(__uint_as_float(zr[2 * kk + 1]), f.z, f.w);
              o[kk] += glu_tc(value, gate);
              if (a.round_out) o[kk] = round_tf32(o[kk]);
            }
            st_global8(xp, o);
            st_global8(xp + 8, o + 8);
          }
        }
      if (S::ALL) {
        // this item's conv2 outputs are read out: the next item's may be written
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        mbar_arrive(&d2_empty[0]);
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

// DConv of a C = 192 layer on the tensor cores, single-pass tf32 (the BF16
// build). Same work items, modes, moments and output arithmetic as
// dconv_tc_row_kernel; what differs is the width:
//  * conv1: per 128-frame block m, tap t and 32-channel K block kb, warp 0
//    loads the x tile at frames ts + 128 m + (t - 1) d (TMA zero-fills
//    frames outside the row) and warp 1 accumulates it against tap t's
//    weights into the block's 32 TMEM columns; a block's centre-tap tiles
//    go first, so the outer taps' loads (the same frames shifted by d)
//    mostly hit L2.
//  * the epilogue warps read y straight out of TMEM (no tap exchange), write
//    g into TMEM as conv2's A operand (with the constant 1 at slot 31), and
//    conv2 runs in 96-column chunks (48 channels) through three TMEM
//    accumulators, overlapping the output of the chunk before.
template <int C>
__global__ void __launch_bounds__(kThreads, 1)
    dconv_tc_wide_kernel(const __grid_constant__ CUtensorMap tmX,
                         const __grid_constant__ CUtensorMap tmW1,
                         const __grid_constant__ CUtensorMap tmW2, const DConvArgs a,
                         const __grid_constant__ DcConst<C> k, int mode) {
  using S = DcTc<C>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ __align__(8) uint64_t full[S::STAGES], empty[S::STAGES];
  __shared__ __align__(8) uint64_t w1_full, w2_full, d1_full, d1_empty, g_ready;
  __shared__ __align__(8) uint64_t d2_full[S::NB2], d2_empty[S::NB2];
  __shared__ uint32_t tmem_slot;
  __shared__ double red[2 * kEpiWarps];

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (a.err && *reinterpret_cast<volatile int*>(a.err) != 0) return;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&w1_full, 1);
    mbar_init(&w2_full, 1);
    mbar_init(&d1_full, 1);
    mbar_init(&d1_empty, kEpiThreads);
    mbar_init(&g_ready, kEpiThreads);
    for (int j = 0; j < S::NB2; ++j) {
      mbar_init(&d2_full[j], 1);
      mbar_init(&d2_empty[j], kEpiThreads);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_slot;
  const int T = a.T;
  const int items = a.rows * a.tiles;
  const bool conv1 = mode == DC_ROW || mode == DC_STATS1;
  const bool conv2 = mode == DC_ROW || mode == DC_OUT;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      if (conv2) {
        mbar_expect_tx(&w2_full, S::W2_BYTES);
        for (int h = 0; h < 2; ++h)
          tma_load_2d(smem + S::OFF_W2 + h * C * 128, &tmW2, &w2_full, 0, h * C);
      }
      if (conv1) {
        mbar_expect_tx(&w1_full, S::W1_BYTES);
        for (int tap = 0; tap < 3; ++tap)
          for (int kb = 0; kb < S::KB; ++kb)
            tma_load_2d(smem + S::OFF_W1 + (tap * S::KB + kb) * S::W1_TILE, &tmW1, &w1_full,
                        tap * C + kb * S::BK, 0);
        uint32_t it = 0;
        bool ok = true;
        for (int w = blockIdx.x; w < items && ok; w += gridDim.x) {
          const int row = w / a.tiles, ts = (w - row * a.tiles) * kTileStride - 2;
          // per block: the centre tap's tiles first, then the outer taps'
          // (the same frames shifted by d, mostly L2 hits by then)
          for (int m = 0; m < 3 && ok; ++m)
            for (int ti = 0; ti < 3 && ok; ++ti)
              for (int kb = 0; kb < S::KB; ++kb, ++it) {
                const int tap = ti == 0 ? 1 : (ti == 1 ? 0 : 2);
                const int s = it % S::STAGES;
                if (!mbar_wait(&empty[s], ((it / S::STAGES) & 1) ^ 1, a.err, 51)) {
                  ok = false;
                  break;
                }
                mbar_expect_tx(&full[s], S::A_BYTES);
                // frames ts + 128 m + (tap - 1) d .. +127 (zero outside the row)
                tma_load_3d(smem + s * S::A_BYTES, &tmX, &full[s], kb * S::BK,
                            ts + m * 128 + (tap - 1) * a.dil, row);
              }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc1 = idesc_tf32(128, S::KS);
      constexpr uint32_t idesc2 = idesc_tf32(128, S::NCH);
      bool ok = (!conv1 || mbar_wait(&w1_full, 0, a.err, 52)) &&
                (!conv2 || mbar_wait(&w2_full, 0, a.err, 53));
      uint32_t it = 0, u = 0;
      // conv2 of item `pend` (-1: none) is issued once its g is in TMEM
      int pend = -1, cur = 0;
      bool g_in = false;
      auto conv2_progress = [&](bool block) {
        if (pend < 0 || !ok) return;
        if (!g_in) {
          if (block) {
            if (!mbar_wait(&g_ready, pend & 1, a.err, 54)) {
              ok = false;
              return;
            }
          } else if (!mbar_test(&g_ready, pend & 1)) {
            return;
          }
          g_in = true;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        }
        while (cur < 3 * S::NCHUNK) {
          const int j = u % S::NB2;
          const uint32_t par = ((u / S::NB2) & 1) ^ 1;
          if (block) {
            if (!mbar_wait(&d2_empty[j], par, a.err, 55)) {
              ok = false;
              return;
            }
          } else if (!mbar_test(&d2_empty[j], par)) {
            return;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const int m = cur / S::NCHUNK, ch = cur % S::NCHUNK;
          const uint32_t wb = smem_u32(smem + S::OFF_W2 + ch * S::NCH * 128);
#pragma unroll
          for (int kk = 0; kk < S::KS / 8; ++kk)
            umma_tf32_ta(tmem + S::TM_D2 + S::NCH * j, tmem + S::TM_G + 32 * m + 8 * kk,
                         umma_desc_k(wb + kk * 32, 128), idesc2, kk != 0);
          umma_commit(&d2_full[j]);
          ++u;
          ++cur;
        }
        pend = -1;
      };
      int ri = 0;
      if (conv1) {
        for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++ri) {
          // D1 is free once the epilogue has read the previous item's conv1
          if (!mbar_wait(&d1_empty, (ri & 1) ^ 1, a.err, 56)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          for (int m = 0; m < 3 && ok; ++m)
            for (int ti = 0; ti < 3 && ok; ++ti)
              for (int kb = 0; kb < S::KB; ++kb, ++it) {
                const int tap = ti == 0 ? 1 : (ti == 1 ? 0 : 2);  // the producer's order
                conv2_progress(false);
                const int s = it % S::STAGES;
                if (!ok || !mbar_wait(&full[s], (it / S::STAGES) & 1, a.err, 57)) {
                  ok = false;
                  break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t xa = smem_u32(smem + s * S::A_BYTES);
                const uint32_t wa = smem_u32(smem + S::OFF_W1 + (tap * S::KB + kb) * S::W1_TILE);
#pragma unroll
                for (int j = 0; j < S::BK / 8; ++j)
                  umma_tf32(tmem + S::TM_D1 + 32 * m, umma_desc_k(xa + j * 32, 128),
                            umma_desc_k(wa + j * 32, 128), idesc1, (kb | ti | j) != 0);
                umma_commit(&empty[s]);
              }
          if (!ok) break;
          umma_commit(&d1_full);
          conv2_progress(true);  // the rest of the previous item's conv2
          if (conv2) {
            pend = ri;
            cur = 0;
            g_in = false;
          }
        }
        conv2_progress(true);
      } else if (conv2) {
        // DC_OUT: conv2 alone, item by item
        for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++ri) {
          pend = ri;
          cur = 0;
          g_in = false;
          conv2_progress(true);
        }
      }
    }
  } else if (warp >= 4) {
    // ---------------- epilogue: warps 4-15 ----------------
    // TMEM lane quarter q = warp % 4 (frames 32q .. 32q+31 of a block); b:
    // the block of this warp's frames for y and g, its third of the columns
    // of each 96-column conv2 chunk for the output
    const int e = warp - 4, q = warp % 4, b = e / 4;
    const int r = q * 32 + lane;
    const int p = 128 * b + r;  // this thread's frame (y, g)
    const int et = threadIdx.x - kEpiBase;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    float4* chan = reinterpret_cast<float4*>(smem + S::OFF_CH);
    for (int c = et; c < C; c += kEpiThreads) {
      chan[2 * c] = make_float4(a.b2[2 * c], a.b2[2 * c + 1], a.n2w[c], a.n2w[c + C]);
      chan[2 * c + 1] = make_float4(a.n2b[c], a.n2b[c + C], a.gamma[c], 0.f);
    }
    epi_bar();
    const double ic1 = 1.0 / ((double)S::HID * T), ic2 = 1.0 / (2.0 * C * T);
    // the row's moments from its tiles' partials, summed by one warp in a
    // fixed order; every epilogue thread gets them
    auto row_sum = [&](const double* part, int row, double& s, double& q2) {
      if (warp == kEpiBase / 32) {
        double ls = 0.0, lq = 0.0;
        for (int t = lane; t < a.tiles; t += 32) {
          ls += part[2 * ((int64_t)row * a.tiles + t)];
          lq += part[2 * ((int64_t)row * a.tiles + t) + 1];
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
          ls += __shfl_xor_sync(0xffffffffu, ls, o);
          lq += __shfl_xor_sync(0xffffffffu, lq, o);
        }
        if (lane == 0) {
          red[0] = ls;
          red[1] = lq;
        }
      }
      epi_bar();
      s = red[0];
      q2 = red[1];
      epi_bar();
    };
    uint32_t u = 0;
    int ri = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < items; w += gridDim.x, ++ri) {
      const int row = w / a.tiles, ts = (w - row * a.tiles) * kTileStride - 2;
      // local frame i = 128 m + r is frame ts + i; owned: 2 <= i < 382, inside the row
      auto owned = [&](int i) { return i >= 2 && i < 382 && ts + i < T; };
      const bool mine = owned(p);
      float yh[S::HID];  // y of frame p by hidden channel
      double s, sq;
      if (conv1) {
        // ---- y = conv1 + bias, straight from block b's accumulator ----
        if (ok && !mbar_wait(&d1_full, ri & 1, a.err, 58)) ok = false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        {
          uint32_t d1[32];
          __syncwarp();
          tmem_ld32_nw(tmem + lane_base + S::TM_D1 + 32 * b, d1);
          tmem_ld_wait<32>(d1);
          // D1 is read out: the next item's conv1 may overwrite it
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          mbar_arrive(&d1_empty);
#pragma unroll
          for (int h = 0; h < S::HID; ++h) yh[h] = __uint_as_float(d1[h]) + k.b1[h];
        }
        float fs = 0.f, fq = 0.f;
#pragma unroll
        for (int h = 0; h < S::HID; ++h) {
          fs += yh[h];
          fq = fmaf(yh[h], yh[h], fq);
        }
        s = mine ? fs : 0.f;
        sq = mine ? fq : 0.f;
        if (mode == DC_STATS1) {
          // y of the owned frames for the later launches
          if (mine) {
            float4* yp = reinterpret_cast<float4*>(a.y + ((int64_t)row * T + ts + p) * S::YS);
#pragma unroll
            for (int c = 0; c < S::YS / 4; ++c)
              yp[c] = make_float4(yh[4 * c], yh[4 * c + 1], yh[4 * c + 2], yh[4 * c + 3]);
          }
          epi_sum2(s, sq, red);
          if (threadIdx.x == kEpiBase) {
            a.part1[2 * (int64_t)w] = s;
            a.part1[2 * (int64_t)w + 1] = sq;
          }
          continue;
        }
        epi_sum2(s, sq, red);
      } else {
        // DC_OUT: y of the owned frames from the buffer
        if (mine) {
          const float4* yp = reinterpret_cast<const float4*>(a.y + ((int64_t)row * T + ts + p) * S::YS);
#pragma unroll
          for (int c = 0; c < S::YS / 4; ++c) {
            const float4 v = yp[c];
            yh[4 * c] = v.x;
            yh[4 * c + 1] = v.y;
            yh[4 * c + 2] = v.z;
            yh[4 * c + 3] = v.w;
          }
        } else {
#pragma unroll
          for (int h = 0; h < S::HID; ++h) yh[h] = 0.f;
        }
        row_sum(a.part1, row, s, sq);
      }
      // ---- g = GELU(GN1(y)) of frame p; conv2's A operand, into TMEM ----
      float mean, inv;
      norm_of(s, sq, ic1, mean, inv);
      float ga[S::ACT];  // g by conv2 input (hidden channels, then the bias input 1)
#pragma unroll
      for (int h = 0; h < S::HID; ++h) {
        const float scale = inv * k.n1w[h];
        ga[h] = mine ? gelu_tc(yh[h] * scale + (k.n1b[h] - mean * scale)) : 0.f;
      }
      ga[S::HID] = 1.0f;
      if (conv2) {
        float gs[S::KS];
#pragma unroll
        for (int j = 0; j < S::KS; ++j) gs[j] = j < S::HID ? ga[j] : (j == S::BIAS ? 1.0f : 0.f);
        __syncwarp();
        tmem_st32(tmem + lane_base + S::TM_G + 32 * b, gs);
        tmem_st_wait();
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        mbar_arrive(&g_ready);
      }

      // ---- moments of z: the sums of v.g and g'Mg over the owned frames ----
      if (mode == DC_OUT) {
        row_sum(a.part2, row, s, sq);
      } else {
        float l = 0.f, qf = 0.f;
        if (mine) {
#pragma unroll
          for (int i = 0, idx = 0; i < S::ACT; ++i) {
            l = fmaf(k.v[i], ga[i], l);
            float t = 0.f;
#pragma unroll
            for (int j = i; j < S::ACT; ++j, ++idx) t = fmaf(k.m[idx], ga[j], t);
            qf = fmaf(ga[i], t, qf);
          }
        }
        s = l;
        sq = qf;
        epi_sum2(s, sq, red);
      }
      float mean2, inv2;
      norm_of(s, sq, ic2, mean2, inv2);
      // GN2 with LayerScale folded in: gamma * value = z_v * a + b, gate = z_g * c + d
      float4* aff = reinterpret_cast<float4*>(smem + S::OFF_AFF);
      for (int c = et; c < C; c += kEpiThreads) {
        const float4 t0 = chan[2 * c], t1 = chan[2 * c + 1];
        const float vs = inv2 * t0.z, gs = inv2 * t0.w;
        aff[c] = make_float4(t1.z * vs, t1.z * (t1.x - mean2 * vs), gs, t1.y - mean2 * gs);
      }
      epi_bar();

      // ---- conv2, the output: x += gamma * GLU(GN2(z)) ----
      // chunk cc = (block, 48-channel group); the residual of the next chunk
      // is loaded from HBM while this one's conv2 completes and is stored
      // (16 channels = 64 bytes at a 64-byte-aligned offset: two 32-byte accesses)
      auto load_res = [&](int cc, float* dst) {
        const int pm = (cc / S::NCHUNK) * 128 + r;
        if (ok && owned(pm)) {
          const float* xp =
              a.x + ((int64_t)row * T + ts + pm) * C + (cc % S::NCHUNK) * (S::NCH / 2) + 16 * b;
          ld_global8(xp, dst);
          ld_global8(xp + 8, dst + 8);
        }
      };
      float nxt[16];
      load_res(0, nxt);
#pragma unroll 1
      for (int cc = 0; cc < 3 * S::NCHUNK; ++cc) {
          const int m = cc / S::NCHUNK, ch = cc % S::NCHUNK;
          const int j = u % S::NB2;
          const int pm = m * 128 + r;
          const bool own = owned(pm);
          const int c0 = ch * (S::NCH / 2) + 16 * b;  // this thread's 16 channels
          float* xp = a.x + ((int64_t)row * T + (own ? ts + pm : 0)) * C + c0;
          float o[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = nxt[i];
          if (cc + 1 < 3 * S::NCHUNK) load_res(cc + 1, nxt);
          if (ok && !mbar_wait(&d2_full[j], (u / S::NB2) & 1, a.err, 59)) ok = false;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          uint32_t zr[32];
          __syncwarp();
          tmem_ld32_nw(tmem + lane_base + S::TM_D2 + S::NCH * j + 32 * b, zr);
          tmem_ld_wait<32>(zr);
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          mbar_arrive(&d2_empty[j]);
          ++u;
          if (ok && own) {
#pragma unroll
            for (int kk = 0; kk < 16; ++kk) {
              const float4 f = aff[c0 + kk];
              const float value = fmaf(__uint_as_float(zr[2 * kk]), f.x, f.y);
              const float gate = fmaf(__uint_as_float(zr[2 * kk + 1]), f.z, f.w);
              o[kk] += glu_tc(value, gate);
              if (a.round_out) o[kk] = round_tf32(o[kk]);
            }
            st_global8(xp, o);
            st_global8(xp + 8, o + 8);
          }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

// DC_STATS2 as a plain kernel: one 384-thread block per tile, thread p on
// local frame p, the same arithmetic in the same order as the persistent
// kernel's epilogue warps (thread p there is epilogue thread p): the row's
// y moments summed over its tiles by one warp, g = GELU(GroupNorm1(y)), the
// quadratic form for the moments of z, and the block sum (lanes, then warps
// in order) into part2. Blocks run many per SM, so the pass moves at the
// speed of its loads instead of one tile per SM at a time.
template <int C>
__global__ void __launch_bounds__(kEpiThreads)
    dconv_tc_stats2_kernel(const DConvArgs a, const __grid_constant__ DcConst<C> k) {
  using S = DcTc<C>;
  __shared__ double red[2 * kEpiWarps];
  const int w = blockIdx.x, p = threadIdx.x, warp = p / 32, lane = p % 32;
  const int T = a.T;
  const int row = w / a.tiles, ts = (w - row * a.tiles) * kTileStride - 2;
  const bool mine = p >= 2 && p < 382 && ts + p < T;
  float yh[S::HID];
  if (mine) {
    const float4* yp = reinterpret_cast<const float4*>(a.y + ((int64_t)row * T + ts + p) * S::YS);
#pragma unroll
    for (int c = 0; c < S::YS / 4; ++c) {
      const float4 v = yp[c];
      const float t4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (4 * c + i < S::HID) yh[4 * c + i] = t4[i];
    }
  } else {
#pragma unroll
    for (int h = 0; h < S::HID; ++h) yh[h] = 0.f;
  }
  // the row's y moments over its tiles, in tile order per lane, then the lanes
  if (warp == 0) {
    double ls = 0.0, lq = 0.0;
    for (int t = lane; t < a.tiles; t += 32) {
      ls += a.part1[2 * ((int64_t)row * a.tiles + t)];
      lq += a.part1[2 * ((int64_t)row * a.tiles + t) + 1];
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      ls += __shfl_xor_sync(0xffffffffu, ls, o);
      lq += __shfl_xor_sync(0xffffffffu, lq, o);
    }
    if (lane == 0) {
      red[0] = ls;
      red[1] = lq;
    }
  }
  __syncthreads();
  const double s1 = red[0], q1 = red[1];
  __syncthreads();
  const double ic1 = 1.0 / ((double)S::HID * T);
  float mean, inv;
  norm_of(s1, q1, ic1, mean, inv);
  float ga[S::ACT];
#pragma unroll
  for (int h = 0; h < S::HID; ++h) {
    const float scale = inv * k.n1w[h];
    ga[h] = mine ? gelu_tc(yh[h] * scale + (k.n1b[h] - mean * scale)) : 0.f;
  }
  ga[S::HID] = 1.0f;
  float l = 0.f, qf = 0.f;
  if (mine) {
#pragma unroll
    for (int i = 0, idx = 0; i < S::ACT; ++i) {
      l = fmaf(k.v[i], ga[i], l);
      float t = 0.f;
#pragma unroll
      for (int j = i; j < S::ACT; ++j, ++idx) t = fmaf(k.m[idx], ga[j], t);
      qf = fmaf(ga[i], t, qf);
    }
  }
  double s = l, q = qf;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    q += __shfl_xor_sync(0xffffffffu, q, o);
  }
  if (lane == 0) {
    red[2 * warp] = s;
    red[2 * warp + 1] = q;
  }
  __syncthreads();
  if (p == 0) {
    s = 0.0;
    q = 0.0;
#pragma unroll
    for (int ww = 0; ww < kEpiWarps; ++ww) {
      s += red[2 * ww];
      q += red[2 * ww + 1];
    }
    a.part2[2 * (int64_t)w] = s;
    a.part2[2 * (int64_t)w + 1] = q;
  }
}

template <int C>
bool launch_c(const DConvArgs& a, cudaStream_t s) {
  using S = DcTc<C>;
  const CUtensorMapSwizzle swz = S::BK == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUtensorMap mx, m1, m1lo, m2, m2lo;
  bool ok;
  {
    const cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)a.T, (cuuint64_t)a.rows};
    const cuuint64_t str[2] = {(cuuint64_t)C * 4, (cuuint64_t)a.T * C * 4};
    const cuuint32_t box[3] = {(cuuint32_t)S::BK, 128, 1};
    ok = make_tensor_map(&mx, a.x, 3, dims, str, box, swz);
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)(3 * C), (cuuint64_t)a.w1_npad};
    const cuuint64_t str[1] = {(cuuint64_t)(3 * C) * 4};
    const cuuint32_t box[2] = {(cuuint32_t)S::BK, (cuuint32_t)S::HP};
    ok = ok && make_tensor_map(&m1, a.w1_tc, 2, dims, str, box, swz);
    ok = ok && make_tensor_map(&m1lo, a.w1_tc_lo, 2, dims, str, box, swz);
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)S::HP, (cuuint64_t)a.w2_npad};
    const cuuint64_t str[1] = {(cuuint64_t)S::HP * 4};
    const cuuint32_t box[2] = {(cuuint32_t)S::HP, (cuuint32_t)(2 * C)};
    ok = ok && make_tensor_map(&m2, a.w2_tc, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_64B);
    ok = ok && make_tensor_map(&m2lo, a.w2_tc_lo, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_64B);
  }
  if (!ok) return false;
  DcConst<C> k;
  const float* src = a.zq_host;
  for (int i = 0; i < S::ACT; ++i) k.v[i] = *src++;
  for (int i = 0; i < S::NQ; ++i) k.m[i] = *src++;
  for (int i = 0; i < S::HID; ++i) k.b1[i] = *src++;
  for (int i = 0; i < S::HID; ++i) k.n1w[i] = *src++;
  for (int i = 0; i < S::HID; ++i) k.n1b[i] = *src++;
  static PerDevice configured;
  if (configured.first()) {
    cudaFuncSetAttribute(dconv_tc_row_kernel<C, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         S::SMEM);
    cudaFuncSetAttribute(dconv_tc_row_kernel<C, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         S::SMEM);
  }
  auto row_kernel = a.single ? dconv_tc_row_kernel<C, false> : dconv_tc_row_kernel<C, true>;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int items = a.rows * a.tiles;
  const int grid = items < sms ? items : sms;
  if (a.tiles == 1) {
    row_kernel<<<grid, kThreads, S::SMEM, s>>>(mx, m1, m1lo, m2, m2lo, a, k, DC_ROW);
  } else {
    row_kernel<<<grid, kThreads, S::SMEM, s>>>(mx, m1, m1lo, m2, m2lo, a, k, DC_STATS1);
    dconv_tc_stats2_kernel<C><<<items, kEpiThreads, 0, s>>>(a, k);
    row_kernel<<<grid, kThreads, S::SMEM, s>>>(mx, m1, m1lo, m2, m2lo, a, k, DC_OUT);
  }
  return true;
}

// C = 192: single-pass only (the split variant's low parts do not fit in
// shared memory beside the weights).
bool launch_wide(const DConvArgs& a, cudaStream_t s) {
  constexpr int C = 192;
  using S = DcTc<C>;
  CUtensorMap mx, m1, m2;
  bool ok;
  {
    const cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)a.T, (cuuint64_t)a.rows};
    const cuuint64_t str[2] = {(cuuint64_t)C * 4, (cuuint64_t)a.T * C * 4};
    const cuuint32_t box[3] = {(cuuint32_t)S::BK, 128, 1};
    ok = make_tensor_map(&mx, a.x, 3, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  {
    // rows = hidden channels (zero beyond HID), columns tap * C + channel
    const cuuint64_t dims[2] = {(cuuint64_t)(3 * C), (cuuint64_t)a.w1_npad};
    const cuuint64_t str[1] = {(cuuint64_t)(3 * C) * 4};
    const cuuint32_t box[2] = {(cuuint32_t)S::BK, (cuuint32_t)S::KS};
    ok = ok && make_tensor_map(&m1, a.w1_tc, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  {
    // rows = conv2 output columns, 32 K slots each; two boxes of C rows
    const cuuint64_t dims[2] = {(cuuint64_t)S::KS, (cuuint64_t)a.w2_npad};
    const cuuint64_t str[1] = {(cuuint64_t)S::KS * 4};
    const cuuint32_t box[2] = {(cuuint32_t)S::KS, (cuuint32_t)C};
    ok = ok && make_tensor_map(&m2, a.w2_tc, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (!ok) return false;
  DcConst<C> k;
  const float* src = a.zq_host;
  for (int i = 0; i < S::ACT; ++i) k.v[i] = *src++;
  for (int i = 0; i < S::NQ; ++i) k.m[i] = *src++;
  for (int i = 0; i < S::HID; ++i) k.b1[i] = *src++;
  for (int i = 0; i < S::HID; ++i) k.n1w[i] = *src++;
  for (int i = 0; i < S::HID; ++i) k.n1b[i] = *src++;
  static PerDevice configured;
  if (configured.first())
    cudaFuncSetAttribute(dconv_tc_wide_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         S::SMEM);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int items = a.rows * a.tiles;
  const int grid = items < sms ? items : sms;
  if (a.tiles == 1) {
    dconv_tc_wide_kernel<C><<<grid, kThreads, S::SMEM, s>>>(mx, m1, m2, a, k, DC_ROW);
  } else {
    dconv_tc_wide_kernel<C><<<grid, kThreads, S::SMEM, s>>>(mx, m1, m2, a, k, DC_STATS1);
    dconv_tc_stats2_kernel<C><<<items, kEpiThreads, 0, s>>>(a, k);
    dconv_tc_wide_kernel<C><<<grid, kThreads, S::SMEM, s>>>(mx, m1, m2, a, k, DC_OUT);
  }
  return true;
}

}  // namespace

bool dconv_tc_supported(int C, int T, bool single) {
  return (C == 48 || C == 96 || (C == 192 && single)) && T > 0 && tensor_map_encoder() != nullptr;
}

int dconv_tc_tiles(int T) { return (T + kTileStride - 1) / kTileStride; }

int dconv_tc_ystride(int C) { return (C / 8 + 3) / 4 * 4; }

int dconv_tc_const_floats(int C) {
  const int hid = C / 8, act = hid + 1;
  return act + act * (act + 1) / 2 + 3 * hid;
}

bool launch_dconv_tc(const DConvArgs& a, cudaStream_t s) {
  if (!dconv_tc_supported(a.C, a.T, a.single != 0) || a.dil < 1 || a.dil > 2 || !a.w1_tc ||
      !a.w1_tc_lo || !a.w2_tc || !a.w2_tc_lo || !a.zq_host || a.w1_npad < (a.C == 192 ? 32 : 16) ||
      a.w2_npad < 2 * a.C || a.tiles != dconv_tc_tiles(a.T) ||
      (a.tiles > 1 && (!a.part1 || !a.part2 || !a.y)) || (int64_t)a.rows * a.tiles > INT32_MAX)
    return false;
  switch (a.C) {
    case 48: return launch_c<48>(a, s);
    case 96: return launch_c<96>(a, s);
    case 192: return launch_wide(a, s);
    default: return false;
  }
}

}  // namespace dmx
