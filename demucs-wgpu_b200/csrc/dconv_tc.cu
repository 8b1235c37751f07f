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
//    (frames outside the row are TMA's zero fill) and the conv1 weights; warps
//    2-5 write each tile's low part (x - tf32(x)); warp 1 issues the MMAs.
//  * warps 6-13 read the conv1 accumulators out of TMEM (which frees them for
//    the next item's conv1), combine the taps through shared memory, reduce
//    the moments of y, and write g (and its low part) to shared memory as the
//    A operand of conv2.
//  * the moments of z come from g alone. With w_c the conv2 weights of output
//    column c (its bias on a constant-1 input slot), sum_c z_c = v.g and
//    sum_c z_c^2 = g'Mg for v = sum_c w_c and M = sum_c w_c w_c', constants
//    computed on the host; so z leaves TMEM once, for the output.
//  * conv2 against the resident conv2 weights (N = 96 columns per MMA) is
//    issued between the next item's conv1 stages; warps 6-13 combine it with
//    the residual straight into x.
//
// K slots: hidden channel h < HID/2 sits at slot h, the others at slot
// 8 + h - HID/2, so each epilogue half (slots 0-7, 8-15) carries half of the
// GroupNorm1 + GELU work; slot 15 is the constant 1 that carries conv2's bias.
// The host packs the tensor-core weight copies in this order.
//
// Precision: 3xTF32 (lo*hi + hi*lo + hi*hi). The high part of an fp32 operand
// is the operand itself (the tensor core reads it truncated to tf32); the low
// part is x - trunc_tf32(x), exact in fp32. The weights' high parts are
// rounded to nearest on the host and their residuals stored beside them. The
// result agrees with fp32 arithmetic to ~1e-6 relative; moments are summed in
// f64 as the reference's GroupNorm does. No load uses cluster multicast.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace dmx {

namespace {

constexpr int kThreads = 448;  // w0 TMA, w1 MMA, w2-5 converter, w6-13 epilogue
constexpr int kEpiThreads = 256;
constexpr int kEpiWarps = 8;

template <int C>
struct DcTc {
  static constexpr int HID = C / 8;
  static constexpr int JA = HID / 2;              // hidden channels per epilogue half
  static constexpr int ACT = HID + 1;             // conv2 K slots in use (hidden, bias)
  static constexpr int NQ = ACT * (ACT + 1) / 2;  // packed upper triangle of M
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
  static constexpr int B_BYTES = N1 * BK * 4;     // one 16-row box per tap
  static constexpr int STAGE = 2 * A_BYTES + 2 * B_BYTES;  // A | A_lo | B | B_lo
  static constexpr int STAGES = 3;
  static constexpr int TX = A_BYTES + 2 * B_BYTES;         // bytes landed by TMA per stage
  static constexpr int G_BYTES = 128 * HP * 4;             // one 128-frame block of g
  static constexpr int W2_BYTES = 2 * C * HP * 4;
  // g hi [3] | g lo [3]; before g is formed the same 48 KB holds the tap-0
  // and tap-2 outputs of all 384 frames for the neighbour exchange
  static constexpr int OFF_G = STAGES * STAGE;
  static constexpr int OFF_W2 = OFF_G + 6 * G_BYTES;       // w2 hi | w2 lo
  static constexpr int OFF_CH = OFF_W2 + 2 * W2_BYTES;     // per-channel constants [C][8]
  static constexpr int OFF_AFF = OFF_CH + C * 32;          // per-item GN2 affine [C] float4
  // ALL: the epilogue threads' residual chunks, prefetched with cp.async
  // while the moments of z are reduced: [18 chunks][256 threads][16 B]
  static constexpr int OFF_RES = OFF_AFF + C * 16;
  static constexpr int RES_BYTES = ALL ? 18 * 256 * 16 : 0;
  static constexpr int SMEM = OFF_RES + RES_BYTES + 1024;
  static_assert(2 * C % NCH == 0 && HID % 2 == 0 && JA <= 7 && SMEM <= 227 * 1024, "shape");
  // K slot of the i-th input of conv2 (the hidden channels, then the bias)
  static constexpr int act_slot(int i) { return i < JA ? i : (i < HID ? 8 + i - JA : 15); }
};

// The moments of z as functions of g (v and M above), over the active K slots
// in act_slot order.
template <int C>
struct DcZq {
  float v[DcTc<C>::ACT];
  float m[DcTc<C>::NQ];  // upper triangle by rows, off-diagonal entries doubled
};

__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

DMX_DEVICE float trunc_tf32(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

DMX_DEVICE void epi_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

DMX_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Sum of (s, q) over the 256 epilogue threads, fixed order; all get the result.
DMX_DEVICE void epi_sum2(double& s, double& q, double* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    q += __shfl_xor_sync(0xffffffffu, q, o);
  }
  const int e = threadIdx.x / 32 - 6;
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
// three launches, each recomputing conv1 from x: DC_STATS1 (moments of y per
// tile), DC_STATS2 (moments of z per tile, with the row's y moments summed
// over its tiles in a fixed order) and DC_OUT (the output).
enum DcMode : int { DC_ROW = 0, DC_STATS1 = 1, DC_STATS2 = 2, DC_OUT = 3 };
constexpr int kTileStride = 380;

template <int C>
__global__ void __launch_bounds__(kThreads, 1)
    dconv_tc_row_kernel(const __grid_constant__ CUtensorMap tmX,
                        const __grid_constant__ CUtensorMap tmW1,
                        const __grid_constant__ CUtensorMap tmW1lo,
                        const __grid_constant__ CUtensorMap tmW2,
                        const __grid_constant__ CUtensorMap tmW2lo, const DConvArgs a,
                        const __grid_constant__ DcZq<C> zq, int mode) {
  using S = DcTc<C>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ __align__(8) uint64_t full[S::STAGES], empty[S::STAGES], conv[S::STAGES];
  __shared__ __align__(8) uint64_t w2_full, d1_full, d1_empty, g_ready, d2_full[2], d2_empty[2];
  __shared__ uint32_t tmem_slot;
  __shared__ double red[2 * kEpiWarps];

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (a.err && *reinterpret_cast<volatile int*>(a.err) != 0) return;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], 128);
    }
    mbar_init(&w2_full, 1);
    mbar_init(&d1_full, 1);
    mbar_init(&d1_empty, kEpiThreads);
    mbar_init(&g_ready, kEpiThreads);
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
  const bool conv2 = mode == DC_ROW || mode == DC_OUT;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      if (conv2) {
        mbar_expect_tx(&w2_full, 2 * S::W2_BYTES);
        tma_load_2d(smem + S::OFF_W2, &tmW2, &w2_full, 0, 0);
        tma_load_2d(smem + S::OFF_W2 + S::W2_BYTES, &tmW2lo, &w2_full, 0, 0);
      }
      uint32_t it = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < items && ok; w += gridDim.x) {
        const int row = w / a.tiles, ts = (w - row * a.tiles) * kTileStride - 2;
        for (int m = 0; m < 3 && ok; ++m) {
          for (int kb = 0; kb < S::KB; ++kb, ++it) {
            const int s = it % S::STAGES;
            if (!mbar_wait(&empty[s], ((it / S::STAGES) & 1) ^ 1, a.err, 31)) {
              ok = false;
              break;
            }
            unsigned char* st = smem + s * S::STAGE;
            mbar_expect_tx(&full[s], S::TX);
            const int c0 = kb * S::BK;
            // frames ts + 128 m .. +127 (zero outside the row), channels c0 .. c0+BK
            tma_load_3d(st, &tmX, &full[s], c0, ts + m * 128, row);
            // B rows 16k .. 16k+15: tap k's weights for these channels
            for (int tap = 0; tap < 3; ++tap) {
              unsigned char* b = st + 2 * S::A_BYTES + tap * S::HP * S::BK * 4;
              tma_load_2d(b, &tmW1, &full[s], tap * C + c0, 0);
              tma_load_2d(b + S::B_BYTES, &tmW1lo, &full[s], tap * C + c0, 0);
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
      bool ok = !conv2 || mbar_wait(&w2_full, 0, a.err, 32);
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
        for (int k = 0; k < 2; ++k) {
          const uint64_t gh = umma_desc_k(g_hi + k * 32, 64);
          const uint64_t wh = umma_desc_k(w_hi + k * 32, 64);
          umma_tf32(d, umma_desc_k(g_lo + k * 32, 64), wh, idesc2, k != 0);
          umma_tf32(d, gh, umma_desc_k(w_lo + k * 32, 64), idesc2, 1);
          umma_tf32(d, gh, wh, idesc2, 1);
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
            const int s = it % S::STAGES;
            if (!ok || !mbar_wait(&conv[s], (it / S::STAGES) & 1, a.err, 33)) {
              ok = false;
              break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a_hi = smem_u32(smem + s * S::STAGE);
            const uint32_t a_lo = a_hi + S::A_BYTES;
            const uint32_t b_hi = a_hi + 2 * S::A_BYTES;
            const uint32_t b_lo = b_hi + S::B_BYTES;
#pragma unroll
            for (int j = 0; j < S::BK / 8; ++j) {
              const uint64_t ah = umma_desc_k(a_hi + j * 32, S::BK * 4);
              const uint64_t bh = umma_desc_k(b_hi + j * 32, S::BK * 4);
              umma_tf32(d, umma_desc_k(a_lo + j * 32, S::BK * 4), bh, idesc1, (kb | j) != 0);
              umma_tf32(d, ah, umma_desc_k(b_lo + j * 32, S::BK * 4), idesc1, 1);
              umma_tf32(d, ah, bh, idesc1, 1);
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
    }
  } else if (warp < 6) {
    // ---------------- converter: the low part of each x tile row ----------------
    const int r = threadIdx.x - 64;
    // visit the 16-byte chunks in swizzle order: 8 lanes, 8 bank groups
    const int swz = S::BK == 32 ? (r & 7) : ((r >> 1) & 3);
    uint32_t it = 0;
    bool live = true;
    for (int w = blockIdx.x; w < items; w += gridDim.x)
      for (int m = 0; m < 3; ++m)
        for (int kb = 0; kb < S::KB; ++kb, ++it) {
          const int s = it % S::STAGES;
          if (live && !mbar_wait(&full[s], (it / S::STAGES) & 1, a.err, 36)) live = false;
          if (live) {
            const float4* x4 = reinterpret_cast<const float4*>(smem + s * S::STAGE + r * S::BK * 4);
            float4* lo4 = reinterpret_cast<float4*>(smem + s * S::STAGE + S::A_BYTES + r * S::BK * 4);
#pragma unroll
            for (int qq = 0; qq < S::BK / 4; ++qq) {
              const int q = qq ^ swz;
              const float4 x = x4[q];
              lo4[q] = make_float4(x.x - trunc_tf32(x.x), x.y - trunc_tf32(x.y),
                                   x.z - trunc_tf32(x.z), x.w - trunc_tf32(x.w));
            }
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          mbar_arrive(&conv[s]);
        }
  } else {
    // ---------------- epilogue: warps 6-13 ----------------
    // TMEM lane quarter q (rows 32q .. 32q+31 of each 128-frame block); half
    // hh takes K slots 8hh .. 8hh+7 (conv1) and columns 48hh.. (conv2)
    const int e = warp - 6, q = warp % 4, hh = e / 4;
    const int r = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    // hidden channels hh*JA + j sit in slots 8hh + j, j < JA
    float b1[S::JA], n1w[S::JA], n1b[S::JA];
#pragma unroll
    for (int j = 0; j < S::JA; ++j) {
      const int h = hh * S::JA + j;
      b1[j] = a.b1[h];
      n1w[j] = a.n1w[h];
      n1b[j] = a.n1b[h];
    }
    // per channel c: conv2 bias (value, gate), GN2 weight and bias (value,
    // gate), LayerScale
    float4* chan = reinterpret_cast<float4*>(smem + S::OFF_CH);
    for (int c = threadIdx.x - 192; c < C; c += kEpiThreads) {
      chan[2 * c] = make_float4(a.b2[2 * c], a.b2[2 * c + 1], a.n2w[c], a.n2w[c + C]);
      chan[2 * c + 1] = make_float4(a.n2b[c], a.n2b[c + C], a.gamma[c], 0.f);
    }
    epi_bar();
    const double ic1 = 1.0 / ((double)S::HID * T), ic2 = 1.0 / (2.0 * C * T);
    // the row's moments from its tiles' partials, summed by one warp in a
    // fixed order; every epilogue thread gets them
    auto row_sum = [&](const double* part, int row, double& s, double& q2) {
      if (threadIdx.x < 192 + 32) {
        double ls = 0.0, lq = 0.0;
        for (int k = lane; k < a.tiles; k += 32) {
          ls += part[2 * ((int64_t)row * a.tiles + k)];
          lq += part[2 * ((int64_t)row * a.tiles + k) + 1];
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
      // ---- y = conv1 + bias, its moments, g into shared memory ----
      // D1 holds Y_k = W_k x (k = tap) per frame; y[p] = Y_0[p-d] + Y_1[p] +
      // Y_2[p+d]. Y_0 and Y_2 go through shared memory to the neighbours
      // (frames 384 x 16 slots each, 64-byte rows with the 64-byte swizzle).
      if (ok && !mbar_wait(&d1_full, ri & 1, a.err, 37)) ok = false;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      float* x0s = reinterpret_cast<float*>(smem + S::OFF_G);
      float* x2s = x0s + 384 * 16;
      constexpr int NC = (S::JA + 3) / 4;  // 16-byte chunks of a half that hold channels
      float y[3][8];
      {
        uint32_t d1[3][3][8];
        __syncwarp();
#pragma unroll
        for (int m = 0; m < 3; ++m)
#pragma unroll
          for (int tap = 0; tap < 3; ++tap)
            tmem_ld8_nw(tm_d1 + lane_base + 64 * m + 16 * tap + 8 * hh, d1[m][tap]);
        tmem_ld_wait<72>(&d1[0][0][0]);
        // D1 is read out: the next item's conv1 may overwrite it
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        mbar_arrive(&d1_empty);
#pragma unroll
        for (int m = 0; m < 3; ++m) {
          const int p = 128 * m + r;
#pragma unroll
          for (int j = 0; j < 8; ++j) y[m][j] = __uint_as_float(d1[m][1][j]);
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            const int off = p * 16 + (((2 * hh + c) ^ ((p >> 1) & 3)) << 2);
            *reinterpret_cast<uint4*>(x0s + off) = make_uint4(
                d1[m][0][4 * c], d1[m][0][4 * c + 1], d1[m][0][4 * c + 2], d1[m][0][4 * c + 3]);
            *reinterpret_cast<uint4*>(x2s + off) = make_uint4(
                d1[m][2][4 * c], d1[m][2][4 * c + 1], d1[m][2][4 * c + 2], d1[m][2][4 * c + 3]);
          }
        }
      }
      epi_bar();
      float fs1 = 0.f, fq1 = 0.f;
#pragma unroll
      for (int m = 0; m < 3; ++m) {
        const int p = 128 * m + r;
        const int pl = p - a.dil, pr = p + a.dil;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          float4 l = make_float4(0.f, 0.f, 0.f, 0.f), rgt = l;
          if (pl >= 0)
            l = *reinterpret_cast<const float4*>(x0s + pl * 16 + (((2 * hh + c) ^ ((pl >> 1) & 3)) << 2));
          if (pr < 384)
            rgt = *reinterpret_cast<const float4*>(x2s + pr * 16 + (((2 * hh + c) ^ ((pr >> 1) & 3)) << 2));
          y[m][4 * c] += l.x + rgt.x;
          y[m][4 * c + 1] += l.y + rgt.y;
          y[m][4 * c + 2] += l.z + rgt.z;
          y[m][4 * c + 3] += l.w + rgt.w;
        }
        const bool valid = owned(p);
#pragma unroll
        for (int j = 0; j < S::JA; ++j) {
          y[m][j] += b1[j];
          if (valid) {
            fs1 += y[m][j];
            fq1 = fmaf(y[m][j], y[m][j], fq1);
          }
        }
      }
      double s = fs1, sq = fq1;  // values of one thread in f32, the CTA sum in f64
      if (mode == DC_ROW || mode == DC_STATS1) epi_sum2(s, sq, red);
      if (mode == DC_STATS1) {
        if (threadIdx.x == 192) {
          a.part1[2 * (int64_t)w] = s;
          a.part1[2 * (int64_t)w + 1] = sq;
        }
        continue;
      }
      if (mode != DC_ROW) row_sum(a.part1, row, s, sq);
      float mean, inv;
      norm_of(s, sq, ic1, mean, inv);
#pragma unroll
      for (int m = 0; m < 3; ++m) {
        float g[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) g[j] = 0.f;
        if (owned(m * 128 + r)) {
#pragma unroll
          for (int j = 0; j < S::JA; ++j) {
            const float scale = inv * n1w[j];
            g[j] = gelu(y[m][j] * scale + (n1b[j] - mean * scale));
          }
        }
        if (hh == 1) g[7] = 1.0f;  // slot 15: conv2's bias input
        // row r of the 128 x 16 K-major tile, 64-byte swizzle: 16-byte chunk
        // c lives at chunk c ^ ((r / 2) % 4)
        unsigned char* hi = smem + S::OFF_G + m * S::G_BYTES + r * 64;
        unsigned char* lo = hi + 3 * S::G_BYTES;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int phys = ((2 * hh + c) ^ ((r >> 1) & 3)) << 4;
          const float4 v = make_float4(g[4 * c], g[4 * c + 1], g[4 * c + 2], g[4 * c + 3]);
          *reinterpret_cast<float4*>(hi + phys) = v;
          if (conv2)
            *reinterpret_cast<float4*>(lo + phys) =
                make_float4(v.x - trunc_tf32(v.x), v.y - trunc_tf32(v.y), v.z - trunc_tf32(v.z),
                            v.w - trunc_tf32(v.w));
        }
      }
      if (conv2) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        mbar_arrive(&g_ready);
      }
      if constexpr (S::ALL) {
        if (conv2) {
          // this thread's residual x[p][24 hh .. 24 hh + 24) of the three
          // blocks, landing while the moments of z are reduced
          const int t = threadIdx.x - 192;
          for (int m = 0; m < 3; ++m) {
            const int p = 128 * m + r;
            if (owned(p)) {
              const float* src = a.x + ((int64_t)row * T + ts + p) * C + 24 * hh;
#pragma unroll
              for (int i = 0; i < 6; ++i) {
                const uint32_t dst = smem_u32(smem + S::OFF_RES + ((6 * m + i) * 256 + t) * 16);
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src + 4 * i)
                             : "memory");
              }
            }
          }
          asm volatile("cp.async.commit_group;" ::: "memory");
        }
      }

      // ---- moments of z: the sums of v.g and g'Mg over the owned frames ----
      if (mode == DC_OUT) {
        row_sum(a.part2, row, s, sq);
      } else {
        epi_bar();  // g of every frame is in shared memory
        float ls = 0.f, lq = 0.f;
        for (int p = threadIdx.x - 192; p < 384; p += kEpiThreads) {
          if (!owned(p)) continue;
          const int rr = p & 127;
          const unsigned char* gp = smem + S::OFF_G + (p >> 7) * S::G_BYTES + rr * 64;
          float gs[16];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const float4 v = *reinterpret_cast<const float4*>(gp + ((c ^ ((rr >> 1) & 3)) << 4));
            gs[4 * c] = v.x;
            gs[4 * c + 1] = v.y;
            gs[4 * c + 2] = v.z;
            gs[4 * c + 3] = v.w;
          }
          float ga[S::ACT];
#pragma unroll
          for (int i = 0; i < S::ACT; ++i) ga[i] = gs[S::act_slot(i)];
          float l = 0.f, qf = 0.f;
#pragma unroll
          for (int i = 0, idx = 0; i < S::ACT; ++i) {
            l = fmaf(zq.v[i], ga[i], l);
            float t = 0.f;
#pragma unroll
            for (int j = i; j < S::ACT; ++j, ++idx) t = fmaf(zq.m[idx], ga[j], t);
            qf = fmaf(ga[i], t, qf);
          }
          ls += l;
          lq += qf;
        }
        s = ls;
        sq = lq;
        epi_sum2(s, sq, red);
        if (mode == DC_STATS2) {
          if (threadIdx.x == 192) {
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
      for (int c = threadIdx.x - 192; c < C; c += kEpiThreads) {
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
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      }
      for (int m = 0; m < 3; ++m)
        for (int ch = 0; ch < S::NCHUNK; ++ch) {
          const int j = u & 1;
          if (!S::ALL) {
            if (ok && !mbar_wait(&d2_full[j], (u >> 1) & 1, a.err, 39)) ok = false;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          }
          const int p = m * 128 + r;
          const bool own = owned(p);
          const int c0 = ch * (S::NCH / 2) + 24 * hh;  // first channel of this thread
          float* xp = a.x + ((int64_t)row * T + (own ? ts + p : 0)) * C + c0;
          uint32_t zr[48];
          __syncwarp();
#pragma unroll
          for (int c = 0; c < 48; c += 16)
            tmem_ld16_nw(tmem + lane_base + d2_col(m, j) + 48 * hh + c, zr + c);
          float4 res[6];
          if (S::ALL) {
            if (m == 0) asm volatile("cp.async.wait_all;" ::: "memory");
            const float4* st = reinterpret_cast<const float4*>(smem + S::OFF_RES) + 6 * m * 256 +
                               (threadIdx.x - 192);
#pragma unroll
            for (int i = 0; i < 6; ++i) res[i] = st[i * 256];
          } else if (ok && own) {
#pragma unroll
            for (int i = 0; i < 6; ++i) res[i] = reinterpret_cast<const float4*>(xp)[i];
          }
          tmem_ld_wait<48>(zr);
          if (!S::ALL) {
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            mbar_arrive(&d2_empty[j]);
            ++u;
          }
          if (ok && own) {
#pragma unroll
            for (int sc = 0; sc < 3; ++sc) {
              float o[8] = {res[2 * sc].x, res[2 * sc].y, res[2 * sc].z, res[2 * sc].w,
                            res[2 * sc + 1].x, res[2 * sc + 1].y, res[2 * sc + 1].z,
                            res[2 * sc + 1].w};
#pragma unroll
              for (int k = 0; k < 8; ++k) {
                const float4 f = aff[c0 + 8 * sc + k];
                // gamma * GN2(value), GN2(gate)
                const float value = fmaf(__uint_as_float(zr[16 * sc + 2 * k]), f.x, f.y);
                const float gate = fmaf(__uint_as_float(zr[16 * sc + 2 * k + 1]), f.z, f.w);
                o[k] += __fdividef(value, 1.0f + __expf(-gate));
              }
              if (a.round_out) {
#pragma unroll
                for (int k = 0; k < 8; ++k) o[k] = round_tf32(o[k]);
              }
              float4* x4 = reinterpret_cast<float4*>(xp + 8 * sc);
              x4[0] = make_float4(o[0], o[1], o[2], o[3]);
              x4[1] = make_float4(o[4], o[5], o[6], o[7]);
            }
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
  DcZq<C> zq;
  for (int i = 0; i < S::ACT; ++i) zq.v[i] = a.zq_host[i];
  for (int i = 0; i < S::NQ; ++i) zq.m[i] = a.zq_host[S::ACT + i];
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(dconv_tc_row_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         S::SMEM);
    configured = true;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int items = a.rows * a.tiles;
  const int grid = items < sms ? items : sms;
  if (a.tiles == 1) {
    dconv_tc_row_kernel<C><<<grid, kThreads, S::SMEM, s>>>(mx, m1, m1lo, m2, m2lo, a, zq, DC_ROW);
  } else {
    for (int mode = DC_STATS1; mode <= DC_OUT; ++mode)
      dconv_tc_row_kernel<C><<<grid, kThreads, S::SMEM, s>>>(mx, m1, m1lo, m2, m2lo, a, zq, mode);
  }
  return true;
}

}  // namespace

bool dconv_tc_supported(int C, int T) {
  return (C == 48 || C == 96) && T > 0 && tensor_map_encoder() != nullptr;
}

int dconv_tc_tiles(int T) { return (T + kTileStride - 1) / kTileStride; }

bool launch_dconv_tc(const DConvArgs& a, cudaStream_t s) {
  if (!dconv_tc_supported(a.C, a.T) || a.dil < 1 || a.dil > 2 || !a.w1_tc || !a.w1_tc_lo ||
      !a.w2_tc || !a.w2_tc_lo || !a.zq_host || a.w1_npad < 16 || a.w2_npad < 2 * a.C ||
      a.tiles != dconv_tc_tiles(a.T) || (a.tiles > 1 && (!a.part1 || !a.part2)) ||
      (int64_t)a.rows * a.tiles > INT32_MAX)
    return false;
  switch (a.C) {
    case 48: return launch_c<48>(a, s);
    case 96: return launch_c<96>(a, s);
    default: return false;
  }
}

}  // namespace dmx
