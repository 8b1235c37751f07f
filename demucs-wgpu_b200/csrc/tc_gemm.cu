// tcgen05 implicit-GEMM kernel (see tc_gemm.cuh for the design).
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "kernels.h"
#include "tc_common.cuh"
#include "tc_gemm.cuh"

namespace dmx {

namespace {

constexpr int BM = 128;
constexpr int kThreads = 448;  // warp 0 TMA, warp 1 MMA, warps 2-5 converter, warps 6-13 epilogue
constexpr int kEpiThreads = 256;

// Arithmetic of the contraction: MODE_TF32 (operands rounded to nearest tf32),
// MODE_SPLIT (3xTF32: hi*hi + hi*lo + lo*hi), MODE_BF16 (kind::f16: A is a
// bf16 activation tile and B a bf16 weight tile, both loaded by TMA as they
// lie in HBM, f32 accumulate; no converter pass).
constexpr int MODE_TF32 = 0, MODE_SPLIT = 1, MODE_BF16 = 2;

// RB (resident B): the single column tile's whole B (every K block) is
// loaded once per CTA and stays in shared memory after the barrier block;
// stages carry A only. For narrow layers (N = 96, 16-channel K blocks) whose
// B is re-read per output tile otherwise.
template <int BN, int BK, int STAGES, int MODE, bool RB = false>
struct Smem {
  static constexpr bool SPLIT = MODE == MODE_SPLIT, BF = MODE == MODE_BF16;
  static constexpr int ELEM = BF ? 2 : 4;
  static constexpr int A_BYTES = BM * BK * ELEM;
  static constexpr int B_BYTES = BN * BK * ELEM;
  // stage: A | B [| A_lo | B_lo]; TMA fills A, B (and B_lo), the converter
  // warps round A in place (and write A_lo)
  static constexpr int STAGE_BYTES =
      RB ? A_BYTES : (SPLIT ? 2 * (A_BYTES + B_BYTES) : A_BYTES + B_BYTES);
  static constexpr int TMA_BYTES = RB ? A_BYTES : (SPLIT ? A_BYTES + 2 * B_BYTES : A_BYTES + B_BYTES);
  // stages, then the barrier block (1024 bytes, keeping resident B aligned)
  static constexpr int TOTAL = STAGES * STAGE_BYTES + 1024 /*align*/ + 1024 /*barriers*/;
  // TMEM columns: two accumulators, rounded up to a power of two
  static constexpr uint32_t TMEM_COLS =
      2 * BN <= 64 ? 64u : (2 * BN <= 128 ? 128u : (2 * BN <= 256 ? 256u : 512u));
  static_assert(!RB || MODE == MODE_TF32, "resident B: single-pass tf32 only");
  static_assert(!BF || BK == 32 || BK == 64,
                "bf16 tiles are 32 or 64 channels: 64- or 128-byte swizzled rows");
  static_assert(STAGE_BYTES % 1024 == 0, "stages keep the 1024-byte swizzle alignment");
};

// GELU of the GEMM epilogue: on the A&S erf (fewer instructions, two of them
// on the special-function unit) in the tf32 GEMMs, on erff in the bf16 GEMMs,
// where the faster MMAs leave the epilogue's special-function operations the
// limit (measured on B200: the BF16 FFN1 took 3.14 ms on the A&S erf, 3.01 ms
// on erff)
template <int MODE>
DMX_DEVICE float gelu_epi(float x) {
  return MODE == MODE_BF16 ? gelu(x) : gelu_tc(x);
}

// two fp32 -> one bf16x2 word, round to nearest even (lo in the low half)
DMX_DEVICE uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __float22bfloat162_rn(make_float2(lo, hi));
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Origin of output-row tile `mt` (see TcAMode).
DMX_DEVICE void tile_origin(const TcParams& p, int mt, int& tb, int& ty0, int& tx0, int64_t& m0) {
  tb = ty0 = tx0 = 0;
  m0 = 0;
  if (p.mode == TC_2D) {
    const int nxb = (p.Wq + 15) / 16, nyb = (p.Hq + 7) / 8;
    tx0 = (mt % nxb) * 16;
    ty0 = ((mt / nxb) % nyb) * 8;
    tb = mt / (nxb * nyb);
  } else if (p.mode == TC_1D) {
    const int nxb = (p.Wq + BM - 1) / BM;
    tx0 = (mt % nxb) * BM;
    tb = mt / nxb;
  } else {
    m0 = (int64_t)mt * BM;
  }
}

// Persistent: CTA c computes tiles c, c + grid, ... of the (row tile, column
// tile) space in row-major order, so the column tiles of one row tile run on
// neighbouring SMs at the same time and its A rows come from HBM once. Two
// TMEM accumulators: the epilogue of one tile overlaps the MMAs of the next.
template <int BN, int BK, int STAGES, int EPI, int MODE, bool RB = false>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmBlo, const TcParams p) {
  using S = Smem<BN, BK, STAGES, MODE, RB>;
  constexpr bool SPLIT = S::SPLIT, BF = S::BF;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * S::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* conv = empty + STAGES;
  uint64_t* acc_full = conv + STAGES;   // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint64_t* bres_full = acc_empty + 2;  // resident B has landed (RB)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bres_full + 1);
  unsigned char* bres = smem + STAGES * S::STAGE_BYTES + 1024;  // resident B (RB)

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // a previous launch on this stream gave up: do nothing (uniform across the CTA)
  if (p.err && *reinterpret_cast<volatile int*>(p.err) != 0) return;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], 128);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kEpiThreads);
    }
    mbar_init(bres_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(S::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const int ktiles = p.Kpad / BK;
  const int total = p.mtiles * p.ntiles;
  // A already rounded to tf32 (and no split): the MMA consumes the TMA tile
  // directly and the converter warps stay idle
  const bool direct = BF || (!SPLIT && p.a_rounded && !p.a_stats);

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      uint32_t it = 0;
      bool ok = true;
      if (RB) {
        // the whole B of the single column tile, once: K block kt at bres + kt B_BYTES
        mbar_expect_tx(bres_full, (uint32_t)ktiles * S::B_BYTES);
        for (int kt = 0; kt < ktiles; ++kt)
          tma_load_2d(bres + kt * S::B_BYTES, &tmB, bres_full, kt * BK, 0);
      }
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const int mt = t / p.ntiles, n0 = (t - mt * p.ntiles) * BN;
        int tb, ty0, tx0;
        int64_t m0;
        tile_origin(p, mt, tb, ty0, tx0, m0);
        for (int kt = 0; kt < ktiles; ++kt, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, p.err, 1)) {
            ok = false;
            break;
          }
          unsigned char* a_dst = smem + s * S::STAGE_BYTES;
          unsigned char* b_dst = a_dst + S::A_BYTES;
          mbar_expect_tx(&full[s], S::TMA_BYTES);
          const int k0 = kt * BK;
          if (p.mode == TC_2D) {
            // with sy = 4 the map traverses H with stride 4: one box is 8 rows
            const int tap = k0 / p.Cin, c0 = k0 - tap * p.Cin;
            tma_load_4d(a_dst, &tmA, &full[s], c0, tx0 + p.dx[tap], ty0 * p.sy + p.dy[tap], tb);
          } else if (p.mode == TC_1D) {
            const int tap = k0 / p.Cin, c0 = k0 - tap * p.Cin;
            const int x0 = tx0 * p.sx + p.dx[tap];
            tma_load_3d(a_dst, &tmA, &full[s], c0, x0, tb);
            // a strided box holds at most 256 / sx rows: two boxes of 64 rows
            // (the swizzle pattern repeats every 8 rows, so the halves line up)
            if (p.sx != 1) tma_load_3d(a_dst + 64 * BK * 4, &tmA, &full[s], c0, x0 + 64 * p.sx, tb);
          } else {
            tma_load_2d(a_dst, &tmA, &full[s], k0, (int)m0);
          }
          if (!RB) tma_load_2d(b_dst, &tmB, &full[s], k0, n0);
          if (SPLIT) tma_load_2d(b_dst + S::B_BYTES + S::A_BYTES, &tmBlo, &full[s], k0, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      // instruction descriptor: f32 accumulator; A and B both tf32 (2) or both bf16 (1)
      constexpr uint32_t ab = BF ? 1u : 2u;
      constexpr uint32_t idesc = (1u << 4) | (ab << 7) | (ab << 10) | ((uint32_t)(BN >> 3) << 17) |
                                 ((uint32_t)(BM >> 4) << 24);
      uint32_t it = 0;
      int tl = 0;
      bool ok = !RB || mbar_wait(bres_full, 0, p.err, 6);
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++tl) {
        const int acc = tl & 1;
        if (!mbar_wait(&acc_empty[acc], ((tl >> 1) & 1) ^ 1, p.err, 5)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        for (int kt = 0; kt < ktiles; ++kt, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(direct ? &full[s] : &conv[s], ph, p.err, 2)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a_addr = smem_u32(smem + s * S::STAGE_BYTES);
          const uint32_t b_addr = RB ? smem_u32(bres + kt * S::B_BYTES) : a_addr + S::A_BYTES;
          const uint32_t alo_addr = b_addr + S::B_BYTES;
          const uint32_t blo_addr = alo_addr + S::A_BYTES;
          if (BF) {
            // K = 16 steps across the 64- or 128-byte bf16 rows of A and B
#pragma unroll
            for (int j = 0; j < BK / 16; ++j)
              umma_bf16(d, umma_desc_k(a_addr + j * 32, BK * 2), umma_desc_k(b_addr + j * 32, BK * 2),
                        idesc, (kt | j) != 0);
          }
#pragma unroll
          for (int j = 0; j < (BF ? 0 : BK / 8); ++j) {
            const uint64_t ad = umma_desc_k(a_addr + j * 32, BK * 4);
            const uint64_t bd = umma_desc_k(b_addr + j * 32, BK * 4);
            if (SPLIT) {
              // small terms first: lo*hi + hi*lo, then hi*hi
              umma_tf32(d, umma_desc_k(alo_addr + j * 32, BK * 4), bd, idesc, (kt | j) != 0);
              umma_tf32(d, ad, umma_desc_k(blo_addr + j * 32, BK * 4), idesc, 1);
              umma_tf32(d, ad, bd, idesc, 1);
            } else {
              umma_tf32(d, ad, bd, idesc, (kt | j) != 0);
            }
          }
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[acc]);
      }
    }
  } else if (warp < 6) {
    // ---------------- converter: warps 2..5, one A row per thread ----------------
    // Round each landed A row to nearest tf32 in place (the tensor core would
    // otherwise truncate); for SPLIT write the residual x - tf32(x) into the
    // A_lo buffer at the same offset.
    const int row = threadIdx.x - 64;
    // visit the row's 16-byte chunks in the order the TMA swizzle permutes
    // them (chunk ^ (128-byte line % 8)), so the 8 lanes of a quarter-warp
    // touch 8 different bank groups
    const int swz = BK == 32 ? (row & 7) : ((row >> 1) & 3);
    uint32_t it = 0;
    bool live = true;
    for (int t = blockIdx.x; t < total && !direct; t += gridDim.x) {
      // optional A transform (TC_ROWS): GELU(GroupNorm(a)) with this row's moments
      float a_mean = 0.f, a_inv = 0.f;
      bool a_row = false;
      if (p.a_stats) {
        const int64_t pos = (int64_t)(t / p.ntiles) * BM + row;
        a_row = pos < (int64_t)p.B * p.Hq * p.Wq;
        if (a_row) {
          const RowNorm rn = row_norm(p.a_stats, (int)(pos / p.a_rowlen), p.a_count);
          a_mean = rn.mean;
          a_inv = rn.inv;
        }
      }
      for (int kt = 0; kt < ktiles; ++kt, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (live && !mbar_wait(&full[s], ph, p.err, 4)) live = false;
        if (live) {
          float4* a = reinterpret_cast<float4*>(smem + s * S::STAGE_BYTES + row * BK * 4);
          float4* alo = reinterpret_cast<float4*>(smem + s * S::STAGE_BYTES + S::A_BYTES +
                                                  S::B_BYTES + row * BK * 4);
#pragma unroll
          for (int qq = 0; qq < BK / 4; ++qq) {
            const int q = qq ^ swz;
            float4 x = a[q];
            if (p.a_stats) {
              float xv[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int k = kt * BK + qq * 4 + e;
                float g = 0.f;
                if (a_row && k < p.a_nvalid) {
                  const float scale = a_inv * p.a_gw[k];
                  g = gelu_tc(xv[e] * scale + (p.a_gb[k] - a_mean * scale));
                }
                xv[e] = g;
              }
              x = make_float4(xv[0], xv[1], xv[2], xv[3]);
            }
            float4 hi;
            hi.x = round_tf32(x.x);
            hi.y = round_tf32(x.y);
            hi.z = round_tf32(x.z);
            hi.w = round_tf32(x.w);
            a[q] = hi;
            if (SPLIT) alo[q] = make_float4(x.x - hi.x, x.y - hi.y, x.z - hi.z, x.w - hi.w);
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&conv[s]))
                     : "memory");
      }
    }
  } else {
    // ---------------- epilogue: warps 6..13, one TMEM lane (row) per thread ----------------
    // two warps per TMEM lane quarter; half hh takes the 32-column chunks
    // 64 k + 32 hh of the tile
    const int e = warp - 6, quarter = warp % 4, hh = e / 4;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    constexpr bool kStats = EPI == EPI_RESIDUAL || EPI == EPI_STORE_STATS || EPI == EPI_STATS;
    bool ok = true;
    int tl = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++tl) {
      const int mt = t / p.ntiles, n0 = (t - mt * p.ntiles) * BN;
      int tb, ty0, tx0;
      int64_t m0;
      tile_origin(p, mt, tb, ty0, tx0, m0);
      const int acc = tl & 1;
      if (ok && !mbar_wait(&acc_full[acc], (tl >> 1) & 1, p.err, 3)) ok = false;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      int b, y, x;
      int64_t pos;
      bool valid;
      if (p.mode == TC_2D) {
        y = ty0 + r / 16;
        x = tx0 + r % 16;
        b = tb;
        valid = y < p.Hq && x < p.Wq;
        pos = ((int64_t)b * p.Hq + y) * p.Wq + x;
      } else if (p.mode == TC_1D) {
        y = 0;
        x = tx0 + r;
        b = tb;
        valid = x < p.Wq;
        pos = (int64_t)b * p.Wq + x;
      } else {
        pos = m0 + r;
        const int64_t plane = (int64_t)p.Hq * p.Wq;
        valid = pos < (int64_t)p.B * plane;
        b = (int)(pos / plane);
        const int64_t rem = pos - (int64_t)b * plane;
        y = (int)(rem / p.Wq);
        x = (int)(rem % p.Wq);
      }
      const int64_t orow = (int64_t)b * p.o_bs + (int64_t)y * p.o_ys + (int64_t)x * p.o_xs + p.o_off;
      // columns stored for this row (o_lim clips the positions 4x + i >= o_lim)
      const int ncol = p.o_lim ? min(p.N, max(0, (p.o_lim - 4 * x) * p.o_lim_ch)) : p.N;
      double ls = 0.0, lq = 0.0;
      // DConv tail: this row's GroupNorm2 statistics, once per tile
      RowNorm nr{0.f, 0.f};
      if (EPI == EPI_DCONV_TAIL && valid) nr = row_norm(p.epi_nstats, (int)(pos / p.epi_rowlen), p.epi_count);
      const uint32_t tacc = tmem + lane_base + (uint32_t)(acc * BN);
      for (int c0 = 32 * hh; c0 < BN; c0 += 64) {
        float v[32];
        __syncwarp();
        tmem_ld32(tacc + (uint32_t)c0, v);
        const int nb = n0 + c0;
        if (ok && valid && nb < ncol) {
          // a full chunk whose row segment is 16-byte aligned moves as float4
          const bool full = nb + 32 <= ncol;
          const bool bias4 = full && ((reinterpret_cast<uintptr_t>(p.bias + nb) & 15) == 0);
          if (bias4) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              const float4 bb = *reinterpret_cast<const float4*>(p.bias + nb + j);
              v[j] += bb.x;
              v[j + 1] += bb.y;
              v[j + 2] += bb.z;
              v[j + 3] += bb.w;
            }
          } else {
            for (int j = 0; j < 32; ++j)
              if (nb + j < ncol) v[j] += p.bias[nb + j];
          }
          if ((EPI == EPI_STORE || EPI == EPI_GELU) && p.o_pcols) {
            // split columns: each 16-column half lies in one group of o_pcols
            // (a multiple of 16) and goes to row orow + group * o_pstride
            if (EPI == EPI_GELU) {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = gelu_epi<MODE>(v[j]);
            }
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              const int n = nb + 16 * hf;
              if (n < ncol) {
                const int grp = n / p.o_pcols;
                const int64_t at = orow + (int64_t)grp * p.o_pstride + (n - grp * p.o_pcols);
                const bool v4 = n + 16 <= ncol && (at & 3) == 0;
                if (p.epi_add) {
                  const float* ad = p.epi_add + at;
                  if (v4) {
#pragma unroll
                    for (int j = 0; j < 16; j += 4) {
                      const float4 t4 = *reinterpret_cast<const float4*>(ad + j);
                      v[16 * hf + j] += t4.x;
                      v[16 * hf + j + 1] += t4.y;
                      v[16 * hf + j + 2] += t4.z;
                      v[16 * hf + j + 3] += t4.w;
                    }
                  } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                      if (n + j < ncol) v[16 * hf + j] += ad[j];
                  }
                }
                if (p.round_out) {
#pragma unroll
                  for (int j = 0; j < 16; ++j) v[16 * hf + j] = round_tf32(v[16 * hf + j]);
                }
                float* o = p.out + at;
                if (v4 && (reinterpret_cast<uintptr_t>(o) & 31) == 0) {
                  st_global8(o, v + 16 * hf);
                  st_global8(o + 8, v + 16 * hf + 8);
                } else if (v4) {
#pragma unroll
                  for (int j = 0; j < 16; j += 4)
                    *reinterpret_cast<float4*>(o + j) =
                        make_float4(v[16 * hf + j], v[16 * hf + j + 1], v[16 * hf + j + 2],
                                    v[16 * hf + j + 3]);
                } else {
#pragma unroll
                  for (int j = 0; j < 16; ++j)
                    if (n + j < ncol) o[j] = v[16 * hf + j];
                }
              }
            }
          } else if (EPI == EPI_STORE || EPI == EPI_GELU || EPI == EPI_STORE_STATS) {
            if (EPI == EPI_GELU) {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = gelu_epi<MODE>(v[j]);
            }
            const bool vec = full && ((orow + nb) & 3) == 0;
            if (p.epi_add) {
              const float* ad = p.epi_add + orow + nb;
              if (vec && (reinterpret_cast<uintptr_t>(ad) & 31) == 0) {
                float a32[32];
#pragma unroll
                for (int j = 0; j < 32; j += 8) ld_global8(ad + j, a32 + j);
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] += a32[j];
              } else if (vec) {
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                  const float4 t4 = *reinterpret_cast<const float4*>(ad + j);
                  v[j] += t4.x;
                  v[j + 1] += t4.y;
                  v[j + 2] += t4.z;
                  v[j + 3] += t4.w;
                }
              } else {
                for (int j = 0; j < 32; ++j)
                  if (nb + j < ncol) v[j] += ad[j];
              }
            }
            if (p.round_out) {  // the output feeds only tf32 GEMMs: round to nearest once
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = round_tf32(v[j]);
            }
            if (EPI == EPI_STORE && p.vt_out && nb >= p.vt_col0) {
              // whole 32-column chunks belong to one head (vt_col0 and 64 are multiples of 32)
              const int c = nb - p.vt_col0, h2 = c / 64, d0 = c % 64;
              const int64_t bb = pos / p.vt_ntok, tok = pos % p.vt_ntok;
              const int64_t at = ((bb * 8 + h2) * 64 + d0) * (int64_t)p.vt_ntok + tok;
              if (p.vt16) {
                uint16_t* vt = reinterpret_cast<uint16_t*>(p.vt_out) + at;
                for (int j = 0; j < 32; ++j)
                  if (nb + j < ncol) vt[(int64_t)j * p.vt_ntok] = (uint16_t)(pack_bf16(v[j], 0.f) & 0xFFFFu);
              } else {
                float* vt = p.vt_out + at;
                for (int j = 0; j < 32; ++j)
                  if (nb + j < ncol) vt[(int64_t)j * p.vt_ntok] = v[j];
              }
            }
            if (p.out16) {
              // bf16 output (the A operand of a bf16 GEMM): 32 values in 64 bytes
              uint16_t* o16 = p.out16 + orow + nb;
              if (full && (reinterpret_cast<uintptr_t>(o16) & 31) == 0) {
                uint32_t w16[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) w16[j] = pack_bf16(v[2 * j], v[2 * j + 1]);
                st_global8(reinterpret_cast<uint32_t*>(o16), w16);
                st_global8(reinterpret_cast<uint32_t*>(o16) + 8, w16 + 8);
              } else if (full && ((orow + nb) & 7) == 0) {
#pragma unroll
                for (int j = 0; j < 32; j += 8)
                  *reinterpret_cast<uint4*>(o16 + j) =
                      make_uint4(pack_bf16(v[j], v[j + 1]), pack_bf16(v[j + 2], v[j + 3]),
                                 pack_bf16(v[j + 4], v[j + 5]), pack_bf16(v[j + 6], v[j + 7]));
              } else {
                for (int j = 0; j < 32; ++j)
                  if (nb + j < ncol) o16[j] = (uint16_t)(pack_bf16(v[j], 0.f) & 0xFFFFu);
              }
            } else {
              float* o = p.out + orow + nb;
              if (vec && (reinterpret_cast<uintptr_t>(o) & 31) == 0) {
#pragma unroll
                for (int j = 0; j < 32; j += 8) st_global8(o + j, v + j);
              } else if (vec) {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                  *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
              } else {
                for (int j = 0; j < 32; ++j)
                  if (nb + j < ncol) o[j] = v[j];
              }
            }
          }
          if (EPI == EPI_GLU || EPI == EPI_GLU_EMB) {
            // 16 outputs: channels nb/2 .. nb/2 + 15
            float g[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) g[j] = glu_tc(v[2 * j], v[2 * j + 1]);
            const int c0o = nb / 2;
            const bool vec = full && ((orow + c0o) & 3) == 0;
            if (EPI == EPI_GLU_EMB) {
              const float* em = p.epi_emb + (int64_t)y * (p.N / 2) + c0o;
              if (vec && ((((int64_t)y * (p.N / 2) + c0o) & 3) == 0)) {
#pragma unroll
                for (int j = 0; j < 16; j += 4) {
                  const float4 t4 = *reinterpret_cast<const float4*>(em + j);
                  g[j] += t4.x;
                  g[j + 1] += t4.y;
                  g[j + 2] += t4.z;
                  g[j + 3] += t4.w;
                }
              } else {
                for (int j = 0; j < 16; ++j)
                  if (nb + 2 * j < ncol) g[j] += em[j];
              }
            }
            float* o = p.out + orow + c0o;
            if (vec && (reinterpret_cast<uintptr_t>(o) & 31) == 0) {
              st_global8(o, g);
              st_global8(o + 8, g + 8);
            } else if (vec) {
#pragma unroll
              for (int j = 0; j < 16; j += 4)
                *reinterpret_cast<float4*>(o + j) = make_float4(g[j], g[j + 1], g[j + 2], g[j + 3]);
            } else {
              for (int j = 0; j < 16; ++j)
                if (nb + 2 * j < ncol) o[j] = g[j];
            }
          }
          if (EPI == EPI_DCONV_TAIL) {
            // channels nb/2 .. nb/2 + 15: out = res + gamma * GLU(GroupNorm(v))
            const int c0o = nb / 2;
            float* o = p.out + orow + c0o;
            const float* rr = p.epi_res + orow + c0o;
            const bool vec = full && ((orow + c0o) & 3) == 0;
            const bool v8 = vec && ((reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(rr)) & 31) == 0;
            float res[16];
            if (v8) {
              ld_global8(rr, res);
              ld_global8(rr + 8, res + 8);
            } else if (vec) {
#pragma unroll
              for (int j = 0; j < 16; j += 4) {
                const float4 r4 = *reinterpret_cast<const float4*>(rr + j);
                res[j] = r4.x;
                res[j + 1] = r4.y;
                res[j + 2] = r4.z;
                res[j + 3] = r4.w;
              }
            } else {
              for (int j = 0; j < 16; ++j) res[j] = nb + 2 * j < ncol ? rr[j] : 0.f;
            }
            if (vec && (p.epi_half & 3) == 0) {
              // per-channel GroupNorm weights / biases (value, gate) and LayerScale, 16 bytes at a time
#pragma unroll
              for (int j4 = 0; j4 < 16; j4 += 4) {
                const int c = c0o + j4;
                const float4 wv = __ldg(reinterpret_cast<const float4*>(p.epi_gw + c));
                const float4 wg = __ldg(reinterpret_cast<const float4*>(p.epi_gw + c + p.epi_half));
                const float4 bv = __ldg(reinterpret_cast<const float4*>(p.epi_gb + c));
                const float4 bg = __ldg(reinterpret_cast<const float4*>(p.epi_gb + c + p.epi_half));
                const float4 gm = __ldg(reinterpret_cast<const float4*>(p.epi_gamma + c));
                const float awv[4] = {wv.x, wv.y, wv.z, wv.w}, awg[4] = {wg.x, wg.y, wg.z, wg.w};
                const float abv[4] = {bv.x, bv.y, bv.z, bv.w}, abg[4] = {bg.x, bg.y, bg.z, bg.w};
                const float agm[4] = {gm.x, gm.y, gm.z, gm.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int j = j4 + e;
                  const float vs = nr.inv * awv[e];
                  const float gsc = nr.inv * awg[e];
                  const float value = v[2 * j] * vs + (abv[e] - nr.mean * vs);
                  const float gate = v[2 * j + 1] * gsc + (abg[e] - nr.mean * gsc);
                  res[j] += agm[e] * glu_tc(value, gate);
                }
              }
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int c = c0o + j;
                if (nb + 2 * j < ncol) {
                  const float vs = nr.inv * p.epi_gw[c];
                  const float gsc = nr.inv * p.epi_gw[c + p.epi_half];
                  const float value = v[2 * j] * vs + (p.epi_gb[c] - nr.mean * vs);
                  const float gate = v[2 * j + 1] * gsc + (p.epi_gb[c + p.epi_half] - nr.mean * gsc);
                  res[j] += p.epi_gamma[c] * glu_tc(value, gate);
                }
              }
            }
            if (p.round_out) {
#pragma unroll
              for (int j = 0; j < 16; ++j) res[j] = round_tf32(res[j]);
            }
            if (v8) {
              st_global8(o, res);
              st_global8(o + 8, res + 8);
            } else if (vec) {
#pragma unroll
              for (int j = 0; j < 16; j += 4)
                *reinterpret_cast<float4*>(o + j) = make_float4(res[j], res[j + 1], res[j + 2], res[j + 3]);
            } else {
              for (int j = 0; j < 16; ++j)
                if (nb + 2 * j < ncol) o[j] = res[j];
            }
          }
          if (EPI == EPI_RESIDUAL) {
            float* o = p.out + orow + nb;
            const float* rr = p.epi_res + orow + nb;
            const bool vec = full && ((orow + nb) & 3) == 0 &&
                             ((reinterpret_cast<uintptr_t>(p.epi_gamma + nb) & 15) == 0);
            if (vec && ((reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(rr)) & 31) == 0) {
              // 32-byte accesses: the row's residual first, then the outputs
              float r32[32];
#pragma unroll
              for (int j = 0; j < 32; j += 8) ld_global8(rr + j, r32 + j);
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                const float4 g4 = *reinterpret_cast<const float4*>(p.epi_gamma + nb + j);
                v[j] = fmaf(g4.x, v[j], r32[j]);
                v[j + 1] = fmaf(g4.y, v[j + 1], r32[j + 1]);
                v[j + 2] = fmaf(g4.z, v[j + 2], r32[j + 2]);
                v[j + 3] = fmaf(g4.w, v[j + 3], r32[j + 3]);
              }
#pragma unroll
              for (int j = 0; j < 32; j += 8) st_global8(o + j, v + j);
            } else if (vec) {
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                const float4 r4 = *reinterpret_cast<const float4*>(rr + j);
                const float4 g4 = *reinterpret_cast<const float4*>(p.epi_gamma + nb + j);
                v[j] = fmaf(g4.x, v[j], r4.x);
                v[j + 1] = fmaf(g4.y, v[j + 1], r4.y);
                v[j + 2] = fmaf(g4.z, v[j + 2], r4.z);
                v[j + 3] = fmaf(g4.w, v[j + 3], r4.w);
                *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
              }
            } else {
              for (int j = 0; j < 32; ++j)
                if (nb + j < ncol) {
                  v[j] = rr[j] + p.epi_gamma[nb + j] * v[j];
                  o[j] = v[j];
                }
            }
          }
          if (kStats) {
            float fs = 0.f, fq = 0.f;
            for (int j = 0; j < 32; ++j)
              if (nb + j < ncol) {
                fs += v[j];
                fq = fmaf(v[j], v[j], fq);
              }
            ls += (double)fs;
            lq += (double)fq;
          }
        }  // ok && valid
      }
      // the accumulator may be overwritten by the next tile's MMAs
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&acc_empty[acc]))
                   : "memory");
      if (kStats && p.epi_rowpart && valid) {
        // this thread's share of the row's moments: one partial per position and
        // (column tile, epilogue half), reduced in a fixed order after the launch
        // (stats.cu), so no atomics and no dependence on the tile's neighbours
        double* e = p.epi_rowpart + (pos * p.epi_nslots + (n0 / BN) * 2 + hh) * 2;
        e[0] = ls;
        e[1] = lq;
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(S::TMEM_COLS));
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
// resident B's shared memory: every K block of one column tile
template <int BN, int BK, int MODE>
int resident_b_bytes(const TcParams& p) {
  return (p.Kpad / BK) * Smem<BN, BK, 1, MODE>::B_BYTES;
}

template <int BN, int BK, int STAGES, int MODE, bool RB = false>
void launch_cfg(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mblo,
                const TcParams& p, int epi, dim3 grid, cudaStream_t s) {
  const int smem = Smem<BN, BK, STAGES, MODE, RB>::TOTAL + (RB ? resident_b_bytes<BN, BK, MODE>(p) : 0);
#define DMX_TC_CASE(E)                                                                        \
  case E: {                                                                                   \
    static PerDevice attr;                                                                    \
    if (attr.first())                                                                         \
      cudaFuncSetAttribute(tc_gemm_kernel<BN, BK, STAGES, E, MODE, RB>,                      \
                           cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);          \
    tc_gemm_kernel<BN, BK, STAGES, E, MODE, RB><<<grid, kThreads, smem, s>>>(ma, mb, mblo, p); \
    break;                                                                                    \
  }
  switch (epi) {
    DMX_TC_CASE(EPI_STORE)
    DMX_TC_CASE(EPI_GELU)
    DMX_TC_CASE(EPI_GLU)
    DMX_TC_CASE(EPI_GLU_EMB)
    DMX_TC_CASE(EPI_RESIDUAL)
    DMX_TC_CASE(EPI_STORE_STATS)
    DMX_TC_CASE(EPI_STATS)
    DMX_TC_CASE(EPI_DCONV_TAIL)
  }
#undef DMX_TC_CASE
}

int pick_bn(int N) { return N <= 64 ? 64 : (N <= 128 ? 128 : 256); }

bool stats_epi(int epi) { return epi == EPI_RESIDUAL || epi == EPI_STORE_STATS || epi == EPI_STATS; }

int sm_count() {
  static int count[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!count[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    count[dev] = n > 0 ? n : 148;
  }
  return count[dev];
}

}  // namespace

int tc_gemm_stat_slots(int N) { return (N + pick_bn(N) - 1) / pick_bn(N) * 2; }

bool tc_gemm_supported(const TcOperandA& a, const TcParams& p) {
  if (!tensor_map_encoder()) return false;
  // row moments: positions of one statistic row are contiguous in the TC_ROWS
  // and TC_1D orders (not across the 8-row boxes of TC_2D)
  if (p.epi_stats && (p.mode == TC_2D || !p.epi_rowpart || p.epi_rowlen <= 0)) return false;
  const int bk = (p.Cin % 32 == 0) ? 32 : (p.Cin % 16 == 0 ? 16 : 0);
  if (bk == 0) return false;
  // bf16: row-major bf16 activations [rows][C] (16-byte row pitch) times the bf16
  // weight copy; stores fp32 or (STORE / GELU, unsplit columns) bf16
  if (p.bf16 && (p.mode != TC_ROWS || bk != 32 || p.Kpad % 32 != 0 || p.a_stats ||
                 (a.sw * 2) % 16 != 0))
    return false;
  if (p.out16 && (!p.bf16 || (p.vt_out && !p.vt16) || p.o_pcols || p.o_lim || p.epi_add ||
                  p.round_out))
    return false;
  if (p.mode == TC_2D || p.mode == TC_1D) {
    if (a.C != p.Cin) return false;
    if ((a.sw * 4) % 16 || (a.sh * 4) % 16 || (a.sb * 4) % 16) return false;
    const bool strided = p.mode == TC_2D ? (p.sy == 4 && p.sx == 1) : (p.sx == 4 && p.sy == 1);
    if (!strided && (p.sy != 1 || p.sx != 1)) return false;
  } else {
    if (p.ntaps != 1 || p.sy != 1 || p.sx != 1) return false;
    if (!p.bf16 && (a.sw * 4) % 16) return false;
  }
  if ((reinterpret_cast<uintptr_t>(a.ptr) & 15) != 0) return false;
  return true;
}

// K channels per stage of a bf16 GEMM: 64 (128-byte rows, half the TMA
// requests per byte) when K allows it, else 32
int bf16_bk(const TcParams& p) { return p.Kpad % 64 == 0 && p.Cin % 64 == 0 ? 64 : 32; }

void launch_tc_gemm(const TcOperandA& a, const float* wk, const float* wk_lo, const TcParams& p0,
                    int epi, cudaStream_t s) {
  TcParams p = p0;
  const int bk = (p.Cin % 32 == 0) ? 32 : 16;
  const int bkb = p.bf16 ? bf16_bk(p) : 0;
  const CUtensorMapSwizzle swz_bf = bkb == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  // resident B: a narrow layer (N = 96 in one exact column tile, 16-channel K
  // blocks) whose whole B fits in shared memory beside six A stages
  const bool rb = !p.bf16 && !wk_lo && bk == 16 && p.N == 96 && p.Npad >= 96 && !p.epi_stats &&
                  Smem<96, 16, 6, MODE_TF32, true>::TOTAL + resident_b_bytes<96, 16, MODE_TF32>(p) <=
                      227 * 1024;
  const CUtensorMapSwizzle swz = bk == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  const int bn = rb ? 96 : pick_bn(p.N);
  CUtensorMap ma, mb, mblo;
  bool ok;
  if (p.mode == TC_2D) {
    const cuuint64_t dims[4] = {(cuuint64_t)a.C, (cuuint64_t)a.W, (cuuint64_t)a.H, (cuuint64_t)a.B};
    const cuuint64_t str[3] = {(cuuint64_t)a.sw * 4, (cuuint64_t)a.sh * 4, (cuuint64_t)a.sb * 4};
    const cuuint32_t box[4] = {(cuuint32_t)bk, 16, (cuuint32_t)(8 * p.sy), 1};
    const cuuint32_t estr[4] = {1, 1, (cuuint32_t)p.sy, 1};
    ok = make_tensor_map(&ma, a.ptr, 4, dims, str, box, swz, estr);
    p.mtiles = ((p.Wq + 15) / 16) * ((p.Hq + 7) / 8) * p.B;
  } else if (p.mode == TC_1D) {
    const cuuint64_t dims[3] = {(cuuint64_t)a.C, (cuuint64_t)a.W, (cuuint64_t)a.B};
    const cuuint64_t str[2] = {(cuuint64_t)a.sw * 4, (cuuint64_t)a.sb * 4};
    // strided: a box of 256 positions at stride 4 holds 64 rows (two per tile)
    const cuuint32_t box[3] = {(cuuint32_t)bk, (cuuint32_t)(p.sx == 1 ? BM : 64 * p.sx), 1};
    const cuuint32_t estr[3] = {1, (cuuint32_t)p.sx, 1};
    ok = make_tensor_map(&ma, a.ptr, 3, dims, str, box, swz, estr);
    p.mtiles = ((p.Wq + BM - 1) / BM) * p.B;
  } else if (p.bf16) {  // bf16 activations [rows][C]: rows of bkb channels
    const cuuint64_t dims[2] = {(cuuint64_t)a.C, (cuuint64_t)a.W};
    const cuuint64_t str[1] = {(cuuint64_t)a.sw * 2};
    const cuuint32_t box[2] = {(cuuint32_t)bkb, (cuuint32_t)BM};
    ok = make_tensor_map(&ma, a.ptr, 2, dims, str, box, swz_bf, nullptr,
                         CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
    p.mtiles = (a.W + BM - 1) / BM;
  } else {
    const cuuint64_t dims[2] = {(cuuint64_t)a.C, (cuuint64_t)a.W};
    const cuuint64_t str[1] = {(cuuint64_t)a.sw * 4};
    const cuuint32_t box[2] = {(cuuint32_t)bk, (cuuint32_t)BM};
    ok = make_tensor_map(&ma, a.ptr, 2, dims, str, box, swz);
    p.mtiles = (a.W + BM - 1) / BM;
  }
  if (p.bf16) {  // bf16 weights [Npad][Kpad]: rows of bkb channels
    const cuuint64_t dims[2] = {(cuuint64_t)p.Kpad, (cuuint64_t)p.Npad};
    const cuuint64_t str[1] = {(cuuint64_t)p.Kpad * 2};
    const cuuint32_t box[2] = {(cuuint32_t)bkb, (cuuint32_t)bn};
    ok = ok && make_tensor_map(&mb, wk, 2, dims, str, box, swz_bf, nullptr,
                               CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
    mblo = mb;
  } else {
    const cuuint64_t dims[2] = {(cuuint64_t)p.Kpad, (cuuint64_t)p.Npad};
    const cuuint64_t str[1] = {(cuuint64_t)p.Kpad * 4};
    const cuuint32_t box[2] = {(cuuint32_t)bk, (cuuint32_t)bn};
    ok = ok && make_tensor_map(&mb, wk, 2, dims, str, box, swz);
    ok = ok && make_tensor_map(&mblo, wk_lo ? wk_lo : wk, 2, dims, str, box, swz);
  }
  if (!ok) return;  // caller checked tc_gemm_supported; a failed encode leaves the output untouched
  p.ntiles = (p.N + bn - 1) / bn;
  const int64_t total = (int64_t)p.mtiles * p.ntiles;
  const dim3 grid((unsigned)std::min<int64_t>(total, sm_count()));
  if (p.bf16 && bkb == 64) {  // bf16 operands, 64-channel K tiles (192 KB of stages)
    if (bn == 64) launch_cfg<64, 64, 8, MODE_BF16>(ma, mb, mblo, p, epi, grid, s);
    else if (bn == 128) launch_cfg<128, 64, 6, MODE_BF16>(ma, mb, mblo, p, epi, grid, s);
    else launch_cfg<256, 64, 4, MODE_BF16>(ma, mb, mblo, p, epi, grid, s);
  } else if (p.bf16) {  // bf16 operands, 32-channel K tiles
    if (bn == 64) launch_cfg<64, 32, 12, MODE_BF16>(ma, mb, mblo, p, epi, grid, s);
    else if (bn == 128) launch_cfg<128, 32, 10, MODE_BF16>(ma, mb, mblo, p, epi, grid, s);
    else launch_cfg<256, 32, 8, MODE_BF16>(ma, mb, mblo, p, epi, grid, s);
  } else if (rb) {
    launch_cfg<96, 16, 6, MODE_TF32, true>(ma, mb, mblo, p, epi, grid, s);
  } else if (wk_lo) {  // 3xTF32: split stages are twice the size
    if (bn == 64) {
      if (bk == 32) launch_cfg<64, 32, 4, MODE_SPLIT>(ma, mb, mblo, p, epi, grid, s);
      else launch_cfg<64, 16, 8, MODE_SPLIT>(ma, mb, mblo, p, epi, grid, s);
    } else if (bn == 128) {
      if (bk == 32) launch_cfg<128, 32, 3, MODE_SPLIT>(ma, mb, mblo, p, epi, grid, s);
      else launch_cfg<128, 16, 6, MODE_SPLIT>(ma, mb, mblo, p, epi, grid, s);
    } else {
      if (bk == 32) launch_cfg<256, 32, 2, MODE_SPLIT>(ma, mb, mblo, p, epi, grid, s);
      else launch_cfg<256, 16, 4, MODE_SPLIT>(ma, mb, mblo, p, epi, grid, s);
    }
  } else if (bn == 64) {
    if (bk == 32) launch_cfg<64, 32, 8, MODE_TF32>(ma, mb, mblo, p, epi, grid, s);
    else launch_cfg<64, 16, 12, MODE_TF32>(ma, mb, mblo, p, epi, grid, s);
  } else if (bn == 128) {
    if (bk == 32) launch_cfg<128, 32, 6, MODE_TF32>(ma, mb, mblo, p, epi, grid, s);
    else launch_cfg<128, 16, 8, MODE_TF32>(ma, mb, mblo, p, epi, grid, s);
  } else {
    if (bk == 32) launch_cfg<256, 32, 4, MODE_TF32>(ma, mb, mblo, p, epi, grid, s);
    else launch_cfg<256, 16, 6, MODE_TF32>(ma, mb, mblo, p, epi, grid, s);
  }
  if (p.epi_stats && stats_epi(epi)) {
    const int64_t positions = (int64_t)p.B * p.Hq * p.Wq;
    launch_row_stats_reduce(p.epi_rowpart, p.epi_nslots, p.epi_rowlen,
                            (int)(positions / p.epi_rowlen), p.epi_stats, s);
  }
}

}  // namespace dmx
