// Flash attention on the tensor cores (tcgen05 kind::tf32, TMEM accumulators)
// for nn.MultiheadAttention with 8 heads of 64 (host.rs:1199-1312,
// ops.rs:1350-1458): softmax(q k^T / 8) v, never materialising the score
// matrix.
//
// One CTA = 128 queries of one (segment, head); two CTAs share an SM, so one's
// softmax overlaps the other's MMAs. Tensor memory holds Q (the A operand of
// S = Q K^T), two S buffers (each overwritten in place by its P, the A operand
// of O += P V) and the O accumulator; shared memory holds only the K / V^T
// ring (3 x 64 keys, both K-major B operands; V^T is written by the projection
// GEMM's epilogue as (segment, head, dim, key)).
//
// Warp 0 streams K and V^T with TMA; warp 1 issues the MMAs, S of key tile
// j+1 ahead of P V of tile j; warps 2-5 own one query row each: they load the
// row of Q into TMEM, then per key tile read S, run the online softmax and
// write P back over S (truncated to tf32, as the tensor core reads it, so the
// row sum adds exactly the weights the MMA uses). The running max is only
// raised when a row's new maximum exceeds it by more than 2^8 (then O is
// rescaled in TMEM); otherwise P = exp(s - m) with the stale m, which is
// exact algebra and stays below 2^8. q, k, v arrive rounded to nearest tf32
// by the projection GEMM, so the tensor core's operand truncation is exact.
//
// The bf16 variant (the BF16 build) runs both products on kind::f16 with
// bf16 q, k and V^T stored so by the projection GEMMs: TMA also brings the
// CTA's Q tile into shared memory, and the softmax warps write P, rounded to
// bf16, into a shared-memory buffer per S buffer instead of over S; both are
// K-major, 128-byte swizzled A operands. The row sum comes from the MMA: 16
// rows of ones after each V^T tile make columns 64..79 of the P V^T
// accumulator the sums of P exactly as the tensor core adds them, so the
// softmax warps do not add the weights themselves. No load uses cluster
// multicast.
#include <cudaTypedefs.h>

#include "common.cuh"
#include <cuda_bf16.h>

#include "tc_common.cuh"
#include "tc_gemm.cuh"

namespace dmx {

namespace {

constexpr int QT = 128;   // queries per CTA
constexpr int KT = 64;    // keys per tile
constexpr int HD = 64;    // head dim
constexpr int STAGES = 3;
constexpr int KCHUNK = KT * 128;             // one 64-row x 128-byte swizzled chunk

// Shared memory: the K / V^T ring (fp32: two 32-column chunks per operand;
// bf16: one 64-column chunk, and after V^T 16 rows of ones, so P V^T's
// columns 64..79 are the row sums of P as the tensor core adds them), then
// for bf16 the Q tile and two P buffers.
template <bool BF>
struct AttnSmem {
  static constexpr int KV_BYTES = BF ? KCHUNK : 2 * KCHUNK;  // 64 x 64 values
  static constexpr int ONES_BYTES = BF ? 16 * 128 : 0;        // 16 rows x 64 bf16 ones
  static constexpr int STAGE_BYTES = 2 * KV_BYTES + ONES_BYTES;  // K, V^T (, ones)
  static constexpr int Q_BYTES = BF ? QT * 128 : 0;           // 128 rows x 64 bf16
  static constexpr int P_BYTES = BF ? QT * 128 : 0;           // one P buffer, 128 x 64 bf16
  static constexpr int OFF_Q = STAGES * STAGE_BYTES;
  static constexpr int OFF_P = OFF_Q + Q_BYTES;
  static constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
  static constexpr int TOTAL = OFF_BAR + 256 + 1024 /*align*/;
};
// TMEM columns. fp32: Q at 0, S buffers at 64 and 128, O at 192. bf16: O
// (64 columns) and the row sums (16 equal columns) at 0, S buffers at 128 and
// 192.
constexpr uint32_t TM_Q = 0, TM_S = 64, TM_O = 192;
constexpr uint32_t TM_S_BF = 128, TM_O_BF = 0;
constexpr float kRescale = 8.0f;  // log2 of the largest P tolerated before O is rescaled

// 2^x by the hardware approximation (PTX ex2.approx.ftz: relative error near
// 2^-22, results below 2^-126 flushed to 0), ample for P that is rounded to
// tf32 next.
DMX_DEVICE float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

DMX_DEVICE float trunc_tf32(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

DMX_DEVICE float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct AttnParams {
  const float* q;  // fp32 variant: the q rows (the bf16 variant loads Q by TMA)
  int ldq;
  int heads;
  int nq, nk;
  int q_col, k_col, v_col;  // column of head 0 in each source matrix
  float* out;
  uint16_t* out16;  // bf16 output instead of `out` (the A operand of a bf16 GEMM)
  int ldo;
  float scale;
  int* err;
};

template <bool BF>
__global__ void __launch_bounds__(192, 2)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmKV,
                        const __grid_constant__ CUtensorMap tmV,
                        const __grid_constant__ CUtensorMap tmQ, const AttnParams p) {
  using L = AttnSmem<BF>;
  constexpr int STAGE_BYTES = L::STAGE_BYTES, KV_BYTES = L::KV_BYTES;
  constexpr uint32_t tmS = BF ? TM_S_BF : TM_S, tmO = BF ? TM_O_BF : TM_O;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* KVs = smem;
  unsigned char* Qs = smem + L::OFF_Q;  // bf16: the Q tile
  unsigned char* Ps = smem + L::OFF_P;  // bf16: P buffers [2]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars;                // Q rows in TMEM (128 arrivals)
  uint64_t* kv_full = q_full + 1;         // [STAGES]
  uint64_t* kv_empty = kv_full + STAGES;  // [STAGES]
  uint64_t* s_full = kv_empty + STAGES;   // [2] S_j in buffer j%2
  uint64_t* p_full = s_full + 2;          // [2] P_j in buffer j%2 (128 arrivals)
  uint64_t* pv_done = p_full + 2;         // [2] P_j V_j complete
  uint64_t* o_final = pv_done + 2;        // every MMA complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_final + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int q0 = blockIdx.x * QT, h = blockIdx.y, b = blockIdx.z;
  if (p.err && *reinterpret_cast<volatile int*>(p.err) != 0) return;

  if (threadIdx.x == 0) {
    mbar_init(q_full, BF ? 1 : 128);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(o_final, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (BF) {
    // the ones rows after each stage's V^T (bf16 1.0; swizzling leaves them as they are)
    for (int i = threadIdx.x; i < STAGES * L::ONES_BYTES / 16; i += blockDim.x) {
      const int s = i / (L::ONES_BYTES / 16), c = i % (L::ONES_BYTES / 16);
      *reinterpret_cast<uint4*>(KVs + s * STAGE_BYTES + 2 * KV_BYTES + 16 * c) =
          make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(256));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const int ntiles = p.nk / KT;
  const int krow0 = b * p.nk;

  if (warp == 0) {
    if (lane == 0) {
      if (BF) {
        // the Q tile: queries q0 .. q0 + 127 of this (segment, head), two 64-row boxes
        // (rows past the segment's queries are read but their outputs are dropped)
        mbar_expect_tx(q_full, L::Q_BYTES);
        for (int c = 0; c < 2; ++c)
          tma_load_2d(Qs + c * KCHUNK, &tmQ, q_full, p.q_col + h * HD, b * p.nq + q0 + 64 * c);
      }
      for (int j = 0; j < ntiles; ++j) {
        const int s = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        if (!mbar_wait(&kv_empty[s], ph ^ 1, p.err, 11)) break;
        unsigned char* st = KVs + s * STAGE_BYTES;
        mbar_expect_tx(&kv_full[s], 2 * KV_BYTES);  // K and V^T (not the ones rows)
        if (BF) {
          // 64 keys x 64 dims of k, and V^T rows (b, h, dim) over this tile's 64 keys
          tma_load_2d(st, &tmKV, &kv_full[s], p.k_col + h * HD, krow0 + j * KT);
          tma_load_2d(st + KV_BYTES, &tmV, &kv_full[s], j * KT, (b * p.heads + h) * HD);
        } else {
          for (int c = 0; c < 2; ++c)
            tma_load_2d(st + c * KCHUNK, &tmKV, &kv_full[s], p.k_col + h * HD + 32 * c, krow0 + j * KT);
          // V^T rows (b, h, dim), keys 32c..32c+31 of this tile per box
          for (int c = 0; c < 2; ++c)
            tma_load_2d(st + KV_BYTES + c * KCHUNK, &tmV, &kv_full[s], j * KT + 32 * c,
                        (b * p.heads + h) * HD);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // S = Q K^T and O = P V: M=128, N=64; B K-major in smem; A from TMEM
      // (tf32) or K-major in smem (bf16)
      constexpr uint32_t ab = BF ? 1u : 2u;
      constexpr uint32_t idesc = (1u << 4) | (ab << 7) | (ab << 10) | ((64u >> 3) << 17) |
                                 ((128u >> 4) << 24);
      // bf16 P V^T: N = 80, V^T's 64 rows and the 16 ones rows after them
      constexpr uint32_t idesc_pv = BF ? (1u << 4) | (ab << 7) | (ab << 10) | ((80u >> 3) << 17) |
                                             ((128u >> 4) << 24)
                                       : idesc;
      bool ok = mbar_wait(q_full, 0, p.err, 12);
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      // S_j = Q K_j^T into buffer j%2
      auto issue_s = [&](int j) -> bool {
        const int s = j % STAGES;
        if (!mbar_wait(&kv_full[s], (j / STAGES) & 1, p.err, 13)) return false;
        // buffer j%2 was last read (as P_{j-2}) by P V of tile j-2
        if (j >= 2 && !mbar_wait(&pv_done[j & 1], ((j - 2) >> 1) & 1, p.err, 17)) return false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t k_addr = smem_u32(KVs + s * STAGE_BYTES);
        const uint32_t d = tmem + tmS + (uint32_t)((j & 1) * 64);
        if (BF) {
          const uint32_t q_addr = smem_u32(Qs);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(d, umma_desc_k(q_addr + kk * 32, 128), umma_desc_k(k_addr + kk * 32, 128), idesc,
                      kk != 0);
        } else {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_tf32_ta(d, tmem + TM_Q + 8 * kk,
                         umma_desc_k(k_addr + (kk / 4) * KCHUNK + (kk % 4) * 32, 128), idesc, kk != 0);
        }
        umma_commit(&s_full[j & 1]);
        return true;
      };
      if (ok && ntiles > 0) ok = issue_s(0);
      for (int j = 0; j < ntiles && ok; ++j) {
        if (j + 1 < ntiles && !issue_s(j + 1)) break;
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1, p.err, 14)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t v_addr = smem_u32(KVs + (j % STAGES) * STAGE_BYTES) + KV_BYTES;
        if (BF) {
          // K = 64 keys in steps of 16 across P's and V^T's 128-byte rows
          const uint32_t p_addr = smem_u32(Ps + (j & 1) * L::P_BYTES);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + tmO, umma_desc_k(p_addr + kk * 32, 128),
                      umma_desc_k(v_addr + kk * 32, 128), idesc_pv, (j | kk) != 0);
        } else {
          const uint32_t pa = tmem + tmS + (uint32_t)((j & 1) * 64);
          // K = 64 keys in steps of 8: V^T chunk kc holds keys 32kc..32kc+31,
          // 32 bytes per step inside its 128-byte rows
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_tf32_ta(tmem + tmO, pa + 8 * kk,
                         umma_desc_k(v_addr + (kk / 4) * KCHUNK + (kk % 4) * 32, 128), idesc,
                         (j | kk) != 0);
        }
        umma_commit(&pv_done[j & 1]);
        umma_commit(&kv_empty[j % STAGES]);
      }
      umma_commit(o_final);
    }
  } else {
    const int quarter = warp % 4;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const float kLog2e = 1.4426950408889634f;
    const float sl = p.scale * kLog2e;  // scores in log2 units
    const bool qvalid = q0 + r < p.nq;
    if (!BF) {
      // this row of Q into TMEM columns [TM_Q, TM_Q + 64)
      float qv[64];
      const float* src = p.q + (int64_t)(b * p.nq + q0 + r) * p.ldq + p.q_col + h * HD;
#pragma unroll
      for (int i = 0; i < HD; i += 4) {
        const float4 t = qvalid ? *reinterpret_cast<const float4*>(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        qv[i] = t.x;
        qv[i + 1] = t.y;
        qv[i + 2] = t.z;
        qv[i + 3] = t.w;
      }
      __syncwarp();
      tmem_st32(tmem + lane_base + TM_Q, qv);
      tmem_st32(tmem + lane_base + TM_Q + 32, qv + 32);
      tmem_st_wait();
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(q_full)) : "memory");
    }
    float m = -INFINITY, l = 0.f;  // running max (log2 units) and row sum
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      if (ok && !mbar_wait(&s_full[j & 1], (j >> 1) & 1, p.err, 15)) ok = false;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t sb = tmem + lane_base + tmS + (uint32_t)((j & 1) * 64);
      float sv[64];
      {
        uint32_t sr[64];
        __syncwarp();
        tmem_ld32_nw(sb, sr);
        tmem_ld32_nw(sb + 32, sr + 32);
        tmem_ld_wait<64>(sr);
#pragma unroll
        for (int i = 0; i < 64; ++i) sv[i] = __uint_as_float(sr[i]);
      }
      // the row's maximum over raw scores (sl > 0 keeps the order): three-
      // input max in eight independent chains
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = sv[i];
#pragma unroll
      for (int i = 8; i < 64; i += 2) mx8[(i / 2) % 8] = fmax3(mx8[(i / 2) % 8], sv[i], sv[i + 1]);
      const float mx = fmaxf(fmax3(mx8[0], mx8[1], mx8[2]),
                             fmax3(fmax3(mx8[3], mx8[4], mx8[5]), mx8[6], mx8[7])) * sl;
      const bool raise = mx > m + kRescale;
      if (__any_sync(0xffffffffu, raise)) {
        const float mnew = raise ? mx : m;
        const float corr = m == -INFINITY ? 0.f : exp2f(m - mnew);
        l *= corr;
        m = mnew;
        if (j > 0) {
          // O holds P V of tiles < j: wait for the last one, then scale it
          if (ok && !mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, p.err, 18)) ok = false;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          __syncwarp();
          // (bf16: the row-sum columns 64..79 too; 80..95 are unused)
          float ov[32];
#pragma unroll
          for (int c = 0; c < (BF ? 96 : 64); c += 32) {
            tmem_ld32(tmem + lane_base + tmO + c, ov);
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] *= corr;
            tmem_st32(tmem + lane_base + tmO + c, ov);
          }
          tmem_st_wait();
        }
      }
      // P = 2^(s sl - m) over S in TMEM, with paired f32 arithmetic. The
      // tensor core reads P truncated to tf32, so the row sum adds the
      // truncated values (four independent pair chains) and O / l stays an
      // exact weighted mean of the V rows.
      const float2 sl2 = make_float2(sl, sl), nm2 = make_float2(-m, -m);
      float2 rs4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) rs4[i] = make_float2(0.f, 0.f);
      if (BF) {
        // P rounded to bf16 into row r of P buffer j%2 (128-byte rows, 16-byte
        // chunk c at chunk c ^ (r % 8)); the row sum is the MMA's (ones rows)
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float2 t = __ffma2_rn(make_float2(sv[2 * i], sv[2 * i + 1]), sl2, nm2);
          const __nv_bfloat162 pb = __floats2bfloat162_rn(ex2_approx(t.x), ex2_approx(t.y));
          pk[i] = *reinterpret_cast<const uint32_t*>(&pb);
        }
        unsigned char* prow = Ps + (j & 1) * L::P_BYTES + r * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) =
              make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float2 t = __ffma2_rn(make_float2(sv[2 * i], sv[2 * i + 1]), sl2, nm2);
          sv[2 * i] = trunc_tf32(ex2_approx(t.x));
          sv[2 * i + 1] = trunc_tf32(ex2_approx(t.y));
          rs4[i % 4] = __fadd2_rn(rs4[i % 4], make_float2(sv[2 * i], sv[2 * i + 1]));
        }
        tmem_st32(sb, sv);
        tmem_st32(sb + 32, sv + 32);
        tmem_st_wait();
      }
      if (!BF) {
        rs4[0] = __fadd2_rn(__fadd2_rn(rs4[0], rs4[1]), __fadd2_rn(rs4[2], rs4[3]));
        l += rs4[0].x + rs4[0].y;
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&p_full[j & 1]))
                   : "memory");
    }
    if (ok && !mbar_wait(o_final, 0, p.err, 16)) ok = false;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    float ov[64];
    __syncwarp();
    tmem_ld32(tmem + lane_base + tmO, ov);
    tmem_ld32(tmem + lane_base + tmO + 32, ov + 32);
    if (BF) {
      float ls[16];
      tmem_ld16(tmem + lane_base + tmO + 64, ls);
      l = ls[0];
    }
    if (ok && qvalid && p.out16) {
      // the output feeds only the bf16 out-projection: stored as bf16
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      uint16_t* o = p.out16 + (int64_t)(b * p.nq + q0 + r) * p.ldo + h * HD;
      if ((reinterpret_cast<uintptr_t>(o) & 31) == 0) {
        // the row's 64 values in 32-byte stores
#pragma unroll
        for (int i = 0; i < HD; i += 16) {
          uint32_t w[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const __nv_bfloat162 t =
                __float22bfloat162_rn(make_float2(ov[i + 2 * e] * inv, ov[i + 2 * e + 1] * inv));
            w[e] = *reinterpret_cast<const uint32_t*>(&t);
          }
          st_global8(reinterpret_cast<uint32_t*>(o + i), w);
        }
      } else {
#pragma unroll
        for (int i = 0; i < HD; i += 8) {
          __nv_bfloat162 w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            w[e] = __float22bfloat162_rn(make_float2(ov[i + 2 * e] * inv, ov[i + 2 * e + 1] * inv));
          *reinterpret_cast<uint4*>(o + i) = *reinterpret_cast<const uint4*>(w);
        }
      }
    } else if (ok && qvalid) {
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      float* o = p.out + (int64_t)(b * p.nq + q0 + r) * p.ldo + h * HD;
#pragma unroll
      // the output feeds only the tf32 out-projection: rounded to nearest here
      for (int i = 0; i < HD; i += 4)
        *reinterpret_cast<float4*>(o + i) =
            make_float4(round_tf32(ov[i] * inv), round_tf32(ov[i + 1] * inv),
                        round_tf32(ov[i + 2] * inv), round_tf32(ov[i + 3] * inv));
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256));
  }
}

}  // namespace

// q (rows, ldq) with head h at column q_col + 64h; k / v in `kv` (rows, ldkv)
// at k_col / v_col + 64h; out (rows, ldo). nk must be a multiple of 64.
// bf16_in: q, kv and vt hold bf16 values (the kind::f16 variant).
bool launch_attention_tc(const float* q, int ldq, int q_col, const float* kv, int ldkv, int k_col,
                         int v_col, const float* vt, float* out, int ldo, int B, int heads, int nq,
                         int nk, float scale, int* err, cudaStream_t s, uint16_t* out16,
                         bool bf16_in) {
  if (nk % KT != 0 || ldq % 4 || (q_col % 4) || (ldkv * 4) % 16 || ldkv % 32) return false;
  if (out16 && ((reinterpret_cast<uintptr_t>(out16) & 15) || ldo % 8)) return false;
  if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(kv) & 15) ||
      (reinterpret_cast<uintptr_t>(vt) & 15) || heads * HD > 4096)
    return false;
  const int esz = bf16_in ? 2 : 4;
  const CUtensorMapDataType dt = bf16_in ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  // boxes of 64 rows x 128 bytes: 32 fp32 or 64 bf16 columns
  const cuuint32_t bw = bf16_in ? 64 : 32;
  CUtensorMap mkv, mv, mq;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)ldkv, (cuuint64_t)B * nk};
    const cuuint64_t str[1] = {(cuuint64_t)ldkv * esz};
    const cuuint32_t box[2] = {bw, KT};
    if (!make_tensor_map(&mkv, kv, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B, nullptr, dt))
      return false;
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)nk, (cuuint64_t)B * heads * HD};
    const cuuint64_t str[1] = {(cuuint64_t)nk * esz};
    const cuuint32_t box[2] = {bw, HD};
    if (!make_tensor_map(&mv, vt, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B, nullptr, dt))
      return false;
  }
  mq = mkv;
  if (bf16_in) {
    const cuuint64_t dims[2] = {(cuuint64_t)ldq, (cuuint64_t)B * nq};
    const cuuint64_t str[1] = {(cuuint64_t)ldq * 2};
    const cuuint32_t box[2] = {64, 64};
    if (!make_tensor_map(&mq, q, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B, nullptr, dt))
      return false;
  }
  AttnParams p;
  p.q = q;
  p.ldq = ldq;
  p.heads = heads;
  p.nq = nq;
  p.nk = nk;
  p.q_col = q_col;
  p.k_col = k_col;
  p.v_col = v_col;
  p.out = out;
  p.out16 = out16;
  p.ldo = ldo;
  p.scale = scale;
  p.err = err;
  static PerDevice attr;
  if (attr.first()) {
    cudaFuncSetAttribute(attention_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         AttnSmem<false>::TOTAL);
    cudaFuncSetAttribute(attention_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         AttnSmem<true>::TOTAL);
  }
  const dim3 grid((nq + QT - 1) / QT, heads, B);
  if (bf16_in)
    attention_tc_kernel<true><<<grid, 192, AttnSmem<true>::TOTAL, s>>>(mkv, mv, mq, p);
  else
    attention_tc_kernel<false><<<grid, 192, AttnSmem<false>::TOTAL, s>>>(mkv, mv, mq, p);
  return true;
}

}  // namespace dmx
