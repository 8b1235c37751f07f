// Flash attention on the tensor cores (tcgen05 kind::tf32, TMEM accumulators)
// for nn.MultiheadAttention with 8 heads of 64 (host.rs:1199-1312,
// ops.rs:1350-1458): softmax(q k^T / 8) v, never materialising the score
// matrix.
//
// One CTA = 128 queries of one (segment, head). Warp 0 streams K and V^T tiles
// of 64 keys with TMA into a 3-deep ring (both K-major B operands: K for
// S = Q K^T, and V^T — written by the projection GEMM's epilogue as
// (segment, head, dim, key) — for O = P V);
// warp 1 issues the MMAs; warps 2-5 own one query row each: they read the
// score row from TMEM, run the online softmax (running max, rescale, row
// sum), write P rounded to nearest tf32 into a 128B-swizzled K-major tile,
// and fold each tile's P V into register accumulators. q, k, v arrive already
// rounded to nearest tf32 by the projection GEMM, so the tensor core's operand
// truncation is exact. No load uses cluster multicast.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "tc_common.cuh"
#include "tc_gemm.cuh"

namespace dmx {

namespace {

constexpr int QT = 128;   // queries per CTA
constexpr int KT = 64;    // keys per tile
constexpr int HD = 64;    // head dim
constexpr int STAGES = 3;
constexpr int CHUNK = 128 * 128;             // one 128-row x 128-byte swizzled chunk
constexpr int KCHUNK = KT * 128;             // one 64-row x 128-byte chunk
constexpr int Q_BYTES = 2 * CHUNK;           // 128 x 64 fp32
constexpr int KV_BYTES = 2 * KCHUNK;         // 64 x 64 fp32 (two 32-column boxes)
constexpr int STAGE_BYTES = 2 * KV_BYTES;    // K then V
constexpr int P_BYTES = 2 * CHUNK;           // 128 x 64 fp32
constexpr int SMEM_BYTES = Q_BYTES + STAGES * STAGE_BYTES + P_BYTES + 1024 + 256;

struct AttnParams {
  int heads;
  int nq, nk;
  int q_col, k_col, v_col;  // column of head 0 in each source matrix
  float* out;
  int ldo;
  float scale;
  int* err;
};

__global__ void __launch_bounds__(192, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmKV,
                        const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* Qs = smem;
  unsigned char* KVs = Qs + Q_BYTES;
  unsigned char* Ps = KVs + STAGES * STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(Ps + P_BYTES);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + STAGES;
  uint64_t* s_full = kv_empty + STAGES;
  uint64_t* p_full = s_full + 1;
  uint64_t* o_full = p_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int q0 = blockIdx.x * QT, h = blockIdx.y, b = blockIdx.z;
  if (p.err && *reinterpret_cast<volatile int*>(p.err) != 0) return;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(o_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(128));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_s = tmem, tmem_o = tmem + 64;
  const int ntiles = p.nk / KT;
  const int qrow0 = b * p.nq + q0, krow0 = b * p.nk;

  if (warp == 0) {
    if (lane == 0) {
      mbar_expect_tx(q_full, Q_BYTES);
      for (int c = 0; c < 2; ++c)
        tma_load_2d(Qs + c * CHUNK, &tmQ, q_full, p.q_col + h * HD + 32 * c, qrow0);
      for (int j = 0; j < ntiles; ++j) {
        const int s = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        if (!mbar_wait(&kv_empty[s], ph ^ 1, p.err, 11)) break;
        unsigned char* st = KVs + s * STAGE_BYTES;
        mbar_expect_tx(&kv_full[s], STAGE_BYTES);
        for (int c = 0; c < 2; ++c)
          tma_load_2d(st + c * KCHUNK, &tmKV, &kv_full[s], p.k_col + h * HD + 32 * c, krow0 + j * KT);
        // V^T rows (b, h, dim), keys 32c..32c+31 of this tile per box
        for (int c = 0; c < 2; ++c)
          tma_load_2d(st + KV_BYTES + c * KCHUNK, &tmV, &kv_full[s], j * KT + 32 * c,
                      (b * p.heads + h) * HD);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // S = Q K^T and O = P V: M=128, N=64, all operands K-major.
      constexpr uint32_t idesc_s = (1u << 4) | (2u << 7) | (2u << 10) | ((64u >> 3) << 17) |
                                   ((128u >> 4) << 24);
      bool ok = mbar_wait(q_full, 0, p.err, 12);
      const uint32_t q_addr = smem_u32(Qs), p_addr = smem_u32(Ps);
      for (int j = 0; j < ntiles && ok; ++j) {
        const int s = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        if (!mbar_wait(&kv_full[s], ph, p.err, 13)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t k_addr = smem_u32(KVs + s * STAGE_BYTES);
        const uint32_t v_addr = k_addr + KV_BYTES;
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_tf32(tmem_s, umma_desc_k(q_addr + c * CHUNK + k * 32, 128),
                      umma_desc_k(k_addr + c * KCHUNK + k * 32, 128), idesc_s, (c | k) != 0);
        umma_commit(s_full);
        if (!mbar_wait(p_full, j & 1, p.err, 14)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        // K = 64 keys in steps of 8: P chunk kc and V^T chunk kc hold keys
        // 32kc..32kc+31, 32 bytes per step inside the 128-byte rows.
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t pa = p_addr + (kk / 4) * CHUNK + (kk % 4) * 32;
          const uint32_t va = v_addr + (kk / 4) * KCHUNK + (kk % 4) * 32;
          umma_tf32(tmem_o, umma_desc_k(pa, 128), umma_desc_k(va, 128), idesc_s, kk != 0);
        }
        umma_commit(o_full);
        umma_commit(&kv_empty[s]);
      }
    }
  } else {
    const int quarter = warp % 4;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const float kLog2e = 1.4426950408889634f;
    float acc[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) acc[i] = 0.f;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      if (ok && !mbar_wait(s_full, j & 1, p.err, 15)) ok = false;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      float sv[64];
      __syncwarp();
      tmem_ld32(tmem_s + lane_base, sv);
      tmem_ld32(tmem_s + lane_base + 32, sv + 32);
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        sv[i] *= p.scale;
        mx = fmaxf(mx, sv[i]);
      }
      const float mnew = fmaxf(m, mx);
      const float corr = exp2f((m - mnew) * kLog2e);
      float rs = 0.f;
      // P, rounded to nearest tf32, into the two swizzled K-major chunks
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        unsigned char* row = Ps + c * CHUNK + r * 128;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          float4 q4;
          const int i = c * 32 + u * 4;
          q4.x = round_tf32(exp2f((sv[i] - mnew) * kLog2e));
          q4.y = round_tf32(exp2f((sv[i + 1] - mnew) * kLog2e));
          q4.z = round_tf32(exp2f((sv[i + 2] - mnew) * kLog2e));
          q4.w = round_tf32(exp2f((sv[i + 3] - mnew) * kLog2e));
          rs += (q4.x + q4.y) + (q4.z + q4.w);
          *reinterpret_cast<float4*>(row + ((u ^ (r & 7)) << 4)) = q4;
        }
      }
      l = l * corr + rs;
      m = mnew;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(p_full)) : "memory");
      if (ok && !mbar_wait(o_full, j & 1, p.err, 16)) ok = false;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      float ov[64];
      __syncwarp();
      tmem_ld32(tmem_o + lane_base, ov);
      tmem_ld32(tmem_o + lane_base + 32, ov + 32);
#pragma unroll
      for (int i = 0; i < HD; ++i) acc[i] = acc[i] * corr + ov[i];
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    if (ok && q0 + r < p.nq) {
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      float* o = p.out + (int64_t)(qrow0 + r) * p.ldo + h * HD;
#pragma unroll
      for (int i = 0; i < HD; i += 4)
        *reinterpret_cast<float4*>(o + i) =
            make_float4(acc[i] * inv, acc[i + 1] * inv, acc[i + 2] * inv, acc[i + 3] * inv);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(128));
  }
}

}  // namespace

// q (rows, ldq) with head h at column q_col + 64h; k / v in `kv` (rows, ldkv)
// at k_col / v_col + 64h; out (rows, ldo). nk must be a multiple of 64.
bool launch_attention_tc(const float* q, int ldq, int q_col, const float* kv, int ldkv, int k_col,
                         int v_col, const float* vt, float* out, int ldo, int B, int heads, int nq,
                         int nk, float scale, int* err, cudaStream_t s) {
  if (nk % KT != 0 || (ldq * 4) % 16 || (ldkv * 4) % 16 || ldkv % 32) return false;
  if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(kv) & 15) ||
      (reinterpret_cast<uintptr_t>(vt) & 15) || heads * HD > 4096)
    return false;
  CUtensorMap mq, mkv;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)ldq, (cuuint64_t)B * nq};
    const cuuint64_t str[1] = {(cuuint64_t)ldq * 4};
    const cuuint32_t box[2] = {32, QT};
    if (!make_tensor_map(&mq, q, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B)) return false;
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)ldkv, (cuuint64_t)B * nk};
    const cuuint64_t str[1] = {(cuuint64_t)ldkv * 4};
    const cuuint32_t box[2] = {32, KT};
    if (!make_tensor_map(&mkv, kv, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B)) return false;
  }
  CUtensorMap mv;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)nk, (cuuint64_t)B * heads * HD};
    const cuuint64_t str[1] = {(cuuint64_t)nk * 4};
    const cuuint32_t box[2] = {32, HD};
    if (!make_tensor_map(&mv, vt, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B)) return false;
  }
  AttnParams p;
  p.heads = heads;
  p.nq = nq;
  p.nk = nk;
  p.q_col = q_col;
  p.k_col = k_col;
  p.v_col = v_col;
  p.out = out;
  p.ldo = ldo;
  p.scale = scale;
  p.err = err;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         SMEM_BYTES);
    attr = true;
  }
  attention_tc_kernel<<<dim3((nq + QT - 1) / QT, heads, B), 192, SMEM_BYTES, s>>>(mq, mkv, mv, p);
  return true;
}

}  // namespace dmx
