// SIMT fp32 implicit-GEMM convolution (the FP32 parity build of every
// contraction). Tile 128 positions x 64 columns x 16 taps-channels, 256
// threads, 8x4 outputs per thread, register-staged double buffering.
#include "conv_gemm.cuh"
#include "kernels.h"

namespace dmx {

namespace {

constexpr int BM = 128, BN = 64, BK = 16, TM = 8, TN = 4;
constexpr int AS = BM + 4;  // padded row of the transposed A tile

struct RowAcc {
  int r0;
  double s[2], q[2];
};

template <int PRO>
DMX_DEVICE float load_a(const ConvParams& p, int64_t boff, int y, int x, int b, int k) {
  if (k >= p.K) return 0.f;
  const int tap = k / p.Cin;
  const int ci = k - tap * p.Cin;
  const int iy = y * p.sy + p.dy[tap];
  const int ix = x * p.sx + p.dx[tap];
  if (iy < 0 || iy >= p.Hin || ix < 0 || ix >= p.Win) return 0.f;
  const int64_t addr = boff + (int64_t)iy * p.i_ys + (int64_t)ix * p.i_xs + (int64_t)ci * p.i_cs;
  float v = __ldg(p.x + addr);
  if (PRO == PRO_ADD) v += __ldg(p.x2 + addr);
  if (PRO == PRO_BATCH_AFFINE) {
    const float4 nz = reinterpret_cast<const float4*>(p.pro_scale)[b];
    v = (v - nz.x) * nz.y;
  }
  return v;
}

template <int PRO, int EPI>
__global__ void __launch_bounds__(256) conv_gemm_kernel(const ConvParams p) {
  __shared__ __align__(16) float As[2][BK][AS];
  __shared__ __align__(16) float Bs[2][BK][BN];
  __shared__ int64_t s_boff[BM];
  __shared__ int s_y[BM], s_x[BM], s_b[BM];

  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int64_t M = (int64_t)p.B * p.Hq * p.Wq;
  const int64_t m0 = (int64_t)blockIdx.x * BM;
  const int n0 = blockIdx.y * BN;
  const int64_t plane = (int64_t)p.Hq * p.Wq;

  if (tid < BM) {
    const int64_t pos = m0 + tid;
    if (pos < M) {
      const int b = (int)(pos / plane);
      const int64_t rem = pos - (int64_t)b * plane;
      s_b[tid] = b;
      s_y[tid] = (int)(rem / p.Wq);
      s_x[tid] = (int)(rem % p.Wq);
      s_boff[tid] = (int64_t)b * p.i_bs;
    } else {
      s_b[tid] = -1;
      s_y[tid] = s_x[tid] = 0;
      s_boff[tid] = 0;
    }
  }
  __syncthreads();

  // Loader mapping: A element (row lm + 16*i, k lk), B float4 (row lbk, col lbn).
  const int lk = tid % 16, lm = tid / 16;
  const int lbk = tid / 16, lbn = (tid % 16) * 4;

  float ra[TM];
  float4 rb;
  auto load_tiles = [&](int k0) {
#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const int r = lm + 16 * i;
      ra[i] = s_b[r] >= 0 ? load_a<PRO>(p, s_boff[r], s_y[r], s_x[r], s_b[r], k0 + lk) : 0.f;
    }
    rb = *reinterpret_cast<const float4*>(p.w + (int64_t)(k0 + lbk) * p.Npad + n0 + lbn);
  };
  auto store_tiles = [&](int buf) {
#pragma unroll
    for (int i = 0; i < TM; ++i) As[buf][lk][lm + 16 * i] = ra[i];
    *reinterpret_cast<float4*>(&Bs[buf][lbk][lbn]) = rb;
  };

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

  const int ktiles = (p.K + BK - 1) / BK;
  load_tiles(0);
  store_tiles(0);
  __syncthreads();
  for (int kt = 0; kt < ktiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < ktiles) load_tiles((kt + 1) * BK);
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][k][ty * TM]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][k][ty * TM + 4]);
      const float4 b = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * TN]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (kt + 1 < ktiles) store_tiles(buf ^ 1);
    __syncthreads();
  }

  // ---------------- epilogue ----------------
  const int nb = n0 + tx * TN;
  float bias[TN];
#pragma unroll
  for (int j = 0; j < TN; ++j) bias[j] = p.bias[nb + j];

  constexpr bool kStats = EPI == EPI_RESIDUAL;
  double rs[TM], rq[TM];  // per row: this thread's TN columns, in order
#pragma unroll
  for (int i = 0; i < TM; ++i) rs[i] = rq[i] = 0.0;

#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int m = ty * TM + i;
    const int b = s_b[m];
    if (b < 0) continue;
    const int64_t pos = m0 + m;
    const int64_t orow =
        (int64_t)b * p.o_bs + (int64_t)s_y[m] * p.o_ys + (int64_t)s_x[m] * p.o_xs + p.o_off;
    (void)pos;
    // columns stored for this row (o_lim clips the positions 4x + i >= o_lim)
    const int ncol = p.o_lim ? min(p.N, max(0, (p.o_lim - 4 * s_x[m]) * p.o_lim_ch)) : p.N;
    float v[TN];
#pragma unroll
    for (int j = 0; j < TN; ++j) v[j] = acc[i][j] + bias[j];
    if (EPI == EPI_STORE || EPI == EPI_GELU) {
      if (EPI == EPI_GELU) {
#pragma unroll
        for (int j = 0; j < TN; ++j) v[j] = gelu(v[j]);
      }
      if (EPI == EPI_STORE && p.round_out) {
#pragma unroll
        for (int j = 0; j < TN; ++j) v[j] = round_tf32(v[j]);
      }
      if (EPI == EPI_STORE && p.vt_out) {
        const int64_t bb = pos / p.vt_ntok, tok = pos % p.vt_ntok;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
          const int n = nb + j;
          if (n >= p.vt_col0 && n < ncol) {
            const int c = n - p.vt_col0;
            p.vt_out[((bb * 8 + c / 64) * 64 + c % 64) * (int64_t)p.vt_ntok + tok] = v[j];
          }
        }
      }
      if (p.epi_add) {
        const float* ad = p.epi_add + orow + nb;
#pragma unroll
        for (int j = 0; j < TN; ++j)
          if (nb + j < ncol) v[j] += ad[j];
      }
      float* o = p.out + orow + nb;
      if (nb + TN <= ncol && ((orow & 3) == 0)) {
        *reinterpret_cast<float4*>(o) = make_float4(v[0], v[1], v[2], v[3]);
      } else {
#pragma unroll
        for (int j = 0; j < TN; ++j)
          if (nb + j < ncol) o[j] = v[j];
      }
    }
    if (EPI == EPI_GLU || EPI == EPI_GLU_EMB) {
#pragma unroll
      for (int j = 0; j < TN; j += 2) {
        const int n = nb + j;
        if (n < ncol) {
          const int c = n / 2;
          float g = v[j] * sigmoid(v[j + 1]);
          if (EPI == EPI_GLU_EMB) g += p.epi_emb[(int64_t)s_y[m] * (p.N / 2) + c];
          p.out[orow + c] = g;
        }
      }
    }
    if (EPI == EPI_RESIDUAL) {
      float* o = p.out + orow + nb;
      const float* r = p.epi_res + orow + nb;
#pragma unroll
      for (int j = 0; j < TN; ++j)
        if (nb + j < ncol) {
          v[j] = r[j] + p.epi_gamma[nb + j] * v[j];
          o[j] = v[j];
        }
    }
    if (kStats && p.epi_stats) {
#pragma unroll
      for (int j = 0; j < TN; ++j)
        if (nb + j < ncol) {
          const double d = v[j];
          rs[i] += d;
          rq[i] += d * d;
        }
    }
  }
  if (kStats && p.epi_stats) {
    // the 16 threads of a row (tx, one half-warp) combine their column sums in a
    // fixed butterfly; one partial per (position, column tile) goes to the
    // scratch for the ordered reduction after the launch (no atomics)
#pragma unroll
    for (int i = 0; i < TM; ++i) {
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], o);
        rq[i] += __shfl_xor_sync(0xffffffffu, rq[i], o);
      }
      const int m = ty * TM + i;
      if (tx == 0 && s_b[m] >= 0) {
        double* e = p.epi_rowpart + ((m0 + m) * gridDim.y + blockIdx.y) * 2;
        e[0] = rs[i];
        e[1] = rq[i];
      }
    }
  }
}

template <int PRO>
void dispatch_epi(const ConvParams& p, int epi, dim3 grid, cudaStream_t s) {
  switch (epi) {
    case EPI_STORE: conv_gemm_kernel<PRO, EPI_STORE><<<grid, 256, 0, s>>>(p); break;
    case EPI_GELU: conv_gemm_kernel<PRO, EPI_GELU><<<grid, 256, 0, s>>>(p); break;
    case EPI_GLU: conv_gemm_kernel<PRO, EPI_GLU><<<grid, 256, 0, s>>>(p); break;
    case EPI_GLU_EMB: conv_gemm_kernel<PRO, EPI_GLU_EMB><<<grid, 256, 0, s>>>(p); break;
    case EPI_RESIDUAL: conv_gemm_kernel<PRO, EPI_RESIDUAL><<<grid, 256, 0, s>>>(p); break;
  }
}

}  // namespace

int conv_gemm_stat_slots(int N) { return (N + BN - 1) / BN; }

void launch_conv_gemm(const ConvParams& p, int pro, int epi, cudaStream_t s) {
  const int64_t M = (int64_t)p.B * p.Hq * p.Wq;
  dim3 grid((unsigned)((M + BM - 1) / BM), (unsigned)((p.N + BN - 1) / BN));
  switch (pro) {
    case PRO_NONE: dispatch_epi<PRO_NONE>(p, epi, grid, s); break;
    case PRO_BATCH_AFFINE: dispatch_epi<PRO_BATCH_AFFINE>(p, epi, grid, s); break;
    case PRO_ADD: dispatch_epi<PRO_ADD>(p, epi, grid, s); break;
  }
  if (epi == EPI_RESIDUAL && p.epi_stats)
    launch_row_stats_reduce(p.epi_rowpart, (int)grid.y, p.epi_rowlen, (int)(M / p.epi_rowlen),
                            p.epi_stats, s);
}

}  // namespace dmx
