// SIMT f32 GEMM, Y[M, N] = X[M, K] . W[N, K]^T (+ bias), for the f32-accurate
// configurations: tf32 tensor-core accumulation changes SPLADE term sets, so
// the f32 path stays on FFMA. 128x128 CTA tile, 16-deep K slices staged
// transposed in shared memory, 8x8 outputs per thread.
//
// Epilogues: plain f32 store, residual add, and the gated activation
// act(gate) * up with gate/up interleaved in 64-row blocks so that one 128-wide
// tile holds matching gate and up columns.
#include "common.cuh"
#include "kernels.h"

namespace inl {

namespace {

constexpr int TM = 128, TN = 128, TK = 16;

template <int ACT>
__device__ __forceinline__ float act_f(float x) {
  if constexpr (ACT == INL_ACT_SILU) return silu_f(x);
  else if constexpr (ACT == INL_ACT_GELU_ERF) return gelu_erf_f(x);
  else return gelu_tanh_f(x);
}

template <int EPI, int ACT>
__global__ void __launch_bounds__(256) gemm_f32_kernel(GemmF32Args g) {
  __shared__ float As[TK][TM + 4];
  __shared__ float Bs[TK][TN + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  for (int k0 = 0; k0 < g.K; k0 += TK) {
    // 128 rows x 16 k per operand = 2048 values, 8 per thread.
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = threadIdx.x + i * 256;
      const int r = idx >> 4, kk = idx & 15;
      const int gk = k0 + kk;
      const int gm = m0 + r, gn = n0 + r;
      As[kk][r] = (gm < g.M && gk < g.K) ? g.A[static_cast<long long>(gm) * g.lda + gk] : 0.f;
      Bs[kk][r] = (gn < g.N && gk < g.K) ? g.W[static_cast<long long>(gn) * g.ldw + gk] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float a[8], b[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = As[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 8; ++j) b[j] = Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = m0 + ty + 16 * i;
    if (r >= g.M) continue;
    if constexpr (EPI == INL_EPI_GATED_BF16) {
      // Tile columns [0,64) = gate, [64,128) = up; output column n0/2 + tx + 16j.
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int cg = n0 + tx + 16 * j;
        if (cg >= g.N) continue;
        float gt = acc[i][j], up = acc[i][j + 4];
        if (g.bias) {
          gt += g.bias[cg];
          up += g.bias[cg + 64];
        }
        g.out[static_cast<long long>(r) * g.ldo + n0 / 2 + tx + 16 * j] = act_f<ACT>(gt) * up;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = n0 + tx + 16 * j;
        if (c >= g.N) continue;
        float v = acc[i][j];
        if (g.bias) v += g.bias[c];
        if constexpr (EPI == INL_EPI_RESID_BF16) v += g.resid[static_cast<long long>(r) * g.ldr + c];
        g.out[static_cast<long long>(r) * g.ldo + c] = v;
      }
    }
  }
}

// Y = X . W^T reduced on the fly into per-segment column maxima: for rows r
// of segment seg[r] (texts), pooled[seg][col] = max over its rows (order-
// encoded ints, atomicMax). Each thread owns 8 consecutive rows x 8 columns
// and flushes one atomic per (segment run, column), so the [M, N] product is
// never stored (the SPLADE decoder: tokens x vocabulary -> texts x vocabulary).
__global__ void __launch_bounds__(256) gemm_f32_segmax_kernel(const float* __restrict__ A, long long lda,
                                                              const float* __restrict__ W, long long ldw, int M,
                                                              int N, int K, const int* __restrict__ seg,
                                                              int* __restrict__ pooled, long long ldp) {
  __shared__ float As[TK][TM + 4];
  __shared__ float Bs[TK][TN + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  for (int k0 = 0; k0 < K; k0 += TK) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = threadIdx.x + i * 256;
      const int r = idx >> 4, kk = idx & 15;
      const int gk = k0 + kk;
      const int gm = m0 + r, gn = n0 + r;
      As[kk][r] = (gm < M && gk < K) ? A[static_cast<long long>(gm) * lda + gk] : 0.f;
      Bs[kk][r] = (gn < N && gk < K) ? W[static_cast<long long>(gn) * ldw + gk] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float a[8], b[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = As[kk][ty * 8 + i];
#pragma unroll
      for (int j = 0; j < 8; ++j) b[j] = Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  int sg[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = m0 + ty * 8 + i;
    sg[i] = r < M ? seg[r] : -1;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int c = n0 + tx + 16 * j;
    if (c >= N) continue;
    int cur = sg[0];
    float mx = acc[0][j];
#pragma unroll
    for (int i = 1; i < 8; ++i) {
      if (sg[i] != cur) {
        if (cur >= 0) atomicMax(pooled + static_cast<long long>(cur) * ldp + c, encode_ordered(mx));
        cur = sg[i];
        mx = acc[i][j];
      } else {
        mx = fmaxf(mx, acc[i][j]);
      }
    }
    if (cur >= 0) atomicMax(pooled + static_cast<long long>(cur) * ldp + c, encode_ordered(mx));
  }
}

}  // namespace

int gemm_f32_tn(const GemmF32Args& g, cudaStream_t s) {
  if (g.M <= 0 || g.N <= 0) return 0;
  if (g.K <= 0) return -1;
  dim3 grid((g.N + TN - 1) / TN, (g.M + TM - 1) / TM);
  switch (g.epi) {
    case INL_EPI_F32: gemm_f32_kernel<INL_EPI_F32, 0><<<grid, 256, 0, s>>>(g); break;
    case INL_EPI_RESID_BF16: gemm_f32_kernel<INL_EPI_RESID_BF16, 0><<<grid, 256, 0, s>>>(g); break;
    case INL_EPI_GATED_BF16:
      if (g.gate_block != 64 || (g.N % 128) != 0) return -1;
      switch (g.act) {
        case INL_ACT_SILU: gemm_f32_kernel<INL_EPI_GATED_BF16, INL_ACT_SILU><<<grid, 256, 0, s>>>(g); break;
        case INL_ACT_GELU_ERF: gemm_f32_kernel<INL_EPI_GATED_BF16, INL_ACT_GELU_ERF><<<grid, 256, 0, s>>>(g); break;
        default: gemm_f32_kernel<INL_EPI_GATED_BF16, INL_ACT_GELU_TANH><<<grid, 256, 0, s>>>(g); break;
      }
      break;
    default: return -1;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int gemm_f32_segmax(const float* A, long long lda, const float* W, long long ldw, int M, int N, int K,
                    const int* seg, int* pooled, long long ldp, cudaStream_t s) {
  if (M <= 0 || N <= 0) return 0;
  if (K <= 0) return -1;
  dim3 grid((N + TN - 1) / TN, (M + TM - 1) / TM);
  gemm_f32_segmax_kernel<<<grid, 256, 0, s>>>(A, lda, W, ldw, M, N, K, seg, pooled, ldp);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace inl
