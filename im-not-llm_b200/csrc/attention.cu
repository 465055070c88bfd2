// Variable-length attention over packed texts: causal, bidirectional and
// sliding-window (|q - k| <= window), grouped-query (query head h reads KV head
// h / (hq / hkv)), masks computed from positions instead of materialised.
//
// bf16 runs on the tcgen05 kernel of attention_sm100.cu (head_dim 64, 128,
// 256). f32: SIMT kernel for the f32-accurate configurations: 32 queries per CTA,
// 32-key tiles in shared memory, one lane per key for the scores and one lane
// per head dimension slice for the output.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace inl {

namespace {

constexpr int kFQ = 32;  // queries per CTA
constexpr int kFK = 32;  // keys per tile

template <int D>
__global__ void __launch_bounds__(128) attn_f32_kernel(AttnArgs a) {
  constexpr int E = D / 32;      // head-dim values per lane
  constexpr int QW = kFQ / 4;    // queries per warp
  extern __shared__ __align__(128) uint8_t smem[];
  float* sQ = reinterpret_cast<float*>(smem);  // [kFQ][D]
  float* sK = sQ + kFQ * D;                    // [kFK][D+1]
  float* sV = sK + kFK * (D + 1);              // [kFK][D]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int2 wk = a.work[blockIdx.x];
  const int text = wk.x, qb = wk.y;
  const int head = blockIdx.y;
  const int kvh = head / (a.hq / a.hkv);
  const int s0 = a.cu[text];
  const int L = a.cu[text + 1] - s0;
  const int q0 = qb * kFQ;
  if (q0 >= L) return;
  int k_lo = 0, k_hi = L;
  if (a.causal) k_hi = min(L, q0 + kFQ);
  if (a.window >= 0) {
    k_lo = max(0, q0 - a.window);
    k_hi = min(k_hi, q0 + kFQ + a.window);
  }
  const float* qbase = static_cast<const float*>(a.q) + static_cast<long long>(s0) * a.ldq + head * D;
  const float* kbase = static_cast<const float*>(a.k) + static_cast<long long>(s0) * a.ldk + kvh * D;
  const float* vbase = static_cast<const float*>(a.v) + static_cast<long long>(s0) * a.ldv + kvh * D;

  for (int idx = tid; idx < kFQ * D; idx += 128) {
    const int r = idx / D, c = idx - (idx / D) * D;
    sQ[idx] = (q0 + r < L) ? qbase[static_cast<long long>(q0 + r) * a.ldq + c] : 0.f;
  }
  float acc[QW][E];
  float m_r[QW], l_r[QW];
#pragma unroll
  for (int i = 0; i < QW; ++i) {
    m_r[i] = -INFINITY;
    l_r[i] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) acc[i][e] = 0.f;
  }

  for (int kt = (k_lo / kFK) * kFK; kt < k_hi; kt += kFK) {
    __syncthreads();
    for (int idx = tid; idx < kFK * D; idx += 128) {
      const int r = idx / D, c = idx - (idx / D) * D;
      const bool valid = kt + r < L;
      sK[r * (D + 1) + c] = valid ? kbase[static_cast<long long>(kt + r) * a.ldk + c] : 0.f;
      sV[r * D + c] = valid ? vbase[static_cast<long long>(kt + r) * a.ldv + c] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < QW; ++i) {
      const int ql = warp * QW + i;
      const int qr = q0 + ql;
      const int key = kt + lane;
      float sc = 0.f;
      const float* qv = sQ + ql * D;
      const float* kv = sK + lane * (D + 1);
#pragma unroll 8
      for (int c = 0; c < D; ++c) sc += qv[c] * kv[c];
      bool valid = key < L && key >= k_lo;
      if (a.causal) valid = valid && key <= qr;
      if (a.window >= 0) valid = valid && abs(qr - key) <= a.window;
      sc = valid ? sc * a.scale : -INFINITY;
      const float mt = warp_max(sc);
      const float m_new = fmaxf(m_r[i], mt);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = expf(m_r[i] - m_use);
      const float p = expf(sc - m_use);
      l_r[i] = l_r[i] * alpha + warp_sum(p);
      m_r[i] = m_new;
#pragma unroll
      for (int e = 0; e < E; ++e) acc[i][e] *= alpha;
      for (int j = 0; j < kFK; ++j) {
        const float pj = __shfl_sync(0xffffffffu, p, j);
#pragma unroll
        for (int e = 0; e < E; ++e) acc[i][e] += pj * sV[j * D + lane + 32 * e];
      }
    }
  }
  float* obase = static_cast<float*>(a.out) + static_cast<long long>(s0) * a.ldo + head * D;
#pragma unroll
  for (int i = 0; i < QW; ++i) {
    const int qr = q0 + warp * QW + i;
    if (qr >= L) continue;
    const float inv = l_r[i] > 0.f ? 1.0f / l_r[i] : 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) obase[static_cast<long long>(qr) * a.ldo + lane + 32 * e] = acc[i][e] * inv;
  }
}

template <int D>
int launch_f32(const AttnArgs& a, cudaStream_t s) {
  auto kern = attn_f32_kernel<D>;
  constexpr int bytes = (kFQ * D + kFK * (D + 1) + kFK * D) * 4;
  static std::atomic<unsigned long long> attr{0};  // one bit per device
  if (set_smem_limit_once(kern, bytes, attr) != cudaSuccess) return -3;
  dim3 grid(a.n_work, a.hq);
  kern<<<grid, 128, bytes, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace

int attention_q_block(int bf16, int d) {
  if (bf16) return 128;  // the tcgen05 kernel's query tile
  return kFQ;
}

bool attention_supported(int bf16, int d) {
  if (bf16) return d == 64 || d == 128 || d == 256;
  return d == 8 || d == 16 || d == 32 || d == 64 || d == 128 || d == 256;
}

int attention(const AttnArgs& a, cudaStream_t s) {
  if (a.n_work <= 0) return 0;
  if (a.hq <= 0 || a.hkv <= 0 || a.hq % a.hkv != 0) return -1;
  if (a.bf16) return attention_tc(a, a.total_rows, s);  // head_dim 64, 128, 256 (others: -1)
  if (a.q_block != kFQ) return -1;
  switch (a.d) {
    case 8:
    case 16: return attention_small(a, s);  // tiny checkpoints
    case 32: return launch_f32<32>(a, s);
    case 64: return launch_f32<64>(a, s);
    case 128: return launch_f32<128>(a, s);
    case 256: return launch_f32<256>(a, s);
    default: return -1;
  }
}

}  // namespace inl
