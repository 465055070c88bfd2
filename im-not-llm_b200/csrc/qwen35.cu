// Qwen3.5 gated full attention around the attention kernel
// (crates/inl-late/src/qwen3_5.rs:251-350), f32, packed texts:
//
//   qk_prep_gated     the q projection holds q | gate per head (2 d columns):
//                     q goes to its own buffer, zero-centred RMSNorm (the
//                     1 + w scale folded at load) and RoPE on the first
//                     rotary_dim features (half-split rotation); k gets the
//                     same in place. The gate is left where it is.
//   gate_sigmoid_mul  attention output times sigmoid(gate).
//   attention_small   f32 attention for head_dim 8 / 16 (tiny checkpoints):
//                     one warp per query row, lane j holds output feature j.
#include <cmath>

#include "common.cuh"
#include "kernels.h"

namespace inl {

namespace {

// One warp per (token, head): q heads first (hq), then k heads (hkv).
__global__ void qk_prep_gated_kernel(Qwen35QkArgs a) {
  extern __shared__ float srow[];  // [warps][d]
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31, wi = threadIdx.x >> 5;
  const long long item = static_cast<long long>(blockIdx.x) * warps + wi;
  const int heads = a.hq + a.hkv;
  if (item >= static_cast<long long>(a.T) * heads) return;
  const int t = static_cast<int>(item / heads);
  const int h = static_cast<int>(item - static_cast<long long>(t) * heads);
  const bool is_q = h < a.hq;
  const int d = a.d;
  const float* src = a.qkv + static_cast<long long>(t) * a.ld +
                     (is_q ? static_cast<long long>(h) * 2 * d : static_cast<long long>(a.hq) * 2 * d +
                                                                     static_cast<long long>(h - a.hq) * d);
  float* dst = is_q ? a.q_out + static_cast<long long>(t) * a.ldq + static_cast<long long>(h) * d
                    : a.qkv + static_cast<long long>(t) * a.ld + static_cast<long long>(a.hq) * 2 * d +
                          static_cast<long long>(h - a.hq) * d;
  const float* w = is_q ? a.qw : a.kw;
  float* x = srow + wi * d;
  float ss = 0.f;
  for (int i = lane; i < d; i += 32) {
    const float v = src[i];
    x[i] = v;
    ss += v * v;
  }
  const float inv = rsqrtf(warp_sum(ss) / static_cast<float>(d) + a.eps);
  __syncwarp();
  for (int i = lane; i < d; i += 32) x[i] = x[i] * inv * w[i];
  __syncwarp();
  int p = a.pos[t];
  if (p < 0 || p >= a.max_pos) {
    if (lane == 0 && a.status) atomicCAS(a.status, 0, INL_DEV_BAD_INDEX);
    p = 0;
  }
  const int half = a.rot / 2;
  const float* cr = a.cos + static_cast<long long>(p) * half;
  const float* sr = a.sin + static_cast<long long>(p) * half;
  for (int i = lane; i < d; i += 32) {
    float y = x[i];
    if (i < half) y = x[i] * cr[i] - x[i + half] * sr[i];
    else if (i < a.rot) y = x[i] * cr[i - half] + x[i - half] * sr[i - half];
    dst[i] = y;
  }
}

__global__ void gate_sigmoid_mul_kernel(float* out, long long ldo, const float* gate_base, long long ldg, int T,
                                        int hq, int d) {
  const long long total = static_cast<long long>(T) * hq * d;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int cols = hq * d;
    const int t = static_cast<int>(idx / cols);
    const int c = static_cast<int>(idx - static_cast<long long>(t) * cols);
    const int h = c / d, j = c - (c / d) * d;
    const float g = gate_base[static_cast<long long>(t) * ldg + static_cast<long long>(h) * 2 * d + d + j];
    out[static_cast<long long>(t) * ldo + c] *= 1.0f / (1.0f + expf(-g));
  }
}

constexpr int kSmallQ = 32;  // queries per work item (the f32 work list's block)

__global__ void __launch_bounds__(128) attention_small_kernel(AttnArgs a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int2 wk = a.work[blockIdx.x];
  const int head = blockIdx.y;
  const int kvh = head / (a.hq / a.hkv);
  const int s0 = a.cu[wk.x];
  const int L = a.cu[wk.x + 1] - s0;
  const int d = a.d;
  const float* qb = static_cast<const float*>(a.q);
  const float* kb = static_cast<const float*>(a.k);
  const float* vb = static_cast<const float*>(a.v);
  float* ob = static_cast<float*>(a.out);
  for (int qi = warp; qi < kSmallQ; qi += 4) {
    const int q = wk.y * kSmallQ + qi;
    if (q >= L) break;
    const float qv = lane < d ? qb[static_cast<long long>(s0 + q) * a.ldq + head * d + lane] : 0.f;
    int k_lo = 0, k_hi = L;
    if (a.causal) k_hi = q + 1;
    if (a.window >= 0) {
      k_lo = max(0, q - a.window);
      k_hi = min(k_hi, q + a.window + 1);
    }
    float m = -INFINITY, l = 0.f, acc = 0.f;
    for (int key = k_lo; key < k_hi; ++key) {
      const long long kr = static_cast<long long>(s0 + key);
      const float kv = lane < d ? kb[kr * a.ldk + kvh * d + lane] : 0.f;
      const float sc = warp_sum(qv * kv) * a.scale;
      const float m_new = fmaxf(m, sc);
      const float alpha = expf(m - m_new);
      const float p = expf(sc - m_new);
      const float vv = lane < d ? vb[kr * a.ldv + kvh * d + lane] : 0.f;
      l = l * alpha + p;
      acc = acc * alpha + p * vv;
      m = m_new;
    }
    if (lane < d) ob[static_cast<long long>(s0 + q) * a.ldo + head * d + lane] = l > 0.f ? acc / l : 0.f;
  }
}

}  // namespace

int qk_prep_gated(const Qwen35QkArgs& a, cudaStream_t s) {
  if (a.T <= 0) return 0;
  if (a.hq <= 0 || a.hkv <= 0 || a.d <= 0 || a.rot < 0 || a.rot > a.d || (a.rot & 1)) return -1;
  const int warps = 4;
  const long long items = static_cast<long long>(a.T) * (a.hq + a.hkv);
  const int blocks = static_cast<int>((items + warps - 1) / warps);
  const size_t smem = static_cast<size_t>(warps) * a.d * sizeof(float);
  if (smem > 48 * 1024) return -1;
  qk_prep_gated_kernel<<<blocks, warps * 32, smem, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int gate_sigmoid_mul(float* out, long long ldo, const float* gate_base, long long ldg, int T, int hq, int d,
                     cudaStream_t s) {
  if (T <= 0) return 0;
  const long long total = static_cast<long long>(T) * hq * d;
  const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
  gate_sigmoid_mul_kernel<<<blocks, 256, 0, s>>>(out, ldo, gate_base, ldg, T, hq, d);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int attention_small(const AttnArgs& a, cudaStream_t s) {
  if (a.n_work <= 0) return 0;
  if (a.bf16 || a.d <= 0 || a.d > 32 || a.q_block != kSmallQ) return -1;
  attention_small_kernel<<<dim3(a.n_work, a.hq), 128, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace inl
