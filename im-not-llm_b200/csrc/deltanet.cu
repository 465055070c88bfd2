// Gated DeltaNet pieces of the Qwen3.5 "linear_attention" layers
// (crates/inl-late/src/qwen3_5.rs:411-545), over packed variable-length
// texts, in f32:
//
//   causal_conv_silu   depthwise causal convolution over each text's tokens
//                      (zero before its first token), then SiLU
//                      (GatedDeltaNet::causal_conv, qwen3_5.rs:463-479);
//   gated_delta_rule   the gated delta rule per (text, value head) in its
//                      recurrent form, with the per-head gated RMSNorm and
//                      the silu(z) gate fused at the end of each token.
//
// The recurrence, per value head with state S (dk x dv), S_0 = 0:
//   g_t = softplus(a_t + dt_bias) * -exp(A_log),  beta_t = sigmoid(b_t)
//   k_t <- k_t / sqrt(|k_t|^2 + 1e-6),  q_t <- q_t / sqrt(|q_t|^2 + 1e-6) / sqrt(dk)
//   u_t = beta_t (v_t - exp(g_t) S_{t-1}^T k_t)
//   S_t = exp(g_t) S_{t-1} + k_t u_t^T,   o_t = S_t^T q_t
// (the definition the reference pins its chunked form against,
// qwen3_5.rs:960-1000; Yang, Kautz and Hatamizadeh, "Gated Delta Networks").
// Thread c of a CTA owns column c of S in registers, so the state update
// needs no exchange between threads; only the q / k norms and the output
// norm are block reductions.
#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/inl_cuda.h"
#include "../../include/inl_cuda_kernels.h"
#include "common.cuh"
#include "kernels.h"

namespace inl {

int record_error(int code, const std::string& msg);

namespace {

__global__ void causal_conv_silu_kernel(const float* __restrict__ x, long long ldx, int T, int C,
                                        const float* __restrict__ w, int K, const int* __restrict__ pos,
                                        float* __restrict__ out, long long ldo) {
  const long long total = static_cast<long long>(T) * C;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(idx / C);
    const int c = static_cast<int>(idx - static_cast<long long>(t) * C);
    const int p = pos[t];  // tokens of this text before t
    float acc = 0.f;
    for (int j = 0; j < K; ++j) {
      const int back = K - 1 - j;
      if (back <= p) acc += w[static_cast<long long>(c) * K + j] * x[static_cast<long long>(t - back) * ldx + c];
    }
    out[static_cast<long long>(t) * ldo + c] = acc / (1.0f + expf(-acc));
  }
}

constexpr int kMaxDeltaThreads = 128;

template <int DK>
__global__ void __launch_bounds__(kMaxDeltaThreads) gated_delta_kernel(DeltaArgs a) {
  const int text = blockIdx.x, vh = blockIdx.y;
  const int c = threadIdx.x;  // value column
  const int warp = c >> 5, lane = c & 31, nw = blockDim.x >> 5;
  const int kh = vh / (a.nv / a.nk);
  const int s0 = a.cu[text];
  const int L = a.cu[text + 1] - s0;
  __shared__ float sk[DK], sq[DK];
  __shared__ float red[3][kMaxDeltaThreads / 32];
  float S[DK];
#pragma unroll
  for (int r = 0; r < DK; ++r) S[r] = 0.f;
  const float neg_a = -expf(a.a_log[vh]);
  const float dt_bias = a.dt_bias[vh];
  const float wn = c < a.dv ? a.norm_w[c] : 0.f;
  const float q_scale = rsqrtf(static_cast<float>(DK));
  for (int i = 0; i < L; ++i) {
    const long long row = s0 + i;
    const float* mrow = a.mixed + row * a.ld_mixed;
    // q and k of key head kh (q block first, then k block), L2-normalised.
    float qv = 0.f, kv = 0.f;
    if (c < DK) {
      qv = mrow[kh * DK + c];
      kv = mrow[a.nk * DK + kh * DK + c];
    }
    const float pk = warp_sum(kv * kv), pq = warp_sum(qv * qv);
    if (lane == 0) {
      red[0][warp] = pk;
      red[1][warp] = pq;
    }
    __syncthreads();
    float tk = 0.f, tq = 0.f;
    for (int w = 0; w < nw; ++w) {
      tk += red[0][w];
      tq += red[1][w];
    }
    if (c < DK) {
      sk[c] = kv * rsqrtf(tk + 1e-6f);
      sq[c] = qv * rsqrtf(tq + 1e-6f) * q_scale;
    }
    // decay and step size of this token (softplus in its stable form)
    const float ar = a.a_in[row * a.ld_ab + vh] + dt_bias;
    const float sp = fmaxf(ar, 0.f) + log1pf(expf(-fabsf(ar)));
    const float alpha = expf(sp * neg_a);
    const float beta = 1.0f / (1.0f + expf(-a.b_in[row * a.ld_ab + vh]));
    __syncthreads();
    float o = 0.f;
    if (c < a.dv) {
      const float v = mrow[2 * a.nk * DK + vh * a.dv + c];
      float mem = 0.f;
#pragma unroll
      for (int r = 0; r < DK; ++r) {
        S[r] *= alpha;
        mem = fmaf(S[r], sk[r], mem);
      }
      const float u = beta * (v - mem);
#pragma unroll
      for (int r = 0; r < DK; ++r) {
        S[r] = fmaf(sk[r], u, S[r]);
        o = fmaf(S[r], sq[r], o);
      }
    }
    // gated RMSNorm over the head's dv outputs (plain weight), times silu(z)
    const float po = warp_sum(o * o);
    if (lane == 0) red[2][warp] = po;
    __syncthreads();
    float to = 0.f;
    for (int w = 0; w < nw; ++w) to += red[2][w];
    if (c < a.dv) {
      const float z = a.z[row * a.ld_z + vh * a.dv + c];
      const float y = o * rsqrtf(to / static_cast<float>(a.dv) + a.eps) * wn * (z / (1.0f + expf(-z)));
      a.out[row * a.ldo + vh * a.dv + c] = y;
    }
    __syncthreads();  // red, sk and sq are rewritten by the next token
  }
}

template <int DK>
int launch_delta(const DeltaArgs& a, cudaStream_t s) {
  const int threads = ((std::max(DK, a.dv) + 31) / 32) * 32;
  gated_delta_kernel<DK><<<dim3(a.n, a.nv), threads, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace

int causal_conv_silu(const float* x, long long ldx, int T, int C, const float* w, int K, const int* pos, float* out,
                     long long ldo, cudaStream_t s) {
  if (T <= 0 || C <= 0) return 0;
  if (K <= 0 || !x || !w || !pos || !out || ldx < C || ldo < C) return -1;
  const long long total = static_cast<long long>(T) * C;
  const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
  causal_conv_silu_kernel<<<blocks, 256, 0, s>>>(x, ldx, T, C, w, K, pos, out, ldo);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int gated_delta_rule(const DeltaArgs& a, cudaStream_t s) {
  if (a.n <= 0) return 0;
  if (a.nk <= 0 || a.nv <= 0 || a.nv % a.nk != 0 || a.dv <= 0 || a.dv > kMaxDeltaThreads) return -1;
  switch (a.dk) {
    case 8: return launch_delta<8>(a, s);
    case 16: return launch_delta<16>(a, s);
    case 32: return launch_delta<32>(a, s);
    case 64: return launch_delta<64>(a, s);
    case 128: return launch_delta<128>(a, s);
    default: return -1;
  }
}

}  // namespace inl

// ------------------------------------------------------------ C-ABI hooks
namespace {

std::mutex g_delta_mu;
std::vector<void*> g_delta_scratch(2, nullptr);  // [0] cu_seqlens, [1] token positions
std::vector<size_t> g_delta_bytes(2, 0);
int g_delta_device = -1;  // device the scratch lives on

// Grow-only device scratch for the hooks' cu_seqlens and positions, on the
// current device (moved there when a call comes from another device).
bool scratch(int i, size_t bytes) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (dev != g_delta_device) {
    if (g_delta_device >= 0 && cudaSetDevice(g_delta_device) == cudaSuccess) {
      for (int j = 0; j < 2; ++j)
        if (g_delta_scratch[j]) cudaFree(g_delta_scratch[j]);
    }
    if (cudaSetDevice(dev) != cudaSuccess) return false;
    for (int j = 0; j < 2; ++j) {
      g_delta_scratch[j] = nullptr;
      g_delta_bytes[j] = 0;
    }
    g_delta_device = dev;
  }
  if (bytes <= g_delta_bytes[i]) return true;
  if (g_delta_scratch[i]) cudaFree(g_delta_scratch[i]);
  g_delta_scratch[i] = nullptr;
  g_delta_bytes[i] = 0;
  if (cudaMalloc(&g_delta_scratch[i], bytes) != cudaSuccess) return false;
  g_delta_bytes[i] = bytes;
  return true;
}

int check_cu(const int32_t* cu, int n, const char* what) {
  if (!cu) return inl::record_error(INL_ERR_CONFIG, std::string(what) + ": NULL cu_seqlens");
  if (cu[0] != 0) return inl::record_error(INL_ERR_INVALID_INPUT, std::string(what) + ": cu_seqlens must start at 0");
  for (int i = 0; i < n; ++i)
    if (cu[i + 1] < cu[i])
      return inl::record_error(INL_ERR_INVALID_INPUT, std::string(what) + ": cu_seqlens must be non-decreasing");
  return INL_OK;
}

// Copies cu_seqlens to the device; with_pos also fills token positions.
int upload_cu(const int32_t* cu, int n, bool with_pos, cudaStream_t s, int** dcu, int** dpos) {
  const int T = cu[n];
  if (!scratch(0, static_cast<size_t>(n + 1) * 4) || (with_pos && !scratch(1, static_cast<size_t>(T + 1) * 4)))
    return inl::record_error(INL_ERR_INFERENCE, "deltanet hook: scratch allocation failed");
  *dcu = static_cast<int*>(g_delta_scratch[0]);
  if (cudaMemcpyAsync(*dcu, cu, static_cast<size_t>(n + 1) * 4, cudaMemcpyHostToDevice, s) != cudaSuccess)
    return inl::record_error(INL_ERR_INFERENCE, "deltanet hook: cu_seqlens upload failed");
  if (with_pos) {
    *dpos = static_cast<int*>(g_delta_scratch[1]);
    if (inl::token_positions(*dcu, n, T, *dpos, s) != 0)
      return inl::record_error(INL_ERR_INFERENCE, "deltanet hook: positions launch failed");
  }
  return INL_OK;
}

}  // namespace

extern "C" {

int inl_cuda_causal_conv_silu(const float* x, int64_t ldx, int C, const float* w, int K, const int32_t* cu_seqlens_host,
                              int n_texts, float* out, int64_t ldo, void* stream) {
  if (n_texts <= 0) return INL_OK;
  int r = check_cu(cu_seqlens_host, n_texts, "causal_conv_silu");
  if (r) return r;
  if (!x || !w || !out || C <= 0 || K <= 0 || ldx < C || ldo < C)
    return inl::record_error(INL_ERR_INVALID_INPUT, "causal_conv_silu: invalid arguments");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  std::lock_guard<std::mutex> lock(g_delta_mu);
  int *dcu = nullptr, *dpos = nullptr;
  if ((r = upload_cu(cu_seqlens_host, n_texts, true, s, &dcu, &dpos))) return r;
  const int T = cu_seqlens_host[n_texts];
  const int k = inl::causal_conv_silu(x, ldx, T, C, w, K, dpos, out, ldo, s);
  cudaStreamSynchronize(s);  // the scratch is reused by the next call
  if (k == -1) return inl::record_error(INL_ERR_INVALID_INPUT, "causal_conv_silu: invalid arguments");
  if (k != 0) return inl::record_error(INL_ERR_INFERENCE, "causal_conv_silu launch failed");
  return INL_OK;
}

int inl_cuda_gated_delta_rule(const float* mixed, int64_t ld_mixed, const float* b_in, const float* a_in,
                              int64_t ld_ab, const float* z, int64_t ld_z, const float* dt_bias, const float* a_log,
                              const float* norm_w, float eps, int nk, int nv, int dk, int dv,
                              const int32_t* cu_seqlens_host, int n_texts, float* out, int64_t ldo, void* stream) {
  if (n_texts <= 0) return INL_OK;
  int r = check_cu(cu_seqlens_host, n_texts, "gated_delta_rule");
  if (r) return r;
  if (!mixed || !b_in || !a_in || !z || !dt_bias || !a_log || !norm_w || !out)
    return inl::record_error(INL_ERR_CONFIG, "gated_delta_rule: NULL argument");
  if (nk <= 0 || nv <= 0 || dk <= 0 || dv <= 0 || ld_mixed < 2LL * nk * dk + static_cast<long long>(nv) * dv ||
      ld_ab < nv || ld_z < static_cast<long long>(nv) * dv || ldo < static_cast<long long>(nv) * dv)
    return inl::record_error(INL_ERR_INVALID_INPUT, "gated_delta_rule: row strides smaller than the rows");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  std::lock_guard<std::mutex> lock(g_delta_mu);
  int *dcu = nullptr, *dpos = nullptr;
  if ((r = upload_cu(cu_seqlens_host, n_texts, false, s, &dcu, &dpos))) return r;
  inl::DeltaArgs a;
  a.mixed = mixed;
  a.ld_mixed = ld_mixed;
  a.b_in = b_in;
  a.a_in = a_in;
  a.ld_ab = ld_ab;
  a.z = z;
  a.ld_z = ld_z;
  a.dt_bias = dt_bias;
  a.a_log = a_log;
  a.norm_w = norm_w;
  a.eps = eps;
  a.nk = nk;
  a.nv = nv;
  a.dk = dk;
  a.dv = dv;
  a.cu = dcu;
  a.n = n_texts;
  a.out = out;
  a.ldo = ldo;
  const int k = inl::gated_delta_rule(a, s);
  cudaStreamSynchronize(s);  // the scratch is reused by the next call
  if (k == -1)
    return inl::record_error(INL_ERR_INVALID_INPUT,
                             "gated_delta_rule: dk must be 8, 16, 32, 64 or 128, dv at most 128, nv a multiple of nk");
  if (k != 0) return inl::record_error(INL_ERR_INFERENCE, "gated_delta_rule launch failed");
  return INL_OK;
}

}  // extern "C"
