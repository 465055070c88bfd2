// Bandwidth-bound kernels of the encoder forward: embedding gather, RMSNorm /
// LayerNorm, per-head q/k norm + RoPE, pooling heads and weight conversion.
// One warp per row (or per token-head) with warp-shuffle reductions; rows are
// read with 16-byte vector loads where the shape allows.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace inl {

namespace {

template <typename T>
__device__ __forceinline__ float ld_f(const T* p, long long i);
template <>
__device__ __forceinline__ float ld_f<float>(const float* p, long long i) { return p[i]; }
template <>
__device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16* p, long long i) {
  return __bfloat162float(p[i]);
}
template <typename T>
__device__ __forceinline__ void st_f(T* p, long long i, float v);
template <>
__device__ __forceinline__ void st_f<float>(float* p, long long i, float v) { p[i] = v; }
template <>
__device__ __forceinline__ void st_f<__nv_bfloat16>(__nv_bfloat16* p, long long i, float v) {
  p[i] = __float2bfloat16_rn(v);
}

// Load 8 consecutive values (16 B for bf16, 32 B for f32) into floats.
template <typename T>
__device__ __forceinline__ void ld8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void ld8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  uint4 w = *reinterpret_cast<const uint4*>(p);
  float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), c = unpack_bf16x2(w.z), d = unpack_bf16x2(w.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}
template <>
__device__ __forceinline__ void ld8<float>(const float* p, float (&v)[8]) {
  float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <typename T>
__device__ __forceinline__ void st8(T* p, const float (&v)[8]);
template <>
__device__ __forceinline__ void st8<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 w;
  w.x = pack_bf16x2(v[0], v[1]); w.y = pack_bf16x2(v[2], v[3]);
  w.z = pack_bf16x2(v[4], v[5]); w.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = w;
}
template <>
__device__ __forceinline__ void st8<float>(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// E = 2, 4 or 8 consecutive values in one vector access (E * sizeof(T) bytes,
// aligned to that size).
template <typename T, int E>
__device__ __forceinline__ void ld_vec(const T* p, float (&v)[E]) {
  if constexpr (E == 8) {
    ld8<T>(p, v);
  } else if constexpr (sizeof(T) == 2) {
    if constexpr (E == 4) {
      const uint2 w = *reinterpret_cast<const uint2*>(p);
      const float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y);
      v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    } else {
      const float2 a = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(p));
      v[0] = a.x; v[1] = a.y;
    }
  } else {
    if constexpr (E == 4) {
      const float4 a = *reinterpret_cast<const float4*>(p);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    } else {
      const float2 a = *reinterpret_cast<const float2*>(p);
      v[0] = a.x; v[1] = a.y;
    }
  }
}
template <typename T, int E>
__device__ __forceinline__ void st_vec(T* p, const float (&v)[E]) {
  if constexpr (E == 8) {
    st8<T>(p, v);
  } else if constexpr (sizeof(T) == 2) {
    if constexpr (E == 4) *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
    else *reinterpret_cast<uint32_t*>(p) = pack_bf16x2(v[0], v[1]);
  } else {
    if constexpr (E == 4) *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    else *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
  }
}

// ------------------------------------------------------------ embedding
template <typename TT, typename TO>
__global__ void embed_gather_kernel(const uint32_t* __restrict__ ids, int T, const TT* __restrict__ table,
                                    int vocab, int H, float scale, TO* __restrict__ out, float* __restrict__ ss_out,
                                    int* status) {
  const int warps = blockDim.x >> 5;
  const long long row = static_cast<long long>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const uint32_t id = ids[row];
  TO* o = out + row * H;
  const bool bad = id >= static_cast<uint32_t>(vocab);
  if (bad && lane == 0 && status) atomicCAS(status, 0, INL_DEV_BAD_INDEX);
  const TT* src = table + static_cast<long long>(bad ? 0u : id) * H;
  if ((H & 7) == 0) {
    const int parts = (H + INL_SS_COLS - 1) / INL_SS_COLS;
    for (int base = 0; base < H; base += 256) {
      const int c = base + lane * 8;
      float s = 0.f;
      if (c < H) {
        float v[8];
        ld8<TT>(src + c, v);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          v[j] = bad ? 0.f : v[j] * scale;
          const float r = sizeof(TO) == 2 ? bf16_round(v[j]) : v[j];
          s = fmaf(r, r, s);
        }
        st8<TO>(o + c, v);
      }
      // 8 lanes x 8 values = one 64-column partial sum of squares
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      s += __shfl_xor_sync(0xffffffffu, s, 4);
      if (ss_out && (lane & 7) == 0 && c < H) ss_out[row * parts + c / INL_SS_COLS] = s;
    }
  } else {
    for (int c = lane; c < H; c += 32) st_f<TO>(o, c, bad ? 0.f : ld_f<TT>(src, c) * scale);
  }
}

// ------------------------------------------------------------ norms
template <bool ACT>
__device__ __forceinline__ float pre_act(float v) {
  if constexpr (ACT) return gelu_erf_f(v);
  else return v;
}

template <typename TI, typename TO, bool LN, bool ACT = false>
__global__ void norm_rows_kernel(const TI* __restrict__ x, long long ldx, const float* __restrict__ w,
                                 const float* __restrict__ b, float eps, int rows, int H, TO* __restrict__ out,
                                 long long ldo) {
  const int warps = blockDim.x >> 5;
  const long long row = static_cast<long long>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const TI* xr = x + row * ldx;
  TO* orow = out + row * ldo;
  const bool vec = (H & 255) == 0;
  float mean = 0.f;
  if (LN) {
    float s = 0.f;
    if (vec) {
      for (int c = lane * 8; c < H; c += 256) {
        float v[8];
        ld8<TI>(xr + c, v);
#pragma unroll
        for (int j = 0; j < 8; ++j) s += pre_act<ACT>(v[j]);
      }
    } else {
      for (int c = lane; c < H; c += 32) s += pre_act<ACT>(ld_f<TI>(xr, c));
    }
    mean = warp_sum(s) / static_cast<float>(H);
  }
  float ss = 0.f;
  if (vec) {
    for (int c = lane * 8; c < H; c += 256) {
      float v[8];
      ld8<TI>(xr + c, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float t = pre_act<ACT>(v[j]) - mean;
        ss += t * t;
      }
    }
  } else {
    for (int c = lane; c < H; c += 32) {
      const float t = pre_act<ACT>(ld_f<TI>(xr, c)) - mean;
      ss += t * t;
    }
  }
  const float inv = rsqrtf(warp_sum(ss) / static_cast<float>(H) + eps);
  if (vec) {
    for (int c = lane * 8; c < H; c += 256) {
      float v[8];
      ld8<TI>(xr + c, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float t = (pre_act<ACT>(v[j]) - mean) * inv;
        if (w) t *= w[c + j];
        if (b) t += b[c + j];
        v[j] = t;
      }
      st8<TO>(orow + c, v);
    }
  } else {
    for (int c = lane; c < H; c += 32) {
      float t = (pre_act<ACT>(ld_f<TI>(xr, c)) - mean) * inv;
      if (w) t *= w[c];
      if (b) t += b[c];
      st_f<TO>(orow, c, t);
    }
  }
}

// The same norm with the row held in registers (H = 256 NC, NC <= 4): one read
// of the row instead of one per pass, the same arithmetic in the same order
// (bit-identical results), weight and bias read as float4.
template <typename TI, typename TO, bool LN, bool ACT, int NC>
__global__ void norm_rows_reg_kernel(const TI* __restrict__ x, long long ldx, const float* __restrict__ w,
                                     const float* __restrict__ b, float eps, int rows, TO* __restrict__ out,
                                     long long ldo) {
  constexpr int H = 256 * NC;
  const int warps = blockDim.x >> 5;
  const long long row = static_cast<long long>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const TI* xr = x + row * ldx;
  TO* orow = out + row * ldo;
  float v[NC][8];
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    ld8<TI>(xr + lane * 8 + 256 * k, v[k]);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[k][j] = pre_act<ACT>(v[k][j]);
  }
  float mean = 0.f;
  if (LN) {
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < NC; ++k)
#pragma unroll
      for (int j = 0; j < 8; ++j) sum += v[k][j];
    mean = warp_sum(sum) / static_cast<float>(H);
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < NC; ++k)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float t = v[k][j] - mean;
      ss += t * t;
    }
  const float inv = rsqrtf(warp_sum(ss) / static_cast<float>(H) + eps);
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    const int c = lane * 8 + 256 * k;
    float wv[8], bv[8];
    if (w) ld8<float>(w + c, wv);
    if (b) ld8<float>(b + c, bv);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float t = (v[k][j] - mean) * inv;
      if (w) t *= wv[j];
      if (b) t += bv[j];
      v[k][j] = t;
    }
    st8<TO>(orow + c, v[k]);
  }
}

// ------------------------------------------------------------ q/k norm + rope
// One warp per (token, head). Lane l holds elements [E*l, E*l+E), E = d/32;
// lanes 0..15 hold the first half of the head, lanes 16..31 the second, so the
// RoPE partner of every element sits in lane l ^ 16.
template <typename T, int E>
__global__ void qk_norm_rope_kernel(QkRopeArgs a) {
  const int warps = blockDim.x >> 5;
  const long long item = static_cast<long long>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int heads = a.hq + a.hkv + (a.v_norm ? a.hkv : 0);
  if (item >= static_cast<long long>(a.T) * heads) return;
  const int t = static_cast<int>(item / heads);
  const int h = static_cast<int>(item - static_cast<long long>(t) * heads);
  const int d = E * 32;
  const int half = d / 2;
  T* row = reinterpret_cast<T*>(a.qkv) + static_cast<long long>(t) * a.ld + static_cast<long long>(h) * d;
  const bool is_q = h < a.hq;
  const bool is_k = !is_q && h < a.hq + a.hkv;
  const float* w = is_q ? a.qw : (is_k ? a.kw : nullptr);
  const bool norm = is_q ? (a.qw != nullptr) : (is_k ? (a.kw != nullptr) : true);
  const bool is_bf16 = sizeof(T) == 2;
  float x[E];
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = ld_f<T>(row, lane * E + e);
  if (norm) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss += x[e] * x[e];
    const float inv = rsqrtf(warp_sum(ss) / static_cast<float>(d) + a.eps);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      float v = x[e] * inv;
      if (w) v *= w[lane * E + e];
      x[e] = is_bf16 ? bf16_round(v) : v;
    }
  }
  if (is_q || is_k) {
    int p = a.pos[t];
    if (p < 0 || p >= a.max_pos) {
      if (lane == 0 && a.status) atomicCAS(a.status, 0, INL_DEV_BAD_INDEX);
      p = 0;
    }
    const float* cr = a.cos + static_cast<long long>(p) * half;
    const float* sr = a.sin + static_cast<long long>(p) * half;
    const bool first = lane < 16;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float other = __shfl_xor_sync(0xffffffffu, x[e], 16);
      const int i = (lane * E + e) - (first ? 0 : half);
      const float c = cr[i], s = sr[i];
      x[e] = first ? (x[e] * c - other * s) : (x[e] * c + other * s);
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e) st_f<T>(row, lane * E + e, x[e]);
}

// Same arithmetic with one vector access per lane for the row (E elements)
// and for its E cos / sin factors, for rows, leading dimension and tables
// aligned to the access size (the host checks).
template <typename T, int E>
__global__ void qk_norm_rope_vec_kernel(QkRopeArgs a) {
  const int warps = blockDim.x >> 5;
  const long long item = static_cast<long long>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int heads = a.hq + a.hkv + (a.v_norm ? a.hkv : 0);
  if (item >= static_cast<long long>(a.T) * heads) return;
  const int t = static_cast<int>(item / heads);
  const int h = static_cast<int>(item - static_cast<long long>(t) * heads);
  constexpr int d = E * 32;
  constexpr int half = d / 2;
  T* row = reinterpret_cast<T*>(a.qkv) + static_cast<long long>(t) * a.ld + static_cast<long long>(h) * d;
  const bool is_q = h < a.hq;
  const bool is_k = !is_q && h < a.hq + a.hkv;
  const float* w = is_q ? a.qw : (is_k ? a.kw : nullptr);
  const bool norm = is_q ? (a.qw != nullptr) : (is_k ? (a.kw != nullptr) : true);
  const bool is_bf16 = sizeof(T) == 2;
  float x[E];
  ld_vec<T, E>(row + lane * E, x);
  if (norm) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss += x[e] * x[e];
    const float inv = rsqrtf(warp_sum(ss) / static_cast<float>(d) + a.eps);
    float wv[E];
    if (w) ld_vec<float, E>(w + lane * E, wv);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      float v = x[e] * inv;
      if (w) v *= wv[e];
      x[e] = is_bf16 ? bf16_round(v) : v;
    }
  }
  if (is_q || is_k) {
    int p = a.pos[t];
    if (p < 0 || p >= a.max_pos) {
      if (lane == 0 && a.status) atomicCAS(a.status, 0, INL_DEV_BAD_INDEX);
      p = 0;
    }
    const bool first = lane < 16;
    const int i0 = lane * E - (first ? 0 : half);
    float c[E], sn[E];
    ld_vec<float, E>(a.cos + static_cast<long long>(p) * half + i0, c);
    ld_vec<float, E>(a.sin + static_cast<long long>(p) * half + i0, sn);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float other = __shfl_xor_sync(0xffffffffu, x[e], 16);
      x[e] = first ? (x[e] * c[e] - other * sn[e]) : (x[e] * c[e] + other * sn[e]);
    }
  }
  st_vec<T, E>(row + lane * E, x);
}

// One warp per token, for heads of 64 or 128 features, where a warp per
// (token, head) has too little to do (a 128- or 256-byte row): the token's
// RoPE factors are read once (E cos and E sin per lane) and its heads are
// processed in groups of four, the group's rows loaded before any is computed.
// Same arithmetic as the per-(token, head) kernels; rows, weights and tables
// aligned to the vector access (the host checks).
template <typename T, int E>
__global__ void qk_norm_rope_tok_kernel(QkRopeArgs a) {
  const int warps = blockDim.x >> 5;
  const long long t = static_cast<long long>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= a.T) return;
  constexpr int d = E * 32;
  constexpr int half = d / 2;
  constexpr int G = 4;
  const int heads = a.hq + a.hkv + (a.v_norm ? a.hkv : 0);
  const bool is_bf16 = sizeof(T) == 2;
  T* base = reinterpret_cast<T*>(a.qkv) + t * a.ld + lane * E;
  const bool first = lane < 16;
  float c[E], sn[E];
  {
    int p = a.pos[t];
    if (p < 0 || p >= a.max_pos) {
      if (lane == 0 && a.status) atomicCAS(a.status, 0, INL_DEV_BAD_INDEX);
      p = 0;
    }
    const int i0 = lane * E - (first ? 0 : half);
    ld_vec<float, E>(a.cos + static_cast<long long>(p) * half + i0, c);
    ld_vec<float, E>(a.sin + static_cast<long long>(p) * half + i0, sn);
  }
  float qw[E], kw[E];
  if (a.qw) ld_vec<float, E>(a.qw + lane * E, qw);
  if (a.kw) ld_vec<float, E>(a.kw + lane * E, kw);
  for (int h0 = 0; h0 < heads; h0 += G) {
    float x[G][E];
#pragma unroll
    for (int g = 0; g < G; ++g)
      if (h0 + g < heads) ld_vec<T, E>(base + static_cast<long long>(h0 + g) * d, x[g]);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int h = h0 + g;
      if (h >= heads) break;  // warp-uniform
      const bool is_q = h < a.hq;
      const bool is_k = !is_q && h < a.hq + a.hkv;
      const bool has_w = is_q ? (a.qw != nullptr) : (is_k ? (a.kw != nullptr) : false);
      const bool norm = is_q ? (a.qw != nullptr) : (is_k ? (a.kw != nullptr) : true);
      if (norm) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) ss += x[g][e] * x[g][e];
        const float inv = rsqrtf(warp_sum(ss) / static_cast<float>(d) + a.eps);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          float v = x[g][e] * inv;
          if (has_w) v *= is_q ? qw[e] : kw[e];
          x[g][e] = is_bf16 ? bf16_round(v) : v;
        }
      }
      if (is_q || is_k) {
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float other = __shfl_xor_sync(0xffffffffu, x[g][e], 16);
          x[g][e] = first ? (x[g][e] * c[e] - other * sn[e]) : (x[g][e] * c[e] + other * sn[e]);
        }
      }
      st_vec<T, E>(base + static_cast<long long>(h) * d, x[g]);
    }
  }
}

// Heads of d <= 32 features (8, 16, 32): one warp per (token, head), lane l < d
// holds element l and its RoPE partner sits in lane l ^ (d / 2).
template <typename T>
__global__ void qk_norm_rope_narrow_kernel(QkRopeArgs a) {
  const int warps = blockDim.x >> 5;
  const long long item = static_cast<long long>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int heads = a.hq + a.hkv + (a.v_norm ? a.hkv : 0);
  if (item >= static_cast<long long>(a.T) * heads) return;
  const int t = static_cast<int>(item / heads);
  const int h = static_cast<int>(item - static_cast<long long>(t) * heads);
  const int d = a.d, half = d / 2;
  const bool on = lane < d;
  T* row = reinterpret_cast<T*>(a.qkv) + static_cast<long long>(t) * a.ld + static_cast<long long>(h) * d;
  const bool is_q = h < a.hq;
  const bool is_k = !is_q && h < a.hq + a.hkv;
  const float* w = is_q ? a.qw : (is_k ? a.kw : nullptr);
  const bool norm = is_q ? (a.qw != nullptr) : (is_k ? (a.kw != nullptr) : true);
  float x = on ? ld_f<T>(row, lane) : 0.f;
  if (norm) {
    const float inv = rsqrtf(warp_sum(x * x) / static_cast<float>(d) + a.eps);
    float v = x * inv;
    if (w && on) v *= w[lane];
    x = sizeof(T) == 2 ? bf16_round(v) : v;
  }
  if (is_q || is_k) {
    int p = a.pos[t];
    if (p < 0 || p >= a.max_pos) {
      if (lane == 0 && a.status) atomicCAS(a.status, 0, INL_DEV_BAD_INDEX);
      p = 0;
    }
    const float other = __shfl_xor_sync(0xffffffffu, x, half);
    if (on) {
      const bool first = lane < half;
      const int i = first ? lane : lane - half;
      const float c = a.cos[static_cast<long long>(p) * half + i], sn = a.sin[static_cast<long long>(p) * half + i];
      x = first ? (x * c - other * sn) : (x * c + other * sn);
    }
  }
  if (on) st_f<T>(row, lane, x);
}

// ------------------------------------------------------------ positions
__global__ void token_positions_kernel(const int* __restrict__ cu, int n, int T, int* __restrict__ pos) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  int lo = 0, hi = n;  // find i with cu[i] <= t < cu[i+1]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (cu[mid] <= t) lo = mid;
    else hi = mid;
  }
  pos[t] = t - cu[lo];
}

// ------------------------------------------------------------ heads
template <typename T>
__global__ void last_token_norm_l2_kernel(const T* __restrict__ h, long long ldh, const int* __restrict__ cu,
                                          int n, const float* __restrict__ w, float eps, int H,
                                          float* __restrict__ out) {
  const int i = blockIdx.x;
  if (i >= n) return;
  __shared__ float red[32];
  const int last = cu[i + 1] - 1;
  float* o = out + static_cast<long long>(i) * H;
  if (last < cu[i]) {  // empty text: zero vector
    for (int c = threadIdx.x; c < H; c += blockDim.x) o[c] = 0.f;
    return;
  }
  const T* row = h + static_cast<long long>(last) * ldh;
  auto block_sum = [&](float v) {
    v = warp_sum(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
    const int nw = blockDim.x >> 5;
    for (int j = 0; j < nw; ++j) t += red[j];
    return t;
  };
  float ss = 0.f;
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    const float v = ld_f<T>(row, c);
    ss += v * v;
  }
  const float inv = rsqrtf(block_sum(ss) / static_cast<float>(H) + eps);
  const bool is_bf16 = sizeof(T) == 2;
  float ss2 = 0.f;
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    float v = ld_f<T>(row, c) * inv * (w ? w[c] : 1.f);
    if (is_bf16) v = bf16_round(v);  // the model-dtype norm output, cast to f32 before L2
    o[c] = v;
    ss2 += v * v;
  }
  const float inv2 = 1.0f / sqrtf(block_sum(ss2) + 1e-12f);
  for (int c = threadIdx.x; c < H; c += blockDim.x) o[c] *= inv2;
}

__global__ void rows_l2_kernel(const float* __restrict__ x, long long ldx, int rows, int D, float clamp_min,
                               float* __restrict__ out, long long ldo) {
  const int warps = blockDim.x >> 5;
  const long long row = static_cast<long long>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + row * ldx;
  float ss = 0.f;
  for (int c = lane; c < D; c += 32) ss += xr[c] * xr[c];
  const float tot = warp_sum(ss);
  const float inv = clamp_min >= 0.f ? 1.0f / fmaxf(sqrtf(tot), clamp_min) : 1.0f / sqrtf(tot - clamp_min);
  for (int c = lane; c < D; c += 32) out[row * ldo + c] = xr[c] * inv;
}

__global__ void bias_rows_l2_kernel(float* x, long long ldx, int rows, int D, const float* __restrict__ bias,
                                    int normalize, float clamp_min) {
  const int warps = blockDim.x >> 5;
  const long long row = static_cast<long long>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float* xr = x + row * ldx;
  float ss = 0.f;
  for (int c = lane; c < D; c += 32) {
    const float v = bias ? xr[c] + bias[c] : xr[c];
    xr[c] = v;
    ss += v * v;
  }
  const float inv = normalize ? 1.0f / fmaxf(sqrtf(warp_sum(ss)), clamp_min) : 1.0f;
  if (normalize)
    for (int c = lane; c < D; c += 32) xr[c] *= inv;
}

// Mean pooling in two passes, deterministic. Pass 1: one CTA of 8 warps per
// (text, chunk of kSegChunk tokens, group of 256 columns); lane l of a warp
// holds columns 8l .. 8l+7 of the group (one 16-byte load per row for bf16),
// warp w sums the chunk's rows w, w + 8, ..., and the eight warp sums are
// added in warp order into partial[text][chunk][:]. Pass 2 adds a text's
// chunks in order and divides by its length. Long texts spread over
// ceil(L / kSegChunk) CTAs instead of one.
constexpr int kSegChunk = 256;

template <typename T>
__global__ void __launch_bounds__(256) segment_sum_chunks_kernel(const T* __restrict__ x, long long ldx,
                                                                 const int* __restrict__ cu, int H, int chunks,
                                                                 float* __restrict__ partial) {
  const int i = blockIdx.x, j = blockIdx.y;
  const int s = cu[i], e = cu[i + 1];
  const int t0 = s + j * kSegChunk;
  if (t0 >= e) return;
  const int t1 = min(e, t0 + kSegChunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c0 = blockIdx.z * 256 + lane * 8;
  const bool on = c0 < H;  // H is a multiple of 8
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (on) {
    for (int t = t0 + warp; t < t1; t += 8) {
      float v[8];
      ld8<T>(x + static_cast<long long>(t) * ldx + c0, v);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] += v[k];
    }
  }
  __shared__ float red[8][256];
#pragma unroll
  for (int k = 0; k < 8; ++k) red[warp][lane * 8 + k] = acc[k];
  __syncthreads();
  const int c = blockIdx.z * 256 + threadIdx.x;
  if (c < H) {
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) sum += red[w][threadIdx.x];
    partial[(static_cast<long long>(i) * chunks + j) * H + c] = sum;
  }
}

__global__ void segment_mean_finish_kernel(const float* __restrict__ partial, const int* __restrict__ cu, int n,
                                           int H, int chunks, float* __restrict__ out) {
  const long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (idx >= static_cast<long long>(n) * H) return;
  const int i = static_cast<int>(idx / H), c = static_cast<int>(idx - static_cast<long long>(i) * H);
  const int L = cu[i + 1] - cu[i];
  const int nch = (L + kSegChunk - 1) / kSegChunk;
  float sum = 0.f;
  for (int j = 0; j < nch; ++j) sum += partial[(static_cast<long long>(i) * chunks + j) * H + c];
  out[idx] = L > 0 ? sum / static_cast<float>(L) : 0.f;
}

__global__ void truncate_normalize_kernel(const float* __restrict__ x, int n, int D, int dim,
                                          float* __restrict__ out) {
  const int warps = blockDim.x >> 5;
  const long long row = static_cast<long long>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n) return;
  const float* xr = x + row * D;
  float ss = 0.f;
  for (int c = lane; c < dim; c += 32) ss += xr[c] * xr[c];
  const float nrm = sqrtf(warp_sum(ss));
  for (int c = lane; c < dim; c += 32) out[row * dim + c] = nrm > 0.f ? xr[c] / nrm : xr[c];
}

template <typename TS, typename TD>
__global__ void convert_rows_kernel(const TS* __restrict__ src, int rows, int cols, TD* __restrict__ dst,
                                    long long ld_dst, int blk, long long blk_stride, long long off,
                                    const float* __restrict__ col_scale) {
  const long long total = static_cast<long long>(rows) * cols;
  for (long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(idx / cols);
    const int c = static_cast<int>(idx - static_cast<long long>(r) * cols);
    const long long dr = static_cast<long long>(r / blk) * blk_stride + off + (r % blk);
    const float v = ld_f<TS>(src, idx);
    st_f<TD>(dst, dr * ld_dst + c, col_scale ? v * col_scale[c] : v);
  }
}

// h[r] = (h[r] + RMSNorm(a[r]) * w) * scale   (the Gemma post-attention / post-feedforward
// norms; with a scale, the PLE block's post norm and the layer scalar)
template <typename T>
__global__ void add_rms_norm_kernel(T* __restrict__ h, const T* __restrict__ a, const float* __restrict__ w,
                                    float eps, int rows, int H, const float* __restrict__ scale) {
  const int warps = blockDim.x >> 5;
  const long long row = static_cast<long long>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* ar = a + row * H;
  T* hr = h + row * H;
  float ss = 0.f;
  for (int c = lane; c < H; c += 32) {
    const float v = ld_f<T>(ar, c);
    ss += v * v;
  }
  const float inv = rsqrtf(warp_sum(ss) / static_cast<float>(H) + eps);
  const bool is_bf16 = sizeof(T) == 2;
  if (scale) {
    // the scalar in the model dtype; the sum rounded before the multiply
    const float sc = is_bf16 ? bf16_round(*scale) : *scale;
    for (int c = lane; c < H; c += 32) {
      float n = ld_f<T>(ar, c) * inv * w[c];
      if (is_bf16) n = bf16_round(n);
      float sum = ld_f<T>(hr, c) + n;
      if (is_bf16) sum = bf16_round(sum);
      st_f<T>(hr, c, sum * sc);
    }
    return;
  }
  for (int c = lane; c < H; c += 32) {
    float n = ld_f<T>(ar, c) * inv * w[c];
    if (is_bf16) n = bf16_round(n);  // the normed branch in the model dtype, then the add
    st_f<T>(hr, c, ld_f<T>(hr, c) + n);
  }
}

// In place, per row of `cols`: x = RMSNorm(x * scale) * w, the product rounded
// to the model dtype first (the per-layer embedding inputs of EmbeddingGemma 2).
template <typename T>
__global__ void scaled_rms_norm_kernel(T* __restrict__ x, long long rows, int cols, float scale,
                                       const float* __restrict__ w, float eps) {
  const int warps = blockDim.x >> 5;
  const long long row = static_cast<long long>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  T* xr = x + row * cols;
  const bool is_bf16 = sizeof(T) == 2;
  float ss = 0.f;
  for (int c = lane; c < cols; c += 32) {
    float v = ld_f<T>(xr, c) * scale;
    if (is_bf16) v = bf16_round(v);
    ss += v * v;
  }
  const float inv = rsqrtf(warp_sum(ss) / static_cast<float>(cols) + eps);
  for (int c = lane; c < cols; c += 32) {
    float v = ld_f<T>(xr, c) * scale;
    if (is_bf16) v = bf16_round(v);
    st_f<T>(xr, c, v * inv * w[c]);
  }
}

// out[r, j] = act(x[r, j]) * y[r, j] with row strides (the PLE gate: the
// activated bottleneck times this layer's slice of the per-layer inputs).
template <typename T, int ACT>
__global__ void act_mul_rows_kernel(const T* x, long long ldx, const T* __restrict__ y, long long ldy, int rows,
                                    int cols, T* out, long long ldo) {
  const long long total = static_cast<long long>(rows) * cols;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / cols;
    const int j = static_cast<int>(i - r * cols);
    const float g = ld_f<T>(x, r * ldx + j);
    float a;
    if constexpr (ACT == INL_ACT_SILU) a = silu_f(g);
    else if constexpr (ACT == INL_ACT_GELU_ERF) a = gelu_erf_f(g);
    else a = gelu_tanh_f(g);
    if (sizeof(T) == 2) a = bf16_round(a);
    st_f<T>(out, r * ldo + j, a * ld_f<T>(y, r * ldy + j));
  }
}

template <typename T>
__global__ void gather_rows_kernel(const T* __restrict__ src, long long lds, const int* __restrict__ idx, int n,
                                   int H, T* __restrict__ dst) {
  const int warps = blockDim.x >> 5;
  const long long r = static_cast<long long>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= n) return;
  const T* s = src + static_cast<long long>(idx[r]) * lds;
  T* d = dst + r * H;
  for (int c = lane; c < H; c += 32) d[c] = s[c];
}

__global__ void fill_i32_kernel(int* __restrict__ p, long long n, int value) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    p[i] = value;
}

// SPLADE finish + fold: w = ln(1 + relu(m + bias - shift) * open); with a canonical
// map, out[i][canon[v]] = max over v (w >= 0, so the int bits order as the floats).
__global__ void splade_finish_kernel(const int* __restrict__ pooled, int n, int V, const float* __restrict__ bias,
                                     float shift, const float* __restrict__ open, const int* __restrict__ canon,
                                     int dim, float* __restrict__ out) {
  const long long total = static_cast<long long>(n) * V;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(i / V);
    const int v = static_cast<int>(i - static_cast<long long>(row) * V);
    const float m = decode_ordered(pooled[i]);
    float x = m + (bias ? bias[v] : 0.f) - shift;
    x = fmaxf(x, 0.f);  // relu before the mask: -inf never meets a zero
    if (open) x *= open[v];
    const float w = logf(1.0f + x);
    if (canon) {
      atomicMax(reinterpret_cast<int*>(out) + static_cast<long long>(row) * dim + canon[v], __float_as_int(w));
    } else {
      out[i] = w;
    }
  }
}

// out[r, j] = act(x[r, j]) * x[r, I + j]: the gated MLP when gate / up are not interleaved.
template <typename T, int ACT>
__global__ void act_mul_kernel(const T* __restrict__ x, int rows, int I, T* __restrict__ out) {
  const long long total = static_cast<long long>(rows) * I;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / I;
    const int j = static_cast<int>(i - r * I);
    const float g = ld_f<T>(x, r * 2 * I + j), u = ld_f<T>(x, r * 2 * I + I + j);
    float a;
    if constexpr (ACT == INL_ACT_SILU) a = silu_f(g);
    else if constexpr (ACT == INL_ACT_GELU_ERF) a = gelu_erf_f(g);
    else a = gelu_tanh_f(g);
    st_f<T>(out, i, a * u);
  }
}

inline int rows_grid(long long rows, int warps_per_block) {
  return static_cast<int>((rows + warps_per_block - 1) / warps_per_block);
}

inline int ok(cudaError_t e) { return e == cudaSuccess ? 0 : -3; }

}  // namespace

int embed_gather(const uint32_t* ids, int T, const void* table, int table_bf16, int vocab, int H, float scale,
                 void* out, int out_bf16, int* status, cudaStream_t s, float* ss_out) {
  if (T <= 0) return 0;
  if (ss_out && (H % INL_SS_COLS) != 0) return -1;
  const int grid = rows_grid(T, 4);
  if (table_bf16 && out_bf16)
    embed_gather_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, 128, 0, s>>>(
        ids, T, static_cast<const __nv_bfloat16*>(table), vocab, H, scale, static_cast<__nv_bfloat16*>(out), ss_out, status);
  else if (table_bf16)
    embed_gather_kernel<__nv_bfloat16, float><<<grid, 128, 0, s>>>(
        ids, T, static_cast<const __nv_bfloat16*>(table), vocab, H, scale, static_cast<float*>(out), ss_out, status);
  else if (out_bf16)
    embed_gather_kernel<float, __nv_bfloat16><<<grid, 128, 0, s>>>(
        ids, T, static_cast<const float*>(table), vocab, H, scale, static_cast<__nv_bfloat16*>(out), ss_out, status);
  else
    embed_gather_kernel<float, float><<<grid, 128, 0, s>>>(ids, T, static_cast<const float*>(table), vocab, H,
                                                           scale, static_cast<float*>(out), ss_out, status);
  return ok(cudaGetLastError());
}

template <bool LN, bool ACT, int NC>
static void norm_reg_launch(const void* x, int x_bf16, long long ldx, const float* w, const float* b, float eps,
                            int rows, void* out, int out_bf16, long long ldo, int grid, cudaStream_t s) {
  if (x_bf16 && out_bf16)
    norm_rows_reg_kernel<__nv_bfloat16, __nv_bfloat16, LN, ACT, NC><<<grid, 128, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), ldx, w, b, eps, rows, static_cast<__nv_bfloat16*>(out), ldo);
  else if (x_bf16)
    norm_rows_reg_kernel<__nv_bfloat16, float, LN, ACT, NC><<<grid, 128, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), ldx, w, b, eps, rows, static_cast<float*>(out), ldo);
  else if (out_bf16)
    norm_rows_reg_kernel<float, __nv_bfloat16, LN, ACT, NC><<<grid, 128, 0, s>>>(
        static_cast<const float*>(x), ldx, w, b, eps, rows, static_cast<__nv_bfloat16*>(out), ldo);
  else
    norm_rows_reg_kernel<float, float, LN, ACT, NC><<<grid, 128, 0, s>>>(static_cast<const float*>(x), ldx, w, b,
                                                                        eps, rows, static_cast<float*>(out), ldo);
}

// Register-resident norm when the rows allow it (H = 256, 512, 768 or 1024;
// rows, strides and weights aligned for the vector accesses); false otherwise.
template <bool LN, bool ACT>
static bool norm_reg(const void* x, int x_bf16, long long ldx, const float* w, const float* b, float eps, int rows,
                     int H, void* out, int out_bf16, long long ldo, cudaStream_t s) {
  const int ei = x_bf16 ? 2 : 4, eo = out_bf16 ? 2 : 4;
  if ((H & 255) || H > 1024 || (ldx * ei) % (8 * ei) || (ldo * eo) % (8 * eo) ||
      (reinterpret_cast<uintptr_t>(x) % (8 * ei)) || (reinterpret_cast<uintptr_t>(out) % (8 * eo)) ||
      (reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(b) & 15))
    return false;
  const int grid = rows_grid(rows, 4);
  switch (H / 256) {
    case 1: norm_reg_launch<LN, ACT, 1>(x, x_bf16, ldx, w, b, eps, rows, out, out_bf16, ldo, grid, s); break;
    case 2: norm_reg_launch<LN, ACT, 2>(x, x_bf16, ldx, w, b, eps, rows, out, out_bf16, ldo, grid, s); break;
    case 3: norm_reg_launch<LN, ACT, 3>(x, x_bf16, ldx, w, b, eps, rows, out, out_bf16, ldo, grid, s); break;
    default: norm_reg_launch<LN, ACT, 4>(x, x_bf16, ldx, w, b, eps, rows, out, out_bf16, ldo, grid, s); break;
  }
  return true;
}

template <bool LN>
static int norm_dispatch(const void* x, int x_bf16, long long ldx, const float* w, const float* b, float eps,
                         int rows, int H, void* out, int out_bf16, long long ldo, cudaStream_t s) {
  if (rows <= 0) return 0;
  if (norm_reg<LN, false>(x, x_bf16, ldx, w, b, eps, rows, H, out, out_bf16, ldo, s)) return ok(cudaGetLastError());
  const int grid = rows_grid(rows, 4);
  if (x_bf16 && out_bf16)
    norm_rows_kernel<__nv_bfloat16, __nv_bfloat16, LN><<<grid, 128, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), ldx, w, b, eps, rows, H, static_cast<__nv_bfloat16*>(out), ldo);
  else if (x_bf16)
    norm_rows_kernel<__nv_bfloat16, float, LN><<<grid, 128, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), ldx, w, b, eps, rows, H, static_cast<float*>(out), ldo);
  else if (out_bf16)
    norm_rows_kernel<float, __nv_bfloat16, LN><<<grid, 128, 0, s>>>(
        static_cast<const float*>(x), ldx, w, b, eps, rows, H, static_cast<__nv_bfloat16*>(out), ldo);
  else
    norm_rows_kernel<float, float, LN><<<grid, 128, 0, s>>>(static_cast<const float*>(x), ldx, w, b, eps, rows, H,
                                                            static_cast<float*>(out), ldo);
  return ok(cudaGetLastError());
}

int rms_norm(const void* x, int x_bf16, long long ldx, const float* w, float eps, int rows, int H, void* out,
             int out_bf16, long long ldo, cudaStream_t s) {
  return norm_dispatch<false>(x, x_bf16, ldx, w, nullptr, eps, rows, H, out, out_bf16, ldo, s);
}

int layer_norm(const void* x, int x_bf16, long long ldx, const float* w, const float* b, float eps, int rows, int H,
               void* out, int out_bf16, long long ldo, cudaStream_t s) {
  return norm_dispatch<true>(x, x_bf16, ldx, w, b, eps, rows, H, out, out_bf16, ldo, s);
}

int qk_norm_rope(const QkRopeArgs& a, cudaStream_t s) {
  if (a.T <= 0) return 0;
  const int heads = a.hq + a.hkv + (a.v_norm ? a.hkv : 0);
  const long long items = static_cast<long long>(a.T) * heads;
  const int grid = rows_grid(items, 8);
  if (a.d == 8 || a.d == 16 || a.d == 32) {
    if (a.bf16) qk_norm_rope_narrow_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(a);
    else qk_norm_rope_narrow_kernel<float><<<grid, 256, 0, s>>>(a);
    return ok(cudaGetLastError());
  }
  const int E = a.d / 32;
  if (a.d % 32 != 0) return -1;
  // One vector access per lane when the rows, the weights and the tables are
  // aligned to it; element by element otherwise.
  const size_t es = a.bf16 ? 2 : 4, vb = es * E;
  const bool vec = (a.ld * es) % vb == 0 && (reinterpret_cast<uintptr_t>(a.qkv) % vb) == 0 &&
                   (reinterpret_cast<uintptr_t>(a.cos) % (4 * E)) == 0 &&
                   (reinterpret_cast<uintptr_t>(a.sin) % (4 * E)) == 0 &&
                   (reinterpret_cast<uintptr_t>(a.qw) % (4 * E)) == 0 && (reinterpret_cast<uintptr_t>(a.kw) % (4 * E)) == 0;
  // Aligned rows: one warp per token for head_dim 64 / 128 (19.1 -> 9.0 us on
  // config 2's bf16 layers), one warp per (token, head) for 256 (0.124
  // against 0.138 ms on config 4's).
  const int tok_grid = rows_grid(a.T, 8);
#define INL_QKR(EE)                                                                               \
  if (vec && EE < 8 && a.bf16) qk_norm_rope_tok_kernel<__nv_bfloat16, EE><<<tok_grid, 256, 0, s>>>(a); \
  else if (vec && EE < 8) qk_norm_rope_tok_kernel<float, EE><<<tok_grid, 256, 0, s>>>(a);         \
  else if (vec && a.bf16) qk_norm_rope_vec_kernel<__nv_bfloat16, EE><<<grid, 256, 0, s>>>(a);     \
  else if (vec) qk_norm_rope_vec_kernel<float, EE><<<grid, 256, 0, s>>>(a);                       \
  else if (a.bf16) qk_norm_rope_kernel<__nv_bfloat16, EE><<<grid, 256, 0, s>>>(a);                \
  else qk_norm_rope_kernel<float, EE><<<grid, 256, 0, s>>>(a);
  switch (E) {
    case 2: INL_QKR(2) break;
    case 4: INL_QKR(4) break;
    case 8: INL_QKR(8) break;
    default: return -1;
  }
#undef INL_QKR
  return ok(cudaGetLastError());
}

int token_positions(const int* cu, int n, int T, int* pos, cudaStream_t s) {
  if (T <= 0) return 0;
  token_positions_kernel<<<(T + 255) / 256, 256, 0, s>>>(cu, n, T, pos);
  return ok(cudaGetLastError());
}

int last_token_norm_l2(const void* h, int h_bf16, long long ldh, const int* cu, int n, const float* w, float eps,
                       int H, float* out, cudaStream_t s) {
  if (n <= 0) return 0;
  if (h_bf16)
    last_token_norm_l2_kernel<__nv_bfloat16><<<n, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(h), ldh, cu, n, w,
                                                                eps, H, out);
  else
    last_token_norm_l2_kernel<float><<<n, 256, 0, s>>>(static_cast<const float*>(h), ldh, cu, n, w, eps, H, out);
  return ok(cudaGetLastError());
}

// f32 rows split into three bf16 K-segments for the 3xBF16 tensor-core
// product: x = hi + lo + O(2^-17 |x|) with hi = bf16(x), lo = bf16(x - hi).
// Activation side (mode 0) [hi | hi | lo], weight side (mode 1) [hi | lo | hi]:
// one bf16 GEMM over K' = 3K then sums hi.hi + hi.lo + lo.hi in f32.
// Mode 2 writes the hi segment alone: the bf16-rounded operand of a plain
// bf16 product over K.
__global__ void split3_kernel(const float* __restrict__ x, long long ldx, int rows, int K, int mode,
                              __nv_bfloat16* __restrict__ out, long long ldo) {
  const int pairs = K / 2;
  const long long total = static_cast<long long>(rows) * pairs;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / pairs);
    const int k = 2 * static_cast<int>(i - static_cast<long long>(r) * pairs);
    const float2 v = *reinterpret_cast<const float2*>(x + static_cast<long long>(r) * ldx + k);
    const __nv_bfloat162 hi = __floats2bfloat162_rn(v.x, v.y);
    const float2 h = __bfloat1622float2(hi);
    const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x - h.x, v.y - h.y);
    __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(out + static_cast<long long>(r) * ldo + k);
    o[0] = hi;
    if (mode == 2) continue;
    o[K / 2] = mode ? lo : hi;
    o[K] = mode ? hi : lo;
  }
}

// The same split four columns at a time (one 16-byte load, 8-byte stores)
// with 32-bit indexing, for rows aligned to it; identical results.
__global__ void split3_vec4_kernel(const float* __restrict__ x, long long ldx, int rows, int K, int mode,
                                   __nv_bfloat16* __restrict__ out, long long ldo) {
  const int q4 = K >> 2;
  const int total = rows * q4;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int r = i / q4;
    const int k = (i - r * q4) << 2;
    const float4 v = *reinterpret_cast<const float4*>(x + static_cast<long long>(r) * ldx + k);
    const __nv_bfloat162 h0 = __floats2bfloat162_rn(v.x, v.y), h1 = __floats2bfloat162_rn(v.z, v.w);
    const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
    const __nv_bfloat162 l0 = __floats2bfloat162_rn(v.x - f0.x, v.y - f0.y);
    const __nv_bfloat162 l1 = __floats2bfloat162_rn(v.z - f1.x, v.w - f1.y);
    uint2 hi, lo;
    hi.x = *reinterpret_cast<const uint32_t*>(&h0);
    hi.y = *reinterpret_cast<const uint32_t*>(&h1);
    lo.x = *reinterpret_cast<const uint32_t*>(&l0);
    lo.y = *reinterpret_cast<const uint32_t*>(&l1);
    __nv_bfloat16* o = out + static_cast<long long>(r) * ldo + k;
    *reinterpret_cast<uint2*>(o) = hi;
    if (mode == 2) continue;
    *reinterpret_cast<uint2*>(o + K) = mode ? lo : hi;
    *reinterpret_cast<uint2*>(o + 2 * K) = mode ? hi : lo;
  }
}

int split3_bf16(const float* x, long long ldx, int rows, int K, int mode, void* out, long long ldo, cudaStream_t s) {
  if (rows <= 0) return 0;
  if ((K & 1) || (ldx & 1) || (ldo & 1) || (reinterpret_cast<uintptr_t>(x) & 7) ||
      (reinterpret_cast<uintptr_t>(out) & 3))
    return -1;
  if ((K & 3) == 0 && (ldx & 3) == 0 && (ldo & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(out) & 7) == 0 && static_cast<long long>(rows) * (K / 4) < (1LL << 31)) {
    const long long total4 = static_cast<long long>(rows) * (K / 4);
    const int blocks = static_cast<int>(std::min<long long>((total4 + 255) / 256, 148LL * 16));
    split3_vec4_kernel<<<blocks, 256, 0, s>>>(x, ldx, rows, K, mode, static_cast<__nv_bfloat16*>(out), ldo);
    return ok(cudaGetLastError());
  }
  const long long total = static_cast<long long>(rows) * (K / 2);
  const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
  split3_kernel<<<blocks, 256, 0, s>>>(x, ldx, rows, K, mode, static_cast<__nv_bfloat16*>(out), ldo);
  return ok(cudaGetLastError());
}

// Split-K partial planes summed in slice order (+ the residual), four
// columns per thread when rows and pointers allow, else one.
template <int V>
__global__ void splits_reduce_kernel(const float* __restrict__ ws, long long plane, long long ldw, int splits, int rows,
                                     int cols, const float* resid, long long ldr, float* out, long long ldo) {
  const int cv = cols / V;
  const long long total = static_cast<long long>(rows) * cv;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / cv);
    const int c = static_cast<int>(i - static_cast<long long>(r) * cv) * V;
    auto ld = [](const float* p, float (&v)[V]) {
      if constexpr (V == 4) {
        const float4 a = *reinterpret_cast<const float4*>(p);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      } else {
        v[0] = *p;
      }
    };
    float acc[V];
    ld(ws + static_cast<long long>(r) * ldw + c, acc);
    for (int sl = 1; sl < splits; ++sl) {
      float p[V];
      ld(ws + sl * plane + static_cast<long long>(r) * ldw + c, p);
#pragma unroll
      for (int j = 0; j < V; ++j) acc[j] += p[j];
    }
    if (resid) {
      float q[V];
      ld(resid + static_cast<long long>(r) * ldr + c, q);
#pragma unroll
      for (int j = 0; j < V; ++j) acc[j] = q[j] + acc[j];
    }
    float* o = out + static_cast<long long>(r) * ldo + c;
    if constexpr (V == 4) *reinterpret_cast<float4*>(o) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    else *o = acc[0];
  }
}

int splits_reduce_f32(const float* ws, long long plane, long long ldw, int splits, int rows, int cols,
                      const float* resid, long long ldr, float* out, long long ldo, cudaStream_t s) {
  if (rows <= 0 || cols <= 0) return 0;
  if (splits < 1) return -1;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool v4 = (cols % 4) == 0 && (ldw % 4) == 0 && (plane % 4) == 0 && (ldo % 4) == 0 && al(ws) && al(out) &&
                  (!resid || (al(resid) && (ldr % 4) == 0));
  const long long total = static_cast<long long>(rows) * (v4 ? cols / 4 : cols);
  const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
  if (v4) splits_reduce_kernel<4><<<blocks, 256, 0, s>>>(ws, plane, ldw, splits, rows, cols, resid, ldr, out, ldo);
  else splits_reduce_kernel<1><<<blocks, 256, 0, s>>>(ws, plane, ldw, splits, rows, cols, resid, ldr, out, ldo);
  return ok(cudaGetLastError());
}

// out = a + b over rows x cols (f32; out may alias a or b).
__global__ void add_rows_f32_kernel(float* out, long long ldo, const float* a, long long lda, const float* b,
                                    long long ldb, int rows, int cols) {
  const long long total = static_cast<long long>(rows) * cols;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / cols), c = static_cast<int>(i - static_cast<long long>(r) * cols);
    out[static_cast<long long>(r) * ldo + c] = a[static_cast<long long>(r) * lda + c] + b[static_cast<long long>(r) * ldb + c];
  }
}

int add_rows_f32(float* out, long long ldo, const float* a, long long lda, const float* b, long long ldb, int rows,
                 int cols, cudaStream_t s) {
  if (rows <= 0 || cols <= 0) return 0;
  const long long total = static_cast<long long>(rows) * cols;
  const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
  add_rows_f32_kernel<<<blocks, 256, 0, s>>>(out, ldo, a, lda, b, ldb, rows, cols);
  return ok(cudaGetLastError());
}

// Gated MLP from the full gate/up product x [rows, 2I] (f32) whose columns come in
// blocks of `blk`: gate block j, then up block j. out[r, c] = act(gate) * up.
template <int ACT>
__global__ void act_mul_blocks_kernel(const float* __restrict__ x, long long ldx, int rows, int I, int blk,
                                      float* __restrict__ out, long long ldo) {
  const long long total = static_cast<long long>(rows) * I;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / I), c = static_cast<int>(i - static_cast<long long>(r) * I);
    const int b = c / blk, o = c - b * blk;
    const float* row = x + static_cast<long long>(r) * ldx + 2LL * b * blk + o;
    float g = row[0];
    if constexpr (ACT == INL_ACT_SILU) g = silu_f(g);
    else if constexpr (ACT == INL_ACT_GELU_ERF) g = gelu_erf_f(g);
    else g = gelu_tanh_f(g);
    out[static_cast<long long>(r) * ldo + c] = g * row[blk];
  }
}

int act_mul_blocks_f32(const float* x, long long ldx, int rows, int I, int blk, int act, float* out, long long ldo,
                       cudaStream_t s) {
  if (rows <= 0 || I <= 0) return 0;
  if (blk <= 0) return -1;
  const long long total = static_cast<long long>(rows) * I;
  const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
  switch (act) {
    case INL_ACT_SILU: act_mul_blocks_kernel<INL_ACT_SILU><<<blocks, 256, 0, s>>>(x, ldx, rows, I, blk, out, ldo); break;
    case INL_ACT_GELU_ERF:
      act_mul_blocks_kernel<INL_ACT_GELU_ERF><<<blocks, 256, 0, s>>>(x, ldx, rows, I, blk, out, ldo);
      break;
    default: act_mul_blocks_kernel<INL_ACT_GELU_TANH><<<blocks, 256, 0, s>>>(x, ldx, rows, I, blk, out, ldo); break;
  }
  return ok(cudaGetLastError());
}

// One CTA per row. Counting: a block sum of the active entries.
__global__ void sparse_count_kernel(const float* __restrict__ rows, int D, int* __restrict__ counts,
                                    int* __restrict__ bad) {
  const float* row = rows + static_cast<long long>(blockIdx.x) * D;
  int c = 0;
  bool finite = true;
  for (int v = threadIdx.x; v < D; v += blockDim.x) {
    const float w = row[v];
    c += w > 0.f;
    finite &= isfinite(w);
  }
  __shared__ int red[32];
  c = __reduce_add_sync(0xffffffffu, c);
  if (!__all_sync(0xffffffffu, finite) && (threadIdx.x & 31) == 0) atomicOr(bad, 1);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
    counts[blockIdx.x] = t;
  }
}

// Order-preserving compaction of one row per CTA: each pass takes blockDim.x
// consecutive columns; a warp's active lanes find their slot from the ballot,
// the warps' totals are scanned in shared memory, and the pass's total moves
// the row's write position.
__global__ void sparse_compact_kernel(const float* __restrict__ rows, int D, const long long* __restrict__ offsets,
                                      int32_t* __restrict__ idx, float* __restrict__ val) {
  const float* row = rows + static_cast<long long>(blockIdx.x) * D;
  long long base = offsets[blockIdx.x];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __shared__ int wsum[32];
  for (int v0 = 0; v0 < D; v0 += blockDim.x) {
    const int v = v0 + threadIdx.x;
    const float w = v < D ? row[v] : 0.f;
    const bool on = w > 0.f;
    const unsigned bal = __ballot_sync(0xffffffffu, on);
    if (lane == 0) wsum[warp] = __popc(bal);
    __syncthreads();
    int before = 0, total = 0;
    for (int k = 0; k < nw; ++k) {
      const int c = wsum[k];
      before += k < warp ? c : 0;
      total += c;
    }
    if (on) {
      const long long at = base + before + __popc(bal & ((1u << lane) - 1u));
      idx[at] = v;
      val[at] = w;
    }
    base += total;
    __syncthreads();  // wsum is rewritten by the next pass
  }
}

int sparse_count(const float* rows, int n, int D, int* counts, int* bad, cudaStream_t s) {
  if (n <= 0) return 0;
  sparse_count_kernel<<<n, 256, 0, s>>>(rows, D, counts, bad);
  return ok(cudaGetLastError());
}

int sparse_compact(const float* rows, int n, int D, const long long* offsets, int32_t* idx, float* val,
                   cudaStream_t s) {
  if (n <= 0) return 0;
  sparse_compact_kernel<<<n, 256, 0, s>>>(rows, D, offsets, idx, val);
  return ok(cudaGetLastError());
}

__global__ void gather_last_rows_kernel(const uint4* __restrict__ in, long long ld_in, const int* __restrict__ cu,
                                        int n, int chunks, uint4* __restrict__ out, long long ld_out) {
  const int i = blockIdx.x;
  if (i >= n) return;
  const uint4* src = in + static_cast<long long>(cu[i + 1] - 1) * ld_in;
  uint4* dst = out + static_cast<long long>(i) * ld_out;
  for (int c = threadIdx.x; c < chunks; c += blockDim.x) dst[c] = src[c];
}

int gather_last_rows_bf16(const void* in, long long ld_in, const int* cu, int n, int cols, void* out,
                          long long ld_out, cudaStream_t s) {
  if (n <= 0) return 0;
  if ((cols % 8) || (ld_in % 8) || (ld_out % 8) || (reinterpret_cast<uintptr_t>(in) & 15) ||
      (reinterpret_cast<uintptr_t>(out) & 15))
    return -1;
  gather_last_rows_kernel<<<n, 128, 0, s>>>(static_cast<const uint4*>(in), ld_in / 8, cu, n, cols / 8,
                                             static_cast<uint4*>(out), ld_out / 8);
  return ok(cudaGetLastError());
}

int rows_l2_f32(const float* x, long long ldx, int rows, int D, float clamp_min, float* out, long long ldo,
                cudaStream_t s) {
  if (rows <= 0) return 0;
  rows_l2_kernel<<<rows_grid(rows, 8), 256, 0, s>>>(x, ldx, rows, D, clamp_min, out, ldo);
  return ok(cudaGetLastError());
}

size_t segment_mean_scratch_bytes(int n, int H, int max_len) {
  const size_t chunks = static_cast<size_t>(std::max(1, (max_len + kSegChunk - 1) / kSegChunk));
  return static_cast<size_t>(std::max(n, 1)) * chunks * H * 4;
}

int segment_mean(const void* x, int x_bf16, long long ldx, const int* cu, int n, int H, int max_len, float* scratch,
                 float* out, cudaStream_t s) {
  if (n <= 0) return 0;
  if ((H % 8) || (ldx % 8) || (reinterpret_cast<uintptr_t>(x) & 15)) return -1;
  const int chunks = std::max(1, (max_len + kSegChunk - 1) / kSegChunk);
  dim3 grid(n, chunks, (H + 255) / 256);
  if (x_bf16)
    segment_sum_chunks_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), ldx, cu, H,
                                                                    chunks, scratch);
  else
    segment_sum_chunks_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(x), ldx, cu, H, chunks, scratch);
  const long long total = static_cast<long long>(n) * H;
  segment_mean_finish_kernel<<<static_cast<int>((total + 255) / 256), 256, 0, s>>>(scratch, cu, n, H, chunks, out);
  return ok(cudaGetLastError());
}

int bias_rows_l2_f32(float* x, long long ldx, int rows, int D, const float* bias, int normalize, float clamp_min,
                     cudaStream_t s) {
  if (rows <= 0) return 0;
  bias_rows_l2_kernel<<<rows_grid(rows, 8), 256, 0, s>>>(x, ldx, rows, D, bias, normalize, clamp_min);
  return ok(cudaGetLastError());
}

int truncate_normalize(const float* x, int n, int D, int dim, float* out, cudaStream_t s) {
  if (n <= 0) return 0;
  truncate_normalize_kernel<<<rows_grid(n, 8), 256, 0, s>>>(x, n, D, dim, out);
  return ok(cudaGetLastError());
}

int convert_rows(const float* src, int rows, int cols, void* dst, int dst_bf16, long long ld_dst, int blk,
                 long long blk_stride, long long off, cudaStream_t s, const float* col_scale) {
  if (rows <= 0 || cols <= 0) return 0;
  const long long total = static_cast<long long>(rows) * cols;
  const int grid = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
  if (dst_bf16)
    convert_rows_kernel<float, __nv_bfloat16><<<grid, 256, 0, s>>>(src, rows, cols, static_cast<__nv_bfloat16*>(dst),
                                                                    ld_dst, blk, blk_stride, off, col_scale);
  else
    convert_rows_kernel<float, float><<<grid, 256, 0, s>>>(src, rows, cols, static_cast<float*>(dst), ld_dst, blk,
                                                           blk_stride, off, col_scale);
  return ok(cudaGetLastError());
}

int convert_bf16_rows(const __nv_bfloat16* src, int rows, int cols, void* dst, int dst_bf16, long long ld_dst,
                      int blk, long long blk_stride, long long off, cudaStream_t s, const float* col_scale) {
  if (rows <= 0 || cols <= 0) return 0;
  const long long total = static_cast<long long>(rows) * cols;
  const int grid = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
  if (dst_bf16)
    convert_rows_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, 256, 0, s>>>(
        src, rows, cols, static_cast<__nv_bfloat16*>(dst), ld_dst, blk, blk_stride, off, col_scale);
  else
    convert_rows_kernel<__nv_bfloat16, float><<<grid, 256, 0, s>>>(src, rows, cols, static_cast<float*>(dst), ld_dst,
                                                                   blk, blk_stride, off, col_scale);
  return ok(cudaGetLastError());
}

int norm_act(const void* x, int x_bf16, long long ldx, const float* w, const float* b, float eps, int rows, int H,
             void* out, int out_bf16, long long ldo, cudaStream_t s) {
  if (rows <= 0) return 0;
  if (x_bf16 == out_bf16 && norm_reg<true, true>(x, x_bf16, ldx, w, b, eps, rows, H, out, out_bf16, ldo, s))
    return ok(cudaGetLastError());
  const int grid = rows_grid(rows, 4);
  if (x_bf16 && out_bf16)
    norm_rows_kernel<__nv_bfloat16, __nv_bfloat16, true, true><<<grid, 128, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), ldx, w, b, eps, rows, H, static_cast<__nv_bfloat16*>(out), ldo);
  else if (!x_bf16 && !out_bf16)
    norm_rows_kernel<float, float, true, true><<<grid, 128, 0, s>>>(static_cast<const float*>(x), ldx, w, b, eps,
                                                                     rows, H, static_cast<float*>(out), ldo);
  else
    return -1;
  return ok(cudaGetLastError());
}

int add_rms_norm(void* h, const void* a, int bf16, const float* w, float eps, int rows, int H, cudaStream_t s,
                 const float* scale) {
  if (rows <= 0) return 0;
  const int grid = rows_grid(rows, 4);
  if (bf16)
    add_rms_norm_kernel<__nv_bfloat16><<<grid, 128, 0, s>>>(
        static_cast<__nv_bfloat16*>(h), static_cast<const __nv_bfloat16*>(a), w, eps, rows, H, scale);
  else
    add_rms_norm_kernel<float><<<grid, 128, 0, s>>>(static_cast<float*>(h), static_cast<const float*>(a), w, eps,
                                                     rows, H, scale);
  return ok(cudaGetLastError());
}

int scaled_rms_norm(void* x, int bf16, long long rows, int cols, float scale, const float* w, float eps,
                    cudaStream_t s) {
  if (rows <= 0 || cols <= 0) return 0;
  const int grid = rows_grid(rows, 4);
  if (bf16)
    scaled_rms_norm_kernel<__nv_bfloat16><<<grid, 128, 0, s>>>(static_cast<__nv_bfloat16*>(x), rows, cols, scale, w,
                                                                eps);
  else
    scaled_rms_norm_kernel<float><<<grid, 128, 0, s>>>(static_cast<float*>(x), rows, cols, scale, w, eps);
  return ok(cudaGetLastError());
}

int act_mul_rows(const void* x, long long ldx, const void* y, long long ldy, int bf16, int rows, int cols, int act,
                 void* out, long long ldo, cudaStream_t s) {
  if (rows <= 0 || cols <= 0) return 0;
  const long long total = static_cast<long long>(rows) * cols;
  const int grid = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
#define INL_AMR(T, A)                                                                                           \
  act_mul_rows_kernel<T, A><<<grid, 256, 0, s>>>(static_cast<const T*>(x), ldx, static_cast<const T*>(y), ldy, \
                                                 rows, cols, static_cast<T*>(out), ldo)
  if (bf16) {
    if (act == INL_ACT_SILU) INL_AMR(__nv_bfloat16, INL_ACT_SILU);
    else if (act == INL_ACT_GELU_ERF) INL_AMR(__nv_bfloat16, INL_ACT_GELU_ERF);
    else INL_AMR(__nv_bfloat16, INL_ACT_GELU_TANH);
  } else {
    if (act == INL_ACT_SILU) INL_AMR(float, INL_ACT_SILU);
    else if (act == INL_ACT_GELU_ERF) INL_AMR(float, INL_ACT_GELU_ERF);
    else INL_AMR(float, INL_ACT_GELU_TANH);
  }
#undef INL_AMR
  return ok(cudaGetLastError());
}

int gather_rows(const void* src, int bf16, long long lds, const int* idx, int n, int H, void* dst, cudaStream_t s) {
  if (n <= 0) return 0;
  const int grid = rows_grid(n, 4);
  if (bf16)
    gather_rows_kernel<__nv_bfloat16><<<grid, 128, 0, s>>>(static_cast<const __nv_bfloat16*>(src), lds, idx, n, H,
                                                            static_cast<__nv_bfloat16*>(dst));
  else
    gather_rows_kernel<float><<<grid, 128, 0, s>>>(static_cast<const float*>(src), lds, idx, n, H,
                                                   static_cast<float*>(dst));
  return ok(cudaGetLastError());
}

int fill_i32(int* p, long long n, int value, cudaStream_t s) {
  if (n <= 0) return 0;
  const int grid = static_cast<int>(std::min<long long>((n + 255) / 256, 148LL * 16));
  fill_i32_kernel<<<grid, 256, 0, s>>>(p, n, value);
  return ok(cudaGetLastError());
}

int splade_finish(const int* pooled, int n, int V, const float* bias, float shift, const float* open,
                  const int* canon, int dim, float* out, cudaStream_t s) {
  if (n <= 0) return 0;
  if (canon) {
    if (cudaMemsetAsync(out, 0, static_cast<size_t>(n) * dim * 4, s) != cudaSuccess) return -3;
  }
  const long long total = static_cast<long long>(n) * V;
  const int grid = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
  splade_finish_kernel<<<grid, 256, 0, s>>>(pooled, n, V, bias, shift, open, canon, dim, out);
  return ok(cudaGetLastError());
}

int act_mul(const void* x, int bf16, int rows, int I, int act, void* out, cudaStream_t s) {
  if (rows <= 0) return 0;
  const long long total = static_cast<long long>(rows) * I;
  const int grid = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
#define INL_AM(T, A) act_mul_kernel<T, A><<<grid, 256, 0, s>>>(static_cast<const T*>(x), rows, I, static_cast<T*>(out))
  if (bf16) {
    if (act == INL_ACT_SILU) INL_AM(__nv_bfloat16, INL_ACT_SILU);
    else if (act == INL_ACT_GELU_ERF) INL_AM(__nv_bfloat16, INL_ACT_GELU_ERF);
    else INL_AM(__nv_bfloat16, INL_ACT_GELU_TANH);
  } else {
    if (act == INL_ACT_SILU) INL_AM(float, INL_ACT_SILU);
    else if (act == INL_ACT_GELU_ERF) INL_AM(float, INL_ACT_GELU_ERF);
    else INL_AM(float, INL_ACT_GELU_TANH);
  }
#undef INL_AM
  return ok(cudaGetLastError());
}

}  // namespace inl
