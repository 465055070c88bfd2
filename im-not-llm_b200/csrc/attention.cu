// Variable-length attention over packed texts: causal, bidirectional and
// sliding-window (|q - k| <= window), grouped-query (query head h reads KV head
// h / (hq / hkv)), masks computed from positions instead of materialised.
//
// bf16 runs on the tcgen05 kernel of attention_sm100.cu (head_dim 64, 128,
// 256). f32 (the f32-accurate configurations): head_dim 64 / 128 on a
// register-tiled SIMT kernel (64 queries per CTA, 8 x 8 output tiles per
// thread); other head dims, and rows not 16-byte aligned, on a plain SIMT
// kernel (32 queries per CTA, 32-key tiles in shared memory, one lane per key
// for the scores and one lane per head dimension slice for the output).
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
  const int q0 = qb * a.q_block + blockIdx.z * kFQ;  // a work item of q_block rows is gridDim.z CTAs
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
  dim3 grid(a.n_work, a.hq, a.q_block / kFQ);
  kern<<<grid, 128, bytes, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// f32 attention for head_dim 64 / 128, register-tiled: a CTA of 64 R threads
// (R = D / 64) takes 64 queries of one head and walks 32-key tiles. Thread t
// owns the QPT = 8 queries of group qg = t / (8 R) and, within the group's
// 8 R threads, slot g = t % (8 R): the scores of keys [g * 4 / R, +4 / R) of
// each tile and the output columns [8 g, 8 g + 8). The 8 R threads of a group sit
// in one warp, so a query row's max and sum combine with shuffles, and every
// thread holds its rows' running max and sum for the output rescale. Q, K, V
// and P live in shared memory row-major with rows padded by 4 floats: the
// 16-byte loads of a warp touch distinct banks, and the lanes of one group
// read the same Q / P addresses (broadcast). Per 4 columns of the scores a
// thread issues QPT + 4 / R loads for 16 QPT / R FMAs, per 4 keys of the
// output 8 + QPT loads for 32 QPT FMAs. For head_dim 128 the K / V tiles
// are double-buffered and copied with cp.async, so the next tile's rows
// arrive while this one is computed. expf and the masks as in
// attn_f32_kernel.
constexpr int kTQ = 64;  // queries per CTA
constexpr int kTK = 32;  // keys per tile

// 16-byte global -> shared copies that bypass registers (cp.async): the
// bytes past src_bytes (0 or 16) are zero-filled.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc, int src_bytes) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(gsrc), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

template <int D>
struct F32Tiled {
  static constexpr int R = D / 64;
  static constexpr int QPT = 8;                     // queries per thread
  static constexpr int G = 8 * R;                   // threads per query group
  static constexpr int THREADS = (kTQ / QPT) * G;   // 64 R
  static constexpr int KPT = 4 / R;     // keys per thread per tile
  static constexpr int LD = D + 4;      // padded row of Q, K, V
  static constexpr int LDP = kTK + 4;   // padded row of P
  // Head_dim 128: tiles copied with cp.async into two K / V buffers, the next
  // tile streaming in during this one (2 CTAs per SM either way; 1.56 -> 1.44
  // ms of config 1's attention). Head_dim 64: one buffer filled by plain
  // loads, which keeps 5 CTAs per SM; the asynchronous forms measured 4-9%
  // slower there (fewer resident CTAs, or 128-thread CTAs at 4 queries per
  // thread).
  static constexpr bool ASYNC = D == 128;
  static constexpr int NBUF = ASYNC ? 2 : 1;
  static constexpr int SMEM = (kTQ * LD + 2 * NBUF * kTK * LD + kTQ * LDP) * 4;  // Q, K / V buffers, P
};

// HX: the head is blockIdx.x and the work item blockIdx.y, so the blocks are
// dispatched item by item (the list is heaviest first) with every head of an
// item together; otherwise (more work items than a grid's y extent) the
// reverse.
template <int D, bool HX>
__global__ void __launch_bounds__(F32Tiled<D>::THREADS) attn_f32_tiled_kernel(AttnArgs a) {
  using C = F32Tiled<D>;
  constexpr int KPT = C::KPT, LD = C::LD, LDP = C::LDP, QPT = C::QPT;
  extern __shared__ __align__(16) float fsm[];
  float* sQ = fsm;                  // [kTQ][LD]
  constexpr int NB = C::NBUF;
  float* sK0 = sQ + kTQ * LD;        // [NB][kTK][LD]
  float* sV0 = sK0 + NB * kTK * LD;  // [NB][kTK][LD]
  float* sP = sV0 + NB * kTK * LD;   // [kTQ][LDP]

  const int tid = threadIdx.x, lane = tid & 31;
  const int qg = tid / C::G, g = tid % C::G;
  const int2 wk = a.work[HX ? blockIdx.y : blockIdx.x];
  const int head = HX ? blockIdx.x : blockIdx.y;
  const int kvh = head / (a.hq / a.hkv);
  const int s0 = a.cu[wk.x];
  const int L = a.cu[wk.x + 1] - s0;
  const int q0 = wk.y * kTQ;
  if (q0 >= L) return;
  int k_lo = 0, k_hi = L;
  if (a.causal) k_hi = min(L, q0 + kTQ);
  if (a.window >= 0) {
    k_lo = max(0, q0 - a.window);
    k_hi = min(k_hi, q0 + kTQ + a.window);
  }
  const float* qbase = static_cast<const float*>(a.q) + static_cast<long long>(s0) * a.ldq + head * D;
  const float* kbase = static_cast<const float*>(a.k) + static_cast<long long>(s0) * a.ldk + kvh * D;
  const float* vbase = static_cast<const float*>(a.v) + static_cast<long long>(s0) * a.ldv + kvh * D;

  // ASYNC: every copy in flight at once (cp.async), K / V tiles double
  // buffered, tile t + 1 streaming in while tile t is computed; otherwise
  // plain 16-byte loads into one buffer. Rows past the text are zero-filled.
  constexpr int C4 = D / 4;  // float4 per row
  if constexpr (C::ASYNC) {
#pragma unroll 4
    for (int i = tid; i < kTQ * C4; i += C::THREADS) {
      const int r = i / C4, c = (i - r * C4) * 4;
      const bool ok = q0 + r < L;
      cp_async16(sQ + r * LD + c, ok ? qbase + static_cast<long long>(q0 + r) * a.ldq + c : qbase, ok ? 16 : 0);
    }
  } else {
    for (int i = tid; i < kTQ * C4; i += C::THREADS) {
      const int r = i / C4, c = (i - r * C4) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (q0 + r < L) v = *reinterpret_cast<const float4*>(qbase + static_cast<long long>(q0 + r) * a.ldq + c);
      *reinterpret_cast<float4*>(sQ + r * LD + c) = v;
    }
  }
  auto load_kv_sync = [&](int kt) {
    for (int i = tid; i < kTK * C4; i += C::THREADS) {
      const int r = i / C4, c = (i - r * C4) * 4;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (kt + r < L) {
        kv = *reinterpret_cast<const float4*>(kbase + static_cast<long long>(kt + r) * a.ldk + c);
        vv = *reinterpret_cast<const float4*>(vbase + static_cast<long long>(kt + r) * a.ldv + c);
      }
      *reinterpret_cast<float4*>(sK0 + r * LD + c) = kv;
      *reinterpret_cast<float4*>(sV0 + r * LD + c) = vv;
    }
  };
  auto load_kv = [&](int kt, int buf) {
    float* dk = sK0 + buf * kTK * LD;
    float* dv = sV0 + buf * kTK * LD;
#pragma unroll 4
    for (int i = tid; i < kTK * C4; i += C::THREADS) {
      const int r = i / C4, c = (i - r * C4) * 4;
      const bool ok = kt + r < L;
      cp_async16(dk + r * LD + c, ok ? kbase + static_cast<long long>(kt + r) * a.ldk + c : kbase, ok ? 16 : 0);
      cp_async16(dv + r * LD + c, ok ? vbase + static_cast<long long>(kt + r) * a.ldv + c : vbase, ok ? 16 : 0);
    }
    cp_async_commit();
  };
  const int kt0 = (k_lo / kTK) * kTK;
  if constexpr (C::ASYNC) load_kv(kt0, 0);  // committed with the Q copies
  float o[QPT][8];
  float m_r[QPT], l_r[QPT];
#pragma unroll
  for (int i = 0; i < QPT; ++i) {
    m_r[i] = -INFINITY;
    l_r[i] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) o[i][j] = 0.f;
  }
  const int qrow0 = qg * QPT;     // first of this thread's query rows in the tile
  const int kc0 = g * KPT;        // first of this thread's keys in a key tile
  const int dc0 = g * 8;          // first of this thread's output columns

  int buf = 0;
  for (int kt = kt0; kt < k_hi; kt += kTK, buf = NB == 2 ? buf ^ 1 : 0) {
    if constexpr (C::ASYNC) {
      // The other buffer was released by the barrier that ended the last tile.
      if (kt + kTK < k_hi) {
        load_kv(kt + kTK, buf ^ 1);
        cp_async_wait<1>();  // this tile's copies (and Q) have landed
      } else {
        cp_async_wait<0>();
      }
    } else {
      load_kv_sync(kt);  // the buffer was released by the last tile's closing barrier
    }
    __syncthreads();  // ... every thread's copies are visible
    const float* sK = sK0 + buf * kTK * LD;
    const float* sV = sV0 + buf * kTK * LD;
    // Scores of this thread's QPT queries x KPT keys.
    float sc[QPT][KPT];
#pragma unroll
    for (int i = 0; i < QPT; ++i)
#pragma unroll
      for (int j = 0; j < KPT; ++j) sc[i][j] = 0.f;
    // Head_dim 128: the 8 query rows of a column step are loaded before the
    // FMAs (3.5% faster there, slower at 64); head_dim 64: the column loop
    // unrolled by 4 (1% faster there).
    constexpr int UNR = D == 64 ? 4 : 2;
#pragma unroll(UNR)
    for (int c = 0; c < D; c += 4) {
      float4 kf[KPT];
#pragma unroll
      for (int j = 0; j < KPT; ++j) kf[j] = *reinterpret_cast<const float4*>(sK + (kc0 + j) * LD + c);
      float4 qa[QPT];
      if constexpr (D == 128) {
#pragma unroll
        for (int i = 0; i < QPT; ++i) qa[i] = *reinterpret_cast<const float4*>(sQ + (qrow0 + i) * LD + c);
      }
#pragma unroll
      for (int i = 0; i < QPT; ++i) {
        const float4 qf = D == 128 ? qa[i] : *reinterpret_cast<const float4*>(sQ + (qrow0 + i) * LD + c);
#pragma unroll
        for (int j = 0; j < KPT; ++j) {
          sc[i][j] = fmaf(qf.x, kf[j].x, sc[i][j]);
          sc[i][j] = fmaf(qf.y, kf[j].y, sc[i][j]);
          sc[i][j] = fmaf(qf.z, kf[j].z, sc[i][j]);
          sc[i][j] = fmaf(qf.w, kf[j].w, sc[i][j]);
        }
      }
    }
    // Online softmax per query row; the row's G threads combine by shuffles.
#pragma unroll
    for (int i = 0; i < QPT; ++i) {
      const int qr = q0 + qrow0 + i;
      float mt = -INFINITY;
#pragma unroll
      for (int j = 0; j < KPT; ++j) {
        const int key = kt + kc0 + j;
        bool valid = key < L && key >= k_lo;
        if (a.causal) valid = valid && key <= qr;
        if (a.window >= 0) valid = valid && abs(qr - key) <= a.window;
        sc[i][j] = valid ? sc[i][j] * a.scale : -INFINITY;
        mt = fmaxf(mt, sc[i][j]);
      }
#pragma unroll
      for (int off = C::G / 2; off > 0; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float m_new = fmaxf(m_r[i], mt);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = expf(m_r[i] - m_use);
      float ps = 0.f;
#pragma unroll
      for (int j = 0; j < KPT; ++j) {
        sc[i][j] = expf(sc[i][j] - m_use);
        ps += sc[i][j];
      }
#pragma unroll
      for (int off = C::G / 2; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l_r[i] = l_r[i] * alpha + ps;
      m_r[i] = m_new;
#pragma unroll
      for (int j = 0; j < 8; ++j) o[i][j] *= alpha;
      float* prow = sP + (qrow0 + i) * LDP + kc0;
      if constexpr (KPT == 4) *reinterpret_cast<float4*>(prow) = make_float4(sc[i][0], sc[i][1], sc[i][2], sc[i][3]);
      else *reinterpret_cast<float2*>(prow) = make_float2(sc[i][0], sc[i][1]);
    }
    __syncthreads();  // P complete
    // O[QPT queries][8 columns] += P[QPT][kTK] . V[kTK][8], four keys at a time.
#pragma unroll 1
    for (int j = 0; j < kTK; j += 4) {
      float4 vf[4][2];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        vf[u][0] = *reinterpret_cast<const float4*>(sV + (j + u) * LD + dc0);
        vf[u][1] = *reinterpret_cast<const float4*>(sV + (j + u) * LD + dc0 + 4);
      }
#pragma unroll
      for (int i = 0; i < QPT; ++i) {
        const float4 pf = *reinterpret_cast<const float4*>(sP + (qrow0 + i) * LDP + j);
        const float p4[4] = {pf.x, pf.y, pf.z, pf.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          o[i][0] = fmaf(p4[u], vf[u][0].x, o[i][0]);
          o[i][1] = fmaf(p4[u], vf[u][0].y, o[i][1]);
          o[i][2] = fmaf(p4[u], vf[u][0].z, o[i][2]);
          o[i][3] = fmaf(p4[u], vf[u][0].w, o[i][3]);
          o[i][4] = fmaf(p4[u], vf[u][1].x, o[i][4]);
          o[i][5] = fmaf(p4[u], vf[u][1].y, o[i][5]);
          o[i][6] = fmaf(p4[u], vf[u][1].z, o[i][6]);
          o[i][7] = fmaf(p4[u], vf[u][1].w, o[i][7]);
        }
      }
    }
    __syncthreads();  // this tile's K, V and P are consumed
  }
  (void)lane;
  float* obase = static_cast<float*>(a.out) + static_cast<long long>(s0) * a.ldo + head * D + dc0;
#pragma unroll
  for (int i = 0; i < QPT; ++i) {
    const int qr = q0 + qrow0 + i;
    if (qr >= L) continue;
    const float inv = l_r[i] > 0.f ? 1.0f / l_r[i] : 0.f;
    float* dst = obase + static_cast<long long>(qr) * a.ldo;
    *reinterpret_cast<float4*>(dst) = make_float4(o[i][0] * inv, o[i][1] * inv, o[i][2] * inv, o[i][3] * inv);
    *reinterpret_cast<float4*>(dst + 4) = make_float4(o[i][4] * inv, o[i][5] * inv, o[i][6] * inv, o[i][7] * inv);
  }
}

template <int D>
int launch_f32_tiled(const AttnArgs& a, cudaStream_t s) {
  using C = F32Tiled<D>;
  static std::atomic<unsigned long long> attr{0}, attr_hx{0};  // one bit per device
  if (a.n_work <= 65535) {
    auto kern = attn_f32_tiled_kernel<D, true>;
    if (set_smem_limit_once(kern, C::SMEM, attr_hx) != cudaSuccess) return -3;
    kern<<<dim3(a.hq, a.n_work), C::THREADS, C::SMEM, s>>>(a);
  } else {
    auto kern = attn_f32_tiled_kernel<D, false>;
    if (set_smem_limit_once(kern, C::SMEM, attr) != cudaSuccess) return -3;
    kern<<<dim3(a.n_work, a.hq), C::THREADS, C::SMEM, s>>>(a);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// The tiled kernel's 16-byte accesses need every row start of q, k, v and
// out 16-byte aligned.
bool f32_tiled_ok(const AttnArgs& a) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return al(a.q) && al(a.k) && al(a.v) && al(a.out) && (a.ldq % 4) == 0 && (a.ldk % 4) == 0 && (a.ldv % 4) == 0 &&
         (a.ldo % 4) == 0;
}

}  // namespace

int attention_q_block(int bf16, int d) {
  if (bf16) return 128;  // the tcgen05 kernel's query tile
  return (d == 64 || d == 128) ? kTQ : kFQ;  // the tiled f32 kernel's, else the SIMT kernel's
}

bool attention_supported(int bf16, int d) {
  if (bf16) return d == 64 || d == 128 || d == 256;
  return d == 8 || d == 16 || d == 32 || d == 64 || d == 128 || d == 256;
}

int attention(const AttnArgs& a, cudaStream_t s) {
  if (a.n_work <= 0) return 0;
  if (a.hq <= 0 || a.hkv <= 0 || a.hq % a.hkv != 0) return -1;
  if (a.bf16) return attention_tc(a, a.total_rows, s);  // head_dim 64, 128, 256 (others: -1)
  if (a.q_block != attention_q_block(0, a.d)) return -1;
  const bool tiled = f32_tiled_ok(a);
  switch (a.d) {
    case 8:
    case 16: return attention_small(a, s);  // tiny checkpoints
    case 32: return launch_f32<32>(a, s);
    case 64: return tiled ? launch_f32_tiled<64>(a, s) : launch_f32<64>(a, s);
    case 128: return tiled ? launch_f32_tiled<128>(a, s) : launch_f32<128>(a, s);
    case 256: return launch_f32<256>(a, s);
    default: return -1;
  }
}

}  // namespace inl
