// Variable-length attention over packed texts: causal, bidirectional and
// sliding-window (|q - k| <= window), grouped-query (query head h reads KV head
// h / (hq / hkv)), masks computed from positions instead of materialised.
//
// bf16: flash-attention style, 4 warps x 16 query rows, 64-key blocks staged
// by cp.async (double-buffered, XOR-swizzled rows), S = Q K^T and O += P V on
// mma.sync.m16n8k16 with f32 accumulation, online softmax in registers; the
// score matrix never leaves registers.
// f32: SIMT kernel for the f32-accurate configurations: 32 queries per CTA,
// 32-key tiles in shared memory, one lane per key for the scores and one lane
// per head dimension slice for the output.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace inl {

namespace {

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Swizzled element offset of (row, col) in a [rows, D] bf16 tile: the 16-byte
// chunk index is XORed with row % 8 so ldmatrix row reads hit distinct banks.
template <int D>
__device__ __forceinline__ int swz(int row, int col) {
  return row * D + ((((col >> 3) ^ (row & 7))) << 3) + (col & 7);
}

constexpr int kBM = 64;
constexpr int kBN = 64;

template <int D>
struct FlashSmem {
  static constexpr int Q = kBM * D;
  static constexpr int KV = kBN * D;
  static constexpr int BYTES = (Q + 4 * KV) * 2;
};

// Copy rows [row0, row0 + ROWS) (text-relative, < L valid) of a head slice into a swizzled tile.
template <int D, int ROWS>
__device__ __forceinline__ void load_tile(__nv_bfloat16* dst, const __nv_bfloat16* base, long long ld, int row0,
                                          int L, int tid) {
  constexpr int CH = D / 8;
  for (int idx = tid; idx < ROWS * CH; idx += 128) {
    const int r = idx / CH, ch = idx - (idx / CH) * CH;
    const int gr = row0 + r;
    const bool valid = gr >= 0 && gr < L;
    const __nv_bfloat16* src = valid ? base + static_cast<long long>(gr) * ld + ch * 8 : base;
    cp_async16(dst + swz<D>(r, ch * 8), src, valid ? 16 : 0);
  }
}

template <int D>
__global__ void __launch_bounds__(128) flash_fwd_bf16_kernel(AttnArgs a) {
  constexpr int NB = kBN / 8;   // key n-blocks per tile
  constexpr int KC = D / 16;    // k chunks over the head dim
  constexpr int DB = D / 8;     // output n-blocks over the head dim
  extern __shared__ __align__(128) uint8_t smem[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* sK = sQ + FlashSmem<D>::Q;
  __nv_bfloat16* sV = sK + 2 * FlashSmem<D>::KV;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int2 wk = a.work[blockIdx.x];
  const int text = wk.x, qb = wk.y;
  const int head = blockIdx.y;
  const int kvh = head / (a.hq / a.hkv);
  const int s0 = a.cu[text];
  const int L = a.cu[text + 1] - s0;
  const int q0 = qb * kBM;
  if (q0 >= L) return;

  int k_lo = 0, k_hi = L;
  if (a.causal) k_hi = min(L, q0 + kBM);
  if (a.window >= 0) {
    k_lo = max(0, q0 - a.window);
    k_hi = min(k_hi, q0 + kBM + a.window);
  }
  const int kb_lo = k_lo / kBN;
  const int kb_hi = (k_hi + kBN - 1) / kBN;

  const __nv_bfloat16* qbase = static_cast<const __nv_bfloat16*>(a.q) + static_cast<long long>(s0) * a.ldq + head * D;
  const __nv_bfloat16* kbase = static_cast<const __nv_bfloat16*>(a.k) + static_cast<long long>(s0) * a.ldk + kvh * D;
  const __nv_bfloat16* vbase = static_cast<const __nv_bfloat16*>(a.v) + static_cast<long long>(s0) * a.ldv + kvh * D;

  load_tile<D, kBM>(sQ, qbase, a.ldq, q0, L, tid);
  if (kb_lo < kb_hi) {
    load_tile<D, kBN>(sK, kbase, a.ldk, kb_lo * kBN, L, tid);
    load_tile<D, kBN>(sV, vbase, a.ldv, kb_lo * kBN, L, tid);
  }
  cp_async_commit();

  float o[DB][4];
#pragma unroll
  for (int j = 0; j < DB; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY};
  float l_r[2] = {0.f, 0.f};
  const float sl2 = a.scale * 1.4426950408889634f;
  const int qrow0 = q0 + warp * 16 + (lane >> 2);  // text-relative query of c0/c1; +8 for c2/c3
  const uint32_t sQa = smem_u32(sQ), sKa = smem_u32(sK), sVa = smem_u32(sV);

  for (int kb = kb_lo; kb < kb_hi; ++kb) {
    const int cur = (kb - kb_lo) & 1;
    if (kb + 1 < kb_hi) {
      load_tile<D, kBN>(sK + (cur ^ 1) * FlashSmem<D>::KV, kbase, a.ldk, (kb + 1) * kBN, L, tid);
      load_tile<D, kBN>(sV + (cur ^ 1) * FlashSmem<D>::KV, vbase, a.ldv, (kb + 1) * kBN, L, tid);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();

    // S = Q K^T for this warp's 16 rows x 64 keys.
    float s[NB][4];
#pragma unroll
    for (int j = 0; j < NB; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    const uint32_t kt = sKa + cur * FlashSmem<D>::KV * 2;
#pragma unroll
    for (int kc = 0; kc < KC; ++kc) {
      uint32_t qa[4];
      {
        const int r = warp * 16 + (lane & 15);
        const int c = kc * 16 + (lane >> 4) * 8;
        ldsm_x4(sQa + swz<D>(r, c) * 2, qa[0], qa[1], qa[2], qa[3]);
      }
#pragma unroll
      for (int np = 0; np < NB / 2; ++np) {
        const int r = np * 16 + (lane & 7) + (lane >> 4) * 8;
        const int c = kc * 16 + ((lane >> 3) & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kt + swz<D>(r, c) * 2, b0, b1, b2, b3);
        mma_bf16_16816(s[2 * np], qa, b0, b1);
        mma_bf16_16816(s[2 * np + 1], qa, b2, b3);
      }
    }

    // Mask + online softmax (rows qrow0 and qrow0 + 8).
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < NB; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kb * kBN + j * 8 + (lane & 3) * 2 + (e & 1);
        const int qr = qrow0 + (e >> 1) * 8;
        bool valid = key < L && key >= 0;
        if (a.causal) valid = valid && key <= qr;
        if (a.window >= 0) valid = valid && abs(qr - key) <= a.window;
        const float v = valid ? s[j][e] * sl2 : -INFINITY;
        s[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float m_new = fmaxf(m_r[r], mx[r]);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      alpha[r] = exp2f(m_r[r] - m_use);
      m_r[r] = m_new;
      mx[r] = m_use;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < NB; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p = exp2f(s[j][e] - mx[e >> 1]);
        s[j][e] = p;
        rs[e >> 1] += p;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l_r[r] = l_r[r] * alpha[r] + rs[r];
    }
#pragma unroll
    for (int j = 0; j < DB; ++j) {
      o[j][0] *= alpha[0];
      o[j][1] *= alpha[0];
      o[j][2] *= alpha[1];
      o[j][3] *= alpha[1];
    }

    // O += P V.
    const uint32_t vt = sVa + cur * FlashSmem<D>::KV * 2;
#pragma unroll
    for (int kc = 0; kc < kBN / 16; ++kc) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(s[2 * kc][0], s[2 * kc][1]);
      pa[1] = pack_bf16x2(s[2 * kc][2], s[2 * kc][3]);
      pa[2] = pack_bf16x2(s[2 * kc + 1][0], s[2 * kc + 1][1]);
      pa[3] = pack_bf16x2(s[2 * kc + 1][2], s[2 * kc + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        const int r = kc * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = dp * 16 + (lane >> 4) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vt + swz<D>(r, c) * 2, b0, b1, b2, b3);
        mma_bf16_16816(o[2 * dp], pa, b0, b1);
        mma_bf16_16816(o[2 * dp + 1], pa, b2, b3);
      }
    }
    __syncthreads();
  }

  // Normalise and store.
  __nv_bfloat16* obase = static_cast<__nv_bfloat16*>(a.out) + static_cast<long long>(s0) * a.ldo + head * D;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qr = qrow0 + r * 8;
    if (qr >= L) continue;
    const float inv = l_r[r] > 0.f ? 1.0f / l_r[r] : 0.f;
    __nv_bfloat16* orow = obase + static_cast<long long>(qr) * a.ldo;
#pragma unroll
    for (int j = 0; j < DB; ++j) {
      const int c = j * 8 + (lane & 3) * 2;
      *reinterpret_cast<uint32_t*>(orow + c) = pack_bf16x2(o[j][2 * r] * inv, o[j][2 * r + 1] * inv);
    }
  }
}

// ------------------------------------------------------------------ f32 SIMT
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
int launch_flash(const AttnArgs& a, cudaStream_t s) {
  auto kern = flash_fwd_bf16_kernel<D>;
  constexpr int bytes = FlashSmem<D>::BYTES;
  static std::atomic<unsigned long long> attr{0};  // one bit per device
  if (set_smem_limit_once(kern, bytes, attr) != cudaSuccess) return -3;
  dim3 grid(a.n_work, a.hq);
  kern<<<grid, 128, bytes, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
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
  if (bf16) return attention_tc_supported(d) ? 128 : kBM;
  return kFQ;
}

bool attention_supported(int bf16, int d) {
  if (bf16) return d == 64 || d == 128 || d == 256;
  return d == 8 || d == 16 || d == 32 || d == 64 || d == 128 || d == 256;
}

int attention(const AttnArgs& a, cudaStream_t s) {
  if (a.n_work <= 0) return 0;
  if (a.hq <= 0 || a.hkv <= 0 || a.hq % a.hkv != 0) return -1;
  if (a.bf16 && attention_tc_supported(a.d)) return attention_tc(a, a.total_rows, s);
  if (a.bf16) {
    if (a.q_block != kBM) return -1;
    switch (a.d) {
      case 64: return launch_flash<64>(a, s);
      case 128: return launch_flash<128>(a, s);
      case 256: return launch_flash<256>(a, s);
      default: return -1;
    }
  }
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
