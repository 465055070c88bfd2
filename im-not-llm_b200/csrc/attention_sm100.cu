// Flash attention on the sm_100a tensor cores for packed variable-length
// texts (bf16, head_dim 64 or 128): causal, bidirectional and sliding-window
// masks computed from positions, grouped-query heads by index.
//
// One CTA = one (text, 128-query tile, query head), 192 threads:
//   warp 0      TMA: the Q tile once, then K_j / V_j tiles of 128 keys into a
//               2-stage ring (kv_full / kv_empty);
//   warp 1      allocates TMEM and issues tcgen05.mma: S_j = Q K_j^T into one of
//               two TMEM score buffers (128 columns each), and O += P_j V_j into
//               the TMEM output (D columns); S_{j+1} is issued before PV_j so
//               the tensor core works while the softmax warps read S_j;
//   warps 2..5  softmax: thread = query row = TMEM lane. Reads S_j with
//               tcgen05.ld, masks, keeps a running row max m and sum l,
//               writes P_j = exp2(s - m) as bf16 into shared memory in the
//               K-major 128-byte-swizzle layout the MMA reads. m is only
//               raised when the block max exceeds it by more than 2^8, and then
//               O is rescaled in TMEM (tcgen05.ld/st), so the common block
//               needs no O round trip. Finally O / l is written as bf16.
// Every mbarrier wait is bounded (status word + early exit, TMEM freed).
#include "common.cuh"
#include "kernels.h"

namespace inl {

namespace {

constexpr int kTQ = 128;   // queries per tile (UMMA M)
constexpr int kTK = 128;   // keys per block (UMMA N of S, K of PV)
constexpr int kBox = 16384;  // one TMA box: 128 rows x 128 bytes
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only when the max grows 256x

template <int D>
struct FaCfg {
  static constexpr int QB = D / 64;  // 64-column boxes per head row
  static constexpr int Q_BYTES = QB * kBox;
  static constexpr int KV_BYTES = QB * kBox;
  static constexpr int P_BYTES = 2 * kBox;  // 128 keys = two 64-key boxes
  static constexpr int SMEM = Q_BYTES + 4 * KV_BYTES + 2 * P_BYTES + 1024 + 256;
  static constexpr int TMEM_COLS = 512;
  static constexpr int O_COL = 2 * kTK;
};

struct FaParams {
  const int* cu;
  const int2* work;
  __nv_bfloat16* out;
  long long ldo;
  int hq, hkv;
  float scale_log2;
  int causal, window;
  int* status;
};

__device__ __forceinline__ bool wait_or_flag(uint64_t* bar, uint32_t parity, int* status, int code, bool& ok) {
  if (!ok) return false;
  ok = mbar_wait(bar, parity, status, code);
  return ok;
}

// Same, with the outcome made uniform across the warp (for the softmax warps,
// whose tcgen05.ld / tcgen05.st must run on all 32 lanes together).
__device__ __forceinline__ bool wait_warp(uint64_t* bar, uint32_t parity, int* status, int code, bool& ok) {
  if (!__all_sync(0xffffffffu, ok)) {
    ok = false;
    return false;
  }
  ok = mbar_wait_warp(bar, parity, status, code);
  return ok;
}

template <int D>
__global__ void __launch_bounds__(192, 1)
    fa_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, FaParams p) {
  using C = FaCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + C::Q_BYTES;            // 2 stages
  uint8_t* sV = sK + 2 * C::KV_BYTES;       // 2 stages
  uint8_t* sP = sV + 2 * C::KV_BYTES;       // 2 buffers
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * C::P_BYTES);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = bars + 3;
  uint64_t* s_full = bars + 5;
  uint64_t* s_free = bars + 7;
  uint64_t* p_full = bars + 9;
  uint64_t* p_free = bars + 11;
  uint64_t* o_done = bars + 13;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 15);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int2 wk = p.work[blockIdx.x];
  const int head = blockIdx.y;
  const int kvh = head / (p.hq / p.hkv);
  const int s0 = p.cu[wk.x];
  const int L = p.cu[wk.x + 1] - s0;
  const int q0 = wk.y * kTQ;
  if (q0 >= L) return;  // uniform for the CTA
  int k_lo = 0, k_hi = L;
  if (p.causal) k_hi = min(L, q0 + kTQ);
  if (p.window >= 0) {
    k_lo = max(0, q0 - p.window);
    k_hi = min(k_hi, q0 + kTQ + p.window);
  }
  const int kb_lo = k_lo / kTK;
  const int n_kv = (k_hi + kTK - 1) / kTK - kb_lo;  // >= 1 because q0 < L

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&p_free[i], 1);
      mbar_init(&o_done[i], 1);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      // Q tile: rows s0 + q0 .. +127, columns head*D .. +D.
      mbar_expect_tx(q_full, C::Q_BYTES);
      for (int b = 0; b < C::QB; ++b) tma_load_2d(sQ + b * kBox, &tmQ, q_full, head * D + b * 64, s0 + q0);
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int st = j & 1;
        if (!wait_or_flag(&kv_empty[st], ((j >> 1) & 1) ^ 1, p.status, INL_DEV_TIMEOUT_PRODUCER, ok)) break;
        mbar_expect_tx(&kv_full[st], 2 * C::KV_BYTES);
        const int row = s0 + (kb_lo + j) * kTK;
        for (int b = 0; b < C::QB; ++b) {
          tma_load_2d(sK + st * C::KV_BYTES + b * kBox, &tmK, &kv_full[st], kvh * D + b * 64, row);
          tma_load_2d(sV + st * C::KV_BYTES + b * kBox, &tmV, &kv_full[st], kvh * D + b * 64, row);
        }
        ++issued;
      }
      // drain: the Q copy and the last two K/V fills must land before exit
      bool dok = true;
      wait_or_flag(q_full, 0, p.status, INL_DEV_TIMEOUT_DRAIN, dok);
      for (int j = max(0, issued - 2); j < issued; ++j) {
        if (!dok) break;
        wait_or_flag(&kv_full[j & 1], (j >> 1) & 1, p.status, INL_DEV_TIMEOUT_DRAIN, dok);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(kTQ, kTK, 0);
      constexpr uint32_t idesc_o = umma_idesc_bf16(kTQ, D, 1);
      const uint32_t q_addr = smem_u32(sQ);
      wait_or_flag(q_full, 0, p.status, INL_DEV_TIMEOUT_MMA, ok);
      for (int j = 0; j <= n_kv && ok; ++j) {
        if (j < n_kv) {
          const int st = j & 1, sb = j & 1;
          if (!wait_or_flag(&kv_full[st], (j >> 1) & 1, p.status, INL_DEV_TIMEOUT_MMA, ok)) break;
          if (!wait_or_flag(&s_free[sb], ((j >> 1) & 1) ^ 1, p.status, INL_DEV_TIMEOUT_MMA, ok)) break;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sK + st * C::KV_BYTES);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kBox + (kk & 3) * 32;
            umma_bf16(tmem + sb * kTK, sw128_kmajor_desc(q_addr + off), sw128_kmajor_desc(k_addr + off), idesc_s,
                      kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[sb]);
        }
        if (j >= 1) {
          const int i = j - 1;
          const int st = i & 1, pb = i & 1;
          if (!wait_or_flag(&p_full[pb], (i >> 1) & 1, p.status, INL_DEV_TIMEOUT_MMA, ok)) break;
          tc_fence_after();
          const uint32_t p_addr = smem_u32(sP + pb * C::P_BYTES);
          const uint32_t v_addr = smem_u32(sV + st * C::KV_BYTES);
#pragma unroll
          for (int kk = 0; kk < kTK / 16; ++kk) {
            const uint32_t a_off = (kk >> 2) * kBox + (kk & 3) * 32;  // P: K-major, 64 keys per box
            const uint32_t b_off = kk * 16 * 128;                      // V: 16 key rows per step
            umma_bf16(tmem + C::O_COL, sw128_kmajor_desc(p_addr + a_off), sw128_mnmajor_desc(v_addr + b_off, kBox),
                      idesc_o, (i > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&o_done[i & 1]);
          umma_commit(&kv_empty[st]);
          umma_commit(&p_free[pb]);
        }
      }
    }
  } else {
    // Softmax warps 2..5: TMEM lane quadrant warp % 4, one query row per thread.
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int q = q0 + r;  // text-relative query
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    float m = -INFINITY, l = 0.f;
    uint8_t* prow_base = sP + r * 128;
    const int sw = r & 7;
    for (int j = 0; j < n_kv; ++j) {
      const int sb = j & 1;
      if (!wait_warp(&s_full[sb], (j >> 1) & 1, p.status, INL_DEV_TIMEOUT_EPILOGUE, ok)) break;
      tc_fence_after();
      uint32_t sv[kTK];
#pragma unroll
      for (int c = 0; c < kTK; c += 32) tmem_ld32(lane_base + sb * kTK + c, *reinterpret_cast<uint32_t(*)[32]>(&sv[c]));
      tmem_ld_wait();
      const int key0 = (kb_lo + j) * kTK;
      const bool full_block = key0 + kTK <= L && (!p.causal || key0 + kTK - 1 <= q0) &&
                              (p.window < 0 || (q0 + kTQ - 1 - key0 <= p.window && key0 + kTK - 1 - q0 <= p.window));
      // Row max with 8 independent partial maxima (a single 128-long chain of
      // fmaxf would serialise on its latency).
      float mp[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) mp[t] = -INFINITY;
      if (full_block) {
#pragma unroll
        for (int c = 0; c < kTK; ++c) mp[c & 7] = fmaxf(mp[c & 7], __uint_as_float(sv[c]));
      } else {
#pragma unroll
        for (int c = 0; c < kTK; ++c) {
          const int key = key0 + c;
          bool valid = key < L;
          if (p.causal) valid = valid && key <= q;
          if (p.window >= 0) valid = valid && abs(q - key) <= p.window;
          if (!valid) sv[c] = __float_as_uint(-INFINITY);
          mp[c & 7] = fmaxf(mp[c & 7], __uint_as_float(sv[c]));
        }
      }
      const float mx = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                             fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
      const float m_blk = mx * p.scale_log2;
      // P_j goes into buffer j & 1: wait until PV_{j-2} released it.
      if (!wait_warp(&p_free[sb], ((j >> 1) & 1) ^ 1, p.status, INL_DEV_TIMEOUT_EPILOGUE, ok)) break;
      // Raise the running max only when the block max exceeds it by > 2^8.
      // Rows that held a finite max and had PV blocks accumulated need O
      // rescaled; the decision is per row, the TMEM round trip per warp.
      const bool raise = m_blk > m + kRescaleThreshold;
      const bool rescale_row = raise && j > 0 && m != -INFINITY;
      const float alpha = rescale_row ? ex2_approx(m - m_blk) : 1.0f;
      if (__any_sync(0xffffffffu, rescale_row)) {
        const int i = j - 1;  // O holds PV_0..PV_{j-1}; wait for PV_{j-1}
        if (!wait_warp(&o_done[i & 1], (i >> 1) & 1, p.status, INL_DEV_TIMEOUT_EPILOGUE, ok)) break;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D; c += 32) {
          uint32_t o[32];
          tmem_ld32(lane_base + C::O_COL + c, o);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 32; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * alpha);
          tmem_st32(lane_base + C::O_COL + c, o);
        }
        tmem_st_wait();
      }
      if (raise) {
        l *= alpha;
        m = m_blk;
      }
      const float m_use = m == -INFINITY ? 0.f : m;
      float rs8[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) rs8[t] = 0.f;
      uint8_t* pb = prow_base + sb * C::P_BYTES;
#pragma unroll
      for (int c = 0; c < kTK; c += 8) {
        uint32_t hb[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const float e = ex2_approx(fmaf(__uint_as_float(sv[c + t]), p.scale_log2, -m_use));
          rs8[t] += e;
          // bf16 round-to-nearest-even on the integer pipe (e >= 0 and finite),
          // keeping the conversion off the MUFU/XU pipe the exp2 needs.
          const uint32_t b = __float_as_uint(e);
          hb[t] = b + 0x7FFFu + ((b >> 16) & 1u);
        }
        uint4 w;
        w.x = __byte_perm(hb[0], hb[1], 0x7632);
        w.y = __byte_perm(hb[2], hb[3], 0x7632);
        w.z = __byte_perm(hb[4], hb[5], 0x7632);
        w.w = __byte_perm(hb[6], hb[7], 0x7632);
        const int chunk = c >> 3;  // 16-byte chunk index 0..15 over 128 keys
        *reinterpret_cast<uint4*>(pb + (chunk >> 3) * kBox + (((chunk & 7) ^ sw) << 4)) = w;
      }
      const float rowsum = ((rs8[0] + rs8[1]) + (rs8[2] + rs8[3])) + ((rs8[4] + rs8[5]) + (rs8[6] + rs8[7]));
      l += rowsum;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
      mbar_arrive(&s_free[sb]);
    }
    // Output: wait for the last PV, then O / l -> bf16.
    const int last = n_kv - 1;
    if (wait_warp(&o_done[last & 1], (last >> 1) & 1, p.status, INL_DEV_TIMEOUT_EPILOGUE, ok)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      __nv_bfloat16* orow = p.out + static_cast<long long>(s0 + q) * p.ldo + head * D;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        uint32_t o[32];
        tmem_ld32(lane_base + C::O_COL + c, o);
        tmem_ld_wait();
        if (q < L) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(o[8 * t + 0]) * inv, __uint_as_float(o[8 * t + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(o[8 * t + 2]) * inv, __uint_as_float(o[8 * t + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(o[8 * t + 4]) * inv, __uint_as_float(o[8 * t + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(o[8 * t + 6]) * inv, __uint_as_float(o[8 * t + 7]) * inv);
            dst[t] = w;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int D>
int launch_fa(const AttnArgs& a, long long total_rows, cudaStream_t s) {
  using C = FaCfg<D>;
  CUtensorMap tq, tk, tv;
  if (!make_tma_2d_bf16(&tq, a.q, total_rows, static_cast<long long>(a.hq) * D, a.ldq, kTQ, 64)) return -2;
  if (!make_tma_2d_bf16(&tk, a.k, total_rows, static_cast<long long>(a.hkv) * D, a.ldk, kTK, 64)) return -2;
  if (!make_tma_2d_bf16(&tv, a.v, total_rows, static_cast<long long>(a.hkv) * D, a.ldv, kTK, 64)) return -2;
  auto kern = fa_sm100_kernel<D>;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess) return -3;
    attr = true;
  }
  FaParams p;
  p.cu = a.cu;
  p.work = a.work;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.ldo = a.ldo;
  p.hq = a.hq;
  p.hkv = a.hkv;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.causal = a.causal;
  p.window = a.window;
  p.status = a.status;
  dim3 grid(a.n_work, a.hq);
  kern<<<grid, 192, C::SMEM, s>>>(tq, tk, tv, p);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace

bool attention_tc_supported(int d) { return d == 64 || d == 128; }

int attention_tc(const AttnArgs& a, long long total_rows, cudaStream_t s) {
  if (a.n_work <= 0) return 0;
  if (a.hq <= 0 || a.hkv <= 0 || a.hq % a.hkv != 0 || a.q_block != kTQ) return -1;
  if ((reinterpret_cast<uintptr_t>(a.q) & 15) || (reinterpret_cast<uintptr_t>(a.k) & 15) ||
      (reinterpret_cast<uintptr_t>(a.v) & 15) || (reinterpret_cast<uintptr_t>(a.out) & 15) || (a.ldq % 8) ||
      (a.ldk % 8) || (a.ldv % 8) || (a.ldo % 8))
    return -1;
  switch (a.d) {
    case 64: return launch_fa<64>(a, total_rows, s);
    case 128: return launch_fa<128>(a, total_rows, s);
    default: return -1;
  }
}

}  // namespace inl
