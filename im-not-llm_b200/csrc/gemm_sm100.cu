// Persistent bf16 GEMM for sm_100a on the 5th-generation tensor cores.
//
//   Y[M, N] = X[M, K] . W[N, K]^T        (X = packed token rows, W = nn.Linear weight)
//
// One CTA per SM, 320 threads, warp-specialised:
//   warp 0      TMA producer: X and W tiles -> shared memory (128-byte swizzle),
//               STAGES-deep ring guarded by full/empty mbarriers;
//   warp 1      allocates TMEM and issues tcgen05.mma (one elected thread),
//               M=128 x N=BN x K=16 per instruction, accumulators in TMEM,
//               two accumulator buffers so the epilogue of tile i overlaps the
//               main loop of tile i+1;
//   warps 2..9  epilogue: tcgen05.ld TMEM -> registers, fused epilogue
//               (plain store, residual add, gated activation, q/k norm + RoPE,
//               f32 store, per-row scale). Warp w reads TMEM lane quadrant
//               w % 4 (tile rows 32*(w%4) .. +31, one row per thread) and half
//               (w - 2) / 4 of the tile's columns. bf16 results leave 32 x 32 at a
//               time through a shared-memory staging area and a TMA tensor store.
// Tiles are walked in row-major tile order by a static stride-gridDim
// schedule, so the CTAs resident at one time share the same few X row blocks
// and read W (a few MB) out of L2.
#include <cstdio>
#include <cstring>

#include "common.cuh"
#include "kernels.h"

namespace inl {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // one 128-byte swizzle row of bf16
constexpr int kEpiWarps = 8;  // two warps per TMEM lane quadrant, each owning half of the tile's columns
constexpr int kThreads = 64 + 32 * kEpiWarps;

template <int BN>
struct GemmCfg {
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_BYTES = BN * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;  // two accumulator buffers
  static constexpr int OUT_STAGE_BYTES = kEpiWarps * 2 * 32 * 64;  // per epilogue warp: 2 chunks of 32 x 32 bf16
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + OUT_STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

struct EpiArgs {
  void* out;
  long long ldo;
  const __nv_bfloat16* resid;
  long long ldr;
  const float* ss_in;
  int ss_in_parts, ss_dim;
  float ss_eps;
  float* ss_out;
  int ss_out_parts;
  const float* qn;
  const float* kn;
  const int* pos;
  const float* cos;
  const float* sin;
  int hq, hkv, d, max_pos;
  float qk_eps;
  int* status;
  int M, N;
  const int* seg;
  int* pooled;
  long long ldp;
  // split-K (f32 output only): the K blocks of a tile are cut into `splits`
  // slices; slice s writes its partial product at out + s * split_stride
  int splits;
  long long split_stride;
};

// A work unit of the persistent schedule: a tile and the K blocks [kb0, kb1)
// of its slice (the whole K without split-K).
struct Unit {
  int tile, kb0, kb1, slice;
};
__device__ __forceinline__ Unit unit_of(int u, int splits, int k_blocks) {
  Unit w;
  w.tile = u / splits;
  w.slice = u - w.tile * splits;
  const int per = (k_blocks + splits - 1) / splits;
  w.kb0 = w.slice * per;
  w.kb1 = min(k_blocks, w.kb0 + per);
  return w;
}

// Output path of one epilogue warp: 32 rows x 32 bf16 columns at a time go
// through a double-buffered 2 KB staging area in shared memory (64-byte rows,
// 64-byte swizzle: the 16-byte piece j of row r sits at piece j ^ ((r >> 1) & 3),
// which keeps each 8-lane group of a warp's stores on distinct banks) and leave
// with one TMA tensor store, instead of 32 scattered 16-byte stores per
// instruction. Rows and columns past the output's extent are clipped by the
// tensor map. Every lane of the warp calls it together.
struct OutStage {
  const CUtensorMap* map;
  uint8_t* buf;  // this warp's 2 x 2048 bytes
  int issued;    // chunks stored so far
};
constexpr int kStageChunkBytes = 32 * 64;

__device__ __forceinline__ void stage_store32(OutStage& st, const float (&v)[32], int col, int row0, int lane) {
  uint8_t* b = st.buf + (st.issued & 1) * kStageChunkBytes;
  if (st.issued >= 2) {
    if (lane == 0) bulk_wait_group_read<1>();  // the store that last used this buffer has read it
    __syncwarp();
  }
  uint8_t* rowp = b + lane * 64;
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 w;
    w.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
    w.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
    w.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
    w.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
    *reinterpret_cast<uint4*>(rowp + ((j ^ sw) << 4)) = w;
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(st.map, b, col, row0);
    bulk_commit_group();
  }
  ++st.issued;
}

template <int ACT>
__device__ __forceinline__ float gate_act(float x) {
  if constexpr (ACT == INL_ACT_SILU) return silu_f(x);
  else if constexpr (ACT == INL_ACT_GELU_ERF) return gelu_erf_f(x);
  else return gelu_tanh_f(x);
}

__device__ __forceinline__ void load_row32_bf16(const __nv_bfloat16* src, float (&v)[32], int ncols_left) {
  if (ncols_left >= 32) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 w = s4[j];
      float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), c = unpack_bf16x2(w.z), d = unpack_bf16x2(w.w);
      v[8 * j + 0] = a.x; v[8 * j + 1] = a.y; v[8 * j + 2] = b.x; v[8 * j + 3] = b.y;
      v[8 * j + 4] = c.x; v[8 * j + 5] = c.y; v[8 * j + 6] = d.x; v[8 * j + 7] = d.y;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = j < ncols_left ? __bfloat162float(src[j]) : 0.f;
  }
}

// Sum of squares of the bf16-rounded values (what the next GEMM reads back).
__device__ __forceinline__ float ss_bf16_32(const float (&v)[32]) {
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    const float2 r = unpack_bf16x2(pack_bf16x2(v[j], v[j + 1]));
    s = fmaf(r.x, r.x, s);
    s = fmaf(r.y, r.y, s);
  }
  return s;
}

// One q or k head of width D in TMEM columns [c0, c0 + D) of this thread's row:
// RMSNorm with weight w, then half-split RoPE at position p, stored through st
// at output columns col0 .. col0 + D of rows row0 .. row0 + 31.
// rp is the RoPE table packed by frequency pairs, [D/4, max_pos] float4 =
// (cos f, cos f+1, sin f, sin f+1) for f = 2i: one 16-byte load serves two
// frequencies, and the 32 threads of a warp (consecutive tokens, mostly
// consecutive positions) read consecutive float4s. w is read as float4.
template <int D>
__device__ __forceinline__ void qk_head(uint32_t t_row, int c0, float rs, const float* __restrict__ w, float eps,
                                        const float4* __restrict__ rp, int p, int max_pos, OutStage& st, int col0,
                                        int row0, int lane) {
  uint32_t r[32], u[32];
  float ss = 0.f;
#pragma unroll 1
  for (int c = 0; c < D; c += 32) {
    tmem_ld32(t_row + c0 + c, r);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float x = __uint_as_float(r[j]) * rs;
      ss = fmaf(x, x, ss);
    }
  }
  const float inv = rsqrtf(ss / static_cast<float>(D) + eps) * rs;
  constexpr int HALF = D / 2;
#pragma unroll 1
  for (int c = 0; c < HALF; c += 32) {
    tmem_ld32(t_row + c0 + c, r);
    tmem_ld32(t_row + c0 + HALF + c, u);
    tmem_ld_wait();
    float lo[32], hi[32];  // rows past M are computed too (p = 0) and clipped by the store
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 wl = __ldg(reinterpret_cast<const float4*>(w + c + j));
      const float4 wh = __ldg(reinterpret_cast<const float4*>(w + HALF + c + j));
      const float4 t0 = __ldg(rp + static_cast<long long>((c + j) >> 1) * max_pos + p);
      const float4 t1 = __ldg(rp + static_cast<long long>(((c + j) >> 1) + 1) * max_pos + p);
      const float a[4] = {wl.x, wl.y, wl.z, wl.w}, b[4] = {wh.x, wh.y, wh.z, wh.w};
      const float cs[4] = {t0.x, t0.y, t1.x, t1.y}, sn[4] = {t0.z, t0.w, t1.z, t1.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float x1 = __uint_as_float(r[j + i]) * inv * a[i];
        const float x2 = __uint_as_float(u[j + i]) * inv * b[i];
        lo[j + i] = x1 * cs[i] - x2 * sn[i];
        hi[j + i] = x2 * cs[i] + x1 * sn[i];
      }
    }
    stage_store32(st, lo, col0 + c, row0, lane);
    stage_store32(st, hi, col0 + HALF + c, row0, lane);
  }
}

// Epilogue of one tile for one warp: TMEM lanes = tile rows (one per thread),
// columns [half * BN/2, (half + 1) * BN/2) of the tile.
template <int BN, int EPI, int ACT>
__device__ __forceinline__ void epilogue_tile(uint32_t t_row, int row, int n0, int half, const EpiArgs& e,
                                              OutStage& st, int lane, long long out_off = 0) {
  constexpr int HW = BN / 2;
  const bool row_ok = row < e.M;
  const int row0 = row - lane;  // first row of this warp's 32
  float rs = 1.0f;
  if (e.ss_in != nullptr && row_ok) {
    const float* sp = e.ss_in + static_cast<long long>(row) * e.ss_in_parts;
    float t = 0.f;
    if ((e.ss_in_parts & 3) == 0) {
      for (int j = 0; j < e.ss_in_parts; j += 4) {
        const float4 v4 = *reinterpret_cast<const float4*>(sp + j);
        t += (v4.x + v4.y) + (v4.z + v4.w);
      }
    } else {
      for (int j = 0; j < e.ss_in_parts; ++j) t += sp[j];
    }
    rs = rsqrtf(t / static_cast<float>(e.ss_dim) + e.ss_eps);
  }
  uint32_t r[32];
  float v[32];
  if constexpr (EPI == INL_EPI_GATED_BF16 || EPI == INL_EPI_GATED_F32) {
    // Tile columns [0, BN/2) are gate, [BN/2, BN) up (weights interleaved in
    // BN/2-row blocks at load time); this warp makes output columns
    // [half * BN/4, (half + 1) * BN/4) of the tile's BN/2.
    constexpr int Q = BN / 4;
    const int out_n = e.N / 2;
    const int o0 = n0 / 2 + half * Q;
#pragma unroll 1
    for (int c = 0; c < Q; c += 32) {
      uint32_t u[32];
      tmem_ld32(t_row + half * Q + c, r);
      tmem_ld32(t_row + HW + half * Q + c, u);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = gate_act<ACT>(__uint_as_float(r[j]) * rs) * (__uint_as_float(u[j]) * rs);
      if (o0 + c >= out_n) continue;  // uniform
      if constexpr (EPI == INL_EPI_GATED_F32) {
        // gate blocks are multiples of 32 columns, so a chunk is whole
        if (row_ok) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(e.out) + static_cast<long long>(row) * e.ldo + o0 + c);
#pragma unroll
          for (int j = 0; j < 8; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
      } else {
        stage_store32(st, v, o0 + c, row0, lane);  // rows past M are clipped
      }
    }
  } else if constexpr (EPI == INL_EPI_SEGMAX) {
    // Rows are vocabulary entries, columns are packed tokens of segment seg[col]:
    // a running max per segment run, flushed with one atomicMax per run.
    // seg[col] is the same for every lane, so the branches stay warp-uniform.
    // The 32 columns' segments arrive with one coalesced load per chunk,
    // requested before the TMEM read so the two latencies overlap; each
    // column's segment is then shuffled from the lane that loaded it. The
    // inner loop is unrolled in full so that r[] stays in registers.
    int cur = -1;
    float mx = -INFINITY;
#pragma unroll 1
    for (int c = 0; c < HW; c += 32) {
      const int c0 = n0 + half * HW + c;
      const int my_seg = c0 + lane < e.N ? __ldg(e.seg + c0 + lane) : -1;
      tmem_ld32(t_row + half * HW + c, r);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int sg = __shfl_sync(0xffffffffu, my_seg, j);
        const float v = __uint_as_float(r[j]);
        if (sg != cur) {
          if (cur >= 0 && row_ok) atomicMax(e.pooled + static_cast<long long>(cur) * e.ldp + row, encode_ordered(mx));
          cur = sg;
          mx = v;
        } else {
          mx = fmaxf(mx, v);
        }
      }
    }
    if (cur >= 0 && row_ok) atomicMax(e.pooled + static_cast<long long>(cur) * e.ldp + row, encode_ordered(mx));
  } else if constexpr (EPI == INL_EPI_QKV) {
    // Heads of width d inside this warp's BN/2 columns; q heads first, then k, then v.
    const int c_begin = n0 + half * HW;
    int p = 0;
    if (row_ok) {
      p = e.pos[row];
      if (p < 0 || p >= e.max_pos) {
        if (e.status) atomicCAS(e.status, 0, INL_DEV_BAD_INDEX);
        p = 0;
      }
    }
    const int hd = e.d;
#pragma unroll 1
    for (int hc = 0; hc < HW; hc += hd) {
      const int col = c_begin + hc;
      if (col >= e.N) break;
      const int head = col / hd;
      if (head < e.hq + e.hkv) {
        const float* w = head < e.hq ? e.qn : e.kn;
        if (hd == 128)
          qk_head<128>(t_row, half * HW + hc, rs, w, e.qk_eps, reinterpret_cast<const float4*>(e.cos), p, e.max_pos,
                       st, col, row0, lane);
        else
          qk_head<64>(t_row, half * HW + hc, rs, w, e.qk_eps, reinterpret_cast<const float4*>(e.cos), p, e.max_pos,
                      st, col, row0, lane);
      } else {
#pragma unroll 1
        for (int c = 0; c < hd; c += 32) {
          tmem_ld32(t_row + half * HW + hc + c, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * rs;
          stage_store32(st, v, col + c, row0, lane);
        }
      }
    }
  } else {
#pragma unroll 1
    for (int c = 0; c < HW; c += 32) {
      tmem_ld32(t_row + half * HW + c, r);
      tmem_ld_wait();
      const int col = n0 + half * HW + c;
      const int left = e.N - col;
      if (left <= 0) continue;  // warp-uniform
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * rs;
      if constexpr (EPI == INL_EPI_F32 || EPI == INL_EPI_RESID_F32) {
        if (!row_ok) continue;
        float* dst = reinterpret_cast<float*>(e.out) + out_off + static_cast<long long>(row) * e.ldo + col;
        if constexpr (EPI == INL_EPI_RESID_F32) {
          // read before the store: out may alias the residual
          const float* src = reinterpret_cast<const float*>(e.resid) + static_cast<long long>(row) * e.ldr + col;
          if (left >= 32) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 q4 = reinterpret_cast<const float4*>(src)[j];
              v[4 * j] += q4.x;
              v[4 * j + 1] += q4.y;
              v[4 * j + 2] += q4.z;
              v[4 * j + 3] += q4.w;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < left) v[j] += src[j];
          }
        }
        if (left >= 32) {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            reinterpret_cast<float4*>(dst)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)  // static indices keep v[] in registers
            if (j < left) dst[j] = v[j];
        }
      } else {
        if constexpr (EPI == INL_EPI_RESID_BF16) {
          if (row_ok) {
          float rr[32];
          load_row32_bf16(e.resid + static_cast<long long>(row) * e.ldr + col, rr, left);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] += rr[j];
          if (e.ss_out != nullptr) {
            // two 32-column chunks per INL_SS_COLS partial: combine in registers
            const float s = ss_bf16_32(v);
            float* so = e.ss_out + static_cast<long long>(row) * e.ss_out_parts + col / INL_SS_COLS;
            if ((c & 32) == 0) *so = s;
            else *so += s;
          }
          }
        }
        stage_store32(st, v, col, row0, lane);  // rows past M / columns past N are clipped
      }
    }
  }
}

template <int BN, int EPI, int ACT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmO, int M, int N, int K, EpiArgs e, int* status) {
  using C = GemmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint8_t* sOut = sB + C::STAGES * C::B_BYTES;  // output staging of the epilogue warps
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + C::OUT_STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);

  pdl_trigger();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tiles = (M + kBM - 1) / kBM;
  const int n_tiles = (N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int k_blocks = (K + kBK - 1) / kBK;
  const int splits = e.splits > 1 ? e.splits : 1;
  const int num_units = num_tiles * splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiWarps);  // one arrival per epilogue warp
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_wait();  // the previous kernel's outputs (A, residual, sums of squares) are complete

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        const Unit w = unit_of(u, splits, k_blocks);
        const int mb = w.tile / n_tiles, nb = w.tile - (w.tile / n_tiles) * n_tiles;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, status, INL_DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[stage], C::STAGE_BYTES);
          tma_load_2d(sA + stage * C::A_BYTES, &tmA, &full[stage], kb * kBK, mb * kBM);
          tma_load_2d(sB + stage * C::B_BYTES, &tmB, &full[stage], kb * kBK, nb * BN);
          ++issued;
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: every copy this thread issued must have landed before the CTA
      // can exit (on the normal path the MMA warp already consumed them all).
      const long long first = issued > C::STAGES ? issued - C::STAGES : 0;
      for (long long f = first; f < issued; ++f) {
        const int s = static_cast<int>(f % C::STAGES);
        const uint32_t ph = static_cast<uint32_t>((f / C::STAGES) & 1);
        if (!mbar_wait(&full[s], ph, status, INL_DEV_TIMEOUT_DRAIN)) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kBM, BN);
      const uint64_t a_desc0 = sw128_kmajor_desc(smem_u32(sA)), b_desc0 = sw128_kmajor_desc(smem_u32(sB));
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        const Unit w = unit_of(u, splits, k_blocks);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, status, INL_DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, status, INL_DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // Descriptors differ from the ring's base descriptors only in the
          // start-address field (address >> 4, 14 bits; shared memory < 256 KB).
          const uint64_t a_desc = a_desc0 + static_cast<uint64_t>((stage * C::A_BYTES) >> 4);
          const uint64_t b_desc = b_desc0 + static_cast<uint64_t>((stage * C::B_BYTES) >> 4);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            umma_bf16(d_tmem, a_desc + static_cast<uint64_t>(kk * 2), b_desc + static_cast<uint64_t>(kk * 2), idesc,
                      (kb != w.kb0 || kk != 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // Epilogue warps 2..9: lane quadrant warp % 4, column half (warp - 2) / 4.
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    OutStage st{&tmO, sOut + (warp - 2) * 2 * kStageChunkBytes, 0};
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
      const Unit w = unit_of(u, splits, k_blocks);
      const int mb = w.tile / n_tiles, nb = w.tile - (w.tile / n_tiles) * n_tiles;
      if (!mbar_wait_warp(&tfull[acc], acc_phase, status, INL_DEV_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
      const int row = mb * kBM + quad * 32 + lane;
      epilogue_tile<BN, EPI, ACT>(t_row, row, nb * BN, half, e, st, lane, w.slice * e.split_stride);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (lane == 0) bulk_wait_group<0>();  // output stores finished before the CTA's shared memory goes away
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ CTA-pair GEMM
// The same GEMM on CTA pairs (clusters of 2) with tcgen05 cta_group::2: a pair
// computes a 256 x 256 tile. Each CTA loads its 128 rows of X and its 128 rows of
// W (its half of the tile's N) per K step, 32 KB instead of the 48 KB a CTA
// loads for a 128 x 256 tile alone, and the leading CTA issues one M = 256
// MMA stream that reads both CTAs' shared memory and writes each CTA's 128
// accumulator rows into its own TMEM. Every CTA then runs the usual epilogue
// on its own rows. Handshake:
//   full[s]   (leading CTA only) armed by the leader's producer for both CTAs'
//             bytes; both producers' TMA loads complete on it;
//   empty[s]  (each CTA) one commit from the leader's MMA thread each;
//   tfull[a]  (each CTA) one commit from the leader's MMA thread each;
//   tempty[a] (leading CTA) one arrival per epilogue warp of both CTAs.
// No load uses multicast.
struct PairCfg {
  static constexpr int BN = 256;
  static constexpr int STAGES = 6;
  static constexpr int A_BYTES = kBM * kBK * 2;         // 128 rows of X
  static constexpr int B_BYTES = 128 * kBK * 2;         // 128 rows of W (half the tile's N)
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // per CTA
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int OUT_STAGE_BYTES = kEpiWarps * 2 * 32 * 64;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + OUT_STAGE_BYTES + 1024 + 256;
};

template <int EPI, int ACT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_bf16_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const __grid_constant__ CUtensorMap tmO, int M, int N, int K, EpiArgs e, int* status) {
  using C = PairCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint8_t* sOut = sB + C::STAGES * C::B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + C::OUT_STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);

  pdl_trigger();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = leading CTA of the pair
  const uint32_t peer = rank ^ 1u;
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  const int m_tiles = (M + 2 * kBM - 1) / (2 * kBM);
  const int n_tiles = (N + C::BN - 1) / C::BN;
  const int num_tiles = m_tiles * n_tiles;
  const int k_blocks = (K + kBK - 1) / kBK;
  const int splits = e.splits > 1 ? e.splits : 1;
  const int num_units = num_tiles * splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * kEpiWarps);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int u = pair; u < num_units && ok; u += n_pairs) {
        const Unit w = unit_of(u, splits, k_blocks);
        const int mb = w.tile / n_tiles, nb = w.tile - (w.tile / n_tiles) * n_tiles;
        const int a_row = mb * 2 * kBM + static_cast<int>(rank) * kBM;
        const int b_row = nb * C::BN + static_cast<int>(rank) * 128;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, status, INL_DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          tma_load_2d_pair(sA + stage * C::A_BYTES, &tmA, bar, kb * kBK, a_row);
          tma_load_2d_pair(sB + stage * C::B_BYTES, &tmB, bar, kb * kBK, b_row);
          ++issued;
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: every stage this CTA filled must have been consumed (its empty
      // barrier released by the leader's commit) before the CTA can go away,
      // since the leader's MMAs read this CTA's shared memory.
      const long long first = issued > C::STAGES ? issued - C::STAGES : 0;
      for (long long f = first; f < issued; ++f) {
        const int s = static_cast<int>(f % C::STAGES);
        const uint32_t ph = static_cast<uint32_t>((f / C::STAGES) & 1);
        if (!mbar_wait(&empty[s], ph, status, INL_DEV_TIMEOUT_DRAIN)) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(2 * kBM, C::BN);
      const uint64_t a_desc0 = sw128_kmajor_desc(smem_u32(sA)), b_desc0 = sw128_kmajor_desc(smem_u32(sB));
      const uint32_t empty_peer0 = mapa_shared(smem_u32(&empty[0]), peer);
      const uint32_t tfull_peer0 = mapa_shared(smem_u32(&tfull[0]), peer);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int u = pair; u < num_units && ok; u += n_pairs) {
        const Unit w = unit_of(u, splits, k_blocks);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, status, INL_DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * C::BN);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, status, INL_DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // Descriptors differ from the ring's base descriptors only in the
          // start-address field (address >> 4, 14 bits; shared memory < 256 KB).
          const uint64_t a_desc = a_desc0 + static_cast<uint64_t>((stage * C::A_BYTES) >> 4);
          const uint64_t b_desc = b_desc0 + static_cast<uint64_t>((stage * C::B_BYTES) >> 4);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            umma_bf16_pair(d_tmem, a_desc + static_cast<uint64_t>(kk * 2), b_desc + static_cast<uint64_t>(kk * 2), idesc,
                           (kb != w.kb0 || kk != 0) ? 1u : 0u);
          }
          umma_commit_pair(smem_u32(&empty[stage]));
          umma_commit_pair(empty_peer0 + static_cast<uint32_t>(stage * sizeof(uint64_t)));
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(&tfull[acc]));
        umma_commit_pair(tfull_peer0 + static_cast<uint32_t>(acc * sizeof(uint64_t)));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // Epilogue warps 2..9 of both CTAs, on this CTA's 128 rows of the tile.
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    OutStage st{&tmO, sOut + (warp - 2) * 2 * kStageChunkBytes, 0};
    const uint32_t tempty_lead0 = mapa_shared(smem_u32(&tempty[0]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = pair; u < num_units; u += n_pairs) {
      const Unit w = unit_of(u, splits, k_blocks);
      const int mb = w.tile / n_tiles, nb = w.tile - (w.tile / n_tiles) * n_tiles;
      if (!mbar_wait_warp(&tfull[acc], acc_phase, status, INL_DEV_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * C::BN);
      const int row = mb * 2 * kBM + static_cast<int>(rank) * kBM + quad * 32 + lane;
      epilogue_tile<C::BN, EPI, ACT>(t_row, row, nb * C::BN, half, e, st, lane, w.slice * e.split_stride);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_lead0 + static_cast<uint32_t>(acc * sizeof(uint64_t)));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (lane == 0) bulk_wait_group<0>();
  }

  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its partner may still touch its shared memory / TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

bool make_kmajor_map(CUtensorMap* map, const void* base, long long rows, long long cols, long long ld,
                     int box_rows) {
  return make_tma_2d_bf16(map, base, rows, cols, ld, box_rows, kBK);
}

int num_sms() {
  // per device: a process may drive GPUs of different SM counts
  static std::atomic<int> count[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = count[dev].load(std::memory_order_relaxed);
  if (!n) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    count[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

template <int BN, int EPI, int ACT>
cudaError_t launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, int M, int N, int K,
                        const EpiArgs& e,
                        int* status, int max_ctas, cudaStream_t stream) {
  using C = GemmCfg<BN>;
  auto kern = gemm_bf16_tn_kernel<BN, EPI, ACT>;
  static std::atomic<unsigned long long> attr_set{0};  // per instantiation, one bit per device
  cudaError_t aerr = set_smem_limit_once(kern, C::SMEM_BYTES, attr_set);
  if (aerr != cudaSuccess) return aerr;
  const int tiles = ((M + kBM - 1) / kBM) * ((N + BN - 1) / BN) * (e.splits > 1 ? e.splits : 1);
  int grid = num_sms();
  if (max_ctas > 0 && max_ctas < grid) grid = max_ctas;
  if (tiles < grid) grid = tiles;
  cudaError_t err = launch_pdl(kern, dim3(grid), dim3(kThreads), C::SMEM_BYTES, stream, ta, tb, to, M, N, K, e, status);
  return err != cudaSuccess ? err : cudaGetLastError();
}

template <int EPI, int ACT>
cudaError_t launch_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, int M, int N, int K,
                             const EpiArgs& e, int* status, int max_ctas, cudaStream_t stream) {
  using C = PairCfg;
  auto kern = gemm_bf16_pair_kernel<EPI, ACT>;
  static std::atomic<unsigned long long> attr_set{0};  // per instantiation, one bit per device
  cudaError_t aerr = set_smem_limit_once(kern, C::SMEM_BYTES, attr_set);
  if (aerr != cudaSuccess) return aerr;
  const int tiles = ((M + 2 * kBM - 1) / (2 * kBM)) * ((N + C::BN - 1) / C::BN) * (e.splits > 1 ? e.splits : 1);
  int pairs = num_sms() / 2;
  if (max_ctas > 0 && max_ctas / 2 < pairs) pairs = max_ctas / 2 > 0 ? max_ctas / 2 : 1;
  if (tiles < pairs) pairs = tiles;
  cudaError_t err =
      launch_pdl(kern, dim3(2 * pairs), dim3(kThreads), C::SMEM_BYTES, stream, ta, tb, to, M, N, K, e, status);
  return err != cudaSuccess ? err : cudaGetLastError();
}

template <int EPI>
cudaError_t dispatch_act_pair(int act, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, int M,
                              int N, int K, const EpiArgs& e, int* status, int max_ctas, cudaStream_t s) {
  switch (act) {
    case INL_ACT_SILU: return launch_gemm_pair<EPI, INL_ACT_SILU>(ta, tb, to, M, N, K, e, status, max_ctas, s);
    case INL_ACT_GELU_ERF: return launch_gemm_pair<EPI, INL_ACT_GELU_ERF>(ta, tb, to, M, N, K, e, status, max_ctas, s);
    default: return launch_gemm_pair<EPI, INL_ACT_GELU_TANH>(ta, tb, to, M, N, K, e, status, max_ctas, s);
  }
}

template <int BN, int EPI>
cudaError_t dispatch_act(int act, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, int M, int N,
                         int K,
                         const EpiArgs& e, int* status, int max_ctas, cudaStream_t s) {
  switch (act) {
    case INL_ACT_SILU: return launch_gemm<BN, EPI, INL_ACT_SILU>(ta, tb, to, M, N, K, e, status, max_ctas, s);
    case INL_ACT_GELU_ERF: return launch_gemm<BN, EPI, INL_ACT_GELU_ERF>(ta, tb, to, M, N, K, e, status, max_ctas, s);
    default: return launch_gemm<BN, EPI, INL_ACT_GELU_TANH>(ta, tb, to, M, N, K, e, status, max_ctas, s);
  }
}

}  // namespace

// Row-major [rows, cols] bf16 with row stride `ld` elements; box [box_rows, box_cols]
// (box_cols * 2 = 128 bytes for the 128-byte swizzle), out-of-range reads fill zeros.
bool make_tma_2d_bf16_swizzled(CUtensorMap* map, const void* base, long long rows, long long cols, long long ld,
                               int box_rows, int box_cols, int swizzle_bytes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                      : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tma_2d_bf16(CUtensorMap* map, const void* base, long long rows, long long cols, long long ld,
                      int box_rows, int box_cols) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int num_sms_cached() { return num_sms(); }

int gemm_bf16_tn(const GemmArgs& g, cudaStream_t stream) {
  if (g.M <= 0 || g.N <= 0) return 0;
  if (g.K <= 0 || (g.K % 8) != 0 || (g.lda % 8) != 0 || (g.ldw % 8) != 0) return -1;
  if ((reinterpret_cast<uintptr_t>(g.A) & 15) || (reinterpret_cast<uintptr_t>(g.W) & 15)) return -1;
  if (g.epi != INL_EPI_SEGMAX && ((reinterpret_cast<uintptr_t>(g.out) & 15) || (g.ldo % 8) != 0)) return -1;
  if (g.epi == INL_EPI_RESID_BF16 && ((reinterpret_cast<uintptr_t>(g.resid) & 15) || (g.ldr % 8) != 0)) return -1;
  if (g.epi == INL_EPI_RESID_F32 && (!g.resid || (reinterpret_cast<uintptr_t>(g.resid) & 15) || (g.ldr % 4) != 0))
    return -1;
  int bn = (g.N <= 128 || (g.N % 256) != 0) ? 128 : 256;
  if (g.epi == INL_EPI_GATED_BF16 || g.epi == INL_EPI_GATED_F32) {
    // Gate/up interleaved in blocks of bn/2 rows; the caller picks the block.
    bn = g.gate_block * 2;
    if ((bn != 128 && bn != 256) || (g.N % bn) != 0) return -1;
  }
  if (g.epi == INL_EPI_QKV) {
    // Each epilogue warp owns 128 columns = whole heads of width 64 or 128.
    bn = 256;
    if ((g.d != 64 && g.d != 128) || (g.N % 256) != 0 || g.N != (g.hq + 2 * g.hkv) * g.d || !g.pos || !g.cos ||
        g.max_pos <= 0 || !g.qn || !g.kn || (reinterpret_cast<uintptr_t>(g.cos) & 15) ||
        (reinterpret_cast<uintptr_t>(g.qn) & 15) || (reinterpret_cast<uintptr_t>(g.kn) & 15))
      return -1;
  }
  if (g.force_bn == 128 || g.force_bn == 256) {
    if ((g.epi == INL_EPI_GATED_BF16 || g.epi == INL_EPI_GATED_F32 || g.epi == INL_EPI_QKV) && g.force_bn != bn)
      return -1;
    bn = g.force_bn;
  }
  if (g.ss_in && (g.ss_in_parts <= 0 || g.ss_dim <= 0)) return -1;
  const int k_blocks = (g.K + kBK - 1) / kBK;
  if (g.splits > 1) {
    // every slice must hold at least one K block
    const int per = (k_blocks + g.splits - 1) / g.splits;
    if (g.epi != INL_EPI_F32 || (g.splits - 1) * per >= k_blocks) return -1;
  }
  if (g.epi == INL_EPI_SEGMAX) {
    if (!g.seg || !g.pooled || g.ldp < g.M) return -1;
    bn = 256;
  }
  // CTA pairs (cta_group::2) take 256-wide tiles of the plain, residual,
  // gated and f32 epilogues; each CTA of a pair loads 128 rows of W, so a K
  // step moves 32 KB per CTA instead of 48 KB (the 3xBF16 f32 products: 3%
  // faster on config 1). The QKV epilogue (q/k norm + RoPE) measured faster on
  // single CTAs, and the segment-max decoder the same on both, so those stay
  // on single CTAs.
  const bool pair = g.cta_pair && bn == 256 &&
                    (g.epi == INL_EPI_BF16 || g.epi == INL_EPI_RESID_BF16 || g.epi == INL_EPI_GATED_BF16 ||
                     g.epi == INL_EPI_F32 || g.epi == INL_EPI_RESID_F32 || g.epi == INL_EPI_GATED_F32);
  CUtensorMap ta, tb, to;
  if (!make_kmajor_map(&ta, g.A, g.M, g.K, g.lda, kBM)) return -2;
  if (!make_kmajor_map(&tb, g.W, g.N, g.K, g.ldw, pair ? 128 : bn)) return -2;
  // bf16 outputs leave through the epilogue warps' staging: boxes of 32 rows x 32
  // columns, 64-byte swizzle; the gated epilogue writes N / 2 columns.
  std::memset(&to, 0, sizeof(to));
  if (g.epi == INL_EPI_BF16 || g.epi == INL_EPI_RESID_BF16 || g.epi == INL_EPI_GATED_BF16 || g.epi == INL_EPI_QKV) {
    const int out_cols = g.epi == INL_EPI_GATED_BF16 ? g.N / 2 : g.N;
    if (!make_tma_2d_bf16_swizzled(&to, g.out, g.M, out_cols, g.ldo, 32, 32, 64)) return -2;
  }
  EpiArgs e{g.out, g.ldo, g.resid, g.ldr, g.ss_in, g.ss_in_parts, g.ss_dim, g.ss_eps, g.ss_out,
            (g.N + INL_SS_COLS - 1) / INL_SS_COLS, g.qn, g.kn, g.pos, g.cos, g.sin, g.hq, g.hkv, g.d, g.max_pos,
            g.qk_eps, g.status, g.M, g.N, g.seg, g.pooled, g.ldp};
  e.splits = g.splits > 1 ? g.splits : 1;
  e.split_stride = static_cast<long long>(g.M) * g.ldo;
  cudaError_t err;
  if (pair) {
    switch (g.epi) {
      case INL_EPI_BF16: err = launch_gemm_pair<INL_EPI_BF16, 0>(ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
      case INL_EPI_RESID_BF16: err = launch_gemm_pair<INL_EPI_RESID_BF16, 0>(ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
      case INL_EPI_F32: err = launch_gemm_pair<INL_EPI_F32, 0>(ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
      case INL_EPI_RESID_F32: err = launch_gemm_pair<INL_EPI_RESID_F32, 0>(ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
      case INL_EPI_GATED_F32: err = dispatch_act_pair<INL_EPI_GATED_F32>(g.act, ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
      default: err = dispatch_act_pair<INL_EPI_GATED_BF16>(g.act, ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
    }
  } else if (bn == 256) {
    switch (g.epi) {
      case INL_EPI_BF16: err = launch_gemm<256, INL_EPI_BF16, 0>(ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
      case INL_EPI_RESID_BF16: err = launch_gemm<256, INL_EPI_RESID_BF16, 0>(ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
      case INL_EPI_F32: err = launch_gemm<256, INL_EPI_F32, 0>(ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
      case INL_EPI_RESID_F32: err = launch_gemm<256, INL_EPI_RESID_F32, 0>(ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
      case INL_EPI_GATED_F32: err = dispatch_act<256, INL_EPI_GATED_F32>(g.act, ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
      case INL_EPI_GATED_BF16: err = dispatch_act<256, INL_EPI_GATED_BF16>(g.act, ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
      case INL_EPI_QKV: err = launch_gemm<256, INL_EPI_QKV, 0>(ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
      case INL_EPI_SEGMAX: err = launch_gemm<256, INL_EPI_SEGMAX, 0>(ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
      default: return -1;
    }
  } else {
    switch (g.epi) {
      case INL_EPI_BF16: err = launch_gemm<128, INL_EPI_BF16, 0>(ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
      case INL_EPI_RESID_BF16: err = launch_gemm<128, INL_EPI_RESID_BF16, 0>(ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
      case INL_EPI_F32: err = launch_gemm<128, INL_EPI_F32, 0>(ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
      case INL_EPI_RESID_F32: err = launch_gemm<128, INL_EPI_RESID_F32, 0>(ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
      case INL_EPI_GATED_F32: err = dispatch_act<128, INL_EPI_GATED_F32>(g.act, ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
      case INL_EPI_GATED_BF16: err = dispatch_act<128, INL_EPI_GATED_BF16>(g.act, ta, tb, to, g.M, g.N, g.K, e, g.status, g.max_ctas, stream); break;
      default: return -1;
    }
  }
  return err == cudaSuccess ? 0 : -3;
}

}  // namespace inl
