// Flash attention on the sm_100a tensor cores for packed variable-length
// texts (bf16, head_dim 64, 128 or 256): causal, bidirectional and
// sliding-window masks computed from positions, grouped-query heads by index.
//
// Persistent: one CTA per SM walks the tiles blockIdx.x, blockIdx.x +
// gridDim.x, ... of the list (work item, query heads), work items heaviest
// first and the heads of one item adjacent (their K / V rows meet in L2).
// For head_dim 64 / 128 the CTA runs two slots side by side; each slot owns a
// Q and a P buffer in shared memory and, in TMEM, a score buffer S (128
// columns) and an output accumulator O (D columns): 2 x 256 of the 512
// columns. When the GQA group size is even, a tile is 128 queries of one text
// and two query heads of one K / V head, one per slot, and each K / V tile is
// loaded once for both. Otherwise a tile is 128 queries and one head, the
// CTA's even tiles run in slot 0 and its odd tiles in slot 1. For head_dim
// 256 the CTA runs one slot (S 128 + O 256 columns). Threads:
//   warp 0     TMA producer: each slot's Q tile, and K / V tiles of 128 keys
//              into one ring, in exactly the order the MMA warp consumes them
//              (so the ring can neither deadlock nor reorder);
//   warp 1     TMEM allocation and tcgen05.mma issue, in units
//              "S = Q K(j)^T; O += P(j-1) V(j-1)": one unit serves both slots
//              of a GQA pair, or the units alternate between the slots. S(j)
//              only needs the softmax warps to have read S(j-1) out of TMEM,
//              so it runs while they still compute P(j-1), and the next
//              block's scores are ready when they finish;
//   8 softmax warps per slot (warps 2-9 slot 0, 10-17 slot 1): two threads
//              per query row. A warp holds 16 rows of one TMEM lane quadrant
//              (tcgen05.ld 16x32bx2): lane t reads keys [0, 64) of row t and
//              lane t + 16 keys [64, 128) of the same row, so a row's max and
//              sum combine with one shuffle, and four softmax warps share each
//              SM sub-partition. Each thread masks its scores, keeps the
//              row's running max m and its share of the sum l, and writes P =
//              exp2(s - m) as bf16 into shared memory in the K-major
//              128-byte-swizzle layout the MMA reads. m is only raised when
//              the block max exceeds it by more than 2^8, and then O is
//              rescaled in TMEM. The exp2 run on the special-function
//              unit. At the end of a tile, O / l goes as bf16 through the slot's P buffer to TMA
//              tensor stores of the warp's 16 rows (whole-row stores for a
//              warp that crosses the end of the text); for head_dim 256 each
//              thread stores its 128 columns straight to the output row.
// Per slot, barriers order the shared buffers: s_free (the scores were read,
// S may be overwritten), pv_done (PV(j-1) is complete: P's buffer may be
// rewritten and O rescaled; the softmax warps compute exp2 into registers
// before they wait on it), p_full, o_full. The first PV of a slot's next tile
// (which overwrites O) is issued only after that slot's softmax warps, having
// read O for the epilogue, delivered the next P.
// Every mbarrier wait is bounded (status word + early exit, TMEM freed).
#include "common.cuh"
#include "kernels.h"

namespace inl {

namespace {

constexpr int kTQ = 128;   // queries per tile (UMMA M)
constexpr int kTK = 128;   // keys per block (UMMA N of S, K of PV)
constexpr int kBox = 16384;  // one TMA box: 128 rows x 128 bytes
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only when the max grows 256x

// head_dim 64 / 128: two slots (S 128 + O D TMEM columns each); head_dim
// 256: one slot (S 128 + O 256 columns), whose Q and K / V tiles are twice
// as large.
template <int D>
struct FaCfg {
  static constexpr int NSLOT = D == 256 ? 1 : 2;
  static constexpr int THREADS = 64 + 256 * NSLOT;  // TMA warp, MMA warp, 8 softmax warps per slot
  static constexpr int QB = D / 64;              // 64-column boxes per head row
  static constexpr int TILE_BYTES = QB * kBox;   // one Q, K or V tile of 128 rows
  static constexpr int P_BYTES = 2 * kBox;       // 128 keys = two 64-key boxes
  static constexpr int NS = D == 64 ? 8 : (D == 128 ? 3 : 2);  // K / V ring slots
  static constexpr int SMEM = NSLOT * TILE_BYTES + NSLOT * P_BYTES + NS * TILE_BYTES + 1024 + 512;
  static constexpr int TMEM_COLS = 512;
  static constexpr int SLOT_COLS = D == 256 ? 512 : 256;  // S at +0, O at +128
  static_assert(SMEM <= 232448, "shared memory of one CTA");
};

struct FaParams {
  const int* cu;
  const int2* work;
  __nv_bfloat16* out;
  long long ldo;
  int hq, hkv, n_tiles;
  int hpt;    // query heads per tile: 2 = the two heads of a GQA pair share every K / V load
  int tstep;  // tile ordinal step of one sequence: 2 = slots take alternate tiles, 1 = paired slots
  float scale_log2;
  int causal, window;
  int* status;
};

struct TileInfo {
  int s0, L, q0, head, kvh, kb_lo, n_kv;
};

// Work entry (text, query block) of the CTA's tile of ordinal k; text -1
// past the end of the list.
__device__ __forceinline__ int2 tile_work(const FaParams& p, int k) {
  const int t = static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x);
  if (t >= p.n_tiles) return make_int2(-1, 0);
  return p.work[t / (p.hq / p.hpt)];
}

// Tile of ordinal k from its work entry and its text's offsets [s0, e).
__device__ __forceinline__ void make_tile(const FaParams& p, int k, int2 wk, int s0, int e, TileInfo& ti) {
  const int t = static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x);
  const int per_item = p.hq / p.hpt;
  const int item = t / per_item;
  ti.head = (t - item * per_item) * p.hpt;
  ti.kvh = ti.head / (p.hq / p.hkv);
  ti.s0 = s0;
  ti.L = e - s0;
  ti.q0 = wk.y * kTQ;
  int k_lo = 0, k_hi = ti.L;
  if (p.causal) k_hi = min(ti.L, ti.q0 + kTQ);
  if (p.window >= 0) {
    k_lo = max(0, ti.q0 - p.window);
    k_hi = min(k_hi, ti.q0 + kTQ + p.window);
  }
  ti.kb_lo = k_lo / kTK;
  ti.n_kv = ti.q0 < ti.L ? (k_hi + kTK - 1) / kTK - ti.kb_lo : 0;
}

// The CTA's tiles of one sequence (ordinals first, first + tstep, ...),
// skipping tiles without key blocks, read ahead: a tile's work entry and its
// text's offsets are dependent global loads, so when a tile becomes current
// the offsets of the next tile and the work entry of the one after it are
// requested; both arrive while the current tile's blocks run, and moving on
// needs no load.
struct TilePipe {
  TileInfo cur;
  int k;        // ordinal of cur
  bool has;     // cur is a tile (false past the end)
  int2 wk1;     // ordinal k + tstep: work entry ...
  int s1, e1;   // ... and its text's offsets
  int2 wk2;     // ordinal k + 2 tstep: work entry

  __device__ __forceinline__ void init(const FaParams& p, int first) {
    k = first - p.tstep;
    wk1 = tile_work(p, first);
    s1 = wk1.x >= 0 ? p.cu[wk1.x] : 0;
    e1 = wk1.x >= 0 ? p.cu[wk1.x + 1] : 0;
    wk2 = tile_work(p, first + p.tstep);
    advance(p);
  }
  __device__ __forceinline__ void advance(const FaParams& p) {
    for (;;) {
      k += p.tstep;
      if (wk1.x < 0) {
        has = false;
        return;
      }
      make_tile(p, k, wk1, s1, e1, cur);
      wk1 = wk2;
      s1 = wk1.x >= 0 ? p.cu[wk1.x] : 0;
      e1 = wk1.x >= 0 ? p.cu[wk1.x + 1] : 0;
      wk2 = tile_work(p, k + 2 * p.tstep);
      if (cur.n_kv > 0) {
        has = true;
        return;
      }
    }
  }
};

// The sequence of MMA units of one slot (or of both slots, paired), walked
// identically by the producer and the MMA warp: unit u issues S op u (if any)
// and PV of S op u-1 (if any); S ops run over the tiles and their key blocks
// in order.
struct SlotSeq {
  TilePipe tp;       // the current tile (tp.cur) and the tiles read ahead
  int j;             // next key block of the current tile
  int tiles, ops;    // tiles whose Q was taken, S ops done
  int pv_row, pv_kvh;
  bool pv, pv_first, pv_last;

  __device__ __forceinline__ void init(const FaParams& p, int first) {
    j = 0;
    tiles = ops = 0;
    pv = false;
    tp.init(p, first);
  }
  __device__ __forceinline__ const TileInfo& ti() const { return tp.cur; }
  __device__ __forceinline__ bool has() const { return tp.has; }
  __device__ __forceinline__ bool live() const { return tp.has || pv; }
  __device__ __forceinline__ int row() const { return tp.cur.s0 + (tp.cur.kb_lo + j) * kTK; }
  // The S op of this unit becomes the next unit's PV.
  __device__ __forceinline__ void advance(const FaParams& p) {
    if (!tp.has) {
      pv = false;
      return;
    }
    pv = true;
    pv_row = row();
    pv_kvh = tp.cur.kvh;
    pv_first = j == 0;
    pv_last = j == tp.cur.n_kv - 1;
    ++ops;
    if (++j == tp.cur.n_kv) {
      j = 0;
      tp.advance(p);
    }
  }
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

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// (d0, d1) = (a0, a1) * (b, b) + (c, c) as one packed f32x2 FMA.
__device__ __forceinline__ void fma2_bcast(float& d0, float& d1, float a0, float a1, float b, float c) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %4};\n\t"
      "mov.b64 rc, {%5, %5};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b), "f"(c));
}

// (s0, s1) += (a0, a1) as one packed f32x2 add.
__device__ __forceinline__ void add2(float& s0, float& s1, float a0, float a1) {
  asm("{\n\t.reg .b64 ra, rs;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rs, {%0, %1};\n\t"
      "add.rn.f32x2 rs, rs, ra;\n\t"
      "mov.b64 {%0, %1}, rs;\n\t}"
      : "+f"(s0), "+f"(s1)
      : "f"(a0), "f"(a1));
}

// bf16x2 {lo, hi} with round-to-nearest-even, one instruction.
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// Columns c of a 128-key block outside [lo, hi) become -inf (lo, hi per row).
template <int N>
__device__ __forceinline__ void mask_range(uint32_t (&sv)[N], int c0, int lo, int hi) {
#pragma unroll
  for (int c = 0; c < N; ++c)
    if (c0 + c < lo || c0 + c >= hi) sv[c] = __float_as_uint(-INFINITY);
}

// PAIR: the two slots take the two query heads of one GQA pair for the same
// 128 queries (one tile), so every K / V tile is loaded once for both; the
// producer and the MMA warp walk one sequence and issue each unit's S and PV
// for both slots. Otherwise the slots take alternate tiles, each with its own
// sequence and K / V loads.
// Warps are dealt round-robin to the SM's four sub-partitions, each with a
// quarter of the register file: 18 warps put 5 on two of them (96 registers
// a thread), 10 warps put 3 on two (168); the launch bounds give ptxas that.
template <int D, bool PAIR>
__global__ void __launch_bounds__(FaCfg<D>::THREADS, 1)
    fa_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                    FaParams p) {
  using C = FaCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                          // NSLOT slots
  uint8_t* sP = sQ + C::NSLOT * C::TILE_BYTES;  // NSLOT slots
  uint8_t* ring = sP + C::NSLOT * C::P_BYTES;  // NS K / V tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + C::NS * C::TILE_BYTES);
  uint64_t* q_full = bars;          // [2]
  uint64_t* q_empty = bars + 2;     // [2]
  uint64_t* s_full = bars + 4;      // [2]
  uint64_t* p_full = bars + 6;      // [2]
  uint64_t* o_full = bars + 8;      // [2]
  uint64_t* s_free = bars + 10;     // [2]
  uint64_t* pv_done = bars + 12;    // [2]
  uint64_t* mma_done = bars + 14;
  uint64_t* ring_full = bars + 15;  // [NS]
  uint64_t* ring_empty = ring_full + C::NS;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(ring_empty + C::NS);

  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 8);  // one arrival per softmax warp of the slot
      mbar_init(&o_full[i], 1);
      mbar_init(&s_free[i], 8);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(mma_done, 1);
    for (int i = 0; i < C::NS; ++i) {
      mbar_init(&ring_full[i], 1);
      mbar_init(&ring_empty[i], 1);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  pdl_wait();  // q / k / v of the previous kernel are complete
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      constexpr int NH = PAIR ? 2 : 1;  // slots served by one unit
      SlotSeq sq0, sq1;
      sq0.init(p, 0);
      if (C::NSLOT == 2) sq1.init(p, 1);
      int g = 0;  // ring loads issued
      auto ring_load = [&](const CUtensorMap* map, int row, int kvh) -> bool {
        const int r = g % C::NS;
        if (!wait_or_flag(&ring_empty[r], ((g / C::NS) & 1) ^ 1, p.status, INL_DEV_TIMEOUT_PRODUCER, ok))
          return false;
        mbar_expect_tx(&ring_full[r], C::TILE_BYTES);
        for (int b = 0; b < C::QB; ++b)
          tma_load_2d(ring + r * C::TILE_BYTES + b * kBox, map, &ring_full[r], kvh * D + b * 64, row);
        ++g;
        return true;
      };
      auto unit = [&](SlotSeq& q, const int s) {
        if (!q.live() || !ok) return;
        if (q.has()) {
          if (q.j == 0) {
            if (q.tiles > 0 &&
                !wait_or_flag(&q_empty[s], (q.tiles - 1) & 1, p.status, INL_DEV_TIMEOUT_PRODUCER, ok))
              return;
            mbar_expect_tx(&q_full[s], NH * C::TILE_BYTES);
            for (int h = 0; h < NH; ++h)
              for (int b = 0; b < C::QB; ++b)
                tma_load_2d(sQ + (s + h) * C::TILE_BYTES + b * kBox, &tmQ, &q_full[s], (q.ti().head + h) * D + b * 64,
                            q.ti().s0 + q.ti().q0);
            ++q.tiles;
          }
          if (!ring_load(&tmK, q.row(), q.ti().kvh)) return;
        }
        if (q.pv && !ring_load(&tmV, q.pv_row, q.pv_kvh)) return;
        q.advance(p);
      };
      if constexpr (PAIR || C::NSLOT == 1) {
        while (ok && sq0.live()) unit(sq0, 0);
      } else {
        while (ok && (sq0.live() || sq1.live())) {
          unit(sq0, 0);
          unit(sq1, 1);
        }
      }
      // Drain: every copy still in flight must land before the CTA exits.
      bool dok = true;
      if (sq0.tiles > 0) wait_or_flag(&q_full[0], (sq0.tiles - 1) & 1, p.status, INL_DEV_TIMEOUT_DRAIN, dok);
      if (!PAIR && C::NSLOT == 2 && sq1.tiles > 0)
        wait_or_flag(&q_full[1], (sq1.tiles - 1) & 1, p.status, INL_DEV_TIMEOUT_DRAIN, dok);
      for (int i = max(0, g - C::NS); i < g; ++i)
        wait_or_flag(&ring_full[i % C::NS], (i / C::NS) & 1, p.status, INL_DEV_TIMEOUT_DRAIN, dok);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(kTQ, kTK, 0);
      constexpr uint32_t idesc_o = umma_idesc_bf16(kTQ, D, 1);
      constexpr int NH = PAIR ? 2 : 1;  // slots served by one unit
      SlotSeq sq0, sq1;
      sq0.init(p, 0);
      if (C::NSLOT == 2) sq1.init(p, 1);
      int g = 0;  // ring tiles consumed
      auto unit = [&](SlotSeq& q, const int s) {
        if (!q.live() || !ok) return;
        if (q.has()) {
          if (q.j == 0) {
            if (!wait_or_flag(&q_full[s], q.tiles & 1, p.status, INL_DEV_TIMEOUT_MMA, ok)) return;
            ++q.tiles;
          }
          const int r = g % C::NS;
          if (!wait_or_flag(&ring_full[r], (g / C::NS) & 1, p.status, INL_DEV_TIMEOUT_MMA, ok)) return;
          const uint32_t k_addr = smem_u32(ring + r * C::TILE_BYTES);
          for (int h = 0; h < NH; ++h) {
            const int sh = s + h;
            // S is rewritten once the softmax warps have read the previous scores.
            if (q.ops > 0 && !wait_or_flag(&s_free[sh], (q.ops - 1) & 1, p.status, INL_DEV_TIMEOUT_MMA, ok)) return;
            tc_fence_after();
            const uint32_t t_s = tmem + sh * C::SLOT_COLS;
            const uint32_t q_addr = smem_u32(sQ + sh * C::TILE_BYTES);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = (kk >> 2) * kBox + (kk & 3) * 32;
              umma_bf16(t_s, sw128_kmajor_desc(q_addr + off), sw128_kmajor_desc(k_addr + off), idesc_s,
                        kk > 0 ? 1u : 0u);
            }
            umma_commit(&s_full[sh]);
          }
          umma_commit(&ring_empty[r]);
          ++g;
          if (q.j == q.ti().n_kv - 1) umma_commit(&q_empty[s]);
        }
        if (q.pv) {
          const int r = g % C::NS;
          if (!wait_or_flag(&ring_full[r], (g / C::NS) & 1, p.status, INL_DEV_TIMEOUT_MMA, ok)) return;
          const uint32_t v_addr = smem_u32(ring + r * C::TILE_BYTES);
          for (int h = 0; h < NH; ++h) {
            const int sh = s + h;
            if (!wait_or_flag(&p_full[sh], (q.ops - 1) & 1, p.status, INL_DEV_TIMEOUT_MMA, ok)) return;
            tc_fence_after();
            const uint32_t t_o = tmem + sh * C::SLOT_COLS + kTK;
            const uint32_t p_addr = smem_u32(sP + sh * C::P_BYTES);
#pragma unroll
            for (int kk = 0; kk < kTK / 16; ++kk) {
              const uint32_t a_off = (kk >> 2) * kBox + (kk & 3) * 32;  // P: K-major, 64 keys per box
              const uint32_t b_off = kk * 16 * 128;                      // V: 16 key rows per step
              umma_bf16(t_o, sw128_kmajor_desc(p_addr + a_off), sw128_mnmajor_desc(v_addr + b_off, kBox),
                        idesc_o, (!q.pv_first || kk > 0) ? 1u : 0u);
            }
            umma_commit(&pv_done[sh]);
            if (q.pv_last) umma_commit(&o_full[sh]);
          }
          umma_commit(&ring_empty[r]);
          ++g;
        }
        q.advance(p);
      };
      if constexpr (PAIR || C::NSLOT == 1) {
        while (ok && sq0.live()) unit(sq0, 0);
      } else {
        while (ok && (sq0.live() || sq1.live())) {
          unit(sq0, 0);
          unit(sq1, 1);
        }
      }
      // Every MMA must be complete before TMEM is released.
      umma_commit(mma_done);
      bool dok = true;
      wait_or_flag(mma_done, 0, p.status, INL_DEV_TIMEOUT_DRAIN, dok);
    }
  } else {
    // Softmax: warps 2..17, eight per slot. Warp w serves slot (w - 2) / 8 and
    // the 16 query rows rw0 .. rw0 + 15 of the slot's tile, rw0 = quad * 32 +
    // sub * 16, where quad = w % 4 is its TMEM lane quadrant and sub picks the
    // quadrant's half. Lanes t and t + 16 hold the same row (tcgen05.ld
    // 16x32bx2): keys [0, 64) and [64, 128) of every block, O columns [0, D/2)
    // and [D/2, D). A row's max and sum combine with one shuffle.
    const int idx = warp - 2;
    const int s = idx >> 3;
    const int sub = (idx >> 2) & 1;
    const int quad = warp & 3;
    const int half = lane >> 4;
    const int rw0 = quad * 32 + sub * 16;
    const int r = rw0 + (lane & 15);
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(rw0) << 16);
    const uint32_t t_s = lane_base + s * C::SLOT_COLS, t_o = t_s + kTK;
    uint8_t* prow = sP + s * C::P_BYTES + half * kBox + r * 128;  // this thread's 64 keys of P
    const int sw = r & 7;
    int u = 0, tiles = 0;
    TilePipe tp;
    tp.init(p, PAIR ? 0 : s);
    while (ok && tp.has) {
      TileInfo ti = tp.cur;
      if constexpr (PAIR) ti.head += s;
      const int q = ti.q0 + r;  // text-relative query
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < ti.n_kv; ++j, ++u) {
        if (!wait_warp(&s_full[s], u & 1, p.status, INL_DEV_TIMEOUT_EPILOGUE, ok)) break;
        tc_fence_after();
        const int key0 = (ti.kb_lo + j) * kTK;
        const bool full_block = key0 + kTK <= ti.L && (!p.causal || key0 + kTK - 1 <= ti.q0) &&
                                (p.window < 0 || (ti.q0 + kTQ - 1 - key0 <= p.window &&
                                                  key0 + kTK - 1 - ti.q0 <= p.window));
        // The keys row q may see in this block: columns [lo, hi).
        int lo = 0, hi = kTK;
        if (!full_block) {
          hi = min(kTK, ti.L - key0);
          if (p.causal) hi = min(hi, q - key0 + 1);
          if (p.window >= 0) {
            hi = min(hi, q + p.window - key0 + 1);
            lo = max(0, q - p.window - key0);
          }
        }
        // This thread's 64 scores of the block, read with one wait.
        uint32_t sv[64];
        tmem_ld32_pair<64>(t_s, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        tmem_ld32_pair<64>(t_s + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
        tmem_ld_wait();
        // The scores are in registers: the next S may overwrite the buffer
        // (one arrival per warp, after all its lanes' reads).
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[s]);
        if (!full_block) mask_range<64>(sv, half * 64, lo, hi);
        float mp[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) mp[t] = fmaxf(__uint_as_float(sv[t]), __uint_as_float(sv[4 + t]));
#pragma unroll
        for (int c = 8; c < 64; c += 8) {
#pragma unroll
          for (int t = 0; t < 4; ++t) mp[t] = fmax3(mp[t], __uint_as_float(sv[c + t]), __uint_as_float(sv[c + 4 + t]));
        }
        float mx = fmax3(mp[0], mp[1], fmaxf(mp[2], mp[3]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));  // the row's other 64 keys
        const float m_blk = mx * p.scale_log2;
        // Raise the running max only when the block max exceeds it by > 2^8.
        // Rows that held a finite max need O rescaled; the decision is per
        // row (both lanes of a row take it alike), the TMEM round trip per warp.
        const bool raise = m_blk > m + kRescaleThreshold;
        const bool rescale_row = raise && j > 0 && m != -INFINITY;
        const float alpha = rescale_row ? ex2_approx(m - m_blk) : 1.0f;
        if (raise) {
          l *= alpha;
          m = m_blk;
        }
        const float neg_m = m == -INFINITY ? 0.f : -m;
        // P = exp2(s * scale - m) into packed bf16 registers while PV(j-1)
        // may still be reading P's buffer.
        float rs[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) rs[t] = 0.f;
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 64; c += 8) {
          float x[8];
#pragma unroll
          for (int t = 0; t < 8; t += 2)
            fma2_bcast(x[t], x[t + 1], __uint_as_float(sv[c + t]), __uint_as_float(sv[c + t + 1]), p.scale_log2,
                       neg_m);
          // Every exponential on the special-function unit (moving a
          // quarter or a half of them to a cubic on the FMA pipe measured
          // 2-3% slower here).
#pragma unroll
          for (int t = 0; t < 8; ++t) x[t] = ex2_approx(x[t]);
          add2(rs[0], rs[1], x[0], x[1]);
          add2(rs[2], rs[3], x[2], x[3]);
          add2(rs[0], rs[1], x[4], x[5]);
          add2(rs[2], rs[3], x[6], x[7]);
#pragma unroll
          for (int t = 0; t < 4; ++t) pk[c / 2 + t] = cvt_bf16x2(x[2 * t], x[2 * t + 1]);
        }
        // PV(u-1) must be complete before O is rescaled and P is rewritten.
        if (u > 0) {
          if (!wait_warp(&pv_done[s], (u - 1) & 1, p.status, INL_DEV_TIMEOUT_EPILOGUE, ok)) break;
          tc_fence_after();
        }
        if (__any_sync(0xffffffffu, rescale_row)) {
#pragma unroll 1
          for (int c = 0; c < D / 2; c += 16) {
            uint32_t o[16];
            tmem_ld16_pair<D / 2>(t_o + c, o);
            tmem_ld_wait();
#pragma unroll
            for (int t = 0; t < 16; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * alpha);
            tmem_st16_pair<D / 2>(t_o + c, o);
          }
          tmem_st_wait();
        }
        // The previous tile's output store (this warp's rows) must have read
        // these rows of the buffer.
        if (lane == 0) bulk_wait_group_read<0>();
        __syncwarp();
#pragma unroll
        for (int chunk = 0; chunk < 8; ++chunk)  // 16-byte chunks over this thread's 64 keys
          *reinterpret_cast<uint4*>(prow + ((chunk ^ sw) << 4)) =
              make_uint4(pk[4 * chunk], pk[4 * chunk + 1], pk[4 * chunk + 2], pk[4 * chunk + 3]);
        l += (rs[0] + rs[1]) + (rs[2] + rs[3]);
        fence_proxy_async_smem();  // each lane's P stores, visible to the tensor core
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[s]);
      }
      if (!ok) break;
      // Tile epilogue: wait for the last PV, then O / l -> bf16. The rows go
      // through the slot's P buffer (free: the last PV has read it) in the
      // 128-byte-swizzled layout of P. A warp whose 16 rows all lie inside the
      // text hands them to TMA tensor stores (16 x 64 boxes); a warp that
      // crosses the end of the text writes its rows back with whole-row
      // stores and skips the rows past it.
      if (!wait_warp(&o_full[s], tiles & 1, p.status, INL_DEV_TIMEOUT_EPILOGUE, ok)) break;
      tc_fence_after();
      const float l_row = l + __shfl_xor_sync(0xffffffffu, l, 16);
      const float inv = l_row > 0.f ? 1.0f / l_row : 0.f;
      constexpr int HC = D / 2;  // O columns of this thread
      if constexpr (D == 256) {
        // A 512-byte output row does not fit the P buffer's staging: each
        // thread writes its 128 columns straight to the output row, 32
        // columns per TMEM read.
        __nv_bfloat16* orow = p.out + static_cast<long long>(ti.s0 + q) * p.ldo + ti.head * D + half * HC;
        const bool row_in = q < ti.L;
#pragma unroll 1
        for (int c = 0; c < HC; c += 32) {
          uint32_t o[32];
          tmem_ld32_pair<HC>(t_o + c, o);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            uint4 w;
            w.x = cvt_bf16x2(__uint_as_float(o[8 * t + 0]) * inv, __uint_as_float(o[8 * t + 1]) * inv);
            w.y = cvt_bf16x2(__uint_as_float(o[8 * t + 2]) * inv, __uint_as_float(o[8 * t + 3]) * inv);
            w.z = cvt_bf16x2(__uint_as_float(o[8 * t + 4]) * inv, __uint_as_float(o[8 * t + 5]) * inv);
            w.w = cvt_bf16x2(__uint_as_float(o[8 * t + 6]) * inv, __uint_as_float(o[8 * t + 7]) * inv);
            if (row_in) *reinterpret_cast<uint4*>(orow + c + 8 * t) = w;
          }
        }
      } else {
        {
          uint32_t o[HC];  // one TMEM read of the half row, one wait
#pragma unroll
          for (int c = 0; c < HC; c += 32) tmem_ld32_pair<HC>(t_o + c, *reinterpret_cast<uint32_t(*)[32]>(&o[c]));
          tmem_ld_wait();
          // staging: column col of row r sits in box col / 64, chunk (col % 64) / 8
          uint8_t* srow = sP + s * C::P_BYTES + r * 128;
#pragma unroll
          for (int t = 0; t < HC / 8; ++t) {
            const int chunk = half * (HC / 8) + t;  // 16-byte chunk of the whole row
            uint4 w;
            w.x = cvt_bf16x2(__uint_as_float(o[8 * t + 0]) * inv, __uint_as_float(o[8 * t + 1]) * inv);
            w.y = cvt_bf16x2(__uint_as_float(o[8 * t + 2]) * inv, __uint_as_float(o[8 * t + 3]) * inv);
            w.z = cvt_bf16x2(__uint_as_float(o[8 * t + 4]) * inv, __uint_as_float(o[8 * t + 5]) * inv);
            w.w = cvt_bf16x2(__uint_as_float(o[8 * t + 6]) * inv, __uint_as_float(o[8 * t + 7]) * inv);
            *reinterpret_cast<uint4*>(srow + (chunk >> 3) * kBox + (((chunk & 7) ^ sw) << 4)) = w;
          }
        }
        const uint8_t* stage = sP + s * C::P_BYTES + rw0 * 128;  // this warp's 16 rows
        if (ti.q0 + rw0 + 16 <= ti.L) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            for (int b = 0; b < D / 64; ++b)
              tma_store_2d(&tmO, stage + b * kBox, ti.head * D + b * 64, ti.s0 + ti.q0 + rw0);
            bulk_commit_group();
          }
        } else {
          __syncwarp();
          constexpr int CPR = D / 8;       // 16-byte chunks per output row
          constexpr int RPI = 32 / CPR;    // rows per store instruction
          const int c = lane % CPR;
          __nv_bfloat16* out_head = p.out + ti.head * D + c * 8;
#pragma unroll 4
          for (int i = 0; i < 16 / RPI; ++i) {
            const int rw = i * RPI + lane / CPR;  // row within the warp's 16
            const int rr = rw0 + rw;              // row within the tile
            const uint4 w = *reinterpret_cast<const uint4*>(stage + (c >> 3) * kBox + rw * 128 +
                                                            (((c & 7) ^ (rr & 7)) << 4));
            if (ti.q0 + rr < ti.L)
              *reinterpret_cast<uint4*>(out_head + static_cast<long long>(ti.s0 + ti.q0 + rr) * p.ldo) = w;
          }
          __syncwarp();  // the next P store rewrites these rows
        }
      }
      tc_fence_before();
      ++tiles;
      tp.advance(p);
    }
    if (lane == 0) bulk_wait_group<0>();  // output stores complete before the CTA exits
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
  CUtensorMap to;  // output rows, 16-row boxes (one warp's rows)
  if (!make_tma_2d_bf16(&to, a.out, total_rows, static_cast<long long>(a.hq) * D, a.ldo, 16, 64)) return -2;
  // Pair the query heads of a GQA group when the group size is even.
  const bool pair = C::NSLOT == 2 && (a.hq / a.hkv) % 2 == 0;
  auto kern = pair ? fa_sm100_kernel<D, true> : fa_sm100_kernel<D, false>;
  static std::atomic<unsigned long long> attr[2] = {};  // per kernel, one bit per device
  if (set_smem_limit_once(kern, C::SMEM, attr[pair]) != cudaSuccess) return -3;
  FaParams p;
  p.cu = a.cu;
  p.work = a.work;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.ldo = a.ldo;
  p.hq = a.hq;
  p.hkv = a.hkv;
  p.hpt = pair ? 2 : 1;
  p.tstep = pair ? 1 : C::NSLOT;
  p.n_tiles = a.n_work * (a.hq / p.hpt);
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.causal = a.causal;
  p.window = a.window;
  p.status = a.status;
  const int grid = std::min(num_sms_cached(), p.n_tiles);
  if (launch_pdl(kern, dim3(grid), dim3(C::THREADS), C::SMEM, s, tq, tk, tv, to, p) != cudaSuccess) return -3;
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace

bool attention_tc_supported(int d) { return d == 64 || d == 128 || d == 256; }

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
    case 256: return launch_fa<256>(a, total_rows, s);
    default: return -1;
  }
}

}  // namespace inl
