// Host-side launchers of the sm_100a kernels (internal interface of
// libinl_cuda.so; the public C ABI is include/inl_cuda.h).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <utility>

// Every bf16 epilogue first multiplies the accumulator by the row scale
// r = rsqrt(sum(ss_in[row, :]) / ss_dim + ss_eps) when ss_in is given (the
// RMSNorm of the A rows, folded: RMSNorm(x) W^T = r * (x (W diag(w))^T)).
enum InlEpilogue : int {
  INL_EPI_BF16 = 0,        // out = bf16(r * acc)
  INL_EPI_RESID_BF16 = 1,  // out = bf16(r * acc + resid) (out may alias resid); ss_out gets the
                           // per-64-column sums of squares of the stored row
  INL_EPI_GATED_BF16 = 2,  // out[:, n/2] = act(r * gate) * (r * up), gate/up interleaved in gate_block rows
  INL_EPI_F32 = 3,         // out = r * acc (f32)
  INL_EPI_QKV = 4,         // q|k|v heads: per-head RMSNorm of q/k (qn/kn) + half-split RoPE at pos[row]
  INL_EPI_SEGMAX = 5,      // pooled[seg[col]][row] = max over columns of the segment (order-encoded atomicMax)
  INL_EPI_RESID_F32 = 6,   // out = r * acc + resid, f32 (resid read as f32; out may alias resid)
  INL_EPI_GATED_F32 = 7,   // as INL_EPI_GATED_BF16 with an f32 output
};

// Columns per partial sum of squares written by the residual epilogue.
constexpr int INL_SS_COLS = 64;

enum InlAct : int { INL_ACT_SILU = 0, INL_ACT_GELU_ERF = 1, INL_ACT_GELU_TANH = 2 };

namespace inl {

struct GemmArgs {
  const __nv_bfloat16* A = nullptr;  // [M, K] row stride lda
  long long lda = 0;
  const __nv_bfloat16* W = nullptr;  // [N, K] row stride ldw
  long long ldw = 0;
  int M = 0, N = 0, K = 0;
  int epi = INL_EPI_BF16;
  int act = INL_ACT_SILU;
  int gate_block = 128;  // rows per gate (or up) block of the interleaved weight
  void* out = nullptr;
  long long ldo = 0;
  const __nv_bfloat16* resid = nullptr;
  long long ldr = 0;
  // folded RMSNorm of the A rows: partial sums of squares [M, ss_in_parts]
  const float* ss_in = nullptr;
  int ss_in_parts = 0;
  int ss_dim = 0;
  float ss_eps = 0.f;
  // residual epilogue: partial sums of squares of the output rows [M, ceil(N / INL_SS_COLS)]
  float* ss_out = nullptr;
  // QKV epilogue; cos is the RoPE table packed by frequency pairs
  // [d/4, max_pos] x float4 (cos f, cos f+1, sin f, sin f+1); sin is unused
  const float* qn = nullptr;
  const float* kn = nullptr;
  const int* pos = nullptr;
  const float* cos = nullptr;
  const float* sin = nullptr;
  int hq = 0, hkv = 0, d = 0, max_pos = 0;
  float qk_eps = 1e-6f;
  // SEGMAX epilogue: column segments and the [segments, ldp] order-encoded maxima
  const int* seg = nullptr;
  int* pooled = nullptr;
  long long ldp = 0;
  int* status = nullptr;
  int max_ctas = 0;   // 0 = one CTA per SM
  int force_bn = 0;   // 0 = automatic tile width
  int cta_pair = 1;   // 1 = 256 x 256 tiles on CTA pairs (cta_group::2) where the epilogue allows, 0 = one CTA per tile
  // split-K (INL_EPI_F32 only): each tile's K blocks in `splits` slices, slice
  // s writing its partial product to out + s * M * ldo (splits_reduce_f32 sums them)
  int splits = 1;
};

// tcgen05 bf16 GEMM; returns 0 on success, <0 on bad arguments / launch error.
int gemm_bf16_tn(const GemmArgs& g, cudaStream_t stream);

// 2D TMA descriptor of a row-major bf16 matrix, 128-byte swizzle, box [box_rows, box_cols].
bool make_tma_2d_bf16(CUtensorMap* map, const void* base, long long rows, long long cols, long long ld,
                      int box_rows, int box_cols);
int num_sms_cached();

// Raises a kernel's dynamic shared-memory limit on the current device, once
// per (kernel, device). The attribute belongs to the device that is current
// when it is set, so a process driving several GPUs sets it on each. `done`
// holds one bit per device and is shared by host threads; setting the
// attribute twice from two threads is harmless.
template <typename Kernel>
inline cudaError_t set_smem_limit_once(Kernel kern, int bytes, std::atomic<unsigned long long>& done) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  const unsigned long long bit = 1ull << dev;
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (err == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
  return err;
}

// Launch with programmatic stream serialization: the kernel may start while
// its predecessor in the stream finishes, and must call pdl_wait() before it
// reads anything the predecessor wrote.
template <typename... Params, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

struct GemmF32Args {
  const float* A = nullptr;
  long long lda = 0;
  const float* W = nullptr;
  long long ldw = 0;
  const float* bias = nullptr;  // [N] or null
  int M = 0, N = 0, K = 0;
  int epi = INL_EPI_F32;  // INL_EPI_F32, INL_EPI_RESID_BF16 (meaning: f32 residual add), INL_EPI_GATED_BF16 (f32)
  int act = INL_ACT_SILU;
  int gate_block = 64;
  float* out = nullptr;
  long long ldo = 0;
  const float* resid = nullptr;
  long long ldr = 0;
};

// SIMT f32 GEMM (f32-accurate path for the f32 configurations).
int gemm_f32_tn(const GemmF32Args& g, cudaStream_t stream);

// f32 X[M,K] . W[N,K]^T reduced to pooled[seg[r]][n] = max over rows r of the segment
// (order-encoded int32, atomicMax; pooled pre-filled with the encoding of -inf).
int gemm_f32_segmax(const float* A, long long lda, const float* W, long long ldw, int M, int N, int K,
                    const int* seg, int* pooled, long long ldp, cudaStream_t s);

// ---------------------------------------------------------------- elementwise
// out[t, :] = table[ids[t], :] * scale ; ids >= vocab set *status = BAD_INDEX and write zeros.
// ss_out (optional, needs H % INL_SS_COLS == 0): per-64-column sums of squares of the stored rows.
int embed_gather(const uint32_t* ids, int T, const void* table, int table_bf16, int vocab, int H, float scale,
                 void* out, int out_bf16, int* status, cudaStream_t s, float* ss_out = nullptr);

// out = x / sqrt(mean(x^2) + eps) * w   (w f32, may be null)  rows x H
int rms_norm(const void* x, int x_bf16, long long ldx, const float* w, float eps, int rows, int H, void* out,
             int out_bf16, long long ldo, cudaStream_t s);

// LayerNorm without bias (bias may be null): (x - mu)/sqrt(var + eps) * w + b
int layer_norm(const void* x, int x_bf16, long long ldx, const float* w, const float* b, float eps, int rows, int H,
               void* out, int out_bf16, long long ldo, cudaStream_t s);

// In place on qkv rows [T, ld]: per head RMSNorm (weights qw/kw, may be null) on the
// q heads (cols [0, hq*d)) and k heads (cols [hq*d, (hq+hkv)*d)), optional weightless
// RMSNorm on v heads, then half-split RoPE on q and k with position pos[t] and the
// table cos/sin [max_pos, d/2]. rope_sel: which of (cos0,sin0)/(cos1,sin1) to use.
struct QkRopeArgs {
  void* qkv = nullptr;
  int bf16 = 1;
  long long ld = 0;
  int T = 0, hq = 0, hkv = 0, d = 0;
  const float* qw = nullptr;
  const float* kw = nullptr;
  int v_norm = 0;
  float eps = 1e-6f;
  const int* pos = nullptr;
  const float* cos = nullptr;
  const float* sin = nullptr;
  int max_pos = 0;
  int* status = nullptr;
};
int qk_norm_rope(const QkRopeArgs& a, cudaStream_t s);

// Position of every packed token inside its text: pos[t] = t - cu[i] for cu[i] <= t < cu[i+1].
int token_positions(const int* cu, int n, int T, int* pos, cudaStream_t s);

// 3xBF16: f32 rows -> bf16 [rows, 3K] at row stride ldo, mode 0 [hi | hi | lo]
// (activation side), mode 1 [hi | lo | hi] (weight side); mode 2 writes [hi]
// alone ([rows, K], a bf16 product); K, ldx, ldo even.
int split3_bf16(const float* x, long long ldx, int rows, int K, int mode, void* out, long long ldo, cudaStream_t s);
// out = sum over s < splits of ws[s * plane + row * ldw + col], in that order,
// plus resid when given (f32; out may alias resid): the second half of a
// split-K product.
int splits_reduce_f32(const float* ws, long long plane, long long ldw, int splits, int rows, int cols,
                      const float* resid, long long ldr, float* out, long long ldo, cudaStream_t s);
// out = a + b (f32 rows; out may alias a or b).
int add_rows_f32(float* out, long long ldo, const float* a, long long lda, const float* b, long long ldb, int rows,
                 int cols, cudaStream_t s);
// out[r, c] = act(gate) * up from x [rows, 2I] f32 whose columns alternate gate / up blocks of blk.
int act_mul_blocks_f32(const float* x, long long ldx, int rows, int I, int blk, int act, float* out, long long ldo,
                       cudaStream_t s);

// Sparse compaction of n dense f32 rows of width D: counts[i] = #{v : row_i[v] > 0};
// *bad set to 1 when a row holds a non-finite value.
int sparse_count(const float* rows, int n, int D, int* counts, int* bad, cudaStream_t s);
// idx / val[offsets[i] ..) = the active entries of row i in ascending column order.
int sparse_compact(const float* rows, int n, int D, const long long* offsets, int32_t* idx, float* val,
                   cudaStream_t s);

// out[i, :] = in[cu[i + 1] - 1, :] for the n texts (bf16 rows; cols, ld_in and
// ld_out multiples of 8, rows 16-byte aligned).
int gather_last_rows_bf16(const void* in, long long ld_in, const int* cu, int n, int cols, void* out,
                          long long ld_out, cudaStream_t s);

// Dense last-token head: out[i] = L2(RMSNorm(h[cu[i+1]-1])) in f32, L2 = x / sqrt(sum x^2 + 1e-12).
int last_token_norm_l2(const void* h, int h_bf16, long long ldh, const int* cu, int n, const float* w, float eps,
                       int H, float* out, cudaStream_t s);

// LayerNorm of gelu_erf(x) (the SPLADE MLM head: LN(gelu(dense(h)))); same dtypes in and out.
int norm_act(const void* x, int x_bf16, long long ldx, const float* w, const float* b, float eps, int rows, int H,
             void* out, int out_bf16, long long ldo, cudaStream_t s);

// h[r] += RMSNorm(a[r]) * w (row-wise, rows x H, both in the model dtype); with
// `scale` (one f32 on the device), h[r] = (h[r] + RMSNorm(a[r]) * w) * scale.
int add_rms_norm(void* h, const void* a, int bf16, const float* w, float eps, int rows, int H, cudaStream_t s,
                 const float* scale = nullptr);

// In place over rows x cols (contiguous): x = RMSNorm(x * scale) * w.
int scaled_rms_norm(void* x, int bf16, long long rows, int cols, float scale, const float* w, float eps,
                    cudaStream_t s);

// out[r, j] = act(x[r, j]) * y[r, j] over rows x cols with row strides (model dtype; out may be x).
int act_mul_rows(const void* x, long long ldx, const void* y, long long ldy, int bf16, int rows, int cols, int act,
                 void* out, long long ldo, cudaStream_t s);

// dst[r] = src[idx[r]] for r < n (rows of H values).
int gather_rows(const void* src, int bf16, long long lds, const int* idx, int n, int H, void* dst, cudaStream_t s);

int fill_i32(int* p, long long n, int value, cudaStream_t s);

// out[r, j] = act(x[r, j]) * x[r, I + j]  (x [rows, 2I], out [rows, I], same dtype).
int act_mul(const void* x, int bf16, int rows, int I, int act, void* out, cudaStream_t s);

// SPLADE finish + fold from order-encoded per-(text, term) maxima [n, V]:
// out = ln(1 + relu(m + bias - shift) * open), folded by max onto canon[v] (dim terms) when canon != null.
int splade_finish(const int* pooled, int n, int V, const float* bias, float shift, const float* open,
                  const int* canon, int dim, float* out, cudaStream_t s);

// Row L2: out = x / max(|x|, clamp) for f32 rows (x may alias out); clamp < 0 means x / sqrt(sum x^2 - clamp).
int rows_l2_f32(const float* x, long long ldx, int rows, int D, float clamp_min, float* out, long long ldo,
                cudaStream_t s);

// In place over rows x D (row stride ldx): x += bias (if given), then, with
// normalize, x /= max(||x||, clamp_min).
int bias_rows_l2_f32(float* x, long long ldx, int rows, int D, const float* bias, int normalize, float clamp_min,
                     cudaStream_t s);

// Segment mean over packed rows: out[i] = mean_{t in text i} x[t] (f32 out),
// the mean of each text's rows (f32 out [n, H]) through scratch of
// segment_mean_scratch_bytes(n, H, max_len) bytes (per-chunk partial sums);
// H and ldx multiples of 8, x 16-byte aligned.
size_t segment_mean_scratch_bytes(int n, int H, int max_len);
int segment_mean(const void* x, int x_bf16, long long ldx, const int* cu, int n, int H, int max_len, float* scratch,
                 float* out, cudaStream_t s);

// Truncate rows of [n, D] f32 to `dim` and renormalise (Matryoshka); out [n, dim].
int truncate_normalize(const float* x, int n, int D, int dim, float* out, cudaStream_t s);

// f32 -> bf16/f32 conversion with row remapping dst_row(r) = (r / blk) * blk_stride + off + r % blk
// and an optional per-column scale (a folded norm weight).
int convert_rows(const float* src, int rows, int cols, void* dst, int dst_bf16, long long ld_dst, int blk,
                 long long blk_stride, long long off, cudaStream_t s, const float* col_scale = nullptr);
int convert_bf16_rows(const __nv_bfloat16* src, int rows, int cols, void* dst, int dst_bf16, long long ld_dst,
                      int blk, long long blk_stride, long long off, cudaStream_t s,
                      const float* col_scale = nullptr);

// ---------------------------------------------------------------- attention
struct AttnArgs {
  const void* q = nullptr;  // [T, ldq] q heads at column h*d
  const void* k = nullptr;  // [T, ldk] kv heads at column g*d
  const void* v = nullptr;
  long long ldq = 0, ldk = 0, ldv = 0;
  void* out = nullptr;  // [T, ldo] q heads at column h*d
  long long ldo = 0;
  int bf16 = 1;
  int hq = 0, hkv = 0, d = 0;
  float scale = 1.0f;
  int causal = 0;
  int window = -1;  // |q - k| > window masked when >= 0
  const int* cu = nullptr;     // device [n+1]
  int n = 0;
  const int2* work = nullptr;  // device [n_work] = (text, q_block)
  int n_work = 0;
  int q_block = 64;
  long long total_rows = 0;    // rows of q/k/v (packed tokens), bounds the TMA maps
  int* status = nullptr;
};
int attention(const AttnArgs& a, cudaStream_t s);

// tcgen05 flash attention (bf16, head_dim 64 / 128, 128-query work items).
bool attention_tc_supported(int d);
int attention_tc(const AttnArgs& a, long long total_rows, cudaStream_t s);

// Number of query rows per work item the attention kernels expect.
int attention_q_block(int bf16, int d);

// Whether attention() has a kernel for this dtype and head_dim.
bool attention_supported(int bf16, int d);

// ---------------------------------------------------------------- Gated DeltaNet (Qwen3.5 linear attention)
// out[t, c] = silu(sum_j w[c, j] x[t - K + 1 + j, c]) over each text's tokens (pos[t] = position in its text).
int causal_conv_silu(const float* x, long long ldx, int T, int C, const float* w, int K, const int* pos, float* out,
                     long long ldo, cudaStream_t s);

struct DeltaArgs {
  const float* mixed = nullptr;  // [T, ld_mixed]: q (nk dk) | k (nk dk) | v (nv dv), after the convolution
  long long ld_mixed = 0;
  const float* b_in = nullptr;   // [T, ld_ab] step-size logits (beta = sigmoid) at column vh
  const float* a_in = nullptr;   // [T, ld_ab] decay inputs (g = softplus(a + dt_bias) * -exp(A_log)) at column vh
  long long ld_ab = 0;
  const float* z = nullptr;      // [T, ld_z] output gate, nv dv columns
  long long ld_z = 0;
  const float* dt_bias = nullptr;  // [nv]
  const float* a_log = nullptr;    // [nv]
  const float* norm_w = nullptr;   // [dv] gated RMSNorm weight
  float eps = 1e-6f;
  int nk = 0, nv = 0, dk = 0, dv = 0;
  const int* cu = nullptr;  // device [n+1]
  int n = 0;
  float* out = nullptr;     // [T, ldo] nv dv columns
  long long ldo = 0;
};
// Recurrent gated delta rule with the gated RMSNorm fused; -1 on unsupported shapes.
int gated_delta_rule(const DeltaArgs& a, cudaStream_t s);

// ---------------------------------------------------------------- Qwen3.5 gated full attention (f32)
struct Qwen35QkArgs {
  float* qkv = nullptr;   // [T, ld]: q | gate per head (2 d each, hq heads), then k (hkv d), then v (hkv d)
  long long ld = 0;
  float* q_out = nullptr; // [T, ldq] normed, rotated q heads (d each)
  long long ldq = 0;
  int T = 0, hq = 0, hkv = 0, d = 0;
  int rot = 0;            // rotary features per head (half-split rotation of the first `rot`)
  const float* qw = nullptr;  // [d] q norm scale (1 + w folded)
  const float* kw = nullptr;  // [d] k norm scale (1 + w folded)
  float eps = 1e-6f;
  const int* pos = nullptr;
  const float* cos = nullptr;  // [max_pos, rot / 2]
  const float* sin = nullptr;
  int max_pos = 0;
  int* status = nullptr;
};
int qk_prep_gated(const Qwen35QkArgs& a, cudaStream_t s);
// out[t, h d + j] *= sigmoid(gate[t, h 2d + d + j]) (gate_base = the q | gate rows).
int gate_sigmoid_mul(float* out, long long ldo, const float* gate_base, long long ldg, int T, int hq, int d,
                     cudaStream_t s);
// f32 attention for head_dim <= 32 on the f32 work list (32-query blocks).
int attention_small(const AttnArgs& a, cudaStream_t s);

}  // namespace inl
