// Packed variable-length attention that allocates no device memory.
//
// inl_cuda_attention keeps its cu_seqlens copy and work list in buffers it
// grows with cudaMalloc. Some callers cannot allow that: a host that has
// handed all of the GPU's memory to its own pool allocator, or that runs
// inside a region where any cudaMalloc/cudaFree would synchronise the device
// or be refused. For them inl_cuda_attention_noalloc keeps that state in
// one file-scope device array instead, sized for at most kMaxTexts texts and
// kMaxWork query blocks per call, and rejects larger calls.
//
// Memory layout of the array (ints):
//   [0]                        status word of the bounded device waits
//   [kCuOffset, +kMaxTexts+1)   cu_seqlens copied from the caller's host array
//   [kWorkOffset, +2*kMaxWork)  work list, one (text, query block) int2 each
// The work list is built on the device from the copied offsets, so nothing is
// staged through host heap memory either. It is ordered heaviest first, as
// the allocating entry point orders it, so the persistent attention kernels,
// which take their tiles in list order, start the long tails early.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "inl_cuda.h"
#include "inl_cuda_kernels.h"
#include "kernels.h"

namespace inl {
int record_error(int code, const std::string& msg);
}

namespace {

constexpr int kMaxTexts = 8192;
constexpr int kMaxWork = 32768;
constexpr int kCuOffset = 64;  // ints; the status word sits alone in the first 256 bytes
constexpr int kWorkOffset = (kCuOffset + kMaxTexts + 1 + 63) / 64 * 64;
constexpr int kScratchInts = kWorkOffset + 2 * kMaxWork;
constexpr int kMaxDevices = 64;
constexpr int kBuildThreads = 1024;
// The build kernel sorts one 32-bit key per text: block count (at most
// kMaxWork = 2^15, 16 bits) above the text index (13 bits).
constexpr int kTextBits = 13;
constexpr int kBuildSmem = (2 * kMaxTexts + 1) * static_cast<int>(sizeof(int));

static_assert(kMaxTexts == 1 << kTextBits, "one sort key slot per text");
static_assert(kMaxWork <= 1 << 16, "block counts fit above the text index");
static_assert(kWorkOffset % 2 == 0, "work list must be int2-aligned");
static_assert(kScratchInts * sizeof(int) == 295424, "288.5 KiB");

// 288.5 KiB on every GPU that loads the library, held until the process exits.
static __device__ __align__(256) int g_attention_scratch[kScratchInts];

// Device address of g_attention_scratch per device, looked up on the first
// call made with that device current. Guarded by g_mu.
int* g_scratch_addr[kMaxDevices] = {};
std::mutex g_mu;
std::atomic<unsigned long long> g_build_smem{0};  // build kernel's shared-memory limit, one bit per device

// Largest r in [0, n) with a[r] <= x, for a non-decreasing a with a[0] <= x.
__device__ __forceinline__ int last_at_most(const int* a, int n, int x) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a[mid] <= x) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// One CTA builds the work list, heaviest first:
//   1. key[t] = (blocks of text t) << 13 | (8191 - t), bitonic-sorted in
//      descending order: texts by block count, ties in text order;
//   2. pre[r] = blocks of the sorted texts before r (exclusive scan);
//   3. every output slot finds its item by binary search.
// Not causal: every block of a text costs the text's length, so the sorted
// texts' blocks follow one another (slot p -> sorted text r with
// pre[r] <= p, block p - pre[r]). Causal: block b attends to b + 1 key
// blocks, so the list runs block index b from the largest down, and within a
// level the sorted texts that have a block b, longest first. The items above
// level b number O(b) = sum_r max(0, nb_r - b - 1) = pre[c] - (b + 1) c with
// c = #{r : nb_r > b + 1}, a prefix of the sorted order; slot p belongs to
// the smallest b with O(b) <= p, as sorted text p - O(b).
__global__ void __launch_bounds__(kBuildThreads) build_work_kernel(const int* __restrict__ cu, int n, int qb,
                                                                   int causal, int2* __restrict__ work,
                                                                   int n_work) {
  extern __shared__ int smem[];
  int* key = smem;              // [kMaxTexts]
  int* pre = smem + kMaxTexts;  // [kMaxTexts + 1]
  const int t = threadIdx.x;
  for (int i = t; i < kMaxTexts; i += kBuildThreads) {
    const int nb = i < n ? (cu[i + 1] - cu[i] + qb - 1) / qb : 0;
    key[i] = i < n ? (nb << kTextBits) | (kMaxTexts - 1 - i) : 0;
  }
  __syncthreads();
  for (int k = 2; k <= kMaxTexts; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = t; i < kMaxTexts; i += kBuildThreads) {
        const int partner = i ^ j;
        if (partner > i) {
          const bool desc = (i & k) == 0;
          const int a = key[i], b = key[partner];
          if (desc ? a < b : a > b) {
            key[i] = b;
            key[partner] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  // exclusive scan of the sorted block counts: each thread sums a run of 8
  constexpr int kRun = kMaxTexts / kBuildThreads;
  int run = 0;
  for (int r = t * kRun; r < (t + 1) * kRun; ++r) run += key[r] >> kTextBits;
  __shared__ int part[kBuildThreads];
  part[t] = run;
  __syncthreads();
  for (int off = 1; off < kBuildThreads; off <<= 1) {
    const int add = t >= off ? part[t - off] : 0;
    __syncthreads();
    part[t] += add;
    __syncthreads();
  }
  int acc = part[t] - run;
  for (int r = t * kRun; r < (t + 1) * kRun; ++r) {
    pre[r] = acc;
    acc += key[r] >> kTextBits;
  }
  if (t == kBuildThreads - 1) pre[kMaxTexts] = acc;
  __syncthreads();
  const int n_sorted = min(n, kMaxTexts);
  for (int p = t; p < n_work; p += kBuildThreads) {
    int r, b;
    if (!causal) {
      r = last_at_most(pre, n_sorted, p);  // texts without blocks share pre with the next and sort last
      b = p - pre[r];
    } else {
      const int top = (key[0] >> kTextBits) - 1;  // largest block index
      int lo = 0, hi = top;                       // smallest b in [0, top] with O(b) <= p
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        // c = #{r : nb_r > mid + 1}, the sorted prefix of texts longer than mid + 1 blocks
        int c_lo = 0, c_hi = n_sorted;
        while (c_lo < c_hi) {
          const int m = (c_lo + c_hi) >> 1;
          if ((key[m] >> kTextBits) > mid + 1) c_lo = m + 1; else c_hi = m;
        }
        const int above = pre[c_lo] - (mid + 1) * c_lo;
        if (above <= p) hi = mid; else lo = mid + 1;
      }
      b = lo;
      int c_lo = 0, c_hi = n_sorted;
      while (c_lo < c_hi) {
        const int m = (c_lo + c_hi) >> 1;
        if ((key[m] >> kTextBits) > b + 1) c_lo = m + 1; else c_hi = m;
      }
      r = p - (pre[c_lo] - (b + 1) * c_lo);
    }
    const int text = kMaxTexts - 1 - (key[r] & (kMaxTexts - 1));
    work[p] = make_int2(text, b);
  }
}

int cuda_fail(cudaError_t e, const char* what) {
  return inl::record_error(INL_ERR_INFERENCE, std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

extern "C" {

int inl_cuda_attention_noalloc(const void* q, const void* k, const void* v, int64_t ldq, int64_t ldk, int64_t ldv,
                               void* out, int64_t ldo, int dtype, int hq, int hkv, int d, float scale, int causal,
                               int window, const int32_t* cu_seqlens_host, int n_texts, void* stream) {
  if (n_texts <= 0) return INL_OK;
  if (!cu_seqlens_host) return inl::record_error(INL_ERR_CONFIG, "NULL cu_seqlens");
  if (n_texts > kMaxTexts)
    return inl::record_error(INL_ERR_INVALID_INPUT, "attention_noalloc: " + std::to_string(n_texts) +
                                                        " texts exceed its limit of " + std::to_string(kMaxTexts));
  if (cu_seqlens_host[0] != 0) return inl::record_error(INL_ERR_INVALID_INPUT, "cu_seqlens[0] must be 0");
  const bool bf16 = dtype == INL_DTYPE_BF16;
  const int qb = inl::attention_q_block(bf16, d);
  long long n_work = 0;
  for (int i = 0; i < n_texts; ++i) {
    const int L = cu_seqlens_host[i + 1] - cu_seqlens_host[i];
    if (L < 0) return inl::record_error(INL_ERR_INVALID_INPUT, "cu_seqlens must be non-decreasing");
    n_work += (L + qb - 1) / qb;
  }
  if (n_work > kMaxWork)
    return inl::record_error(INL_ERR_INVALID_INPUT,
                             "attention_noalloc: " + std::to_string(n_work) + " query blocks of " +
                                 std::to_string(qb) + " rows exceed its limit of " + std::to_string(kMaxWork));
  if (n_work == 0) return INL_OK;
  // Everything the attention launcher can refuse is checked here, before any
  // work is queued on the stream: an error return never leaves a build of
  // the shared list running behind it.
  if (hq <= 0 || hkv <= 0 || hq % hkv != 0 || !inl::attention_supported(bf16, d))
    return inl::record_error(INL_ERR_INVALID_INPUT, "attention: unsupported head_dim / heads");
  if (!q || !k || !v || !out) return inl::record_error(INL_ERR_CONFIG, "NULL q, k, v or out");
  if (bf16 && inl::attention_tc_supported(d) &&
      ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
        reinterpret_cast<uintptr_t>(out)) & 15 || (ldq | ldk | ldv | ldo) % 8))
    return inl::record_error(INL_ERR_INVALID_INPUT,
                             "attention: q, k, v and out need 16-byte alignment and row strides of 8 elements");

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The call waits for its stream before it returns (the array is shared), so
  // a stream that is capturing is refused before anything is queued on it.
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(s, &capture);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamIsCapturing");
  if (capture != cudaStreamCaptureStatusNone)
    return inl::record_error(INL_ERR_CONFIG, "attention_noalloc: the stream is capturing; this call waits for "
                                             "its stream, which a capture does not allow");
  std::lock_guard<std::mutex> lock(g_mu);
  int dev = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return inl::record_error(INL_ERR_CONFIG, "device index out of range");
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attention_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(attention scratch)");
    g_scratch_addr[dev] = static_cast<int*>(p);
  }
  if ((e = inl::set_smem_limit_once(build_work_kernel, kBuildSmem, g_build_smem)) != cudaSuccess)
    return cuda_fail(e, "work list build");
  int* status = g_scratch_addr[dev];
  int* dcu = status + kCuOffset;
  int2* dwork = reinterpret_cast<int2*>(status + kWorkOffset);

  // From the first queued operation on, every return drains the stream while
  // the lock is held: the next call rewrites the array.
  auto drained = [&](int code) {
    cudaStreamSynchronize(s);
    return code;
  };
  // The status word must start at zero; cu and the work list are overwritten.
  if ((e = cudaMemsetAsync(status, 0, sizeof(int), s)) != cudaSuccess) return drained(cuda_fail(e, "status clear"));
  if ((e = cudaMemcpyAsync(dcu, cu_seqlens_host, static_cast<size_t>(n_texts + 1) * sizeof(int),
                           cudaMemcpyHostToDevice, s)) != cudaSuccess)
    return drained(cuda_fail(e, "cu_seqlens copy"));
  build_work_kernel<<<1, kBuildThreads, kBuildSmem, s>>>(dcu, n_texts, qb, causal != 0, dwork,
                                                         static_cast<int>(n_work));
  if ((e = cudaGetLastError()) != cudaSuccess) return drained(cuda_fail(e, "work list build"));
  inl::AttnArgs a;
  a.q = q;
  a.k = k;
  a.v = v;
  a.ldq = ldq;
  a.ldk = ldk;
  a.ldv = ldv;
  a.out = out;
  a.ldo = ldo;
  a.bf16 = bf16;
  a.hq = hq;
  a.hkv = hkv;
  a.d = d;
  a.scale = scale;
  a.causal = causal;
  a.window = window;
  a.cu = dcu;
  a.n = n_texts;
  a.work = dwork;
  a.n_work = static_cast<int>(n_work);
  a.q_block = qb;
  a.total_rows = cu_seqlens_host[n_texts];
  a.status = status;
  const int r = inl::attention(a, s);
  if (r == -1) return drained(inl::record_error(INL_ERR_INVALID_INPUT, "attention: unsupported head_dim / heads"));
  if (r != 0) return drained(inl::record_error(INL_ERR_INFERENCE, "attention launch failed"));
  int device_status = 0;
  if ((e = cudaMemcpyAsync(&device_status, status, sizeof(int), cudaMemcpyDeviceToHost, s)) != cudaSuccess)
    return drained(cuda_fail(e, "status read"));
  if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return cuda_fail(e, "attention");
  if (device_status != 0)
    return inl::record_error(INL_ERR_TIMEOUT, "attention: a device wait ran past its limit (code " +
                                                  std::to_string(device_status) + ")");
  return INL_OK;
}

}  // extern "C"
