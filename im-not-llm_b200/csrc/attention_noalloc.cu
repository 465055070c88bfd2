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
// staged through host heap memory either.
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

static_assert(kWorkOffset % 2 == 0, "work list must be int2-aligned");
static_assert(kScratchInts * sizeof(int) == 295424, "288.5 KiB");

// 288.5 KiB on every GPU that loads the library, held until the process exits.
static __device__ __align__(256) int g_attention_scratch[kScratchInts];

// Device address of g_attention_scratch per device, looked up on the first
// call made with that device current. Guarded by g_mu.
int* g_scratch_addr[kMaxDevices] = {};
std::mutex g_mu;

// One CTA: each thread counts the query blocks of a contiguous run of texts,
// a shared-memory scan gives every run its first slot, then each thread writes
// its (text, block) pairs in text order. Slots at or past `cap` are skipped.
__global__ void __launch_bounds__(kBuildThreads) build_work_kernel(const int* __restrict__ cu, int n, int qb,
                                                                   int2* __restrict__ work, int cap) {
  __shared__ int part[kBuildThreads];
  const int t = threadIdx.x;
  const int chunk = (n + kBuildThreads - 1) / kBuildThreads;
  const int lo = min(n, t * chunk), hi = min(n, lo + chunk);
  int count = 0;
  for (int i = lo; i < hi; ++i) count += (cu[i + 1] - cu[i] + qb - 1) / qb;
  part[t] = count;
  __syncthreads();
  for (int off = 1; off < kBuildThreads; off <<= 1) {
    const int add = t >= off ? part[t - off] : 0;
    __syncthreads();
    part[t] += add;
    __syncthreads();
  }
  int slot = part[t] - count;
  for (int i = lo; i < hi; ++i) {
    const int blocks = (cu[i + 1] - cu[i] + qb - 1) / qb;
    for (int b = 0; b < blocks; ++b, ++slot)
      if (slot < cap) work[slot] = make_int2(i, b);
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
  const int qb = inl::attention_q_block(dtype == INL_DTYPE_BF16, d);
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

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  std::lock_guard<std::mutex> lock(g_mu);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return inl::record_error(INL_ERR_CONFIG, "device index out of range");
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attention_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(attention scratch)");
    g_scratch_addr[dev] = static_cast<int*>(p);
  }
  int* status = g_scratch_addr[dev];
  int* dcu = status + kCuOffset;
  int2* dwork = reinterpret_cast<int2*>(status + kWorkOffset);

  // The status word must start at zero; cu and the work list are overwritten.
  if ((e = cudaMemsetAsync(status, 0, sizeof(int), s)) != cudaSuccess) return cuda_fail(e, "status clear");
  if ((e = cudaMemcpyAsync(dcu, cu_seqlens_host, static_cast<size_t>(n_texts + 1) * sizeof(int),
                           cudaMemcpyHostToDevice, s)) != cudaSuccess)
    return cuda_fail(e, "cu_seqlens copy");
  if (n_work > 0) {
    build_work_kernel<<<1, kBuildThreads, 0, s>>>(dcu, n_texts, qb, dwork, kMaxWork);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e, "work list build");
  }
  inl::AttnArgs a;
  a.q = q;
  a.k = k;
  a.v = v;
  a.ldq = ldq;
  a.ldk = ldk;
  a.ldv = ldv;
  a.out = out;
  a.ldo = ldo;
  a.bf16 = dtype == INL_DTYPE_BF16;
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
  if (r == -1) return inl::record_error(INL_ERR_INVALID_INPUT, "attention: unsupported head_dim / heads");
  if (r != 0) return inl::record_error(INL_ERR_INFERENCE, "attention launch failed");
  // Drain the stream while holding the lock: the next call rewrites the array.
  int device_status = 0;
  if ((e = cudaMemcpyAsync(&device_status, status, sizeof(int), cudaMemcpyDeviceToHost, s)) != cudaSuccess)
    return cuda_fail(e, "status read");
  if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return cuda_fail(e, "attention");
  if (device_status != 0)
    return inl::record_error(INL_ERR_TIMEOUT, "attention: a device wait ran past its limit (code " +
                                                  std::to_string(device_status) + ")");
  return INL_OK;
}

}  // extern "C"
