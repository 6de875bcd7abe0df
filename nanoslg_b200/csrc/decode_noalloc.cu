// nslg_paged_decode_noalloc: the paged decode attention of nslg_paged_decode for callers
// that cannot allocate device memory.
//
// Who needs it. nslg_paged_decode takes a caller-provided workspace for its split-KV
// partials, which the caller usually gets from cudaMalloc or a framework allocator. Some
// callers have neither: a serving process that hands nearly all HBM to its KV page pool
// at start-up and then runs with a fixed budget (a later cudaMalloc may fail or fragment
// what is left); a host program in another language that binds this C ABI and owns no
// device allocator; a latency-critical decode loop that cannot afford the device-wide
// synchronisation cudaMalloc and cudaFree can imply. This entry point takes the same
// inputs and outputs but keeps its scratch in a fixed array that lives in this library.
//
// The array. g_noalloc_scratch below is a file-scope __device__ array of
// NSLG_NOALLOC_SCRATCH_BYTES (8 MiB). Every GPU on which the library's code is loaded
// holds these 8 MiB until the process exits. Host code cannot pass the array's name to
// a kernel: on the host that name is only a stand-in, not a device address. So on the
// first call on each device (with that device current) we look its device address up
// once with cudaGetSymbolAddress and reuse it afterwards; make that first call before
// any stream capture. The first call on a device also loads this module if it is not
// loaded yet. The address is kept together with the CUDA context it was looked up in;
// a call made in another context (after cudaDeviceReset, or in a context the caller
// created) looks it up again, so make the first call in each new context before any
// stream capture too.
//
// Sharing. Every call on a device uses the same array and it keeps whatever the last
// call left there. The decode kernel needs the array's first words (its per-CTA arrival
// counts) to be zero before a call and leaves them zero after it; a __device__ array
// starts zeroed when the module is loaded, so that holds from the first call on. The
// partial results behind them need no initial value: a call reads only partials that
// its own CTAs have just written. Two calls whose kernels overlap on the GPU (for
// example on two streams without an ordering between them) race on the array and
// corrupt each other's results; order them.
//
// Limit. The scratch a call needs is (batch + #SMs) * num_qo_heads * (head_dim + 1) * 4
// bytes, plus the arrival counts (#SMs words rounded up to 256 bytes) and 256 bytes for
// alignment; calls needing more than 8 MiB are rejected with
// NSLG_ERR_WORKSPACE and a message. Shapes the tensor-core kernel does not cover run the
// CUDA-core kernel, which needs no scratch. No call allocates or frees device memory.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "launch.h"

namespace nslg {
namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[NSLG_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};
CUcontext g_scratch_ctx[kMaxDevices] = {};   // the context each address belongs to

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// cuCtxGetCurrent through the runtime's driver entry point (the library does not link
// libcuda itself); null if the driver does not provide it.
CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(ptr);
  });
  return fn;
}

// Device address of g_noalloc_scratch on the current device, looked up once per device
// and context: the address is cached with the context that was current when it was
// looked up, and looked up again when the calling thread's current context differs (a
// new primary context after cudaDeviceReset, or a context the caller created), since
// the module, and with it the array, is loaded at another address in each context.
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return set_error(NSLG_ERR_CUDA, cudaGetErrorString(err));
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(NSLG_ERR_UNSUPPORTED, "paged_decode_noalloc: device index >= 64");
  CtxGetCurrentFn get = ctx_get_current_fn();
  if (get == nullptr)
    return set_error(NSLG_ERR_CUDA, "paged_decode_noalloc: driver has no cuCtxGetCurrent");
  // null until the runtime has bound a context to this thread; the lookup below does that
  CUcontext ctx = nullptr;
  if (get(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (ctx == nullptr || g_scratch_addr[dev] == nullptr || g_scratch_ctx[dev] != ctx) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess || p == nullptr)
      return set_error(NSLG_ERR_CUDA, std::string("paged_decode_noalloc: cudaGetSymbolAddress: ") +
                                          cudaGetErrorString(err));
    if (get(&ctx) != CUDA_SUCCESS || ctx == nullptr)
      return set_error(NSLG_ERR_CUDA, "paged_decode_noalloc: no current CUDA context");
    g_scratch_addr[dev] = p;
    g_scratch_ctx[dev] = ctx;
  }
  *out = g_scratch_addr[dev];
  return NSLG_OK;
}

}  // namespace
}  // namespace nslg

using namespace nslg;

extern "C" int nslg_paged_decode_noalloc(int dtype, int batch, int num_qo_heads,
                                         int num_kv_heads, int head_dim, int page_size,
                                         const void* q, int64_t q_stride, void* out,
                                         int64_t out_stride, const void* pool_k,
                                         const void* pool_v, int64_t num_pages,
                                         const int32_t* kv_indptr, const int32_t* kv_indices,
                                         const int32_t* kv_last_page_len, float sm_scale,
                                         uint32_t* dev_status, void* stream) {
  clear_error();
  if (dtype != NSLG_DTYPE_BF16 && dtype != NSLG_DTYPE_F16 && dtype != NSLG_DTYPE_F32)
    return set_error(NSLG_ERR_ARG, "paged_decode_noalloc: bad dtype");
  if (batch < 0) return set_error(NSLG_ERR_ARG, "paged_decode_noalloc: batch < 0");
  if (batch == 0) return NSLG_OK;
  if (num_qo_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || num_qo_heads % num_kv_heads)
    return set_error(NSLG_ERR_ARG,
                     "paged_decode_noalloc: need num_qo_heads % num_kv_heads == 0");
  if (page_size <= 0 || num_pages <= 0)
    return set_error(NSLG_ERR_ARG, "paged_decode_noalloc: page_size and num_pages must be positive");
  if (!q || !out || !pool_k || !pool_v || !kv_indptr || !kv_indices || !kv_last_page_len)
    return set_error(NSLG_ERR_ARG, "paged_decode_noalloc: null pointer");
  if (!(sm_scale > 0.f)) return set_error(NSLG_ERR_ARG, "paged_decode_noalloc: sm_scale must be > 0");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool aligned = (reinterpret_cast<uintptr_t>(pool_k) & 15u) == 0 &&
                       (reinterpret_cast<uintptr_t>(pool_v) & 15u) == 0 &&
                       (reinterpret_cast<uintptr_t>(q) & 3u) == 0 &&
                       (reinterpret_cast<uintptr_t>(out) & 3u) == 0 && q_stride % 2 == 0 &&
                       out_stride % 2 == 0;
  if (!(decode_tc_supported(dtype, num_qo_heads, num_kv_heads, head_dim, page_size) && aligned))
    return launch_paged_attention_simt(dtype, batch, num_qo_heads, num_kv_heads, head_dim,
                                       page_size, q, q_stride, out, out_stride, nullptr, nullptr,
                                       1, pool_k, pool_v, num_pages, kv_indptr, kv_indices,
                                       kv_last_page_len, sm_scale, 0, dev_status, st);
  const int64_t need = decode_tc_workspace_bytes(batch, num_qo_heads, head_dim);
  if (need > NSLG_NOALLOC_SCRATCH_BYTES)
    return set_error(NSLG_ERR_WORKSPACE,
                     "paged_decode_noalloc: this batch needs " + std::to_string(need) +
                         " bytes of scratch, more than the fixed " +
                         std::to_string(static_cast<long long>(NSLG_NOALLOC_SCRATCH_BYTES)) +
                         "; use nslg_paged_decode with a workspace");
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc != NSLG_OK) return rc;
  return launch_paged_decode_tc(dtype, batch, num_qo_heads, num_kv_heads, head_dim, q, q_stride, out,
                                out_stride, pool_k, pool_v, num_pages, kv_indptr, kv_indices,
                                kv_last_page_len, sm_scale, scratch, NSLG_NOALLOC_SCRATCH_BYTES,
                                dev_status, st);
}
