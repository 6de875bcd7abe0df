// Device-side planning of a decode step: the per-forward plan of
// FlashInferCacheContext.__init__ + _plan_flashinfer (kv_cache.py:547-632) for the case
// where every sequence adds one token, built on the GPU from block tables that live in
// device memory.
//
// The host keeps the page bookkeeping (pool, radix tree, block tables) and sends, per
// step, only the batch's table rows ("slots"), the sequences' token counts before the
// step and the block-table entries that changed since the last step (new pages, copies
// on write). Kernel 1 (one CTA) applies the changes, then computes every sequence's
// position, write location (page * page_size + slot), page count and last-page length,
// and the page-list offsets kv_indptr with a block-wide exclusive scan; kernel 2 (one
// CTA per sequence) gathers each sequence's page ids into kv_indices. Output layout and
// values are those of the host plan, element for element.
//
// nslg_plan_decode_host does the same step from HOST arrays in one call: it copies them
// into a pinned, device-mapped staging slot owned by the library (a ring of slots per
// device, each reused only after the kernels that read it have finished, tracked with
// one event per slot) and the kernels read the few hundred bytes straight from there;
// the pages allocated since the last forward are zeroed (K and V pools) in the same
// call. No device upload buffer, no separate copy: one host call per decode step, and
// for batches up to kFusedMaxBatch one kernel launch (plan_decode_fused_kernel). A
// step whose arrays fit PlanInline (up to 128 sequences, 192 table changes, 96 pages to
// zero: a decode step's steady state) skips the staging too: the arrays travel in the
// launch's parameters, and the kernel reads no host memory (each dependent read of the
// mapped staging is a PCIe round trip: 23 us per step on B200 for the C2 batch of 64).
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "launch.h"

namespace nslg {
namespace {

constexpr int kScanThreads = 1024;
constexpr int kMaxItems = 4;                 // sequences per scan thread (batch <= 4096)

struct PlanParams {
  int batch, page_size, num_updates;
  const int32_t* slots;
  const int32_t* starts;
  const int32_t* updates;   // [num_updates][3] = (slot, index, page id)
  int32_t* bt;
  int64_t bt_stride, bt_rows;
  int32_t *positions, *write_loc, *indptr, *lpl, *qo, *row_start, *indices;
  int64_t max_indices;
  uint32_t* status;
};

__global__ void __launch_bounds__(kScanThreads) plan_decode_scan_kernel(const PlanParams p) {
  __shared__ int32_t warp_sums[kScanThreads / 32];
  const int t = threadIdx.x, lane = t % 32, warp = t / 32;
  // 1. block-table changes
  for (int i = t; i < p.num_updates; i += kScanThreads) {
    const int s = p.updates[3 * i], j = p.updates[3 * i + 1], pg = p.updates[3 * i + 2];
    if (s >= 0 && s < p.bt_rows && j >= 0 && j < p.bt_stride)
      p.bt[s * p.bt_stride + j] = pg;
    else
      report(p.status, NSLG_DEV_BAD_PLAN);
  }
  __syncthreads();
  // 2. per-sequence values; thread t owns sequences [t * k, t * k + k)
  const int k = (p.batch + kScanThreads - 1) / kScanThreads;
  int npg[kMaxItems];
  int local = 0;
#pragma unroll
  for (int e = 0; e < kMaxItems; ++e) {
    const int b = t * k + e;
    npg[e] = 0;
    if (e >= k || b >= p.batch) continue;
    const int s = p.slots[b];
    const int pos = p.starts[b];
    const int len = pos + 1;
    const int n = (len + p.page_size - 1) / p.page_size;
    const int pi = pos / p.page_size;
    int loc = -1;
    if (s >= 0 && s < p.bt_rows && pi < p.bt_stride) {
      loc = p.bt[s * p.bt_stride + pi] * p.page_size + pos % p.page_size;
    } else {
      report(p.status, NSLG_DEV_BAD_PLAN);
    }
    p.positions[b] = pos;
    p.write_loc[b] = loc;
    p.lpl[b] = len - (n - 1) * p.page_size;
    p.qo[b] = b;
    p.row_start[b] = b;
    npg[e] = n;
    local += n;
  }
  // 3. exclusive scan of the page counts
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += v;
    }
    warp_sums[lane] = w;   // inclusive over warps
  }
  __syncthreads();
  int run = incl - local + (warp > 0 ? warp_sums[warp - 1] : 0);
#pragma unroll
  for (int e = 0; e < kMaxItems; ++e) {
    const int b = t * k + e;
    if (e >= k || b >= p.batch) continue;
    p.indptr[b] = run;
    run += npg[e];
  }
  if (t == kScanThreads - 1) {
    p.indptr[p.batch] = run;
    p.qo[p.batch] = p.batch;
    if (run > p.max_indices) report(p.status, NSLG_DEV_BAD_PLAN);
  }
}

__global__ void __launch_bounds__(128) plan_decode_gather_kernel(const PlanParams p) {
  const int b = blockIdx.x;
  const int beg = p.indptr[b], end = p.indptr[b + 1];
  const int s = p.slots[b];
  if (s < 0 || s >= p.bt_rows || end - beg > p.bt_stride || end > p.max_indices) {
    if (threadIdx.x == 0) report(p.status, NSLG_DEV_BAD_PLAN);
    return;
  }
  const int32_t* row = p.bt + s * p.bt_stride;
  for (int j = threadIdx.x; j < end - beg; j += blockDim.x) p.indices[beg + j] = row[j];
}

// Zeroes `pages` of one or two pool tensors [layers, pages_total, page elements]: block
// (i, l, z) clears page pages[i] of layer l of pool z with 16-byte stores.
__global__ void __launch_bounds__(256) zero_pages_kernel(const int32_t* pages, int n,
                                                         uint8_t* pool0, uint8_t* pool1,
                                                         int64_t num_pages,
                                                         int64_t layer_stride,
                                                         int64_t page_bytes, uint32_t* status) {
  const int i = blockIdx.x, l = blockIdx.y;
  const int pg = pages[i];
  if (pg < 0 || pg >= num_pages) {
    if (threadIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) report(status, NSLG_DEV_BAD_PLAN);
    return;
  }
  uint8_t* pool = blockIdx.z ? pool1 : pool0;
  uint4* dst = reinterpret_cast<uint4*>(pool + l * layer_stride + pg * page_bytes);
  const int64_t nv = page_bytes / 16;
  for (int64_t v = threadIdx.x; v < nv; v += blockDim.x) dst[v] = make_uint4(0u, 0u, 0u, 0u);
}

// Small batches in one launch: block b < batch plans sequence b alone (its page-list
// offset is the sum of the page counts of sequences 0..b-1, each block summing them
// itself; it applies the table updates of its own row, then writes its fields and
// gathers its page ids); blocks from `batch` on zero the new pages (page i, layer l,
// pool k or v). Saves the scan launch and the separate zeroing launch of the two-kernel
// path; each block reads the start positions of the sequences before it and the whole
// update list, so it is used up to kFusedMaxBatch sequences and kFusedMaxUpdates table
// changes (the steady state of a decode batch: a few new pages per step). The first step
// of a batch, which uploads whole tables, takes the two-kernel path.
constexpr int kFusedMaxBatch = 128;
constexpr int kFusedMaxUpdates = 256;   // every block scans the update list
constexpr int kFusedThreads = 128;

struct ZeroParams {
  const int32_t* pages;
  int n, layers;
  uint8_t *pool0, *pool1;
  int64_t num_pages, layer_stride, page_bytes;
};

// The host arrays of a decode step small enough to travel in the launch itself (kernel
// parameter space, read in place through a __grid_constant__ parameter): the kernel then
// reads no host memory, where each dependent read of mapped staging is a PCIe round trip.
// Sized so that the fused kernel's parameters stay within the classic 4 KiB.
constexpr int kInlineBatch = 128;
constexpr int kInlineUpdates = 192;
constexpr int kInlineZero = 96;
struct PlanInline {
  int32_t slots[kInlineBatch];
  int32_t starts[kInlineBatch];
  int32_t updates[3 * kInlineUpdates];
  int32_t zero[kInlineZero];
};

__global__ void __launch_bounds__(kFusedThreads) plan_decode_fused_kernel(
    const PlanParams p, const ZeroParams z, const __grid_constant__ PlanInline in,
    const int use_inline) {
  // launched with programmatic dependent launch: nothing is read or written before the
  // previous kernel on the stream (which may still read the plan being replaced) is done
  pdl_wait();
  pdl_trigger();
  const int t = threadIdx.x;
  const int32_t* slots = use_inline ? in.slots : p.slots;
  const int32_t* starts = use_inline ? in.starts : p.starts;
  const int32_t* updates = use_inline ? in.updates : p.updates;
  const int32_t* zero = use_inline ? in.zero : z.pages;
  if (static_cast<int>(blockIdx.x) >= p.batch) {
    // ---- page zeroing
    const int zb = blockIdx.x - p.batch;
    const int pool = zb & 1, rest = zb >> 1;
    const int l = rest % z.layers, i = rest / z.layers;
    const int pg = zero[i];
    if (pg < 0 || pg >= z.num_pages) {
      if (t == 0 && l == 0 && pool == 0) report(p.status, NSLG_DEV_BAD_PLAN);
      return;
    }
    uint4* dst = reinterpret_cast<uint4*>((pool ? z.pool1 : z.pool0) + l * z.layer_stride +
                                          pg * z.page_bytes);
    const int64_t nv = z.page_bytes / 16;
    for (int64_t v = t; v < nv; v += kFusedThreads) dst[v] = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  // ---- sequence b
  __shared__ int32_t warp_sums[kFusedThreads / 32];
  const int b = blockIdx.x;
  const int s = slots[b];
  const int pos = starts[b];
  const bool row_ok = s >= 0 && s < p.bt_rows;
  int part = 0;
  for (int j = t; j < b; j += kFusedThreads) part += starts[j] / p.page_size + 1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if ((t & 31) == 0) warp_sums[t >> 5] = part;
  // this row's table changes
  for (int i = t; i < p.num_updates; i += kFusedThreads) {
    if (updates[3 * i] != s) continue;
    const int j = updates[3 * i + 1], pg = updates[3 * i + 2];
    if (row_ok && j >= 0 && j < p.bt_stride)
      p.bt[s * p.bt_stride + j] = pg;
    else
      report(p.status, NSLG_DEV_BAD_PLAN);
  }
  __syncthreads();
  int run = 0;
#pragma unroll
  for (int w = 0; w < kFusedThreads / 32; ++w) run += warp_sums[w];
  const int n = pos / p.page_size + 1;    // ceil((pos + 1) / page_size)
  const bool fits = row_ok && n <= p.bt_stride && run + n <= p.max_indices;
  if (t == 0) {
    const int pi = pos / p.page_size;
    p.positions[b] = pos;
    p.write_loc[b] = fits ? p.bt[s * p.bt_stride + pi] * p.page_size + pos % p.page_size : -1;
    p.lpl[b] = pos + 1 - (n - 1) * p.page_size;
    p.qo[b] = b;
    p.row_start[b] = b;
    p.indptr[b] = run;
    if (b == p.batch - 1) {
      p.indptr[p.batch] = run + n;
      p.qo[p.batch] = p.batch;
    }
    if (!fits) report(p.status, NSLG_DEV_BAD_PLAN);
  }
  if (!fits) return;
  const int32_t* row = p.bt + s * p.bt_stride;
  for (int j = t; j < n; j += kFusedThreads) p.indices[run + j] = row[j];
}

// Split-heads plan: sequence b' = b * hkv + h of the split-heads decode is kv head h of
// sequence b, with b's pages, its last-page length, and page ids page * hkv + h (the
// decode kernel takes the head from the id). Block b' writes its pages; the CSR offsets
// follow from kv_indptr alone: v_indptr[b * hkv + h] = hkv * kv_indptr[b] + h * n_b.
__global__ void __launch_bounds__(128) split_heads_plan_kernel(
    int batch, int hkv, const int32_t* kv_indptr, const int32_t* kv_indices,
    const int32_t* kv_lpl, int32_t* v_indptr, int32_t* v_indices, int32_t* v_lpl,
    int64_t max_v, uint32_t* status) {
  pdl_wait();
  pdl_trigger();
  const int bv = blockIdx.x, b = bv / hkv, h = bv % hkv;
  const int beg = kv_indptr[b], n = kv_indptr[b + 1] - beg;
  const int64_t vbeg = static_cast<int64_t>(hkv) * beg + static_cast<int64_t>(h) * n;
  if (threadIdx.x == 0) {
    v_indptr[bv] = static_cast<int32_t>(vbeg);
    v_lpl[bv] = kv_lpl[b];
    if (bv == batch * hkv - 1) v_indptr[batch * hkv] = hkv * kv_indptr[batch];
  }
  if (n < 0 || vbeg + n > max_v) {
    if (threadIdx.x == 0) report(status, NSLG_DEV_BAD_PLAN);
    return;
  }
  for (int j = threadIdx.x; j < n; j += blockDim.x)
    v_indices[vbeg + j] = kv_indices[beg + j] * hkv + h;
}

int check_plan_args(int batch, int page_size, int64_t bt_stride, int64_t bt_rows,
                    int num_updates, int64_t max_indices) {
  if (batch < 1 || batch > kScanThreads * kMaxItems)
    return set_error(NSLG_ERR_UNSUPPORTED, "plan_decode: batch must be in [1, 4096]");
  if (page_size <= 0 || bt_stride <= 0 || bt_rows <= 0 || num_updates < 0 || max_indices < 1)
    return set_error(NSLG_ERR_ARG, "plan_decode: bad sizes");
  if (bt_rows * bt_stride >= (int64_t{1} << 31))
    return set_error(NSLG_ERR_UNSUPPORTED, "plan_decode: block tables larger than 2^31 entries");
  return NSLG_OK;
}

int check_zero_args(int n, const void* pool, int64_t layers, int64_t num_pages,
                    int64_t page_bytes) {
  if (n < 0 || layers <= 0 || num_pages <= 0 || page_bytes <= 0 || page_bytes % 16 ||
      layers > 65535)
    return set_error(NSLG_ERR_ARG, "zero_pages: bad sizes");
  if (!pool || (reinterpret_cast<uintptr_t>(pool) & 15u))
    return set_error(NSLG_ERR_ARG, "zero_pages: null or misaligned pointer");
  return NSLG_OK;
}

int launch_plan(const PlanParams& p, cudaStream_t st) {
  plan_decode_scan_kernel<<<1, kScanThreads, 0, st>>>(p);
  int rc = check_launch("plan_decode_scan");
  if (rc != NSLG_OK) return rc;
  plan_decode_gather_kernel<<<p.batch, 128, 0, st>>>(p);
  return check_launch("plan_decode_gather");
}

// Pinned, device-mapped staging of nslg_plan_decode_host: kStageSlots slots per device,
// used round robin; a slot's event is recorded after the kernels that read it, and the
// slot is written again only once that event has completed.
constexpr int kMaxDevices = 64;
constexpr int kStageSlots = 8;
struct StageSlot {
  int32_t* host = nullptr;
  size_t cap = 0;              // int32 entries
  cudaEvent_t done = nullptr;
  bool pending = false;
};
struct DeviceStage {
  std::mutex mu;
  StageSlot slot[kStageSlots];
  int next = 0;
};
DeviceStage g_stage[kMaxDevices];

}  // namespace
}  // namespace nslg

using namespace nslg;

extern "C" int nslg_zero_pages(const int32_t* pages, int num_pages_to_zero, void* pool,
                               int64_t layers, int64_t num_pages, int64_t page_bytes,
                               uint32_t* dev_status, void* stream) {
  if (num_pages_to_zero == 0) return NSLG_OK;
  int rc = check_zero_args(num_pages_to_zero, pool, layers, num_pages, page_bytes);
  if (rc != NSLG_OK) return rc;
  if (!pages) return set_error(NSLG_ERR_ARG, "zero_pages: null or misaligned pointer");
  uint8_t* p8 = static_cast<uint8_t*>(pool);
  zero_pages_kernel<<<dim3(num_pages_to_zero, static_cast<unsigned>(layers), 1), 256, 0,
                      static_cast<cudaStream_t>(stream)>>>(
      pages, num_pages_to_zero, p8, p8, num_pages, num_pages * page_bytes, page_bytes,
      dev_status);
  return check_launch("zero_pages");
}

extern "C" int nslg_plan_decode(int batch, int page_size, const int32_t* slots,
                                const int32_t* starts, int num_updates, const int32_t* updates,
                                int32_t* block_tables, int64_t bt_stride, int64_t bt_rows,
                                int32_t* positions, int32_t* write_loc, int32_t* kv_indptr,
                                int32_t* kv_last_page_len, int32_t* qo_indptr,
                                int32_t* q_row_start, int32_t* kv_indices, int64_t max_indices,
                                uint32_t* dev_status, void* stream) {
  int rc = check_plan_args(batch, page_size, bt_stride, bt_rows, num_updates, max_indices);
  if (rc != NSLG_OK) return rc;
  if (!slots || !starts || (num_updates && !updates) || !block_tables || !positions ||
      !write_loc || !kv_indptr || !kv_last_page_len || !qo_indptr || !q_row_start || !kv_indices)
    return set_error(NSLG_ERR_ARG, "plan_decode: null pointer");
  PlanParams p{batch, page_size, num_updates, slots, starts, updates, block_tables, bt_stride,
               bt_rows, positions, write_loc, kv_indptr, kv_last_page_len, qo_indptr,
               q_row_start, kv_indices, max_indices, dev_status};
  return launch_plan(p, static_cast<cudaStream_t>(stream));
}

extern "C" int nslg_plan_decode_host(int batch, int page_size, const int32_t* slots,
                                     const int32_t* starts, int num_updates,
                                     const int32_t* updates, int num_zero,
                                     const int32_t* zero_pages, void* pool_k, void* pool_v,
                                     int64_t layers, int64_t num_pages, int64_t page_bytes,
                                     int32_t* block_tables, int64_t bt_stride, int64_t bt_rows,
                                     int32_t* plan, int64_t max_indices, uint32_t* dev_status,
                                     void* stream) {
  int rc = check_plan_args(batch, page_size, bt_stride, bt_rows, num_updates, max_indices);
  if (rc != NSLG_OK) return rc;
  if (!slots || !starts || (num_updates && !updates) || !block_tables || !plan)
    return set_error(NSLG_ERR_ARG, "plan_decode_host: null pointer");
  if (num_zero < 0) return set_error(NSLG_ERR_ARG, "zero_pages: bad sizes");
  if (num_zero) {
    if (!zero_pages) return set_error(NSLG_ERR_ARG, "plan_decode_host: null pointer");
    rc = check_zero_args(num_zero, pool_k, layers, num_pages, page_bytes);
    if (rc == NSLG_OK) rc = check_zero_args(num_zero, pool_v, layers, num_pages, page_bytes);
    if (rc != NSLG_OK) return rc;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaError_t err = cudaStreamIsCapturing(st, &cs);
  if (err != cudaSuccess) return set_error(NSLG_ERR_CUDA, cudaGetErrorString(err));
  if (cs != cudaStreamCaptureStatusNone)
    return set_error(NSLG_ERR_UNSUPPORTED,
                     "plan_decode_host: reads host staging, cannot be captured in a graph");
  const int64_t B = batch;
  const int64_t zero_blocks = static_cast<int64_t>(num_zero) * layers * 2;
  if (batch <= kInlineBatch && num_updates <= kInlineUpdates && num_zero <= kInlineZero &&
      zero_blocks < (int64_t{1} << 24)) {
    // the step's host arrays go with the launch: no staging slot, no host memory read
    static_assert(sizeof(PlanParams) + sizeof(ZeroParams) + sizeof(PlanInline) + 16 <= 4096,
                  "plan_decode_fused_kernel parameters must fit 4 KiB");
    PlanInline in;
    std::memcpy(in.slots, slots, sizeof(int32_t) * batch);
    std::memcpy(in.starts, starts, sizeof(int32_t) * batch);
    if (num_updates) std::memcpy(in.updates, updates, sizeof(int32_t) * 3 * num_updates);
    if (num_zero) std::memcpy(in.zero, zero_pages, sizeof(int32_t) * num_zero);
    PlanParams p{batch, page_size, num_updates, nullptr, nullptr, nullptr, block_tables,
                 bt_stride, bt_rows, plan, plan + B, plan + 2 * B, plan + 3 * B + 1,
                 plan + 4 * B + 1, plan + 5 * B + 2, plan + 6 * B + 2, max_indices, dev_status};
    ZeroParams z{nullptr, num_zero, static_cast<int>(layers), static_cast<uint8_t*>(pool_k),
                 static_cast<uint8_t*>(pool_v), num_pages, num_pages * page_bytes, page_bytes};
    return launch_pdl("plan_decode_fused", plan_decode_fused_kernel,
                      dim3(static_cast<unsigned>(batch + zero_blocks)), dim3(kFusedThreads), 0,
                      st, p, z, in, 1);
  }

  int dev = 0;
  err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return set_error(NSLG_ERR_CUDA, cudaGetErrorString(err));
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(NSLG_ERR_UNSUPPORTED, "plan_decode_host: device index >= 64");

  const size_t need = 2 * static_cast<size_t>(batch) + 3 * static_cast<size_t>(num_updates) +
                      static_cast<size_t>(num_zero);
  DeviceStage& ds = g_stage[dev];
  std::lock_guard<std::mutex> lock(ds.mu);
  StageSlot& sl = ds.slot[ds.next];
  if (sl.pending) {
    err = cudaEventSynchronize(sl.done);   // the kernels of kStageSlots calls ago
    if (err != cudaSuccess)
      return set_error(NSLG_ERR_CUDA, std::string("plan_decode_host: ") + cudaGetErrorString(err));
    sl.pending = false;
  }
  if (sl.done == nullptr) {
    err = cudaEventCreateWithFlags(&sl.done, cudaEventDisableTiming);
    if (err != cudaSuccess) return set_error(NSLG_ERR_CUDA, cudaGetErrorString(err));
  }
  if (sl.cap < need) {
    if (sl.host) cudaFreeHost(sl.host);
    sl.host = nullptr;
    sl.cap = 0;
    size_t cap = need > 16384 ? need : 16384;
    err = cudaHostAlloc(reinterpret_cast<void**>(&sl.host), cap * sizeof(int32_t),
                        cudaHostAllocMapped | cudaHostAllocPortable);
    if (err != cudaSuccess)
      return set_error(NSLG_ERR_CUDA, std::string("plan_decode_host: cudaHostAlloc: ") +
                                          cudaGetErrorString(err));
    sl.cap = cap;
  }
  int32_t* h = sl.host;
  std::memcpy(h, slots, sizeof(int32_t) * batch);
  std::memcpy(h + batch, starts, sizeof(int32_t) * batch);
  if (num_updates) std::memcpy(h + 2 * batch, updates, sizeof(int32_t) * 3 * num_updates);
  if (num_zero) std::memcpy(h + 2 * batch + 3 * num_updates, zero_pages, sizeof(int32_t) * num_zero);
  int32_t* d = nullptr;   // the same memory as the device sees it (UVA: normally h)
  err = cudaHostGetDevicePointer(reinterpret_cast<void**>(&d), h, 0);
  if (err != cudaSuccess) return set_error(NSLG_ERR_CUDA, cudaGetErrorString(err));

  PlanParams p{batch, page_size, num_updates, d, d + batch,
               num_updates ? d + 2 * batch : nullptr, block_tables, bt_stride, bt_rows, plan,
               plan + B, plan + 2 * B, plan + 3 * B + 1, plan + 4 * B + 1, plan + 5 * B + 2,
               plan + 6 * B + 2, max_indices, dev_status};
  if (batch <= kFusedMaxBatch && num_updates <= kFusedMaxUpdates &&
      zero_blocks < (int64_t{1} << 24)) {
    ZeroParams z{d + 2 * batch + 3 * num_updates, num_zero, static_cast<int>(layers),
                 static_cast<uint8_t*>(pool_k), static_cast<uint8_t*>(pool_v), num_pages,
                 num_pages * page_bytes, page_bytes};
    static const PlanInline unused{};
    rc = launch_pdl("plan_decode_fused", plan_decode_fused_kernel,
                    dim3(static_cast<unsigned>(batch + zero_blocks)), dim3(kFusedThreads), 0, st,
                    p, z, unused, 0);
  } else {
    if (num_zero) {
      zero_pages_kernel<<<dim3(num_zero, static_cast<unsigned>(layers), 2), 256, 0, st>>>(
          d + 2 * batch + 3 * num_updates, num_zero, static_cast<uint8_t*>(pool_k),
          static_cast<uint8_t*>(pool_v), num_pages, num_pages * page_bytes, page_bytes,
          dev_status);
      rc = check_launch("zero_pages");
    }
    if (rc == NSLG_OK) rc = launch_plan(p, st);
  }
  // whatever was launched may still read the slot: it is handed out again only after this
  err = cudaEventRecord(sl.done, st);
  if (err == cudaSuccess) {
    sl.pending = true;
    ds.next = (ds.next + 1) % kStageSlots;
  } else if (rc == NSLG_OK) {
    rc = set_error(NSLG_ERR_CUDA, cudaGetErrorString(err));
  }
  return rc;
}

extern "C" int nslg_split_heads_plan(int batch, int num_kv_heads, const int32_t* kv_indptr,
                                     const int32_t* kv_indices,
                                     const int32_t* kv_last_page_len, int32_t* v_indptr,
                                     int32_t* v_indices, int32_t* v_last_page_len,
                                     int64_t max_v_indices, int64_t num_pages,
                                     uint32_t* dev_status, void* stream) {
  if (batch < 0 || num_kv_heads < 1 || max_v_indices < 1 || num_pages < 1)
    return set_error(NSLG_ERR_ARG, "split_heads_plan: bad sizes");
  if (batch == 0) return NSLG_OK;
  if (static_cast<int64_t>(batch) * num_kv_heads > (int64_t{1} << 20) ||
      num_pages * num_kv_heads >= (int64_t{1} << 31))
    return set_error(NSLG_ERR_UNSUPPORTED, "split_heads_plan: too many sequences or pages");
  if (!kv_indptr || !kv_indices || !kv_last_page_len || !v_indptr || !v_indices ||
      !v_last_page_len)
    return set_error(NSLG_ERR_ARG, "split_heads_plan: null pointer");
  return launch_pdl("split_heads_plan", split_heads_plan_kernel,
                    dim3(static_cast<unsigned>(batch * num_kv_heads)), dim3(128), 0,
                    static_cast<cudaStream_t>(stream), batch, num_kv_heads, kv_indptr,
                    kv_indices, kv_last_page_len, v_indptr, v_indices, v_last_page_len,
                    max_v_indices, dev_status);
}
