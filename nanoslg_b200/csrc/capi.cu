// extern "C" entry points declared in include/nslg_b200.h: argument validation,
// per-thread error messages, and the choice between the tensor-core kernels and the
// CUDA-core kernel for shapes the former do not cover.
#include <cuda_runtime.h>

#include <atomic>
#include <string>

#include "launch.h"

namespace nslg {

namespace {
thread_local std::string g_last_error;
std::atomic<int> g_sm_count[64];
}  // namespace

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

void clear_error() { g_last_error.clear(); }

int check_launch(const char* what) {
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess)
    return set_error(NSLG_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
  return NSLG_OK;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = g_sm_count[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_sm_count[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int esize(int dtype) { return dtype_bytes(dtype); }

bool valid_dtype(int dtype) {
  return dtype == NSLG_DTYPE_BF16 || dtype == NSLG_DTYPE_F16 || dtype == NSLG_DTYPE_F32;
}

int check_heads(const char* what, int hq, int hkv, int d) {
  if (hq <= 0 || hkv <= 0 || d <= 0 || hq % hkv != 0)
    return set_error(NSLG_ERR_ARG, std::string(what) + ": need num_qo_heads % num_kv_heads == 0");
  return NSLG_OK;
}

}  // namespace
}  // namespace nslg

using namespace nslg;

extern "C" {

const char* nslg_version(void) { return "nanoslg-b200 0.1 (sm_100a)"; }

const char* nslg_last_error(void) { return g_last_error.c_str(); }

int nslg_rope_kv_append(int dtype, int num_tokens, int num_qo_heads, int num_kv_heads,
                        int head_dim, const void* q, int64_t q_stride, const void* k,
                        int64_t k_stride, const void* v, int64_t v_stride, void* q_out,
                        const int32_t* positions, const float* cos_table,
                        const float* sin_table, int64_t table_rows, const int32_t* write_loc,
                        void* pool_k, void* pool_v, int64_t pool_slots, uint32_t* dev_status,
                        void* stream) {
  g_last_error.clear();
  if (!valid_dtype(dtype)) return set_error(NSLG_ERR_ARG, "rope_kv_append: bad dtype");
  if (num_tokens < 0) return set_error(NSLG_ERR_ARG, "rope_kv_append: num_tokens < 0");
  if (num_tokens == 0) return NSLG_OK;
  int rc = check_heads("rope_kv_append", num_qo_heads, num_kv_heads, head_dim);
  if (rc) return rc;
  const int vec = 16 / esize(dtype);
  if (head_dim % (2 * vec) != 0)
    return set_error(NSLG_ERR_UNSUPPORTED, "rope_kv_append: head_dim must be a multiple of " +
                                                std::to_string(2 * vec));
  if (k == nullptr || v == nullptr)
    return set_error(NSLG_ERR_ARG, "rope_kv_append: k and v are required");
  if (q_out != nullptr && q == nullptr)
    return set_error(NSLG_ERR_ARG, "rope_kv_append: q_out given without q");
  if (positions != nullptr && (cos_table == nullptr || sin_table == nullptr || table_rows <= 0))
    return set_error(NSLG_ERR_ARG, "rope_kv_append: positions need cos/sin tables");
  if (write_loc != nullptr && (pool_k == nullptr || pool_v == nullptr || pool_slots <= 0))
    return set_error(NSLG_ERR_ARG, "rope_kv_append: write_loc needs pool_k/pool_v");
  const int64_t es = esize(dtype);
  if ((q_out && (!aligned16(q) || !aligned16(q_out) || (q_stride * es) % 16)) || !aligned16(k) ||
      !aligned16(v) || (k_stride * es) % 16 || (v_stride * es) % 16 ||
      (pool_k && !aligned16(pool_k)) || (pool_v && !aligned16(pool_v)) ||
      (cos_table && !aligned16(cos_table)) || (sin_table && !aligned16(sin_table)))
    return set_error(NSLG_ERR_ARG, "rope_kv_append: pointers and row strides must be 16-byte aligned");
  return launch_rope_kv_append(dtype, num_tokens, num_qo_heads, num_kv_heads, head_dim, q,
                               q_stride, k, k_stride, v, v_stride, q_out, positions, cos_table,
                               sin_table, table_rows, write_loc, pool_k, pool_v, pool_slots,
                               dev_status, static_cast<cudaStream_t>(stream));
}

int64_t nslg_decode_workspace_bytes(int batch, int num_qo_heads, int head_dim) {
  if (batch < 0 || num_qo_heads <= 0 || head_dim <= 0) return 0;
  return decode_tc_workspace_bytes(batch, num_qo_heads, head_dim);
}

int nslg_paged_decode(int dtype, int batch, int num_qo_heads, int num_kv_heads, int head_dim,
                      int page_size, const void* q, int64_t q_stride, void* out,
                      int64_t out_stride, const void* pool_k, const void* pool_v,
                      int64_t num_pages, const int32_t* kv_indptr, const int32_t* kv_indices,
                      const int32_t* kv_last_page_len, float sm_scale, void* workspace,
                      int64_t workspace_bytes, uint32_t* dev_status, void* stream) {
  g_last_error.clear();
  if (!valid_dtype(dtype)) return set_error(NSLG_ERR_ARG, "paged_decode: bad dtype");
  if (batch < 0) return set_error(NSLG_ERR_ARG, "paged_decode: batch < 0");
  if (batch == 0) return NSLG_OK;
  int rc = check_heads("paged_decode", num_qo_heads, num_kv_heads, head_dim);
  if (rc) return rc;
  if (page_size <= 0 || num_pages <= 0)
    return set_error(NSLG_ERR_ARG, "paged_decode: page_size and num_pages must be positive");
  if (!q || !out || !pool_k || !pool_v || !kv_indptr || !kv_indices || !kv_last_page_len)
    return set_error(NSLG_ERR_ARG, "paged_decode: null pointer");
  if (!(sm_scale > 0.f)) return set_error(NSLG_ERR_ARG, "paged_decode: sm_scale must be > 0");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (decode_tc_supported(dtype, num_qo_heads, num_kv_heads, head_dim, page_size) &&
      aligned16(pool_k) && aligned16(pool_v) && (reinterpret_cast<uintptr_t>(q) & 3u) == 0 &&
      (reinterpret_cast<uintptr_t>(out) & 3u) == 0 && q_stride % 2 == 0 && out_stride % 2 == 0)
    return launch_paged_decode_tc(dtype, batch, num_qo_heads, num_kv_heads, head_dim, q, q_stride, out,
                                  out_stride, pool_k, pool_v, num_pages, kv_indptr, kv_indices,
                                  kv_last_page_len, sm_scale, workspace, workspace_bytes,
                                  dev_status, st);
  // decode is the one-row case of the general kernel (qo_indptr == NULL: row b of q is
  // the single query of sequence b)
  return launch_paged_attention_simt(dtype, batch, num_qo_heads, num_kv_heads, head_dim,
                                     page_size, q, q_stride, out, out_stride, nullptr, nullptr, 1,
                                     pool_k, pool_v, num_pages, kv_indptr, kv_indices,
                                     kv_last_page_len, sm_scale, 0, dev_status, st);
}

int nslg_paged_decode_split_heads(int dtype, int batch, int num_qo_heads, int num_kv_heads,
                                  int head_dim, int page_size, const void* q, void* out,
                                  const void* pool_k, const void* pool_v, int64_t num_pages,
                                  const int32_t* v_indptr, const int32_t* v_indices,
                                  const int32_t* v_last_page_len, float sm_scale,
                                  void* workspace, int64_t workspace_bytes,
                                  uint32_t* dev_status, void* stream) {
  g_last_error.clear();
  if (!valid_dtype(dtype)) return set_error(NSLG_ERR_ARG, "paged_decode_split_heads: bad dtype");
  if (batch < 0) return set_error(NSLG_ERR_ARG, "paged_decode_split_heads: batch < 0");
  if (batch == 0) return NSLG_OK;
  int rc = check_heads("paged_decode_split_heads", num_qo_heads, num_kv_heads, head_dim);
  if (rc) return rc;
  if (page_size <= 0 || num_pages <= 0)
    return set_error(NSLG_ERR_ARG, "paged_decode_split_heads: page_size and num_pages must be positive");
  if (!q || !out || !pool_k || !pool_v || !v_indptr || !v_indices || !v_last_page_len)
    return set_error(NSLG_ERR_ARG, "paged_decode_split_heads: null pointer");
  if (!(sm_scale > 0.f)) return set_error(NSLG_ERR_ARG, "paged_decode_split_heads: sm_scale must be > 0");
  const int group = num_qo_heads / num_kv_heads;
  if (num_kv_heads < 2 || static_cast<int64_t>(batch) * num_kv_heads > (int64_t{1} << 20) ||
      num_pages * num_kv_heads >= (int64_t{1} << 31) ||
      !decode_tc_supported(dtype, group, 1, head_dim, page_size) || !aligned16(pool_k) ||
      !aligned16(pool_v) || (reinterpret_cast<uintptr_t>(q) & 3u) ||
      (reinterpret_cast<uintptr_t>(out) & 3u))
    return set_error(NSLG_ERR_UNSUPPORTED,
                     "paged_decode_split_heads: needs the tensor-core decode path, 2 or more "
                     "kv heads and 4-byte aligned q / out");
  // sequence b * hkv + h: the group of query heads of kv head h of sequence b, rows of
  // group * head_dim elements in the contiguous [batch, num_qo_heads, head_dim] q / out
  const int64_t row = static_cast<int64_t>(group) * head_dim;
  return launch_paged_decode_tc(dtype, batch * num_kv_heads, group, 1, head_dim, q, row, out,
                                row, pool_k, pool_v, num_pages, v_indptr, v_indices,
                                v_last_page_len, sm_scale, workspace, workspace_bytes,
                                dev_status, static_cast<cudaStream_t>(stream), num_kv_heads);
}

int nslg_append_paged_decode(int dtype, int batch, int num_qo_heads, int num_kv_heads,
                             int head_dim, int page_size, const void* q, int64_t q_stride,
                             const void* k, int64_t k_stride, const void* v, int64_t v_stride,
                             const int32_t* write_loc, void* out, int64_t out_stride,
                             void* pool_k, void* pool_v, int64_t num_pages,
                             const int32_t* kv_indptr, const int32_t* kv_indices,
                             const int32_t* kv_last_page_len, float sm_scale, void* workspace,
                             int64_t workspace_bytes, uint32_t* dev_status, void* stream) {
  g_last_error.clear();
  if (batch < 0) return set_error(NSLG_ERR_ARG, "append_paged_decode: batch < 0");
  if (batch == 0) return NSLG_OK;
  if (!write_loc) return set_error(NSLG_ERR_ARG, "append_paged_decode: null write_loc");
  if (page_size <= 0 || num_pages <= 0)
    return set_error(NSLG_ERR_ARG, "append_paged_decode: page_size and num_pages must be positive");
  int rc = nslg_rope_kv_append(dtype, batch, num_kv_heads, num_kv_heads, head_dim, nullptr, 0, k,
                               k_stride, v, v_stride, nullptr, nullptr, nullptr, nullptr, 0,
                               write_loc, pool_k, pool_v, num_pages * page_size, dev_status,
                               stream);
  if (rc != NSLG_OK) return rc;
  return nslg_paged_decode(dtype, batch, num_qo_heads, num_kv_heads, head_dim, page_size, q,
                           q_stride, out, out_stride, pool_k, pool_v, num_pages, kv_indptr,
                           kv_indices, kv_last_page_len, sm_scale, workspace, workspace_bytes,
                           dev_status, stream);
}

int nslg_paged_prefill(int dtype, int batch, int num_qo_heads, int num_kv_heads, int head_dim,
                       int page_size, const void* q, int64_t q_stride, int64_t q_rows, void* out,
                       int64_t out_stride, const int32_t* qo_indptr, const int32_t* q_row_start,
                       int max_qo_len, const void* pool_k, const void* pool_v, int64_t num_pages,
                       const int32_t* kv_indptr, const int32_t* kv_indices,
                       const int32_t* kv_last_page_len, float sm_scale, int causal,
                       uint32_t* dev_status, void* stream) {
  g_last_error.clear();
  if (!valid_dtype(dtype)) return set_error(NSLG_ERR_ARG, "paged_prefill: bad dtype");
  if (batch < 0 || max_qo_len < 0)
    return set_error(NSLG_ERR_ARG, "paged_prefill: negative batch or max_qo_len");
  if (batch == 0 || max_qo_len == 0) return NSLG_OK;
  int rc = check_heads("paged_prefill", num_qo_heads, num_kv_heads, head_dim);
  if (rc) return rc;
  if (page_size <= 0 || num_pages <= 0)
    return set_error(NSLG_ERR_ARG, "paged_prefill: page_size and num_pages must be positive");
  if (!q || !out || !qo_indptr || !pool_k || !pool_v || !kv_indptr || !kv_indices ||
      !kv_last_page_len)
    return set_error(NSLG_ERR_ARG, "paged_prefill: null pointer");
  if (!(sm_scale > 0.f)) return set_error(NSLG_ERR_ARG, "paged_prefill: sm_scale must be > 0");
  if (max_qo_len > 65535) return set_error(NSLG_ERR_UNSUPPORTED, "paged_prefill: max_qo_len > 65535");
  if (q_rows <= 0) return set_error(NSLG_ERR_ARG, "paged_prefill: q_rows must be positive");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (prefill_tc_supported(dtype, num_qo_heads, num_kv_heads, head_dim, page_size) &&
      aligned16(q) && aligned16(out) && aligned16(pool_k) && aligned16(pool_v) &&
      (q_stride * 2) % 16 == 0 && (out_stride * 2) % 16 == 0)
    return launch_paged_prefill_tc(dtype, batch, num_qo_heads, num_kv_heads, q, q_stride, q_rows, out,
                                   out_stride, qo_indptr, q_row_start, max_qo_len, pool_k,
                                   pool_v, num_pages, kv_indptr, kv_indices, kv_last_page_len,
                                   sm_scale, causal, dev_status, st);
  return launch_paged_attention_simt(dtype, batch, num_qo_heads, num_kv_heads, head_dim,
                                     page_size, q, q_stride, out, out_stride, qo_indptr,
                                     q_row_start, max_qo_len, pool_k, pool_v, num_pages,
                                     kv_indptr, kv_indices, kv_last_page_len, sm_scale, causal,
                                     dev_status, st);
}

int nslg_rmsnorm_residual(int dtype, int rows, int hidden, const void* x, int64_t x_stride,
                          void* residual, int64_t residual_stride, const void* weight, void* out,
                          int64_t out_stride, float eps, void* stream) {
  g_last_error.clear();
  if (!valid_dtype(dtype)) return set_error(NSLG_ERR_ARG, "rmsnorm_residual: bad dtype");
  if (rows < 0 || hidden <= 0) return set_error(NSLG_ERR_ARG, "rmsnorm_residual: bad shape");
  if (rows == 0) return NSLG_OK;
  if (!x || !weight || !out) return set_error(NSLG_ERR_ARG, "rmsnorm_residual: null pointer");
  const int64_t es = esize(dtype);
  if ((hidden * es) % 16 || !aligned16(x) || !aligned16(weight) || !aligned16(out) ||
      (residual && !aligned16(residual)) || (x_stride * es) % 16 || (out_stride * es) % 16 ||
      (residual && (residual_stride * es) % 16))
    return set_error(NSLG_ERR_ARG, "rmsnorm_residual: rows must be 16-byte aligned");
  return launch_rmsnorm_residual(dtype, rows, hidden, x, x_stride, residual, residual_stride,
                                 weight, out, out_stride, eps, static_cast<cudaStream_t>(stream));
}

int nslg_silu_mul(int dtype, int rows, int inter, const void* gate_up, int64_t gate_up_stride,
                  void* out, int64_t out_stride, void* stream) {
  g_last_error.clear();
  if (!valid_dtype(dtype)) return set_error(NSLG_ERR_ARG, "silu_mul: bad dtype");
  if (rows < 0 || inter <= 0) return set_error(NSLG_ERR_ARG, "silu_mul: bad shape");
  if (rows == 0) return NSLG_OK;
  if (!gate_up || !out) return set_error(NSLG_ERR_ARG, "silu_mul: null pointer");
  const int64_t es = esize(dtype);
  if ((inter * es) % 16 || !aligned16(gate_up) || !aligned16(out) || (gate_up_stride * es) % 16 ||
      (out_stride * es) % 16)
    return set_error(NSLG_ERR_ARG, "silu_mul: rows must be 16-byte aligned");
  return launch_silu_mul(dtype, rows, inter, gate_up, gate_up_stride, out, out_stride,
                         static_cast<cudaStream_t>(stream));
}

int nslg_linear(int dtype, int rows, int out_features, int in_features, const void* x,
                int64_t x_stride, const void* weight, int64_t w_stride, void* y,
                int64_t y_stride, uint32_t* dev_status, void* stream) {
  g_last_error.clear();
  if (dtype != NSLG_DTYPE_BF16 && dtype != NSLG_DTYPE_F16)
    return set_error(NSLG_ERR_ARG, "linear: dtype must be bfloat16 or float16");
  if (rows < 0 || out_features <= 0 || in_features <= 0)
    return set_error(NSLG_ERR_ARG, "linear: bad shape");
  if (rows == 0) return NSLG_OK;
  if (!linear_tc_supported(dtype, rows, out_features, in_features))
    return set_error(NSLG_ERR_UNSUPPORTED, "linear: needs 1 <= rows <= " +
                                               std::to_string(kLinearMaxRows) +
                                               " and in_features a multiple of 64");
  if (!x || !weight || !y) return set_error(NSLG_ERR_ARG, "linear: null pointer");
  if (!aligned16(x) || !aligned16(weight) || (x_stride * 2) % 16 || (w_stride * 2) % 16 ||
      x_stride < in_features || w_stride < in_features || y_stride < out_features ||
      (reinterpret_cast<uintptr_t>(y) & 1u))
    return set_error(NSLG_ERR_ARG,
                     "linear: x and weight rows must be 16-byte aligned and strides cover the rows");
  return launch_linear_tc(dtype, rows, out_features, in_features, x, x_stride, weight, w_stride,
                          y, y_stride, nullptr, dev_status, static_cast<cudaStream_t>(stream));
}

int nslg_linear_swiglu(int dtype, int rows, int inter, int in_features, const void* x,
                       int64_t x_stride, const void* gate_up, int64_t w_stride, void* out,
                       int64_t out_stride, uint32_t* dev_status, void* stream) {
  g_last_error.clear();
  if (dtype != NSLG_DTYPE_BF16 && dtype != NSLG_DTYPE_F16)
    return set_error(NSLG_ERR_ARG, "linear_swiglu: dtype must be bfloat16 or float16");
  if (rows < 0 || inter <= 0 || in_features <= 0)
    return set_error(NSLG_ERR_ARG, "linear_swiglu: bad shape");
  if (rows == 0) return NSLG_OK;
  if (!linear_tc_supported(dtype, rows, inter, in_features) || inter > (1 << 22))
    return set_error(NSLG_ERR_UNSUPPORTED, "linear_swiglu: needs 1 <= rows <= " +
                                               std::to_string(kLinearMaxRows) +
                                               ", inter <= 4194304 and in_features a multiple of 64");
  if (!x || !gate_up || !out) return set_error(NSLG_ERR_ARG, "linear_swiglu: null pointer");
  if (!aligned16(x) || !aligned16(gate_up) || (x_stride * 2) % 16 || (w_stride * 2) % 16 ||
      x_stride < in_features || w_stride < in_features || out_stride < inter ||
      (reinterpret_cast<uintptr_t>(out) & 1u))
    return set_error(NSLG_ERR_ARG, "linear_swiglu: x and weight rows must be 16-byte aligned "
                                   "and strides cover the rows");
  return launch_linear_tc(dtype, rows, inter, in_features, x, x_stride, gate_up, w_stride, out,
                          out_stride, nullptr, dev_status, static_cast<cudaStream_t>(stream),
                          true);
}

int nslg_linear_rope_append(int dtype, int rows, int num_qo_heads, int num_kv_heads,
                            int head_dim, int in_features, const void* x, int64_t x_stride,
                            const void* w_qkv, int64_t w_stride, void* q_out,
                            const int32_t* positions, const float* cos_table,
                            const float* sin_table, int64_t table_rows,
                            const int32_t* write_loc, void* pool_k, void* pool_v,
                            int64_t pool_slots, uint32_t* dev_status, void* stream) {
  g_last_error.clear();
  if (dtype != NSLG_DTYPE_BF16 && dtype != NSLG_DTYPE_F16)
    return set_error(NSLG_ERR_ARG, "linear_rope_append: dtype must be bfloat16 or float16");
  if (rows < 0 || num_qo_heads <= 0 || num_kv_heads <= 0 || in_features <= 0 ||
      num_qo_heads > 4096 || num_kv_heads > 4096)
    return set_error(NSLG_ERR_ARG, "linear_rope_append: bad shape");
  if (rows == 0) return NSLG_OK;
  const int n = (num_qo_heads + 2 * num_kv_heads) * 128;
  if (head_dim != 128 || !linear_tc_supported(dtype, rows, n, in_features))
    return set_error(NSLG_ERR_UNSUPPORTED, "linear_rope_append: needs head_dim 128, 1 <= rows <= " +
                                               std::to_string(kLinearMaxRows) +
                                               " and in_features a multiple of 64");
  if (!x || !w_qkv || !q_out || !pool_k || !pool_v || (positions && (!cos_table || !sin_table)))
    return set_error(NSLG_ERR_ARG, "linear_rope_append: null pointer");
  if (!aligned16(x) || !aligned16(w_qkv) || !aligned16(q_out) || !aligned16(pool_k) ||
      !aligned16(pool_v) || (x_stride * 2) % 16 || (w_stride * 2) % 16 ||
      x_stride < in_features || w_stride < in_features)
    return set_error(NSLG_ERR_ARG, "linear_rope_append: x, weight, q_out and pool rows must be "
                                   "16-byte aligned and strides cover the rows");
  LinearRope r{};
  r.hq = num_qo_heads;
  r.hkv = num_kv_heads;
  r.q_out = q_out;
  r.positions = positions;
  r.cos_t = cos_table;
  r.sin_t = sin_table;
  r.table_rows = table_rows;
  r.write_loc = write_loc;
  r.pool_k = pool_k;
  r.pool_v = pool_v;
  r.pool_slots = pool_slots;
  return launch_linear_tc(dtype, rows, n, in_features, x, x_stride, w_qkv, w_stride, nullptr, n,
                          nullptr, dev_status, static_cast<cudaStream_t>(stream), false, &r);
}

int nslg_linear_tp_push(int dtype, int rows, int out_features, int in_features, const void* x,
                        int64_t x_stride, const void* weight, int64_t w_stride, void* y,
                        int64_t y_stride, int world, int rank, void* const* stage_bufs,
                        int64_t stage_bytes, const void* counters, uint32_t* dev_status,
                        void* stream) {
  g_last_error.clear();
  if (dtype != NSLG_DTYPE_BF16 && dtype != NSLG_DTYPE_F16)
    return set_error(NSLG_ERR_ARG, "linear_tp_push: dtype must be bfloat16 or float16");
  if (rows < 0 || out_features <= 0 || in_features <= 0)
    return set_error(NSLG_ERR_ARG, "linear_tp_push: bad shape");
  if (world < 2 || world > NSLG_TP_MAX_WORLD || rank < 0 || rank >= world)
    return set_error(NSLG_ERR_ARG, "linear_tp_push: need 2 <= world <= 8 and 0 <= rank < world");
  if (rows == 0) return NSLG_OK;
  if (!linear_tc_supported(dtype, rows, out_features, in_features))
    return set_error(NSLG_ERR_UNSUPPORTED, "linear_tp_push: needs 1 <= rows <= " +
                                               std::to_string(kLinearMaxRows) +
                                               " and in_features a multiple of 64");
  if (out_features % 8)
    return set_error(NSLG_ERR_ARG, "linear_tp_push: out_features must be a multiple of 8");
  if (!x || !weight || !y || !stage_bufs || !counters)
    return set_error(NSLG_ERR_ARG, "linear_tp_push: null pointer");
  if (!aligned16(x) || !aligned16(weight) || !aligned16(y) || !aligned16(counters) ||
      (x_stride * 2) % 16 || (w_stride * 2) % 16 || (y_stride * 2) % 16 ||
      x_stride < in_features || w_stride < in_features || y_stride < out_features)
    return set_error(NSLG_ERR_ARG,
                     "linear_tp_push: x, weight and y rows must be 16-byte aligned and strides "
                     "cover the rows");
  TpPush push{};
  int64_t region = 0, slot = 0;
  tp_stage_geometry(stage_bytes, world, &region, &slot);
  if (2 * static_cast<int64_t>(out_features) * 2 * rows > region)
    return set_error(NSLG_ERR_WORKSPACE, "linear_tp_push: " + std::to_string(rows) +
                                             " rows do not fit the stage buffers");
  for (int i = 0; i < world; ++i) {
    if (!stage_bufs[i] || !aligned16(stage_bufs[i]))
      return set_error(NSLG_ERR_ARG, "linear_tp_push: bad stage buffer");
    push.stage[i] = static_cast<uint8_t*>(stage_bufs[i]);
  }
  push.counters = static_cast<const uint32_t*>(counters);
  push.slot_bytes = slot;
  push.region_bytes = region;
  push.world = world;
  push.rank = rank;
  return launch_linear_tc(dtype, rows, out_features, in_features, x, x_stride, weight, w_stride,
                          y, y_stride, &push, dev_status, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
