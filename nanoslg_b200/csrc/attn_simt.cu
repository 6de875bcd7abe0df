// Paged attention on CUDA cores: one warp per (query row, query head), online softmax
// in fp32 over the row's visible kv positions, lanes splitting head_dim.
//
// This is the kernel for the fp32 model (the tiny config is fp32 end to end, and a
// tf32 tensor-core path would change its greedy tokens) and for shapes the
// tensor-core kernels do not cover (head_dim other than 128, page size other than 16,
// more than 8 kv heads). Decode is the qo_len == 1 case of the same kernel.
//
// Semantics (kv_cache.py:192-224 and 312-322): row i of sequence b sits at absolute
// position kv_len - qo_len + i and, with causal != 0, sees kv positions <= that
// position; kv position j of sequence b lives in page kv_indices[kv_indptr[b] + j / P]
// at slot j % P.
#include "common.cuh"
#include "launch.h"

namespace nslg {
namespace {

struct SimtParams {
  const void* q;
  void* out;
  const void* pool_k;
  const void* pool_v;
  const int32_t* qo_indptr;
  const int32_t* q_row_start;
  const int32_t* kv_indptr;
  const int32_t* kv_indices;
  const int32_t* kv_lpl;
  int64_t q_stride, out_stride, num_pages;
  int batch, hq, hkv, d, page_size, causal;
  float sm_scale;
  uint32_t* status;
};

template <typename T, int DV>
__global__ void __launch_bounds__(128) paged_attn_simt_kernel(const SimtParams p) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int h = blockIdx.x * 4 + warp;
  const int i = blockIdx.y;
  const int b = blockIdx.z;
  if (h >= p.hq) return;
  // qo_indptr == NULL: decode, one query row per sequence (row b)
  const int qo_len = p.qo_indptr != nullptr ? p.qo_indptr[b + 1] - p.qo_indptr[b] : 1;
  if (i >= qo_len) return;
  const int kv_beg = p.kv_indptr[b];
  const int np = p.kv_indptr[b + 1] - kv_beg;
  const int kv_len = np > 0 ? (np - 1) * p.page_size + p.kv_lpl[b] : 0;
  const int qpos = kv_len - qo_len + i;
  const int limit = p.causal ? min(kv_len, qpos + 1) : kv_len;
  const int64_t row =
      static_cast<int64_t>(p.q_row_start   ? p.q_row_start[b]
                           : p.qo_indptr ? p.qo_indptr[b]
                                         : b) +
      i;
  const int kvh = h / (p.hq / p.hkv);
  const int d0 = lane * DV;  // head_dim == 32 * DV: every lane owns DV dims

  float qv[DV], acc[DV];
  const T* qp = static_cast<const T*>(p.q) + row * p.q_stride + static_cast<int64_t>(h) * p.d;
#pragma unroll
  for (int e = 0; e < DV; ++e) {
    qv[e] = Elem<T>::to_f(qp[d0 + e]);
    acc[e] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const T* pk = static_cast<const T*>(p.pool_k);
  const T* pv = static_cast<const T*>(p.pool_v);
  for (int j = 0; j < limit; ++j) {
    int page = p.kv_indices[kv_beg + j / p.page_size];
    if (page < 0 || page >= p.num_pages) {
      if (lane == 0 && h == 0 && i == 0) report(p.status, NSLG_DEV_BAD_PAGE);
      continue;
    }
    const int64_t off =
        ((static_cast<int64_t>(page) * p.page_size + j % p.page_size) * p.hkv + kvh) * p.d + d0;
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < DV; ++e) s = fmaf(qv[e], Elem<T>::to_f(pk[off + e]), s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    s *= p.sm_scale;
    const float m_new = fmaxf(m, s);
    const float alpha = expf(m - m_new);
    const float pw = expf(s - m_new);
    l = l * alpha + pw;
#pragma unroll
    for (int e = 0; e < DV; ++e) acc[e] = fmaf(pw, Elem<T>::to_f(pv[off + e]), acc[e] * alpha);
    m = m_new;
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  T* op = static_cast<T*>(p.out) + row * p.out_stride + static_cast<int64_t>(h) * p.d;
#pragma unroll
  for (int e = 0; e < DV; ++e) op[d0 + e] = Elem<T>::from_f(acc[e] * inv);
}

template <typename T>
int launch_typed(const SimtParams& p, int max_qo_len, cudaStream_t stream) {
  dim3 grid((p.hq + 3) / 4, max_qo_len, p.batch);
  if (p.d % 32 != 0) return set_error(NSLG_ERR_UNSUPPORTED, "paged attention: head_dim % 32");
  const int dv = p.d / 32;
  switch (dv) {
    case 1: paged_attn_simt_kernel<T, 1><<<grid, 128, 0, stream>>>(p); break;
    case 2: paged_attn_simt_kernel<T, 2><<<grid, 128, 0, stream>>>(p); break;
    case 3: paged_attn_simt_kernel<T, 3><<<grid, 128, 0, stream>>>(p); break;
    case 4: paged_attn_simt_kernel<T, 4><<<grid, 128, 0, stream>>>(p); break;
    case 5: paged_attn_simt_kernel<T, 5><<<grid, 128, 0, stream>>>(p); break;
    case 6: paged_attn_simt_kernel<T, 6><<<grid, 128, 0, stream>>>(p); break;
    case 7: paged_attn_simt_kernel<T, 7><<<grid, 128, 0, stream>>>(p); break;
    case 8: paged_attn_simt_kernel<T, 8><<<grid, 128, 0, stream>>>(p); break;
    default: return set_error(NSLG_ERR_UNSUPPORTED, "paged attention: head_dim > 256");
  }
  return check_launch("paged_attn_simt");
}

}  // namespace

int launch_paged_attention_simt(int dtype, int batch, int hq, int hkv, int d, int page_size,
                                const void* q, int64_t q_stride, void* out,
                                int64_t out_stride, const int32_t* qo_indptr,
                                const int32_t* q_row_start, int max_qo_len,
                                const void* pool_k, const void* pool_v, int64_t num_pages,
                                const int32_t* kv_indptr, const int32_t* kv_indices,
                                const int32_t* kv_last_page_len, float sm_scale, int causal,
                                uint32_t* status, cudaStream_t stream) {
  if (batch == 0 || max_qo_len == 0) return NSLG_OK;
  SimtParams p{q,         out,        pool_k,     pool_v,           qo_indptr, q_row_start,
               kv_indptr, kv_indices, kv_last_page_len, q_stride,   out_stride, num_pages,
               batch,     hq,         hkv,        d,                page_size, causal,
               sm_scale,  status};
  if (dtype == NSLG_DTYPE_BF16) return launch_typed<__nv_bfloat16>(p, max_qo_len, stream);
  if (dtype == NSLG_DTYPE_F16) return launch_typed<__half>(p, max_qo_len, stream);
  return launch_typed<float>(p, max_qo_len, stream);
}

}  // namespace nslg
