// Greedy sampling of the LM head: per row of logits, the maximum and the index of its
// first occurrence, with torch.argmax's ordering (NaN above every number, ties to the
// lowest index). Replaces `logits[:, -1].argmax(-1)` (worker.py greedy path on the
// all-gathered logits of tp_layers.py:89); with a vocab-parallel LM head every rank
// reduces its own shard (index_offset = its first vocabulary id) and only the
// (maximum, index) pairs cross the TP group.
//
// One CTA per row: every thread streams 16-byte vectors of the row (all loads of a
// thread independent, so a CTA keeps many in flight), keeps its best (value, index) in
// visiting order, then a warp-shuffle and a shared-memory reduction pick the row's best.
#include <string>

#include "common.cuh"
#include "launch.h"

namespace nslg {
namespace {

constexpr int kArgmaxThreads = 1024;

// (a, ai) ranks before (b, bi)
__device__ __forceinline__ bool ranks_before(float a, int ai, float b, int bi) {
  const bool an = isnan(a), bn = isnan(b);
  if (an != bn) return an;
  if (!an && a != b) return a > b;
  return ai < bi;
}

template <typename T>
__global__ void __launch_bounds__(kArgmaxThreads) argmax_rows_kernel(
    const T* __restrict__ x, int64_t stride, int cols, int64_t index_offset, int vec_ok,
    float* out_val, int64_t* out_idx) {
  constexpr int VEC = 16 / sizeof(T);
  const T* xr = x + static_cast<int64_t>(blockIdx.x) * stride;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  if (vec_ok) {
    const int nv = cols / VEC;
    const uint4* xv = reinterpret_cast<const uint4*>(xr);
#pragma unroll 4
    for (int v = threadIdx.x; v < nv; v += blockDim.x) {
      union {
        uint4 u;
        T e[VEC];
      } w;
      w.u = __ldg(xv + v);
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float f = Elem<T>::to_f(w.e[j]);
        if (ranks_before(f, v * VEC + j, best, bi)) { best = f; bi = v * VEC + j; }
      }
    }
  } else {
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
      const float f = Elem<T>::to_f(xr[c]);
      if (ranks_before(f, c, best, bi)) { best = f; bi = c; }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ranks_before(ov, oi, best, bi)) { best = ov; bi = oi; }
  }
  __shared__ float s_val[kArgmaxThreads / 32];
  __shared__ int s_idx[kArgmaxThreads / 32];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) { s_val[warp] = best; s_idx[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x / 32;
    best = lane < nw ? s_val[lane] : -INFINITY;
    bi = lane < nw ? s_idx[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ranks_before(ov, oi, best, bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) {
      if (out_val) out_val[blockIdx.x] = best;
      out_idx[blockIdx.x] = static_cast<int64_t>(bi) + index_offset;
    }
  }
}

}  // namespace
}  // namespace nslg

using namespace nslg;

extern "C" int nslg_argmax_rows(int dtype, int rows, int cols, const void* x, int64_t x_stride,
                                int64_t index_offset, float* out_val, int64_t* out_idx,
                                void* stream) {
  if (dtype != NSLG_DTYPE_BF16 && dtype != NSLG_DTYPE_F16 && dtype != NSLG_DTYPE_F32)
    return set_error(NSLG_ERR_ARG, "argmax_rows: bad dtype");
  if (rows < 0 || cols <= 0 || x_stride < cols)
    return set_error(NSLG_ERR_ARG, "argmax_rows: bad shape");
  if (rows == 0) return NSLG_OK;
  if (!x || !out_idx) return set_error(NSLG_ERR_ARG, "argmax_rows: null pointer");
  const int esz = dtype_bytes(dtype);
  const int vec_ok = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && ((x_stride * esz) % 16 == 0) &&
                     ((static_cast<int64_t>(cols) * esz) % 16 == 0);
  int threads = kArgmaxThreads;
  const int work = vec_ok ? cols / (16 / esz) : cols;
  while (threads > 32 && threads / 2 >= work) threads /= 2;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == NSLG_DTYPE_BF16)
    argmax_rows_kernel<__nv_bfloat16><<<rows, threads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), x_stride, cols, index_offset, vec_ok, out_val,
        out_idx);
  else if (dtype == NSLG_DTYPE_F16)
    argmax_rows_kernel<__half><<<rows, threads, 0, st>>>(static_cast<const __half*>(x), x_stride,
                                                         cols, index_offset, vec_ok, out_val,
                                                         out_idx);
  else
    argmax_rows_kernel<float><<<rows, threads, 0, st>>>(static_cast<const float*>(x), x_stride,
                                                        cols, index_offset, vec_ok, out_val,
                                                        out_idx);
  return check_launch("argmax_rows");
}
