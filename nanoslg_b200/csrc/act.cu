// SwiGLU activation of the MLP on a fused gate|up GEMM output.
//
// The reference computes F.silu(gate_proj(x)) * up_proj(x) (models.py:156-157) as two
// GEMMs and two elementwise kernels. With the gate and up weights stacked, one GEMM
// writes [rows, 2*I] (gate in columns [0, I), up in [I, 2I)) and this kernel produces
// silu(gate) * up with the reference's rounding points: silu in fp32 rounded to the
// activation type, then the product rounded again (bf16: silu from the hardware
// exponential and an approximate division, within the bf16 rounding). 16-byte vector
// loads and stores.
#include "common.cuh"
#include "launch.h"

namespace nslg {
namespace {

template <typename T, int VEC>
union AVec {
  uint4 u;
  T e[VEC];
};

template <typename T>
__global__ void __launch_bounds__(256) silu_mul_kernel(const T* gu, int64_t gu_stride, T* out,
                                                       int64_t out_stride, int rows, int inter) {
  pdl_wait();
  pdl_trigger();
  constexpr int VEC = 16 / sizeof(T);
  const int per_row = inter / VEC;
  const int64_t total = static_cast<int64_t>(rows) * per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / per_row;
    const int c = static_cast<int>(i % per_row) * VEC;
    AVec<T, VEC> g, u, y;
    g.u = *reinterpret_cast<const uint4*>(gu + r * gu_stride + c);
    u.u = *reinterpret_cast<const uint4*>(gu + r * gu_stride + inter + c);
#pragma unroll
    for (int j = 0; j < VEC; ++j) y.e[j] = swiglu<T>(g.e[j], u.e[j]);
    *reinterpret_cast<uint4*>(out + r * out_stride + c) = y.u;
  }
}

}  // namespace

int launch_silu_mul(int dtype, int rows, int inter, const void* gate_up, int64_t gu_stride,
                    void* out, int64_t out_stride, cudaStream_t stream) {
  if (rows == 0) return NSLG_OK;
  const int vec = 16 / dtype_bytes(dtype);
  const int64_t total = static_cast<int64_t>(rows) * (inter / vec);
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  const dim3 grid(static_cast<unsigned>(blocks));
  if (dtype == NSLG_DTYPE_BF16)
    return launch_pdl("silu_mul", silu_mul_kernel<__nv_bfloat16>, grid, dim3(threads), 0, stream,
                      static_cast<const __nv_bfloat16*>(gate_up), gu_stride,
                      static_cast<__nv_bfloat16*>(out), out_stride, rows, inter);
  if (dtype == NSLG_DTYPE_F16)
    return launch_pdl("silu_mul", silu_mul_kernel<__half>, grid, dim3(threads), 0, stream,
                      static_cast<const __half*>(gate_up), gu_stride, static_cast<__half*>(out),
                      out_stride, rows, inter);
  return launch_pdl("silu_mul", silu_mul_kernel<float>, grid, dim3(threads), 0, stream,
                    static_cast<const float*>(gate_up), gu_stride, static_cast<float*>(out),
                    out_stride, rows, inter);
}

}  // namespace nslg
