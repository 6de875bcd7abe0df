// Fused residual add + RMSNorm, one CTA per row, 16-byte vector loads/stores.
//
// Rounding points follow the reference (models.py:31-34 and the residual adds at
// models.py:169-172): h = x + residual is rounded to the activation type, statistics are
// taken in fp32 on that rounded h, the normalised value is rounded to the activation
// type, and the weight multiply is one more rounded elementwise op.
#include "common.cuh"
#include "launch.h"

namespace nslg {
namespace {

struct NormParams {
  const void* x;
  void* residual;
  const void* weight;
  void* out;
  int64_t x_stride, r_stride, o_stride;
  int rows, hidden;
  float eps;
};

template <typename T, int VEC>
union NVec {
  uint4 u;
  T e[VEC];
};

// Vectors per thread kept in registers between the two passes (with their weights,
// loaded in the first pass): at hidden 4096 in bf16 (512 vectors, 256 threads) the
// second pass then reads no memory, one dependent L2 round trip less per row.
constexpr int kHeld = 4;

template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_residual_kernel(const NormParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int VEC = 16 / sizeof(T);
  const int row = blockIdx.x;
  const int nv = p.hidden / VEC;
  const int bd = blockDim.x;
  const T* x = static_cast<const T*>(p.x) + row * p.x_stride;
  T* res = p.residual != nullptr ? static_cast<T*>(p.residual) + row * p.r_stride : nullptr;
  const T* w = static_cast<const T*>(p.weight);
  T* out = static_cast<T*>(p.out) + row * p.o_stride;

  // h = x (+ residual, rounded; written back), sum of squares in the order i = t, t + bd, ..
  auto load_h = [&](int i, NVec<T, VEC>& a) {
    a.u = reinterpret_cast<const uint4*>(x)[i];
    if (res != nullptr) {
      NVec<T, VEC> r;
      r.u = reinterpret_cast<const uint4*>(res)[i];
#pragma unroll
      for (int j = 0; j < VEC; ++j)
        a.e[j] = Elem<T>::from_f(__fadd_rn(Elem<T>::to_f(a.e[j]), Elem<T>::to_f(r.e[j])));
      reinterpret_cast<uint4*>(res)[i] = a.u;
    }
  };
  float ss = 0.f;
  NVec<T, VEC> held[kHeld], wheld[kHeld];
#pragma unroll
  for (int k = 0; k < kHeld; ++k) {
    const int i = threadIdx.x + k * bd;
    if (i < nv) {
      load_h(i, held[k]);
      wheld[k].u = reinterpret_cast<const uint4*>(w)[i];
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float f = Elem<T>::to_f(held[k].e[j]);
        ss = fmaf(f, f, ss);
      }
    }
  }
  for (int i = threadIdx.x + kHeld * bd; i < nv; i += bd) {
    NVec<T, VEC> a;
    load_h(i, a);
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float f = Elem<T>::to_f(a.e[j]);
      ss = fmaf(f, f, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  __shared__ float red[32];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float v = lane < (bd + 31) / 32 ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  const float inv = rsqrtf(__fadd_rn(__fdiv_rn(red[0], static_cast<float>(p.hidden)), p.eps));

  auto norm_store = [&](int i, const NVec<T, VEC>& a, const NVec<T, VEC>& ww) {
    NVec<T, VEC> o;
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float y = Elem<T>::round(__fmul_rn(Elem<T>::to_f(a.e[j]), inv));
      o.e[j] = Elem<T>::from_f(__fmul_rn(Elem<T>::to_f(ww.e[j]), y));
    }
    reinterpret_cast<uint4*>(out)[i] = o.u;
  };
#pragma unroll
  for (int k = 0; k < kHeld; ++k) {
    const int i = threadIdx.x + k * bd;
    if (i < nv) norm_store(i, held[k], wheld[k]);
  }
  const T* h = res != nullptr ? res : x;
  for (int i = threadIdx.x + kHeld * bd; i < nv; i += bd) {
    NVec<T, VEC> a, ww;
    a.u = reinterpret_cast<const uint4*>(h)[i];
    ww.u = reinterpret_cast<const uint4*>(w)[i];
    norm_store(i, a, ww);
  }
}

}  // namespace

int launch_rmsnorm_residual(int dtype, int rows, int hidden, const void* x, int64_t x_stride,
                            void* residual, int64_t residual_stride, const void* weight,
                            void* out, int64_t out_stride, float eps, cudaStream_t stream) {
  if (rows == 0) return NSLG_OK;
  NormParams p{x, residual, weight, out, x_stride, residual_stride, out_stride, rows, hidden, eps};
  const int esz = dtype_bytes(dtype);
  const int nv = hidden * esz / 16;
  int threads = 32;
  while (threads < nv && threads < 256) threads *= 2;
  if (dtype == NSLG_DTYPE_BF16)
    return launch_pdl("rmsnorm_residual", rmsnorm_residual_kernel<__nv_bfloat16>, dim3(rows),
                      dim3(threads), 0, stream, p);
  if (dtype == NSLG_DTYPE_F16)
    return launch_pdl("rmsnorm_residual", rmsnorm_residual_kernel<__half>, dim3(rows),
                      dim3(threads), 0, stream, p);
  return launch_pdl("rmsnorm_residual", rmsnorm_residual_kernel<float>, dim3(rows),
                    dim3(threads), 0, stream, p);
}

}  // namespace nslg
