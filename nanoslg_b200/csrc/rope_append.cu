// Fused rotary embedding + paged KV append.
//
// One thread owns 16 bytes of a head row. For q and k it owns the matching 16 bytes
// of both halves of the row (rotate-half pairs dimension d with d + D/2), rotates
// them and stores them with 16-byte vector stores: q into q_out, k into the page
// slot the context assigned to the token. v is copied unrotated. The arithmetic
// repeats the reference's elementwise ops with their rounding points
// (models.py:79-83): cos/sin are first cast to the activation type, then
//   out = x*cos + cat(-x2, x1)*sin
// with every product and the sum rounded to the activation type. fp32 uses the
// explicitly rounded intrinsics so no fused multiply-add changes the result.
#include "common.cuh"
#include "launch.h"

namespace nslg {
namespace {

struct RopeParams {
  const void* q;
  const void* k;
  const void* v;
  void* q_out;
  const int32_t* positions;
  const float* cos_t;
  const float* sin_t;
  const int32_t* write_loc;
  void* pool_k;
  void* pool_v;
  int64_t q_stride, k_stride, v_stride;
  int64_t table_rows, pool_slots;
  int num_tokens, hq, hkv, d;
  uint32_t* status;
};

template <typename T, int VEC>
union Vec {
  uint4 u;
  T e[VEC];
};

template <typename T>
__device__ __forceinline__ float rot_term(float x, float c) {
  return Elem<T>::round(__fmul_rn(x, c));
}

template <typename T>
__global__ void __launch_bounds__(256) rope_kv_append_kernel(const RopeParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int VEC = 16 / sizeof(T);
  const int half = p.d / 2;
  const int vh = half / VEC;   // 16-byte vectors per half row
  const int vrow = p.d / VEC;  // 16-byte vectors per row
  const int q_items = p.q_out != nullptr ? p.hq * vh : 0;
  const int k_items = p.hkv * vh;
  const int v_items = p.hkv * vrow;
  const int per_tok = q_items + k_items + v_items;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= static_cast<int64_t>(p.num_tokens) * per_tok) return;
  const int t = static_cast<int>(gid / per_tok);
  const int w = static_cast<int>(gid % per_tok);

  int64_t loc = p.write_loc != nullptr ? p.write_loc[t] : -1;
  if (loc >= p.pool_slots) {
    if (w == 0) report(p.status, NSLG_DEV_BAD_SLOT);
    loc = -1;
  }

  if (w < q_items + k_items) {
    const bool is_q = w < q_items;
    const int idx = is_q ? w : w - q_items;
    const int h = idx / vh;
    const int c = idx % vh;
    const T* src = is_q ? static_cast<const T*>(p.q) + t * p.q_stride + h * p.d
                        : static_cast<const T*>(p.k) + t * p.k_stride + h * p.d;
    T* dst;
    if (is_q) {
      dst = static_cast<T*>(p.q_out) + (static_cast<int64_t>(t) * p.hq + h) * p.d;
    } else {
      if (loc < 0) return;
      dst = static_cast<T*>(p.pool_k) + (loc * p.hkv + h) * p.d;
    }
    Vec<T, VEC> x1, x2, o1, o2;
    x1.u = *reinterpret_cast<const uint4*>(src + c * VEC);
    x2.u = *reinterpret_cast<const uint4*>(src + half + c * VEC);
    int64_t pos = p.positions != nullptr ? p.positions[t] : -1;
    if (p.positions != nullptr && (pos < 0 || pos >= p.table_rows)) {
      if (w == 0) report(p.status, NSLG_DEV_BAD_POSITION);
      pos = -1;
    }
    if (pos < 0) {
      o1 = x1;
      o2 = x2;
    } else {
      const float* cs = p.cos_t + pos * p.d + c * VEC;
      const float* sn = p.sin_t + pos * p.d + c * VEC;
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const float a = Elem<T>::to_f(x1.e[i]);
        const float b = Elem<T>::to_f(x2.e[i]);
        const float c1 = Elem<T>::round(cs[i]);
        const float s1 = Elem<T>::round(sn[i]);
        const float c2 = Elem<T>::round(cs[half + i]);
        const float s2 = Elem<T>::round(sn[half + i]);
        // d <  D/2:  x[d]*cos[d] + (-x[d+D/2])*sin[d]
        // d >= D/2:  x[d]*cos[d] + ( x[d-D/2])*sin[d]
        o1.e[i] = Elem<T>::from_f(__fadd_rn(rot_term<T>(a, c1), rot_term<T>(-b, s1)));
        o2.e[i] = Elem<T>::from_f(__fadd_rn(rot_term<T>(b, c2), rot_term<T>(a, s2)));
      }
    }
    *reinterpret_cast<uint4*>(dst + c * VEC) = o1.u;
    *reinterpret_cast<uint4*>(dst + half + c * VEC) = o2.u;
  } else {
    if (loc < 0) return;
    const int idx = w - q_items - k_items;
    const int h = idx / vrow;
    const int c = idx % vrow;
    const T* src = static_cast<const T*>(p.v) + t * p.v_stride + h * p.d + c * VEC;
    T* dst = static_cast<T*>(p.pool_v) + (loc * p.hkv + h) * p.d + c * VEC;
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
  }
}

}  // namespace

int launch_rope_kv_append(int dtype, int num_tokens, int hq, int hkv, int d, const void* q,
                          int64_t q_stride, const void* k, int64_t k_stride, const void* v,
                          int64_t v_stride, void* q_out, const int32_t* positions,
                          const float* cos_t, const float* sin_t, int64_t table_rows,
                          const int32_t* write_loc, void* pool_k, void* pool_v,
                          int64_t pool_slots, uint32_t* status, cudaStream_t stream) {
  RopeParams p{q,        k,        v,          q_out,    positions, cos_t,      sin_t,
               write_loc, pool_k,  pool_v,     q_stride, k_stride,  v_stride,   table_rows,
               pool_slots, num_tokens, hq,     hkv,      d,         status};
  const int esz = dtype == NSLG_DTYPE_BF16 ? 2 : 4;
  const int vec = 16 / esz;
  const int per_tok = (q_out ? hq * (d / 2 / vec) : 0) + hkv * (d / 2 / vec) + hkv * (d / vec);
  const int64_t total = static_cast<int64_t>(num_tokens) * per_tok;
  if (total == 0) return NSLG_OK;
  const int threads = 256;
  const int64_t blocks = (total + threads - 1) / threads;
  const dim3 grid(static_cast<unsigned>(blocks));
  if (dtype == NSLG_DTYPE_BF16)
    return launch_pdl("rope_kv_append", rope_kv_append_kernel<__nv_bfloat16>, grid,
                      dim3(threads), 0, stream, p);
  return launch_pdl("rope_kv_append", rope_kv_append_kernel<float>, grid, dim3(threads), 0,
                    stream, p);
}

}  // namespace nslg
