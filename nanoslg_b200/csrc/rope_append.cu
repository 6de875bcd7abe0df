// Fused rotary embedding + paged KV append.
//
// A thread owns 16 bytes of a head row. For q and k it owns the matching 16 bytes of
// both halves of the row (rotate-half pairs dimension d with d + D/2), rotates them and
// stores them with 16-byte vector stores: q into q_out, k into the page slot the
// context assigned to the token. v is copied unrotated. The arithmetic repeats the
// reference's elementwise ops with their rounding points (models.py:79-83): cos/sin
// are first cast to the activation type, then
//   out = x*cos + cat(-x2, x1)*sin
// with every product and the sum rounded to the activation type.
//
// bf16 (rope_kv_append_bf16_kernel): one CTA per token, two 16-byte items per thread,
// both read before anything else. The token's cos/sin row is rounded to bf16 once, into
// shared memory, and every q/k head of the token reads it from there; the products and sums run as paired bf16 instructions (mul/add/sub.rn
// .bf16x2: each rounds the exact result once, as torch does after computing the op in
// fp32, and explicit .rn keeps them from being contracted into a fused multiply-add).
// Per 16-byte output: 4 multiplies and 2 adds of bf16 pairs, no conversions.
// fp32 (rope_kv_append_kernel): the explicitly rounded fp32 intrinsics, so no fused
// multiply-add changes the result.
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

__device__ __forceinline__ uint32_t bf2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf2_add(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

constexpr int kBf16MaxThreads = 512;

template <int D>
__global__ void __launch_bounds__(kBf16MaxThreads) rope_kv_append_bf16_kernel(const RopeParams p) {
  constexpr int HALF = D / 2;
  constexpr int VH = HALF / 8;    // 16-byte chunks per half row
  constexpr int VROW = D / 8;     // 16-byte chunks per row
  // bf16 pairs of the token's cos / sin row, rounded: word i = dims 2i, 2i + 1
  __shared__ __align__(16) uint32_t cs2[HALF];
  __shared__ __align__(16) uint32_t sn2[HALF];
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int q_items = p.q_out != nullptr ? p.hq * VH : 0;
  const int k_items = p.hkv * VH;
  const int per_tok = q_items + k_items + p.hkv * VROW;
  const __nv_bfloat16* qb = static_cast<const __nv_bfloat16*>(p.q) + t * p.q_stride;
  const __nv_bfloat16* kb = static_cast<const __nv_bfloat16*>(p.k) + t * p.k_stride;
  const __nv_bfloat16* vb = static_cast<const __nv_bfloat16*>(p.v) + t * p.v_stride;
  // item w: q/k head idx / VH, 16-byte chunk idx % VH of both halves; or v head
  // idx / VROW, chunk idx % VROW
  auto load = [&](int w, uint4& x1, uint4& x2) {
    if (w < q_items + k_items) {
      const bool is_q = w < q_items;
      const int idx = is_q ? w : w - q_items;
      const __nv_bfloat16* src = (is_q ? qb : kb) + (idx / VH) * D + (idx % VH) * 8;
      x1 = *reinterpret_cast<const uint4*>(src);
      x2 = *reinterpret_cast<const uint4*>(src + HALF);
    } else {
      const int idx = w - q_items - k_items;
      x1 = *reinterpret_cast<const uint4*>(vb + (idx / VROW) * D + (idx % VROW) * 8);
    }
  };
  // Each thread owns two items, w = tid and tid + blockDim; both are read before the
  // table row is staged, so every thread has 32-64 bytes in flight while the position
  // and the cos/sin row arrive.
  uint4 f1[2], f2[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    f1[u] = f2[u] = make_uint4(0u, 0u, 0u, 0u);
    const int w = threadIdx.x + u * blockDim.x;
    if (w < per_tok) load(w, f1[u], f2[u]);
  }
  int64_t loc = p.write_loc != nullptr ? p.write_loc[t] : -1;
  if (loc >= p.pool_slots) {
    if (threadIdx.x == 0) report(p.status, NSLG_DEV_BAD_SLOT);
    loc = -1;
  }
  bool rot = false;
  if (p.positions != nullptr) {
    const int64_t pos = p.positions[t];
    if (pos < 0 || pos >= p.table_rows) {
      if (threadIdx.x == 0) report(p.status, NSLG_DEV_BAD_POSITION);
    } else {
      rot = true;
      const float2* c = reinterpret_cast<const float2*>(p.cos_t + pos * D);
      const float2* sn = reinterpret_cast<const float2*>(p.sin_t + pos * D);
      for (int i = threadIdx.x; i < HALF; i += blockDim.x) {
        const __nv_bfloat162 cb = __float22bfloat162_rn(c[i]);
        const __nv_bfloat162 sb = __float22bfloat162_rn(sn[i]);
        cs2[i] = *reinterpret_cast<const uint32_t*>(&cb);
        sn2[i] = *reinterpret_cast<const uint32_t*>(&sb);
      }
    }
  }
  __syncthreads();
  auto finish = [&](int w, uint4 x1, uint4 x2) {
    if (w < q_items + k_items) {
      const bool is_q = w < q_items;
      const int idx = is_q ? w : w - q_items;
      const int h = idx / VH, c = idx % VH;
      __nv_bfloat16* dst;
      if (is_q) {
        dst = static_cast<__nv_bfloat16*>(p.q_out) + (static_cast<int64_t>(t) * p.hq + h) * D;
      } else {
        if (loc < 0) return;
        dst = static_cast<__nv_bfloat16*>(p.pool_k) + (loc * p.hkv + h) * D;
      }
      if (rot) {
        const uint4 c1 = *reinterpret_cast<const uint4*>(&cs2[c * 4]);
        const uint4 s1 = *reinterpret_cast<const uint4*>(&sn2[c * 4]);
        const uint4 c2 = *reinterpret_cast<const uint4*>(&cs2[HALF / 2 + c * 4]);
        const uint4 s2 = *reinterpret_cast<const uint4*>(&sn2[HALF / 2 + c * 4]);
        // d <  D/2:  x[d]*cos[d] - x[d+D/2]*sin[d];  d >= D/2:  x[d]*cos[d] + x[d-D/2]*sin[d]
        const uint4 o1{bf2_sub(bf2_mul(x1.x, c1.x), bf2_mul(x2.x, s1.x)),
                       bf2_sub(bf2_mul(x1.y, c1.y), bf2_mul(x2.y, s1.y)),
                       bf2_sub(bf2_mul(x1.z, c1.z), bf2_mul(x2.z, s1.z)),
                       bf2_sub(bf2_mul(x1.w, c1.w), bf2_mul(x2.w, s1.w))};
        const uint4 o2{bf2_add(bf2_mul(x2.x, c2.x), bf2_mul(x1.x, s2.x)),
                       bf2_add(bf2_mul(x2.y, c2.y), bf2_mul(x1.y, s2.y)),
                       bf2_add(bf2_mul(x2.z, c2.z), bf2_mul(x1.z, s2.z)),
                       bf2_add(bf2_mul(x2.w, c2.w), bf2_mul(x1.w, s2.w))};
        x1 = o1;
        x2 = o2;
      }
      *reinterpret_cast<uint4*>(dst + c * 8) = x1;
      *reinterpret_cast<uint4*>(dst + HALF + c * 8) = x2;
    } else {
      if (loc < 0) return;
      const int idx = w - q_items - k_items;
      __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.pool_v) +
                           (loc * p.hkv + idx / VROW) * D + (idx % VROW) * 8;
      *reinterpret_cast<uint4*>(dst) = x1;
    }
  };
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int w = threadIdx.x + u * blockDim.x;
    if (w < per_tok) finish(w, f1[u], f2[u]);
  }
  // rows wider than two items per thread (a block has at most kBf16MaxThreads threads)
  for (int w = threadIdx.x + 2 * blockDim.x; w < per_tok; w += blockDim.x) {
    uint4 x1 = make_uint4(0u, 0u, 0u, 0u), x2 = x1;
    load(w, x1, x2);
    finish(w, x1, x2);
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
  if (dtype == NSLG_DTYPE_BF16 && (d == 128 || d == 64) && num_tokens > 0) {
    const int per_tok = (q_out ? hq * (d / 16) : 0) + hkv * (d / 16) + hkv * (d / 8);
    if (per_tok == 0) return NSLG_OK;
    int threads = ((per_tok + 1) / 2 + 31) / 32 * 32;   // two items per thread
    if (threads > kBf16MaxThreads) threads = kBf16MaxThreads;
    const dim3 grid(static_cast<unsigned>(num_tokens));
    if (d == 128)
      return launch_pdl("rope_kv_append", rope_kv_append_bf16_kernel<128>, grid, dim3(threads),
                        0, stream, p);
    return launch_pdl("rope_kv_append", rope_kv_append_bf16_kernel<64>, grid, dim3(threads), 0,
                      stream, p);
  }
  const int esz = dtype_bytes(dtype);
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
  if (dtype == NSLG_DTYPE_F16)
    return launch_pdl("rope_kv_append", rope_kv_append_kernel<__half>, grid, dim3(threads), 0,
                      stream, p);
  return launch_pdl("rope_kv_append", rope_kv_append_kernel<float>, grid, dim3(threads), 0,
                    stream, p);
}

}  // namespace nslg
