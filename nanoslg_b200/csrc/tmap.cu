// TMA tensor-map encoding (host side) shared by the decode and prefill kernels.
//
// cuTensorMapEncodeTiled is a driver entry point; it is fetched through the runtime's
// cudaGetDriverEntryPoint so the library does not link libcuda directly.
#include <cuda.h>

#include <mutex>
#include <string>

#include "launch.h"

namespace nslg {
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// Pool maps are cached per (layer pointer, pages, heads, head_dim): the pool is allocated
// once and each layer's K and V maps are reused on every step.
struct MapEntry {
  const void* ptr = nullptr;
  int64_t pages = 0;
  int hkv = 0, d = 0;
  int all_heads = 0;
  CUtensorMap map;
};
constexpr int kMapCache = 512;
MapEntry g_maps[kMapCache];
int g_map_next = 0;
std::mutex g_map_mu;

}  // namespace

int encode_tiled_3d_bf16(CUtensorMap* out, const void* base, uint64_t d0, uint64_t d1,
                         uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes,
                         uint32_t box0, uint32_t box1, uint32_t box2) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return set_error(NSLG_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  const cuuint32_t box[3] = {box0, box1, box2};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(NSLG_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(r));
  return NSLG_OK;
}

int cached_pool_map(const void* pool, int64_t pages, int hkv, int d, int all_heads,
                    CUtensorMap* out) {
  std::lock_guard<std::mutex> lock(g_map_mu);
  for (int i = 0; i < kMapCache; ++i) {
    const MapEntry& e = g_maps[i];
    if (e.ptr == pool && e.pages == pages && e.hkv == hkv && e.d == d &&
        e.all_heads == all_heads) {
      *out = e.map;
      return NSLG_OK;
    }
  }
  MapEntry& e = g_maps[g_map_next];
  e.ptr = nullptr;
  const uint64_t tok = static_cast<uint64_t>(pages) * 16;
  const uint64_t tok_stride = static_cast<uint64_t>(hkv) * d * 2, head_stride = static_cast<uint64_t>(d) * 2;
  const int rc =
      all_heads
          // dims: head_dim, token row, kv head (token stride listed before the smaller head
          // stride); box 64 dims x 16 tokens x all heads -> smem [head][token][64 dims]
          ? encode_tiled_3d_bf16(&e.map, pool, d, tok, hkv, tok_stride, head_stride, 64, 16, hkv)
          // dims: head_dim, kv head, token row; box 64 dims x 1 head x 16 tokens
          : encode_tiled_3d_bf16(&e.map, pool, d, hkv, tok, head_stride, tok_stride, 64, 1, 16);
  if (rc != NSLG_OK) return rc;
  e.ptr = pool;
  e.pages = pages;
  e.hkv = hkv;
  e.d = d;
  e.all_heads = all_heads;
  *out = e.map;
  g_map_next = (g_map_next + 1) % kMapCache;
  return NSLG_OK;
}

int pool_tensor_map(const void* pool, int64_t pages, int hkv, int d, CUtensorMap* out) {
  return cached_pool_map(pool, pages, hkv, d, 0, out);
}

int pool_tensor_map_all_heads(const void* pool, int64_t pages, int hkv, int d, CUtensorMap* out) {
  return cached_pool_map(pool, pages, hkv, d, 1, out);
}

}  // namespace nslg
