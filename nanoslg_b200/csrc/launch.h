// Host-side declarations shared by the kernel files and the C ABI in capi.cu.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/nslg_b200.h"

namespace nslg {

// Records `msg` as this thread's last error and returns `code`.
int set_error(int code, const std::string& msg);

// Empties this thread's last error (every entry point does this first, so that
// nslg_last_error() returns "" after a call that succeeded).
void clear_error();

// Bytes per element of an NSLG_DTYPE_* code (4 for float32, 2 for bfloat16 / float16).
inline int dtype_bytes(int dtype) { return dtype == NSLG_DTYPE_F32 ? 4 : 2; }

// Turns a pending launch error into NSLG_ERR_CUDA with the kernel's name.
int check_launch(const char* what);

// Number of SMs of the current device (cached per device).
int sm_count();

// Launches `kern` with programmatic dependent launch allowed: the grid may be scheduled
// while the previous kernel on the stream drains, which hides the launch gap between
// consecutive kernels (also inside CUDA graphs). The kernel must execute pdl_wait()
// (common.cuh) before it reads anything the previous kernel wrote.
template <typename... KArgs, typename... Args>
int launch_pdl(const char* what, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
               cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kern, args...);
  if (err != cudaSuccess) return set_error(NSLG_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
  return check_launch(what);
}

// 3-D tiled tensor map of 2-byte elements (bf16 and fp16 alike: TMA moves bytes, and its
// out-of-bounds fill, 0, is +0.0 in both) with 128-byte swizzle (strides in bytes, dims
// innermost first).
int encode_tiled_3d_bf16(CUtensorMap* out, const void* base, uint64_t d0, uint64_t d1,
                         uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes,
                         uint32_t box0, uint32_t box1, uint32_t box2);

// Cached map of one pool layer [pages, 16, hkv, d] with a [16 tok x 1 head x 64 dim] box.
int pool_tensor_map(const void* pool, int64_t pages, int hkv, int d, CUtensorMap* out);
// Same pool with a [16 tok x hkv heads x 64 dim] box landing as [head][token][64] in smem
// (dims listed token-major); fails if the driver rejects the stride order.
int pool_tensor_map_all_heads(const void* pool, int64_t pages, int hkv, int d, CUtensorMap* out);

int launch_rope_kv_append(int dtype, int num_tokens, int hq, int hkv, int d, const void* q,
                          int64_t q_stride, const void* k, int64_t k_stride, const void* v,
                          int64_t v_stride, void* q_out, const int32_t* positions,
                          const float* cos_t, const float* sin_t, int64_t table_rows,
                          const int32_t* write_loc, void* pool_k, void* pool_v,
                          int64_t pool_slots, uint32_t* status, cudaStream_t stream);

int launch_rmsnorm_residual(int dtype, int rows, int hidden, const void* x, int64_t x_stride,
                            void* residual, int64_t residual_stride, const void* weight,
                            void* out, int64_t out_stride, float eps, cudaStream_t stream);

int launch_silu_mul(int dtype, int rows, int inter, const void* gate_up, int64_t gu_stride,
                    void* out, int64_t out_stride, cudaStream_t stream);

// CUDA-core paged attention (any page size, head_dim <= 256, fp32, bf16 or fp16): decode is
// the qo_len == 1 case.
int launch_paged_attention_simt(int dtype, int batch, int hq, int hkv, int d, int page_size,
                                const void* q, int64_t q_stride, void* out,
                                int64_t out_stride, const int32_t* qo_indptr,
                                const int32_t* q_row_start, int max_qo_len,
                                const void* pool_k, const void* pool_v, int64_t num_pages,
                                const int32_t* kv_indptr, const int32_t* kv_indices,
                                const int32_t* kv_last_page_len, float sm_scale, int causal,
                                uint32_t* status, cudaStream_t stream);

// TMA-fed split-KV decode for bf16 / fp16, page_size 16, head_dim 128 or 64.
bool decode_tc_supported(int dtype, int hq, int hkv, int d, int page_size);
int64_t decode_tc_workspace_bytes(int batch, int hq, int d);
int launch_paged_decode_tc(int dtype, int batch, int hq, int hkv, int d, const void* q,
                           int64_t q_stride,
                           void* out, int64_t out_stride, const void* pool_k,
                           const void* pool_v, int64_t num_pages, const int32_t* kv_indptr,
                           const int32_t* kv_indices, const int32_t* kv_last_page_len,
                           float sm_scale, void* workspace, int64_t workspace_bytes,
                           uint32_t* status, cudaStream_t stream, int vheads = 1);

// tcgen05 causal prefill for bf16 / fp16, page_size 16, head_dim 128, group <= 16
// dividing 128.
bool prefill_tc_supported(int dtype, int hq, int hkv, int d, int page_size);
int launch_paged_prefill_tc(int dtype, int batch, int hq, int hkv, const void* q,
                            int64_t q_stride,
                            int64_t q_rows, void* out, int64_t out_stride,
                            const int32_t* qo_indptr, const int32_t* q_row_start, int max_qo_len,
                            const void* pool_k, const void* pool_v, int64_t num_pages,
                            const int32_t* kv_indptr, const int32_t* kv_indices,
                            const int32_t* kv_last_page_len, float sm_scale, int causal,
                            uint32_t* status, cudaStream_t stream);

// tcgen05 linear layer y = x . W^T for at most kLinearMaxRows rows of x (decode steps),
// bf16 / fp16, K a multiple of 64 (linear_tc.cu).
constexpr int kLinearMaxRows = 256;
bool linear_tc_supported(int dtype, int M, int N, int K);

// Blocks of every tensor-parallel reduction call (tp_allreduce.cu). Block b numbers its
// calls with counter word b and handles rows b, b + kTpReduceGrid, ...; a producer that
// pushes row m into the peers' stage buffers tags it with counter word m % kTpReduceGrid.
constexpr int kTpReduceGrid = 128;

// Where a linear layer pushes its output rows as this rank's partial of a one-shot
// tensor-parallel reduction: the stage buffers of every rank (this one's included, not
// written), this rank's call counters, and the slot / source-region geometry the
// reduction kernel uses for `world` ranks (tp_stage_geometry).
struct TpPush {
  uint8_t* stage[NSLG_TP_MAX_WORLD];
  const uint32_t* counters;
  int64_t slot_bytes, region_bytes;
  int world, rank;
};
// [2 slots][world sources][rows][2 x row bytes]: region (one source's rows of one slot)
// and slot sizes of a stage buffer of stage_bytes.
inline void tp_stage_geometry(int64_t stage_bytes, int world, int64_t* region, int64_t* slot) {
  *region = (stage_bytes / 2 / world) & ~static_cast<int64_t>(15);
  *slot = *region * world;
}

// push == nullptr: y only. Otherwise also every row of y, packed with this rank's call
// numbers, into every peer's stage buffer (out_features is then the reduced row length).
// swiglu: w is a stacked [2N, K] gate|up weight and y[m][c] = silu(x.gate_c) * (x.up_c)
// with the reference's rounding points (no push; NSLG_ERR_UNSUPPORTED where the split-K
// sum of the shape would not be pushed).
// rope: N = (hq + 2 hkv) * 128 rows of a stacked q|k|v weight, y unused; the epilogue
// rotates q into q_out and appends rotated k and v to the pool (nslg_rope_kv_append's
// operation), NSLG_ERR_UNSUPPORTED like swiglu.
struct LinearRope {
  int hq, hkv;
  void* q_out;
  const int32_t* positions;
  const float* cos_t;
  const float* sin_t;
  int64_t table_rows;
  const int32_t* write_loc;
  void* pool_k;
  void* pool_v;
  int64_t pool_slots;
};
int launch_linear_tc(int dtype, int M, int N, int K, const void* x, int64_t x_stride,
                     const void* w, int64_t w_stride, void* y, int64_t y_stride,
                     const TpPush* push, uint32_t* status, cudaStream_t stream,
                     bool swiglu = false, const LinearRope* rope = nullptr);

}  // namespace nslg
