// Decode-sized linear layers on the 5th-generation tensor cores: y = x . W^T for a few
// rows of activations (the batch of a decode step) against a large weight matrix,
// bf16 or fp16, fp32 accumulation, the result rounded once to the activation type.
//
// Replaces, for forwards of at most 256 rows, the cuBLAS GEMMs behind the projections
// the decode step runs per layer (ColumnParallelLinear / RowParallelLinear's F.linear,
// tp_layers.py:28-158, and the stacked q|k|v and gate|up products) and the LM head on
// the last position. At these shapes the product is a stream over the weights (64 rows
// of x against 4096 x 14336 weights is 64 flop per weight byte), so the kernel is built
// to keep HBM busy: every weight byte is read once, with TMA, in 16 KiB boxes.
//
// Shape of the MMA ("swap AB"). A tile is 128 weight rows: the MMA's M dimension is the
// weight rows (A = W tile [128 x 64] from shared memory, K-major, 128-byte swizzle), its
// N dimension the activation rows (B = x tile [Mp x 64], Mp = rows rounded up to 16;
// TMA fills the rows past the end with zeros), and the accumulator D [128 x Mp] fp32
// lives in TMEM. Four tcgen05.mma (K = 16 each) per 64-element chunk of K.
//
// Work split ("stream-K"). The (tile, K-chunk) iterations of the whole product form one
// list, n_tiles x kc long; CTA c of `grid` takes the contiguous range
// [total * c / grid, total * (c + 1) / grid), so every CTA streams the same number of
// weight bytes whatever the shape (no wave quantisation: a 224-tile product on 148 SMs
// costs 1.5 tiles per SM, not 2). A CTA's range covers the tail of one tile, whole
// tiles, and the head of another. Whole tiles are written to y directly. A tile shared
// by several CTAs: each writes its fp32 partial tile to the workspace (slot 2c for the
// first tile of CTA c, 2c + 1 for its last), fences, and increments the tile's counter;
// the CTA that arrives last sums the partials in CTA order (the same order on every
// call, so the result does not depend on timing), rounds once, writes y and sets the
// counter back to zero.
//
// Pipeline (one CTA per SM, 256 threads):
//   warp 0     TMA producer: per iteration one W box [64 x 128] and one x box [64 x Mp]
//              into a ring of stages guarded by full / empty mbarriers;
//   warp 1     MMA issuer: per tile segment, waits for an accumulator the epilogue has
//              drained, 4 MMAs per stage, commits the stage back to the producer and the
//              accumulator to the epilogue (two accumulators, so the next segment's MMAs
//              overlap the epilogue of this one);
//   warps 4-7  epilogue: thread r owns TMEM lane r = weight row n0 + r; reads D in
//              16-column pieces and writes y[m][n0 + r] (each store instruction of a warp
//              covers 32 consecutive n of one row m), or the fp32 partial.
// Every mbarrier wait is bounded (2 s); on a timeout the kernel records
// NSLG_DEV_WAIT_TIMEOUT, stops, drains what it issued (bounded), frees TMEM and returns.
#include <cuda.h>

#include <string>

#include "common.cuh"
#include "launch.h"
#include "tcgen05.cuh"

namespace nslg {
namespace {

constexpr int kTileN = 128;       // weight rows per tile (MMA M)
constexpr int kChunk = 64;        // K elements per stage: one 128-byte swizzle row
constexpr int kThreads = 256;     // warp 0 TMA, warp 1 MMA, warps 4-7 epilogue
constexpr int kMaxStages = 8;
constexpr int kMinChunksPerCta = 4;
constexpr int kWBytes = kTileN * 128;   // 16 KiB W box per stage
constexpr int kLinearSmemBudget = 232448 - 1024 - 256;  // opt-in smem minus alignment, barriers

struct LinParams {
  void* y;
  int64_t y_stride;
  float* part;          // [2 * grid][Mp][kTileN] fp32 partial tiles
  uint32_t* counters;   // [n_tiles], zero between calls
  int M, N, Mp, n_tiles, kc, grid, stages, tmem_cols;
  int64_t total;        // n_tiles * kc iterations
  uint32_t* status;
};

__device__ __forceinline__ int64_t iter_begin(const LinParams& p, int c) {
  return p.total * c / p.grid;
}
// CTA whose range holds iteration i: the largest c with floor(total * c / grid) <= i
__device__ __forceinline__ int cta_of_iter(const LinParams& p, int64_t i) {
  return static_cast<int>((static_cast<int64_t>(p.grid) * (i + 1) - 1) / p.total);
}
// partial-tile slot of CTA c for tile t (its first tile: 2c, its last: 2c + 1)
__device__ __forceinline__ int64_t part_slot(const LinParams& p, int c, int t) {
  const int first = static_cast<int>(iter_begin(p, c) / p.kc);
  return 2 * static_cast<int64_t>(c) + (t == first ? 0 : 1);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap tmap_w,
                     const __grid_constant__ CUtensorMap tmap_x, const LinParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int xbytes = p.Mp * 128;
  const int sbytes = kWBytes + xbytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.stages * sbytes);
  uint64_t* empty = full + kMaxStages;
  uint64_t* acc_full = empty + kMaxStages;   // [2]
  uint64_t* acc_empty = acc_full + 2;        // [2]
  uint64_t* mma_drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = abort_flag + 1;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int c = blockIdx.x;
  const int64_t b0 = iter_begin(p, c), b1 = iter_begin(p, c + 1);
  const int t_first = static_cast<int>(b0 / p.kc);
  const int t_last = static_cast<int>((b1 - 1) / p.kc);

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    mbar_init(mma_drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(p.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();     // the next kernel may start its prologue; it waits for our completion

  if (warp == 0) {
    // -------------------------------------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&tmap_w);
      prefetch_tmap(&tmap_x);
      const uint64_t stream_w = l2_policy_evict_first();   // every weight byte used once
      const uint64_t keep_x = l2_policy_evict_last();      // x is re-read by every CTA
      pdl_wait();      // x is the previous kernel's output
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      bool ok = true;
      for (int64_t it = b0; it < b1; ++it) {
        if (*abort_flag || !mbar_wait(&empty[stage], phase ^ 1)) { ok = false; break; }
        const int t = static_cast<int>(it / p.kc);
        const int k = static_cast<int>(it - static_cast<int64_t>(t) * p.kc);
        uint8_t* sb = smem + stage * sbytes;
        mbar_arrive_expect_tx(&full[stage], sbytes);
        tma_load_3d(sb, &tmap_w, &full[stage], k * kChunk, t * kTileN, 0, stream_w);
        tma_load_3d(sb + kWBytes, &tmap_x, &full[stage], k * kChunk, 0, 0, keep_x);
        ++issued;
        if (++stage == p.stages) { stage = 0; phase ^= 1; }
      }
      if (!ok) {
        report(p.status, NSLG_DEV_WAIT_TIMEOUT);
        *abort_flag = 1;
        // no load may still be writing shared memory when the CTA leaves (bounded)
        for (int64_t u = issued - p.stages < 0 ? 0 : issued - p.stages; u < issued; ++u)
          (void)mbar_wait(&full[u % p.stages], (u / p.stages) & 1);
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(Mma16<T>::kFormat, p.Mp, false);
      constexpr uint32_t kDescHi = smem_desc_hi(1024);
      const uint32_t lo0 = smem_desc_lo(smem_u32(smem), 16);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int seg = 0;
      int64_t it = b0;
      for (int t = t_first; ok && t <= t_last; ++t, ++seg) {
        const int a = seg & 1;
        const int64_t seg_end = min(b1, static_cast<int64_t>(t + 1) * p.kc);
        // the epilogue has drained this accumulator's previous segment
        if (seg >= 2 && !(ok = mbar_wait(&acc_empty[a], ((seg - 2) >> 1) & 1))) break;
        tc_fence_after();
        const uint32_t d = tmem + a * p.Mp;
        for (bool first = true; it < seg_end; ++it, first = false) {
          if (*abort_flag || !(ok = mbar_wait(&full[stage], phase))) break;
          tc_fence_after();
          const uint32_t w_lo = lo0 + (stage * sbytes >> 4);
          const uint32_t x_lo = lo0 + ((stage * sbytes + kWBytes) >> 4);
#pragma unroll
          for (int ks = 0; ks < kChunk / 16; ++ks)
            mma_ss_w(d, w_lo + ks * 2, x_lo + ks * 2, kDescHi, idesc,
                     (first && ks == 0) ? 0u : 1u);
          mma_commit(&empty[stage]);
          if (++stage == p.stages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        mma_commit(&acc_full[a]);
      }
      if (!ok) {
        report(p.status, NSLG_DEV_WAIT_TIMEOUT);
        *abort_flag = 1;
      }
      // every MMA issued so far has completed once this arrives (bounded wait)
      mma_commit(mma_drain);
      (void)mbar_wait(mma_drain, 0);
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------- epilogue
    const int r = (warp & 3) * 32 + lane;          // TMEM lane = row of the tile
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int et = threadIdx.x - 128;              // 0..127
    T* y = static_cast<T*>(p.y);
    int seg = 0;
    bool ok = true;
    for (int t = t_first; t <= t_last; ++t, ++seg) {
      const int a = seg & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[a], (seg >> 1) & 1))) { ok = false; break; }
      tc_fence_after();
      const int n = t * kTileN + r;
      const int64_t t_beg = static_cast<int64_t>(t) * p.kc, t_end = t_beg + p.kc;
      const bool whole = b0 <= t_beg && t_end <= b1;
      float* dst = whole ? nullptr
                         : p.part + (part_slot(p, c, t) * p.Mp) * kTileN + r;
      for (int c0 = 0; c0 < p.Mp; c0 += 16) {
        float v[16];
        tmem_ld16(lane_base + a * p.Mp + c0, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = c0 + j;
          if (m >= p.M) break;
          if (whole) {
            if (n < p.N) y[static_cast<int64_t>(m) * p.y_stride + n] = Elem<T>::from_f(v[j]);
          } else {
            dst[static_cast<int64_t>(m) * kTileN] = v[j];
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[a]);               // the MMA warp may reuse this accumulator
      if (whole) continue;
      // shared tile: publish the partial, count it, and the last contributor finishes
      __threadfence();
      named_barrier_sync(2, 128);
      const int cf = cta_of_iter(p, t_beg), cl = cta_of_iter(p, t_end - 1);
      if (et == 0) {
        const uint32_t old = atomicAdd(&p.counters[t], 1u);
        const bool last = old == static_cast<uint32_t>(cl - cf);
        if (last) p.counters[t] = 0u;           // every contributor has arrived
        *last_flag = last ? 1 : 0;
      }
      named_barrier_sync(2, 128);
      if (*last_flag) {
        __threadfence();
        for (int m = 0; m < p.M; ++m) {
          float s = 0.f;
          for (int cc = cf; cc <= cl; ++cc)
            s += __ldcg(p.part + (part_slot(p, cc, t) * p.Mp + m) * kTileN + r);
          if (n < p.N) y[static_cast<int64_t>(m) * p.y_stride + n] = Elem<T>::from_f(s);
        }
      }
      named_barrier_sync(2, 128);               // last_flag is rewritten by the next tile
    }
    if (!ok) {
      if (lane == 0) report(p.status, NSLG_DEV_WAIT_TIMEOUT);
      *abort_flag = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(p.tmem_cols)
                 : "memory");
  }
}

int64_t counters_bytes(int n_tiles) { return (static_cast<int64_t>(n_tiles) * 4 + 255) & ~255ll; }

struct Plan {
  int Mp, n_tiles, kc, grid, stages, tmem_cols;
  int64_t total;
};

Plan plan_for(int M, int N, int K) {
  Plan pl{};
  pl.Mp = (M + 15) / 16 * 16;
  pl.n_tiles = (N + kTileN - 1) / kTileN;
  pl.kc = K / kChunk;
  pl.total = static_cast<int64_t>(pl.n_tiles) * pl.kc;
  int64_t g = pl.total / kMinChunksPerCta;
  if (g > sm_count()) g = sm_count();
  if (g < 1) g = 1;
  pl.grid = static_cast<int>(g);
  const int sbytes = kWBytes + pl.Mp * 128;
  int st = (kLinearSmemBudget - 2048) / sbytes;
  pl.stages = st > kMaxStages ? kMaxStages : st;
  int cols = 32;
  while (cols < 2 * pl.Mp) cols *= 2;
  pl.tmem_cols = cols;
  return pl;
}

}  // namespace

int64_t linear_tc_workspace_bytes(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const Plan pl = plan_for(M, N, K);
  return counters_bytes(pl.n_tiles) + 2ll * pl.grid * pl.Mp * kTileN * 4;
}

bool linear_tc_supported(int dtype, int M, int N, int K) {
  return (dtype == NSLG_DTYPE_BF16 || dtype == NSLG_DTYPE_F16) && M >= 1 && M <= kLinearMaxRows &&
         N >= 1 && K >= kChunk && K % kChunk == 0;
}

int launch_linear_tc(int dtype, int M, int N, int K, const void* x, int64_t x_stride,
                     const void* w, int64_t w_stride, void* y, int64_t y_stride,
                     void* workspace, int64_t workspace_bytes, uint32_t* status,
                     cudaStream_t stream) {
  const Plan pl = plan_for(M, N, K);
  const int64_t need = linear_tc_workspace_bytes(M, N, K);
  if (workspace == nullptr || workspace_bytes < need)
    return set_error(NSLG_ERR_WORKSPACE, "linear: workspace needs " + std::to_string(need) + " bytes");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return set_error(NSLG_ERR_ARG, "linear: workspace must be 256-byte aligned");
  CUtensorMap tw, tx;
  // W [N, K] and x [M, K], K innermost; boxes [64 x 128] and [64 x Mp] with 128-byte swizzle
  int rc = encode_tiled_3d_bf16(&tw, w, K, N, 1, static_cast<uint64_t>(w_stride) * 2,
                                static_cast<uint64_t>(w_stride) * 2 * N, kChunk, kTileN, 1);
  if (rc != NSLG_OK) return rc;
  rc = encode_tiled_3d_bf16(&tx, x, K, M, 1, static_cast<uint64_t>(x_stride) * 2,
                            static_cast<uint64_t>(x_stride) * 2 * M, kChunk, pl.Mp, 1);
  if (rc != NSLG_OK) return rc;
  LinParams p{};
  p.y = y;
  p.y_stride = y_stride;
  p.counters = static_cast<uint32_t*>(workspace);
  p.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + counters_bytes(pl.n_tiles));
  p.M = M;
  p.N = N;
  p.Mp = pl.Mp;
  p.n_tiles = pl.n_tiles;
  p.kc = pl.kc;
  p.grid = pl.grid;
  p.stages = pl.stages;
  p.tmem_cols = pl.tmem_cols;
  p.total = pl.total;
  p.status = status;
  const size_t smem = 1024 + static_cast<size_t>(pl.stages) * (kWBytes + pl.Mp * 128) + 256;
  auto kern = dtype == NSLG_DTYPE_F16 ? linear_tc_kernel<__half> : linear_tc_kernel<__nv_bfloat16>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return set_error(NSLG_ERR_CUDA, cudaGetErrorString(err));
  return launch_pdl("linear_tc", kern, dim3(pl.grid), dim3(kThreads), smem, stream, tw, tx, p);
}

}  // namespace nslg
