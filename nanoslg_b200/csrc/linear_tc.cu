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
// Work split. CTA c computes tile c / s over the K-chunk range of split c % s, where
// the host picks s (splits per tile, at most 8) so that n_tiles * s fills the SMs twice
// over (two CTAs fit on an SM) without cutting K into pieces of fewer than
// kMinChunksPerSplit chunks, as a power of two when the grid exceeds the SM count (so
// the clusters pack into the GPCs in one wave): s = 1 for wide products (each CTA one whole tile, written straight to y; a 224-tile
// product runs at once on 148 SMs), s > 1 for narrow ones (o_proj, down_proj, TP
// shards). The s CTAs of a tile form one thread-block cluster, and the split-K sum
// never leaves the chip: CTA j owns rows [8 floor(16 j / s), 8 floor(16 (j + 1) / s))
// of the tile, sums them over the s fp32 partials in rank order (the same order on
// every call), rounds once and writes them to y. Decode batches (up to 64 rows): every
// CTA stores its partial of each owner's rows straight into that owner's shared memory
// (st.async, 4 bytes per store, each counted on the owner's mbarrier), and the owner
// waits for its mbarrier alone -- one cluster arrive at the start, no cluster barrier
// at the end (about 1 us less per call than the pulled sum). Larger batches: each CTA
// stages its partial tile in its own shared memory (the stage ring, idle once the MMAs
// are done), the cluster synchronises, the owners read the partials through
// distributed shared memory, and a second cluster barrier keeps every partial in place
// until all readers are done.
//
// Fused tensor-parallel push (nslg_linear_tp_push). For a RowParallel product (o_proj,
// down_proj) of a TP decode step, y is this rank's partial of the all-reduce that
// follows. With the push on, each CTA, once its rows of y are final, also stores them
// packed with the reduction's call numbers straight into every peer's stage buffer over
// NVLink (the layout nslg_tp_allreduce_rmsnorm's one-shot mode reads), so the transfer
// runs while other tiles are still on the tensor cores and the reduction kernel that
// follows only waits for, sums and normalises the rows (nslg_tp_reduce_pushed_rmsnorm).
// The compute and the collective's data movement are one kernel; no load ever reads a
// peer's memory.
//
// Paired epilogues. Two modes keep row r < 64 of a tile together with row r + 64 (in the
// staged tile, and in each split owner's share: columns [lo, hi) of 64 mean rows
// [lo, hi) and [64 + lo, 64 + hi)). SwiGLU (nslg_linear_swiglu): tile t is loaded as
// gate rows [64t, 64t + 64) and up rows [I + 64t, ...) of a stacked gate|up weight (two
// 64-row boxes into the one swizzled A tile), and the epilogue writes silu(gate) * up.
// RoPE + KV append (nslg_linear_rope_append): with head_dim 128 a tile of the stacked
// q|k|v product is one head, whose rotate-half pairs are rows r and r + 64; the epilogue
// rotates q into q_out and k into the paged pool and copies v there. Both round as the
// separate kernels do, so their results are bit for bit the two-kernel results.
//
// Pipeline (up to two CTAs per SM, 256 threads each):
//   warp 0     TMA producer: the first ring's worth of weight boxes before waiting for
//              the previous kernel (programmatic dependent launch: the weights do not
//              depend on it), then per chunk one W box [64 x 128] and one x box
//              [64 x Mp] into a ring of stages guarded by full / empty mbarriers;
//   warp 1     MMA issuer: 4 MMAs per stage, commits each stage back to the producer and
//              the accumulator to the epilogue;
//   warps 4-7  epilogue: thread r owns TMEM lane r = weight row n0 + r; reads D in
//              32-column pieces into shared memory (the idle stage ring): the rounded y
//              tile, or the fp32 partial tile; then all 256 threads of the CTA write the
//              tile's rows of y with 16-byte stores, or do its share of the cluster's
//              sum (16-byte loads of the partials, 8-byte stores of y).
// Every wait is bounded (2 s); on a timeout the kernel records NSLG_DEV_WAIT_TIMEOUT,
// stops, drains what it issued (bounded), frees TMEM and returns.
#include <cooperative_groups.h>
#include <cuda.h>

#include <cstdlib>
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
constexpr int kMinStages = 3;
constexpr int kMinChunksPerSplit = 2;   // 32 KiB of weights per CTA at least
constexpr int kCtasPerSm = 2;           // K splits may fill the SMs twice over
constexpr int kMaxSplits = 8;           // portable cluster size
constexpr int kWBytes = kTileN * 128;   // 16 KiB W box per stage
// Row stride (floats) of a staged fp32 partial tile: 128 + 16, so that rows m and m + 1
// sit 16 banks apart. Mp * 576 bytes fit in the stage ring for every Mp <= 256 (at
// least three stages of 16 KiB + Mp * 128 bytes).
constexpr int kPartStride = kTileN + 16;
// Stage ring of about 112 KiB, so that two CTAs fit on an SM: a wide product's whole
// grid runs at once, and the next launch's CTA can set up and start its weight loads
// while this one drains (a 200 KiB ring of 8 stages, one CTA per SM, measured slower on
// the 8B shapes: 19.5 against 12.3 us for q|k|v at one row).
constexpr int kLinearSmemBudget = 112 * 1024;
constexpr int kMaxTiles = 1 << 16;      // out_features <= 8,388,608
// Split-K sums of batches up to this many (padded) rows are pushed: each CTA stores its
// partial rows straight into the shared memory of the CTA that owns them (st.async,
// completing on the owner's mbarrier), instead of staging them and pulling them through
// distributed shared memory between two cluster barriers. The receive buffer,
// s * Mp * (largest row share) floats <= 168 * Mp * 4 bytes, comes out of the ring; the
// push is used where it leaves at least kMinStages stages (at 64 rows: every s but 7).
// Measured on the 8B shapes: 0.7-1.2 us faster per call at 1-16 rows, 2.5-4 us at 64.
constexpr int kPushMaxMp = 64;

// RoPE + paged KV append in the epilogue of a stacked q|k|v product with head_dim 128
// (one tile = one head: q heads 0..hq-1, k heads, v heads), the operation and the
// rounding of nslg_rope_kv_append: q rotated into q_out [rows, hq, 128], k rotated and
// v copied into the pool slot write_loc[m] (< 0: not written).
struct RopeAppend {
  int on, hq, hkv;
  void* q_out;
  const int32_t* positions;   // NULL: no rotation
  const float* cos_t;
  const float* sin_t;
  int64_t table_rows;
  const int32_t* write_loc;
  void* pool_k;
  void* pool_v;
  int64_t pool_slots;
};

struct LinParams {
  void* y;
  int64_t y_stride;
  int M, N, Mp, kc, splits, stages, tmem_cols;
  int do_push;      // also push y's rows to the peers (push)
  int y_vec;        // y's rows start on 16-byte boundaries (base and stride)
  int push_sum;     // split-K partials pushed to their owners (splits > 1, Mp <= 64)
  int swiglu;       // tile t = gate rows [64t, 64t + 64) and up rows [I + 64t, ...) of a
                    // stacked gate|up weight; y[m][c] = silu(gate) * up, N = I
  int paired;       // epilogue pairs row r < 64 of a tile with row r + 64 (SwiGLU, RoPE)
  RopeAppend rope;  // rope.on: tile t is q / k / v head t of a stacked q|k|v product
  TpPush push;
  uint32_t* status;
};

// y[m][n0 .. n0 + 8) = the eight values packed in v: one 16-byte store where the row is
// aligned and the eight columns exist, else element by element up to out_features.
template <typename T>
__device__ __forceinline__ void store_y8(const LinParams& p, int m, int n0, uint4 v) {
  T* dst = static_cast<T*>(p.y) + static_cast<int64_t>(m) * p.y_stride + n0;
  if (p.y_vec && n0 + 8 <= p.N) {
    *reinterpret_cast<uint4*>(dst) = v;
  } else {
    const T* e = reinterpret_cast<const T*>(&v);
    for (int i = 0; i < 8 && n0 + i < p.N; ++i) dst[i] = e[i];
  }
}

// y[m][n0 .. n0 + 4) = v rounded to T: one 8-byte store where the row is aligned and
// the four columns exist, else element by element up to out_features.
template <typename T>
__device__ __forceinline__ void store_y4(const LinParams& p, int m, int n0, const float (&v)[4]) {
  T* dst = static_cast<T*>(p.y) + static_cast<int64_t>(m) * p.y_stride + n0;
  if (p.y_vec && n0 + 4 <= p.N) {
    uint2 out;
    T* e = reinterpret_cast<T*>(&out);
#pragma unroll
    for (int i = 0; i < 4; ++i) e[i] = Elem<T>::from_f(v[i]);
    *reinterpret_cast<uint2*>(dst) = out;
  } else {
    for (int i = 0; i < 4 && n0 + i < p.N; ++i) dst[i] = Elem<T>::from_f(v[i]);
  }
}

// First row of the tile that CTA j of s sums in the split-K reduction: a multiple of 8
// (whole 16-byte vectors of a y row for the push), every CTA at least 16 rows.
__device__ __forceinline__ int split_row_lo(int j, int s) { return 8 * ((16 * j) / s); }

// The RoPE epilogue's output for activation row m (a token), tile t (a head) and the
// head dims [c, c + n) and [64 + c, 64 + c + n): a holds the product's values (rounded)
// of the first dims, b of the second. q and k heads are rotated as
// rope_kv_append_kernel does (rotate-half, cos/sin rounded to T, every product and sum
// rounded to T); v heads are copied. q goes to q_out, k and v to the pool slot.
template <typename T, int n>
__device__ void rope_store(const LinParams& p, int m, int t, int c, const T (&a)[n],
                           const T (&b)[n]) {
  const RopeAppend& r = p.rope;
  const bool is_q = t < r.hq, is_v = t >= r.hq + r.hkv;
  T* dst;
  if (is_q) {
    dst = static_cast<T*>(r.q_out) + (static_cast<int64_t>(m) * r.hq + t) * 128;
  } else {
    int64_t loc = r.write_loc != nullptr ? r.write_loc[m] : -1;
    if (loc >= r.pool_slots) {
      report(p.status, NSLG_DEV_BAD_SLOT);
      loc = -1;
    }
    if (loc < 0) return;
    const int h = is_v ? t - r.hq - r.hkv : t - r.hq;
    dst = static_cast<T*>(is_v ? r.pool_v : r.pool_k) + (loc * r.hkv + h) * 128;
  }
  alignas(16) T o1[n];
  alignas(16) T o2[n];
  int64_t pos = -1;
  if (!is_v && r.positions != nullptr) {
    pos = r.positions[m];
    if (pos < 0 || pos >= r.table_rows) {   // reported, row left unrotated
      report(p.status, NSLG_DEV_BAD_POSITION);
      pos = -1;
    }
  }
  if (pos < 0) {
#pragma unroll
    for (int i = 0; i < n; ++i) { o1[i] = a[i]; o2[i] = b[i]; }
  } else {
    const float* cs = r.cos_t + pos * 128 + c;
    const float* sn = r.sin_t + pos * 128 + c;
#pragma unroll
    for (int i = 0; i < n; ++i) {
      const float x1 = Elem<T>::to_f(a[i]), x2 = Elem<T>::to_f(b[i]);
      const float c1 = Elem<T>::round(cs[i]), s1 = Elem<T>::round(sn[i]);
      const float c2 = Elem<T>::round(cs[64 + i]), s2 = Elem<T>::round(sn[64 + i]);
      o1[i] = Elem<T>::from_f(__fadd_rn(Elem<T>::round(__fmul_rn(x1, c1)),
                                        Elem<T>::round(__fmul_rn(-x2, s1))));
      o2[i] = Elem<T>::from_f(__fadd_rn(Elem<T>::round(__fmul_rn(x2, c2)),
                                        Elem<T>::round(__fmul_rn(x1, s2))));
    }
  }
  if constexpr (n == 8) {
    *reinterpret_cast<uint4*>(dst + c) = *reinterpret_cast<const uint4*>(o1);
    *reinterpret_cast<uint4*>(dst + 64 + c) = *reinterpret_cast<const uint4*>(o2);
  } else {
    static_assert(n == 4, "4 or 8 dims");
    *reinterpret_cast<uint2*>(dst + c) = *reinterpret_cast<const uint2*>(o1);
    *reinterpret_cast<uint2*>(dst + 64 + c) = *reinterpret_cast<const uint2*>(o2);
  }
}

// SwiGLU mode: CTA j of s owns the output columns [half_lo(j), half_lo(j + 1)) of its
// tile's 64, i.e. gate rows [lo, hi) and up rows [64 + lo, 64 + hi) of the tile.
__device__ __forceinline__ int half_lo(int j, int s) { return 8 * ((8 * j) / s); }

// Rows of the tile (of D, 128) that CTA j sums, and the position of row r among them.
__device__ __forceinline__ int owned_rows(const LinParams& p, int j) {
  return p.paired ? 2 * (half_lo(j + 1, p.splits) - half_lo(j, p.splits))
                  : split_row_lo(j + 1, p.splits) - split_row_lo(j, p.splits);
}

// The CTA of the cluster whose share of the tile's rows holds row r.
__device__ __forceinline__ int split_owner(int r, int s) {
  int o = 0;
  for (int j = 1; j < s; ++j)
    if (split_row_lo(j, s) <= r) o = j;
  return o;
}
__device__ __forceinline__ int half_owner(int c, int s) {
  int o = 0;
  for (int j = 1; j < s; ++j)
    if (half_lo(j, s) <= c) o = j;
  return o;
}

// Address of this CTA's shared-memory word `local` in the shared memory of cluster CTA
// `rank`.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}

// 4-byte store into another cluster CTA's shared memory that counts 4 bytes of
// transaction on that CTA's mbarrier `bar` when it lands (both cluster addresses).
__device__ __forceinline__ void st_async_f32(uint32_t addr, float v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(
                   addr),
               "r"(__float_as_uint(v)), "r"(bar)
               : "memory");
}

__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}

// Bounded wait (the same limit as mbar_wait) for a phase completed by other CTAs'
// st.async transactions: acquire at cluster scope, so their stores are visible.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = global_ns();
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    if (global_ns() - t0 > kWaitLimitNs) return false;
  }
}

__device__ __forceinline__ void st_sys_v4(void* ptr, uint32_t a, uint32_t b, uint32_t c,
                                          uint32_t d) {
  asm volatile("st.relaxed.sys.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(ptr), "r"(a),
               "r"(b), "r"(c), "r"(d)
               : "memory");
}

// The push of a fused RowParallel product: the rows [r_lo, r_hi) of tile t of y that
// this CTA wrote, for every activation row m, go to every peer's stage buffer as this
// rank's partial of the one-shot reduction that tp_allreduce.cu runs next (source
// region `rank` of slot call & 1, row m, 16-byte vector n / 8), packed as that kernel
// reads them: {d0, call, d1, call} per 16-byte store, call = this rank's counter word of
// the reduction block that owns row m, plus one. Plain stores over NVLink (no multicast,
// no loads from peer memory); nothing waits here: the reduction kernel polls for the
// words.
template <typename T>
__device__ void push_rows(const LinParams& p, int t, int r_lo, int r_hi) {
  const int nvec = (r_hi - r_lo) / 8;
  const int64_t units_per_row = 2 * static_cast<int64_t>(p.N / 8);
  const T* y = static_cast<const T*>(p.y);
  for (int u = threadIdx.x; u < p.M * nvec; u += kThreads) {
    const int m = u / nvec;
    const int n = t * kTileN + r_lo + 8 * (u % nvec);
    if (n >= p.N) continue;
    const uint4 v =
        __ldcg(reinterpret_cast<const uint4*>(y + static_cast<int64_t>(m) * p.y_stride + n));
    const uint32_t call =
        *reinterpret_cast<const volatile uint32_t*>(p.push.counters + m % kTpReduceGrid) + 1u;
    const int64_t off = static_cast<int64_t>(call & 1u) * p.push.slot_bytes +
                        p.push.rank * p.push.region_bytes +
                        (static_cast<int64_t>(m) * units_per_row + 2 * (n / 8)) * 16;
    for (int d = 0; d < p.push.world; ++d) {
      if (d == p.push.rank) continue;
      uint8_t* dst = p.push.stage[d] + off;
      st_sys_v4(dst, v.x, call, v.y, call);
      st_sys_v4(dst + 16, v.z, call, v.w, call);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 2)
    linear_tc_kernel(const __grid_constant__ CUtensorMap tmap_w,
                     const __grid_constant__ CUtensorMap tmap_w2,
                     const __grid_constant__ CUtensorMap tmap_x, const LinParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int sbytes = kWBytes + p.Mp * 128;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.stages * sbytes);
  uint64_t* empty = full + kMaxStages;
  uint64_t* acc_full = empty + kMaxStages;
  uint64_t* mma_drain = acc_full + 1;
  uint64_t* recv_full = mma_drain + 1;            // push_sum: every partial row has landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* partial = reinterpret_cast<float*>(smem);   // [Mp][kPartStride], over the stage ring
  // push_sum: [s][M][rows of this CTA's share] received partials, after the barriers
  float* recv = reinterpret_cast<float*>(smem + p.stages * sbytes + 256);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int t = blockIdx.x / p.splits;            // tile
  const int j = blockIdx.x - t * p.splits;        // split of its K range
  const int k_lo = p.kc * j / p.splits, k_hi = p.kc * (j + 1) / p.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(mma_drain, 1);
    mbar_init(recv_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
    if (p.push_sum)   // every CTA of the cluster sends its partial of this CTA's rows
      mbar_arrive_expect_tx(recv_full,
                            static_cast<uint32_t>(p.splits * p.M * 4 * owned_rows(p, j)));
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
  // push_sum: the receive barriers of the cluster are armed once every CTA has passed
  // this arrive; senders wait for it before their first remote store
  if (p.push_sum) cluster_arrive_release();
  pdl_trigger();     // the next kernel may start its prologue; it waits for our completion

  if (warp == 0) {
    // -------------------------------------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&tmap_w);
      if (p.swiglu) prefetch_tmap(&tmap_w2);
      prefetch_tmap(&tmap_x);
      const uint64_t stream_w = l2_policy_evict_first();   // every weight byte used once
      const uint64_t keep_x = l2_policy_evict_last();      // x is re-read by every CTA
      const int n = k_hi - k_lo;
      const int pre = n < p.stages ? n : p.stages;
      for (int i = 0; i < pre; ++i) {                 // first use of stages 0 .. pre-1
        mbar_arrive_expect_tx(&full[i], sbytes);
        if (p.swiglu) {   // gate rows into the A tile's first 64 rows, up rows below
          tma_load_3d(smem + i * sbytes, &tmap_w, &full[i], (k_lo + i) * kChunk, t * 64, 0,
                      stream_w);
          tma_load_3d(smem + i * sbytes + kWBytes / 2, &tmap_w2, &full[i], (k_lo + i) * kChunk,
                      t * 64, 0, stream_w);
        } else {
          tma_load_3d(smem + i * sbytes, &tmap_w, &full[i], (k_lo + i) * kChunk, t * kTileN, 0,
                      stream_w);
        }
      }
      pdl_wait();      // x is the previous kernel's output
      for (int i = 0; i < pre; ++i)
        tma_load_3d(smem + i * sbytes + kWBytes, &tmap_x, &full[i], (k_lo + i) * kChunk, 0, 0,
                    keep_x);
      int stage = pre % p.stages;
      uint32_t phase = pre == p.stages ? 1u : 0u;
      int issued = pre;
      bool ok = true;
      for (int k = k_lo + pre; k < k_hi; ++k) {
        if (*abort_flag || !mbar_wait(&empty[stage], phase ^ 1)) { ok = false; break; }
        uint8_t* sb = smem + stage * sbytes;
        mbar_arrive_expect_tx(&full[stage], sbytes);
        if (p.swiglu) {
          tma_load_3d(sb, &tmap_w, &full[stage], k * kChunk, t * 64, 0, stream_w);
          tma_load_3d(sb + kWBytes / 2, &tmap_w2, &full[stage], k * kChunk, t * 64, 0, stream_w);
        } else {
          tma_load_3d(sb, &tmap_w, &full[stage], k * kChunk, t * kTileN, 0, stream_w);
        }
        tma_load_3d(sb + kWBytes, &tmap_x, &full[stage], k * kChunk, 0, 0, keep_x);
        ++issued;
        if (++stage == p.stages) { stage = 0; phase ^= 1; }
      }
      if (!ok) {
        report(p.status, NSLG_DEV_WAIT_TIMEOUT);
        *abort_flag = 1;
        // no load may still be writing shared memory when the CTA leaves (bounded)
        for (int u = issued - p.stages < 0 ? 0 : issued - p.stages; u < issued; ++u)
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
      for (int k = k_lo; k < k_hi; ++k) {
        if (*abort_flag || !(ok = mbar_wait(&full[stage], phase))) break;
        tc_fence_after();
        const uint32_t w_lo = lo0 + (stage * sbytes >> 4);
        const uint32_t x_lo = lo0 + ((stage * sbytes + kWBytes) >> 4);
#pragma unroll
        for (int ks = 0; ks < kChunk / 16; ++ks)
          mma_ss_w(tmem, w_lo + ks * 2, x_lo + ks * 2, kDescHi, idesc,
                   (k == k_lo && ks == 0) ? 0u : 1u);
        mma_commit(&empty[stage]);
        if (++stage == p.stages) { stage = 0; phase ^= 1; }
      }
      if (ok) {
        mma_commit(acc_full);
      } else {
        report(p.status, NSLG_DEV_WAIT_TIMEOUT);
        *abort_flag = 1;
      }
      // every MMA issued so far has completed once this arrives (bounded wait)
      mma_commit(mma_drain);
      (void)mbar_wait(mma_drain, 0);
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------- epilogue
    if (p.push_sum) cluster_wait_acquire();
    const int r = (warp & 3) * 32 + lane;          // TMEM lane = row of the tile
    // push_sum: the owner of row r, and where this CTA's values of row r go there
    // (SwiGLU: the owner of output column r % 64 takes gate row r and up row r + 64;
    // its rows are [its gate rows, its up rows])
    const int own = !p.push_sum ? 0
                    : p.paired  ? half_owner(r & 63, p.splits)
                                : split_owner(r, p.splits);
    const int own_rows = owned_rows(p, own);
    int own_pos;
    if (p.paired) {
      const int lo = half_lo(own, p.splits);
      own_pos = (r < 64 ? 0 : own_rows / 2) + (r & 63) - lo;
    } else {
      own_pos = r - split_row_lo(own, p.splits);
    }
    const uint32_t dst0 =
        p.push_sum ? cluster_addr(smem_u32(recv) + 4u * static_cast<uint32_t>(
                                                           j * p.M * own_rows + own_pos),
                                  own)
                   : 0u;
    const uint32_t dst_bar = p.push_sum ? cluster_addr(smem_u32(recv_full), own) : 0u;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0));
    if (!ok) {
      if (lane == 0) report(p.status, NSLG_DEV_WAIT_TIMEOUT);
      *abort_flag = 1;
    }
    if (ok) {
      tc_fence_after();
      // this thread's row of D, 32 columns (activation rows) per wait, into shared
      // memory: the rounded y tile [Mp][128] (splits == 1) or the fp32 partial tile
      // [Mp][128]; each store instruction of a warp covers 32 consecutive tile rows
      T* tile_y = reinterpret_cast<T*>(smem);
      for (int c0 = 0; c0 < p.Mp; c0 += 32) {
        float v[32];
        tmem_ld16(lane_base + c0, *reinterpret_cast<float(*)[16]>(v));
        if (c0 + 16 < p.Mp) tmem_ld16(lane_base + c0 + 16, *reinterpret_cast<float(*)[16]>(v + 16));
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 32; ++q) {
          const int m = c0 + q;
          if (m >= p.M) break;
          if (p.splits == 1)
            tile_y[m * kTileN + r] = Elem<T>::from_f(v[q]);
          else if (p.push_sum)
            st_async_f32(dst0 + 4u * static_cast<uint32_t>(m * own_rows), v[q], dst_bar);
          else
            partial[m * kPartStride + r] = v[q];
        }
      }
    }
  }

  if (p.push_sum && warp < 4) cluster_wait_acquire();
  tc_fence_before();
  __syncthreads();
  if (p.splits == 1) {
    // the staged tile to y, 8 consecutive outputs (16 bytes) of one row per store
    if (!*abort_flag && p.rope.on) {
      // head t of token m: dims c.. and 64 + c.. of the staged tile, rotated, stored
      const T* tile_y = reinterpret_cast<const T*>(smem);
      for (int u = threadIdx.x; u < p.M * 8; u += kThreads) {
        const int m = u / 8, c = 8 * (u % 8);
        alignas(16) T a[8];
        alignas(16) T b[8];
        *reinterpret_cast<uint4*>(a) = *reinterpret_cast<const uint4*>(tile_y + m * kTileN + c);
        *reinterpret_cast<uint4*>(b) =
            *reinterpret_cast<const uint4*>(tile_y + m * kTileN + 64 + c);
        rope_store<T, 8>(p, m, t, c, a, b);
      }
    } else if (!*abort_flag && p.swiglu) {
      // y[m][64t + c] = silu(gate) * up from rows c and 64 + c of the staged tile
      const T* tile_y = reinterpret_cast<const T*>(smem);
      for (int u = threadIdx.x; u < p.M * 8; u += kThreads) {
        const int m = u / 8, c = 8 * (u % 8);
        const uint4 g = *reinterpret_cast<const uint4*>(tile_y + m * kTileN + c);
        const uint4 up = *reinterpret_cast<const uint4*>(tile_y + m * kTileN + 64 + c);
        uint4 o;
        const T* ge = reinterpret_cast<const T*>(&g);
        const T* ue = reinterpret_cast<const T*>(&up);
        T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
        for (int i = 0; i < 8; ++i) oe[i] = swiglu<T>(ge[i], ue[i]);
        store_y8<T>(p, m, t * 64 + c, o);
      }
    } else if (!*abort_flag) {
      const T* tile_y = reinterpret_cast<const T*>(smem);
      for (int u = threadIdx.x; u < p.M * (kTileN / 8); u += kThreads) {
        const int m = u / (kTileN / 8), c = 8 * (u % (kTileN / 8));
        store_y8<T>(p, m, t * kTileN + c, *reinterpret_cast<const uint4*>(tile_y + m * kTileN + c));
      }
    }
  } else if (p.push_sum) {
    // this CTA's rows of the tile: wait (bounded) for the s partials to land, sum them
    // in split order (the order of the pulled sum below), round once, store
    const bool landed = mbar_wait_cluster(recv_full, 0);
    if (!landed) {
      if (threadIdx.x == 0) report(p.status, NSLG_DEV_WAIT_TIMEOUT);
    } else if (!*abort_flag && p.paired) {
      // sums of this CTA's rows [lo, hi) and [64 + lo, 64 + hi) of the tile (gate and
      // up, or the two halves of a head), rounded, then activated or rotated
      const int lo = half_lo(j, p.splits);
      const int h = half_lo(j + 1, p.splits) - lo;
      const int quads = h / 4;
      for (int e = threadIdx.x; e < p.M * quads; e += kThreads) {
        const int m = e / quads, q4 = 4 * (e % quads);
        float g[4] = {0.f, 0.f, 0.f, 0.f}, u[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int sp = 0; sp < kMaxSplits; ++sp) {
          const float* row = recv + (sp * p.M + m) * 2 * h;
          const float4 a = sp < p.splits ? *reinterpret_cast<const float4*>(row + q4)
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
          const float4 b = sp < p.splits ? *reinterpret_cast<const float4*>(row + h + q4)
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
          g[0] += a.x; g[1] += a.y; g[2] += a.z; g[3] += a.w;
          u[0] += b.x; u[1] += b.y; u[2] += b.z; u[3] += b.w;
        }
        if (p.rope.on) {
          alignas(16) T a[4];
          alignas(16) T b[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            a[i] = Elem<T>::from_f(g[i]);
            b[i] = Elem<T>::from_f(u[i]);
          }
          rope_store<T, 4>(p, m, t, lo + q4, a, b);
        } else {
          float o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            o[i] = Elem<T>::to_f(swiglu<T>(Elem<T>::from_f(g[i]), Elem<T>::from_f(u[i])));
          store_y4<T>(p, m, t * 64 + lo + q4, o);
        }
      }
    } else if (!*abort_flag) {
      const int r_lo = split_row_lo(j, p.splits);
      const int rows_s = split_row_lo(j + 1, p.splits) - r_lo;
      const int quads = rows_s / 4;
      for (int e = threadIdx.x; e < p.M * quads; e += kThreads) {
        const int m = e / quads, q4 = 4 * (e % quads);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int sp = 0; sp < kMaxSplits; ++sp) {
          const float4 a = sp < p.splits ? *reinterpret_cast<const float4*>(
                                               recv + (sp * p.M + m) * rows_s + q4)
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
          acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
        }
        store_y4<T>(p, m, t * kTileN + r_lo + q4, acc);
      }
    }
  } else {
    // split-K sum across the cluster (the s CTAs of this tile) through distributed
    // shared memory; rank order = split order. Unit = 4 consecutive rows of the tile for
    // one activation row m: one 16-byte load from each of the s partials, all issued
    // before the sum, one 8-byte store of y. With 32 or 16 rows per CTA (s = 4, 8) the
    // eight threads of a quarter warp read 128 bytes of one row m, or 64 of each of
    // two rows m 16 banks apart (the padded row stride): one wavefront per quarter warp.
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();                                 // every partial is staged
    if (!*abort_flag) {
      const int r_lo = split_row_lo(j, p.splits);
      const int quads = (split_row_lo(j + 1, p.splits) - r_lo) / 4;
      const float* src[kMaxSplits];
#pragma unroll
      for (int sp = 0; sp < kMaxSplits; ++sp)
        src[sp] = cluster.map_shared_rank(partial, sp < p.splits ? sp : 0);
      for (int e = threadIdx.x; e < p.M * quads; e += kThreads) {
        const int m = e / quads, row = r_lo + 4 * (e % quads);
        float4 a[kMaxSplits];
#pragma unroll
        for (int sp = 0; sp < kMaxSplits; ++sp)
          a[sp] = sp < p.splits
                      ? *reinterpret_cast<const float4*>(src[sp] + m * kPartStride + row)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int sp = 0; sp < kMaxSplits; ++sp) {
          acc[0] += a[sp].x; acc[1] += a[sp].y; acc[2] += a[sp].z; acc[3] += a[sp].w;
        }
        store_y4<T>(p, m, t * kTileN + row, acc);
      }
    }
    cluster.sync();                                 // no partial is read any more
  }
  if (p.do_push) {
    __syncthreads();      // y's rows of this CTA are written (read back through L2)
    if (!*abort_flag)
      push_rows<T>(p, t, p.splits == 1 ? 0 : split_row_lo(j, p.splits),
                   p.splits == 1 ? kTileN : split_row_lo(j + 1, p.splits));
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(p.tmem_cols)
                 : "memory");
  }
}

struct Plan {
  int Mp, n_tiles, kc, splits, grid, stages, tmem_cols, push_sum, recv_bytes;
};

// Split policy overrides, for measurements: NSLG_LINEAR_CTAS_PER_SM (1 or 2: the grid
// may fill the SMs once or twice over with K splits), NSLG_LINEAR_MIN_CHUNKS (the
// fewest 64-element K chunks a split may have, 1 to 64), NSLG_LINEAR_SPLITS (1 to 8
// splits per tile, at most one per chunk, instead of the rule) and NSLG_LINEAR_PUSH_SUM
// (0: the pulled split-K sum at every batch size).
int env_int(const char* name, int dflt, int lo, int hi) {
  const char* e = std::getenv(name);
  if (e == nullptr || e[0] == '\0') return dflt;
  const int v = std::atoi(e);
  return v < lo ? lo : (v > hi ? hi : v);
}

size_t smem_bytes(int stages, int Mp, int recv_bytes) {
  return 1024 + static_cast<size_t>(stages) * (kWBytes + Mp * 128) + 256 + recv_bytes;
}

int stages_for(int Mp, int recv_bytes) {
  const int st = (kLinearSmemBudget - recv_bytes) / (kWBytes + Mp * 128);
  return st < kMinStages ? kMinStages : (st > kMaxStages ? kMaxStages : st);
}

// Receive buffer of a pushed split-K sum: s partials of the largest row share (SwiGLU
// mode: twice the largest share of the tile's 64 output columns).
int recv_bytes_for(int splits, int Mp, bool paired) {
  int rows = 0;
  for (int j = 0; j < splits; ++j) {
    const int r = paired ? 2 * (8 * ((8 * (j + 1)) / splits) - 8 * ((8 * j) / splits))
                         : 8 * ((16 * (j + 1)) / splits) - 8 * ((16 * j) / splits);
    rows = r > rows ? r : rows;
  }
  return splits * Mp * rows * 4;
}

// Splits per tile: as many as fill the SMs `cps` times over (two CTAs fit on an SM),
// at most kMaxSplits and at least kMinChunksPerSplit chunks each. When the grid takes
// more than one CTA per SM the cluster size is rounded down to a power of two, so that
// the clusters pack into the GPCs' CTA slots in one wave (measured on the 8B q|k|v
// product at one row: 48 clusters of 6, 288 CTAs, 15.7 us; of 3, 144 CTAs, 12.3 us).
Plan plan_for(int M, int N, int K, bool swiglu, bool paired) {
  Plan pl{};
  pl.Mp = (M + 15) / 16 * 16;
  // a tile is 128 weight rows: 128 outputs, or 64 gate|up pairs (SwiGLU)
  pl.n_tiles = swiglu ? (N + 63) / 64 : (N + kTileN - 1) / kTileN;
  pl.kc = K / kChunk;
  const int cps = env_int("NSLG_LINEAR_CTAS_PER_SM", kCtasPerSm, 1, 2);
  int s = sm_count() * cps / pl.n_tiles;
  int s_max = pl.kc / env_int("NSLG_LINEAR_MIN_CHUNKS", kMinChunksPerSplit, 1, 64);
  if (s_max > kMaxSplits) s_max = kMaxSplits;
  if (s > s_max) s = s_max;
  if (s < 1) s = 1;
  if (pl.n_tiles * s > sm_count())
    while (s & (s - 1)) --s;                   // a power of two
  const int forced = env_int("NSLG_LINEAR_SPLITS", 0, 0, kMaxSplits);
  if (forced > 0) s = forced <= pl.kc ? forced : pl.kc;
  pl.splits = s;
  pl.grid = pl.n_tiles * s;
  pl.push_sum = (s > 1 && pl.Mp <= kPushMaxMp && env_int("NSLG_LINEAR_PUSH_SUM", 1, 0, 1) &&
                 recv_bytes_for(s, pl.Mp, paired) + kMinStages * (kWBytes + pl.Mp * 128) <=
                     kLinearSmemBudget)
                    ? 1
                    : 0;
  pl.recv_bytes = pl.push_sum ? recv_bytes_for(s, pl.Mp, paired) : 0;
  pl.stages = stages_for(pl.Mp, pl.recv_bytes);
  int cols = 32;
  while (cols < pl.Mp) cols *= 2;
  pl.tmem_cols = cols;
  return pl;
}

}  // namespace

bool linear_tc_supported(int dtype, int M, int N, int K) {
  return (dtype == NSLG_DTYPE_BF16 || dtype == NSLG_DTYPE_F16) && M >= 1 && M <= kLinearMaxRows &&
         N >= 1 && N <= kMaxTiles * kTileN && K >= kChunk && K % kChunk == 0;
}

int launch_linear_tc(int dtype, int M, int N, int K, const void* x, int64_t x_stride,
                     const void* w, int64_t w_stride, void* y, int64_t y_stride,
                     const TpPush* push, uint32_t* status, cudaStream_t stream, bool swiglu,
                     const LinearRope* rope) {
  const bool paired = swiglu || rope != nullptr;
  const Plan pl = plan_for(M, N, K, swiglu, paired);
  if (paired && (push != nullptr || (pl.splits > 1 && !pl.push_sum)))
    return set_error(NSLG_ERR_UNSUPPORTED,
                     std::string(swiglu ? "linear_swiglu" : "linear_rope_append") +
                         ": the split-K sum of this shape does not fit the push");
  CUtensorMap tw, tw2, tx;
  // W [N, K] and x [M, K], K innermost; boxes [64 x 128] and [64 x Mp] with 128-byte
  // swizzle. SwiGLU: W is [2N, K] (gate rows, then up rows), one map per half, each with
  // N rows (so a ragged last tile reads zeros, not the other half) and [64 x 64] boxes.
  int rc;
  if (swiglu) {
    const uint64_t sb = static_cast<uint64_t>(w_stride) * 2;
    rc = encode_tiled_3d_bf16(&tw, w, K, N, 1, sb, sb * N, kChunk, 64, 1);
    if (rc != NSLG_OK) return rc;
    rc = encode_tiled_3d_bf16(&tw2, static_cast<const uint8_t*>(w) + sb * N, K, N, 1, sb, sb * N,
                              kChunk, 64, 1);
  } else {
    rc = encode_tiled_3d_bf16(&tw, w, K, N, 1, static_cast<uint64_t>(w_stride) * 2,
                              static_cast<uint64_t>(w_stride) * 2 * N, kChunk, kTileN, 1);
    tw2 = tw;
  }
  if (rc != NSLG_OK) return rc;
  rc = encode_tiled_3d_bf16(&tx, x, K, M, 1, static_cast<uint64_t>(x_stride) * 2,
                            static_cast<uint64_t>(x_stride) * 2 * M, kChunk, pl.Mp, 1);
  if (rc != NSLG_OK) return rc;
  LinParams p{};
  p.y = y;
  p.y_stride = y_stride;
  p.M = M;
  p.N = N;
  p.Mp = pl.Mp;
  p.kc = pl.kc;
  p.splits = pl.splits;
  p.stages = pl.stages;
  p.tmem_cols = pl.tmem_cols;
  p.do_push = push != nullptr ? 1 : 0;
  p.y_vec = (reinterpret_cast<uintptr_t>(y) % 16 == 0 && y_stride % 8 == 0) ? 1 : 0;
  p.push_sum = pl.push_sum;
  p.swiglu = swiglu ? 1 : 0;
  p.paired = paired ? 1 : 0;
  if (rope != nullptr) {
    p.rope.on = 1;
    p.rope.hq = rope->hq;
    p.rope.hkv = rope->hkv;
    p.rope.q_out = rope->q_out;
    p.rope.positions = rope->positions;
    p.rope.cos_t = rope->cos_t;
    p.rope.sin_t = rope->sin_t;
    p.rope.table_rows = rope->table_rows;
    p.rope.write_loc = rope->write_loc;
    p.rope.pool_k = rope->pool_k;
    p.rope.pool_v = rope->pool_v;
    p.rope.pool_slots = rope->pool_slots;
  }
  if (push != nullptr) p.push = *push;
  p.status = status;
  const size_t smem = smem_bytes(pl.stages, pl.Mp, pl.recv_bytes);
  auto kern = dtype == NSLG_DTYPE_F16 ? linear_tc_kernel<__half> : linear_tc_kernel<__nv_bfloat16>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return set_error(NSLG_ERR_CUDA, cudaGetErrorString(err));
  // one cluster per tile (its K splits), launched with programmatic dependent launch
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = pl.splits;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  err = cudaLaunchKernelEx(&cfg, kern, tw, tw2, tx, p);
  if (err != cudaSuccess) return set_error(NSLG_ERR_CUDA, std::string("linear_tc: ") + cudaGetErrorString(err));
  return check_launch("linear_tc");
}

}  // namespace nslg
