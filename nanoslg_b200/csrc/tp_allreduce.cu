// Tensor-parallel all-reduce fused with the residual add and RMSNorm that follow it,
// over peer memory (CUDA IPC mappings across NVLink / NVSwitch), and the IPC helpers
// that set the peer memory up.
//
// Replaces, for the rows of one decode step, RowParallelLinear's NCCL all-reduce
// (tp_layers.py:148-158 -> parallel.py:167-172) and the block's residual add + RMSNorm
// (models.py:169-172, 25-34): one kernel per RowParallel output instead of an NCCL
// all-reduce, an add and a norm.
//
// Protocol: one-shot push with flags inside the data ("low-latency" packing). Each
// 16-byte store carries 8 bytes of activations and, in each of its 8-byte halves, the
// 32-bit call number: {d0, call, d1, call}. An 8-byte store is single-copy atomic, so a
// reader that sees the call number in both halves has both data words of this call; no
// fence and no separate flag are needed, and the only cross-GPU latency on the critical
// path is one NVLink write. Rank r writes its partial rows into slot (call & 1), source
// region r, of every peer's stage buffer; each rank then polls its own buffer (local
// memory) for the other ranks' words, sums all ranks' rows in fp32 in rank order (its
// own partial read directly), rounds once to the activation type (one NCCL bf16 sum of
// two ranks rounds the same way), adds the residual (rounded), stores the new residual,
// and writes weight * round(h * rsqrt(mean(h^2) + eps)) as the rmsnorm kernel does.
//
// Calls are numbered per block: block b keeps its call count in this rank's counter
// buffer (word b) and the grid is always kGrid blocks, so block b of every rank sees
// the same sequence of call numbers (every rank makes the same calls). The count lives
// in device memory, so the launch can be captured in a CUDA graph and replayed. Two
// slots suffice: a peer can be at most one call ahead (its call e + 1 needs this rank's
// words of call e + 1, written only after this rank finished call e), and words left
// from call e - 1 carry another call number.
//
// Two-shot mode, for many rows on many ranks: the one-shot push sends world - 1 copies of
// every row out of each GPU, which at TP=8 and 64 rows is 7 MiB per call (packed). The
// two-shot mode splits each row into `world` column slices: rank r sends slice j of its
// partial rows to rank j only (reduce-scatter), rank j sums slice j over the ranks in
// the same fp32 rank order and rounds it once, then pushes the reduced slice to every
// rank (all-gather); each rank then has the whole reduced row and does the residual add
// and RMSNorm as before. Results are identical to the one-shot mode's; each rank sends
// 2 (world - 1) / world of a row instead of world - 1 rows, for a second NVLink round
// trip. Both phases use the same in-band call numbers, so the mode may change from call
// to call. The mode is chosen per call by size (kTwoShotSavingBytes) unless
// NSLG_TP_TWO_SHOT forces one; both were checked bit for bit with every rank of a group
// of 2, 4 and 8 emulated in one cooperative grid on one GPU (nslg_tp_allreduce_rmsnorm_
// emulated, which runs this same kernel).
//
// Stage buffer of each rank: [2 slots][world sources][rows][2 x row bytes] (the packed
// rows are twice the activations); in two-shot mode a slot holds [2 phases][world
// sources][rows][2 x slice bytes] instead. Every wait is bounded by `timeout_ns` of
// %globaltimer; a block that gives up records NSLG_DEV_WAIT_TIMEOUT and leaves its rows
// unwritten, so the context stays usable.
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <string>

#include "common.cuh"
#include "launch.h"

namespace nslg {
namespace {

constexpr int kGrid = kTpReduceGrid;   // blocks per call, the same on every rank and call
constexpr int kThreads = 256;
constexpr int kVecPerThread = 4;    // 16-byte vectors of a row per thread (hidden <= 8192 bf16)
// Two-shot sends 2 (world - 2) / world x the one-shot's bytes fewer out of each GPU but
// adds a second NVLink round trip: it is chosen when the packed bytes it saves exceed
// kTwoShotSavingBytes. Measured at TP=4 on B200 (8 KiB rows, CUDA-graph loops, max over
// ranks): one-shot 7.5 / 14.1 / 40.3 us, two-shot 7.9 / 9.5 / 20.5 us at 1 / 64 / 256
// rows, i.e. the second round trip costs about 0.4 us and two-shot wins from about 5
// rows (~120 KB saved).
constexpr int64_t kTwoShotSavingBytes = 128 << 10;

// NSLG_TP_TWO_SHOT, read at every call: "0" -> one-shot, "1" -> two-shot (where the shape
// allows it), unset or anything else ("auto") -> -1, chosen by size
int two_shot_override() {
  const char* e = getenv("NSLG_TP_TWO_SHOT");
  if (e == nullptr || e[0] == '\0') return -1;
  if (strcmp(e, "0") == 0) return 0;
  if (strcmp(e, "1") == 0) return 1;
  return -1;
}
static_assert(kGrid * 4 <= NSLG_TP_COUNTER_BYTES, "counter buffer too small");

struct ArParams {
  const void* partial;
  int64_t p_stride;
  uint8_t* stage[NSLG_TP_MAX_WORLD];
  int64_t slot_bytes, region_bytes;
  uint32_t* counters;
  void* residual;
  int64_t r_stride;
  const void* weight;
  void* out;
  int64_t o_stride;
  int rows, hidden, world, rank, two_shot;
  int pushed;       // phase 1 already done by the producer (nslg_linear_tp_push)
  float eps;
  uint64_t timeout_ns;
  uint32_t* status;
  // Every rank of the group in one cooperative grid on one GPU (nslg_tp_allreduce_
  // rmsnorm_emulated): blocks [r * e_grid, (r + 1) * e_grid) are rank r, with its own
  // partial, residual, output and counters; the scalar fields above are then unused.
  int emulate, e_grid;
  const void* e_partial[NSLG_TP_MAX_WORLD];
  void* e_residual[NSLG_TP_MAX_WORLD];
  void* e_out[NSLG_TP_MAX_WORLD];
  uint32_t* e_counters[NSLG_TP_MAX_WORLD];
};

__device__ __forceinline__ void st_relaxed_v4(void* p, uint4 v) {
  asm volatile("st.relaxed.sys.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_relaxed_v4(const void* p) {
  uint4 v;
  asm volatile("ld.relaxed.sys.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

template <typename T, int VEC>
union NVec {
  uint4 u;
  T e[VEC];
};

template <typename T>
__global__ void __launch_bounds__(kThreads) tp_allreduce_rmsnorm_kernel(const ArParams p) {
  pdl_wait();      // the partial is the previous kernel's output
  pdl_trigger();
  constexpr int VEC = 16 / sizeof(T);
  const int nv = p.hidden / VEC;                  // 16-byte vectors per row
  const int64_t units_per_row = 2 * static_cast<int64_t>(nv);
  // this block's rank, its index among the rank's blocks, and the rank's buffers
  const int nblk = p.emulate ? p.e_grid : static_cast<int>(gridDim.x);
  const int rank = p.emulate ? static_cast<int>(blockIdx.x) / nblk : p.rank;
  const int bid = p.emulate ? static_cast<int>(blockIdx.x) % nblk : static_cast<int>(blockIdx.x);
  const void* partial = p.emulate ? p.e_partial[rank] : p.partial;
  void* residual = p.emulate ? p.e_residual[rank] : p.residual;
  void* out_rows = p.emulate ? p.e_out[rank] : p.out;
  uint32_t* counter = (p.emulate ? p.e_counters[rank] : p.counters) + bid;
  const uint32_t call = *reinterpret_cast<volatile uint32_t*>(counter) + 1;
  const int64_t slot_off = (call & 1u) * p.slot_bytes;
  __shared__ volatile int bad;      // a wait of this block gave up: the others stop too
  __shared__ float red[kThreads / 32];
  if (threadIdx.x == 0) bad = 0;

  // Polls the packed 32-byte unit at q until both of its 16-byte halves carry this call
  // number (bounded); returns its 16 data bytes. On a timeout sets `bad` (the block's
  // other threads stop polling too) and records NSLG_DEV_WAIT_TIMEOUT.
  // Second half of a fetch: (a, b) were loaded from q already (the caller issues the
  // loads of a whole set of units first, so they cost one memory latency together rather
  // than one each); polls q again only if they did not carry this call's number yet.
  auto settle = [&](const uint4* q, uint4& a, uint4& b) {
    if (!(a.y == call && a.w == call && b.y == call && b.w == call)) {
      const uint64_t t0 = global_ns();
      while (true) {
        a = ld_relaxed_v4(q);
        b = ld_relaxed_v4(q + 1);
        if (a.y == call && a.w == call && b.y == call && b.w == call) break;
        if (bad) break;
        if (global_ns() - t0 > p.timeout_ns) {
          bad = 1;
          report(p.status, NSLG_DEV_WAIT_TIMEOUT);
          break;
        }
      }
    }
  };
  auto push = [&](uint4* dst, const uint4 v) {
    st_relaxed_v4(dst, make_uint4(v.x, call, v.y, call));
    st_relaxed_v4(dst + 1, make_uint4(v.z, call, v.w, call));
  };
  // two-shot layout of a slot, per phase and source rank: [rows][2 * nvs] packed units
  const int nvs = nv / p.world;                   // 16-byte vectors per column slice
  const int64_t units_src = 2 * static_cast<int64_t>(p.rows) * nvs;

  // 1. push this rank's partial rows, packed with the call number: one-shot, the whole
  //    row to every peer; two-shot, column slice j of the row to rank j only
  for (int row = p.pushed ? p.rows : bid; row < p.rows; row += nblk) {
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const T*>(partial) +
                                                      row * p.p_stride);
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
      const uint4 v = src[i];
      if (p.two_shot) {
        const int j = i / nvs;
        if (j == rank) continue;
        push(reinterpret_cast<uint4*>(p.stage[j] + slot_off) + rank * units_src +
                 row * 2 * nvs + 2 * (i - j * nvs), v);
        continue;
      }
      for (int d = 0; d < p.world; ++d) {
        if (d == rank) continue;
        push(reinterpret_cast<uint4*>(p.stage[d] + slot_off + rank * p.region_bytes) +
                 row * units_per_row + 2 * i, v);
      }
    }
  }
  __syncthreads();   // `bad` is initialised before anyone can set it

  // 2. per row: wait for and sum every rank's words, then residual add and RMSNorm
  const T* w = static_cast<const T*>(p.weight);
  for (int row = bid; row < p.rows; row += nblk) {
    const uint4* mine = reinterpret_cast<const uint4*>(static_cast<const T*>(partial) +
                                                       row * p.p_stride);
    const uint4* own = reinterpret_cast<const uint4*>(p.stage[rank] + slot_off);
    float acc[kVecPerThread][VEC];
    if (p.two_shot) {
      // 2a. reduce this rank's column slice over the ranks (fp32, rank order, one
      //     rounding) and push the reduced slice to every rank, this one included
      for (int u = threadIdx.x; u < nvs; u += blockDim.x) {
        float a[VEC];
#pragma unroll
        for (int j = 0; j < VEC; ++j) a[j] = 0.f;
        uint4 ua[NSLG_TP_MAX_WORLD], ub[NSLG_TP_MAX_WORLD];
#pragma unroll
        for (int s = 0; s < NSLG_TP_MAX_WORLD; ++s) {
          if (s >= p.world || s == rank) continue;
          const uint4* q = own + s * units_src + row * 2 * nvs + 2 * u;
          ua[s] = ld_relaxed_v4(q);
          ub[s] = ld_relaxed_v4(q + 1);
        }
#pragma unroll
        for (int s = 0; s < NSLG_TP_MAX_WORLD; ++s) {
          if (s >= p.world) continue;
          NVec<T, VEC> v;
          if (s == rank) {
            v.u = mine[rank * nvs + u];
          } else {
            settle(own + s * units_src + row * 2 * nvs + 2 * u, ua[s], ub[s]);
            v.u = make_uint4(ua[s].x, ua[s].z, ub[s].x, ub[s].z);
          }
#pragma unroll
          for (int j = 0; j < VEC; ++j) a[j] = __fadd_rn(a[j], Elem<T>::to_f(v.e[j]));
        }
        if (bad) break;   // never push a slice built from words that did not arrive
        NVec<T, VEC> r;
#pragma unroll
        for (int j = 0; j < VEC; ++j) r.e[j] = Elem<T>::from_f(a[j]);
        for (int d = 0; d < p.world; ++d)
          push(reinterpret_cast<uint4*>(p.stage[d] + slot_off) + (p.world + rank) * units_src +
                   row * 2 * nvs + 2 * u, r.u);
      }
      // 2b. gather the reduced slices of every rank (all loads of the thread first)
      uint4 ua[kVecPerThread], ub[kVecPerThread];
#pragma unroll
      for (int k = 0; k < kVecPerThread; ++k) {
        const int i = threadIdx.x + k * kThreads;
        if (i >= nv) continue;
        const int s = i / nvs;
        const uint4* q = own + (p.world + s) * units_src + row * 2 * nvs + 2 * (i - s * nvs);
        ua[k] = ld_relaxed_v4(q);
        ub[k] = ld_relaxed_v4(q + 1);
      }
#pragma unroll
      for (int k = 0; k < kVecPerThread; ++k) {
        const int i = threadIdx.x + k * kThreads;
#pragma unroll
        for (int j = 0; j < VEC; ++j) acc[k][j] = 0.f;
        if (i >= nv) continue;
        const int s = i / nvs;
        settle(own + (p.world + s) * units_src + row * 2 * nvs + 2 * (i - s * nvs), ua[k], ub[k]);
        NVec<T, VEC> v;
        v.u = make_uint4(ua[k].x, ua[k].z, ub[k].x, ub[k].z);
#pragma unroll
        for (int j = 0; j < VEC; ++j) acc[k][j] = Elem<T>::to_f(v.e[j]);
      }
    } else {
#pragma unroll
      for (int k = 0; k < kVecPerThread; ++k) {
        const int i = threadIdx.x + k * kThreads;
#pragma unroll
        for (int j = 0; j < VEC; ++j) acc[k][j] = 0.f;
        if (i >= nv) continue;
        // every peer's unit of this vector loaded at once, then settled and summed in
        // rank order
        uint4 ua[NSLG_TP_MAX_WORLD], ub[NSLG_TP_MAX_WORLD];
#pragma unroll
        for (int s = 0; s < NSLG_TP_MAX_WORLD; ++s) {
          if (s >= p.world || s == rank) continue;
          const uint4* q = reinterpret_cast<const uint4*>(p.stage[rank] + slot_off +
                                                          s * p.region_bytes) +
                           row * units_per_row + 2 * i;
          ua[s] = ld_relaxed_v4(q);
          ub[s] = ld_relaxed_v4(q + 1);
        }
#pragma unroll
        for (int s = 0; s < NSLG_TP_MAX_WORLD; ++s) {
          if (s >= p.world) continue;
          NVec<T, VEC> v;
          if (s == rank) {
            v.u = mine[i];
          } else {
            const uint4* q = reinterpret_cast<const uint4*>(p.stage[rank] + slot_off +
                                                            s * p.region_bytes) +
                             row * units_per_row + 2 * i;
            settle(q, ua[s], ub[s]);
            v.u = make_uint4(ua[s].x, ua[s].z, ub[s].x, ub[s].z);
          }
#pragma unroll
          for (int j = 0; j < VEC; ++j) acc[k][j] = __fadd_rn(acc[k][j], Elem<T>::to_f(v.e[j]));
        }
      }
    }
    __syncthreads();
    if (bad) break;     // block-uniform: a peer never delivered; nothing is written
    T* res = static_cast<T*>(residual) + row * p.r_stride;
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < kVecPerThread; ++k) {
      const int i = threadIdx.x + k * kThreads;
      if (i >= nv) continue;
      NVec<T, VEC> r;
      r.u = reinterpret_cast<const uint4*>(res)[i];
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float sum = Elem<T>::round(acc[k][j]);              // the all-reduced output
        r.e[j] = Elem<T>::from_f(__fadd_rn(Elem<T>::to_f(r.e[j]), sum));
        const float h = Elem<T>::to_f(r.e[j]);
        ss = fmaf(h, h, ss);
      }
      reinterpret_cast<uint4*>(res)[i] = r.u;
    }
    if (w == nullptr) continue;
    // the same reduction tree as the rmsnorm kernel, so both give the same statistics
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (warp == 0) {
      float v = lane < kThreads / 32 ? red[lane] : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red[0] = v;
    }
    __syncthreads();
    const float inv = rsqrtf(__fadd_rn(__fdiv_rn(red[0], static_cast<float>(p.hidden)), p.eps));
    T* out = static_cast<T*>(out_rows) + row * p.o_stride;
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
      NVec<T, VEC> a, ww, o;
      a.u = reinterpret_cast<const uint4*>(res)[i];
      ww.u = reinterpret_cast<const uint4*>(w)[i];
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float y = Elem<T>::round(__fmul_rn(Elem<T>::to_f(a.e[j]), inv));
        o.e[j] = Elem<T>::from_f(__fmul_rn(Elem<T>::to_f(ww.e[j]), y));
      }
      reinterpret_cast<uint4*>(out)[i] = o.u;
    }
    __syncthreads();   // red[] is rewritten by the next row
  }
  // 3. this block's call count (read by the next launch on this stream)
  if (threadIdx.x == 0) *counter = call;
}

}  // namespace
}  // namespace nslg

using namespace nslg;

extern "C" int nslg_ipc_alloc(int64_t bytes, void** dev_ptr, void* handle_out) {
  if (bytes <= 0 || dev_ptr == nullptr || handle_out == nullptr)
    return set_error(NSLG_ERR_ARG, "ipc_alloc: bytes must be > 0 and pointers non-null");
  void* p = nullptr;
  cudaError_t err = cudaMalloc(&p, static_cast<size_t>(bytes));
  if (err != cudaSuccess) return set_error(NSLG_ERR_CUDA, std::string("ipc_alloc: ") + cudaGetErrorString(err));
  err = cudaMemset(p, 0, static_cast<size_t>(bytes));
  if (err == cudaSuccess) err = cudaDeviceSynchronize();
  if (err == cudaSuccess) err = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle_out), p);
  if (err != cudaSuccess) {
    cudaFree(p);
    return set_error(NSLG_ERR_CUDA, std::string("ipc_alloc: ") + cudaGetErrorString(err));
  }
  *dev_ptr = p;
  return NSLG_OK;
}

extern "C" int nslg_ipc_open(const void* handle, void** dev_ptr) {
  if (handle == nullptr || dev_ptr == nullptr) return set_error(NSLG_ERR_ARG, "ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t err = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) return set_error(NSLG_ERR_CUDA, std::string("ipc_open: ") + cudaGetErrorString(err));
  return NSLG_OK;
}

extern "C" int nslg_ipc_close(void* dev_ptr) {
  const cudaError_t err = cudaIpcCloseMemHandle(dev_ptr);
  if (err != cudaSuccess) return set_error(NSLG_ERR_CUDA, std::string("ipc_close: ") + cudaGetErrorString(err));
  return NSLG_OK;
}

extern "C" int nslg_ipc_free(void* dev_ptr) {
  const cudaError_t err = cudaFree(dev_ptr);
  if (err != cudaSuccess) return set_error(NSLG_ERR_CUDA, std::string("ipc_free: ") + cudaGetErrorString(err));
  return NSLG_OK;
}

namespace {
// Per-rank buffers of a group emulated on one GPU (nslg_tp_allreduce_rmsnorm_emulated).
struct EmulatedRanks {
  const void* const* partials;
  void* const* counters;
  void* const* residuals;
  void* const* outs;
};

template <typename T>
int launch_emulated(ArParams p, int world, cudaStream_t st) {
  // every block of every rank must be resident at once (they wait on one another): the
  // cooperative launch fails, rather than hangs, when they cannot be
  auto kern = tp_allreduce_rmsnorm_kernel<T>;
  int per_sm = 0;
  cudaError_t err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, 0);
  if (err != cudaSuccess) return set_error(NSLG_ERR_CUDA, cudaGetErrorString(err));
  int g = per_sm * sm_count() / world;
  if (g > kGrid) g = kGrid;
  if (g < 1) return set_error(NSLG_ERR_UNSUPPORTED, "tp_allreduce_rmsnorm_emulated: no room");
  p.emulate = 1;
  p.e_grid = g;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(g * world);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  err = cudaLaunchKernelEx(&cfg, kern, p);
  if (err != cudaSuccess)
    return set_error(NSLG_ERR_CUDA, std::string("tp_allreduce_rmsnorm_emulated: ") +
                                        cudaGetErrorString(err));
  return check_launch("tp_allreduce_rmsnorm_emulated");
}

int tp_reduce(int dtype, int rows, int hidden, int world, int rank, const void* partial,
              int64_t partial_stride, void* const* stage_bufs, int64_t stage_bytes,
              void* counters, void* residual, int64_t residual_stride, const void* weight,
              void* out, int64_t out_stride, float eps, int64_t timeout_ns,
              uint32_t* dev_status, void* stream, int pushed,
              const EmulatedRanks* emu = nullptr) {
  if (dtype != NSLG_DTYPE_BF16 && dtype != NSLG_DTYPE_F16 && dtype != NSLG_DTYPE_F32)
    return set_error(NSLG_ERR_ARG, "tp_allreduce_rmsnorm: bad dtype");
  if (world < 2 || world > NSLG_TP_MAX_WORLD || rank < 0 || rank >= world)
    return set_error(NSLG_ERR_ARG, "tp_allreduce_rmsnorm: need 2 <= world <= 8 and 0 <= rank < world");
  if (rows < 0 || hidden <= 0) return set_error(NSLG_ERR_ARG, "tp_allreduce_rmsnorm: bad shape");
  const int esz = dtype_bytes(dtype);
  if ((static_cast<int64_t>(hidden) * esz) % 16)
    return set_error(NSLG_ERR_ARG, "tp_allreduce_rmsnorm: hidden * element size must be a multiple of 16 bytes");
  if (static_cast<int64_t>(hidden) * esz > 16ll * kThreads * kVecPerThread)
    return set_error(NSLG_ERR_UNSUPPORTED, "tp_allreduce_rmsnorm: rows longer than 16 KiB");
  if (!partial || !stage_bufs || !counters || !residual || (weight && !out))
    return set_error(NSLG_ERR_ARG, "tp_allreduce_rmsnorm: null pointer");
  // [2 slots][world][rows][2 * row bytes]
  const int64_t row_bytes = static_cast<int64_t>(hidden) * esz;
  int64_t region = 0, slot = 0;
  tp_stage_geometry(stage_bytes, world, &region, &slot);
  if (2 * row_bytes * rows > region)
    return set_error(NSLG_ERR_WORKSPACE, "tp_allreduce_rmsnorm: " + std::to_string(rows) +
                                             " rows need " + std::to_string(4 * row_bytes * rows * world) +
                                             " stage bytes per rank, have " + std::to_string(stage_bytes));
  if (timeout_ns <= 0) return set_error(NSLG_ERR_ARG, "tp_allreduce_rmsnorm: timeout_ns must be > 0");
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  if (!a16(partial) || !a16(residual) || !a16(counters) || (weight && (!a16(weight) || !a16(out))) ||
      (partial_stride * esz) % 16 || (residual_stride * esz) % 16 || (weight && (out_stride * esz) % 16))
    return set_error(NSLG_ERR_ARG, "tp_allreduce_rmsnorm: rows must be 16-byte aligned");
  ArParams p{};
  for (int i = 0; i < world; ++i) {
    if (!stage_bufs[i] || !a16(stage_bufs[i]))
      return set_error(NSLG_ERR_ARG, "tp_allreduce_rmsnorm: bad stage buffer");
    p.stage[i] = static_cast<uint8_t*>(stage_bufs[i]);
    if (emu == nullptr) continue;
    if (!emu->partials[i] || !emu->counters[i] || !emu->residuals[i] ||
        (weight && !emu->outs[i]) || !a16(emu->partials[i]) || !a16(emu->counters[i]) ||
        !a16(emu->residuals[i]) || (weight && !a16(emu->outs[i])))
      return set_error(NSLG_ERR_ARG, "tp_allreduce_rmsnorm_emulated: bad rank buffer");
    p.e_partial[i] = emu->partials[i];
    p.e_counters[i] = static_cast<uint32_t*>(emu->counters[i]);
    p.e_residual[i] = emu->residuals[i];
    p.e_out[i] = weight ? emu->outs[i] : nullptr;
  }
  p.partial = partial;
  p.p_stride = partial_stride;
  p.region_bytes = region;
  p.slot_bytes = slot;
  p.counters = static_cast<uint32_t*>(counters);
  p.residual = residual;
  p.r_stride = residual_stride;
  p.weight = weight;
  p.out = out;
  p.o_stride = out_stride;
  p.rows = rows;
  p.hidden = hidden;
  p.world = world;
  p.rank = rank;
  p.eps = eps;
  // Two-shot (reduce-scatter of column slices, then all-gather of the reduced slices)
  // when the one-shot's (world - 1) full-row pushes per rank are large: it moves
  // 2 (world - 1) / world of a row per rank instead of (world - 1) rows, at the price of a
  // second NVLink round trip. Same fp32 rank-order sums, so both give identical results.
  // By size unless NSLG_TP_TWO_SHOT forces a mode: the packed one-shot push is
  // 2 (world - 1) rows x row bytes out of each GPU, two-shot's 4 (world - 1) / world of
  // that; e.g. 8B decode rows (8 KiB): one-shot up to 5 rows at TP=4, 1 at TP=8.
  const int vec = 16 / esz;
  const bool two_ok = world > 2 && hidden % (world * vec) == 0;
  const int force = two_shot_override();
  const int64_t saved = 2 * static_cast<int64_t>(rows) * row_bytes * (world - 1) * (world - 2) /
                        world;
  p.two_shot = !pushed && two_ok && (force >= 0 ? force == 1 : saved >= kTwoShotSavingBytes);
  p.pushed = pushed;
  p.timeout_ns = static_cast<uint64_t>(timeout_ns);
  p.status = dev_status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (emu != nullptr) {
    if (dtype == NSLG_DTYPE_BF16) return launch_emulated<__nv_bfloat16>(p, world, st);
    if (dtype == NSLG_DTYPE_F16) return launch_emulated<__half>(p, world, st);
    return launch_emulated<float>(p, world, st);
  }
  if (dtype == NSLG_DTYPE_BF16)
    return launch_pdl("tp_allreduce_rmsnorm", tp_allreduce_rmsnorm_kernel<__nv_bfloat16>,
                      dim3(kGrid), dim3(kThreads), 0, st, p);
  if (dtype == NSLG_DTYPE_F16)
    return launch_pdl("tp_allreduce_rmsnorm", tp_allreduce_rmsnorm_kernel<__half>,
                      dim3(kGrid), dim3(kThreads), 0, st, p);
  return launch_pdl("tp_allreduce_rmsnorm", tp_allreduce_rmsnorm_kernel<float>, dim3(kGrid),
                    dim3(kThreads), 0, st, p);
}
}  // namespace

extern "C" int nslg_tp_allreduce_rmsnorm(int dtype, int rows, int hidden, int world, int rank,
                                         const void* partial, int64_t partial_stride,
                                         void* const* stage_bufs, int64_t stage_bytes,
                                         void* counters, void* residual, int64_t residual_stride,
                                         const void* weight, void* out, int64_t out_stride,
                                         float eps, int64_t timeout_ns, uint32_t* dev_status,
                                         void* stream) {
  return tp_reduce(dtype, rows, hidden, world, rank, partial, partial_stride, stage_bufs,
                   stage_bytes, counters, residual, residual_stride, weight, out, out_stride,
                   eps, timeout_ns, dev_status, stream, 0);
}

extern "C" int nslg_tp_allreduce_rmsnorm_emulated(
    int dtype, int rows, int hidden, int world, const void* const* partials,
    int64_t partial_stride, void* const* stage_bufs, int64_t stage_bytes, void* const* counters,
    void* const* residuals, int64_t residual_stride, const void* weight, void* const* outs,
    int64_t out_stride, float eps, int64_t timeout_ns, uint32_t* dev_status, void* stream) {
  clear_error();
  if (!partials || !counters || !residuals || (weight && !outs))
    return set_error(NSLG_ERR_ARG, "tp_allreduce_rmsnorm_emulated: null pointer array");
  if (world < 2 || world > NSLG_TP_MAX_WORLD)
    return set_error(NSLG_ERR_ARG, "tp_allreduce_rmsnorm_emulated: need 2 <= world <= 8");
  const EmulatedRanks emu{partials, counters, residuals, outs};
  return tp_reduce(dtype, rows, hidden, world, 0, partials[0], partial_stride, stage_bufs,
                   stage_bytes, counters[0], residuals[0], residual_stride, weight,
                   weight ? outs[0] : nullptr, out_stride, eps, timeout_ns, dev_status, stream,
                   0, &emu);
}

extern "C" int nslg_tp_reduce_pushed_rmsnorm(int dtype, int rows, int hidden, int world,
                                             int rank, const void* partial,
                                             int64_t partial_stride, void* const* stage_bufs,
                                             int64_t stage_bytes, void* counters,
                                             void* residual, int64_t residual_stride,
                                             const void* weight, void* out,
                                             int64_t out_stride, float eps,
                                             int64_t timeout_ns, uint32_t* dev_status,
                                             void* stream) {
  return tp_reduce(dtype, rows, hidden, world, rank, partial, partial_stride, stage_bufs,
                   stage_bytes, counters, residual, residual_stride, weight, out, out_stride,
                   eps, timeout_ns, dev_status, stream, 1);
}
