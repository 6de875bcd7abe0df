// Split-KV GQA decode attention for bf16 or fp16, page_size 16, head_dim 128 (or 64).
//
// Work split. The pages of all sequences form one flat list (the CSR kv_indices,
// kv_cache.py:598-615). CTA c of n takes the contiguous slice
// [floor(T*c/n), floor(T*(c+1)/n)) of it, T = kv_indptr[B], so every CTA streams the
// same number of pages whatever the sequence lengths are. n = min(#SMs, ceil(T/m)), m =
// the pages of at least 2 and 32 KiB of K/V, and n is computed on the device from
// kv_indptr, so the launch needs no host-side plan and
// can be replayed inside a CUDA graph. A CTA's slice is cut into segments at sequence
// boundaries; segment (b, c) writes its softmax partial (o, lse) to slot b + c of the
// workspace (unique: along the flat list either b or c grows by one at each new
// segment). A sequence lying inside one CTA's slice is finished in place and written
// straight to `out`.
//
// Combining split sequences, two modes chosen per call by the host (merge_inline).
// In-kernel, with no second launch: a sequence spread over CTAs cf..cl is combined by
// the last of those CTAs to finish its segment: each writes its partial, fences, and adds
// one to the arrival count of slot cf (at most one sequence that continues past its
// slice starts in any CTA's slice, so the counts are indexed by CTA, [#SMs] words at
// the head of the workspace whatever the batch); the CTA that brings the count to
// cl - cf + 1 merges the partials (log-sum-exp weights in fp32, partials summed in slot
// order, so the result does not depend on which CTA merges) and puts the count back to
// zero. The counts are zero between calls: a new workspace must start zeroed. No CTA
// waits for another. Merge kernel: decode_merge_kernel, launched behind the decode grid
// with programmatic dependent launch, combines them on (hq / 4) x batch CTAs. In both
// modes sequences without pages are written as zeros by decode CTA b % grid.
//
// Data movement. One producer warp issues TMA tile loads (no multicast) of each page:
// per kv head and per 64-dim half, a [16 tokens x 64 dims] box with 128-byte swizzle,
// into a ring of `stages` stage buffers guarded by full/empty mbarriers. A stage holds
// 8/HKV pages of all HKV heads, K and V: 64 KiB for head_dim 128.
//
// Math. Eight consumer warps; warp w owns kv head w % HKV and page w / HKV of every
// stage. Its G = Hq/Hkv query heads are the rows of a 16-row mma tile (rows >= G are
// zero), so one K/V page serves all heads of the GQA group:
//   S[16 x 16 tokens] = Q[16 x D] . K^T   (mma.m16n8k16, K via ldmatrix from the
//                                          swizzled tile, conflict free)
//   online softmax in fp32 (exp2, row max/sum over the 4-lane quad)
//   O[16 x D] += P[16 x 16] . V          (P reused from the S accumulators as the A
//                                          fragment, V via ldmatrix.trans)
// Warps that share a kv head (HKV < 8) merge their states through shared memory at
// the end of each segment.
#include <cuda.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <string>

#include "common.cuh"
#include "launch.h"

namespace nslg {
namespace {

constexpr int kPS = 16;             // tokens per page
constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kMinPagesPerCta = 2;
// ... and at least this many K/V bytes per CTA (a page holds 64 * hkv * head_dim bytes:
// 64 KiB at 8 kv heads, 8 KiB at 1): every extra CTA of a sequence is one more partial
// to merge, every missing one a slower stream. Measured at the TP=8 shard (1 kv head),
// batch 1, 512 tokens, 32 layers per graph: 16 / 32 / 64 / 128 KiB per CTA (16, 8, 4,
// 2 CTAs) gave 6.67 / 6.48 / 6.72 / 8.02 us per layer; the 8 kv head shapes keep 2
// pages (64 KiB each) per CTA.
constexpr int kMinCtaBytes = 32 << 10;
constexpr int kBoxBytes = kPS * 64 * 2;  // one [16 x 64] bf16 box: 2 KiB
constexpr int kMaxSmem = 232448;         // 227 KiB opt-in per CTA on sm_100
constexpr int kSmemCsrBatch = 1024;      // batches up to this size keep the CSR in smem

struct DecodeParams {
  const void* q;    // [B, hq, D] of the activation type T (bf16 or fp16)
  void* out;
  const int32_t* indptr;
  const int32_t* indices;
  const int32_t* lpl;
  float* part_o;    // [slots, hq, D]
  float* part_lse;  // [slots, hq]
  uint32_t* arrive; // [grid] arrival counts of the split sequences, by first CTA
  int64_t q_stride, out_stride, num_pages;
  int batch, hq, group, stages, grid;
  int smem_csr;       // kv_indptr and kv_last_page_len are staged in shared memory
  int inline_merge;   // 1: split sequences merged by their last CTA; 0: by the merge kernel
  int min_pages;      // fewest pages a CTA streams (kMinPagesPerCta, kMinCtaBytes)
  int vheads;         // > 1: split-heads call, page id = pool page * vheads + kv head
  int box_all_heads;  // tensor maps with a [64 dim x 16 tok x HKV head] box (token-major)
  float scale_log2;
  uint32_t* status;
};

__device__ __forceinline__ int num_ctas(int64_t total_pages, int grid, int min_pages) {
  const int64_t want = (total_pages + min_pages - 1) / min_pages;
  return static_cast<int>(want < grid ? want : grid);
}

// CTA whose slice holds flat page p: the largest c with floor(T*c/n) <= p.
__device__ __forceinline__ int cta_of(int64_t p, int64_t total, int n) {
  return static_cast<int>((static_cast<int64_t>(n) * (p + 1) - 1) / total);
}

// Sequence holding flat page p (kv_indptr non-decreasing, kv_indptr[B] > p).
__device__ __forceinline__ int seq_of(const int32_t* indptr, int batch, int64_t p) {
  int lo = 1, hi = batch;  // first j in [1, B] with indptr[j] > p
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (indptr[mid] > p) hi = mid; else lo = mid + 1;
  }
  return lo - 1;
}

constexpr int kMaxHq = 128;        // 8 kv heads x 16 query heads per group
constexpr int kMergeThreads = kConsumerWarps * 32;
constexpr int kStaticSmem = 2 * kMaxHq * 4 + 16;   // s_stat + s_merge, rounded up

// Sequences without pages (no CTA streams them) are zeros; CTA c writes sequences
// c, c + grid, ... Run after the PDL wait: the kernel before may still read `out`.
template <typename T, int D>
__device__ void zero_empty_sequences(const DecodeParams& p, const int32_t* indptr, int c,
                                     int tid, int nthreads) {
  const int words = p.hq * D / 2;
  for (int b = c; b < p.batch; b += p.grid) {
    if (indptr[b] != indptr[b + 1]) continue;
    uint32_t* ob = reinterpret_cast<uint32_t*>(static_cast<T*>(p.out) +
                                               static_cast<int64_t>(b) * p.out_stride);
    for (int e = tid; e < words; e += nthreads) ob[e] = 0u;
  }
}

// Combines the `cnt` partials of sequence b (slots b + cf .. b + cf + cnt - 1) into
// out[b]; run by the kConsumerWarps warps of the CTA that arrived last. The partials
// were written by other CTAs and published by their arrivals; they are read through L2
// (ld.global.cg), never from this SM's L1. Up to kFastMerge partials: one pass (below).
// More:
//   pass 1: per query head, m = max_i lse_i and 1 / sum_i 2^(lse_i - m); 8 lanes per
//           head split the partials (32 heads per pass of the CTA);
//   pass 2: per (head, 4 dims), sum_i 2^(lse_i - m) o_i, times 1 / sum; with many
//           outputs each thread takes 4 at once (8 independent loads per step of its
//           loop over the partials, two steps unrolled), with few (hq x D / 4 <= 128)
//           2 to 8 lanes share one output's partials and add up by shuffles. The order
//           of the sums depends only on the shapes, not on which CTA merges.
constexpr int kFastMerge = 4;   // partials merged in one pass of loads

template <typename T, int D>
__device__ void merge_sequence(const DecodeParams& p, int b, int cf, int cnt, float* stat,
                               int tid) {
  const int warp = tid / 32, lane = tid % 32;
  const int64_t slot0 = static_cast<int64_t>(b) + cf;
  const float* lse0 = p.part_lse + slot0 * p.hq;
  if (cnt <= kFastMerge) {
    // Few partials (a sequence over at most 4 CTAs): each thread takes (head, 4 dims)
    // outputs e, e + 256, ... and issues every load it needs -- the log-sum-exp and the
    // 4 partial values of each of its outputs' partials -- before any arithmetic, so the
    // merge costs one L2 round trip. Per output: m = max_i lse_i, w_i = 2^(lse_i - m),
    // out = (sum_i w_i o_i) / (sum_i w_i), sums in partial order.
    constexpr int DQ = D / 4;
    constexpr int kE = 4;
    const int n_out = p.hq * DQ;
    const int64_t step = static_cast<int64_t>(p.hq) * D;
    for (int e0 = tid; e0 < n_out; e0 += kE * kMergeThreads) {
      float l[kE][kFastMerge];
      float4 v[kE][kFastMerge];
#pragma unroll
      for (int k = 0; k < kE; ++k) {
        const int e = e0 + k * kMergeThreads;
        const int ec = e < n_out ? e : n_out - 1;     // clamped: loads stay in range
        const int hq = ec / DQ;
        const float* po = p.part_o + (slot0 * p.hq + hq) * D + (ec % DQ) * 4;
#pragma unroll
        for (int i = 0; i < kFastMerge; ++i) {
          if (i < cnt && e < n_out) {
            l[k][i] = __ldcg(lse0 + static_cast<int64_t>(i) * p.hq + hq);
            v[k][i] = __ldcg(reinterpret_cast<const float4*>(po + i * step));
          } else {
            l[k][i] = -INFINITY;
            v[k][i] = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
      }
#pragma unroll
      for (int k = 0; k < kE; ++k) {
        const int e = e0 + k * kMergeThreads;
        if (e >= n_out) continue;
        float m = l[k][0];
#pragma unroll
        for (int i = 1; i < kFastMerge; ++i) m = fmaxf(m, l[k][i]);
        float s = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int i = 0; i < kFastMerge; ++i) {
          const float w = l[k][i] == -INFINITY ? 0.f : fast_exp2(l[k][i] - m);
          s += w;
          acc.x = fmaf(w, v[k][i].x, acc.x);
          acc.y = fmaf(w, v[k][i].y, acc.y);
          acc.z = fmaf(w, v[k][i].z, acc.z);
          acc.w = fmaf(w, v[k][i].w, acc.w);
        }
        const float inv = s > 0.f ? 1.f / s : 0.f;
        T* ob = static_cast<T*>(p.out) + static_cast<int64_t>(b) * p.out_stride +
                static_cast<int64_t>(e / DQ) * D + (e % DQ) * 4;
        reinterpret_cast<uint32_t*>(ob)[0] = Mma16<T>::pack(acc.x * inv, acc.y * inv);
        reinterpret_cast<uint32_t*>(ob)[1] = Mma16<T>::pack(acc.z * inv, acc.w * inv);
      }
    }
    return;
  }
  for (int h0 = warp * 4; h0 < p.hq; h0 += kConsumerWarps * 4) {
    const int hq = h0 + lane / 8, sub = lane % 8;
    float m = -INFINITY, s = 0.f;
    if (hq < p.hq) {
#pragma unroll 4
      for (int i = sub; i < cnt; i += 8) {
        const float l = __ldcg(lse0 + static_cast<int64_t>(i) * p.hq + hq);
        const float nm = fmaxf(m, l);
        if (nm != -INFINITY) s = s * fast_exp2(m - nm) + fast_exp2(l - nm);
        m = nm;
      }
    }
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, m, o);
      const float os = __shfl_xor_sync(0xffffffffu, s, o);
      const float nm = fmaxf(m, om);
      s = nm == -INFINITY ? 0.f : s * fast_exp2(m - nm) + os * fast_exp2(om - nm);
      m = nm;
    }
    if (sub == 0 && hq < p.hq) {
      stat[2 * hq] = m;
      stat[2 * hq + 1] = s > 0.f ? 1.f / s : 0.f;
    }
  }
  named_barrier_sync(1, kMergeThreads);
  constexpr int DQ = D / 4;
  constexpr int kE = 4;                                   // outputs per thread per round
  const int n_out = p.hq * DQ;
  const int64_t step = static_cast<int64_t>(p.hq) * D;   // from one partial to the next
  int tpo = 1;   // threads per output: 2..8 neighbouring lanes when the outputs are few
  while (tpo < 8 && n_out * tpo * 2 <= kMergeThreads) tpo *= 2;
  if (tpo > 1) {
    // lanes e*tpo .. e*tpo + tpo - 1 (one aligned group inside a warp) split the
    // partials of output e (i = sub, sub + tpo, ...) and add their sums by shuffles
    const int e = tid / tpo, sub = tid % tpo;
    const bool live = e < n_out;
    const int ec = live ? e : n_out - 1;   // idle lanes load a valid address, store nothing
    const int hq = ec / DQ;
    const float m = stat[2 * hq];
    const float* po = p.part_o + (slot0 * p.hq + hq) * D + (ec % DQ) * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int i = sub; i < cnt; i += tpo) {
      const float l = __ldcg(lse0 + static_cast<int64_t>(i) * p.hq + hq);
      const float4 v = __ldcg(reinterpret_cast<const float4*>(po + i * step));
      const float w = l == -INFINITY ? 0.f : fast_exp2(l - m);
      acc.x = fmaf(w, v.x, acc.x);
      acc.y = fmaf(w, v.y, acc.y);
      acc.z = fmaf(w, v.z, acc.z);
      acc.w = fmaf(w, v.w, acc.w);
    }
    for (int o = tpo / 2; o > 0; o >>= 1) {
      acc.x += __shfl_xor_sync(0xffffffffu, acc.x, o);
      acc.y += __shfl_xor_sync(0xffffffffu, acc.y, o);
      acc.z += __shfl_xor_sync(0xffffffffu, acc.z, o);
      acc.w += __shfl_xor_sync(0xffffffffu, acc.w, o);
    }
    if (live && sub == 0) {
      const float inv = stat[2 * hq + 1];
      T* ob = static_cast<T*>(p.out) + static_cast<int64_t>(b) * p.out_stride +
              static_cast<int64_t>(hq) * D + (ec % DQ) * 4;
      reinterpret_cast<uint32_t*>(ob)[0] = Mma16<T>::pack(acc.x * inv, acc.y * inv);
      reinterpret_cast<uint32_t*>(ob)[1] = Mma16<T>::pack(acc.z * inv, acc.w * inv);
    }
    return;
  }
  for (int e0 = tid; e0 < n_out; e0 += kE * kMergeThreads) {
    int hq[kE];
    float m[kE];
    const float* po[kE];
    float4 acc[kE];
#pragma unroll
    for (int k = 0; k < kE; ++k) {
      const int e = min(e0 + k * kMergeThreads, n_out - 1);   // clamped: loads stay in range
      hq[k] = e / DQ;
      m[k] = stat[2 * hq[k]];
      po[k] = p.part_o + (slot0 * p.hq + hq[k]) * D + (e % DQ) * 4;
      acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll 2
    for (int i = 0; i < cnt; ++i) {
      float l[kE];
      float4 v[kE];
#pragma unroll
      for (int k = 0; k < kE; ++k) {
        if (e0 + k * kMergeThreads < n_out) {
          l[k] = __ldcg(lse0 + static_cast<int64_t>(i) * p.hq + hq[k]);
          v[k] = __ldcg(reinterpret_cast<const float4*>(po[k] + i * step));
        } else {
          l[k] = -INFINITY;
          v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int k = 0; k < kE; ++k) {
        const float w = l[k] == -INFINITY ? 0.f : fast_exp2(l[k] - m[k]);
        acc[k].x = fmaf(w, v[k].x, acc[k].x);
        acc[k].y = fmaf(w, v[k].y, acc[k].y);
        acc[k].z = fmaf(w, v[k].z, acc[k].z);
        acc[k].w = fmaf(w, v[k].w, acc[k].w);
      }
    }
#pragma unroll
    for (int k = 0; k < kE; ++k) {
      const int e = e0 + k * kMergeThreads;
      if (e >= n_out) continue;
      const float inv = stat[2 * hq[k] + 1];
      T* ob = static_cast<T*>(p.out) + static_cast<int64_t>(b) * p.out_stride +
              static_cast<int64_t>(hq[k]) * D + (e % DQ) * 4;
      // 4-byte stores: `out` and its row stride are only required to be 4-byte aligned
      reinterpret_cast<uint32_t*>(ob)[0] = Mma16<T>::pack(acc[k].x * inv, acc[k].y * inv);
      reinterpret_cast<uint32_t*>(ob)[1] = Mma16<T>::pack(acc[k].z * inv, acc[k].w * inv);
    }
  }
}

template <int HKV, int D>
struct Cfg {
  static constexpr int kPPS = kConsumerWarps / HKV;  // pages per stage
  static constexpr int kHalves = D / 64;
  static constexpr int kStageBytes = kPPS * 2 * kHalves * HKV * kBoxBytes;
  // byte offset of the box (page j, K=0/V=1, half, head) inside a stage
  __device__ static constexpr int box(int j, int kv, int half, int h) {
    return (((j * 2 + kv) * kHalves + half) * HKV + h) * kBoxBytes;
  }
};

template <typename T, int HKV, int D>
__global__ void __launch_bounds__(kThreads, 1)
    decode_tc_kernel(const __grid_constant__ CUtensorMap tmap_k,
                     const __grid_constant__ CUtensorMap tmap_v, const DecodeParams p) {
  using C = Cfg<HKV, D>;
  constexpr int NT = D / 8;   // 8-wide n tiles of the output
  constexpr int KS = D / 16;  // 16-deep k steps of Q.K^T
  extern __shared__ uint8_t smem_raw[];
  __shared__ float s_stat[2 * kMaxHq];   // merge: per query head, max lse and 1 / sum
  __shared__ int s_merge;                // this CTA merges the segment's sequence
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int stages = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + stages * C::kStageBytes);
  uint64_t* empty = full + stages;
  float* comb = reinterpret_cast<float*>(empty + stages);  // [8 warps][G][D] o, then m, l

  // Programmatic dependent launch: this grid may start while the kernel before it (the
  // KV append, which also writes the rotated q) is still running. Everything up to the
  // first page load and the first q read -- staging the CSR, barrier set-up, the first
  // page ids -- uses only data of kernels that finished before that one started (the
  // plan), so it runs before the wait; the producer waits before its first TMA load and
  // the consumers before they read q.
  // The CSR lookups (slice bounds, sequence of a page, segment ends, last-page lengths)
  // are chains of dependent loads; with the arrays in shared memory (one coalesced load
  // by the whole CTA) they no longer delay the first TMA issue or each new segment.
  const int32_t* indptr = p.indptr;
  const int32_t* lpl = p.lpl;
  if (p.smem_csr) {
    int32_t* s_ip = reinterpret_cast<int32_t*>(
        reinterpret_cast<uint8_t*>(comb) +
        (C::kPPS > 1 ? static_cast<size_t>(kConsumerWarps) * p.group * (D + 2) * 4 : 0));
    int32_t* s_lpl = s_ip + p.batch + 1;
    for (int i = threadIdx.x; i <= p.batch; i += blockDim.x) s_ip[i] = p.indptr[i];
    for (int i = threadIdx.x; i < p.batch; i += blockDim.x) s_lpl[i] = p.lpl[i];
    __syncthreads();
    indptr = s_ip;
    lpl = s_lpl;
  }

  const int64_t total = indptr[p.batch];
  const int n = num_ctas(total, p.grid, p.min_pages);
  const int c = blockIdx.x;
  if (c >= n) {
    pdl_wait();
    zero_empty_sequences<T, D>(p, indptr, c, threadIdx.x, blockDim.x);
    return;
  }
  const int64_t p0 = total * c / n;
  const int64_t p1 = total * (c + 1) / n;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // let the next kernel (if launched with programmatic stream serialisation) be
  // scheduled as SMs free up; it waits for this grid's completion before reading `out`
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    // The whole warp issues the TMA boxes of a stage (lane L takes boxes L, L + 32, ...),
    // so stages of many small boxes (few kv heads) go out in a few instructions; lane jj
    // holds the page id of the stage's page jj.
    prefetch_tmap(&tmap_k);
    prefetch_tmap(&tmap_v);
    const uint64_t policy = l2_policy_evict_first();
    constexpr int kHB = 1;  // boxes per (page, K/V, half) with the all-heads map
    int stage = 0;
    uint32_t phase = 0;
    uint32_t armed[4] = {0u, 0u, 0u, 0u};  // arms of each stage's full barrier (lane 0)
    // Stages in order: (first flat page, page count) over the segments of this CTA's
    // slice. The page ids of the next stage are loaded one stage ahead so their latency
    // overlaps the wait for a free stage.
    int b = seq_of(indptr, p.batch, p0);
    int64_t seg_end = min(p1, static_cast<int64_t>(indptr[b + 1]));
    int64_t cursor = p0;
    auto next_stage = [&](int64_t& q0, int& np) -> bool {
      if (cursor >= p1) return false;
      if (cursor >= seg_end) {
        ++b;
        while (b < p.batch && indptr[b + 1] <= cursor) ++b;
        seg_end = min(p1, static_cast<int64_t>(indptr[b + 1]));
      }
      q0 = cursor;
      np = static_cast<int>(min(static_cast<int64_t>(C::kPPS), seg_end - cursor));
      cursor += np;
      return true;
    };
    int64_t q0 = 0;
    int np = 0;
    bool have = next_stage(q0, np);
    int my_id = (have && lane < np) ? p.indices[q0 + lane] : 0;
    pdl_wait();   // the pages hold the keys and values the previous kernel appended
    while (have) {
      int64_t nq0 = 0;
      int nnp = 0;
      const bool nhave = next_stage(nq0, nnp);
      const int my_nid = (nhave && lane < nnp) ? p.indices[nq0 + lane] : 0;
      if (!__all_sync(0xffffffffu, mbar_wait(&empty[stage], phase ^ 1))) {
        if (lane == 0) {
          report(p.status, NSLG_DEV_WAIT_TIMEOUT);
          // The consumers stopped releasing stages. Issue nothing more, wait (bounded)
          // for the loads already in flight, and leave.
          for (int s = 0; s < stages; ++s)
            if (armed[s] > 0) (void)mbar_wait(&full[s], (armed[s] - 1) & 1);
        }
        return;
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[stage], np * 2 * C::kHalves * HKV * kBoxBytes);
        ++armed[stage];
      }
      __syncwarp();
      if (lane < np && (my_id < 0 || my_id >= p.num_pages * (p.vheads > 1 ? p.vheads : 1))) {
        report(p.status, NSLG_DEV_BAD_PAGE);
        my_id = 0;  // keep the transaction count; page 0 is the pool's null page
      }
      uint8_t* sb = smem + stage * C::kStageBytes;
      const int per_page = 2 * C::kHalves * (p.box_all_heads ? kHB : HKV);
      const int nbox = np * per_page;
      // every lane runs the same rounds (the shuffle needs the whole warp)
      for (int k0 = 0; k0 < C::kPPS * per_page; k0 += 32) {
        const int k = k0 + lane;
        const int jj = min(k / per_page, C::kPPS - 1);
        const int pid = __shfl_sync(0xffffffffu, my_id, jj);
        if (k >= nbox) continue;
        int r = k - jj * per_page;
        const int kv = r & 1;
        r >>= 1;
        const CUtensorMap* map = kv ? &tmap_v : &tmap_k;
        if (p.box_all_heads) {
          // one box covers every kv head of the page half (token-major map)
          const int half = r;
          tma_load_3d(sb + C::box(jj, kv, half, 0), map, &full[stage], half * 64, pid * kPS, 0,
                      policy);
        } else {
          const int half = r % C::kHalves, h = r / C::kHalves;
          // split-heads calls: the page id carries the kv head (the map's head coordinate)
          const int vh = p.vheads > 1 ? pid % p.vheads : 0;
          const int pg = p.vheads > 1 ? pid / p.vheads : pid;
          tma_load_3d(sb + C::box(jj, kv, half, h), map, &full[stage], half * 64, h + vh,
                      pg * kPS, policy);
        }
      }
      if (++stage == stages) { stage = 0; phase ^= 1; }
      have = nhave;
      q0 = nq0;
      np = nnp;
      my_id = my_nid;
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  pdl_wait();   // q comes from the previous kernel
  zero_empty_sequences<T, D>(p, indptr, c, threadIdx.x, kMergeThreads);
  const int h = warp % HKV;
  const int j = warp / HKV;
  const int g = lane >> 2;        // mma row group: query head g (and g + 8)
  const int tq = lane & 3;        // thread in quad
  const int G = p.group;
  const float sl = p.scale_log2;
  int stage = 0;
  uint32_t phase = 0;
  bool ok = true;
  int b = seq_of(indptr, p.batch, p0);
  for (int64_t pp = p0; pp < p1;) {
    const int64_t seq_beg = indptr[b];
    const int64_t seq_end = indptr[b + 1];
    const int64_t seg_beg = pp;
    const int64_t seg_end = min(p1, seq_end);
    const int last_len = lpl[b];

    // Q fragments (A operand, 16 rows = query heads h*G + r, r < G).
    uint32_t qa[KS][4];
    {
      const T* qb = static_cast<const T*>(p.q) + static_cast<int64_t>(b) * p.q_stride +
                                static_cast<int64_t>(h) * G * D;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        const int col = ks * 16 + tq * 2;
        qa[ks][0] = g < G ? *reinterpret_cast<const uint32_t*>(qb + g * D + col) : 0u;
        qa[ks][1] = g + 8 < G ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * D + col) : 0u;
        qa[ks][2] = g < G ? *reinterpret_cast<const uint32_t*>(qb + g * D + col + 8) : 0u;
        qa[ks][3] =
            g + 8 < G ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * D + col + 8) : 0u;
      }
    }
    float o[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    for (int64_t q0 = seg_beg; q0 < seg_end; q0 += C::kPPS) {
      const int np = static_cast<int>(min(static_cast<int64_t>(C::kPPS), seg_end - q0));
      if (ok) {
        // warp-uniform: a warp that gives up stops consuming and stops releasing
        // stages, but keeps the control flow (and the named barriers) of the others
        ok = __all_sync(0xffffffffu, mbar_wait(&full[stage], phase));
        if (!ok && lane == 0) report(p.status, NSLG_DEV_WAIT_TIMEOUT);
      }
      if (ok && j < np) {
        const int nvalid = (q0 + j == seq_end - 1) ? last_len : kPS;
        const uint32_t sb = smem_u32(smem + stage * C::kStageBytes);
        // ---- S = Q . K^T over the page's 16 tokens
        float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        {
          const int mi = lane >> 3, r = lane & 7;
          const int tok = (mi >> 1) * 8 + r;
#pragma unroll
          for (int ks = 0; ks < KS; ++ks) {
            const int half = ks >> 2;
            const int chunk = ((ks & 3) << 1) + (mi & 1);
            const uint32_t addr = sb + C::box(j, 0, half, h) + tok * 128 + ((chunk ^ (tok & 7)) << 4);
            uint32_t b00, b01, b10, b11;
            ldmatrix_x4(addr, b00, b01, b10, b11);
            Mma16<T>::mma(s[0], qa[ks], b00, b01);
            Mma16<T>::mma(s[1], qa[ks], b10, b11);
          }
        }
        // ---- mask the tail of the last page, online softmax
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (nt * 8 + tq * 2 + (e & 1) >= nvalid) s[nt][e] = -INFINITY;
        float mx0 = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
        float mx1 = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float base0 = mn0 == -INFINITY ? 0.f : mn0 * sl;
        const float base1 = mn1 == -INFINITY ? 0.f : mn1 * sl;
        const float a0 = fast_exp2(fmaf(m0, sl, -base0));
        const float a1 = fast_exp2(fmaf(m1, sl, -base1));
        m0 = mn0;
        m1 = mn1;
        float ps[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          ps[nt][0] = fast_exp2(fmaf(s[nt][0], sl, -base0));
          ps[nt][1] = fast_exp2(fmaf(s[nt][1], sl, -base0));
          ps[nt][2] = fast_exp2(fmaf(s[nt][2], sl, -base1));
          ps[nt][3] = fast_exp2(fmaf(s[nt][3], sl, -base1));
        }
        l0 = fmaf(l0, a0, ps[0][0] + ps[0][1] + ps[1][0] + ps[1][1]);
        l1 = fmaf(l1, a1, ps[0][2] + ps[0][3] + ps[1][2] + ps[1][3]);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          o[t][0] *= a0; o[t][1] *= a0;
          o[t][2] *= a1; o[t][3] *= a1;
        }
        uint32_t pa[4];
        pa[0] = Mma16<T>::pack(ps[0][0], ps[0][1]);
        pa[1] = Mma16<T>::pack(ps[0][2], ps[0][3]);
        pa[2] = Mma16<T>::pack(ps[1][0], ps[1][1]);
        pa[3] = Mma16<T>::pack(ps[1][2], ps[1][3]);
        // ---- O += P . V
        {
          const int mi = lane >> 3, r = lane & 7;
          const int tok = (mi & 1) * 8 + r;
#pragma unroll
          for (int qd = 0; qd < D / 16; ++qd) {
            const int cg = qd * 2 + (mi >> 1);  // 8-dim chunk of the head row
            const int half = cg >> 3, ch = cg & 7;
            const uint32_t addr = sb + C::box(j, 1, half, h) + tok * 128 + ((ch ^ (tok & 7)) << 4);
            uint32_t v0, v1, v2, v3;
            ldmatrix_x4_trans(addr, v0, v1, v2, v3);
            Mma16<T>::mma(o[2 * qd], pa, v0, v1);
            Mma16<T>::mma(o[2 * qd + 1], pa, v2, v3);
          }
        }
      }
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == stages) { stage = 0; phase ^= 1; }
    }
    pp = seg_end;

    // ---- finish the segment: row sums over the quad
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const bool whole = cta_of(seq_beg, total, n) == cta_of(seq_end - 1, total, n);
    const int64_t slot = static_cast<int64_t>(b) + c;

    if constexpr (C::kPPS == 1) {
      // one warp per kv head: its state is the segment's
      if (ok) {
        const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
        const float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const int r = g + rr * 8;
          if (r >= G) continue;
          const int hq = h * G + r;
          const float inv = rr ? inv1 : inv0;
          if (whole) {
            T* ob = static_cast<T*>(p.out) + static_cast<int64_t>(b) * p.out_stride +
                    static_cast<int64_t>(hq) * D;
#pragma unroll
            for (int t = 0; t < NT; ++t)
              *reinterpret_cast<uint32_t*>(ob + t * 8 + tq * 2) =
                  Mma16<T>::pack(o[t][rr * 2] * inv, o[t][rr * 2 + 1] * inv);
          } else {
            float* po = p.part_o + (slot * p.hq + hq) * D;
#pragma unroll
            for (int t = 0; t < NT; ++t)
              *reinterpret_cast<float2*>(po + t * 8 + tq * 2) =
                  make_float2(o[t][rr * 2] * inv, o[t][rr * 2 + 1] * inv);
            if (tq == 0) {
              const float m = rr ? m1 : m0, l = rr ? l1 : l0;
              p.part_lse[slot * p.hq + hq] = l > 0.f ? m * sl + __log2f(l) : -INFINITY;
            }
          }
        }
      }
    } else {
      // The kPPS warps of kv head h (pages j = 0..kPPS-1 of each stage) each hold a
      // partial softmax state. All of them store it in shared memory; then warp j merges
      // the kPPS states for D / kPPS of the head dims (every row of the group) and writes
      // them, so the combine costs one pass instead of kPPS - 1 serial ones.
      float* cw = comb + static_cast<size_t>(warp) * G * (D + 2);
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const int col = t * 8 + tq * 2;
        if (g < G) { cw[g * D + col] = o[t][0]; cw[g * D + col + 1] = o[t][1]; }
        if (g + 8 < G) { cw[(g + 8) * D + col] = o[t][2]; cw[(g + 8) * D + col + 1] = o[t][3]; }
      }
      if (tq == 0) {
        if (g < G) { cw[G * D + g] = m0; cw[G * D + G + g] = l0; }
        if (g + 8 < G) { cw[G * D + g + 8] = m1; cw[G * D + G + g + 8] = l1; }
      }
      named_barrier_sync(1, kConsumerWarps * 32);
      if (ok) {
        constexpr int DS = D / C::kPPS;          // head dims merged and written by this warp
        for (int e = lane; e < G * DS; e += 32) {
          const int r = e / DS, col = j * DS + e % DS;
          float mx = -INFINITY;
#pragma unroll
          for (int jj = 0; jj < C::kPPS; ++jj)
            mx = fmaxf(mx, comb[static_cast<size_t>(jj * HKV + h) * G * (D + 2) + G * D + r]);
          const float base = mx == -INFINITY ? 0.f : mx * sl;
          float lsum = 0.f, acc = 0.f;
#pragma unroll
          for (int jj = 0; jj < C::kPPS; ++jj) {
            const float* cx = comb + static_cast<size_t>(jj * HKV + h) * G * (D + 2);
            const float w = fast_exp2(fmaf(cx[G * D + r], sl, -base));
            lsum = fmaf(cx[G * D + G + r], w, lsum);
            acc = fmaf(cx[r * D + col], w, acc);
          }
          const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
          const int hq = h * G + r;
          if (whole) {
            static_cast<T*>(p.out)[static_cast<int64_t>(b) * p.out_stride +
                                   static_cast<int64_t>(hq) * D + col] = Elem<T>::from_f(acc * inv);
          } else {
            p.part_o[(slot * p.hq + hq) * D + col] = acc * inv;
            if (j == 0 && e % DS == 0)
              p.part_lse[slot * p.hq + hq] = lsum > 0.f ? mx * sl + __log2f(lsum) : -INFINITY;
          }
        }
      }
    }
    if constexpr (C::kPPS > 1) named_barrier_sync(1, kConsumerWarps * 32);
    if (!whole && p.inline_merge) {
      // Publish this segment's partial and count it in; the last CTA of the sequence
      // merges. Every CTA of the sequence arrives exactly once, also after a timed-out
      // wait (its partial is then garbage, and the status word says so), so the counts
      // always return to zero.
      // One barrier, then one acquire-release increment by thread 0: its release
      // publishes the partial all warps stored before the barrier, its acquire makes the
      // partials of the CTAs that arrived earlier visible to the merge (one round trip
      // instead of a fence per thread followed by the increment).
      named_barrier_sync(1, kMergeThreads);
      const int cf = cta_of(seq_beg, total, n);
      const int cnt = cta_of(seq_end - 1, total, n) - cf + 1;
      if (threadIdx.x == 0) {
        const uint32_t prev = atom_add_acq_rel_u32(&p.arrive[cf], 1u);
        const bool last = prev + 1u == static_cast<uint32_t>(cnt);
        if (last) atomicExch(&p.arrive[cf], 0u);
        s_merge = last ? 1 : 0;
      }
      named_barrier_sync(1, kMergeThreads);
      if (s_merge) merge_sequence<T, D>(p, b, cf, cnt, s_stat, threadIdx.x);
    }
    ++b;
    while (b < p.batch && indptr[b + 1] <= pp) ++b;
  }
}

// The merge-kernel mode (DecodeParams::inline_merge == 0): the partials of sequences
// that span several CTAs are combined by this second kernel, launched with programmatic
// dependent launch right behind the decode grid; one warp per (sequence, query head).
// Sequences finished in place by the decode kernel, and sequences without pages (written
// as zeros there), need no merge. The lanes read the partials' log-sum-exps in parallel
// (lane i: partial i, i + 32, ...) and the weighted partial outputs are loaded four
// partials at a time, so the merge costs a few load latencies however many CTAs the
// sequence spans, spread over (hq / 4) x batch CTAs.
template <typename T, int D>
__global__ void __launch_bounds__(128) decode_merge_kernel(const DecodeParams p) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int hq = blockIdx.x * 4 + warp;
  const int b = blockIdx.y;
  constexpr int DV = D / 32;
  static_assert(DV == 4 || DV == 2, "head_dim 128 or 64");
  // the CSR is an input of both kernels: read it before waiting for the decode grid
  const int64_t total = p.indptr[p.batch];
  const int64_t beg = p.indptr[b], end = p.indptr[b + 1];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (hq >= p.hq) return;
  T* ob = static_cast<T*>(p.out) + static_cast<int64_t>(b) * p.out_stride + static_cast<int64_t>(hq) * D;
  if (beg == end) return;
  const int n = num_ctas(total, p.grid, p.min_pages);
  const int cf = cta_of(beg, total, n), cl = cta_of(end - 1, total, n);
  if (cf == cl) return;
  const int cnt = cl - cf + 1;
  auto lse_of = [&](int i) {   // partial i of this sequence (CTA cf + i)
    return p.part_lse[(static_cast<int64_t>(b) + cf + i) * p.hq + hq];
  };
  const int64_t step = static_cast<int64_t>(p.hq) * D;   // from one partial to the next
  if (cnt <= 8) {
    // every load in flight at once: lane i's log-sum-exp and all partial outputs
    const float* po0 = p.part_o + ((static_cast<int64_t>(b) + cf) * p.hq + hq) * D + lane * DV;
    const float l = lane < cnt ? lse_of(lane) : -INFINITY;
    float v[8][DV];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k < cnt) {
#pragma unroll
        for (int e = 0; e < DV; ++e) v[k][e] = po0[k * step + e];
      }
    }
    float mx = l;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float w = l == -INFINITY ? 0.f : fast_exp2(l - mx);
    float wsum = w;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
    float acc[DV];
#pragma unroll
    for (int e = 0; e < DV; ++e) acc[e] = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float wk = __shfl_sync(0xffffffffu, w, k);
      if (k < cnt) {
#pragma unroll
        for (int e = 0; e < DV; ++e) acc[e] = fmaf(wk, v[k][e], acc[e]);
      }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
    for (int e = 0; e < DV; ++e) ob[lane * DV + e] = Elem<T>::from_f(acc[e] * inv);
    return;
  }
  float mx = -INFINITY;
  for (int i = lane; i < cnt; i += 32) mx = fmaxf(mx, lse_of(i));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float acc[DV];
#pragma unroll
  for (int e = 0; e < DV; ++e) acc[e] = 0.f;
  float wsum = 0.f;
  for (int base = 0; base < cnt; base += 32) {
    const int i = base + lane;
    const float l = i < cnt ? lse_of(i) : -INFINITY;
    const float w = l == -INFINITY ? 0.f : fast_exp2(l - mx);
    wsum += w;
    const int m = min(32, cnt - base);
    const float* po0 = p.part_o + ((static_cast<int64_t>(b) + cf + base) * p.hq + hq) * D + lane * DV;
#pragma unroll 4
    for (int k = 0; k < m; ++k) {
      const float wk = __shfl_sync(0xffffffffu, w, k);
      const float* po = po0 + k * step;
      if constexpr (DV == 4) {
        const float4 v = *reinterpret_cast<const float4*>(po);
        acc[0] = fmaf(wk, v.x, acc[0]);
        acc[1] = fmaf(wk, v.y, acc[1]);
        acc[2] = fmaf(wk, v.z, acc[2]);
        acc[3] = fmaf(wk, v.w, acc[3]);
      } else {
        const float2 v = *reinterpret_cast<const float2*>(po);
        acc[0] = fmaf(wk, v.x, acc[0]);
        acc[1] = fmaf(wk, v.y, acc[1]);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
  for (int e = 0; e < DV; ++e) ob[lane * DV + e] = Elem<T>::from_f(acc[e] * inv);
}

// ------------------------------------------------------------------ host side
template <typename T, int HKV, int D>
int launch_typed(const CUtensorMap& tk, const CUtensorMap& tv, DecodeParams p,
                 cudaStream_t stream) {
  using C = Cfg<HKV, D>;
  const size_t comb = C::kPPS > 1 ? static_cast<size_t>(kConsumerWarps) * p.group * (D + 2) * 4 : 0;
  p.smem_csr = p.batch <= kSmemCsrBatch ? 1 : 0;
  const size_t csr = p.smem_csr ? static_cast<size_t>(2 * p.batch + 1) * 4 : 0;
  // the static __shared__ merge state counts against the same per-CTA limit
  const size_t fixed = 1024 + comb + csr + 2 * 8 * 8 + kStaticSmem;
  int stages = static_cast<int>((kMaxSmem - fixed) / C::kStageBytes);
  if (stages > 4) stages = 4;
  if (stages < 2) return set_error(NSLG_ERR_UNSUPPORTED, "decode: group too large for smem");
  p.stages = stages;
  const size_t smem =
      1024 + static_cast<size_t>(stages) * C::kStageBytes + 2 * stages * 8 + comb + csr;
  auto kern = decode_tc_kernel<T, HKV, D>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return set_error(NSLG_ERR_CUDA, cudaGetErrorString(err));
  const int rc = launch_pdl("decode_tc", kern, dim3(p.grid), dim3(kThreads), smem, stream, tk,
                            tv, p);
  if (rc != NSLG_OK || p.inline_merge) return rc;
  // merge-kernel mode: launched with programmatic dependent launch while the decode grid
  // drains; it starts its work once the decode grid has completed
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.hq + 3) / 4, p.batch);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  err = cudaLaunchKernelEx(&cfg, decode_merge_kernel<T, D>, p);
  if (err != cudaSuccess)
    return set_error(NSLG_ERR_CUDA, std::string("decode_merge: ") + cudaGetErrorString(err));
  return check_launch("decode_merge");
}

template <typename T>
int launch_for_type(int hkv, int d, const CUtensorMap& tk, const CUtensorMap& tv,
                    DecodeParams p, cudaStream_t stream) {
  if (d == 128) {
    switch (hkv) {
      case 1: return launch_typed<T, 1, 128>(tk, tv, p, stream);
      case 2: return launch_typed<T, 2, 128>(tk, tv, p, stream);
      case 4: return launch_typed<T, 4, 128>(tk, tv, p, stream);
      case 8: return launch_typed<T, 8, 128>(tk, tv, p, stream);
    }
  } else if (d == 64) {
    switch (hkv) {
      case 1: return launch_typed<T, 1, 64>(tk, tv, p, stream);
      case 2: return launch_typed<T, 2, 64>(tk, tv, p, stream);
      case 4: return launch_typed<T, 4, 64>(tk, tv, p, stream);
      case 8: return launch_typed<T, 8, 64>(tk, tv, p, stream);
    }
  }
  return set_error(NSLG_ERR_UNSUPPORTED, "decode: unsupported head count / head_dim");
}

}  // namespace

bool decode_tc_supported(int dtype, int hq, int hkv, int d, int page_size) {
  return (dtype == NSLG_DTYPE_BF16 || dtype == NSLG_DTYPE_F16) && page_size == kPS &&
         (d == 128 || d == 64) &&
         (hkv == 1 || hkv == 2 || hkv == 4 || hkv == 8) && hq % hkv == 0 && hq / hkv <= 16;
}

namespace {
// The arrival counts: one 32-bit word per CTA at the head of the workspace, padded to
// 256 bytes so that the partials behind them keep their alignment.
int64_t arrive_bytes(int grid) { return (static_cast<int64_t>(grid) * 4 + 255) / 256 * 256; }

// Which CTA combines a split sequence. In-kernel (the last CTA of the sequence to finish)
// saves the second launch and its wait for the whole decode grid (about 1 us per call on
// B200), but one SM then reads all the sequence's partials; the merge kernel spreads the
// same reads over ceil(hq / 4) CTAs per sequence. The host cannot see the lengths (they
// are on the device), so it estimates the partials per split sequence from the batch
// alone, as for sequences of equal length: about #SMs / batch + 1 CTAs, each hq x
// head_dim fp32 values. In-kernel when that is at most 64 KiB, or when the merge kernel
// would get no more than 2 CTAs per sequence anyway (hq <= 8). Measured at the 8B decode
// shapes (32 layers per graph): hq 32, batch 64: 30.7 us per layer in-kernel against
// 31.9; hq 32, batch 1: 11.0 against 8.6; hq 4, batch 64: 14.0 against 14.8; hq 4,
// batch 1: 7.2 against 8.1. NSLG_DECODE_MERGE=inline or =kernel forces a mode.
constexpr int64_t kInlineMergeBytes = 64 << 10;
int merge_inline(int batch, int hq, int d, int grid) {
  const char* e = std::getenv("NSLG_DECODE_MERGE");
  if (e != nullptr && std::strcmp(e, "inline") == 0) return 1;
  if (e != nullptr && std::strcmp(e, "kernel") == 0) return 0;
  if (hq <= 8) return 1;
  const int64_t per_merge =
      static_cast<int64_t>((grid + batch - 1) / batch + 1) * hq * static_cast<int64_t>(d) * 4;
  return per_merge <= kInlineMergeBytes ? 1 : 0;
}
}  // namespace

int64_t decode_tc_workspace_bytes(int batch, int hq, int d) {
  const int grid = sm_count();
  const int64_t slots = static_cast<int64_t>(batch) + grid;
  return arrive_bytes(grid) + slots * hq * (static_cast<int64_t>(d) + 1) * 4 + 256;
}

int launch_paged_decode_tc(int dtype, int batch, int hq, int hkv, int d, const void* q,
                           int64_t q_stride, void* out, int64_t out_stride, const void* pool_k,
                           const void* pool_v, int64_t num_pages, const int32_t* kv_indptr,
                           const int32_t* kv_indices, const int32_t* kv_last_page_len,
                           float sm_scale, void* workspace, int64_t workspace_bytes,
                           uint32_t* status, cudaStream_t stream, int vheads) {
  if (batch == 0) return NSLG_OK;
  const int64_t need = decode_tc_workspace_bytes(batch, hq, d);
  if (workspace == nullptr || workspace_bytes < need)
    return set_error(NSLG_ERR_WORKSPACE, "decode workspace needs " + std::to_string(need) + " bytes");
  if (num_pages * kPS > (int64_t{1} << 31))
    return set_error(NSLG_ERR_UNSUPPORTED, "decode: pool larger than 2^31 token rows");
  CUtensorMap tk, tv;
  // -1 unknown, 1 the driver takes the token-major all-heads map, 0 it does not
  static std::atomic<int> all_heads_ok{-1};
  // split-heads calls (vheads > 1, hkv == 1) read one head per box from the real pool
  int box_all = vheads <= 1 && all_heads_ok.load(std::memory_order_relaxed) != 0 ? 1 : 0;
  const int map_heads = vheads > 1 ? vheads : hkv;
  int rc = NSLG_ERR_UNSUPPORTED;
  if (box_all) {
    rc = pool_tensor_map_all_heads(pool_k, num_pages, hkv, d, &tk);
    if (rc == NSLG_OK) rc = pool_tensor_map_all_heads(pool_v, num_pages, hkv, d, &tv);
    if (all_heads_ok.load(std::memory_order_relaxed) < 0)
      all_heads_ok.store(rc == NSLG_OK ? 1 : 0, std::memory_order_relaxed);
  }
  if (rc != NSLG_OK) {
    // the driver did not take the token-major strides: one box per kv head instead
    box_all = 0;
    rc = pool_tensor_map(pool_k, num_pages, map_heads, d, &tk);
    if (rc != NSLG_OK) return rc;
    rc = pool_tensor_map(pool_v, num_pages, map_heads, d, &tv);
    if (rc != NSLG_OK) return rc;
  }
  const int grid = sm_count();
  const int64_t slots = static_cast<int64_t>(batch) + grid;
  uintptr_t ws = (reinterpret_cast<uintptr_t>(workspace) + 255) & ~static_cast<uintptr_t>(255);
  DecodeParams p{};
  p.q = q;
  p.out = out;
  p.indptr = kv_indptr;
  p.indices = kv_indices;
  p.lpl = kv_last_page_len;
  p.arrive = reinterpret_cast<uint32_t*>(ws);
  p.part_o = reinterpret_cast<float*>(ws + arrive_bytes(grid));
  p.part_lse = p.part_o + slots * hq * d;
  p.q_stride = q_stride;
  p.out_stride = out_stride;
  p.num_pages = num_pages;
  p.batch = batch;
  p.hq = hq;
  p.group = hq / hkv;
  p.grid = grid;
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.status = status;
  p.box_all_heads = box_all;
  p.vheads = vheads > 1 ? vheads : 1;
  p.inline_merge = merge_inline(batch, hq, d, grid);
  {
    // NSLG_DECODE_MIN_CTA_KB overrides kMinCtaBytes (1 to 4096 KiB), for measurements
    int min_bytes = kMinCtaBytes;
    if (const char* e = std::getenv("NSLG_DECODE_MIN_CTA_KB")) {
      const int kb = std::atoi(e);
      if (kb >= 1 && kb <= 4096) min_bytes = kb << 10;
    }
    const int page_bytes = 64 * hkv * d;
    const int by_bytes = (min_bytes + page_bytes - 1) / page_bytes;
    p.min_pages = by_bytes > kMinPagesPerCta ? by_bytes : kMinPagesPerCta;
  }
  if (dtype == NSLG_DTYPE_F16) return launch_for_type<__half>(hkv, d, tk, tv, p, stream);
  return launch_for_type<__nv_bfloat16>(hkv, d, tk, tv, p, stream);
}


}  // namespace nslg
