// Causal paged prefill / extend attention on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in TMEM), bf16, page_size 16, head_dim 128.
//
// Work unit. One CTA computes 128 query rows of one kv head h: T = 128/G new tokens of
// sequence b times the G query heads h*G .. h*G+G-1 that share h (GQA), row r = token
// r/G, head r%G. Q arrives by TMA as two [T tok x G heads x 64 dims] boxes straight out
// of the caller's [rows, Hq, D] tensor (no packing: sequence b's rows start at
// q_row_start[b]), so each K/V tile is loaded once for all G heads.
//
// Pipeline (per kv tile of 64 tokens = 4 pages, 2 smem stages):
//   producer warp   TMA: per page, per 64-dim half, a [16 tok x 64] box of K and of V
//                   (128-byte swizzle; pages past the sequence are loaded from outside
//                   the tensor, which TMA fills with zeros)
//   MMA warp        S(j) = Q . K(j)^T     M=128 N=64  K=128  A,B K-major from smem
//                   O   += P(j) . V(j)    M=128 N=128 K=64   A = P from TMEM,
//                                                            B = V MN-major from smem
//   softmax WG      thread r owns TMEM lane r = row r: loads S(j), masks kpos > qpos,
//                   keeps a running max m (log2 domain) and sum l; O is rescaled in
//                   TMEM only when the max grows by more than 8 (2^8 headroom for P in
//                   bf16), P is written back to TMEM as bf16 for the PV MMA.
//   epilogue        O / l -> bf16 -> out row (q_row_start[b] + token, head).
// TMEM: S 64 columns, P 32, O 128 -> 256 allocated, two CTAs per SM.
// The MMA warp issues S(j+1) before PV(j), so the softmax of tile j+1 overlaps PV(j).
//
// Persistent grid of 2 CTAs per SM walking the (query tile, sequence, kv head) items,
// longest causal spans first; TMEM, barriers and the TMA pipeline carry across items.
//
// Every mbarrier wait is bounded (2 s); on a timeout the kernel records
// NSLG_DEV_WAIT_TIMEOUT, stops issuing work, drains what it issued (bounded), frees its
// TMEM and returns.
#include <cuda.h>

#include <string>

#include "common.cuh"
#include "launch.h"

namespace nslg {
namespace {

constexpr int kD = 128;
constexpr int kBM = 128;           // rows per CTA
constexpr int kBN = 64;            // kv tokens per tile
constexpr int kPS = 16;
constexpr int kPagesPerTile = kBN / kPS;
constexpr int kThreads = 192;      // warp 0 TMA, warp 1 MMA, warps 2-5 softmax
constexpr int kTmemCols = 256;
constexpr int kColS = 0, kColP = 64, kColO = 128;

constexpr int kQBytes = kBM * kD * 2;           // 32 KiB: [2 halves][128 rows][128 B]
constexpr int kQHalf = kBM * 128;               // 16 KiB
constexpr int kKVHalf = kBN * 128;              // 8 KiB: [64 tok][128 B]
constexpr int kKVTile = 2 * kKVHalf;            // 16 KiB per K (or V) tile
constexpr int kStageBytes = 2 * kKVTile;        // K + V: 32 KiB
constexpr int kStages = 2;
constexpr int kSmemBytes = 1024 + kQBytes + kStages * kStageBytes + 256;

struct PrefillParams {
  __nv_bfloat16* out;
  const int32_t* qo_indptr;
  const int32_t* q_row_start;
  const int32_t* indptr;
  const int32_t* indices;
  const int32_t* lpl;
  int64_t out_stride, num_pages;
  int batch, hq, hkv, group, tokens_per_tile, causal, n_items;
  float scale_log2;
  uint32_t* status;
};

// ----------------------------------------------------------------- tcgen05 wrappers
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  // start>>4 [0,14) | LBO>>4 [16,30) | SBO>>4 [32,46) | version 1 [46,48) | SWIZZLE_128B (2) [61,64)
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) |
         (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: f32 accumulate, bf16 A and B, M = 128.
__host__ __device__ constexpr uint32_t idesc_bf16(int n, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((static_cast<uint32_t>(n) >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, "
      "%10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, "
      "%27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ----------------------------------------------------------------- work items
// Item = (query tile, sequence, kv head), ordered with the query tiles that sit latest in
// their sequences -- the longest causal spans -- first; CTA c takes items c, c + grid, ...
struct Item {
  int b, h, i0, qo_len, kv_beg, npages, kv_len, ntiles, row0;
};

__device__ __forceinline__ bool load_item(const PrefillParams& p, int item, Item& it) {
  const int per = p.batch * p.hkv;
  const int tq_rev = item / per;
  const int rem = item - tq_rev * per;
  it.b = rem / p.hkv;
  it.h = rem - it.b * p.hkv;
  it.qo_len = p.qo_indptr[it.b + 1] - p.qo_indptr[it.b];
  const int ntile_q = (it.qo_len + p.tokens_per_tile - 1) / p.tokens_per_tile;
  const int tq = ntile_q - 1 - tq_rev;
  if (tq < 0) return false;
  it.i0 = tq * p.tokens_per_tile;
  it.kv_beg = p.indptr[it.b];
  it.npages = p.indptr[it.b + 1] - it.kv_beg;
  it.kv_len = it.npages > 0 ? (it.npages - 1) * kPS + p.lpl[it.b] : 0;
  const int last_tok = min(it.i0 + p.tokens_per_tile, it.qo_len) - 1;
  const int last_qpos = it.kv_len - it.qo_len + last_tok;
  const int kv_span = p.causal ? min(it.kv_len, last_qpos + 1) : it.kv_len;
  it.ntiles = (kv_span + kBN - 1) / kBN;
  if (it.ntiles <= 0) return false;
  it.row0 = (p.q_row_start ? p.q_row_start[it.b] : p.qo_indptr[it.b]) + it.i0;
  return true;
}

// ----------------------------------------------------------------- the kernel
// Persistent: each CTA walks its items with one TMEM allocation and one set of barriers.
// A global tile counter t (over all items of the CTA) drives the barrier phases, so the
// producer streams Q and K/V of the next item while the current one is still computing.
// q_empty (MMA commit after an item's last S MMA) frees the single Q buffer, o_free (the
// softmax warpgroup after reading O in an item's epilogue) frees the O accumulator for
// the next item's first P.V MMA.
__global__ void __launch_bounds__(kThreads, 2)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmap_q,
                      const __grid_constant__ CUtensorMap tmap_k,
                      const __grid_constant__ CUtensorMap tmap_v, const PrefillParams p) {
  const int G = p.group;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sq = smem;
  uint8_t* skv = smem + kQBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(skv + kStages * kStageBytes);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;        // [2]
  uint64_t* kv_empty = bars + 3;       // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* p_full = bars + 6;
  uint64_t* pv_done = bars + 7;
  uint64_t* mma_drain = bars + 8;
  uint64_t* q_empty = bars + 9;
  uint64_t* o_free = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 12);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    mbar_init(o_free, 128);
    mbar_init(mma_drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // -------------------------------------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&tmap_q);
      prefetch_tmap(&tmap_k);
      prefetch_tmap(&tmap_v);
      const uint64_t keep = l2_policy_evict_last();
      int t = 0, n_it = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
        Item it;
        if (!load_item(p, item, it)) continue;
        if (n_it > 0 && (*abort_flag || !mbar_wait(q_empty, (n_it - 1) & 1))) { ok = false; break; }
        mbar_arrive_expect_tx(q_full, kQBytes);
        tma_load_3d(sq, &tmap_q, q_full, 0, it.h * G, it.row0, keep);
        tma_load_3d(sq + kQHalf, &tmap_q, q_full, 64, it.h * G, it.row0, keep);
        ++n_it;
        // page ids of a tile are fetched together, one tile ahead of their TMA loads
        auto fetch_ids = [&](int j, int (&ids)[kPagesPerTile]) {
#pragma unroll
          for (int pg = 0; pg < kPagesPerTile; ++pg) {
            const int pi = j * kPagesPerTile + pg;
            ids[pg] = (j < it.ntiles && pi < it.npages) ? p.indices[it.kv_beg + pi] : -1;
          }
        };
        int ids[kPagesPerTile];
        fetch_ids(0, ids);
        for (int j = 0; j < it.ntiles; ++j, ++t) {
          const int s = t & 1;
          int next_ids[kPagesPerTile];
          fetch_ids(j + 1, next_ids);
          if (*abort_flag || !mbar_wait(&kv_empty[s], ((t >> 1) & 1) ^ 1)) { ok = false; break; }
          mbar_arrive_expect_tx(&kv_full[s], kStageBytes);
          uint8_t* kt = skv + s * kStageBytes;
          uint8_t* vt = kt + kKVTile;
#pragma unroll
          for (int pg = 0; pg < kPagesPerTile; ++pg) {
            const int pi = j * kPagesPerTile + pg;
            int tok_row = static_cast<int>(p.num_pages) * kPS;  // outside the pool: zeros
            if (pi < it.npages) {
              const int pid = ids[pg];
              if (pid >= 0 && pid < p.num_pages) tok_row = pid * kPS;
              else report(p.status, NSLG_DEV_BAD_PAGE);
            }
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              tma_load_3d(kt + half * kKVHalf + pg * kPS * 128, &tmap_k, &kv_full[s], half * 64,
                          it.h, tok_row, keep);
              tma_load_3d(vt + half * kKVHalf + pg * kPS * 128, &tmap_v, &kv_full[s], half * 64,
                          it.h, tok_row, keep);
            }
          }
#pragma unroll
          for (int pg = 0; pg < kPagesPerTile; ++pg) ids[pg] = next_ids[pg];
        }
      }
      if (!ok) {
        report(p.status, NSLG_DEV_WAIT_TIMEOUT);
        *abort_flag = 1;
        // no load may still be writing shared memory when the CTA leaves (bounded waits)
        if (n_it > 0) (void)mbar_wait(q_full, (n_it - 1) & 1);
        for (int u = t - 2 < 0 ? 0 : t - 2; u < t; ++u)
          (void)mbar_wait(&kv_full[u & 1], (u >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdescS = idesc_bf16(kBN, false);
      constexpr uint32_t kIdescO = idesc_bf16(kD, true);
      const uint32_t q_base = smem_u32(sq);
      auto issue_s = [&](int t) {
        const uint32_t k_base = smem_u32(skv + (t & 1) * kStageBytes);
#pragma unroll
        for (int ks = 0; ks < kD / 16; ++ks) {
          const uint32_t off = (ks >> 2) * kQHalf + (ks & 3) * 32;
          const uint32_t koff = (ks >> 2) * kKVHalf + (ks & 3) * 32;
          mma_ss(tmem + kColS, smem_desc(q_base + off, 16, 1024),
                 smem_desc(k_base + koff, 16, 1024), kIdescS, ks > 0 ? 1u : 0u);
        }
        mma_commit(s_full);
      };
      int t = 0, n_it = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
        Item it;
        if (!load_item(p, item, it)) continue;
        if (*abort_flag || !mbar_wait(q_full, n_it & 1)) { ok = false; break; }
        tc_fence_after();
        for (int j = 0; j < it.ntiles; ++j, ++t) {
          // q_empty is committed right after an item's last S MMA: Q is free once it is done
          if (j == 0) {
            if (!(ok = mbar_wait(&kv_full[t & 1], (t >> 1) & 1))) break;
            tc_fence_after();
            issue_s(t);
            if (it.ntiles == 1) mma_commit(q_empty);
          }
          if (!(ok = mbar_wait(p_full, t & 1))) break;
          tc_fence_after();
          if (j + 1 < it.ntiles) {
            if (!(ok = mbar_wait(&kv_full[(t + 1) & 1], ((t + 1) >> 1) & 1))) break;
            tc_fence_after();
            issue_s(t + 1);
            if (j + 2 == it.ntiles) mma_commit(q_empty);
          }
          if (j == 0 && n_it > 0) {
            if (!(ok = mbar_wait(o_free, (n_it - 1) & 1))) break;
            tc_fence_after();
          }
          const uint32_t v_base = smem_u32(skv + (t & 1) * kStageBytes + kKVTile);
#pragma unroll
          for (int kt = 0; kt < kBN / 16; ++kt)
            mma_ts(tmem + kColO, tmem + kColP + kt * 8,
                   smem_desc(v_base + kt * 2048, kKVHalf, 1024), kIdescO,
                   (j > 0 || kt > 0) ? 1u : 0u);
          mma_commit(pv_done);
          mma_commit(&kv_empty[t & 1]);
          if (*abort_flag) { ok = false; break; }
        }
        ++n_it;
      }
      if (!ok) {
        report(p.status, NSLG_DEV_WAIT_TIMEOUT);
        *abort_flag = 1;
      }
      // every MMA issued so far has completed once this arrives (bounded wait)
      mma_commit(mma_drain);
      (void)mbar_wait(mma_drain, 0);
    }
  } else {
    // -------------------------------------------------------------- softmax warpgroup
    const int quarter = warp & 3;              // TMEM lanes 32*quarter .. +31
    const int r = quarter * 32 + lane;         // row = TMEM lane
    const int tok = r / G, g = r % G;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const float sl = p.scale_log2;
    int t = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
      Item it;
      if (!load_item(p, item, it)) continue;
      const bool row_valid = (it.i0 + tok) < it.qo_len;
      const int qpos = it.kv_len - it.qo_len + it.i0 + tok;
      float m_ref = -INFINITY, l = 0.f;
      for (int j = 0; j < it.ntiles; ++j, ++t) {
        if (!__all_sync(0xffffffffu, mbar_wait(s_full, t & 1))) { ok = false; break; }
        tc_fence_after();
        float s[2][32];
        tmem_ld32(lane_base + kColS, s[0]);
        tmem_ld32(lane_base + kColS + 32, s[1]);
        tmem_wait_ld();
        const int kbase = j * kBN;
        float mt = -INFINITY;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const int kpos = kbase + hh * 32 + c;
            const bool vis = row_valid && kpos < it.kv_len && (!p.causal || kpos <= qpos);
            s[hh][c] = vis ? s[hh][c] * sl : -INFINITY;
            mt = fmaxf(mt, s[hh][c]);
          }
        const float m_new = fmaxf(m_ref, mt);
        const bool rescale = m_new > m_ref + 8.0f;   // also true on the first finite max
        const float alpha = (rescale && m_ref != -INFINITY) ? fast_exp2(m_ref - m_new) : 1.f;
        if (rescale) m_ref = m_new;
        float rs = 0.f;
        uint32_t pk[32];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const float p0 = m_ref == -INFINITY ? 0.f : fast_exp2(s[hh][c] - m_ref);
            const float p1 = m_ref == -INFINITY ? 0.f : fast_exp2(s[hh][c + 1] - m_ref);
            rs += p0 + p1;
            pk[hh * 16 + c / 2] = pack_bf16x2(p0, p1);
          }
        // PV of the previous tile must be done before P is overwritten or O is rescaled
        // (for j == 0 the previous item's epilogue already waited for it)
        if (j > 0) {
          if (!__all_sync(0xffffffffu, mbar_wait(pv_done, (t - 1) & 1))) { ok = false; break; }
          tc_fence_after();
          // tcgen05.ld/st are warp-collective: the whole warp takes the rescale branch
          // when any of its rows needs it (rows that do not multiply by 1)
          if (__any_sync(0xffffffffu, alpha != 1.f)) {
            for (int cb = 0; cb < kD; cb += 32) {
              float o[32];
              tmem_ld32(lane_base + kColO + cb, o);
              tmem_wait_ld();
              uint32_t w[32];
#pragma unroll
              for (int c = 0; c < 32; ++c) w[c] = __float_as_uint(o[c] * alpha);
              tmem_st32(lane_base + kColO + cb, w);
            }
          }
        }
        l = l * alpha + rs;
        tmem_st32(lane_base + kColP, pk);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(p_full);
        if (__any_sync(0xffffffffu, *abort_flag != 0)) { ok = false; break; }
      }
      if (!ok) break;
      // epilogue: O of this item -> bf16 rows, then hand O back to the MMA warp
      if (!__all_sync(0xffffffffu, mbar_wait(pv_done, (t - 1) & 1))) { ok = false; break; }
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.out + static_cast<int64_t>(it.row0 + tok) * p.out_stride +
                            static_cast<int64_t>(it.h * G + g) * kD;
      for (int cb = 0; cb < kD; cb += 32) {
        float o[32];
        tmem_ld32(lane_base + kColO + cb, o);
        tmem_wait_ld();
        if (row_valid) {
          uint4 pkt[4];
          uint32_t* u = reinterpret_cast<uint32_t*>(pkt);
#pragma unroll
          for (int c = 0; c < 32; c += 2) u[c / 2] = pack_bf16x2(o[c] * inv, o[c + 1] * inv);
#pragma unroll
          for (int v = 0; v < 4; ++v) reinterpret_cast<uint4*>(orow + cb)[v] = pkt[v];
        }
      }
      tc_fence_before();
      mbar_arrive(o_free);
    }
    if (!ok) report(p.status, NSLG_DEV_WAIT_TIMEOUT);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

}  // namespace

bool prefill_tc_supported(int dtype, int hq, int hkv, int d, int page_size) {
  if (dtype != NSLG_DTYPE_BF16 || d != kD || page_size != kPS) return false;
  if (hq % hkv) return false;
  const int g = hq / hkv;
  return g >= 1 && g <= 16 && (kBM % g) == 0;
}

int launch_paged_prefill_tc(int batch, int hq, int hkv, const void* q, int64_t q_stride,
                            int64_t q_rows, void* out, int64_t out_stride,
                            const int32_t* qo_indptr, const int32_t* q_row_start, int max_qo_len,
                            const void* pool_k, const void* pool_v, int64_t num_pages,
                            const int32_t* kv_indptr, const int32_t* kv_indices,
                            const int32_t* kv_last_page_len, float sm_scale, int causal,
                            uint32_t* status, cudaStream_t stream) {
  const int G = hq / hkv;
  const int tpt = kBM / G;
  if (num_pages * kPS >= (int64_t{1} << 31))
    return set_error(NSLG_ERR_UNSUPPORTED, "prefill: pool larger than 2^31 token rows");
  if (q_rows <= 0 || q_rows >= (int64_t{1} << 31))
    return set_error(NSLG_ERR_ARG, "prefill: q_rows out of range");
  CUtensorMap tq, tk, tv;
  int rc = pool_tensor_map(pool_k, num_pages, hkv, kD, &tk);
  if (rc != NSLG_OK) return rc;
  rc = pool_tensor_map(pool_v, num_pages, hkv, kD, &tv);
  if (rc != NSLG_OK) return rc;
  rc = encode_tiled_3d_bf16(&tq, q, kD, hq, q_rows, static_cast<uint64_t>(kD) * 2,
                            static_cast<uint64_t>(q_stride) * 2, 64, G, tpt);
  if (rc != NSLG_OK) return rc;
  PrefillParams p{};
  p.out = static_cast<__nv_bfloat16*>(out);
  p.qo_indptr = qo_indptr;
  p.q_row_start = q_row_start;
  p.indptr = kv_indptr;
  p.indices = kv_indices;
  p.lpl = kv_last_page_len;
  p.out_stride = out_stride;
  p.num_pages = num_pages;
  p.batch = batch;
  p.hq = hq;
  p.hkv = hkv;
  p.group = G;
  p.tokens_per_tile = tpt;
  p.causal = causal;
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.status = status;
  cudaError_t err = cudaFuncSetAttribute(prefill_tc_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (err != cudaSuccess) return set_error(NSLG_ERR_CUDA, cudaGetErrorString(err));
  const int64_t items = static_cast<int64_t>((max_qo_len + tpt - 1) / tpt) * batch * hkv;
  if (items >= (int64_t{1} << 31)) return set_error(NSLG_ERR_UNSUPPORTED, "prefill: too many tiles");
  p.n_items = static_cast<int>(items);
  const int64_t grid = items < 2 * static_cast<int64_t>(sm_count()) ? items : 2 * sm_count();
  prefill_tc_kernel<<<static_cast<unsigned>(grid), kThreads, kSmemBytes, stream>>>(tq, tk, tv, p);
  return check_launch("prefill_tc");
}

}  // namespace nslg
