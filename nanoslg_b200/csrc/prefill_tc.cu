// Causal paged prefill / extend attention on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in TMEM), bf16, page_size 16, head_dim 128.
//
// Work item. 128 query rows of one kv head h: T = 128/G new tokens of sequence b times
// the G query heads h*G .. h*G+G-1 that share h (GQA), row r = token r/G, head r%G. Q
// arrives by TMA as two [T tok x G heads x 64 dims] boxes straight out of the caller's
// [rows, Hq, D] tensor (no packing: sequence b's rows start at q_row_start[b]), so each
// K/V tile is loaded once for all G heads. A persistent grid (2 CTAs per SM) walks the
// items, longest causal spans first; TMEM, barriers and the TMA pipeline carry across
// items.
//
// Pipeline over kv tiles of 64 tokens (4 pages), t counting every tile of the CTA:
//   producer warp   TMA, per page and 64-dim half, a [16 tok x 64] box of K (ring of 2)
//                   and of V (ring of 2); K runs one tile ahead of V. Pages past the
//                   sequence are loaded from outside the tensor, which TMA fills with
//                   zeros.
//   MMA warp        S(t) = Q . K(t)^T  M=128 N=64  K=128, A and B K-major (smem),
//                   into TMEM buffer S[t%2];
//                   O += P(t) . V(t)   M=128 N=128 K=64, A = P(t) in TMEM (written over
//                   S[t%2]), B = V MN-major (smem).
//                   S(t+2) goes into S[t%2] as soon as P(t) . V(t) is done, so the
//                   softmax of tile t+1 overlaps P(t).V(t) and S(t+2).
//   softmax WG      thread r owns TMEM lane r = row r: loads S(t), masks only on tiles
//                   that cross the causal or length edge, keeps a running max (log2
//                   domain) and sum, writes P as bf16 over S, rescales O in TMEM only when
//                   the max grows by more than 8 (2^8 headroom for P in bf16).
//   epilogue        O / l -> bf16 -> out row (q_row_start[b] + token, head); then O is
//                   handed back to the MMA warp for the next item.
// TMEM: S[0] 64 columns, S[1] 64, O 128 = 256, two CTAs per SM.
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
constexpr int kBM = 128;           // rows per item
constexpr int kBN = 64;            // kv tokens per tile
constexpr int kPS = 16;
constexpr int kPagesPerTile = kBN / kPS;
constexpr int kThreads = 192;      // warp 0 TMA, warp 1 MMA, warps 2-5 softmax
constexpr int kTmemCols = 256;
constexpr int kColS = 0;           // S[b] at kColS + 64*b, P(t) over S[t%2]
constexpr int kColO = 128;

constexpr int kQBytes = kBM * kD * 2;           // 32 KiB: [2 halves][128 rows][128 B]
constexpr int kQHalf = kBM * 128;               // 16 KiB
constexpr int kKVHalf = kBN * 128;              // 8 KiB: [64 tok][128 B]
constexpr int kTile = 2 * kKVHalf;              // 16 KiB per K (or V) tile
constexpr int kRing = 2;                        // K ring and V ring depth
constexpr int kSmemBytes = 1024 + kQBytes + 2 * kRing * kTile + 256;

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
// Barrier phases. Every per-buffer barrier (k/v full/empty, s_full, p_full, pv_done)
// completes once per tile that uses its buffer, so the tile t's phase parity there is
// (t >> 1) & 1; q_full, q_empty and o_free complete once per item.
__global__ void __launch_bounds__(kThreads, 2)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmap_q,
                      const __grid_constant__ CUtensorMap tmap_k,
                      const __grid_constant__ CUtensorMap tmap_v, const PrefillParams p) {
  const int G = p.group;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sq = smem;
  uint8_t* sk = smem + kQBytes;                 // [kRing][2 halves][64 tok][128 B]
  uint8_t* sv = sk + kRing * kTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sv + kRing * kTile);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;     // [2]
  uint64_t* k_empty = bars + 4;    // [2]
  uint64_t* v_full = bars + 6;     // [2]
  uint64_t* v_empty = bars + 8;    // [2]
  uint64_t* s_full = bars + 10;    // [2]
  uint64_t* p_full = bars + 12;    // [2]
  uint64_t* pv_done = bars + 14;   // [2]
  uint64_t* o_free = bars + 16;
  uint64_t* mma_drain = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 19);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
    }
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
      int tk = 0, tv = 0, n_it = 0;      // K tiles, V tiles, Q loads issued
      bool ok = true;
      // page ids of tile j of the item (-1 past the sequence)
      auto fetch_ids = [&](const Item& it, int j, int (&ids)[kPagesPerTile]) {
#pragma unroll
        for (int pg = 0; pg < kPagesPerTile; ++pg) {
          const int pi = j * kPagesPerTile + pg;
          ids[pg] = (j < it.ntiles && pi < it.npages) ? p.indices[it.kv_beg + pi] : -1;
        }
      };
      // loads one [64 tok x 128 dim] tile (K or V) of the item into ring slot `slot`
      auto load_tile = [&](const Item& it, int j, const int (&ids)[kPagesPerTile],
                           const CUtensorMap* map, uint8_t* dst, uint64_t* bar) {
        mbar_arrive_expect_tx(bar, kTile);
#pragma unroll
        for (int pg = 0; pg < kPagesPerTile; ++pg) {
          const int pi = j * kPagesPerTile + pg;
          int tok_row = static_cast<int>(p.num_pages) * kPS;  // outside the pool: zeros
          if (pi < it.npages) {
            if (ids[pg] >= 0 && ids[pg] < p.num_pages) tok_row = ids[pg] * kPS;
            else report(p.status, NSLG_DEV_BAD_PAGE);
          }
#pragma unroll
          for (int half = 0; half < 2; ++half)
            tma_load_3d(dst + half * kKVHalf + pg * kPS * 128, map, bar, half * 64, it.h,
                        tok_row, keep);
        }
      };
      for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
        Item it;
        if (!load_item(p, item, it)) continue;
        if (n_it > 0 && (*abort_flag || !mbar_wait(q_empty, (n_it - 1) & 1))) { ok = false; break; }
        mbar_arrive_expect_tx(q_full, kQBytes);
        tma_load_3d(sq, &tmap_q, q_full, 0, it.h * G, it.row0, keep);
        tma_load_3d(sq + kQHalf, &tmap_q, q_full, 64, it.h * G, it.row0, keep);
        ++n_it;
        // K(j) before V(j-1): keys run one tile ahead of values. The page ids of tile j+1
        // are fetched before waiting for K(j)'s slot, so their latency is hidden, and are
        // reused for V one tile later.
        int ids_v[kPagesPerTile], ids_k[kPagesPerTile], ids_n[kPagesPerTile];
        fetch_ids(it, 0, ids_k);
        for (int j = 0; j <= it.ntiles; ++j) {
          fetch_ids(it, j + 1, ids_n);
          if (j < it.ntiles) {
            const int s = tk & 1;
            if (*abort_flag || !mbar_wait(&k_empty[s], ((tk >> 1) & 1) ^ 1)) { ok = false; break; }
            load_tile(it, j, ids_k, &tmap_k, sk + s * kTile, &k_full[s]);
            ++tk;
          }
          if (j > 0) {
            const int s = tv & 1;
            if (*abort_flag || !mbar_wait(&v_empty[s], ((tv >> 1) & 1) ^ 1)) { ok = false; break; }
            load_tile(it, j - 1, ids_v, &tmap_v, sv + s * kTile, &v_full[s]);
            ++tv;
          }
#pragma unroll
          for (int pg = 0; pg < kPagesPerTile; ++pg) {
            ids_v[pg] = ids_k[pg];
            ids_k[pg] = ids_n[pg];
          }
        }
      }
      if (!ok) {
        report(p.status, NSLG_DEV_WAIT_TIMEOUT);
        *abort_flag = 1;
        // no load may still be writing shared memory when the CTA leaves (bounded waits)
        if (n_it > 0) (void)mbar_wait(q_full, (n_it - 1) & 1);
        for (int u = tk - 2 < 0 ? 0 : tk - 2; u < tk; ++u)
          (void)mbar_wait(&k_full[u & 1], (u >> 1) & 1);
        for (int u = tv - 2 < 0 ? 0 : tv - 2; u < tv; ++u)
          (void)mbar_wait(&v_full[u & 1], (u >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdescS = idesc_bf16(kBN, false);
      constexpr uint32_t kIdescO = idesc_bf16(kD, true);
      const uint32_t q_base = smem_u32(sq);
      bool ok = true;
      // S(u) into S[u%2]; the buffer is free once P(u-2).V(u-2) is done
      auto issue_s = [&](int u) -> bool {
        const int b = u & 1;
        if (!mbar_wait(&k_full[b], (u >> 1) & 1)) return false;
        if (u >= 2 && !mbar_wait(&pv_done[b], ((u - 2) >> 1) & 1)) return false;
        tc_fence_after();
        const uint32_t k_base = smem_u32(sk + b * kTile);
#pragma unroll
        for (int ks = 0; ks < kD / 16; ++ks) {
          const uint32_t off = (ks >> 2) * kQHalf + (ks & 3) * 32;
          const uint32_t koff = (ks >> 2) * kKVHalf + (ks & 3) * 32;
          mma_ss(tmem + kColS + 64 * b, smem_desc(q_base + off, 16, 1024),
                 smem_desc(k_base + koff, 16, 1024), kIdescS, ks > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[b]);
        mma_commit(&k_empty[b]);
        return true;
      };
      int t = 0, n_it = 0;
      for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
        Item it;
        if (!load_item(p, item, it)) continue;
        if (*abort_flag || !mbar_wait(q_full, n_it & 1)) { ok = false; break; }
        tc_fence_after();
        const int t0 = t;
        const int last = t0 + it.ntiles - 1;
        for (int u = t0; ok && u <= last && u < t0 + 2; ++u) {
          ok = issue_s(u);
          if (ok && u == last) mma_commit(q_empty);   // Q is free once the last S is done
        }
        for (int j = 0; ok && j < it.ntiles; ++j, ++t) {
          const int b = t & 1;
          if (!(ok = mbar_wait(&p_full[b], (t >> 1) & 1))) break;
          if (j == 0 && n_it > 0 && !(ok = mbar_wait(o_free, (n_it - 1) & 1))) break;
          if (!(ok = mbar_wait(&v_full[b], (t >> 1) & 1))) break;
          tc_fence_after();
          const uint32_t v_base = smem_u32(sv + b * kTile);
#pragma unroll
          for (int kt = 0; kt < kBN / 16; ++kt)
            mma_ts(tmem + kColO, tmem + kColS + 64 * b + kt * 8,
                   smem_desc(v_base + kt * 2048, kKVHalf, 1024), kIdescO,
                   (j > 0 || kt > 0) ? 1u : 0u);
          mma_commit(&pv_done[b]);
          mma_commit(&v_empty[b]);
          if (t + 2 <= last) {
            ok = issue_s(t + 2);
            if (ok && t + 2 == last) mma_commit(q_empty);
          }
          if (*abort_flag) ok = false;
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
      // last kv position the row sees (-1: none)
      const int lim = row_valid ? (p.causal ? min(it.kv_len - it.qo_len + it.i0 + tok,
                                                  it.kv_len - 1)
                                            : it.kv_len - 1)
                                : -1;
      float m_ref = -INFINITY, l = 0.f;   // m_ref in log2 units (raw score * sl)
      for (int j = 0; j < it.ntiles; ++j, ++t) {
        const int b = t & 1;
        const uint32_t scol = kColS + 64 * b;
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[b], (t >> 1) & 1))) { ok = false; break; }
        tc_fence_after();
        float s[64];
        tmem_ld32(lane_base + scol, *reinterpret_cast<float(*)[32]>(&s[0]));
        tmem_ld32(lane_base + scol + 32, *reinterpret_cast<float(*)[32]>(&s[32]));
        tmem_wait_ld();
        const int kbase = j * kBN;
        // columns past `lim` are masked; interior tiles (every row of the warp sees the
        // whole tile) skip the per-column test
        if (!__all_sync(0xffffffffu, kbase + kBN - 1 <= lim)) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (kbase + c > lim) s[c] = -INFINITY;
        }
        float mt = s[0];
#pragma unroll
        for (int c = 1; c < 64; ++c) mt = fmaxf(mt, s[c]);
        const float m_new = fmaxf(m_ref, mt * sl);
        const bool rescale = m_new > m_ref + 8.0f;   // also true on the first finite max
        const float alpha = (rescale && m_ref != -INFINITY) ? fast_exp2(m_ref - m_new) : 1.f;
        if (rescale) m_ref = m_new;
        const float neg = m_ref == -INFINITY ? 0.f : -m_ref;
        float rs = 0.f;
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 64; c += 2) {
          const float p0 = fast_exp2(fmaf(s[c], sl, neg));
          const float p1 = fast_exp2(fmaf(s[c + 1], sl, neg));
          rs += p0 + p1;
          pk[c / 2] = pack_bf16x2(p0, p1);
        }
        // O may only be rescaled once P(t-1).V(t-1) is done (warp-uniform branch: the
        // tcgen05.ld/st are warp-collective; rows with alpha == 1 multiply by 1)
        if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
          if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[b ^ 1], ((t - 1) >> 1) & 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
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
        l = l * alpha + rs;
        tmem_st32(lane_base + scol, pk);           // P(t) over S(t)
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[b]);
        if (__any_sync(0xffffffffu, *abort_flag != 0)) { ok = false; break; }
      }
      if (!ok) break;
      // epilogue: O of this item -> bf16 rows, then hand O back to the MMA warp
      const int tl = t - 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[tl & 1], (tl >> 1) & 1))) { ok = false; break; }
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
