// Causal paged prefill / extend attention on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in TMEM), bf16 or fp16, page_size 16, head_dim 128.
//
// Work item. Two adjacent query tiles ("halves" A and B) of one sequence b and one kv
// head h, each 128 rows: T = 128/G new tokens times the G query heads h*G .. h*G+G-1
// that share h (GQA), row r = token r/G, head r%G. Both halves read the same K/V tiles,
// so every K/V byte brought on chip feeds two 128-row MMAs. Q arrives by TMA as
// [T tok x G heads x 64 dims] boxes straight out of the caller's [rows, Hq, D] tensor (no
// packing: sequence b's rows start at q_row_start[b]). A persistent grid (one CTA per
// SM) walks the items, longest causal spans first (CTA c takes items c, c + grid, ...);
// TMEM, barriers and the TMA pipeline carry across items, and the next item's Q is
// loaded while the current one runs. (Dealing the items instead in equal-work units of
// a long and a short span of one (sequence, kv head) on neighbouring CTAs, so that they
// share its K/V through L2, measured 0.315 ms against 0.264 ms at the 64 x 512 bench
// shape, and the K/V re-reads this order causes are not what bounds the kernel.)
//
// Pipeline over kv tiles of 64 tokens (4 pages), t counting every tile of the CTA:
//   producer warp   TMA: Q of the next item (two Q slots), and per page and 64-dim half
//                   a [16 tok x 64] box of K (ring of 3 tiles) and of V (ring of 3); K runs
//                   one tile ahead of V. Pages past the sequence are loaded from outside
//                   the tensor (TMA fills zeros).
//   MMA warp        for X in {A, B}:
//                   S_X(t) = Q_X . K(t)^T  M=128 N=64  K=128, A and B K-major (smem),
//                   into TMEM buffer S_X[t%2];
//                   O_X += P_X(t) . V(t)   M=128 N=128 K=64, A = P_X(t) in TMEM (written
//                   over S_X[t%2]), B = V MN-major (smem).
//                   Issue order per tile: P_A(t).V(t), S_A(t+1), P_B(t).V(t), S_B(t+1).
//                   S_X(t+1) reuses the buffer of P_X(t-1), whose P.V was issued a tile
//                   earlier, so the issuer never waits on an MMA still in the pipe, and
//                   the softmax of S_A(t+1) runs while the pipe does half B's MMAs (and
//                   the other way round).
//   softmax WG X    (two warpgroups, one per half) thread r owns TMEM lane r = row r:
//                   loads S_X(t), masks only on tiles that cross the causal or length
//                   edge, keeps a running max (log2 domain) and sum, writes P in the
//                   activation type (bf16 or fp16) over S, rescales O_X in TMEM only when
//                   the max grows by more than 8 (2^8 headroom for P, within range for
//                   both types).
//   epilogue        softmax WG X reads O_X out of TMEM (then hands O_X back to the MMA
//                   warp), scales by 1/l and writes rows of the activation type into its half of the item's
//                   Q slot (dead once the item's last S is done), in the 128-byte swizzled
//                   layout of the Q load;
//   store warp      writes each staged half to `out` with two TMA stores (the Q box
//                   shape), or, for a tile that ends inside the sequence's last rows, with
//                   plain coalesced stores of the valid rows only; frees the Q slot.
// Both halves run the item's tile count (the longer span); the other half's extra
// columns are masked. TMEM: per half S[0] 64 + S[1] 64 + O 128 columns = 512.
//
// Every mbarrier wait is bounded (2 s); on a timeout the kernel records
// NSLG_DEV_WAIT_TIMEOUT, stops issuing work, drains what it issued (bounded), frees its
// TMEM and returns.
#include <cuda.h>

#include <string>

#include "common.cuh"
#include "launch.h"
#include "tcgen05.cuh"

namespace nslg {
namespace {

constexpr int kD = 128;
constexpr int kBM = 128;           // rows per half
constexpr int kBN = 64;            // kv tokens per tile
constexpr int kPS = 16;
constexpr int kPagesPerTile = kBN / kPS;
constexpr int kThreads = 352;      // warp 0 TMA, 1 MMA, 2-5 / 6-9 softmax A / B, 10 stores
constexpr int kTmemCols = 512;
constexpr int kHalfCols = 256;     // per half: S[0] at +0, S[1] at +64, O at +128
constexpr int kColO = 128;

constexpr int kQBytes = kBM * kD * 2;           // 32 KiB per half: [2 dims halves][128 rows][128 B]
constexpr int kQHalf = kBM * 128;               // 16 KiB
constexpr int kQSlot = 2 * kQBytes;             // one item's Q (both halves); two slots
constexpr int kKVHalf = kBN * 128;              // 8 KiB: [64 tok][128 B]
constexpr int kTile = 2 * kKVHalf;              // 16 KiB per K (or V) tile
constexpr int kRing = 3;                        // K ring and V ring depth
constexpr int kSmemBytes = 1024 + 2 * kQSlot + 2 * kRing * kTile + 512;

struct PrefillParams {
  void* out;        // rows of the activation type T (bf16 or fp16)
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

// ----------------------------------------------------------------- work items
// Item = (pair of query tiles, sequence, kv head), pairs latest in their sequences (the
// longest causal spans) first; CTA c takes items c, c + grid, ... Half X of pair k is
// query tile 2k + X.
struct Half {
  int i0, row0, lim_base;  // first new token, first row, kv_len - qo_len (+ i for causal)
  bool any;                // the half has rows of this sequence
};
struct Item {
  int b, h, qo_len, kv_beg, npages, kv_len, ntiles;
  Half x[2];
};

// The per-sequence values of an item, read with independent loads. A warp issues them
// one item ahead (issue_item) and turns them into the Item at the next item boundary
// (finish_item), so the loads' latency overlaps the current item instead of delaying
// the first MMA of the next one.
struct ItemLoads {
  int b, h, pk_rev;
  int qo0, qo1, ip0, ip1, lpl, rs;
};
// CTA c takes items c, c + grid, c + 2 grid, ...
__device__ __forceinline__ int first_item() { return static_cast<int>(blockIdx.x); }
__device__ __forceinline__ int next_item_id(int item) { return item + static_cast<int>(gridDim.x); }

__device__ __forceinline__ void issue_item(const PrefillParams& p, int item, ItemLoads& L) {
  if (item >= p.n_items) return;
  const int per = p.batch * p.hkv;
  L.pk_rev = item / per;
  const int rem = item - L.pk_rev * per;
  L.b = rem / p.hkv;
  L.h = rem - L.b * p.hkv;
  L.qo0 = p.qo_indptr[L.b];
  L.qo1 = p.qo_indptr[L.b + 1];
  L.ip0 = p.indptr[L.b];
  L.ip1 = p.indptr[L.b + 1];
  L.lpl = p.lpl[L.b];
  L.rs = p.q_row_start ? p.q_row_start[L.b] : L.qo0;
}

__device__ __forceinline__ bool finish_item(const PrefillParams& p, const ItemLoads& L,
                                            Item& it) {
  it.b = L.b;
  it.h = L.h;
  const int tpt = p.tokens_per_tile;
  it.qo_len = L.qo1 - L.qo0;
  const int ntile_q = (it.qo_len + tpt - 1) / tpt;
  const int npairs = (ntile_q + 1) / 2;
  const int pk = npairs - 1 - L.pk_rev;
  if (pk < 0) return false;
  it.kv_beg = L.ip0;
  it.npages = L.ip1 - L.ip0;
  it.kv_len = it.npages > 0 ? (it.npages - 1) * kPS + L.lpl : 0;
  int last_tok = -1;
  for (int x = 0; x < 2; ++x) {
    Half& hx = it.x[x];
    hx.i0 = (2 * pk + x) * tpt;
    hx.row0 = L.rs + hx.i0;
    hx.any = hx.i0 < it.qo_len;
    hx.lim_base = it.kv_len - it.qo_len + hx.i0;
    if (hx.any) last_tok = min(hx.i0 + tpt, it.qo_len) - 1;
  }
  const int kv_span = p.causal ? min(it.kv_len, it.kv_len - it.qo_len + last_tok + 1) : it.kv_len;
  it.ntiles = (kv_span + kBN - 1) / kBN;
  return it.ntiles > 0;
}

__device__ __forceinline__ bool load_item(const PrefillParams& p, int item, Item& it) {
  ItemLoads L;
  issue_item(p, item, L);
  return finish_item(p, L, it);
}

// ----------------------------------------------------------------- the kernel
// Barrier phases. K/V ring barriers complete once per use of their slot (tile t uses slot
// t % 3, parity (t / 3) & 1); per-half S-buffer barriers (s_full, p_full, pv_done) once
// per use of their buffer (parity (t >> 1) & 1); Q-slot barriers (q_full, q_empty,
// o_staged) once per use of their slot (item n uses slot n & 1, parity (n >> 1) & 1);
// o_free once per item.
template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmap_q,
                      const __grid_constant__ CUtensorMap tmap_k,
                      const __grid_constant__ CUtensorMap tmap_v,
                      const __grid_constant__ CUtensorMap tmap_o, const PrefillParams p) {
  const int G = p.group;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sq = smem;                            // [2 slots][2 halves][32 KiB]
  uint8_t* sk = smem + 2 * kQSlot;               // [kRing][2 dim halves][64 tok][128 B]
  uint8_t* sv = sk + kRing * kTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sv + kRing * kTile);
  uint64_t* q_full = bars + 0;     // [slot]
  uint64_t* q_empty = bars + 2;    // [slot]: last S done (MMA) + staged O stored (store warp)
  uint64_t* k_full = bars + 4;     // [kRing]
  uint64_t* k_empty = bars + 7;    // [kRing]
  uint64_t* v_full = bars + 10;    // [kRing]
  uint64_t* v_empty = bars + 13;   // [kRing]
  uint64_t* s_full = bars + 16;    // [half][2]
  uint64_t* p_full = bars + 20;    // [half][2]
  uint64_t* pv_done = bars + 24;   // [half][2]
  uint64_t* o_free = bars + 28;    // [half]
  uint64_t* o_staged = bars + 30;  // [half][slot]
  uint64_t* mma_drain = bars + 34;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 35);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 36);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 2);
      mbar_init(&o_free[i], 128);
    }
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
      mbar_init(&o_staged[i], 128);
    }
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
      int tk = 0, tv = 0, nq = 0;      // K tiles, V tiles, Q loads issued
      bool ok = true;
      auto q_slot_free = [&](bool block) {   // the slot of Q load nq has been released
        const uint32_t par = ((nq >> 1) & 1) ^ 1;
        return block ? mbar_wait(&q_empty[nq & 1], par) : mbar_try_wait(&q_empty[nq & 1], par);
      };
      auto load_q = [&](const Item& it) {
        const int s = nq & 1;
        mbar_arrive_expect_tx(&q_full[s], 2 * kQBytes);
        for (int x = 0; x < 2; ++x) {
          uint8_t* dst = sq + s * kQSlot + x * kQBytes;
          tma_load_3d(dst, &tmap_q, &q_full[s], 0, it.h * G, it.x[x].row0, keep);
          tma_load_3d(dst + kQHalf, &tmap_q, &q_full[s], 64, it.h * G, it.x[x].row0, keep);
        }
        ++nq;
      };
      auto fetch_ids = [&](const Item& it, int j, int (&ids)[kPagesPerTile]) {
#pragma unroll
        for (int pg = 0; pg < kPagesPerTile; ++pg) {
          const int pi = j * kPagesPerTile + pg;
          ids[pg] = (j < it.ntiles && pi < it.npages) ? p.indices[it.kv_beg + pi] : -1;
        }
      };
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
      auto next_item = [&](int from, Item& it) {
        int item = from;
        while (item < p.n_items && !load_item(p, item, it)) item = next_item_id(item);
        return item;
      };
      Item it;
      int item = next_item(first_item(), it);
      if (item < p.n_items) load_q(it);      // slot 0 starts free
      while (ok && item < p.n_items) {
        Item nx;
        const int nitem = next_item(next_item_id(item), nx);
        bool nx_q = nitem >= p.n_items;       // next item's Q issued (or no next item)
        // K(j) before V(j-1); page ids of tile j+1 fetched before waiting for K(j)'s slot;
        // the next item's Q goes out as soon as its slot is released
        int ids_v[kPagesPerTile], ids_k[kPagesPerTile], ids_n[kPagesPerTile];
        fetch_ids(it, 0, ids_k);
        for (int j = 0; j <= it.ntiles; ++j) {
          fetch_ids(it, j + 1, ids_n);
          if (!nx_q && q_slot_free(false)) {
            load_q(nx);
            nx_q = true;
          }
          if (j < it.ntiles) {
            const int s = tk % kRing;
            if (*abort_flag || !mbar_wait(&k_empty[s], ((tk / kRing) & 1) ^ 1)) { ok = false; break; }
            load_tile(it, j, ids_k, &tmap_k, sk + s * kTile, &k_full[s]);
            ++tk;
          }
          if (j > 0) {
            const int s = tv % kRing;
            if (*abort_flag || !mbar_wait(&v_empty[s], ((tv / kRing) & 1) ^ 1)) { ok = false; break; }
            load_tile(it, j - 1, ids_v, &tmap_v, sv + s * kTile, &v_full[s]);
            ++tv;
          }
#pragma unroll
          for (int pg = 0; pg < kPagesPerTile; ++pg) {
            ids_v[pg] = ids_k[pg];
            ids_k[pg] = ids_n[pg];
          }
        }
        if (!ok) break;
        if (!nx_q) {
          if (*abort_flag || !q_slot_free(true)) { ok = false; break; }
          load_q(nx);
        }
        it = nx;
        item = nitem;
      }
      if (!ok) {
        report(p.status, NSLG_DEV_WAIT_TIMEOUT);
        *abort_flag = 1;
        // no load may still be writing shared memory when the CTA leaves (bounded waits)
        for (int u = nq - 2 < 0 ? 0 : nq - 2; u < nq; ++u)
          (void)mbar_wait(&q_full[u & 1], (u >> 1) & 1);
        for (int u = tk - kRing < 0 ? 0 : tk - kRing; u < tk; ++u)
          (void)mbar_wait(&k_full[u % kRing], (u / kRing) & 1);
        for (int u = tv - kRing < 0 ? 0 : tv - kRing; u < tv; ++u)
          (void)mbar_wait(&v_full[u % kRing], (u / kRing) & 1);
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdescS = idesc_f16(Mma16<T>::kFormat, kBN, false);
      constexpr uint32_t kIdescO = idesc_f16(Mma16<T>::kFormat, kD, true);
      constexpr uint32_t kDescHi = smem_desc_hi(1024);
      // descriptor low words of the first Q slot, K slot and V slot (K-major Q and K:
      // LBO 16; MN-major V: LBO = the 64-dim half stride)
      const uint32_t q_lo0 = smem_desc_lo(smem_u32(sq), 16);
      const uint32_t k_lo0 = smem_desc_lo(smem_u32(sk), 16);
      const uint32_t v_lo0 = smem_desc_lo(smem_u32(sv), kKVHalf);
      bool ok = true;
      // S_X(u) = Q_X . K(u)^T into S_X[u%2]; the buffer is free once P_X(u-2).V is done.
      // Issued per half, right after that half's P_X(u-1).V: the wait is then on an MMA
      // issued a whole tile earlier (long complete), so the tensor pipe never drains
      // while the issuer waits, and the softmax of S_X(u) overlaps the other half's MMAs.
      auto issue_s = [&](int u, int qs, int x) -> bool {
        const int slot = u % kRing, b = u & 1;
        if (x == 0 && !mbar_wait(&k_full[slot], (u / kRing) & 1)) return false;
        const uint32_t k_lo = k_lo0 + slot * (kTile >> 4);
        if (u >= 2 && !mbar_wait(&pv_done[x * 2 + b], ((u - 2) >> 1) & 1)) return false;
        tc_fence_after();
        const uint32_t q_lo = q_lo0 + (qs * kQSlot + x * kQBytes) / 16;
        const uint32_t dcol = tmem + x * kHalfCols + 64 * b;
#pragma unroll
        for (int ks = 0; ks < kD / 16; ++ks) {
          const uint32_t off = ((ks >> 2) * kQHalf + (ks & 3) * 32) >> 4;
          const uint32_t koff = ((ks >> 2) * kKVHalf + (ks & 3) * 32) >> 4;
          mma_ss_w(dcol, q_lo + off, k_lo + koff, kDescHi, kIdescS, ks > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[x * 2 + b]);
        if (x == 1) mma_commit(&k_empty[slot]);
        return true;
      };
      int t = 0, n_it = 0;
      ItemLoads nxt;
      issue_item(p, first_item(), nxt);
      for (int item = first_item(); ok && item < p.n_items; item = next_item_id(item)) {
        const ItemLoads cur = nxt;
        issue_item(p, next_item_id(item), nxt);
        Item it;
        if (!finish_item(p, cur, it)) continue;
        const int qs = n_it & 1;
        if (*abort_flag || !mbar_wait(&q_full[qs], (n_it >> 1) & 1)) { ok = false; break; }
        tc_fence_after();
        const int t0 = t;
        const int last = t0 + it.ntiles - 1;
        for (int x = 0; ok && x < 2; ++x) ok = issue_s(t0, qs, x);
        if (ok && t0 == last) mma_commit(&q_empty[qs]);   // Q is read for the last time
        for (int j = 0; ok && j < it.ntiles; ++j, ++t) {
          const int slot = t % kRing, b = t & 1;
          if (!(ok = mbar_wait(&v_full[slot], (t / kRing) & 1))) break;
          const uint32_t v_lo = v_lo0 + slot * (kTile >> 4);
          for (int x = 0; x < 2; ++x) {
            if (!(ok = mbar_wait(&p_full[x * 2 + b], (t >> 1) & 1))) break;
            if (j == 0 && n_it > 0 && !(ok = mbar_wait(&o_free[x], (n_it - 1) & 1))) break;
            tc_fence_after();
            const uint32_t hb = tmem + x * kHalfCols;
#pragma unroll
            for (int kt = 0; kt < kBN / 16; ++kt)
              mma_ts_w(hb + kColO, hb + 64 * b + kt * 8, v_lo + (kt * 2048 >> 4), kDescHi,
                       kIdescO, (j > 0 || kt > 0) ? 1u : 0u);
            mma_commit(&pv_done[x * 2 + b]);
            if (x == 1) mma_commit(&v_empty[slot]);
            if (t + 1 <= last && !(ok = issue_s(t + 1, qs, x))) break;
          }
          if (!ok) break;
          if (t + 1 == last) mma_commit(&q_empty[qs]);
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
  } else if (warp == 10) {
    // -------------------------------------------------------------- output stores
    int n_it = 0;
    bool ok = true;
    ItemLoads nxt;
    issue_item(p, first_item(), nxt);
    for (int item = first_item(); ok && item < p.n_items; item = next_item_id(item)) {
      const ItemLoads cur = nxt;
      issue_item(p, next_item_id(item), nxt);
      Item it;
      if (!finish_item(p, cur, it)) continue;
      const int qs = n_it & 1;
      for (int x = 0; x < 2; ++x) {
        if (!__all_sync(0xffffffffu, mbar_wait(&o_staged[x * 2 + qs], (n_it >> 1) & 1))) {
          ok = false;
          break;
        }
        const Half& hx = it.x[x];
        if (!hx.any) continue;
        const uint8_t* stage = sq + qs * kQSlot + x * kQBytes;
        const int ntok = min(p.tokens_per_tile, it.qo_len - hx.i0);
        if (ntok == p.tokens_per_tile) {
          if (lane == 0) {
            tma_store_3d(&tmap_o, stage, 0, it.h * G, hx.row0);
            tma_store_3d(&tmap_o, stage + kQHalf, 64, it.h * G, hx.row0);
          }
        } else {
          // the tile ends inside the sequence: only its first ntok tokens are written
          const int rows = ntok * G;
          for (int idx = lane; idx < rows * 16; idx += 32) {
            const int r = idx >> 4, c = idx & 15, cc = c & 7;
            const uint4 v = *reinterpret_cast<const uint4*>(stage + (c >> 3) * kQHalf + r * 128 +
                                                            ((cc ^ (r & 7)) << 4));
            T* dst = static_cast<T*>(p.out) + static_cast<int64_t>(hx.row0 + r / G) * p.out_stride +
                                 static_cast<int64_t>(it.h * G + r % G) * kD + c * 8;
            *reinterpret_cast<uint4*>(dst) = v;
          }
        }
      }
      if (!ok) break;
      if (lane == 0) {
        bulk_commit_group();
        bulk_wait_read_all();   // the slot may be refilled once the stores have read it
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&q_empty[qs]);
      ++n_it;
    }
    if (lane == 0) bulk_wait_all();
    if (!ok && lane == 0) {
      report(p.status, NSLG_DEV_WAIT_TIMEOUT);
      *abort_flag = 1;
    }
  } else {
    // -------------------------------------------------------------- softmax warpgroups
    const int x = (warp - 2) / 4;                 // half A (warps 2-5) or B (warps 6-9)
    const int quarter = warp & 3;                 // TMEM lanes 32*quarter .. +31
    const int r = quarter * 32 + lane;            // row = TMEM lane
    const int tok = r / G;
    const uint32_t lane_base = tmem + x * kHalfCols + (static_cast<uint32_t>(quarter * 32) << 16);
    const float sl = p.scale_log2;
    int t = 0, n_it = 0;
    bool ok = true;
    ItemLoads nxt;
    issue_item(p, first_item(), nxt);
    for (int item = first_item(); ok && item < p.n_items; item = next_item_id(item)) {
      const ItemLoads cur = nxt;
      issue_item(p, next_item_id(item), nxt);
      Item it;
      if (!finish_item(p, cur, it)) continue;
      const Half& hx = it.x[x];
      const bool row_valid = (hx.i0 + tok) < it.qo_len;
      // last kv position the row sees (-1: none)
      const int lim = row_valid ? (p.causal ? min(hx.lim_base + tok, it.kv_len - 1) : it.kv_len - 1)
                                : -1;
      float m_ref = -INFINITY, l = 0.f;   // m_ref in log2 units (raw score * sl)
      for (int j = 0; j < it.ntiles; ++j, ++t) {
        const int b = t & 1;
        const uint32_t scol = 64 * b;
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[x * 2 + b], (t >> 1) & 1))) { ok = false; break; }
        tc_fence_after();
        float s[64];
        tmem_ld64(lane_base + scol, s);
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
          pk[c / 2] = Mma16<T>::pack(p0, p1);
        }
        // O may only be rescaled once P(t-1).V(t-1) is done (warp-uniform branch: the
        // tcgen05.ld/st are warp-collective; rows with alpha == 1 multiply by 1)
        if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
          if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[x * 2 + (b ^ 1)], ((t - 1) >> 1) & 1))) {
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
        mbar_arrive(&p_full[x * 2 + b]);
        if (__any_sync(0xffffffffu, *abort_flag != 0)) { ok = false; break; }
      }
      if (!ok) break;
      // epilogue: O of this half -> TMEM is handed back -> bf16 rows staged in this half of
      // the item's Q slot (128-byte swizzle: 16-byte chunk c of row r at c ^ (r & 7)), for
      // the store warp
      const int tl = t - 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[x * 2 + (tl & 1)], (tl >> 1) & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int qs = n_it & 1;
      uint8_t* stage = sq + qs * kQSlot + x * kQBytes + r * 128;
      for (int cb = 0; cb < kD; cb += 64) {
        float o0[32], o1[32];
        tmem_ld32(lane_base + kColO + cb, o0);
        tmem_ld32(lane_base + kColO + cb + 32, o1);
        tmem_wait_ld();
        if (cb + 64 == kD) {
          tc_fence_before();
          mbar_arrive(&o_free[x]);                  // O_X may be overwritten now
        }
        uint8_t* row = stage + (cb >> 6) * kQHalf;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float* src = c < 4 ? &o0[c * 8] : &o1[(c - 4) * 8];
          uint4 pkt;
          pkt.x = Mma16<T>::pack(src[0] * inv, src[1] * inv);
          pkt.y = Mma16<T>::pack(src[2] * inv, src[3] * inv);
          pkt.z = Mma16<T>::pack(src[4] * inv, src[5] * inv);
          pkt.w = Mma16<T>::pack(src[6] * inv, src[7] * inv);
          *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) << 4)) = pkt;
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&o_staged[x * 2 + qs]);
      ++n_it;
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
  if ((dtype != NSLG_DTYPE_BF16 && dtype != NSLG_DTYPE_F16) || d != kD || page_size != kPS)
    return false;
  if (hq % hkv) return false;
  const int g = hq / hkv;
  return g >= 1 && g <= 16 && (kBM % g) == 0;
}

int launch_paged_prefill_tc(int dtype, int batch, int hq, int hkv, const void* q,
                            int64_t q_stride,
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
  CUtensorMap tq, tk, tv, to;
  int rc = pool_tensor_map(pool_k, num_pages, hkv, kD, &tk);
  if (rc != NSLG_OK) return rc;
  rc = pool_tensor_map(pool_v, num_pages, hkv, kD, &tv);
  if (rc != NSLG_OK) return rc;
  rc = encode_tiled_3d_bf16(&tq, q, kD, hq, q_rows, static_cast<uint64_t>(kD) * 2,
                            static_cast<uint64_t>(q_stride) * 2, 64, G, tpt);
  if (rc != NSLG_OK) return rc;
  // out rows have the Q layout; the store box is the Q box
  rc = encode_tiled_3d_bf16(&to, out, kD, hq, q_rows, static_cast<uint64_t>(kD) * 2,
                            static_cast<uint64_t>(out_stride) * 2, 64, G, tpt);
  if (rc != NSLG_OK) return rc;
  PrefillParams p{};
  p.out = out;
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
  auto kern = dtype == NSLG_DTYPE_F16 ? prefill_tc_kernel<__half> : prefill_tc_kernel<__nv_bfloat16>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemBytes);
  if (err != cudaSuccess) return set_error(NSLG_ERR_CUDA, cudaGetErrorString(err));
  const int64_t pairs = ((max_qo_len + tpt - 1) / tpt + 1) / 2;
  const int64_t items = pairs * batch * hkv;
  p.n_items = static_cast<int>(items);
  const int64_t grid = items < static_cast<int64_t>(sm_count()) ? items : sm_count();
  kern<<<static_cast<unsigned>(grid), kThreads, kSmemBytes, stream>>>(tq, tk, tv, to, p);
  return check_launch("prefill_tc");
}

}  // namespace nslg
