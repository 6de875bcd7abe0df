"""B200 paged KV cache behind NanoSLG's ``CacheContext`` boundary.

Drop-in for ``nanoslg/kv_cache.py``: the same ``KVCacheConfig``, ``CacheContext`` and
``KVCacheManager`` ABCs, the same page pool (page 0 = null page, refcounts, a free *set*
whose ``pop()`` order decides page ids, zero-on-alloc, copy-on-write) and the same
per-token radix prefix tree, so page tables, write slots and CSR arrays are bit-exact
with the reference's (kv_cache.py:382-531, 694-777).  What changes is behind
``attend()``: instead of FlashInfer's wrappers (kv_cache.py:703-705, 618-632, 650, 654)
or contiguous SDPA (kv_cache.py:312-322), each layer launches the sm_100a kernels of
``nanoslg_b200/csrc`` through the C ABI -- the KV append (optionally fused with RoPE,
see ``attend_rope``) and split-KV decode or causal prefill attention reading the pages
in place.  The per-forward plan (positions, write slots, CSR) is built once per
``begin_forward``: for decode steps on a CUDA pool it is built on the GPU from block
tables mirrored in device memory (one ``nslg_plan_decode_host`` call per step, which
also zeroes the newly allocated pages), otherwise on the host and shipped to the
device in one host-to-device copy.

``create_cache_manager`` always returns the B200 backend: there is no second backend
and no CPU fallback; the bookkeeping itself runs on any device (tests drive it with
CPU tensors), the kernels need CUDA.
"""
import math
import threading
from abc import ABC, abstractmethod
from dataclasses import dataclass
from typing import Dict, List, Optional, Set, Tuple

import numpy as np
import torch

from . import _native as N
from . import ops


@dataclass
class KVCacheConfig:
    """Cache sizing (kv_cache.py:59-145). ``backend`` is kept for config compatibility;
    every value selects the B200 paged backend."""
    num_layers: int
    num_kv_heads: int          # per TP rank
    num_qo_heads: int          # per TP rank
    head_dim: int
    page_size: int = 16
    max_pages: int = 0         # 0 = auto
    max_batch_size: int = 8
    max_seq_len: int = 4096
    memory_fraction: float = 0.30
    dtype: torch.dtype = torch.bfloat16
    device: torch.device = None
    enable_prefix_caching: bool = True
    backend: str = "b200"

    def __post_init__(self):
        if self.backend not in ("auto", "b200", "flashinfer", "contiguous"):
            raise ValueError(f"unknown kv backend {self.backend!r}")
        self.backend = "b200"
        if self.max_pages <= 0:
            self.max_pages = self._auto_pages()

    def _elem_bytes(self) -> int:
        return {torch.float16: 2, torch.bfloat16: 2, torch.float32: 4}.get(self.dtype, 2)

    def _auto_pages(self) -> int:
        """Same budget rule as the reference (kv_cache.py:88-102): free memory minus a
        max(2 GiB, 15%) headroom, times memory_fraction, capped at 65536 pages."""
        if self.device is None or torch.device(self.device).type != "cuda":
            return 256
        try:
            free, total = torch.cuda.mem_get_info(self.device)
        except Exception:
            return 256
        headroom = max(2 << 30, int(total * 0.15))
        budget = int(max(0, free - headroom) * self.memory_fraction)
        per_page = (2 * self.num_layers * self.page_size * self.num_kv_heads
                    * self.head_dim * self._elem_bytes())
        return max(64, min(budget // max(per_page, 1), 65536))

    @classmethod
    def from_hf_config(cls, hf_config, parallel_config=None, device=None, **kw):
        """Per-rank shape from an HF config (kv_cache.py:119-145)."""
        nl = getattr(hf_config, "num_hidden_layers", getattr(hf_config, "num_layers", 32))
        nkv = getattr(hf_config, "num_key_value_heads",
                      getattr(hf_config, "multi_query_group_num",
                              getattr(hf_config, "num_attention_heads", 32)))
        nq = getattr(hf_config, "num_attention_heads", 32)
        hd = getattr(hf_config, "head_dim",
                     getattr(hf_config, "kv_channels", hf_config.hidden_size // nq))
        if parallel_config is not None:
            tp = parallel_config.tp_size
            if tp > 1:
                nkv //= tp
                nq //= tp
            if parallel_config.pp_size > 1 and parallel_config.pp_layer_splits:
                try:
                    from .parallel import ParallelContext
                    ctx = ParallelContext.get()
                    if ctx and ctx.pp_rank in parallel_config.pp_layer_splits:
                        nl = len(parallel_config.pp_layer_splits[ctx.pp_rank])
                except Exception:
                    pass
        return cls(num_layers=nl, num_kv_heads=nkv, num_qo_heads=nq, head_dim=hd,
                   device=device, **kw)


class CacheContext(ABC):
    """Per-forward context handed to every layer (kv_cache.py:149-163)."""
    seq_ids: List[str]
    new_token_counts: List[int]
    input_offsets: List[int]
    batch_size: int
    seq_lens: List[int]

    @abstractmethod
    def get_position_ids(self, max_input_len: int) -> torch.Tensor: ...

    @abstractmethod
    def attend(self, layer_idx: int, q: torch.Tensor, k_new: torch.Tensor,
               v_new: torch.Tensor, n_heads: int, n_kv_heads: int) -> torch.Tensor: ...

    @abstractmethod
    def get_start_pos(self, batch_idx: int = 0) -> int: ...


class KVCacheManager(ABC):
    """Cache manager interface (kv_cache.py:166-189)."""
    cfg: KVCacheConfig

    @abstractmethod
    def allocate_sequence(self, seq_id: str, token_ids: Optional[List[int]] = None,
                          num_tokens: int = 0) -> int: ...

    @abstractmethod
    def extend_sequence(self, seq_id: str, num_new: int = 1): ...

    @abstractmethod
    def begin_forward(self, seq_ids: List[str], new_token_counts: List[int],
                      input_offsets: Optional[List[int]] = None) -> CacheContext: ...

    @abstractmethod
    def end_forward(self, ctx: CacheContext): ...

    @abstractmethod
    def release_sequence(self, seq_id: str): ...

    @abstractmethod
    def append_token_ids(self, seq_id: str, new_ids: List[int]): ...

    @abstractmethod
    def reset(self): ...

    @property
    @abstractmethod
    def stats(self) -> Dict: ...


class PagePool:
    """K/V pages ``[num_layers, max_pages, page_size, num_kv_heads, head_dim]``; page 0 is
    the permanent null page (kv_cache.py:382-442).

    Page ids come from ``set.pop()`` on a free set built and updated exactly as the
    reference does, so the same call sequence hands out the same ids.  The reference
    zeroes a page on every allocation with two small copies per page; here the ids are
    queued and zeroed together by ``flush_zero()`` before the device next touches the
    pool (the context calls it when it is built, ``cow`` before its copy), which leaves
    the same pool contents."""

    def __init__(self, cfg: KVCacheConfig):
        self.cfg = cfg
        shape = (cfg.num_layers, cfg.max_pages, cfg.page_size, cfg.num_kv_heads, cfg.head_dim)
        self.k = torch.zeros(shape, dtype=cfg.dtype, device=cfg.device)
        self.v = torch.zeros(shape, dtype=cfg.dtype, device=cfg.device)
        self.ref_count = [0] * cfg.max_pages
        # numpy, so a decode step updates the pages of a whole batch in one indexed op
        self.tokens_used = np.zeros(cfg.max_pages, dtype=np.int32)
        self.ref_count[0] = 1
        self.free_set: Set[int] = set(range(1, cfg.max_pages))
        self._lock = threading.Lock()
        self._pending_zero: List[int] = []
        # per-layer views, made once (indexing the pool tensor every call costs more
        # than the views themselves)
        self.k_layers = [self.k[i] for i in range(cfg.num_layers)]
        self.v_layers = [self.v[i] for i in range(cfg.num_layers)]
        self.layer_ptrs = [(a.data_ptr(), b.data_ptr())
                           for a, b in zip(self.k_layers, self.v_layers)]

    def alloc(self, n=1) -> Optional[List[int]]:
        with self._lock:
            if len(self.free_set) < n:
                return None
            out = []
            for _ in range(n):
                pid = self.free_set.pop()
                self.ref_count[pid] = 1
                self.tokens_used[pid] = 0
                out.append(pid)
            self._pending_zero.extend(out)
            return out

    def alloc_one(self) -> Optional[int]:
        """The page ``alloc(1)`` would hand out (same free-set pop), or None when the pool
        is empty."""
        with self._lock:
            fs = self.free_set
            if not fs:
                return None
            pid = fs.pop()
            self.ref_count[pid] = 1
            self.tokens_used[pid] = 0
            self._pending_zero.append(pid)
            return pid

    def take_pending_zero(self) -> List[int]:
        """The pages allocated since the last flush (sorted, unique); the caller zeroes
        them (``nslg_plan_decode_host`` on the device-planned path, ``flush_zero``
        otherwise)."""
        with self._lock:
            if not self._pending_zero:
                return []
            ids = sorted(set(self._pending_zero))
            self._pending_zero.clear()
            return ids

    def flush_zero(self):
        """Zeroes every page allocated since the last flush (all layers, K and V)."""
        ids = self.take_pending_zero()
        if not ids:
            return
        idx = torch.tensor(ids, dtype=torch.long).to(self.k.device, non_blocking=True)
        self.k.index_fill_(1, idx, 0)
        self.v.index_fill_(1, idx, 0)

    def release(self, pid):
        if pid <= 0:
            return
        with self._lock:
            self.ref_count[pid] -= 1
            if self.ref_count[pid] <= 0:
                self.ref_count[pid] = 0
                self.tokens_used[pid] = 0
                self.free_set.add(pid)

    def add_ref(self, pid):
        with self._lock:
            self.ref_count[pid] += 1

    def is_shared(self, pid):
        return self.ref_count[pid] > 1

    def cow(self, pid):
        new = self.alloc(1)
        if new is None:
            return None
        d = new[0]
        self.flush_zero()
        self.k[:, d].copy_(self.k[:, pid])
        self.v[:, d].copy_(self.v[:, pid])
        self.tokens_used[d] = self.tokens_used[pid]
        return d

    @property
    def num_free(self):
        return len(self.free_set)

    @property
    def utilization(self):
        return 1.0 - self.num_free / max(self.cfg.max_pages - 1, 1)


class _RNode:
    __slots__ = ("children", "page_id", "ref", "last_access", "depth")

    def __init__(self, d=0):
        self.children: Dict[int, "_RNode"] = {}
        self.page_id = -1
        self.ref = 0
        self.last_access = 0
        self.depth = d


class RadixTree:
    """Per-token prefix trie with a page id at every page-aligned depth
    (kv_cache.py:453-531).  ``last_access`` is a logical clock ticked once per
    match/insert call: the eviction order equals the reference's wall-clock order."""

    def __init__(self, ps, pool):
        self.root = _RNode()
        self.ps = ps
        self.pool = pool
        self._lock = threading.Lock()
        self._clock = 0

    def _tick(self):
        self._clock += 1
        return self._clock

    def match(self, tokens):
        with self._lock:
            node, pages, now = self.root, [], self._tick()
            for i, tok in enumerate(tokens):
                ch = node.children.get(tok)
                if ch is None:
                    break
                node = ch
                node.last_access = now
                if (i + 1) % self.ps == 0 and node.page_id >= 0:
                    if self.pool.ref_count[node.page_id] > 0:
                        pages.append(node.page_id)
                    else:
                        node.page_id = -1
                        break
            return len(pages) * self.ps, pages

    def insert(self, tokens, page_ids):
        with self._lock:
            node, pi, now = self.root, 0, self._tick()
            for i, tok in enumerate(tokens):
                if tok not in node.children:
                    node.children[tok] = _RNode(i + 1)
                node = node.children[tok]
                node.last_access = now
                if (i + 1) % self.ps == 0 and pi < len(page_ids):
                    incoming = page_ids[pi]
                    pi += 1
                    if node.page_id < 0:
                        node.page_id = incoming
                        self.pool.add_ref(incoming)

    def add_refs(self, tokens, n=1):
        with self._lock:
            node = self.root
            for tok in tokens:
                ch = node.children.get(tok)
                if ch is None:
                    break
                node = ch
                node.ref += n

    def dec_refs(self, tokens, n=1):
        with self._lock:
            node = self.root
            for tok in tokens:
                ch = node.children.get(tok)
                if ch is None:
                    break
                node = ch
                node.ref = max(0, node.ref - n)

    def evict_lru(self, need):
        with self._lock:
            cands = []
            self._collect(self.root, cands)
            cands.sort(key=lambda x: x[0])
            freed = 0
            for _, nd, par, edge in cands:
                if freed >= need:
                    break
                if nd.ref > 0:
                    continue
                if nd.page_id >= 0:
                    self.pool.release(nd.page_id)
                    nd.page_id = -1
                    freed += 1
                if not nd.children and par is not None:
                    par.children.pop(edge, None)
            return freed

    def _collect(self, node, out, par=None, edge=-1):
        # iterative pre-order walk in the reference's visiting order (deep tries of
        # long prompts would overflow Python's recursion limit)
        stack = [(node, par, edge)]
        while stack:
            nd, pa, ed = stack.pop()
            if nd.page_id >= 0 and nd.ref == 0:
                out.append((nd.last_access, nd, pa, ed))
            for t, ch in reversed(list(nd.children.items())):
                stack.append((ch, nd, t))

    @property
    def cached_pages(self):
        c, stack = 0, [self.root]
        while stack:
            n = stack.pop()
            if n.page_id >= 0:
                c += 1
            stack.extend(n.children.values())
        return c


class _BlockTable(list):
    """A sequence's page list -- the reference's ``block_table`` list, same contents and
    list behaviour -- with an int32 numpy mirror kept in step on every append, extend and
    item assignment, so a forward's CSR page list is a concatenation of array prefixes
    instead of a Python loop over every page of every sequence."""
    __slots__ = ("arr", "dirty_from")

    def __init__(self, pages=()):
        super().__init__(pages)
        self.dirty_from = 0    # entries [dirty_from, len) differ from the device copy
        self.arr = np.empty(max(16, 2 * len(self)), dtype=np.int32)
        if len(self):
            self.arr[:len(self)] = np.asarray(self, dtype=np.int32)

    def _reserve(self, n, keep):
        """Capacity for n entries, preserving the first ``keep``."""
        if n > self.arr.size:
            grown = np.empty(max(n, 2 * self.arr.size), dtype=np.int32)
            grown[:keep] = self.arr[:keep]
            self.arr = grown

    def extend(self, pages):
        pages = list(pages)
        old = len(self)
        self._reserve(old + len(pages), old)
        super().extend(pages)
        self.arr[old:len(self)] = pages
        if old < self.dirty_from:
            self.dirty_from = old

    def append(self, page):
        old = len(self)
        if old >= self.arr.size:
            self._reserve(old + 1, old)
        super().append(page)
        self.arr[old] = page
        if old < self.dirty_from:
            self.dirty_from = old

    def __setitem__(self, i, v):
        super().__setitem__(i, v)
        if isinstance(i, slice):
            self._resync()
        else:
            j = i if i >= 0 else i + len(self)
            self.arr[j] = v
            if j < self.dirty_from:
                self.dirty_from = j

    def _resync(self):
        """Mirror rebuilt from the list, every entry marked for upload (after the list
        operations the bookkeeping never uses on a block table)."""
        self._reserve(len(self), 0)
        self.arr[:len(self)] = np.asarray(self, dtype=np.int32)
        self.dirty_from = 0

    def __iadd__(self, pages):
        self.extend(pages)
        return self

    def __imul__(self, n):
        super().__imul__(n)
        self._resync()
        return self

    def __delitem__(self, i):
        super().__delitem__(i)
        self._resync()

    def insert(self, i, page):
        super().insert(i, page)
        self._resync()

    def pop(self, i=-1):
        page = super().pop(i)
        self._resync()
        return page

    def remove(self, page):
        super().remove(page)
        self._resync()

    def clear(self):
        super().clear()
        self._resync()

    def sort(self, *args, **kw):
        super().sort(*args, **kw)
        self._resync()

    def reverse(self):
        super().reverse()
        self._resync()

    def prefix(self, n):
        """int32 array of the first n page ids, 0 (the null page) past the end."""
        if n <= len(self):
            return self.arr[:n]
        return np.concatenate([self.arr[:len(self)], np.zeros(n - len(self), np.int32)])


class _PagedSeqState:
    __slots__ = ("seq_id", "block_table", "_n", "prefix_len", "token_ids", "slot")
    # bumped by every assignment to num_tokens (a decode batch cached by the manager is
    # only reused while nothing outside its own begin/end changed a token count)
    version = 0

    def __init__(self, sid, prefix_pages=None, plen=0, tids=None):
        self.slot = -1          # row of the device block tables (device planning)
        self.seq_id = sid
        self.block_table = _BlockTable(prefix_pages or [])
        self._n = plen
        self.prefix_len = plen
        self.token_ids = list(tids or [])

    @property
    def num_tokens(self):
        return self._n

    @num_tokens.setter
    def num_tokens(self, v):
        self._n = v
        _PagedSeqState.version += 1


class _DecodeBatch:
    """A decode batch planned on the device, kept for the next step of the same batch:
    its sequence states, table rows, token counts before the step, the page holding each
    sequence's next position, and the longest block table; ``open`` is the context of
    its step begun and not yet ended. Every step moves all start positions on by one, so
    the sequences whose next position opens a page at step ``t`` (counted from when the
    batch was built) are ``buckets[t % page_size]``, and ``total``, the number of page
    ids in the step's plan, grows by that bucket's size."""
    __slots__ = ("ids", "mut", "ver", "sts", "slots", "n0", "ptrs", "cur_pid", "longest",
                 "open", "t", "buckets", "total")


class B200CacheContext(CacheContext):
    """Per-forward context of the B200 backend.

    Host side (once per forward) it computes what ``FlashInferCacheContext.__init__``
    computes (kv_cache.py:547-632): start positions and sequence lengths, the per-token
    (page, slot) write targets with copy-on-write of shared pages, and the CSR page list
    ``kv_indptr / kv_indices / kv_last_page_len`` (+ ``qo_indptr`` for prefill).  On a
    CUDA pool a decode step (one new token per sequence, no copy-on-write) is planned on
    the GPU instead (``B200PagedKVCache._begin_decode_device``, ``nslg_plan_decode_host``);
    otherwise the arrays travel to the device in one copy. Either way they are int32
    views of one buffer:

      positions [B*iw]  absolute position of every input cell (0 for left padding)
      write_loc [B*iw]  page*page_size + slot of every input cell, -1 = not written
      kv_indptr [B+1], kv_indices [T], kv_last_page_len [B], qo_indptr [B+1],
      q_row_start [B] = b*iw + input_offsets[b]  (first real row of sequence b)

    Per layer, ``attend`` / ``attend_rope`` launch the append kernel and the decode
    (all counts == 1) or prefill kernel; no Python loop runs per layer.
    """

    def __init__(self, cache: "B200PagedKVCache", seq_ids, new_token_counts, input_offsets,
                 states=None):
        self.cache = cache
        self.seq_ids = seq_ids
        self.new_token_counts = new_token_counts
        self.input_offsets = input_offsets or [0] * len(seq_ids)
        self.batch_size = B = len(seq_ids)
        cfg = cache.cfg
        pool = cache.pool
        ps = cfg.page_size
        dev = cfg.device

        sts = states if states is not None else [cache.seqs[s] for s in seq_ids]
        self.start_positions = [st.num_tokens for st in sts]
        self.seq_lens = [self.start_positions[i] + new_token_counts[i] for i in range(B)]
        self.max_kv_len = max(self.seq_lens) if self.seq_lens else 0
        self._is_decode = all(n == 1 for n in new_token_counts)
        self._split_plan = None      # split-heads page list, built by the first decode call
        self._iw = (max(o + n for o, n in zip(self.input_offsets, new_token_counts))
                    if B else 1)
        iw = self._iw

        # Decode fast path: one new token per sequence, every target page allocated and
        # private (no copy-on-write): the write targets are whole-batch array arithmetic.
        # Anything else takes the general loop below.
        self._wi = None
        self._wi_src = None
        self._direct_ptrs = None
        fast = self._is_decode and iw == 1 and B > 0
        if fast:
            rc = pool.ref_count
            pids = []
            for st, start in zip(sts, self.start_positions):
                bt = st.block_table
                pi = start // ps
                if pi >= len(bt) or rc[bt[pi]] > 1:
                    fast = False
                    break
                pids.append(bt[pi])
        if fast:
            start = np.asarray(self.start_positions, dtype=np.int64)
            slots = start % ps
            tu = pool.tokens_used
            pa = np.asarray(pids, dtype=np.int64)     # distinct: every page is private
            tu[pa] = np.maximum(tu[pa], slots + 1)
            self._wi_src = (pids, slots.tolist())
            positions = start.astype(np.int32).reshape(B, 1)
            write_loc = (np.asarray(pids, dtype=np.int64) * ps + slots).astype(np.int32).reshape(B, 1)
        else:
            positions, write_loc = self._general_write_targets(sts, new_token_counts, iw, ps)

        self._finish_plan(B, iw, ps, sts, positions, write_loc, new_token_counts, dev)

    _PLAN_VIEWS = frozenset(("_pos_i32", "_write_loc", "kv_indptr", "kv_last_page_len",
                             "qo_indptr", "q_row_start", "kv_indices"))

    def __getattr__(self, name):
        # a device-planned decode step builds its plan views and its per-sequence lists on
        # first use (most steps only need the raw pointers)
        d = self.__dict__
        if name in B200CacheContext._PLAN_VIEWS:
            src = d.get("_plan_src")
            if src is not None:
                self._set_plan_views(*src)
                return d[name]
        elif name in ("start_positions", "seq_lens", "max_kv_len"):
            n0 = d.get("_n0")
            if n0 is not None:
                d["start_positions"] = n0.tolist()
                d["seq_lens"] = (n0 + 1).tolist()
                d["max_kv_len"] = int(n0.max()) + 1
                return d[name]
        raise AttributeError(name)

    def _set_plan_views(self, d, B, iw, total):
        """Slices the plan arrays out of the flat int32 device buffer ``d`` (layout of the
        class docstring, page ids last)."""
        sizes = [B * iw, B * iw, B + 1, max(B, 1), B + 1, B, total]
        offs = np.cumsum([0] + sizes)
        views = [d[offs[i]:offs[i + 1]] for i in range(len(sizes))]
        (self._pos_i32, self._write_loc, self.kv_indptr, self.kv_last_page_len,
         self.qo_indptr, self.q_row_start, self.kv_indices) = views
        self.kv_last_page_len = self.kv_last_page_len[:max(B, 1)]
        return int(offs[-1])

    @property
    def _write_info(self) -> List[List[Tuple[int, int]]]:
        """(page, slot) of every new token of every sequence (kv_cache.py:575-594)."""
        if self._wi is None:
            if self._wi_src is not None:           # a decode step: one token each
                pids, slots = self._wi_src
                self._wi = [[(int(p_), int(s_))] for p_, s_ in zip(pids, slots)]
            else:                                  # the general path's array part
                wi, fast, pids, slots, beg = self._wi_parts
                pl, sl = pids.tolist(), slots.tolist()
                for j, b in enumerate(fast):
                    wi[b] = list(zip(pl[beg[j]:beg[j + 1]], sl[beg[j]:beg[j + 1]]))
                self._wi = wi
        return self._wi

    def _general_write_targets(self, sts, new_token_counts, iw, ps):
        """Write targets of any forward, with copy-on-write (kv_cache.py:575-594).

        A sequence whose new tokens land in pages shared with another owner goes through
        the reference's page-by-page order (the first token written into a shared page
        copies it); all other sequences -- every sequence of a prefill into fresh pages
        -- are computed together as arrays. Copy-on-write only allocates new private
        pages and drops references to shared ones, so a sequence found to write private
        pages only still does after the copies of the sequences before it."""
        B = self.batch_size
        pool = self.cache.pool
        rc = pool.ref_count
        positions = np.zeros((B, iw), dtype=np.int32)
        write_loc = np.full((B, iw), -1, dtype=np.int32)
        wi: List = [None] * B
        fast = []
        distinct = len(set(self.seq_ids)) == B
        for b in range(B):
            st = sts[b]
            n = new_token_counts[b]
            if n <= 0:
                wi[b] = []
                continue
            start = st.num_tokens
            p0, p1 = start // ps, (start + n - 1) // ps
            bt = st.block_table
            if distinct and p1 < len(bt) and max(map(rc.__getitem__, bt[p0:p1 + 1])) <= 1:
                fast.append(b)
                continue
            try:
                wi[b] = self._write_targets_in_order(st, n, self.input_offsets[b],
                                                     positions[b], write_loc[b], ps)
            except RuntimeError:
                # out of pages for a copy: the sequences before this one have marked
                # their pages (tokens_used), as in the reference's token loop
                if fast:
                    self._private_targets(fast, sts, new_token_counts, iw, ps, positions,
                                          write_loc)
                raise
        if not fast:
            self._wi = wi
            return positions, write_loc
        pids, slots, beg = self._private_targets(fast, sts, new_token_counts, iw, ps,
                                                 positions, write_loc)
        self._wi = None
        self._wi_parts = (wi, fast, pids, slots, beg)
        return positions, write_loc

    def _private_targets(self, fast, sts, new_token_counts, iw, ps, positions, write_loc):
        """Write targets of the sequences ``fast``, which write only private pages, in
        position order, as arrays: fills their cells of positions / write_loc, raises
        tokens_used of their pages, returns (page ids, slots, per-sequence bounds)."""
        fb = np.asarray(fast, dtype=np.int64)
        n = np.asarray([new_token_counts[b] for b in fast], dtype=np.int64)
        start = np.asarray([sts[b].num_tokens for b in fast], dtype=np.int64)
        off = np.asarray([self.input_offsets[b] for b in fast], dtype=np.int64)
        beg = np.zeros(len(fast) + 1, dtype=np.int64)
        np.cumsum(n, out=beg[1:])
        seq = np.repeat(np.arange(len(fast)), n)
        i = np.arange(int(beg[-1]), dtype=np.int64) - beg[seq]
        pos = start[seq] + i
        tabs = [sts[b].block_table for b in fast]
        tbase = np.zeros(len(fast) + 1, dtype=np.int64)
        np.cumsum([len(t) for t in tabs], out=tbase[1:])
        flat = np.concatenate([t.arr[:len(t)] for t in tabs])
        pids = flat[tbase[seq] + pos // ps].astype(np.int64)
        slots = pos % ps
        cells = fb[seq] * iw + off[seq] + i
        positions.reshape(-1)[cells] = pos
        write_loc.reshape(-1)[cells] = pids * ps + slots
        # tokens_used: the last token written into each page has its highest slot (a
        # private page belongs to one sequence, whose tokens arrive in order)
        last = np.empty(pids.shape[0], dtype=bool)
        last[:-1] = pids[1:] != pids[:-1]
        last[-1] = True
        tu = self.cache.pool.tokens_used
        lp = pids[last]
        tu[lp] = np.maximum(tu[lp], slots[last] + 1)
        return pids, slots, beg

    def _write_targets_in_order(self, st, n, o, pos_row, loc_row, ps):
        """One sequence's write targets page by page in the reference's order, copying
        each shared page it writes into; fills its rows of positions / write_loc and
        returns its (page, slot) list."""
        pool = self.cache.pool
        start = st.num_tokens
        info: List[Tuple[int, int]] = []
        pos_row[o:o + n] = np.arange(start, start + n, dtype=np.int32)
        ap = start
        end = start + n
        while ap < end:
            pi = ap // ps
            stop = min(end, (pi + 1) * ps)
            if pi >= len(st.block_table):
                info.extend([(0, 0)] * (stop - ap))
            else:
                pid = st.block_table[pi]
                if pool.is_shared(pid):
                    np_ = pool.cow(pid)
                    if np_ is None:
                        raise RuntimeError("KV OOM during CoW")
                    st.block_table[pi] = np_
                    pool.release(pid)
                    pid = np_
                info.extend((pid, sl) for sl in range(ap % ps, stop - pi * ps))
                pool.tokens_used[pid] = max(pool.tokens_used[pid], stop - pi * ps)
            ap = stop
        loc_row[o:o + n] = [p_ * ps + s_ for p_, s_ in info]
        return info

    def _finish_plan(self, B, iw, ps, sts, positions, write_loc, new_token_counts, dev):
        cache = self.cache
        cfg = cache.cfg
        pool = cache.pool
        # CSR page list (kv_cache.py:598-615)
        kv_lens = np.asarray(self.seq_lens, dtype=np.int64)
        npgs = (kv_lens + ps - 1) // ps
        indptr = np.zeros(B + 1, dtype=np.int32)
        indptr[1:] = np.cumsum(npgs)
        # an empty batch still gets one page id and one last-page length of 0, like the
        # reference's `indices or [0]` / `lpl or [0]` (kv_cache.py:612-615)
        lpl = (np.where(npgs > 0, kv_lens - (npgs - 1) * ps, 0).astype(np.int32) if B
               else np.zeros(1, dtype=np.int32))
        total = int(indptr[B])
        indices = (np.concatenate([st.block_table.prefix(n)
                                   for st, n in zip(sts, npgs.tolist())])
                   if total else np.zeros(1, dtype=np.int32))
        qo = np.zeros(B + 1, dtype=np.int32)
        qo[1:] = np.cumsum(new_token_counts, dtype=np.int64) if B else []
        row_start = (np.arange(B, dtype=np.int32) * iw
                     + np.asarray(self.input_offsets, dtype=np.int32)) if B else \
            np.zeros(0, dtype=np.int32)

        # one int32 buffer, page ids last so that every other view sits at an offset that
        # depends only on (B, input width): a fixed plan buffer keeps them in place
        parts = [positions.ravel(), write_loc.ravel(), indptr, lpl, qo, row_start,
                 indices]
        offs = np.cumsum([0] + [p.size for p in parts])
        size = int(offs[-1])
        dev_t = torch.device(dev) if dev is not None else torch.device("cpu")
        if dev_t.type == "cuda":
            # assembled straight into a reused pinned buffer (one host->device copy)
            host = cache._pinned_plan(size)
            np.concatenate(parts, out=host.numpy())
        else:
            host = torch.from_numpy(np.concatenate(parts))
        flat_size = size
        pool.flush_zero()
        static = cache.static_plan_for(B, iw, flat_size)
        self.plan_static = static is not None
        if static is not None:
            static[:flat_size].copy_(host, non_blocking=True)
            d = static
        else:
            d = host.to(dev_t, non_blocking=True)
        if dev_t.type == "cuda":
            cache._plan_copied()
        views = [d[offs[i]:offs[i + 1]] for i in range(len(parts))]
        (self._pos_i32, self._write_loc, self.kv_indptr, self.kv_last_page_len,
         self.qo_indptr, self.q_row_start, self.kv_indices) = views
        self.kv_last_page_len = self.kv_last_page_len[:max(B, 1)]
        self._plan_bytes = flat_size * 4
        self._pos64 = None
        self._sm_scale = 1.0 / math.sqrt(cfg.head_dim)

    # -- CacheContext ------------------------------------------------------------
    def get_position_ids(self, S):
        if self._pos64 is None:
            self._pos64 = self._pos_i32.view(self.batch_size, self._iw).long()
        pos = self._pos64
        if S <= self._iw:
            return pos[:, :S]
        return torch.cat([pos, pos.new_zeros(self.batch_size, S - self._iw)], 1)

    def get_start_pos(self, idx=0):
        return self.start_positions[idx]

    def attend(self, layer_idx, q, k_new, v_new, n_heads, n_kv_heads):
        """q, k_new already rotated (the ABC contract, models.py:99-105)."""
        self._check_width(q)
        if self._is_decode:
            out = self._decode_direct(layer_idx, q, k_new, v_new)
            if out is not None:
                return out
        pool = self.cache.pool
        ops.rope_kv_append(None, k_new, v_new, None, None, None, self._write_loc,
                           pool.k_layers[layer_idx], pool.v_layers[layer_idx], rotate=False)
        return self._attention(layer_idx, q)

    def attend_rope(self, layer_idx, q, k_new, v_new, cos, sin):
        """Fused path: RoPE on q and k (positions from this context, rows of the fp32
        cos/sin tables of models.py:37-66), KV append, attention."""
        self._check_width(q)
        pool = self.cache.pool
        B, S, hq, d = q.shape
        q_rot = ops.rope_kv_append(q, k_new, v_new, self._pos_i32, cos, sin, self._write_loc,
                                   pool.k_layers[layer_idx], pool.v_layers[layer_idx])
        return self._attention(layer_idx, q_rot.view(B, S, hq, d))

    def attend_qkv(self, layer_idx, x, w_qkv, n_heads, n_kv_heads, cos, sin):
        """Decode steps: the layer's q|k|v product, RoPE and KV append in one kernel
        (``ops.linear_rope_append``, x [B, 1, hidden] against the stacked [q; k; v]
        weight), then attention -- what the projections followed by ``attend_rope`` do.
        Returns None (nothing launched) where that kernel does not take the operands;
        the caller then projects and calls ``attend_rope``."""
        if not self._is_decode or x.dim() != 3:
            return None
        B, S, _ = x.shape
        if B != self.batch_size or S != self._iw:
            return None
        pool = self.cache.pool
        q_rot = ops.linear_rope_append(x, w_qkv, n_heads, n_kv_heads, self._pos_i32, cos, sin,
                                       self._write_loc, pool.k_layers[layer_idx],
                                       pool.v_layers[layer_idx])
        if q_rot is None:
            return None
        return self._attention(layer_idx, q_rot.view(B, S, n_heads, -1))

    def _decode_direct(self, layer_idx, q, k, v):
        """Decode ``attend`` straight through one C call (``nslg_append_paged_decode``: KV
        append, then paged decode), skipping the generic wrappers' per-call checks, for
        the common inputs:
        dense CUDA q [B, 1, Hq, D] and k, v [B, 1, Hkv, D] of the pool's dtype and head
        sizes. Returns None for anything else (the caller takes the generic path)."""
        pool = self.cache.pool
        pk = pool.k_layers[layer_idx]
        dt = pk.dtype
        if not (q.is_cuda and q.dtype == dt and k.dtype == dt and v.dtype == dt
                and q.dim() == 4 and k.dim() == 4 and k.shape == v.shape
                and k.shape[0] == q.shape[0] and k.shape[1] == 1
                and k.shape[2] == pk.shape[2] and k.shape[3] == pk.shape[3]
                and q.shape[3] == pk.shape[3] and q.shape[2] % k.shape[2] == 0
                and q.is_contiguous() and k.is_contiguous() and v.is_contiguous()):
            return None
        B, _, hq, d = q.shape
        P, ps, hkv, _ = pk.shape
        lib, dtc, status, ws_t = self.cache._direct_state(B, hq, d, q.device)
        ws, wsb = ws_t.data_ptr(), ws_t.numel()
        ptrs = self._direct_ptrs
        if ptrs is None:
            ptrs = self._direct_ptrs = (self._write_loc.data_ptr(), self.kv_indptr.data_ptr(),
                                        self.kv_indices.data_ptr(),
                                        self.kv_last_page_len.data_ptr())
        stream = ops._stream(q)
        pkp, pvp = pool.layer_ptrs[layer_idx]
        out = torch.empty((B, 1, hq * d), dtype=dt, device=q.device)
        rc = lib.nslg_append_paged_decode(dtc, B, hq, hkv, d, ps, q.data_ptr(), hq * d,
                                          k.data_ptr(), hkv * d, v.data_ptr(), hkv * d, ptrs[0],
                                          out.data_ptr(), hq * d, pkp, pvp, P, ptrs[1], ptrs[2],
                                          ptrs[3], self._sm_scale, ws, wsb, status, stream)
        if rc:
            raise N.NativeError("nslg_append_paged_decode", rc, lib.nslg_last_error().decode())
        return out

    def _check_width(self, q):
        if q.shape[0] != self.batch_size or q.shape[1] != self._iw:
            raise ValueError(f"attend: q is {tuple(q.shape[:2])}, the context was planned for "
                             f"{(self.batch_size, self._iw)} (batch, input width)")

    def _attention(self, layer_idx, q):
        B, S, hq, d = q.shape
        pool = self.cache.pool
        pk, pv = pool.k_layers[layer_idx], pool.v_layers[layer_idx]
        if self._is_decode:
            hkv = pk.shape[2]
            if (2 <= hkv and B * hkv <= ops.DECODE_SPLIT_HEADS_PAIRS and q.dtype != torch.float32
                    and d in (64, 128) and pk.shape[1] == 16 and hq // hkv <= 16):
                # small batches: the decode split by kv head as well as by pages (the split
                # page list built once per step, at the first layer)
                if self._split_plan is None:
                    self._split_plan = ops.split_heads_plan(self.kv_indptr, self.kv_indices,
                                                            self.kv_last_page_len, hkv,
                                                            pk.shape[0])
                out = ops.paged_decode_split_heads(q[:, 0].contiguous(), pk, pv,
                                                   self._split_plan, self._sm_scale)
                return out.view(B, 1, hq * d)
            out = ops.paged_decode(q[:, 0], pk, pv, self.kv_indptr, self.kv_indices,
                                   self.kv_last_page_len, self._sm_scale)
            return out.view(B, 1, hq * d)
        out = torch.zeros((B, S, hq, d), dtype=q.dtype, device=q.device)
        ops.paged_prefill(q, self.qo_indptr, S, pk, pv, self.kv_indptr, self.kv_indices,
                          self.kv_last_page_len, self._sm_scale, causal=True,
                          q_row_start=self.q_row_start, out=out)
        return out.view(B, S, hq * d)


class B200PagedKVCache(KVCacheManager):
    """Paged manager (kv_cache.py:694-777) with the FlashInfer wrappers removed."""

    def __init__(self, cfg: KVCacheConfig):
        self.cfg = cfg
        self.pool = PagePool(cfg)
        self.tree = RadixTree(cfg.page_size, self.pool) if cfg.enable_prefix_caching else None
        self.seqs: Dict[str, _PagedSeqState] = {}
        self._static_plans: Dict[Tuple[int, int], torch.Tensor] = {}
        self._direct = {}             # (batch, heads, head_dim) -> direct decode state
        self._mut = 0                 # bumped by every bookkeeping change outside the
        self._dc = None               # cached decode batch's own steps (_DecodeBatch)
        self._pin_buf = None          # pinned host staging of the plan, reused per forward
        self._pin_event = None        # recorded after the copy out of it
        # device planning of decode steps (CUDA pools): block tables mirrored on the GPU,
        # one row ("slot") per live sequence, rows reused after release
        dev = torch.device(cfg.device) if cfg.device is not None else torch.device("cpu")
        self.device_plan = dev.type == "cuda"
        self._dbt = None              # int32 [rows, stride] device block tables
        self._slot_free: List[int] = []
        self._slot_next = 0
        self._up_dev = None           # device copy of (slots, starts, table updates, zeroes)
        self._plan_dev = None         # device plan buffer of the forwards without a static one
        self._hs = None               # host scratch of table updates and pages to zero
        self._hs_ptr = 0
        self._pc = None               # constant arguments of nslg_plan_decode_host

    def use_static_plan(self, batch, input_width=1, max_pages=None):
        """From now on, forwards of exactly (batch, input_width) put their plan into one
        fixed device buffer (page-id capacity ``max_pages``, default the whole pool), so a
        CUDA graph captured over one such forward can be replayed for the later ones."""
        # page-list capacity: every sequence lists its shared prefix pages again, so the
        # list can be longer than the pool; size it for full-length sequences
        ps = self.cfg.page_size
        cap = max_pages if max_pages is not None else max(
            self.cfg.max_pages, batch * -(-self.cfg.max_seq_len // ps))
        n = 2 * batch * input_width + (batch + 1) + max(batch, 1) + (batch + 1) + batch + cap
        self._static_plans[(batch, input_width)] = torch.zeros(
            n, dtype=torch.int32, device=self.cfg.device)

    def static_plan_for(self, batch, input_width, size):
        """The fixed plan buffer of (batch, input_width), or None when there is none or
        this plan does not fit it (the forward then gets a buffer of its own, and
        ``plan_static`` of its context is False)."""
        buf = self._static_plans.get((batch, input_width))
        if buf is not None and size > buf.numel():
            return None
        return buf

    def _direct_state(self, batch, hq, d, device):
        """(library, dtype code, status word pointer, decode workspace pointer and size)
        for the direct decode path, looked up once per (batch, heads, head_dim)."""
        key = (batch, hq, d)
        st = self._direct.get(key)
        if st is None:
            lib = N.lib()
            wsb = lib.nslg_decode_workspace_bytes(batch, hq, d)
            ws = ops._STATE.workspace(device, wsb)
            # the tuple holds the workspace tensor itself: it stays allocated even if the
            # shared workspace is regrown for a larger call later
            st = (lib, ops._dtype_code(self.pool.k), ops.status_word(device).data_ptr(), ws)
            self._direct[key] = st
        return st

    def _pinned_plan(self, size):
        """A pinned int32 host buffer of ``size`` entries for this forward's plan; the
        previous forward's copy out of it has completed before it is handed out again."""
        buf = self._pin_buf
        if buf is None or buf.numel() < size:
            cap = max(size, 4096, 2 * (buf.numel() if buf is not None else 0))
            if self._pin_event is not None:
                self._pin_event.synchronize()
            self._pin_buf = buf = torch.empty(cap, dtype=torch.int32).pin_memory()
        elif self._pin_event is not None:
            self._pin_event.synchronize()
        return buf[:size]

    def _plan_copied(self, stream=None):
        if self._pin_event is None:
            self._pin_event = torch.cuda.Event()
        self._pin_event.record(stream if stream is not None
                               else torch.cuda.current_stream(self.cfg.device))

    def _ensure_tables(self, rows, stride):
        cur = self._dbt
        r0, s0 = (cur.shape if cur is not None else (0, 0))
        if rows <= r0 and stride <= s0:
            return
        nr = max(rows, r0 if rows <= r0 else 2 * r0, 64)
        ns = max(stride, s0 if stride <= s0 else 2 * s0, 256)
        new = torch.zeros((nr, ns), dtype=torch.int32, device=self.cfg.device)
        if cur is not None:
            new[:r0, :s0].copy_(cur)
        self._dbt = new

    def _begin_decode_device(self, seq_ids, ntoks):
        """begin_forward for a decode step (one new token per sequence) planned on the
        device, in one pass over the batch: page extension (in batch order, as
        extend_sequence), the write page, tokens_used, the device table row and the table
        entries to upload. Returns None -- with nothing done but page extensions, which
        the general path repeats idempotently -- when a target page is shared (copy on
        write)."""
        ps = self.cfg.page_size
        rc = self.pool.ref_count
        tu = self.pool.tokens_used
        seqs = self.seqs
        sts, starts, pids, slots, dirty = [], [], [], [], []
        longest = 0
        for sid in seq_ids:
            st = seqs[sid]
            n0 = st.num_tokens
            bt = st.block_table
            nb = len(bt)
            if n0 >= nb * ps:
                bt.extend(self._alloc(n0 // ps + 1 - nb))
                nb = len(bt)
            pid = bt[n0 // ps]
            if rc[pid] > 1:
                return None
            if st.slot < 0:
                if self._slot_free:
                    st.slot = self._slot_free.pop()
                else:
                    st.slot = self._slot_next
                    self._slot_next += 1
                bt.dirty_from = 0
            if bt.dirty_from < nb:
                dirty.append(st)
            if nb > longest:
                longest = nb
            sts.append(st)
            starts.append(n0)
            pids.append(pid)
            slots.append(st.slot)
        B = len(sts)
        pa = np.asarray(pids, dtype=np.int64)         # distinct: every page is private
        st0 = np.asarray(starts, dtype=np.int64)
        tu[pa] = np.maximum(tu[pa], st0 % ps + 1)
        nu = self._stage_updates(dirty)
        self._ensure_tables(self._slot_next, longest)
        c = _DecodeBatch()
        c.ids = list(seq_ids)
        c.mut = self._mut
        c.ver = _PagedSeqState.version
        c.sts = sts
        c.slots = np.asarray(slots, dtype=np.int32)
        c.n0 = np.asarray(starts, dtype=np.int32)
        c.ptrs = (c.slots.ctypes.data, c.n0.ctypes.data)
        c.cur_pid = np.asarray(pids, dtype=np.int64)
        c.longest = longest
        c.t = 0
        c.buckets = [[] for _ in range(ps)]
        for i, x in enumerate(starts):
            c.buckets[-x % ps].append(i)
        c.total = int((st0 // ps).sum()) + B
        self._dc = c
        ctx = self._decode_context(c, seq_ids, ntoks, c.n0 % ps)
        ctx._wi_src = (pids, ctx._wi_src[1])
        self._launch_device_plan(ctx, c, nu)
        return ctx

    def _begin_decode_cached(self, c, seq_ids, ntoks):
        """Next decode step of the cached batch ``c``: only the sequences whose next
        position opens a page are visited (page extension in batch order, copy-on-write
        check); everything else is array arithmetic. None (cache dropped) when a page to
        write is shared: the general path takes the step."""
        ps = self.cfg.page_size
        n0 = c.n0
        rem = n0 % ps
        dirty = []
        opening = c.buckets[c.t % ps]
        if opening:
            rc = self.pool.ref_count
            alloc_one = self.pool.alloc_one
            sts = c.sts
            for i in opening:
                st = sts[i]
                bt = st.block_table
                pi = int(n0[i]) // ps
                nb = len(bt)
                if pi >= nb:
                    pid = alloc_one() if pi == nb else None
                    if pid is not None:
                        bt.append(pid)
                    else:       # several pages, or eviction / the OOM error of _alloc
                        bt.extend(self._alloc(pi + 1 - nb))
                    nb = len(bt)
                    if nb > c.longest:
                        c.longest = nb
                pid = bt[pi]
                if rc[pid] > 1:
                    self._dc = None
                    return None
                c.cur_pid[i] = pid
                if bt.dirty_from < nb:
                    dirty.append(st)
        # tokens_used of each sequence's page: positions fill a private page in order
        # (the pages are private, so the ids are distinct)
        tu = self.pool.tokens_used
        tu[c.cur_pid] = np.maximum(tu[c.cur_pid], rem + 1)
        nu = self._stage_updates(dirty) if dirty else 0
        self._ensure_tables(self._slot_next, c.longest)
        ctx = self._decode_context(c, seq_ids, ntoks, rem)
        self._launch_device_plan(ctx, c, nu)
        return ctx

    def _decode_context(self, c, seq_ids, ntoks, rem):
        """The context of a device-planned decode step of batch ``c`` (start positions
        ``c.n0``, in-page slots ``rem``); its plan arrays come from _launch_device_plan."""
        n0 = c.n0
        B = n0.shape[0]
        ctx = B200CacheContext.__new__(B200CacheContext)
        ctx.cache = self
        ctx.seq_ids = seq_ids
        ctx.new_token_counts = ntoks
        ctx.input_offsets = [0] * B
        ctx.batch_size = B
        ctx._n0 = n0.copy()       # start_positions / seq_lens / max_kv_len, built on use
        ctx._is_decode = True
        ctx._split_plan = None
        ctx._iw = 1
        ctx._wi = None
        ctx._wi_src = (c.cur_pid.copy(), rem)
        ctx._sm_scale = 1.0 / math.sqrt(self.cfg.head_dim)
        ctx._pos64 = None
        ctx._dc = c
        c.open = ctx
        return ctx

    def _host_scratch(self, n):
        """The int32 host array the table updates and pages to zero are written into
        (at least ``n`` entries; reallocation moves it)."""
        hs = self._hs
        if hs is None or hs.size < n:
            new = np.empty(max(n, 4096, 2 * (hs.size if hs is not None else 0)), dtype=np.int32)
            if hs is not None:
                new[:hs.size] = hs
            self._hs = hs = new
            self._hs_ptr = new.ctypes.data
        return hs

    def _stage_updates(self, dirty):
        """Writes the block-table entries of every sequence in ``dirty`` changed since its
        last upload, as (table row, index, page id) triples, to the start of the host
        scratch; returns how many."""
        k = 0
        for st in dirty:
            bt = st.block_table
            d, nb = bt.dirty_from, len(bt)
            n = nb - d
            hs = self._host_scratch(3 * (k + n))
            if n == 1:
                j = 3 * k
                hs[j] = st.slot
                hs[j + 1] = d
                hs[j + 2] = bt.arr[d]
            else:
                v = hs[3 * k:3 * (k + n)].reshape(n, 3)
                v[:, 0] = st.slot
                v[:, 1] = np.arange(d, nb, dtype=np.int32)
                v[:, 2] = bt.arr[d:nb]
            k += n
            bt.dirty_from = nb
        return k

    def _plan_consts(self):
        pc = self._pc
        if pc is None:
            pool = self.pool
            dev = torch.device(self.cfg.device)
            idx = dev.index if dev.index is not None else torch.cuda.current_device()
            page_bytes = pool.k[0, 0].numel() * pool.k.element_size()
            pc = self._pc = (N.lib(), pool.k.data_ptr(), pool.v.data_ptr(), pool.k.shape[0],
                             pool.k.shape[1], page_bytes,
                             ops.status_word(torch.device("cuda", idx)).data_ptr(), idx)
        return pc

    def _launch_device_plan(self, ctx, c, nu):
        """One nslg_plan_decode_host call: the batch's table rows and start positions
        (arrays of ``c``), the ``nu`` table updates at the start of the host scratch and
        the pages to zero after them; the plan goes to the static buffer of this batch
        size when there is one and it fits, else to the manager's own plan buffer."""
        n0 = c.n0
        B = n0.shape[0]
        ps = self.cfg.page_size
        total = c.total                                # sum of ceil((start + 1) / ps)
        zero = self.pool.take_pending_zero()           # pages allocated since the last forward
        nz = len(zero)
        if nz:
            self._host_scratch(3 * nu + nz)[3 * nu:3 * nu + nz] = zero
        elif self._hs is None:
            self._host_scratch(1)
        plan_size = 6 * B + 2 + total
        d = self.static_plan_for(B, 1, plan_size)
        ctx.plan_static = d is not None
        if d is None:
            # one buffer reused by every forward: its readers are earlier launches on the
            # same stream
            if self._plan_dev is None or self._plan_dev.numel() < plan_size:
                grown = 2 * self._plan_dev.numel() if self._plan_dev is not None else 0
                self._plan_dev = torch.empty(max(plan_size, 65536, grown), dtype=torch.int32,
                                             device=self.cfg.device)
            d = self._plan_dev
        base = d.data_ptr()
        # plan views are sliced from d on first use (B200CacheContext.__getattr__); the
        # direct decode path takes these pointers
        ctx._plan_src = (d, B, 1, total)
        ctx._direct_ptrs = (base + 4 * B, base + 8 * B, base + 4 * (6 * B + 2),
                            base + 4 * (3 * B + 1))
        ctx._plan_bytes = 4 * (2 * B + 3 * nu + nz)
        lib, pk, pv, layers, pages, page_bytes, status, idx = self._plan_consts()
        stream = (ops._raw_stream(idx) if ops._raw_stream is not None
                  else torch.cuda.current_stream(idx).cuda_stream)
        dbt = self._dbt
        hp = self._hs_ptr
        rc = lib.nslg_plan_decode_host(B, ps, c.ptrs[0], c.ptrs[1], nu, hp, nz, hp + 12 * nu,
                                       pk, pv, layers, pages, page_bytes, dbt.data_ptr(),
                                       dbt.shape[1], dbt.shape[0], base, max(total, 1), status,
                                       stream)
        if rc:
            raise N.NativeError("nslg_plan_decode_host", rc, lib.nslg_last_error().decode())

    def allocate_sequence(self, seq_id, token_ids=None, num_tokens=0):
        self._mut += 1
        tids = token_ids or []
        total = len(tids) if tids else num_tokens
        plen, ppages = 0, []
        if self.tree and len(tids) >= self.cfg.page_size:
            plen, ppages = self.tree.match(tids)
            for p in ppages:
                self.pool.add_ref(p)
            if ppages:
                self.tree.add_refs(tids[:plen])
        st = _PagedSeqState(seq_id, ppages, plen, tids)
        st.num_tokens = plen
        new = total - plen
        if new > 0:
            st.block_table.extend(self._alloc(math.ceil(new / self.cfg.page_size)))
        self.seqs[seq_id] = st
        return plen

    def extend_sequence(self, seq_id, num_new=1):
        self._mut += 1
        st = self.seqs[seq_id]
        need = math.ceil((st.num_tokens + num_new) / self.cfg.page_size)
        if need > len(st.block_table):
            st.block_table.extend(self._alloc(need - len(st.block_table)))

    def begin_forward(self, seq_ids, ntoks, offsets=None):
        if (self.device_plan and 0 < len(seq_ids) <= 4096 and not any(offsets or ())
                and (ntoks.count(1) == len(ntoks) if isinstance(ntoks, list)
                     else all(n == 1 for n in ntoks))):
            c = self._dc
            if (c is not None and c.mut == self._mut and c.ver == _PagedSeqState.version
                    and c.ids == (seq_ids if type(seq_ids) is list else list(seq_ids))):
                ctx = self._begin_decode_cached(c, seq_ids, ntoks)
                if ctx is not None:
                    return ctx
            ctx = self._begin_decode_device(seq_ids, ntoks)
            if ctx is not None:
                return ctx
        self._mut += 1
        # extend_sequence for every sequence, inlined (sequences in order, so the page
        # allocation order is the reference's)
        sts = [self.seqs[s] for s in seq_ids]
        ps = self.cfg.page_size
        for st, n in zip(sts, ntoks):
            bt = st.block_table
            if st.num_tokens + n > len(bt) * ps:
                need = -(-(st.num_tokens + n) // ps)
                bt.extend(self._alloc(need - len(bt)))
        return B200CacheContext(self, seq_ids, ntoks, offsets, sts)

    def end_forward(self, ctx):
        c = getattr(ctx, "_dc", None)
        if c is not None and c is self._dc and c.open is ctx:
            # the open step of the cached decode batch: one token each, cache kept in
            # step (any other context, e.g. one ended twice, takes the general path,
            # which drops the cache)
            c.open = None
            for st in c.sts:
                st._n += 1
            c.n0 += 1
            c.t += 1
            c.total += len(c.buckets[c.t % self.cfg.page_size])
            return
        self._mut += 1
        for b in range(ctx.batch_size):
            st = self.seqs[ctx.seq_ids[b]]
            st._n += ctx.new_token_counts[b]

    def release_sequence(self, seq_id):
        if seq_id not in self.seqs:
            return
        self._mut += 1
        st = self.seqs[seq_id]
        if self.tree and st.token_ids:
            nf = st.num_tokens // self.cfg.page_size
            if nf:
                self.tree.insert(st.token_ids[:nf * self.cfg.page_size], st.block_table[:nf])
            if st.prefix_len:
                self.tree.dec_refs(st.token_ids[:st.prefix_len])
        for p in st.block_table:
            self.pool.release(p)
        if st.slot >= 0:
            self._slot_free.append(st.slot)
        del self.seqs[seq_id]

    def append_token_ids(self, seq_id, ids):
        if seq_id in self.seqs:
            self.seqs[seq_id].token_ids.extend(ids)

    def reset(self):
        for s in list(self.seqs):
            self.release_sequence(s)

    def _alloc(self, n):
        pages = self.pool.alloc(n)
        if pages:
            return pages
        if self.tree:
            if self.tree.evict_lru(n) > 0:
                pages = self.pool.alloc(n)
                if pages:
                    return pages
        raise RuntimeError(f"KV OOM: need {n}, free {self.pool.num_free}")

    @property
    def stats(self):
        return {"backend": "b200",
                "active_seqs": len(self.seqs),
                "pages_used": self.cfg.max_pages - 1 - self.pool.num_free,
                "pages_free": self.pool.num_free,
                "util": f"{self.pool.utilization:.1%}",
                "radix": self.tree.cached_pages if self.tree else 0}


def create_cache_manager(hf_config, parallel_config, device, dtype, model_config,
                         max_batch_size=4) -> KVCacheManager:
    """Factory with the reference's signature (kv_cache.py:780-804); always the B200
    paged backend."""
    dev = torch.device(device) if device is not None else None
    if dev is not None and dev.type == "cuda":
        torch.cuda.synchronize(dev)
        torch.cuda.empty_cache()
    kv_cfg = KVCacheConfig.from_hf_config(
        hf_config, parallel_config=parallel_config, device=device,
        page_size=getattr(model_config, "page_size", 16),
        max_pages=getattr(model_config, "max_kv_pages", 0),
        max_batch_size=max_batch_size,
        max_seq_len=getattr(model_config, "max_seq_len", 4096),
        memory_fraction=getattr(model_config, "kv_memory_fraction", 0.30),
        dtype=dtype,
        enable_prefix_caching=getattr(model_config, "enable_prefix_caching", True),
        backend=getattr(model_config, "kv_backend", "auto"),
    )
    return B200PagedKVCache(kv_cfg)
