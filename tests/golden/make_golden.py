"""Generate the golden fixtures in this directory from the NanoSLG reference itself.

Run in a container that has the reference checked out (read-only is fine):

    python tests/golden/make_golden.py --reference /path/to/nanoslg-checkout

It imports the reference's own Python (``nanoslg/kv_cache.py``, ``nanoslg/models.py``)
on CPU and records what it computes, so that the oracle restatement under ``oracle/``
and the CUDA path can be pinned to the reference without the reference being present:

* ``paged_scenarios.json``   -- page-pool / radix-tree / CSR-plan bookkeeping (hand-written
  scenarios and seeded random workloads) of
  ``FlashInferPagedKVCache`` + ``FlashInferCacheContext`` (kv_cache.py:382-777) with the
  two FlashInfer wrappers replaced by recorders (their ``plan`` arguments are the CSR
  arrays ``indptr / indices / last_page_len / qo_indptr``).
* ``attention_cases.pt``     -- ``ContiguousCacheContext.attend`` (kv_cache.py:247-325:
  KV write + ``_build_causal_mask`` + ``_sdpa``) on seeded q/k/v, decode and ragged
  prefill/extend, fp32 and bf16.
* ``rope_norm.pt``           -- ``precompute_rope_frequencies`` / ``apply_rotary_emb`` /
  ``RMSNorm`` (models.py:25-83) on seeded inputs.
* ``tiny_llama.json``        -- greedy tokens of the tiny fp32 Llama (2 layers, hidden 256,
  4/2 heads, vocab 1024) driven exactly like ``worker.py`` drives a TP=1 batch, on the
  contiguous-SDPA backend.
* ``tiny_llama_kv8.json``    -- the same for a batch of two prompts (32 and 19 tokens,
  left-padded prefill) on the tiny model widened to hidden 512 with 8 query / 8 KV heads,
  so that tensor-parallel degrees 1, 2, 4 and 8 all divide its heads
  (``--only-kv8`` writes this file alone).

The shims are the minimum needed to run on CPU: ``ParallelContext.device = cpu``,
backend ``contiguous`` (or ``flashinfer`` with the wrappers stubbed), and building the
managers directly instead of through ``create_cache_manager`` (kv_cache.py:780-782 calls
``torch.cuda.synchronize``).
"""
import argparse
import json
import os
import sys
from types import SimpleNamespace

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


# ----------------------------------------------------------------------------------------
# paged bookkeeping
# ----------------------------------------------------------------------------------------
class _Recorder:
    """Stands in for flashinfer.Batch{Decode,Prefill}WithPagedKVCacheWrapper: keeps the
    last plan() arguments (the CSR the reference would hand to FlashInfer)."""

    def __init__(self):
        self.last = None

    def plan(self, *args, **kw):
        self.last = ([a.tolist() if torch.is_tensor(a) else a for a in args], dict(kw))


def _make_paged(kvc, page_size, max_pages, prefix=True, num_layers=1, nkv=1, nq=1, hd=16):
    cfg = kvc.KVCacheConfig(num_layers=num_layers, num_kv_heads=nkv, num_qo_heads=nq,
                            head_dim=hd, page_size=page_size, max_pages=max_pages,
                            dtype=torch.float32, device=torch.device("cpu"),
                            enable_prefix_caching=prefix, backend="flashinfer")
    mgr = object.__new__(kvc.FlashInferPagedKVCache)
    mgr.cfg = cfg
    mgr.pool = kvc.PagePool(cfg)
    mgr.tree = kvc.RadixTree(cfg.page_size, mgr.pool) if prefix else None
    mgr.seqs = {}
    mgr._dec_wrap = _Recorder()
    mgr._pf_wrap = _Recorder()
    return mgr


def _snapshot(mgr):
    return {
        "block_tables": {s: list(st.block_table) for s, st in sorted(mgr.seqs.items())},
        "num_tokens": {s: st.num_tokens for s, st in sorted(mgr.seqs.items())},
        "num_free": mgr.pool.num_free,
        "ref_count": list(mgr.pool.ref_count),
        "tokens_used": list(mgr.pool.tokens_used),
        "stats": {k: v for k, v in mgr.stats.items() if k != "backend"},
    }


def run_paged_script(kvc, setup, ops):
    """Replays ``ops`` on a reference manager and returns one record per op."""
    mgr = _make_paged(kvc, **setup)
    records = []
    ctx = None
    for op in ops:
        kind = op[0]
        rec = {"op": op}
        try:
            if kind == "alloc":
                _, sid, toks, ntok = op
                rec["ret"] = mgr.allocate_sequence(sid, toks, ntok)
            elif kind == "extend":
                mgr.extend_sequence(op[1], op[2])
            elif kind == "begin":
                _, sids, counts, offsets = op
                mgr._dec_wrap.last = mgr._pf_wrap.last = None
                ctx = mgr.begin_forward(sids, counts, offsets)
                rec["write_info"] = [[list(x) for x in wi] for wi in ctx._write_info]
                rec["positions"] = ctx._pos.tolist()
                rec["start_positions"] = list(ctx.start_positions)
                rec["seq_lens"] = list(ctx.seq_lens)
                rec["is_decode"] = ctx._is_decode
                rec["indptr"] = ctx._fi_ind.tolist()
                rec["indices"] = ctx._fi_idx.tolist()
                rec["last_page_len"] = ctx._fi_lpl.tolist()
                if not ctx._is_decode:
                    rec["qo_indptr"] = ctx._fi_qo.tolist()
                wrap = mgr._dec_wrap if ctx._is_decode else mgr._pf_wrap
                rec["plan_args"] = wrap.last[0][:4] if wrap.last else None
            elif kind == "end":
                mgr.end_forward(ctx)
            elif kind == "release":
                mgr.release_sequence(op[1])
            elif kind == "append":
                mgr.append_token_ids(op[1], op[2])
            elif kind == "rewind":          # test hook: move a sequence's write cursor back
                mgr.seqs[op[1]].num_tokens = op[2]
            elif kind == "reset":
                mgr.reset()
            else:
                raise ValueError(kind)
        except RuntimeError as e:
            rec["error"] = str(e)
        rec["state"] = _snapshot(mgr)
        records.append(rec)
    return records


def paged_scenarios(kvc):
    g = torch.Generator().manual_seed(1234)

    def rt(n, hi=50):
        return torch.randint(0, hi, (n,), generator=g).tolist()

    scen = []
    # 1. the survey's hand example at page 4: 10 tokens -> 3 pages; re-match of 8 tokens.
    t10 = list(range(100, 110))
    scen.append({"name": "page4_basic", "setup": {"page_size": 4, "max_pages": 16},
                 "ops": [["alloc", "a", t10, 0], ["begin", ["a"], [10], [0]], ["end"],
                         ["release", "a"],
                         ["alloc", "b", t10[:8] + [7, 7], 0], ["begin", ["b"], [2], [0]],
                         ["end"], ["release", "b"]]})
    # 2. worker-style batches with radix hits, left padding and decode across pages.
    pre = rt(9)
    a_t, b_t, c_t = pre + rt(4), pre + rt(7), rt(5)
    ops = [["alloc", "a", a_t, 0], ["alloc", "b", b_t, 0], ["alloc", "c", c_t, 0],
           ["begin", ["a", "b", "c"], [13, 16, 5], [3, 0, 11]], ["end"]]
    for step in range(6):
        ops += [["begin", ["a", "b", "c"], [1, 1, 1], None], ["end"],
                ["append", "a", [step]], ["append", "b", [step + 1]], ["append", "c", [2]]]
    ops += [["release", "a"], ["release", "b"], ["release", "c"]]
    # second batch: d shares a's first 12 tokens (3 pages), e is a full-prompt hit of 8
    d_t, e_t = a_t[:12] + rt(6), b_t[:8]
    ops += [["alloc", "d", d_t, 0], ["alloc", "e", e_t, 0]]
    # worker clamps e's prefix to pl-1=7 but the state keeps num_tokens=8 (quirk)
    ops += [["begin", ["d", "e"], [6, 1], [0, 5]], ["end"]]
    for step in range(5):
        ops += [["begin", ["d", "e"], [1, 1], None], ["end"]]
    ops += [["release", "d"], ["release", "e"]]
    scen.append({"name": "radix_batches", "setup": {"page_size": 4, "max_pages": 40}, "ops": ops})
    # 3. copy-on-write of a shared page (reached by rewinding a sequence's cursor).
    s_t = rt(8)
    scen.append({"name": "cow", "setup": {"page_size": 4, "max_pages": 16},
                 "ops": [["alloc", "x", s_t, 0], ["begin", ["x"], [8], [0]], ["end"],
                         ["release", "x"], ["alloc", "y", s_t + [1, 2], 0],
                         ["rewind", "y", 6], ["begin", ["y"], [2], [0]], ["end"],
                         ["begin", ["y"], [1], None], ["end"], ["release", "y"]]})
    # 4. LRU eviction and OOM in a small pool.
    ops = []
    for i in range(4):
        t = rt(8, 1000)
        ops += [["alloc", f"p{i}", t, 0], ["begin", [f"p{i}"], [8], [0]], ["end"],
                ["release", f"p{i}"]]
    ops += [["alloc", "big", rt(20, 1000), 0], ["begin", ["big"], [20], [0]], ["end"],
            ["alloc", "huge", rt(40, 1000), 0], ["release", "big"]]
    scen.append({"name": "evict_oom", "setup": {"page_size": 4, "max_pages": 12}, "ops": ops})
    # 5. page 16, several worker batches, no prefix caching on a second manager.
    for prefix in (True, False):
        ops = []
        shared = rt(40, 1000)
        for bi in range(3):
            sids = [f"b{bi}s{j}" for j in range(4)]
            toks = [shared[:16 + 8 * j] + rt(5 + 7 * j + bi, 1000) for j in range(4)]
            for s, t in zip(sids, toks):
                ops.append(["alloc", s, t, 0])
            # counts/offsets are left for the replayer to derive from the alloc returns
            ops.append(["prefill_auto", sids])
            ops.append(["end"])
            for step in range(18):
                ops += [["begin", sids, [1] * 4, None], ["end"]]
                for s in sids:
                    ops.append(["append", s, [step]])
            for s in sids:
                ops.append(["release", s])
        scen.append({"name": f"page16_batches_prefix{int(prefix)}",
                     "setup": {"page_size": 16, "max_pages": 64, "prefix": prefix},
                     "ops": ops})
    # 6. continuous batching (drawn last, so the scenarios above keep their draws):
    # requests arrive while others decode, are prefilled as a batch of their own
    # (worker-style clamp and left padding), join the decode batch, and finish at random;
    # the pool is small enough that the tree evicts cached prefixes.
    for ps, pages in ((4, 72), (1, 200)):
        def ri(lo, hi):
            return int(torch.randint(lo, hi, (1,), generator=g))

        sysp = rt(3 * ps + 5, 1000)
        ops, running, nxt = [], [], 0
        for step in range(48):
            if step == 0 or (len(running) < 6 and ri(0, 4) == 0):
                new = []
                for _ in range(ri(1, 4)):
                    sid = f"r{nxt}"
                    nxt += 1
                    kind = ri(0, 3)
                    if kind == 0:      # the shared system prompt and a question
                        toks = sysp + rt(ri(1, 3 * ps + 2), 1000)
                    elif kind == 1:     # a prefix of the system prompt (a whole-prompt hit)
                        toks = sysp[:ri(1, len(sysp) + 1)]
                    else:
                        toks = rt(ri(2, 6 * ps + 3), 1000)
                    ops.append(["alloc", sid, toks, 0])
                    new.append(sid)
                ops += [["prefill_auto", new], ["end"]]
                running += new
            if step == 20 and running:
                ops.append(["extend", running[0], 2])
            ops += [["begin", list(running), [1] * len(running), None], ["end"]]
            for s in running:
                ops.append(["append", s, [ri(0, 1000)]])
            keep = []
            for s in running:
                if ri(0, 8) == 0:
                    ops.append(["release", s])
                else:
                    keep.append(s)
            running = keep
        for s in running:
            ops.append(["release", s])
        scen.append({"name": f"continuous_batching_page{ps}",
                     "setup": {"page_size": ps, "max_pages": pages}, "ops": ops})
    # 7. a batch whose second sequence must copy a shared page when no page is free: the
    # first sequence (a private page) has already marked its page when the copy fails.
    a_t, b_t, c_t = list(range(200, 208)), list(range(300, 305)), list(range(400, 408))
    scen.append({"name": "cow_out_of_pages", "setup": {"page_size": 4, "max_pages": 8},
                 "ops": [["alloc", "x", a_t, 0], ["begin", ["x"], [8], [0]], ["end"],
                         ["release", "x"],
                         ["alloc", "y", a_t + [1, 2], 0], ["begin", ["y"], [2], [0]], ["end"],
                         ["alloc", "z", b_t, 0], ["begin", ["z"], [5], [0]], ["end"],
                         ["alloc", "w", c_t, 0], ["begin", ["w"], [8], [0]], ["end"],
                         ["rewind", "y", 6], ["begin", ["z", "y"], [1, 1], None],
                         ["release", "y"], ["begin", ["z"], [1], None], ["end"]]})
    return scen


def random_workloads(kvc, seeds=range(12)):
    """Seeded random workloads over small pools (pages 1, 2, 4 and 16): requests with
    shared, repeated or fresh prompts arrive in batches, are prefilled (worker-style clamp
    and left padding), decode in whole or partial batches, sometimes extend by several
    tokens at once or with mixed counts, have their cursor moved back into shared pages,
    finish at random, and now and then the manager is reset. Operations that the
    reference cannot run (a sequence already gone) are dropped while the script is
    resolved against a shadow reference manager, so every recorded op is a valid call;
    out-of-pages errors are part of the record. Some scripts also end a context a second
    time after a begin that failed (the cached decode batch must not mistake that for
    its own step)."""
    import random
    out = []
    for seed in seeds:
        rng = random.Random(1000 + seed)
        ps = [1, 2, 4, 16][seed % 4]
        pages = rng.choice([10, 16, 24]) if ps > 1 else rng.choice([30, 48])
        ops, live, nxt, toks_of, finished = [], [], 0, {}, []
        shared = [rng.randrange(1000) for _ in range(rng.randrange(1, 4 * ps + 3))]
        for _ in range(rng.randrange(15, 40)):
            if rng.random() < 0.3 or not live:
                new = []
                for _ in range(rng.randrange(1, 4)):
                    sid = f"r{nxt}"
                    nxt += 1
                    k = rng.random()
                    if k < 0.3:
                        t = shared + [rng.randrange(1000) for _ in range(rng.randrange(0, 3 * ps))]
                    elif k < 0.45 and finished:
                        t = list(rng.choice(finished))
                        t = t[:rng.randrange(1, len(t) + 1)]
                    elif k < 0.55:
                        t = shared[:rng.randrange(1, len(shared) + 1)]
                    else:
                        t = [rng.randrange(1000) for _ in range(rng.randrange(1, 6 * ps + 3))]
                    ops.append(["alloc", sid, t or [1], 0])
                    new.append(sid)
                    toks_of[sid] = list(t or [1])
                ops += [["prefill_auto", new], ["end"]]
                live += new
            if rng.random() < 0.1 and live:
                ops.append(["extend", rng.choice(live), rng.randrange(1, 2 * ps + 2)])
            if rng.random() < 0.05 and live:
                ops.append(["rewind_rel", rng.choice(live), rng.randrange(1, 2 * ps + 1)])
            if rng.random() < 0.15 and live:
                sub = rng.sample(live, rng.randrange(1, len(live) + 1))
                cnt = [rng.randrange(1, 3 * ps + 2) for _ in sub]
                ops += [["begin", sub, cnt, [max(cnt) - c for c in cnt]], ["end"]]
            batch = list(live) if rng.random() < 0.7 else rng.sample(live, rng.randrange(1, len(live) + 1))
            ops += [["begin", batch, [1] * len(batch), None], ["end"]]
            for sid in batch:
                t = rng.randrange(1000)
                ops.append(["append", sid, [t]])
                toks_of[sid].append(t)
            keep = []
            for sid in live:
                if rng.random() < 0.12:
                    ops.append(["release", sid])
                    finished.append(toks_of[sid])
                else:
                    keep.append(sid)
            live = keep
            if rng.random() < 0.02:
                ops.append(["reset"])
                live = []
        ops += [["release", sid] for sid in live]
        setup = {"page_size": ps, "max_pages": pages}
        out.append({"name": f"random_{seed}_page{ps}", "setup": setup,
                    "ops": _resolve_random(kvc, setup, ops, stale_end=seed % 3 == 2)})
    return out


def _resolve_random(kvc, setup, ops, stale_end):
    """Turns a random script into valid reference calls (see random_workloads)."""
    mgr = _make_paged(kvc, **setup)
    out, rets, ctx, begin_ok = [], {}, None, False
    for op in ops:
        k = op[0]
        if k == "prefill_auto":
            sids = [s for s in op[1] if s in mgr.seqs]
            if not sids:
                continue
            counts = []
            for s in sids:
                pl = len(mgr.seqs[s].token_ids)
                counts.append(pl - (min(rets[s], pl - 1) if pl > 1 else 0))
            op = ["begin", sids, counts, [max(counts) - c for c in counts]]
        elif k == "rewind_rel":
            if op[1] not in mgr.seqs:
                continue
            op = ["rewind", op[1], max(mgr.seqs[op[1]].num_tokens - op[2], 0)]
        elif k == "begin":
            keep = [(s, c, o) for s, c, o in zip(op[1], op[2], op[3] or [0] * len(op[1]))
                    if s in mgr.seqs]
            if not keep:
                continue
            if all(c == 1 for _, c, _ in keep):
                op = ["begin", [s for s, _, _ in keep], [1] * len(keep), None]
            else:
                mx = max(c for _, c, _ in keep)
                op = ["begin", [s for s, _, _ in keep], [c for _, c, _ in keep],
                      [mx - c for _, c, _ in keep]]
        elif k in ("extend", "append", "release") and op[1] not in mgr.seqs:
            continue
        elif k == "end":
            if not out or out[-1][0] != "begin" or (not begin_ok and not stale_end):
                continue
            if any(s not in mgr.seqs for s in ctx.seq_ids):
                continue
        k = op[0]
        try:
            if k == "alloc":
                rets[op[1]] = mgr.allocate_sequence(op[1], op[2], op[3])
            elif k == "begin":
                begin_ok = False
                ctx = mgr.begin_forward(op[1], op[2], op[3])
                begin_ok = True
            elif k == "end":
                mgr.end_forward(ctx)
            elif k == "release":
                mgr.release_sequence(op[1])
            elif k == "append":
                mgr.append_token_ids(op[1], op[2])
            elif k == "rewind":
                mgr.seqs[op[1]].num_tokens = op[2]
            elif k == "extend":
                mgr.extend_sequence(op[1], op[2])
            elif k == "reset":
                mgr.reset()
        except RuntimeError:
            pass
        out.append(op)
    return out


def expand_prefill_auto(kvc, scen):
    """``prefill_auto`` mirrors worker.py:169-213: per sequence the prefix returned by
    allocate_sequence is clamped to pl-1 and the batch is left-padded.  The generator
    resolves it to a plain ``begin`` op with the counts and offsets the worker computes."""
    mgr = _make_paged(kvc, **scen["setup"])
    out, rets = [], {}
    for op in scen["ops"]:
        if op[0] == "prefill_auto":
            sids = op[1]
            counts = []
            for s in sids:
                pl = len(mgr.seqs[s].token_ids)
                plen = min(rets[s], pl - 1) if pl > 1 else 0
                counts.append(pl - plen)
            mx = max(counts)
            op = ["begin", sids, counts, [mx - c for c in counts]]
        out.append(op)
        # advance the shadow manager so that later prefix matches are right
        k = op[0]
        try:
            if k == "alloc":
                rets[op[1]] = mgr.allocate_sequence(op[1], op[2], op[3])
            elif k == "begin":
                ctx = mgr.begin_forward(op[1], op[2], op[3])
            elif k == "end":
                mgr.end_forward(ctx)
            elif k == "release":
                mgr.release_sequence(op[1])
            elif k == "append":
                mgr.append_token_ids(op[1], op[2])
            elif k == "rewind":
                mgr.seqs[op[1]].num_tokens = op[2]
        except RuntimeError:
            pass
    return out


# ----------------------------------------------------------------------------------------
# contiguous SDPA attention
# ----------------------------------------------------------------------------------------
def attention_cases(kvc):
    cases = []
    specs = [
        # name, dtype, Hq, Hkv, D, prefill lens, decode steps, extend chunk
        ("f32_gqa2", torch.float32, 4, 2, 64, [5, 17, 33], 3, 0),
        ("bf16_gqa4", torch.bfloat16, 8, 2, 128, [1, 12, 29, 40], 2, 0),
        ("bf16_extend", torch.bfloat16, 8, 2, 128, [7, 20], 1, 5),
        ("f32_single", torch.float32, 4, 2, 64, [24], 2, 0),
        ("bf16_mha", torch.bfloat16, 4, 4, 64, [3, 9], 2, 0),
    ]
    g = torch.Generator().manual_seed(7)
    for name, dt, hq, hkv, d, lens, ndec, ext in specs:
        B = len(lens)
        cfg = kvc.KVCacheConfig(num_layers=2, num_kv_heads=hkv, num_qo_heads=hq,
                                head_dim=d, max_batch_size=B, max_seq_len=128,
                                dtype=dt, device=torch.device("cpu"), backend="contiguous")
        mgr = kvc.ContiguousKVCache(cfg)
        sids = [f"s{i}" for i in range(B)]
        for s in sids:
            mgr.allocate_sequence(s)
        steps = []
        # prefill (ragged, left padded), then optional extend chunk, then decode steps
        plan = [("prefill", list(lens))]
        if ext:
            plan.append(("prefill", [ext] * B))
        plan += [("decode", [1] * B)] * ndec
        for kind, counts in plan:
            mx = max(counts)
            offs = [mx - c for c in counts]
            ctx = mgr.begin_forward(sids, counts, offs)
            S = mx
            rec = {"kind": kind, "counts": counts, "offsets": offs,
                   "start_positions": list(ctx.start_positions), "layers": []}
            for layer in range(2):
                q = torch.randn(B, S, hq, d, generator=g).to(dt)
                k = torch.randn(B, S, hkv, d, generator=g).to(dt)
                v = torch.randn(B, S, hkv, d, generator=g).to(dt)
                out = ctx.attend(layer, q, k, v, hq, hkv)
                rec["layers"].append({"q": q, "k": k, "v": v, "out": out})
            rec["positions"] = ctx.get_position_ids(S).clone()
            mgr.end_forward(ctx)
            steps.append(rec)
        cases.append({"name": name, "dtype": str(dt), "hq": hq, "hkv": hkv, "d": d,
                      "lens": lens, "steps": steps})
    return cases


# ----------------------------------------------------------------------------------------
# RoPE / RMSNorm
# ----------------------------------------------------------------------------------------
def rope_norm_cases(M):
    g = torch.Generator().manual_seed(11)
    out = {}
    cfg_plain = SimpleNamespace()
    cfg_l3 = SimpleNamespace(rope_scaling={"rope_type": "llama3", "factor": 8.0,
                                           "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                                           "original_max_position_embeddings": 8192})
    for key, d, mx, th, c in [("t64_1e4", 64, 128, 10000.0, cfg_plain),
                              ("t128_5e5", 128, 4096, 500000.0, cfg_plain),
                              ("t128_l3", 128, 4096, 500000.0, cfg_l3)]:
        cos, sin = M.precompute_rope_frequencies(d, mx, th, c)
        rows = torch.cat([torch.arange(16), torch.randint(16, mx, (48,), generator=g)])
        out[f"table_{key}"] = {"rows": rows, "cos": cos[rows].clone(), "sin": sin[rows].clone(),
                               "dim": d, "max": mx, "theta": th, "llama3": c is cfg_l3}
        if key == "t128_5e5":
            full_cos, full_sin = cos, sin
    cos, sin = full_cos, full_sin
    for dt in (torch.float32, torch.bfloat16):
        x = torch.randn(3, 5, 4, 128, generator=g).to(dt)
        pos = torch.randint(0, 4096, (3, 5), generator=g)
        y = M.apply_rotary_emb(x, cos[pos], sin[pos])
        out[f"rope_{str(dt)[6:]}"] = {"x": x, "pos": pos, "y": y}
        h = 256
        xs = (torch.randn(7, h, generator=g) * 3).to(dt)
        w = (1 + 0.1 * torch.randn(h, generator=g)).to(dt)
        norm = M.RMSNorm(h, eps=1e-5).to(dt)
        norm.weight.data.copy_(w)
        with torch.no_grad():
            out[f"rmsnorm_{str(dt)[6:]}"] = {"x": xs, "w": w, "eps": 1e-5, "y": norm(xs)}
            r = torch.randn(7, h, generator=g).to(dt)
            hsum = xs + r
            out[f"addnorm_{str(dt)[6:]}"] = {"x": xs, "r": r, "w": w, "eps": 1e-5,
                                             "h": hsum, "y": norm(hsum)}
    return out


def fp16_cases(kvc, M):
    """float16 activations (worker.py:22-26 allows them): the contiguous path's attention
    (its mask fills with -65504 in fp16, kv_cache.py:208), RoPE and RMSNorm, recorded the
    same way as the bf16 cases."""
    g = torch.Generator().manual_seed(13)
    out = {"attention": []}
    specs = [("f16_gqa4", 8, 2, 128, [1, 12, 29, 40], 2, 0),
             ("f16_extend", 8, 2, 128, [7, 20], 1, 5),
             ("f16_gqa4_d64", 8, 2, 64, [3, 17], 2, 0)]
    dt = torch.float16
    for name, hq, hkv, d, lens, ndec, ext in specs:
        B = len(lens)
        cfg = kvc.KVCacheConfig(num_layers=2, num_kv_heads=hkv, num_qo_heads=hq,
                                head_dim=d, max_batch_size=B, max_seq_len=128,
                                dtype=dt, device=torch.device("cpu"), backend="contiguous")
        mgr = kvc.ContiguousKVCache(cfg)
        sids = [f"s{i}" for i in range(B)]
        for s in sids:
            mgr.allocate_sequence(s)
        steps = []
        plan = [("prefill", list(lens))]
        if ext:
            plan.append(("prefill", [ext] * B))
        plan += [("decode", [1] * B)] * ndec
        for kind, counts in plan:
            mx = max(counts)
            offs = [mx - c for c in counts]
            ctx = mgr.begin_forward(sids, counts, offs)
            rec = {"kind": kind, "counts": counts, "offsets": offs,
                   "start_positions": list(ctx.start_positions), "layers": []}
            for layer in range(2):
                q = torch.randn(B, mx, hq, d, generator=g).to(dt)
                k = torch.randn(B, mx, hkv, d, generator=g).to(dt)
                v = torch.randn(B, mx, hkv, d, generator=g).to(dt)
                o = ctx.attend(layer, q, k, v, hq, hkv)
                rec["layers"].append({"q": q, "k": k, "v": v, "out": o})
            rec["positions"] = ctx.get_position_ids(mx).clone()
            mgr.end_forward(ctx)
            steps.append(rec)
        out["attention"].append({"name": name, "dtype": str(dt), "hq": hq, "hkv": hkv, "d": d,
                                 "lens": lens, "steps": steps})
    cos, sin = M.precompute_rope_frequencies(128, 4096, 500000.0, SimpleNamespace())
    x = torch.randn(3, 5, 4, 128, generator=g).to(dt)
    pos = torch.randint(0, 4096, (3, 5), generator=g)
    out["rope"] = {"x": x, "pos": pos, "y": M.apply_rotary_emb(x, cos[pos], sin[pos])}
    h = 256
    xs = (torch.randn(7, h, generator=g) * 3).to(dt)
    w = (1 + 0.1 * torch.randn(h, generator=g)).to(dt)
    norm = M.RMSNorm(h, eps=1e-5).to(dt)
    norm.weight.data.copy_(w)
    with torch.no_grad():
        out["rmsnorm"] = {"x": xs, "w": w, "eps": 1e-5, "y": norm(xs)}
        r = torch.randn(7, h, generator=g).to(dt)
        hsum = xs + r
        out["addnorm"] = {"x": xs, "r": r, "w": w, "eps": 1e-5, "h": hsum, "y": norm(hsum)}
    return out


# ----------------------------------------------------------------------------------------
# tiny Llama (config C1)
# ----------------------------------------------------------------------------------------
TINY = dict(num_hidden_layers=2, hidden_size=256, num_attention_heads=4,
            num_key_value_heads=2, intermediate_size=512, vocab_size=1024,
            rms_norm_eps=1e-5, rope_theta=10000.0, max_position_embeddings=128)


def tiny_llama(kvc, M, ParallelContext, ParallelConfig, ParallelMode):
    pctx = ParallelContext.initialize(ParallelConfig(ParallelMode.TENSOR, 1), 0)
    pctx.device = torch.device("cpu")
    hf = SimpleNamespace(**TINY)
    model = M.create_model(hf, pctx.config).float()
    torch.manual_seed(0)
    names = []
    with torch.no_grad():
        for n, p in model.named_parameters():
            names.append(n)
            if "norm" in n:
                continue
            p.normal_(0.0, 0.02)
    prompt = torch.randint(0, 1024, (1, 32), generator=torch.Generator().manual_seed(1))
    cfg = kvc.KVCacheConfig(num_layers=2, num_kv_heads=2, num_qo_heads=4, head_dim=64,
                            max_batch_size=1, max_seq_len=64, dtype=torch.float32,
                            device=torch.device("cpu"), backend="contiguous")
    mgr = kvc.ContiguousKVCache(cfg)
    toks, margins = [], []
    with torch.inference_mode():
        mgr.allocate_sequence("s0", prompt[0].tolist())
        ctx = mgr.begin_forward(["s0"], [32], [0])
        logits = model(prompt, ctx, None)
        mgr.end_forward(ctx)
        first_logits = logits[0, -1].clone()
        for step in range(16):
            last = logits[0, -1]
            top2 = torch.topk(last, 2).values
            margins.append(float(top2[0] - top2[1]))
            t = int(last.argmax())
            toks.append(t)
            if step == 15:
                break
            ctx = mgr.begin_forward(["s0"], [1])
            logits = model(torch.tensor([[t]]), ctx, None)
            mgr.end_forward(ctx)
    return {"config": TINY, "init": "torch.manual_seed(0); normal_(0, 0.02) over "
            "named_parameters() in order, skipping *norm* weights (kept at 1)",
            "param_order": names, "prompt": prompt[0].tolist(), "tokens": toks,
            "min_margin": min(margins), "first_logits_head": first_logits[:16].tolist()}


# The tiny model widened to 8 query and 8 KV heads, so that every tensor-parallel degree
# of one 8-GPU node (1, 2, 4, 8) divides its heads; two prompts of different lengths.
TINY_KV8 = dict(num_hidden_layers=2, hidden_size=512, num_attention_heads=8,
                num_key_value_heads=8, intermediate_size=1024, vocab_size=1024,
                rms_norm_eps=1e-5, rope_theta=10000.0, max_position_embeddings=128)


def tiny_llama_batch(kvc, M, ParallelContext, ParallelConfig, ParallelMode, cfg=TINY_KV8,
                     prompt_lens=(32, 19), steps=16):
    """Greedy tokens of a batch driven like worker.py:365-426 drives one TP batch: one
    left-padded prefill forward (input_offsets = width - count, worker.py:375-378), then
    decode steps of the whole batch (worker.py:398-412), on the contiguous-SDPA backend."""
    pctx = ParallelContext.initialize(ParallelConfig(ParallelMode.TENSOR, 1), 0)
    pctx.device = torch.device("cpu")
    hf = SimpleNamespace(**cfg)
    model = M.create_model(hf, pctx.config).float()
    torch.manual_seed(0)
    names = []
    with torch.no_grad():
        for n, p in model.named_parameters():
            names.append(n)
            if "norm" in n:
                continue
            p.normal_(0.0, 0.02)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg["vocab_size"], (n,), generator=g).tolist()
               for n in prompt_lens]
    B = len(prompts)
    nq, nkv = cfg["num_attention_heads"], cfg["num_key_value_heads"]
    kcfg = kvc.KVCacheConfig(num_layers=cfg["num_hidden_layers"], num_kv_heads=nkv,
                             num_qo_heads=nq, head_dim=cfg["hidden_size"] // nq,
                             max_batch_size=B, max_seq_len=max(prompt_lens) + steps + 8,
                             dtype=torch.float32, device=torch.device("cpu"),
                             backend="contiguous")
    mgr = kvc.ContiguousKVCache(kcfg)
    sids = [f"s{i}" for i in range(B)]
    width = max(prompt_lens)
    ids = torch.zeros(B, width, dtype=torch.long)
    for i, p in enumerate(prompts):
        ids[i, width - len(p):] = torch.tensor(p)
    toks = [[] for _ in range(B)]
    margins = []
    with torch.inference_mode():
        for sid, p in zip(sids, prompts):
            mgr.allocate_sequence(sid, p)
        ctx = mgr.begin_forward(sids, [len(p) for p in prompts],
                                [width - len(p) for p in prompts])
        logits = model(ids, ctx, None)
        mgr.end_forward(ctx)
        for step in range(steps):
            last = logits[:, -1]
            top2 = torch.topk(last, 2, dim=-1).values
            margins.append(float((top2[:, 0] - top2[:, 1]).min()))
            t = last.argmax(-1)
            for i in range(B):
                toks[i].append(int(t[i]))
            if step + 1 == steps:
                break
            ctx = mgr.begin_forward(sids, [1] * B)
            logits = model(t[:, None], ctx, None)
            mgr.end_forward(ctx)
    return {"config": cfg, "init": "torch.manual_seed(0); normal_(0, 0.02) over "
            "named_parameters() in order, skipping *norm* weights (kept at 1)",
            "param_order": names, "prompts": prompts, "tokens": toks,
            "min_margin": min(margins)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of Guney-olu/nanoslg")
    ap.add_argument("--only-paged", action="store_true",
                    help="write paged_scenarios.json only")
    ap.add_argument("--only-kv8", action="store_true",
                    help="write tiny_llama_kv8.json only")
    ap.add_argument("--only-fp16", action="store_true",
                    help="write fp16_cases.pt only")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import nanoslg.kv_cache as kvc
    import nanoslg.models as M
    from nanoslg.parallel import ParallelContext, ParallelConfig, ParallelMode

    torch.set_num_threads(1)
    if args.only_fp16:
        torch.save(fp16_cases(kvc, M), os.path.join(HERE, "fp16_cases.pt"))
        return
    if args.only_kv8:
        tb = tiny_llama_batch(kvc, M, ParallelContext, ParallelConfig, ParallelMode)
        with open(os.path.join(HERE, "tiny_llama_kv8.json"), "w") as f:
            json.dump(tb, f, indent=1)
        print("tiny llama (8 kv heads, batch 2) tokens:", tb["tokens"], "min margin",
              tb["min_margin"])
        return
    scen = paged_scenarios(kvc)
    for s in scen:
        s["ops"] = expand_prefill_auto(kvc, s)
    scen += random_workloads(kvc)
    for s in scen:
        s["records"] = run_paged_script(kvc, s["setup"], s["ops"])
    with open(os.path.join(HERE, "paged_scenarios.json"), "w") as f:
        json.dump(scen, f)
    if args.only_paged:
        return
    torch.save(attention_cases(kvc), os.path.join(HERE, "attention_cases.pt"))
    torch.save(rope_norm_cases(M), os.path.join(HERE, "rope_norm.pt"))
    torch.save(fp16_cases(kvc, M), os.path.join(HERE, "fp16_cases.pt"))
    tl = tiny_llama(kvc, M, ParallelContext, ParallelConfig, ParallelMode)
    with open(os.path.join(HERE, "tiny_llama.json"), "w") as f:
        json.dump(tl, f, indent=1)
    print("tiny llama tokens:", tl["tokens"], "min margin", tl["min_margin"])
    tb = tiny_llama_batch(kvc, M, ParallelContext, ParallelConfig, ParallelMode)
    with open(os.path.join(HERE, "tiny_llama_kv8.json"), "w") as f:
        json.dump(tb, f, indent=1)
    print("tiny llama (8 kv heads, batch 2) tokens:", tb["tokens"], "min margin",
          tb["min_margin"])


if __name__ == "__main__":
    main()
