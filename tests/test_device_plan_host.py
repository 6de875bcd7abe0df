"""Host side of the device-planned decode step, on CPU.

The manager of a CUDA pool plans decode steps on the GPU (csrc/plan.cu,
nslg_plan_decode_host) from block tables mirrored in device memory: per step it sends the
batch's table rows, the token counts before the step and the table entries changed since
the last step. When the same batch steps again with nothing else changed, a cached copy
of the batch's state is advanced instead of walking every sequence. Here the launch is
replaced by a recorder that applies the uploads to a numpy mirror of the device tables,
and three managers run
the same random workload: device planning with the cache, device planning without it,
and the host plan (kv_cache.py:547-632 restated). Page ids, block tables, refcounts,
tokens_used, write targets and the mirrored tables must agree at every step."""
import random

import numpy as np
import pytest
import torch

from nanoslg_b200.kv_cache import B200PagedKVCache, KVCacheConfig


class _Mirror:
    """Stands in for the nslg_plan_decode_host launch: applies the table updates, records
    the step."""

    def __init__(self, mgr):
        self.mgr = mgr
        self.rows = {}
        self.last = None

    def __call__(self, ctx, c, nu):
        if nu:
            for s, j, pg in self.mgr._hs[:3 * nu].reshape(nu, 3).tolist():
                self.rows.setdefault(s, {})[j] = pg
        self.mgr.pool.take_pending_zero()
        ps = self.mgr.cfg.page_size
        # the page-id count kept by the batch is the one the plan is sized with
        assert c.total == int(((c.n0.astype(np.int64) + ps) // ps).sum())
        self.last = (c.slots.tolist(), c.n0.tolist())
        ctx.plan_static = False


def _managers(page_size, max_pages):
    out = []
    for mode in ("cached", "uncached", "host"):
        cfg = KVCacheConfig(num_layers=1, num_kv_heads=1, num_qo_heads=1, head_dim=16,
                            page_size=page_size, max_pages=max_pages, dtype=torch.float32,
                            device=torch.device("cpu"), enable_prefix_caching=True)
        m = B200PagedKVCache(cfg)
        m.device_plan = mode != "host"
        m._mode = mode
        if m.device_plan:
            m._mirror = _Mirror(m)
            m._launch_device_plan = m._mirror
        out.append(m)
    return out


@pytest.mark.parametrize("page_size", [1, 4, 16])
def test_cached_decode_batches_match_host_plan(page_size):
    mgrs = _managers(page_size, 6000)
    rng = random.Random(11 + page_size)
    shared = [rng.randrange(1000) for _ in range(3 * page_size)]
    live, nxt = [], 0
    hits = {"cached": 0}

    def add(n_new):
        nonlocal nxt
        for _ in range(n_new):
            sid = f"q{nxt}"
            nxt += 1
            r = rng.random()
            if r < 0.15:
                # the whole prompt matched in the tree and the last tokens recomputed: the
                # pages to write are shared, copy on write on the host path
                toks, back = list(shared), rng.randrange(1, 2 * page_size + 1)
            elif r < 0.4:
                toks, back = shared + [rng.randrange(1000) for _ in range(rng.randrange(1, 40))], 0
            else:
                toks, back = [rng.randrange(1000) for _ in range(rng.randrange(1, 120))], 0
            for m in mgrs:
                m.allocate_sequence(sid, toks)
                m.seqs[sid].num_tokens = max(len(toks) - back, 0)
            live.append(sid)

    def drop(k):
        for _ in range(k):
            sid = live.pop(rng.randrange(len(live)))
            for m in mgrs:
                m.append_token_ids(sid, [1, 2, 3])
                m.release_sequence(sid)

    add(20)
    for step in range(80):
        if step in (20, 50):
            drop(6)
            add(8)
        if step == 35:                      # another bookkeeping call drops the cache
            for m in mgrs:
                m.extend_sequence(live[0], 1)
        if step == 65:                      # so does a direct token-count change
            for m in mgrs:
                m.seqs[live[1]].num_tokens += 0
        ctxs = []
        for m in mgrs:
            if m._mode == "uncached":
                m._dc = None
            was = m._dc
            c = m.begin_forward(list(live), [1] * len(live))
            if m._mode == "cached" and was is not None and getattr(c, "_dc", None) is was:
                hits["cached"] += 1
            ctxs.append(c)
        host = ctxs[2]
        for m, c in zip(mgrs, ctxs):
            assert c.start_positions == host.start_positions, (step, m._mode)
            assert c._write_info == host._write_info, (step, m._mode)
        for m in mgrs[1:]:
            assert {s: list(st.block_table) for s, st in m.seqs.items()} == \
                   {s: list(st.block_table) for s, st in mgrs[0].seqs.items()}, step
            assert m.pool.ref_count == mgrs[0].pool.ref_count, step
            assert list(m.pool.tokens_used) == list(mgrs[0].pool.tokens_used), step
        for m, c in zip(mgrs[:2], ctxs[:2]):
            if getattr(c, "_dc", None) is None:
                continue                    # the host path took this step
            slots, starts = m._mirror.last
            assert starts == host.start_positions
            for sid, slot, n0 in zip(live, slots, starts):
                row = m._mirror.rows.get(slot, {})
                bt = list(m.seqs[sid].block_table)
                npg = n0 // page_size + 1
                assert [row.get(j) for j in range(npg)] == bt[:npg], (step, sid, m._mode)
        for m, c in zip(mgrs, ctxs):
            m.end_forward(c)
        for m in mgrs[1:]:
            assert {s: st.num_tokens for s, st in m.seqs.items()} == \
                   {s: st.num_tokens for s, st in mgrs[0].seqs.items()}
    assert hits["cached"] > 40


def test_device_planned_context_builds_its_lists_lazily():
    """A device-planned decode context keeps its start positions as an array and builds
    start_positions / seq_lens / max_kv_len (and the plan views) on first use; unknown
    attributes still raise AttributeError."""
    m = _managers(16, 512)[0]
    for sid, n in (("a", 40), ("b", 16), ("c", 3)):
        m.allocate_sequence(sid, None, num_tokens=n)
        m.seqs[sid].num_tokens = n
    ctx = m.begin_forward(["a", "b", "c"], [1, 1, 1])
    assert "start_positions" not in ctx.__dict__
    assert ctx.get_start_pos(1) == 16
    assert ctx.start_positions == [40, 16, 3]
    assert ctx.seq_lens == [41, 17, 4] and ctx.max_kv_len == 41
    assert not hasattr(ctx, "no_such_attribute")
    m.end_forward(ctx)
    ctx2 = m.begin_forward(["a", "b", "c"], [1, 1, 1])       # the cached batch
    assert ctx2.start_positions == [41, 17, 4]
    assert ctx.start_positions == [40, 16, 3]                # the old context is unchanged
    m.end_forward(ctx2)


def _golden_scenarios():
    import json
    import os
    from conftest import GOLDEN
    with open(os.path.join(GOLDEN, "paged_scenarios.json")) as f:
        return json.load(f)


_SCEN = _golden_scenarios()


@pytest.mark.parametrize("sc", _SCEN, ids=[s["name"] for s in _SCEN])
def test_device_planned_manager_replays_reference_scenarios(sc):
    """Every golden scenario (recorded from the reference's FlashInferPagedKVCache) replayed
    on a device-planning manager: the state after each op is the reference's, and on the
    decode steps the device plans, the CSR and write targets that follow from what was
    sent (the mirrored table rows and the start positions) are the reference's."""
    from oracle import paged_plan
    setup = dict(sc["setup"])
    ps = setup["page_size"]
    cfg = KVCacheConfig(num_layers=1, num_kv_heads=1, num_qo_heads=1, head_dim=16,
                        page_size=ps, max_pages=setup["max_pages"], dtype=torch.float32,
                        device=torch.device("cpu"),
                        enable_prefix_caching=setup.get("prefix", True))
    m = B200PagedKVCache(cfg)
    m.device_plan = True
    m._mirror = _Mirror(m)
    m._launch_device_plan = m._mirror
    ctx, device_steps = None, 0
    for i, rec in enumerate(sc["records"]):
        op = rec["op"]
        kind = op[0]
        err = None
        try:
            if kind == "alloc":
                assert m.allocate_sequence(op[1], op[2], op[3]) == rec["ret"], i
            elif kind == "extend":
                m.extend_sequence(op[1], op[2])
            elif kind == "begin":
                ctx = m.begin_forward(op[1], op[2], op[3])
                assert ctx.start_positions == rec["start_positions"], i
                assert ctx.seq_lens == rec["seq_lens"], i
                assert ctx._is_decode == rec["is_decode"], i
                if getattr(ctx, "_dc", None) is not None:
                    device_steps += 1
                    slots, starts = m._mirror.last
                    assert starts == rec["start_positions"], i
                    tables = []
                    for slot, n0 in zip(slots, starts):
                        row = m._mirror.rows.get(slot, {})
                        tables.append([row.get(j) for j in range(n0 // ps + 1)])
                    ind, idx, lpl = paged_plan.csr(tables, rec["seq_lens"], ps)
                    assert (ind, idx, lpl) == (rec["indptr"], rec["indices"],
                                               rec["last_page_len"]), i
                    wi = paged_plan.write_targets(tables, starts, [1] * len(starts), ps)
                    assert [[list(x) for x in w] for w in wi] == rec["write_info"], i
                else:
                    assert [[list(x) for x in w] for w in ctx._write_info] == \
                        rec["write_info"], i
                    assert ctx.kv_indptr.tolist() == rec["indptr"], i
                    assert ctx.kv_indices.tolist() == rec["indices"], i
                    assert ctx.kv_last_page_len.tolist() == rec["last_page_len"], i
            elif kind == "end":
                m.end_forward(ctx)
            elif kind == "release":
                m.release_sequence(op[1])
            elif kind == "append":
                m.append_token_ids(op[1], op[2])
            elif kind == "rewind":
                m.seqs[op[1]].num_tokens = op[2]
            elif kind == "reset":
                m.reset()
        except RuntimeError as e:
            err = str(e)
        assert (err is None) == ("error" not in rec), (i, err)
        st = rec["state"]
        assert {s: list(x.block_table) for s, x in sorted(m.seqs.items())} == \
            st["block_tables"], i
        assert {s: x.num_tokens for s, x in sorted(m.seqs.items())} == st["num_tokens"], i
        assert m.pool.num_free == st["num_free"], i
        assert list(m.pool.ref_count) == st["ref_count"], i
        assert list(m.pool.tokens_used) == st["tokens_used"], i
    n_dec = sum(1 for r in sc["records"] if r["op"][0] == "begin" and r.get("is_decode"))
    assert n_dec == 0 or device_steps > 0


def test_context_ended_twice_drops_the_cached_batch():
    """Ending a decode context a second time (after the next begin ran out of pages)
    advances the token counts like the reference's end_forward does; the cached batch
    must not take that step for its own, or the next begin would skip the page the
    reference allocates (and fails to allocate) there."""
    mgrs = _managers(4, 3)                 # pages 1 and 2 only
    outcomes = []
    for m in mgrs:
        m.allocate_sequence("a", [1, 2, 3])
        m.allocate_sequence("b", [4, 5, 6, 7])
        m.end_forward(m.begin_forward(["a", "b"], [3, 4], [1, 0]))
        ctx1 = m.begin_forward(["a"], [1])           # position 3: page 1 still has room
        m.end_forward(ctx1)
        with pytest.raises(RuntimeError, match="KV OOM"):
            m.begin_forward(["a"], [1])              # position 4 needs a page: none left
        m.end_forward(ctx1)                          # the old context once more
        assert m.seqs["a"].num_tokens == 5
        try:
            m.begin_forward(["a"], [1])
            outcomes.append("ok")
        except RuntimeError as e:
            outcomes.append(str(e))
    assert outcomes[0] == outcomes[2] and outcomes[1] == outcomes[2], outcomes
    assert outcomes[2].startswith("KV OOM")


def test_block_table_mirror_follows_every_list_operation():
    """The int32 mirror of a block table equals the list after any list operation, and
    the entries marked for upload cover every entry that changed."""
    from nanoslg_b200.kv_cache import _BlockTable
    rng = random.Random(5)
    bt = _BlockTable([3, 1, 4])
    shadow = [3, 1, 4]
    uploaded = list(shadow)          # what the device copy holds

    def upload():
        nonlocal uploaded
        d = bt.dirty_from
        uploaded = uploaded[:d] + list(bt)[d:]
        bt.dirty_from = len(bt)

    upload()
    for step in range(400):
        op = rng.randrange(12)
        if op == 0:
            x = [rng.randrange(100) for _ in range(rng.randrange(0, 40))]
            bt.extend(x); shadow.extend(x)
        elif op == 1:
            x = rng.randrange(100)
            bt.append(x); shadow.append(x)
        elif op == 2 and shadow:
            i = rng.randrange(-len(shadow), len(shadow)); x = rng.randrange(100)
            bt[i] = x; shadow[i] = x
        elif op == 3 and shadow:
            i = rng.randrange(len(shadow)); j = rng.randrange(i, len(shadow) + 1)
            x = [rng.randrange(100) for _ in range(rng.randrange(0, 5))]
            bt[i:j] = x; shadow[i:j] = x
        elif op == 4:
            x = [rng.randrange(100) for _ in range(rng.randrange(0, 5))]
            bt += x; shadow += x
        elif op == 5 and shadow:
            i = rng.randrange(len(shadow))
            assert bt.pop(i) == shadow.pop(i)
        elif op == 6:
            i = rng.randrange(len(shadow) + 1); x = rng.randrange(100)
            bt.insert(i, x); shadow.insert(i, x)
        elif op == 7 and shadow:
            x = rng.choice(shadow)
            bt.remove(x); shadow.remove(x)
        elif op == 8 and shadow:
            i = rng.randrange(len(shadow))
            del bt[i:]; del shadow[i:]
        elif op == 9:
            bt.sort(); shadow.sort()
        elif op == 10:
            bt.reverse(); shadow.reverse()
        elif op == 11 and rng.random() < 0.05:
            bt.clear(); shadow.clear()
        assert list(bt) == shadow
        assert bt.arr[:len(bt)].tolist() == shadow
        if rng.random() < 0.5:
            upload()
            assert uploaded[:len(shadow)] == shadow
