"""The B200 manager's host bookkeeping replayed against the reference's own run.

Every op of every scenario in tests/golden/paged_scenarios.json (recorded from
FlashInferPagedKVCache with the FlashInfer wrappers stubbed) is replayed on
nanoslg_b200.kv_cache.B200PagedKVCache with CPU tensors; page ids, block tables,
refcounts, write targets, positions and the CSR arrays must be identical."""
import json
import os

import pytest
import torch

from conftest import GOLDEN
from nanoslg_b200.kv_cache import B200PagedKVCache, KVCacheConfig

with open(os.path.join(GOLDEN, "paged_scenarios.json")) as f:
    SCEN = json.load(f)


def _manager(page_size, max_pages, prefix=True):
    cfg = KVCacheConfig(num_layers=1, num_kv_heads=1, num_qo_heads=1, head_dim=16,
                        page_size=page_size, max_pages=max_pages, dtype=torch.float32,
                        device=torch.device("cpu"), enable_prefix_caching=prefix)
    return B200PagedKVCache(cfg)


def _snapshot(mgr):
    return {
        "block_tables": {s: list(st.block_table) for s, st in sorted(mgr.seqs.items())},
        "num_tokens": {s: st.num_tokens for s, st in sorted(mgr.seqs.items())},
        "num_free": mgr.pool.num_free,
        "ref_count": list(mgr.pool.ref_count),
        "tokens_used": list(mgr.pool.tokens_used),
        "stats": {k: v for k, v in mgr.stats.items() if k != "backend"},
    }


@pytest.mark.parametrize("sc", SCEN, ids=[s["name"] for s in SCEN])
def test_scenario_bit_exact(sc):
    mgr = _manager(**sc["setup"])
    ctx = None
    for i, rec in enumerate(sc["records"]):
        op = rec["op"]
        kind = op[0]
        got = {}
        try:
            if kind == "alloc":
                got["ret"] = mgr.allocate_sequence(op[1], op[2], op[3])
            elif kind == "extend":
                mgr.extend_sequence(op[1], op[2])
            elif kind == "begin":
                ctx = mgr.begin_forward(op[1], op[2], op[3])
                B, iw = ctx.batch_size, ctx._iw
                got["write_info"] = [[list(x) for x in wi] for wi in ctx._write_info]
                got["positions"] = ctx._pos_i32.view(B, iw).tolist()
                got["start_positions"] = list(ctx.start_positions)
                got["seq_lens"] = list(ctx.seq_lens)
                got["is_decode"] = ctx._is_decode
                got["indptr"] = ctx.kv_indptr.tolist()
                got["indices"] = ctx.kv_indices.tolist()
                got["last_page_len"] = ctx.kv_last_page_len.tolist()
                if not ctx._is_decode:
                    got["qo_indptr"] = ctx.qo_indptr.tolist()
                # the position tensor handed to models (kv_cache.py:635-637): int64,
                # zero-padded past the input width
                pids = ctx.get_position_ids(iw + 2)
                assert pids.dtype == torch.long and pids.shape == (B, iw + 2)
                assert pids[:, :iw].tolist() == rec["positions"]
                assert not bool(pids[:, iw:].any())
                assert ctx.get_position_ids(max(iw - 1, 0)).tolist() == \
                    [row[:max(iw - 1, 0)] for row in rec["positions"]]
            elif kind == "end":
                mgr.end_forward(ctx)
            elif kind == "release":
                mgr.release_sequence(op[1])
            elif kind == "append":
                mgr.append_token_ids(op[1], op[2])
            elif kind == "rewind":
                mgr.seqs[op[1]].num_tokens = op[2]
            elif kind == "reset":
                mgr.reset()
        except RuntimeError as e:
            got["error"] = str(e)
        for key, val in got.items():
            assert val == rec[key], f"op {i} {op[:2]}: {key} differs"
        assert ("error" in got) == ("error" in rec), f"op {i}: error mismatch"
        assert _snapshot(mgr) == rec["state"], f"op {i} {op[:2]}: state differs"


def test_write_locations_follow_write_info():
    mgr = _manager(4, 32)
    mgr.allocate_sequence("a", list(range(10)))
    mgr.allocate_sequence("b", list(range(50, 53)))
    ctx = mgr.begin_forward(["a", "b"], [10, 3], [0, 7])
    loc = ctx._write_loc.view(2, 10).tolist()
    assert loc[0] == [p * 4 + s for p, s in ctx._write_info[0]]
    assert loc[1][:7] == [-1] * 7
    assert loc[1][7:] == [p * 4 + s for p, s in ctx._write_info[1]]
    assert ctx.q_row_start.tolist() == [0, 17]


def test_pool_pages_zeroed_on_alloc():
    mgr = _manager(4, 8)
    mgr.pool.k.fill_(3.0)
    mgr.pool.v.fill_(3.0)
    mgr.allocate_sequence("a", list(range(6)))
    mgr.begin_forward(["a"], [6], [0])
    for pid in mgr.seqs["a"].block_table:
        assert mgr.pool.k[:, pid].abs().sum() == 0 and mgr.pool.v[:, pid].abs().sum() == 0
    assert mgr.pool.k[:, 0].abs().sum() > 0      # the null page is never handed out


def test_factory_returns_b200_backend():
    from types import SimpleNamespace
    from nanoslg_b200.kv_cache import create_cache_manager
    hf = SimpleNamespace(num_hidden_layers=2, num_key_value_heads=2, num_attention_heads=4,
                         hidden_size=256)
    mc = SimpleNamespace(page_size=16, max_kv_pages=32, kv_backend="contiguous")
    mgr = create_cache_manager(hf, None, torch.device("cpu"), torch.float32, mc)
    assert isinstance(mgr, B200PagedKVCache) and mgr.cfg.backend == "b200"
    assert tuple(mgr.pool.k.shape) == (2, 32, 16, 2, 64)


def test_csr_matches_plain_loop_restatement_at_c2_size():
    """At the full C2 batch (64 sequences, lengths U[512, 8192]) the vectorised CSR of a
    decode step equals the reference's per-page loop restated in oracle/paged_plan.py."""
    from oracle import paged_plan
    g = torch.Generator().manual_seed(0)
    lens = torch.randint(512, 8193, (64,), generator=g).tolist()
    mgr = _manager(16, 40000)
    sids = [f"s{i}" for i in range(64)]
    for s, n in zip(sids, lens):
        mgr.allocate_sequence(s, None, num_tokens=n)
        mgr.seqs[s].num_tokens = n
    for step in range(3):
        ctx = mgr.begin_forward(sids, [1] * 64)
        bts = [list(mgr.seqs[s].block_table) for s in sids]
        ind, idx, lpl = paged_plan.csr(bts, ctx.seq_lens, 16)
        assert ctx.kv_indptr.tolist() == ind
        assert ctx.kv_indices.tolist() == idx
        assert ctx.kv_last_page_len.tolist() == lpl
        wi = paged_plan.write_targets(bts, ctx.start_positions, [1] * 64, 16)
        assert [[list(x) for x in w] for w in ctx._write_info] == [[list(x) for x in w] for w in wi]
        mgr.end_forward(ctx)
