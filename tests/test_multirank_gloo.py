"""N > 1 host logic on CPU with gloo ranks: the TP linear layers and collectives of
nanoslg_b200.tp_layers / parallel (Megatron column/row split, SUM all-reduce, LM-head
all-gather) against one unsplit layer, identical page tables on every TP rank (each
rank runs the same bookkeeping on the same token ids, so attention needs no exchange),
and the pipeline micro-batch schedule of LlamaRunner.decode_microbatched over 2 and 3
stages."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from nanoslg_b200 import parallel, tp_layers
        from nanoslg_b200.kv_cache import B200PagedKVCache, KVCacheConfig
        cfg = parallel.ParallelConfig(parallel.ParallelMode.TENSOR, world)
        ctx = parallel.ParallelContext.initialize(cfg, rank, device="cpu")
        ctx.setup_groups()
        g = torch.Generator().manual_seed(0)
        x = torch.randn(3, 5, 16, generator=g)
        w_col = torch.randn(8, 16, generator=g)
        w_row = torch.randn(16, 8, generator=g)
        col = tp_layers.ColumnParallelLinear(16, 8, gather_output=True)
        row = tp_layers.RowParallelLinear(8, 16)
        with torch.no_grad():
            col.weight.copy_(w_col.chunk(world, 0)[rank])          # models.py:409-421 split
            row.weight.copy_(w_row.chunk(world, 1)[rank])          # models.py:424-427 split
            y_col = col(x)
            y_row = row(torch.nn.functional.linear(x, w_col).chunk(world, -1)[rank].contiguous())
        ok_col = torch.allclose(y_col, torch.nn.functional.linear(x, w_col), atol=1e-5)
        ok_row = torch.allclose(y_row, torch.nn.functional.linear(
            torch.nn.functional.linear(x, w_col), w_row), atol=1e-4)
        # bookkeeping: same ops on every rank -> same CSR
        kc = KVCacheConfig(num_layers=1, num_kv_heads=8 // world, num_qo_heads=32 // world,
                           head_dim=16, page_size=16, max_pages=256, dtype=torch.float32,
                           device=torch.device("cpu"))
        mgr = B200PagedKVCache(kc)
        for i, n in enumerate([40, 17, 300]):
            mgr.allocate_sequence(f"s{i}", list(range(i, i + n)))
        c = mgr.begin_forward(["s0", "s1", "s2"], [40, 17, 300], [260, 283, 0])
        sig = torch.tensor([hash((tuple(c.kv_indices.tolist()), tuple(c._write_loc.tolist())))
                            % (1 << 31)], dtype=torch.int64)
        sigs = [torch.zeros_like(sig) for _ in range(world)]
        dist.all_gather(sigs, sig)
        same = all(int(s) == int(sigs[0]) for s in sigs)
        out[rank] = (ok_col, ok_row, same, tuple(col.weight.shape), tuple(row.weight.shape))
    finally:
        dist.destroy_process_group()


def test_two_rank_tp_layers_and_bookkeeping():
    world = 2
    port = _free_port()
    with mp.get_context("spawn").Manager() as m:
        out = m.dict()
        mp.start_processes(_worker, args=(world, port, out), nprocs=world, start_method="spawn",
                           join=True)
        res = dict(out)
    assert set(res) == {0, 1}
    for rank, (ok_col, ok_row, same, wc, wr) in res.items():
        assert ok_col and ok_row and same, (rank, res[rank])
        assert wc == (4, 16) and wr == (16, 4)


def _pp_worker(rank, world, port, num_micro, steps, out):
    """One pipeline stage per rank (TP 1): LlamaRunner.decode_microbatched's tick schedule
    and neighbour exchange, with the stage forward replaced by a known function."""
    import datetime
    import types
    from types import SimpleNamespace
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from nanoslg_b200.runner import LlamaRunner
        P, p, H, B = world, rank, 4, 2 * num_micro

        class _Cache:
            def __init__(self):
                self.begun = []

            def begin_forward(self, sids, counts, offsets=None):
                assert counts == [1] * len(sids)
                self.begun.append(tuple(sids))
                return tuple(sids)

            def end_forward(self, ctx):
                assert self.begun and self.begun[-1] == ctx

        def stage(self, x, ctx, mb):
            # stage p adds p + 1 to the hidden state; the first embeds the token as a
            # constant row, the last turns the row back into a token
            h = x.float().view(mb, 1, 1).expand(mb, 1, H) if p == 0 else x
            h = h + (p + 1)
            if p == P - 1:
                return (h[:, 0, 0].long() * 3 + 1) % 997
            return h.contiguous()

        r = object.__new__(LlamaRunner)
        r.pctx = SimpleNamespace(pp_rank=p, tp_rank=0, get_pp_next_rank=lambda: p + 1,
                                 get_pp_prev_rank=lambda: p - 1)
        r.pcfg = SimpleNamespace(pp_size=P, tp_size=1)
        r.seq_ids = [f"s{i}" for i in range(B)]
        r.hf = SimpleNamespace(hidden_size=H)
        r.dtype = torch.float32
        r.device = torch.device("cpu")
        r.cache = _Cache()
        r._stage_decode_forward = types.MethodType(stage, r)
        tokens = torch.arange(B, dtype=torch.long) * 11 + 5
        got = r.decode_microbatched(tokens, num_micro, steps)
        out[rank] = (None if got is None else got.tolist(), len(r.cache.begun))
    finally:
        dist.destroy_process_group()


def _lock_step(tokens, P, steps):
    shift = P * (P + 1) // 2
    rows = []
    for t in tokens:
        seq = []
        for _ in range(steps):
            t = ((t + shift) * 3 + 1) % 997
            seq.append(t)
        rows.append(seq)
    return rows



@pytest.mark.parametrize("world,num_micro", [(2, 2), (3, 3), (3, 4)])
def test_pp_microbatch_schedule_matches_lock_step(world, num_micro):
    """Micro-batches flowing through 2-3 gloo stages give every sequence the tokens of
    running the stages in lock step, on the first and the last stage; every stage runs
    steps x num_micro micro-batch forwards."""
    steps = 3
    port = _free_port()
    with mp.get_context("spawn").Manager() as m:
        out = m.dict()
        mp.start_processes(_pp_worker, args=(world, port, num_micro, steps, out), nprocs=world,
                           start_method="spawn", join=True)
        res = dict(out)
    B = 2 * num_micro
    want = _lock_step([i * 11 + 5 for i in range(B)], world, steps)
    assert set(res) == set(range(world))
    for rank, (got, nfwd) in res.items():
        assert nfwd == steps * num_micro, rank
        if rank in (0, world - 1):
            assert got == want, rank
        else:
            assert got is None


def _greedy_worker(rank, world, port, out):
    """models._LlamaStage._greedy under TP over gloo: each rank reduces its vocabulary
    shard and the ranks exchange (max, index) pairs; the argmax kernel is replaced by
    torch.argmax (CPU), which is what it is GPU-tested against."""
    import types
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from nanoslg_b200 import models, parallel, tp_layers
        cfg = parallel.ParallelConfig(parallel.ParallelMode.TENSOR, world)
        ctx = parallel.ParallelContext.initialize(cfg, rank, device="cpu")
        ctx.setup_groups()

        def argmax_rows(x, index_offset=0, values=False):
            idx = x.argmax(-1) + index_offset
            val = x.max(-1).values.float()
            return (idx, val) if values else idx

        models.ops.argmax_rows = argmax_rows
        V, H, rows = 24, 6, 7
        head = tp_layers.ParallelLMHead(H, V, gather_output=True)
        g = torch.Generator().manual_seed(3)
        w = torch.randn(V, H, generator=g)
        # rows 1-3: the maximum ties across shards (equal weight rows in both halves, and
        # an exact tie between indices 5 and 17 / 2 and 22); row 4: all logits equal
        w[17] = w[5]
        w[22] = w[2]
        h = torch.randn(rows, 1, H, generator=g)
        h[1, 0] = w[5] * 3
        h[2, 0] = w[2] * 3
        h[3, 0] = w[17] * 3
        h[4, 0] = 0.0
        with torch.no_grad():
            head.lm_head.weight.copy_(w.chunk(world, 0)[rank])
        stage = types.SimpleNamespace(lm_head=head)
        with torch.inference_mode():                 # as in the runner's decode steps
            got = models._LlamaStage._greedy(stage, h)
        want = torch.nn.functional.linear(h[:, -1], w).argmax(-1)
        out[rank] = (got.tolist(), want.tolist())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_vocab_parallel_greedy_exchange_matches_argmax_of_gathered_logits(world):
    """The (max, index) exchange of the vocab-parallel LM head picks the token argmax over
    the all-gathered logits would (the reference's path, tp_layers.py:89 then argmax),
    including exact ties across shards, which go to the lowest index."""
    port = _free_port()
    with mp.get_context("spawn").Manager() as m:
        out = m.dict()
        mp.start_processes(_greedy_worker, args=(world, port, out), nprocs=world,
                           start_method="spawn", join=True)
        res = dict(out)
    assert set(res) == set(range(world))
    for rank, (got, want) in res.items():
        assert got == want, rank
    assert res[0][1][1] == 5 and res[0][1][2] == 2 and res[0][1][4] == 0
