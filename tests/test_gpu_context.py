"""The B200 CacheContext / model path on the GPU against the reference's recorded
outputs (tests/golden): contiguous-SDPA attention cases (fp32, bf16 and fp16) and the
tiny fp32 Llama's greedy tokens."""
import json
import os
from types import SimpleNamespace

import pytest
import torch

from conftest import GOLDEN
from oracle.attention import attend_sequences
from oracle.rope_norm import apply_rotary, rope_table
from nanoslg_b200 import ops
from nanoslg_b200.kv_cache import B200PagedKVCache, KVCacheConfig, create_cache_manager

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
ATT = torch.load(os.path.join(GOLDEN, "attention_cases.pt")) + \
    torch.load(os.path.join(GOLDEN, "fp16_cases.pt"))["attention"]
DTYPES = {"torch.float32": torch.float32, "torch.bfloat16": torch.bfloat16,
          "torch.float16": torch.float16}


@pytest.fixture(autouse=True)
def _clean_status():
    ops.status_word(DEV).zero_()
    yield
    ops.check_device_status(DEV)


@pytest.mark.parametrize("case", ATT, ids=[c["name"] for c in ATT])
def test_context_attend_matches_reference(case):
    dt = DTYPES[case["dtype"]]
    tol = dict(rtol=1e-4, atol=1e-5) if dt == torch.float32 else dict(rtol=1e-2, atol=2e-2)
    B = len(case["lens"])
    cfg = KVCacheConfig(num_layers=2, num_kv_heads=case["hkv"], num_qo_heads=case["hq"],
                        head_dim=case["d"], page_size=16, max_pages=64, dtype=dt, device=DEV)
    mgr = B200PagedKVCache(cfg)
    sids = [f"s{i}" for i in range(B)]
    for s in sids:
        mgr.allocate_sequence(s)
    for step in case["steps"]:
        ctx = mgr.begin_forward(sids, step["counts"], step["offsets"])
        assert ctx.start_positions == step["start_positions"]
        for li, lay in enumerate(step["layers"]):
            out = ctx.attend(li, lay["q"].to(DEV), lay["k"].to(DEV), lay["v"].to(DEV),
                             case["hq"], case["hkv"]).cpu()
            for b, (o, n) in enumerate(zip(step["offsets"], step["counts"])):
                torch.testing.assert_close(out[b, o:o + n], lay["out"][b, o:o + n], **tol)
        mgr.end_forward(ctx)


def test_attend_rope_equals_unfused_path(monkeypatch):
    """attend_rope (fused kernel) == torch RoPE (the reference's ops) + attend, both on
    the plain decode split (the split-heads decode of small batches merges in another
    order; it is compared with the plain one in test_gpu_kernels)."""
    monkeypatch.setattr(ops, "DECODE_SPLIT_HEADS_PAIRS", 0)
    hq, hkv, d = 32, 8, 128
    cos, sin = rope_table(d, 8192, 500000.0)
    cos_d, sin_d = cos.to(DEV), sin.to(DEV)
    outs = []
    for fused in (True, False):
        cfg = KVCacheConfig(num_layers=1, num_kv_heads=hkv, num_qo_heads=hq, head_dim=d,
                            page_size=16, max_pages=256, dtype=torch.bfloat16, device=DEV)
        mgr = B200PagedKVCache(cfg)
        g = torch.Generator().manual_seed(21)
        sids = ["a", "b", "c"]
        for s, n in zip(sids, (300, 17, 64)):
            mgr.allocate_sequence(s, list(range(n)))
        res = []
        plan = [([300, 17, 64], [0, 283, 236])] + [([1, 1, 1], None)] * 3
        for counts, offs in plan:
            ctx = mgr.begin_forward(sids, counts, offs)
            S = max(counts)
            q = torch.randn(3, S, hq, d, generator=g).to(torch.bfloat16).to(DEV)
            k = torch.randn(3, S, hkv, d, generator=g).to(torch.bfloat16).to(DEV)
            v = torch.randn(3, S, hkv, d, generator=g).to(torch.bfloat16).to(DEV)
            if fused:
                o = ctx.attend_rope(0, q, k, v, cos_d, sin_d)
            else:
                pos = ctx.get_position_ids(S)
                o = ctx.attend(0, apply_rotary(q, cos_d[pos], sin_d[pos]),
                               apply_rotary(k, cos_d[pos], sin_d[pos]), v, hq, hkv)
            res.append(o.cpu())
            mgr.end_forward(ctx)
        outs.append(res)
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_llama8b_layer_shapes_prefill_then_decode():
    """One 8B-shaped layer (32/8 heads, D 128): prompt prefill of 512 then decode, against
    the oracle over the rotated q/k the kernel produced."""
    hq, hkv, d, B = 32, 8, 128, 4
    cos, sin = rope_table(d, 8192, 500000.0)
    cfg = KVCacheConfig(num_layers=1, num_kv_heads=hkv, num_qo_heads=hq, head_dim=d,
                        page_size=16, max_pages=512, dtype=torch.bfloat16, device=DEV)
    mgr = B200PagedKVCache(cfg)
    sids = [f"s{i}" for i in range(B)]
    lens = [512, 300, 511, 17]
    for s, n in zip(sids, lens):
        mgr.allocate_sequence(s, list(range(n)))
    g = torch.Generator().manual_seed(8)
    hist_k = [torch.zeros(0, hkv, d, dtype=torch.bfloat16) for _ in range(B)]
    hist_v = [torch.zeros(0, hkv, d, dtype=torch.bfloat16) for _ in range(B)]
    plan = [(lens, [512 - n for n in lens])] + [([1] * B, None)] * 4
    for counts, offs in plan:
        ctx = mgr.begin_forward(sids, counts, offs)
        S = max(counts)
        offs = offs or [0] * B
        q = torch.randn(B, S, hq, d, generator=g).to(torch.bfloat16)
        k = torch.randn(B, S, hkv, d, generator=g).to(torch.bfloat16)
        v = torch.randn(B, S, hkv, d, generator=g).to(torch.bfloat16)
        out = ctx.attend_rope(0, q.to(DEV), k.to(DEV), v.to(DEV), cos.to(DEV), sin.to(DEV)).cpu()
        pos = ctx.get_position_ids(S).cpu()
        qr, kr = apply_rotary(q, cos[pos], sin[pos]), apply_rotary(k, cos[pos], sin[pos])
        qs = []
        for b in range(B):
            o, n = offs[b], counts[b]
            hist_k[b] = torch.cat([hist_k[b], kr[b, o:o + n]])
            hist_v[b] = torch.cat([hist_v[b], v[b, o:o + n]])
            qs.append(qr[b, o:o + n])
        ref = attend_sequences(qs, hist_k, hist_v)
        for b in range(B):
            o, n = offs[b], counts[b]
            torch.testing.assert_close(out[b, o:o + n].view(n, hq, d), ref[b],
                                       rtol=1e-2, atol=2e-2)
        mgr.end_forward(ctx)


def test_tiny_llama_greedy_tokens_match_reference():
    """Config C1 (fp32, 2 layers, hidden 256) through nanoslg_b200.models + the B200 cache,
    driven like worker.py drives a TP=1 request: identical greedy tokens."""
    from nanoslg_b200 import models
    from nanoslg_b200.parallel import ParallelConfig, ParallelContext, ParallelMode
    with open(os.path.join(GOLDEN, "tiny_llama.json")) as f:
        g = json.load(f)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    pcfg = ParallelConfig(ParallelMode.TENSOR, 1)
    ParallelContext.initialize(pcfg, 0, device=DEV)
    hf = SimpleNamespace(**g["config"])
    model = models.create_model(hf, pcfg).float()
    assert [n for n, _ in model.named_parameters()] == g["param_order"]
    models.init_random_(model, seed=0)
    model = model.to(DEV)
    mc = SimpleNamespace(page_size=16, max_kv_pages=64, enable_prefix_caching=True)
    mgr = create_cache_manager(hf, pcfg, DEV, torch.float32, mc, max_batch_size=1)
    prompt = torch.tensor([g["prompt"]], device=DEV)
    toks = []
    with torch.inference_mode():
        mgr.allocate_sequence("s0", g["prompt"])
        ctx = mgr.begin_forward(["s0"], [len(g["prompt"])], [0])
        logits = model(prompt, ctx)
        mgr.end_forward(ctx)
        for step in range(len(g["tokens"])):
            t = int(logits[0, -1].argmax())
            toks.append(t)
            mgr.append_token_ids("s0", [t])
            if step + 1 == len(g["tokens"]):
                break
            ctx = mgr.begin_forward(["s0"], [1])
            logits = model(torch.tensor([[t]], device=DEV), ctx)
            mgr.end_forward(ctx)
    assert toks == g["tokens"]


def test_runner_tiny_llama_matches_reference_tokens():
    """The batch runner (worker.py's loop) on config C1 gives the reference's tokens; a
    second batch whose prompt is the first prompt plus 8 generated tokens reuses the two
    cached prompt pages through the radix tree and continues the same greedy sequence."""
    from nanoslg_b200 import models
    from nanoslg_b200.runner import LlamaRunner
    with open(os.path.join(GOLDEN, "tiny_llama.json")) as f:
        g = json.load(f)
    torch.backends.cuda.matmul.allow_tf32 = False
    hf = SimpleNamespace(**g["config"])
    r = LlamaRunner(hf, DEV, dtype=torch.float32, max_kv_pages=64)
    # the runner draws its weights on the device; load the fixture's CPU draw instead
    cpu = models.init_random_(models.create_model(hf, r.pcfg).float())
    r.model.load_state_dict(cpu.state_dict())
    want = g["tokens"]
    tok = r.prefill([g["prompt"]])
    toks = [int(tok[0])]
    for _ in range(len(want) - 1):
        tok = r.decode_step(tok)
        toks.append(int(tok[0]))
    assert toks == want
    r.release([toks])
    tok = r.prefill([g["prompt"] + want[:8]])
    assert r.prefix_lens == [32]                 # two 16-token pages from the radix tree
    toks2 = [int(tok[0])]
    for _ in range(7):
        tok = r.decode_step(tok)
        toks2.append(int(tok[0]))
    assert toks2 == want[8:16]
    r.release([toks2])


def test_runner_cuda_graph_decode_matches_reference_tokens():
    """Decode steps replayed from a captured CUDA graph (fixed plan buffer, fixed token
    input) give the reference's greedy tokens; a second batch (radix hit on the first
    prompt's pages) replays the same graph and continues the sequence."""
    from nanoslg_b200 import models
    from nanoslg_b200.runner import LlamaRunner
    with open(os.path.join(GOLDEN, "tiny_llama.json")) as f:
        g = json.load(f)
    torch.backends.cuda.matmul.allow_tf32 = False
    hf = SimpleNamespace(**g["config"])
    r = LlamaRunner(hf, DEV, dtype=torch.float32, max_kv_pages=64)
    cpu = models.init_random_(models.create_model(hf, r.pcfg).float())
    r.model.load_state_dict(cpu.state_dict())
    r.enable_cuda_graphs([1])
    want = g["tokens"]
    tok = r.prefill([g["prompt"]])
    toks = [int(tok[0])]
    for _ in range(len(want) - 1):
        tok = r.decode_step(tok)
        toks.append(int(tok[0]))
    assert toks == want
    assert 1 in r._graphs
    r.release([toks])
    tok = r.prefill([g["prompt"] + want[:8]])
    assert r.prefix_lens == [32]
    toks2 = [int(tok[0])]
    for _ in range(7):
        tok = r.decode_step(tok)
        toks2.append(int(tok[0]))
    assert toks2 == want[8:16]
    r.release([toks2])


@pytest.mark.parametrize("n_live", [24, 160])
def test_device_plan_matches_host_plan(n_live):
    """nslg_plan_decode_host (device block tables, csrc/plan.cu) builds the same decode
    plan as the host path (kv_cache.py:547-632 restated) over a run with page-boundary
    crossings, sequences joining and leaving (table rows reused, tables grown) and
    radix-shared prefixes (copy on write takes the host path for that step, then the
    device tables are refreshed). 24 sequences take the one-launch planner, 160 the
    scan + gather kernels."""
    import random
    from nanoslg_b200.kv_cache import B200PagedKVCache, KVCacheConfig
    dev = torch.device("cuda:0")
    cfg = dict(num_layers=1, num_kv_heads=2, num_qo_heads=4, head_dim=64, page_size=16,
               max_pages=4096, dtype=torch.bfloat16, device=dev, enable_prefix_caching=True)
    mgrs = [B200PagedKVCache(KVCacheConfig(**cfg)) for _ in range(2)]
    mgrs[1].device_plan = False
    assert mgrs[0].device_plan
    rng = random.Random(3)
    shared = [rng.randrange(1000) for _ in range(48)]
    live, nxt = [], 0

    def add(n_new):
        nonlocal nxt
        for _ in range(n_new):
            sid = f"q{nxt}"
            nxt += 1
            if rng.random() < 0.3:      # a prompt starting with a page-aligned shared prefix
                toks = shared + [rng.randrange(1000) for _ in range(rng.randrange(1, 40))]
            else:
                toks = [rng.randrange(1000) for _ in range(rng.randrange(1, 300))]
            for m in mgrs:
                m.allocate_sequence(sid, toks)
                st = m.seqs[sid]
                st.num_tokens = len(toks)        # prompt already cached
            live.append(sid)

    def drop(k):
        for _ in range(k):
            sid = live.pop(rng.randrange(len(live)))
            for m in mgrs:
                m.append_token_ids(sid, [1, 2, 3])
                m.release_sequence(sid)

    add(n_live)
    fields = ("_pos_i32", "_write_loc", "kv_indptr", "kv_indices", "kv_last_page_len",
              "qo_indptr", "q_row_start")
    for step in range(60):
        if step in (15, 35):
            drop(8)
            add(12)
        if n_live > 100 and step > 20:
            break
        ctxs = [m.begin_forward(list(live), [1] * len(live)) for m in mgrs]
        for f in fields:
            a, b = getattr(ctxs[0], f), getattr(ctxs[1], f)
            assert a.tolist() == b.tolist(), f"step {step}: {f} differs"
        assert ctxs[0]._write_info == ctxs[1]._write_info
        assert [list(m.seqs[s].block_table) for s in live for m in mgrs[:1]] == \
               [list(m.seqs[s].block_table) for s in live for m in mgrs[1:]]
        assert list(mgrs[0].pool.tokens_used) == list(mgrs[1].pool.tokens_used)
        for m, c in zip(mgrs, ctxs):
            m.end_forward(c)
    from nanoslg_b200 import ops
    ops.check_device_status(dev)


def test_device_plan_zeroes_new_pages():
    """Pages allocated since the last forward are zeroed in every layer (PagePool.alloc,
    kv_cache.py:411) by nslg_zero_pages on the device-planned decode path; the null page
    and pages of other sequences are left alone."""
    from nanoslg_b200.kv_cache import B200PagedKVCache, KVCacheConfig
    dev = torch.device("cuda:0")
    mgr = B200PagedKVCache(KVCacheConfig(num_layers=3, num_kv_heads=2, num_qo_heads=4,
                                         head_dim=64, page_size=16, max_pages=64,
                                         dtype=torch.bfloat16, device=dev,
                                         enable_prefix_caching=False))
    assert mgr.device_plan
    mgr.pool.k.fill_(3.0)
    mgr.pool.v.fill_(3.0)
    for s, n in (("a", 40), ("b", 16)):
        mgr.allocate_sequence(s, None, num_tokens=n)
        mgr.seqs[s].num_tokens = n
    ctx = mgr.begin_forward(["a", "b"], [1, 1])
    torch.cuda.synchronize(dev)
    pages = set(mgr.seqs["a"].block_table) | set(mgr.seqs["b"].block_table)
    for pid in pages:
        assert mgr.pool.k[:, pid].abs().sum() == 0 and mgr.pool.v[:, pid].abs().sum() == 0
    untouched = [p for p in range(64) if p not in pages]
    assert bool((mgr.pool.k[:, untouched] == 3.0).all())
    mgr.end_forward(ctx)


@pytest.mark.parametrize("batch", [5, 100, 300])
def test_plan_decode_device_arrays_match_host_arrays(batch):
    """nslg_plan_decode (inputs in device memory, scan + gather kernels) and
    nslg_plan_decode_host (inputs from host arrays; one launch up to 128 sequences) give
    the same plan for the same tables, rows, start positions and table updates."""
    import ctypes
    import numpy as np
    from nanoslg_b200 import _native as N
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(batch)
    ps, stride, rows = 16, 64, batch + 7
    slots = rng.permutation(rows)[:batch].astype(np.int32)
    starts = rng.integers(0, stride * ps - 1, batch).astype(np.int32)
    tables = rng.integers(1, 50000, (rows, stride)).astype(np.int32)
    nu = 40
    upd = np.stack([rng.choice(slots, nu), rng.integers(0, stride, nu),
                    rng.integers(1, 50000, nu)], 1).astype(np.int32)
    upd = upd[np.unique(upd[:, :2], axis=0, return_index=True)[1]]   # one value per entry
    nu = upd.shape[0]
    total = int((starts // ps + 1).sum())
    size = 6 * batch + 2 + total
    outs = []
    status = ops.status_word(dev)
    lib = N.lib()
    stream = torch.cuda.current_stream(dev).cuda_stream
    for host in (False, True):
        bt = torch.from_numpy(tables).to(dev)
        plan = torch.full((size,), -7, dtype=torch.int32, device=dev)
        B = batch
        if host:
            hs, hst, hu = (np.ascontiguousarray(a) for a in (slots, starts, upd))
            rc = lib.nslg_plan_decode_host(B, ps, hs.ctypes.data, hst.ctypes.data, nu,
                                           hu.ctypes.data, 0, None, None, None, 1, 1, 16,
                                           bt.data_ptr(), stride, rows, plan.data_ptr(), total,
                                           status.data_ptr(), stream)
        else:
            ds, dst, du = (torch.from_numpy(a).to(dev) for a in (slots, starts, upd))
            p = plan.data_ptr()
            rc = lib.nslg_plan_decode(B, ps, ds.data_ptr(), dst.data_ptr(), nu, du.data_ptr(),
                                      bt.data_ptr(), stride, rows, p, p + 4 * B, p + 8 * B,
                                      p + 4 * (3 * B + 1), p + 4 * (4 * B + 1),
                                      p + 4 * (5 * B + 2), p + 4 * (6 * B + 2), total,
                                      status.data_ptr(), stream)
        assert rc == 0, lib.nslg_last_error()
        torch.cuda.synchronize(dev)
        outs.append((plan.cpu(), bt.cpu()))
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1], outs[1][1])
    # and against the plan restated on the host
    tab = tables.copy()
    tab[upd[:, 0], upd[:, 1]] = upd[:, 2]
    n = starts // ps + 1
    indptr = np.concatenate([[0], np.cumsum(n)])
    want = np.concatenate([starts, tab[slots, starts // ps] * ps + starts % ps, indptr,
                           starts + 1 - (n - 1) * ps, np.arange(batch + 1), np.arange(batch),
                           np.concatenate([tab[s, :k] for s, k in zip(slots, n)])])
    assert outs[1][0].numpy().tolist() == want.tolist()


def test_zero_pages_entry_point():
    """nslg_zero_pages zeroes exactly the listed pages of every layer of one pool."""
    from nanoslg_b200 import _native as N
    dev = torch.device("cuda:0")
    pool = torch.full((3, 10, 16, 2, 64), 3.0, dtype=torch.bfloat16, device=dev)
    pages = torch.tensor([2, 5, 9], dtype=torch.int32, device=dev)
    page_bytes = pool[0, 0].numel() * 2
    N.call("nslg_zero_pages", pages.data_ptr(), 3, pool.data_ptr(), 3, 10, page_bytes,
           ops.status_word(dev).data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize(dev)
    z = [2, 5, 9]
    assert int(pool[:, z].float().abs().sum()) == 0
    keep = [p for p in range(10) if p not in z]
    assert bool((pool[:, keep] == 3.0).all())


def test_plan_decode_host_refuses_graph_capture():
    """nslg_plan_decode_host reads host staging, so it cannot be baked into a CUDA graph:
    inside a capture it returns NSLG_ERR_UNSUPPORTED without enqueuing anything, and the
    capture ends normally."""
    import numpy as np
    from nanoslg_b200 import _native as N
    dev = torch.device("cuda:0")
    lib = N.lib()
    slots = np.zeros(1, dtype=np.int32)
    starts = np.zeros(1, dtype=np.int32)
    bt = torch.ones((4, 8), dtype=torch.int32, device=dev)
    plan = torch.zeros(64, dtype=torch.int32, device=dev)
    side = torch.cuda.Stream(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(g, stream=side):
            rc = lib.nslg_plan_decode_host(1, 16, slots.ctypes.data, starts.ctypes.data, 0, None,
                                           0, None, None, None, 1, 1, 16, bt.data_ptr(), 8, 4,
                                           plan.data_ptr(), 8, None, side.cuda_stream)
            plan.add_(0)                  # the graph holds something to replay
    assert rc == N.ERR_UNSUPPORTED and b"graph" in lib.nslg_last_error()
    g.replay()
    torch.cuda.synchronize(dev)
    assert int(plan.abs().sum()) == 0


def test_small_batch_decode_takes_the_split_heads_path(monkeypatch):
    """Decode steps of a small batch through the context split the work by kv head as
    well as by pages (its page list built once per step) and agree with the plain split
    within fp32 rounding of the merge order, step after step."""
    hq, hkv, d = 32, 8, 128
    cos, sin = rope_table(d, 8192, 500000.0)
    cos_d, sin_d = cos.to(DEV), sin.to(DEV)
    outs = {}
    for pairs in (64, 0):
        monkeypatch.setattr(ops, "DECODE_SPLIT_HEADS_PAIRS", pairs)
        cfg = KVCacheConfig(num_layers=1, num_kv_heads=hkv, num_qo_heads=hq, head_dim=d,
                            page_size=16, max_pages=256, dtype=torch.bfloat16, device=DEV)
        mgr = B200PagedKVCache(cfg)
        g = torch.Generator().manual_seed(5)
        sids = ["a", "b"]
        for s, n in zip(sids, (700, 33)):
            mgr.allocate_sequence(s, None, num_tokens=n)
            mgr.seqs[s].num_tokens = n          # history already cached
        res = []
        for _ in range(3):
            ctx = mgr.begin_forward(sids, [1, 1])
            q = torch.randn(2, 1, hq, d, generator=g).to(torch.bfloat16).to(DEV)
            k = torch.randn(2, 1, hkv, d, generator=g).to(torch.bfloat16).to(DEV)
            v = torch.randn(2, 1, hkv, d, generator=g).to(torch.bfloat16).to(DEV)
            res.append(ctx.attend_rope(0, q, k, v, cos_d, sin_d).cpu())
            assert (ctx._split_plan is not None) == (pairs > 0)
            mgr.end_forward(ctx)
        outs[pairs] = res
    for a, b in zip(outs[64], outs[0]):
        torch.testing.assert_close(a, b, rtol=1e-2, atol=1e-2)
