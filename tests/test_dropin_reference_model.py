"""Drop-in check with the reference's own model code: NanoSLG's unmodified
``nanoslg/models.py`` (LlamaTP, its RoPE, its ``_attention_forward`` calling
``cache_ctx.get_position_ids`` and ``cache_ctx.attend``, models.py:86-105) runs the tiny
fp32 Llama of config C1 over this package's ``create_cache_manager`` (the manager,
contexts, page pool, radix tree and the plans they build), driven in the order
worker.py:365-426 drives a batch: allocate, prefill forward, then begin / forward / end
decode steps. The greedy tokens must be the ones the reference produced on its own
contiguous backend (tests/golden/tiny_llama.json).

The reference is importable only where its checkout is present (set NANOSLG_REFERENCE
to it; this test is skipped otherwise). There is no GPU here, so the three native calls
behind ``attend`` (KV append into the pool, paged decode, paged prefill) are replaced,
for this test only, by a CPU stand-in that reads and writes the same pool through the
same plan arrays (write slots, CSR page lists, query row starts) with the oracle's
attention. What this covers is the boundary: the reference's model driving this
package's bookkeeping and plans. The kernels themselves are compared with the oracle on
the same plans by the GPU tests."""
import importlib
import json
import os
import sys
from types import SimpleNamespace

import pytest
import torch

from conftest import GOLDEN, REFERENCE
from oracle.attention import attend_sequences

pytestmark = pytest.mark.skipif(
    REFERENCE is None or not os.path.isdir(os.path.join(REFERENCE or "", "nanoslg")),
    reason="the reference checkout is not available (NANOSLG_REFERENCE)")


def _seq_kv(pool, indptr, indices, lpl, b):
    ps = pool.shape[1]
    s, e = int(indptr[b]), int(indptr[b + 1])
    if e == s:
        return pool.new_zeros(0, pool.shape[2], pool.shape[3])
    n = (e - s - 1) * ps + int(lpl[b])
    return pool[indices[s:e].long()].reshape(-1, pool.shape[2], pool.shape[3])[:n]


def _append(q, k, v, positions, cos, sin, write_loc, pool_k, pool_v, q_out=None,
            rotate=True):
    assert q is None and not rotate          # the reference rotates in its model
    ps = pool_k.shape[1]
    kk = k.reshape(-1, k.shape[-2], k.shape[-1])
    vv = v.reshape(-1, v.shape[-2], v.shape[-1])
    for i, w in enumerate(write_loc.reshape(-1).tolist()):
        if w >= 0:
            pool_k[w // ps, w % ps] = kk[i]
            pool_v[w // ps, w % ps] = vv[i]
    return None


def _decode(q, pool_k, pool_v, kv_indptr, kv_indices, kv_last_page_len, sm_scale, out=None):
    res = []
    for b in range(q.shape[0]):
        k = _seq_kv(pool_k, kv_indptr, kv_indices, kv_last_page_len, b)
        v = _seq_kv(pool_v, kv_indptr, kv_indices, kv_last_page_len, b)
        res.append(attend_sequences([q[b:b + 1]], [k], [v])[0][0])
    return torch.stack(res)


def _prefill(q, qo_indptr, max_qo_len, pool_k, pool_v, kv_indptr, kv_indices,
             kv_last_page_len, sm_scale, causal=True, q_row_start=None, out=None):
    rows = q.reshape(-1, q.shape[-2], q.shape[-1])
    o = out.view(-1, q.shape[-2], q.shape[-1])
    for b in range(qo_indptr.numel() - 1):
        n = int(qo_indptr[b + 1] - qo_indptr[b])
        r0 = int(q_row_start[b]) if q_row_start is not None else int(qo_indptr[b])
        k = _seq_kv(pool_k, kv_indptr, kv_indices, kv_last_page_len, b)
        v = _seq_kv(pool_v, kv_indptr, kv_indices, kv_last_page_len, b)
        o[r0:r0 + n] = attend_sequences([rows[r0:r0 + n]], [k], [v], causal=causal)[0]
    return out


def test_reference_models_py_drives_the_b200_cache_manager(monkeypatch):
    sys.path.insert(0, REFERENCE)
    try:
        M = importlib.import_module("nanoslg.models")
        P = importlib.import_module("nanoslg.parallel")
    finally:
        sys.path.remove(REFERENCE)
    from nanoslg_b200 import kv_cache, ops

    monkeypatch.setattr(ops, "rope_kv_append", _append)
    monkeypatch.setattr(ops, "paged_decode", _decode)
    monkeypatch.setattr(ops, "paged_prefill", _prefill)
    monkeypatch.setattr(ops, "flush_zero_pages", lambda *a, **k: None, raising=False)

    with open(os.path.join(GOLDEN, "tiny_llama.json")) as f:
        g = json.load(f)
    torch.set_num_threads(1)
    pconf = P.ParallelConfig(P.ParallelMode.TENSOR, 1)
    pctx = P.ParallelContext.initialize(pconf, 0)
    pctx.device = torch.device("cpu")
    hf = SimpleNamespace(**g["config"])
    model = M.create_model(hf, pconf).float()            # the reference's LlamaTP
    torch.manual_seed(0)
    with torch.no_grad():
        for n, p in model.named_parameters():
            if "norm" not in n:
                p.normal_(0.0, 0.02)
    # this package's factory, called with the reference's own config objects
    mgr = kv_cache.create_cache_manager(
        hf, pconf, torch.device("cpu"), torch.float32,
        SimpleNamespace(page_size=16, max_kv_pages=32), max_batch_size=1)
    assert isinstance(mgr, kv_cache.B200PagedKVCache)
    prompt = g["prompt"]
    toks = []
    with torch.inference_mode():
        plen = mgr.allocate_sequence("s0", list(prompt))
        assert plen == 0
        ctx = mgr.begin_forward(["s0"], [len(prompt)], [0])
        logits = model(torch.tensor([prompt]), ctx, None)
        mgr.end_forward(ctx)
        for step in range(len(g["tokens"])):
            t = int(logits[0, -1].argmax())
            toks.append(t)
            if step + 1 == len(g["tokens"]):
                break
            mgr.append_token_ids("s0", [t])
            ctx = mgr.begin_forward(["s0"], [1])
            assert ctx.get_start_pos(0) == len(prompt) + step
            logits = model(torch.tensor([[t]]), ctx, None)
            mgr.end_forward(ctx)
        mgr.release_sequence("s0")
    assert toks == g["tokens"]
