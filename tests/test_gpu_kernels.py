"""GPU parity of each kernel against the CPU oracle, through the C ABI.

Tolerances (north star): RoPE/KV append bit-exact; attention in bf16 within 2e-2 abs /
1e-2 rel of the fp32 oracle over the same bf16 inputs; fp32 attention within 1e-5."""
import math

import pytest
import torch

from oracle.attention import attend_sequences
from oracle.rope_norm import apply_rotary, rmsnorm, rope_table
from nanoslg_b200 import ops
from paged_util import make_paged, sequence_kv

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
BF16_TOL = dict(rtol=1e-2, atol=2e-2)
F32_TOL = dict(rtol=1e-5, atol=1e-5)


def _tol(dt):
    return BF16_TOL if dt == torch.bfloat16 else F32_TOL


@pytest.fixture(autouse=True)
def _clean_status():
    ops.status_word(DEV).zero_()
    yield
    ops.check_device_status(DEV)


@pytest.mark.parametrize("dt,hq,hkv,d", [(torch.bfloat16, 32, 8, 128), (torch.float32, 4, 2, 64),
                                         (torch.bfloat16, 8, 1, 64)])
def test_rope_kv_append_bit_exact(dt, hq, hkv, d):
    g = torch.Generator().manual_seed(3)
    T, ps, P = 37, 16, 20
    cos, sin = rope_table(d, 4096, 500000.0)
    q = torch.randn(T, hq, d, generator=g).to(dt)
    k = torch.randn(T, hkv, d, generator=g).to(dt)
    v = torch.randn(T, hkv, d, generator=g).to(dt)
    pos = torch.randint(0, 4096, (T,), generator=g, dtype=torch.int32)
    loc = torch.randperm(P * ps, generator=g)[:T].to(torch.int32)
    loc[::5] = -1                                        # padded cells are not written
    pk = torch.full((P, ps, hkv, d), 7.0, dtype=dt, device=DEV)
    pv = torch.full((P, ps, hkv, d), 7.0, dtype=dt, device=DEV)
    q_out = ops.rope_kv_append(q.to(DEV), k.to(DEV), v.to(DEV), pos.to(DEV), cos.to(DEV),
                               sin.to(DEV), loc.to(DEV), pk, pv)
    p64 = pos.long()[None]
    q_ref = apply_rotary(q[None], cos[p64], sin[p64])[0]
    k_ref = apply_rotary(k[None], cos[p64], sin[p64])[0]
    assert torch.equal(q_out.cpu(), q_ref)
    fk, fv = pk.view(-1, hkv, d).cpu(), pv.view(-1, hkv, d).cpu()
    w = loc >= 0
    assert torch.equal(fk[loc[w].long()], k_ref[w])
    assert torch.equal(fv[loc[w].long()], v[w])
    untouched = torch.ones(P * ps, dtype=torch.bool)
    untouched[loc[w].long()] = False
    assert bool((fk[untouched] == 7.0).all()) and bool((fv[untouched] == 7.0).all())


@pytest.mark.parametrize("d", [128, 64])
def test_rope_kv_append_bf16_wide_range(d):
    """bf16 path (paired bf16 multiplies and adds) against the reference's torch ops over
    many tokens whose values span 2^-40 .. 2^20 (products down to the bf16 subnormal
    range), positions across the whole table, and the unrotated append (rotate=False)."""
    g = torch.Generator().manual_seed(17)
    T, hq, hkv, ps, P = 3000, 16, 4, 16, 200
    bf = torch.bfloat16
    cos, sin = rope_table(d, 8192, 500000.0)
    scale = lambda *s: torch.exp2(torch.randint(-40, 21, s, generator=g).float())
    q = (torch.randn(T, hq, d, generator=g) * scale(T, hq, 1)).to(bf)
    k = (torch.randn(T, hkv, d, generator=g) * scale(T, hkv, 1)).to(bf)
    v = torch.randn(T, hkv, d, generator=g).to(bf)
    pos = torch.randint(0, 8192, (T,), generator=g, dtype=torch.int32)
    loc = torch.randperm(P * ps, generator=g)[:T].to(torch.int32)
    pk = torch.zeros((P, ps, hkv, d), dtype=bf, device=DEV)
    pv = torch.zeros_like(pk)
    q_out = ops.rope_kv_append(q.to(DEV), k.to(DEV), v.to(DEV), pos.to(DEV), cos.to(DEV),
                               sin.to(DEV), loc.to(DEV), pk, pv)
    p64 = pos.long()[None]
    assert torch.equal(q_out.cpu(), apply_rotary(q[None], cos[p64], sin[p64])[0])
    fk = pk.view(-1, hkv, d).cpu()
    assert torch.equal(fk[loc.long()], apply_rotary(k[None], cos[p64], sin[p64])[0])
    assert torch.equal(pv.view(-1, hkv, d).cpu()[loc.long()], v)
    # already-rotated k (the attend() path): copied as is
    pk.zero_()
    ops.rope_kv_append(None, k.to(DEV), v.to(DEV), None, None, None, loc.to(DEV), pk, pv,
                       rotate=False)
    assert torch.equal(pk.view(-1, hkv, d).cpu()[loc.long()], k)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("hidden", [256, 4096, 8192])
def test_rmsnorm_residual(dt, hidden):
    g = torch.Generator().manual_seed(4)
    x = (torch.randn(9, hidden, generator=g) * 2).to(dt)
    r = torch.randn(9, hidden, generator=g).to(dt)
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(dt)
    y = ops.rmsnorm_residual(x.to(DEV), w.to(DEV), 1e-5)
    tol = dict(rtol=1e-2, atol=1e-2) if dt == torch.bfloat16 else dict(rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(y.cpu(), rmsnorm(x, w, 1e-5), **tol)
    rd = r.to(DEV)
    y2 = ops.rmsnorm_residual(x.to(DEV), w.to(DEV), 1e-5, residual=rd)
    h = x + r
    assert torch.equal(rd.cpu(), h)                      # the residual add is bit-exact
    torch.testing.assert_close(y2.cpu(), rmsnorm(h, w, 1e-5), **tol)


DECODE_CASES = [
    # hq, hkv, d, lens
    (32, 8, 128, [1, 15, 16, 17, 100, 1000, 2049]),
    (16, 4, 128, [3, 33, 700, 1500]),
    (16, 2, 128, [5, 16, 900]),
    (4, 1, 128, [1, 2, 31, 32, 33, 600]),
    (8, 1, 128, [77, 1200]),
    (64, 8, 128, [40, 513]),
    (8, 8, 128, [19, 260]),
    (8, 2, 64, [9, 300, 1024]),
    (32, 8, 128, [0, 50, 0, 3]),                         # sequences without pages
]


@pytest.mark.parametrize("mode", ["auto", "inline", "kernel"])
@pytest.mark.parametrize("hq,hkv,d,lens", DECODE_CASES)
def test_paged_decode_bf16(hq, hkv, d, lens, mode, monkeypatch):
    if mode != "auto":
        monkeypatch.setenv("NSLG_DECODE_MERGE", mode)
    pk = make_paged(lens, hkv, d, 4096, torch.bfloat16, DEV, seed=len(lens) + hq)
    g = torch.Generator().manual_seed(5)
    q = torch.randn(len(lens), hq, d, generator=g).to(torch.bfloat16)
    out = ops.paged_decode(q.to(DEV), pk["pool_k"], pk["pool_v"], pk["indptr"], pk["indices"],
                           pk["lpl"], 1 / math.sqrt(d)).cpu()
    ks = [sequence_kv(pk, b, "k") for b in range(len(lens))]
    vs = [sequence_kv(pk, b, "v") for b in range(len(lens))]
    ref = attend_sequences([q[b:b + 1] for b in range(len(lens))], ks, vs)
    for b, n in enumerate(lens):
        exp = ref[b][0] if n > 0 else torch.zeros(hq, d, dtype=torch.bfloat16)
        torch.testing.assert_close(out[b], exp, **BF16_TOL)


@pytest.mark.parametrize("hq,hkv,d,lens", [
    (32, 8, 128, [512]),                                 # 8B TP=1, batch 1
    (32, 8, 128, [1, 17, 300, 2049]),
    (16, 4, 128, [0, 700, 33]),                          # a sequence without pages
    (16, 2, 128, [5000]),
    (8, 2, 64, [9, 300, 1024]),
])
def test_paged_decode_split_heads(hq, hkv, d, lens):
    """The decode split by kv head as well as by pages (each (sequence, kv head) a
    sequence of the group's query heads, page ids page * hkv + head from
    split_heads_plan): the oracle's attention within the bf16 tolerance, and the plain
    decode's within fp32 rounding of the merge order."""
    pk = make_paged(lens, hkv, d, 4096, torch.bfloat16, DEV, seed=len(lens) + 3 * hq)
    g = torch.Generator().manual_seed(11)
    q = torch.randn(len(lens), hq, d, generator=g).to(torch.bfloat16)
    qd = q.to(DEV)
    plan = ops.split_heads_plan(pk["indptr"], pk["indices"], pk["lpl"], hkv,
                                pk["pool_k"].shape[0])
    out = ops.paged_decode_split_heads(qd, pk["pool_k"], pk["pool_v"], plan,
                                       1 / math.sqrt(d))
    plain = ops.paged_decode(qd, pk["pool_k"], pk["pool_v"], pk["indptr"], pk["indices"],
                             pk["lpl"], 1 / math.sqrt(d))
    torch.testing.assert_close(out, plain, rtol=1e-2, atol=1e-2)
    out = out.cpu()
    ks = [sequence_kv(pk, b, "k") for b in range(len(lens))]
    vs = [sequence_kv(pk, b, "v") for b in range(len(lens))]
    ref = attend_sequences([q[b:b + 1] for b in range(len(lens))], ks, vs)
    for b, n in enumerate(lens):
        exp = ref[b][0] if n > 0 else torch.zeros(hq, d, dtype=torch.bfloat16)
        torch.testing.assert_close(out[b], exp, **BF16_TOL)
    # deterministic
    again = ops.paged_decode_split_heads(qd, pk["pool_k"], pk["pool_v"], plan, 1 / math.sqrt(d))
    assert torch.equal(again.cpu(), out)


def test_paged_decode_many_sequences_split_across_ctas():
    g = torch.Generator().manual_seed(6)
    lens = torch.randint(1, 3000, (97,), generator=g).tolist()
    pk = make_paged(lens, 8, 128, 30000, torch.bfloat16, DEV, seed=9)
    q = torch.randn(len(lens), 32, 128, generator=g).to(torch.bfloat16)
    out = ops.paged_decode(q.to(DEV), pk["pool_k"], pk["pool_v"], pk["indptr"], pk["indices"],
                           pk["lpl"], 1 / math.sqrt(128)).cpu()
    for b in range(len(lens)):
        ref = attend_sequences([q[b:b + 1]], [sequence_kv(pk, b, "k")], [sequence_kv(pk, b, "v")])
        torch.testing.assert_close(out[b], ref[0][0], **BF16_TOL)


@pytest.mark.parametrize("mode", ["inline", "kernel"])
def test_paged_decode_merge_modes_and_arrival_counts(mode, monkeypatch):
    """Both ways of combining sequences split across CTAs: inside the one decode launch by
    the last CTA of each sequence to finish ("inline"), or by the merge kernel behind it
    ("kernel"). After every call the per-CTA arrival counts at the workspace's head are
    zero again, whatever the batch; the same call twice gives bit-identical outputs (the
    inline merge does not depend on which CTA runs it). Spans from 2 to all CTAs per
    sequence (a 40000-token sequence over every SM), empty sequences among them."""
    monkeypatch.setenv("NSLG_DECODE_MERGE", mode)
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    g = torch.Generator().manual_seed(12)
    for i, lens in enumerate([[5000], [1, 0, 40000, 17], [700] * 40, [3000, 0, 2]]):
        pk = make_paged(lens, 8, 128, sum(-(-n // 16) for n in lens) + 64, torch.bfloat16,
                        DEV, seed=70 + i)
        q = torch.randn(len(lens), 32, 128, generator=g).to(torch.bfloat16)
        args = (q.to(DEV), pk["pool_k"], pk["pool_v"], pk["indptr"], pk["indices"], pk["lpl"],
                1 / math.sqrt(128))
        out = ops.paged_decode(*args)
        torch.cuda.synchronize(DEV)
        ws = ops._STATE.ws[DEV]
        assert int(ws[:sms * 4].count_nonzero()) == 0
        assert torch.equal(ops.paged_decode(*args), out)
        out = out.cpu()
        for b, n in enumerate(lens):
            if n == 0:
                assert not bool(out[b].any())
                continue
            ref = attend_sequences([q[b:b + 1]], [sequence_kv(pk, b, "k")],
                                   [sequence_kv(pk, b, "v")])
            torch.testing.assert_close(out[b], ref[0][0], **BF16_TOL)


def test_paged_decode_c2_shape_sampled():
    """The benchmark's decode workload (64 sequences, lengths U[512, 8192], 32/8 heads,
    pages shuffled over a large pool): all outputs finite, ten sequences against the
    oracle."""
    g = torch.Generator().manual_seed(0)
    lens = torch.randint(512, 8193, (64,), generator=g).tolist()
    pk = make_paged(lens, 8, 128, sum(-(-n // 16) for n in lens) + 2000, torch.bfloat16, DEV,
                    seed=41)
    q = torch.randn(64, 32, 128, generator=g).to(torch.bfloat16)
    out = ops.paged_decode(q.to(DEV), pk["pool_k"], pk["pool_v"], pk["indptr"], pk["indices"],
                           pk["lpl"], 1 / math.sqrt(128))
    assert bool(torch.isfinite(out).all())
    out = out.cpu()
    for b in (0, 3, 9, 20, 33, 40, 51, 58, 62, 63):
        ref = attend_sequences([q[b:b + 1]], [sequence_kv(pk, b, "k")], [sequence_kv(pk, b, "v")])
        torch.testing.assert_close(out[b], ref[0][0], **BF16_TOL)


def test_paged_decode_fp32_and_other_page_sizes():
    for dt, ps, d in [(torch.float32, 16, 64), (torch.float32, 4, 128), (torch.bfloat16, 8, 128)]:
        lens = [1, 7, 64, 301]
        pk = make_paged(lens, 2, d, 1024, dt, DEV, seed=11, page_size=ps)
        q = torch.randn(len(lens), 8, d, generator=torch.Generator().manual_seed(2)).to(dt)
        out = ops.paged_decode(q.to(DEV), pk["pool_k"], pk["pool_v"], pk["indptr"],
                               pk["indices"], pk["lpl"], 1 / math.sqrt(d)).cpu()
        for b in range(len(lens)):
            ref = attend_sequences([q[b:b + 1]], [sequence_kv(pk, b, "k")],
                                   [sequence_kv(pk, b, "v")])
            torch.testing.assert_close(out[b], ref[0][0], **_tol(dt))


@pytest.mark.parametrize("dt,hq,hkv,d", [(torch.bfloat16, 32, 8, 128), (torch.float32, 4, 2, 64),
                                         (torch.bfloat16, 16, 2, 128), (torch.bfloat16, 8, 8, 128),
                                         (torch.bfloat16, 16, 1, 128), (torch.bfloat16, 8, 2, 64)])
def test_paged_prefill_causal_ragged(dt, hq, hkv, d):
    # (history already in the cache, new rows): covers plain prefill, extend after a
    # prefix hit, single-token rows and empty sequences
    spec = [(0, 37), (16, 20), (5, 1), (0, 130), (64, 0), (200, 77)]
    lens = [h + n for h, n in spec]
    pk = make_paged(lens, hkv, d, 2048, dt, DEV, seed=13)
    g = torch.Generator().manual_seed(7)
    S = max(n for _, n in spec)
    B = len(spec)
    q = torch.randn(B, S, hq, d, generator=g).to(dt)
    offsets = [S - n for _, n in spec]                    # left padded like the worker
    counts = [n for _, n in spec]
    qo = torch.tensor([0] + list(torch.cumsum(torch.tensor(counts), 0)), dtype=torch.int32)
    row_start = torch.tensor([b * S + o for b, o in enumerate(offsets)], dtype=torch.int32)
    out = ops.paged_prefill(q.to(DEV), qo.to(DEV), S, pk["pool_k"], pk["pool_v"], pk["indptr"],
                            pk["indices"], pk["lpl"], 1 / math.sqrt(d), causal=True,
                            q_row_start=row_start.to(DEV)).cpu()
    ks = [sequence_kv(pk, b, "k") for b in range(B)]
    vs = [sequence_kv(pk, b, "v") for b in range(B)]
    ref = attend_sequences([q[b, offsets[b]:] for b in range(B)], ks, vs)
    for b in range(B):
        torch.testing.assert_close(out[b, offsets[b]:], ref[b], **_tol(dt))
        assert bool((out[b, :offsets[b]] == 0).all())     # padded rows stay zero


@pytest.mark.parametrize("scale", [1.0, 6.0])
def test_paged_prefill_long_prompts(scale):
    """Long prompts through the tcgen05 kernel (many work items and kv tiles per item,
    prompts that end mid-tile), plain and with query values scaled up so that the row
    maxima keep growing past the lazy-rescale threshold (2^8) within a row."""
    hq, hkv, d = 32, 8, 128
    spec = [(0, 2100), (0, 1500), (300, 700), (0, 129)]
    lens = [h + n for h, n in spec]
    pk = make_paged(lens, hkv, d, 2048, torch.bfloat16, DEV, seed=21)
    g = torch.Generator().manual_seed(22)
    counts = [n for _, n in spec]
    T = sum(counts)
    q = (torch.randn(T, hq, d, generator=g) * scale).to(torch.bfloat16)
    qo = torch.tensor([0] + list(torch.cumsum(torch.tensor(counts), 0)), dtype=torch.int32)
    out = ops.paged_prefill(q.to(DEV), qo.to(DEV), max(counts), pk["pool_k"], pk["pool_v"],
                            pk["indptr"], pk["indices"], pk["lpl"], 1 / math.sqrt(d),
                            causal=True).cpu()
    ks = [sequence_kv(pk, b, "k") for b in range(len(spec))]
    vs = [sequence_kv(pk, b, "v") for b in range(len(spec))]
    rows = [q[int(qo[b]):int(qo[b + 1])] for b in range(len(spec))]
    ref = attend_sequences(rows, ks, vs)
    for b in range(len(spec)):
        torch.testing.assert_close(out[int(qo[b]):int(qo[b + 1])], ref[b], **BF16_TOL)


def test_paged_prefill_c3_shape_sampled():
    """The benchmark's prefill workload (64 prompts x 512 tokens, 32/8 heads, shuffled
    pages): every output finite, and eight sequences checked against the oracle."""
    hq, hkv, d, B, P = 32, 8, 128, 64, 512
    pk = make_paged([P] * B, hkv, d, B * P // 16 + 1, torch.bfloat16, DEV, seed=31)
    g = torch.Generator().manual_seed(32)
    q = torch.randn(B * P, hq, d, generator=g).to(torch.bfloat16)
    qo = torch.arange(0, B * P + 1, P, dtype=torch.int32)
    out = ops.paged_prefill(q.to(DEV), qo.to(DEV), P, pk["pool_k"], pk["pool_v"], pk["indptr"],
                            pk["indices"], pk["lpl"], 1 / math.sqrt(d), causal=True)
    assert bool(torch.isfinite(out).all())
    out = out.cpu()
    for b in (0, 1, 17, 31, 32, 45, 62, 63):
        ref = attend_sequences([q[b * P:(b + 1) * P]], [sequence_kv(pk, b, "k")],
                               [sequence_kv(pk, b, "v")])[0]
        torch.testing.assert_close(out[b * P:(b + 1) * P], ref, **BF16_TOL)


def test_bad_page_id_sets_status_without_fault():
    pk = make_paged([40, 40], 8, 128, 64, torch.bfloat16, DEV, seed=1)
    bad = pk["indices"].clone()
    bad[1] = 10 ** 6                                      # outside the 64-page pool
    q = torch.randn(2, 32, 128, device=DEV).to(torch.bfloat16)
    ops.paged_decode(q, pk["pool_k"], pk["pool_v"], pk["indptr"], bad, pk["lpl"], 0.1)
    with pytest.raises(RuntimeError, match="page id outside the pool"):
        ops.check_device_status(DEV)
    ops.paged_prefill(q[:, None], torch.tensor([0, 1, 2], dtype=torch.int32, device=DEV), 1,
                      pk["pool_k"], pk["pool_v"], pk["indptr"], bad, pk["lpl"], 0.1)
    with pytest.raises(RuntimeError, match="page id outside the pool"):
        ops.check_device_status(DEV)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_silu_mul_matches_reference_ops(dt):
    g = torch.Generator().manual_seed(12)
    gu = (torch.randn(37, 2 * 1024, generator=g) * 3).to(dt).to(DEV)
    out = ops.silu_mul(gu)
    ref = torch.nn.functional.silu(gu[:, :1024]) * gu[:, 1024:]     # models.py:156-157
    tol = dict(rtol=1e-2, atol=1e-2) if dt == torch.bfloat16 else dict(rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(out, ref, **tol)


def test_fused_projections_match_separate_layers():
    """One stacked q/k/v GEMM and one gate/up GEMM + silu*mul give the same block output
    as the reference's separate projections (bf16, GEMM rounding tolerance)."""
    from nanoslg_b200 import models
    from nanoslg_b200.kv_cache import B200PagedKVCache, KVCacheConfig
    from nanoslg_b200.parallel import ParallelConfig, ParallelContext, ParallelMode
    from nanoslg_b200.runner import llama_config
    hf = llama_config("tiny")
    pc = ParallelConfig(ParallelMode.TENSOR, 1)
    ParallelContext.initialize(pc, 0, device=DEV)
    m = models.init_random_(models.create_model(hf, pc)).to(DEV).to(torch.bfloat16)
    ids = torch.randint(0, 1024, (3, 20), device=DEV)
    outs = []
    for fused in (False, True):
        if fused:
            models.fuse_projections(m)
        cfg = KVCacheConfig(num_layers=2, num_kv_heads=2, num_qo_heads=4, head_dim=64,
                            page_size=16, max_pages=32, dtype=torch.bfloat16, device=DEV)
        mgr = B200PagedKVCache(cfg)
        for i in range(3):
            mgr.allocate_sequence(f"s{i}")
        ctx = mgr.begin_forward(["s0", "s1", "s2"], [20, 20, 20], [0, 0, 0])
        with torch.inference_mode():
            outs.append(m(ids, ctx).float())
    assert models._views_intact(m.layers[0].mlp._gu, [m.layers[0].mlp.gate_proj,
                                                      m.layers[0].mlp.up_proj])
    torch.testing.assert_close(outs[1], outs[0], rtol=2e-2, atol=2e-2)


def test_rope_kv_append_reports_bad_position_and_slot():
    """A position outside the cos/sin table and a write slot outside the pool are not
    accessed: the token is copied unrotated / not written, and the status word names
    both errors (the call itself succeeds; the GPU never faults)."""
    bf = torch.bfloat16
    hq, hkv, d, ps, P = 8, 2, 128, 16, 4
    g = torch.Generator().manual_seed(23)
    cos, sin = rope_table(d, 64, 500000.0)
    q = torch.randn(4, hq, d, generator=g).to(bf)
    k = torch.randn(4, hkv, d, generator=g).to(bf)
    v = torch.randn(4, hkv, d, generator=g).to(bf)
    pos = torch.tensor([3, 64, 5, 7], dtype=torch.int32)        # 64: one past the table
    loc = torch.tensor([0, 1, P * ps + 5, 2], dtype=torch.int32)  # token 2: past the pool
    pk = torch.zeros((P, ps, hkv, d), dtype=bf, device=DEV)
    pv = torch.zeros_like(pk)
    q_out = ops.rope_kv_append(q.to(DEV), k.to(DEV), v.to(DEV), pos.to(DEV), cos.to(DEV),
                               sin.to(DEV), loc.to(DEV), pk, pv)
    with pytest.raises(RuntimeError) as err:
        ops.check_device_status(DEV)
    assert "position outside the RoPE table" in str(err.value)
    assert "write slot outside the pool" in str(err.value)
    ok = torch.tensor([0, 2, 3])
    p64 = pos.long()[ok][None]
    assert torch.equal(q_out.cpu()[ok], apply_rotary(q[ok][None], cos[p64], sin[p64])[0])
    assert torch.equal(q_out.cpu()[1], q[1])                    # left unrotated
    fk = pk.view(-1, hkv, d).cpu()
    assert torch.equal(fk[[0, 2]], apply_rotary(k[[0, 3]][None], cos[pos.long()[[0, 3]]][None],
                                                sin[pos.long()[[0, 3]]][None])[0])
    assert torch.equal(fk[1], k[1])
    assert int((fk[3:] != 0).sum()) == 0


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_argmax_rows_matches_torch(dt):
    """nslg_argmax_rows against torch.argmax: first index of the maximum, NaN above every
    number, all -inf rows to index 0; vector and scalar (odd column count) paths, row
    strides, the shard offset and the returned maxima."""
    g = torch.Generator().manual_seed(31)
    for rows, cols in ((64, 128256), (1, 128256), (5, 1003), (3, 7), (2, 40000)):
        x = (torch.randn(rows, cols, generator=g) * 4).to(dt)
        if rows > 2:
            x[1, cols // 3] = x[1, 2 * cols // 3] = x[1].max() + 1        # tie: first wins
            x[2] = float("-inf")
        if rows > 3:
            x[3, cols - 1] = float("nan")
            x[3, cols // 2] = float("nan")
            x[4, :] = x[4, 0]                                               # all equal
        xd = x.to(DEV)
        idx = ops.argmax_rows(xd).cpu()
        assert torch.equal(idx, x.argmax(-1)), (rows, cols)
        idx2, val = ops.argmax_rows(xd, index_offset=1000, values=True)
        assert torch.equal(idx2.cpu(), x.argmax(-1) + 1000)
        ref = x.float().gather(1, x.argmax(-1, keepdim=True))[:, 0]
        assert torch.equal(val.cpu(), ref) or torch.allclose(val.cpu(), ref, equal_nan=True)
    # a strided view: the last position of [B, S, V] logits
    x = torch.randn(4, 3, 1000, generator=g).to(dt)
    assert torch.equal(ops.argmax_rows(x.to(DEV)[:, -1]).cpu(), x[:, -1].argmax(-1))
