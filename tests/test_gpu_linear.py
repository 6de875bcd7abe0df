"""The tcgen05 linear layer of decode steps (nslg_linear, ops.linear) against a plain
torch fp32 reference of the same product, y = x . W^T rounded once to the activation
type, at the shapes the Llama-3.1-8B decode step runs per layer and rank (TP = 1 and 8),
the LM head, ragged tiles, and through CUDA-graph replay.

Tolerance: the fp32 sums differ from the reference's only in order, so y is within one
rounding of the activation type (bf16 2^-8, fp16 2^-11 relative) plus a small absolute
floor for outputs near zero."""
import pytest
import torch

from nanoslg_b200 import _native as N
from nanoslg_b200 import ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
TOL = {torch.bfloat16: dict(rtol=8e-3, atol=8e-3), torch.float16: dict(rtol=2e-3, atol=2e-3)}


@pytest.fixture(autouse=True)
def _clean_status():
    ops.status_word(DEV).zero_()
    yield
    ops.check_device_status(DEV)


def _problem(m, n, k, dt, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(m, k, device=DEV, generator=g).to(dt)
    w = (torch.randn(n, k, device=DEV, generator=g) / k ** 0.5).to(dt)
    return x, w


def _ref(x, w):
    return (x.float() @ w.float().t()).to(x.dtype)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", [
    (64, 6144, 4096),      # stacked q|k|v, TP=1
    (64, 4096, 4096),      # o_proj, TP=1
    (64, 28672, 4096),     # stacked gate|up, TP=1
    (64, 4096, 14336),     # down_proj, TP=1
    (1, 4096, 4096),       # batch 1
    (64, 768, 4096),       # q|k|v at TP=8
    (64, 4096, 512),       # o_proj at TP=8
    (64, 4096, 1792),      # down_proj at TP=8
    (17, 1000, 512),       # ragged rows and a partial last tile
    (256, 640, 128),       # the largest row count, few chunks per tile
])
def test_linear_matches_fp32_reference(dt, m, n, k):
    x, w = _problem(m, n, k, dt, seed=m * 7 + n + k)
    y = ops.linear(x, w, max_rows=ops.LINEAR_MAX_ROWS)
    assert ops.linear_supported(x, w)
    torch.testing.assert_close(y, _ref(x, w), **TOL[dt])
    # deterministic: the split-K partials are summed in a fixed order
    assert torch.equal(ops.linear(x, w, max_rows=ops.LINEAR_MAX_ROWS), y)


def test_linear_lm_head_on_a_strided_last_position():
    """The LM head on the last position of [B, S, hidden] (a strided view) at the TP=8
    vocabulary shard (128256 / 8 = 16032 rows: a partial last tile)."""
    dt = torch.bfloat16
    g = torch.Generator(device=DEV).manual_seed(5)
    h = torch.randn(8, 3, 4096, device=DEV, generator=g).to(dt)
    w = (torch.randn(16032, 4096, device=DEV, generator=g) / 64).to(dt)
    last = h[:, -1]
    y = ops.linear(last, w, max_rows=ops.LINEAR_MAX_ROWS)
    torch.testing.assert_close(y, _ref(last.contiguous(), w), **TOL[dt])


@pytest.mark.parametrize("m,n,k", [(17, 1001, 512), (5, 4093, 1792), (64, 3000, 4096)])
@pytest.mark.parametrize("pad", [0, 3])
def test_linear_output_rows_unaligned_or_ragged(m, n, k, pad):
    """y written into rows of stride n + pad (pad 3: no row starts on a 16-byte
    boundary, so every store is element-wise) with out_features not a multiple of 4 or
    8 (the last vector of a row is cut at out_features), for whole tiles (n = 1001,
    3000) and cluster-split tiles (4093 x 1792); nothing past out_features is written."""
    dt = torch.bfloat16
    x, w = _problem(m, n, k, dt, seed=m + n + pad)
    buf = torch.full((m, n + pad), 7.0, dtype=dt, device=DEV)
    y = buf[:, :n]
    ops.linear(x, w, out=y, max_rows=ops.LINEAR_MAX_ROWS)
    torch.testing.assert_close(y, _ref(x, w), **TOL[dt])
    assert bool((buf[:, n:] == 7.0).all())
    assert torch.equal(y, ops.linear(x, w, max_rows=ops.LINEAR_MAX_ROWS))


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("splits", [2, 3, 5, 6, 7, 8])
@pytest.mark.parametrize("m", [1, 17, 64, 100])
def test_linear_pushed_and_pulled_split_sums_agree(dt, splits, m, monkeypatch):
    """The two ways of summing a tile's K splits inside its cluster -- partials pushed
    into the owning CTA's shared memory (st.async on its mbarrier; up to 64 rows where
    the receive buffer fits) and partials staged and pulled through distributed shared
    memory between cluster barriers (NSLG_LINEAR_PUSH_SUM=0, and past 64 rows) -- add
    the same fp32 values in the same order: bit-identical outputs, at every split count
    (uneven row shares at 3, 5, 6, 7) and a ragged last tile."""
    x, w = _problem(m, 1000, 1024, dt, seed=splits * 100 + m)
    monkeypatch.setenv("NSLG_LINEAR_SPLITS", str(splits))
    pushed = ops.linear(x, w, max_rows=ops.LINEAR_MAX_ROWS)
    monkeypatch.setenv("NSLG_LINEAR_PUSH_SUM", "0")
    pulled = ops.linear(x, w, max_rows=ops.LINEAR_MAX_ROWS)
    assert torch.equal(pushed, pulled)
    torch.testing.assert_close(pushed, _ref(x, w), **TOL[dt])


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,inter,k", [
    (1, 14336, 4096),      # TP=1: whole tiles
    (16, 7168, 4096),      # TP=2: 2-way K split
    (5, 3584, 4096),       # TP=4
    (64, 1792, 4096),      # TP=8: 8-way split, 64 rows
    (3, 1000, 512),        # ragged: the last tile has 40 gate|up pairs
    (100, 512, 1024),      # past 64 rows with a K split: the kernel declines, two kernels run
])
def test_linear_swiglu_matches_linear_then_silu_mul(dt, m, inter, k):
    """The gate|up product with SwiGLU in the kernel's epilogue gives exactly the values of
    the product (rounded) followed by the silu*mul kernel, and is within one rounding of
    the torch fp32 reference of silu(x.gate) * (x.up)."""
    x, w = _problem(m, 2 * inter, k, dt, seed=m + inter + k)
    fused = ops.linear_swiglu(x, w, max_rows=ops.LINEAR_MAX_ROWS)
    two = ops.silu_mul(ops.linear(x, w, max_rows=ops.LINEAR_MAX_ROWS))
    assert fused.shape == (m, inter)
    assert torch.equal(fused, two)
    g = (x.float() @ w[:inter].float().t()).to(dt).float()
    u = (x.float() @ w[inter:].float().t()).to(dt).float()
    ref = (torch.nn.functional.silu(g).to(dt).float() * u).to(dt)
    torch.testing.assert_close(fused, ref, **TOL[dt])


@pytest.mark.parametrize("splits", [3, 5, 6, 7])
@pytest.mark.parametrize("m", [1, 64])
def test_linear_swiglu_uneven_split_shares(splits, m, monkeypatch):
    """Forced K splits whose shares of a tile's 64 gate|up pairs are uneven: each owner
    sums its gate rows and the matching up rows; equal to the two-kernel path (which
    splits the same way), or the two-kernel path itself where the push does not fit."""
    monkeypatch.setenv("NSLG_LINEAR_SPLITS", str(splits))
    x, w = _problem(m, 2 * 1000, 1024, torch.bfloat16, seed=splits + m)
    fused = ops.linear_swiglu(x, w, max_rows=ops.LINEAR_MAX_ROWS)
    assert torch.equal(fused, ops.silu_mul(ops.linear(x, w, max_rows=ops.LINEAR_MAX_ROWS)))


def test_linear_graph_replay():
    dt = torch.bfloat16
    x, w = _problem(64, 4096, 4096, dt, seed=11)
    y = torch.empty(64, 4096, dtype=dt, device=DEV)
    ops.linear(x, w, out=y, max_rows=ops.LINEAR_MAX_ROWS)
    torch.cuda.synchronize(DEV)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ops.linear(x, w, out=y, max_rows=ops.LINEAR_MAX_ROWS)
    for seed in (12, 13):
        x2, _ = _problem(64, 4096, 4096, dt, seed=seed)
        x.copy_(x2)
        graph.replay()
        torch.cuda.synchronize(DEV)
        torch.testing.assert_close(y, _ref(x2, w), **TOL[dt])
    del graph


def test_linear_products_of_different_shapes_back_to_back():
    """Calls of different shapes (whole tiles and cluster-split tiles) back to back,
    each overlapping the previous one's tail (programmatic dependent launch)."""
    dt = torch.bfloat16
    shapes = [(17, 1000, 512), (8, 16032, 4096), (64, 4096, 512), (64, 28672, 4096),
              (1, 640, 128)]
    probs = [_problem(m, n, k, dt, seed=i) for i, (m, n, k) in enumerate(shapes)]
    for _ in range(3):
        for x, w in probs:
            torch.testing.assert_close(ops.linear(x, w, max_rows=ops.LINEAR_MAX_ROWS),
                                       _ref(x, w), **TOL[dt])


def test_linear_refuses_what_it_does_not_cover():
    x = torch.zeros(300, 128, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(256, 128, dtype=torch.bfloat16, device=DEV)
    assert not ops.linear_supported(x, w)                       # too many rows: cuBLAS
    assert not ops.linear_supported(x[:8, :100], w[:, :100])    # K not a multiple of 64
    assert not ops.linear_supported(x[:8].float(), w.float())   # fp32: cuBLAS
    lib = N.lib()
    rc = lib.nslg_linear(N.DTYPE_BF16, 300, 256, 128, x.data_ptr(), 128, w.data_ptr(), 128,
                         x.data_ptr(), 256, None, torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == N.ERR_UNSUPPORTED and b"rows" in lib.nslg_last_error()


@pytest.mark.parametrize("cps,minc", [(2, 8), (1, 2), (2, 2), (2, 1)])
@pytest.mark.parametrize("m,n,k", [(64, 6144, 4096), (1, 4096, 512), (16, 4096, 1792),
                                   (64, 768, 4096), (5, 1000, 192)])
def test_linear_split_policies(cps, minc, m, n, k, monkeypatch):
    """Other split rules (two CTAs per SM's worth of K splits, splits of 1 to 8 chunks,
    clusters up to 8): the same products within the same tolerance, still deterministic."""
    monkeypatch.setenv("NSLG_LINEAR_CTAS_PER_SM", str(cps))
    monkeypatch.setenv("NSLG_LINEAR_MIN_CHUNKS", str(minc))
    dt = torch.bfloat16
    x, w = _problem(m, n, k, dt, seed=m + n + k + cps + minc)
    y = ops.linear(x, w, max_rows=ops.LINEAR_MAX_ROWS)
    torch.testing.assert_close(y, _ref(x, w), **TOL[dt])
    assert torch.equal(ops.linear(x, w, max_rows=ops.LINEAR_MAX_ROWS), y)


def _rope_case(m, hq, hkv, k, dt, seed, pages=64):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(m, 1, k, device=DEV, generator=g).to(dt)
    w = (torch.randn((hq + 2 * hkv) * 128, k, device=DEV, generator=g) / k ** 0.5).to(dt)
    pool_k = torch.randn(pages, 16, hkv, 128, device=DEV, generator=g).to(dt)
    pool_v = torch.randn(pages, 16, hkv, 128, device=DEV, generator=g).to(dt)
    pos = torch.randint(0, 4000, (m,), device=DEV, generator=g).to(torch.int32)
    loc = torch.randperm(pages * 16, device=DEV, generator=g)[:m].to(torch.int32)
    inv = 1.0 / (500000.0 ** (torch.arange(0, 64, device=DEV).float() / 64))
    ang = torch.outer(torch.arange(4096, device=DEV).float(), inv)
    cos = torch.cat([ang.cos(), ang.cos()], -1).contiguous()
    sin = torch.cat([ang.sin(), ang.sin()], -1).contiguous()
    return x, w, pool_k, pool_v, pos, loc, cos, sin


def _rope_two_kernels(x, w, hq, hkv, pos, loc, cos, sin, pool_k, pool_v):
    qkv = ops.linear(x, w, max_rows=ops.LINEAR_MAX_ROWS)
    q = qkv[..., :hq * 128].view(-1, hq, 128)
    kk = qkv[..., hq * 128:(hq + hkv) * 128].view(-1, hkv, 128)
    v = qkv[..., (hq + hkv) * 128:].view(-1, hkv, 128)
    return ops.rope_kv_append(q, kk, v, pos, cos, sin, loc, pool_k, pool_v)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,hq,hkv,k", [
    (1, 32, 8, 4096),      # TP=1: 48 heads, 4-way K split
    (16, 16, 4, 4096),     # TP=2
    (5, 4, 1, 4096),       # TP=8 shard: 6 heads, 8-way split
    (64, 8, 2, 1024),      # 64 rows
    (3, 2, 2, 128),        # 2 chunks: whole tiles
])
def test_linear_rope_append_matches_linear_then_rope_kv_append(dt, m, hq, hkv, k):
    """The q|k|v product with RoPE and the paged KV append in its epilogue writes exactly
    what the product (rounded) followed by rope_kv_append writes: the rotated q, and the
    rotated k and plain v in the pool slots."""
    x, w, pk, pv, pos, loc, cos, sin = _rope_case(m, hq, hkv, k, dt, seed=m + hq + k)
    pk2, pv2 = pk.clone(), pv.clone()
    q_fused = ops.linear_rope_append(x, w, hq, hkv, pos, cos, sin, loc, pk, pv,
                                     max_rows=ops.LINEAR_MAX_ROWS)
    assert q_fused is not None
    q_two = _rope_two_kernels(x, w, hq, hkv, pos, loc, cos, sin, pk2, pv2)
    assert torch.equal(q_fused, q_two)
    assert torch.equal(pk, pk2) and torch.equal(pv, pv2)


def test_linear_rope_append_out_of_range_positions_and_slots():
    """A position outside the cos/sin table leaves that token unrotated and sets the
    position bit of the status word; a write slot < 0 is skipped, one past the pool sets
    the slot bit and is skipped -- as rope_kv_append does."""
    x, w, pk, pv, pos, loc, cos, sin = _rope_case(4, 8, 2, 512, torch.bfloat16, seed=3)
    pos[1] = 5000                        # the table has 4096 rows
    loc[2] = -1
    loc[3] = pk.shape[0] * 16            # one past the last slot
    pk2, pv2 = pk.clone(), pv.clone()
    q_fused = ops.linear_rope_append(x, w, 8, 2, pos, cos, sin, loc, pk, pv,
                                     max_rows=ops.LINEAR_MAX_ROWS)
    st = int(ops.status_word(DEV).item())
    assert st & N.DEV_BAD_POSITION and st & N.DEV_BAD_SLOT
    ops.status_word(DEV).zero_()
    q_two = _rope_two_kernels(x, w, 8, 2, pos, loc, cos, sin, pk2, pv2)
    ops.status_word(DEV).zero_()
    assert torch.equal(q_fused, q_two)
    assert torch.equal(pk, pk2) and torch.equal(pv, pv2)


def test_linear_rope_append_declines_what_it_does_not_cover():
    """head_dim 64 and more rows than allowed: None, nothing launched (the caller runs the
    two kernels)."""
    x, w, pk, pv, pos, loc, cos, sin = _rope_case(2, 4, 2, 256, torch.bfloat16, seed=4)
    pk64 = torch.zeros(8, 16, 2, 64, dtype=torch.bfloat16, device=DEV)
    assert ops.linear_rope_append(x, w, 4, 2, pos, cos, sin, loc, pk64, pk64) is None
    assert ops.linear_rope_append(x, w, 4, 2, pos, cos, sin, loc, pk, pv, max_rows=1) is None
