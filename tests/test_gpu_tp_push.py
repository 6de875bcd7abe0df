"""The RowParallel product fused with the push of its partial rows to the peers
(nslg_linear_tp_push) and the reduction that then only gathers, sums and normalises
(nslg_tp_reduce_pushed_rmsnorm), with every rank of a TP group emulated on ONE GPU.

Each emulated rank has its own stage buffer, call counters, partial and residual, all in
this GPU's memory; the "peer mappings" are the other ranks' buffers themselves. All the
ranks' fused products run first (each pushes its rows into the other ranks' buffers),
then all the ranks' reductions: every word a reduction polls for has been written by a
kernel that already finished, so no kernel waits on one that has not run. This checks
the whole protocol -- packing, call numbers, slots, source regions, row layout -- on one
GPU: each partial against a torch fp32 product (bf16 tolerance), the new residual
bit-exact against the fp32 rank-order sum of the partials (the reference's
RowParallelLinear all-reduce + residual add, tp_layers.py:148-158, models.py:169-172),
the RMSNorm output within one rounding, over consecutive calls that alternate the two
stage slots."""
import ctypes

import pytest
import torch

from nanoslg_b200 import _native as N
from nanoslg_b200 import ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
EPS = 1e-5


@pytest.fixture(autouse=True)
def _clean_status():
    ops.status_word(DEV).zero_()
    yield
    ops.check_device_status(DEV)


def _expected(parts, res, w):
    s = parts[0].float()
    for p in parts[1:]:
        s = s + p.float()
    s = s.to(res.dtype)
    h = (res.float() + s.float()).to(res.dtype)
    hf = h.float()
    y = (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + EPS)).to(res.dtype)
    return h, (w.float() * y.float()).to(res.dtype)


def _close(a, b):
    return bool(((a.float() - b.float()).abs() <= b.float().abs() * 2 ** -7 + 1e-6).all())


@pytest.mark.parametrize("world,hidden,k_rank,rows_seq", [
    (2, 4096, 2048, [1, 16, 5]),        # o_proj of the 8B model at TP=2 (4 K splits)
    (4, 4096, 3584, [16, 1, 9]),        # down_proj at TP=4 (4 K splits)
    (8, 4096, 512, [1, 16, 16, 3]),     # o_proj at TP=8 (whole tiles)
    (8, 1024, 192, [7, 64]),            # a narrow row, three K chunks, up to 64 rows
])
def test_fused_push_and_reduce_emulated_ranks(world, hidden, k_rank, rows_seq):
    lib = N.lib()
    bf = torch.bfloat16
    status = ops.status_word(DEV)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    max_rows = max(rows_seq)
    stage_bytes = 4 * world * max_rows * hidden * 2
    stages = [torch.zeros(stage_bytes, dtype=torch.uint8, device=DEV) for _ in range(world)]
    arr = (ctypes.c_void_p * world)(*[s.data_ptr() for s in stages])
    counters = [torch.zeros(N.TP_COUNTER_BYTES // 4, dtype=torch.int32, device=DEV)
                for _ in range(world)]
    g = torch.Generator(device=DEV).manual_seed(world * 100 + hidden)
    for call, rows in enumerate(rows_seq):
        xs = [torch.randn(rows, k_rank, generator=g, device=DEV).to(bf) for _ in range(world)]
        ws = [(torch.randn(hidden, k_rank, generator=g, device=DEV) / k_rank ** 0.5).to(bf)
              for _ in range(world)]
        res0 = torch.randn(rows, hidden, generator=g, device=DEV).to(bf)
        nw = (1 + 0.1 * torch.randn(hidden, generator=g, device=DEV)).to(bf)
        parts = [torch.empty(rows, hidden, dtype=bf, device=DEV) for _ in range(world)]
        for r in range(world):
            rc = lib.nslg_linear_tp_push(
                N.DTYPE_BF16, rows, hidden, k_rank, xs[r].data_ptr(), k_rank,
                ws[r].data_ptr(), k_rank, parts[r].data_ptr(), hidden, world, r,
                ctypes.cast(arr, ctypes.c_void_p), stage_bytes, counters[r].data_ptr(),
                status.data_ptr(), stream)
            assert rc == N.OK, lib.nslg_last_error()
        resid = [res0.clone() for _ in range(world)]
        outs = [torch.empty(rows, hidden, dtype=bf, device=DEV) for _ in range(world)]
        for r in range(world):
            rc = lib.nslg_tp_reduce_pushed_rmsnorm(
                N.DTYPE_BF16, rows, hidden, world, r, parts[r].data_ptr(), hidden,
                ctypes.cast(arr, ctypes.c_void_p), stage_bytes, counters[r].data_ptr(),
                resid[r].data_ptr(), hidden, nw.data_ptr(), outs[r].data_ptr(), hidden,
                EPS, 2_000_000_000, status.data_ptr(), stream)
            assert rc == N.OK, lib.nslg_last_error()
        torch.cuda.synchronize(DEV)
        assert int(status.item()) == 0, f"device status {int(status.item()):#x} at call {call}"
        for r in range(world):
            want = (xs[r].float() @ ws[r].float().t()).to(bf)
            torch.testing.assert_close(parts[r], want, rtol=8e-3, atol=8e-3)
        h_want, o_want = _expected(parts, res0, nw)
        for r in range(world):
            assert torch.equal(resid[r], h_want), f"rank {r} residual, call {call}"
            assert _close(outs[r], o_want), f"rank {r} norm output, call {call}"
        for r in range(world):
            assert int(counters[r][0].item()) == call + 1      # one reduction call per call


def test_fused_push_rejects_what_it_does_not_cover():
    lib = N.lib()
    x = torch.zeros(4, 128, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(1000, 128, dtype=torch.bfloat16, device=DEV)   # 1000 % 8 == 0
    y = torch.zeros(4, 1000, dtype=torch.bfloat16, device=DEV)
    st = torch.zeros(1 << 16, dtype=torch.uint8, device=DEV)
    arr = (ctypes.c_void_p * 2)(st.data_ptr(), st.data_ptr())
    cnt = torch.zeros(256, dtype=torch.int32, device=DEV)
    s = torch.cuda.current_stream(DEV).cuda_stream
    call = lambda world, rank, ob, nbytes: lib.nslg_linear_tp_push(
        N.DTYPE_BF16, 4, 1000, 128, x.data_ptr(), 128, w.data_ptr(), 128, y.data_ptr(), 1000,
        world, rank, ctypes.cast(arr, ctypes.c_void_p), nbytes, cnt.data_ptr(), None, s)
    assert call(1, 0, None, 1 << 16) == N.ERR_ARG                   # world < 2
    assert call(2, 2, None, 1 << 16) == N.ERR_ARG                   # rank out of range
    assert call(2, 0, None, 1024) == N.ERR_WORKSPACE                # rows do not fit
    assert b"fit" in lib.nslg_last_error()


def _emulated_call(world, rows, hidden, parts, stages, stage_bytes, counters, resid, nw, outs,
                   timeout_ns=2_000_000_000):
    lib = N.lib()
    P = ctypes.c_void_p * world
    rc = lib.nslg_tp_allreduce_rmsnorm_emulated(
        N.DTYPE_BF16, rows, hidden, world,
        ctypes.cast(P(*[t.data_ptr() for t in parts]), ctypes.c_void_p), hidden,
        ctypes.cast(P(*[s.data_ptr() for s in stages]), ctypes.c_void_p), stage_bytes,
        ctypes.cast(P(*[c.data_ptr() for c in counters]), ctypes.c_void_p),
        ctypes.cast(P(*[r.data_ptr() for r in resid]), ctypes.c_void_p), hidden,
        nw.data_ptr(), ctypes.cast(P(*[o.data_ptr() for o in outs]), ctypes.c_void_p), hidden,
        EPS, timeout_ns, ops.status_word(DEV).data_ptr(),
        torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == N.OK, lib.nslg_last_error()


@pytest.mark.parametrize("world,mode", [(2, "0"), (4, "0"), (4, "1"), (8, "0"), (8, "1"),
                                        (8, "auto")])
def test_reduction_protocol_emulated_group_one_gpu(world, mode, monkeypatch):
    """The reduction kernel with every rank of a TP group in one cooperative grid on one
    GPU (nslg_tp_allreduce_rmsnorm_emulated): the one-shot push and the two-shot
    reduce-scatter + all-gather, on consecutive calls that alternate the stage slots and
    change the row count. The new residual must be bit-exact against the fp32 rank-order
    sum on every rank, the norm output within one rounding."""
    monkeypatch.setenv("NSLG_TP_TWO_SHOT", mode)
    hidden, bf = 4096, torch.bfloat16
    rows_seq = [64, 1, 17, 64, 5]
    stage_bytes = 4 * world * max(rows_seq) * hidden * 2
    stages = [torch.zeros(stage_bytes, dtype=torch.uint8, device=DEV) for _ in range(world)]
    counters = [torch.zeros(N.TP_COUNTER_BYTES // 4, dtype=torch.int32, device=DEV)
                for _ in range(world)]
    g = torch.Generator(device=DEV).manual_seed(world * 10 + len(mode))
    for call, rows in enumerate(rows_seq):
        parts = [torch.randn(rows, hidden, generator=g, device=DEV).to(bf) for _ in range(world)]
        res0 = torch.randn(rows, hidden, generator=g, device=DEV).to(bf)
        nw = (1 + 0.1 * torch.randn(hidden, generator=g, device=DEV)).to(bf)
        resid = [res0.clone() for _ in range(world)]
        outs = [torch.empty(rows, hidden, dtype=bf, device=DEV) for _ in range(world)]
        _emulated_call(world, rows, hidden, parts, stages, stage_bytes, counters, resid, nw,
                       outs)
        torch.cuda.synchronize(DEV)
        assert int(ops.status_word(DEV).item()) == 0, f"status at call {call}"
        h_want, o_want = _expected(parts, res0, nw)
        for r in range(world):
            assert torch.equal(resid[r], h_want), f"rank {r} residual, call {call}"
            assert _close(outs[r], o_want), f"rank {r} norm output, call {call}"
