"""The peer-memory TP reduction (nslg_tp_allreduce_rmsnorm, tp_comm.PeerAllReduce)
against a torch restatement of what it replaces: RowParallelLinear's SUM all-reduce
(tp_layers.py:148-158), the residual add and the next RMSNorm (models.py:169-172,
25-34).  The sum is taken in fp32 in rank order and rounded once, so the new residual
is bit-exact; the normalised output may differ by one rounding of the rsqrt."""
import ctypes
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT

pytestmark = pytest.mark.gpu

HIDDEN = 4096
EPS = 1e-5


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _expected(parts, res, w, eps):
    s = parts[0].float()
    for p in parts[1:]:
        s = s + p.float()
    s = s.to(res.dtype)
    h = (res.float() + s.float()).to(res.dtype)
    hf = h.float()
    inv = torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + eps)
    y = (hf * inv).to(res.dtype)
    return h, (w.float() * y.float()).to(res.dtype)


def _close(a, b):
    # one bf16 rounding step of slack for the rsqrt (2^-7 relative) plus a tiny floor
    return bool(((a.float() - b.float()).abs() <= b.float().abs() * 2 ** -7 + 1e-6).all())


def _peer_main(rank, world, port, out, mode="0"):
    import sys
    sys.path.insert(0, ROOT)
    os.environ["NSLG_TP_TWO_SHOT"] = mode
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device(f"cuda:{rank}")
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    res_out = {}
    try:
        from nanoslg_b200 import ops
        from nanoslg_b200.tp_comm import PeerAllReduce
        bf = torch.bfloat16
        peer = PeerAllReduce(dist.group.WORLD, rank, world, dev, 64, HIDDEN, bf)

        def data(it, rows):
            gp = torch.Generator(device=dev).manual_seed(1000 * it + rank)
            part = torch.randn(rows, HIDDEN, generator=gp, device=dev).to(bf)
            gs = torch.Generator(device=dev).manual_seed(99 + it)
            res = torch.randn(rows, HIDDEN, generator=gs, device=dev).to(bf)
            w = (1 + 0.1 * torch.randn(HIDDEN, generator=gs, device=dev)).to(bf)
            parts = [torch.empty_like(part) for _ in range(world)]
            dist.all_gather(parts, part)
            return part, res, w, parts

        # eager calls: changing row counts, both stage slots, with and without the norm
        ok = []
        for it, rows in enumerate([64, 1, 17, 64, 3, 40]):
            part, res, w, parts = data(it, rows)
            h_want, o_want = _expected(parts, res, w, EPS)
            r = res.clone()
            if it == 4:
                got = peer.allreduce_add_norm(part, r, None, EPS)
                ok.append(got is r and torch.equal(r, h_want))
            else:
                o = peer.allreduce_add_norm(part, r, w, EPS)
                ok.append(torch.equal(r, h_want) and _close(o, o_want))
        res_out["eager"] = ok

        # CUDA graph: two calls captured, replayed with fresh inputs each time
        rows = 64
        part_s = torch.zeros(rows, HIDDEN, dtype=bf, device=dev)
        res_s = torch.zeros_like(part_s)
        w_s = torch.ones(HIDDEN, dtype=bf, device=dev)
        part2_s = torch.zeros_like(part_s)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            o1 = peer.allreduce_add_norm(part_s, res_s, w_s, EPS)
            o2 = peer.allreduce_add_norm(part2_s, res_s, w_s, EPS)
        gok = []
        for it in range(10, 13):
            part, res, w, parts = data(it, rows)
            part2, _, _, parts2 = data(it + 100, rows)
            part_s.copy_(part)
            part2_s.copy_(part2)
            res_s.copy_(res)
            w_s.copy_(w)
            graph.replay()
            torch.cuda.synchronize(dev)
            h1, o1_want = _expected(parts, res, w, EPS)
            h2, o2_want = _expected(parts2, h1, w, EPS)
            gok.append(torch.equal(res_s, h2) and _close(o1, o1_want) and _close(o2, o2_want))
        res_out["graph"] = gok
        del graph
        ops.check_device_status(dev)
        peer.close()
        res_out["done"] = True
    finally:
        out[rank] = res_out
        dist.destroy_process_group()


@pytest.mark.parametrize("world,mode", [(2, "0"), (4, "0"), (8, "0"), (4, "1"), (8, "1"),
                                        (8, "auto")])
def test_peer_allreduce_rmsnorm(world, mode):
    """One-shot ("0"), two-shot ("1": reduce-scatter of column slices + all-gather) and
    the size-based choice ("auto", which mixes both over the test's row counts): the
    same bit-exact residual in every mode."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with mp.get_context("spawn").Manager() as m:
        out = m.dict()
        mp.start_processes(_peer_main, args=(world, _free_port(), out, mode), nprocs=world,
                           start_method="spawn", join=True)
        res = dict(out)
    for rank in range(world):
        r = res[rank]
        assert r.get("done"), f"rank {rank}: {r}"
        assert all(r["eager"]), f"rank {rank} eager: {r['eager']}"
        assert all(r["graph"]), f"rank {rank} graph: {r['graph']}"


def test_peer_wait_gives_up_with_status():
    """A peer that never stages its rows: the kernel's bounded wait runs out, the status
    word says so, the residual is left as it was and the context stays usable."""
    from nanoslg_b200 import _native as N
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    rows = 4
    bf = torch.bfloat16
    ptrs = []

    def alloc(n):
        p = ctypes.c_void_p()
        h = ctypes.create_string_buffer(N.IPC_HANDLE_BYTES)
        N.call("nslg_ipc_alloc", n, ctypes.byref(p), h)
        ptrs.append(p.value)
        return p.value

    stage_bytes = 4 * 2 * rows * HIDDEN * 2
    # rank 0 is this process; "rank 1" is a second local buffer that nobody writes to
    stages = (ctypes.c_void_p * 2)(alloc(stage_bytes), alloc(stage_bytes))
    counters = torch.zeros(N.TP_COUNTER_BYTES // 4, dtype=torch.int32, device=dev)
    try:
        part = torch.randn(rows, HIDDEN, device=dev).to(bf)
        res = torch.randn(rows, HIDDEN, device=dev).to(bf)
        keep = res.clone()
        w = torch.ones(HIDDEN, dtype=bf, device=dev)
        out = torch.empty_like(part)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        N.call("nslg_tp_allreduce_rmsnorm", N.DTYPE_BF16, rows, HIDDEN, 2, 0, part.data_ptr(),
               HIDDEN, ctypes.cast(stages, ctypes.c_void_p), stage_bytes,
               counters.data_ptr(), res.data_ptr(), HIDDEN, w.data_ptr(),
               out.data_ptr(), HIDDEN, EPS, 200_000_000, status.data_ptr(),
               torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize(dev)
        assert int(status.item()) & N.DEV_WAIT_TIMEOUT
        assert torch.equal(res, keep)
        # the context is still usable
        assert float((part.float() * 2).sum()) == pytest.approx(float(part.float().sum() * 2),
                                                                rel=1e-5)
    finally:
        torch.cuda.synchronize(dev)
        for p in ptrs:
            N.call("nslg_ipc_free", p)
