"""Benchmark of the per-layer paged decode-attention path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload C2: batch 64, 32 query / 8 KV heads, head_dim 128, page 16, per-sequence KV
lengths uniform in [512, 8192] (seed 0), page ids a random draw from a 600k-page pool
(one layer, 39.3 GB of K+V), q/K/V ~ N(0, 1).  A step is one decode-attention pass over
the batch (64 query tokens); the metric is decode tokens/s of that pass.

* ``value``     -- kernel path, inputs resident in HBM: ops.paged_decode (the C ABI
                   nslg_paged_decode: one split-KV kernel launch, split sequences
                   merged in-kernel by their last CTA), CUDA events on the
                   launching stream.  The 1.13 GB of KV read per step is 9x the 126 MB L2,
                   so no L2 flush is needed between steps.
* ``e2e``       -- the same decode step through the reference-facing API:
                   manager.begin_forward -> CacheContext.attend -> end_forward, with q/k/v
                   copied from pinned host memory and the output read back every step;
                   two steps in flight with the copies on copy streams (``e2e.serial``:
                   one step at a time on one stream).
* ``roofline``  -- algorithmic bytes per step / mean step time vs the measured HBM copy
                   bandwidth (MEASURED_PEAKS.json).
* ``cpu_baseline`` / ``--impl reference`` -- the reference's contiguous-SDPA attend
                   (restated in oracle/attention.py) on the host cores.

N > 1 (torchrun): every rank runs its own independent C2 batch (weak scaling, no
collective on the data path); ``value`` is the sum over ranks of tokens / the slowest
rank's time.

Beside the headline, the same line carries, at every N:

* ``parity``          -- the sharded path checked in this run: greedy tokens of a tiny
                         fp32 Llama (8/8 heads) at TP=N and TP=N/2 x PP=2 (eager and CUDA
                         graphs, lock step and 2 micro-batches) against tokens recorded from
                         the reference, and the fused peer reduction bit-exact (N > 1);
* ``llama8b_decode``  -- the Llama-3.1-8B-shaped model's decode at TP=N, batch 64 and 1,
                         with a per-category split of a step (GEMM / attention / TP
                         reduction / other) naming the limiter, and at N > 1 the TP=1 figure
                         of the same batch measured on rank 0 alone (strong scaling);
* ``cpu_baseline``    -- rank 0's host cores running the reference's attend.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, HQ, HKV, D, PS = 64, 32, 8, 128, 16
POOL_PAGES = 600_000
LEN_LO, LEN_HI = 512, 8192
FALLBACK_HBM_GBS = 6650.0


def c2_lens(seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(LEN_LO, LEN_HI + 1, (B,), generator=g).tolist()


def alg_bytes(lens):
    """Bytes a decode step must move: K and V of every cached token, q in, out, the page
    ids and the small CSR arrays."""
    pages = sum(math.ceil(n / PS) for n in lens)
    kv = sum(lens) * HKV * D * 2 * 2
    return kv + 2 * B * HQ * D * 2 + 4 * pages + 4 * (2 * B + 1)


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.out, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        self.out.flush()
        try:
            rows = [r.split(",") for r in open(self.out.name).read().strip().splitlines()]
        except Exception:
            rows = []
        os.unlink(self.out.name)
        rows = [[c.strip() for c in r] for r in rows if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


# ---------------------------------------------------------------------------- ours
def build_c2_device(device, seed, pool_pages=POOL_PAGES):
    """Pool [600k, 16, 8, 128] x2 bf16 ~ N(0,1), page table drawn from randperm(600k)."""
    lens = c2_lens(seed)
    npg = [math.ceil(n / PS) for n in lens]
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(pool_pages, generator=g)
    perm = perm[perm != 0][:sum(npg)].to(torch.int32)
    indptr = torch.zeros(B + 1, dtype=torch.int32)
    indptr[1:] = torch.cumsum(torch.tensor(npg), 0).to(torch.int32)
    lpl = torch.tensor([n - (p - 1) * PS for n, p in zip(lens, npg)], dtype=torch.int32)
    gd = torch.Generator(device=device).manual_seed(seed)
    shape = (pool_pages, PS, HKV, D)
    pool_k = torch.empty(shape, dtype=torch.bfloat16, device=device)
    pool_v = torch.empty(shape, dtype=torch.bfloat16, device=device)
    for t in (pool_k, pool_v):
        for i in range(0, pool_pages, 50_000):      # bounded fp32 temporaries
            t[i:i + 50_000] = torch.randn(t[i:i + 50_000].shape, device=device, generator=gd)
    q = torch.randn(B, HQ, D, device=device, generator=gd).to(torch.bfloat16)
    return dict(lens=lens, pool_k=pool_k, pool_v=pool_v, indptr=indptr.to(device),
                indices=perm.to(device), lpl=lpl.to(device), q=q)


def run_kernel(device, steps, warmup, seed, pool_pages=POOL_PAGES):
    """The headline: C2 decode steps on resident inputs."""
    from nanoslg_b200 import ops
    c = build_c2_device(device, seed, pool_pages)
    out = torch.empty(B, HQ, D, dtype=torch.bfloat16, device=device)
    scale = 1.0 / math.sqrt(D)

    def step():
        ops.paged_decode(c["q"], c["pool_k"], c["pool_v"], c["indptr"], c["indices"], c["lpl"],
                         scale, out=out)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(device)
    ops.check_device_status(device)
    stream = torch.cuda.current_stream(device)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    with ClockSampler(device.index) as clk:
        ev[0].record(stream)
        for i in range(steps):
            step()
            ev[i + 1].record(stream)
        torch.cuda.synchronize(device)
    per = [ev[i].elapsed_time(ev[i + 1]) for i in range(steps)]
    total_ms = ev[0].elapsed_time(ev[-1])
    ops.check_device_status(device)
    res = dict(total_ms=total_ms, per_ms=per, lens=c["lens"], clocks=clk.summary())
    del c
    torch.cuda.empty_cache()
    return res


def pipelined(n, launch, finish, depth=1):
    """Runs ``launch(i)`` for steps i = 0..n-1 and ``finish(i)`` for each once ``depth``
    steps are in flight (depth 1: every step is finished before the next is launched;
    depth 2: step i+1 is launched before step i is finished), in step order."""
    for i in range(n):
        launch(i)
        if i - depth + 1 >= 0:
            finish(i - depth + 1)
    for j in range(max(n - depth + 1, 0), n):
        finish(j)


def run_e2e(device, steps, warmup, seed, depth=1):
    """Decode steps through B200PagedKVCache / CacheContext.attend with host buffers.

    Each step copies its q/k/v from pinned host memory to the device, plans, appends and
    attends, copies the output to pinned host memory and ends the forward; a step is
    finished when its output is on the host. ``depth`` 1 finishes every step before the
    next begins (one stream). ``depth`` 2 begins step i+1 before waiting for step i's
    output, and on a GPU moves the copies to two copy streams with a device input buffer
    and a host output buffer per step in flight: step i+1's inputs go up while step i's
    kernels run and step i's output comes down while step i+1's run, so the compute
    stream only runs the plan, append and attention kernels back to back. The kernels
    stay in step order on one stream (each step appends to the same sequences)."""
    from nanoslg_b200.kv_cache import B200PagedKVCache, KVCacheConfig
    lens = c2_lens(seed)
    cfg = KVCacheConfig(num_layers=1, num_kv_heads=HKV, num_qo_heads=HQ, head_dim=D,
                        page_size=PS, max_pages=POOL_PAGES, dtype=torch.bfloat16, device=device,
                        enable_prefix_caching=True)
    mgr = B200PagedKVCache(cfg)
    sids = [f"s{b}" for b in range(B)]
    for s, n in zip(sids, lens):
        mgr.allocate_sequence(s, None, num_tokens=n)
        mgr.seqs[s].num_tokens = n            # history already cached
    mgr.pool.flush_zero()
    gd = torch.Generator(device=device).manual_seed(seed)
    for t in (mgr.pool.k, mgr.pool.v):       # history values ~ N(0, 1)
        for i in range(0, POOL_PAGES, 50_000):
            t[0, i:i + 50_000] = torch.randn(t[0, i:i + 50_000].shape, device=device, generator=gd)
    g = torch.Generator().manual_seed(seed + 1)
    nbuf = 4
    # each step's q | k | v packed in one pinned host buffer, copied with one transfer
    # into the device buffer of its slot (one slot per step in flight)
    qn, kn = B * HQ * D, B * HKV * D
    hin = [torch.randn(qn + 2 * kn, generator=g).to(torch.bfloat16).pin_memory()
           for _ in range(nbuf)]
    din = [torch.empty(qn + 2 * kn, dtype=torch.bfloat16, device=device) for _ in range(depth)]
    qkv = [(d[:qn].view(B, 1, HQ, D), d[qn:qn + kn].view(B, 1, HKV, D),
            d[qn + kn:].view(B, 1, HKV, D)) for d in din]
    hout = [torch.empty(B, 1, HQ * D, dtype=torch.bfloat16).pin_memory() for _ in range(depth)]
    done = [torch.cuda.Event() for _ in range(depth)]
    stream = torch.cuda.current_stream(device)
    split = depth > 1 and device.type == "cuda"
    if split:
        cp_in, cp_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
        in_ready = [torch.cuda.Event() for _ in range(depth)]
        consumed = [torch.cuda.Event() for _ in range(depth)]
        keep = [None] * depth       # each slot's output, alive until its copy is finished
    stats = {"h2d": 0, "d2h": 0}

    def launch(i):
        s = i % depth
        q, k, v = qkv[s]
        if split:
            # the slot's previous step has finished reading its inputs (and the host has
            # read its output: ``pipelined`` finishes step i - depth before this launch)
            cp_in.wait_event(consumed[s])
            with torch.cuda.stream(cp_in):
                din[s].copy_(hin[i % nbuf], non_blocking=True)
            in_ready[s].record(cp_in)
            stream.wait_event(in_ready[s])
        else:
            din[s].copy_(hin[i % nbuf], non_blocking=True)
        ctx = mgr.begin_forward(sids, [1] * B)
        out = ctx.attend(0, q, k, v, HQ, HKV)
        if split:
            consumed[s].record(stream)
            cp_out.wait_event(consumed[s])
            with torch.cuda.stream(cp_out):
                hout[s].copy_(out, non_blocking=True)
            done[s].record(cp_out)
            keep[s] = out
        else:
            hout[s].copy_(out, non_blocking=True)
            done[s].record(stream)
        mgr.end_forward(ctx)      # the reference's order: begin, forward, end, read
        stats["h2d"] = q.numel() * 2 + k.numel() * 2 + v.numel() * 2 + ctx._plan_bytes
        stats["d2h"] = hout[0].numel() * 2

    def finish(i):
        done[i % depth].synchronize()     # step i's output is on the host

    pipelined(warmup, launch, finish, depth)
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    pipelined(steps, lambda i: launch(warmup + i), lambda i: finish(warmup + i), depth)
    e1.record(stream)      # every step's output is on the host by now
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1)
    del mgr
    torch.cuda.empty_cache()
    return dict(total_ms=ms, h2d=stats["h2d"], d2h=stats["d2h"])


# ------------------------------------------------------------------ prefill kernel
def c3_prefill_inputs(device, batch=64, prompt=512):
    """The C3 prefill prompts as one ragged batch: q [batch * prompt, 32, 128] and its
    qo_indptr, a pool holding every prompt's K/V (pages drawn from a permutation), the
    CSR page table and last-page lengths; seeded N(0, 1) bf16."""
    npg = -(-prompt // PS)
    pages = batch * npg + 1
    g = torch.Generator(device=device).manual_seed(7)
    pool_k = torch.randn(pages, PS, HKV, D, device=device, generator=g).to(torch.bfloat16)
    pool_v = torch.randn(pages, PS, HKV, D, device=device, generator=g).to(torch.bfloat16)
    indices = (torch.randperm(pages - 1, device=device, generator=g)[:batch * npg] + 1).int()
    indptr = torch.arange(0, batch * npg + 1, npg, device=device, dtype=torch.int32)
    lpl = torch.full((batch,), prompt - (npg - 1) * PS, device=device, dtype=torch.int32)
    qo = torch.arange(0, batch * prompt + 1, prompt, device=device, dtype=torch.int32)
    q = torch.randn(batch * prompt, HQ, D, device=device, generator=g).to(torch.bfloat16)
    return q, qo, pool_k, pool_v, indptr, indices, lpl


def _median_ms(fn, reps, warm=3):
    """Median CUDA-event time of ``fn`` over ``reps`` back-to-back calls, after ``warm``."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
    ev[0].record()
    for i in range(reps):
        fn()
        ev[i + 1].record()
    torch.cuda.synchronize()
    return statistics.median(ev[i].elapsed_time(ev[i + 1]) for i in range(reps))


def run_reference_backend(device, reps=20):
    """The reference's GPU attention backend, FlashInfer (kv_cache.py:704-705: one
    BatchDecodeWithPagedKVCacheWrapper and one BatchPrefillWithPagedKVCacheWrapper, NHD;
    planned as kv_cache.py:617-633 does, with the same CSR page table; run as
    kv_cache.py:650-654), on the C2 decode batch and the C3 prefill prompts, timed beside
    this repo's kernels on the same inputs. FlashInfer is the build installed in the image
    (library code, not part of this repository); its first call JIT-compiles or loads its
    kernels, outside the timing. Prefill is timed on the backend the reference gets
    (the wrapper's default) and on FlashInfer's TensorRT-LLM Blackwell kernels
    (backend "trtllm-gen", prebuilt), the fastest library prefill on this GPU."""
    try:
        import flashinfer
    except Exception as e:                 # not in this environment
        return {"unavailable": f"flashinfer not importable: {type(e).__name__}: {e}"}
    from nanoslg_b200 import ops
    hbm, _ = peaks()
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tpk = float(json.load(f)["bf16_tflops"])
    except Exception:
        tpk = 1590.0
    scale = 1.0 / math.sqrt(D)
    res = {"library": f"flashinfer {flashinfer.__version__}",
           "timing": f"median of {reps} back-to-back calls, CUDA events, eager launches"}
    ws = torch.empty(128 << 20, dtype=torch.uint8, device=device)
    c2 = None
    try:
        c2 = build_c2_device(device, 0)
        dec = flashinfer.BatchDecodeWithPagedKVCacheWrapper(ws, "NHD")
        dec.plan(c2["indptr"], c2["indices"], c2["lpl"], HQ, HKV, D, PS,
                 q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16)
        o_fi = dec.run(c2["q"], (c2["pool_k"], c2["pool_v"]))
        o_us = torch.empty_like(c2["q"])
        ops.paged_decode(c2["q"], c2["pool_k"], c2["pool_v"], c2["indptr"], c2["indices"],
                         c2["lpl"], scale, out=o_us)
        torch.cuda.synchronize()
        ab = alg_bytes(c2["lens"])
        fi_ms = _median_ms(lambda: dec.run(c2["q"], (c2["pool_k"], c2["pool_v"]), out=o_fi), reps)
        us_ms = _median_ms(lambda: ops.paged_decode(
            c2["q"], c2["pool_k"], c2["pool_v"], c2["indptr"], c2["indices"], c2["lpl"], scale,
            out=o_us), reps)
        res["c2_decode"] = {
            "flashinfer_ms": fi_ms, "ours_ms": us_ms, "speedup": fi_ms / us_ms,
            "flashinfer_hbm_frac": ab / (fi_ms / 1e3) / 1e9 / hbm,
            "ours_hbm_frac": ab / (us_ms / 1e3) / 1e9 / hbm,
            "max_abs_diff": float((o_fi.float() - o_us.float()).abs().max())}
        del o_fi, o_us, dec
    except Exception as e:
        res["c2_decode"] = {"error": f"{type(e).__name__}: {str(e)[:300]}"}
    del c2
    torch.cuda.empty_cache()
    q, qo, pool_k, pool_v, indptr, indices, lpl = c3_prefill_inputs(device)
    flops = 64 * 4 * HQ * D * (512 * 513 // 2)
    o_us = torch.empty_like(q)
    run_us = lambda: ops.paged_prefill(q, qo, 512, pool_k, pool_v, indptr, indices, lpl, scale,
                                       causal=True, out=o_us)
    us_ms = _median_ms(run_us, reps)
    for backend in ("auto", "trtllm-gen"):
        try:
            pf = flashinfer.BatchPrefillWithPagedKVCacheWrapper(ws, "NHD", backend=backend)
            pf.plan(qo, indptr, indices, lpl, HQ, HKV, D, PS, causal=True,
                    q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16)
            o_fi = pf.run(q, (pool_k, pool_v))
            torch.cuda.synchronize()
            fi_ms = _median_ms(lambda: pf.run(q, (pool_k, pool_v), out=o_fi), reps)
            res[f"c3_prefill_{backend}"] = {
                "flashinfer_ms": fi_ms, "ours_ms": us_ms, "speedup": fi_ms / us_ms,
                "flashinfer_tensor_frac": flops / (fi_ms / 1e3) / 1e12 / tpk,
                "ours_tensor_frac": flops / (us_ms / 1e3) / 1e12 / tpk,
                "max_abs_diff": float((o_fi.float() - o_us.float()).abs().max())}
            del o_fi, pf
        except Exception as e:
            res[f"c3_prefill_{backend}"] = {"error": f"{type(e).__name__}: {str(e)[:300]}"}
    del q, pool_k, pool_v, o_us, ws
    torch.cuda.empty_cache()
    return res


def run_prefill_kernel(device, reps=10, batch=64, prompt=512):
    """Causal prefill attention of the C3 batch-64 prompts (32/8 heads, D=128) on the
    tcgen05 kernel: algorithmic FLOPs = sum_b sum_i 4*Hq*D*(i+1) over the causal rows."""
    from nanoslg_b200 import ops
    q, qo, pool_k, pool_v, indptr, indices, lpl = c3_prefill_inputs(device, batch, prompt)
    out = torch.empty_like(q)
    scale = 1.0 / math.sqrt(D)

    def run():
        ops.paged_prefill(q, qo, prompt, pool_k, pool_v, indptr, indices, lpl, scale,
                          causal=True, out=out)

    for _ in range(3):
        run()
    torch.cuda.synchronize(device)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
    ev[0].record()
    for i in range(reps):
        run()
        ev[i + 1].record()
    torch.cuda.synchronize(device)
    per = [ev[i].elapsed_time(ev[i + 1]) for i in range(reps)]
    flops = batch * 4 * HQ * D * (prompt * (prompt + 1) // 2)
    ms = statistics.median(per)
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops"])
        src = "measured burst bf16_tflops"
    except Exception:
        peak, src = 1590.0, "fallback 1590 TFLOP/s"
    tf = flops / (ms / 1e3) / 1e12
    del pool_k, pool_v, q, out
    torch.cuda.empty_cache()
    return {"workload": f"causal prefill attention, batch {batch} x {prompt} tokens, 32/8 heads, "
                        "D=128, page 16 (C3 prompts)", "kernel": "prefill_tc_kernel (tcgen05)",
            "ms_median": ms, "tflops": tf, "peak_tflops": peak, "frac": tf / peak,
            "peak_source": src, "algorithmic_flops": flops}


def run_decode_model_shapes(device, reps=10, layers=32):
    """Decode attention at the Llama-3.1-8B model's decode shapes, as the model runs it:
    ``layers`` layers, each with its own pool (so no layer's K/V is still in L2 from the
    last), one decode call per layer captured back to back in a CUDA graph, replayed
    ``reps`` times (CUDA events). Cases: batch 64 with contexts U[512, 640] and batch 1
    with a 512-token context, at TP=1 (32/8 heads) and at the TP=8 shard (4/1 heads).
    Algorithmic bytes per layer: every cached K and V byte, q in, out, and the page ids.
    Each case is timed with the library's choice of how split sequences are combined, and
    with each of the two modes forced (in the decode kernel / by the merge kernel)."""
    from nanoslg_b200 import ops
    peak, src = _hbm_peak()
    g = torch.Generator().manual_seed(5)
    res = {}
    for name, batch, lo, hi, hq, hkv in (("tp1_batch64", 64, 512, 640, 32, 8),
                                         ("tp1_batch1", 1, 512, 512, 32, 8),
                                         ("tp8_batch64", 64, 512, 640, 4, 1),
                                         ("tp8_batch1", 1, 512, 512, 4, 1)):
        lens = torch.randint(lo, hi + 1, (batch,), generator=g).tolist()
        npg = [-(-n // PS) for n in lens]
        pages = sum(npg) + 1
        indptr = torch.tensor([0] + torch.cumsum(torch.tensor(npg), 0).tolist(),
                              dtype=torch.int32, device=device)
        lpl = torch.tensor([n - (p - 1) * PS for n, p in zip(lens, npg)], dtype=torch.int32,
                           device=device)
        pools = []
        for _ in range(layers):
            idx = (torch.randperm(pages - 1, generator=g)[:sum(npg)] + 1).to(torch.int32)
            pk = torch.randn(pages, PS, hkv, D, device=device).to(torch.bfloat16)
            pv = torch.randn(pages, PS, hkv, D, device=device).to(torch.bfloat16)
            pools.append((pk, pv, idx.to(device)))
        q = torch.randn(batch, hq, D, device=device).to(torch.bfloat16)
        outs = [torch.empty_like(q) for _ in range(layers)]
        scale = 1.0 / math.sqrt(D)

        def step():
            for (pk, pv, idx), o in zip(pools, outs):
                ops.paged_decode(q, pk, pv, indptr, idx, lpl, scale, out=o)

        def time_layers(mode):
            # mode None: the library's own choice of merge; "inline" / "kernel" force one
            # (the choice is made when the graph is captured)
            old = os.environ.pop("NSLG_DECODE_MERGE", None)
            if mode is not None:
                os.environ["NSLG_DECODE_MERGE"] = mode
            try:
                step()
                torch.cuda.synchronize(device)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    step()
            finally:
                os.environ.pop("NSLG_DECODE_MERGE", None)
                if old is not None:
                    os.environ["NSLG_DECODE_MERGE"] = old
            graph.replay()
            torch.cuda.synchronize(device)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                graph.replay()
            e1.record()
            torch.cuda.synchronize(device)
            ops.check_device_status(device)
            del graph
            return e0.elapsed_time(e1) / reps / layers

        ms_layer = time_layers(None)
        by_mode = {m: time_layers(m) * 1e3 for m in ("inline", "kernel")}
        nbytes = (sum(lens) * hkv * D * 2 * 2 + 2 * batch * hq * D * 2 + 4 * sum(npg)
                  + 4 * (2 * batch + 1))
        gbs = nbytes / (ms_layer / 1e3) / 1e9
        res[name] = {"batch": batch, "ctx": f"U[{lo},{hi}]", "heads": f"{hq}/{hkv}",
                     "us_per_layer": ms_layer * 1e3, "algorithmic_bytes_per_layer": nbytes,
                     "gbs": gbs, "frac": gbs / peak,
                     "us_per_layer_merge_inline": by_mode["inline"],
                     "us_per_layer_merge_kernel": by_mode["kernel"]}
        del pools, outs
        torch.cuda.empty_cache()
    return {"workload": "decode attention at the 8B decode shapes, 32 layers per CUDA graph",
            "peak_gbs": peak, "peak_source": src, **res}


LINEAR_SHAPES = [(f"tp{tp}_{m}rows_{name}", m, n // (tp if split == "out" else 1),
                  k // (tp if split == "in" else 1))
                 for tp in (1, 2, 8) for m in (1, 64)
                 for name, n, k, split in (("qkv", 6144, 4096, "out"), ("o", 4096, 4096, "in"),
                                           ("gate_up", 28672, 4096, "out"),
                                           ("down", 4096, 14336, "in"))]


def run_linear_shapes(device, shapes=None, reps=20, copies=8, policies=None):
    """The tcgen05 linear kernel (ops.linear, every row count allowed) against cuBLAS
    (F.linear) on the 8B model's per-layer projections at TP = 1, 2 and 8 and 1 or 64
    rows: ``copies`` weight copies rotated between calls (the large ones then come from
    DRAM; the TP=8 ones still fit in L2 together), ``reps`` calls per CUDA graph, five
    replays, CUDA events; frac = weight bytes / time / measured HBM bandwidth.
    ``policies``: (CTAs per SM, fewest K chunks per split) pairs of the kernel's split
    rule, or ("splits", s) for a fixed split count, to time as well (through its
    NSLG_LINEAR_* overrides)."""
    import torch.nn.functional as F
    from nanoslg_b200 import ops
    peak, _ = _hbm_peak()
    out = {}

    def timeit(fn):
        fn()
        torch.cuda.synchronize(device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(reps):
                fn()
        g.replay()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(5):
            g.replay()
        e1.record()
        torch.cuda.synchronize(device)
        del g
        return e0.elapsed_time(e1) * 1e3 / (5 * reps)

    for name, m, n, k in (shapes or LINEAR_SHAPES):
        ws = [(torch.randn(n, k, device=device) / 64).to(torch.bfloat16) for _ in range(copies)]
        x = torch.randn(m, k, device=device).to(torch.bfloat16)
        i = [0]

        def ours():
            i[0] = (i[0] + 1) % copies
            ops.linear(x, ws[i[0]], max_rows=ops.LINEAR_MAX_ROWS)

        def cublas():
            i[0] = (i[0] + 1) % copies
            F.linear(x, ws[i[0]])

        t_o, t_c = timeit(ours), timeit(cublas)
        gb = n * k * 2 / 1e9
        out[name] = {"shape": [m, n, k], "ours_us": t_o, "cublas_us": t_c,
                     "ours_frac": gb / (t_o * 1e-6) / peak, "cublas_frac": gb / (t_c * 1e-6) / peak}
        for pol in policies or ():
            env = ({"NSLG_LINEAR_SPLITS": str(pol[1])} if pol[0] == "splits" else
                   {"NSLG_LINEAR_CTAS_PER_SM": str(pol[0]), "NSLG_LINEAR_MIN_CHUNKS": str(pol[1])})
            key = (f"splits{pol[1]}" if pol[0] == "splits" else f"cps{pol[0]}_min{pol[1]}")
            os.environ.update(env)
            try:
                out[name].setdefault("ours_us_by_policy", {})[key] = timeit(ours)
            finally:
                for e in env:
                    os.environ.pop(e, None)
        del ws
        torch.cuda.empty_cache()
    ops.check_device_status(device)
    return out


def _hbm_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        return 6650.0, "fallback 6650 GB/s"


def run_elementwise_kernels(device, reps=10, batch=64, prompt=512, hidden=4096):
    """The two bandwidth-bound kernels of the layer at the C3 prefill shape (64 prompts x
    512 tokens = 32768 rows; inputs larger than L2, no flush):
      rope_kv_append_bf16_kernel: q [T, 32, 128], k, v [T, 8, 128] bf16, positions 0..511 per
        prompt, fp32 cos/sin table [8192, 128]; writes q_rot and K/V into a shuffled pool.
        Algorithmic bytes: q, k, v read + q_rot written + K/V written + the touched table
        rows (512 x 128 x 4 B x 2) + positions and write slots (4 B each per row);
      rmsnorm_residual_kernel: x, residual [T, 4096] bf16 with weight; residual <- x +
        residual, out = rmsnorm(residual) * weight. Algorithmic bytes: x, residual read,
        residual and out written, weight once;
      silu_mul_kernel: the stacked gate|up GEMM output [T, 2 x 14336] bf16 read, silu(gate)
        * up [T, 14336] written.
    CUDA events, median of ``reps`` launches each."""
    from nanoslg_b200 import ops
    from nanoslg_b200.models import precompute_rope_frequencies
    bf = torch.bfloat16
    T = batch * prompt
    g = torch.Generator(device=device).manual_seed(11)
    npg = -(-prompt // PS)
    pages = batch * npg + 1
    q = torch.randn(T, HQ, D, device=device, generator=g).to(bf)
    k = torch.randn(T, HKV, D, device=device, generator=g).to(bf)
    v = torch.randn(T, HKV, D, device=device, generator=g).to(bf)
    q_out = torch.empty_like(q)
    pool_k = torch.zeros(pages, PS, HKV, D, device=device, dtype=bf)
    pool_v = torch.zeros_like(pool_k)
    perm = torch.randperm(pages - 1, device=device, generator=g)[:batch * npg] + 1
    pos = torch.arange(prompt, device=device, dtype=torch.int32).repeat(batch)
    page_of = perm.view(batch, npg)[:, (pos[:prompt] // PS).long()].reshape(-1)
    write_loc = (page_of * PS + (pos % PS)).to(torch.int32)
    cos, sin = precompute_rope_frequencies(D, 8192, 500000.0, None)
    cos, sin = cos.to(device).float().contiguous(), sin.to(device).float().contiguous()
    x = torch.randn(T, hidden, device=device, generator=g).to(bf)
    res = torch.randn(T, hidden, device=device, generator=g).to(bf)
    w = torch.ones(hidden, device=device, dtype=bf)
    out = torch.empty_like(x)

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(device)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
        ev[0].record()
        for i in range(reps):
            fn()
            ev[i + 1].record()
        torch.cuda.synchronize(device)
        return statistics.median(ev[i].elapsed_time(ev[i + 1]) for i in range(reps))

    peak, src = _hbm_peak()
    rope_ms = timed(lambda: ops.rope_kv_append(q, k, v, pos, cos, sin, write_loc, pool_k,
                                               pool_v, q_out=q_out))
    rope_bytes = (T * HQ * D * 2) * 2 + (T * HKV * D * 2) * 4 + 2 * prompt * D * 4 + 8 * T
    norm_ms = timed(lambda: ops.rmsnorm_residual(x, w, 1e-5, residual=res, out=out))
    norm_bytes = 4 * T * hidden * 2 + hidden * 2
    del q, k, v, q_out, pool_k, pool_v, x, res, out
    torch.cuda.empty_cache()
    inter = 14336
    gu = torch.randn(T, 2 * inter, device=device, generator=g).to(bf)
    act = torch.empty(T, inter, device=device, dtype=bf)
    silu_ms = timed(lambda: ops.silu_mul(gu, out=act))
    silu_bytes = 3 * T * inter * 2
    del gu, act
    torch.cuda.empty_cache()
    leg = lambda name, ms, nbytes: {
        "kernel": name, "ms_median": ms, "algorithmic_bytes": nbytes,
        "gbs": nbytes / (ms / 1e3) / 1e9, "frac": nbytes / (ms / 1e3) / 1e9 / peak}
    return {"workload": f"C3 prefill shape: {batch} prompts x {prompt} tokens "
                        f"({T} rows), 32/8 heads, D=128, hidden {hidden}, bf16",
            "peak_gbs": peak, "peak_source": src,
            "rope_kv_append": leg("rope_kv_append_bf16_kernel", rope_ms, rope_bytes),
            "rmsnorm_residual": leg("rmsnorm_residual_kernel", norm_ms, norm_bytes),
            "silu_mul": leg("silu_mul_kernel", silu_ms, silu_bytes)}


# ------------------------------------------------------------------ model decode
def run_llama_decode(device, world, rank, batch, prompt, steps, warmup, runner=None,
                     peer_allreduce=True, split=False, solo=False):
    """Llama-3.1-8B-architecture decode (BASELINE config C3 at TP=1, TP=world under
    torchrun): prefill of ``prompt`` random token ids per sequence, then ``steps`` timed
    greedy decode steps of the whole batch through the B200 path. ``split`` adds the
    per-category split of a step (run_step_split); ``solo`` runs TP=world on this rank
    alone, with no collective, while other ranks of a process group wait."""
    from nanoslg_b200.runner import LlamaRunner, llama_config
    hf = llama_config("llama-3.1-8b")
    if runner is None:
        pages = 2 * 64 * (-(-(prompt + 8 + 64 + 2) // PS)) + 64
        # room for one batch of 64 x 512-token prompts, or the C4 batches of
        # 1024 + 128 + 136 tokens per request (shared prefix pages counted once)
        pages = max(pages, 64 * (-(-(128 + 136) // PS)) * 2 + 2 * (1024 // PS) + 64)
        runner = LlamaRunner(hf, device, tp_size=world, rank=rank, max_kv_pages=pages,
                             peer_allreduce=peer_allreduce)
        runner.enable_cuda_graphs([64, 16, 4, 1])
    g = torch.Generator().manual_seed(123 + batch)
    prompts = torch.randint(0, hf.vocab_size, (batch, prompt), generator=g).tolist()
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    tok = runner.prefill(prompts)
    torch.cuda.synchronize(device)
    prefill_ms = (time.perf_counter() - t0) * 1e3
    for _ in range(warmup):
        tok = runner.decode_step(tok)
    coll = torch.distributed.is_initialized() and not solo
    if coll:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        tok = runner.decode_step(tok)
    e1.record()
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1)
    if coll:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    sp = run_step_split(runner, device) if split else None
    runner.release()
    roof = _decode_roofline(runner, batch, prompt + warmup + (steps + 1) / 2)
    res = {"batch": batch, "prompt": prompt, "steps": steps, "ms_per_step": ms / steps,
           "tok_s": batch * steps / (ms / 1e3), "prefill_ms": prefill_ms,
           "hbm_roofline": dict(roof, frac=roof["ms_per_step"] / (ms / steps))}
    if sp is not None:
        res["step_split"] = sp
    return runner, res


def run_step_split(runner, device, reps=10):
    """Where one decode step of the current batch spends its time, by category: each
    category's kernels for every layer, with the step's exact shapes, captured alone in a
    CUDA graph and replayed ``reps`` times (CUDA events, max over ranks):

      gemm       the projections (stacked q|k|v, o, stacked gate|up, down) of every layer
                 and the LM head on the last position, through ops.linear as the model
                 runs them;
      attention  RoPE + KV append + paged decode attention (CacheContext.attend_rope) of
                 every layer on the step's own plan;
      tp_reduce  the two residual-add + RMSNorm calls per layer, fused with the RowParallel
                 all-reduce over peer memory at TP > 1 (NCCL all-reduce + the norm kernel
                 when the peer path is off);
      other      SwiGLU, the embedding gather and the greedy argmax (+ the (max, index)
                 exchange at TP > 1).

    ``step_ms`` is the whole step replayed the same way; ``limiter`` the largest category.
    The categories are timed apart, so their sum exceeds the step only by what the step
    overlaps (programmatic dependent launch) and is below it by launch gaps."""
    import torch.nn.functional as F
    from nanoslg_b200 import ops
    model, mgr = runner.model, runner.cache
    B = len(runner.seq_ids)
    hf = runner.hf
    hid = hf.hidden_size
    dt = runner.dtype
    ctx = mgr.begin_forward(runner.seq_ids, [1] * B)
    if not getattr(ctx, "plan_static", False):
        mgr.end_forward(ctx)
        return None
    layers = list(model.layers)
    att0 = layers[0].self_attn
    hq, hkv, hd = att0.n_heads_tp, att0.n_kv_heads_tp, att0.head_dim
    x = torch.randn(B, 1, hid, device=device).to(dt)
    qkv = torch.randn(B, 1, (hq + 2 * hkv) * hd, device=device).to(dt)
    a = torch.randn(B, 1, hq * hd, device=device).to(dt)
    inter = layers[0].mlp.down_proj.weight.shape[1]
    gu = torch.randn(B, 1, 2 * inter, device=device).to(dt)
    act = torch.randn(B, 1, inter, device=device).to(dt)
    res = torch.randn(B, 1, hid, device=device).to(dt)
    ids = torch.zeros(B, 1, dtype=torch.long, device=device)
    peer = runner.peer
    if peer is not None:
        peer.active = peer.fits(B)
    head = getattr(model.lm_head, "lm_head", model.lm_head)

    def gemm():
        for L in layers:
            ops.linear(x, L.self_attn._qkv)
            ops.linear(a, L.self_attn.o_proj.weight)
            ops.linear(x, L.mlp._gu)
            ops.linear(act, L.mlp.down_proj.weight)
        ops.linear(x[:, -1], head.weight)

    def attention():
        q = qkv[..., :hq * hd].view(B, 1, hq, hd)
        k = qkv[..., hq * hd:(hq + hkv) * hd].view(B, 1, hkv, hd)
        v = qkv[..., (hq + hkv) * hd:].view(B, 1, hkv, hd)
        for L in layers:
            ctx.attend_rope(L.self_attn.layer_idx, q, k, v, model.cos, model.sin)

    def tp_reduce():
        for L in layers:
            for norm in (L.input_layernorm, L.post_attention_layernorm):
                if peer is not None and peer.active:
                    peer.allreduce_add_norm(x, res, norm.weight, norm.eps)
                else:
                    y = x
                    if runner.pcfg.tp_size > 1:
                        y = x.clone()
                        torch.distributed.all_reduce(y, group=runner.pctx.tp_group)
                    ops.rmsnorm_residual(y, norm.weight, norm.eps, residual=res)

    logits = F.linear(x[:, -1], head.weight)
    tp = runner.pcfg.tp_size

    def other():
        model.embed_tokens(ids)
        for _ in layers:
            ops.silu_mul(gu, out=act)
        if tp > 1:
            idx, val = ops.argmax_rows(logits, 0, values=True)
            pair = torch.stack([val, idx.float()], -1)
            allp = torch.empty((tp * pair.shape[0], 2), dtype=pair.dtype, device=device)
            torch.distributed.all_gather_into_tensor(allp, pair, group=runner.pctx.tp_group)
        else:
            ops.argmax_rows(logits)

    def step():
        model(ids, ctx, last_only=True, greedy=True)

    def timed(fn):
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream(device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        graph.replay()
        torch.cuda.synchronize(device)
        if torch.distributed.is_initialized():
            torch.distributed.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1) / reps
        del graph
        if torch.distributed.is_initialized():
            t = torch.tensor([ms], device=device, dtype=torch.float64)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    with torch.inference_mode():
        cats = {name: timed(fn) for name, fn in (("gemm", gemm), ("attention", attention),
                                                ("tp_reduce", tp_reduce), ("other", other))}
        step_ms = timed(step)
    mgr.end_forward(ctx)
    ops.check_device_status(device)
    total = sum(cats.values())
    return {"step_ms": step_ms, **{f"{k}_ms": v for k, v in cats.items()},
            "sum_ms": total, "share": {k: v / total for k, v in cats.items()},
            "limiter": max(cats, key=cats.get),
            "method": "each category's kernels of every layer captured alone in a CUDA graph, "
                      f"{reps} replays, CUDA events, max over ranks"}


def _decode_roofline(runner, batch, avg_ctx):
    """Lower bound of one decode step of this rank from HBM traffic alone: every weight
    of the rank read once (embedding: only the batch's rows) plus the K/V of every
    sequence and layer (average context ``avg_ctx`` tokens over the timed steps), at the
    measured HBM bandwidth."""
    hidden = runner.hf.hidden_size
    wbytes = 0
    for name, prm in runner.model.named_parameters():
        n = prm.numel() * prm.element_size()
        if "embed_tokens" in name:
            n = batch * hidden * prm.element_size()
        wbytes += n
    cfg = runner.cache.cfg
    kv = batch * avg_ctx * cfg.num_layers * 2 * cfg.num_kv_heads * cfg.head_dim * 2
    peak, src = _hbm_peak()
    return {"weight_bytes": wbytes, "kv_bytes": int(kv), "peak_gbs": peak,
            "peak_source": src, "ms_per_step": (wbytes + kv) / (peak * 1e9) * 1e3}


def run_llama_c4(device, world, rank, runner, batches=(4, 16, 64), prefix_len=1024,
                 suffix_len=128, steps=128):
    """BASELINE config C4 on the TP=world runner: every request shares one random
    1024-token prefix and has a unique random 128-token suffix. A priming batch (prefill
    + 4 decode steps + release, which inserts its pages into the radix tree) precedes each
    measured batch; the measured batch's prefill reuses the shared pages (prefix_skip
    tokens per request) and then decodes ``steps`` greedy tokens, CUDA events around the
    decode loop, max over ranks."""
    from nanoslg_b200.runner import llama_config
    hf = llama_config("llama-3.1-8b")
    g = torch.Generator().manual_seed(77)
    prefix = torch.randint(0, hf.vocab_size, (prefix_len,), generator=g).tolist()
    out = {}
    for bsz in batches:
        def batch():
            return [prefix + torch.randint(0, hf.vocab_size, (suffix_len,), generator=g).tolist()
                    for _ in range(bsz)]
        tok = runner.prefill(batch())                          # priming batch
        gen = [[int(t)] for t in tok.tolist()]
        for _ in range(4):
            tok = runner.decode_step(tok)
            for gl, t in zip(gen, tok.tolist()):
                gl.append(int(t))
        runner.release(gen)
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        tok = runner.prefill(batch())                          # measured batch
        torch.cuda.synchronize(device)
        prefill_ms = (time.perf_counter() - t0) * 1e3
        skip = list(runner.prefix_lens)
        for _ in range(3):
            tok = runner.decode_step(tok)
        if torch.distributed.is_initialized():
            torch.distributed.barrier()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            tok = runner.decode_step(tok)
        e1.record()
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1)
        if torch.distributed.is_initialized():
            t = torch.tensor([ms, prefill_ms], device=device, dtype=torch.float64)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms, prefill_ms = t.tolist()
        runner.release()
        out[f"batch{bsz}"] = {"decode_tok_s": bsz * steps / (ms / 1e3),
                              "ms_per_step": ms / steps, "prefill_ms": prefill_ms,
                              "prefix_skip_tokens": min(skip), "steps": steps}
    return out


def run_llama70b_c5(device, world, rank, steps=256, batch=32, prompt=2048):
    """BASELINE C5: Llama-3-70B architecture (random init), bf16, TP=4 x PP=2 on 8 GPUs,
    batch 32, 2048-token random prompts, 256 greedy decode tokens. The prefill runs the
    reference's lock-step pipeline; decode is measured with the config's 4 pipeline
    micro-batches (LlamaRunner.decode_microbatched), with 2, and lock step (the
    reference's schedule), every stage forward a CUDA graph. CUDA events around the
    decode loop, max over ranks."""
    from nanoslg_b200.runner import LlamaRunner, llama_config
    if world != 8:
        raise ValueError("C5 runs on 8 GPUs (TP=4 x PP=2)")
    hf = llama_config("llama-3-70b")
    pages = batch * (-(-(prompt + steps + 16) // PS)) + 64
    runner = LlamaRunner(hf, device, tp_size=4, pp_size=2, rank=rank, max_kv_pages=pages,
                         prefix_caching=False)
    runner.enable_cuda_graphs([batch, batch // 2, batch // 4])
    g = torch.Generator().manual_seed(70)
    prompts = torch.randint(0, hf.vocab_size, (batch, prompt), generator=g).tolist()
    out = {"model": "Llama-3-70B architecture, random init N(0, 0.02), bf16",
           "parallelism": "TP=4 x PP=2", "batch": batch, "prompt": prompt, "steps": steps}

    def maxed(x):
        t = torch.tensor([x], device=device, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    for name, micro in (("microbatch4", 4), ("microbatch2", 2), ("lockstep", 1)):
        torch.distributed.barrier()
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        tok = runner.prefill(prompts)
        torch.cuda.synchronize(device)
        prefill_ms = maxed((time.perf_counter() - t0) * 1e3)

        def decode(n, tok):
            if micro > 1:
                gen = runner.decode_microbatched(tok, micro, n)
                return gen[:, -1].contiguous()
            for _ in range(n):
                tok = runner.decode_step(tok)
            return tok

        tok = decode(2, tok)                                   # graph capture, warm-up
        torch.distributed.barrier()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        tok = decode(steps, tok)
        e1.record()
        torch.cuda.synchronize(device)
        ms = maxed(e0.elapsed_time(e1))
        runner.release()
        out[name] = {"decode_tok_s": batch * steps / (ms / 1e3), "ms_per_step": ms / steps,
                     "prefill_ms": prefill_ms}
    runner.close()
    return out


def run_allreduce(device, world, rank, hidden=4096, rows_list=(1, 64, 256), calls=50,
                  replays=10):
    """The fused TP reduction (nslg_tp_allreduce_rmsnorm: all-reduce of a RowParallel
    partial + residual add + RMSNorm over NVLink peer memory) against what it replaces
    (NCCL all-reduce + the rmsnorm kernel), bf16 [rows, hidden], each timed as ``calls``
    back-to-back calls captured in one CUDA graph and replayed ``replays`` times; CUDA
    events, max over ranks, microseconds per call."""
    from nanoslg_b200 import ops
    from nanoslg_b200.tp_comm import PeerAllReduce
    bf = torch.bfloat16
    peer = PeerAllReduce(torch.distributed.group.WORLD, rank, world, device, max(rows_list),
                         hidden, bf)
    w = torch.ones(hidden, dtype=bf, device=device)
    out = {}
    for rows in rows_list:
        x = torch.randn(rows, hidden, device=device).to(bf)
        r = torch.randn(rows, hidden, device=device).to(bf)

        def nccl():
            torch.distributed.all_reduce(x)
            return ops.rmsnorm_residual(x, w, 1e-5, residual=r)

        def fused():
            return peer.allreduce_add_norm(x, r, w, 1e-5)

        legs = [("nccl_allreduce_plus_rmsnorm_us", nccl, None), ("fused_us", fused, None)]
        if world > 2:       # the fused kernel's two modes, forced (decided at capture)
            legs += [("fused_one_shot_us", fused, "0"), ("fused_two_shot_us", fused, "1")]
        for name, fn, mode in legs:
            if mode is None:
                os.environ.pop("NSLG_TP_TWO_SHOT", None)
            else:
                os.environ["NSLG_TP_TWO_SHOT"] = mode
            for _ in range(3):
                fn()
            torch.cuda.synchronize(device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(calls):
                    fn()
            g.replay()
            torch.cuda.synchronize(device)
            torch.distributed.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(replays):
                g.replay()
            e1.record()
            torch.cuda.synchronize(device)
            t = torch.tensor([e0.elapsed_time(e1) * 1e3 / (calls * replays)], device=device)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            out.setdefault(f"rows{rows}", {})[name] = round(float(t.item()), 2)
            del g
    os.environ.pop("NSLG_TP_TWO_SHOT", None)
    ops.check_device_status(device)
    out["gemm_then_reduce"] = _gemm_reduce_timing(device, world, rank, peer, hidden, calls,
                                                  replays)
    peer.close()
    return {"world": world, "hidden": hidden, "dtype": "bf16", **out}


def _gemm_reduce_timing(device, world, rank, peer, hidden, calls, replays):
    """A RowParallel product (o_proj of the 8B model at TP=world: [rows, 4096/world] x
    [4096, 4096/world]^T) followed by the fused reduction + residual + RMSNorm, as the
    decode step runs it: with the push in the reduction kernel (``separate_us``) and with
    the GEMM pushing its own rows (nslg_linear_tp_push, ``fused_push_us``). Pairs of calls
    captured back to back in a CUDA graph; CUDA events, max over ranks, us per pair."""
    from nanoslg_b200 import ops
    bf = torch.bfloat16
    k = 4096 // world
    res = {}
    for rows in (1, 4):
        x = torch.randn(rows, k, device=device).to(bf)
        wt = (torch.randn(hidden, k, device=device) / k ** 0.5).to(bf)
        r = torch.randn(rows, hidden, device=device).to(bf)
        nw = torch.ones(hidden, dtype=bf, device=device)
        for name, fuse in (("separate_us", False), ("fused_push_us", True)):
            peer.fuse_push = fuse

            def pair():
                y = peer.linear_push(x, wt) if fuse else None
                if y is None:
                    y = ops.linear(x, wt)
                return peer.allreduce_add_norm(y, r, nw, 1e-5)

            for _ in range(3):
                pair()
            torch.cuda.synchronize(device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(calls):
                    pair()
            g.replay()
            torch.cuda.synchronize(device)
            torch.distributed.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(replays):
                g.replay()
            e1.record()
            torch.cuda.synchronize(device)
            t = torch.tensor([e0.elapsed_time(e1) * 1e3 / (calls * replays)], device=device)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            res.setdefault(f"rows{rows}", {})[name] = round(float(t.item()), 2)
            del g
    peer.fuse_push = True
    ops.check_device_status(device)
    return {"shape": f"[rows, {k}] x [{hidden}, {k}]^T", **res}


# ------------------------------------------------------------------------ parity
def _tokens_run(runner, prompts, steps, micro=0):
    """Greedy tokens [B, steps] of a prefill and ``steps - 1`` decode steps (``micro``:
    the decode steps as pipeline micro-batches). None on ranks that do not hold them."""
    tok = runner.prefill(prompts)
    first = tok.clone()
    if micro:
        gen = runner.decode_microbatched(tok, micro, steps - 1)
        if gen is None:
            return None
        return torch.cat([first[:, None], gen.to(first.device)], 1).tolist()
    toks = [first]
    for _ in range(steps - 1):
        tok = runner.decode_step(tok)
        toks.append(tok.clone())
    return torch.stack(toks, 1).tolist()


def run_parity(device, world, rank):
    """Correctness of the sharded path at this world size, checked inside the benchmark
    run against fixtures recorded from the reference (tests/golden/tiny_llama_kv8.json:
    the reference's contiguous-SDPA path on a 2-prompt batch of a tiny fp32 Llama with 8
    query / 8 KV heads, so TP = 1, 2, 4 and 8 all divide it):

    * ``tp``: TP=world, RowParallel reductions through the fused peer-memory kernel
      (world > 1), greedy tokens through the vocab-parallel (max, index) exchange; eager
      and with CUDA-graph decode steps;
    * ``tp_x_pp2`` (world >= 2): TP=world/2 x PP=2 (PP=2 alone at world 2), lock-step
      stages and the 2-micro-batch pipeline schedule;
    * ``allreduce``: nslg_tp_allreduce_rmsnorm's new residual bit-equal to an fp32
      rank-order sum of the ranks' bf16 partials + residual (hidden 4096; 1 and 64 rows);
    * ``tp_exchange_one_gpu`` (rank 0, every world size): the same check with all ranks of
      a TP=8 group on this GPU -- the reduction's one-shot, two-shot and size-chosen
      modes in one cooperative grid, and the RowParallel GEMM's own push followed by the
      push-less reduction.

    Every rank takes part; ``ok`` is true only if every check held on every rank."""
    from types import SimpleNamespace
    from nanoslg_b200.models import reference_random_state_dict
    from nanoslg_b200.runner import LlamaRunner
    with open(os.path.join(ROOT, "tests", "golden", "tiny_llama_kv8.json")) as f:
        g = json.load(f)
    hf = SimpleNamespace(**g["config"])
    full = reference_random_state_dict(hf)
    want = g["tokens"]
    steps = len(want[0])
    prev_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    checks = {}
    layouts = [("tp", world, 1, False), ("tp_graphs", world, 1, True)]
    if world >= 2:
        layouts += [("tp_x_pp2", world // 2, 2, False), ("tp_x_pp2_graphs", world // 2, 2, True)]
    for name, tp, pp, graphs in layouts:
        # no prefix caching: the second batch of a runner must not hit the first one's
        # pages (a full-prompt hit re-feeds the last token one position later, a
        # reference quirk the fixture does not contain)
        r = LlamaRunner(hf, device, dtype=torch.float32, tp_size=tp, pp_size=pp, rank=rank,
                        max_kv_pages=64, prefix_caching=False)
        r.load_full_state_dict(full)
        if graphs:
            r.enable_cuda_graphs([len(want), 1])
        got = _tokens_run(r, g["prompts"], steps)
        ok = got == want
        r.release()
        if pp > 1:
            got_mb = _tokens_run(r, g["prompts"], steps, micro=2)
            ok = ok and (got_mb is None or got_mb == want)
            r.release()
        r.close()
        checks[name] = {"tp": tp, "pp": pp, "cuda_graphs": graphs, "ok": bool(ok)}
    torch.backends.cuda.matmul.allow_tf32 = prev_tf32
    if world > 1:
        checks["allreduce"] = _allreduce_parity(device, world, rank)
    if rank == 0:
        checks["tp_exchange_one_gpu"] = _emulated_exchange_parity(device)
    flags = torch.tensor([int(all(c["ok"] for c in checks.values()))], device=device)
    if world > 1:
        torch.distributed.all_reduce(flags, op=torch.distributed.ReduceOp.MIN)
    return {"ok": bool(flags.item()), "fixture": "tests/golden/tiny_llama_kv8.json "
            "(reference contiguous SDPA, fp32, batch 2, 16 greedy tokens)", "checks": checks}


def _emulated_exchange_parity(device, world=8, hidden=4096):
    """All ranks of a TP group emulated on this GPU (see run_parity): residual bit-equal
    to bf16(bf16(fp32 rank-order sum of the partials) + residual) on every rank."""
    import ctypes
    from nanoslg_b200 import _native as N
    from nanoslg_b200 import ops
    lib = N.lib()
    bf = torch.bfloat16
    stream = torch.cuda.current_stream(device).cuda_stream
    status = ops.status_word(device)
    P = ctypes.c_void_p * world
    arr = lambda ts: ctypes.cast(P(*[t.data_ptr() for t in ts]), ctypes.c_void_p)
    stage_bytes = 4 * world * 64 * hidden * 2
    g = torch.Generator(device=device).manual_seed(123)

    def want(parts, res):
        s = parts[0].float()
        for p in parts[1:]:
            s = s + p.float()
        return (res.float() + s.to(bf).float()).to(bf)

    out = {}
    for name, mode in (("one_shot", "0"), ("two_shot", "1"), ("by_size", None)):
        old = os.environ.pop("NSLG_TP_TWO_SHOT", None)
        if mode is not None:
            os.environ["NSLG_TP_TWO_SHOT"] = mode
        try:
            stages = [torch.zeros(stage_bytes, dtype=torch.uint8, device=device)
                      for _ in range(world)]
            cnt = [torch.zeros(N.TP_COUNTER_BYTES // 4, dtype=torch.int32, device=device)
                   for _ in range(world)]
            ok = True
            for rows in (64, 1, 17):
                parts = [torch.randn(rows, hidden, generator=g, device=device).to(bf)
                         for _ in range(world)]
                res = torch.randn(rows, hidden, generator=g, device=device).to(bf)
                resid = [res.clone() for _ in range(world)]
                rc = lib.nslg_tp_allreduce_rmsnorm_emulated(
                    N.DTYPE_BF16, rows, hidden, world, arr(parts), hidden, arr(stages),
                    stage_bytes, arr(cnt), arr(resid), hidden, None, None, 0, 1e-5,
                    2_000_000_000, status.data_ptr(), stream)
                torch.cuda.synchronize(device)
                h = want(parts, res)
                ok = ok and rc == 0 and all(torch.equal(r, h) for r in resid)
            out[name] = bool(ok)
        finally:
            os.environ.pop("NSLG_TP_TWO_SHOT", None)
            if old is not None:
                os.environ["NSLG_TP_TWO_SHOT"] = old
    # the RowParallel GEMM pushing its own rows, then the reductions without a push
    stages = [torch.zeros(stage_bytes, dtype=torch.uint8, device=device) for _ in range(world)]
    cnt = [torch.zeros(N.TP_COUNTER_BYTES // 4, dtype=torch.int32, device=device)
           for _ in range(world)]
    k = hidden // world
    ok = True
    for rows in (1, 16):
        xs = [torch.randn(rows, k, generator=g, device=device).to(bf) for _ in range(world)]
        ws = [(torch.randn(hidden, k, generator=g, device=device) / k ** 0.5).to(bf)
              for _ in range(world)]
        parts = [torch.empty(rows, hidden, dtype=bf, device=device) for _ in range(world)]
        res = torch.randn(rows, hidden, generator=g, device=device).to(bf)
        resid = [res.clone() for _ in range(world)]
        for r in range(world):
            ok = ok and lib.nslg_linear_tp_push(
                N.DTYPE_BF16, rows, hidden, k, xs[r].data_ptr(), k, ws[r].data_ptr(), k,
                parts[r].data_ptr(), hidden, world, r, arr(stages), stage_bytes,
                cnt[r].data_ptr(), status.data_ptr(), stream) == 0
        for r in range(world):
            ok = ok and lib.nslg_tp_reduce_pushed_rmsnorm(
                N.DTYPE_BF16, rows, hidden, world, r, parts[r].data_ptr(), hidden,
                arr(stages), stage_bytes, cnt[r].data_ptr(), resid[r].data_ptr(), hidden,
                None, None, 0, 1e-5, 2_000_000_000, status.data_ptr(), stream) == 0
        torch.cuda.synchronize(device)
        h = want(parts, res)
        ok = ok and all(torch.equal(r, h) for r in resid)
    out["gemm_push"] = bool(ok)
    try:
        ops.check_device_status(device)
    except RuntimeError:
        out = {n: False for n in out}
    return {"world": world, "ok": all(out.values()), "modes": out,
            "check": "every emulated rank's new residual bit-equal to bf16(bf16(fp32 "
                     "rank-order sum) + residual)"}


def _allreduce_parity(device, world, rank, hidden=4096):
    from nanoslg_b200 import ops
    from nanoslg_b200.tp_comm import PeerAllReduce
    bf = torch.bfloat16
    peer = PeerAllReduce(torch.distributed.group.WORLD, rank, world, device, 64, hidden, bf)
    modes = {"one_shot": "0", "two_shot": "1"} if world > 2 else {"one_shot": "0"}
    res_ok = {}
    for name, env in modes.items():
        if env is None:
            os.environ.pop("NSLG_TP_TWO_SHOT", None)
        else:
            os.environ["NSLG_TP_TWO_SHOT"] = env
        ok = True
        for it, rows in enumerate((64, 1, 64)):
            parts = [torch.randn(rows, hidden, generator=torch.Generator().manual_seed(1000 * it + r))
                     .to(bf) for r in range(world)]
            gs = torch.Generator().manual_seed(99 + it)
            res = torch.randn(rows, hidden, generator=gs).to(bf)
            w = (1 + 0.1 * torch.randn(hidden, generator=gs)).to(bf)
            s = parts[0].float()
            for p in parts[1:]:
                s = s + p.float()
            h_want = (res.float() + s.to(bf).float()).to(bf)
            r_dev = res.to(device)
            peer.allreduce_add_norm(parts[rank].to(device), r_dev, w.to(device), 1e-5)
            ok = ok and torch.equal(r_dev.cpu(), h_want)
        try:
            ops.check_device_status(device)
        except RuntimeError:
            ok = False
        res_ok[name] = bool(ok)
    os.environ.pop("NSLG_TP_TWO_SHOT", None)
    # the RowParallel GEMM pushing its own rows (nslg_linear_tp_push), then the reduction
    # (decode batches of up to tp_comm.FUSED_PUSH_MAX_ROWS rows take this path)
    from nanoslg_b200.tp_comm import FUSED_PUSH_MAX_ROWS, FUSED_PUSH_MIN_WORLD
    min_world = FUSED_PUSH_MIN_WORLD
    peer_world_ok = world >= min_world
    ok = True
    k = 4096 // world
    for it, rows in enumerate(sorted({1, FUSED_PUSH_MAX_ROWS, max(1, FUSED_PUSH_MAX_ROWS - 1)})):
        g = torch.Generator().manual_seed(500 + 10 * it + rank)
        x = torch.randn(rows, k, generator=g).to(bf).to(device)
        wt = (torch.randn(hidden, k, generator=g) / k ** 0.5).to(bf).to(device)
        gs = torch.Generator().manual_seed(77 + it)
        res = torch.randn(rows, hidden, generator=gs).to(bf)
        w = (1 + 0.1 * torch.randn(hidden, generator=gs)).to(bf)
        part = peer.linear_push(x, wt) if peer_world_ok else None
        if part is None:
            if peer_world_ok:
                ok = False
            break
        r_dev = res.to(device)
        peer.allreduce_add_norm(part, r_dev, w.to(device), 1e-5)
        parts = [torch.empty_like(part) for _ in range(world)]
        torch.distributed.all_gather(parts, part)
        s = parts[0].float()
        for p in parts[1:]:
            s = s + p.float()
        h_want = (res.to(device).float() + s.to(bf).float()).to(bf)
        ok = ok and torch.equal(r_dev, h_want)
    try:
        ops.check_device_status(device)
    except RuntimeError:
        ok = False
    if peer_world_ok:                     # below FUSED_PUSH_MIN_WORLD the path is unused
        res_ok["fused_gemm_push"] = bool(ok)
    peer.close()
    return {"world": world, "rows": [64, 1, 64], "ok": all(res_ok.values()), "modes": res_ok,
            "check": "new residual bit-equal to bf16(bf16(fp32 rank-order sum) + residual)"}


# ------------------------------------------------------------------------ CPU side
def cpu_reference(max_seconds, n_calls=None, seed=0, warmup=1):
    """The reference's contiguous attend (oracle/attention.py restating
    kv_cache.py:247-325) on the C2 workload, all host threads: ``warmup`` untimed calls,
    then timed calls until ``n_calls`` are done or ``max_seconds`` have passed (whichever
    comes first; at least one)."""
    from oracle.attention import ContiguousOracle
    torch.set_num_threads(os.cpu_count() or 1)
    lens = c2_lens(seed)
    smax = max(lens) + 1
    orc = ContiguousOracle(1, B, smax, HKV, D, torch.bfloat16)
    g = torch.Generator().manual_seed(seed)
    blk = torch.randn(1024, HKV, D, generator=g).to(torch.bfloat16)
    for b, n in enumerate(lens):                        # history: tiled random rows
        reps = -(-n // 1024)
        orc.k[0, b, :n] = blk.repeat(reps, 1, 1)[:n]
        orc.v[0, b, :n] = blk.flip(0).repeat(reps, 1, 1)[:n]
    q = torch.randn(B, 1, HQ, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, 1, HKV, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, 1, HKV, D, generator=g).to(torch.bfloat16)
    starts = list(lens)
    for _ in range(max(1, warmup)):
        orc.attend(0, q, k, v, starts, [1] * B, [0] * B)
    times = []
    t_end = time.perf_counter() + max_seconds
    while not times or ((n_calls is None or len(times) < n_calls)
                        and time.perf_counter() < t_end):
        t0 = time.perf_counter()
        orc.attend(0, q, k, v, starts, [1] * B, [0] * B)
        times.append(time.perf_counter() - t0)
    mean = sum(times) / len(times)
    return dict(value=B / mean, calls=len(times), s_per_call=mean, cores=torch.get_num_threads(),
                sample=f"{len(times)} full C2 decode-attention calls (64 seqs, sum(len)="
                       f"{sum(lens)}, one layer) through the contiguous cache + SDPA, bf16")


def run_model_legs(a, device, world, rank):
    """The Llama-3.1-8B decode legs at TP=world: batch 64 and batch 1 with the per-step
    split, at world > 1 also the TP=1 batch-64 decode on rank 0 alone (the scaling
    denominator) and the C4 radix workload."""
    out = {}
    tp1 = None
    if world > 1:
        # the same batch-64 decode at TP=1 on rank 0 alone: the denominator of this
        # line's TP scaling figures
        if rank == 0:
            run1, tp1 = run_llama_decode(device, 1, 0, 64, 512, a.model_steps, 4, solo=True)
            run1.close()
            del run1
            torch.cuda.empty_cache()
        torch.distributed.barrier()
    runner, r64 = run_llama_decode(device, world, rank, 64, 512, a.model_steps, 4,
                                   peer_allreduce=a.tp_reduce == "peer", split=True)
    _, r1 = run_llama_decode(device, world, rank, 1, 512, a.model_steps, 4, runner=runner,
                             split=True)
    out["llama8b_decode"] = {
        "model": "Llama-3.1-8B architecture, random init N(0, 0.02), bf16 (BASELINE C3)",
        "parallelism": f"TP={world}", "batch64": r64, "batch1": r1,
        "tp_reduce": a.tp_reduce if world > 1 else None,
        "note": "greedy decode steps through models.LlamaTP + B200PagedKVCache; projections "
                "through the tcgen05 linear kernel for batches of up to 16 rows, cuBLAS "
                "above; attention, RoPE/append, RMSNorm, SwiGLU, argmax and the TP "
                "reduction the nslg kernels"}
    if tp1 is not None:
        out["llama8b_decode"]["tp_scaling_batch64"] = {
            "tp1_tok_s": tp1["tok_s"], "tp1_ms_per_step": tp1["ms_per_step"],
            "speedup_vs_tp1": r64["tok_s"] / tp1["tok_s"],
            "efficiency_vs_tp1": r64["tok_s"] / (world * tp1["tok_s"]),
            "note": "strong scaling (fixed batch 64); TP=1 measured on rank 0 alone in "
                    "this run"}
    if world > 1:
        out["llama8b_c4_radix"] = {
            "config": "BASELINE C4: TP=N, shared 1024-token prefix + unique 128-token "
                      "suffix per request, 128 greedy decode tokens, radix prefix caching",
            **run_llama_c4(device, world, rank, runner)}
    runner.close()
    del runner
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--pool-pages", type=int, default=POOL_PAGES,
                    help="page pool size; the profiling case uses a smaller pool with the same "
                         "batch (still 1.13 GB of KV per step)")
    ap.add_argument("--no-model", action="store_true", help="skip the Llama-3.1-8B decode leg")
    ap.add_argument("--model-steps", type=int, default=32)
    ap.add_argument("--c5", action="store_true",
                    help="only BASELINE C5 (Llama-3-70B, TP=4 x PP=2, needs --gpus 8)")
    ap.add_argument("--tp-reduce", choices=["peer", "nccl"], default="peer",
                    help="TP>1 decode: RowParallel reductions over NVLink peer memory fused "
                         "with residual add + RMSNorm (peer), or NCCL all-reduce (nccl)")
    ap.add_argument("--only", choices=["all", "kernel", "model", "prefill", "allreduce",
                                       "elementwise", "e2e", "parity", "decode-shapes",
                                       "linear", "refbackend"],
                    default="all",
                    help="kernel: only the resident-input kernel timing (profiling case); "
                         "model: only the Llama-3.1-8B decode leg; elementwise: the RoPE + "
                         "KV-append and RMSNorm + residual kernels at the C3 prefill shape; "
                         "e2e: only the two end-to-end legs (one and two steps in flight); "
                         "parity: only the sharded-path token / reduction checks; "
                         "decode-shapes: decode attention at the 8B model's decode shapes; "
                         "linear: the tcgen05 linear kernel against cuBLAS per 8B shape; "
                         "refbackend: the reference's FlashInfer backend against these "
                         "kernels on C2 decode and C3 prefill")
    ap.add_argument("--no-ref-backend", action="store_true",
                    help="skip the FlashInfer (reference GPU backend) leg of the default run")
    ap.add_argument("--linear-sweep", action="store_true",
                    help="--only linear: also time the kernel under other split policies")
    ap.add_argument("--linear-shape", default=None,
                    help="with --only linear: one shape 'rows,out,in' (e.g. 64,6144,4096)")
    a = ap.parse_args()
    if a.warmup < 3:
        a.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    metric = "decode tok/s (paged decode attention, C2: B=64, 32/8 heads, D=128, len U[512,8192])"
    config = {"workload": "C2 decode-attention microbenchmark (BASELINE configs[1])",
              "batch": B, "num_qo_heads": HQ, "num_kv_heads": HKV, "head_dim": D,
              "page_size": PS, "pool_pages": POOL_PAGES, "kv_len": f"U[{LEN_LO},{LEN_HI}] seed 0",
              "l2": "inputs larger than L2 (1.13 GB KV per step vs 126 MB L2), no flush",
              "parallelism": f"{world} independent replicas" if world > 1 else "single GPU"}

    if a.impl == "reference":
        if rank != 0:
            return 0
        # a.warmup untimed calls, then up to a.steps timed ones within 150 s
        r = cpu_reference(150.0, n_calls=a.steps, warmup=a.warmup)
        line = {"metric": metric, "value": r["value"], "unit": "tok/s", "n_gpus": a.gpus,
                "steps": r["calls"], "warmup": a.warmup, "ms_per_step": r["s_per_call"] * 1e3,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic (seeded N(0,1) K/V, random page table)",
                "config": config, "impl": "reference",
                "cpu_baseline": {"value": r["value"], "unit": "tok/s", "cores": r["cores"],
                                 "kind": "port", "sample": r["sample"]},
                "e2e": {"value": r["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    if not torch.cuda.is_available():
        print(json.dumps({"error": "no CUDA device"}))
        return 1
    torch.cuda.set_device(local)
    device = torch.device(f"cuda:{local}")
    if world > 1:
        import datetime
        # rank 0 alone runs the CPU baseline and the TP=1 reference decode while the
        # other ranks wait in a barrier: the group timeout covers that wait
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=420),
                                             device_id=device)
    from nanoslg_b200 import build as nbuild
    if not os.path.exists(nbuild.LIB):
        nbuild.build()
    if a.only == "parity":
        r = run_parity(device, world, rank)
        if rank == 0:
            print(json.dumps({"case": "parity only", "n_gpus": world, "parity": r}), flush=True)
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        return 0 if r["ok"] else 1

    if a.only == "e2e":
        steps = a.e2e_steps or max(10, a.steps // 2)
        res = {}
        for depth in (1, 2):
            r = run_e2e(device, steps, a.warmup, seed=rank, depth=depth)
            res[f"depth{depth}"] = {"ms_per_step": r["total_ms"] / steps,
                                    "tok_s": B * steps / (r["total_ms"] / 1e3),
                                    "h2d_bytes_per_step": r["h2d"],
                                    "d2h_bytes_per_step": r["d2h"]}
        if rank == 0:
            print(json.dumps({"case": "e2e only", "steps": steps, "e2e": res}), flush=True)
        if world > 1:
            torch.distributed.destroy_process_group()
        return 0
    if a.only == "prefill":
        if rank == 0:
            print(json.dumps({"case": "prefill only", "prefill_attention":
                              run_prefill_kernel(device)}), flush=True)
        if world > 1:
            torch.distributed.destroy_process_group()
        return 0
    if a.only == "linear":
        shapes = None
        if a.linear_shape:
            m, n, k = (int(v) for v in a.linear_shape.split(","))
            shapes = [(f"rows{m}_out{n}_in{k}", m, n, k)]
        policies = ([(1, 8), (2, 8), (1, 2)] + [("splits", n) for n in (1, 2, 3, 4, 6, 8)]
                    if a.linear_sweep else None)
        if rank == 0:
            print(json.dumps({"case": "linear only", "linear_shapes":
                              run_linear_shapes(device, shapes, policies=policies)}),
                  flush=True)
        if world > 1:
            torch.distributed.destroy_process_group()
        return 0
    if a.only == "refbackend":
        if rank == 0:
            print(json.dumps({"case": "reference GPU backend only", "reference_gpu_backend":
                              run_reference_backend(device)}), flush=True)
        if world > 1:
            torch.distributed.destroy_process_group()
        return 0
    if a.only == "decode-shapes":
        if rank == 0:
            print(json.dumps({"case": "decode shapes only", "decode_model_shapes":
                              run_decode_model_shapes(device)}), flush=True)
        if world > 1:
            torch.distributed.destroy_process_group()
        return 0
    if a.only == "elementwise":
        if rank == 0:
            print(json.dumps({"case": "elementwise only", "elementwise":
                              run_elementwise_kernels(device)}), flush=True)
        if world > 1:
            torch.distributed.destroy_process_group()
        return 0
    if a.only == "allreduce":
        if world < 2:
            raise SystemExit("--only allreduce needs torchrun with 2 or more GPUs")
        r = run_allreduce(device, world, rank)
        if rank == 0:
            print(json.dumps({"case": "allreduce", "tp_allreduce_rmsnorm": r}), flush=True)
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
        return 0
    if a.c5:
        r = run_llama70b_c5(device, world, rank)
        if rank == 0:
            print(json.dumps({"case": "C5", "llama70b_c5": r}), flush=True)
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
        return 0
    if a.only == "model":
        r = run_model_legs(a, device, world, rank)
        if rank == 0:
            print(json.dumps({"case": "model only", "n_gpus": world, **r}), flush=True)
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        return 0
    parity = run_parity(device, world, rank) if a.only == "all" else None
    kr = run_kernel(device, a.steps, a.warmup, seed=rank, pool_pages=a.pool_pages)
    if a.only == "kernel":
        if rank == 0:
            mean_ms = statistics.mean(kr["per_ms"])
            print(json.dumps({"case": "kernel only", "pool_pages": a.pool_pages,
                              "kernel_ms_mean": mean_ms,
                              "achieved_gbs": alg_bytes(kr["lens"]) / mean_ms / 1e6}), flush=True)
        if world > 1:
            torch.distributed.destroy_process_group()
        return 0
    e2e_steps = a.e2e_steps or max(10, a.steps // 2)
    er = run_e2e(device, e2e_steps, a.warmup, seed=rank)
    # the same steps with two in flight (host work of step i+1 under step i's kernels)
    overlap_err, ov_ms = None, -1.0
    try:
        ov_ms = run_e2e(device, e2e_steps, a.warmup, seed=rank, depth=2)["total_ms"]
    except Exception as e:       # reported in the line; the serial figure stands alone
        overlap_err = f"{type(e).__name__}: {e}"

    total_ms, e2e_ms = kr["total_ms"], er["total_ms"]
    if world > 1:
        t = torch.tensor([total_ms, e2e_ms, ov_ms], device=device, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms, e2e_ms, ov_ms = t.tolist()
    value = world * B * a.steps / (total_ms / 1e3)
    serial = {"value": world * B * e2e_steps / (e2e_ms / 1e3), "unit": "tok/s",
              "ms_per_step": e2e_ms / e2e_steps, "steps_in_flight": 1,
              "path": "one stream; each step's output on the host before the next step "
                      "begins"}
    if overlap_err is None and ov_ms > 0:
        # headline: two steps in flight, copies on copy streams (each step still copies
        # its own inputs up and its own output down inside the timed region)
        e2e = {"value": world * B * e2e_steps / (ov_ms / 1e3), "unit": "tok/s",
               "ms_per_step": ov_ms / e2e_steps, "steps_in_flight": 2,
               "path": "B200PagedKVCache.begin_forward -> CacheContext.attend -> "
                       "end_forward per step, pinned host q/k/v copied up and the output "
                       "copied down every step on two copy streams, step i+1 begun before "
                       "step i's output is read",
               "serial": serial}
    else:
        e2e = dict(serial, overlapped_error=overlap_err)
    e2e.update({"steps": e2e_steps, "h2d_bytes_per_step": er["h2d"],
                "d2h_bytes_per_step": er["d2h"]})
    mean_ms = statistics.mean(kr["per_ms"])
    ab = alg_bytes(kr["lens"])
    hbm, src = peaks()
    achieved = ab / (mean_ms / 1e3) / 1e9
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "decode_tc_c2_traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            traffic = json.load(f).get("dram_bytes_per_launch")
    line = {"metric": metric, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": total_ms / a.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) K/V, random page table over a 600k-page pool)",
            "config": config,
            "e2e": e2e,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "traffic": traffic,
                         "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)" if src ==
                         "measured" else "fallback 6650 GB/s",
                         "algorithmic_bytes_per_step": ab,
                         "kernel_ms_mean": mean_ms,
                         "kernel_ms_median": statistics.median(kr["per_ms"])},
            "gpu_launches": a.steps,
            "clocks": kr["clocks"]}
    line["parity"] = parity
    line["prefill_attention"] = run_prefill_kernel(device) if rank == 0 else None
    line["decode_model_shapes"] = run_decode_model_shapes(device) if rank == 0 else None
    if world > 1:
        torch.distributed.barrier()
    if not a.no_model:
        line.update(run_model_legs(a, device, world, rank))
    if a.only == "all" and world == 1 and not a.no_ref_backend:
        # last of the GPU legs: the library's kernels run after every leg of this repo
        line["reference_gpu_backend"] = run_reference_backend(device)
    if rank == 0 and not a.no_cpu:
        r = cpu_reference(a.cpu_seconds)
        line["cpu_baseline"] = {"value": r["value"], "unit": "tok/s", "cores": r["cores"],
                                "kind": "port", "sample": r["sample"]}
    if world > 1:
        torch.distributed.barrier()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
