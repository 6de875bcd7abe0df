"""float16 activations on the GPU (the reference's worker runs float16 as well as
bfloat16, worker.py:22-26): every kernel of the path in fp16, through the C ABI, against
the CPU oracle (itself pinned to fp16 outputs recorded from the reference,
tests/golden/fp16_cases.pt).

Tolerances: RoPE/KV append bit-exact (the reference's fp16 elementwise ops); attention
within the north star's 2e-2 abs / 1e-2 rel of the fp32 oracle over the same fp16
inputs; RMSNorm within one fp16 rounding of the rsqrt."""
import math
import os

import pytest
import torch

from conftest import GOLDEN
from oracle.attention import attend_sequences
from oracle.rope_norm import apply_rotary, rmsnorm, rope_table
from nanoslg_b200 import ops
from paged_util import make_paged, sequence_kv

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
TOL = dict(rtol=1e-2, atol=2e-2)
F16 = torch.float16


@pytest.fixture(autouse=True)
def _clean_status():
    ops.status_word(DEV).zero_()
    yield
    ops.check_device_status(DEV)


@pytest.mark.parametrize("hq,hkv,d", [(32, 8, 128), (8, 1, 64)])
def test_fp16_rope_kv_append_bit_exact(hq, hkv, d):
    g = torch.Generator().manual_seed(31)
    T, ps, P = 300, 16, 40
    cos, sin = rope_table(d, 8192, 500000.0)
    q = (torch.randn(T, hq, d, generator=g) * 4).to(F16)
    k = (torch.randn(T, hkv, d, generator=g) * 4).to(F16)
    v = torch.randn(T, hkv, d, generator=g).to(F16)
    pos = torch.randint(0, 8192, (T,), generator=g, dtype=torch.int32)
    loc = torch.randperm(P * ps, generator=g)[:T].to(torch.int32)
    loc[::7] = -1
    pk = torch.zeros((P, ps, hkv, d), dtype=F16, device=DEV)
    pv = torch.zeros_like(pk)
    q_out = ops.rope_kv_append(q.to(DEV), k.to(DEV), v.to(DEV), pos.to(DEV), cos.to(DEV),
                               sin.to(DEV), loc.to(DEV), pk, pv)
    p64 = pos.long()[None]
    assert torch.equal(q_out.cpu(), apply_rotary(q[None], cos[p64], sin[p64])[0])
    w = loc >= 0
    fk, fv = pk.view(-1, hkv, d).cpu(), pv.view(-1, hkv, d).cpu()
    assert torch.equal(fk[loc[w].long()], apply_rotary(k[None], cos[p64], sin[p64])[0][w])
    assert torch.equal(fv[loc[w].long()], v[w])


def test_fp16_rope_and_rmsnorm_on_the_reference_cases():
    gold = torch.load(os.path.join(GOLDEN, "fp16_cases.pt"))
    cos, sin = rope_table(128, 4096, 500000.0)
    r = gold["rope"]
    x = r["x"].reshape(-1, 4, 128)
    pos = r["pos"].reshape(-1).to(torch.int32)
    kv = x[:, :1].contiguous().to(DEV)
    pool = torch.zeros((2, 16, 1, 128), dtype=F16, device=DEV)
    nowrite = torch.full((x.shape[0],), -1, dtype=torch.int32, device=DEV)
    q_out = ops.rope_kv_append(x.to(DEV), kv, kv, pos.to(DEV), cos.to(DEV), sin.to(DEV),
                               nowrite, pool, pool.clone())
    assert torch.equal(q_out.cpu().reshape(r["y"].shape), r["y"])
    for key in ("rmsnorm", "addnorm"):
        c = gold[key]
        xd = c["x"].to(DEV)
        if key == "addnorm":
            res = c["r"].to(DEV).clone()
            y = ops.rmsnorm_residual(xd, c["w"].to(DEV), c["eps"], residual=res)
            assert torch.equal(res.cpu(), c["h"])
        else:
            y = ops.rmsnorm_residual(xd, c["w"].to(DEV), c["eps"])
        want = c["y"].float()
        assert bool(((y.cpu().float() - want).abs() <= want.abs() * 2 ** -10 + 1e-6).all())


@pytest.mark.parametrize("hq,hkv,d", [(32, 8, 128), (8, 2, 64), (32, 1, 128)])
def test_fp16_paged_decode_tensor_cores(hq, hkv, d):
    g = torch.Generator().manual_seed(41)
    lens = torch.randint(1, 2500, (37,), generator=g).tolist()
    pk = make_paged(lens, hkv, d, 8000, F16, DEV, seed=42)
    q = torch.randn(len(lens), hq, d, generator=g).to(F16)
    out = ops.paged_decode(q.to(DEV), pk["pool_k"], pk["pool_v"], pk["indptr"], pk["indices"],
                           pk["lpl"], 1 / math.sqrt(d)).cpu()
    assert out.dtype == F16
    for b in range(len(lens)):
        want = attend_sequences([q[b:b + 1]], [sequence_kv(pk, b, "k")],
                                [sequence_kv(pk, b, "v")])[0][0]
        torch.testing.assert_close(out[b], want, **TOL)


def test_fp16_causal_prefill_tensor_cores():
    g = torch.Generator().manual_seed(43)
    hq, hkv, d = 32, 8, 128
    qo = [300, 129, 1, 64]
    prefix = [0, 40, 500, 0]
    lens = [a + b for a, b in zip(qo, prefix)]
    pk = make_paged(lens, hkv, d, 400, F16, DEV, seed=44)
    q = torch.randn(sum(qo), hq, d, generator=g).to(F16)
    qo_indptr = torch.tensor([0] + torch.cumsum(torch.tensor(qo), 0).tolist(), dtype=torch.int32)
    out = ops.paged_prefill(q.to(DEV), qo_indptr.to(DEV), max(qo), pk["pool_k"], pk["pool_v"],
                            pk["indptr"], pk["indices"], pk["lpl"], 1 / math.sqrt(d),
                            causal=True).cpu()
    for b in range(len(qo)):
        lo, hi = int(qo_indptr[b]), int(qo_indptr[b + 1])
        want = attend_sequences([q[lo:hi]], [sequence_kv(pk, b, "k")],
                                [sequence_kv(pk, b, "v")])[0]
        torch.testing.assert_close(out[lo:hi], want, **TOL)


def test_fp16_silu_mul_and_argmax():
    g = torch.Generator().manual_seed(45)
    gu = (torch.randn(33, 2 * 1024, generator=g) * 3).to(F16)
    got = ops.silu_mul(gu.to(DEV)).cpu()
    want = torch.nn.functional.silu(gu[:, :1024].float()).to(F16).float() * gu[:, 1024:].float()
    assert torch.equal(got, want.to(F16))
    logits = torch.randn(17, 5000, generator=g).to(F16)
    logits[3, 100] = logits[3, 4000] = 70.0          # a tie goes to the lower index
    idx = ops.argmax_rows(logits.to(DEV)).cpu()
    assert torch.equal(idx, logits.argmax(-1))


def test_fp16_cuda_core_fallback_shape():
    """A shape the tensor-core kernels do not cover (page size 8) runs the CUDA-core
    kernel in fp16."""
    g = torch.Generator().manual_seed(47)
    lens = [5, 77, 300]
    pk = make_paged(lens, 2, 64, 100, F16, DEV, seed=48, page_size=8)
    q = torch.randn(len(lens), 4, 64, generator=g).to(F16)
    out = ops.paged_decode(q.to(DEV), pk["pool_k"], pk["pool_v"], pk["indptr"], pk["indices"],
                           pk["lpl"], 1 / math.sqrt(64)).cpu()
    for b in range(len(lens)):
        want = attend_sequences([q[b:b + 1]], [sequence_kv(pk, b, "k")],
                                [sequence_kv(pk, b, "v")])[0][0]
        torch.testing.assert_close(out[b], want, **TOL)
