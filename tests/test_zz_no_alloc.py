"""GPU test of nslg_paged_decode_noalloc, the decode entry point that allocates nothing.

It exists for callers that cannot allocate device memory (a serving process whose HBM is
all given to its KV page pool, a host program in another language binding the C ABI
without a device allocator, a loop that cannot take cudaMalloc's synchronisation). It must
give the same result as nslg_paged_decode, which uses a caller-provided workspace, and
keep giving it when called again: the fixed scratch array it uses still holds the previous
call's partials. Both entry points run the same kernels with the same split of the pages,
so the outputs must be bit-equal. This file is named so that pytest collects it last."""
import math

import pytest
import torch

from nanoslg_b200 import _native as N
from nanoslg_b200 import ops
from oracle.attention import attend_sequences
from paged_util import make_paged, sequence_kv

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
TOL = dict(rtol=1e-2, atol=2e-2)      # the bf16 attention tolerance of the other tests


def _noalloc(q, pk, out, status, page_size=16):
    hkv = pk["pool_k"].shape[2]
    return N.lib().nslg_paged_decode_noalloc(
        N.DTYPE_BF16, q.shape[0], q.shape[1], hkv, q.shape[2], page_size, q.data_ptr(),
        q.stride(0), out.data_ptr(), out.stride(0), pk["pool_k"].data_ptr(),
        pk["pool_v"].data_ptr(), pk["pool_k"].shape[0], pk["indptr"].data_ptr(),
        pk["indices"].data_ptr(), pk["lpl"].data_ptr(), 1 / math.sqrt(q.shape[2]),
        status.data_ptr(), torch.cuda.current_stream(DEV).cuda_stream)


def test_noalloc_decode_matches_workspace_entry_point_twice():
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    g = torch.Generator().manual_seed(77)
    # two calls in a row with different batches: the second reuses the scratch array
    for call, (nseq, hq, hkv) in enumerate([(40, 32, 8), (23, 16, 2)]):
        lens = torch.randint(1, 3000, (nseq,), generator=g).tolist()
        pk = make_paged(lens, hkv, 128, 20000, torch.bfloat16, DEV, seed=100 + call)
        q = torch.randn(nseq, hq, 128, generator=g).to(torch.bfloat16).to(DEV)
        ref = ops.paged_decode(q, pk["pool_k"], pk["pool_v"], pk["indptr"], pk["indices"],
                               pk["lpl"], 1 / math.sqrt(128))
        out = torch.full_like(q, float("nan"))
        rc = _noalloc(q, pk, out, status)
        assert rc == N.OK, N.lib().nslg_last_error()
        assert N.lib().nslg_last_error() == b""
        torch.cuda.synchronize(DEV)
        assert int(status.item()) == 0
        assert torch.equal(out, ref)


def test_noalloc_decode_cuda_core_branch_matches_oracle():
    """Page size 8 is not a tensor-core shape: the entry point runs the CUDA-core kernel,
    which needs no scratch."""
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    lens = [1, 9, 130, 517]
    pk = make_paged(lens, 2, 64, 200, torch.bfloat16, DEV, seed=5, page_size=8)
    q = torch.randn(len(lens), 8, 64, generator=torch.Generator().manual_seed(6)) \
        .to(torch.bfloat16).to(DEV)
    out = torch.full_like(q, float("nan"))
    rc = _noalloc(q, pk, out, status, page_size=8)
    assert rc == N.OK, N.lib().nslg_last_error()
    torch.cuda.synchronize(DEV)
    assert int(status.item()) == 0
    qc = q.cpu()
    for b in range(len(lens)):
        want = attend_sequences([qc[b:b + 1]], [sequence_kv(pk, b, "k")],
                                [sequence_kv(pk, b, "v")])[0][0]
        torch.testing.assert_close(out[b].cpu(), want, **TOL)


def test_noalloc_decode_rejects_batches_beyond_the_scratch():
    big = 4096                                      # needs ~71 MB of partials > 8 MiB
    pk = make_paged([1] * big, 8, 128, big + 8, torch.bfloat16, DEV, seed=1)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    q = torch.zeros(big, 32, 128, dtype=torch.bfloat16, device=DEV)
    out = torch.empty_like(q)
    rc = _noalloc(q, pk, out, status)
    assert rc == N.ERR_WORKSPACE
    assert b"scratch" in N.lib().nslg_last_error()
