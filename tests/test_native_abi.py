"""The C-ABI library loads without a GPU and exports what include/*.h declares."""
import ctypes
import glob
import os
import re

import pytest

from conftest import ROOT
from nanoslg_b200 import _native as N
from nanoslg_b200 import build


@pytest.fixture(scope="module")
def lib():
    build.build()
    return N.lib()


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        names |= set(re.findall(r"\b(nslg_\w+)\s*\(", text))
    return names


def test_every_declared_symbol_is_exported(lib):
    declared = _declared()
    assert {"nslg_paged_decode", "nslg_paged_prefill", "nslg_rope_kv_append",
            "nslg_rmsnorm_residual"} <= declared
    for name in declared:
        assert hasattr(lib, name), name
    # and every declared symbol has a ctypes signature in the binding
    assert declared <= set(N.SIGNATURES)


def test_version_and_argument_errors_without_gpu(lib):
    assert "sm_100a" in N.version()
    # rejected on the host before any CUDA call
    rc = lib.nslg_rmsnorm_residual(7, 1, 16, None, 0, None, 0, None, None, 0, 1e-5, None)
    assert rc == N.ERR_ARG
    assert b"dtype" in lib.nslg_last_error()
    rc = lib.nslg_paged_decode(N.DTYPE_BF16, 2, 6, 4, 128, 16, None, 0, None, 0, None, None, 1,
                               None, None, None, 1.0, None, 0, None, None)
    assert rc == N.ERR_ARG and b"num_kv_heads" in lib.nslg_last_error()
    with pytest.raises(N.NativeError):
        N.call("nslg_paged_prefill", N.DTYPE_F32, 1, 4, 2, 64, 16, None, 0, 1, None, 0, None,
               None, 4, None, None, 1, None, None, None, 0.125, 1, None, None)
    # batch 0 is a no-op
    assert lib.nslg_paged_decode(N.DTYPE_BF16, 0, 32, 8, 128, 16, None, 0, None, 0, None, None,
                                 1, None, None, None, 1.0, None, 0, None, None) == N.OK


def test_ops_refuse_cpu_tensors(lib):
    import torch
    from nanoslg_b200 import ops
    x = torch.zeros(2, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.rmsnorm_residual(x, torch.ones(16), 1e-5)
