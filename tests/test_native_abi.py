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


def test_ops_refuse_unsupported_dtypes():
    """bf16, fp16 and fp32 (the reference's activation types): anything else is refused,
    never converted."""
    import torch
    from nanoslg_b200 import ops
    assert ops._dtype_code(torch.zeros(1, dtype=torch.bfloat16)) == N.DTYPE_BF16
    assert ops._dtype_code(torch.zeros(1, dtype=torch.float16)) == N.DTYPE_F16
    assert ops._dtype_code(torch.zeros(1, dtype=torch.float32)) == N.DTYPE_F32
    for dt in (torch.float64, torch.int32, torch.float8_e4m3fn):
        with pytest.raises(TypeError, match="bfloat16, float16 and float32"):
            ops._dtype_code(torch.zeros(1, dtype=dt))


def test_tp_plan_and_ipc_argument_errors_without_gpu(lib):
    """The tensor-parallel reduction, the decode planner, page zeroing and the IPC helpers
    reject bad arguments on the host, before any CUDA call."""
    vp = ctypes.c_void_p
    stages = (vp * 2)(vp(16), vp(32))
    # world 1 is not a tensor-parallel group
    rc = lib.nslg_tp_allreduce_rmsnorm(N.DTYPE_BF16, 4, 4096, 1, 0, vp(16), 4096,
                                       ctypes.cast(stages, vp), 1 << 20, vp(16), vp(16), 4096,
                                       vp(16), vp(16), 4096, 1e-5, 10**9, None, None)
    assert rc == N.ERR_ARG and b"world" in lib.nslg_last_error()
    # stage buffers too small for the rows: 4 * world * rows * hidden * 2 bytes needed
    rc = lib.nslg_tp_allreduce_rmsnorm(N.DTYPE_BF16, 64, 4096, 2, 0, vp(16), 4096,
                                       ctypes.cast(stages, vp), 1 << 20, vp(16), vp(16), 4096,
                                       vp(16), vp(16), 4096, 1e-5, 10**9, None, None)
    assert rc == N.ERR_WORKSPACE and b"stage bytes" in lib.nslg_last_error()
    # rows longer than 16 KiB are not supported
    rc = lib.nslg_tp_allreduce_rmsnorm(N.DTYPE_BF16, 1, 16384, 2, 1, vp(16), 16384,
                                       ctypes.cast(stages, vp), 1 << 30, vp(16), vp(16), 16384,
                                       vp(16), vp(16), 16384, 1e-5, 10**9, None, None)
    assert rc == N.ERR_UNSUPPORTED
    # a non-positive wait limit would make every wait give up at once
    rc = lib.nslg_tp_allreduce_rmsnorm(N.DTYPE_BF16, 1, 4096, 2, 1, vp(16), 4096,
                                       ctypes.cast(stages, vp), 1 << 20, vp(16), vp(16), 4096,
                                       vp(16), vp(16), 4096, 1e-5, 0, None, None)
    assert rc == N.ERR_ARG and b"timeout" in lib.nslg_last_error()
    # the planner takes 1..4096 sequences
    args = [vp(16)] * 2 + [0, None, vp(16), 512, 64] + [vp(16)] * 7 + [1024, None, None]
    assert lib.nslg_plan_decode(0, 16, *args) == N.ERR_UNSUPPORTED
    assert lib.nslg_plan_decode(4097, 16, *args) == N.ERR_UNSUPPORTED
    assert lib.nslg_plan_decode(4, 0, *args) == N.ERR_ARG
    # page zeroing: nothing to do is fine, bad sizes are not
    assert lib.nslg_zero_pages(None, 0, None, 1, 1, 16, None, None) == N.OK
    assert lib.nslg_zero_pages(vp(16), 2, vp(16), 1, 64, 24, None, None) == N.ERR_ARG
    # one-call append + decode: batch 0 is a no-op, bad sizes are refused
    dec = lambda b, ps, wl: lib.nslg_append_paged_decode(
        N.DTYPE_BF16, b, 32, 8, 128, ps, vp(16), 4096, vp(16), 1024, vp(16), 1024, wl, vp(16),
        4096, vp(16), vp(16), 64, vp(16), vp(16), vp(16), 0.08, vp(16), 1 << 20, None, None)
    assert dec(0, 16, None) == N.OK
    assert dec(-1, 16, vp(16)) == N.ERR_ARG
    assert dec(4, 16, None) == N.ERR_ARG
    assert dec(4, 0, vp(16)) == N.ERR_ARG
    # greedy argmax: shapes, dtype and pointers are checked before any launch
    assert lib.nslg_argmax_rows(N.DTYPE_BF16, 0, 10, None, 10, 0, None, None, None) == N.OK
    assert lib.nslg_argmax_rows(7, 1, 10, vp(16), 10, 0, None, vp(16), None) == N.ERR_ARG
    assert lib.nslg_argmax_rows(N.DTYPE_BF16, -1, 10, vp(16), 10, 0, None, vp(16), None) == N.ERR_ARG
    assert lib.nslg_argmax_rows(N.DTYPE_BF16, 1, 0, vp(16), 10, 0, None, vp(16), None) == N.ERR_ARG
    assert lib.nslg_argmax_rows(N.DTYPE_BF16, 1, 10, vp(16), 9, 0, None, vp(16), None) == N.ERR_ARG
    assert lib.nslg_argmax_rows(N.DTYPE_BF16, 1, 10, vp(16), 10, 0, None, None, None) == N.ERR_ARG
    # the one-call planner from host arrays: same batch limits, its own argument checks
    # (all of them before any CUDA call)
    hbuf = (ctypes.c_int32 * 64)()
    h = ctypes.cast(hbuf, vp)
    hargs = lambda b, ps, nz, pk, pb, plan: (b, ps, h, h, 0, None, nz, h, pk, pk, 1, 64, pb,
                                             vp(16), 512, 64, plan, 1024, None, None)
    assert lib.nslg_plan_decode_host(*hargs(0, 16, 0, None, 16, vp(16))) == N.ERR_UNSUPPORTED
    assert lib.nslg_plan_decode_host(*hargs(4097, 16, 0, None, 16, vp(16))) == N.ERR_UNSUPPORTED
    assert lib.nslg_plan_decode_host(*hargs(4, 0, 0, None, 16, vp(16))) == N.ERR_ARG
    assert lib.nslg_plan_decode_host(*hargs(4, 16, 0, None, 16, None)) == N.ERR_ARG
    assert lib.nslg_plan_decode_host(*hargs(4, 16, -1, None, 16, vp(16))) == N.ERR_ARG
    assert lib.nslg_plan_decode_host(*hargs(4, 16, 2, None, 16, vp(16))) == N.ERR_ARG
    assert lib.nslg_plan_decode_host(*hargs(4, 16, 2, vp(16), 24, vp(16))) == N.ERR_ARG
    assert lib.nslg_plan_decode_host(*hargs(4, 16, 2, vp(8), 16, vp(16))) == N.ERR_ARG
    # IPC helpers
    ptr = vp()
    assert lib.nslg_ipc_alloc(0, ctypes.byref(ptr), ctypes.create_string_buffer(64)) == N.ERR_ARG
    assert lib.nslg_ipc_open(None, ctypes.byref(ptr)) == N.ERR_ARG


C_HOST = r"""
#include <stdio.h>
#include <string.h>
#include "nslg_b200.h"

/* A C99 host bound to the library the way another language's FFI would be: version,
 * host-side argument checks and the error text, no GPU needed. */
int main(void) {
  const char* v = nslg_version();
  if (v == NULL || strstr(v, "sm_100a") == NULL) return 2;
  int rc = nslg_rmsnorm_residual(7, 1, 16, NULL, 0, NULL, 0, NULL, NULL, 0, 1e-5f, NULL);
  if (rc != NSLG_ERR_ARG || strstr(nslg_last_error(), "dtype") == NULL) return 3;
  rc = nslg_paged_decode(NSLG_DTYPE_BF16, 2, 6, 4, 128, 16, NULL, 0, NULL, 0, NULL, NULL, 1,
                         NULL, NULL, NULL, 1.0f, NULL, 0, NULL, NULL);
  if (rc != NSLG_ERR_ARG || strstr(nslg_last_error(), "num_kv_heads") == NULL) return 4;
  rc = nslg_paged_decode(NSLG_DTYPE_BF16, 0, 32, 8, 128, 16, NULL, 0, NULL, 0, NULL, NULL, 1,
                         NULL, NULL, NULL, 1.0f, NULL, 0, NULL, NULL);
  if (rc != NSLG_OK) return 5;
  printf("c host ok: %s\n", v);
  return 0;
}
"""


def test_c_host_compiles_links_and_calls_the_abi(lib, tmp_path):
    """include/nslg_b200.h is plain C99 and the shared library links into a C program,
    whose calls behave as through ctypes."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    src = tmp_path / "host.c"
    src.write_text(C_HOST)
    libdir = os.path.join(ROOT, "nanoslg_b200", "lib")
    exe = tmp_path / "host"
    subprocess.run([gcc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror",
                    "-I", os.path.join(ROOT, "include"), str(src), "-L", libdir, "-lnslg_b200",
                    "-Wl,-rpath," + libdir, "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    assert "c host ok" in r.stdout and "sm_100a" in r.stdout


def _header_prototypes():
    """name -> (return type, [parameter types]) of every nslg_* prototype in include/*.h,
    types as written (qualifiers and pointer stars kept, parameter names dropped)."""
    out = {}
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        text = re.sub(r"^\s*#.*$", "", text, flags=re.M)
        for m in re.finditer(r"([A-Za-z_][\w\s\*]*?)\b(nslg_\w+)\s*\(([^)]*)\)\s*;", text):
            ret, name, params = " ".join(m.group(1).split()), m.group(2), m.group(3).strip()
            types = []
            if params and params != "void":
                for prm in params.split(","):
                    prm = " ".join(prm.split())
                    # drop the parameter name (the last identifier not followed by '*')
                    types.append(re.sub(r"\s*\b\w+$", "", prm).replace(" *", "*"))
            out[name] = (ret.replace(" *", "*"), types)
    return out


def _ctype_of(ctype_str):
    if ctype_str.endswith("*"):
        return "pointer"
    base = ctype_str.replace("const ", "")
    return {"int": ctypes.c_int, "int64_t": ctypes.c_int64, "float": ctypes.c_float,
            "uint32_t": ctypes.c_uint32, "size_t": ctypes.c_size_t}[base]


def test_binding_signatures_match_the_header_types():
    """Every parameter of every prototype has the ctypes type of its C type in
    nanoslg_b200._native.SIGNATURES (pointers as void*, char* or POINTER), in order, and
    the return types agree: a mismatch would pass arguments in the wrong registers."""
    protos = _header_prototypes()
    assert set(protos) == set(N.SIGNATURES), set(protos) ^ set(N.SIGNATURES)
    ptr_types = (ctypes.c_void_p, ctypes.c_char_p)
    for name, (ret, params) in protos.items():
        res, args = N.SIGNATURES[name]
        assert len(args) == len(params), (name, len(args), len(params))
        for i, (c, a) in enumerate(zip(params, args)):
            want = _ctype_of(c)
            if want == "pointer":
                assert a in ptr_types or (isinstance(a, type) and
                                          issubclass(a, ctypes._Pointer)), (name, i, c, a)
            else:
                assert a is want, (name, i, c, a)
        want_ret = _ctype_of(ret)
        if want_ret == "pointer":
            assert res in ptr_types, (name, ret, res)
        else:
            assert res is want_ret, (name, ret, res)
