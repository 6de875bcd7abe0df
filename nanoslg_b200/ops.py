"""Torch-tensor wrappers over the C ABI (``include/nslg_b200.h``).

Each op checks devices, dtypes and layouts, passes raw pointers and the current CUDA
stream to the native library, and raises on any non-zero status.  Nothing here
computes on the CPU: the ops need CUDA tensors and the built library.
"""
import os
import threading

import torch
import torch.nn.functional as F

from . import _native as N

_DTYPES = {torch.bfloat16: N.DTYPE_BF16, torch.float16: N.DTYPE_F16, torch.float32: N.DTYPE_F32}


def _dtype_code(t):
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise TypeError(f"nanoslg_b200 kernels support bfloat16, float16 and float32, got {t.dtype}")


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("nanoslg_b200 kernels need CUDA tensors (no CPU path)")


def _ptr(t):
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(t):
    """cudaStream_t of the current stream of t's device (the raw handle when torch
    exposes it, which avoids building a Stream object per launch)."""
    if _raw_stream is not None:
        return _raw_stream(t.device.index if t.device.index is not None
                           else torch.cuda.current_device())
    return torch.cuda.current_stream(t.device).cuda_stream


def _rows(x, name):
    """Views ``x`` ([..., H, D] with contiguous heads) as rows: returns (rows, stride)."""
    if x.dim() < 2 or x.stride(-1) != 1 or x.stride(-2) != x.shape[-1]:
        raise ValueError(f"{name}: heads and head_dim must be contiguous, got strides {x.stride()}")
    n = 1
    for s in x.shape[:-2]:
        n *= s
    # the leading dims must collapse into one row index with a single stride; size-1 dims
    # carry no stride information (views give them arbitrary strides) and are skipped
    dims = [(x.shape[i], x.stride(i)) for i in range(x.dim() - 2) if x.shape[i] != 1]
    if not dims:
        return n, x.shape[-1] * x.shape[-2]
    stride = dims[-1][1]
    expect = stride
    for size, st in reversed(dims):
        if st != expect:
            raise ValueError(f"{name}: leading dims do not form one row stride {x.stride()}")
        expect *= size
    return n, stride


class _DeviceState:
    """Per-device scratch: the decode workspace and the device status word."""

    def __init__(self):
        self.lock = threading.Lock()
        self.ws = {}
        self.status = {}

    def workspace(self, device, nbytes):
        """The decode workspace: zeroed when allocated (the kernel's arrival counts at its
        head must start at zero; every call leaves them zero)."""
        buf = self.ws.get(device)
        if buf is not None and buf.numel() >= nbytes:
            return buf
        with self.lock:
            buf = self.ws.get(device)
            if buf is None or buf.numel() < nbytes:
                buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
                self.ws[device] = buf
            return buf

    def status_word(self, device):
        st = self.status.get(device)
        if st is not None:
            return st
        with self.lock:
            st = self.status.get(device)
            if st is None:
                st = torch.zeros(1, dtype=torch.int32, device=device)
                self.status[device] = st
            return st


_STATE = _DeviceState()


def status_word(device):
    """The int32 device word the kernels OR their NSLG_DEV_* error bits into."""
    if not isinstance(device, torch.device):
        device = torch.device(device)
    if device.index is None and device.type == "cuda":
        device = torch.device("cuda", torch.cuda.current_device())
    return _STATE.status_word(device)


def check_device_status(device, reset=True):
    """Synchronises and raises RuntimeError if a kernel on ``device`` flagged an error."""
    st = status_word(device)
    v = int(st.item())
    if reset and v:
        st.zero_()
    if v:
        names = [n for bit, n in ((N.DEV_BAD_PAGE, "page id outside the pool"),
                                  (N.DEV_BAD_SLOT, "write slot outside the pool"),
                                  (N.DEV_BAD_POSITION, "position outside the RoPE table"),
                                  (N.DEV_WAIT_TIMEOUT, "pipeline wait timed out"),
                                  (N.DEV_BAD_PLAN, "plan entry outside the device block "
                                                   "tables")) if v & bit]
        raise RuntimeError("nanoslg_b200 device error: " + ", ".join(names))


def rope_kv_append(q, k, v, positions, cos, sin, write_loc, pool_k, pool_v, q_out=None,
                   rotate=True):
    """Rotates q and k (rotate-half RoPE) and appends rotated k and plain v to the pool.

    q: [..., Hq, D]; k, v: [..., Hkv, D] with the same leading token dims;
    positions: int32 [T] (row of the cos/sin tables per token);
    write_loc: int32 [T] flat slot page*page_size+slot, -1 = do not write;
    pool_k / pool_v: one layer of the pool, [num_pages, page_size, Hkv, D].
    Returns q_out ([T, Hq, D], rotated q), or None when q is None.
    With ``rotate=False`` q and k are taken as already rotated (positions ignored).
    """
    _need_cuda(q, k, v, positions, cos, sin, write_loc, pool_k, pool_v)
    dt = _dtype_code(k)
    nk, ks = _rows(k, "k")
    nv, vs = _rows(v, "v")
    hkv, d = k.shape[-2], k.shape[-1]
    if nk != nv:
        raise ValueError("k and v token counts differ")
    qs, hq = 0, hkv
    if q is not None:
        nq, qs = _rows(q, "q")
        hq = q.shape[-2]
        if nq != nk or q.dtype != k.dtype:
            raise ValueError("q must match k in token count and dtype")
        if q_out is None:
            q_out = torch.empty((nq, hq, d), dtype=q.dtype, device=q.device)
    if pool_k.dtype != k.dtype or pool_v.dtype != k.dtype:
        raise TypeError("pool dtype must match k/v")
    if not (pool_k.is_contiguous() and pool_v.is_contiguous()):
        raise ValueError("pool layers must be contiguous")
    slots = pool_k.shape[0] * pool_k.shape[1]
    if write_loc is not None and (write_loc.dtype != torch.int32 or write_loc.numel() != nk):
        raise ValueError("write_loc must be int32 with one entry per token")
    if rotate:
        if positions is None or positions.dtype != torch.int32 or positions.numel() != nk:
            raise ValueError("positions must be int32 with one entry per token")
        if cos.dtype != torch.float32 or not cos.is_contiguous() or not sin.is_contiguous():
            raise ValueError("cos/sin tables must be contiguous float32 [rows, D]")
        rows = cos.shape[0]
    else:
        positions = cos = sin = None
        rows = 0
    N.call("nslg_rope_kv_append", dt, nk, hq, hkv, d, _ptr(q), qs, _ptr(k), ks, _ptr(v), vs,
           _ptr(q_out), _ptr(positions), _ptr(cos), _ptr(sin), rows, _ptr(write_loc),
           _ptr(pool_k), _ptr(pool_v), slots, _ptr(status_word(k.device)), _stream(k))
    return q_out


def paged_decode(q, pool_k, pool_v, kv_indptr, kv_indices, kv_last_page_len, sm_scale,
                 out=None):
    """Decode attention, one query per sequence. q: [B, Hq, D] -> out [B, Hq, D]."""
    _need_cuda(q, pool_k, pool_v, kv_indptr, kv_indices, kv_last_page_len)
    dt = _dtype_code(q)
    nb, qs = _rows(q, "q")
    hq, d = q.shape[-2], q.shape[-1]
    num_pages, ps, hkv = pool_k.shape[0], pool_k.shape[1], pool_k.shape[2]
    if out is None:
        out = torch.empty((nb, hq, d), dtype=q.dtype, device=q.device)
    _, os_ = _rows(out, "out")
    for t in (kv_indptr, kv_indices, kv_last_page_len):
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise ValueError("CSR arrays must be contiguous int32")
    wsb = N.lib().nslg_decode_workspace_bytes(nb, hq, d)
    ws = _STATE.workspace(q.device, wsb)
    N.call("nslg_paged_decode", dt, nb, hq, hkv, d, ps, _ptr(q), qs, _ptr(out), os_,
           _ptr(pool_k), _ptr(pool_v), num_pages, _ptr(kv_indptr), _ptr(kv_indices),
           _ptr(kv_last_page_len), float(sm_scale), _ptr(ws), ws.numel(),
           _ptr(status_word(q.device)), _stream(q))
    return out


# Decode batches of at most this many (sequence, kv head) pairs take the split-heads path
# in the paged context (the work split by kv head as well as by pages). Off by default:
# alone it is faster (one B200, 32 decode calls per CUDA graph, us per layer, plain ->
# split: TP=1 batch 1, 512 tokens, 8.9 -> 7.3; TP=4 batch 1 10.0 -> 6.8; TP=1 batch 8
# 15.4 -> 13.6; TP=2 batch 16 20.4 -> 16.7; slower from 128 pairs: TP=1 batch 16 20.8 ->
# 23.8), but inside the 8B decode step, between the q|k|v and o_proj products, it was
# slower (same-box A/B: batch 1 3.17-3.20 -> 3.27 ms per step, batch 4 3.27-3.30 ->
# 3.31-3.35). NSLG_DECODE_SPLIT_HEADS=1 (read at import) enables it up to 64 pairs.
_SPLIT_ENV = os.environ.get("NSLG_DECODE_SPLIT_HEADS")
DECODE_SPLIT_HEADS_PAIRS = 64 if _SPLIT_ENV == "1" else 0


def split_heads_plan(kv_indptr, kv_indices, kv_last_page_len, hkv, num_pages):
    """The page list of ``paged_decode_split_heads`` from a decode plan's CSR (int32 device
    arrays): returns (v_indptr, v_indices, v_last_page_len) for batch * hkv sequences, one
    per (sequence, kv head), page ids page * hkv + head (nslg_split_heads_plan)."""
    _need_cuda(kv_indptr, kv_indices, kv_last_page_len)
    batch = kv_indptr.numel() - 1
    dev = kv_indptr.device
    v_indptr = torch.empty(batch * hkv + 1, dtype=torch.int32, device=dev)
    v_indices = torch.empty(max(hkv * kv_indices.numel(), 1), dtype=torch.int32, device=dev)
    v_lpl = torch.empty(batch * hkv, dtype=torch.int32, device=dev)
    N.call("nslg_split_heads_plan", batch, hkv, _ptr(kv_indptr), _ptr(kv_indices),
           _ptr(kv_last_page_len), _ptr(v_indptr), _ptr(v_indices), _ptr(v_lpl),
           v_indices.numel(), int(num_pages), _ptr(status_word(dev)), _stream(kv_indptr))
    return v_indptr, v_indices, v_lpl


def paged_decode_split_heads(q, pool_k, pool_v, split_plan, sm_scale, out=None):
    """``paged_decode`` with the work split by kv head as well as by pages
    (nslg_paged_decode_split_heads): q contiguous [B, Hq, D] -> out [B, Hq, D];
    ``split_plan`` from ``split_heads_plan``. The same attention within fp32 rounding
    of the merge order."""
    _need_cuda(q, pool_k, pool_v)
    dt = _dtype_code(q)
    if q.dim() != 3 or not q.is_contiguous():
        raise ValueError("paged_decode_split_heads: q must be contiguous [B, Hq, D]")
    b, hq, d = q.shape
    num_pages, ps, hkv = pool_k.shape[0], pool_k.shape[1], pool_k.shape[2]
    if out is None:
        out = torch.empty_like(q)
    v_indptr, v_indices, v_lpl = split_plan
    wsb = N.lib().nslg_decode_workspace_bytes(b * hkv, hq // hkv, d)
    ws = _STATE.workspace(q.device, wsb)
    N.call("nslg_paged_decode_split_heads", dt, b, hq, hkv, d, ps, _ptr(q), _ptr(out),
           _ptr(pool_k), _ptr(pool_v), num_pages, _ptr(v_indptr), _ptr(v_indices), _ptr(v_lpl),
           float(sm_scale), _ptr(ws), ws.numel(), _ptr(status_word(q.device)), _stream(q))
    return out


def paged_prefill(q, qo_indptr, max_qo_len, pool_k, pool_v, kv_indptr, kv_indices,
                  kv_last_page_len, sm_scale, causal=True, q_row_start=None, out=None):
    """Causal prefill/extend attention over the paged KV.

    q: [rows, Hq, D] (or [B, S, Hq, D], viewed as rows); sequence b's qo_len rows start at
    row q_row_start[b] (default qo_indptr[b]).  out has q's row layout; rows that belong
    to no sequence are left as they are (zero them first if they must read as zero).
    """
    _need_cuda(q, qo_indptr, pool_k, pool_v, kv_indptr, kv_indices, kv_last_page_len,
               q_row_start)
    dt = _dtype_code(q)
    nrows, qs = _rows(q, "q")
    hq, d = q.shape[-2], q.shape[-1]
    num_pages, ps, hkv = pool_k.shape[0], pool_k.shape[1], pool_k.shape[2]
    if out is None:
        out = torch.zeros(q.shape, dtype=q.dtype, device=q.device)
    _, os_ = _rows(out, "out")
    batch = qo_indptr.numel() - 1
    N.call("nslg_paged_prefill", dt, batch, hq, hkv, d, ps, _ptr(q), qs, nrows, _ptr(out), os_,
           _ptr(qo_indptr), _ptr(q_row_start), int(max_qo_len), _ptr(pool_k), _ptr(pool_v),
           num_pages, _ptr(kv_indptr), _ptr(kv_indices), _ptr(kv_last_page_len),
           float(sm_scale), 1 if causal else 0, _ptr(status_word(q.device)), _stream(q))
    return out


def rmsnorm_residual(x, weight, eps, residual=None, out=None):
    """out = rmsnorm(x [+ residual]) * weight; with a residual, residual <- x + residual."""
    _need_cuda(x, weight, residual, out)
    dt = _dtype_code(x)
    hidden = x.shape[-1]
    if x.stride(-1) != 1 or weight.dtype != x.dtype or weight.numel() != hidden:
        raise ValueError("rmsnorm_residual: bad layout or weight")
    rows = x.numel() // hidden
    x2 = x.reshape(rows, hidden)
    if out is None:
        out = torch.empty_like(x2)
    out2 = out.view(rows, hidden)
    r2 = None
    if residual is not None:
        r2 = residual.view(rows, hidden)
    N.call("nslg_rmsnorm_residual", dt, rows, hidden, _ptr(x2), x2.stride(0), _ptr(r2),
           r2.stride(0) if r2 is not None else 0, _ptr(weight), _ptr(out2), out2.stride(0),
           float(eps), _stream(x))
    return out.view(x.shape)


def silu_mul(gate_up, out=None):
    """silu(gate) * up of a fused [..., 2*I] gate|up tensor -> [..., I]."""
    _need_cuda(gate_up, out)
    dt = _dtype_code(gate_up)
    two_i = gate_up.shape[-1]
    inter = two_i // 2
    if gate_up.stride(-1) != 1 or two_i % 2:
        raise ValueError("silu_mul: last dim must be contiguous and even")
    rows = gate_up.numel() // two_i
    g2 = gate_up.reshape(rows, two_i)
    if out is None:
        out = torch.empty(gate_up.shape[:-1] + (inter,), dtype=gate_up.dtype,
                          device=gate_up.device)
    o2 = out.view(rows, inter)
    N.call("nslg_silu_mul", dt, rows, inter, _ptr(g2), g2.stride(0), _ptr(o2), o2.stride(0),
           _stream(gate_up))
    return out


LINEAR_MAX_ROWS = 256     # what nslg_linear accepts
# What ``linear`` sends the kernel by default: batches of up to LINEAR_AUTO_ROWS rows, and
# of up to LINEAR_WIDE_ROWS rows for products of at least LINEAR_WIDE_BYTES of weights
# (at 64 rows the kernel is level with or ahead of cuBLAS on the 8B model's TP=1 gate|up
# and down products, 235 and 117 MB, and behind on the narrower ones). NSLG_LINEAR_ROWS
# (read at import, 1 to LINEAR_MAX_ROWS) replaces both limits, for measurements.
_ROWS_ENV = os.environ.get("NSLG_LINEAR_ROWS")
LINEAR_AUTO_ROWS = max(1, min(int(_ROWS_ENV or "16"), 256))
LINEAR_WIDE_ROWS = LINEAR_AUTO_ROWS if _ROWS_ENV else 64
LINEAR_WIDE_BYTES = 96 << 20


def auto_rows(weight):
    """The default row limit of ``linear`` / ``linear_swiglu`` / ``linear_rope_append``
    for this weight."""
    big = weight.numel() * weight.element_size() >= LINEAR_WIDE_BYTES
    return LINEAR_WIDE_ROWS if big else LINEAR_AUTO_ROWS


def linear_supported(x, weight, bias=None, max_rows=LINEAR_MAX_ROWS):
    """Whether the tcgen05 kernel takes these operands: CUDA bf16 / fp16 x and weight of
    one type, no bias, at most ``max_rows`` rows of x, in_features a multiple of 64, rows
    of x and weight contiguous and 16-byte aligned."""
    if bias is not None or not (x.is_cuda and weight.is_cuda):
        return False
    if x.dtype not in (torch.bfloat16, torch.float16) or weight.dtype != x.dtype:
        return False
    k = x.shape[-1]
    if weight.dim() != 2 or weight.shape[1] != k or k % 64 or x.stride(-1) != 1:
        return False
    if weight.stride(1) != 1 or weight.stride(0) % 8 or weight.data_ptr() % 16:
        return False
    rows = x.numel() // k if k else 0
    return 1 <= rows <= max_rows


def linear(x, weight, bias=None, out=None, max_rows=None):
    """F.linear(x, weight, bias): the tcgen05 kernel (nslg_linear) for forwards of at most
    ``max_rows`` rows (``linear_supported``), the cuBLAS GEMM of F.linear for the rest.
    The default (``auto_rows``) sends the kernel the small decode batches (up to 16 rows),
    where it streams the weights faster than cuBLAS on the 8B model's shapes at every TP
    degree, and batches of up to 64 rows on the largest products; prefill, fp32 and
    biased layers stay cuBLAS."""
    if max_rows is None:
        max_rows = auto_rows(weight)
    if not linear_supported(x, weight, bias, max_rows):
        return F.linear(x, weight, bias)
    k, n = x.shape[-1], weight.shape[0]
    try:
        rows, xs = _rows(x.unsqueeze(-2), "x")
    except ValueError:                     # leading dims that do not form one row stride
        return F.linear(x, weight, bias)
    if xs % 8 or x.data_ptr() % 16:
        return F.linear(x, weight, bias)
    if out is None:
        out = torch.empty(x.shape[:-1] + (n,), dtype=x.dtype, device=x.device)
    _, ys = _rows(out.unsqueeze(-2), "out")
    N.call("nslg_linear", _dtype_code(x), rows, n, k, _ptr(x), xs, _ptr(weight),
           weight.stride(0), _ptr(out), ys, _ptr(status_word(x.device)), _stream(x))
    return out


def linear_swiglu(x, gate_up, max_rows=None):
    """silu(x . gate^T) * (x . up^T) for a stacked [gate; up] weight ([2 I, in]): the
    tcgen05 linear kernel with the activation in its epilogue (nslg_linear_swiglu) where
    ``linear_supported(x, gate_up)`` holds; ``silu_mul(linear(x, gate_up))`` otherwise,
    and where the kernel reports that the shape's split-K sum would not be pushed. Both
    give the same values: each product rounded to the activation type, silu rounded, the
    product rounded."""
    if max_rows is None:
        max_rows = auto_rows(gate_up)
    two_i = gate_up.shape[0]
    if two_i % 2 or not linear_supported(x, gate_up, None, max_rows):
        return silu_mul(linear(x, gate_up, max_rows=max_rows))
    k, inter = x.shape[-1], two_i // 2
    try:
        rows, xs = _rows(x.unsqueeze(-2), "x")
    except ValueError:
        return silu_mul(linear(x, gate_up, max_rows=max_rows))
    if xs % 8 or x.data_ptr() % 16:
        return silu_mul(linear(x, gate_up, max_rows=max_rows))
    out = torch.empty(x.shape[:-1] + (inter,), dtype=x.dtype, device=x.device)
    lib = N.lib()
    rc = lib.nslg_linear_swiglu(_dtype_code(x), rows, inter, k, _ptr(x), xs, _ptr(gate_up),
                                gate_up.stride(0), _ptr(out), inter,
                                _ptr(status_word(x.device)), _stream(x))
    if rc == N.ERR_UNSUPPORTED:
        return silu_mul(linear(x, gate_up, max_rows=max_rows), out=out)
    if rc != N.OK:
        raise N.NativeError("nslg_linear_swiglu", rc,
                            lib.nslg_last_error().decode(errors="replace"))
    return out


def linear_rope_append(x, w_qkv, hq, hkv, positions, cos, sin, write_loc, pool_k, pool_v,
                       max_rows=None):
    """The q|k|v product of x with a stacked [q; k; v] weight, then rope_kv_append's
    RoPE and KV append, in one kernel (nslg_linear_rope_append): returns the rotated q
    ([rows, hq, 128]) after k and v went to the pool slots ``write_loc``. Returns None
    where that kernel does not take the operands (head_dim other than 128, more than
    ``max_rows`` rows, a split-K sum it would not push, ...); the caller then runs
    ``linear`` and ``rope_kv_append``, which give the same values."""
    if max_rows is None:
        max_rows = auto_rows(w_qkv)
    d = pool_k.shape[-1]
    if (d != 128 or w_qkv.shape[0] != (hq + 2 * hkv) * d
            or not linear_supported(x, w_qkv, None, max_rows)):
        return None
    if (pool_k.dtype != x.dtype or pool_v.dtype != x.dtype or not pool_k.is_contiguous()
            or not pool_v.is_contiguous() or pool_k.shape[-2] != hkv):
        return None
    try:
        rows, xs = _rows(x.unsqueeze(-2), "x")
    except ValueError:
        return None
    if xs % 8 or x.data_ptr() % 16:
        return None
    if (positions is None or positions.dtype != torch.int32 or positions.numel() != rows
            or write_loc is None or write_loc.dtype != torch.int32 or write_loc.numel() != rows
            or cos.dtype != torch.float32 or not cos.is_contiguous() or not sin.is_contiguous()):
        return None
    q_out = torch.empty((rows, hq, d), dtype=x.dtype, device=x.device)
    lib = N.lib()
    rc = lib.nslg_linear_rope_append(
        _dtype_code(x), rows, hq, hkv, d, x.shape[-1], _ptr(x), xs, _ptr(w_qkv),
        w_qkv.stride(0), _ptr(q_out), _ptr(positions), _ptr(cos), _ptr(sin), cos.shape[0],
        _ptr(write_loc), _ptr(pool_k), _ptr(pool_v), pool_k.shape[0] * pool_k.shape[1],
        _ptr(status_word(x.device)), _stream(x))
    if rc == N.ERR_UNSUPPORTED:
        return None
    if rc != N.OK:
        raise N.NativeError("nslg_linear_rope_append", rc,
                            lib.nslg_last_error().decode(errors="replace"))
    return q_out


def argmax_rows(x, index_offset=0, values=False):
    """Per row of ``x`` [rows, cols] (last dim contiguous): the index of the first
    maximum plus ``index_offset`` (int64 [rows]), ordered as torch.argmax (NaN above
    every number, ties to the lowest index); with ``values`` also the maxima (fp32)."""
    _need_cuda(x)
    if x.dim() != 2 or x.stride(-1) != 1:
        raise ValueError("argmax_rows: x must be [rows, cols] with contiguous rows")
    rows, cols = x.shape
    idx = torch.empty(rows, dtype=torch.int64, device=x.device)
    val = torch.empty(rows, dtype=torch.float32, device=x.device) if values else None
    N.call("nslg_argmax_rows", _dtype_code(x), rows, cols, _ptr(x), x.stride(0),
           int(index_offset), _ptr(val), _ptr(idx), _stream(x))
    return (idx, val) if values else idx
