"""Peer-memory tensor-parallel reduction fused with the residual add and RMSNorm.

In the reference every RowParallelLinear (o_proj, down_proj) ends with an NCCL SUM
all-reduce (tp_layers.py:148-158 -> parallel.py:167-172), after which the block adds
the residual and applies the next RMSNorm (models.py:169-172).  ``PeerAllReduce`` does
the three in one kernel (``nslg_tp_allreduce_rmsnorm``) over buffers that every rank of
the TP group maps from every other rank with CUDA IPC (plain NVLink peer stores, no
multicast objects).  The model marks forwards whose rows fit the buffers
(decode steps) ``active``; larger forwards (prefill) keep the NCCL all-reduce.  For
decode batches the tcgen05 linear kernel takes, the RowParallel GEMM itself pushes its
output rows to the peers (``linear_push``, one kernel for the product and the
collective's transfer) and the reduction kernel only gathers, sums and normalises.

Every rank of the group has to run the same sequence of calls with the same row
counts, as the TP ranks of the reference already do (they run the same forward on the
same broadcast token ids).
"""
import ctypes
import os

import torch
import torch.distributed as dist

from . import _native as N
from . import ops


# Rows up to which, and group sizes from which, the RowParallel GEMM pushes its own rows.
# Measured on B200s (o_proj shard, then the reduction + RMSNorm, CUDA-graph loops, max
# over ranks): TP=4, 1 row 11.0 us fused against 11.6 separate, 16 rows 14.8 against
# 14.2; TP=2, 1 row 10.4 against 10.0, 4 rows 10.9 against 10.4.
FUSED_PUSH_MAX_ROWS = 4
FUSED_PUSH_MIN_WORLD = 4


class PeerAllReduce:
    """One TP group's peer buffers (per rank a stage buffer of two slots x ``world``
    sources x ``max_rows`` packed rows, mapped by every peer, and private call counters)
    and the fused call."""

    def __init__(self, group, rank, world, device, max_rows, hidden, dtype,
                 timeout_s=10.0):
        if not 2 <= world <= N.TP_MAX_WORLD:
            raise ValueError(f"PeerAllReduce: world must be in [2, {N.TP_MAX_WORLD}]")
        if dtype not in (torch.bfloat16, torch.float16, torch.float32):
            raise TypeError("PeerAllReduce supports bfloat16, float16 and float32 activations")
        self.group, self.rank, self.world = group, rank, world
        self.device = torch.device(device)
        self.max_rows, self.hidden, self.dtype = max_rows, hidden, dtype
        self.timeout_ns = int(timeout_s * 1e9)
        esz = torch.tensor([], dtype=dtype).element_size()
        self.stage_bytes = 4 * world * max_rows * hidden * esz
        self.active = False
        # RowParallel products of decode batches the tcgen05 linear kernel takes push their
        # partial rows to the peers from inside the GEMM (nslg_linear_tp_push);
        # NSLG_TP_FUSED_PUSH=0 keeps the push in the reduction kernel instead
        self.fuse_push = os.environ.get("NSLG_TP_FUSED_PUSH", "1") != "0"
        self._pushed_ptr = None        # the partial whose rows were pushed by the GEMM
        self._own, self._opened = [], []
        with torch.cuda.device(self.device):
            stage, h_stage = self._alloc(self.stage_bytes)
            handles = [None] * world
            dist.all_gather_object(handles, h_stage, group=group)
            stage_ptrs = [stage if i == rank else self._open(h) for i, h in enumerate(handles)]
        self._stage_arr = (ctypes.c_void_p * world)(*stage_ptrs)
        self.counters = torch.zeros(N.TP_COUNTER_BYTES // 4, dtype=torch.int32,
                                    device=self.device)
        self.status = ops.status_word(self.device)
        dist.barrier(group=group)          # every rank has mapped every buffer

    def _alloc(self, nbytes):
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(N.IPC_HANDLE_BYTES)
        N.call("nslg_ipc_alloc", nbytes, ctypes.byref(ptr), handle)
        self._own.append(ptr.value)
        return ptr.value, handle.raw

    def _open(self, handle):
        ptr = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(handle, N.IPC_HANDLE_BYTES)
        N.call("nslg_ipc_open", buf, ctypes.byref(ptr))
        self._opened.append(ptr.value)
        return ptr.value

    def fits(self, rows):
        return rows <= self.max_rows

    def linear_push(self, x, weight):
        """This rank's RowParallel product y = x . weight^T with its rows pushed into every
        peer's stage buffer by the same kernel (nslg_linear_tp_push: the GEMM and the
        collective's data movement in one launch). Returns y, the partial that the next
        ``allreduce_add_norm`` reduces (it then skips its own push), or None when the
        fused kernel does not take these operands (the caller runs the plain product)."""
        if (not self.fuse_push or self.world < FUSED_PUSH_MIN_WORLD
                or not ops.linear_supported(x, weight)):
            return None
        k, n = x.shape[-1], weight.shape[0]
        if n != self.hidden or x.dtype != self.dtype:
            return None
        try:
            rows, xs = ops._rows(x.unsqueeze(-2), "x")
        except ValueError:
            return None
        if rows > min(self.max_rows, FUSED_PUSH_MAX_ROWS) or xs % 8 or x.data_ptr() % 16:
            return None
        out = torch.empty(x.shape[:-1] + (n,), dtype=x.dtype, device=x.device)
        N.call("nslg_linear_tp_push", ops._dtype_code(x), rows, n, k, ops._ptr(x), xs,
               ops._ptr(weight), weight.stride(0), ops._ptr(out), n, self.world, self.rank,
               ctypes.cast(self._stage_arr, ctypes.c_void_p), self.stage_bytes,
               ops._ptr(self.counters), ops._ptr(self.status), ops._stream(x))
        self._pushed_ptr = out.data_ptr()
        return out

    def allreduce_add_norm(self, partial, residual, weight, eps, out=None):
        """residual <- residual + sum over the group of ``partial`` (in place); returns
        rmsnorm(residual) * weight, or ``residual`` itself when ``weight`` is None."""
        ops._need_cuda(partial, residual, weight, out)
        hidden = partial.shape[-1]
        rows = partial.numel() // hidden
        if hidden != self.hidden or rows > self.max_rows:
            raise ValueError(f"PeerAllReduce: [{rows}, {hidden}] does not fit "
                             f"[{self.max_rows}, {self.hidden}]")
        if partial.dtype != self.dtype or residual.dtype != self.dtype:
            raise TypeError("PeerAllReduce: activation dtype mismatch")
        p2 = partial.reshape(rows, hidden)
        r2 = residual.view(rows, hidden)
        o2 = None
        if weight is not None:
            if out is None:
                out = torch.empty_like(p2)
            o2 = out.view(rows, hidden)
        # the GEMM that produced ``partial`` already pushed its rows: reduce only
        pushed = self._pushed_ptr is not None and partial.data_ptr() == self._pushed_ptr
        self._pushed_ptr = None
        fn = "nslg_tp_reduce_pushed_rmsnorm" if pushed else "nslg_tp_allreduce_rmsnorm"
        N.call(fn, ops._dtype_code(partial), rows, hidden,
               self.world, self.rank, ops._ptr(p2), p2.stride(0),
               ctypes.cast(self._stage_arr, ctypes.c_void_p), self.stage_bytes,
               ops._ptr(self.counters), ops._ptr(r2), r2.stride(0),
               ops._ptr(weight), ops._ptr(o2), o2.stride(0) if o2 is not None else 0,
               float(eps), self.timeout_ns, ops._ptr(self.status), ops._stream(partial))
        if weight is None:
            return residual
        return out.view(partial.shape)

    def close(self):
        """Unmaps the peers' buffers and frees this rank's (after a group barrier, so no
        peer still reads them)."""
        if not self._own:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                N.call("nslg_ipc_close", p)
            for p in self._own:
                N.call("nslg_ipc_free", p)
        self._own, self._opened = [], []
