"""Tensor-parallel linear layers with the reference's surface (nanoslg/tp_layers.py:28-158,
210-234): Column splits the output features, Row splits the input features and
all-reduces its output over the TP group (NCCL), the LM head is a gathered Column layer.
The products go through ``ops.linear``: the tcgen05 kernel for decode-sized forwards
(at most 256 rows, bf16 / fp16), the cuBLAS GEMM of ``F.linear`` otherwise (prefill,
fp32, CPU tensors), as in the reference."""
import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .parallel import all_gather_tp, all_reduce_tp, get_parallel_context


class ColumnParallelLinear(nn.Module):
    """Weight [out/tp, in]; output [..., out/tp] (all-gathered when gather_output)."""

    def __init__(self, in_features, out_features, bias=False, gather_output=False,
                 init_method=None):
        super().__init__()
        tp = get_parallel_context().config.tp_size
        if out_features % tp:
            raise ValueError(f"out_features ({out_features}) must be divisible by tp ({tp})")
        self.in_features, self.out_features, self.tp_size = in_features, out_features, tp
        self.gather_output = gather_output
        self.out_features_per_partition = out_features // tp
        self.weight = nn.Parameter(torch.empty(self.out_features_per_partition, in_features))
        self.bias = nn.Parameter(torch.empty(self.out_features_per_partition)) if bias else None
        if init_method is not None:
            init_method(self.weight)
        else:
            nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            bound = 1 / math.sqrt(in_features) if in_features > 0 else 0
            nn.init.uniform_(self.bias, -bound, bound)

    def forward(self, x):
        out = ops.linear(x, self.weight, self.bias)
        if self.gather_output and self.tp_size > 1:
            out = all_gather_tp(out, dim=-1)
        return out


class RowParallelLinear(nn.Module):
    """Weight [out, in/tp]; the partial products are summed by an all-reduce."""

    def __init__(self, in_features, out_features, bias=False, input_is_parallel=True,
                 init_method=None):
        super().__init__()
        tp = get_parallel_context().config.tp_size
        if in_features % tp:
            raise ValueError(f"in_features ({in_features}) must be divisible by tp ({tp})")
        self.in_features, self.out_features, self.tp_size = in_features, out_features, tp
        self.input_is_parallel = input_is_parallel
        self.in_features_per_partition = in_features // tp
        self.weight = nn.Parameter(torch.empty(out_features, self.in_features_per_partition))
        self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None
        if init_method is not None:
            init_method(self.weight)
        else:
            nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))

    # A PeerAllReduce set here (models.enable_peer_allreduce) takes over the reduction
    # while it is active: forward returns this rank's partial product and the RMSNorm
    # that consumes it sums the partials, adds the residual and normalises in one kernel.
    peer_reduce = None

    def forward(self, x):
        if (self.tp_size > 1 and self.peer_reduce is not None and self.peer_reduce.active
                and self.bias is None):
            # the partial product; the GEMM pushes it to the peers itself when it can
            out = self.peer_reduce.linear_push(x, self.weight)
            return out if out is not None else ops.linear(x, self.weight)
        out = ops.linear(x, self.weight)
        if self.tp_size > 1:
            out = all_reduce_tp(out)
        if self.bias is not None:
            out = out + self.bias
        return out


class ParallelLMHead(nn.Module):
    """Vocab-split LM head whose logits are all-gathered (tp_layers.py:210-234)."""

    def __init__(self, hidden_size, vocab_size, gather_output=True):
        super().__init__()
        self.hidden_size, self.vocab_size = hidden_size, vocab_size
        self.tp_size = get_parallel_context().config.tp_size
        self.gather_output = gather_output
        self.lm_head = ColumnParallelLinear(hidden_size, vocab_size, bias=False,
                                            gather_output=gather_output)

    def forward(self, x):
        return self.lm_head(x)
