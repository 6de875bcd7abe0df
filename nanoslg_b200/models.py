"""Llama-architecture models driving the per-layer path (nanoslg/models.py:25-383).

Same module tree and parameter names as the reference's LlamaTP / LlamaPP / LlamaHybrid
(so its weight loaders and init rules apply unchanged), with these changes on the hot
path:

* ``RMSNorm`` runs the fused residual-add + RMSNorm kernel.  The blocks carry the
  residual stream explicitly: block i returns (mlp_out, residual) and block i+1 adds
  them inside its input norm.  The sums are the reference's ``h = x + attn`` and
  ``x + mlp`` (models.py:169-172) with the same bf16 rounding, one kernel instead of
  an add and ~7 norm kernels.
* ``_attention_forward`` (models.py:86-105) hands q, k, v and the RoPE tables to
  ``cache_ctx.attend_rope`` when the context has it (the B200 context does): RoPE, the
  KV append and attention become kernels behind the context.  Any other CacheContext
  gets the reference's torch RoPE followed by ``attend``.
* Greedy decoding reduces the LM-head logits with the ``nslg_argmax_rows`` kernel; a
  vocab-parallel head reduces its shard and the ranks exchange (max, index) pairs
  instead of all-gathering the logits.
* The projections of decode-sized forwards (at most 256 rows: decode steps, the LM head
  on the last position) run the tcgen05 linear kernel (``ops.linear``, nslg_linear);
  larger forwards (prefill) stay cuBLAS GEMMs. The collectives are NCCL or the fused
  peer-memory reduction; with the latter, a RowParallel product the tcgen05 kernel
  takes also pushes its partial rows to the peers from inside the GEMM.
"""
import math
from typing import List

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .parallel import ParallelMode, get_parallel_context
from .tp_layers import ColumnParallelLinear, ParallelLMHead, RowParallelLinear


class RMSNorm(nn.Module):
    """weight * bf16(x * rsqrt(mean(x^2) + eps)) with fp32 statistics (models.py:25-34)."""

    def __init__(self, dim, eps=1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        return ops.rmsnorm_residual(x, self.weight, self.eps)

    def add_forward(self, x, residual, peer=None):
        """residual <- x + residual (in place); returns (rmsnorm(residual), residual).
        With an active PeerAllReduce ``peer``, ``x`` is this rank's partial RowParallel
        output and is summed over the TP group first (one fused kernel)."""
        if peer is not None:
            return peer.allreduce_add_norm(x, residual, self.weight, self.eps), residual
        out = ops.rmsnorm_residual(x, self.weight, self.eps, residual=residual)
        return out, residual


def precompute_rope_frequencies(dim, max_seq_len, theta, config):
    """fp32 (cos, sin) tables [max_seq_len, dim] of cat(f, f) (models.py:37-66)."""
    freqs = 1.0 / (theta ** (torch.arange(0, dim, 2)[: dim // 2].float() / dim))
    sc = getattr(config, "rope_scaling", None)
    if sc and sc.get("rope_type") == "llama3":
        factor = sc.get("factor", 8.0)
        lo, hi = sc.get("low_freq_factor", 1.0), sc.get("high_freq_factor", 4.0)
        old_ctx = sc.get("original_max_position_embeddings", 8192)
        wl = 2 * math.pi / freqs
        smooth = (old_ctx / wl - lo) / (hi - lo)
        mid = (1 - smooth) * freqs / factor + smooth * freqs
        freqs = torch.where(wl < old_ctx / hi, freqs,
                            torch.where(wl > old_ctx / lo, freqs / factor, mid))
    t = torch.arange(max_seq_len, dtype=torch.float32)
    f = torch.outer(t, freqs)
    f = torch.cat((f, f), dim=-1)
    return f.cos(), f.sin()


def apply_rotary_emb(x, cos, sin):
    """Rotate-half RoPE with cos/sin cast to x's dtype (models.py:69-83)."""
    if cos.dim() == 2:
        cos, sin = cos[None, :, None, :], sin[None, :, None, :]
    elif cos.dim() == 3:
        cos, sin = cos[:, :, None, :], sin[:, :, None, :]
    cos = cos.to(x.device, dtype=x.dtype)
    sin = sin.to(x.device, dtype=x.dtype)
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return x * cos + torch.cat((-x2, x1), dim=-1) * sin


def _attention_forward(q, k_new, v_new, layer_idx, n_heads, n_kv_heads, cos, sin, cache_ctx):
    attend_rope = getattr(cache_ctx, "attend_rope", None)
    if attend_rope is not None:
        return attend_rope(layer_idx, q, k_new, v_new, cos, sin)
    S = q.shape[1]
    pos_ids = cache_ctx.get_position_ids(S)
    q = apply_rotary_emb(q, cos[pos_ids], sin[pos_ids])
    k_new = apply_rotary_emb(k_new, cos[pos_ids], sin[pos_ids])
    return cache_ctx.attend(layer_idx, q, k_new, v_new, n_heads, n_kv_heads)


class TPAttention(nn.Module):
    def __init__(self, config, layer_idx):
        super().__init__()
        tp = get_parallel_context().config.tp_size
        self.hidden_size = config.hidden_size
        self.n_heads = config.num_attention_heads
        self.n_kv_heads = getattr(config, "num_key_value_heads",
                                  getattr(config, "multi_query_group_num", self.n_heads))
        self.head_dim = config.hidden_size // self.n_heads   # models.py:117
        self.layer_idx = layer_idx
        if self.n_heads % tp or self.n_kv_heads % tp:
            raise ValueError("head counts must be divisible by tp_size")
        self.n_heads_tp = self.n_heads // tp
        self.n_kv_heads_tp = self.n_kv_heads // tp
        h, d = self.hidden_size, self.head_dim
        self.q_proj = ColumnParallelLinear(h, self.n_heads * d, gather_output=False)
        self.k_proj = ColumnParallelLinear(h, self.n_kv_heads * d, gather_output=False)
        self.v_proj = ColumnParallelLinear(h, self.n_kv_heads * d, gather_output=False)
        self.o_proj = RowParallelLinear(self.n_heads * d, h, input_is_parallel=True)
        self._qkv = None

    def fuse_projections(self):
        """Stacks the q, k and v weights into one buffer and makes the three Parameters
        views of it (same names, shapes and state-dict entries), so one GEMM produces
        q, k and v and reads the layer's input once."""
        self._qkv = _stack_as_views([self.q_proj, self.k_proj, self.v_proj])

    def forward(self, x, cos, sin, cache_ctx, mask=None):
        B, S, _ = x.shape
        hd = self.head_dim
        if _views_intact(self._qkv, [self.q_proj, self.k_proj, self.v_proj]):
            # decode batches: projections, RoPE and KV append in one kernel when the
            # context offers it (B200CacheContext.attend_qkv)
            attend_qkv = getattr(cache_ctx, "attend_qkv", None)
            if attend_qkv is not None:
                a = attend_qkv(self.layer_idx, x, self._qkv, self.n_heads_tp,
                               self.n_kv_heads_tp, cos, sin)
                if a is not None:
                    return self.o_proj(a)
            qkv = ops.linear(x, self._qkv)
            nq, nk = self.n_heads_tp * hd, self.n_kv_heads_tp * hd
            q = qkv[..., :nq].view(B, S, self.n_heads_tp, hd)
            k = qkv[..., nq:nq + nk].view(B, S, self.n_kv_heads_tp, hd)
            v = qkv[..., nq + nk:].view(B, S, self.n_kv_heads_tp, hd)
        else:
            q = self.q_proj(x).view(B, S, self.n_heads_tp, hd)
            k = self.k_proj(x).view(B, S, self.n_kv_heads_tp, hd)
            v = self.v_proj(x).view(B, S, self.n_kv_heads_tp, hd)
        a = _attention_forward(q, k, v, self.layer_idx, self.n_heads_tp, self.n_kv_heads_tp,
                               cos, sin, cache_ctx)
        return self.o_proj(a)


class TPMLP(nn.Module):
    def __init__(self, config):
        super().__init__()
        h, i = config.hidden_size, config.intermediate_size
        self.gate_proj = ColumnParallelLinear(h, i, gather_output=False)
        self.up_proj = ColumnParallelLinear(h, i, gather_output=False)
        self.down_proj = RowParallelLinear(i, h, input_is_parallel=True)
        self._gu = None

    def fuse_projections(self):
        """Stacks gate and up weights (views, as in TPAttention.fuse_projections): for
        decode batches one kernel (the gate|up product with SwiGLU in its epilogue), for
        larger ones one GEMM and one silu*mul kernel, instead of two GEMMs and two
        elementwise kernels."""
        self._gu = _stack_as_views([self.gate_proj, self.up_proj])

    def forward(self, x):
        if _views_intact(self._gu, [self.gate_proj, self.up_proj]):
            return self.down_proj(ops.linear_swiglu(x, self._gu))
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


def _stack_as_views(linears):
    """Concatenates the layers' weights along the output dim into one tensor and turns each
    layer's weight Parameter into a view of its rows (in-place loads keep them views)."""
    stacked = torch.cat([m.weight.data for m in linears], 0)
    row = 0
    for m in linears:
        n = m.weight.shape[0]
        m.weight = nn.Parameter(stacked[row:row + n], requires_grad=m.weight.requires_grad)
        row += n
    return stacked


def _views_intact(stacked, linears):
    """True while every weight is still the view of ``stacked`` made by _stack_as_views
    (a later model.to(...) replaces Parameters with fresh tensors and ends the fusion)."""
    if stacked is None:
        return False
    ptr, es = stacked.data_ptr(), stacked.element_size()
    row = 0
    for m in linears:
        w = m.weight
        if w.dtype != stacked.dtype or w.data_ptr() != ptr + row * stacked.shape[1] * es:
            return False
        row += w.shape[0]
    return True


class TPTransformerBlock(nn.Module):
    """models.py:160-172 with the residual carried between blocks (see module doc)."""

    def __init__(self, config, layer_idx):
        super().__init__()
        self.self_attn = TPAttention(config, layer_idx)
        self.mlp = TPMLP(config)
        eps = getattr(config, "rms_norm_eps", 1e-5)
        self.input_layernorm = RMSNorm(config.hidden_size, eps=eps)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, eps=eps)

    peer_reduce = None      # PeerAllReduce of the TP group (enable_peer_allreduce)

    def forward(self, x, cos, sin, cache_ctx, residual=None):
        peer = self.peer_reduce if self.peer_reduce is not None and self.peer_reduce.active else None
        if residual is None:
            residual = x.clone()
            h = self.input_layernorm(x)
        else:
            h, residual = self.input_layernorm.add_forward(x, residual, peer)
        a = self.self_attn(h, cos, sin, cache_ctx)
        h, residual = self.post_attention_layernorm.add_forward(a, residual, peer)
        return self.mlp(h), residual


# The reference's PP blocks (models.py:175-239) are the TP blocks with plain nn.Linear;
# at tp_size 1 the TP layers are exactly that, with the same parameter names.
PPTransformerBlock = TPTransformerBlock


class _LlamaStage(nn.Module):
    """Layers [layer_indices] of a Llama model, with the embedding on the first stage and
    the final norm + LM head on the last."""

    def __init__(self, hf_config, layer_indices: List[int], is_first, is_last, lm_head_tp):
        super().__init__()
        self.device = get_parallel_context().device
        self.layer_indices = layer_indices
        self.is_first, self.is_last = is_first, is_last
        self.n_layers = len(layer_indices)
        if is_first:
            self.embed_tokens = nn.Embedding(hf_config.vocab_size, hf_config.hidden_size)
        self.layers = nn.ModuleList(
            [TPTransformerBlock(hf_config, i) for i in range(len(layer_indices))])
        if is_last:
            self.norm = RMSNorm(hf_config.hidden_size, eps=getattr(hf_config, "rms_norm_eps", 1e-5))
            if lm_head_tp:
                self.lm_head = ParallelLMHead(hf_config.hidden_size, hf_config.vocab_size,
                                              gather_output=True)
            else:
                self.lm_head = nn.Linear(hf_config.hidden_size, hf_config.vocab_size, bias=False)
        theta = getattr(hf_config, "rope_theta", 500000.0)
        mx = getattr(hf_config, "max_position_embeddings", 8192)
        hd = hf_config.hidden_size // hf_config.num_attention_heads
        # plain fp32 attributes on the rank's device, untouched by model.to(dtype), as in
        # the reference (models.py:265-270)
        cos, sin = precompute_rope_frequencies(hd, mx, theta, hf_config)
        self.cos = cos.to(self.device)
        self.sin = sin.to(self.device)

    peer_reduce = None      # PeerAllReduce of the TP group (enable_peer_allreduce)

    def forward(self, x, cache_ctx, mask=None, last_only=False, greedy=False):
        """Reference semantics (models.py:272-276): logits for every input position.
        ``last_only`` computes the final norm and LM head for the last position only
        (the only one the decode loop reads), which saves the [B, S, vocab] logits of a
        long prefill. ``greedy`` (last stage, with ``last_only``) returns the greedy token
        of the last position, [B] int64, instead of its logits: under TP each rank takes
        the argmax of its vocabulary shard and only (max, index) pairs are gathered."""
        h = self.embed_tokens(x) if self.is_first and x.dtype == torch.long else x
        peer = self.peer_reduce
        if peer is not None:
            # the same decision on every TP rank: they run the same shapes
            peer.active = peer.fits(h.shape[0] * h.shape[1])
            peer = peer if peer.active else None
        residual = None
        for layer in self.layers:
            h, residual = layer(h, self.cos, self.sin, cache_ctx, residual)
        if residual is not None:
            # the stage's output is the residual stream after its last block (with an
            # active peer reduction, h is still this rank's partial down_proj output)
            if self.is_last:
                if last_only and peer is None:
                    h, residual = h[:, -1:].contiguous(), residual[:, -1:].contiguous()
                # with an active peer reduction every row is reduced (the GEMM may already
                # have pushed them all to the peers) and the last position taken after
                h, _ = self.norm.add_forward(h, residual, peer)
                if last_only and peer is not None:
                    h = h[:, -1:].contiguous()
                if greedy and last_only:
                    return self._greedy(h)
                return self.lm_head(h)
            if peer is not None:
                return peer.allreduce_add_norm(h, residual, None, 0.0)
            return _add(h, residual)
        if self.is_last and last_only:
            h = h[:, -1:].contiguous()
        if self.is_last and greedy and last_only:
            return self._greedy(self.norm(h))
        return self.lm_head(self.norm(h)) if self.is_last else h

    def _greedy(self, h):
        """argmax over the vocabulary of the LM head applied to h [B, 1, hidden]: the
        first index of the maximum, as torch.argmax over the all-gathered logits
        (tp_layers.py:89 gathers them in the reference). With a vocab-parallel head each
        rank reduces its shard and one all-gather of [B, 2] fp32 (max, global index)
        pairs replaces the gather of [B, vocab] logits; the lowest rank holding the
        maximum wins, and its shard holds the lowest indices."""
        head = getattr(self.lm_head, "lm_head", None)
        tp = getattr(head, "tp_size", 1)
        if (head is None or tp == 1 or not getattr(head, "gather_output", False)
                or head.out_features >= (1 << 24)):
            return ops.argmax_rows(self.lm_head(h)[:, -1])
        local = ops.linear(h[:, -1], head.weight, head.bias)            # [B, V/tp]
        ctx = get_parallel_context()
        offset = ctx.tp_rank * head.out_features_per_partition
        idx, val = ops.argmax_rows(local, offset, values=True)
        pair = torch.stack([val, idx.float()], -1)                        # exact below 2^24
        # gathered as the rank-major concatenation [tp * B, 2] (the layout every backend
        # accepts), viewed as [tp, B, 2]
        allp = torch.empty((tp * pair.shape[0], 2), dtype=pair.dtype, device=pair.device)
        dist.all_gather_into_tensor(allp, pair.contiguous(), group=ctx.tp_group)
        allp = allp.view(tp, pair.shape[0], 2)
        best = allp[..., 0].argmax(0)                                      # first max rank
        return allp[..., 1].gather(0, best[None]).squeeze(0).long()


def _add(a, b):
    return b.add_(a)


def enable_peer_allreduce(model, peer):
    """Routes the RowParallel reductions of ``model`` (o_proj, down_proj) through
    ``peer`` (a tp_comm.PeerAllReduce of this rank's TP group) for forwards whose rows
    fit its buffers; ``None`` restores the NCCL all-reduce everywhere."""
    model.peer_reduce = peer
    for layer in model.layers:
        layer.peer_reduce = peer
        layer.self_attn.o_proj.peer_reduce = peer
        layer.mlp.down_proj.peer_reduce = peer
    return model


def fuse_projections(model):
    """Fuses the q/k/v and gate/up GEMMs of every block of ``model`` (call once the model
    is on its final device and dtype)."""
    for layer in model.layers:
        layer.self_attn.fuse_projections()
        layer.mlp.fuse_projections()
    return model


class LlamaTP(_LlamaStage):
    """All layers on every rank, weights split by TP (models.py:246-276)."""

    def __init__(self, hf_config):
        super().__init__(hf_config, list(range(hf_config.num_hidden_layers)), True, True,
                         lm_head_tp=True)


class LlamaPP(_LlamaStage):
    """A pipeline stage without TP (models.py:279-318)."""

    def __init__(self, hf_config, layer_indices, is_first, is_last):
        super().__init__(hf_config, layer_indices, is_first, is_last, lm_head_tp=False)


class LlamaHybrid(_LlamaStage):
    """A pipeline stage whose layers are TP-split (models.py:321-360)."""

    def __init__(self, hf_config, layer_indices, is_first, is_last):
        super().__init__(hf_config, layer_indices, is_first, is_last, lm_head_tp=True)


def create_model(hf_config, parallel_config):
    """models.py:362-383."""
    ctx = get_parallel_context()
    if parallel_config.mode == ParallelMode.TENSOR:
        return LlamaTP(hf_config)
    li = parallel_config.pp_layer_splits[ctx.pp_rank]
    first, last = ctx.pp_rank == 0, ctx.pp_rank == parallel_config.pp_size - 1
    if parallel_config.mode == ParallelMode.PIPELINE:
        return LlamaPP(hf_config, li, first, last)
    if parallel_config.mode == ParallelMode.HYBRID:
        return LlamaHybrid(hf_config, li, first, last)
    raise ValueError(f"Unknown mode: {parallel_config.mode}")


_COLUMN = ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj", "lm_head")
_ROW = ("o_proj", "down_proj")


def load_full_state_dict(model, full, tp_size=1, tp_rank=0):
    """Copies this rank's shard of an unsharded LlamaTP state dict ``full`` into ``model``
    (in place, so stacked q/k/v and gate/up buffers stay fused), with the reference's
    split rule (models.py:386-573): column layers (q, k, v, gate, up, LM head) take chunk
    ``tp_rank`` of dim 0, row layers (o, down) of dim 1, the rest is copied whole; a
    pipeline stage's local layer i is global layer ``model.layer_indices[i]``."""
    with torch.no_grad():
        for name, p in model.named_parameters():
            src = name
            if name.startswith("layers."):
                parts = name.split(".")
                parts[1] = str(model.layer_indices[int(parts[1])])
                src = ".".join(parts)
            elif name == "lm_head.weight":                  # LlamaPP's plain nn.Linear
                src = "lm_head.lm_head.weight"
            t = full[src]
            if tp_size > 1 and any(k in name for k in _COLUMN):
                t = t.chunk(tp_size, 0)[tp_rank]
            elif tp_size > 1 and any(k in name for k in _ROW):
                t = t.chunk(tp_size, 1)[tp_rank]
            p.data.copy_(t.to(p.device, p.dtype))
    return model


def reference_param_shapes(hf_config):
    """Names and shapes of an unsharded LlamaTP's parameters, in the order of the
    reference's ``named_parameters()`` (models.py:108-172, 246-276)."""
    h, inter, vocab = hf_config.hidden_size, hf_config.intermediate_size, hf_config.vocab_size
    nq = hf_config.num_attention_heads
    nkv = getattr(hf_config, "num_key_value_heads", nq)
    d = h // nq
    out = [("embed_tokens.weight", (vocab, h))]
    for i in range(hf_config.num_hidden_layers):
        p = f"layers.{i}."
        out += [(p + "self_attn.q_proj.weight", (nq * d, h)),
                (p + "self_attn.k_proj.weight", (nkv * d, h)),
                (p + "self_attn.v_proj.weight", (nkv * d, h)),
                (p + "self_attn.o_proj.weight", (h, nq * d)),
                (p + "mlp.gate_proj.weight", (inter, h)), (p + "mlp.up_proj.weight", (inter, h)),
                (p + "mlp.down_proj.weight", (h, inter)),
                (p + "input_layernorm.weight", (h,)),
                (p + "post_attention_layernorm.weight", (h,))]
    return out + [("norm.weight", (h,)), ("lm_head.lm_head.weight", (vocab, h))]


def reference_random_state_dict(hf_config, seed=0, std=0.02):
    """Unsharded fp32 state dict of the BASELINE init rule on the CPU: manual_seed(seed),
    then normal_(0, std) over the parameters in the reference's order, norm weights 1.
    Sharded with ``load_full_state_dict``, every TP/PP layout gets the same model."""
    shapes = reference_param_shapes(hf_config)
    sd = {n: (torch.ones(s) if "norm" in n else torch.empty(s)) for n, s in shapes}
    torch.manual_seed(seed)
    for n, _ in shapes:
        if "norm" not in n:
            sd[n].normal_(0.0, std)
    return sd


def init_random_(model, seed=0, std=0.02):
    """Random init of the BASELINE configs: manual_seed(seed), normal_(0, std) over
    named_parameters() in order, norm weights kept at 1 (the golden fixture's rule)."""
    torch.manual_seed(seed)
    with torch.no_grad():
        for n, p in model.named_parameters():
            if "norm" in n:
                p.fill_(1.0)
            else:
                p.normal_(0.0, std)
    return model
