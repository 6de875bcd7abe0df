"""Batch runner driving the per-layer path the way NanoSLG's worker drives it.

``LlamaRunner`` is the core of ``run_tp_worker``'s batch loop (nanoslg/worker.py:365-426):
prefix-aware allocation with the prompt clamp of ``allocate_batch_with_prefix``
(worker.py:169-213), one left-padded prefill forward, then greedy decode steps of
``begin_forward -> model -> end_forward -> argmax``, and release (which inserts the
sequences into the radix tree for later batches).  The scheduler, queues, HTTP server
and broadcasts of the worker are not part of the path and are left out; under
torch.distributed every TP rank runs the same runner on the same token ids, as the
worker's ranks do after their metadata broadcasts.
"""
from types import SimpleNamespace

import torch

import torch.distributed as dist

from . import models
from .kv_cache import create_cache_manager
from .parallel import ParallelConfig, ParallelContext, ParallelMode, get_layers_for_pp_rank


def llama_config(name):
    """Architectures of the BASELINE configs (random init; no checkpoint is read)."""
    cfgs = {
        "tiny": dict(num_hidden_layers=2, hidden_size=256, num_attention_heads=4,
                     num_key_value_heads=2, intermediate_size=512, vocab_size=1024,
                     rms_norm_eps=1e-5, rope_theta=10000.0, max_position_embeddings=128),
        "llama-3.1-8b": dict(num_hidden_layers=32, hidden_size=4096, num_attention_heads=32,
                             num_key_value_heads=8, intermediate_size=14336, vocab_size=128256,
                             rms_norm_eps=1e-5, rope_theta=500000.0,
                             max_position_embeddings=8192),
        "llama-3-70b": dict(num_hidden_layers=80, hidden_size=8192, num_attention_heads=64,
                            num_key_value_heads=8, intermediate_size=28672, vocab_size=128256,
                            rms_norm_eps=1e-5, rope_theta=500000.0,
                            max_position_embeddings=8192),
    }
    return SimpleNamespace(**cfgs[name])


class LlamaRunner:
    """One rank of a TP, PP or hybrid TP x PP deployment (parallel.py:15-68 layout: rank =
    pp_rank * tp_size + tp_rank).  With pp_size > 1 each rank holds its stage's layers
    (get_layers_for_pp_rank) and its stage-local KV cache; a forward runs the stages in
    turn, each TP rank sending the hidden state to the same TP rank of the next stage
    (NCCL send/recv, the reference's handoff of worker.py:561-593 / 654-685 without the
    TP-master funnel: every TP rank already holds the all-reduced hidden), and the last
    stage broadcasts the greedy tokens to every rank."""

    def __init__(self, hf_config, device, dtype=torch.bfloat16, tp_size=1, rank=0,
                 max_kv_pages=0, page_size=16, prefix_caching=True, seed=0, pp_size=1,
                 peer_allreduce=True, peer_max_rows=256):
        self.device = torch.device(device)
        self.dtype = dtype
        world = tp_size * pp_size
        if pp_size == 1:
            self.pcfg = ParallelConfig(ParallelMode.TENSOR, world)
        else:
            mode = ParallelMode.PIPELINE if tp_size == 1 else ParallelMode.HYBRID
            self.pcfg = ParallelConfig(mode, world, tp_size=tp_size, pp_size=pp_size)
            L = hf_config.num_hidden_layers
            self.pcfg.pp_layer_splits = {r: get_layers_for_pp_rank(L, pp_size, r)
                                         for r in range(pp_size)}
        ctx = ParallelContext.initialize(self.pcfg, rank, device=self.device)
        if world > 1:
            ctx.setup_groups()
        self.pctx = ctx
        self.hf = hf_config
        prev = torch.get_default_dtype()
        torch.set_default_dtype(dtype)
        try:
            with torch.device(self.device):
                self.model = models.create_model(hf_config, self.pcfg)
        finally:
            torch.set_default_dtype(prev)
        models.init_random_(self.model, seed=seed + ctx.tp_rank)
        models.fuse_projections(self.model)
        self.model.eval()
        # decode-sized RowParallel reductions over NVLink peer memory, fused with the
        # residual add and RMSNorm (tp_comm.PeerAllReduce); prefill keeps NCCL
        self.peer = None
        if tp_size > 1 and peer_allreduce:
            from .tp_comm import PeerAllReduce
            self.peer = PeerAllReduce(ctx.tp_group, ctx.tp_rank, tp_size, self.device,
                                      peer_max_rows, hf_config.hidden_size, dtype)
            models.enable_peer_allreduce(self.model, self.peer)
        mc = SimpleNamespace(page_size=page_size, max_kv_pages=max_kv_pages,
                             enable_prefix_caching=prefix_caching)
        self.cache = create_cache_manager(hf_config, self.pcfg, self.device, dtype, mc,
                                          max_batch_size=0)
        self.seq_ids = []
        self.use_graphs = False
        self._graphs = {}        # batch -> (graph, static tokens in, static tokens out)

    def load_full_state_dict(self, full):
        """Loads this rank's shard of an unsharded state dict (reference split rule)."""
        models.load_full_state_dict(self.model, full, self.pcfg.tp_size, self.pctx.tp_rank)

    def _forward_tokens(self, x, ctx, width):
        """One forward of the whole deployment for this step's cache context; returns the
        greedy token of every sequence on every rank."""
        if self.pcfg.pp_size == 1:
            return self.model(x, ctx, last_only=True, greedy=True)
        pc = self.pctx
        B = len(self.seq_ids)
        if not pc.is_first_pp_stage:
            x = torch.empty(B, width, self.hf.hidden_size, dtype=self.dtype, device=self.device)
            dist.recv(x, src=pc.get_pp_prev_rank())
        if width == 1 and self.use_graphs:
            # decode step: the stage forward replays its CUDA graph
            res = self._stage_decode_forward(x, ctx, B)
            if pc.is_last_pp_stage:
                tok = res.clone()
            else:
                dist.send(res.contiguous(), dst=pc.get_pp_next_rank())
                tok = torch.empty(B, dtype=torch.long, device=self.device)
            dist.broadcast(tok, src=(self.pcfg.pp_size - 1) * self.pcfg.tp_size)
            return tok
        out = self.model(x, ctx, last_only=pc.is_last_pp_stage, greedy=pc.is_last_pp_stage)
        if pc.is_last_pp_stage:
            tok = out
        else:
            dist.send(out.contiguous(), dst=pc.get_pp_next_rank())
            tok = torch.empty(B, dtype=torch.long, device=self.device)
        dist.broadcast(tok, src=(self.pcfg.pp_size - 1) * self.pcfg.tp_size)
        return tok

    def enable_cuda_graphs(self, batches):
        """Decode steps of these batch sizes run as one captured CUDA graph each: the plan
        goes into a fixed device buffer (built there by the device planner before every
        replay), the token ids into a fixed input tensor, and the whole model forward plus
        argmax replays without per-kernel launches from Python."""
        for b in batches:
            self.cache.use_static_plan(b, 1)
        self.use_graphs = True

    @torch.inference_mode()
    def prefill(self, prompts):
        """Allocates the batch (radix hits clamped to len-1, worker.py:190-195), runs the
        left-padded prefill and returns the first greedy token of every sequence."""
        mgr = self.cache
        self.seq_ids = [f"s{i}" for i in range(len(prompts))]
        prefix = []
        for sid, toks in zip(self.seq_ids, prompts):
            plen = mgr.allocate_sequence(sid, list(toks))
            pl = len(toks)
            prefix.append(min(plen, pl - 1) if pl > 1 else 0)
        counts = [len(t) - p for t, p in zip(prompts, prefix)]
        width = max(counts)
        offsets = [width - n for n in counts]
        ids = torch.zeros(len(prompts), width, dtype=torch.long)
        for i, (t, p, n) in enumerate(zip(prompts, prefix, counts)):
            ids[i, width - n:] = torch.tensor(t[p:p + n])
        self.prefix_lens = prefix
        ctx = mgr.begin_forward(self.seq_ids, counts, offsets)
        tok = self._forward_tokens(ids.to(self.device, non_blocking=True), ctx, width)
        mgr.end_forward(ctx)
        return tok

    @torch.inference_mode()
    def decode_step(self, tokens):
        mgr = self.cache
        B = len(self.seq_ids)
        ctx = mgr.begin_forward(self.seq_ids, [1] * B)
        if not (self.use_graphs and self.pcfg.pp_size == 1
                and getattr(ctx, "plan_static", False)):
            tok = self._forward_tokens(tokens[:, None], ctx, 1)
            mgr.end_forward(ctx)
            return tok
        entry = self._graphs.get(B)
        if entry is None:
            tok_in = tokens.clone()
            # warm-up forwards on a side stream, then capture; each re-writes this step's
            # K/V slots with the same values
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                for _ in range(2):
                    self.model(tok_in[:, None], ctx, last_only=True)
            torch.cuda.current_stream(self.device).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                tok_out = self.model(tok_in[:, None], ctx, last_only=True, greedy=True)
            entry = (graph, tok_in, tok_out)
            self._graphs[B] = entry
        else:
            entry[1].copy_(tokens)
        entry[0].replay()
        mgr.end_forward(ctx)
        return entry[2].clone()

    def _stage_decode_forward(self, x, ctx, B):
        """Decode forward of this rank's pipeline stage for B sequences: the last stage
        returns their greedy tokens [B], the others the hidden state [B, 1, hidden].
        With graphs enabled and the plan in the static buffer, the stage forward replays
        one CUDA graph per B (no collective inside: the stage's TP reductions are the
        peer-memory kernel, or NCCL in the graph as in ``decode_step``). The result is the
        graph's static output: use it before the next call with the same B."""
        last = self.pctx.is_last_pp_stage
        if not (self.use_graphs and getattr(ctx, "plan_static", False)):
            return self.model(x, ctx, last_only=last, greedy=last)
        key = ("stage", B)
        entry = self._graphs.get(key)
        if entry is None:
            x_in = x.clone()
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                for _ in range(2):       # rewrites this step's K/V slots with the same values
                    self.model(x_in, ctx, last_only=last)
            torch.cuda.current_stream(self.device).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                res = self.model(x_in, ctx, last_only=last, greedy=last)
            entry = (graph, x_in, res)
            self._graphs[key] = entry
        else:
            entry[1].copy_(x)
        entry[0].replay()
        return entry[2]

    @torch.inference_mode()
    def decode_microbatched(self, tokens, num_micro, steps):
        """``steps`` greedy decode steps of the current batch split into ``num_micro``
        micro-batches flowing through the pipeline stages (BASELINE C5; the reference runs
        its PP stages in lock step, worker.py:580-607). Tick i: stage p runs micro-batch
        (i - p) mod M; after every tick each rank exchanges, in one grouped NCCL
        send/recv, the hidden state with the neighbouring stages (same TP rank) and the
        last stage returns the micro-batch's tokens to the first, which needs them M - P
        + 1 ticks later (M >= P). Returns the generated tokens [B, steps] on every rank
        of the first and last stage (other stages: None)."""
        pc = self.pctx
        P = self.pcfg.pp_size
        if P < 2:
            raise ValueError("decode_microbatched needs pipeline stages")
        p = pc.pp_rank
        B = len(self.seq_ids)
        M = num_micro
        if B % M or M < P:
            raise ValueError("batch must split into num_micro >= pp_size equal micro-batches")
        mb = B // M
        tp = self.pcfg.tp_size
        groups = [self.seq_ids[j * mb:(j + 1) * mb] for j in range(M)]
        first_rank = pc.tp_rank
        last_rank = (P - 1) * tp + pc.tp_rank
        H = self.hf.hidden_size
        tok_mb = [tokens[j * mb:(j + 1) * mb].clone() for j in range(M)]
        gen = [[] for _ in range(M)]
        recv_h = None
        n_work = steps * M
        for i in range(n_work + P - 1):
            k = i - p
            active = 0 <= k < n_work
            out = None
            if active:
                m = k % M
                ctx = self.cache.begin_forward(groups[m], [1] * mb)
                x = tok_mb[m][:, None] if p == 0 else recv_h
                out = self._stage_decode_forward(x, ctx, mb)
                self.cache.end_forward(ctx)
                if p == P - 1:
                    gen[m].append(out.clone())
            ops = []
            if active and p < P - 1:
                ops.append(dist.P2POp(dist.isend, out.contiguous(), pc.get_pp_next_rank()))
            if p > 0 and 0 <= i + 1 - p < n_work:
                recv_h = torch.empty(mb, 1, H, dtype=self.dtype, device=self.device)
                ops.append(dist.P2POp(dist.irecv, recv_h, pc.get_pp_prev_rank()))
            if active and p == P - 1:
                ops.append(dist.P2POp(dist.isend, out.contiguous(), first_rank))
            pending = None
            if p == 0 and 0 <= i - (P - 1) < n_work:
                t = torch.empty(mb, dtype=torch.long, device=self.device)
                ops.append(dist.P2POp(dist.irecv, t, last_rank))
                pending = ((i - (P - 1)) % M, t)
            if ops:
                for r in dist.batch_isend_irecv(ops):
                    r.wait()
            if pending is not None:
                tok_mb[pending[0]] = pending[1]
                gen[pending[0]].append(pending[1])
        if p != 0 and p != P - 1:
            return None
        return torch.cat([torch.stack(g, 1) for g in gen], 0)

    def close(self):
        """Drops the captured graphs (they may hold NCCL calls, which must be gone before
        the process group is destroyed), the model and the cache."""
        self._graphs.clear()
        self.model = None
        self.cache = None
        torch.cuda.synchronize(self.device)
        if self.peer is not None:
            self.peer.close()
            self.peer = None
        torch.cuda.empty_cache()

    def release(self, generated=None):
        """Records generated ids (for radix insertion) and releases the batch."""
        if generated is not None:
            for sid, ids in zip(self.seq_ids, generated):
                self.cache.append_token_ids(sid, list(ids))
        for sid in self.seq_ids:
            self.cache.release_sequence(sid)
        self.seq_ids = []
