"""Tiny Llama forward on the contiguous oracle (TEST INFRASTRUCTURE ONLY; see
oracle/__init__.py).

Restates LlamaTP at TP=1 (nanoslg/models.py:86-172, 246-276): embedding, per layer
RMSNorm -> q/k/v projections -> RoPE -> attend -> o_proj -> residual, RMSNorm -> SwiGLU
MLP -> residual, final RMSNorm, LM head; driven like worker.py:365-426 drives one
request (prefill of the prompt, then greedy decode).
"""
import torch
import torch.nn.functional as F

from .attention import ContiguousOracle
from .rope_norm import apply_rotary, rmsnorm, rope_table


def param_names(n_layers):
    """Parameter order of the reference's LlamaTP.named_parameters()."""
    names = ["embed_tokens.weight"]
    for i in range(n_layers):
        p = f"layers.{i}."
        names += [p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight",
                  p + "self_attn.v_proj.weight", p + "self_attn.o_proj.weight",
                  p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight",
                  p + "mlp.down_proj.weight", p + "input_layernorm.weight",
                  p + "post_attention_layernorm.weight"]
    return names + ["norm.weight", "lm_head.lm_head.weight"]


def param_shapes(cfg):
    h, i, v = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    nq, nkv = cfg["num_attention_heads"], cfg["num_key_value_heads"]
    d = h // nq
    shapes = {"embed_tokens.weight": (v, h), "norm.weight": (h,),
              "lm_head.lm_head.weight": (v, h)}
    for li in range(cfg["num_hidden_layers"]):
        p = f"layers.{li}."
        shapes.update({p + "self_attn.q_proj.weight": (nq * d, h),
                       p + "self_attn.k_proj.weight": (nkv * d, h),
                       p + "self_attn.v_proj.weight": (nkv * d, h),
                       p + "self_attn.o_proj.weight": (h, nq * d),
                       p + "mlp.gate_proj.weight": (i, h), p + "mlp.up_proj.weight": (i, h),
                       p + "mlp.down_proj.weight": (h, i),
                       p + "input_layernorm.weight": (h,),
                       p + "post_attention_layernorm.weight": (h,)})
    return shapes


def init_params(cfg, seed=0, std=0.02):
    """The fixture's init rule: manual_seed(seed), then normal_(0, std) over the
    parameters in named_parameters() order, norm weights kept at 1."""
    shapes = param_shapes(cfg)
    params = {}
    for n in param_names(cfg["num_hidden_layers"]):
        params[n] = torch.ones(shapes[n]) if "norm" in n else torch.empty(shapes[n])
    torch.manual_seed(seed)
    for n in param_names(cfg["num_hidden_layers"]):
        if "norm" not in n:
            params[n].normal_(0.0, std)
    return params


class TinyLlamaOracle:
    def __init__(self, cfg, params, max_seq=128):
        self.cfg, self.p = cfg, params
        self.nq, self.nkv = cfg["num_attention_heads"], cfg["num_key_value_heads"]
        self.d = cfg["hidden_size"] // self.nq
        self.eps = cfg.get("rms_norm_eps", 1e-5)
        self.cos, self.sin = rope_table(self.d, cfg.get("max_position_embeddings", 8192),
                                        cfg.get("rope_theta", 500000.0), cfg.get("rope_scaling"))
        self.cache = ContiguousOracle(cfg["num_hidden_layers"], 1, max_seq, self.nkv, self.d,
                                      torch.float32)
        self.n = 0

    def forward(self, ids):
        B, S = ids.shape
        p = self.p
        start = [self.n]
        pos = torch.arange(self.n, self.n + S)[None]
        h = F.embedding(ids, p["embed_tokens.weight"])
        for li in range(self.cfg["num_hidden_layers"]):
            pre = f"layers.{li}."
            x = rmsnorm(h, p[pre + "input_layernorm.weight"], self.eps)
            q = F.linear(x, p[pre + "self_attn.q_proj.weight"]).view(B, S, self.nq, self.d)
            k = F.linear(x, p[pre + "self_attn.k_proj.weight"]).view(B, S, self.nkv, self.d)
            v = F.linear(x, p[pre + "self_attn.v_proj.weight"]).view(B, S, self.nkv, self.d)
            q = apply_rotary(q, self.cos[pos], self.sin[pos])
            k = apply_rotary(k, self.cos[pos], self.sin[pos])
            a = self.cache.attend(li, q, k, v, start, [S], [0])
            h = h + F.linear(a, p[pre + "self_attn.o_proj.weight"])
            x = rmsnorm(h, p[pre + "post_attention_layernorm.weight"], self.eps)
            m = F.silu(F.linear(x, p[pre + "mlp.gate_proj.weight"])) * \
                F.linear(x, p[pre + "mlp.up_proj.weight"])
            h = h + F.linear(m, p[pre + "mlp.down_proj.weight"])
        self.n += S
        return F.linear(rmsnorm(h, p["norm.weight"], self.eps), p["lm_head.lm_head.weight"])

    def greedy(self, prompt, steps):
        toks = []
        logits = self.forward(torch.tensor([prompt]))
        for step in range(steps):
            t = int(logits[0, -1].argmax())
            toks.append(t)
            if step + 1 < steps:
                logits = self.forward(torch.tensor([[t]]))
        return toks
