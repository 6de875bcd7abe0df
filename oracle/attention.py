"""Contiguous-SDPA attention oracle (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py).

Restates nanoslg/kv_cache.py:
  _sdpa                      44-56   softmax(q k^T / sqrt(D) + mask) v, GQA by head groups
  _build_causal_mask         192-224 kpos <= start + i  and  kpos < seq_len, -inf elsewhere,
                                     None on the three fast paths
  ContiguousCacheContext     247-325 write the new k/v at [start, start+n), transpose the
                                     [B, max_kv] slab, attend
The ``ContiguousOracle`` keeps a ``[L, Bmax, Smax, Hkv, D]`` cache exactly like
``_ContiguousPool`` so the timed CPU baseline does the reference's work per call.
"""
import torch
import torch.nn.functional as F


def sdpa(q, k, v, attn_mask=None, is_causal=False):
    """q [B,Hq,Sq,D], k/v [B,Hkv,Skv,D] (kv_cache.py:44-56)."""
    if q.shape[1] != k.shape[1]:
        return F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask,
                                              is_causal=is_causal, enable_gqa=True)
    return F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask, is_causal=is_causal)


def build_causal_mask(batch_size, input_width, start_positions, new_token_counts,
                      input_offsets, seq_lens, max_kv_len, dtype):
    """[B,1,Q,KV] additive mask or None (kv_cache.py:192-224)."""
    B = batch_size
    if B == 1 and start_positions[0] == 0 and input_offsets[0] == 0:
        return None
    if all(n == 1 for n in new_token_counts) and len(set(seq_lens)) == 1:
        return None
    if (all(s == 0 for s in start_positions) and all(o == 0 for o in input_offsets)
            and len(set(new_token_counts)) == 1):
        return None
    neg = -65504.0 if dtype == torch.float16 else float("-inf")
    mask = torch.full((B, 1, input_width, max_kv_len), neg, dtype=dtype)
    kp = torch.arange(max_kv_len)
    for b in range(B):
        off, ntok, base, kv = input_offsets[b], new_token_counts[b], start_positions[b], seq_lens[b]
        if ntok == 0:
            continue
        qp = torch.arange(ntok) + base
        ok = (kp[None, :] <= qp[:, None]) & (kp[None, :] < kv)
        mask[b, 0, off:off + ntok] = torch.where(ok, torch.tensor(0.0, dtype=dtype),
                                                 torch.tensor(neg, dtype=dtype))
    return mask


class ContiguousOracle:
    """A contiguous KV cache plus the attend() of ContiguousCacheContext."""

    def __init__(self, num_layers, max_batch, max_seq, hkv, d, dtype):
        shape = (num_layers, max_batch, max_seq, hkv, d)
        self.k = torch.zeros(shape, dtype=dtype)
        self.v = torch.zeros(shape, dtype=dtype)
        self.dtype = dtype

    def attend(self, layer, q, k_new, v_new, start_positions, new_token_counts, input_offsets):
        """One layer, sequences in slots 0..B-1 (kv_cache.py:297-322).

        q [B,S,Hq,D] and k_new/v_new [B,S,Hkv,D] are left-padded; row offsets[b] + i holds
        token i of sequence b, written at cache position start_positions[b] + i."""
        B, S = q.shape[0], q.shape[1]
        seq_lens = [s + n for s, n in zip(start_positions, new_token_counts)]
        kv = max(seq_lens) if seq_lens else 0
        if all(n == 1 for n in new_token_counts):
            bi = torch.arange(B)
            pos = torch.tensor(start_positions, dtype=torch.long)
            self.k[layer, bi, pos] = k_new[:, 0]
            self.v[layer, bi, pos] = v_new[:, 0]
        else:
            for b in range(B):
                o, n, s = input_offsets[b], new_token_counts[b], start_positions[b]
                if n > 0:
                    self.k[layer, b, s:s + n] = k_new[b, o:o + n]
                    self.v[layer, b, s:s + n] = v_new[b, o:o + n]
        iw = max(o + n for o, n in zip(input_offsets, new_token_counts)) if B else 1
        mask = build_causal_mask(B, iw, start_positions, new_token_counts, input_offsets,
                                 seq_lens, kv, self.dtype)
        k_t = self.k[layer, :B, :kv].transpose(1, 2).contiguous()
        v_t = self.v[layer, :B, :kv].transpose(1, 2).contiguous()
        q_t = q.transpose(1, 2)
        if mask is not None:
            mask = mask[:, :, :S, :kv].to(dtype=q.dtype)
        out = sdpa(q_t, k_t, v_t, attn_mask=mask, is_causal=(mask is None and S > 1))
        return out.transpose(1, 2).contiguous().reshape(B, S, -1)


def attend_sequences(q_rows, k_hist, v_hist, causal=True):
    """Per-sequence reference for tests of arbitrary size.

    q_rows[b]: [n_b, Hq, D] new query rows of sequence b; k_hist[b] / v_hist[b]:
    [len_b, Hkv, D] its whole KV (history + new rows, new rows last).  Row i sits at
    position len_b - n_b + i.  Returns a list of [n_b, Hq, D] in q's dtype, computed in
    fp32 with the same mask rule as build_causal_mask.
    """
    outs = []
    for q, k, v in zip(q_rows, k_hist, v_hist):
        n, hq, d = q.shape
        L, hkv = k.shape[0], k.shape[1]
        if n == 0:
            outs.append(q.new_zeros(q.shape))
            continue
        qt = q.float().transpose(0, 1)[None]           # [1, Hq, n, D]
        kt = k.float().transpose(0, 1)[None]           # [1, Hkv, L, D]
        vt = v.float().transpose(0, 1)[None]
        mask = None
        if causal:
            qp = torch.arange(n) + (L - n)
            ok = torch.arange(L)[None, :] <= qp[:, None]
            mask = torch.zeros(n, L).masked_fill(~ok, float("-inf"))[None, None]
        o = sdpa(qt, kt, vt, attn_mask=mask)
        outs.append(o[0].transpose(0, 1).to(q.dtype))
    return outs
