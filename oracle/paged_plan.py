"""Paged write-target and CSR plan oracle (TEST INFRASTRUCTURE ONLY; see
oracle/__init__.py).

Restates, as the reference's plain per-token / per-page Python loops, what
FlashInferCacheContext computes from the sequences' block tables:
  write targets   nanoslg/kv_cache.py:575-594  (page, slot) = (block_table[pos // P], pos % P),
                                                (0, 0) past the end of the block table
  CSR page list   nanoslg/kv_cache.py:598-615  indptr / indices / last_page_len
  qo_indptr       nanoslg/kv_cache.py:623-626
Copy-on-write is not restated here: the golden scenarios pin it against the reference.
"""


def write_targets(block_tables, start_positions, new_token_counts, page_size):
    out = []
    for bt, start, n in zip(block_tables, start_positions, new_token_counts):
        info = []
        for t in range(n):
            ap = start + t
            pi, sl = ap // page_size, ap % page_size
            info.append((0, 0) if pi >= len(bt) else (bt[pi], sl))
        out.append(info)
    return out


def csr(block_tables, seq_lens, page_size):
    indptr, indices, lpl = [0], [], []
    for bt, kv in zip(block_tables, seq_lens):
        np_ = -(-kv // page_size) if kv > 0 else 0
        for p in range(np_):
            indices.append(bt[p] if p < len(bt) else 0)
        indptr.append(indptr[-1] + np_)
        lpl.append((kv - (np_ - 1) * page_size) if np_ > 0 else 0)
    return indptr, indices, lpl


def qo_indptr(new_token_counts):
    qo = [0]
    for n in new_token_counts:
        qo.append(qo[-1] + n)
    return qo
