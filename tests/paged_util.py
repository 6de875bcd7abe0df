"""Builds seeded paged-KV problems and their per-sequence views for parity tests."""
import math

import torch


def make_paged(lens, hkv, d, num_pages, dtype, device, seed=0, page_size=16, fill="randn"):
    """Random page tables over a pool of ``num_pages`` pages (page 0 never used).

    Returns dict with pool_k/pool_v [P, page, Hkv, D] on ``device`` and the CSR arrays
    (int32, on device) plus host copies."""
    g = torch.Generator().manual_seed(seed)
    npg = [math.ceil(n / page_size) if n > 0 else 0 for n in lens]
    total = sum(npg)
    assert total < num_pages
    perm = (torch.randperm(num_pages - 1, generator=g)[:total] + 1).to(torch.int32)
    indptr = torch.zeros(len(lens) + 1, dtype=torch.int32)
    indptr[1:] = torch.cumsum(torch.tensor(npg, dtype=torch.int64), 0).to(torch.int32)
    lpl = torch.tensor([(n - (p - 1) * page_size) if p > 0 else 0 for n, p in zip(lens, npg)],
                       dtype=torch.int32)
    shape = (num_pages, page_size, hkv, d)
    gd = torch.Generator(device=device).manual_seed(seed + 1)
    pool_k = torch.randn(shape, dtype=torch.float32, device=device, generator=gd).to(dtype) \
        if fill == "randn" else torch.zeros(shape, dtype=dtype, device=device)
    pool_v = torch.randn(shape, dtype=torch.float32, device=device, generator=gd).to(dtype) \
        if fill == "randn" else torch.zeros(shape, dtype=dtype, device=device)
    return {"pool_k": pool_k, "pool_v": pool_v, "indptr": indptr.to(device),
            "indices": (perm if total else torch.zeros(1, dtype=torch.int32)).to(device),
            "lpl": lpl.to(device), "indptr_h": indptr, "indices_h": perm, "lpl_h": lpl,
            "lens": list(lens), "page_size": page_size}


def sequence_kv(pk, b, which="k"):
    """[len_b, Hkv, D] of sequence b gathered from the pool, on the CPU."""
    ps = pk["page_size"]
    s, e = int(pk["indptr_h"][b]), int(pk["indptr_h"][b + 1])
    pages = pk["indices_h"][s:e].long()
    pool = pk["pool_k"] if which == "k" else pk["pool_v"]
    rows = pool[pages.to(pool.device)].reshape(-1, pool.shape[2], pool.shape[3])
    return rows[:pk["lens"][b]].cpu()
