"""Radix-style prefix sharing with refcounted pages and copy-on-write
(BASELINE config 3's layout at reduced size, Qwen2.5-7B attention shapes).

One owner writes a shared prompt prefix whose last page is only partly full;
every sequence lists the prefix pages (one reference each on the host page
pool), and before its first own token lands in the shared partial page it
takes a private copy of that page (page copy kernel), then appends its
suffix.  Checked: page-level K/V bit-exact through gather, decode attention
against the f32 oracle on each sequence's logical cache, the refcounts, and
that the owner's copy of the partial page is untouched.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from mitten_b200 import host, paged

pytestmark = pytest.mark.gpu

HQ, HKV, D, PS = 28, 4, 128, 16
TOL = 2e-2


def test_shared_prefix_pages_with_copy_on_write(cuda_device):
    rng = np.random.default_rng(5)
    prefix_len = 4 * PS + 8                 # four full pages and a partial one (the 1032-token case, scaled)
    suffixes = [20, 1, 40, 16, 9, 33]
    n = len(suffixes)
    num_pages = 64
    pool = paged.PagedKVPool(1, num_pages, PS, HKV, D)
    pages = host.KvCachePool(num_pages, PS)

    def rows(t):
        return (rng.standard_normal((t, HKV, D)).astype(np.float32),
                rng.standard_normal((t, HKV, D)).astype(np.float32))

    def write(table, start, k, v):
        pos = np.arange(start, start + len(k))
        slots = np.array([table[p // PS] * PS + p % PS for p in pos], np.int64)
        pool.append(0, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), torch.from_numpy(slots).cuda())

    # the owner (request 0) allocates and fills the prefix
    owner_table = [pages.allocate(0) for _ in range((prefix_len + PS - 1) // PS)]
    kp, vp = rows(prefix_len)
    write(owner_table, 0, kp, vp)
    partial = owner_table[-1]

    tables, ks, vs, n_cow = [], [], [], 0
    for i, sl in enumerate(suffixes):
        t = list(owner_table)
        for p in t:
            pages.retain(p)                  # the sequence's reference to a shared page
        # the first suffix token goes to position prefix_len, inside the shared partial page
        idx = prefix_len // PS
        if pages.refcount(t[idx]) > 1:
            fresh = pages.allocate(i + 1)
            pool.page_copy(torch.tensor([t[idx]], dtype=torch.int32, device="cuda"),
                           torch.tensor([fresh], dtype=torch.int32, device="cuda"))
            pages.release(t[idx])
            t[idx] = fresh
            n_cow += 1
        while len(t) * PS < prefix_len + sl:
            t.append(pages.allocate(i + 1))
        ks_, vs_ = rows(sl)
        write(t, prefix_len, ks_, vs_)
        tables.append(t)
        ks.append(np.concatenate([kp, ks_]))
        vs.append(np.concatenate([vp, vs_]))
    torch.cuda.synchronize()

    assert n_cow == n
    for p in owner_table[:-1]:
        assert pages.refcount(p) == 1 + n     # owner + every sequence
    assert pages.refcount(partial) == 1       # every sequence copied it away

    lens = [prefix_len + s for s in suffixes]
    indptr = np.concatenate([[0], np.cumsum([len(t) for t in tables])]).astype(np.int32)
    indices = np.concatenate(tables).astype(np.int32)
    kv_indptr = torch.from_numpy(indptr).cuda()
    kv_indices = torch.from_numpy(indices).cuda()
    seq_lens = torch.tensor(lens, dtype=torch.int32, device="cuda")

    # page contents bit-exact: every sequence sees prefix + its own suffix, rounded to bf16 once
    gk, gv = pool.gather(0, kv_indptr, kv_indices, seq_lens)
    for r in range(n):
        want_k = oracle.round_bf16(ks[r].transpose(1, 0, 2))
        want_v = oracle.round_bf16(vs[r].transpose(1, 0, 2))
        np.testing.assert_array_equal(gk[r].float().cpu().numpy(), want_k)
        np.testing.assert_array_equal(gv[r].float().cpu().numpy(), want_v)
    # the owner's partial page still holds only the prefix rows (copy-on-write left it alone)
    ok_, ov_ = pool.gather(0, torch.tensor([0, len(owner_table)], dtype=torch.int32, device="cuda"),
                           torch.tensor(owner_table, dtype=torch.int32, device="cuda"),
                           torch.tensor([prefix_len], dtype=torch.int32, device="cuda"))
    np.testing.assert_array_equal(ok_[0].float().cpu().numpy(), oracle.round_bf16(kp.transpose(1, 0, 2)))

    q = rng.standard_normal((n, HQ, D)).astype(np.float32)
    out = paged.paged_decode(pool, 0, torch.from_numpy(q).cuda(), kv_indptr, kv_indices, seq_lens,
                             out_dtype=torch.float32).cpu().numpy()
    for r in range(n):
        want = oracle.attention(q[r:r + 1], ks[r].transpose(1, 0, 2).copy(), vs[r].transpose(1, 0, 2).copy(),
                                D ** -0.5)[0]
        assert float(np.abs(out[r] - want).max()) <= TOL
    assert paged.device_error(0) == (0, 0)
