"""Seeded paged-KV test cases shared by the GPU tests: random page tables,
K/V written through the library's own append kernel, and the oracle's view
of the same data as contiguous per-request caches."""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

import oracle
from mitten_b200 import paged


@dataclass
class Case:
    pool: paged.PagedKVPool
    lens: list[int]
    tables: list[list[int]]
    k: list[np.ndarray]   # per sequence [len, Hkv, D] f32 (pre-rounding)
    v: list[np.ndarray]
    kv_indptr: torch.Tensor
    kv_indices: torch.Tensor
    seq_lens: torch.Tensor
    max_pages: int

    def oracle_cache(self, r: int, layer_round: bool = True, phantom: bool = True):
        """[Hkv, T, D] f32 contiguous cache of sequence r as the reference holds it."""
        k = self.k[r].transpose(1, 0, 2)
        v = self.v[r].transpose(1, 0, 2)
        if layer_round:
            k, v = oracle.round_bf16(k), oracle.round_bf16(v)
        if phantom:
            z = np.zeros((k.shape[0], 1, k.shape[2]), np.float32)
            k = np.concatenate([z, k], axis=1)
            v = np.concatenate([z, v], axis=1)
        return k, v


def make_case(lens, hkv, d, page_size=16, num_pages=None, extra_pages=0, seed=0, layers=1, layer=0,
              device="cuda", scale_kv=1.0) -> Case:
    rng = np.random.default_rng(seed)
    need = [(n + page_size - 1) // page_size + extra_pages for n in lens]
    total = sum(need)
    if num_pages is None:
        num_pages = max(total + 7, 8)
    pool = paged.PagedKVPool(layers, num_pages, page_size, hkv, d, device=device)
    perm = rng.permutation(num_pages)[:total].astype(np.int32)
    tables, indptr, off = [], [0], 0
    for n in need:
        tables.append(perm[off:off + n].tolist())
        off += n
        indptr.append(off)
    ks = [(rng.standard_normal((n, hkv, d)) * scale_kv).astype(np.float32) for n in lens]
    vs = [(rng.standard_normal((n, hkv, d)) * scale_kv).astype(np.float32) for n in lens]
    # write through the append kernel, one slot per token
    slots = []
    for r, n in enumerate(lens):
        for t in range(n):
            slots.append(tables[r][t // page_size] * page_size + t % page_size)
    if slots:
        kt = torch.from_numpy(np.concatenate(ks)).to(device)
        vt = torch.from_numpy(np.concatenate(vs)).to(device)
        st = torch.tensor(slots, dtype=torch.int64, device=device)
        pool.append(layer, kt, vt, st)
    return Case(pool, list(lens), tables, ks, vs,
                torch.tensor(indptr, dtype=torch.int32, device=device),
                torch.tensor(perm[:total] if total else [0], dtype=torch.int32, device=device),
                torch.tensor(lens, dtype=torch.int32, device=device) if lens else torch.zeros(0, dtype=torch.int32,
                                                                                            device=device),
                max(need) if need else 0)
