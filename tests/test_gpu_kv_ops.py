"""KV append / page copy / gather / slot mapping / argmax on the GPU, bit-exact
against the oracle (every comparison is on bf16 bit patterns or integers)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import oracle.host_ref as ref
from mitten_b200 import paged
from tests.paged_case import make_case

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("hkv,d,ps", [(2, 64, 16), (4, 128, 16), (1, 256, 16), (2, 64, 8), (3, 64, 32)])
def test_append_gather_bit_exact(cuda_device, hkv, d, ps):
    lens = [1, 15, 16, 17, 100, 0, 333]
    case = make_case(lens, hkv, d, page_size=ps, seed=11, extra_pages=1)
    ks, vs = case.pool.gather(0, case.kv_indptr, case.kv_indices, case.seq_lens)
    torch.cuda.synchronize()
    for r, n in enumerate(lens):
        want_k = oracle.rne_bf16_bits(case.k[r].transpose(1, 0, 2))
        want_v = oracle.rne_bf16_bits(case.v[r].transpose(1, 0, 2))
        np.testing.assert_array_equal(_bits(ks[r]), want_k)
        np.testing.assert_array_equal(_bits(vs[r]), want_v)
    assert paged.device_error(0) == (0, 0)


def test_append_bf16_source_and_strided_rows(cuda_device):
    # k/v as column slices of a fused [n, (Hq + 2 Hkv) * D] projection output.
    n, hq, hkv, d, ps = 50, 14, 2, 64, 16
    pool = paged.PagedKVPool(2, 16, ps, hkv, d, device=cuda_device)
    fused = torch.randn(n, (hq + 2 * hkv) * d, device=cuda_device).to(torch.bfloat16)
    k = fused[:, hq * d:(hq + hkv) * d]
    v = fused[:, (hq + hkv) * d:]
    pages = [5, 2, 9, 14]
    slots = torch.tensor([pages[t // ps] * ps + t % ps for t in range(n)], dtype=torch.int64, device=cuda_device)
    pool.append(1, k, v, slots)
    torch.cuda.synchronize()
    kp = pool.k_pages(1)  # [pages, hkv, ps, d]
    for t in range(n):
        p, o = pages[t // ps], t % ps
        assert torch.equal(kp[p, :, o, :].reshape(-1).view(torch.int16), k[t].reshape(-1).view(torch.int16))
        assert torch.equal(pool.v_pages(1)[p, :, o, :].reshape(-1).view(torch.int16),
                           v[t].reshape(-1).view(torch.int16))
    # layer 0 untouched
    assert int(pool.storage[0].view(torch.int16).abs().sum()) == 0


def test_append_negative_slot_skips(cuda_device):
    pool = paged.PagedKVPool(1, 4, 16, 1, 64, device=cuda_device)
    k = torch.ones(3, 1, 64, device=cuda_device)
    slots = torch.tensor([-1, 5, -1], dtype=torch.int64, device=cuda_device)
    pool.append(0, k, k, slots)
    torch.cuda.synchronize()
    written = (pool.storage != 0).sum().item()
    assert written == 2 * 64  # one token row in K and one in V


def test_page_copy_all_layers(cuda_device):
    layers, pages, ps, hkv, d = 3, 32, 16, 2, 64
    pool = paged.PagedKVPool(layers, pages, ps, hkv, d, device=cuda_device)
    pool.storage.copy_(torch.randn_like(pool.storage, dtype=torch.float32).to(torch.bfloat16))
    before = pool.storage.clone()
    src = torch.tensor([3, 7, 30, 11], dtype=torch.int32, device=cuda_device)
    dst = torch.tensor([4, 0, 31, 11], dtype=torch.int32, device=cuda_device)
    pool.page_copy(src, dst)
    torch.cuda.synchronize()
    want = before.clone()
    for s, t in zip(src.tolist(), dst.tolist()):
        want[:, :, t] = before[:, :, s]
    assert torch.equal(pool.storage.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("layers,ps,hkv,d", [(2, 16, 2, 64), (1, 8, 1, 64), (2, 16, 4, 128), (1, 16, 1, 256),
                                             (1, 32, 8, 128)])
def test_page_copy_many_pairs(cuda_device, layers, ps, hkv, d):
    """Slabs of 1-16 KB take the bulk-copy kernel (several units per CTA, so
    every ring wraps); 64 KB slabs the vector kernel.  Bit-exact, including a
    pair whose source is its destination."""
    pages = 2048
    pool = paged.PagedKVPool(layers, pages, ps, hkv, d, device=cuda_device)
    pool.storage.copy_(torch.randn_like(pool.storage, dtype=torch.float32).to(torch.bfloat16))
    before = pool.storage.clone()
    rng = np.random.default_rng(ps * hkv + d)
    perm = rng.permutation(pages)
    n = 700
    src_l, dst_l = perm[:n].tolist(), perm[n:2 * n].tolist()
    dst_l[5] = src_l[5]
    src = torch.tensor(src_l, dtype=torch.int32, device=cuda_device)
    dst = torch.tensor(dst_l, dtype=torch.int32, device=cuda_device)
    paged.device_error(0, clear=True)
    pool.page_copy(src, dst)
    torch.cuda.synchronize()
    want = before.clone()
    want[:, :, torch.tensor(dst_l)] = before[:, :, torch.tensor(src_l)]
    assert torch.equal(pool.storage.view(torch.int16), want.view(torch.int16))
    assert paged.device_error(0) == (0, 0)


def test_page_copy_bad_page_is_flagged_not_faulted(cuda_device):
    pool = paged.PagedKVPool(1, 64, 16, 2, 64, device=cuda_device)
    pool.storage.copy_(torch.randn_like(pool.storage, dtype=torch.float32).to(torch.bfloat16))
    before = pool.storage.clone()
    src = torch.tensor([1, 2, 10 ** 6], dtype=torch.int32, device=cuda_device)
    dst = torch.tensor([3, 4, 5], dtype=torch.int32, device=cuda_device)
    paged.device_error(0, clear=True)
    pool.page_copy(src, dst)
    torch.cuda.synchronize()
    code, detail = paged.device_error(0, clear=True)
    assert code == 1 and detail == 2
    want = before.clone()
    want[:, :, 3] = before[:, :, 1]
    want[:, :, 4] = before[:, :, 2]
    assert torch.equal(pool.storage.view(torch.int16), want.view(torch.int16))


def test_slot_mapping_matches_python(cuda_device):
    rng = np.random.default_rng(5)
    ps = 16
    q_lens = [3, 0, 1, 40, 7]
    starts = [0, 0, 33, 5, 200]
    qo, pos, tables, kvp = [0], [], [], [0]
    for ql, st in zip(q_lens, starts):
        npg = (st + ql + ps - 1) // ps + 1
        tables.append(rng.choice(1000, npg, replace=False).tolist())
        kvp.append(kvp[-1] + npg)
        pos.extend(range(st, st + ql))
        qo.append(qo[-1] + ql)
    kvi = sum(tables, [])
    dev = cuda_device
    slots = paged.build_slot_mapping(torch.tensor(qo, dtype=torch.int32, device=dev),
                                     torch.tensor(pos, dtype=torch.int32, device=dev),
                                     torch.tensor(kvp, dtype=torch.int32, device=dev),
                                     torch.tensor(kvi, dtype=torch.int32, device=dev), ps)
    want = []
    for r, (ql, st) in enumerate(zip(q_lens, starts)):
        for p in range(st, st + ql):
            want.append(tables[r][p // ps] * ps + p % ps)
    assert slots.cpu().tolist() == want


def test_slot_mapping_flags_position_past_pages(cuda_device):
    dev = cuda_device
    paged.device_error(0, clear=True)
    slots = paged.build_slot_mapping(torch.tensor([0, 1], dtype=torch.int32, device=dev),
                                     torch.tensor([40], dtype=torch.int32, device=dev),
                                     torch.tensor([0, 2], dtype=torch.int32, device=dev),
                                     torch.tensor([3, 4], dtype=torch.int32, device=dev), 16)
    assert slots.cpu().tolist() == [-1]
    code, _ = paged.device_error(0, clear=True)
    assert code == 5


def test_argmax_first_strict_max(cuda_device):
    rng = np.random.default_rng(9)
    rows = rng.standard_normal((6, 151936)).astype(np.float32)
    rows[1, 100] = rows[1, 5000] = 50.0          # tie -> first index
    rows[2, :] = -np.inf                         # nothing beats -inf -> 0
    rows[3, 10] = np.nan                         # NaN never wins
    rows[3, 11] = 99.0
    rows[4, :] = 0.0
    rows[5, -1] = 1e30
    got = paged.argmax_rows(torch.from_numpy(rows).to(cuda_device)).cpu().tolist()
    want = [ref.sample_token(r.tolist(), 0.0) for r in rows]
    assert got == want
