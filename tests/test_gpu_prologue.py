"""The fused attention prologue (mtn_qkv_prologue) against the unfused path
it replaces (torch RMSNorm (1 + w) and rotate-half RoPE, then the append
kernel), on the GPU.

q: within 1e-5 relative (the RMSNorm sum runs in another order).  K/V in the
pool: the bf16 of the same values, so at most one bf16 ulp apart and almost
all bit-identical (a last-bit f32 difference can flip the rounding of an
element lying on a bf16 boundary).  Tokens with slot -1 store nothing."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from mitten_b200 import _lib, paged
from mitten_b200.model import _rms

pytestmark = pytest.mark.gpu


def _rope_ref(x, pos, inv_freq, rd):
    half = rd // 2
    ang = pos.float()[:, None, None] * inv_freq[None, None, :]
    c, s = torch.cos(ang), torch.sin(ang)
    x1, x2 = x[..., :half], x[..., half:rd]
    out = torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)
    return torch.cat([out, x[..., rd:]], dim=-1) if rd < x.shape[-1] else out


@pytest.mark.parametrize("d,hq,hkv,gated,dtype,rd", [(64, 14, 2, True, torch.float32, 64),
                                                     (128, 28, 4, True, torch.bfloat16, 128),
                                                     (256, 8, 1, False, torch.float32, 256),
                                                     (128, 8, 2, False, torch.float32, 64)])
def test_prologue_matches_unfused_path(cuda_device, d, hq, hkv, gated, dtype, rd):
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(d + hq)
    T, ps, num_pages = 300, 16, 64
    pool = paged.PagedKVPool(2, num_pages, ps, hkv, d, device=dev)
    qg = 2 if gated else 1
    qp = torch.randn((T, hq * qg * d), generator=g, device=dev).to(dtype)
    k = torch.randn((T, hkv * d), generator=g, device=dev).to(dtype)
    v = torch.randn((T, hkv * d), generator=g, device=dev).to(dtype)
    qw = (1.0 + 0.1 * torch.randn(d, generator=g, device=dev)).float()
    kw = (1.0 + 0.1 * torch.randn(d, generator=g, device=dev)).float()
    pos = torch.randint(0, 30000, (T,), generator=g, device=dev, dtype=torch.int32)
    inv = (1.0 / (1e6 ** (torch.arange(0, rd, 2, device=dev, dtype=torch.float32) / rd))).contiguous()
    slots = torch.randperm(num_pages * ps, generator=g, device=dev)[:T].to(torch.int64)
    slots[::7] = -1
    q_out = torch.empty((T, hq, d), dtype=torch.float32, device=dev)
    layer = 1
    _lib.check(_lib.lib().mtn_qkv_prologue(paged.C.byref(pool.layout), layer, qp.data_ptr(), k.data_ptr(), v.data_ptr(),
                                           paged._dtype_code(dtype), qp.shape[1], hkv * d, hkv * d, int(gated), hq,
                                           qw.data_ptr(), kw.data_ptr(), 1e-6, inv.data_ptr(), rd, pos.data_ptr(),
                                           slots.data_ptr(), T, q_out.data_ptr(), paged._stream(None)))
    torch.cuda.synchronize()
    q_in = qp.view(T, hq, qg, d)[:, :, 0, :].float()
    q_ref = _rope_ref(_rms(q_in, qw, 1e-6), pos, inv, rd)
    torch.testing.assert_close(q_out, q_ref, rtol=1e-5, atol=1e-5)
    k_ref = _rope_ref(_rms(k.view(T, hkv, d).float(), kw, 1e-6), pos, inv, rd).to(torch.bfloat16)
    v_ref = v.view(T, hkv, d).float().to(torch.bfloat16)
    # the pool rows at each stored slot: storage [layers][K|V][page][hkv][ps][d]
    ok = slots >= 0
    pg, off = slots[ok] // ps, slots[ok] % ps
    k_pool = pool.storage[layer, 0][pg, :, off]
    v_pool = pool.storage[layer, 1][pg, :, off]
    assert torch.equal(v_pool.view(torch.int16), v_ref[ok].view(torch.int16))
    kb, rb = k_pool.view(torch.int16).int(), k_ref[ok].view(torch.int16).int()
    same = (kb == rb).float().mean().item()
    assert same > 0.999 and (kb - rb).abs().max().item() <= 1, same
    # skipped tokens left the pool alone (it started zeroed and slots are distinct)
    assert paged.device_error(0) == (0, 0)


def test_prologue_rejects_bad_rotary_dim(cuda_device):
    pool = paged.PagedKVPool(1, 4, 16, 1, 64, device="cuda")
    z = torch.zeros(64, device="cuda")
    st = _lib.lib().mtn_qkv_prologue(paged.C.byref(pool.layout), 0, z.data_ptr(), z.data_ptr(), z.data_ptr(),
                                     _lib.MTN_DTYPE_F32, 64, 64, 64, 0, 1, None, None, 1e-6, z.data_ptr(), 32,
                                     z.data_ptr(), z.data_ptr(), 1, z.data_ptr(), None)
    assert st == _lib.MTN_EINVAL
