"""KV offload and the prefill -> decode handoff on the GPU.

Pages pack bit-exactly into a flat buffer (device, or pinned host memory)
and unpack into other pages.  Then the handoff through the engine: a
prefill worker (its own pool and scheduler) prefills three requests and
exports them; their pages are packed, the decode worker imports them onto
pages of its own pool, unpacks, and decodes to the end; and an offload
round trip exports a request to pinned host memory, lets its pages be
reused, and brings it back onto new pages of the same pool.  Greedy tokens
equal the oracle model's in every case."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from mitten_b200 import host, model as M, paged
from oracle import model_ref as R
from tests.paged_case import make_case

pytestmark = pytest.mark.gpu

CFG = R.QwenShape(hidden=256, layers=2, hq=14, hkv=2, head_dim=64, inter=512, vocab=4096)
STEPS = 10


def _shape(cfg):
    return M.DecoderShape(hidden=cfg.hidden, layers=cfg.layers, hq=cfg.hq, hkv=cfg.hkv, head_dim=cfg.head_dim,
                          inter=cfg.inter, vocab=cfg.vocab)


@pytest.mark.parametrize("where", ["device", "host"])
def test_pack_unpack_round_trip(cuda_device, where):
    case = make_case([300, 77, 1000], 2, 64, seed=3, layers=3, layer=1, extra_pages=4)
    pool = case.pool
    src = torch.tensor([5, 0, 17, 9], dtype=torch.int32, device="cuda")
    shape = (4, pool.num_layers, 2, pool.num_kv_heads, pool.page_size, pool.head_dim)
    buf = torch.empty(shape, dtype=torch.bfloat16, device="cuda") if where == "device" \
        else torch.empty(shape, dtype=torch.bfloat16).pin_memory()
    paged.pack_pages(pool, src, out=buf)
    torch.cuda.synchronize()
    want = pool.storage[:, :, src.long()].permute(2, 0, 1, 3, 4, 5).cpu()
    assert torch.equal(buf.cpu().view(torch.int16), want.view(torch.int16))
    dst = torch.tensor([pool.num_pages - 1, pool.num_pages - 2, 3, 30], dtype=torch.int32, device="cuda")
    paged.unpack_pages(pool, buf, dst)
    torch.cuda.synchronize()
    assert torch.equal(pool.storage[:, :, dst.long()].view(torch.int16), pool.storage[:, :, src.long()].view(torch.int16))
    assert paged.device_error(0) == (0, 0)


def _decode_loop(model, sched):
    while sched.num_active():
        b = sched.schedule()
        if b is None:
            break
        tok = paged.argmax_rows(model.forward(b)).cpu().numpy().astype(np.uint32)
        sched.process_tokens(tok)


def test_prefill_worker_hands_off_to_decode_worker(cuda_device):
    w = R.random_weights(CFG, seed=21)
    rng = np.random.default_rng(22)
    prompts = [rng.integers(0, CFG.vocab, n).astype(np.uint32) for n in (70, 33, 129)]
    pre_model, dec_model = M.QwenPagedModel(_shape(CFG), w, 128, 16), M.QwenPagedModel(_shape(CFG), w, 256, 16)
    pre = host.Scheduler(128, 16, max_prefill_tokens_per_iter=1024, max_decode_batch_size=8, eos_token_ids=(CFG.vocab,))
    dec = host.Scheduler(256, 16, max_prefill_tokens_per_iter=1024, max_decode_batch_size=8, eos_token_ids=(CFG.vocab,))
    for rid, p in enumerate(prompts):
        pre.add_request(rid, p, temperature=0.0, max_new_tokens=STEPS)
    b = pre.schedule()
    assert b.n_prefill == 3
    tok = paged.argmax_rows(pre_model.forward(b)).cpu().numpy().astype(np.uint32)
    pre.process_tokens(tok)
    for rid, p in enumerate(prompts):
        h = pre.export_request(rid)  # KvHandoff: pages, device_len, first token
        staged = paged.pack_pages(pre_model.pool, torch.tensor(h["pages"], dtype=torch.int32, device="cuda"))
        pages = dec.import_request(rid, p, h["outputs"], h["device_len"], 0.0, STEPS)
        paged.unpack_pages(dec_model.pool, staged, torch.tensor(pages, dtype=torch.int32, device="cuda"))
    assert pre.num_active() == 0 and pre.free_pages() + pre.cached_pages() == 128
    _decode_loop(dec_model, dec)
    want = R.generate(R.RefModel(CFG, w, kv_round=True), [p.astype(np.int64) for p in prompts], STEPS)
    assert [dec.request_output(r) for r in range(3)] == want
    assert paged.device_error(0) == (0, 0)


def test_offload_to_host_and_back(cuda_device):
    w = R.random_weights(CFG, seed=31)
    rng = np.random.default_rng(32)
    prompts = [rng.integers(0, CFG.vocab, n).astype(np.uint32) for n in (90, 40)]
    model = M.QwenPagedModel(_shape(CFG), w, 64, 16)
    s = host.Scheduler(64, 16, max_prefill_tokens_per_iter=1024, max_decode_batch_size=8, eos_token_ids=(CFG.vocab,))
    for rid, p in enumerate(prompts):
        s.add_request(rid, p, temperature=0.0, max_new_tokens=STEPS)
    for _ in range(4):  # prefill + 3 decode steps
        b = s.schedule()
        s.process_tokens(paged.argmax_rows(model.forward(b)).cpu().numpy().astype(np.uint32))
    h = s.export_request(0)  # swap request 0 out to pinned host memory
    idx = torch.tensor(h["pages"], dtype=torch.int32, device="cuda")
    host_buf = torch.empty((len(h["pages"]), CFG.layers, 2, CFG.hkv, 16, CFG.head_dim), dtype=torch.bfloat16).pin_memory()
    paged.pack_pages(model.pool, idx, out=host_buf)
    torch.cuda.synchronize()
    model.pool.storage[:, :, idx.long()] = 0  # its pages are reused meanwhile
    for _ in range(3):  # request 1 keeps decoding alone
        b = s.schedule()
        s.process_tokens(paged.argmax_rows(model.forward(b)).cpu().numpy().astype(np.uint32))
    pages = s.import_request(0, prompts[0], h["outputs"], h["device_len"], 0.0, STEPS)
    paged.unpack_pages(model.pool, host_buf, torch.tensor(pages, dtype=torch.int32, device="cuda"))
    _decode_loop(model, s)
    want = R.generate(R.RefModel(CFG, w, kv_round=True), [p.astype(np.int64) for p in prompts], STEPS)
    assert [s.request_output(r) for r in range(2)] == want
    assert paged.device_error(0) == (0, 0)
