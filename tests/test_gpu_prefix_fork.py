"""Prefix sharing with copy-on-write driven by the scheduler, through the
whole engine loop, on a reduced BASELINE config 3 (Qwen2.5-7B attention
shapes: 28 query / 4 kv heads, head_dim 128; 2 narrow layers).

A parent request prefills a 1032-token random prefix: 64 full pages of 16
plus one page holding 8 tokens.  Eight children fork off it
(mtn_sched_fork), each with a unique suffix of U[64, 512] tokens, and
share every prefix page, the partial one included.  The first write into
the shared partial page -- a child's suffix, or the parent's next decode
token -- arrives with a copy-on-write pair in the batch; the engine's
forward runs mtn_page_copy on it before any kernel reads or writes.

Checked every iteration: each CoW pair copies the shared partial page onto
a page only its writer holds, each request copies at most once, and every
page's reference count equals its holders.  At the end: every request's
greedy tokens equal the oracle model's on its full prompt (parent: the
prefix; child: prefix + suffix), and every page is back (free or held by
the radix cache alone).
"""
from __future__ import annotations

from collections import Counter

import numpy as np
import pytest
import torch

from mitten_b200 import _lib, host, model as M
from oracle import model_ref as R

pytestmark = pytest.mark.gpu

CFG = R.QwenShape(hidden=256, layers=2, hq=28, hkv=4, head_dim=128, inter=512, vocab=4096)
PREFIX, PS, STEPS = 1032, 16, 8


def _shape(cfg):
    return M.DecoderShape(hidden=cfg.hidden, layers=cfg.layers, hq=cfg.hq, hkv=cfg.hkv, head_dim=cfg.head_dim,
                          inter=cfg.inter, vocab=cfg.vocab)


def _check_refcounts(s, ids, num_pages):
    holders = Counter()
    for r in ids:
        if s.request_info(r)["state"] in (_lib.MTN_REQ_WAITING, _lib.MTN_REQ_PREFILLING, _lib.MTN_REQ_DECODING):
            holders.update(s.request_pages(r))
    holders.update(s.tree_pages())
    for p in range(num_pages):
        assert s.page_refcount(p) == holders.get(p, 0), p


def test_forked_prefix_copy_on_write_through_engine(cuda_device):
    w = R.random_weights(CFG, seed=5)
    rng = np.random.default_rng(5)
    prefix = rng.integers(0, CFG.vocab, PREFIX).astype(np.uint32)
    srng = np.random.default_rng(6)
    suffixes = [srng.integers(0, CFG.vocab, int(srng.integers(64, 513))).astype(np.uint32) for _ in range(8)]
    num_pages = 2048
    model = M.QwenPagedModel(_shape(CFG), w, num_pages, PS)
    s = host.Scheduler(num_pages, PS, max_prefill_tokens_per_iter=4096, max_decode_batch_size=16,
                       eos_token_ids=(CFG.vocab,))
    s.add_request(0, prefix, temperature=0.0, max_new_tokens=STEPS)
    ids = [0]
    cow_writers = []
    partial = None
    it = 0
    while s.num_active():
        b = s.schedule()
        assert b is not None
        if it == 1:  # the parent's prompt is done: fork the children off it
            assert s.request_info(0)["device_len"] == PREFIX
        for src, dst in zip(b.cow_src.tolist(), b.cow_dst.tolist()):
            assert src == partial, "only the shared partial prefix page is ever copied"
            (writer,) = [int(b.req_ids[i]) for i in range(b.n_reqs) if dst in b.page_table()[i]]
            cow_writers.append(writer)
            assert s.page_refcount(dst) == 1
        _check_refcounts(s, ids, num_pages)
        lg = model.forward(b)
        tok = M.paged.argmax_rows(lg).cpu().numpy().astype(np.uint32)
        s.process_tokens(tok)
        if it == 0:
            partial = s.request_pages(0)[PREFIX // PS]
            for k, suf in enumerate(suffixes):
                s.fork(0, k + 1, suf, temperature=0.0, max_new_tokens=STEPS)
                ids.append(k + 1)
            assert s.page_refcount(partial) == 9  # the parent and eight children
        it += 1
        assert it < 200
    assert M.paged.device_error(0) == (0, 0)
    # every holder of the partial page but the last one to write copied it, once
    assert len(cow_writers) == len(set(cow_writers)) == 8
    # tokens equal the oracle model's on each full prompt
    ref = R.RefModel(CFG, w, kv_round=True)
    prompts = [prefix.astype(np.int64)] + [np.concatenate([prefix, suf]).astype(np.int64) for suf in suffixes]
    want = R.generate(ref, prompts, STEPS)
    got = [s.request_output(r) for r in range(9)]
    assert got == want
    tree = s.tree_pages()
    assert all(s.page_refcount(p) == 1 for p in tree)
    assert s.free_pages() + len(tree) == num_pages


def test_forked_prefix_decode_graph_lists_more_table_entries_than_pages(cuda_device):
    """The decode CUDA graph's page-table buffer holds the batch's table
    entries, which with shared prefix pages outnumber the pool's pages: nine
    requests list the 65 prefix pages each (585 entries) in a pool of 256
    pages.  The graph-replayed engine must emit the oracle model's tokens."""
    w = R.random_weights(CFG, seed=5)
    rng = np.random.default_rng(15)
    prefix = rng.integers(0, CFG.vocab, PREFIX).astype(np.uint32)
    suffixes = [rng.integers(0, CFG.vocab, 20).astype(np.uint32) for _ in range(8)]
    num_pages = 256
    model = M.QwenPagedModel(_shape(CFG), w, num_pages, PS)
    s = host.Scheduler(num_pages, PS, max_prefill_tokens_per_iter=4096, max_decode_batch_size=16,
                       eos_token_ids=(CFG.vocab,))
    s.add_request(0, prefix, temperature=0.0, max_new_tokens=STEPS)
    eng = M.Engine(model, s, cuda_graphs=True)
    eng.step()  # the parent's prefill
    for k, suf in enumerate(suffixes):
        s.fork(0, k + 1, suf, temperature=0.0, max_new_tokens=STEPS)
    entries = 0
    while s.num_active():
        b = s.schedule()
        assert b is not None
        if not b.n_prefill:
            entries = max(entries, int(b.kv_indptr[-1]))
        lg = model.decode_step(b)
        s.process_tokens(M.paged.argmax_rows(lg).cpu().numpy().astype(np.uint32))
    assert entries > num_pages
    assert M.paged.device_error(0) == (0, 0)
    ref = R.RefModel(CFG, w, kv_round=True)
    prompts = [prefix.astype(np.int64)] + [np.concatenate([prefix, suf]).astype(np.int64) for suf in suffixes]
    want = R.generate(ref, prompts, STEPS)
    got = [s.request_output(r) for r in range(9)]
    assert got == want
