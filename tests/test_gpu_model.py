"""The model call site end to end: scheduler mirror + paged model + kernels
against the numpy restatement of Qwen3_5Model (oracle/model_ref.py).

Pass criteria: greedy tokens equal to the oracle's for
all 32 steps of every request, and the logits every token is chosen from
within a stated tolerance.  The oracle stores its cache rows rounded to
bf16 (the pool's storage precision; the reference f32 path with bf16 K/V).
The model's attention runs with MTN_ATTN_SPLIT_BF16 (Q and P reach the
tensor cores as bf16 hi + lo pairs), so what remains is f32 summation order
(BLAS vs numpy, tensor-core accumulation) and the occasional K/V element
whose f32 value rounds to a different bf16 neighbour on the two sides.

The oracle is also run teacher-forced on the kernel path's own tokens; the
largest logit error over every sampled step is printed and bounded.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from mitten_b200 import host, model as M
from oracle import model_ref as R

pytestmark = pytest.mark.gpu

# max |logit_gpu - logit_oracle| over every sampled step (teacher-forced)
LOGIT_TOL_SMALL = 1e-2
LOGIT_TOL_CONFIG1 = 1e-2  # 24 layers of N(0, 0.02) weights


def shape_of(cfg: R.QwenShape) -> M.DecoderShape:
    return M.DecoderShape(hidden=cfg.hidden, layers=cfg.layers, hq=cfg.hq, hkv=cfg.hkv, head_dim=cfg.head_dim,
                          inter=cfg.inter, vocab=cfg.vocab, eps=cfg.eps, theta=cfg.theta,
                          partial_rotary=cfg.partial_rotary, gated_q=cfg.gated_q, qk_norm=cfg.qk_norm,
                          phantom=cfg.phantom, mlp=cfg.mlp)


def run_engine(cfg, weights, prompts, steps, num_pages=256, budget=512, max_decode=8):
    model = M.QwenPagedModel(shape_of(cfg), weights, num_pages, 16)
    sched = host.Scheduler(num_pages, 16, max_prefill_tokens_per_iter=budget, max_decode_batch_size=max_decode,
                           eos_token_ids=(cfg.vocab,))  # no token id stops a request early
    for rid, p in enumerate(prompts):
        sched.add_request(rid, p.astype(np.uint32), temperature=0.0, max_new_tokens=steps)
    logits_by_req = {rid: [] for rid in range(len(prompts))}
    iters = 0
    while sched.num_active():
        b = sched.schedule()
        assert b is not None
        lg = model.forward(b)
        done_prompt = [sched.request_info(int(r))["device_len"] + int(b.qo_indptr[i + 1] - b.qo_indptr[i])
                       >= len(prompts[int(r)]) for i, r in enumerate(b.req_ids)]
        lg_h = lg.cpu().numpy()
        for i, r in enumerate(b.req_ids):
            if done_prompt[i]:
                logits_by_req[int(r)].append(lg_h[i])
        tok = M.paged.argmax_rows(lg).cpu().numpy().astype(np.uint32)
        sched.process_tokens(tok)
        iters += 1
        assert iters < 10_000
    outs = [sched.request_output(rid) for rid in range(len(prompts))]
    return outs, logits_by_req, model, sched


def compare(cfg, weights, prompts, steps, tol, **kw):
    """Free-running greedy tokens must equal the oracle's, every request, every step.  The oracle is
    also run teacher-forced on the kernel path's tokens to measure the logit error of every sampled
    step (the first-strict-max choice is compared with the oracle's at each step too)."""
    outs, lg_gpu, model, sched = run_engine(cfg, weights, prompts, steps, **kw)
    ref = R.RefModel(cfg, weights, kv_round=True)
    want = R.generate(ref, prompts, steps)
    forced = R.RefModel(cfg, weights, kv_round=True)
    err, gaps = 0.0, []
    for rid, prompt in enumerate(prompts):
        assert len(outs[rid]) == steps
        lg = forced.forward(rid, prompt, np.arange(len(prompt)))
        for s in range(steps):
            err = max(err, float(np.abs(lg_gpu[rid][s] - lg).max()))
            best = R.greedy_first_max(lg)
            top2 = np.partition(lg, -2)[-2:]
            gaps.append(float(top2[1] - top2[0]))
            assert outs[rid][s] == best, (rid, s, outs[rid][s], best)
            if s + 1 < steps:
                lg = forced.forward(rid, np.array([outs[rid][s]]), np.array([len(prompt) + s]))
    print(f"max |logit error| (teacher forced) {err:.3e}; smallest top-2 logit gap {min(gaps):.3e}")
    assert outs == want
    assert err <= tol, err
    assert sched.num_active() == 0
    return err


def test_small_model_chunked_prefill_and_mixed_batches(cuda_device):
    cfg = R.QwenShape(hidden=256, layers=3, hq=14, hkv=2, head_dim=64, inter=512, vocab=4096)
    w = R.random_weights(cfg, seed=0)
    rng = np.random.default_rng(1)
    prompts = [rng.integers(0, cfg.vocab, n).astype(np.int64) for n in (40, 17, 63, 5)]
    # a 48-token prefill budget cuts prompts into chunks and mixes prefill with decode rows
    compare(cfg, w, prompts, 12, LOGIT_TOL_SMALL, budget=48)


def test_gemma_shaped_mqa_call_site(cuda_device):
    """The Gemma attention call site (MQA, head_dim 256, GeGLU, theta 1e4, no phantom row) at reduced
    width and depth, with chunked prefill mixed into decode batches."""
    import dataclasses

    cfg = dataclasses.replace(R.GEMMA_2B, hidden=512, layers=3, inter=1024, vocab=8192)
    w = R.random_weights(cfg, seed=7)
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, cfg.vocab, n).astype(np.int64) for n in (90, 33, 140, 12)]
    compare(cfg, w, prompts, 10, LOGIT_TOL_SMALL, budget=96)


def test_config1_greedy_32_steps(cuda_device):
    """Qwen2.5-0.5B shape, N(0, 0.02) weights (seed 0), 4 prompts of 128 ids (seed 1)."""
    cfg = R.CONFIG1
    w = R.random_weights(cfg, seed=0)
    rng = np.random.default_rng(1)
    prompts = [rng.integers(0, cfg.vocab, 128).astype(np.int64) for _ in range(4)]
    compare(cfg, w, prompts, 32, LOGIT_TOL_CONFIG1, num_pages=512)


def test_engine_cuda_graph_decode_matches_eager(cuda_device):
    """Engine with the decode forward replayed from CUDA graphs (static metadata buffers refreshed per
    step) emits the same tokens as the eager engine, across page growth and a shrinking batch."""
    cfg = R.QwenShape(hidden=256, layers=3, hq=14, hkv=2, head_dim=64, inter=512, vocab=4096)
    w = R.random_weights(cfg, seed=3)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, cfg.vocab, n).astype(np.uint32) for n in (30, 7, 50)]
    steps = [40, 25, 33]  # requests finish at different iterations: batch sizes 3, 2, 1 all replay
    outs = {}
    for graphs in (False, True):
        model = M.QwenPagedModel(shape_of(cfg), w, 128, 16)
        sched = host.Scheduler(128, 16, max_prefill_tokens_per_iter=512, max_decode_batch_size=8,
                               eos_token_ids=(cfg.vocab,))
        for rid, (p, n) in enumerate(zip(prompts, steps)):
            sched.add_request(rid, p, temperature=0.0, max_new_tokens=n)
        M.Engine(model, sched, cuda_graphs=graphs).run()
        outs[graphs] = [sched.request_output(r) for r in range(len(prompts))]
        assert [len(o) for o in outs[graphs]] == steps
    assert outs[True] == outs[False]
    assert M.paged.device_error(0) == (0, 0)
