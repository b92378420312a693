"""The model call site end to end: scheduler mirror + paged model + kernels
against the numpy restatement of Qwen3_5Model (oracle/model_ref.py).

Pass criteria: greedy tokens equal to the oracle's for
32 steps, and the logits every token is chosen from within a stated
tolerance.  The oracle stores its cache rows rounded to bf16 (the pool's
storage precision; the reference f32 path with bf16 K/V), so the remaining
differences are BLAS summation order and the bf16 Q and P operands of the
tensor-core attention (measured: with those two roundings emulated in the
oracle the logit error falls from ~3e-2 to ~5e-3 at config 1).

The oracle is also run teacher-forced on the kernel path's own tokens, so a
free-running divergence is checked where it happens: it passes only at a
near-tie, where the oracle's logit for the kernel path's token is within
2 x the logit tolerance of the oracle's maximum.  At config 1 (seeds 0 and
1) 3 of 4 requests match for all 32 steps; request 3 matches for 20 steps
and then takes a token whose oracle logit is 0.0073 below the maximum.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from mitten_b200 import host, model as M
from oracle import model_ref as R

pytestmark = pytest.mark.gpu

# max |logit_gpu - logit_oracle| over every sampled step (teacher-forced)
LOGIT_TOL_SMALL = 1e-2   # 3 layers: measured 4.1e-3
LOGIT_TOL_CONFIG1 = 5e-2  # 24 layers of N(0, 0.02) weights: measured 3.3e-2


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
    """Free-running greedy tokens must equal the oracle's; the oracle is then also run teacher-forced on
    the kernel path's tokens so a divergence can be told apart: it is accepted only at a near-tie,
    where the oracle's logit for the kernel path's token is within 2 * tol of its maximum."""
    outs, lg_gpu, model, sched = run_engine(cfg, weights, prompts, steps, **kw)
    ref = R.RefModel(cfg, weights, kv_round=True)
    lg_ref = []
    want = R.generate(ref, prompts, steps, logits_out=lg_ref)
    # teacher-forced oracle: the same prompts followed by the kernel path's tokens
    forced = R.RefModel(cfg, weights, kv_round=True)
    err, report = 0.0, []
    for rid, prompt in enumerate(prompts):
        assert len(outs[rid]) == steps
        lg = forced.forward(rid, prompt, np.arange(len(prompt)))
        for s in range(steps):
            err = max(err, float(np.abs(lg_gpu[rid][s] - lg).max()))
            tok = outs[rid][s]
            best = R.greedy_first_max(lg)
            gap = float(lg[best] - lg[tok])
            if tok != best:
                report.append((rid, s, tok, best, gap))
                assert gap <= 2 * tol, (rid, s, tok, best, gap)
            if s + 1 < steps:
                lg = forced.forward(rid, np.array([tok]), np.array([len(prompt) + s]))
    print(f"max |logit error| (teacher forced) {err:.3e}; near-tie divergences {report}")
    assert err <= tol, err
    if not report:
        assert outs == want
    assert sched.num_active() == 0
    return err, report


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
    err, report = compare(cfg, w, prompts, 32, LOGIT_TOL_CONFIG1, num_pages=512)
    assert len(report) <= 1  # near-ties, each a free-running divergence


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
