"""Device sampling (mtn_sample_rows) against the C restatement of the
reference's sample_token (oracle.sample_token, scheduler.rs:186-223):
token for token, on every row kind the CPU agreement test uses, on a mixed
greedy / temperature batch at config 1's vocabulary, and inside the engine
loop (each step's device pick equals the oracle's pick of the same logits
row; the reference's hash of logit bits makes a free-running comparison
with a CPU model meaningless, since any last-bit difference reseeds it)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from mitten_b200 import host, model as M, paged
from oracle import model_ref as R
from tests.test_sample_oracle import _rows

pytestmark = pytest.mark.gpu


@pytest.mark.filterwarnings("ignore::RuntimeWarning")
def test_sample_rows_match_oracle(cuda_device):
    by_vocab = {}
    for row, t in _rows():
        by_vocab.setdefault(row.size, []).append((row, t))
    for vocab, items in by_vocab.items():
        lg = torch.from_numpy(np.stack([r for r, _ in items])).cuda()
        temps = torch.tensor([t for _, t in items], dtype=torch.float32)
        got = paged.sample_rows(lg, temps).cpu().numpy().tolist()
        want = [oracle.sample_token(r, t) for r, t in items]
        assert got == want, (vocab, got, want)


def test_mixed_batch_config1_vocab(cuda_device):
    rng = np.random.default_rng(5)
    n, vocab = 64, 151936
    rows = (rng.standard_normal((n, vocab)) * 2.0).astype(np.float32)
    temps = np.where(np.arange(n) % 3 == 0, 0.0, rng.uniform(0.3, 1.5, n)).astype(np.float32)
    lg = torch.from_numpy(rows).cuda()
    t = torch.from_numpy(temps)
    paged.sample_rows(lg, t)  # warm
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    got = paged.sample_rows(lg, t)
    b.record()
    b.synchronize()
    print(f"64 rows x {vocab}: {a.elapsed_time(b):.3f} ms")
    want = [oracle.sample_token(rows[i], float(temps[i])) for i in range(n)]
    assert got.cpu().numpy().tolist() == want
    greedy = paged.argmax_rows(lg).cpu().numpy()
    assert all(got.cpu().numpy()[i] == greedy[i] for i in range(n) if temps[i] <= 0)


def test_engine_temperature_sampling_picks_the_oracles_token(cuda_device):
    cfg = R.QwenShape(hidden=256, layers=2, hq=14, hkv=2, head_dim=64, inter=512, vocab=4096)
    w = R.random_weights(cfg, seed=11)
    shape = M.DecoderShape(hidden=cfg.hidden, layers=cfg.layers, hq=cfg.hq, hkv=cfg.hkv, head_dim=cfg.head_dim,
                           inter=cfg.inter, vocab=cfg.vocab)
    model = M.QwenPagedModel(shape, w, 128, 16)
    sched = host.Scheduler(128, 16, max_prefill_tokens_per_iter=256, max_decode_batch_size=8,
                           eos_token_ids=(cfg.vocab,))
    rng = np.random.default_rng(12)
    temps = [0.0, 0.8, 1.0, 1.7]
    for rid, t in enumerate(temps):
        sched.add_request(rid, rng.integers(0, cfg.vocab, 20 + rid).astype(np.uint32), temperature=t,
                          max_new_tokens=12)
    steps = 0
    while sched.num_active():
        b = sched.schedule()
        lg = model.forward(b)
        tok = paged.sample_rows(lg, torch.from_numpy(b.temperatures)).cpu().numpy()
        lh = lg.cpu().numpy()
        for i in range(b.n_reqs):
            assert tok[i] == oracle.sample_token(lh[i], float(b.temperatures[i])), (steps, i)
        sched.process_tokens(tok.astype(np.uint32))
        steps += 1
    assert [len(sched.request_output(r)) for r in range(4)] == [12] * 4
    # the Engine class takes the same path
    sched2 = host.Scheduler(128, 16, max_prefill_tokens_per_iter=256, max_decode_batch_size=8,
                            eos_token_ids=(cfg.vocab,))
    for rid, t in enumerate(temps):
        sched2.add_request(rid, rng.integers(0, cfg.vocab, 9).astype(np.uint32), temperature=t, max_new_tokens=5)
    M.Engine(M.QwenPagedModel(shape, w, 128, 16), sched2, cuda_graphs=True).run()
    assert [len(sched2.request_output(r)) for r in range(4)] == [5] * 4
