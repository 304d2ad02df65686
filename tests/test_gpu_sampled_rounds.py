"""Non-greedy batches through the served worker (``SelfSpecDiffusionWorker.forward_batch_generation``) on a B200.

* A greedy request keeps exactly its greedy stream when its batch takes the sampled path (same batch shape): with
  top_k = 1 the target distribution is the argmax, so the accept test and the draws reduce to the greedy verify.
* A stateful grammar (each token must flip the parity of the previous one) holds on every committed token: the verify
  rows' masks follow the chain a0, d1..dj, and committed tokens advance the grammar.
* A large presence penalty forbids repeats inside one round too (the in-block verify ids are penalised row by row).
* min_new_tokens keeps a strongly favoured stop id out until the output is long enough, then it ends the request.
* Same seed, same tokens; another seed, other tokens.
"""
import os
import types

import pytest
import torch

from gravityocr_b200.compat.sglang_worker import ReqToPagePool, SelfSpecDiffusionWorker
from gravityocr_b200.compat.types import ForwardMode, Req, SamplingParams, ScheduleBatch
from gravityocr_b200.config import small_model
from gravityocr_b200.engine import Engine
from gravityocr_b200.weights import random_weights, request_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def model():
    cfg = small_model(2)
    return cfg, random_weights(cfg, 7, torch.bfloat16, embed_std=0.25)


def _worker(cfg, w, seed=0, pool=8, K=17):
    eng = Engine(cfg, w, max_rows=max(pool * K, 4 * 64), n_pages=pool * 64 + 8)
    target = types.SimpleNamespace(engine=eng, req_to_page=ReqToPagePool(eng, size=pool, max_context=1024))
    args = types.SimpleNamespace(speculative_num_draft_tokens=K, page_size=16, model_path="", random_seed=seed)
    os.environ["SELFSPEC_MASK_ID"] = str(cfg.mask_id)
    return SelfSpecDiffusionWorker(args, 0, 0, None, 0, 0, 0, 0, target)


def _req(cfg, i, sp, eos=None):
    img, txt = request_inputs(cfg, 5, 48, 12, i, torch.bfloat16)
    return Req(i, img, txt.tolist(), sp, cfg.vocab, eos_token_ids=eos)


def _run(wk, reqs, slots, rounds):
    wk.forward_batch_generation(ScheduleBatch(reqs, torch.tensor(slots, device=DEV),
                                              torch.zeros(len(reqs), dtype=torch.int64, device=DEV),
                                              ForwardMode.EXTEND))
    seq = {s: len(r.origin_input_ids) for r, s in zip(reqs, slots)}
    live = [(r, s) for r, s in zip(reqs, slots) if not r.finished()]
    for _ in range(rounds):
        if not live:
            break
        rr, ss = [x[0] for x in live], [x[1] for x in live]
        b = ScheduleBatch(rr, torch.tensor(ss, device=DEV), torch.tensor([seq[s] for s in ss], device=DEV),
                          ForwardMode.DECODE, torch.tensor([seq[s] for s in ss]))
        res = wk.forward_batch_generation(b)
        for i, s in enumerate(ss):
            seq[s] += res.accept_length_per_req_cpu[i] + 1
        live = [(r, s) for r, s in live if not r.finished()]


def test_greedy_request_unchanged_in_a_sampled_batch(model):
    cfg, w = model
    a = [_req(cfg, 0, SamplingParams(max_new_tokens=1 << 20)), _req(cfg, 1, SamplingParams(max_new_tokens=1 << 20))]
    _run(_worker(cfg, w), a, [0, 1], 5)
    b = [_req(cfg, 0, SamplingParams(max_new_tokens=1 << 20)),
         _req(cfg, 1, SamplingParams(max_new_tokens=1 << 20, temperature=0.9, top_p=0.95))]
    _run(_worker(cfg, w), b, [0, 1], 5)
    n = min(len(a[0].output_ids), len(b[0].output_ids))
    assert n >= 10 and a[0].output_ids[:n] == b[0].output_ids[:n]
    assert b[1].output_ids != a[1].output_ids[: len(b[1].output_ids)]   # the sampled one really sampled


class _ParityGrammar:
    """Each token must have the other parity than the previous one (the first token is free)."""

    def __init__(self, vocab):
        self.vocab, self.hist, self.finished = vocab, [], False
        self.ids = torch.arange(vocab)

    def allowed_tokens(self):
        if not self.hist:
            return torch.ones(self.vocab, dtype=torch.bool)
        return (self.ids % 2) != (self.hist[-1] % 2)

    def accept_token(self, t):
        if self.hist and t % 2 == self.hist[-1] % 2:
            raise ValueError(f"token {t} breaks the parity chain")
        self.hist.append(int(t))

    def rollback(self, n):
        del self.hist[len(self.hist) - n:]

    def is_terminated(self):
        return False


def test_grammar_masks_follow_the_draft_chain(model):
    cfg, w = model
    reqs = [_req(cfg, i, SamplingParams(max_new_tokens=1 << 20, temperature=t)) for i, t in enumerate((0.0, 1.0))]
    for r in reqs:
        r.grammar = _ParityGrammar(cfg.vocab)
    _run(_worker(cfg, w), reqs, [2, 3], 6)
    for r in reqs:
        out = r.output_ids
        assert len(out) >= 10
        # the prefill's token is the first the grammar sees; every later one flips parity
        assert all(out[i] % 2 != out[i - 1] % 2 for i in range(1, len(out))), out
        assert r.grammar.hist == out


def test_presence_penalty_forbids_repeats_within_rounds(model):
    cfg, w = model
    sp = SamplingParams(max_new_tokens=1 << 20, temperature=0.7, presence_penalty=1e4)
    reqs = [_req(cfg, 4, sp)]
    # a strong logit bias on two tokens makes repeats likely without the penalty
    sp.logit_bias = {101: 15.0, 202: 15.0}
    _run(_worker(cfg, w), reqs, [1], 6)
    out = reqs[0].output_ids
    assert len(out) >= 10 and len(set(out)) == len(out), out
    assert 101 in out and 202 in out


def test_min_new_tokens_holds_back_a_favoured_stop_id(model):
    cfg, w = model
    eos = 4242
    sp = SamplingParams(max_new_tokens=64, temperature=1.0, min_new_tokens=6, logit_bias={eos: 40.0})
    r = _req(cfg, 6, sp, eos=[eos])
    _run(_worker(cfg, w), [r], [0], 20)
    assert r.finished_reason.kind == "stop"
    assert len(r.output_ids) == 7 and r.output_ids[-1] == eos and eos not in r.output_ids[:6]


def test_same_seed_same_tokens(model):
    cfg, w = model
    outs = []
    for seed in (11, 11, 12):
        reqs = [_req(cfg, i, SamplingParams(max_new_tokens=1 << 20, temperature=1.0, top_k=50, top_p=0.9,
                                            repetition_penalty=1.3, frequency_penalty=0.2)) for i in range(2)]
        _run(_worker(cfg, w, seed=seed), reqs, [0, 1], 4)
        outs.append([r.output_ids for r in reqs])
    assert outs[0] == outs[1]
    assert outs[0] != outs[2]
