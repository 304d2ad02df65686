"""Draft-ahead in the served worker (the reference's SELFSPEC_DRAFT_AHEAD=1, selfspec_diffusion_worker.py:1000-1125,
selfspec_fast_commit.py:357-440) on a B200: with it on, every request commits exactly the tokens it commits with it off,
under the same schedule -- including rounds where a request finishes (no draft is launched ahead then), a stash
released by the scheduler hook, and a batch that changes after a draft was launched ahead (the stash is dropped)."""
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


def _schedule(ahead: bool, w, cfg):
    eng = Engine(cfg, w, max_rows=8 * 64, n_pages=8 * 64 + 8)
    target = types.SimpleNamespace(engine=eng, req_to_page=ReqToPagePool(eng, size=8, max_context=1024))
    os.environ["SELFSPEC_MASK_ID"] = str(cfg.mask_id)
    wk = SelfSpecDiffusionWorker(types.SimpleNamespace(speculative_num_draft_tokens=17, page_size=16, model_path="",
                                                       ss_draft_ahead=ahead), 0, 0, None, 0, 0, 0, 0, target)
    budgets = [1 << 20, 9, 1 << 20]
    reqs = []
    for i, mx in enumerate(budgets):
        img, txt = request_inputs(cfg, 5, 48, 12, i, torch.bfloat16)
        reqs.append(Req(i, img, txt.tolist(), SamplingParams(max_new_tokens=mx), cfg.vocab))
    slots = [0, 3, 5]
    wk.forward_batch_generation(ScheduleBatch(reqs, torch.tensor(slots, device=DEV),
                                              torch.zeros(3, dtype=torch.int64, device=DEV), ForwardMode.EXTEND))
    seq = {s: len(r.origin_input_ids) for r, s in zip(reqs, slots)}

    def batch_of(rr, ss):
        return ScheduleBatch(rr, torch.tensor(ss, device=DEV), torch.tensor([seq[s] for s in ss], device=DEV),
                             ForwardMode.DECODE, torch.tensor([seq[s] for s in ss]))

    live = list(zip(reqs, slots))
    b = batch_of([x[0] for x in live], [x[1] for x in live])
    for rnd in range(14):
        if rnd == 8:
            wk.ss_release_stash("test: scheduler hook")
        res = wk.forward_batch_generation(b)
        for i, s in enumerate([x[1] for x in live]):
            seq[s] += res.accept_length_per_req_cpu[i] + 1
        if any(r.finished() for r, _ in live) or rnd == 10:
            # the batch changes: finished requests leave; at round 10 the last request also leaves
            live = [(r, s) for r, s in live if not r.finished()]
            if rnd == 10:
                live = live[:-1]
            b = batch_of([x[0] for x in live], [x[1] for x in live])
    return [r.output_ids for r in reqs], wk.ahead_stats


def test_draft_ahead_commits_the_same_tokens():
    cfg = small_model(2)
    w = random_weights(cfg, 7, torch.bfloat16, embed_std=0.25)
    off, _ = _schedule(False, w, cfg)
    on, stats = _schedule(True, w, cfg)
    assert on == off
    assert len(on[1]) == 9
    assert stats["launched"] >= 8 and stats["used"] >= 6, stats
    assert stats["skip_finish"] >= 1 and stats["released"] >= 2, stats
