"""Host commit rules of the package (gravityocr_b200.commit_rules) against the reference's own rules module
(golden vectors from tests/golden/make_golden.py) and the SGLang-shaped request objects of gravityocr_b200.compat."""
import json
import os

import pytest

from gravityocr_b200 import commit_rules as R
from gravityocr_b200.compat.types import Req, SamplingParams


def _load(golden_dir, name):
    p = os.path.join(golden_dir, name)
    if not os.path.exists(p):
        pytest.skip(f"{name} not generated")
    return json.load(open(p))


def test_cut_index_golden(golden_dir):
    for c in _load(golden_dir, "commit_rules.json")["cut_index"]:
        assert R.cut_index(c["T"], c["budget"], frozenset(c["stop"]), c["vocab"]) == c["j"]


class _SP:
    def __init__(self, mx):
        self.max_new_tokens = mx
        self.ignore_eos = False
        self.stop_token_ids = [7]
        self.stop_strs = None
        self.stop_regex_strs = None


class _Req:
    def __init__(self, mx, prev):
        self.sampling_params = _SP(mx)
        self.eos_token_ids = {11}
        self.tokenizer = None
        self.grammar = None
        self.to_finish = None
        self.vocab_size = 59392
        self.output_ids = [1] * prev
        self.spec_verify_ct = 0
        self.spec_accepted_tokens = 0

    def finished(self):
        return False

    def check_finished(self, n=1):
        pass

    def update_spec_acceptance_histogram(self, a):
        pass


def test_host_commit_golden(golden_dir):
    for c in _load(golden_dir, "commit_rules.json")["host_commit"]:
        reqs = []
        for r, b in zip(c["rows"], c["budgets"]):
            prev = 10
            reqs.append(_Req(prev + b, prev))
        toks, js, accs = R.host_commit(reqs, c["rows"])
        assert (toks, js, accs) == (c["toks"], c["js"], c["accs"])
        assert [q.spec_accepted_tokens for q in reqs] == c["accepted_counters"]


def test_req_finish_order_and_cut():
    import torch
    V = 100
    r = Req("a", torch.zeros((2, 4)), [5, 6], SamplingParams(max_new_tokens=4, stop_token_ids=[9]), V)
    r.output_ids = [1]
    j = R.commit_fast(r, [3, 9, 4])           # stop id at index 1
    assert j == 1 and r.output_ids == [1, 3, 9] and r.finished_reason.kind == "stop"
    r2 = Req("b", torch.zeros((2, 4)), [5], SamplingParams(max_new_tokens=3), V)
    r2.output_ids = [1]
    j = R.commit_fast(r2, [3, 4, 5, 6])       # budget 2
    assert j == 1 and r2.output_ids == [1, 3, 4] and r2.finished_reason.kind == "length"
    r3 = Req("c", torch.zeros((2, 4)), [5], SamplingParams(max_new_tokens=50), V)
    assert R.cannot_finish(r3, [1, 2, 3]) and not R.cannot_finish(r3, [1, V + 1])
