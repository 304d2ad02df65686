"""Non-greedy verify kernels on a B200 against the sampling oracle (oracle/sampling_ref.py, pinned to the reference's
selfspec_sampling.py), all through the C ABI.

* gr_logits_process: bit-exact against the oracle's row processing (penalizers in either orchestrator order with
  in-block verify ids, min_new_tokens stop mask, grammar mask, logit bias) at the baseline vocabulary.
* gr_penalty_cumulate: the penalizer state equals the oracle's cumulation bit for bit.
* gr_sample_rows: on the same processed logits and the same Philox coins, every accept bit and every draw equals the
  oracle's (float64 target distribution), except listed near-ties: an accept test whose coin is within 1e-5 of
  p_j(d_{j+1}), or a draw whose CDF position is within 1e-5 of the total mass from a token boundary.  Every draw lies
  in the oracle's kept set.  Filters: joint top-k / top-p, sequential (with min-p), "pytorch".
* gr_commit_sampled: acc, verified tokens, packed row and the rng round follow the accept bits exactly.
* The whole chain is exact in distribution: with rows shared by many requests, the first verified token follows p_0.
"""
import math

import numpy as np
import pytest
import torch

from gravityocr_b200 import _lib as L
from gravityocr_b200.sampling import RequestSampling, SamplerState, pack_allowed
from oracle import sampling_ref as S

pytestmark = pytest.mark.gpu
DEV = "cuda"
V = 59392
EPS = 1e-5


def _state_and_params(bs, pool, seed, order, g):
    st = SamplerState(V, pool, DEV, seed=seed, order=order)
    reqs = []
    for b in range(bs):
        reqs.append(RequestSampling(temperature=0.7 + 0.2 * b, top_k=[-1, 50, 4000][b % 3],
                                    top_p=[0.9, 1.0, 0.6][b % 3], min_p=[0.0, 0.05, 0.0][b % 3],
                                    repetition_penalty=1.0 + 0.3 * (b % 2), frequency_penalty=0.2 * (b % 3),
                                    presence_penalty=0.5 * ((b + 1) % 2), min_new_tokens=[0, 40, 3][b % 3],
                                    stop_ids=[7, 11 + b], logit_bias={5: 2.0, 9 + b: -1.5} if b % 2 else None))
    rpi = torch.tensor([(3 * b + 1) % pool for b in range(bs)], dtype=torch.int64)
    # some history in the penalizer state (oracle and device alike)
    ost = {}
    for b in range(bs):
        slot = int(rpi[b])
        toks = torch.randint(0, V, (20,), generator=g).tolist() + [5, 5, 17]
        o = S.PenaltyState(V)
        r = reqs[b]
        o.cumulate(toks, r.repetition_penalty, r.frequency_penalty, r.presence_penalty)
        ost[b] = o
        st.st_rep[slot] = o.rep.to(DEV)
        st.st_freq[slot] = o.freq.to(DEV)
        st.st_pres[slot] = o.pres.to(DEV)
        st.st_len[slot] = o.len_out
    return st, reqs, rpi, ost


@pytest.mark.parametrize("order", [S.NAMES.values(), [S.REP, S.PRES, S.MIN_NEW, S.FREQ]])
def test_logits_process_bit_exact(order):
    g = torch.Generator().manual_seed(3)
    bs, K, pool = 3, 5, 11
    order = list(order)
    st, reqs, rpi, ost = _state_and_params(bs, pool, 1, order, g)
    cand = torch.randint(0, V, (bs, K), generator=g, dtype=torch.int32)
    cand[:, 2] = cand[:, 1]
    cand[0, 3] = 5
    allowed = torch.rand((bs * K, V), generator=g) < 0.97
    allowed[:, 5] = True
    logits = torch.randn((bs * K, V), generator=g) * 4
    smp = st.batch(reqs, rpi.to(DEV), pack_allowed(allowed).to(DEV))
    dev = logits.to(DEV)
    L.logits_process(dev, bs, K, cand.to(DEV), smp)
    torch.cuda.synchronize()
    got = dev.cpu()
    used = [op for op in order if {S.REP: any(r.repetition_penalty != 1 for r in reqs),
                                   S.FREQ: any(r.frequency_penalty != 0 for r in reqs),
                                   S.PRES: any(r.presence_penalty != 0 for r in reqs),
                                   S.MIN_NEW: any(r.min_new_tokens > 0 for r in reqs)}[op]]
    for b in range(bs):
        r = reqs[b]
        bias = None
        if r.logit_bias:
            bias = torch.zeros(V)
            for t, v in r.logit_bias.items():
                bias[t] = v
        for j in range(K):
            ref = S.process_row(logits[b * K + j], ost[b], cand[b, 1: j + 1].tolist(), j, used, r.repetition_penalty,
                                r.frequency_penalty, r.presence_penalty, r.min_new_tokens, list(r.stop_ids),
                                allowed[b * K + j], bias)
            assert torch.equal(got[b * K + j], ref), (b, j)


def test_logits_process_without_grammar_or_bias_bit_exact():
    """No grammar mask and no logit bias: the kernel leaves every entry that no op changes unread and unwritten, and
    rewrites the rest (generated tokens, the block's draft ids, stop ids under min_new_tokens).  Every row equals the
    oracle's, and the untouched entries keep their exact bits (-0.0 and infinities included)."""
    import dataclasses
    g = torch.Generator().manual_seed(8)
    bs, K, pool = 3, 17, 11
    order = list(S.NAMES.values())
    st, reqs, rpi, ost = _state_and_params(bs, pool, 2, order, g)
    reqs = [dataclasses.replace(r, logit_bias=None) for r in reqs]
    cand = torch.randint(0, V, (bs, K), generator=g, dtype=torch.int32)
    cand[:, 4] = cand[:, 2]
    cand[1, 6] = 7   # a stop id drafted inside the block
    logits = torch.randn((bs * K, V), generator=g) * 4
    logits[:, 100:110] = -0.0
    logits[:, 200] = float("inf")
    logits[:, 201] = -float("inf")
    smp = st.batch(reqs, rpi.to(DEV))
    dev = logits.to(DEV)
    L.logits_process(dev, bs, K, cand.to(DEV), smp)
    torch.cuda.synchronize()
    got = dev.cpu()
    used = [op for op in order if {S.REP: any(r.repetition_penalty != 1 for r in reqs),
                                   S.FREQ: any(r.frequency_penalty != 0 for r in reqs),
                                   S.PRES: any(r.presence_penalty != 0 for r in reqs),
                                   S.MIN_NEW: any(r.min_new_tokens > 0 for r in reqs)}[op]]
    changed = 0
    for b in range(bs):
        r = reqs[b]
        for j in range(K):
            ref = S.process_row(logits[b * K + j], ost[b], cand[b, 1: j + 1].tolist(), j, used, r.repetition_penalty,
                                r.frequency_penalty, r.presence_penalty, r.min_new_tokens, list(r.stop_ids), None,
                                None)
            row = got[b * K + j]
            assert torch.equal(row.view(torch.int32), ref.view(torch.int32)), (b, j)
            changed += int((row.view(torch.int32) != logits[b * K + j].view(torch.int32)).sum())
    assert 0 < changed < bs * K * V // 100   # a few entries rewritten, the rest left as they were


def test_penalty_cumulate_bit_exact():
    g = torch.Generator().manual_seed(4)
    bs, K, pool = 3, 6, 8
    order = list(S.NAMES.values())
    st, reqs, rpi, ost = _state_and_params(bs, pool, 1, order, g)
    toks = torch.randint(0, V, (bs, K), generator=g, dtype=torch.int32)
    toks[:, 3] = toks[:, 1]
    counts = torch.tensor([0, 3, K - 1], dtype=torch.int32)
    smp = st.batch(reqs, rpi.to(DEV))
    L.penalty_cumulate(bs, toks.to(DEV), K, counts.to(DEV), 1, smp)
    torch.cuda.synchronize()
    for b in range(bs):
        r = reqs[b]
        ost[b].cumulate(toks[b, : int(counts[b]) + 1].tolist(), r.repetition_penalty, r.frequency_penalty,
                        r.presence_penalty)
        slot = int(rpi[b])
        assert torch.equal(st.st_rep[slot].cpu(), ost[b].rep) and torch.equal(st.st_pres[slot].cpu(), ost[b].pres)
        assert torch.equal(st.st_freq[slot].cpu(), ost[b].freq)
        assert int(st.st_len[slot]) == ost[b].len_out


def _oracle_probs64(lg, T, k, p, mp, mode):
    """float64 target distribution with the kernels' tie rule (ties kept together)."""
    x = lg.double() / T
    probs = torch.softmax(x, -1).view(1, -1)
    kk, pp, mm = torch.tensor([k]), torch.tensor([p], dtype=torch.float64), torch.tensor([mp], dtype=torch.float64)
    if mode == L.FILTER_JOINT:
        return S.joint_top_k_top_p(probs, kk, pp)[0]
    if mode == L.FILTER_SEQUENTIAL:
        return S.sequential_filter(probs, kk, pp, mm)[0]
    s, order = probs.sort(dim=-1, descending=True)
    first = torch.ones_like(s, dtype=torch.bool)
    first[:, 1:] = s[:, 1:] < s[:, :-1]
    pos = torch.arange(probs.shape[1]).expand_as(s)
    n_greater = torch.where(first, pos, torch.zeros_like(pos)).cummax(dim=-1).values
    gsum = (torch.cumsum(s, -1) - s).gather(1, n_greater)
    keep_s = (n_greater < k) & (gsum <= p) & (s >= s[:, :1] * mp)
    keep = torch.zeros_like(keep_s).scatter_(1, order, keep_s)
    return S._renorm(probs, keep)[0]


def _draw_margin(p, u, exclude):
    w = p.clone()
    if exclude >= 0:
        w[exclude] = 0
    c = torch.cumsum(w, 0)
    t = u * float(c[-1])
    return float((c - t).abs().min() / c[-1])


# (6, 5, 3): 30 rows, fewer than the SMs (the launch runs 1,024-thread CTAs); (10, 17, 1): 170 rows (two
# 512-thread CTAs per SM), one round
@pytest.mark.parametrize("bs,K,rounds", [(6, 5, 3), (10, 17, 1)])
@pytest.mark.parametrize("shape", ["peaked", "flat"])
@pytest.mark.parametrize("mode", [L.FILTER_JOINT, L.FILTER_SEQUENTIAL, L.FILTER_TORCH])
def test_sample_rows_match_oracle(mode, shape, bs, K, rounds):
    g = torch.Generator().manual_seed(10 + mode + (100 if shape == "flat" else 0) + bs)
    seed = 1234567
    st = SamplerState(V, bs, DEV, seed=seed, filter=mode)
    reqs = [RequestSampling(temperature=[0.6, 1.0, 1.3, 0.9, 0.0, 1.0][b % 6],
                            top_k=[-1, 40, 1000, 5, -1, -1][b % 6], top_p=[0.9, 1.0, 0.8, 0.95, 1.0, 0.5][b % 6],
                            min_p=0.0 if mode == L.FILTER_JOINT else [0.0, 0.1, 0.02, 0.0, 0.0, 0.3][b % 6])
            for b in range(bs)]   # a flashinfer batch with min-p takes the sequential filter (tested on its own)
    if shape == "peaked":   # a few dominant tokens over a spread-out bulk
        logits = torch.randn((bs * K, V), generator=g) * 2
        logits[:, :20] += torch.randn((bs * K, 20), generator=g) * 3 + 6
    else:   # mean weight above 1/32 of the maximum: the kernel's first select pass aggregates in registers
        logits = torch.randn((bs * K, V), generator=g) * 0.3
    cand = torch.randint(0, 20, (bs, K), generator=g, dtype=torch.int32)
    rpi = torch.arange(bs, dtype=torch.int64)
    smp = st.batch(reqs, rpi.to(DEV))
    assert smp.filter == mode
    ties, mism = [], []
    for rnd in range(rounds):
        dev = logits.to(DEV)
        accept = torch.zeros(bs * K, dtype=torch.int32, device=DEV)
        sample = torch.zeros(bs * K, dtype=torch.int32, device=DEV)
        p_next = torch.zeros(bs * K, dtype=torch.float32, device=DEV)
        status = torch.zeros(1, dtype=torch.int32, device=DEV)
        L.sample_rows(dev, bs, K, cand.to(DEV), smp, L.COIN_FIRST, accept, sample, p_next, status=status)
        torch.cuda.synchronize()
        assert int(status) == 0
        acc_g, smp_g, pn_g = accept.cpu().tolist(), sample.cpu().tolist(), p_next.cpu()
        for b in range(bs):
            T, k = reqs[b].normalised()
            for j in range(K):
                r = b * K + j
                p = _oracle_probs64(logits[r], T, min(k, V), reqs[b].top_p, reqs[b].min_p, mode)
                d = int(cand[b, j + 1]) if j + 1 < K else -1
                uf = S.coin(seed, rnd, b, 0, S.COIN_FINAL)
                assert float(p[smp_g[r]]) > 0, f"draw {smp_g[r]} outside the kept set (row {r})"
                want = S.draw(p, uf, exclude=d)
                if want != smp_g[r]:
                    m = _draw_margin(p, uf, d)
                    (ties if m < EPS else mism).append(("draw", rnd, r, want, smp_g[r], m))
                if d >= 0:
                    ua = S.coin(seed, rnd, b, j, S.COIN_ACCEPT)
                    pd = float(p[d])
                    assert abs(float(pn_g[r]) - pd) <= 1e-4 * max(pd, 1e-6) + 1e-7, (r, float(pn_g[r]), pd)
                    if (ua <= pd) != bool(acc_g[r]):
                        (ties if abs(ua - pd) < EPS else mism).append(("accept", rnd, r, ua, pd))
        st.rng[1] += 1
    assert not mism, mism[:5]
    print(f"filter {mode}: near-ties listed {ties}")


def test_first_token_draws_and_status():
    g = torch.Generator().manual_seed(5)
    bs = 4
    st = SamplerState(V, bs, DEV, seed=99)
    reqs = [RequestSampling(temperature=1.0, top_p=0.9)] * bs
    logits = torch.randn((bs, V), generator=g)
    logits[3] = float("-inf")                       # a row that allows nothing
    smp = st.batch(reqs, torch.arange(bs, dtype=torch.int64, device=DEV))
    out = torch.zeros(bs, dtype=torch.int32, device=DEV)
    am = torch.full((bs * 3,), -5, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    L.sample_rows(logits.to(DEV), bs, 1, None, smp, L.COIN_FIRST, None, out, first_out=am, first_stride=3,
                  status=status)
    torch.cuda.synchronize()
    assert int(status) == L.GR_ERR_NO_TOKEN
    o = out.cpu().tolist()
    assert am.cpu().view(bs, 3)[:, 0].tolist() == o and am.cpu().view(bs, 3)[:, 1:].eq(-5).all()
    for b in range(3):
        p = _oracle_probs64(logits[b], 1.0, V, 0.9, 0.0, L.FILTER_JOINT)
        want = S.draw(p, S.coin(99, 0, b, 0, S.COIN_FIRST))
        assert o[b] == want or _draw_margin(p, S.coin(99, 0, b, 0, S.COIN_FIRST), -1) < EPS


def test_commit_sampled_chain():
    bs, K = 4, 5
    am = torch.tensor([[10, 11, 12, 13, 14], [20, 21, 22, 23, 24], [30, 31, 32, 33, 34], [40, 41, 42, 43, 44]],
                      dtype=torch.int32)
    accept = torch.tensor([[1, 1, 0, 1, 0], [0, 1, 1, 1, 0], [1, 1, 1, 1, 0], [1, 0, 0, 0, 0]], dtype=torch.int32)
    sample = torch.arange(bs * K, dtype=torch.int32).view(bs, K) + 100
    d = lambda t: t.contiguous().view(-1).to(DEV)
    seeds = torch.zeros(8, dtype=torch.int64, device=DEV)
    rpi = torch.tensor([5, 0, 2, 7], dtype=torch.int64, device=DEV)
    seq = torch.tensor([100, 200, 300, 400], dtype=torch.int64, device=DEV)
    predict = torch.zeros(bs * K, dtype=torch.int32, device=DEV)
    packed = torch.zeros((bs, K + 2), dtype=torch.int32, device=DEV)
    released = torch.zeros(bs * K, dtype=torch.int64, device=DEV)
    n_rel = torch.zeros(1, dtype=torch.int32, device=DEV)
    out_next = torch.zeros(bs, dtype=torch.int64, device=DEV)
    acc_len = torch.zeros(bs, dtype=torch.int32, device=DEV)
    rng = torch.tensor([7, 41], dtype=torch.int64, device=DEV)
    L.commit_sampled(bs, K, d(am), d(accept), d(sample), seeds, rpi, seq, predict, packed, released, out_next,
                     n_released=n_rel, accept_len=acc_len, rng=rng)
    torch.cuda.synchronize()
    accs = [2, 0, 4, 1]
    assert acc_len.cpu().tolist() == accs
    pv = predict.cpu().view(bs, K).tolist()
    for b, a in enumerate(accs):
        ver = am[b, 1: a + 1].tolist() + [int(sample[b, a])]
        assert pv[b][: a + 1] == ver and not any(pv[b][a + 1:])
        assert packed.cpu()[b].tolist() == [int(am[b, 0]), a] + ver + [0] * (K - 1 - a)
        assert int(seeds[rpi[b]]) == ver[-1] == int(out_next[b])
        assert int(seq[b]) == [100, 200, 300, 400][b] + a + 2
    assert int(n_rel) == sum(K - 1 - a for a in accs)
    assert rng.cpu().tolist() == [7, 42]


def test_speculative_chain_exact_in_distribution():
    """4096 requests share the same three rows (different coins): the first verified token follows p_0 and, given d1
    accepted, the second follows p_1 -- whatever the drafts."""
    g = torch.Generator().manual_seed(8)
    bs, K, Vs = 4096, 3, 64
    st = SamplerState(Vs, bs, DEV, seed=2024)
    reqs = [RequestSampling(temperature=1.0)] * bs
    base = torch.randn((K, Vs), generator=g) * 1.5
    logits = base.repeat(bs, 1).to(DEV)
    cand = torch.tensor([0, 2, 4], dtype=torch.int32).repeat(bs, 1).to(DEV)
    smp = st.batch(reqs, torch.arange(bs, dtype=torch.int64, device=DEV))
    accept = torch.zeros(bs * K, dtype=torch.int32, device=DEV)
    sample = torch.zeros(bs * K, dtype=torch.int32, device=DEV)
    L.sample_rows(logits, bs, K, cand, smp, L.COIN_FIRST, accept, sample)
    torch.cuda.synchronize()
    a = accept.cpu().view(bs, K)
    s = sample.cpu().view(bs, K)
    first = torch.where(a[:, 0] == 1, torch.full((bs,), 2), s[:, 0])
    p0 = torch.softmax(base[0].double(), -1)
    emp = torch.bincount(first, minlength=Vs).double() / bs
    assert float((emp - p0).abs().max()) < 4 * math.sqrt(float(p0.max()) / bs)
    sel = a[:, 0] == 1
    second = torch.where(a[sel, 1] == 1, torch.full((int(sel.sum()),), 4), s[sel, 1])
    p1 = torch.softmax(base[1].double(), -1)
    emp1 = torch.bincount(second, minlength=Vs).double() / int(sel.sum())
    assert float((emp1 - p1).abs().max()) < 4 * math.sqrt(float(p1.max()) / int(sel.sum())) + 1e-3
