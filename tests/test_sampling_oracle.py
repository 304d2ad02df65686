"""The sampling oracle (oracle/sampling_ref.py) against the reference's own selfspec_sampling.py outputs
(tests/golden/sampling.json, made by tests/golden/make_golden.py), plus properties of the speculative decision."""
import json
import os

import numpy as np
import pytest
import torch

from oracle import sampling_ref as S


@pytest.fixture(scope="module")
def golden(golden_dir):
    p = os.path.join(golden_dir, "sampling.json")
    if not os.path.exists(p):
        pytest.skip("sampling.json not generated")
    return json.load(open(p))


def _state(c, b, V):
    st = S.PenaltyState(V)
    seen = c["seen"][b]
    st.rep[torch.tensor(seen)] = float(np.float32(c["rep"][b]))
    st.pres[torch.tensor(seen)] = float(np.float32(c["pres"][b]))
    st.freq.scatter_add_(0, torch.tensor(seen), torch.full((len(seen),), float(np.float32(c["freq"][b]))))
    st.len_out = c["len_out"][b]
    return st


def test_penalties_equal_reference_penalize_rows(golden):
    V, bs, K = golden["V"], golden["bs"], golden["K"]
    for c in golden["penalize"]:
        order = [S.NAMES[n] for n in c["order"]]
        logits = S.f32(c["logits"], (bs * K, V))
        ref = S.f32(c["out"], (bs * K, V))
        for b in range(bs):
            st = _state(c, b, V)
            for r in range(K):
                row = S.process_row(logits[b * K + r], st, c["cand"][b][1: r + 1], r, order, c["rep"][b],
                                    c["freq"][b], c["pres"][b], c["min_new"][b], c["stop_ids"][b])
                assert torch.equal(row, ref[b * K + r]), (c["order"], b, r)


def test_cumulation_equals_reference_cumulate_block(golden):
    V, bs = golden["V"], golden["bs"]
    for c in golden["penalize"]:
        a = c["after"]
        rep, freq, pres = (S.f32(a[k], (bs, V)) for k in ("rep", "freq", "pres"))
        for b in range(bs):
            st = _state(c, b, V)
            toks = [t for t, v in zip(c["cum_tok"][b], c["cum_valid"][b]) if v]
            st.cumulate(toks, c["rep"][b], c["freq"][b], c["pres"][b])
            assert torch.equal(st.rep, rep[b]) and torch.equal(st.pres, pres[b]) and torch.equal(st.freq, freq[b])
            assert st.len_out == a["len_out"][b]


def test_filters_equal_reference(golden):
    V = golden["V"]
    for c in golden["filters"]:
        probs = S.f32(c["probs"], (6, V))
        k, p, mp = torch.tensor(c["top_k"]), torch.tensor(c["top_p"]), torch.tensor(c["min_p"])
        assert torch.equal(S.joint_top_k_top_p(probs, k, p), S.f32(c["joint"], (6, V)))
        assert torch.equal(S.torch_filter(probs, k, p, mp, True), S.f32(c["torch"], (6, V)))
        assert torch.equal(S.torch_filter(probs, k, p, mp, False), S.f32(c["torch_no_min_p"], (6, V)))
        assert torch.equal(S.min_p_filter(probs, mp), S.f32(c["min_p_filtered"], (6, V)))


def test_target_distribution_equals_reference(golden):
    V, bs, K = golden["V"], golden["bs"], golden["K"]
    for c in golden["target"]:
        lg = S.f32(c["logits"], (bs * K, V))
        rep = lambda x: torch.tensor(x).repeat_interleave(K)
        fi = S.target_probs(lg, rep(c["temperature"]), rep(c["top_k"]), rep(c["top_p"]), rep(c["min_p"]),
                            S.FILTER_JOINT)
        assert torch.equal(fi, S.f32(c["flashinfer"], (bs * K, V)))
        pt = S.target_probs(lg, rep(c["temperature"]), rep(c["top_k"]), rep(c["top_p"]), rep(c["min_p"]),
                            S.FILTER_TORCH)
        assert torch.equal(pt, S.f32(c["pytorch_min_p"], (bs * K, V)))


def test_philox_known_answers():
    # Random123's published known-answer vectors for philox4x32-10
    assert S.philox4x32_10([0, 0, 0, 0], [0, 0]) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert S.philox4x32_10([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2) == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    assert S.philox4x32_10([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0]) == \
        [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]
    c = [S.coin(12345, 7, b, j, k) for b in range(4) for j in range(5) for k in range(3)]
    assert all(0.0 < x <= 1.0 for x in c) and len(set(c)) == len(c)


def test_speculative_chain_is_exact_in_distribution():
    """Speculative sampling with a point-mass draft commits AR samples: the first verified token follows p_0 whatever
    the draft, and given that d_1 was accepted the next one follows p_1."""
    g = torch.Generator().manual_seed(0)
    V, K, n = 6, 3, 40000
    probs = torch.softmax(torch.randn(K, V, generator=g) * 1.5, dim=-1)
    cand = [0, 2, 4]          # a0, d1, d2
    rng = np.random.default_rng(1)
    first, second = np.zeros(V), np.zeros(V)
    n_acc1 = 0
    for _ in range(n):
        coins = 1.0 - rng.random(K)
        acc, pred = S.speculative_chain(probs, cand, coins, 1.0 - rng.random())
        first[pred[0]] += 1
        if acc >= 1:
            n_acc1 += 1
            second[pred[1]] += 1
    p0 = probs[0].double().numpy()
    assert np.abs(first / n - p0).max() < 4 * np.sqrt(p0.max() / n)
    assert abs(n_acc1 / n - p0[2]) < 4 * np.sqrt(0.25 / n)
    p1 = probs[1].double().numpy()
    assert np.abs(second / n_acc1 - p1).max() < 4 * np.sqrt(p1.max() / n_acc1)
