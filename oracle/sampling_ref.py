"""CPU oracle for non-greedy verify (sampling, penalties, grammar mask, logit bias).  TEST INFRASTRUCTURE ONLY.

Restates, in torch on the CPU:
  * the logits processing AR decode gives every row (``patches/sglang/python/sglang/srt/speculative/
    selfspec_sampling.py``: ``penalize_rows`` :120-170 with SGLang's four penalizers in the orchestrator's order --
    repetition ``where(l < 0, l * S, l / S)``, presence and frequency subtraction, min_new_tokens masking the stop ids
    while the output is shorter than min_new_tokens; then the grammar vocab mask, then logit_bias, ``:150-195`` of
    ``selfspec_fast_commit.py``).  Row j of a request also sees the in-block verify ids cand[1..j];
  * the penalizer cumulation of committed tokens (``cumulate_block`` :60-100);
  * AR's target distribution (``verify_target_probs`` :245-275): softmax(logits / T), then the flashinfer backend's
    joint top-k / top-p (``joint_top_k_top_p`` :205-222: keep q iff #{p > p_q} < k and sum{p > p_q} < top_p), or its
    sequential top-k renorm -> top-p renorm -> min-p when min-p is in use, or the "pytorch" backend
    (``torch_backend_filter`` :232-243);
  * the speculative decision of ``tree_speculative_sampling_target_only`` (sgl_kernel 0.4.1, not vendored; its use is
    ``selfspec_fast_commit.py:197-230``) for a linear chain with thresholds 1.0: walking j = 0, 1, ...: d_{j+1} is
    accepted iff coin_j <= p_j(d_{j+1}); at the first rejection the token is drawn from p_j with d_{j+1} removed and
    renormalised; when every draft is accepted the bonus is drawn from the last row.  Draws invert the CDF of the
    (unnormalised) kept mass in vocabulary order at u * total;
  * the coins: Philox-4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC'11),
    keyed by the round's seed, counter = (round, request, row | kind << 24, 0); a coin is ((x0 >> 8) + 1) * 2^-24,
    uniform in (0, 1] as ``acceptance_coins`` (:280-284) asks.

``tests/golden/sampling.json`` holds the reference module's own outputs on seeded inputs; ``tests/test_sampling_oracle.py``
checks this file against them.
"""
from __future__ import annotations

import base64
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

REP, FREQ, PRES, MIN_NEW = 0, 1, 2, 3
NAMES = {"BatchedRepetitionPenalizer": REP, "BatchedFrequencyPenalizer": FREQ, "BatchedPresencePenalizer": PRES,
         "BatchedMinNewTokensPenalizer": MIN_NEW}
FILTER_JOINT, FILTER_SEQUENTIAL, FILTER_TORCH = 0, 1, 2
COIN_ACCEPT, COIN_FINAL, COIN_FIRST = 0, 1, 2


def f32(b64: str, shape) -> torch.Tensor:
    return torch.from_numpy(np.frombuffer(base64.b64decode(b64), dtype="<f4").copy()).view(*shape)


# ---------------------------------------------------------------------- coins
_M0, _M1, _W0, _W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85


def philox4x32_10(ctr: Sequence[int], key: Sequence[int]) -> List[int]:
    c0, c1, c2, c3 = (int(x) & 0xFFFFFFFF for x in ctr)
    k0, k1 = (int(x) & 0xFFFFFFFF for x in key)
    for _ in range(10):
        p0 = _M0 * c0
        p1 = _M1 * c2
        hi0, lo0 = p0 >> 32, p0 & 0xFFFFFFFF
        hi1, lo1 = p1 >> 32, p1 & 0xFFFFFFFF
        c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
        k0 = (k0 + _W0) & 0xFFFFFFFF
        k1 = (k1 + _W1) & 0xFFFFFFFF
    return [c0, c1, c2, c3]


def coin(seed: int, rnd: int, b: int, j: int, kind: int) -> float:
    """Uniform in (0, 1], a float32 value exactly."""
    x = philox4x32_10((rnd, b, (j & 0xFFFFFF) | (kind << 24), 0), (seed & 0xFFFFFFFF, seed >> 32))[0]
    return float(np.float32(((x >> 8) + 1) * (2.0 ** -24)))


# ---------------------------------------------------------------------- logits processing
class PenaltyState:
    """One request slot's penalizer state, as SGLang's penalizers hold it: repetition (1 where unseen, the penalty where
    seen), frequency (the penalty added once per occurrence), presence (the penalty where seen), output length."""

    def __init__(self, vocab: int):
        self.rep = torch.ones(vocab)
        self.freq = torch.zeros(vocab)
        self.pres = torch.zeros(vocab)
        self.len_out = 0

    def cumulate(self, tokens: Sequence[int], rep_p: float, freq_p: float, pres_p: float) -> None:
        for t in tokens:
            self.rep[t] = rep_p
            self.pres[t] = pres_p
            self.freq[t] += np.float32(freq_p)
        self.len_out += len(tokens)


def process_row(logits: torch.Tensor, st: PenaltyState, in_block: Sequence[int], j: int, order: Sequence[int],
                rep_p: float, freq_p: float, pres_p: float, min_new: int, stop_ids: Sequence[int],
                allowed: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One row (float32, returned as a new tensor): penalizers in `order` (only the active ones), grammar mask, bias.
    in_block = cand[1..j] (the verify ids between the committed tokens and this row)."""
    l = logits.clone().float()
    rep_p, freq_p, pres_p = (float(np.float32(x)) for x in (rep_p, freq_p, pres_p))
    for op in order:
        if op == REP and rep_p != 1.0:
            S = st.rep.clone()
            for t in in_block:
                S[t] = rep_p
            l = torch.where(l < 0, l * S, l / S)
        elif op == PRES and pres_p != 0.0:
            S = st.pres.clone()
            for t in in_block:
                S[t] = pres_p
            l = l - S
        elif op == FREQ and freq_p != 0.0:
            S = st.freq.clone()
            for t in in_block:
                S[t] += np.float32(freq_p)
            l = l - S
        elif op == MIN_NEW and st.len_out + j < min_new:
            for t in stop_ids:
                l[t] = float("-inf")
    if allowed is not None:
        l = torch.where(allowed, l, torch.full_like(l, float("-inf")))
    if bias is not None:
        l = l + bias.float()
    return l


# ---------------------------------------------------------------------- target distributions
def _renorm(p, keep):
    out = torch.where(keep, p, torch.zeros_like(p))
    return out / out.sum(-1, keepdim=True)


def joint_top_k_top_p(probs: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor) -> torch.Tensor:
    """keep q iff #{v : p_v > p_q} < k and (sum{p_v > p_q} < top_p or top_p >= 1); renormalised."""
    s, order = probs.sort(dim=-1, descending=True)
    V = probs.shape[-1]
    pos = torch.arange(V).expand_as(s)
    first = torch.ones_like(s, dtype=torch.bool)
    first[:, 1:] = s[:, 1:] < s[:, :-1]
    n_greater = torch.where(first, pos, torch.zeros_like(pos)).cummax(dim=-1).values
    excl = torch.cumsum(s, dim=-1) - s
    greater_sum = excl.gather(1, n_greater)
    keep_s = (n_greater < top_k.view(-1, 1).to(n_greater.dtype)) & ((greater_sum < top_p.view(-1, 1)) |
                                                                    (top_p.view(-1, 1) >= 1.0))
    keep = torch.zeros_like(keep_s).scatter_(1, order, keep_s)
    return _renorm(probs, keep)


def min_p_filter(probs: torch.Tensor, min_p: torch.Tensor) -> torch.Tensor:
    keep = probs >= probs.max(dim=-1, keepdim=True).values * min_p.view(-1, 1)
    return _renorm(probs, keep)


def torch_filter(probs, top_k, top_p, min_p, need_min_p: bool) -> torch.Tensor:
    """The "pytorch" backend: sorted order, position < k, exclusive cumsum <= top_p, p >= p_max * min_p."""
    s, order = probs.sort(dim=-1, descending=True)
    csum = torch.cumsum(s, dim=-1)
    V = probs.shape[-1]
    keep_s = torch.arange(V).view(1, -1) < top_k.view(-1, 1)
    keep_s &= ~((csum - s) > top_p.view(-1, 1))
    if need_min_p:
        keep_s &= ~(s < (s[:, 0] * min_p).view(-1, 1))
    keep = torch.zeros_like(keep_s).scatter_(1, order, keep_s)
    return _renorm(probs, keep)


def sequential_filter(probs, top_k, top_p, min_p) -> torch.Tensor:
    """flashinfer with min-p: top-k renorm, then top-p renorm on that, then min-p (ties kept together, as the joint
    rule keeps them)."""
    inf = torch.full_like(top_p, 2.0)
    p = joint_top_k_top_p(probs, top_k, inf)
    p = joint_top_k_top_p(p, torch.full_like(top_k, 1 << 30), top_p)
    return min_p_filter(p, min_p)


def target_probs(logits: torch.Tensor, temperature, top_k, top_p, min_p, mode: int) -> torch.Tensor:
    """AR's sampling distribution of each row (logits [R, V] processed; per-row parameters)."""
    T = torch.as_tensor(temperature, dtype=torch.float32).view(-1, 1)
    probs = torch.softmax(logits.float() / T, dim=-1)
    k = torch.as_tensor(top_k, dtype=torch.int64).view(-1)
    p = torch.as_tensor(top_p, dtype=torch.float32).view(-1)
    mp = torch.as_tensor(min_p, dtype=torch.float32).view(-1)
    if mode == FILTER_JOINT:
        return joint_top_k_top_p(probs, k, p)
    if mode == FILTER_SEQUENTIAL:
        return sequential_filter(probs, k, p, mp)
    return torch_filter(probs, k, p, mp, True)


# ---------------------------------------------------------------------- draws and the speculative decision
def draw(p: torch.Tensor, u: float, exclude: int = -1) -> int:
    """Inverse CDF in vocabulary order over p (excluding `exclude`) at u * total: the first index whose inclusive
    cumulative mass exceeds it (the last index with mass when rounding leaves none)."""
    w = p.double().clone()
    if exclude >= 0:
        w[exclude] = 0.0
    c = torch.cumsum(w, 0)
    tot = float(c[-1])
    if tot <= 0:
        return int(torch.argmax(p))
    idx = int(torch.searchsorted(c, torch.tensor([u * tot], dtype=torch.float64), right=True)[0])
    if idx >= w.shape[0]:
        idx = int(torch.nonzero(w > 0)[-1])
    return idx


def speculative_chain(probs: torch.Tensor, cand: Sequence[int], coins: Sequence[float], final_coin: float):
    """probs [K, V] = p_0..p_{K-1} (row j predicts the token after cand[j]); cand = [a0, d1..d_{K-1}].
    Returns (acc, predict [acc + 1]): predict[j] = d_{j+1} for j < acc, predict[acc] = the draw."""
    K = probs.shape[0]
    for j in range(K - 1):
        d = int(cand[j + 1])
        if not coins[j] <= float(probs[j, d]):
            return j, [int(t) for t in cand[1: j + 1]] + [draw(probs[j], final_coin, exclude=d)]
    return K - 1, [int(t) for t in cand[1:K]] + [draw(probs[K - 1], final_coin)]
