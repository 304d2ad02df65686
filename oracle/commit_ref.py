"""CPU oracle for the accept-and-commit step.  TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates, in numpy / plain Python:
  * ``chain_accept``: the linear-chain greedy verify (sgl_kernel 0.4.1 ``verify_tree_greedy`` as the worker drives it
    through ``_chain_retrieve``, ``selfspec_diffusion_worker.py:530-548``; its linear-chain result is pinned by
    ``selfspec_fast_commit.py:443-452``: accepted indices i*K + 0..acc) -- equivalently the natcache accept
    ``src/fast_sampling.py:577-584``: acc = number of leading draft tokens d_j (j >= 1) equal to the verify argmax of
    the row before them.
  * ``ss_commit``: the Triton ``_ss_commit_kernel`` (``patches/sglang/python/sglang/srt/speculative/
    selfspec_fast_commit.py:108-147``): packed row (a0, acc, predict row zeroed past acc), seed pool write,
    seq_lens += acc + 1, rejected verify slots compacted in row order.
  * the dependency-free host rules of ``selfspec_commit_rules.py:94-170`` (``cut_index``, ``commit_fast``,
    ``host_commit`` for requests with no grammar / stop strings).

The golden vectors in ``tests/golden/commit_kernel.json`` come from the reference kernel itself run under the Triton
CPU interpreter, and ``tests/golden/commit_rules.json`` from the reference rules module; ``tests/test_oracle_golden.py``
checks this file against both.
"""
from __future__ import annotations

from typing import Dict, List, Sequence, Tuple

import numpy as np


def chain_accept(draft: Sequence[int], verify_argmax: Sequence[int]) -> int:
    """draft = [a0, d1..d_{K-1}] (the verify input row), verify_argmax[t] = argmax of verify row t.
    Returns acc in [0, K-1]: d_j accepted for j = 1..acc."""
    K = len(draft)
    acc = 0
    while acc + 1 < K and int(draft[acc + 1]) == int(verify_argmax[acc]):
        acc += 1
    return acc


def batch_accept(draft: np.ndarray, verify_argmax: np.ndarray) -> np.ndarray:
    """[bs, K] x [bs, K] -> acc [bs] int32."""
    return np.array([chain_accept(d, v) for d, v in zip(draft.tolist(), verify_argmax.tolist())], dtype=np.int32)


def ss_commit(predict: np.ndarray, acc: np.ndarray, a0: np.ndarray, rpi: np.ndarray, seeds: np.ndarray,
              seq_lens: np.ndarray, loc: np.ndarray, K: int) -> Dict[str, np.ndarray]:
    """Numpy restatement of ``_ss_commit_kernel`` for bs = len(acc) rows.

    predict [bs*K (+1)] int32 verify predicts (row i: i*K + 0..acc valid); acc [bs] int32; a0 [bs] int64;
    rpi [bs] int64 req pool indices; seeds [pool] int64 (updated copy returned); seq_lens [bs] int64 (updated copy
    returned); loc [bs*K] int64 verify slots.  Returns packed [bs, K+2] int32, seeds, seq_lens, free (the compacted
    rejected slots, length sum(K-1-acc)), out [bs] int64 next seeds."""
    bs = int(acc.shape[0])
    seeds = seeds.copy()
    seq_lens = seq_lens.copy()
    packed = np.zeros((bs, K + 2), dtype=np.int32)
    out = np.zeros((bs,), dtype=np.int64)
    free: List[int] = []
    for i in range(bs):
        a = int(acc[i])
        row = predict[i * K: i * K + K].astype(np.int64)
        packed[i, 0] = np.int32(np.int64(a0[i]).astype(np.int32))
        packed[i, 1] = a
        packed[i, 2: 2 + a + 1] = row[: a + 1].astype(np.int32)
        seed = int(predict[i * K + a])
        seeds[int(rpi[i])] = seed
        out[i] = seed
        seq_lens[i] += a + 1
        free += [int(loc[i * K + j]) for j in range(a + 1, K)]
    return {"packed": packed, "seeds": seeds, "seq_lens": seq_lens, "free": np.array(free, dtype=np.int64), "out": out}


# ---------------------------------------------------------------------- host rules (selfspec_commit_rules.py)
def cut_index(T: Sequence[int], budget: int, stop: frozenset, vocab: int) -> int:
    """selfspec_commit_rules.py:94-103: index of the last token the per-token loop appends,
    min(budget - 1, first stop id, first out-of-vocab id, len(T) - 1)."""
    lim = len(T) - 1
    if budget - 1 < lim:
        lim = budget - 1 if budget > 0 else 0
    for t in range(lim):
        x = T[t]
        if x in stop or x > vocab or x < 0:
            return t
    return lim


def commit_rows(rows: Sequence[Sequence[int]], budgets: Sequence[int], stop: frozenset, vocab: int
                ) -> Tuple[List[List[int]], List[int], List[int]]:
    """host_commit for fast requests (selfspec_commit_rules.py:121-126,150-170) over packed rows (a0, acc, predict..):
    T = [a0] + predict[0..acc]; j = cut_index(T, budget, stop, vocab); tokens T[:j+1].  Returns (tokens, js, accs)."""
    toks, js, accs = [], [], []
    for r, b in zip(rows, budgets):
        a = int(r[1])
        T = [int(r[0])] + [int(x) for x in r[2: 3 + a]]
        j = cut_index(T, b, stop, vocab)
        toks.append(T[: j + 1])
        js.append(j)
        accs.append(a)
    return toks, js, accs


def released_positions(seq_len_before: int, acc: int, K: int) -> List[int]:
    """Logical KV positions the round rolls back: the verify window occupies S+1..S+K; positions S+acc+2..S+K are not
    kept (the page-1 reference frees the same verify slots acc+1..K-1)."""
    return list(range(seq_len_before + acc + 2, seq_len_before + K + 1))
