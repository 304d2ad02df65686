"""The persistent small-batch forward (one cooperative kernel per forward, gr_small_*) against the per-launch
forward: the same device code on the same parameters, so every output must be bit-identical (argmaxes, top-1 logits,
top-2 gaps, the K/V rows written, the commit bookkeeping), eagerly and from CUDA graphs."""
import math

import pytest
import torch

from gravityocr_b200.config import small_model
from gravityocr_b200.engine import Engine
from gravityocr_b200.weights import prefix_embeddings, random_weights, request_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"
K = 17


def _setup(bs, n_layers=2, n_image=96, n_prompt=16, seed=4):
    cfg = small_model(n_layers)
    w = random_weights(cfg, seed, torch.bfloat16)
    w32 = {k: v.float() for k, v in w.items()}
    reqs = []
    for b in range(bs):
        img, txt = request_inputs(cfg, seed, n_image + 40 * b, n_prompt, b, torch.bfloat16)
        x = prefix_embeddings(w32, cfg, img, txt)
        ids = torch.cat([torch.full((n_image + 40 * b,), -1, dtype=torch.int64), txt])
        reqs.append((x, ids))
    cap = n_image + 40 * bs + n_prompt + 8 * (K + 1) + 64
    ppr = (cap + 15) // 16
    eng = Engine(cfg, w, max_rows=max(64 * bs, bs * K), n_pages=bs * ppr + 4)
    eng.reserve(bs * K)
    rb = eng.new_round_buffers(bs, K, ppr, max_len=cap, avg_len=cap // 2)
    rb.attn_chunk, rb.attn_splits = 64, int(math.ceil((cap + K + 1) / 64))  # several splits: the merge runs too
    for b in range(bs):
        rb.page_table[b] = torch.tensor(eng.pool.alloc(ppr), dtype=torch.int32, device=DEV)
    eng.prefill(rb, [x for x, _ in reqs], [i for _, i in reqs])
    return eng, rb


def _state(rb):
    return [t.clone() for t in (rb.seq_lens, rb.seeds, rb.n_committed, rb.rounds)]


def _restore(rb, snap):
    for t, s in zip((rb.seq_lens, rb.seeds, rb.n_committed, rb.rounds), snap):
        t.copy_(s)


def _outputs(eng, rb):
    return [t.clone() for t in (rb.am, rb.v, rb.top_d, rb.top_v, rb.gap_d, rb.gap_v, rb.readback, rb.seq_lens,
                                rb.seeds)]


def _cache(eng):
    # compared after the last round only: a replay from the restored lengths finds the first run's later rows
    return [t.clone() for t in eng.pool.k] + [t.clone() for t in eng.pool.v]


def _rounds(eng, rb, n, small):
    eng.small_rows = 64 if small else 0
    out = []
    for _ in range(n):
        eng.round_launch(rb)
        torch.cuda.synchronize()
        eng.check_status(rb)
        out.append(_outputs(eng, rb))
    return out


@pytest.mark.parametrize("bs", [1, 2, 3])
def test_small_forward_equals_per_launch(bs):
    """The persistent kernel runs the mma.sync attention body: the per-launch reference uses the same kernel for
    every grid size (large grids would otherwise take the tcgen05 kernel, equal only to rounding)."""
    from gravityocr_b200 import _lib as L
    eng, rb = _setup(bs)
    snap = _state(rb)
    L.set_attention_tc(False)
    try:
        ref = _rounds(eng, rb, 3, small=False)
    finally:
        L.set_attention_tc(True)
    ref_cache = _cache(eng)
    _restore(rb, snap)
    got = _rounds(eng, rb, 3, small=True)
    assert len(eng._small) == 2  # one plan per forward kind (draft, verify)
    for r, (a, b) in enumerate(zip(ref, got)):
        for i, (x, y) in enumerate(zip(a, b)):
            assert torch.equal(x, y), f"round {r}: output {i} differs"
    for i, (x, y) in enumerate(zip(ref_cache, _cache(eng))):
        assert torch.equal(x, y), f"K/V cache tensor {i} differs"


def test_small_forward_graph_replay():
    eng, rb = _setup(1)
    snap = _state(rb)
    eng.small_rows = 64
    ref = _rounds(eng, rb, 2, small=True)
    _restore(rb, snap)
    eng.round_launch(rb)  # builds nothing new: the plans exist
    torch.cuda.synchronize()
    _restore(rb, snap)
    gd, gv = eng.capture_split(rb)
    got = []
    for _ in range(2):
        gd.replay()
        gv.replay()
        torch.cuda.synchronize()
        eng.check_status(rb)
        got.append(_outputs(eng, rb))
    for r, (a, b) in enumerate(zip(ref, got)):
        for i, (x, y) in enumerate(zip(a, b)):
            assert torch.equal(x, y), f"graph round {r}: output {i} differs"
