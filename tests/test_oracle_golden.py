"""The CPU oracle against golden vectors produced by the reference itself (tests/golden/make_golden.py)."""
import json
import os

import numpy as np
import pytest
import torch

from oracle.commit_ref import batch_accept, commit_rows, cut_index, ss_commit
from oracle.decoder_ref import OracleDecoder, natcache_generate, spec_generate


def _load(golden_dir, name):
    p = os.path.join(golden_dir, name)
    if not os.path.exists(p):
        pytest.skip(f"{name} not generated")
    return json.load(open(p))


def test_ss_commit_matches_reference_triton_kernel(golden_dir):
    data = _load(golden_dir, "commit_kernel.json")
    assert len(data["cases"]) >= 20
    for c in data["cases"]:
        i, o, K = c["in"], c["out"], c["K"]
        r = ss_commit(np.array(i["predict"], dtype=np.int64), np.array(i["acc"]), np.array(i["a0"]),
                      np.array(i["rpi"]), np.array(i["seeds"], dtype=np.int64), np.array(i["seq_lens"], dtype=np.int64),
                      np.array(i["loc"], dtype=np.int64), K)
        assert r["packed"].tolist() == o["packed"]
        assert r["seeds"].tolist() == o["seeds"]
        assert r["seq_lens"].tolist() == o["seq_lens"]
        assert r["free"].tolist() == o["free"]
        assert r["out"].tolist() == o["out"]
        assert all(x == -1 for x in o["free_tail"])


def test_chain_accept_agrees_with_packed_rows(golden_dir):
    data = _load(golden_dir, "commit_kernel.json")
    for c in data["cases"]:
        K, bs = c["K"], c["bs"]
        pred = np.array(c["in"]["predict"][: bs * K]).reshape(bs, K)
        acc = np.array(c["in"]["acc"])
        am = np.zeros((bs, K), dtype=np.int64)
        for b in range(bs):
            am[b, 1: acc[b] + 1] = pred[b, : acc[b]]
            if acc[b] + 1 < K:
                am[b, acc[b] + 1] = pred[b, acc[b]] + 1
        assert batch_accept(am, pred).tolist() == acc.tolist()


def test_cut_index_matches_reference_rules(golden_dir):
    data = _load(golden_dir, "commit_rules.json")
    for c in data["cut_index"]:
        assert cut_index(c["T"], c["budget"], frozenset(c["stop"]), c["vocab"]) == c["j"], c


def test_host_commit_matches_reference_rules(golden_dir):
    data = _load(golden_dir, "commit_rules.json")
    for c in data["host_commit"]:
        toks, js, accs = commit_rows(c["rows"], c["budgets"], frozenset(c["stop"]), c["vocab"])
        assert (toks, js, accs) == (c["toks"], c["js"], c["accs"])


def _natcache_case(golden_dir, name):
    from gravityocr_b200.config import small_model
    from gravityocr_b200.weights import prefix_embeddings, random_weights, request_inputs
    g = _load(golden_dir, name)
    cfg = small_model(g["n_layers"])
    w = random_weights(cfg, g["weight_seed"], torch.float32)
    img, txt = request_inputs(cfg, g["input_seed"], g["n_image"], g["n_prompt"], 0, torch.float32)
    assert txt.tolist() == g["prompt_ids"]
    return g, cfg, OracleDecoder(cfg, w), prefix_embeddings(w, cfg, img, txt)


def test_natcache_restatement_reproduces_reference_small(golden_dir):
    g, cfg, m, x = _natcache_case(golden_dir, "natcache_small.json")
    tr = []
    s = natcache_generate(m, x, g["max_new_tokens"], g["bd"], tr)
    assert s == g["stream"]
    assert [d["k"] for d in tr] == [d["k"] for d in g["trace"]]
    assert [d["draft"] for d in tr] == [d["draft"] for d in g["trace"]]
    # the served full-draft form commits the same (AR-greedy) stream
    s2 = spec_generate(m, x, g["max_new_tokens"], g["bd"] + 1)
    assert s2 == g["stream"][: len(s2)]
    assert g["teacher_force_argmax"] == g["stream"][: len(g["teacher_force_argmax"])]


@pytest.mark.slow
def test_natcache_restatement_reproduces_reference_config0(golden_dir):
    g, cfg, m, x = _natcache_case(golden_dir, "natcache_config0.json")
    tf, gap, _ = m.teacher_force(x, g["stream"][: g["max_new_tokens"]])
    assert tf == g["teacher_force_argmax"]
    s2 = spec_generate(m, x, 32, g["bd"] + 1)
    assert s2 == g["stream"][:32]


def _natcache_varied(golden_dir, name):
    from gravityocr_b200.config import ModelConfig
    from gravityocr_b200.config import small_model
    from gravityocr_b200.weights import prefix_embeddings, request_inputs, variant_weights
    g = _load(golden_dir, name)
    cfg = small_model(g["n_layers"])
    w = variant_weights(cfg, g["weight_seed"], g["embed_std"], g.get("weight_variant"))
    img, txt = request_inputs(cfg, g["input_seed"], g["n_image"], g["n_prompt"], 0, torch.float32)
    assert txt.tolist() == g["prompt_ids"]
    return g, OracleDecoder(cfg, w), prefix_embeddings(w, cfg, img, txt)


def test_reference_stream_does_not_depend_on_block_size(golden_dir):
    """The reference's own runs at B = 4, 16 and 32 commit one stream (its docs: output invariant to the draft block),
    and that stream is varied (not one repeated token), so it exercises rejections."""
    streams = [_load(golden_dir, f"natcache_varied_bd{b}.json")["stream"] for b in (4, 16, 32)]
    assert streams[0] == streams[1] == streams[2]
    assert len(set(streams[0])) > 0.9 * len(streams[0])


@pytest.mark.slow
def test_natcache_restatement_reproduces_reference_varied(golden_dir):
    g, m, x = _natcache_varied(golden_dir, "natcache_varied_bd16.json")
    tr = []
    s = natcache_generate(m, x, g["max_new_tokens"], g["bd"], tr)
    assert s == g["stream"]
    assert [d["k"] for d in tr] == [d["k"] for d in g["trace"]]
    assert [d["draft"] for d in tr] == [d["draft"] for d in g["trace"]]


@pytest.mark.slow
def test_natcache_restatement_reproduces_reference_mrope(golden_dir):
    """Image tokens on a grid (2-D multimodal RoPE positions): the oracle's natcache reproduces the reference's run."""
    from gravityocr_b200.weights import grid_positions
    g, m, x = _natcache_varied(golden_dir, "natcache_mrope.json")
    pos3 = grid_positions(g["n_image"], g["n_prompt"], g["grid_w"])
    tr = []
    s = natcache_generate(m, x, g["max_new_tokens"], g["bd"], tr, pos3=pos3)
    assert s == g["stream"]
    assert [d["k"] for d in tr] == [d["k"] for d in g["trace"]]
    tf, _, _ = m.teacher_force(x, g["stream"][: g["max_new_tokens"]], pos3=pos3)
    assert tf == g["teacher_force_argmax"]
    # the positions matter: the 1-D layout gives another stream
    assert natcache_generate(m, x, 16, g["bd"]) != s[:16]
