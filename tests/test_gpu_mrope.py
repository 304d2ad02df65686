"""Multimodal (2-D image) RoPE positions on a B200.

* The QKV epilogue with per-row (t, h, w) positions: pair i rotates by the axis of its M-RoPE section ([8, 12, 12]),
  against an fp32 reference (rtol 2e-2 as the 1-D RoPE test).
* The natcache drop-in called as the reference's make_sampler calls it, with get_rope_index returning image tokens on
  a 16 x 16 grid: stream, per-round k and stats equal the reference's own run (tests/golden/natcache_mrope.json), up to
  a first divergence that may only be an fp32 near-tie.
* The served worker with a request carrying the same positions commits the fp32 AR-greedy stream of that prefix
  (teacher-forced argmax with the same positions; near-ties listed).
"""
import json
import os
import types

import pytest
import torch

from gravityocr_b200 import _lib as L
from gravityocr_b200.config import ModelConfig
from gravityocr_b200.engine import rope_inv_freq
from gravityocr_b200.weights import grid_positions, prefix_embeddings, random_weights, request_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"
TIE = 1e-3


def _mrope_ref(x, pos3, inv_freq, rd, sec):
    axis = torch.cat([torch.full((n,), a, dtype=torch.int64) for a, n in enumerate(sec)]).to(x.device)
    f = (pos3.float()[:, axis] * inv_freq.float()[None, :])
    c, s = f.cos()[:, None, :], f.sin()[:, None, :]
    out = x.clone()
    x0, x1 = x[..., 0:rd:2], x[..., 1:rd:2]
    out[..., 0:rd:2] = x0 * c - x1 * s
    out[..., 1:rd:2] = x1 * c + x0 * s
    return out


@pytest.mark.parametrize("m", [17, 300])
def test_qkv_epilogue_with_multimodal_positions(m):
    cfg = ModelConfig()
    g = torch.Generator().manual_seed(31 + m)
    H, nq, nkv, D = cfg.hidden, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
    w = (torch.randn((cfg.qkv_dim, H), generator=g) * 0.02).to(DEV, torch.bfloat16)
    x = torch.randn((m, H), generator=g).to(DEV, torch.bfloat16)
    n_pages, ps = m // 16 + 16, 16
    pos3 = torch.randint(0, 3000, (m, 3), generator=g, dtype=torch.int32)
    slots = torch.randperm(n_pages * ps, generator=g)[:m].to(torch.int64)
    kc = torch.zeros((n_pages, nkv, ps, D), dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    q = torch.zeros((m, nq * D), dtype=torch.bfloat16, device=DEV)
    inv = rope_inv_freq(cfg).to(DEV)
    dummy = torch.zeros((m,), dtype=torch.int32, device=DEV)
    pos3_d, slots_d = pos3.to(DEV).contiguous(), slots.to(DEV)
    e = L.Epilogue()
    e.mode = L.EPI_QKV_ROPE
    e.q_out, e.k_cache, e.v_cache = q.data_ptr(), kc.data_ptr(), vc.data_ptr()
    e.row_pos, e.row_slot, e.inv_freq = dummy.data_ptr(), slots_d.data_ptr(), inv.data_ptr()
    e.row_pos3 = pos3_d.data_ptr()
    for i in range(3):
        e.mrope_section[i] = cfg.mrope_section[i]
    e.rotary_dim, e.n_q_heads, e.n_kv_heads, e.page_size = cfg.rotary_dim, nq, nkv, ps
    ws = torch.zeros((L.linear_workspace_bytes(cfg.qkv_dim, m, L.linear_default_splits(cfg.qkv_dim, H, m, L.EPI_QKV_ROPE)),),
                     dtype=torch.uint8, device=DEV)
    L.linear(w, x, m, e, ws)
    torch.cuda.synchronize()
    y = x.float() @ w.float().T
    qr = _mrope_ref(y[:, : nq * D].view(m, nq, D), pos3_d, inv, cfg.rotary_dim, cfg.mrope_section)
    kr = _mrope_ref(y[:, nq * D: (nq + nkv) * D].view(m, nkv, D), pos3_d, inv, cfg.rotary_dim, cfg.mrope_section)
    torch.testing.assert_close(q.float().view(m, nq, D), qr, rtol=2e-2, atol=2e-2)
    kg = kc.permute(0, 2, 1, 3).reshape(n_pages * ps, nkv, D)[slots_d]
    torch.testing.assert_close(kg.float(), kr, rtol=2e-2, atol=2e-2)
    # a 1-D rotation would differ: the test really exercises the per-axis positions
    assert (pos3[:, 1] != pos3[:, 0]).any()


def test_natcache_with_grid_positions_equals_reference(golden_dir):
    from test_gpu_dropins import _natcache_vs_golden
    if not os.path.exists(os.path.join(golden_dir, "natcache_mrope.json")):
        pytest.skip("natcache_mrope.json not generated")
    _natcache_vs_golden(golden_dir, "natcache_mrope.json", via_reference_model=True)


def test_worker_with_grid_positions_commits_the_ar_stream():
    from oracle.decoder_ref import OracleDecoder
    from gravityocr_b200.compat.sglang_worker import ReqToPagePool, SelfSpecDiffusionWorker
    from gravityocr_b200.compat.types import ForwardMode, Req, SamplingParams, ScheduleBatch
    from gravityocr_b200.config import small_model
    from gravityocr_b200.engine import Engine
    cfg = small_model(2)
    # norm weights near one: the stream depends on the positions (checked below)
    w = random_weights(cfg, 7, torch.bfloat16, norm_center=1.0)
    w32 = {k: v.float() for k, v in w.items()}
    eng = Engine(cfg, w, max_rows=4 * 64, n_pages=8 * 64 + 8)
    target = types.SimpleNamespace(engine=eng, req_to_page=ReqToPagePool(eng, size=8, max_context=1024))
    os.environ["SELFSPEC_MASK_ID"] = str(cfg.mask_id)
    wk = SelfSpecDiffusionWorker(types.SimpleNamespace(speculative_num_draft_tokens=17, page_size=16, model_path=""),
                                 0, 0, None, 0, 0, 0, 0, target)
    reqs = []
    for i in range(2):
        img, txt = request_inputs(cfg, 5, 64, 12, i, torch.bfloat16)
        r = Req(i, img, txt.tolist(), SamplingParams(max_new_tokens=1 << 20), cfg.vocab)
        r.mrope_positions = grid_positions(64, 12, 8)
        reqs.append(r)
    wk.forward_batch_generation(ScheduleBatch(reqs, torch.tensor([1, 4], device=DEV),
                                              torch.zeros(2, dtype=torch.int64, device=DEV), ForwardMode.EXTEND))
    seq = [76, 76]
    for _ in range(5):
        b = ScheduleBatch(reqs, torch.tensor([1, 4], device=DEV), torch.tensor(seq, device=DEV), ForwardMode.DECODE,
                          torch.tensor(seq))
        res = wk.forward_batch_generation(b)
        seq = [s + j + 1 for s, j in zip(seq, res.accept_length_per_req_cpu)]
    for r in reqs:
        img = r.image_embeds.float()
        txt = torch.tensor(r.origin_input_ids[64:])
        x = prefix_embeddings(w32, cfg, img, txt)
        out = r.output_ids
        tf, gap, _ = OracleDecoder(cfg, w32).teacher_force(x, out, pos3=r.mrope_positions)
        bad = [(i, out[i], tf[i], gap[i]) for i in range(len(out)) if out[i] != tf[i] and gap[i] >= TIE]
        assert not bad, bad[:4]
        # and the 1-D layout would have given another stream
        tf1, _, _ = OracleDecoder(cfg, w32).teacher_force(x, out)
        assert tf1 != tf
