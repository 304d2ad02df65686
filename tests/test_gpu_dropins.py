"""The two drop-ins at the reference's own boundary, on a B200.

natcache (``compat.natcache.generate_speculative_natcache``):
  * called exactly as the reference's ``make_sampler`` calls it (``src/infer_omnidocbench.py:441-446``): a model object
    with the reference ``GlmOcrBlockDiffusion``'s handles (processor, tokenizer, mm_model.get_image_features /
    get_rope_index, text_model, glm.lm_head, bd_size, mask_id, image_token_id) around transformers'
    ``GlmOcrForConditionalGeneration`` holding the seeded weights, and a PIL crop;
  * its stream, per-round trace (k, new tokens) and stats must be the reference's own (tests/golden/natcache_*.json,
    produced by running ``src/fast_sampling.py:425`` on CPU), up to a first divergence that may only sit at an fp32
    argmax near-tie (top-2 gap < 1e-3).
SelfSpecDiffusionWorker (``compat.sglang_worker``), result contract of ``selfspec_diffusion_worker.py:954-961,990-998``:
  * extend then decode rounds for a batch of 3: every request's committed tokens are the fp32 AR-greedy stream of that
    request alone (near-ties listed), next_token_ids = the device next seeds, accept lengths = j;
  * a request cut inside a round by its length budget or by a stop id keeps exactly T[:j+1] and its K/V length is
    S + j + 1 (``kv_committed += j + 1``);
  * batch composition changes between rounds (a request leaves, a new one joins) keep every stream intact.
"""
import json
import os
import types

import pytest
import torch

from gravityocr_b200.compat.natcache import SelfSpecModel, generate_speculative_natcache
from gravityocr_b200.compat.sglang_worker import ReqToPagePool, SelfSpecDiffusionWorker
from gravityocr_b200.compat.types import ForwardMode, Req, SamplingParams, ScheduleBatch
from gravityocr_b200.config import ModelConfig, small_model
from gravityocr_b200.engine import Engine
from gravityocr_b200.weights import (grid_positions, prefix_embeddings, prefix_token_ids, random_weights,
                                     request_inputs, variant_weights)

pytestmark = pytest.mark.gpu
DEV = "cuda"
TIE = 1e-3


# ---------------------------------------------------------------------- natcache
class _RefShapedModel(torch.nn.Module):
    """The handles the reference's natcache reads from ``GlmOcrBlockDiffusion`` (``src/models/glm_ocr_dllm.py:139-183``),
    around a transformers GlmOcrForConditionalGeneration; the processor and vision tower are stand-ins that hand the
    seeded image embeddings and 1-D positions to the caller, as the golden generator's run of the reference did."""

    def __init__(self, cfg, w32, n_img, txt, img, bd, pos3=None):
        super().__init__()
        from transformers import GlmOcrConfig, GlmOcrForConditionalGeneration
        hf = GlmOcrConfig()
        tc = hf.text_config
        tc.num_hidden_layers, tc.hidden_size = cfg.n_layers, cfg.hidden
        tc.num_attention_heads, tc.num_key_value_heads, tc.head_dim = cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
        tc.intermediate_size, tc.vocab_size, tc.rms_norm_eps = cfg.intermediate, cfg.vocab, cfg.rms_eps
        tc.rope_parameters = {"rope_theta": cfg.rope_theta, "rope_type": "default",
                              "partial_rotary_factor": cfg.rotary_dim / cfg.head_dim, "mrope_section": [8, 12, 12]}
        hf.vision_config.depth = 1
        with torch.device("meta"):   # parameters are assigned from the seeded weights below (the vision tower unused)
            self.glm = GlmOcrForConditionalGeneration(hf).eval()
        sd = {}
        for k, t in w32.items():
            if k == "lm_head":
                sd["lm_head.weight"] = t
            elif k.startswith("layers."):
                _, l, n = k.split(".", 2)
                mod = "self_attn." if n.endswith("_proj") and n[0] in "qkvo" else ("mlp." if n.endswith("_proj") else "")
                sd[f"model.language_model.layers.{l}.{mod}{n}.weight"] = t
            else:
                sd[f"model.language_model.{k}.weight"] = t
        missing, unexpected = self.glm.load_state_dict(sd, strict=False, assign=True)
        assert not unexpected and all("visual" in m for m in missing)
        self.bd_size, self.mask_id, self.image_token_id = bd, cfg.mask_id, cfg.image_token_id
        ids = prefix_token_ids(cfg, n_img, txt)[None]

        class _Enc(dict):
            def to(self, dev):
                return self

        class _Proc:
            def apply_chat_template(self, *a, **k):
                return ""

            def __call__(self, *a, **k):
                return _Enc({"input_ids": ids, "mm_token_type_ids": torch.zeros_like(ids), "pixel_values": torch.zeros(1),
                             "image_grid_thw": None})

        self.processor = _Proc()
        self.tokenizer = types.SimpleNamespace(eos_token_id=None)
        mm = self.glm.model
        mm.get_image_features = lambda pv, thw, return_dict=True: types.SimpleNamespace(pooler_output=[img])
        p3 = torch.arange(ids.shape[1]).expand(3, -1) if pos3 is None else pos3
        mm.get_rope_index = lambda i, t, image_grid_thw=None, video_grid_thw=None, attention_mask=None: (
            p3[:, None, :].clone(), None)

    @property
    def mm_model(self):
        return self.glm.model

    @property
    def text_model(self):
        return self.glm.model.language_model


def _natcache_vs_golden(golden_dir, name, via_reference_model):
    from oracle.decoder_ref import OracleDecoder
    g = json.load(open(os.path.join(golden_dir, name)))
    cfg = small_model(g["n_layers"]) if g["n_layers"] != 16 else ModelConfig()
    w32 = variant_weights(cfg, g["weight_seed"], g.get("embed_std", 0.02), g.get("weight_variant"))
    img, txt = request_inputs(cfg, g["input_seed"], g["n_image"], g["n_prompt"], 0, torch.float32)
    assert txt.tolist() == g["prompt_ids"]
    n, bd = g["max_new_tokens"], g["bd"]
    pos3 = grid_positions(g["n_image"], g["n_prompt"], g["grid_w"]) if g.get("grid_w") else None
    tr = []
    if via_reference_model:
        from PIL import Image
        model = _RefShapedModel(cfg, w32, g["n_image"], txt, img, bd, pos3)
        _, st = generate_speculative_natcache(model, Image.new("RGB", (8, 8)), max_new_tokens=n, return_stats=True,
                                              trace=tr)
        assert model.gr_engine.engine.cfg == cfg
        del model
    else:
        eng = Engine(cfg, {k: v.to(torch.bfloat16) for k, v in w32.items()}, max_rows=64,
                     n_pages=4 * ((g["n_image"] + g["n_prompt"] + n + 200) // 16))
        _, st = generate_speculative_natcache(SelfSpecModel(eng, bd_size=bd), img, prompt=txt, max_new_tokens=n,
                                              return_stats=True, trace=tr)
    ours = [t for d in tr for t in d["new_tokens"]]
    ref = g["stream"]
    m = min(len(ours), len(ref))
    first_div = next((i for i in range(m) if ours[i] != ref[i]), m)
    if first_div < m or len(ours) != len(ref):
        # only an fp32 argmax near-tie may separate the streams (teacher-forced gap of the reference model)
        x = prefix_embeddings(w32, cfg, img, txt)
        _, gap, _ = OracleDecoder(cfg, w32).teacher_force(x, ours[: first_div + 1], pos3=pos3)
        assert first_div < m and gap[first_div] < TIE, f"{name}: diverges at {first_div} with gap {gap[first_div]}"
        print(f"{name}: same stream for {first_div} tokens, then an fp32 near-tie (gap {gap[first_div]:.2e})")
        return
    assert st == g["stats"], (st, g["stats"])
    assert [d["k"] for d in tr] == [d["k"] for d in g["trace"]]
    assert [d["new_tokens"] for d in tr] == [d["new_tokens"] for d in g["trace"]]
    same_drafts = sum(a["draft"] == b["draft"] for a, b in zip(tr, g["trace"]))
    print(f"{name}: stream, k and stats identical to the reference; drafts identical in {same_drafts}/{len(tr)} rounds")


def test_natcache_small_equals_reference(golden_dir):
    _natcache_vs_golden(golden_dir, "natcache_small.json", via_reference_model=False)


@pytest.mark.parametrize("name", ["natcache_varied_bd16.json", "natcache_varied_bd4.json",
                                  "natcache_varied_bd32.json", "natcache_config0.json"])
def test_natcache_reference_call_equals_reference(golden_dir, name):
    if not os.path.exists(os.path.join(golden_dir, name)):
        pytest.skip(f"{name} not generated")
    _natcache_vs_golden(golden_dir, name, via_reference_model=True)


def test_natcache_refuses_accept_conf():
    cfg = small_model(2)
    eng = Engine(cfg, random_weights(cfg, 0, torch.bfloat16), max_rows=64, n_pages=64)
    img, txt = request_inputs(cfg, 0, 16, 4, 0, torch.float32)
    with pytest.raises(ValueError, match="accept_conf"):
        generate_speculative_natcache(SelfSpecModel(eng), img, prompt=txt, max_new_tokens=8, accept_conf=0.5)


# ---------------------------------------------------------------------- served worker
def _worker(cfg, w, pool_size=8, max_context=1024, K=17):
    eng = Engine(cfg, w, max_rows=max(pool_size * K, 4 * 64), n_pages=pool_size * (max_context // 16) + 8)
    target = types.SimpleNamespace(engine=eng, req_to_page=ReqToPagePool(eng, size=pool_size, max_context=max_context))
    args = types.SimpleNamespace(speculative_num_draft_tokens=K, page_size=16, model_path="")
    os.environ["SELFSPEC_MASK_ID"] = str(cfg.mask_id)
    return SelfSpecDiffusionWorker(args, 0, 0, None, 0, 0, 0, 0, target), eng


def _req(cfg, i, max_new, stop=None, n_img=48, n_prompt=12):
    img, txt = request_inputs(cfg, 5, n_img, n_prompt, i, torch.bfloat16)
    return Req(i, img, txt.tolist(), SamplingParams(max_new_tokens=max_new, stop_token_ids=stop), cfg.vocab)


def _extend(wk, reqs, slots):
    b = ScheduleBatch(reqs, torch.tensor(slots, dtype=torch.int64, device=DEV),
                      torch.zeros((len(reqs),), dtype=torch.int64, device=DEV), ForwardMode.EXTEND)
    return wk.forward_batch_generation(b)


def _decode_batch(reqs, slots, seq_lens):
    return ScheduleBatch(reqs, torch.tensor(slots, dtype=torch.int64, device=DEV),
                         torch.tensor(seq_lens, dtype=torch.int64, device=DEV), ForwardMode.DECODE,
                         torch.tensor(seq_lens, dtype=torch.int64))


def _ar_check(cfg, w32, req, stream):
    """Every committed token equals the fp32 teacher-forced argmax of that request alone, or is a near-tie."""
    from oracle.decoder_ref import OracleDecoder
    img = req.image_embeds.float()
    txt = torch.tensor(req.origin_input_ids[img.shape[0]:])
    x = prefix_embeddings(w32, cfg, img, txt)
    tf, gap, _ = OracleDecoder(cfg, w32).teacher_force(x, stream)
    bad = [(i, stream[i], tf[i], gap[i]) for i in range(len(stream)) if stream[i] != tf[i] and gap[i] >= TIE]
    assert not bad, f"request {req.rid}: tokens off the AR argmax beyond near-ties {bad[:4]}"


def test_worker_rounds_commit_ar_streams_and_contract():
    cfg = small_model(2)
    w = random_weights(cfg, 7, torch.bfloat16, embed_std=0.25)
    w32 = {k: v.float() for k, v in w.items()}
    wk, eng = _worker(cfg, w)
    reqs = [_req(cfg, i, 1 << 20) for i in range(3)]
    slots = [5, 1, 3]
    res = _extend(wk, reqs, slots)
    assert res.finish_checked and [r.output_ids for r in reqs] == res.next_token_ids_cpu
    seq = [len(r.origin_input_ids) for r in reqs]
    batch = _decode_batch(reqs, slots, seq)
    for _ in range(5):
        before = [len(r.output_ids) for r in reqs]
        sl0 = batch.seq_lens_cpu.clone()
        res = wk.forward_batch_generation(batch)
        assert res.finish_checked
        for i, r in enumerate(reqs):
            assert r.output_ids[before[i]:] == res.next_token_ids_cpu[i]
            j = res.accept_length_per_req_cpu[i]
            assert len(res.next_token_ids_cpu[i]) == j + 1
            assert int(batch.seq_lens_cpu[i]) == int(sl0[i]) + j + 1 == int(batch.seq_lens[i])
            assert int(res.next_token_ids[i]) == r.output_ids[-1]       # the next seed is the last committed token
        assert res.num_accepted_tokens == sum(res.accept_length_per_req_cpu)
    for r in reqs:
        _ar_check(cfg, w32, r, r.output_ids)


def test_worker_cut_inside_round_and_batch_changes():
    cfg = small_model(2)
    w = random_weights(cfg, 7, torch.bfloat16, embed_std=0.25)
    w32 = {k: v.float() for k, v in w.items()}
    # reference streams of two requests, to pick a stop id that falls inside a round
    wk0, _ = _worker(cfg, w)
    probe = [_req(cfg, i, 1 << 20) for i in range(2)]
    _extend(wk0, probe, [0, 1])
    b0 = _decode_batch(probe, [0, 1], [r.image_embeds.shape[0] + 12 for r in probe])
    for _ in range(4):
        wk0.forward_batch_generation(b0)
    stop_tok = probe[1].output_ids[5]   # a0 of a later round: the cut falls inside that round
    del wk0, b0
    wk, eng = _worker(cfg, w)
    # request 0: a length budget of 4 (ends inside its second round); request 1: a stop id; request 2 joins later
    reqs = [_req(cfg, 0, 4), _req(cfg, 1, 1 << 20, stop=[stop_tok]), _req(cfg, 2, 1 << 20)]
    live, slots = reqs[:2], [4, 2]
    _extend(wk, live, slots)
    P = [r.image_embeds.shape[0] + 12 for r in reqs]
    seq = {4: P[0], 2: P[1]}
    rounds = 0
    while live and rounds < 40:
        batch = _decode_batch(live, slots, [seq[s] for s in slots])
        res = wk.forward_batch_generation(batch)
        rounds += 1
        for i, (r, s) in enumerate(zip(live, slots)):
            j = res.accept_length_per_req_cpu[i]
            assert int(batch.seq_lens[i]) == seq[s] + j + 1      # K/V keeps x0 and T[:j]
            seq[s] += j + 1
        keep = [(r, s) for r, s in zip(live, slots) if not r.finished()]
        for r, s in zip(live, slots):
            if r.finished():
                wk.req_to_page.release(s)
        live, slots = [k[0] for k in keep], [k[1] for k in keep]
        if rounds == 2:   # a new request joins a running batch
            _extend(wk, [reqs[2]], [6])
            live.append(reqs[2])
            slots.append(6)
            seq[6] = P[2]
        if reqs[2].output_ids and len(reqs[2].output_ids) > 40:
            reqs[2].to_finish = types.SimpleNamespace(kind="abort")
            reqs[2].check_finished()
    assert reqs[0].finished_reason.kind == "length" and len(reqs[0].output_ids) == 4
    assert reqs[1].finished_reason.kind == "stop" and reqs[1].output_ids[-1] == stop_tok
    assert stop_tok not in reqs[1].output_ids[:-1]
    for r in reqs:
        _ar_check(cfg, w32, r, r.output_ids)
