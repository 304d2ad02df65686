"""Generate the golden vectors that pin the CPU oracle to the reference implementation.

Run in the build container, where the reference tree is readable (it is never read on the GPU box):

    python tests/golden/make_golden.py --ref /path/to/GravityOCR [--only natcache_small,commit_kernel,...]

Outputs (small JSON files next to this script):
  * ``natcache_<case>.json``: the reference's own ``generate_speculative_natcache`` (``src/fast_sampling.py:425``) and
    ``teacher_force_argmax`` (``:631``) run unmodified on CPU on a random-init transformers ``GlmOcrForConditionalGeneration``
    holding ``gravityocr_b200.weights.random_weights`` -- per-round trace, committed stream, teacher-forced argmax.
    Settings follow the reference's own ``--no_dynamo`` (``src/infer_omnidocbench.py:614-616``); the processor and the
    vision tower are stubbed so the seeded image embeddings are injected as inputs_embeds at image-token positions and
    positions are 1-D (``get_rope_index`` -> arange).
  * ``commit_kernel.json``: the reference Triton ``_ss_commit_kernel`` (``selfspec_fast_commit.py:108-147``) executed
    by the Triton CPU interpreter on seeded inputs (its source is parsed out of the reference file at generation time).
  * ``commit_rules.json``: ``cut_index`` and ``host_commit`` of ``selfspec_commit_rules.py`` on seeded rows.
  * ``sampling.json``: ``selfspec_sampling.py``'s penalties, penalizer cumulation and target distributions on seeded
    small-vocabulary rows (the penalizers are stand-ins carrying SGLang's class names and state tensors).
"""
from __future__ import annotations

import argparse
import ast
import json
import os
import random
import sys
import time
import types

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

NATCACHE_CASES = {
    # name: (n_layers, n_image, n_prompt, max_new_tokens, bd, weight_seed, input_seed, embed_std, grid_w)
    "small": (2, 64, 16, 48, 16, 0, 0, 0.02, 0),
    "config0": (16, 256, 32, 128, 16, 0, 0, 0.02, 0),
    # the config-0 model with its token-embedding table drawn at std 0.25: a varied stream (the baseline's 0.02 settles
    # on one repeated token), drafted at three block sizes -- the committed stream must not depend on B
    "varied_bd16": (16, 256, 32, 128, 16, 0, 0, 0.25, 0),
    "varied_bd4": (16, 256, 32, 128, 4, 0, 0, 0.25, 0),
    "varied_bd32": (16, 256, 32, 128, 32, 0, 0, 0.25, 0),
    # image tokens on a 16 x 16 grid: 2-D multimodal RoPE positions (get_rope_index returns them), response tokens at
    # max position + 1 + r; 4 layers with norm weights near one (WEIGHT_VARIANTS) so the stream depends on them
    "mrope": (4, 256, 32, 64, 16, 0, 0, 0.02, 16),
}
# extra random_weights arguments per case (the rest use the baseline draw); "bf16_weights": the reference runs on the
# bf16-rounded weights the CUDA path holds.  Sharper attention (q/k std 0.05) or 16 such layers make the bf16 and fp32
# streams part at non-tied tokens within a few tokens even with 1-D positions, so the case stays at 4 layers.
WEIGHT_VARIANTS = {"mrope": {"norm_center": 1.0, "bf16_weights": True}}


def _dump(name, obj):
    path = os.path.join(HERE, name)
    with open(path, "w") as f:
        json.dump(obj, f, separators=(",", ":"))
    print(f"wrote {path} ({os.path.getsize(path)} B)")


def gen_natcache(ref: str, case: str):
    import torch
    torch._dynamo.config.disable = True
    sys.path.insert(0, os.path.join(ref, "src"))
    import fast_sampling as fs
    from models.glm_ocr_dllm import GlmOcrBlockDiffusion
    from transformers import GlmOcrConfig, GlmOcrForConditionalGeneration
    from gravityocr_b200.config import small_model
    from gravityocr_b200.weights import grid_positions, request_inputs, prefix_token_ids, variant_weights

    L, n_img, n_txt, new, bd, wseed, iseed, estd, grid_w = NATCACHE_CASES[case]
    cfg = small_model(L)
    hf = GlmOcrConfig()
    tc = hf.text_config
    tc.num_hidden_layers = L
    tc.hidden_size = cfg.hidden
    tc.num_attention_heads = cfg.n_q_heads
    tc.num_key_value_heads = cfg.n_kv_heads
    tc.head_dim = cfg.head_dim
    tc.intermediate_size = cfg.intermediate
    tc.vocab_size = cfg.vocab
    tc.rms_norm_eps = cfg.rms_eps
    tc.rope_parameters = {"rope_theta": cfg.rope_theta, "rope_type": "default",
                          "partial_rotary_factor": cfg.rotary_dim / cfg.head_dim, "mrope_section": [8, 12, 12]}
    hf.vision_config.depth = 1
    torch.manual_seed(0)
    glm = GlmOcrForConditionalGeneration(hf).float().eval()
    wv = WEIGHT_VARIANTS.get(case, {})
    w = variant_weights(cfg, wseed, estd, wv)
    sd = {}
    for k, t in w.items():
        if k == "lm_head":
            sd["lm_head.weight"] = t
        elif k.startswith("layers."):
            _, l, n = k.split(".", 2)
            mod = "self_attn." if n.endswith("_proj") and n[0] in "qkvo" else ("mlp." if n.endswith("_proj") else "")
            sd[f"model.language_model.layers.{l}.{mod}{n}.weight"] = t
        else:
            sd[f"model.language_model.{k}.weight"] = t
    missing, unexpected = glm.load_state_dict(sd, strict=False)
    assert not unexpected and all("visual" in m for m in missing), (missing, unexpected)

    m = object.__new__(GlmOcrBlockDiffusion)
    torch.nn.Module.__init__(m)
    m.glm = glm
    m.bd_size = bd
    m.mask_id = cfg.mask_id
    m.image_token_id = hf.image_token_id
    m.loop_enabled = False
    glm.model.language_model.config._attn_implementation = "flex_attention"
    img, txt = request_inputs(cfg, iseed, n_img, n_txt, 0, torch.float32)
    ids = prefix_token_ids(cfg, n_img, txt)[None]

    class _Enc(dict):
        def to(self, dev):
            return self

    class _Proc:
        def apply_chat_template(self, *a, **k):
            return ""

        def __call__(self, *a, **k):
            return _Enc({"input_ids": ids, "mm_token_type_ids": torch.zeros_like(ids),
                         "pixel_values": torch.zeros(1), "image_grid_thw": None})

    m.processor = _Proc()
    m.tokenizer = types.SimpleNamespace(eos_token_id=None, decode=lambda *a, **k: "")
    mm = glm.model
    mm.get_image_features = lambda pv, thw, return_dict=True: types.SimpleNamespace(pooler_output=[img])
    pos3 = (grid_positions(n_img, n_txt, grid_w) if grid_w else torch.arange(n_img + n_txt).expand(3, -1))
    mm.get_rope_index = lambda ids_, mmtt, image_grid_thw=None, video_grid_thw=None, attention_mask=None: (
        pos3[:, None, :].clone(), None)
    from PIL import Image
    im = Image.new("RGB", (8, 8))
    t0 = time.time()
    tr = []
    _, st = fs.generate_speculative_natcache(m, im, max_new_tokens=new, return_stats=True, trace=tr)
    t1 = time.time()
    stream = [t for d in tr for t in d["new_tokens"]]
    tf = fs.teacher_force_argmax(m, im, "x", stream[:new])
    t2 = time.time()
    print(f"natcache {case}: {t1 - t0:.1f}s, teacher force {t2 - t1:.1f}s, stats {st}")
    _dump(f"natcache_{case}.json", {
        "source": "reference src/fast_sampling.py generate_speculative_natcache + teacher_force_argmax (CPU, fp32)",
        "n_layers": L, "n_image": n_img, "n_prompt": n_txt, "max_new_tokens": new, "bd": bd,
        "weight_seed": wseed, "input_seed": iseed, "embed_std": estd, "grid_w": grid_w, "weight_variant": wv,
        "mask_id": cfg.mask_id,
        "prompt_ids": txt.tolist(),
        "stream": stream, "teacher_force_argmax": tf, "stats": st,
        "trace": [{"k": d["k"], "draft": d["draft"], "ar_pred": d["ar_pred"], "new_tokens": d["new_tokens"]} for d in tr],
        "seconds": round(t1 - t0, 2), "threads": torch.get_num_threads(),
    })


def gen_commit_kernel(ref: str):
    os.environ["TRITON_INTERPRET"] = "1"
    import torch
    import triton
    import triton.language as tl
    src = os.path.join(ref, "patches/sglang/python/sglang/srt/speculative/selfspec_fast_commit.py")
    tree = ast.parse(open(src).read())
    fn = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "_ss_commit_kernel"][0]
    ns = {"triton": triton, "tl": tl}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), src, "exec"), ns)
    kern = ns["_ss_commit_kernel"]
    rng = random.Random(1234)
    cases = []
    for K in (5, 9, 17, 33):
        for bs in (1, 2, 3, 8, 33):
            pool = 2 * bs + 3
            predict = torch.tensor([rng.randrange(0, 59392) for _ in range(bs * K + 1)], dtype=torch.int32)
            accs = [rng.choice([0, K - 1, rng.randrange(0, K)]) for _ in range(bs)]
            acc = torch.tensor(accs, dtype=torch.int32)
            a0m = torch.tensor([[rng.randrange(0, 59392) for _ in range(K)] for _ in range(bs)], dtype=torch.int64)
            a0 = a0m[:, 0]
            rpi = torch.tensor(rng.sample(range(pool), bs), dtype=torch.int64)
            seeds = torch.tensor([rng.randrange(0, 59392) for _ in range(pool)], dtype=torch.int64)
            sl = torch.tensor([rng.randrange(1, 9000) for _ in range(bs)], dtype=torch.int64)
            loc = torch.tensor(rng.sample(range(10 * bs * K + 100), bs * K), dtype=torch.int64)
            packed = torch.zeros((bs, K + 2), dtype=torch.int32)
            free = torch.full((bs * K,), -1, dtype=torch.int64)
            out = torch.zeros((bs,), dtype=torch.int64)
            inp = {"predict": predict.tolist(), "acc": accs, "a0": a0.tolist(), "rpi": rpi.tolist(),
                   "seeds": seeds.tolist(), "seq_lens": sl.tolist(), "loc": loc.tolist()}
            kern[(bs,)](predict, acc, a0, a0.stride(0), rpi, seeds, sl, loc, packed, free, out,
                        K=K, KP2=triton.next_power_of_2(K), BS_POW2=triton.next_power_of_2(max(bs, 2)))
            n_free = sum(K - 1 - a for a in accs)
            cases.append({"K": K, "bs": bs, "pool": pool, "in": inp,
                          "out": {"packed": packed.tolist(), "seeds": seeds.tolist(), "seq_lens": sl.tolist(),
                                  "free": free[:n_free].tolist(), "free_tail": free[n_free:].tolist(), "out": out.tolist()}})
    _dump("commit_kernel.json", {"source": "reference selfspec_fast_commit.py _ss_commit_kernel under TRITON_INTERPRET=1",
                                 "cases": cases})


def gen_commit_rules(ref: str):
    sys.path.insert(0, os.path.join(ref, "patches/sglang/python/sglang/srt/speculative"))
    import selfspec_commit_rules as R
    rng = random.Random(99)
    V = 59392
    cut = []
    for _ in range(400):
        n = rng.randrange(1, 35)
        T = [rng.choice([rng.randrange(0, V), rng.randrange(0, V), rng.choice([-1, V + 1, V, 7, 11])]) for _ in range(n)]
        budget = rng.choice([0, 1, 2, n - 1, n, n + 1, rng.randrange(0, 2 * n + 2)])
        stop = frozenset(rng.sample([7, 11, 13, 151329, 59246], rng.randrange(0, 3)))
        cut.append({"T": T, "budget": budget, "stop": sorted(stop), "vocab": V, "j": R.cut_index(T, budget, stop, V)})

    class _SP:
        def __init__(self, mx):
            self.max_new_tokens = mx
            self.ignore_eos = False
            self.stop_token_ids = [7]
            self.stop_strs = None
            self.stop_regex_strs = None

    class _Req:
        """Minimal stand-in: the fast path only reads these attributes; finish state is not recorded."""

        def __init__(self, mx, out):
            self.sampling_params = _SP(mx)
            self.eos_token_ids = {11}
            self.tokenizer = None
            self.grammar = None
            self.to_finish = None
            self.vocab_size = V
            self.output_ids = list(out)
            self.spec_verify_ct = 0
            self.spec_accepted_tokens = 0
            self.hist = []

        def finished(self):
            return False

        def check_finished(self, n=1):
            pass

        def update_spec_acceptance_histogram(self, a):
            self.hist.append(a)

    hc = []
    for _ in range(60):
        bs = rng.randrange(1, 6)
        K = rng.choice([5, 17, 33])
        reqs, rows, budgets = [], [], []
        for _ in range(bs):
            prev = rng.randrange(0, 40)
            mx = prev + rng.randrange(1, K + 4)
            r = _Req(mx, [1] * prev)
            a = rng.randrange(0, K)
            row = [rng.randrange(0, V), a] + [rng.choice([rng.randrange(0, V), 7, 11, 12]) for _ in range(a + 1)] + [0] * (K - 1 - a)
            reqs.append(r)
            rows.append(row)
            budgets.append(mx - prev)
        toks, js, accs = R.host_commit(reqs, rows)
        hc.append({"K": K, "rows": rows, "budgets": budgets, "stop": [7, 11], "vocab": V,
                   "toks": toks, "js": js, "accs": accs, "accepted_counters": [q.spec_accepted_tokens for q in reqs]})
    _dump("commit_rules.json", {"source": "reference selfspec_commit_rules.py cut_index / host_commit",
                                "cut_index": cut, "host_commit": hc})


def gen_sampling(ref: str):
    """The reference's selfspec_sampling.py (torch only) on seeded small-vocabulary inputs: penalize_rows with stand-in
    penalizers carrying SGLang's class names and state tensors, cumulate_block, joint_top_k_top_p, torch_backend_filter,
    min_p_filter and verify_target_probs."""
    import torch
    sys.path.insert(0, os.path.join(ref, "patches/sglang/python/sglang/srt/speculative"))
    import selfspec_sampling as S
    import base64
    import numpy as np
    g = torch.Generator().manual_seed(4242)
    V, bs, K = 48, 3, 5

    def b64(t):   # exact float32 values, compactly
        return base64.b64encode(np.ascontiguousarray(t.detach().float().numpy(), dtype="<f4").tobytes()).decode()

    def rnd(*shape):
        return torch.randn(*shape, generator=g)

    def mk(name, **attrs):
        cls = type(name, (), {"is_prepared": lambda self: True})
        o = cls()
        for k, v in attrs.items():
            setattr(o, k, v)
        return o

    def apply_scaling(logits, pen):   # SGLang's apply_scaling_penalties
        logits[:] = torch.where(logits < 0, logits * pen, logits / pen)

    out = {"V": V, "bs": bs, "K": K, "penalize": [], "filters": [], "target": []}
    for case in range(4):
        order = [["BatchedFrequencyPenalizer", "BatchedMinNewTokensPenalizer", "BatchedPresencePenalizer",
                  "BatchedRepetitionPenalizer"], ["BatchedRepetitionPenalizer", "BatchedPresencePenalizer",
                  "BatchedFrequencyPenalizer", "BatchedMinNewTokensPenalizer"]][case % 2]
        rep_p = 1.0 + torch.rand(bs, 1, generator=g)
        fre_p = torch.rand(bs, 1, generator=g)
        pre_p = torch.rand(bs, 1, generator=g)
        seen = torch.randint(0, V, (bs, 12), generator=g)
        cum_rep = torch.ones(bs, V)
        cum_rep.scatter_(1, seen, rep_p.expand(-1, 12))
        cum_fre = torch.zeros(bs, V)
        cum_fre.scatter_add_(1, seen, fre_p.expand(-1, 12).contiguous())
        cum_pre = torch.zeros(bs, V)
        cum_pre.scatter_(1, seen, pre_p.expand(-1, 12))
        len_out = torch.randint(0, 6, (bs, 1), generator=g)
        min_new = torch.randint(0, 8, (bs, 1), generator=g)
        stop_ids = torch.randint(0, V, (bs, 2), generator=g)
        stop_pen = torch.zeros(bs, V)
        stop_pen.scatter_(1, stop_ids, float("-inf"))
        pens = {
            "BatchedRepetitionPenalizer": mk("BatchedRepetitionPenalizer", cumulated_repetition_penalties=cum_rep.clone(),
                                             repetition_penalties=rep_p),
            "BatchedFrequencyPenalizer": mk("BatchedFrequencyPenalizer", cumulated_frequency_penalties=cum_fre.clone(),
                                            frequency_penalties=fre_p),
            "BatchedPresencePenalizer": mk("BatchedPresencePenalizer", cumulated_presence_penalties=cum_pre.clone(),
                                           presence_penalties=pre_p),
            "BatchedMinNewTokensPenalizer": mk("BatchedMinNewTokensPenalizer", len_output_tokens=len_out.clone(),
                                               min_new_tokens=min_new, stop_token_penalties=stop_pen),
        }
        orch = types.SimpleNamespace(is_required=True, penalizers={n: pens[n] for n in order})
        cand = torch.randint(0, V, (bs, K), generator=g)
        cand[:, 2] = cand[:, 1]                     # repeated in-block tokens
        logits = rnd(bs * K, V) * 3
        lg = logits.clone()
        S.penalize_rows(orch, lg, cand, apply_scaling)
        tok = torch.randint(0, V, (bs, 7), generator=g)
        valid = torch.rand(bs, 7, generator=g) < 0.6
        valid[0] = False
        S.cumulate_block(orch, tok, valid)
        out["penalize"].append({
            "order": order, "rep": rep_p.view(-1).tolist(), "freq": fre_p.view(-1).tolist(),
            "pres": pre_p.view(-1).tolist(), "seen": seen.tolist(), "len_out": len_out.view(-1).tolist(),
            "min_new": min_new.view(-1).tolist(), "stop_ids": stop_ids.tolist(), "cand": cand.tolist(),
            "logits": b64(logits), "out": b64(lg),
            "cum_tok": tok.tolist(), "cum_valid": valid.tolist(),
            "after": {"rep": b64(pens["BatchedRepetitionPenalizer"].cumulated_repetition_penalties),
                      "freq": b64(pens["BatchedFrequencyPenalizer"].cumulated_frequency_penalties),
                      "pres": b64(pens["BatchedPresencePenalizer"].cumulated_presence_penalties),
                      "len_out": pens["BatchedMinNewTokensPenalizer"].len_output_tokens.view(-1).tolist()}})
    for case in range(4):
        rows = 6
        # probabilities with tie groups (quantised logits)
        lo = torch.round(rnd(rows, V) * 2) / 2
        probs = torch.softmax(lo, dim=-1)
        top_k = torch.tensor([1, 3, 8, V, 20, 1 << 30], dtype=torch.int64)[torch.randperm(6, generator=g)]
        top_p = torch.tensor([0.3, 0.9, 1.0, 0.5, 0.99, 0.7])[torch.randperm(6, generator=g)]
        min_p = torch.tensor([0.0, 0.05, 0.2, 0.0, 0.5, 0.1])[torch.randperm(6, generator=g)]
        out["filters"].append({
            "probs": b64(probs), "top_k": top_k.tolist(), "top_p": top_p.tolist(), "min_p": min_p.tolist(),
            "joint": b64(S.joint_top_k_top_p(probs, top_k, top_p)),
            "torch": b64(S.torch_backend_filter(probs, top_k, top_p, min_p, True)),
            "torch_no_min_p": b64(S.torch_backend_filter(probs, top_k, top_p, min_p, False)),
            "min_p_filtered": b64(S.min_p_filter(probs, min_p))})
    for case in range(2):
        lg = rnd(bs * K, V) * 2
        si = types.SimpleNamespace(temperatures=(0.3 + torch.rand(bs, 1, generator=g)),
                                   top_ks=torch.tensor([1, 5, 1 << 30], dtype=torch.int32),
                                   top_ps=torch.tensor([1.0, 0.8, 0.6]), min_ps=torch.tensor([0.0, 0.1, 0.0]),
                                   need_top_p_sampling=True, need_top_k_sampling=True, need_min_p_sampling=False)
        fi = S.verify_target_probs(lg.clone(), si, K, "flashinfer")
        si.need_min_p_sampling = True
        pt = S.verify_target_probs(lg.clone(), si, K, "pytorch")
        out["target"].append({"logits": b64(lg), "temperature": si.temperatures.view(-1).tolist(),
                              "top_k": si.top_ks.tolist(), "top_p": si.top_ps.tolist(), "min_p": si.min_ps.tolist(),
                              "flashinfer": b64(fi), "pytorch_min_p": b64(pt)})
    _dump("sampling.json", {"source": "reference selfspec_sampling.py (penalize_rows, cumulate_block, "
                                      "joint_top_k_top_p, torch_backend_filter, min_p_filter, verify_target_probs)",
                            "encoding": "float tensors: base64 of little-endian float32, row-major", **out})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("GRAVITYOCR_REF"),
                    help="path of the GravityOCR source tree (or set GRAVITYOCR_REF)")
    ap.add_argument("--only", default="commit_kernel,commit_rules,sampling," +
                    ",".join(f"natcache_{c}" for c in NATCACHE_CASES))
    a = ap.parse_args()
    if not a.ref or not os.path.isdir(a.ref):
        ap.error("--ref (or GRAVITYOCR_REF) must name the GravityOCR source tree")
    only = a.only.split(",")
    if "commit_rules" in only:
        gen_commit_rules(a.ref)
    if "commit_kernel" in only:
        gen_commit_kernel(a.ref)
    if "sampling" in only:
        gen_sampling(a.ref)
    for case in NATCACHE_CASES:
        if f"natcache_{case}" in only:
            gen_natcache(a.ref, case)


if __name__ == "__main__":
    main()
