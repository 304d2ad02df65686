"""In-process drop-in for the reference's ``generate_speculative_natcache`` (``src/fast_sampling.py:425-628``), the
entry ``src/infer_omnidocbench.py:433-459`` (``--spec_natcache``, ``make_sampler``) calls as

    txt, s = generate_speculative_natcache(model, crop, prompt=prompt, max_new_tokens=mnt, temperature=...,
                                           top_p=..., max_long_side=..., draft_steps=..., return_stats=True, trace=tr)

Same signature, the same rounds and the same return contract: text, or (text, stats) with ``return_stats``; one dict
per round appended to ``trace`` with the reference's keys (``round``, ``k``, ``draft``, ``ar_pred``, ``new_tokens``).

``model`` is either the reference's own ``GlmOcrBlockDiffusion`` (the object ``make_sampler`` holds: ``processor``,
``tokenizer``, ``mm_model``, ``text_model``, ``glm.lm_head``, ``bd_size``, ``mask_id``, ``image_token_id``) or a
``SelfSpecModel`` around an ``Engine``.  For the reference model the decoder weights are copied once into an Engine on
the model's GPU (``attach_engine``); the crop goes through the caller's own processor and vision tower
(``get_image_features``, ``get_rope_index``, as ``:456-488`` does) and the image embeddings are injected at the
image-token rows; 2-D multimodal positions of the image tokens go to the prefill's RoPE, and response token r sits at
max position + 1 + r (``comb_pos``, :505-506).  ``image`` may also be the image-embedding prefix itself (tensor
[n_image, hidden], or an object with ``.embeds`` and ``.positions``).

The rounds are the reference's, on the CUDA path:
  * round 0 (no pending token): draft over B mask rows that all see each other (the draft mask of ``:508-510`` with
    ``pre = 0``); the draft is [a0, d1..dB] with a0 the prefill's argmax; causal verify over it (``:561-575``);
  * rounds 1+: the pending token plus B masks (pending causal, masks bidirectional), causal verify over
    [a0, d1..dB] with the pending token's K/V kept from the draft -- the served full-draft round, replayed from one
    CUDA graph per (B, request capacity);
  * accept: the leading drafts equal to the verify argmax; commit [draft[:k], ar_pred[k]] or the full draft plus the
    bonus token (``:577-605``).
So the committed stream is AR greedy and, with equal arithmetic, the trace and stats are the reference's.

Options that only change what is drafted (``temperature``, ``top_p``, ``draft_threshold``, ``draft_steps``,
``full_draft``) leave the committed text unchanged, because the reference's verify is always the causal argmax: the
CUDA path drafts greedily in one step with the full draft and commits the same text.  ``accept_conf > 0`` accepts
drafts that are not the argmax and changes the text, so it raises ``ValueError``; the reference's caller catches any
exception and falls back.
"""
from __future__ import annotations

import re
from typing import Dict, List, Optional

import torch

from .. import _lib as L
from ..config import ModelConfig
from ..engine import Engine


class SelfSpecModel:
    """The handles natcache reads from the reference's ``GlmOcrBlockDiffusion`` (bd_size, mask_id, tokenizer), around
    an ``Engine`` holding the decoder on one GPU."""

    def __init__(self, engine: Engine, bd_size: int = 16, tokenizer=None, image_token_id: Optional[int] = None):
        self.engine = engine
        self.bd_size = bd_size
        self.mask_id = engine.cfg.mask_id
        self.tokenizer = tokenizer
        self.image_token_id = engine.cfg.image_token_id if image_token_id is None else image_token_id
        self._rb: Dict[tuple, object] = {}

    def round_buffers(self, K: int, pages: int, max_len: int, avg_len: int):
        key = (K, pages)
        rb = self._rb.get(key)
        if rb is None:
            eng = self.engine
            eng.reserve(K)
            rb = eng.new_round_buffers(1, K, pages, max_len=max_len, avg_len=avg_len)
            rb.page_table[0] = torch.tensor(eng.pool.alloc(pages), dtype=torch.int32, device=eng.device)
            rb.graph = None
            rb.host = torch.zeros_like(rb.readback, device="cpu").pin_memory()
            rb.event = torch.cuda.Event()
            rb.tmp_idx = torch.zeros((K,), dtype=torch.int32, device=eng.device)
            rb.ids64 = torch.zeros((K,), dtype=torch.int64, device=eng.device)
            self._rb[key] = rb
        return rb


# ---------------------------------------------------------------------- the reference model -> an engine
def _text_config(model) -> ModelConfig:
    tc = model.text_model.config
    rp = getattr(tc, "rope_parameters", None) or {}
    head_dim = int(getattr(tc, "head_dim", None) or tc.hidden_size // tc.num_attention_heads)
    factor = float(rp.get("partial_rotary_factor", getattr(tc, "partial_rotary_factor", 1.0)))
    return ModelConfig(n_layers=int(tc.num_hidden_layers), hidden=int(tc.hidden_size),
                       n_q_heads=int(tc.num_attention_heads), n_kv_heads=int(tc.num_key_value_heads),
                       head_dim=head_dim, intermediate=int(tc.intermediate_size), vocab=int(tc.vocab_size),
                       rms_eps=float(tc.rms_norm_eps), rope_theta=float(rp.get("rope_theta", 10000.0)),
                       rotary_dim=int(head_dim * factor), mask_id=int(model.mask_id),
                       image_token_id=int(model.image_token_id),
                       mrope_section=tuple(int(x) for x in rp.get("mrope_section", (8, 12, 12))))


def _text_weights(model) -> Dict[str, torch.Tensor]:
    """transformers GlmOcrTextModel parameter names -> this package's (``weights.weight_shapes``)."""
    tm = model.text_model
    w = {"embed_tokens": tm.embed_tokens.weight, "norm": tm.norm.weight, "lm_head": model.glm.lm_head.weight}
    for l, layer in enumerate(tm.layers):
        p = f"layers.{l}."
        at, mlp = layer.self_attn, layer.mlp
        w.update({p + "q_proj": at.q_proj.weight, p + "k_proj": at.k_proj.weight, p + "v_proj": at.v_proj.weight,
                  p + "o_proj": at.o_proj.weight, p + "gate_up_proj": mlp.gate_up_proj.weight,
                  p + "down_proj": mlp.down_proj.weight, p + "input_layernorm": layer.input_layernorm.weight,
                  p + "post_self_attn_layernorm": layer.post_self_attn_layernorm.weight,
                  p + "post_attention_layernorm": layer.post_attention_layernorm.weight,
                  p + "post_mlp_layernorm": layer.post_mlp_layernorm.weight})
    return {k: v.detach() for k, v in w.items()}


def attach_engine(model, max_context: int = 16384, device: Optional[torch.device] = None) -> SelfSpecModel:
    """Copy the reference model's decoder weights (bf16) into an Engine on `device` (default: the model's device if
    it is a GPU, else the current GPU) and keep it on the model as ``model.gr_engine``.  Pages for one request of up to
    `max_context` tokens per distinct block size."""
    cfg = _text_config(model)
    if device is None:
        d = next(model.parameters()).device
        device = d if d.type == "cuda" else torch.device("cuda", torch.cuda.current_device())
    pages = 4 * ((max_context + 15) // 16) + 16
    eng = Engine(cfg, _text_weights(model), max_rows=64, n_pages=pages, device=device)
    sm = SelfSpecModel(eng, bd_size=int(model.bd_size), tokenizer=getattr(model, "tokenizer", None),
                       image_token_id=cfg.image_token_id)
    model.gr_engine = sm
    return sm


def _resolve(model) -> SelfSpecModel:
    if isinstance(model, SelfSpecModel):
        return model
    sm = getattr(model, "gr_engine", None)
    return sm if sm is not None else attach_engine(model)


# ---------------------------------------------------------------------- the prefix
def _prefix_from_embeds(sm: SelfSpecModel, image, prompt):
    """image: the image-embedding prefix [n_image, hidden], or an object with ``.embeds`` and optionally
    ``.positions`` (int [3, n_image + n_prompt] multimodal positions of the whole prefix)."""
    eng = sm.engine
    img = getattr(image, "embeds", image)
    if img.dim() != 2 or img.shape[1] != eng.cfg.hidden:
        raise ValueError(f"image must be the image-embedding prefix [n_image, {eng.cfg.hidden}]")
    if isinstance(prompt, str):
        if sm.tokenizer is None or not hasattr(sm.tokenizer, "encode"):
            raise ValueError("a text prompt needs model.tokenizer; pass prompt token ids instead")
        prompt = sm.tokenizer.encode(prompt)
    ids = torch.as_tensor(prompt, dtype=torch.int64).view(-1)
    emb = eng.w.embed[ids.to(eng.device)].float().cpu()
    x = torch.cat([img.float().cpu(), emb], dim=0)
    pid = torch.cat([torch.full((img.shape[0],), -1, dtype=torch.int64), ids])
    pos = getattr(image, "positions", None)
    return x, pid, (None if pos is None else _pos3_or_none(torch.as_tensor(pos), x.shape[0]))


def _pos3_or_none(pos: torch.Tensor, P: int) -> Optional[torch.Tensor]:
    """[3, P] multimodal positions, or None when they are the plain 0..P-1 on every axis."""
    pos = pos.reshape(3, -1)[:, :P].to(torch.int64).cpu()
    plain = torch.arange(P)
    if all(torch.equal(pos[a], plain) for a in range(3)):
        return None
    return pos


def _prefix_from_processor(model, sm: SelfSpecModel, image, prompt, max_long_side):
    """The reference's own preprocessing (``src/fast_sampling.py:456-488``) through the caller's model: resize, chat
    template, processor, vision tower, M-RoPE index; image embeddings replace the image-token rows."""
    from PIL import Image
    eng = sm.engine
    if image.mode != "RGB":
        image = image.convert("RGB")
    w, h = image.size
    if max(w, h) > max_long_side:
        s = max_long_side / max(w, h)
        image = image.resize((int(w * s), int(h * s)), Image.LANCZOS)
    msgs = [{"role": "user", "content": [{"type": "image"}, {"type": "text", "text": prompt}]}]
    text = model.processor.apply_chat_template(msgs, add_generation_prompt=True, tokenize=False)
    enc = model.processor(text=[text], images=[image], return_tensors="pt")
    dev = next(model.parameters()).device
    enc = enc.to(dev) if hasattr(enc, "to") else enc
    input_ids = enc["input_ids"]
    pixel_values, thw = enc.get("pixel_values"), enc.get("image_grid_thw")
    ids = input_ids[0].to(torch.int64).cpu()
    P = ids.shape[0]
    pos, _ = model.mm_model.get_rope_index(input_ids, enc["mm_token_type_ids"], image_grid_thw=thw,
                                           video_grid_thw=None,
                                           attention_mask=torch.ones((1, P), dtype=torch.long, device=dev))
    pos3 = _pos3_or_none(pos, P)
    img_rows = ids == sm.image_token_id
    x = eng.w.embed[ids.clamp(min=0).to(eng.device)].float().cpu()
    pid = ids.clone()
    if pixel_values is not None and bool(img_rows.any()):
        feats = model.mm_model.get_image_features(pixel_values, thw, return_dict=True).pooler_output
        emb = torch.cat(list(feats), dim=0).float().cpu()
        if emb.shape[0] != int(img_rows.sum()):
            raise ValueError(f"{emb.shape[0]} image embeddings for {int(img_rows.sum())} image tokens")
        x[img_rows] = emb
        pid[img_rows] = -1
    return x, pid, pos3


# ---------------------------------------------------------------------- the rounds
def _first_round(eng: Engine, rb, bd: int) -> None:
    """Round 0 of the reference (no pending token; a0 = the prefill's argmax, held in the seed pool): draft over B
    mask rows at positions S..S+B-1, every row seeing the whole block; draft = [a0, argmax of the B rows]; causal verify
    over the draft at positions S..S+B; accept and commit with a0 counted as a verify row (K/V kept for a0, d1..d_acc)."""
    K = bd + 1
    cfg = eng.cfg
    rb.ids64[:bd].fill_(cfg.mask_id)
    eng.forward(L.ROWS_EXPLICIT, 1, bd, rb.seq_lens, rb.page_table, out_idx=rb.tmp_idx, ids64=rb.ids64[:bd],
                attn_chunk=rb.attn_chunk, attn_splits=rb.attn_splits, status=rb.status, attn_draft=2,
                rope_delta=rb.pos_delta)
    rb.am[0:1].copy_(rb.seeds[rb.rpi[0:1]])
    rb.am[1:K].copy_(rb.tmp_idx[:bd])
    rb.ids64.copy_(rb.am)
    eng.forward(L.ROWS_EXPLICIT, 1, K, rb.seq_lens, rb.page_table, out_idx=rb.v, out_top1=rb.top_v,
                out_gap=rb.gap_v, ids64=rb.ids64, attn_chunk=rb.attn_chunk, attn_splits=rb.attn_splits,
                status=rb.status, attn_draft=0, rope_delta=rb.pos_delta)
    L.accept_commit(1, K, rb.am, rb.v, rb.seeds, rb.rpi, rb.seq_lens, rb.packed, rb.released, rb.out_next,
                    x0_committed=True, n_released=rb.n_released, n_committed=rb.n_committed, rounds=rb.rounds,
                    accept_len=rb.accept_len)


def _read_round(rb, K: int):
    rb.host.copy_(rb.readback, non_blocking=True)
    rb.event.record()
    rb.event.synchronize()
    h = rb.host
    st = int(h[K + 2 + 1])
    if st:
        raise RuntimeError(f"device status {st}: {L.load().gr_status_string(st).decode()}")
    return h[: K + 2].tolist()


@torch.no_grad()
def generate_speculative_natcache(model, image, prompt="Text Recognition:", max_new_tokens=512,
                                  draft_threshold=0.9, temperature=0.0, top_p=0.95, max_long_side=1344,
                                  accept_conf=0.0, draft_steps=1, return_stats=False, trace=None, draft_bd=None,
                                  full_draft=True):
    if accept_conf > 0:
        raise ValueError("accept_conf > 0 commits drafts that are not the verify argmax; not on the CUDA path")
    sm = _resolve(model)
    eng = sm.engine
    if int(getattr(model, "mask_id", sm.mask_id)) != eng.cfg.mask_id:
        raise ValueError(f"mask id {model.mask_id} != the engine's {eng.cfg.mask_id}")
    bd = int(draft_bd) if draft_bd else int(getattr(model, "bd_size", sm.bd_size))
    K = bd + 1
    if torch.is_tensor(getattr(image, "embeds", image)):
        x, pid, pos3 = _prefix_from_embeds(sm, image, prompt)
    else:
        x, pid, pos3 = _prefix_from_processor(model, sm, image, prompt, max_long_side)
    P = x.shape[0]
    max_len = P + max_new_tokens + 2 * K + 64
    pages = eng.pages_for(max_len)
    rb = sm.round_buffers(K, pages, max_len, P + max_new_tokens // 2)
    eng.prefill(rb, [x], [pid], prefix_pos3=[pos3])
    tok = getattr(model, "tokenizer", None) or sm.tokenizer
    eos = getattr(tok, "eos_token_id", None) if tok is not None else None
    committed: List[int] = []
    n_rounds = n_acc = 0
    done = False
    while not done and len(committed) < max_new_tokens:
        if n_rounds == 0:
            _first_round(eng, rb, bd)
        else:
            if rb.graph is None:
                # captured once per (K, pages): replays read the device-resident lengths / seeds / page table
                snap = (rb.seq_lens.clone(), rb.seeds.clone(), rb.n_committed.clone(), rb.rounds.clone())
                eng.round_launch(rb)
                torch.cuda.synchronize()
                for t, s0 in zip((rb.seq_lens, rb.seeds, rb.n_committed, rb.rounds), snap):
                    t.copy_(s0)
                rb.graph = eng.capture(rb)
            rb.graph.replay()
        row = _read_round(rb, K)
        acc = row[1]
        new = [row[0]] + row[2: 3 + acc]
        n_rounds += 1
        n_acc += len(new)
        if trace is not None:
            am = rb.am[:K].tolist()
            v = rb.v[:K].tolist()
            trace.append({"round": n_rounds, "k": acc + 1, "draft": am, "ar_pred": [am[0]] + v[: K - 1],
                          "new_tokens": new})
        committed += new
        if eos is not None and eos in new:
            done = True
    gen = committed
    if eos is not None and eos in gen:
        gen = gen[: gen.index(eos)]
    txt = gen
    if tok is not None and hasattr(tok, "decode"):
        txt = ""
        if gen:
            txt = re.sub(r"<think>.*?</think>\s*", "", tok.decode(gen, skip_special_tokens=True), flags=re.S)
    if return_stats:
        fwd = 2 * n_rounds
        return txt, {"rounds": n_rounds, "draft_fwd": n_rounds, "verify_fwd": n_rounds, "commit_fwd": 0,
                     "total_fwd": fwd, "resp_tokens": len(gen), "tokens_per_fwd": round(len(gen) / max(1, fwd), 3),
                     "accept_per_round": round(n_acc / max(1, n_rounds), 2)}
    return txt
