"""In-process drop-in for the reference's ``generate_speculative_natcache`` (``src/fast_sampling.py:425-628``), the
entry ``src/infer_omnidocbench.py:433-459`` (``--spec_natcache``) calls.

Same signature, same greedy full-draft semantics and the same return contract (text, or (text, stats) with
``return_stats``; per-round dicts appended to ``trace``).  The round underneath is the served full-draft round on the
CUDA path (draft [x0 | mask x B], causal verify [a0, d1..dB], accept-and-commit) replayed from one CUDA graph per
(B, batch 1); it commits the same AR-greedy token stream as the reference's natcache round.

What differs, because the vision tower, processor and tokenizer are outside this path:
  * ``image`` is the image-embedding prefix (fp32 / bf16 tensor [n_image, hidden], or an object with ``.embeds``)
    that the reference gets from ``get_image_features`` and injects with ``masked_scatter`` (``:467-488``);
  * ``prompt`` is the prompt token ids (list / 1-D tensor); a str is accepted only when ``model.tokenizer`` can encode
    it;
  * without a tokenizer the "text" is the committed id list.
Unsupported options (sampling, ``accept_conf``, ``draft_steps != 1``, ``full_draft=False``) raise ``ValueError``;
the reference's caller (``make_sampler``) catches exceptions and falls back, so the contract holds.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional

import torch

from ..engine import Engine


class SelfSpecModel:
    """The handles natcache reads from the reference's ``GlmOcrBlockDiffusion`` (bd_size, mask_id, tokenizer), around
    an ``Engine`` holding the decoder on one GPU."""

    def __init__(self, engine: Engine, bd_size: int = 16, tokenizer=None):
        self.engine = engine
        self.bd_size = bd_size
        self.mask_id = engine.cfg.mask_id
        self.tokenizer = tokenizer
        self._rb: Dict[int, object] = {}

    def round_buffers(self, K: int, pages: int, max_len: int, avg_len: int):
        key = (K, pages)
        rb = self._rb.get(key)
        if rb is None:
            eng = self.engine
            eng.reserve(K)
            rb = eng.new_round_buffers(1, K, pages, max_len=max_len, avg_len=avg_len)
            rb.page_table[0] = torch.tensor(eng.pool.alloc(pages), dtype=torch.int32, device=eng.device)
            rb.graph = None
            self._rb[key] = rb
        return rb


def _prefix(model: SelfSpecModel, image, prompt):
    eng = model.engine
    img = getattr(image, "embeds", image)
    if not torch.is_tensor(img) or img.dim() != 2 or img.shape[1] != eng.cfg.hidden:
        raise ValueError(f"image must be the image-embedding prefix [n_image, {eng.cfg.hidden}]")
    if isinstance(prompt, str):
        if model.tokenizer is None or not hasattr(model.tokenizer, "encode"):
            raise ValueError("a text prompt needs model.tokenizer; pass prompt token ids instead")
        prompt = model.tokenizer.encode(prompt)
    ids = torch.as_tensor(prompt, dtype=torch.int64).view(-1)
    emb = eng.w.embed[ids.to(eng.device)].float().cpu()
    x = torch.cat([img.float().cpu(), emb], dim=0)
    pid = torch.cat([torch.full((img.shape[0],), -1, dtype=torch.int64), ids])
    return x, pid


@torch.no_grad()
def generate_speculative_natcache(model: SelfSpecModel, image, prompt="Text Recognition:", max_new_tokens=512,
                                  draft_threshold=0.9, temperature=0.0, top_p=0.95, max_long_side=1344,
                                  accept_conf=0.0, draft_steps=1, return_stats=False, trace=None, draft_bd=None,
                                  full_draft=True):
    if temperature > 0:
        raise ValueError("only greedy decoding (temperature <= 0) is on the CUDA path")
    if accept_conf > 0 or draft_steps != 1 or not full_draft:
        raise ValueError("the CUDA path runs the full-draft round with draft_steps=1 and exact accept")
    eng = model.engine
    bd = int(draft_bd) if draft_bd else model.bd_size
    K = bd + 1
    x, pid = _prefix(model, image, prompt)
    P = x.shape[0]
    max_len = P + max_new_tokens + 2 * K + 64
    pages = eng.pages_for(max_len)
    rb = model.round_buffers(K, pages, max_len, P + max_new_tokens // 2)
    eng.prefill(rb, [x], [pid])
    eos = getattr(model.tokenizer, "eos_token_id", None) if model.tokenizer is not None else None
    committed: List[int] = [int(rb.seeds[0])]
    if rb.graph is None:
        # capture once per (K, pages): replays read the device-resident lengths / seeds / page table
        snap = (rb.seq_lens.clone(), rb.seeds.clone(), rb.n_committed.clone(), rb.rounds.clone())
        eng.round_launch(rb)
        torch.cuda.synchronize()
        rb.seq_lens.copy_(snap[0]); rb.seeds.copy_(snap[1]); rb.n_committed.copy_(snap[2]); rb.rounds.copy_(snap[3])
        rb.graph = eng.capture(rb)
        rb.host = torch.zeros_like(rb.readback, device="cpu").pin_memory()
        rb.event = torch.cuda.Event()
    n_rounds = n_acc = 0
    done = eos is not None and committed[0] == eos
    while not done and len(committed) < max_new_tokens:
        rb.graph.replay()
        rb.host.copy_(rb.readback, non_blocking=True)
        rb.event.record()
        rb.event.synchronize()
        h = rb.host
        st = int(h[K + 2 + 1])
        if st:
            raise RuntimeError(f"device status {st} in the self-spec round")
        row = h[: K + 2].tolist()
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
    if model.tokenizer is not None and hasattr(model.tokenizer, "decode") and gen:
        txt = model.tokenizer.decode(gen, skip_special_tokens=True)
    if return_stats:
        fwd = 2 * n_rounds
        return txt, {"rounds": n_rounds, "draft_fwd": n_rounds, "verify_fwd": n_rounds, "commit_fwd": 0,
                     "total_fwd": fwd, "resp_tokens": len(gen), "tokens_per_fwd": round(len(gen) / max(1, fwd), 3),
                     "accept_per_round": round(n_acc / max(1, n_rounds), 2)}
    return txt


_ = math
