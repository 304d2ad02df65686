"""Minimal stand-ins for the SGLang scheduler objects the self-spec worker reads (duck typed: SGLang's own
``ScheduleBatch`` / ``Req`` / ``GenerationBatchResult`` work the same way).  Finish semantics of ``Req.check_finished``
follow SGLang's order for requests without grammar or stop strings: length, then stop token, then vocab boundary."""
from __future__ import annotations

import enum
from dataclasses import dataclass, field
from typing import List, Optional

import torch


class ForwardMode(enum.Enum):
    EXTEND = 1
    DECODE = 2

    def is_extend(self) -> bool:
        return self is ForwardMode.EXTEND


@dataclass
class SamplingParams:
    """SGLang's per-request sampling fields the round reads (temperature 0 = greedy)."""
    max_new_tokens: int = 128
    ignore_eos: bool = False
    stop_token_ids: Optional[List[int]] = None
    stop_strs: Optional[List[str]] = None
    stop_regex_strs: Optional[List[str]] = None
    temperature: float = 0.0
    top_p: float = 1.0
    top_k: int = -1
    min_p: float = 0.0
    repetition_penalty: float = 1.0
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0
    min_new_tokens: int = 0
    logit_bias: Optional[dict] = None
    # f(logits [n, vocab] fp32, params list) -> logits: SGLang's custom logit processor interface; each param dict
    # carries "__req__" (a read-only request view whose output_ids hold the row's prefix)
    custom_logit_processor: Optional[object] = None
    custom_params: Optional[dict] = None


@dataclass
class FinishReason:
    kind: str
    matched: Optional[int] = None


class Req:
    """One request: an image-embedding prefix plus prompt ids (vision and tokenizer stay outside this path)."""

    def __init__(self, rid, image_embeds: torch.Tensor, prompt_ids, sampling_params: SamplingParams,
                 vocab_size: int, eos_token_ids=None):
        self.rid = rid
        self.image_embeds = image_embeds
        self.origin_input_ids = [-1] * image_embeds.shape[0] + [int(t) for t in prompt_ids]
        self.sampling_params = sampling_params
        self.vocab_size = vocab_size
        self.eos_token_ids = set(eos_token_ids or ())
        self.tokenizer = None
        self.grammar = None
        self.to_finish = None
        self.output_ids: List[int] = []
        self.finished_reason: Optional[FinishReason] = None
        self.spec_verify_ct = 0
        self.spec_accepted_tokens = 0
        self.hist: List[int] = []
        self._spec_seed_ready = False
        # multimodal (t, h, w) positions [3, prefix length] of the prefix (image tokens on a grid), or None for 1-D
        self.mrope_positions = None

    def prefix_rows(self, engine):
        ids = torch.tensor(self.origin_input_ids, dtype=torch.int64)
        img = self.image_embeds.float().cpu()
        tok = ids[img.shape[0]:]
        emb = engine.w.embed[tok.to(engine.device)].float().cpu()
        return torch.cat([img, emb], 0), ids

    def finished(self) -> bool:
        return self.finished_reason is not None

    def update_spec_acceptance_histogram(self, a: int) -> None:
        self.hist.append(a)

    def check_finished(self, new_accepted_len: int = 1) -> None:
        if self.finished():
            return
        if self.to_finish is not None:
            self.finished_reason, self.to_finish = self.to_finish, None
            return
        if len(self.output_ids) >= self.sampling_params.max_new_tokens:
            self.finished_reason = FinishReason("length")
            return
        sp = self.sampling_params
        stop = set() if sp.ignore_eos else (set(sp.stop_token_ids or ()) | self.eos_token_ids)
        for t in self.output_ids[-new_accepted_len:]:
            if t in stop:
                self.finished_reason = FinishReason("stop", t)
                return
            if t > self.vocab_size or t < 0:
                self.finished_reason = FinishReason("vocab", t)
                return


@dataclass
class ScheduleBatch:
    reqs: List[Req]
    req_pool_indices: torch.Tensor
    seq_lens: torch.Tensor
    forward_mode: ForwardMode = ForwardMode.EXTEND
    seq_lens_cpu: Optional[torch.Tensor] = None

    def batch_size(self) -> int:
        return len(self.reqs)


@dataclass
class GenerationBatchResult:
    logits_output: object = None
    next_token_ids: Optional[torch.Tensor] = None
    num_accepted_tokens: int = 0
    accept_length_per_req_cpu: Optional[List[int]] = None
    accept_lens: Optional[torch.Tensor] = None
    can_run_cuda_graph: bool = True
    next_token_ids_cpu: Optional[List[List[int]]] = None
    finish_checked: bool = False
