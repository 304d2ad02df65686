"""Host side of non-greedy rounds: sampling parameters, penalizer state, grammar masks, and the sampled round.

A batch is *plain* when every request is greedy and nothing else changes its logits (no penalty, logit bias, grammar
or custom logit processor); a plain batch runs the greedy round unchanged (argmax fused into lm_head, one CUDA graph).
Any other batch runs the round below (the reference's non-plain path: ``selfspec_diffusion_worker.py:504-528``
``_sample_a0``, ``selfspec_fast_commit.py:150-230`` ``verify_logits`` / ``process_verify_logits`` /
``sampling_verify``, ``selfspec_sampling.py``):

  draft   the draft forward as usual (argmax of the mask rows = the drafts d1..dB); the boundary rows' lm_head writes
          fp32 logits, which get AR's logits processing (penalties of every committed token, the grammar mask of the
          request's current state, logit bias, custom logit processors) and a0 is drawn from AR's target distribution;
          a0 is cumulated into the penalizer state;
  verify  the causal verify forward over [a0, d1..dB]; lm_head writes fp32 logits of every row; row j gets the
          processing AR decode gives the token after cand[0..j] (penalties of the committed tokens plus d1..dj, the
          grammar mask after a0, d1..dj); AR's target distribution per row; d_{j+1} is accepted with probability
          p_j(d_{j+1}); at the first rejection a token is drawn from p_j without d_{j+1}, or the bonus from the last
          row; the commit and the penalizer cumulation of the verified tokens follow on the device.

Coins are Philox-4x32-10 draws keyed by this state's seed and a device-resident round counter (advanced by the
commit), so a sampled round needs no host sync before its commit readback and can replay from a CUDA graph once the
host has written the batch's parameter and mask buffers.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence

import torch

from . import _lib as L

TOP_K_ALL = 1 << 30
# SGLang's penalizers in the order its orchestrator holds them (SamplingBatchInfo builds it from this set)
DEFAULT_ORDER = (L.PEN_FREQUENCY, L.PEN_MIN_NEW_TOKENS, L.PEN_PRESENCE, L.PEN_REPETITION)
PENALIZER_NAMES = {"BatchedRepetitionPenalizer": L.PEN_REPETITION, "BatchedFrequencyPenalizer": L.PEN_FREQUENCY,
                   "BatchedPresencePenalizer": L.PEN_PRESENCE, "BatchedMinNewTokensPenalizer": L.PEN_MIN_NEW_TOKENS}


@dataclass
class RequestSampling:
    """One request's sampling settings, normalised as SGLang's SamplingParams normalises them (a temperature below
    1e-6 means greedy: temperature 1, top_k 1; top_k <= 0 means every token)."""

    temperature: float = 0.0
    top_k: int = -1
    top_p: float = 1.0
    min_p: float = 0.0
    repetition_penalty: float = 1.0
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0
    min_new_tokens: int = 0
    stop_ids: Sequence[int] = ()
    logit_bias: Optional[Dict[int, float]] = None

    @staticmethod
    def of(sp, stop_ids: Sequence[int] = ()) -> "RequestSampling":
        g = lambda n, d: getattr(sp, n, d) if getattr(sp, n, None) is not None else d
        return RequestSampling(float(g("temperature", 0.0)), int(g("top_k", -1)), float(g("top_p", 1.0)),
                               float(g("min_p", 0.0)), float(g("repetition_penalty", 1.0)),
                               float(g("frequency_penalty", 0.0)), float(g("presence_penalty", 0.0)),
                               int(g("min_new_tokens", 0)), tuple(stop_ids), g("logit_bias", None))

    def normalised(self):
        T, k = self.temperature, self.top_k
        if T < 1e-6:
            T, k = 1.0, 1
        if k <= 0:
            k = TOP_K_ALL
        return T, k

    @property
    def greedy(self) -> bool:
        return self.normalised()[1] == 1

    @property
    def plain(self) -> bool:
        return (self.greedy and self.repetition_penalty == 1.0 and self.frequency_penalty == 0.0 and
                self.presence_penalty == 0.0 and self.min_new_tokens <= 0 and not self.logit_bias)


class SamplerState:
    """Penalizer state by request pool slot, the coins' rng and the per-batch buffers of one engine.  `filter` names
    the sampling backend: FILTER_JOINT for flashinfer (a batch with min-p then takes FILTER_SEQUENTIAL, as SGLang's
    flashinfer path does), FILTER_TORCH for the "pytorch" backend."""

    def __init__(self, vocab: int, pool_size: int, device, seed: int = 0, filter: int = L.FILTER_JOINT,
                 order: Sequence[int] = DEFAULT_ORDER):
        self.vocab, self.pool_size, self.device = vocab, pool_size, torch.device(device)
        self.filter = filter
        self.order = tuple(order)
        f32 = dict(dtype=torch.float32, device=self.device)
        self.st_rep = torch.ones((pool_size, vocab), **f32)
        self.st_freq = torch.zeros((pool_size, vocab), **f32)
        self.st_pres = torch.zeros((pool_size, vocab), **f32)
        self.st_len = torch.zeros((pool_size,), dtype=torch.int32, device=self.device)
        self.rng = torch.tensor([seed & ((1 << 63) - 1), 0], dtype=torch.int64, device=self.device)
        self._keep: List[torch.Tensor] = []

    def reset_slot(self, slot: int) -> None:
        """A new request in this pool slot: no token seen yet."""
        self.st_rep[slot].fill_(1.0)
        self.st_freq[slot].zero_()
        self.st_pres[slot].zero_()
        self.st_len[slot] = 0

    def batch(self, reqs: Sequence[RequestSampling], rpi: torch.Tensor, allowed: Optional[torch.Tensor] = None
              ) -> L.Sampling:
        """The gr_sampling block of a batch (rpi: device int64 pool slots in batch order).  The arrays it points to
        are kept alive until the next call."""
        dev, bs = self.device, len(reqs)
        norm = [r.normalised() for r in reqs]
        t = lambda xs, dt: torch.tensor(xs, dtype=dt, device=dev)
        arrays = {
            "temperature": t([T for T, _ in norm], torch.float32),
            "top_k": t([min(k, TOP_K_ALL) for _, k in norm], torch.int32),
            "top_p": t([r.top_p for r in reqs], torch.float32),
            "min_p": t([r.min_p for r in reqs], torch.float32),
            "repetition": t([r.repetition_penalty for r in reqs], torch.float32),
            "frequency": t([r.frequency_penalty for r in reqs], torch.float32),
            "presence": t([r.presence_penalty for r in reqs], torch.float32),
            "min_new_tokens": t([r.min_new_tokens for r in reqs], torch.int32),
        }
        n_stop = max([len(r.stop_ids) for r in reqs] + [1])
        stops = torch.full((bs, n_stop), -1, dtype=torch.int32)
        for i, r in enumerate(reqs):
            if r.stop_ids:
                stops[i, : len(r.stop_ids)] = torch.tensor(list(r.stop_ids), dtype=torch.int32)
        arrays["stop_ids"] = stops.to(dev)
        bias = None
        if any(r.logit_bias for r in reqs):
            bias = torch.zeros((bs, self.vocab), dtype=torch.float32)
            for i, r in enumerate(reqs):
                for tok, v in (r.logit_bias or {}).items():
                    bias[i, int(tok)] = float(v)
            bias = bias.to(dev)
        used = {L.PEN_REPETITION: any(r.repetition_penalty != 1.0 for r in reqs),
                L.PEN_FREQUENCY: any(r.frequency_penalty != 0.0 for r in reqs),
                L.PEN_PRESENCE: any(r.presence_penalty != 0.0 for r in reqs),
                L.PEN_MIN_NEW_TOKENS: any(r.min_new_tokens > 0 for r in reqs)}
        order = [op for op in self.order if used[op]]
        s = L.Sampling()
        s.vocab = self.vocab
        # the flashinfer backend switches to renorm-then-min-p as soon as one request of the batch uses min-p
        # (verify_target_probs, selfspec_sampling.py:278-282)
        s.filter = L.FILTER_SEQUENTIAL if self.filter == L.FILTER_JOINT and any(r.min_p > 0 for r in reqs) \
            else self.filter
        for k, v in arrays.items():
            setattr(s, k, v.data_ptr())
        s.n_order = len(order)
        for i, op in enumerate(order):
            s.order[i] = op
        s.n_stop = n_stop
        s.st_rep, s.st_freq, s.st_pres = self.st_rep.data_ptr(), self.st_freq.data_ptr(), self.st_pres.data_ptr()
        s.st_len = self.st_len.data_ptr()
        s.req_pool_idx = rpi.data_ptr()
        s.allowed = 0 if allowed is None else allowed.data_ptr()
        s.logit_bias = 0 if bias is None else bias.data_ptr()
        s.rng = self.rng.data_ptr()
        self._keep = list(arrays.values()) + [rpi] + [x for x in (allowed, bias) if x is not None]
        return s


# ---------------------------------------------------------------------- grammar masks
def mask_words(vocab: int) -> int:
    return (vocab + 31) // 32


def pack_allowed(allowed: torch.Tensor) -> torch.Tensor:
    """bool [rows, vocab] -> int32 [rows, ceil(vocab / 32)] bit masks (bit v % 32 of word v / 32 set = allowed)."""
    rows, V = allowed.shape
    W = mask_words(V)
    pad = torch.zeros((rows, W * 32), dtype=torch.bool)
    pad[:, :V] = allowed.cpu()
    bits = pad.view(rows, W, 32).to(torch.int64) << torch.arange(32, dtype=torch.int64)
    words = bits.sum(-1)
    return torch.where(words >= (1 << 31), words - (1 << 32), words).to(torch.int32)


def verify_row_masks(grammars: Sequence, cand: torch.Tensor, vocab: int) -> Optional[torch.Tensor]:
    """Allowed-token masks of the verify rows (bool [bs*K, vocab]) or None when no request has a grammar.
    Row j of request i allows what its grammar allows after a0, d1..dj; the walk stops at the first draft its parent
    row does not allow (later rows stay all-allowed, they are never reached) and every token it accepted is rolled
    back (the grammar leaves as it came; ``selfspec_sampling.fulldraft_bitmask``).  A grammar object needs
    ``allowed_tokens() -> bool [vocab]``, ``accept_token(id)`` (ValueError on rejection) and ``rollback(n)``."""
    if not any(g is not None for g in grammars):
        return None
    bs, K = cand.shape
    out = torch.ones((bs * K, vocab), dtype=torch.bool)
    c = cand.tolist()
    for i, g in enumerate(grammars):
        if g is None or getattr(g, "finished", False):
            continue
        n = 0
        try:
            g.accept_token(int(c[i][0]))
            n = 1
            for j in range(K):
                row = g.allowed_tokens()
                out[i * K + j] = row
                if j + 1 >= K or not bool(row[int(c[i][j + 1])]):
                    break
                g.accept_token(int(c[i][j + 1]))
                n += 1
        except ValueError:
            pass
        finally:
            if n:
                g.rollback(n)
    return out


def current_masks(grammars: Sequence, vocab: int) -> Optional[torch.Tensor]:
    """Allowed-token masks of each request's current grammar state (bool [bs, vocab]) or None."""
    if not any(g is not None for g in grammars):
        return None
    out = torch.ones((len(grammars), vocab), dtype=torch.bool)
    for i, g in enumerate(grammars):
        if g is not None and not getattr(g, "finished", False):
            out[i] = g.allowed_tokens()
    return out


# ---------------------------------------------------------------------- the sampled round on an engine
class SampledRound:
    """Buffers and launches of a non-greedy round for one (B, batch) of an Engine."""

    def __init__(self, engine, rb):
        self.eng, self.rb = engine, rb
        bs, K, V, H = rb.bs, rb.K, engine.cfg.vocab, engine.cfg.hidden
        dev = engine.device
        self.logits = torch.empty((bs * K, V), dtype=torch.float32, device=dev)
        self.x_first = torch.empty((bs, H), dtype=torch.bfloat16, device=dev)
        self.first = torch.zeros((bs,), dtype=torch.int32, device=dev)
        self.accept = torch.zeros((bs * K,), dtype=torch.int32, device=dev)
        self.sample = torch.zeros((bs * K,), dtype=torch.int32, device=dev)
        self.p_next = torch.zeros((bs * K,), dtype=torch.float32, device=dev)

    def _lm_head_f32(self, x: torch.Tensor, m: int, out: torch.Tensor) -> None:
        e = L.Epilogue()
        e.mode = L.EPI_STORE_F32
        e.out = out.data_ptr()
        e.ld_out = self.eng.cfg.vocab
        self.eng.reserve(m)
        L.linear(self.eng.w.lm_head, x, m, e, self.eng.lin_ws, status=self.rb.status)

    def draft(self, smp: L.Sampling, custom: Optional[Callable[[torch.Tensor], None]] = None) -> None:
        """Draft forward, then a0 drawn from AR's distribution of the boundary rows (written into am[:, 0])."""
        eng, rb = self.eng, self.rb
        bs, K = rb.bs, rb.K
        eng.draft_launch(rb)
        L.gather_rows(eng.x, bs, K, self.x_first)
        lg = self.logits[:bs]
        self._lm_head_f32(self.x_first, bs, lg)
        L.logits_process(lg, bs, 1, None, smp)
        if custom is not None:
            custom(lg)
        L.sample_rows(lg, bs, 1, None, smp, L.COIN_FIRST, None, self.first, first_out=rb.am, first_stride=K,
                      status=rb.status)
        L.penalty_cumulate(bs, rb.am, K, None, 1, smp)

    def verify(self, smp: L.Sampling, rng: torch.Tensor,
               custom: Optional[Callable[[torch.Tensor], None]] = None) -> None:
        """Causal verify forward, AR's distribution of every row, the speculative decision and the commit."""
        eng, rb = self.eng, self.rb
        bs, K = rb.bs, rb.K
        eng.forward(L.ROWS_VERIFY, bs, K, rb.seq_lens, rb.page_table, out_idx=rb.v, ids32=rb.am,
                    attn_chunk=rb.attn_chunk, attn_splits=rb.attn_splits, status=rb.status, order=rb.order,
                    head=False, rope_delta=rb.pos_delta)
        self._lm_head_f32(eng.x, bs * K, self.logits)
        L.logits_process(self.logits, bs, K, rb.am, smp)
        if custom is not None:
            custom(self.logits)
        L.sample_rows(self.logits, bs, K, rb.am, smp, L.COIN_FIRST, self.accept, self.sample, self.p_next,
                      status=rb.status)
        L.commit_sampled(bs, K, rb.am, self.accept, self.sample, rb.seeds, rb.rpi, rb.seq_lens, rb.v, rb.packed,
                         rb.released, rb.out_next, n_released=rb.n_released, n_committed=rb.n_committed,
                         rounds=rb.rounds, accept_len=rb.accept_len, rng=rng)
        L.penalty_cumulate(bs, rb.v, K, rb.accept_len, 1, smp)


def first_tokens(engine, rows: torch.Tensor, n: int, smp: L.Sampling, status=None,
                 custom: Optional[Callable[[torch.Tensor], None]] = None) -> torch.Tensor:
    """The prefill's first token of n requests (rows: their normed last prefix rows, bf16 [n, H]) drawn from AR's
    distribution with GR_COIN_PREFILL coins; cumulated into the penalizer state.  Returns int32 [n] on the device."""
    V = engine.cfg.vocab
    lg = torch.empty((n, V), dtype=torch.float32, device=engine.device)
    e = L.Epilogue()
    e.mode = L.EPI_STORE_F32
    e.out = lg.data_ptr()
    e.ld_out = V
    engine.reserve(n)
    L.linear(engine.w.lm_head, rows, n, e, engine.lin_ws, status=status)
    L.logits_process(lg, n, 1, None, smp)
    if custom is not None:
        custom(lg)
    out = torch.zeros((n,), dtype=torch.int32, device=engine.device)
    L.sample_rows(lg, n, 1, None, smp, L.COIN_PREFILL, None, out, status=status)
    L.penalty_cumulate(n, out, 1, None, 1, smp)
    return out


_ = math
