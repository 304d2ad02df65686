"""Drop-in for the served boundary: a ``SelfSpecDiffusionWorker`` with the reference's constructor and hooks
(``patches/sglang/python/sglang/srt/speculative/selfspec_diffusion_worker.py:313-1341``), running the full-draft
round (``SELFSPEC_FULLDRAFT=1``, ``SELFSPEC_FAST_COMMIT=1``, device positions) on the CUDA path.

Hooks kept 1:1 -- ``forward_batch_generation`` (:1127), ``_draft_block`` (:660), ``_fulldraft_verify`` (:822),
``_fast_commit_round`` (:963), ``clear_cache_pool`` / ``update_weights_from_tensor`` (:472-487) and the scheduler
hooks ``ss_bind_scheduler`` / ``ss_release_stash`` (:1001, :1019).

Draft-ahead (``SELFSPEC_DRAFT_AHEAD=1`` or ``draft_ahead=True``; :1000-1125 and ``selfspec_fast_commit.py:357-440``):
when the next scheduler iteration is expected to decode the same batch, a plain round's readback copy is followed at
once by the next round's draft graph (the commit kernel has already advanced the device lengths and seeds), so the GPU
runs it while the host waits for and reads the rows.  The reference replays it only after its host pre-check
``cannot_finish``; here the check runs on the rows afterwards and decides whether the draft is kept, which leaves the
GPU no gap between the verify and the next draft.  The next call with the same batch (same requests, pool slots and
lengths) replays only the verify + commit graph.  Anything else discards the pre-launched draft: a request that can
end this round, ``ss_release_stash`` before a prefill admission, a changed batch, a non-plain batch.
Pages are owned per request here, so a discarded draft frees nothing: its K/V rows sit at positions the next draft
rewrites before anything reads them.  The result carries the reference's contract (:954-961, :990-998): ``next_token_ids`` = the
device next seeds [bs], ``next_token_ids_cpu`` = the committed tokens per request, ``accept_length_per_req_cpu``
= j per request, ``num_accepted_tokens`` = sum(j), ``finish_checked=True``.

Ownership as in the reference: the K/V pages and the request -> page table belong to the target worker (an
``Engine`` plus a ``ReqToPagePool``); the seed pool, the penalizer state and the pinned readback buffer belong to this
worker.  A plain batch (every request greedy; no penalty, logit bias, grammar or custom logit processor: the reference's
``selfspec_sampling.is_plain``) replays the greedy round's CUDA graph; any other batch runs the sampled round of
``gravityocr_b200.sampling`` (a0 drawn as AR decode draws it, speculative sampling of the verify rows against AR's
distribution, penalizer cumulation on the device), with the per-round grammar masks and custom logit processors applied
on the host side of the launches.

SGLang itself is not a dependency: ``ScheduleBatch``-, ``Req``- and ``GenerationBatchResult``-shaped objects are
duck typed; ``gravityocr_b200.compat.types`` provides minimal ones for tests and standalone serving.
"""
from __future__ import annotations

import json
import os
from typing import List, Optional

import torch

from .. import _lib as L
from ..commit_rules import cannot_finish, grammar_accept_or_abort, host_commit, stop_set
from ..engine import Engine
from ..sampling import (RequestSampling, SampledRound, SamplerState, current_masks, first_tokens, pack_allowed,
                        verify_row_masks)
from .types import GenerationBatchResult


def _resolve_block_diffusion(server_args):
    """mask id / bd_size: SELFSPEC_MASK_ID env > <model_path>/block_diffusion.json; neither -> ValueError
    (selfspec_diffusion_worker.py:208-229)."""
    bd_size = None
    path = os.path.join(str(getattr(server_args, "model_path", "")), "block_diffusion.json")
    bd = None
    if os.path.isfile(path):
        with open(path) as f:
            bd = json.load(f)
        bd_size = int(bd["bd_size"]) if "bd_size" in bd else None
    env = os.environ.get("SELFSPEC_MASK_ID", "")
    if env:
        return int(env), bd_size, "env SELFSPEC_MASK_ID"
    if bd is not None and "mask_id" in bd:
        return int(bd["mask_id"]), bd_size, path
    raise ValueError(f"SELFSPEC_DIFFUSION: no mask id — {path} missing/without mask_id and SELFSPEC_MASK_ID unset")


class ReqToPagePool:
    """Request slot -> physical K/V pages (the page-16 counterpart of SGLang's req_to_token pool)."""

    def __init__(self, engine: Engine, size: int, max_context: int):
        self.engine = engine
        self.size = size
        self.pages_per_req = engine.pages_for(max_context)
        self.table = torch.zeros((size, self.pages_per_req), dtype=torch.int32, device=engine.device)
        self.owned: dict = {}

    def assign(self, idx: int) -> None:
        if idx in self.owned:
            return
        pages = self.engine.pool.alloc(self.pages_per_req)
        self.owned[idx] = pages
        self.table[idx] = torch.tensor(pages, dtype=torch.int32, device=self.engine.device)

    def release(self, idx: int) -> None:
        pages = self.owned.pop(idx, None)
        if pages is not None:
            self.engine.pool.release(pages)


class SelfSpecDiffusionWorker:
    def __init__(self, server_args, gpu_id: int, tp_rank: int, dp_rank: Optional[int], moe_ep_rank: int,
                 attn_cp_rank: int, moe_dp_rank: int, nccl_port: int, target_worker):
        self.target_worker = target_worker
        self.engine: Engine = getattr(target_worker, "engine", target_worker)
        self.req_to_page: ReqToPagePool = getattr(target_worker, "req_to_page", None)
        if self.req_to_page is None:
            raise ValueError("target_worker must provide req_to_page (a ReqToPagePool)")
        self.tp_rank = tp_rank
        self.page_size = int(getattr(server_args, "page_size", 16) or 16)
        if self.page_size != self.engine.page_size:
            raise ValueError(f"page_size {self.page_size} != the K/V pool's {self.engine.page_size}")
        self.draft_token_num = int(server_args.speculative_num_draft_tokens)
        self.mask_id, bd_size, src = _resolve_block_diffusion(server_args)
        if self.mask_id != self.engine.cfg.mask_id:
            raise ValueError(f"mask id {self.mask_id} ({src}) != the model's {self.engine.cfg.mask_id}")
        if bd_size is not None and self.draft_token_num != bd_size + 1:
            raise ValueError(f"speculative_num_draft_tokens {self.draft_token_num} != bd_size + 1 = {bd_size + 1}")
        if tp_rank != 0:
            raise ValueError("the self-spec round runs one replica per GPU (no tensor parallelism)")
        self.device = self.engine.device
        self._seed_pool: Optional[torch.Tensor] = None
        self._rb = {}
        self._graphs = bool(int(os.environ.get("GR_GRAPHS", "1")))
        self.n_rounds = 0
        self._sampler: Optional[SamplerState] = None
        self._draft_ahead = bool(int(os.environ.get("SELFSPEC_DRAFT_AHEAD", "0"))) or \
            bool(getattr(server_args, "ss_draft_ahead", False))
        self._sched = None
        self._stash = None
        self.ahead_stats = {"launched": 0, "used": 0, "released": 0, "skip_finish": 0, "skip_sched": 0}
        self._random_seed = int(getattr(server_args, "random_seed", 0) or 0)
        self._filter = L.FILTER_TORCH if getattr(server_args, "sampling_backend", "flashinfer") == "pytorch" \
            else L.FILTER_JOINT

    # ------------------------------------------------------------------ pools / buffers
    def update_weights_from_tensor(self, recv_req):
        return self.target_worker.update_weights_from_tensor(recv_req)

    def clear_cache_pool(self):
        # captured graphs hold the pool's address: clear it in place
        if self._seed_pool is not None:
            self._seed_pool.zero_()

    def ss_bind_scheduler(self, scheduler) -> None:
        """Read-only access to the scheduler's running batch and waiting queue, for the draft-ahead gate."""
        self._sched = scheduler

    def ss_release_stash(self, reason: str = "") -> None:
        """Drop a pre-launched draft (the scheduler calls this before a prefill admission)."""
        if self._stash is not None:
            self._stash = None
            self.ahead_stats["released"] += 1

    def _ahead_allowed(self, batch) -> bool:
        """The next iteration is expected to decode this same batch (no prefill admission pending)."""
        s = self._sched
        if s is None:
            return True   # no scheduler bound: the caller either repeats the batch or releases the stash
        if batch is not getattr(s, "running_batch", None):
            return False
        waiting = getattr(s, "waiting_queue", None) or []
        full = getattr(getattr(s, "running_batch", None), "batch_is_full", False)
        return getattr(s, "chunked_req", None) is None and (not waiting or full)

    def _stash_matches(self, st, batch) -> bool:
        if batch is not st["batch"] or batch.req_pool_indices is not st["rpi"] or len(batch.reqs) != len(st["reqs"]):
            return False
        if any(a is not b for a, b in zip(batch.reqs, st["reqs"])):
            return False
        return batch.seq_lens_cpu is not None and batch.seq_lens_cpu.tolist() == st["seq_lens"]

    def _sampler_state(self) -> SamplerState:
        if self._sampler is None:
            self._sampler = SamplerState(self.engine.cfg.vocab, self.req_to_page.size, self.device,
                                         seed=self._random_seed, filter=self._filter)
        return self._sampler

    @staticmethod
    def _request_sampling(reqs) -> List[RequestSampling]:
        return [RequestSampling.of(r.sampling_params, stop_ids=sorted(stop_set(r))) for r in reqs]

    def _plain(self, reqs, rs: List[RequestSampling]) -> bool:
        """selfspec_sampling.is_plain (selfspec_sampling.py:40-70): every request greedy, no penalty, logit bias,
        grammar or custom logit processor."""
        return all(x.plain for x in rs) and not any(getattr(r, "grammar", None) is not None for r in reqs) and \
            not any(getattr(r.sampling_params, "custom_logit_processor", None) for r in reqs)

    @staticmethod
    def _custom_hook(reqs, K: int, cand: Optional[List[List[int]]]):
        """Custom logit processors on rows (b, j): one call per (processor, j) over its requests, each with a request
        view whose output_ids hold the row's prefix (output_ids + cand[b][0..j]; none for first-token rows)."""
        users = [(i, r.sampling_params.custom_logit_processor) for i, r in enumerate(reqs)
                 if getattr(r.sampling_params, "custom_logit_processor", None)]
        if not users:
            return None

        class _View:
            def __init__(self, req, extra):
                self._req, self.output_ids = req, list(req.output_ids) + list(extra)

            def __getattr__(self, n):
                return getattr(self._req, n)

        def hook(logits: torch.Tensor) -> None:
            for j in range(K):
                groups = {}
                for i, fn in users:
                    groups.setdefault(id(fn), (fn, []))[1].append(i)
                for fn, idx in groups.values():
                    rows = torch.tensor([i * K + j for i in idx], device=logits.device)
                    params = []
                    for i in idx:
                        prm = dict(reqs[i].sampling_params.custom_params or {})
                        prm["__req__"] = _View(reqs[i], cand[i][: j + 1] if cand is not None else [])
                        params.append(prm)
                    logits[rows] = fn(logits[rows], params)
        return hook

    def _pos_delta(self) -> torch.Tensor:
        """RoPE position - cache position of each pool slot (nonzero for a prefix with 2-D image positions)."""
        if getattr(self, "_delta_pool", None) is None:
            self._delta_pool = torch.zeros((self.req_to_page.size,), dtype=torch.int32, device=self.device)
        return self._delta_pool

    def _seeds(self) -> torch.Tensor:
        if self._seed_pool is None:
            self._seed_pool = torch.zeros((self.req_to_page.size,), dtype=torch.int64, device=self.device)
        return self._seed_pool

    def _buffers(self, bs: int):
        K = self.draft_token_num
        rb = self._rb.get(bs)
        if rb is None:
            eng = self.engine
            eng.reserve(bs * K)
            rb = eng.new_round_buffers(bs, K, self.req_to_page.pages_per_req, pool_size=self.req_to_page.size)
            rb.seeds = self._seeds()
            rb.graph = None
            rb.host = torch.zeros(rb.readback.shape, dtype=torch.int32).pin_memory()
            rb.event = torch.cuda.Event()
            rb.order = torch.arange(bs, dtype=torch.int32, device=self.device)  # exists before any capture
            self._rb[bs] = rb
        rb.seeds = self._seeds()
        return rb

    # ------------------------------------------------------------------ hooks
    def forward_batch_generation(self, batch) -> GenerationBatchResult:
        if batch.forward_mode.is_extend():
            self.ss_release_stash("prefill")
            return self._prefill(batch)
        st, self._stash = self._stash, None
        if st is not None:
            if self._stash_matches(st, batch):
                # this round's draft already ran right after the previous readback
                self.ahead_stats["used"] += 1
                self._cur = st["rb"]
                st["rb"].gv.replay()
                return self._fast_commit_round(batch, None, None)
            self.ahead_stats["released"] += 1
        draft_tokens = self._draft_block(batch)
        return self._fulldraft_verify(batch, draft_tokens)

    def _prefill(self, batch) -> GenerationBatchResult:
        eng = self.engine
        rpi = [int(i) for i in batch.req_pool_indices.tolist()]
        for i in rpi:
            self.req_to_page.assign(i)
        rb = self._buffers(len(rpi))
        rb.rpi.copy_(batch.req_pool_indices)
        rb.page_table.copy_(self.req_to_page.table[batch.req_pool_indices])
        xs, ids = [], []
        for req in batch.reqs:
            x, pid = req.prefix_rows(eng)
            xs.append(x)
            ids.append(pid)
        rs = self._request_sampling(batch.reqs)
        first_fn = None
        if not self._plain(batch.reqs, rs):
            st = self._sampler_state()
            for i in rpi:
                st.reset_slot(i)

            def first_fn(rows, which):
                sub = [batch.reqs[b] for b in which]
                masks = current_masks([getattr(r, "grammar", None) for r in sub], eng.cfg.vocab)
                smp = st.batch([rs[b] for b in which], rb.rpi[torch.tensor(which, device=self.device)].contiguous(),
                               None if masks is None else pack_allowed(masks).to(self.device))
                return first_tokens(eng, rows, len(which), smp, status=rb.status,
                                    custom=self._custom_hook(sub, 1, None))
        pos3 = [getattr(r, "mrope_positions", None) for r in batch.reqs]
        first = eng.prefill(rb, xs, ids, first_fn=first_fn, prefix_pos3=pos3)
        self._pos_delta()[batch.req_pool_indices] = rb.pos_delta
        batch.seq_lens.copy_(rb.seq_lens)
        batch.seq_lens_cpu = rb.seq_lens.cpu()
        for req, t in zip(batch.reqs, first):
            req.output_ids.append(t)
            req.check_finished()
            if getattr(req, "grammar", None) is not None and not req.finished():
                grammar_accept_or_abort(req, t)   # AR decode feeds every output token to the grammar
            req._spec_seed_ready = True
        return GenerationBatchResult(next_token_ids=torch.tensor(first, dtype=torch.int64, device=self.device),
                                     next_token_ids_cpu=[[t] for t in first], finish_checked=True)

    def _draft_block(self, batch) -> Optional[torch.Tensor]:
        """Stage the batch into the round buffers and enqueue the draft forward (device positions: its argmax
        [a0, d1..d_{K-1}] stays on the device as the verify input, so nothing is returned)."""
        if not all(getattr(r, "_spec_seed_ready", False) for r in batch.reqs):
            raise AssertionError("no carried seed (prefill/extend must seed the pool)")
        bs = len(batch.reqs)
        rb = self._buffers(bs)
        rb.rpi.copy_(batch.req_pool_indices)
        rb.page_table.copy_(self.req_to_page.table[batch.req_pool_indices])
        rb.seq_lens.copy_(batch.seq_lens)
        rb.pos_delta.copy_(self._pos_delta()[batch.req_pool_indices])
        # longest-first attention launch order for this batch (the captured graph reads it in place)
        self.engine.refresh_order(rb)
        self._cur = rb
        return None

    def _fulldraft_verify(self, batch, draft_tokens) -> GenerationBatchResult:
        """Verify over [a0, d1..d_{K-1}] at positions seq_lens + 1 + j and the commit: the whole round is one CUDA
        graph (draft, verify, accept-and-commit) replayed per batch-size bucket."""
        rb = self._cur
        eng = self.engine
        rs = self._request_sampling(batch.reqs)
        if not self._plain(batch.reqs, rs):
            return self._sampled_round(batch, rb, rs)
        if self._graphs:
            if rb.graph is None:
                snap = (rb.seq_lens.clone(), rb.seeds.clone(), rb.n_committed.clone(), rb.rounds.clone())
                eng.round_launch(rb)
                torch.cuda.synchronize()
                rb.seq_lens.copy_(snap[0]); rb.seeds.copy_(snap[1])
                rb.n_committed.copy_(snap[2]); rb.rounds.copy_(snap[3])
                rb.gd, rb.gv = eng.capture_split(rb)   # draft, and verify + commit (draft-ahead replays them apart)
                rb.graph = True
            rb.gd.replay()
            rb.gv.replay()
        else:
            eng.round_launch(rb)
        return self._fast_commit_round(batch, None, None)

    def _sampled_round(self, batch, rb, rs: List[RequestSampling]) -> GenerationBatchResult:
        """A non-plain batch: a0 drawn from AR's distribution of the draft's boundary rows (grammar mask of the current
        state), then the verify rows' speculative sampling (grammar rows after a0, d1..dj), the commit and the
        penalizer cumulation, all on the device; the host builds the grammar masks and runs custom processors."""
        eng, reqs, K = self.engine, batch.reqs, self.draft_token_num
        bs, V = len(reqs), eng.cfg.vocab
        st = self._sampler_state()
        sr = getattr(rb, "sampled", None)
        if sr is None:
            sr = rb.sampled = SampledRound(eng, rb)
        grammars = [getattr(r, "grammar", None) for r in reqs]
        m0 = current_masks(grammars, V)
        smp = st.batch(rs, rb.rpi, None if m0 is None else pack_allowed(m0).to(self.device))
        sr.draft(smp, custom=self._custom_hook(reqs, 1, None))
        cand = None
        need_host = any(g is not None for g in grammars) or \
            any(getattr(r.sampling_params, "custom_logit_processor", None) for r in reqs)
        if need_host:
            cand = rb.am.view(bs, K).cpu()
        m1 = verify_row_masks(grammars, cand, V) if cand is not None else None
        smp = st.batch(rs, rb.rpi, None if m1 is None else pack_allowed(m1).to(self.device))
        sr.verify(smp, st.rng, custom=self._custom_hook(reqs, K, None if cand is None else cand.tolist()))
        return self._fast_commit_round(batch, None, None, plain=False)

    def _fast_commit_round(self, batch, verify_input, batch_result, plain: bool = True,
                           vocab_mask: Optional[torch.Tensor] = None) -> GenerationBatchResult:
        """One pinned readback (packed rows + status), the host finish rules, K/V length fix-ups for requests that
        finished inside the round (selfspec_fast_commit.py:291-355)."""
        rb = self._cur
        K = self.draft_token_num
        bs = len(batch.reqs)
        rb.host.copy_(rb.readback, non_blocking=True)
        rb.event.record()
        # Draft-ahead goes out before the readback is waited on, so the GPU runs it while the host reads the rows.  It
        # is kept only if no request can end this round; otherwise it is dropped, which is harmless: the draft writes
        # K/V beyond the committed lengths (rewritten before anything reads them) and its own outputs, and the
        # readback was copied before it in stream order.
        launched = False
        if plain and self._draft_ahead and self._graphs and getattr(rb, "gd", None) is not None:
            if self._ahead_allowed(batch):
                # the longest-first attention order only schedules (results do not depend on it), and lengths move by
                # at most K + 1 a round: on an unchanged batch it is refreshed every 8th round, not between every
                # verify and the next draft
                if self.n_rounds % 8 == 0:
                    self.engine.refresh_order(rb)
                rb.gd.replay()
                launched = True
                self.ahead_stats["launched"] += 1
            else:
                self.ahead_stats["skip_sched"] += 1
        rb.event.synchronize()
        h = rb.host
        st = int(h[bs * (K + 2) + 1])
        if st:
            raise RuntimeError(f"device status {st}: {L.load().gr_status_string(st).decode()}")
        rows = h[: bs * (K + 2)].view(bs, K + 2).tolist()
        ahead = False
        if launched:
            if all(cannot_finish(q, [r[0]] + r[2: 3 + r[1]]) for q, r in zip(batch.reqs, rows)):
                ahead = True  # no request ends this round: the device lengths and seeds were the next round's
            else:
                self.ahead_stats["skip_finish"] += 1
        toks, js, accs = host_commit(batch.reqs, rows)
        # the kernel advanced seq_lens by acc + 2 (x0 + verify rows 0..acc); a request cut inside the round keeps j + 1
        fix = [accs[i] + 1 - js[i] for i in range(bs)]
        if any(fix):
            rb.seq_lens.sub_(torch.tensor(fix, dtype=torch.int64, device=self.device))
        batch.seq_lens.copy_(rb.seq_lens)
        sl = batch.seq_lens_cpu
        for i in range(bs):
            sl[i] += js[i] + 1
        self.n_rounds += 1
        if ahead:
            if any(fix) or any(r.finished() for r in batch.reqs):
                raise RuntimeError("draft-ahead: cannot_finish disagreed with the host finish rules")
            self._stash = {"batch": batch, "rpi": batch.req_pool_indices, "reqs": list(batch.reqs), "rb": rb,
                           "seq_lens": sl.tolist()}
        return GenerationBatchResult(next_token_ids=rb.out_next.clone(), num_accepted_tokens=sum(js),
                                     accept_length_per_req_cpu=js, next_token_ids_cpu=toks, finish_checked=True)
