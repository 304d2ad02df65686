"""Drop-in for the served boundary: a ``SelfSpecDiffusionWorker`` with the reference's constructor and hooks
(``patches/sglang/python/sglang/srt/speculative/selfspec_diffusion_worker.py:313-1341``), running the full-draft
round (``SELFSPEC_FULLDRAFT=1``, ``SELFSPEC_FAST_COMMIT=1``, device positions) on the CUDA path.

Hooks kept 1:1 -- ``forward_batch_generation`` (:1127), ``_draft_block`` (:660), ``_fulldraft_verify`` (:822),
``_fast_commit_round`` (:963), ``clear_cache_pool`` / ``update_weights_from_tensor`` (:472-487) and the scheduler
hooks ``ss_bind_scheduler`` / ``ss_release_stash`` (:1001, :1019; no draft is launched ahead, so there is never a
stash to release).  The result carries the reference's contract (:954-961, :990-998): ``next_token_ids`` = the
device next seeds [bs], ``next_token_ids_cpu`` = the committed tokens per request, ``accept_length_per_req_cpu``
= j per request, ``num_accepted_tokens`` = sum(j), ``finish_checked=True``.

Ownership as in the reference: the K/V pages and the request -> page table belong to the target worker (an
``Engine`` plus a ``ReqToPagePool``); the seed pool and the pinned readback buffer belong to this worker.  Greedy
batches only (non-greedy sampling is a later step; such a batch raises ``ValueError``).

SGLang itself is not a dependency: ``ScheduleBatch``-, ``Req``- and ``GenerationBatchResult``-shaped objects are
duck typed; ``gravityocr_b200.compat.types`` provides minimal ones for tests and standalone serving.
"""
from __future__ import annotations

import json
import os
from typing import List, Optional

import torch

from .. import _lib as L
from ..commit_rules import host_commit
from ..engine import Engine
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

    # ------------------------------------------------------------------ pools / buffers
    def update_weights_from_tensor(self, recv_req):
        return self.target_worker.update_weights_from_tensor(recv_req)

    def clear_cache_pool(self):
        # captured graphs hold the pool's address: clear it in place
        if self._seed_pool is not None:
            self._seed_pool.zero_()

    def ss_bind_scheduler(self, scheduler) -> None:
        self._scheduler = scheduler

    def ss_release_stash(self, reason: str = "") -> None:
        return None

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
            return self._prefill(batch)
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
        first = eng.prefill(rb, xs, ids)
        batch.seq_lens.copy_(rb.seq_lens)
        batch.seq_lens_cpu = rb.seq_lens.cpu()
        for req, t in zip(batch.reqs, first):
            req.output_ids.append(t)
            req.check_finished()
            req._spec_seed_ready = True
        return GenerationBatchResult(next_token_ids=torch.tensor(first, dtype=torch.int64, device=self.device),
                                     next_token_ids_cpu=[[t] for t in first], finish_checked=True)

    def _draft_block(self, batch) -> Optional[torch.Tensor]:
        """Stage the batch into the round buffers and enqueue the draft forward (device positions: its argmax
        [a0, d1..d_{K-1}] stays on the device as the verify input, so nothing is returned)."""
        if not all(getattr(r, "_spec_seed_ready", False) for r in batch.reqs):
            raise AssertionError("no carried seed (prefill/extend must seed the pool)")
        for r in batch.reqs:
            sp = r.sampling_params
            if getattr(sp, "temperature", 0.0) not in (0.0, None) and not getattr(sp, "greedy", True):
                raise ValueError("non-greedy sampling is not on the CUDA path")
        bs = len(batch.reqs)
        rb = self._buffers(bs)
        rb.rpi.copy_(batch.req_pool_indices)
        rb.page_table.copy_(self.req_to_page.table[batch.req_pool_indices])
        rb.seq_lens.copy_(batch.seq_lens)
        # longest-first attention launch order for this batch (the captured graph reads it in place)
        self.engine.refresh_order(rb)
        self._cur = rb
        return None

    def _fulldraft_verify(self, batch, draft_tokens) -> GenerationBatchResult:
        """Verify over [a0, d1..d_{K-1}] at positions seq_lens + 1 + j and the commit: the whole round is one CUDA
        graph (draft, verify, accept-and-commit) replayed per batch-size bucket."""
        rb = self._cur
        eng = self.engine
        if self._graphs:
            if rb.graph is None:
                snap = (rb.seq_lens.clone(), rb.seeds.clone(), rb.n_committed.clone(), rb.rounds.clone())
                eng.round_launch(rb)
                torch.cuda.synchronize()
                rb.seq_lens.copy_(snap[0]); rb.seeds.copy_(snap[1])
                rb.n_committed.copy_(snap[2]); rb.rounds.copy_(snap[3])
                rb.graph = eng.capture(rb)
            rb.graph.replay()
        else:
            eng.round_launch(rb)
        return self._fast_commit_round(batch, None, None)

    def _fast_commit_round(self, batch, verify_input, batch_result, plain: bool = True,
                           vocab_mask: Optional[torch.Tensor] = None) -> GenerationBatchResult:
        """One pinned readback (packed rows + status), the host finish rules, K/V length fix-ups for requests that
        finished inside the round (selfspec_fast_commit.py:291-355)."""
        rb = self._cur
        K = self.draft_token_num
        bs = len(batch.reqs)
        rb.host.copy_(rb.readback, non_blocking=True)
        rb.event.record()
        rb.event.synchronize()
        h = rb.host
        st = int(h[bs * (K + 2) + 1])
        if st:
            raise RuntimeError(f"device status {st}: {L.load().gr_status_string(st).decode()}")
        rows = h[: bs * (K + 2)].view(bs, K + 2).tolist()
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
        return GenerationBatchResult(next_token_ids=rb.out_next.clone(), num_accepted_tokens=sum(js),
                                     accept_length_per_req_cpu=js, next_token_ids_cpu=toks, finish_checked=True)
