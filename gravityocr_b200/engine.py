"""The self-speculative round on one B200: device weights, the paged K/V pool, the forward composed from the C-ABI
kernels, the draft / verify / accept-commit round and its CUDA-graph capture per (B, batch).

Data layout in HBM (bf16 unless noted):
  * weights per layer: ``qkv`` [q_dim + 2 kv_dim, H] (q, k, v rows stacked), ``o`` [H, q_dim], ``gate_up`` [2I, H]
    with gate and up rows interleaved pairwise (row 2j = gate j, 2j+1 = up j), ``down`` [H, I], 4 norm vectors;
    ``embed`` [V, H], ``norm`` [H], ``lm_head`` [V, H].
  * K/V cache: two tensors [layers, pages, kv_heads, page_size=16, head_dim] -- one (page, head) block of a layer is
    4 KiB contiguous, the TMA box of the attention kernel; requests own fixed page tables [bs, pages_per_req] int32.
  * per-forward activations for M = bs*K rows: residual ``h`` fp32 x2 (ping-pong), ``x`` bf16 (normed GEMM input),
    ``q`` / ``attn`` bf16 [M, q_dim], ``y`` fp32 [M, H] (o_proj / down_proj output), ``act`` bf16 [M, I].
  * round state (device, int64 like the reference's ``seq_lens`` / seed pool): ``seq_lens`` (K/V length; x0 not yet
    in K/V), ``seeds`` pool by req_pool_idx, ``n_committed`` / ``rounds`` int32; ``packed`` [bs, K+2] int32 + status
    word -- the round's only device->host copy.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import _lib as L
from .config import ModelConfig


def rope_inv_freq(cfg: ModelConfig) -> torch.Tensor:
    """transformers modeling_glm_ocr.py:708-710, computed on the CPU in fp32 exactly as there."""
    rd = cfg.rotary_dim
    return 1.0 / (cfg.rope_theta ** (torch.arange(0, rd, 2, dtype=torch.int64).to(dtype=torch.float32) / rd))


class DeviceWeights:
    """bf16 weights on one GPU in the kernels' layout."""

    def __init__(self, cfg: ModelConfig, weights: Dict[str, torch.Tensor], device: torch.device):
        self.cfg = cfg
        dev = device
        bf = torch.bfloat16
        up = lambda t: t.to(device=dev, dtype=bf).contiguous()
        self.embed = up(weights["embed_tokens"])
        self.norm = up(weights["norm"])
        self.lm_head = up(weights["lm_head"])
        self.layers = []
        for l in range(cfg.n_layers):
            p = f"layers.{l}."
            qkv = up(torch.cat([weights[p + "q_proj"], weights[p + "k_proj"], weights[p + "v_proj"]], 0))
            gu_raw = up(weights[p + "gate_up_proj"])
            gu = torch.empty_like(gu_raw)
            L.pack_gate_up(gu_raw, gu, cfg.intermediate)
            del gu_raw
            self.layers.append({
                "qkv": qkv, "o": up(weights[p + "o_proj"]), "gate_up": gu, "down": up(weights[p + "down_proj"]),
                "in": up(weights[p + "input_layernorm"]), "psa": up(weights[p + "post_self_attn_layernorm"]),
                "pa": up(weights[p + "post_attention_layernorm"]), "pm": up(weights[p + "post_mlp_layernorm"]),
            })
        self.inv_freq = rope_inv_freq(cfg).to(dev)
        torch.cuda.synchronize(dev)

    def streamed_bytes(self) -> int:
        n = self.norm.numel() + self.lm_head.numel()
        for d in self.layers:
            n += sum(d[k].numel() for k in ("qkv", "o", "gate_up", "down", "in", "psa", "pa", "pm"))
        return 2 * n


class PagePool:
    """Fixed-size page pool of the paged K/V cache; pages are handed out per request and returned on release."""

    def __init__(self, cfg: ModelConfig, n_pages: int, page_size: int, device: torch.device):
        self.cfg = cfg
        self.page_size = page_size
        self.n_pages = n_pages
        shape = (cfg.n_layers, n_pages, cfg.n_kv_heads, page_size, cfg.head_dim)
        self.k = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.v = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.free: List[int] = list(range(n_pages - 1, -1, -1))

    def alloc(self, n: int) -> List[int]:
        if n > len(self.free):
            raise RuntimeError(f"K/V pool exhausted: need {n} pages, {len(self.free)} free")
        return [self.free.pop() for _ in range(n)]

    def release(self, pages: Sequence[int]) -> None:
        self.free.extend(int(p) for p in pages)

    @staticmethod
    def bytes_needed(cfg: ModelConfig, n_pages: int, page_size: int) -> int:
        return 2 * cfg.n_layers * n_pages * cfg.n_kv_heads * page_size * cfg.head_dim * 2


# Split chunk (cache tokens per CTA) by (request, kv head) pairs: measured on a B200 with the config-3 prefix mix
# (U[256, 4096] + 32) at batch 4-32 and 2,738-token prefixes at batch 1-2, both kernels, chunks 256-4096.  A CTA has a
# large fixed cost (TMEM allocation, query staging, pipeline fill, the split merge), so fewer, longer splits win until
# the longest request's chain dominates: e.g. batch 32 takes 55.6 us at 2 splits against 70.6 at 4 and 102 at 12.
_CHUNK_BY_PAIRS = ((16, 640), (64, 1024), (192, 1536))


def attention_split(bs: int, K: int, max_len: int, avg_len: int, n_kv: int, sms: int) -> Tuple[int, int]:
    """Cache tokens per split and the split-grid extent.  With enough (request, head) pairs to fill the GPU twice the
    requests run in 4096-token splits (2560 just above twice); below that the chunk grows with the number of pairs
    (_CHUNK_BY_PAIRS, then 2048 tokens), never so small that a request needs more splits than the merges take: 8 while the grid stays within one
    CTA per SM (those splits merge inside one portable thread-block cluster), 16 otherwise.  A single request keeps a
    finer cut (about 16 splits of its length, capped at 8 by the cluster), which measured fastest inside its
    forward."""
    L = max_len + K + 1
    units = max(1, bs * n_kv)
    if units >= 2 * sms:
        # just above two CTAs per SM a 4096-token chunk leaves a thin second wave (measured: 40 requests 71.5 us at
        # 2560 against 86.4 at 4096); from ~2.4 CTAs per SM on, the widest chunk wins
        chunk = 2560 if units < (12 * sms) // 5 else 4096
    elif bs == 1:
        chunk = max(128, -(-max(1, avg_len) // 16))
    else:
        chunk = next((c for lim, c in _CHUNK_BY_PAIRS if units <= lim), 2048)
    chunk = max(chunk, -(-L // (8 if units < 2 * sms else 16)))
    chunk = min(4096, -(-chunk // 64) * 64)
    return chunk, max(1, -(-L // chunk))


@dataclass
class RoundBuffers:
    bs: int
    K: int
    seq_lens: torch.Tensor      # int64 [bs]
    page_table: torch.Tensor    # int32 [bs, pages_per_req]
    rpi: torch.Tensor           # int64 [bs]
    seeds: torch.Tensor         # int64 [pool]
    n_committed: torch.Tensor   # int32 [bs]
    rounds: torch.Tensor        # int32 [bs]
    am: torch.Tensor            # int32 [bs*K]  draft argmax = verify input [a0, d1..]
    v: torch.Tensor             # int32 [bs*K]  verify argmax
    gap_d: torch.Tensor         # fp32 [bs*K]
    gap_v: torch.Tensor
    top_d: torch.Tensor
    top_v: torch.Tensor
    readback: torch.Tensor      # int32 [bs*(K+2) + 4]: packed rows, then n_released, status
    released: torch.Tensor      # int64 [bs*K]
    out_next: torch.Tensor      # int64 [bs]
    accept_len: torch.Tensor    # int32 [bs]
    attn_chunk: int
    attn_splits: int
    order: Optional[torch.Tensor] = None            # int32 [bs] attention launch order (longest first)
    pos_delta: Optional[torch.Tensor] = None        # int32 [bs] RoPE position - cache position (M-RoPE delta)
    override_g: Optional[torch.Tensor] = None      # int32 [bs, g_len] forced-accept replay stream
    override_plan: Optional[torch.Tensor] = None   # int32 [bs, max_rounds]

    @property
    def packed(self) -> torch.Tensor:
        return self.readback[: self.bs * (self.K + 2)].view(self.bs, self.K + 2)

    @property
    def n_released(self) -> torch.Tensor:
        return self.readback[self.bs * (self.K + 2): self.bs * (self.K + 2) + 1]

    @property
    def status(self) -> torch.Tensor:
        return self.readback[self.bs * (self.K + 2) + 1: self.bs * (self.K + 2) + 2]


class Engine:
    """One model replica on one GPU: the forward, the round and graph capture."""

    def __init__(self, cfg: ModelConfig, weights: Dict[str, torch.Tensor], *, max_rows: int, n_pages: int,
                 page_size: int = 16, device: Optional[torch.device] = None, pdl: bool = True):
        L.load()
        if page_size != 16:
            raise ValueError("the attention kernel's TMA box is one 16-token page")
        self.cfg = cfg
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.page_size = page_size
        L.set_pdl(pdl)
        self.w = DeviceWeights(cfg, weights, self.device)
        self.pool = PagePool(cfg, n_pages, page_size, self.device)
        self.max_rows = max_rows
        dev, H = self.device, cfg.hidden
        self.h = [torch.zeros((max_rows, H), dtype=torch.float32, device=dev) for _ in range(2)]
        self.x = torch.zeros((max_rows, H), dtype=torch.bfloat16, device=dev)
        self.q = torch.zeros((max_rows, cfg.q_dim), dtype=torch.bfloat16, device=dev)
        self.attn = torch.zeros((max_rows, cfg.q_dim), dtype=torch.bfloat16, device=dev)
        self.y = torch.zeros((0,), dtype=torch.float32, device=dev)   # split-K partials of o_proj / down_proj
        self._grow_y(max_rows)
        self.act = torch.zeros((max_rows, cfg.intermediate), dtype=torch.bfloat16, device=dev)
        self.row_pos = torch.zeros((max_rows,), dtype=torch.int32, device=dev)
        self.row_slot = torch.zeros((max_rows,), dtype=torch.int64, device=dev)
        self.row_ids = torch.zeros((max_rows,), dtype=torch.int32, device=dev)
        self.status = torch.zeros((4,), dtype=torch.int32, device=dev)
        self.lin_ws = torch.zeros((self.linear_ws_bytes(max_rows),), dtype=torch.uint8, device=dev)
        self.attn_ws: Optional[torch.Tensor] = None
        self.sms = L.num_sms()
        self.graphs: Dict[Tuple[int, int], torch.cuda.CUDAGraph] = {}

    # ------------------------------------------------------------------ workspace
    def gemm_shapes(self) -> List[Tuple[int, int, int]]:
        """(n_out, k_in, epilogue mode) of every projection a forward or a sampled round runs."""
        c = self.cfg
        return [(c.qkv_dim, c.hidden, L.EPI_QKV_ROPE), (c.hidden, c.q_dim, L.EPI_PARTIAL_F32),
                (2 * c.intermediate, c.hidden, L.EPI_SWIGLU), (c.hidden, c.intermediate, L.EPI_PARTIAL_F32),
                (c.vocab, c.hidden, L.EPI_ARGMAX), (c.vocab, c.hidden, L.EPI_STORE_F32)]

    def linear_ws_bytes(self, m: int) -> int:
        """Scratch of every projection at M = m rows with its default split-K (tickets, partials, argmax tiles)."""
        return max(L.linear_workspace_bytes(n, m, L.linear_default_splits(n, k, m, mode))
                   for n, k, mode in self.gemm_shapes())

    def splits(self, n_out: int, k_in: int, m: int) -> int:
        """Split-K count of o_proj / down_proj writing partials for gr_residual_norm."""
        return L.linear_default_splits(n_out, k_in, m, L.EPI_PARTIAL_F32)

    def _grow_y(self, m: int) -> None:
        c = self.cfg
        parts = max(self.splits(c.hidden, c.q_dim, m), self.splits(c.hidden, c.intermediate, m))
        need = parts * m * c.hidden
        if self.y.numel() < need:
            self.y = torch.zeros((need,), dtype=torch.float32, device=self.device)

    def reserve(self, m: int) -> None:
        """Grow the projection scratch and the partial-sum buffer for M = m rows (never during graph capture)."""
        need = self.linear_ws_bytes(m)
        if self.lin_ws.numel() < need:
            self.lin_ws = torch.zeros((need,), dtype=torch.uint8, device=self.device)
        self._grow_y(m)

    def _attn_workspace(self, bs: int, K: int, splits: int) -> torch.Tensor:
        need = L.attention_workspace_bytes(bs, K, self.cfg.n_q_heads, self.cfg.n_kv_heads, splits)
        if self.attn_ws is None or self.attn_ws.numel() < need:
            self.attn_ws = torch.zeros((max(need, 256),), dtype=torch.uint8, device=self.device)
        return self.attn_ws

    # ------------------------------------------------------------------ forward
    def forward(self, rows_mode: int, bs: int, K: int, seq_lens: torch.Tensor, page_table: torch.Tensor, *,
                out_idx: torch.Tensor, out_top1: Optional[torch.Tensor] = None, out_gap: Optional[torch.Tensor] = None,
                seeds=None, rpi=None, ids32=None, ids64=None, row_embeds=None, attn_chunk: int = 64,
                attn_splits: int = 1, status: Optional[torch.Tensor] = None, head: bool = True,
                order: Optional[torch.Tensor] = None, attn_draft: Optional[int] = None,
                rope_delta: Optional[torch.Tensor] = None, rope_pos3: Optional[torch.Tensor] = None) -> None:
        """One pass of the decoder over M = bs*K rows; writes each row's argmax (and top-1 / gap) to out_idx.
        head=False stops before lm_head (the normed final hidden rows stay in ``self.x``).  attn_draft overrides the
        attention mask the row mode implies (1 for draft rows, else causal); 2 = every row sees the whole window.
        rope_delta (int32 [bs]): RoPE position = cache position + delta; rope_pos3 (int32 [M, 3]): explicit
        multimodal (t, h, w) positions of the rows instead."""
        cfg, w, M = self.cfg, self.w, bs * K
        if M > self.max_rows:
            raise ValueError(f"{M} rows > max_rows {self.max_rows}")
        st = status if status is not None else self.status
        c_ = self.cfg
        y_need = max(self.splits(c_.hidden, c_.q_dim, M), self.splits(c_.hidden, c_.intermediate, M)) * M * c_.hidden
        if self.lin_ws.numel() < self.linear_ws_bytes(M) or self.y.numel() < y_need:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError(f"scratch too small for M={M}; call reserve() before capture")
            self.reserve(M)
        L.embed_rows(rows_mode, bs, K, seeds=seeds, rpi=rpi, ids32=ids32, ids64=ids64, row_embeds=row_embeds,
                     seq_lens=seq_lens, page_table=page_table, page_size=self.page_size, embed=w.embed, vocab=cfg.vocab,
                     mask_id=cfg.mask_id, norm_w=w.layers[0]["in"], eps=cfg.rms_eps, h_out=self.h[0], x_out=self.x,
                     row_pos=self.row_pos, row_slot=self.row_slot, row_ids=self.row_ids, rope_delta=rope_delta,
                     status=st)
        ws_attn = self._attn_workspace(bs, K, attn_splits) if attn_splits > 1 else None
        draft = int(rows_mode == L.ROWS_DRAFT) if attn_draft is None else int(attn_draft)
        self._forward_body(rows_mode, bs, K, seq_lens, page_table, out_idx, out_top1, out_gap, attn_chunk,
                           attn_splits, st, head, order, ws_attn, draft, rope_pos3)

    def _forward_body(self, rows_mode, bs, K, seq_lens, page_table, out_idx, out_top1, out_gap, attn_chunk,
                      attn_splits, st, head, order, ws_attn, draft, rope_pos3=None) -> None:
        """The layers and lm_head after the embedding rows."""
        ops = L
        cfg, w, M = self.cfg, self.w, bs * K
        base_add = 1 if rows_mode == L.ROWS_VERIFY else 0
        cur = 0
        for l, d in enumerate(w.layers):
            nxt = w.layers[l + 1] if l + 1 < len(w.layers) else None
            e = L.Epilogue()
            e.mode = L.EPI_QKV_ROPE
            e.q_out = self.q.data_ptr()
            e.k_cache = self.pool.k[l].data_ptr()
            e.v_cache = self.pool.v[l].data_ptr()
            e.row_pos = self.row_pos.data_ptr()
            e.row_slot = self.row_slot.data_ptr()
            e.inv_freq = w.inv_freq.data_ptr()
            e.rotary_dim = cfg.rotary_dim
            if rope_pos3 is not None:
                e.row_pos3 = rope_pos3.data_ptr()
                for i in range(3):
                    e.mrope_section[i] = cfg.mrope_section[i]
            e.n_q_heads = cfg.n_q_heads
            e.n_kv_heads = cfg.n_kv_heads
            e.page_size = self.page_size
            ops.linear(d["qkv"], self.x, M, e, self.lin_ws, prefetch=d["o"], status=st)
            ops.bd_attention(self.q, self.pool.k[l], self.pool.v[l], page_table, seq_lens, bs, K, draft, base_add,
                           cfg.n_q_heads, cfg.n_kv_heads, self.page_size, attn_chunk, attn_splits, self.attn, ws_attn,
                           status=st, order=order)
            e = L.Epilogue()
            e.mode = L.EPI_PARTIAL_F32
            e.out = self.y.data_ptr()
            e.ld_out = cfg.hidden
            sp_o = self.splits(cfg.hidden, cfg.q_dim, M)
            ops.linear(d["o"], self.attn, M, e, self.lin_ws, splits=sp_o, prefetch=d["gate_up"], status=st)
            ops.residual_norm(M, self.h[cur], self.y, d["psa"], d["pa"], cfg.rms_eps, self.h[1 - cur], self.x,
                              y_parts=sp_o)
            cur ^= 1
            e = L.Epilogue()
            e.mode = L.EPI_SWIGLU
            e.out = self.act.data_ptr()
            e.ld_out = cfg.intermediate
            ops.linear(d["gate_up"], self.x, M, e, self.lin_ws, prefetch=d["down"], status=st)
            e = L.Epilogue()
            e.mode = L.EPI_PARTIAL_F32
            e.out = self.y.data_ptr()
            e.ld_out = cfg.hidden
            sp_d = self.splits(cfg.hidden, cfg.intermediate, M)
            pf = nxt["qkv"] if nxt is not None else w.lm_head[: min(w.lm_head.shape[0], 16384)]
            ops.linear(d["down"], self.act, M, e, self.lin_ws, splits=sp_d, prefetch=pf, status=st)
            ops.residual_norm(M, self.h[cur], self.y, d["pm"], nxt["in"] if nxt is not None else w.norm, cfg.rms_eps,
                              self.h[1 - cur], self.x, y_parts=sp_d)
            cur ^= 1
        if not head:
            return
        e = L.Epilogue()
        e.mode = L.EPI_ARGMAX
        e.out_idx = out_idx.data_ptr()
        e.out_top1 = 0 if out_top1 is None else out_top1.data_ptr()
        e.out_gap = 0 if out_gap is None else out_gap.data_ptr()
        ops.linear(w.lm_head, self.x, M, e, self.lin_ws, status=st)

    def final_hidden(self) -> torch.Tensor:
        """Normed input of lm_head of the last forward (bf16 [max_rows, H]); for logits checks in tests."""
        return self.x

    # ------------------------------------------------------------------ requests
    def pages_for(self, max_len: int) -> int:
        return (max_len + self.page_size - 1) // self.page_size

    def new_round_buffers(self, bs: int, K: int, pages_per_req: int, pool_size: Optional[int] = None,
                          max_len: Optional[int] = None, avg_len: Optional[int] = None) -> RoundBuffers:
        dev = self.device
        pool_size = pool_size or bs
        ml = max_len or pages_per_req * self.page_size
        chunk, splits = attention_split(bs, K, ml, avg_len or ml, self.cfg.n_kv_heads, self.sms)
        i32 = dict(dtype=torch.int32, device=dev)
        i64 = dict(dtype=torch.int64, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        return RoundBuffers(
            bs=bs, K=K, seq_lens=torch.zeros((bs,), **i64), page_table=torch.zeros((bs, pages_per_req), **i32),
            rpi=torch.arange(bs, **i64), seeds=torch.zeros((pool_size,), **i64), n_committed=torch.zeros((bs,), **i32),
            rounds=torch.zeros((bs,), **i32), am=torch.zeros((bs * K,), **i32), v=torch.zeros((bs * K,), **i32),
            gap_d=torch.zeros((bs * K,), **f32), gap_v=torch.zeros((bs * K,), **f32),
            top_d=torch.zeros((bs * K,), **f32), top_v=torch.zeros((bs * K,), **f32),
            readback=torch.zeros((bs * (K + 2) + 4,), **i32), released=torch.zeros((bs * K,), **i64),
            out_next=torch.zeros((bs,), **i64), accept_len=torch.zeros((bs,), **i32),
            attn_chunk=chunk, attn_splits=splits, pos_delta=torch.zeros((bs,), **i32))

    def prefill(self, rb: RoundBuffers, prefixes: List[torch.Tensor], prefix_ids: List[torch.Tensor],
                chunk: int = 64, attn_chunk: Optional[int] = None, first_fn=None,
                prefix_pos3: Optional[List[Optional[torch.Tensor]]] = None) -> List[int]:
        """Causal prefill of each request's prefix through the same kernels (chunks of ``chunk`` rows, causal
        attention).  prefixes[b]: fp32 [P_b, H] layer-0 input rows (image embeddings + prompt embeddings);
        prefix_ids[b]: int64 [P_b] ids (< 0 where the row comes from ``prefixes``).  Sets seq_lens = P_b, the seed
        pool (seeds[rpi[b]] = first generated token), n_committed = 1.  Returns the first tokens: the argmax of the
        last prefix row, or first_fn(rows [n, H] bf16, request indices) for a batch that samples.
        prefix_pos3[b] (int [3, P_b], optional): the request's multimodal (t, h, w) prefix positions (image tokens on a
        grid); its decode rows then rotate by cache position + (max position + 1 - P_b), kept in rb.pos_delta."""
        bs = rb.bs
        dev = self.device
        lens = [int(p.shape[0]) for p in prefixes]
        cap = rb.page_table.shape[1] * self.page_size
        for n in lens:
            if ((n + chunk - 1) // chunk) * chunk > cap:
                raise ValueError(f"prefix of {n} rows needs {((n + chunk - 1) // chunk) * chunk} slots, capacity {cap}")
        n_chunks = max((n + chunk - 1) // chunk for n in lens)
        mm = prefix_pos3 is not None and any(p is not None for p in prefix_pos3)
        H = self.cfg.hidden
        self.reserve(bs * chunk)
        out_idx = torch.zeros((bs * chunk,), dtype=torch.int32, device=dev)
        # Every prefix row and id goes to the device once; a chunk gathers its rows there (row `pad` is zeros, for the
        # rows past a prefix that ends inside the chunk).  The first tokens stay on the device until the end, so the
        # host never waits for a chunk and stays ahead of the GPU.
        offs = [0]
        for n in lens:
            offs.append(offs[-1] + n)
        pad = offs[-1]
        all_rows = torch.empty((pad + 1, H), dtype=torch.float32, device=dev)
        all_ids = torch.empty((pad + 1,), dtype=torch.int64, device=dev)
        for b in range(bs):
            all_rows[offs[b]: offs[b + 1]].copy_(prefixes[b])
            all_ids[offs[b]: offs[b + 1]].copy_(prefix_ids[b])
        all_rows[pad].zero_()
        all_ids[pad] = 0
        first_dev = torch.zeros((bs,), dtype=torch.int64, device=dev)
        for c in range(n_chunks):
            active = [b for b in range(bs) if lens[b] > c * chunk]
            nb = len(active)
            gather = torch.full((nb * chunk,), pad, dtype=torch.int64)
            for i, b in enumerate(active):
                s0, s1 = c * chunk, min(lens[b], (c + 1) * chunk)
                gather[i * chunk: i * chunk + s1 - s0] = torch.arange(offs[b] + s0, offs[b] + s1)
            gather = gather.to(dev)
            rows_e = all_rows.index_select(0, gather)
            ids = all_ids.index_select(0, gather)
            seq = torch.full((nb,), c * chunk, dtype=torch.int64).to(dev)
            pt = rb.page_table[torch.tensor(active, device=dev)].contiguous()
            pos3 = None
            if mm:
                pos3 = (torch.arange(c * chunk, (c + 1) * chunk, dtype=torch.int32)[None, :, None]
                        .expand(nb, chunk, 3).contiguous())
                for i, b in enumerate(active):
                    if prefix_pos3[b] is not None:
                        s0, s1 = c * chunk, min(lens[b], (c + 1) * chunk)
                        pos3[i, : s1 - s0] = prefix_pos3[b][:, s0:s1].T.to(torch.int32)
                pos3 = pos3.view(nb * chunk, 3).to(dev)
            ml = (c + 1) * chunk
            ach, asp = attention_split(nb, chunk, ml, ml, self.cfg.n_kv_heads, self.sms)
            if attn_chunk:
                ach, asp = attn_chunk, int(math.ceil(ml / attn_chunk))
            self.forward(L.ROWS_EXPLICIT, nb, chunk, seq, pt, out_idx=out_idx, ids64=ids, row_embeds=rows_e,
                         attn_chunk=ach, attn_splits=asp, status=rb.status, head=False, rope_pos3=pos3)
            # lm_head only on the rows that end a prefix (the first generated token of those requests)
            ends = [(b, i * chunk + (lens[b] - 1 - c * chunk)) for i, b in enumerate(active)
                    if c * chunk <= lens[b] - 1 < (c + 1) * chunk]
            if ends:
                rows = self.x[torch.tensor([r for _, r in ends], device=dev)].contiguous()
                if first_fn is not None:
                    res = first_fn(rows, [b for b, _ in ends])
                else:
                    e = L.Epilogue()
                    e.mode = L.EPI_ARGMAX
                    e.out_idx = out_idx.data_ptr()
                    L.linear(self.w.lm_head, rows, len(ends), e, self.lin_ws, status=rb.status)
                    res = out_idx[: len(ends)]
                first_dev[torch.tensor([b for b, _ in ends], device=dev)] = res.to(device=dev, dtype=torch.int64)
        rb.seq_lens.copy_(torch.tensor(lens, dtype=torch.int64))
        delta = [0] * bs
        for b in range(bs):
            if prefix_pos3 is not None and prefix_pos3[b] is not None:
                delta[b] = int(prefix_pos3[b].max()) + 1 - lens[b]
        rb.pos_delta.copy_(torch.tensor(delta, dtype=torch.int32))
        self.refresh_order(rb)
        rb.seeds[rb.rpi] = first_dev
        rb.n_committed.fill_(1)
        rb.rounds.zero_()
        self.check_status(rb)
        return first_dev.cpu().tolist()

    def refresh_order(self, rb: RoundBuffers) -> None:
        """Longest-first attention launch order from the current lengths (scheduling only; results do not depend on
        it).  The buffer is updated in place, so captured graphs pick it up."""
        order = torch.argsort(rb.seq_lens, descending=True, stable=True).to(torch.int32)
        if rb.order is None:
            rb.order = order.contiguous()
        else:
            rb.order.copy_(order)

    def check_status(self, rb: RoundBuffers) -> None:
        s = int(rb.status.item())
        if s != 0:
            raise RuntimeError(f"device status {s}: {L.load().gr_status_string(s).decode()}")

    # ------------------------------------------------------------------ the round
    def draft_launch(self, rb: RoundBuffers, override: bool = False) -> None:
        """Enqueue the draft forward over [x0 | mask x (K-1)] (+ the forced-accept override when asked)."""
        bs, K = rb.bs, rb.K
        self.forward(L.ROWS_DRAFT, bs, K, rb.seq_lens, rb.page_table, out_idx=rb.am, out_top1=rb.top_d,
                     out_gap=rb.gap_d, seeds=rb.seeds, rpi=rb.rpi, attn_chunk=rb.attn_chunk,
                     attn_splits=rb.attn_splits, status=rb.status, order=rb.order, rope_delta=rb.pos_delta)
        if override:
            L.draft_override(bs, K, rb.am, rb.override_g, rb.n_committed, rb.override_plan, rb.rounds,
                             self.cfg.vocab, self.cfg.mask_id)

    def verify_launch(self, rb: RoundBuffers) -> None:
        """Enqueue the causal verify forward over [a0, d1..d_{K-1}] and the accept-and-commit kernel."""
        bs, K = rb.bs, rb.K
        self.forward(L.ROWS_VERIFY, bs, K, rb.seq_lens, rb.page_table, out_idx=rb.v, out_top1=rb.top_v,
                     out_gap=rb.gap_v, ids32=rb.am, attn_chunk=rb.attn_chunk, attn_splits=rb.attn_splits,
                     status=rb.status, order=rb.order, rope_delta=rb.pos_delta)
        L.accept_commit(bs, K, rb.am, rb.v, rb.seeds, rb.rpi, rb.seq_lens, rb.packed, rb.released, rb.out_next,
                        x0_committed=False, n_released=rb.n_released, n_committed=rb.n_committed, rounds=rb.rounds,
                        accept_len=rb.accept_len)

    def round_launch(self, rb: RoundBuffers, override: bool = False) -> None:
        """Enqueue one round: draft forward, optional forced-accept override, verify forward, accept-and-commit."""
        self.draft_launch(rb, override)
        self.verify_launch(rb)

    def kernels_per_forward(self, rows: int = 0) -> int:
        """Kernel launches of one forward of `rows` rows: embed + per layer (4 projections, attention, 2 residual
        norms) + lm_head (projection + per-token argmax reduction)."""
        return 3 + 7 * self.cfg.n_layers

    def capture(self, rb: RoundBuffers, override: bool = False, warmup: int = 0) -> torch.cuda.CUDAGraph:
        """Capture one round (both forwards and the commit) into a CUDA graph; replays read the device-resident
        lengths, seeds and page tables, so one graph serves every round of this (B, batch) bucket."""
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self.round_launch(rb, override)
        torch.cuda.current_stream().wait_stream(s)
        self.graphs[(rb.K, rb.bs)] = g
        return g

    def capture_split(self, rb: RoundBuffers, override: bool = False) -> Tuple[torch.cuda.CUDAGraph, torch.cuda.CUDAGraph]:
        """Two graphs per (B, batch): the draft forward, and the verify forward + commit (timed separately)."""
        gd, gv = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(gd, stream=s):
                self.draft_launch(rb, override)
            with torch.cuda.graph(gv, stream=s):
                self.verify_launch(rb)
        torch.cuda.current_stream().wait_stream(s)
        return gd, gv


def host_rows(readback_host: torch.Tensor, bs: int, K: int) -> List[List[int]]:
    return readback_host[: bs * (K + 2)].view(bs, K + 2).tolist()
