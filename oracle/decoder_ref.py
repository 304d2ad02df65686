"""CPU oracle for the GLM-OCR-shaped decoder and the self-speculative round.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this module, and only as the
checker (or as the timed CPU port).  The product path never calls it.

What it restates, in plain torch fp32 on the CPU:
  * the decoder layer of transformers 5.5 ``models/glm_ocr/modeling_glm_ocr.py`` (RMSNorm :50-64, interleaved-pair
    partial RoPE :121-165 with the inverse frequencies of :700-711 and the 1-D M-RoPE of :715-735, GQA attention
    :168-235 with ``repeat_kv`` :86-95, SwiGLU MLP with the gate in the first half of gate_up :237-252, the sandwich
    norms of the decoder layer :255-302);
  * the in-process natcache round, ``src/fast_sampling.py:425-628`` (``generate_speculative_natcache``), greedy,
    draft_steps=1, full_draft=True: draft mask :508-510, verify mask :512-514, token shift :531-536, accept
    :577-584, cache truncation :600-605;
  * the served full-draft round of ``patches/sglang/python/sglang/srt/speculative/selfspec_diffusion_worker.py``:
    draft window ``[seed | mask x (K-1)]`` at positions ``seq_lens + j`` (:691-706, :575-605), x0's row causal and
    the mask rows bidirectional (:702-704), verify over ``am[:, :K]`` at positions ``seq_lens + 1 + j`` (:849-884),
    and the linear-chain greedy accept (``oracle.commit_ref.chain_accept``);
  * greedy AR decoding and the one-pass teacher-forced argmax (``src/fast_sampling.py:631-690``), with the top-2
    logit gap used to list argmax near-ties.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own ``generate_speculative_natcache`` and
``teacher_force_argmax`` (imported from the reference tree in the build container) on the same seeded weights and
inputs and stores the streams; ``tests/test_oracle_golden.py`` checks this module against them.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch


@dataclass
class OracleCache:
    """Contiguous per-request K/V by logical position: [layers, capacity, kv_heads, head_dim] fp32."""

    k: torch.Tensor
    v: torch.Tensor


class OracleDecoder:
    def __init__(self, cfg, weights: Dict[str, torch.Tensor], device: str = "cpu"):
        self.cfg = cfg
        self.device = torch.device(device)
        self.w = {k: t.to(device=self.device, dtype=torch.float32) for k, t in weights.items()}
        rd = cfg.rotary_dim
        # modeling_glm_ocr.py:708-710 (int64 arange, float division, fp32 reciprocal)
        self.inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, rd, 2, dtype=torch.int64).to(
            device=self.device, dtype=torch.float32) / rd))

    # ------------------------------------------------------------------ primitives
    def rms(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        x = x.float()
        var = x.pow(2).mean(-1, keepdim=True)
        return w * (x * torch.rsqrt(var + self.cfg.rms_eps))

    def rope(self, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """x [T, heads, head_dim]; rotates pairs (2i, 2i+1) of the first rotary_dim lanes by pos * inv_freq[i].
        pos [T] (1-D) or [T, 3] multimodal (t, h, w): pair i then takes the axis of its M-RoPE section
        (modeling_glm_ocr.py:730-735 apply_mrope: chunks of mrope_section along the frequencies, chunk c from axis c)."""
        rd = self.cfg.rotary_dim
        pos = pos.to(self.device)
        if pos.dim() == 2:
            sec = getattr(self.cfg, "mrope_section", (8, 12, 12))
            axis = torch.cat([torch.full((n,), a, dtype=torch.int64) for a, n in enumerate(sec)]).to(self.device)
            f = pos.float()[:, axis] * self.inv_freq[None, :]                        # [T, rd/2]
        else:
            f = pos.float()[:, None] * self.inv_freq[None, :]                        # [T, rd/2]
        c, s = f.cos()[:, None, :], f.sin()[:, None, :]
        x0, x1 = x[..., 0:rd:2], x[..., 1:rd:2]
        out = x.clone()
        out[..., 0:rd:2] = x0 * c - x1 * s
        out[..., 1:rd:2] = x1 * c + x0 * s
        return out

    def new_cache(self, capacity: int) -> OracleCache:
        c = self.cfg
        shape = (c.n_layers, capacity, c.n_kv_heads, c.head_dim)
        return OracleCache(torch.zeros(shape, device=self.device), torch.zeros(shape, device=self.device))

    def embed(self, ids: torch.Tensor) -> torch.Tensor:
        return self.w["embed_tokens"][ids.to(self.device)].float()

    # ------------------------------------------------------------------ forward
    def forward(self, x: torch.Tensor, pos: torch.Tensor, cache: OracleCache, write_pos: torch.Tensor,
                visible: torch.Tensor) -> torch.Tensor:
        """One decoder pass over T rows.

        x [T, hidden] layer-0 input; pos [T] RoPE positions; write_pos [T] cache positions the rows' K/V are stored at
        (before attention, as ``past_key_values.update`` does); visible [T, L] bool: row t attends to cache positions
        j < L with visible[t, j].  Returns the last layer's output (before the final norm)."""
        c, w = self.cfg, self.w
        T = x.shape[0]
        L = visible.shape[1]
        g = c.n_q_heads // c.n_kv_heads
        scale = c.head_dim ** -0.5
        wp = write_pos.to(self.device).long()
        neg = torch.zeros((T, L), device=self.device)
        neg[~visible.to(self.device)] = float("-inf")
        h = x.float()
        for l in range(c.n_layers):
            p = f"layers.{l}."
            xn = self.rms(h, w[p + "input_layernorm"])
            q = (xn @ w[p + "q_proj"].T).view(T, c.n_q_heads, c.head_dim)
            k = (xn @ w[p + "k_proj"].T).view(T, c.n_kv_heads, c.head_dim)
            v = (xn @ w[p + "v_proj"].T).view(T, c.n_kv_heads, c.head_dim)
            q, k = self.rope(q, pos), self.rope(k, pos)
            cache.k[l, wp] = k
            cache.v[l, wp] = v
            kk, vv = cache.k[l, :L], cache.v[l, :L]                                   # [L, kvh, d]
            qg = q.view(T, c.n_kv_heads, g, c.head_dim)
            s = torch.einsum("tngd,lnd->ngtl", qg, kk) * scale + neg                  # [kvh, g, T, L]
            pr = torch.softmax(s, dim=-1)
            o = torch.einsum("ngtl,lnd->tngd", pr, vv).reshape(T, c.q_dim)
            a = o @ w[p + "o_proj"].T
            h = h + self.rms(a, w[p + "post_self_attn_layernorm"])
            xm = self.rms(h, w[p + "post_attention_layernorm"])
            gu = xm @ w[p + "gate_up_proj"].T
            gate, up = gu[:, : c.intermediate], gu[:, c.intermediate:]
            m = (up * torch.nn.functional.silu(gate)) @ w[p + "down_proj"].T
            h = h + self.rms(m, w[p + "post_mlp_layernorm"])
        return h

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        return self.rms(h, self.w["norm"]) @ self.w["lm_head"].T

    # ------------------------------------------------------------------ prefill / AR
    def prefill(self, x: torch.Tensor, capacity: int, pos3: Optional[torch.Tensor] = None
                ) -> Tuple[OracleCache, torch.Tensor]:
        """Causal pass over the prefix rows x [P, hidden] (RoPE positions 0..P-1, or pos3 [3, P] multimodal);
        returns (cache, last-row logits [V])."""
        P = x.shape[0]
        cache = self.new_cache(capacity)
        wpos = torch.arange(P)
        rpos = wpos if pos3 is None else pos3.T.contiguous()
        vis = torch.ones((P, P), dtype=torch.bool).tril()
        h = self.forward(x, rpos, cache, wpos, vis)
        return cache, self.logits(h[-1:])[0]

    def ar_greedy(self, x: torch.Tensor, n_new: int) -> List[int]:
        """Greedy AR decode (argmax of the fp32 logits, lowest index on ties) of n_new tokens after the prefix."""
        P = x.shape[0]
        cache, lg = self.prefill(x, P + n_new + 1)
        out = [int(lg.argmax())]
        for t in range(1, n_new):
            p = P + t - 1
            vis = torch.ones((1, p + 1), dtype=torch.bool)
            h = self.forward(self.embed(torch.tensor([out[-1]])), torch.tensor([p]), cache, torch.tensor([p]), vis)
            out.append(int(self.logits(h)[0].argmax()))
        return out

    def teacher_force(self, x: torch.Tensor, gen: List[int], chunk: int = 512, pos3: Optional[torch.Tensor] = None
                      ) -> Tuple[List[int], List[float], torch.Tensor]:
        """One causal pass over prefix + gen (``src/fast_sampling.py:631-690``): for every i, the argmax (and the top-2
        logit gap) of the logits that predict gen[i] from gen[:i].  pos3 [3, P]: multimodal prefix positions, gen
        token i then at max + 1 + i on every axis.  Returns (argmax list, gap list, logits [n, V])."""
        P, n = x.shape[0], len(gen)
        seq = torch.cat([x.float(), self.embed(torch.tensor(gen[:-1], dtype=torch.int64))], dim=0) if n > 1 else x.float()
        T = seq.shape[0]
        cache = self.new_cache(T)
        rope = None
        if pos3 is not None:
            nxt = int(pos3.max()) + 1
            rope = torch.cat([pos3.T, (torch.arange(T - P) + nxt)[:, None].expand(-1, 3)], dim=0)
        hs = []
        for s0 in range(0, T, chunk):
            s1 = min(T, s0 + chunk)
            pos = torch.arange(s0, s1)
            vis = torch.arange(s1)[None, :] <= pos[:, None]
            hs.append(self.forward(seq[s0:s1], pos if rope is None else rope[s0:s1], cache, pos, vis))
        h = torch.cat(hs, dim=0)[P - 1: P - 1 + n]
        lg = self.logits(h)
        top = torch.topk(lg, 2, dim=-1).values
        return lg.argmax(-1).tolist(), (top[:, 0] - top[:, 1]).tolist(), lg


# ---------------------------------------------------------------------- natcache form (pins the oracle to the reference)
def natcache_generate(model: OracleDecoder, x: torch.Tensor, max_new_tokens: int, bd: int,
                      trace: Optional[list] = None, pos3: Optional[torch.Tensor] = None) -> List[int]:
    """Restatement of ``generate_speculative_natcache`` (``src/fast_sampling.py:425-612``) with temperature 0,
    draft_steps=1, full_draft=True, accept_conf=0 and no EOS.  Greedy picks are ``softmax(logits.float()).argmax``
    (``src/models/glm_ocr_dllm.py:997-1002``).  pos3 [3, P]: the prefix's multimodal positions; response token r then
    sits at position next_pos + r on every axis, next_pos = max(pos3) + 1 (``comb_pos``, :505-506)."""
    c = model.cfg
    mask_id = c.mask_id
    P = x.shape[0]
    next_pos = P if pos3 is None else int(pos3.max()) + 1
    cap = P + max_new_tokens + 2 * bd + 8
    cache, seed_logit = model.prefill(x, cap, pos3)
    seed_logit = seed_logit[None]                                            # [1, V]
    clen = P
    committed: List[int] = []
    pending: Optional[int] = None
    greedy = lambda lg: torch.softmax(lg.float(), dim=-1).argmax(-1)
    while len(committed) < max_new_tokens:
        pre = 1 if pending is not None else 0
        Q = pre + bd
        r0 = clen - P
        ids = ([pending] if pre else []) + [mask_id] * bd
        pos = torch.arange(next_pos + r0, next_pos + r0 + Q)
        wpos = torch.arange(clen, clen + Q)
        qi = torch.arange(Q)[:, None]
        kv = torch.arange(clen + Q)[None, :]
        vis = (kv < clen) | (qi >= pre) | ((kv - clen) <= qi)                # fast_sampling.py:508-510
        raw = model.logits(model.forward(model.embed(torch.tensor(ids)), pos, cache, wpos, vis))    # [Q, V]
        used = torch.cat([raw[:1], raw[:-1]], 0) if pre else torch.cat([seed_logit, raw[:-1]], 0)
        block = greedy(used[pre:])                                           # [bd]
        x_extra = greedy(raw[-1:])                                           # the last mask predicts d_bd
        draft = torch.cat([block, x_extra]).tolist()                         # a0, d1..d_bd
        Qv = Q + 1
        vids = ([pending] if pre else []) + draft
        pos_v = torch.arange(next_pos + r0, next_pos + r0 + Qv)
        wpos_v = torch.arange(clen, clen + Qv)
        qi = torch.arange(Qv)[:, None]
        kv = torch.arange(clen + Qv)[None, :]
        vis_v = (kv < clen) | ((kv - clen) <= qi)                            # fast_sampling.py:512-514
        lv = model.logits(model.forward(model.embed(torch.tensor(vids)), pos_v, cache, wpos_v, vis_v))
        pred = torch.cat([lv[:1] if pre else seed_logit, lv[:-1]], 0)[pre:]
        ar_pred = greedy(pred).tolist()
        bonus = int(lv[-1].float().argmax())
        k = next((i for i in range(len(draft)) if draft[i] != ar_pred[i]), len(draft))
        new = draft[:k] + [ar_pred[k]] if k < len(draft) else draft + [bonus]
        m = len(new)
        clen = clen + pre + (m - 1)
        pending = new[-1]
        committed += new
        if trace is not None:
            trace.append({"k": k, "draft": draft, "ar_pred": ar_pred, "new_tokens": new})
    return committed


# ---------------------------------------------------------------------- served full-draft form (what the CUDA path does)
@dataclass
class SpecState:
    """One request's round state by logical position: ``seq_len`` tokens have K/V, ``seed`` (x0) is committed but has
    no K/V yet, ``out`` holds every committed token (the prefill's first token included)."""

    cache: OracleCache
    seq_len: int
    seed: int
    out: List[int]
    prefix_len: int
    pos_delta: int = 0          # RoPE position - cache position (multimodal prefixes)


def spec_start(model: OracleDecoder, x: torch.Tensor, capacity: int, pos3: Optional[torch.Tensor] = None
               ) -> SpecState:
    """Prefill; the first generated token (argmax of the last prefix logit) becomes the first seed."""
    cache, lg = model.prefill(x, capacity, pos3)
    s = int(lg.argmax())
    delta = 0 if pos3 is None else int(pos3.max()) + 1 - x.shape[0]
    return SpecState(cache, x.shape[0], s, [s], x.shape[0], delta)


def spec_draft(model: OracleDecoder, st: SpecState, K: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Draft forward over [seed | mask x (K-1)] at positions S..S+K-1: row 0 sees kv[0..S], mask rows see
    kv[0..S+K-1].  Returns (am [K] argmax per row = [a0, d1..d_{K-1}], logits [K, V])."""
    S = st.seq_len
    ids = torch.tensor([st.seed] + [model.cfg.mask_id] * (K - 1))
    pos = torch.arange(S, S + K)
    kv = torch.arange(S + K)[None, :]
    lim = torch.full((K, 1), S + K)
    lim[0, 0] = S + 1
    lg = model.logits(model.forward(model.embed(ids), pos + st.pos_delta, st.cache, pos, kv < lim))
    return lg.argmax(-1), lg


def spec_verify(model: OracleDecoder, st: SpecState, vids: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Causal verify over vids = [a0, d1..d_{K-1}] at positions S+1..S+K (x0's draft K/V at S is kept).
    Returns (v [K] argmax per row, logits [K, V])."""
    S, K = st.seq_len, vids.shape[0]
    pos = torch.arange(S + 1, S + 1 + K)
    kv = torch.arange(S + 1 + K)[None, :]
    lim = torch.arange(S + 2, S + 2 + K)[:, None]
    lg = model.logits(model.forward(model.embed(vids), pos + st.pos_delta, st.cache, pos, kv < lim))
    return lg.argmax(-1), lg


def forced_draft(am: torch.Tensor, g: List[int], c: int, A: int, vocab: int, mask_id: int) -> torch.Tensor:
    """Forced-accept replay: d_j = g[c + j] for 1 <= j <= A, then d_{A+1} = (g[c + A + 1] + 1) mod V (skipping
    mask_id), where c is the stream index of a0.  Entries past A+1 keep the model's draft."""
    d = am.clone()
    K = d.shape[0]
    for j in range(1, min(A, K - 1) + 1):
        d[j] = g[c + j]
    if A + 1 <= K - 1:
        t = (g[c + A + 1] + 1) % vocab
        if t == mask_id:
            t = (t + 1) % vocab
        d[A + 1] = t
    return d


def spec_commit(st: SpecState, am: Sequence[int], v: Sequence[int]) -> Dict[str, object]:
    """Accept (linear chain) and commit by logical positions: T = [a0] + v[0..acc], K/V kept through x0 and the
    verify rows 0..acc, next seed = v[acc], released positions S+acc+2..S+K."""
    from .commit_ref import chain_accept, released_positions

    am, v = [int(t) for t in am], [int(t) for t in v]
    K = len(am)
    acc = chain_accept(am, v)
    T = [am[0]] + v[: acc + 1]
    S0 = st.seq_len
    released = released_positions(S0, acc, K)
    st.seq_len = S0 + acc + 2
    st.seed = T[-1]
    st.out += T
    return {"am": am, "v": v, "acc": acc, "T": T, "S0": S0, "released": released}


def spec_round(model: OracleDecoder, st: SpecState, K: int,
               override: Optional[Callable[[torch.Tensor, SpecState], torch.Tensor]] = None) -> Dict[str, object]:
    """One full-draft round: draft, (optional draft override), verify, chain accept, commit by logical positions."""
    am, dlg = spec_draft(model, st, K)
    if override is not None:
        am = override(am, st)
    v, vlg = spec_verify(model, st, am)
    r = spec_commit(st, am.tolist(), v.tolist())
    r["draft_logits"], r["verify_logits"] = dlg, vlg
    return r


def spec_generate(model: OracleDecoder, x: torch.Tensor, n_new: int, K: int,
                  override=None, trace: Optional[list] = None) -> List[int]:
    st = spec_start(model, x, x.shape[0] + n_new + 2 * K + 8)
    while len(st.out) < n_new:
        r = spec_round(model, st, K, override)
        if trace is not None:
            trace.append({k: v for k, v in r.items() if not k.endswith("logits")})
    return st.out[:n_new]


def near_tie_report(stream: List[int], tf_argmax: List[int], tf_gap: List[float], tol: float = 1e-3) -> Dict[str, list]:
    """Positions where ``stream`` differs from the teacher-forced argmax; each must be a near-tie (gap < tol)."""
    bad, ties = [], []
    for i, (a, b) in enumerate(zip(stream, tf_argmax)):
        if a != b:
            (ties if tf_gap[i] < tol else bad).append((i, a, b, tf_gap[i]))
    return {"near_ties": ties, "mismatches": bad}


def hbm_bytes_per_forward(cfg, seq_lens: List[int], K: int, verify: bool) -> int:
    """Algorithmic bytes of one forward: streamed weights + K/V read + K/V written (bf16).  K/V read counts the
    committed prefix S plus delta (1 for the draft, 2 for the verify, which also sees x0)."""
    per_tok = cfg.kv_bytes_per_token()
    delta = 2 if verify else 1
    rd = sum((s + delta) for s in seq_lens) * per_tok
    wr = len(seq_lens) * K * per_tok
    return cfg.streamed_params() * 2 + rd + wr


__all__ = ["OracleDecoder", "OracleCache", "natcache_generate", "SpecState", "spec_start", "spec_draft",
           "spec_verify", "spec_commit", "spec_round", "spec_generate", "forced_draft", "near_tie_report", "hbm_bytes_per_forward"]

_ = math
