"""Algorithmic byte and FLOP counts of the round (the roofline numerators).

Per forward over a batch with committed lengths S_b (x0 not in K/V) and K = B + 1 rows per request:
  weights  W     = streamed parameters (every layer weight, final norm, lm_head) x 2 B
  K/V read KV_rd = sum_b (S_b + delta) x 65,536 B   (delta 1 for the draft, 2 for the verify, which also sees x0)
  K/V write KV_wr = bs x K x 65,536 B
  logits   0     (lm_head is fused with the argmax)
FLOPs = 2 x streamed params x bs x K  +  4 x K x n_q_heads x head_dim x sum_b (S_b + delta) x layers.
"""
from __future__ import annotations

from typing import Sequence

from .config import ModelConfig


def forward_bytes(cfg: ModelConfig, seq_lens: Sequence[int], K: int, verify: bool) -> int:
    per_tok = cfg.kv_bytes_per_token()
    delta = 2 if verify else 1
    return cfg.streamed_params() * 2 + sum(int(s) + delta for s in seq_lens) * per_tok + len(seq_lens) * K * per_tok


def forward_flops(cfg: ModelConfig, seq_lens: Sequence[int], K: int, verify: bool) -> int:
    delta = 2 if verify else 1
    attn = 4 * K * cfg.n_q_heads * cfg.head_dim * sum(int(s) + delta for s in seq_lens) * cfg.n_layers
    return 2 * cfg.streamed_params() * len(seq_lens) * K + attn


def attention_bytes(cfg: ModelConfig, seq_lens: Sequence[int], K: int, base_add: int) -> int:
    """One attention launch (one layer): K and V of every visible position, q in, out out."""
    kv = sum(int(s) + base_add + K for s in seq_lens) * cfg.n_kv_heads * cfg.head_dim * 2 * 2
    qo = 2 * len(seq_lens) * K * cfg.q_dim * 2
    return kv + qo


def prefill_flops(cfg: ModelConfig, prefix_lens: Sequence[int]) -> int:
    """Dense causal prefill of each prefix (the algorithmic work, whatever the chunking): every decoder weight once per
    prefix token, causal attention (token t sees t + 1 positions), and lm_head for each request's last token."""
    decoder = cfg.streamed_params() - cfg.vocab * cfg.hidden - cfg.hidden
    n = sum(int(x) for x in prefix_lens)
    causal = sum(int(x) * (int(x) + 1) // 2 for x in prefix_lens)
    attn = 4 * cfg.n_q_heads * cfg.head_dim * causal * cfg.n_layers
    return 2 * decoder * n + attn + 2 * cfg.vocab * cfg.hidden * len(prefix_lens)
