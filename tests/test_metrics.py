"""The roofline numerators: a one-token prefill is one one-row forward with one visible position (less the final
norm's weights, which the prefill's lm_head row skips), the counts add over requests, and causal attention grows with
n (n + 1) / 2 visible positions."""
from gravityocr_b200.config import ModelConfig, small_model
from gravityocr_b200.metrics import forward_flops, prefill_flops


def test_one_token_prefill_is_one_forward_row():
    for cfg in (ModelConfig(), small_model(2)):
        assert prefill_flops(cfg, [1]) == forward_flops(cfg, [0], 1, False) - 2 * cfg.hidden


def test_prefill_flops_add_over_requests_and_attention_is_causal():
    cfg = ModelConfig()
    a, b = prefill_flops(cfg, [300]), prefill_flops(cfg, [4128])
    assert prefill_flops(cfg, [300, 4128]) == a + b
    per_pos = 4 * cfg.n_q_heads * cfg.head_dim * cfg.n_layers
    # one more token: its weights, its row of lm_head replaces the previous last token's, and n + 1 more positions
    step = prefill_flops(cfg, [301]) - a
    weights = 2 * (cfg.streamed_params() - cfg.vocab * cfg.hidden - cfg.hidden)
    assert step == weights + per_pos * 301
