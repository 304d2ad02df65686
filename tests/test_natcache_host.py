"""Host side of the natcache drop-in (no GPU): the reference model's decoder configuration and weights are read from
the transformers module tree exactly as the engine lays them out."""
import types

import torch

from gravityocr_b200.compat.natcache import _text_config, _text_weights
from gravityocr_b200.config import small_model
from gravityocr_b200.weights import weight_shapes


def _ref_shaped(cfg):
    from transformers import GlmOcrConfig, GlmOcrForConditionalGeneration
    hf = GlmOcrConfig()
    tc = hf.text_config
    tc.num_hidden_layers, tc.hidden_size = cfg.n_layers, cfg.hidden
    tc.num_attention_heads, tc.num_key_value_heads, tc.head_dim = cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
    tc.intermediate_size, tc.vocab_size, tc.rms_norm_eps = cfg.intermediate, cfg.vocab, cfg.rms_eps
    tc.rope_parameters = {"rope_theta": cfg.rope_theta, "rope_type": "default",
                          "partial_rotary_factor": cfg.rotary_dim / cfg.head_dim, "mrope_section": [8, 12, 12]}
    hf.vision_config.depth = 1
    with torch.device("meta"):
        glm = GlmOcrForConditionalGeneration(hf)
    m = types.SimpleNamespace(glm=glm, mask_id=cfg.mask_id, image_token_id=cfg.image_token_id,
                              text_model=glm.model.language_model)
    return m


def test_reference_model_maps_to_engine_layout():
    cfg = small_model(2)
    m = _ref_shaped(cfg)
    assert _text_config(m) == cfg
    w = _text_weights(m)
    assert sorted(w) == sorted(n for n, _ in weight_shapes(cfg))
    for name, shape in weight_shapes(cfg):
        assert tuple(w[name].shape) == shape, name
    assert w["lm_head"] is m.glm.lm_head.weight.detach() or w["lm_head"].shape == m.glm.lm_head.weight.shape
    assert w["layers.1.gate_up_proj"].shape == (2 * cfg.intermediate, cfg.hidden)
