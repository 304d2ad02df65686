"""Seeded random-init weights and synthetic request inputs (no checkpoint or dataset is available).

Weights follow the baseline: every parameter (norm weights included) is drawn N(0, 0.02).  The draw order is fixed
here so the CUDA path, the CPU oracle and the reference's own transformers model (loaded with the same tensors by
``tests/golden/make_golden.py``) all hold identical values.  Names are transformers' GLM-OCR parameter names with
the ``model.language_model.`` prefix dropped.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import torch

from .config import ModelConfig

INIT_STD = 0.02


def weight_shapes(cfg: ModelConfig) -> List[Tuple[str, Tuple[int, ...]]]:
    h, i = cfg.hidden, cfg.intermediate
    out: List[Tuple[str, Tuple[int, ...]]] = [("embed_tokens", (cfg.vocab, h))]
    for l in range(cfg.n_layers):
        p = f"layers.{l}."
        out += [
            (p + "q_proj", (cfg.q_dim, h)),
            (p + "k_proj", (cfg.kv_dim, h)),
            (p + "v_proj", (cfg.kv_dim, h)),
            (p + "o_proj", (h, cfg.q_dim)),
            (p + "gate_up_proj", (2 * i, h)),
            (p + "down_proj", (h, i)),
            (p + "input_layernorm", (h,)),
            (p + "post_self_attn_layernorm", (h,)),
            (p + "post_attention_layernorm", (h,)),
            (p + "post_mlp_layernorm", (h,)),
        ]
    out += [("norm", (h,)), ("lm_head", (cfg.vocab, h))]
    return out


def random_weights(cfg: ModelConfig, seed: int, dtype: torch.dtype = torch.bfloat16,
                   embed_std: float = INIT_STD, norm_center: float = 0.0,
                   qk_std: float = INIT_STD) -> Dict[str, torch.Tensor]:
    """N(0, 0.02) for every tensor, drawn in ``weight_shapes`` order from one CPU generator.

    The values are drawn in fp32 and rounded once to ``dtype``; with dtype=float32 nothing is rounded.
    ``embed_std`` scales the token-embedding table only (same draw, multiplied by embed_std / 0.02).  At the baseline's
    0.02 every sublayer adds a vector of the same size as the token's own embedding, the context dominates and greedy
    streams settle on one repeated token within a few steps; at 0.25 the token identity carries through the 16 layers
    and streams stay varied, which the parity fixtures use to exercise rejections and rollbacks.
    ``norm_center`` is added to every RMSNorm weight (1.0 gives norm weights near one, as a trained model has, so each
    sublayer's output carries weight in the residual) and ``qk_std`` rescales the q/k projections (sharper attention);
    together they make the committed stream depend on the RoPE positions, which the multimodal-position fixtures
    need.  Defaults reproduce the baseline draw exactly."""
    g = torch.Generator().manual_seed(int(seed))
    w: Dict[str, torch.Tensor] = {}
    for name, shape in weight_shapes(cfg):
        t = torch.empty(shape, dtype=torch.float32)
        t.normal_(0.0, INIT_STD, generator=g)
        if name == "embed_tokens" and embed_std != INIT_STD:
            t.mul_(embed_std / INIT_STD)
        if (name.endswith("_proj") and name.split(".")[-1] in ("q_proj", "k_proj")) and qk_std != INIT_STD:
            t.mul_(qk_std / INIT_STD)
        if (name.endswith("layernorm") or name == "norm") and norm_center:
            t.add_(norm_center)
        w[name] = t if dtype == torch.float32 else t.to(dtype)
    return w


def request_inputs(cfg: ModelConfig, seed: int, n_image: int, n_prompt: int, index: int = 0,
                   dtype: torch.dtype = torch.bfloat16) -> Tuple[torch.Tensor, torch.Tensor]:
    """Synthetic prefix of one request: ``n_image`` image-embedding vectors N(0,1)*0.02 (injected as inputs_embeds at
    image-token positions) followed by ``n_prompt`` prompt ids uniform in [0, vocab-1) excluding mask_id.

    Returns (image_embeds [n_image, hidden] fp32 holding ``dtype``-rounded values, prompt_ids [n_prompt] int64)."""
    g = torch.Generator().manual_seed(int(seed) * 1_000_003 + 7919 * int(index) + 1)
    img = torch.randn((n_image, cfg.hidden), generator=g, dtype=torch.float32) * 0.02
    if dtype != torch.float32:
        img = img.to(dtype).float()
    ids = torch.randint(0, cfg.vocab - 1, (n_prompt,), generator=g, dtype=torch.int64)
    bad = ids == cfg.mask_id
    while bool(bad.any()):
        ids[bad] = torch.randint(0, cfg.vocab - 1, (int(bad.sum()),), generator=g, dtype=torch.int64)
        bad = ids == cfg.mask_id
    return img, ids


def prefix_token_ids(cfg: ModelConfig, n_image: int, prompt_ids: torch.Tensor) -> torch.Tensor:
    """Prefix ids as the processor lays them out: image placeholder ids, then the prompt ids."""
    return torch.cat([torch.full((n_image,), cfg.image_token_id, dtype=torch.int64), prompt_ids.to(torch.int64)])


def prefix_embeddings(weights: Dict[str, torch.Tensor], cfg: ModelConfig, image_embeds: torch.Tensor,
                      prompt_ids: torch.Tensor) -> torch.Tensor:
    """Layer-0 input of the prefix in fp32: image vectors at image positions, embedding rows elsewhere
    (reference ``src/fast_sampling.py:483-488`` masked_scatter)."""
    e = weights["embed_tokens"][prompt_ids.to(torch.int64)].float()
    return torch.cat([image_embeds.float(), e], dim=0)


def grid_positions(n_image: int, n_prompt: int, grid_w: int) -> torch.Tensor:
    """Multimodal (t, h, w) positions [3, n_image + n_prompt] of a prefix whose image tokens lie on a grid of width
    grid_w (token k at row k // grid_w, column k % grid_w, temporal position 0), followed by the prompt tokens at
    start, start + 1, ... on every axis, start = the largest image position + 1 -- the layout of an image in a
    multimodal RoPE index (transformers GlmOcrModel.get_rope_index), as a synthetic stand-in for a real crop."""
    k = torch.arange(n_image)
    img = torch.stack([torch.zeros_like(k), k // grid_w, k % grid_w])
    start = int(img.max()) + 1 if n_image else 0
    txt = torch.arange(start, start + n_prompt).expand(3, -1)
    return torch.cat([img, txt], dim=1).to(torch.int64)


def variant_weights(cfg: ModelConfig, seed: int, embed_std: float = INIT_STD, variant: Optional[dict] = None
                    ) -> Dict[str, torch.Tensor]:
    """fp32 weights of a fixture: ``random_weights`` with the variant's norm_center / qk_std, rounded through bf16 when
    the variant says ``bf16_weights`` (the values the CUDA path holds)."""
    v = dict(variant or {})
    bf16 = v.pop("bf16_weights", False)
    w = random_weights(cfg, seed, torch.bfloat16 if bf16 else torch.float32, embed_std=embed_std, **v)
    return {k: t.float() for k, t in w.items()}
