"""Model, round and workload configuration for the self-speculative decode round.

The decoder is GLM-OCR's text stack (transformers ``GlmOcrTextDecoderLayer``): sandwich RMSNorm, GQA attention with
interleaved-pair partial RoPE, SwiGLU MLP whose ``gate_up_proj`` holds the gate in its first half.  The round is the
full-draft round of the reference SGLang worker
(``patches/sglang/python/sglang/srt/speculative/selfspec_diffusion_worker.py:660-998``): a draft forward over
``[x0 | mask x B]`` (K = B + 1 rows), a causal verify forward over ``[a0, d1..dB]`` (K rows) and one accept-and-commit.

Workload presets restate the five configurations the baseline names (seeded synthetic inputs stand in for the
OmniDocBench crops, which are not available).
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass, field
from typing import List, Tuple


@dataclass(frozen=True)
class ModelConfig:
    """GLM-OCR-shaped decoder.  Defaults are the baseline architecture (configs 0-4)."""

    n_layers: int = 16
    hidden: int = 1536
    n_q_heads: int = 16
    n_kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 4608
    vocab: int = 59392
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    # partial_rotary_factor 0.5: at head_dim 128 the default M-RoPE sections [8, 12, 12] (sum 32 frequencies)
    # require a rotary dimension of 64 (transformers modeling_glm_ocr.py GlmOcrTextRotaryEmbedding).
    rotary_dim: int = 64
    # GLM-OCR's <|mask|> id (reference MODEL_CARD.md:98-100; worker _resolve_block_diffusion error text).
    mask_id: int = 59282
    image_token_id: int = 59280
    # M-RoPE: rotary pairs [0, 8) rotate by the temporal position, [8, 20) by the row, [20, 32) by the column
    # (transformers GlmOcrTextRotaryEmbedding mrope_section); text tokens have three equal positions.
    mrope_section: Tuple[int, int, int] = (8, 12, 12)

    @property
    def q_dim(self) -> int:
        return self.n_q_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return self.q_dim + 2 * self.kv_dim

    def streamed_params(self) -> int:
        """Parameters read per forward: every layer weight, the final norm and lm_head (embedding rows excluded)."""
        h, i = self.hidden, self.intermediate
        per_layer = self.qkv_dim * h + h * self.q_dim + 2 * i * h + h * i + 4 * h
        return self.n_layers * per_layer + h + self.vocab * h

    def kv_bytes_per_token(self) -> int:
        """bf16 K and V bytes of one token over all layers."""
        return 2 * self.n_kv_heads * self.head_dim * 2 * self.n_layers


@dataclass(frozen=True)
class RoundConfig:
    """Self-spec round shape: bd_size B draft tokens behind the boundary token x0 (K = B + 1 rows per forward)."""

    bd_size: int = 16
    page_size: int = 16

    @property
    def K(self) -> int:
        return self.bd_size + 1


@dataclass
class Workload:
    """One of the baseline's workloads, restated with seeded synthetic inputs."""

    name: str
    model: ModelConfig
    seed: int
    batch: int
    n_image: Tuple[int, int]          # image-embedding prefix length range (inclusive)
    n_prompt: int
    out_len: Tuple[int, int]          # generated tokens range (inclusive)
    bd_sizes: List[int] = field(default_factory=lambda: [16])
    dtype: str = "bf16"


def preset(idx: int) -> Workload:
    m = ModelConfig()
    if idx == 0:
        return Workload("config0-cpu-roundtrip", m, seed=0, batch=1, n_image=(256, 256), n_prompt=32,
                        out_len=(128, 128), dtype="fp32")
    if idx == 2:
        return Workload("config2-bs1-crop", m, seed=2, batch=1, n_image=(256, 256), n_prompt=32,
                        out_len=(1024, 1024))
    if idx == 3:
        return Workload("config3-bs64-serving", m, seed=3, batch=64, n_image=(256, 4096), n_prompt=32,
                        out_len=(256, 2048))
    if idx == 4:
        return Workload("config4-fullpage-sweep", m, seed=4, batch=128, n_image=(4096, 4096), n_prompt=64,
                        out_len=(4096, 4096), bd_sizes=[4, 8, 16, 32])
    raise ValueError(f"no preset {idx} (config 1 is the attention op alone)")


def small_model(n_layers: int = 2, vocab: int = 59392) -> ModelConfig:
    """Reduced-depth model with the baseline's per-layer geometry, for quick parity tests."""
    return dataclasses.replace(ModelConfig(), n_layers=n_layers, vocab=vocab)
