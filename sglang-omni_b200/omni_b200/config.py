"""Talker / code-predictor geometry and sampling defaults.

Field names follow the Qwen3 talker configs the reference reads
(sglang_omni/models/qwen3_omni/hf_config.py:271-342;
sglang_omni/models/qwen3_tts/sglang_model.py:447-490): hidden_size,
num_attention_heads, num_key_value_heads, head_dim, intermediate_size,
num_code_groups, rope_theta, rms_norm_eps.
"""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass(frozen=True)
class PredictorConfig:
    """The residual-codebook predictor (the Qwen3-TTS "subtalker")."""

    num_hidden_layers: int = 5
    hidden_size: int = 1024
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 64
    intermediate_size: int = 3072
    vocab_size: int = 2048
    num_code_groups: int = 16  # layer-0 code + 15 residual codebooks
    rope_theta: float = 1e6
    rms_norm_eps: float = 1e-6

    @property
    def cache_len(self) -> int:
        # slots per request: the talker hidden, the layer-0 embedding, 14 residual inputs (+1 spare)
        return self.num_code_groups + 1


@dataclass(frozen=True)
class MoEConfig:
    num_experts: int = 128
    num_experts_per_tok: int = 8
    moe_intermediate_size: int = 384
    shared_expert_intermediate_size: int = 1536
    norm_topk_prob: bool = True
    fp8_block: int = 128  # e4m3 experts with per-128x128 fp32 scales


@dataclass(frozen=True)
class TalkerConfig:
    num_hidden_layers: int = 20
    hidden_size: int = 1024
    num_attention_heads: int = 16
    num_key_value_heads: int = 2
    head_dim: int = 128
    intermediate_size: int = 3072
    vocab_size: int = 3072  # codec vocabulary of the layer-0 head
    rope_theta: float = 1e6
    rms_norm_eps: float = 1e-6
    page_size: int = 16
    max_context: int = 8192
    moe: MoEConfig | None = None
    predictor: PredictorConfig = field(default_factory=PredictorConfig)


@dataclass(frozen=True)
class SamplingParams:
    """Per-request sampling of the layer-0 codec token and of the residual codebooks
    (request_builders.py:135-143, 162-166, 1796)."""

    temperature: float = 0.9
    top_k: int = 50
    top_p: float = 0.8
    min_p: float = 0.0
    repetition_penalty: float = 1.05
    subtalker_dosample: bool = True
    subtalker_temperature: float = 0.9
    subtalker_top_k: int = 50
    subtalker_top_p: float = 0.8


# The configurations of the benchmark (BASELINE.json "configs").
CONFIG0_PREDICTOR = PredictorConfig()
CONFIG1_DENSE = TalkerConfig()
CONFIG3_MOE = TalkerConfig(moe=MoEConfig(), predictor=PredictorConfig(vocab_size=1024, num_code_groups=32))
