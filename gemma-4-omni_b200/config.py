"""Shape/constant configuration of the streaming listener step.

Constants mirror the reference contracts:
- duplex_kernel/streaming_conformer.py:18-23 (MEL_TICK_ROWS, MEL_BINS, Q2_TOKENS,
  MAX_PAST_TOKENS, CACHED_PAST_TOKENS, ATTENTION_CHUNK_SIZE)
- duplex_kernel/microbatch_contract.py:19-33 (PCM_SAMPLES_PER_FRAME,
  PCM_TAIL_SAMPLES, CONTROL_HIDDEN_WIDTH, MEL_BINS)
- transformers Gemma4AudioConfig defaults (models/gemma4/configuration_gemma4.py:52-72)
"""
from __future__ import annotations

import math
from dataclasses import asdict, dataclass

MEL_TICK_ROWS = 8
MEL_BINS = 128
Q2_TOKENS = 2
MAX_PAST_TOKENS = 12
CACHED_PAST_TOKENS = 13
ATTENTION_CHUNK_SIZE = 12
PCM_SAMPLES_PER_FRAME = 1280
PCM_TAIL_SAMPLES = 160
CONTROL_HIDDEN_WIDTH = 1536
SAMPLE_RATE_HZ = 16_000
FRAME_PERIOD_S = 0.080

WEIGHT_BF16 = 0
WEIGHT_INT8 = 1


@dataclass(frozen=True)
class ListenerConfig:
    """One audio tower (+ optional FiLM adapter) served by a listener context."""

    hidden: int = 1536
    layers: int = 12
    heads: int = 8
    ffn: int = 6144
    sub_ch0: int = 128
    sub_ch1: int = 32
    output_dims: int = 1536
    text_hidden: int = 1536
    conv_kernel: int = 5
    rms_eps: float = 1e-6
    softcap: float = 50.0
    invalid_logit: float = -1.0e9
    gradient_clipping: float = 1e10
    residual_weight: float = 0.5
    film_enabled: bool = True
    film_query_dim: int = 2048
    film_bottleneck: int = 256
    film_max_scale: float = 0.25

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def sub_freq0(self) -> int:
        return (MEL_BINS + 1) // 2

    @property
    def sub_freq1(self) -> int:
        return (self.sub_freq0 + 1) // 2

    @property
    def sub_proj_in(self) -> int:
        return self.sub_ch1 * self.sub_freq1

    def validate(self) -> None:
        if self.hidden % self.heads:
            raise ValueError("hidden must divide evenly across heads")
        if self.conv_kernel != 5:
            raise ValueError("the streaming listener requires conv_kernel_size 5")
        for name in ("hidden", "ffn", "output_dims", "text_hidden"):
            if getattr(self, name) % 128:
                raise ValueError(f"{name} must be a multiple of 128 for the tensor-core tiles")
        if self.sub_proj_in % 64:
            raise ValueError("subsampler projection width must be a multiple of 64")
        if self.head_dim % 32 or self.head_dim > 256:
            raise ValueError("head_dim must be a multiple of 32 and at most 256")
        if self.sub_ch0 != 128 or self.sub_ch1 % 32:
            raise ValueError("subsampler channels must be (128, multiple of 32)")
        if self.film_enabled and (self.film_query_dim % 128 or self.film_bottleneck % 128):
            raise ValueError("FiLM widths must be multiples of 128")

    def to_dict(self) -> dict:
        return asdict(self)


# BASELINE config 0..4 audio tower: d=1536, 12 layers, 8 heads, FFN 6144, conv 5,
# chunk 12 / left 13 / right 0, subsampling (128, 32), output 1536.
FULL = ListenerConfig()
# Small tower used for fast parity cases (same code paths, smaller widths).
SMALL = ListenerConfig(hidden=256, layers=2, heads=2, ffn=1024, output_dims=256, text_hidden=256,
                       film_query_dim=256, film_bottleneck=128)

FILM_ALPHA = 0.0513  # BASELINE: FiLM scale = 0.25 * sigmoid(scale_logit)
FILM_SCALE_LOGIT = math.log((FILM_ALPHA / 0.25) / (1.0 - FILM_ALPHA / 0.25))
