"""B200-native streaming listener step (PCM -> log-mel -> Gemma 4 audio Conformer
with per-session caches -> soft tokens -> FiLM residual).

The package directory is ``gemma-4-omni_b200``; it is imported under the name
``gemma4_omni_b200`` (see ``load_package`` in the repository's entry points).
"""
from .config import FULL, SMALL, WEIGHT_BF16, WEIGHT_INT8, ListenerConfig  # noqa: F401

__all__ = ["ListenerConfig", "FULL", "SMALL", "WEIGHT_BF16", "WEIGHT_INT8"]
