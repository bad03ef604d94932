"""Kernel package: importing it registers the attention specifications."""

from tklab.kernels.flash_attention import ATTENTION_CAUSAL, ATTENTION_NONCAUSAL
from tklab.kernels.rope_attention import ATTENTION_ROPE_CAUSAL, ATTENTION_ROPE_NONCAUSAL

__all__ = ["ATTENTION_CAUSAL", "ATTENTION_NONCAUSAL", "ATTENTION_ROPE_CAUSAL", "ATTENTION_ROPE_NONCAUSAL"]
