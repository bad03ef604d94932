"""Kernel package: importing it registers the attention specifications."""

from tklab.kernels.flash_attention import ATTENTION_CAUSAL, ATTENTION_NONCAUSAL

__all__ = ["ATTENTION_CAUSAL", "ATTENTION_NONCAUSAL"]
