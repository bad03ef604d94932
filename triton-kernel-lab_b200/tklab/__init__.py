"""B200 (sm_100a) drop-in for triton-kernel-lab's flash-attention path.

Import names mirror the reference package (``tklab.registry``,
``tklab.kernels.flash_attention``, ``tklab.harness.tolerances`` ...), so code
and tests written against the reference run unchanged with this directory on
``sys.path``.  The kernels themselves live in ``libtklab_attn.so`` (CUDA for
sm_100a, built from ``csrc/``) and are reached through its C ABI.
"""

__version__ = "0.1.0"
