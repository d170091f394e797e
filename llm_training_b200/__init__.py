"""B200-native (sm_100a) two-level sqrt-block attention for the LLM_training GPT trainer.

``ops.sqrt_block_attention`` is the differentiable op; ``model`` holds the
``BaseAttention`` plugin registry and the ``sqrt_block`` plugin; the kernels and
the C ABI (include/sqrtblock.h) live in ``csrc`` and build into ``lib/``.
"""

__version__ = "0.1.0"
