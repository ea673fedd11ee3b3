"""B200 (sm_100a) decode megakernel for Llama-3.2-1B.

One persistent CUDA launch decodes a token for every sequence in the batch:
all decoder layers, the final norm, the tied lm_head and greedy argmax. The
kernel lives in ``csrc/`` behind a C ABI (``include/mk.h``) and is driven from
the PyTorch module in ``model.py``.
"""
from .config import LLAMA_3_2_1B, SMALL, TINY, LlamaDecodeConfig

__all__ = ["LlamaDecodeConfig", "LLAMA_3_2_1B", "SMALL", "TINY"]
