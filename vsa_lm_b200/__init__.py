"""B200-native (sm_100a) Bolt-3 dual-field attention: drop-in `Bolt3Attn` and `Bolt3Decoder`.

The kernels live in libbolt3.so (C-ABI: include/bolt3.h), built in-tree by `vsa_lm_b200.build`.
"""
from .bolt3 import AnchorKV, Bolt3Attn, Bolt3Decoder, Bolt3LayerState, LlamaRMSNorm, LlamaRoPE, StaticKV, llama_inv_freq

__all__ = ["AnchorKV", "Bolt3Attn", "Bolt3Decoder", "Bolt3LayerState", "LlamaRMSNorm", "LlamaRoPE", "StaticKV",
           "llama_inv_freq"]
