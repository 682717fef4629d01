"""B200-native fused 4-bit AdamW (drop-in for nubank/adamw4bit's optimizer API).

``optimizer.step()`` runs hand-written sm_100a CUDA kernels (libadamw4bit_b200.so,
C ABI in include/adamw4bit_b200.h) through ctypes; there is no CPU path.
"""

from .optimizer import AdamW8bit, QuantizedAdamW, ZEEDENAdamW4Bit, ZIPSRAdamW4Bit

__all__ = ["QuantizedAdamW", "ZIPSRAdamW4Bit", "ZEEDENAdamW4Bit", "AdamW8bit"]
