"""flash_uma_b200: B200-native (sm_100a) eSCN/UMA message-passing hot path.

Drop-in for FlashUMA's ``ZeroAllocBackbone(backbone, dtype)``; the fused ops run
as hand-written CUDA kernels in ``lib/libflashuma_b200.so`` behind a C ABI
(``include/flash_uma_b200.h``). Importing the package needs no GPU; calling an
op without the built library or without a CUDA device raises.
"""
__version__ = "0.1.0"
