"""B200-native (sm_100a) hot path of wan-dit-lab's Wan-5B DiT block forward: W4A4 linears, 3D RoPE, FP8 KV cache
and SageAttention, behind the reference's Python module API. The kernels live in libwdl_b200.so (C ABI,
include/wdl_b200.h) and are reached through `_native`; nothing here falls back to PyTorch compute or the CPU."""

__version__ = "0.1.0"
