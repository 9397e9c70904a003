"""Attention, KV cache and RoPE operators on the B200 kernels."""
