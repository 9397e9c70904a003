"""W4A4 quantized linears on the B200 kernels."""
