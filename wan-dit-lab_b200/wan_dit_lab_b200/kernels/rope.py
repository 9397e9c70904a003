"""3D RoPE of Wan on the B200 kernel, with the API and validation of the reference's
src/wan_dit_lab/kernels/rope_triton.py (rope_apply, rope_apply_wan), forward only.

Input (batch, token, heads, dim), any strides; frequencies (cos/sin, position, pair) in float32 or float64.
Token t of the grid (f, h, w) of its sample has positions (start_frame + t / (h w), t / w % h, t % w); the
pairs of a head split into time / height / width as dim/2 - 2 (dim/2 // 3), dim/2 // 3, dim/2 // 3.
x1' = x1 c - x2 s, x2' = x2 c + x1 s with both products and the sum rounded separately, in float32 (float64
when the input or the table is float64); padding tokens past f h w are copied unchanged.
"""

import torch

from wan_dit_lab_b200 import _native

_CODES = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2, torch.float64: 3}


def rope_apply(x, grid_sizes, freq, start_frame=0, *, output_dtype=None):
    """Rotate, preserving the input dtype by default (reference rope_triton.py:101-144)."""
    if x.device.type != "cuda" or freq.device != x.device:
        raise ValueError("Input and frequencies must be on the same CUDA device")
    dtypes = (torch.float16, torch.bfloat16, torch.float32, torch.float64)
    if x.dtype not in dtypes or freq.dtype not in (torch.float32, torch.float64):
        raise TypeError("Floating input and real FP32/FP64 frequencies required")
    if x.ndim != 4 or x.shape[-1] < 2 or x.shape[-1] % 2:
        raise ValueError("Input must be (batch, token, heads, even dim)")
    if freq.ndim != 3 or freq.shape[0] != 2 or freq.shape[2] != x.shape[-1] // 2:
        raise ValueError("Frequencies must be (2, positions, dim/2)")
    if freq.requires_grad:
        raise ValueError("Trainable frequencies are not supported")
    if isinstance(grid_sizes, torch.Tensor):
        if grid_sizes.device.type != "cpu":
            raise ValueError("Grid sizes must be host metadata, not CUDA tensors")
        grid_sizes = grid_sizes.tolist()
    grids = [list(g) for g in grid_sizes]
    if len(grids) != x.shape[0] or not grids:
        raise ValueError("One grid is required per nonempty batch")
    if not isinstance(start_frame, int) or start_frame < 0:
        raise ValueError("start_frame must be a nonnegative integer")
    for g in grids:
        if len(g) != 3 or any(not isinstance(v, int) for v in g):
            raise ValueError("Each grid must contain three integers")
        f, h, w = g
        if f < 0 or h <= 0 or w <= 0 or f * h * w > x.shape[1]:
            raise ValueError("Grid exceeds sequence length or has invalid dimensions")
        spatial = (x.shape[-1] // 2) // 3
        if start_frame + f > freq.shape[1] or (spatial and max(h, w) > freq.shape[1]):
            raise ValueError("Grid or offset exceeds frequency bounds")
    output_dtype = x.dtype if output_dtype is None else output_dtype
    if output_dtype not in dtypes:
        raise TypeError("Floating output dtype required")
    if x.requires_grad:
        raise ValueError("The B200 RoPE is a forward (inference) operator")
    out = torch.empty(x.shape, device=x.device, dtype=output_dtype)
    B, L, H, D = x.shape
    flat = torch.tensor([v for g in grids for v in g], dtype=torch.int32)
    xs = torch.tensor(x.stride(), dtype=torch.int64)
    fs = torch.tensor(freq.stride(), dtype=torch.int64)
    with torch.cuda.device(x.device):
        _native.check(_native.lib().wdl_rope_apply(
            x.data_ptr(), _CODES[x.dtype], xs.data_ptr(), B, L, H, D, flat.data_ptr(), freq.data_ptr(),
            _CODES[freq.dtype], fs.data_ptr(), freq.shape[1], start_frame, out.data_ptr(), _CODES[output_dtype],
            _native.stream()))
    return out


def rope_apply_wan(x, grid_sizes, freqs, start_frame=0):
    """Upstream Wan adapter: complex frequencies, float32 output (reference rope_triton.py:147-152)."""
    if freqs.dtype not in (torch.complex64, torch.complex128):
        raise TypeError("Wan adapter requires complex frequencies")
    real_freqs = torch.view_as_real(freqs).permute(2, 0, 1)
    return rope_apply(x, grid_sizes, real_freqs, start_frame, output_dtype=torch.float32)
