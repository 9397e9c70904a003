"""The operators live::* of the reference's native/ops (native/ops/w4a4_ops.cpp:79-95, native/ops/sage_ops.cpp:28-35),
loaded the way its kernels/operators.py:19-25 loads them (load() registers them once and returns torch.ops.live),
here as torch.library custom operators over libwdl_b200.so, each with a fake (meta) implementation for shape
inference as the reference's Meta kernels give:

    live::w4a4_linear(x, qweight, wscales, proj_down, proj_up, smooth, bias) -> [M, N] bfloat16
    live::w4a4_gelu_mlp(x, six parts of layer 1, six parts of layer 2)    -> [M, N2] bfloat16
    live::sage_sm89(q, k, v, q_scale, k_scale, v_scale, sm_scale)        -> [B, n, H, 128] bfloat16

The W4A4 operators take the parts of quantization/w4a4.py's quantize (the logical packed format of this build) and
run w4a4_linear / w4a4_gelu_mlp. sage_sm89 takes SageAttention's operands in the layouts the reference's
quantizers write (kernels/sage_kv.py:60-124): q INT8 [B, n, H, 128] with scales [B, H, blocks of 32 x 8], k INT8
[B, L, H, 128] with scales [B, H, blocks of 64 x 4], v E4M3 [B, 128, H, padded] whose keys are permuted within
every 16 ([0, 1, 8, 9, 2, 3, 10, 11, 4, 5, 12, 13, 6, 7, 14, 15]) and v_scale [B, H, 128]; they are rearranged
into the attention kernel's layouts (sage_operands) and run by wdl_sage_attention. The fast path of attention over
the FP8 cache (kernels/sage_kv.py attend) never materializes these layouts; this operator serves call sites that
hold Sage's operands already."""

import torch

from wan_dit_lab_b200 import _native

HEAD_DIM = 128
# where Sage's V layout keeps key j of each 16 (reference kernels/sage_kv.py:102-104): pairs of keys, the first
# four pairs at positions 0, 4, 8, 12, the last four at 2, 6, 10, 14
_V_POSITION = [(p % 4) * 4 + (p // 4) * 2 + j % 2 for j in range(16) for p in [j // 2]]


def sage_operands(q, k, v, q_scale, k_scale, v_scale):
    """Sage's layouts (batch element b already taken: q [n, H, 128], k [L, H, 128], v [128, H, padded], q_scale
    [H, *], k_scale [H, *], v_scale [H, 128]) -> the attention kernel's: q_i8 [H, npad, 128], q_scale [H, npad / 4],
    k_i8 [H, Lpad, 128], k_scale [H, Lpad / 16], v_f8 [H, 128, Lpad] (keys in order), v_scale [H, 128]; npad and
    Lpad rounded up to 128, padding zero codes and zero scales. Plain tensor operations on q's device."""
    n, H, D = q.shape
    L = k.shape[0]
    npad, lpad = -(-n // 128) * 128, -(-L // 128) * 128
    dev = q.device
    qi = torch.zeros(H, npad, D, dtype=torch.int8, device=dev)
    qi[:, :n] = q.transpose(0, 1)
    qs = torch.zeros(H, npad // 32 * 8, dtype=torch.float32, device=dev)
    qs[:, :q_scale.shape[-1]] = q_scale
    ki = torch.zeros(H, lpad, D, dtype=torch.int8, device=dev)
    ki[:, :L] = k.transpose(0, 1)
    ks = torch.zeros(H, lpad // 64 * 4, dtype=torch.float32, device=dev)
    ks[:, :k_scale.shape[-1]] = k_scale
    padded = v.shape[-1]
    order = torch.tensor(_V_POSITION, device=dev)
    natural = v.view(torch.uint8).permute(1, 0, 2).reshape(H, D, padded // 16, 16).index_select(3, order)
    vf = torch.zeros(H, D, lpad, dtype=torch.uint8, device=dev)
    vf[:, :, :min(padded, lpad)] = natural.reshape(H, D, padded)[:, :, :lpad]
    return qi, qs, ki, ks, vf, v_scale.float().contiguous()


def _check_sage(q, k, v, q_scale, k_scale, v_scale):
    if q.dtype != torch.int8 or k.dtype != torch.int8:
        raise TypeError("q and k must be int8")
    if v.dtype not in (torch.float8_e4m3fn, torch.uint8):
        raise TypeError("v must be float8_e4m3fn")
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4 or q.shape[-1] != HEAD_DIM or k.shape[-1] != HEAD_DIM:
        raise ValueError("q [B, n, H, 128], k [B, L, H, 128] and v [B, 128, H, padded] expected")
    B, n, H, _ = q.shape
    L = k.shape[1]
    padded = -(-L // 64) * 64
    if k.shape[0] != B or k.shape[2] != H or tuple(v.shape) != (B, HEAD_DIM, H, padded):
        raise ValueError(f"k must be [{B}, L, {H}, 128] and v [{B}, 128, {H}, {padded}]")
    if tuple(q_scale.shape) != (B, H, -(-n // 128) * 32) or tuple(k_scale.shape) != (B, H, padded // 16):
        raise ValueError("q_scale must be [B, H, blocks of 32 x 8] and k_scale [B, H, blocks of 64 x 4]")
    if tuple(v_scale.shape) != (B, H, HEAD_DIM):
        raise ValueError("v_scale must be [B, H, 128]")
    if L == 0:
        raise ValueError("attention over no keys")


def _register():
    lib = torch.library

    @lib.custom_op("live::w4a4_linear", mutates_args=(), device_types="cuda")
    def w4a4_linear(x: torch.Tensor, qweight: torch.Tensor, wscales: torch.Tensor, proj_down: torch.Tensor,
                    proj_up: torch.Tensor, smooth: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
        from wan_dit_lab_b200.quantization import w4a4
        return w4a4.w4a4_linear(x, qweight, wscales, proj_down, proj_up, smooth, bias)

    @w4a4_linear.register_fake
    def _(x, qweight, wscales, proj_down, proj_up, smooth, bias):
        return x.new_empty(x.shape[0], qweight.shape[0])

    @lib.custom_op("live::w4a4_gelu_mlp", mutates_args=(), device_types="cuda")
    def w4a4_gelu_mlp(x: torch.Tensor, qweight1: torch.Tensor, wscales1: torch.Tensor, proj_down1: torch.Tensor,
                      proj_up1: torch.Tensor, smooth1: torch.Tensor, bias1: torch.Tensor, qweight2: torch.Tensor,
                      wscales2: torch.Tensor, proj_down2: torch.Tensor, proj_up2: torch.Tensor, smooth2: torch.Tensor,
                      bias2: torch.Tensor) -> torch.Tensor:
        from wan_dit_lab_b200.quantization import w4a4
        return w4a4.w4a4_gelu_mlp(x, qweight1, wscales1, proj_down1, proj_up1, smooth1, bias1, qweight2, wscales2,
                                  proj_down2, proj_up2, smooth2, bias2)

    @w4a4_gelu_mlp.register_fake
    def _(x, qweight1, wscales1, proj_down1, proj_up1, smooth1, bias1, qweight2, wscales2, proj_down2, proj_up2,
          smooth2, bias2):
        return x.new_empty(x.shape[0], qweight2.shape[0])

    @lib.custom_op("live::sage_sm89", mutates_args=(), device_types="cuda")
    def sage_sm89(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_scale: torch.Tensor, k_scale: torch.Tensor,
                  v_scale: torch.Tensor, sm_scale: float) -> torch.Tensor:
        _check_sage(q, k, v, q_scale, k_scale, v_scale)
        B, n, H, D = q.shape
        L = k.shape[1]
        out = torch.empty(B, n, H, D, dtype=torch.bfloat16, device=q.device)
        lib_, st = _native.lib(), _native.stream()
        for b in range(B):
            qi, qs, ki, ks, vf, vs = sage_operands(q[b], k[b], v[b], q_scale[b].float(), k_scale[b].float(),
                                                   v_scale[b])
            _native.check(lib_.wdl_sage_attention(qi.data_ptr(), qs.data_ptr(), ki.data_ptr(), ks.data_ptr(),
                                                  vf.data_ptr(), vs.data_ptr(), n, L, H, sm_scale,
                                                  out[b].data_ptr(), H * D, st))
        return out

    @sage_sm89.register_fake
    def _(q, k, v, q_scale, k_scale, v_scale, sm_scale):
        return q.new_empty(q.shape, dtype=torch.bfloat16)


def load():
    """Registers live::w4a4_linear, live::w4a4_gelu_mlp and live::sage_sm89 in this process, once (unless another
    library registered them already), and returns torch.ops.live."""
    if not hasattr(torch.ops.live, "sage_sm89"):
        _register()
    return torch.ops.live
