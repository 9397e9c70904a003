"""W4A4 linear layers (SVDQuant: INT4 weights and activations in groups of 64 input channels) on the B200
kernels, with the module API of the reference's src/wan_dit_lab/quantization/w4a4.py.

Same names, arguments and meaning as the reference: GROUP, GELU_SHIFT, PARTS, int4_groups, quantize,
linear, gelu_mlp, w4a4_linear, w4a4_gelu_mlp, PackedW4A4Linear, PackedW4A4GeluMLP. The arithmetic runs in
libwdl_b200.so (tcgen05 kind::i8 GEMM with per-group scale promotion, and the INT4 group quantizer).

The packed weight format is the logical one, not Nunchaku's MMA-tile order (whose packer is not part of the
reference): qweight [N, K/2] uint8 with two INT4 codes per byte (low nibble = even input channel, two's
complement), wscales [K/64, N] in bfloat16 (or float16), proj_down [K, r], proj_up [N, r], smooth [K] and
bias [N] in bfloat16, as w4a4.quantize returns them (reference w4a4.py:141-180). At load (PackedW4A4Linear)
or on first use (w4a4_linear) the codes are unpacked once into the GEMM's device layout: one code per byte
[N, K] and fp32 scales [K/64, N]. HBM holds 180 GB here, so the weights are kept one code per byte and no
nibble is unpacked inside the GEMM's main loop.
"""

import math
import weakref
from pathlib import Path

import torch

from wan_dit_lab_b200 import _native

GROUP = 64  # input channels per INT4 scale (reference w4a4.py:29)
# How the GEMM's operands hold the 4-bit codes in HBM, one per byte: E4M3 (the code's value as an FP8 number,
# tcgen05 kind::f8f6f4, float32 group partials) or int8 (kind::i8, int32 partials). All exact; E4M3 spares
# the promotion an int-to-float conversion per accumulator element and group.
# "f16fold" holds float16 operands: activation codes, and weights folded with their bf16 group scales (exact),
# so that the GEMM's promotion is one fused multiply-add by the activation scale (same results bit for bit); a
# layer whose folded weights would not be exact (non-bf16 scales) falls back to "e4m3". "f16pre" keeps the folded
# weights and folds the activation scales into the activations too (code * sx * 2^-E per row, exact): the GEMM
# accumulates all of K on the tensor cores and scales each row once (float32 rounding of the sum, not bit-identical
# to the per-group promotion); the fused MLP's unsigned hidden layer stays in "f16fold".
CODE_FORMAT = "f16pre"
GELU_SHIFT = 0.171875  # GELU(x) + GELU_SHIFT >= 0: the hidden layer of gelu_mlp is quantized unsigned (w4a4.py:195)
PARTS = ("qweight", "wscales", "proj_down", "proj_up", "smooth", "bias")  # w4a4.py:207


def _cuda(t, name):
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor")
    return t


def _scale_code(dtype):
    if dtype not in (torch.bfloat16, torch.float16):
        raise TypeError("INT4 scales are stored in bfloat16 or float16")
    return _native.DTYPE_CODE[dtype]


def _code_format(name):
    return {"e4m3": _native.CODES_E4M3, "int8": _native.CODES_INT8, "f16fold": _native.CODES_F16_FOLD,
            "f16pre": _native.CODES_F16_PRE}[name]


def hidden_format(code_format):
    """The code format (int) of the fused MLP's hidden layer, which a GELU epilogue of a GEMM in `code_format`
    writes and the second layer's GEMM reads: the prescaled format's is the folded one (unsigned codes)."""
    return _native.CODES_F16_FOLD if code_format == _native.CODES_F16_PRE else code_format


def scale_shape(groups, rows, code_format):
    """Shape of a [groups, rows] scale array in the given code format (one power of two per row for "f16pre")."""
    return (rows,) if _code_format(code_format) == _native.CODES_F16_PRE else (groups, rows)


def quantize_rows(x, scale_dtype=torch.bfloat16, smooth=None, packed=False, code_format="int8"):
    """Rows of x [M, K] (bfloat16 or float32, CUDA) in symmetric INT4 groups of GROUP: codes [M, K] int8, scales
    [K / GROUP, M] float32 (holding values rounded to scale_dtype) and, with packed, the nibbles [M, K / 2] uint8.
    code_format "int8" gives the codes as int8 integers, "e4m3" as the GEMM's E4M3 bytes (a uint8 tensor),
    "f16fold" float16 codes, "f16pre"
    float16 code * scale * 2^-E_m with the rows' 2^E_m [M] as scales (bf16 scales only).
    scale = max(max|x_g|, 1e-8) / 7, code = round-half-even(x / scale) clamped to [-8, 7] (the rule of
    int4_groups, reference w4a4.py:86-100); smooth [K] bfloat16 divides x first."""
    _cuda(x, "x")
    if x.ndim != 2 or x.shape[1] % GROUP:
        raise ValueError("x must be [M, K] with K a multiple of 64")
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("x must be bfloat16 or float32")
    if x.stride(1) != 1:
        x = x.contiguous()
    M, K = x.shape
    dtype = {"int8": torch.int8, "f16fold": torch.float16, "f16pre": torch.float16}.get(code_format, torch.uint8)
    codes = torch.empty(M, K, dtype=dtype, device=x.device)
    scales = torch.empty(scale_shape(K // GROUP, M, code_format), dtype=torch.float32, device=x.device)
    nib = torch.empty(M, K // 2, dtype=torch.uint8, device=x.device) if packed else None
    if smooth is not None:
        smooth = _cuda(smooth, "smooth").to(torch.bfloat16).contiguous()
    with torch.cuda.device(x.device):
        _native.check(_native.lib().wdl_w4a4_quantize_rows(
            x.data_ptr(), _native.DTYPE_CODE[x.dtype], x.stride(0), _native.ptr(smooth), M, K,
            _scale_code(scale_dtype), _code_format(code_format), codes.data_ptr(), scales.data_ptr(),
            _native.ptr(nib), _native.stream()))
    return (codes, scales, nib) if packed else (codes, scales)


MSE_STEPS = torch.linspace(0.5, 1.0, 26).tolist()  # the scales the "mse" rule tries, x max|x| / 7 (w4a4.py:76)


@torch.no_grad()
def int4_groups(R, rule="max"):
    """R [N, K] in symmetric INT4 groups of GROUP input channels: the integers [N, K] (int32) and the scales
    [N, K / GROUP] (float32), as the reference's int4_groups (w4a4.py:80-100). "max": scale = max|x| / 7, the
    forward path's rule, by the quantizer kernel (R on a GPU). "mse" (offline, R on any device): of the scales
    c max|x| / 7 for c in MSE_STEPS the one with the least squared error over the group, the smallest c among equal
    errors; values beyond the grid are clipped to -8 / 7."""
    N, K = R.shape
    if rule == "max":
        codes, _ = quantize_rows(R.float().contiguous(), torch.bfloat16)
        return codes.to(torch.int32), _group_scales(R.float())
    if rule != "mse":
        raise ValueError(rule)
    groups = R.float().reshape(N, K // GROUP, GROUP)
    top = _group_scales(R.float())
    scale = torch.empty_like(top)
    # every candidate of a slice of rows at once ([candidates, rows, groups, 64], about 64 MB), the first minimum
    rows = max(1, (16 << 20) // (len(MSE_STEPS) * K))
    for r0 in range(0, N, rows):
        g = groups[r0:r0 + rows]
        cand = torch.stack([top[r0:r0 + rows] * c for c in MSE_STEPS])  # [C, rows, groups]
        back = torch.round(g / cand[..., None]).clamp(-8, 7) * cand[..., None]
        err = ((g - back) ** 2).sum(-1)
        scale[r0:r0 + rows] = cand.gather(0, err.argmin(0, keepdim=True))[0]
    codes = torch.round(groups / scale[..., None]).clamp(-8, 7).to(torch.int32).reshape(N, K)
    return codes, scale


@torch.no_grad()
def gptq(R, H, damp=0.01, block=128):
    """GPTQ (Frantar et al., "GPTQ: Accurate Post-Training Quantization for Generative Pre-trained Transformers",
    ICLR 2023) of R [N, K] into symmetric INT4 groups of GROUP input channels (reference w4a4.py:103-137), for the
    inputs X of the layer through H = X^T X [K, K]: the columns are rounded left to right; a group's scale
    max|x| / 7 is taken from its columns when the first of them is rounded, as earlier errors have moved them; each
    column's error over the diagonal of U (the upper Cholesky factor of H^-1) is spread over the columns to its
    right along U's row, inside a block of `block` columns column by column and onto the columns past the block
    with one product. H gets damp x mean(diag H) on its diagonal; an input channel with H_jj = 0 carries nothing:
    its weights are rounded from 0. Returns codes int32 [N, K] and scales float32 [N, K / GROUP]."""
    W = R.detach().float().clone()
    N, K = W.shape
    Hd = H.detach().float().to(W.device).clone()
    idle = Hd.diagonal() == 0
    Hd[idle, idle] = 1
    W[:, idle] = 0
    Hd.diagonal().add_(damp * Hd.diagonal().mean())
    U = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(Hd)), upper=True)
    del Hd
    codes = torch.zeros(N, K, dtype=torch.int32, device=W.device)
    scales = torch.zeros(N, K // GROUP, device=W.device)
    for b0 in range(0, K, block):
        b1 = min(b0 + block, K)
        part = W[:, b0:b1]  # a view: the block's columns move in place as their left neighbours are rounded
        errors = torch.zeros(N, b1 - b0, device=W.device)
        for j in range(b1 - b0):
            c = b0 + j
            if c % GROUP == 0:
                scales[:, c // GROUP] = W[:, c:c + GROUP].abs().amax(dim=1).clamp(min=1e-8) / 7
            s = scales[:, c // GROUP]
            w = part[:, j]
            q = torch.round(w / s).clamp(-8, 7)
            codes[:, c] = q.to(torch.int32)
            e = (w - q * s) / U[c, c]
            part[:, j:] -= e[:, None] * U[c, c:b1][None, :]
            errors[:, j] = e
        W[:, b1:] -= errors @ U[b0:b1, b1:]
    return codes, scales


def _pack_nibbles(codes):
    """int codes [N, K] in [-8, 7] -> uint8 [N, K / 2], two per byte, the even input channel in the low nibble."""
    lo, hi = codes[:, 0::2] & 0xF, codes[:, 1::2] & 0xF
    return (lo | (hi << 4)).to(torch.uint8)


def _group_scales(R):
    """The fp32 scales max(max|R_g|, 1e-8) / 7 the quantizer used, [N, K / GROUP]. The division by 7 is done as
    an IEEE division (as the kernel does it): on a CUDA tensor PyTorch divides by a scalar through its reciprocal,
    which rounds differently in a few cases."""
    N, K = R.shape
    top = R.view(N, K // GROUP, GROUP).abs().amax(dim=-1).clamp(min=1e-8)
    return (top.cpu() / 7).to(R.device)


def _lowrank_split(Ws, rank):
    """W diag(s) = U V + R: the rank-r branch, up [N, r] (left singular vectors times their singular values) and
    down [r, K], from the SVD of the smoothed weight, and the residual R left to INT4. rank 0: no branch, R = Ws."""
    if not rank:
        return Ws.new_zeros(Ws.shape[0], 0), Ws.new_zeros(0, Ws.shape[1]), Ws
    left, sigma, right = torch.linalg.svd(Ws, full_matrices=False)
    up, down = left[:, :rank] * sigma[:rank], right[:rank]
    return up, down, Ws - up @ down


def _round_residual(R, s, hessian, rule, scale_dtype):
    """(codes [N, K], float32 group scales [N, K/64], packed nibbles [N, K/2]) of the residual. Without a Hessian
    and with the "max" rule: to the nearest, by the quantizer kernel (the rounding of the forward path). Else on the
    host side: the scale rule of int4_groups, or GPTQ with the second moment of what the INT4 branch multiplies R by,
    x / s: H divided by s along both axes (a layer with K > 8192, whose H alone takes 0.8 GB, on the CPU)."""
    if hessian is None and rule == "max":
        codes, _, packed = quantize_rows(R.contiguous(), scale_dtype, packed=True)
        return codes, _group_scales(R), packed
    if hessian is None:
        codes, scales = int4_groups(R, rule)
    else:
        host = torch.device("cpu") if R.shape[1] > 8192 else R.device
        sh = s.to(host)
        codes, scales = gptq(R.to(host), hessian.float().to(host).div(sh[:, None]).div(sh[None, :]))
        codes, scales = codes.to(R.device), scales.to(R.device)
    return codes, scales, _pack_nibbles(codes)


def _shifted_bias(bias, shift, codes, scales, s):
    """The layer's bias as float32; for a layer whose INT4 branch quantizes x + shift (gelu_mlp's second layer), less
    what the shift adds through that branch, shift (R_q / s) 1, R_q being R as the codes and scales hold it
    (w4a4.py:168-170): the low-rank branch reads x without the shift."""
    N = codes.shape[0]
    out = codes.new_zeros(N, dtype=torch.float32) if bias is None else bias.float().to(codes.device)
    if not shift:
        return out
    held = (codes.view(N, -1, GROUP).float() * scales[..., None]).view(N, -1)
    return out - shift * held.div(s[None, :]).sum(dim=1)


@torch.no_grad()
def quantize(weight, bias=None, smooth=None, rank=32, shift=0.0, hessian=None, rule="max", scale_dtype=torch.bfloat16):
    """The tensors of a W4A4 layer for y = x W^T + b (reference w4a4.py:141-180): dict(qweight [N, K/2] uint8,
    wscales [K/64, N], proj_down [K, r], proj_up [N, r], smooth [K], bias [N]), bfloat16 where not INT4, in the
    logical packed format of this module. weight [N, K] (on a CUDA device for the kernel's "max" rounding; the
    offline rules run where it is); smooth [K] (ones when None): x is divided by it and W multiplied; rank: of the
    16-bit low-rank branch (0: none); shift: the second layer of gelu_mlp quantizes x + shift unsigned
    (_shifted_bias). hessian [K, K]: X^T X of the inputs the INT4 branch multiplies by R (x + shift for gelu_mlp's
    second layer, before smoothing): R is rounded by GPTQ instead of to the nearest. rule: the INT4 scale rule of
    int4_groups."""
    if hessian is None and rule == "max":
        _cuda(weight, "weight")
    W = weight.float()
    s = W.new_ones(W.shape[1]) if smooth is None else smooth.float().to(W.device)
    up, down, R = _lowrank_split(W * s[None, :], rank)
    codes, scales, packed = _round_residual(R, s, hessian, rule, scale_dtype)
    bf = torch.bfloat16
    return dict(qweight=packed,
                wscales=scales.t().contiguous().to(scale_dtype),  # [K/64, N]
                proj_down=(down / s[None, :]).t().contiguous().to(bf),  # [K, r]: the branch reads x, not x / s
                proj_up=up.contiguous().to(bf),  # [N, r]
                smooth=s.to(bf),
                bias=_shifted_bias(bias, shift, codes, scales, s).to(bf))


def smoothing(act_amax, weight, alpha=0.5):
    """SmoothQuant's s_j = max|x_j|^alpha / max|W_:j|^(1 - alpha) (reference w4a4.py:183-186)."""
    w = weight.float().abs().amax(dim=0).clamp(min=1e-5)
    return (act_amax.float().to(w.device).clamp(min=1e-5) ** alpha / w ** (1 - alpha)).clamp(min=1e-2, max=1e2)


class PreparedW4A4:
    """A W4A4 layer in the GEMM's device layout: codes [N, K] one byte each (CODE_FORMAT), scales [K/64, N]
    float32, bias [N] float32 (or None), smooth [K] bfloat16 (or None when it is all ones), made once from the
    packed parts."""

    def __init__(self, qweight, wscales, proj_down, proj_up, smooth, bias, code_format=None):
        _cuda(qweight, "qweight")
        N, half = qweight.shape
        K = 2 * half
        if wscales.shape != (K // GROUP, N):
            raise ValueError(f"wscales must be [K/64, N] = [{K // GROUP}, {N}], got {tuple(wscales.shape)}")
        self.N, self.K = N, K
        # the SVDQuant low-rank branch (rank r, bf16 factors): proj_down [K, r] (already divided by the smoothing:
        # the branch reads x itself), proj_up [N, r]; y += (x proj_down) proj_up^T: the down-projection a thin
        # float32 product, the up-projection formed in the GEMM epilogue (wdl_lowrank). The factors are kept in
        # float32 with the rank padded to a multiple of 4 by zero columns (the epilogue takes four ranks at a time).
        self.rank = 0 if proj_down is None or proj_down.numel() == 0 else int(proj_down.shape[-1])
        if self.rank:
            if proj_down.shape != (K, self.rank) or proj_up is None or proj_up.shape != (N, self.rank):
                raise ValueError(f"proj_down must be [K, r] = [{K}, r] and proj_up [N, r] = [{N}, r]")
            r4 = -(-self.rank // 4) * 4
            self.down = torch.zeros(K, r4, dtype=torch.float32, device=proj_down.device)
            self.up = torch.zeros(N, r4, dtype=torch.float32, device=proj_up.device)
            self.down[:, :self.rank] = proj_down.float()
            self.up[:, :self.rank] = proj_up.float()
        self.scale_dtype = wscales.dtype
        self._parts = (qweight, wscales, proj_down, proj_up, smooth, bias)
        fmt = code_format or CODE_FORMAT
        q = qweight.contiguous().view(torch.uint8)
        ws = wscales.contiguous()
        if fmt in ("f16fold", "f16pre") and not self._fold(q, ws, N, K):
            fmt = "e4m3"  # the folded weights would not be exact: keep the 8-bit codes
        self.code_format = _code_format(fmt)
        if fmt not in ("f16fold", "f16pre"):
            self.codes = torch.empty(N, K, dtype=torch.uint8, device=qweight.device)
            self.scales = torch.empty(scale_shape(K // GROUP, N, fmt), dtype=torch.float32, device=qweight.device)
            with torch.cuda.device(q.device):
                _native.check(_native.lib().wdl_w4a4_unpack_weight(
                    q.data_ptr(), ws.data_ptr(), _scale_code(ws.dtype), N, K, self.code_format, self.codes.data_ptr(),
                    self.scales.data_ptr(), _native.stream()))
        self.bias = None if bias is None else bias.float().contiguous()
        ones = smooth is None or bool((smooth == 1).all())
        self.smooth = None if ones else smooth.to(torch.bfloat16).contiguous()
        self.out_features = N

    def _fold(self, q, ws, N, K):
        """The folded format's weights: codes [N, K] float16 = code * wscale * 2^-F with one power of two per layer
        (the largest product lands below 2^15), and scales = the float 2^F the GEMM multiplies back. False when
        any element would not be an exact normal float16 number."""
        if ws.dtype != torch.bfloat16:
            return False
        top = float(ws.float().abs().max())
        shift = math.ceil(math.log2(8 * top)) - 15 if top > 0 else 0
        codes = torch.empty(N, K, dtype=torch.float16, device=q.device)
        inexact = torch.zeros(1, dtype=torch.int32, device=q.device)
        with torch.cuda.device(q.device):
            _native.check(_native.lib().wdl_w4a4_fold_weight(q.data_ptr(), ws.data_ptr(), _scale_code(ws.dtype), N,
                                                             K, shift, codes.data_ptr(), inexact.data_ptr(),
                                                             _native.stream()))
        if int(inexact.item()) != 0:
            return False
        self.codes = codes
        self.scales = torch.tensor([2.0 ** shift], dtype=torch.float32, device=q.device)
        return True

    def lowrank(self, x):
        """The low-rank branch's contribution (x proj_down) proj_up^T [M, N] float32 for x [M, K] (the layer's
        input before smoothing), or None at rank 0, as two plain float32 products: the addend form that the _add
        GEMM entry points take (the tensor-parallel shards' partial products use it); the layers themselves form
        the up-projection in the GEMM epilogue (lowrank_act, lowrank_arg)."""
        if not self.rank:
            return None
        return ((x.float() @ self.down) @ self.up.t()).contiguous()

    def lowrank_act(self, x):
        """The branch's down-projection x proj_down [M, r] float32 for x [M, K] bfloat16 or float32 (the layer's
        input before smoothing; Nunchaku forms it beside its quantizer, w4a4_ops.cpp:27), by wdl_lowrank_down, or
        None at rank 0."""
        if not self.rank:
            return None
        if x.dtype not in (torch.bfloat16, torch.float32):
            raise TypeError("the low-rank branch reads a bfloat16 or float32 input")
        if x.stride(1) != 1 or (x.stride(0) * x.element_size()) % 16 or x.data_ptr() % 16:
            x = x.contiguous()
        M, r4 = x.shape[0], self.down.shape[1]
        act = torch.empty(M, r4, dtype=torch.float32, device=x.device)
        with torch.cuda.device(x.device):
            _native.check(_native.lib().wdl_lowrank_down(
                x.data_ptr(), _native.DTYPE_CODE[x.dtype], x.stride(0), M, self.K, self.down.data_ptr(), r4,
                act.data_ptr(), r4, _native.stream()))
        return act

    def lowrank_arg(self, act):
        """The wdl_lowrank that the _lowrank GEMM entry points take for act = lowrank_act(x) (None for None): the
        epilogue adds act proj_up^T before the bias (w4a4_ops.cpp:36), the [M, N] product never written."""
        if act is None:
            return None
        arg = _native.LowRank(act.data_ptr(), act.stride(0), self.up.data_ptr(), self.up.shape[1])
        arg.tensors = (act, self.up)  # alive as long as the argument
        return arg

    def quantize_input(self, x, work):
        """x [M, K] bfloat16 -> (codes, scales) of this layer's code format, in the workspace `work`."""
        M, K = x.shape
        lib = _native.lib()
        codes = work[: M * K * 2]
        scales = work[(M * K * 2 + 255) // 256 * 256:].view(torch.float32)
        _native.check(lib.wdl_w4a4_quantize_rows(x.data_ptr(), _native.BF16, x.stride(0), _native.ptr(self.smooth), M,
                                                 K, _scale_code(self.scale_dtype), self.code_format, codes.data_ptr(),
                                                 scales.data_ptr(), None, _native.stream()))
        return codes, scales

    def __call__(self, x):
        """y [M, N] bfloat16 = x W^T + b for x [M, K] bfloat16."""
        M, K = x.shape
        if K != self.K:
            raise ValueError(f"x has {K} input channels, the layer {self.K}")
        if x.dtype != torch.bfloat16:
            raise TypeError("x must be bfloat16")
        if x.stride(1) != 1 or (x.stride(0) * 2) % 16:
            x = x.contiguous()
        y = torch.empty(M, self.N, dtype=torch.bfloat16, device=x.device)
        lib = _native.lib()
        work = torch.empty(lib.wdl_w4a4_linear_workspace(M, K), dtype=torch.uint8, device=x.device)
        with torch.cuda.device(x.device):
            if not self.rank:
                _native.check(lib.wdl_w4a4_linear(
                    x.data_ptr(), x.stride(0), M, K, _native.ptr(self.smooth), _scale_code(self.scale_dtype),
                    self.codes.data_ptr(), self.scales.data_ptr(), self.code_format, _native.ptr(self.bias), self.N,
                    y.data_ptr(), self.N, work.data_ptr(), work.numel(), _native.stream()))
            else:
                branch = self.lowrank_arg(self.lowrank_act(x))
                codes, scales = self.quantize_input(x, work)
                _native.check(lib.wdl_w4a4_gemm_lowrank(
                    codes.data_ptr(), scales.data_ptr(), self.codes.data_ptr(), self.scales.data_ptr(),
                    self.code_format, _native.ptr(self.bias), branch, M, self.N, K, y.data_ptr(), self.N,
                    _native.stream()))
        return y


def _stamp(parts):
    """What a prepared layer was made from: for each part a weak reference to the tensor object and its in-place
    version counter (None for an absent part)."""
    return tuple(None if t is None else (weakref.ref(t), t._version) for t in parts)


def _same_parts(stamp, parts):
    return all((a is None) == (t is None) and (t is None or (a[0]() is t and a[1] == t._version))
               for a, t in zip(stamp, parts))


def _prepare(qweight, wscales, proj_down, proj_up, smooth, bias):
    """The device layout of these packed parts, made once and kept on the qweight tensor itself (attribute
    `_wdl_prepared`), so that it lives exactly as long as the weight does. A later call reuses it only with the very
    same tensor objects, none modified in place since (object identity and version counter): a weight freed and
    another allocated at its address never matches, and any number of layers and models keep their own."""
    parts = (qweight, wscales, proj_down, proj_up, smooth, bias)
    held = getattr(qweight, "_wdl_prepared", None)
    if held is not None and _same_parts(held[0], parts):
        return held[1]
    layer = PreparedW4A4(*parts)
    qweight._wdl_prepared = (_stamp(parts), layer)
    return layer


def w4a4_linear(x, qweight, wscales, proj_down, proj_up, smooth, bias):
    """live::w4a4_linear (reference native/ops/w4a4_ops.cpp:31-40): y [M, N] bfloat16 for x [M, K] bfloat16."""
    return _prepare(qweight, wscales, proj_down, proj_up, smooth, bias)(x)


def linear(x, t):
    """y = x W^T + b for x [M, K] bfloat16 and t the tensors of quantize (reference w4a4.py:189-192)."""
    return w4a4_linear(x, *(t[part] for part in PARTS))


def _same_format(l1, l2):
    if l1.code_format == l2.code_format:
        return l1, l2
    # the hidden codes are written in the first layer's format and read in the second's: one format for both
    parts = lambda l: l._parts  # noqa: E731
    return (PreparedW4A4(*parts(l1), code_format="e4m3"), PreparedW4A4(*parts(l2), code_format="e4m3"))


def w4a4_gelu_mlp(x, *parts):
    """live::w4a4_gelu_mlp (reference native/ops/w4a4_ops.cpp:44-63, w4a4.py:198-204): y [M, N2] bfloat16 =
    GELU(x W1^T + b1) W2^T + b2 for x [M, K] bfloat16 and the six parts of each layer (the second made with
    shift=GELU_SHIFT). The first GEMM's epilogue applies GELU, adds the shift and quantizes the hidden layer to
    unsigned INT4 straight into the second GEMM's operand; with low-rank branches it also keeps GELU's output for
    the second layer's branch (which reads it without the shift)."""
    if len(parts) != 12:
        raise ValueError("w4a4_gelu_mlp takes the six parts of each of the two layers")
    l1, l2 = _same_format(_prepare(*parts[:6]), _prepare(*parts[6:]))
    if x.dtype != torch.bfloat16:
        raise TypeError("x must be bfloat16")
    if x.ndim != 2 or x.shape[1] != l1.K or l2.K != l1.N:
        raise ValueError("x must be [M, K] of the first layer, whose N is the second layer's K")
    x = x.contiguous()
    M, lib, st = x.shape[0], _native.lib(), _native.stream()
    work = torch.empty(lib.wdl_w4a4_linear_workspace(M, l1.K), dtype=torch.uint8, device=x.device)
    hidden = torch.empty(M * l1.N * 2, dtype=torch.uint8, device=x.device)  # the hidden codes, 1 or 2 bytes each
    hscales = torch.empty(scale_shape(l1.N // GROUP, M, "e4m3"), dtype=torch.float32, device=x.device)
    gelu = torch.empty(M, l1.N, dtype=torch.float32, device=x.device) if l2.rank else None
    y = torch.empty(M, l2.N, dtype=torch.bfloat16, device=x.device)
    with torch.cuda.device(x.device):
        branch1 = l1.lowrank_arg(l1.lowrank_act(x))
        codes, scales = l1.quantize_input(x, work)
        _native.check(lib.wdl_w4a4_gemm_gelu_u4_lowrank(
            codes.data_ptr(), scales.data_ptr(), l1.codes.data_ptr(), l1.scales.data_ptr(), l1.code_format,
            _native.ptr(l1.bias), branch1, _native.ptr(l2.smooth), GELU_SHIFT, _scale_code(l2.scale_dtype), M, l1.N,
            l1.K, hidden.data_ptr(), l1.N, hscales.data_ptr(), _native.ptr(gelu), l1.N, st))
        branch2 = l2.lowrank_arg(l2.lowrank_act(gelu) if l2.rank else None)
        _native.check(lib.wdl_w4a4_gemm_lowrank(
            hidden.data_ptr(), hscales.data_ptr(), l2.codes.data_ptr(), l2.scales.data_ptr(), hidden_format(l2.code_format),
            _native.ptr(l2.bias), branch2, M, l2.N, l2.K, y.data_ptr(), l2.N, st))
    return y


def gelu_mlp(x, t1, t2):
    """y = GELU(x W1^T + b1) W2^T + b2 (GELU in tanh form, Wan's feed forward) for x [M, K] bfloat16 and t1, t2
    the tensors of quantize, t2 made with shift=GELU_SHIFT (reference w4a4.py:198-204)."""
    return w4a4_gelu_mlp(x, *(t1[part] for part in PARTS), *(t2[part] for part in PARTS))


class PackedW4A4Linear(torch.nn.Module):
    """A linear layer in W4A4 over the parts of quantize (reference w4a4.py:220-231); unpacked once, here."""

    def __init__(self, **parts):
        super().__init__()
        self.layer = PreparedW4A4(*(parts[name] for name in PARTS))
        self.out_features = self.layer.out_features

    def forward(self, X):
        y = self.layer(X.reshape(-1, X.shape[-1]).to(torch.bfloat16).contiguous())
        return y.reshape(*X.shape[:-1], self.out_features)


class PackedW4A4GeluMLP(torch.nn.Module):
    """Wan's feed forward (Linear, GELU in tanh form, Linear) in W4A4 as one gelu_mlp (reference w4a4.py:234-245)."""

    def __init__(self, fc1, fc2):
        super().__init__()
        self.parts = [fc1[name] for name in PARTS] + [fc2[name] for name in PARTS]
        self.out_features = fc2["proj_up"].shape[0] if fc2["proj_up"].numel() else fc2["wscales"].shape[-1]

    def forward(self, X):
        y = w4a4_gelu_mlp(X.reshape(-1, X.shape[-1]).to(torch.bfloat16).contiguous(), *self.parts)
        return y.reshape(*X.shape[:-1], self.out_features)


# ---- block packs: the W4A4 tensors of every block as one uint8 row per block, mapped read-only
# (reference w4a4.py:264-416). The file is the reference's: rows of bytes_per_block bytes, every entry 16-byte
# aligned at the offset the manifest (<pack>.json) gives, named "<layer>.<part>" for a W4A4 layer and by the
# parameter's name for the rest (bfloat16). What differs is the byte order of the parts: the logical one of
# quantize here, recorded as "packing": "logical" in the manifest; the reference's packs hold Nunchaku's
# MMA-tile order (its packer, nunchaku/lora/flux/packer.py at 302e0e9, is not in the reference tree) and are
# refused by mapped_pack rather than misread.

FORMATS = ("block_w4a4_v1", "block_w4a4_v2")  # w4a4.py:30: a layer per nn.Linear; v2 fuses q, k, v and the FFN
PACKING = "logical"
QKV = ("self_attn.q", "self_attn.k", "self_attn.v")  # w4a4.py:265: one layer self_attn.qkv in a fused pack
FFN = ("ffn.0", "ffn.2")  # w4a4.py:266: one gelu_mlp in a fused pack
FUSED_LAYERS = ("self_attn.qkv", "self_attn.o", "cross_attn.q", "cross_attn.k", "cross_attn.v", "cross_attn.o",
                "ffn.0", "ffn.2")  # the W4A4 layers of a block_w4a4_v2 row, which the B200 block runs


class BlockShape:
    """The shape of a Wan block for the pack functions when no block is at hand: model width, feed-forward width,
    the norms' eps."""

    def __init__(self, dim, ffn_dim, eps=1e-6):
        self.dim, self.ffn_dim, self.eps = dim, ffn_dim, eps


def block_parameters(dim, ffn_dim):
    """[(name, shape)] of a WanBlock's parameters in named_parameters order (reference models/block.py:13-20,
    models/multi_head_attention.py:13-18): the block's own modulation [1, 6, dim] first, then per attention the q,
    k, v, o weights and biases, norm_q and norm_k; the feed forward; norm3's weight and bias (norm1 and norm2
    have none)."""
    out = [("modulation", (1, 6, dim))]
    for attention in ("self_attn", "cross_attn"):
        for linear in "qkvo":
            out += [(f"{attention}.{linear}.weight", (dim, dim)), (f"{attention}.{linear}.bias", (dim,))]
        out += [(f"{attention}.norm_q.weight", (dim,)), (f"{attention}.norm_k.weight", (dim,))]
    out += [("ffn.0.weight", (ffn_dim, dim)), ("ffn.0.bias", (ffn_dim,)), ("ffn.2.weight", (dim, ffn_dim)),
            ("ffn.2.bias", (dim,)), ("norm3.weight", (dim,)), ("norm3.bias", (dim,))]
    return out


def _state(block):
    """{name: tensor} of a block given as a module (named_parameters) or as a state dict."""
    return dict(block.named_parameters()) if hasattr(block, "named_parameters") else dict(block)


def _parameters(like):
    """[(name, shape)] of the block `like`, in registration order: a module's named_parameters (the reference's
    WanBlock, on the meta device too), BlockShape, or a WanBlock state dict (any order; checked name by name)."""
    if hasattr(like, "named_parameters"):
        return [(name, tuple(p.shape)) for name, p in like.named_parameters()]
    if isinstance(like, BlockShape):
        return block_parameters(like.dim, like.ffn_dim)
    state = dict(like)
    if "modulation" not in state or "ffn.0.weight" not in state:
        raise ValueError("a WanBlock state dict needs modulation and ffn.0.weight")
    want = block_parameters(state["modulation"].shape[-1], state["ffn.0.weight"].shape[0])
    numel = lambda shape: math.prod(shape)  # noqa: E731
    if set(state) != {name for name, _ in want} or any(state[n].numel() != numel(s) for n, s in want):
        raise ValueError("the state dict does not hold a WanBlock's parameters: "
                         f"{sorted(set(state) ^ {name for name, _ in want})[:4]}")
    return want


def layers(block, fused=False, keep=()):
    """{layer: [names of the nn.Linear it is made of, stacked by output]} of a Wan block (reference
    w4a4.py:269-276): every weight of two dimensions is a linear layer's; fused takes q, k, v of self-attention as
    one layer self_attn.qkv; keep: names of linears left in bfloat16."""
    out = {}
    for name, shape in _parameters(block):
        if name.endswith(".weight") and len(shape) == 2 and name[:-7] not in keep:
            linear = name[:-7]
            out.setdefault("self_attn.qkv" if fused and linear in QKV else linear, []).append(linear)
    return out


def part_shapes(N, K, rank, scale_dtype=torch.bfloat16):
    """{part: (dtype name, shape, bytes)} of quantize's tensors for a weight [N, K] at `rank`, in PARTS order."""
    if K % GROUP:
        raise ValueError(f"a W4A4 layer's input width must be a multiple of {GROUP}, got {K}")
    scale = str(scale_dtype).removeprefix("torch.")
    size = torch.empty(0, dtype=scale_dtype).element_size()
    return dict(qweight=("uint8", (N, K // 2), N * K // 2), wscales=(scale, (K // GROUP, N), K // GROUP * N * size),
                proj_down=("bfloat16", (K, rank), K * rank * 2), proj_up=("bfloat16", (N, rank), N * rank * 2),
                smooth=("bfloat16", (K,), K * 2), bias=("bfloat16", (N,), N * 2))


def pack_layout(block, fused=False, rank=32, keep=(), scale_dtype=torch.bfloat16):
    """(layout, bytes per row) of a block's pack row (reference w4a4.py:279-313): entries dict(name, dtype, shape,
    offset, bytes) in the block's parameter order, a W4A4 layer's six parts where its first member's weight is
    (its biases are the part bias), every other parameter in bfloat16; each entry starts 16-byte aligned. In a
    fused pack the second feed-forward layer's parts carry gelu_mlp: True (made for GELU's shifted output)."""
    params = _parameters(block)
    groups = layers(block, fused, keep)
    group_of = {member: g for g, members in groups.items() for member in members}
    shapes = dict(params)
    layout, offset = [], 0

    def add(name, dtype, shape, size, **extra):
        nonlocal offset
        layout.append(dict(name=name, dtype=dtype, shape=list(shape), offset=offset, bytes=size, **extra))
        offset += -(-size // 16) * 16

    for name, shape in params:
        owner = name.rsplit(".", 1)[0]
        g = group_of.get(owner)
        if g is None:
            add(name, "bfloat16", shape, math.prod(shape) * 2)
        elif name.endswith(".weight") and groups[g][0] == owner:
            N = sum(shapes[f"{member}.weight"][0] for member in groups[g])
            extra = {"gelu_mlp": True} if fused and g == FFN[1] else {}
            for part, (dtype, part_shape, size) in part_shapes(N, shape[1], rank, scale_dtype).items():
                add(f"{g}.{part}", dtype, part_shape, size, **extra)
    return layout, offset


@torch.no_grad()
def layer_parts(block, index, amax, alpha=0.5, rank=32, fused=False, keep=(), hessians=None, rule="max",
                scale_dtype=torch.bfloat16, device="cuda"):
    """{layer: quantize tensors} of block number `index` (reference w4a4.py:316-333), quantized on `device`: the
    members' weights stacked by output, the smoothing from amax {"<index>.<first member>": largest |x| of each input
    channel} (SmoothQuant, alpha); in a fused pack the second feed-forward layer is made for gelu_mlp's shifted
    input (its smoothing from amax + GELU_SHIFT)."""
    state = _state(block)
    out = {}
    for g, members in layers(block, fused, keep).items():
        W = torch.cat([state[f"{m}.weight"].detach().to(device, torch.float32) for m in members])
        biases = [state.get(f"{m}.bias") for m in members]
        b = None
        if any(x is not None for x in biases):
            b = torch.cat([torch.zeros(state[f"{m}.weight"].shape[0], device=device) if x is None else
                           x.detach().to(device, torch.float32) for m, x in zip(members, biases)])
        shift = GELU_SHIFT if fused and g == FFN[1] else 0.0
        a = amax.get(f"{index}.{members[0]}")  # the members share their input
        s = None if a is None else smoothing(a.to(device) + shift, W, alpha)
        H = None if hessians is None else hessians.get(g)
        out[g] = quantize(W, b, smooth=s, rank=rank, shift=shift, hessian=H, rule=rule, scale_dtype=scale_dtype)
    return out


def _put(row, entry, tensor, exact_shape):
    """tensor's bytes into row at entry's place; the dtype and shape (or, for a raw parameter, the element count)
    must be the entry's."""
    if exact_shape and (str(tensor.dtype).removeprefix("torch.") != entry["dtype"] or
                        list(tensor.shape) != entry["shape"]):
        raise ValueError(f"{entry['name']}: {tensor.dtype} {list(tensor.shape)} where the layout has "
                         f"{entry['dtype']} {entry['shape']}")
    data = tensor.detach().contiguous().cpu().reshape(-1).view(torch.uint8)
    if data.numel() != entry["bytes"]:
        raise ValueError(f"{entry['name']}: {data.numel()} bytes where the layout has {entry['bytes']}")
    row[entry["offset"]:entry["offset"] + entry["bytes"]] = data


class _PackFile:
    """A pack being written: rows go to <path>.tmp as they come, hashed on the way; commit() makes the file durable,
    moves it to <path> and writes the manifest beside it; abandon() removes every file it made. It never replaces an
    existing pack, manifest or temporary file (FileExistsError before anything is opened)."""

    def __init__(self, path):
        import hashlib
        self.path = Path(path)
        self.manifest = self.path.with_name(self.path.name + ".json")
        self.partial = self.path.with_name(self.path.name + ".tmp")
        taken = next((f for f in (self.path, self.manifest, self.partial) if f.exists()), None)
        if taken is not None:
            raise FileExistsError(taken)
        self.out = open(self.partial, "xb")
        self.sha = hashlib.sha256()

    def append(self, row):
        data = memoryview(row.numpy())
        self.sha.update(data)
        self.out.write(data)

    def commit(self, metadata):
        import json
        import os
        self.out.flush()
        os.fsync(self.out.fileno())
        self.out.close()
        os.replace(self.partial, self.path)
        metadata = dict(metadata, sha256=self.sha.hexdigest())
        self.manifest.write_text(json.dumps(metadata, indent=1), encoding="utf-8")
        return metadata

    def abandon(self):
        self.out.close()
        for f in (self.partial, self.path, self.manifest):
            f.unlink(missing_ok=True)


def _block_row(block, tensors, layout, size, groups, index):
    """One block's uint8 row: its W4A4 parts (tensors: {layer: quantize tensors}) at their entries, then every other
    parameter of the layout in bfloat16 (a W4A4 layer's float bias is not stored: its part is)."""
    if set(tensors) != set(groups):
        raise ValueError(f"block {index}: W4A4 tensors for {sorted(tensors)}, the layout has {sorted(groups)}")
    entry = {e["name"]: e for e in layout}
    row = torch.zeros(size, dtype=torch.uint8)
    quantized = {f"{layer}.{part}" for layer in tensors for part in PARTS}
    for name in sorted(quantized):
        layer, part = name.rsplit(".", 1)
        _put(row, entry[name], tensors[layer][part], True)
    state = _state(block)
    for e in layout:
        if e["name"] not in quantized and e["name"] in state:
            _put(row, e, state[e["name"]].detach().to(torch.bfloat16), False)
    return row


@torch.no_grad()
def build_pack(blocks, amax, path, source, alpha=0.5, rank=32, fused=False, keep=(), hessians=None, rule="max",
               scale_dtype=torch.bfloat16, parts=None):
    """The blocks (modules or state dicts with WanBlock's names) as a pack at `path`, one uint8 row per block
    (pack_layout), and its manifest <path>.json, with the keys of the reference's (w4a4.py:361-394): block_w4a4_v2
    when fused, else block_w4a4_v1, and "packing": "logical" for this build's part order. Written to <path>.tmp,
    synced, then renamed; nothing is left behind on failure, and an existing pack, manifest or temporary file is
    never overwritten (FileExistsError). parts: per block the W4A4 tensors already made ({layer: quantize tensors},
    e.g. WanBlockB200.parts), instead of quantizing here."""
    from wan_dit_lab_b200.quantization.weight_pack import source_identity
    layout, size = pack_layout(blocks[0], fused, rank, keep, scale_dtype)
    groups = layers(blocks[0], fused, keep)
    before = source_identity(source)
    pack = _PackFile(path)
    try:
        for index, block in enumerate(blocks):
            if pack_layout(block, fused, rank, keep, scale_dtype) != (layout, size):
                raise ValueError("Packed blocks must share one layout")
            if parts is not None:
                tensors = parts[index]
            else:
                tensors = layer_parts(_state(block), index, amax, alpha, rank, fused, keep,
                                      None if hessians is None else hessians(index), rule, scale_dtype)
            pack.append(_block_row(block, tensors, layout, size, groups, index))
        if source_identity(source) != before:
            raise RuntimeError("Checkpoint changed during conversion")
        what = (f"W4A4 of SVDQuant: INT4 codes in groups of {GROUP} input channels, a bfloat16 low-rank branch of rank "
                f"{rank}, activation maxima folded in by SmoothQuant smoothing; parts in logical order")
        if fused:
            what += ("; self-attention's q, k, v stacked into one layer and the feed forward stored for the fused GELU "
                     f"MLP, whose hidden activation is shifted by {GELU_SHIFT} and quantized unsigned")
        metadata = pack.commit(dict(
            format=FORMATS[1] if fused else FORMATS[0], packing=PACKING, blocks=len(blocks), layout=layout,
            bytes_per_block=size, bytes=size * len(blocks), source=before, alpha=alpha, rank=rank,
            calibrated=sorted(amax), bfloat16_layers=sorted(keep),
            rounding="nearest" if hessians is None else "GPTQ", scale_rule=rule, quantization=what))
    except BaseException:
        pack.abandon()
        raise
    return {k: v for k, v in metadata.items() if k not in ("layout", "calibrated")}


def _pack_manifest(path, source):
    """The manifest beside the pack at `path`, refused (ValueError) unless it names `source` as its checkpoint, one
    of the block formats and this build's logical part order."""
    import json

    from wan_dit_lab_b200.quantization.weight_pack import source_identity
    manifest = json.loads(path.with_name(path.name + ".json").read_text(encoding="utf-8"))
    if manifest["format"] not in FORMATS or manifest["source"] != source_identity(source):
        raise ValueError("Weight pack has a different checkpoint or format")
    if manifest.get("packing") != PACKING:
        raise ValueError("W4A4 weight pack holds its parts in Nunchaku's MMA-tile order (the reference's packer); "
                         "this build reads packs in the logical order that build_pack writes")
    return manifest


def mapped_pack(blocks, path, source):
    """(rows uint8 [blocks, bytes per block] over the file mapped read-only, layout) of a pack (the reference's
    mapped_pack, w4a4.py:418-437). blocks: the model's blocks (a sequence) or their number. ValueError when the
    manifest names another checkpoint or format, when the parts are not in this build's logical order, or when the
    file is not blocks x bytes_per_block long. The rows read the page cache directly: nothing is copied until a
    row is moved to a device."""
    import mmap
    import warnings

    path = Path(path)
    manifest = _pack_manifest(path, source)
    count = blocks if isinstance(blocks, int) else len(blocks)
    size = manifest["bytes_per_block"]
    if count == 0 or manifest["blocks"] != count or path.stat().st_size != size * count:
        raise ValueError("W4A4 weight pack is incomplete")
    with open(path, "rb") as f:
        pages = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)  # stays mapped after the file is closed
    with warnings.catch_warnings():  # the mapping is read-only, and torch warns that the tensor is not writable
        warnings.simplefilter("ignore", UserWarning)
        flat = torch.frombuffer(pages, dtype=torch.uint8)
    return flat.view(count, size), manifest["layout"]


def slot_parts(row, layout):
    """(parts {layer: {part: tensor}}, params {name: tensor}) of a pack row: views of `row`, no copy, each entry at
    its offset with its dtype and shape."""
    def view(e):
        return row[e["offset"]:e["offset"] + e["bytes"]].view(getattr(torch, e["dtype"])).view(e["shape"])

    entries = {e["name"]: e for e in layout}
    names = [e["name"][:-len(".qweight")] for e in layout if e["name"].endswith(".qweight")]
    parts = {g: {part: view(entries[f"{g}.{part}"]) for part in PARTS} for g in names}
    taken = {f"{g}.{part}" for g in names for part in PARTS}
    return parts, {e["name"]: view(e) for e in layout if e["name"] not in taken}


def slot(row, like, layout, code_format=None, shard=None, reduce=None, device="cuda"):
    """The block of a block_w4a4_v2 pack row as a WanBlockB200 (reference w4a4.py:399-416, which builds a module over
    the row): a row elsewhere is copied to `device` once, the parts are views of that copy, and each layer is
    prepared in the kernels' layout. like: the block's eps (from a WanBlock or a BlockShape; None: 1e-6). The
    shapes come from the layout. shard (rank, world): shard `rank` of the tensor-parallel block instead
    (WanBlockTP, with `reduce` summing across shards). Refused (ValueError): block_w4a4_v1 rows and rows that keep
    layers in bfloat16, since the B200 block runs q, k, v as one W4A4 layer and the feed forward as the fused GELU
    MLP, whose second layer is quantized for GELU's shifted output."""
    from wan_dit_lab_b200.models import block, block_tp
    kept = [e["name"][:-7] for e in layout if e["name"].endswith(".weight") and len(e["shape"]) == 2]
    if kept:
        raise ValueError(f"the B200 block runs every linear layer in W4A4; this pack keeps {kept} in bfloat16")
    gelu = all(e.get("gelu_mlp") for e in layout if e["name"].startswith(FFN[1] + "."))
    names = [e["name"][:-len(".qweight")] for e in layout if e["name"].endswith(".qweight")]
    if sorted(names) != sorted(FUSED_LAYERS) or not gelu:
        raise ValueError("a block_w4a4_v1 row (a layer per nn.Linear) cannot drive the B200 block, which runs q, k, "
                         "v as one W4A4 layer and the feed forward as the fused GELU MLP: pack with fused=True")
    device = torch.device(device)
    if row.device != device and not (device.type == row.device.type and device.index is None):
        row = row.to(device)
    parts, params = slot_parts(row, layout)
    dim = params["modulation"].numel() // 6
    eps = getattr(like, "eps", None)
    if eps is None and hasattr(like, "norm1"):
        eps = like.norm1.eps
    eps = 1e-6 if eps is None else eps
    ffn_dim, heads = parts["ffn.0"]["qweight"].shape[0], dim // block.HEAD_DIM
    if shard is None:
        return block.WanBlockB200(params, dim, ffn_dim, heads, eps, device=row.device, parts=parts,
                                  code_format=code_format)
    rank, world = shard
    return block_tp.WanBlockTP(params, dim, ffn_dim, heads, rank, world, eps, device=row.device, parts=parts,
                               code_format=code_format, reduce=reduce)
