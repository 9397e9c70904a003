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

import torch

from wan_dit_lab_b200 import _native

GROUP = 64  # input channels per INT4 scale (reference w4a4.py:29)
# How the GEMM's operands hold the 4-bit codes in HBM, one per byte: E4M3 (the code's value as an FP8 number,
# tcgen05 kind::f8f6f4, float32 group partials) or int8 (kind::i8, int32 partials). All exact; E4M3 spares
# the promotion an int-to-float conversion per accumulator element and group. "e4m3ts" keeps E4M3 codes and
# stores each group scale padded to 16 bytes (s, 0, 0, 0), so that the GEMM forms the scale products on the
# tensor cores too (same results bit for bit, one CUDA-core operation per element and group instead of two).
# "f16fold" holds float16 operands: activation codes, and weights folded with their bf16 group scales (exact),
# so that the GEMM's promotion is one fused multiply-add by the activation scale (same results bit for bit); a
# layer whose folded weights would not be exact (non-bf16 scales) falls back to "e4m3".
CODE_FORMAT = "f16fold"
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
    return {"e4m3": _native.CODES_E4M3, "int8": _native.CODES_INT8, "e4m3ts": _native.CODES_E4M3_TS,
            "f16fold": _native.CODES_F16_FOLD}[name]


def scale_shape(groups, rows, code_format):
    """Shape of a [groups, rows] scale array in the given code format (padded to 4 float32 for "e4m3ts")."""
    return (groups, rows, 4) if _code_format(code_format) == _native.CODES_E4M3_TS else (groups, rows)


def quantize_rows(x, scale_dtype=torch.bfloat16, smooth=None, packed=False, code_format="int8"):
    """Rows of x [M, K] (bfloat16 or float32, CUDA) in symmetric INT4 groups of GROUP: codes [M, K] int8, scales
    [K / GROUP, M] float32 (holding values rounded to scale_dtype) and, with packed, the nibbles [M, K / 2] uint8.
    code_format "int8" gives the codes as int8 integers, "e4m3" as the GEMM's E4M3 bytes (a uint8 tensor),
    "e4m3ts" E4M3 bytes with scales [K / GROUP, M, 4] holding (s, 0, 0, 0), "f16fold" float16 codes.
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
    dtype = {"int8": torch.int8, "f16fold": torch.float16}.get(code_format, torch.uint8)
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


@torch.no_grad()
def int4_groups(R, rule="max"):
    """R [N, K] in symmetric INT4 groups of GROUP input channels: the integers [N, K] (int32) and the scales
    [N, K / GROUP] (float32), as the reference's int4_groups (w4a4.py:81-100). Rule "max" only: the "mse" search
    and GPTQ are offline calibration options of the reference outside the forward path."""
    if rule != "max":
        raise NotImplementedError("only the 'max' scale rule is implemented on the B200 path")
    N, K = R.shape
    codes, _ = quantize_rows(R.float().contiguous(), torch.bfloat16)
    return codes.to(torch.int32), _group_scales(R.float())


def _group_scales(R):
    """The fp32 scales max(max|R_g|, 1e-8) / 7 the quantizer used, [N, K / GROUP]. The division by 7 is done as
    an IEEE division (as the kernel does it): on a CUDA tensor PyTorch divides by a scalar through its reciprocal,
    which rounds differently in a few cases."""
    N, K = R.shape
    top = R.view(N, K // GROUP, GROUP).abs().amax(dim=-1).clamp(min=1e-8)
    return (top.cpu() / 7).to(R.device)


@torch.no_grad()
def quantize(weight, bias=None, smooth=None, rank=32, shift=0.0, hessian=None, rule="max", scale_dtype=torch.bfloat16):
    """The tensors of a W4A4 layer for y = x W^T + b (reference w4a4.py:141-180): dict(qweight [N, K/2] uint8,
    wscales [K/64, N], proj_down [K, r], proj_up [N, r], smooth [K], bias [N]), bfloat16 where not INT4, in the
    logical packed format of this module. weight [N, K] on a CUDA device; smooth [K] (ones when None); rank: of
    the 16-bit low-rank branch taken from the SVD of W diag(s) (0: none); shift: the second layer of gelu_mlp
    quantizes x + shift unsigned, and the bias takes off shift (R / s) 1 (w4a4.py:168-170)."""
    if hessian is not None:
        raise NotImplementedError("GPTQ rounding is an offline calibration option, not implemented here")
    W = _cuda(weight, "weight").float()
    N, K = W.shape
    s = torch.ones(K, device=W.device) if smooth is None else smooth.float().to(W.device)
    Ws = W * s[None, :]
    if rank:
        U, S, Vh = torch.linalg.svd(Ws, full_matrices=False)
        up, down = U[:, :rank] * S[:rank], Vh[:rank]
        R = Ws - up @ down
    else:
        up, down = W.new_zeros(N, 0), W.new_zeros(0, K)
        R = Ws
    codes, scales_t, packed = quantize_rows(R.contiguous(), scale_dtype, packed=True)
    top = _group_scales(R)  # the fp32 scales of the codes
    b = torch.zeros(N, device=W.device) if bias is None else bias.float().to(W.device)
    if shift:
        Rq = (codes.view(N, K // GROUP, GROUP).float() * top[..., None]).view(N, K)  # R as INT4 holds it
        b = b - shift * (Rq / s[None, :]).sum(dim=1)
    return dict(
        qweight=packed,
        wscales=top.t().contiguous().to(scale_dtype),  # [K/64, N]
        proj_down=(down / s[None, :]).t().contiguous().to(torch.bfloat16),  # [K, r]: the branch reads x itself
        proj_up=up.contiguous().to(torch.bfloat16),  # [N, r]
        smooth=s.to(torch.bfloat16),
        bias=b.to(torch.bfloat16),
    )


def smoothing(act_amax, weight, alpha=0.5):
    """SmoothQuant's s_j = max|x_j|^alpha / max|W_:j|^(1 - alpha) (reference w4a4.py:183-186)."""
    w = weight.float().abs().amax(dim=0).clamp(min=1e-5)
    return (act_amax.float().to(w.device).clamp(min=1e-5) ** alpha / w ** (1 - alpha)).clamp(min=1e-2, max=1e2)


class PreparedW4A4:
    """A W4A4 layer in the GEMM's device layout: codes [N, K] one byte each (CODE_FORMAT), scales [K/64, N]
    float32 ([K/64, N, 4] padded in "e4m3ts"), bias [N] float32 (or None), smooth [K] bfloat16 (or None when it is all ones), made once from the
    packed parts."""

    def __init__(self, qweight, wscales, proj_down, proj_up, smooth, bias, code_format=None):
        _cuda(qweight, "qweight")
        N, half = qweight.shape
        K = 2 * half
        if wscales.shape != (K // GROUP, N):
            raise ValueError(f"wscales must be [K/64, N] = [{K // GROUP}, {N}], got {tuple(wscales.shape)}")
        if proj_down is not None and proj_down.numel() and proj_down.shape[-1] > 0:
            raise NotImplementedError("the low-rank branch (proj_down/proj_up of rank > 0) is not implemented yet")
        self.N, self.K = N, K
        self.scale_dtype = wscales.dtype
        fmt = code_format or CODE_FORMAT
        q = qweight.contiguous().view(torch.uint8)
        ws = wscales.contiguous()
        if fmt == "f16fold" and not self._fold(q, ws, N, K):
            fmt = "e4m3"  # the folded weights would not be exact: keep the 8-bit codes
        self.code_format = _code_format(fmt)
        if fmt != "f16fold":
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
            _native.check(lib.wdl_w4a4_linear(
                x.data_ptr(), x.stride(0), M, K, _native.ptr(self.smooth), _scale_code(self.scale_dtype),
                self.codes.data_ptr(), self.scales.data_ptr(), self.code_format, _native.ptr(self.bias), self.N,
                y.data_ptr(), self.N, work.data_ptr(), work.numel(), _native.stream()))
        return y


_prepared = {}


def _prepare(qweight, wscales, proj_down, proj_up, smooth, bias):
    key = (qweight.data_ptr(), qweight._version, wscales.data_ptr(), wscales._version,
           None if bias is None else (bias.data_ptr(), bias._version),
           None if smooth is None else (smooth.data_ptr(), smooth._version))
    layer = _prepared.get(key)
    if layer is None:
        if len(_prepared) > 256:
            _prepared.clear()
        layer = _prepared[key] = PreparedW4A4(qweight, wscales, proj_down, proj_up, smooth, bias)
    return layer


def w4a4_linear(x, qweight, wscales, proj_down, proj_up, smooth, bias):
    """live::w4a4_linear (reference native/ops/w4a4_ops.cpp:31-40): y [M, N] bfloat16 for x [M, K] bfloat16."""
    return _prepare(qweight, wscales, proj_down, proj_up, smooth, bias)(x)


def linear(x, t):
    """y = x W^T + b for x [M, K] bfloat16 and t the tensors of quantize (reference w4a4.py:189-192)."""
    return w4a4_linear(x, *(t[part] for part in PARTS))


class PackedW4A4Linear(torch.nn.Module):
    """A linear layer in W4A4 over the parts of quantize (reference w4a4.py:220-231); unpacked once, here."""

    def __init__(self, **parts):
        super().__init__()
        self.layer = PreparedW4A4(*(parts[name] for name in PARTS))
        self.out_features = self.layer.out_features

    def forward(self, X):
        y = self.layer(X.reshape(-1, X.shape[-1]).to(torch.bfloat16).contiguous())
        return y.reshape(*X.shape[:-1], self.out_features)
