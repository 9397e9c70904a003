"""The Wan block forward (src/wan_dit_lab/models/block.py WanBlock with the W4A4 layers of
quantization/w4a4.py: FusedQKVAttention, PackedW4A4Linear, PackedW4A4GeluMLP, and KVCache.attend over the FP8
cache with SageAttention) on the B200 kernels, one chunk of one video stream at a time (batch 1).

    shift_a, scale_a, gate_a, shift_f, scale_f, gate_f = (time_in + modulation).chunk(6)
    X = X + self_attn(norm1(X) (1 + scale_a) + shift_a) * gate_a        W4A4 qkv, RMSNorm q / k, RoPE,
                                                                         FP8 KV store, Sage over the cache, W4A4 o
    X = X + cross_attn(norm3(X))                                         W4A4 q, RMSNorm q, Sage over the
                                                                         prompt's keys / values, W4A4 o
    X = X + ffn(norm2(X) (1 + scale_f) + shift_f) * gate_f              W4A4 fc1 + GELU + unsigned INT4 requant
                                                                         fused, W4A4 fc2

Kernels per block and chunk (libwdl_b200.so): ln_quant, GEMM (qkv), qkv_prep, Sage prep (3) + quant_q +
attention, quantize_rows + GEMM with gated residual (o), ln_quant, GEMM (cross q), rms_rows, quant_q,
attention, quantize_rows + GEMM with residual (cross o), ln_quant, GEMM with the GELU requant epilogue (fc1),
GEMM with gated residual (fc2). The residual stream is float32 (after the first block of a model the
reference's X is float32 too: the float32 gates promote it), updated in place.

Cross-attention runs on the Sage kernel as in the reference's Live experiments ("Sage cross"); its keys and
values depend on the prompt alone and are projected, normalized and quantized once per prompt
(Stream.cross, generation/causal.py:558-568).
"""

import math

import torch

from wan_dit_lab_b200 import _native
from wan_dit_lab_b200.quantization import w4a4

HEAD_DIM = 128


def _f32(t):
    return t.detach().float().contiguous()


class Buffers:
    """Scratch of one chunk of n tokens, shared by all the blocks of a model (they run one after another). heads:
    the heads this process holds (all of them, or a tensor-parallel shard's), ffn_dim its hidden channels; dim the
    model's width (the residual stream). sharded: also the fp32 partial products and RMS statistics that a
    tensor-parallel block sums across shards."""

    def __init__(self, n, dim, ffn_dim, heads, max_keys, text_tokens, device, sharded=False, lowrank=False):
        self.n, self.dim, self.ffn = n, dim, ffn_dim
        u8 = dict(dtype=torch.uint8, device=device)
        f32 = dict(dtype=torch.float32, device=device)
        bf = dict(dtype=torch.bfloat16, device=device)
        hd = heads * HEAD_DIM
        width = max(dim, ffn_dim)
        self.codes = torch.empty(n, 2 * width, **u8)  # room for the float16 codes of "f16fold"
        self.scales = torch.empty(width // 64, n, **f32)
        self.hcodes = torch.empty(n, 2 * ffn_dim, **u8)  # rows of ffn_dim codes, one or two bytes each
        self.hscales = torch.empty(ffn_dim // 64, n, **f32)
        self.qkv = torch.empty(n, 3 * hd, **bf)
        self.q = torch.empty(n, hd, **f32)
        self.k = torch.empty(n, hd, **f32)
        self.attn = torch.empty(n, hd, **bf)
        self.cq = torch.empty(n, hd, **bf)
        npad = -(-n // 128) * 128
        self.q_i8 = torch.empty(heads, npad, HEAD_DIM, dtype=torch.int8, device=device)
        self.q_scale = torch.empty(heads, npad // 32 * 8, **f32)
        lib = _native.lib()
        self.sage = torch.empty(lib.wdl_sage_attend_workspace(n, max_keys, heads), **u8)
        if sharded:
            self.partial = torch.empty(n, dim, **f32)  # a row-parallel layer's share of its product
            self.sumsq = torch.empty(n, 2, **f32)  # the shard's share of the q / k RMS statistics
        if lowrank:  # the inputs of SVDQuant low-rank branches that no other buffer holds
            self.xin = torch.empty(n, dim, **bf)  # a layer's bf16 input after LayerNorm / modulation
            self.gelu = torch.empty(n, ffn_dim, **f32)  # GELU's output in the feed forward (before the shift)


def quantize_block(p, scale_dtype=torch.bfloat16, rank=0):
    """The W4A4 parts {layer: quantize() tensors} of a block's float weights p (the reference's names; SVDQuant
    low-rank branches of `rank`, 0 for none; q, k and v of self-attention as one qkv layer, FusedQKVAttention; ffn.2
    made for gelu_mlp's shifted input)."""
    parts = {}
    cat = lambda *names: torch.cat([p[n] for n in names])  # noqa: E731
    parts["self_attn.qkv"] = w4a4.quantize(cat("self_attn.q.weight", "self_attn.k.weight", "self_attn.v.weight"),
                                           cat("self_attn.q.bias", "self_attn.k.bias", "self_attn.v.bias"),
                                           rank=rank, scale_dtype=scale_dtype)
    for name in ("self_attn.o", "cross_attn.q", "cross_attn.k", "cross_attn.v", "cross_attn.o", "ffn.0"):
        parts[name] = w4a4.quantize(p[f"{name}.weight"], p[f"{name}.bias"], rank=rank, scale_dtype=scale_dtype)
    parts["ffn.2"] = w4a4.quantize(p["ffn.2.weight"], p["ffn.2.bias"], rank=rank, shift=w4a4.GELU_SHIFT,
                                   scale_dtype=scale_dtype)
    return parts


def attention_scale(keys, entropy_ratio=None, head_dim=HEAD_DIM):
    """The softmax scale of Q K^T over `keys` keys (reference KVCache.scale, causal.py:138-142): 1 / sqrt(d), or
    with an entropy ratio r, sqrt(log_T N / d) for N = keys and T = N r, which keeps attention's entropy at that of
    the training length."""
    if entropy_ratio is None:
        return head_dim ** -0.5
    return math.sqrt(math.log(keys) / math.log(keys * entropy_ratio) / head_dim)


def attend_forcing(buf, n, H, cache, at, forcing, entropy_ratio=None):
    """Self-attention of a chunk with Forcing-KV's head split (reference causal.py:222-240), over the H heads this
    process holds (buf.q / buf.k float32 [n, H 128], the chunk's values in buf.qkv[:, 2 H 128:], output buf.attn):
    forcing = (static, dynamic, anchor rows) int32 device tensors in this process's head numbers. The dynamic
    heads attend to the cached window [0, at) and the chunk, the static heads to the anchor rows (the sink and the
    newest finished frame) and the chunk, each group through the attention's head / token maps
    (wdl_sage_attend_maps) on gathered copies of its heads' queries, keys and values; each group's softmax scale is
    attention_scale of its own key count (causal.py:236-238)."""
    lib, st = _native.lib(), _native.stream()
    ck, cks, cv, cvs, capacity = cache
    static, dynamic, anchors = forcing
    width = H * HEAD_DIM
    heads_of = lambda t, idx: t.view(n, H, HEAD_DIM).index_select(1, idx).reshape(n, -1)  # noqa: E731
    out = buf.attn[:n].view(n, H, HEAD_DIM)
    for idx, tokens, length in ((dynamic, None, at), (static, anchors, anchors.numel())):
        if idx.numel() == 0:
            continue
        il = idx.long()
        q_s, k_s = heads_of(buf.q[:n], il).contiguous(), heads_of(buf.k[:n], il).contiguous()
        v_s = heads_of(buf.qkv[:n, 2 * width:3 * width], il).contiguous()
        hs = idx.numel()
        o_s = torch.empty(n, hs * HEAD_DIM, dtype=torch.bfloat16, device=buf.attn.device)
        _native.check(lib.wdl_sage_attend_maps(
            q_s.data_ptr(), hs * HEAD_DIM, n, ck.data_ptr(), cks.data_ptr(), cv.data_ptr(), cvs.data_ptr(),
            capacity, H, idx.data_ptr(), _native.ptr(tokens), length, k_s.data_ptr(), _native.F32,
            hs * HEAD_DIM, v_s.data_ptr(), _native.BF16, hs * HEAD_DIM, n, hs,
            attention_scale(length + n, entropy_ratio), o_s.data_ptr(), hs * HEAD_DIM, buf.sage.data_ptr(), buf.sage.numel(), st))
        out[:, il] = o_s.view(n, hs, HEAD_DIM)


class CrossKV:
    """The keys and values of one block's cross-attention over a prompt, quantized for the Sage kernel."""

    def __init__(self, k_i8, k_scale, v_f8, v_scale, tokens):
        self.k_i8, self.k_scale, self.v_f8, self.v_scale, self.tokens = k_i8, k_scale, v_f8, v_scale, tokens


class WanBlockB200:
    """One Wan block with its weights in the kernels' layouts, made from a WanBlock state dict (the reference's
    parameter names: self_attn.{q,k,v,o}, cross_attn.{q,k,v,o}, ffn.{0,2}, norm3, *.norm_q / norm_k, modulation).
    Every linear layer is W4A4 (INT4 groups of 64): quantized here from float weights (with SVDQuant low-rank
    branches of svd_rank, 0 for none), or given as `parts` {layer: quantize() tensors} of a converted pack, with
    low-rank branches of any rank and smoothing vectors."""

    def __init__(self, state, dim, ffn_dim, heads, eps=1e-6, device="cuda", parts=None, scale_dtype=torch.bfloat16,
                 code_format=None, svd_rank=0):
        self.dim, self.ffn_dim, self.heads, self.eps = dim, ffn_dim, heads, eps
        self.kv_heads = heads  # the heads of this process's KV cache and attention
        if dim != heads * HEAD_DIM:
            raise ValueError("head_dim must be 128")
        p = {k: v.to(device) for k, v in state.items()}
        if parts is None:
            parts = quantize_block(p, scale_dtype, rank=svd_rank)
        self.parts = parts
        self.layers = {name: w4a4.PreparedW4A4(*(t[k] for k in w4a4.PARTS), code_format=code_format)
                       for name, t in parts.items()}
        # SVDQuant low-rank branches (rank r > 0): their [n, N] products, (x proj_down) proj_up^T in float32,
        # enter the GEMM epilogues before the bias (wdl_w4a4_gemm_add and relatives)
        self.lowrank = any(layer.rank for layer in self.layers.values())
        if len({layer.code_format for layer in self.layers.values()}) > 1:
            # a layer could not take the requested format: the block's quantizers feed every layer one format
            self.layers = {name: w4a4.PreparedW4A4(*(t[k] for k in w4a4.PARTS), code_format="e4m3")
                           for name, t in parts.items()}
        self.code_format = self.layers["self_attn.qkv"].code_format
        self.norm_q, self.norm_k = _f32(p["self_attn.norm_q.weight"]), _f32(p["self_attn.norm_k.weight"])
        self.cross_norm_q, self.cross_norm_k = _f32(p["cross_attn.norm_q.weight"]), _f32(p["cross_attn.norm_k.weight"])
        self.norm3_w, self.norm3_b = _f32(p["norm3.weight"]), _f32(p["norm3.bias"])
        self.modulation = _f32(p["modulation"]).reshape(6, dim)
        self.act_scale_dtype = _native.BF16  # activation scales are bf16, as Nunchaku stores them (x's dtype)

    # ---- prompt
    def cross_kv(self, context):
        """CrossKV of the prompt context [tokens, dim] bfloat16 (after the model's text embedding):
        K = RMSNorm(k(C)), V = v(C) (models/multi_head_attention.py:21-26), quantized for the Sage kernel."""
        lib, st = _native.lib(), _native.stream()
        T = context.shape[0]
        k = self.layers["cross_attn.k"](context)
        v = self.layers["cross_attn.v"](context)
        kf = torch.empty(T, self.dim, device=context.device)
        _native.check(lib.wdl_rms_rows(k.data_ptr(), self.dim, T, self.dim, self.cross_norm_k.data_ptr(), self.eps,
                                       kf.data_ptr(), self.dim, st))
        lpad = -(-T // 128) * 128
        H = self.heads
        k_i8 = torch.zeros(H, lpad, HEAD_DIM, dtype=torch.int8, device=context.device)
        k_scale = torch.zeros(H, lpad // 64 * 4, device=context.device)
        v_f8 = torch.zeros(H, HEAD_DIM, lpad, dtype=torch.uint8, device=context.device)
        v_scale = torch.zeros(H, HEAD_DIM, device=context.device)
        work = torch.empty(lib.wdl_sage_prep_workspace(T, H), dtype=torch.uint8, device=context.device)
        _native.check(lib.wdl_sage_prep_kv(None, None, None, None, 0, kf.data_ptr(), _native.F32, self.dim,
                                           v.data_ptr(), _native.BF16, self.dim, T, H, k_i8.data_ptr(),
                                           k_scale.data_ptr(), v_f8.data_ptr(), v_scale.data_ptr(), work.data_ptr(),
                                           work.numel(), st))
        return CrossKV(k_i8, k_scale, v_f8, v_scale, T)

    # ---- chunk
    # When set (a callable taking (start, stop) CUDA events and the layer's int ops), every GEMM launch of forward
    # is bracketed by CUDA events on the current stream: the benchmark's per-kernel timing of the W4A4 GEMMs.
    gemm_timer = None

    def forward(self, X, mod, cache, at, freq, grid, start, cross, buf, x_is_bf16=False, trace=None, forcing=None,
                entropy_ratio=None):
        """X [n, dim] float32, updated in place (the block's output). mod [6, dim] float32: this block's
        time_in + modulation. cache: (k, ks, v, vs, capacity) FP8 cache buffers of this block
        [capacity, heads, 128] / [capacity, heads]; the chunk's keys and values are stored at `at` and attention
        runs over [0, at + n). freq [2, positions, 64] float32 RoPE table, grid (frames, h, w) of the chunk,
        start its first frame's time position. cross: CrossKV of the prompt. x_is_bf16: the stream held bf16
        values (the first block of a model): the first norm rounds to bf16 as .type_as does (the reference's
        LayerNorm, models/layer_norm.py:5-7); its residual update makes the stream float32 (the gates are float32),
        so the two later norms do not. trace: a dict that, when
        given, receives copies of the intermediate tensors (debugging; synchronizes). forcing: Forcing-KV's
        (static heads, dynamic heads, anchor rows) of the cache (KVCache.forcing()), or None: with it, the dynamic
        heads attend to the whole cached window and the static ones to the anchor rows (the sink and the newest
        finished frame), both with the chunk, through the attention's head / token maps (causal.py:222-240).
        entropy_ratio: the cache's attention entropy ratio (self-attention's softmax scale, attention_scale), or None
        for 1 / sqrt(128)."""
        if X.dtype != torch.float32 or X.dim() != 2 or not X.is_contiguous():
            raise ValueError("X must be the float32 residual stream [n, dim], contiguous: the kernels read and update "
                             "it as rows")
        lib, st = _native.lib(), _native.stream()
        n, dim, H = X.shape[0], self.dim, self.heads
        ck, cks, cv, cvs, capacity = cache

        def keep(name, t):
            if trace is not None:
                trace[name] = t.clone()
        fmt, sd = self.code_format, self.act_scale_dtype
        L = self.layers
        mod_ptr = lambda i: mod.data_ptr() + i * dim * 4  # noqa: E731

        timer = WanBlockB200.gemm_timer

        def timed(layer, launch):
            if timer is None:
                return launch()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            launch()
            e1.record()
            timer(e0, e1, 2 * n * layer.N * layer.K)

        def lora(layer, x):
            """The layer's low-rank branch for its bf16 / float32 input x (its down-projection [n, r] here, its
            up-projection in the GEMM epilogue: a wdl_lowrank), or None at rank 0."""
            return layer.lowrank_arg(layer.lowrank_act(x[:n])) if layer.rank else None

        def gemm(layer, out, add=None):
            timed(layer, lambda: _native.check(lib.wdl_w4a4_gemm_lowrank(
                buf.codes.data_ptr(), buf.scales.data_ptr(), layer.codes.data_ptr(), layer.scales.data_ptr(), fmt,
                _native.ptr(layer.bias), add, n, layer.N, layer.K, out.data_ptr(), out.stride(0), st)))

        def gemm_residual(layer, gate_row, codes=None, scales=None, add=None):
            c = buf.codes if codes is None else codes
            s = buf.scales if scales is None else scales
            f = fmt if codes is None else w4a4.hidden_format(fmt)  # the hidden layer's own format
            timed(layer, lambda: _native.check(lib.wdl_w4a4_gemm_residual_lowrank(
                c.data_ptr(), s.data_ptr(), layer.codes.data_ptr(), layer.scales.data_ptr(), f,
                _native.ptr(layer.bias), add, None if gate_row is None else mod_ptr(gate_row),
                X.data_ptr(), dim, n, layer.N, layer.K, X.data_ptr(), dim, st)))

        def ln_quant(shift_row, scale_row, affine, layer, round_bf16):
            """Codes and scales of the layer's input; with a low-rank branch also the bf16 input itself (buf.xin),
            whose product with the branch is returned (else None)."""
            keep = buf.xin if layer.rank else None
            _native.check(lib.wdl_ln_quant_keep(
                X.data_ptr(), _native.F32, dim, n, dim, self.eps, self.norm3_w.data_ptr() if affine else None,
                self.norm3_b.data_ptr() if affine else None, 1 if round_bf16 else 0,
                None if shift_row is None else mod_ptr(shift_row), None if scale_row is None else mod_ptr(scale_row),
                _native.ptr(layer.smooth), sd, fmt, buf.codes.data_ptr(), buf.scales.data_ptr(), _native.ptr(keep),
                dim, st))
            return None if keep is None else lora(layer, keep)

        def quantize(x, layer):
            _native.check(lib.wdl_w4a4_quantize_rows(x.data_ptr(), _native.BF16, x.stride(0), _native.ptr(layer.smooth),
                                                     n, layer.K, sd, fmt, buf.codes.data_ptr(), buf.scales.data_ptr(),
                                                     None, st))

        # self-attention
        add = ln_quant(0, 1, False, L["self_attn.qkv"], x_is_bf16)
        gemm(L["self_attn.qkv"], buf.qkv, add)
        keep("qkv", buf.qkv)
        _native.check(lib.wdl_qkv_prep(buf.qkv.data_ptr(), 3 * dim, n, dim, self.norm_q.data_ptr(),
                                       self.norm_k.data_ptr(), self.eps, freq.data_ptr(), freq.shape[1], grid[1],
                                       grid[2], start, buf.q.data_ptr(), buf.k.data_ptr(), ck.data_ptr(),
                                       cks.data_ptr(), cv.data_ptr(), cvs.data_ptr(), capacity, at, st))
        if forcing is None:
            _native.check(lib.wdl_sage_attend(
                buf.q.data_ptr(), dim, n, ck.data_ptr(), cks.data_ptr(), cv.data_ptr(), cvs.data_ptr(), at,
                buf.k.data_ptr(), _native.F32, dim, None, _native.BF16, 3 * dim, n, H,  # V: in the cache (qkv_prep)
                attention_scale(at + n, entropy_ratio), buf.attn.data_ptr(), dim, buf.sage.data_ptr(), buf.sage.numel(),
                st))
        else:
            attend_forcing(buf, n, H, cache, at, forcing, entropy_ratio)
        keep("q", buf.q), keep("k", buf.k), keep("attn", buf.attn)
        quantize(buf.attn, L["self_attn.o"])
        gemm_residual(L["self_attn.o"], 2, add=lora(L["self_attn.o"], buf.attn))
        keep("x_after_self", X)
        # cross-attention
        # the first residual update made the stream float32 (float32 gates): the later norms round only at the linear
        add = ln_quant(None, None, True, L["cross_attn.q"], False)
        gemm(L["cross_attn.q"], buf.cq, add)
        keep("cq", buf.cq)
        _native.check(lib.wdl_rms_rows(buf.cq.data_ptr(), dim, n, dim, self.cross_norm_q.data_ptr(), self.eps,
                                       buf.q.data_ptr(), dim, st))
        _native.check(lib.wdl_sage_quant_q(buf.q.data_ptr(), dim, n, H, buf.q_i8.data_ptr(), buf.q_scale.data_ptr(), st))
        _native.check(lib.wdl_sage_attention(buf.q_i8.data_ptr(), buf.q_scale.data_ptr(), cross.k_i8.data_ptr(),
                                             cross.k_scale.data_ptr(), cross.v_f8.data_ptr(), cross.v_scale.data_ptr(),
                                             n, cross.tokens, H, HEAD_DIM ** -0.5, buf.attn.data_ptr(), dim, st))
        keep("cattn", buf.attn)
        quantize(buf.attn, L["cross_attn.o"])
        gemm_residual(L["cross_attn.o"], None, add=lora(L["cross_attn.o"], buf.attn))
        keep("x_after_cross", X)
        # feed forward
        fc1, fc2 = L["ffn.0"], L["ffn.2"]
        add = ln_quant(3, 4, False, fc1, False)
        gelu = buf.gelu if fc2.rank else None  # the second layer's branch reads GELU's output without the shift
        timed(fc1, lambda: _native.check(lib.wdl_w4a4_gemm_gelu_u4_lowrank(
            buf.codes.data_ptr(), buf.scales.data_ptr(), fc1.codes.data_ptr(), fc1.scales.data_ptr(), fmt,
            _native.ptr(fc1.bias), add, _native.ptr(fc2.smooth), w4a4.GELU_SHIFT, sd, n, fc1.N, fc1.K,
            buf.hcodes.data_ptr(), fc1.N, buf.hscales.data_ptr(), _native.ptr(gelu), fc1.N, st)))
        if trace is not None:  # the hidden codes [n, ffn] as float values, whatever their operand format
            raw = buf.hcodes.view(-1)
            if w4a4.hidden_format(fmt) == _native.CODES_F16_FOLD:
                trace["hcodes"] = raw[:n * fc1.N * 2].view(torch.float16).view(n, fc1.N).float()
            else:
                trace["hcodes"] = raw[:n * fc1.N].view(torch.float8_e4m3fn).view(n, fc1.N).float()
        if trace is not None:  # the hidden scales [ffn / 64, n] as the GEMM reads them
            G = buf.hscales.shape[0]
            keep("hscales", buf.hscales.view(-1)[:G * n].view(G, n))
        gemm_residual(fc2, 5, buf.hcodes, buf.hscales, add=None if gelu is None else lora(fc2, gelu))
        return X

    def buffers(self, n, max_keys, text_tokens, device, lowrank=None):
        """Scratch for chunks of n tokens attending to up to max_keys keys (lowrank: with the inputs of low-rank
        branches; default: whether this block has any)."""
        return Buffers(n, self.dim, self.ffn_dim, self.kv_heads, max_keys, text_tokens, device,
                       lowrank=self.lowrank if lowrank is None else lowrank)

    def modulation_of(self, time_in):
        """time_in [6, dim] float32 + this block's modulation (models/block.py:75)."""
        out = torch.empty(6, self.dim, device=time_in.device)
        _native.check(_native.lib().wdl_modulation(time_in.data_ptr(), self.modulation.data_ptr(), 1, self.dim,
                                                   out.data_ptr(), _native.stream()))
        return out
