"""One video stream split across GPUs (tensor parallelism of the Wan block): heads for self- and cross-attention,
hidden channels for the feed forward, one NCCL all-reduce (sum) after each row-parallel layer.

The reference runs a stream on one GPU; the split follows its block (models/block.py:22-29, 75-79) and linears
(quantization/w4a4.py:220-262):

    layer            split                      shard of the packed parts
    self_attn.qkv    column (its heads' q, k, v) rows of qweight / bias / proj_up, columns of wscales
    self_attn.o      row (its heads' channels)  K slice: qweight columns, wscales groups, smooth, proj_down
    cross_attn.q     column (its heads)
    cross_attn.k, v  replicated                 (once per prompt; each shard keeps its heads' keys / values)
    cross_attn.o     row
    ffn.0            column (hidden channels)   the GELU + INT4 requantization stays local
    ffn.2            row

A 64-channel INT4 group never straddles shards (head and hidden splits are multiples of 64), so every shard
quantizes its activations exactly as the whole layer does. A row-parallel layer's shards write their fp32 partial
products (wdl_w4a4_gemm_f32); after the all-reduce, wdl_residual_update applies bias, bf16 rounding, gate and
residual once. The q / k RMSNorms (and cross-attention's query norm) span all heads: each shard sums the squares
of its slice (wdl_rows_sumsq), the sums are all-reduced ([tokens, 2] floats), and the norm divides by the
whole row's statistics (wdl_qkv_prep_sharded, wdl_rms_rows_sharded). LayerNorms, AdaLN and the residual stream
are replicated: every shard holds the same X (the all-reduce gives all ranks the same sums).

WanBlockTP.steps is a generator that yields each tensor to sum across shards, in the same order on every shard;
forward drives it with a reduce callable (torch.distributed.all_reduce over NCCL in a process per GPU).
run_lockstep drives the shards of one block in one process instead (each yielded tensor replaced by the sum of
all shards'), which is how the split is tested against the whole block on one GPU.
"""

import torch

from wan_dit_lab_b200 import _native
from wan_dit_lab_b200.models.block import (HEAD_DIM, Buffers, CrossKV, WanBlockB200, _f32, attend_forcing,
                                          attention_scale, quantize_block)
from wan_dit_lab_b200.quantization import w4a4

ROW_PARALLEL = ("self_attn.o", "cross_attn.o", "ffn.2")
COLUMN_PARALLEL = ("self_attn.qkv", "cross_attn.q", "ffn.0")
REPLICATED = ("cross_attn.k", "cross_attn.v")


def _take(t, dim, index):
    """A copy of t's entries `index` along dim (a copy: the whole layer's storage is not kept alive)."""
    return t.index_select(dim, index.to(t.device)).contiguous().clone()


def shard_columns(parts, index):
    """The parts of a column-parallel shard: output features `index` (a LongTensor) of a W4A4 layer."""
    out = dict(parts)
    out["qweight"] = _take(parts["qweight"], 0, index)
    out["wscales"] = _take(parts["wscales"], 1, index)
    out["bias"] = None if parts["bias"] is None else _take(parts["bias"], 0, index)
    if parts["proj_up"] is not None and parts["proj_up"].numel():
        out["proj_up"] = _take(parts["proj_up"], 0, index)
    return out


def shard_rows(parts, k0, k1):
    """The parts of a row-parallel shard: input channels [k0, k1) (multiples of 64) of a W4A4 layer, without its
    bias (added once, after the shards' partial products are summed). Returns (shard parts, the layer's bias)."""
    if k0 % w4a4.GROUP or k1 % w4a4.GROUP:
        raise ValueError("a row-parallel shard must hold whole groups of 64 input channels")
    out = dict(parts)
    out["qweight"] = parts["qweight"][:, k0 // 2:k1 // 2].contiguous().clone()
    out["wscales"] = parts["wscales"][k0 // w4a4.GROUP:k1 // w4a4.GROUP].contiguous().clone()
    if parts["smooth"] is not None:
        out["smooth"] = parts["smooth"][k0:k1].contiguous().clone()
    if parts["proj_down"] is not None and parts["proj_down"].numel():
        out["proj_down"] = parts["proj_down"][k0:k1].contiguous().clone()
    out["bias"] = None
    return out, parts["bias"]


def shard_block_parts(parts, dim, ffn_dim, heads, rank, world):
    """The parts of shard `rank` of `world` of one block's W4A4 layers (quantize_block), and the biases of its
    row-parallel layers: ({layer: parts}, {layer: bias [dim]})."""
    if heads % world or ffn_dim % (world * 128):
        raise ValueError(f"{world} shards need heads ({heads}) and ffn_dim / 128 ({ffn_dim // 128}) divisible by it")
    d = dim // world
    h0, h1 = rank * d, (rank + 1) * d
    f = ffn_dim // world
    f0, f1 = rank * f, (rank + 1) * f
    heads_cols = torch.arange(h0, h1)
    out, bias = {}, {}
    out["self_attn.qkv"] = shard_columns(parts["self_attn.qkv"], torch.cat([heads_cols + j * dim for j in range(3)]))
    out["cross_attn.q"] = shard_columns(parts["cross_attn.q"], heads_cols)
    out["ffn.0"] = shard_columns(parts["ffn.0"], torch.arange(f0, f1))
    out["self_attn.o"], bias["self_attn.o"] = shard_rows(parts["self_attn.o"], h0, h1)
    out["cross_attn.o"], bias["cross_attn.o"] = shard_rows(parts["cross_attn.o"], h0, h1)
    out["ffn.2"], bias["ffn.2"] = shard_rows(parts["ffn.2"], f0, f1)
    for name in REPLICATED:
        out[name] = parts[name]
    return out, bias


def run_lockstep(gens):
    """Drives the step generators of all shards of one block in one process: every tensor they yield (one per
    shard, in the same order) is replaced by the sum over shards, as an all-reduce would."""
    gens = list(gens)
    while True:
        ts = [next(g, None) for g in gens]
        if all(t is None for t in ts):
            return
        if any(t is None for t in ts):
            raise RuntimeError("the shards yielded different numbers of tensors")
        total = ts[0].clone()
        for t in ts[1:]:
            total += t
        for t in ts:
            t.copy_(total)


class WanBlockTP:
    """Shard `rank` of `world` of one Wan block (WanBlockB200's arguments and state-dict names; every linear W4A4,
    any rank, with smoothing). reduce: a callable summing a CUDA tensor in place across the shards (None: only steps() is used)."""

    def __init__(self, state, dim, ffn_dim, heads, rank, world, eps=1e-6, device="cuda", parts=None,
                 scale_dtype=torch.bfloat16, code_format=None, reduce=None):
        if dim != heads * HEAD_DIM:
            raise ValueError("head_dim must be 128")
        if not 0 <= rank < world:
            raise ValueError("rank must be in [0, world)")
        self.dim, self.ffn_dim, self.heads, self.eps = dim, ffn_dim, heads, eps
        self.rank, self.world, self.reduce = rank, world, reduce
        self.kv_heads = heads // world
        self.local_dim = dim // world
        self.local_ffn = ffn_dim // world
        p = {k: v.to(device) for k, v in state.items()}
        if parts is None:
            parts = quantize_block(p, scale_dtype)
        shard, bias = shard_block_parts(parts, dim, ffn_dim, heads, rank, world)
        fmt = code_format or w4a4.CODE_FORMAT
        self.layers = {name: w4a4.PreparedW4A4(*(t[k] for k in w4a4.PARTS), code_format=fmt)
                       for name, t in shard.items()}
        # SVDQuant low-rank branches: a column shard's branch is (x proj_down) proj_up_shard^T, its own output
        # columns; a row shard's, (x_shard proj_down_shard) proj_up^T, is a share of the whole branch that enters the
        # shard's fp32 partial and is summed with the partials across shards
        self.lowrank = any(layer.rank for layer in self.layers.values())
        if len({layer.code_format for layer in self.layers.values()}) > 1:
            self.layers = {name: w4a4.PreparedW4A4(*(t[k] for k in w4a4.PARTS), code_format="e4m3")
                           for name, t in shard.items()}
        self.code_format = self.layers["self_attn.qkv"].code_format
        self.bias = {name: None if b is None else _f32(b) for name, b in bias.items()}
        sl = slice(rank * self.local_dim, (rank + 1) * self.local_dim)
        self.norm_q = _f32(p["self_attn.norm_q.weight"][sl])
        self.norm_k = _f32(p["self_attn.norm_k.weight"][sl])
        self.cross_norm_q = _f32(p["cross_attn.norm_q.weight"][sl])
        self.cross_norm_k = _f32(p["cross_attn.norm_k.weight"])  # the whole prompt keys are normalized per shard
        self.norm3_w, self.norm3_b = _f32(p["norm3.weight"]), _f32(p["norm3.bias"])
        self.modulation = _f32(p["modulation"]).reshape(6, dim)
        self.act_scale_dtype = _native.BF16

    def buffers(self, n, max_keys, text_tokens, device, lowrank=None):
        """WanBlockB200.buffers for this shard's heads and hidden channels, with the partials and statistics that
        are summed across shards."""
        return Buffers(n, self.dim, self.local_ffn, self.kv_heads, max_keys, text_tokens, device, sharded=True,
                       lowrank=self.lowrank if lowrank is None else lowrank)

    def modulation_of(self, time_in):
        return WanBlockB200.modulation_of(self, time_in)

    # ---- prompt
    def cross_kv(self, context):
        """CrossKV of this shard's heads: the prompt's keys and values are projected and normalized whole (once per
        prompt, replicated), then this shard's heads are quantized for the Sage kernel."""
        lib, st = _native.lib(), _native.stream()
        T, H, d = context.shape[0], self.kv_heads, self.local_dim
        k = self.layers["cross_attn.k"](context)
        v = self.layers["cross_attn.v"](context)
        kf = torch.empty(T, self.dim, device=context.device)
        _native.check(lib.wdl_rms_rows(k.data_ptr(), self.dim, T, self.dim, self.cross_norm_k.data_ptr(), self.eps,
                                       kf.data_ptr(), self.dim, st))
        lpad = -(-T // 128) * 128
        k_i8 = torch.zeros(H, lpad, HEAD_DIM, dtype=torch.int8, device=context.device)
        k_scale = torch.zeros(H, lpad // 64 * 4, device=context.device)
        v_f8 = torch.zeros(H, HEAD_DIM, lpad, dtype=torch.uint8, device=context.device)
        v_scale = torch.zeros(H, HEAD_DIM, device=context.device)
        work = torch.empty(lib.wdl_sage_prep_workspace(T, H), dtype=torch.uint8, device=context.device)
        off = self.rank * d
        _native.check(lib.wdl_sage_prep_kv(None, None, None, None, 0, kf.data_ptr() + off * 4, _native.F32, self.dim,
                                           v.data_ptr() + off * 2, _native.BF16, self.dim, T, H, k_i8.data_ptr(),
                                           k_scale.data_ptr(), v_f8.data_ptr(), v_scale.data_ptr(), work.data_ptr(),
                                           work.numel(), st))
        return CrossKV(k_i8, k_scale, v_f8, v_scale, T)

    # ---- chunk
    # When set (a callable taking (start, stop) CUDA events and the layer's int ops), every GEMM launch of steps is
    # bracketed by CUDA events on the current stream: the benchmark's per-kernel timing of the W4A4 GEMMs.
    gemm_timer = None

    def forward(self, X, mod, cache, at, freq, grid, start, cross, buf, x_is_bf16=False, trace=None, forcing=None,
                entropy_ratio=None):
        """WanBlockB200.forward on this shard: every tensor steps() yields is summed across shards by reduce."""
        if self.reduce is None:
            raise RuntimeError("a tensor-parallel block needs a reduce callable (or run_lockstep over its steps)")
        for t in self.steps(X, mod, cache, at, freq, grid, start, cross, buf, x_is_bf16, forcing, entropy_ratio):
            self.reduce(t)
        return X

    def steps(self, X, mod, cache, at, freq, grid, start, cross, buf, x_is_bf16=False, forcing=None,
              entropy_ratio=None):
        """The block on this shard's heads and hidden channels (WanBlockB200.forward's arguments; cache holds this
        shard's heads, forcing its Forcing-KV split in this shard's head numbers, which changes no collective).
        Yields, in order: the q / k sums of squares [n, 2], the self-attention O partial [n, dim],
        the cross query's sums of squares [n], the cross O partial, the FFN-2 partial; each must hold the sum over
        shards when the generator resumes."""
        if X.dtype != torch.float32 or X.dim() != 2 or not X.is_contiguous():
            raise ValueError("X must be the float32 residual stream [n, dim], contiguous: the kernels read and update "
                             "it as rows")
        lib, st = _native.lib(), _native.stream()
        n, dim, H, d = X.shape[0], self.dim, self.kv_heads, self.local_dim
        ck, cks, cv, cvs, capacity = cache
        fmt, sd = self.code_format, self.act_scale_dtype
        L = self.layers
        mod_ptr = lambda i: mod.data_ptr() + i * dim * 4  # noqa: E731
        timer = WanBlockTP.gemm_timer

        def timed(layer, launch):
            if timer is None:
                return launch()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            launch()
            e1.record()
            timer(e0, e1, 2 * n * layer.N * layer.K)

        def lora(layer, x):
            """The shard's low-rank branch for its input x (its down-projection here, the up-projection onto the
            layer's N in the GEMM epilogue: a wdl_lowrank), or None at rank 0."""
            return layer.lowrank_arg(layer.lowrank_act(x[:n])) if layer.rank else None

        def gemm(layer, out, add=None):
            timed(layer, lambda: _native.check(lib.wdl_w4a4_gemm_lowrank(
                buf.codes.data_ptr(), buf.scales.data_ptr(), layer.codes.data_ptr(), layer.scales.data_ptr(), fmt,
                _native.ptr(layer.bias), add, n, layer.N, layer.K, out.data_ptr(), out.stride(0), st)))

        def partial(layer, codes, scales, add=None):
            f = w4a4.hidden_format(fmt) if codes is buf.hcodes else fmt  # the hidden layer's own format
            timed(layer, lambda: _native.check(lib.wdl_w4a4_gemm_f32_lowrank(
                codes.data_ptr(), scales.data_ptr(), layer.codes.data_ptr(), layer.scales.data_ptr(), f, None, add,
                n, dim, layer.K, buf.partial.data_ptr(), dim, st)))

        def residual(name, gate_row):
            _native.check(lib.wdl_residual_update(buf.partial.data_ptr(), dim, _native.ptr(self.bias[name]),
                                                  None if gate_row is None else mod_ptr(gate_row), X.data_ptr(), dim,
                                                  n, dim, st))

        def ln_quant(shift_row, scale_row, affine, layer, round_bf16):
            """Codes and scales of a column-parallel layer's (whole) input; with a low-rank branch also the bf16
            input itself (buf.xin), whose product with the shard's branch is returned (else None)."""
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

        sumsq = buf.sumsq[:n]
        # self-attention on this shard's heads
        add = ln_quant(0, 1, False, L["self_attn.qkv"], x_is_bf16)
        gemm(L["self_attn.qkv"], buf.qkv, add)  # [n, 3 d]: q | k | v of this shard's heads
        _native.check(lib.wdl_rows_sumsq(buf.qkv.data_ptr(), 3 * d, n, d, 2, d, sumsq.data_ptr(), st))
        yield sumsq
        _native.check(lib.wdl_qkv_prep_sharded(
            buf.qkv.data_ptr(), 3 * d, n, d, self.norm_q.data_ptr(), self.norm_k.data_ptr(), self.eps,
            sumsq.data_ptr(), dim, freq.data_ptr(), freq.shape[1], grid[1], grid[2], start, buf.q.data_ptr(),
            buf.k.data_ptr(), ck.data_ptr(), cks.data_ptr(), cv.data_ptr(), cvs.data_ptr(), capacity, at, st))
        if forcing is None:
            _native.check(lib.wdl_sage_attend(
                buf.q.data_ptr(), d, n, ck.data_ptr(), cks.data_ptr(), cv.data_ptr(), cvs.data_ptr(), at,
                buf.k.data_ptr(), _native.F32, d, None, _native.BF16, 3 * d, n, H,  # V: in the cache (qkv_prep)
                attention_scale(at + n, entropy_ratio), buf.attn.data_ptr(), d, buf.sage.data_ptr(), buf.sage.numel(),
                st))
        else:
            attend_forcing(buf, n, H, cache, at, forcing, entropy_ratio)
        quantize(buf.attn, L["self_attn.o"])
        partial(L["self_attn.o"], buf.codes, buf.scales, lora(L["self_attn.o"], buf.attn))
        yield buf.partial
        residual("self_attn.o", 2)
        # cross-attention on this shard's heads
        # the first residual update made the stream float32 (float32 gates): the later norms round only at the linear
        add = ln_quant(None, None, True, L["cross_attn.q"], False)
        gemm(L["cross_attn.q"], buf.cq, add)
        row_sums = buf.sumsq.view(-1)[:n]
        _native.check(lib.wdl_rows_sumsq(buf.cq.data_ptr(), d, n, d, 1, 0, row_sums.data_ptr(), st))
        yield row_sums
        _native.check(lib.wdl_rms_rows_sharded(buf.cq.data_ptr(), d, n, d, self.cross_norm_q.data_ptr(), self.eps,
                                               row_sums.data_ptr(), dim, buf.q.data_ptr(), d, st))
        _native.check(lib.wdl_sage_quant_q(buf.q.data_ptr(), d, n, H, buf.q_i8.data_ptr(), buf.q_scale.data_ptr(), st))
        _native.check(lib.wdl_sage_attention(buf.q_i8.data_ptr(), buf.q_scale.data_ptr(), cross.k_i8.data_ptr(),
                                             cross.k_scale.data_ptr(), cross.v_f8.data_ptr(), cross.v_scale.data_ptr(),
                                             n, cross.tokens, H, HEAD_DIM ** -0.5, buf.attn.data_ptr(), d, st))
        quantize(buf.attn, L["cross_attn.o"])
        partial(L["cross_attn.o"], buf.codes, buf.scales, lora(L["cross_attn.o"], buf.attn))
        yield buf.partial
        residual("cross_attn.o", None)
        # feed forward on this shard's hidden channels
        fc1, fc2 = L["ffn.0"], L["ffn.2"]
        add = ln_quant(3, 4, False, fc1, False)
        gelu = buf.gelu if fc2.rank else None  # the second layer's branch reads GELU's output (its shard's channels)
        timed(fc1, lambda: _native.check(lib.wdl_w4a4_gemm_gelu_u4_lowrank(
            buf.codes.data_ptr(), buf.scales.data_ptr(), fc1.codes.data_ptr(), fc1.scales.data_ptr(), fmt,
            _native.ptr(fc1.bias), add, _native.ptr(fc2.smooth), w4a4.GELU_SHIFT, sd, n, fc1.N, fc1.K,
            buf.hcodes.data_ptr(), fc1.N, buf.hscales.data_ptr(), _native.ptr(gelu), fc1.N, st)))
        partial(fc2, buf.hcodes, buf.hscales, None if gelu is None else lora(fc2, gelu))
        yield buf.partial
        residual("ffn.2", 5)
