"""Makes the golden vectors of tests/golden/*.npz by running the reference's own code (wan-dit-lab, imported
from its source tree) on small seeded inputs on the CPU. The vectors pin the CPU oracle (oracle/); the
reference itself is not needed afterwards and is never read at test time.

    python tests/golden/make_golden.py /path/to/wan-dit-lab

What each file holds and which reference code made it:
  w4a4_int4_groups.npz  quantization/w4a4.py:81-100 int4_groups(R, "max") on heavy-tailed weights and on
                        bf16 activations with outlier channels
  fp8_rows.npz          quantization/fp8.py:37-41 quantize_rows (the FP8 KV-cache bytes and scales), with
                        the boundary values of the reference's tests/test_cache_fp8.py
  rope.npz              models/rope.py:4-31 rope() tables and rope_apply() on float32 and float64 tables
  norms.npz             models/rms_norm.py:10-13 RMSNorm, models/layer_norm.py:5-7 LayerNorm
  sage_quant.npz        kernels/sage_kv.py:112-124 quant_q, and its Triton _sum_max/_quant_k/_quant_v run by
                        Triton's CPU interpreter (TRITON_INTERPRET=1) over an FP8 cache plus a bf16 chunk
  kv_attend.npz         generation/causal.py:193-273 KVCache(fp8=True).attend (exact SDPA over the cache
                        read back from FP8, the chunk unquantized)
  block.npz             models/block.py:22-29 WanBlock (nn.Linear, float32) on a small seeded block
  kvcache.npz           generation/causal.py:160-337 KVCache bookkeeping (ring slots, eviction, anchors)
  w4a4_calibration.npz  quantization/w4a4.py:80-137 int4_groups(R, "mse") on heavy-tailed weights and gptq(R, H)
                        on correlated inputs with an idle channel (both on the CPU)
  rope_stretched.npz    models/positions.py rope_at / stretch and runtime/live_presets.py:50-59 rope_table's rule:
                        the time / height / width table with height and width stretched over the trained grid
                        (the W4A4 Live preset: native 704x1280, 480x864, VAE stride 16), 256 positions, float32
  model_edges.npz       models/model.py:32-41, 81-84 and models/head.py:13-18: WanModel's text embedding, time
                        embedding / projection, patch embedding, head and unpatchify on a small seeded model,
                        under bfloat16 autocast on the CPU as Stream runs it
  schedule.json         generation/causal.py:36-45 sigmas() at the default shift and at 3, STEPS, CHUNK, CONTEXT
  block_pack_layout.json  quantization/w4a4.py:269-313 layers() and pack_layout() of a small WanBlock, the
                        reference's own functions run with its quantize replaced by one that returns zero tensors
                        of this build's part shapes (its Nunchaku packer is not in the tree), on the CPU
"""

import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"  # before triton is imported: its kernels run on the CPU

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent


def save(name, **arrays):
    np.savez_compressed(HERE / name, **{k: np.asarray(v) for k, v in arrays.items()})
    print(f"{name}: " + ", ".join(f"{k}{tuple(np.asarray(v).shape)}" for k, v in arrays.items()))


def bf16_bits(t):
    return t.to(torch.bfloat16).view(torch.int16).numpy()


def main(reference):
    sys.path.insert(0, str(Path(reference) / "src"))
    from wan_dit_lab.quantization import w4a4
    from wan_dit_lab.quantization.fp8 import quantize_rows
    from wan_dit_lab.models.rope import rope, rope_apply
    from wan_dit_lab.models.rms_norm import RMSNorm
    from wan_dit_lab.models.layer_norm import LayerNorm

    # ---- W4A4 int4 groups
    g = torch.Generator().manual_seed(100)
    R = torch.distributions.StudentT(3.0).sample((48, 256)) * 0.02
    q, s = w4a4.int4_groups(R, rule="max")
    X = torch.randn(37, 512, generator=g)
    X[:, torch.randperm(512, generator=g)[:6]] *= 20
    Xb = X.to(torch.bfloat16)
    qx, sx = w4a4.int4_groups(Xb.float(), rule="max")
    save("w4a4_int4_groups.npz", R=R.numpy(), q=q.numpy(), scale=s.numpy(), x_bf16=bf16_bits(Xb), qx=qx.numpy(),
         sx=sx.numpy(), scale_bf16=bf16_bits(s), scale_f16=s.to(torch.float16).numpy())

    # ---- FP8 rows (KV cache store)
    torch.manual_seed(23)
    k32 = torch.randn(2, 7, 3, 128)
    edge = torch.tensor([0., -0., 1e-15, -1e-15, .5, -.5, 1., -1., 3., -3., 448., -448.]).repeat(8).reshape(1, 1, 1, 96)
    mid = torch.tensor([448., 84.021, -84.021, 1.06251, -1.06251, 1.06249, -1.06249, 0.]).reshape(1, 1, 1, 8)
    out = {}
    for name, x in (("k32", k32), ("edge", edge), ("mid", mid)):
        for dt in (torch.float32, torch.bfloat16, torch.float16):
            xd = x.to(dt)
            f8, sc = quantize_rows(xd)
            key = f"{name}_{str(dt).split('.')[1]}"
            out[key + "_x"] = xd.float().numpy()
            out[key + "_fp8"] = f8.view(torch.uint8).numpy()
            out[key + "_scale"] = sc.numpy()
    save("fp8_rows.npz", **out)

    # ---- RoPE
    d = 128
    tables64 = torch.cat([rope(64, d - 4 * (d // 6)), rope(64, 2 * (d // 6)), rope(64, 2 * (d // 6))], dim=-1)
    tables32 = tables64.float()
    torch.manual_seed(19)
    grid = ((2, 3, 5),)
    x32 = torch.randn(1, 30, 3, 128)  # exactly the 2 x 3 x 5 grid (models/rope.py has no padding)
    xb = x32.to(torch.bfloat16)
    save("rope.npz", freq64=tables64.numpy(), freq32=tables32.numpy(), x32=x32.numpy(), xbf16=bf16_bits(xb),
         start=np.int64(7), grid=np.array(grid[0]),
         out32_f32table=rope_apply(x32, grid, tables32, 7).numpy(),
         out32_f64table=rope_apply(x32, grid, tables64, 7).numpy(),
         outbf16_f32table=bf16_bits(rope_apply(xb, grid, tables32, 7)))

    # ---- norms
    torch.manual_seed(7)
    xn = torch.randn(5, 3072)
    rms = RMSNorm(3072, eps=1e-6)
    with torch.no_grad():
        rms.weight.copy_(torch.randn(3072) * 0.02 + 1.0)
    ln = LayerNorm(3072, eps=1e-6, elementwise_affine=False)
    ln3 = LayerNorm(3072, eps=1e-6, elementwise_affine=True)
    with torch.no_grad():
        ln3.weight.copy_(torch.randn(3072) * 0.1 + 1.0)
        ln3.bias.copy_(torch.randn(3072) * 0.1)
        save("norms.npz", x=xn.numpy(), xbf16=bf16_bits(xn), rms_weight=rms.weight.numpy(),
             rms_f32=rms(xn).numpy(), rms_bf16=rms(xn.to(torch.bfloat16)).float().numpy(),
             ln_f32=ln(xn).numpy(), ln_bf16=bf16_bits(ln(xn.to(torch.bfloat16))),
             ln3_weight=ln3.weight.numpy(), ln3_bias=ln3.bias.numpy(), ln3_f32=ln3(xn).numpy())

    # ---- Sage quantizers over an FP8 cache (Triton under the CPU interpreter) and quant_q
    from wan_dit_lab.kernels import sage_kv
    import triton
    at, n, H, D = 200, 150, 2, 128
    torch.manual_seed(0)
    total = at + n + 64
    ck = (torch.randn(1, total, H, D) + 0.5).to(torch.float8_e4m3fn)
    cv = (torch.randn(1, total, H, D) * 0.7).to(torch.float8_e4m3fn)
    ks = torch.rand(1, total, H, 1) + 0.5
    vs = torch.rand(1, total, H, 1) + 0.5
    K = (torch.randn(1, n, H, D) + 0.5).float()
    V = torch.randn(1, n, H, D).to(torch.bfloat16)
    Q = torch.randn(1, n, H, D).float()
    L = at + n
    T = 64
    tiles = triton.cdiv(L, T)
    unused = lambda: torch.empty(1, dtype=torch.int32)  # noqa: E731
    strides = lambda x: (x.stride(0), x.stride(1), x.stride(2))  # noqa: E731
    k_args = (*strides(ck), *strides(ks), *strides(K))
    v_args = (*strides(cv), *strides(vs), *strides(V))
    k_sum = torch.zeros(1, H, D)
    sage_kv._sum_max[(tiles, H, 1)](ck, ks, K, k_sum, torch.empty_like(k_sum), at, L, *k_args, unused(), unused(),
                                    D=D, T=T, SUM=True, HMAP=False, TMAP=False)
    k_mean = k_sum / L
    blocks = triton.cdiv(L, sage_kv.BLKK)
    k_int8 = torch.empty(1, L, H, D, dtype=torch.int8)
    k_scale = torch.empty(1, H, blocks * 4)
    sage_kv._quant_k[(blocks * 4, H, 1)](ck, ks, K, k_mean, k_int8, k_scale, at, L, *k_args, *strides(k_int8),
                                         unused(), unused(), D=D, BLK=sage_kv.BLKK, HMAP=False, TMAP=False)
    v_max = torch.zeros(1, H, D)
    sage_kv._sum_max[(tiles, H, 1)](cv, vs, V, torch.empty_like(v_max), v_max, at, L, *v_args, unused(), unused(),
                                    D=D, T=T, SUM=False, HMAP=False, TMAP=False)
    v_scale = v_max.clamp(min=1e-8) / sage_kv.V_MAX
    padded = blocks * sage_kv.BLKK
    v_fp8 = torch.zeros(1, D, H, padded, dtype=torch.float8_e4m3fn)
    sage_kv._quant_v[(padded // T, H, 1)](cv, vs, V, v_scale, v_fp8, at, L, *v_args, v_fp8.stride(0),
                                          v_fp8.stride(1), v_fp8.stride(2), unused(), unused(), D=D, T=T,
                                          HMAP=False, TMAP=False)
    q_int8, q_scale = sage_kv.quant_q(Q)
    save("sage_quant.npz", at=np.int64(at), cache_k=ck.view(torch.uint8).numpy(), cache_v=cv.view(torch.uint8).numpy(),
         cache_ks=ks.numpy(), cache_vs=vs.numpy(), K=K.numpy(), V=bf16_bits(V), Q=Q.numpy(), k_sum=k_sum.numpy(),
         k_int8=k_int8.numpy(), k_scale=k_scale.numpy(), v_max=v_max.numpy(), v_scale=v_scale.numpy(),
         v_fp8=v_fp8.view(torch.uint8).numpy(), q_int8=q_int8.numpy(), q_scale=q_scale.numpy())

    # ---- KV cache attention (exact SDPA over the FP8 cache read back)
    from wan_dit_lab.generation.causal import KVCache
    torch.manual_seed(3)
    per, chunk, H, D = 39, 2, 2, 128
    cache = KVCache(4 * chunk * per, chunk * per, fp8=True, chunk=chunk)
    steps = {}
    for step in range(3):
        nq = chunk * per
        Qs = torch.randn(1, nq, H, D)
        Ks = torch.randn(1, nq, H, D) + 0.3
        Vs = torch.randn(1, nq, H, D)  # float32 throughout (the cache reads back in V's dtype)
        at = cache.saved
        A = cache.attend(Qs, Ks, Vs)
        steps.update({f"q{step}": Qs.numpy(), f"k{step}": Ks.numpy(), f"v{step}": Vs.numpy(),
                      f"at{step}": np.int64(at), f"out{step}": A.float().numpy()})
        cache.commit()
    save("kv_attend.npz", per=np.int64(per), chunk=np.int64(chunk), **steps)

    # ---- a small WanBlock in float32
    from wan_dit_lab.models.block import WanBlock
    torch.manual_seed(1)
    block = WanBlock(256, 1024, 2, 1e-6).eval()
    with torch.no_grad():
        for name, p in block.named_parameters():  # N(0, 0.02), norm weights around 1
            p.copy_(torch.randn_like(p) * 0.02 + (1.0 if "norm" in name and name.endswith("weight") else 0.0))
    freqs = torch.cat([rope(1024, d - 4 * (d // 6)), rope(1024, 2 * (d // 6)), rope(1024, 2 * (d // 6))], dim=-1).float()
    Xb = torch.randn(1, 2 * 8 * 16, 256)
    e = torch.randn(1, 6, 256) * 0.1
    context = torch.randn(1, 16, 256)
    with torch.no_grad():
        out = block(Xb, e, grid_sizes=((2, 8, 16),), freqs=freqs, context=context, start_frame=3)
    state = {f"p::{k}": v.numpy() for k, v in block.state_dict().items()}
    save("block.npz", x=Xb.numpy(), e=e.numpy(), context=context.numpy(), out=out.numpy(), start=np.int64(3),
         grid=np.array((2, 8, 16)), **state)


def kvcache_golden(reference):
    """The reference KVCache's bookkeeping (generation/causal.py:160-337) on CPU tensors: six commits of a chunk of
    3 frames x 4 tokens into a window of 6 ring frames, without and with a 3-frame sink, Forcing-KV static head 1;
    after every commit the ring slots the chunk went to (last_slots), frame_of and place_in_frame, and the anchor
    rows (sink + newest finished frame, place_anchor) from the first full cache on."""
    sys.path.insert(0, str(Path(reference) / "src"))
    from wan_dit_lab.generation import causal
    per, chunk, ring_frames, heads, commits = 4, 3, 6, 2, 6
    n = chunk * per
    out = {}
    for sink_frames in (0, 3):
        c = causal.KVCache((ring_frames + sink_frames) * per, sink_frames * per, fp8=True, chunk=chunk)
        c.allocate(torch.zeros(1, n, heads, 8))
        c.set_heads([1], heads)
        slots, frame_of, place, anchors = [], [], [], []
        for step in range(commits):
            c.commit()
            slots.append(np.full(n, -1) if c.last_slots is None else
                         np.pad(c.last_slots.numpy(), (0, n - len(c.last_slots)), constant_values=-1))
            frame_of.append(c.frame_of.numpy().copy())
            place.append(c.place_in_frame.numpy().copy())
            if c.full():
                if not hasattr(c, "anchor_tokens"):  # as attend_split makes it on the first full pass
                    c.anchor_tokens = torch.zeros(c.sink_tokens + c.per_frame, dtype=torch.int32)
                    c.anchor_tokens[:c.sink_tokens] = torch.arange(c.sink_tokens, dtype=torch.int32)
                c.place_anchor()
                anchors.append(c.anchor_tokens.numpy().copy())
            else:
                anchors.append(np.full(c.sink_tokens + c.per_frame, -1, dtype=np.int32))
        key = f"sink{sink_frames}"
        out[key + "_slots"] = np.stack(slots)
        out[key + "_frame_of"] = np.stack(frame_of)
        out[key + "_place"] = np.stack(place)
        out[key + "_anchors"] = np.stack(anchors)
    save("kvcache.npz", **out)


def calibration_golden(reference):
    """The reference's offline rounding options on the CPU: int4_groups(R, "mse") (w4a4.py:80-100) on Student-t
    weights, and gptq(R, H) (w4a4.py:104-137) with H = X^T X of correlated inputs, one input channel idle (H_jj = 0)."""
    sys.path.insert(0, str(Path(reference) / "src"))
    from wan_dit_lab.quantization import w4a4
    torch.manual_seed(41)  # StudentT samples from the global generator
    g = torch.Generator().manual_seed(41)
    R = torch.distributions.StudentT(3.0).sample((64, 512))
    q_mse, s_mse = w4a4.int4_groups(R, rule="mse")
    K, N = 256, 80
    mix = torch.randn(K, K, generator=g) / K ** 0.5
    X = torch.randn(2048, K, generator=g) @ mix + 0.3 * torch.randn(2048, K, generator=g)
    X[:, 77] = 0  # an idle channel
    Rg = torch.randn(N, K, generator=g)
    H = X.T @ X
    q_gptq, s_gptq = w4a4.gptq(Rg, H)
    save("w4a4_calibration.npz", R=R.numpy(), q_mse=q_mse.numpy(), s_mse=s_mse.numpy(), Rg=Rg.numpy(), H=H.numpy(),
         q_gptq=q_gptq.numpy(), s_gptq=s_gptq.numpy())


def rope_stretched_golden(reference):
    """The RoPE table of the W4A4 Live preset by the reference's own functions (runtime/live_presets.py:50-59 with
    models/positions.py): time pairs from rope(), height and width from rope_at() at the positions stretched over
    the trained token grid (stretch()), concatenated and cast to float32 as the preset's rope_dtype says; 256
    positions instead of the preset's 65536 (the table's rows do not depend on the count)."""
    sys.path.insert(0, str(Path(reference) / "src"))
    from wan_dit_lab.models.positions import rope_at, stretch
    from wan_dit_lab.models.rope import rope
    d, count, cell = 128, 256, 2 * 16
    scales = stretch([s // cell for s in (704, 1280)], [480 // cell, 864 // cell])
    tables = [rope(count, d - 4 * (d // 6))] + [rope_at(count, 2 * (d // 6), sc) for sc in scales]
    save("rope_stretched.npz", scales=np.array(scales), table=torch.cat(tables, dim=-1).to(torch.float32).numpy(),
         at_half=rope_at(count, 42, 0.5).numpy())


def model_edges_golden(reference):
    """The edges of the reference's WanModel around the blocks (models/model.py:32-41 text / patch / time
    embeddings, :81-84 head and unpatchify, models/head.py:13-18) on a small seeded model (dim 128, text_dim 64,
    in / out 16), run under bfloat16 autocast on the CPU as its Stream runs the model (one chunk of 2 frames of
    8 x 12 latents, t = 750); the state dict is saved with the outputs."""
    sys.path.insert(0, str(Path(reference) / "src"))
    from wan_dit_lab.models.model import WanModel
    torch.manual_seed(61)
    model = WanModel(dim=128, eps=1e-6, ffn_dim=512, freq_dim=256, in_dim=16, num_heads=1, num_layers=0, out_dim=16,
                     text_len=8, text_dim=64).eval()
    g = torch.Generator().manual_seed(62)
    context = torch.randn(1, 8, 64, generator=g)
    x = torch.randn(1, 16, 2, 8, 12, generator=g)
    tokens = torch.randn(1, 2 * 4 * 6, 128, generator=g)  # the residual stream the head reads (float32)
    t = torch.tensor([750.0])
    with torch.no_grad(), torch.autocast("cpu", dtype=torch.bfloat16):
        text = model.text_embedding(context)
        patches = model.patch_embedding(x).flatten(2).transpose(1, 2)
        omega = 10000 ** (-torch.arange(128, dtype=torch.float64) / 128)
        theta = t.double()[:, None] * omega[None, :]
        temb = model.time_embedding(torch.cat([torch.cos(theta), torch.sin(theta)], dim=1).float())
        e0 = model.time_projection(temb).unflatten(1, (6, -1))
        y = model.head(tokens, temb)
        f, h, w = 2, 4, 6
        out = y.view(1, f, h, w, 1, 2, 2, 16).permute(0, 7, 1, 4, 2, 5, 3, 6).reshape(1, 16, f, h * 2, w * 2)
    state = {k: v.detach().numpy() for k, v in model.state_dict().items()}
    save("model_edges.npz", context=context.numpy(), x=x.numpy(), tokens=tokens.numpy(),
         text=text.float().numpy(), patches=patches.float().numpy(), temb=temb.float().numpy(),
         e0=e0.float().numpy(), out=out.float().numpy(), **{"state." + k: v for k, v in state.items()})


def schedule_golden(reference):
    """The rollout's noise levels and sizes by the reference's own generation/causal.py (sigmas, STEPS, CHUNK,
    CONTEXT, SHIFT)."""
    import json
    sys.path.insert(0, str(Path(reference) / "src"))
    from wan_dit_lab.generation import causal
    out = dict(shift=causal.SHIFT, steps=list(causal.STEPS), chunk=causal.CHUNK, context=causal.CONTEXT,
               sigmas=causal.sigmas(), sigmas_shift3=causal.sigmas(shift=3.0))
    (HERE / "schedule.json").write_text(json.dumps(out, indent=1), encoding="utf-8")
    print("schedule.json:", out)


def block_pack_golden(reference):
    """The reference's pack layout rule (quantization/w4a4.py:269-313) on a WanBlock(256, 512, 2 heads): its
    parameter names and shapes, layers() fused and not, and pack_layout() for packs v1 and v2, rank 32 and 0, with
    and without a layer kept in bfloat16. pack_layout quantizes a zero weight on the GPU to learn the parts'
    shapes; here its quantize is a stand-in returning zero tensors of this build's logical parts (qweight
    [N, K/2] uint8, wscales [K/64, N], proj_down [K, r], proj_up [N, r], smooth [K], bias [N] in bfloat16) and
    its torch.zeros ignores the device, so the rule runs unchanged on the CPU."""
    import json
    import types
    sys.path.insert(0, str(Path(reference) / "src"))
    from wan_dit_lab.models.block import WanBlock
    from wan_dit_lab.quantization import w4a4
    block = WanBlock(256, 512, 2, 1e-6)
    bf = torch.bfloat16

    def stand_in(W, b=None, smooth=None, rank=32, **_):
        N, K = W.shape
        return dict(qweight=torch.zeros(N, K // 2, dtype=torch.uint8), wscales=torch.zeros(K // 64, N, dtype=bf),
                    proj_down=torch.zeros(K, rank, dtype=bf), proj_up=torch.zeros(N, rank, dtype=bf),
                    smooth=torch.zeros(K, dtype=bf), bias=torch.zeros(N, dtype=bf))

    shim = types.ModuleType("torch_zeros_on_cpu")
    shim.__dict__.update(torch.__dict__)
    shim.zeros = lambda *a, device=None, **k: torch.zeros(*a, **k)
    saved = w4a4.torch, w4a4.quantize
    w4a4.torch, w4a4.quantize = shim, stand_in
    try:
        cases = []
        for fused, rank, keep in ((False, 32, ()), (True, 32, ()), (True, 0, ()), (True, 16, ("cross_attn.k",))):
            layout, size = w4a4.pack_layout(block, fused, rank, keep)
            cases.append(dict(fused=fused, rank=rank, keep=list(keep), layout=layout, bytes_per_block=size))
    finally:
        w4a4.torch, w4a4.quantize = saved
    out = dict(dim=256, ffn_dim=512, parameters=[[n, list(p.shape)] for n, p in block.named_parameters()],
               layers={str(f): {g: [n for n, _ in m] for g, m in w4a4.layers(block, f).items()} for f in (False, True)},
               cases=cases)
    (HERE / "block_pack_layout.json").write_text(json.dumps(out, indent=1), encoding="utf-8")
    print(f"block_pack_layout.json: {len(out['parameters'])} parameters, {len(cases)} layouts")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <wan-dit-lab checkout>")
    main(sys.argv[1])
    kvcache_golden(sys.argv[1])
    block_pack_golden(sys.argv[1])
    calibration_golden(sys.argv[1])
    rope_stretched_golden(sys.argv[1])
    model_edges_golden(sys.argv[1])
    schedule_golden(sys.argv[1])
