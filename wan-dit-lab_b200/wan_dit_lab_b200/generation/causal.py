"""Chunked autoregressive generation (Self-Forcing's DMD sampler) on the B200 Wan model, after the reference's
src/wan_dit_lab/generation/causal.py (sigmas, KVCache, Stream.next_chunk) and models/model.py (WanModel).

A chunk of `chunk` latent frames is denoised in len(STEPS) passes of the model while it attends to itself and to
the keys / values of the frames before it, kept in an FP8 cache per block; one more pass with t = 0 writes its
clean keys / values, and commit keeps them. The cache is a buffer of max_tokens + chunk tokens: a sink of the
first frames that is never evicted, then a ring; once the ring is full the chunk's tokens replace those of the
oldest frames (the reference's default eviction, causal.py:298-337 without Participative Compression).

The model's edges (patch embedding, time embedding and projection, text embedding, head, unpatchify;
models/model.py:32-84, models/head.py:13-18) run as plain bf16 PyTorch ops (cuBLAS / cuDNN library calls); the
30 blocks run on the B200 kernels (models/block.py).
"""

import math

import torch

from wan_dit_lab_b200 import _native
from wan_dit_lab_b200.models.block import WanBlockB200

SHIFT = 5.0  # timestep_shift of the distilled model (reference causal.py:35)
STEPS = (1000, 750, 500, 250)  # its four timesteps before the shift (causal.py:36)
CHUNK = 3  # latent frames generated together (causal.py:37)
CONTEXT = 21  # latent frames attention looks back at (causal.py:38)


def sigmas(shift=SHIFT, steps=STEPS):
    """sigma = shift u / (1 + (shift - 1) u), u = t / 1000 (reference causal.py:41-45): 1, 0.9375, 0.8333, 0.625."""
    u = torch.tensor(steps, dtype=torch.float64) / 1000
    return (shift * u / (1 + (shift - 1) * u)).tolist()


def rope_at(count, dim, scale=1.0):
    """cos / sin [2, count, dim / 2] float64 of one axis at the positions i * scale (models/rope.py:4-10 at scale 1,
    models/positions.py rope_at otherwise): angle = position * 10000^(-2 j / dim)."""
    pos = torch.arange(count, dtype=torch.float64)[:, None] * scale
    ang = pos * 10000 ** (-2 * torch.arange(dim // 2, dtype=torch.float64) / dim)
    return torch.stack((torch.cos(ang), torch.sin(ang)))


def stretch(trained, now, strength=1.0):
    """Position Interpolation of height and width (models/positions.py stretch): per side (trained / now) ** strength,
    sizes in tokens, 1 where they are equal."""
    return [(t / n) ** strength for t, n in zip(trained, now)]


def rope_table(positions, head_dim=128, scales=None):
    """cos / sin [2, positions, head_dim / 2] float32 of the time / height / width axes (models/rope.py:4-10,
    runtime/live_presets.py:50-59 with float32 tables): dims d - 4 (d // 6), 2 (d // 6), 2 (d // 6); scales (height,
    width): their positions stretched over a trained grid (stretch), as the W4A4 Live preset's table."""
    d = head_dim
    hw = [rope_at(positions, 2 * (d // 6), s) for s in (scales or (1.0, 1.0))]
    return torch.cat([rope_at(positions, d - 4 * (d // 6)), *hw], dim=-1).float()


def shard_heads(static, rank, world, heads):
    """The static heads (Forcing-KV, numbered over the model's heads) that tensor-parallel shard `rank` of `world`
    holds, each holding `heads` consecutive heads, renumbered from 0; ValueError for a head outside the model."""
    first, total = rank * heads, world * heads
    static = list(static or ())
    if any(h < 0 or h >= total for h in static):
        raise ValueError("static heads out of range")
    return [h - first for h in static if first <= h < first + heads]


class KVCache:
    """FP8 keys / values of the finished frames of one block: [max_tokens + chunk tokens, heads, 128] E4M3 with
    one float32 scale per (token, head), the first sink_tokens never evicted (reference KVCache,
    causal.py:48-337, fp8=True, positions "video", no Participative Compression / decay). Forcing-KV's head split
    (set_heads; causal.py:92-102, 222-248): once the cache is full, the static heads attend to the sink, the newest
    finished frame and the chunk only (anchor_tokens, read through the attention's token map), the others to the
    whole window."""

    fp8 = True

    def __init__(self, max_tokens, sink_tokens, n, heads, device, entropy_ratio=None):
        self.max_tokens, self.sink_tokens, self.n, self.heads = max_tokens, sink_tokens, n, heads
        # attention entropy scaling (reference causal.py:80-85, 138-142): with a ratio r, Q K^T over N keys is scaled
        # by sqrt(log_{N r} N / d) instead of 1 / sqrt(d); None: 1 / sqrt(d), as trained
        self.entropy_ratio = entropy_ratio
        cap = max_tokens + n
        self.capacity = cap
        self.k = torch.zeros(cap, heads, 128, dtype=torch.uint8, device=device)
        self.v = torch.zeros_like(self.k)
        self.ks = torch.zeros(cap, heads, device=device)
        self.vs = torch.zeros_like(self.ks)
        ring = max_tokens - sink_tokens
        self.frame_of = torch.zeros(ring, dtype=torch.long, device=device)  # frame number of each ring token
        self.place_in_frame = torch.zeros_like(self.frame_of)  # its index among the tokens of its frame
        self.saved = 0
        self.frames = 0
        self.per_frame = None
        self.static_heads = None
        self.anchor_tokens = None

    def buffers(self):
        return self.k, self.ks, self.v, self.vs, self.capacity

    def full(self):
        return self.saved == self.max_tokens

    def reset(self):
        """An empty cache (buffers kept): nothing saved, frames counted from 0."""
        self.saved, self.frames = 0, 0
        self.frame_of.zero_()
        self.place_in_frame.zero_()

    def set_heads(self, static, heads=None):
        """Forcing-KV: the head numbers that attend to the sink, the newest finished frame and the chunk only, once
        the cache is full (reference KVCache.set_heads, causal.py:98-102); None or empty: every head sees the whole
        window. heads: the cache's head count (checked)."""
        if heads is not None and heads != self.heads:
            raise ValueError(f"the cache holds {self.heads} heads, not {heads}")
        static = sorted(set(static or ()))
        if any(h < 0 or h >= self.heads for h in static):
            raise ValueError("static heads out of range")
        self.static_heads = static or None
        dev = self.k.device
        if self.static_heads is None:
            self.anchor_tokens = None
            return
        self.static_idx = torch.tensor(self.static_heads, dtype=torch.int32, device=dev)
        self.dynamic_idx = torch.tensor([h for h in range(self.heads) if h not in static], dtype=torch.int32,
                                        device=dev)
        self.anchor_tokens = None  # made at the first commit that knows the frame size

    def _order(self):
        """Position in the video of each ring token (reference causal.py:331): frame, then place in its frame."""
        return self.frame_of * self.per_frame + self.place_in_frame

    def place_anchor(self):
        """The cache rows of the sink and of the newest finished frame, into anchor_tokens in place (a recorded
        CUDA graph reads them; reference KVCache.place_anchor, causal.py:243-248)."""
        sink, per = self.sink_tokens, self.per_frame
        if self.anchor_tokens is None:
            self.anchor_tokens = torch.zeros(sink + per, dtype=torch.int32, device=self.k.device)
            self.anchor_tokens[:sink] = torch.arange(sink, dtype=torch.int32, device=self.k.device)
        newest = torch.topk(self._order(), per).indices
        self.anchor_tokens[sink:] = (sink + newest).to(torch.int32)

    def forcing(self):
        """(static heads, dynamic heads, anchor rows) int32 device tensors when the head split applies (static
        heads set, the cache full, a ring beyond the sink), else None."""
        if self.static_heads is None or not self.full() or self.anchor_tokens is None:
            return None
        return self.static_idx, self.dynamic_idx, self.anchor_tokens

    def commit(self, chunk_frames, per_frame):
        """Keeps the chunk last written at `saved` (reference KVCache.commit / evicted, causal.py:298-337): while
        filling it stays where it was written; once full it replaces the ring tokens earliest in the video, the
        chunk's token i going to the i-th earliest."""
        n, at, sink = self.n, self.saved, self.sink_tokens
        self.per_frame = per_frame
        dev = self.k.device
        slots, i = None, None
        if at + n <= self.max_tokens:
            o = torch.arange(max(at, sink), max(at + n, sink), device=dev)  # its tokens past the sink
            slots, i = o - sink, o - at
            self.saved += n
        elif self.max_tokens > sink:
            slots = torch.topk(self._order(), n, largest=False).indices  # ascending: the earliest first
            to = sink + slots
            for buf in (self.k, self.v, self.ks, self.vs):
                buf[to] = buf[at:at + n].clone()
            i = torch.arange(n, device=dev)
        if slots is not None and len(slots):
            self.frame_of[slots] = self.frames + i // per_frame
            self.place_in_frame[slots] = i % per_frame
        self.frames += chunk_frames
        if self.static_heads is not None and self.max_tokens > sink and self.full():
            self.place_anchor()


class WanModelB200:
    """Wan2.2-TI2V-5B-shaped DiT (reference models/model.py WanModel with the Live preset's W4A4 blocks).
    state: the model's state dict (reference parameter names); its blocks are quantized to W4A4 at load."""

    def __init__(self, state, dim=3072, ffn_dim=14336, freq_dim=256, in_dim=48, out_dim=48, num_heads=24,
                 num_layers=30, eps=1e-6, device="cuda", block_parts=None, blocks=None):
        self.dim, self.heads, self.out_dim, self.freq_dim, self.eps = dim, num_heads, out_dim, freq_dim, eps
        self.ffn_dim = ffn_dim
        dev = torch.device(device)
        g = lambda k: state[k].to(dev)  # noqa: E731
        bf = lambda k: state[k].to(dev, torch.bfloat16)  # noqa: E731
        self.patch_w, self.patch_b = bf("patch_embedding.weight"), bf("patch_embedding.bias")
        self.text = [(bf(f"text_embedding.{i}.weight"), bf(f"text_embedding.{i}.bias")) for i in (0, 2)]
        self.time = [(bf(f"time_embedding.{i}.weight"), bf(f"time_embedding.{i}.bias")) for i in (0, 2)]
        self.proj = (bf("time_projection.1.weight"), bf("time_projection.1.bias"))
        self.head_w, self.head_b = bf("head.head.weight"), bf("head.head.bias")
        self.head_mod = g("head.modulation").float()
        if blocks is None:
            blocks = []
            for i in range(num_layers):
                prefix = f"blocks.{i}."
                sub = {k[len(prefix):]: v for k, v in state.items() if k.startswith(prefix)}
                blocks.append(WanBlockB200(sub, dim, ffn_dim, num_heads, eps, device=dev,
                                           parts=None if block_parts is None else block_parts[i]))
        self.blocks = blocks
        # (time_in + modulation) of all blocks in one launch per pass
        self.modulation = torch.stack([b.modulation for b in blocks]).contiguous()  # [layers, 6, dim]
        self.mods = torch.empty_like(self.modulation)
        self.device = dev
        self._times = {}

    # ---- edges (bf16 PyTorch ops, as the reference runs them under autocast)
    def text_embedding(self, context):
        (w0, b0), (w2, b2) = self.text
        h = torch.nn.functional.gelu(torch.nn.functional.linear(context.to(torch.bfloat16), w0, b0), approximate="tanh")
        return torch.nn.functional.linear(h, w2, b2)

    def time_in(self, t):
        """e0 [6, dim] float32 and t_emb [dim] of timestep t (models/model.py:38-41)."""
        omega = 10000 ** (-torch.arange(self.freq_dim // 2, dtype=torch.float64, device=self.device) / (self.freq_dim // 2))
        theta = torch.tensor([float(t)], dtype=torch.float64, device=self.device)[:, None] * omega[None, :]
        s = torch.cat([torch.cos(theta), torch.sin(theta)], dim=1).float().to(torch.bfloat16)
        (w0, b0), (w2, b2) = self.time
        temb = torch.nn.functional.linear(torch.nn.functional.silu(torch.nn.functional.linear(s, w0, b0)), w2, b2)
        e0 = torch.nn.functional.linear(torch.nn.functional.silu(temb), *self.proj).unflatten(1, (6, -1))
        return e0[0].float().contiguous(), temb[0]

    def patch_embed(self, x):
        """[C, f, H, W] latents -> [f (H/2) (W/2), dim] bf16 tokens (Conv3d kernel / stride (1, 2, 2)), row-major: the
        block kernels read and update the stream as contiguous rows (the convolution's tokens come out transposed)."""
        y = torch.nn.functional.conv3d(x[None].to(torch.bfloat16), self.patch_w, self.patch_b, stride=(1, 2, 2))
        return y.flatten(2).transpose(1, 2)[0].contiguous()

    def head(self, X, temb, grid):
        """Head.forward (models/head.py:13-18) and unpatchify (models/model.py:81-84): [out_dim, f, 2h, 2w]."""
        shift, scale = (self.head_mod + temb.float()[None, None]).chunk(2, dim=1)
        xn = torch.nn.functional.layer_norm(X, (self.dim,), eps=self.eps)
        y = torch.nn.functional.linear((xn * (1 + scale[0]) + shift[0]).to(torch.bfloat16), self.head_w, self.head_b)
        f, h, w = grid
        y = y.view(1, f, h, w, 1, 2, 2, self.out_dim)
        return y.permute(0, 7, 1, 4, 2, 5, 3, 6).reshape(self.out_dim, f, h * 2, w * 2)

    def time_cached(self, t):
        """time_in(t), kept per timestep (a rollout uses the same five): no host-to-device copy on later passes."""
        key = float(t)
        got = self._times.get(key)
        if got is None:
            got = self.time_in(t)
            self._times[key] = got
        return got

    def cross_kvs(self, context):
        ctx = self.text_embedding(context)
        return [b.cross_kv(ctx[0] if ctx.ndim == 3 else ctx) for b in self.blocks]

    def forward(self, x, t, grid, freq, start, caches, cross, buf):
        """One pass over a chunk x [C, f, H, W] at timestep t: the flow prediction [out_dim, f, H, W] (float32).
        Every block stores the chunk's keys / values into its cache at cache.saved and attends to [0, saved + n)."""
        e0, temb = self.time_cached(t)
        return self.forward_embedded(x, e0, temb, grid, freq, start, caches, cross, buf)

    def forward_embedded(self, x, e0, temb, grid, freq, start, caches, cross, buf):
        """forward with the timestep already embedded (e0 [6, dim] float32, temb [dim]): every tensor it reads is
        on the device, so that a pass can be recorded into a CUDA graph over fixed buffers."""
        X = self.patch_embed(x).float()
        _native.check(_native.lib().wdl_modulation(e0.data_ptr(), self.modulation.data_ptr(), len(self.blocks), self.dim,
                                                   self.mods.data_ptr(), _native.stream()))
        for i, blk in enumerate(self.blocks):
            forcing = caches[i].forcing()
            kw = {} if forcing is None else {"forcing": forcing}
            if caches[i].entropy_ratio is not None:
                kw["entropy_ratio"] = caches[i].entropy_ratio
            blk.forward(X, self.mods[i], caches[i].buffers(), caches[i].saved, freq, grid, start, cross[i], buf,
                        x_is_bf16=(i == 0), **kw)
        return self.head(X, temb, grid).float()


class PassGraphs:
    """Passes of the model over a chunk replayed from CUDA graphs (reference Pass, causal.py:381-413). A pass reads
    fixed buffers (latents, time embedding, the chunk's RoPE table, caches, prompt keys / values, scratch); what
    changes between chunks on the device side is the cache fill `saved` (where the chunk's keys go and how many
    keys attention reads), so there is one graph per fill level: one per chunk until the cache is full, then one
    for every later chunk. Each is recorded on its first use after one eager run of the same pass (which writes
    the same cache rows the recorded pass then writes again), and a pass is then three device copies and one
    replay: no kernel launched from Python."""

    def __init__(self, model, shape, max_graphs=16):
        dev = model.device
        self.model, self.max_graphs = model, max_graphs
        self.x = torch.empty(shape, device=dev)
        self.e0 = torch.empty(6, model.dim, device=dev)
        self.temb = torch.empty(model.dim, dtype=torch.bfloat16, device=dev)
        self.pool = torch.cuda.graph_pool_handle()
        self.graphs = {}  # saved -> (graph, output)

    def run(self, x, t, grid, freq, caches, cross, buf):
        e0, temb = self.model.time_cached(t)
        self.x.copy_(x)
        self.e0.copy_(e0)
        self.temb.copy_(temb)
        key = caches[0].saved
        entry = self.graphs.pop(key, None)
        if entry is None:
            args = (self.x, self.e0, self.temb, grid, freq, 0, caches, cross, buf)
            self.model.forward_embedded(*args)  # warm-up: lazy initializations happen outside the capture
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, pool=self.pool, capture_error_mode="thread_local"):
                out = self.model.forward_embedded(*args)
            entry = (graph, out)
            if len(self.graphs) >= self.max_graphs:
                self.graphs.pop(next(iter(self.graphs)))
        self.graphs[key] = entry  # most recently used last
        entry[0].replay()
        return entry[1]


class Stream:
    """A video, chunk by chunk (reference Stream with sampler "dmd", kv_fp8, attention "sage", positions "video",
    cross_cache True, causal.py:450-758): next_chunk denoises a chunk in len(levels) passes, writes its keys and
    values with one more pass (write_pass; at t = context_noise, the clean chunk noised to it, 0 as trained), and
    commits them. frames: the video's length when known (the window is no longer than it); shift: of the noise
    levels (sigmas); rope_scales: height and width positions stretched over a trained grid (rope_table)."""

    def __init__(self, model, context, height, width, generator=None, max_frames=CONTEXT, sink_frames=0, chunk=CHUNK,
                 vae_stride=8, positions=1024, cuda_graph=False, static_heads=None, attention_entropy_ratio=None,
                 frames=None, shift=SHIFT, write_pass=True, context_noise=0, rope_scales=None):
        h, w = height // vae_stride, width // vae_stride
        self.tokens = (h // 2) * (w // 2)
        self.grid = (chunk, h // 2, w // 2)
        self.chunk, self.model = chunk, model
        n = chunk * self.tokens
        self.shape = (model.out_dim, chunk, h, w)
        # attention sees at most max_frames with the chunk itself (reference causal.py:471-479); the ring takes a
        # whole chunk at a time: no ring at all (sink and chunk fill the window) or at least a chunk's worth
        window = max_frames if frames is None else min(max_frames, frames)
        if not (sink_frames == window - chunk or 0 <= sink_frames <= window - 2 * chunk):
            raise ValueError(f"sink_frames {sink_frames} leaves no whole chunk of ring in a window of {window}")
        self.window = window
        heads = model.blocks[0].kv_heads  # all of them, or this tensor-parallel shard's
        self.caches = [KVCache((window - chunk) * self.tokens, sink_frames * self.tokens, n, heads, model.device,
                               attention_entropy_ratio) for _ in model.blocks]
        if static_heads:  # Forcing-KV: {block: [static heads]} (reference Stream, causal.py:490-494)
            rank, world = getattr(model.blocks[0], "rank", 0), getattr(model.blocks[0], "world", 1)
            for index, cache in enumerate(self.caches):
                static = static_heads.get(index, static_heads.get(str(index), []))
                cache.set_heads(shard_heads(static, rank, world, heads), heads)
        self.freq = rope_table(positions, scales=rope_scales).to(model.device)
        # the chunk's table: its frames' time angles in rows 0.. (the kernels run with start 0), height / width
        # angles as in the whole table (reference Stream's chunk_freqs), refreshed in place before every chunk
        self.chunk_freq = self.freq.clone()
        self.cross = model.cross_kvs(context.to(model.device))
        text_tokens = self.cross[0].tokens
        self.buf = model.blocks[0].buffers(n, window * self.tokens, text_tokens, model.device,
                                           lowrank=any(getattr(b, "lowrank", False) for b in model.blocks))
        self.levels = sigmas(shift=shift)
        # write_pass False: no pass at t = 0, the cache keeps the keys and values of the last step (of x at the last
        # noise level); context_noise: the timestep the chunk is written at (causal.py:534-538)
        self.write_pass, self.context_noise = write_pass, context_noise
        self.generator = generator
        self.start = 0
        self.graphs = PassGraphs(model, self.shape) if cuda_graph else None
        self.use_graphs = cuda_graph

    def reset(self):
        """A new video under the same prompt: caches emptied (buffers kept), frames counted from 0 again."""
        for cache in self.caches:
            cache.reset()
        self.start = 0

    @torch.no_grad()
    def next_chunk(self, noise=None):
        """Latents [C, chunk, H, W] of the next chunk (reference causal.py:681-758, dmd sampler)."""
        dev = self.model.device
        x = torch.randn(self.shape, generator=self.generator, device=dev) if noise is None else noise
        time_pairs = 64 - 2 * 21  # head_dim 128: the first 22 angle pairs are the time axis
        self.chunk_freq[:, :self.chunk, :time_pairs].copy_(self.freq[:, self.start:self.start + self.chunk, :time_pairs])
        if self.use_graphs:
            run = lambda xx, t: self.graphs.run(xx, t, self.grid, self.chunk_freq, self.caches, self.cross, self.buf)  # noqa: E731
        else:
            run = lambda xx, t: self.model.forward(xx, t, self.grid, self.chunk_freq, 0, self.caches, self.cross,  # noqa: E731
                                                   self.buf)
        x0 = x
        for i, sigma in enumerate(self.levels):
            flow = run(x, 1000 * sigma)
            x0 = x - sigma * flow
            if i + 1 < len(self.levels):
                fresh = torch.randn(x0.shape, generator=self.generator, device=dev)
                x = (1 - self.levels[i + 1]) * x0 + self.levels[i + 1] * fresh
        if self.write_pass:  # the chunk's keys and values for the cache (causal.py:725-738)
            sigma = self.context_noise / 1000
            if sigma > 0:
                fresh = torch.randn(x0.shape, generator=self.generator, device=dev)
                run((1 - sigma) * x0 + sigma * fresh, float(self.context_noise))
            else:
                run(x0, 0.0)
        for cache in self.caches:
            cache.commit(self.chunk, self.tokens)
        self.start += self.chunk
        return x0


def random_block_state(g, dim, ffn_dim, device):
    """One block's random-init weights: N(0, 0.02), norm weights around 1, modulation N(0, 1) / sqrt(dim)."""
    r = lambda *s: torch.randn(*s, generator=g, device=device) * 0.02  # noqa: E731
    st = {}
    for attn in ("self_attn", "cross_attn"):
        for name in ("q", "k", "v", "o"):
            st[f"{attn}.{name}.weight"], st[f"{attn}.{name}.bias"] = r(dim, dim), r(dim)
        st[f"{attn}.norm_q.weight"] = 1 + r(dim)
        st[f"{attn}.norm_k.weight"] = 1 + r(dim)
    st["ffn.0.weight"], st["ffn.0.bias"] = r(ffn_dim, dim), r(ffn_dim)
    st["ffn.2.weight"], st["ffn.2.bias"] = r(dim, ffn_dim), r(dim)
    st["norm3.weight"], st["norm3.bias"] = 1 + r(dim), r(dim)
    st["modulation"] = torch.randn(1, 6, dim, generator=g, device=device) / math.sqrt(dim)
    return st


def random_model(dim=3072, ffn_dim=14336, freq_dim=256, in_dim=48, out_dim=48, num_heads=24, num_layers=30,
                 text_dim=4096, seed=6, device="cuda", shard=None, reduce=None, svd_rank=0):
    """A WanModelB200 of the Wan2.2-TI2V-5B shape with random-init weights (N(0, 0.02)),
    generated on `device` from one seed, one block at a time (each block's float weights are dropped once it
    is quantized to W4A4). shard = (rank, world): this rank's tensor-parallel shard of every block (every rank
    generates the same weights from the seed and keeps its heads and hidden channels); reduce: the in-place sum
    across ranks (torch.distributed.all_reduce). svd_rank: every layer's SVDQuant low-rank branch (0: none; the
    LongLive W4A4 packs carry rank 32), one stream per GPU only."""
    if svd_rank and shard is not None:
        raise ValueError("svd_rank applies to one stream per GPU (the tensor-parallel blocks quantize at rank 0)")
    g = torch.Generator(device=device).manual_seed(seed)
    edges = random_state(dim, freq_dim=freq_dim, in_dim=in_dim, out_dim=out_dim, num_layers=0, text_dim=text_dim,
                         generator=g, device=device)
    if shard is None:
        make = lambda st: WanBlockB200(st, dim, ffn_dim, num_heads, device=device, svd_rank=svd_rank)  # noqa: E731
    else:
        from wan_dit_lab_b200.models.block_tp import WanBlockTP
        make = lambda st: WanBlockTP(st, dim, ffn_dim, num_heads, shard[0], shard[1], device=device,  # noqa: E731
                                     reduce=reduce)
    blocks = [make(random_block_state(g, dim, ffn_dim, device)) for _ in range(num_layers)]
    return WanModelB200(edges, dim, ffn_dim, freq_dim, in_dim, out_dim, num_heads, num_layers, device=device,
                        blocks=blocks)


def random_state(dim=3072, ffn_dim=14336, freq_dim=256, in_dim=48, out_dim=48, num_layers=30, text_dim=4096, seed=6,
                 device="cuda", generator=None):
    """Random-init weights of the Wan2.2-TI2V-5B shape, N(0, 0.02) (norm weights around 1, modulations
    N(0, 1) / sqrt(dim) as WanBlock initializes them), generated on `device` from one seed."""
    g = torch.Generator(device=device).manual_seed(seed) if generator is None else generator
    r = lambda *s: torch.randn(*s, generator=g, device=device) * 0.02  # noqa: E731
    st = {"patch_embedding.weight": r(dim, in_dim, 1, 2, 2), "patch_embedding.bias": r(dim),
          "text_embedding.0.weight": r(dim, text_dim), "text_embedding.0.bias": r(dim),
          "text_embedding.2.weight": r(dim, dim), "text_embedding.2.bias": r(dim),
          "time_embedding.0.weight": r(dim, freq_dim), "time_embedding.0.bias": r(dim),
          "time_embedding.2.weight": r(dim, dim), "time_embedding.2.bias": r(dim),
          "time_projection.1.weight": r(6 * dim, dim), "time_projection.1.bias": r(6 * dim),
          "head.head.weight": r(4 * out_dim, dim), "head.head.bias": r(4 * out_dim),
          "head.modulation": torch.randn(1, 2, dim, generator=g, device=device) / math.sqrt(dim)}
    for i in range(num_layers):
        st.update({f"blocks.{i}.{k}": v for k, v in random_block_state(g, dim, ffn_dim, device).items()})
    return st
