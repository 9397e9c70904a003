"""The chunked rollout against the oracle: a 2-layer model (dim 1024, 8 heads, FFN 4096) at 512 x 928's token grid
(1392-token chunks of 3 latent frames of 16 x 29), four chunks of the dmd sampler (4 denoising passes and a write
pass each) with a window of 9 frames whose first 3 are a sink: the cache fills (0, 1392, 2784 keys before the
chunk), then the ring evicts its oldest chunk (the fourth chunk attends to the sink, the third chunk and itself).

The GPU rollout runs eagerly through Stream.next_chunk; every pass records the stream entering the first block and
leaving the last, and the blocks' modulations, cache fill and RoPE table. The oracle replays the block stack on
each recorded input over caches of its own, which only its own write passes fill and which it commits and evicts
by the reference's rule (generation/causal.py:298-337, KVCache.commit): so the cache's growth and eviction across
chunks is the oracle's, not copied from the GPU. Checked per chunk, on the first denoising pass and on the write
pass: the stack's residual update within the block bar of the full-size test (tests/test_block_full_gpu.py:
sqrt(2 (1 - 0.999)) + 1e-2), and after each chunk's commit the cache rows of both layers equal byte for byte but
for values within one rounding of a boundary."""

import math

import numpy as np
import pytest
import torch

from oracle import block as ob
from test_block_gpu import numpy_parts

pytestmark = pytest.mark.gpu

COS_BAR, LINEAR_BAR = 0.999, 1e-2
BLOCK_BAR = math.sqrt(2 * (1 - COS_BAR)) + LINEAR_BAR
DIM, FFN, HEADS, LAYERS, CHUNKS = 1024, 4096, 8, 2, 4
ROWS = np.r_[0:64, 672:704, 1344:1392]


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


class OracleCache:
    """One layer's FP8 cache in the oracle's numpy layout, with the reference's commit and eviction (ring tokens
    replaced earliest in the video first: frame number * tokens per frame + place in the frame)."""

    def __init__(self, max_tokens, sink, n, heads):
        cap = max_tokens + n
        self.buf = dict(k=np.zeros((1, cap, heads, 128), np.uint8), ks=np.zeros((1, cap, heads, 1), np.float32),
                        v=np.zeros((1, cap, heads, 128), np.uint8), vs=np.zeros((1, cap, heads, 1), np.float32))
        self.max_tokens, self.sink, self.n = max_tokens, sink, n
        ring = max_tokens - sink
        self.frame_of, self.place = np.zeros(ring, np.int64), np.zeros(ring, np.int64)
        self.saved, self.frames = 0, 0

    def commit(self, chunk_frames, per_frame):
        at, n, sink = self.saved, self.n, self.sink
        slots = None
        if at + n <= self.max_tokens:
            o = np.arange(max(at, sink), max(at + n, sink))
            slots, i = o - sink, o - at
            self.saved += n
        elif self.max_tokens > sink:
            order = self.frame_of * per_frame + self.place
            slots = np.argsort(order, kind="stable")[:n]  # the n earliest ring tokens, earliest first
            for b in self.buf.values():
                b[:, sink + slots] = b[:, at:at + n].copy()
            i = np.arange(n)
        if slots is not None and len(slots):
            self.frame_of[slots] = self.frames + i // per_frame
            self.place[slots] = i % per_frame
        self.frames += chunk_frames


def test_rollout_matches_the_oracle_over_a_growing_and_evicting_cache():
    from wan_dit_lab_b200 import _native
    from wan_dit_lab_b200.generation.causal import Stream, random_model
    model = random_model(dim=DIM, ffn_dim=FFN, num_heads=HEADS, num_layers=LAYERS, seed=41)
    g = torch.Generator().manual_seed(42)
    context = torch.randn(1, 64, 4096, generator=g).to(torch.bfloat16)
    stream = Stream(model, context.cuda(), 256, 464, generator=torch.Generator(device="cuda").manual_seed(43),
                    max_frames=9, sink_frames=3, cuda_graph=False)
    n, per_frame = stream.chunk * stream.tokens, stream.tokens
    assert n == 1392

    records = []
    original = [b.forward for b in model.blocks]

    def recorder(i):
        def forward(X, mod, cache, at, freq, grid, start, cross, buf, **kw):
            if i == 0:
                records.append(dict(x0=X.clone(), at=at, freq=freq.clone(), grid=tuple(grid), start=start, mods=[],
                                    trace={}))
                kw["trace"] = records[-1]["trace"]  # the first layer's stages, for the report of a failure
            records[-1]["mods"].append(mod.clone())
            out = original[i](X, mod, cache, at, freq, grid, start, cross, buf, **kw)
            if i == LAYERS - 1:
                records[-1]["out"] = X.clone()
            return out
        return forward

    for i, b in enumerate(model.blocks):
        b.forward = recorder(i)
    caches_after = []
    for _ in range(CHUNKS):
        stream.next_chunk()
        caches_after.append([[t.cpu().numpy() for t in (c.k, c.ks, c.v, c.vs)] for c in stream.caches])
    assert _native.device_error() == 0
    passes = len(stream.levels) + 1
    assert len(records) == CHUNKS * passes

    ctx = model.text_embedding(context.cuda())[0].float().cpu().numpy()
    parts = [numpy_parts(b.parts) for b in model.blocks]
    norms = [dict(norm_q=b.norm_q.cpu().numpy(), norm_k=b.norm_k.cpu().numpy(),
                  cross_norm_q=b.cross_norm_q.cpu().numpy(), cross_norm_k=b.cross_norm_k.cpu().numpy(),
                  norm3_w=b.norm3_w.cpu().numpy(), norm3_b=b.norm3_b.cpu().numpy()) for b in model.blocks]
    c0 = stream.caches[0]
    ocaches = [OracleCache(c0.max_tokens, c0.sink_tokens, n, HEADS) for _ in range(LAYERS)]

    def replay(rec, rows=None, trace=None):
        """The oracle's block stack on the recorded input of a pass; rows: the last layer finishes only these;
        trace: receives the first layer's stages."""
        X = rec["x0"].cpu().numpy()
        for layer in range(LAYERS):
            last = layer == LAYERS - 1
            X = ob.block(X, rec["mods"][layer].cpu().numpy(), parts[layer], norms[layer], ocaches[layer].buf,
                         rec["at"], rec["freq"].cpu().numpy(), rec["grid"], rec["start"], ctx, HEADS,
                         rows=rows if last else None, x_is_bf16=layer == 0, trace=trace if layer == 0 else None)
        return X

    report, updates, caches_equal = [], [], []
    for chunk in range(CHUNKS):
        first, write = records[chunk * passes], records[chunk * passes + passes - 1]
        assert first["at"] == ocaches[0].saved == write["at"]
        x0 = first["x0"].cpu().numpy()[ROWS]
        got = replay(first, ROWS)
        updates.append((f"chunk {chunk} pass 0", rel(first["out"].cpu().numpy()[ROWS] - x0, got - x0)))
        x0 = write["x0"].cpu().numpy()
        stages = {}
        got = replay(write, trace=stages)  # every row of both layers: its keys and values are what the cache keeps
        updates.append((f"chunk {chunk} write pass", rel(write["out"].cpu().numpy() - x0, got - x0)))
        report.append(f"chunk {chunk} write pass, first layer: " + ", ".join(
            f"{k} {rel(write['trace'][k].float().cpu().numpy(), stages[k]):.2e}" for k in ("qkv", "q", "k", "attn")))
        for c in ocaches:
            c.commit(stream.chunk, per_frame)
        kept = ocaches[0].saved
        for layer in range(LAYERS):
            gk, gks, gv, gvs = caches_after[chunk][layer]
            o = ocaches[layer].buf
            for name, gpu, ours, gs, os_ in (("k", gk, o["k"][0], gks, o["ks"][0, ..., 0]),
                                             ("v", gv, o["v"][0], gvs, o["vs"][0, ..., 0])):
                equal = float((gpu[:kept] == ours[:kept]).mean())
                caches_equal.append((f"chunk {chunk} layer {layer} cache {name}", equal))
                report.append(f"chunk {chunk} layer {layer} cache {name}: bytes equal {equal:.4f}, scales relative "
                              f"L2 {rel(gs[:kept], os_[:kept]):.2e}")
    print("\n".join(report + [f"{k}: stack update relative L2 {v:.4f}" for k, v in updates]))
    assert min(v for _, v in caches_equal) >= 0.99
    worst = max(v for _, v in updates)
    assert worst <= BLOCK_BAR, f"stack update relative L2 {worst:.4f} > {BLOCK_BAR:.4f}"
