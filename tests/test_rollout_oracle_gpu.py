"""The chunked rollout against the oracle: a 2-layer model (dim 1024, 8 heads, FFN 4096) at 512 x 928's token grid
(1392-token chunks of 3 latent frames of 16 x 29), four chunks of the dmd sampler (4 denoising passes and a write
pass each) with a window of 9 frames whose first 3 are a sink: the cache fills (0, 1392, 2784 keys before the
chunk), then the ring evicts its oldest chunk (the fourth chunk attends to the sink, the third chunk and itself).

The GPU rollout runs eagerly through Stream.next_chunk; every layer of every pass records the stream entering and
leaving it, its modulation, the cache fill and the RoPE table, and the caches are copied after every chunk.
Checked against the oracle:
- every layer of the first denoising pass and of the write pass of every chunk, each on its own input and on the
  cache as it stood before the pass: the oracle block (oracle/block.py, the query rows of the full-size test,
  P V over the cache's per-token V as the kernel computes it) updates the stream within the block bar of the
  full-size test (tests/test_block_full_gpu.py: sqrt(2 (1 - 0.999)) + 1e-2);
- the cache's growth and eviction, exactly: the reference's commit (generation/causal.py:298-337, KVCache.commit,
  restated in OracleCache), fed each chunk's keys and values as the write pass stored them, gives the GPU's cache
  byte for byte after every commit, through the fills and the eviction of the ring's oldest chunk.
The oracle's own chained rollout (every layer on the oracle's output of the layer before, over caches of its own) is
reported as well: its distance grows with depth, because the INT4 / INT8 / FP8 requantizations carry every float32
summation-order difference across rounding boundaries; it is printed, not gated."""

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

    records = []  # per pass: per layer the stream in and out, the modulation; the pass's fill and RoPE table
    original = [b.forward for b in model.blocks]

    def recorder(i):
        def forward(X, mod, cache, at, freq, grid, start, cross, buf, **kw):
            if i == 0:
                records.append(dict(at=at, freq=freq.clone(), grid=tuple(grid), start=start, x_in=[], out=[], mods=[]))
            rec = records[-1]
            rec["x_in"].append(X.clone())
            rec["mods"].append(mod.clone())
            out = original[i](X, mod, cache, at, freq, grid, start, cross, buf, **kw)
            rec["out"].append(X.clone())
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
    cap = c0.capacity

    def gpu_cache(chunk, layer):
        """The layer's cache as it stood before the chunk's passes (empty before the first), in the oracle's layout."""
        if chunk == 0:
            return dict(k=np.zeros((1, cap, HEADS, 128), np.uint8), ks=np.zeros((1, cap, HEADS, 1), np.float32),
                        v=np.zeros((1, cap, HEADS, 128), np.uint8), vs=np.zeros((1, cap, HEADS, 1), np.float32))
        k, ks, v, vs = caches_after[chunk - 1][layer]
        return dict(k=k[None].copy(), ks=ks[None, ..., None].copy(), v=v[None].copy(), vs=vs[None, ..., None].copy())

    def oracle_block(rec, layer, X, cache, rows):
        return ob.block(X, rec["mods"][layer].cpu().numpy(), parts[layer], norms[layer], cache, rec["at"],
                        rec["freq"].cpu().numpy(), rec["grid"], rec["start"], ctx, HEADS, rows=rows,
                        x_is_bf16=layer == 0, token_v=True)

    report, isolated = [], []
    for chunk in range(CHUNKS):
        for p in (0, passes - 1):
            rec = records[chunk * passes + p]
            for layer in range(LAYERS):
                X = rec["x_in"][layer].cpu().numpy()
                got = oracle_block(rec, layer, X, gpu_cache(chunk, layer), ROWS)
                err = rel(rec["out"][layer].cpu().numpy()[ROWS] - X[ROWS], got - X[ROWS])
                isolated.append(err)
                report.append(f"chunk {chunk} {'write pass' if p else 'pass 0'} layer {layer}: update relative L2 "
                              f"{err:.4f} (on its own input and the GPU's cache)")

    # the cache's growth and eviction, exactly: the oracle's bookkeeping fed the chunks the GPU wrote
    books = [OracleCache(c0.max_tokens, c0.sink_tokens, n, HEADS) for _ in range(LAYERS)]
    for chunk in range(CHUNKS):
        at = records[chunk * passes]["at"]
        assert at == books[0].saved
        for layer, book in enumerate(books):
            k, ks, v, vs = caches_after[chunk][layer]  # the chunk itself is still at [at, at + n) after commit
            for name, arr in (("k", k[None]), ("ks", ks[None, ..., None]), ("v", v[None]), ("vs", vs[None, ..., None])):
                book.buf[name][:, at:at + n] = arr[:, at:at + n]
            book.commit(stream.chunk, per_frame)
            kept = book.saved
            for name, arr in (("k", k), ("ks", ks), ("v", v), ("vs", vs)):
                ours = book.buf[name][0, :kept].reshape(arr[:kept].shape)
                assert np.array_equal(arr[:kept], ours), (chunk, layer, name)
        report.append(f"chunk {chunk}: cache of {books[0].saved} keys after commit equals the oracle's bookkeeping "
                      f"byte for byte ({'ring evicted' if at + n > c0.max_tokens else 'filling'})")

    # for information: the oracle's own chained rollout over its own caches
    chained = [OracleCache(c0.max_tokens, c0.sink_tokens, n, HEADS) for _ in range(LAYERS)]
    for chunk in range(CHUNKS):
        for p in (0, passes - 1):
            rec = records[chunk * passes + p]
            X = rec["x_in"][0].cpu().numpy()
            x0 = X[ROWS] if p == 0 else X
            for layer in range(LAYERS):
                X = oracle_block(rec, layer, X, chained[layer].buf, ROWS if (p == 0 and layer == LAYERS - 1) else None)
            gpu = rec["out"][LAYERS - 1].cpu().numpy()
            gpu = gpu[ROWS] if p == 0 else gpu
            report.append(f"chunk {chunk} {'write pass' if p else 'pass 0'}: oracle's own chain, stack update "
                          f"relative L2 {rel(gpu - x0, X - x0):.4f} (not gated)")
        for c in chained:
            c.commit(stream.chunk, per_frame)
    print("\n".join(report))
    assert max(isolated) <= BLOCK_BAR, f"a layer's update relative L2 {max(isolated):.4f} > {BLOCK_BAR:.4f}"
