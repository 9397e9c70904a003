"""The FP8 KV cache's bookkeeping on CPU tensors (generation/causal.py::KVCache): which ring slots a full cache's
chunk replaces (the ring tokens earliest in the video, the chunk's token i into the i-th earliest: reference
KVCache.commit / evicted, causal.py:298-337), and Forcing-KV's anchor rows (the sink and the newest finished
frame, causal.py:243-248), checked against a plain restatement of those rules and the reference's own KVCache
(tests/golden/kvcache.npz). Also the host logic of Stream around the passes (the chunk schedule, the write pass,
the window, the Forcing-KV and entropy-ratio wiring), with stand-in models on the CPU."""

import sys
from pathlib import Path

import pytest
import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "wan-dit-lab_b200"))


def restated(frames_done, per, ring_frames, chunk_frames):
    """Frame number and place in frame of every ring slot after `frames_done` chunks, by the reference's rules."""
    ring = ring_frames * per
    frame_of = [0] * ring
    place = [0] * ring
    saved, frames, history = 0, 0, []
    n = chunk_frames * per
    for _ in range(frames_done):
        if saved + n <= ring:
            for i in range(n):
                frame_of[saved + i], place[saved + i] = frames + i // per, i % per
            saved += n
        else:
            order = sorted(range(ring), key=lambda s: frame_of[s] * per + place[s])[:n]
            history.append(order)
            for i, s in enumerate(order):
                frame_of[s], place[s] = frames + i // per, i % per
        frames += chunk_frames
    return frame_of, place, history


def test_eviction_order_and_anchors_follow_the_reference():
    from wan_dit_lab_b200.generation.causal import KVCache
    per, chunk, ring_frames, heads = 4, 3, 6, 2
    n = chunk * per
    cache = KVCache(ring_frames * per, 0, n, heads, "cpu")
    cache.set_heads([1], heads)
    moved = []
    for c in range(5):
        at = cache.saved
        marker = torch.full((n, heads, 128), c + 1, dtype=torch.uint8)
        cache.k[at:at + n] = marker  # the chunk's keys, as a pass writes them at `saved`
        full_before = cache.full()
        cache.commit(chunk, per)
        if full_before:
            moved.append([int(r) for r in (cache.k[:, 0, 0] == c + 1).nonzero().flatten() if r < ring_frames * per])
    frame_of, place, history = restated(5, per, ring_frames, chunk)
    assert cache.frame_of.tolist() == frame_of and cache.place_in_frame.tolist() == place
    assert [sorted(h) for h in history] == moved
    # the newest finished frame's rows, after the (empty) sink
    newest = max(frame_of)
    want = sorted(s for s in range(len(frame_of)) if frame_of[s] == newest)
    assert sorted(cache.anchor_tokens.tolist()) == want
    static, dynamic, anchors = cache.forcing()
    assert static.tolist() == [1] and dynamic.tolist() == [0] and anchors is cache.anchor_tokens


def test_forcing_applies_only_to_a_full_cache_with_static_heads():
    from wan_dit_lab_b200.generation.causal import KVCache
    cache = KVCache(24, 0, 12, 3, "cpu")
    assert cache.forcing() is None
    cache.set_heads([0, 2], 3)
    cache.commit(3, 4)
    assert cache.forcing() is None  # not full yet
    cache.commit(3, 4)
    assert cache.full() and cache.forcing() is not None
    cache.set_heads([], 3)
    assert cache.forcing() is None
    cache.reset()
    assert cache.saved == 0 and not cache.place_in_frame.any()
    try:
        cache.set_heads([5], 3)
    except ValueError:
        pass
    else:
        raise AssertionError("a head out of range must be refused")


def test_cache_matches_reference_golden():
    """Against the reference KVCache itself (tests/golden/kvcache.npz, made by tests/golden/make_golden.py): the
    slots every commit fills, frame_of and place_in_frame after it, and the anchor rows once full."""
    import numpy as np
    from wan_dit_lab_b200.generation.causal import KVCache
    d = np.load(Path(__file__).resolve().parent / "golden" / "kvcache.npz")
    per, chunk, ring_frames, heads = 4, 3, 6, 2
    n = chunk * per
    for sink_frames in (0, 3):
        key = f"sink{sink_frames}"
        cache = KVCache((ring_frames + sink_frames) * per, sink_frames * per, n, heads, "cpu")
        cache.set_heads([1], heads)
        for step in range(d[key + "_slots"].shape[0]):
            at = cache.saved
            ring_before = cache.k[:, 0, 0].clone()
            cache.k[at:at + n] = step + 1  # mark the chunk's rows
            full = cache.full()
            cache.commit(chunk, per)
            want = d[key + "_slots"][step]
            want = want[want >= 0]
            if full:  # the chunk's token i went to ring slot want[i]
                got = [int(cache.k[sink_frames * per + s, 0, 0]) for s in want]
                assert got == [step + 1] * len(want)
                assert not torch.equal(cache.k[:, 0, 0], ring_before)
            np.testing.assert_array_equal(cache.frame_of.numpy(), d[key + "_frame_of"][step])
            np.testing.assert_array_equal(cache.place_in_frame.numpy(), d[key + "_place"][step])
            if d[key + "_anchors"][step][0] >= 0:
                np.testing.assert_array_equal(cache.anchor_tokens.numpy(), d[key + "_anchors"][step])


def test_static_heads_split_across_shards():
    """Forcing-KV's static heads in the model's numbering go to the shards that hold them, renumbered; out of
    range is an error; one shard is the whole model."""
    from wan_dit_lab_b200.generation.causal import shard_heads
    static = [1, 5, 6]
    assert shard_heads(static, 0, 1, 8) == [1, 5, 6]
    assert [shard_heads(static, r, 2, 4) for r in range(2)] == [[1], [1, 2]]
    assert [shard_heads(static, r, 4, 2) for r in range(4)] == [[1], [], [1], [0]]
    assert shard_heads(None, 0, 2, 4) == []
    with pytest.raises(ValueError):
        shard_heads([8], 1, 2, 4)
    with pytest.raises(ValueError):
        shard_heads([-1], 0, 2, 4)


def test_stream_gives_each_cache_its_shards_static_heads():
    """Stream(static_heads=...) on a tensor-parallel shard: every block's cache gets the static heads among the
    shard's own, renumbered (keys may be ints or strings, as the reference's presets give them). A stand-in model
    on the CPU: the constructor only sizes and wires the caches and scratch."""
    from types import SimpleNamespace
    from wan_dit_lab_b200.generation.causal import Stream

    class Shard:
        kv_heads, rank, world, lowrank = 4, 1, 2, False

        def buffers(self, *args, **kwargs):
            return None

    model = SimpleNamespace(blocks=[Shard(), Shard(), Shard()], out_dim=48, device="cpu",
                            cross_kvs=lambda context: [SimpleNamespace(tokens=context.shape[1])])
    s = Stream(model, torch.zeros(1, 8, 16), 64, 64, vae_stride=16, max_frames=9, static_heads={0: [1, 5], "2": [6, 7]})
    assert [c.static_heads for c in s.caches] == [[1], None, [2, 3]]
    assert all(c.heads == 4 for c in s.caches)
    with pytest.raises(ValueError):
        Stream(model, torch.zeros(1, 8, 16), 64, 64, vae_stride=16, max_frames=9, static_heads={1: [8]})


def test_attention_entropy_scale_follows_the_reference():
    """attention_scale (reference KVCache.scale, causal.py:138-142): 1 / sqrt(d) without a ratio, else
    sqrt(log(N) / log(N r) / d); Stream hands its ratio to every cache."""
    import math
    from types import SimpleNamespace
    from wan_dit_lab_b200.generation.causal import Stream
    from wan_dit_lab_b200.models.block import attention_scale
    assert attention_scale(5568) == 128 ** -0.5
    for keys, r in ((5568, 0.5), (1392, 0.25), (9744, 2.0)):
        assert attention_scale(keys, r) == math.sqrt(math.log(keys) / math.log(keys * r) / 128)
    assert abs(attention_scale(1392, 1.0) - 128 ** -0.5) < 1e-15  # T = N: the trained scale

    class Block:
        kv_heads, lowrank = 2, False

        def buffers(self, *args, **kwargs):
            return None

    model = SimpleNamespace(blocks=[Block(), Block()], out_dim=48, device="cpu",
                            cross_kvs=lambda context: [SimpleNamespace(tokens=context.shape[1])])
    s = Stream(model, torch.zeros(1, 8, 16), 64, 64, vae_stride=16, max_frames=9, attention_entropy_ratio=0.5)
    assert [c.entropy_ratio for c in s.caches] == [0.5, 0.5]
    assert Stream(model, torch.zeros(1, 8, 16), 64, 64, vae_stride=16, max_frames=9).caches[0].entropy_ratio is None


class _Recorder:
    """A stand-in model on the CPU that records each pass (its timestep and input) and predicts a zero flow; the
    stream's schedule, write pass and cache bookkeeping run as they do around the real model."""

    def __init__(self, layers=2):
        from types import SimpleNamespace

        class Block:
            kv_heads, lowrank = 2, False

            def buffers(self, *args, **kwargs):
                return None

        self.blocks = [Block() for _ in range(layers)]
        self.out_dim, self.device, self.calls = 4, "cpu", []
        self.cross_kvs = lambda context: [SimpleNamespace(tokens=context.shape[1])]

    def forward(self, x, t, grid, freq, start, caches, cross, buf):
        self.calls.append((t, x.clone(), [c.saved for c in caches]))
        return torch.zeros_like(x)


def test_stream_schedule_write_pass_and_context_noise():
    """The reference Stream's options around the passes (causal.py:705-738): four denoising passes at 1000 sigma for
    the shifted levels, then the write pass at t = 0 on the clean chunk, or at t = context_noise on the chunk noised
    to it, or none (write_pass False); every cache commits once per chunk either way."""
    import math
    from wan_dit_lab_b200.generation.causal import Stream, sigmas
    ctx = torch.zeros(1, 8, 16)
    for kw, last in ((dict(), 0.0), (dict(context_noise=100), 100.0), (dict(write_pass=False), None),
                     (dict(shift=3.0), 0.0)):
        model = _Recorder()
        s = Stream(model, ctx, 64, 64, generator=torch.Generator().manual_seed(1), vae_stride=16, max_frames=9, **kw)
        noise = torch.randn(s.shape, generator=torch.Generator().manual_seed(2))
        x0 = s.next_chunk(noise)
        levels = sigmas(shift=kw.get("shift", 5.0))
        ts = [c[0] for c in model.calls]
        assert all(math.isclose(t, 1000 * sg) for t, sg in zip(ts, levels))
        assert len(ts) == len(levels) + (last is not None)
        if last is not None:
            assert ts[-1] == last
        # a zero flow: x0 is the pass's input, so the last denoising pass saw the levels' mix of x0 and noise
        assert torch.equal(model.calls[0][1], noise)
        if last == 0.0:
            assert torch.equal(model.calls[-1][1], x0)
        elif last == 100.0:
            assert not torch.equal(model.calls[-1][1], x0)
        # every pass wrote at the same place; the commit after the chunk moved it on
        assert all(c[2] == [0, 0] for c in model.calls)
        assert [c.saved for c in s.caches] == [s.tokens * 3] * 2 and s.start == 3


def test_stream_window_of_a_known_length_and_sink_rule():
    from wan_dit_lab_b200.generation.causal import Stream
    ctx = torch.zeros(1, 8, 16)
    s = Stream(_Recorder(), ctx, 64, 64, vae_stride=16, max_frames=21, frames=9)
    assert s.window == 9 and s.caches[0].max_tokens == 6 * s.tokens
    assert Stream(_Recorder(), ctx, 64, 64, vae_stride=16, max_frames=9, sink_frames=3).caches[0].sink_tokens == 3 * 4
    assert Stream(_Recorder(), ctx, 64, 64, vae_stride=16, max_frames=9, sink_frames=6).caches[0].max_tokens == 24
    with pytest.raises(ValueError):  # 4 sink frames leave 2 ring frames: less than a chunk
        Stream(_Recorder(), ctx, 64, 64, vae_stride=16, max_frames=9, sink_frames=4)



def test_schedule_equals_the_reference():
    """sigmas, STEPS, CHUNK, CONTEXT and SHIFT equal the reference's generation/causal.py (tests/golden/schedule.json,
    made by its own functions)."""
    import json
    from wan_dit_lab_b200.generation import causal
    g = json.loads((Path(__file__).resolve().parent / "golden" / "schedule.json").read_text())
    assert causal.sigmas() == g["sigmas"] and causal.sigmas(shift=3.0) == g["sigmas_shift3"]
    assert (causal.SHIFT, list(causal.STEPS), causal.CHUNK, causal.CONTEXT) == (g["shift"], g["steps"], g["chunk"],
                                                                                 g["context"])
