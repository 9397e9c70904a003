"""The RoPE tables of the rollout (generation/causal.py: rope_at, stretch, rope_table) against the reference's own
functions: the plain time / height / width table equals models/rope.py's rows (tests/golden/rope.npz), and the
W4A4 Live preset's table, height and width stretched over the trained token grid (runtime/live_presets.py:50-59,
models/positions.py: native 704x1280 at 480x864, VAE stride 16), equals the one its functions build
(tests/golden/rope_stretched.npz), bit for bit in float32; Stream(rope_scales=...) builds that table."""

from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_plain_table_equals_the_reference_rows():
    from wan_dit_lab_b200.generation.causal import rope_table
    plain = np.load(GOLDEN / "rope.npz")["freq32"]
    np.testing.assert_array_equal(rope_table(plain.shape[1]).numpy(), plain)


def test_stretched_table_equals_the_live_presets():
    from wan_dit_lab_b200.generation.causal import rope_at, rope_table, stretch
    g = np.load(GOLDEN / "rope_stretched.npz")
    scales = stretch([704 // 32, 1280 // 32], [480 // 32, 864 // 32])
    np.testing.assert_array_equal(np.array(scales), g["scales"])
    np.testing.assert_array_equal(rope_table(256, scales=scales).numpy(), g["table"])
    np.testing.assert_array_equal(rope_at(256, 42, 0.5).numpy(), g["at_half"])
    # stretching changes only the height and width pairs
    plain = rope_table(256)
    assert torch.equal(rope_table(256, scales=scales)[..., :22], plain[..., :22])
    assert not torch.equal(rope_table(256, scales=scales)[..., 22:], plain[..., 22:])


def test_stream_builds_the_stretched_table():
    from wan_dit_lab_b200.generation.causal import Stream, rope_table

    class Block:
        kv_heads, lowrank = 2, False

        def buffers(self, *args, **kwargs):
            return None

    model = SimpleNamespace(blocks=[Block()], out_dim=4, device="cpu",
                            cross_kvs=lambda context: [SimpleNamespace(tokens=context.shape[1])])
    scales = [22 / 15, 40 / 27]
    s = Stream(model, torch.zeros(1, 8, 16), 64, 64, vae_stride=16, max_frames=9, rope_scales=scales)
    assert torch.equal(s.freq, rope_table(1024, scales=scales)) and torch.equal(s.chunk_freq, s.freq)
