"""The model's edges around the blocks (generation/causal.py::WanModelB200: text embedding, time embedding and
projection, patch embedding, head and unpatchify) against the reference's WanModel (models/model.py:32-41, 81-84,
models/head.py:13-18) run by its own code under bfloat16 autocast on the CPU, as its Stream runs the model
(tests/golden/model_edges.npz): the same bfloat16 operations on the same weights, equal bit for bit on the CPU.
A stand-in block carries the modulation the constructor stacks; the edges need no GPU."""

from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

G = np.load(Path(__file__).resolve().parent / "golden" / "model_edges.npz")


def model():
    from wan_dit_lab_b200.generation.causal import WanModelB200
    state = {k[len("state."):]: torch.from_numpy(G[k]) for k in G.files if k.startswith("state.")}
    block = SimpleNamespace(modulation=torch.zeros(6, 128))
    return WanModelB200(state, dim=128, ffn_dim=512, freq_dim=256, in_dim=16, out_dim=16, num_heads=1, num_layers=1,
                        device="cpu", blocks=[block])


def test_embeddings_equal_the_reference():
    m = model()
    text = m.text_embedding(torch.from_numpy(G["context"])[0])
    np.testing.assert_array_equal(text.float().numpy(), G["text"][0])
    patches = m.patch_embed(torch.from_numpy(G["x"])[0])
    np.testing.assert_array_equal(patches.float().numpy(), G["patches"][0])
    e0, temb = m.time_in(750.0)
    np.testing.assert_array_equal(temb.float().numpy(), G["temb"][0])
    np.testing.assert_array_equal(e0.numpy(), G["e0"][0])


def test_head_and_unpatchify_equal_the_reference():
    m = model()
    _, temb = m.time_in(750.0)
    out = m.head(torch.from_numpy(G["tokens"])[0], temb, (2, 4, 6))
    assert out.shape == (16, 2, 8, 12)
    np.testing.assert_array_equal(out.float().numpy(), G["out"][0])
