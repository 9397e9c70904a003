"""The chunked rollout (generation/causal.py) on a small random model: passes replayed from CUDA graphs give the
same latents bit for bit as passes launched from Python, through cache filling, a full cache with eviction and a
graph shared by every chunk after it; and the per-chunk RoPE table (time angles of the chunk's frames in rows
0.., run with start 0) gives the same flow as the whole table with the chunk's start."""

import pytest
import torch

pytestmark = pytest.mark.gpu

DIM, HEADS, FFN, LAYERS, TEXT_DIM = 1024, 8, 2048, 2, 512


def model_and_prompt():
    from wan_dit_lab_b200.generation import causal
    model = causal.random_model(dim=DIM, ffn_dim=FFN, num_heads=HEADS, num_layers=LAYERS, text_dim=TEXT_DIM, seed=3,
                                device="cuda")
    text = torch.randn(1, 64, TEXT_DIM, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16).cuda()
    return model, text


def stream(model, text, graphs):
    from wan_dit_lab_b200.generation import causal
    return causal.Stream(model, text, 256, 256, torch.Generator(device="cuda").manual_seed(5), max_frames=9,
                         vae_stride=16, cuda_graph=graphs)


def test_graph_replay_equals_eager_rollout():
    from wan_dit_lab_b200 import _native
    model, text = model_and_prompt()
    eager, graphed = stream(model, text, False), stream(model, text, True)
    noise = torch.randn(48, 15, 16, 16, generator=torch.Generator().manual_seed(6)).cuda()
    for c in range(5):  # the cache (6 frames) is full after two chunks; chunks 3-5 evict and share one graph
        a = eager.next_chunk(noise[:, 3 * c:3 * c + 3])
        b = graphed.next_chunk(noise[:, 3 * c:3 * c + 3])
        torch.cuda.synchronize()
        assert torch.equal(a, b), f"chunk {c}"
        assert torch.isfinite(a).all()
    assert len(graphed.graphs.graphs) == 3  # fill levels 0, 192, then full (384)
    for ce, cg in zip(eager.caches, graphed.caches):
        assert torch.equal(ce.k, cg.k) and torch.equal(ce.vs, cg.vs)
    graphed.reset()  # a new video reuses the recorded graphs
    eager.reset()
    for c in range(2):
        assert torch.equal(eager.next_chunk(noise[:, 3 * c:3 * c + 3]), graphed.next_chunk(noise[:, 3 * c:3 * c + 3]))
    assert len(graphed.graphs.graphs) == 3
    assert _native.device_error() == 0


def test_chunk_rope_table_equals_start_offset():
    model, text = model_and_prompt()
    s = stream(model, text, False)
    noise = torch.randn(48, 6, 16, 16, generator=torch.Generator().manual_seed(7)).cuda()
    s.next_chunk(noise[:, :3])  # the second chunk starts at frame 3
    x = noise[:, 3:6]
    s.chunk_freq[:, :3, :22].copy_(s.freq[:, 3:6, :22])
    shifted = model.forward(x, 750.0, s.grid, s.chunk_freq, 0, s.caches, s.cross, s.buf).clone()
    whole = model.forward(x, 750.0, s.grid, s.freq, 3, s.caches, s.cross, s.buf)
    assert torch.equal(shifted, whole)


def test_graph_replay_with_lowrank_blocks():
    """Blocks with SVDQuant low-rank branches (their float32 products formed by library GEMMs inside the recorded
    pass) replay as they run eagerly."""
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from test_block_gpu import lowrank_parts, random_state
    from wan_dit_lab_b200.generation import causal
    from wan_dit_lab_b200.models.block import WanBlockB200
    edges = causal.random_state(DIM, num_layers=0, text_dim=TEXT_DIM, seed=8, device="cuda")
    blocks = []
    for i in range(LAYERS):
        st = random_state(DIM, FFN, 20 + i)
        blocks.append(WanBlockB200(st, DIM, FFN, HEADS, parts=lowrank_parts(st, 16, 30 + i)))
    model = causal.WanModelB200(edges, DIM, FFN, num_heads=HEADS, num_layers=LAYERS, device="cuda", blocks=blocks)
    text = torch.randn(1, 64, TEXT_DIM, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16).cuda()
    eager, graphed = stream(model, text, False), stream(model, text, True)
    assert hasattr(eager.buf, "xin")
    noise = torch.randn(48, 9, 16, 16, generator=torch.Generator().manual_seed(9)).cuda()
    for c in range(3):
        a = eager.next_chunk(noise[:, 3 * c:3 * c + 3])
        b = graphed.next_chunk(noise[:, 3 * c:3 * c + 3])
        torch.cuda.synchronize()
        assert torch.equal(a, b), f"chunk {c}"
