"""A W4A4 block pack drives the B200 block (quantization/w4a4.py: build_pack -> mapped_pack -> slot), as the
reference's pack tests make and stream theirs (tests/test_w4a4_pack.py:38-62, tests/test_w4a4.py:95-130): blocks
quantized by build_pack itself (SmoothQuant smoothing from calibration maxima, SVDQuant rank 32, the second
feed-forward layer made for the fused GELU MLP) and slotted from a host row or a device row run bit for bit as the
block made directly from the same parts and the same bfloat16 parameters; the parts equal what layer_parts
makes again (the INT4 codes all but a few, which the GPU's SVD may round across a code boundary)."""

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))

pytestmark = pytest.mark.gpu

DIM, HEADS, FFN = 1024, 8, 4096


def run(blk, seed=3):
    from oracle import fp8 as of
    from oracle import rope as orope
    frames, h, w, at, text = 2, 4, 8, 128, 32
    n = frames * h * w
    g = torch.Generator().manual_seed(seed)
    X = torch.randn(n, DIM, generator=g).cuda()
    time_in = (torch.randn(6, DIM, generator=g) * 0.1).cuda()
    ctx = torch.randn(text, DIM, generator=g).to(torch.bfloat16).cuda()
    cap = at + n + 16
    ck8, cks = of.quantize_rows((torch.randn(1, cap, HEADS, 128, generator=g) + 0.3).numpy())
    cv8, cvs = of.quantize_rows(torch.randn(1, cap, HEADS, 128, generator=g).numpy())
    cache = (torch.from_numpy(ck8[0]).cuda(), torch.from_numpy(cks[0, ..., 0]).cuda(),
             torch.from_numpy(cv8[0]).cuda(), torch.from_numpy(cvs[0, ..., 0]).cuda(), cap)
    freq = torch.from_numpy(orope.table(1024).astype(np.float32)).cuda()
    blk.forward(X, blk.modulation_of(time_in), cache, at, freq, (frames, h, w), at // (h * w), blk.cross_kv(ctx),
                blk.buffers(n, at + n, text, "cuda"))
    torch.cuda.synchronize()
    return X.cpu()


def test_pack_rows_run_as_the_blocks_they_were_made_from(tmp_path):
    from test_block_gpu import random_state
    from wan_dit_lab_b200 import _native
    from wan_dit_lab_b200.models.block import WanBlockB200
    from wan_dit_lab_b200.quantization import w4a4
    states = [random_state(DIM, FFN, 70 + i) for i in range(2)]
    g = torch.Generator().manual_seed(72)
    amax = {}
    for i in range(2):
        for first, K in (("self_attn.q", DIM), ("self_attn.o", DIM), ("cross_attn.q", DIM), ("cross_attn.k", DIM),
                         ("cross_attn.v", DIM), ("cross_attn.o", DIM), ("ffn.0", DIM), ("ffn.2", FFN)):
            a = torch.rand(K, generator=g) * 2 + 0.1
            a[torch.randperm(K, generator=g)[:K // 100]] *= 30  # outlier channels
            amax[f"{i}.{first}"] = a
    source = tmp_path / "source.pt"
    source.write_bytes(b"checkpoint identity")
    path = tmp_path / "blocks.w4a4"
    info = w4a4.build_pack(states, amax, path, source, rank=32, fused=True)
    assert info["format"] == "block_w4a4_v2" and info["rank"] == 32
    rows, layout = w4a4.mapped_pack(len(states), path, source)
    for i, state in enumerate(states):
        parts, params = w4a4.slot_parts(rows[i], layout)
        cuda_parts = {layer: {k: v.cuda() for k, v in t.items()} for layer, t in parts.items()}
        # the smoothing and the low-rank branches are in the pack
        assert all(t["proj_down"].shape[1] == 32 for t in parts.values())
        assert not bool((parts["self_attn.qkv"]["smooth"] == 1).all())
        direct = WanBlockB200({k: v.to(torch.bfloat16) for k, v in state.items()}, DIM, FFN, HEADS, parts=cuda_parts)
        expected = run(direct)
        for row in (rows[i], rows[i].cuda()):
            blk = w4a4.slot(row, w4a4.BlockShape(DIM, FFN), layout)
            assert blk.lowrank and blk.code_format == direct.code_format
            assert torch.equal(run(blk), expected)
        assert torch.isfinite(expected).all()
        # the pack holds what layer_parts makes
        again = w4a4.layer_parts(state, i, amax, rank=32, fused=True)
        for layer, t in again.items():
            same = (t["qweight"].cpu() == parts[layer]["qweight"]).float().mean().item()
            assert same >= 0.999, (layer, same)
            for name in ("smooth", "bias", "wscales"):
                a, b = t[name].float().cpu(), parts[layer][name].float()
                assert float((a - b).norm() / b.norm().clamp(min=1e-30)) <= 1e-2, (layer, name)
    assert _native.device_error() == 0
