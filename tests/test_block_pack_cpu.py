"""W4A4 block packs without a GPU (quantization/w4a4.py: pack_layout, build_pack, mapped_pack, slot_parts, slot):
the layout rule equals the reference's own pack_layout (tests/golden/block_pack_layout.json, made by running it);
rows written from given W4A4 tensors map back to the same bytes, name for name; the manifest's digest is the
file's; and the reader refuses what it cannot run, as the reference's mapped_pack does (w4a4.py:397-414):
another checkpoint, another format, a truncated file, the Nunchaku tile order, v1 rows and bfloat16 layers."""

import hashlib
import json
from pathlib import Path

import pytest
import torch

from wan_dit_lab_b200.quantization import w4a4

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "block_pack_layout.json").read_text())
DIM, FFN = GOLDEN["dim"], GOLDEN["ffn_dim"]


def random_block(seed):
    g = torch.Generator().manual_seed(seed)
    return {name: torch.randn(*shape, generator=g) for name, shape in w4a4.block_parameters(DIM, FFN)}


def random_parts(block, fused, rank, seed, keep=()):
    """Tensors of each W4A4 layer with the dtypes and shapes of quantize (random bytes: the pack is bytes)."""
    g = torch.Generator().manual_seed(seed)
    out = {}
    for layer, members in w4a4.layers(block, fused, keep).items():
        N, K = sum(block[f"{m}.weight"].shape[0] for m in members), block[f"{members[0]}.weight"].shape[1]
        t = {}
        for part, (dtype, shape, _) in w4a4.part_shapes(N, K, rank).items():
            if dtype == "uint8":
                t[part] = torch.randint(0, 256, shape, generator=g, dtype=torch.uint8)
            else:
                t[part] = torch.randn(*shape, generator=g).to(getattr(torch, dtype))
        out[layer] = t
    return out


def test_parameters_and_layers_equal_the_reference_block():
    assert [[n, list(s)] for n, s in w4a4.block_parameters(DIM, FFN)] == GOLDEN["parameters"]
    shape = w4a4.BlockShape(DIM, FFN)
    for fused in (False, True):
        assert w4a4.layers(shape, fused) == GOLDEN["layers"][str(fused)]
    # a state dict in another order gives the same layers
    block = random_block(0)
    assert w4a4.layers(dict(reversed(list(block.items()))), True) == GOLDEN["layers"]["True"]


@pytest.mark.parametrize("case", range(len(GOLDEN["cases"])))
def test_layout_equals_the_reference_rule(case):
    c = GOLDEN["cases"][case]
    layout, size = w4a4.pack_layout(w4a4.BlockShape(DIM, FFN), c["fused"], c["rank"], tuple(c["keep"]))
    assert size == c["bytes_per_block"]
    assert layout == c["layout"]
    assert all(e["offset"] % 16 == 0 for e in layout)


@pytest.mark.parametrize("fused,rank,keep", [(True, 32, ()), (True, 0, ()), (False, 16, ()),
                                             (True, 8, ("cross_attn.k",))])
def test_rows_map_back_to_the_written_tensors(tmp_path, fused, rank, keep):
    source = tmp_path / "source.pt"
    source.write_bytes(b"checkpoint identity")
    blocks = [random_block(s) for s in (1, 2, 3)]
    parts = [random_parts(b, fused, rank, 10 + i, keep) for i, b in enumerate(blocks)]
    path = tmp_path / "blocks.w4a4"
    info = w4a4.build_pack(blocks, {}, path, source, rank=rank, fused=fused, keep=keep, parts=parts)
    assert info["format"] == ("block_w4a4_v2" if fused else "block_w4a4_v1") and info["packing"] == "logical"
    assert info["sha256"] == hashlib.sha256(path.read_bytes()).hexdigest()
    rows, layout = w4a4.mapped_pack(blocks, path, source)
    assert rows.shape == (3, info["bytes_per_block"]) and rows.dtype == torch.uint8
    for row, block, p in zip(rows, blocks, parts):
        got_parts, params = w4a4.slot_parts(row, layout)
        assert set(got_parts) == set(p)
        for layer, t in p.items():
            for name in w4a4.PARTS:
                assert got_parts[layer][name].dtype == t[name].dtype, (layer, name)
                assert torch.equal(got_parts[layer][name], t[name]), (layer, name)
        # the other parameters in bfloat16; a W4A4 layer's float bias is not stored (its part is)
        stacked = {m for members in w4a4.layers(block, fused, keep).values() for m in members}
        want = {n for n in block if n.rsplit(".", 1)[0] not in stacked}
        assert set(params) == want
        for name in want:
            assert torch.equal(params[name].reshape(-1), block[name].to(torch.bfloat16).reshape(-1)), name
    with pytest.raises(FileExistsError):
        w4a4.build_pack(blocks, {}, path, source, rank=rank, fused=fused, keep=keep, parts=parts)


def test_reader_refuses_what_it_cannot_run(tmp_path):
    source = tmp_path / "source.pt"
    source.write_bytes(b"checkpoint identity")
    blocks = [random_block(4), random_block(5)]
    path = tmp_path / "blocks.w4a4"
    w4a4.build_pack(blocks, {}, path, source, rank=4, fused=True, parts=[random_parts(b, True, 4, 6) for b in blocks])
    manifest = path.with_suffix(".w4a4.json")
    meta = json.loads(manifest.read_text())
    with pytest.raises(ValueError, match="incomplete"):
        w4a4.mapped_pack(3, path, source)
    other = tmp_path / "other.pt"
    other.write_bytes(b"another checkpoint")
    with pytest.raises(ValueError, match="different checkpoint or format"):
        w4a4.mapped_pack(blocks, path, other)
    for change, message in ((dict(format="block_bf16_v1"), "different checkpoint or format"),
                            (dict(packing=None), "Nunchaku")):
        manifest.write_text(json.dumps({**meta, **change}))
        with pytest.raises(ValueError, match=message):
            w4a4.mapped_pack(blocks, path, source)
    manifest.write_text(json.dumps(meta))
    with path.open("r+b") as f:
        f.truncate(meta["bytes"] - 16)
    with pytest.raises(ValueError, match="incomplete"):
        w4a4.mapped_pack(blocks, path, source)


def test_slot_refuses_v1_rows_and_bfloat16_layers():
    """Checked from the layout alone, before the row goes to a GPU."""
    shape = w4a4.BlockShape(DIM, FFN)
    row = torch.zeros(1, dtype=torch.uint8)
    v1, _ = w4a4.pack_layout(shape, fused=False, rank=0)
    with pytest.raises(ValueError, match="fused=True"):
        w4a4.slot(row, shape, v1)
    kept, _ = w4a4.pack_layout(shape, fused=True, rank=0, keep=("cross_attn.k",))
    with pytest.raises(ValueError, match="bfloat16"):
        w4a4.slot(row, shape, kept)


def test_failed_build_leaves_nothing(tmp_path):
    source = tmp_path / "source.pt"
    source.write_bytes(b"x")
    blocks = [random_block(7), random_block(8)]
    parts = [random_parts(b, True, 4, 9) for b in blocks]
    parts[1]["ffn.0"]["proj_up"] = parts[1]["ffn.0"]["proj_up"][:, :2].contiguous()  # another rank: a wrong shape
    path = tmp_path / "blocks.w4a4"
    with pytest.raises(ValueError, match="ffn.0.proj_up"):
        w4a4.build_pack(blocks, {}, path, source, rank=4, fused=True, parts=parts)
    assert not any(tmp_path.glob("blocks.w4a4*"))
    with pytest.raises(ValueError, match="layout has"):
        w4a4.build_pack(blocks, {}, path, source, rank=4, fused=True, parts=[{}, {}])
    assert not any(tmp_path.glob("blocks.w4a4*"))


def test_slot_builds_the_block_or_a_shard_over_the_rows_views(tmp_path, monkeypatch):
    """slot hands the row's views (no copy on the row's own device) and the shapes from the layout to the block
    class: WanBlockB200, or with shard=(rank, world) WanBlockTP with its reduce callable. The block classes are
    stand-ins here (they need a GPU); what they receive is checked."""
    from wan_dit_lab_b200.models import block, block_tp
    source = tmp_path / "source.pt"
    source.write_bytes(b"checkpoint identity")
    blocks = [random_block(20)]
    path = tmp_path / "blocks.w4a4"
    w4a4.build_pack(blocks, {}, path, source, rank=4, fused=True, parts=[random_parts(blocks[0], True, 4, 21)])
    rows, layout = w4a4.mapped_pack(1, path, source)
    seen = []

    def stand_in(kind):
        def make(state, dim, ffn_dim, heads, *args, **kwargs):
            seen.append((kind, state, dim, ffn_dim, heads, args, kwargs))
            return kind
        return make

    monkeypatch.setattr(block, "WanBlockB200", stand_in("whole"))
    monkeypatch.setattr(block_tp, "WanBlockTP", stand_in("shard"))
    row = rows[0].clone()
    assert w4a4.slot(row, w4a4.BlockShape(DIM, FFN, eps=1e-5), layout, device="cpu") == "whole"
    kind, state, dim, ffn_dim, heads, args, kwargs = seen[-1]
    assert (dim, ffn_dim, heads, args) == (DIM, FFN, DIM // 128, (1e-5,))
    assert kwargs["parts"]["ffn.2"]["qweight"].data_ptr() >= row.data_ptr()  # views of the row, not copies
    assert kwargs["parts"]["ffn.2"]["qweight"].untyped_storage().data_ptr() == row.untyped_storage().data_ptr()
    assert torch.equal(state["norm3.weight"], blocks[0]["norm3.weight"].to(torch.bfloat16))
    reduce = object()
    assert w4a4.slot(row, None, layout, shard=(1, 2), reduce=reduce, device="cpu") == "shard"
    kind, state, dim, ffn_dim, heads, args, kwargs = seen[-1]
    assert args == (1, 2, 1e-6) and kwargs["reduce"] is reduce and kwargs["device"] == torch.device("cpu")
