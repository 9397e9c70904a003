"""integration.install on stand-ins for the reference's modules (no GPU, no reference import): every step rebinds
exactly the call sites the reference's own install() and call sites use (runtime/pipeline.py:92-122,
quantization/w4a4.py:210-215, generation/causal.py:203-210, kernels/operators.py:19-25), the FP8 store routes
through store_kv_fp8 only for FP8 caches, restore() puts every original back, and a bad request changes nothing."""

from types import SimpleNamespace

import pytest


def stand_ins():
    calls = []

    class KVCache:
        def __init__(self, fp8):
            self.fp8, self.k, self.ks, self.v, self.vs = fp8, "k", "ks", "v", "vs"

        def store(self, at, k, v):
            calls.append(("original store", self.fp8))

    return dict(attention=SimpleNamespace(rope_apply="ref rope"),
                w4a4=SimpleNamespace(rope_apply="ref rope", quantize="ref quantize", w4a4_linear="ref linear",
                                     w4a4_gelu_mlp="ref mlp"),
                causal=SimpleNamespace(KVCache=KVCache), sage_kv=SimpleNamespace(attend="ref attend"),
                operators=SimpleNamespace(load="ref load")), calls


def test_install_rebinds_every_call_site_and_restores_them():
    from wan_dit_lab_b200 import integration
    from wan_dit_lab_b200.kernels import cache_fp8, operators, rope, sage_kv
    from wan_dit_lab_b200.quantization import w4a4
    mods, calls = stand_ins()
    original_store = mods["causal"].KVCache.store
    restore = integration.install(**mods)
    assert mods["attention"].rope_apply is rope.rope_apply and mods["w4a4"].rope_apply is rope.rope_apply
    assert mods["w4a4"].quantize is w4a4.quantize and mods["w4a4"].w4a4_linear is w4a4.w4a4_linear
    assert mods["w4a4"].w4a4_gelu_mlp is w4a4.w4a4_gelu_mlp
    assert mods["sage_kv"].attend is sage_kv.attend and mods["operators"].load is operators.load
    # the bfloat16 cache keeps the reference's store; the FP8 one goes to store_kv_fp8
    mods["causal"].KVCache(fp8=False).store(0, None, None)
    assert calls == [("original store", False)]
    seen = []
    saved, cache_fp8.store_kv_fp8 = cache_fp8.store_kv_fp8, lambda *a: seen.append(a[-1])
    try:
        mods["causal"].KVCache(fp8=True).store(7, None, None)
    finally:
        cache_fp8.store_kv_fp8 = saved
    assert seen == [7]
    restore()
    assert mods["attention"].rope_apply == "ref rope" and mods["w4a4"].rope_apply == "ref rope"
    assert (mods["w4a4"].quantize, mods["w4a4"].w4a4_linear, mods["w4a4"].w4a4_gelu_mlp) == (
        "ref quantize", "ref linear", "ref mlp")
    assert mods["sage_kv"].attend == "ref attend" and mods["operators"].load == "ref load"
    assert mods["causal"].KVCache.store is original_store


def test_bad_requests_change_nothing():
    from wan_dit_lab_b200 import integration
    mods, _ = stand_ins()
    with pytest.raises(ValueError, match="unknown step"):
        integration.install(("rope", "flash"), **mods)
    with pytest.raises(ValueError, match="sage_kv"):
        integration.install(("rope", "attention"), attention=mods["attention"], w4a4=mods["w4a4"])
    assert mods["attention"].rope_apply == "ref rope" and mods["sage_kv"].attend == "ref attend"
    restore = integration.install(("rope",), attention=mods["attention"], w4a4=mods["w4a4"])
    assert mods["sage_kv"].attend == "ref attend"  # only the steps asked for
    restore()
    assert mods["attention"].rope_apply == "ref rope"


def test_a_step_that_fails_part_of_the_way_undoes_the_steps_before_it():
    """A module that lacks an attribute a later step rebinds (here the operators module has no `load`): install
    raises, and the rope / w4a4 / attention call sites it had already swapped are back to the reference's."""
    from types import SimpleNamespace

    from wan_dit_lab_b200 import integration
    mods, _ = stand_ins()
    original_store = mods["causal"].KVCache.store
    mods["operators"] = SimpleNamespace()
    with pytest.raises(AttributeError):
        integration.install(**mods)
    assert mods["attention"].rope_apply == "ref rope" and mods["w4a4"].rope_apply == "ref rope"
    assert (mods["w4a4"].quantize, mods["w4a4"].w4a4_linear, mods["w4a4"].w4a4_gelu_mlp) == (
        "ref quantize", "ref linear", "ref mlp")
    assert mods["sage_kv"].attend == "ref attend"
    assert mods["causal"].KVCache.store is original_store
