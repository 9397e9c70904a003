"""This build's operators swapped into the reference's modules, in this process only: the steps of the reference's
runtime/pipeline.py:92-122 install() with a "b200" backend, plus the W4A4, attention and operator call sites.

    restore = install(("rope", "kv_store", "w4a4", "attention", "operators"),
                      attention=wan_dit_lab.models.multi_head_attention, w4a4=wan_dit_lab.quantization.w4a4,
                      causal=wan_dit_lab.generation.causal, sage_kv=wan_dit_lab.kernels.sage_kv,
                      operators=wan_dit_lab.kernels.operators)
    ...                     # the reference's pipeline runs on the B200 kernels
    restore()               # the reference's own functions again

What each step rebinds:
    rope        attention.rope_apply and w4a4.rope_apply (FusedQKVAttention's) -> kernels.rope.rope_apply
    kv_store    causal.KVCache.store's FP8 path -> kernels.cache_fp8.store_kv_fp8 (install_cache_store)
    w4a4        w4a4.quantize, w4a4.w4a4_linear, w4a4.w4a4_gelu_mlp -> quantization.w4a4's: the reference's
                convert / layer_parts / build_pack then make parts in this build's logical format, and its
                PackedW4A4Linear / PackedW4A4GeluMLP run them (they call the module-level functions)
    attention   sage_kv.attend (KVCache.attend imports it at each call) -> kernels.sage_kv.attend
    operators   operators.load -> kernels.operators.load (torch.ops.live.* over this library)
A module a step needs must be given (the reference's module object); nothing here imports the reference."""

STEPS = ("rope", "kv_store", "w4a4", "attention", "operators")
_NEEDS = {"rope": ("attention", "w4a4"), "kv_store": ("causal",), "w4a4": ("w4a4",), "attention": ("sage_kv",),
          "operators": ("operators",)}


def install(steps=STEPS, **modules):
    """Rebinds the call sites of `steps` in the reference's `modules` (attention, w4a4, causal, sage_kv,
    operators) to this build's functions; returns a callable that puts every original back (in reverse order).
    ValueError for an unknown step or a missing module, before anything is changed; if a step raises part of the
    way (an attribute the module lacks, a failed import), the steps already done are undone before it propagates."""
    steps = tuple(steps)
    for step in steps:
        if step not in _NEEDS:
            raise ValueError(f"unknown step {step!r}; steps are {STEPS}")
        missing = [m for m in _NEEDS[step] if modules.get(m) is None]
        if missing:
            raise ValueError(f"step {step!r} needs the reference's module(s) {missing}")
    undo = []

    def rebind(owner, name, value):
        undo.append((owner, name, getattr(owner, name)))
        setattr(owner, name, value)

    def restore():
        while undo:
            owner, name, value = undo.pop()
            setattr(owner, name, value)

    try:
        for step in steps:
            if step == "rope":
                from wan_dit_lab_b200.kernels.rope import rope_apply
                rebind(modules["attention"], "rope_apply", rope_apply)
                rebind(modules["w4a4"], "rope_apply", rope_apply)
            elif step == "kv_store":
                from wan_dit_lab_b200.kernels.cache_fp8 import install_cache_store
                cls = modules["causal"].KVCache
                undo.append((cls, "store", install_cache_store(cls)))
            elif step == "w4a4":
                from wan_dit_lab_b200.quantization import w4a4
                for name in ("quantize", "w4a4_linear", "w4a4_gelu_mlp"):
                    rebind(modules["w4a4"], name, getattr(w4a4, name))
            elif step == "attention":
                from wan_dit_lab_b200.kernels import sage_kv
                rebind(modules["sage_kv"], "attend", sage_kv.attend)
            else:
                from wan_dit_lab_b200.kernels import operators
                rebind(modules["operators"], "load", operators.load)
    except BaseException:
        restore()  # a step that fails part of the way leaves no module half swapped
        raise
    return restore
