"""CPU oracle of the Wan-5B DiT block hot path: a plain restatement of the reference's arithmetic (numpy, and
PyTorch CPU tensors only where a bfloat16 / float8 rounding is needed), each function citing the file:line of
wan-dit-lab it follows.

TEST INFRASTRUCTURE. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may
import it, and only as the checker or the timed CPU baseline. The product path (the package under
wan-dit-lab_b200/) never imports it.

Parity pins: every function is checked against golden vectors made by the reference's own code
(tests/golden/make_golden.py imports the reference's src tree and runs it on seeded inputs; the vectors are
committed as tests/golden/*.npz). The W4A4 GEMM and the activation quantizer of Nunchaku, and SageAttention's
kernel, are third-party code absent from the reference tree; their oracle here follows the published
algorithm and the reference's call sites, pinned where the reference pins it (int4_groups rounding, the Sage
quantizer layouts, the FP8 store bytes). Parity unpinned: the W4A4 GEMM's promotion of the exact group
partials (Nunchaku @ 302e0e9), the fused MLP's unsigned hidden quantizer, and the Sage kernel's P V rounding
(SageAttention 2.2.0) have no golden vector from their own code.
"""
