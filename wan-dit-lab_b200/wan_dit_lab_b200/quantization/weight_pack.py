"""The identity of the checkpoint a weight pack was converted from (reference
src/wan_dit_lab/quantization/weight_pack.py:21-24): a pack's manifest records it, and a reader refuses a pack whose
recorded identity differs from the checkpoint it is asked to stand for."""

from pathlib import Path


def source_identity(path):
    """dict(path, size, mtime_ns) of the resolved checkpoint file: the same three keys as the reference's manifests,
    so that packs written by either side name their source alike."""
    resolved = Path(path).resolve()
    info = resolved.stat()
    return dict(path=str(resolved), size=info.st_size, mtime_ns=info.st_mtime_ns)
