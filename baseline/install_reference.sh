#!/bin/bash
# Installs the reference package (wan-dit-lab, unmodified) into baseline/_ref, where bench.py --impl reference and
# the CPU baseline of bench.py import it from: its own WanBlock, KVCache and RoPE, timed on the host cores. The source
# tree is copied first (the build writes next to it); dependencies are not installed (torch and the rest are the
# environment's own). baseline/_ref is not committed; it travels with the working tree.
#
#   bash baseline/install_reference.sh [path of the reference checkout]
set -euo pipefail
here="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
source_tree="${1:-/root/reference}"
work="$(mktemp -d)"
trap 'rm -rf "$work"' EXIT
cp -r "$source_tree/src" "$source_tree/pyproject.toml" "$source_tree/README.md" "$work/"
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
    --target "$here/_ref" "$work"
python -c "import sys; sys.path.insert(0, '$here/_ref'); import wan_dit_lab.models.block as b; print('installed', b.__file__)"
