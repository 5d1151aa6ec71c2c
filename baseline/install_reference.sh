#!/bin/sh
# Places the reference's Python package (osuT5/, unmodified) in baseline/_ref so
# that bench.py --impl reference can import its logits processors by path.
# `pip install --target baseline/_ref <reference>` is not possible: the reference
# has neither setup.py nor pyproject.toml.  baseline/_ref is git-ignored and
# travels to the GPU box with the rest of the tree.
#   usage: sh baseline/install_reference.sh [REFERENCE_DIR]   (default: /root/reference)
set -e
REF="${1:-/root/reference}"
HERE="$(cd "$(dirname "$0")" && pwd)"
rm -rf "$HERE/_ref"
mkdir -p "$HERE/_ref"
cp -r "$REF/osuT5" "$HERE/_ref/osuT5"
find "$HERE/_ref" -name "__pycache__" -type d -prune -exec rm -rf {} +
echo "reference package copied to $HERE/_ref"
