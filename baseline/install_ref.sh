#!/usr/bin/env bash
# Installs the unmodified reference (sdivyanshu90/build-your-own-distributed-training)
# into baseline/_ref, where `bench.py --impl reference` imports it from.
#
#   bash baseline/install_ref.sh [REFERENCE_SOURCE_DIR]    (default: /root/reference)
#
# Steps, all offline:
#   1. copy the reference to a scratch dir (its source tree is read-only and the
#      setuptools build writes build/ and *.egg-info/ next to it);
#   2. pip install --no-index --no-build-isolation --no-deps from /opt/wheelhouse
#      into baseline/_ref (--no-deps: the reference pins torch<2.7 and only torch
#      2.11 is installed; its other deps, numpy and pyyaml, are present);
#   3. the reference's pyproject packages only `src` itself (not its subpackages),
#      so the install is completed with a verbatim copy of its src/ tree, then
#      checked identical with diff -r.
# baseline/_ref is git-ignored (not product source) but is not gpurun-ignored,
# so it travels with the working tree to the GPU box.
set -euo pipefail
SRC="${1:-/root/reference}"
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
DEST="$HERE/_ref"
TMP="$(mktemp -d /tmp/refcopy.XXXXXX)"
trap 'rm -rf "$TMP"' EXIT
cp -r "$SRC/." "$TMP/"
rm -rf "$DEST"
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
    --target "$DEST" "$TMP" >/dev/null
rm -rf "$DEST/src"
cp -r "$SRC/src" "$DEST/src"
find "$DEST/src" -name '__pycache__' -prune -exec rm -rf {} +
diff -r -x __pycache__ "$SRC/src" "$DEST/src"
echo "reference installed under $DEST"
