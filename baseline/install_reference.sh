#!/bin/bash
# Installs the unmodified reference into baseline/_ref for `bench.py --impl reference`,
# offline: no index, the image's wheelhouse only, no dependency resolution (one of the
# reference's build requirements is not in the wheelhouse; its runtime imports are).
# The source tree is copied first because the build writes into it.
# usage: bash baseline/install_reference.sh <path to the reference source tree>
set -e
SRC=${1:?usage: install_reference.sh <path to the reference source tree>}
HERE=$(cd "$(dirname "$0")" && pwd)
TMP=$(mktemp -d)
cp -r "$SRC" "$TMP/src"
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
    --target "$HERE/_ref" "$TMP/src"
rm -rf "$TMP"
