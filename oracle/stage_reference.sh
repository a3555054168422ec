#!/usr/bin/env bash
# Stages the reference's own Python package (DWDP) under oracle/_ref for the CPU
# reference arm of bench.py and the oracle checks. Test infrastructure only: the
# staged copy is git-ignored and is never imported by the product path.
#
#   oracle/stage_reference.sh [reference_root]    (default /root/reference)
#
# The reference tree is read-only, so it is copied to a scratch directory first and
# installed from there with pip, offline, without dependencies (torch is present).
set -euo pipefail
SRC="${1:-/root/reference}"
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
DEST="$HERE/_ref"
if [ ! -d "$SRC/DWDP" ]; then
  echo "stage_reference: no reference package under $SRC" >&2
  exit 1
fi
TMP="$(mktemp -d)"
trap 'rm -rf "$TMP"' EXIT
cp -r "$SRC" "$TMP/src"
rm -rf "$DEST"
python -m pip install --quiet --no-index --no-build-isolation --no-deps --target "$DEST" "$TMP/src"
echo "staged the reference package under $DEST"
