#!/usr/bin/env bash
# Installs the unmodified reference (ckswjd99-lab/AppCorr) into baseline/_ref for
# `bench.py --impl reference`. Offline: wheels come from /opt/wheelhouse only.
#
#   bash baseline/install_reference.sh [REFERENCE_SOURCE_DIR]
#
# The reference's setup.py lists numpy / torchao / realesrgan / triton; torchao and realesrgan
# have no wheel offline, so the install runs with --no-deps (torch, numpy and triton are already
# in the interpreter). Its `offload/` tree has no top-level __init__.py, so setuptools'
# find_packages() skips it; it is copied verbatim next to the installed packages.
set -euo pipefail
SRC="${1:-${APPCORR_REFERENCE_SRC:-/root/reference}}"
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
DEST="$HERE/_ref"
PY="${PYTHON:-python}"
if [ ! -f "$SRC/setup.py" ]; then
  echo "reference source not found at $SRC" >&2
  exit 1
fi
TMP="$(mktemp -d /tmp/appcorr_ref_src.XXXXXX)"
trap 'rm -rf "$TMP"' EXIT
# build from a copy: setuptools writes build/ and *.egg-info into the source tree
cp -a "$SRC/." "$TMP/"
rm -rf "$DEST"
"$PY" -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
  --target "$DEST" "$TMP" >/dev/null
cp -a "$SRC/offload" "$DEST/offload"
echo "installed reference into $DEST"
ls "$DEST"
