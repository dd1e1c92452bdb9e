#!/usr/bin/env bash
# Install the unmodified reference (noamelata/SAGA) into baseline/_ref.
#
# The reference ships no packaging metadata (no setup.py, no pyproject.toml),
# so `pip install <checkout>` refuses it. This recipe copies the checkout to a
# scratch directory, adds a packaging file that only lists the reference's own
# modules (the `attention` package, `speedup`, `lm_eval_saga`), and installs
# that copy offline into baseline/_ref. No reference source file is changed.
# baseline/_ref is git-ignored; it travels to the GPU box with the snapshot.
#
# Usage: bash baseline/install_reference.sh [REFERENCE_CHECKOUT]
set -euo pipefail
REF="${1:-${SAGA_REFERENCE:-/root/reference}}"
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
DEST="$HERE/_ref"
TMP="$(mktemp -d)"
trap 'rm -rf "$TMP"' EXIT
cp -r "$REF" "$TMP/saga_ref"
chmod -R u+w "$TMP/saga_ref"
cat > "$TMP/saga_ref/pyproject.toml" <<'TOML'
[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "saga-reference"
version = "0.0.0"
description = "noamelata/SAGA, installed unmodified as the benchmark's reference arm"

[tool.setuptools]
packages = ["attention"]
py-modules = ["speedup", "lm_eval_saga"]
TOML
rm -rf "$DEST"
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
    --target "$DEST" "$TMP/saga_ref"
python - "$DEST" "$REF" <<'PY'
import filecmp, os, sys
dest, ref = sys.argv[1], sys.argv[2]
for rel in ("attention/attention.py", "attention/triton_atopn.py", "speedup.py", "lm_eval_saga.py"):
    assert filecmp.cmp(os.path.join(dest, rel), os.path.join(ref, rel), shallow=False), rel
print("reference installed unmodified into", dest)
PY
