#!/bin/bash
# Installs the reference (berattunca21-byte/radeon-igpu-forge) into
# baseline/_ref for bench.py's reference arm. The reference ships no
# packaging metadata, so `pip install ... /path/to/reference` fails; this
# copies it to a temporary directory, adds a minimal pyproject.toml that names
# its own ml.fxlm and ml.fxgpu packages (no code is changed), and installs
# that copy offline. Usage: baseline/install_ref.sh <reference source tree>
set -euo pipefail
SRC=${1:?usage: baseline/install_ref.sh <reference source tree>}
HERE=$(cd "$(dirname "$0")" && pwd)
TMP=$(mktemp -d)
trap 'rm -rf "$TMP"' EXIT
cp -r "$SRC" "$TMP/ref"
cat > "$TMP/ref/pyproject.toml" <<'TOML'
[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "radeon-igpu-forge-ref"
version = "0.0.0"

[tool.setuptools]
packages = ["ml.fxlm", "ml.fxgpu"]

[tool.setuptools.package-data]
"ml.fxlm" = ["kernels/*"]
"ml.fxgpu" = ["*.hip"]
TOML
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
    --target "$HERE/_ref" "$TMP/ref"
