#!/usr/bin/env bash
# Offline install of the unmodified reference (haohq19/ssla) into baseline/_ref, so that the
# GPU box (where the reference checkout does not exist) can import it for the reference arms:
# its Triton chunk_gla / scan timed on the B200 (bench.py) and its model_mos.py run over the
# ssla_b200 layers (tests/test_reference_model.py).
#
# The reference checkout has no packaging metadata (no setup.py / pyproject.toml), so pip
# cannot install it directly; the checkout is read-only, so this copies it under /tmp, adds a
# pyproject.toml that lists its modules as they are, and installs the copy with
# `pip --no-index --no-build-isolation --target`.  No reference source file is changed.
#
#   bash baseline/install_ref.sh [/path/to/ssla]
set -euo pipefail
SRC=${1:-/root/reference}
HERE=$(cd "$(dirname "$0")" && pwd)
TMP=$(mktemp -d /tmp/ssla_ref_pkg.XXXXXX)
cp -r "$SRC"/. "$TMP"/
MODS=$(cd "$TMP" && ls *.py | sed 's/\.py$//' | awk '{printf "\"%s\", ", $1}')
cat > "$TMP/pyproject.toml" <<TOML
[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "ssla-reference"
version = "0.0.0"

[tool.setuptools]
py-modules = [${MODS%, }]

[tool.setuptools.packages.find]
where = ["."]
include = ["ops*", "layers*", "utils*", "dataset*"]
namespaces = true

[tool.setuptools.package-data]
"*" = ["*.yaml"]
TOML
rm -rf "$HERE/_ref"
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse --target "$HERE/_ref" "$TMP"
# the model configs are data the reference reads by path (configs/model/*.yaml)
cp -r "$SRC/configs" "$HERE/_ref/ssla_configs"
rm -rf "$TMP"
echo "installed the reference into $HERE/_ref"
