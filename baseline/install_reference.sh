#!/usr/bin/env bash
# Offline install of the unmodified reference (its model/ and engine/ packages) into
# baseline/_ref, where bench.py's reference legs and the drop-in GPU tests import it.
#
#   bash baseline/install_reference.sh <path of the reference checkout>
#
# The reference ships no packaging metadata, so pip refuses the checkout itself.  The two
# packages are copied to a temporary directory, a minimal pyproject.toml naming them is added
# there (no source file is changed), and that copy is installed with pip from the local wheel
# house only.  baseline/_ref is git-ignored (it is the reference's code, not this project's).
set -euo pipefail
src="${1:?path of the reference checkout}"
here="$(cd "$(dirname "$0")" && pwd)"
tmp="$(mktemp -d)"
trap 'rm -rf "$tmp"' EXIT
cp -r "$src/model" "$src/engine" "$tmp/"
cat > "$tmp/pyproject.toml" <<'TOML'
[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "uttt-reference"
version = "0.0.0"

[tool.setuptools]
packages = ["model", "engine"]
TOML
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
    --target "$here/_ref" --upgrade "$tmp"
