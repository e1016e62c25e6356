#!/bin/sh
# Installs the unmodified reference solution into baseline/_ref (git-ignored; it travels to the
# GPU box with the working tree). The reference cannot be pip-installed: it has neither setup.py
# nor pyproject.toml, so its solution tree and config are copied as they are. bench.py's Triton
# timing leg imports baseline/_ref/solution/triton/kernel.py::run from here.
set -e
SRC=${1:?usage: install_ref.sh <reference checkout>}
DST=$(dirname "$0")/_ref
[ -d "$SRC/solution" ] || { echo "no reference at $SRC" >&2; exit 1; }
rm -rf "$DST"
mkdir -p "$DST"
cp -r "$SRC/solution" "$SRC/config.toml" "$DST/"
echo "installed $SRC/solution -> $DST"
