#!/bin/sh
# Install the reference optimizer package (pykeio/THORN, the `thorn` module) into
# baseline/_ref, unmodified, for the baseline arms of bench.py: the reference's own
# CPU step (`--impl reference`, the `cpu_baseline` object) and its own GPU step
# (`--impl reference_gpu`).  baseline/_ref is git-ignored and travels with the
# working tree to the GPU box.
#
#     sh oracle/install_reference.sh <directory of the reference project>
#
# The project declares hatchling as its build backend, which is not installed
# here, and pip may not write into the project's directory.  So pip builds a
# copy in a temporary directory whose pyproject.toml names setuptools instead;
# the package sources themselves are copied byte for byte, and the script
# checks that the installed module equals the project's.
set -eu
SRC="$1"
HERE="$(cd "$(dirname "$0")" && pwd)"
DEST="$HERE/../baseline/_ref"
TMP="$(mktemp -d)"
trap 'rm -rf "$TMP"' EXIT
cp -r "$SRC/." "$TMP/src"
sed -i 's/requires = \["hatchling"\]/requires = ["setuptools"]/; s/build-backend = "hatchling.build"/build-backend = "setuptools.build_meta"/' \
    "$TMP/src/pyproject.toml"
python -m pip install --quiet --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
    --upgrade --target "$DEST" "$TMP/src"
cmp "$SRC/thorn/thorn.py" "$DEST/thorn/thorn.py"
cmp "$SRC/thorn/__init__.py" "$DEST/thorn/__init__.py"
echo "reference installed into $DEST"
