#!/bin/sh
# Installs the unmodified reference (COMP, package `komp`) into baseline/_ref, for bench.py's reference arm (COMP under
# TRITON_INTERPRET=1 on the host cores, COMP's Triton kernels on the GPU) and tests/test_gpu_vs_komp.py.
#
#   sh baseline/install_ref.sh /path/to/reference-checkout
#
# pip builds the package from a copy of the checkout (the build writes into its source tree; the checkout itself is
# only read), without dependencies: `kurn` and the pinned triton 3.8.0 are not in the offline wheelhouse, and COMP's
# kernels and host code need neither (the image's triton runs them). The reference's patch series is placed beside the
# package, where komp.fork loads the Triton extension module (triton.language.extra.kurn) from (KOMP_PATCHES).
set -eu
SRC=${1:?usage: install_ref.sh REFERENCE_DIR}
HERE=$(cd "$(dirname "$0")" && pwd)
TMP=$(mktemp -d)
cp -r "$SRC" "$TMP/ref"
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse --target "$HERE/_ref" \
    "$TMP/ref"
mkdir -p "$HERE/_ref/patches"
cp "$SRC"/patches/* "$HERE/_ref/patches/"
rm -rf "$TMP"
echo "installed komp into $HERE/_ref"
