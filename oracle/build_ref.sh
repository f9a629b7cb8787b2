#!/usr/bin/env bash
# Builds the reference ParaConv2d op (GeoND-tech/ParaConv2d) from its own
# unmodified source files into oracle/_ref/libptparaconv2d_ref.so.
#
# Test infrastructure only: the library is the ground truth that the CPU
# restatement in oracle/pc2d_oracle.c is pinned against, the generator of the
# golden fixtures in tests/golden/, and the timed CPU baseline of bench.py.
# It is never part of the product path.
#
# The reference's TORCH_LIBRARY namespace is renamed at compile time
# (-Dptparaconv2d=ptparaconv2d_ref) so that the reference op
# (torch.ops.ptparaconv2d_ref.*) and the product op (torch.ops.ptparaconv2d.*)
# can be loaded into one process.  The source is compiled where it lies;
# nothing is copied.  Unlike the reference's own build script (which passes no
# -O flag) the host code is compiled with -O2; ORACLE_OPT=-O0 reproduces the
# as-shipped build.
#
# Usage: oracle/build_ref.sh [reference_dir]     (default /root/reference)
set -euo pipefail

REF=${1:-/root/reference}
HERE=$(cd "$(dirname "$0")" && pwd)
OUT="$HERE/_ref"
OPT=${ORACLE_OPT:--O2}
PY=${PYTHON:-python}

if [ ! -f "$REF/paraconv2d.cc" ]; then
  echo "reference sources not found under $REF" >&2
  exit 2
fi
mkdir -p "$OUT"
TMP=$(mktemp -d)
trap 'rm -rf "$TMP"' EXIT

TORCH_DIR=$($PY -c 'import torch, os; print(os.path.dirname(torch.__file__))')
PY_INC=$($PY -c 'import sysconfig; print(sysconfig.get_path("include"))')
SITE=$(dirname "$TORCH_DIR")
CUDNN_INC="$SITE/nvidia/cudnn/include"
INC=(-isystem "$TORCH_DIR/include" -isystem "$TORCH_DIR/include/torch/csrc/api/include" -isystem "$PY_INC" -I/usr/local/cuda/include)
DEFS=(-D_GLIBCXX_USE_CXX11_ABI=1 -Dptparaconv2d=ptparaconv2d_ref)
ARCH=(-gencode arch=compute_100a,code=sm_100a)

# The CUDA translation units are only compiled so that the host wrappers in
# paraconv2d.cc link; the oracle never calls them.
for f in paraconv2dkernels paraconv2dgradkernels paraconv2d; do
  nvcc -std=c++17 -c -o "$TMP/$f.cu.o" "$REF/$f.cu" -x cu -Xcompiler -fPIC \
    --expt-relaxed-constexpr "${ARCH[@]}" --device-c "${INC[@]}" -I"$CUDNN_INC" "${DEFS[@]}" -w
done
nvcc "$TMP/paraconv2d.cu.o" "$TMP/paraconv2dkernels.cu.o" "$TMP/paraconv2dgradkernels.cu.o" \
  --output-file "$TMP/link.o" --device-link "${ARCH[@]}" -Xcompiler -fPIC
g++ -std=c++17 $OPT -fPIC "${DEFS[@]}" "${INC[@]}" -c "$REF/paraconv2d.cc" -o "$TMP/paraconv2d.cc.o" -w
g++ -shared -fPIC -o "$OUT/libptparaconv2d_ref.so" "$TMP/paraconv2d.cc.o" "$TMP/paraconv2d.cu.o" \
  "$TMP/paraconv2dkernels.cu.o" "$TMP/paraconv2dgradkernels.cu.o" "$TMP/link.o" \
  -L"$TORCH_DIR/lib" -Wl,-rpath,"$TORCH_DIR/lib" -ltorch -ltorch_cpu -lc10 -lc10_cuda -ltorch_cuda \
  -L/usr/local/cuda/lib64 -Wl,-rpath,/usr/local/cuda/lib64 -lcudart
echo "built $OUT/libptparaconv2d_ref.so ($OPT)"
