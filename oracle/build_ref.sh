#!/usr/bin/env bash
# Builds the reference's own op sources, unmodified, against the mock TF/Eigen
# headers in oracle/tf_shim/, into oracle/_ref/:
#   libsdpa_ref_cpu.so  sdpa/sdpa_cpu.cc (CPU OpKernels + CPU functors)
#   libsdpa_ref_gpu.so  the same plus sdpa/sdpa_fwd.cu.cc and sdpa/sdpa_bwd.cu.cc
#                       compiled for sm_100a (the reference's GPU op)
# Test infrastructure only.  Needs the reference checkout (REF_DIR; its
# default is set below); on a machine without it the prebuilt oracle/_ref/*.so
# are used.
# Flags follow the reference's build.sh: -O2, -march=native for the host code
# (here -march=x86-64-v3 so the library also runs on the GPU box's host CPU).
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
REF_DIR="${REF_DIR:-/root/reference}"
SRC="$REF_DIR/sdpa"
OUT="$HERE/_ref"
CUDA="${CUDA_HOME:-/usr/local/cuda}"
if [ ! -f "$SRC/sdpa_cpu.cc" ]; then
  echo "build_ref: reference sources not found at $SRC; keeping prebuilt $OUT" >&2
  exit 0
fi
mkdir -p "$OUT"
TMP="$(mktemp -d)"
trap 'rm -rf "$TMP"' EXIT
SHIM="-I$HERE/tf_shim -I$SRC"
HOSTFLAGS="-O2 -march=x86-64-v3 -fPIC -std=c++17 -Wno-deprecated-declarations -Wno-attributes"

# CPU-only library (GOOGLE_CUDA undefined: exactly the reference's CPU registrations)
g++ $HOSTFLAGS $SHIM -c "$SRC/sdpa_cpu.cc" -o "$TMP/cpu.o"
g++ $HOSTFLAGS -I"$HERE" -c "$HERE/ref_wrap.cc" -o "$TMP/wrap_cpu.o"
g++ -shared -o "$OUT/libsdpa_ref_cpu.so" "$TMP/cpu.o" "$TMP/wrap_cpu.o" -lpthread

# GPU library: the reference kernels for sm_100a (the reference's build.sh gives no -arch)
if [ -x "$CUDA/bin/nvcc" ]; then
  NV="$CUDA/bin/nvcc -std=c++17 -O2 -gencode arch=compute_100a,code=sm_100a -lineinfo -Xcompiler -fPIC --expt-relaxed-constexpr -diag-suppress 2810,611,177,550"
  $NV $SHIM -DGOOGLE_CUDA=1 -x cu -c "$SRC/sdpa_fwd.cu.cc" -o "$TMP/fwd.o"
  $NV $SHIM -DGOOGLE_CUDA=1 -x cu -c "$SRC/sdpa_bwd.cu.cc" -o "$TMP/bwd.o"
  g++ $HOSTFLAGS $SHIM -I"$CUDA/include" -DGOOGLE_CUDA=1 -DTFS_WITH_CUDA_RUNTIME -c "$SRC/sdpa_cpu.cc" -o "$TMP/cpu_g.o"
  g++ $HOSTFLAGS -I"$HERE" -I"$CUDA/include" -DTFS_WITH_CUDA_RUNTIME -c "$HERE/ref_wrap.cc" -o "$TMP/wrap_g.o"
  $CUDA/bin/nvcc -shared -gencode arch=compute_100a,code=sm_100a -o "$OUT/libsdpa_ref_gpu.so" \
    "$TMP/cpu_g.o" "$TMP/wrap_g.o" "$TMP/fwd.o" "$TMP/bwd.o" -lcudart -lpthread
fi
echo "build_ref: built $(ls "$OUT")"
