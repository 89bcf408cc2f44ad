#!/usr/bin/env bash
# Builds the TensorFlow op library `sdpa.so.2.16` (the file name users load
# with tf.load_op_library) from tf_op/ against an installed TensorFlow, linking
# the sm_100a kernels of libsdpa_b200.so.  Needs TensorFlow's headers; run
# `python tf-custom-flash-attention_b200/build.py` first.
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
PKG="$(dirname "$HERE")"
CUDA="${CUDA_HOME:-/usr/local/cuda}"
read -r -a TF_CFLAGS <<< "$(python -c 'import tensorflow as tf; print(" ".join(tf.sysconfig.get_compile_flags()))')"
read -r -a TF_LFLAGS <<< "$(python -c 'import tensorflow as tf; print(" ".join(tf.sysconfig.get_link_flags()))')"
g++ -std=c++17 -O2 -fPIC -shared -DGOOGLE_CUDA=1 "${TF_CFLAGS[@]}" -I"$CUDA/include" \
  "$HERE/sdpa_ops.cc" "$HERE/sdpa_kernels.cc" -o "$PKG/sdpa.so.2.16" \
  "${TF_LFLAGS[@]}" -L"$PKG" -lsdpa_b200 -Wl,-rpath,'$ORIGIN' -L"$CUDA/lib64" -lcudart
echo "built $PKG/sdpa.so.2.16"
