#!/bin/bash
# Tensor-pipe probes (not part of libg2v.so): standalone sm_100a programs that measure the tcgen05 MMA
# rate for the operand layouts and shapes the kernels use, alone and inside a producer/consumer ring.
set -e
HERE="$(cd "$(dirname "$0")" && pwd)"
for p in tc_rate_probe tc_pipe_probe tc_pipe_probe2; do
    nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -I "$HERE/.." -o "$HERE/$p" "$HERE/$p.cu"
done
