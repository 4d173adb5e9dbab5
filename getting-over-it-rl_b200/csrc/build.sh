#!/bin/sh
# Build libgoib2d.so for sm_100a (the engine), and beside it libgoib2d_rotcheck.so (the rot_of self-check the GPU
# tests run). __graft_entry__.build() runs this script.
set -e
cd "$(dirname "$0")"
OUT=${1:-../goib2d/libgoib2d.so}
FLAGS="-gencode arch=compute_100a,code=sm_100a -O3 -lineinfo -fmad=false -prec-div=true -prec-sqrt=true -ftz=false -std=c++17 -Xcompiler -fPIC"
nvcc $FLAGS -c step.cu -o step.o
nvcc $FLAGS -c api.cu -o api.o
nvcc -gencode arch=compute_100a,code=sm_100a -shared -o "$OUT" step.o api.o
nvcc $FLAGS -shared -o "$(dirname "$OUT")/libgoib2d_rotcheck.so" rot_check.cu
rm -f step.o api.o
