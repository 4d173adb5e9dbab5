#!/bin/sh
# Build libgoib2d.so for sm_100a (see goib2d/build.py, which runs the same commands).
set -e
cd "$(dirname "$0")"
OUT=${1:-../goib2d/libgoib2d.so}
FLAGS="-gencode arch=compute_100a,code=sm_100a -O3 -lineinfo -fmad=false -prec-div=true -prec-sqrt=true -ftz=false -std=c++17 -Xcompiler -fPIC"
nvcc $FLAGS -c step.cu -o step.o
nvcc $FLAGS -c api.cu -o api.o
nvcc -gencode arch=compute_100a,code=sm_100a -shared -o "$OUT" step.o api.o
rm -f step.o api.o
