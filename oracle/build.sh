#!/bin/sh
# Builds the CPU oracle (test infrastructure; see rwq_oracle.cpp header).
# -ffp-contract=off: the reference never fuses d*q+m or the dot products'
# mul+add, so neither may the restatement.  No -ffast-math.
set -e
here=$(cd "$(dirname "$0")" && pwd)
mkdir -p "$here/_build"
g++ -O2 -std=c++17 -fPIC -shared -ffp-contract=off -fno-fast-math -pthread \
    "$here/rwq_oracle.cpp" -o "$here/_build/librwq_oracle.so.tmp"
mv "$here/_build/librwq_oracle.so.tmp" "$here/_build/librwq_oracle.so"
