#!/bin/sh
# Build recipe for the CPU oracle (test infrastructure): oracle/liboracle.so.
# -ffp-contract=off keeps every a*b+c as two roundings, as in the Rust reference.
set -e
cd "$(dirname "$0")"
g++ -O2 -std=c++17 -fPIC -shared -pthread -ffp-contract=off -fno-fast-math \
    -o liboracle.so tensor.cpp model.cpp synth.cpp capi.cpp
