#!/bin/bash
# Builds libfsattn_b200.so in the package directory from the .cu files beside this script (sm_100a only).
set -euo pipefail
here="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
out="$here/../libfsattn_b200.so"
nvcc=${NVCC:-/usr/local/cuda/bin/nvcc}
flags=(-gencode arch=compute_100a,code=sm_100a -O3 -lineinfo -std=c++17 -Xcompiler -fPIC -Xcompiler -fvisibility=hidden
       --expt-relaxed-constexpr ${FSATTN_PTXAS_V:+-Xptxas -v} ${FSATTN_EXTRA_FLAGS:-})
objs=()
mkdir -p "$here/build"
pids=()
for f in "$here"/*.cu; do
    o="$here/build/$(basename "${f%.cu}").o"
    objs+=("$o")
    if [ ! -f "$o" ] || [ "$f" -nt "$o" ] || [ -n "$(find "$here" "$here/../../include" -name '*.cuh' -newer "$o" -o -name '*.h' -newer "$o" 2>/dev/null | head -1)" ]; then
        "$nvcc" "${flags[@]}" -c "$f" -o "$o" &
        pids+=($!)
    fi
done
for p in "${pids[@]:-}"; do [ -n "$p" ] && wait "$p"; done
"$nvcc" -shared -o "$out" "${objs[@]}" -lcudart
echo "built $out"
