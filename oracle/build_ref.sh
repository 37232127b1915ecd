#!/usr/bin/env bash
# Compile the reference decoder from its own sources (read in place, never
# copied) plus oracle/ref_harness.cc into oracle/_ref/libref_asr.so.
# TEST INFRASTRUCTURE: the resulting library is a parity checker only.
# Usage: oracle/build_ref.sh REFERENCE_ROOT   (or ORATOR_REFERENCE=... oracle/build_ref.sh)
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
R="${1:-${ORATOR_REFERENCE:-}}"
if [ -z "$R" ]; then
  echo "usage: $0 REFERENCE_ROOT (or set ORATOR_REFERENCE)" >&2
  exit 2
fi
OUT="$HERE/_ref"
if [ ! -f "$R/src/model/asr_text_decoder.cu" ]; then
  echo "reference sources not found under $R; skipping" >&2
  exit 0
fi
mkdir -p "$OUT/obj"
NVCC="${NVCC:-nvcc}"
GEN="-gencode arch=compute_100a,code=sm_100a"
objs=()
for f in src/model/asr_text_decoder.cu src/model/asr_gemm.cu src/model/asr_ops.cu \
         src/pipeline/gpu_vad.cu src/model/asr_audio_tower.cu \
         src/model/conformer_preencode.cu src/model/conformer_layer.cu \
         src/model/sortformer_decoder.cu; do
  o="$OUT/obj/$(basename "$f").o"
  "$NVCC" -std=c++20 -O3 $GEN -Xcompiler -fPIC -I"$R/include" -c "$R/$f" -o "$o"
  objs+=("$o")
done
for f in src/gpu/memory.cc src/gpu/gpu_lock.cc src/io/safetensor.cc \
         src/io/sharded_safetensor.cc src/core/tensor.cc; do
  o="$OUT/obj/$(basename "$f").o"
  g++ -std=c++20 -O2 -fPIC -I"$R/include" -I/usr/local/cuda/include -c "$R/$f" -o "$o"
  objs+=("$o")
done
g++ -std=c++20 -O2 -fPIC -I"$R/include" -I/usr/local/cuda/include \
  -c "$HERE/ref_harness.cc" -o "$OUT/obj/ref_harness.o"
"$NVCC" -shared $GEN -o "$OUT/libref_asr.so" "${objs[@]}" "$OUT/obj/ref_harness.o" -lcudart
# the reference's CPU speech detector (a test utility of the reference)
g++ -std=c++20 -O2 -fPIC -shared -I"$R/include" -I"$R/test/utils" -I/usr/local/cuda/include \
  "$R/test/utils/asr_vad_cpu.cc" "$R/src/io/safetensor.cc" "$R/src/core/tensor.cc" \
  "$R/src/gpu/memory.cc" "$HERE/ref_vad_harness.cc" -L/usr/local/cuda/lib64 -lcudart \
  -o "$OUT/libref_vad_cpu.so"
echo "built $OUT/libref_asr.so $OUT/libref_vad_cpu.so"
