#!/bin/sh
# Extracts the host-compilable part of trench-gguf's gpuq/gpuq.hip (its per-block quantizers, dequantizers and the
# source decoder: everything but the HIP/CUDA runtime host code) into oracle/_ref/, where ref_host.cpp includes it.
# The reference sources are read where they lie; nothing of them is copied into the repository.
#   extract_ref.sh <gpuq.hip> <out.inc>
set -e
SRC=$1; OUT=$2
[ -f "$SRC" ] || { echo "extract_ref.sh: $SRC not found" >&2; exit 2; }
awk '
  /^#include <cstdint>/ { on = 1 }
  /^namespace \{/       { ns++; on = 0 }
  /^enum \{ S_F32/      { on = 1 }
  on { print }
' "$SRC" > "$OUT.tmp"
# sanity: the pieces ref_host.cpp calls must be there
for sym in q_iq2_xxs q_iq1_s q_iq1_m q_iq2_s q_iq2_xs q_iq3_xxs q_iq3_s q_iq4_xs q_iq4_nl q_q2_k q_q3_k q_q4_k \
           q_q5_k q_q6_k q_q8_0 dq_iq2_xxs dq_iq4_xs "void kq" "void kdqq" "void kdq" fp16_to_fp32; do
  grep -q "$sym" "$OUT.tmp" || { echo "extract_ref.sh: '$sym' missing from the extract" >&2; exit 3; }
done
mv "$OUT.tmp" "$OUT"
