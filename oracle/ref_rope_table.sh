#!/usr/bin/env bash
# Compiles the reference's own BF16 RoPE-table code (bf16_rne_to_f32 and
# make_bf16_rope_table, src/higgs_pipeline.cpp:471-487) from its source into
# oracle/_ref/libref_rope.so, so the oracle's and the engine's tables can be
# compared with the reference's bit for bit.
#
# The rest of higgs_pipeline.cpp needs the absent ggml submodule, so only
# these two functions are compiled: they are cut from the reference file by
# their signatures (not by line numbers) into oracle/_ref/ (git-ignored, never
# committed), next to a shim for the two ggml bf16 conversions they call
# (upstream ggml's published round-to-nearest-even conversion) and the
# reference's own include/higgs_audio.h for TextConfig.
#
# Usage: oracle/ref_rope_table.sh <reference checkout>   (or HKV_REFERENCE=<checkout>)
# There is no default location: without one the script says so and exits 2.
set -euo pipefail
REF=${1:-${HKV_REFERENCE:-}}
[ -n "$REF" ] || { echo "no reference checkout given (argument or HKV_REFERENCE)" >&2; exit 2; }
HERE="$(cd "$(dirname "$0")" && pwd)"
OUT="$HERE/_ref"
SRC="$REF/src/higgs_pipeline.cpp"
[ -f "$SRC" ] || { echo "reference source not found at $SRC" >&2; exit 2; }
mkdir -p "$OUT"
# From `float bf16_rne_to_f32(` through the closing brace of make_bf16_rope_table.
awk '
  /^float bf16_rne_to_f32\(float value\) \{/ { on = 1 }
  on { print }
  on && /^std::vector<float> make_bf16_rope_table\(/ { in_table = 1 }
  in_table && /^}/ { exit }
' "$SRC" > "$OUT/ref_rope_extract.inc"
grep -q "make_bf16_rope_table" "$OUT/ref_rope_extract.inc" || { echo "extraction failed" >&2; exit 3; }
cat > "$OUT/ref_rope_table.cpp" <<'CPP'
#include "higgs_audio.h"
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
namespace higgs_audio {
struct ggml_bf16_t { uint16_t bits; };
static inline ggml_bf16_t ggml_fp32_to_bf16(float s) {
    uint32_t u; std::memcpy(&u, &s, 4);
    ggml_bf16_t h;
    if ((u & 0x7fffffffu) > 0x7f800000u) { h.bits = (uint16_t)((u >> 16) | 64u); return h; }
    h.bits = (uint16_t)((u + (0x7fffu + ((u >> 16) & 1u))) >> 16);
    return h;
}
static inline float ggml_bf16_to_fp32(ggml_bf16_t h) {
    uint32_t u = (uint32_t)h.bits << 16; float f; std::memcpy(&f, &u, 4); return f;
}
#include "ref_rope_extract.inc"
}  // namespace higgs_audio
extern "C" void ref_rope_table(int64_t context_length, int64_t key_length, float base,
                               float *cos_out, float *sin_out) {
    higgs_audio::TextConfig cfg;
    cfg.context_length = context_length;
    cfg.key_length = key_length;
    cfg.rope_freq_base = base;
    const std::vector<float> c = higgs_audio::make_bf16_rope_table(cfg, false);
    const std::vector<float> s = higgs_audio::make_bf16_rope_table(cfg, true);
    std::memcpy(cos_out, c.data(), c.size() * sizeof(float));
    std::memcpy(sin_out, s.data(), s.size() * sizeof(float));
}
CPP
g++ -O2 -std=c++17 -fPIC -shared -ffp-contract=off -I"$REF/include" -I"$OUT" \
    "$OUT/ref_rope_table.cpp" -o "$OUT/libref_rope.so"
echo "$OUT/libref_rope.so"
