#!/usr/bin/env bash
# Builds oracle/_ref/libref.so from the reference's own C++ sources (test
# infrastructure: the result is a checker, never part of the product).
#
#   server/paged_attention.cpp, server/speculative_decoder.cpp,
#   server/mtp_heads.cpp, server/chunked_prefill.cpp
#                                        compiled in place, unmodified;
#   server/radix_kv_cache.cpp            compiled in place, unmodified, with
#                                        <functional> force-included;
#   server/paged_kv_cache.cpp            compiled unmodified from a scratch copy
#                                        under oracle/_ref/src whose header has
#                                        the one-word shim the reference needs
#                                        to compile (`mutable` on cache_mutex,
#                                        required by get_utilization() const);
#   oracle/ref_shim.cpp + oracle C files provide the Rust kernel symbols those
#                                        files call (C restatements of lib.rs).
#
# Outputs only into oracle/_ref/ (git-ignored).  Needs the reference tree at
# $SME_LLM_EDGE_REF (default: a directory named "reference" beside the
# repository root); without it the script exits 0 and leaves any previously
# built library in place.
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
REF="${SME_LLM_EDGE_REF:-$(cd "$HERE/../.." && pwd)/reference}"
OUT="$HERE/_ref"
if [ ! -d "$REF/server" ]; then
  echo "build_ref: reference tree not found at $REF; skipping" >&2
  exit 0
fi
CXX=/usr/bin/g++
CC=/usr/bin/gcc
mkdir -p "$OUT/src" "$OUT/obj"
cp "$REF/server/paged_kv_cache.cpp" "$OUT/src/paged_kv_cache.cpp"
sed 's/^\(\s*\)std::mutex cache_mutex;/\1mutable std::mutex cache_mutex;/' "$REF/server/paged_kv_cache.h" > "$OUT/src/paged_kv_cache.h"
grep -q "mutable std::mutex cache_mutex" "$OUT/src/paged_kv_cache.h"

CXXFLAGS="-std=c++20 -O2 -fPIC -fopenmp -ffp-contract=off -w"
CFLAGS="-O2 -fPIC -fopenmp -ffp-contract=off -std=gnu11 -w"
$CXX $CXXFLAGS -c "$REF/server/paged_attention.cpp" -o "$OUT/obj/paged_attention.o"
$CXX $CXXFLAGS -c "$REF/server/speculative_decoder.cpp" -o "$OUT/obj/speculative_decoder.o"
$CXX $CXXFLAGS -c "$REF/server/mtp_heads.cpp" -o "$OUT/obj/mtp_heads.o"
$CXX $CXXFLAGS -c "$REF/server/chunked_prefill.cpp" -o "$OUT/obj/chunked_prefill.o"
$CXX $CXXFLAGS -c "$OUT/src/paged_kv_cache.cpp" -o "$OUT/obj/paged_kv_cache.o"
# radix_kv_cache.cpp uses std::function without including <functional>; the
# header is supplied on the command line (-include), the source is unmodified
$CXX $CXXFLAGS -include functional -c "$REF/server/radix_kv_cache.cpp" -o "$OUT/obj/radix_kv_cache.o"
$CXX $CXXFLAGS -I"$OUT/src" -I"$REF/server" -I"$HERE" -c "$HERE/ref_shim.cpp" -o "$OUT/obj/ref_shim.o"
for f in orc_sample orc_model orc_kv; do
  $CC $CFLAGS -c "$HERE/$f.c" -o "$OUT/obj/$f.o"
done
$CXX -shared -fopenmp -o "$OUT/libref.so" "$OUT"/obj/*.o -lm
echo "build_ref: built $OUT/libref.so"

# The reference's callers linked against the CUDA library instead of the Rust
# kernels: server/speculative_decoder.cpp, server/mtp_heads.cpp,
# server/paged_kv_cache.cpp (scratch copy above) and
# server/flash_decoding_tracker.cpp, unmodified, plus oracle/ref_callers.cpp.
# --no-undefined: every kernel symbol they call must come from
# libspecdec_sm100.so (found at run time through the rpath, relative to
# oracle/_ref/).
SPECDEC_DIR="$(cd "$HERE/.." && pwd)/sme-llm-edge_b200/specdec"
if [ -f "$SPECDEC_DIR/libspecdec_sm100.so" ]; then
  mkdir -p "$OUT/obj_callers"
  $CXX $CXXFLAGS -c "$REF/server/flash_decoding_tracker.cpp" -o "$OUT/obj_callers/flash_decoding_tracker.o"
  $CXX $CXXFLAGS -I"$REF/server" -c "$HERE/ref_callers.cpp" -o "$OUT/obj_callers/ref_callers.o"
  $CXX -shared -o "$OUT/libref_callers.so" "$OUT/obj_callers/ref_callers.o" "$OUT/obj_callers/flash_decoding_tracker.o" \
    "$OUT/obj/speculative_decoder.o" "$OUT/obj/mtp_heads.o" "$OUT/obj/paged_kv_cache.o" \
    -L"$SPECDEC_DIR" -lspecdec_sm100 -Wl,-rpath,'$ORIGIN/../../sme-llm-edge_b200/specdec' -Wl,--no-undefined -ldl
  echo "build_ref: built $OUT/libref_callers.so (reference callers -> libspecdec_sm100.so)"
fi
