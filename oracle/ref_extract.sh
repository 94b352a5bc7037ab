#!/bin/sh
# Builds oracle/_ref/libref_pins.so: the reference's own self-contained lines for the seeded-key
# expander and the periodic encoder's NTT, compiled where they lie in the reference tree, behind
# the extern "C" shim ref_pins.cpp.  Test infrastructure: it only pins the oracle (tests/golden/
# make_ref_vectors.py writes fixtures from it; tests/test_ref_pins.py compares live when built).
#
#   ref_extract.sh <reference root> <output dir>
#
# The line ranges are the reference's (hpc_gpu_port/seeded_keys.hpp:80-134, ChaCha20, SeedStream,
# fillUniformMod; :195, :302-317, :321-325 and :352-375, the part-file layout, byte I/O and
# header reader; hpc_gpu_port/periodic_encode.hpp:102-120 the scalar helpers, :150-160 the root
# table, :241-260 the NTT).  Each range is checked against its first and last lines, so a changed
# reference stops the build instead of compiling the wrong lines.  The extracted text goes to the
# output directory only (a build product, not part of the repository).
set -eu
REF="$1"
OUT="$2"
SK="$REF/hpc_gpu_port/seeded_keys.hpp"
PE="$REF/hpc_gpu_port/periodic_encode.hpp"
[ -r "$SK" ] && [ -r "$PE" ] || { echo "ref_extract: reference sources not found under $REF" >&2; exit 2; }
mkdir -p "$OUT"

take() {  # file first last first-line-pattern last-line-pattern output
    first=$(sed -n "$2p" "$1")
    last=$(sed -n "$3p" "$1")
    case "$first" in *"$4"*) ;; *) echo "ref_extract: $1:$2 is not '$4'" >&2; exit 3 ;; esac
    case "$last" in *"$5"*) ;; *) echo "ref_extract: $1:$3 is not '$5'" >&2; exit 3 ;; esac
    sed -n "$2,$3p" "$1" > "$6"
}
take "$SK" 80 134 "RFC 8439 ChaCha20 block function" "}" "$OUT/seeded_core.inc"
take "$SK" 195 195 "struct Layout {" "moduli; };" "$OUT/part_layout.inc"
take "$SK" 302 317 "namespace io {" "}  // namespace io" "$OUT/part_io.inc"
take "$SK" 321 325 "inline size_t bytesPerKey" "}" "$OUT/part_sizes.inc"
take "$SK" 352 375 "struct PartHeader {" "}" "$OUT/part_reader.inc"
take "$PE" 102 120 "static uint32_t bitReverse" "}" "$OUT/pe_helpers.inc"
take "$PE" 150 160 "q[l] = ql;" "}" "$OUT/pe_table.inc"
take "$PE" 241 260 "void ntt(uint64_t* a, uint32_t l) const {" "}" "$OUT/pe_ntt.inc"
grep -q "fillUniformMod" "$OUT/seeded_core.inc" && grep -q "class SeedStream" "$OUT/seeded_core.inc" &&
    grep -q "readSeededPartHeader" "$OUT/part_reader.inc" && grep -q "getWords" "$OUT/part_io.inc" &&
    grep -q "mulShoup" "$OUT/pe_helpers.inc" && grep -q "rootShoup\[l\]\[ir\]" "$OUT/pe_table.inc" ||
    { echo "ref_extract: extracted ranges lack their expected contents" >&2; exit 3; }
${CXX:-g++} -O2 -std=c++17 -fPIC -shared -I"$OUT" -o "$OUT/libref_pins.so" "$(dirname "$0")/ref_pins.cpp"
