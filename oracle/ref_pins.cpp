// ref_pins.cpp -- extern "C" entry points over the reference's own code for two pieces of the
// hot path's arithmetic, so the oracle can be compared with the reference word for word:
//   * the seeded-key a-half expander (ChaCha20 block, SeedStream, fillUniformMod:
//     hpc_gpu_port/seeded_keys.hpp:80-134), the normative stream of the key a-halves;
//   * the periodic encoder's NTT and its root table (hpc_gpu_port/periodic_encode.hpp:102-120,
//     :150-160, :241-260), OpenFHE's transform order (natural in, bit-reversed out,
//     Table[brev(i)] = psi^i);
//   * the seeded part-file header reader and byte I/O (hpc_gpu_port/seeded_keys.hpp:195,
//     :302-317, :321-325, :352-375), which any FSSMSKY1 file must satisfy.
// TEST INFRASTRUCTURE ONLY (built by ref_extract.sh into oracle/_ref/, never linked by the engine).
// The included .inc files are the reference's lines, extracted at build time from the reference
// tree; this file supplies only the declarations those lines expect around them.
#include <array>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <istream>
#include <ostream>
#include <string>
#include <vector>

namespace refpins {

// names the extracted lines refer to (declared before them in seeded_keys.hpp:74-78)
using Seed32 = std::array<uint8_t, 32>;
static constexpr char kMagic[8] = {'F', 'S', 'S', 'M', 'S', 'K', 'Y', '1'};
static constexpr uint32_t kVersion = 1;
static constexpr uint32_t kExpander = 1;
static constexpr uint32_t kNonceTag = 0x59454b53u;   // "SKEY" little-endian

#include "seeded_core.inc"
#include "part_layout.inc"
#include "part_io.inc"
#include "part_sizes.inc"
#include "part_reader.inc"

// the members of PeriodicEncoder that its ntt() and root-table lines use, for one tower
struct PeriodicNtt {
    uint32_t Np = 0, REP = 1;
    std::vector<uint64_t> q, psiRep;
    std::vector<std::vector<uint64_t>> rootTab, rootShoup;
#include "pe_helpers.inc"
#include "pe_ntt.inc"
    // root table of tower 0 for modulus ql, ring-N primitive root psi, REP = 2^logRep, N' = N / REP
    void build(uint64_t ql, uint64_t psi, uint32_t logNp) {
        const uint32_t l = 0;
        q.assign(1, 0);
        psiRep.assign(1, 0);
        rootTab.assign(1, {});
        rootShoup.assign(1, {});
#include "pe_table.inc"
    }
};

}  // namespace refpins

extern "C" {

void ref_chacha20_block(const uint32_t key[8], uint32_t counter, const uint32_t nonce[3], uint32_t out[16]) {
    refpins::ChaCha20::block(key, counter, nonce, out);
}

// a-half words of (seed, digit, limb) for modulus q: the expander of seeded_keys.hpp
void ref_expand_a(const uint8_t seed[32], uint32_t digit, uint32_t limb, uint64_t q, uint64_t* out, size_t n) {
    refpins::Seed32 s;
    std::memcpy(s.data(), seed, 32);
    refpins::SeedStream ss(s, digit, limb);
    refpins::fillUniformMod(ss, q, out, n);
}

// the periodic encoder's forward NTT at ring N' = 2^(logN - logRep) with root psi^(2^logRep), psi a
// primitive 2^(logN+1)-th root mod q; a: N' words, transformed in place
void ref_periodic_ntt(uint64_t q, uint64_t psi, uint32_t logN, uint32_t logRep, uint64_t* a) {
    refpins::PeriodicNtt t;
    t.REP = 1u << logRep;
    t.Np = 1u << (logN - logRep);
    t.build(q, psi, logN - logRep);
    t.ntt(a, 0);
}

// a part file read by the reference's own header reader and byte I/O: head = {version, expander,
// N, sizeQ, sizeP, numPartQ, numPerPartQ, count}, the moduli, the tag, then every record's index,
// seed and its first `nb` b-words; returns 0, or 1 with the reader's message in err
int ref_read_part(const char* path, uint32_t head[8], uint64_t* moduli, char* tag, int tag_cap, uint32_t* indices,
                  uint8_t* seeds, uint64_t* bhead, int nb, char* err, int err_cap) {
    std::ifstream is(path, std::ios::binary);
    refpins::PartHeader H;
    std::string e;
    auto fail = [&](const std::string& m) {
        std::snprintf(err, err_cap, "%s", m.c_str());
        return 1;
    };
    if (!refpins::readSeededPartHeader(is, H, &e)) return fail(e);
    const uint32_t h[8] = {H.version, H.expander, H.L.N, H.L.sizeQ, H.L.sizeP, H.L.numPartQ, H.L.numPerPartQ, H.count};
    std::memcpy(head, h, sizeof h);
    std::memcpy(moduli, H.L.moduli.data(), H.L.moduli.size() * 8);
    std::snprintf(tag, tag_cap, "%s", H.keyTag.c_str());
    const size_t words = (refpins::bytesPerKey(H.L) - 36) / 8;
    std::vector<uint64_t> bw;
    for (uint32_t k = 0; k < H.count; k++) {
        if (!refpins::io::get32(is, indices[k]) || !is.read((char*)seeds + 32 * (size_t)k, 32) ||
            !refpins::io::getWords(is, bw, words))
            return fail("short key record");
        std::memcpy(bhead + (size_t)k * nb, bw.data(), (size_t)nb * 8);
    }
    return 0;
}

}  // extern "C"
