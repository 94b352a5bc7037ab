// sampling.h -- deterministic samplers for keys and encryption randomness (host side).
//
// Every random polynomial is drawn from a ChaCha20 (RFC 8439) keystream; the seed expander
// for key a-halves follows the reference's normative spec (hpc_gpu_port/seeded_keys.hpp:
// 36-49): key = 32-byte seed as 8 LE words, nonce = {n0, n1, tag}, counter 0,1,2,..., the
// 16 output words read as LE uint64 pairs, rejection w >= 2^64 - (2^64 mod q).
// The other samplers use the same stream with their own tags:
//   "SECR": sparse ternary with exactly h nonzeros (position u & (N-1), sign = bit 63)
//   "TERN": uniform ternary (u mod 3) - 1
//   "GAUS": rounded Gaussian by a cumulative table over |x| <= ceil(6 sigma)
//   "SEED": per-object 32-byte seeds derived from a master seed (first 8 words of block 0)
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

namespace fhe {

enum : uint32_t {
    kTagSKEY = 0x59454b53u, kTagGAUS = 0x53554147u, kTagSECR = 0x52434553u,
    kTagTERN = 0x4e524554u, kTagSEED = 0x44454553u, kTagPKEY = 0x59454b50u,
};
// seed identifiers under the master seed
enum : uint32_t { kSeedPublic = 0xFFFFFFF0u, kSeedSecret = 0xFFFFFFF1u, kSeedEncrypt = 0xFFFFFFF2u };

struct ChaChaStream {
    uint32_t key[8], nonce[3], w[16], counter = 0;
    int pos = 8;
    static inline uint32_t rotl(uint32_t v, int c) { return (v << c) | (v >> (32 - c)); }
    static void block(const uint32_t k[8], uint32_t ctr, const uint32_t n[3], uint32_t out[16]) {
        const uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u, k[0], k[1], k[2], k[3],
                                k[4], k[5], k[6], k[7], ctr, n[0], n[1], n[2]};
        uint32_t x[16];
        for (int i = 0; i < 16; i++) x[i] = s[i];
        auto qr = [](uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
            a += b; d ^= a; d = rotl(d, 16);
            c += d; b ^= c; b = rotl(b, 12);
            a += b; d ^= a; d = rotl(d, 8);
            c += d; b ^= c; b = rotl(b, 7);
        };
        for (int r = 0; r < 10; r++) {
            qr(x[0], x[4], x[8], x[12]); qr(x[1], x[5], x[9], x[13]);
            qr(x[2], x[6], x[10], x[14]); qr(x[3], x[7], x[11], x[15]);
            qr(x[0], x[5], x[10], x[15]); qr(x[1], x[6], x[11], x[12]);
            qr(x[2], x[7], x[8], x[13]); qr(x[3], x[4], x[9], x[14]);
        }
        for (int i = 0; i < 16; i++) out[i] = x[i] + s[i];
    }
    ChaChaStream(const uint8_t seed[32], uint32_t n0, uint32_t n1, uint32_t tag) {
        for (int k = 0; k < 8; k++)
            key[k] = (uint32_t)seed[4 * k] | ((uint32_t)seed[4 * k + 1] << 8) | ((uint32_t)seed[4 * k + 2] << 16) |
                     ((uint32_t)seed[4 * k + 3] << 24);
        nonce[0] = n0; nonce[1] = n1; nonce[2] = tag;
    }
    uint64_t next() {
        if (pos == 8) { block(key, counter++, nonce, w); pos = 0; }
        const uint64_t v = (uint64_t)w[2 * pos] | ((uint64_t)w[2 * pos + 1] << 32);
        pos++;
        return v;
    }
};

inline void derive_seed(const uint8_t master[32], uint32_t id, uint32_t sub, uint8_t out[32]) {
    ChaChaStream s(master, id, sub, kTagSEED);
    uint32_t w[16];
    ChaChaStream::block(s.key, 0, s.nonce, w);
    for (int k = 0; k < 8; k++)
        for (int b = 0; b < 4; b++) out[4 * k + b] = (uint8_t)(w[k] >> (8 * b));
}

inline void sample_uniform(const uint8_t seed[32], uint32_t n0, uint32_t n1, uint32_t tag, uint64_t q, uint64_t* out,
                           size_t n) {
    ChaChaStream s(seed, n0, n1, tag);
    const uint64_t r = (0 - q) % q, lim = 0 - r;
    for (size_t k = 0; k < n; k++) {
        uint64_t w = s.next();
        while (r != 0 && w >= lim) w = s.next();
        out[k] = w % q;
    }
}

inline void sample_ternary_hw(const uint8_t seed[32], uint32_t n0, uint32_t n1, int h, int8_t* out, int n) {
    ChaChaStream s(seed, n0, n1, kTagSECR);
    std::memset(out, 0, (size_t)n);
    int placed = 0;
    while (placed < h && placed < n) {
        const uint64_t u = s.next();
        const uint32_t pos = (uint32_t)(u & (uint64_t)(n - 1));
        if (out[pos]) continue;
        out[pos] = (u >> 63) ? -1 : 1;
        placed++;
    }
}

inline void sample_ternary(const uint8_t seed[32], uint32_t n0, uint32_t n1, int8_t* out, int n) {
    ChaChaStream s(seed, n0, n1, kTagTERN);
    for (int k = 0; k < n; k++) out[k] = (int8_t)((int)(s.next() % 3) - 1);
}

inline void sample_gauss(const uint8_t seed[32], uint32_t n0, uint32_t n1, double sigma, int64_t* out, int n) {
    int B = (int)std::ceil(6.0 * sigma);
    if (B > 63) B = 63;
    double w[64], tot = 0.0, cum = 0.0;
    uint64_t T[64];
    for (int x = 0; x <= B; x++) {
        w[x] = (x == 0 ? 1.0 : 2.0) * std::exp(-(double)x * x / (2.0 * sigma * sigma));
        tot += w[x];
    }
    for (int x = 0; x < B; x++) {
        cum += w[x];
        T[x] = (uint64_t)(cum / tot * 9223372036854775808.0);
    }
    T[B] = 0x8000000000000000ull;
    ChaChaStream s(seed, n0, n1, kTagGAUS);
    for (int k = 0; k < n; k++) {
        const uint64_t u = s.next();
        const uint64_t r = u >> 1;
        int mag = 0;
        while (mag < B && r >= T[mag]) mag++;
        out[k] = (u & 1) ? -mag : mag;
    }
}

}  // namespace fhe
