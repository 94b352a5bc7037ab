// modarith.cuh -- 64-bit modular arithmetic for RNS limbs (moduli < 2^61).
//
// All helpers return canonical residues in [0, q) unless the name says "lazy".
//  * mul_shoup:   x * w mod q for a constant w with w' = floor(w * 2^64 / q) (Shoup).
//  * mul_barrett: a * b mod q for variable a, b < q (Barrett, HAC 14.42 with base 2,
//                 mu = floor(2^(2k) / q), k = bit length of q).
//  * redc:        Montgomery reduction of a 128-bit T < q * 2^64 (R = 2^64); used for the
//                 key inner product whose key words are stored multiplied by R.
#pragma once
#include <cstdint>

struct ModConst {
    uint64_t q;       // modulus
    uint64_t mu;      // floor(2^(2k) / q)
    uint64_t qinv;    // -q^-1 mod 2^64 (Montgomery)
    uint64_t r2;      // 2^128 mod q (to enter the Montgomery domain)
    uint32_t k;       // bit length of q
    uint32_t pad;
};

__host__ __device__ __forceinline__ uint64_t mod_add(uint64_t a, uint64_t b, uint64_t q) {
    uint64_t s = a + b;
    return s >= q ? s - q : s;
}
__host__ __device__ __forceinline__ uint64_t mod_sub(uint64_t a, uint64_t b, uint64_t q) {
    return a >= b ? a - b : a + q - b;
}
__host__ __device__ __forceinline__ uint64_t mod_neg(uint64_t a, uint64_t q) { return a ? q - a : 0; }

__device__ __forceinline__ uint64_t mul_shoup_lazy(uint64_t x, uint64_t w, uint64_t wp, uint64_t q) {
    const uint64_t hi = __umul64hi(x, wp);
    return x * w - hi * q;  // in [0, 2q)
}
__device__ __forceinline__ uint64_t mul_shoup(uint64_t x, uint64_t w, uint64_t wp, uint64_t q) {
    uint64_t r = mul_shoup_lazy(x, w, wp, q);
    return r >= q ? r - q : r;
}

// Barrett reduction of x = hi:lo < 2^(2k) (in particular any product of two residues).
__device__ __forceinline__ uint64_t barrett128(uint64_t hi, uint64_t lo, const ModConst& m) {
    const uint32_t k = m.k;
    const uint64_t x1 = (hi << (65 - k)) | (lo >> (k - 1));      // x >> (k-1)
    const uint64_t ph = __umul64hi(x1, m.mu), pl = x1 * m.mu;
    const uint64_t q3 = (ph << (63 - k)) | (pl >> (k + 1));      // (x1 * mu) >> (k+1)
    uint64_t r = lo - q3 * m.q;                                   // exact: r < 3q < 2^64
    if (r >= m.q) r -= m.q;
    if (r >= m.q) r -= m.q;
    return r;
}
// s < 16q (a sum of up to eight lazy Shoup products) -> [0, q); needs 16q < 2^64
__device__ __forceinline__ uint64_t reduce_lazy16(uint64_t s, uint64_t q) {
    if (s >= (q << 3)) s -= (q << 3);
    if (s >= (q << 2)) s -= (q << 2);
    if (s >= (q << 1)) s -= (q << 1);
    return s >= q ? s - q : s;
}
// any 64-bit value mod q (valid for q >= 2^32: 64 <= 2k)
__device__ __forceinline__ uint64_t reduce64(uint64_t v, const ModConst& m) { return barrett128(0, v, m); }
__device__ __forceinline__ uint64_t mul_barrett(uint64_t a, uint64_t b, const ModConst& m) {
    return barrett128(__umul64hi(a, b), a * b, m);
}

// 128-bit accumulator helpers
struct u128acc {
    uint64_t lo, hi;
};
__device__ __forceinline__ void acc_mad(u128acc& acc, uint64_t a, uint64_t b) {
    const uint64_t pl = a * b, ph = __umul64hi(a, b);
    asm("add.cc.u64 %0, %0, %2;\n\taddc.u64 %1, %1, %3;" : "+l"(acc.lo), "+l"(acc.hi) : "l"(pl), "l"(ph));
}
// The same sum, column by column in 32-bit words with three carry chains: the products a0 b0 and
// a1 b1 land in their own columns in one chain, the two cross products in one chain each (ten
// multiply-adds and carry adds).  Fewer instructions than acc_mad, but it keeps more registers
// live: it pays in the kernels with few loads in flight (the base conversion, the bootstrap's
// diagonal sums) and costs occupancy in the key inner products, which keep acc_mad.
__device__ __forceinline__ void acc_mad32(u128acc& acc, uint64_t a, uint64_t b) {
    asm("{\n\t"
        ".reg .u32 a0, a1, b0, b1, s0, s1, s2, s3;\n\t"
        "mov.b64 {a0, a1}, %2;\n\t"
        "mov.b64 {b0, b1}, %3;\n\t"
        "mov.b64 {s0, s1}, %0;\n\t"
        "mov.b64 {s2, s3}, %1;\n\t"
        "mad.lo.cc.u32 s0, a0, b0, s0;\n\t"
        "madc.hi.cc.u32 s1, a0, b0, s1;\n\t"
        "madc.lo.cc.u32 s2, a1, b1, s2;\n\t"
        "madc.hi.u32 s3, a1, b1, s3;\n\t"
        "mad.lo.cc.u32 s1, a0, b1, s1;\n\t"
        "madc.hi.cc.u32 s2, a0, b1, s2;\n\t"
        "addc.u32 s3, s3, 0;\n\t"
        "mad.lo.cc.u32 s1, a1, b0, s1;\n\t"
        "madc.hi.cc.u32 s2, a1, b0, s2;\n\t"
        "addc.u32 s3, s3, 0;\n\t"
        "mov.b64 %0, {s0, s1};\n\t"
        "mov.b64 %1, {s2, s3};\n\t"
        "}"
        : "+l"(acc.lo), "+l"(acc.hi)
        : "l"(a), "l"(b));
}
// Montgomery: returns T * 2^-64 mod q for T = hi:lo < q * 2^64, canonical.
__device__ __forceinline__ uint64_t redc(uint64_t hi, uint64_t lo, const ModConst& m) {
    const uint64_t mq = lo * m.qinv;                 // m = T * (-q^-1) mod 2^64
    const uint64_t mh = __umul64hi(mq, m.q);         // (m q) >> 64; low half cancels T's low half
    // (T + m q) / 2^64 = hi + mh + carry(lo + mq*q low)
    const uint64_t carry = lo != 0 ? 1 : 0;          // lo + (mq*q mod 2^64) == 0 mod 2^64 exactly
    uint64_t r = hi + mh + carry;
    return r >= m.q ? r - m.q : r;
}

// host-side constant construction
inline ModConst make_modconst(uint64_t q) {
    ModConst m{};
    m.q = q;
    uint32_t k = 0;
    while (k < 64 && (q >> k)) k++;
    m.k = k;
    // mu = floor(2^(2k) / q) via long division on 128-bit
    unsigned __int128 num = (unsigned __int128)1 << (2 * k);
    m.mu = (uint64_t)(num / q);
    // -q^-1 mod 2^64 by Newton iteration
    uint64_t inv = q;  // q * q = 1 mod 8 for odd q
    for (int i = 0; i < 6; i++) inv *= 2 - q * inv;
    m.qinv = (uint64_t)(0 - inv);
    unsigned __int128 r = ((unsigned __int128)1 << 64) % q;
    m.r2 = (uint64_t)((r * r) % q);
    return m;
}

inline uint64_t host_mulmod(uint64_t a, uint64_t b, uint64_t q) { return (uint64_t)(((unsigned __int128)a * b) % q); }
inline uint64_t host_powmod(uint64_t a, uint64_t e, uint64_t q) {
    uint64_t r = 1 % q;
    a %= q;
    while (e) {
        if (e & 1) r = host_mulmod(r, a, q);
        a = host_mulmod(a, a, q);
        e >>= 1;
    }
    return r;
}
inline uint64_t host_invmod(uint64_t a, uint64_t q) { return host_powmod(a, q - 2, q); }
inline uint64_t shoup_of(uint64_t w, uint64_t q) { return (uint64_t)(((unsigned __int128)w << 64) / q); }
inline uint64_t mont_of(uint64_t w, uint64_t q) { return (uint64_t)(((unsigned __int128)w << 64) % q); }   // w 2^64 mod q
