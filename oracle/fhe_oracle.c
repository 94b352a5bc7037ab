/*
 * fhe_oracle.c -- CPU restatement of the CKKS/RNS arithmetic on the fhe-ssm hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker; see fhe_oracle.h).  Parity against OpenFHE:
 * unpinned (OpenFHE v1.5.1 and FIDESlib are third-party, absent from the reference tree).
 *
 * Conventions restated from the reference's own sources:
 *   - NTT order: natural-order coefficients in, bit-reversed evaluations out, root table
 *     Table[brev(i)] = psi^i (hpc_gpu_port/periodic_encode.hpp:141-161, :240-260).
 *   - Encode rounding: scale, llround, MAX_BITS 61 approx factor, negative -> q - |c|
 *     (hpc_gpu_port/periodic_encode.hpp:186-237).
 *   - Rotation index 5^s mod 2N, conjugation 2N-1 (hpc_gpu_port/gpu_real_model.cu:1355-1369).
 *   - Hybrid key structure: numPartQ digits over QP, a_j uniform in EVAL form from the seed
 *     expander, b_j = -a_j * tau_{k^-1}(s) + e_j + [P]_{q_i} * s_i on the digit's limbs
 *     (hpc_gpu_port/seeded_keys.hpp:36-49, :139-195, :216-221).
 *   - ChaCha20 expander with rejection sampling (hpc_gpu_port/seeded_keys.hpp:36-49).
 * Everything else (ModUp/ModDown base conversion, rescale by the last limb) is the
 * textbook RNS-CKKS algorithm (Cheon-Han-Kim-Kim-Song 2018; Han-Ki 2020 hybrid key
 * switching) written from the mathematics.
 */
#include "fhe_oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

typedef unsigned __int128 u128;

#define TAG_SKEY 0x59454b53u /* "SKEY" */
#define TAG_GAUS 0x53554147u /* "GAUS" */
#define TAG_SECR 0x52434553u /* "SECR" */
#define TAG_TERN 0x4e524554u /* "TERN" */
#define TAG_SEED 0x44454553u /* "SEED" */

/* ================================ scalar arithmetic ================================ */
uint64_t oc_mulmod(uint64_t a, uint64_t b, uint64_t q) { return (uint64_t)(((u128)a * b) % q); }
static inline uint64_t addm(uint64_t a, uint64_t b, uint64_t q) { uint64_t s = a + b; return s >= q ? s - q : s; }
static inline uint64_t subm(uint64_t a, uint64_t b, uint64_t q) { return a >= b ? a - b : a + q - b; }
uint64_t oc_powmod(uint64_t a, uint64_t e, uint64_t q) {
    uint64_t r = 1 % q;
    a %= q;
    while (e) {
        if (e & 1) r = oc_mulmod(r, a, q);
        a = oc_mulmod(a, a, q);
        e >>= 1;
    }
    return r;
}
uint64_t oc_invmod(uint64_t a, uint64_t q) { return oc_powmod(a, q - 2, q); } /* q prime */

int oc_is_prime(uint64_t n) {
    static const uint64_t bases[] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37};
    if (n < 2) return 0;
    for (int i = 0; i < 12; i++) {
        if (n == bases[i]) return 1;
        if (n % bases[i] == 0) return 0;
    }
    uint64_t d = n - 1;
    int s = 0;
    while ((d & 1) == 0) { d >>= 1; s++; }
    for (int i = 0; i < 12; i++) {
        uint64_t x = oc_powmod(bases[i], d, n);
        if (x == 1 || x == n - 1) continue;
        int comp = 1;
        for (int r = 1; r < s; r++) {
            x = oc_mulmod(x, x, n);
            if (x == n - 1) { comp = 0; break; }
        }
        if (comp) return 0;
    }
    return 1;
}

/* ================================ moduli chain ===================================== */
static uint64_t first_prime(int bits, uint64_t M) {
    uint64_t x = 1ull << bits;
    uint64_t q = x - (x % M) + 1;
    if (q <= x) q += M;
    while (!oc_is_prime(q)) q += M;
    return q;
}
static uint64_t prev_prime(uint64_t q, uint64_t M) {
    do { q -= M; } while (!oc_is_prime(q));
    return q;
}
static uint64_t next_prime(uint64_t q, uint64_t M) {
    do { q += M; } while (!oc_is_prime(q));
    return q;
}
static int in_list(uint64_t v, const uint64_t* a, int n) {
    for (int i = 0; i < n; i++) if (a[i] == v) return 1;
    return 0;
}

int oc_gen_chain(int logN, int L, int q0bits, int qbits, int K, int pbits, uint64_t* q, uint64_t* p) {
    const uint64_t M = 2ull << logN;
    if (L < 1 || q0bits > 61 || qbits > 61 || pbits > 61) return -1;
    if (L > 1) {
        uint64_t qs = first_prime(qbits, M), qPrev = qs, qNext = qs;
        q[L - 1] = qs;
        int cnt = 0;
        for (int i = L - 2; i >= 1; i--) {
            if (cnt % 2 == 0) { qPrev = prev_prime(qPrev, M); q[i] = qPrev; }
            else { qNext = next_prime(qNext, M); q[i] = qNext; }
            cnt++;
        }
    }
    uint64_t q0 = prev_prime(first_prime(q0bits, M), M);
    while (L > 1 && in_list(q0, q + 1, L - 1)) q0 = prev_prime(q0, M);
    q[0] = q0;
    uint64_t pp = first_prime(pbits, M);
    for (int k = 0; k < K; k++) {
        pp = prev_prime(pp, M);
        while (in_list(pp, q, L) || in_list(pp, p, k)) pp = prev_prime(pp, M);
        p[k] = pp;
    }
    return 0;
}

uint64_t oc_min_root(uint64_t q, int logN) {
    const uint64_t N = 1ull << logN, M = 2 * N;
    uint64_t psi = 0;
    for (uint64_t x = 2; x < q; x++) {
        uint64_t g = oc_powmod(x, (q - 1) / M, q);
        if (oc_powmod(g, N, q) == q - 1) { psi = g; break; }
    }
    /* all primitive 2N-th roots are psi^j, j odd: take the smallest */
    uint64_t best = psi, sq = oc_mulmod(psi, psi, q), cur = psi;
    for (uint64_t j = 1; j < M; j += 2) {
        if (cur < best) best = cur;
        cur = oc_mulmod(cur, sq, q);
    }
    return best;
}

/* ================================ context ========================================== */
struct oc_ctx {
    int logN, N, nq, np, alpha;
    uint64_t* mod;  /* nq + np */
    uint64_t* psi;
    uint64_t** tab;  /* tab[m][brev(i)] = psi^i */
    uint64_t** itab; /* itab[m][brev(i)] = psi^-i */
};

static uint32_t brev(uint32_t v, int bits) {
    uint32_t r = 0;
    for (int b = 0; b < bits; b++) { r = (r << 1) | (v & 1u); v >>= 1; }
    return r;
}

oc_ctx* oc_ctx_new(int logN, int nq, const uint64_t* q, int np, const uint64_t* p, int alpha) {
    oc_ctx* c = (oc_ctx*)calloc(1, sizeof(oc_ctx));
    c->logN = logN; c->N = 1 << logN; c->nq = nq; c->np = np; c->alpha = alpha;
    int nm = nq + np;
    c->mod = (uint64_t*)malloc(sizeof(uint64_t) * nm);
    c->psi = (uint64_t*)malloc(sizeof(uint64_t) * nm);
    c->tab = (uint64_t**)malloc(sizeof(uint64_t*) * nm);
    c->itab = (uint64_t**)malloc(sizeof(uint64_t*) * nm);
    for (int m = 0; m < nm; m++) {
        uint64_t mm = m < nq ? q[m] : p[m - nq];
        c->mod[m] = mm;
        c->psi[m] = oc_min_root(mm, logN);
        c->tab[m] = (uint64_t*)malloc(sizeof(uint64_t) * c->N);
        c->itab[m] = (uint64_t*)malloc(sizeof(uint64_t) * c->N);
        uint64_t x = 1, xi = 1, pinv = oc_invmod(c->psi[m], mm);
        for (int i = 0; i < c->N; i++) {
            uint32_t r = brev((uint32_t)i, logN);
            c->tab[m][r] = x;
            c->itab[m][r] = xi;
            x = oc_mulmod(x, c->psi[m], mm);
            xi = oc_mulmod(xi, pinv, mm);
        }
    }
    return c;
}

void oc_ctx_free(oc_ctx* c) {
    if (!c) return;
    for (int m = 0; m < c->nq + c->np; m++) { free(c->tab[m]); free(c->itab[m]); }
    free(c->tab); free(c->itab); free(c->mod); free(c->psi); free(c);
}
uint64_t oc_modulus(const oc_ctx* c, int m) { return c->mod[m]; }
uint64_t oc_root(const oc_ctx* c, int m) { return c->psi[m]; }

/* ================================ NTT ============================================== */
/* Cooley-Tukey, natural in -> bit-reversed out (periodic_encode.hpp:241-260 loop shape). */
static void ntt_ct(uint64_t q, const uint64_t* tab, int n, uint64_t* a) {
    for (int mm = 1, t = n >> 1; mm < n; mm <<= 1, t >>= 1) {
        for (int i = 0; i < mm; i++) {
            const int j1 = i * 2 * t;
            const uint64_t w = tab[mm + i];
            for (int j = j1; j < j1 + t; j++) {
                uint64_t x = oc_mulmod(a[j + t], w, q);
                uint64_t u = a[j];
                a[j] = addm(u, x, q);
                a[j + t] = subm(u, x, q);
            }
        }
    }
}
void oc_ntt(const oc_ctx* c, uint64_t* a, int m) { ntt_ct(c->mod[m], c->tab[m], c->N, a); }
/* The same transform at ring 2^logN with an explicit primitive 2^(logN+1)-th root psi: the
 * table Tab[brev(i)] = psi^i is built as the context builds its own (the periodic encoder's
 * small-ring transform, periodic_encode.hpp:150-160, takes psi' = psi^REP). */
void oc_ntt_root(int logN, uint64_t q, uint64_t psi, uint64_t* a) {
    const int n = 1 << logN;
    uint64_t* tab = (uint64_t*)malloc(sizeof(uint64_t) * n);
    uint64_t x = 1;
    for (int i = 0; i < n; i++) {
        tab[brev((uint32_t)i, logN)] = x;
        x = oc_mulmod(x, psi, q);
    }
    ntt_ct(q, tab, n, a);
    free(tab);
}
/* Gentleman-Sande, bit-reversed in -> natural out, then * N^-1. */
void oc_intt(const oc_ctx* c, uint64_t* a, int m) {
    const uint64_t q = c->mod[m];
    const uint64_t* itab = c->itab[m];
    const int n = c->N;
    for (int mm = n >> 1, t = 1; mm >= 1; mm >>= 1, t <<= 1) {
        for (int i = 0; i < mm; i++) {
            const int j1 = i * 2 * t;
            const uint64_t w = itab[mm + i];
            for (int j = j1; j < j1 + t; j++) {
                uint64_t u = a[j], v = a[j + t];
                a[j] = addm(u, v, q);
                a[j + t] = oc_mulmod(subm(u, v, q), w, q);
            }
        }
    }
    const uint64_t ninv = oc_invmod((uint64_t)n, q);
    for (int j = 0; j < n; j++) a[j] = oc_mulmod(a[j], ninv, q);
}

uint64_t oc_rot_index(int logN, int64_t r) {
    const int64_t n = (int64_t)1 << (logN - 1);
    int64_t rr = r % n;
    if (rr < 0) rr += n;
    return oc_powmod(5, (uint64_t)rr, 2ull << logN);
}

void oc_automorph_eval(const oc_ctx* c, const uint64_t* in, uint64_t* out, uint64_t k) {
    const uint64_t M = 2ull * c->N;
    for (int i = 0; i < c->N; i++) {
        uint64_t e = 2ull * brev((uint32_t)i, c->logN) + 1;
        uint64_t f = (e * k) % M;
        uint32_t j = brev((uint32_t)((f - 1) / 2), c->logN);
        out[i] = in[j];
    }
}

void oc_automorph_coeff(const oc_ctx* c, const uint64_t* in, uint64_t* out, uint64_t k, int m) {
    const uint64_t q = c->mod[m], M = 2ull * c->N;
    for (int i = 0; i < c->N; i++) {
        uint64_t f = ((uint64_t)i * k) % M;
        if (f < (uint64_t)c->N) out[f] = in[i];
        else out[f - c->N] = in[i] ? q - in[i] : 0;
    }
}

/* ================================ rescale ========================================== */
/* Divide by the last modulus q_l with a centred lift of the last limb:
 * out_i = (x_i - [x_l]_centred mod q_i) * q_l^-1 mod q_i. */
void oc_rescale(const oc_ctx* c, const uint64_t* in, int nl, uint64_t* out) {
    const int N = c->N;
    const int l = nl - 1;
    const uint64_t ql = c->mod[l];
    uint64_t* last = (uint64_t*)malloc(sizeof(uint64_t) * N);
    uint64_t* tmp = (uint64_t*)malloc(sizeof(uint64_t) * N);
    memcpy(last, in + (size_t)l * N, sizeof(uint64_t) * N);
    oc_intt(c, last, l);
    for (int i = 0; i < l; i++) {
        const uint64_t qi = c->mod[i];
        for (int k = 0; k < N; k++) {
            uint64_t v = last[k];
            tmp[k] = v > ql / 2 ? subm(v % qi, ql % qi, qi) : v % qi;
        }
        oc_ntt(c, tmp, i);
        const uint64_t inv = oc_invmod(ql % qi, qi);
        for (int k = 0; k < N; k++) out[(size_t)i * N + k] = oc_mulmod(subm(in[(size_t)i * N + k], tmp[k], qi), inv, qi);
    }
    free(last); free(tmp);
}

/* ================================ key switching ==================================== */
static int ceil_div(int a, int b) { return (a + b - 1) / b; }

/* Q limbs 0..nl-1 map to modulus index t; P limbs map to nq + k.  "ext" limb index e in
 * [0, nl + np) maps to modulus ext_mod(e). */
static int ext_mod(const oc_ctx* c, int nl, int e) { return e < nl ? e : c->nq + (e - nl); }

void oc_modup(const oc_ctx* c, const uint64_t* in, int nl, uint64_t* out) {
    const int N = c->N, np = c->np, alpha = c->alpha;
    const int dnum = ceil_div(nl, alpha), ne = nl + np;
    uint64_t* coef = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)nl * N);
    memcpy(coef, in, sizeof(uint64_t) * (size_t)nl * N);
    for (int i = 0; i < nl; i++) oc_intt(c, coef + (size_t)i * N, i);
    uint64_t* t = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)alpha * N);
    for (int j = 0; j < dnum; j++) {
        const int lo = j * alpha, hi = (lo + alpha < nl) ? lo + alpha : nl, sz = hi - lo;
        /* t_i = [x_i * (Q_j/q_i)^-1]_{q_i} */
        for (int a = 0; a < sz; a++) {
            const int i = lo + a;
            const uint64_t qi = c->mod[i];
            uint64_t qhat = 1;
            for (int b = 0; b < sz; b++) if (b != a) qhat = oc_mulmod(qhat, c->mod[lo + b] % qi, qi);
            const uint64_t qhinv = oc_invmod(qhat, qi);
            for (int k = 0; k < N; k++) t[(size_t)a * N + k] = oc_mulmod(coef[(size_t)i * N + k], qhinv, qi);
        }
        uint64_t* oj = out + (size_t)j * ne * N;
        for (int e = 0; e < ne; e++) {
            const int m = ext_mod(c, nl, e);
            uint64_t* dst = oj + (size_t)e * N;
            if (e >= lo && e < hi) { memcpy(dst, in + (size_t)e * N, sizeof(uint64_t) * N); continue; }
            const uint64_t pm = c->mod[m];
            uint64_t qh[64];
            for (int a = 0; a < sz; a++) {
                uint64_t v = 1;
                for (int b = 0; b < sz; b++) if (b != a) v = oc_mulmod(v, c->mod[lo + b] % pm, pm);
                qh[a] = v;
            }
            for (int k = 0; k < N; k++) {
                u128 acc = 0;
                for (int a = 0; a < sz; a++) acc += (u128)t[(size_t)a * N + k] * qh[a];
                dst[k] = (uint64_t)(acc % pm);
            }
            oc_ntt(c, dst, m);
        }
    }
    free(coef); free(t);
}

void oc_moddown(const oc_ctx* c, const uint64_t* in, int nl, uint64_t* out) {
    const int N = c->N, np = c->np;
    uint64_t* coef = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)np * N);
    uint64_t* tmp = (uint64_t*)malloc(sizeof(uint64_t) * N);
    for (int k = 0; k < np; k++) {
        const int m = c->nq + k;
        const uint64_t pk = c->mod[m];
        memcpy(coef + (size_t)k * N, in + (size_t)(nl + k) * N, sizeof(uint64_t) * N);
        oc_intt(c, coef + (size_t)k * N, m);
        uint64_t phat = 1;
        for (int b = 0; b < np; b++) if (b != k) phat = oc_mulmod(phat, c->mod[c->nq + b] % pk, pk);
        const uint64_t phinv = oc_invmod(phat, pk);
        for (int x = 0; x < N; x++) coef[(size_t)k * N + x] = oc_mulmod(coef[(size_t)k * N + x], phinv, pk);
    }
    for (int i = 0; i < nl; i++) {
        const uint64_t qi = c->mod[i];
        uint64_t ph[64];
        uint64_t P = 1;
        for (int k = 0; k < np; k++) {
            uint64_t v = 1;
            for (int b = 0; b < np; b++) if (b != k) v = oc_mulmod(v, c->mod[c->nq + b] % qi, qi);
            ph[k] = v;
            P = oc_mulmod(P, c->mod[c->nq + k] % qi, qi);
        }
        const uint64_t Pinv = oc_invmod(P, qi);
        for (int x = 0; x < N; x++) {
            u128 acc = 0;
            for (int k = 0; k < np; k++) acc += (u128)coef[(size_t)k * N + x] * ph[k];
            tmp[x] = (uint64_t)(acc % qi);
        }
        oc_ntt(c, tmp, i);
        for (int x = 0; x < N; x++)
            out[(size_t)i * N + x] = oc_mulmod(subm(in[(size_t)i * N + x], tmp[x], qi), Pinv, qi);
    }
    free(coef); free(tmp);
}

void oc_key_inner(const oc_ctx* c, const uint64_t* ext, int nl, const uint64_t* key, uint64_t* out0, uint64_t* out1) {
    const int N = c->N, np = c->np, ne = nl + np, nk = c->nq + np;
    const int dnum = ceil_div(nl, c->alpha);
    for (int e = 0; e < ne; e++) {
        const int m = ext_mod(c, nl, e);
        const uint64_t q = c->mod[m];
        for (int x = 0; x < N; x++) {
            u128 a0 = 0, a1 = 0;
            for (int j = 0; j < dnum; j++) {
                const uint64_t d = ext[((size_t)j * ne + e) * N + x];
                const uint64_t kb = key[(((size_t)j * 2 + 0) * nk + m) * N + x];
                const uint64_t ka = key[(((size_t)j * 2 + 1) * nk + m) * N + x];
                a0 = (a0 + (u128)d * kb) % q;
                a1 = (a1 + (u128)d * ka) % q;
            }
            out0[(size_t)e * N + x] = (uint64_t)a0;
            out1[(size_t)e * N + x] = (uint64_t)a1;
        }
    }
}

void oc_keyswitch(const oc_ctx* c, const uint64_t* d, int nl, const uint64_t* key, uint64_t* out0, uint64_t* out1) {
    const int N = c->N, np = c->np, ne = nl + np;
    const int dnum = ceil_div(nl, c->alpha);
    uint64_t* ext = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)dnum * ne * N);
    uint64_t* i0 = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)ne * N);
    uint64_t* i1 = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)ne * N);
    oc_modup(c, d, nl, ext);
    oc_key_inner(c, ext, nl, key, i0, i1);
    oc_moddown(c, i0, nl, out0);
    oc_moddown(c, i1, nl, out1);
    free(ext); free(i0); free(i1);
}

/* ====================== limb-partitioned key switching (one rank's share) ============ */
/* A rank owns Q limbs [qlo, qlo + nqo) and P limbs [plo, plo + npo); its "own ext limbs" are those
 * Q limbs then those P limbs.  After the first exchange every rank holds all nl limbs of d in
 * coefficient form (dcoef); after the second, the np P limbs of the inner product (both
 * polynomials) in coefficient form.  These three pieces are the rank-local arithmetic. */
static int own_ext_mod(const oc_ctx* c, int nl, int qlo, int nqo, int plo, int o) {
    return o < nqo ? qlo + o : ext_mod(c, nl, nl + plo + (o - nqo));
}
static int own_ext_index(int nl, int qlo, int nqo, int plo, int o) { return o < nqo ? qlo + o : nl + plo + (o - nqo); }

void oc_ks_part_ext(const oc_ctx* c, const uint64_t* dcoef, int nl, int qlo, int nqo, int plo, int npo,
                    uint64_t* ext_own) {
    const int N = c->N, alpha = c->alpha, dnum = ceil_div(nl, alpha), no = nqo + npo;
    for (int j = 0; j < dnum; j++) {
        const int lo = j * alpha, hi = (lo + alpha < nl) ? lo + alpha : nl, sz = hi - lo;
        for (int o = 0; o < no; o++) {
            const int e = own_ext_index(nl, qlo, nqo, plo, o), m = own_ext_mod(c, nl, qlo, nqo, plo, o);
            const uint64_t pm = c->mod[m];
            uint64_t* dst = ext_own + ((size_t)j * no + o) * N;
            if (e >= lo && e < hi) {   /* the digit's own limb: d itself, back in eval form */
                memcpy(dst, dcoef + (size_t)e * N, sizeof(uint64_t) * N);
                oc_ntt(c, dst, m);
                continue;
            }
            uint64_t qhinv[64], qh[64];
            for (int a = 0; a < sz; a++) {
                const uint64_t qi = c->mod[lo + a];
                uint64_t v = 1, w = 1;
                for (int b = 0; b < sz; b++)
                    if (b != a) {
                        v = oc_mulmod(v, c->mod[lo + b] % qi, qi);
                        w = oc_mulmod(w, c->mod[lo + b] % pm, pm);
                    }
                qhinv[a] = oc_invmod(v, qi);
                qh[a] = w;
            }
            for (int k = 0; k < N; k++) {
                u128 acc = 0;
                for (int a = 0; a < sz; a++)
                    acc += (u128)oc_mulmod(dcoef[(size_t)(lo + a) * N + k], qhinv[a], c->mod[lo + a]) * qh[a];
                dst[k] = (uint64_t)(acc % pm);
            }
            oc_ntt(c, dst, m);
        }
    }
}

void oc_ks_part_inner(const oc_ctx* c, const uint64_t* ext_own, int nl, const uint64_t* key, int qlo, int nqo,
                      int plo, int npo, uint64_t* out0, uint64_t* out1) {
    const int N = c->N, nk = c->nq + c->np, dnum = ceil_div(nl, c->alpha), no = nqo + npo;
    for (int o = 0; o < no; o++) {
        const int m = own_ext_mod(c, nl, qlo, nqo, plo, o);
        const uint64_t q = c->mod[m];
        for (int x = 0; x < N; x++) {
            u128 a0 = 0, a1 = 0;
            for (int j = 0; j < dnum; j++) {
                const uint64_t d = ext_own[((size_t)j * no + o) * N + x];
                a0 = (a0 + (u128)d * key[(((size_t)j * 2 + 0) * nk + m) * N + x]) % q;
                a1 = (a1 + (u128)d * key[(((size_t)j * 2 + 1) * nk + m) * N + x]) % q;
            }
            out0[(size_t)o * N + x] = (uint64_t)a0;
            out1[(size_t)o * N + x] = (uint64_t)a1;
        }
    }
}

/* own Q limbs of one inner-product polynomial (eval) and all its np P limbs (coefficient form,
 * NOT yet multiplied by phat^-1) -> own Q limbs of the key-switch output */
void oc_ks_part_moddown(const oc_ctx* c, const uint64_t* in_own, const uint64_t* pcoef, int nl, int qlo, int nqo,
                        uint64_t* out_own) {
    const int N = c->N, np = c->np;
    uint64_t* t = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)np * N);
    uint64_t* tmp = (uint64_t*)malloc(sizeof(uint64_t) * N);
    for (int k = 0; k < np; k++) {
        const uint64_t pk = c->mod[c->nq + k];
        uint64_t phat = 1;
        for (int b = 0; b < np; b++) if (b != k) phat = oc_mulmod(phat, c->mod[c->nq + b] % pk, pk);
        const uint64_t phinv = oc_invmod(phat, pk);
        for (int x = 0; x < N; x++) t[(size_t)k * N + x] = oc_mulmod(pcoef[(size_t)k * N + x], phinv, pk);
    }
    for (int o = 0; o < nqo; o++) {
        const int i = qlo + o;
        const uint64_t qi = c->mod[i];
        uint64_t ph[64], P = 1;
        for (int k = 0; k < np; k++) {
            uint64_t v = 1;
            for (int b = 0; b < np; b++) if (b != k) v = oc_mulmod(v, c->mod[c->nq + b] % qi, qi);
            ph[k] = v;
            P = oc_mulmod(P, c->mod[c->nq + k] % qi, qi);
        }
        const uint64_t Pinv = oc_invmod(P, qi);
        for (int x = 0; x < N; x++) {
            u128 acc = 0;
            for (int k = 0; k < np; k++) acc += (u128)t[(size_t)k * N + x] * ph[k];
            tmp[x] = (uint64_t)(acc % qi);
        }
        oc_ntt(c, tmp, i);
        for (int x = 0; x < N; x++)
            out_own[(size_t)o * N + x] = oc_mulmod(subm(in_own[(size_t)o * N + x], tmp[x], qi), Pinv, qi);
    }
    free(t); free(tmp);
}

/* ================================ ciphertext ops =================================== */
void oc_ct_add(const oc_ctx* c, const uint64_t* a, const uint64_t* b, int nl, uint64_t* out) {
    const int N = c->N;
    for (int p = 0; p < 2; p++)
        for (int i = 0; i < nl; i++)
            for (int x = 0; x < N; x++) {
                size_t o = ((size_t)p * nl + i) * N + x;
                out[o] = addm(a[o], b[o], c->mod[i]);
            }
}

void oc_ct_mul_pt(const oc_ctx* c, const uint64_t* a, const uint64_t* pt, int nl, uint64_t* out) {
    const int N = c->N;
    for (int p = 0; p < 2; p++)
        for (int i = 0; i < nl; i++)
            for (int x = 0; x < N; x++) {
                size_t o = ((size_t)p * nl + i) * N + x;
                out[o] = oc_mulmod(a[o], pt[(size_t)i * N + x], c->mod[i]);
            }
}

void oc_ct_mul_relin(const oc_ctx* c, const uint64_t* a, const uint64_t* b, int nl, const uint64_t* rlk, uint64_t* out) {
    const int N = c->N;
    const size_t P = (size_t)nl * N;
    uint64_t* d2 = (uint64_t*)malloc(sizeof(uint64_t) * P);
    uint64_t* k0 = (uint64_t*)malloc(sizeof(uint64_t) * P);
    uint64_t* k1 = (uint64_t*)malloc(sizeof(uint64_t) * P);
    for (int i = 0; i < nl; i++) {
        const uint64_t q = c->mod[i];
        for (int x = 0; x < N; x++) {
            size_t o = (size_t)i * N + x;
            uint64_t a0 = a[o], a1 = a[P + o], b0 = b[o], b1 = b[P + o];
            out[o] = oc_mulmod(a0, b0, q);
            out[P + o] = addm(oc_mulmod(a0, b1, q), oc_mulmod(a1, b0, q), q);
            d2[o] = oc_mulmod(a1, b1, q);
        }
    }
    oc_keyswitch(c, d2, nl, rlk, k0, k1);
    for (int i = 0; i < nl; i++)
        for (int x = 0; x < N; x++) {
            size_t o = (size_t)i * N + x;
            out[o] = addm(out[o], k0[o], c->mod[i]);
            out[P + o] = addm(out[P + o], k1[o], c->mod[i]);
        }
    free(d2); free(k0); free(k1);
}

void oc_ct_rescale(const oc_ctx* c, const uint64_t* in, int nl, uint64_t* out) {
    const size_t P = (size_t)nl * c->N, Po = (size_t)(nl - 1) * c->N;
    oc_rescale(c, in, nl, out);
    oc_rescale(c, in + P, nl, out + Po);
}

/* (c0, c1) -> tau_k(c0 + KS(c1)_0, KS(c1)_1) with the key for s -> tau_{k^-1}(s). */
void oc_ct_automorph(const oc_ctx* c, const uint64_t* in, int nl, uint64_t k, const uint64_t* key, uint64_t* out) {
    const int N = c->N;
    const size_t P = (size_t)nl * N;
    uint64_t* k0 = (uint64_t*)malloc(sizeof(uint64_t) * P);
    uint64_t* k1 = (uint64_t*)malloc(sizeof(uint64_t) * P);
    oc_keyswitch(c, in + P, nl, key, k0, k1);
    for (int i = 0; i < nl; i++) {
        for (int x = 0; x < N; x++) k0[(size_t)i * N + x] = addm(k0[(size_t)i * N + x], in[(size_t)i * N + x], c->mod[i]);
        oc_automorph_eval(c, k0 + (size_t)i * N, out + (size_t)i * N, k);
        oc_automorph_eval(c, k1 + (size_t)i * N, out + P + (size_t)i * N, k);
    }
    free(k0); free(k1);
}

/* ================================ ChaCha20 + samplers ============================== */
static inline uint32_t rotl32(uint32_t v, int c) { return (v << c) | (v >> (32 - c)); }
#define QR(a, b, c, d)                          \
    a += b; d ^= a; d = rotl32(d, 16);          \
    c += d; b ^= c; b = rotl32(b, 12);          \
    a += b; d ^= a; d = rotl32(d, 8);           \
    c += d; b ^= c; b = rotl32(b, 7);

void oc_chacha20_block(const uint32_t key[8], uint32_t counter, const uint32_t nonce[3], uint32_t out[16]) {
    uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u, key[0], key[1], key[2], key[3],
                      key[4], key[5], key[6], key[7], counter, nonce[0], nonce[1], nonce[2]};
    uint32_t x[16];
    memcpy(x, s, sizeof x);
    for (int r = 0; r < 10; r++) {
        QR(x[0], x[4], x[8], x[12]); QR(x[1], x[5], x[9], x[13]);
        QR(x[2], x[6], x[10], x[14]); QR(x[3], x[7], x[11], x[15]);
        QR(x[0], x[5], x[10], x[15]); QR(x[1], x[6], x[11], x[12]);
        QR(x[2], x[7], x[8], x[13]); QR(x[3], x[4], x[9], x[14]);
    }
    for (int i = 0; i < 16; i++) out[i] = x[i] + s[i];
}

typedef struct { uint32_t key[8], nonce[3], w[16], counter; int pos; } stream_t;
static void stream_init(stream_t* s, const uint8_t seed[32], uint32_t n0, uint32_t n1, uint32_t tag) {
    for (int k = 0; k < 8; k++)
        s->key[k] = (uint32_t)seed[4 * k] | ((uint32_t)seed[4 * k + 1] << 8) | ((uint32_t)seed[4 * k + 2] << 16) |
                    ((uint32_t)seed[4 * k + 3] << 24);
    s->nonce[0] = n0; s->nonce[1] = n1; s->nonce[2] = tag;
    s->counter = 0; s->pos = 8;
}
static uint64_t stream_next(stream_t* s) {
    if (s->pos == 8) { oc_chacha20_block(s->key, s->counter++, s->nonce, s->w); s->pos = 0; }
    uint64_t v = (uint64_t)s->w[2 * s->pos] | ((uint64_t)s->w[2 * s->pos + 1] << 32);
    s->pos++;
    return v;
}

void oc_sample_uniform(const uint8_t seed[32], uint32_t n0, uint32_t n1, uint32_t tag, uint64_t q, uint64_t* out, int n) {
    stream_t s;
    stream_init(&s, seed, n0, n1, tag);
    const uint64_t r = (0 - q) % q, lim = 0 - r;
    for (int k = 0; k < n; k++) {
        uint64_t w = stream_next(&s);
        while (r != 0 && w >= lim) w = stream_next(&s);
        out[k] = w % q;
    }
}

void oc_sample_ternary_hw(const uint8_t seed[32], uint32_t n0, uint32_t n1, int h, int8_t* out, int n) {
    stream_t s;
    stream_init(&s, seed, n0, n1, TAG_SECR);
    memset(out, 0, (size_t)n);
    int placed = 0;
    while (placed < h && placed < n) {
        uint64_t u = stream_next(&s);
        uint32_t pos = (uint32_t)(u & (uint64_t)(n - 1));
        if (out[pos]) continue;
        out[pos] = (u >> 63) ? -1 : 1;
        placed++;
    }
}

void oc_sample_ternary(const uint8_t seed[32], uint32_t n0, uint32_t n1, int8_t* out, int n) {
    stream_t s;
    stream_init(&s, seed, n0, n1, TAG_TERN);
    for (int k = 0; k < n; k++) out[k] = (int8_t)((int)(stream_next(&s) % 3) - 1);
}

/* CDT of the rounded Gaussian: weights w_0 = 1, w_x = 2 exp(-x^2 / 2 sigma^2), x <= B. */
static int gauss_table(double sigma, uint64_t* T) {
    int B = (int)ceil(6.0 * sigma);
    if (B > 63) B = 63;
    double w[64], tot = 0.0, cum = 0.0;
    for (int x = 0; x <= B; x++) { w[x] = (x == 0 ? 1.0 : 2.0) * exp(-(double)x * x / (2.0 * sigma * sigma)); tot += w[x]; }
    for (int x = 0; x < B; x++) { cum += w[x]; T[x] = (uint64_t)(cum / tot * 9223372036854775808.0); }
    T[B] = 0x8000000000000000ull;
    return B;
}

void oc_sample_gauss(const uint8_t seed[32], uint32_t n0, uint32_t n1, double sigma, int32_t* out, int n) {
    uint64_t T[64];
    int B = gauss_table(sigma, T);
    stream_t s;
    stream_init(&s, seed, n0, n1, TAG_GAUS);
    for (int k = 0; k < n; k++) {
        uint64_t u = stream_next(&s);
        uint64_t r = u >> 1;
        int mag = 0;
        while (mag < B && r >= T[mag]) mag++;
        out[k] = (u & 1) ? -mag : mag;
    }
}

void oc_derive_seed(const uint8_t master[32], uint32_t id, uint32_t sub, uint8_t out[32]) {
    uint32_t key[8], nonce[3] = {id, sub, TAG_SEED}, w[16];
    for (int k = 0; k < 8; k++)
        key[k] = (uint32_t)master[4 * k] | ((uint32_t)master[4 * k + 1] << 8) | ((uint32_t)master[4 * k + 2] << 16) |
                 ((uint32_t)master[4 * k + 3] << 24);
    oc_chacha20_block(key, 0, nonce, w);
    for (int k = 0; k < 8; k++) {
        out[4 * k] = (uint8_t)w[k]; out[4 * k + 1] = (uint8_t)(w[k] >> 8);
        out[4 * k + 2] = (uint8_t)(w[k] >> 16); out[4 * k + 3] = (uint8_t)(w[k] >> 24);
    }
}

/* ================================ small polys / keys =============================== */
void oc_small_to_eval_i8(const oc_ctx* c, const int8_t* s, int m, uint64_t* out) {
    const uint64_t q = c->mod[m];
    for (int k = 0; k < c->N; k++) out[k] = s[k] >= 0 ? (uint64_t)s[k] : q - (uint64_t)(-s[k]);
    oc_ntt(c, out, m);
}
void oc_small_to_eval_i32(const oc_ctx* c, const int32_t* s, int m, uint64_t* out) {
    const uint64_t q = c->mod[m];
    for (int k = 0; k < c->N; k++) out[k] = s[k] >= 0 ? (uint64_t)s[k] % q : q - ((uint64_t)(-(int64_t)s[k]) % q);
    oc_ntt(c, out, m);
}

void oc_secret_eval(const oc_ctx* c, const int8_t* s, uint64_t* out) {
    for (int m = 0; m < c->nq + c->np; m++) oc_small_to_eval_i8(c, s, m, out + (size_t)m * c->N);
}

void oc_keygen_switch(const oc_ctx* c, const uint64_t* s_src_eval, const uint64_t* s_key_eval,
                      const uint8_t key_seed[32], double sigma, uint64_t* out) {
    const int N = c->N, nk = c->nq + c->np;
    const int dnum = ceil_div(c->nq, c->alpha);
    int32_t* e = (int32_t*)malloc(sizeof(int32_t) * N);
    uint64_t* ee = (uint64_t*)malloc(sizeof(uint64_t) * N);
    uint64_t P[64];
    for (int i = 0; i < c->nq; i++) {
        uint64_t v = 1;
        for (int k = 0; k < c->np; k++) v = oc_mulmod(v, c->mod[c->nq + k] % c->mod[i], c->mod[i]);
        P[i] = v;
    }
    for (int j = 0; j < dnum; j++) {
        oc_sample_gauss(key_seed, (uint32_t)j, 0, sigma, e, N);
        const int lo = j * c->alpha, hi = lo + c->alpha;
        for (int m = 0; m < nk; m++) {
            const uint64_t q = c->mod[m];
            uint64_t* b = out + (((size_t)j * 2 + 0) * nk + m) * N;
            uint64_t* a = out + (((size_t)j * 2 + 1) * nk + m) * N;
            oc_sample_uniform(key_seed, (uint32_t)j, (uint32_t)m, TAG_SKEY, q, a, N);
            oc_small_to_eval_i32(c, e, m, ee);
            const int in_digit = (m < c->nq && m >= lo && m < hi);
            for (int x = 0; x < N; x++) {
                uint64_t v = subm(ee[x], oc_mulmod(a[x], s_key_eval[(size_t)m * N + x], q), q);
                if (in_digit) v = addm(v, oc_mulmod(P[m], s_src_eval[(size_t)m * N + x], q), q);
                b[x] = v;
            }
        }
    }
    free(e); free(ee);
}

#define TAG_PKEY 0x59454b50u /* "PKEY" */

void oc_keygen_public(const oc_ctx* c, const uint64_t* s_eval, const uint8_t seed[32], double sigma, uint64_t* out) {
    const int N = c->N, nq = c->nq;
    int32_t* e = (int32_t*)malloc(sizeof(int32_t) * N);
    uint64_t* ee = (uint64_t*)malloc(sizeof(uint64_t) * N);
    oc_sample_gauss(seed, 0xFFFFFFFFu, 0, sigma, e, N);
    for (int m = 0; m < nq; m++) {
        const uint64_t q = c->mod[m];
        uint64_t* b = out + (size_t)m * N;
        uint64_t* a = out + ((size_t)nq + m) * N;
        oc_sample_uniform(seed, 0, (uint32_t)m, TAG_PKEY, q, a, N);
        oc_small_to_eval_i32(c, e, m, ee);
        for (int x = 0; x < N; x++) b[x] = subm(ee[x], oc_mulmod(a[x], s_eval[(size_t)m * N + x], q), q);
    }
    free(e); free(ee);
}

void oc_encrypt(const oc_ctx* c, const uint64_t* pk, const uint64_t* pt, int nl, const uint8_t seed[32],
                double sigma, uint64_t* out) {
    const int N = c->N, nq = c->nq;
    int8_t* v = (int8_t*)malloc((size_t)N);
    int32_t* e0 = (int32_t*)malloc(sizeof(int32_t) * N);
    int32_t* e1 = (int32_t*)malloc(sizeof(int32_t) * N);
    uint64_t* vv = (uint64_t*)malloc(sizeof(uint64_t) * N);
    uint64_t* ev = (uint64_t*)malloc(sizeof(uint64_t) * N);
    oc_sample_ternary(seed, 0, 3, v, N);
    oc_sample_gauss(seed, 0, 1, sigma, e0, N);
    oc_sample_gauss(seed, 0, 2, sigma, e1, N);
    const size_t P = (size_t)nl * N;
    for (int m = 0; m < nl; m++) {
        const uint64_t q = c->mod[m];
        oc_small_to_eval_i8(c, v, m, vv);
        oc_small_to_eval_i32(c, e0, m, ev);
        for (int x = 0; x < N; x++) {
            uint64_t t = addm(oc_mulmod(vv[x], pk[(size_t)m * N + x], q), ev[x], q);
            out[(size_t)m * N + x] = addm(t, pt[(size_t)m * N + x], q);
        }
        oc_small_to_eval_i32(c, e1, m, ev);
        for (int x = 0; x < N; x++)
            out[P + (size_t)m * N + x] = addm(oc_mulmod(vv[x], pk[((size_t)nq + m) * N + x], q), ev[x], q);
    }
    free(v); free(e0); free(e1); free(vv); free(ev);
}

void oc_decrypt(const oc_ctx* c, const uint64_t* ct, int nl, const uint64_t* s_eval, uint64_t* pt_out) {
    const int N = c->N;
    const size_t P = (size_t)nl * N;
    for (int m = 0; m < nl; m++) {
        const uint64_t q = c->mod[m];
        for (int x = 0; x < N; x++) {
            size_t o = (size_t)m * N + x;
            pt_out[o] = addm(ct[o], oc_mulmod(ct[P + o], s_eval[o], q), q);
        }
    }
}

/* ================================ CKKS encoding ==================================== */
/* Special FFT over the rotation group 5^j mod M (slot j <-> root zeta^{5^j}):
 * fwd: z_j = sum_k u_k zeta^{k 5^j};  inv: its inverse.  Radix-2 structure of the
 * CKKS "special FFT" (Cheon et al. 2018, HEAAN), written from that definition. */
static void bitrev_cplx(double* re, double* im, int n) {
    for (int i = 1, j = 0; i < n; i++) {
        int bit = n >> 1;
        for (; j & bit; bit >>= 1) j ^= bit;
        j ^= bit;
        if (i < j) {
            double t = re[i]; re[i] = re[j]; re[j] = t;
            t = im[i]; im[i] = im[j]; im[j] = t;
        }
    }
}

void oc_fft_special_fwd(double* re, double* im, int n, int M) {
    uint64_t* rg = (uint64_t*)malloc(sizeof(uint64_t) * n);
    uint64_t g = 1;
    for (int j = 0; j < n; j++) { rg[j] = g; g = (g * 5) % (uint64_t)M; }
    bitrev_cplx(re, im, n);
    for (int len = 2; len <= n; len <<= 1) {
        const int lenh = len >> 1, lenq = len << 2;
        for (int i = 0; i < n; i += len)
            for (int j = 0; j < lenh; j++) {
                const uint64_t idx = (rg[j] % (uint64_t)lenq) * (uint64_t)(M / lenq);
                const double wr = cos(2.0 * M_PI * (double)idx / M), wi = sin(2.0 * M_PI * (double)idx / M);
                const double ur = re[i + j], ui = im[i + j];
                const double xr = re[i + j + lenh], xi = im[i + j + lenh];
                const double vr = xr * wr - xi * wi, vi = xr * wi + xi * wr;
                re[i + j] = ur + vr; im[i + j] = ui + vi;
                re[i + j + lenh] = ur - vr; im[i + j + lenh] = ui - vi;
            }
    }
    free(rg);
}

void oc_fft_special_inv(double* re, double* im, int n, int M) {
    uint64_t* rg = (uint64_t*)malloc(sizeof(uint64_t) * n);
    uint64_t g = 1;
    for (int j = 0; j < n; j++) { rg[j] = g; g = (g * 5) % (uint64_t)M; }
    for (int len = n; len >= 1; len >>= 1) {
        const int lenh = len >> 1, lenq = len << 2;
        for (int i = 0; i < n; i += len)
            for (int j = 0; j < lenh; j++) {
                const uint64_t idx = ((uint64_t)lenq - (rg[j] % (uint64_t)lenq)) * (uint64_t)(M / lenq);
                const double wr = cos(2.0 * M_PI * (double)idx / M), wi = sin(2.0 * M_PI * (double)idx / M);
                const double ar = re[i + j], ai = im[i + j], br = re[i + j + lenh], bi = im[i + j + lenh];
                re[i + j] = ar + br; im[i + j] = ai + bi;
                const double dr = ar - br, di = ai - bi;
                re[i + j + lenh] = dr * wr - di * wi; im[i + j + lenh] = dr * wi + di * wr;
            }
    }
    bitrev_cplx(re, im, n);
    for (int i = 0; i < n; i++) { re[i] /= n; im[i] /= n; }
    free(rg);
}

int oc_encode(const oc_ctx* c, const double* re, const double* im, double scale, int nl, uint64_t* out) {
    const int N = c->N, n = N / 2;
    double* vr = (double*)malloc(sizeof(double) * n);
    double* vi = (double*)malloc(sizeof(double) * n);
    memcpy(vr, re, sizeof(double) * n);
    if (im) memcpy(vi, im, sizeof(double) * n); else memset(vi, 0, sizeof(double) * n);
    oc_fft_special_inv(vr, vi, n, 2 * N);
    int logc = -100000;
    for (int i = 0; i < n; i++) {
        vr[i] *= scale; vi[i] *= scale;
        if (vr[i] != 0.0) { int l = (int)ceil(log2(fabs(vr[i]))); if (l > logc) logc = l; }
        if (vi[i] != 0.0) { int l = (int)ceil(log2(fabs(vi[i]))); if (l > logc) logc = l; }
    }
    if (logc == -100000) logc = 0;
    if (logc < 0) { free(vr); free(vi); return 2; }
    const int logValid = logc <= 61 ? logc : 61, logApprox = logc - logValid;
    const double approx = pow(2.0, logApprox);
    const double maxv = (double)(int64_t)((1ull << 63) - (1ull << 9) - 1);
    int64_t* coef = (int64_t*)malloc(sizeof(int64_t) * N);
    for (int i = 0; i < n; i++) {
        double dr = vr[i] / approx, di = vi[i] / approx;
        if (fabs(dr) > maxv || fabs(di) > maxv) { free(vr); free(vi); free(coef); return 3; }
        coef[i] = llround(dr);
        coef[i + n] = llround(di);
    }
    for (int m = 0; m < nl; m++) {
        const uint64_t q = c->mod[m];
        uint64_t* o = out + (size_t)m * N;
        for (int k = 0; k < N; k++) o[k] = coef[k] >= 0 ? (uint64_t)coef[k] % q : (q - ((uint64_t)(-coef[k]) % q)) % q;
        oc_ntt(c, o, m);
        if (logApprox > 0) {
            const uint64_t f = oc_powmod(2, (uint64_t)logApprox, q);
            for (int k = 0; k < N; k++) o[k] = oc_mulmod(o[k], f, q);
        }
    }
    free(vr); free(vi); free(coef);
    return 0;
}

void oc_decode(const oc_ctx* c, const uint64_t* pt, double scale, double* re, double* im) {
    const int N = c->N, n = N / 2;
    const uint64_t q = c->mod[0];
    uint64_t* a = (uint64_t*)malloc(sizeof(uint64_t) * N);
    memcpy(a, pt, sizeof(uint64_t) * N);
    oc_intt(c, a, 0);
    for (int i = 0; i < n; i++) {
        uint64_t x = a[i], y = a[i + n];
        re[i] = (x > q / 2 ? -(double)(q - x) : (double)x) / scale;
        im[i] = (y > q / 2 ? -(double)(q - y) : (double)y) / scale;
    }
    oc_fft_special_fwd(re, im, n, 2 * N);
    free(a);
}
