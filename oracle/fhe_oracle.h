/*
 * fhe_oracle.h -- CPU restatement of the CKKS/RNS arithmetic on the fhe-ssm hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA engine in
 * fhe-ssm_b200/: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg
 * load it.  The engine never links it and never falls back to it.
 *
 * PARITY STATUS: unpinned against OpenFHE.  The reference's arithmetic lives in the
 * third-party OpenFHE v1.5.1 (harness/build_openfhe.sh:13-16) and FIDESlib
 * (docs/RUNBOOK.md:17), neither of which is in the reference tree or installable here.
 * Every routine below is written from the mathematics, following the conventions the
 * reference states in its own sources (cited per function), and the pieces that have
 * published known answers (ChaCha20, RFC 8439 section 2.3.2) are checked against them.
 *
 * Integer arithmetic uses unsigned __int128 products and the C '%' operator throughout:
 * slow, but obviously exact.  All residues are canonical, in [0, q).
 */
#ifndef FHE_ORACLE_H
#define FHE_ORACLE_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar modular arithmetic ---------------------------------------------------- */
uint64_t oc_mulmod(uint64_t a, uint64_t b, uint64_t q);
uint64_t oc_powmod(uint64_t a, uint64_t e, uint64_t q);
uint64_t oc_invmod(uint64_t a, uint64_t q);
int oc_is_prime(uint64_t n);

/* ---- moduli chain (OpenFHE-style selection, ParameterGenerationCKKSRNS rules) ----- */
/* q[0]: largest prime = 1 mod 2N below 2^q0bits; q[L-1]: smallest prime = 1 mod 2N above
 * 2^qbits, q[L-2..1] alternate below/above it; p[0..K-1]: successive primes = 1 mod 2N
 * below 2^pbits, skipping any already in q.  Returns 0 on success. */
int oc_gen_chain(int logN, int L, int q0bits, int qbits, int K, int pbits, uint64_t* q, uint64_t* p);
/* smallest primitive 2N-th root of unity mod q */
uint64_t oc_min_root(uint64_t q, int logN);

/* ---- context: ring degree + moduli (Q chain then P chain) ------------------------ */
typedef struct oc_ctx oc_ctx;
oc_ctx* oc_ctx_new(int logN, int nq, const uint64_t* q, int np, const uint64_t* p, int alpha);
void oc_ctx_free(oc_ctx* c);
uint64_t oc_modulus(const oc_ctx* c, int m);   /* m < nq: q_m; else p_{m-nq} */
uint64_t oc_root(const oc_ctx* c, int m);

/* ---- NTT (periodic_encode.hpp:241-260 ordering: natural in, bit-reversed out) ----- */
void oc_ntt(const oc_ctx* c, uint64_t* a, int m);
/* the same transform at ring 2^logN with an explicit primitive 2^(logN+1)-th root psi */
void oc_ntt_root(int logN, uint64_t q, uint64_t psi, uint64_t* a);
void oc_intt(const oc_ctx* c, uint64_t* a, int m);
/* eval-form automorphism X -> X^k (k odd): out[i] = in[j], 2brev(j)+1 = k(2brev(i)+1) mod 2N */
void oc_automorph_eval(const oc_ctx* c, const uint64_t* in, uint64_t* out, uint64_t k);
/* coefficient-form automorphism (negacyclic index map with sign) */
void oc_automorph_coeff(const oc_ctx* c, const uint64_t* in, uint64_t* out, uint64_t k, int m);
uint64_t oc_rot_index(int logN, int64_t r);   /* 5^r mod 2N (r reduced mod N/2) */

/* ---- polynomials with nl limbs (Q limbs 0..nl-1), eval form, layout [limb][N] ------ */
/* rescale: drop limb nl-1 with a centred lift, out has nl-1 limbs */
void oc_rescale(const oc_ctx* c, const uint64_t* in, int nl, uint64_t* out);
/* ModUp: in (nl Q-limbs, eval) -> out[dnum_l][nl + np][N], dnum_l = ceil(nl/alpha) */
void oc_modup(const oc_ctx* c, const uint64_t* in, int nl, uint64_t* out);
/* ModDown: in (nl Q-limbs then np P-limbs, eval) -> out (nl Q-limbs) */
void oc_moddown(const oc_ctx* c, const uint64_t* in, int nl, uint64_t* out);
/* key inner product: ext [dnum_l][nl+np][N]; key [dnum_top][2][nq+np][N] -> out0/out1 [nl+np][N] */
void oc_key_inner(const oc_ctx* c, const uint64_t* ext, int nl, const uint64_t* key, uint64_t* out0, uint64_t* out1);
/* full key switch of d (nl limbs, eval) -> (out0, out1) (nl limbs each) */
void oc_keyswitch(const oc_ctx* c, const uint64_t* d, int nl, const uint64_t* key, uint64_t* out0, uint64_t* out1);

/* ---- limb-partitioned key switching: one rank's share ------------------------------
 * The rank owns Q limbs [qlo, qlo+nqo) and P limbs [plo, plo+npo) ("own ext limbs": those Q limbs
 * then those P limbs).  ext: dcoef = all nl Q limbs of d in coefficient form (after the first
 * all-gather) -> ext_own [dnum][nqo+npo][N] eval.  inner: -> out0/out1 [nqo+npo][N].  moddown:
 * in_own = own Q limbs of one inner-product polynomial (eval), pcoef = its np P limbs in
 * coefficient form (after the second all-gather) -> out_own [nqo][N]. */
void oc_ks_part_ext(const oc_ctx* c, const uint64_t* dcoef, int nl, int qlo, int nqo, int plo, int npo,
                    uint64_t* ext_own);
void oc_ks_part_inner(const oc_ctx* c, const uint64_t* ext_own, int nl, const uint64_t* key, int qlo, int nqo,
                      int plo, int npo, uint64_t* out0, uint64_t* out1);
void oc_ks_part_moddown(const oc_ctx* c, const uint64_t* in_own, const uint64_t* pcoef, int nl, int qlo, int nqo,
                        uint64_t* out_own);

/* ---- ciphertext ops; a ct with nl limbs is [2][nl][N] ---------------------------- */
void oc_ct_add(const oc_ctx* c, const uint64_t* a, const uint64_t* b, int nl, uint64_t* out);
void oc_ct_mul_pt(const oc_ctx* c, const uint64_t* a, const uint64_t* pt, int nl, uint64_t* out);
/* ct x ct -> relinearised (no rescale) */
void oc_ct_mul_relin(const oc_ctx* c, const uint64_t* a, const uint64_t* b, int nl, const uint64_t* rlk, uint64_t* out);
void oc_ct_rescale(const oc_ctx* c, const uint64_t* in, int nl, uint64_t* out);
/* rotation / conjugation by automorphism index k with the key for tau_{k^-1}(s) */
void oc_ct_automorph(const oc_ctx* c, const uint64_t* in, int nl, uint64_t k, const uint64_t* key, uint64_t* out);

/* ---- ChaCha20 (RFC 8439) and the seeded samplers (seeded_keys.hpp:36-49) ---------- */
void oc_chacha20_block(const uint32_t key[8], uint32_t counter, const uint32_t nonce[3], uint32_t out[16]);
/* uniform mod q by rejection, stream nonce {n0, n1, tag} */
void oc_sample_uniform(const uint8_t seed[32], uint32_t n0, uint32_t n1, uint32_t tag, uint64_t q, uint64_t* out, int n);
/* sparse ternary with exactly h nonzeros, as signed int8 coefficients */
void oc_sample_ternary_hw(const uint8_t seed[32], uint32_t n0, uint32_t n1, int h, int8_t* out, int n);
/* uniform ternary {-1,0,1} */
void oc_sample_ternary(const uint8_t seed[32], uint32_t n0, uint32_t n1, int8_t* out, int n);
/* rounded discrete Gaussian of width sigma (CDT over |x| <= ceil(6 sigma)) */
void oc_sample_gauss(const uint8_t seed[32], uint32_t n0, uint32_t n1, double sigma, int32_t* out, int n);
/* 32-byte per-object seed from a master seed: ChaCha20(master, 0, {id, sub, 'SEED'}) */
void oc_derive_seed(const uint8_t master[32], uint32_t id, uint32_t sub, uint8_t out[32]);

/* ---- small signed polynomial -> eval form over modulus m -------------------------- */
void oc_small_to_eval_i8(const oc_ctx* c, const int8_t* s, int m, uint64_t* out);
void oc_small_to_eval_i32(const oc_ctx* c, const int32_t* s, int m, uint64_t* out);

/* ---- keys ------------------------------------------------------------------------- */
/* hybrid key from s_src to s_key (both given as signed small polys? no: eval form over all
 * nq+np moduli, layout [nq+np][N]); key_seed drives a_j (tag SKEY), e_j (tag GAUS).
 * out: [dnum_top][2][nq+np][N] with component 0 = b, 1 = a. */
void oc_keygen_switch(const oc_ctx* c, const uint64_t* s_src_eval, const uint64_t* s_key_eval,
                      const uint8_t key_seed[32], double sigma, uint64_t* out);
/* eval-form secret over all moduli from its signed coefficients */
void oc_secret_eval(const oc_ctx* c, const int8_t* s, uint64_t* out);
/* public key (b = -a s + e, a) over nq limbs, out [2][nq][N] */
void oc_keygen_public(const oc_ctx* c, const uint64_t* s_eval, const uint8_t seed[32], double sigma, uint64_t* out);
/* encrypt plaintext pt (nl limbs, eval) with pk: out [2][nl][N]; randomness from seed */
void oc_encrypt(const oc_ctx* c, const uint64_t* pk, const uint64_t* pt, int nl, const uint8_t seed[32],
                double sigma, uint64_t* out);
/* decrypt to eval-form plaintext (nl limbs) */
void oc_decrypt(const oc_ctx* c, const uint64_t* ct, int nl, const uint64_t* s_eval, uint64_t* pt_out);

/* ---- CKKS encoding (special FFT; periodic_encode.hpp:186-237 rounding) ------------ */
void oc_fft_special_inv(double* re, double* im, int n, int M);
void oc_fft_special_fwd(double* re, double* im, int n, int M);
/* encode n=N/2 complex slots at scale into nl limbs (eval form); returns 0 or an error */
int oc_encode(const oc_ctx* c, const double* re, const double* im, double scale, int nl, uint64_t* out);
/* decode from an eval-form plaintext, reading limb 0 only (|value| < q0/2 assumed) */
void oc_decode(const oc_ctx* c, const uint64_t* pt, double scale, double* re, double* im);

#ifdef __cplusplus
}
#endif
#endif
