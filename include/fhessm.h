/*
 * fhessm.h -- C-ABI of the B200 CKKS evaluation engine (libfhessm.so).
 *
 * The drop-in boundary for the hot path of xelananv/fhe-ssm.  The reference's server calls
 * the OpenFHE / FIDESlib CryptoContext API with C++ shared pointers and exceptions
 * (hpc_gpu_port/gpu_real_model.cu, harness/cpu_real_model.cpp); this header exports the same
 * operations as plain C: opaque handles, host pointers and sizes, integer status codes.
 * Each entry point names the reference call it replaces (file:line in the reference tree).
 *
 * Conventions
 *  - Every function returns FHE_OK (0) or a negative status; fhe_last_error() returns the
 *    message of the last failure on the calling thread.  Nothing degrades silently: a
 *    request the engine cannot serve exactly is refused (the reference's "refuse loudly"
 *    rule, gpu_real_model.cu:924-928, :975-993).
 *  - A context owns one CUDA device and one stream; every handle it creates lives in that
 *    device's memory.  Calls on one context must come from one thread at a time.
 *  - "level" counts consumed levels as the reference's TrackedCt::used does
 *    (gpu_real_model.cu:1547-1551): level 0 = all L limbs, level L-1 = one limb.
 *  - Word layouts for raw import/export: a polynomial is [limb][N] uint64 residues in
 *    evaluation (NTT) form, bit-reversed order; a ciphertext is [2][limbs][N]; a switching
 *    key is [digit][2 (b, a)][L + K][N] with digit = ceil(L / alpha).
 *  - Handles are freed with their fhe_*_free function; freeing NULL is a no-op.
 */
#ifndef FHESSM_H
#define FHESSM_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

#define FHE_OK 0
#define FHE_ERR_ARG (-1)        /* bad argument */
#define FHE_ERR_CUDA (-3)       /* CUDA runtime error */
#define FHE_ERR_LEVEL (-4)      /* level / scale mismatch between operands */
#define FHE_ERR_KEY (-5)        /* a required key is missing */
#define FHE_ERR_RANGE (-6)      /* value out of the encodable range (refused) */
#define FHE_ERR_PROTO (-7)      /* malformed request / file (server step) */

typedef struct fhe_ctx fhe_ctx;
typedef struct fhe_ct fhe_ct;
typedef struct fhe_pt fhe_pt;

typedef struct {
    int logN;       /* ring degree 2^logN, 12..16 */
    int L;          /* Q limbs at the top level (q0 + L-1 scaling primes) */
    int K;          /* special primes */
    int alpha;      /* limbs per key-switching digit (dnum = ceil(L / alpha)) */
    int q0bits;     /* first modulus size (60) */
    int qbits;      /* scaling modulus size (45) */
    int pbits;      /* special modulus size (60) */
    int hw;         /* secret Hamming weight (192); 0 = uniform ternary */
    double sigma;   /* error width (3.19) */
    int device;     /* CUDA device ordinal */
    int boot_primes;  /* top limbs drawn as boot_bits-bit primes for the bootstrap circuit (0: none) */
    int boot_bits;    /* size of those primes (58) */
} fhe_params;

const char* fhe_last_error(void);

/* ---- context ----------------------------------------------------------------------------
 * replaces CCParams + GenCryptoContext + Enable (gpu_real_model.cu:1138-1164) and
 * LoadContext / SetDevices (:1530, :1161): the chain, NTT tables and keys live on `device`. */
int fhe_ctx_create(const fhe_params* p, fhe_ctx** out);
void fhe_ctx_destroy(fhe_ctx* cx);
/* the moduli chain: L Q-moduli then K special moduli */
int fhe_ctx_moduli(const fhe_ctx* cx, uint64_t* out);
/* FLEXIBLEAUTO scaling factor at `level` (CryptoParametersRNS::GetScalingFactorReal) */
double fhe_ctx_scale(const fhe_ctx* cx, int level);
int fhe_ctx_sync(fhe_ctx* cx);
/* device memory: out[0] free bytes, out[1] total, out[2] bytes the stream-ordered pool holds,
 * out[3] bytes of it in live buffers, out[4] bytes of cached BSGS plaintexts */
int fhe_ctx_memory(fhe_ctx* cx, long long* out);
/* kernel launches issued by this context so far */
long long fhe_ctx_launches(const fhe_ctx* cx);
/* key switches issued so far and the sum of their limb counts (operation census) */
int fhe_ctx_counters(const fhe_ctx* cx, long long* keyswitches, long long* ks_limbs);
/* a named statistic of the context: "launches", "keyswitches", "ks_limbs", "pt_encodes" (plaintexts
 * encoded on a cache miss), "pt_cached" (plaintexts held by the encode cache), "host_waits" (times a
 * host-to-device upload had to wait for an earlier one's staging buffer).  Unknown name: error. */
int fhe_ctx_stat(const fhe_ctx* cx, const char* name, long long* value);
/* the context's CUDA stream (cudaStream_t), for callers that time it with CUDA events */
void* fhe_ctx_stream(const fhe_ctx* cx);
/* engine options: "matvec_tensor_cores" (default 1): BSGS products on the tcgen05 tensor cores
 * (byte-split integer MMA); 0 selects the CUDA-core kernel (same results, bit for bit).
 * "merged_rescale" (default 1): circuit products divide by P q_l once (ModDown and rescale
 * merged); 0 runs ModDown and rescale separately.
 * "profile_every" (default 1): the per-kernel timer times one scope in this many of each kind
 * and scales the totals (keeps the timer's own cost out of a timed region).
 * "plaintext_cache" (default 0): 1 = a BSGS plan keeps the plaintext words of its last call
 * (level and scale) resident and reuses them when the next call has the same level and scale,
 * the reference's --cache-diags (gpu_real_model.cu:1647-1652, also off by default there).
 * "plaintext_cache_reserve_mib" (default 24576): a plan caches only while this much device
 * memory would stay free.
 * "pdl" (default 1): programmatic dependent launch of the hot kernels.
 * "ntt_cluster" (default 0): N = 2^16 transforms as one 8-CTA cluster launch per limb.
 * "ntt_arith" (default 1): NTT butterflies with the cheaper Shoup quotient; 0: exact quotient
 * (the same words either way).
 * "baby_limbs" (default 8): limbs walked by one thread of the baby key inner products.
 * "boot_compress" (default 1): bootstrap levels with slot-periodic diagonals keep their
 * plaintexts compressed (read by the next fhe_bootstrap_setup; the same words).
 * "boot_delta_log2" (default 0 = 2^(bits(q0) - 11)): the bootstrap input scale, read by the
 * next fhe_bootstrap_setup; -1 = the chain's canonical level-1 scale, 30..56 = 2^value. */
int fhe_ctx_set_option(fhe_ctx* cx, const char* name, int value);
/* per-kernel CUDA-event timing on the context's stream (off by default).  collect
 * synchronises, writes {"kernel": [launches, total_ms, algorithmic_bytes], ...} as JSON
 * into buf (cap bytes) and resets the counters. */
int fhe_prof_enable(fhe_ctx* cx, int on);
int fhe_prof_collect(fhe_ctx* cx, char* buf, int cap);

/* ---- keys -------------------------------------------------------------------------------
 * replaces KeyGen + EvalMultKeyGen (gpu_real_model.cu:1293-1298); all randomness from the
 * 32-byte seed through the ChaCha20 expander of hpc_gpu_port/seeded_keys.hpp:36-49. */
int fhe_keygen(fhe_ctx* cx, const uint8_t seed[32]);
/* replaces EvalRotateKeyGen(rots) (:1299-1336); conj != 0 adds the conjugation key */
int fhe_keygen_rotations(fhe_ctx* cx, const int32_t* steps, int n, int conj);
/* switching keys for the automorphism indices idx[0..n) (odd, < 2N; 1 is skipped): the client
 * minting the index list of a rotation-index contract (fhe_model_rot_contract's autoIndices) */
int fhe_keygen_auto(fhe_ctx* cx, const uint64_t* idx, int n);
/* raw key material (canonical residues), for parity checks and key files:
 * which = 0: relinearisation key; otherwise the automorphism index (5^r mod 2N, or 2N-1). */
int fhe_key_export(fhe_ctx* cx, uint64_t which, uint64_t* words);
int fhe_key_import(fhe_ctx* cx, uint64_t which, const uint64_t* words);
int fhe_secret_export(fhe_ctx* cx, int8_t* coeffs);
int fhe_pubkey_export(fhe_ctx* cx, uint64_t* words);   /* [2][L][N] (b, a) */
uint64_t fhe_rot_index(const fhe_ctx* cx, int32_t step);

/* ---- encoding ---------------------------------------------------------------------------
 * replaces MakeCKKSPackedPlaintext(v, 1, level) (gpu_real_model.cu:1577-1589): n complex
 * slot values (n divides N/2; a shorter vector repeats across the slots) encoded at `level`
 * with the given scale (scale <= 0: the level's FLEXIBLEAUTO factor). */
int fhe_encode(fhe_ctx* cx, const double* re, const double* im, int n, int level, double scale, fhe_pt** out);
/* replaces Plaintext::GetRealPackedValue / GetCKKSPackedValue (:2211): N/2 slots */
int fhe_decode(fhe_ctx* cx, const fhe_pt* pt, double* re, double* im);
/* The compressed store entry of a periodic slot vector (replaces periodicEncodeComp,
 * hpc_gpu_port/periodic_encode.hpp:263-276, the store entry of buildComp, gpu_real_model.cu:
 * 2888-2925): count vectors of `period` complex slots (re, im: [count][period]; im may be NULL),
 * each tiled N/(2 period) times across the slots, encoded at `level` and `scale` (<= 0: the
 * level's scale) into words [count][L - level][2 period], canonical.  Word j2 of limb l equals
 * word j2 << log2(N / (2 period)) of fhe_encode of the tiled vector.  period: a power of two in
 * [4, 2048] dividing N/2.  The words come from the device generator the matvec plans use. */
int fhe_encode_periodic(fhe_ctx* cx, const double* re, const double* im, int period, int count, int level,
                        double scale, uint64_t* words);
void fhe_pt_free(fhe_pt* pt);
int fhe_pt_level(const fhe_pt* pt);

/* ---- encryption -------------------------------------------------------------------------
 * replaces Encrypt(pk, pt) / Decrypt(sk, ct) (gpu_real_model.cu:2202-2221, encCh/decCh) */
int fhe_encrypt(fhe_ctx* cx, const fhe_pt* pt, fhe_ct** out);
int fhe_decrypt(fhe_ctx* cx, const fhe_ct* ct, fhe_pt** out);
void fhe_ct_free(fhe_ct* ct);
int fhe_ct_level(const fhe_ct* ct);
double fhe_ct_scale(const fhe_ct* ct);
int fhe_ct_copy(fhe_ctx* cx, const fhe_ct* a, fhe_ct** out);

/* ---- evaluation -------------------------------------------------------------------------
 * EvalMult(ct, pt) without rescale (mulPt = this + fhe_rescale, gpu_real_model.cu:2629-2632) */
int fhe_mul_ct_pt(fhe_ctx* cx, const fhe_ct* a, const fhe_pt* pt, fhe_ct** out);
/* EvalMult(ct, ct) with relinearisation, no rescale (rmsnorm x^2 :3520, polyGate3 :4627) */
int fhe_mul_ct_ct_relin(fhe_ctx* cx, const fhe_ct* a, const fhe_ct* b, fhe_ct** out);
/* EvalAdd / EvalSub with the levels and scales reconciled, as OpenFHE's FLEXIBLEAUTO EvalAdd
   does for addAligned (:2692-2743, the add at :2743): the operand with more limbs is aligned down
   to the other's level and scale; at equal levels an integer scale ratio is fixed by an exact
   integer product and any other ratio by aligning both one level down.  Operands already at one
   level and scale are added as they are. */
int fhe_add(fhe_ctx* cx, const fhe_ct* a, const fhe_ct* b, fhe_ct** out);
int fhe_sub(fhe_ctx* cx, const fhe_ct* a, const fhe_ct* b, fhe_ct** out);
/* EvalAdd(ct, pt) (addPtV :2756-2759) */
int fhe_add_pt(fhe_ctx* cx, const fhe_ct* a, const fhe_pt* pt, fhe_ct** out);
/* EvalMult by a real constant encoded at `scale` (scale <= 0: the ct's level factor), no rescale */
int fhe_mul_const(fhe_ctx* cx, const fhe_ct* a, double v, double scale, fhe_ct** out);
/* EvalAdd of a real constant in every slot */
int fhe_add_const(fhe_ctx* cx, const fhe_ct* a, double v, fhe_ct** out);
/* RescaleInPlace (:2631, :2820) */
int fhe_rescale(fhe_ctx* cx, fhe_ct* ct);
/* LevelReduceInternalInPlace (experimental/gpu_real_model_x.cu:2778): drop limbs, no rescale */
int fhe_level_reduce(fhe_ctx* cx, fhe_ct* ct, int levels);
/* EvalRotate(ct, k) (:2762-2765): slot i of the result = slot i+k of the input */
int fhe_rotate(fhe_ctx* cx, const fhe_ct* a, int32_t k, fhe_ct** out);
/* hoisted rotations: one ModUp shared by n rotations (EvalFastRotation; used by the BSGS babies) */
int fhe_rotate_hoisted(fhe_ctx* cx, const fhe_ct* a, const int32_t* ks, int n, fhe_ct** outs);
/* sum_i EvalRotate(in[i], ks[i]) for inputs at one level and scale (the BSGS giant step,
 * matvecBatch :3407): the rotations share one batched ModUp and a single ModDown of the sum
 * (at most one ks[i] may be 0) */
int fhe_rotate_sum(fhe_ctx* cx, const fhe_ct* const* in, const int32_t* ks, int n, fhe_ct** out);
/* EvalConj: complex conjugation of every slot (automorphism 2N-1, :1355-1369) */
int fhe_conjugate(fhe_ctx* cx, const fhe_ct* a, fhe_ct** out);

/* ---- circuit-level operations ----------------------------------------------------------
 * mulPt (gpu_real_model.cu:2629-2632): EvalMult by a per-slot vector (re/im, n slots
 * repeated across N/2) + RescaleInPlace; the plaintext scale is chosen so the result sits on
 * the next level's FLEXIBLEAUTO factor */
int fhe_mul_vec_rescale(fhe_ctx* cx, const fhe_ct* a, const double* re, const double* im, int n, fhe_ct** out);
/* alignTo (:2636-2641): bring a ciphertext down to `level` at that level's factor (one
 * integer product + rescale whatever the gap); in place */
int fhe_align(fhe_ctx* cx, fhe_ct* ct, int level);
/* EvalMult(ct, ct) + relinearise + rescale, operands aligned to the lower level first */
int fhe_mul_rescale(fhe_ctx* cx, const fhe_ct* a, const fhe_ct* b, fhe_ct** out);
/* polyGate3 / channel-mix polynomials (:4609-4649, :5130-5163): sum_i c_i (.) x^i, power
 * basis, c = [deg+1][n] real per-slot coefficients (n slots, repeated) */
int fhe_poly_eval(fhe_ctx* cx, const fhe_ct* x, const double* coeffs, int deg, int n, fhe_ct** out);
/* sum_i c_i T_i(x) (Chebyshev basis, |x| <= 1), baby-step / giant-step, depth
 * ceil(log2(ncoef)) + 1 */
int fhe_cheb_eval(fhe_ctx* cx, const fhe_ct* x, const double* coeffs, int ncoef, fhe_ct** out);
/* levels fhe_cheb_eval consumes on a canonical-scale input for these coefficients (host only:
 * the bootstrap plans SlotToCoeff's level with it) */
int fhe_cheb_depth(const double* coeffs, int ncoef, int* depth);
/* the same series on `count` ciphertexts of one level and scale, every ciphertext product of
 * the evaluations batched (the bootstrap's EvalMod runs its real and imaginary parts this way) */
int fhe_cheb_eval_n(fhe_ctx* cx, const fhe_ct* const* xs, int count, const double* coeffs, int ncoef,
                    fhe_ct** outs);
/* EvalBootstrapSetup + EvalBootstrapKeyGen (gpu_real_model.cu:1436-1444, :1293-1336):
 * CoeffToSlot / SlotToCoeff plaintexts, the EvalMod interpolant (degree `degree` on
 * [-bound, bound] before 3 double angles) and the rotation + conjugation keys */
int fhe_bootstrap_setup(fhe_ctx* cx, double bound, int degree);
/* the same with the number of double-angle steps of EvalMod (fhe_bootstrap_setup: 3); the
 * interpolant is of cos(2 pi (B x - 1/4) / 2^double_angles) */
int fhe_bootstrap_setup_r(fhe_ctx* cx, double bound, int degree, int double_angles);
/* EvalBootstrap (:2544): refresh to level fhe_bootstrap_level() */
int fhe_bootstrap(fhe_ctx* cx, const fhe_ct* a, fhe_ct** out);
/* a batch of n ciphertexts, one after another on the context's stream (the batched
 * EvalBootstrap of baseline config 3, 32 ciphertexts per call); out[i] refreshes in[i] */
int fhe_bootstrap_n(fhe_ctx* cx, const fhe_ct* const* in, int n, fhe_ct** out);
int fhe_bootstrap_level(const fhe_ctx* cx);
/* diagnostics: the bootstrap pipeline stopped after stage `upto` (1 ModRaise, 2 CoeffToSlot,
 * 3 EvalMod, 4 complete) */
int fhe_bootstrap_stage(fhe_ctx* cx, const fhe_ct* a, int upto, fhe_ct** out);

/* ---- BSGS matvec (matvecBatch / matvecBatchChunked, gpu_real_model.cu:2883-3431) ---------
 * A plan holds the masked block-cyclic diagonals of W (rows x cols, row-major, rows <= D)
 * for a layout of one D-channel vector per block of D slots; column chunk s of W multiplies
 * input ciphertext s.  b1 = baby steps (D / b1 giant steps). */
typedef struct fhe_mvplan fhe_mvplan;
int fhe_matvec_plan(fhe_ctx* cx, const double* W, int rows, int cols, int D, int b1, fhe_mvplan** out);
void fhe_mvplan_free(fhe_mvplan* pl);
/* rotation keys the matvec needs: j, j - D (babies), g b1 (giants; one giant family: the
 * plan's D-periodic diagonals let every family share the g b1 rotation) */
int fhe_matvec_keygen(fhe_ctx* cx, int D, int b1);
/* out = W [in_0 | in_1 | ...], one level consumed, canonical scale */
int fhe_matvec_bsgs(fhe_ctx* cx, const fhe_mvplan* pl, const fhe_ct* const* in, int nin, fhe_ct** out);

/* ---- the encrypted model step -------------------------------------------------------------
 * The layer loop of gpu_real_model.cu:4744-5264 (+ carry :4688-4737, :5271-5300, output norm
 * :5389) for the polynomial SSM of train_fhe_native_ssm.py (_fwd_np :829-890).  Lanes: one
 * conversation per block of D slots, complex packing (lane r real part, lane r + N/2D
 * imaginary part).  vecs: d-length decay, 1-decay, g1, mix, c, dd, p0, p1, p2, g2 then
 * dff-length q0, q1, q2, q3, r0, r1, r2; seeds (18 values): rmsnorm Newton seeds (a, b, iters)
 * of the time-mix and channel-mix norms (the bundle's L{i}.{tm,cm}.rsqrt,
 * train_fhe_native_ssm.py:1121-1124), then the bootstrap gains of the refresh sites tm.x,
 * tm.ms, u, s, g, cm.x, cm.ms, v, f, tm.y, cm.y, z (a site is refreshed at value * gain: a
 * bootstrap's error is absolute, so small-valued sites are scaled up by relabelling the scale).
 * fhe_model_set_output: seed3 = (a, b, iters, gain x, gain ms, gain y) of the output norm. */
typedef struct fhe_model fhe_model;
typedef struct {
    int d, dff, n_layer, D, b1;
    double a_min, a_max, alpha, eps;
    int shift_mix;
} fhe_model_cfg;
int fhe_model_create(fhe_ctx* cx, const fhe_model_cfg* cfg, fhe_model** out);
void fhe_model_free(fhe_model* m);
int fhe_model_set_layer(fhe_model* m, int layer, const double* win, const double* wout, const double* wk,
                        const double* wr, const double* wv, const double* vecs, const double* seeds);
int fhe_model_set_output(fhe_model* m, const double* g_out, const double* seed3);
/* rotation keys of the matvecs and the norm reductions (bootstrap keys: fhe_bootstrap_setup) */
int fhe_model_keygen(fhe_model* m);
/* drop the carried state (req.N.reset, gpu_real_model.cu:4465-4469) */
int fhe_model_reset(fhe_model* m);
/* one token for every lane: in = embedded rows, out = rmsnorm(h, g_out) (the client applies
 * the tied head in plaintext, --dec-out :2444-2533) */
int fhe_model_step(fhe_model* m, const fhe_ct* in, fhe_ct** out);
int fhe_model_stats(const fhe_model* m, long long* bootstraps, long long* steps);
/* bootstraps per refresh site since creation (the refresh rule of gpu_real_model.cu:2573-2599):
 * 0 norm input x, 1 norm mean square, 2 norm Newton y, 3 norm Newton -ms/2, 4 norm tail y,
 * 5 shift-mix input, 6 previous u, 7 matvec input u, 8 carried state, 9 new state, 10 readout
 * z, 11 gate output, 12 channel-mix input v, 13 channel-mix product f */
int fhe_model_refresh_census(const fhe_model* m, long long* counts, int n);
/* diagnostics: k > 0 makes fhe_model_step return the layer-0 intermediate k (1 norm,
 * 2 shift-mix, 3 Win x, 4 scan, 5 readout, 6 gate, 7 h+attn, 8 norm 2, 9 k_0, 10 f_0, 11 h+ffn) */
int fhe_model_probe(fhe_model* m, int k);
/* server step (the request/response of the serve loop :4385-4483): n_in input ciphertexts
 * (one per pack), flags bit 0 = reset the carry first; *n_out outputs */
int fhe_server_step(fhe_model* m, const fhe_ct* const* in, int n_in, fhe_ct** out, int* n_out, int flags);

/* ---- the serve loop (the --serve REQDIR --stateful loop of gpu_real_model.cu:4363-4483) ----
 * req.<N>.{0..count-1} + req.<N>.meta (+ req.<N>.reset) + req.<N>.ready in, resp.<N>.* +
 * resp.<N>.meta + resp.<N>.done (or resp.<N>.error) out, serve.status kept current, a `stop`
 * file (or timeout_ms idle, or max_requests > 0 served) ends it.  Ciphertext files: "FSSMCT01",
 * int32 level, limbs, logN, pad, double scale, [2][limbs][N] uint64 words. */
typedef struct {
    int level, nl, logN;
    double scale;
    uint64_t* words;   /* [2][nl][2^logN] */
} fhe_wire_ct;
/* one step: n_in request ciphertexts in; fill out[0..*n_out) with 1 <= *n_out <= n_in.  out[i].words
 * has room for the words of in[i] only, so output i must keep in[i].logN and at most in[i].nl limbs;
 * the loop answers a request whose outputs break this with resp.<N>.error (the callback itself must
 * not write past that room).  reset != 0: a new session.  Returns FHE_OK or a status (message via
 * fhe_last_error).  Request meta fields of the reference (ringDim, level, interleave, packTokens) are
 * checked when present; lanes, tokensReal, dpad and packTokens are echoed in resp.<N>.meta. */
typedef int (*fhe_serve_step_fn)(void* user, int reset, int n_in, const fhe_wire_ct* in, int* n_out,
                                 fhe_wire_ct* out);
int fhe_serve_files(const char* dir, int timeout_ms, int max_requests, fhe_serve_step_fn step, void* user,
                    int* served);
/* the serve loop over fhe_server_step of model m (one pack per request) */
int fhe_serve_model(fhe_model* m, const char* dir, int timeout_ms, int max_requests, int* served);

/* ---- key material: seeded part files and the rotation-index contract --------------------
 * Part files follow the reference's FSSMSKY1 format (hpc_gpu_port/seeded_keys.hpp:44-52; written
 * by writeSeededPart :327-349, read by readSeededPartHeader :354-370 and expandSeededKeys
 * :382-420): a header with the ring, chain and digit layout, then per key its automorphism index,
 * the 32-byte seed of its a-halves and its b-halves [numPartQ][sizeQ + sizeP][N] in evaluation
 * form.  Index 0 carries the relinearisation key (this engine's extension).  The a-halves are
 * re-expanded from the seeds on the device when a file is loaded. */
typedef struct {
    uint32_t version, expander, N, sizeQ, sizeP, numPartQ, numPerPartQ, count;
} fhe_part_layout;
/* header of a part file (no GPU needed): moduli[sizeQ + sizeP] and the key tag when non-NULL */
int fhe_part_header(const char* path, fhe_part_layout* lay, uint64_t* moduli, int moduli_cap, char* tag, int tag_cap);
/* write a part file from caller-held words (no GPU needed): lay->count records of indices[k],
 * seeds[k][32], b[k][numPartQ][sizeQ + sizeP][N] */
int fhe_part_write_words(const char* path, const fhe_part_layout* lay, const uint64_t* moduli, const char* tag,
                         const uint32_t* indices, const uint8_t* seeds, const uint64_t* b);
/* write the context's keys `which[0..n)` (0 = relinearisation, else automorphism indices); every one
 * must have been generated from a seed in this context (replaces writeSeededPart) */
int fhe_keys_save_part(fhe_ctx* cx, const char* path, const uint64_t* which, int n, const char* tag);
/* load a part file minted for this context's chain (else FHE_ERR_ARG, as the reference's loader
 * refuses): b words from the file, a-halves expanded from the seeds on the device; keys the context
 * already holds are kept; *inserted = keys added (replaces expandSeededKeys + LoadContext) */
int fhe_keys_load_part(fhe_ctx* cx, const char* path, int* inserted);
/* the rotation-index contract of a model ("fhe-ssm-rot-indices-v1", the --dump-rot-indices JSON of
 * gpu_real_model.cu:1337-1394): rotationAmounts, bootstrapSteps, and autoIndices = every
 * automorphism index the server will look up (5^s mod 2N, and 2N - 1) */
int fhe_model_rot_contract(const fhe_model* m, char* buf, int cap);

/* ---- raw words (parity tests, serialisation) -------------------------------------------- */
int fhe_ct_import(fhe_ctx* cx, const uint64_t* words, int level, double scale, fhe_ct** out);
int fhe_ct_export(fhe_ctx* cx, const fhe_ct* ct, uint64_t* words);
int fhe_pt_import(fhe_ctx* cx, const uint64_t* words, int level, double scale, fhe_pt** out);
int fhe_pt_export(fhe_ctx* cx, const fhe_pt* pt, uint64_t* words);
/* forward / inverse NTT of n limb-polynomials in host memory; mod_idx[i] names the modulus
 * (0..L-1: q_i, L..L+K-1: p_{i-L}) of polynomial i */
int fhe_ntt_host(fhe_ctx* cx, uint64_t* words, int n, const int* mod_idx, int inverse);
/* key switching of one polynomial (limbs = L - level, eval form) with a raw key
 * ([digit][2][L+K][N], canonical) -> out0, out1 (same limbs) */
int fhe_keyswitch_host(fhe_ctx* cx, const uint64_t* d, int level, const uint64_t* key, uint64_t* out0,
                       uint64_t* out1);

/* ---- limb-partitioned key switching over several GPUs (single-pack latency) -------------
 * Replaces the reference's multi-device context (gpu_real_model.cu:847-884 --devices; FIDESlib's
 * limb placement :995-997 and SetDevices :1158-1161).  Rank g of `world` owns a block of the Q
 * limbs and of the K special limbs of every polynomial: per = ceil(n / world) limbs, rank g the
 * limbs [g per, (g + 1) per) that exist (fhe_dist_limbs gives its Q block).  A key switch
 * all-gathers the ranks' Q limbs of d in coefficient form before ModUp and their special limbs of
 * the inner products before ModDown (NCCL, on the context's own communication stream); all other
 * work stays on the rank's limbs, and every rank's limbs equal the single-GPU key switch's. */
/* an NCCL unique id (128 bytes): rank 0 makes it and shares it with the other ranks */
int fhe_dist_unique_id(uint8_t* out);
/* join a group of `world` ranks (one context per GPU, same chain and keys) */
int fhe_dist_init(fhe_ctx* cx, int world, int rank, const uint8_t* id);
/* this rank's block of the L - level Q limbs: *first, *count (count may be 0) */
int fhe_dist_limbs(const fhe_ctx* cx, int level, int* first, int* count);
/* key switch with the resident key `which` (0 = relinearisation, else an automorphism index):
 * d_own = the rank's Q limbs of d (eval form, device memory, [count][N]) -> out0, out1, the rank's
 * limbs of the result (device memory).  Every rank of the group must call it (a collective),
 * enqueued on the context's stream. */
int fhe_keyswitch_dist(fhe_ctx* cx, uint64_t which, const uint64_t* d_own, int level, uint64_t* out0,
                       uint64_t* out1);

/* ---- key switching without device allocation -------------------------------------------
 * No counterpart in the reference (its key switch allocates through OpenFHE / FIDESlib).
 * For callers that must not allocate device memory during a pass: a server that has given
 * nearly all HBM to long-lived arenas (resident conversations' state, keys, plaintexts), or a
 * host runtime whose own pool owns the device.  Key-switches d (device memory, limbs =
 * L - level, eval form) with the context's resident key `which` (0 = relinearisation, else
 * an automorphism index from fhe_rot_index) into out0, out1 (device memory, same limbs);
 * enqueued on the context's stream (fhe_ctx_stream), results bit-identical to
 * fhe_keyswitch_host.  Working memory is a static 64 MiB device array per GPU
 * (FHE_NOALLOC_SCRATCH_MIB): at N = 2^16, K = 4, alpha = 4 at most 16 limbs; larger requests
 * return FHE_ERR_ARG.  Overlapping calls on one GPU (different contexts or threads) race on
 * that array.  The first call on a GPU does the set-up; make it before any stream capture (a
 * failed set-up returns an error and is retried by the next call).
 * Per-kernel profiling must be off. */
#define FHE_NOALLOC_SCRATCH_MIB 64
int fhe_keyswitch_noalloc(fhe_ctx* cx, uint64_t which, const uint64_t* d, int level, uint64_t* out0,
                          uint64_t* out1);

#ifdef __cplusplus
}
#endif
#endif
