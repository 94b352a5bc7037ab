// engine.h -- the B200 CKKS evaluation engine: context, device objects and operations.
//
// One Context owns one CUDA device and one stream.  Every ciphertext / plaintext / key
// lives in that device's HBM; the host only drives launches.  Words are uint64 residues
// (canonical, [0, q)).  Layouts:
//   polynomial with nl limbs : [limb][N]                     (limb i uses modulus q_i)
//   ciphertext               : 2 polynomials, poly p at d + p * stride
//   extended basis Q_l u P   : limbs 0..nl-1 are q_0..q_{nl-1}, then the K special primes
//   switching key            : [digit][2 (b, a)][L + K][N], Montgomery form (x * 2^64 mod q)
#pragma once
#include <cuda_runtime.h>

#include <complex>
#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "modarith.cuh"

namespace fhe {

struct Error : std::runtime_error {
    int code;
    explicit Error(const std::string& s, int c = -1) : std::runtime_error(s), code(c) {}
};

#define CUDA_CHECK(x)                                                                            \
    do {                                                                                         \
        cudaError_t err__ = (x);                                                                 \
        if (err__ != cudaSuccess)                                                                \
            throw ::fhe::Error(std::string("CUDA error: ") + cudaGetErrorString(err__) + " at " + \
                                   __FILE__ + ":" + std::to_string(__LINE__),                    \
                               -3);                                                              \
    } while (0)

constexpr int kMaxMod = 64;
constexpr int kMaxDevices = 64;

// constant-memory copy of every modulus' constants (index: Q chain then P chain)
// defined once: the library is one translation unit (fhessm.cu)
__constant__ ModConst c_mod[kMaxMod];

// Which limbs a batched kernel walks: count = npoly * nl limb-polynomials.
struct LimbMap {
    uint64_t* base;
    long long poly_stride;   // words between consecutive polynomials
    int nl;                  // limbs per polynomial
    int skip_alpha;          // >0: skip limbs [dg*alpha, min(dg*alpha+alpha, skip_nq)) (ModUp own digit),
    int skip_nq;             //     dg = poly, or poly % skip_period for a batch of ModUp outputs
    int skip_period;
    // modulus index of limb l: l < split ? l + off0 : l - split + off1
    int split, off0, off1;
    __host__ __device__ int mod(int l) const { return l < split ? l + off0 : l - split + off1; }
};

struct Params {
    int logN = 16;
    int L = 20;        // Q limbs at the top level
    int K = 4;         // special primes
    int alpha = 4;     // limbs per key-switching digit
    int q0bits = 60, qbits = 45, pbits = 60;
    int hw = 192;      // secret Hamming weight (0: uniform ternary)
    double sigma = 3.19;
    int device = 0;
    int boot_primes = 0;   // top limbs drawn as boot_bits-bit primes (the levels a bootstrap consumes)
    int boot_bits = 58;
};

struct Context;

// ---- device objects -------------------------------------------------------------------
struct DevBuf {
    uint64_t* p = nullptr;
    size_t words = 0;
    cudaStream_t st = nullptr;
    DevBuf() = default;
    DevBuf(size_t w, cudaStream_t s);
    ~DevBuf();
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept { *this = std::move(o); }
    DevBuf& operator=(DevBuf&& o) noexcept;
};

struct Ciphertext {
    DevBuf buf;
    int nl = 0;            // current limb count
    size_t stride = 0;     // words between c0 and c1
    double scale = 1.0;
    uint64_t* c(int p) const { return buf.p + (size_t)p * stride; }
};

struct Plaintext {
    DevBuf buf;            // [nl][N] eval form (or [nl][N/rep] when compressed)
    int nl = 0;
    double scale = 1.0;
    int log_rep = 0;       // >0: REP-periodic compressed plaintext, word i of a limb = comp[i >> log_rep]
};

struct SwitchKey {
    DevBuf buf;            // [dnum_top][2][L+K][N], Montgomery form
    uint64_t index = 0;    // automorphism index (0 for relinearisation)
    uint8_t seed[32] = {0};   // the a-halves' expander seed (seeded keys: part files carry it)
    bool seeded = false;
    DevBuf fwd;            // rotation keys: the same key with the automorphism applied (the key
                           // of the rotate-then-switch order), built on first use by rotate_sum
};

// ---- context ----------------------------------------------------------------------------
struct Context {
    Params prm;
    int logN = 0, N = 0, L = 0, K = 0, alpha = 0, dnum_top = 0;
    std::vector<uint64_t> mods;      // L + K
    std::vector<ModConst> mc;
    std::vector<uint64_t> psi;       // minimal primitive 2N-th roots
    std::vector<double> scale_at;    // FLEXIBLEAUTO-style scaling factor by limb count (index nl)
    cudaStream_t stream = nullptr;
    int device = 0;
    uint64_t *d_tw = nullptr, *d_twp = nullptr, *d_itw = nullptr, *d_itwp = nullptr, *d_ninv = nullptr;
    uint64_t *d_tw2 = nullptr, *d_itw2 = nullptr;   // the same tables as (twiddle, Shoup) pairs for the NTT kernels
    uint64_t *d_twrow = nullptr, *d_itwrow = nullptr;   // last-four-stage twiddles in the row kernel's access order
    uint64_t* d_rmont = nullptr;     // [L+K][2]: 2^64 mod q (+ Shoup), the factor into Montgomery form
    // ModDown / rescale constants (level independent): see build_tables()
    uint64_t* d_md = nullptr;        // ModDown: [K] phatinv (+shoup), [L][K] phat mod q_i (+shoup), [L] Pinv (+shoup)
    uint64_t* d_rs = nullptr;        // rescale: [L][L] (ql mod qi, ql^-1 mod qi, shoup)
    unsigned int* d_err = nullptr;   // set by a kernel whose bounded wait ran out (checked at syncs)
    int use_tc = 1;                  // BSGS products on the tensor cores (tcgen05) where the shape allows
    int use_pdl = 1;                 // programmatic dependent launch for the hot kernels (launch_pdl)
    int ntt_cluster = 0;             // N = 2^16: one cluster launch per transform (ntt.cu, k_ntt_cluster)
    int baby_limbs = 8;              // k_baby_pq: limbs walked by one thread
    int boot_compress = 1;           // bootstrap_setup: slot-periodic level plaintexts stored compressed
    int ntt_arith = 1;               // NTT butterflies: 1 cheaper Shoup quotient in 32-bit steps (ntt.cu, mul_shoup_q4), 0 exact
    int merged_rescale = 1;          // circuit products: ModDown and rescale in one division by P q_l
    // bootstrap input scale: the message is brought to one limb (q0) at scale 2^boot_delta_log2.
    // q0 / scale is the factor by which SlotToCoeff amplifies the error of EvalMod's output, and
    // 2 pi |m| scale / q0 the argument whose sine EvalMod returns in place of it (relative error
    // (2 pi |m| scale / q0)^2 / 6 on the largest coefficients).  0 (default): scale = 2^(bits(q0)
    // - 11), 2^49 for a 60-bit q0 (17.7 bits on U[-1, 1] slots at N = 2^16 against 13.8 at the
    // canonical scale; 1.5e-5 on constant slots of magnitude 2); -1: the chain's canonical
    // level-1 scale; read by bootstrap_setup
    int boot_delta_log2 = 0;
    // BSGS plaintext cache (the reference's --cache-diags, gpu_real_model.cu:1647-1652, off by
    // default as there): a plan keeps the plaintext words of its last call while at least
    // pt_cache_reserve_mib of device memory stays free
    int pt_cache = 0;
    long long pt_cache_reserve_mib = 24 * 1024;
    long long pt_cache_bytes = 0;    // held by the plans of this context
    std::map<int, uint64_t*> modup_tab;   // per nl: [dnum][alpha][2] qhat^-1, [dnum][ne][alpha][2] qhat mod t
    std::map<int, uint64_t*> mdr_tab;     // per nl: ModDown + rescale in one step (ct_mul_relin_rescale)
    // keys
    DevBuf sk;                       // secret, eval form over all L+K moduli, [L+K][N]
    std::vector<int8_t> sk_coeff;    // signed coefficients (client side)
    DevBuf pk;                       // [2][L][N]
    std::unique_ptr<SwitchKey> rlk;
    std::map<uint64_t, std::unique_ptr<SwitchKey>> rot_keys;   // by automorphism index
    uint8_t master[32] = {0};
    uint32_t enc_counter = 0;
    mutable long long launches = 0;  // kernel launches issued (for the launch count claim)
    long long ks_count = 0, ks_limbs = 0;   // key switches issued and the sum of their limb counts
    long long pt_encodes = 0;        // plaintexts encoded on an encode-cache miss
    long long host_waits = 0;        // uploads that waited for a staging slot still in flight
    // Pinned host staging for uploads on the hot path (upload_async): kStageSlots slots of
    // kStageBytes, used round robin; slot i is reused once the event recorded after its copy
    // has completed, so an upload never waits for the stream's other work.
    static constexpr int kStageSlots = 8;
    static constexpr size_t kStageBytes = (size_t)1 << 20;
    uint8_t* stage = nullptr;
    cudaEvent_t stage_ev[kStageSlots] = {};
    int stage_next = 0;
    // optional per-kernel CUDA-event timing (bench roofline): name -> pending event pairs
    // Sampled: one scope in prof_every of each name is timed; the totals are scaled by
    // seen / sampled (the average duration of a timed scope is exact for what was timed).
    struct ProfEntry {
        std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pending;
        long long seen = 0, sampled = 0;
        double ms = 0.0, bytes = 0.0;
        double ops = 0.0;   // tensor-core kernels: int8 multiply-accumulates issued (0 for the others)
    };
    bool prof = false;
    int prof_every = 1;
    void check_device_error();
    // Makes this context's moduli the ones in the device's constant table c_mod (one table per
    // device, shared by every context on it): when another context with a different chain wrote
    // it last, the device is synchronised and the table rewritten.  Every C-ABI entry calls it.
    void activate();
    mutable std::map<std::string, ProfEntry> prof_acc;
    std::unique_ptr<Plaintext> pt_i;         // NTT of X^{N/2}: multiplication by i
    std::map<uint64_t, std::shared_ptr<Plaintext>> ptcache;   // encode_cached: (content, level, scale)
    std::shared_ptr<void> boot;              // bootstrapping precomputation (bootstrap.cu)
    std::shared_ptr<void> dist;              // limb-partitioned group: NCCL communicator and stream (dist.cu)

    explicit Context(const Params& p);
    ~Context();
    Context(const Context&) = delete;

    int dnum(int nl) const { return (nl + alpha - 1) / alpha; }
    int ext_mod(int nl, int e) const { return e < nl ? e : L + (e - nl); }
    const uint64_t* modup_table(int nl);
    const uint64_t* mdr_table(int nl);
    LimbMap qmap(uint64_t* base, int nl, long long poly_stride) const;
    LimbMap extmap(uint64_t* base, int nl, long long poly_stride) const;   // Q_l u P
};

enum EwOp : int { EW_ADD = 0, EW_SUB = 1, EW_MULPT = 2, EW_ADDPT = 3, EW_NEG = 4 };

// per-limb constants passed by value to k_mul_const (1.5 KB of kernel parameters)
struct LimbConst {
    uint64_t w[kMaxMod], wp[kMaxMod], add[kMaxMod];
    int has_w, has_add;
};
// out = a * w (+ add on c0), limb-wise; out may alias a
void apply_limb_const(Context& cx, const Ciphertext& a, const LimbConst& k, Ciphertext& out);
// round(v) mod q_i for each limb (|v| < 2^126)
void limb_residues(const Context& cx, long double v, int nl, uint64_t* out);
Plaintext encode_pq(Context& cx, const std::complex<double>* z, int nslots, int nl, double scale);
// host -> device copy of `bytes` (<= Context::kStageBytes) through a pinned staging slot, ordered
// on the context's stream: the host buffer may be reused as soon as the call returns, and the
// stream is not drained (a pageable-memory copy would wait for all earlier work first)
void upload_async(Context& cx, void* dev, const void* host, size_t bytes);

// Brackets the launches of one kernel (or kernel pair) with CUDA events on the context's
// stream when profiling is on; `bytes` is the algorithmic DRAM traffic of the bracket.
struct ProfScope {
    const Context& cx;
    cudaEvent_t a = nullptr, b = nullptr;
    const char* name;
    double bytes;
    bool timed = false;
    ProfScope(const Context& c, const char* n, double by, double ops = 0.0) : cx(c), name(n), bytes(by) {
        if (!cx.prof) return;
        auto& e = cx.prof_acc[name];
        timed = (e.seen++ % std::max(1, cx.prof_every)) == 0;
        e.bytes += bytes;
        e.ops += ops;
        if (!timed) return;
        cudaEventCreate(&a);
        cudaEventCreate(&b);
        cudaEventRecord(a, cx.stream);
    }
    ~ProfScope() {
        if (!timed) return;
        cudaEventRecord(b, cx.stream);
        auto& e = cx.prof_acc[name];
        e.pending.emplace_back(a, b);
        e.sampled++;
    }
};

// ---- programmatic dependent launch ------------------------------------------------------
// A kernel launched by launch_pdl may be scheduled while the previous kernel on the stream is
// still running: its CTAs start, run pdl_wait() -- which returns once the previous grid has
// completed and its writes are visible -- and only then touch memory.  Every kernel launched this
// way calls pdl_wait() before its first global load or store; pdl_trigger() lets the next grid be
// scheduled as soon as all of this grid's CTAs have started.  For a kernel launched the ordinary
// way both are no-ops.  What is gained is the gap between dependent kernels (scheduling the next
// grid, its CTAs' start-up), which dominates the short launches of small batches.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" :::); }

template <typename... P, typename... A>
inline void launch_pdl(const Context& cx, void (*k)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       A&&... args);

// ---- low-level launches (ntt.cu, kernels.cu, keys.cu) --------------------------------------
void expand_uniform_dev(Context& cx, const uint8_t seed[32], int digit0, int ndigit, int limb0, int nlimb,
                        uint32_t tag, uint64_t* out, long long digit_stride);
void ntt(const Context& cx, const LimbMap& mp, int npoly, bool inv, cudaStream_t st);
// rescale by the last of l + 1 limbs, the dropped limbs already inverse-transformed in place (ntt.cu)
void ntt_rescale(const Context& cx, uint64_t* a, long long stride, int l, uint64_t* y, cudaStream_t st);
constexpr int kFuseMax = 16;   // polynomials of one fused rescale transform (ntt_rescale_n)
void ntt_rescale_n(const Context& cx, const uint64_t* src, long long src_stride, uint64_t* const* dst, int npoly,
                   int l, uint64_t* y, cudaStream_t st);

// ---- operations (engine.cu) ---------------------------------------------------------------
// key switching of d (nl limbs, eval) -> (out0, out1) added into add0/add1 (may be null),
// then permuted by the automorphism `perm_k` (1 = identity).  out may alias add.
void keyswitch(Context& cx, const uint64_t* d, int nl, const SwitchKey& key, const uint64_t* add0,
               const uint64_t* add1, uint64_t* out0, uint64_t* out1, uint64_t perm_k);

Ciphertext ct_alloc(Context& cx, int nl);
Ciphertext ct_copy(Context& cx, const Ciphertext& a);
void ct_add(Context& cx, const Ciphertext& a, const Ciphertext& b, Ciphertext& out);
void ct_sub(Context& cx, const Ciphertext& a, const Ciphertext& b, Ciphertext& out);
void ct_add_raw(Context& cx, const Ciphertext& a, const Ciphertext& b, Ciphertext& out);
void ct_mul_pt(Context& cx, const Ciphertext& a, const Plaintext& pt, Ciphertext& out);
void ct_add_pt(Context& cx, const Ciphertext& a, const Plaintext& pt, Ciphertext& out);
void ct_mul_relin(Context& cx, const Ciphertext& a, const Ciphertext& b, Ciphertext& out);
// a * b, relinearised and rescaled with one division by P q_l (ModDown and rescale merged):
// nl - 1 limbs out; not bit-identical to ct_mul_relin + ct_rescale (one rounding instead of two)
void ct_mul_relin_rescale(Context& cx, const Ciphertext& a, const Ciphertext& b, Ciphertext& out);
void ct_mul_relin_rescale_n(Context& cx, const Ciphertext* const* a, const Ciphertext* const* b, int B,
                            Ciphertext* out);
void ct_rescale(Context& cx, Ciphertext& a);
void ct_rescale_n(Context& cx, Ciphertext* const* a, int K);   // K rescales of one limb count, batched
void ct_level_drop(Context& cx, Ciphertext& a, int nl_target);   // drop limbs, no scaling
void ct_automorph(Context& cx, const Ciphertext& a, uint64_t k, Ciphertext& out);
// out = extra + sum_b rot((c0s[b], c1s[b]), steps[b]) for n inputs of nl limbs at `scale`
// (no zero steps; extra0/extra1 may be null): one batched ModUp, the inner products summed
// in QP, one ModDown (ksbatch.cu)
void rotate_sum(Context& cx, const uint64_t* const* c0s, const uint64_t* const* c1s, const int* steps, int n,
                int nl, double scale, const uint64_t* extra0, const uint64_t* extra1, Ciphertext& out);
void ct_rotate(Context& cx, const Ciphertext& a, int r, Ciphertext& out);
void ct_conjugate(Context& cx, const Ciphertext& a, Ciphertext& out);
void ct_rotate_hoisted(Context& cx, const Ciphertext& a, const int* rs, int n, Ciphertext* outs);
void ct_mul_const(Context& cx, const Ciphertext& a, double v, double scale, Ciphertext& out);  // by round(v*scale)
void ct_add_const(Context& cx, const Ciphertext& a, double v, Ciphertext& out);
void ct_mul_int(Context& cx, const Ciphertext& a, int64_t v, Ciphertext& out);

// encoding (host special FFT + device reduction/NTT)
Plaintext encode(Context& cx, const std::complex<double>* z, int nslots, int nl, double scale);
void decode(Context& cx, const Plaintext& pt, std::complex<double>* z);
// client-side crypto (keys held by the context)
void keygen(Context& cx, const uint8_t seed[32]);
void keygen_rotations(Context& cx, const int* rs, int n, bool conj);
void keygen_auto(Context& cx, const uint64_t* ks, int n);   // keys for automorphism indices
uint64_t rot_index(const Context& cx, int r);
Ciphertext encrypt(Context& cx, const Plaintext& pt);
Plaintext decrypt(Context& cx, const Ciphertext& ct);

// circuit layer (circuit.cu)
double canon(const Context& cx, int nl);
void mul_integer(Context& cx, const Ciphertext& a, long double M, Ciphertext& out);
void mul_integer_add_const(Context& cx, const Ciphertext& a, long double M, double v, Ciphertext& out);
void mul_const_rescale(Context& cx, const Ciphertext& a, double c, Ciphertext& out, double target = 0);
void align(Context& cx, Ciphertext& a, int nl_t, double target = 0);
void align_n(Context& cx, Ciphertext* const* a, int K, int nl_t, double target = 0);
void mul_const_rescale_n(Context& cx, const Ciphertext* const* a, const double* c, int K, Ciphertext* out,
                         double target = 0);
void mul_vec_rescale_n(Context& cx, const Ciphertext* const* a, const std::complex<double>* const* v, int n, int K,
                       Ciphertext* out, double target = 0);
void match(Context& cx, Ciphertext& a, Ciphertext& b);
void add_any(Context& cx, const Ciphertext& a, const Ciphertext& b, Ciphertext& out);
void sub_any(Context& cx, const Ciphertext& a, const Ciphertext& b, Ciphertext& out);
void mul_rescale(Context& cx, const Ciphertext& a, const Ciphertext& b, Ciphertext& out);
void mul_vec_rescale(Context& cx, const Ciphertext& a, const std::complex<double>* v, int n, Ciphertext& out,
                     double target = 0);
void add_vec(Context& cx, const Ciphertext& a, const std::complex<double>* v, int n, Ciphertext& out);
void mul_i(Context& cx, const Ciphertext& a, Ciphertext& out);
void split_complex(Context& cx, const Ciphertext& z, Ciphertext& re, Ciphertext& im, bool halve = true);
void merge_complex(Context& cx, Ciphertext re, Ciphertext im, Ciphertext& z);
void rotate_sum(Context& cx, const Ciphertext& a, int step, int count, Ciphertext& out);
void cheb_eval(Context& cx, const Ciphertext& x, const std::vector<double>& coeffs, Ciphertext& out);
std::vector<double> cheb_fit(double (*f)(double, const void*), const void* arg, double a, double b, int n);
void poly_eval_vec(Context& cx, const Ciphertext& x, const std::vector<std::vector<std::complex<double>>>& c, int n,
                   Ciphertext& out);
void poly_eval_vec_n(Context& cx, const Ciphertext* const* xs, int K,
                     const std::vector<std::vector<std::complex<double>>>* const* cs, int n, Ciphertext* outs);
void mul_rescale_n(Context& cx, const Ciphertext* const* a, const Ciphertext* const* b, int K, Ciphertext* out);
// encode with a cache keyed by (content, slots, level, scale); periodic vectors (n < N/2)
// are stored compressed (matvec.cu)
const Plaintext& encode_cached(Context& cx, const std::complex<double>* z, int n, int nl, double scale);
// BSGS matvec (matvec.cu)
struct MatvecPlan;
std::shared_ptr<MatvecPlan> matvec_plan(Context& cx, const double* W, int rows, int cols, int D, int b1);
std::vector<int> matvec_rotations(int D, int b1);
void encode_periodic_words(Context& cx, const std::complex<double>* z, int period, int count, int nl, double scale,
                           uint64_t* host_out);
void matvec(Context& cx, const MatvecPlan& pl, const Ciphertext* const* us, Ciphertext& out);
struct BabySet;
void matvec_babies(Context& cx, const Ciphertext& u, int D, int b1, BabySet& bs);
void matvec_apply(Context& cx, const MatvecPlan& pl, const BabySet* const* sets, Ciphertext& out);
// model (model.cu)
struct Model;
struct ModelCfg;
// bootstrapping (bootstrap.cu)
std::vector<int> boot_rotations(const Context& cx);
void bootstrap_setup(Context& cx, double B, int deg, int r = 3);
void bootstrap(Context& cx, const Ciphertext& in, Ciphertext& out);
void bootstrap_upto(Context& cx, const Ciphertext& in, Ciphertext& out, int upto);
int bootstrap_levels_after(const Context& cx);

template <typename... P, typename... A>
inline void launch_pdl(const Context& cx, void (*k)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       A&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = cx.use_pdl ? 1 : 0;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    CUDA_CHECK(cudaLaunchKernelEx(&cfg, k, std::forward<A>(args)...));
}

// raw access (parity tests)
void upload(Context& cx, uint64_t* dst, const uint64_t* src, size_t words);
void download(Context& cx, uint64_t* dst, const uint64_t* src, size_t words);
void key_to_mont(Context& cx, uint64_t* key, bool to_mont);   // in place, [dnum_top][2][L+K][N]

}  // namespace fhe
