// bootstrap.cu -- full-slot CKKS bootstrapping (replaces EvalBootstrap, gpu_real_model.cu
// :2535-2556, whose refresh rule is :2573-2599).
//
// Pipeline (baseline config 3): ModRaise -> CoeffToSlot (3 merged FFT levels) -> split into
// real / imaginary parts -> EvalMod (degree-59 Chebyshev interpolant of a scaled cosine + 3
// double-angle steps) -> merge -> SlotToCoeff (3 merged FFT levels).
//
//  * ModRaise: the ciphertext is reduced to the first modulus q0 and its centred residues are
//    lifted to all L limbs, so it decrypts to t = m + q0 I with |I| small (sparse secret).
//  * CoeffToSlot evaluates (1/n) Stages_inv, the special FFT's inverse without its final
//    bit reversal (slot order stays bit-reversed; EvalMod is slot-wise so the order is free)
//    and SlotToCoeff evaluates Stages_fwd, the forward special FFT without its initial bit
//    reversal.  15 butterfly stages are merged into 3 levels of 5 stages: each level is a
//    sum of at most 63 rotated diagonals, evaluated by baby-step / giant-step (7 hoisted
//    babies, 7 giants).  CoeffToSlot keeps the ciphertext at scale q0 (the plaintext scale of
//    each level is the level's prime), so its plaintexts carry 45 bits of precision.
//  * EvalMod: with y = t / q0, sin(2 pi y) = cos(2 pi (y - 1/4)) is computed as the 8-fold
//    angle of cos(2 pi (y - 1/4) / 8), whose Chebyshev interpolant on [-B, B] is degree 59.
//    sin(2 pi y) ~ 2 pi m / q0; the factor q0 / (2 pi Delta) is folded into SlotToCoeff.
#include <cmath>
#include <set>

#include "engine.h"

namespace fhe {

constexpr int kDiagMax = 16;   // babies / giants of one bootstrap linear-transform level
// Baby steps of a linear-transform level.  Every level is a sum of at most 63 rotated diagonals
// (offsets -31..31 times the level's base): b1 = 16 gives 15 babies and 4 giants.  The babies
// stay in QP (double hoisting: one ModUp, no ModDown per baby), the diagonal products run over
// the extended basis, and only the 4 giant inputs are brought down to Q before their rotations.
constexpr int kBootB1 = 16;

// circuit.cu
double canon(const Context& cx, int nl);
void align(Context& cx, Ciphertext& a, int nl_t, double target);
void split_complex(Context& cx, const Ciphertext& z, Ciphertext& re, Ciphertext& im, bool halve);
void merge_complex(Context& cx, Ciphertext re, Ciphertext im, Ciphertext& z);
void cheb_eval(Context& cx, const Ciphertext& x, const std::vector<double>& coeffs, Ciphertext& out);
void cheb_eval_n(Context& cx, const Ciphertext* const* x, int K, const std::vector<double>& coeffs, Ciphertext* out);
int cheb_depth(const std::vector<double>& coeffs);
void mul_rescale_n(Context& cx, const Ciphertext* const* a, const Ciphertext* const* b, int K, Ciphertext* out);
std::vector<double> cheb_fit(double (*f)(double, const void*), const void* arg, double a, double b, int n);
void mul_integer(Context& cx, const Ciphertext& a, long double M, Ciphertext& out);
void mul_integer_add_const(Context& cx, const Ciphertext& a, long double M, double v, Ciphertext& out);
void mul_rescale(Context& cx, const Ciphertext& a, const Ciphertext& b, Ciphertext& out);
__global__ void k_rescale_lift(const uint64_t*, uint64_t*, int, int, int);

using cvec = std::vector<std::complex<double>>;
using Diags = std::map<int, cvec>;   // signed rotation offset -> diagonal

static cvec rotv(const cvec& d, int s) {   // rot(d, s)[p] = d[(p + s) mod n]
    const int n = (int)d.size();
    cvec r(n);
    for (int p = 0; p < n; p++) r[p] = d[((p + s) % n + n) % n];
    return r;
}
static int signed_off(int o, int n) {
    o = ((o % n) + n) % n;
    return o > n / 2 ? o - n : o;
}

// one butterfly stage of the special FFT as three diagonals (offsets 0, +lenh, -lenh)
static Diags stage(int n, int M, int len, bool inverse) {
    const int lenh = len / 2, lenq = len * 4, gap = M / lenq;
    std::vector<uint64_t> rg(n);
    uint64_t g = 1;
    for (int j = 0; j < n; j++) { rg[j] = g; g = (g * 5) % (uint64_t)M; }
    cvec d0(n), dp(n), dm(n);
    for (int i = 0; i < n; i += len)
        for (int j = 0; j < lenh; j++) {
            const int p = i + j, p2 = i + j + lenh;
            if (!inverse) {
                const uint64_t idx = (rg[j] % (uint64_t)lenq) * (uint64_t)gap;
                const std::complex<double> w(std::cos(2 * M_PI * idx / M), std::sin(2 * M_PI * idx / M));
                d0[p] = 1.0; dp[p] = w;          // out[p]  = v[p] + w v[p+lenh]
                dm[p2] = 1.0; d0[p2] = -w;       // out[p2] = v[p] - w v[p2]
            } else {
                const uint64_t idx = ((uint64_t)lenq - (rg[j] % (uint64_t)lenq)) * (uint64_t)gap;
                const std::complex<double> w(std::cos(2 * M_PI * idx / M), std::sin(2 * M_PI * idx / M));
                d0[p] = 0.5; dp[p] = 0.5;        // out[p]  = (v[p] + v[p+lenh]) / 2
                dm[p2] = 0.5 * w; d0[p2] = -0.5 * w;   // out[p2] = (v[p] - v[p2]) w / 2
            }
        }
    // +lenh and -lenh coincide mod n when lenh = n/2: the two diagonals have disjoint
    // supports, so they are summed into one
    Diags D;
    D[0] = d0;
    for (auto* pr : {&dp, &dm}) {
        const int o = signed_off(pr == &dp ? lenh : -lenh, n);
        auto& dst = D[o];
        if (dst.empty()) dst.assign(n, 0.0);
        for (int p = 0; p < n; p++) dst[p] += (*pr)[p];
    }
    return D;
}

// (A o B): sum_{a,b} (A_a . rot(B_b, a)) at offset a + b
static Diags compose(const Diags& A, const Diags& B, int n) {
    Diags R;
    for (auto& a : A)
        for (auto& b : B) {
            const int o = signed_off(a.first + b.first, n);
            cvec rb = rotv(b.second, a.first);
            auto& dst = R[o];
            if (dst.empty()) dst.assign(n, 0.0);
            for (int p = 0; p < n; p++) dst[p] += a.second[p] * rb[p];
        }
    return R;
}

struct BootLevel {
    int base = 1, b1 = kBootB1;
    bool pq = true;   // plaintexts over QP (double-hoisted evaluation)
    int log_rep = 0;  // > 0: every plaintext is REP-compressed (its diagonals are slot-periodic)
    int nl_in = 0;
    double s_in = 0, s_out = 0;
    std::map<std::pair<int, int>, Plaintext> pts;   // (g, j) -> plaintext of rot(D_k, -g b1 base)
    std::vector<int> gs;                            // giant indices in use
};

struct BootCtx {
    double B = 24.0;
    int r = 3, deg = 59;
    std::vector<double> cheb;
    std::vector<BootLevel> cts;
    // SlotToCoeff plaintexts per (EvalMod output scale, folded relabel factor): a canonical
    // one-limb input is relabelled to delta_in, and the factor is folded into the first level's
    // constant so that its output lands on the canonical scale
    struct StcSet {
        double s_in = 0, relabel = 1;
        std::vector<BootLevel> levels;
    };
    std::vector<StcSet> stcs;
    int nl_top = 0;   // limbs of the ModRaise output
    int nl_stc = 0, nl_out = 0;
    double delta_in = 0;
};

struct CosArg {
    double B;
    int r;
};
// cos(2 pi (B x - 1/4) / 2^r): after r double angles, sin(2 pi B x)
static double cos_target(double x, const void* arg) {
    const CosArg* c = (const CosArg*)arg;
    return std::cos(2 * M_PI * (c->B * x - 0.25) / (double)(1 << c->r));
}

// rotation steps the bootstrap needs (babies j*base, giants g*b1*base).  SlotToCoeff's levels
// start at stage 0, 1 per, 2 per; CoeffToSlot's are cut from the top (logn - per, logn - 2 per,
// 0), which is the same split only when per divides logn (n = 2^12, 2^15): both sets of bases.
std::vector<int> boot_rotations(const Context& cx) {
    const int n = cx.N / 2;
    int logn = 0;
    while ((1 << logn) < n) logn++;
    std::set<int> r;
    const int per = (logn + 2) / 3;   // stages per level (5 at n = 2^15)
    std::set<int> los;
    for (int lv = 0; lv < 3; lv++) {
        if (lv * per < logn) los.insert(lv * per);                         // SlotToCoeff
        los.insert(std::max(0, logn - (lv + 1) * per));                    // CoeffToSlot
    }
    for (int lo : los) {
        const int base = 1 << lo;
        for (int j = 1; j < kBootB1; j++)
            if ((j * base) % n != 0) r.insert(j * base);
        for (int g = -32 / kBootB1; g < 32 / kBootB1; g++)
            if (g && (g * kBootB1 * base) % n != 0) r.insert(g * kBootB1 * base);   // a full turn needs no key
    }
    return std::vector<int>(r.begin(), r.end());
}

// the smallest power-of-two period of a slot vector (exact comparison: the entries of a
// periodic diagonal are computed by the same operations in every period)
static int slot_period(const cvec& d) {
    const int n = (int)d.size();
    int p = 1;
    for (;; p <<= 1) {
        if (p >= n) return n;
        bool ok = true;
        for (int i = p; i < n && ok; i++) ok = d[i] == d[i % p];
        if (ok) return p;
    }
}

// build one merged level (stages with lenh = 2^lo .. 2^hi-1) as BSGS plaintexts
static BootLevel build_level(Context& cx, int lo, int hi, bool inverse, int nl_in, double s_in, double s_out,
                             std::complex<double> fold) {
    const int n = cx.N / 2, M = 2 * cx.N;
    Diags D;
    bool first = true;
    if (inverse) {   // CoeffToSlot applies the largest lenh first
        for (int e = hi - 1; e >= lo; e--) {
            Diags S = stage(n, M, 2 << e, true);
            D = first ? S : compose(S, D, n);
            first = false;
        }
    } else {
        for (int e = lo; e < hi; e++) {
            Diags S = stage(n, M, 2 << e, false);
            D = first ? S : compose(S, D, n);
            first = false;
        }
    }
    BootLevel L;
    L.base = 1 << lo;
    L.b1 = kBootB1;
    L.pq = true;
    L.nl_in = nl_in;
    L.s_in = s_in;
    L.s_out = s_out;
    const double spt = s_out * (double)cx.mods[nl_in - 1] / s_in;
    // The diagonals of stages with lenh < 2^hi repeat every 2^hi slots (a stage's entries depend
    // on the slot's position in its block of 2 lenh).  Below the full slot count such a level's
    // plaintexts are stored compressed: 2P words per limb for period P, read at x >> log_rep.
    int period = 1;
    for (auto& kv : D) period = std::max(period, slot_period(kv.second));
    const bool comp = cx.boot_compress && period < n && period <= 4096 && period >= 8;
    std::set<int> gset;
    for (auto& kv : D) {
        const int o = kv.first;
        if (o % L.base) throw Error("bootstrap: merged offset not a multiple of the level base");
        const int k = o / L.base;
        const int g = (int)std::floor((double)k / L.b1), j = k - g * L.b1;
        cvec d = rotv(kv.second, -g * L.b1 * L.base);
        for (auto& x : d) x *= fold;
        Plaintext pt;
        if (comp) {
            // Montgomery form, over QP or Q (k_diag_mac accumulates 128-bit products, reduces once)
            pt = encode_periodic_ext(cx, d.data(), period, nl_in, spt, L.pq, true);
            L.log_rep = pt.log_rep;
        } else {
            pt = L.pq ? encode_pq(cx, d.data(), n, nl_in, spt) : encode(cx, d.data(), n, nl_in, spt);
            LimbMap mm = cx.extmap(pt.buf.p, nl_in, 0);
            if (!L.pq) { mm.nl = nl_in; mm.split = nl_in; }
            k_mont_map<<<dim3(cx.N / 256, mm.nl), 256, 0, cx.stream>>>(pt.buf.p, mm, cx.logN);
            CUDA_CHECK(cudaGetLastError());
        }
        L.pts.emplace(std::make_pair(g, j), std::move(pt));
        gset.insert(g);
    }
    L.gs.assign(gset.begin(), gset.end());
    if ((int)L.gs.size() > kDiagMax || L.b1 > kDiagMax) throw Error("bootstrap: level too wide for k_diag_mac", -1);
    return L;
}

// All giants of one linear-transform level in one pass over the babies:
// out_g[c][i][x] = sum_j pt_gj[i][x] * baby_j[c][i][x] (pt in Montgomery form, <= kDiagMax
// products per 128-bit sum: hi < q for words < 2^60).  A pair of threads shares slot x: the
// even thread takes babies 0..7, the odd one babies 8..15; the two partial sums are added with
// one shuffle and the even thread writes c = 0, the odd one c = 1.  grid (N / 128, nl).
struct DiagArgs {
    const uint64_t* b0[kDiagMax];
    const uint64_t* b1[kDiagMax];
    const uint64_t* pt[kDiagMax][kDiagMax];   // [g][j] or null; word x of limb i at [i][x >> lr]
    uint64_t* o0[kDiagMax];
    uint64_t* o1[kDiagMax];
    int nb, ng, lr;
};
__global__ void __launch_bounds__(256, 4) k_diag_mac(const DiagArgs a, int logN, int nq, int L) {
    constexpr int H = kDiagMax / 2;
    const int N = 1 << logN;
    const int x = blockIdx.x * (blockDim.x / 2) + (threadIdx.x >> 1);
    const int half = threadIdx.x & 1;
    const int i = blockIdx.y;   // limb: Q limbs below nq, then the special limbs
    const ModConst mc = c_mod[i < nq ? i : L + (i - nq)];
    const size_t w = (size_t)i * N + x;
    const size_t wp = ((size_t)i << (logN - a.lr)) + (x >> a.lr);   // the plaintext word of slot x
    const int j0 = half * H;
    uint64_t v0[H], v1[H];
#pragma unroll
    for (int j = 0; j < H; j++)
        if (j0 + j < a.nb) { v0[j] = a.b0[j0 + j][w]; v1[j] = a.b1[j0 + j][w]; }
    for (int g = 0; g < a.ng; g++) {
        u128acc s0{0, 0}, s1{0, 0};
#pragma unroll
        for (int j = 0; j < H; j++) {
            if (j0 + j >= a.nb || !a.pt[g][j0 + j]) continue;
            const uint64_t p = a.pt[g][j0 + j][wp];
            acc_mad32(s0, p, v0[j]);
            acc_mad32(s1, p, v1[j]);
        }
        // the partner's sum of the output this thread writes
        const uint64_t mlo = half ? s0.lo : s1.lo, mhi = half ? s0.hi : s1.hi;
        const uint64_t plo = __shfl_xor_sync(0xffffffffu, mlo, 1), phi = __shfl_xor_sync(0xffffffffu, mhi, 1);
        u128acc t = half ? s1 : s0;
        asm("add.cc.u64 %0, %0, %2;\n\taddc.u64 %1, %1, %3;" : "+l"(t.lo), "+l"(t.hi) : "l"(plo), "l"(phi));
        (half ? a.o1 : a.o0)[g][w] = redc(t.hi, t.lo, mc);
    }
}

// One linear-transform level: sum over the level's diagonals k of pt_k . rot(v, k base), by
// baby steps j and giant steps g (k = g b1 + j; the plaintexts carry the -g b1 base pre-rotation).
static void eval_level(Context& cx, const BootLevel& L, const Ciphertext& v, Ciphertext& out) {
    if (v.nl != L.nl_in) throw Error("bootstrap: level mismatch in linear transform", -4);
    const int N = cx.N, K = cx.K, nl = v.nl, ne = nl + K, dn = cx.dnum(nl);
    cudaStream_t st = cx.stream;
    const int nb = L.b1, nw = L.pq ? ne : nl;   // limbs of babies, plaintexts and products
    // babies: QP images P rot(v, j base) from one ModUp (L.pq), or Q rotations (hoisted)
    DevBuf bq;
    std::vector<Ciphertext> baby;
    std::vector<const uint64_t*> b0(nb), b1v(nb);
    if (L.pq) {
        bq = DevBuf((size_t)nb * 2 * ne * N, st);
        DevBuf ext = modup(cx, v.c(1), nl);
        BabyArgs ba{};
        for (int i = 0; i < nl; i++) {
            uint64_t pm = 1;
            for (int k = 0; k < K; k++) pm = host_mulmod(pm, cx.mods[cx.L + k] % cx.mods[i], cx.mods[i]);
            ba.pw[i] = pm;
            ba.pwp[i] = shoup_of(pm, cx.mods[i]);
        }
        for (int j = 0; j < nb; j++) {
            const uint64_t k = j == 0 ? 1 : rot_index(cx, j * L.base);
            ba.perm[j] = k;
            ba.fkey[j] = k == 1 ? nullptr : forward_key(cx, k);
        }
        {
            ProfScope ps(cx, "baby_pq", 8.0 * N * nb * ((double)dn * ne * 2 + 2 * ne));
            const int per = std::max(1, cx.baby_limbs);
            k_baby_pq<<<dim3(N / 256, (ne + per - 1) / per, nb), 256, 0, st>>>(ext.p, v.c(0), v.c(1), ba, bq.p, nl, ne,
                                                                           dn, cx.L, K, cx.logN, per);
            CUDA_CHECK(cudaGetLastError());
        }
        cx.launches++;
        cx.ks_count += nb - 1;
        cx.ks_limbs += (long long)(nb - 1) * nl;
        for (int j = 0; j < nb; j++) {
            b0[j] = bq.p + (size_t)j * 2 * ne * N;
            b1v[j] = b0[j] + (size_t)ne * N;
        }
    } else {
        std::vector<int> steps;
        for (int j = 1; j < nb; j++) steps.push_back(j * L.base);
        baby.resize(nb);
        baby[0] = ct_copy(cx, v);
        std::vector<Ciphertext> rs(steps.size());
        ct_rotate_hoisted(cx, v, steps.data(), (int)steps.size(), rs.data());
        for (size_t i = 0; i < rs.size(); i++) baby[i + 1] = std::move(rs[i]);
        for (int j = 0; j < nb; j++) { b0[j] = baby[j].c(0); b1v[j] = baby[j].c(1); }
    }
    // giant g: inner_g = sum_j pt_gj . baby_j (one k_diag_mac for all g)
    DiagArgs da{};
    da.nb = nb;
    da.lr = L.log_rep;
    for (int j = 0; j < nb; j++) { da.b0[j] = b0[j]; da.b1[j] = b1v[j]; }
    std::vector<int> gl;   // giants in use, in output order
    double spt = 0;
    for (int g : L.gs) {
        bool any = false;
        for (int j = 0; j < nb; j++) {
            auto it = L.pts.find(std::make_pair(g, j));
            if (it == L.pts.end()) continue;
            da.pt[gl.size()][j] = it->second.buf.p;
            spt = it->second.scale;
            any = true;
        }
        if (any) gl.push_back(g);
    }
    if (gl.empty()) throw Error("bootstrap: empty linear-transform level", -1);
    const int G = (int)gl.size();
    DevBuf inner((size_t)G * 2 * nw * N, st);
    for (int gi = 0; gi < G; gi++) {
        da.o0[gi] = inner.p + (size_t)gi * 2 * nw * N;
        da.o1[gi] = da.o0[gi] + (size_t)nw * N;
    }
    da.ng = G;
    {
        ProfScope ps(cx, "diag_mac", 8.0 * N * nw * (2.0 * nb + 2.0 * G + (double)L.pts.size() / (1 << L.log_rep)));
        k_diag_mac<<<dim3(N / 128, nw), 256, 0, st>>>(da, cx.logN, nl, cx.L);
        CUDA_CHECK(cudaGetLastError());
        cx.launches++;
    }
    // back to Q (QP path: one ModDown per giant input), then sum_g rot(inner_g, g b1 base)
    DevBuf innq;
    const uint64_t* iq = inner.p;
    if (L.pq) {
        innq = DevBuf((size_t)G * 2 * nl * N, st);
        moddown_many(cx, inner.p, G, nl, innq.p);
        iq = innq.p;
    }
    // giants whose rotation is the identity (g = 0, or a full turn of the slots) are summed
    // into the unrotated term
    std::vector<const uint64_t*> c0s, c1s, flat;
    std::vector<int> gsteps;
    for (int gi = 0; gi < G; gi++) {
        const uint64_t* p = iq + (size_t)gi * 2 * nl * N;
        const int step = gl[gi] * nb * L.base;
        if (rot_index(cx, step) == 1) { flat.push_back(p); continue; }
        c0s.push_back(p);
        c1s.push_back(p + (size_t)nl * N);
        gsteps.push_back(step);
    }
    DevBuf fsum;
    const uint64_t* g0 = flat.empty() ? nullptr : flat[0];
    if (flat.size() > 1) {
        fsum = DevBuf((size_t)2 * nl * N, st);
        ProfScope pe(cx, "ewise", 8.0 * N * nl * 2 * 3 * (double)(flat.size() - 1));
        const long long ps = (long long)nl * N;
        launch_pdl(cx, k_ewise, dim3(N / 256, nl, 2), dim3(256), 0, st, EW_ADD, flat[0], ps, flat[1], ps, fsum.p, ps, 0, cx.logN);
        for (size_t f = 2; f < flat.size(); f++)
            launch_pdl(cx, k_ewise, dim3(N / 256, nl, 2), dim3(256), 0, st, EW_ADD, fsum.p, ps, flat[f], ps, fsum.p, ps, 0, cx.logN);
        CUDA_CHECK(cudaGetLastError());
        cx.launches += (long long)flat.size() - 1;
        g0 = fsum.p;
    }
    Ciphertext acc;
    rotate_sum(cx, c0s.data(), c1s.data(), gsteps.data(), (int)gsteps.size(), nl, v.scale * spt, g0,
               g0 ? g0 + (size_t)nl * N : nullptr, acc);
    ct_rescale(cx, acc);
    acc.scale = L.s_out;
    out = std::move(acc);
}

void bootstrap_setup(Context& cx, double B, int deg, int r) {
    if (r < 1 || r > 8 || deg < 3) throw Error("bootstrap_setup: need degree >= 3 and 1..8 double angles", -1);
    auto bc = std::make_shared<BootCtx>();
    bc->B = B;
    bc->deg = deg;
    bc->r = r;
    const int n = cx.N / 2;
    int logn = 0;
    while ((1 << logn) < n) logn++;
    const int per = (logn + 2) / 3;
    // ModRaise lifts to all limbs but the top one: CoeffToSlot takes three levels and carries
    // the EvalMod argument's 1/(2B) in its last level, so the chain's top prime is not needed
    const int Lt = cx.L - 1;
    bc->nl_top = Lt;
    const double q0 = (double)cx.mods[0];
    // CoeffToSlot at scale q0 (each level's plaintext scale is its own prime); the last level
    // also carries the factor 1/(2B) of the EvalMod argument and lands on the canonical scale,
    // so no level is spent on that constant
    int nl = Lt;
    for (int lv = 0; lv < 3; lv++) {
        const int hi = logn - lv * per, lo = std::max(0, hi - per);
        const bool last = lv == 2;
        bc->cts.push_back(build_level(cx, lo, hi, true, nl, q0, last ? canon(cx, nl - 1) : q0,
                                      last ? 1.0 / (2.0 * B) : 1.0));
        nl--;
    }
    const int nl_em = nl;
    const CosArg ca{B, r};
    bc->cheb = cheb_fit(cos_target, &ca, -1.0, 1.0, deg);
    // EvalMod depth: the levels the Chebyshev evaluation of these coefficients takes (its
    // baby / giant / leaf tree, cheb_depth) + r double angles
    nl = nl_em - cheb_depth(bc->cheb) - bc->r;
    // SlotToCoeff is built on the first bootstrap, when the (data-independent) scale of the
    // EvalMod output is known; its first level absorbs that scale and q0 / (2 pi Delta_in)
    {
        int q0bits = 0;
        while (q0bits < 64 && (cx.mods[0] >> q0bits)) q0bits++;
        bc->delta_in = cx.boot_delta_log2 > 0    ? std::ldexp(1.0, cx.boot_delta_log2)
                       : cx.boot_delta_log2 < 0 ? canon(cx, 1)
                                                : std::ldexp(1.0, q0bits - 11);
    }
    bc->nl_stc = nl;
    bc->nl_out = nl - 3;
    cx.boot = bc;
}

static const std::vector<BootLevel>& stc_for(Context& cx, BootCtx* bc, double s_in, double relabel) {
    for (auto& st : bc->stcs)
        if (std::fabs(st.s_in / s_in - 1) < 1e-12 && std::fabs(st.relabel / relabel - 1) < 1e-12) return st.levels;
    const int n = cx.N / 2;
    int logn = 0;
    while ((1 << logn) < n) logn++;
    const int per = (logn + 2) / 3;
    const double q0 = (double)cx.mods[0];
    // q0 / (2 pi delta_in) turns EvalMod's sine back into the message; 1 / relabel puts a
    // relabelled input's message back on its own scale
    const std::complex<double> fold(q0 / (2 * M_PI * bc->delta_in) / relabel);
    BootCtx::StcSet st;
    st.s_in = s_in;
    st.relabel = relabel;
    int nl = bc->nl_stc;
    for (int lv = 0; lv < 3; lv++) {
        const int lo = lv * per, hi = std::min(logn, lo + per);
        st.levels.push_back(build_level(cx, lo, hi, false, nl, lv == 0 ? s_in : canon(cx, nl), canon(cx, nl - 1),
                                        lv == 0 ? fold : 1.0));
        nl--;
    }
    bc->stcs.push_back(std::move(st));
    return bc->stcs.back().levels;
}

int bootstrap_levels_after(const Context& cx) {
    auto* bc = (BootCtx*)cx.boot.get();
    return bc ? bc->nl_out : 0;
}

// ct (any level, nl >= 2 or canonical at 1 limb) -> refreshed ct at nl_out limbs, canonical scale.
// upto < 4 stops early (diagnostics): 1 after ModRaise, 2 after CoeffToSlot, 3 after EvalMod.
void bootstrap_upto(Context& cx, const Ciphertext& in, Ciphertext& out, int upto);
void bootstrap(Context& cx, const Ciphertext& in, Ciphertext& out) { bootstrap_upto(cx, in, out, 4); }

void bootstrap_upto(Context& cx, const Ciphertext& in, Ciphertext& out, int upto) {
    ProfScope op(cx, "op:bootstrap", 0);
    auto* bc = (BootCtx*)cx.boot.get();
    if (!bc) throw Error("bootstrap: no bootstrap precomputation (call bootstrap_setup)", -5);
    const int N = cx.N;
    Ciphertext a = ct_copy(cx, in);
    // 1. to one limb at the canonical scale of level L-1.  A one-limb input with another scale
    //    is relabelled (its integer message is what the pipeline refreshes) and the factor put
    //    back at the end: folded into SlotToCoeff for a canonical input (the output is then
    //    canonical), on the output's scale otherwise.
    double relabel = 1.0;
    if (a.nl > 1) align(cx, a, 1, bc->delta_in);
    else {
        relabel = a.scale / bc->delta_in;
        a.scale = bc->delta_in;
    }
    // 2. ModRaise: centred lift of the q0 residues to the bootstrap's top limbs
    const int Lt = bc->nl_top;
    Ciphertext raised = ct_alloc(cx, Lt);
    {
        DevBuf c((size_t)2 * N, cx.stream);
        CUDA_CHECK(cudaMemcpyAsync(c.p, a.c(0), N * 8, cudaMemcpyDeviceToDevice, cx.stream));
        CUDA_CHECK(cudaMemcpyAsync(c.p + N, a.c(1), N * 8, cudaMemcpyDeviceToDevice, cx.stream));
        LimbMap lm{};
        lm.base = c.p; lm.poly_stride = N; lm.nl = 1; lm.split = 1; lm.off0 = 0; lm.off1 = 0;
        ntt(cx, lm, 2, true, cx.stream);
        // k_rescale_lift writes y[c][i] for i < nlm1, layout [2][nlm1][N]: lift into a temp then copy
        DevBuf y((size_t)2 * Lt * N, cx.stream);
        launch_pdl(cx, k_rescale_lift, dim3(N / 256, Lt, 2), dim3(256), 0, cx.stream, c.p, y.p, Lt, 0, cx.logN);
        CUDA_CHECK(cudaGetLastError());
        cx.launches++;
        ntt(cx, cx.qmap(y.p, Lt, (long long)Lt * N), 2, false, cx.stream);
        CUDA_CHECK(cudaMemcpyAsync(raised.buf.p, y.p, (size_t)2 * Lt * N * 8, cudaMemcpyDeviceToDevice, cx.stream));
    }
    raised.scale = (double)cx.mods[0];
    if (upto == 1) { out = std::move(raised); return; }
    // 3. CoeffToSlot
    Ciphertext v = std::move(raised);
    auto* ps_cts = new ProfScope(cx, "op:boot_cts", 0);
    for (auto& L : bc->cts) {
        Ciphertext t;
        eval_level(cx, L, v, t);
        v = std::move(t);
    }
    delete ps_cts;
    if (upto == 2) { out = std::move(v); return; }
    // 4. EvalMod on 2 Re and 2 Im (values t/(q0 B) in [-1, 1])
    auto* ps_mod = new ProfScope(cx, "op:boot_evalmod", 0);
    Ciphertext re, im;
    split_complex(cx, v, re, im, false);
    Ciphertext parts[2] = {std::move(re), std::move(im)};
    {
        // the two evaluations run side by side: every ciphertext product is one batched product
        const Ciphertext* px[2] = {&parts[0], &parts[1]};
        Ciphertext c[2];
        cheb_eval_n(cx, px, 2, bc->cheb, c);
        for (int k = 0; k < bc->r; k++) {   // cos(2a) = 2 cos^2(a) - 1
            const Ciphertext* pc[2] = {&c[0], &c[1]};
            Ciphertext sq[2];
            mul_rescale_n(cx, pc, pc, 2, sq);
            for (int j = 0; j < 2; j++) mul_integer_add_const(cx, sq[j], 2, -1.0, c[j]);
        }
        parts[0] = std::move(c[0]);
        parts[1] = std::move(c[1]);
    }
    Ciphertext w;
    merge_complex(cx, std::move(parts[0]), std::move(parts[1]), w);
    delete ps_mod;
    if (upto == 3) { out = std::move(w); return; }
    ProfScope ps_stc(cx, "op:boot_stc", 0);
    // 5. SlotToCoeff
    if (w.nl > bc->nl_stc) align(cx, w, bc->nl_stc, 0);
    if (w.nl != bc->nl_stc) throw Error("bootstrap: EvalMod used more levels than planned", -4);
    // a canonical one-limb input (one factor, one cached set) comes out on the canonical scale;
    // any other scale keeps the relabelled output scale rather than a SlotToCoeff set per scale
    const bool fold = relabel != 1.0 && in.nl == 1 && std::fabs(in.scale / canon(cx, 1) - 1) < 1e-12;
    for (auto& L : stc_for(cx, bc, w.scale, fold ? relabel : 1.0)) {
        Ciphertext t;
        eval_level(cx, L, w, t);
        w = std::move(t);
    }
    if (!fold) w.scale *= relabel;
    out = std::move(w);
}

}  // namespace fhe
