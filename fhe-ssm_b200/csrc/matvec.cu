// matvec.cu -- the baby-step / giant-step plaintext-ciphertext matvec of the model
// (replaces matvec / matvecBatch / matvecBatchChunked, gpu_real_model.cu:2777-2833,
// :2883-3431; diagonal rule with the -g pre-rotation, harness/cpu_real_model.cpp:15-35).
//
// Layout.  A ciphertext carries one D-channel vector per block of D slots (slot r*D + c is
// channel c of lane r; with complex packing the real and imaginary parts are two lanes).
// y = W u needs a rotation of each block by k modulo D, while a ciphertext rotation moves
// data across block boundaries, so the block-cyclic rotation is split by masks:
//   rho_k(u) = M_k . rot(u, k) + (1 - M_k) . rot(u, k - D),   M_k[c] = [c + k < D].
// With k = g b1 + j the baby masks (M_j) and the giant masks (pushed through the giant
// rotation) are folded into three families of D-periodic plaintexts (AA, AB, BA; BB is
// empty), so the matvec is
//   y = sum_g rot(IA_g, g b1) + rot(IB_g, g b1 - D),
//   IA_g = sum_j AA_gj . rot(u, j) + AB_gj . rot(u, j - D),  IB_g = sum_j BA_gj . rot(u, j)
// i.e. 2 b1 - 1 hoisted baby rotations and 2 (D/b1 - 1) giant rotations.
//
// Plaintexts.  Every family vector is D-periodic, so its ring-N encoding is the ring-2D
// encoding of one period embedded at stride N/(2D) (hpc_gpu_port/periodic_encode.hpp:1-40
// states and checks this identity), and its NTT is the 2D-point NTT broadcast to
// word i >> log2(N/2D) (the compressed store, gpu_real_model.cu:145-175).  The plan keeps
// the 2D real small-ring coefficients of each family vector (fp64) in HBM; k_ptgen turns
// them into residues at the level and scale of the call (scale, round, reduce, 2D-point
// NTT, Montgomery form) and k_bsgs_mac accumulates all baby products of all giants in one
// pass over the babies.
#include <cmath>
#include <cstring>

#include "engine.h"

namespace fhe {

// small-ring special inverse FFT (n' = D slots, M' = 4D): same routine as encode
static void fft_special_inv_small(std::complex<double>* v, int n, int M);

// --------------------------------------------------------------------------- kernels ----
// coef [P][2D] fp64 -> out [P][nl][2D] words: round(c * scale) mod q_i, 2D-point NTT with the
// first 2D entries of the ring-N root table (they are the powers of psi^(N/2D) in the same
// bit-reversed order), then (mont != 0) * 2^64 mod q (Montgomery form for k_bsgs_mac)
__global__ void __launch_bounds__(256) k_ptgen(const double* __restrict__ coef, double scale, uint64_t* __restrict__ out,
                                               int nl, int logD2, const uint64_t* __restrict__ tw,
                                               const uint64_t* __restrict__ twp, int N, int mont) {
    extern __shared__ uint64_t sa[];
    const int D2 = 1 << logD2;
    const int id = blockIdx.x, i = blockIdx.y;
    const ModConst mc = c_mod[i];
    const double* c = coef + (size_t)id * D2;
    for (int k = threadIdx.x; k < D2; k += blockDim.x) {
        const double v = c[k] * scale;
        const long long r = llrint(v);
        sa[k] = r >= 0 ? reduce64((uint64_t)r, mc) : mod_neg(reduce64((uint64_t)(-r), mc), mc.q);
    }
    __syncthreads();
    const uint64_t* T = tw + (size_t)i * N;
    const uint64_t* Tp = twp + (size_t)i * N;
    for (int m = 1, t = D2 >> 1; m < D2; m <<= 1, t >>= 1) {
        for (int b = threadIdx.x; b < D2 / 2; b += blockDim.x) {
            const int grp = b / t, off = b % t;
            const int j1 = grp * 2 * t + off, j2 = j1 + t;
            const uint64_t w = T[m + grp], wp = Tp[m + grp];
            const uint64_t x = mul_shoup(sa[j2], w, wp, mc.q);
            const uint64_t u = sa[j1];
            sa[j1] = mod_add(u, x, mc.q);
            sa[j2] = mod_sub(u, x, mc.q);
        }
        __syncthreads();
    }
    uint64_t* o = out + ((size_t)id * nl + i) * D2;
    for (int k = threadIdx.x; k < D2; k += blockDim.x)
        o[k] = mont ? redc(__umul64hi(sa[k], mc.r2), sa[k] * mc.r2, mc) : sa[k];
}

// ------------------------------------------------------- periodic encode + plaintext cache ----
// A slot vector of period n < N/2 encodes as the ring-2n encoding of one period at stride
// N/2n (the identity of hpc_gpu_port/periodic_encode.hpp): a 2n-word compressed plaintext per
// limb, read by the element-wise kernels at word x >> log2(N/2n).  Plaintexts of the model's
// fixed vectors are cached by (content, level, scale), so a step re-encodes nothing.
static Plaintext encode_periodic(Context& cx, const std::complex<double>* z, int n, int nl, double scale) {
    std::vector<std::complex<double>> v(z, z + n);
    fft_special_inv(v.data(), n, 4 * n);
    std::vector<double> co(2 * n);
    const double maxv = (double)((1ull << 61) - 1);
    for (int k = 0; k < n; k++) {
        co[k] = v[k].real();
        co[k + n] = v[k].imag();
        if (std::fabs(co[k] * scale) > maxv || std::fabs(co[k + n] * scale) > maxv)
            throw Error("encode: value * scale exceeds 61 bits (refused)", -6);
    }
    DevBuf dc(co.size(), cx.stream);
    CUDA_CHECK(cudaMemcpyAsync(dc.p, co.data(), co.size() * 8, cudaMemcpyHostToDevice, cx.stream));
    int log2n = 0;
    while ((1 << log2n) < 2 * n) log2n++;
    Plaintext pt;
    pt.buf = DevBuf((size_t)nl * 2 * n, cx.stream);
    pt.nl = nl;
    pt.scale = scale;
    int lr = 0;
    while ((cx.N >> lr) > 2 * n) lr++;
    pt.log_rep = lr;
    k_ptgen<<<dim3(1, nl), 256, 2 * n * 8, cx.stream>>>((const double*)dc.p, scale, pt.buf.p, nl, log2n, cx.d_tw,
                                                       cx.d_twp, cx.N, 0);
    CUDA_CHECK(cudaGetLastError());
    cx.launches++;
    return pt;
}

const Plaintext& encode_cached(Context& cx, const std::complex<double>* z, int n, int nl, double scale) {
    uint64_t h = 1469598103934665603ull;   // FNV-1a over the bytes of (values, n, nl, scale)
    auto mix = [&](const void* p, size_t bytes) {
        const uint8_t* b = (const uint8_t*)p;
        for (size_t i = 0; i < bytes; i++) { h ^= b[i]; h *= 1099511628211ull; }
    };
    mix(z, sizeof(std::complex<double>) * n);
    mix(&n, sizeof n);
    mix(&nl, sizeof nl);
    mix(&scale, sizeof scale);
    auto it = cx.ptcache.find(h);
    if (it != cx.ptcache.end()) return *it->second;
    if (cx.ptcache.size() > 50000) cx.ptcache.clear();
    auto pt = std::make_shared<Plaintext>(n < cx.N / 2 && (cx.N / 2) % n == 0 && n >= 8
                                              ? encode_periodic(cx, z, n, nl, scale)
                                              : encode(cx, z, n, nl, scale));
    return *cx.ptcache.emplace(h, pt).first->second;
}

constexpr int kMaxBabies = 256;   // sets * 2 * b1 (kernel-parameter array)
struct MacArgs {
    const uint64_t* babies[kMaxBabies];   // [set][2][b1] ciphertext bases (Y = 0: rot(u, j), Y = 1: rot(u, j - D))
    long long bstride;               // words between c0 and c1 of a baby
    const int* ids;                  // [set][3][G][b1] plaintext id or -1 (families AA, AB, BA)
    const uint64_t* pts;             // [P][nl][2D] Montgomery words
    uint64_t* out;                   // [2G][2][nl][N] (IA_0..IA_{G-1}, IB_0..IB_{G-1})
    int nsets, b1, G, nl, logN, lr, D2;
};

// one CTA: 64 consecutive evaluation slots of one limb, 512 threads = 64 slots x 8 output
// groups; the babies' words for those slots are staged in shared memory per input set
__global__ void __launch_bounds__(512) k_bsgs_mac(MacArgs a) {
    extern __shared__ uint64_t sb[];   // [2][b1][2][64]
    const int N = 1 << a.logN;
    const int i = blockIdx.y;
    const int xs = threadIdx.x & 63, og = threadIdx.x >> 6;
    const int x = blockIdx.x * 64 + xs;
    const ModConst mc = c_mod[i];
    const int nout = 2 * a.G;
    constexpr int MAXO = 16;
    uint64_t acc[MAXO][2];
#pragma unroll
    for (int t = 0; t < MAXO; t++) acc[t][0] = acc[t][1] = 0;
    const int ptw = x >> a.lr;
    for (int s = 0; s < a.nsets; s++) {
        __syncthreads();
        for (int e = threadIdx.x; e < 2 * a.b1 * 2 * 64; e += blockDim.x) {
            const int xx = e & 63, p = (e >> 6) & 1, bj = e >> 7;   // bj = Y * b1 + j
            const uint64_t* base = a.babies[(size_t)s * 2 * a.b1 + bj];
            sb[e] = base[(size_t)p * a.bstride + (size_t)i * N + (size_t)blockIdx.x * 64 + xx];
        }
        __syncthreads();
        for (int t = 0; t < MAXO; t++) {
            const int o = og + 8 * t;
            if (o >= nout) break;
            const int X = o / a.G, g = o % a.G;
            for (int Y = 0; Y < 2; Y++) {
                const int fam = X == 0 ? Y : (Y == 0 ? 2 : -1);
                if (fam < 0) continue;
                const int* idrow = a.ids + (((size_t)s * 3 + fam) * a.G + g) * a.b1;
                for (int j0 = 0; j0 < a.b1; j0 += 8) {
                    u128acc p0{0, 0}, p1{0, 0};
                    bool any = false;
#pragma unroll
                    for (int jj = 0; jj < 8; jj++) {
                        const int j = j0 + jj;
                        if (j >= a.b1) break;
                        const int id = idrow[j];
                        if (id < 0) continue;
                        any = true;
                        const uint64_t w = a.pts[((size_t)id * a.nl + i) * a.D2 + ptw];
                        const uint64_t* bb = sb + ((Y * a.b1 + j) * 2) * 64 + xs;
                        acc_mad(p0, w, bb[0]);
                        acc_mad(p1, w, bb[64]);
                    }
                    if (!any) continue;
                    acc[t][0] += redc(p0.hi, p0.lo, mc);
                    acc[t][1] += redc(p1.hi, p1.lo, mc);
                    acc[t][0] = reduce_lazy16(acc[t][0], mc.q);
                    acc[t][1] = reduce_lazy16(acc[t][1], mc.q);
                }
            }
        }
    }
    for (int t = 0; t < MAXO; t++) {
        const int o = og + 8 * t;
        if (o >= nout) break;
        uint64_t* dst = a.out + (((size_t)o * 2) * a.nl + i) * N + x;
        dst[0] = acc[t][0];
        dst[(size_t)a.nl * N] = acc[t][1];
    }
}

// -------------------------------------------------------------------------- the plan ----
struct MatvecPlan {
    int D = 0, b1 = 0, G = 0, nsets = 0, P = 0, rows = 0, cols = 0;
    std::vector<int> ids;     // [set][3][G][b1]
    DevBuf d_ids;             // int table (packed into uint64 words)
    DevBuf coef;              // [P][2D] fp64 bit patterns
};

static void fft_special_inv_small(std::complex<double>* v, int n, int M) {
    std::vector<uint64_t> rg(n);
    uint64_t g = 1;
    for (int j = 0; j < n; j++) { rg[j] = g; g = (g * 5) % (uint64_t)M; }
    for (int len = n; len >= 1; len >>= 1) {
        const int lenh = len >> 1, lenq = len << 2;
        for (int i = 0; i < n; i += len)
            for (int j = 0; j < lenh; j++) {
                const uint64_t idx = ((uint64_t)lenq - (rg[j] % (uint64_t)lenq)) * (uint64_t)(M / lenq);
                const std::complex<double> w(std::cos(2.0 * M_PI * idx / M), std::sin(2.0 * M_PI * idx / M));
                const std::complex<double> u = v[i + j] + v[i + j + lenh];
                const std::complex<double> x = (v[i + j] - v[i + j + lenh]) * w;
                v[i + j] = u;
                v[i + j + lenh] = x;
            }
    }
    for (int i = 1, j = 0; i < n; i++) {
        int bit = n >> 1;
        for (; j & bit; bit >>= 1) j ^= bit;
        j ^= bit;
        if (i < j) std::swap(v[i], v[j]);
    }
    for (int i = 0; i < n; i++) v[i] /= (double)n;
}

// W: rows x cols row-major (rows <= D); column chunk s multiplies input ciphertext s
std::shared_ptr<MatvecPlan> matvec_plan(Context& cx, const double* W, int rows, int cols, int D, int b1) {
    const int n = cx.N / 2;
    if (D < 2 || (D & (D - 1)) || n % D || rows > D || b1 < 1 || D % b1)
        throw Error("matvec_plan: need D | N/2 (power of two), rows <= D, b1 | D", -1);
    auto pl = std::make_shared<MatvecPlan>();
    pl->D = D; pl->b1 = b1; pl->G = D / b1; pl->rows = rows; pl->cols = cols;
    pl->nsets = (cols + D - 1) / D;
    const int G = pl->G, S = pl->nsets;
    if (2 * G > 8 * 16) throw Error("matvec_plan: too many giant steps (2 D / b1 must be <= 128)", -1);
    pl->ids.assign((size_t)S * 3 * G * b1, -1);
    // family vectors, then small-ring coefficients (in parallel)
    struct Job { int s, fam, g, j; };
    std::vector<Job> jobs;
    for (int s = 0; s < S; s++)
        for (int g = 0; g < G; g++)
            for (int j = 0; j < b1; j++)
                for (int fam = 0; fam < 3; fam++) {
                    if (fam == 2 && g == 0) continue;   // giant-B mask [p < 0] is empty
                    jobs.push_back({s, fam, g, j});
                }
    std::vector<std::vector<double>> co(jobs.size());
    std::vector<char> nz(jobs.size(), 0);
#pragma omp parallel for schedule(dynamic, 16)
    for (long jb = 0; jb < (long)jobs.size(); jb++) {
        const Job J = jobs[jb];
        const int k = J.g * b1 + J.j;
        std::vector<std::complex<double>> v(D);
        bool any = false;
        for (int p = 0; p < D; p++) {
            const bool ga = p >= J.g * b1;                 // giant A keeps inner slots p >= g b1
            const bool mj = p + J.j < D;                   // baby A (rot(u, j)) is valid where p + j < D
            const bool use = J.fam == 0 ? (ga && mj) : J.fam == 1 ? (ga && !mj) : (!ga && mj);
            double w = 0.0;
            if (use) {
                const int c = ((p - J.g * b1) % D + D) % D;     // output channel of this inner slot
                const int col = (c + k) % D + J.s * D;
                if (c < rows && col < cols) w = W[(size_t)c * cols + col];
            }
            v[p] = w;
            if (w != 0.0) any = true;
        }
        if (!any) continue;
        nz[jb] = 1;
        fft_special_inv_small(v.data(), D, 4 * D);
        co[jb].resize(2 * D);
        for (int t = 0; t < D; t++) { co[jb][t] = v[t].real(); co[jb][t + D] = v[t].imag(); }
    }
    int P = 0;
    for (size_t jb = 0; jb < jobs.size(); jb++) if (nz[jb]) P++;
    std::vector<double> flat((size_t)std::max(P, 1) * 2 * D, 0.0);
    int id = 0;
    for (size_t jb = 0; jb < jobs.size(); jb++) {
        if (!nz[jb]) continue;
        const Job J = jobs[jb];
        pl->ids[(((size_t)J.s * 3 + J.fam) * G + J.g) * b1 + J.j] = id;
        std::copy(co[jb].begin(), co[jb].end(), flat.begin() + (size_t)id * 2 * D);
        id++;
    }
    pl->P = P;
    pl->coef = DevBuf(flat.size(), cx.stream);
    CUDA_CHECK(cudaMemcpyAsync(pl->coef.p, flat.data(), flat.size() * 8, cudaMemcpyHostToDevice, cx.stream));
    std::vector<uint64_t> idw((pl->ids.size() + 1) / 2, 0);
    std::memcpy(idw.data(), pl->ids.data(), pl->ids.size() * sizeof(int));
    pl->d_ids = DevBuf(idw.size(), cx.stream);
    CUDA_CHECK(cudaMemcpyAsync(pl->d_ids.p, idw.data(), idw.size() * 8, cudaMemcpyHostToDevice, cx.stream));
    CUDA_CHECK(cudaStreamSynchronize(cx.stream));
    return pl;
}

std::vector<int> matvec_rotations(int D, int b1) {
    std::vector<int> r;
    for (int j = 1; j < b1; j++) r.push_back(j);
    for (int j = 0; j < b1; j++) r.push_back(j - D);
    for (int g = 1; g < D / b1; g++) { r.push_back(g * b1); r.push_back(g * b1 - D); }
    return r;
}

// the 2 b1 babies of one input: rot(u, j) (j = 0..b1-1) and rot(u, j - D) (j = 0..b1-1),
// all with stride nl*N; one hoisted ModUp
struct BabySet {
    int D = 0, b1 = 0, nl = 0;
    double scale = 0;
    std::vector<Ciphertext> cts;   // [2 b1]: Y = 0 then Y = 1
};

void matvec_babies(Context& cx, const Ciphertext& u, int D, int b1, BabySet& bs) {
    if (u.nl < 2) throw Error("matvec: no level left", -4);
    std::vector<int> steps;
    for (int j = 1; j < b1; j++) steps.push_back(j);
    for (int j = 0; j < b1; j++) steps.push_back(j - D);
    std::vector<Ciphertext> r(steps.size());
    ct_rotate_hoisted(cx, u, steps.data(), (int)steps.size(), r.data());
    bs.D = D; bs.b1 = b1; bs.nl = u.nl; bs.scale = u.scale;
    bs.cts.clear();
    bs.cts.resize(2 * b1);
    bs.cts[0] = ct_copy(cx, u);
    for (int j = 1; j < b1; j++) bs.cts[j] = std::move(r[j - 1]);
    for (int j = 0; j < b1; j++) bs.cts[b1 + j] = std::move(r[b1 - 1 + j]);
}

void matvec_apply(Context& cx, const MatvecPlan& pl, const BabySet* const* sets, Ciphertext& out);

// y = W [u_0 | u_1 | ...]: inputs (one per column chunk) at a common level and scale;
// the output is rescaled once and lands on the canonical scale of level nl - 1
void matvec(Context& cx, const MatvecPlan& pl, const Ciphertext* const* us, Ciphertext& out) {
    std::vector<BabySet> bs(pl.nsets);
    std::vector<const BabySet*> ptr(pl.nsets);
    for (int s = 0; s < pl.nsets; s++) {
        matvec_babies(cx, *us[s], pl.D, pl.b1, bs[s]);
        ptr[s] = &bs[s];
    }
    matvec_apply(cx, pl, ptr.data(), out);
}

void matvec_apply(Context& cx, const MatvecPlan& pl, const BabySet* const* sets, Ciphertext& out) {
    const int N = cx.N, S = pl.nsets, b1 = pl.b1, G = pl.G, D = pl.D;
    const int nl = sets[0]->nl;
    for (int s = 0; s < S; s++)
        if (sets[s]->nl != nl || std::fabs(sets[s]->scale / sets[0]->scale - 1) > 1e-9 || sets[s]->D != D ||
            sets[s]->b1 != b1)
            throw Error("matvec: input chunks must share level, scale and baby geometry", -4);
    cudaStream_t st = cx.stream;
    if ((size_t)S * 2 * b1 > (size_t)kMaxBabies) throw Error("matvec: too many babies for one launch", -1);
    // plaintexts at this level: scale so that the rescaled output is canonical
    const double target = canon(cx, nl - 1);
    const double spt = target * (double)cx.mods[nl - 1] / sets[0]->scale;
    int logD2 = 0;
    while ((1 << logD2) < 2 * D) logD2++;
    DevBuf pts((size_t)std::max(pl.P, 1) * nl * 2 * D, st);
    if (pl.P > 0) {
        ProfScope ps(cx, "ptgen", 8.0 * pl.P * 2 * D * (1 + nl));
        k_ptgen<<<dim3(pl.P, nl), 256, 2 * D * 8, st>>>((const double*)pl.coef.p, spt, pts.p, nl, logD2, cx.d_tw,
                                                        cx.d_twp, N, 1);
        CUDA_CHECK(cudaGetLastError());
        cx.launches++;
    }
    DevBuf inner((size_t)2 * G * 2 * nl * N, st);
    {
        MacArgs a;
        for (int s = 0; s < S; s++)
            for (int k = 0; k < 2 * b1; k++) a.babies[(size_t)s * 2 * b1 + k] = sets[s]->cts[k].buf.p;
        a.bstride = (long long)nl * N;
        a.ids = (const int*)pl.d_ids.p;
        a.pts = pts.p;
        a.out = inner.p;
        a.nsets = S; a.b1 = b1; a.G = G; a.nl = nl; a.logN = cx.logN; a.D2 = 2 * D;
        int lr = 0;
        while ((N >> lr) > 2 * D) lr++;
        a.lr = lr;
        const size_t smem = (size_t)2 * b1 * 2 * 64 * 8;
        ProfScope ps(cx, "bsgs_mac", 8.0 * N * nl * (2.0 * S * 2 * b1 + 2.0 * 2 * G));
        if (smem > 48 * 1024)
            CUDA_CHECK(cudaFuncSetAttribute(k_bsgs_mac, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        k_bsgs_mac<<<dim3(N / 64, nl), 512, smem, st>>>(a);
        CUDA_CHECK(cudaGetLastError());
        cx.launches++;
    }
    // giants: sum_g rot(IA_g, g b1) + rot(IB_g, g b1 - D)
    // (IA_0 unrotated; IB_0 is empty: rot(u, j) with j < b1 never needs the -D giant)
    const double sc = sets[0]->scale * spt;
    std::vector<const uint64_t*> c0s, c1s;
    std::vector<int> steps;
    for (int g = 1; g < G; g++)
        for (int X = 0; X < 2; X++) {
            const uint64_t* p = inner.p + (size_t)(X * G + g) * 2 * nl * N;
            c0s.push_back(p);
            c1s.push_back(p + (size_t)nl * N);
            steps.push_back(X == 0 ? g * b1 : g * b1 - D);
        }
    Ciphertext acc;
    rotate_sum(cx, c0s.data(), c1s.data(), steps.data(), (int)steps.size(), nl, sc, inner.p,
               inner.p + (size_t)nl * N, acc);
    ct_rescale(cx, acc);
    acc.scale = target;
    out = std::move(acc);
}

}  // namespace fhe
