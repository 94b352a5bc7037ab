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
// empty): y = sum_g rot(IA_g, g b1) + rot(IB_g, g b1 - D) with
//   IA_g = sum_j AA_gj . rot(u, j) + AB_gj . rot(u, j - D),  IB_g = sum_j BA_gj . rot(u, j).
// A D-periodic plaintext is invariant under rot(., -D), so rot(BA . rot(u, j), g b1 - D) =
// rot(BA . rot(u, j - D), g b1): the BA family joins AB on the baby rot(u, j - D) under the
// same giant, and
//   y = sum_g rot(I_g, g b1),  I_g = sum_j AA_gj . rot(u, j) + (AB_gj + BA_gj) . rot(u, j - D),
// i.e. 2 b1 - 1 hoisted baby rotations and D/b1 - 1 giant rotations (the masks of AB and BA
// are disjoint, so the merged family is one plaintext per (g, j)).
//
// Plaintexts.  Every family vector is D-periodic, so its ring-N encoding is the ring-2D
// encoding of one period embedded at stride N/(2D) (hpc_gpu_port/periodic_encode.hpp:1-40
// states and checks this identity), and its NTT is the 2D-point NTT broadcast to
// word i >> log2(N/2D) (the compressed store, gpu_real_model.cu:145-175).  The plan keeps
// the 2D real small-ring coefficients of each family vector (fp64) in HBM; k_ptgen turns
// them into residues at the level and scale of the call (scale, round, reduce, 2D-point
// NTT, Montgomery form), for the Q limbs and the special limbs P.
//
// Evaluation (double hoisting, Bossuat et al., Eurocrypt 2021, section 4):
//  * babies: one ModUp of u, then every baby rot(u, r) is left in the extended basis QP as
//    P rot(u, r) (no ModDown): k_baby_pq computes the key inner product at the permuted
//    slots of the shared ModUp output with the rotate-then-switch key;
//  * k_bsgs_gemm: for every REP-group of slots (the slots that share one compressed
//    plaintext word) the products are a dense (G x 2b1) x (2b1 x slots) product of words
//    mod q; the kernel stages babies and plaintext words in shared memory and accumulates
//    128-bit;
//  * one ModDown per giant input (G of them, batched), then the giant rotations summed by
//    rotate_sum (one batched ModUp, one ModDown of the sum).
#include <cmath>
#include <cstring>

#include "engine.h"

namespace fhe {

// small-ring special inverse FFT (n' = D slots, M' = 4D): same routine as encode
static void fft_special_inv_small(std::complex<double>* v, int n, int M);

// --------------------------------------------------------------------------- kernels ----
// coef [P][2D] fp64 -> out [limb][2D][P] words (word k of every plaintext of a limb is
// contiguous, the order k_bsgs_gemm reads): round(c * scale) mod m(i), 2D-point NTT with the
// first 2D entries of the ring-N root table (the powers of psi^(N/2D) in the same
// bit-reversed order), then (mont != 0) * 2^64 mod q (Montgomery form for the products).
// Limb i uses modulus i for i < nq and the special modulus L + i - nq above; IPC plaintexts
// per CTA (their words are written together).
template <int IPC>
__global__ void __launch_bounds__(256) k_ptgen(const double* __restrict__ coef, double scale, uint64_t* __restrict__ out,
                                               int P, int nq, int L, int logD2, const uint64_t* __restrict__ tw,
                                               const uint64_t* __restrict__ twp, int N, int mont) {
    extern __shared__ uint64_t sa[];   // [IPC][2D]
    const int D2 = 1 << logD2;
    const int id0 = blockIdx.x * IPC, i = blockIdx.y;
    const int m = i < nq ? i : L + (i - nq);
    const ModConst mc = c_mod[m];
    for (int e = threadIdx.x; e < IPC * D2; e += blockDim.x) {
        const int t = e >> logD2, k = e & (D2 - 1);
        uint64_t r0 = 0;
        if (id0 + t < P) {
            const long long r = llround(coef[(size_t)(id0 + t) * D2 + k] * scale);   // ties away from zero, as llround in encode
            r0 = r >= 0 ? reduce64((uint64_t)r, mc) : mod_neg(reduce64((uint64_t)(-r), mc), mc.q);
        }
        sa[e] = r0;
    }
    __syncthreads();
    const uint64_t* T = tw + (size_t)m * N;
    const uint64_t* Tp = twp + (size_t)m * N;
    for (int mm = 1, t = D2 >> 1; mm < D2; mm <<= 1, t >>= 1) {
        for (int bi = threadIdx.x; bi < IPC * (D2 / 2); bi += blockDim.x) {
            const int v = bi / (D2 / 2), b = bi % (D2 / 2);
            const int grp = b / t, off = b % t;
            const int j1 = grp * 2 * t + off, j2 = j1 + t;
            uint64_t* s2 = sa + (size_t)v * D2;
            const uint64_t x = mul_shoup(s2[j2], T[mm + grp], Tp[mm + grp], mc.q);
            const uint64_t u = s2[j1];
            s2[j1] = mod_add(u, x, mc.q);
            s2[j2] = mod_sub(u, x, mc.q);
        }
        __syncthreads();
    }
    for (int e = threadIdx.x; e < IPC * D2; e += blockDim.x) {
        const int t = e % IPC, k = e / IPC;
        if (id0 + t >= P) continue;
        const uint64_t v = sa[(size_t)t * D2 + k];
        out[((size_t)i * D2 + k) * P + id0 + t] = mont ? redc(__umul64hi(v, mc.r2), v * mc.r2, mc) : v;
    }
}

// 2048-point specialisation of k_ptgen (D = 1024, the model's block): one plaintext at a time
// in registers, 8 words per thread, 11 butterfly stages in 4 passes (3 + 3 + 3 + 2) with three
// exchanges through shared memory; the limb's twiddles are staged in shared memory once per CTA,
// and 4 plaintexts are written together (32-byte runs of the transposed layout).  The
// butterflies are the lazy ones of the ring NTT with the cheaper quotient (values in
// [0, 8q + 2^32), twiddle and Shoup companion read as one 16-byte pair); the output is made
// canonical, or taken to Montgomery form by a Shoup product with 2^64 mod q: the same words as
// k_ptgen.
__device__ __forceinline__ void pgl(uint64_t& a, uint64_t& b, const ulonglong2 t, uint64_t q) {
    bfly<false, 1>(a, b, t.x, t.y, q);
}
__global__ void __launch_bounds__(256) k_ptgen2048(const double* __restrict__ coef, double scale,
                                                   uint64_t* __restrict__ out, int P, int nq, int L,
                                                   const ulonglong2* __restrict__ tw2,
                                                   const uint64_t* __restrict__ rmont, int N, int mont) {
    constexpr int D2 = 2048, IPC = 4;
    extern __shared__ uint64_t pg[];
    ulonglong2* T = reinterpret_cast<ulonglong2*>(pg);   // [D2] (twiddle, Shoup companion) pairs
    uint64_t* S = pg + 2 * D2;     // [IPC][D2]: exchange buffer of plaintext t, then its result
    const int tid = threadIdx.x;
    const int id0 = blockIdx.x * IPC, i = blockIdx.y;
    const int m = i < nq ? i : L + (i - nq);
    const ModConst mc = c_mod[m];
    const uint64_t q = mc.q;
    // the coefficients of all IPC plaintexts are loaded up front (one latency for the CTA)
    double cf[IPC][8];
#pragma unroll
    for (int t = 0; t < IPC; t++)
#pragma unroll
        for (int k = 0; k < 8; k++)
            cf[t][k] = id0 + t < P ? coef[(size_t)(id0 + t) * D2 + tid + 256 * k] : 0.0;
    for (int k = tid; k < D2; k += 256) T[k] = tw2[(size_t)m * N + k];
    const uint64_t rq = rmont[2 * m], rqp = rmont[2 * m + 1];   // 2^64 mod q (+ Shoup): Montgomery form
    __syncthreads();
#pragma unroll
    for (int t = 0; t < IPC; t++) {
        uint64_t* Sb = S + (size_t)t * D2;
        uint64_t x[8];
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const long long r = llround(cf[t][k] * scale);   // ties away from zero, as llround in encode
            x[k] = r >= 0 ? reduce64((uint64_t)r, mc) : mod_neg(reduce64((uint64_t)(-r), mc), q);
        }
        // pass 1: elements tid + 256 k, distances 1024, 512, 256
        pgl(x[0], x[4], T[1], q); pgl(x[1], x[5], T[1], q);
        pgl(x[2], x[6], T[1], q); pgl(x[3], x[7], T[1], q);
#pragma unroll
        for (int k = 0; k < 8; k++) if ((k & 2) == 0) pgl(x[k], x[k + 2], T[2 + k / 4], q);
#pragma unroll
        for (int k = 0; k < 8; k += 2) pgl(x[k], x[k + 1], T[4 + k / 2], q);
#pragma unroll
        for (int k = 0; k < 8; k++) Sb[tid + 256 * k] = x[k];
        __syncthreads();
        // pass 2: elements blk*256 + r + 32 k (blk = tid / 32, r = tid % 32), distances 128, 64, 32
        {
            const int blk = tid >> 5, r = tid & 31;
#pragma unroll
            for (int k = 0; k < 8; k++) x[k] = Sb[blk * 256 + r + 32 * k];
#pragma unroll
            for (int k = 0; k < 4; k++) pgl(x[k], x[k + 4], T[8 + blk], q);
#pragma unroll
            for (int k = 0; k < 8; k++) if ((k & 2) == 0) pgl(x[k], x[k + 2], T[16 + 2 * blk + k / 4], q);
#pragma unroll
            for (int k = 0; k < 8; k += 2) pgl(x[k], x[k + 1], T[32 + 4 * blk + k / 2], q);
            __syncthreads();
#pragma unroll
            for (int k = 0; k < 8; k++) Sb[blk * 256 + r + 32 * k] = x[k];
        }
        __syncthreads();
        // pass 3: elements g*32 + r + 4 k (g = tid / 4, r = tid % 4), distances 16, 8, 4
        {
            const int g = tid >> 2, r = tid & 3;
#pragma unroll
            for (int k = 0; k < 8; k++) x[k] = Sb[g * 32 + r + 4 * k];
#pragma unroll
            for (int k = 0; k < 4; k++) pgl(x[k], x[k + 4], T[64 + g], q);
#pragma unroll
            for (int k = 0; k < 8; k++) if ((k & 2) == 0) pgl(x[k], x[k + 2], T[128 + 2 * g + k / 4], q);
#pragma unroll
            for (int k = 0; k < 8; k += 2) pgl(x[k], x[k + 1], T[256 + 4 * g + k / 2], q);
            __syncthreads();
#pragma unroll
            for (int k = 0; k < 8; k++) Sb[g * 32 + r + 4 * k] = x[k];
        }
        __syncthreads();
        // pass 4: elements 8 tid + k, distances 2, 1
        {
#pragma unroll
            for (int k = 0; k < 8; k++) x[k] = Sb[8 * tid + k];
#pragma unroll
            for (int k = 0; k < 8; k++) if ((k & 2) == 0) pgl(x[k], x[k + 2], T[512 + 2 * tid + k / 4], q);
#pragma unroll
            for (int k = 0; k < 8; k += 2) pgl(x[k], x[k + 1], T[1024 + 4 * tid + k / 2], q);
            __syncthreads();
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const uint64_t v = x[k];
                Sb[8 * tid + k] = mont ? mul_shoup(v, rq, rqp, q) : canon_out<1>(v, q);
            }
        }
        __syncthreads();
    }
    for (int e = tid; e < IPC * D2; e += 256) {
        const int t = e % IPC, k = e / IPC;
        if (id0 + t >= P) continue;
        out[((size_t)i * D2 + k) * P + id0 + t] = S[(size_t)t * D2 + k];
    }
}

// ------------------------------------------------------- periodic encode + plaintext cache ----
// A slot vector of period n < N/2 encodes as the ring-2n encoding of one period at stride
// N/2n (the identity of hpc_gpu_port/periodic_encode.hpp): a 2n-word compressed plaintext per
// limb, read by the element-wise kernels at word x >> log2(N/2n).  Plaintexts of the model's
// fixed vectors are cached by (content, level, scale), so a step re-encodes nothing.
// A slot vector of period n (n | N/2, n <= 4096) as a REP-compressed plaintext (word x of a
// limb = comp[x >> log_rep], 2n words per limb): nl Q limbs, then (pq) the K special limbs, in
// Montgomery form when `mont` is set.
Plaintext encode_periodic_ext(Context& cx, const std::complex<double>* z, int n, int nl, double scale, bool pq,
                              bool mont) {
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
    upload_async(cx, dc.p, co.data(), co.size() * 8);
    cx.pt_encodes++;
    int log2n = 0;
    while ((1 << log2n) < 2 * n) log2n++;
    const int nlimb = nl + (pq ? cx.K : 0);
    Plaintext pt;
    pt.buf = DevBuf((size_t)nlimb * 2 * n, cx.stream);
    pt.nl = nlimb;
    pt.scale = scale;
    int lr = 0;
    while ((cx.N >> lr) > 2 * n) lr++;
    pt.log_rep = lr;
    if (2 * n * 8 > 48 * 1024)
        CUDA_CHECK(cudaFuncSetAttribute(k_ptgen<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * n * 8));
    k_ptgen<1><<<dim3(1, nlimb), 256, 2 * n * 8, cx.stream>>>((const double*)dc.p, scale, pt.buf.p, 1, nl, cx.L,
                                                             log2n, cx.d_tw, cx.d_twp, cx.N, mont ? 1 : 0);
    CUDA_CHECK(cudaGetLastError());
    cx.launches++;
    return pt;
}
static Plaintext encode_periodic(Context& cx, const std::complex<double>* z, int n, int nl, double scale) {
    return encode_periodic_ext(cx, z, n, nl, scale, false, false);
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
    auto pt = std::make_shared<Plaintext>(n < cx.N / 2 && (cx.N / 2) % n == 0 && n >= 8 && n <= 4096
                                              ? encode_periodic(cx, z, n, nl, scale)
                                              : encode(cx, z, n, nl, scale));
    return *cx.ptcache.emplace(h, pt).first->second;
}

constexpr int kMaxSets = 8;      // input chunks of one matvec (column blocks of D)
constexpr int kKc = 64;          // babies per shared-memory chunk (<= 128 products per 128-bit sum)

struct GemmArgs {
    const uint64_t* babies[kMaxSets];   // per set: [2 b1][2][ne][N], QP basis (Y = 0: rot(u, j), Y = 1: rot(u, j - D))
    const int* ids;                     // [set][3][G][b1] plaintext id or -1 (families AA, AB+BA; the
                                        // third, BA alone, is empty in merged plans)
    const uint64_t* pts;                // [ne][2D][P] Montgomery words
    uint64_t* out;                      // [M][2][ne][N] (I_0..I_{G-1}, then zero outputs up to M), QP
    int nsets, b1, G, M, nl, ne, L, logN, lr, D2, P, TW;
};

// One CTA: limb e of TW consecutive slots that share one compressed plaintext word (TW <= REP),
// both polynomials: out[o][c][x] = sum_k W[o][k] * baby[k][c][x] with W[o][k] the word of
// family fam(o, k), giant g(o), baby j(k).  Thread (to, tn) owns outputs 2to, 2to+1 and the 4
// columns 4tn..4tn+3 (column n = c * TW + slot).  Babies and plaintext words are staged in
// shared memory kKc at a time, split into 30-bit halves (words < q < 2^60): a b =
// a0 b0 + (a0 b1 + a1 b0) 2^30 + a1 b1 2^60 with every partial product a 32x32->64-bit
// multiply-add.  The three 64-bit partial sums absorb 8 terms (< 2^64) before they are folded
// into a 128-bit sum; each chunk sum (< kKc q^2 < 2^127) is Montgomery-reduced (W carries the
// factor 2^64) into a running sum mod q.
__device__ __forceinline__ void fold128(u128acc& t, uint64_t s00, uint64_t smid, uint64_t s11) {
    // t += s00 + smid 2^30 + s11 2^60
    uint64_t lo = s00, hi = 0;
    const uint64_t ml = smid << 30, mh = smid >> 34;
    const uint64_t hl = s11 << 60, hh = s11 >> 4;
    asm("add.cc.u64 %0, %0, %2;\n\taddc.u64 %1, %1, %3;" : "+l"(lo), "+l"(hi) : "l"(ml), "l"(mh));
    asm("add.cc.u64 %0, %0, %2;\n\taddc.u64 %1, %1, %3;" : "+l"(lo), "+l"(hi) : "l"(hl), "l"(hh));
    asm("add.cc.u64 %0, %0, %2;\n\taddc.u64 %1, %1, %3;" : "+l"(t.lo), "+l"(t.hi) : "l"(lo), "l"(hi));
}

__global__ void __launch_bounds__(512) k_bsgs_gemm(const GemmArgs a) {
    extern __shared__ uint32_t sm32[];
    const int M = a.M, TW = a.TW, NC = 2 * TW;
    uint32_t* Bs = sm32;                        // [kKc][NC][2]  (lo30, hi30)
    uint32_t* Ws = sm32 + (size_t)kKc * NC * 2; // [kKc][M][2]
    const int N = 1 << a.logN;
    const int e = blockIdx.y;
    const int x0 = blockIdx.x * TW;
    const int m = e < a.nl ? e : a.L + (e - a.nl);
    const ModConst mc = c_mod[m];
    const int nth = blockDim.x, tid = threadIdx.x;
    const int tn = tid % (TW / 2), to = tid / (TW / 2);
    const int o0 = 2 * to, n0 = 4 * tn;
    const int ptw = x0 >> a.lr;
    const int K = 2 * a.b1;
    constexpr uint64_t M30 = (1ull << 30) - 1;
    uint64_t sum[2][4];
#pragma unroll
    for (int u = 0; u < 2; u++)
#pragma unroll
        for (int v = 0; v < 4; v++) sum[u][v] = 0;
    for (int s = 0; s < a.nsets; s++) {
        const uint64_t* bb = a.babies[s];
        for (int k0 = 0; k0 < K; k0 += kKc) {
            const int kc = min(kKc, K - k0);
            __syncthreads();
            for (int t = tid; t < kc * NC; t += nth) {
                const int kk = t / NC, n = t % NC, c = n / TW, xs = n % TW;
                const uint64_t v = bb[(((size_t)(k0 + kk) * 2 + c) * a.ne + e) * N + x0 + xs];
                Bs[2 * t] = (uint32_t)(v & M30);
                Bs[2 * t + 1] = (uint32_t)(v >> 30);
            }
            for (int t = tid; t < kc * M; t += nth) {
                const int kk = t / M, o = t % M;
                const int k = k0 + kk, Y = k / a.b1, j = k % a.b1;
                const int X = o / a.G, g = o % a.G;
                const int fam = X == 0 ? Y : (Y == 0 ? 2 : -1);
                int id = -1;
                if (fam >= 0) id = a.ids[(((size_t)s * 3 + fam) * a.G + g) * a.b1 + j];
                const uint64_t v = id < 0 ? 0 : a.pts[((size_t)e * a.D2 + ptw) * a.P + id];
                Ws[2 * t] = (uint32_t)(v & M30);
                Ws[2 * t + 1] = (uint32_t)(v >> 30);
            }
            __syncthreads();
            // outputs o >= G (the zero second output when G = 1) have no products with the
            // babies rot(u, j - D) (k >= b1): those warps stop early (the split is warp-uniform)
            const int kend = o0 >= a.G ? max(0, min(kc, a.b1 - k0)) : kc;
            u128acc tot[2][4];
#pragma unroll
            for (int u = 0; u < 2; u++)
#pragma unroll
                for (int v = 0; v < 4; v++) tot[u][v] = u128acc{0, 0};
            for (int kb = 0; kb < kend; kb += 8) {
                uint64_t s00[2][4], smd[2][4], s11[2][4];
#pragma unroll
                for (int u = 0; u < 2; u++)
#pragma unroll
                    for (int v = 0; v < 4; v++) s00[u][v] = smd[u][v] = s11[u][v] = 0;
                const int ke = min(kend, kb + 8);
                for (int kk = kb; kk < ke; kk++) {
                    const uint4 wv = *reinterpret_cast<const uint4*>(Ws + (size_t)(kk * M + o0) * 2);
                    const uint4 bA = *reinterpret_cast<const uint4*>(Bs + (size_t)(kk * NC + n0) * 2);
                    const uint4 bB = *reinterpret_cast<const uint4*>(Bs + (size_t)(kk * NC + n0) * 2 + 4);
                    const uint32_t w0[2] = {wv.x, wv.z}, w1[2] = {wv.y, wv.w};
                    const uint32_t b0[4] = {bA.x, bA.z, bB.x, bB.z}, b1[4] = {bA.y, bA.w, bB.y, bB.w};
#pragma unroll
                    for (int u = 0; u < 2; u++)
#pragma unroll
                        for (int v = 0; v < 4; v++) {
                            s00[u][v] += (uint64_t)w0[u] * b0[v];
                            smd[u][v] += (uint64_t)w0[u] * b1[v];
                            smd[u][v] += (uint64_t)w1[u] * b0[v];
                            s11[u][v] += (uint64_t)w1[u] * b1[v];
                        }
                }
#pragma unroll
                for (int u = 0; u < 2; u++)
#pragma unroll
                    for (int v = 0; v < 4; v++) fold128(tot[u][v], s00[u][v], smd[u][v], s11[u][v]);
            }
#pragma unroll
            for (int u = 0; u < 2; u++)
#pragma unroll
                for (int v = 0; v < 4; v++) {
                    // <= 64 products of words < q < 2^60: hi < 64 q^2 / 2^64 < 4q; bring it below q
                    // (T changes by a multiple of q 2^64) before the Montgomery step
                    uint64_t hi = tot[u][v].hi;
                    if (hi >= 2 * mc.q) hi -= 2 * mc.q;
                    if (hi >= mc.q) hi -= mc.q;
                    sum[u][v] = mod_add(sum[u][v], redc(hi, tot[u][v].lo, mc), mc.q);
                }
        }
    }
#pragma unroll
    for (int u = 0; u < 2; u++)
#pragma unroll
        for (int v = 0; v < 4; v++) {
            const int n = n0 + v, c = n / TW, xs = n % TW;
            a.out[(((size_t)(o0 + u) * 2 + c) * a.ne + e) * N + x0 + xs] = sum[u][v];
        }
}

#include "tc_gemm.cuh"   // (inside namespace fhe)

// Babies in QP: out[b] = P rot(u, r_b), i.e. c0 = tau(ip0) + P tau(u0), c1 = tau(ip1) with
// ip = <ModUp(u1), key_b> evaluated at the permuted slots of the shared ModUp output `ext`
// against the rotate-then-switch key (fkey[x] = key[auto_src(x)]); perm == 1: P u.
struct BabyArgs {
    const uint64_t* fkey[64];
    uint64_t perm[64];
    uint64_t pw[kMaxMod], pwp[kMaxMod];   // P mod q_i (Shoup)
};
// Each thread owns one slot x of one baby and walks `per` consecutive limbs e (Context::
// baby_limbs): the permuted source slot, the baby's key pointer and its index are computed once
// per thread, not once per limb.
__global__ void __launch_bounds__(256) k_baby_pq(const uint64_t* __restrict__ ext, const uint64_t* __restrict__ u0,
                                                 const uint64_t* __restrict__ u1, const __grid_constant__ BabyArgs a,
                                                 uint64_t* __restrict__ out, int nl, int ne, int dn, int L, int K,
                                                 int logN, int per) {
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int b = blockIdx.z;
    const int e0 = blockIdx.y * per, e1 = min(ne, e0 + per);
    uint64_t* o = out + (size_t)b * 2 * ne * N;
    const uint64_t k = a.perm[b];
    if (k == 1) {
        for (int e = e0; e < e1; e++) {
            const uint64_t q = c_mod[e < nl ? e : L + (e - nl)].q;
            uint64_t v0 = 0, v1 = 0;
            if (e < nl) {
                v0 = mul_shoup(u0[(size_t)e * N + x], a.pw[e], a.pwp[e], q);
                v1 = mul_shoup(u1[(size_t)e * N + x], a.pw[e], a.pwp[e], q);
            }
            o[(size_t)e * N + x] = v0;
            o[((size_t)ne + e) * N + x] = v1;
        }
        return;
    }
    const uint32_t sx = auto_src((uint32_t)x, k, logN);
    const uint64_t* key = a.fkey[b];
    const size_t nk = (size_t)(L + K);
#pragma unroll 1
    for (int e = e0; e < e1; e++) {
        const int m = e < nl ? e : L + (e - nl);
        const ModConst mc = c_mod[m];
        u128acc a0{0, 0}, a1{0, 0};
        digit_dot2(ext + (size_t)e * N + sx, (size_t)ne * N, key + (size_t)m * N + x, key + (nk + m) * N + x,
                   2 * nk * N, dn, a0, a1);
        uint64_t v0 = redc(a0.hi, a0.lo, mc);
        const uint64_t v1 = redc(a1.hi, a1.lo, mc);
        if (e < nl) v0 = mod_add(v0, mul_shoup(u0[(size_t)e * N + sx], a.pw[e], a.pwp[e], mc.q), mc.q);
        o[(size_t)e * N + x] = v0;
        o[((size_t)ne + e) * N + x] = v1;
    }
}

// -------------------------------------------------------------------------- the plan ----
struct MatvecPlan {
    int D = 0, b1 = 0, G = 0, nsets = 0, P = 0, rows = 0, cols = 0;
    std::vector<int> ids;     // [set][3][G][b1]
    DevBuf d_ids;             // int table (packed into uint64 words)
    DevBuf coef;              // [P][2D] fp64 bit patterns
    // plaintext words of the last call ([ne][2D][P] at level cached_nl, plaintext scale
    // cached_spt), kept under the context's plaintext-cache budget: a recurrent model applies
    // every matrix at the same level and scale on every step
    mutable DevBuf cached;
    mutable int cached_nl = 0;
    mutable double cached_spt = 0.0;
    Context* owner = nullptr;
    ~MatvecPlan() {
        if (owner && cached.p) owner->pt_cache_bytes -= (long long)(cached.words * 8);
    }
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
    pl->owner = &cx;
    pl->D = D; pl->b1 = b1; pl->G = D / b1; pl->rows = rows; pl->cols = cols;
    pl->nsets = (cols + D - 1) / D;
    const int G = pl->G, S = pl->nsets;
    // matvec_apply's product tile pairs the M = max(2, G) outputs of one giant family: G <= 64
    if (G > 64) throw Error("matvec_plan: too many giant steps (D / b1 must be <= 64)", -1);
    pl->ids.assign((size_t)S * 3 * G * b1, -1);
    // family vectors, then small-ring coefficients (in parallel)
    struct Job { int s, fam, g, j; };
    std::vector<Job> jobs;
    for (int s = 0; s < S; s++)
        for (int g = 0; g < G; g++)
            for (int j = 0; j < b1; j++)
                for (int fam = 0; fam < 2; fam++) jobs.push_back({s, fam, g, j});   // AA, AB + BA
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
            // family 0: AA (ga, mj); family 1: AB (ga, !mj) + BA (!ga, mj) on the baby rot(u, j - D)
            const bool use = J.fam == 0 ? (ga && mj) : (ga != mj);
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

// The compressed store entries of `count` period-`period` slot vectors (the reference's
// periodicEncodeComp, hpc_gpu_port/periodic_encode.hpp:263-276): the plan's small-ring inverse
// FFT on the host, then the plan's device generator (k_ptgen2048 at period 1024, else k_ptgen)
// in canonical form.  host_out: [count][nl][2 period]; word j2 of limb l is word
// j2 << log2(N / (2 period)) of the dense encoding of the tiled vector.
void encode_periodic_words(Context& cx, const std::complex<double>* z, int period, int count, int nl, double scale,
                           uint64_t* host_out) {
    const int D = period, D2 = 2 * period;
    if (D < 4 || (D & (D - 1)) || (cx.N / 2) % D || D > 2048 || count < 1 || nl < 1 || nl > cx.L)
        throw Error("encode_periodic: period must be a power of two in [4, 2048] dividing N/2; 1 <= limbs <= L", -1);
    std::vector<double> flat((size_t)count * D2);
    const double maxv = (double)((1ull << 61) - 1);
#pragma omp parallel for schedule(dynamic, 4)
    for (int t = 0; t < count; t++) {
        std::vector<std::complex<double>> v(z + (size_t)t * D, z + (size_t)(t + 1) * D);
        fft_special_inv_small(v.data(), D, 4 * D);
        for (int k = 0; k < D; k++) {
            flat[(size_t)t * D2 + k] = v[k].real();
            flat[(size_t)t * D2 + k + D] = v[k].imag();
        }
    }
    for (double c : flat)
        if (std::fabs(c * scale) > maxv) throw Error("encode: value * scale exceeds 61 bits (refused)", -6);
    DevBuf dc(flat.size(), cx.stream), out((size_t)nl * D2 * count, cx.stream);
    CUDA_CHECK(cudaMemcpyAsync(dc.p, flat.data(), flat.size() * 8, cudaMemcpyHostToDevice, cx.stream));
    if (D2 == 2048) {
        const size_t smem = (size_t)(2 + 4) * 2048 * 8;
        CUDA_CHECK(cudaFuncSetAttribute(k_ptgen2048, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        k_ptgen2048<<<dim3((count + 3) / 4, nl), 256, smem, cx.stream>>>((const double*)dc.p, scale, out.p, count, nl,
                                                                        cx.L, (const ulonglong2*)cx.d_tw2, cx.d_rmont,
                                                                        cx.N, 0);
    } else {
        constexpr int IPC = 4;
        int logD2 = 0;
        while ((1 << logD2) < D2) logD2++;
        const size_t smem = (size_t)IPC * D2 * 8;
        if (smem > 48 * 1024)
            CUDA_CHECK(cudaFuncSetAttribute(k_ptgen<IPC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        k_ptgen<IPC><<<dim3((count + IPC - 1) / IPC, nl), 256, smem, cx.stream>>>((const double*)dc.p, scale, out.p,
                                                                                count, nl, cx.L, logD2, cx.d_tw,
                                                                                cx.d_twp, cx.N, 0);
    }
    CUDA_CHECK(cudaGetLastError());
    cx.launches++;
    // [limb][2D][count] on the device -> [count][limb][2D] for the caller
    std::vector<uint64_t> tr(out.words);
    CUDA_CHECK(cudaMemcpyAsync(tr.data(), out.p, tr.size() * 8, cudaMemcpyDeviceToHost, cx.stream));
    CUDA_CHECK(cudaStreamSynchronize(cx.stream));
    for (int l = 0; l < nl; l++)
        for (int k = 0; k < D2; k++)
            for (int t = 0; t < count; t++)
                host_out[((size_t)t * nl + l) * D2 + k] = tr[((size_t)l * D2 + k) * count + t];
}

std::vector<int> matvec_rotations(int D, int b1) {
    std::vector<int> r;
    for (int j = 1; j < b1; j++) r.push_back(j);
    for (int j = 0; j < b1; j++) r.push_back(j - D);
    for (int g = 1; g < D / b1; g++) r.push_back(g * b1);
    return r;
}

// the 2 b1 babies of one input in QP: P rot(u, j) (j = 0..b1-1) then P rot(u, j - D)
struct BabySet {
    int D = 0, b1 = 0, nl = 0;
    double scale = 0;
    DevBuf pq;              // [2 b1][2][nl + K][N]
    mutable DevBuf split;   // tensor-core image: [nl + K][N/32][8 byte slices][64 Kp] (built on first use)
    mutable int split_Kp = 0;
};

void matvec_babies(Context& cx, const Ciphertext& u, int D, int b1, BabySet& bs) {
    ProfScope op(cx, "op:matvec_babies", 0);
    if (u.nl < 2) throw Error("matvec: no level left", -4);
    const int N = cx.N, K = cx.K, L = cx.L, nl = u.nl, ne = nl + K, dn = cx.dnum(nl);
    cudaStream_t st = cx.stream;
    bs.D = D; bs.b1 = b1; bs.nl = nl; bs.scale = u.scale;
    bs.pq = DevBuf((size_t)2 * b1 * 2 * ne * N, st);
    DevBuf ext = modup(cx, u.c(1), nl);
    BabyArgs ba{};
    for (int i = 0; i < nl; i++) {
        uint64_t pm = 1;
        for (int k = 0; k < K; k++) pm = host_mulmod(pm, cx.mods[L + k] % cx.mods[i], cx.mods[i]);
        ba.pw[i] = pm;
        ba.pwp[i] = shoup_of(pm, cx.mods[i]);
    }
    const int nb = 2 * b1;
    for (int b0 = 0; b0 < nb; b0 += 64) {
        const int B = std::min(64, nb - b0);
        for (int b = 0; b < B; b++) {
            const int t = b0 + b, Y = t / b1, j = t % b1;
            const uint64_t k = rot_index(cx, Y == 0 ? j : j - D);
            ba.perm[b] = k;
            ba.fkey[b] = k == 1 ? nullptr : forward_key(cx, k);
        }
        ProfScope ps(cx, "baby_pq", 8.0 * N * B * ((double)dn * ne * 2 + 2 * ne));
        const int per = std::max(1, cx.baby_limbs);
        k_baby_pq<<<dim3(N / 256, (ne + per - 1) / per, B), 256, 0, st>>>(ext.p, u.c(0), u.c(1), ba,
                                                                     bs.pq.p + (size_t)b0 * 2 * ne * N, nl, ne, dn, L,
                                                                     K, cx.logN, per);
        CUDA_CHECK(cudaGetLastError());
        cx.launches++;
        cx.ks_count += B;
        cx.ks_limbs += (long long)B * nl;
    }
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

// ModDown of B polynomial pairs in QP ([B][2][nl+K][N], destroyed) into out [B][2][nl][N]
static void moddown_many(Context& cx, uint64_t* in, int B, int nl, uint64_t* out) {
    const int N = cx.N, K = cx.K, L = cx.L, ne = nl + K;
    cudaStream_t st = cx.stream;
    LimbMap pm{};
    pm.base = in + (size_t)nl * N; pm.poly_stride = (long long)ne * N; pm.nl = K;
    pm.split = 0; pm.off0 = 0; pm.off1 = L;
    ntt(cx, pm, 2 * B, true, st);
    DevBuf y((size_t)B * 2 * nl * N, st);
    {
        ProfScope ps(cx, "moddown_bconv", 8.0 * N * B * (2 * K + 2 * nl));
        launch_pdl(cx, k_moddown_bconv, dim3(N / 256, 2, B), dim3(256), 0, st, in, y.p, cx.d_md, nl, ne, L, K, cx.logN,
                                                             (long long)2 * ne * N, (long long)2 * nl * N);
    }
    ntt(cx, cx.qmap(y.p, nl, (long long)nl * N), 2 * B, false, st);
    for (int b0 = 0; b0 < B; b0 += 64) {
        const int Bc = std::min(64, B - b0);
        FinalBatch fb{};
        for (int b = 0; b < Bc; b++) {
            fb.out0[b] = out + (size_t)(b0 + b) * 2 * nl * N;
            fb.out1[b] = fb.out0[b] + (size_t)nl * N;
            fb.perm[b] = 1;
        }
        ProfScope ps(cx, "moddown_final", 8.0 * N * nl * Bc * 6);
        launch_pdl(cx, k_moddown_final_b, dim3(N / 256, nl, 2 * Bc), dim3(256), 0, st, in + (size_t)b0 * 2 * ne * N,
                                                                     y.p + (size_t)b0 * 2 * nl * N, nullptr, fb,
                                                                     cx.d_md, nl, ne, L, K, cx.logN);
    }
    CUDA_CHECK(cudaGetLastError());
    cx.launches += 2 + (B + 63) / 64;
}

void matvec_apply(Context& cx, const MatvecPlan& pl, const BabySet* const* sets, Ciphertext& out) {
    ProfScope op(cx, "op:matvec_apply", 0);
    const int N = cx.N, S = pl.nsets, b1 = pl.b1, G = pl.G, D = pl.D, K = cx.K;
    const int nl = sets[0]->nl, ne = nl + K;
    for (int s = 0; s < S; s++)
        if (sets[s]->nl != nl || std::fabs(sets[s]->scale / sets[0]->scale - 1) > 1e-9 || sets[s]->D != D ||
            sets[s]->b1 != b1)
            throw Error("matvec: input chunks must share level, scale and baby geometry", -4);
    if (S > kMaxSets) throw Error("matvec: too many input chunks for one launch", -1);
    cudaStream_t st = cx.stream;
    // plaintexts at this level: scale so that the rescaled output is canonical
    const double target = canon(cx, nl - 1);
    const double spt = target * (double)cx.mods[nl - 1] / sets[0]->scale;
    int logD2 = 0;
    while ((1 << logD2) < 2 * D) logD2++;
    int lr = 0;
    while ((N >> lr) > 2 * D) lr++;
    const int TW = std::min(32, 1 << lr);
    if (TW < 8) throw Error("matvec: D too large for the ring (need N / 2D >= 8)", -1);
    const int M = std::max(2, G);   // outputs I_g (a second, zero output when G = 1: the kernels pair outputs)
    if ((TW / 2) * (M / 2) > 512 || M % 2) throw Error("matvec: too many giant steps for one CTA", -1);
    const bool hit = pl.cached.p && pl.cached_nl == nl && pl.cached_spt == spt;
    DevBuf pts(hit ? 0 : (size_t)std::max(pl.P, 1) * ne * 2 * D, st);
    if (hit) {
        // words of an earlier call at this level and scale
    } else if (pl.P > 0 && logD2 == 11) {
        const size_t smem = (size_t)(2 + 4) * 2048 * 8;
        CUDA_CHECK(cudaFuncSetAttribute(k_ptgen2048, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        ProfScope ps(cx, "ptgen", 8.0 * pl.P * 2 * D * (1 + ne));
        k_ptgen2048<<<dim3((pl.P + 3) / 4, ne), 256, smem, st>>>((const double*)pl.coef.p, spt, pts.p, pl.P, nl, cx.L,
                                                                (const ulonglong2*)cx.d_tw2, cx.d_rmont, N, 1);
        CUDA_CHECK(cudaGetLastError());
        cx.launches++;
    } else if (pl.P > 0) {
        constexpr int IPC = 4;
        const size_t smem = (size_t)IPC * 2 * D * 8;
        if (smem > 48 * 1024)
            CUDA_CHECK(cudaFuncSetAttribute(k_ptgen<IPC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        ProfScope ps(cx, "ptgen", 8.0 * pl.P * 2 * D * (1 + ne));
        k_ptgen<IPC><<<dim3((pl.P + IPC - 1) / IPC, ne), 256, smem, st>>>(
            (const double*)pl.coef.p, spt, pts.p, pl.P, nl, cx.L, logD2, cx.d_tw, cx.d_twp, N, 1);
        CUDA_CHECK(cudaGetLastError());
        cx.launches++;
    }
    if (!hit && cx.pt_cache && pl.P > 0) {
        // keep these words for the next call if the budget allows (replacing an entry of
        // another level or scale)
        const long long bytes = (long long)(pts.words * 8);
        if (pl.cached.p) {
            cx.pt_cache_bytes -= (long long)(pl.cached.words * 8);
            pl.cached = DevBuf();
        }
        size_t fr = 0, tot = 0;
        CUDA_CHECK(cudaMemGetInfo(&fr, &tot));
        if ((long long)fr - bytes >= cx.pt_cache_reserve_mib * (1ll << 20)) {
            pl.cached = std::move(pts);
            pl.cached_nl = nl;
            pl.cached_spt = spt;
            cx.pt_cache_bytes += bytes;
        }
    }
    const uint64_t* ptsrc = pts.p ? pts.p : pl.cached.p;   // this call's words, or the cached ones
    DevBuf inner((size_t)M * 2 * ne * N, st);
    {
        GemmArgs a{};
        for (int s = 0; s < S; s++) a.babies[s] = sets[s]->pq.p;
        a.ids = (const int*)pl.d_ids.p;
        a.pts = ptsrc;
        a.out = inner.p;
        a.nsets = S; a.b1 = b1; a.G = G; a.M = M; a.nl = nl; a.ne = ne; a.L = cx.L; a.logN = cx.logN; a.lr = lr;
        a.D2 = 2 * D; a.P = std::max(pl.P, 1); a.TW = TW;
        const double bytes = 8.0 * N * ne * (2.0 * S * 2 * b1 + 2.0 * M) + 8.0 * pl.P * ne * 2 * D;
        if (cx.use_tc && TW == 32 && (M == 16 || M == 32 || M == 64)) {
            // tensor cores: babies split into byte slices once per baby set, plaintext words packed
            // per call, both in the shared-memory image the product kernel bulk-copies.  8
            // accumulator tiles of M columns; a 512-column tile takes all of an SM's tensor
            // memory, so its CTAs ask for enough shared memory to run one per SM.
            const int Kp = (2 * b1 + 31) / 32 * 32;
            const int R = N / 32;
            const uint32_t tcols = M == 16 ? 128u : M == 32 ? 256u : 512u;
            Tc2Args t{};
            for (int s = 0; s < S; s++) {
                const BabySet& b = *sets[s];
                if (!b.split.p || b.split_Kp != Kp) {
                    const size_t bytes = (size_t)ne * R * 8 * 64 * Kp;
                    b.split = DevBuf(bytes / 8, st);
                    b.split_Kp = Kp;
                    const size_t sm = (size_t)8 * 64 * Kp;
                    if (sm > 48 * 1024)
                        CUDA_CHECK(cudaFuncSetAttribute(k_tc_split_babies, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
                    ProfScope ps(cx, "tc_split", 2.0 * bytes);
                    k_tc_split_babies<<<dim3(R, ne), 256, sm, st>>>(b.pq.p, (uint8_t*)b.split.p, 2 * b1, Kp, ne, nl,
                                                                    cx.L, cx.logN);
                    CUDA_CHECK(cudaGetLastError());
                    cx.launches++;
                }
                t.bsplit[s] = (const uint8_t*)b.split.p;
            }
            const size_t wblk = (size_t)8 * M * Kp;
            DevBuf wpack((size_t)S * ne * 2 * D * wblk / 8, st);
            {
                if (wblk > 48 * 1024)
                    CUDA_CHECK(cudaFuncSetAttribute(k_tc_pack_w, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wblk));
                ProfScope ps(cx, "tc_pack_w", (double)S * ne * 2 * D * wblk + 8.0 * pl.P * ne * 2 * D);
                for (int s = 0; s < S; s++) {
                    k_tc_pack_w<<<dim3(2 * D, ne), 256, wblk, st>>>(ptsrc, (const int*)pl.d_ids.p,
                                                                  (uint8_t*)wpack.p + (size_t)s * ne * 2 * D * wblk, s, G,
                                                                  b1, Kp, M, 2 * D, std::max(pl.P, 1), nl, cx.L);
                    cx.launches++;
                }
                CUDA_CHECK(cudaGetLastError());
            }
            t.wpack = (const uint8_t*)wpack.p;
            t.out = inner.p;
            t.nsets = S; t.G = G; t.M = M; t.nl = nl; t.ne = ne; t.L = cx.L; t.logN = cx.logN; t.lr = lr;
            t.D2 = 2 * D;
            t.Kp = Kp;
            size_t smem = tc_smem_bytes(M, Kp);
            if (tcols == 512) smem = std::max<size_t>(smem, 120 * 1024);
            // int8 MACs the tensor cores are given: per CTA and input set, for each diagonal pair p of
            // the limb's byte width, one 128 x M x 32 MMA per (byte slice, 32-deep K chunk)
            double macs = 0.0;
            for (int e = 0; e < ne; e++) {
                uint64_t q = cx.mods[cx.ext_mod(nl, e)];
                int nbyte = 0;
                while (q) { nbyte++; q >>= 8; }
                for (int p = 0; p < nbyte; p++)
                    macs += (double)(std::min(nbyte - 1, 2 * p + 1) - std::max(0, 2 * p - (nbyte - 1)) + 1) * (Kp / 32);
            }
            macs *= (double)R * S * 128.0 * M * 32.0;
            ProfScope ps(cx, "bsgs_tc", bytes, macs);
            auto launch = [&](auto kern) {
                CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
                kern<<<dim3(R, ne), kTcThreads, smem, st>>>(t, tcols, cx.d_err);
            };
            if (M == 16) launch(k_bsgs_tc2<16>);
            else if (M == 32) launch(k_bsgs_tc2<32>);
            else launch(k_bsgs_tc2<64>);
        } else {
            const size_t smem = (size_t)kKc * (2 * TW + M) * 8;
            if (smem > 48 * 1024)
                CUDA_CHECK(cudaFuncSetAttribute(k_bsgs_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            ProfScope ps(cx, "bsgs_gemm", bytes);
            k_bsgs_gemm<<<dim3(N / TW, ne), (TW / 2) * (M / 2), smem, st>>>(a);
        }
        CUDA_CHECK(cudaGetLastError());
        cx.launches++;
    }
    // back to Q: one ModDown per giant input, then sum_g rot(I_g, g b1) (I_0 unrotated)
    DevBuf innq((size_t)G * 2 * nl * N, st);
    moddown_many(cx, inner.p, G, nl, innq.p);
    const double sc = sets[0]->scale * spt;
    std::vector<const uint64_t*> c0s, c1s;
    std::vector<int> steps;
    for (int g = 1; g < G; g++) {
        const uint64_t* p = innq.p + (size_t)g * 2 * nl * N;
        c0s.push_back(p);
        c1s.push_back(p + (size_t)nl * N);
        steps.push_back(g * b1);
    }
    Ciphertext acc;
    rotate_sum(cx, c0s.data(), c1s.data(), steps.data(), (int)steps.size(), nl, sc, innq.p,
               innq.p + (size_t)nl * N, acc);
    ct_rescale(cx, acc);
    acc.scale = target;
    out = std::move(acc);
}

}  // namespace fhe
