// engine.cu -- host side of the CKKS engine: context set-up, key material, encoding and
// the ciphertext operations, each a short sequence of launches on the context's stream.
//
// The operations replace the OpenFHE / FIDESlib CryptoContext calls of the reference's
// server (hpc_gpu_port/gpu_real_model.cu: EvalMult+RescaleInPlace :2629-2632, EvalRotate
// :2762-2765, EvalAdd :2692-2743, Encrypt/Decrypt :2202-2221, MakeCKKSPackedPlaintext
// :1577-1589) with the same semantics: FLEXIBLEAUTO scaling factors per level, rotation
// index 5^r mod 2N, conjugation 2N-1 (:1355-1369).
#include <omp.h>

#include <mutex>

#include <algorithm>
#include <cstdlib>
#include <cmath>
#include <cstring>

#include "engine.h"
#include "sampling.h"

namespace fhe {

// kernels.cu
__global__ void k_modup_bconv(const uint64_t*, const uint64_t*, uint64_t*, const uint64_t*, int, int, int, int, int,
                              long long, long long, long long);
__global__ void k_key_inner(const uint64_t*, const uint64_t*, uint64_t*, int, int, int, int, int, int);
__global__ void k_moddown_bconv(const uint64_t*, uint64_t*, const uint64_t*, int, int, int, int, int, long long,
                                long long);
__global__ void k_moddown_final(const uint64_t*, const uint64_t*, const uint64_t*, const uint64_t*, uint64_t*,
                                uint64_t*, const uint64_t*, int, int, int, int, int, uint64_t);
__global__ void k_rescale_lift(const uint64_t*, uint64_t*, int, int, int);
__global__ void k_mdr_bconv(const uint64_t*, uint64_t*, const uint64_t*, int, int, int, int, long long, long long);
__global__ void k_mdr_final(const uint64_t*, long long, const uint64_t*, const uint64_t*, const uint64_t*, uint64_t*,
                            long long, int, int, int, int);
__global__ void k_mdr_gather(const uint64_t*, long long, const uint64_t*, const uint64_t*, uint64_t*, int, int, int,
                             int);
__global__ void k_rescale_final(uint64_t*, long long, const uint64_t*, const uint64_t*, int, int, int, int);
__global__ void k_ewise(int, const uint64_t*, long long, const uint64_t*, long long, uint64_t*, long long, int, int);
__global__ void k_tensor(const uint64_t*, long long, const uint64_t*, long long, uint64_t*, long long, uint64_t*, int);
__global__ void k_signed_to_limbs(const int64_t*, uint64_t*, LimbMap, int);
__global__ void k_automorph(const uint64_t*, uint64_t*, uint64_t, int);
__global__ void k_keyb(const uint64_t*, const uint64_t*, const uint64_t*, const uint64_t*, const uint64_t*, uint64_t*,
                       int, int, int);
__global__ void k_mont(uint64_t*, int, int, int);
__global__ void k_encrypt(const uint64_t*, const uint64_t*, const uint64_t*, const uint64_t*, int, const uint64_t*,
                          uint64_t*, uint64_t*, int);
__global__ void k_decrypt(const uint64_t*, const uint64_t*, const uint64_t*, uint64_t*, int);
__global__ void k_pkb(const uint64_t*, const uint64_t*, const uint64_t*, uint64_t*, int);
__global__ void k_square(const uint64_t*, uint64_t*, int);


// ============================================================================ buffers ====
DevBuf::DevBuf(size_t w, cudaStream_t s) : words(w), st(s) {
    if (!w) return;
    cudaError_t e = cudaMallocAsync((void**)&p, w * sizeof(uint64_t), s);
    if (e == cudaErrorMemoryAllocation) {
        // the pool keeps freed buffers (the context sets no release threshold): hand the unused
        // ones back to the driver and try once more before failing
        (void)cudaGetLastError();
        int dev = 0;
        cudaMemPool_t pool;
        if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess &&
            cudaStreamSynchronize(s) == cudaSuccess && cudaMemPoolTrimTo(pool, 0) == cudaSuccess)
            e = cudaMallocAsync((void**)&p, w * sizeof(uint64_t), s);
    }
    if (e != cudaSuccess) p = nullptr;
    CUDA_CHECK(e);
}
DevBuf::~DevBuf() {
    if (p) cudaFreeAsync(p, st);
}
DevBuf& DevBuf::operator=(DevBuf&& o) noexcept {
    if (this != &o) {
        if (p) cudaFreeAsync(p, st);
        p = o.p; words = o.words; st = o.st;
        o.p = nullptr; o.words = 0;
    }
    return *this;
}

// ======================================================================= prime chain ====
static bool is_prime(uint64_t n) {
    static const uint64_t bases[] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37};
    if (n < 2) return false;
    for (uint64_t b : bases) {
        if (n == b) return true;
        if (n % b == 0) return false;
    }
    uint64_t d = n - 1;
    int s = 0;
    while (!(d & 1)) { d >>= 1; s++; }
    for (uint64_t b : bases) {
        uint64_t x = host_powmod(b, d, n);
        if (x == 1 || x == n - 1) continue;
        bool comp = true;
        for (int r = 1; r < s; r++) {
            x = host_mulmod(x, x, n);
            if (x == n - 1) { comp = false; break; }
        }
        if (comp) return false;
    }
    return true;
}

// OpenFHE-style selection (ParameterGenerationCKKSRNS): the top scaling prime = first prime
// = 1 mod 2N above 2^qbits, the ones below it alternating below/above it, q_0 the largest
// below 2^q0bits, special primes descending below 2^pbits skipping the Q chain.  With
// Bt > 0 the top Bt limbs (the levels a bootstrap consumes) form a second region of
// bbits-bit primes chosen the same way; q_1..q_{L-1-Bt} are the qbits-bit user primes.
static void gen_chain(int logN, int L, int q0bits, int qbits, int K, int pbits, int Bt, int bbits,
                      std::vector<uint64_t>& mods) {
    const uint64_t M = 2ull << logN;
    auto first = [&](int bits) {
        uint64_t x = 1ull << bits, q = x - (x % M) + 1;
        if (q <= x) q += M;
        while (!is_prime(q)) q += M;
        return q;
    };
    auto prev = [&](uint64_t q) { do { q -= M; } while (!is_prime(q)); return q; };
    auto next = [&](uint64_t q) { do { q += M; } while (!is_prime(q)); return q; };
    std::vector<uint64_t> q(L), p(K);
    auto region = [&](int top, int bottom, int bits) {   // fills q[bottom..top]
        if (top < bottom) return;
        uint64_t qs = first(bits), qp = qs, qn = qs;
        q[top] = qs;
        int cnt = 0;
        for (int i = top - 1; i >= bottom; i--) {
            if (cnt % 2 == 0) { qp = prev(qp); q[i] = qp; }
            else { qn = next(qn); q[i] = qn; }
            cnt++;
        }
    };
    if (L > 1) {
        region(L - 1 - Bt, 1, qbits);
        region(L - 1, L - Bt, bbits);
    }
    auto in = [](uint64_t v, const std::vector<uint64_t>& a, int from, int to) {
        for (int i = from; i < to; i++) if (a[i] == v) return true;
        return false;
    };
    uint64_t q0 = prev(first(q0bits));
    while (L > 1 && in(q0, q, 1, L)) q0 = prev(q0);
    q[0] = q0;
    uint64_t pp = first(pbits);
    for (int k = 0; k < K; k++) {
        pp = prev(pp);
        while (in(pp, q, 0, L) || in(pp, p, 0, k)) pp = prev(pp);
        p[k] = pp;
    }
    mods = q;
    mods.insert(mods.end(), p.begin(), p.end());
}

static uint64_t min_root(uint64_t q, int logN) {
    const uint64_t N = 1ull << logN, M = 2 * N;
    uint64_t psi = 0;
    for (uint64_t x = 2; x < q; x++) {
        uint64_t g = host_powmod(x, (q - 1) / M, q);
        if (host_powmod(g, N, q) == q - 1) { psi = g; break; }
    }
    uint64_t best = psi, sq = host_mulmod(psi, psi, q), cur = psi;
    for (uint64_t j = 1; j < M; j += 2) {
        if (cur < best) best = cur;
        cur = host_mulmod(cur, sq, q);
    }
    return best;
}

static uint32_t brev(uint32_t v, int bits) {
    uint32_t r = 0;
    for (int b = 0; b < bits; b++) { r = (r << 1) | (v & 1u); v >>= 1; }
    return r;
}

static uint64_t* dev_upload(const std::vector<uint64_t>& h) {
    uint64_t* d = nullptr;
    CUDA_CHECK(cudaMalloc((void**)&d, h.size() * sizeof(uint64_t)));
    CUDA_CHECK(cudaMemcpy(d, h.data(), h.size() * sizeof(uint64_t), cudaMemcpyHostToDevice));
    return d;
}

// ========================================================================== context ====
Context::Context(const Params& p) : prm(p) {
    if (p.logN < 12 || p.logN > 16) throw Error("logN must be in [12, 16]");
    if (p.L < 1 || p.K < 1 || p.L + p.K > kMaxMod || p.alpha < 1 || p.alpha > 8 || p.K > 8)
        throw Error("bad chain shape (need 1 <= L, 1 <= K <= 8, L + K <= 64, 1 <= alpha <= 8)");
    if (p.q0bits > 60 || p.qbits > 60 || p.pbits > 60 || p.qbits < 33 || p.boot_bits > 60 ||
        (p.boot_primes > 0 && p.boot_bits < 33))
        throw Error("moduli must be 33..60 bits");
    if (p.boot_primes < 0 || p.boot_primes > p.L - 1) throw Error("boot_primes must be in [0, L-1]");
    logN = p.logN; N = 1 << logN; L = p.L; K = p.K; alpha = p.alpha; device = p.device;
    dnum_top = dnum(L);
    CUDA_CHECK(cudaSetDevice(device));
    CUDA_CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    {
        // keep freed transient buffers in the stream-ordered pool across synchronisations
        // (the default threshold of 0 returns them to the driver at every sync)
        cudaMemPool_t pool;
        CUDA_CHECK(cudaDeviceGetDefaultMemPool(&pool, device));
        uint64_t keep = UINT64_MAX;
        CUDA_CHECK(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
    }
    CUDA_CHECK(cudaMalloc((void**)&d_err, sizeof(unsigned int)));
    CUDA_CHECK(cudaMemset(d_err, 0, sizeof(unsigned int)));
    gen_chain(logN, L, p.q0bits, p.qbits, K, p.pbits, p.boot_primes, p.boot_bits, mods);
    const int nm = L + K;
    mc.resize(nm);
    psi.resize(nm);
    std::vector<uint64_t> tw((size_t)nm * N), twp((size_t)nm * N), itw((size_t)nm * N), itwp((size_t)nm * N),
        ninv(2 * nm);
#pragma omp parallel for
    for (int m = 0; m < nm; m++) {
        const uint64_t q = mods[m];
        mc[m] = make_modconst(q);
        psi[m] = min_root(q, logN);
        const uint64_t pinv = host_invmod(psi[m], q);
        uint64_t x = 1, xi = 1;
        for (int i = 0; i < N; i++) {
            const uint32_t r = brev((uint32_t)i, logN);
            tw[(size_t)m * N + r] = x; twp[(size_t)m * N + r] = shoup_of(x, q);
            itw[(size_t)m * N + r] = xi; itwp[(size_t)m * N + r] = shoup_of(xi, q);
            x = host_mulmod(x, psi[m], q);
            xi = host_mulmod(xi, pinv, q);
        }
        const uint64_t ni = host_invmod((uint64_t)N % q, q);
        ninv[2 * m] = ni; ninv[2 * m + 1] = shoup_of(ni, q);
    }
    activate();
    // FHESSM_NTT_CLUSTER=0/1 overrides the default transform path at N = 2^16 (tuning and A/B runs)
    if (const char* e = std::getenv("FHESSM_NTT_CLUSTER")) ntt_cluster = std::atoi(e) != 0;
    d_tw = dev_upload(tw); d_twp = dev_upload(twp); d_itw = dev_upload(itw); d_itwp = dev_upload(itwp);
    {
        std::vector<uint64_t> f(2 * tw.size()), v(2 * itw.size());
        for (size_t i = 0; i < tw.size(); i++) { f[2 * i] = tw[i]; f[2 * i + 1] = twp[i]; }
        for (size_t i = 0; i < itw.size(); i++) { v[2 * i] = itw[i]; v[2 * i + 1] = itwp[i]; }
        d_tw2 = dev_upload(f);
        d_itw2 = dev_upload(v);
        // the row kernel's table: block bg, slot 2^sp - 1 + j (stage sp of the last four), thread r0
        const int nb = N >> 8, S1 = logN - 8;
        std::vector<uint64_t> fr((size_t)nm * nb * 240 * 2), vr(fr.size());
#pragma omp parallel for
        for (int m = 0; m < nm; m++)
            for (int bg = 0; bg < nb; bg++)
                for (int sp = 0; sp < 4; sp++)
                    for (int j = 0; j < (1 << sp); j++)
                        for (int r0 = 0; r0 < 16; r0++) {
                            const size_t src = (size_t)m * N + (1u << (S1 + 4 + sp)) + ((size_t)bg << (4 + sp)) +
                                               ((size_t)r0 << sp) + j;
                            const size_t dst = ((size_t)m * nb + bg) * 240 + (size_t)((1 << sp) - 1 + j) * 16 + r0;
                            fr[2 * dst] = tw[src]; fr[2 * dst + 1] = twp[src];
                            vr[2 * dst] = itw[src]; vr[2 * dst + 1] = itwp[src];
                        }
        d_twrow = dev_upload(fr);
        d_itwrow = dev_upload(vr);
    }
    d_ninv = dev_upload(ninv);
    {
        std::vector<uint64_t> rm(2 * nm);
        for (int m = 0; m < nm; m++) {
            rm[2 * m] = (uint64_t)(((unsigned __int128)1 << 64) % mods[m]);
            rm[2 * m + 1] = shoup_of(rm[2 * m], mods[m]);
        }
        d_rmont = dev_upload(rm);
    }
    // FLEXIBLEAUTO scaling factors: scale_at[top] = q_{top-1}; scale_at[nl] = scale_at[nl+1]^2 / q_nl,
    // anchored separately at the top of each prime region (user region, bootstrap region)
    scale_at.assign(L + 1, 0.0);
    auto fill = [&](int top, int bottom) {
        scale_at[top] = (double)mods[top - 1];
        for (int nl = top - 1; nl >= bottom; nl--) scale_at[nl] = scale_at[nl + 1] * scale_at[nl + 1] / (double)mods[nl];
    };
    const int utop = L - p.boot_primes;   // limb count at the top of the user region
    if (p.boot_primes == 0) fill(L, 1);
    else { fill(L, utop + 1); fill(utop, 1); }
    // ModDown constants
    {
        std::vector<uint64_t> md(2 * K + (size_t)L * K * 2 + (size_t)L * 2);
        for (int k = 0; k < K; k++) {
            const uint64_t pk = mods[L + k];
            uint64_t ph = 1;
            for (int b = 0; b < K; b++) if (b != k) ph = host_mulmod(ph, mods[L + b] % pk, pk);
            const uint64_t inv = host_invmod(ph, pk);
            md[2 * k] = inv; md[2 * k + 1] = shoup_of(inv, pk);
        }
        for (int i = 0; i < L; i++) {
            const uint64_t qi = mods[i];
            uint64_t P = 1;
            for (int k = 0; k < K; k++) {
                uint64_t v = 1;
                for (int b = 0; b < K; b++) if (b != k) v = host_mulmod(v, mods[L + b] % qi, qi);
                md[2 * K + ((size_t)i * K + k) * 2] = v;
                md[2 * K + ((size_t)i * K + k) * 2 + 1] = shoup_of(v, qi);
                P = host_mulmod(P, mods[L + k] % qi, qi);
            }
            const uint64_t pinv = host_invmod(P, qi);
            md[2 * K + (size_t)L * K * 2 + 2 * i] = pinv;
            md[2 * K + (size_t)L * K * 2 + 2 * i + 1] = shoup_of(pinv, qi);
        }
        d_md = dev_upload(md);
    }
    // rescale constants: (q_l^-1 mod q_i, shoup) at [l][i]
    {
        std::vector<uint64_t> rs((size_t)L * L * 2, 0);
        for (int l = 1; l < L; l++)
            for (int i = 0; i < l; i++) {
                const uint64_t inv = host_invmod(mods[l] % mods[i], mods[i]);
                rs[((size_t)l * L + i) * 2] = inv;
                rs[((size_t)l * L + i) * 2 + 1] = shoup_of(inv, mods[i]);
            }
        d_rs = dev_upload(rs);
    }
}

Context::~Context() {
    cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    boot.reset();
    pt_i.reset();
    ptcache.clear();
    rlk.reset();
    rot_keys.clear();
    sk = DevBuf();
    pk = DevBuf();
    if (stream) cudaStreamSynchronize(stream);
    for (auto* p : {d_tw, d_twp, d_itw, d_itwp, d_ninv, d_md, d_rs, d_tw2, d_itw2, d_twrow, d_itwrow, d_rmont})
        if (p) cudaFree(p);
    if (d_err) cudaFree(d_err);
    for (auto& e : stage_ev)
        if (e) cudaEventDestroy(e);
    if (stage) cudaFreeHost(stage);
    for (auto& kv : modup_tab) cudaFree(kv.second);
    for (auto& kv : mdr_tab) cudaFree(kv.second);
    if (stream) cudaStreamDestroy(stream);
}

const uint64_t* Context::modup_table(int nl) {
    auto it = modup_tab.find(nl);
    if (it != modup_tab.end()) return it->second;
    const int dn = dnum(nl), ne = nl + K;
    std::vector<uint64_t> tab((size_t)dn * alpha * 2 + (size_t)dn * ne * alpha * 2, 0);
    for (int j = 0; j < dn; j++) {
        const int lo = j * alpha, sz = std::min(alpha, nl - lo);
        for (int a = 0; a < sz; a++) {
            const uint64_t qi = mods[lo + a];
            uint64_t qh = 1;
            for (int b = 0; b < sz; b++) if (b != a) qh = host_mulmod(qh, mods[lo + b] % qi, qi);
            const uint64_t inv = host_invmod(qh, qi);
            tab[((size_t)j * alpha + a) * 2] = inv;
            tab[((size_t)j * alpha + a) * 2 + 1] = shoup_of(inv, qi);
        }
        for (int e = 0; e < ne; e++) {
            if (e >= lo && e < lo + sz) continue;
            const uint64_t t = mods[ext_mod(nl, e)];
            for (int a = 0; a < sz; a++) {
                uint64_t v = 1;
                for (int b = 0; b < sz; b++) if (b != a) v = host_mulmod(v, mods[lo + b] % t, t);
                const size_t o = (size_t)dn * alpha * 2 + (((size_t)j * ne + e) * alpha + a) * 2;
                tab[o] = v;
                tab[o + 1] = mont_of(v, t);
            }
        }
    }
    uint64_t* d = dev_upload(tab);
    modup_tab[nl] = d;
    return d;
}

// ModDown and rescale in one division by M = q_l P (l = nl - 1): see k_mdr_bconv for the layout
const uint64_t* Context::mdr_table(int nl) {
    auto it = mdr_tab.find(nl);
    if (it != mdr_tab.end()) return it->second;
    const int J = K + 1, nq = nl - 1, l = nl - 1;
    std::vector<uint64_t> m(J);
    m[0] = mods[l];
    for (int k = 0; k < K; k++) m[1 + k] = mods[L + k];
    auto hat_mod = [&](int j, uint64_t t) {   // (M / m_j) mod t
        uint64_t v = 1;
        for (int u = 0; u < J; u++) if (u != j) v = host_mulmod(v, m[u] % t, t);
        return v;
    };
    std::vector<uint64_t> tab((size_t)2 * J + (size_t)nq * J * 2 + 6 * (size_t)nq + 2 + J, 0);
    for (int j = 0; j < J; j++) {
        const uint64_t inv = host_invmod(hat_mod(j, m[j]), m[j]);
        tab[2 * j] = inv;
        tab[2 * j + 1] = shoup_of(inv, m[j]);
    }
    for (int i = 0; i < nq; i++) {
        const uint64_t qi = mods[i];
        for (int j = 0; j < J; j++) {
            const uint64_t v = hat_mod(j, qi);
            tab[2 * J + ((size_t)i * J + j) * 2] = v;
            tab[2 * J + ((size_t)i * J + j) * 2 + 1] = shoup_of(v, qi);
        }
        uint64_t Mq = 1, Pq = 1;
        for (int u = 0; u < J; u++) Mq = host_mulmod(Mq, m[u] % qi, qi);
        for (int k = 0; k < K; k++) Pq = host_mulmod(Pq, mods[L + k] % qi, qi);
        const uint64_t minv = host_invmod(Mq, qi);
        tab[2 * J + (size_t)nq * J * 2 + 2 * i] = minv;
        tab[2 * J + (size_t)nq * J * 2 + 2 * i + 1] = shoup_of(minv, qi);
        tab[2 * J + (size_t)nq * J * 2 + 2 * nq + 2 * i] = Pq;
        tab[2 * J + (size_t)nq * J * 2 + 2 * nq + 2 * i + 1] = shoup_of(Pq, qi);
    }
    uint64_t Pl = 1;
    for (int k = 0; k < K; k++) Pl = host_mulmod(Pl, mods[L + k] % mods[l], mods[l]);
    tab[2 * J + (size_t)nq * J * 2 + 4 * (size_t)nq] = Pl;
    tab[2 * J + (size_t)nq * J * 2 + 4 * (size_t)nq + 1] = shoup_of(Pl, mods[l]);
    const size_t mo = 2 * J + (size_t)nq * J * 2 + 4 * (size_t)nq + 2;   // M mod q_i, then 1/m_j
    for (int i = 0; i < nq; i++) {
        uint64_t Mq = 1;
        for (int u = 0; u < J; u++) Mq = host_mulmod(Mq, m[u] % mods[i], mods[i]);
        tab[mo + 2 * i] = Mq;
        tab[mo + 2 * i + 1] = shoup_of(Mq, mods[i]);
    }
    for (int j = 0; j < J; j++) {
        const double r = 1.0 / (double)m[j];
        std::memcpy(&tab[mo + 2 * (size_t)nq + j], &r, sizeof r);
    }
    uint64_t* d = dev_upload(tab);
    mdr_tab[nl] = d;
    return d;
}

LimbMap Context::qmap(uint64_t* base, int nl, long long poly_stride) const {
    LimbMap mp{};
    mp.base = base; mp.poly_stride = poly_stride; mp.nl = nl; mp.skip_alpha = 0; mp.skip_nq = 0;
    mp.split = nl; mp.off0 = 0; mp.off1 = 0;
    return mp;
}
LimbMap Context::extmap(uint64_t* base, int nl, long long poly_stride) const {
    LimbMap mp{};
    mp.base = base; mp.poly_stride = poly_stride; mp.nl = nl + K; mp.skip_alpha = 0; mp.skip_nq = nl;
    mp.split = nl; mp.off0 = 0; mp.off1 = L;
    return mp;
}

static inline dim3 g2(const Context& cx, int y, int z = 1) { return dim3(cx.N / 256, y, z); }

// ==================================================================== key switching ====
static void moddown(Context& cx, uint64_t* ip, int nl, const uint64_t* add0, const uint64_t* add1, uint64_t* out0,
                    uint64_t* out1, uint64_t perm_k) {
    const int N = cx.N, K = cx.K, L = cx.L, ne = nl + K;
    cudaStream_t st = cx.stream;
    LimbMap pm{};
    pm.base = ip + (size_t)nl * N; pm.poly_stride = (long long)ne * N; pm.nl = K;
    pm.split = 0; pm.off0 = 0; pm.off1 = L;
    ntt(cx, pm, 2, true, st);
    DevBuf y((size_t)2 * nl * N, st);
    {
        ProfScope ps(cx, "moddown_bconv", 8.0 * N * (2 * K + 2 * nl));
        launch_pdl(cx, k_moddown_bconv, g2(cx, 2), dim3(256), 0, st, ip, y.p, cx.d_md, nl, ne, L, K, cx.logN, 0, 0);
    }
    ntt(cx, cx.qmap(y.p, nl, (long long)nl * N), 2, false, st);
    {
        ProfScope ps(cx, "moddown_final", 8.0 * N * nl * (6 + (add0 ? 1 : 0) + (add1 ? 1 : 0)));
        launch_pdl(cx, k_moddown_final, g2(cx, nl, 2), dim3(256), 0, st, ip, y.p, add0, add1, out0, out1, cx.d_md, nl, ne, L, K,
                                                       cx.logN, perm_k);
    }
    CUDA_CHECK(cudaGetLastError());
    cx.launches += 2;
}

// ModUp of d (nl limbs, eval form): ext [dnum][nl+K][N], eval form
static DevBuf modup(Context& cx, const uint64_t* d, int nl) {
    const int N = cx.N, K = cx.K, ne = nl + K, dn = cx.dnum(nl);
    cudaStream_t st = cx.stream;
    DevBuf dc((size_t)nl * N, st);
    CUDA_CHECK(cudaMemcpyAsync(dc.p, d, (size_t)nl * N * 8, cudaMemcpyDeviceToDevice, st));
    ntt(cx, cx.qmap(dc.p, nl, (long long)nl * N), 1, true, st);
    DevBuf ext((size_t)dn * ne * N, st);
    {
        ProfScope ps(cx, "modup_bconv", 8.0 * N * (2 * nl + (double)dn * ne));
        launch_pdl(cx, k_modup_bconv, g2(cx, dn), dim3(256), 0, st, dc.p, d, ext.p, cx.modup_table(nl), nl, ne, cx.alpha, cx.L,
                                                  cx.logN, 0, 0, 0);
    }
    LimbMap em = cx.extmap(ext.p, nl, (long long)ne * N);
    em.skip_alpha = cx.alpha;
    ntt(cx, em, dn, false, st);
    CUDA_CHECK(cudaGetLastError());
    cx.launches += 1;
    return ext;
}

static void inner_moddown(Context& cx, const DevBuf& ext, int nl, const SwitchKey& key, const uint64_t* add0,
                          const uint64_t* add1, uint64_t* out0, uint64_t* out1, uint64_t perm_k) {
    const int N = cx.N, K = cx.K, ne = nl + K, dn = cx.dnum(nl);
    cudaStream_t st = cx.stream;
    cx.ks_count++;
    cx.ks_limbs += nl;
    DevBuf ip((size_t)2 * ne * N, st);
    {
        ProfScope ps(cx, "key_inner", 8.0 * N * ((double)dn * ne * 3 + 2 * ne));
        launch_pdl(cx, k_key_inner, g2(cx, ne), dim3(256), 0, st, ext.p, key.buf.p, ip.p, nl, ne, dn, cx.L, K, cx.logN);
    }
    cx.launches += 1;
    moddown(cx, ip.p, nl, add0, add1, out0, out1, perm_k);
}

void keyswitch(Context& cx, const uint64_t* d, int nl, const SwitchKey& key, const uint64_t* add0,
               const uint64_t* add1, uint64_t* out0, uint64_t* out1, uint64_t perm_k) {
    DevBuf ext = modup(cx, d, nl);
    inner_moddown(cx, ext, nl, key, add0, add1, out0, out1, perm_k);
}

// ======================================================================= ciphertexts ====
Ciphertext ct_alloc(Context& cx, int nl) {
    Ciphertext c;
    c.buf = DevBuf((size_t)2 * nl * cx.N, cx.stream);
    c.nl = nl;
    c.stride = (size_t)nl * cx.N;
    return c;
}

Ciphertext ct_copy(Context& cx, const Ciphertext& a) {
    Ciphertext c = ct_alloc(cx, a.nl);
    c.scale = a.scale;
    const size_t bytes = (size_t)a.nl * cx.N * 8;
    CUDA_CHECK(cudaMemcpyAsync(c.c(0), a.c(0), bytes, cudaMemcpyDeviceToDevice, cx.stream));
    CUDA_CHECK(cudaMemcpyAsync(c.c(1), a.c(1), bytes, cudaMemcpyDeviceToDevice, cx.stream));
    return c;
}

static void ensure_out(Context& cx, Ciphertext& out, int nl) {
    if (!out.buf.p || out.stride < (size_t)nl * cx.N) out = ct_alloc(cx, nl);
    out.nl = nl;
}

static void check_same(const Ciphertext& a, const Ciphertext& b, const char* op) {
    if (a.nl != b.nl) throw Error(std::string(op) + ": level mismatch (" + std::to_string(a.nl) + " vs " +
                                  std::to_string(b.nl) + " limbs)", -4);
    const double r = a.scale / b.scale;
    if (r > 1.0 + 1e-9 || r < 1.0 - 1e-9) throw Error(std::string(op) + ": scale mismatch", -4);
}

static void ewise(Context& cx, int op, const Ciphertext& a, const uint64_t* b, long long sb, int log_rep,
                  Ciphertext& out) {
    ensure_out(cx, out, a.nl);
    ProfScope ps(cx, "ewise", 8.0 * cx.N * a.nl * 2 * 3);
    launch_pdl(cx, k_ewise, g2(cx, a.nl, 2), dim3(256), 0, cx.stream, op, a.buf.p, (long long)a.stride, b, sb, out.buf.p,
                                                    (long long)out.stride, log_rep, cx.logN);
    CUDA_CHECK(cudaGetLastError());
    cx.launches++;
}

void ct_add(Context& cx, const Ciphertext& a, const Ciphertext& b, Ciphertext& out) {
    check_same(a, b, "add");
    ewise(cx, EW_ADD, a, b.buf.p, (long long)b.stride, 0, out);
    out.scale = a.scale;
}
// addition of residues whose scales the caller has already made equal (no scale check)
void ct_add_raw(Context& cx, const Ciphertext& a, const Ciphertext& b, Ciphertext& out) {
    if (a.nl != b.nl) throw Error("add: level mismatch", -4);
    const double sc = a.scale;
    ewise(cx, EW_ADD, a, b.buf.p, (long long)b.stride, 0, out);
    out.scale = sc;
}
void ct_sub(Context& cx, const Ciphertext& a, const Ciphertext& b, Ciphertext& out) {
    check_same(a, b, "sub");
    ewise(cx, EW_SUB, a, b.buf.p, (long long)b.stride, 0, out);
    out.scale = a.scale;
}
void ct_mul_pt(Context& cx, const Ciphertext& a, const Plaintext& pt, Ciphertext& out) {
    if (pt.nl < a.nl) throw Error("mul_pt: plaintext has fewer limbs than the ciphertext", -4);
    const double sc = a.scale * pt.scale;
    ewise(cx, EW_MULPT, a, pt.buf.p, 0, pt.log_rep, out);
    out.scale = sc;
}
void ct_add_pt(Context& cx, const Ciphertext& a, const Plaintext& pt, Ciphertext& out) {
    if (pt.nl < a.nl) throw Error("add_pt: plaintext has fewer limbs than the ciphertext", -4);
    const double r = a.scale / pt.scale;
    if (r > 1.0 + 1e-9 || r < 1.0 - 1e-9) throw Error("add_pt: scale mismatch", -4);
    const double sc = a.scale;
    ewise(cx, EW_ADDPT, a, pt.buf.p, 0, pt.log_rep, out);
    out.scale = sc;
}

void ct_mul_relin(Context& cx, const Ciphertext& a, const Ciphertext& b, Ciphertext& out) {
    if (a.nl != b.nl) throw Error("mul: level mismatch", -4);
    if (!cx.rlk) throw Error("mul: no relinearisation key", -5);
    const int nl = a.nl;
    const double sc = a.scale * b.scale;
    Ciphertext t = ct_alloc(cx, nl);
    DevBuf d2((size_t)nl * cx.N, cx.stream);
    {
        ProfScope ps(cx, "tensor", 8.0 * cx.N * nl * 7);
        launch_pdl(cx, k_tensor, g2(cx, nl), dim3(256), 0, cx.stream, a.buf.p, (long long)a.stride, b.buf.p, (long long)b.stride,
                                                    t.buf.p, (long long)t.stride, d2.p, cx.logN);
    }
    CUDA_CHECK(cudaGetLastError());
    cx.launches++;
    keyswitch(cx, d2.p, nl, *cx.rlk, t.c(0), t.c(1), t.c(0), t.c(1), 1);
    t.scale = sc;
    out = std::move(t);
}

void ct_mul_relin_rescale(Context& cx, const Ciphertext& a, const Ciphertext& b, Ciphertext& out) {
    if (a.nl != b.nl) throw Error("mul: level mismatch", -4);
    if (a.nl < 2) throw Error("mul_rescale: no level left", -4);
    if (!cx.rlk) throw Error("mul: no relinearisation key", -5);
    if (cx.K > 6) throw Error("mul_relin_rescale: at most 6 special primes", -1);
    const int N = cx.N, K = cx.K, L = cx.L, nl = a.nl, ne = nl + K, dn = cx.dnum(nl), J = K + 1;
    cudaStream_t st = cx.stream;
    Ciphertext d = ct_alloc(cx, nl);
    DevBuf d2((size_t)nl * N, st);
    {
        ProfScope ps(cx, "tensor", 8.0 * N * nl * 7);
        launch_pdl(cx, k_tensor, g2(cx, nl), dim3(256), 0, st, a.buf.p, (long long)a.stride, b.buf.p, (long long)b.stride, d.buf.p,
                                             (long long)d.stride, d2.p, cx.logN);
    }
    DevBuf ext = modup(cx, d2.p, nl);
    DevBuf ip((size_t)2 * ne * N, st);
    {
        ProfScope ps(cx, "key_inner", 8.0 * N * ((double)dn * ne * 3 + 2 * ne));
        launch_pdl(cx, k_key_inner, g2(cx, ne), dim3(256), 0, st, ext.p, cx.rlk->buf.p, ip.p, nl, ne, dn, L, K, cx.logN);
    }
    cx.ks_count++;
    cx.ks_limbs += nl;
    const uint64_t* tab = cx.mdr_table(nl);
    DevBuf z((size_t)2 * J * N, st);
    {
        ProfScope ps(cx, "mdr_gather", 8.0 * N * 2 * (1 + 2 * J));
        launch_pdl(cx, k_mdr_gather, dim3(N / 256, J, 2), dim3(256), 0, st, d.buf.p, (long long)d.stride, ip.p, tab, z.p, nl, ne, K,
                                                          cx.logN);
    }
    LimbMap zm{};
    zm.base = z.p; zm.poly_stride = (long long)J * N; zm.nl = J;
    zm.split = 1; zm.off0 = nl - 1; zm.off1 = L;
    ntt(cx, zm, 2, true, st);
    DevBuf y((size_t)2 * (nl - 1) * N, st);
    {
        ProfScope ps(cx, "moddown_bconv", 8.0 * N * (2 * J + 2 * (nl - 1)));
        launch_pdl(cx, k_mdr_bconv, g2(cx, 2), dim3(256), 0, st, z.p, y.p, tab, nl, K, L, cx.logN, 0, 0);
    }
    ntt(cx, cx.qmap(y.p, nl - 1, (long long)(nl - 1) * N), 2, false, st);
    Ciphertext r = ct_alloc(cx, nl - 1);
    {
        ProfScope ps(cx, "moddown_final", 8.0 * N * (nl - 1) * 2 * 5);
        launch_pdl(cx, k_mdr_final, g2(cx, nl - 1, 2), dim3(256), 0, st, d.buf.p, (long long)d.stride, ip.p, y.p, tab, r.buf.p,
                                                       (long long)r.stride, nl, ne, K, cx.logN);
    }
    CUDA_CHECK(cudaGetLastError());
    cx.launches += 6;
    r.scale = a.scale * b.scale / (double)cx.mods[nl - 1];
    out = std::move(r);
}


// dst[p] = src[p] (one limb of N words each), p < npoly = gridDim.y
struct LimbPtrs {
    const uint64_t* src[kFuseMax];
};
__global__ void __launch_bounds__(256) k_gather_limbs(const __grid_constant__ LimbPtrs g, uint64_t* __restrict__ dst,
                                                      int logN) {
    pdl_wait();
    pdl_trigger();
    const int x = blockIdx.x * blockDim.x + threadIdx.x, p = blockIdx.y;
    dst[((size_t)p << logN) + x] = g.src[p][x];
}

// The rescale of K ciphertexts of one limb count as one batch: their dropped limbs gathered into
// one buffer and inverse-transformed by one launch pair, then one fused forward transform for
// all of them (ntt_rescale_n), kFuseMax / 2 ciphertexts at a time.  The words equal K calls of
// ct_rescale.
void ct_rescale_n(Context& cx, Ciphertext* const* a, int K) {
    if (K < 1) return;
    if (K == 1 || cx.logN < 13) {
        for (int k = 0; k < K; k++) ct_rescale(cx, *a[k]);
        return;
    }
    const int nl = a[0]->nl;
    for (int k = 0; k < K; k++)
        if (a[k]->nl != nl) throw Error("rescale_n: the ciphertexts differ in limb count", -4);
    if (nl < 2) throw Error("rescale: no limb left to drop", -4);
    const int N = cx.N, l = nl - 1;
    cudaStream_t st = cx.stream;
    for (int k0 = 0; k0 < K; k0 += kFuseMax / 2) {
        const int B = std::min(kFuseMax / 2, K - k0);
        LimbPtrs g{};
        uint64_t* dst[kFuseMax];
        for (int b = 0; b < B; b++) {
            Ciphertext& c = *a[k0 + b];
            g.src[2 * b] = c.c(0) + (size_t)l * N;
            g.src[2 * b + 1] = c.c(1) + (size_t)l * N;
            dst[2 * b] = c.c(0);
            dst[2 * b + 1] = c.c(1);
        }
        DevBuf t((size_t)2 * B * N, st);
        launch_pdl(cx, k_gather_limbs, dim3(N / 256, 2 * B), dim3(256), 0, st, g, t.p, cx.logN);
        CUDA_CHECK(cudaGetLastError());
        cx.launches++;
        LimbMap lm{};
        lm.base = t.p; lm.poly_stride = N; lm.nl = 1; lm.split = 1; lm.off0 = l; lm.off1 = 0;
        ntt(cx, lm, 2 * B, true, st);
        DevBuf y((size_t)2 * B * l * N, st);
        {
            ProfScope ps(cx, "rescale_ntt", 8.0 * N * B * (4.0 * l + 2));
            ntt_rescale_n(cx, t.p, N, dst, 2 * B, l, y.p, st);
        }
        for (int b = 0; b < B; b++) {
            a[k0 + b]->scale /= (double)cx.mods[l];
            a[k0 + b]->nl = l;
        }
    }
}

void ct_rescale(Context& cx, Ciphertext& a) {
    if (a.nl < 2) throw Error("rescale: no limb left to drop", -4);
    const int N = cx.N, l = a.nl - 1;
    cudaStream_t st = cx.stream;
    if (cx.logN >= 13) {
        // the dropped limb of both polynomials to coefficient form in place, then one fused
        // forward transform: lift on load, (a_i - y) q_l^-1 on store (ntt.cu, ntt_rescale)
        LimbMap lm{};
        lm.base = a.c(0) + (size_t)l * N; lm.poly_stride = (long long)a.stride; lm.nl = 1;
        lm.split = 1; lm.off0 = l; lm.off1 = 0;
        ntt(cx, lm, 2, true, st);
        DevBuf y((size_t)2 * l * N, st);
        {
            ProfScope ps(cx, "rescale_ntt", 8.0 * N * (4.0 * l + 2));
            ntt_rescale(cx, a.buf.p, (long long)a.stride, l, y.p, st);
        }
        a.scale /= (double)cx.mods[l];
        a.nl = l;
        return;
    }
    DevBuf last((size_t)2 * N, st);
    CUDA_CHECK(cudaMemcpyAsync(last.p, a.c(0) + (size_t)l * N, N * 8, cudaMemcpyDeviceToDevice, st));
    CUDA_CHECK(cudaMemcpyAsync(last.p + N, a.c(1) + (size_t)l * N, N * 8, cudaMemcpyDeviceToDevice, st));
    LimbMap lm{};
    lm.base = last.p; lm.poly_stride = N; lm.nl = 1; lm.split = 1; lm.off0 = l; lm.off1 = 0;
    ntt(cx, lm, 2, true, st);
    DevBuf y((size_t)2 * l * N, st);
    {
        ProfScope ps(cx, "rescale_lift", 8.0 * N * 2 * (1 + l));
        launch_pdl(cx, k_rescale_lift, g2(cx, l, 2), dim3(256), 0, st, last.p, y.p, l, l, cx.logN);
    }
    ntt(cx, cx.qmap(y.p, l, (long long)l * N), 2, false, st);
    {
        ProfScope ps(cx, "rescale_final", 8.0 * N * 2 * l * 3);
        launch_pdl(cx, k_rescale_final, g2(cx, l, 2), dim3(256), 0, st, a.buf.p, (long long)a.stride, y.p, cx.d_rs, l, l, cx.L,
                                                      cx.logN);
    }
    CUDA_CHECK(cudaGetLastError());
    cx.launches += 2;
    a.scale /= (double)cx.mods[l];
    a.nl = l;
}

void ct_level_drop(Context& cx, Ciphertext& a, int nl_target) {
    if (nl_target < 1 || nl_target > a.nl) throw Error("level_drop: bad target", -4);
    a.nl = nl_target;   // the remaining limbs are a valid encryption modulo the smaller Q
}

void ct_automorph(Context& cx, const Ciphertext& a, uint64_t k, Ciphertext& out) {
    auto it = cx.rot_keys.find(k);
    if (it == cx.rot_keys.end()) throw Error("automorphism: no key for index " + std::to_string(k), -5);
    Ciphertext t = ct_alloc(cx, a.nl);
    keyswitch(cx, a.c(1), a.nl, *it->second, a.c(0), nullptr, t.c(0), t.c(1), k);
    t.scale = a.scale;
    out = std::move(t);
}

uint64_t rot_index(const Context& cx, int r) {
    const int64_t n = cx.N / 2;
    int64_t rr = r % n;
    if (rr < 0) rr += n;
    return host_powmod(5, (uint64_t)rr, 2ull * cx.N);
}

void ct_rotate(Context& cx, const Ciphertext& a, int r, Ciphertext& out) {
    const uint64_t k = rot_index(cx, r);
    if (k == 1) { out = ct_copy(cx, a); return; }
    ct_automorph(cx, a, k, out);
}
void ct_conjugate(Context& cx, const Ciphertext& a, Ciphertext& out) { ct_automorph(cx, a, 2ull * cx.N - 1, out); }

// ct_rotate_hoisted: ksbatch.cu

// per-limb constant (v mod q_i) with shoup, uploaded to a small device buffer
static DevBuf limb_consts(Context& cx, const std::vector<uint64_t>& v, bool with_shoup) {
    std::vector<uint64_t> h(with_shoup ? 2 * v.size() : v.size());
    for (size_t i = 0; i < v.size(); i++) {
        if (with_shoup) { h[2 * i] = v[i]; h[2 * i + 1] = shoup_of(v[i], cx.mods[i]); }
        else h[i] = v[i];
    }
    DevBuf d(h.size(), cx.stream);
    CUDA_CHECK(cudaMemcpyAsync(d.p, h.data(), h.size() * 8, cudaMemcpyHostToDevice, cx.stream));
    CUDA_CHECK(cudaStreamSynchronize(cx.stream));   // h is a host temporary
    return d;
}

static uint64_t signed_mod(long double v, uint64_t q) {
    // round(v) mod q for |v| < 2^126
    const bool neg = v < 0;
    long double a = neg ? -v : v;
    a = std::floor(a + 0.5L);
    unsigned __int128 u = (unsigned __int128)a;
    uint64_t r = (uint64_t)(u % q);
    return neg ? (r ? q - r : 0) : r;
}

void limb_residues(const Context& cx, long double v, int nl, uint64_t* out) {
    for (int i = 0; i < nl; i++) out[i] = signed_mod(v, cx.mods[i]);
}

void apply_limb_const(Context& cx, const Ciphertext& a, const LimbConst& k, Ciphertext& out) {
    ProfScope ps(cx, "mul_const", 8.0 * cx.N * a.nl * 2 * 2);
    if (&out == &a) {
        launch_pdl(cx, k_mul_const, g2(cx, a.nl, 2), dim3(256), 0, cx.stream, a.buf.p, (long long)a.stride, a.buf.p, (long long)a.stride,
                                                            k, cx.logN);
    } else {
        Ciphertext t;
        ensure_out(cx, t, a.nl);
        launch_pdl(cx, k_mul_const, g2(cx, a.nl, 2), dim3(256), 0, cx.stream, a.buf.p, (long long)a.stride, t.buf.p, (long long)t.stride,
                                                            k, cx.logN);
        t.scale = a.scale;
        out = std::move(t);
    }
    CUDA_CHECK(cudaGetLastError());
    cx.launches++;
}

static LimbConst mul_consts(const Context& cx, long double c, int nl) {
    LimbConst k{};
    k.has_w = 1;
    limb_residues(cx, c, nl, k.w);
    for (int i = 0; i < nl; i++) k.wp[i] = shoup_of(k.w[i], cx.mods[i]);
    return k;
}

void ct_mul_const(Context& cx, const Ciphertext& a, double v, double scale, Ciphertext& out) {
    const double sc = a.scale * scale;
    apply_limb_const(cx, a, mul_consts(cx, (long double)v * (long double)scale, a.nl), out);
    out.scale = sc;
}

void ct_mul_int(Context& cx, const Ciphertext& a, int64_t v, Ciphertext& out) {
    const double sc = a.scale;
    apply_limb_const(cx, a, mul_consts(cx, (long double)v, a.nl), out);
    out.scale = sc;
}

// adds the constant v (every slot) at the ciphertext's scale: constant polynomial round(v*scale)
void ct_add_const(Context& cx, const Ciphertext& a, double v, Ciphertext& out) {
    LimbConst k{};
    k.has_add = 1;
    limb_residues(cx, (long double)v * (long double)a.scale, a.nl, k.add);
    const double sc = a.scale;
    apply_limb_const(cx, a, k, out);
    out.scale = sc;
}

// ========================================================================= encoding ====
// Special FFT over the rotation group 5^j mod M (slot j <-> root zeta^{5^j}), the CKKS
// canonical embedding restricted to the N/2 slots (Cheon-Kim-Kim-Song 2017).
struct FFTPlan {
    int n = 0, M = 0;
    std::vector<uint64_t> rg;
    std::vector<std::complex<double>> ksi;
};
static const FFTPlan& fft_plan(int n, int M) {
    static std::map<std::pair<int, int>, FFTPlan> plans;
    auto key = std::make_pair(n, M);
    auto it = plans.find(key);
    if (it != plans.end()) return it->second;
    FFTPlan p;
    p.n = n; p.M = M;
    p.rg.resize(n);
    uint64_t g = 1;
    for (int j = 0; j < n; j++) { p.rg[j] = g; g = (g * 5) % (uint64_t)M; }
    p.ksi.resize(M);
    for (int k = 0; k < M; k++) p.ksi[k] = std::complex<double>(std::cos(2.0 * M_PI * k / M), std::sin(2.0 * M_PI * k / M));
    return plans.emplace(key, std::move(p)).first->second;
}
static void bitrev_c(std::complex<double>* v, int n) {
    for (int i = 1, j = 0; i < n; i++) {
        int bit = n >> 1;
        for (; j & bit; bit >>= 1) j ^= bit;
        j ^= bit;
        if (i < j) std::swap(v[i], v[j]);
    }
}
static void fft_special_inv(std::complex<double>* v, int n, int M) {
    const FFTPlan& p = fft_plan(n, M);
    for (int len = n; len >= 1; len >>= 1) {
        const int lenh = len >> 1, lenq = len << 2;
        for (int i = 0; i < n; i += len)
            for (int j = 0; j < lenh; j++) {
                const uint64_t idx = ((uint64_t)lenq - (p.rg[j] % (uint64_t)lenq)) * (uint64_t)(M / lenq);
                const std::complex<double> u = v[i + j] + v[i + j + lenh];
                const std::complex<double> w = (v[i + j] - v[i + j + lenh]) * p.ksi[idx];
                v[i + j] = u;
                v[i + j + lenh] = w;
            }
    }
    bitrev_c(v, n);
    for (int i = 0; i < n; i++) v[i] /= (double)n;
}
static void fft_special_fwd(std::complex<double>* v, int n, int M) {
    const FFTPlan& p = fft_plan(n, M);
    bitrev_c(v, n);
    for (int len = 2; len <= n; len <<= 1) {
        const int lenh = len >> 1, lenq = len << 2;
        for (int i = 0; i < n; i += len)
            for (int j = 0; j < lenh; j++) {
                const uint64_t idx = (p.rg[j] % (uint64_t)lenq) * (uint64_t)(M / lenq);
                const std::complex<double> u = v[i + j], w = v[i + j + lenh] * p.ksi[idx];
                v[i + j] = u + w;
                v[i + j + lenh] = u - w;
            }
    }
}

// slots -> int64 coefficients with the reference encoder's rounding (periodic_encode.hpp:
// 186-237): scale, refuse when a coefficient needs more than 61 bits, llround.
static void encode_coeffs(Context& cx, const std::complex<double>* z, int nslots, double scale, int64_t* coef) {
    const int N = cx.N, n = N / 2;
    if (nslots > n || nslots < 1 || (n % nslots) != 0) throw Error("encode: slot count must divide N/2", -4);
    std::vector<std::complex<double>> v(n);
    for (int i = 0; i < n; i++) v[i] = z[i % nslots];   // a shorter vector repeats across the slots
    fft_special_inv(v.data(), n, 2 * N);
    const double maxv = (double)((1ull << 61) - 1);
    for (int i = 0; i < n; i++) {
        const double re = v[i].real() * scale, im = v[i].imag() * scale;
        if (std::fabs(re) > maxv || std::fabs(im) > maxv)
            throw Error("encode: value * scale exceeds 61 bits (refused)", -6);
        coef[i] = std::llround(re);
        coef[i + n] = std::llround(im);
    }
}

void upload_async(Context& cx, void* dev, const void* host, size_t bytes) {
    if (bytes > Context::kStageBytes) {   // larger than a slot: a plain copy, then wait for it
        CUDA_CHECK(cudaMemcpyAsync(dev, host, bytes, cudaMemcpyHostToDevice, cx.stream));
        CUDA_CHECK(cudaStreamSynchronize(cx.stream));
        return;
    }
    if (!cx.stage) {
        CUDA_CHECK(cudaHostAlloc((void**)&cx.stage, Context::kStageSlots * Context::kStageBytes,
                                 cudaHostAllocDefault));
        for (auto& e : cx.stage_ev) CUDA_CHECK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    }
    const int i = cx.stage_next;
    cx.stage_next = (i + 1) % Context::kStageSlots;
    if (cudaEventQuery(cx.stage_ev[i]) == cudaErrorNotReady) {   // the slot's last copy is still queued
        cx.host_waits++;
        CUDA_CHECK(cudaEventSynchronize(cx.stage_ev[i]));
    }
    uint8_t* slot = cx.stage + (size_t)i * Context::kStageBytes;
    std::memcpy(slot, host, bytes);
    CUDA_CHECK(cudaMemcpyAsync(dev, slot, bytes, cudaMemcpyHostToDevice, cx.stream));
    CUDA_CHECK(cudaEventRecord(cx.stage_ev[i], cx.stream));
}

Plaintext encode(Context& cx, const std::complex<double>* z, int nslots, int nl, double scale) {
    if (nl < 1 || nl > cx.L) throw Error("encode: bad level", -4);
    const int N = cx.N;
    std::vector<int64_t> coef(N);
    encode_coeffs(cx, z, nslots, scale, coef.data());
    DevBuf dc((size_t)N, cx.stream);
    upload_async(cx, dc.p, coef.data(), (size_t)N * 8);
    Plaintext pt;
    pt.buf = DevBuf((size_t)nl * N, cx.stream);
    pt.nl = nl;
    pt.scale = scale;
    LimbMap mp = cx.qmap(pt.buf.p, nl, (long long)nl * N);
    k_signed_to_limbs<<<g2(cx, nl), 256, 0, cx.stream>>>((const int64_t*)dc.p, pt.buf.p, mp, cx.logN);
    CUDA_CHECK(cudaGetLastError());
    ntt(cx, mp, 1, false, cx.stream);
    cx.launches += 1;
    cx.pt_encodes++;
    return pt;
}

// the same plaintext over the extended basis: nl Q limbs then the K special limbs
Plaintext encode_pq(Context& cx, const std::complex<double>* z, int nslots, int nl, double scale) {
    if (nl < 1 || nl > cx.L) throw Error("encode: bad level", -4);
    const int N = cx.N, ne = nl + cx.K;
    std::vector<int64_t> coef(N);
    encode_coeffs(cx, z, nslots, scale, coef.data());
    DevBuf dc((size_t)N, cx.stream);
    upload_async(cx, dc.p, coef.data(), (size_t)N * 8);
    Plaintext pt;
    pt.buf = DevBuf((size_t)ne * N, cx.stream);
    pt.nl = ne;
    pt.scale = scale;
    LimbMap mp = cx.extmap(pt.buf.p, nl, (long long)ne * N);
    k_signed_to_limbs<<<g2(cx, ne), 256, 0, cx.stream>>>((const int64_t*)dc.p, pt.buf.p, mp, cx.logN);
    CUDA_CHECK(cudaGetLastError());
    ntt(cx, mp, 1, false, cx.stream);
    cx.launches += 1;
    cx.pt_encodes++;
    return pt;
}

void decode(Context& cx, const Plaintext& pt, std::complex<double>* z) {
    const int N = cx.N, n = N / 2;
    DevBuf t((size_t)N, cx.stream);
    CUDA_CHECK(cudaMemcpyAsync(t.p, pt.buf.p, N * 8, cudaMemcpyDeviceToDevice, cx.stream));
    LimbMap mp = cx.qmap(t.p, 1, N);
    ntt(cx, mp, 1, true, cx.stream);
    std::vector<uint64_t> h(N);
    CUDA_CHECK(cudaMemcpyAsync(h.data(), t.p, N * 8, cudaMemcpyDeviceToHost, cx.stream));
    CUDA_CHECK(cudaStreamSynchronize(cx.stream));
    const uint64_t q = cx.mods[0];
    std::vector<std::complex<double>> v(n);
    for (int i = 0; i < n; i++) {
        const uint64_t a = h[i], b = h[i + n];
        const double re = a > q / 2 ? -(double)(q - a) : (double)a;
        const double im = b > q / 2 ? -(double)(q - b) : (double)b;
        v[i] = std::complex<double>(re / pt.scale, im / pt.scale);
    }
    fft_special_fwd(v.data(), n, 2 * N);
    for (int i = 0; i < n; i++) z[i] = v[i];
}

// ============================================================================= keys ====
// signed coefficient polynomials (npoly x N int64, host) -> eval form over the limbs of `mp`
static void small_to_eval(Context& cx, const int64_t* h, int npoly, LimbMap mp) {
    const int N = cx.N;
    DevBuf d((size_t)npoly * N, cx.stream);
    CUDA_CHECK(cudaMemcpyAsync(d.p, h, (size_t)npoly * N * 8, cudaMemcpyHostToDevice, cx.stream));
    k_signed_to_limbs<<<dim3(N / 256, npoly * mp.nl), 256, 0, cx.stream>>>((const int64_t*)d.p, mp.base, mp, cx.logN);
    CUDA_CHECK(cudaGetLastError());
    ntt(cx, mp, npoly, false, cx.stream);
    CUDA_CHECK(cudaStreamSynchronize(cx.stream));
    cx.launches += 1;
}

static LimbMap fullmap(const Context& cx, uint64_t* base) {
    LimbMap mp{};
    mp.base = base; mp.poly_stride = (long long)(cx.L + cx.K) * cx.N; mp.nl = cx.L + cx.K;
    mp.split = cx.L + cx.K; mp.off0 = 0; mp.off1 = 0;
    return mp;
}

// hybrid switching key from s_src to s_key (both eval form over all L+K moduli)
static std::unique_ptr<SwitchKey> gen_switch_key(Context& cx, const uint64_t* s_src, const uint64_t* s_key,
                                                 const uint8_t key_seed[32]) {
    const int N = cx.N, nm = cx.L + cx.K;
    auto key = std::make_unique<SwitchKey>();
    key->buf = DevBuf((size_t)cx.dnum_top * 2 * nm * N, cx.stream);
    std::vector<uint64_t> pm(nm, 0);
    for (int i = 0; i < cx.L; i++) {
        uint64_t v = 1;
        for (int k = 0; k < cx.K; k++) v = host_mulmod(v, cx.mods[cx.L + k] % cx.mods[i], cx.mods[i]);
        pm[i] = v;
    }
    DevBuf dpm = limb_consts(cx, pm, false);
    std::memcpy(key->seed, key_seed, 32);
    key->seeded = true;
    // every digit's a-half on the device, straight from the seed (the seeded expander, tag SKEY)
    expand_uniform_dev(cx, key_seed, 0, cx.dnum_top, 0, nm, kTagSKEY, key->buf.p + (size_t)nm * N,
                       (long long)2 * nm * N);
    // the digits' Gaussian errors (host), uploaded together
    std::vector<int64_t> e((size_t)cx.dnum_top * N);
    for (int j = 0; j < cx.dnum_top; j++)
        sample_gauss(key_seed, (uint32_t)j, 0, cx.prm.sigma, e.data() + (size_t)j * N, N);
    DevBuf de((size_t)nm * N, cx.stream), d((size_t)cx.dnum_top * N, cx.stream);
    CUDA_CHECK(cudaMemcpyAsync(d.p, e.data(), e.size() * 8, cudaMemcpyHostToDevice, cx.stream));
    for (int j = 0; j < cx.dnum_top; j++) {
        uint64_t* kb = key->buf.p + ((size_t)j * 2 + 0) * nm * N;
        uint64_t* ka = key->buf.p + ((size_t)j * 2 + 1) * nm * N;
        // e in eval form over every modulus: broadcast the single polynomial to all limbs
        LimbMap mp = fullmap(cx, de.p);
        mp.poly_stride = 0;
        k_signed_to_limbs<<<dim3(N / 256, nm), 256, 0, cx.stream>>>((const int64_t*)d.p + (size_t)j * N, de.p, mp,
                                                                    cx.logN);
        CUDA_CHECK(cudaGetLastError());
        ntt(cx, fullmap(cx, de.p), 1, false, cx.stream);
        const int lo = j * cx.alpha, hi = std::min(lo + cx.alpha, cx.L);
        k_keyb<<<dim3(N / 256, nm), 256, 0, cx.stream>>>(ka, de.p, s_key, s_src, dpm.p, kb, lo, hi, cx.logN);
        CUDA_CHECK(cudaGetLastError());
        cx.launches += 2;
    }
    k_mont<<<dim3(N / 256, cx.dnum_top * 2 * nm), 256, 0, cx.stream>>>(key->buf.p, nm, 1, cx.logN);
    CUDA_CHECK(cudaGetLastError());
    CUDA_CHECK(cudaStreamSynchronize(cx.stream));   // e is a host temporary
    cx.launches++;
    return key;
}

void keygen(Context& cx, const uint8_t seed[32]) {
    const int N = cx.N, nm = cx.L + cx.K;
    std::memcpy(cx.master, seed, 32);
    cx.enc_counter = 0;
    uint8_t s_seed[32], p_seed[32], r_seed[32];
    derive_seed(seed, kSeedSecret, 0, s_seed);
    derive_seed(seed, kSeedPublic, 0, p_seed);
    derive_seed(seed, 2, 0, r_seed);
    cx.sk_coeff.assign(N, 0);
    if (cx.prm.hw > 0) sample_ternary_hw(s_seed, 0, 0, cx.prm.hw, cx.sk_coeff.data(), N);
    else sample_ternary(s_seed, 0, 0, cx.sk_coeff.data(), N);
    std::vector<int64_t> s64(cx.sk_coeff.begin(), cx.sk_coeff.end());
    cx.sk = DevBuf((size_t)nm * N, cx.stream);
    small_to_eval(cx, s64.data(), 1, fullmap(cx, cx.sk.p));
    // public key over the L Q-limbs
    cx.pk = DevBuf((size_t)2 * cx.L * N, cx.stream);
    {
        expand_uniform_dev(cx, p_seed, 0, 1, 0, cx.L, kTagPKEY, cx.pk.p + (size_t)cx.L * N, 0);
        std::vector<int64_t> e(N);
        sample_gauss(p_seed, 0xFFFFFFFFu, 0, cx.prm.sigma, e.data(), N);
        DevBuf de((size_t)cx.L * N, cx.stream);
        LimbMap mp = cx.qmap(de.p, cx.L, 0);
        small_to_eval(cx, e.data(), 1, mp);
        k_pkb<<<dim3(N / 256, cx.L), 256, 0, cx.stream>>>(cx.pk.p + (size_t)cx.L * N, de.p, cx.sk.p, cx.pk.p, cx.logN);
        CUDA_CHECK(cudaGetLastError());
        CUDA_CHECK(cudaStreamSynchronize(cx.stream));
    }
    // relinearisation key: s^2 -> s
    DevBuf s2((size_t)nm * N, cx.stream);
    k_square<<<dim3(N / 256, nm), 256, 0, cx.stream>>>(cx.sk.p, s2.p, cx.logN);
    CUDA_CHECK(cudaGetLastError());
    cx.rlk = gen_switch_key(cx, s2.p, cx.sk.p, r_seed);
    cx.rot_keys.clear();
    CUDA_CHECK(cudaStreamSynchronize(cx.stream));
}

// rotation / conjugation keys: index k switches s -> tau_{k^-1}(s) (seeded_keys.hpp:162-170)
static void gen_auto_key(Context& cx, uint64_t k) {
    if (cx.rot_keys.count(k)) return;
    const int N = cx.N, nm = cx.L + cx.K;
    const uint64_t M = 2ull * N;
    // k^-1 mod 2N (k odd): Newton on 64-bit then reduce
    uint64_t inv = k;
    for (int i = 0; i < 6; i++) inv *= 2 - k * inv;
    inv &= (M - 1);
    DevBuf sp((size_t)nm * N, cx.stream);
    k_automorph<<<dim3(N / 256, nm), 256, 0, cx.stream>>>(cx.sk.p, sp.p, inv, cx.logN);
    CUDA_CHECK(cudaGetLastError());
    uint8_t seed[32];
    derive_seed(cx.master, (uint32_t)k, 0, seed);
    auto key = gen_switch_key(cx, cx.sk.p, sp.p, seed);
    key->index = k;
    cx.rot_keys[k] = std::move(key);
    CUDA_CHECK(cudaStreamSynchronize(cx.stream));
}

void keygen_auto(Context& cx, const uint64_t* ks, int n) {
    for (int i = 0; i < n; i++) {
        const uint64_t k = ks[i];
        if (!(k & 1) || k >= 2ull * cx.N) throw Error("keygen_auto: automorphism index must be odd and below 2N", -1);
        if (k == 1 || cx.rot_keys.count(k)) continue;
        if (!cx.sk.p) throw Error("keygen_auto: no secret key", -5);
        gen_auto_key(cx, k);
    }
}

void keygen_rotations(Context& cx, const int* rs, int n, bool conj) {
    // keys already held (generated earlier, or loaded from part files) are kept; only a missing
    // key needs the secret
    auto need = [&](uint64_t k) {
        if (k == 1 || cx.rot_keys.count(k)) return;
        if (!cx.sk.p) throw Error("keygen_rotations: no key for automorphism " + std::to_string(k) + " and no secret", -5);
        gen_auto_key(cx, k);
    };
    for (int i = 0; i < n; i++) need(rot_index(cx, rs[i]));
    if (conj) need(2ull * cx.N - 1);
}

Ciphertext encrypt(Context& cx, const Plaintext& pt) {
    if (!cx.pk.p) throw Error("encrypt: no public key", -5);
    const int N = cx.N, nl = pt.nl;
    uint8_t seed[32];
    derive_seed(cx.master, kSeedEncrypt, cx.enc_counter++, seed);
    std::vector<int8_t> v(N);
    std::vector<int64_t> h((size_t)3 * N);
    sample_ternary(seed, 0, 3, v.data(), N);
    for (int i = 0; i < N; i++) h[i] = v[i];
    sample_gauss(seed, 0, 1, cx.prm.sigma, h.data() + N, N);
    sample_gauss(seed, 0, 2, cx.prm.sigma, h.data() + 2 * N, N);
    DevBuf sm((size_t)3 * nl * N, cx.stream);
    small_to_eval(cx, h.data(), 3, cx.qmap(sm.p, nl, (long long)nl * N));
    Ciphertext c = ct_alloc(cx, nl);
    k_encrypt<<<g2(cx, nl), 256, 0, cx.stream>>>(sm.p, sm.p + (size_t)nl * N, sm.p + (size_t)2 * nl * N, cx.pk.p, cx.L,
                                                 pt.buf.p, c.c(0), c.c(1), cx.logN);
    CUDA_CHECK(cudaGetLastError());
    cx.launches++;
    c.scale = pt.scale;
    return c;
}

Plaintext decrypt(Context& cx, const Ciphertext& ct) {
    if (!cx.sk.p) throw Error("decrypt: no secret key", -5);
    Plaintext pt;
    pt.buf = DevBuf((size_t)ct.nl * cx.N, cx.stream);
    pt.nl = ct.nl;
    pt.scale = ct.scale;
    k_decrypt<<<g2(cx, ct.nl), 256, 0, cx.stream>>>(ct.c(0), ct.c(1), cx.sk.p, pt.buf.p, cx.logN);
    CUDA_CHECK(cudaGetLastError());
    cx.launches++;
    return pt;
}

// ========================================================================= raw access ====
void upload(Context& cx, uint64_t* dst, const uint64_t* src, size_t words) {
    CUDA_CHECK(cudaMemcpyAsync(dst, src, words * 8, cudaMemcpyHostToDevice, cx.stream));
    CUDA_CHECK(cudaStreamSynchronize(cx.stream));
}
void download(Context& cx, uint64_t* dst, const uint64_t* src, size_t words) {
    CUDA_CHECK(cudaMemcpyAsync(dst, src, words * 8, cudaMemcpyDeviceToHost, cx.stream));
    CUDA_CHECK(cudaStreamSynchronize(cx.stream));
    cx.check_device_error();
}
// A kernel whose bounded wait ran out left its flag: report it (the results of the work in
// flight since the last check are not trustworthy) and clear it.
// the moduli table each device's c_mod holds now (what the last activate() on it wrote)
static std::mutex g_cmod_mu;
static std::vector<ModConst> g_cmod_loaded[kMaxDevices];

void Context::activate() {
    if (device < 0 || device >= kMaxDevices) throw Error("device index out of range", -1);
    std::lock_guard<std::mutex> lk(g_cmod_mu);
    auto& cur = g_cmod_loaded[device];
    if (cur.size() == mc.size() && std::memcmp(cur.data(), mc.data(), mc.size() * sizeof(ModConst)) == 0) return;
    // another chain's constants are in the table: let the kernels that read them finish first
    if (!cur.empty()) CUDA_CHECK(cudaDeviceSynchronize());
    CUDA_CHECK(cudaMemcpyToSymbol(c_mod, mc.data(), sizeof(ModConst) * mc.size()));
    cur = mc;
}

void Context::check_device_error() {
    unsigned int f = 0;
    CUDA_CHECK(cudaMemcpy(&f, d_err, sizeof f, cudaMemcpyDeviceToHost));
    if (f) {
        CUDA_CHECK(cudaMemset(d_err, 0, sizeof f));
        throw Error("a tensor-core wait ran out of iterations (results since the last sync are invalid)", -3);
    }
}
void key_to_mont(Context& cx, uint64_t* key, bool to_mont) {
    const int nm = cx.L + cx.K;
    k_mont<<<dim3(cx.N / 256, cx.dnum_top * 2 * nm), 256, 0, cx.stream>>>(key, nm, to_mont ? 1 : 0, cx.logN);
    CUDA_CHECK(cudaGetLastError());
}

}  // namespace fhe
