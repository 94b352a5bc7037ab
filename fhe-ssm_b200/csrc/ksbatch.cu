// ksbatch.cu -- key switching batched over many rotations.
//
// A 1024-wide BSGS matvec issues ~125 rotations of a ciphertext of ~12 limbs, and a
// bootstrap level ~14.  One rotation at a time is a chain of ~10 launches of a few hundred
// CTAs each, far from filling 148 SMs, so the engine batches them:
//
//  * ct_rotate_hoisted (the babies): one ModUp of the input, then the key inner products,
//    the ModDown transforms and base conversions of up to kKsBatch rotations each run as
//    one launch over the whole batch (keys and output pointers travel in the kernel
//    parameters).  Bit-identical to rotating one at a time.
//  * rotate_sum (the giants): out = sum_b rot(in_b, r_b).  Each input is permuted first
//    (tau_b(c0), tau_b(c1) in evaluation form), so the key switch runs in the
//    rotate-then-switch order with the forward key tau_b(key_b); the batch shares one ModUp
//    launch sequence, the inner products of all inputs are summed in the extended basis QP in
//    one kernel, and a single ModDown finishes the sum (lazy ModDown: the sum of the
//    ModDowns and the ModDown of the sum differ only by the rounding of the P-division).
//    This is the double-hoisting arrangement of the BSGS giant step (Bossuat, Mouchet,
//    Troncoso-Pastoriza, Hubaux, Eurocrypt 2021, section 4).
#include "engine.h"

namespace fhe {

constexpr int kKsBatch = 64;

struct KeyBatch {
    const uint64_t* k[kKsBatch];
};
struct FinalBatch {
    uint64_t* out0[kKsBatch];
    uint64_t* out1[kKsBatch];
    uint64_t perm[kKsBatch];
};
struct RotBatch {
    const uint64_t* c0[kKsBatch];
    const uint64_t* c1[kKsBatch];
    uint64_t perm[kKsBatch];
};

// ------------------------------------------------------------------------------ kernels ----
// Batched key inner product.  ext_b = ext + b * ext_stride (stride 0: one shared ModUp).
//  sum == 0: out[b][c][e] = sum_j ext_b[j][e] * key_b[j][c][m(e)]       (grid z = batch)
//  sum == 1: out[c][e] (+)= sum_b sum_j ext_b[j][e] * key_b[j][c][m(e)] (accumulate != 0: add)
__global__ void __launch_bounds__(256) k_key_inner_b(const uint64_t* __restrict__ ext, long long ext_stride,
                                                     const KeyBatch kb, int B, uint64_t* __restrict__ out, int nl,
                                                     int ne, int dnum, int L, int K, int logN, int sum,
                                                     int accumulate) {
    pdl_wait();   // launched by launch_pdl: the previous kernel's writes first
    pdl_trigger();
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int e = blockIdx.y;
    const int m = e < nl ? e : L + (e - nl);
    const ModConst mc = c_mod[m];
    const size_t nk = (size_t)(L + K);
    if (!sum) {
        const int b = blockIdx.z;
        const uint64_t* eb = ext + b * ext_stride;
        const uint64_t* key = kb.k[b];
        u128acc a0{0, 0}, a1{0, 0};
        digit_dot2(eb + (size_t)e * N + x, (size_t)ne * N, key + (size_t)m * N + x, key + (nk + m) * N + x,
                   2 * nk * N, dnum, a0, a1);
        uint64_t* o = out + (size_t)b * 2 * ne * N;
        o[(size_t)e * N + x] = redc(a0.hi, a0.lo, mc);
        o[((size_t)ne + e) * N + x] = redc(a1.hi, a1.lo, mc);
        return;
    }
    uint64_t s0 = 0, s1 = 0;
    if (accumulate) {
        s0 = out[(size_t)e * N + x];
        s1 = out[((size_t)ne + e) * N + x];
    }
    for (int b = 0; b < B; b++) {
        const uint64_t* eb = ext + b * ext_stride;
        const uint64_t* key = kb.k[b];
        u128acc a0{0, 0}, a1{0, 0};
        digit_dot2(eb + (size_t)e * N + x, (size_t)ne * N, key + (size_t)m * N + x, key + (nk + m) * N + x,
                   2 * nk * N, dnum, a0, a1);
        s0 = mod_add(s0, redc(a0.hi, a0.lo, mc), mc.q);
        s1 = mod_add(s1, redc(a1.hi, a1.lo, mc), mc.q);
    }
    out[(size_t)e * N + x] = s0;
    out[((size_t)ne + e) * N + x] = s1;
}

// Key inner products of B ModUp outputs against one shared key (the relinearisation key of a
// batch of products): out[b][c][e] = sum_j ext_b[j][e] * key[j][c][m(e)].  A thread serves
// kKeyShare outputs of one slot, so each key word is read once per kKeyShare products.
constexpr int kKeyShare = 4;
__global__ void __launch_bounds__(256) k_key_inner_shared(const uint64_t* __restrict__ ext, long long ext_stride,
                                                          const uint64_t* __restrict__ key, int B,
                                                          uint64_t* __restrict__ out, int nl, int ne, int dnum, int L,
                                                          int K, int logN) {
    pdl_wait();   // launched by launch_pdl: the previous kernel's writes first
    pdl_trigger();
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int e = blockIdx.y;
    const int b0 = blockIdx.z * kKeyShare, nb = min(kKeyShare, B - b0);
    const int m = e < nl ? e : L + (e - nl);
    const ModConst mc = c_mod[m];
    const size_t nk = (size_t)(L + K);
    const uint64_t pol = evict_first_policy();
    const uint64_t* k0 = key + (size_t)m * N + x;
    const uint64_t* k1 = key + (nk + m) * N + x;
    const uint64_t* eb = ext + (size_t)b0 * ext_stride + (size_t)e * N + x;
    u128acc a0[kKeyShare], a1[kKeyShare];
#pragma unroll
    for (int i = 0; i < kKeyShare; i++) a0[i] = a1[i] = u128acc{0, 0};
#pragma unroll 2
    for (int j = 0; j < dnum; j++) {
        const uint64_t v0 = ld_stream(k0 + (size_t)j * 2 * nk * N, pol);
        const uint64_t v1 = ld_stream(k1 + (size_t)j * 2 * nk * N, pol);
        uint64_t dv[kKeyShare];
#pragma unroll
        for (int i = 0; i < kKeyShare; i++)
            if (i < nb) dv[i] = eb[(size_t)i * ext_stride + (size_t)j * ne * N];
#pragma unroll
        for (int i = 0; i < kKeyShare; i++)
            if (i < nb) {
                acc_mad(a0[i], dv[i], v0);
                acc_mad(a1[i], dv[i], v1);
            }
    }
#pragma unroll
    for (int i = 0; i < kKeyShare; i++)
        if (i < nb) {
            uint64_t* o = out + (size_t)(b0 + i) * 2 * ne * N;
            o[(size_t)e * N + x] = redc(a0[i].hi, a0[i].lo, mc);
            o[((size_t)ne + e) * N + x] = redc(a1[i].hi, a1[i].lo, mc);
        }
}

// Batched ModDown epilogue: out_c(b)[i][x] = add_c[i][s] + (buf_b[c][i][s] - y_b[c][i][s]) P^-1
// with s = auto_src(x, perm_b); add_0 = add0 (shared), add_1 = none.  grid z = 2 * batch.
__global__ void __launch_bounds__(256) k_moddown_final_b(const uint64_t* __restrict__ buf,
                                                         const uint64_t* __restrict__ y, const uint64_t* add0,
                                                         const FinalBatch fb, const uint64_t* __restrict__ md,
                                                         int nl, int ne, int L, int K, int logN) {
    pdl_wait();   // launched by launch_pdl: the previous kernel's writes first
    pdl_trigger();
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int i = blockIdx.y, c = blockIdx.z & 1, b = blockIdx.z >> 1;
    const uint64_t q = c_mod[i].q;
    const uint64_t* pinv = md + 2 * K + (size_t)L * K * 2 + (size_t)i * 2;
    const uint64_t k = fb.perm[b];
    const uint32_t s = k == 1 ? (uint32_t)x : auto_src((uint32_t)x, k, logN);
    const uint64_t* bb = buf + (size_t)b * 2 * ne * N;
    const uint64_t* yb = y + (size_t)b * 2 * nl * N;
    uint64_t v = mod_sub(bb[((size_t)c * ne + i) * N + s], yb[((size_t)c * nl + i) * N + s], q);
    v = mul_shoup(v, pinv[0], pinv[1], q);
    if (c == 0 && add0) v = mod_add(v, add0[(size_t)i * N + s], q);
    uint64_t* out = c == 0 ? fb.out0[b] : fb.out1[b];
    out[(size_t)i * N + x] = v;
}

// rotate_sum input stage: for each input b, tau_b(c1_b) (eval form) into dev[b] and dc[b]
// (dc is transformed to coefficient form next), and cs0 (+)= sum_b tau_b(c0_b) (+ init0).
__global__ void __launch_bounds__(256) k_gather_rot(const RotBatch rb, int B, uint64_t* __restrict__ dev,
                                                    uint64_t* __restrict__ dc, uint64_t* __restrict__ cs0,
                                                    const uint64_t* init0, int nl, int logN, int accumulate) {
    pdl_wait();   // launched by launch_pdl: the previous kernel's writes first
    pdl_trigger();
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int i = blockIdx.y;
    const uint64_t q = c_mod[i].q;
    uint64_t s0 = accumulate ? cs0[(size_t)i * N + x] : (init0 ? init0[(size_t)i * N + x] : 0);
    for (int b = 0; b < B; b++) {
        const uint32_t s = auto_src((uint32_t)x, rb.perm[b], logN);
        s0 = mod_add(s0, rb.c0[b][(size_t)i * N + s], q);
        const uint64_t v = rb.c1[b][(size_t)i * N + s];
        dev[((size_t)b * nl + i) * N + x] = v;
        dc[((size_t)b * nl + i) * N + x] = v;
    }
    cs0[(size_t)i * N + x] = s0;
}

// fwd[w][x] = key[w][auto_src(x, k)] for every limb-polynomial w of a switching key
__global__ void __launch_bounds__(256) k_key_permute(const uint64_t* __restrict__ key, uint64_t* __restrict__ fwd,
                                                     uint64_t k, int logN) {
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const size_t w = blockIdx.y;
    fwd[w * N + x] = key[w * N + auto_src((uint32_t)x, k, logN)];
}

// ------------------------------------------------------------------------------ host side ----
static inline dim3 gb(const Context& cx, int y, int z = 1) { return dim3(cx.N / 256, y, z); }

static const SwitchKey& rot_key(const Context& cx, uint64_t k, const char* who) {
    auto it = cx.rot_keys.find(k);
    if (it == cx.rot_keys.end())
        throw Error(std::string(who) + ": no rotation key for automorphism " + std::to_string(k), -5);
    return *it->second;
}

static const uint64_t* forward_key(Context& cx, uint64_t k) {
    SwitchKey& key = const_cast<SwitchKey&>(rot_key(cx, k, "rotate_sum"));
    if (!key.fwd.p) {
        key.fwd = DevBuf(key.buf.words, cx.stream);
        const int polys = (int)(key.buf.words / cx.N);
        k_key_permute<<<gb(cx, polys), 256, 0, cx.stream>>>(key.buf.p, key.fwd.p, k, cx.logN);
        CUDA_CHECK(cudaGetLastError());
        cx.launches++;
    }
    return key.fwd.p;
}

void ct_rotate_hoisted(Context& cx, const Ciphertext& a, const int* rs, int n, Ciphertext* outs) {
    const int N = cx.N, K = cx.K, L = cx.L, nl = a.nl, ne = nl + K, dn = cx.dnum(nl);
    cudaStream_t st = cx.stream;
    std::vector<int> todo;
    for (int i = 0; i < n; i++) {
        const uint64_t k = rot_index(cx, rs[i]);
        if (k == 1) outs[i] = ct_copy(cx, a);
        else {
            rot_key(cx, k, "rotate_hoisted");
            todo.push_back(i);
        }
    }
    if (todo.empty()) return;
    DevBuf ext = modup(cx, a.c(1), nl);
    for (size_t c0 = 0; c0 < todo.size(); c0 += kKsBatch) {
        const int B = (int)std::min<size_t>(kKsBatch, todo.size() - c0);
        KeyBatch kb{};
        FinalBatch fb{};
        for (int b = 0; b < B; b++) {
            const int i = todo[c0 + b];
            const uint64_t k = rot_index(cx, rs[i]);
            kb.k[b] = rot_key(cx, k, "rotate_hoisted").buf.p;
            outs[i] = ct_alloc(cx, nl);
            outs[i].scale = a.scale;
            fb.out0[b] = outs[i].c(0);
            fb.out1[b] = outs[i].c(1);
            fb.perm[b] = k;
        }
        DevBuf ip((size_t)B * 2 * ne * N, st);
        {
            ProfScope ps(cx, "key_inner", 8.0 * N * B * ((double)dn * ne * 2 + 2 * ne) + 8.0 * N * dn * ne);
            launch_pdl(cx, k_key_inner_b, gb(cx, ne, B), dim3(256), 0, st, ext.p, 0, kb, B, ip.p, nl, ne, dn, L, K, cx.logN, 0, 0);
        }
        LimbMap pm{};
        pm.base = ip.p + (size_t)nl * N; pm.poly_stride = (long long)ne * N; pm.nl = K;
        pm.split = 0; pm.off0 = 0; pm.off1 = L;
        ntt(cx, pm, 2 * B, true, st);
        DevBuf y((size_t)B * 2 * nl * N, st);
        {
            ProfScope ps(cx, "moddown_bconv", 8.0 * N * B * (2 * K + 2 * nl));
            launch_pdl(cx, k_moddown_bconv, gb(cx, 2, B), dim3(256), 0, st, ip.p, y.p, cx.d_md, nl, ne, L, K, cx.logN,
                                                          (long long)2 * ne * N, (long long)2 * nl * N);
        }
        ntt(cx, cx.qmap(y.p, nl, (long long)nl * N), 2 * B, false, st);
        {
            ProfScope ps(cx, "moddown_final", 8.0 * N * nl * B * 7);
            launch_pdl(cx, k_moddown_final_b, gb(cx, nl, 2 * B), dim3(256), 0, st, ip.p, y.p, a.c(0), fb, cx.d_md, nl, ne, L, K,
                                                                 cx.logN);
        }
        CUDA_CHECK(cudaGetLastError());
        cx.launches += 3;
        cx.ks_count += B;
        cx.ks_limbs += (long long)B * nl;
    }
}

void rotate_sum(Context& cx, const uint64_t* const* c0s, const uint64_t* const* c1s, const int* steps, int n,
                int nl, double scale, const uint64_t* extra0, const uint64_t* extra1, Ciphertext& out) {
    const int N = cx.N, K = cx.K, L = cx.L, ne = nl + K, dn = cx.dnum(nl);
    cudaStream_t st = cx.stream;
    for (int i = 0; i < n; i++)
        if (rot_index(cx, steps[i]) == 1) throw Error("rotate_sum: a zero rotation belongs in extra", -1);
    Ciphertext r = ct_alloc(cx, nl);
    r.scale = scale;
    if (n == 0) {
        if (!extra0) throw Error("rotate_sum: nothing to sum", -1);
        CUDA_CHECK(cudaMemcpyAsync(r.c(0), extra0, (size_t)nl * N * 8, cudaMemcpyDeviceToDevice, st));
        CUDA_CHECK(cudaMemcpyAsync(r.c(1), extra1, (size_t)nl * N * 8, cudaMemcpyDeviceToDevice, st));
        out = std::move(r);
        return;
    }
    DevBuf cs0((size_t)nl * N, st), acc((size_t)2 * ne * N, st);
    const uint64_t* tab = cx.modup_table(nl);
    for (int c0 = 0; c0 < n; c0 += kKsBatch) {
        const int B = std::min(kKsBatch, n - c0);
        RotBatch rb{};
        KeyBatch kb{};
        for (int b = 0; b < B; b++) {
            const uint64_t k = rot_index(cx, steps[c0 + b]);
            rb.c0[b] = c0s[c0 + b];
            rb.c1[b] = c1s[c0 + b];
            rb.perm[b] = k;
            kb.k[b] = forward_key(cx, k);
        }
        DevBuf dev((size_t)B * nl * N, st), dc((size_t)B * nl * N, st);
        {
            ProfScope ps(cx, "gather_rot", 8.0 * N * nl * (3.0 * B + 2));
            launch_pdl(cx, k_gather_rot, gb(cx, nl), dim3(256), 0, st, rb, B, dev.p, dc.p, cs0.p, extra0, nl, cx.logN, c0 > 0);
        }
        ntt(cx, cx.qmap(dc.p, nl, (long long)nl * N), B, true, st);
        DevBuf ext((size_t)B * dn * ne * N, st);
        {
            ProfScope ps(cx, "modup_bconv", 8.0 * N * B * (2 * nl + (double)dn * ne));
            launch_pdl(cx, k_modup_bconv, gb(cx, dn, B), dim3(256), 0, st, dc.p, dev.p, ext.p, tab, nl, ne, cx.alpha, L, cx.logN,
                                                         (long long)nl * N, (long long)nl * N,
                                                         (long long)dn * ne * N);
        }
        LimbMap em = cx.extmap(ext.p, nl, (long long)ne * N);
        em.skip_alpha = cx.alpha;
        em.skip_period = dn;
        ntt(cx, em, B * dn, false, st);
        {
            ProfScope ps(cx, "key_inner", 8.0 * N * ((double)B * dn * ne * 3 + 2 * ne));
            launch_pdl(cx, k_key_inner_b, gb(cx, ne), dim3(256), 0, st, ext.p, (long long)dn * ne * N, kb, B, acc.p, nl, ne, dn, L, K,
                                                      cx.logN, 1, c0 > 0);
        }
        CUDA_CHECK(cudaGetLastError());
        cx.launches += 3;
        cx.ks_count += B;
        cx.ks_limbs += (long long)B * nl;
    }
    moddown(cx, acc.p, nl, cs0.p, extra1, r.c(0), r.c(1), 1);
    out = std::move(r);
}

// B products a[k] * b[k] at one level, relinearised and rescaled together: one batched ModUp,
// one key-inner launch, one merged ModDown + rescale (the same arithmetic as
// ct_mul_relin_rescale, product by product)
void ct_mul_relin_rescale_n(Context& cx, const Ciphertext* const* a, const Ciphertext* const* b, int B,
                            Ciphertext* out) {
    if (B < 1 || B > 64) throw Error("mul_relin_rescale_n: 1..64 products", -1);
    const int nl = a[0]->nl;
    for (int k = 0; k < B; k++)
        if (a[k]->nl != nl || b[k]->nl != nl) throw Error("mul: level mismatch", -4);
    if (nl < 2) throw Error("mul_rescale: no level left", -4);
    if (!cx.rlk) throw Error("mul: no relinearisation key", -5);
    if (cx.K > 6) throw Error("mul_relin_rescale: at most 6 special primes", -1);
    const int N = cx.N, K = cx.K, L = cx.L, ne = nl + K, dn = cx.dnum(nl), J = K + 1;
    cudaStream_t st = cx.stream;
    DevBuf d((size_t)B * 2 * nl * N, st), d2((size_t)B * nl * N, st);
    for (int k = 0; k < B; k++) {
        ProfScope ps(cx, "tensor", 8.0 * N * nl * 7);
        launch_pdl(cx, k_tensor, g2(cx, nl), dim3(256), 0, st, a[k]->buf.p, (long long)a[k]->stride, b[k]->buf.p,
                                             (long long)b[k]->stride, d.p + (size_t)k * 2 * nl * N,
                                             (long long)nl * N, d2.p + (size_t)k * nl * N, cx.logN);
    }
    // ModUp of the B d2 polynomials
    DevBuf dc((size_t)B * nl * N, st);
    CUDA_CHECK(cudaMemcpyAsync(dc.p, d2.p, (size_t)B * nl * N * 8, cudaMemcpyDeviceToDevice, st));
    ntt(cx, cx.qmap(dc.p, nl, (long long)nl * N), B, true, st);
    DevBuf ext((size_t)B * dn * ne * N, st);
    {
        ProfScope ps(cx, "modup_bconv", 8.0 * N * B * (2 * nl + (double)dn * ne));
        launch_pdl(cx, k_modup_bconv, g2(cx, dn, B), dim3(256), 0, st, dc.p, d2.p, ext.p, cx.modup_table(nl), nl, ne, cx.alpha, L,
                                                     cx.logN, (long long)nl * N, (long long)nl * N,
                                                     (long long)dn * ne * N);
    }
    LimbMap em = cx.extmap(ext.p, nl, (long long)ne * N);
    em.skip_alpha = cx.alpha;
    em.skip_period = dn;
    ntt(cx, em, B * dn, false, st);
    DevBuf ip((size_t)B * 2 * ne * N, st);
    {
        // the relinearisation key is read once per kKeyShare products
        const int nz = (B + kKeyShare - 1) / kKeyShare;
        ProfScope ps(cx, "key_inner", 8.0 * N * ((double)dn * ne * (B + 2.0 * nz) + 2.0 * B * ne));
        launch_pdl(cx, k_key_inner_shared, g2(cx, ne, nz), dim3(256), 0, st, ext.p, (long long)dn * ne * N,
                   (const uint64_t*)cx.rlk->buf.p, B, ip.p, nl, ne, dn, L, K, cx.logN);
    }
    cx.ks_count += B;
    cx.ks_limbs += (long long)B * nl;
    // ModDown + rescale in one division by P q_l, all products together
    const uint64_t* tab = cx.mdr_table(nl);
    DevBuf z((size_t)B * 2 * J * N, st);
    {
        ProfScope ps(cx, "mdr_gather", 8.0 * N * B * 2 * (1 + 2 * J));
        for (int k = 0; k < B; k++)
            launch_pdl(cx, k_mdr_gather, dim3(N / 256, J, 2), dim3(256), 0, st, d.p + (size_t)k * 2 * nl * N, (long long)nl * N,
                                                              ip.p + (size_t)k * 2 * ne * N, tab,
                                                              z.p + (size_t)k * 2 * J * N, nl, ne, K, cx.logN);
    }
    LimbMap zm{};
    zm.base = z.p; zm.poly_stride = (long long)J * N; zm.nl = J;
    zm.split = 1; zm.off0 = nl - 1; zm.off1 = L;
    ntt(cx, zm, 2 * B, true, st);
    DevBuf y((size_t)B * 2 * (nl - 1) * N, st);
    {
        ProfScope ps(cx, "moddown_bconv", 8.0 * N * B * (2 * J + 2 * (nl - 1)));
        launch_pdl(cx, k_mdr_bconv, g2(cx, 2, B), dim3(256), 0, st, z.p, y.p, tab, nl, K, L, cx.logN, (long long)2 * J * N,
                                                  (long long)2 * (nl - 1) * N);
    }
    ntt(cx, cx.qmap(y.p, nl - 1, (long long)(nl - 1) * N), 2 * B, false, st);
    for (int k = 0; k < B; k++) {
        Ciphertext r = ct_alloc(cx, nl - 1);
        {
            ProfScope ps(cx, "moddown_final", 8.0 * N * (nl - 1) * 2 * 5);
            launch_pdl(cx, k_mdr_final, g2(cx, nl - 1, 2), dim3(256), 0, st, d.p + (size_t)k * 2 * nl * N, (long long)nl * N,
                                                           ip.p + (size_t)k * 2 * ne * N,
                                                           y.p + (size_t)k * 2 * (nl - 1) * N, tab, r.buf.p,
                                                           (long long)r.stride, nl, ne, K, cx.logN);
        }
        r.scale = a[k]->scale * b[k]->scale / (double)cx.mods[nl - 1];
        out[k] = std::move(r);
    }
    CUDA_CHECK(cudaGetLastError());
    cx.launches += 7 + 4 * (long long)B;
}

}  // namespace fhe
