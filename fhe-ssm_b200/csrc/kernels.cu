// kernels.cu -- element-wise RNS kernels, base conversions and key-switching pieces.
//
// Grids are (N / 256, limbs, polys) with 256 threads; thread x of block (bx, i, p) owns
// coefficient / evaluation slot bx*256 + x of limb i of polynomial p.  All residues are
// canonical.  The base conversions are the approximate (fast) CRT basis switch of RNS
// CKKS: y_t = sum_i [x_i * qhat_i^-1]_{q_i} * [qhat_i]_t mod t, with no correction of the
// small multiple of the source modulus it leaves -- the hybrid key switching of
// Han-Ki 2020 as OpenFHE implements it (keyswitch-hybrid ModUp/ModDown).
#include "engine.h"

namespace fhe {


// eval-form automorphism source index: out[i] = in[src], 2brev(src)+1 = k (2brev(i)+1) mod 2N
__device__ __forceinline__ uint32_t auto_src(uint32_t i, uint64_t k, int logN) {
    const uint32_t br = __brev(i) >> (32 - logN);
    const uint64_t e = ((2ull * br + 1) * k) & ((2ull << logN) - 1);
    const uint32_t f = (uint32_t)((e - 1) >> 1);
    return __brev(f) >> (32 - logN);
}

// ---------------------------------------------------------------------------- ModUp ----
// dcoef: the nl Q-limbs in coefficient form; deval: the same limbs in eval form.
// ext[j][e] for digit j: own limbs copied from deval, all others base-converted (coefficient
// form, NTT'd afterwards).  blockIdx.z indexes a batch of inputs (strides sdc, sdv, sext).  tab: [dnum][alpha][2] (qhat^-1 mod q_i, shoup) then
// [dnum][ne][alpha][2] (qhat mod t, qhat 2^64 mod t): each output is one 128-bit sum of
// products with the Montgomery-form constants and one Montgomery reduction.
__global__ void __launch_bounds__(256) k_modup_bconv(const uint64_t* __restrict__ dcoef,
                                                     const uint64_t* __restrict__ deval, uint64_t* __restrict__ ext,
                                                     const uint64_t* __restrict__ tab, int nl, int ne, int alpha, int L,
                                                     int logN, long long sdc, long long sdv, long long sext) {
    pdl_wait();   // launched by launch_pdl: the previous kernel's writes first
    pdl_trigger();
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int j = blockIdx.y;
    const int dn = gridDim.y;
    dcoef += blockIdx.z * sdc;   // batch of inputs (blockIdx.z), same limb count
    deval += blockIdx.z * sdv;
    ext += blockIdx.z * sext;
    const int lo = j * alpha, sz = min(alpha, nl - lo);
    const uint64_t* qhinv = tab + (size_t)j * alpha * 2;
    const uint64_t* qh = tab + (size_t)dn * alpha * 2 + (size_t)j * ne * alpha * 2;
    __shared__ uint64_t sw[kMaxMod * 8 * 2];   // this digit's [ne][alpha][2] constants
    for (int i = threadIdx.x; i < ne * alpha * 2; i += blockDim.x) sw[i] = qh[i];
    __syncthreads();
    uint64_t t[8];
#pragma unroll
    for (int a = 0; a < 8; a++) {
        if (a < sz) {
            const uint64_t q = c_mod[lo + a].q;
            t[a] = mul_shoup(dcoef[(size_t)(lo + a) * N + x], qhinv[2 * a], qhinv[2 * a + 1], q);
        }
    }
    uint64_t* out = ext + (size_t)j * ne * N;
    for (int e = 0; e < ne; e++) {
        if (e >= lo && e < lo + sz) {
            out[(size_t)e * N + x] = deval[(size_t)e * N + x];
            continue;
        }
        const ModConst mt = c_mod[e < nl ? e : L + (e - nl)];
        const uint64_t* w = sw + e * alpha * 2;
        u128acc s{0, 0};
#pragma unroll
        for (int a = 0; a < 8; a++)   // constants in Montgomery form: sum < 8 2^60 t < t 2^64
            if (a < sz) acc_mad32(s, t[a], w[2 * a + 1]);
        out[(size_t)e * N + x] = redc(s.hi, s.lo, mt);
    }
}

// ----------------------------------------------------- digit dot products (key switching) ----
// Switching keys are streamed once per launch and are larger than L2: their loads skip L1 and
// carry an L2 evict-first hint, so that the ModUp outputs and the NTT tables stay resident.
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t p;
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t ld_stream(const uint64_t* a, uint64_t pol) {
    uint64_t v;
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.u64 %0, [%1], %2;" : "=l"(v) : "l"(a), "l"(pol));
    return v;
}
constexpr int kDigitBatch = 4;
// a0 += sum_j d[j ds] k0[j ks], a1 += sum_j d[j ds] k1[j ks] over the digits j < dn (128-bit
// sums; key words in Montgomery form).  The 3 loads of up to kDigitBatch digits are all issued
// before the first multiply, so a thread keeps them in flight together.
__device__ __forceinline__ void digit_dot2(const uint64_t* __restrict__ d, size_t ds, const uint64_t* __restrict__ k0,
                                           const uint64_t* __restrict__ k1, size_t ks, int dn, u128acc& a0,
                                           u128acc& a1) {
    const uint64_t pol = evict_first_policy();
    for (int j0 = 0; j0 < dn; j0 += kDigitBatch) {
        uint64_t dv[kDigitBatch], v0[kDigitBatch], v1[kDigitBatch];
#pragma unroll
        for (int j = 0; j < kDigitBatch; j++)
            if (j0 + j < dn) {
                dv[j] = d[(size_t)(j0 + j) * ds];
                v0[j] = ld_stream(k0 + (size_t)(j0 + j) * ks, pol);
                v1[j] = ld_stream(k1 + (size_t)(j0 + j) * ks, pol);
            }
#pragma unroll
        for (int j = 0; j < kDigitBatch; j++)
            if (j0 + j < dn) {
                acc_mad(a0, dv[j], v0[j]);
                acc_mad(a1, dv[j], v1[j]);
            }
    }
}

// ------------------------------------------------------------------- key inner product ----
// out[c][e] = sum_j ext[j][e] * key[j][c][m(e)]  (key in Montgomery form -> canonical result)
__global__ void k_key_inner(const uint64_t* __restrict__ ext, const uint64_t* __restrict__ key,
                            uint64_t* __restrict__ out, int nl, int ne, int dnum, int L, int K, int logN) {
    pdl_wait();   // launched by launch_pdl: the previous kernel's writes first
    pdl_trigger();
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int e = blockIdx.y;
    const int m = e < nl ? e : L + (e - nl);
    const ModConst mc = c_mod[m];
    const size_t nk = (size_t)(L + K);
    u128acc a0{0, 0}, a1{0, 0};
    digit_dot2(ext + (size_t)e * N + x, (size_t)ne * N, key + (size_t)m * N + x, key + (nk + m) * N + x, 2 * nk * N,
               dnum, a0, a1);
    out[(size_t)e * N + x] = redc(a0.hi, a0.lo, mc);
    out[((size_t)ne + e) * N + x] = redc(a1.hi, a1.lo, mc);
}

// ---------------------------------------------------------------------------- ModDown ----
// buf: [2][ne][N], P limbs (e >= nl) already in coefficient form.  y[c][i] = BConv_{P->q_i}.
// md: [K][2] phat^-1 mod p_k (+shoup); [L][K][2] phat_k mod q_i (+shoup); [L][2] P^-1 mod q_i.
__global__ void k_moddown_bconv(const uint64_t* __restrict__ buf, uint64_t* __restrict__ y,
                                const uint64_t* __restrict__ md, int nl, int ne, int L, int K, int logN,
                                long long sbuf, long long sy) {
    pdl_wait();   // launched by launch_pdl: the previous kernel's writes first
    pdl_trigger();
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int c = blockIdx.y;
    buf += blockIdx.z * sbuf;   // batch of key-switch outputs (blockIdx.z)
    y += blockIdx.z * sy;
    uint64_t t[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
        if (k < K) {
            const uint64_t p = c_mod[L + k].q;
            t[k] = mul_shoup(buf[((size_t)c * ne + nl + k) * N + x], md[2 * k], md[2 * k + 1], p);
        }
    }
    const uint64_t* ph = md + 2 * K;
    for (int i = 0; i < nl; i++) {
        const uint64_t q = c_mod[i].q;
        const uint64_t* w = ph + (size_t)i * K * 2;
        uint64_t s = 0;
#pragma unroll
        for (int k = 0; k < 8; k++)
            if (k < K) s += mul_shoup_lazy(t[k], w[2 * k], w[2 * k + 1], q);
        y[((size_t)c * nl + i) * N + x] = reduce_lazy16(s, q);
    }
}

// out_c[i][x] = add_c[i][s] + (buf[c][i][s] - y[c][i][s]) * P^-1,  s = auto_src(x, k)
__global__ void k_moddown_final(const uint64_t* __restrict__ buf, const uint64_t* __restrict__ y,
                                const uint64_t* add0, const uint64_t* add1, uint64_t* out0, uint64_t* out1,
                                const uint64_t* __restrict__ md, int nl, int ne, int L, int K, int logN,
                                uint64_t perm_k) {
    pdl_wait();   // launched by launch_pdl: the previous kernel's writes first
    pdl_trigger();
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int i = blockIdx.y, c = blockIdx.z;
    const uint64_t q = c_mod[i].q;
    const uint64_t* pinv = md + 2 * K + (size_t)L * K * 2 + (size_t)i * 2;
    const uint32_t s = perm_k == 1 ? (uint32_t)x : auto_src((uint32_t)x, perm_k, logN);
    uint64_t v = mod_sub(buf[((size_t)c * ne + i) * N + s], y[((size_t)c * nl + i) * N + s], q);
    v = mul_shoup(v, pinv[0], pinv[1], q);
    const uint64_t* add = c == 0 ? add0 : add1;
    if (add) v = mod_add(v, add[(size_t)i * N + s], q);
    uint64_t* out = c == 0 ? out0 : out1;
    out[(size_t)i * N + x] = v;
}

// ---------------------------------------------------------------- ModDown + rescale merged ----
// z: [2][K+1][N] coefficient form of x on the moduli M = q_l p_0 .. p_{K-1} (x = P d + ip on q_l,
// ip on the p_k).  y[c][i] = [x]_M mod q_i for i < nl - 1, with [x]_M the centred residue
// (-M/2 <= [x]_M < M/2): sum_j t_j (M/m_j) - u M with t_j = x (M/m_j)^-1 mod m_j and
// u = rint(sum_j t_j / m_j) evaluated in double precision (Halevi-Polyakov-Shoup, CT-RSA 2019).
// The division (x - [x]_M) / M is then an exact rounding: no bias is left in the coefficients
// (the fast conversion without u would leave floor() plus up to K+1 units on every coefficient).
// tab: [K+1][2] (M/m_j)^-1 mod m_j (+shoup), [nl-1][K+1][2] (M/m_j) mod q_i (+shoup), then
// [nl-1][2] M^-1 mod q_i, [nl-1][2] P mod q_i, [2] P mod q_l, [nl-1][2] M mod q_i, [K+1] 1/m_j
// (double bit patterns).
__global__ void __launch_bounds__(256) k_mdr_bconv(const uint64_t* __restrict__ z, uint64_t* __restrict__ y,
                                                   const uint64_t* __restrict__ tab, int nl, int K, int L, int logN,
                                                   long long sz, long long sy) {
    pdl_wait();   // launched by launch_pdl: the previous kernel's writes first
    pdl_trigger();
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int c = blockIdx.y;
    z += blockIdx.z * sz;   // a batch of products (blockIdx.z)
    y += blockIdx.z * sy;
    const int J = K + 1, nq = nl - 1;
    const uint64_t* mmod = tab + 2 * J + (size_t)nq * J * 2 + 4 * (size_t)nq + 2;   // [nq][2] M mod q_i
    const double* rinv = reinterpret_cast<const double*>(mmod + 2 * (size_t)nq);      // [J] 1 / m_j
    uint64_t t[8];
    double v = 0.0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        if (j < J) {
            const uint64_t m = c_mod[j == 0 ? nl - 1 : L + j - 1].q;
            t[j] = mul_shoup(z[((size_t)c * J + j) * N + x], tab[2 * j], tab[2 * j + 1], m);
            v += (double)t[j] * rinv[j];
        }
    }
    const uint64_t u = (uint64_t)rint(v);   // 0 <= u <= J
    const uint64_t* hat = tab + 2 * J;
    for (int i = 0; i < nq; i++) {
        const uint64_t q = c_mod[i].q;
        const uint64_t* w = hat + (size_t)i * J * 2;
        uint64_t s = 0;
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (j < J) s += mul_shoup_lazy(t[j], w[2 * j], w[2 * j + 1], q);   // J <= 7 terms < 14q
        s += 2 * q - mul_shoup_lazy(u, mmod[2 * i], mmod[2 * i + 1], q);       // - u M, still < 16q
        y[((size_t)c * nq + i) * N + x] = reduce_lazy16(s, q);
    }
}
// out_c[i] = (P d_c[i] + ip_c[i] - y_c[i]) * M^-1 for i < nl - 1 (eval form)
__global__ void __launch_bounds__(256) k_mdr_final(const uint64_t* __restrict__ d, long long sd,
                                                   const uint64_t* __restrict__ ip, const uint64_t* __restrict__ y,
                                                   const uint64_t* __restrict__ tab, uint64_t* out, long long so,
                                                   int nl, int ne, int K, int logN) {
    pdl_wait();   // launched by launch_pdl: the previous kernel's writes first
    pdl_trigger();
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int i = blockIdx.y, c = blockIdx.z;
    const int J = K + 1, nq = nl - 1;
    const uint64_t q = c_mod[i].q;
    const uint64_t* minv = tab + 2 * J + (size_t)nq * J * 2 + 2 * i;
    const uint64_t* pm = tab + 2 * J + (size_t)nq * J * 2 + 2 * nq + 2 * i;
    uint64_t v = mul_shoup(d[(size_t)c * sd + (size_t)i * N + x], pm[0], pm[1], q);
    v = mod_add(v, ip[((size_t)c * ne + i) * N + x], q);
    v = mod_sub(v, y[((size_t)c * nq + i) * N + x], q);
    out[(size_t)c * so + (size_t)i * N + x] = mul_shoup(v, minv[0], minv[1], q);
}
// z[c][0] = P d_c[l] + ip_c[l] (the dropped limb l = nl - 1), z[c][1 + k] = ip_c[nl + k]
__global__ void __launch_bounds__(256) k_mdr_gather(const uint64_t* __restrict__ d, long long sd,
                                                    const uint64_t* __restrict__ ip, const uint64_t* __restrict__ tab,
                                                    uint64_t* __restrict__ z, int nl, int ne, int K, int logN) {
    pdl_wait();   // launched by launch_pdl: the previous kernel's writes first
    pdl_trigger();
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int j = blockIdx.y, c = blockIdx.z;
    const int J = K + 1, l = nl - 1;
    uint64_t v;
    if (j == 0) {
        const uint64_t q = c_mod[l].q;
        // P mod q_l sits after the per-i entries: tab[2J + nq J 2 + 2 nq + 2 nq] (+shoup)
        const uint64_t* pl = tab + 2 * J + (size_t)(nl - 1) * J * 2 + 4 * (size_t)(nl - 1);
        v = mod_add(mul_shoup(d[(size_t)c * sd + (size_t)l * N + x], pl[0], pl[1], q), ip[((size_t)c * ne + l) * N + x], q);
    } else {
        v = ip[((size_t)c * ne + nl + j - 1) * N + x];
    }
    z[((size_t)c * J + j) * N + x] = v;
}

// ---------------------------------------------------------------------------- rescale ----
// last: [2][N] the dropped limb (index l) in coefficient form; y[c][i] = centred lift mod q_i
__global__ void k_rescale_lift(const uint64_t* __restrict__ last, uint64_t* __restrict__ y, int nlm1, int l,
                               int logN) {
    pdl_wait();   // launched by launch_pdl: the previous kernel's writes first
    pdl_trigger();
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int i = blockIdx.y, c = blockIdx.z;
    const uint64_t ql = c_mod[l].q;
    const ModConst mi = c_mod[i];
    const uint64_t v = last[(size_t)c * N + x];
    uint64_t r;
    if (v > (ql >> 1)) r = mod_sub(reduce64(v, mi), reduce64(ql, mi), mi.q);
    else r = reduce64(v, mi);
    y[((size_t)c * nlm1 + i) * N + x] = r;
}
// a_c[i] = (a_c[i] - y[c][i]) * q_l^-1   (rs: [l][i][2] = (q_l^-1 mod q_i, shoup))
__global__ void k_rescale_final(uint64_t* a, long long stride, const uint64_t* __restrict__ y,
                                const uint64_t* __restrict__ rs, int nlm1, int l, int L, int logN) {
    pdl_wait();   // launched by launch_pdl: the previous kernel's writes first
    pdl_trigger();
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int i = blockIdx.y, c = blockIdx.z;
    const uint64_t q = c_mod[i].q;
    const uint64_t* w = rs + ((size_t)l * L + i) * 2;
    uint64_t* p = a + (size_t)c * stride + (size_t)i * N + x;
    *p = mul_shoup(mod_sub(*p, y[((size_t)c * nlm1 + i) * N + x], q), w[0], w[1], q);
}

// ------------------------------------------------------------------------ element-wise ----

// ct op ct / ct op pt.  pt has log_rep: word x of limb i = pt[i][x >> log_rep] (x in eval order).
__global__ void k_ewise(int op, const uint64_t* a, long long sa, const uint64_t* b, long long sb, uint64_t* o,
                        long long so, int log_rep, int logN) {
    pdl_wait();   // launched by launch_pdl: the previous kernel's writes first
    pdl_trigger();
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int i = blockIdx.y, c = blockIdx.z;
    const ModConst mc = c_mod[i];
    const uint64_t av = a[(size_t)c * sa + (size_t)i * N + x];
    uint64_t r;
    switch (op) {
        case EW_ADD: r = mod_add(av, b[(size_t)c * sb + (size_t)i * N + x], mc.q); break;
        case EW_SUB: r = mod_sub(av, b[(size_t)c * sb + (size_t)i * N + x], mc.q); break;
        case EW_MULPT: {
            const uint64_t pv = b[(size_t)i * (N >> log_rep) + (x >> log_rep)];
            r = mul_barrett(av, pv, mc);
            break;
        }
        case EW_ADDPT: {
            if (c == 0) r = mod_add(av, b[(size_t)i * (N >> log_rep) + (x >> log_rep)], mc.q);
            else r = av;
            break;
        }
        default: r = mod_neg(av, mc.q); break;
    }
    o[(size_t)c * so + (size_t)i * N + x] = r;
}

// multiply every limb i by a per-limb constant (shoup pair), optionally add a per-limb constant
// to c0.  The constants travel in the kernel parameters (no host-to-device copy, no sync).
__global__ void k_mul_const(const uint64_t* a, long long sa, uint64_t* o, long long so, const LimbConst k, int logN) {
    pdl_wait();   // launched by launch_pdl: the previous kernel's writes first
    pdl_trigger();
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int i = blockIdx.y, c = blockIdx.z;
    const uint64_t q = c_mod[i].q;
    uint64_t v = a[(size_t)c * sa + (size_t)i * N + x];
    if (k.has_w) v = mul_shoup(v, k.w[i], k.wp[i], q);
    if (k.has_add && c == 0) v = mod_add(v, k.add[i], q);
    o[(size_t)c * so + (size_t)i * N + x] = v;
}

// tensor: d0 = a0 b0, d1 = a0 b1 + a1 b0 (into o), d2 = a1 b1 (into d2)
__global__ void k_tensor(const uint64_t* a, long long sa, const uint64_t* b, long long sb, uint64_t* o, long long so,
                         uint64_t* d2, int logN) {
    pdl_wait();   // launched by launch_pdl: the previous kernel's writes first
    pdl_trigger();
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int i = blockIdx.y;
    const ModConst mc = c_mod[i];
    const size_t off = (size_t)i * N + x;
    const uint64_t a0 = a[off], a1 = a[sa + off], b0 = b[off], b1 = b[sb + off];
    const uint64_t d0 = mul_barrett(a0, b0, mc);
    const uint64_t d1 = mod_add(mul_barrett(a0, b1, mc), mul_barrett(a1, b0, mc), mc.q);
    d2[off] = mul_barrett(a1, b1, mc);
    o[off] = d0;
    o[so + off] = d1;
}

// signed small/int64 coefficients -> residues of limbs (mods[] of map), coefficient form
__global__ void k_signed_to_limbs(const int64_t* __restrict__ s, uint64_t* out, LimbMap mp, int logN) {
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int y = blockIdx.y;
    const int poly = y / mp.nl, limb = y % mp.nl;
    const ModConst mc = c_mod[mp.mod(limb)];
    const int64_t v = s[(size_t)poly * N + x];
    const uint64_t r = v >= 0 ? reduce64((uint64_t)v, mc) : mod_neg(reduce64((uint64_t)(-v), mc), mc.q);
    out[(size_t)poly * mp.poly_stride + (size_t)limb * N + x] = r;
}

// out = in permuted by automorphism k (eval form), per limb
__global__ void k_automorph(const uint64_t* in, uint64_t* out, uint64_t k, int logN) {
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const size_t l = blockIdx.y;
    out[l * N + x] = in[l * N + auto_src((uint32_t)x, k, logN)];
}

// b = -a * skey + e + [limb in digit] P * ssrc  (all eval form), one digit j; limbs of the
// full basis (L+K); result written in Montgomery form together with a.
__global__ void k_keyb(const uint64_t* a, const uint64_t* e, const uint64_t* skey, const uint64_t* ssrc,
                       const uint64_t* __restrict__ pmodq, uint64_t* b, int lo, int hi, int logN) {
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int m = blockIdx.y;
    const ModConst mc = c_mod[m];
    const size_t off = (size_t)m * N + x;
    uint64_t v = mod_sub(e[off], mul_barrett(a[off], skey[off], mc), mc.q);
    if (m >= lo && m < hi) v = mod_add(v, mul_barrett(pmodq[m], ssrc[off], mc), mc.q);
    b[off] = v;
}

// Montgomery domain conversion in place over limbs of the full basis
__global__ void k_mont(uint64_t* a, int nmod, int to_mont, int logN) {
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int m = blockIdx.y % nmod;
    const ModConst mc = c_mod[m];
    uint64_t* p = a + (size_t)blockIdx.y * N + x;
    if (to_mont) *p = redc(__umul64hi(*p, mc.r2), *p * mc.r2, mc);
    else *p = redc(0, *p, mc);
}

// every limb l of a polynomial into Montgomery form (x 2^64 mod m(l)), modulus m(l) = mp.mod(l)
__global__ void k_mont_map(uint64_t* a, LimbMap mp, int logN) {
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int l = blockIdx.y;
    const ModConst mc = c_mod[mp.mod(l)];
    uint64_t* p = mp.base + (size_t)l * N + x;
    *p = redc(__umul64hi(*p, mc.r2), *p * mc.r2, mc);
}

// encrypt: c0 = v*pk0 + e0 + m, c1 = v*pk1 + e1 over nl limbs; small polys in eval form
__global__ void k_encrypt(const uint64_t* v, const uint64_t* e0, const uint64_t* e1, const uint64_t* pk, int L,
                          const uint64_t* m, uint64_t* c0, uint64_t* c1, int logN) {
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int i = blockIdx.y;
    const ModConst mc = c_mod[i];
    const size_t off = (size_t)i * N + x;
    const uint64_t vv = v[off];
    c0[off] = mod_add(mod_add(mul_barrett(vv, pk[off], mc), e0[off], mc.q), m[off], mc.q);
    c1[off] = mod_add(mul_barrett(vv, pk[(size_t)L * N + off], mc), e1[off], mc.q);
}

// decrypt: m = c0 + c1 * s
__global__ void k_decrypt(const uint64_t* c0, const uint64_t* c1, const uint64_t* s, uint64_t* m, int logN) {
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int i = blockIdx.y;
    const ModConst mc = c_mod[i];
    const size_t off = (size_t)i * N + x;
    m[off] = mod_add(c0[off], mul_barrett(c1[off], s[off], mc), mc.q);
}

// public key: b = -a*s + e
__global__ void k_pkb(const uint64_t* a, const uint64_t* e, const uint64_t* s, uint64_t* b, int logN) {
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int i = blockIdx.y;
    const ModConst mc = c_mod[i];
    const size_t off = (size_t)i * N + x;
    b[off] = mod_sub(e[off], mul_barrett(a[off], s[off], mc), mc.q);
}

// elementwise square of an eval-form polynomial over nmod limbs (s -> s^2)
__global__ void k_square(const uint64_t* a, uint64_t* o, int logN) {
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int m = blockIdx.y;
    const size_t off = (size_t)m * N + x;
    o[off] = mul_barrett(a[off], a[off], c_mod[m]);
}

}  // namespace fhe
