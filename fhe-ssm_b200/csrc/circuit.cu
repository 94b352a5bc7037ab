// circuit.cu -- scale-managed building blocks of the encrypted model circuit.
//
// The reference threads a TrackedCt (ciphertext + consumed levels, gpu_real_model.cu
// :1547-1551) through FLEXIBLEAUTO operations: EvalMult + RescaleInPlace (mulPt :2629-2632),
// the mult-by-one level alignment (alignTo :2636-2641), EvalAdd with level reconcile
// (addAligned :2692-2743).  Here every ciphertext carries its limb count and its exact scale
// (a double), and these helpers keep the scale at the level's FLEXIBLEAUTO factor:
//   * a plaintext or constant product picks its encoding scale so that the rescaled result
//     lands exactly on scale_at[nl-1];
//   * alignment to a lower level drops limbs for free and fixes the scale with one integer
//     constant product + rescale (one level, whatever the gap);
//   * constants are multiplied as exact integers; rounding is absorbed into the tracked scale.
#include <cmath>
#include <tuple>

#include "engine.h"

namespace fhe {

__global__ void k_signed_to_limbs(const int64_t*, uint64_t*, LimbMap, int);

static void require(bool c, const char* msg) {
    if (!c) throw Error(msg, -4);
}

double canon(const Context& cx, int nl) { return cx.scale_at[nl]; }

// out = a * M (integer, |M| < 2^126), no rescale; out may alias a (scale unchanged)
void mul_integer(Context& cx, const Ciphertext& a, long double M, Ciphertext& out) {
    LimbConst k{};
    k.has_w = 1;
    limb_residues(cx, M, a.nl, k.w);
    for (int i = 0; i < a.nl; i++) k.wp[i] = shoup_of(k.w[i], cx.mods[i]);
    const double sc = a.scale;
    apply_limb_const(cx, a, k, out);
    out.scale = sc;
}

// out = a * M + v (v at a's scale) in one pass over the limbs: the same words as mul_integer
// followed by ct_add_const (the Chebyshev doubling 2 T^2 - 1 and the double angles)
void mul_integer_add_const(Context& cx, const Ciphertext& a, long double M, double v, Ciphertext& out) {
    LimbConst k{};
    k.has_w = 1;
    limb_residues(cx, M, a.nl, k.w);
    for (int i = 0; i < a.nl; i++) k.wp[i] = shoup_of(k.w[i], cx.mods[i]);
    k.has_add = 1;
    limb_residues(cx, (long double)v * (long double)a.scale, a.nl, k.add);
    const double sc = a.scale;
    apply_limb_const(cx, a, k, out);
    out.scale = sc;
}

// value * c, rescaled once; the integer factor round(c * S) is chosen so that the output
// scale is `target` (default: the canonical factor of the output level).
void mul_const_rescale(Context& cx, const Ciphertext& a, double c, Ciphertext& out, double target) {
    require(a.nl >= 2, "mul_const_rescale: no level left");
    const int nl = a.nl;
    if (target <= 0) target = canon(cx, nl - 1);
    const long double S = (long double)target * (long double)cx.mods[nl - 1] / (long double)a.scale;
    const long double M = std::floor((long double)c * S + 0.5L);
    Ciphertext t;
    mul_integer(cx, a, M, t);
    // the value represented is a * M / S_eff with S_eff = M / c: keep the exact scale
    t.scale = (c != 0.0) ? a.scale * (double)(M / (long double)c) : a.scale * (double)S;
    ct_rescale(cx, t);
    out = std::move(t);
}

// K constant products a[k] * c[k] (one limb count), rescaled as one batch (mul_const_rescale each)
void mul_const_rescale_n(Context& cx, const Ciphertext* const* a, const double* c, int K, Ciphertext* out,
                         double target) {
    const int nl = a[0]->nl;
    require(nl >= 2, "mul_const_rescale: no level left");
    if (target <= 0) target = canon(cx, nl - 1);
    std::vector<Ciphertext*> t(K);
    for (int k = 0; k < K; k++) {
        require(a[k]->nl == nl, "mul_const_rescale_n: the ciphertexts differ in limb count");
        const long double S = (long double)target * (long double)cx.mods[nl - 1] / (long double)a[k]->scale;
        const long double M = std::floor((long double)c[k] * S + 0.5L);
        const double sc = a[k]->scale;
        mul_integer(cx, *a[k], M, out[k]);
        out[k].scale = (c[k] != 0.0) ? sc * (double)(M / (long double)c[k]) : sc * (double)S;
        t[k] = &out[k];
    }
    ct_rescale_n(cx, t.data(), K);
}

// bring a to nl_t limbs at scale `target` (default canonical).  nl_t < a.nl: one level used.
void align(Context& cx, Ciphertext& a, int nl_t, double target) {
    if (target <= 0) target = canon(cx, nl_t);
    require(nl_t >= 1 && nl_t <= a.nl, "align: bad target level");
    if (nl_t == a.nl) {
        const double r = a.scale / target;
        require(r > 1 - 1e-9 && r < 1 + 1e-9, "align: same level but different scale");
        return;
    }
    ct_level_drop(cx, a, nl_t + 1);
    Ciphertext t;
    mul_const_rescale(cx, a, 1.0, t, target);
    a = std::move(t);
}

// a and b to a common level (the lower one) with equal scales.  Equal-level operands whose
// scales differ by an integer factor are fixed by an exact integer product; any other ratio (a
// bootstrap's output against a product of canonical operands, say) by aligning both one level
// down onto the canonical scale there.
void match(Context& cx, Ciphertext& a, Ciphertext& b) {
    if (a.nl > b.nl) {
        align(cx, a, b.nl, b.scale);
        return;
    }
    if (b.nl > a.nl) {
        align(cx, b, a.nl, a.scale);
        return;
    }
    const double r = a.scale / b.scale;
    if (r > 1 - 1e-9 && r < 1 + 1e-9) return;
    Ciphertext* lo = r > 1 ? &b : &a;
    const double f = r > 1 ? r : 1.0 / r;
    const double fi = std::round(f);
    if (std::fabs(f - fi) < 1e-9 * f) {
        mul_integer(cx, *lo, fi, *lo);
        lo->scale *= fi;
        return;
    }
    require(a.nl >= 2, "match: equal levels with a non-integer scale ratio and no level left");
    align(cx, a, a.nl - 1, 0);
    align(cx, b, b.nl - 1, 0);
}

static bool same_level_scale(const Ciphertext& a, const Ciphertext& b) {
    const double r = a.scale / b.scale;
    return a.nl == b.nl && r > 1 - 1e-9 && r < 1 + 1e-9;
}

void add_any(Context& cx, const Ciphertext& a0, const Ciphertext& b0, Ciphertext& out) {
    if (same_level_scale(a0, b0)) {
        ct_add(cx, a0, b0, out);
        return;
    }
    Ciphertext a = ct_copy(cx, a0), b = ct_copy(cx, b0);
    match(cx, a, b);
    ct_add(cx, a, b, out);
}
void sub_any(Context& cx, const Ciphertext& a0, const Ciphertext& b0, Ciphertext& out) {
    if (same_level_scale(a0, b0)) {
        ct_sub(cx, a0, b0, out);
        return;
    }
    Ciphertext a = ct_copy(cx, a0), b = ct_copy(cx, b0);
    match(cx, a, b);
    ct_sub(cx, a, b, out);
}

// ct x ct at the common level, relinearised and rescaled
void mul_rescale(Context& cx, const Ciphertext& a, const Ciphertext& b, Ciphertext& out) {
    auto prod = [&](const Ciphertext& x, const Ciphertext& y) {
        if (cx.merged_rescale && cx.K <= 6) {   // the merged conversion sums K + 1 <= 7 lazy products
            ct_mul_relin_rescale(cx, x, y, out);
        } else {
            ct_mul_relin(cx, x, y, out);
            ct_rescale(cx, out);
        }
    };
    if (a.nl == b.nl) {
        prod(a, b);
    } else {
        Ciphertext x = ct_copy(cx, a.nl > b.nl ? a : b);
        const Ciphertext& y = a.nl > b.nl ? b : a;
        align(cx, x, y.nl, 0);
        prod(x, y);
    }
}

// per-slot product with a (complex) vector of n slots (n | N/2, repeated), then rescale; the
// plaintext scale makes the output scale `target` (default canonical)
void mul_vec_rescale(Context& cx, const Ciphertext& a, const std::complex<double>* v, int n, Ciphertext& out,
                     double target) {
    require(a.nl >= 2, "mul_vec_rescale: no level left");
    if (target <= 0) target = canon(cx, a.nl - 1);
    const double s = target * (double)cx.mods[a.nl - 1] / a.scale;
    const Plaintext& pt = encode_cached(cx, v, n, a.nl, s);
    Ciphertext t;
    ct_mul_pt(cx, a, pt, t);
    ct_rescale(cx, t);
    t.scale = target;   // exact by construction (a.scale * s / q)
    out = std::move(t);
}

// K per-slot products a[k] * v[k] (n slots each), one level of limbs for all, rescaled as one
// batch; each output lands on `target` (default: the canonical scale of the level below)
void mul_vec_rescale_n(Context& cx, const Ciphertext* const* a, const std::complex<double>* const* v, int n, int K,
                       Ciphertext* out, double target) {
    if (K == 1) { mul_vec_rescale(cx, *a[0], v[0], n, out[0], target); return; }
    const int nl = a[0]->nl;
    require(nl >= 2, "mul_vec_rescale: no level left");
    if (target <= 0) target = canon(cx, nl - 1);
    std::vector<Ciphertext*> t(K);
    for (int k = 0; k < K; k++) {
        require(a[k]->nl == nl, "mul_vec_rescale_n: the ciphertexts differ in limb count");
        const double s = target * (double)cx.mods[nl - 1] / a[k]->scale;
        const Plaintext& pt = encode_cached(cx, v[k], n, nl, s);
        ct_mul_pt(cx, *a[k], pt, out[k]);
        t[k] = &out[k];
    }
    ct_rescale_n(cx, t.data(), K);
    for (int k = 0; k < K; k++) out[k].scale = target;   // exact by construction
}

// align() of K ciphertexts to nl_t limbs and scale `target` (default canonical), the rescales batched
void align_n(Context& cx, Ciphertext* const* a, int K, int nl_t, double target) {
    if (target <= 0) target = canon(cx, nl_t);
    std::vector<Ciphertext*> todo;
    for (int k = 0; k < K; k++) {
        require(nl_t >= 1 && nl_t <= a[k]->nl, "align: bad target level");
        if (a[k]->nl == nl_t) {
            const double r = a[k]->scale / target;
            require(r > 1 - 1e-9 && r < 1 + 1e-9, "align: same level but different scale");
            continue;
        }
        ct_level_drop(cx, *a[k], nl_t + 1);
        const long double S = (long double)target * (long double)cx.mods[nl_t] / (long double)a[k]->scale;
        const long double M = std::floor(S + 0.5L);
        const double sc = a[k]->scale;
        mul_integer(cx, *a[k], M, *a[k]);
        a[k]->scale = sc * (double)M;
        todo.push_back(a[k]);
    }
    ct_rescale_n(cx, todo.data(), (int)todo.size());
}

// + vector (n slots, repeated) at the ciphertext's scale
void add_vec(Context& cx, const Ciphertext& a, const std::complex<double>* v, int n, Ciphertext& out) {
    const Plaintext& pt = encode_cached(cx, v, n, a.nl, a.scale);
    ct_add_pt(cx, a, pt, out);
}

// multiply by i in every slot: the monomial X^{N/2} (exact, no level, no scale change)
void mul_i(Context& cx, const Ciphertext& a, Ciphertext& out) {
    if (!cx.pt_i) {
        // coefficient form X^{N/2} -> NTT over all Q limbs
        std::vector<int64_t> coef(cx.N, 0);
        coef[cx.N / 2] = 1;
        auto pt = std::make_unique<Plaintext>();
        pt->buf = DevBuf((size_t)cx.L * cx.N, cx.stream);
        pt->nl = cx.L;
        pt->scale = 1.0;
        DevBuf dc((size_t)cx.N, cx.stream);
        CUDA_CHECK(cudaMemcpyAsync(dc.p, coef.data(), cx.N * 8, cudaMemcpyHostToDevice, cx.stream));
        LimbMap mp = cx.qmap(pt->buf.p, cx.L, (long long)cx.L * cx.N);
        k_signed_to_limbs<<<dim3(cx.N / 256, cx.L), 256, 0, cx.stream>>>((const int64_t*)dc.p, pt->buf.p, mp, cx.logN);
        CUDA_CHECK(cudaGetLastError());
        ntt(cx, mp, 1, false, cx.stream);
        CUDA_CHECK(cudaStreamSynchronize(cx.stream));
        cx.pt_i = std::move(pt);
    }
    const double sc = a.scale;
    Ciphertext t;
    ct_mul_pt(cx, a, *cx.pt_i, t);
    t.scale = sc;
    out = std::move(t);
}

// real and imaginary parts of every slot: re = (z + conj z), im = -i (z - conj z).  With
// halve (default) both carry twice the input scale, so they represent Re z and Im z exactly;
// without it they keep the input scale and represent 2 Re z and 2 Im z.
void split_complex(Context& cx, const Ciphertext& z, Ciphertext& re, Ciphertext& im, bool halve) {
    Ciphertext c;
    ct_conjugate(cx, z, c);
    Ciphertext s, d;
    ct_add(cx, z, c, s);
    ct_sub(cx, z, c, d);
    Ciphertext di;
    mul_i(cx, d, di);
    ct_mul_int(cx, di, -1, im);   // -i (z - conj z) = 2 Im(z)
    im.scale = (halve ? 2 : 1) * z.scale;
    re = std::move(s);
    re.scale = (halve ? 2 : 1) * z.scale;
}

// z = re + i im  (re, im real-valued ciphertexts)
void merge_complex(Context& cx, Ciphertext re, Ciphertext im, Ciphertext& z) {
    match(cx, re, im);
    Ciphertext ii;
    mul_i(cx, im, ii);
    ct_add(cx, re, ii, z);
}

// sum over a power-of-two window: out[i] = sum_{k < count} a[i + k*step] (log-doubling)
void rotate_sum(Context& cx, const Ciphertext& a, int step, int count, Ciphertext& out) {
    Ciphertext s = ct_copy(cx, a);
    for (int k = 1; k < count; k <<= 1) {
        Ciphertext r, t;
        ct_rotate(cx, s, k * step, r);
        ct_add(cx, s, r, t);
        s = std::move(t);
    }
    out = std::move(s);
}

// ---------------------------------------------------------------- Chebyshev evaluation ----
// p(x) = sum_i c_i T_i(x) on a ciphertext x with |x| <= 1, by the recursive baby-step /
// giant-step split p = q * T_{2^m} + r (Chebyshev division, T_i T_M = (T_{i+M} + T_{|i-M|})/2).
// Depth ceil(log2(deg+1)) + 1.  The babies T_1..T_{bs-1} are aligned to one level first.
// out = sum_t w_t . in_t over nl limbs and both polynomials, w_t a per-limb integer residue
// (Shoup): the leaf combinations of the Chebyshev evaluation in one pass.  <= kLinMax terms,
// each lazy product < 2q, so the sum stays below 16q.
constexpr int kLinMax = 8;
struct LinArgs {
    const uint64_t* in[kLinMax];
    long long stride[kLinMax];   // words between c0 and c1 of input t
    uint64_t w[kLinMax][kMaxMod], wp[kLinMax][kMaxMod];
    int nt;
};
__global__ void __launch_bounds__(256) k_lincomb(const LinArgs a, uint64_t* out, long long ostride, int logN) {
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int i = blockIdx.y, c = blockIdx.z;
    const uint64_t q = c_mod[i].q;
    uint64_t s = 0;
#pragma unroll
    for (int t = 0; t < kLinMax; t++) {
        if (t >= a.nt) break;
        const uint64_t v = a.in[t][(size_t)c * a.stride[t] + (size_t)i * N + x];
        s += mul_shoup_lazy(v, a.w[t][i], a.wp[t][i], q);
    }
    out[(size_t)c * ostride + (size_t)i * N + x] = reduce_lazy16(s, q);
}

// K products a[k] * b[k] relinearised and rescaled together (ct_mul_relin_rescale_n); operands
// of unequal levels are aligned first.  Falls back to one product at a time when the batch
// does not share a level.
void mul_rescale_n(Context& cx, const Ciphertext* const* a, const Ciphertext* const* b, int K, Ciphertext* out) {
    if (K == 1 || !cx.merged_rescale || cx.K > 6) {
        for (int k = 0; k < K; k++) mul_rescale(cx, *a[k], *b[k], out[k]);
        return;
    }
    std::vector<Ciphertext> tmp;
    tmp.reserve(K);
    std::vector<const Ciphertext*> A(K), B(K);
    for (int k = 0; k < K; k++) {
        if (a[k]->nl == b[k]->nl) { A[k] = a[k]; B[k] = b[k]; continue; }
        const bool ah = a[k]->nl > b[k]->nl;
        tmp.push_back(ct_copy(cx, ah ? *a[k] : *b[k]));
        align(cx, tmp.back(), (ah ? b[k] : a[k])->nl, 0);
        A[k] = ah ? &tmp.back() : a[k];
        B[k] = ah ? b[k] : &tmp.back();
    }
    for (int k = 1; k < K; k++)
        if (A[k]->nl != A[0]->nl) {
            for (int j = 0; j < K; j++) mul_rescale(cx, *A[j], *B[j], out[j]);
            return;
        }
    ct_mul_relin_rescale_n(cx, A.data(), B.data(), K, out);
}

// Chebyshev series sum_i c_i T_i(x) over K ciphertexts at once (same level and scale, same
// polynomial): every ciphertext product of the K evaluations is one batched product.
// Babies T_1 .. T_{bs-1} by T_i = 2 T_a T_b - T_{a-b} (a = ceil(i/2), b = floor(i/2)), giants
// T_{bs}, T_{2bs}, ... by doubling, and the series split recursively as p = q T_M + r down to
// leaves of degree < bs.
//   * A product or a difference of operands at two levels reads the higher one brought down to
//     the lower level (align: one constant product and rescale).  Such an aligned copy of a baby
//     or a giant is made once per level and kept (T_1 serves T_3, T_5 and T_7, a giant both
//     halves of the series below it).
//   * A leaf is one integer-weighted sum and one rescale.  Its babies are not aligned: baby i
//     enters through its first nl limbs (dropping limbs is free) with the integer weight
//     round(c_i tq / scale_i), so every term carries the common scale tq before the rescale.
struct ChebEvalN {
    Context& cx;
    int bs, K, lo = 0;
    std::vector<std::vector<Ciphertext>> T;         // T[i][k]
    std::map<int, std::vector<Ciphertext>> giant;   // T_{2^m}[k]
    std::map<std::tuple<const void*, int, double>, std::vector<Ciphertext>> memo;   // aligned copies

    // src (a baby or a giant of this evaluator) at nl limbs and scale `target`: src itself, or
    // its aligned copy, made on first use
    const std::vector<Ciphertext>& at(const std::vector<Ciphertext>& src, int nl, double target) {
        const double r = src[0].scale / target;
        if (src[0].nl == nl && r > 1 - 1e-9 && r < 1 + 1e-9) return src;
        const auto key = std::make_tuple((const void*)&src, nl, target);
        auto it = memo.find(key);
        if (it != memo.end()) return it->second;
        std::vector<Ciphertext> v(K);
        std::vector<Ciphertext*> pv(K);
        for (int k = 0; k < K; k++) {
            v[k] = ct_copy(cx, src[k]);
            pv[k] = &v[k];
        }
        align_n(cx, pv.data(), K, nl, target);
        return memo.emplace(key, std::move(v)).first->second;
    }
    void prod(const std::vector<Ciphertext>& a, const std::vector<Ciphertext>& b, std::vector<Ciphertext>& o) {
        std::vector<const Ciphertext*> pa(K), pb(K);
        for (int k = 0; k < K; k++) { pa[k] = &a[k]; pb[k] = &b[k]; }
        o.clear();
        o.resize(K);
        mul_rescale_n(cx, pa.data(), pb.data(), K, o.data());
    }
    // a * b for two persistent operands (babies, giants), the higher one read at the lower level
    void prod_at(const std::vector<Ciphertext>& a, const std::vector<Ciphertext>& b, std::vector<Ciphertext>& o) {
        if (a[0].nl == b[0].nl) prod(a, b, o);
        else if (a[0].nl > b[0].nl) prod(at(a, b[0].nl, canon(cx, b[0].nl)), b, o);
        else prod(a, at(b, a[0].nl, canon(cx, a[0].nl)), o);
    }
    // 2 a b - c (c = null: 2 a b - 1)
    std::vector<Ciphertext> cheb_step(const std::vector<Ciphertext>& a, const std::vector<Ciphertext>& b,
                                      const std::vector<Ciphertext>* c) {
        std::vector<Ciphertext> p;
        prod_at(a, b, p);
        std::vector<Ciphertext> r(K);
        if (!c) {
            for (int k = 0; k < K; k++) mul_integer_add_const(cx, p[k], 2, -1.0, r[k]);
            return r;
        }
        const std::vector<Ciphertext>& ca = at(*c, p[0].nl, p[0].scale);
        for (int k = 0; k < K; k++) {
            mul_integer(cx, p[k], 2, p[k]);
            ct_sub(cx, p[k], ca[k], r[k]);
        }
        return r;
    }
    ChebEvalN(Context& c, const Ciphertext* const* x, int K_, int degree) : cx(c), K(K_) {
        bs = 1;
        while (bs * bs < degree + 1) bs <<= 1;   // babies up to ~sqrt(deg)
        if (bs < 2) bs = 2;
        T.resize(bs);
        T[1].resize(K);
        for (int k = 0; k < K; k++) T[1][k] = ct_copy(cx, *x[k]);
        for (int i = 2; i < bs; i++) {
            const int a = (i + 1) / 2, b = i / 2;
            T[i] = cheb_step(T[a], T[b], a == b ? nullptr : &T[a - b]);
        }
        int M = bs;
        giant[M] = cheb_step(T[bs / 2], T[bs / 2], nullptr);
        while (2 * M <= degree) {
            giant[2 * M] = cheb_step(giant[M], giant[M], nullptr);
            M *= 2;
        }
        lo = T[1][0].nl;
        for (int i = 1; i < bs; i++) lo = std::min(lo, T[i][0].nl);
    }
    std::vector<Ciphertext> leaf(const std::vector<double>& c) {
        const int nl = lo;
        const double target = canon(cx, nl - 1);
        const double tq = target * (double)cx.mods[nl - 1];
        std::vector<Ciphertext> out(K);
        LinArgs la{};
        std::vector<int> terms;
        for (int i = 1; i < (int)c.size() && i < bs; i++) {
            if (c[i] == 0.0) continue;
            if (la.nt == kLinMax) throw Error("chebyshev: too many baby terms in one leaf", -1);
            const int t = la.nt++;
            terms.push_back(i);
            limb_residues(cx, std::floor((long double)c[i] * (long double)(tq / T[i][0].scale) + 0.5L), nl, la.w[t]);
            for (int l = 0; l < nl; l++) la.wp[t][l] = shoup_of(la.w[t][l], cx.mods[l]);
        }
        if (la.nt == 0) { la.nt = 1; terms.push_back(1); }   // constant-only leaf: 0 * T_1
        std::vector<Ciphertext*> pacc(K);
        for (int k = 0; k < K; k++) {
            for (int t = 0; t < la.nt; t++) {
                la.in[t] = T[terms[t]][k].c(0);
                la.stride[t] = (long long)T[terms[t]][k].stride;
            }
            out[k] = ct_alloc(cx, nl);
            {
                ProfScope ps(cx, "lincomb", 8.0 * cx.N * nl * 2 * (la.nt + 1));
                k_lincomb<<<dim3(cx.N / 256, nl, 2), 256, 0, cx.stream>>>(la, out[k].c(0), (long long)out[k].stride,
                                                                          cx.logN);
                CUDA_CHECK(cudaGetLastError());
                cx.launches++;
            }
            out[k].scale = tq;
            pacc[k] = &out[k];
        }
        ct_rescale_n(cx, pacc.data(), K);
        for (int k = 0; k < K; k++) {
            out[k].scale = target;
            if (!c.empty() && c[0] != 0.0) {
                Ciphertext u;
                ct_add_const(cx, out[k], c[0], u);
                out[k] = std::move(u);
            }
        }
        return out;
    }
    std::vector<Ciphertext> eval(std::vector<double> c) {
        int deg = (int)c.size() - 1;
        while (deg > 0 && c[deg] == 0.0) deg--;
        c.resize(deg + 1);
        if (deg < bs) return leaf(c);
        int M = bs;
        while (2 * M <= deg) M *= 2;
        // p = q T_M + r
        std::vector<double> q(deg - M + 1), r(c.begin(), c.begin() + M);
        q[0] = c[M];
        for (int i = M + 1; i <= deg; i++) {
            q[i - M] = 2 * c[i];
            r[2 * M - i] -= c[i];
        }
        std::vector<Ciphertext> qv = eval(q), rv = eval(r), pr;
        if (qv[0].nl <= giant[M][0].nl) {
            prod(qv, at(giant[M], qv[0].nl, qv[0].scale), pr);
        } else {   // never for the trees of cheb_depth (a leaf sits below every giant it meets)
            for (int k = 0; k < K; k++) align(cx, qv[k], giant[M][0].nl, giant[M][0].scale);
            prod(qv, giant[M], pr);
        }
        std::vector<Ciphertext> out(K);
        if (rv[0].nl > pr[0].nl) {
            std::vector<Ciphertext*> prv(K);
            for (int k = 0; k < K; k++) prv[k] = &rv[k];
            align_n(cx, prv.data(), K, pr[0].nl, pr[0].scale);
        }
        for (int k = 0; k < K; k++) {
            if (rv[k].nl == pr[k].nl) ct_add(cx, pr[k], rv[k], out[k]);
            else add_any(cx, pr[k], rv[k], out[k]);
        }
        return out;
    }
};

// Levels consumed by ChebEvalN on a canonical-scale input: the same tree on depths (a product
// is one level below its deeper operand; a leaf is one level below the deepest baby).
static int cheb_depth_rec(std::vector<double> c, int bs, int lo, const std::map<int, int>& gd) {
    int deg = (int)c.size() - 1;
    while (deg > 0 && c[deg] == 0.0) deg--;
    c.resize(deg + 1);
    if (deg < bs) return lo + 1;
    int M = bs;
    while (2 * M <= deg) M *= 2;
    std::vector<double> q(deg - M + 1), r(c.begin(), c.begin() + M);
    q[0] = c[M];
    for (int i = M + 1; i <= deg; i++) {
        q[i - M] = 2 * c[i];
        r[2 * M - i] -= c[i];
    }
    const int dq = cheb_depth_rec(q, bs, lo, gd), dr = cheb_depth_rec(r, bs, lo, gd);
    return std::max(std::max(dq, gd.at(M)) + 1, dr);
}
int cheb_depth(const std::vector<double>& coeffs) {
    const int degree = (int)coeffs.size() - 1;
    int bs = 1;
    while (bs * bs < degree + 1) bs <<= 1;
    if (bs < 2) bs = 2;
    std::vector<int> d(bs, 0);
    for (int i = 2; i < bs; i++) d[i] = std::max(d[(i + 1) / 2], d[i / 2]) + 1;
    int lo = 0;
    for (int i = 1; i < bs; i++) lo = std::max(lo, d[i]);
    std::map<int, int> gd;
    int M = bs;
    gd[M] = d[bs / 2] + 1;
    while (2 * M <= degree) {
        gd[2 * M] = gd[M] + 1;
        M *= 2;
    }
    return cheb_depth_rec(coeffs, bs, lo, gd);
}

// cheb_eval over K ciphertexts at one level and scale, products batched
void cheb_eval_n(Context& cx, const Ciphertext* const* x, int K, const std::vector<double>& coeffs, Ciphertext* out) {
    std::vector<Ciphertext> y;
    std::vector<const Ciphertext*> px(x, x + K);
    if (x[0]->scale / canon(cx, x[0]->nl) > 1 + 1e-9 || x[0]->scale / canon(cx, x[0]->nl) < 1 - 1e-9) {
        y.reserve(K);
        for (int k = 0; k < K; k++) {
            y.push_back(ct_copy(cx, *x[k]));
            align(cx, y.back(), y.back().nl - 1, 0);
            px[k] = &y.back();
        }
    }
    ChebEvalN ev(cx, px.data(), K, (int)coeffs.size() - 1);
    std::vector<Ciphertext> r = ev.eval(coeffs);
    for (int k = 0; k < K; k++) out[k] = std::move(r[k]);
}

void cheb_eval(Context& cx, const Ciphertext& x, const std::vector<double>& coeffs, Ciphertext& out) {
    const Ciphertext* px[1] = {&x};
    cheb_eval_n(cx, px, 1, coeffs, &out);
}

// sum_i c_i (.) x^i with per-slot coefficient vectors c_i (n slots each, repeated), power
// basis, depth ceil(log2 deg) + 1, for K inputs at once (each with its own coefficients; the
// power products of the K evaluations are batched products).  The powers are not aligned to one
// level: each is level-dropped (free) to the lowest power's level, multiplied by its coefficient
// plaintext, whose encoding scale lands the product on the canonical scale of the level below,
// and the terms are summed; c_0 is added last.  (polyGate3 and the channel-mix polynomials of
// gpu_real_model.cu:4609-4649, :5130-5163, evaluated without the reference's per-term alignTo
// chain.)
void poly_eval_vec_n(Context& cx, const Ciphertext* const* xs, int K,
                     const std::vector<std::vector<std::complex<double>>>* const* cs, int n, Ciphertext* outs) {
    std::vector<std::vector<Ciphertext>> pw(K);
    int maxdeg = 0;
    for (int k = 0; k < K; k++) {
        const int deg = (int)cs[k]->size() - 1;
        require(deg >= 1, "poly_eval_vec: degree must be >= 1");
        maxdeg = std::max(maxdeg, deg);
        pw[k].resize(deg + 1);
        pw[k][1] = ct_copy(cx, *xs[k]);
        const double r = pw[k][1].scale / canon(cx, xs[k]->nl);
        if (r > 1 + 1e-9 || r < 1 - 1e-9) align(cx, pw[k][1], xs[k]->nl - 1, 0);
    }
    for (int i = 2; i <= maxdeg; i++) {   // x^i = x^a x^b for every input of degree >= i
        const int a = (i + 1) / 2, b = i / 2;
        std::vector<const Ciphertext*> pa, pb;
        std::vector<int> who;
        for (int k = 0; k < K; k++)
            if ((int)pw[k].size() > i) { pa.push_back(&pw[k][a]); pb.push_back(&pw[k][b]); who.push_back(k); }
        std::vector<Ciphertext> o(who.size());
        mul_rescale_n(cx, pa.data(), pb.data(), (int)who.size(), o.data());
        for (size_t j = 0; j < who.size(); j++) pw[who[j]][i] = std::move(o[j]);
    }
    // the coefficient products of every input, one batch per limb count
    std::vector<std::complex<double>> zero(n, 0.0);
    struct Term { int k, i; const std::complex<double>* v; };
    std::map<int, std::vector<Term>> by_nl;
    for (int k = 0; k < K; k++) {
        const auto& c = *cs[k];
        const int deg = (int)c.size() - 1;
        int lo = pw[k][1].nl;
        for (int i = 1; i <= deg; i++) lo = std::min(lo, pw[k][i].nl);
        bool have = false;
        for (int i = 1; i <= deg; i++) {
            bool nz = false;
            for (auto& v : c[i]) if (v != 0.0) { nz = true; break; }
            if (!nz) continue;
            ct_level_drop(cx, pw[k][i], lo);
            by_nl[lo].push_back({k, i, c[i].data()});
            have = true;
        }
        if (!have) {   // all-zero polynomial: 0 * x keeps a valid ciphertext
            ct_level_drop(cx, pw[k][1], lo);
            by_nl[lo].push_back({k, 1, zero.data()});
        }
    }
    std::vector<Ciphertext> acc(K);
    std::vector<char> have(K, 0);
    for (auto& g : by_nl) {
        const auto& terms = g.second;
        const int B = (int)terms.size();
        std::vector<const Ciphertext*> in(B);
        std::vector<const std::complex<double>*> vs(B);
        for (int j = 0; j < B; j++) { in[j] = &pw[terms[j].k][terms[j].i]; vs[j] = terms[j].v; }
        std::vector<Ciphertext> prod(B);
        mul_vec_rescale_n(cx, in.data(), vs.data(), n, B, prod.data(), 0);
        for (int j = 0; j < B; j++) {
            const int k = terms[j].k;
            if (!have[k]) { acc[k] = std::move(prod[j]); have[k] = 1; }
            else { Ciphertext u; ct_add(cx, acc[k], prod[j], u); acc[k] = std::move(u); }
        }
    }
    for (int k = 0; k < K; k++) add_vec(cx, acc[k], (*cs[k])[0].data(), n, outs[k]);
}

void poly_eval_vec(Context& cx, const Ciphertext& x, const std::vector<std::vector<std::complex<double>>>& c, int n,
                   Ciphertext& out) {
    const Ciphertext* px[1] = {&x};
    const std::vector<std::vector<std::complex<double>>>* pc[1] = {&c};
    poly_eval_vec_n(cx, px, 1, pc, n, &out);
}

// Chebyshev interpolant of f on [a, b] of degree n (Chebyshev nodes of the first kind)
std::vector<double> cheb_fit(double (*f)(double, const void*), const void* arg, double a, double b, int n) {
    std::vector<double> c(n + 1, 0.0), fx(n + 1);
    for (int k = 0; k <= n; k++) {
        const double t = std::cos(M_PI * (k + 0.5) / (n + 1));
        fx[k] = f(0.5 * (b - a) * t + 0.5 * (a + b), arg);
    }
    for (int j = 0; j <= n; j++) {
        double s = 0;
        for (int k = 0; k <= n; k++) s += fx[k] * std::cos(M_PI * j * (k + 0.5) / (n + 1));
        c[j] = (j == 0 ? 1.0 : 2.0) * s / (n + 1);
    }
    return c;
}

}  // namespace fhe
