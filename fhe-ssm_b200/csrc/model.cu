// model.cu -- the encrypted recurrent step of the polynomial SSM language model over a pack
// of conversations (the layer loop of gpu_real_model.cu:4744-5264, the carry :4688-4737 /
// :5271-5300, the output norm :5380-5389), float64 semantics of train_fhe_native_ssm.py
// `_fwd_np` (:829-890).
//
// Packing.  The residual stream of every conversation is a d-vector (padded to D = 2^k >= d);
// slot r*D + c holds channel c of lane r (R = N/2/D blocks), and each complex slot carries two
// lanes: lane r in the real part and lane r + R in the imaginary part, so one ciphertext holds
// 2R conversations (64 at N = 2^16, D = 1024).  Linear maps with real coefficients act on both
// parts at once; the polynomial nonlinearities (gate, activations, the Newton rsqrt) act on
// the real and imaginary parts separately (split by a conjugation, merged after).
//
// Per layer (sequential block):
//   u  = rmsnorm(h, g1)                          (rotate-sum of x^2 over a block, linear seed,
//                                                 depth-2 Newton y' = 1.5y + (-ms/2 y)(y^2))
//   u  = mix . u + (1 - mix) . u_prev            (shift-mix; u_prev carried)
//   x  = Win u;  s = a . s_prev + (1 - a) . x    (scan state s carried)
//   z  = c . s + dd . x;  g = z (p0 + p1 z + p2 z^2);  h += alpha Wout g
//   v  = rmsnorm(h, g2);  k_j = Wk_j v, r_j = Wr_j v (dff in chunks of D, shared babies)
//   f  = (q0 + q1 k + q2 k^2 + q3 k^3) (r0 + r1 r + r2 r^2);  h += Wv [f_0 | f_1 | ...]
// then y = rmsnorm(h, g_out).  A ciphertext is bootstrapped when it cannot cover the levels
// of the next operation (the reference's refresh rule, gpu_real_model.cu:2573-2599).
#include <cmath>

#include "engine.h"

namespace fhe {

struct NormSeed {
    double a = 1.0, b = 0.0;
    int iters = 0;
    double gx = 1.0, gms = 1.0;   // bootstrap gains of the input and of mean(x^2) + eps
    double gy = 1.0;              // bootstrap gain of the Newton iterate (~ 1/sqrt(ms))
};

struct ModelCfg {
    int d = 0, dff = 0, n_layer = 0, D = 0, b1 = 32;
    double a_min = 0.9, a_max = 0.9995, alpha = 1.0, eps = 1e-5;
    bool shift_mix = true;
};

struct LayerParams {
    std::shared_ptr<MatvecPlan> win, wout, wv;
    std::vector<std::shared_ptr<MatvecPlan>> wk, wr;
    std::vector<double> decay, bco, g1, mix, c, dd, p0, p1, p2, g2;
    std::vector<double> q[4], r[3];
    NormSeed tm, cm;
    // bootstrap gains of the refresh sites (shift-mix output, scan state, gate output,
    // channel-mix input, channel-mix products): a bootstrap's error is absolute, so a site
    // whose values are small is refreshed at value * gain (a relabelling of the scale,
    // exact) and relabelled back
    double g_u = 1, g_s = 1, g_g = 1, g_v = 1, g_f = 1, g_z = 1;
    bool ready = false;
};

struct Model {
    Context& cx;
    ModelCfg cfg;
    int C = 1;   // dff chunks of D
    std::vector<LayerParams> L;
    std::vector<double> g_out;
    NormSeed out_seed;
    std::vector<Ciphertext> s, up;   // carried state per layer
    bool have_state = false;
    long long boots = 0, steps = 0;
    // diagnostics: when > 0, step() returns the layer-0 intermediate number `probe`
    // (1 norm, 2 shift-mix, 3 Win x, 4 scan s, 5 readout z, 6 gate g, 7 h + attn, 8 norm 2,
    //  9 k_0, 10 f_0, 11 h + ffn)
    int probe = 0;
    explicit Model(Context& c) : cx(c) {}

    // ------------------------------------------------------------------ helpers ----
    // channels [off, off + D) of a per-channel vector as one block period (zero padded)
    std::vector<std::complex<double>> slots(const std::vector<double>& v, int off = 0) const {
        std::vector<std::complex<double>> z(cfg.D, 0.0);
        for (int i = 0; i < cfg.D && off + i < (int)v.size(); i++) z[i] = v[off + i];
        return z;
    }
    // refresh sites (bootstrap census, fhe_model_refresh_census)
    enum Site { kNormX, kNormMs, kNormY, kNormM, kNormTail, kXn, kUp, kU, kSp, kSnew, kZ, kG, kV, kF, kSites };
    long long site_boots[kSites] = {};
    void refresh(Ciphertext& a, int need, double gain, Site site) {
        if (a.nl - 1 >= need) return;
        site_boots[site]++;
        ProfScope op(cx, "op:refresh", 0);
        Ciphertext t;
        a.scale /= gain;   // the ciphertext now represents value * gain
        bootstrap(cx, a, t);
        t.scale *= gain;
        a = std::move(t);
        boots++;
        if (a.nl - 1 < need) throw Error("model: a bootstrap does not leave enough levels for this operation", -4);
    }
    Ciphertext mulv(const Ciphertext& a, const std::vector<double>& v) {
        auto z = slots(v);
        Ciphertext o;
        mul_vec_rescale(cx, a, z.data(), cfg.D, o, 0);
        return o;
    }
    // a * va + b * vb (per-channel vectors): both inputs read at the lower of their levels (a
    // limb drop, free) so that the two products are one batch and land on one level and scale
    Ciphertext mulv_sum(const Ciphertext& a, const std::vector<double>& va, const Ciphertext& b,
                        const std::vector<double>& vb) {
        const int lo = std::min(a.nl, b.nl);
        Ciphertext& ma = const_cast<Ciphertext&>(a);
        Ciphertext& mb = const_cast<Ciphertext&>(b);
        const int na = a.nl, nb = b.nl;
        ma.nl = lo;
        mb.nl = lo;
        auto za = slots(va), zb = slots(vb);
        const Ciphertext* in[2] = {&a, &b};
        const std::complex<double>* vs[2] = {za.data(), zb.data()};
        Ciphertext o[2];
        mul_vec_rescale_n(cx, in, vs, cfg.D, 2, o, 0);
        ma.nl = na;
        mb.nl = nb;
        Ciphertext r;
        ct_add(cx, o[0], o[1], r);
        return r;
    }
    Ciphertext addc(const Ciphertext& a, const Ciphertext& b) {
        Ciphertext o;
        add_any(cx, a, b, o);
        return o;
    }

    // polynomials with per-channel coefficient vectors on complex-packed ciphertexts: zs[j]
    // with coefficients cs[j] (channels from offs[j]); out[2 j] and out[2 j + 1] are the real
    // and imaginary parts of the result.  The power products of all 2 J parts run batched.
    void poly_parts(const std::vector<const Ciphertext*>& zs,
                    const std::vector<std::vector<const std::vector<double>*>>& cs, const std::vector<int>& offs,
                    std::vector<Ciphertext>& out) {
        ProfScope op(cx, "op:poly", 0);
        const int J = (int)zs.size();
        std::vector<Ciphertext> parts(2 * J);
        std::vector<std::vector<std::vector<std::complex<double>>>> c(J);
        for (int j = 0; j < J; j++) {
            split_complex(cx, *zs[j], parts[2 * j], parts[2 * j + 1], true);
            for (auto* v : cs[j]) c[j].push_back(slots(*v, offs[j]));
        }
        std::vector<const Ciphertext*> px(2 * J);
        std::vector<const std::vector<std::vector<std::complex<double>>>*> pc(2 * J);
        for (int k = 0; k < 2 * J; k++) { px[k] = &parts[k]; pc[k] = &c[k / 2]; }
        out.clear();
        out.resize(2 * J);
        poly_eval_vec_n(cx, px.data(), 2 * J, pc.data(), cfg.D, out.data());
    }
    Ciphertext poly_complex(const Ciphertext& z, const std::vector<const std::vector<double>*>& coeffs, int off = 0) {
        std::vector<Ciphertext> p;
        poly_parts({&z}, {coeffs}, {off}, p);
        Ciphertext o;
        merge_complex(cx, std::move(p[0]), std::move(p[1]), o);
        return o;
    }
    // K products a[k] * b[k], relinearised and rescaled as one batch
    void mul_n(const std::vector<const Ciphertext*>& a, const std::vector<const Ciphertext*>& b,
               std::vector<Ciphertext>& out) {
        out.clear();
        out.resize(a.size());
        mul_rescale_n(cx, a.data(), b.data(), (int)a.size(), out.data());
    }

    // rmsnorm: x / sqrt(mean(x^2) + eps) * g per lane (rmsnorm, gpu_real_model.cu:3451-3657)
    Ciphertext rmsnorm(const Ciphertext& x0, const std::vector<double>& g, const NormSeed& sd) {
        ProfScope op(cx, "op:rmsnorm", 0);
        const int D = cfg.D;
        Ciphertext x = ct_copy(cx, x0);
        refresh(x, 3, sd.gx, kNormX);
        Ciphertext xr, xi;
        split_complex(cx, x, xr, xi, true);
        Ciphertext sq;
        {
            std::vector<Ciphertext> s2;
            mul_n({&xr, &xi}, {&xr, &xi}, s2);
            merge_complex(cx, std::move(s2[0]), std::move(s2[1]), sq);
        }
        // block sums land on channel 0 of every block, then are broadcast back
        Ciphertext t;
        rotate_sum(cx, sq, 1, D, t);
        std::vector<double> mask(D, 0.0);
        mask[0] = 1.0 / cfg.d;
        Ciphertext m = mulv(t, mask);
        Ciphertext ms;
        rotate_sum(cx, m, -1, D, ms);
        {   // + eps for the lanes of both parts: eps (1 + i) in every slot
            std::vector<std::complex<double>> ee(D, std::complex<double>(cfg.eps, cfg.eps));
            Ciphertext e;
            add_vec(cx, ms, ee.data(), D, e);
            ms = std::move(e);
        }
        const int maxlv = bootstrap_levels_after(cx) - 1;
        refresh(ms, std::min(2 + 2 * sd.iters, maxlv), sd.gms, kNormMs);
        // the Newton chain runs on complex-packed (y, -ms/2) pairs: seed and iterations act on
        // the real and imaginary parts separately, and a pair that runs out of levels between
        // iterations is merged and bootstrapped once (one bootstrap serves both parts)
        Ciphertext mr, mi;
        split_complex(cx, ms, mr, mi, true);
        Ciphertext yp[2], mh[2];
        Ciphertext* mparts[2] = {&mr, &mi};
        {   // seed a + b ms and -ms/2 of both parts: four constant products, one batched rescale
            const Ciphertext* in[4] = {mparts[0], mparts[0], mparts[1], mparts[1]};
            const double cs4[4] = {sd.b, -0.5, sd.b, -0.5};
            Ciphertext o[4];
            mul_const_rescale_n(cx, in, cs4, 4, o, 0);
            for (int P = 0; P < 2; P++) {
                ct_add_const(cx, o[2 * P], sd.a, yp[P]);
                mh[P] = std::move(o[2 * P + 1]);
            }
        }
        for (int it = 0; it < sd.iters; it++) {
            if (yp[0].nl - 1 < 2 + (it + 1 == sd.iters ? 1 : 0)) {
                Ciphertext yc, mc;
                merge_complex(cx, std::move(yp[0]), std::move(yp[1]), yc);
                merge_complex(cx, std::move(mh[0]), std::move(mh[1]), mc);
                const int rest = 2 * (sd.iters - it) + 1;
                refresh(yc, std::min(rest, maxlv), sd.gy, kNormY);
                refresh(mc, std::min(rest, maxlv), sd.gms * 2, kNormM);
                split_complex(cx, yc, yp[0], yp[1], true);
                split_complex(cx, mc, mh[0], mh[1], true);
            }
            // y <- 1.5 y + (-ms/2) y^3 on both parts: {y^2, (-ms/2) y} of both parts as one batch
            // of four products, then their product as one batch of two
            std::vector<Ciphertext> sq2, u;
            mul_n({&yp[0], &mh[0], &yp[1], &mh[1]}, {&yp[0], &yp[0], &yp[1], &yp[1]}, sq2);
            mul_n({&sq2[1], &sq2[3]}, {&sq2[0], &sq2[2]}, u);
            for (int P = 0; P < 2; P++) {
                Ciphertext y3;
                mul_integer(cx, yp[P], 3, y3);   // 1.5 y at twice the scale
                y3.scale = yp[P].scale * 2;
                Ciphertext yn;
                add_any(cx, y3, u[P], yn);
                yp[P] = std::move(yn);
            }
        }
        if (yp[0].nl < 2) {
            Ciphertext yc;
            merge_complex(cx, std::move(yp[0]), std::move(yp[1]), yc);
            refresh(yc, 1, sd.gy, kNormTail);
            split_complex(cx, yc, yp[0], yp[1], true);
        }
        // x g at the level of y: the parts of x are level-dropped (free) to one limb above y,
        // so that the gain product lands on y's level and scale without an alignment
        if (xr.nl > yp[0].nl + 1) { ct_level_drop(cx, xr, yp[0].nl + 1); ct_level_drop(cx, xi, yp[0].nl + 1); }
        Ciphertext xgr = mulv(xr, g), xgi = mulv(xi, g);
        std::vector<Ciphertext> outp;
        mul_n({&xgr, &xgi}, {&yp[0], &yp[1]}, outp);
        Ciphertext out;
        merge_complex(cx, std::move(outp[0]), std::move(outp[1]), out);
        return out;
    }

    // ---------------------------------------------------------------------- step ----
    Ciphertext step(const Ciphertext& emb) {
        const int nL = cfg.n_layer;
        if (!have_state) { s.clear(); up.clear(); s.resize(nL); up.resize(nL); }
        Ciphertext h = ct_copy(cx, emb);
        // the model runs in the user region of the chain (the top limbs are the bootstrap's)
        const int utop = cx.L - cx.prm.boot_primes;
        if (h.nl > utop) align(cx, h, utop, 0);
        for (int l = 0; l < nL; l++) {
            LayerParams& P = L[l];
            if (!P.ready) throw Error("model: layer weights not set", -1);
            // ---- time mix
#define FHE_PROBE(k, ct) \
    if (probe % 100 == (k) && l == probe / 100) return ct_copy(cx, ct);
            Ciphertext xn = rmsnorm(h, P.g1, P.tm);
            FHE_PROBE(1, xn)
            Ciphertext u;
            if (cfg.shift_mix) {
                std::vector<double> om(P.mix.size());
                for (size_t i = 0; i < om.size(); i++) om[i] = 1.0 - P.mix[i];
                refresh(xn, 1, P.g_u, kXn);
                if (have_state) {
                    refresh(up[l], 1, P.g_u, kUp);
                    u = mulv_sum(xn, P.mix, up[l], om);
                } else {
                    u = mulv(xn, P.mix);
                }
                up[l] = ct_copy(cx, xn);
            } else {
                u = std::move(xn);
            }
            FHE_PROBE(2, u)
            refresh(u, 7, P.g_u, kU);
            Ciphertext x;
            {
                const Ciphertext* in[1] = {&u};
                matvec(cx, *P.win, in, x);
            }
            FHE_PROBE(3, x)
            Ciphertext snew;
            if (have_state) {
                Ciphertext sp = ct_copy(cx, s[l]);
                refresh(sp, 1, P.g_s, kSp);
                snew = mulv_sum(sp, P.decay, x, P.bco);
            } else {
                snew = mulv(x, P.bco);
            }
            // the carried state loses a level per step: refresh it (and keep the refreshed copy
            // as the carry) when the readout z could not cover the gate polynomial
            refresh(snew, 5, P.g_s, kSnew);
            s[l] = ct_copy(cx, snew);
            FHE_PROBE(4, snew)
            Ciphertext z = mulv_sum(snew, P.c, x, P.dd);
            refresh(z, 4, P.g_z, kZ);
            FHE_PROBE(5, z)
            std::vector<double> zero(cfg.d, 0.0);
            Ciphertext g = poly_complex(z, {&zero, &P.p0, &P.p1, &P.p2});
            FHE_PROBE(6, g)
            refresh(g, 1, P.g_g, kG);
            Ciphertext attn;
            {
                const Ciphertext* in[1] = {&g};
                matvec(cx, *P.wout, in, attn);
            }
            if (cfg.alpha != 1.0) {
                Ciphertext t;
                mul_const_rescale(cx, attn, cfg.alpha, t, 0);
                attn = std::move(t);
            }
            h = addc(h, attn);
            FHE_PROBE(7, h)
            // ---- channel mix
            Ciphertext v = rmsnorm(h, P.g2, P.cm);
            FHE_PROBE(8, v)
            refresh(v, 6, P.g_v, kV);
            BabySet bs;
            matvec_babies(cx, v, cfg.D, cfg.b1, bs);
            const BabySet* bsp[1] = {&bs};
            // k_j = Wk_j v and r_j = Wr_j v for every chunk, then the activation and gate
            // polynomials of all chunks on their real and imaginary parts (power products
            // batched over the 4 C parts), then act * gate part by part (one batch of 2 C
            // products), merged per chunk
            std::vector<Ciphertext> kr(2 * C);
            for (int ch = 0; ch < C; ch++) {
                matvec_apply(cx, *P.wk[ch], bsp, kr[2 * ch]);
                matvec_apply(cx, *P.wr[ch], bsp, kr[2 * ch + 1]);
                if (ch == 0) FHE_PROBE(9, kr[0])
            }
            std::vector<const Ciphertext*> zs(2 * C);
            std::vector<std::vector<const std::vector<double>*>> pcs(2 * C);
            std::vector<int> offs(2 * C);
            for (int ch = 0; ch < C; ch++) {
                zs[2 * ch] = &kr[2 * ch];
                pcs[2 * ch] = {&P.q[0], &P.q[1], &P.q[2], &P.q[3]};
                zs[2 * ch + 1] = &kr[2 * ch + 1];
                pcs[2 * ch + 1] = {&P.r[0], &P.r[1], &P.r[2]};
                offs[2 * ch] = offs[2 * ch + 1] = ch * cfg.D;
            }
            std::vector<Ciphertext> pp;   // [chunk][act / gate][re / im]
            poly_parts(zs, pcs, offs, pp);
            std::vector<const Ciphertext*> pa, pg;
            for (int ch = 0; ch < C; ch++)
                for (int q = 0; q < 2; q++) { pa.push_back(&pp[4 * ch + q]); pg.push_back(&pp[4 * ch + 2 + q]); }
            std::vector<Ciphertext> fp;
            mul_n(pa, pg, fp);
            std::vector<Ciphertext> f(C);
            for (int ch = 0; ch < C; ch++) merge_complex(cx, std::move(fp[2 * ch]), std::move(fp[2 * ch + 1]), f[ch]);
            FHE_PROBE(10, f[0])
            // the chunks ran identical pipelines: bring any stragglers to the lowest one
            int lo = 0;
            for (int ch = 1; ch < C; ch++) if (f[ch].nl < f[lo].nl) lo = ch;
            for (int ch = 0; ch < C; ch++)
                if (f[ch].nl > f[lo].nl) align(cx, f[ch], f[lo].nl, f[lo].scale);
            if (f[0].nl < 2)
                for (auto& c : f) refresh(c, 1, P.g_f, kF);
            std::vector<const Ciphertext*> fin(C);
            for (int ch = 0; ch < C; ch++) fin[ch] = &f[ch];
            FHE_PROBE(12, f[C - 1])
            Ciphertext ffn;
            matvec(cx, *P.wv, fin.data(), ffn);
            FHE_PROBE(13, ffn)
            h = addc(h, ffn);
            FHE_PROBE(11, h)
#undef FHE_PROBE
        }
        have_state = true;
        steps++;
        return rmsnorm(h, g_out, out_seed);
    }
};

// the rotation amounts of a step: the BSGS matvec's babies and giants and the rmsnorm's block
// sums (+2^k up, -2^k back down); the conjugation (complex split) comes on top
std::vector<int> model_rotation_steps(const ModelCfg& cfg) {
    std::vector<int> r = matvec_rotations(cfg.D, cfg.b1);
    for (int k = 1; k < cfg.D; k <<= 1) { r.push_back(k); r.push_back(-k); }
    return r;
}

// ------------------------------------------------------------------ construction API ----
std::shared_ptr<Model> model_create(Context& cx, const ModelCfg& cfg) {
    if (cfg.d < 1 || cfg.D < cfg.d || (cfg.D & (cfg.D - 1)) || (cx.N / 2) % cfg.D)
        throw Error("model: D must be a power of two >= d dividing N/2", -1);
    if (cfg.dff % cfg.D && cfg.dff > cfg.D) throw Error("model: dff must be a multiple of D", -1);
    auto m = std::make_shared<Model>(cx);
    m->cfg = cfg;
    m->C = std::max(1, (cfg.dff + cfg.D - 1) / cfg.D);
    m->L.resize(cfg.n_layer);
    return m;
}

// vecs: d-length decay, bco, g1, mix, c, dd, p0, p1, p2, g2 then dff-length q0..q3, r0..r2
// seeds: tm (a, b, iters), cm (a, b, iters)
void model_set_layer(Model& m, int l, const double* win, const double* wout, const double* wk, const double* wr,
                     const double* wv, const double* vecs, const double* seeds) {
    if (l < 0 || l >= m.cfg.n_layer) throw Error("model: layer index out of range", -1);
    const int d = m.cfg.d, dff = m.cfg.dff, D = m.cfg.D, b1 = m.cfg.b1;
    LayerParams& P = m.L[l];
    P.win = matvec_plan(m.cx, win, d, d, D, b1);
    P.wout = matvec_plan(m.cx, wout, d, d, D, b1);
    P.wv = matvec_plan(m.cx, wv, d, dff, D, b1);
    P.wk.clear();
    P.wr.clear();
    for (int ch = 0; ch < m.C; ch++) {
        const int r0 = ch * D, rows = std::min(D, dff - r0);
        P.wk.push_back(matvec_plan(m.cx, wk + (size_t)r0 * d, rows, d, D, b1));
        P.wr.push_back(matvec_plan(m.cx, wr + (size_t)r0 * d, rows, d, D, b1));
    }
    std::vector<double>* dv[] = {&P.decay, &P.bco, &P.g1, &P.mix, &P.c, &P.dd, &P.p0, &P.p1, &P.p2, &P.g2};
    for (int i = 0; i < 10; i++) dv[i]->assign(vecs + (size_t)i * d, vecs + (size_t)(i + 1) * d);
    const double* fv = vecs + (size_t)10 * d;
    for (int i = 0; i < 4; i++) P.q[i].assign(fv + (size_t)i * dff, fv + (size_t)(i + 1) * dff);
    for (int i = 0; i < 3; i++) P.r[i].assign(fv + (size_t)(4 + i) * dff, fv + (size_t)(5 + i) * dff);
    // seeds: tm (a, b, iters), cm (a, b, iters), then the bootstrap gains
    // tm.x, tm.ms, u, s, g, cm.x, cm.ms, v, f
    P.tm = {seeds[0], seeds[1], (int)seeds[2], seeds[6], seeds[7], seeds[15]};
    P.cm = {seeds[3], seeds[4], (int)seeds[5], seeds[11], seeds[12], seeds[16]};
    P.g_u = seeds[8]; P.g_s = seeds[9]; P.g_g = seeds[10]; P.g_v = seeds[13]; P.g_f = seeds[14];
    P.g_z = seeds[17];
    P.ready = true;
}

}  // namespace fhe
