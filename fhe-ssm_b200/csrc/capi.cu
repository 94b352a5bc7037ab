// capi.cu -- the extern "C" surface declared in include/fhessm.h.
//
// Every entry point catches the engine's exceptions and turns them into a status code plus
// a thread-local message; no C++ exception crosses the boundary.
#include <cmath>
#include <cstring>
#include <string>

#include "../../include/fhessm.h"
#include "engine.h"

struct fhe_ctx {
    fhe::Context cx;
    explicit fhe_ctx(const fhe::Params& p) : cx(p) {}
};
struct fhe_ct {
    fhe::Ciphertext c;
    fhe_ctx* owner;
};
struct fhe_pt {
    fhe::Plaintext p;
    fhe_ctx* owner;
};

static thread_local std::string g_err;

template <class F>
static int guard(F&& f) {
    try {
        f();
        return FHE_OK;
    } catch (const fhe::Error& e) {
        g_err = e.what();
        return e.code < 0 ? e.code : FHE_ERR_ARG;
    } catch (const std::exception& e) {
        g_err = e.what();
        return FHE_ERR_ARG;
    }
}

#define REQUIRE(cond, msg) \
    do {                   \
        if (!(cond)) throw fhe::Error(msg, FHE_ERR_ARG); \
    } while (0)

static int nl_of(const fhe::Context& cx, int level) {
    if (level < 0 || level >= cx.L) throw fhe::Error("level out of range", FHE_ERR_ARG);
    return cx.L - level;
}
static void bind(fhe_ctx* c) {
    CUDA_CHECK(cudaSetDevice(c->cx.device));
    c->cx.activate();
}

static fhe_ct* wrap(fhe_ctx* c, fhe::Ciphertext&& x) {
    auto* r = new fhe_ct{std::move(x), c};
    return r;
}

extern "C" {

const char* fhe_last_error(void) { return g_err.c_str(); }

int fhe_ctx_create(const fhe_params* p, fhe_ctx** out) {
    return guard([&] {
        REQUIRE(p && out, "null argument");
        fhe::Params q;
        q.logN = p->logN; q.L = p->L; q.K = p->K; q.alpha = p->alpha;
        q.q0bits = p->q0bits; q.qbits = p->qbits; q.pbits = p->pbits;
        q.hw = p->hw; q.sigma = p->sigma; q.device = p->device;
        q.boot_primes = p->boot_primes; q.boot_bits = p->boot_bits > 0 ? p->boot_bits : 58;
        *out = new fhe_ctx(q);
    });
}
void fhe_ctx_destroy(fhe_ctx* cx) {
    if (!cx) return;
    try { delete cx; } catch (...) {}
}
int fhe_ctx_moduli(const fhe_ctx* cx, uint64_t* out) {
    return guard([&] {
        REQUIRE(cx && out, "null argument");
        std::memcpy(out, cx->cx.mods.data(), cx->cx.mods.size() * 8);
    });
}
double fhe_ctx_scale(const fhe_ctx* cx, int level) {
    if (!cx || level < 0 || level >= cx->cx.L) return 0.0;
    return cx->cx.scale_at[cx->cx.L - level];
}
int fhe_ctx_sync(fhe_ctx* cx) {
    return guard([&] {
        REQUIRE(cx, "null argument");
        bind(cx);
        CUDA_CHECK(cudaStreamSynchronize(cx->cx.stream));
        cx->cx.check_device_error();
    });
}
int fhe_ctx_set_option(fhe_ctx* cx, const char* name, int value) {
    return guard([&] {
        REQUIRE(cx && name, "null argument");
        if (std::strcmp(name, "matvec_tensor_cores") == 0) cx->cx.use_tc = value != 0;
        else if (std::strcmp(name, "merged_rescale") == 0) cx->cx.merged_rescale = value != 0;
        else if (std::strcmp(name, "pdl") == 0) cx->cx.use_pdl = value != 0;
        else if (std::strcmp(name, "ntt_cluster") == 0) cx->cx.ntt_cluster = value != 0;
        else if (std::strcmp(name, "ntt_arith") == 0) cx->cx.ntt_arith = value == 1 ? 1 : 0;
        else if (std::strcmp(name, "baby_limbs") == 0) cx->cx.baby_limbs = value < 1 ? 1 : value > 64 ? 64 : value;
        else if (std::strcmp(name, "boot_compress") == 0) cx->cx.boot_compress = value != 0;
        else if (std::strcmp(name, "boot_delta_log2") == 0) {
            if (value != 0 && value != -1 && (value < 30 || value > 56))
                throw fhe::Error("boot_delta_log2: 0 (auto), -1 (canonical) or 30..56", -1);
            cx->cx.boot_delta_log2 = value;
        }
        else if (std::strcmp(name, "profile_every") == 0) cx->cx.prof_every = value < 1 ? 1 : value;
        else if (std::strcmp(name, "plaintext_cache") == 0) cx->cx.pt_cache = value != 0;
        else if (std::strcmp(name, "plaintext_cache_reserve_mib") == 0) cx->cx.pt_cache_reserve_mib = value < 0 ? 0 : value;
        else throw fhe::Error(std::string("unknown option ") + name, FHE_ERR_ARG);
    });
}
int fhe_ctx_memory(fhe_ctx* cx, long long* out) {
    return guard([&] {
        REQUIRE(cx && out, "null argument");
        bind(cx);
        size_t fr = 0, tot = 0;
        CUDA_CHECK(cudaMemGetInfo(&fr, &tot));
        cudaMemPool_t pool;
        CUDA_CHECK(cudaDeviceGetDefaultMemPool(&pool, cx->cx.prm.device));
        uint64_t res = 0, used = 0;
        CUDA_CHECK(cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReservedMemCurrent, &res));
        CUDA_CHECK(cudaMemPoolGetAttribute(pool, cudaMemPoolAttrUsedMemCurrent, &used));
        out[0] = (long long)fr;
        out[1] = (long long)tot;
        out[2] = (long long)res;
        out[3] = (long long)used;
        out[4] = cx->cx.pt_cache_bytes;
    });
}
long long fhe_ctx_launches(const fhe_ctx* cx) { return cx ? cx->cx.launches : 0; }
void* fhe_ctx_stream(const fhe_ctx* cx) { return cx ? (void*)cx->cx.stream : nullptr; }
int fhe_ctx_counters(const fhe_ctx* cx, long long* keyswitches, long long* ks_limbs) {
    return guard([&] {
        REQUIRE(cx, "null argument");
        if (keyswitches) *keyswitches = cx->cx.ks_count;
        if (ks_limbs) *ks_limbs = cx->cx.ks_limbs;
    });
}
int fhe_ctx_stat(const fhe_ctx* cx, const char* name, long long* value) {
    return guard([&] {
        REQUIRE(cx && name && value, "null argument");
        const fhe::Context& c = cx->cx;
        if (std::strcmp(name, "launches") == 0) *value = c.launches;
        else if (std::strcmp(name, "keyswitches") == 0) *value = c.ks_count;
        else if (std::strcmp(name, "ks_limbs") == 0) *value = c.ks_limbs;
        else if (std::strcmp(name, "pt_encodes") == 0) *value = c.pt_encodes;
        else if (std::strcmp(name, "pt_cached") == 0) *value = (long long)c.ptcache.size();
        else if (std::strcmp(name, "host_waits") == 0) *value = c.host_waits;
        else throw fhe::Error(std::string("unknown statistic: ") + name, -1);
    });
}
int fhe_prof_enable(fhe_ctx* cx, int on) {
    return guard([&] {
        REQUIRE(cx, "null argument");
        cx->cx.prof = on != 0;
    });
}
int fhe_prof_collect(fhe_ctx* cx, char* buf, int cap) {
    return guard([&] {
        REQUIRE(cx && buf && cap > 2, "null argument");
        bind(cx);
        auto& c = cx->cx;
        CUDA_CHECK(cudaStreamSynchronize(c.stream));
        std::string js = "{";
        bool first = true;
        for (auto& kv : c.prof_acc) {
            auto& e = kv.second;
            for (auto& pr : e.pending) {
                float ms = 0.f;
                CUDA_CHECK(cudaEventElapsedTime(&ms, pr.first, pr.second));
                e.ms += ms;
                cudaEventDestroy(pr.first);
                cudaEventDestroy(pr.second);
            }
            e.pending.clear();
            if (!first) js += ", ";
            first = false;
            const double ms = e.sampled ? e.ms * (double)e.seen / (double)e.sampled : 0.0;
            js += "\"" + kv.first + "\": [" + std::to_string(e.seen) + ", " + std::to_string(ms) + ", " +
                  std::to_string(e.bytes) + ", " + std::to_string(e.ops) + "]";
        }
        js += "}";
        c.prof_acc.clear();
        REQUIRE((int)js.size() < cap, "buffer too small");
        std::memcpy(buf, js.c_str(), js.size() + 1);
    });
}

int fhe_keygen(fhe_ctx* cx, const uint8_t seed[32]) {
    return guard([&] {
        REQUIRE(cx && seed, "null argument");
        bind(cx);
        fhe::keygen(cx->cx, seed);
    });
}
int fhe_keygen_rotations(fhe_ctx* cx, const int32_t* steps, int n, int conj) {
    return guard([&] {
        REQUIRE(cx && (steps || n == 0), "null argument");
        bind(cx);
        std::vector<int> v(steps, steps + n);
        fhe::keygen_rotations(cx->cx, v.data(), n, conj != 0);
    });
}
int fhe_keygen_auto(fhe_ctx* cx, const uint64_t* idx, int n) {
    return guard([&] {
        REQUIRE(cx && (idx || n == 0), "null argument");
        bind(cx);
        fhe::keygen_auto(cx->cx, idx, n);
    });
}
static fhe::SwitchKey* find_key(fhe::Context& c, uint64_t which) {
    if (which == 0) {
        if (!c.rlk) throw fhe::Error("no relinearisation key", FHE_ERR_KEY);
        return c.rlk.get();
    }
    auto it = c.rot_keys.find(which);
    if (it == c.rot_keys.end()) throw fhe::Error("no key for automorphism " + std::to_string(which), FHE_ERR_KEY);
    return it->second.get();
}
int fhe_key_export(fhe_ctx* cx, uint64_t which, uint64_t* words) {
    return guard([&] {
        REQUIRE(cx && words, "null argument");
        bind(cx);
        auto& c = cx->cx;
        fhe::SwitchKey* k = find_key(c, which);
        fhe::DevBuf t(k->buf.words, c.stream);
        CUDA_CHECK(cudaMemcpyAsync(t.p, k->buf.p, k->buf.words * 8, cudaMemcpyDeviceToDevice, c.stream));
        fhe::key_to_mont(c, t.p, false);
        fhe::download(c, words, t.p, t.words);
    });
}
int fhe_key_import(fhe_ctx* cx, uint64_t which, const uint64_t* words) {
    return guard([&] {
        REQUIRE(cx && words, "null argument");
        bind(cx);
        auto& c = cx->cx;
        auto key = std::make_unique<fhe::SwitchKey>();
        const size_t w = (size_t)c.dnum_top * 2 * (c.L + c.K) * c.N;
        key->buf = fhe::DevBuf(w, c.stream);
        key->index = which;
        fhe::upload(c, key->buf.p, words, w);
        fhe::key_to_mont(c, key->buf.p, true);
        if (which == 0) c.rlk = std::move(key);
        else c.rot_keys[which] = std::move(key);
    });
}
int fhe_secret_export(fhe_ctx* cx, int8_t* coeffs) {
    return guard([&] {
        REQUIRE(cx && coeffs, "null argument");
        REQUIRE(!cx->cx.sk_coeff.empty(), "no secret key");
        std::memcpy(coeffs, cx->cx.sk_coeff.data(), cx->cx.sk_coeff.size());
    });
}
int fhe_pubkey_export(fhe_ctx* cx, uint64_t* words) {
    return guard([&] {
        REQUIRE(cx && words, "null argument");
        REQUIRE(cx->cx.pk.p, "no public key");
        bind(cx);
        fhe::download(cx->cx, words, cx->cx.pk.p, cx->cx.pk.words);
    });
}
uint64_t fhe_rot_index(const fhe_ctx* cx, int32_t step) { return cx ? fhe::rot_index(cx->cx, step) : 0; }

int fhe_encode(fhe_ctx* cx, const double* re, const double* im, int n, int level, double scale, fhe_pt** out) {
    return guard([&] {
        REQUIRE(cx && re && out && n > 0, "null argument");
        bind(cx);
        auto& c = cx->cx;
        const int nl = nl_of(c, level);
        std::vector<std::complex<double>> z(n);
        for (int i = 0; i < n; i++) z[i] = std::complex<double>(re[i], im ? im[i] : 0.0);
        const double sc = scale > 0 ? scale : c.scale_at[nl];
        *out = new fhe_pt{fhe::encode(c, z.data(), n, nl, sc), cx};
    });
}
int fhe_encode_periodic(fhe_ctx* cx, const double* re, const double* im, int period, int count, int level,
                        double scale, uint64_t* words) {
    return guard([&] {
        REQUIRE(cx && re && words && period > 0 && count > 0, "bad argument");
        bind(cx);
        auto& c = cx->cx;
        const int nl = nl_of(c, level);
        std::vector<std::complex<double>> z((size_t)period * count);
        for (size_t i = 0; i < z.size(); i++) z[i] = std::complex<double>(re[i], im ? im[i] : 0.0);
        fhe::encode_periodic_words(c, z.data(), period, count, nl, scale > 0 ? scale : c.scale_at[nl], words);
    });
}
int fhe_decode(fhe_ctx* cx, const fhe_pt* pt, double* re, double* im) {
    return guard([&] {
        REQUIRE(cx && pt && re, "null argument");
        bind(cx);
        auto& c = cx->cx;
        std::vector<std::complex<double>> z(c.N / 2);
        fhe::decode(c, pt->p, z.data());
        for (int i = 0; i < c.N / 2; i++) {
            re[i] = z[i].real();
            if (im) im[i] = z[i].imag();
        }
    });
}
void fhe_pt_free(fhe_pt* pt) { delete pt; }
int fhe_pt_level(const fhe_pt* pt) { return pt ? pt->owner->cx.L - pt->p.nl : -1; }

int fhe_encrypt(fhe_ctx* cx, const fhe_pt* pt, fhe_ct** out) {
    return guard([&] {
        REQUIRE(cx && pt && out, "null argument");
        bind(cx);
        *out = wrap(cx, fhe::encrypt(cx->cx, pt->p));
    });
}
int fhe_decrypt(fhe_ctx* cx, const fhe_ct* ct, fhe_pt** out) {
    return guard([&] {
        REQUIRE(cx && ct && out, "null argument");
        bind(cx);
        *out = new fhe_pt{fhe::decrypt(cx->cx, ct->c), cx};
    });
}
void fhe_ct_free(fhe_ct* ct) { delete ct; }
int fhe_ct_level(const fhe_ct* ct) { return ct ? ct->owner->cx.L - ct->c.nl : -1; }
double fhe_ct_scale(const fhe_ct* ct) { return ct ? ct->c.scale : 0.0; }
int fhe_ct_copy(fhe_ctx* cx, const fhe_ct* a, fhe_ct** out) {
    return guard([&] {
        REQUIRE(cx && a && out, "null argument");
        bind(cx);
        *out = wrap(cx, fhe::ct_copy(cx->cx, a->c));
    });
}

#define BINOP(name, fn)                                                     \
    int name(fhe_ctx* cx, const fhe_ct* a, const fhe_ct* b, fhe_ct** out) { \
        return guard([&] {                                                  \
            REQUIRE(cx && a && b && out, "null argument");                  \
            bind(cx);                                                       \
            fhe::Ciphertext r;                                              \
            fn(cx->cx, a->c, b->c, r);                                      \
            *out = wrap(cx, std::move(r));                                  \
        });                                                                 \
    }
BINOP(fhe_add, fhe::add_any)
BINOP(fhe_sub, fhe::sub_any)
BINOP(fhe_mul_ct_ct_relin, fhe::ct_mul_relin)

int fhe_mul_ct_pt(fhe_ctx* cx, const fhe_ct* a, const fhe_pt* pt, fhe_ct** out) {
    return guard([&] {
        REQUIRE(cx && a && pt && out, "null argument");
        bind(cx);
        fhe::Ciphertext r;
        fhe::ct_mul_pt(cx->cx, a->c, pt->p, r);
        *out = wrap(cx, std::move(r));
    });
}
int fhe_add_pt(fhe_ctx* cx, const fhe_ct* a, const fhe_pt* pt, fhe_ct** out) {
    return guard([&] {
        REQUIRE(cx && a && pt && out, "null argument");
        bind(cx);
        fhe::Ciphertext r;
        fhe::ct_add_pt(cx->cx, a->c, pt->p, r);
        *out = wrap(cx, std::move(r));
    });
}
int fhe_mul_const(fhe_ctx* cx, const fhe_ct* a, double v, double scale, fhe_ct** out) {
    return guard([&] {
        REQUIRE(cx && a && out, "null argument");
        bind(cx);
        fhe::Ciphertext r;
        const double sc = scale > 0 ? scale : cx->cx.scale_at[a->c.nl];
        fhe::ct_mul_const(cx->cx, a->c, v, sc, r);
        *out = wrap(cx, std::move(r));
    });
}
int fhe_add_const(fhe_ctx* cx, const fhe_ct* a, double v, fhe_ct** out) {
    return guard([&] {
        REQUIRE(cx && a && out, "null argument");
        bind(cx);
        fhe::Ciphertext r;
        fhe::ct_add_const(cx->cx, a->c, v, r);
        *out = wrap(cx, std::move(r));
    });
}
int fhe_rescale(fhe_ctx* cx, fhe_ct* ct) {
    return guard([&] {
        REQUIRE(cx && ct, "null argument");
        bind(cx);
        fhe::ct_rescale(cx->cx, ct->c);
    });
}
int fhe_level_reduce(fhe_ctx* cx, fhe_ct* ct, int levels) {
    return guard([&] {
        REQUIRE(cx && ct && levels >= 0, "bad argument");
        bind(cx);
        fhe::ct_level_drop(cx->cx, ct->c, ct->c.nl - levels);
    });
}
int fhe_rotate(fhe_ctx* cx, const fhe_ct* a, int32_t k, fhe_ct** out) {
    return guard([&] {
        REQUIRE(cx && a && out, "null argument");
        bind(cx);
        fhe::Ciphertext r;
        fhe::ct_rotate(cx->cx, a->c, k, r);
        *out = wrap(cx, std::move(r));
    });
}
int fhe_rotate_hoisted(fhe_ctx* cx, const fhe_ct* a, const int32_t* ks, int n, fhe_ct** outs) {
    return guard([&] {
        REQUIRE(cx && a && ks && outs && n > 0, "null argument");
        bind(cx);
        std::vector<fhe::Ciphertext> r(n);
        std::vector<int> v(ks, ks + n);
        fhe::ct_rotate_hoisted(cx->cx, a->c, v.data(), n, r.data());
        for (int i = 0; i < n; i++) outs[i] = wrap(cx, std::move(r[i]));
    });
}
int fhe_rotate_sum(fhe_ctx* cx, const fhe_ct* const* in, const int32_t* ks, int n, fhe_ct** out) {
    return guard([&] {
        REQUIRE(cx && in && ks && out && n > 0, "null argument");
        bind(cx);
        auto& c = cx->cx;
        const int nl = in[0]->c.nl;
        const double sc = in[0]->c.scale;
        std::vector<const uint64_t*> c0s, c1s;
        std::vector<int> steps;
        const fhe::Ciphertext* extra = nullptr;
        for (int i = 0; i < n; i++) {
            REQUIRE(in[i], "null argument");
            if (in[i]->c.nl != nl || std::fabs(in[i]->c.scale / sc - 1) > 1e-9)
                throw fhe::Error("rotate_sum: inputs differ in level or scale", FHE_ERR_LEVEL);
            if (fhe::rot_index(c, ks[i]) == 1) {
                REQUIRE(!extra, "rotate_sum: at most one zero rotation");
                extra = &in[i]->c;
                continue;
            }
            c0s.push_back(in[i]->c.c(0));
            c1s.push_back(in[i]->c.c(1));
            steps.push_back(ks[i]);
        }
        fhe::Ciphertext r;
        fhe::rotate_sum(c, c0s.data(), c1s.data(), steps.data(), (int)steps.size(), nl, sc,
                        extra ? extra->c(0) : nullptr, extra ? extra->c(1) : nullptr, r);
        *out = wrap(cx, std::move(r));
    });
}
int fhe_conjugate(fhe_ctx* cx, const fhe_ct* a, fhe_ct** out) {
    return guard([&] {
        REQUIRE(cx && a && out, "null argument");
        bind(cx);
        fhe::Ciphertext r;
        fhe::ct_conjugate(cx->cx, a->c, r);
        *out = wrap(cx, std::move(r));
    });
}

int fhe_mul_vec_rescale(fhe_ctx* cx, const fhe_ct* a, const double* re, const double* im, int n, fhe_ct** out) {
    return guard([&] {
        REQUIRE(cx && a && re && out && n > 0, "null argument");
        bind(cx);
        std::vector<std::complex<double>> v(n);
        for (int i = 0; i < n; i++) v[i] = std::complex<double>(re[i], im ? im[i] : 0.0);
        fhe::Ciphertext r;
        fhe::mul_vec_rescale(cx->cx, a->c, v.data(), n, r, 0);
        *out = wrap(cx, std::move(r));
    });
}
int fhe_align(fhe_ctx* cx, fhe_ct* ct, int level) {
    return guard([&] {
        REQUIRE(cx && ct, "null argument");
        bind(cx);
        fhe::align(cx->cx, ct->c, nl_of(cx->cx, level), 0);
    });
}
int fhe_mul_rescale(fhe_ctx* cx, const fhe_ct* a, const fhe_ct* b, fhe_ct** out) {
    return guard([&] {
        REQUIRE(cx && a && b && out, "null argument");
        bind(cx);
        fhe::Ciphertext r;
        fhe::mul_rescale(cx->cx, a->c, b->c, r);
        *out = wrap(cx, std::move(r));
    });
}
int fhe_poly_eval(fhe_ctx* cx, const fhe_ct* x, const double* coeffs, int deg, int n, fhe_ct** out) {
    return guard([&] {
        REQUIRE(cx && x && coeffs && out && deg >= 1 && n > 0, "bad argument");
        bind(cx);
        std::vector<std::vector<std::complex<double>>> c(deg + 1, std::vector<std::complex<double>>(n));
        for (int i = 0; i <= deg; i++)
            for (int k = 0; k < n; k++) c[i][k] = coeffs[(size_t)i * n + k];
        fhe::Ciphertext r;
        fhe::poly_eval_vec(cx->cx, x->c, c, n, r);
        *out = wrap(cx, std::move(r));
    });
}
int fhe_cheb_eval(fhe_ctx* cx, const fhe_ct* x, const double* coeffs, int ncoef, fhe_ct** out) {
    return guard([&] {
        REQUIRE(cx && x && coeffs && out && ncoef >= 2, "bad argument");
        bind(cx);
        std::vector<double> c(coeffs, coeffs + ncoef);
        fhe::Ciphertext r;
        fhe::cheb_eval(cx->cx, x->c, c, r);
        *out = wrap(cx, std::move(r));
    });
}
int fhe_cheb_depth(const double* coeffs, int ncoef, int* depth) {
    return guard([&] {
        REQUIRE(coeffs && depth && ncoef >= 2, "bad argument");
        *depth = fhe::cheb_depth(std::vector<double>(coeffs, coeffs + ncoef));
    });
}
int fhe_cheb_eval_n(fhe_ctx* cx, const fhe_ct* const* xs, int count, const double* coeffs, int ncoef,
                    fhe_ct** outs) {
    return guard([&] {
        REQUIRE(cx && xs && coeffs && outs && ncoef >= 2 && count >= 1 && count <= 64, "bad argument");
        bind(cx);
        std::vector<const fhe::Ciphertext*> in(count);
        for (int k = 0; k < count; k++) {
            REQUIRE(xs[k], "null ciphertext");
            REQUIRE(xs[k]->c.nl == xs[0]->c.nl && xs[k]->c.scale == xs[0]->c.scale,
                    "batched Chebyshev series: the inputs must share level and scale");
            in[k] = &xs[k]->c;
        }
        std::vector<double> c(coeffs, coeffs + ncoef);
        std::vector<fhe::Ciphertext> r(count);
        fhe::cheb_eval_n(cx->cx, in.data(), count, c, r.data());
        for (int k = 0; k < count; k++) outs[k] = wrap(cx, std::move(r[k]));
    });
}
int fhe_bootstrap_setup(fhe_ctx* cx, double bound, int degree) {
    return guard([&] {
        REQUIRE(cx && bound > 0 && degree >= 3, "bad argument");
        bind(cx);
        std::vector<int> rots = fhe::boot_rotations(cx->cx);
        fhe::keygen_rotations(cx->cx, rots.data(), (int)rots.size(), true);
        fhe::bootstrap_setup(cx->cx, bound, degree);
    });
}

int fhe_bootstrap_setup_r(fhe_ctx* cx, double bound, int degree, int double_angles) {
    return guard([&] {
        REQUIRE(cx && bound > 0 && degree >= 3, "bad argument");
        bind(cx);
        std::vector<int> rots = fhe::boot_rotations(cx->cx);
        fhe::keygen_rotations(cx->cx, rots.data(), (int)rots.size(), true);
        fhe::bootstrap_setup(cx->cx, bound, degree, double_angles);
    });
}
int fhe_bootstrap(fhe_ctx* cx, const fhe_ct* a, fhe_ct** out) {
    return guard([&] {
        REQUIRE(cx && a && out, "null argument");
        bind(cx);
        fhe::Ciphertext r;
        fhe::bootstrap(cx->cx, a->c, r);
        *out = wrap(cx, std::move(r));
    });
}
int fhe_bootstrap_n(fhe_ctx* cx, const fhe_ct* const* in, int n, fhe_ct** out) {
    return guard([&] {
        REQUIRE(cx && in && out && n > 0, "null argument");
        for (int i = 0; i < n; i++) REQUIRE(in[i], "null ciphertext");
        bind(cx);
        std::vector<fhe::Ciphertext> r((size_t)n);
        for (int i = 0; i < n; i++) fhe::bootstrap(cx->cx, in[i]->c, r[i]);
        for (int i = 0; i < n; i++) out[i] = wrap(cx, std::move(r[i]));
    });
}
int fhe_bootstrap_stage(fhe_ctx* cx, const fhe_ct* a, int upto, fhe_ct** out) {
    return guard([&] {
        REQUIRE(cx && a && out && upto >= 1 && upto <= 4, "bad argument");
        bind(cx);
        fhe::Ciphertext r;
        fhe::bootstrap_upto(cx->cx, a->c, r, upto);
        *out = wrap(cx, std::move(r));
    });
}
int fhe_bootstrap_level(const fhe_ctx* cx) {
    if (!cx) return -1;
    const int nl = fhe::bootstrap_levels_after(cx->cx);
    return nl ? cx->cx.L - nl : -1;
}

struct fhe_mvplan {
    std::shared_ptr<fhe::MatvecPlan> p;
};
int fhe_matvec_plan(fhe_ctx* cx, const double* W, int rows, int cols, int D, int b1, fhe_mvplan** out) {
    return guard([&] {
        REQUIRE(cx && W && out && rows > 0 && cols > 0, "bad argument");
        bind(cx);
        *out = new fhe_mvplan{fhe::matvec_plan(cx->cx, W, rows, cols, D, b1)};
    });
}
void fhe_mvplan_free(fhe_mvplan* pl) { delete pl; }
int fhe_matvec_keygen(fhe_ctx* cx, int D, int b1) {
    return guard([&] {
        REQUIRE(cx && D > 0 && b1 > 0, "bad argument");
        bind(cx);
        std::vector<int> r = fhe::matvec_rotations(D, b1);
        fhe::keygen_rotations(cx->cx, r.data(), (int)r.size(), false);
    });
}
int fhe_matvec_bsgs(fhe_ctx* cx, const fhe_mvplan* pl, const fhe_ct* const* in, int nin, fhe_ct** out) {
    return guard([&] {
        REQUIRE(cx && pl && in && out && nin > 0, "null argument");
        bind(cx);
        std::vector<const fhe::Ciphertext*> us(nin);
        for (int i = 0; i < nin; i++) us[i] = &in[i]->c;
        fhe::Ciphertext r;
        fhe::matvec(cx->cx, *pl->p, us.data(), r);
        *out = wrap(cx, std::move(r));
    });
}

struct fhe_model {
    std::shared_ptr<fhe::Model> m;
    fhe_ctx* owner;
};
int fhe_model_create(fhe_ctx* cx, const fhe_model_cfg* c, fhe_model** out) {
    return guard([&] {
        REQUIRE(cx && c && out, "null argument");
        bind(cx);
        fhe::ModelCfg mc;
        mc.d = c->d; mc.dff = c->dff; mc.n_layer = c->n_layer; mc.D = c->D; mc.b1 = c->b1;
        mc.a_min = c->a_min; mc.a_max = c->a_max; mc.alpha = c->alpha; mc.eps = c->eps;
        mc.shift_mix = c->shift_mix != 0;
        *out = new fhe_model{fhe::model_create(cx->cx, mc), cx};
    });
}
void fhe_model_free(fhe_model* m) { delete m; }
int fhe_model_set_layer(fhe_model* m, int layer, const double* win, const double* wout, const double* wk,
                        const double* wr, const double* wv, const double* vecs, const double* seeds) {
    return guard([&] {
        REQUIRE(m && win && wout && wk && wr && wv && vecs && seeds, "null argument");
        bind(m->owner);
        fhe::model_set_layer(*m->m, layer, win, wout, wk, wr, wv, vecs, seeds);
    });
}
int fhe_model_set_output(fhe_model* m, const double* g_out, const double* seed3) {
    return guard([&] {
        REQUIRE(m && g_out && seed3, "null argument");
        m->m->g_out.assign(g_out, g_out + m->m->cfg.d);
        m->m->out_seed = {seed3[0], seed3[1], (int)seed3[2], seed3[3], seed3[4], seed3[5]};
    });
}
int fhe_model_keygen(fhe_model* m) {
    return guard([&] {
        REQUIRE(m, "null argument");
        bind(m->owner);
        std::vector<int> r = fhe::model_rotation_steps(m->m->cfg);
        fhe::keygen_rotations(m->owner->cx, r.data(), (int)r.size(), true);
    });
}
int fhe_model_reset(fhe_model* m) {
    return guard([&] {
        REQUIRE(m, "null argument");
        m->m->have_state = false;
        m->m->s.clear();
        m->m->up.clear();
    });
}
int fhe_model_step(fhe_model* m, const fhe_ct* in, fhe_ct** out) {
    return guard([&] {
        REQUIRE(m && in && out, "null argument");
        bind(m->owner);
        *out = wrap(m->owner, m->m->step(in->c));
    });
}
int fhe_model_stats(const fhe_model* m, long long* bootstraps, long long* steps) {
    return guard([&] {
        REQUIRE(m, "null argument");
        if (bootstraps) *bootstraps = m->m->boots;
        if (steps) *steps = m->m->steps;
    });
}
int fhe_model_refresh_census(const fhe_model* m, long long* counts, int n) {
    return guard([&] {
        REQUIRE(m && counts && n >= 0, "null argument");
        for (int i = 0; i < n; i++) counts[i] = i < fhe::Model::kSites ? m->m->site_boots[i] : 0;
    });
}
int fhe_model_probe(fhe_model* m, int k) {
    return guard([&] {
        REQUIRE(m && k >= 0 && k % 100 <= 13, "bad argument");
        m->m->probe = k;
    });
}
int fhe_server_step(fhe_model* m, const fhe_ct* const* in, int n_in, fhe_ct** out, int* n_out, int flags) {
    return guard([&] {
        REQUIRE(m && in && out && n_out && n_in == 1, "one input pack per model (one ciphertext of 2N/2D lanes)");
        bind(m->owner);
        if (flags & 1) {
            m->m->have_state = false;
            m->m->s.clear();
            m->m->up.clear();
        }
        out[0] = wrap(m->owner, m->m->step(in[0]->c));
        *n_out = 1;
    });
}

int fhe_ct_import(fhe_ctx* cx, const uint64_t* words, int level, double scale, fhe_ct** out) {
    return guard([&] {
        REQUIRE(cx && words && out, "null argument");
        bind(cx);
        auto& c = cx->cx;
        const int nl = nl_of(c, level);
        fhe::Ciphertext r = fhe::ct_alloc(c, nl);
        r.scale = scale;
        fhe::upload(c, r.buf.p, words, (size_t)2 * nl * c.N);
        *out = wrap(cx, std::move(r));
    });
}
int fhe_ct_export(fhe_ctx* cx, const fhe_ct* ct, uint64_t* words) {
    return guard([&] {
        REQUIRE(cx && ct && words, "null argument");
        bind(cx);
        auto& c = cx->cx;
        const size_t w = (size_t)ct->c.nl * c.N;
        fhe::download(c, words, ct->c.c(0), w);
        fhe::download(c, words + w, ct->c.c(1), w);
    });
}
int fhe_pt_import(fhe_ctx* cx, const uint64_t* words, int level, double scale, fhe_pt** out) {
    return guard([&] {
        REQUIRE(cx && words && out, "null argument");
        bind(cx);
        auto& c = cx->cx;
        const int nl = nl_of(c, level);
        fhe::Plaintext p;
        p.buf = fhe::DevBuf((size_t)nl * c.N, c.stream);
        p.nl = nl;
        p.scale = scale;
        fhe::upload(c, p.buf.p, words, (size_t)nl * c.N);
        *out = new fhe_pt{std::move(p), cx};
    });
}
int fhe_pt_export(fhe_ctx* cx, const fhe_pt* pt, uint64_t* words) {
    return guard([&] {
        REQUIRE(cx && pt && words, "null argument");
        bind(cx);
        fhe::download(cx->cx, words, pt->p.buf.p, (size_t)pt->p.nl * (cx->cx.N >> pt->p.log_rep));
    });
}
int fhe_ntt_host(fhe_ctx* cx, uint64_t* words, int n, const int* mod_idx, int inverse) {
    return guard([&] {
        REQUIRE(cx && words && mod_idx && n > 0, "null argument");
        bind(cx);
        auto& c = cx->cx;
        for (int i = 0; i < n; i++) REQUIRE(mod_idx[i] >= 0 && mod_idx[i] < c.L + c.K, "modulus index out of range");
        fhe::DevBuf d((size_t)n * c.N, c.stream);
        fhe::upload(c, d.p, words, d.words);
        // a run of consecutive moduli, repeated back to back, is one batched transform
        for (int s = 0; s < n;) {
            int run = 1;
            while (s + run < n && mod_idx[s + run] == mod_idx[s] + run) run++;
            int reps = 1;
            while (s + (reps + 1) * run <= n && std::equal(mod_idx + s, mod_idx + s + run, mod_idx + s + reps * run))
                reps++;
            fhe::LimbMap mp{};
            mp.base = d.p + (size_t)s * c.N; mp.poly_stride = (long long)run * c.N; mp.nl = run;
            mp.split = run; mp.off0 = mod_idx[s]; mp.off1 = 0;
            fhe::ntt(c, mp, reps, inverse != 0, c.stream);
            s += run * reps;
        }
        fhe::download(c, words, d.p, d.words);
    });
}
int fhe_keyswitch_host(fhe_ctx* cx, const uint64_t* d, int level, const uint64_t* key, uint64_t* out0,
                       uint64_t* out1) {
    return guard([&] {
        REQUIRE(cx && d && key && out0 && out1, "null argument");
        bind(cx);
        auto& c = cx->cx;
        const int nl = nl_of(c, level);
        fhe::SwitchKey k;
        const size_t kw = (size_t)c.dnum_top * 2 * (c.L + c.K) * c.N;
        k.buf = fhe::DevBuf(kw, c.stream);
        fhe::upload(c, k.buf.p, key, kw);
        fhe::key_to_mont(c, k.buf.p, true);
        fhe::DevBuf dd((size_t)nl * c.N, c.stream), o((size_t)2 * nl * c.N, c.stream);
        fhe::upload(c, dd.p, d, dd.words);
        fhe::keyswitch(c, dd.p, nl, k, nullptr, nullptr, o.p, o.p + (size_t)nl * c.N, 1);
        fhe::download(c, out0, o.p, (size_t)nl * c.N);
        fhe::download(c, out1, o.p + (size_t)nl * c.N, (size_t)nl * c.N);
    });
}

}  // extern "C"
