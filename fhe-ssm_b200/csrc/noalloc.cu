// noalloc.cu -- hybrid key switching that allocates no device memory.
//
// fhe_keyswitch_noalloc launches the same kernels, in the same order and on the same stream,
// as the allocating key switch in engine.cu (ModUp, key inner product, ModDown), so its output
// is bit-identical to fhe_keyswitch_host for the same input and key.  Only the working buffers
// differ: they live in one file-scope __device__ array that is reserved when the module loads
// on a device, and the ModUp base-conversion table (which the allocating path caches in
// cudaMalloc'd memory per limb count) is rebuilt on the host per call and passed to the
// device as a kernel parameter.
//
// Who cannot allocate, and why: a serving process that has handed nearly all of a GPU's HBM
// to long-lived arenas (the carried recurrent state of every resident conversation, the
// rotation keys, the plaintext cache) must not have a key switch fail with out-of-memory or
// stall in the allocator halfway through a pass; and a host runtime that owns device memory
// through its own pool (a Go or C++ server binding this library) may forbid any other code
// from calling cudaMalloc / cudaMallocAsync on its devices.  Such callers pass device
// buffers they own for the input and the outputs, and this entry point takes nothing else.
//
// Limits and hazards:
//  * kNoAllocScratchBytes (64 MiB) bounds the working set: at N = 2^16 (K = 4, alpha = 4) a
//    key switch of at most 16 limbs fits; larger requests are refused with FHE_ERR_ARG.
//  * the scratch is one array per device, shared by every context on that device: calls
//    that overlap in time (different contexts' streams, or different host threads) race on
//    it.  Calls through one context are ordered by that context's stream and do not.
//  * the first call on a device does the set-up (cudaGetSymbolAddress, which may load the
//    module on that device); make it before any stream capture on that device.  A set-up
//    that fails is reported and retried by the next call; it does not disable the entry point.
//  * per-kernel profiling (fhe_prof_enable) creates CUDA events, so it must be off.
//  * no word of the scratch is read before this call writes it (the table is copied in
//    first, ModUp writes every extended limb, the inner product and ModDown write every word
//    they later read), so nothing in it has to start at zero and nothing is cleared.

#include <cstdio>
#include <mutex>

namespace fhe {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;
constexpr int kNoAllocTabWords = 3584;     // 28 KiB: fits the 32 KiB kernel-parameter limit
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) uint64_t g_noalloc_scratch[kNoAllocScratchBytes / 8];

struct NoAllocTab {
    uint64_t w[kNoAllocTabWords];
};

// copies the by-value ModUp table into the scratch (the only host-to-device transfer)
__global__ void k_noalloc_tab(const NoAllocTab t, uint64_t* __restrict__ dst, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) dst[i] = t.w[i];
}

static std::mutex g_noalloc_mu;
static uint64_t* g_noalloc_ptr[kNoAllocMaxDevices];

// Device address of the scratch on `dev`, which the caller has made current.  Looked up on the
// first call that succeeds on a device and kept; a failed lookup (for example one made during a
// stream capture) is not remembered: its error is cleared from the runtime's sticky last-error
// slot and reported, and the next call tries again.
static uint64_t* noalloc_scratch(int dev) {
    if (dev < 0 || dev >= kNoAllocMaxDevices) throw Error("fhe_keyswitch_noalloc: device index out of range", -1);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            cudaGetLastError();
            throw Error(std::string("fhe_keyswitch_noalloc: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e),
                        -3);
        }
        g_noalloc_ptr[dev] = static_cast<uint64_t*>(p);
    }
    return g_noalloc_ptr[dev];
}

// ModUp table words for nl limbs (same layout as Context::modup_table)
static int noalloc_tab_words(const Context& cx, int nl) {
    const int dn = cx.dnum(nl), ne = nl + cx.K;
    return dn * cx.alpha * 2 + dn * ne * cx.alpha * 2;
}

// Scratch words for a key switch of nl limbs: region A holds d in coefficient form (nl
// limbs), then the inner product (2 x (nl+K)); region B holds the ModUp output (dnum x
// (nl+K)), then ModDown's converted P part (2 x nl); the table follows, 256-word aligned.
static size_t noalloc_words(const Context& cx, int nl) {
    const size_t N = cx.N, ne = nl + cx.K, dn = cx.dnum(nl);
    const size_t a = std::max<size_t>(nl, 2 * ne), b = std::max<size_t>(dn * ne, 2 * (size_t)nl);
    const size_t t = ((size_t)noalloc_tab_words(cx, nl) + 255) / 256 * 256;
    return (a + b) * N + t;
}

static bool noalloc_fits(const Context& cx, int nl) {
    return noalloc_tab_words(cx, nl) <= kNoAllocTabWords && noalloc_words(cx, nl) * 8 <= kNoAllocScratchBytes;
}

static void keyswitch_noalloc(Context& cx, const uint64_t* d, int nl, const SwitchKey& key, uint64_t* out0,
                              uint64_t* out1, uint64_t* scratch) {
    const int N = cx.N, K = cx.K, L = cx.L, ne = nl + K, dn = cx.dnum(nl), alpha = cx.alpha;
    cudaStream_t st = cx.stream;
    uint64_t* A = scratch;
    uint64_t* B = A + (size_t)std::max(nl, 2 * ne) * N;
    uint64_t* T = B + (size_t)std::max(dn * ne, 2 * nl) * N;

    // ModUp table (the layout of Context::modup_table): [dn][alpha] (Q_j/q_a)^-1 mod q_a with its
    // Shoup companion, then [dn][ne][alpha] (Q_j/q_a) mod m(e) with its Montgomery form
    NoAllocTab tab;
    const int tw = noalloc_tab_words(cx, nl);
    for (int i = 0; i < tw; i++) tab.w[i] = 0;
    for (int j = 0; j < dn; j++) {
        const int lo = j * alpha, sz = std::min(alpha, nl - lo);
        for (int a = 0; a < sz; a++) {
            const uint64_t qi = cx.mods[lo + a];
            uint64_t qh = 1;
            for (int b = 0; b < sz; b++) if (b != a) qh = host_mulmod(qh, cx.mods[lo + b] % qi, qi);
            const uint64_t inv = host_invmod(qh, qi);
            tab.w[(j * alpha + a) * 2] = inv;
            tab.w[(j * alpha + a) * 2 + 1] = shoup_of(inv, qi);
        }
        for (int e = 0; e < ne; e++) {
            if (e >= lo && e < lo + sz) continue;
            const uint64_t t = cx.mods[cx.ext_mod(nl, e)];
            for (int a = 0; a < sz; a++) {
                uint64_t v = 1;
                for (int b = 0; b < sz; b++) if (b != a) v = host_mulmod(v, cx.mods[lo + b] % t, t);
                const int o = dn * alpha * 2 + ((j * ne + e) * alpha + a) * 2;
                tab.w[o] = v;
                tab.w[o + 1] = mont_of(v, t);
            }
        }
    }
    k_noalloc_tab<<<(tw + 255) / 256, 256, 0, st>>>(tab, T, tw);

    // ModUp (engine.cu modup): d -> coefficient form in A, base-convert each digit into B
    CUDA_CHECK(cudaMemcpyAsync(A, d, (size_t)nl * N * 8, cudaMemcpyDeviceToDevice, st));
    ntt(cx, cx.qmap(A, nl, (long long)nl * N), 1, true, st);
    k_modup_bconv<<<g2(cx, dn), 256, 0, st>>>(A, d, B, T, nl, ne, alpha, L, cx.logN, 0, 0, 0);
    LimbMap em = cx.extmap(B, nl, (long long)ne * N);
    em.skip_alpha = alpha;
    ntt(cx, em, dn, false, st);

    // key inner product (engine.cu inner_moddown) into A; the coefficient copy of d is dead
    k_key_inner<<<g2(cx, ne), 256, 0, st>>>(B, key.buf.p, A, nl, ne, dn, L, K, cx.logN);

    // ModDown (engine.cu moddown) with the converted P part in B; the ModUp output is dead
    LimbMap pm{};
    pm.base = A + (size_t)nl * N; pm.poly_stride = (long long)ne * N; pm.nl = K;
    pm.split = 0; pm.off0 = 0; pm.off1 = L;
    ntt(cx, pm, 2, true, st);
    k_moddown_bconv<<<g2(cx, 2), 256, 0, st>>>(A, B, cx.d_md, nl, ne, L, K, cx.logN, 0, 0);
    ntt(cx, cx.qmap(B, nl, (long long)nl * N), 2, false, st);
    k_moddown_final<<<g2(cx, nl, 2), 256, 0, st>>>(A, B, nullptr, nullptr, out0, out1, cx.d_md, nl, ne, L, K,
                                                   cx.logN, 1);
    CUDA_CHECK(cudaGetLastError());
    cx.launches += 5;
    cx.ks_count++;
    cx.ks_limbs += nl;
}

}  // namespace fhe

// A device pointer of this context's device (plain device memory or managed memory).
static void require_device_ptr(const fhe::Context& c, const void* p, const char* what) {
    cudaPointerAttributes at{};
    const cudaError_t e = cudaPointerGetAttributes(&at, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        throw fhe::Error(std::string("fhe_keyswitch_noalloc: cannot query ") + what, FHE_ERR_ARG);
    }
    const bool dev = at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
    if (!dev || at.device != c.device)
        throw fhe::Error(std::string("fhe_keyswitch_noalloc: ") + what + " is not device memory of the context's GPU",
                         FHE_ERR_ARG);
    if (reinterpret_cast<uintptr_t>(p) % 8 != 0)
        throw fhe::Error(std::string("fhe_keyswitch_noalloc: ") + what + " is not 8-byte aligned", FHE_ERR_ARG);
}

extern "C" int fhe_keyswitch_noalloc(fhe_ctx* cx, uint64_t which, const uint64_t* d, int level, uint64_t* out0,
                                     uint64_t* out1) {
    return guard([&] {
        REQUIRE(cx && d && out0 && out1, "null argument");
        auto& c = cx->cx;
        REQUIRE(!c.prof, "fhe_keyswitch_noalloc: per-kernel profiling is on (it creates CUDA events); turn it off");
        bind(cx);
        const int nl = nl_of(c, level);
        fhe::SwitchKey* key = find_key(c, which);
        if (!fhe::noalloc_fits(c, nl)) {
            int most = 0;
            for (int n = 1; n <= c.L; n++) if (fhe::noalloc_fits(c, n)) most = n;
            char msg[256];
            std::snprintf(msg, sizeof msg,
                          "fhe_keyswitch_noalloc: %d limbs need %.1f MiB of scratch; the static scratch holds "
                          "%zu MiB (at most %d limbs in this context)",
                          nl, fhe::noalloc_words(c, nl) * 8.0 / (1 << 20), fhe::kNoAllocScratchBytes >> 20, most);
            throw fhe::Error(msg, FHE_ERR_ARG);
        }
        require_device_ptr(c, d, "d");
        require_device_ptr(c, out0, "out0");
        require_device_ptr(c, out1, "out1");
        uint64_t* s = fhe::noalloc_scratch(c.device);
        fhe::keyswitch_noalloc(c, d, nl, *key, out0, out1, s);
    });
}
