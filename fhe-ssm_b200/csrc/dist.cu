// dist.cu -- limb-partitioned hybrid key switching over several GPUs (single-pack latency).
//
// The reference runs one context's RNS limbs on several GPUs (gpu_real_model.cu:847-884, the
// --devices flag; FIDESlib places limb i on device i mod G, :995-997, SetDevices :1158-1161).
// Here rank g of G owns a contiguous block of the Q limbs and of the K special limbs of every
// polynomial (limb_block: per = ceil(n / G) limbs, rank g the limbs [g per, (g + 1) per) that
// exist).  A key switch of d (the rank's Q limbs, eval form) is:
//   1. inverse NTT of the rank's limbs, ncclAllGather of them in coefficient form (every rank
//      then holds all of d in coefficient form: what each digit's base conversion reads);
//   2. ModUp to the rank's own extended limbs (its Q block, then its P block), NTT, and the key
//      inner product with the resident key on those limbs only;
//   3. inverse NTT of the rank's special limbs of both products, ncclAllGather of them;
//   4. ModDown on the rank's Q limbs: base conversion of the gathered P part, NTT, subtract,
//      multiply by P^-1.
// Every base conversion and reduction is the single-GPU kernel's formula with the same constant
// tables (Context::modup_table, d_md), so the ranks' limbs equal the single-GPU key switch word
// for word.  The collectives run on the context's own communication stream, ordered against
// the compute stream by events; remote limbs land in this GPU's memory before a kernel reads
// them (no kernel touches peer memory).  NCCL is loaded at run time (dlopen), so single-GPU use
// of the library needs no NCCL.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>

namespace fhe {

// ----------------------------------------------------------------------------- NCCL ----
struct NcclApi {
    ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*commInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*allGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*errorString)(ncclResult_t) = nullptr;
};
static const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    static std::string err;
    std::call_once(once, [] {
        // a libnccl already in the process (torch's) first, else the loader's search path
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) { err = dlerror() ? dlerror() : "dlopen failed"; return; }
        api.getUniqueId = (decltype(api.getUniqueId))dlsym(h, "ncclGetUniqueId");
        api.commInitRank = (decltype(api.commInitRank))dlsym(h, "ncclCommInitRank");
        api.commDestroy = (decltype(api.commDestroy))dlsym(h, "ncclCommDestroy");
        api.allGather = (decltype(api.allGather))dlsym(h, "ncclAllGather");
        api.errorString = (decltype(api.errorString))dlsym(h, "ncclGetErrorString");
    });
    if (!api.allGather || !api.commInitRank || !api.getUniqueId)
        throw Error("NCCL is not available: " + (err.empty() ? std::string("missing symbols") : err), -3);
    return api;
}
#define NCCL_CHECK(x)                                                                                  \
    do {                                                                                               \
        ncclResult_t r__ = (x);                                                                        \
        if (r__ != ncclSuccess)                                                                        \
            throw Error(std::string("NCCL error: ") + (nccl().errorString ? nccl().errorString(r__) : "?") + \
                            " at " + __FILE__ + ":" + std::to_string(__LINE__),                        \
                        -3);                                                                           \
    } while (0)

struct DistState {
    ncclComm_t comm = nullptr;
    cudaStream_t cs = nullptr;          // communication stream
    cudaEvent_t ev_ready = nullptr, ev_done = nullptr;
    int world = 1, rank = 0;
    ~DistState() {
        if (comm && nccl().commDestroy) nccl().commDestroy(comm);
        if (ev_ready) cudaEventDestroy(ev_ready);
        if (ev_done) cudaEventDestroy(ev_done);
        if (cs) cudaStreamDestroy(cs);
    }
};

struct LimbBlock {
    int lo, cnt, per;
};
// rank's block of n limbs (per = ceil(n / world); ranks past the end own nothing)
static LimbBlock limb_block(int n, int world, int rank) {
    const int per = (n + world - 1) / world;
    const int lo = std::min(n, rank * per);
    return {lo, std::min(n, lo + per) - lo, per};
}

// ---------------------------------------------------------------------------- kernels ----
// ModUp onto the rank's own extended limbs o < no (Q limbs qlo.., then P limbs plo..; blockIdx.y
// = o, blockIdx.z = digit j): the digit's own limbs are copied from dcoef (coefficient form, the
// NTT that follows brings them back to d's eval words), the others are the base conversion of
// k_modup_bconv with its table (indexed by the global extended limb).
__global__ void __launch_bounds__(256) k_dist_modup(const uint64_t* __restrict__ dcoef, uint64_t* __restrict__ ext,
                                                    const uint64_t* __restrict__ tab, int nl, int ne, int alpha, int L,
                                                    int logN, int qlo, int nqo, int plo, int no) {
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int o = blockIdx.y, j = blockIdx.z, dn = gridDim.z;
    const int e = o < nqo ? qlo + o : nl + plo + (o - nqo);
    const int lo = j * alpha, sz = min(alpha, nl - lo);
    uint64_t* out = ext + ((size_t)j * no + o) * N + x;
    if (e >= lo && e < lo + sz) {
        *out = dcoef[(size_t)e * N + x];
        return;
    }
    const uint64_t* qhinv = tab + (size_t)j * alpha * 2;
    const uint64_t* w = tab + (size_t)dn * alpha * 2 + ((size_t)j * ne + e) * alpha * 2;
    const ModConst mt = c_mod[e < nl ? e : L + (e - nl)];
    u128acc s{0, 0};
#pragma unroll
    for (int a = 0; a < 8; a++)
        if (a < sz) {
            const uint64_t t = mul_shoup(dcoef[(size_t)(lo + a) * N + x], qhinv[2 * a], qhinv[2 * a + 1], c_mod[lo + a].q);
            acc_mad32(s, t, w[2 * a + 1]);
        }
    *out = redc(s.hi, s.lo, mt);
}

// key inner product on the rank's own extended limbs: out[c][o] = sum_j ext[j][o] key[j][c][m(o)]
__global__ void k_dist_inner(const uint64_t* __restrict__ ext, const uint64_t* __restrict__ key,
                             uint64_t* __restrict__ out, int nl, int dnum, int L, int K, int logN, int qlo, int nqo,
                             int plo, int no) {
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int o = blockIdx.y;
    const int m = o < nqo ? qlo + o : L + plo + (o - nqo);
    const ModConst mc = c_mod[m];
    const size_t nk = (size_t)(L + K);
    u128acc a0{0, 0}, a1{0, 0};
    digit_dot2(ext + (size_t)o * N + x, (size_t)no * N, key + (size_t)m * N + x, key + (nk + m) * N + x, 2 * nk * N,
               dnum, a0, a1);
    out[(size_t)o * N + x] = redc(a0.hi, a0.lo, mc);
    out[((size_t)no + o) * N + x] = redc(a1.hi, a1.lo, mc);
}

// the rank's special limbs of both products into the all-gather block [per][2][N]
__global__ void k_dist_pack_p(const uint64_t* __restrict__ ip, uint64_t* __restrict__ send, int nqo, int no,
                              int logN) {
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int i = blockIdx.y, c = blockIdx.z;
    send[((size_t)i * 2 + c) * N + x] = ip[((size_t)c * no + nqo + i) * N + x];
}

// ModDown conversion of the gathered P part (pc [K][2][N], coefficient form) to the rank's Q
// limbs: the formula of k_moddown_bconv with its table d_md
__global__ void k_dist_moddown_bconv(const uint64_t* __restrict__ pc, uint64_t* __restrict__ y,
                                     const uint64_t* __restrict__ md, int L, int K, int logN, int qlo, int nqo) {
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int c = blockIdx.y;
    uint64_t t[8];
#pragma unroll
    for (int k = 0; k < 8; k++)
        if (k < K) t[k] = mul_shoup(pc[((size_t)k * 2 + c) * N + x], md[2 * k], md[2 * k + 1], c_mod[L + k].q);
    const uint64_t* ph = md + 2 * K;
    for (int o = 0; o < nqo; o++) {
        const int i = qlo + o;
        const uint64_t q = c_mod[i].q;
        const uint64_t* w = ph + (size_t)i * K * 2;
        uint64_t s = 0;
#pragma unroll
        for (int k = 0; k < 8; k++)
            if (k < K) s += mul_shoup_lazy(t[k], w[2 * k], w[2 * k + 1], q);
        y[((size_t)c * nqo + o) * N + x] = reduce_lazy16(s, q);
    }
}

// out_c[o] = (ip[c][o] - y[c][o]) P^-1 mod q_{qlo + o}
__global__ void k_dist_moddown_final(const uint64_t* __restrict__ ip, const uint64_t* __restrict__ y,
                                     uint64_t* out0, uint64_t* out1, const uint64_t* __restrict__ md, int L, int K,
                                     int logN, int qlo, int nqo, int no) {
    const int N = 1 << logN;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int o = blockIdx.y, c = blockIdx.z, i = qlo + o;
    const uint64_t q = c_mod[i].q;
    const uint64_t* pinv = md + 2 * K + (size_t)L * K * 2 + (size_t)i * 2;
    const uint64_t v = mod_sub(ip[((size_t)c * no + o) * N + x], y[((size_t)c * nqo + o) * N + x], q);
    (c == 0 ? out0 : out1)[(size_t)o * N + x] = mul_shoup(v, pinv[0], pinv[1], q);
}

// ------------------------------------------------------------------------------ host ----
static DistState& dist_state(Context& cx) {
    auto* d = static_cast<DistState*>(cx.dist.get());
    if (!d) throw Error("keyswitch_dist: the context has not joined a group (fhe_dist_init)", -1);
    return *d;
}

void dist_init(Context& cx, int world, int rank, const uint8_t id[128]) {
    if (world < 1 || rank < 0 || rank >= world) throw Error("dist_init: bad world size or rank", -1);
    auto st = std::make_shared<DistState>();
    st->world = world;
    st->rank = rank;
    ncclUniqueId uid;
    std::memcpy(uid.internal, id, sizeof uid.internal);
    NCCL_CHECK(nccl().commInitRank(&st->comm, world, uid, rank));
    CUDA_CHECK(cudaStreamCreateWithFlags(&st->cs, cudaStreamNonBlocking));
    CUDA_CHECK(cudaEventCreateWithFlags(&st->ev_ready, cudaEventDisableTiming));
    CUDA_CHECK(cudaEventCreateWithFlags(&st->ev_done, cudaEventDisableTiming));
    cx.dist = st;
}

void dist_unique_id(uint8_t out[128]) {
    ncclUniqueId uid;
    NCCL_CHECK(nccl().getUniqueId(&uid));
    std::memcpy(out, uid.internal, sizeof uid.internal);
}

// all-gather of `count` words per rank from send into recv, on the communication stream,
// ordered after the compute stream's work so far and before its next launch
static void dist_allgather(Context& cx, DistState& ds, const uint64_t* send, uint64_t* recv, size_t count) {
    CUDA_CHECK(cudaEventRecord(ds.ev_ready, cx.stream));
    CUDA_CHECK(cudaStreamWaitEvent(ds.cs, ds.ev_ready, 0));
    NCCL_CHECK(nccl().allGather(send, recv, count, ncclUint64, ds.comm, ds.cs));
    CUDA_CHECK(cudaEventRecord(ds.ev_done, ds.cs));
    CUDA_CHECK(cudaStreamWaitEvent(cx.stream, ds.ev_done, 0));
}

// d_own: the rank's Q limbs of d (nl = L - level limbs in all), eval form, device memory;
// out0/out1: the rank's Q limbs of the key-switched pair (same block)
void keyswitch_dist(Context& cx, const uint64_t* d_own, int nl, const SwitchKey& key, uint64_t* out0,
                    uint64_t* out1) {
    DistState& ds = dist_state(cx);
    const int N = cx.N, K = cx.K, L = cx.L, ne = nl + K, dn = cx.dnum(nl);
    const LimbBlock qb = limb_block(nl, ds.world, ds.rank), pb = limb_block(K, ds.world, ds.rank);
    const int no = qb.cnt + pb.cnt;
    cudaStream_t st = cx.stream;
    // 1. the rank's limbs of d in coefficient form, gathered
    DevBuf send1((size_t)qb.per * N, st), dcoef((size_t)ds.world * qb.per * N, st);
    if (qb.cnt) {
        CUDA_CHECK(cudaMemcpyAsync(send1.p, d_own, (size_t)qb.cnt * N * 8, cudaMemcpyDeviceToDevice, st));
        LimbMap m1 = cx.qmap(send1.p, qb.cnt, (long long)qb.cnt * N);
        m1.off0 = qb.lo;
        ntt(cx, m1, 1, true, st);
    }
    dist_allgather(cx, ds, send1.p, dcoef.p, (size_t)qb.per * N);
    // 2. ModUp to the own extended limbs, NTT, key inner product
    DevBuf ext((size_t)std::max(1, dn * no) * N, st), ip((size_t)2 * std::max(1, no) * N, st);
    if (no) {
        k_dist_modup<<<dim3(N / 256, no, dn), 256, 0, st>>>(dcoef.p, ext.p, cx.modup_table(nl), nl, ne, cx.alpha, L,
                                                           cx.logN, qb.lo, qb.cnt, pb.lo, no);
        LimbMap em{};
        em.base = ext.p; em.poly_stride = (long long)no * N; em.nl = no;
        em.split = qb.cnt; em.off0 = qb.lo; em.off1 = L + pb.lo;
        ntt(cx, em, dn, false, st);
        k_dist_inner<<<dim3(N / 256, no), 256, 0, st>>>(ext.p, key.buf.p, ip.p, nl, dn, L, K, cx.logN, qb.lo, qb.cnt,
                                                        pb.lo, no);
        cx.launches += 2;
    }
    // 3. the own special limbs of both products in coefficient form, gathered
    DevBuf send2((size_t)pb.per * 2 * N, st), pc((size_t)ds.world * pb.per * 2 * N, st);
    if (pb.cnt) {
        LimbMap pm{};
        pm.base = ip.p + (size_t)qb.cnt * N; pm.poly_stride = (long long)no * N; pm.nl = pb.cnt;
        pm.split = 0; pm.off0 = 0; pm.off1 = L + pb.lo;
        ntt(cx, pm, 2, true, st);
        k_dist_pack_p<<<dim3(N / 256, pb.cnt, 2), 256, 0, st>>>(ip.p, send2.p, qb.cnt, no, cx.logN);
        cx.launches++;
    }
    dist_allgather(cx, ds, send2.p, pc.p, (size_t)pb.per * 2 * N);
    // 4. ModDown on the own Q limbs
    if (qb.cnt) {
        DevBuf y((size_t)2 * qb.cnt * N, st);
        k_dist_moddown_bconv<<<dim3(N / 256, 2), 256, 0, st>>>(pc.p, y.p, cx.d_md, L, K, cx.logN, qb.lo, qb.cnt);
        LimbMap ym = cx.qmap(y.p, qb.cnt, (long long)qb.cnt * N);
        ym.off0 = qb.lo;
        ntt(cx, ym, 2, false, st);
        k_dist_moddown_final<<<dim3(N / 256, qb.cnt, 2), 256, 0, st>>>(ip.p, y.p, out0, out1, cx.d_md, L, K, cx.logN,
                                                                      qb.lo, qb.cnt, no);
        cx.launches += 2;
    }
    CUDA_CHECK(cudaGetLastError());
    cx.ks_count++;
    cx.ks_limbs += nl;
}

}  // namespace fhe

extern "C" {

int fhe_dist_unique_id(uint8_t* out) {
    return guard([&] {
        REQUIRE(out, "null argument");
        fhe::dist_unique_id(out);
    });
}

int fhe_dist_init(fhe_ctx* cx, int world, int rank, const uint8_t* id) {
    return guard([&] {
        REQUIRE(cx && id, "null argument");
        bind(cx);
        fhe::dist_init(cx->cx, world, rank, id);
    });
}

int fhe_dist_limbs(const fhe_ctx* cx, int level, int* first, int* count) {
    return guard([&] {
        REQUIRE(cx && first && count, "null argument");
        const auto* d = static_cast<fhe::DistState*>(cx->cx.dist.get());
        REQUIRE(d, "the context has not joined a group (fhe_dist_init)");
        const fhe::LimbBlock b = fhe::limb_block(nl_of(cx->cx, level), d->world, d->rank);
        *first = b.lo;
        *count = b.cnt;
    });
}

int fhe_keyswitch_dist(fhe_ctx* cx, uint64_t which, const uint64_t* d_own, int level, uint64_t* out0,
                       uint64_t* out1) {
    return guard([&] {
        REQUIRE(cx && d_own && out0 && out1, "null argument");
        bind(cx);
        auto& c = cx->cx;
        fhe::keyswitch_dist(c, d_own, nl_of(c, level), *find_key(c, which), out0, out1);
    });
}

}  // extern "C"
