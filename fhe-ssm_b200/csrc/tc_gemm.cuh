// tc_gemm.cuh -- the BSGS product of matvec.cu on the 5th-generation tensor cores (tcgen05).
//
// Per CTA (limb e, one group of 32 slots sharing a compressed plaintext word, both polynomials:
// 64 columns n) the product is C[o][n] = sum_k W[o][k] B[k][n] over words < q < 2^60, exact.
// Words are split into bytes, W = sum_a W_a 256^a, B = sum_b B_b 256^b, and grouped by
// diagonal d = a + b:
//     C = sum_d 256^d D_d,   D_d[n][o] = sum_a sum_k B_{d-a}[k][n] W_a[o][k]     (< 2^26, int32)
// D_d for all 15 diagonals is a sequence of u8 x u8 -> s32 tcgen05.mma (kind::i8) with
// accumulators in tensor memory: the M side (128 rows) stacks the 64 columns n of two
// diagonals d, d+1, the N side is the M_out outputs o, K runs over byte slice a and the babies
// k.  Shared memory holds B as byte slices -1..8 (slices -1 and 8 are zero, so the two
// stacked diagonals can share one descriptor) and W as byte slices 0..7, both K-major in the
// no-swizzle canonical layout (core matrix = 8 rows x 16 bytes; LBO = 128 B between K chunks,
// SBO = 8 Kp B between 8-row groups).  The epilogue reads the accumulators with tcgen05.ld,
// rebuilds the 128-bit value sum_d 256^d D_d (< K q^2 < 2^127) and Montgomery-reduces it.
//
// Descriptor layouts follow the sm100 UMMA descriptor definitions of CUTLASS/CuTe
// (cute/arch/mma_sm100_desc.hpp: SmemDescriptor, InstrDescriptor).
//
// Included by matvec.cu inside namespace fhe (it uses GemmArgs).

constexpr int kTcThreads = 128;
constexpr int kTcMaxIters = 1 << 26;   // bounded mbarrier wait (a few seconds)

__device__ __forceinline__ uint32_t tc_smem(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// K-major, no swizzle; addresses and offsets in bytes (multiples of 16)
__device__ __forceinline__ uint64_t tc_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}
// kind::i8, D s32, A u8, B u8, both K-major, M = 128, N = n
__host__ __device__ constexpr uint32_t tc_idesc(int n) {
    return (2u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t phase) {
    for (int it = 0; it < kTcMaxIters; it++) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(ok)
            : "r"(tc_smem(bar)), "r"(phase)
            : "memory");
        if (ok) return true;
    }
    return false;
}

__device__ __forceinline__ void tc_ld8(uint32_t taddr, uint32_t* v) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
}

// Shared memory of k_bsgs_tc2 (dynamic, bytes): [M side: 10 slices x 64 Kp][N side: 8 slices x
// MP Kp][2 barriers][tmem address].  Slices 0..7 of the M side double as the epilogue exchange buffer.
__host__ __device__ inline size_t tc_smem_bytes(int Mp, int Kp) {
    return (size_t)10 * 64 * Kp + (size_t)8 * Mp * Kp + 24;
}

// ---------------------------------------------------------------------------------------------
// Operands packed in global memory as the exact shared-memory image of a tile, so that the
// product kernel only issues bulk copies (cp.async.bulk, completion counted on an mbarrier).

// Babies of one set -> per (limb e, group r of 32 slots) a block of byte slices 0..7, each 64
// rows (n = c * 32 + slot) x Kp bytes (k), K-major core-matrix order.  One CTA per (r, e); the
// block is assembled in shared memory and written with 16-byte stores.
__global__ void __launch_bounds__(256) k_tc_split_babies(const uint64_t* __restrict__ bb, uint8_t* __restrict__ out,
                                                         int K, int Kp, int ne, int nl, int L, int logN) {
    extern __shared__ __align__(16) uint8_t ss[];   // [8][64 Kp]
    const int N = 1 << logN;
    const int r = blockIdx.x, e = blockIdx.y, x0 = r * 32;
    // words of this limb are < q: only byte slices 0..nbyte-1 are written (the product kernel
    // reads no others)
    const int nbyte = (int)((c_mod[e < nl ? e : L + (e - nl)].k + 7) / 8);
    const uint32_t SB = 8u * Kp;
    for (int t = threadIdx.x; t < 64 * (Kp / 4); t += blockDim.x) {
        const int n = t & 63, k4 = t >> 6, c = n >> 5, xs = n & 31;
        uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int k = 4 * k4 + u;
            if (k < K) {
                const uint64_t v = bb[(((size_t)k * 2 + c) * ne + e) * N + x0 + xs];
#pragma unroll
                for (int b = 0; b < 8; b++) w[b] |= (uint32_t)((v >> (8 * b)) & 0xFF) << (8 * u);
            }
        }
        const int k = 4 * k4;
        const size_t off = (size_t)(n >> 3) * SB + (size_t)(k >> 4) * 128 + (size_t)(n & 7) * 16 + (k & 15);
#pragma unroll
        for (int b = 0; b < 8; b++)
            if (b < nbyte) *reinterpret_cast<uint32_t*>(ss + (size_t)b * 64 * Kp + off) = w[b];
    }
    __syncthreads();
    uint4* dst = reinterpret_cast<uint4*>(out + ((size_t)e * (N / 32) + r) * 8 * 64 * Kp);
    const uint4* src = reinterpret_cast<const uint4*>(ss);
    for (int i = threadIdx.x; i < nbyte * 64 * Kp / 16; i += blockDim.x) dst[i] = src[i];
}

// Plaintext words of set s of a plan -> per (limb e, compressed word w) a block of byte slices
// 0..7, each Mp rows (outputs o) x Kp bytes (babies k): W[o][k] is the word of family
// fam(o, k), giant g(o), baby j(k), or 0.
__global__ void __launch_bounds__(256) k_tc_pack_w(const uint64_t* __restrict__ pts, const int* __restrict__ ids,
                                                   uint8_t* __restrict__ out, int s, int G, int b1, int Kp, int Mp,
                                                   int D2, int P, int nl, int L) {
    extern __shared__ __align__(16) uint8_t sw[];   // [8][Mp Kp]
    const int wi = blockIdx.x, e = blockIdx.y;
    const int nbyte = (int)((c_mod[e < nl ? e : L + (e - nl)].k + 7) / 8);   // slices the product reads
    const int M = Mp, K = 2 * b1;   // outputs o: giant g = o % G of family X = o / G (X = 1: none)
    const uint32_t SB = 8u * Kp;
    const uint64_t* row = pts + ((size_t)e * D2 + wi) * P;
    for (int t = threadIdx.x; t < Mp * (Kp / 4); t += blockDim.x) {
        const int o = t % Mp, k4 = t / Mp;
        uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (o < M) {
            const int X = o / G, g = o % G;
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int k = 4 * k4 + u;
                if (k >= K) continue;
                const int Y = k / b1, j = k % b1;
                const int fam = X == 0 ? Y : (Y == 0 ? 2 : -1);
                const int id = fam >= 0 ? ids[(((size_t)s * 3 + fam) * G + g) * b1 + j] : -1;
                if (id < 0) continue;
                const uint64_t v = row[id];
#pragma unroll
                for (int b = 0; b < 8; b++) w[b] |= (uint32_t)((v >> (8 * b)) & 0xFF) << (8 * u);
            }
        }
        const int k = 4 * k4;
        const size_t off = (size_t)(o >> 3) * SB + (size_t)(k >> 4) * 128 + (size_t)(o & 7) * 16 + (k & 15);
#pragma unroll
        for (int b = 0; b < 8; b++)
            if (b < nbyte) *reinterpret_cast<uint32_t*>(sw + (size_t)b * Mp * Kp + off) = w[b];
    }
    __syncthreads();
    const size_t blk = (size_t)8 * Mp * Kp;
    uint4* dst = reinterpret_cast<uint4*>(out + ((size_t)e * D2 + wi) * blk);
    const uint4* src = reinterpret_cast<const uint4*>(sw);
    for (int i = threadIdx.x; i < (int)((size_t)nbyte * Mp * Kp / 16); i += blockDim.x) dst[i] = src[i];
}

struct Tc2Args {
    const uint8_t* bsplit[kMaxSets];   // per set: [ne][N/32][8][64 Kp]
    const uint8_t* wpack;              // [set][ne][2D][8][Mp Kp]
    uint64_t* out;                     // [M][2][ne][N]
    int nsets, G, M, nl, ne, L, logN, lr, D2, Kp;
};

__device__ __forceinline__ void tc_bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                     tc_smem(dst)),
                 "l"(src), "r"(bytes), "r"(tc_smem(bar))
                 : "memory");
}

// The product kernel on packed operands: per set, two bulk copies (babies 8 x 64 Kp bytes,
// plaintext words 8 x Mp Kp bytes) into the slices of the shared-memory image, then the MMAs
// and the epilogue of k_bsgs_tc.
template <int MP>
__global__ void __launch_bounds__(kTcThreads, 1) k_bsgs_tc2(const Tc2Args a, uint32_t tcols, unsigned int* err) {
    extern __shared__ __align__(1024) uint8_t tsm[];
    constexpr int Mp = MP;
    const int Kp = a.Kp;
    uint8_t* Ms = tsm;                                        // slice s (-1..8) at (s + 1) * 64 Kp
    uint8_t* Ns = tsm + (size_t)10 * 64 * Kp;                 // slice a at a * Mp Kp
    uint64_t* bar = (uint64_t*)(Ns + (size_t)8 * Mp * Kp);    // [0] copies, [1] MMAs
    uint32_t* tslot = (uint32_t*)(bar + 2);
    const int N = 1 << a.logN;
    const int r = blockIdx.x, e = blockIdx.y, x0 = r * 32;
    const int m = e < a.nl ? e : a.L + (e - a.nl);
    const ModConst mc = c_mod[m];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int M = a.M, ptw = x0 >> a.lr;
    const uint32_t SB = 8u * Kp;
    // words of this limb are < q: their bytes nbyte.. are zero, and so are the diagonals
    // d > 2 (nbyte - 1): only those MMAs and tensor-memory columns are used (45-bit limbs:
    // 6 bytes, 6 diagonal pairs, 84 of 144 MMAs), and only byte slices 0..nbyte-1 are copied
    const int nbyte = (int)((mc.k + 7) / 8);
    const int npairs = nbyte;   // pairs p with 2p <= 2 (nbyte - 1)
    const uint32_t bbytes = (uint32_t)nbyte * 64u * Kp, wbytes = (uint32_t)nbyte * Mp * Kp;

    // zero M-side slots: slot 0 (slice -1) and slots nbyte+1..9 (slices nbyte..8, read by the
    // stacked second diagonal of the top pairs and never copied)
    for (int i = tid; i < 64 * Kp / 16; i += kTcThreads) {
        reinterpret_cast<uint4*>(Ms)[i] = make_uint4(0, 0, 0, 0);
        for (int sl = nbyte + 1; sl <= 9; sl++)
            reinterpret_cast<uint4*>(Ms + (size_t)sl * 64 * Kp)[i] = make_uint4(0, 0, 0, 0);
    }
    uint64_t run[Mp];
#pragma unroll
    for (int o = 0; o < Mp; o++) run[o] = 0;
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tc_smem(bar)));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tc_smem(bar + 1)));
        asm volatile("fence.mbarrier_init.release.cluster;");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc_smem(tslot)),
                     "r"(tcols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("fence.proxy.async.shared::cta;");   // zero slices, before the tensor cores read them
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t taddr = *tslot;
    const uint32_t idesc = tc_idesc(Mp);
    bool ok = true;

    for (int s = 0; s < a.nsets && ok; s++) {
        if (tid == 0) {
            asm volatile("fence.proxy.async.shared::cta;");   // the previous epilogue's exchange writes
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc_smem(bar)),
                         "r"(bbytes + wbytes)
                         : "memory");
            tc_bulk_g2s(Ms + (size_t)64 * Kp, a.bsplit[s] + ((size_t)e * (N / 32) + r) * 8 * 64 * Kp, bbytes, bar);
            tc_bulk_g2s(Ns, a.wpack + (((size_t)s * a.ne + e) * a.D2 + ptw) * 8 * Mp * Kp, wbytes, bar);
        }
        ok = __syncthreads_and(tc_wait(bar, (uint32_t)(s & 1)) ? 1 : 0) != 0;
        if (!ok) {
            if (tid == 0) atomicExch(err, 1u);
            tc_wait(bar, (uint32_t)(s & 1));
            break;
        }
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;");
            const uint32_t mbase = tc_smem(Ms), nbase = tc_smem(Ns);
            for (int p = 0; p < npairs; p++) {
                const int d = 2 * p;
                bool first = true;
                for (int aa = max(0, d - (nbyte - 1)); aa <= min(nbyte - 1, d + 1); aa++) {
                    const uint32_t ma = mbase + (uint32_t)(d - aa + 1) * 64u * Kp;
                    const uint32_t na = nbase + (uint32_t)aa * Mp * Kp;
                    for (int ks = 0; ks < Kp / 32; ks++) {
                        tc_mma(taddr + (uint32_t)(p * Mp), tc_desc(ma + ks * 256, 128, SB), tc_desc(na + ks * 256, 128, SB),
                               idesc, first ? 0u : 1u);
                        first = false;
                    }
                }
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                tc_smem(bar + 1)));
        }
        ok = __syncthreads_and(tc_wait(bar + 1, (uint32_t)(s & 1)) ? 1 : 0) != 0;
        if (!ok) {
            if (tid == 0) atomicExch(err, 1u);
            tc_wait(bar + 1, (uint32_t)(s & 1));
            break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;");
        const int row = 32 * warp + lane, n = row & 63, h = row >> 6;
        unsigned __int128* xch = reinterpret_cast<unsigned __int128*>(Ms + (size_t)64 * Kp);
#pragma unroll
        for (int oc = 0; oc < Mp / 8; oc++) {
            unsigned __int128 acc[8];
#pragma unroll
            for (int j = 0; j < 8; j++) acc[j] = 0;
            // the accumulators of PB diagonal pairs are loaded together before one wait (one
            // tensor-memory round trip per group instead of one per pair)
            constexpr int PB = MP >= 64 ? 4 : 8;
#pragma unroll
            for (int p0 = 0; p0 < 8; p0 += PB) {
                if (p0 >= npairs) break;   // uniform: all diagonals beyond are zero
                uint32_t v[PB][8];
#pragma unroll
                for (int p = 0; p < PB; p++)   // columns of all 8 pairs are allocated (tcols = 8 Mp)
                    tc_ld8(taddr + ((uint32_t)(32 * warp) << 16) + (uint32_t)((p0 + p) * Mp + oc * 8), v[p]);
                asm volatile("tcgen05.wait::ld.sync.aligned;");
#pragma unroll
                for (int p = 0; p < PB; p++) {
                    if (p0 + p >= npairs) break;
                    const int sh = 8 * (2 * (p0 + p) + h);
#pragma unroll
                    for (int j = 0; j < 8; j++) acc[j] += (unsigned __int128)v[p][j] << sh;
                }
            }
            __syncthreads();
            if (h == 1) {
#pragma unroll
                for (int j = 0; j < 8; j++) xch[n * 8 + j] = acc[j];
            }
            __syncthreads();
            if (h == 0) {
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int o = oc * 8 + j;
                    if (o >= M) continue;
                    const unsigned __int128 tot = acc[j] + xch[n * 8 + j];
                    uint64_t hi = (uint64_t)(tot >> 64);
                    const uint64_t lo = (uint64_t)tot;
                    if (hi >= 4 * mc.q) hi -= 4 * mc.q;
                    if (hi >= 2 * mc.q) hi -= 2 * mc.q;
                    if (hi >= mc.q) hi -= mc.q;
                    run[o] = mod_add(run[o], redc(hi, lo, mc), mc.q);
                }
            }
        }
        // the next bulk copy (async proxy) overwrites the exchange buffer written here
        asm volatile("fence.proxy.async.shared::cta;");
        asm volatile("tcgen05.fence::before_thread_sync;");
        __syncthreads();
    }
    if (ok && tid < 64) {
        const int c = tid >> 5, xs = tid & 31;
#pragma unroll
        for (int o = 0; o < Mp; o++)
            if (o < M) a.out[(((size_t)o * 2 + c) * a.ne + e) * N + x0 + xs] = run[o];
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(tcols));
}
