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

// Shared memory (dynamic, bytes): [Mside: 10 slices x 64 Kp][Nside: 8 slices x MP Kp][barrier 8]
// [tmem address 4].  Slices 0..7 of the M side double as the epilogue exchange buffer.
__host__ __device__ inline size_t tc_smem_bytes(int Mp, int Kp) {
    return (size_t)10 * 64 * Kp + (size_t)8 * Mp * Kp + 16;
}

template <int MP>
__global__ void __launch_bounds__(kTcThreads, 1) k_bsgs_tc(const GemmArgs a, int Kp, uint32_t tcols,
                                                           unsigned int* err) {
    extern __shared__ __align__(1024) uint8_t tsm[];
    constexpr int Mp = MP;
    uint8_t* Ms = tsm;                                        // slice s (-1..8) at (s + 1) * 64 Kp
    uint8_t* Ns = tsm + (size_t)10 * 64 * Kp;                 // slice a at a * Mp Kp
    uint64_t* bar = (uint64_t*)(Ns + (size_t)8 * Mp * Kp);
    uint32_t* tslot = (uint32_t*)(bar + 1);
    const int N = 1 << a.logN;
    const int e = blockIdx.y, x0 = blockIdx.x * 32;
    const int m = e < a.nl ? e : a.L + (e - a.nl);
    const ModConst mc = c_mod[m];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int M = 2 * a.G, K = 2 * a.b1, ptw = x0 >> a.lr;
    const uint32_t SB = 8u * Kp;   // bytes between 8-row groups

    // zero: slices -1 and 8 (never written again), the running sums
    for (int i = tid; i < 64 * Kp / 16; i += kTcThreads) {
        reinterpret_cast<uint4*>(Ms)[i] = make_uint4(0, 0, 0, 0);
        reinterpret_cast<uint4*>(Ms + (size_t)9 * 64 * Kp)[i] = make_uint4(0, 0, 0, 0);
    }
    uint64_t run[Mp];   // threads of rows 0..63 (h = 0): running sums mod q of column n, all outputs
#pragma unroll
    for (int o = 0; o < Mp; o++) run[o] = 0;
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tc_smem(bar)));
        asm volatile("fence.mbarrier_init.release.cluster;");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc_smem(tslot)),
                     "r"(tcols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t taddr = *tslot;
    const uint32_t idesc = tc_idesc(Mp);
    bool ok = true;

    for (int s = 0; s < a.nsets && ok; s++) {
        const uint64_t* bb = a.babies[s];
        // ---- stage B (M side): byte b of word B[k][n] -> slice b, row n, K byte k
        for (int t = tid; t < 64 * (Kp / 4); t += kTcThreads) {
            const int n = t & 63, k4 = t >> 6, c = n >> 5, xs = n & 31;
            uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int k = 4 * k4 + u;
                if (k < K) {
                    const uint64_t v = bb[(((size_t)k * 2 + c) * a.ne + e) * N + x0 + xs];
#pragma unroll
                    for (int b = 0; b < 8; b++) w[b] |= (uint32_t)((v >> (8 * b)) & 0xFF) << (8 * u);
                }
            }
            const int k = 4 * k4;
            const size_t off = (size_t)(n >> 3) * SB + (size_t)(k >> 4) * 128 + (size_t)(n & 7) * 16 + (k & 15);
#pragma unroll
            for (int b = 0; b < 8; b++) *reinterpret_cast<uint32_t*>(Ms + (size_t)(b + 1) * 64 * Kp + off) = w[b];
        }
        // ---- stage W (N side): byte a of W[o][k] -> slice a, row o, K byte k (rows o >= M are zero)
        for (int t = tid; t < Mp * (Kp / 4); t += kTcThreads) {
            const int o = t % Mp, k4 = t / Mp;
            uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            if (o < M) {
                const int X = o / a.G, g = o % a.G;
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int k = 4 * k4 + u;
                    if (k >= K) continue;
                    const int Y = k / a.b1, j = k % a.b1;
                    const int fam = X == 0 ? Y : (Y == 0 ? 2 : -1);
                    int id = -1;
                    if (fam >= 0) id = a.ids[(((size_t)s * 3 + fam) * a.G + g) * a.b1 + j];
                    if (id < 0) continue;
                    const uint64_t v = a.pts[((size_t)e * a.D2 + ptw) * a.P + id];
#pragma unroll
                    for (int b = 0; b < 8; b++) w[b] |= (uint32_t)((v >> (8 * b)) & 0xFF) << (8 * u);
                }
            }
            const int k = 4 * k4;
            const size_t off = (size_t)(o >> 3) * SB + (size_t)(k >> 4) * 128 + (size_t)(o & 7) * 16 + (k & 15);
#pragma unroll
            for (int b = 0; b < 8; b++) *reinterpret_cast<uint32_t*>(Ns + (size_t)b * Mp * Kp + off) = w[b];
        }
        asm volatile("fence.proxy.async.shared::cta;");
        __syncthreads();
        // ---- MMAs: pair p = diagonals (2p, 2p+1) into tensor-memory columns [p Mp, (p+1) Mp)
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;");
            const uint32_t mbase = tc_smem(Ms), nbase = tc_smem(Ns);
            for (int p = 0; p < 8; p++) {
                const int d = 2 * p;
                bool first = true;
                for (int aa = max(0, d - 7); aa <= min(7, d + 1); aa++) {
                    const uint32_t ma = mbase + (uint32_t)(d - aa + 1) * 64u * Kp;   // slice d - aa (rows 64..127: d + 1 - aa)
                    const uint32_t na = nbase + (uint32_t)aa * Mp * Kp;
                    for (int ks = 0; ks < Kp / 32; ks++) {
                        tc_mma(taddr + (uint32_t)(p * Mp), tc_desc(ma + ks * 256, 128, SB), tc_desc(na + ks * 256, 128, SB),
                               idesc, first ? 0u : 1u);
                        first = false;
                    }
                }
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                tc_smem(bar)));
        }
        // every thread waits; the outcome is made uniform so that no thread leaves a barrier early
        ok = __syncthreads_and(tc_wait(bar, (uint32_t)(s & 1)) ? 1 : 0) != 0;
        if (!ok) {
            if (tid == 0) atomicExch(err, 1u);
            tc_wait(bar, (uint32_t)(s & 1));   // a second bounded wait for the MMAs in flight
            break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;");
        // ---- epilogue: warp w holds rows 32w..32w+31: n = row % 64, half h = row / 64 (d = 2p + h)
        const int row = 32 * warp + lane, n = row & 63, h = row >> 6;
        unsigned __int128* xch = reinterpret_cast<unsigned __int128*>(Ms + (size_t)64 * Kp);   // slices 0.., [64 n][8]
#pragma unroll
        for (int oc = 0; oc < Mp / 8; oc++) {
            unsigned __int128 acc[8];
#pragma unroll
            for (int j = 0; j < 8; j++) acc[j] = 0;
#pragma unroll
            for (int p = 0; p < 8; p++) {
                uint32_t v[8];
                tc_ld8(taddr + ((uint32_t)(32 * warp) << 16) + (uint32_t)(p * Mp + oc * 8), v);
                asm volatile("tcgen05.wait::ld.sync.aligned;");
                const int sh = 8 * (2 * p + h);
#pragma unroll
                for (int j = 0; j < 8; j++) acc[j] += (unsigned __int128)v[j] << sh;
            }
            __syncthreads();   // previous readers of xch are done
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
                    // < 128 q^2 / 2^64 < 8q for 60-bit words
                    if (hi >= 4 * mc.q) hi -= 4 * mc.q;
                    if (hi >= 2 * mc.q) hi -= 2 * mc.q;
                    if (hi >= mc.q) hi -= mc.q;
                    run[o] = mod_add(run[o], redc(hi, lo, mc), mc.q);
                }
            }
        }
        asm volatile("tcgen05.fence::before_thread_sync;");
        __syncthreads();   // tensor memory and the exchange buffer are free for the next set
    }
    // ---- outputs: out[o][c][e][x0 + xs] for column n = 32 c + xs (threads of rows 0..63)
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
