// ntt.cu -- batched negacyclic NTT / inverse NTT for RNS limbs, N = 2^12 .. 2^16.
//
// Ordering (the reference's encoder states it for OpenFHE, hpc_gpu_port/periodic_encode.hpp:
// 141-161 and :240-260): the forward transform takes natural-order coefficients to
// bit-reversed evaluations with the root table Tab[brev(i)] = psi^i (Cooley-Tukey); the
// inverse takes bit-reversed evaluations back to natural-order coefficients
// (Gentleman-Sande) and multiplies by N^-1.
//
// Decomposition.  With N = R * 256 (R = 2^(logN-8), 16 <= R <= 256) the transform splits in
// two kernels of 4096-word tiles held in shared memory, 256 threads, 16 words per thread:
//   phase "col": the logN-8 stages with butterfly distance >= 256.  The limb is an R x 256
//                row-major matrix and each column is an independent R-point transform;
//                a tile is R rows x (4096/R) columns (>= 16 columns: 128-byte row segments).
//   phase "row": the last 8 stages, distance < 256: each 256-word block is independent.
// Inside a tile each thread runs 4 stages on 16 registers, the tile is exchanged through
// shared memory, and the thread runs the remaining stages on another 16 registers.  Every
// twiddle is Shoup-precomputed; all residues stay canonical.
#include "engine.h"

namespace fhe {

// Harvey lazy butterflies.  Forward: inputs in [0, 4q + 2^32) -> outputs in [0, 4q + 2^32);
// the conditional subtraction of 2q looks at the high words only (subtract when u >> 32 exceeds
// 2q >> 32), which leaves u < 2q + 2^32 and saves the low-word compare.  Inverse: inputs in
// [0, 2q) -> outputs in [0, 2q).  4q + 2^32 < 2^63 for the moduli below 2^61; the transforms
// correct to [0, q) at their output.
// Twiddle pairs are loaded with an L2 evict-last policy (a per-load cache hint): the tables are
// re-read by every transform of the same modulus and should outlive the data streaming past them.
__device__ __forceinline__ uint64_t tw_policy() {
    uint64_t p;
    asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ ulonglong2 ld_tw(const ulonglong2* a, uint64_t pol) {
    ulonglong2 v;
    asm("ld.global.nc.L2::cache_hint.v2.u64 {%0, %1}, [%2], %3;" : "=l"(v.x), "=l"(v.y) : "l"(a), "l"(pol));
    return v;
}

// Shoup product with a cheaper quotient (AR = 1 butterflies), written as explicit 32-bit steps.
// est = x1 p1 + hi(x0 p1) + hi(x1 p0) is the high 64 bits of x * wp without the x0 * p0 term and
// the carries out of the cross terms' low halves (x = x1:x0, wp = p1:p0 in 32-bit words): 0 to 2
// below floor(x wp / 2^64), so x w - est q lies in [0, 4q) (Shoup's exact quotient: [0, 2q)).
// x w - est q is formed modulo 2^64 as x w + est (2^64 - q) (nq = 2^64 - q), the subtraction
// folded into the multiply-adds: nine 32-bit multiplies in all, no product at or above bit 64.
__device__ __forceinline__ uint64_t mul_shoup_q4(uint64_t x, uint64_t w, uint64_t wp, uint64_t nq) {
    uint64_t r;
    asm("{\n\t"
        ".reg .u32 x0, x1, w0, w1, p0, p1, n0, n1, h0, h1, e0, e1, r0, r1;\n\t"
        ".reg .u64 e, t;\n\t"
        "mov.b64 {x0, x1}, %1;\n\t"
        "mov.b64 {w0, w1}, %2;\n\t"
        "mov.b64 {p0, p1}, %3;\n\t"
        "mov.b64 {n0, n1}, %4;\n\t"
        "mul.hi.u32 h0, x0, p1;\n\t"
        "mul.hi.u32 h1, x1, p0;\n\t"
        "cvt.u64.u32 t, h0;\n\t"
        "mad.wide.u32 e, x1, p1, t;\n\t"       // est = x1 p1 + hi(x0 p1)
        "cvt.u64.u32 t, h1;\n\t"
        "add.u64 e, e, t;\n\t"                  //     + hi(x1 p0)
        "mov.b64 {e0, e1}, e;\n\t"
        "mul.wide.u32 t, x0, w0;\n\t"
        "mad.wide.u32 t, e0, n0, t;\n\t"        // low words: x0 w0 + e0 n0
        "mov.b64 {r0, r1}, t;\n\t"
        "mad.lo.u32 r1, x0, w1, r1;\n\t"
        "mad.lo.u32 r1, x1, w0, r1;\n\t"
        "mad.lo.u32 r1, e0, n1, r1;\n\t"
        "mad.lo.u32 r1, e1, n0, r1;\n\t"
        "mov.b64 %0, {r0, r1};\n\t"
        "}"
        : "=l"(r)
        : "l"(x), "l"(w), "l"(wp), "l"(nq));
    return r;
}

// AR = 0: the Harvey butterflies above.  AR = 1: the same with mul_shoup_q4; forward values in
// [0, 8q + 2^32) (u is brought below 4q + 2^32 by the high-word test against 4q), inverse values
// in [0, 4q).  8q + 2^33 < 2^64 for the moduli below 2^61.  The output words are the same.
template <bool INV, int AR = 0>
__device__ __forceinline__ void bfly(uint64_t& lo, uint64_t& hi, uint64_t w, uint64_t wp, uint64_t q) {
    if (AR == 1) {
        const uint64_t q4 = q << 2;
        if (!INV) {
            uint64_t u = lo;
            if ((uint32_t)(u >> 32) > (uint32_t)(q4 >> 32)) u -= q4;
            const uint64_t x = mul_shoup_q4(hi, w, wp, 0 - q);
            lo = u + x;
            hi = u - x + q4;
        } else {
            uint64_t u = lo + hi;
            if (u >= q4) u -= q4;
            const uint64_t t = lo - hi + q4;
            hi = mul_shoup_q4(t, w, wp, 0 - q);
            lo = u;
        }
        return;
    }
    const uint64_t q2 = q << 1;
    if (!INV) {
        uint64_t u = lo;
        if ((uint32_t)(u >> 32) > (uint32_t)(q2 >> 32)) u -= q2;
        const uint64_t x = mul_shoup_lazy(hi, w, wp, q);
        lo = u + x;
        hi = u - x + q2;
    } else {
        uint64_t u = lo + hi;
        if (u >= q2) u -= q2;
        const uint64_t t = lo - hi + q2;
        hi = mul_shoup_lazy(t, w, wp, q);
        lo = u;
    }
}
__device__ __forceinline__ uint64_t canon4(uint64_t v, uint64_t q) {   // [0, 4q + 2^32) -> [0, q)
    const uint64_t q2 = q << 1;
    if (v >= q2) v -= q2;   // < 2q + 2^32
    if (v >= q2) v -= q2;   // < 2q
    return v >= q ? v - q : v;
}
// the forward transform's output range of butterflies AR -> [0, q)  (2^32 < q)
template <int AR>
__device__ __forceinline__ uint64_t canon_out(uint64_t v, uint64_t q) {
    if (AR == 0) return canon4(v, q);
    const uint64_t q4 = q << 2, q2 = q << 1;
    if (v >= q4) v -= q4;   // [0, 8q + 2^32) -> [0, 4q + 2^32) < 5q
    if (v >= q2) v -= q2;   // < 3q
    if (v >= q) v -= q;     // < 2q
    return v >= q ? v - q : v;
}

__device__ __forceinline__ bool limb_skipped(const LimbMap& mp, int poly, int limb) {
    if (mp.skip_alpha == 0) return false;
    const int lo = (mp.skip_period > 0 ? poly % mp.skip_period : poly) * mp.skip_alpha;
    return limb >= lo && limb < min(lo + mp.skip_alpha, mp.skip_nq);
}

// One radix-2 stage over a thread's 16 registers at register distance H: butterfly (k, k + H)
// for every k with k & H == 0, using twiddle number k / (2H) of the stage, tw(j).  Each of the
// 8/H distinct twiddles is loaded once.
template <bool INV, int H, int AR, class TW>
__device__ __forceinline__ void stage16h(uint64_t (&x)[16], uint64_t q, TW tw) {
#pragma unroll
    for (int j = 0; j < 8 / H; j++) {
        const ulonglong2 t2 = tw(j);
#pragma unroll
        for (int kk = 0; kk < H; kk++) bfly<INV, AR>(x[2 * H * j + kk], x[2 * H * j + kk + H], t2.x, t2.y, q);
    }
}
template <bool INV, int AR = 0, class TW>
__device__ __forceinline__ void stage16(uint64_t (&x)[16], uint64_t q, int h, TW tw) {
    if (h == 8) stage16h<INV, 8, AR>(x, q, tw);
    else if (h == 4) stage16h<INV, 4, AR>(x, q, tw);
    else if (h == 2) stage16h<INV, 2, AR>(x, q, tw);
    else stage16h<INV, 1, AR>(x, q, tw);
}

// A forward transform with a fused prologue and epilogue (FUSE = true): the rescale of up to
// kFuseMax / 2 ciphertexts.  The column pass reads, in place of its input limb i, the centred
// lift of the dropped limb (coefficient form, src + poly * src_stride) modulo q_i; the row pass
// writes, in place of the transformed lift y, the rescaled limb dst[poly]_i = (dst[poly]_i - y)
// * q_l^-1 (rs: [l][i][2], q_l^-1 mod q_i with its Shoup companion).  The words equal
// k_rescale_lift -> NTT -> k_rescale_final.
struct NttFuse {
    const uint64_t* src;
    long long src_stride;
    uint64_t* dst[kFuseMax];   // polynomial p's limbs 0..l-1 at dst[p] (limb stride N)
    const uint64_t* rs;
    int l, L;
};

// ---- phase "col": stages with distance >= 256 ----------------------------------------
template <int LOGN, bool INV, bool FUSE = false, int AR = 0>
__global__ void __launch_bounds__(256, 3) k_ntt_col(LimbMap mp, const ulonglong2* __restrict__ tw2,
                                                  const uint64_t* __restrict__ ninv,
                                                  const __grid_constant__ NttFuse fz) {
    pdl_wait();   // launched by launch_pdl: the previous kernel's writes first
    pdl_trigger();
    constexpr int N = 1 << LOGN;
    constexpr int R = N >> 8;            // rows
    constexpr int TC = 4096 / R;         // columns per tile
    constexpr int G = R / 16;            // row groups (part A stride)
    __shared__ uint64_t sm[4096];
    const int y = blockIdx.y;
    const int poly = y / mp.nl, limb = y % mp.nl;
    if (limb_skipped(mp, poly, limb)) return;
    const int m = mp.mod(limb);
    uint64_t* a = mp.base + (size_t)poly * mp.poly_stride + (size_t)limb * N;
    const uint64_t q = c_mod[m].q;
    const ulonglong2* T2 = tw2 + (size_t)m * N;   // (twiddle, Shoup companion) pairs: one 16-byte load
    const uint64_t pol = tw_policy();
    const int t = threadIdx.x;
    const int c = t % TC, g = t / TC;    // part A: column c, rows g + G*k
    const int col = blockIdx.x * TC + c;
    const int a2 = t / TC;               // part B: rows 16*a2 + k
    uint64_t x[16];
    if (!INV) {
        if (FUSE) {   // centred lift of the dropped limb: v > q_l / 2 stands for v - q_l
            const uint64_t* src = fz.src + (size_t)poly * fz.src_stride;
            const ModConst mi = c_mod[m];
            const uint64_t ql = c_mod[fz.l].q, qlm = reduce64(ql, mi);
#pragma unroll
            for (int k = 0; k < 16; k++) {
                const uint64_t v = src[(size_t)(g + G * k) * 256 + col];
                x[k] = v > (ql >> 1) ? mod_sub(reduce64(v, mi), qlm, q) : reduce64(v, mi);
            }
        } else {
#pragma unroll
            for (int k = 0; k < 16; k++) x[k] = a[(size_t)(g + G * k) * 256 + col];
        }
        // part A: distances R/2 .. R/16 (register distance h = 8,4,2,1); twiddle 2^s + k/(2h)
#pragma unroll
        for (int s = 0; s < 4; s++)
            stage16<false, AR>(x, q, 8 >> s, [&](int j) { return ld_tw(T2 + (1 << s) + j, pol); });
        if (R == 16) {
#pragma unroll
            for (int k = 0; k < 16; k++) a[(size_t)(g + G * k) * 256 + col] = x[k];
            return;
        }
#pragma unroll
        for (int k = 0; k < 16; k++) sm[(g + G * k) * TC + c] = x[k];
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; k++) x[k] = sm[(16 * a2 + k) * TC + c];
        // part B: distances R/32 .. 1 (h = t_r), m_row = R/(2h), twiddle m_row + a2*(8/h) + k/(2h)
#pragma unroll
        for (int h = R / 32; h >= 1; h >>= 1)
            stage16<false, AR>(x, q, h, [&](int j) { return ld_tw(T2 + R / (2 * h) + a2 * (8 / h) + j, pol); });
#pragma unroll
        for (int k = 0; k < 16; k++) a[(size_t)(16 * a2 + k) * 256 + col] = x[k];
    } else {
        if (R == 16) {
#pragma unroll
            for (int k = 0; k < 16; k++) x[k] = a[(size_t)(g + G * k) * 256 + col];
        } else {
#pragma unroll
            for (int k = 0; k < 16; k++) x[k] = a[(size_t)(16 * a2 + k) * 256 + col];
            // inverse part B first: distances 1 .. R/32
#pragma unroll
            for (int h = 1; h <= R / 32; h <<= 1)
                stage16<true, AR>(x, q, h, [&](int j) { return ld_tw(T2 + R / (2 * h) + a2 * (8 / h) + j, pol); });
#pragma unroll
            for (int k = 0; k < 16; k++) sm[(16 * a2 + k) * TC + c] = x[k];
            __syncthreads();
#pragma unroll
            for (int k = 0; k < 16; k++) x[k] = sm[(g + G * k) * TC + c];
        }
#pragma unroll
        for (int s = 3; s >= 0; s--)
            stage16<true, AR>(x, q, 8 >> s, [&](int j) { return ld_tw(T2 + (1 << s) + j, pol); });
        const uint64_t ni = ninv[2 * m], nip = ninv[2 * m + 1];
#pragma unroll
        for (int k = 0; k < 16; k++) a[(size_t)(g + G * k) * 256 + col] = mul_shoup(x[k], ni, nip, q);
    }
}

// ---- phase "row": the last 8 stages, 256-word blocks ---------------------------------------
// Shared memory holds each 256-word block as a 16 x 16 matrix with rows padded to 17 words:
// both the row-wise (fixed row, column = lane) and the column-wise (fixed column, row = lane)
// accesses of a half-warp fall on 16 distinct 8-byte bank pairs, and every access is a
// per-thread base plus an immediate offset.
// Part B (the last four stages) reads its twiddles from the row table `rtab`: for block bg,
// thread r0 and stage sp (distance h = 8 >> sp), twiddle j of the 2^sp the thread needs is
// rtab[bg][2^sp - 1 + j][r0] = Tab[2^(logN-4+sp) + bg * 2^(4+sp) + r0 * 2^sp + j], so a warp's
// load covers consecutive pairs.
constexpr int kRowTab = 240;   // pairs per 256-word block: 16 threads x (1 + 2 + 4 + 8)
template <int LOGN, bool INV, bool FUSE = false, int AR = 0>
__global__ void __launch_bounds__(256, 3) k_ntt_row(LimbMap mp, const ulonglong2* __restrict__ tw2,
                                                  const ulonglong2* __restrict__ rtab,
                                                  const __grid_constant__ NttFuse fz) {
    pdl_wait();   // launched by launch_pdl: the previous kernel's writes first
    pdl_trigger();
    constexpr int N = 1 << LOGN;
    constexpr int S1 = LOGN - 8;
    __shared__ uint64_t sm[16 * 272];
    const int y = blockIdx.y;
    const int poly = y / mp.nl, limb = y % mp.nl;
    if (limb_skipped(mp, poly, limb)) return;
    const int m = mp.mod(limb);
    uint64_t* a = mp.base + (size_t)poly * mp.poly_stride + (size_t)limb * N + (size_t)blockIdx.x * 4096;
    const uint64_t q = c_mod[m].q;
    const ulonglong2* T2 = tw2 + (size_t)m * N;   // (twiddle, Shoup companion) pairs: one 16-byte load
    const uint64_t pol = tw_policy();
    const int t = threadIdx.x;
    const int b = t >> 4, r0 = t & 15;
    const int bg = blockIdx.x * 16 + b;  // global 256-block index
    const ulonglong2* RB = rtab + ((size_t)m * (N >> 8) + bg) * kRowTab + r0;
    uint64_t* sA = sm + b * 272 + r0;        // entry (k, r0) at sA[17 k]
    uint64_t* sB = sm + b * 272 + 17 * r0;   // entry (r0, k) at sB[k]
    uint64_t x[16];
    if (!INV) {
#pragma unroll
        for (int k = 0; k < 16; k++) x[k] = a[b * 256 + r0 + 16 * k];
        // part A: distances 128,64,32,16 (h = 8..1), twiddle 2^(S1+s) + bg*2^s + k/(2h)
#pragma unroll
        for (int s = 0; s < 4; s++)
            stage16<false, AR>(x, q, 8 >> s, [&](int j) { return ld_tw(T2 + (1 << (S1 + s)) + (bg << s) + j, pol); });
#pragma unroll
        for (int k = 0; k < 16; k++) sA[17 * k] = x[k];
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; k++) x[k] = sB[k];
        // part B: distances 8,4,2,1
#pragma unroll
        for (int sp = 0; sp < 4; sp++)
            stage16<false, AR>(x, q, 8 >> sp, [&](int j) { return ld_tw(RB + ((1 << sp) - 1 + j) * 16, pol); });
        // each thread rewrites only the row it read: no barrier before the write
#pragma unroll
        for (int k = 0; k < 16; k++) sB[k] = canon_out<AR>(x[k], q);
        __syncthreads();
        if (FUSE) {   // the rescaled limb in place of the transformed lift
            uint64_t* d = fz.dst[poly] + (size_t)limb * N + (size_t)blockIdx.x * 4096;
            const uint64_t* w = fz.rs + ((size_t)fz.l * fz.L + m) * 2;
            const uint64_t w0 = w[0], w1 = w[1];
#pragma unroll
            for (int k = 0; k < 16; k++) {
                uint64_t* p = d + b * 256 + r0 + 16 * k;
                *p = mul_shoup(mod_sub(*p, sA[17 * k], q), w0, w1, q);
            }
        } else {
#pragma unroll
            for (int k = 0; k < 16; k++) a[b * 256 + r0 + 16 * k] = sA[17 * k];
        }
    } else {
#pragma unroll
        for (int k = 0; k < 16; k++) sA[17 * k] = a[b * 256 + r0 + 16 * k];
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; k++) x[k] = sB[k];
#pragma unroll
        for (int sp = 3; sp >= 0; sp--)
            stage16<true, AR>(x, q, 8 >> sp, [&](int j) { return ld_tw(RB + ((1 << sp) - 1 + j) * 16, pol); });
#pragma unroll
        for (int k = 0; k < 16; k++) sB[k] = x[k];   // own row: no barrier
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; k++) x[k] = sA[17 * k];
#pragma unroll
        for (int s = 3; s >= 0; s--)
            stage16<true, AR>(x, q, 8 >> s, [&](int j) { return ld_tw(T2 + (1 << (S1 + s)) + (bg << s) + j, pol); });
#pragma unroll
        for (int k = 0; k < 16; k++) a[b * 256 + r0 + 16 * k] = x[k];
    }
}

// ---- one launch per transform at N = 2^16: a cluster of 8 CTAs per limb ------------------
// The limb is a 256 x 256 row-major matrix.  CTA k of the cluster (512 threads, 16 words each)
// owns columns [32k, 32k + 32) for the 8 stages with distance >= 256 (column transforms) and rows
// [32k, 32k + 32) for the last 8 (row transforms); between the two the CTAs read each other's
// blocks from shared memory across the cluster (distributed shared memory), so the limb crosses
// HBM once in each direction and the transform is one launch.  Butterflies, twiddle indices and
// value ranges are those of k_ntt_col / k_ntt_row (the words are identical).
//   forward: load columns (layout A: rows g + 16m) -> stages 0-3 -> smem -> layout B (rows
//            16 a2 + k) -> stages 4-7 -> own smem; cluster barrier; read rows from the 8 CTAs
//            (layout C: columns u + 16m) -> cluster barrier -> stages 8-11 -> smem (swizzled) ->
//            layout D (columns 16 j + e) -> stages 12-15 -> smem -> layout C -> store rows.
//   inverse: the same steps in reverse order with the inverse tables, then * N^-1.
// Shared memory: one 80 KB buffer: [256][40] words for the column phase (row stride 40 = 8 mod 16:
// the two rows a warp touches in a cross-CTA read fall on different banks), [32][264] for the row
// phase with the word of column c at c ^ ((c >> 4) & 15) (conflict-free for both layouts).
constexpr int kClC = 8, kClT = 512, kClP1 = 40, kClP2 = 264;
constexpr size_t kClSmem = (size_t)256 * kClP1 * 8;   // >= 32 * kClP2 * 8

__device__ __forceinline__ void cl_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint64_t cl_ld(uint32_t laddr, uint32_t rank) {
    uint32_t ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(laddr), "r"(rank));
    uint64_t v;
    asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(ra) : "memory");
    return v;
}
__device__ __forceinline__ int cl_swz(int c) { return c ^ ((c >> 4) & 15); }

template <bool INV>
__global__ void __cluster_dims__(kClC, 1, 1) __launch_bounds__(kClT, 1)
    k_ntt_cluster(LimbMap mp, const ulonglong2* __restrict__ tw2, const ulonglong2* __restrict__ rtab,
                  const uint64_t* __restrict__ ninv) {
    pdl_wait();   // launched by launch_pdl: the previous kernel's writes first
    pdl_trigger();
    constexpr int N = 1 << 16;
    extern __shared__ __align__(16) uint64_t cs[];
    const int y = blockIdx.y;
    const int poly = y / mp.nl, limb = y % mp.nl;
    if (limb_skipped(mp, poly, limb)) return;   // uniform over the cluster: no barrier is reached
    const int m = mp.mod(limb);
    uint64_t* a = mp.base + (size_t)poly * mp.poly_stride + (size_t)limb * N;
    const uint64_t q = c_mod[m].q;
    const ulonglong2* T2 = tw2 + (size_t)m * N;
    const uint64_t pol = tw_policy();
    const int k = blockIdx.x;                    // rank in the cluster
    const int t = threadIdx.x;
    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(cs);
    // layout A / B (column phase): column 32k + cc
    const int cc = t & 31, g = t >> 5;           // A: rows g + 16 mm; B: rows 16 g + kk
    // layout C / D (row phase): row 32k + rr
    const int rr = t >> 4, u = t & 15;           // C: columns u + 16 mm; D: columns 16 u + e
    const int r = 32 * k + rr;
    const ulonglong2* RB = rtab + ((size_t)m * (N >> 8) + r) * kRowTab + u;
    uint64_t x[16];
    if (!INV) {
#pragma unroll
        for (int i = 0; i < 16; i++) x[i] = a[(size_t)(g + 16 * i) * 256 + 32 * k + cc];
#pragma unroll
        for (int s = 0; s < 4; s++)
            stage16<false>(x, q, 8 >> s, [&](int j) { return ld_tw(T2 + (1 << s) + j, pol); });
#pragma unroll
        for (int i = 0; i < 16; i++) cs[(g + 16 * i) * kClP1 + cc] = x[i];
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 16; i++) x[i] = cs[(16 * g + i) * kClP1 + cc];
#pragma unroll
        for (int h = 8, s = 4; h >= 1; h >>= 1, s++)
            stage16<false>(x, q, h, [&](int j) { return ld_tw(T2 + (1 << s) + g * (8 / h) + j, pol); });
#pragma unroll
        for (int i = 0; i < 16; i++) cs[(16 * g + i) * kClP1 + cc] = x[i];   // own rows only: no barrier
        cl_sync();
        // row r, columns u + 16 i: CTA i >> 1 holds them at [r][u + 16 (i & 1)]
#pragma unroll
        for (int i = 0; i < 16; i++)
            x[i] = cl_ld(sbase + (uint32_t)((r * kClP1 + u + 16 * (i & 1)) * 8), (uint32_t)(i >> 1));
        cl_sync();   // every CTA has read what it needs: the buffer is free
#pragma unroll
        for (int s = 0; s < 4; s++)
            stage16<false>(x, q, 8 >> s, [&](int j) { return ld_tw(T2 + (1 << (8 + s)) + (r << s) + j, pol); });
#pragma unroll
        for (int i = 0; i < 16; i++) cs[rr * kClP2 + cl_swz(u + 16 * i)] = x[i];
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 16; i++) x[i] = cs[rr * kClP2 + cl_swz(16 * u + i)];
#pragma unroll
        for (int sp = 0; sp < 4; sp++)
            stage16<false>(x, q, 8 >> sp, [&](int j) { return ld_tw(RB + ((1 << sp) - 1 + j) * 16, pol); });
#pragma unroll
        for (int i = 0; i < 16; i++) cs[rr * kClP2 + cl_swz(16 * u + i)] = canon4(x[i], q);   // own words
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 16; i++) a[(size_t)r * 256 + u + 16 * i] = cs[rr * kClP2 + cl_swz(u + 16 * i)];
    } else {
#pragma unroll
        for (int i = 0; i < 16; i++) cs[rr * kClP2 + cl_swz(u + 16 * i)] = a[(size_t)r * 256 + u + 16 * i];
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 16; i++) x[i] = cs[rr * kClP2 + cl_swz(16 * u + i)];
#pragma unroll
        for (int sp = 3; sp >= 0; sp--)
            stage16<true>(x, q, 8 >> sp, [&](int j) { return ld_tw(RB + ((1 << sp) - 1 + j) * 16, pol); });
#pragma unroll
        for (int i = 0; i < 16; i++) cs[rr * kClP2 + cl_swz(16 * u + i)] = x[i];   // own words
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 16; i++) x[i] = cs[rr * kClP2 + cl_swz(u + 16 * i)];
#pragma unroll
        for (int s = 3; s >= 0; s--)
            stage16<true>(x, q, 8 >> s, [&](int j) { return ld_tw(T2 + (1 << (8 + s)) + (r << s) + j, pol); });
        // the row block as [32][264] (unswizzled) for the other CTAs' column reads
        __syncthreads();   // every thread is done reading the swizzled block
#pragma unroll
        for (int i = 0; i < 16; i++) cs[rr * kClP2 + u + 16 * i] = x[i];
        cl_sync();
        // column 32k + cc, rows 16 g + i: CTA g >> 1 holds them at [(16 g + i) & 31][32k + cc]
#pragma unroll
        for (int i = 0; i < 16; i++)
            x[i] = cl_ld(sbase + (uint32_t)((((16 * g + i) & 31) * kClP2 + 32 * k + cc) * 8), (uint32_t)(g >> 1));
        cl_sync();
#pragma unroll
        for (int h = 1, s = 7; h <= 8; h <<= 1, s--)
            stage16<true>(x, q, h, [&](int j) { return ld_tw(T2 + (1 << s) + g * (8 / h) + j, pol); });
#pragma unroll
        for (int i = 0; i < 16; i++) cs[(16 * g + i) * kClP1 + cc] = x[i];
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 16; i++) x[i] = cs[(g + 16 * i) * kClP1 + cc];
#pragma unroll
        for (int s = 3; s >= 0; s--)
            stage16<true>(x, q, 8 >> s, [&](int j) { return ld_tw(T2 + (1 << s) + j, pol); });
        const uint64_t ni = ninv[2 * m], nip = ninv[2 * m + 1];
#pragma unroll
        for (int i = 0; i < 16; i++) a[(size_t)(g + 16 * i) * 256 + 32 * k + cc] = mul_shoup(x[i], ni, nip, q);
    }
}

static void launch_ntt_cluster(const Context& cx, const LimbMap& mp, int count, bool inv, cudaStream_t st) {
    auto kern = inv ? k_ntt_cluster<true> : k_ntt_cluster<false>;
    static bool attr_set[2] = {false, false};
    if (!attr_set[inv ? 1 : 0]) {
        CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kClSmem));
        attr_set[inv ? 1 : 0] = true;
    }
    if (inv)
        launch_pdl(cx, k_ntt_cluster<true>, dim3(kClC, count), dim3(kClT), kClSmem, st, mp,
                   (const ulonglong2*)cx.d_itw2, (const ulonglong2*)cx.d_itwrow, cx.d_ninv);
    else
        launch_pdl(cx, k_ntt_cluster<false>, dim3(kClC, count), dim3(kClT), kClSmem, st, mp,
                   (const ulonglong2*)cx.d_tw2, (const ulonglong2*)cx.d_twrow, cx.d_ninv);
}

template <int LOGN, int AR>
static void launch_ntt_ar(const Context& cx, const LimbMap& mp, int count, bool inv, cudaStream_t st) {
    constexpr int N = 1 << LOGN;
    constexpr int R = N >> 8;
    dim3 gcol(R / 16, count), grow(N / 4096, count);
    if (!inv) {
        launch_pdl(cx, k_ntt_col<LOGN, false, false, AR>, gcol, dim3(256), 0, st, mp, (const ulonglong2*)cx.d_tw2,
                   cx.d_ninv, NttFuse{});
        launch_pdl(cx, k_ntt_row<LOGN, false, false, AR>, grow, dim3(256), 0, st, mp, (const ulonglong2*)cx.d_tw2,
                   (const ulonglong2*)cx.d_twrow, NttFuse{});
    } else {
        launch_pdl(cx, k_ntt_row<LOGN, true, false, AR>, grow, dim3(256), 0, st, mp, (const ulonglong2*)cx.d_itw2,
                   (const ulonglong2*)cx.d_itwrow, NttFuse{});
        launch_pdl(cx, k_ntt_col<LOGN, true, false, AR>, gcol, dim3(256), 0, st, mp, (const ulonglong2*)cx.d_itw2,
                   cx.d_ninv, NttFuse{});
    }
}
template <int LOGN>
static void launch_ntt(const Context& cx, const LimbMap& mp, int count, bool inv, cudaStream_t st) {
    if (cx.ntt_arith == 1) launch_ntt_ar<LOGN, 1>(cx, mp, count, inv, st);
    else launch_ntt_ar<LOGN, 0>(cx, mp, count, inv, st);
}

void ntt(const Context& cx, const LimbMap& mp, int npoly, bool inv, cudaStream_t st) {
    const int count = npoly * mp.nl;
    if (count == 0) return;
    int work = count;   // limb-polynomials actually transformed (ModUp skips its own digit)
    if (mp.skip_alpha)
        for (int p = 0; p < npoly; p++) {
            const int dg = mp.skip_period > 0 ? p % mp.skip_period : p;
            work -= std::max(0, std::min(mp.skip_alpha, mp.skip_nq - dg * mp.skip_alpha));
        }
    // the launch's batch size class as an inclusive "op:" entry (where the transforms' time goes)
    static const char* kCls[2][3] = {{"op:ntt_fwd_le16", "op:ntt_fwd_le64", "op:ntt_fwd_gt64"},
                                     {"op:ntt_inv_le16", "op:ntt_inv_le64", "op:ntt_inv_gt64"}};
    ProfScope pc(cx, kCls[inv ? 1 : 0][work <= 16 ? 0 : work <= 64 ? 1 : 2], 16.0 * cx.N * work);
    ProfScope ps(cx, inv ? "ntt_inv" : "ntt_fwd", 16.0 * cx.N * work);
    switch (cx.logN) {
        case 12: launch_ntt<12>(cx, mp, count, inv, st); break;
        case 13: launch_ntt<13>(cx, mp, count, inv, st); break;
        case 14: launch_ntt<14>(cx, mp, count, inv, st); break;
        case 15: launch_ntt<15>(cx, mp, count, inv, st); break;
        case 16:
            if (cx.ntt_cluster) {
                launch_ntt_cluster(cx, mp, count, inv, st);
                CUDA_CHECK(cudaGetLastError());
                cx.launches += 1;
                return;
            }
            launch_ntt<16>(cx, mp, count, inv, st);
            break;
        default: throw Error("ntt: logN must be in [12, 16]");
    }
    CUDA_CHECK(cudaGetLastError());
    cx.launches += 2;
}

template <int LOGN, int AR>
static void launch_ntt_rescale_ar(const Context& cx, const LimbMap& mp, int count, const NttFuse& fz,
                                  cudaStream_t st) {
    constexpr int N = 1 << LOGN;
    constexpr int R = N >> 8;
    launch_pdl(cx, k_ntt_col<LOGN, false, true, AR>, dim3(R / 16, count), dim3(256), 0, st, mp,
               (const ulonglong2*)cx.d_tw2, cx.d_ninv, fz);
    launch_pdl(cx, k_ntt_row<LOGN, false, true, AR>, dim3(N / 4096, count), dim3(256), 0, st, mp,
               (const ulonglong2*)cx.d_tw2, (const ulonglong2*)cx.d_twrow, fz);
}
template <int LOGN>
static void launch_ntt_rescale(const Context& cx, const LimbMap& mp, int count, const NttFuse& fz, cudaStream_t st) {
    if (cx.ntt_arith == 1) launch_ntt_rescale_ar<LOGN, 1>(cx, mp, count, fz, st);
    else launch_ntt_rescale_ar<LOGN, 0>(cx, mp, count, fz, st);
}

// The rescale of npoly polynomials with l + 1 limbs each (npoly <= kFuseMax), past the inverse
// transform of their dropped limbs (coefficient form, polynomial p's at src + p * src_stride):
// the limbs 0..l-1 at dst[p] become (a_i - lift_i(a_l)) q_l^-1, the lifts' transforms held in y
// ([npoly][l][N] scratch).  Two launches instead of lift, transform and final.
void ntt_rescale_n(const Context& cx, const uint64_t* src, long long src_stride, uint64_t* const* dst, int npoly,
                   int l, uint64_t* y, cudaStream_t st) {
    if (cx.logN < 13) throw Error("ntt_rescale: logN must be >= 13", -1);
    if (npoly < 1 || npoly > kFuseMax) throw Error("ntt_rescale: 1 to 16 polynomials", -1);
    LimbMap mp = cx.qmap(y, l, (long long)l * cx.N);
    NttFuse fz{};
    fz.src = src;
    fz.src_stride = src_stride;
    for (int p = 0; p < npoly; p++) fz.dst[p] = dst[p];
    fz.rs = cx.d_rs;
    fz.l = l;
    fz.L = cx.L;
    switch (cx.logN) {
        case 13: launch_ntt_rescale<13>(cx, mp, npoly * l, fz, st); break;
        case 14: launch_ntt_rescale<14>(cx, mp, npoly * l, fz, st); break;
        case 15: launch_ntt_rescale<15>(cx, mp, npoly * l, fz, st); break;
        case 16: launch_ntt_rescale<16>(cx, mp, npoly * l, fz, st); break;
        default: throw Error("ntt_rescale: logN must be in [13, 16]");
    }
    CUDA_CHECK(cudaGetLastError());
    cx.launches += 2;
}
// one ciphertext: the dropped limb transformed in place (a + l N, poly stride `stride`)
void ntt_rescale(const Context& cx, uint64_t* a, long long stride, int l, uint64_t* y, cudaStream_t st) {
    uint64_t* dst[2] = {a, a + stride};
    ntt_rescale_n(cx, a + (size_t)l * cx.N, stride, dst, 2, l, y, st);
}

}  // namespace fhe
