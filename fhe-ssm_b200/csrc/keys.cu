// keys.cu -- the seeded uniform expander on the device.
//
// A key's a-half (and the public key's a) is a stream of words uniform mod q drawn from a
// ChaCha20 keystream: the reference's normative expander (hpc_gpu_port/seeded_keys.hpp:23-43,
// :80-134): key = the 32-byte seed as 8 little-endian words, nonce = {digit, limb, tag},
// counter 0, 1, 2, ..., the 16 output words of a block read as little-endian 64-bit words, and
// rejection of w >= 2^64 - (2^64 mod q).  The host restatement is sampling.h; this kernel
// produces the same words on the GPU, so keys are expanded where they are used (key
// generation, and loading seeded part files whose a-halves travel as 32-byte seeds).
//
// Parallel form of a sequential rejection sampler: one CTA owns one (digit, limb) stream.  In a
// round, thread t expands blocks base + 8t .. base + 8t + 7 (64 consecutive stream words), counts
// the words it accepts, and a block-wide exclusive scan of the counts gives each thread the
// output position of its first accepted word; accepted words keep their stream order.  Rounds
// continue until N words are placed (the rejection rate is below 1/16 for the 60-bit moduli, so a
// limb of 2^16 words takes 5 rounds of 16,384 words); a stream that would need more than
// kExpandMaxRounds rounds (never, for an odd modulus above 2^32) raises the context's error flag.
#include "engine.h"

namespace fhe {

constexpr int kExpandThreads = 256;
constexpr int kExpandBlocksPerThread = 8;   // 64 words per thread per round
constexpr int kExpandMaxRounds = 64;

__device__ __forceinline__ uint32_t cc_rotl(uint32_t v, int c) { return __funnelshift_l(v, v, c); }
__device__ __forceinline__ void cc_qr(uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
    a += b; d ^= a; d = cc_rotl(d, 16);
    c += d; b ^= c; b = cc_rotl(b, 12);
    a += b; d ^= a; d = cc_rotl(d, 8);
    c += d; b ^= c; b = cc_rotl(b, 7);
}
// RFC 8439 section 2.3: 20 rounds (10 double rounds), then the input state added back
__device__ __forceinline__ void cc_block(const uint32_t (&k)[8], uint32_t ctr, uint32_t n0, uint32_t n1, uint32_t n2,
                                         uint32_t (&x)[16]) {
    const uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u, k[0], k[1], k[2], k[3],
                            k[4], k[5], k[6], k[7], ctr, n0, n1, n2};
#pragma unroll
    for (int i = 0; i < 16; i++) x[i] = s[i];
#pragma unroll 1
    for (int r = 0; r < 10; r++) {
        cc_qr(x[0], x[4], x[8], x[12]); cc_qr(x[1], x[5], x[9], x[13]);
        cc_qr(x[2], x[6], x[10], x[14]); cc_qr(x[3], x[7], x[11], x[15]);
        cc_qr(x[0], x[5], x[10], x[15]); cc_qr(x[1], x[6], x[11], x[12]);
        cc_qr(x[2], x[7], x[8], x[13]); cc_qr(x[3], x[4], x[9], x[14]);
    }
#pragma unroll
    for (int i = 0; i < 16; i++) x[i] += s[i];
}

struct ExpandArgs {
    uint32_t key[8];        // the seed as 8 little-endian words
    uint32_t tag;           // third nonce word
    int digit0;             // first nonce word = digit0 + blockIdx.y
    int limb0;              // second nonce word and modulus index = limb0 + blockIdx.x (Q then P chain)
    long long digit_stride; // words between the outputs of consecutive digits
    int logN;
};

// out + blockIdx.y * digit_stride + blockIdx.x * N: N words uniform mod q(limb0 + blockIdx.x),
// canonical; rmont[2 m] = 2^64 mod q_m gives the rejection bound
__global__ void __launch_bounds__(kExpandThreads) k_expand_uniform(const ExpandArgs a, uint64_t* __restrict__ out,
                                                                    const uint64_t* __restrict__ rmont,
                                                                    unsigned int* err) {
    __shared__ uint32_t warp_tot[kExpandThreads / 32];
    __shared__ uint32_t s_filled;
    const int N = 1 << a.logN;
    const int m = a.limb0 + blockIdx.x;
    const uint32_t digit = (uint32_t)(a.digit0 + blockIdx.y);
    const ModConst mc = c_mod[m];
    const uint64_t r = rmont[2 * m];            // 2^64 mod q
    const uint64_t lim = 0 - r;                  // q * floor(2^64 / q); every word is accepted when r == 0
    uint64_t* o = out + (size_t)blockIdx.y * a.digit_stride + (size_t)blockIdx.x * N;
    uint32_t key[8];
#pragma unroll
    for (int i = 0; i < 8; i++) key[i] = a.key[i];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) s_filled = 0;
    __syncthreads();
    for (int round = 0; round < kExpandMaxRounds; round++) {
        const uint32_t filled = s_filled;
        if (filled >= (uint32_t)N) return;
        const uint32_t ctr0 = (uint32_t)(round * kExpandThreads + tid) * kExpandBlocksPerThread;
        // pass 1: how many of this thread's 64 words are accepted
        uint32_t cnt = 0;
        for (int b = 0; b < kExpandBlocksPerThread; b++) {
            uint32_t x[16];
            cc_block(key, ctr0 + b, (uint32_t)digit, (uint32_t)m, a.tag, x);
#pragma unroll
            for (int w = 0; w < 8; w++) {
                const uint64_t v = (uint64_t)x[2 * w] | ((uint64_t)x[2 * w + 1] << 32);
                cnt += (r == 0 || v < lim) ? 1u : 0u;
            }
        }
        // block-wide exclusive scan of the counts
        uint32_t inc = cnt;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, inc, d);
            if (lane >= d) inc += t;
        }
        if (lane == 31) warp_tot[warp] = inc;
        __syncthreads();
        uint32_t before = 0, total = 0;
        for (int w2 = 0; w2 < kExpandThreads / 32; w2++) {
            if (w2 < warp) before += warp_tot[w2];
            total += warp_tot[w2];
        }
        uint32_t pos = filled + before + inc - cnt;
        // pass 2: regenerate the same blocks and place the accepted words in stream order
        if (pos < (uint32_t)N) {
            for (int b = 0; b < kExpandBlocksPerThread && pos < (uint32_t)N; b++) {
                uint32_t x[16];
                cc_block(key, ctr0 + b, (uint32_t)digit, (uint32_t)m, a.tag, x);
#pragma unroll
                for (int w = 0; w < 8; w++) {
                    const uint64_t v = (uint64_t)x[2 * w] | ((uint64_t)x[2 * w + 1] << 32);
                    if ((r == 0 || v < lim) && pos < (uint32_t)N) {
                        o[pos] = mc.k > 32 ? reduce64(v, mc) : v % mc.q;
                        pos++;
                    }
                }
            }
        }
        __syncthreads();   // every thread has read warp_tot and s_filled
        if (tid == 0) s_filled = filled + total;
        __syncthreads();
    }
    if (tid == 0 && s_filled < (uint32_t)N) atomicExch(err, 2u);
}

// Words of the streams {digit0 + j, limb0 + i, tag} of `seed` for j < ndigit, i < nlimb, each N
// words uniform mod q(limb0 + i), written to out + j * digit_stride + i * N (device memory),
// enqueued on the context's stream.
void expand_uniform_dev(Context& cx, const uint8_t seed[32], int digit0, int ndigit, int limb0, int nlimb,
                        uint32_t tag, uint64_t* out, long long digit_stride) {
    if (nlimb < 1 || ndigit < 1 || limb0 < 0 || limb0 + nlimb > cx.L + cx.K)
        throw Error("expand_uniform: limb range outside the chain", -1);
    ExpandArgs a{};
    for (int k = 0; k < 8; k++)
        a.key[k] = (uint32_t)seed[4 * k] | ((uint32_t)seed[4 * k + 1] << 8) | ((uint32_t)seed[4 * k + 2] << 16) |
                   ((uint32_t)seed[4 * k + 3] << 24);
    a.tag = tag;
    a.digit0 = digit0;
    a.limb0 = limb0;
    a.digit_stride = digit_stride;
    a.logN = cx.logN;
    k_expand_uniform<<<dim3(nlimb, ndigit), kExpandThreads, 0, cx.stream>>>(a, out, cx.d_rmont, cx.d_err);
    CUDA_CHECK(cudaGetLastError());
    cx.launches++;
}

}  // namespace fhe
