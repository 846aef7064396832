// Router top-k, token permutation into ragged per-expert groups, the gather
// of permuted activation rows and the weighted unpermute/combine.
//
// Routing is bit-exact with the reference CPU path:
//   logits   moe_dot_bf16_row (raw_forward_utils.cpp.inc:174-216): per
//            (token, expert) 16 FMA chains over i = l, l+16, ..., lane sums
//            b_l = s_l + s_{l+8}, then ((b0+b1)+b2)+...+b7;
//   softmax  generation_router.cpp.inc:606-622: exp in double, denominator
//            summed in double in expert order, p *= (float)(1/denom);
//   sigmoid  :239-245, 1/(1+expf(-l)) in float, expf being the host C
//            library's (libm_expf below reproduces it bit for bit);
//   top-k    :640-674, k largest scores descending (equal scores: lower
//            expert index first), optional renormalisation and scaling.
// The permutation is the order of moe_pc_group_tokens_by_expert
// (token_grouping.cpp.inc:47-55): sorted by expert, then token index.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace moe_b200 {

// ---------------------------------------------------------------------------
// Router logits for large batches.  A block computes a 32-token x 64-expert
// tile.  The reference accumulates each dot product in 16 FMA chains (chain l
// takes elements l, l+16, ...).  Here lane l of a 16-lane half-warp runs chain
// l for 16 tokens x 8 experts (128 independent chains), two tokens at a time
// with packed fp32 FMAs (fma.rn.f32x2, each half an IEEE fp32 FMA).  Per 16
// elements a lane does 24 four-byte shared loads for 128 FMAs; the two
// half-warps read the same token rows (one broadcast wavefront) and adjacent
// router rows whose fp32 row stride is 16 words past a multiple of 32 (disjoint
// banks, one wavefront): 0.19 wavefronts per FMA, under the shared-memory
// pipe's 0.25 at the FMA peak.  The chains read an fp32 copy of each
// 128-element chunk of the rows, so the FMA loop does no conversions.  At the
// end each lane's chain sums go through shared memory so that one lane holds
// all 16 chains of a dot, which it combines exactly as the reference does:
// b_l = s_l + s_{l+8}, then ((b0+b1)+b2)+...+b7, then the 4-way and scalar
// tails (H % 16 != 0).
//
// router_logits_tma_kernel (16-byte aligned rows) specialises warps: one
// lane brings each chunk's token and router rows in with two TMA copies into
// a 3-deep bf16 ring, two warps convert ring entries into a 2-deep fp32 ring,
// eight warps run the FMA chains; mbarriers hand the buffers along, so
// copies, conversion and FMAs of different chunks overlap.
// router_logits_kernel (rows only 8-byte aligned) stages with 8-byte
// cp.async and converts in lockstep with the FMAs.
// ---------------------------------------------------------------------------
constexpr int kRtTok = 32, kRtExp = 64;          // block tile
constexpr int kRtK = 128;                        // elements per chunk (multiple of 16)
constexpr int kRtS = kRtK + 16;                  // fp32 row stride in words (== 16 mod 32)
constexpr int kRtRows = kRtTok + kRtExp;
constexpr int kRtRing = 3;                       // bf16 chunk buffers
constexpr int kRtF32Ring = 2;                    // fp32 chunk buffers (TMA kernel)
constexpr size_t kRtF32Bytes = (size_t)kRtRows * kRtS * 4;
constexpr size_t kRtRawBytes = (size_t)kRtRows * kRtK * 2;
constexpr int kRtDots = 256;                     // dots per warp (16 tokens x 16 experts)
constexpr int kRtScratch = kRtDots * 17 + 16;    // floats of a warp's transpose area
constexpr size_t kRtScratchBytes = 8ull * kRtScratch * 4;
constexpr size_t kRtSmem = std::max(kRtF32Bytes + kRtRing * kRtRawBytes, kRtScratchBytes);
constexpr size_t kRtTmaRings = kRtF32Ring * kRtF32Bytes + kRtRing * kRtRawBytes;
static_assert(kRtScratchBytes <= kRtTmaRings, "transpose area inside the rings");
constexpr size_t kRtTmaSmem = kRtTmaRings + 128;
constexpr int kRtFmaWarps = 8, kRtCvtWarps = 2;
constexpr int kRtTmaThreads = 32 * (kRtFmaWarps + kRtCvtWarps + 1);

__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ unsigned long long pack_f32x2(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
// d.lo += a.lo * b.lo, d.hi += a.hi * b.hi, each rounded once (IEEE fp32 FMA)
__device__ __forceinline__ void fma_f32x2(unsigned long long& d, unsigned long long a, unsigned long long b) {
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(d) : "l"(a), "l"(b));
}

// 8 bf16 of raw row r, column group v -> fp32 row r of `fs`
__device__ __forceinline__ void rt_convert8(const uint16_t* raw, float* fs, uint32_t r, uint32_t v) {
    const uint4 u = *reinterpret_cast<const uint4*>(raw + (size_t)r * kRtK + v * 8);
    float4 lo, hi;
    lo.x = __uint_as_float(u.x << 16); lo.y = __uint_as_float(u.x & 0xffff0000u);
    lo.z = __uint_as_float(u.y << 16); lo.w = __uint_as_float(u.y & 0xffff0000u);
    hi.x = __uint_as_float(u.z << 16); hi.y = __uint_as_float(u.z & 0xffff0000u);
    hi.z = __uint_as_float(u.w << 16); hi.w = __uint_as_float(u.w & 0xffff0000u);
    float4* d = reinterpret_cast<float4*>(fs + (size_t)r * kRtS + v * 8);
    d[0] = lo;
    d[1] = hi;
}

// One FMA warp's share of the block tile: tokens tg*16 + a (a < 16), experts
// eg*16 + 2j + p (j < 8) for half-warp p, chain l = lane % 16.
struct RtLane {
    int l, p, tg, eg;
    unsigned long long acc[8][8];  // [token pair i][expert j]: lo token 2i, hi token 2i+1
    __device__ __forceinline__ RtLane(int warp, int lane) {
        l = lane & 15;
        p = lane >> 4;
        tg = warp & 1;
        eg = warp >> 1;
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[i][j] = 0ull;
    }
    // the 16-element steps of one chunk of the fp32 tile `fs`
    __device__ __forceinline__ void chunk(const float* fs, uint32_t clen) {
        const float* xp = fs + (size_t)(tg * 16) * kRtS + l;
        const float* wp = fs + (size_t)(kRtTok + eg * 16 + p) * kRtS + l;
#pragma unroll 1
        for (uint32_t k = 0; k < clen; k += 16) {
            unsigned long long wd[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float wv = wp[(size_t)(2 * j) * kRtS + k];
                wd[j] = pack_f32x2(wv, wv);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const unsigned long long xv = pack_f32x2(xp[(size_t)(2 * i) * kRtS + k], xp[(size_t)(2 * i + 1) * kRtS + k]);
#pragma unroll
                for (int j = 0; j < 8; ++j) fma_f32x2(acc[i][j], xv, wd[j]);
            }
        }
    }
    // `sc`: this warp's transpose area (kRtScratch floats), free for its use.
    __device__ __forceinline__ void finish(float* sc, const uint16_t* __restrict__ x,
                                           const uint16_t* __restrict__ w, uint32_t t0, uint32_t e0, uint32_t T,
                                           uint32_t E, uint32_t H, float* __restrict__ logits) {
        // dot d = p*128 + a*8 + j keeps its 16 chain sums at d*17 + (d/128)*16
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int d0 = p * 128 + (2 * i) * 8 + j;
                sc[d0 * 17 + p * 16 + l] = __uint_as_float((uint32_t)acc[i][j]);
                sc[(d0 + 8) * 17 + p * 16 + l] = __uint_as_float((uint32_t)(acc[i][j] >> 32));
            }
        __syncwarp();
        const int lane = threadIdx.x & 31;
        const uint32_t main_end = H & ~15u;
#pragma unroll 1
        for (int m = 0; m < kRtDots / 32; ++m) {
            const int d = lane + 32 * m;
            const int dp = d >> 7, a = (d & 127) >> 3, j = d & 7;
            const float* s = sc + d * 17 + dp * 16;
            float sum = __fadd_rn(s[0], s[8]);
#pragma unroll
            for (int c = 1; c < 8; ++c) sum = __fadd_rn(sum, __fadd_rn(s[c], s[c + 8]));
            const uint32_t tt = t0 + tg * 16 + a, e = e0 + eg * 16 + 2 * j + dp;
            if (tt < T && e < E) {
                float out = 0.0f + sum;
                if (main_end < H) {
                    const uint16_t* wr = w + (uint64_t)e * H;
                    const uint16_t* xr = x + (uint64_t)tt * H;
                    uint32_t i = main_end;
                    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
                    for (; i + 3 < H; i += 4) {
                        a0 = __fmaf_rn(bf16_bits_to_f32(wr[i]), bf16_bits_to_f32(xr[i]), a0);
                        a1 = __fmaf_rn(bf16_bits_to_f32(wr[i + 1]), bf16_bits_to_f32(xr[i + 1]), a1);
                        a2 = __fmaf_rn(bf16_bits_to_f32(wr[i + 2]), bf16_bits_to_f32(xr[i + 2]), a2);
                        a3 = __fmaf_rn(bf16_bits_to_f32(wr[i + 3]), bf16_bits_to_f32(xr[i + 3]), a3);
                    }
                    out = __fadd_rn(out, __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3)));
                    for (; i < H; ++i) out = __fmaf_rn(bf16_bits_to_f32(wr[i]), bf16_bits_to_f32(xr[i]), out);
                }
                logits[(uint64_t)tt * E + e] = out;
            }
        }
    }
};

__global__ void __launch_bounds__(kRtTmaThreads, 1)
    router_logits_tma_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                             const uint16_t* __restrict__ x, const uint16_t* __restrict__ w, uint32_t T, uint32_t E,
                             uint32_t H, float* __restrict__ logits, uint32_t* err) {
    extern __shared__ __align__(128) unsigned char rt_smem[];
    float* fs = reinterpret_cast<float*>(rt_smem);                                       // [kRtF32Ring][rows][kRtS]
    uint16_t* raw = reinterpret_cast<uint16_t*>(rt_smem + kRtF32Ring * kRtF32Bytes);      // [kRtRing][rows][kRtK]
    uint64_t* bars = reinterpret_cast<uint64_t*>(rt_smem + kRtTmaRings);
    uint64_t* raw_full = bars;                      // TMA bytes landed
    uint64_t* raw_empty = bars + kRtRing;           // converters done reading
    uint64_t* f32_full = bars + 2 * kRtRing;        // converters done writing
    uint64_t* f32_empty = bars + 2 * kRtRing + kRtF32Ring;  // FMA warps done reading
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t e0 = blockIdx.x * kRtExp, t0 = blockIdx.y * kRtTok;
    const uint32_t main_end = H & ~15u;
    const uint32_t nchunks = (main_end + kRtK - 1) / kRtK;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRtRing; ++i) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], kRtCvtWarps);
        }
        for (int i = 0; i < kRtF32Ring; ++i) {
            mbar_init(&f32_full[i], kRtCvtWarps);
            mbar_init(&f32_empty[i], kRtFmaWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp < kRtFmaWarps) {
        RtLane ln(warp, lane);
        for (uint32_t c = 0; c < nchunks; ++c) {
            const uint32_t s = c % kRtF32Ring;
            mbar_wait(&f32_full[s], (c / kRtF32Ring) & 1, err, kErrTimeoutRouterLoad);
            ln.chunk(fs + (size_t)s * kRtRows * kRtS, min((uint32_t)kRtK, main_end - c * kRtK));
            __syncwarp();
            if (lane == 0) mbar_arrive(&f32_empty[s]);
        }
        // every FMA warp is past its last chunk; the converters and the
        // producer finished before the last chunk could be read, so both
        // rings are free for the transpose
        asm volatile("bar.sync 1, %0;" ::"n"(32 * kRtFmaWarps) : "memory");
        ln.finish(reinterpret_cast<float*>(rt_smem) + (size_t)warp * kRtScratch, x, w, t0, e0, T, E, H, logits);
    } else if (warp < kRtFmaWarps + kRtCvtWarps) {
        const uint32_t ct = threadIdx.x - 32 * kRtFmaWarps;  // 0..63
        constexpr int kVpr = kRtK / 8, kPer = kRtRows * kVpr / (32 * kRtCvtWarps);
        static_assert(kRtRows * kVpr % (32 * kRtCvtWarps) == 0, "whole conversion rounds");
        for (uint32_t c = 0; c < nchunks; ++c) {
            const uint32_t rs = c % kRtRing, s = c % kRtF32Ring;
            mbar_wait(&raw_full[rs], (c / kRtRing) & 1, err, kErrTimeoutRouterLoad);
            mbar_wait(&f32_empty[s], ((c / kRtF32Ring) & 1) ^ 1, err, kErrTimeoutRouterLoad);
            const uint16_t* src = raw + (size_t)rs * kRtRows * kRtK;
            float* dst = fs + (size_t)s * kRtRows * kRtS;
#pragma unroll 8
            for (int j = 0; j < kPer; ++j) {
                const uint32_t i = ct + 32u * kRtCvtWarps * j;
                rt_convert8(src, dst, i / kVpr, i % kVpr);
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&f32_full[s]);
                mbar_arrive(&raw_empty[rs]);
            }
        }
    } else if (lane == 0) {  // producer
        for (uint32_t c = 0; c < nchunks; ++c) {
            const uint32_t rs = c % kRtRing;
            mbar_wait(&raw_empty[rs], ((c / kRtRing) & 1) ^ 1, err, kErrTimeoutRouterLoad, true);
            mbar_arrive_expect_tx(&raw_full[rs], (uint32_t)kRtRawBytes);
            uint16_t* dst = raw + (size_t)rs * kRtRows * kRtK;
            tma_load_2d(dst, &tmap_x, (int32_t)(c * kRtK), (int32_t)t0, &raw_full[rs]);
            tma_load_2d(dst + (size_t)kRtTok * kRtK, &tmap_w, (int32_t)(c * kRtK), (int32_t)e0, &raw_full[rs]);
        }
    }
}

__global__ void __launch_bounds__(256, 1) router_logits_kernel(const uint16_t* __restrict__ x,
                                                               const uint16_t* __restrict__ w, uint32_t T,
                                                               uint32_t E, uint32_t H, float* __restrict__ logits) {
    extern __shared__ __align__(128) unsigned char rt_smem[];
    float* fs = reinterpret_cast<float*>(rt_smem);                        // [rows][kRtS]
    uint16_t* raw = reinterpret_cast<uint16_t*>(rt_smem + kRtF32Bytes);  // [kRtRing][rows][kRtK]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t e0 = blockIdx.x * kRtExp, t0 = blockIdx.y * kRtTok;
    const uint32_t main_end = H & ~15u;
    const uint32_t nchunks = (main_end + kRtK - 1) / kRtK;

    // Row r of the tile: a token row (r < kRtTok) or a router row; rows past
    // T or E repeat the last one (their dots are computed and not stored).
    auto row_ptr = [&](uint32_t r) -> const uint16_t* {
        if (r < (uint32_t)kRtTok) return x + (uint64_t)min(t0 + r, T - 1) * H;
        return w + (uint64_t)min(e0 + r - kRtTok, E - 1) * H;
    };
    auto stage = [&](uint32_t c) {  // chunk c into ring slot c % kRtRing
        const uint32_t c0 = c * kRtK;
        const uint32_t vpr = min((uint32_t)kRtK, main_end - c0) / 4;
        uint16_t* dst = raw + (size_t)(c % kRtRing) * kRtRows * kRtK;
        for (uint32_t i = threadIdx.x; i < kRtRows * vpr; i += blockDim.x) {
            const uint32_t r = i / vpr, v = i % vpr;
            cp_async8(dst + (size_t)r * kRtK + v * 4, row_ptr(r) + c0 + v * 4);
        }
        cp_async_commit();
    };

    RtLane ln(warp, lane);
    for (uint32_t c = 0; c + 1 < kRtRing && c < nchunks; ++c) stage(c);
    for (uint32_t c = 0; c < nchunks; ++c) {
        if (c + 1 < nchunks) cp_async_wait<kRtRing - 2>();
        else cp_async_wait<0>();
        __syncthreads();  // chunk c visible to all; every lane done with chunk c - 1's fp32 tile
        if (c + kRtRing - 1 < nchunks) stage(c + kRtRing - 1);  // into the slot chunk c - 1 used
        const uint32_t clen = min((uint32_t)kRtK, main_end - c * kRtK);
        const uint16_t* src = raw + (size_t)(c % kRtRing) * kRtRows * kRtK;
        const uint32_t vpr = clen / 8;
        for (uint32_t i = threadIdx.x; i < kRtRows * vpr; i += blockDim.x) rt_convert8(src, fs, i / vpr, i % vpr);
        __syncthreads();
        ln.chunk(fs, clen);
    }
    __syncthreads();  // tile and ring free for the transpose
    ln.finish(reinterpret_cast<float*>(rt_smem) + (size_t)warp * kRtScratch, x, w, t0, e0, T, E, H, logits);
}

constexpr int kMaxExperts = 1024;

// ---------------------------------------------------------------------------
// expf as the reference's host C library computes it (glibc >= 2.28 on
// x86-64 with FMA; the algorithm published in ARM's optimized-routines):
// with N = 32, z = x * N / ln2 is split into k = round(z) and r = z - k
// (r by one FMA, |r| <= 1/2); 2^(k/N) is a table entry 2^((k mod N)/N) with
// k / N added to its exponent; 2^(r/N) is the cubic 1 + c2 r + c1 r^2 +
// c0 r^3 evaluated by FMAs in double; the product is rounded once to float.
// The table holds 2^(i/32) rounded to double, minus i/32 in the exponent
// field.  Checked equal to the C library's expf for every float in
// [-103.97, 88.72]; outside that range expf is 0 or +inf.
// ---------------------------------------------------------------------------
__device__ const uint64_t kExp2Tab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull};

__device__ __forceinline__ float libm_expf(float x) {
    if (x != x) return x;
    if (x > 0x1.62e42ep6f) return INFINITY;
    if (x < -0x1.9fe368p6f) return 0.0f;
    const double inv_ln2_n = 0x1.71547652b82fep+0 * 32.0;
    const double c0 = 0x1.c6af84b912394p-5 / (32.0 * 32.0 * 32.0);
    const double c1 = 0x1.ebfce50fac4f3p-3 / (32.0 * 32.0);
    const double c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    const double shift = 0x1.8p+52;
    const double xd = (double)x;
    const double z = __dmul_rn(inv_ln2_n, xd);
    double kd = __dadd_rn(z, shift);
    const uint64_t ki = (uint64_t)__double_as_longlong(kd);
    kd = __dsub_rn(kd, shift);
    const double r = __fma_rn(inv_ln2_n, xd, -kd);
    const double s = __longlong_as_double((long long)(kExp2Tab[ki % 32] + (ki << 47)));
    const double p = __fma_rn(__fma_rn(c0, r, c1), __dmul_rn(r, r), __fma_rn(c2, r, 1.0));
    return __double2float_rn(__dmul_rn(p, s));
}

// Group limit of sigmoid routers (generation_router.cpp.inc:484-558) on the
// scores p[0, E) of one token, by one warp (p in shared memory).  Group g is
// experts [g*E/G, (g+1)*E/G); its score is the sum of its two largest scores
// (the largest alone for one expert per group), kept by the reference's
// running best0/best1 update from 0.  The TG groups with the largest scores
// keep their experts' scores, the others' are set to 0.  Equal group scores
// resolve to the lower group index (the reference's nth_element leaves that
// order open).  G <= 256.
__device__ void group_limit_warp(float* p, uint32_t E, uint32_t G, uint32_t TG) {
    const unsigned full = 0xffffffffu;
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t epg = E / G;
    float gs[8];  // scores of groups lane + 32 m
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const uint32_t g = lane + 32 * m;
        float b0 = 0.0f, b1 = 0.0f;
        if (g < G) {
            for (uint32_t e = g * epg; e < (g + 1) * epg; ++e) {
                const float v = p[e];
                if (v > b0) {
                    b1 = b0;
                    b0 = v;
                } else if (v > b1) {
                    b1 = v;
                }
            }
        }
        gs[m] = epg > 1 ? __fadd_rn(b0, b1) : b0;
    }
    uint32_t kept = 0;  // bit m: group lane + 32 m kept
    for (uint32_t j = 0; j < TG; ++j) {
        float best = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const uint32_t g = lane + 32 * m;
            if (g < G && !((kept >> m) & 1u) && (bi == 0x7fffffff || gs[m] > best)) {
                best = gs[m];
                bi = (int)g;
            }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(full, best, o);
            const int oi = __shfl_xor_sync(full, bi, o);
            if (oi != 0x7fffffff && (bi == 0x7fffffff || ob > best || (ob == best && oi < bi))) {
                best = ob;
                bi = oi;
            }
        }
        if ((uint32_t)(bi & 31) == lane) kept |= 1u << (bi >> 5);
    }
    __syncwarp();
    for (uint32_t r = 0; r < (E + 31) / 32; ++r) {
        const uint32_t e = lane + 32 * r;
        const uint32_t g = (e < E ? e : 0) / epg;
        const uint32_t owner_bits = __shfl_sync(full, kept, g & 31);
        if (e < E && !((owner_bits >> (g >> 5)) & 1u)) p[e] = 0.0f;
    }
    __syncwarp();
}

__device__ void topk_token(float* p, uint32_t t, uint32_t E, uint32_t K, const RouteCfg& rc,
                           int32_t* __restrict__ ids, float* __restrict__ wout, float* __restrict__ scores_out) {
    const int sigmoid = rc.sigmoid, norm_topk = rc.norm_topk;
    const float routed_scale = rc.routed_scale;
    const int lane = threadIdx.x & 31;
    if (sigmoid) {
        for (uint32_t e = lane; e < E; e += 32) {
            const float ex = libm_expf(-p[e]);
            p[e] = __fdiv_rn(1.0f, __fadd_rn(1.0f, ex));
        }
        __syncwarp();
        if (rc.n_group) group_limit_warp(p, E, rc.n_group, rc.topk_group);
    } else {
        float mx = -INFINITY;
        for (uint32_t e = lane; e < E; e += 32) mx = fmaxf(mx, p[e]);
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        for (uint32_t e = lane; e < E; e += 32) p[e] = (float)exp((double)p[e] - (double)mx);
        __syncwarp();
        double denom = 0.0;
        if (lane == 0) {
            for (uint32_t e = 0; e < E; ++e) denom = __dadd_rn(denom, (double)p[e]);
        }
        denom = __shfl_sync(0xffffffffu, denom, 0);
        const float inv = (float)(1.0 / denom);
        for (uint32_t e = lane; e < E; e += 32) p[e] = __fmul_rn(p[e], inv);
        __syncwarp();
    }
    if (scores_out) {
        for (uint32_t e = lane; e < E; e += 32) scores_out[(uint64_t)t * E + e] = p[e];
    }
    // k rounds of arg-max; equal scores resolve to the lower expert index.
    float sel_w[32];
    int sel_i[32];
    uint32_t taken_mask[kMaxExperts / 32];
    for (uint32_t q = 0; q < (E + 31) / 32; ++q) taken_mask[q] = 0;
    for (uint32_t j = 0; j < K; ++j) {
        float best = -INFINITY;
        int bi = 0x7fffffff;
        for (uint32_t e = lane; e < E; e += 32) {
            if ((taken_mask[e >> 5] >> (e & 31)) & 1u) continue;
            const float v = p[e];
            // e grows within a lane, so an equal score never displaces an
            // earlier (lower) index here
            if (bi == 0x7fffffff || v > best) {
                best = v;
                bi = (int)e;
            }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != 0x7fffffff && (bi == 0x7fffffff || ob > best || (ob == best && oi < bi))) {
                best = ob;
                bi = oi;
            }
        }
        taken_mask[bi >> 5] |= 1u << (bi & 31);
        if (j < 32) {
            sel_w[j] = best;
            sel_i[j] = bi;
        }
    }
    if (lane == 0) {
        float denom = 0.f;
        for (uint32_t j = 0; j < K; ++j) denom = __fadd_rn(denom, sel_w[j]);
        if (norm_topk && denom <= 0.f) denom = 1e-8f;
        const float scale = sigmoid ? routed_scale : 1.0f;
        for (uint32_t j = 0; j < K; ++j) {
            float wv = sel_w[j];
            if (norm_topk) wv = __fdiv_rn(wv, denom);
            if (scale != 1.0f) wv = __fmul_rn(wv, scale);
            ids[(uint64_t)t * K + j] = sel_i[j];
            wout[(uint64_t)t * K + j] = wv;
        }
    }
}

// ---------------------------------------------------------------------------
// Scores + top-k of one token for E <= 32 * EPL experts, by one warp, all in
// registers (expert e = lane + 32 q in slot q).  Same arithmetic and order as
// topk_token: double exp, the softmax denominator summed in double in expert
// order (every lane runs the same chain), equal scores to the lower index.
// Requires K <= 32.
// ---------------------------------------------------------------------------
template <int EPL>
__device__ void topk_token_reg(float* lg, uint32_t t, uint32_t E, uint32_t K, const RouteCfg& rc,
                               int32_t* __restrict__ ids, float* __restrict__ wout, float* __restrict__ scores_out) {
    const int sigmoid = rc.sigmoid, norm_topk = rc.norm_topk;
    const float routed_scale = rc.routed_scale;
    const uint32_t lane = threadIdx.x & 31;
    const unsigned full = 0xffffffffu;
    float v[EPL];
#pragma unroll
    for (int q = 0; q < EPL; ++q) {
        const uint32_t e = lane + 32 * q;
        v[q] = e < E ? lg[e] : 0.f;
    }
    if (sigmoid) {
#pragma unroll
        for (int q = 0; q < EPL; ++q) {
            const float ex = libm_expf(-v[q]);
            v[q] = __fdiv_rn(1.0f, __fadd_rn(1.0f, ex));
        }
        if (rc.n_group) {  // through the token's shared-memory row
            __syncwarp();
#pragma unroll
            for (int q = 0; q < EPL; ++q)
                if (lane + 32 * q < E) lg[lane + 32 * q] = v[q];
            __syncwarp();
            group_limit_warp(lg, E, rc.n_group, rc.topk_group);
#pragma unroll
            for (int q = 0; q < EPL; ++q) v[q] = lane + 32 * q < E ? lg[lane + 32 * q] : 0.f;
        }
    } else {
        float mx = -INFINITY;
#pragma unroll
        for (int q = 0; q < EPL; ++q)
            if (lane + 32 * q < E) mx = fmaxf(mx, v[q]);
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(full, mx, o));
#pragma unroll
        for (int q = 0; q < EPL; ++q) v[q] = (float)exp((double)v[q] - (double)mx);
        double denom = 0.0;
#pragma unroll
        for (int q = 0; q < EPL; ++q) {
            float all[32];
#pragma unroll
            for (int s = 0; s < 32; ++s) all[s] = __shfl_sync(full, v[q], s);
#pragma unroll
            for (int s = 0; s < 32; ++s)
                if (32 * q + s < (int)E) denom = __dadd_rn(denom, (double)all[s]);
        }
        const float inv = (float)(1.0 / denom);
#pragma unroll
        for (int q = 0; q < EPL; ++q) v[q] = __fmul_rn(v[q], inv);
    }
    if (scores_out) {
#pragma unroll
        for (int q = 0; q < EPL; ++q)
            if (lane + 32 * q < E) scores_out[(uint64_t)t * E + lane + 32 * q] = v[q];
    }
    uint32_t taken = 0;  // bit q: slot q selected
    float my_w = 0.f;
    int my_i = 0;
    for (uint32_t j = 0; j < K; ++j) {
        float best = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int q = 0; q < EPL; ++q) {
            const uint32_t e = lane + 32 * q;
            if (e < E && !((taken >> q) & 1u) && (bi == 0x7fffffff || v[q] > best)) {
                best = v[q];
                bi = (int)e;
            }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(full, best, o);
            const int oi = __shfl_xor_sync(full, bi, o);
            if (oi != 0x7fffffff && (bi == 0x7fffffff || ob > best || (ob == best && oi < bi))) {
                best = ob;
                bi = oi;
            }
        }
        if ((uint32_t)(bi & 31) == lane) taken |= 1u << (bi >> 5);
        if (lane == j) {
            my_w = best;
            my_i = bi;
        }
    }
    float denom = 0.f;
    for (uint32_t j = 0; j < K; ++j) denom = __fadd_rn(denom, __shfl_sync(full, my_w, j));
    if (lane < K) {
        if (norm_topk && denom <= 0.f) denom = 1e-8f;
        const float scale = sigmoid ? routed_scale : 1.0f;
        float wv = my_w;
        if (norm_topk) wv = __fdiv_rn(wv, denom);
        if (scale != 1.0f) wv = __fmul_rn(wv, scale);
        ids[(uint64_t)t * K + lane] = my_i;
        wout[(uint64_t)t * K + lane] = wv;
    }
}

// Top-k over logits in global memory: one warp per token.
__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ logits, uint32_t T, uint32_t E,
                                                          uint32_t K, RouteCfg rc,
                                                          int32_t* __restrict__ ids, float* __restrict__ wout,
                                                          float* __restrict__ scores_out) {
    __shared__ float ps[8][kMaxExperts];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t t = blockIdx.x * 8 + warp;
    if (t >= T) return;
    for (uint32_t e = lane; e < E; e += 32) ps[warp][e] = logits[(uint64_t)t * E + e];
    __syncwarp();
    if (K <= 32 && E <= 32) {
        topk_token_reg<1>(ps[warp], t, E, K, rc, ids, wout, scores_out);
    } else if (K <= 32 && E <= 64) {
        topk_token_reg<2>(ps[warp], t, E, K, rc, ids, wout, scores_out);
    } else if (K <= 32 && E <= 128) {
        topk_token_reg<4>(ps[warp], t, E, K, rc, ids, wout, scores_out);
    } else if (K <= 32 && E <= 256) {
        topk_token_reg<8>(ps[warp], t, E, K, rc, ids, wout, scores_out);
    } else {
        topk_token(ps[warp], t, E, K, rc, ids, wout, scores_out);
    }
}

// ---------------------------------------------------------------------------
// Router for small batches, logits and top-k in one kernel.  A block holds
// the rows of `tb` tokens and all E <= 64 router rows in shared memory (row
// pitch 2H + 32 bytes, so the rows a warp reads fall in different banks),
// brought in by one bulk copy per row before any arithmetic.  Eight threads
// per (token, expert) dot product: thread m owns the reference's FMA chains
// 2m and 2m + 1 (elements 16 i + 2m, 16 i + 2m + 1, one 4-byte load per
// operand), so the 16-chain order of router_logits_kernel is kept exactly.
// Then one warp per token runs the top-k.
// ---------------------------------------------------------------------------
constexpr int kRfMaxDots = 64;          // tb * E per block (8 threads each, 512 threads)
constexpr int kRfMaxE = 64;
constexpr uint32_t kRfSmemMax = 200 * 1024;

__global__ void __launch_bounds__(512) router_fused_kernel(const uint16_t* __restrict__ x,
                                                           const uint16_t* __restrict__ w, uint32_t T, uint32_t E,
                                                           uint32_t H, uint32_t K, uint32_t tb, RouteCfg rc,
                                                           float* __restrict__ logits, int32_t* __restrict__ ids,
                                                           float* __restrict__ wout, float* __restrict__ scores,
                                                           uint32_t* __restrict__ err) {
    extern __shared__ __align__(16) uint8_t rf_smem[];
    __shared__ uint64_t bar;
    const uint32_t pitch = H * 2 + 32;  // bytes per staged row
    uint8_t* xs = rf_smem;                               // [tb] rows
    uint8_t* ws = rf_smem + (size_t)tb * pitch;          // [E] rows
    float* lg = reinterpret_cast<float*>(ws + (size_t)E * pitch);  // [tb][E]
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t t0 = blockIdx.x * tb;
    const uint32_t nt = min(tb, T - t0);
    pdl_trigger();  // the permutation kernel may launch now; it waits for the ids
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == 0) {
        const uint32_t rowb = H * 2;
        if (lane == 0) mbar_arrive_expect_tx(&bar, (nt + E) * rowb);
        __syncwarp();
        for (uint32_t r = lane; r < nt + E; r += 32) {
            if (r < nt) {
                bulk_g2s(xs + (size_t)r * pitch, x + (uint64_t)(t0 + r) * H, rowb, &bar);
            } else {
                bulk_g2s(ws + (size_t)(r - nt) * pitch, w + (uint64_t)(r - nt) * H, rowb, &bar);
            }
        }
    }
    const bool ok = mbar_wait(&bar, 0, err, kErrTimeoutLoadFull);
    if (!__syncthreads_and(ok)) return;

    const uint32_t m = threadIdx.x & 7;
    const uint32_t d = threadIdx.x >> 3;  // dot: token d / E, expert d % E
    const uint32_t ndots = nt * E;
    const uint32_t dv = d < ndots ? d : 0;  // idle threads shadow dot 0 (the shuffles span 8 lanes)
    const uint8_t* xr = xs + (size_t)(dv / E) * pitch;
    const uint8_t* wr = ws + (size_t)(dv % E) * pitch;
    const uint32_t main_end = H & ~15u;
    float a0 = 0.f, a1 = 0.f;
#pragma unroll 4
    for (uint32_t i = 0; i < main_end; i += 16) {
        const uint32_t xv = *reinterpret_cast<const uint32_t*>(xr + (i + 2 * m) * 2);
        const uint32_t wv = *reinterpret_cast<const uint32_t*>(wr + (i + 2 * m) * 2);
        a0 = __fmaf_rn(__uint_as_float(wv << 16), __uint_as_float(xv << 16), a0);
        a1 = __fmaf_rn(__uint_as_float(wv & 0xffff0000u), __uint_as_float(xv & 0xffff0000u), a1);
    }
    // b_c = s_c + s_{c+8} (chains c = 2m + q, m < 4), then ((b0 + b1) + b2) + ... + b7
    const unsigned full = 0xffffffffu;
    const float b0 = a0 + __shfl_down_sync(full, a0, 4, 8);
    const float b1 = a1 + __shfl_down_sync(full, a1, 4, 8);
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float c0 = __shfl_sync(full, b0, q, 8);
        const float c1 = __shfl_sync(full, b1, q, 8);
        s = q == 0 ? __fadd_rn(c0, c1) : __fadd_rn(__fadd_rn(s, c0), c1);
    }
    if (m == 0 && d < ndots) {
        const uint16_t* xe = reinterpret_cast<const uint16_t*>(xr);
        const uint16_t* we = reinterpret_cast<const uint16_t*>(wr);
        float out = 0.0f + s;
        uint32_t i = main_end;
        float t0a = 0.f, t1a = 0.f, t2a = 0.f, t3a = 0.f;
        for (; i + 3 < H; i += 4) {
            t0a = __fmaf_rn(bf16_bits_to_f32(we[i]), bf16_bits_to_f32(xe[i]), t0a);
            t1a = __fmaf_rn(bf16_bits_to_f32(we[i + 1]), bf16_bits_to_f32(xe[i + 1]), t1a);
            t2a = __fmaf_rn(bf16_bits_to_f32(we[i + 2]), bf16_bits_to_f32(xe[i + 2]), t2a);
            t3a = __fmaf_rn(bf16_bits_to_f32(we[i + 3]), bf16_bits_to_f32(xe[i + 3]), t3a);
        }
        out = __fadd_rn(out, __fadd_rn(__fadd_rn(t0a, t1a), __fadd_rn(t2a, t3a)));
        for (; i < H; ++i) out = __fmaf_rn(bf16_bits_to_f32(we[i]), bf16_bits_to_f32(xe[i]), out);
        lg[d] = out;
        logits[(uint64_t)t0 * E + d] = out;
    }
    __syncthreads();
    for (uint32_t tt = warp; tt < nt; tt += 16) {
        if (E <= 32 && K <= 32) {
            topk_token_reg<1>(lg + (size_t)tt * E, t0 + tt, E, K, rc, ids, wout, scores);
        } else if (K <= 32) {
            topk_token_reg<2>(lg + (size_t)tt * E, t0 + tt, E, K, rc, ids, wout, scores);
        } else {
            topk_token(lg + (size_t)tt * E, t0 + tt, E, K, rc, ids, wout, scores);
        }
    }
}

// ---------------------------------------------------------------------------
// Stable counting sort of n items by bucket (deterministic).
//   count:   per 2048-item tile, per-bucket counts and each item's rank among
//            earlier items of its bucket in the tile;
//   scan:    per-bucket prefix over tiles, group sizes and offsets;
//   scatter: destination = offset[bucket] + tile base + rank.
// ---------------------------------------------------------------------------
static_assert(kSortTile == 8 * 8 * 32, "a sort tile is 8 warps x 8 steps x 32 lanes");

__global__ void __launch_bounds__(256) sort_count_kernel(const int32_t* __restrict__ keys, uint32_t n,
                                                         uint32_t nb, uint32_t* __restrict__ tile_counts,
                                                         uint32_t* __restrict__ rank, uint32_t* __restrict__ err) {
    extern __shared__ uint32_t cnt[];  // [8][nb]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (uint32_t i = threadIdx.x; i < 8 * nb; i += blockDim.x) cnt[i] = 0;
    __syncthreads();
    const uint32_t base = blockIdx.x * kSortTile + warp * 256;
    const unsigned lt = (1u << lane) - 1u;
    uint32_t* wc = cnt + warp * nb;
    for (int s = 0; s < 8; ++s) {
        const uint32_t item = base + s * 32 + lane;
        int32_t b = -1;
        if (item < n) {
            b = keys[item];
            if (b < 0 || (uint32_t)b >= nb) {
                record_error(err, kErrBadExpert);
                b = -1;
            }
        }
        const unsigned peers = __match_any_sync(0xffffffffu, b);
        const uint32_t before = (b >= 0) ? wc[b] : 0;
        __syncwarp();
        if (b >= 0) {
            rank[item] = before + __popc(peers & lt);
            if ((int)(__ffs(peers) - 1) == lane) wc[b] = before + __popc(peers);
        }
        __syncwarp();
    }
    __syncthreads();
    // exclusive prefix over the 8 warps per bucket; tile totals to global
    for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) {
        uint32_t run = 0;
        for (int w = 0; w < 8; ++w) {
            const uint32_t c = cnt[w * nb + b];
            cnt[w * nb + b] = run;
            run += c;
        }
        tile_counts[(uint64_t)blockIdx.x * nb + b] = run;
    }
    __syncthreads();
    for (int s = 0; s < 8; ++s) {
        const uint32_t item = base + s * 32 + lane;
        if (item < n) {
            const int32_t b = keys[item];
            if (b >= 0 && (uint32_t)b < nb) rank[item] += cnt[warp * nb + b];
        }
    }
}

// Single block: per-bucket prefix over tiles (in place: counts become
// bases), group sizes, group offsets and the GEMM tile prefixes.
// Group layout: buckets 0..nb-1 then, when `extra_rows` > 0, one extra group
// (the shared expert) of `extra_rows` rows.
__global__ void __launch_bounds__(1024) sort_scan_kernel(uint32_t* __restrict__ tile_counts, uint32_t ntiles,
                                                         uint32_t nb, uint32_t extra_rows,
                                                         GroupInfo gi) {
    __shared__ uint32_t warp_sums[32];
    const uint32_t G = nb + (extra_rows ? 1 : 0);
    // 1) per-bucket column scan over tiles
    for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) {
        uint32_t run = 0;
        for (uint32_t t = 0; t < ntiles; ++t) {
            const uint32_t c = tile_counts[(uint64_t)t * nb + b];
            tile_counts[(uint64_t)t * nb + b] = run;
            run += c;
        }
        gi.count[b] = run;
    }
    if (threadIdx.x == 0 && extra_rows) gi.count[nb] = extra_rows;
    __syncthreads();
    // 2) exclusive scans over groups of: rows, gate/up tiles, down tiles
    uint32_t carry_rows = 0, carry_gu = 0, carry_dn = 0;
    for (uint32_t g0 = 0; g0 < G; g0 += blockDim.x) {
        const uint32_t g = g0 + threadIdx.x;
        const uint32_t c = g < G ? gi.count[g] : 0;
        const uint32_t ntile_n = ceil_div(c, gi.block_n);
        uint32_t v[3] = {c, ntile_n * gi.gu_row_tiles, ntile_n * gi.dn_row_tiles};
        uint32_t incl[3];
        for (int q = 0; q < 3; ++q) {
            uint32_t x = v[q];
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
                if ((threadIdx.x & 31) >= o) x += y;
            }
            if ((threadIdx.x & 31) == 31) warp_sums[threadIdx.x >> 5] = x;
            __syncthreads();
            if (threadIdx.x < 32) {
                uint32_t s = warp_sums[threadIdx.x];
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
                    if (threadIdx.x >= o) s += y;
                }
                warp_sums[threadIdx.x] = s;
            }
            __syncthreads();
            const uint32_t warp_prefix = (threadIdx.x >= 32) ? warp_sums[(threadIdx.x >> 5) - 1] : 0;
            incl[q] = x + warp_prefix;
            const uint32_t chunk_total = warp_sums[31];
            __syncthreads();
            const uint32_t carry = q == 0 ? carry_rows : (q == 1 ? carry_gu : carry_dn);
            uint32_t* dst = q == 0 ? gi.offset : (q == 1 ? gi.gu_tile_off : gi.dn_tile_off);
            if (g < G) dst[g] = carry + incl[q] - v[q];
            if (q == 0) carry_rows += chunk_total;
            else if (q == 1) carry_gu += chunk_total;
            else carry_dn += chunk_total;
        }
    }
    if (threadIdx.x == 0) {
        gi.offset[G] = carry_rows;
        gi.gu_tile_off[G] = carry_gu;
        gi.dn_tile_off[G] = carry_dn;
    }
}

// ---------------------------------------------------------------------------
// The whole permutation of a decode-sized batch in one block: the stable
// counting sort (same order as sort_count/sort_scan/scatter: by expert, then
// assignment index), the group sizes, offsets and GEMM tile prefixes, and
// the two tile tables of the block-scaled GEMMs (build_tiles_kernel's
// entries).  1024 threads; warp w sorts the contiguous segment
// [w * seg, (w + 1) * seg) of the assignments, seg a multiple of 32.
// ---------------------------------------------------------------------------
constexpr uint32_t kSmallN = 8192;  // assignments (8 per lane)
constexpr uint32_t kSmallE = 256;   // experts

__device__ __forceinline__ void fill_tiles(const uint32_t* cnt, const uint32_t* off, const uint32_t* toff,
                                           uint32_t G, uint32_t m_tiles, uint32_t block_n, TileEntry* tiles,
                                           uint32_t max_tiles) {
    const uint32_t total = toff[G];
    for (uint32_t t = threadIdx.x; t < total && t < max_tiles; t += blockDim.x) {
        uint32_t lo = 0, hi = G;
        while (hi - lo > 1) {
            const uint32_t mid = (lo + hi) >> 1;
            if (toff[mid] <= t) lo = mid;
            else hi = mid;
        }
        const uint32_t local = t - toff[lo];
        const uint32_t ntn = ceil_div(cnt[lo], block_n);
        const uint32_t nt = local % ntn;
        const uint32_t n0 = nt * block_n;
        TileEntry e;
        e.group = lo;
        e.mt = local / ntn;
        e.row0 = off[lo] + n0;
        e.nn_ntile = min(block_n, cnt[lo] - n0) | ((toff[lo] / m_tiles + nt) << 8);
        tiles[t] = e;
    }
}

// Gate/up token tile of the n-th row of a group whose gate/up tiles start at
// tile_off, and the row's index inside that tile: (tile << 8) | index.
__device__ __forceinline__ uint32_t row_tile_info(uint32_t tile_off, uint32_t n, const GroupInfo& gi) {
    return ((tile_off / gi.gu_row_tiles + n / gi.block_n) << 8) | (n % gi.block_n);
}

__global__ void __launch_bounds__(1024) route_small_kernel(const int32_t* __restrict__ ids, uint32_t n, uint32_t K,
                                                           uint32_t E, uint32_t shared_rows, uint32_t shared_base,
                                                           GroupInfo gi,
                                                           TileEntry* __restrict__ gu_tiles, uint32_t gu_max,
                                                           TileEntry* __restrict__ dn_tiles, uint32_t dn_max,
                                                           uint32_t* __restrict__ pos_of,
                                                           uint32_t* __restrict__ row_token,
                                                           uint32_t* __restrict__ row_assign,
                                                           uint32_t* __restrict__ row_info,
                                                           uint32_t* __restrict__ err) {
    __shared__ uint32_t cnt[32][kSmallE];  // per-warp counts, then each warp's base within the expert
    __shared__ uint32_t gcnt[kSmallE + 2], goff[kSmallE + 2], gut[kSmallE + 2], dnt[kSmallE + 2];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t G = E + (shared_rows ? 1 : 0);
    pdl_wait();  // the router's ids
    pdl_trigger();
    for (uint32_t i = threadIdx.x; i < 32 * kSmallE; i += blockDim.x) (&cnt[0][0])[i] = 0;
    __syncthreads();
    const uint32_t seg = ceil_div(ceil_div(n, 32u), 32u) * 32u;
    const uint32_t s0 = warp * seg;
    const unsigned lt = (1u << lane) - 1u;
    uint32_t rk[kSmallN / 1024];
    int32_t bk[kSmallN / 1024];
#pragma unroll
    for (uint32_t s = 0; s < kSmallN / 1024; ++s) {
        const uint32_t i = s0 + s * 32 + lane;
        int32_t b = -1;
        if (s * 32 < seg && i < n) {
            b = ids[i];
            if (b < 0 || (uint32_t)b >= E) {
                record_error(err, kErrBadExpert);
                b = -1;
            }
        }
        const unsigned peers = __match_any_sync(0xffffffffu, b);
        const uint32_t before = b >= 0 ? cnt[warp][b] : 0;
        __syncwarp();
        rk[s] = before + __popc(peers & lt);
        bk[s] = b;
        if (b >= 0 && (int)(__ffs(peers) - 1) == (int)lane) cnt[warp][b] = before + __popc(peers);
        __syncwarp();
    }
    __syncthreads();
    // per expert: exclusive prefix over the warps (stable: warp w's
    // assignments precede warp w + 1's), and the expert's total
    for (uint32_t b = threadIdx.x; b < E; b += blockDim.x) {
        uint32_t run = 0;
        for (uint32_t w = 0; w < 32; ++w) {
            const uint32_t c = cnt[w][b];
            cnt[w][b] = run;
            run += c;
        }
        gcnt[b] = run;
    }
    if (threadIdx.x == 0 && shared_rows) gcnt[E] = shared_rows;
    __syncthreads();
    // exclusive scans over the groups (warp 0, up to 9 groups per lane)
    if (warp == 0) {
        const uint32_t per = ceil_div(G, 32u);
        uint32_t a = 0, bsum = 0, c = 0;
        for (uint32_t q = 0; q < per; ++q) {
            const uint32_t g = lane * per + q;
            if (g < G) {
                const uint32_t ntn = ceil_div(gcnt[g], gi.block_n);
                a += gcnt[g];
                bsum += ntn * gi.gu_row_tiles;
                c += ntn * gi.dn_row_tiles;
            }
        }
        uint32_t ia = a, ib = bsum, ic = c;
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t ya = __shfl_up_sync(0xffffffffu, ia, o);
            const uint32_t yb = __shfl_up_sync(0xffffffffu, ib, o);
            const uint32_t yc = __shfl_up_sync(0xffffffffu, ic, o);
            if ((int)lane >= o) {
                ia += ya;
                ib += yb;
                ic += yc;
            }
        }
        uint32_t ra = ia - a, rb = ib - bsum, rc = ic - c;
        for (uint32_t q = 0; q < per; ++q) {
            const uint32_t g = lane * per + q;
            if (g < G) {
                const uint32_t ntn = ceil_div(gcnt[g], gi.block_n);
                goff[g] = ra;
                gut[g] = rb;
                dnt[g] = rc;
                ra += gcnt[g];
                rb += ntn * gi.gu_row_tiles;
                rc += ntn * gi.dn_row_tiles;
            }
        }
        if (lane == 31) {
            goff[G] = ia;
            gut[G] = ib;
            dnt[G] = ic;
        }
    }
    __syncthreads();
    for (uint32_t g = threadIdx.x; g <= G; g += blockDim.x) {
        if (g < G) gi.count[g] = gcnt[g];
        gi.offset[g] = goff[g];
        gi.gu_tile_off[g] = gut[g];
        gi.dn_tile_off[g] = dnt[g];
    }
    // destinations
#pragma unroll
    for (uint32_t s = 0; s < kSmallN / 1024; ++s) {
        const uint32_t i = s0 + s * 32 + lane;
        const int32_t b = bk[s];
        if (b >= 0) {
            const uint32_t n = cnt[warp][b] + rk[s];
            const uint32_t pos = goff[b] + n;
            pos_of[i] = pos;
            row_token[pos] = i / K;
            row_assign[pos] = i;
            if (row_info) row_info[pos] = row_tile_info(gut[b], n, gi);
        }
    }
    for (uint32_t t = threadIdx.x; t < shared_rows; t += blockDim.x) {
        const uint32_t pos = goff[E] + t;
        row_token[pos] = shared_base + t;
        row_assign[pos] = 0xffffffffu;
        if (row_info) row_info[pos] = row_tile_info(gut[E], t, gi);
    }
    if (gu_tiles) fill_tiles(gcnt, goff, gut, G, gi.gu_row_tiles, gi.block_n, gu_tiles, gu_max);
    if (dn_tiles) fill_tiles(gcnt, goff, dnt, G, gi.dn_row_tiles, gi.block_n, dn_tiles, dn_max);
}

// Destination of every assignment a = t*K + j, and for every permuted row:
// its source token and assignment.  Shared-expert rows follow the routed
// rows in token order.
__global__ void scatter_kernel(const int32_t* __restrict__ ids, uint32_t n, uint32_t K, uint32_t nb,
                               const uint32_t* __restrict__ tile_base, const uint32_t* __restrict__ rank,
                               GroupInfo gi, uint32_t shared_rows, uint32_t shared_base, uint32_t* __restrict__ pos_of,
                               uint32_t* __restrict__ row_token, uint32_t* __restrict__ row_assign,
                               uint32_t* __restrict__ row_info) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const int32_t b = ids[i];
        if (b >= 0 && (uint32_t)b < nb) {
            const uint32_t n = tile_base[(uint64_t)(i / kSortTile) * nb + b] + rank[i];
            const uint32_t pos = gi.offset[b] + n;
            pos_of[i] = pos;
            row_token[pos] = i / K;
            row_assign[pos] = i;
            if (row_info) row_info[pos] = row_tile_info(gi.gu_tile_off[b], n, gi);
        }
    } else if (i < n + shared_rows) {
        const uint32_t t = i - n;
        const uint32_t pos = gi.offset[nb] + t;
        row_token[pos] = shared_base + t;
        row_assign[pos] = 0xffffffffu;
        if (row_info) row_info[pos] = row_tile_info(gi.gu_tile_off[nb], t, gi);
    }
}

// X_perm[p][0..Kp) = x[row_token[p]][0..H) followed by zeros; 16-byte
// vectors, one warp per row.
__global__ void gather_rows_kernel(const uint16_t* __restrict__ x, uint32_t H, uint32_t Kp,
                                   const uint32_t* __restrict__ row_token, uint32_t rows,
                                   uint16_t* __restrict__ xp) {
    const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
    const uint32_t lane = threadIdx.x & 31;
    for (uint32_t r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
        const uint4* src = reinterpret_cast<const uint4*>(x + (uint64_t)row_token[r] * H);
        uint4* dst = reinterpret_cast<uint4*>(xp + (uint64_t)r * Kp);
        const uint32_t nv = H / 8, nvp = Kp / 8;
        for (uint32_t v = lane; v < nvp; v += 32) dst[v] = v < nv ? __ldg(src + v) : make_uint4(0, 0, 0, 0);
    }
}

// y[t] = ys[t] + sum_j w[t,j] * yp[pos(t,j)], one fused multiply-add per
// term in router order (generation_mlp.cpp.inc:1417-1431 via moe_axpy_f32);
// ys (the shared expert's rows) may be null.
__global__ void combine_kernel(const float* __restrict__ yp, uint32_t H, const uint32_t* __restrict__ pos_of,
                               const float* __restrict__ w, uint32_t T, uint32_t K, const float* __restrict__ ys,
                               uint16_t* __restrict__ y_bf16, float* __restrict__ y_f32) {
    pdl_wait();  // the down GEMM's rows
    for (uint32_t t = blockIdx.y; t < T; t += gridDim.y)
    for (uint32_t h4 = blockIdx.x * blockDim.x + threadIdx.x; h4 * 4 < H; h4 += gridDim.x * blockDim.x) {
        const uint32_t h = h4 * 4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        if (ys) {
            const float4 s = *reinterpret_cast<const float4*>(ys + (uint64_t)t * H + h);
            acc.x = 0.f + s.x;
            acc.y = 0.f + s.y;
            acc.z = 0.f + s.z;
            acc.w = 0.f + s.w;
        }
        for (uint32_t j = 0; j < K; ++j) {
            const uint32_t p = pos_of[(uint64_t)t * K + j];
            const float wt = w[(uint64_t)t * K + j];
            const float4 v = *reinterpret_cast<const float4*>(yp + (uint64_t)p * H + h);
            acc.x = __fmaf_rn(wt, v.x, acc.x);
            acc.y = __fmaf_rn(wt, v.y, acc.y);
            acc.z = __fmaf_rn(wt, v.z, acc.z);
            acc.w = __fmaf_rn(wt, v.w, acc.w);
        }
        if (y_f32) *reinterpret_cast<float4*>(y_f32 + (uint64_t)t * H + h) = acc;
        if (y_bf16) {
            uint2 o;
            o.x = (uint32_t)f32_to_bf16_bits(acc.x) | ((uint32_t)f32_to_bf16_bits(acc.y) << 16);
            o.y = (uint32_t)f32_to_bf16_bits(acc.z) | ((uint32_t)f32_to_bf16_bits(acc.w) << 16);
            *reinterpret_cast<uint2*>(y_bf16 + (uint64_t)t * H + h) = o;
        }
    }
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
// Tokens per block for router_fused_kernel, or 0 when that kernel does not
// apply (rows not 16-byte aligned, too many experts for one block's shared
// memory, or a batch large enough that the tiled kernel's reuse wins).
static uint32_t router_fused_tb(const uint16_t* x, const uint16_t* w, uint32_t T, uint32_t E, uint32_t H) {
    if (H % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15)) return 0;
    if (E == 0 || E > (uint32_t)kRfMaxE) return 0;
    auto smem = [&](uint32_t tb) { return (uint64_t)(tb + E) * (H * 2 + 32) + (uint64_t)tb * E * 4; };
    uint32_t tb = std::max(1u, ceil_div(T, 148u));
    tb = std::min(tb, (uint32_t)kRfMaxDots / E);
    while (tb > 1 && smem(tb) > kRfSmemMax) --tb;
    if (smem(tb) > kRfSmemMax) return 0;
    if (ceil_div(T, tb) > 4u * 148u) return 0;
    return tb;
}

uint32_t router_box_rows(bool tokens) { return tokens ? kRtTok : kRtExp; }

bool router_wants_tma(const uint16_t* x, const uint16_t* w, uint32_t T, uint32_t E, uint32_t H) {
    if (T == 0 || router_fused_tb(x, w, T, E, H)) return false;
    return H % 8 == 0 && !(reinterpret_cast<uintptr_t>(x) & 15) && !(reinterpret_cast<uintptr_t>(w) & 15) &&
           (H & ~15u) > 0;
}

cudaError_t launch_router(const uint16_t* x, const uint16_t* w, uint32_t T, uint32_t E, uint32_t H, uint32_t K,
                          const RouteCfg& rc_in, float* logits, int32_t* ids, float* wout, float* scores,
                          uint32_t* err, cudaStream_t st, uint32_t* launches, const CUtensorMap* tmap_x,
                          const CUtensorMap* tmap_w) {
    if (T == 0) return cudaSuccess;
    RouteCfg rc = rc_in;
    // the group limit applies under the reference's conditions only
    if (!(rc.sigmoid && rc.n_group > 1 && rc.topk_group > 0 && rc.topk_group < rc.n_group && E % rc.n_group == 0))
        rc.n_group = rc.topk_group = 0;
    if (rc.n_group > 256) return cudaErrorInvalidValue;
    const uint32_t tb = router_fused_tb(x, w, T, E, H);
    if (tb) {
        static uint64_t attr_set = 0;  // one bit per device
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev < 64 && !((attr_set >> dev) & 1u)) {
            e = cudaFuncSetAttribute(router_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kRfSmemMax);
            if (e != cudaSuccess) return e;
            attr_set |= 1ull << dev;
        }
        const size_t smem = (size_t)(tb + E) * (H * 2 + 32) + (size_t)tb * E * 4;
        router_fused_kernel<<<ceil_div(T, tb), 512, smem, st>>>(x, w, T, E, H, K, tb, rc, logits, ids, wout,
                                                               scores, err);
        if (launches) *launches += 1;
        return cudaGetLastError();
    }
    static uint64_t rt_attr = 0;  // one bit per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && !((rt_attr >> dev) & 1u)) {
        e = cudaFuncSetAttribute(router_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRtSmem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(router_logits_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kRtTmaSmem);
        if (e != cudaSuccess) return e;
        rt_attr |= 1ull << dev;
    }
    if (ceil_div(T, kRtTok) > 65535u) return cudaErrorInvalidValue;  // grid y limit: T <= 2,097,120
    dim3 g1(ceil_div(E, kRtExp), ceil_div(T, kRtTok));
    if (tmap_x && tmap_w)
        router_logits_tma_kernel<<<g1, kRtTmaThreads, kRtTmaSmem, st>>>(*tmap_x, *tmap_w, x, w, T, E, H, logits,
                                                                         err);
    else
        router_logits_kernel<<<g1, 256, kRtSmem, st>>>(x, w, T, E, H, logits);
    router_topk_kernel<<<ceil_div(T, 8), 256, 0, st>>>(logits, T, E, K, rc, ids, wout, scores);
    if (launches) *launches += 2;
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Router logits from fp32 token rows (a Gemma-style block whose router reads
// RMSNorm(hidden) or the scaled residual stream), in the reference's order:
// a half-warp per (token, expert) dot, lane l running chain l over elements
// l, l + 16, ... of the 16-aligned part, then b_c = s_c + s_{c+8} and
// ((b0 + b1) + b2) + ... + b7, then the 4-way and scalar tails on lane 0 --
// the same arithmetic as RtLane::finish, so bf16-valued rows give the bf16
// kernels' logits bit for bit.  One block per token, its 16 half-warps take
// the experts in turn.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) router_logits_f32in_kernel(const float* __restrict__ x,
                                                                  const uint16_t* __restrict__ w, uint32_t T,
                                                                  uint32_t E, uint32_t H, float* __restrict__ logits) {
    const uint32_t t = blockIdx.x;
    const uint32_t hw = threadIdx.x >> 4, l = threadIdx.x & 15;
    const uint32_t main_end = H & ~15u;
    const float* xr = x + (uint64_t)t * H;
    const unsigned mask = 0xFFFFu << (threadIdx.x & 16);
    for (uint32_t e = hw; e < E; e += 16) {
        const uint16_t* wr = w + (uint64_t)e * H;
        float s = 0.0f;
        for (uint32_t i = l; i < main_end; i += 16) s = __fmaf_rn(__ldg(xr + i), bf16_bits_to_f32(__ldg(wr + i)), s);
        const float b = __fadd_rn(s, __shfl_down_sync(mask, s, 8, 16));  // lanes 0..7: b_l
        float sum = __shfl_sync(mask, b, 0, 16);
        for (int c = 1; c < 8; ++c) sum = __fadd_rn(sum, __shfl_sync(mask, b, c, 16));
        if (l == 0) {
            float out = 0.0f + sum;
            if (main_end < H) {
                uint32_t i = main_end;
                float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
                for (; i + 3 < H; i += 4) {
                    a0 = __fmaf_rn(bf16_bits_to_f32(wr[i]), xr[i], a0);
                    a1 = __fmaf_rn(bf16_bits_to_f32(wr[i + 1]), xr[i + 1], a1);
                    a2 = __fmaf_rn(bf16_bits_to_f32(wr[i + 2]), xr[i + 2], a2);
                    a3 = __fmaf_rn(bf16_bits_to_f32(wr[i + 3]), xr[i + 3], a3);
                }
                out = __fadd_rn(out, __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3)));
                for (; i < H; ++i) out = __fmaf_rn(bf16_bits_to_f32(wr[i]), xr[i], out);
            }
            logits[(uint64_t)t * E + e] = out;
        }
    }
}

cudaError_t launch_router_f32(const float* x, const uint16_t* w, uint32_t T, uint32_t E, uint32_t H, uint32_t K,
                              const RouteCfg& rc_in, float* logits, int32_t* ids, float* wout, float* scores,
                              cudaStream_t st, uint32_t* launches) {
    if (T == 0) return cudaSuccess;
    RouteCfg rc = rc_in;
    if (!(rc.sigmoid && rc.n_group > 1 && rc.topk_group > 0 && rc.topk_group < rc.n_group && E % rc.n_group == 0))
        rc.n_group = rc.topk_group = 0;
    if (rc.n_group > 256) return cudaErrorInvalidValue;
    router_logits_f32in_kernel<<<T, 256, 0, st>>>(x, w, T, E, H, logits);
    router_topk_kernel<<<ceil_div(T, 8), 256, 0, st>>>(logits, T, E, K, rc, ids, wout, scores);
    if (launches) *launches += 2;
    return cudaGetLastError();
}

uint32_t sort_tiles(uint32_t n) { return ceil_div(n, kSortTile); }

cudaError_t launch_sort_count(const int32_t* keys, uint32_t n, uint32_t nb, uint32_t* tile_counts, uint32_t* rank,
                              uint32_t* err, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    sort_count_kernel<<<sort_tiles(n), 256, 8 * nb * sizeof(uint32_t), st>>>(keys, n, nb, tile_counts, rank, err);
    return cudaGetLastError();
}

cudaError_t launch_sort_scan(uint32_t* tile_counts, uint32_t ntiles, uint32_t nb, GroupInfo gi, cudaStream_t st) {
    sort_scan_kernel<<<1, 1024, 0, st>>>(tile_counts, ntiles, nb, 0, gi);
    return cudaGetLastError();
}

cudaError_t launch_permute(const int32_t* ids, uint32_t T, uint32_t K, uint32_t E, uint32_t shared_rows,
                           uint32_t shared_base, uint32_t* tile_counts, uint32_t* rank, GroupInfo gi, uint32_t* pos_of,
                           uint32_t* row_token, uint32_t* row_assign, uint32_t* row_info, uint32_t* err,
                           cudaStream_t st) {
    const uint32_t n = T * K;
    const uint32_t nt = sort_tiles(n);
    if (n > 0) {
        sort_count_kernel<<<nt, 256, 8 * E * sizeof(uint32_t), st>>>(ids, n, E, tile_counts, rank, err);
    }
    sort_scan_kernel<<<1, 1024, 0, st>>>(tile_counts, nt, E, shared_rows, gi);
    const uint32_t total = n + shared_rows;
    if (total > 0) {
        scatter_kernel<<<ceil_div(total, 256), 256, 0, st>>>(ids, n, K, E, tile_counts, rank, gi, shared_rows,
                                                             shared_base, pos_of, row_token, row_assign, row_info);
    }
    return cudaGetLastError();
}

bool route_small_fits(uint32_t n, uint32_t E) { return n <= kSmallN && E <= kSmallE; }

cudaError_t launch_route_small(const int32_t* ids, uint32_t T, uint32_t K, uint32_t E, uint32_t shared_rows,
                               uint32_t shared_base, GroupInfo gi, TileEntry* gu_tiles, uint32_t gu_max,
                               TileEntry* dn_tiles, uint32_t dn_max, uint32_t* pos_of, uint32_t* row_token,
                               uint32_t* row_assign, uint32_t* row_info, uint32_t* err, cudaStream_t st, bool pdl) {
    return launch_kernel(route_small_kernel, dim3(1), dim3(1024), 0, st, pdl, ids, T * K, K, E, shared_rows,
                         shared_base, gi, gu_tiles, gu_max, dn_tiles, dn_max, pos_of, row_token, row_assign,
                         row_info, err);
}

cudaError_t launch_gather(const uint16_t* x, uint32_t H, uint32_t Kp, const uint32_t* row_token, uint32_t rows,
                          uint16_t* xp, cudaStream_t st) {
    if (rows == 0) return cudaSuccess;
    const uint32_t blocks = min(ceil_div(rows, 8), 148u * 8u);
    gather_rows_kernel<<<blocks, 256, 0, st>>>(x, H, Kp, row_token, rows, xp);
    return cudaGetLastError();
}

cudaError_t launch_combine(const float* yp, uint32_t H, const uint32_t* pos_of, const float* w, uint32_t T,
                           uint32_t K, const float* ys, uint16_t* y_bf16, float* y_f32, cudaStream_t st, bool pdl) {
    if (T == 0) return cudaSuccess;
    const uint32_t threads = 128;
    dim3 grid(ceil_div(ceil_div(H, 4), threads), min(T, 65535u));
    return launch_kernel(combine_kernel, grid, dim3(threads), 0, st, pdl, yp, H, pos_of, w, T, K, ys, y_bf16,
                         y_f32);
}

// Combine weights of a layer with missing experts (generation_mlp.cpp.inc:
// 1219-1282): per token the missing experts' weights are 0 and, when the
// router renormalises its top-k (norm), the others' are multiplied by
// 1 / (their sum, added in router order); a token whose experts are all
// missing records kErrAllExpertsMissing (the reference fails the layer
// there).  One thread per token.
__global__ void combine_weights_kernel(const int32_t* __restrict__ ids, const float* __restrict__ w,
                                       const uint8_t* __restrict__ present, uint32_t T, uint32_t K, uint32_t E,
                                       int norm, float* __restrict__ cw, uint32_t* __restrict__ err) {
    const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    const int32_t* id = ids + (uint64_t)t * K;
    const float* wt = w + (uint64_t)t * K;
    float* out = cw + (uint64_t)t * K;
    auto here = [&](uint32_t j) { return (uint32_t)id[j] < E && present[id[j]] != 0; };
    uint32_t mapped = 0;
    float wsum = 0.0f;
    for (uint32_t j = 0; j < K; ++j) {
        if (here(j)) {
            ++mapped;
            wsum = __fadd_rn(wsum, wt[j]);
        }
    }
    if (mapped == 0) record_error(err, kErrAllExpertsMissing);
    const bool renorm = norm && mapped < K && wsum > 1e-9f;
    const float scale = renorm ? __fdiv_rn(1.0f, wsum) : 1.0f;
    for (uint32_t j = 0; j < K; ++j) out[j] = !here(j) ? 0.0f : (renorm ? __fmul_rn(wt[j], scale) : wt[j]);
}

cudaError_t launch_combine_weights(const int32_t* ids, const float* w, const uint8_t* present, uint32_t T,
                                   uint32_t K, uint32_t E, bool norm, float* cw, uint32_t* err, cudaStream_t st) {
    if (T == 0) return cudaSuccess;
    combine_weights_kernel<<<ceil_div(T, 256u), 256, 0, st>>>(ids, w, present, T, K, E, norm ? 1 : 0, cw, err);
    return cudaGetLastError();
}

}  // namespace moe_b200
