// Router top-k, token permutation into ragged per-expert groups, the gather
// of permuted activation rows and the weighted unpermute/combine.
//
// Routing is bit-exact with the reference CPU path:
//   logits   moe_dot_bf16_row (raw_forward_utils.cpp.inc:174-216): per
//            (token, expert) 16 FMA chains over i = l, l+16, ..., lane sums
//            b_l = s_l + s_{l+8}, then ((b0+b1)+b2)+...+b7;
//   softmax  generation_router.cpp.inc:606-622: exp in double, denominator
//            summed in double in expert order, p *= (float)(1/denom);
//   sigmoid  :239-245, 1/(1+exp(-l)) in float;
//   top-k    :640-674, k largest scores descending (equal scores: lower
//            expert index first), optional renormalisation and scaling.
// The permutation is the order of moe_pc_group_tokens_by_expert
// (token_grouping.cpp.inc:47-55): sorted by expert, then token index.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace moe_b200 {

// ---------------------------------------------------------------------------
// Router logits.  A block computes a 16-token x 16-expert tile: 256 threads =
// 16 lane groups x 16 lanes, lane l of a group owning the reference's FMA
// chain l (elements l, l+16, ...) for the group's 4 tokens x 4 experts (16
// independent chains per thread).  Token and router rows are staged through
// shared memory in 256-element chunks with cp.async, double-buffered.
// ---------------------------------------------------------------------------
constexpr int kRtTok = 16, kRtExp = 16;
constexpr int kRtChunk = 256;               // elements per staged chunk (multiple of 16)
constexpr int kRtStride = kRtChunk + 8;     // padded row (bf16) against bank conflicts

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
    const uint32_t d = smem_u32(dst);
    const int n = valid ? 16 : 0;  // 0 source bytes -> zero fill
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__global__ void __launch_bounds__(256) router_logits_kernel(const uint16_t* __restrict__ x,
                                                            const uint16_t* __restrict__ w, uint32_t T,
                                                            uint32_t E, uint32_t H, float* __restrict__ logits) {
    __shared__ __align__(16) uint16_t xs[2][kRtTok][kRtStride];
    __shared__ __align__(16) uint16_t ws[2][kRtExp][kRtStride];
    const int l = threadIdx.x & 15;
    const int grp = threadIdx.x >> 4;
    const int gt = (grp >> 2) * 4, ge = (grp & 3) * 4;  // the group's first token / expert in the tile
    const uint32_t t0 = blockIdx.x * kRtTok, e0 = blockIdx.y * kRtExp;
    const uint32_t main_end = H & ~15u;  // the 16-step main loop of the reference
    const uint32_t nchunks = (main_end + kRtChunk - 1) / kRtChunk;

    auto stage = [&](uint32_t c, int buf) {
        const uint32_t c0 = c * kRtChunk;
        const uint32_t clen = min((uint32_t)kRtChunk, main_end - c0);
        const uint32_t vpr = clen / 8;  // 16-byte vectors per row
        for (uint32_t i = threadIdx.x; i < 32 * vpr; i += blockDim.x) {
            const uint32_t row = i / vpr, v = i % vpr;
            if (row < kRtTok) {
                const uint32_t t = t0 + row;
                cp_async16(&xs[buf][row][v * 8], x + (uint64_t)min(t, T - 1) * H + c0 + v * 8, t < T);
            } else {
                const uint32_t e = e0 + row - kRtTok;
                cp_async16(&ws[buf][row - kRtTok][v * 8], w + (uint64_t)min(e, E - 1) * H + c0 + v * 8, e < E);
            }
        }
        cp_async_commit();
    };

    float acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
    if (nchunks > 0) stage(0, 0);
    for (uint32_t c = 0; c < nchunks; ++c) {
        const int buf = c & 1;
        if (c + 1 < nchunks) {
            stage(c + 1, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const uint32_t clen = min((uint32_t)kRtChunk, main_end - c * kRtChunk);
        for (uint32_t i = l; i < clen; i += 16) {
            float xv[4], wv[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) xv[a] = bf16_bits_to_f32(xs[buf][gt + a][i]);
#pragma unroll
            for (int b = 0; b < 4; ++b) wv[b] = bf16_bits_to_f32(ws[buf][ge + b][i]);
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) acc[a][b] = __fmaf_rn(wv[b], xv[a], acc[a][b]);
        }
        __syncthreads();
    }
    // lane sums b_l = s_l + s_{l+8}, then the ordered 8-term sum, then the
    // reference's 4-way and scalar tails (H % 16 != 0).
    const unsigned full = 0xffffffffu;
#pragma unroll
    for (int a = 0; a < 4; ++a) {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const float hi = __shfl_down_sync(full, acc[a][b], 8, 16);
            const float bl = acc[a][b] + hi;  // valid on lanes 0..7
            float s = __shfl_sync(full, bl, 0, 16);
#pragma unroll
            for (int j = 1; j < 8; ++j) s = __fadd_rn(s, __shfl_sync(full, bl, j, 16));
            const uint32_t tt = t0 + gt + a, e = e0 + ge + b;
            if (l == 0 && tt < T && e < E) {
                float out = 0.0f + s;
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
                logits[(uint64_t)tt * E + e] = out;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Scores + top-k of one token, by one warp.  `p` holds the token's E logits
// on entry (shared memory; may alias nothing else) and its scores on exit.
// ---------------------------------------------------------------------------
constexpr int kMaxExperts = 1024;

__device__ void topk_token(float* p, uint32_t t, uint32_t E, uint32_t K, int sigmoid, int norm_topk,
                           float routed_scale, int32_t* __restrict__ ids, float* __restrict__ wout,
                           float* __restrict__ scores_out) {
    const int lane = threadIdx.x & 31;
    if (sigmoid) {
        for (uint32_t e = lane; e < E; e += 32) {
            const float ex = (float)exp(-(double)p[e]);
            p[e] = __fdiv_rn(1.0f, __fadd_rn(1.0f, ex));
        }
        __syncwarp();
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

// Top-k over logits in global memory: one warp per token.
__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ logits, uint32_t T, uint32_t E,
                                                          uint32_t K, int sigmoid, int norm_topk, float routed_scale,
                                                          int32_t* __restrict__ ids, float* __restrict__ wout,
                                                          float* __restrict__ scores_out) {
    __shared__ float ps[8][kMaxExperts];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t t = blockIdx.x * 8 + warp;
    if (t >= T) return;
    for (uint32_t e = lane; e < E; e += 32) ps[warp][e] = logits[(uint64_t)t * E + e];
    __syncwarp();
    topk_token(ps[warp], t, E, K, sigmoid, norm_topk, routed_scale, ids, wout, scores_out);
}

// ---------------------------------------------------------------------------
// Scores + top-k of one token for E <= 32 * EPL experts, by one warp, all in
// registers (expert e = lane + 32 q in slot q).  Same arithmetic and order as
// topk_token: double exp, the softmax denominator summed in double in expert
// order (every lane runs the same chain), equal scores to the lower index.
// Requires K <= 32.
// ---------------------------------------------------------------------------
template <int EPL>
__device__ void topk_token_reg(const float* lg, uint32_t t, uint32_t E, uint32_t K, int sigmoid, int norm_topk,
                               float routed_scale, int32_t* __restrict__ ids, float* __restrict__ wout,
                               float* __restrict__ scores_out) {
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
            const float ex = (float)exp(-(double)v[q]);
            v[q] = __fdiv_rn(1.0f, __fadd_rn(1.0f, ex));
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
                                                           uint32_t H, uint32_t K, uint32_t tb, int sigmoid,
                                                           int norm_topk, float routed_scale,
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
            topk_token_reg<1>(lg + (size_t)tt * E, t0 + tt, E, K, sigmoid, norm_topk, routed_scale, ids, wout,
                              scores);
        } else if (K <= 32) {
            topk_token_reg<2>(lg + (size_t)tt * E, t0 + tt, E, K, sigmoid, norm_topk, routed_scale, ids, wout,
                              scores);
        } else {
            topk_token(lg + (size_t)tt * E, t0 + tt, E, K, sigmoid, norm_topk, routed_scale, ids, wout, scores);
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
constexpr int kSortTile = 2048;  // 8 warps x 8 steps x 32 lanes

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

cudaError_t launch_router(const uint16_t* x, const uint16_t* w, uint32_t T, uint32_t E, uint32_t H, uint32_t K,
                          int sigmoid, int norm_topk, float routed_scale, float* logits, int32_t* ids, float* wout,
                          float* scores, uint32_t* err, cudaStream_t st, uint32_t* launches) {
    if (T == 0) return cudaSuccess;
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
        router_fused_kernel<<<ceil_div(T, tb), 512, smem, st>>>(x, w, T, E, H, K, tb, sigmoid, norm_topk,
                                                               routed_scale, logits, ids, wout, scores, err);
        if (launches) *launches += 1;
        return cudaGetLastError();
    }
    dim3 g1(ceil_div(T, kRtTok), ceil_div(E, kRtExp));
    router_logits_kernel<<<g1, 256, 0, st>>>(x, w, T, E, H, logits);
    router_topk_kernel<<<ceil_div(T, 8), 256, 0, st>>>(logits, T, E, K, sigmoid, norm_topk, routed_scale, ids, wout,
                                                       scores);
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

}  // namespace moe_b200
