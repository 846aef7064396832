// Gemma-style MoE block parts around the experts (generation_mlp.cpp.inc:
// 94-104, 145-175, 234-250, 380-429, 478-570; generation_router.cpp.inc:
// 316-359):
//   * the routed input RMSNorm(hidden) with the MoE pre-norm weight, and the
//     router input hidden * rms^-1 * scale / sqrt(H) of a router input
//     scale -- both read by the router, so computed exactly as the
//     reference does (sum of squares in double, one fused multiply-add per
//     element in element order; 1 / sqrt in float; the products left to
//     right), which keeps the routing bit-exact;
//   * the block combine: per token the shared expert's row (RMSNorm with
//     post-norm 1, times the shared-expert gate), then in router order each
//     routed row (RMSNorm with post-norm 2, the down scale) added with one
//     fused multiply-add per element, then the output RMSNorm.  These norms
//     change only the output values, so their sums of squares are reduced
//     in parallel (tolerance parity).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace moe_b200 {

// 32 rows per warp: each chunk of 128 columns of the warp's rows is staged in
// shared memory (coalesced loads), then lane r runs row r's sequential
// double-precision chain over the chunk; finally the warp writes the rows
// out, coalesced.  mode 0: out = in * norm * w (or (1 + w) with the unit
// offset), norm = 1 / sqrt(mean + eps); mode 1 (router input scale):
// out = in * norm * scale * (1 / sqrt(H)), norm with eps 1e-6, scale[0]
// for all elements (count 1), scale[i] (count >= H) or 1.
__global__ void __launch_bounds__(32) row_norm_exact_kernel(const float* __restrict__ in, uint32_t rows, uint32_t H,
                                                            const float* __restrict__ w, uint64_t w_count,
                                                            int mode, float eps, int unit_offset,
                                                            float* __restrict__ out_f32,
                                                            uint16_t* __restrict__ out_bf16) {
    __shared__ float tile[32][129];
    const uint32_t lane = threadIdx.x;
    const uint32_t r0 = blockIdx.x * 32;
    double ss = 0.0;
    for (uint32_t c0 = 0; c0 < H; c0 += 128) {
        const uint32_t cn = min(128u, H - c0);
        for (uint32_t rr = 0; rr < 32; ++rr) {
            const uint32_t r = r0 + rr;
            for (uint32_t c = lane; c < cn; c += 32) tile[rr][c] = r < rows ? in[(uint64_t)r * H + c0 + c] : 0.0f;
        }
        __syncwarp();
        for (uint32_t c = 0; c < cn; ++c) {
            const double v = (double)tile[lane][c];
            ss = __fma_rn(v, v, ss);
        }
        __syncwarp();
    }
    const float eps_used = mode == 1 ? 1.0e-6f : (eps > 0.0f ? eps : 1.0e-6f);
    const float my_norm = 1.0f / sqrtf(__double2float_rn(__ddiv_rn(ss, (double)H)) + eps_used);
    const float inv_sqrt_h = 1.0f / sqrtf((float)H);
    for (uint32_t rr = 0; rr < 32; ++rr) {
        const uint32_t r = r0 + rr;
        const float norm = __shfl_sync(0xffffffffu, my_norm, rr);
        if (r >= rows) break;  // uniform across the warp
        for (uint32_t c = lane; c < H; c += 32) {
            const float v = in[(uint64_t)r * H + c];
            float o;
            if (mode == 1) {
                const float s = w_count == 1 ? w[0] : (w_count >= H ? w[c] : 1.0f);
                o = __fmul_rn(__fmul_rn(__fmul_rn(v, norm), s), inv_sqrt_h);
            } else {
                o = __fmul_rn(__fmul_rn(v, norm), unit_offset ? __fadd_rn(1.0f, w[c]) : w[c]);
            }
            if (out_f32) out_f32[(uint64_t)r * H + c] = o;
            if (out_bf16) out_bf16[(uint64_t)r * H + c] = f32_to_bf16_bits(o);
        }
    }
}

cudaError_t launch_row_norm_exact(const float* in, uint32_t rows, uint32_t H, const float* w, uint64_t w_count,
                                  int mode, float eps, int unit_offset, float* out_f32, uint16_t* out_bf16,
                                  cudaStream_t st) {
    if (rows == 0) return cudaSuccess;
    row_norm_exact_kernel<<<ceil_div(rows, 32), 32, 0, st>>>(in, rows, H, w, w_count, mode, eps, unit_offset, out_f32,
                                                           out_bf16);
    return cudaGetLastError();
}

// Block-wide sum of squares of v[0, H) in double (parallel order).
__device__ float block_rms_norm(const float* v, uint32_t H, float eps, double* red) {
    double ss = 0.0;
    for (uint32_t c = threadIdx.x; c < H; c += blockDim.x) ss = __fma_rn((double)v[c], (double)v[c], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    double t = 0.0;
    for (uint32_t i = 0; i < blockDim.x / 32; ++i) t += red[i];
    return 1.0f / sqrtf(__double2float_rn(t / (double)H) + (eps > 0.0f ? eps : 1.0e-6f));
}

// One block per token; mlp (H floats) and the row being normed (H floats)
// in shared memory.
__global__ void __launch_bounds__(512) block_combine_kernel(const float* __restrict__ yp, uint32_t H,
                                                            const uint32_t* __restrict__ pos_of,
                                                            const int32_t* __restrict__ ids,
                                                            const float* __restrict__ w, uint32_t T, uint32_t K,
                                                            uint32_t E, const float* __restrict__ ys,
                                                            const float* __restrict__ gate, BlockParts bp,
                                                            uint16_t* __restrict__ y_bf16,
                                                            float* __restrict__ y_f32) {
    extern __shared__ float sm[];
    float* mlp = sm;          // [H]
    float* row = sm + H;      // [H]
    __shared__ double red[16];
    const uint32_t t = blockIdx.x;
    pdl_wait();
    auto norm_row = [&](const float* src, const float* nw) {
        // row = RMSNorm(src) * (nw or 1 + nw), or src itself
        for (uint32_t c = threadIdx.x; c < H; c += blockDim.x) row[c] = src[c];
        if (nw) {
            __syncthreads();
            const float n = block_rms_norm(row, H, bp.eps, red);
            __syncthreads();
            for (uint32_t c = threadIdx.x; c < H; c += blockDim.x)
                row[c] = __fmul_rn(__fmul_rn(row[c], n), bp.unit_offset ? __fadd_rn(1.0f, nw[c]) : nw[c]);
        }
        __syncthreads();
    };
    for (uint32_t c = threadIdx.x; c < H; c += blockDim.x) mlp[c] = 0.0f;
    if (ys) {
        norm_row(ys + (uint64_t)t * H, bp.post_norm1);
        const float g = gate ? gate[t] : 1.0f;
        for (uint32_t c = threadIdx.x; c < H; c += blockDim.x) mlp[c] = __fmaf_rn(row[c], g, mlp[c]);
        __syncthreads();
    }
    for (uint32_t j = 0; j < K; ++j) {
        const uint64_t a = (uint64_t)t * K + j;
        const uint32_t e = (uint32_t)ids[a];
        norm_row(yp + (uint64_t)pos_of[a] * H, bp.post_norm2);
        const float wj = w[a];
        const uint64_t n = bp.down_scale_count;
        for (uint32_t c = threadIdx.x; c < H; c += blockDim.x) {
            float v = row[c];
            if (bp.down_scale && n) {
                if (n == 1) v = __fmul_rn(v, bp.down_scale[0]);
                else if (n == E && e < E) v = __fmul_rn(v, bp.down_scale[e]);
                else if ((uint64_t)e * H <= n && H <= n - (uint64_t)e * H) v = __fmul_rn(v, bp.down_scale[(uint64_t)e * H + c]);
            }
            mlp[c] = __fmaf_rn(wj, v, mlp[c]);
        }
        __syncthreads();
    }
    float n_out = 1.0f;
    if (bp.post_norm) n_out = block_rms_norm(mlp, H, bp.eps, red);
    for (uint32_t c = threadIdx.x; c < H; c += blockDim.x) {
        float o = mlp[c];
        if (bp.post_norm) o = __fmul_rn(__fmul_rn(o, n_out), bp.unit_offset ? __fadd_rn(1.0f, bp.post_norm[c]) : bp.post_norm[c]);
        if (y_f32) y_f32[(uint64_t)t * H + c] = o;
        if (y_bf16) y_bf16[(uint64_t)t * H + c] = f32_to_bf16_bits(o);
    }
}

cudaError_t launch_block_combine(const float* yp, uint32_t H, const uint32_t* pos_of, const int32_t* ids,
                                 const float* w, uint32_t T, uint32_t K, uint32_t E, const float* ys,
                                 const float* gate, const BlockParts& bp, uint16_t* y_bf16, float* y_f32,
                                 cudaStream_t st, bool pdl) {
    if (T == 0) return cudaSuccess;
    const size_t smem = (size_t)2 * H * sizeof(float);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    static uint64_t attr_set = 0;  // one bit per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && !((attr_set >> dev) & 1u)) {
        e = cudaFuncSetAttribute(block_combine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        attr_set |= 1ull << dev;
    }
    return launch_kernel(block_combine_kernel, dim3(T), dim3(512), smem, st, pdl, yp, H, pos_of, ids, w, T, K, E, ys,
                         gate, bp, y_bf16, y_f32);
}

}  // namespace moe_b200
