// CUDA-core kernels over the repacked MXFP4 tiles.
//
// * gemm_simt_kernel: a plain grouped GEMM (one thread per output element)
//   that shares the tcgen05 kernels' tile decode and epilogue math.  It exists
//   to cross-check the tensor-core path in the GPU tests and is never used by
//   the layer forward.
// * triplet kernels: the fp32 single-token expert of
//   moe_pc_engine_run_expert_triplet_f32 (expert_triplet_cpu.cpp.inc:22-106).
//   Its input is an fp32 hidden vector, so it runs as a warp-per-row GEMV in
//   fp32 -- one token reads each weight once, which is HBM-bound work with no
//   use for the tensor cores.
#include "common.cuh"
#include "kernels.h"

namespace moe_b200 {

// Decodes element k (0..63) of row rr of a repacked tile to float.
__device__ __forceinline__ float tile_elem(const uint8_t* tile, uint32_t rr, uint32_t k) {
    const uint32_t w = reinterpret_cast<const uint32_t*>(tile)[(k / 8) * kTileRows + rr];
    const uint32_t s = tile[kTileCodeBytes + (k / 32) * kTileRows + rr];
    const uint32_t e = k % 8;
    uint32_t v = bf16x2_mul(e2m1_pair_bits(w, e / 2), e8m0_f1(s));
    if (s > 128u) v = bf16x2_mul(v, e8m0_f2(s));
    const uint16_t h = (e & 1) ? (uint16_t)(v >> 16) : (uint16_t)(v & 0xFFFF);
    return bf16_bits_to_f32(h);
}

template <int MODE>
__global__ void gemm_simt_kernel(const uint16_t* __restrict__ b, uint32_t b_stride, uint32_t rows,
                                 const GemmParams p, uint32_t m_rows) {
    const uint32_t m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= m_rows) return;
    for (uint32_t prow = blockIdx.y; prow < rows; prow += gridDim.y) {
    uint32_t lo = 0, hi = p.groups;  // group owning permuted row prow
    while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (p.offset[mid] <= prow) lo = mid;
        else hi = mid;
    }
    const uint32_t raw = MODE == kGateUp ? 2 * kTileBytes : kTileBytes;
    const uint8_t* wrow = p.wt + (uint64_t)lo * p.group_stride + (uint64_t)(m / kTileRows) * p.k_tiles * raw;
    const uint16_t* brow = b + (uint64_t)prow * b_stride;
    float acc0 = 0.f, acc1 = 0.f;
    for (uint32_t kt = 0; kt < p.k_tiles; ++kt) {
        const uint8_t* tile = wrow + (uint64_t)kt * raw;
        for (uint32_t k = 0; k < kTileK; ++k) {
            const float xv = bf16_bits_to_f32(brow[kt * kTileK + k]);
            acc0 = __fmaf_rn(tile_elem(tile, m % kTileRows, k), xv, acc0);
            if (MODE == kGateUp) acc1 = __fmaf_rn(tile_elem(tile + kTileBytes, m % kTileRows, k), xv, acc1);
        }
    }
    if (MODE == kGateUp) {
        const float g = acc0;
        const float hv = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), acc1);
        if (m < p.m_valid) p.h_out[(uint64_t)prow * p.h_stride + m] = f32_to_bf16_bits(hv);
    } else {
        if (m < p.m_valid) p.y_out[(uint64_t)prow * p.y_stride + m] = acc0;
    }
    }
}

cudaError_t launch_gemm_simt(int mode, const uint16_t* b, uint32_t b_stride, uint32_t rows, const GemmParams& p,
                             uint32_t m_rows, cudaStream_t st) {
    if (rows == 0) return cudaSuccess;
    dim3 grid(ceil_div(m_rows, 128), min(rows, 65535u));
    if (mode == kGateUp) gemm_simt_kernel<kGateUp><<<grid, 128, 0, st>>>(b, b_stride, rows, p, m_rows);
    else gemm_simt_kernel<kDown><<<grid, 128, 0, st>>>(b, b_stride, rows, p, m_rows);
    return cudaGetLastError();
}

// One warp per weight row; lane l covers elements l, l+32, ... of every
// 64-element tile.  gate_out receives SiLU(gate)*up and up_out receives up,
// as the reference's scratch buffers do (expert_triplet_cpu.cpp.inc:76-89).
__global__ void triplet_gate_up_kernel(const uint8_t* __restrict__ gu, const float* __restrict__ x, uint32_t H,
                                       uint32_t I, float* __restrict__ gate_out, float* __restrict__ up_out) {
    const uint32_t row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint32_t lane = threadIdx.x & 31;
    if (row >= I) return;
    const uint32_t kt_n = ceil_div(H, kTileK);
    const uint8_t* base = gu + (uint64_t)(row / kTileRows) * kt_n * 2 * kTileBytes;
    float g = 0.f, u = 0.f;
    for (uint32_t kt = 0; kt < kt_n; ++kt) {
        const uint8_t* tile = base + (uint64_t)kt * 2 * kTileBytes;
        for (uint32_t k = lane; k < kTileK; k += 32) {
            const uint32_t col = kt * kTileK + k;
            if (col < H) {
                const float xv = x[col];
                g = __fmaf_rn(tile_elem(tile, row % kTileRows, k), xv, g);
                u = __fmaf_rn(tile_elem(tile + kTileBytes, row % kTileRows, k), xv, u);
            }
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        g += __shfl_xor_sync(0xffffffffu, g, o);
        u += __shfl_xor_sync(0xffffffffu, u, o);
    }
    if (lane == 0) {
        gate_out[row] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
        up_out[row] = u;
    }
}

__global__ void triplet_down_kernel(const uint8_t* __restrict__ dn, const float* __restrict__ h, uint32_t I,
                                    uint32_t H, float* __restrict__ out) {
    const uint32_t row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint32_t lane = threadIdx.x & 31;
    if (row >= H) return;
    const uint32_t kt_n = ceil_div(I, kTileK);
    const uint8_t* base = dn + (uint64_t)(row / kTileRows) * kt_n * kTileBytes;
    float acc = 0.f;
    for (uint32_t kt = 0; kt < kt_n; ++kt) {
        const uint8_t* tile = base + (uint64_t)kt * kTileBytes;
        for (uint32_t k = lane; k < kTileK; k += 32) {
            const uint32_t col = kt * kTileK + k;
            if (col < I) acc = __fmaf_rn(tile_elem(tile, row % kTileRows, k), h[col], acc);
        }
    }
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) out[row] = acc;
}

cudaError_t launch_triplet_f32(const uint8_t* gu_tiles, const uint8_t* dn_tiles, const float* x, uint32_t H,
                               uint32_t I, float* gate_out, float* up_out, float* out, cudaStream_t st) {
    triplet_gate_up_kernel<<<ceil_div(I * 32, 256), 256, 0, st>>>(gu_tiles, x, H, I, gate_out, up_out);
    triplet_down_kernel<<<ceil_div(H * 32, 256), 256, 0, st>>>(dn_tiles, gate_out, I, H, out);
    return cudaGetLastError();
}

}  // namespace moe_b200
