// GPU form of moe_pc_group_tokens_by_expert (token_grouping.cpp.inc:1-83):
// an LSD radix sort of (layer, expert, token_index) with 8-bit digits, each
// pass the same deterministic stable counting sort as the layer's
// permutation, then a device run-length scan into batches.
#include "common.cuh"
#include "kernels.h"

namespace moe_b200 {

__global__ void iota_kernel(uint32_t* v, uint32_t n) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) v[i] = i;
}

__global__ void digit_kernel(const AssignRec* __restrict__ a, const uint32_t* __restrict__ order, uint32_t n,
                             int field, int shift, int32_t* __restrict__ keys) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const AssignRec r = a[order[i]];
    const uint32_t v = field == 0 ? r.token_index : (field == 1 ? r.expert : r.layer);
    keys[i] = (int32_t)((v >> shift) & 0xFFu);
}

__global__ void scatter_order_kernel(const int32_t* __restrict__ keys, uint32_t n, uint32_t nb,
                                     const uint32_t* __restrict__ tile_base, const uint32_t* __restrict__ rank,
                                     const uint32_t* __restrict__ offset, const uint32_t* __restrict__ order_in,
                                     uint32_t* __restrict__ order_out) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t b = (uint32_t)keys[i];
    const uint32_t pos = offset[b] + tile_base[(uint64_t)(i / 2048) * nb + b] + rank[i];
    order_out[pos] = order_in[i];
}

__global__ void gather_sorted_kernel(const AssignRec* __restrict__ a, const uint32_t* __restrict__ order, uint32_t n,
                                     AssignRec* __restrict__ out) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = a[order[i]];
}

// One block: head flags where (layer, expert) changes, a block-wide scan to
// number the batches, then batch sizes from consecutive heads.
__global__ void __launch_bounds__(1024) batches_kernel(const AssignRec* __restrict__ s, uint32_t n,
                                                       uint32_t* __restrict__ batches, uint32_t* __restrict__ count) {
    __shared__ uint32_t warp_sums[32];
    __shared__ uint32_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (uint32_t c0 = 0; c0 < n; c0 += blockDim.x) {
        const uint32_t i = c0 + threadIdx.x;
        uint32_t head = 0;
        if (i < n) head = (i == 0 || s[i].layer != s[i - 1].layer || s[i].expert != s[i - 1].expert) ? 1u : 0u;
        uint32_t x = head;
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
            if ((threadIdx.x & 31) >= o) x += y;
        }
        if ((threadIdx.x & 31) == 31) warp_sums[threadIdx.x >> 5] = x;
        __syncthreads();
        if (threadIdx.x < 32) {
            uint32_t v = warp_sums[threadIdx.x];
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, v, o);
                if (threadIdx.x >= o) v += y;
            }
            warp_sums[threadIdx.x] = v;
        }
        __syncthreads();
        const uint32_t incl = x + ((threadIdx.x >= 32) ? warp_sums[(threadIdx.x >> 5) - 1] : 0) + carry;
        if (head) {
            const uint32_t b = incl - 1;
            batches[b * 4 + 0] = s[i].layer;
            batches[b * 4 + 1] = s[i].expert;
            batches[b * 4 + 2] = i;
        }
        __syncthreads();
        if (threadIdx.x == 0) carry += warp_sums[31];
        __syncthreads();
    }
    const uint32_t nb = carry;
    for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) {
        const uint32_t end = (b + 1 < nb) ? batches[(b + 1) * 4 + 2] : n;
        batches[b * 4 + 3] = end - batches[b * 4 + 2];
    }
    if (threadIdx.x == 0) *count = nb;
}

cudaError_t launch_iota(uint32_t* v, uint32_t n, cudaStream_t st) {
    iota_kernel<<<ceil_div(n, 256), 256, 0, st>>>(v, n);
    return cudaGetLastError();
}

cudaError_t launch_group_pass(const AssignRec* a, const uint32_t* order_in, uint32_t* order_out, uint32_t n,
                              int field, int shift, int32_t* keys, uint32_t* tile_counts, uint32_t* rank,
                              GroupInfo gi, uint32_t* err, cudaStream_t st) {
    digit_kernel<<<ceil_div(n, 256), 256, 0, st>>>(a, order_in, n, field, shift, keys);
    cudaError_t e = launch_sort_count(keys, n, 256, tile_counts, rank, err, st);
    if (e != cudaSuccess) return e;
    e = launch_sort_scan(tile_counts, sort_tiles(n), 256, gi, st);
    if (e != cudaSuccess) return e;
    scatter_order_kernel<<<ceil_div(n, 256), 256, 0, st>>>(keys, n, 256, tile_counts, rank, gi.offset, order_in,
                                                           order_out);
    return cudaGetLastError();
}

cudaError_t launch_group_finish(const AssignRec* a, const uint32_t* order, uint32_t n, AssignRec* sorted,
                                uint32_t* batches, uint32_t* batch_count, cudaStream_t st) {
    gather_sorted_kernel<<<ceil_div(n, 256), 256, 0, st>>>(a, order, n, sorted);
    batches_kernel<<<1, 1024, 0, st>>>(sorted, n, batches, batch_count);
    return cudaGetLastError();
}

}  // namespace moe_b200
