// One-time repack of the reference's GGUF MXFP4 expert bytes into the
// TMA-friendly tile layout described in common.cuh ("wtile").
//
// The reference stores each expert projection as rows of ceil(K/32) 17-byte
// blocks (tensor_layout.cpp.inc:174-176; decode order
// tensor_dot_cpu_kernels.cpp.inc:576-599).  Row strides such as 1530 B are
// not 16-byte multiples, so the bytes cannot be tiled by TMA or bulk copies
// directly; they are rewritten once when an expert becomes resident.
#include "common.cuh"
#include "kernels.h"

namespace moe_b200 {

// One thread per output code word (row r, k-tile kt, word c).
__global__ void repack_mxfp4_kernel(const uint8_t* __restrict__ gguf, uint32_t rows, uint32_t cols,
                                    uint8_t* __restrict__ out, uint32_t row_tiles, uint32_t k_tiles,
                                    uint32_t tile_stride) {
    const uint32_t gguf_row_bytes = ceil_div(cols, 32) * 17;
    const uint64_t total_words = (uint64_t)row_tiles * k_tiles * kTileRows * 8;
    for (uint64_t idx = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; idx < total_words;
         idx += (uint64_t)gridDim.x * blockDim.x) {
        // idx = ((rt * k_tiles + kt) * 8 + c) * 128 + rr : consecutive threads
        // write consecutive words of one tile.
        const uint32_t rr = (uint32_t)(idx % kTileRows);
        const uint32_t c = (uint32_t)((idx / kTileRows) % 8);
        const uint64_t tile = idx / (kTileRows * 8);
        const uint32_t kt = (uint32_t)(tile % k_tiles);
        const uint32_t rt = (uint32_t)(tile / k_tiles);
        const uint32_t r = rt * kTileRows + rr;
        uint8_t* tile_base = out + tile * tile_stride;
        uint32_t word = 0;
        if (r < rows) {
            const uint8_t* row = gguf + (uint64_t)r * gguf_row_bytes;
            for (int e = 0; e < 8; ++e) {
                const uint32_t k = kt * kTileK + c * 8 + e;
                uint32_t code = 0;
                if (k < cols) {
                    const uint8_t* blk = row + (k / 32) * 17;
                    const uint32_t i = k % 32;
                    code = i < 16 ? (blk[1 + i] & 0x0Fu) : (blk[1 + i - 16] >> 4);
                }
#pragma unroll
                for (int b = 0; b < 4; ++b) word |= ((code >> b) & 1u) << code_bit_pos(e, b);
            }
        }
        reinterpret_cast<uint32_t*>(tile_base)[c * kTileRows + rr] = word;
        if (c < 2) {
            // scale bytes: sub-block c of this k tile
            const uint32_t k0 = kt * kTileK + c * 32;
            uint8_t s = 0;
            if (r < rows && k0 < cols) s = gguf[(uint64_t)r * gguf_row_bytes + (k0 / 32) * 17];
            tile_base[kTileCodeBytes + c * kTileRows + rr] = s;
        }
    }
}

// Decodes repacked tiles back to bf16 [rows x cols] with the same arithmetic
// the GEMM converters use (e2m1_pair_bits and the two E8M0 factors).  Used
// by the tests to prove the decode is exact.
__global__ void dequant_wtiles_kernel(const uint8_t* __restrict__ tiles, uint32_t rows, uint32_t cols,
                                      uint32_t k_tiles, uint32_t tile_stride, uint16_t* __restrict__ out) {
    const uint64_t total = (uint64_t)rows * ceil_div(cols, 8);
    for (uint64_t idx = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t r = (uint32_t)(idx / ceil_div(cols, 8));
        const uint32_t k8 = (uint32_t)(idx % ceil_div(cols, 8)) * 8;
        const uint32_t kt = k8 / kTileK;
        const uint32_t c = (k8 % kTileK) / 8;
        const uint8_t* tile = tiles + ((uint64_t)(r / kTileRows) * k_tiles + kt) * tile_stride;
        const uint32_t rr = r % kTileRows;
        const uint32_t w = reinterpret_cast<const uint32_t*>(tile)[c * kTileRows + rr];
        const uint32_t s = tile[kTileCodeBytes + (c / 4) * kTileRows + rr];
        const uint32_t f1 = e8m0_f1(s), f2 = e8m0_f2(s);
        for (int i = 0; i < 4; ++i) {
            uint32_t v = bf16x2_mul(e2m1_pair_bits(w, i), f1);
            if (s > 128u) v = bf16x2_mul(v, f2);
            const uint32_t k = k8 + 2 * i;
            if (k < cols) out[(uint64_t)r * cols + k] = (uint16_t)(v & 0xFFFF);
            if (k + 1 < cols) out[(uint64_t)r * cols + k + 1] = (uint16_t)(v >> 16);
        }
    }
}

static int grid_for(uint64_t work, int threads) {
    const uint64_t blocks = (work + threads - 1) / threads;
    return (int)(blocks < 148 * 16 ? (blocks ? blocks : 1) : 148 * 16);
}

// `tile_stride` is the distance between consecutive tiles: kTileBytes for a
// lone matrix, 2 * kTileBytes when gate and up tiles are interleaved.
cudaError_t launch_repack_mxfp4(const uint8_t* gguf, uint32_t rows, uint32_t cols, uint8_t* out,
                                uint32_t tile_stride, cudaStream_t stream) {
    const uint32_t rt = ceil_div(rows, kTileRows), kt = ceil_div(cols, kTileK);
    const uint64_t words = (uint64_t)rt * kt * kTileRows * 8;
    repack_mxfp4_kernel<<<grid_for(words, 256), 256, 0, stream>>>(gguf, rows, cols, out, rt, kt, tile_stride);
    return cudaGetLastError();
}

cudaError_t launch_dequant_wtiles(const uint8_t* tiles, uint32_t rows, uint32_t cols, uint32_t tile_stride,
                                  uint16_t* out, cudaStream_t stream) {
    const uint64_t work = (uint64_t)rows * ceil_div(cols, 8);
    dequant_wtiles_kernel<<<grid_for(work, 256), 256, 0, stream>>>(tiles, rows, cols, ceil_div(cols, kTileK),
                                                                   tile_stride, out);
    return cudaGetLastError();
}

}  // namespace moe_b200
