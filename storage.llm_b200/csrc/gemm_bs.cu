// Block-scaled tcgen05 grouped GEMMs: the tensor core consumes the MXFP4
// weights as they are stored -- E2M1 codes plus one E8M0 scale per 32 K --
// so no SM instruction is spent decoding weights.
//
//   A  E2M1 weight codes, packed two per byte in HBM, TMA'd with the
//      16U4_ALIGN16B type (each 16 codes land in 16 bytes of shared memory,
//      the operand form kind::mxf8f6f4 reads), 128 rows x 128 K per box;
//   SFA the rows' E8M0 scales, one 512-byte block per 128 x 128 tile laid out
//      as tcgen05.cp.32x128b.warpx4 expects (row r, K block j at byte
//      (r%32)*16 + (r/32)*4 + j), copied to TMEM each stage;
//   B  activations as two E4M3 terms, hi and lo, each with its own E8M0
//      scale per 32 K (SFB).  A bf16 value has 8 significant bits and splits
//      exactly into hi (4 bits) + lo (4 bits), so W.x = W.x_hi + W.x_lo is
//      the same product the bf16 path computes;
//   D  fp32 in TMEM: per K step, MMA(A, B_hi) then MMA(A, B_lo) accumulate.
//
// kGateUp: gate and up tiles of the same 128 intermediate rows share B; the
//          epilogue computes h = SiLU(gate) * up and writes it already split
//          into hi/lo E4M3 + scales (a warp's 32 rows are one 32-element K
//          block of the down GEMM), so the down GEMM reads it directly.
// kDown:   the epilogue writes fp32 expert outputs for the combine.
//
// Warp roles (192 threads, one CTA per SM, persistent over all tiles):
//   warp 0     producer: TMA of the A and B boxes and bulk copies of the
//              weight and activation scale blocks -- all asynchronous, so a
//              stage costs the producer no memory round trip
//   warp 1     TMEM owner, scale-factor copies and MMA issue
//   warps 2-5  epilogue, one TMEM lane quarter each
// All waits are bounded and report through p.err.
#include <cuda_fp8.h>

#include "common.cuh"
#include "kernels.h"

namespace moe_b200 {

template <int MODE, int BN>
struct BsCfg {
    static constexpr int kNA = MODE == kGateUp ? 2 : 1;       // A operands per stage
    static constexpr int kABytes = 128 * 128;                 // smem bytes per A box
    static constexpr int kATx = 128 * 128 / 2;                // packed bytes the A box moves
    static constexpr int kBBytes = BN * 128;                  // smem bytes per B term (hi or lo)
    static constexpr int kSF = 512;
    static constexpr int kStageBytes = kNA * kABytes + 2 * kBBytes + (kNA + 2) * kSF;
    static constexpr int kStages = (200 * 1024) / kStageBytes;
    static constexpr int kAccCols = kNA * BN;
    static constexpr int kAccs = 256 / kAccCols >= 2 ? 2 : 1;
    static constexpr int kSFCols = (kNA + 2) * 4;             // TMEM columns of scale factors per stage
    static constexpr int kSmem = kStages * kStageBytes + 2048 /*two 1024 alignments*/ + 512 /*barriers*/;
    static_assert(kStages >= 3, "pipeline too shallow");
    static_assert(256 + kStages * kSFCols <= 512, "TMEM budget");
};

__device__ __forceinline__ float pow2f(int e) {
    // exact 2^e for e in [-127, 127]
    return e >= -126 ? __int_as_float((e + 127) << 23) : __int_as_float(0x00400000);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Scale exponent for a 32-value block with absolute maximum `amax`: the block
// maps into [128, 256) of E4M3's range (no overflow; E4M3 keeps 4 significant
// bits anywhere in its normal range, so the exact choice costs no precision).
__device__ __forceinline__ int block_exp(float amax) {
    if (!(amax > 0.f)) return -127;
    const int e = (int)((__float_as_uint(amax) >> 23) & 0xFF) - 127 - 7;
    return e < -127 ? -127 : (e > 127 ? 127 : e);
}

__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
    const __half_raw hr = __nv_cvt_fp8_to_halfraw(b, __NV_E4M3);
    return __half2float(__half(hr));
}

// Splits the 32 values held by a warp (one per lane, one 32-element K block)
// into hi + lo E4M3 terms with E8M0 scale bytes.  Warp-collective.
__device__ __forceinline__ void split_e4m3_warp(float v, uint8_t& hi, uint8_t& lo, uint8_t& s_hi, uint8_t& s_lo) {
    const int e1 = block_exp(warp_max(fabsf(v)));
    hi = __nv_cvt_float_to_fp8(v * pow2f(-e1), __NV_SATFINITE, __NV_E4M3);
    const float r = v - e4m3_to_f32(hi) * pow2f(e1);
    const int e2 = block_exp(warp_max(fabsf(r)));
    lo = __nv_cvt_float_to_fp8(r * pow2f(-e2), __NV_SATFINITE, __NV_E4M3);
    s_hi = (uint8_t)(e1 + 127);
    s_lo = (uint8_t)(e2 + 127);
}

// ---------------------------------------------------------------------------
// Activation quantisation: one warp per (token, 32-element block).
//   q_hi/q_lo [T][Kp] E4M3 bytes, s_hi/s_lo [T][Kp/32] E8M0 bytes.
// ---------------------------------------------------------------------------
__global__ void quantize_rows_kernel(const uint16_t* __restrict__ x, uint32_t T, uint32_t H, uint32_t Kp,
                                     uint8_t* __restrict__ q_hi, uint8_t* __restrict__ q_lo,
                                     uint8_t* __restrict__ s_hi, uint8_t* __restrict__ s_lo) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t nblk = Kp / 32;
    const uint64_t total = (uint64_t)T * nblk;
    const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
    for (uint64_t wb = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; wb < total; wb += warps) {
        const uint32_t t = (uint32_t)(wb / nblk), b = (uint32_t)(wb % nblk);
        const uint32_t k = b * 32 + lane;
        const float v = k < H ? bf16_bits_to_f32(x[(uint64_t)t * H + k]) : 0.f;
        uint8_t hi, lo, sh, sl;
        split_e4m3_warp(v, hi, lo, sh, sl);
        q_hi[(uint64_t)t * Kp + k] = hi;
        q_lo[(uint64_t)t * Kp + k] = lo;
        if (lane == 0) {
            s_hi[(uint64_t)t * nblk + b] = sh;
            s_lo[(uint64_t)t * nblk + b] = sl;
        }
    }
}

// Permuted rows for the block-scaled GEMM: the E4M3 bytes of each row's token
// and its scale bytes, the latter written straight into the scale blocks the
// GEMM's producer bulk-copies: one 1024-byte block per (token tile, 128-K
// stage) holding the hi block then the lo block, row r of the tile at byte
// (r%32)*16 + (r/32)*4 + j for K block j -- the tcgen05.cp.32x128b layout.
// Token tile t of group g is tile_off[g]/m_tiles + (row - offset[g]) / BN.
__global__ void gather_bs_kernel(const uint8_t* __restrict__ q_hi, const uint8_t* __restrict__ q_lo,
                                 const uint8_t* __restrict__ s_hi, const uint8_t* __restrict__ s_lo, uint32_t Kp,
                                 const uint32_t* __restrict__ row_token, uint32_t rows,
                                 const uint32_t* __restrict__ offset, const uint32_t* __restrict__ tile_off,
                                 uint32_t groups, uint32_t m_tiles, uint32_t block_n, uint8_t* __restrict__ x_hi,
                                 uint8_t* __restrict__ x_lo, uint8_t* __restrict__ sf_atoms) {
    const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t nv = Kp / 16, nkt = Kp / 128;
    for (uint32_t r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
        const uint32_t t = row_token[r];
        const uint4* sh = reinterpret_cast<const uint4*>(q_hi + (uint64_t)t * Kp);
        const uint4* sl = reinterpret_cast<const uint4*>(q_lo + (uint64_t)t * Kp);
        uint4* dh = reinterpret_cast<uint4*>(x_hi + (uint64_t)r * Kp);
        uint4* dl = reinterpret_cast<uint4*>(x_lo + (uint64_t)r * Kp);
        for (uint32_t v = lane; v < nv; v += 32) {
            dh[v] = __ldg(sh + v);
            dl[v] = __ldg(sl + v);
        }
        uint32_t lo = 0, hi = groups;  // group owning row r
        while (hi - lo > 1) {
            const uint32_t mid = (lo + hi) >> 1;
            if (offset[mid] <= r) lo = mid;
            else hi = mid;
        }
        const uint32_t n = r - offset[lo];
        const uint64_t tile = tile_off[lo] / m_tiles + n / block_n;
        const uint32_t rr = n % block_n;
        const uint32_t pos = (rr % 32) * 16 + (rr / 32) * 4;
        const uint32_t* wh = reinterpret_cast<const uint32_t*>(s_hi + (uint64_t)t * (Kp / 32));
        const uint32_t* wl = reinterpret_cast<const uint32_t*>(s_lo + (uint64_t)t * (Kp / 32));
        for (uint32_t kt = lane; kt < nkt; kt += 32) {
            uint8_t* atom = sf_atoms + (tile * nkt + kt) * 1024;
            *reinterpret_cast<uint32_t*>(atom + pos) = __ldg(wh + kt);
            *reinterpret_cast<uint32_t*>(atom + 512 + pos) = __ldg(wl + kt);
        }
    }
}

// ---------------------------------------------------------------------------
// Weight repack for the block-scaled path (once per expert at upload).
//   codes: row r of the matrix at codes + r * Kp/2, element 2j in the low
//          nibble of byte j (zero past `cols`);
//   sfa:   [row_tile][k_tile][512] scale blocks in the tcgen05.cp layout.
// ---------------------------------------------------------------------------
__global__ void repack_bs_kernel(const uint8_t* __restrict__ gguf, uint32_t rows, uint32_t cols, uint32_t rows_pad,
                                 uint32_t Kp, uint8_t* __restrict__ codes, uint8_t* __restrict__ sfa) {
    const uint32_t gguf_row_bytes = ceil_div(cols, 32) * 17;
    const uint32_t kt_n = Kp / 128;
    const uint64_t nbytes = (uint64_t)rows_pad * (Kp / 2);
    const uint64_t nsf = (uint64_t)rows_pad * (Kp / 32);
    for (uint64_t idx = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; idx < nbytes + nsf;
         idx += (uint64_t)gridDim.x * blockDim.x) {
        if (idx < nbytes) {
            const uint32_t r = (uint32_t)(idx / (Kp / 2));
            const uint32_t j = (uint32_t)(idx % (Kp / 2));
            uint32_t b = 0;
            if (r < rows) {
                const uint8_t* row = gguf + (uint64_t)r * gguf_row_bytes;
                for (int h = 0; h < 2; ++h) {
                    const uint32_t k = 2 * j + h;
                    if (k < cols) {
                        const uint8_t* blk = row + (k / 32) * 17;
                        const uint32_t i = k % 32;
                        const uint32_t code = i < 16 ? (blk[1 + i] & 0x0Fu) : (blk[1 + i - 16] >> 4);
                        b |= code << (4 * h);
                    }
                }
            }
            codes[idx] = (uint8_t)b;
        } else {
            const uint64_t q = idx - nbytes;
            const uint32_t r = (uint32_t)(q / (Kp / 32));
            const uint32_t blk = (uint32_t)(q % (Kp / 32));
            uint8_t s = 0;
            if (r < rows && blk * 32 < cols) s = gguf[(uint64_t)r * gguf_row_bytes + blk * 17];
            const uint32_t mt = r / 128, rr = r % 128, kt = blk / 4, j = blk % 4;
            sfa[((uint64_t)mt * kt_n + kt) * 512 + (rr % 32) * 16 + (rr / 32) * 4 + j] = s;
        }
    }
}

cudaError_t launch_repack_bs(const uint8_t* gguf, uint32_t rows, uint32_t cols, uint32_t rows_pad, uint32_t Kp,
                             uint8_t* codes, uint8_t* sfa, cudaStream_t st) {
    const uint64_t work = (uint64_t)rows_pad * (Kp / 2) + (uint64_t)rows_pad * (Kp / 32);
    const uint64_t blocks = (work + 255) / 256;
    repack_bs_kernel<<<(unsigned)(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, st>>>(gguf, rows, cols, rows_pad,
                                                                                       Kp, codes, sfa);
    return cudaGetLastError();
}

cudaError_t launch_quantize_rows(const uint16_t* x, uint32_t T, uint32_t H, uint32_t Kp, uint8_t* q_hi,
                                 uint8_t* q_lo, uint8_t* s_hi, uint8_t* s_lo, cudaStream_t st) {
    if (T == 0) return cudaSuccess;
    const uint64_t warps = (uint64_t)T * (Kp / 32);
    const uint64_t blocks = (warps + 7) / 8;
    quantize_rows_kernel<<<(unsigned)(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, st>>>(x, T, H, Kp, q_hi, q_lo,
                                                                                           s_hi, s_lo);
    return cudaGetLastError();
}

cudaError_t launch_gather_bs(const uint8_t* q_hi, const uint8_t* q_lo, const uint8_t* s_hi, const uint8_t* s_lo,
                             uint32_t Kp, const uint32_t* row_token, uint32_t rows, const uint32_t* offset,
                             const uint32_t* tile_off, uint32_t groups, uint32_t m_tiles, uint32_t block_n,
                             uint8_t* x_hi, uint8_t* x_lo, uint8_t* sf_atoms, cudaStream_t st) {
    if (rows == 0) return cudaSuccess;
    const uint32_t blocks = min(ceil_div(rows, 8), 148u * 8u);
    gather_bs_kernel<<<blocks, 256, 0, st>>>(q_hi, q_lo, s_hi, s_lo, Kp, row_token, rows, offset, tile_off, groups,
                                             m_tiles, block_n, x_hi, x_lo, sf_atoms);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// The grouped GEMM
// ---------------------------------------------------------------------------
struct BsTile {
    uint32_t g, mt, n0, nn;
};

template <int BN>
__device__ __forceinline__ void bs_tile_coord(const BsParams& p, uint32_t tile, BsTile& tc) {
    uint32_t lo = 0, hi = p.groups;
    while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (p.tile_off[mid] <= tile) lo = mid;
        else hi = mid;
    }
    const uint32_t local = tile - p.tile_off[lo];
    const uint32_t cnt = p.count[lo];
    const uint32_t ntn = ceil_div(cnt, BN);
    tc.g = lo;
    tc.mt = local / ntn;
    tc.n0 = (local % ntn) * BN;
    tc.nn = min((uint32_t)BN, cnt - tc.n0);
}

__device__ __forceinline__ float silu_fast(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

template <int MODE, int BN>
__global__ void __launch_bounds__(192, 1) gemm_bs_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                                         const __grid_constant__ CUtensorMap tmap_b_hi,
                                                         const __grid_constant__ CUtensorMap tmap_b_lo,
                                                         const BsParams p) {
    using C = BsCfg<MODE, BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // scale-factor blocks first (small), then the 1024-aligned operand tiles
    uint8_t* sf_base = smem;                                                  // [stages][kNA+2][512]
    uint8_t* a_base = smem + C::kStages * (C::kNA + 2) * C::kSF;              // [stages][kNA][16 KB]
    a_base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(a_base) + 1023) & ~uintptr_t(1023));
    uint8_t* b_base = a_base + C::kStages * C::kNA * C::kABytes;              // [stages][2][kBBytes]
    uint64_t* bars = reinterpret_cast<uint64_t*>(b_base + C::kStages * 2 * C::kBBytes);
    uint64_t* load_full = bars;
    uint64_t* load_empty = load_full + C::kStages;
    uint64_t* acc_full = load_empty + C::kStages;
    uint64_t* acc_empty = acc_full + C::kAccs;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + C::kAccs);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < C::kStages; ++i) {
            mbar_init(&load_full[i], 1);
            mbar_init(&load_empty[i], 1);
        }
        for (int i = 0; i < C::kAccs; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 128);
        }
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b_hi);
        prefetch_tmap(&tmap_b_lo);
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    const uint32_t total = p.tile_off[p.groups];
    constexpr uint32_t kSfCol0 = 256;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        uint32_t stage = 0, phase = 0;
        bool ok = true;
        for (uint32_t tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
            BsTile tc;
            bs_tile_coord<BN>(p, tile, tc);
            const uint32_t row0 = p.offset[tc.g] + tc.n0;
            const uint32_t n_sub = ceil_div(tc.nn, 32);
            const uint32_t ntile = p.tile_off[tc.g] / p.m_tiles + tc.n0 / BN;
            for (uint32_t kt = 0; kt < p.k_tiles; ++kt) {
                ok = mbar_wait(&load_empty[stage], phase ^ 1, p.err, kErrTimeoutLoadEmpty);
                if (!__all_sync(0xffffffffu, ok)) {
                    ok = false;
                    break;
                }
                uint8_t* sf = sf_base + stage * (C::kNA + 2) * C::kSF;
                if (lane == 0) {
                    mbar_arrive_expect_tx(&load_full[stage],
                                          C::kNA * (C::kATx + C::kSF) + 2 * C::kSF + 2 * n_sub * 32 * 128);
                    // activation scales: hi and lo blocks of this token tile and stage
                    bulk_g2s(sf + C::kNA * C::kSF, p.sfb_atoms + ((uint64_t)ntile * p.k_tiles + kt) * 1024,
                             2 * C::kSF, &load_full[stage]);
#pragma unroll
                    for (int pj = 0; pj < C::kNA; ++pj) {
                        const int32_t arow = (int32_t)(((uint64_t)tc.g * C::kNA + pj) * p.rows_pad + tc.mt * 128);
                        tma_load_2d(a_base + (stage * C::kNA + pj) * C::kABytes, &tmap_a, (int32_t)(kt * 128), arow,
                                    &load_full[stage]);
                        const uint8_t* sfa_src =
                            p.sfa + ((((uint64_t)tc.g * C::kNA + pj) * p.m_tiles + tc.mt) * p.k_tiles + kt) * 512;
                        bulk_g2s(sf + pj * C::kSF, sfa_src, C::kSF, &load_full[stage]);
                    }
                    uint8_t* bh = b_base + stage * 2 * C::kBBytes;
                    for (uint32_t sb = 0; sb < n_sub; ++sb) {
                        tma_load_2d(bh + sb * 32 * 128, &tmap_b_hi, (int32_t)(kt * 128), (int32_t)(row0 + sb * 32),
                                    &load_full[stage]);
                        tma_load_2d(bh + C::kBBytes + sb * 32 * 128, &tmap_b_lo, (int32_t)(kt * 128),
                                    (int32_t)(row0 + sb * 32), &load_full[stage]);
                    }
                }
                __syncwarp();
                if (++stage == C::kStages) {
                    stage = 0;
                    phase ^= 1;
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, acc = 0, accphase = 0;
            bool ok = true;
            for (uint32_t tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
                BsTile tc;
                bs_tile_coord<BN>(p, tile, tc);
                const uint32_t n_mma = max(16u, (tc.nn + 15u) & ~15u);
                if (!(ok = mbar_wait(&acc_empty[acc], accphase ^ 1, p.err, kErrTimeoutAccEmpty))) break;
                tc_fence_after();
                const uint32_t d0 = tmem + acc * C::kAccCols;
                for (uint32_t kt = 0; kt < p.k_tiles; ++kt) {
                    if (!(ok = mbar_wait(&load_full[stage], phase, p.err, kErrTimeoutLoadFull))) break;
                    tc_fence_after();
                    const uint8_t* sf = sf_base + stage * (C::kNA + 2) * C::kSF;
                    const uint32_t sfc = tmem + kSfCol0 + stage * C::kSFCols;
#pragma unroll
                    for (int q = 0; q < C::kNA + 2; ++q) tmem_cp_sf(sfc + q * 4, smem_desc_sf(smem_u32(sf + q * C::kSF)));
                    const uint32_t a_addr = smem_u32(a_base + stage * C::kNA * C::kABytes);
                    const uint32_t bh_addr = smem_u32(b_base + stage * 2 * C::kBBytes);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint32_t idesc = idesc_bs_m128(n_mma, kk);
                        const uint64_t bhi = smem_desc_sw128(bh_addr + kk * 32);
                        const uint64_t blo = smem_desc_sw128(bh_addr + C::kBBytes + kk * 32);
#pragma unroll
                        for (int pj = 0; pj < C::kNA; ++pj) {
                            const uint64_t adesc = smem_desc_sw128(a_addr + pj * C::kABytes + kk * 32);
                            const uint32_t d = d0 + pj * BN;
                            mma_bs(d, adesc, bhi, idesc, sfc + pj * 4, sfc + C::kNA * 4, (kt | kk) != 0);
                            mma_bs(d, adesc, blo, idesc, sfc + pj * 4, sfc + C::kNA * 4 + 4, 1);
                        }
                    }
                    mma_commit(&load_empty[stage]);
                    if (++stage == C::kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                mma_commit(&acc_full[acc]);
                if (++acc == C::kAccs) {
                    acc = 0;
                    accphase ^= 1;
                }
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const uint32_t quarter = warp & 3;
        const uint32_t r = quarter * 32 + lane;
        const uint32_t lane_addr = (quarter * 32) << 16;
        uint32_t acc = 0, accphase = 0;
        bool ok = true;
        for (uint32_t tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
            BsTile tc;
            bs_tile_coord<BN>(p, tile, tc);
            ok = mbar_wait(&acc_full[acc], accphase, p.err, kErrTimeoutAccFull, true);
            if (!__all_sync(0xffffffffu, ok)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t m = tc.mt * 128 + r;
            const uint64_t row0 = p.offset[tc.g] + tc.n0;
            const uint32_t dbase = tmem + lane_addr + acc * C::kAccCols;
            // scale block of the down GEMM for this token tile and 128-K stage (= mt)
            uint8_t* h_atom = MODE == kGateUp
                                  ? p.sfh_atoms + (((uint64_t)p.tile_off[tc.g] / p.m_tiles + tc.n0 / BN) *
                                                       p.m_tiles + tc.mt) * 1024
                                  : nullptr;
            for (uint32_t c0 = 0; c0 < tc.nn; c0 += 32) {
                uint32_t d[32];
                MOE_TMEM_LD32(dbase + c0, d);
                if (MODE == kGateUp) {
                    uint32_t u[32];
                    MOE_TMEM_LD32(dbase + BN + c0, u);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const uint32_t col = c0 + i;
                        if (col >= tc.nn) continue;  // uniform across the warp
                        const float hv = silu_fast(__uint_as_float(d[i])) * __uint_as_float(u[i]);
                        uint8_t hi, lo, sh, sl;
                        split_e4m3_warp(hv, hi, lo, sh, sl);
                        const uint64_t prow = row0 + col;
                        p.h_hi[prow * p.h_stride + m] = hi;
                        p.h_lo[prow * p.h_stride + m] = lo;
                        if (lane == 0) {
                            const uint32_t pos = (col % 32) * 16 + (col / 32) * 4 + quarter;
                            h_atom[pos] = sh;
                            h_atom[512 + pos] = sl;
                        }
                    }
                } else {
                    tmem_wait_ld();
                    if (m < p.m_valid) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            if (c0 + i < tc.nn) p.y_out[(row0 + c0 + i) * p.y_stride + m] = __uint_as_float(d[i]);
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[acc]);
            if (++acc == C::kAccs) {
                acc = 0;
                accphase ^= 1;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

template <int MODE, int BN>
static cudaError_t launch_bs_mode(const CUtensorMap& ta, const CUtensorMap& tbh, const CUtensorMap& tbl,
                                  const BsParams& p, int num_sms, cudaStream_t st) {
    using C = BsCfg<MODE, BN>;
    static uint64_t attr_set = 0;  // one bit per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && !((attr_set >> dev) & 1u)) {
        e = cudaFuncSetAttribute(gemm_bs_kernel<MODE, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
        if (e != cudaSuccess) return e;
        attr_set |= 1ull << dev;
    }
    gemm_bs_kernel<MODE, BN><<<num_sms, 192, C::kSmem, st>>>(ta, tbh, tbl, p);
    return cudaGetLastError();
}

cudaError_t launch_gemm_bs(int mode, int block_n, const CUtensorMap& ta, const CUtensorMap& tbh,
                           const CUtensorMap& tbl, const BsParams& p, int num_sms, cudaStream_t st) {
    if (mode == kGateUp) {
        return block_n == 64 ? launch_bs_mode<kGateUp, 64>(ta, tbh, tbl, p, num_sms, st)
                             : launch_bs_mode<kGateUp, 128>(ta, tbh, tbl, p, num_sms, st);
    }
    return block_n == 64 ? launch_bs_mode<kDown, 64>(ta, tbh, tbl, p, num_sms, st)
                         : launch_bs_mode<kDown, 128>(ta, tbh, tbl, p, num_sms, st);
}

}  // namespace moe_b200
