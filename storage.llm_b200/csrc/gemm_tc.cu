// tcgen05 grouped GEMMs over the ragged per-expert groups.
//
// Swap-AB formulation: the MMA's M side is 128 weight rows, its N side the
// group's tokens (16..128 per tile, a runtime N per tile), so a decode-sized
// group of a few tokens wastes no tensor work on padding.
//
//   A  MXFP4 weights, decoded by converter warps straight into TMEM as bf16
//      (tcgen05.st): E2M1 code bits placed in a bf16 exponent/mantissa and
//      scaled by the E8M0 factor with one bf16x2 multiply -- exact, and the
//      decoded weights never touch shared memory;
//   B  permuted bf16 activation rows, TMA 64 x N boxes, 128-byte swizzle;
//   D  fp32 accumulators in TMEM; 4 K-steps of 16 per 64-element stage.
//
// kGateUp: one tile = 128 gate rows + the same 128 up rows (two MMAs sharing
//          B), epilogue h = SiLU(gate) * up -> bf16 permuted intermediate.
// kDown:   one tile = 128 down rows, epilogue writes fp32 expert outputs.
//
// Warp roles (704 threads, one CTA per SM, persistent over all tiles):
//   warp 0      producer: bulk copy of the raw weight tile + TMA boxes of
//               32 token rows, only as many as the tile's N needs
//   warp 1      TMEM owner and MMA issuer
//   warps 2-17  converters: four groups of four warps, each group covering
//               the four TMEM lane quarters; group g decodes a quarter of
//               the stage (gate/up: projection g/2, K half g%2; down: K
//               quarter g)
//   warps 18-21 epilogue (one TMEM lane quarter each)
// Every wait is bounded (common.cuh mbar_wait) and reports through p.err.
#include "common.cuh"
#include "kernels.h"

namespace moe_b200 {

template <int MODE>
struct TcCfg {
    static constexpr int kBN = kBlockN;                                    // max tokens per tile
    static constexpr int kRaw = MODE == kGateUp ? 2 * kTileBytes : kTileBytes;
    static constexpr int kBBytes = kBN * 128;                              // 64 bf16 per row
    static constexpr int kSubRows = 32;                                    // rows per TMA box
    static constexpr int kStages = MODE == kGateUp ? 8 : 10;
    static constexpr int kACols = MODE == kGateUp ? 64 : 32;               // TMEM columns per A stage
    static constexpr int kAStages = 256 / kACols;
    static constexpr int kAccCols = MODE == kGateUp ? 2 * kBN : kBN;
    static constexpr int kAccs = 256 / kAccCols;
    static constexpr int kSmem = kStages * (kBBytes + kRaw) + 1024 /*align*/ + 512 /*barriers*/;
};

struct TileCoord {
    uint32_t g, mt, n0, nn;
};

__device__ __forceinline__ void tile_coord(const GemmParams& p, uint32_t tile, TileCoord& tc) {
    uint32_t lo = 0, hi = p.groups;
    while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (p.tile_off[mid] <= tile) lo = mid;
        else hi = mid;
    }
    const uint32_t local = tile - p.tile_off[lo];
    const uint32_t cnt = p.count[lo];
    const uint32_t ntn = ceil_div(cnt, kBlockN);
    tc.g = lo;
    tc.mt = local / ntn;
    tc.n0 = (local % ntn) * kBlockN;
    tc.nn = min(kBlockN, cnt - tc.n0);
}

// SiLU with the fast exponential and division: its error (a few ulp of
// fp32) is far below the bf16 rounding of the intermediate it feeds.
__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

constexpr int kConvWarps = 16;
constexpr int kFirstEpiWarp = 2 + kConvWarps;
constexpr int kThreads = (kFirstEpiWarp + 4) * 32;

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_b,
                                                         const GemmParams p) {
    using C = TcCfg<MODE>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* b_tiles = smem;                                   // [kStages][kBBytes]
    uint8_t* raw_tiles = smem + C::kStages * C::kBBytes;       // [kStages][kRaw]
    uint64_t* bars = reinterpret_cast<uint64_t*>(raw_tiles + C::kStages * C::kRaw);
    uint64_t* load_full = bars;
    uint64_t* load_empty = load_full + C::kStages;
    uint64_t* a_full = load_empty + C::kStages;
    uint64_t* a_empty = a_full + C::kAStages;
    uint64_t* acc_full = a_empty + C::kAStages;
    uint64_t* acc_empty = acc_full + C::kAccs;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + C::kAccs);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < C::kStages; ++i) {
            mbar_init(&load_full[i], 1);
            mbar_init(&load_empty[i], 1);
        }
        for (int i = 0; i < C::kAStages; ++i) {
            mbar_init(&a_full[i], kConvWarps * 32);
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < C::kAccs; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 128);
        }
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) prefetch_tmap(&tmap_b);
    if (warp == 1) {
        tmem_alloc(tmem_holder, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    const uint32_t total = p.tile_off[p.groups];
    const uint32_t a_col0 = 256;  // A stages live in columns [256, 512)

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            bool ok = true;
            for (uint32_t tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
                TileCoord tc;
                tile_coord(p, tile, tc);
                const uint8_t* wbase =
                    p.wt + (uint64_t)tc.g * p.group_stride + (uint64_t)tc.mt * p.k_tiles * C::kRaw;
                const int32_t row0 = (int32_t)(p.offset[tc.g] + tc.n0);
                const uint32_t n_sub = ceil_div(tc.nn, C::kSubRows);
                for (uint32_t kt = 0; kt < p.k_tiles; ++kt) {
                    if (!(ok = mbar_wait(&load_empty[stage], phase ^ 1, p.err, kErrTimeoutLoadEmpty, true))) break;
                    mbar_arrive_expect_tx(&load_full[stage], n_sub * C::kSubRows * 128 + C::kRaw);
                    bulk_g2s(raw_tiles + stage * C::kRaw, wbase + (uint64_t)kt * C::kRaw, C::kRaw, &load_full[stage]);
                    for (uint32_t sb = 0; sb < n_sub; ++sb) {
                        tma_load_2d(b_tiles + stage * C::kBBytes + sb * C::kSubRows * 128, &tmap_b,
                                    (int32_t)(kt * kTileK), row0 + (int32_t)(sb * C::kSubRows), &load_full[stage]);
                    }
                    if (++stage == C::kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, astage = 0, aphase = 0, acc = 0, accphase = 0;
            bool ok = true;
            for (uint32_t tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
                TileCoord tc;
                tile_coord(p, tile, tc);
                const uint32_t n_mma = max(16u, (tc.nn + 15u) & ~15u);
                const uint32_t idesc = idesc_bf16_m128(n_mma);
                if (!(ok = mbar_wait(&acc_empty[acc], accphase ^ 1, p.err, kErrTimeoutAccEmpty))) break;
                tc_fence_after();
                const uint32_t d0 = tmem + acc * C::kAccCols;
                for (uint32_t kt = 0; kt < p.k_tiles; ++kt) {
                    if (!(ok = mbar_wait(&a_full[astage], aphase, p.err, kErrTimeoutAFull))) break;
                    if (!(ok = mbar_wait(&load_full[stage], phase, p.err, kErrTimeoutLoadFull))) break;
                    tc_fence_after();
                    const uint32_t b_addr = smem_u32(b_tiles + stage * C::kBBytes);
                    const uint32_t a0 = tmem + a_col0 + astage * C::kACols;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t bdesc = smem_desc_sw128(b_addr + kk * 32);
                        const uint32_t accum = (kt | kk) != 0;
                        mma_ts_bf16(d0, a0 + kk * 8, bdesc, idesc, accum);
                        if (MODE == kGateUp) mma_ts_bf16(d0 + C::kBN, a0 + 32 + kk * 8, bdesc, idesc, accum);
                    }
                    mma_commit(&a_empty[astage]);
                    mma_commit(&load_empty[stage]);
                    if (++stage == C::kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                    if (++astage == C::kAStages) {
                        astage = 0;
                        aphase ^= 1;
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
    } else if (warp < kFirstEpiWarp) {
        // ------------------------------------------------------------ converters
        const uint32_t quarter = warp & 3;
        const uint32_t group = (warp - 2) >> 2;  // 0..3
        const uint32_t r = quarter * 32 + lane;  // weight row inside the tile == TMEM lane
        const uint32_t lane_addr = (quarter * 32) << 16;
        // gate/up: projection group/2, words 4*(group%2) .. +3 (one scale block)
        // down:    words 2*group, 2*group+1 (scale block group/2)
        const uint32_t proj = MODE == kGateUp ? (group >> 1) : 0;
        const uint32_t word0 = MODE == kGateUp ? (group & 1) * 4 : group * 2;
        const uint32_t sblk = MODE == kGateUp ? (group & 1) : (group >> 1);
        const uint32_t col = MODE == kGateUp ? proj * 32 + (group & 1) * 16 : group * 8;
        uint32_t stage = 0, phase = 0, astage = 0, aphase = 0;
        bool ok = true;
        for (uint32_t tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
            for (uint32_t kt = 0; kt < p.k_tiles; ++kt) {
                if (!(ok = mbar_wait(&load_full[stage], phase, p.err, kErrTimeoutLoadFull))) break;
                const uint8_t* raw = raw_tiles + stage * C::kRaw + proj * kTileBytes;
                const uint32_t* words = reinterpret_cast<const uint32_t*>(raw) + word0 * kTileRows + r;
                const uint32_t sc = raw[kTileCodeBytes + sblk * kTileRows + r];
                constexpr int kWords = MODE == kGateUp ? 4 : 2;
                uint32_t w[kWords];
#pragma unroll
                for (int c = 0; c < kWords; ++c) w[c] = words[c * kTileRows];
                const uint32_t f1 = e8m0_f1(sc);
                uint32_t v[kWords * 4];
#pragma unroll
                for (int c = 0; c < kWords; ++c) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) v[c * 4 + i] = bf16x2_mul(e2m1_pair_bits(w[c], i), f1);
                }
                if (sc > 128u) {  // scales above 2^1: second factor
                    const uint32_t f2 = e8m0_f2(sc);
#pragma unroll
                    for (int j = 0; j < kWords * 4; ++j) v[j] = bf16x2_mul(v[j], f2);
                }
                fence_proxy_async_smem();
                if (!(ok = mbar_wait(&a_empty[astage], aphase ^ 1, p.err, kErrTimeoutAEmpty))) break;
                tc_fence_after();
                const uint32_t taddr = tmem + lane_addr + a_col0 + astage * C::kACols + col;
                if (MODE == kGateUp) {
                    MOE_TMEM_ST16(taddr, v);
                } else {
                    MOE_TMEM_ST8(taddr, v);
                }
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&a_full[astage]);
                if (++stage == C::kStages) {
                    stage = 0;
                    phase ^= 1;
                }
                if (++astage == C::kAStages) {
                    astage = 0;
                    aphase ^= 1;
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
            TileCoord tc;
            tile_coord(p, tile, tc);
            if (!(ok = mbar_wait(&acc_full[acc], accphase, p.err, kErrTimeoutAccFull, true))) break;
            tc_fence_after();
            const uint32_t m = tc.mt * kTileRows + r;
            const bool valid = m < p.m_valid;
            const uint64_t row0 = p.offset[tc.g] + tc.n0;
            const uint32_t dbase = tmem + lane_addr + acc * C::kAccCols;
            for (uint32_t c0 = 0; c0 < tc.nn; c0 += 32) {
                uint32_t d[32];
                MOE_TMEM_LD32(dbase + c0, d);
                if (MODE == kGateUp) {
                    uint32_t u[32];
                    MOE_TMEM_LD32(dbase + C::kBN + c0, u);
                    tmem_wait_ld();
                    if (valid) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            if (c0 + i < tc.nn) {
                                const float hv = __fmul_rn(silu_f(__uint_as_float(d[i])), __uint_as_float(u[i]));
                                p.h_out[(row0 + c0 + i) * p.h_stride + m] = f32_to_bf16_bits(hv);
                            }
                        }
                    }
                } else {
                    tmem_wait_ld();
                    if (valid) {
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

template <int MODE>
static cudaError_t launch_mode(const CUtensorMap& tmap_b, const GemmParams& p, int num_sms, cudaStream_t st) {
    using C = TcCfg<MODE>;
    static uint64_t attr_set = 0;  // one bit per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && !((attr_set >> dev) & 1u)) {
        e = cudaFuncSetAttribute(gemm_tc_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
        if (e != cudaSuccess) return e;
        attr_set |= 1ull << dev;
    }
    gemm_tc_kernel<MODE><<<num_sms, kThreads, C::kSmem, st>>>(tmap_b, p);
    return cudaGetLastError();
}

cudaError_t launch_gemm_tc(int mode, const CUtensorMap& tmap_b, const GemmParams& p, int num_sms,
                           cudaStream_t st) {
    return mode == kGateUp ? launch_mode<kGateUp>(tmap_b, p, num_sms, st)
                           : launch_mode<kDown>(tmap_b, p, num_sms, st);
}

}  // namespace moe_b200
