// Block-scaled tcgen05 grouped GEMMs: the tensor core consumes the MXFP4
// weights as they are stored -- E2M1 codes plus one E8M0 scale per 32 K --
// so no SM instruction is spent decoding weights.
//
//   A   E2M1 weight codes, packed two per byte in HBM as contiguous 8 KB
//       blocks of 128 rows x 128 K, TMA'd with the 16U4_ALIGN16B type (each
//       16 codes land in 16 bytes of shared memory, the operand form
//       kind::mxf8f6f4 reads);
//   SFA the rows' E8M0 scales, one 512-byte block per 128 x 128 tile (row r,
//       K block j at byte (r%32)*16 + (r/32)*4 + j); the gate and up blocks
//       of a tile are adjacent so one bulk copy brings both.  Scale-factor
//       warps store every block into each TMEM lane quarter (lane l holds
//       bytes [16 l, 16 l + 16)) with tcgen05.st, off the tensor pipe;
//   B   activations as two E4M3 terms, hi and lo, each with an E8M0 scale per
//       32 K (SFB).  A bf16 value has 8 significant bits and splits exactly
//       into hi (4 bits) + lo (4 bits), so W.x = W.x_hi + W.x_lo is the product
//       the bf16 path computes.  The hi and lo planes sit in one allocation
//       and one 3-D TMA box brings both;
//   D   fp32 in TMEM.
//
// Two tile shapes:
//   32-token tiles (decode-sized groups): B rows 0-31 hi, 32-63 lo, one
//     MMA of N = 64 per K step, so the A tile is read from shared memory once;
//     the accumulator halves are summed in the epilogue;
//   128-token tiles (prefill): the hi and lo MMAs accumulate into the same
//     columns (N up to 128 each).
//
// kGateUp: gate and up tiles of the same 128 intermediate rows share B; the
//          epilogue computes h = SiLU(gate) * up and writes it already split
//          into hi/lo E4M3 + scales (a warp's 32 rows are one 32-element K
//          block of the down GEMM), so the down GEMM reads it directly.
// kDown:   the epilogue writes fp32 expert outputs for the combine.
//
// Warp roles (320 threads, one CTA per SM -- or per SM of a CTA pair --,
// persistent over a precomputed tile table):
//   warp 0      producer: per 128-K block one bulk copy of the weight scales,
//               one of the activation scales, the A boxes and one B box
//   warp 1      TMEM owner and MMA issue (in a CTA pair, the rank-0 CTA's)
//   warps 2-5   epilogue, one TMEM lane quarter each
//   warps 6-9   scale factors into TMEM, one lane quarter each; for gate/up
//               tiles with one accumulator also a share of the epilogue
//   warps 10-17 (576 threads: 128-token gate/up tiles with one accumulator)
//               two more epilogue groups
// All waits are bounded and report through p.err.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace moe_b200 {

// FP4: the fast mode (kind::mxf4): A and B packed E2M1 in shared memory, one
// B term, 64-byte swizzled rows (one 128-K stage per row).
// KB: 128-K blocks per pipeline stage (2 on CTA pairs, whose smaller B
// halves leave room for stages twice as deep in K; 2 on the stacked 32- and
// 64-token down tiles and 2 or 4 in the fast mode, whose 128-K blocks are
// only 8 or 4 MMAs): fewer stage hand-offs per MMA.  A tile's last stage holds the
// K blocks that are left (K blocks need not divide by KB).
template <int MODE, int BN, bool FP4 = false, bool PAIR = false, int KB = 1>
struct BsCfg {
    static_assert(BN == 32 || BN == 64 || BN == 128, "tile width");
    static_assert(!PAIR || (BN == 128 && !FP4), "CTA pairs run the exact path's 128-token tiles");
    static constexpr bool kStackN = !FP4 && BN <= 64;
    static_assert(KB == 1 || (KB == 2 && (PAIR || kStackN)) || ((KB == 2 || KB == 4) && FP4),
                  "several K blocks per stage: CTA pairs, stacked tiles and the fast mode's small stages");
    static constexpr int kNA = MODE == kGateUp ? 2 : 1;       // A operands per stage
    static constexpr int kABytes = FP4 ? 128 * 64 : 128 * 128;  // smem bytes per A box
    static constexpr int kATx = 128 * 128 / 2;                // packed bytes the A box moves
    static constexpr int kBTerms = FP4 ? 1 : 2;               // B terms per stage (hi, lo)
    static constexpr int kBRows = PAIR ? BN / 2 : BN;         // B rows in this CTA's shared memory
    static constexpr int kBBytes = FP4 ? kBRows * 64 : kBRows * 128;  // smem bytes per B term
    static constexpr int kSFA = kNA * 512;                    // weight scale bytes per K block
    static constexpr int kSFB = (FP4 || kStackN) ? 512 : 1024;  // activation scale bytes per K block
    static constexpr int kSFBlock = kSFA + kSFB;
    static constexpr int kSFStage = KB * kSFBlock;
    static constexpr int kStageBytes = KB * (kNA * kABytes + kBTerms * kBBytes) + kSFStage;
    static constexpr int kStages = (210 * 1024) / kStageBytes;
    static constexpr int kAccCols = kNA * (kStackN ? 2 * BN : BN);
    static constexpr int kAccs = 256 / kAccCols >= 2 ? 2 : 1;
    static constexpr int kSFCols = kSFStage / 128;            // TMEM columns of scale factors per stage
    static constexpr int kSFBlockCols = kSFBlock / 128;       // ... per K block
    static constexpr int kSmem = kStages * kStageBytes + 2048 /*two 1024 alignments*/ + 512 /*barriers*/;
    // gate/up with one accumulator: its epilogue holds up the next tile's
    // MMAs, so more warps share it -- for 128-token tiles four groups of four
    // warps (the scale-factor warps are one of them, 576 threads), else two
    static constexpr bool kGuSplit = MODE == kGateUp && kAccs == 1;
    static constexpr int kEpiGroups = kGuSplit ? (BN == 128 ? 4 : 2) : 1;
    static constexpr int kThreads = kEpiGroups == 4 ? 576 : 320;
    static_assert(kStages >= (KB >= 2 ? 2 : 3), "pipeline too shallow");
    static_assert(256 + kStages * kSFCols <= 512, "TMEM budget");
    static_assert(kSmem <= 227 * 1024, "shared memory budget");
    static_assert(((PAIR ? 4 : 3) * kStages + 2 * kAccs) * 8 + 4 <= 512, "barrier space");
};

// Byte offsets of a token row's hi and lo scale words inside a stage's
// activation scale block (the tcgen05.cp layout over the B rows).
// Stacked tiles (32 or 64 tokens): hi rows [0, BN), lo rows [BN, 2 BN) of one
// 512-byte block; 128-token tiles: a hi block, then a lo block.
__device__ __forceinline__ uint32_t sf_row_pos(uint32_t row) { return (row % 32) * 16 + (row / 32) * 4; }
template <int BN>
__device__ __forceinline__ uint32_t sfb_pos_hi(uint32_t rr) {
    return sf_row_pos(rr);
}
template <int BN>
__device__ __forceinline__ uint32_t sfb_pos_lo(uint32_t rr) {
    return BN <= 64 ? sf_row_pos(BN + rr) : 512 + sf_row_pos(rr);
}

__device__ __forceinline__ float pow2f(int e) {
    // exact 2^e for e in [-127, 127]
    return e >= -126 ? __int_as_float((e + 127) << 23) : __int_as_float(0x00400000);
}

// Warp-wide maximum of non-negative floats in one redux.sync: their bit
// patterns order like unsigned integers.
__device__ __forceinline__ float warp_max_abs(float v) {
    return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v))));
}

// Scale exponent for a 32-value block with absolute maximum `amax`: the block
// maps into [128, 256) of E4M3's range (no overflow; E4M3 keeps 4 significant
// bits anywhere in its normal range, so the exact choice costs no precision).
__device__ __forceinline__ int block_exp(float amax) {
    const int e = (int)((__float_as_uint(amax) >> 23) & 0xFF) - 127 - 7;
    return amax > 0.f ? max(-127, min(127, e)) : -127;
}

// Two fp32 values to E4M3 codes by the hardware conversion (round to nearest
// even, saturating finite; no saturation happens for |y| < 448): the first
// argument in the low byte.  One conversion per two values.
__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
    uint16_t d;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(d) : "f"(hi), "f"(lo));
    return d;
}

// The values of the two E4M3 codes in the low 16 bits of `code2` (low byte
// first), exactly: every E4M3 value is an f16 value, so the hardware
// conversion to f16x2 and then to fp32 loses nothing.  The residual of the
// hi/lo split needs the rounded hi value; this is it, two at a time.
__device__ __forceinline__ void e4m3x2_values(uint32_t code2, float& lo, float& hi) {
    asm("{\n\t.reg .b32 h2;\n\t.reg .b16 l, h;\n\t"
        "cvt.rn.f16x2.e4m3x2 h2, %2;\n\t"
        "mov.b32 {l, h}, h2;\n\t"
        "cvt.f32.f16 %0, l;\n\t"
        "cvt.f32.f16 %1, h;\n\t}"
        : "=f"(lo), "=f"(hi)
        : "h"((uint16_t)code2));
}

// Splits the 32 values held by a warp (one per lane, one 32-element K block)
// into hi + lo E4M3 terms with E8M0 scale bytes.  Warp-collective.
__device__ __forceinline__ void split_e4m3_warp(float v, uint8_t& hi, uint8_t& lo, uint8_t& s_hi, uint8_t& s_lo) {
    const int e1 = block_exp(warp_max_abs(v));
    const float y = v * pow2f(-e1);
    const uint32_t c = cvt_e4m3x2(y, 0.0f);
    hi = (uint8_t)c;
    float q, q_unused;
    e4m3x2_values(c, q, q_unused);
    const float r = v - q * pow2f(e1);
    const int e2 = block_exp(warp_max_abs(r));
    lo = (uint8_t)cvt_e4m3x2(r * pow2f(-e2), 0.0f);
    s_hi = (uint8_t)(e1 + 127);
    s_lo = (uint8_t)(e2 + 127);
}

// Hi/lo split of four consecutive values held by each lane, a 32-element
// block spanning 8 consecutive lanes (lanes 8j .. 8j+7 hold block j): the
// same block maximum, exponents and rounding as split_e4m3_warp, with the
// maximum taken by three shuffles inside the 8-lane group.  Returns the four
// hi and four lo code bytes packed low-to-high and the block's scale bytes.
__device__ __forceinline__ void split_e4m3_x4(const float v[4], uint32_t& hi4, uint32_t& lo4, uint8_t& s_hi,
                                              uint8_t& s_lo) {
    auto group_max = [](float a) {
        uint32_t u = __float_as_uint(a);
        u = max(u, __shfl_xor_sync(0xffffffffu, u, 1));
        u = max(u, __shfl_xor_sync(0xffffffffu, u, 2));
        u = max(u, __shfl_xor_sync(0xffffffffu, u, 4));
        return __uint_as_float(u);  // non-negative floats order like their bit patterns
    };
    float m = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    const int e1 = block_exp(group_max(m));
    float r[4];
    const float inv1 = pow2f(-e1), sc1 = pow2f(e1);
    float y[4], q[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) y[i] = v[i] * inv1;
    const uint32_t c01 = cvt_e4m3x2(y[0], y[1]), c23 = cvt_e4m3x2(y[2], y[3]);
    hi4 = c01 | (c23 << 16);
    e4m3x2_values(c01, q[0], q[1]);
    e4m3x2_values(c23, q[2], q[3]);
#pragma unroll
    for (int i = 0; i < 4; ++i) r[i] = v[i] - q[i] * sc1;
    m = fmaxf(fmaxf(fabsf(r[0]), fabsf(r[1])), fmaxf(fabsf(r[2]), fabsf(r[3])));
    const int e2 = block_exp(group_max(m));
    const float inv2 = pow2f(-e2);
    lo4 = cvt_e4m3x2(r[0] * inv2, r[1] * inv2) | (cvt_e4m3x2(r[2] * inv2, r[3] * inv2) << 16);
    s_hi = (uint8_t)(e1 + 127);
    s_lo = (uint8_t)(e2 + 127);
}

// Scale exponent of a 32-value block for E2M1 codes (fast mode): the
// smallest e with amax <= 6 * 2^e, so the block maximum is never clipped.
__device__ __forceinline__ int fp4_block_exp(float amax) {
    if (!(amax > 0.f)) return -127;
    int e = max(-127, (int)((__float_as_uint(amax) >> 23) & 0xFF) - 127 - 2);  // amax / 2^e in [4, 8)
    if (amax > 6.0f * pow2f(e)) ++e;
    return min(127, e);
}

// ---------------------------------------------------------------------------
// Permuted activation rows for the block-scaled GEMM, quantised on the way:
// one warp per (permuted row, chunk of kGqChunk 128-element K stages).  For
// stage kt lane l holds elements 128 kt + 4 l .. + 3 (one 8-byte load), so
// 32-element block j is lanes 8j .. 8j+7; the lane writes its four hi and
// four lo code bytes with one 4-byte store per plane of xb ([2][rows_cap][Kp]).
// The stage's four hi and four lo scale bytes go, as one 32-bit word each,
// straight into the scale block the GEMM's producer bulk-copies for (token
// tile, kt), at sfb_pos_hi / sfb_pos_lo.  The row's token tile and index in
// it come from the permutation (row_info).
// ---------------------------------------------------------------------------
constexpr uint32_t kGqChunk = 4;

template <int BN>
__global__ void __launch_bounds__(256) gather_quant_bs_kernel(const uint16_t* __restrict__ x, uint32_t H,
                                                              uint32_t Kp, const uint32_t* __restrict__ row_token,
                                                              const uint32_t* __restrict__ row_info, uint32_t rows,
                                                              uint32_t rows_cap, uint8_t* __restrict__ xb,
                                                              uint8_t* __restrict__ sf_atoms) {
    constexpr uint32_t kAtom = BN <= 64 ? 512 : 1024;
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t nkt = Kp / 128;
    const uint32_t chunks = (nkt + kGqChunk - 1) / kGqChunk;
    const uint64_t tasks = (uint64_t)rows * chunks;
    const uint64_t xplane = (uint64_t)rows_cap * Kp;
    const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
    // the permutation first; only then may the gate/up GEMM launch (its
    // prologue reads the tile table the permutation wrote)
    pdl_wait();
    pdl_trigger();
    for (uint64_t task = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; task < tasks; task += warps) {
        const uint32_t r = (uint32_t)(task / chunks);
        const uint32_t kt0 = (uint32_t)(task % chunks) * kGqChunk;
        const uint16_t* xr = x + (uint64_t)__ldg(row_token + r) * H;
        const uint32_t info = __ldg(row_info + r);
        uint8_t* atoms = sf_atoms + (uint64_t)(info >> 8) * nkt * kAtom;
        const uint32_t pos_h = sfb_pos_hi<BN>(info & 0xFFu), pos_l = sfb_pos_lo<BN>(info & 0xFFu);
        uint32_t* dh = reinterpret_cast<uint32_t*>(xb + (uint64_t)r * Kp) + lane;
        uint32_t* dl = reinterpret_cast<uint32_t*>(xb + xplane + (uint64_t)r * Kp) + lane;
        uint2 raw[kGqChunk];
#pragma unroll
        for (uint32_t c = 0; c < kGqChunk; ++c) {
            const uint32_t k = (kt0 + c) * 128 + lane * 4;  // H % 8 == 0: four elements all in or all out
            raw[c] = (kt0 + c < nkt && k < H) ? __ldg(reinterpret_cast<const uint2*>(xr + k)) : make_uint2(0, 0);
        }
#pragma unroll
        for (uint32_t c = 0; c < kGqChunk; ++c) {
            const uint32_t kt = kt0 + c;
            if (kt >= nkt) break;  // uniform across the warp
            const float v[4] = {__uint_as_float(raw[c].x << 16), __uint_as_float(raw[c].x & 0xffff0000u),
                                __uint_as_float(raw[c].y << 16), __uint_as_float(raw[c].y & 0xffff0000u)};
            uint32_t hi4, lo4;
            uint8_t sh, sl;
            split_e4m3_x4(v, hi4, lo4, sh, sl);
            dh[kt * 32] = hi4;
            dl[kt * 32] = lo4;
            // block j's scale bytes sit in lane 8j; gather them into one word
            uint32_t shw = 0, slw = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                shw |= (uint32_t)(uint8_t)__shfl_sync(0xffffffffu, (uint32_t)sh, 8 * j) << (8 * j);
                slw |= (uint32_t)(uint8_t)__shfl_sync(0xffffffffu, (uint32_t)sl, 8 * j) << (8 * j);
            }
            if (lane == 0) {
                uint8_t* atom = atoms + (uint64_t)kt * kAtom;
                *reinterpret_cast<uint32_t*>(atom + pos_h) = shw;
                *reinterpret_cast<uint32_t*>(atom + pos_l) = slw;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Weight repack for the block-scaled path (once per expert at upload).
//   codes: blocks [row_tile][k_tile] of 128 rows x 128 K, 8 KB each, row r of
//          a block at r*64 bytes, element 2j in the low nibble of byte j
//          (zero past `rows` / `cols`);
//   sfa:   one 512-byte scale block per (row_tile, k_tile) in the tcgen05.cp
//          layout, consecutive blocks `sf_stride` bytes apart (the gate and up
//          blocks of a tile are interleaved: stride 1024, up at +512).
// ---------------------------------------------------------------------------
__global__ void repack_bs_kernel(const uint8_t* __restrict__ gguf, uint32_t rows, uint32_t cols, uint32_t rows_pad,
                                 uint32_t Kp, uint8_t* __restrict__ codes, uint8_t* __restrict__ sfa,
                                 uint32_t sf_stride) {
    const uint32_t gguf_row_bytes = ceil_div(cols, 32) * 17;
    const uint32_t kt_n = Kp / 128;
    const uint64_t nbytes = (uint64_t)rows_pad * (Kp / 2);
    const uint64_t nsf = (uint64_t)rows_pad * (Kp / 32);
    for (uint64_t idx = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; idx < nbytes + nsf;
         idx += (uint64_t)gridDim.x * blockDim.x) {
        if (idx < nbytes) {
            const uint64_t blk = idx / 8192;
            const uint32_t within = (uint32_t)(idx % 8192);
            const uint32_t mt = (uint32_t)(blk / kt_n), kt = (uint32_t)(blk % kt_n);
            const uint32_t r = mt * 128 + within / 64;
            const uint32_t j = kt * 64 + within % 64;  // byte index along the row
            uint32_t b = 0;
            if (r < rows) {
                const uint8_t* row = gguf + (uint64_t)r * gguf_row_bytes;
                for (int h = 0; h < 2; ++h) {
                    const uint32_t k = 2 * j + h;
                    if (k < cols) {
                        const uint8_t* gb = row + (k / 32) * 17;
                        const uint32_t i = k % 32;
                        const uint32_t code = i < 16 ? (gb[1 + i] & 0x0Fu) : (gb[1 + i - 16] >> 4);
                        b |= code << (4 * h);
                    }
                }
            }
            codes[idx] = (uint8_t)b;
        } else {
            const uint64_t q = idx - nbytes;
            const uint32_t r = (uint32_t)(q / (Kp / 32));
            const uint32_t blk = (uint32_t)(q % (Kp / 32));
            uint8_t sv = 0;
            if (r < rows && blk * 32 < cols) sv = gguf[(uint64_t)r * gguf_row_bytes + blk * 17];
            const uint32_t mt = r / 128, rr = r % 128, kt = blk / 4, j = blk % 4;
            sfa[((uint64_t)mt * kt_n + kt) * sf_stride + (rr % 32) * 16 + (rr / 32) * 4 + j] = sv;
        }
    }
}

cudaError_t launch_repack_bs(const uint8_t* gguf, uint32_t rows, uint32_t cols, uint32_t rows_pad, uint32_t Kp,
                             uint8_t* codes, uint8_t* sfa, uint32_t sf_stride, cudaStream_t st) {
    const uint64_t work = (uint64_t)rows_pad * (Kp / 2) + (uint64_t)rows_pad * (Kp / 32);
    const uint64_t blocks = (work + 255) / 256;
    repack_bs_kernel<<<(unsigned)(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, st>>>(gguf, rows, cols, rows_pad,
                                                                                       Kp, codes, sfa, sf_stride);
    return cudaGetLastError();
}

// The inverse of repack_bs_kernel: GGUF MXFP4 rows (per 32 elements one E8M0
// byte, then 16 bytes holding element i in the low nibble of byte i and
// element i + 16 in its high nibble) of one projection, rebuilt from its
// block-scaled form.  Only the cross-check paths need the GGUF bytes again
// (they repack them into their own tile form), so the upload keeps a single
// copy of every expert.  One thread per output byte.
__global__ void bs_to_gguf_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ sfa,
                                  uint32_t sf_stride, uint32_t rows, uint32_t cols, uint32_t Kp,
                                  uint8_t* __restrict__ gguf) {
    const uint32_t nblk = ceil_div(cols, 32);
    const uint32_t row_bytes = nblk * 17;
    const uint32_t kt_n = Kp / 128;
    const uint64_t total = (uint64_t)rows * row_bytes;
    for (uint64_t idx = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t r = (uint32_t)(idx / row_bytes);
        const uint32_t rem = (uint32_t)(idx % row_bytes);
        const uint32_t b = rem / 17, j = rem % 17;
        const uint32_t mt = r / 128, rr = r % 128;
        uint8_t v;
        if (j == 0) {
            const uint32_t kt = b / 4, q = b % 4;
            v = sfa[((uint64_t)mt * kt_n + kt) * sf_stride + (rr % 32) * 16 + (rr / 32) * 4 + q];
        } else {
            auto code = [&](uint32_t k) -> uint32_t {
                const uint64_t blk = (uint64_t)mt * kt_n + k / 128;
                const uint8_t byte = codes[blk * 8192 + rr * 64 + (k % 128) / 2];
                return (k & 1u) ? (byte >> 4) : (byte & 0x0Fu);
            };
            const uint32_t k_lo = b * 32 + (j - 1);
            v = (uint8_t)(code(k_lo) | (code(k_lo + 16) << 4));  // past `cols` the block-scaled codes are 0
        }
        gguf[idx] = v;
    }
}

cudaError_t launch_bs_to_gguf(const uint8_t* codes, const uint8_t* sfa, uint32_t sf_stride, uint32_t rows,
                              uint32_t cols, uint32_t Kp, uint8_t* gguf, cudaStream_t st) {
    const uint64_t work = (uint64_t)rows * ceil_div(cols, 32) * 17;
    const uint64_t blocks = (work + 255) / 256;
    bs_to_gguf_kernel<<<(unsigned)(blocks < 148 * 16 ? (blocks ? blocks : 1) : 148 * 16), 256, 0, st>>>(
        codes, sfa, sf_stride, rows, cols, Kp, gguf);
    return cudaGetLastError();
}

// The same planes and scale words as gather_quant_bs_kernel, computed once
// per token instead of once per permuted row: a warp takes (token t, chunk
// of kGqChunk K stages), reads and splits the token's row once, and stores
// the codes and scale words at each of the token's permuted rows:
// pos_of[t*K + j] for its K routed assignments, and shared_off[0] + t for
// the shared expert's row when shared_off is set.  Positions at or past
// `rows` (an assignment the permutation rejected) are skipped.  The split
// depends only on the values, so the bytes equal the per-row gather's.
template <int BN>
__global__ void __launch_bounds__(256) scatter_quant_bs_kernel(const uint16_t* __restrict__ x, uint32_t H,
                                                               uint32_t Kp, uint32_t T, uint32_t K,
                                                               const uint32_t* __restrict__ pos_of,
                                                               const uint32_t* __restrict__ shared_off,
                                                               const uint32_t* __restrict__ row_info, uint32_t rows,
                                                               uint32_t rows_cap, uint8_t* __restrict__ xb,
                                                               uint8_t* __restrict__ sf_atoms) {
    constexpr uint32_t kAtom = BN <= 64 ? 512 : 1024;
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t nkt = Kp / 128;
    const uint32_t chunks = (nkt + kGqChunk - 1) / kGqChunk;
    const uint64_t tasks = (uint64_t)T * chunks;
    const uint64_t xplane = (uint64_t)rows_cap * Kp;
    const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
    pdl_wait();  // the permutation (positions, row info) first
    pdl_trigger();
    for (uint64_t task = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; task < tasks; task += warps) {
        const uint32_t t = (uint32_t)(task / chunks);
        const uint32_t kt0 = (uint32_t)(task % chunks) * kGqChunk;
        // lane j < K: the token's j-th routed row; the shared row separately
        uint32_t my_pos = 0xFFFFFFFFu, my_info = 0;
        if (lane < K) {
            const uint32_t q = __ldg(pos_of + (uint64_t)t * K + lane);
            if (q < rows) {
                my_pos = q;
                my_info = __ldg(row_info + q);
            }
        }
        uint32_t sh_pos = 0xFFFFFFFFu, sh_info = 0;
        if (shared_off) {
            const uint32_t q = __ldg(shared_off) + t;
            if (q < rows) {
                sh_pos = q;
                sh_info = __ldg(row_info + q);
            }
        }
        const uint16_t* xr = x + (uint64_t)t * H;
        uint2 raw[kGqChunk];
#pragma unroll
        for (uint32_t c = 0; c < kGqChunk; ++c) {
            const uint32_t k = (kt0 + c) * 128 + lane * 4;  // H % 8 == 0: four elements all in or all out
            raw[c] = (kt0 + c < nkt && k < H) ? __ldg(reinterpret_cast<const uint2*>(xr + k)) : make_uint2(0, 0);
        }
        // the chunk's K blocks split first, then each destination row
        // resolved once and written for all of them
        const uint32_t nc = min(kGqChunk, nkt - kt0);
        uint32_t hi4[kGqChunk], lo4[kGqChunk], shw[kGqChunk], slw[kGqChunk];
#pragma unroll
        for (uint32_t c = 0; c < kGqChunk; ++c) {
            const float v[4] = {__uint_as_float(raw[c].x << 16), __uint_as_float(raw[c].x & 0xffff0000u),
                                __uint_as_float(raw[c].y << 16), __uint_as_float(raw[c].y & 0xffff0000u)};
            uint8_t sh, sl;
            split_e4m3_x4(v, hi4[c], lo4[c], sh, sl);
            // block j's scale bytes sit in lane 8j; gather them into one word
            shw[c] = 0;
            slw[c] = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                shw[c] |= (uint32_t)(uint8_t)__shfl_sync(0xffffffffu, (uint32_t)sh, 8 * j) << (8 * j);
                slw[c] |= (uint32_t)(uint8_t)__shfl_sync(0xffffffffu, (uint32_t)sl, 8 * j) << (8 * j);
            }
        }
        auto put = [&](uint32_t pos, uint32_t info) {
            uint32_t* dh = reinterpret_cast<uint32_t*>(xb + (uint64_t)pos * Kp) + lane + kt0 * 32;
            uint32_t* dl = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(dh) + xplane);
            if (nc == kGqChunk) {
#pragma unroll
                for (uint32_t c = 0; c < kGqChunk; ++c) {
                    dh[c * 32] = hi4[c];
                    dl[c * 32] = lo4[c];
                }
            } else {
#pragma unroll
                for (uint32_t c = 0; c < kGqChunk; ++c) {
                    if (c < nc) {
                        dh[c * 32] = hi4[c];
                        dl[c * 32] = lo4[c];
                    }
                }
            }
            if (lane < nc) {  // lane c stores K block kt0 + c's scale words
                uint32_t h = shw[0], l = slw[0];
#pragma unroll
                for (uint32_t c = 1; c < kGqChunk; ++c) {
                    h = lane == c ? shw[c] : h;
                    l = lane == c ? slw[c] : l;
                }
                uint8_t* atom = sf_atoms + ((uint64_t)(info >> 8) * nkt + kt0 + lane) * kAtom;
                *reinterpret_cast<uint32_t*>(atom + sfb_pos_hi<BN>(info & 0xFFu)) = h;
                *reinterpret_cast<uint32_t*>(atom + sfb_pos_lo<BN>(info & 0xFFu)) = l;
            }
        };
        for (uint32_t j = 0; j < K; ++j) {
            const uint32_t pos = __shfl_sync(0xffffffffu, my_pos, j);
            const uint32_t info = __shfl_sync(0xffffffffu, my_info, j);
            if (pos != 0xFFFFFFFFu) put(pos, info);  // uniform across the warp
        }
        if (sh_pos != 0xFFFFFFFFu) put(sh_pos, sh_info);
    }
}

cudaError_t launch_scatter_quant_bs(const uint16_t* x, uint32_t H, uint32_t Kp, uint32_t T, uint32_t K,
                                    const uint32_t* pos_of, const uint32_t* shared_off, const uint32_t* row_info,
                                    uint32_t rows, uint32_t rows_cap, uint32_t block_n, uint8_t* xb,
                                    uint8_t* sf_atoms, cudaStream_t st, bool pdl) {
    if (T == 0) return cudaSuccess;
    if (K > 32) return cudaErrorInvalidValue;
    const uint64_t tasks = (uint64_t)T * ((Kp / 128 + kGqChunk - 1) / kGqChunk);
    const uint32_t blocks = (uint32_t)std::min<uint64_t>((tasks + 7) / 8, 148ull * 8ull);
    if (block_n == 32) {
        return launch_kernel(scatter_quant_bs_kernel<32>, dim3(blocks), dim3(256), 0, st, pdl, x, H, Kp, T, K,
                             pos_of, shared_off, row_info, rows, rows_cap, xb, sf_atoms);
    }
    if (block_n == 64) {
        return launch_kernel(scatter_quant_bs_kernel<64>, dim3(blocks), dim3(256), 0, st, pdl, x, H, Kp, T, K,
                             pos_of, shared_off, row_info, rows, rows_cap, xb, sf_atoms);
    }
    return launch_kernel(scatter_quant_bs_kernel<128>, dim3(blocks), dim3(256), 0, st, pdl, x, H, Kp, T, K, pos_of,
                         shared_off, row_info, rows, rows_cap, xb, sf_atoms);
}

// Fast mode: each token row split once into E2M1 codes with one E8M0 scale
// per 32 elements (the smallest scale that keeps the block maximum at or
// below 6; codes rounded to nearest even by the hardware conversion), stored
// at each of the token's permuted rows like scatter_quant_bs_kernel:
// xq [rows_cap][Kp/2] bytes, element 2j in the low nibble of byte j; the
// four scale bytes of a 128-K stage as one word in the stage's 512-byte
// scale block of the row's token tile, at sf_row_pos(index in tile).
__global__ void __launch_bounds__(256) scatter_quant_fp4_kernel(const uint16_t* __restrict__ x, uint32_t H,
                                                                uint32_t Kp, uint32_t T, uint32_t K,
                                                                const uint32_t* __restrict__ pos_of,
                                                                const uint32_t* __restrict__ shared_off,
                                                                const uint32_t* __restrict__ row_info, uint32_t rows,
                                                                uint8_t* __restrict__ xq,
                                                                uint8_t* __restrict__ sf_atoms) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t nkt = Kp / 128;
    const uint32_t chunks = (nkt + kGqChunk - 1) / kGqChunk;
    const uint64_t tasks = (uint64_t)T * chunks;
    const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
    pdl_wait();  // the permutation (positions, row info) first
    pdl_trigger();
    for (uint64_t task = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; task < tasks; task += warps) {
        const uint32_t t = (uint32_t)(task / chunks);
        const uint32_t kt0 = (uint32_t)(task % chunks) * kGqChunk;
        uint32_t my_pos = 0xFFFFFFFFu, my_info = 0;
        if (lane < K) {
            const uint32_t q = __ldg(pos_of + (uint64_t)t * K + lane);
            if (q < rows) {
                my_pos = q;
                my_info = __ldg(row_info + q);
            }
        }
        uint32_t sh_pos = 0xFFFFFFFFu, sh_info = 0;
        if (shared_off) {
            const uint32_t q = __ldg(shared_off) + t;
            if (q < rows) {
                sh_pos = q;
                sh_info = __ldg(row_info + q);
            }
        }
        const uint16_t* xr = x + (uint64_t)t * H;
        uint2 raw[kGqChunk];
#pragma unroll
        for (uint32_t c = 0; c < kGqChunk; ++c) {
            const uint32_t k = (kt0 + c) * 128 + lane * 4;  // H % 8 == 0: four elements all in or all out
            raw[c] = (kt0 + c < nkt && k < H) ? __ldg(reinterpret_cast<const uint2*>(xr + k)) : make_uint2(0, 0);
        }
#pragma unroll
        for (uint32_t c = 0; c < kGqChunk; ++c) {
            const uint32_t kt = kt0 + c;
            if (kt >= nkt) break;  // uniform across the warp
            const float v[4] = {__uint_as_float(raw[c].x << 16), __uint_as_float(raw[c].x & 0xffff0000u),
                                __uint_as_float(raw[c].y << 16), __uint_as_float(raw[c].y & 0xffff0000u)};
            uint32_t m = __float_as_uint(fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3]))));
            m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
            m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
            m = max(m, __shfl_xor_sync(0xffffffffu, m, 4));
            const int e = fp4_block_exp(__uint_as_float(m));
            const float inv = pow2f(-e);
            const uint32_t codes = cvt_e2m1x2(v[0] * inv, v[1] * inv) | (cvt_e2m1x2(v[2] * inv, v[3] * inv) << 8);
            uint32_t sw = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) sw |= (uint32_t)(__shfl_sync(0xffffffffu, (uint32_t)(e + 127), 8 * j) & 0xFFu)
                                              << (8 * j);
            auto put = [&](uint32_t pos, uint32_t info) {
                *reinterpret_cast<uint16_t*>(xq + (uint64_t)pos * (Kp / 2) + kt * 64 + lane * 2) = (uint16_t)codes;
                if (lane == 0) {
                    uint8_t* atom = sf_atoms + ((uint64_t)(info >> 8) * nkt + kt) * 512;
                    *reinterpret_cast<uint32_t*>(atom + sf_row_pos(info & 0xFFu)) = sw;
                }
            };
            for (uint32_t j = 0; j < K; ++j) {
                const uint32_t pos = __shfl_sync(0xffffffffu, my_pos, j);
                const uint32_t info = __shfl_sync(0xffffffffu, my_info, j);
                if (pos != 0xFFFFFFFFu) put(pos, info);  // uniform across the warp
            }
            if (sh_pos != 0xFFFFFFFFu) put(sh_pos, sh_info);
        }
    }
}

cudaError_t launch_scatter_quant_fp4(const uint16_t* x, uint32_t H, uint32_t Kp, uint32_t T, uint32_t K,
                                     const uint32_t* pos_of, const uint32_t* shared_off, const uint32_t* row_info,
                                     uint32_t rows, uint8_t* xq, uint8_t* sf_atoms, cudaStream_t st, bool pdl) {
    if (T == 0) return cudaSuccess;
    if (K > 32) return cudaErrorInvalidValue;
    const uint64_t tasks = (uint64_t)T * ((Kp / 128 + kGqChunk - 1) / kGqChunk);
    const uint32_t blocks = (uint32_t)std::min<uint64_t>((tasks + 7) / 8, 148ull * 8ull);
    return launch_kernel(scatter_quant_fp4_kernel, dim3(blocks), dim3(256), 0, st, pdl, x, H, Kp, T, K, pos_of,
                         shared_off, row_info, rows, xq, sf_atoms);
}

cudaError_t launch_gather_quant_bs(const uint16_t* x, uint32_t H, uint32_t Kp, const uint32_t* row_token,
                                   const uint32_t* row_info, uint32_t rows, uint32_t rows_cap, uint32_t block_n,
                                   uint8_t* xb, uint8_t* sf_atoms, cudaStream_t st, bool pdl) {
    if (rows == 0) return cudaSuccess;
    const uint64_t tasks = (uint64_t)rows * ((Kp / 128 + kGqChunk - 1) / kGqChunk);
    const uint32_t blocks = (uint32_t)std::min<uint64_t>((tasks + 7) / 8, 148ull * 8ull);
    if (block_n == 32) {
        return launch_kernel(gather_quant_bs_kernel<32>, dim3(blocks), dim3(256), 0, st, pdl, x, H, Kp, row_token,
                             row_info, rows, rows_cap, xb, sf_atoms);
    }
    if (block_n == 64) {
        return launch_kernel(gather_quant_bs_kernel<64>, dim3(blocks), dim3(256), 0, st, pdl, x, H, Kp, row_token,
                             row_info, rows, rows_cap, xb, sf_atoms);
    }
    return launch_kernel(gather_quant_bs_kernel<128>, dim3(blocks), dim3(256), 0, st, pdl, x, H, Kp, row_token,
                         row_info, rows, rows_cap, xb, sf_atoms);
}

// ---------------------------------------------------------------------------
// The grouped GEMM
// ---------------------------------------------------------------------------
struct BsTileX {
    uint32_t g, mt, row0, nn, ntile;
};

__device__ __forceinline__ BsTileX load_tile(const BsParams& p, uint32_t tile) {
    const uint4 e = __ldg(reinterpret_cast<const uint4*>(p.tiles) + tile);
    return BsTileX{e.x, e.y, e.z, e.w & 0xFFu, e.w >> 8};
}

// Tile table: tile index -> (group, weight row tile, first row, tokens, token
// tile), in the order (group, row tile, token tile).  One thread per entry.
__global__ void build_tiles_kernel(const uint32_t* __restrict__ count, const uint32_t* __restrict__ offset,
                                   const uint32_t* __restrict__ tile_off, uint32_t groups, uint32_t m_tiles,
                                   uint32_t block_n, uint32_t max_tiles, TileEntry* __restrict__ tiles) {
    const uint32_t total = tile_off[groups];
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < total && t < max_tiles;
         t += gridDim.x * blockDim.x) {
        uint32_t lo = 0, hi = groups;
        while (hi - lo > 1) {
            const uint32_t mid = (lo + hi) >> 1;
            if (tile_off[mid] <= t) lo = mid;
            else hi = mid;
        }
        const uint32_t local = t - tile_off[lo];
        const uint32_t ntn = ceil_div(count[lo], block_n);
        const uint32_t nt = local % ntn;
        const uint32_t n0 = nt * block_n;
        TileEntry e;
        e.group = lo;
        e.mt = local / ntn;
        e.row0 = offset[lo] + n0;
        e.nn_ntile = min(block_n, count[lo] - n0) | ((tile_off[lo] / m_tiles + nt) << 8);
        tiles[t] = e;
    }
}

cudaError_t launch_build_tiles(const uint32_t* count, const uint32_t* offset, const uint32_t* tile_off,
                               uint32_t groups, uint32_t m_tiles, uint32_t block_n, uint32_t max_tiles,
                               TileEntry* tiles, cudaStream_t st) {
    const uint32_t blocks = max(1u, min(ceil_div(max_tiles, 256), 148u * 4u));
    build_tiles_kernel<<<blocks, 256, 0, st>>>(count, offset, tile_off, groups, m_tiles, block_n, max_tiles, tiles);
    return cudaGetLastError();
}

__device__ __forceinline__ float silu_fast(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// The gated activation of the gate projection (moe_generation_gated_activation_cached,
// generation_mlp.cpp.inc:94-104): SiLU, GELU in its erf form, or GELU in its
// tanh form with x + 0.044715 x^3 as one multiply-add (CUDA's erff / tanhf;
// tolerance parity like the rest of the expert math).
// The GELU forms are kept out of line and chosen once per 8 values, so the
// SiLU path of the epilogue is the same code as without them (an inline
// select per value would be if-converted into evaluating every form).
__device__ __noinline__ float gelu_act(int act, float g) {
    if (act == 1) return 0.5f * g * (1.0f + erff(g * 0.70710678118654752440f));
    return 0.5f * g * (1.0f + tanhf(0.7978845608028654f * fmaf(0.044715f * g * g, g, g)));
}

// Gate/up epilogue for 8 token columns of one row m: h = SiLU(gate) * up,
// split into hi/lo E4M3 with the down GEMM's block scales, stored.  The 8 chains
// are independent and the code is branch-free (columns at or past nn are
// computed; their stores are predicated off, and lane j stores column j's
// scale bytes), so the latencies overlap and no per-column divergence
// handling is needed.
template <int BN>
__device__ __forceinline__ void h_store8(const float* hv, uint32_t c0, uint32_t nn, uint64_t row0, uint32_t m,
                                         uint32_t lane, uint32_t quarter, const BsParams& p, uint8_t* h_atom) {
    // split_e4m3_warp for the 8 values, written phase by phase (all block
    // maxima of a phase back to back) so the independent chains overlap
    // around the warp reductions
    // (codes two columns per conversion, the rounded hi values from the
    // reverse conversion)
    uint8_t hi[8], lo[8], sh[8], sl[8];
    float mx[8], r[8], y[8];
    int e[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) mx[j] = warp_max_abs(hv[j]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        e[j] = block_exp(mx[j]);
        y[j] = hv[j] * pow2f(-e[j]);
        sh[j] = (uint8_t)(e[j] + 127);
    }
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
        const uint32_t c = cvt_e4m3x2(y[j], y[j + 1]);
        hi[j] = (uint8_t)c;
        hi[j + 1] = (uint8_t)(c >> 8);
        float q0, q1;
        e4m3x2_values(c, q0, q1);
        r[j] = hv[j] - q0 * pow2f(e[j]);
        r[j + 1] = hv[j + 1] - q1 * pow2f(e[j + 1]);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) mx[j] = warp_max_abs(r[j]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        e[j] = block_exp(mx[j]);
        sl[j] = (uint8_t)(e[j] + 127);
    }
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
        const uint32_t c = cvt_e4m3x2(r[j] * pow2f(-e[j]), r[j + 1] * pow2f(-e[j + 1]));
        lo[j] = (uint8_t)c;
        lo[j + 1] = (uint8_t)(c >> 8);
    }
    uint8_t* hp = p.h_out + (row0 + c0) * p.h_stride + m;
    uint8_t* lp = hp + p.h_plane;
    if (c0 + 8 <= nn) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            hp[(uint64_t)j * p.h_stride] = hi[j];
            lp[(uint64_t)j * p.h_stride] = lo[j];
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (c0 + j < nn) {
                hp[(uint64_t)j * p.h_stride] = hi[j];
                lp[(uint64_t)j * p.h_stride] = lo[j];
            }
        }
    }
    uint8_t s_h = sh[0], s_l = sl[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) {
        s_h = lane == (uint32_t)j ? sh[j] : s_h;
        s_l = lane == (uint32_t)j ? sl[j] : s_l;
    }
    if (lane < 8 && c0 + lane < nn) {
        h_atom[sfb_pos_hi<BN>(c0 + lane) + quarter] = s_h;
        h_atom[sfb_pos_lo<BN>(c0 + lane) + quarter] = s_l;
    }
}

// Fast mode: the same 8 columns of SiLU(gate) * up as E2M1 codes for the
// down GEMM -- per column one 32-element K block (the warp's 32 rows) with
// one E8M0 scale; lanes 2i and 2i+1 form byte i of the row's packed codes
// ([rows][h_stride] bytes, element 2i in the low nibble), stored by the even
// lane; lane j stores column j's scale byte.
template <int BN>
__device__ __forceinline__ void h_store8_fp4(const float* hv, uint32_t c0, uint32_t nn, uint64_t row0, uint32_t m,
                                             uint32_t lane, uint32_t quarter, const BsParams& p, uint8_t* h_atom) {
    float mx[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) mx[j] = warp_max_abs(hv[j]);
    uint32_t byte[8];
    uint8_t sc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int e = fp4_block_exp(mx[j]);
        const uint32_t code = cvt_e2m1x2(hv[j] * pow2f(-e), 0.0f) & 0xFu;
        byte[j] = code | (__shfl_down_sync(0xffffffffu, code, 1) << 4);
        sc[j] = (uint8_t)(e + 127);
    }
    uint8_t* hp = p.h_out + (row0 + c0) * p.h_stride + (m >> 1);
    if ((lane & 1u) == 0) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (c0 + j < nn) hp[(uint64_t)j * p.h_stride] = (uint8_t)byte[j];
        }
    }
    uint8_t s = sc[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) s = lane == (uint32_t)j ? sc[j] : s;
    if (lane < 8 && c0 + lane < nn) h_atom[sfb_pos_hi<BN>(c0 + lane) + quarter] = s;
}

template <int BN, bool FP4 = false>
__device__ __forceinline__ void gu_store8(const float* g, const float* u, uint32_t c0, uint32_t nn, uint64_t row0,
                                          uint32_t m, uint32_t lane, uint32_t quarter, const BsParams& p,
                                          uint8_t* h_atom) {
    float hv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) hv[j] = silu_fast(g[j]) * u[j];
    if (p.act != 0) {  // uniform across the grid
#pragma unroll
        for (int j = 0; j < 8; ++j) hv[j] = gelu_act(p.act, g[j]) * u[j];
    }
    if constexpr (FP4) {
        h_store8_fp4<BN>(hv, c0, nn, row0, m, lane, quarter, p, h_atom);
    } else {
        h_store8<BN>(hv, c0, nn, row0, m, lane, quarter, p, h_atom);
    }
}

// One warp group's share [cb, cb + W) of a gate/up tile's token columns (the
// group's four warps cover the 128 TMEM lanes): drain, release the group's
// share of the accumulator, then SiLU * up, the hi/lo split and the stores.
// Stacked tiles drain into registers first, so the release comes before the
// math and the next tile's MMAs overlap it.
// Hands an accumulator back to the MMA issuer after this thread's last TMEM
// read (tc_fence_before already done): one arrival per thread on the local
// barrier, or, in a CTA pair, one per warp on the rank-0 CTA's barrier
// (acc_empty_cl, a shared::cluster address).
template <bool PAIR>
__device__ __forceinline__ void acc_release(uint64_t* acc_empty_bar, uint32_t acc_empty_cl) {
    if constexpr (PAIR) {
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive_cluster(acc_empty_cl);
    } else {
        mbar_arrive(acc_empty_bar);
    }
}

template <int BN, int W, bool FP4 = false, bool PAIR = false>
__device__ __forceinline__ void gu_tile_part(const BsParams& p, const BsTileX& tc, uint32_t dbase, uint32_t cb,
                                             uint32_t m, uint32_t lane, uint32_t quarter, uint8_t* h_atom,
                                             uint64_t* acc_empty_bar, uint32_t acc_empty_cl) {
    constexpr bool kStackN = !FP4 && BN <= 64;
    constexpr uint32_t kLoOff = kStackN ? BN : 0;  // stacked: lo half follows hi
    constexpr uint32_t kProjOff = kStackN ? 2 * BN : BN;
    if constexpr (kStackN) {
        float g[W], u[W];
#pragma unroll
        for (uint32_t j0 = 0; j0 < (uint32_t)W; j0 += 16) {
            const uint32_t c0 = cb + j0;
            if (c0 < tc.nn) {  // uniform across the warp
                uint32_t a[16], b[16], c[16], d[16];
                MOE_TMEM_LD16(dbase + c0, a);
                MOE_TMEM_LD16(dbase + kLoOff + c0, b);
                MOE_TMEM_LD16(dbase + kProjOff + c0, c);
                MOE_TMEM_LD16(dbase + kProjOff + kLoOff + c0, d);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    g[j0 + i] = __uint_as_float(a[i]) + __uint_as_float(b[i]);
                    u[j0 + i] = __uint_as_float(c[i]) + __uint_as_float(d[i]);
                }
            }
        }
        tc_fence_before();
        acc_release<PAIR>(acc_empty_bar, acc_empty_cl);
#pragma unroll
        for (uint32_t j0 = 0; j0 < (uint32_t)W; j0 += 8) {
            const uint32_t c0 = cb + j0;
            if (c0 >= tc.nn) break;  // uniform across the warp
            gu_store8<BN>(g + j0, u + j0, c0, tc.nn, tc.row0, m, lane, quarter, p, h_atom);
        }
    } else {
        for (uint32_t c0 = cb; c0 < cb + W && c0 < tc.nn; c0 += 16) {
            uint32_t a[16], c[16];
            MOE_TMEM_LD16(dbase + c0, a);
            MOE_TMEM_LD16(dbase + kProjOff + c0, c);
            tmem_wait_ld();
            float v0[16], v1[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                v0[i] = __uint_as_float(a[i]);
                v1[i] = __uint_as_float(c[i]);
            }
            gu_store8<BN, FP4>(v0, v1, c0, tc.nn, tc.row0, m, lane, quarter, p, h_atom);
            if (c0 + 8 < tc.nn) {
                gu_store8<BN, FP4>(v0 + 8, v1 + 8, c0 + 8, tc.nn, tc.row0, m, lane, quarter, p, h_atom);
            }
        }
        tc_fence_before();
        acc_release<PAIR>(acc_empty_bar, acc_empty_cl);
    }
}

template <int MODE, int BN, bool FP4, bool PAIR, int KB>
__global__ void __launch_bounds__(BsCfg<MODE, BN, FP4, PAIR, KB>::kThreads, 1)
    gemm_bs_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                                         const __grid_constant__ CUtensorMap tmap_b,
                                                         const BsParams p) {
    using C = BsCfg<MODE, BN, FP4, PAIR, KB>;
    // gate/up with one accumulator: the epilogue warps, the scale-factor
    // warps and (128-token tiles) warps 10-17 drain and store one group of
    // each tile's columns each (the MMAs wait for the whole accumulator
    // anyway), dividing the epilogue's time per tile
    constexpr bool kGuSplit = C::kGuSplit;
    constexpr int kGuW = BN / C::kEpiGroups;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // scale blocks first (small), then the 1024-aligned operand tiles
    uint8_t* sf_base = smem;                                         // [stages][KB][kSFBlock]
    uint8_t* a_base = smem + C::kStages * C::kSFStage;               // [stages][KB][kNA][16 KB]
    a_base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(a_base) + 1023) & ~uintptr_t(1023));
    uint8_t* b_base = a_base + C::kStages * KB * C::kNA * C::kABytes;  // [stages][KB][terms][kBBytes]
    uint64_t* bars = reinterpret_cast<uint64_t*>(b_base + C::kStages * KB * C::kBTerms * C::kBBytes);
    uint64_t* load_full = bars;
    uint64_t* load_empty = load_full + C::kStages;
    uint64_t* sf_full = load_empty + C::kStages;   // scale factors stored in TMEM
    uint64_t* acc_full = sf_full + C::kStages;
    uint64_t* acc_empty = acc_full + C::kAccs;
    uint64_t* sf_load = acc_empty + C::kAccs;      // CTA pairs: this CTA's scale blocks landed
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(sf_load + (PAIR ? C::kStages : 0));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // CTA pairs walk the tile table per pair (a tile entry's row tile is a
    // pair of 128-row tiles; rank 1 takes the second) and the rank-0 CTA
    // issues the M = 256 MMAs.  The MMA waits on the rank-0 CTA's load_full
    // (both CTAs' operand copies complete there), sf_full (both CTAs' scale-
    // factor warps) and acc_empty (both CTAs' epilogues); its commits arrive
    // on load_empty and acc_full in both CTAs.  Each CTA's scale blocks land
    // on its own sf_load.
    const uint32_t rank = PAIR ? cluster_ctarank() : 0;
    const uint32_t first = PAIR ? blockIdx.x >> 1 : blockIdx.x;
    const uint32_t step = PAIR ? gridDim.x >> 1 : gridDim.x;
    auto tile_at = [&](uint32_t t) {
        BsTileX tc = load_tile(p, t);
        if constexpr (PAIR) tc.mt = tc.mt * 2 + rank;
        return tc;
    };
    // token columns of a tile's MMAs (stacked: hi rows [0, BN), lo rows [BN, 2 BN))
    auto tile_n = [](uint32_t nn) { return C::kStackN ? 2u * BN : max(16u, (nn + 15u) & ~15u); };
    if (threadIdx.x == 0) {
        for (int i = 0; i < C::kStages; ++i) {
            mbar_init(&load_full[i], PAIR ? 2 : 1);
            mbar_init(&load_empty[i], 1);
            mbar_init(&sf_full[i], PAIR ? 8 : 4);
            if (PAIR) mbar_init(&sf_load[i], 1);
        }
        for (int i = 0; i < C::kAccs; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], PAIR ? 2 * 4 * C::kEpiGroups : 128 * C::kEpiGroups);
        }
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
    }
    if (warp == 1) {
        if constexpr (PAIR) {
            tmem_alloc_pair(tmem_holder, 512);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_holder, 512);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    if constexpr (PAIR) {
        cluster_sync();  // both CTAs' barriers initialised before any remote arrival
    } else {
        __syncthreads();
    }
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    // The tile table and weights were ready before this grid launched (the
    // previous kernel triggers only after its own wait); the activations
    // (B and its scales) come from the previous kernel and are read only
    // after pdl_wait() in the producer.
    pdl_trigger();
    const uint32_t total = p.tile_off[p.groups];
    constexpr uint32_t kSfCol0 = 256;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            bool ok = true;
            constexpr uint32_t kOpBytes = C::kNA * C::kATx + C::kBTerms * C::kBBytes;  // per K block
            // arms stage s for this CTA's copies of one use (nk K blocks)
            auto arm = [&](uint32_t s, uint32_t nk) {
                if constexpr (PAIR) {
                    mbar_arrive_expect_tx(&sf_load[s], nk * C::kSFBlock);
                    mbar_arrive_expect_tx_cluster(mapa_cluster(&load_full[s], 0), nk * kOpBytes);
                } else {
                    mbar_arrive_expect_tx(&load_full[s], nk * (kOpBytes + C::kSFBlock));
                }
            };
            auto sf_bar = [&](uint32_t s) { return PAIR ? &sf_load[s] : &load_full[s]; };
            // the weight blocks and weight scales of the stage's K blocks kt..
            auto load_a = [&](uint32_t s, uint64_t ablk0, uint64_t sblk0, uint32_t kt, uint32_t nk) {
#pragma unroll
                for (int kb = 0; kb < KB; ++kb) {
                    if ((uint32_t)kb >= nk) break;
                    bulk_g2s(sf_base + s * C::kSFStage + kb * C::kSFBlock, p.sfa + (sblk0 + kt + kb) * C::kSFA,
                             C::kSFA, sf_bar(s));
#pragma unroll
                    for (int pj = 0; pj < C::kNA; ++pj) {
                        const uint64_t b = ablk0 + (uint64_t)pj * p.m_tiles * p.k_tiles + kt + kb;  // weight block
                        uint8_t* dst = a_base + ((s * KB + kb) * C::kNA + pj) * C::kABytes;
                        if constexpr (PAIR) {
                            tma_load_2d_pair(dst, &tmap_a, 0, (int32_t)(b * 128), mapa_cluster(&load_full[s], 0));
                        } else {
                            tma_load_2d(dst, &tmap_a, 0, (int32_t)(b * 128), &load_full[s]);
                        }
                    }
                }
            };
            // weights of the first tile's first stages before waiting for the
            // previous kernel: they do not depend on it
            uint32_t pre = 0;
            if (first < total) {
                const BsTileX tc = tile_at(first);
                const uint32_t slot = p.group_slot ? __ldg(p.group_slot + tc.g) : tc.g;
                const uint64_t ablk0 = ((uint64_t)slot * C::kNA * p.m_tiles + tc.mt) * p.k_tiles;
                const uint64_t sblk0 = ((uint64_t)slot * p.m_tiles + tc.mt) * p.k_tiles;
                pre = min((uint32_t)C::kStages, ceil_div(p.k_tiles, KB));
                for (uint32_t s = 0; s < pre; ++s) {
                    const uint32_t nk = (KB == 1 ? 1u : min((uint32_t)KB, p.k_tiles - s * KB));
                    arm(s, nk);
                    load_a(s, ablk0, sblk0, s * KB, nk);
                }
            }
            pdl_wait();
            for (uint32_t tile = first; ok && tile < total; tile += step) {
                const BsTileX tc = tile_at(tile);
                const uint32_t slot = p.group_slot ? __ldg(p.group_slot + tc.g) : tc.g;  // weights of the group
                const uint64_t ablk0 = ((uint64_t)slot * C::kNA * p.m_tiles + tc.mt) * p.k_tiles;
                const uint64_t sblk0 = ((uint64_t)slot * p.m_tiles + tc.mt) * p.k_tiles;
                // a pair's rank 1 holds B rows [N/2, N) of the tile
                const int32_t b_row = (int32_t)(tc.row0 + (PAIR ? rank * (tile_n(tc.nn) / 2) : 0));
                for (uint32_t kt = 0; kt < p.k_tiles; kt += KB) {
                    if (!(ok = mbar_wait(&load_empty[stage], phase ^ 1, p.err, kErrTimeoutLoadEmpty))) break;
                    uint8_t* sf = sf_base + stage * C::kSFStage;
                    const uint32_t nk = (KB == 1 ? 1u : min((uint32_t)KB, p.k_tiles - kt));
                    const bool prefetched = tile == first && kt / KB < pre;
                    if (!prefetched) {
                        arm(stage, nk);
                        load_a(stage, ablk0, sblk0, kt, nk);
                    }
#pragma unroll
                    for (int kb = 0; kb < KB; ++kb) {
                        if ((uint32_t)kb >= nk) break;
                        bulk_g2s(sf + kb * C::kSFBlock + C::kSFA,
                                 p.sfb_atoms + ((uint64_t)tc.ntile * p.k_tiles + kt + kb) * C::kSFB, C::kSFB,
                                 sf_bar(stage));
                        uint8_t* bdst = b_base + (stage * KB + kb) * C::kBTerms * C::kBBytes;
                        if constexpr (FP4) {
                            // the tile's token rows: 64 bytes (128 codes) of each
                            tma_load_2d(bdst, &tmap_b, (int32_t)((kt + kb) * 64), (int32_t)tc.row0, &load_full[stage]);
                        } else if constexpr (PAIR) {
                            tma_load_3d_pair(bdst, &tmap_b, (int32_t)((kt + kb) * 128), b_row, 0,
                                             mapa_cluster(&load_full[stage], 0));
                        } else {
                            // hi and lo planes of the tile's token rows in one 3-D box
                            tma_load_3d(bdst, &tmap_b, (int32_t)((kt + kb) * 128), (int32_t)tc.row0, 0,
                                        &load_full[stage]);
                        }
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
        if (lane == 0 && rank == 0) {
            uint32_t stage = 0, phase = 0, acc = 0, accphase = 0;
            bool ok = true;
            for (uint32_t tile = first; ok && tile < total; tile += step) {
                const BsTileX tc = load_tile(p, tile);
                const uint32_t n_mma = tile_n(tc.nn);
                if (!(ok = mbar_wait(&acc_empty[acc], accphase ^ 1, p.err, kErrTimeoutAccEmpty))) break;
                tc_fence_after();
                const uint32_t d0 = tmem + acc * C::kAccCols;
                // The next stage's barriers are tested (without blocking) while
                // this stage's MMAs still fill the tensor pipe's queue; when both
                // have completed, the stage boundary needs no wait.
                bool next_ready = false;
                for (uint32_t kt = 0; kt < p.k_tiles; kt += KB) {
                    // operands landed (observed here too, so this thread's MMAs
                    // are ordered after the copies) and the scale factors are in TMEM
                    if (!next_ready) {
                        if (!(ok = mbar_wait(&load_full[stage], phase, p.err, kErrTimeoutLoadFull))) break;
                        if (!(ok = mbar_wait(&sf_full[stage], phase, p.err, kErrTimeoutAFull))) break;
                    }
                    next_ready = false;
                    const bool look = kt + KB < p.k_tiles;
                    const uint32_t nstage = stage + 1 == (uint32_t)C::kStages ? 0u : stage + 1;
                    const uint32_t nphase = stage + 1 == (uint32_t)C::kStages ? phase ^ 1 : phase;
                    auto look_ahead = [&]() {
                        next_ready = look && mbar_test_wait(&load_full[nstage], nphase) &&
                                     mbar_test_wait(&sf_full[nstage], nphase);
                    };
                    tc_fence_after();
                    const uint32_t nk = (KB == 1 ? 1u : min((uint32_t)KB, p.k_tiles - kt));
#pragma unroll
                    for (int kb = 0; kb < KB; ++kb) {
                    if ((uint32_t)kb >= nk) break;
                    const uint32_t sfc = tmem + kSfCol0 + stage * C::kSFCols + kb * C::kSFBlockCols;
                    const uint32_t sfb = sfc + C::kNA * 4;
                    const uint32_t a_addr = smem_u32(a_base + (stage * KB + kb) * C::kNA * C::kABytes);
                    const uint32_t b_addr = smem_u32(b_base + (stage * KB + kb) * C::kBTerms * C::kBBytes);
                    const uint32_t kacc = kt + kb;  // 0 only for the tile's first K block
                    if constexpr (FP4) {
                        // two K = 64 MMAs per 128-K stage, scale bytes {0, 1} then {2, 3}
#pragma unroll
                        for (int kk = 0; kk < 2; ++kk) {
                            const uint32_t idesc = idesc_fp4_m128(n_mma, 2 * kk);
                            const uint64_t bdesc = smem_desc_sw64(b_addr + kk * 32);
#pragma unroll
                            for (int pj = 0; pj < C::kNA; ++pj) {
                                const uint64_t adesc = smem_desc_sw64(a_addr + pj * C::kABytes + kk * 32);
                                mma_fp4(d0 + pj * BN, adesc, bdesc, idesc, sfc + pj * 4, sfb, (kacc | kk) != 0);
                            }
                            if ((uint32_t)kb + 1 == nk && kk == 0) look_ahead();
                        }
                    } else {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint32_t idesc = idesc_bs(PAIR ? 256 : 128, n_mma, kk);
                        const uint64_t bhi = smem_desc_sw128(b_addr + kk * 32);
#pragma unroll
                        for (int pj = 0; pj < C::kNA; ++pj) {
                            const uint64_t adesc = smem_desc_sw128(a_addr + pj * C::kABytes + kk * 32);
                            if (C::kStackN) {
                                mma_bs(d0 + pj * 2 * BN, adesc, bhi, idesc, sfc + pj * 4, sfb, (kacc | kk) != 0);
                            } else {
                                const uint64_t blo = smem_desc_sw128(b_addr + C::kBBytes + kk * 32);
                                const uint32_t d = d0 + pj * BN;
                                if constexpr (PAIR) {
                                    mma_bs_pair(d, adesc, bhi, idesc, sfc + pj * 4, sfb, (kacc | kk) != 0);
                                    mma_bs_pair(d, adesc, blo, idesc, sfc + pj * 4, sfb + 4, 1);
                                } else {
                                    mma_bs(d, adesc, bhi, idesc, sfc + pj * 4, sfb, (kacc | kk) != 0);
                                    mma_bs(d, adesc, blo, idesc, sfc + pj * 4, sfb + 4, 1);
                                }
                            }
                        }
                        if ((uint32_t)kb + 1 == nk && kk == 2) look_ahead();
                    }
                    }
                    }
                    if constexpr (PAIR) {
                        mma_commit_pair(&load_empty[stage], 0x3);
                    } else {
                        mma_commit(&load_empty[stage]);
                    }
                    if (++stage == C::kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                if constexpr (PAIR) {
                    mma_commit_pair(&acc_full[acc], 0x3);
                } else {
                    mma_commit(&acc_full[acc]);
                }
                if (++acc == C::kAccs) {
                    acc = 0;
                    accphase ^= 1;
                }
            }
        }
    } else if (warp >= 6 && warp < 10) {
        // ------------------------------------------------------------ scale factors (warps 6-9)
        // Each warp stores the stage's scale blocks into its TMEM lane quarter
        // of the stage's scale columns: lane l of every quarter holds bytes
        // [16 l, 16 l + 16) of each 512-byte block (the layout the MMA reads).
        // Doing this with tcgen05.st here keeps it off the tensor pipe.  The
        // slot of stage u is free once stage u's scale blocks have landed: the
        // producer reloaded them only after the MMAs of stage u - kStages were
        // done.  In a pair each CTA stores its own rows' A scales and all the
        // tile's B scales.
        const uint32_t lane_addr = ((warp & 3) * 32) << 16;
        uint32_t stage = 0, phase = 0, eaccphase = 0;
        bool ok = true;
        for (uint32_t tile = first; ok && tile < total; tile += step) {
            for (uint32_t kt = 0; kt < p.k_tiles; kt += KB) {
                ok = mbar_wait(PAIR ? &sf_load[stage] : &load_full[stage], phase, p.err, kErrTimeoutLoadFull);
                if (!__all_sync(0xffffffffu, ok)) {
                    ok = false;
                    break;
                }
                const uint8_t* sf = sf_base + stage * C::kSFStage + lane * 16;
                const uint32_t col = tmem + lane_addr + kSfCol0 + stage * C::kSFCols;
                const int nq = (int)(KB == 1 ? 1u : min((uint32_t)KB, p.k_tiles - kt)) * (C::kSFBlock / 512);
#pragma unroll
                for (int q = 0; q < C::kSFStage / 512; ++q) {
                    if (q >= nq) break;
                    const uint4 v = *reinterpret_cast<const uint4*>(sf + q * 512);
                    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
                    MOE_TMEM_ST4(col + q * 4, w);
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if constexpr (PAIR) {
                        mbar_arrive_cluster(mapa_cluster(&sf_full[stage], 0));
                    } else {
                        mbar_arrive(&sf_full[stage]);
                    }
                }
                if (++stage == C::kStages) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if constexpr (kGuSplit) {
                if (!ok) break;
                const BsTileX tc = tile_at(tile);
                ok = mbar_wait(&acc_full[0], eaccphase, p.err, kErrTimeoutAccFull, true);
                if (!__all_sync(0xffffffffu, ok)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t quarter = warp & 3;
                uint8_t* h_atom = p.sfh_atoms + ((uint64_t)tc.ntile * p.m_tiles + tc.mt) * C::kSFB;
                gu_tile_part<BN, kGuW, FP4, PAIR>(p, tc, tmem + lane_addr, kGuW, tc.mt * 128 + quarter * 32 + lane,
                                                  lane, quarter, h_atom, &acc_empty[0],
                                                  PAIR ? mapa_cluster(&acc_empty[0], 0) : 0u);
                eaccphase ^= 1;
            }
        }
    } else if (warp >= 10) {
        // ------------------------------------------------------------ epilogue groups 2 and 3
        // (gate/up 128-token tiles with one accumulator: columns
        // [group * kGuW, (group + 1) * kGuW) of each tile)
        if constexpr (C::kEpiGroups == 4) {
            const uint32_t quarter = warp & 3;
            const uint32_t lane_addr = (quarter * 32) << 16;
            const uint32_t group = (warp - 2) >> 2;
            uint32_t eaccphase = 0;
            bool ok = true;
            for (uint32_t tile = first; ok && tile < total; tile += step) {
                const BsTileX tc = tile_at(tile);
                ok = mbar_wait(&acc_full[0], eaccphase, p.err, kErrTimeoutAccFull, true);
                if (!__all_sync(0xffffffffu, ok)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint8_t* h_atom = p.sfh_atoms + ((uint64_t)tc.ntile * p.m_tiles + tc.mt) * C::kSFB;
                gu_tile_part<BN, kGuW, FP4, PAIR>(p, tc, tmem + lane_addr, group * kGuW,
                                                  tc.mt * 128 + quarter * 32 + lane, lane, quarter, h_atom,
                                                  &acc_empty[0], PAIR ? mapa_cluster(&acc_empty[0], 0) : 0u);
                eaccphase ^= 1;
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const uint32_t quarter = warp & 3;
        const uint32_t r = quarter * 32 + lane;
        const uint32_t lane_addr = (quarter * 32) << 16;
        uint32_t acc = 0, accphase = 0;
        bool ok = true;
        for (uint32_t tile = first; ok && tile < total; tile += step) {
            const BsTileX tc = tile_at(tile);
            ok = mbar_wait(&acc_full[acc], accphase, p.err, kErrTimeoutAccFull, true);
            if (!__all_sync(0xffffffffu, ok)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t m = tc.mt * 128 + r;
            const uint64_t row0 = tc.row0;
            const uint32_t dbase = tmem + lane_addr + acc * C::kAccCols;
            const uint32_t acc_empty_cl = PAIR ? mapa_cluster(&acc_empty[acc], 0) : 0u;
            // the down GEMM's scale block for this token tile and 128-K stage (= mt)
            uint8_t* h_atom =
                MODE == kGateUp ? p.sfh_atoms + ((uint64_t)tc.ntile * p.m_tiles + tc.mt) * C::kSFB : nullptr;
            constexpr uint32_t kLoOff = C::kStackN ? BN : 0;        // stacked: lo half follows hi
            if constexpr (MODE == kGateUp) {
                gu_tile_part<BN, kGuW, FP4, PAIR>(p, tc, dbase, 0, m, lane, quarter, h_atom, &acc_empty[acc],
                                                  acc_empty_cl);
                if (++acc == C::kAccs) {
                    acc = 0;
                    accphase ^= 1;
                }
                continue;
            }
            {
                // 32 token columns per round: all TMEM loads, one wait, the stores
                for (uint32_t c0 = 0; c0 < tc.nn; c0 += 32) {
                    uint32_t a0[16], a1[16], b0[16], b1[16];
                    MOE_TMEM_LD16(dbase + c0, a0);
                    MOE_TMEM_LD16(dbase + c0 + 16, a1);
                    if (C::kStackN) {
                        MOE_TMEM_LD16(dbase + kLoOff + c0, b0);
                        MOE_TMEM_LD16(dbase + kLoOff + c0 + 16, b1);
                    }
                    tmem_wait_ld();
                    float v0[32];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        v0[i] = __uint_as_float(a0[i]) + (C::kStackN ? __uint_as_float(b0[i]) : 0.f);
                        v0[16 + i] = __uint_as_float(a1[i]) + (C::kStackN ? __uint_as_float(b1[i]) : 0.f);
                    }
                    if (!p.ret_ptrs && !p.y_row_map) {
                        // permuted rows in order: straight-line stores (the tail
                        // chunk's are predicated)
                        float* yp = p.y_out + (row0 + c0) * p.y_stride + m;
                        if (m < p.m_valid) {
                            if (c0 + 32 <= tc.nn) {
#pragma unroll
                                for (int i = 0; i < 32; ++i) yp[(uint64_t)i * p.y_stride] = v0[i];
                            } else {
#pragma unroll
                                for (int i = 0; i < 32; ++i)
                                    if (c0 + i < tc.nn) yp[(uint64_t)i * p.y_stride] = v0[i];
                            }
                        }
                    } else {
                        // rows by source token (and, with expert parallelism,
                        // other ranks' rows into their return buffers over
                        // NVLink): lane i resolves the destination row of chunk
                        // column i once, the pointers are shuffled out
                        uint64_t my_dst = 0;
                        if (c0 + lane < tc.nn) {
                            const uint64_t prow = row0 + c0 + lane;
                            const uint64_t orow = p.y_row_map ? __ldg(p.y_row_map + prow) : prow;
                            float* dst = p.y_out + orow * p.y_stride;
                            if (p.ret_ptrs && orow < p.ret_rows) {
                                uint32_t r = 0;
                                while (r + 1 < p.ret_world && __ldg(p.ret_roff + r + 1) <= orow) ++r;
                                dst = p.ret_ptrs[r] +
                                      ((uint64_t)__ldg(p.ret_base + r) + orow - __ldg(p.ret_roff + r)) * p.y_stride;
                            }
                            my_dst = reinterpret_cast<uint64_t>(dst);
                        }
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            float* dst = reinterpret_cast<float*>(__shfl_sync(0xffffffffu, my_dst, i));
                            if (m < p.m_valid && c0 + i < tc.nn) dst[m] = v0[i];
                        }
                    }
                }
            }
            tc_fence_before();
            acc_release<PAIR>(&acc_empty[acc], acc_empty_cl);
            if (++acc == C::kAccs) {
                acc = 0;
                accphase ^= 1;
            }
        }
        if (MODE == kDown && p.ret_ptrs) __threadfence_system();  // peer stores before the exchange barrier
    }

    tc_fence_before();
    if constexpr (PAIR) {
        cluster_sync();  // no MMA, remote arrival or TMEM access of either CTA is left
    } else {
        __syncthreads();
    }
    tc_fence_after();
    if (warp == 1) {
        if constexpr (PAIR) {
            tmem_dealloc_pair(tmem, 512);
        } else {
            tmem_dealloc(tmem, 512);
        }
    }
}

// CTA-pair grids: two CTAs per cluster, as many clusters as can be resident
// at once (the SMs of a GPC pair up by TPC), found once per device and mode.
template <typename K>
static int pair_grid(K kernel, int smem, int threads, int num_sms, int* cache) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return 0;
    if (cache[dev] == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(num_sms & ~1));
        cfg.blockDim = dim3((unsigned)threads);
        cfg.dynamicSmemBytes = (size_t)smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess) clusters = 0;
        cache[dev] = clusters > 0 ? std::min(2 * clusters, num_sms & ~1) : -1;
    }
    return cache[dev];
}

template <int MODE, int BN, bool FP4, bool PAIR, int KB = 1>
static cudaError_t launch_bs_mode(const CUtensorMap& ta, const CUtensorMap& tb, const BsParams& p, int num_sms,
                                  cudaStream_t st, bool pdl) {
    using C = BsCfg<MODE, BN, FP4, PAIR, KB>;
    static uint64_t attr_set = 0;  // one bit per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && !((attr_set >> dev) & 1u)) {
        e = cudaFuncSetAttribute(gemm_bs_kernel<MODE, BN, FP4, PAIR, KB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 C::kSmem);
        if (e != cudaSuccess) return e;
        attr_set |= 1ull << dev;
    }
    if constexpr (PAIR) {
        static int grid_cache[64] = {};
        const int grid = pair_grid(gemm_bs_kernel<MODE, BN, FP4, PAIR, KB>, C::kSmem, C::kThreads, num_sms,
                                   grid_cache);
        if (grid <= 0) return cudaErrorNotSupported;
        return launch_kernel_cluster2(gemm_bs_kernel<MODE, BN, FP4, PAIR, KB>, dim3(grid), dim3(C::kThreads),
                                      C::kSmem, st, pdl, ta, tb, p);
    } else {
        return launch_kernel(gemm_bs_kernel<MODE, BN, FP4, PAIR, KB>, dim3(num_sms), dim3(C::kThreads), C::kSmem,
                             st, pdl, ta, tb, p);
    }
}

template <int MODE, bool FP4>
static cudaError_t launch_bs_width(int block_n, bool pair, const CUtensorMap& ta, const CUtensorMap& tb,
                                   const BsParams& p, int num_sms, cudaStream_t st, bool pdl) {
    if constexpr (!FP4 && MODE == kDown) {
        // stacked down tiles: two K blocks per stage (3 stages of 66 KB at 64
        // tokens; measured at config 1, 256 tokens: 68 -> 65 us).  The gate/up
        // ones keep one: two 99 KB stages are too shallow for their weight
        // stream (105 -> 116 us).
        if (block_n == 32) return launch_bs_mode<MODE, 32, false, false, 2>(ta, tb, p, num_sms, st, pdl);
        if (block_n == 64) return launch_bs_mode<MODE, 64, false, false, 2>(ta, tb, p, num_sms, st, pdl);
    }
    if (block_n == 32) return launch_bs_mode<MODE, 32, FP4, false>(ta, tb, p, num_sms, st, pdl);
    if (block_n == 64) return launch_bs_mode<MODE, 64, FP4, false>(ta, tb, p, num_sms, st, pdl);
    if constexpr (FP4) {
        // the fast mode's 128-token tiles: 2 K blocks per stage for gate/up,
        // 4 for down (measured at config 4: gate/up 3.56 / 3.02 / 3.21 ms and
        // down 2.50 / 2.08 / 1.86 ms with 1 / 2 / 4 blocks per stage)
        constexpr int kFkb = MODE == kGateUp ? 2 : 4;
        return launch_bs_mode<MODE, 128, true, false, kFkb>(ta, tb, p, num_sms, st, pdl);
    }
    if constexpr (!FP4) {
        if (pair) {
            // two 128-K blocks per stage
            return launch_bs_mode<MODE, 128, false, true, 2>(ta, tb, p, num_sms, st, pdl);
        }
    }
    return launch_bs_mode<MODE, 128, FP4, false>(ta, tb, p, num_sms, st, pdl);
}

cudaError_t launch_gemm_bs(int mode, int block_n, const CUtensorMap& ta, const CUtensorMap& tb, const BsParams& p,
                           int num_sms, cudaStream_t st, bool pdl, bool fp4, bool pair) {
    if (pair && (fp4 || block_n != 128)) return cudaErrorInvalidValue;
    if (mode == kGateUp) {
        return fp4 ? launch_bs_width<kGateUp, true>(block_n, false, ta, tb, p, num_sms, st, pdl)
                   : launch_bs_width<kGateUp, false>(block_n, pair, ta, tb, p, num_sms, st, pdl);
    }
    return fp4 ? launch_bs_width<kDown, true>(block_n, false, ta, tb, p, num_sms, st, pdl)
               : launch_bs_width<kDown, false>(block_n, pair, ta, tb, p, num_sms, st, pdl);
}

}  // namespace moe_b200
