// Kernel launchers shared by the C-ABI layer (api.cu).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace moe_b200 {

// Per-group (expert) routing results on the device, written by the scan
// kernel and read by the grouped GEMMs' tile schedulers.
struct GroupInfo {
    uint32_t* count;        // [G] rows (token assignments) per group
    uint32_t* offset;       // [G+1] first permuted row of each group
    uint32_t* gu_tile_off;  // [G+1] prefix of gate/up GEMM tiles
    uint32_t* dn_tile_off;  // [G+1] prefix of down GEMM tiles
    uint32_t block_n;       // tokens per GEMM tile
    uint32_t gu_row_tiles;  // ceil(I / 128)
    uint32_t dn_row_tiles;  // ceil(H / 128)
};

struct GemmParams {
    const uint8_t* wt;        // repacked weights of group 0; group g at wt + g * group_stride
    uint64_t group_stride;    // bytes per group
    uint32_t k_tiles;         // K / 64 (K padded to 64)
    uint32_t m_valid;         // output columns to write (I padded to 64 for gate/up, H for down)
    uint32_t groups;          // G
    const uint32_t* count;
    const uint32_t* offset;
    const uint32_t* tile_off;
    uint16_t* h_out;          // gate/up: [rows][h_stride] bf16 SiLU(gate)*up
    uint32_t h_stride;
    float* y_out;             // down: [rows][y_stride] f32
    uint32_t y_stride;
    uint32_t* err;
};

enum GemmMode : int { kGateUp = 0, kDown = 1 };

// One grouped-GEMM tile, precomputed after routing so the GEMM roles read
// their work with a single 16-byte load.
struct TileEntry {
    uint32_t group;       // expert slot
    uint32_t mt;          // weight row tile
    uint32_t row0;        // first permuted row of the tile's tokens
    uint32_t nn_ntile;    // tokens in the tile (low 8 bits) | token-tile index << 8
};

// Block-scaled grouped GEMM parameters (gemm_bs.cu).
struct BsParams {
    uint32_t groups;
    const uint32_t* count;
    const uint32_t* offset;
    const uint32_t* tile_off;
    const TileEntry* tiles;   // [tile_off[groups]] entries
    const uint8_t* a_codes;   // weight blocks (8 KB each) in the order of the A tensor map
    uint32_t rows_pad;        // weight rows per matrix, padded to 128
    uint32_t m_tiles;         // rows_pad / 128
    uint32_t k_tiles;         // K (padded to 128) / 128
    const uint8_t* sfa;       // weight scale blocks, [groups][m_tiles][k_tiles][proj][512]
    const uint8_t* sfb_atoms; // activation scale blocks, [token tiles][k_tiles][512 (32-token) | 1024 (128-token)]
    uint8_t* h_out;           // gate/up output: [hi, lo][rows][h_stride] E4M3 terms of SiLU(gate)*up
    uint64_t h_plane;         // bytes between the hi and lo planes of h_out
    uint32_t h_stride;
    uint8_t* sfh_atoms;       // gate/up output: the down GEMM's scale blocks (same layout as sfb_atoms)
    float* y_out;             // down: [rows][y_stride] f32
    uint32_t y_stride;
    uint32_t m_valid;         // output rows to write (down)
    const uint32_t* group_slot;  // weight slot of each group; null: the group index itself
    const uint32_t* y_row_map;   // down: output row of each permuted row; null: the permuted row
    // down, expert parallelism: output rows below ret_rows belong to other
    // ranks' tokens and are stored straight into the source rank's return
    // buffer (peer memory): rows [ret_roff[r], ret_roff[r+1]) came from rank
    // r and go to ret_ptrs[r] starting at row ret_base[r].  Null: y_out only.
    float* const* ret_ptrs;
    const uint32_t* ret_roff;
    const uint32_t* ret_base;
    uint32_t ret_rows;
    uint32_t ret_world;
    int32_t act;              // gate/up: 0 SiLU, 1 GELU (erf form), 2 GELU (tanh form)
    uint32_t* err;
};

// Block parts the combine applies (block.cu); null pointers are absent parts.
struct BlockParts {
    const float* post_norm1;   // [H] RMSNorm weight of the shared expert's output
    const float* post_norm2;   // [H] RMSNorm weight of each routed expert's output
    const float* post_norm;    // [H] RMSNorm weight of the block output
    const float* down_scale;   // 1, E or E*H scales of the routed outputs
    uint64_t down_scale_count;
    float eps;                 // RMSNorm epsilon (<= 0: 1e-6)
    int unit_offset;           // RMSNorm by (1 + w)
};
// Exact-order row RMSNorm (block.cu): mode 0 the MoE pre-norm with weight w,
// mode 1 the router input scale (w = the scale, w_count values).
cudaError_t launch_row_norm_exact(const float* in, uint32_t rows, uint32_t H, const float* w, uint64_t w_count,
                                  int mode, float eps, int unit_offset, float* out_f32, uint16_t* out_bf16,
                                  cudaStream_t st);
// y[t] = post_norm(post_norm1(ys[t]) * gate[t] + sum_j w[t,j] * down_scale(post_norm2(yp[pos_of[t*K+j]])));
// ys, gate may be null.  H <= 25600.
cudaError_t launch_block_combine(const float* yp, uint32_t H, const uint32_t* pos_of, const int32_t* ids,
                                 const float* w, uint32_t T, uint32_t K, uint32_t E, const float* ys,
                                 const float* gate, const BlockParts& bp, uint16_t* y_bf16, float* y_f32,
                                 cudaStream_t st, bool pdl);

cudaError_t launch_repack_mxfp4(const uint8_t* gguf, uint32_t rows, uint32_t cols, uint8_t* out,
                                uint32_t tile_stride, cudaStream_t stream);
cudaError_t launch_dequant_wtiles(const uint8_t* tiles, uint32_t rows, uint32_t cols, uint32_t tile_stride,
                                  uint16_t* out, cudaStream_t stream);

// Logits + top-k; adds the number of kernels it launched to *launches.
// tmap_x / tmap_w (both or neither): router_tmap_x / router_tmap_w maps of
// x and w, for the TMA-fed logits kernel of large batches.
// Routing semantics (generation_router.cpp.inc:560-682).
struct RouteCfg {
    int sigmoid;          // sigmoid scores (else softmax)
    int norm_topk;        // renormalise the k weights
    float routed_scale;   // sigmoid routers: weights scaled by this
    uint32_t n_group;     // group limit (sigmoid routers): groups ...
    uint32_t topk_group;  // ... of which this many keep their scores; 0: none
};
cudaError_t launch_router(const uint16_t* x, const uint16_t* w, uint32_t T, uint32_t E, uint32_t H, uint32_t K,
                          const RouteCfg& rc, float* logits, int32_t* ids, float* wout, float* scores, uint32_t* err,
                          cudaStream_t st, uint32_t* launches, const CUtensorMap* tmap_x = nullptr,
                          const CUtensorMap* tmap_w = nullptr);
// The same routing from fp32 token rows x [T x H] (the logits in the
// reference's FMA order, then the same top-k).
cudaError_t launch_router_f32(const float* x, const uint16_t* w, uint32_t T, uint32_t E, uint32_t H, uint32_t K,
                              const RouteCfg& rc, float* logits, int32_t* ids, float* wout, float* scores,
                              cudaStream_t st, uint32_t* launches);
// Box of the router's tensor maps: 128 bf16 columns x box_rows rows, no
// swizzle (router_box_rows(true) for x, (false) for w).
uint32_t router_box_rows(bool tokens);
// Whether launch_router would use the TMA-fed kernel for this batch.
bool router_wants_tma(const uint16_t* x, const uint16_t* w, uint32_t T, uint32_t E, uint32_t H);
// Items per tile of the stable counting sort (8 warps x 8 steps x 32 lanes);
// sort_tiles(n) = ceil(n / kSortTile) tiles, each with a row of per-bucket
// counts in the tile_counts buffer.
constexpr uint32_t kSortTile = 2048;
uint32_t sort_tiles(uint32_t n);
// Permutation of T*K assignments (assignment a reads source row a / K) into
// E groups, plus an extra group of `shared_rows` rows whose source rows are
// shared_base + t.  row_info (may be null): per permuted row, its gate/up
// token tile << 8 | its index in the tile (gi.block_n, gi.gu_row_tiles).
cudaError_t launch_permute(const int32_t* ids, uint32_t T, uint32_t K, uint32_t E, uint32_t shared_rows,
                           uint32_t shared_base, uint32_t* tile_counts, uint32_t* rank, GroupInfo gi,
                           uint32_t* pos_of, uint32_t* row_token, uint32_t* row_assign, uint32_t* row_info,
                           uint32_t* err, cudaStream_t st);
// Single-block permutation + tile tables for n <= 8192 assignments and
// E <= 256 experts (route_small_fits); tile tables may be null.
bool route_small_fits(uint32_t n, uint32_t E);
cudaError_t launch_route_small(const int32_t* ids, uint32_t T, uint32_t K, uint32_t E, uint32_t shared_rows,
                               uint32_t shared_base, GroupInfo gi, TileEntry* gu_tiles, uint32_t gu_max,
                               TileEntry* dn_tiles, uint32_t dn_max, uint32_t* pos_of, uint32_t* row_token,
                               uint32_t* row_assign, uint32_t* row_info, uint32_t* err, cudaStream_t st, bool pdl);
// Generic pieces of the stable counting sort, used by the grouping utility.
struct AssignRec {
    uint32_t token_index, layer, expert;
    float router_score;
};
cudaError_t launch_sort_count(const int32_t* keys, uint32_t n, uint32_t nb, uint32_t* tile_counts, uint32_t* rank,
                              uint32_t* err, cudaStream_t st);
cudaError_t launch_sort_scan(uint32_t* tile_counts, uint32_t ntiles, uint32_t nb, GroupInfo gi, cudaStream_t st);
cudaError_t launch_group_pass(const AssignRec* a, const uint32_t* order_in, uint32_t* order_out, uint32_t n,
                              int field, int shift, int32_t* keys, uint32_t* tile_counts, uint32_t* rank,
                              GroupInfo gi, uint32_t* err, cudaStream_t st);
cudaError_t launch_group_finish(const AssignRec* a, const uint32_t* order, uint32_t n, AssignRec* sorted,
                                uint32_t* batches /* [n][4] */, uint32_t* batch_count, cudaStream_t st);
cudaError_t launch_iota(uint32_t* v, uint32_t n, cudaStream_t st);
cudaError_t launch_gather(const uint16_t* x, uint32_t H, uint32_t Kp, const uint32_t* row_token, uint32_t rows,
                          uint16_t* xp, cudaStream_t st);
// y[t] = ys[t] (shared expert rows, may be null) + sum_j w[t,j] * yp[pos_of[t*K+j]].
cudaError_t launch_combine(const float* yp, uint32_t H, const uint32_t* pos_of, const float* w, uint32_t T,
                           uint32_t K, const float* ys, uint16_t* y_bf16, float* y_f32, cudaStream_t st, bool pdl);
// cw [T x K]: the combine weights when some experts are missing (present
// [E] bytes, 0 = missing): 0 for missing experts; for the others w, times
// 1 / (the sum of the present experts' w, router order) when norm (a
// renormalising router); kErrAllExpertsMissing when a token has none (the
// reference's partial-failure policy, generation_mlp.cpp.inc:1219-1282).
cudaError_t launch_combine_weights(const int32_t* ids, const float* w, const uint8_t* present, uint32_t T,
                                   uint32_t K, uint32_t E, bool norm, float* cw, uint32_t* err, cudaStream_t st);

// tcgen05 grouped GEMMs (gemm_tc.cu).  `tmap_b` covers the permuted
// activation rows [rows x Kp] bf16 with a 64 x block_n box, 128-byte swizzle.
constexpr uint32_t kBlockN = 128;
cudaError_t launch_gemm_tc(int mode, const CUtensorMap& tmap_b, const GemmParams& p, int num_sms,
                           cudaStream_t st);
// Block-scaled tcgen05 grouped GEMMs (gemm_bs.cu) and their data preparation.
// Launchers taking `pdl` launch with programmatic stream serialization: the
// kernel may start while its predecessor drains and waits (griddepcontrol)
// before reading what the predecessor wrote.
cudaError_t launch_repack_bs(const uint8_t* gguf, uint32_t rows, uint32_t cols, uint32_t rows_pad, uint32_t Kp,
                             uint8_t* codes, uint8_t* sfa, uint32_t sf_stride, cudaStream_t st);
// GGUF MXFP4 rows [rows x ceil(cols/32)*17] of one projection, rebuilt from
// its block-scaled codes and scale blocks (the inverse of launch_repack_bs).
cudaError_t launch_bs_to_gguf(const uint8_t* codes, const uint8_t* sfa, uint32_t sf_stride, uint32_t rows,
                              uint32_t cols, uint32_t Kp, uint8_t* gguf, cudaStream_t st);
// xb [2][rows_cap][Kp]: permuted rows of x as exact hi/lo E4M3 terms; their
// scale words go to sf_atoms, one block per (token tile, 128-K stage), at the
// tile and index the permutation recorded in row_info.
cudaError_t launch_gather_quant_bs(const uint16_t* x, uint32_t H, uint32_t Kp, const uint32_t* row_token,
                                   const uint32_t* row_info, uint32_t rows, uint32_t rows_cap, uint32_t block_n,
                                   uint8_t* xb, uint8_t* sf_atoms, cudaStream_t st, bool pdl);
// The same planes, split once per token row of x [T x H] and stored at the
// token's permuted rows pos_of[t*K + j] (and shared_off[0] + t when set).
cudaError_t launch_scatter_quant_bs(const uint16_t* x, uint32_t H, uint32_t Kp, uint32_t T, uint32_t K,
                                    const uint32_t* pos_of, const uint32_t* shared_off, const uint32_t* row_info,
                                    uint32_t rows, uint32_t rows_cap, uint32_t block_n, uint8_t* xb,
                                    uint8_t* sf_atoms, cudaStream_t st, bool pdl);
cudaError_t launch_build_tiles(const uint32_t* count, const uint32_t* offset, const uint32_t* tile_off,
                               uint32_t groups, uint32_t m_tiles, uint32_t block_n, uint32_t max_tiles,
                               TileEntry* tiles, cudaStream_t st);
// `tb` is a 3-D map over [2][rows][K] E4M3 bytes with a {128, block_n, 2} box.
// fp4 (fast mode, kind::mxf4): `ta` is a byte map over the weight codes with
// a {64, 128} box and `tb` a byte map over [rows][K/2] packed E2M1 codes with
// a {64, block_n} box, both 64-byte swizzled; h_out is then [rows][I/2]
// packed codes and the scale blocks are 512 bytes for every tile width.
// pair (exact path, 128-token tiles): CTA pairs run cta_group::2 MMAs of 256
// weight rows; the tile table's row tiles are then pairs of 128-row tiles
// (m_tiles even) and `tb`'s box is {128, 64, 2}, half a tile's token rows.
cudaError_t launch_gemm_bs(int mode, int block_n, const CUtensorMap& ta, const CUtensorMap& tb, const BsParams& p,
                           int num_sms, cudaStream_t st, bool pdl, bool fp4 = false, bool pair = false);
// Fast mode: token rows of x as packed E2M1 codes [rows][Kp/2] with E8M0
// scale words in 512-byte blocks per (token tile, 128-K stage), stored at
// each of the token's permuted rows (as launch_scatter_quant_bs).
cudaError_t launch_scatter_quant_fp4(const uint16_t* x, uint32_t H, uint32_t Kp, uint32_t T, uint32_t K,
                                     const uint32_t* pos_of, const uint32_t* shared_off, const uint32_t* row_info,
                                     uint32_t rows, uint8_t* xq, uint8_t* sf_atoms, cudaStream_t st, bool pdl);

// CUDA-core grouped GEMMs used only to cross-check the tcgen05 kernels.
cudaError_t launch_gemm_simt(int mode, const uint16_t* b, uint32_t b_stride, uint32_t rows, const GemmParams& p,
                             uint32_t m_rows, cudaStream_t st);
// fp32 single-token expert (gate/up/SiLU/down) for the triplet entry point.
cudaError_t launch_triplet_f32(const uint8_t* gu_tiles, const uint8_t* dn_tiles, const float* x, uint32_t H,
                               uint32_t I, float* gate_out, float* up_out, float* out, cudaStream_t st);

}  // namespace moe_b200
