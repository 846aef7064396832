// C ABI of the B200 MoE expert-FFN hot path (include/moe_b200.h): engine,
// device weight cache, workspace and the per-layer launch sequence
//   router -> permute (count/scan/scatter) -> gather -> gate/up GEMM ->
//   down GEMM -> combine
// all enqueued on the caller's stream with no host synchronisation.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <new>
#include <vector>

#include "engine.h"

using namespace moe_b200;


namespace moe_b200 {

int check_dims(const moe_b200_layer_cfg_t* c, char* err) {
    if (!c) {
        set_err(err, "null layer config");
        return 0;
    }
    if (c->hidden == 0 || c->hidden % 8 != 0 || c->hidden > 65536) {
        set_err(err, "hidden=%u must be a positive multiple of 8 (<= 65536)", c->hidden);
        return 0;
    }
    if (c->intermediate == 0 || c->intermediate > 100000) {
        set_err(err, "invalid intermediate size %u", c->intermediate);
        return 0;
    }
    if (c->experts == 0 || c->experts > 1024) {
        set_err(err, "experts=%u outside 1..1024", c->experts);
        return 0;
    }
    if (c->gemm_path < MOE_B200_GEMM_BLOCKSCALED || c->gemm_path > MOE_B200_GEMM_MXF4_FAST) {
        set_err(err, "unknown gemm_path %d", c->gemm_path);
        return 0;
    }
    if (c->top_k == 0 || c->top_k > 32 || c->top_k > c->experts) {
        set_err(err, "top_k=%u outside 1..min(32, experts)", c->top_k);
        return 0;
    }
    if (c->score_func == MOE_B200_SCORE_SIGMOID && c->n_group > 256 && c->topk_group > 0 &&
        c->topk_group < c->n_group && c->experts % c->n_group == 0) {
        set_err(err, "n_group=%u: group limits of more than 256 groups are not supported", c->n_group);
        return 0;
    }
    return 1;
}

int get_encoder(moe_b200_engine* eng, char* err) {
    if (eng->encode) return 1;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
    if (!fn || q != cudaDriverEntryPointSuccess) {
        set_err(err, "cuTensorMapEncodeTiled unavailable");
        return 0;
    }
    eng->encode = reinterpret_cast<EncodeTiledFn>(fn);
    return 1;
}

// 2-D tiled tensor map with 128-byte swizzle.  `cols` counts elements of
// `dtype`; `row_bytes` is the global row stride.
int make_tmap2d(moe_b200_engine* eng, CUtensorMap* map, CUtensorMapDataType dtype, void* base, uint64_t cols,
                uint64_t rows, uint64_t row_bytes, uint32_t box_cols, uint32_t box_rows, char* err,
                CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    if (!get_encoder(eng, err)) return 0;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = eng->encode(map, dtype, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_err(err, "cuTensorMapEncodeTiled failed (%d)", (int)r);
        return 0;
    }
    return 1;
}

// 3-D map over [2][rows][cols] bytes (hi plane, lo plane) with a
// {128, box_rows, 2} box and 128-byte swizzle: one copy brings both terms.
int make_tmap_planes(moe_b200_engine* eng, CUtensorMap* map, void* base, uint64_t cols, uint64_t rows,
                     uint32_t box_rows, char* err) {
    if (!get_encoder(eng, err)) return 0;
    const cuuint64_t dims[3] = {cols, rows, 2};
    const cuuint64_t strides[2] = {cols, cols * rows};
    const cuuint32_t box[3] = {128, box_rows, 2};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = eng->encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base, dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_err(err, "cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
        return 0;
    }
    return 1;
}

// bf16 activation rows for the TMEM-decode path: 64-element x 32-row boxes.
int make_tmap(moe_b200_engine* eng, CUtensorMap* map, void* base, uint64_t cols, uint64_t rows, char* err) {
    return make_tmap2d(eng, map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, cols, rows, cols * 2, 64, 32, err);
}

// Tensor maps for the TMA-fed router logits kernel (x [T x H] and the router
// rows w [E x H], bf16, no swizzle).  Returns false when the batch takes
// another router kernel or a map cannot be made (the router then stages
// rows itself).
bool router_tmaps(moe_b200_engine* eng, const uint16_t* x, const uint16_t* w, uint32_t T, uint32_t E, uint32_t H,
                  CUtensorMap* tx, CUtensorMap* tw) {
    if (!router_wants_tma(x, w, T, E, H)) return false;
    char err[MOE_B200_ERR_LEN];
    if (!get_encoder(eng, err)) return false;
    auto enc = [&](CUtensorMap* m, const uint16_t* base, uint32_t rows, uint32_t box_rows) {
        const cuuint64_t dims[2] = {H, rows};
        const cuuint64_t strides[1] = {(cuuint64_t)H * 2};
        const cuuint32_t box[2] = {128, box_rows};
        const cuuint32_t estr[2] = {1, 1};
        return eng->encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    return enc(tx, x, T, router_box_rows(true)) && enc(tw, w, E, router_box_rows(false));
}

LayerWeights* get_layer(moe_b200_engine* eng, int32_t layer, char* err) {
    if (!eng) {
        set_err(err, "null engine");
        return nullptr;
    }
    if (layer < 0 || (size_t)layer >= eng->layers.size()) {
        set_err(err, "layer %d outside 0..%zu", layer, eng->layers.size() - 1);
        return nullptr;
    }
    return &eng->layers[layer];
}

// The layer's block-scaled expert store for experts of I = intermediate
// rows (H = the router's): allocated, zeroed and mapped on the first expert
// of a shape; a new intermediate size drops the layer's experts.
int ensure_bs_layout(moe_b200_engine* eng, LayerWeights* L, uint32_t intermediate, char* err) {
    if (L->I == intermediate && L->bs_gu_codes.ptr) return 1;
    const uint32_t hidden = L->H;
    L->I = 0;  // set once the store is complete, so a failure here starts over next time
    // a new shape drops the layer's tile form; it is derived again on demand
    L->gu.release();
    L->dn.release();
    L->gu_stride = 0;
    L->dn_stride = 0;
    L->rp_i = round_up(intermediate, 128);
    L->rp_h = round_up(hidden, 128);
    L->kq = round_up(hidden, 128);
    L->iq = round_up(intermediate, 128);
    const uint64_t slots = L->E + 1;
    L->bs_gu_codes.release();
    L->bs_gu_sfa.release();
    L->bs_dn_codes.release();
    L->bs_dn_sfa.release();
    L->present.assign(L->E + 1, 0);
    L->tile_ready.assign(L->E + 1, 0);
    CK(L->bs_gu_codes.reserve(slots * 2 * L->rp_i * (L->kq / 2)));
    CK(L->bs_gu_sfa.reserve(slots * 2 * (L->rp_i / 128) * (L->kq / 128) * 512));
    CK(L->bs_dn_codes.reserve(slots * L->rp_h * (L->iq / 2)));
    CK(L->bs_dn_sfa.reserve(slots * (L->rp_h / 128) * (L->iq / 128) * 512));
    // slots never uploaded hold zero codes: such an expert computes an
    // exact zero row, which is what skipping it adds (skip_missing)
    CK(cudaMemsetAsync(L->bs_gu_codes.ptr, 0, L->bs_gu_codes.bytes, eng->ustream));
    CK(cudaMemsetAsync(L->bs_gu_sfa.ptr, 0, L->bs_gu_sfa.bytes, eng->ustream));
    CK(cudaMemsetAsync(L->bs_dn_codes.ptr, 0, L->bs_dn_codes.bytes, eng->ustream));
    CK(cudaMemsetAsync(L->bs_dn_sfa.ptr, 0, L->bs_dn_sfa.bytes, eng->ustream));
    // codes are 8 KB blocks of 128 rows x 128 K: a "tall" tensor of 128-element
    // rows, one 128 x 128 box per block
    if (!make_tmap2d(eng, &L->tmap_gu_codes, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, L->bs_gu_codes.ptr, 128,
                     slots * 2 * L->rp_i * (L->kq / 128), 64, 128, 128, err) ||
        !make_tmap2d(eng, &L->tmap_dn_codes, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, L->bs_dn_codes.ptr, 128,
                     slots * L->rp_h * (L->iq / 128), 64, 128, 128, err) ||
        !make_tmap2d(eng, &L->tmap_gu_fp4, CU_TENSOR_MAP_DATA_TYPE_UINT8, L->bs_gu_codes.ptr, 64,
                     slots * 2 * L->rp_i * (L->kq / 128), 64, 64, 128, err, CU_TENSOR_MAP_SWIZZLE_64B) ||
        !make_tmap2d(eng, &L->tmap_dn_fp4, CU_TENSOR_MAP_DATA_TYPE_UINT8, L->bs_dn_codes.ptr, 64,
                     slots * L->rp_h * (L->iq / 128), 64, 64, 128, err, CU_TENSOR_MAP_SWIZZLE_64B)) {
        return 0;
    }
    L->I = intermediate;
    return 1;
}

// One expert slot's block-scaled form as the four byte ranges of an expert
// record, in record order: gate and up codes, their scale blocks, down codes,
// down scale blocks.
struct RecordPart {
    uint8_t* dev;
    uint64_t bytes;
};
void record_parts(const LayerWeights* L, uint32_t slot, RecordPart out[4]) {
    const uint64_t gu_codes = 2ull * L->rp_i * (L->kq / 2);
    const uint64_t gu_sfa = 2ull * (L->rp_i / 128) * (L->kq / 128) * 512;
    const uint64_t dn_codes = (uint64_t)L->rp_h * (L->iq / 2);
    const uint64_t dn_sfa = (uint64_t)(L->rp_h / 128) * (L->iq / 128) * 512;
    out[0] = {L->bs_gu_codes.as<uint8_t>() + slot * gu_codes, gu_codes};
    out[1] = {L->bs_gu_sfa.as<uint8_t>() + slot * gu_sfa, gu_sfa};
    out[2] = {L->bs_dn_codes.as<uint8_t>() + slot * dn_codes, dn_codes};
    out[3] = {L->bs_dn_sfa.as<uint8_t>() + slot * dn_sfa, dn_sfa};
}

int ensure_tile_form(moe_b200_engine* eng, LayerWeights* L, uint32_t slot, char* err) {
    if (slot >= L->present.size() || !L->present[slot]) {
        set_err(err, "expert slot %u not uploaded", slot);
        return 0;
    }
    if (L->tile_ready[slot]) return 1;
    const uint32_t H = L->H, I = L->I;
    if (!L->gu.ptr) {
        L->gu_stride = (uint64_t)ceil_div(I, kTileRows) * ceil_div(H, kTileK) * 2 * kTileBytes;
        L->dn_stride = (uint64_t)ceil_div(H, kTileRows) * ceil_div(I, kTileK) * kTileBytes;
        CK(L->gu.reserve(L->gu_stride * (L->E + 1)));
        CK(L->dn.reserve(L->dn_stride * (L->E + 1)));
    }
    const uint64_t gu_need = (uint64_t)I * ceil_div(H, 32) * 17;
    const uint64_t dn_need = (uint64_t)H * ceil_div(I, 32) * 17;
    cudaStream_t st = eng->ustream;
    CK(eng->staging.reserve(2 * gu_need + dn_need));
    uint8_t* stg = eng->staging.as<uint8_t>();
    const uint64_t mti = L->rp_i / 128, kth = L->kq / 128, mth = L->rp_h / 128, kti = L->iq / 128;
    for (int pj = 0; pj < 2; ++pj) {
        CK(launch_bs_to_gguf(L->bs_gu_codes.as<uint8_t>() + ((uint64_t)slot * 2 + pj) * L->rp_i * (L->kq / 2),
                             L->bs_gu_sfa.as<uint8_t>() + (uint64_t)slot * mti * kth * 1024 + pj * 512, 1024, I, H,
                             L->kq, stg + pj * gu_need, st));
    }
    CK(launch_bs_to_gguf(L->bs_dn_codes.as<uint8_t>() + (uint64_t)slot * L->rp_h * (L->iq / 2),
                         L->bs_dn_sfa.as<uint8_t>() + (uint64_t)slot * mth * kti * 512, 512, H, I, L->iq,
                         stg + 2 * gu_need, st));
    uint8_t* gu_dst = L->gu.as<uint8_t>() + L->gu_stride * slot;
    uint8_t* dn_dst = L->dn.as<uint8_t>() + L->dn_stride * slot;
    CK(launch_repack_mxfp4(stg, I, H, gu_dst, 2 * kTileBytes, st));
    CK(launch_repack_mxfp4(stg + gu_need, I, H, gu_dst + kTileBytes, 2 * kTileBytes, st));
    CK(launch_repack_mxfp4(stg + 2 * gu_need, H, I, dn_dst, kTileBytes, st));
    CK(cudaStreamSynchronize(st));
    L->tile_ready[slot] = 1;
    return 1;
}

int run_blockscaled(moe_b200_engine* eng, LayerWeights* L, const BsJob& job, cudaStream_t st, cudaEvent_t* ev,
                    uint32_t* launches, char* err) {
    auto mark = [&](int i) {
        if (ev) cudaEventRecord(ev[i], st);
    };
    const uint32_t H = L->H;
    const uint32_t n = job.T * job.K;
    if (reinterpret_cast<uintptr_t>(job.src) & 7) {
        set_err(err, "activation rows must start on an 8-byte boundary");
        return 0;
    }
    const uint32_t P = n + job.shared_rows;
    const uint32_t G = job.E + (job.shared_rows ? 1 : 0);
    const uint32_t Kq = L->kq, Iq = L->iq;  // K padded to 128
    const uint32_t rows_cap = std::max(P, 32u);
    // tokens per GEMM tile: 32 while the groups average at most 16 rows, 64
    // up to 160 rows, else 128: wider tiles re-read each weight block from L2
    // fewer times and issue fewer MMAs per token (measured: 256 tokens of
    // config 1, 32 rows per group, are 5 % faster with 64; config 3, 256 rows
    // per group, 3 % faster with 128)
    const uint64_t avg_x = G ? (uint64_t)P / G : 0;
    const uint32_t block_n = avg_x <= 16 ? 32u : (avg_x <= 160 ? 64u : kBlockN);
    const uint32_t ntiles = sort_tiles(n);
    const uint32_t token_tiles = P / block_n + G;  // upper bound of sum_g ceil(count_g / block_n)
    uint32_t* errw = eng->err_word.as<uint32_t>();

    CK(eng->tile_counts.reserve((size_t)std::max(ntiles, 1u) * std::max(job.E, 1u) * 4));
    CK(eng->rank.reserve((size_t)std::max(n, 1u) * 4));
    CK(eng->pos_of.reserve((size_t)std::max(n, 1u) * 4));
    CK(eng->row_token.reserve((size_t)P * 4));
    CK(eng->row_assign.reserve((size_t)P * 4));
    CK(eng->row_info.reserve((size_t)P * 4));
    CK(eng->g_count.reserve((size_t)(G + 1) * 4));
    CK(eng->g_offset.reserve((size_t)(G + 1) * 4));
    CK(eng->g_gu_off.reserve((size_t)(G + 1) * 4));
    CK(eng->g_dn_off.reserve((size_t)(G + 1) * 4));
    CK(eng->xb.reserve((size_t)2 * rows_cap * Kq));
    CK(eng->hb.reserve((size_t)2 * rows_cap * Iq));
    CK(eng->sfx_atoms.reserve((size_t)token_tiles * (Kq / 128) * 1024));
    CK(eng->sfh_atoms.reserve((size_t)token_tiles * (Iq / 128) * 1024));
    CK(eng->gu_tiles.reserve((size_t)token_tiles * (L->rp_i / 128) * sizeof(TileEntry)));
    CK(eng->dn_tiles.reserve((size_t)token_tiles * (L->rp_h / 128) * sizeof(TileEntry)));
    // the planes' row count is fixed by the buffer, so the maps only change
    // when a buffer is reallocated or the geometry changes
    struct MapSpec {
        CUtensorMap* maps;
        DevBuf* buf;
        uint32_t cols;
    } specs[2] = {{eng->tmap_xb, &eng->xb, Kq}, {eng->tmap_hb, &eng->hb, Iq}};
    for (int i = 0; i < 2 && job.fp4; ++i) {
        // fast mode: [rows][cols / 2] packed E2M1 bytes at the start of the
        // same buffer, 64-byte boxes of 32, 64 or 128 rows
        CUtensorMap* maps = i == 0 ? eng->tmap_xq : eng->tmap_hq;
        const uint64_t rows = specs[i].buf->bytes / (2ull * specs[i].cols);
        const uint64_t rb = specs[i].cols / 2;
        if (eng->fp4_map_key[i] != specs[i].buf->ptr || eng->fp4_map_dims[i][0] != specs[i].cols ||
            eng->fp4_map_dims[i][1] != rows) {
            for (int b = 0; b < 3; ++b) {
                if (!make_tmap2d(eng, &maps[b], CU_TENSOR_MAP_DATA_TYPE_UINT8, specs[i].buf->ptr, rb, rows, rb, 64,
                                 32u << b, err, CU_TENSOR_MAP_SWIZZLE_64B)) {
                    return 0;
                }
            }
            eng->fp4_map_key[i] = specs[i].buf->ptr;
            eng->fp4_map_dims[i][0] = specs[i].cols;
            eng->fp4_map_dims[i][1] = rows;
        }
    }
    for (int i = 0; i < 2; ++i) {
        const uint64_t rows = specs[i].buf->bytes / (2ull * specs[i].cols);
        if (eng->bs_map_key[i] != specs[i].buf->ptr || eng->bs_map_dims[i][0] != specs[i].cols ||
            eng->bs_map_dims[i][1] != rows) {
            if (!make_tmap_planes(eng, &specs[i].maps[0], specs[i].buf->ptr, specs[i].cols, rows, 32, err) ||
                !make_tmap_planes(eng, &specs[i].maps[1], specs[i].buf->ptr, specs[i].cols, rows, 64, err) ||
                !make_tmap_planes(eng, &specs[i].maps[2], specs[i].buf->ptr, specs[i].cols, rows, 128, err)) {
                return 0;
            }
            eng->bs_map_key[i] = specs[i].buf->ptr;
            eng->bs_map_dims[i][0] = specs[i].cols;
            eng->bs_map_dims[i][1] = rows;
        }
    }

    // CTA pairs take the 128-token tiles of the exact path when the weight
    // row tiles pair up; the tile table then counts pairs of row tiles
    const bool pair_ok = eng->cta_pairs && !job.fp4 && block_n == kBlockN;
    const bool pair_gu = pair_ok && (L->rp_i / 128) % 2 == 0;
    const bool pair_dn = pair_ok && (L->rp_h / 128) % 2 == 0;
    GroupInfo gi;
    gi.count = eng->g_count.as<uint32_t>();
    gi.offset = eng->g_offset.as<uint32_t>();
    gi.gu_tile_off = eng->g_gu_off.as<uint32_t>();
    gi.dn_tile_off = eng->g_dn_off.as<uint32_t>();
    gi.block_n = block_n;
    gi.gu_row_tiles = L->rp_i / (pair_gu ? 256 : 128);
    gi.dn_row_tiles = L->rp_h / (pair_dn ? 256 : 128);
    if (route_small_fits(n, job.E)) {
        // decode-sized batch: sort, offsets and both tile tables in one block
        CK(launch_route_small(job.ids, job.T, job.K, job.E, job.shared_rows, job.shared_base, gi,
                              eng->gu_tiles.as<TileEntry>(), token_tiles * (L->rp_i / 128),
                              eng->dn_tiles.as<TileEntry>(), token_tiles * (L->rp_h / 128),
                              eng->pos_of.as<uint32_t>(), eng->row_token.as<uint32_t>(),
                              eng->row_assign.as<uint32_t>(), eng->row_info.as<uint32_t>(), errw, st, true));
        *launches += 1;
    } else {
        CK(launch_permute(job.ids, job.T, job.K, job.E, job.shared_rows, job.shared_base,
                          eng->tile_counts.as<uint32_t>(), eng->rank.as<uint32_t>(), gi, eng->pos_of.as<uint32_t>(),
                          eng->row_token.as<uint32_t>(), eng->row_assign.as<uint32_t>(),
                          eng->row_info.as<uint32_t>(), errw, st));
        CK(launch_build_tiles(gi.count, gi.offset, gi.gu_tile_off, G, gi.gu_row_tiles, block_n,
                              token_tiles * (L->rp_i / 128), eng->gu_tiles.as<TileEntry>(), st));
        CK(launch_build_tiles(gi.count, gi.offset, gi.dn_tile_off, G, gi.dn_row_tiles, block_n,
                              token_tiles * (L->rp_h / 128), eng->dn_tiles.as<TileEntry>(), st));
        *launches += 5;
    }
    mark(2);
    // permuted source rows as exact hi/lo E4M3 terms + their scale blocks
    const uint64_t xb_rows = eng->xb.bytes / (2ull * Kq), hb_rows = eng->hb.bytes / (2ull * Iq);
    const bool per_token = job.K <= 32 && (job.shared_rows == 0 || (job.shared_base == 0 && job.shared_rows == job.T));
    if (job.src_shared && !per_token) {
        set_err(err, "separate shared-expert rows need the single-device layer");
        return 0;
    }
    if (job.src_shared) {
        // the routed rows from src, then the shared rows from src_shared
        const uint32_t* soff = job.shared_rows ? gi.offset + job.E : nullptr;
        if (job.fp4) {
            CK(launch_scatter_quant_fp4(job.src, H, Kq, job.T, job.K, eng->pos_of.as<uint32_t>(), nullptr,
                                        eng->row_info.as<uint32_t>(), P, eng->xb.as<uint8_t>(),
                                        eng->sfx_atoms.as<uint8_t>(), st, true));
            CK(launch_scatter_quant_fp4(job.src_shared, H, Kq, job.T, 0, eng->pos_of.as<uint32_t>(), soff,
                                        eng->row_info.as<uint32_t>(), P, eng->xb.as<uint8_t>(),
                                        eng->sfx_atoms.as<uint8_t>(), st, true));
        } else {
            CK(launch_scatter_quant_bs(job.src, H, Kq, job.T, job.K, eng->pos_of.as<uint32_t>(), nullptr,
                                       eng->row_info.as<uint32_t>(), P, (uint32_t)xb_rows, block_n,
                                       eng->xb.as<uint8_t>(), eng->sfx_atoms.as<uint8_t>(), st, true));
            CK(launch_scatter_quant_bs(job.src_shared, H, Kq, job.T, 0, eng->pos_of.as<uint32_t>(), soff,
                                       eng->row_info.as<uint32_t>(), P, (uint32_t)xb_rows, block_n,
                                       eng->xb.as<uint8_t>(), eng->sfx_atoms.as<uint8_t>(), st, true));
        }
        *launches += 1;
    } else if (job.fp4) {
        if (!per_token) {
            set_err(err, "the fast mode runs the single-device layer only");
            return 0;
        }
        CK(launch_scatter_quant_fp4(job.src, H, Kq, job.T, job.K, eng->pos_of.as<uint32_t>(),
                                    job.shared_rows ? gi.offset + job.E : nullptr, eng->row_info.as<uint32_t>(), P,
                                    eng->xb.as<uint8_t>(), eng->sfx_atoms.as<uint8_t>(), st, true));
    } else if (job.K > 1 && per_token) {
        // each token row feeds K (+1 shared) permuted rows: split it once
        CK(launch_scatter_quant_bs(job.src, H, Kq, job.T, job.K, eng->pos_of.as<uint32_t>(),
                                   job.shared_rows ? gi.offset + job.E : nullptr, eng->row_info.as<uint32_t>(), P,
                                   (uint32_t)xb_rows, block_n, eng->xb.as<uint8_t>(), eng->sfx_atoms.as<uint8_t>(),
                                   st, true));
    } else {
        CK(launch_gather_quant_bs(job.src, H, Kq, eng->row_token.as<uint32_t>(), eng->row_info.as<uint32_t>(), P,
                                  (uint32_t)xb_rows, block_n, eng->xb.as<uint8_t>(), eng->sfx_atoms.as<uint8_t>(),
                                  st, true));
    }
    *launches += 1;
    mark(3);
    BsParams bp{};
    bp.groups = G;
    bp.count = gi.count;
    bp.offset = gi.offset;
    bp.err = errw;
    bp.act = job.act;
    bp.group_slot = job.group_slot;
    // gate/up: K = H (padded Kq), M = I rows (padded rp_i), output h hi/lo
    bp.tile_off = gi.gu_tile_off;
    bp.tiles = eng->gu_tiles.as<TileEntry>();
    bp.rows_pad = L->rp_i;
    bp.m_tiles = L->rp_i / 128;
    bp.k_tiles = Kq / 128;
    bp.sfa = L->bs_gu_sfa.as<uint8_t>();
    bp.a_codes = L->bs_gu_codes.as<uint8_t>();
    bp.sfb_atoms = eng->sfx_atoms.as<uint8_t>();
    bp.h_out = eng->hb.as<uint8_t>();
    bp.h_plane = hb_rows * Iq;
    bp.h_stride = job.fp4 ? Iq / 2 : Iq;
    bp.sfh_atoms = eng->sfh_atoms.as<uint8_t>();
    bp.m_valid = Iq;
    const int bi = block_n == 32 ? 0 : (block_n == 64 ? 1 : 2);
    // a pair's CTAs each load half of the tile's token rows (the 64-row box)
    CK(launch_gemm_bs(kGateUp, (int)block_n, job.fp4 ? L->tmap_gu_fp4 : L->tmap_gu_codes,
                      job.fp4 ? eng->tmap_xq[bi] : eng->tmap_xb[pair_gu ? 1 : bi], bp, eng->num_sms, st, true,
                      job.fp4, pair_gu));
    *launches += 1;
    mark(4);
    // down: K = I (padded Iq), M = H rows (padded rp_h), output fp32 rows
    bp.tile_off = gi.dn_tile_off;
    bp.tiles = eng->dn_tiles.as<TileEntry>();
    bp.rows_pad = L->rp_h;
    bp.m_tiles = L->rp_h / 128;
    bp.k_tiles = Iq / 128;
    bp.sfa = L->bs_dn_sfa.as<uint8_t>();
    bp.a_codes = L->bs_dn_codes.as<uint8_t>();
    bp.sfb_atoms = eng->sfh_atoms.as<uint8_t>();
    bp.y_out = job.y;
    bp.y_stride = H;
    bp.m_valid = H;
    bp.y_row_map = job.y_by_source ? eng->row_token.as<uint32_t>() : nullptr;
    bp.ret_ptrs = job.ret_ptrs;
    bp.ret_roff = job.ret_roff;
    bp.ret_base = job.ret_base;
    bp.ret_rows = job.ret_rows;
    bp.ret_world = job.ret_world;
    CK(launch_gemm_bs(kDown, (int)block_n, job.fp4 ? L->tmap_dn_fp4 : L->tmap_dn_codes,
                      job.fp4 ? eng->tmap_hq[bi] : eng->tmap_hb[pair_dn ? 1 : bi], bp, eng->num_sms, st, true,
                      job.fp4, pair_dn));
    *launches += 1;
    mark(5);
    return 1;
}

}  // namespace

extern "C" {

moe_b200_engine_t* moe_b200_create(const moe_b200_init_t* init, char* err) {
    const int device = init ? init->device : 0;
    const uint32_t layers = (init && init->max_layers) ? init->max_layers : 1;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
        set_err(err, "CUDA device %d not available (%d devices)", device, count);
        return nullptr;
    }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
        set_err(err, "cudaGetDeviceProperties failed");
        return nullptr;
    }
    if (prop.major != 10) {
        set_err(err, "device %d is sm_%d%d; this library is built for sm_100a (B200)", device, prop.major,
                prop.minor);
        return nullptr;
    }
    if (cudaSetDevice(device) != cudaSuccess) {
        set_err(err, "cudaSetDevice(%d) failed", device);
        return nullptr;
    }
    auto* eng = new (std::nothrow) moe_b200_engine();
    if (!eng) {
        set_err(err, "out of host memory");
        return nullptr;
    }
    eng->device = device;
    eng->num_sms = prop.multiProcessorCount;
    {
        const char* v = std::getenv("MOE_B200_CTA_PAIRS");
        eng->cta_pairs = !(v && v[0] == '0');
    }
    eng->layers.resize(layers);
    if (eng->err_word.reserve(sizeof(uint32_t)) != cudaSuccess ||
        cudaMemset(eng->err_word.ptr, 0, sizeof(uint32_t)) != cudaSuccess ||
        cudaStreamCreateWithFlags(&eng->hstream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreate(&eng->ustream) != cudaSuccess ||
        cudaMallocHost(&eng->h_err, sizeof(uint32_t)) != cudaSuccess) {
        set_err(err, "device allocation failed");
        if (eng->hstream) cudaStreamDestroy(eng->hstream);
        if (eng->ustream) cudaStreamDestroy(eng->ustream);
        eng->err_word.release();
        delete eng;
        return nullptr;
    }
    *eng->h_err = 0;
    return eng;
}

void moe_b200_destroy(moe_b200_engine_t* eng) {
    if (!eng) return;
    cudaSetDevice(eng->device);
    cudaDeviceSynchronize();
    for (auto& l : eng->layers) l.release_all();
    DevBuf* bufs[] = {&eng->staging, &eng->logits, &eng->scores, &eng->ids, &eng->wts, &eng->tile_counts,
                      &eng->rank, &eng->pos_of, &eng->row_token, &eng->row_assign, &eng->row_info, &eng->g_count,
                      &eng->g_offset, &eng->g_gu_off, &eng->g_dn_off, &eng->xperm, &eng->hperm,
                      &eng->yperm, &eng->err_word, &eng->hx, &eng->hy, &eng->hyf, &eng->hids,
                      &eng->hw, &eng->hperm_out, &eng->tri, &eng->xb,
                      &eng->sfx_atoms, &eng->hb, &eng->sfh_atoms, &eng->gu_tiles, &eng->dn_tiles,
                      &eng->pipe_ys, &eng->pipe_zero_ids, &eng->pipe_slot, &eng->present_dev, &eng->comb_w};
    for (DevBuf* b : bufs) b->release();
    for (cudaEvent_t e : eng->prof_events) cudaEventDestroy(e);
    ep_release(eng->ep);
    if (eng->hstream) cudaStreamDestroy(eng->hstream);
    if (eng->ustream) cudaStreamDestroy(eng->ustream);
    if (eng->pipe_in) cudaStreamDestroy(eng->pipe_in);
    if (eng->pipe_out) cudaStreamDestroy(eng->pipe_out);
    for (cudaEvent_t e : eng->pipe_ev) cudaEventDestroy(e);
    if (eng->h_err) cudaFreeHost(eng->h_err);
    delete eng;
}

int moe_b200_upload_router(moe_b200_engine_t* eng, int32_t layer, const uint16_t* w, uint32_t experts,
                           uint32_t hidden, int32_t src_on_device, char* err) {
    LayerWeights* L = get_layer(eng, layer, err);
    if (!L) return 0;
    if (!w || experts == 0 || experts > 1024 || hidden == 0 || hidden % 8) {
        set_err(err, "invalid router upload (experts=%u hidden=%u)", experts, hidden);
        return 0;
    }
    CK(cudaSetDevice(eng->device));
    if (L->E && (L->E != experts || L->H != hidden)) {
        // a new shape invalidates the layer's experts
        DevBuf keep;
        std::swap(keep, L->router);
        L->release_all();
        std::swap(keep, L->router);
        L->present.clear();
        L->I = 0;
    }
    const size_t bytes = (size_t)experts * hidden * 2;
    CK(L->router.reserve(bytes));
    CK(cudaMemcpy(L->router.ptr, w, bytes, src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice));
    L->E = experts;
    L->H = hidden;
    return 1;
}

int moe_b200_upload_expert(moe_b200_engine_t* eng, int32_t layer, int32_t expert, const uint8_t* gate,
                           uint64_t gate_bytes, const uint8_t* up, uint64_t up_bytes, const uint8_t* down,
                           uint64_t down_bytes, uint32_t hidden, uint32_t intermediate, int32_t src_on_device,
                           char* err) {
    LayerWeights* L = get_layer(eng, layer, err);
    if (!L) return 0;
    if (!L->E) {
        set_err(err, "upload the router of layer %d before its experts", layer);
        return 0;
    }
    if (hidden != L->H || intermediate == 0 || intermediate > 100000) {
        set_err(err, "expert shape H=%u I=%u does not match layer H=%u", hidden, intermediate, L->H);
        return 0;
    }
    if (expert < -1 || expert >= (int32_t)L->E) {
        set_err(err, "expert %d outside -1..%u", expert, L->E - 1);
        return 0;
    }
    const uint64_t gu_need = (uint64_t)intermediate * ceil_div(hidden, 32) * 17;
    const uint64_t dn_need = (uint64_t)hidden * ceil_div(intermediate, 32) * 17;
    if (!gate || !up || !down || gate_bytes < gu_need || up_bytes < gu_need || down_bytes < dn_need) {
        set_err(err, "expert %d: MXFP4 byte counts %llu/%llu/%llu below %llu/%llu/%llu", expert,
                (unsigned long long)gate_bytes, (unsigned long long)up_bytes, (unsigned long long)down_bytes,
                (unsigned long long)gu_need, (unsigned long long)gu_need, (unsigned long long)dn_need);
        return 0;
    }
    CK(cudaSetDevice(eng->device));
    if (!ensure_bs_layout(eng, L, intermediate, err)) return 0;
    const uint32_t slot = expert < 0 ? L->E : (uint32_t)expert;
    const uint8_t* src[3] = {gate, up, down};
    const uint64_t need[3] = {gu_need, gu_need, dn_need};
    const uint8_t* dsrc[3] = {gate, up, down};
    cudaStream_t st = eng->ustream;
    if (!src_on_device) {
        CK(eng->staging.reserve(2 * gu_need + dn_need));
        uint8_t* stg = eng->staging.as<uint8_t>();
        uint64_t off = 0;
        for (int i = 0; i < 3; ++i) {
            CK(cudaMemcpyAsync(stg + off, src[i], need[i], cudaMemcpyHostToDevice, st));
            dsrc[i] = stg + off;
            off += need[i];
        }
    }
    {
        const uint64_t mti = L->rp_i / 128, kth = L->kq / 128, mth = L->rp_h / 128, kti = L->iq / 128;
        for (int pj = 0; pj < 2; ++pj) {
            const uint64_t m = (uint64_t)slot * 2 + pj;
            // scale blocks [slot][mt][kt][gate | up]: one bulk copy per stage brings both
            CK(launch_repack_bs(dsrc[pj], intermediate, hidden, L->rp_i, L->kq,
                                L->bs_gu_codes.as<uint8_t>() + m * L->rp_i * (L->kq / 2),
                                L->bs_gu_sfa.as<uint8_t>() + (uint64_t)slot * mti * kth * 1024 + pj * 512, 1024,
                                st));
        }
        CK(launch_repack_bs(dsrc[2], hidden, intermediate, L->rp_h, L->iq,
                            L->bs_dn_codes.as<uint8_t>() + (uint64_t)slot * L->rp_h * (L->iq / 2),
                            L->bs_dn_sfa.as<uint8_t>() + (uint64_t)slot * mth * kti * 512, 512, st));
    }
    // the caller may reuse its buffers (and the next upload the staging
    // buffer) once this returns: wait for this upload only, not the device
    CK(cudaStreamSynchronize(st));
    L->present[slot] = 1;
    L->tile_ready[slot] = 0;
    return 1;
}

uint64_t moe_b200_expert_record_bytes(uint32_t hidden, uint32_t intermediate) {
    if (hidden == 0 || intermediate == 0 || intermediate > 100000 || hidden > 100000) return 0;
    const uint64_t rp_i = round_up(intermediate, 128), rp_h = round_up(hidden, 128);
    const uint64_t kq = rp_h, iq = rp_i;
    return 2 * rp_i * (kq / 2) + 2 * (rp_i / 128) * (kq / 128) * 512 + rp_h * (iq / 2) + (rp_h / 128) * (iq / 128) * 512;
}

int moe_b200_export_expert(moe_b200_engine_t* eng, int32_t layer, int32_t expert, uint8_t* dst, uint64_t dst_bytes,
                           int32_t dst_on_device, char* err) {
    LayerWeights* L = get_layer(eng, layer, err);
    if (!L) return 0;
    if (!L->E || !L->I || expert < -1 || expert >= (int32_t)L->E) {
        set_err(err, "layer %d has no expert %d", layer, expert);
        return 0;
    }
    const uint32_t slot = expert < 0 ? L->E : (uint32_t)expert;
    if (slot >= L->present.size() || !L->present[slot]) {
        set_err(err, "expert %d of layer %d is not resident", expert, layer);
        return 0;
    }
    const uint64_t need = moe_b200_expert_record_bytes(L->H, L->I);
    if (!dst || dst_bytes < need) {
        set_err(err, "expert record needs %llu bytes, got %llu", (unsigned long long)need,
                (unsigned long long)dst_bytes);
        return 0;
    }
    CK(cudaSetDevice(eng->device));
    RecordPart parts[4];
    record_parts(L, slot, parts);
    uint64_t off = 0;
    for (const RecordPart& r : parts) {
        CK(cudaMemcpyAsync(dst + off, r.dev, r.bytes, dst_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost,
                           eng->ustream));
        off += r.bytes;
    }
    CK(cudaStreamSynchronize(eng->ustream));
    return 1;
}

int moe_b200_import_expert(moe_b200_engine_t* eng, int32_t layer, int32_t expert, const uint8_t* src,
                           uint64_t src_bytes, uint32_t hidden, uint32_t intermediate, int32_t src_on_device,
                           char* err) {
    LayerWeights* L = get_layer(eng, layer, err);
    if (!L) return 0;
    if (!L->E) {
        set_err(err, "upload the router of layer %d before its experts", layer);
        return 0;
    }
    if (hidden != L->H || intermediate == 0 || intermediate > 100000) {
        set_err(err, "expert shape H=%u I=%u does not match layer H=%u", hidden, intermediate, L->H);
        return 0;
    }
    if (expert < -1 || expert >= (int32_t)L->E) {
        set_err(err, "expert %d outside -1..%u", expert, L->E - 1);
        return 0;
    }
    const uint64_t need = moe_b200_expert_record_bytes(hidden, intermediate);
    if (!src || src_bytes != need) {
        set_err(err, "expert record of H=%u I=%u is %llu bytes, got %llu", hidden, intermediate,
                (unsigned long long)need, (unsigned long long)src_bytes);
        return 0;
    }
    CK(cudaSetDevice(eng->device));
    if (!ensure_bs_layout(eng, L, intermediate, err)) return 0;
    const uint32_t slot = expert < 0 ? L->E : (uint32_t)expert;
    RecordPart parts[4];
    record_parts(L, slot, parts);
    uint64_t off = 0;
    for (const RecordPart& r : parts) {
        CK(cudaMemcpyAsync(r.dev, src + off, r.bytes, src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                           eng->ustream));
        off += r.bytes;
    }
    // the caller may reuse its buffer once this returns
    CK(cudaStreamSynchronize(eng->ustream));
    L->present[slot] = 1;
    L->tile_ready[slot] = 0;
    return 1;
}

}  // extern "C"

namespace {

// Host-buffer calls on large batches overlap the copies with the per-token
// stages: x arrives in token chunks (pipe_in), the router and the shared
// expert run on each chunk as it lands, and the combine runs chunk by chunk
// with each chunk's rows, ids and weights copied back (pipe_out) while the
// next is combined.  Every token's result comes from the same kernels as
// without the chunks; where both calls pick the same GEMM tile widths (every
// batch averaging more than 160 rows per expert) the bytes are the same.
constexpr uint32_t kPipeChunks = 8;
constexpr uint32_t kPipeMinTokens = 4096;

struct HostPipe {
    const uint16_t* x;  // host rows of the batch
    uint16_t* y_bf16;   // host outputs (null: not wanted)
    float* y_f32;
    int32_t* ids;
    float* w;
};

// Token range of chunk c.
inline void pipe_range(uint32_t T, uint32_t c, uint32_t* t0, uint32_t* t1) {
    const uint32_t tc = ceil_div(T, kPipeChunks);
    *t0 = std::min(T, c * tc);
    *t1 = std::min(T, *t0 + tc);
}

// The single-device layer (moe_b200_layer_forward and moe_b200_block_forward):
// `hidden` is the residual stream the block parts may read (may be null).
// `pipe`: the call's host buffers (moe_b200_layer_forward_host), x then being
// the device buffer the chunks are copied into.
int forward_impl(moe_b200_engine_t* eng, const moe_b200_layer_cfg_t* cfg, const uint16_t* x, const float* hidden,
                 uint32_t T, uint16_t* y_bf16, float* y_f32, int32_t* topk_ids, float* topk_w, uint32_t* perm,
                 void* stream, char* err, const HostPipe* pipe = nullptr) {
    if (!check_dims(cfg, err)) return 0;
    LayerWeights* L = get_layer(eng, cfg->layer, err);
    if (!L) return 0;
    const uint32_t H = cfg->hidden, I = cfg->intermediate, E = cfg->experts, K = cfg->top_k;
    if (L->E != E || L->H != H || L->I != I) {
        set_err(err, "layer %d holds E=%u H=%u I=%u, config asks E=%u H=%u I=%u", cfg->layer, L->E, L->H, L->I, E,
                H, I);
        return 0;
    }
    if (L->present.size() != (size_t)E + 1) {
        set_err(err, "layer %d has no experts uploaded", cfg->layer);
        return 0;
    }
    const bool skip_missing = cfg->skip_missing != 0;
    for (uint32_t e = 0; e < E && !skip_missing; ++e) {
        if (!L->present[e]) {
            set_err(err, "expert %u of layer %d was never uploaded", e, cfg->layer);
            return 0;
        }
    }
    const bool shared = cfg->use_shared != 0;
    if (shared && !L->present[E] && !skip_missing) {
        set_err(err, "layer %d has no shared expert uploaded", cfg->layer);
        return 0;
    }
    const bool fp4 = cfg->gemm_path == MOE_B200_GEMM_MXF4_FAST;
    const bool bs = cfg->gemm_path == MOE_B200_GEMM_BLOCKSCALED || fp4;
    const bool block = L->has_block() || cfg->activation != MOE_B200_ACT_SILU;
    if (cfg->activation < MOE_B200_ACT_SILU || cfg->activation > MOE_B200_ACT_GELU_TANH) {
        set_err(err, "unknown activation %d", cfg->activation);
        return 0;
    }
    if (block && !bs) {
        set_err(err, "block parts and GELU activations run on the block-scaled GEMM paths (gemm_path 0 or 3)");
        return 0;
    }
    if (skip_missing && !bs) {
        set_err(err, "skip_missing runs on the block-scaled GEMM paths (gemm_path 0 or 3)");
        return 0;
    }
    if (L->has_block() && H > 25600) {
        set_err(err, "block parts support H <= 25600 (H=%u)", H);
        return 0;
    }
    if (T == 0) return 1;
    if (!x) {
        set_err(err, "null input");
        return 0;
    }
    if (L->needs_hidden() && !hidden) {
        set_err(err, "layer %d has a pre-norm or router input scale: give the residual stream "
                     "(moe_b200_block_forward)", cfg->layer);
        return 0;
    }
    if ((uint64_t)T * K > 0x7fffffffull) {
        set_err(err, "tokens x top_k too large");
        return 0;
    }
    CK(cudaSetDevice(eng->device));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const uint32_t n = T * K;
    const uint32_t shared_rows = shared ? T : 0;
    const uint32_t P = n + shared_rows;
    const uint32_t G = E + (shared ? 1 : 0);
    const uint32_t Kp = round_up(H, kTileK), Ip = round_up(I, kTileK);
    const uint32_t rows_cap = std::max(P, 32u);
    const uint32_t ntiles = sort_tiles(n);

    CK(eng->logits.reserve((size_t)T * E * 4));
    CK(eng->scores.reserve((size_t)T * E * 4));
    CK(eng->ids.reserve((size_t)n * 4));
    CK(eng->wts.reserve((size_t)n * 4));
    CK(eng->tile_counts.reserve((size_t)std::max(ntiles, 1u) * E * 4));
    CK(eng->rank.reserve((size_t)n * 4));
    CK(eng->pos_of.reserve((size_t)n * 4));
    CK(eng->row_token.reserve((size_t)P * 4));
    CK(eng->row_assign.reserve((size_t)P * 4));
    CK(eng->g_count.reserve((size_t)(G + 1) * 4));
    CK(eng->g_offset.reserve((size_t)(G + 1) * 4));
    CK(eng->g_gu_off.reserve((size_t)(G + 1) * 4));
    CK(eng->g_dn_off.reserve((size_t)(G + 1) * 4));
    CK(eng->yperm.reserve((size_t)P * H * 4));
    if (!bs) {
        // the cross-check GEMMs read the tile form
        for (uint32_t e = 0; e < E; ++e) {
            if (!ensure_tile_form(eng, L, e, err)) return 0;
        }
        if (shared && !ensure_tile_form(eng, L, E, err)) return 0;
        CK(eng->xperm.reserve((size_t)rows_cap * Kp * 2));
        CK(eng->hperm.reserve((size_t)rows_cap * Ip * 2));
        // tensor maps over the permuted activations and the intermediate
        const uint64_t xrows = eng->xperm.bytes / ((uint64_t)Kp * 2), hrows = eng->hperm.bytes / ((uint64_t)Ip * 2);
        if (eng->tmap_x_base != eng->xperm.ptr || eng->tmap_x_dims[0] != Kp || eng->tmap_x_dims[1] != xrows) {
            if (!make_tmap(eng, &eng->tmap_x, eng->xperm.ptr, Kp, xrows, err)) return 0;
            eng->tmap_x_base = eng->xperm.ptr;
            eng->tmap_x_dims[0] = Kp;
            eng->tmap_x_dims[1] = xrows;
        }
        if (eng->tmap_h_base != eng->hperm.ptr || eng->tmap_h_dims[0] != Ip || eng->tmap_h_dims[1] != hrows) {
            if (!make_tmap(eng, &eng->tmap_h, eng->hperm.ptr, Ip, hrows, err)) return 0;
            eng->tmap_h_base = eng->hperm.ptr;
            eng->tmap_h_dims[0] = Ip;
            eng->tmap_h_dims[1] = hrows;
        }
    }

    cudaEvent_t* ev = nullptr;
    if (eng->prof_max && eng->prof_calls < eng->prof_max) {
        ev = &eng->prof_events[(size_t)eng->prof_calls * (MOE_B200_STAGES + 1)];
        ++eng->prof_calls;
    }
    auto mark = [&](int i) {
        if (ev) cudaEventRecord(ev[i], st);
    };
    mark(0);
    int32_t* ids = topk_ids ? topk_ids : eng->ids.as<int32_t>();
    float* w = topk_w ? topk_w : eng->wts.as<float>();
    uint32_t* errw = eng->err_word.as<uint32_t>();
    uint32_t launches = 0;

    const int sigmoid = cfg->score_func == MOE_B200_SCORE_SIGMOID;
    const float rscale = cfg->routed_scale > 0.f ? cfg->routed_scale : 1.0f;
    const RouteCfg rcfg{sigmoid, cfg->norm_topk, rscale, cfg->n_group, cfg->topk_group};
    // host-buffer calls: the shared expert needs no routing, so its pipeline
    // runs on each token chunk right after the chunk lands, under the copies
    // of the chunks after it; the routed pass then leaves it out
    const bool pipe_shared = pipe && shared && bs;
    if (pipe_shared) {
        CK(eng->pipe_ys.reserve((size_t)T * H * 4));
        if (eng->pipe_zero_ids.bytes < (size_t)T * 4) {
            CK(eng->pipe_zero_ids.reserve((size_t)T * 4));
            CK(cudaMemsetAsync(eng->pipe_zero_ids.ptr, 0, eng->pipe_zero_ids.bytes, st));
        }
        CK(eng->pipe_slot.reserve(4));
        CK(cudaMemcpyAsync(eng->pipe_slot.ptr, &L->E, 4, cudaMemcpyHostToDevice, st));
    }
    // block parts: the routed input RMSNorm(hidden) * pre_norm2, exactly as
    // the reference computes it (fp32 for the router, bf16 for the experts)
    const uint16_t* x_routed = x;
    if (L->blk_pre_norm2.ptr) {
        CK(eng->xr_f32.reserve((size_t)T * H * 4));
        CK(eng->xr_bf16.reserve((size_t)T * H * 2));
        CK(launch_row_norm_exact(hidden, T, H, L->blk_pre_norm2.as<float>(), H, 0, cfg->norm_eps,
                                 cfg->norm_unit_offset, eng->xr_f32.as<float>(), eng->xr_bf16.as<uint16_t>(), st));
        x_routed = eng->xr_bf16.as<uint16_t>();
        launches += 1;
    }
    if (L->blk_router_scale.ptr || L->blk_pre_norm2.ptr) {
        // the router reads an fp32 row: the scaled residual stream, or the
        // pre-normed routed input
        const float* rin = eng->xr_f32.as<float>();
        if (L->blk_router_scale.ptr) {
            CK(eng->rin_f32.reserve((size_t)T * H * 4));
            CK(launch_row_norm_exact(hidden, T, H, L->blk_router_scale.as<float>(), L->blk_router_scale_count, 1, 0.f,
                                     0, eng->rin_f32.as<float>(), nullptr, st));
            rin = eng->rin_f32.as<float>();
            launches += 1;
        }
        CK(launch_router_f32(rin, L->router.as<uint16_t>(), T, E, H, K, rcfg, eng->logits.as<float>(), ids, w,
                             eng->scores.as<float>(), st, &launches));
    } else if (pipe) {
        for (uint32_t c = 0; c < kPipeChunks; ++c) {
            uint32_t t0, t1;
            pipe_range(T, c, &t0, &t1);
            if (t0 == t1) continue;
            uint16_t* xc = const_cast<uint16_t*>(x) + (size_t)t0 * H;
            CK(cudaMemcpyAsync(xc, pipe->x + (size_t)t0 * H, (size_t)(t1 - t0) * H * 2, cudaMemcpyHostToDevice,
                               eng->pipe_in));
            CK(cudaEventRecord(eng->pipe_ev[c], eng->pipe_in));
            CK(cudaStreamWaitEvent(st, eng->pipe_ev[c], 0));
            CUtensorMap rtx, rtw;
            const bool rt_tma = router_tmaps(eng, xc, L->router.as<uint16_t>(), t1 - t0, E, H, &rtx, &rtw);
            CK(launch_router(xc, L->router.as<uint16_t>(), t1 - t0, E, H, K, rcfg,
                             eng->logits.as<float>() + (size_t)t0 * E, ids + (size_t)t0 * K, w + (size_t)t0 * K,
                             eng->scores.as<float>() + (size_t)t0 * E, errw, st, &launches, rt_tma ? &rtx : nullptr,
                             rt_tma ? &rtw : nullptr));
            if (pipe_shared) {
                // the shared expert on this chunk: one group, its own output rows
                BsJob sj{};
                sj.ids = eng->pipe_zero_ids.as<int32_t>();
                sj.T = t1 - t0;
                sj.K = 1;
                sj.E = 1;
                sj.shared_rows = 0;
                sj.shared_base = 0;
                sj.src = xc;
                sj.act = cfg->activation;
                sj.group_slot = eng->pipe_slot.as<uint32_t>();
                sj.y = eng->pipe_ys.as<float>() + (size_t)t0 * H;
                sj.y_by_source = true;
                sj.fp4 = fp4;
                if (!run_blockscaled(eng, L, sj, st, nullptr, &launches, err)) return 0;
            }
        }
    } else {
        CUtensorMap rtx, rtw;
        const bool rt_tma = router_tmaps(eng, x, L->router.as<uint16_t>(), T, E, H, &rtx, &rtw);
        CK(launch_router(x, L->router.as<uint16_t>(), T, E, H, K, rcfg, eng->logits.as<float>(), ids, w,
                         eng->scores.as<float>(), errw, st, &launches, rt_tma ? &rtx : nullptr,
                         rt_tma ? &rtw : nullptr));
    }
    // the shared-expert gate sigmoid(gate_inp . x): the router's exact dot and
    // sigmoid with one expert
    const bool gated = shared && L->blk_gate_inp.ptr;
    if (gated) {
        CK(eng->gate_logits.reserve((size_t)T * 4));
        CK(eng->gate_ids.reserve((size_t)T * 4));
        CK(eng->gate_w.reserve((size_t)T * 4));
        CK(eng->gate_scores.reserve((size_t)T * 4));
        CK(launch_router(x, L->blk_gate_inp.as<uint16_t>(), T, 1, H, 1, RouteCfg{1, 0, 1.0f, 0, 0},
                         eng->gate_logits.as<float>(), eng->gate_ids.as<int32_t>(), eng->gate_w.as<float>(),
                         eng->gate_scores.as<float>(), errw, st, &launches, nullptr, nullptr));
    }
    mark(1);

    if (bs) {
        BsJob job{};
        job.ids = ids;
        job.T = T;
        job.K = K;
        job.E = E;
        job.shared_rows = pipe_shared ? 0 : shared_rows;
        job.shared_base = 0;
        job.src = x_routed;
        job.src_shared = (x_routed != x && shared_rows) ? x : nullptr;
        job.act = cfg->activation;
        job.group_slot = nullptr;
        job.y = eng->yperm.as<float>();
        job.y_by_source = false;
        job.fp4 = fp4;
        if (!run_blockscaled(eng, L, job, st, ev, &launches, err)) return 0;
    } else {
    GroupInfo gi;
    gi.count = eng->g_count.as<uint32_t>();
    gi.offset = eng->g_offset.as<uint32_t>();
    gi.gu_tile_off = eng->g_gu_off.as<uint32_t>();
    gi.dn_tile_off = eng->g_dn_off.as<uint32_t>();
    gi.block_n = kBlockN;
    gi.gu_row_tiles = ceil_div(I, kTileRows);
    gi.dn_row_tiles = ceil_div(H, kTileRows);
    CK(launch_permute(ids, T, K, E, shared_rows, 0, eng->tile_counts.as<uint32_t>(), eng->rank.as<uint32_t>(), gi,
                      eng->pos_of.as<uint32_t>(), eng->row_token.as<uint32_t>(), eng->row_assign.as<uint32_t>(),
                      nullptr, errw, st));
    launches += 3;
    mark(2);
    CK(launch_gather(x, H, Kp, eng->row_token.as<uint32_t>(), P, eng->xperm.as<uint16_t>(), st));
    launches += 1;
    mark(3);

    GemmParams gp{};
    gp.groups = G;
    gp.count = gi.count;
    gp.offset = gi.offset;
    gp.err = errw;
    // gate/up: K = H, output columns = Ip
    gp.wt = L->gu.as<uint8_t>();
    gp.group_stride = L->gu_stride;
    gp.k_tiles = Kp / kTileK;
    gp.m_valid = Ip;
    gp.tile_off = gi.gu_tile_off;
    gp.h_out = eng->hperm.as<uint16_t>();
    gp.h_stride = Ip;
    if (cfg->gemm_path == MOE_B200_GEMM_SIMT) {
        CK(launch_gemm_simt(kGateUp, eng->xperm.as<uint16_t>(), Kp, P, gp, Ip, st));
    } else {
        CK(launch_gemm_tc(kGateUp, eng->tmap_x, gp, eng->num_sms, st));
    }
    launches += 1;
    mark(4);
    // down: K = Ip, output columns = H
    gp.wt = L->dn.as<uint8_t>();
    gp.group_stride = L->dn_stride;
    gp.k_tiles = Ip / kTileK;
    gp.m_valid = H;
    gp.tile_off = gi.dn_tile_off;
    gp.y_out = eng->yperm.as<float>();
    gp.y_stride = H;
    if (cfg->gemm_path == MOE_B200_GEMM_SIMT) {
        CK(launch_gemm_simt(kDown, eng->hperm.as<uint16_t>(), Ip, P, gp, H, st));
    } else {
        CK(launch_gemm_tc(kDown, eng->tmap_h, gp, eng->num_sms, st));
    }
    launches += 1;
    mark(5);
    }

    // missing experts (skip_missing): the combine weights of the reference's
    // partial-failure policy -- 0 for a missing expert (whose zero codes add
    // nothing anyway), the others renormalised when the router renormalises
    // its top-k -- and an error for a token whose experts are all missing
    const float* cw = w;
    if (skip_missing &&
        std::find(L->present.begin(), L->present.begin() + E, (uint8_t)0) != L->present.begin() + E) {
        CK(eng->present_dev.reserve(E));
        CK(cudaMemcpyAsync(eng->present_dev.ptr, L->present.data(), E, cudaMemcpyHostToDevice, st));
        CK(eng->comb_w.reserve((size_t)T * K * 4));
        CK(launch_combine_weights(ids, w, eng->present_dev.as<uint8_t>(), T, K, E, cfg->norm_topk != 0,
                                  eng->comb_w.as<float>(), errw, st));
        launches += 1;
        cw = eng->comb_w.as<float>();
    }
    // tokens [t0, t1): the combine, then (host-buffer calls) their copy back
    auto combine = [&](uint32_t t0, uint32_t t1) -> int {
        const float* ys = !shared      ? nullptr
                          : pipe_shared ? eng->pipe_ys.as<float>() + (size_t)t0 * H
                                        : eng->yperm.as<float>() + (size_t)(n + t0) * H;
        uint16_t* yb = y_bf16 ? y_bf16 + (size_t)t0 * H : nullptr;
        float* yf = y_f32 ? y_f32 + (size_t)t0 * H : nullptr;
        if (L->has_block_combine()) {
            BlockParts parts{L->blk_post_norm1.as<float>(), L->blk_post_norm2.as<float>(),
                             L->blk_post_norm.as<float>(), L->blk_down_scale.as<float>(), L->blk_down_scale_count,
                             cfg->norm_eps, cfg->norm_unit_offset};
            CK(launch_block_combine(eng->yperm.as<float>(), H, eng->pos_of.as<uint32_t>() + (size_t)t0 * K,
                                    ids + (size_t)t0 * K, cw + (size_t)t0 * K, t1 - t0, K, E, ys,
                                    gated ? eng->gate_w.as<float>() + t0 : nullptr, parts, yb, yf, st, bs));
        } else {
            CK(launch_combine(eng->yperm.as<float>(), H, eng->pos_of.as<uint32_t>() + (size_t)t0 * K,
                              cw + (size_t)t0 * K, t1 - t0, K, ys, yb, yf, st, bs));
        }
        launches += 1;
        return 1;
    };
    if (pipe) {
        for (uint32_t c = 0; c < kPipeChunks; ++c) {
            uint32_t t0, t1;
            pipe_range(T, c, &t0, &t1);
            if (t0 == t1) continue;
            if (!combine(t0, t1)) return 0;
            cudaEvent_t e = eng->pipe_ev[kPipeChunks + c];
            CK(cudaEventRecord(e, st));
            CK(cudaStreamWaitEvent(eng->pipe_out, e, 0));
            const size_t rows = t1 - t0;
            if (pipe->y_bf16) {
                CK(cudaMemcpyAsync(pipe->y_bf16 + (size_t)t0 * H, y_bf16 + (size_t)t0 * H, rows * H * 2,
                                   cudaMemcpyDeviceToHost, eng->pipe_out));
            }
            if (pipe->y_f32) {
                CK(cudaMemcpyAsync(pipe->y_f32 + (size_t)t0 * H, y_f32 + (size_t)t0 * H, rows * H * 4,
                                   cudaMemcpyDeviceToHost, eng->pipe_out));
            }
            if (pipe->ids) {
                CK(cudaMemcpyAsync(pipe->ids + (size_t)t0 * K, ids + (size_t)t0 * K, rows * K * 4,
                                   cudaMemcpyDeviceToHost, eng->pipe_out));
            }
            if (pipe->w) {
                CK(cudaMemcpyAsync(pipe->w + (size_t)t0 * K, w + (size_t)t0 * K, rows * K * 4,
                                   cudaMemcpyDeviceToHost, eng->pipe_out));
            }
        }
    } else if (!combine(0, T)) {
        return 0;
    }
    mark(6);
    if (perm) {
        CK(cudaMemcpyAsync(perm, eng->row_assign.ptr, (size_t)n * 4, cudaMemcpyDeviceToDevice, st));
    }
    eng->last_T = T;
    eng->last_E = E;
    eng->last_G = G;
    eng->last_P = P;
    eng->last_Kp = Kp;
    eng->last_Ip = Ip;
    eng->last_H = H;
    eng->last_launches = launches;
    return 1;
}

}  // namespace

extern "C" {

int moe_b200_layer_forward(moe_b200_engine_t* eng, const moe_b200_layer_cfg_t* cfg, const uint16_t* x,
                           uint32_t T, uint16_t* y_bf16, float* y_f32, int32_t* topk_ids, float* topk_w,
                           uint32_t* perm, void* stream, char* err) {
    return forward_impl(eng, cfg, x, nullptr, T, y_bf16, y_f32, topk_ids, topk_w, perm, stream, err);
}

int moe_b200_block_forward(moe_b200_engine_t* eng, const moe_b200_layer_cfg_t* cfg, const uint16_t* x,
                           const float* hidden, uint32_t T, uint16_t* y_bf16, float* y_f32, int32_t* topk_ids,
                           float* topk_w, void* stream, char* err) {
    return forward_impl(eng, cfg, x, hidden, T, y_bf16, y_f32, topk_ids, topk_w, nullptr, stream, err);
}

int moe_b200_block_forward_host(moe_b200_engine_t* eng, const moe_b200_layer_cfg_t* cfg, const uint16_t* x,
                                const float* hidden, uint32_t T, uint16_t* y_bf16, float* y_f32, int32_t* topk_ids,
                                float* topk_w, char* err) {
    if (!check_dims(cfg, err)) return 0;
    if (!eng) {
        set_err(err, "null engine");
        return 0;
    }
    if (T == 0) return 1;
    if (!x) {
        set_err(err, "null input");
        return 0;
    }
    CK(cudaSetDevice(eng->device));
    const uint32_t H = cfg->hidden, K = cfg->top_k;
    CK(eng->hx.reserve((size_t)T * H * 2));
    CK(eng->hy.reserve((size_t)T * H * 2));
    CK(eng->hyf.reserve((size_t)T * H * 4));
    CK(eng->hids.reserve((size_t)T * K * 4));
    CK(eng->hw.reserve((size_t)T * K * 4));
    if (hidden) CK(eng->hhid.reserve((size_t)T * H * 4));
    cudaStream_t st = eng->hstream;
    CK(cudaMemcpyAsync(eng->hx.ptr, x, (size_t)T * H * 2, cudaMemcpyHostToDevice, st));
    if (hidden) CK(cudaMemcpyAsync(eng->hhid.ptr, hidden, (size_t)T * H * 4, cudaMemcpyHostToDevice, st));
    if (!forward_impl(eng, cfg, eng->hx.as<uint16_t>(), hidden ? eng->hhid.as<float>() : nullptr, T,
                      y_bf16 ? eng->hy.as<uint16_t>() : nullptr, y_f32 ? eng->hyf.as<float>() : nullptr,
                      eng->hids.as<int32_t>(), eng->hw.as<float>(), nullptr, st, err)) {
        return 0;
    }
    if (y_bf16) CK(cudaMemcpyAsync(y_bf16, eng->hy.ptr, (size_t)T * H * 2, cudaMemcpyDeviceToHost, st));
    if (y_f32) CK(cudaMemcpyAsync(y_f32, eng->hyf.ptr, (size_t)T * H * 4, cudaMemcpyDeviceToHost, st));
    if (topk_ids) CK(cudaMemcpyAsync(topk_ids, eng->hids.ptr, (size_t)T * K * 4, cudaMemcpyDeviceToHost, st));
    if (topk_w) CK(cudaMemcpyAsync(topk_w, eng->hw.ptr, (size_t)T * K * 4, cudaMemcpyDeviceToHost, st));
    return moe_b200_sync(eng, st, err);
}

int moe_b200_upload_block(moe_b200_engine_t* eng, int32_t layer, const moe_b200_block_tensors_t* t,
                          int32_t src_on_device, char* err) {
    LayerWeights* L = get_layer(eng, layer, err);
    if (!L) return 0;
    if (!L->E) {
        set_err(err, "upload the router of layer %d before its block tensors", layer);
        return 0;
    }
    CK(cudaSetDevice(eng->device));
    CK(cudaStreamSynchronize(eng->ustream));
    L->release_block();
    if (!t) return 1;
    const uint64_t H = L->H, E = L->E;
    if ((t->down_scale && t->down_scale_count == 0) || (t->router_scale && t->router_scale_count == 0)) {
        set_err(err, "a block scale tensor with zero values");
        return 0;
    }
    const cudaMemcpyKind kind = src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    auto put = [&](DevBuf& dst, const void* src, uint64_t bytes) -> int {
        if (!src) return 1;
        CK(dst.reserve(bytes));
        CK(cudaMemcpyAsync(dst.ptr, src, bytes, kind, eng->ustream));
        return 1;
    };
    (void)E;
    if (!put(L->blk_pre_norm2, t->pre_norm2, H * 4) || !put(L->blk_post_norm1, t->post_norm1, H * 4) ||
        !put(L->blk_post_norm2, t->post_norm2, H * 4) || !put(L->blk_post_norm, t->post_norm, H * 4) ||
        !put(L->blk_down_scale, t->down_scale, t->down_scale_count * 4) ||
        !put(L->blk_gate_inp, t->shared_gate_inp, H * 2) ||
        !put(L->blk_router_scale, t->router_scale, t->router_scale_count * 4)) {
        L->release_block();
        return 0;
    }
    L->blk_down_scale_count = t->down_scale ? t->down_scale_count : 0;
    L->blk_router_scale_count = t->router_scale ? t->router_scale_count : 0;
    CK(cudaStreamSynchronize(eng->ustream));
    return 1;
}

int moe_b200_sync(moe_b200_engine_t* eng, void* stream, char* err) {
    if (!eng) {
        set_err(err, "null engine");
        return 0;
    }
    CK(cudaSetDevice(eng->device));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the error word rides the stream: one synchronisation covers both
    CK(cudaMemcpyAsync(eng->h_err, eng->err_word.ptr, 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    const uint32_t code = *eng->h_err;
    if (code != kErrNone) {
        CK(cudaMemsetAsync(eng->err_word.ptr, 0, 4, st));
        CK(cudaStreamSynchronize(st));
        const char* what = code == kErrBadExpert            ? "expert id out of range"
                           : code == kErrAllExpertsMissing  ? "every expert of a token is missing (skip_missing)"
                           : code == kErrTimeoutRouterLoad  ? "bounded wait timed out in the router"
                           : code == kErrTimeoutPeer        ? "bounded wait for another rank timed out"
                                                            : "bounded wait timed out in a GEMM pipeline";
        set_err(err, "device error %u (%s)", code, what);
        return 0;
    }
    return 1;
}

int moe_b200_layer_forward_host(moe_b200_engine_t* eng, const moe_b200_layer_cfg_t* cfg, const uint16_t* x,
                                uint32_t T, uint16_t* y_bf16, float* y_f32, int32_t* topk_ids, float* topk_w,
                                uint32_t* perm, char* err) {
    if (!check_dims(cfg, err)) return 0;
    if (!eng) {
        set_err(err, "null engine");
        return 0;
    }
    if (T == 0) return 1;
    if (!x) {
        set_err(err, "null input");
        return 0;
    }
    CK(cudaSetDevice(eng->device));
    const uint32_t H = cfg->hidden, K = cfg->top_k;
    CK(eng->hx.reserve((size_t)T * H * 2));
    CK(eng->hy.reserve((size_t)T * H * 2));
    CK(eng->hyf.reserve((size_t)T * H * 4));
    CK(eng->hids.reserve((size_t)T * K * 4));
    CK(eng->hw.reserve((size_t)T * K * 4));
    CK(eng->hperm_out.reserve((size_t)T * K * 4));
    cudaStream_t st = eng->hstream;
    // large batches without the permutation output: chunked copies (the
    // plain router path only; the f32 router of the block parts reads the
    // residual stream, which this call does not take)
    const LayerWeights* Lp = (cfg->layer >= 0 && (size_t)cfg->layer < eng->layers.size()) ? &eng->layers[cfg->layer]
                                                                                            : nullptr;
    const bool chunked = T >= kPipeMinTokens && !perm && Lp && !Lp->blk_pre_norm2.ptr && !Lp->blk_router_scale.ptr;
    if (chunked) {
        if (!eng->pipe_in) {
            CK(cudaStreamCreateWithFlags(&eng->pipe_in, cudaStreamNonBlocking));
            CK(cudaStreamCreateWithFlags(&eng->pipe_out, cudaStreamNonBlocking));
        }
        while (eng->pipe_ev.size() < 2 * kPipeChunks) {
            cudaEvent_t e;
            CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
            eng->pipe_ev.push_back(e);
        }
        const HostPipe pipe{x, y_bf16, y_f32, topk_ids, topk_w};
        if (!forward_impl(eng, cfg, eng->hx.as<uint16_t>(), nullptr, T, y_bf16 ? eng->hy.as<uint16_t>() : nullptr,
                          y_f32 ? eng->hyf.as<float>() : nullptr, eng->hids.as<int32_t>(), eng->hw.as<float>(),
                          nullptr, st, err, &pipe)) {
            return 0;
        }
        if (!moe_b200_sync(eng, st, err)) return 0;
        CK(cudaStreamSynchronize(eng->pipe_out));
        return 1;
    }
    CK(cudaMemcpyAsync(eng->hx.ptr, x, (size_t)T * H * 2, cudaMemcpyHostToDevice, st));
    if (!moe_b200_layer_forward(eng, cfg, eng->hx.as<uint16_t>(), T, y_bf16 ? eng->hy.as<uint16_t>() : nullptr,
                                y_f32 ? eng->hyf.as<float>() : nullptr, eng->hids.as<int32_t>(),
                                eng->hw.as<float>(), perm ? eng->hperm_out.as<uint32_t>() : nullptr, st, err)) {
        return 0;
    }
    if (y_bf16) CK(cudaMemcpyAsync(y_bf16, eng->hy.ptr, (size_t)T * H * 2, cudaMemcpyDeviceToHost, st));
    if (y_f32) CK(cudaMemcpyAsync(y_f32, eng->hyf.ptr, (size_t)T * H * 4, cudaMemcpyDeviceToHost, st));
    if (topk_ids) CK(cudaMemcpyAsync(topk_ids, eng->hids.ptr, (size_t)T * K * 4, cudaMemcpyDeviceToHost, st));
    if (topk_w) CK(cudaMemcpyAsync(topk_w, eng->hw.ptr, (size_t)T * K * 4, cudaMemcpyDeviceToHost, st));
    if (perm) CK(cudaMemcpyAsync(perm, eng->hperm_out.ptr, (size_t)T * K * 4, cudaMemcpyDeviceToHost, st));
    return moe_b200_sync(eng, st, err);
}

int moe_b200_run_expert_triplet_f32(moe_b200_engine_t* eng, int layer, int expert, const float* hidden,
                                    uint32_t hidden_count, float* scratch_gate, float* scratch_up,
                                    uint32_t intermediate_count, float* out_hidden, uint32_t out_count) {
    char* err = nullptr;
    if (!eng || !hidden || !scratch_gate || !scratch_up || !out_hidden) return 0;
    if (layer < 0 || (size_t)layer >= eng->layers.size()) return 0;
    LayerWeights* L = &eng->layers[layer];
    if (!L->E || !L->I || hidden_count != L->H || out_count != L->H || intermediate_count != L->I) return 0;
    if (expert < -1 || expert >= (int)L->E) return 0;
    const uint32_t slot = expert < 0 ? L->E : (uint32_t)expert;
    if (!L->present[slot]) return 0;
    CK(cudaSetDevice(eng->device));
    if (!ensure_tile_form(eng, L, slot, err)) return 0;
    const uint32_t H = L->H, I = L->I;
    CK(eng->tri.reserve((size_t)(H + 2 * I + H) * 4));
    float* dx = eng->tri.as<float>();
    float* dg = dx + H;
    float* du = dg + I;
    float* dout = du + I;
    CK(cudaMemcpy(dx, hidden, (size_t)H * 4, cudaMemcpyHostToDevice));
    CK(launch_triplet_f32(L->gu.as<uint8_t>() + L->gu_stride * slot, L->dn.as<uint8_t>() + L->dn_stride * slot, dx,
                          H, I, dg, du, dout, 0));
    CK(cudaMemcpy(scratch_gate, dg, (size_t)I * 4, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(scratch_up, du, (size_t)I * 4, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(out_hidden, dout, (size_t)H * 4, cudaMemcpyDeviceToHost));
    return 1;
}

int moe_b200_debug_dequant(moe_b200_engine_t* eng, int32_t layer, int32_t expert, int32_t proj, uint16_t* out,
                           uint64_t out_elems, char* err) {
    LayerWeights* L = get_layer(eng, layer, err);
    if (!L) return 0;
    if (expert < -1 || expert >= (int32_t)L->E || !L->I) {
        set_err(err, "no such expert %d", expert);
        return 0;
    }
    const uint32_t slot = expert < 0 ? L->E : (uint32_t)expert;
    if (!L->present[slot]) {
        set_err(err, "expert %d not uploaded", expert);
        return 0;
    }
    const uint32_t rows = proj == MOE_B200_PROJ_DOWN ? L->H : L->I;
    const uint32_t cols = proj == MOE_B200_PROJ_DOWN ? L->I : L->H;
    if (!out || out_elems < (uint64_t)rows * cols) {
        set_err(err, "output needs %llu elements", (unsigned long long)rows * cols);
        return 0;
    }
    CK(cudaSetDevice(eng->device));
    if (!ensure_tile_form(eng, L, slot, err)) return 0;
    const uint8_t* tiles = proj == MOE_B200_PROJ_DOWN ? L->dn.as<uint8_t>() + L->dn_stride * slot
                                                      : L->gu.as<uint8_t>() + L->gu_stride * slot +
                                                            (proj == MOE_B200_PROJ_UP ? kTileBytes : 0);
    const uint32_t stride = proj == MOE_B200_PROJ_DOWN ? kTileBytes : 2 * kTileBytes;
    DevBuf tmp;
    CK(tmp.reserve((size_t)rows * cols * 2));
    CK(launch_dequant_wtiles(tiles, rows, cols, stride, tmp.as<uint16_t>(), 0));
    CK(cudaMemcpy(out, tmp.ptr, (size_t)rows * cols * 2, cudaMemcpyDeviceToHost));
    tmp.release();
    return 1;
}

int moe_b200_debug_read(moe_b200_engine_t* eng, int32_t which, void* dst, uint64_t bytes, char* err) {
    if (!eng || !dst) {
        set_err(err, "null argument");
        return 0;
    }
    CK(cudaSetDevice(eng->device));
    CK(cudaDeviceSynchronize());
    const void* src = nullptr;
    uint64_t have = 0;
    switch (which) {
        case MOE_B200_BUF_LOGITS: src = eng->logits.ptr; have = (uint64_t)eng->last_T * eng->last_E * 4; break;
        case MOE_B200_BUF_SCORES: src = eng->scores.ptr; have = (uint64_t)eng->last_T * eng->last_E * 4; break;
        case MOE_B200_BUF_GROUP_COUNT: src = eng->g_count.ptr; have = (uint64_t)eng->last_G * 4; break;
        case MOE_B200_BUF_GROUP_OFFSET: src = eng->g_offset.ptr; have = (uint64_t)(eng->last_G + 1) * 4; break;
        case MOE_B200_BUF_ROW_TOKEN: src = eng->row_token.ptr; have = (uint64_t)eng->last_P * 4; break;
        case MOE_B200_BUF_XPERM: src = eng->xperm.ptr; have = eng->xperm.bytes; break;
        case MOE_B200_BUF_HPERM: src = eng->hperm.ptr; have = eng->hperm.bytes; break;
        case MOE_B200_BUF_YPERM: src = eng->yperm.ptr; have = (uint64_t)eng->last_P * eng->last_H * 4; break;
        default: set_err(err, "unknown buffer %d", which); return 0;
    }
    if (!src || bytes > have) {
        set_err(err, "buffer %d holds %llu bytes, %llu requested", which, (unsigned long long)have,
                (unsigned long long)bytes);
        return 0;
    }
    CK(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost));
    return 1;
}

uint32_t moe_b200_last_launch_count(const moe_b200_engine_t* eng) { return eng ? eng->last_launches : 0; }

int moe_b200_profile_enable(moe_b200_engine_t* eng, uint32_t max_calls, char* err) {
    if (!eng) {
        set_err(err, "null engine");
        return 0;
    }
    CK(cudaSetDevice(eng->device));
    for (cudaEvent_t e : eng->prof_events) cudaEventDestroy(e);
    eng->prof_events.clear();
    eng->prof_max = 0;
    eng->prof_calls = 0;
    if (max_calls == 0) return 1;
    eng->prof_events.resize((size_t)max_calls * (MOE_B200_STAGES + 1));
    for (auto& e : eng->prof_events) CK(cudaEventCreate(&e));
    eng->prof_max = max_calls;
    return 1;
}

int moe_b200_profile_read(moe_b200_engine_t* eng, float* stage_ms, uint32_t* calls, char* err) {
    if (!eng || !stage_ms) {
        set_err(err, "null argument");
        return 0;
    }
    CK(cudaSetDevice(eng->device));
    for (int s = 0; s < MOE_B200_STAGES; ++s) stage_ms[s] = 0.f;
    for (uint32_t c = 0; c < eng->prof_calls; ++c) {
        cudaEvent_t* ev = &eng->prof_events[(size_t)c * (MOE_B200_STAGES + 1)];
        CK(cudaEventSynchronize(ev[MOE_B200_STAGES]));
        for (int s = 0; s < MOE_B200_STAGES; ++s) {
            float ms = 0.f;
            CK(cudaEventElapsedTime(&ms, ev[s], ev[s + 1]));
            stage_ms[s] += ms;
        }
    }
    if (calls) *calls = eng->prof_calls;
    return 1;
}

int moe_b200_group_tokens_by_expert(const moe_b200_assignment_t* assignments, uint32_t n,
                                    moe_b200_assignment_t* out_sorted, moe_b200_batch_t* out_batches,
                                    uint32_t max_batches, uint32_t* out_batch_count) {
    static_assert(sizeof(moe_b200_assignment_t) == sizeof(AssignRec), "assignment layout");
    static_assert(sizeof(moe_b200_batch_t) == 4 * sizeof(uint32_t), "batch layout");
    if (!assignments || n == 0 || !out_batch_count) {
        if (out_batch_count) *out_batch_count = 0;
        return 0;
    }
    if (n > (1u << 30)) return 0;
    // Process-wide workspace on the current device; the utility has no
    // engine handle (its signature is the reference's).
    static std::mutex mu;
    static DevBuf a, sorted, ord0, ord1, keys, tiles, rank, cnt, off, z0, z1, batches, bcount, errw;
    static int dev = -1;
    std::lock_guard<std::mutex> lock(mu);
    char* err = nullptr;
    int cur = 0;
    CK(cudaGetDevice(&cur));
    if (dev != cur) {
        DevBuf* all[] = {&a, &sorted, &ord0, &ord1, &keys, &tiles, &rank, &cnt, &off, &z0, &z1, &batches, &bcount, &errw};
        for (DevBuf* b : all) { b->ptr = nullptr; b->bytes = 0; }  // buffers of another device are abandoned
        dev = cur;
    }
    const size_t rec = sizeof(AssignRec);
    CK(a.reserve(n * rec));
    CK(sorted.reserve(n * rec));
    CK(ord0.reserve(n * 4));
    CK(ord1.reserve(n * 4));
    CK(keys.reserve(n * 4));
    CK(tiles.reserve((size_t)sort_tiles(n) * 256 * 4));
    CK(rank.reserve(n * 4));
    CK(cnt.reserve(257 * 4));
    CK(off.reserve(257 * 4));
    CK(z0.reserve(257 * 4));
    CK(z1.reserve(257 * 4));
    CK(batches.reserve((size_t)n * 16));
    CK(bcount.reserve(4));
    CK(errw.reserve(4));
    CK(cudaMemset(errw.ptr, 0, 4));
    CK(cudaMemcpy(a.ptr, assignments, n * rec, cudaMemcpyHostToDevice));
    // digit passes needed per field (least significant key first)
    uint32_t mx[3] = {0, 0, 0};
    for (uint32_t i = 0; i < n; ++i) {
        mx[0] = std::max(mx[0], assignments[i].token_index);
        mx[1] = std::max(mx[1], assignments[i].expert);
        mx[2] = std::max(mx[2], assignments[i].layer);
    }
    GroupInfo gi{cnt.as<uint32_t>(), off.as<uint32_t>(), z0.as<uint32_t>(), z1.as<uint32_t>(), 1, 0, 0};
    cudaStream_t st = 0;
    CK(launch_iota(ord0.as<uint32_t>(), n, st));
    uint32_t* in = ord0.as<uint32_t>();
    uint32_t* out = ord1.as<uint32_t>();
    for (int field = 0; field < 3; ++field) {
        for (int shift = 0; shift < 32 && (shift == 0 || (mx[field] >> shift) != 0); shift += 8) {
            if (mx[field] == 0) break;
            CK(launch_group_pass(a.as<AssignRec>(), in, out, n, field, shift, keys.as<int32_t>(),
                                 tiles.as<uint32_t>(), rank.as<uint32_t>(), gi, errw.as<uint32_t>(), st));
            std::swap(in, out);
        }
    }
    CK(launch_group_finish(a.as<AssignRec>(), in, n, sorted.as<AssignRec>(), batches.as<uint32_t>(),
                           bcount.as<uint32_t>(), st));
    uint32_t nb = 0;
    CK(cudaMemcpy(&nb, bcount.ptr, 4, cudaMemcpyDeviceToHost));
    if (out_sorted) CK(cudaMemcpy(out_sorted, sorted.ptr, n * rec, cudaMemcpyDeviceToHost));
    if (out_batches && max_batches) {
        CK(cudaMemcpy(out_batches, batches.ptr, (size_t)std::min(nb, max_batches) * 16, cudaMemcpyDeviceToHost));
    }
    *out_batch_count = nb;
    return (!out_batches || nb <= max_batches) ? 1 : 0;
}

}  // extern "C"
