// Engine internals shared by the C-ABI translation units (api.cu, ep.cu):
// device buffers, the per-layer weight cache, the engine handle and the
// block-scaled expert pipeline both the single-device and the
// expert-parallel forward run.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "../../include/moe_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace moe_b200 {

inline void set_err(char* err, const char* fmt, ...) {
    if (!err) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, MOE_B200_ERR_LEN, fmt, ap);
    va_end(ap);
}

#define CK(call)                                                                                   \
    do {                                                                                           \
        cudaError_t e_ = (call);                                                                   \
        if (e_ != cudaSuccess) {                                                                   \
            set_err(err, "%s failed: %s", #call, cudaGetErrorString(e_));                          \
            return 0;                                                                              \
        }                                                                                          \
    } while (0)

// Device buffer that only grows.
struct DevBuf {
    void* ptr = nullptr;
    size_t bytes = 0;
    cudaError_t reserve(size_t want) {
        if (want <= bytes) return cudaSuccess;
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
        cudaError_t e = cudaMalloc(&ptr, want);
        if (e == cudaSuccess) bytes = want;
        return e;
    }
    void release() {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
    }
    template <class T>
    T* as() const {
        return static_cast<T*>(ptr);
    }
};

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct LayerWeights {
    uint32_t E = 0, H = 0, I = 0;
    DevBuf router;          // bf16 [E x H]
    // the one resident form of the experts, block-scaled: packed E2M1 codes
    // + E8M0 scale blocks (what the product GEMMs read)
    DevBuf bs_gu_codes, bs_gu_sfa, bs_dn_codes, bs_dn_sfa;
    std::vector<uint8_t> present;  // [E+1]; slot E = shared expert
    // tile form of the cross-check GEMMs, the fp32 triplet and the dequant
    // hook ("wtile", common.cuh): allocated and derived from the
    // block-scaled form only when one of those is first called
    DevBuf gu;              // [E+1] groups of interleaved gate/up tiles
    DevBuf dn;              // [E+1] groups of down tiles
    uint64_t gu_stride = 0, dn_stride = 0;
    std::vector<uint8_t> tile_ready;  // [E+1]: slot's tile form is current
    // Gemma-style block parts (moe_b200_upload_block); empty = absent
    DevBuf blk_pre_norm2, blk_post_norm1, blk_post_norm2, blk_post_norm, blk_down_scale, blk_gate_inp,
        blk_router_scale;
    uint64_t blk_down_scale_count = 0, blk_router_scale_count = 0;
    bool has_block_combine() const {
        return blk_post_norm1.ptr || blk_post_norm2.ptr || blk_post_norm.ptr || blk_down_scale.ptr || blk_gate_inp.ptr;
    }
    bool needs_hidden() const { return blk_pre_norm2.ptr || blk_router_scale.ptr; }
    bool has_block() const { return has_block_combine() || needs_hidden(); }
    void release_block() {
        DevBuf* b[] = {&blk_pre_norm2, &blk_post_norm1, &blk_post_norm2, &blk_post_norm, &blk_down_scale,
                       &blk_gate_inp, &blk_router_scale};
        for (DevBuf* x : b) x->release();
        blk_down_scale_count = blk_router_scale_count = 0;
    }
    uint32_t rp_i = 0, rp_h = 0, kq = 0, iq = 0;  // rows padded to 128, K padded to 128
    CUtensorMap tmap_gu_codes{}, tmap_dn_codes{};
    // the same codes as packed bytes (64-byte rows, 64-byte swizzle) for the
    // fast mode's kind::mxf4 GEMMs
    CUtensorMap tmap_gu_fp4{}, tmap_dn_fp4{};
    void release_all() {
        release_block();
        router.release();
        gu.release();
        dn.release();
        bs_gu_codes.release();
        bs_gu_sfa.release();
        bs_dn_codes.release();
        bs_dn_sfa.release();
    }
};

inline uint32_t round_up(uint32_t v, uint32_t m) { return (v + m - 1) / m * m; }

struct EpState;
void ep_release(EpState* ep);

}  // namespace moe_b200

struct moe_b200_engine {
    using DevBuf = moe_b200::DevBuf;
    using LayerWeights = moe_b200::LayerWeights;
    using EncodeTiledFn = moe_b200::EncodeTiledFn;
    int device = 0;
    int num_sms = 148;
    // 128-token tiles of the exact path run on CTA pairs (cta_group::2);
    // MOE_B200_CTA_PAIRS=0 in the environment at engine creation selects the
    // one-CTA kernels instead
    bool cta_pairs = true;
    std::vector<LayerWeights> layers;
    DevBuf staging;  // GGUF bytes copied from the host before the repack
    // uploads and tile-form derivations run here and wait only for
    // themselves; a blocking stream, so it is ordered after work the caller
    // queued on the legacy default stream (e.g. the copy that produced a
    // device-resident source)
    cudaStream_t ustream = nullptr;
    // workspace
    DevBuf logits, scores, ids, wts, tile_counts, rank, pos_of, row_token, row_assign, row_info;
    DevBuf g_count, g_offset, g_gu_off, g_dn_off;
    DevBuf xperm, hperm, yperm;
    DevBuf err_word;
    // skip_missing with a renormalising router: the layer's expert presence
    // and the combine weights computed from it
    DevBuf present_dev, comb_w;
    // block-scaled path: quantised activations and intermediate
    // (xb, hb hold a hi plane followed by a lo plane)
    DevBuf xb, sfx_atoms, hb, sfh_atoms, gu_tiles, dn_tiles;
    // block parts: pre-normed routed input (fp32 for the router, bf16 for the
    // experts), the router's fp32 input, the shared-expert gate's routing
    DevBuf xr_f32, xr_bf16, rin_f32, gate_logits, gate_ids, gate_w, gate_scores;
    // 3-D maps over xb / hb: [0] 32-token box, [1] 64-token box, [2] 128-token box
    CUtensorMap tmap_xb[3]{}, tmap_hb[3]{};
    const void* bs_map_key[2] = {nullptr, nullptr};
    uint64_t bs_map_dims[2][2] = {};
    // fast mode: 2-D byte maps over the same buffers holding packed E2M1 rows
    CUtensorMap tmap_xq[3]{}, tmap_hq[3]{};
    const void* fp4_map_key[2] = {nullptr, nullptr};
    uint64_t fp4_map_dims[2][2] = {};
    // host-call staging
    DevBuf hx, hy, hyf, hids, hw, hperm_out, tri, hhid;
    // host-buffer entry points: their own non-blocking stream, and a pinned
    // word the error code is copied into before the one synchronisation
    cudaStream_t hstream = nullptr;
    // host-buffer calls on large batches: token chunks of x are copied in on
    // pipe_in and routed as they land; the combined rows go back on pipe_out
    // chunk by chunk (events: kPipeChunks copy-ins, then kPipeChunks combines)
    cudaStream_t pipe_in = nullptr, pipe_out = nullptr;
    std::vector<cudaEvent_t> pipe_ev;
    // ... and the shared expert runs on each chunk as it lands: its output
    // rows by token, its all-zero group ids, its one-entry group -> slot map
    DevBuf pipe_ys, pipe_zero_ids, pipe_slot;
    uint32_t* h_err = nullptr;
    CUtensorMap tmap_x{}, tmap_h{};
    void* tmap_x_base = nullptr;
    void* tmap_h_base = nullptr;
    uint64_t tmap_x_dims[2] = {0, 0}, tmap_h_dims[2] = {0, 0};
    EncodeTiledFn encode = nullptr;
    // last-forward geometry (debug reads)
    uint32_t last_T = 0, last_E = 0, last_G = 0, last_P = 0, last_Kp = 0, last_Ip = 0, last_H = 0;
    uint32_t last_launches = 0;
    // stage profiling
    std::vector<cudaEvent_t> prof_events;  // [max_calls][MOE_B200_STAGES + 1]
    uint32_t prof_max = 0, prof_calls = 0;
    // expert parallelism (ep.cu); null until moe_b200_ep_init
    moe_b200::EpState* ep = nullptr;
};


namespace moe_b200 {

int check_dims(const moe_b200_layer_cfg_t* c, char* err);
LayerWeights* get_layer(moe_b200_engine* eng, int32_t layer, char* err);
// Makes the tile form of `slot` current (allocating the layer's tile buffers
// on first use) from its block-scaled form; synchronises the upload stream.
int ensure_tile_form(moe_b200_engine* eng, LayerWeights* L, uint32_t slot, char* err);
bool router_tmaps(moe_b200_engine* eng, const uint16_t* x, const uint16_t* w, uint32_t T, uint32_t E, uint32_t H,
                  CUtensorMap* tx, CUtensorMap* tw);

// One run of the block-scaled expert pipeline: permutation of T*K
// assignments into E routed groups (+ an extra shared-expert group of
// `shared_rows` rows), quantise-on-gather, gate/up GEMM, down GEMM.
struct BsJob {
    const int32_t* ids;          // group of each assignment a, device [T*K]
    uint32_t T, K;               // assignment a reads source row a / K
    uint32_t E;                  // routed groups
    uint32_t shared_rows;        // rows of the shared-expert group (0: none) ...
    uint32_t shared_base;        // ... reading source rows shared_base + t
    const uint16_t* src;         // source rows, bf16 [*, H], device
    const uint16_t* src_shared = nullptr;  // the shared group's source rows when they differ from src
    int32_t act = 0;             // gated activation (MOE_B200_ACT_*)
    const uint32_t* group_slot;  // weight slot of each group (device); null: routed group g -> slot g,
                                 // shared group -> slot E of the layer
    float* y;                    // expert outputs, fp32 rows [*, H]
    bool y_by_source;            // row of y: the source row (else the permuted row)
    // expert parallelism: source rows below ret_rows are other ranks' tokens,
    // stored by the down GEMM into their return buffers (see BsParams)
    float* const* ret_ptrs = nullptr;
    const uint32_t* ret_roff = nullptr;
    const uint32_t* ret_base = nullptr;
    uint32_t ret_rows = 0;
    uint32_t ret_world = 0;
    bool fp4 = false;            // fast mode: E2M1 activations, kind::mxf4 GEMMs
};

// Enqueues the pipeline on `st`; fills the engine's permutation buffers
// (pos_of: permuted row of each assignment).  `ev`, when not null, receives
// stage marks 2..5.  Adds its kernel launches to *launches.
int run_blockscaled(moe_b200_engine* eng, LayerWeights* L, const BsJob& job, cudaStream_t st, cudaEvent_t* ev,
                    uint32_t* launches, char* err);

}  // namespace moe_b200
