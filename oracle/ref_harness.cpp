// TEST INFRASTRUCTURE ONLY -- never part of the shipped product path.
//
// Compiles the reference's own CPU MoE hot path (jujumelona/storage.llm,
// moe_engine) into oracle/_ref/libmoe_ref.so so the tests and the bench's
// reference arm can call it.  This file contains no reference source: it
// textually includes the reference's single translation unit
// (moe_engine/src/moe_pc_engine.cpp, which itself includes every
// src/parts/*.cpp.inc) from the read-only reference checkout, and adds thin
// extern "C" entry points around the reference's `static` hot-path functions.
//
// The layer entry point composes the reference leaves in exactly the order
// of moe_layer_moe_mlp_f32 (generation_mlp.cpp.inc:776-1442) for one token at
// a time, which is how the engine runs a layer (generation_forward.cpp.inc:
// 212-215 / generation_api_main.cpp.inc:261-283):
//   router     moe_router_topk_f32            generation_router.cpp.inc:560-682
//   shared     dense MLP (gate/up/act, down)  generation_mlp.cpp.inc:596-727, 839-860
//   gate/up    moe_parallel_rows(k*I) -> moe_dot_gguf_mxfp4_row x2 -> act
//                                             generation_mlp.cpp.inc:1335-1376
//   down       moe_parallel_rows(k*H) -> moe_dot_gguf_mxfp4_row
//                                             generation_mlp.cpp.inc:1378-1413
//   combine    moe_axpy_f32 in router order   generation_mlp.cpp.inc:1415-1431
// ref_moe_block adds the optional parts of Gemma-style blocks around the
// experts through the reference's own functions for them (the MoE pre-norm,
// post-FFW norms 1/2/final, expert down scales, shared-expert gate).
// ref_moe_layer_engine runs moe_layer_moe_mlp_f32 itself, its experts filed
// as tensor records over a shard file, which pins the leaf composition above
// to the layer function the engine calls.
// Weights are passed in the reference's GGUF MXFP4 byte layout (17-byte
// blocks per 32 K-elements, tensor_layout.cpp.inc:174-176).
#include "moe_engine/src/moe_pc_engine.cpp"

#include <xmmintrin.h>
#include <pmmintrin.h>

namespace {

// Restores the caller thread's MXCSR: the reference's row pool switches the
// calling thread to FTZ/DAZ (parallel_rows.cpp.inc:39-46, 215) and the
// Python test process must not inherit that.
struct mxcsr_guard {
    unsigned int saved;
    mxcsr_guard() : saved(_mm_getcsr()) {}
    ~mxcsr_guard() { _mm_setcsr(saved); }
};

uint64_t router_cache_key(int32_t layer) {
    // Same key the reference builds in moe_map_router_tensor
    // (generation_router.cpp.inc:159-160).
    const uint32_t suffix_hash = moe_router_fnv1a_hash_string("ffn_gate_inp.weight");
    return ((uint64_t)(uint32_t)layer << 32) | suffix_hash | 0x80000000ull;
}

// Key of the router's input scale tensor (moe_map_router_scale_tensor,
// generation_router.cpp.inc:272-314).
uint64_t router_scale_key(int32_t layer) {
    return ((uint64_t)(uint32_t)layer << 32) | moe_router_fnv1a_hash_string("ffn_gate_inp.scale") | 0x80000000ull;
}

// The plain router and layer entry points model layers without a router
// input scale: drop one a block call may have left in this engine's cache.
void clear_router_scale(moe_pc_engine* engine, int32_t layer) {
    std::unique_lock<std::shared_mutex> lock(engine->raw_tensor_cache_mutex);
    engine->raw_tensor_cache.erase(router_scale_key(layer));
}

float bf16_to_f32(uint16_t v) {
    uint32_t bits = (uint32_t)v << 16;
    float out;
    std::memcpy(&out, &bits, sizeof(out));
    return out;
}

}  // namespace

extern "C" {

typedef struct {
    uint32_t hidden;        // H
    uint32_t intermediate;  // I
    uint32_t experts;       // E
    uint32_t top_k;         // k (also written to the engine metadata)
    const uint16_t* router_bf16;  // [E x H] row-major bf16 (ffn_gate_inp.weight)
    const uint8_t* gate;    // [E][I rows][ceil(H/32)*17 B]
    const uint8_t* up;      // [E][I rows][ceil(H/32)*17 B]
    const uint8_t* down;    // [E][H rows][ceil(I/32)*17 B]
    const uint8_t* shared_gate;  // [I][ceil(H/32)*17] or null
    const uint8_t* shared_up;
    const uint8_t* shared_down;  // [H][ceil(I/32)*17]
} ref_layer_desc;

// Creates a reference engine whose GGUF metadata JSON is `metadata_json`
// (e.g. {"num_experts_per_tok":4,"norm_topk_prob":false}).  Routing semantics
// come from those keys exactly as in the engine (generation_router.cpp.inc:
// 361-482).
void* ref_engine_create(const char* metadata_json) {
    mxcsr_guard guard;
    moe_pc_engine_config_t cfg = moe_pc_default_config();
    cfg.prefer_gpu = 0;
    cfg.vram_budget_bytes = 0;
    moe_pc_engine_t* engine = moe_pc_engine_create(&cfg);
    if (!engine) return nullptr;
    engine->offload_gguf_metadata_json = metadata_json ? metadata_json : "";
    return engine;
}

void ref_engine_destroy(void* engine) {
    mxcsr_guard guard;
    moe_pc_engine_destroy(static_cast<moe_pc_engine_t*>(engine));
}

uint32_t ref_row_threads(void) { return row_hw_threads(); }

float ref_e8m0_to_f32(uint8_t v) { return moe_e8m0_to_f32_half(v); }

float ref_mxfp4_value(uint8_t code) { return moe_mxfp4_value_from_code(code); }

// One reference MXFP4 row dot per row (tensor_dot_cpu_kernels.cpp.inc:601-667).
void ref_mxfp4_dot_rows(const uint8_t* packed, uint32_t rows, uint32_t cols,
                        const float* x, float* out) {
    mxcsr_guard guard;
    const uint64_t row_bytes = (uint64_t)((cols + 31u) / 32u) * 17u;
    for (uint32_t r = 0; r < rows; ++r) {
        out[r] = moe_dot_gguf_mxfp4_row(packed + (uint64_t)r * row_bytes, x, cols);
    }
}

// Reference bf16 router row dot (raw_forward_utils.cpp.inc:174-216).
void ref_bf16_dot_rows(const uint16_t* w, uint32_t rows, uint32_t cols,
                       const float* x, float* out) {
    mxcsr_guard guard;
    for (uint32_t r = 0; r < rows; ++r) {
        out[r] = moe_dot_bf16_row(reinterpret_cast<const uint8_t*>(w + (uint64_t)r * cols), x, cols);
    }
}

float ref_silu(float x) { return moe_generation_silu(x); }

// Router top-k for T tokens through moe_router_topk_f32 itself.  `logits`
// (optional, [T x E]) receives the router's post-softmax scores.
int ref_router_topk(void* eng, const uint16_t* router_bf16, uint32_t experts,
                    uint32_t hidden, const uint16_t* x_bf16, uint32_t tokens,
                    uint32_t top_k, int32_t* out_ids, float* out_w, float* out_scores) {
    mxcsr_guard guard;
    moe_pc_engine* engine = static_cast<moe_pc_engine*>(eng);
    if (!engine || !router_bf16 || !x_bf16) return 0;
    const int32_t layer = 0;
    clear_router_scale(engine, layer);
    moe_raw_tensor_cache_entry entry{};
    entry.base = reinterpret_cast<const uint8_t*>(router_bf16);
    entry.bytes = (uint64_t)experts * hidden * 2ull;
    entry.rows = experts;
    entry.cols = hidden;
    entry.scalar_encoding = moe_RAW_SCALAR_BF16;
    entry.weight_format = moe_WEIGHT_ENCODING_RAW_BF16;
    {
        std::unique_lock<std::shared_mutex> lock(engine->raw_tensor_cache_mutex);
        engine->raw_tensor_cache[router_cache_key(layer)] = entry;
    }
    std::vector<float> x(hidden);
    std::vector<int> ids;
    std::vector<float> w, logits;
    std::vector<uint32_t> order;
    for (uint32_t t = 0; t < tokens; ++t) {
        for (uint32_t h = 0; h < hidden; ++h) x[h] = bf16_to_f32(x_bf16[(uint64_t)t * hidden + h]);
        if (!moe_router_topk_f32(engine, layer, x.data(), hidden, experts, top_k,
                                 &ids, &w, &logits, &order)) {
            return 0;
        }
        if (ids.size() != top_k) return 0;
        for (uint32_t j = 0; j < top_k; ++j) {
            out_ids[(uint64_t)t * top_k + j] = ids[j];
            out_w[(uint64_t)t * top_k + j] = w[j];
        }
        if (out_scores) {
            for (uint32_t e = 0; e < experts; ++e) out_scores[(uint64_t)t * experts + e] = logits[e];
        }
    }
    return 1;
}

// Whole MoE FFN layer for T tokens, one token at a time, in the order of
// moe_layer_moe_mlp_f32.  y_f32 receives the MoE block output `mlp`
// (shared + sum_e w_e * y_e) before the residual add of
// moe_add_mlp_residual_f32 (generation_mlp.cpp.inc:572-594).
int ref_moe_layer(void* eng, const ref_layer_desc* d, const uint16_t* x_bf16,
                  uint32_t tokens, float* y_f32, int32_t* out_ids, float* out_w) {
    mxcsr_guard guard;
    moe_pc_engine* engine = static_cast<moe_pc_engine*>(eng);
    if (!engine || !d || !x_bf16 || !y_f32) return 0;
    const uint32_t H = d->hidden, I = d->intermediate, E = d->experts, K = d->top_k;
    const int32_t layer = 0;
    clear_router_scale(engine, layer);
    const uint64_t row_h = (uint64_t)((H + 31u) / 32u) * 17u;
    const uint64_t row_i = (uint64_t)((I + 31u) / 32u) * 17u;
    const uint64_t expert_gu_bytes = (uint64_t)I * row_h;
    const uint64_t expert_d_bytes = (uint64_t)H * row_i;

    moe_raw_tensor_cache_entry entry{};
    entry.base = reinterpret_cast<const uint8_t*>(d->router_bf16);
    entry.bytes = (uint64_t)E * H * 2ull;
    entry.rows = E;
    entry.cols = H;
    entry.scalar_encoding = moe_RAW_SCALAR_BF16;
    entry.weight_format = moe_WEIGHT_ENCODING_RAW_BF16;
    {
        std::unique_lock<std::shared_mutex> lock(engine->raw_tensor_cache_mutex);
        engine->raw_tensor_cache[router_cache_key(layer)] = entry;
    }
    const int activation_mode = moe_engine_gelu_activation_mode(engine);

    std::vector<float> x(H), mlp(H), shared_gate(I), shared_out(H);
    std::vector<float> gate_pool((uint64_t)K * I), up_pool((uint64_t)K * I), out_pool((uint64_t)K * H);
    std::vector<int> ids;
    std::vector<float> w, logits;
    std::vector<uint32_t> order;
    for (uint32_t t = 0; t < tokens; ++t) {
        for (uint32_t h = 0; h < H; ++h) x[h] = bf16_to_f32(x_bf16[(uint64_t)t * H + h]);
        std::fill(mlp.begin(), mlp.end(), 0.0f);
        // Shared expert first (generation_mlp.cpp.inc:839-860, dense MLP :707-727).
        if (d->shared_gate && d->shared_up && d->shared_down) {
            if (!moe_parallel_rows(engine, I, 0, [&](uint32_t row) {
                    const float g = moe_dot_gguf_mxfp4_row(d->shared_gate + row * row_h, x.data(), H);
                    const float u = moe_dot_gguf_mxfp4_row(d->shared_up + row * row_h, x.data(), H);
                    shared_gate[row] = moe_generation_gated_activation_cached(activation_mode, g, u);
                    return 1;
                })) return 0;
            if (!moe_parallel_rows(engine, H, 0, [&](uint32_t row) {
                    shared_out[row] = moe_dot_gguf_mxfp4_row(d->shared_down + row * row_i, shared_gate.data(), I);
                    return 1;
                })) return 0;
            const float gate_scalar = 1.0f;  // no shared gate tensor (:478-512)
            for (uint32_t i = 0; i < H; ++i) mlp[i] += shared_out[i] * gate_scalar;
        }
        if (!moe_router_topk_f32(engine, layer, x.data(), H, E, K, &ids, &w, &logits, &order)) {
            return 0;
        }
        const size_t sel = ids.size();
        if (sel != K) return 0;
        // Phase 2a: gate + up + activation over k*I flat rows (:1346-1370).
        if (!moe_parallel_rows(engine, (uint32_t)(sel * I), 0, [&](uint32_t flat_row) {
                const uint32_t e = flat_row / I;
                const uint32_t r = flat_row % I;
                const uint64_t ex = (uint64_t)ids[e];
                const float g = moe_dot_gguf_mxfp4_row(d->gate + ex * expert_gu_bytes + r * row_h, x.data(), H);
                const float u = moe_dot_gguf_mxfp4_row(d->up + ex * expert_gu_bytes + r * row_h, x.data(), H);
                gate_pool[(uint64_t)e * I + r] = moe_generation_gated_activation_cached(activation_mode, g, u);
                return 1;
            })) return 0;
        // Phase 2b: down over k*H flat rows (:1385-1404).
        if (!moe_parallel_rows(engine, (uint32_t)(sel * H), 0, [&](uint32_t flat_row) {
                const uint32_t e = flat_row / H;
                const uint32_t r = flat_row % H;
                const uint64_t ex = (uint64_t)ids[e];
                out_pool[(uint64_t)e * H + r] = moe_dot_gguf_mxfp4_row(
                    d->down + ex * expert_d_bytes + r * row_i, gate_pool.data() + (uint64_t)e * I, I);
                return 1;
            })) return 0;
        // Phase 3: weighted combine in router order (:1417-1431).
        for (size_t e = 0; e < sel; ++e) {
            moe_axpy_f32(mlp.data(), out_pool.data() + e * H, w[e], H);
        }
        std::memcpy(y_f32 + (uint64_t)t * H, mlp.data(), (size_t)H * sizeof(float));
        if (out_ids) for (uint32_t j = 0; j < K; ++j) out_ids[(uint64_t)t * K + j] = ids[j];
        if (out_w) for (uint32_t j = 0; j < K; ++j) out_w[(uint64_t)t * K + j] = w[j];
    }
    return 1;
}

// Optional parts of Gemma-style MoE blocks around the experts.  Each is
// registered under the first tensor-name suffix the reference looks up for
// it, exactly where moe_map_layer_common_tensor (generation_mlp.cpp.inc:25-62)
// finds its cached tensors; absent parts are removed from that cache.
typedef struct {
    ref_layer_desc base;
    float eps;                     // RMSNorm epsilon (the model's rms_norm_eps)
    const float* pre_norm2;        // [H]  pre_ffw_norm_2.weight
    const float* post_norm1;       // [H]  post_ffw_norm_1.weight
    const float* post_norm2;       // [H]  post_ffw_norm_2.weight
    const float* post_norm;        // [H]  post_ffw_norm.weight
    const float* down_scale;       // [down_scale_count]  ffn_down_exps.scale
    uint64_t down_scale_count;
    const uint16_t* shared_gate_inp;  // [H] bf16  shared_expert_gate.weight
    const float* router_scale;        // [router_scale_count]  ffn_gate_inp.scale
    uint64_t router_scale_count;
} ref_block_desc;

namespace {

uint64_t common_key(int32_t layer, const char* suffix) {
    return ((uint64_t)(uint32_t)layer << 32) | moe_fnv1a_hash_string(suffix) | 0x80000000ull;
}

void put_common(moe_pc_engine* engine, int32_t layer, const char* suffix, const void* data, uint64_t count,
                uint32_t rows, uint32_t cols, uint8_t encoding, uint8_t format) {
    std::unique_lock<std::shared_mutex> lock(engine->raw_tensor_cache_mutex);
    const uint64_t key = common_key(layer, suffix);
    if (!data) {
        engine->raw_tensor_cache.erase(key);
        return;
    }
    moe_raw_tensor_cache_entry e{};
    e.base = reinterpret_cast<const uint8_t*>(data);
    e.bytes = count * (encoding == moe_RAW_SCALAR_F32 ? 4ull : 2ull);
    e.rows = rows;
    e.cols = cols;
    e.scalar_encoding = encoding;
    e.weight_format = format;
    engine->raw_tensor_cache[key] = e;
}

}  // namespace

namespace {

// The optional block parts of `bd` in this engine's tensor cache, each under
// the first suffix the reference looks it up by (absent ones removed).
void install_block_parts(moe_pc_engine* engine, int32_t layer, const ref_block_desc* bd) {
    const uint32_t H = bd->base.hidden;
    const uint8_t F32 = moe_RAW_SCALAR_F32, BF16 = moe_RAW_SCALAR_BF16;
    const uint8_t RAW_F32 = moe_WEIGHT_ENCODING_RAW_FP32, RAW_BF16 = moe_WEIGHT_ENCODING_RAW_BF16;
    put_common(engine, layer, "pre_ffw_norm_2.weight", bd->pre_norm2, H, H, 0, F32, RAW_F32);
    put_common(engine, layer, "post_ffw_norm_1.weight", bd->post_norm1, H, H, 0, F32, RAW_F32);
    put_common(engine, layer, "post_ffw_norm_2.weight", bd->post_norm2, H, H, 0, F32, RAW_F32);
    put_common(engine, layer, "post_ffw_norm.weight", bd->post_norm, H, H, 0, F32, RAW_F32);
    put_common(engine, layer, "ffn_down_exps.scale", bd->down_scale, bd->down_scale_count,
               (uint32_t)bd->down_scale_count, 0, F32, RAW_F32);
    put_common(engine, layer, "shared_expert_gate.weight", bd->shared_gate_inp, H, 1, H, BF16, RAW_BF16);
    // the router's own lookup of its input scale (moe_map_router_scale_tensor,
    // generation_router.cpp.inc:272-314) keys it with the router's hash
    const uint64_t key = router_scale_key(layer);
    std::unique_lock<std::shared_mutex> lock(engine->raw_tensor_cache_mutex);
    if (bd->router_scale && bd->router_scale_count) {
        moe_raw_tensor_cache_entry e{};
        e.base = reinterpret_cast<const uint8_t*>(bd->router_scale);
        e.bytes = bd->router_scale_count * 4ull;
        e.rows = (uint32_t)bd->router_scale_count;
        e.cols = 0;
        e.scalar_encoding = F32;
        e.weight_format = RAW_F32;
        engine->raw_tensor_cache[key] = e;
    } else {
        engine->raw_tensor_cache.erase(key);
    }
}

}  // namespace

// The MoE block for T tokens, one token at a time, composed from the
// reference's own functions in moe_layer_moe_mlp_f32's order
// (generation_mlp.cpp.inc:776-1442): the routed input is
// moe_layer_moe_norm_f32(hidden) when pre_ffw_norm_2 exists (:826-831), the
// shared expert is gated by moe_layer_shared_expert_gate_f32 and normalised
// by moe_layer_post_ffw_norm1_f32 (:849-859), each routed output goes
// through moe_layer_post_ffw_norm2_f32 and moe_layer_apply_expert_down_scale_f32
// before moe_axpy_f32 (:1417-1430), and the block output through
// moe_layer_post_ffw_norm_f32 (moe_add_mlp_residual_f32 :572-594).  The
// activation and the norms' unit offset come from the engine metadata.
// y_f32 receives what the block adds to `hidden`.
int ref_moe_block(void* eng, const ref_block_desc* bd, const uint16_t* x_bf16, const float* hidden,
                  uint32_t tokens, float* y_f32, int32_t* out_ids, float* out_w) {
    mxcsr_guard guard;
    moe_pc_engine* engine = static_cast<moe_pc_engine*>(eng);
    if (!engine || !bd || !x_bf16 || !y_f32) return 0;
    if ((bd->pre_norm2 || bd->router_scale) && !hidden) return 0;
    const ref_layer_desc* d = &bd->base;
    const uint32_t H = d->hidden, I = d->intermediate, E = d->experts, K = d->top_k;
    const int32_t layer = 0;
    const uint64_t row_h = (uint64_t)((H + 31u) / 32u) * 17u;
    const uint64_t row_i = (uint64_t)((I + 31u) / 32u) * 17u;
    const uint64_t expert_gu_bytes = (uint64_t)I * row_h;
    const uint64_t expert_d_bytes = (uint64_t)H * row_i;
    {
        moe_raw_tensor_cache_entry r{};
        r.base = reinterpret_cast<const uint8_t*>(d->router_bf16);
        r.bytes = (uint64_t)E * H * 2ull;
        r.rows = E;
        r.cols = H;
        r.scalar_encoding = moe_RAW_SCALAR_BF16;
        r.weight_format = moe_WEIGHT_ENCODING_RAW_BF16;
        std::unique_lock<std::shared_mutex> lock(engine->raw_tensor_cache_mutex);
        engine->raw_tensor_cache[router_cache_key(layer)] = r;
    }
    install_block_parts(engine, layer, bd);
    const int activation_mode = moe_engine_gelu_activation_mode(engine);
    const float eps = bd->eps;

    std::vector<float> x(H), xe(H), mlp(H), tmp(H), shared_gate(I), shared_out(H);
    std::vector<float> gate_pool((uint64_t)K * I), out_pool((uint64_t)K * H);
    std::vector<int> ids;
    std::vector<float> w, logits;
    std::vector<uint32_t> order;
    for (uint32_t t = 0; t < tokens; ++t) {
        for (uint32_t h = 0; h < H; ++h) x[h] = bf16_to_f32(x_bf16[(uint64_t)t * H + h]);
        std::fill(mlp.begin(), mlp.end(), 0.0f);
        const float* expert_input = x.data();
        if (hidden && moe_layer_moe_norm_f32(engine, layer, hidden + (uint64_t)t * H, H, xe.data(), eps)) {
            expert_input = xe.data();
        }
        if (d->shared_gate && d->shared_up && d->shared_down) {
            if (!moe_parallel_rows(engine, I, 0, [&](uint32_t row) {
                    const float g = moe_dot_gguf_mxfp4_row(d->shared_gate + row * row_h, x.data(), H);
                    const float u = moe_dot_gguf_mxfp4_row(d->shared_up + row * row_h, x.data(), H);
                    shared_gate[row] = moe_generation_gated_activation_cached(activation_mode, g, u);
                    return 1;
                })) return 0;
            if (!moe_parallel_rows(engine, H, 0, [&](uint32_t row) {
                    shared_out[row] = moe_dot_gguf_mxfp4_row(d->shared_down + row * row_i, shared_gate.data(), I);
                    return 1;
                })) return 0;
            float g = 1.0f;
            if (!moe_layer_shared_expert_gate_f32(engine, layer, x.data(), H, &g)) return 0;
            const float* so = shared_out.data();
            if (moe_layer_post_ffw_norm1_f32(engine, layer, shared_out.data(), H, tmp.data(), eps)) so = tmp.data();
            for (uint32_t i = 0; i < H; ++i) mlp[i] += so[i] * g;
        }
        // a router with its own input scale reads the residual stream
        // (generation_mlp.cpp.inc:866-871) and scales it inside
        // moe_router_topk_f32 (generation_router.cpp.inc:584-587)
        const float* router_input = bd->router_scale ? hidden + (uint64_t)t * H : expert_input;
        if (!moe_router_topk_f32(engine, layer, router_input, H, E, K, &ids, &w, &logits, &order)) return 0;
        if (ids.size() != K) return 0;
        if (!moe_parallel_rows(engine, K * I, 0, [&](uint32_t flat_row) {
                const uint32_t e = flat_row / I;
                const uint32_t r = flat_row % I;
                const uint64_t ex = (uint64_t)ids[e];
                const float g = moe_dot_gguf_mxfp4_row(d->gate + ex * expert_gu_bytes + r * row_h, expert_input, H);
                const float u = moe_dot_gguf_mxfp4_row(d->up + ex * expert_gu_bytes + r * row_h, expert_input, H);
                gate_pool[(uint64_t)e * I + r] = moe_generation_gated_activation_cached(activation_mode, g, u);
                return 1;
            })) return 0;
        if (!moe_parallel_rows(engine, K * H, 0, [&](uint32_t flat_row) {
                const uint32_t e = flat_row / H;
                const uint32_t r = flat_row % H;
                const uint64_t ex = (uint64_t)ids[e];
                out_pool[(uint64_t)e * H + r] = moe_dot_gguf_mxfp4_row(
                    d->down + ex * expert_d_bytes + r * row_i, gate_pool.data() + (uint64_t)e * I, I);
                return 1;
            })) return 0;
        for (uint32_t e = 0; e < K; ++e) {
            float* out = out_pool.data() + (uint64_t)e * H;
            if (moe_layer_post_ffw_norm2_f32(engine, layer, out, H, tmp.data(), eps)) {
                std::memcpy(out, tmp.data(), (size_t)H * sizeof(float));
            }
            if (!moe_layer_apply_expert_down_scale_f32(engine, layer, ids[e], E, out, H)) return 0;
            moe_axpy_f32(mlp.data(), out, w[e], H);
        }
        float* yt = y_f32 + (uint64_t)t * H;
        if (!moe_layer_post_ffw_norm_f32(engine, layer, mlp.data(), H, yt, eps)) {
            std::memcpy(yt, mlp.data(), (size_t)H * sizeof(float));
        }
        if (out_ids) for (uint32_t j = 0; j < K; ++j) out_ids[(uint64_t)t * K + j] = ids[j];
        if (out_w) for (uint32_t j = 0; j < K; ++j) out_w[(uint64_t)t * K + j] = w[j];
    }
    return 1;
}

// The reference's gated activation for an explicit mode
// (generation_mlp.cpp.inc:99-104) and RMSNorm with a weight vector
// (moe_apply_rmsnorm_common_weight_f32 :145-175; the unit offset follows
// the engine's metadata), for direct known-answer tables.
float ref_gated_activation(int32_t mode, float gate, float up) {
    mxcsr_guard guard;
    return moe_generation_gated_activation_cached(mode, gate, up);
}

int ref_rmsnorm(void* eng, const float* w, uint32_t n, const float* in, float eps, float* out) {
    mxcsr_guard guard;
    moe_pc_engine* engine = static_cast<moe_pc_engine*>(eng);
    moe_raw_tensor_cache_entry e{};
    e.base = reinterpret_cast<const uint8_t*>(w);
    e.bytes = (uint64_t)n * 4ull;
    e.rows = n;
    e.cols = 0;
    e.scalar_encoding = moe_RAW_SCALAR_F32;
    e.weight_format = moe_WEIGHT_ENCODING_RAW_FP32;
    return moe_apply_rmsnorm_common_weight_f32(engine, e, in, n, out, eps);
}

// The reference's public grouping utility (token_grouping.cpp.inc:1-83) is
// already extern "C" (moe_pc_group_tokens_by_expert); this alias keeps the
// oracle's symbols in one namespace.
int ref_group_tokens_by_expert(const moe_token_expert_assignment_t* a, uint32_t n,
                               moe_token_expert_assignment_t* sorted,
                               moe_expert_batch_t* batches, uint32_t max_batches,
                               uint32_t* batch_count) {
    return moe_pc_group_tokens_by_expert(a, n, sorted, batches, max_batches, batch_count);
}

// The layer through moe_layer_moe_mlp_f32 itself (generation_mlp.cpp.inc:
// 776-1442), one call per token as the engine makes it
// (generation_forward.cpp.inc:212-215).  The experts become tensor records
// the way the codec table makes them: their GGUF MXFP4 bytes are written to
// `shard_path` (gate, up, down of expert 0, then expert 1, ...), each
// projection gets a moe_tensor_record over its byte range finished by the
// reference's finalize_tensor_layout with the MXFP4 encoding, and
// tensor_slots_set files it under (layer 0, expert, projection); the layer
// function then finds, maps and decodes them through find_tensor_record,
// get_or_map_tensor_shard and moe_dot_tensor_record_row.  The shared expert
// is the layer's dense MLP (ffn_gate/ffn_up/ffn_down.weight as MXFP4 tensors,
// which moe_layer_common_dense_mlp_f32 finds first, :596-727, 833-860), the
// router as in ref_moe_layer.  The engine's residency bookkeeping (expert
// states, which the prefetch and heat updates consult) is emptied, so the
// call computes without tier moves; the phase is prefill (no speculative
// prefetch).  Input: s->norm = the token's row; hidden = 0, so the residual
// add leaves hidden = mlp; y_f32 receives s->mlp, ids and w the router's
// selection.  Without `bd` (the plain layer) any block parts a
// ref_moe_block call left in the engine are removed first; with it, they are
// installed and `hidden_in` is the residual stream (ref_moe_block_engine).
static int run_layer_function(moe_pc_engine* engine, const ref_layer_desc* d, const ref_block_desc* bd,
                              const uint16_t* x_bf16, const float* hidden_in, uint32_t tokens, float* y_f32,
                              int32_t* out_ids, float* out_w, const char* shard_path,
                              const uint8_t* present = nullptr) {
    if (!engine || !d || !x_bf16 || !y_f32 || !shard_path) return 0;
    if (bd && (bd->pre_norm2 || bd->router_scale) && !hidden_in) return 0;
    const uint32_t H = d->hidden, I = d->intermediate, E = d->experts, K = d->top_k;
    const int32_t layer = 0;
    const uint64_t row_h = (uint64_t)((H + 31u) / 32u) * 17u;
    const uint64_t row_i = (uint64_t)((I + 31u) / 32u) * 17u;
    const uint64_t gu_bytes = (uint64_t)I * row_h, dn_bytes = (uint64_t)H * row_i;

    // the shard file: [expert][gate, up, down]
    {
        FILE* f = std::fopen(shard_path, "wb");
        if (!f) return 0;
        bool ok = true;
        for (uint32_t e = 0; e < E && ok; ++e) {
            ok = std::fwrite(d->gate + (uint64_t)e * gu_bytes, 1, gu_bytes, f) == gu_bytes &&
                 std::fwrite(d->up + (uint64_t)e * gu_bytes, 1, gu_bytes, f) == gu_bytes &&
                 std::fwrite(d->down + (uint64_t)e * dn_bytes, 1, dn_bytes, f) == dn_bytes;
        }
        ok = std::fclose(f) == 0 && ok;
        if (!ok) return 0;
    }
    // a shard number of its own per call (past the fast-slot cache), so a
    // mapping of an earlier call's file is never reused
    static std::atomic<uint32_t> next_shard{moe_SOURCE_MMAP_FAST_SLOTS + 1u};
    const uint32_t shard = next_shard.fetch_add(1u);
    engine->tensor_paths.push_back(shard_path);
    const uint16_t path_index = (uint16_t)(engine->tensor_paths.size() - 1u);
    tensor_slots_reset(engine);
    const moe_projection_t projs[3] = {moe_PROJ_GATE, moe_PROJ_UP, moe_PROJ_DOWN};
    uint64_t offset = 0;
    for (uint32_t e = 0; e < E; ++e) {
        for (int p = 0; p < 3; ++p) {
            const bool down = projs[p] == moe_PROJ_DOWN;
            moe_tensor_record rec{};
            rec.info.weight_byte_offset = offset;
            rec.info.weight_byte_length = down ? dn_bytes : gu_bytes;
            rec.info.part = 0;
            rec.info.shard = shard;
            rec.info.layer = (uint32_t)layer;
            rec.info.expert = e;
            rec.info.proj = projs[p];
            rec.info.rows = down ? H : I;
            rec.info.cols = down ? I : H;
            rec.info.groups = (rec.info.cols + 31u) / 32u;
            rec.info.group_size = 32u;
            rec.resolved_path_index = path_index;
            finalize_tensor_layout(&rec, moe_WEIGHT_ENCODING_MXFP4);
            engine->tensors.push_back(rec);
            // a missing expert has no record: the layer's partial-failure path
            if (!present || present[e]) tensor_slots_set(engine, layer, (int)e, projs[p], engine->tensors.size() - 1u);
            offset += rec.info.weight_byte_length;
        }
    }

    // router, and the shared expert as the layer's dense MLP
    if (!bd) clear_router_scale(engine, layer);
    {
        moe_raw_tensor_cache_entry r{};
        r.base = reinterpret_cast<const uint8_t*>(d->router_bf16);
        r.bytes = (uint64_t)E * H * 2ull;
        r.rows = E;
        r.cols = H;
        r.scalar_encoding = moe_RAW_SCALAR_BF16;
        r.weight_format = moe_WEIGHT_ENCODING_RAW_BF16;
        std::unique_lock<std::shared_mutex> lock(engine->raw_tensor_cache_mutex);
        engine->raw_tensor_cache[router_cache_key(layer)] = r;
    }
    {
        // whether the router reads the residual stream is decided from the
        // model's tensor names (moe_engine_has_common_tensor_suffix, which
        // also remembers its answers): name the scale tensor exactly when the
        // block has one.  Its slot is out of range, so a lookup of the tensor
        // itself still finds the cached copy installed below.
        const std::string scale_name = "blk." + std::to_string(layer) + ".ffn_gate_inp.scale";
        if (bd && bd->router_scale && bd->router_scale_count) {
            engine->gguf_common_tensor_slots[scale_name] = SIZE_MAX;
        } else {
            engine->gguf_common_tensor_slots.erase(scale_name);
        }
        std::unique_lock<std::shared_mutex> lock(engine->common_tensor_suffix_cache_mutex);
        engine->common_tensor_suffix_cache.clear();
    }
    if (bd) {
        install_block_parts(engine, layer, bd);
        // the layer function takes its RMSNorm epsilon from the model's config
        moe_attn_config_t acfg = moe_generation_attn_config(engine);
        acfg.rms_norm_eps = bd->eps;
        engine->attn_config = acfg;
        engine->attn_config_valid.store(true, std::memory_order_release);
    } else {
        const char* block_parts[] = {"pre_ffw_norm_2.weight", "post_ffw_norm_1.weight", "post_ffw_norm_2.weight",
                                     "post_ffw_norm.weight", "ffn_down_exps.scale", "shared_expert_gate.weight"};
        for (const char* sfx : block_parts) put_common(engine, layer, sfx, nullptr, 0, 0, 0, 0, 0);
    }
    const bool shared = d->shared_gate && d->shared_up && d->shared_down && (!present || present[E]);
    struct {
        const char* suffix;
        const uint8_t* data;
        uint32_t rows, cols;
    } dense[3] = {{"ffn_gate.weight", d->shared_gate, I, H},
                  {"ffn_up.weight", d->shared_up, I, H},
                  {"ffn_down.weight", d->shared_down, H, I}};
    for (const auto& t : dense) {
        std::unique_lock<std::shared_mutex> lock(engine->raw_tensor_cache_mutex);
        const uint64_t key = common_key(layer, t.suffix);
        if (!shared) {
            engine->raw_tensor_cache.erase(key);
            continue;
        }
        moe_raw_tensor_cache_entry e{};
        e.base = t.data;
        e.weight_row_bytes = (uint64_t)((t.cols + 31u) / 32u) * 17u;
        e.bytes = (uint64_t)t.rows * e.weight_row_bytes;
        e.rows = t.rows;
        e.cols = t.cols;
        e.scalar_encoding = moe_RAW_SCALAR_UNKNOWN;
        e.weight_format = moe_WEIGHT_ENCODING_MXFP4;
        engine->raw_tensor_cache[key] = e;
    }

    {
        std::lock_guard<std::mutex> lock(engine->map_mutex);
        engine->expert_states.clear();
    }
    engine->generation_phase.store(moe_GEN_PHASE_PREFILL, std::memory_order_release);
    moe_storage_constants_t c = moe_engine_storage_constants_or_static(engine);
    c.hidden_size = H;
    c.expert_intermediate_size = I;
    c.experts_per_moe_layer = E;
    c.first_moe_layer = 0;
    c.last_moe_layer = 0;

    moe_decode_scratch s;
    s.mlp.resize(H);
    s.shared.resize(H);
    s.expert.resize(H);
    s.norm.resize(H);
    s.residual.resize(H);
    s.gate.resize(I);
    s.up.resize(I);
    s.expert_work.resize(K);
    std::vector<float> hidden(H);
    // what the layer adds to hidden: the final post-FFW norm's output when
    // the block has one (moe_add_mlp_residual_f32 leaves it in s.shared), else mlp
    const std::vector<float>& added = (bd && bd->post_norm) ? s.shared : s.mlp;
    for (uint32_t t = 0; t < tokens; ++t) {
        for (uint32_t h = 0; h < H; ++h) s.norm[h] = bf16_to_f32(x_bf16[(uint64_t)t * H + h]);
        if (hidden_in) {
            std::memcpy(hidden.data(), hidden_in + (uint64_t)t * H, (size_t)H * sizeof(float));
        } else {
            std::fill(hidden.begin(), hidden.end(), 0.0f);
        }
        if (!moe_layer_moe_mlp_f32(engine, layer, &s, hidden.data(), &c)) return 0;
        if (s.selected_experts.size() != K || s.selected_weights.size() != K) return 0;
        std::memcpy(y_f32 + (uint64_t)t * H, added.data(), (size_t)H * sizeof(float));
        if (out_ids) for (uint32_t j = 0; j < K; ++j) out_ids[(uint64_t)t * K + j] = s.selected_experts[j];
        if (out_w) for (uint32_t j = 0; j < K; ++j) out_w[(uint64_t)t * K + j] = s.selected_weights[j];
    }
    return 1;
}

int ref_moe_layer_engine(void* eng, const ref_layer_desc* d, const uint16_t* x_bf16, uint32_t tokens,
                         float* y_f32, int32_t* out_ids, float* out_w, const char* shard_path) {
    mxcsr_guard guard;
    return run_layer_function(static_cast<moe_pc_engine*>(eng), d, nullptr, x_bf16, nullptr, tokens, y_f32, out_ids,
                              out_w, shard_path);
}

// The same with some experts missing: present[e] == 0 (e < E) files no
// records for routed expert e, present[E] == 0 leaves the shared expert out,
// so the layer function takes its partial-failure path
// (generation_mlp.cpp.inc:1219-1282, 833-860).
int ref_moe_layer_engine_present(void* eng, const ref_layer_desc* d, const uint16_t* x_bf16, uint32_t tokens,
                                 float* y_f32, int32_t* out_ids, float* out_w, const char* shard_path,
                                 const uint8_t* present) {
    mxcsr_guard guard;
    return run_layer_function(static_cast<moe_pc_engine*>(eng), d, nullptr, x_bf16, nullptr, tokens, y_f32, out_ids,
                              out_w, shard_path, present);
}

// The same with the Gemma-style block parts of `bd` (ref_moe_block's inputs:
// x the normalised row the shared expert reads, hidden the fp32 residual
// stream the pre-norm and a scaled router read); y receives what the block
// adds to hidden.  The engine's metadata must carry the block's activation
// and unit offset, as for ref_moe_block; its RMSNorm epsilon is set here.
int ref_moe_block_engine(void* eng, const ref_block_desc* bd, const uint16_t* x_bf16, const float* hidden,
                         uint32_t tokens, float* y_f32, int32_t* out_ids, float* out_w, const char* shard_path) {
    mxcsr_guard guard;
    if (!bd) return 0;
    return run_layer_function(static_cast<moe_pc_engine*>(eng), &bd->base, bd, x_bf16, hidden, tokens, y_f32,
                              out_ids, out_w, shard_path);
}

}  // extern "C"
