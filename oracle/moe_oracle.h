/* TEST INFRASTRUCTURE ONLY -- the CPU checker for the CUDA path, never the
 * product.  Plain-C restatement of the reference's MoE expert-FFN hot path
 * (jujumelona/storage.llm, moe_engine).  Only tests/, the smoke check and the
 * bench's CPU-baseline / reference arms load it. */
#ifndef MOE_ORACLE_H
#define MOE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    uint32_t token_index;
    uint32_t layer;
    uint32_t expert;
    float router_score;
} mo_assignment_t;  /* = moe_token_expert_assignment_t (moe_tensor_types.h.inc:62-67) */

typedef struct {
    uint32_t layer;
    uint32_t expert;
    uint32_t first_sorted_index;
    uint32_t token_count;
} mo_batch_t;       /* = moe_expert_batch_t (moe_tensor_types.h.inc:69-74) */

typedef struct {
    uint32_t hidden, intermediate, experts, top_k;
    int32_t score_sigmoid;   /* 0 softmax (default), 1 sigmoid */
    int32_t norm_topk;       /* renormalise the k weights */
    float routed_scale;      /* sigmoid only; 1.0 = none */
    const uint16_t* router_bf16;   /* [E x H] */
    const uint8_t* gate;           /* [E][I][ceil(H/32)*17] GGUF MXFP4 */
    const uint8_t* up;
    const uint8_t* down;           /* [E][H][ceil(I/32)*17] */
    const uint8_t* shared_gate;    /* optional always-on expert */
    const uint8_t* shared_up;
    const uint8_t* shared_down;
    uint32_t n_group;        /* group limit of sigmoid routers: groups ... */
    uint32_t topk_group;     /* ... of which this many keep their scores; 0 = none */
    /* Optional parts of Gemma-style MoE blocks around the experts; zero /
     * NULL = absent, which is the plain layer above. */
    int32_t activation;      /* 0 SiLU, 1 GELU (erf), 2 GELU (tanh form) */
    int32_t norm_unit_offset;      /* RMSNorm multiplies by (1 + w) instead of w */
    float norm_eps;                /* RMSNorm epsilon; <= 0 means 1e-6 */
    const float* pre_norm2;        /* [H] routed experts and router read RMSNorm(hidden) */
    const float* post_norm1;       /* [H] RMSNorm of the shared expert's output */
    const float* post_norm2;       /* [H] RMSNorm of each routed expert's output */
    const float* post_norm;        /* [H] RMSNorm of the block output */
    const float* down_scale;       /* 1 (all experts), E (per expert) or E*H (per element) */
    uint64_t down_scale_count;
    const uint16_t* shared_gate_inp;  /* [H] bf16: shared expert x sigmoid(row . x) */
    /* Router input scale (ffn_gate_inp.scale): the router then reads
     * hidden * rms^-1 * scale / sqrt(H) of the residual stream (needs hidden). */
    const float* router_scale;     /* 1 (one for all elements) or H values */
    uint64_t router_scale_count;
    /* Experts the layer cannot use (generation_mlp.cpp.inc:1219-1282): E + 1
     * bytes, 0 = missing, the last one the shared expert; NULL = all present.
     * A missing routed expert is left out and, when the router renormalises
     * its top-k, the others' combine weights are divided by their sum; a
     * token whose experts are all missing fails, as the reference's layer
     * does.  The router's ids and weights themselves are unchanged. */
    const uint8_t* present;
} mo_layer_t;

float mo_e8m0_to_f32(uint8_t v);
float mo_mxfp4_value(uint8_t code);
float mo_mxfp4_dot_row(const uint8_t* packed, const float* x, uint32_t cols);
float mo_bf16_dot_row(const uint16_t* w, const float* x, uint32_t cols);
float mo_silu(float x);
float mo_gated_activation(int32_t mode, float gate, float up);
int mo_rmsnorm(const float* in, const float* w, uint32_t n, float eps, int32_t unit_offset, float* out);
void mo_router_scores(const mo_layer_t* L, const float* x, float* scores);
int mo_router_topk(const mo_layer_t* L, const float* x, int32_t* ids, float* w, uint32_t* ties);
int mo_group_tokens_by_expert(const mo_assignment_t* a, uint32_t n, mo_assignment_t* sorted,
                              mo_batch_t* batches, uint32_t max_batches, uint32_t* batch_count);
int mo_expert_triplet(const uint8_t* gate, const uint8_t* up, const uint8_t* down,
                      const float* x, uint32_t hidden, uint32_t intermediate,
                      float* scratch_gate, float* scratch_up, float* out);
int mo_moe_layer(const mo_layer_t* L, const uint16_t* x_bf16, uint32_t tokens,
                 float* y, int32_t* ids, float* w, uint32_t threads, uint32_t* ties);
/* The layer with the residual stream `hidden` [T x H] beside its normed
 * form x (needed only with pre_norm2); y = what the block adds to hidden. */
int mo_moe_block(const mo_layer_t* L, const uint16_t* x_bf16, const float* hidden, uint32_t tokens,
                 float* y, int32_t* ids, float* w, uint32_t threads, uint32_t* ties);

#ifdef __cplusplus
}
#endif
#endif
