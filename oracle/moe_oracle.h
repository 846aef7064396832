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
} mo_layer_t;

float mo_e8m0_to_f32(uint8_t v);
float mo_mxfp4_value(uint8_t code);
float mo_mxfp4_dot_row(const uint8_t* packed, const float* x, uint32_t cols);
float mo_bf16_dot_row(const uint16_t* w, const float* x, uint32_t cols);
float mo_silu(float x);
void mo_router_scores(const mo_layer_t* L, const float* x, float* scores);
int mo_router_topk(const mo_layer_t* L, const float* x, int32_t* ids, float* w, uint32_t* ties);
int mo_group_tokens_by_expert(const mo_assignment_t* a, uint32_t n, mo_assignment_t* sorted,
                              mo_batch_t* batches, uint32_t max_batches, uint32_t* batch_count);
int mo_expert_triplet(const uint8_t* gate, const uint8_t* up, const uint8_t* down,
                      const float* x, uint32_t hidden, uint32_t intermediate,
                      float* scratch_gate, float* scratch_up, float* out);
int mo_moe_layer(const mo_layer_t* L, const uint16_t* x_bf16, uint32_t tokens,
                 float* y, int32_t* ids, float* w, uint32_t threads, uint32_t* ties);

#ifdef __cplusplus
}
#endif
#endif
