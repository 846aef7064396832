/* TEST INFRASTRUCTURE ONLY -- never part of the shipped product path.
 *
 * Plain-C restatement of the reference's MoE expert-FFN hot path
 * (jujumelona/storage.llm, moe_engine/src/parts).  It is the checker the
 * CUDA kernels are compared against, and the "port" CPU baseline.  Every
 * function cites the reference code it follows.  Floating-point operations
 * are spelled out in the order the reference's x86 build (AVX2 + FMA,
 * -O3, GCC's default fp-contract) evaluates them, so results are bit-exact
 * against oracle/_ref/libmoe_ref.so on the same host; that is checked by
 * tests/test_oracle.py.  This file is compiled with -ffp-contract=off so the
 * fmaf() calls below are the only fused operations.
 */
#include "moe_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* E8M0 scale -> float: v>0 -> 2^(v-127) (v=255 gives +inf), v=0 -> 2^-127.
 * tensor_dot_cpu_kernels.cpp.inc:576-581 */
float mo_e8m0_to_f32(uint8_t v) {
    uint32_t bits = v ? ((uint32_t)v << 23) : 0x00400000u;
    float out;
    memcpy(&out, &bits, sizeof(out));
    return out;
}

/* OCP E2M1 code table, tensor_dot_cpu_kernels.cpp.inc:583-589. */
static const float kE2M1[16] = {
    0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
    -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f,
};

float mo_mxfp4_value(uint8_t code) { return kE2M1[code & 0x0f]; }

/* Element i of a 32-element block: low nibble of qs[i] for i<16, high nibble
 * of qs[i-16] otherwise.  tensor_dot_cpu_kernels.cpp.inc:595-599 */
static uint8_t mo_code_at(const uint8_t* qs, uint32_t i) {
    return i < 16u ? (qs[i] & 0x0f) : (qs[i - 16u] >> 4);
}

/* _mm256 horizontal sum as the reference does it (moe_dot_hsum256_ps,
 * tensor_dot_cpu_kernels.cpp.inc:252-259): lanes i and i+4 are added, then two
 * hadd steps give (a0+a1)+(a2+a3). */
static float mo_hsum8(const float v[8]) {
    float a0 = v[0] + v[4], a1 = v[1] + v[5], a2 = v[2] + v[6], a3 = v[3] + v[7];
    return (a0 + a1) + (a2 + a3);
}

/* MXFP4 row dot, AVX2+FMA branch of moe_dot_gguf_mxfp4_row
 * (tensor_dot_cpu_kernels.cpp.inc:601-667): per full block two 8-lane FMA
 * accumulators (low nibbles x x[0..15], high nibbles x x[16..31]) over two
 * 8-element steps, horizontal sums, then acc += (low + high) * scale (fused
 * by the compiler); a ragged last block accumulates serially without fusion
 * (the compiled reference keeps that loop's multiply and add separate). */
float mo_mxfp4_dot_row(const uint8_t* packed, const float* x, uint32_t cols) {
    float acc = 0.0f;
    uint32_t start = 0;
    const uint32_t full = cols & ~31u;
    for (; start < full; start += 32u) {
        const float scale = mo_e8m0_to_f32(packed[0]);
        const uint8_t* qs = packed + 1;
        const float* xb = x + start;
        float lo[8] = {0}, hi[8] = {0};
        for (uint32_t j = 0; j < 16u; j += 8u) {
            for (uint32_t l = 0; l < 8u; ++l) {
                const uint8_t b = qs[j + l];
                lo[l] = fmaf(kE2M1[b & 0x0f], xb[j + l], lo[l]);
                hi[l] = fmaf(kE2M1[b >> 4], xb[j + l + 16u], hi[l]);
            }
        }
        const float low = mo_hsum8(lo);
        const float high = mo_hsum8(hi);
        acc = fmaf(low + high, scale, acc);
        packed += 17;
    }
    if (start < cols) {
        const float scale = mo_e8m0_to_f32(packed[0]);
        const uint8_t* qs = packed + 1;
        const uint32_t limit = cols - start;
        float block_acc = 0.0f;
        for (uint32_t i = 0; i < limit; ++i) {
            block_acc = block_acc + kE2M1[mo_code_at(qs, i)] * x[start + i];
        }
        acc = fmaf(block_acc, scale, acc);
    }
    return acc;
}

static float mo_bf16(uint16_t v) {
    uint32_t bits = (uint32_t)v << 16;
    float f;
    memcpy(&f, &bits, sizeof(f));
    return f;
}

/* bf16 router row dot, AVX2 branch of moe_dot_bf16_row
 * (raw_forward_utils.cpp.inc:174-216): 16-element steps into two 8-lane FMA
 * accumulators, lane-wise sum0+sum1, left-to-right sum of the 8 lanes, then
 * a 4-way tail and a scalar tail. */
float mo_bf16_dot_row(const uint16_t* w, const float* x, uint32_t n) {
    uint32_t i = 0;
    float acc = 0.0f;
    float s0[8] = {0}, s1[8] = {0};
    for (; i + 15u < n; i += 16u) {
        for (uint32_t l = 0; l < 8u; ++l) {
            s0[l] = fmaf(mo_bf16(w[i + l]), x[i + l], s0[l]);
            s1[l] = fmaf(mo_bf16(w[i + 8u + l]), x[i + 8u + l], s1[l]);
        }
    }
    {
        float b[8];
        for (uint32_t l = 0; l < 8u; ++l) b[l] = s0[l] + s1[l];
        float s = b[0];
        for (uint32_t l = 1; l < 8u; ++l) s = s + b[l];
        acc = acc + s;
    }
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    for (; i + 3u < n; i += 4u) {
        a0 = fmaf(mo_bf16(w[i + 0u]), x[i + 0u], a0);
        a1 = fmaf(mo_bf16(w[i + 1u]), x[i + 1u], a1);
        a2 = fmaf(mo_bf16(w[i + 2u]), x[i + 2u], a2);
        a3 = fmaf(mo_bf16(w[i + 3u]), x[i + 3u], a3);
    }
    acc = acc + ((a0 + a1) + (a2 + a3));
    for (; i < n; ++i) acc = fmaf(mo_bf16(w[i]), x[i], acc);
    return acc;
}

/* x / (1 + exp(-x)) with the exact libm exp: generation_silu.cpp.inc:20-26. */
float mo_silu(float x) { return x / (1.0f + expf(-x)); }

/* GELU, erf form: 0.5 x (1 + erf(x / sqrt 2)) (generation_silu.cpp.inc:28-30). */
static float mo_gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f)); }

/* GELU, tanh form (generation_mlp.cpp.inc:94-97).  The reference's build
 * fuses x + 0.044715 x^3 into one multiply-add on the last product. */
static float mo_gelu_tanh(float x) {
    const float k = 0.7978845608028654f;
    return 0.5f * x * (1.0f + tanhf(k * fmaf(0.044715f * x * x, x, x)));
}

/* act(gate) * up for activation mode 0 SiLU, 1 GELU (erf), 2 GELU (tanh)
 * (moe_generation_gated_activation_cached, generation_mlp.cpp.inc:99-104). */
float mo_gated_activation(int32_t mode, float gate, float up) {
    if (mode == 2) return mo_gelu_tanh(gate) * up;
    return (mode == 1 ? mo_gelu_erf(gate) : mo_silu(gate)) * up;
}

/* RMSNorm with a weight vector (moe_apply_rmsnorm_common_weight_f32,
 * generation_mlp.cpp.inc:145-175): the sum of squares in double, in element
 * order (the reference's build fuses each step into a double multiply-add),
 * the mean rounded to float, 1 / sqrt(mean + eps) in float, then
 * x * norm * w -- or x * norm * (1 + w) for Gemma models (the unit offset,
 * raw_forward_utils.cpp.inc:322-328).  eps <= 0 means 1e-6. */
int mo_rmsnorm(const float* in, const float* w, uint32_t n, float eps, int32_t unit_offset, float* out) {
    if (!in || !w || !out || n == 0) return 0;
    double ss = 0.0;
    for (uint32_t i = 0; i < n; ++i) ss = fma((double)in[i], (double)in[i], ss);
    const float norm = 1.0f / sqrtf((float)(ss / (double)n) + (eps > 0.0f ? eps : 1.0e-6f));
    for (uint32_t i = 0; i < n; ++i) out[i] = in[i] * norm * (unit_offset ? (1.0f + w[i]) : w[i]);
    return 1;
}

/* Group limit of sigmoid routers (generation_router.cpp.inc:484-558),
 * applied when n_group > 1, 0 < topk_group < n_group and E % n_group == 0:
 * each group's score is the sum of its two largest scores (best0/best1
 * updated from 0 in expert order; the largest alone for one expert per
 * group), the topk_group best groups keep their scores and the other groups'
 * scores become 0.  The reference picks the groups with std::nth_element,
 * whose order among equal group scores is unspecified; this restatement
 * takes the lower group index first and counts such ties in *ties. */
static void mo_group_limit(const mo_layer_t* L, float* p, uint32_t* ties) {
    const uint32_t E = L->experts, G = L->n_group, TG = L->topk_group;
    if (G <= 1 || TG == 0 || TG >= G || E % G != 0) return;
    const uint32_t epg = E / G;
    float* gs = (float*)malloc(sizeof(float) * G);
    unsigned char* keep = (unsigned char*)calloc(G, 1);
    if (!gs || !keep) { free(gs); free(keep); return; }
    for (uint32_t g = 0; g < G; ++g) {
        float b0 = 0.0f, b1 = 0.0f;
        for (uint32_t e = g * epg; e < (g + 1) * epg; ++e) {
            const float v = p[e];
            if (v > b0) { b1 = b0; b0 = v; } else if (v > b1) { b1 = v; }
        }
        gs[g] = epg > 1 ? b0 + b1 : b0;
    }
    for (uint32_t j = 0; j < TG; ++j) {
        int32_t best = -1;
        for (uint32_t g = 0; g < G; ++g)
            if (!keep[g] && (best < 0 || gs[g] > gs[best])) best = (int32_t)g;
        keep[best] = 1;
    }
    if (ties) {
        for (uint32_t g = 0; g < G; ++g) {
            if (!keep[g]) continue;
            for (uint32_t h = 0; h < G; ++h)
                if (!keep[h] && gs[h] == gs[g]) { ++*ties; break; }
        }
    }
    for (uint32_t g = 0; g < G; ++g)
        if (!keep[g])
            for (uint32_t e = g * epg; e < (g + 1) * epg; ++e) p[e] = 0.0f;
    free(gs);
    free(keep);
}

/* Router scores (generation_router.cpp.inc:188-237, 587-623): logits by the
 * bf16 row dot, then softmax with exp in double, the denominator summed in
 * double in expert order, and each score multiplied by (float)(1/denom); or
 * sigmoid 1/(1+exp(-l)) in float (:239-245) followed by the group limit. */
/* Scaled router input (moe_prepare_scaled_router_input_f32,
 * generation_router.cpp.inc:316-359), used when the layer has an
 * ffn_gate_inp.scale tensor: x * norm * scale * (1 / sqrt(H)) with norm =
 * 1 / sqrt(mean(x^2) + 1e-6) (sum of squares in double, fused as in the
 * reference's build), one scale for every element or one per element; any
 * other count scales by 1. */
static void mo_scaled_router_input(const mo_layer_t* L, const float* x, float* out) {
    const uint32_t H = L->hidden;
    double ss = 0.0;
    for (uint32_t i = 0; i < H; ++i) ss = fma((double)x[i], (double)x[i], ss);
    const float norm = 1.0f / sqrtf((float)(ss / (double)H) + 1.0e-6f);
    const float inv_sqrt_hidden = 1.0f / sqrtf((float)H);
    for (uint32_t i = 0; i < H; ++i) {
        float scale = 1.0f;
        if (L->router_scale_count == 1u) scale = L->router_scale[0];
        else if (L->router_scale_count >= H) scale = L->router_scale[i];
        out[i] = x[i] * norm * scale * inv_sqrt_hidden;
    }
}

static void mo_router_scores_t(const mo_layer_t* L, const float* x, float* p, uint32_t* ties) {
    const uint32_t E = L->experts, H = L->hidden;
    float* xs = NULL;
    if (L->router_scale && L->router_scale_count) {
        xs = (float*)malloc(sizeof(float) * H);
        if (xs) {
            mo_scaled_router_input(L, x, xs);
            x = xs;
        }
    }
    for (uint32_t e = 0; e < E; ++e) p[e] = mo_bf16_dot_row(L->router_bf16 + (uint64_t)e * H, x, H);
    free(xs);
    if (L->score_sigmoid) {
        for (uint32_t e = 0; e < E; ++e) p[e] = 1.0f / (1.0f + expf(-p[e]));
        mo_group_limit(L, p, ties);
        return;
    }
    float mx = -INFINITY;
    for (uint32_t e = 0; e < E; ++e) if (p[e] > mx) mx = p[e];
    double denom = 0.0;
    for (uint32_t e = 0; e < E; ++e) {
        p[e] = (float)exp((double)p[e] - (double)mx);
        denom += (double)p[e];
    }
    const float inv = (float)(1.0 / denom);
    for (uint32_t e = 0; e < E; ++e) p[e] *= inv;
}

void mo_router_scores(const mo_layer_t* L, const float* x, float* p) { mo_router_scores_t(L, x, p, NULL); }

/* Top-k of the router scores (generation_router.cpp.inc:640-674): the k
 * largest scores in descending order.  The reference uses
 * std::nth_element + std::sort, whose order among exactly equal scores is
 * unspecified; this restatement and the CUDA kernel both put the lower
 * expert index first, and `ties` counts how often a tie touched the
 * selection so callers can assert it never happened.  Weights are the raw
 * scores, divided by their float sum when norm_topk is set (:655-668), and
 * multiplied by routed_scale for sigmoid routers (:669-674). */
int mo_router_topk(const mo_layer_t* L, const float* x, int32_t* ids, float* w, uint32_t* ties) {
    const uint32_t E = L->experts;
    uint32_t K = L->top_k < E ? L->top_k : E;
    float* p = (float*)malloc(sizeof(float) * E);
    unsigned char* taken = (unsigned char*)calloc(E, 1);
    if (!p || !taken) { free(p); free(taken); return 0; }
    mo_router_scores_t(L, x, p, ties);
    for (uint32_t j = 0; j < K; ++j) {
        int32_t best = -1;
        for (uint32_t e = 0; e < E; ++e) {
            if (taken[e]) continue;
            if (best < 0 || p[e] > p[best]) best = (int32_t)e;
        }
        if (best < 0) break;
        taken[best] = 1;
        ids[j] = best;
        w[j] = p[best];
    }
    if (ties) {
        /* a tie matters when an unselected score equals a selected one, or
         * two selected scores are equal */
        for (uint32_t j = 0; j < K; ++j) {
            for (uint32_t e = 0; e < E; ++e) {
                if ((uint32_t)ids[j] != e && p[e] == w[j]) { ++*ties; break; }
            }
        }
    }
    float denom = 0.0f;
    for (uint32_t j = 0; j < K; ++j) denom += w[j];
    if (L->norm_topk) {
        if (denom <= 0.0f) denom = 1e-8f;
        for (uint32_t j = 0; j < K; ++j) w[j] /= denom;
    }
    const float scale = L->score_sigmoid ? L->routed_scale : 1.0f;
    if (scale != 1.0f) for (uint32_t j = 0; j < K; ++j) w[j] *= scale;
    free(p);
    free(taken);
    return 1;
}

/* Sort (layer, expert, token_index) and emit contiguous batches:
 * token_grouping.cpp.inc:1-83.  Insertion into a merge sort keeps it O(n log n);
 * the key is total so stability does not matter. */
static int mo_assign_less(const mo_assignment_t* a, const mo_assignment_t* b) {
    if (a->layer != b->layer) return a->layer < b->layer;
    if (a->expert != b->expert) return a->expert < b->expert;
    return a->token_index < b->token_index;
}

static void mo_merge_sort(mo_assignment_t* v, mo_assignment_t* tmp, uint32_t n) {
    if (n < 2) return;
    const uint32_t h = n / 2;
    mo_merge_sort(v, tmp, h);
    mo_merge_sort(v + h, tmp, n - h);
    uint32_t i = 0, j = h, o = 0;
    while (i < h && j < n) tmp[o++] = mo_assign_less(&v[j], &v[i]) ? v[j++] : v[i++];
    while (i < h) tmp[o++] = v[i++];
    while (j < n) tmp[o++] = v[j++];
    memcpy(v, tmp, sizeof(*v) * n);
}

int mo_group_tokens_by_expert(const mo_assignment_t* a, uint32_t n, mo_assignment_t* sorted,
                              mo_batch_t* batches, uint32_t max_batches, uint32_t* batch_count) {
    if (!a || n == 0 || !batch_count) {
        if (batch_count) *batch_count = 0;
        return 0;
    }
    mo_assignment_t* buf = sorted ? sorted : (mo_assignment_t*)malloc(sizeof(*buf) * n);
    mo_assignment_t* tmp = (mo_assignment_t*)malloc(sizeof(*tmp) * n);
    if (!buf || !tmp) { if (!sorted) free(buf); free(tmp); return 0; }
    memcpy(buf, a, sizeof(*buf) * n);
    mo_merge_sort(buf, tmp, n);
    uint32_t count = 0, start = 0;
    while (start < n) {
        uint32_t end = start + 1;
        while (end < n && buf[end].layer == buf[start].layer && buf[end].expert == buf[start].expert) ++end;
        if (batches && count < max_batches) {
            batches[count].layer = buf[start].layer;
            batches[count].expert = buf[start].expert;
            batches[count].first_sorted_index = start;
            batches[count].token_count = end - start;
        }
        ++count;
        start = end;
    }
    *batch_count = count;
    if (!sorted) free(buf);
    free(tmp);
    return (!batches || count <= max_batches) ? 1 : 0;
}

/* One expert: gate/up row dots, SiLU(gate)*up, then down row dots
 * (expert_triplet_cpu.cpp.inc:22-106, generation_mlp.cpp.inc:1346-1404). */
static void mo_triplet_act(int32_t mode, const uint8_t* gate, const uint8_t* up, const uint8_t* down,
                           const float* x, uint32_t H, uint32_t I, float* sg, float* su, float* out) {
    const uint64_t row_h = (uint64_t)((H + 31u) / 32u) * 17u;
    const uint64_t row_i = (uint64_t)((I + 31u) / 32u) * 17u;
    for (uint32_t r = 0; r < I; ++r) {
        sg[r] = mo_mxfp4_dot_row(gate + r * row_h, x, H);
        su[r] = mo_mxfp4_dot_row(up + r * row_h, x, H);
        sg[r] = mo_gated_activation(mode, sg[r], su[r]);
    }
    for (uint32_t r = 0; r < H; ++r) out[r] = mo_mxfp4_dot_row(down + r * row_i, sg, I);
}

int mo_expert_triplet(const uint8_t* gate, const uint8_t* up, const uint8_t* down,
                      const float* x, uint32_t H, uint32_t I,
                      float* sg, float* su, float* out) {
    mo_triplet_act(0, gate, up, down, x, H, I, sg, su, out);
    return 1;
}

/* Per-expert output scale (moe_layer_apply_expert_down_scale_f32,
 * generation_mlp.cpp.inc:514-570): one scale for every expert, one per
 * expert, or one per (expert, element); a count that fits none of these
 * leaves the row unscaled, as in the reference. */
static void mo_down_scale(const mo_layer_t* L, uint32_t expert, float* v) {
    const uint64_t n = L->down_scale_count, E = L->experts, H = L->hidden;
    if (!L->down_scale || n == 0) return;
    if (n == 1) {
        for (uint64_t i = 0; i < H; ++i) v[i] *= L->down_scale[0];
    } else if (n == E && expert < E) {
        for (uint64_t i = 0; i < H; ++i) v[i] *= L->down_scale[expert];
    } else if ((uint64_t)expert * H <= n && H <= n - (uint64_t)expert * H) {
        for (uint64_t i = 0; i < H; ++i) v[i] *= L->down_scale[(uint64_t)expert * H + i];
    }
}

/* dst += alpha * src with one fused multiply-add per element: the AVX2
 * _mm256_fmadd_ps loop of moe_axpy_f32 (generation_simd_helpers.cpp.inc:63-84)
 * and its compiler-fused scalar tail. */
static void mo_axpy(float* dst, const float* src, float alpha, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i) dst[i] = fmaf(alpha, src[i], dst[i]);
}

typedef struct {
    const mo_layer_t* L;
    const uint16_t* x_bf16;
    const float* hidden;
    float* y;
    int32_t* ids;
    float* w;
    uint32_t t0, t1;
    uint32_t ties;
    int ok;
} mo_layer_job;

/* One token through the block in moe_layer_moe_mlp_f32 order
 * (generation_mlp.cpp.inc:776-1442):
 *   shared input = x; routed input = RMSNorm(hidden) with pre_norm2 when
 *     given (:820-831, moe_layer_moe_norm_f32 :234-250), else x; the router
 *     reads the routed input, or hidden when the layer has a router input
 *     scale, which it then scales itself (:866-876);
 *   shared expert (:839-860): act(gate)*up, down; RMSNorm with post_norm1
 *     (:853-856); mlp += out * g, g = sigmoid(shared_gate_inp . x) or 1
 *     (moe_layer_shared_expert_gate_f32 :478-512) -- mlp is still 0 there,
 *     so the reference's fused multiply-add is the plain product;
 *   router top-k, gate/up/act and down for each selected expert;
 *   per expert in router order (:1417-1431): RMSNorm with post_norm2, the
 *     down scale, mlp += w_e * y_e;
 *   y = RMSNorm(mlp) with post_norm (moe_add_mlp_residual_f32 :572-594),
 *     else mlp: what the block adds to hidden. */
static void* mo_layer_worker(void* arg) {
    mo_layer_job* j = (mo_layer_job*)arg;
    const mo_layer_t* L = j->L;
    const uint32_t H = L->hidden, I = L->intermediate, K = L->top_k;
    const uint64_t gu_bytes = (uint64_t)I * ((H + 31u) / 32u) * 17u;
    const uint64_t d_bytes = (uint64_t)H * ((I + 31u) / 32u) * 17u;
    const int32_t act = L->activation;
    float* x = (float*)malloc(sizeof(float) * H);
    float* xe = (float*)malloc(sizeof(float) * H);
    float* mlp = (float*)malloc(sizeof(float) * H);
    float* out = (float*)malloc(sizeof(float) * H);
    float* tmp = (float*)malloc(sizeof(float) * H);
    float* sg = (float*)malloc(sizeof(float) * I);
    float* su = (float*)malloc(sizeof(float) * I);
    int32_t* ids = (int32_t*)malloc(sizeof(int32_t) * K);
    float* w = (float*)malloc(sizeof(float) * K);
    float* cw = (float*)malloc(sizeof(float) * K);  /* the combine's weights */
    j->ok = x && xe && mlp && out && tmp && sg && su && ids && w && cw &&
            (!(L->pre_norm2 || L->router_scale) || j->hidden);
    for (uint32_t t = j->t0; j->ok && t < j->t1; ++t) {
        for (uint32_t h = 0; h < H; ++h) x[h] = mo_bf16(j->x_bf16[(uint64_t)t * H + h]);
        const float* xr = x;
        if (L->pre_norm2) {
            mo_rmsnorm(j->hidden + (uint64_t)t * H, L->pre_norm2, H, L->norm_eps, L->norm_unit_offset, xe);
            xr = xe;
        }
        memset(mlp, 0, sizeof(float) * H);
        if (L->shared_gate && L->shared_up && L->shared_down && (!L->present || L->present[L->experts])) {
            mo_triplet_act(act, L->shared_gate, L->shared_up, L->shared_down, x, H, I, sg, su, out);
            float g = 1.0f;
            if (L->shared_gate_inp) g = 1.0f / (1.0f + expf(-mo_bf16_dot_row(L->shared_gate_inp, x, H)));
            const float* so = out;
            if (L->post_norm1) {
                mo_rmsnorm(out, L->post_norm1, H, L->norm_eps, L->norm_unit_offset, tmp);
                so = tmp;
            }
            for (uint32_t h = 0; h < H; ++h) mlp[h] = fmaf(so[h], g, mlp[h]);
        }
        /* with a router scale the router reads the residual stream itself
         * (generation_mlp.cpp.inc:866-871) */
        const float* rin = L->router_scale ? j->hidden + (uint64_t)t * H : xr;
        if (!mo_router_topk(L, rin, ids, w, &j->ties)) { j->ok = 0; break; }
        /* partial failure (generation_mlp.cpp.inc:1219-1282): missing experts
         * drop out; with a renormalising router the others' weights are
         * multiplied by 1 / (their sum, in router order) */
        memcpy(cw, w, sizeof(float) * K);
        if (L->present) {
            uint32_t mapped = 0;
            float wsum = 0.0f;
            for (uint32_t e = 0; e < K; ++e) {
                if (L->present[ids[e]]) {
                    ++mapped;
                    wsum += w[e];
                }
            }
            if (mapped == 0) { j->ok = 0; break; }
            if (mapped < K) {
                const float scale = 1.0f / wsum;
                const int renorm = L->norm_topk && wsum > 1e-9f;
                for (uint32_t e = 0; e < K; ++e) {
                    cw[e] = !L->present[ids[e]] ? 0.0f : (renorm ? w[e] * scale : w[e]);
                }
            }
        }
        for (uint32_t e = 0; e < K; ++e) {
            const uint64_t ex = (uint64_t)ids[e];
            if (L->present && !L->present[ex]) continue;
            mo_triplet_act(act, L->gate + ex * gu_bytes, L->up + ex * gu_bytes, L->down + ex * d_bytes,
                           xr, H, I, sg, su, out);
            if (L->post_norm2) {
                mo_rmsnorm(out, L->post_norm2, H, L->norm_eps, L->norm_unit_offset, tmp);
                memcpy(out, tmp, sizeof(float) * H);
            }
            mo_down_scale(L, (uint32_t)ex, out);
            mo_axpy(mlp, out, cw[e], H);
        }
        float* yt = j->y + (uint64_t)t * H;
        if (L->post_norm) {
            mo_rmsnorm(mlp, L->post_norm, H, L->norm_eps, L->norm_unit_offset, yt);
        } else {
            memcpy(yt, mlp, sizeof(float) * H);
        }
        if (j->ids) memcpy(j->ids + (uint64_t)t * K, ids, sizeof(int32_t) * K);
        if (j->w) memcpy(j->w + (uint64_t)t * K, w, sizeof(float) * K);
    }
    free(x); free(xe); free(mlp); free(out); free(tmp); free(sg); free(su); free(ids); free(w); free(cw);
    return NULL;
}

/* Tokens are independent, so splitting them over threads does not change
 * any result. */
int mo_moe_block(const mo_layer_t* L, const uint16_t* x_bf16, const float* hidden, uint32_t tokens,
                 float* y, int32_t* ids, float* w, uint32_t threads, uint32_t* ties) {
    if (!L || !x_bf16 || !y || L->top_k == 0 || L->top_k > L->experts) return 0;
    if ((L->pre_norm2 || L->router_scale) && !hidden) return 0;
    if (threads == 0) threads = 1;
    if (threads > tokens) threads = tokens ? tokens : 1;
    mo_layer_job* jobs = (mo_layer_job*)calloc(threads, sizeof(mo_layer_job));
    pthread_t* th = (pthread_t*)calloc(threads, sizeof(pthread_t));
    if (!jobs || !th) { free(jobs); free(th); return 0; }
    for (uint32_t i = 0; i < threads; ++i) {
        jobs[i].L = L; jobs[i].x_bf16 = x_bf16; jobs[i].hidden = hidden;
        jobs[i].y = y; jobs[i].ids = ids; jobs[i].w = w;
        jobs[i].t0 = (uint32_t)((uint64_t)tokens * i / threads);
        jobs[i].t1 = (uint32_t)((uint64_t)tokens * (i + 1) / threads);
        if (i > 0) pthread_create(&th[i], NULL, mo_layer_worker, &jobs[i]);
    }
    mo_layer_worker(&jobs[0]);
    int ok = jobs[0].ok;
    uint32_t tie_total = jobs[0].ties;
    for (uint32_t i = 1; i < threads; ++i) {
        pthread_join(th[i], NULL);
        ok = ok && jobs[i].ok;
        tie_total += jobs[i].ties;
    }
    if (ties) *ties += tie_total;
    free(jobs);
    free(th);
    return ok;
}

int mo_moe_layer(const mo_layer_t* L, const uint16_t* x_bf16, uint32_t tokens,
                 float* y, int32_t* ids, float* w, uint32_t threads, uint32_t* ties) {
    return mo_moe_block(L, x_bf16, NULL, tokens, y, ids, w, threads, ties);
}
