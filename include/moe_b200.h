/*
 * moe_b200.h -- C ABI of the B200 (sm_100a) MoE expert-FFN hot path.
 *
 * Drop-in for the CPU expert dispatch of jujumelona/storage.llm's moe_engine:
 * router top-k, token permutation into ragged per-expert groups, MXFP4
 * gate/up grouped GEMM with fused SwiGLU, down grouped GEMM and the weighted
 * combine.  Conventions follow the reference C API
 * (moe_engine/include/moe_pc_engine.h and include/parts/*.h.inc):
 *   - functions return int 1 on success and 0 on failure, never throw;
 *   - a caller-owned `err` buffer of MOE_B200_ERR_LEN bytes (may be NULL)
 *     receives a human-readable message, like moe_generation_stats_t.error
 *     (moe_forward_api.h.inc:63-69);
 *   - buffers are caller-owned with explicit element counts that are checked
 *     against the layer shape (expert_triplet_cpu.cpp.inc:34-43);
 *   - weights are given in the reference's GGUF MXFP4 byte layout (17-byte
 *     blocks per 32 K-elements, rows of ceil(K/32)*17 bytes,
 *     tensor_layout.cpp.inc:174-176) and router weights as bf16 [E x H];
 *   - one engine per CUDA device; calls on one engine are not reentrant.
 * No torch types cross this boundary.
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_B200_ERR_LEN 160

#if defined(__GNUC__)
#define MOE_B200_API __attribute__((visibility("default")))
#else
#define MOE_B200_API
#endif

typedef struct moe_b200_engine moe_b200_engine_t;

typedef struct {
    int32_t device;      /* CUDA device ordinal */
    uint32_t max_layers; /* number of layer weight slots (0 -> 1) */
} moe_b200_init_t;

enum {
    MOE_B200_SCORE_SOFTMAX = 0, /* generation_router.cpp.inc:606-622 (default) */
    MOE_B200_SCORE_SIGMOID = 1  /* generation_router.cpp.inc:600-605 */
};

enum {
    MOE_B200_GEMM_BLOCKSCALED = 0, /* tcgen05 kind::mxf8f6f4 block-scaled MMA on the E2M1 codes (default) */
    MOE_B200_GEMM_SIMT = 1,        /* CUDA-core grouped GEMMs, a cross-check for tests */
    MOE_B200_GEMM_TMEM_DECODE = 2, /* tcgen05 kind::f16 with weights decoded to bf16 in TMEM */
    /* Opt-in fast mode, NOT within the layer tolerance: the activations and
     * the SwiGLU intermediate are quantised to E2M1 with one E8M0 scale per
     * 32 elements (like the weights) and both grouped GEMMs run tcgen05
     * kind::mxf4 (FP4 x FP4).  Routing (ids, weights, permutation) is the
     * exact path's; the output error is a few percent (measured figures are
     * in the tests and the bench).  Single-device forward only. */
    MOE_B200_GEMM_MXF4_FAST = 3
};

/* Explicit form of the routing metadata the reference reads from GGUF JSON
 * keys (num_experts_per_tok, scoring_func, norm_topk_prob,
 * routed_scaling_factor: generation_router.cpp.inc:361-482), and of the
 * block style it reads from the model's metadata (hidden_activation, and
 * the Gemma unit offset of its RMSNorms: raw_forward_utils.cpp.inc:322-350).
 * The tensors of a Gemma-style block around the experts (norms, down
 * scales, shared-expert gate, router input scale) are uploaded per layer
 * with moe_b200_upload_block.  A zero-initialised config is the plain
 * SiLU-gated layer. */
typedef struct {
    uint32_t hidden;       /* H, multiple of 8 */
    uint32_t intermediate; /* I */
    uint32_t experts;      /* E routed experts, <= 1024 */
    uint32_t top_k;        /* k, 1..32 and <= E */
    int32_t layer;         /* weight slot */
    int32_t score_func;    /* MOE_B200_SCORE_* */
    int32_t norm_topk;     /* renormalise the k weights (:659-668) */
    float routed_scale;    /* applied for sigmoid routers only (:669-674); 0 -> 1 */
    int32_t use_shared;    /* add the layer's always-on shared expert (generation_mlp.cpp.inc:833-860) */
    int32_t gemm_path;     /* MOE_B200_GEMM_* */
    /* Group limit of sigmoid routers (generation_router.cpp.inc:484-558):
     * with n_group > 1, 0 < topk_group < n_group and experts % n_group == 0,
     * only the topk_group groups with the largest top-2 score sums keep their
     * scores, the others' are zeroed before the top-k.  0 = none (the
     * reference skips the limit for any other combination, and so does this
     * library); n_group <= 256. */
    uint32_t n_group;
    uint32_t topk_group;
    /* Gated activation of the gate projection (moe_generation_gated_activation_cached,
     * generation_mlp.cpp.inc:94-104): MOE_B200_ACT_*.  Block-scaled paths only. */
    int32_t activation;
    /* RMSNorms of the layer's block parts multiply by (1 + w) (Gemma models) */
    int32_t norm_unit_offset;
    float norm_eps;        /* RMSNorm epsilon of the block parts; <= 0 -> 1e-6 */
    /* Partial-failure policy.  0: an expert (or the shared expert, with
     * use_shared) that was never uploaded makes the call fail.  1: the
     * reference's policy (generation_mlp.cpp.inc:1219-1282, 833-860): such an
     * expert contributes nothing; when norm_topk is set the combine divides
     * the weights of the token's other experts by their sum; a token whose
     * selected experts are all missing fails the call, as the reference's
     * layer fails.  The routing and the returned weights are unchanged.
     * (The expert-parallel forward leaves missing terms out without the
     * renormalisation.) */
    int32_t skip_missing;
} moe_b200_layer_cfg_t;

enum {
    MOE_B200_ACT_SILU = 0,      /* generation_silu.cpp.inc:20-26 */
    MOE_B200_ACT_GELU_ERF = 1,  /* generation_silu.cpp.inc:28-30 */
    MOE_B200_ACT_GELU_TANH = 2  /* generation_mlp.cpp.inc:94-97 */
};

/* Optional tensors of a Gemma-style MoE block around the experts, in the
 * order the reference applies them per token (moe_layer_moe_mlp_f32,
 * generation_mlp.cpp.inc:776-1442).  NULL = the part is absent.  fp32 [H]
 * vectors unless stated:
 *   pre_norm2        the routed experts and the router read
 *                    RMSNorm(hidden) * pre_norm2 (:234-250, :820-831);
 *   post_norm1       RMSNorm of the shared expert's output (:853-856);
 *   post_norm2       RMSNorm of each routed expert's output (:414-429);
 *   post_norm        RMSNorm of the block output (:572-594);
 *   down_scale       scales of the routed outputs: 1 value (all experts), E
 *                    (per expert) or E*H (per element); other counts leave
 *                    them unscaled, as the reference does (:514-570);
 *   shared_gate_inp  bf16 [H] row: the shared expert is scaled by
 *                    sigmoid(row . x) (:478-512);
 *   router_scale     1 or H values: the router reads hidden * rms(hidden)^-1
 *                    * scale / sqrt(H) (generation_router.cpp.inc:316-359). */
typedef struct {
    const float* pre_norm2;
    const float* post_norm1;
    const float* post_norm2;
    const float* post_norm;
    const float* down_scale;
    uint64_t down_scale_count;
    const uint16_t* shared_gate_inp;
    const float* router_scale;
    uint64_t router_scale_count;
} moe_b200_block_tensors_t;

/* Same layout as moe_token_expert_assignment_t / moe_expert_batch_t
 * (include/parts/moe_tensor_types.h.inc:62-74). */
typedef struct {
    uint32_t token_index;
    uint32_t layer;
    uint32_t expert;
    float router_score;
} moe_b200_assignment_t;

typedef struct {
    uint32_t layer;
    uint32_t expert;
    uint32_t first_sorted_index;
    uint32_t token_count;
} moe_b200_batch_t;

/* Engine lifetime.  Replaces moe_pc_engine_create/destroy
 * (include/parts/moe_lifecycle_api.h.inc:6-7) for the GPU hot path. */
MOE_B200_API moe_b200_engine_t* moe_b200_create(const moe_b200_init_t* init, char* err);
MOE_B200_API void moe_b200_destroy(moe_b200_engine_t* engine);

/* Router weight ffn_gate_inp.weight, bf16 [experts x hidden] row-major
 * (the tensor moe_map_router_tensor resolves, generation_router.cpp.inc:
 * 140-186).  `src_on_device` = 1 when `w_bf16` is device memory. */
MOE_B200_API int moe_b200_upload_router(moe_b200_engine_t* engine, int32_t layer, const uint16_t* w_bf16, uint32_t experts,
                           uint32_t hidden, int32_t src_on_device, char* err);

/* One expert's gate [I x H], up [I x H] and down [H x I] projections in the
 * reference's GGUF MXFP4 bytes (per-expert records of codec_table.cpp.inc:
 * 1586-1646).  expert = -1 uploads the layer's shared expert.  The bytes are
 * repacked once into the block-scaled layout the GEMMs read, the only copy
 * the engine keeps (0.53 bytes per weight, like GGUF); the caller keeps
 * ownership of its buffers.  Replaces the residency upload of
 * device_copy_tensor_from_host (device_tensor_copy_ops.cpp.inc:73) for
 * expert triplets.  `src_on_device` = 1 takes the bytes from device memory
 * (e.g. the engine's own resident copy) with no host round trip.  The work
 * runs on the engine's upload stream, which is ordered after work queued on
 * the legacy default stream (device sources written on another stream must
 * be complete before the call); the call returns once its repack is done and
 * stalls no other stream.  The router of the layer must be uploaded first. */
MOE_B200_API int moe_b200_upload_expert(moe_b200_engine_t* engine, int32_t layer, int32_t expert, const uint8_t* gate,
                           uint64_t gate_bytes, const uint8_t* up, uint64_t up_bytes, const uint8_t* down,
                           uint64_t down_bytes, uint32_t hidden, uint32_t intermediate, int32_t src_on_device,
                           char* err);

/* Repacked-expert records: the second half of the residency upload hook
 * (device_tensor_copy_ops.cpp.inc:73), so that a persisted cache beside the
 * model's JUJU sections makes re-residency a plain copy with no repack.
 * A record is one expert's block-scaled form exactly as the engine stores
 * it, four byte ranges back to back (Ip = I and Hp = H rounded up to 128):
 *   gate/up codes  [2][Ip][Hp/2]   E2M1 pairs, 8 KB blocks of 128 rows x 128 K
 *   gate/up scales [Ip/128][Hp/128][gate, up][512]  E8M0, the MMA's layout
 *   down codes     [Hp][Ip/2]
 *   down scales    [Hp/128][Ip/128][512]
 * Its size depends only on H and I (0 for a shape the engine rejects).
 * Export copies a resident expert's record (expert -1: the shared expert)
 * to host or device memory; import installs a record as upload_expert would
 * have left it, without the repack.  Both run on the upload stream and return
 * when their copies are done.  A record carries no shape or checksum of its
 * own: the file that keeps it does (storage.llm_b200/expert_cache.py). */
MOE_B200_API uint64_t moe_b200_expert_record_bytes(uint32_t hidden, uint32_t intermediate);
MOE_B200_API int moe_b200_export_expert(moe_b200_engine_t* engine, int32_t layer, int32_t expert, uint8_t* dst,
                           uint64_t dst_bytes, int32_t dst_on_device, char* err);
MOE_B200_API int moe_b200_import_expert(moe_b200_engine_t* engine, int32_t layer, int32_t expert, const uint8_t* src,
                           uint64_t src_bytes, uint32_t hidden, uint32_t intermediate, int32_t src_on_device,
                           char* err);

/* The cache file of such records, read from C (host code, no device needed).
 * The file is the one storage.llm_b200/expert_cache.py writes:
 *   - a 4096-byte header: magic "MOEB200R", version, H, I, record size,
 *     entry count, the entry table's offset and CRC-32;
 *   - 64-byte entries: layer, expert, source key, record offset, CRC-32;
 *   - records at 4096-aligned offsets.
 * Each record is keyed by the source bytes it was made from:
 * moe_b200_source_key is BLAKE2b-64 (RFC 7693) over the gate, up and down
 * GGUF bytes, each preceded by its byte count as 8 little-endian bytes.
 * open maps the file read-only and checks the header and the entry table;
 * it returns NULL with `err` set otherwise.  record returns the record of
 * (layer, expert) (expert -1: the shared expert) inside the mapping, valid
 * until close.  It returns NULL with err[0] == 0 when the file holds no
 * record of that slot made from `source_key`.  With verify != 0 it also
 * checks the record's CRC-32, and returns NULL with `err` set on a mismatch.
 * A record found goes to moe_b200_import_expert with
 * moe_b200_expert_record_bytes(H, I) bytes. */
typedef struct moe_b200_expert_cache moe_b200_expert_cache_t;
MOE_B200_API uint64_t moe_b200_source_key(const uint8_t* gate, uint64_t gate_bytes, const uint8_t* up,
                           uint64_t up_bytes, const uint8_t* down, uint64_t down_bytes);
MOE_B200_API moe_b200_expert_cache_t* moe_b200_expert_cache_open(const char* path, char* err);
MOE_B200_API void moe_b200_expert_cache_close(moe_b200_expert_cache_t* cache);
MOE_B200_API int moe_b200_expert_cache_info(const moe_b200_expert_cache_t* cache, uint32_t* hidden,
                           uint32_t* intermediate, uint64_t* record_bytes, uint32_t* entries);
MOE_B200_API const uint8_t* moe_b200_expert_cache_record(const moe_b200_expert_cache_t* cache, int32_t layer,
                           int32_t expert, uint64_t source_key, int32_t verify, char* err);

/* The block tensors of a layer (copied into the engine; NULL clears them).
 * The router of the layer must be uploaded first.  The layer's forward then
 * applies them (moe_b200_block_forward when pre_norm2 or router_scale is
 * set, since those read the residual stream).  Block parts need H <= 25600
 * and run on the single-device, block-scaled forward (gemm_path 0 or 3).
 * Replaces the CPU application of those tensors in moe_layer_moe_mlp_f32. */
MOE_B200_API int moe_b200_upload_block(moe_b200_engine_t* engine, int32_t layer, const moe_b200_block_tensors_t* t,
                                       int32_t src_on_device, char* err);

/* The MoE FFN for `tokens` tokens, all pointers device memory, enqueued on
 * `stream` (a cudaStream_t; NULL = legacy default stream).  Replaces the
 * per-token moe_layer_moe_mlp_f32 expert phase (generation_mlp.cpp.inc:
 * 874-1431) and fills the batched slot moe_layer_moe_mlp_batched_f32
 * (generation_api_batch.cpp.inc:68-78).
 *   x_bf16    [tokens x H] expert input (the router input); 8-byte aligned
 *             (16-byte aligned rows take the single-kernel router)
 *   y_bf16    [tokens x H] output mlp = shared + sum_j w_j * expert_j(x) (may be NULL)
 *   y_f32     [tokens x H] the same in fp32 (may be NULL)
 *   topk_ids  [tokens x k] selected experts, descending score (may be NULL)
 *   topk_w    [tokens x k] their weights (may be NULL)
 *   perm      [tokens x k] assignment index t*k+j at each sorted position,
 *             the order of moe_pc_group_tokens_by_expert (may be NULL)
 * The residual add (generation_mlp.cpp.inc:572-594) stays with the caller.
 * Errors found on the device are reported by moe_b200_sync. */
MOE_B200_API int moe_b200_layer_forward(moe_b200_engine_t* engine, const moe_b200_layer_cfg_t* cfg, const uint16_t* x_bf16,
                           uint32_t tokens, uint16_t* y_bf16, float* y_f32, int32_t* topk_ids, float* topk_w,
                           uint32_t* perm, void* stream, char* err);

/* Same with host buffers: copies in, runs, copies out and synchronises. */
MOE_B200_API int moe_b200_layer_forward_host(moe_b200_engine_t* engine, const moe_b200_layer_cfg_t* cfg,
                                const uint16_t* x_bf16, uint32_t tokens, uint16_t* y_bf16, float* y_f32,
                                int32_t* topk_ids, float* topk_w, uint32_t* perm, char* err);

/* The layer with its block parts (moe_b200_upload_block), device pointers:
 * x_bf16 is the expert input (the shared expert's, and the routed experts'
 * and the router's without pre_norm2), hidden_f32 [tokens x H] the residual
 * stream the pre-norm and the router input scale read (may be NULL when the
 * layer has neither).  y = what the block adds to hidden.  The routing is
 * bit-exact with the reference also when the router reads RMSNorm(hidden) or
 * the scaled residual stream; the pre-normed routed input is rounded to
 * bf16 before the experts (tolerance parity). */
MOE_B200_API int moe_b200_block_forward(moe_b200_engine_t* engine, const moe_b200_layer_cfg_t* cfg,
                                        const uint16_t* x_bf16, const float* hidden_f32, uint32_t tokens,
                                        uint16_t* y_bf16, float* y_f32, int32_t* topk_ids, float* topk_w,
                                        void* stream, char* err);
/* Host-buffer variant (copies in, runs, copies out, synchronises). */
MOE_B200_API int moe_b200_block_forward_host(moe_b200_engine_t* engine, const moe_b200_layer_cfg_t* cfg,
                                             const uint16_t* x_bf16, const float* hidden_f32, uint32_t tokens,
                                             uint16_t* y_bf16, float* y_f32, int32_t* topk_ids, float* topk_w,
                                             char* err);

/* Waits for the engine's work and reports any error a kernel recorded
 * (bounded waits that timed out, out-of-range expert ids). */
MOE_B200_API int moe_b200_sync(moe_b200_engine_t* engine, void* stream, char* err);

/* Drop-in for moe_pc_engine_run_expert_triplet_f32
 * (include/parts/moe_forward_api.h.inc:85-96, expert_triplet_cpu.cpp.inc:
 * 22-106): one expert on one fp32 hidden vector, host buffers; scratch_gate
 * receives SiLU(gate)*up, scratch_up receives up.  Synchronous. */
MOE_B200_API int moe_b200_run_expert_triplet_f32(moe_b200_engine_t* engine, int layer, int expert, const float* hidden,
                                    uint32_t hidden_count, float* scratch_gate, float* scratch_up,
                                    uint32_t intermediate_count, float* out_hidden, uint32_t out_count);

/* Drop-in for moe_pc_group_tokens_by_expert (include/parts/moe_names_api.h.inc:
 * 1-8, token_grouping.cpp.inc:1-83), same signature, host buffers: sorts by
 * (layer, expert, token_index) on the current CUDA device and emits the
 * contiguous batches.  Assignments with equal keys keep their input order. */
MOE_B200_API int moe_b200_group_tokens_by_expert(const moe_b200_assignment_t* assignments, uint32_t assignment_count,
                                    moe_b200_assignment_t* out_sorted_assignments, moe_b200_batch_t* out_batches,
                                    uint32_t max_batches, uint32_t* out_batch_count);

/* Allocation-free form of moe_b200_group_tokens_by_expert, for callers that
 * must not allocate device memory while they run: an engine whose residency
 * cache owns the whole VRAM budget (every byte it has not handed out already
 * holds expert weights, so a cudaMalloc mid-layer would fail or evict).  No
 * counterpart in the reference.  Same inputs and outputs (host buffers) plus
 * an error buffer; the result is identical to
 * moe_b200_group_tokens_by_expert's, including the return of 0 with
 * *out_batch_count = the full batch count when more than max_batches
 * batches exist.  It calls no cudaMalloc, cudaFree or allocating library
 * routine: its scratch is a fixed device array of about 4.3 MB inside this
 * library, which every GPU that loads the library holds until the process
 * exits.  Limits and caveats:
 *   - at most MOE_B200_NOALLOC_MAX_ASSIGNMENTS assignments; more returns 0
 *     with a message in `err`;
 *   - it copies the assignments in and the results out with synchronous
 *     copies on the current device's legacy default stream, so it must run
 *     outside any stream capture (before or between captures, never while
 *     a stream of the process is being recorded into a graph);
 *   - the first call on a device resolves the array's device address with
 *     cudaGetSymbolAddress (with that device current) and keeps it; the kept
 *     address does not survive cudaDeviceReset, so do not call it again
 *     after resetting a device in the same process;
 *   - every call shares the one array, which keeps the last call's contents;
 *     calls are serialised within the process, and any other work that
 *     overlaps a call on the GPU and touches the array would race with it. */
#define MOE_B200_NOALLOC_MAX_ASSIGNMENTS 65536u
MOE_B200_API int moe_b200_group_tokens_by_expert_noalloc(const moe_b200_assignment_t* assignments,
                                                         uint32_t assignment_count,
                                                         moe_b200_assignment_t* out_sorted_assignments,
                                                         moe_b200_batch_t* out_batches, uint32_t max_batches,
                                                         uint32_t* out_batch_count, char* err);

/* ------------------------------------------------------------------------
 * Expert parallelism over GPUs (one process and one engine per GPU).
 * Replaces the reference's single-process expert loop
 * (generation_mlp.cpp.inc:1023-1431) when the experts are spread over
 * several devices; the reference has no multi-device counterpart.
 *
 * By default rank r of `world` owns experts [r*E/world, (r+1)*E/world);
 * moe_b200_ep_set_placement spreads and replicates them instead.  The
 * router and the shared expert are replicated and each rank feeds its own
 * tokens.  Every rank uploads the router, its own experts and (if used) the
 * shared expert, then all ranks call moe_b200_ep_layer_forward together.
 * Rows move over NVLink peer memory (CUDA IPC mappings of every rank's
 * receive and return buffers), stored by this library's own kernels; the
 * per-rank row counts and the barriers between the phases are device-side
 * peer stores too (bounded waits).  NCCL, opened at run time
 * (libnccl.so.2), is used only at set-up: to create the communicator and to
 * exchange the IPC handles when the buffers grow.  The host reads the W x W
 * row counts from mapped memory while the dispatch runs, to size the local
 * expert work, and does not synchronise the stream.
 * ------------------------------------------------------------------------ */
#define MOE_B200_EP_UID_BYTES 128
/* A fresh communicator id (ncclGetUniqueId); create it on one rank and
 * hand the bytes to every rank. */
MOE_B200_API int moe_b200_ep_unique_id(uint8_t* out_uid, char* err);
/* Joins the communicator (collective over all `world` ranks). */
MOE_B200_API int moe_b200_ep_init(moe_b200_engine_t* engine, int rank, int world, const uint8_t* uid, char* err);
/* This rank's expert block for a layer of `experts` experts under the
 * default placement (contiguous blocks). */
MOE_B200_API int moe_b200_ep_local_experts(moe_b200_engine_t* engine, uint32_t experts, uint32_t* first,
                                           uint32_t* count, char* err);
/* Expert placement with replication (load balance under skewed routing):
 * expert e lives on replica_count[e] ranks, listed consecutively in
 * replica_ranks; the tokens routed to a replicated expert are spread over its
 * replicas in turn (token index modulo the replica count).  Every rank must
 * set the same placement, upload the experts of its list
 * (moe_b200_ep_local_expert_list) and call the forward afterwards. */
MOE_B200_API int moe_b200_ep_set_placement(moe_b200_engine_t* engine, uint32_t experts,
                                           const uint32_t* replica_count, const uint32_t* replica_ranks, char* err);
/* This rank's experts under the current placement (the default one when none
 * was set), ascending; `capacity` entries available in `out`. */
MOE_B200_API int moe_b200_ep_local_expert_list(moe_b200_engine_t* engine, uint32_t experts, uint32_t* out,
                                               uint32_t capacity, uint32_t* count, char* err);
/* The layer on this rank's T tokens (device pointers, caller's stream; the
 * same outputs as moe_b200_layer_forward for those tokens).  Block-scaled
 * GEMM path only.  T may be 0 (the rank still serves its experts).
 * Collective: every rank calls it, in the same order.  The host returns once
 * the row counts are known (the device work continues on the stream).  If a
 * rank misses a call, the others' device waits give up after about a second
 * each and the call (or the next moe_b200_sync) reports "bounded wait for
 * another rank timed out"; the group is then out of step and must be set up
 * again with moe_b200_ep_init on every rank. */
MOE_B200_API int moe_b200_ep_layer_forward(moe_b200_engine_t* engine, const moe_b200_layer_cfg_t* cfg,
                                           const uint16_t* x_bf16, uint32_t tokens, uint16_t* y_bf16, float* y_f32,
                                           int32_t* topk_ids, float* topk_w, void* stream, char* err);
/* Host-pointer variant (copies in, runs, copies out, synchronises). */
MOE_B200_API int moe_b200_ep_layer_forward_host(moe_b200_engine_t* engine, const moe_b200_layer_cfg_t* cfg,
                                                const uint16_t* x_bf16, uint32_t tokens, uint16_t* y_bf16,
                                                float* y_f32, int32_t* topk_ids, float* topk_w, char* err);
/* Rows this rank sent to / received from each rank in its last call
 * (arrays of `world` entries): the load balance of the exchange. */
MOE_B200_API int moe_b200_ep_last_counts(moe_b200_engine_t* engine, uint32_t* sent, uint32_t* received, char* err);

/* Test and diagnostics hooks (no reference counterpart). */
enum {
    MOE_B200_PROJ_GATE = 0,
    MOE_B200_PROJ_UP = 1,
    MOE_B200_PROJ_DOWN = 2
};
/* Decodes an uploaded projection from the device tile layout back to bf16
 * [rows x cols] in host memory, with the kernels' own decode arithmetic. */
MOE_B200_API int moe_b200_debug_dequant(moe_b200_engine_t* engine, int32_t layer, int32_t expert, int32_t proj,
                           uint16_t* out_bf16, uint64_t out_elems, char* err);

enum {
    MOE_B200_BUF_LOGITS = 0,     /* float  [T x E] */
    MOE_B200_BUF_SCORES = 1,     /* float  [T x E] router scores after softmax/sigmoid */
    MOE_B200_BUF_GROUP_COUNT = 2,/* uint32 [G] */
    MOE_B200_BUF_GROUP_OFFSET = 3,/* uint32 [G+1] */
    MOE_B200_BUF_ROW_TOKEN = 4,  /* uint32 [P] source token of each permuted row */
    MOE_B200_BUF_XPERM = 5,      /* bf16   [P x Kp] */
    MOE_B200_BUF_HPERM = 6,      /* bf16   [P x Ip] */
    MOE_B200_BUF_YPERM = 7       /* float  [P x H] */
};
/* Copies an internal buffer of the last forward call to host memory. */
MOE_B200_API int moe_b200_debug_read(moe_b200_engine_t* engine, int32_t which, void* dst, uint64_t bytes, char* err);

/* Stage timing with CUDA events recorded on the forward's own stream.
 * Stages: 0 router (logits + top-k), 1 permutation (count/scan/scatter),
 * 2 gather of permuted rows, 3 gate/up GEMM, 4 down GEMM, 5 combine.
 * enable(max_calls > 0) starts recording for up to max_calls forwards
 * (0 stops); read() synchronises and returns the summed milliseconds per
 * stage and the number of forwards recorded. */
#define MOE_B200_STAGES 6
MOE_B200_API int moe_b200_profile_enable(moe_b200_engine_t* engine, uint32_t max_calls, char* err);
MOE_B200_API int moe_b200_profile_read(moe_b200_engine_t* engine, float* stage_ms, uint32_t* calls, char* err);

/* Number of kernel launches issued by the last moe_b200_layer_forward. */
MOE_B200_API uint32_t moe_b200_last_launch_count(const moe_b200_engine_t* engine);

#ifdef __cplusplus
}
#endif
#endif /* MOE_B200_H */
