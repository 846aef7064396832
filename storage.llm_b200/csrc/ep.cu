// Expert parallelism across GPUs (one process and one engine per GPU).
//
// Rank r of W owns the contiguous expert block [r*E/W, (r+1)*E/W); the
// router and the shared expert are replicated, tokens are data-parallel.
// One layer call on the rank's own T tokens:
//   1. router + top-k on the local tokens (full E);
//   2. dispatch: a stable sort of the T*K assignments by owner rank, then a
//      pack kernel writing each assignment's token row (bf16 [H]) and its
//      expert index local to the owner into the send buffers;
//   3. NCCL: per-rank row counts (one 4-byte send/recv per peer), one host
//      read of the counts to size the exchange, then grouped send/recv of
//      the rows and their expert indices (an all-to-allv);
//   4. the block-scaled pipeline on the received rows, grouped by (local
//      expert, source rank, source order); the shared expert's rows (the
//      rank's own tokens) ride along as the extra group.  The down GEMM
//      writes each output row at its receive position;
//   5. NCCL: the fp32 expert rows go back to their source ranks (the
//      reverse all-to-allv), landing at the positions they were sent from;
//   6. the combine of the single-device path: shared row + the K expert rows
//      in router order, one fused multiply-add each.
// Because every row's expert output and the combine order are the same as on
// one device, a rank's result equals the single-device result for its
// tokens wherever both pick the same GEMM tile width.
//
// NCCL is opened at run time (the copy the process already loaded, e.g.
// PyTorch's, else libnccl.so.2), so the library loads without it and only
// these entry points report its absence.
#include <dlfcn.h>
#include <nccl.h>  // types and prototypes only; no link-time dependency

#include <algorithm>
#include <mutex>

#include "engine.h"

namespace moe_b200 {

namespace {

struct NcclApi {
    bool ok = false;
    decltype(&ncclGetUniqueId) GetUniqueId = nullptr;
    decltype(&ncclCommInitRank) CommInitRank = nullptr;
    decltype(&ncclCommDestroy) CommDestroy = nullptr;
    decltype(&ncclGroupStart) GroupStart = nullptr;
    decltype(&ncclGroupEnd) GroupEnd = nullptr;
    decltype(&ncclSend) Send = nullptr;
    decltype(&ncclRecv) Recv = nullptr;
    decltype(&ncclGetErrorString) GetErrorString = nullptr;
};

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
        api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
        api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
        api.GroupStart = reinterpret_cast<decltype(api.GroupStart)>(dlsym(h, "ncclGroupStart"));
        api.GroupEnd = reinterpret_cast<decltype(api.GroupEnd)>(dlsym(h, "ncclGroupEnd"));
        api.Send = reinterpret_cast<decltype(api.Send)>(dlsym(h, "ncclSend"));
        api.Recv = reinterpret_cast<decltype(api.Recv)>(dlsym(h, "ncclRecv"));
        api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
        api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.GroupStart && api.GroupEnd &&
                 api.Send && api.Recv && api.GetErrorString;
    });
    return api;
}

#define NCK(call)                                                                      \
    do {                                                                               \
        ncclResult_t r_ = (call);                                                      \
        if (r_ != ncclSuccess) {                                                       \
            set_err(err, "%s failed: %s", #call, nccl().GetErrorString(r_));           \
            return 0;                                                                  \
        }                                                                              \
    } while (0)

// dest[a] = owner rank of assignment a's expert.
__global__ void ep_owner_kernel(const int32_t* __restrict__ ids, uint32_t n, uint32_t e_per,
                                int32_t* __restrict__ dest) {
    for (uint32_t a = blockIdx.x * blockDim.x + threadIdx.x; a < n; a += gridDim.x * blockDim.x) {
        dest[a] = ids[a] / (int32_t)e_per;
    }
}

// Send buffers in owner order: row p carries the token row of assignment
// row_asg[p] and that assignment's expert index local to its owner.  One
// warp per row, 16-byte vectors (H is a multiple of 8).
__global__ void ep_pack_kernel(const uint16_t* __restrict__ x, uint32_t H, uint32_t K, uint32_t e_per,
                               const int32_t* __restrict__ ids, const uint32_t* __restrict__ row_asg, uint32_t n,
                               uint16_t* __restrict__ send_x, int32_t* __restrict__ send_meta) {
    pdl_wait();
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
    for (uint32_t p = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; p < n; p += warps) {
        const uint32_t a = row_asg[p];
        const uint4* src = reinterpret_cast<const uint4*>(x + (uint64_t)(a / K) * H);
        uint4* dst = reinterpret_cast<uint4*>(send_x + (uint64_t)p * H);
        for (uint32_t v = lane; v < H / 8; v += 32) dst[v] = __ldg(src + v);
        if (lane == 0) send_meta[p] = ids[a] % (int32_t)e_per;
    }
}

}  // namespace

struct EpState {
    void* comm = nullptr;  // ncclComm_t
    int rank = 0, world = 1;
    // dispatch permutation (by owner rank)
    DevBuf dest, pos, row_tok, row_asg, cnt, off, gu_off, dn_off, tile_counts, rank_buf;
    DevBuf recv_cnt, slots;
    DevBuf send_x, send_meta, recv_x, recv_meta, yloc, ret;
    uint32_t* h_cnt = nullptr;  // pinned: [world] sent, [world] received
    std::vector<uint32_t> last_sent, last_recv;
    uint32_t slots_key[3] = {~0u, ~0u, ~0u};
};

void ep_release(EpState* ep) {
    if (!ep) return;
    if (ep->comm && nccl().ok) nccl().CommDestroy(static_cast<ncclComm_t>(ep->comm));
    DevBuf* bufs[] = {&ep->dest, &ep->pos, &ep->row_tok, &ep->row_asg, &ep->cnt, &ep->off, &ep->gu_off,
                      &ep->dn_off, &ep->tile_counts, &ep->rank_buf, &ep->recv_cnt, &ep->slots, &ep->send_x,
                      &ep->send_meta, &ep->recv_x, &ep->recv_meta, &ep->yloc, &ep->ret};
    for (DevBuf* b : bufs) b->release();
    if (ep->h_cnt) cudaFreeHost(ep->h_cnt);
    delete ep;
}

}  // namespace moe_b200

using namespace moe_b200;

extern "C" {

int moe_b200_ep_unique_id(uint8_t* out, char* err) {
    if (!out) {
        set_err(err, "null output");
        return 0;
    }
    if (!nccl().ok) {
        set_err(err, "NCCL (libnccl.so.2) not available");
        return 0;
    }
    static_assert(sizeof(ncclUniqueId) == MOE_B200_EP_UID_BYTES, "unique id size");
    ncclUniqueId id;
    NCK(nccl().GetUniqueId(&id));
    memcpy(out, &id, sizeof(id));
    return 1;
}

int moe_b200_ep_init(moe_b200_engine_t* eng, int rank, int world, const uint8_t* uid, char* err) {
    if (!eng || !uid) {
        set_err(err, "null engine or unique id");
        return 0;
    }
    if (world < 1 || rank < 0 || rank >= world) {
        set_err(err, "rank %d outside 0..%d", rank, world - 1);
        return 0;
    }
    if (!nccl().ok) {
        set_err(err, "NCCL (libnccl.so.2) not available");
        return 0;
    }
    CK(cudaSetDevice(eng->device));
    if (eng->ep) {
        ep_release(eng->ep);
        eng->ep = nullptr;
    }
    auto* ep = new (std::nothrow) EpState();
    if (!ep) {
        set_err(err, "out of host memory");
        return 0;
    }
    ep->rank = rank;
    ep->world = world;
    ncclUniqueId id;
    memcpy(&id, uid, sizeof(id));
    ncclComm_t comm = nullptr;
    const ncclResult_t r = nccl().CommInitRank(&comm, world, id, rank);
    if (r != ncclSuccess) {
        set_err(err, "ncclCommInitRank failed: %s", nccl().GetErrorString(r));
        delete ep;
        return 0;
    }
    ep->comm = comm;
    if (cudaMallocHost(&ep->h_cnt, sizeof(uint32_t) * 2 * world) != cudaSuccess) {
        set_err(err, "pinned allocation failed");
        ep_release(ep);
        return 0;
    }
    eng->ep = ep;
    return 1;
}

int moe_b200_ep_local_experts(moe_b200_engine_t* eng, uint32_t experts, uint32_t* first, uint32_t* count,
                              char* err) {
    if (!eng || !eng->ep) {
        set_err(err, "expert parallelism not initialised (moe_b200_ep_init)");
        return 0;
    }
    const uint32_t W = (uint32_t)eng->ep->world;
    if (experts == 0 || experts % W != 0) {
        set_err(err, "%u experts do not split evenly over %u ranks", experts, W);
        return 0;
    }
    if (first) *first = (uint32_t)eng->ep->rank * (experts / W);
    if (count) *count = experts / W;
    return 1;
}

int moe_b200_ep_layer_forward(moe_b200_engine_t* eng, const moe_b200_layer_cfg_t* cfg, const uint16_t* x,
                              uint32_t T, uint16_t* y_bf16, float* y_f32, int32_t* topk_ids, float* topk_w,
                              void* stream, char* err) {
    if (!check_dims(cfg, err)) return 0;
    if (!eng || !eng->ep) {
        set_err(err, "expert parallelism not initialised (moe_b200_ep_init)");
        return 0;
    }
    if (cfg->gemm_path != MOE_B200_GEMM_BLOCKSCALED) {
        set_err(err, "the expert-parallel forward runs the block-scaled GEMM path only");
        return 0;
    }
    EpState* ep = eng->ep;
    LayerWeights* L = get_layer(eng, cfg->layer, err);
    if (!L) return 0;
    const uint32_t H = cfg->hidden, I = cfg->intermediate, E = cfg->experts, K = cfg->top_k;
    const uint32_t W = (uint32_t)ep->world;
    if (L->E != E || L->H != H || L->I != I) {
        set_err(err, "layer %d holds E=%u H=%u I=%u, config asks E=%u H=%u I=%u", cfg->layer, L->E, L->H, L->I, E,
                H, I);
        return 0;
    }
    if (E % W != 0) {
        set_err(err, "%u experts do not split evenly over %u ranks", E, W);
        return 0;
    }
    const uint32_t e_per = E / W, e0 = (uint32_t)ep->rank * e_per;
    for (uint32_t e = e0; e < e0 + e_per; ++e) {
        if (!L->present[e]) {
            set_err(err, "local expert %u of layer %d was never uploaded", e, cfg->layer);
            return 0;
        }
    }
    const bool shared = cfg->use_shared != 0;
    if (shared && !L->present[E]) {
        set_err(err, "layer %d has no shared expert uploaded", cfg->layer);
        return 0;
    }
    if ((uint64_t)T * K > 0x7fffffffull) {
        set_err(err, "tokens x top_k too large");
        return 0;
    }
    if (T > 0 && !x) {
        set_err(err, "null input");
        return 0;
    }
    CK(cudaSetDevice(eng->device));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    ncclComm_t comm = static_cast<ncclComm_t>(ep->comm);
    const uint32_t n = T * K;
    uint32_t* errw = eng->err_word.as<uint32_t>();
    uint32_t launches = 0;
    // stage marks (moe_b200_profile_enable): 0 start, 1 router, 2 dispatch
    // sort + pack, 3 count exchange + host read, 4 row exchange, 5 local
    // experts, 6 return exchange + combine
    cudaEvent_t* ev = nullptr;
    if (eng->prof_max && eng->prof_calls < eng->prof_max) {
        ev = &eng->prof_events[(size_t)eng->prof_calls * (MOE_B200_STAGES + 1)];
        ++eng->prof_calls;
    }
    auto mark = [&](int i) {
        if (ev) cudaEventRecord(ev[i], st);
    };
    mark(0);

    // 1. router on the local tokens
    CK(eng->logits.reserve((size_t)std::max(T, 1u) * E * 4));
    CK(eng->scores.reserve((size_t)std::max(T, 1u) * E * 4));
    CK(eng->ids.reserve((size_t)std::max(n, 1u) * 4));
    CK(eng->wts.reserve((size_t)std::max(n, 1u) * 4));
    int32_t* ids = topk_ids ? topk_ids : eng->ids.as<int32_t>();
    float* w = topk_w ? topk_w : eng->wts.as<float>();
    if (T > 0) {
        const int sigmoid = cfg->score_func == MOE_B200_SCORE_SIGMOID;
        const float rscale = cfg->routed_scale > 0.f ? cfg->routed_scale : 1.0f;
        CK(launch_router(x, L->router.as<uint16_t>(), T, E, H, K, sigmoid, cfg->norm_topk, rscale,
                         eng->logits.as<float>(), ids, w, eng->scores.as<float>(), errw, st, &launches));
    }

    mark(1);
    // 2. dispatch: stable sort by owner rank, then pack the send buffers
    CK(ep->dest.reserve((size_t)std::max(n, 1u) * 4));
    CK(ep->pos.reserve((size_t)std::max(n, 1u) * 4));
    CK(ep->row_tok.reserve((size_t)std::max(n, 1u) * 4));
    CK(ep->row_asg.reserve((size_t)std::max(n, 1u) * 4));
    CK(ep->rank_buf.reserve((size_t)std::max(n, 1u) * 4));
    CK(ep->tile_counts.reserve((size_t)std::max(sort_tiles(n), 1u) * W * 4));
    CK(ep->cnt.reserve((size_t)(W + 1) * 4));
    CK(ep->off.reserve((size_t)(W + 1) * 4));
    CK(ep->gu_off.reserve((size_t)(W + 1) * 4));
    CK(ep->dn_off.reserve((size_t)(W + 1) * 4));
    CK(ep->recv_cnt.reserve((size_t)W * 4));
    CK(ep->send_x.reserve((size_t)std::max(n, 1u) * H * 2));
    CK(ep->send_meta.reserve((size_t)std::max(n, 1u) * 4));
    GroupInfo gd;
    gd.count = ep->cnt.as<uint32_t>();
    gd.offset = ep->off.as<uint32_t>();
    gd.gu_tile_off = ep->gu_off.as<uint32_t>();
    gd.dn_tile_off = ep->dn_off.as<uint32_t>();
    gd.block_n = 1;
    gd.gu_row_tiles = 1;
    gd.dn_row_tiles = 1;
    if (n > 0) {
        ep_owner_kernel<<<std::min(ceil_div(n, 256u), 148u * 4u), 256, 0, st>>>(ids, n, e_per,
                                                                               ep->dest.as<int32_t>());
        CK(cudaGetLastError());
        if (route_small_fits(n, W)) {
            CK(launch_route_small(ep->dest.as<int32_t>(), T, K, W, 0, 0, gd, nullptr, 0, nullptr, 0,
                                  ep->pos.as<uint32_t>(), ep->row_tok.as<uint32_t>(), ep->row_asg.as<uint32_t>(),
                                  nullptr, errw, st, true));
        } else {
            CK(launch_permute(ep->dest.as<int32_t>(), T, K, W, 0, 0, ep->tile_counts.as<uint32_t>(),
                              ep->rank_buf.as<uint32_t>(), gd, ep->pos.as<uint32_t>(), ep->row_tok.as<uint32_t>(),
                              ep->row_asg.as<uint32_t>(), nullptr, errw, st));
        }
        CK(launch_kernel(ep_pack_kernel, dim3(std::min(ceil_div(n, 8u), 148u * 8u)), dim3(256), 0, st, true, x, H,
                         K, e_per, (const int32_t*)ids, (const uint32_t*)ep->row_asg.as<uint32_t>(), n,
                         ep->send_x.as<uint16_t>(), ep->send_meta.as<int32_t>()));
        launches += 4;
    } else {
        CK(cudaMemsetAsync(ep->cnt.ptr, 0, (size_t)(W + 1) * 4, st));
    }

    mark(2);
    // 3. counts, then the rows and their local expert indices
    const NcclApi& nc = nccl();
    NCK(nc.GroupStart());
    for (uint32_t q = 0; q < W; ++q) {
        NCK(nc.Send(ep->cnt.as<uint32_t>() + q, 1, ncclUint32, (int)q, comm, st));
        NCK(nc.Recv(ep->recv_cnt.as<uint32_t>() + q, 1, ncclUint32, (int)q, comm, st));
    }
    NCK(nc.GroupEnd());
    CK(cudaMemcpyAsync(ep->h_cnt, ep->cnt.ptr, W * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(ep->h_cnt + W, ep->recv_cnt.ptr, W * 4, cudaMemcpyDeviceToHost, st));
    mark(3);
    CK(cudaStreamSynchronize(st));
    std::vector<uint32_t> scnt(ep->h_cnt, ep->h_cnt + W), rcnt(ep->h_cnt + W, ep->h_cnt + 2 * W);
    std::vector<uint64_t> soff(W + 1, 0), roff(W + 1, 0);
    for (uint32_t q = 0; q < W; ++q) {
        soff[q + 1] = soff[q] + scnt[q];
        roff[q + 1] = roff[q] + rcnt[q];
    }
    if (soff[W] != n) {
        set_err(err, "dispatch counted %llu rows for %u assignments", (unsigned long long)soff[W], n);
        return 0;
    }
    ep->last_sent = scnt;
    ep->last_recv = rcnt;
    const uint32_t n_recv = (uint32_t)roff[W];
    const uint32_t shared_rows = shared ? T : 0;
    const uint32_t rows = n_recv + shared_rows;  // rows the local experts run on
    CK(ep->recv_x.reserve((size_t)std::max(rows, 1u) * H * 2));
    CK(ep->recv_meta.reserve((size_t)std::max(n_recv, 1u) * 4));
    CK(ep->yloc.reserve((size_t)std::max(rows, 1u) * H * 4));
    CK(ep->ret.reserve((size_t)std::max(n, 1u) * H * 4));
    const uint32_t me = (uint32_t)ep->rank;
    // this rank's own rows: a device copy, not a NCCL self-exchange
    if (scnt[me]) {
        CK(cudaMemcpyAsync(ep->recv_x.as<uint16_t>() + roff[me] * H, ep->send_x.as<uint16_t>() + soff[me] * H,
                           (size_t)scnt[me] * H * 2, cudaMemcpyDeviceToDevice, st));
        CK(cudaMemcpyAsync(ep->recv_meta.as<int32_t>() + roff[me], ep->send_meta.as<int32_t>() + soff[me],
                           (size_t)scnt[me] * 4, cudaMemcpyDeviceToDevice, st));
    }
    if (W > 1) {
        NCK(nc.GroupStart());
        for (uint32_t q = 0; q < W; ++q) {
            if (q == me) continue;
            if (scnt[q]) {
                NCK(nc.Send(ep->send_x.as<uint16_t>() + soff[q] * H, (size_t)scnt[q] * H * 2, ncclUint8, (int)q,
                            comm, st));
                NCK(nc.Send(ep->send_meta.as<int32_t>() + soff[q], scnt[q], ncclInt32, (int)q, comm, st));
            }
            if (rcnt[q]) {
                NCK(nc.Recv(ep->recv_x.as<uint16_t>() + roff[q] * H, (size_t)rcnt[q] * H * 2, ncclUint8, (int)q,
                            comm, st));
                NCK(nc.Recv(ep->recv_meta.as<int32_t>() + roff[q], rcnt[q], ncclInt32, (int)q, comm, st));
            }
        }
        NCK(nc.GroupEnd());
    }
    if (shared_rows) {
        CK(cudaMemcpyAsync(ep->recv_x.as<uint16_t>() + (size_t)n_recv * H, x, (size_t)T * H * 2,
                           cudaMemcpyDeviceToDevice, st));
    }

    mark(4);
    // 4. local experts (+ the shared expert on the local tokens)
    if (ep->slots_key[0] != e0 || ep->slots_key[1] != e_per || ep->slots_key[2] != E) {
        std::vector<uint32_t> slots(e_per + 1);
        for (uint32_t g = 0; g < e_per; ++g) slots[g] = e0 + g;
        slots[e_per] = E;  // the shared expert's slot
        CK(ep->slots.reserve(slots.size() * 4));
        CK(cudaMemcpy(ep->slots.ptr, slots.data(), slots.size() * 4, cudaMemcpyHostToDevice));
        ep->slots_key[0] = e0;
        ep->slots_key[1] = e_per;
        ep->slots_key[2] = E;
    }
    if (rows > 0) {
        BsJob job{};
        job.ids = ep->recv_meta.as<int32_t>();
        job.T = n_recv;
        job.K = 1;
        job.E = e_per;
        job.shared_rows = shared_rows;
        job.shared_base = n_recv;
        job.src = ep->recv_x.as<uint16_t>();
        job.group_slot = ep->slots.as<uint32_t>();
        job.y = ep->yloc.as<float>();
        job.y_by_source = true;
        if (!run_blockscaled(eng, L, job, st, nullptr, &launches, err)) return 0;
    }

    mark(5);
    // 5. expert rows back to their sources
    if (scnt[me]) {
        CK(cudaMemcpyAsync(ep->ret.as<float>() + soff[me] * H, ep->yloc.as<float>() + roff[me] * H,
                           (size_t)scnt[me] * H * 4, cudaMemcpyDeviceToDevice, st));
    }
    if (W > 1) {
        NCK(nc.GroupStart());
        for (uint32_t q = 0; q < W; ++q) {
            if (q == me) continue;
            if (rcnt[q]) {
                NCK(nc.Send(ep->yloc.as<float>() + roff[q] * H, (size_t)rcnt[q] * H, ncclFloat32, (int)q, comm,
                            st));
            }
            if (scnt[q]) {
                NCK(nc.Recv(ep->ret.as<float>() + soff[q] * H, (size_t)scnt[q] * H, ncclFloat32, (int)q, comm,
                            st));
            }
        }
        NCK(nc.GroupEnd());
    }

    // 6. combine in router order
    if (T > 0) {
        CK(launch_combine(ep->ret.as<float>(), H, ep->pos.as<uint32_t>(), w, T, K,
                          shared ? ep->yloc.as<float>() + (size_t)n_recv * H : nullptr, y_bf16, y_f32, st, false));
        launches += 1;
    }
    mark(6);
    eng->last_launches = launches;
    return 1;
}

int moe_b200_ep_layer_forward_host(moe_b200_engine_t* eng, const moe_b200_layer_cfg_t* cfg, const uint16_t* x,
                                   uint32_t T, uint16_t* y_bf16, float* y_f32, int32_t* topk_ids, float* topk_w,
                                   char* err) {
    if (!check_dims(cfg, err)) return 0;
    if (!eng) {
        set_err(err, "null engine");
        return 0;
    }
    if (T > 0 && !x) {
        set_err(err, "null input");
        return 0;
    }
    CK(cudaSetDevice(eng->device));
    const uint32_t H = cfg->hidden, K = cfg->top_k;
    const size_t t1 = std::max(T, 1u);
    CK(eng->hx.reserve(t1 * H * 2));
    CK(eng->hy.reserve(t1 * H * 2));
    CK(eng->hyf.reserve(t1 * H * 4));
    CK(eng->hids.reserve(t1 * K * 4));
    CK(eng->hw.reserve(t1 * K * 4));
    cudaStream_t st = 0;
    if (T > 0) CK(cudaMemcpyAsync(eng->hx.ptr, x, (size_t)T * H * 2, cudaMemcpyHostToDevice, st));
    if (!moe_b200_ep_layer_forward(eng, cfg, eng->hx.as<uint16_t>(), T, y_bf16 ? eng->hy.as<uint16_t>() : nullptr,
                                   y_f32 ? eng->hyf.as<float>() : nullptr, eng->hids.as<int32_t>(),
                                   eng->hw.as<float>(), st, err)) {
        return 0;
    }
    if (T > 0) {
        if (y_bf16) CK(cudaMemcpyAsync(y_bf16, eng->hy.ptr, (size_t)T * H * 2, cudaMemcpyDeviceToHost, st));
        if (y_f32) CK(cudaMemcpyAsync(y_f32, eng->hyf.ptr, (size_t)T * H * 4, cudaMemcpyDeviceToHost, st));
        if (topk_ids) CK(cudaMemcpyAsync(topk_ids, eng->hids.ptr, (size_t)T * K * 4, cudaMemcpyDeviceToHost, st));
        if (topk_w) CK(cudaMemcpyAsync(topk_w, eng->hw.ptr, (size_t)T * K * 4, cudaMemcpyDeviceToHost, st));
    }
    return moe_b200_sync(eng, st, err);
}

int moe_b200_ep_last_counts(moe_b200_engine_t* eng, uint32_t* sent, uint32_t* received, char* err) {
    if (!eng || !eng->ep) {
        set_err(err, "expert parallelism not initialised (moe_b200_ep_init)");
        return 0;
    }
    const EpState* ep = eng->ep;
    for (size_t q = 0; q < ep->last_sent.size(); ++q) {
        if (sent) sent[q] = ep->last_sent[q];
        if (received) received[q] = ep->last_recv[q];
    }
    return 1;
}

}  // extern "C"
