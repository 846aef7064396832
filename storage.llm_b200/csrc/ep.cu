// Expert parallelism across GPUs (one process and one engine per GPU).
//
// By default rank r of W owns the contiguous expert block
// [r*E/W, (r+1)*E/W); moe_b200_ep_set_placement installs any other placement,
// with an expert replicated on several ranks (its tokens then take the
// replicas in turn).  The router and the shared expert are replicated, tokens
// are data-parallel.  One layer call on the rank's own T tokens:
//   1. router + top-k on the local tokens (full E);
//   2. owner rank of each assignment (the replica tables), then a stable
//      sort of the T*K assignments by owner rank;
//   3. count exchange kernel: this rank's per-owner row counts are stored
//      into row `me` of every rank's W x W count matrix (peer memory), a
//      device barrier, then the matrix goes to mapped host memory and the
//      kernel derives where this rank's rows land in every owner's receive
//      buffer;
//   4. dispatch kernel, enqueued before the host reads the counts: each
//      assignment's token row (bf16 [H]) and its owner-local expert index
//      are stored straight into the owner's receive buffer over NVLink (peer
//      memory opened with CUDA IPC); the host meanwhile reads the matrix
//      (polling the mapped flag, no stream synchronisation), and in the rare
//      call where a buffer must grow, all ranks grow and dispatch again;
//   5. the block-scaled pipeline on the received rows, grouped by (local
//      expert, source rank, source order).  The down GEMM's epilogue stores
//      every expert row straight into its source rank's return buffer, at
//      the position the row was sent from: compute and the return exchange
//      are one kernel, tile by tile.  The shared expert on the rank's own
//      tokens needs nothing from the exchange: its pipeline is enqueued on a
//      side stream right after the router and runs while steps 2-4 move the
//      counts and rows over NVLink;
//   6. device barrier, then the single-device combine: shared row + the K
//      expert rows in router order, one fused multiply-add each.
// The device barriers store an epoch into every rank's control words
// (st.release.sys over NVLink) and wait, bounded, for every rank's; NCCL
// remains for set-up (IPC handle exchange when buffers grow).
// Every row's expert output and the combine order are those of one device,
// so a rank's result equals the single-device result for its tokens wherever
// both pick the same GEMM tile width.
//
// The receive and return buffers are symmetric: each rank allocates its own
// and maps every peer's; they grow collectively (all ranks decide from the
// same count matrix) and their IPC handles are re-exchanged then.  NCCL is
// opened at run time (the copy the process already loaded, e.g. PyTorch's,
// else libnccl.so.2), so the library loads without it and only these entry
// points report its absence.
#include <dlfcn.h>
#include <nccl.h>  // types and prototypes only; no link-time dependency

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstring>
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
    decltype(&ncclAllGather) AllGather = nullptr;
    decltype(&ncclAllReduce) AllReduce = nullptr;
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
        api.AllGather = reinterpret_cast<decltype(api.AllGather)>(dlsym(h, "ncclAllGather"));
        api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(dlsym(h, "ncclAllReduce"));
        api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
        api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.GroupStart && api.GroupEnd &&
                 api.Send && api.Recv && api.AllGather && api.AllReduce && api.GetErrorString;
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

// Destination of assignment a (token a / K, expert e = ids[a]): the expert's
// replicas are rep_ranks[rep_off[e] .. rep_off[e+1]); tokens take them in
// turn (token index modulo the replica count).  meta[a] = the expert's index
// in the destination's local expert list.
__global__ void ep_owner_kernel(const int32_t* __restrict__ ids, uint32_t n, uint32_t K, uint32_t E,
                                const uint32_t* __restrict__ rep_off, const uint32_t* __restrict__ rep_ranks,
                                const uint32_t* __restrict__ local_idx, int32_t* __restrict__ dest,
                                int32_t* __restrict__ meta) {
    for (uint32_t a = blockIdx.x * blockDim.x + threadIdx.x; a < n; a += gridDim.x * blockDim.x) {
        const uint32_t e = (uint32_t)ids[a];
        const uint32_t r0 = __ldg(rep_off + e), nr = __ldg(rep_off + e + 1) - r0;
        const uint32_t q = __ldg(rep_ranks + r0 + (a / K) % nr);
        dest[a] = (int32_t)q;
        meta[a] = (int32_t)__ldg(local_idx + (uint64_t)q * E + e);
    }
}

// Dispatch: row p of the owner-ordered assignment list (p in [soff[q],
// soff[q+1]) goes to rank q) is stored into rank q's receive buffer at row
// dst_off[q] + p - soff[q]: the assignment's token row and its expert index
// in q's local list (meta).  One warp per row, 16-byte stores (H is a
// multiple of 8), into peer memory for q != this rank.  Rows past rank q's
// capacity (cap_rows[q]) are skipped: the host, which learns the counts while
// this runs, grows the buffers and dispatches again.
__global__ void ep_dispatch_kernel(const uint16_t* __restrict__ x, uint32_t H, uint32_t K,
                                   const int32_t* __restrict__ meta, const uint32_t* __restrict__ row_asg, uint32_t n,
                                   const uint32_t* __restrict__ soff, const uint32_t* __restrict__ dst_off,
                                   const uint32_t* __restrict__ cap_rows, uint16_t* const* __restrict__ peer_x,
                                   int32_t* const* __restrict__ peer_meta, uint32_t world) {
    pdl_wait();
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
    for (uint32_t p = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; p < n; p += warps) {
        uint32_t q = 0;
        while (q + 1 < world && __ldg(soff + q + 1) <= p) ++q;
        const uint64_t row = (uint64_t)dst_off[q] + p - __ldg(soff + q);
        if (row >= __ldg(cap_rows + q)) continue;  // rank q's buffer grows first; this call then dispatches again
        const uint32_t a = row_asg[p];
        const uint4* src = reinterpret_cast<const uint4*>(x + (uint64_t)(a / K) * H);
        uint4* dst = reinterpret_cast<uint4*>(peer_x[q] + row * H);
        for (uint32_t v = lane; v < H / 8; v += 32) dst[v] = __ldg(src + v);
        if (lane == 0) peer_meta[q][row] = meta[a];
    }
    __threadfence_system();  // peer stores before the exchange barrier
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Barrier over the ranks through their control buffers (word q of rank r's
// buffer: the last barrier epoch rank q reached, as seen by r).  One block,
// thread q < W handles rank q: this rank's earlier stores (peer memory
// included) are fenced, its arrival is stored into every rank's word `me`,
// then thread q waits until rank q's arrival shows here.  Epochs only grow,
// so a rank that is already one barrier ahead still counts.  Each wait gives
// up after ~1 s of SM clocks, recording kErrTimeoutPeer.
__device__ void ep_barrier(uint32_t* const* peer_ctrl, uint32_t me, uint32_t W, uint32_t epoch, uint32_t* err) {
    const uint32_t q = threadIdx.x;
    __threadfence_system();
    __syncthreads();
    if (q < W) st_release_sys(peer_ctrl[q] + me, epoch);
    if (q < W) {
        const uint32_t* f = peer_ctrl[me] + q;
        const long long t0 = clock64();
        while ((int32_t)(ld_acquire_sys(f) - epoch) < 0) {
            if (clock64() - t0 > (1ll << 31)) {
                record_error(err, kErrTimeoutPeer);
                break;
            }
            __nanosleep(100);
        }
    }
    __syncthreads();
}

__global__ void ep_barrier_kernel(uint32_t* const* peer_ctrl, uint32_t me, uint32_t W, uint32_t epoch,
                                  uint32_t* err) {
    ep_barrier(peer_ctrl, me, W, epoch, err);
}

// The W x W row-count matrix without NCCL: this rank's counts cnt[W] go into
// row `me` of every rank's matrix (words W + me*W .. of its control buffer),
// a barrier, then the whole matrix is copied to pinned host memory followed by
// the epoch in the word after it (stored last, release), which the host polls.
__global__ void ep_counts_kernel(const uint32_t* __restrict__ cnt, uint32_t* const* peer_ctrl, uint32_t me,
                                 uint32_t W, uint32_t epoch, uint32_t* host_ctrl, uint32_t* __restrict__ small,
                                 uint32_t* err) {
    pdl_wait();
    for (uint32_t i = threadIdx.x; i < W * W; i += blockDim.x) {
        const uint32_t q = i / W, j = i % W;
        peer_ctrl[q][W + me * W + j] = cnt[j];
    }
    ep_barrier(peer_ctrl, me, W, epoch, err);
    const uint32_t* mat = peer_ctrl[me] + W;
    for (uint32_t i = threadIdx.x; i < W * W; i += blockDim.x) host_ctrl[i] = ld_relaxed_sys(mat + i);
    // small: dst_off[q] = where this rank's rows start in rank q's receive
    // buffer; roff[r] = where rank r's rows start in this rank's; sbase[r] =
    // where rank r expects the rows it sent here, in its return buffer
    if (threadIdx.x == 0) {
        uint32_t acc = 0;
        small[W] = 0;
        for (uint32_t r = 0; r < W; ++r) {
            acc += ld_relaxed_sys(mat + r * W + me);
            small[W + 1 + r] = acc;
        }
        for (uint32_t q = 0; q < W; ++q) {
            uint32_t o = 0, b = 0;
            for (uint32_t r = 0; r < me; ++r) o += ld_relaxed_sys(mat + r * W + q);
            for (uint32_t j = 0; j < me; ++j) b += ld_relaxed_sys(mat + q * W + j);
            small[q] = o;
            small[2 * W + 1 + q] = b;
        }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) st_release_sys(host_ctrl + W * W, epoch);
}

}  // namespace

// A buffer every rank allocates and every peer maps (CUDA IPC).
struct SymBuf {
    DevBuf local;
    std::vector<void*> peer;  // peer[q]: rank q's buffer as mapped here (this rank's own: local)
};

struct EpState {
    void* comm = nullptr;  // ncclComm_t
    int rank = 0, world = 1;
    // dispatch permutation (by owner rank)
    DevBuf dest, pos, row_tok, row_asg, cnt, off, gu_off, dn_off, tile_counts, rank_buf;
    DevBuf small;      // per call, written on the device: dst_off[W], roff[W+1], sbase[W]
    DevBuf ptrs;       // device copies of the peer pointers: x[W], meta[W], ret[W]
    DevBuf barrier_word, slots, yloc, handles;
    SymBuf recv_x, recv_meta, ret;  // receive rows, their expert indices; returned expert rows
    std::vector<uint64_t> cap_x, cap_meta, cap_ret;  // every rank's capacities (bytes), the same on all ranks
    // control words for the device-side count exchange and barriers: per rank
    // [W] barrier epochs + [W x W] count matrix, mapped on every peer
    SymBuf ctrl;
    DevBuf ctrl_ptrs;             // device copy of ctrl.peer
    uint32_t epoch = 0;           // barriers taken so far (the same on every rank)
    uint32_t* h_ctrl = nullptr;   // mapped pinned [W x W] matrix + [1] epoch
    uint32_t* d_h_ctrl = nullptr; // its device address
    DevBuf cap_rows;              // [W] rows each rank's receive buffers hold (for H = cap_rows_H)
    uint32_t cap_rows_H = 0, cap_gen = 0, cap_rows_gen = ~0u;
    std::vector<uint32_t> last_sent, last_recv;
    // expert placement (identical on every rank): replicas of expert e are
    // rep_ranks[rep_off[e] .. rep_off[e+1]); this rank's experts in order
    uint32_t place_E = 0;
    std::vector<uint32_t> rep_off, rep_ranks, local_list;
    DevBuf d_rep_off, d_rep_ranks, d_local_idx, meta;
    bool slots_dirty = true;
    // the shared expert's rows (this rank's own tokens) run on a side stream
    // while the token rows cross NVLink: its group map, its all-zero group
    // ids, its output rows, and the fork / join events
    cudaStream_t side = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    DevBuf shared_slot, zero_ids, yshared;
};

void close_peers(EpState* ep, SymBuf& b) {
    for (size_t q = 0; q < b.peer.size(); ++q) {
        if ((int)q != ep->rank && b.peer[q]) cudaIpcCloseMemHandle(b.peer[q]);
    }
    b.peer.assign(ep->world, nullptr);
}

void ep_release(EpState* ep) {
    if (!ep) return;
    close_peers(ep, ep->recv_x);
    close_peers(ep, ep->recv_meta);
    close_peers(ep, ep->ret);
    close_peers(ep, ep->ctrl);
    if (ep->comm && nccl().ok) nccl().CommDestroy(static_cast<ncclComm_t>(ep->comm));
    DevBuf* bufs[] = {&ep->dest, &ep->pos, &ep->row_tok, &ep->row_asg, &ep->cnt, &ep->off, &ep->gu_off,
                      &ep->dn_off, &ep->tile_counts, &ep->rank_buf, &ep->small, &ep->ptrs,
                      &ep->barrier_word, &ep->slots, &ep->yloc, &ep->handles, &ep->recv_x.local,
                      &ep->recv_meta.local, &ep->ret.local, &ep->d_rep_off, &ep->d_rep_ranks,
                      &ep->d_local_idx, &ep->meta, &ep->ctrl.local, &ep->ctrl_ptrs, &ep->cap_rows};
    for (DevBuf* b : bufs) b->release();
    ep->shared_slot.release();
    ep->zero_ids.release();
    ep->yshared.release();
    if (ep->side) cudaStreamDestroy(ep->side);
    if (ep->ev_fork) cudaEventDestroy(ep->ev_fork);
    if (ep->ev_join) cudaEventDestroy(ep->ev_join);
    if (ep->h_ctrl) cudaFreeHost(ep->h_ctrl);
    delete ep;
}

// Installs a placement (replica lists per expert) and its device tables.
int ep_apply_placement(EpState* ep, uint32_t E, const std::vector<uint32_t>& rep_off,
                       const std::vector<uint32_t>& rep_ranks, char* err) {
    const uint32_t W = (uint32_t)ep->world, me = (uint32_t)ep->rank;
    std::vector<uint32_t> local_idx((size_t)W * E, 0xFFFFFFFFu);
    std::vector<uint32_t> next(W, 0), mine;
    for (uint32_t e = 0; e < E; ++e) {
        for (uint32_t i = rep_off[e]; i < rep_off[e + 1]; ++i) {
            const uint32_t q = rep_ranks[i];
            local_idx[(size_t)q * E + e] = next[q]++;
            if (q == me) mine.push_back(e);
        }
    }
    CK(ep->d_rep_off.reserve(rep_off.size() * 4));
    CK(ep->d_rep_ranks.reserve(std::max<size_t>(rep_ranks.size(), 1) * 4));
    CK(ep->d_local_idx.reserve(local_idx.size() * 4));
    CK(cudaMemcpy(ep->d_rep_off.ptr, rep_off.data(), rep_off.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(ep->d_rep_ranks.ptr, rep_ranks.data(), rep_ranks.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(ep->d_local_idx.ptr, local_idx.data(), local_idx.size() * 4, cudaMemcpyHostToDevice));
    ep->place_E = E;
    ep->rep_off = rep_off;
    ep->rep_ranks = rep_ranks;
    ep->local_list = mine;
    ep->slots_dirty = true;
    return 1;
}

// The default placement: contiguous blocks of E/W experts, one replica each.
int ep_default_placement(EpState* ep, uint32_t E, char* err) {
    const uint32_t W = (uint32_t)ep->world;
    if (E == 0 || E % W != 0) {
        set_err(err, "%u experts do not split evenly over %u ranks (set a placement)", E, W);
        return 0;
    }
    std::vector<uint32_t> off(E + 1), ranks(E);
    for (uint32_t e = 0; e <= E; ++e) off[e] = e;
    for (uint32_t e = 0; e < E; ++e) ranks[e] = e / (E / W);
    return ep_apply_placement(ep, E, off, ranks, err);
}

// Makes every rank's receive/return buffers at least as large as this call
// needs (all ranks decide from the same count matrix and token counts, so
// they agree without talking), then re-exchanges the IPC handles.
// Collective.  Before any mapping closes, this rank's stream is drained (a
// dispatch into the old buffers may still run), and a barrier makes sure no
// rank still uses a mapping its owner is about to free.  These collectives
// are NCCL's and have no timeout: after a peer timed out in the count
// exchange, ranks can disagree on growing, and the next such call can block.
int ep_ensure_capacity(EpState* ep, const std::vector<uint64_t>& need_x, const std::vector<uint64_t>& need_meta,
                       const std::vector<uint64_t>& need_ret, cudaStream_t st, char* err) {
    const uint32_t W = (uint32_t)ep->world, me = (uint32_t)ep->rank;
    bool grow = false;
    for (uint32_t q = 0; q < W; ++q) {
        grow = grow || need_x[q] > ep->cap_x[q] || need_meta[q] > ep->cap_meta[q] || need_ret[q] > ep->cap_ret[q];
    }
    if (!grow) return 1;
    ++ep->cap_gen;
    // this rank's own kernels (a dispatch into the old buffers) finish
    // before any mapping closes
    CK(cudaStreamSynchronize(st));
    const NcclApi& nc = nccl();
    ncclComm_t comm = static_cast<ncclComm_t>(ep->comm);
    auto bump = [](uint64_t need, uint64_t cap) {
        return need > cap ? std::max<uint64_t>(need + need / 4, 1u << 16) : cap;
    };
    for (uint32_t q = 0; q < W; ++q) {
        ep->cap_x[q] = bump(need_x[q], ep->cap_x[q]);
        ep->cap_meta[q] = bump(need_meta[q], ep->cap_meta[q]);
        ep->cap_ret[q] = bump(need_ret[q], ep->cap_ret[q]);
    }
    // nobody may still use an old mapping when a rank frees its old buffer
    close_peers(ep, ep->recv_x);
    close_peers(ep, ep->recv_meta);
    close_peers(ep, ep->ret);
    NCK(nc.AllReduce(ep->barrier_word.ptr, ep->barrier_word.ptr, 1, ncclUint32, ncclSum, comm, st));
    CK(cudaStreamSynchronize(st));
    SymBuf* bufs[3] = {&ep->recv_x, &ep->recv_meta, &ep->ret};
    const uint64_t caps[3] = {ep->cap_x[me], ep->cap_meta[me], ep->cap_ret[me]};
    for (int i = 0; i < 3; ++i) CK(bufs[i]->local.reserve(caps[i]));
    cudaIpcMemHandle_t mine[3];
    for (int i = 0; i < 3; ++i) CK(cudaIpcGetMemHandle(&mine[i], bufs[i]->local.ptr));
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    CK(ep->handles.reserve(hb * 3 * (W + 1)));
    uint8_t* d_h = ep->handles.as<uint8_t>();
    CK(cudaMemcpyAsync(d_h, mine, hb * 3, cudaMemcpyHostToDevice, st));
    NCK(nc.AllGather(d_h, d_h + hb * 3, hb * 3, ncclUint8, comm, st));
    std::vector<cudaIpcMemHandle_t> all(3 * W);
    CK(cudaMemcpyAsync(all.data(), d_h + hb * 3, hb * 3 * W, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    for (uint32_t q = 0; q < W; ++q) {
        for (int i = 0; i < 3; ++i) {
            if (q == me) {
                bufs[i]->peer[q] = bufs[i]->local.ptr;
            } else {
                void* ptr = nullptr;
                CK(cudaIpcOpenMemHandle(&ptr, all[3 * q + i], cudaIpcMemLazyEnablePeerAccess));
                bufs[i]->peer[q] = ptr;
            }
        }
    }
    std::vector<void*> dev_ptrs(3 * W);
    for (uint32_t q = 0; q < W; ++q) {
        dev_ptrs[q] = ep->recv_x.peer[q];
        dev_ptrs[W + q] = ep->recv_meta.peer[q];
        dev_ptrs[2 * W + q] = ep->ret.peer[q];
    }
    CK(ep->ptrs.reserve(sizeof(void*) * 3 * W));
    CK(cudaMemcpy(ep->ptrs.ptr, dev_ptrs.data(), sizeof(void*) * 3 * W, cudaMemcpyHostToDevice));
    return 1;
}

// Maps every rank's control buffer (collective, once per group).
int ep_map_ctrl(EpState* ep, char* err) {
    const uint32_t W = (uint32_t)ep->world, me = (uint32_t)ep->rank;
    const NcclApi& nc = nccl();
    ncclComm_t comm = static_cast<ncclComm_t>(ep->comm);
    cudaIpcMemHandle_t mine;
    CK(cudaIpcGetMemHandle(&mine, ep->ctrl.local.ptr));
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    DevBuf& d_h = ep->handles;
    CK(d_h.reserve(hb * (W + 1)));
    CK(cudaMemcpy(d_h.ptr, &mine, hb, cudaMemcpyHostToDevice));
    NCK(nc.AllGather(d_h.ptr, d_h.as<uint8_t>() + hb, hb, ncclUint8, comm, 0));
    std::vector<cudaIpcMemHandle_t> all(W);
    CK(cudaMemcpy(all.data(), d_h.as<uint8_t>() + hb, hb * W, cudaMemcpyDeviceToHost));
    for (uint32_t q = 0; q < W; ++q) {
        if (q == me) {
            ep->ctrl.peer[q] = ep->ctrl.local.ptr;
        } else {
            void* ptr = nullptr;
            CK(cudaIpcOpenMemHandle(&ptr, all[q], cudaIpcMemLazyEnablePeerAccess));
            ep->ctrl.peer[q] = ptr;
        }
    }
    CK(ep->ctrl_ptrs.reserve(sizeof(void*) * W));
    CK(cudaMemcpy(ep->ctrl_ptrs.ptr, ep->ctrl.peer.data(), sizeof(void*) * W, cudaMemcpyHostToDevice));
    // every rank has mapped every buffer before anyone stores into them
    NCK(nc.AllReduce(ep->barrier_word.ptr, ep->barrier_word.ptr, 1, ncclUint32, ncclSum, comm, 0));
    CK(cudaDeviceSynchronize());
    return 1;
}

// Waits (host) for the count matrix of barrier `epoch`; ~10 s at most.
int ep_wait_counts(EpState* ep, uint32_t epoch, char* err) {
    const uint32_t W = (uint32_t)ep->world;
    volatile uint32_t* flag = ep->h_ctrl + W * W;
    const auto t0 = std::chrono::steady_clock::now();
    for (uint64_t i = 0; *flag != epoch; ++i) {
        if ((i & 1023) == 0 && std::chrono::steady_clock::now() - t0 > std::chrono::seconds(10)) {
            set_err(err, "expert-parallel count exchange timed out (a rank missing?)");
            return 0;
        }
    }
    std::atomic_thread_fence(std::memory_order_acquire);
    return 1;
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
    if (world > 32) {  // one lane per rank in the device barriers; one node holds at most 8 GPUs anyway
        set_err(err, "world of %d ranks: at most 32 supported", world);
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
    ep->recv_x.peer.assign(world, nullptr);
    ep->recv_meta.peer.assign(world, nullptr);
    ep->ret.peer.assign(world, nullptr);
    ep->cap_x.assign(world, 0);
    ep->cap_meta.assign(world, 0);
    ep->cap_ret.assign(world, 0);
    ep->ctrl.peer.assign(world, nullptr);
    const size_t ctrl_bytes = sizeof(uint32_t) * (world + world * world);
    if (cudaHostAlloc(&ep->h_ctrl, sizeof(uint32_t) * (world * world + 1), cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer(&ep->d_h_ctrl, ep->h_ctrl, 0) != cudaSuccess ||
        ep->barrier_word.reserve(4) != cudaSuccess || cudaMemset(ep->barrier_word.ptr, 0, 4) != cudaSuccess ||
        ep->ctrl.local.reserve(ctrl_bytes) != cudaSuccess ||
        cudaMemset(ep->ctrl.local.ptr, 0, ctrl_bytes) != cudaSuccess ||
        cudaStreamCreateWithFlags(&ep->side, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&ep->ev_fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ep->ev_join, cudaEventDisableTiming) != cudaSuccess) {
        set_err(err, "allocation failed");
        ep_release(ep);
        return 0;
    }
    memset(ep->h_ctrl, 0, sizeof(uint32_t) * (world * world + 1));
    if (!ep_map_ctrl(ep, err)) {
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

int moe_b200_ep_set_placement(moe_b200_engine_t* eng, uint32_t experts, const uint32_t* replica_count,
                              const uint32_t* replica_ranks, char* err) {
    if (!eng || !eng->ep) {
        set_err(err, "expert parallelism not initialised (moe_b200_ep_init)");
        return 0;
    }
    if (experts == 0 || !replica_count || !replica_ranks) {
        set_err(err, "empty placement");
        return 0;
    }
    const uint32_t W = (uint32_t)eng->ep->world;
    std::vector<uint32_t> off(experts + 1, 0);
    for (uint32_t e = 0; e < experts; ++e) {
        if (replica_count[e] == 0 || replica_count[e] > W) {
            set_err(err, "expert %u has %u replicas (1..%u)", e, replica_count[e], W);
            return 0;
        }
        off[e + 1] = off[e] + replica_count[e];
    }
    std::vector<uint32_t> ranks(replica_ranks, replica_ranks + off[experts]);
    for (uint32_t e = 0; e < experts; ++e) {
        for (uint32_t i = off[e]; i < off[e + 1]; ++i) {
            if (ranks[i] >= W) {
                set_err(err, "expert %u placed on rank %u of %u", e, ranks[i], W);
                return 0;
            }
            for (uint32_t j = off[e]; j < i; ++j) {
                if (ranks[j] == ranks[i]) {
                    set_err(err, "expert %u placed twice on rank %u", e, ranks[i]);
                    return 0;
                }
            }
        }
    }
    CK(cudaSetDevice(eng->device));
    return ep_apply_placement(eng->ep, experts, off, ranks, err);
}

int moe_b200_ep_local_expert_list(moe_b200_engine_t* eng, uint32_t experts, uint32_t* out, uint32_t capacity,
                                  uint32_t* count, char* err) {
    if (!eng || !eng->ep) {
        set_err(err, "expert parallelism not initialised (moe_b200_ep_init)");
        return 0;
    }
    EpState* ep = eng->ep;
    if (ep->place_E != experts) {
        CK(cudaSetDevice(eng->device));
        if (!ep_default_placement(ep, experts, err)) return 0;
    }
    if (count) *count = (uint32_t)ep->local_list.size();
    if (out) {
        if (capacity < ep->local_list.size()) {
            set_err(err, "%zu local experts do not fit in %u entries", ep->local_list.size(), capacity);
            return 0;
        }
        for (size_t i = 0; i < ep->local_list.size(); ++i) out[i] = ep->local_list[i];
    }
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
    if (cfg->activation != MOE_B200_ACT_SILU ||
        (cfg->layer >= 0 && (size_t)cfg->layer < eng->layers.size() && eng->layers[cfg->layer].has_block())) {
        set_err(err, "block parts and GELU activations run on the single-device forward");
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
    if (ep->place_E != E && !ep_default_placement(ep, E, err)) return 0;
    const uint32_t e_loc = (uint32_t)ep->local_list.size();
    if (L->present.size() != (size_t)E + 1) {
        set_err(err, "layer %d has no experts uploaded", cfg->layer);
        return 0;
    }
    for (uint32_t e : ep->local_list) {
        if (!L->present[e] && !cfg->skip_missing) {
            set_err(err, "local expert %u of layer %d was never uploaded", e, cfg->layer);
            return 0;
        }
    }
    const bool shared = cfg->use_shared != 0;
    if (shared && !L->present[E] && !cfg->skip_missing) {
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
        CUtensorMap rtx, rtw;
        const bool rt_tma = router_tmaps(eng, x, L->router.as<uint16_t>(), T, E, H, &rtx, &rtw);
        CK(launch_router(x, L->router.as<uint16_t>(), T, E, H, K,
                         RouteCfg{sigmoid, cfg->norm_topk, rscale, cfg->n_group, cfg->topk_group},
                         eng->logits.as<float>(), ids, w, eng->scores.as<float>(), errw, st, &launches,
                         rt_tma ? &rtx : nullptr, rt_tma ? &rtw : nullptr));
    }

    mark(1);
    // the shared expert's pass may start once the previous call's local
    // experts are done with the workspace, i.e. from here on
    CK(cudaEventRecord(ep->ev_fork, st));
    if (ep->slots_dirty) {
        std::vector<uint32_t> slots(ep->local_list);
        CK(ep->slots.reserve(std::max<size_t>(slots.size(), 1) * 4));
        if (!slots.empty()) {
            CK(cudaMemcpy(ep->slots.ptr, slots.data(), slots.size() * 4, cudaMemcpyHostToDevice));
        }
        const uint32_t ss = E;  // the shared expert's slot
        CK(ep->shared_slot.reserve(4));
        CK(cudaMemcpy(ep->shared_slot.ptr, &ss, 4, cudaMemcpyHostToDevice));
        ep->slots_dirty = false;
    }
    // The shared expert on this rank's own tokens needs nothing from the
    // exchange: its pipeline (one group, all token ids 0, the shared slot)
    // runs on the side stream while the counts and rows cross NVLink.  A
    // workspace that the received rows' pass grows later is reallocated by
    // cudaFree / cudaMalloc, which wait for this pass first.
    const uint32_t shared_rows = shared ? T : 0;
    if (shared_rows) {
        if (ep->zero_ids.bytes < (size_t)T * 4) {
            CK(ep->zero_ids.reserve((size_t)T * 4));
            CK(cudaMemset(ep->zero_ids.ptr, 0, ep->zero_ids.bytes));
        }
        CK(ep->yshared.reserve((size_t)T * H * 4));
        BsJob sj{};
        sj.ids = ep->zero_ids.as<int32_t>();
        sj.T = T;
        sj.K = 1;
        sj.E = 1;
        sj.src = x;
        sj.group_slot = ep->shared_slot.as<uint32_t>();
        sj.y = ep->yshared.as<float>();
        sj.y_by_source = true;
        CK(cudaStreamWaitEvent(ep->side, ep->ev_fork, 0));
        if (!run_blockscaled(eng, L, sj, ep->side, nullptr, &launches, err)) return 0;
        CK(cudaEventRecord(ep->ev_join, ep->side));
    }
    // 2. stable sort of the assignments by owner rank
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
    GroupInfo gd;
    gd.count = ep->cnt.as<uint32_t>();
    gd.offset = ep->off.as<uint32_t>();
    gd.gu_tile_off = ep->gu_off.as<uint32_t>();
    gd.dn_tile_off = ep->dn_off.as<uint32_t>();
    gd.block_n = 1;
    gd.gu_row_tiles = 1;
    gd.dn_row_tiles = 1;
    if (n > 0) {
        CK(ep->meta.reserve((size_t)n * 4));
        ep_owner_kernel<<<std::min(ceil_div(n, 256u), 148u * 4u), 256, 0, st>>>(
            ids, n, K, E, ep->d_rep_off.as<uint32_t>(), ep->d_rep_ranks.as<uint32_t>(),
            ep->d_local_idx.as<uint32_t>(), ep->dest.as<int32_t>(), ep->meta.as<int32_t>());
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
        launches += 2;
    } else {
        CK(cudaMemsetAsync(ep->cnt.ptr, 0, (size_t)(W + 1) * 4, st));
        CK(cudaMemsetAsync(ep->off.ptr, 0, (size_t)(W + 1) * 4, st));
    }
    mark(2);

    // 3. the W x W count matrix (peer stores + a device barrier; copied to
    //    mapped host memory, and the offsets derived on the device), then
    // 4. the dispatch into the owners' receive buffers, enqueued before the
    //    host reads the counts (rows that do not fit are skipped and sent
    //    again below after the buffers grow)
    const uint32_t me = (uint32_t)ep->rank;
    uint32_t* const* d_ctrl = ep->ctrl_ptrs.as<uint32_t*>();
    CK(ep->small.reserve((size_t)(3 * W + 1) * 4));
    const uint32_t* d_dst_off = ep->small.as<uint32_t>();
    const uint32_t* d_roff = d_dst_off + W;
    const uint32_t* d_sbase = d_roff + W + 1;
    auto upload_caps = [&]() -> int {
        std::vector<uint32_t> c(W);
        for (uint32_t q = 0; q < W; ++q)
            c[q] = (uint32_t)std::min<uint64_t>({ep->cap_x[q] / (2ull * H), ep->cap_meta[q] / 4, 0xFFFFFFFFull});
        CK(ep->cap_rows.reserve((size_t)W * 4));
        CK(cudaMemcpyAsync(ep->cap_rows.ptr, c.data(), (size_t)W * 4, cudaMemcpyHostToDevice, st));
        ep->cap_rows_H = H;
        ep->cap_rows_gen = ep->cap_gen;
        return 1;
    };
    auto dispatch = [&]() -> int {
        if (ep->cap_rows_H != H || ep->cap_rows_gen != ep->cap_gen) {
            if (!upload_caps()) return 0;
        }
        // the peer pointer table as of now: growing the buffers replaces it
        void** d_ptrs = ep->ptrs.as<void*>();
        if (n > 0 && d_ptrs) {
            CK(launch_kernel(ep_dispatch_kernel, dim3(std::min(ceil_div(n, 8u), 148u * 8u)), dim3(256), 0, st, false,
                             x, H, K, (const int32_t*)ep->meta.as<int32_t>(),
                             (const uint32_t*)ep->row_asg.as<uint32_t>(), n, (const uint32_t*)ep->off.as<uint32_t>(),
                             d_dst_off, (const uint32_t*)ep->cap_rows.as<uint32_t>(),
                             reinterpret_cast<uint16_t* const*>(d_ptrs), reinterpret_cast<int32_t* const*>(d_ptrs + W),
                             W));
            launches += 1;
        }
        CK(launch_kernel(ep_barrier_kernel, dim3(1), dim3(32), 0, st, false, d_ctrl, me, W, ++ep->epoch, errw));
        launches += 1;
        return 1;
    };
    const uint32_t e_counts = ++ep->epoch;
    CK(launch_kernel(ep_counts_kernel, dim3(1), dim3(32), 0, st, false, (const uint32_t*)ep->cnt.as<uint32_t>(),
                     d_ctrl, me, W, e_counts, ep->d_h_ctrl, ep->small.as<uint32_t>(), errw));
    launches += 1;
    if (!dispatch()) return 0;
    if (!ep_wait_counts(ep, e_counts, err)) return 0;
    auto M = [&](uint32_t r, uint32_t q) -> uint64_t { return ep->h_ctrl[(size_t)r * W + q]; };
    std::vector<uint64_t> n_of(W, 0), recv_of(W, 0);
    for (uint32_t r = 0; r < W; ++r) {
        for (uint32_t q = 0; q < W; ++q) {
            n_of[r] += M(r, q);
            recv_of[q] += M(r, q);
        }
    }
    if (n_of[me] != n) {
        set_err(err, "dispatch counted %llu rows for %u assignments", (unsigned long long)n_of[me], n);
        return 0;
    }
    const uint32_t n_recv = (uint32_t)recv_of[me];
    {
        std::vector<uint64_t> need_x(W), need_meta(W), need_ret(W);
        for (uint32_t q = 0; q < W; ++q) {
            need_x[q] = recv_of[q] * H * 2 + 16;
            need_meta[q] = recv_of[q] * 4 + 16;
            need_ret[q] = n_of[q] * H * 4 + 16;
        }
        const uint32_t gen = ep->cap_gen;
        if (!ep_ensure_capacity(ep, need_x, need_meta, need_ret, st, err)) return 0;
        // grown (every rank decides alike): send again into the new buffers
        if (ep->cap_gen != gen && !dispatch()) return 0;
    }
    ep->last_sent.assign(W, 0);
    ep->last_recv.assign(W, 0);
    for (uint32_t q = 0; q < W; ++q) {
        ep->last_sent[q] = (uint32_t)M(me, q);
        ep->last_recv[q] = (uint32_t)M(q, me);
    }
    uint16_t* recv_x = ep->recv_x.local.as<uint16_t>();
    void** d_ptrs = ep->ptrs.as<void*>();
    mark(3);
    mark(4);

    // 5. local experts on the received rows (after the shared expert's pass,
    //    which used the same workspace); the down GEMM stores other ranks'
    //    rows into their return buffers
    if (shared_rows) CK(cudaStreamWaitEvent(st, ep->ev_join, 0));
    CK(ep->yloc.reserve((size_t)std::max(n_recv, 1u) * H * 4));
    BsJob mj{};
    mj.ids = ep->recv_meta.local.as<int32_t>();
    mj.T = n_recv;
    mj.K = 1;
    mj.E = e_loc;
    mj.src = recv_x;
    mj.group_slot = ep->slots.as<uint32_t>();
    mj.y = ep->yloc.as<float>();
    mj.y_by_source = true;
    mj.ret_ptrs = reinterpret_cast<float* const*>(d_ptrs + 2 * W);
    mj.ret_roff = d_roff;
    mj.ret_base = d_sbase;
    mj.ret_rows = n_recv;
    mj.ret_world = W;
    if (n_recv > 0) {
        if (!run_blockscaled(eng, L, mj, st, nullptr, &launches, err)) return 0;
    }
    mark(5);

    // 6. once every rank's rows are back: combine in router order
    CK(launch_kernel(ep_barrier_kernel, dim3(1), dim3(32), 0, st, false, d_ctrl, me, W, ++ep->epoch, errw));
    launches += 1;
    if (T > 0) {
        CK(launch_combine(ep->ret.local.as<float>(), H, ep->pos.as<uint32_t>(), w, T, K,
                          shared ? ep->yshared.as<float>() : nullptr, y_bf16, y_f32, st, false));
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
    cudaStream_t st = eng->hstream;
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
