// Allocation-free variant of moe_b200_group_tokens_by_expert.
//
// Some callers cannot allocate device memory while they run a layer: an
// engine whose residency cache owns the whole VRAM budget (every byte it does
// not hand out is already holding expert weights).  This entry point
// therefore never calls cudaMalloc, cudaFree or any allocating library
// routine.  Its working memory is the fixed array below, which every GPU that
// loads this library holds for the life of the process.
//
// The kernels are the same ones the allocating entry point launches (the
// deterministic radix passes of group.cu), so the two produce identical
// output for any input both accept.
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/moe_b200.h"
#include "common.cuh"
#include "kernels.h"

using namespace moe_b200;

namespace {

constexpr uint32_t kMaxN = MOE_B200_NOALLOC_MAX_ASSIGNMENTS;
// rows of per-bucket counts the sort needs at the maximum size: one per
// kSortTile items (sort_tiles in route.cu)
constexpr uint32_t kTilesMax = (kMaxN + kSortTile - 1) / kSortTile;
static_assert(kTilesMax * kSortTile >= kMaxN, "scratch tile-count rows cover the largest accepted input");

// Carve-up of the scratch array (byte offsets, each 256-aligned).
constexpr size_t align256(size_t v) { return (v + 255) / 256 * 256; }
constexpr size_t kOffIn = 0;                                               // AssignRec[kMaxN] input copy
constexpr size_t kOffSorted = align256(kOffIn + kMaxN * 16);               // AssignRec[kMaxN] sorted
constexpr size_t kOffOrd0 = align256(kOffSorted + kMaxN * 16);             // uint32[kMaxN]
constexpr size_t kOffOrd1 = align256(kOffOrd0 + kMaxN * 4);                // uint32[kMaxN]
constexpr size_t kOffKeys = align256(kOffOrd1 + kMaxN * 4);                // int32[kMaxN]
constexpr size_t kOffRank = align256(kOffKeys + kMaxN * 4);                // uint32[kMaxN]
constexpr size_t kOffBatches = align256(kOffRank + kMaxN * 4);             // uint32[kMaxN][4]
constexpr size_t kOffTiles = align256(kOffBatches + kMaxN * 16);           // uint32[kTilesMax][256]
constexpr size_t kOffGroup = align256(kOffTiles + kTilesMax * 256 * 4);    // 4 x uint32[257]
constexpr size_t kOffCount = align256(kOffGroup + 4 * 257 * 4);            // uint32 batch count
constexpr size_t kOffErr = kOffCount + 4;                                  // uint32 error word
constexpr size_t kScratchBytes = align256(kOffErr + 4);

}  // namespace

// The scratch.  In host code this name is only a host-side stand-in for the
// device array; its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

namespace {

std::mutex g_noalloc_mu;           // one call at a time in this process
uint8_t* g_noalloc_ptr[64] = {};   // device address of the array, per device

void noalloc_err(char* err, const char* msg) {
    if (err) snprintf(err, MOE_B200_ERR_LEN, "%s", msg);
}

}  // namespace

extern "C" MOE_B200_API int moe_b200_group_tokens_by_expert_noalloc(
    const moe_b200_assignment_t* assignments, uint32_t n, moe_b200_assignment_t* out_sorted,
    moe_b200_batch_t* out_batches, uint32_t max_batches, uint32_t* out_batch_count, char* err) {
    if (!assignments || n == 0 || !out_batch_count) {
        if (out_batch_count) *out_batch_count = 0;
        noalloc_err(err, "no assignments");
        return 0;
    }
    if (n > kMaxN) {
        *out_batch_count = 0;
        if (err) {
            snprintf(err, MOE_B200_ERR_LEN, "%u assignments exceed the allocation-free maximum of %u", n, kMaxN);
        }
        return 0;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        noalloc_err(err, "no current CUDA device");
        return 0;
    }
    if (!g_noalloc_ptr[dev]) {
        // First call on this device (with it current): resolve the array's
        // device address once.
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            if (err) snprintf(err, MOE_B200_ERR_LEN, "cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
            return 0;
        }
        g_noalloc_ptr[dev] = static_cast<uint8_t*>(p);
    }
    uint8_t* base = g_noalloc_ptr[dev];
    AssignRec* d_in = reinterpret_cast<AssignRec*>(base + kOffIn);
    AssignRec* d_sorted = reinterpret_cast<AssignRec*>(base + kOffSorted);
    uint32_t* ord0 = reinterpret_cast<uint32_t*>(base + kOffOrd0);
    uint32_t* ord1 = reinterpret_cast<uint32_t*>(base + kOffOrd1);
    int32_t* keys = reinterpret_cast<int32_t*>(base + kOffKeys);
    uint32_t* rank = reinterpret_cast<uint32_t*>(base + kOffRank);
    uint32_t* batches = reinterpret_cast<uint32_t*>(base + kOffBatches);
    uint32_t* tiles = reinterpret_cast<uint32_t*>(base + kOffTiles);
    uint32_t* grp = reinterpret_cast<uint32_t*>(base + kOffGroup);
    uint32_t* bcount = reinterpret_cast<uint32_t*>(base + kOffCount);
    uint32_t* errw = reinterpret_cast<uint32_t*>(base + kOffErr);

    cudaStream_t st = 0;
    // The array keeps the previous call's contents: the only word that must
    // start at zero is the error word (every other region is fully written
    // before it is read).
    if (cudaMemsetAsync(errw, 0, 4, st) != cudaSuccess ||
        cudaMemcpyAsync(d_in, assignments, (size_t)n * sizeof(AssignRec), cudaMemcpyHostToDevice, st) !=
            cudaSuccess) {
        noalloc_err(err, "copy of the assignments to the device failed");
        return 0;
    }
    uint32_t mx[3] = {0, 0, 0};
    for (uint32_t i = 0; i < n; ++i) {
        mx[0] = assignments[i].token_index > mx[0] ? assignments[i].token_index : mx[0];
        mx[1] = assignments[i].expert > mx[1] ? assignments[i].expert : mx[1];
        mx[2] = assignments[i].layer > mx[2] ? assignments[i].layer : mx[2];
    }
    GroupInfo gi{grp, grp + 257, grp + 2 * 257, grp + 3 * 257, 1, 0, 0};
    if (launch_iota(ord0, n, st) != cudaSuccess) {
        noalloc_err(err, "kernel launch failed");
        return 0;
    }
    uint32_t* in = ord0;
    uint32_t* out = ord1;
    for (int field = 0; field < 3; ++field) {
        if (mx[field] == 0) continue;
        for (int shift = 0; shift < 32 && (shift == 0 || (mx[field] >> shift) != 0); shift += 8) {
            if (launch_group_pass(d_in, in, out, n, field, shift, keys, tiles, rank, gi, errw, st) != cudaSuccess) {
                noalloc_err(err, "kernel launch failed");
                return 0;
            }
            uint32_t* t = in;
            in = out;
            out = t;
        }
    }
    if (launch_group_finish(d_in, in, n, d_sorted, batches, bcount, st) != cudaSuccess) {
        noalloc_err(err, "kernel launch failed");
        return 0;
    }
    uint32_t nb = 0;
    if (cudaMemcpy(&nb, bcount, 4, cudaMemcpyDeviceToHost) != cudaSuccess ||
        (out_sorted &&
         cudaMemcpy(out_sorted, d_sorted, (size_t)n * sizeof(AssignRec), cudaMemcpyDeviceToHost) != cudaSuccess) ||
        (out_batches && max_batches &&
         cudaMemcpy(out_batches, batches, (size_t)(nb < max_batches ? nb : max_batches) * 16,
                    cudaMemcpyDeviceToHost) != cudaSuccess)) {
        noalloc_err(err, "copy of the results to the host failed");
        return 0;
    }
    *out_batch_count = nb;
    if (out_batches && nb > max_batches) {
        noalloc_err(err, "more batches than max_batches");
        return 0;
    }
    return 1;
}
