// Shared device helpers for the B200 (sm_100a) MoE expert-FFN kernels:
// mbarriers with bounded waits, bulk / tensor (TMA) copies, tcgen05
// (TMEM alloc, MMA, commit, loads and stores), and the repacked MXFP4 tile
// geometry.
#pragma once

#include <utility>

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace moe_b200 {

// ---------------------------------------------------------------------------
// Repacked MXFP4 weight tile ("wtile").
//
// A weight matrix [R rows x K cols] in the reference's GGUF layout (per row,
// ceil(K/32) blocks of 17 bytes: E8M0 scale, then 16 code bytes holding
// element j in the low nibble of byte j and element j+16 in the high nibble)
// is repacked once at upload into tiles of 128 rows x 64 K-elements:
//   bytes [0, 4096)     code words: word c (0..7) of row r (0..127) at
//                       (c*128 + r)*4 holds elements 8c..8c+7 of the tile's
//                       64.  Element 2i sits in the low half-word and 2i+1 at
//                       the same place in the high half-word, so pair i
//                       decodes to one bf16x2.  Within a half-word (sign s,
//                       magnitude bits m2 m1 m0 of an E2M1 code):
//                         pair 0: m at bits 0-2,  s at 9
//                         pair 1: m at bits 3-5,  s at 12
//                         pair 2: m at bits 6-8,  s at 15
//                         pair 3: m0 m1 at 10-11, m2 at 14, s at 13
//                       Pairs 0-2 then need one shift and one mask to land
//                       on bf16 bits (m at 6-8, s at 15); pair 3 needs three.
//   bytes [4096, 4352)  E8M0 scale bytes: sub-block s (0..1, 32 elements
//                       each) of row r at 4096 + s*128 + r.
// Tiles are ordered (row_tile, k_tile) row-tile major.  Rows past R and
// elements past K are zero codes.  Consecutive threads of a converter warp
// read consecutive words, so the shared-memory reads are conflict-free.
// ---------------------------------------------------------------------------
constexpr int kTileRows = 128;
constexpr int kTileK = 64;
constexpr int kTileCodeBytes = kTileRows * kTileK / 2;        // 4096
constexpr int kTileBytes = kTileCodeBytes + kTileRows * 2;    // 4352

__host__ __device__ constexpr uint32_t ceil_div(uint32_t a, uint32_t b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------------------
// Error word shared by all kernels of one engine.  A wait that exceeds its
// bound records where it gave up and returns instead of hanging the GPU.
// ---------------------------------------------------------------------------
enum : uint32_t {
    kErrNone = 0,
    kErrTimeoutLoadFull = 1,
    kErrTimeoutLoadEmpty = 2,
    kErrTimeoutAFull = 3,
    kErrTimeoutAEmpty = 4,
    kErrTimeoutAccFull = 5,
    kErrTimeoutAccEmpty = 6,
    kErrTimeoutRouterLoad = 7,
    kErrTimeoutPeer = 8,
    kErrBadExpert = 16,
    kErrAllExpertsMissing = 17,
};

__device__ __forceinline__ void record_error(uint32_t* err, uint32_t code) {
    if (err) atomicCAS(err, 0u, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking test of the phase with the given parity (no suspension).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity; gives up after ~2^31 SM clocks
// (about one second), records `code` and returns false.  `backoff` parks
// the warp for a short sleep between polls, for waiters whose latency does
// not matter (it leaves the issue slots to the warps on the critical path).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err, uint32_t code,
                                          bool backoff = false) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long start = clock64();
    while (true) {
        for (int i = 0; i < 32; ++i) {
            if (mbar_try_wait(bar, parity)) return true;
            if (backoff) __nanosleep(200);
        }
        if (clock64() - start > (1ll << 31)) {
            record_error(err, code);
            return false;
        }
    }
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  A kernel launched with the programmatic
// stream-serialization attribute may start while its predecessor in the
// stream still runs; pdl_wait() blocks the calling thread until the
// predecessor grid has completed and its writes are visible.  pdl_trigger()
// lets this grid's own dependent launch early.  Both are no-ops for a
// kernel launched the ordinary way.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... Exp, typename... Act>
inline cudaError_t launch_kernel(void (*kernel)(Exp...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                 bool pdl, Act&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl ? attr : nullptr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Act>(args)...);
}

// launch_kernel for clusters of two CTAs (grid.x even).
template <typename... Exp, typename... Act>
inline cudaError_t launch_kernel_cluster2(void (*kernel)(Exp...), dim3 grid, dim3 block, size_t smem,
                                          cudaStream_t st, bool pdl, Act&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Act>(args)...);
}

// ---------------------------------------------------------------------------
// Bulk and tensor copies; each one fills only the issuing CTA's shared memory.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t c0, int32_t c1,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int32_t c0, int32_t c1, int32_t c2,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
        "%4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

// Pulls a contiguous global range into L2 (no shared memory involved).
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulate).
__device__ __forceinline__ void mma_ts_bf16(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives on `bar` once every tcgen05 operation this thread issued so far
// has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// Instruction descriptor for kind::f16: fp32 D, bf16 A and B, both K-major,
// M = 128, N = n (multiple of 16, 16..256).
__device__ __forceinline__ uint32_t idesc_bf16_m128(uint32_t n) {
    return (1u << 4)            // D format f32
           | (1u << 7)          // A format bf16
           | (1u << 10)         // B format bf16
           | ((n >> 3) << 17)   // N / 8
           | ((128u >> 4) << 24);  // M / 16
}

// ---------------------------------------------------------------------------
// CTA pairs (a cluster of two CTAs on the two SMs of a TPC running one
// cta_group::2 MMA of M = 256): each CTA holds its 128 rows of A and half of
// the B rows in its own shared memory; the even CTA (rank 0) issues the MMAs
// and owns the barriers the MMA waits on.  Addresses of the rank-0 CTA's
// barriers are shared::cluster addresses from mapa.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// shared::cluster address of the variable at `p` in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_cluster(const void* p, uint32_t rank) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
    return a;
}

// Arrivals on another CTA's barrier.  Default (release, CTA-scope)
// semantics as for local arrivals: what the barriers order here is tensor-
// core and copy work (tcgen05 fences, complete_tx), not generic memory, and a
// cluster-scope release would first drain this thread's global stores.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cl) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cl) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx_cluster(uint32_t bar_cl, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cluster.b64 _, [%0], %1;" ::"r"(bar_cl), "r"(bytes)
                 : "memory");
}

// Every thread of both CTAs: arrive (release) and wait (acquire).
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Tensor loads into this CTA's shared memory whose completion is counted on
// the rank-0 CTA's barrier (bar_cl, a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int32_t c0, int32_t c1,
                                                 uint32_t bar_cl) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
        "%3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar_cl)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, int32_t c0, int32_t c1,
                                                 int32_t c2, uint32_t bar_cl) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
        "%3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar_cl)
        : "memory");
}

// TMEM of a CTA pair: one warp with the same warp index in each CTA executes
// these; both CTAs get the same columns.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Arrives on the barrier at this offset in each CTA of `mask` once the
// pair MMAs this thread issued so far have completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar, uint16_t mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(mask)
        : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (the layout a TMA SWIZZLE_128B box of 64 bf16 per row
// writes).  `addr` must lie in a 1024-byte aligned tile; advancing K by 16
// elements inside the 128-byte swizzle row adds 32 bytes to the address.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFF) >> 4);   // start address
    d |= (uint64_t)1 << 16;                   // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;         // stride byte offset: 8 rows x 128 B
    d |= (uint64_t)1 << 46;                   // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;                   // SWIZZLE_128B
    return d;
}

#define MOE_TMEM_ST32(taddr, v)                                                                              \
    asm volatile(                                                                                            \
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "  \
        "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, "    \
        "%32};" ::"r"(taddr),                                                                                \
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),  \
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),      \
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),     \
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])                  \
        : "memory")

// ---------------------------------------------------------------------------
// Block-scaled MMA (kind::mxf8f6f4): A = E2M1 weights, B = E4M3 activations,
// E8M0 scale factors for both in TMEM.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_bs(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
}

// The same MMA over a CTA pair (M = 256: rows 0-127 from the rank-0 CTA's
// A, 128-255 from the rank-1 CTA's at the same shared-memory offset; B rows
// [0, N/2) from the rank-0 CTA, [N/2, N) from the rank-1 CTA; each CTA's
// TMEM holds its rows' accumulator, its rows' A scales and all N B scales).
__device__ __forceinline__ void mma_bs_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
}

// Same MMA with A read from tensor memory ([a_tmem]: lane 0, first column of
// the 128-row A slice; one 32-bit column per 4 bytes of each row).
__device__ __forceinline__ void mma_bs_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], [%1], %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
}

// Instruction descriptor for kind::mxf8f6f4 block_scale: A E2M1, B E4M3,
// E8M0 scales, both operands K-major, M = m (128; 256 for a CTA pair),
// N = n; `sf_id` selects the byte of each 32-bit scale word (the 32-element
// K block inside a 128-K stage).
__device__ __forceinline__ uint32_t idesc_bs(uint32_t m, uint32_t n, uint32_t sf_id) {
    return (sf_id << 4)          // B scale-factor id
           | (5u << 7)           // A format E2M1
           | (0u << 10)          // B format E4M3
           | ((n >> 3) << 17)    // N / 8
           | (1u << 23)          // scale format E8M0
           | ((m >> 4) << 24)    // M / 16
           | (sf_id << 29);      // A scale-factor id
}
__device__ __forceinline__ uint32_t idesc_bs_m128(uint32_t n, uint32_t sf_id) { return idesc_bs(128, n, sf_id); }

// ---------------------------------------------------------------------------
// Block-scaled MMA on packed FP4 operands (kind::mxf4, the fast mode): A and
// B both E2M1, two codes per byte in shared memory, K = 64 per instruction,
// one E8M0 scale per 32 K (scale_vec::2X: the two scale bytes of an MMA are
// bytes sf_id and sf_id + 1 of each row's scale word, sf_id = 0 or 2).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_fp4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.scale_vec::2X [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
            d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
}

// Instruction descriptor for kind::mxf4: A and B E2M1, E8M0 scales, both
// K-major, M = 128, N = n, K = 64; `sf_id` (0 or 2) picks the scale bytes.
__device__ __forceinline__ uint32_t idesc_fp4_m128(uint32_t n, uint32_t sf_id) {
    return (sf_id << 4)          // B scale-factor id
           | (1u << 7)           // A format E2M1
           | (1u << 10)          // B format E2M1
           | ((n >> 3) << 17)    // N / 8
           | (1u << 23)          // scale format E8M0
           | ((128u >> 4) << 24) // M / 16
           | (sf_id << 29);      // A scale-factor id
}

// Shared-memory descriptor, K-major with 64-byte swizzle: 64-byte rows (128
// packed FP4 codes), 8-row groups 512 bytes apart (what a TMA SWIZZLE_64B box
// of 64 bytes per row writes).  `addr` lies in a 512-byte aligned tile;
// advancing K by 64 codes adds 32 bytes.
__device__ __forceinline__ uint64_t smem_desc_sw64(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFF) >> 4);   // start address
    d |= (uint64_t)1 << 16;                   // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(512 >> 4) << 32;          // stride byte offset: 8 rows x 64 B
    d |= (uint64_t)1 << 46;                   // descriptor version (sm_100)
    d |= (uint64_t)4 << 61;                   // SWIZZLE_64B
    return d;
}

// Two fp32 values to E2M1 codes by the hardware conversion (round to nearest
// even, saturating at +-6): the first argument in the low nibble.
__device__ __forceinline__ uint32_t cvt_e2m1x2(float lo, float hi) {
    uint32_t d;
    asm("{\n\t.reg .b8 t;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\t"
        "cvt.u32.u8 %0, t;\n\t}"
        : "=r"(d)
        : "f"(hi), "f"(lo));
    return d;
}

// Shared-memory descriptor of a 32 x 128-bit scale-factor block (no swizzle,
// 16-byte rows, 8-row core matrices 128 bytes apart), the source of
// tcgen05.cp.32x128b.
__device__ __forceinline__ uint64_t smem_desc_sf(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFF) >> 4);
    d |= (uint64_t)(128 >> 4) << 16;   // leading byte offset
    d |= (uint64_t)(128 >> 4) << 32;   // stride byte offset: next 8 rows
    d |= (uint64_t)1 << 46;            // descriptor version (sm_100)
    return d;                          // layout type 0: no swizzle
}

// Copies a 32-row x 128-bit scale block from shared memory to TMEM columns
// [taddr, taddr+4), replicated into all four lane quarters.
__device__ __forceinline__ void tmem_cp_sf(uint32_t taddr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

#define MOE_TMEM_ST16(taddr, v)                                                                              \
    asm volatile(                                                                                            \
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "  \
        "%13, %14, %15, %16};" ::"r"(taddr),                                                                 \
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),  \
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])                   \
        : "memory")

#define MOE_TMEM_ST8(taddr, v)                                                                               \
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr), \
                 "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])      \
                 : "memory")

#define MOE_TMEM_ST4(taddr, v)                                                                               \
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(v[0]),      \
                 "r"(v[1]), "r"(v[2]), "r"(v[3])                                                              \
                 : "memory")

#define MOE_TMEM_LD16(taddr, v)                                                                              \
    asm volatile(                                                                                            \
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "   \
        "%13, %14, %15}, [%16];"                                                                             \
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),   \
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),          \
          "=r"(v[15])                                                                                        \
        : "r"(taddr)                                                                                         \
        : "memory")

#define MOE_TMEM_LD32(taddr, v)                                                                              \
    asm volatile(                                                                                            \
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "   \
        "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "  \
        "[%32];"                                                                                             \
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),   \
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),          \
          "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),        \
          "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),        \
          "=r"(v[29]), "=r"(v[30]), "=r"(v[31])                                                              \
        : "r"(taddr)                                                                                         \
        : "memory")

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------
// MXFP4 decode helpers
// ---------------------------------------------------------------------------
// bf16x2 bit pattern of pair i (0..3) of a repacked code word (layout
// above).  A code (sign s, 3 magnitude bits m) becomes bf16 bits
// (s<<15)|(m<<6), the E2M1 value times 2^-126 (exactly; subnormal for m=1).
__device__ __forceinline__ uint32_t e2m1_pair_bits(uint32_t w, int i) {
    constexpr uint32_t kMask = 0x81C081C0u;
    if (i == 0) return (w << 6) & kMask;
    if (i == 1) return (w << 3) & kMask;
    if (i == 2) return w & kMask;
    return ((w >> 4) & 0x00C000C0u) | ((w >> 6) & 0x01000100u) | ((w << 2) & 0x80008000u);
}

// Bit positions of element e (0..7) of a code word: returns the position of
// magnitude bit b (0..2) or, for b == 3, of the sign.
__host__ __device__ constexpr int code_bit_pos(int e, int b) {
    const int base = (e & 1) ? 16 : 0;
    const int pair = e >> 1;
    if (pair < 3) return base + (b < 3 ? pair * 3 + b : pair * 3 + 9);
    constexpr int p3[4] = {10, 11, 14, 13};
    return base + p3[b];
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// Scale factors for E8M0 byte s: value = bits * 2^(s-1), applied as
// f1 = 2^(min(s,128)-1) and, only for s > 128, f2 = 2^(s-128) so neither
// factor overflows bf16.  Both are returned broadcast as bf16x2.
__device__ __forceinline__ uint32_t e8m0_f1(uint32_t s) {
    const uint32_t e = (s > 128u ? 128u : s) + 126u;
    const uint32_t h = e << 7;
    return h | (h << 16);
}
__device__ __forceinline__ uint32_t e8m0_f2(uint32_t s) {
    const uint32_t h = (s - 1u) << 7;
    return h | (h << 16);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

}  // namespace moe_b200
