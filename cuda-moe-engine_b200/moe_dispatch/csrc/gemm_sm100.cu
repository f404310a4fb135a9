// Persistent grouped GEMM on 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces the reference's expert stage (src/moe_dispatch/layer.py:159-182):
// grouped_linear over packed rows (experts.py:21-35, Triton in
// _triton_gemm.py:16-104) followed by swiglu_out (csrc/dispatch.cu:277-323).
//
// For expert e, packed rows [offsets[e], offsets[e+1]) are multiplied by the
// expert's K-major weight block:
//   plain :  out[r, c] = bf16( sum_k a[r,k] * w[e, c, k] )
//   swiglu:  g = bf16(a[r].w[e,c]),  u = bf16(a[r].w[e,I+c]),  out = bf16(silu(g)*u)
// The bf16 rounding of g and u reproduces the reference's materialised bf16
// projection before its SwiGLU kernel, so fusing does not change results.
//
// Structure (one CTA per SM, 320 threads):
//   warp 0       TMA producer: A tile 128x64 and B tile 256x64 (two 128-row
//                boxes) per stage, 128-byte swizzle, 4 stages of 48 KiB.
//   warp 1       TMEM allocator and single-thread MMA issuer:
//                tcgen05.mma.cta_group::1.kind::f16, M=128 N=256 K=16, fp32
//                accumulators in TMEM, two 256-column buffers so the epilogue
//                of one tile overlaps the main loop of the next.
//   warps 2..9   epilogue, two warps per TMEM lane quarter, each on half of
//                the tile's columns: tcgen05.ld 32 lanes x 32 columns, SwiGLU
//                or cast, masked 16-byte stores (rows past the expert's end
//                are skipped).
// Tiles are numbered on the device from `offsets` (no host sync): expert by
// expert, and inside an expert n-tile by n-tile over its m-tiles.  CTAs claim
// them in that order with an atomic counter as they become free, so the tiles
// in flight form one compact window: they share the expert's A rows, and each
// B tile streams from DRAM once.
//
// Every mbarrier wait is bounded (globaltimer); when one runs out the kernel
// records an error in its status word, stops issuing, waits (bounded) for its
// copies and MMAs in flight, frees its TMEM and returns.
#include "common.cuh"
#include "launch.h"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstring>
#include <mutex>

namespace moe {
namespace {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kUmmaK = 16;
constexpr int kStages = 4;
constexpr int kTileABytes = kBM * kBK * 2;
constexpr int kTileBBytes = kBN * kBK * 2;
constexpr int kStageBytes = kTileABytes + kTileBBytes;
constexpr int kBoxRows = 128;
constexpr int kBoxBytes = kBoxRows * kBK * 2;
constexpr int kPairBM = 2 * kBM;  // rows of the CTA-pair tile
constexpr int kTmemCols = 2 * kBN;
// Warps 0 and 1 load and issue; warps 2..9 are the epilogue, two per TMEM lane
// quarter (and so two per SM sub-partition), each taking half of a tile's
// output columns, so one warp's TMEM loads and SiLU latency hide the other's.
// (Measured with ncu: one warp per quarter left the MMA waiting for the SwiGLU
// epilogue, 2.19 M vs 1.97 M cycles; four per quarter gave 1.98 M.)
constexpr int kEpilogueThreads = 256;
constexpr int kEpilogueGroups = kEpilogueThreads / 128;  // warps per TMEM lane quarter
constexpr int kThreads = 64 + kEpilogueThreads;
constexpr int kMaxExperts = 1024;
constexpr uint64_t kWaitLimitNs = 4000000000ull;   // a wait that takes 4 s is an error
constexpr uint64_t kDrainLimitNs = 200000000ull;   // bounded drain after an error

constexpr int kTileRing = 4;                      // tiles claimed ahead of the consumers
constexpr int kBarrierBytes = (2 * kStages + 5 + 2 * kTileRing) * 8;
// shared tables: m-tile prefix [pairs+1], offsets [E+1], first row of each pair [pairs]
constexpr int kTableBytes = (3 * kMaxExperts + 2) * 4;
constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kBarrierBytes + 16 + kTileRing * 4 +
                           kTableBytes;

enum GemmStatus : int32_t {
    kStatusOk = 0,
    kStatusWaitTimeout = 1,
    kStatusSlotShared = 5,
    kStatusArrivalTimeout = 6,  // rows from a peer rank did not arrive in time
};

__device__ int32_t g_gemm_status;

// Dynamic tile scheduling.  Each launch owns one slot {claim counter, CTAs
// finished, CTAs entered}: a CTA's producer thread claims the next tile with one atomicAdd,
// so tiles are handed out in order as SMs become free (no SM idles while
// another still holds a queue of tiles, and the tiles in flight stay a
// compact window whose weights and rows are shared in L2).  The last CTA to
// finish zeroes the slot for its next user.  Eager launches cycle through
// the first kSchedEagerSlots slots; launches captured into a CUDA graph get
// the others, so a graph's slot is not handed to eager launches that may run
// beside it.  Two launches collide only if they run at the same time with
// hundreds of other launches issued between them, or if one captured graph is
// replayed on two streams at once.  Every CTA counts itself in on entry; a
// count past the grid size means a second launch is using the slot before the
// first has released it, and the kernel records status 5 (kStatusSlotShared):
// the tiles are then split between the two launches and both results are void.
constexpr int kSchedEagerSlots = 512;
constexpr int kSchedCaptureSlots = 512;
__device__ uint32_t g_tile_sched[kSchedEagerSlots + kSchedCaptureSlots][4];

struct GemmParams {
    const int32_t* offsets;
    __nv_bfloat16* out;
    int64_t ldo;         // output row stride in elements
    int n_out;           // output columns (intermediate for SwiGLU)
    int k_dim;
    int experts;
    int n_tiles;         // output column tiles
    int b_rows;          // weight rows per expert (2*I for SwiGLU, N otherwise)
    int up_offset;       // row offset of the "up" half inside an expert (SwiGLU)
    uint32_t* sched;     // this launch's {claim counter, CTAs finished, CTAs entered}
    const float* a_scale;  // e4m3 operands: dequantisation scale per A row
    const float* b_scale;  // e4m3 operands: dequantisation scale per weight row
    // Arrival groups (expert parallelism): an expert's rows come from `groups`
    // ranks one after another; group_rows[e * (groups + 1) + g] is the first row
    // (relative to the expert's span) of group g, group_rows[.. + groups] the
    // expert's real rows.  A tile belongs to the group of its last real row
    // and is loaded once arrival[source of that group and every group before]
    // reaches *epoch (group g comes from rank (me - g) mod ranks; group 0 is
    // this rank's own rows, already in place).  groups == 1: no waits.
    int groups;
    const int32_t* group_rows;
    const uint32_t* arrival;
    const int32_t* epoch;
    int ranks, me;
    uint64_t arrival_limit_ns;
};

// m-tile table of a launch, built by one warp: for every (group, expert) pair
// j = g * experts + e, the first row of its first tile and the exclusive prefix
// of the pairs' m-tile counts; with one group j = e.  Tiles of BM rows.
template <int BM>
__device__ void build_tile_table(const GemmParams& p, int lane, int* mt_prefix, int* offs,
                                 int* tbase) {
    for (int e = lane; e <= p.experts; e += 32) offs[e] = p.offsets[e];
    __syncwarp();
    const int pairs = p.experts * p.groups;
    int carry = 0;
    for (int j0 = 0; j0 < pairs; j0 += 32) {
        const int j = j0 + lane;
        int mt = 0;
        if (j < pairs) {
            const int e = j % p.experts, g = j / p.experts;
            const int lo = offs[e], hi = offs[e + 1];
            const int rows = hi - lo;
            const int tiles = rows > 0 ? (rows + BM - 1) / BM : 0;
            int first = 0;  // first m-tile of the pair
            mt = tiles;
            if (p.groups > 1) {
                // tiles whose last real row lies in groups 0..g-1, and 0..g
                const int* b = p.group_rows + static_cast<int64_t>(e) * (p.groups + 1);
                const int real = b[p.groups];
                first = g == 0 ? 0 : (b[g] >= real ? tiles : b[g] / BM);
                mt = (b[g + 1] >= real ? tiles : b[g + 1] / BM) - first;
            }
            tbase[j] = lo + first * BM;
        }
        int inclusive = mt;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, inclusive, off);
            if (lane >= off) inclusive += y;
        }
        if (j < pairs) mt_prefix[j] = carry + inclusive - mt;
        carry += __shfl_sync(0xffffffffu, inclusive, 31);
    }
    if (lane == 0) mt_prefix[pairs] = carry;
}

// ---------------------------------------------------------------- PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// The same with cluster-scope acquire: for phases completed by the other CTA
// of a pair, whose shared-memory writes must be visible after the wait.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ void record_status(int32_t code) { atomicCAS(&g_gemm_status, 0, code); }

// Bounded wait for the phase of `bar` with the given parity.  Returns false
// when the CTA is aborting (another role gave up) or this wait ran out.
template <bool kCluster = false>
__device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity,
                                            volatile int* abort_flag, uint64_t limit_ns) {
    const uint64_t start = global_timer();
    for (uint32_t i = 1;; ++i) {
        if (kCluster ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity)) return true;
        if ((i & 31) == 0) {
            if (*abort_flag) return false;
            if (global_timer() - start > limit_ns) {
                record_status(kStatusWaitTimeout);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          uint64_t limit_ns) {
    return mbar_try_wait(bar, parity) || mbar_wait_slow<false>(bar, parity, abort_flag, limit_ns);
}

__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort_flag, uint64_t limit_ns) {
    return mbar_try_wait_cluster(bar, parity) ||
           mbar_wait_slow<true>(bar, parity, abort_flag, limit_ns);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x,
                                            int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// K-major operand, 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes
// apart (SBO); the leading offset is unused for this layout (encoded as 1).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
           (static_cast<uint64_t>(2) << 61);
}

// Instruction descriptor: D fp32, both operands K-major, M x N; A and B bf16
// (format 1 for kind::f16) or e4m3 (format 0 for kind::f8f6f4).
constexpr uint32_t make_idesc(int m, int n, bool fp8 = false) {
    const uint32_t ab = fp8 ? 0u : ((1u << 7) | (1u << 10));
    return (1u << 4) | ab | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

// Elements of one 128-byte swizzled row: one k-block per pipeline stage.
template <bool kFp8> constexpr int stage_k() { return kFp8 ? 128 : kBK; }

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate));
}

// e4m3 x e4m3 -> fp32, K = 32 per instruction (32 bytes of each operand row).
__device__ __forceinline__ void umma_e4m3(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate));
}

template <bool kFp8>
__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b,
                                     uint32_t idesc, uint32_t accumulate) {
    if constexpr (kFp8) umma_e4m3(tmem_d, desc_a, desc_b, idesc, accumulate);
    else umma_bf16(tmem_d, desc_a, desc_b, idesc, accumulate);
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float round_bf16(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
}

// Next tile of this launch, or -1 once every tile has been claimed.
__device__ __forceinline__ int claim_tile(uint32_t* sched, int total_tiles) {
    const uint32_t t = atomicAdd(sched, 1u);
    return t < static_cast<uint32_t>(total_tiles) ? static_cast<int>(t) : -1;
}

// Called by one thread per CTA on entry: a slot already entered by a whole
// grid belongs to another launch still in flight.
__device__ __forceinline__ void enter_schedule(uint32_t* sched) {
    if (atomicAdd(sched + 2, 1u) >= gridDim.x) record_status(kStatusSlotShared);
}

// Called by one thread per CTA after the CTA's producer stopped claiming:
// the last CTA of the grid resets the slot.
__device__ __forceinline__ void finish_schedule(uint32_t* sched) {
    __threadfence();
    if (atomicAdd(sched + 1, 1u) == gridDim.x - 1) {
        atomicExch(sched, 0u);
        atomicExch(sched + 2, 0u);
        atomicExch(sched + 1, 0u);
    }
}

// Tile t -> (pair j, m-tile inside the pair, n-tile).  Tiles are ordered by
// pair (group-major, then expert); inside a pair by n-tile, then m-tile.
__device__ __forceinline__ void decode_tile(int t, const int* mt_prefix, int pairs, int n_tiles,
                                            int& j, int& m, int& n) {
    const int q = t / n_tiles;
    int lo = 0, hi = pairs - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (mt_prefix[mid] <= q) lo = mid;
        else hi = mid - 1;
    }
    j = lo;
    const int mt = mt_prefix[j + 1] - mt_prefix[j];
    const int local = t - mt_prefix[j] * n_tiles;
    n = local / mt;
    m = local - n * mt;
}

__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* addr) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
    return v;
}

// Producer side of the arrival groups: before the loads of a tile of group g,
// wait (bounded) until the rows of groups arrived+1..g are in place.  The
// rows were written by peers; the proxy fence orders the acquire before the
// TMA (async proxy) reads of them.  Returns false when the CTA is aborting.
__device__ __noinline__ bool wait_arrival(const GemmParams& p, int g, int& arrived,
                                          volatile int* abort_flag) {
    const uint32_t epoch = static_cast<uint32_t>(*p.epoch);
    for (int gg = arrived + 1; gg <= g; ++gg) {
        const int src = (p.me - gg + p.ranks) % p.ranks;
        const uint64_t start = global_timer();
        for (uint32_t i = 0; load_acquire_sys(p.arrival + src) < epoch; ++i) {
            if (*abort_flag) return false;
            if ((i & 63) == 63 && global_timer() - start > p.arrival_limit_ns) {
                record_status(kStatusArrivalTimeout);
                *abort_flag = 1;
                return false;
            }
            __nanosleep(128);
        }
        arrived = gg;
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");
    return true;
}

// Called by one thread of every CTA of a scatter launch after its stores: the
// last CTA to finish raises this rank's return flag on every rank.
__device__ __forceinline__ void raise_return_flags(const GemmScatter& scatter) {
    __threadfence_system();
    if (atomicAdd(scatter.ticket, 1) == static_cast<int>(gridDim.x) - 1) {
        __threadfence_system();
        const uint32_t epoch = static_cast<uint32_t>(*scatter.epoch);
        for (int r = 0; r < scatter.ranks; ++r) {
            uint32_t* flag = reinterpret_cast<uint32_t*>(scatter.base[r] + scatter.flags_offset) +
                             2 * kGemmScatterMaxRanks + scatter.me;
            asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(epoch) : "memory");
        }
        *scatter.ticket = 0;
    }
}

template <bool kSwiglu, bool kScatter = false, bool kFp8 = false>
__global__ void __launch_bounds__(kThreads, 1)
grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                    const __grid_constant__ CUtensorMap tmap_b, const GemmParams p,
                    const GemmScatter scatter) {
    static_assert(!(kSwiglu && kScatter), "the scatter epilogue is for the down GEMM");
    static_assert(!(kFp8 && kScatter), "the scatter epilogue takes bf16 operands");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* tiles = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    uint64_t* tmem_full = empty + kStages;
    uint64_t* tmem_empty = tmem_full + 2;
    uint64_t* drain = tmem_empty + 2;
    uint64_t* tile_full = drain + 1;
    uint64_t* tile_empty = tile_full + kTileRing;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tile_empty + kTileRing);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* tile_ring = reinterpret_cast<volatile int*>(tmem_slot + 4);
    int* mt_prefix = reinterpret_cast<int*>(tmem_slot + 4 + kTileRing);
    int* offs = mt_prefix + kMaxExperts + 1;  // shared copy of p.offsets: no global load per tile
    int* tbase = offs + kMaxExperts + 1;      // first row of each pair's first tile

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int kOutTile = kSwiglu ? kBN / 2 : kBN;
    constexpr int kStageK = stage_k<kFp8>();
    const int k_blocks = (p.k_dim + kStageK - 1) / kStageK;
    if (threadIdx.x == 32) enter_schedule(p.sched);
    pdl_trigger();  // the next kernel may launch and run its prologue

    // m-tile table (warp 0).
    if (warp == 0) {
        pdl_wait();  // offsets and rows come from the kernels before this launch
        build_tile_table<kBM>(p, lane, mt_prefix, offs, tbase);
    } else if (warp == 1) {
        if (lane == 0) {
            for (int s = 0; s < kStages; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], 1);
            }
            for (int a = 0; a < 2; ++a) {
                mbar_init(&tmem_full[a], 1);
                mbar_init(&tmem_empty[a], kEpilogueThreads);
            }
            for (int r = 0; r < kTileRing; ++r) {
                mbar_init(&tile_full[r], 1);
                mbar_init(&tile_empty[r], 1 + kEpilogueThreads);  // MMA thread + epilogue
            }
            mbar_init(drain, 1);
            *abort_flag = 0;
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        __syncwarp();
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (warp != 0) pdl_wait();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int pairs = p.experts * p.groups;
    const int total_tiles = mt_prefix[pairs] * p.n_tiles;

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------ TMA producer
            int stage = 0;
            uint32_t phase = 0;
            uint32_t armed = 0;            // stages armed at least once
            uint32_t last_parity = 0;      // parity of each stage's latest arm
            int ring = 0;
            uint32_t ring_phase = 0;
            int arrived = 0;  // arrival groups known to be in place
            // One claim is kept in reserve, so the atomic's round trip overlaps
            // the previous tile's loads instead of stalling the pipeline.
            int next = claim_tile(p.sched, total_tiles);
            for (;;) {
                const int t = *abort_flag ? -1 : next;
                // publish the claim (or the end) to the MMA thread and the epilogue
                if (!mbar_wait(&tile_empty[ring], ring_phase ^ 1u, abort_flag, kWaitLimitNs)) break;
                tile_ring[ring] = t;
                mbar_arrive(&tile_full[ring]);
                if (++ring == kTileRing) {
                    ring = 0;
                    ring_phase ^= 1u;
                }
                if (t < 0) break;
                next = claim_tile(p.sched, total_tiles);
                int j, m, n;
                decode_tile(t, mt_prefix, pairs, p.n_tiles, j, m, n);
                const int e = j % p.experts;
                if (j / p.experts > arrived && !wait_arrival(p, j / p.experts, arrived, abort_flag)) break;
                const int row0 = tbase[j] + m * kBM;
                const int brow = e * p.b_rows + n * kOutTile;
                const int brow2 = kSwiglu ? brow + p.up_offset : brow + kBoxRows;
                bool ok = true;
                for (int kb = 0; kb < k_blocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kWaitLimitNs)) {
                        ok = false;
                        break;
                    }
                    uint8_t* sa = tiles + stage * kStageBytes;
                    uint8_t* sb = sa + kTileABytes;
                    mbar_expect_tx(&full[stage], kStageBytes);
                    tma_load_2d(sa, &tmap_a, &full[stage], kb * kStageK, row0);
                    tma_load_2d(sb, &tmap_b, &full[stage], kb * kStageK, brow);
                    tma_load_2d(sb + kBoxBytes, &tmap_b, &full[stage], kb * kStageK, brow2);
                    armed |= 1u << stage;
                    last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
            }
            if (*abort_flag) {
                // Let every copy this thread started land before the CTA exits.
                for (int s = 0; s < kStages; ++s)
                    if (armed & (1u << s)) {
                        volatile int never = 0;
                        mbar_wait(&full[s], (last_parity >> s) & 1u, &never, kDrainLimitNs);
                    }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------------------------ MMA issuer
            constexpr uint32_t idesc = make_idesc(kBM, kBN, kFp8);
            int stage = 0;
            uint32_t phase = 0;
            int ring = 0;
            uint32_t ring_phase = 0;
            bool issued = false;
            for (int local = 0;; ++local) {
                if (!mbar_wait(&tile_full[ring], ring_phase, abort_flag, kWaitLimitNs)) break;
                const int t = tile_ring[ring];
                mbar_arrive(&tile_empty[ring]);
                if (++ring == kTileRing) {
                    ring = 0;
                    ring_phase ^= 1u;
                }
                if (t < 0) break;
                const int acc = local & 1;
                const uint32_t acc_phase = (local >> 1) & 1;
                if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, abort_flag, kWaitLimitNs)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + acc * kBN;
                bool ok = true;
                for (int kb = 0; kb < k_blocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, kWaitLimitNs)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(tiles + stage * kStageBytes);
                    const uint32_t b_addr = a_addr + kTileABytes;
#pragma unroll
                    for (int k = 0; k < kBK / kUmmaK; ++k)
                        umma<kFp8>(d, smem_desc_sw128(a_addr + k * kUmmaK * 2),
                                  smem_desc_sw128(b_addr + k * kUmmaK * 2), idesc,
                                  (kb | k) != 0 ? 1u : 0u);
                    issued = true;
                    umma_commit(&empty[stage]);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit(&tmem_full[acc]);
            }
            if (*abort_flag && issued) {
                // Wait for the MMAs in flight before TMEM is released.
                umma_commit(drain);
                volatile int never = 0;
                mbar_wait(drain, 0, &never, kDrainLimitNs);
            }
        }
    } else {
        // ---------------------------------------------------- epilogue
        const int quarter = warp & 3;  // TMEM lanes this warp may access
        const int group = (warp - 2) >> 2;  // which share of the output columns
        int ring = 0;
        uint32_t ring_phase = 0;
        for (int local = 0;; ++local) {
            if (!mbar_wait(&tile_full[ring], ring_phase, abort_flag, kWaitLimitNs)) break;
            const int t = tile_ring[ring];
            mbar_arrive(&tile_empty[ring]);
            if (++ring == kTileRing) {
                ring = 0;
                ring_phase ^= 1u;
            }
            if (t < 0) break;
            int j, m, n;
            decode_tile(t, mt_prefix, pairs, p.n_tiles, j, m, n);
            const int e = j % p.experts;
            const int acc = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            if (!mbar_wait(&tmem_full[acc], acc_phase, abort_flag, kWaitLimitNs)) break;
            tc_fence_after();
            const int64_t row = static_cast<int64_t>(tbase[j]) + m * kBM + quarter * 32 + lane;
            bool valid = row < offs[e + 1];
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kBN;
            __nv_bfloat16* dst_row = p.out + row * p.ldo;
            // e4m3: out = bf16((acc * row scale) * column scale); the row scale is
            // read once per tile, the column scales once per 32-column chunk
            float rscale = 1.0f, gscale = 1.0f, uscale = 1.0f;
            if constexpr (kFp8) rscale = valid ? __ldg(p.a_scale + row) : 0.0f;
            if constexpr (kScatter) {
                // the source rank and packed row this grouped row returns to
                valid = false;
                for (int src = 0; src < scatter.ranks; ++src) {
                    const int seg = src * scatter.local_experts + e;
                    const int64_t start = scatter.seg_start[seg];
                    if (row >= start && row < start + scatter.seg_count[seg]) {
                        const int64_t back = scatter.ret_dst[seg] + (row - start);
                        if (back < scatter.back_rows) {
                            valid = true;
                            dst_row = reinterpret_cast<__nv_bfloat16*>(
                                          scatter.base[src] + scatter.back_offset) + back * p.ldo;
                        }
                    }
                }
            }
#pragma unroll 1
            for (int c = group * (kOutTile / kEpilogueGroups); c < (group + 1) * (kOutTile / kEpilogueGroups);
                 c += 32) {
                uint32_t v[32];
                uint32_t outw[16];
                if constexpr (kSwiglu) {
                    uint32_t u[32];
                    tmem_ld32(taddr + c, v);
                    tmem_ld32(taddr + kBN / 2 + c, u);
                    if constexpr (kFp8) {
                        // lane l holds the scales of column col0 + l (gate and up rows)
                        const int col = n * kOutTile + c + lane;
                        const bool in = col < p.n_out;
                        gscale = in ? __ldg(p.b_scale + static_cast<int64_t>(e) * p.b_rows + col) : 0.0f;
                        uscale = in ? __ldg(p.b_scale + static_cast<int64_t>(e) * p.b_rows + p.up_offset + col) : 0.0f;
                    }
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        float a2[2];
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            float gv = __uint_as_float(v[2 * j + h]);
                            float uv = __uint_as_float(u[2 * j + h]);
                            if constexpr (kFp8) {
                                gv = (gv * rscale) * __shfl_sync(0xffffffffu, gscale, 2 * j + h);
                                uv = (uv * rscale) * __shfl_sync(0xffffffffu, uscale, 2 * j + h);
                            }
                            const float g = round_bf16(gv);
                            const float up = round_bf16(uv);
                            a2[h] = (g / (1.0f + expf(-g))) * up;
                        }
                        outw[j] = pack_bf16x2(a2[0], a2[1]);
                    }
                } else {
                    tmem_ld32(taddr + c, v);
                    if constexpr (kFp8) {
                        const int col = n * kOutTile + c + lane;
                        gscale = col < p.n_out ? __ldg(p.b_scale + static_cast<int64_t>(e) * p.b_rows + col) : 0.0f;
                    }
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        float lo = __uint_as_float(v[2 * j]), hi = __uint_as_float(v[2 * j + 1]);
                        if constexpr (kFp8) {
                            lo = (lo * rscale) * __shfl_sync(0xffffffffu, gscale, 2 * j);
                            hi = (hi * rscale) * __shfl_sync(0xffffffffu, gscale, 2 * j + 1);
                        }
                        outw[j] = pack_bf16x2(lo, hi);
                    }
                }
                if (valid) {
                    const int col0 = n * kOutTile + c;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        if (col0 + q * 8 + 8 <= p.n_out)
                            *reinterpret_cast<uint4*>(dst_row + col0 + q * 8) =
                                make_uint4(outw[4 * q], outw[4 * q + 1], outw[4 * q + 2], outw[4 * q + 3]);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&tmem_empty[acc]);
        }
        if constexpr (kScatter) __threadfence_system();  // results visible on their ranks
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                     "r"(kTmemCols));
    }
    if (threadIdx.x == 0) finish_schedule(p.sched);
    if constexpr (kScatter) {
        if (threadIdx.x == 0) raise_return_flags(scatter);
    }
}

// ------------------------------------------------- CTA-pair (cta_group::2) variant
//
// Two CTAs of a cluster share one 256 x 256 tile: each CTA stages its own 128
// rows of A and 128 rows of B (the gate half and the up half for SwiGLU,
// otherwise two consecutive 128-row halves), 6 stages of 32 KiB.  The even
// (leader) CTA issues tcgen05.mma.cta_group::2 with M=256, N=256, reading both
// CTAs' shared memory; each CTA's TMEM receives the accumulator of its own 128
// rows.  Both CTAs' TMA loads complete on the leader's full barrier (only the
// leader arms its byte count); the leader's commits arrive on both CTAs'
// barriers (multicast commit); both CTAs' epilogues release an accumulator on
// the leader's barrier.  Per SM this halves the B bytes of the 1-CTA tile.

constexpr int kPairStages = 6;
constexpr int kPairTileABytes = kBM * kBK * 2;     // this CTA's 128 rows of A
constexpr int kPairTileBBytes = kBoxRows * kBK * 2; // this CTA's 128 rows of B
constexpr int kPairStageBytes = kPairTileABytes + kPairTileBBytes;
constexpr int kPairBarrierBytes = (2 * kPairStages + 5 + 2 * kTileRing) * 8;
constexpr int kPairSmemBytes = 1024 + kPairStages * kPairStageBytes + kPairBarrierBytes + 16 +
                               kTileRing * 4 + kTableBytes;
// The scatter (fused return) epilogue stages each warp's 32 x 32 output chunk
// in 2 KiB of shared memory after the tables, to store it as row segments.
constexpr int kScatterStageOffset =
    (kPairStages * kPairStageBytes + kPairBarrierBytes + 16 + kTileRing * 4 + kTableBytes + 15) / 16 * 16;
constexpr int kScatterStageBytes = (kEpilogueThreads / 32) * 2048;
constexpr int kPairScatterSmemBytes = 1024 + kScatterStageOffset + kScatterStageBytes;
static_assert(kPairScatterSmemBytes <= 227 * 1024, "scatter epilogue staging fits in shared memory");

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of the same shared variable in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t map_to_cta(uint32_t local_addr, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
    return remote;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
                 : "memory");
}

__device__ __forceinline__ void st_cluster_s32(uint32_t cluster_addr, int value) {
    asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(cluster_addr), "r"(value) : "memory");
}

__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map,
                                                 uint32_t leader_bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void umma_bf16_pair(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b,
                                               uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_e4m3_pair(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b,
                                               uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate));
}

template <bool kFp8>
__device__ __forceinline__ void umma_pair(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b,
                                          uint32_t idesc, uint32_t accumulate) {
    if constexpr (kFp8) umma_e4m3_pair(tmem_d, desc_a, desc_b, idesc, accumulate);
    else umma_bf16_pair(tmem_d, desc_a, desc_b, idesc, accumulate);
}

// Arrives (once) on the barrier at this shared offset in both CTAs of the pair
// when every tcgen05 operation issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;" ::"r"(smem_u32(bar)), "h"(static_cast<uint16_t>(0x3))
        : "memory");
}

template <bool kSwiglu, bool kFp8 = false, bool kScatter = false>
__global__ void __launch_bounds__(kThreads, 1)
grouped_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a,
                         const __grid_constant__ CUtensorMap tmap_b, const GemmParams p,
                         const GemmScatter scatter) {
    static_assert(!(kScatter && (kSwiglu || kFp8)), "the scatter epilogue is for the bf16 down GEMM");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* tiles = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPairStages * kPairStageBytes);
    uint64_t* empty = full + kPairStages;
    uint64_t* tmem_full = empty + kPairStages;
    uint64_t* tmem_empty = tmem_full + 2;
    uint64_t* drain = tmem_empty + 2;
    uint64_t* tile_full = drain + 1;
    uint64_t* tile_empty = tile_full + kTileRing;   // used in the leader only
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tile_empty + kTileRing);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* tile_ring = reinterpret_cast<volatile int*>(tmem_slot + 4);
    int* mt_prefix = reinterpret_cast<int*>(tmem_slot + 4 + kTileRing);
    int* offs = mt_prefix + kMaxExperts + 1;  // shared copy of p.offsets: no global load per tile
    int* tbase = offs + kMaxExperts + 1;      // first row of each pair's first tile

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();  // 0 = leader, 1 = peer
    const bool leader = rank == 0;
    constexpr int kOutTile = kSwiglu ? kBN / 2 : kBN;
    constexpr int kStageK = stage_k<kFp8>();
    const int k_blocks = (p.k_dim + kStageK - 1) / kStageK;
    if (threadIdx.x == 32) enter_schedule(p.sched);
    pdl_trigger();  // the next kernel may launch and run its prologue

    // m-tile table of 256-row tiles (warp 0, both CTAs).
    if (warp == 0) {
        pdl_wait();  // offsets and rows come from the kernels before this launch
        build_tile_table<kPairBM>(p, lane, mt_prefix, offs, tbase);
    } else if (warp == 1) {
        if (lane == 0) {
            for (int s = 0; s < kPairStages; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], 1);
            }
            for (int a = 0; a < 2; ++a) {
                mbar_init(&tmem_full[a], 1);
                mbar_init(&tmem_empty[a], 2 * kEpilogueThreads);
            }
            // tile ring: the leader's producer claims; the leader's MMA thread,
            // both epilogues and the peer's producer release a slot
            for (int r = 0; r < kTileRing; ++r) {
                mbar_init(&tile_full[r], 1);
                mbar_init(&tile_empty[r], 2 + 2 * kEpilogueThreads);
            }
            mbar_init(drain, 1);
            *abort_flag = 0;
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        __syncwarp();
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    if (warp != 0) pdl_wait();
    tc_fence_before();
    cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int pairs = p.experts * p.groups;
    const int total_tiles = mt_prefix[pairs] * p.n_tiles;

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------ TMA producer (both CTAs)
            int stage = 0;
            uint32_t phase = 0;
            uint32_t armed = 0, last_parity = 0;
            int ring = 0;
            uint32_t ring_phase = 0;
            int arrived = 0;  // arrival groups known to be in place (each CTA waits for its own rows)
            // the leader keeps one claim in reserve (see the one-CTA kernel)
            int next = leader ? claim_tile(p.sched, total_tiles) : -1;
            for (;;) {
                int t;
                if (leader) {
                    t = *abort_flag ? -1 : next;
                    if (!mbar_wait(&tile_empty[ring], ring_phase ^ 1u, abort_flag, kWaitLimitNs)) break;
                    tile_ring[ring] = t;
                    st_cluster_s32(map_to_cta(smem_u32(const_cast<int*>(&tile_ring[ring])), 1), t);
                    mbar_arrive(&tile_full[ring]);
                    mbar_arrive_cluster(map_to_cta(smem_u32(&tile_full[ring]), 1));
                } else {
                    if (!mbar_wait_cluster(&tile_full[ring], ring_phase, abort_flag, kWaitLimitNs)) break;
                    t = tile_ring[ring];
                    mbar_arrive_cluster(map_to_cta(smem_u32(&tile_empty[ring]), 0));
                }
                if (++ring == kTileRing) {
                    ring = 0;
                    ring_phase ^= 1u;
                }
                if (t < 0) break;
                if (leader) next = claim_tile(p.sched, total_tiles);
                int j, m, n;
                decode_tile(t, mt_prefix, pairs, p.n_tiles, j, m, n);
                const int e = j % p.experts;
                if (j / p.experts > arrived && !wait_arrival(p, j / p.experts, arrived, abort_flag)) break;
                const int row0 = tbase[j] + m * kPairBM + static_cast<int>(rank) * kBM;
                const int brow0 = e * p.b_rows + n * kOutTile;
                const int brow = kSwiglu ? brow0 + (leader ? 0 : p.up_offset)
                                         : brow0 + static_cast<int>(rank) * kBoxRows;
                bool ok = true;
                for (int kb = 0; kb < k_blocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kWaitLimitNs)) {
                        ok = false;
                        break;
                    }
                    const uint32_t leader_full = map_to_cta(smem_u32(&full[stage]), 0);
                    uint8_t* sa = tiles + stage * kPairStageBytes;
                    if (leader) mbar_expect_tx(&full[stage], 2 * kPairStageBytes);
                    tma_load_2d_pair(sa, &tmap_a, leader_full, kb * kStageK, row0);
                    tma_load_2d_pair(sa + kPairTileABytes, &tmap_b, leader_full, kb * kStageK, brow);
                    armed |= 1u << stage;
                    last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == kPairStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
            }
            if (*abort_flag && leader) {
                for (int s = 0; s < kPairStages; ++s)
                    if (armed & (1u << s)) {
                        volatile int never = 0;
                        mbar_wait(&full[s], (last_parity >> s) & 1u, &never, kDrainLimitNs);
                    }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ------------------------------------------------ MMA issuer (leader only)
            constexpr uint32_t idesc = make_idesc(kPairBM, kBN, kFp8);
            int stage = 0;
            uint32_t phase = 0;
            int ring = 0;
            uint32_t ring_phase = 0;
            bool issued = false;
            for (int local = 0;; ++local) {
                if (!mbar_wait(&tile_full[ring], ring_phase, abort_flag, kWaitLimitNs)) break;
                const int t = tile_ring[ring];
                mbar_arrive(&tile_empty[ring]);
                if (++ring == kTileRing) {
                    ring = 0;
                    ring_phase ^= 1u;
                }
                if (t < 0) break;
                const int acc = local & 1;
                const uint32_t acc_phase = (local >> 1) & 1;
                if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, abort_flag, kWaitLimitNs)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + acc * kBN;
                bool ok = true;
                for (int kb = 0; kb < k_blocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, kWaitLimitNs)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(tiles + stage * kPairStageBytes);
                    const uint32_t b_addr = a_addr + kPairTileABytes;
#pragma unroll
                    for (int k = 0; k < kBK / kUmmaK; ++k)
                        umma_pair<kFp8>(d, smem_desc_sw128(a_addr + k * kUmmaK * 2),
                                       smem_desc_sw128(b_addr + k * kUmmaK * 2), idesc,
                                       (kb | k) != 0 ? 1u : 0u);
                    issued = true;
                    umma_commit_pair(&empty[stage]);
                    if (++stage == kPairStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit_pair(&tmem_full[acc]);
            }
            if (*abort_flag && issued) {
                umma_commit_pair(drain);
                volatile int never = 0;
                mbar_wait(drain, 0, &never, kDrainLimitNs);
            }
        }
    } else {
        // ---------------------------------------------------- epilogue (both CTAs)
        const int quarter = warp & 3;
        const int group = (warp - 2) >> 2;
        const uint32_t leader_empty0 = map_to_cta(smem_u32(&tmem_empty[0]), 0);
        const uint32_t leader_empty1 = map_to_cta(smem_u32(&tmem_empty[1]), 0);
        int ring = 0;
        uint32_t ring_phase = 0;
        for (int local = 0;; ++local) {
            if (!mbar_wait_cluster(&tile_full[ring], ring_phase, abort_flag, kWaitLimitNs)) break;
            const int t = tile_ring[ring];
            mbar_arrive_cluster(map_to_cta(smem_u32(&tile_empty[ring]), 0));
            if (++ring == kTileRing) {
                ring = 0;
                ring_phase ^= 1u;
            }
            if (t < 0) break;
            int j, m, n;
            decode_tile(t, mt_prefix, pairs, p.n_tiles, j, m, n);
            const int e = j % p.experts;
            const int acc = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            if (!mbar_wait(&tmem_full[acc], acc_phase, abort_flag, kWaitLimitNs)) break;
            tc_fence_after();
            const int64_t row = static_cast<int64_t>(tbase[j]) + m * kPairBM +
                                static_cast<int>(rank) * kBM + quarter * 32 + lane;
            bool valid = row < offs[e + 1];
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kBN;
            __nv_bfloat16* dst_row = p.out + row * p.ldo;
            // e4m3: out = bf16((acc * row scale) * column scale); the row scale is
            // read once per tile, the column scales once per 32-column chunk
            float rscale = 1.0f, gscale = 1.0f, uscale = 1.0f;
            if constexpr (kFp8) rscale = valid ? __ldg(p.a_scale + row) : 0.0f;
            if constexpr (kScatter) {
                // the source rank and packed row this grouped row returns to
                valid = false;
                for (int src = 0; src < scatter.ranks; ++src) {
                    const int seg = src * scatter.local_experts + e;
                    const int64_t start = scatter.seg_start[seg];
                    if (row >= start && row < start + scatter.seg_count[seg]) {
                        const int64_t back = scatter.ret_dst[seg] + (row - start);
                        if (back < scatter.back_rows) {
                            valid = true;
                            dst_row = reinterpret_cast<__nv_bfloat16*>(
                                          scatter.base[src] + scatter.back_offset) + back * p.ldo;
                        }
                    }
                }
            }
#pragma unroll 1
            for (int c = group * (kOutTile / kEpilogueGroups); c < (group + 1) * (kOutTile / kEpilogueGroups);
                 c += 32) {
                uint32_t v[32];
                uint32_t outw[16];
                if constexpr (kSwiglu) {
                    uint32_t u[32];
                    tmem_ld32(taddr + c, v);
                    tmem_ld32(taddr + kBN / 2 + c, u);
                    if constexpr (kFp8) {
                        // lane l holds the scales of column col0 + l (gate and up rows)
                        const int col = n * kOutTile + c + lane;
                        const bool in = col < p.n_out;
                        gscale = in ? __ldg(p.b_scale + static_cast<int64_t>(e) * p.b_rows + col) : 0.0f;
                        uscale = in ? __ldg(p.b_scale + static_cast<int64_t>(e) * p.b_rows + p.up_offset + col) : 0.0f;
                    }
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        float a2[2];
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            float gv = __uint_as_float(v[2 * j + h]);
                            float uv = __uint_as_float(u[2 * j + h]);
                            if constexpr (kFp8) {
                                gv = (gv * rscale) * __shfl_sync(0xffffffffu, gscale, 2 * j + h);
                                uv = (uv * rscale) * __shfl_sync(0xffffffffu, uscale, 2 * j + h);
                            }
                            const float g = round_bf16(gv);
                            const float up = round_bf16(uv);
                            a2[h] = (g / (1.0f + expf(-g))) * up;
                        }
                        outw[j] = pack_bf16x2(a2[0], a2[1]);
                    }
                } else {
                    tmem_ld32(taddr + c, v);
                    if constexpr (kFp8) {
                        const int col = n * kOutTile + c + lane;
                        gscale = col < p.n_out ? __ldg(p.b_scale + static_cast<int64_t>(e) * p.b_rows + col) : 0.0f;
                    }
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        float lo = __uint_as_float(v[2 * j]), hi = __uint_as_float(v[2 * j + 1]);
                        if constexpr (kFp8) {
                            lo = (lo * rscale) * __shfl_sync(0xffffffffu, gscale, 2 * j);
                            hi = (hi * rscale) * __shfl_sync(0xffffffffu, gscale, 2 * j + 1);
                        }
                        outw[j] = pack_bf16x2(lo, hi);
                    }
                }
                if constexpr (kScatter) {
                    // Rows go to peer ranks: instead of 32 scattered 16-byte
                    // pieces per store instruction (one row per lane), stage
                    // the 32 x 32 chunk in shared memory and store 64-byte row
                    // segments (lanes 4r..4r+3 write row r, 8 rows per
                    // instruction).  16-byte chunk q of row r sits at slot
                    // q ^ ((r >> 1) & 3): conflict-free writes and reads.
                    uint4* stage = reinterpret_cast<uint4*>(smem + kScatterStageOffset) + (warp - 2) * 128;
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        stage[lane * 4 + (q ^ ((lane >> 1) & 3))] =
                            make_uint4(outw[4 * q], outw[4 * q + 1], outw[4 * q + 2], outw[4 * q + 3]);
                    __syncwarp();
                    const int col0 = n * kOutTile + c;
                    const unsigned long long my_dst = reinterpret_cast<unsigned long long>(dst_row);
#pragma unroll
                    for (int step = 0; step < 4; ++step) {
                        const int r = step * 8 + (lane >> 2), q = lane & 3;
                        const uint4 v = stage[r * 4 + (q ^ ((r >> 1) & 3))];
                        const unsigned long long d = __shfl_sync(0xffffffffu, my_dst, r);
                        const int ok = __shfl_sync(0xffffffffu, valid ? 1 : 0, r);
                        if (ok && col0 + q * 8 + 8 <= p.n_out)
                            *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(d) + col0 + q * 8) = v;
                    }
                    __syncwarp();
                } else if (valid) {
                    const int col0 = n * kOutTile + c;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        if (col0 + q * 8 + 8 <= p.n_out)
                            *reinterpret_cast<uint4*>(dst_row + col0 + q * 8) =
                                make_uint4(outw[4 * q], outw[4 * q + 1], outw[4 * q + 2], outw[4 * q + 3]);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive_cluster(acc ? leader_empty1 : leader_empty0);
        }
        if constexpr (kScatter) __threadfence_system();  // results visible on their ranks
    }

    tc_fence_before();
    cluster_sync();  // no CTA leaves while its peer may still touch its memory
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                     "r"(kTmemCols));
    }
    if (threadIdx.x == 0) finish_schedule(p.sched);
    if constexpr (kScatter) {
        if (threadIdx.x == 0) raise_return_flags(scatter);
    }
}

// ------------------------------------------------------ operand-swapped pair tile
//
// The pair tile pads each expert's rows up to a multiple of 256, the MMA's M.
// Here the operands trade places: the weights are the M side (256 weight rows
// per tile, 128 in each CTA) and an expert's packed rows are the N side, which
// the instruction descriptor sets per tile in steps of 16.  An expert of R
// rows runs mt = ceil(R / 256) tiles of N = round_up(ceil(R / mt), 16) rows,
// so 1032 rows cost 5 x 208 MMA columns instead of 5 x 256 padded rows.  TMEM
// then holds out^T (lane = output column, TMEM column = packed row); the
// epilogue transposes each 32 x 32 chunk through shared memory and stores
// 64-byte row segments.
//
// SwiGLU: each CTA's 128 weight rows are 64 gate rows (TMEM lanes 0..63) and
// the matching 64 up rows (lanes 64..127).  A gate warp and the up warp of the
// same lanes and column group swap halves of each 32 x 32 chunk through shared
// memory (the gate warp gives its bf16-rounded g of rows 16..31, the up warp
// its u of rows 0..15; two buffers per warp pair, an mbarrier handshake with
// bounded waits), then each applies silu(g) * u to its 16 rows and stores
// them, so all eight epilogue warps share the SwiGLU work.
//
// The fp32 accumulation is the same sum over k in the same order as the other
// tiles, so the results are bit-identical to them (tested).
constexpr int kSwapPairs = 4;  // SwiGLU warp pairs (gate warp + up warp)
constexpr int kSwapBarrierBytes = (2 * kPairStages + 5 + 2 * kTileRing + 4 * kSwapPairs) * 8;
constexpr int kSwapStageOffset = (kPairStages * kPairStageBytes + kSwapBarrierBytes + 16 +
                                  kTileRing * 4 + kTableBytes + 127) / 128 * 128;
constexpr int kSwapStageBytes = (kEpilogueThreads / 32) * 2048;  // a 32 x 32 bf16 chunk per warp
constexpr int kSwapSmemBytes = 1024 + kSwapStageOffset + kSwapStageBytes;
static_assert(kSwapSmemBytes <= 227 * 1024, "swapped pair tile fits in shared memory");

// Packed rows in each of an expert's mt tiles (the MMA's N): the rows spread
// evenly over the tiles, rounded up to the N step of 16.  Never above 256,
// and the last tile always holds at least one real row.
__device__ __forceinline__ int swap_tile_cols(int rows, int mt) {
    return ((rows + mt - 1) / mt + 15) & ~15;
}

template <bool kSwiglu>
__global__ void __launch_bounds__(kThreads, 1)
grouped_gemm_swap_kernel(const __grid_constant__ CUtensorMap tmap_a,
                         const __grid_constant__ CUtensorMap tmap_b, const GemmParams p,
                         const GemmScatter) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* tiles = smem;  // per stage: 128 weight rows, then 128 packed rows
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPairStages * kPairStageBytes);
    uint64_t* empty = full + kPairStages;
    uint64_t* tmem_full = empty + kPairStages;
    uint64_t* tmem_empty = tmem_full + 2;
    uint64_t* drain = tmem_empty + 2;
    uint64_t* tile_full = drain + 1;
    uint64_t* tile_empty = tile_full + kTileRing;   // used in the leader only
    uint64_t* x_ready = tile_empty + kTileRing;     // [pair][buffer] up values written
    uint64_t* x_free = x_ready + 2 * kSwapPairs;    // [pair][buffer] buffer consumed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(x_free + 2 * kSwapPairs);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* tile_ring = reinterpret_cast<volatile int*>(tmem_slot + 4);
    int* mt_prefix = reinterpret_cast<int*>(tmem_slot + 4 + kTileRing);
    int* offs = mt_prefix + kMaxExperts + 1;
    int* tbase = offs + kMaxExperts + 1;
    __nv_bfloat16* chunks = reinterpret_cast<__nv_bfloat16*>(smem + kSwapStageOffset);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();  // 0 = leader, 1 = peer
    const bool leader = rank == 0;
    constexpr int kOutTile = kSwiglu ? kBN / 2 : kBN;  // output columns of a tile (both CTAs)
    const int k_blocks = (p.k_dim + kBK - 1) / kBK;
    if (threadIdx.x == 32) enter_schedule(p.sched);
    pdl_trigger();  // the next kernel may launch and run its prologue

    if (warp == 0) {
        pdl_wait();  // offsets and rows come from the kernels before this launch
        build_tile_table<kPairBM>(p, lane, mt_prefix, offs, tbase);
    } else if (warp == 1) {
        if (lane == 0) {
            for (int s = 0; s < kPairStages; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], 1);
            }
            for (int a = 0; a < 2; ++a) {
                mbar_init(&tmem_full[a], 1);
                mbar_init(&tmem_empty[a], 2 * kEpilogueThreads);
            }
            for (int r = 0; r < kTileRing; ++r) {
                mbar_init(&tile_full[r], 1);
                mbar_init(&tile_empty[r], 2 + 2 * kEpilogueThreads);
            }
            for (int i = 0; i < 2 * kSwapPairs; ++i) {  // both warps of a pair arrive
                mbar_init(&x_ready[i], 64);
                mbar_init(&x_free[i], 64);
            }
            mbar_init(drain, 1);
            *abort_flag = 0;
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        __syncwarp();
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    if (warp != 0) pdl_wait();
    tc_fence_before();
    cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int pairs = p.experts;  // one arrival group
    const int total_tiles = mt_prefix[pairs] * p.n_tiles;

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------ TMA producer (both CTAs)
            int stage = 0;
            uint32_t phase = 0;
            uint32_t armed = 0, last_parity = 0;
            int ring = 0;
            uint32_t ring_phase = 0;
            int next = leader ? claim_tile(p.sched, total_tiles) : -1;
            for (;;) {
                int t;
                if (leader) {
                    t = *abort_flag ? -1 : next;
                    if (!mbar_wait(&tile_empty[ring], ring_phase ^ 1u, abort_flag, kWaitLimitNs)) break;
                    tile_ring[ring] = t;
                    st_cluster_s32(map_to_cta(smem_u32(const_cast<int*>(&tile_ring[ring])), 1), t);
                    mbar_arrive(&tile_full[ring]);
                    mbar_arrive_cluster(map_to_cta(smem_u32(&tile_full[ring]), 1));
                } else {
                    if (!mbar_wait_cluster(&tile_full[ring], ring_phase, abort_flag, kWaitLimitNs)) break;
                    t = tile_ring[ring];
                    mbar_arrive_cluster(map_to_cta(smem_u32(&tile_empty[ring]), 0));
                }
                if (++ring == kTileRing) {
                    ring = 0;
                    ring_phase ^= 1u;
                }
                if (t < 0) break;
                if (leader) next = claim_tile(p.sched, total_tiles);
                int j, m, n;
                decode_tile(t, mt_prefix, pairs, p.n_tiles, j, m, n);
                const int cols = swap_tile_cols(offs[j + 1] - offs[j], mt_prefix[j + 1] - mt_prefix[j]);
                // this CTA's packed rows: the first or second half of the tile's N
                const int row0 = tbase[j] + m * cols + static_cast<int>(rank) * (cols >> 1);
                // this CTA's weight rows: 64 gate (+ 64 up) or 128 output columns
                const int wrow = j * p.b_rows + n * kOutTile + static_cast<int>(rank) * (kOutTile / 2);
                bool ok = true;
                for (int kb = 0; kb < k_blocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kWaitLimitNs)) {
                        ok = false;
                        break;
                    }
                    const uint32_t leader_full = map_to_cta(smem_u32(&full[stage]), 0);
                    uint8_t* sw = tiles + stage * kPairStageBytes;
                    if (leader) mbar_expect_tx(&full[stage], 2 * kPairStageBytes);
                    if constexpr (kSwiglu) {
                        // two 64-row boxes: gate rows, then the matching up rows
                        tma_load_2d_pair(sw, &tmap_b, leader_full, kb * kBK, wrow);
                        tma_load_2d_pair(sw + kPairTileABytes / 2, &tmap_b, leader_full, kb * kBK,
                                         wrow + p.up_offset);
                    } else {
                        tma_load_2d_pair(sw, &tmap_b, leader_full, kb * kBK, wrow);
                    }
                    tma_load_2d_pair(sw + kPairTileABytes, &tmap_a, leader_full, kb * kBK, row0);
                    armed |= 1u << stage;
                    last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == kPairStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
            }
            if (*abort_flag && leader) {
                for (int s = 0; s < kPairStages; ++s)
                    if (armed & (1u << s)) {
                        volatile int never = 0;
                        mbar_wait(&full[s], (last_parity >> s) & 1u, &never, kDrainLimitNs);
                    }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ------------------------------------------------ MMA issuer (leader only)
            constexpr uint32_t idesc_m = make_idesc(kPairBM, 0);  // N is set per tile
            int stage = 0;
            uint32_t phase = 0;
            int ring = 0;
            uint32_t ring_phase = 0;
            bool issued = false;
            for (int local = 0;; ++local) {
                if (!mbar_wait(&tile_full[ring], ring_phase, abort_flag, kWaitLimitNs)) break;
                const int t = tile_ring[ring];
                mbar_arrive(&tile_empty[ring]);
                if (++ring == kTileRing) {
                    ring = 0;
                    ring_phase ^= 1u;
                }
                if (t < 0) break;
                int j, m, n;
                decode_tile(t, mt_prefix, pairs, p.n_tiles, j, m, n);
                const int cols = swap_tile_cols(offs[j + 1] - offs[j], mt_prefix[j + 1] - mt_prefix[j]);
                const uint32_t idesc = idesc_m | (static_cast<uint32_t>(cols >> 3) << 17);
                const int acc = local & 1;
                const uint32_t acc_phase = (local >> 1) & 1;
                if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, abort_flag, kWaitLimitNs)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + acc * kBN;
                bool ok = true;
                for (int kb = 0; kb < k_blocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, kWaitLimitNs)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t w_addr = smem_u32(tiles + stage * kPairStageBytes);
                    const uint32_t r_addr = w_addr + kPairTileABytes;
#pragma unroll
                    for (int k = 0; k < kBK / kUmmaK; ++k)
                        umma_bf16_pair(d, smem_desc_sw128(w_addr + k * kUmmaK * 2),
                                       smem_desc_sw128(r_addr + k * kUmmaK * 2), idesc,
                                       (kb | k) != 0 ? 1u : 0u);
                    issued = true;
                    umma_commit_pair(&empty[stage]);
                    if (++stage == kPairStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit_pair(&tmem_full[acc]);
            }
            if (*abort_flag && issued) {
                umma_commit_pair(drain);
                volatile int never = 0;
                mbar_wait(drain, 0, &never, kDrainLimitNs);
            }
        }
    } else {
        // ---------------------------------------------------- epilogue (both CTAs)
        const int quarter = warp & 3;
        const int group = (warp - 2) >> 2;  // even or odd 32-column chunks of the tile
        const bool up_warp = kSwiglu && quarter >= 2;
        const int xpair = (quarter & 1) + 2 * group;  // SwiGLU: gate warp + up warp
        __nv_bfloat16* mine = chunks + (kSwiglu ? 2 * xpair : warp - 2) * 1024;
        // first output column of this warp's 32 TMEM lanes
        const int lane_col = static_cast<int>(rank) * (kOutTile / 2) + (kSwiglu ? (quarter & 1) : quarter) * 32;
        const uint32_t leader_empty0 = map_to_cta(smem_u32(&tmem_empty[0]), 0);
        const uint32_t leader_empty1 = map_to_cta(smem_u32(&tmem_empty[1]), 0);
        uint32_t handed = 0;  // chunks passed between the SwiGLU warp pair so far
        int ring = 0;
        uint32_t ring_phase = 0;
        bool ok = true;
        for (int local = 0; ok; ++local) {
            if (!mbar_wait_cluster(&tile_full[ring], ring_phase, abort_flag, kWaitLimitNs)) break;
            const int t = tile_ring[ring];
            mbar_arrive_cluster(map_to_cta(smem_u32(&tile_empty[ring]), 0));
            if (++ring == kTileRing) {
                ring = 0;
                ring_phase ^= 1u;
            }
            if (t < 0) break;
            int j, m, n;
            decode_tile(t, mt_prefix, pairs, p.n_tiles, j, m, n);
            const int cols = swap_tile_cols(offs[j + 1] - offs[j], mt_prefix[j + 1] - mt_prefix[j]);
            const int first = tbase[j] + m * cols;           // packed row of TMEM column 0
            const int real = min(cols, offs[j + 1] - first);  // columns holding real rows
            const int acc = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            if (!mbar_wait(&tmem_full[acc], acc_phase, abort_flag, kWaitLimitNs)) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kBN;
            const int col0 = n * kOutTile + lane_col;
#pragma unroll 1
            for (int c = group * 32; c < real; c += 64) {
                uint32_t v[32];
                tmem_ld32(taddr + c, v);
                tmem_wait_ld();
                // chunk[i][l]: packed row c + i, output column col0 + l
                __nv_bfloat16* chunk = mine;
                int buffer = 0;
                int first_row = 0, steps = 4;  // rows of the chunk this warp stores
                if constexpr (kSwiglu) {
                    buffer = 2 * xpair + (handed & 1);
                    const uint32_t use = (handed >> 1) & 1;
                    ++handed;
                    chunk = chunks + buffer * 1024;
                    // the gate warp keeps rows 0..15, the up warp rows 16..31
                    first_row = up_warp ? 16 : 0;
                    steps = 2;
                    const int give = 16 - first_row;
                    if (!mbar_wait(&x_free[buffer], use ^ 1u, abort_flag, kWaitLimitNs)) {
                        ok = false;
                        break;
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i)  // constant register indices, a warp-uniform select
                        chunk[(give + i) * 32 + lane] =
                            __float2bfloat16_rn(__uint_as_float(up_warp ? v[i] : v[16 + i]));
                    mbar_arrive(&x_ready[buffer]);
                    if (!mbar_wait(&x_ready[buffer], use, abort_flag, kWaitLimitNs)) {
                        ok = false;
                        break;
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int row = first_row + i;
                        const float mine_v = round_bf16(__uint_as_float(up_warp ? v[16 + i] : v[i]));
                        const float other = __bfloat162float(chunk[row * 32 + lane]);
                        const float g = up_warp ? other : mine_v;
                        const float up = up_warp ? mine_v : other;
                        chunk[row * 32 + lane] = __float2bfloat16_rn((g / (1.0f + expf(-g))) * up);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        chunk[i * 32 + lane] = __float2bfloat16_rn(__uint_as_float(v[i]));
                }
                __syncwarp();
                // packed row r of the chunk: 32 outputs, four 16-byte pieces;
                // lanes 4r..4r+3 store row r, eight rows per instruction
                const uint4* pieces = reinterpret_cast<const uint4*>(chunk);
#pragma unroll
                for (int step = 0; step < steps; ++step) {
                    const int r = first_row + step * 8 + (lane >> 2), q = lane & 3;
                    const int col = col0 + q * 8;
                    if (c + r < real && col + 8 <= p.n_out)
                        *reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(first + c + r) * p.ldo + col) =
                            pieces[r * 4 + q];
                }
                __syncwarp();
                if constexpr (kSwiglu) mbar_arrive(&x_free[buffer]);
            }
            tc_fence_before();
            mbar_arrive_cluster(acc ? leader_empty1 : leader_empty0);
        }
    }

    tc_fence_before();
    cluster_sync();  // no CTA leaves while its peer may still touch its memory
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                     "r"(kTmemCols));
    }
    if (threadIdx.x == 0) finish_schedule(p.sched);
}

// ------------------------------------------------------------------ host side

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult query;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &query) ==
                cudaSuccess &&
            query == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// Row-major matrix [rows, cols] of bf16 (or e4m3 bytes with fp8), boxes of
// box_rows rows x 128 bytes, 128B swizzle.
bool make_tensor_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                     bool fp8 = false, uint32_t box_rows = kBoxRows) {
    auto encode = tensor_map_encoder();
    if (!encode) return false;
    const uint64_t elem = fp8 ? 1 : 2;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * elem};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / elem), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t elem_strides[2] = {1, 1};
    return encode(map, fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, elem_strides,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct DeviceInfo {
    int sms = 0;
    int pair_clusters = 0;
    uint32_t* sched = nullptr;  // device address of g_tile_sched
    bool configured[2][2] = {};       // [fp8][swiglu]
    bool pair_configured[2][2] = {};  // [fp8][swiglu]
    bool swap_configured[2] = {};     // [swiglu]
    int swap_clusters = 0;
};

DeviceInfo& device_info(int device) {
    static DeviceInfo infos[64];
    return infos[device & 63];
}

// The scheduling slot of the next launch on `stream` (see g_tile_sched).
cudaError_t schedule_slot(DeviceInfo& info, cudaStream_t stream, uint32_t** slot) {
    static std::atomic<uint32_t> eager{0}, captured{0};
    if (!info.sched) {
        void* base = nullptr;
        MOE_CUDA_TRY(cudaGetSymbolAddress(&base, g_tile_sched));
        info.sched = static_cast<uint32_t*>(base);
    }
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    MOE_CUDA_TRY(cudaStreamIsCapturing(stream, &capture));
    const uint32_t index = capture == cudaStreamCaptureStatusActive
                               ? kSchedEagerSlots + captured.fetch_add(1) % kSchedCaptureSlots
                               : eager.fetch_add(1) % kSchedEagerSlots;
    *slot = info.sched + 4 * index;
    return cudaSuccess;
}

enum class Tile { kSingle, kPair };

// Tile shape selection (MOE_B200_GEMM_TILE=single|pair overrides).  The
// 256-row CTA-pair tile streams half the weight bytes per output row, and
// with claimed tiles and two epilogue warps per lane quarter it keeps the
// tensor pipe 90-95 % busy.  Measured in SM cycles on B200 (ncu), it wins or
// ties wherever experts average 512 rows or more (Mixtral gate/up 1.97 M vs
// 2.08 M, down 0.98 M vs 1.17 M; 64 experts x 1536 rows: 1.34 M vs 1.34 M,
// 0.69 M vs 0.77 M; 256 experts x 1024 rows: 15.2 M vs 16.2 M, 8.5 M vs
// 9.4 M).  With 256 rows per expert the rows it pads above each expert's
// last multiple of 256 make the one-CTA tile as fast or faster (5.12 M vs
// 4.94 M, 2.89 M vs 2.87 M).
Tile pick_tile(int64_t rows, int experts) {
    const char* env = getenv("MOE_B200_GEMM_TILE");
    if (env && strcmp(env, "pair") == 0) return Tile::kPair;
    if (env && strcmp(env, "single") == 0) return Tile::kSingle;
    return rows >= 512 * static_cast<int64_t>(experts) ? Tile::kPair : Tile::kSingle;
}

// The operand-swapped pair tile (MOE_B200_GEMM_SWAP=0 keeps the row-padded
// one): bf16 operands, rows of one arrival group.
bool use_swapped_pair() {
    const char* env = getenv("MOE_B200_GEMM_SWAP");
    return !(env && env[0] == '0');
}

template <typename Kernel>
cudaError_t launch_pair(Kernel kernel, int smem_bytes, bool& configured, int& resident_clusters,
                        int sms, int64_t max_tiles, const CUtensorMap& map_a, const CUtensorMap& map_b,
                        const GemmParams& p, cudaStream_t stream, const GemmScatter& scatter = {}) {
    cudaLaunchConfig_t config = {};
    cudaLaunchAttribute attribute[2];
    attribute[0].id = cudaLaunchAttributeClusterDimension;
    attribute[0].val.clusterDim.x = 2;
    attribute[0].val.clusterDim.y = 1;
    attribute[0].val.clusterDim.z = 1;
    // a dependent launch of the kernel before it (see pdl_wait)
    attribute[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[1].val.programmaticStreamSerializationAllowed = 1;
    config.blockDim = dim3(kThreads);
    config.dynamicSmemBytes = smem_bytes;
    config.stream = stream;
    config.attrs = attribute;
    config.numAttrs = 2;
    if (!configured) {
        MOE_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          smem_bytes));
        configured = true;
    }
    if (resident_clusters == 0) {
        config.gridDim = dim3(sms & ~1);
        int clusters = 0;
        MOE_CUDA_TRY(cudaOccupancyMaxActiveClusters(&clusters, kernel, &config));
        resident_clusters = clusters > 0 ? clusters : sms / 2;
    }
    const int64_t clusters = max_tiles < resident_clusters ? max_tiles : resident_clusters;
    config.gridDim = dim3(static_cast<unsigned>(2 * clusters));
    return cudaLaunchKernelEx(&config, kernel, map_a, map_b, p, scatter);
}

}  // namespace

cudaError_t launch_grouped_gemm(const void* a, const void* b, const int32_t* offsets, void* out,
                                int64_t rows, int64_t n_out, int64_t k_dim, int experts,
                                bool swiglu, cudaStream_t stream, const char** error,
                                const float* a_scale, const float* b_scale,
                                const GemmArrival* arrival) {
    const bool fp8 = a_scale != nullptr;
    *error = nullptr;
    if (rows == 0 || experts == 0) return cudaSuccess;
    const int groups = arrival ? arrival->groups : 1;
    if (groups < 1 || static_cast<int64_t>(experts) * groups > kMaxExperts) {
        *error = "grouped GEMM supports at most 1024 experts (times arrival groups)";
        return cudaErrorInvalidValue;
    }
    int device = 0;
    MOE_CUDA_TRY(cudaGetDevice(&device));
    DeviceInfo& info = device_info(device);
    if (info.sms == 0) MOE_CUDA_TRY(cudaDeviceGetAttribute(&info.sms, cudaDevAttrMultiProcessorCount, device));
    const int64_t b_rows = swiglu ? 2 * n_out : n_out;
    CUtensorMap map_a, map_b;
    if (!make_tensor_map(&map_a, a, static_cast<uint64_t>(rows), static_cast<uint64_t>(k_dim), fp8) ||
        !make_tensor_map(&map_b, b, static_cast<uint64_t>(b_rows * experts), static_cast<uint64_t>(k_dim), fp8)) {
        *error = "cuTensorMapEncodeTiled rejected an operand (pointer alignment or shape)";
        return cudaErrorInvalidValue;
    }
    GemmParams p;
    p.a_scale = a_scale;
    p.b_scale = b_scale;
    p.offsets = offsets;
    p.out = static_cast<__nv_bfloat16*>(out);
    p.ldo = n_out;
    p.n_out = static_cast<int>(n_out);
    p.k_dim = static_cast<int>(k_dim);
    p.experts = experts;
    const int out_tile = swiglu ? kBN / 2 : kBN;
    p.n_tiles = static_cast<int>((n_out + out_tile - 1) / out_tile);
    p.b_rows = static_cast<int>(b_rows);
    p.up_offset = swiglu ? static_cast<int>(n_out) : 0;
    p.groups = groups;
    p.group_rows = arrival ? arrival->group_rows : nullptr;
    p.arrival = arrival ? arrival->flags : nullptr;
    p.epoch = arrival ? arrival->epoch : nullptr;
    p.ranks = arrival ? arrival->ranks : 1;
    p.me = arrival ? arrival->me : 0;
    p.arrival_limit_ns = arrival ? arrival->limit_ns : 0;
    MOE_CUDA_TRY(schedule_slot(info, stream, &p.sched));

    const Tile tile = pick_tile(rows, experts);
    if (tile == Tile::kPair) {
        const int64_t max_tiles =
            ((rows + kPairBM - 1) / kPairBM + experts) * static_cast<int64_t>(p.n_tiles);
        if (!fp8 && groups == 1 && use_swapped_pair()) {
            // SwiGLU loads each CTA's gate and up weight rows as two 64-row boxes
            CUtensorMap map_w;
            if (swiglu && !make_tensor_map(&map_w, b, static_cast<uint64_t>(b_rows * experts),
                                           static_cast<uint64_t>(k_dim), false, kBoxRows / 2)) {
                *error = "cuTensorMapEncodeTiled rejected an operand (pointer alignment or shape)";
                return cudaErrorInvalidValue;
            }
            auto swapped = swiglu ? grouped_gemm_swap_kernel<true> : grouped_gemm_swap_kernel<false>;
            return launch_pair(swapped, kSwapSmemBytes, info.swap_configured[swiglu], info.swap_clusters,
                               info.sms, max_tiles, map_a, swiglu ? map_w : map_b, p, stream);
        }
        auto pair = fp8 ? (swiglu ? grouped_gemm_pair_kernel<true, true> : grouped_gemm_pair_kernel<false, true>)
                        : (swiglu ? grouped_gemm_pair_kernel<true, false> : grouped_gemm_pair_kernel<false, false>);
        return launch_pair(pair, kPairSmemBytes, info.pair_configured[fp8][swiglu], info.pair_clusters,
                           info.sms, max_tiles, map_a, map_b, p, stream);
    }
    auto kernel = fp8 ? (swiglu ? grouped_gemm_kernel<true, false, true> : grouped_gemm_kernel<false, false, true>)
                      : (swiglu ? grouped_gemm_kernel<true> : grouped_gemm_kernel<false>);
    if (!info.configured[fp8][swiglu]) {
        MOE_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
        info.configured[fp8][swiglu] = true;
    }
    const int64_t max_tiles = ((rows + kBM - 1) / kBM + experts) * static_cast<int64_t>(p.n_tiles);
    const int grid = static_cast<int>(max_tiles < info.sms ? max_tiles : info.sms);
    const GemmScatter none = {};
    return launch_dependent(kernel, dim3(grid), dim3(kThreads), kSmemBytes, stream, map_a, map_b, p,
                            none);
}

cudaError_t launch_grouped_gemm_scatter(const void* a, const void* b, const int32_t* offsets,
                                        int64_t rows, int64_t n_out, int64_t k_dim, int experts,
                                        const GemmScatter& scatter, cudaStream_t stream,
                                        const char** error) {
    *error = nullptr;
    if (experts > kMaxExperts) {
        *error = "grouped GEMM supports at most 1024 experts";
        return cudaErrorInvalidValue;
    }
    int device = 0;
    MOE_CUDA_TRY(cudaGetDevice(&device));
    DeviceInfo& info = device_info(device);
    if (info.sms == 0) MOE_CUDA_TRY(cudaDeviceGetAttribute(&info.sms, cudaDevAttrMultiProcessorCount, device));
    static bool configured[64] = {};
    static bool pair_configured[64] = {};
    auto kernel = grouped_gemm_kernel<false, true>;
    if (!configured[device & 63]) {
        MOE_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
        configured[device & 63] = true;
    }
    CUtensorMap map_a, map_b;
    const uint64_t a_rows = static_cast<uint64_t>(rows > 0 ? rows : 1);
    if (!make_tensor_map(&map_a, a, a_rows, static_cast<uint64_t>(k_dim)) ||
        !make_tensor_map(&map_b, b, static_cast<uint64_t>(n_out * experts), static_cast<uint64_t>(k_dim))) {
        *error = "cuTensorMapEncodeTiled rejected an operand (pointer alignment or shape)";
        return cudaErrorInvalidValue;
    }
    GemmParams p;
    p.offsets = offsets;
    p.out = nullptr;
    p.ldo = n_out;
    p.n_out = static_cast<int>(n_out);
    p.k_dim = static_cast<int>(k_dim);
    p.experts = experts;
    p.n_tiles = static_cast<int>((n_out + kBN - 1) / kBN);
    p.b_rows = static_cast<int>(n_out);
    p.up_offset = 0;
    p.a_scale = p.b_scale = nullptr;
    p.groups = 1;
    p.group_rows = nullptr;
    p.arrival = nullptr;
    p.epoch = nullptr;
    p.ranks = 1;
    p.me = 0;
    p.arrival_limit_ns = 0;
    MOE_CUDA_TRY(schedule_slot(info, stream, &p.sched));
    // Every CTA takes part in the completion ticket, so the grid never depends
    // on the rows (rows = the grouped capacity, an upper bound).
    if (pick_tile(rows, experts) == Tile::kPair) {
        static int resident[64] = {};  // every resident cluster, whatever the rows
        return launch_pair(grouped_gemm_pair_kernel<false, false, true>, kPairScatterSmemBytes,
                           pair_configured[device & 63], resident[device & 63], info.sms, INT64_MAX,
                           map_a, map_b, p, stream, scatter);
    }
    return launch_dependent(kernel, dim3(info.sms), dim3(kThreads), kSmemBytes, stream, map_a, map_b,
                            p, scatter);
}

bool grouped_gemm_uses_pair(int64_t rows, int experts) {
    return pick_tile(rows, experts) == Tile::kPair;
}

cudaError_t read_gemm_status(int32_t* code, bool clear) {
    MOE_CUDA_TRY(cudaMemcpyFromSymbol(code, g_gemm_status, sizeof(int32_t)));
    if (clear) {
        const int32_t zero = 0;
        MOE_CUDA_TRY(cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(int32_t)));
    }
    return cudaSuccess;
}

}  // namespace moe
