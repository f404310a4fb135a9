// Expert-parallel exchange over NVLink peer memory, with no host synchronisation.
//
// Every rank owns one "region" in its own HBM, shared with the other ranks of
// one node through CUDA IPC (moe_peer_alloc / moe_peer_open).  Its layout is the
// same on every rank (moe_ep_p2p_region_bytes):
//   inbox   int32 [P][E]     rank s writes its per-expert row counts into row s
//   flags   uint32 [3][P]    count / rows / return flags; source s sets slot s
//   grouped bf16 [G][H]      rows for this rank's experts, expert-major (written by senders)
//   back    bf16 [B][H]      this rank's packed rows after the experts (written by owners)
//
// One forward step on rank `me` (all ranks run the same sequence):
//   1. exchange_counts: write counts[E] into every rank's inbox row `me`, raise
//      the count flag, wait for all P flags; then, with the full [P][E] count
//      matrix local, compute every table below in one CTA.
//   2. send_rows: copy each packed row to its expert owner's grouped buffer, at
//      offsets[e] + sum_{s < me} counts[s][e] + slot (16-byte peer stores); the
//      last CTA raises the rows flag on every rank.
//   3. wait(rows), then the grouped GEMMs run on the local grouped buffer.
//   4. return_rows: copy each result row back to its source's `back` buffer at
//      the source's packed position; the last CTA raises the return flags.
//   5. wait(return), then combine reads `back` in packed order.
// Flags carry a step number (epoch) kept in device memory, so no flag is ever
// reset and the whole step can be captured in a CUDA graph.  Inside an
// expert, rows are source-major -- the global token order -- so the grouped rows
// equal what one GPU packs for these experts.
//
// Every wait is bounded by `timeout_ms`; when it runs out the kernel records
// status 2 in the status word read by moe_device_status and returns.
#include "common.cuh"
#include "launch.h"

#include <cstdlib>

namespace moe {
namespace {

constexpr int kMaxRanks = kEpP2pMaxRanks;

__device__ int32_t g_ep_status;

struct Regions {
    char* base[kMaxRanks];
};

struct Layout {
    int64_t inbox, flags, grouped, back, total;
};

__host__ __device__ inline int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline Layout region_layout(int ranks, int experts, int64_t hidden,
                                                int64_t grouped_rows, int64_t back_rows) {
    Layout l;
    l.inbox = 0;
    l.flags = align_up(static_cast<int64_t>(ranks) * experts * 4, 256);
    l.grouped = align_up(l.flags + 3 * kMaxRanks * 4, 1024);
    l.back = align_up(l.grouped + grouped_rows * hidden * 2, 1024);
    l.total = align_up(l.back + back_rows * hidden * 2, 1024);
    return l;
}

// Local state words (int32), per rank: see state_words().
struct State {
    int32_t* epoch;        // [1]  step number of the current step
    int32_t* counters;     // [2]  last-CTA tickets for send / return
    int32_t* send_dst;     // [E]  grouped row on the owner where my rows of expert e start
    int32_t* offsets;      // [E_l + 1] my grouped expert spans (aligned)
    int32_t* seg_start;    // [P][E_l] grouped row where source s's rows of my expert start
    int32_t* seg_count;    // [P][E_l] rows from source s for my expert
    int32_t* ret_dst;      // [P][E_l] packed row on source s where they go back
    int32_t* recv_prefix;  // [P*E_l + 1] source-major prefix of seg_count
    int32_t* owner_total;  // [P]  rows I send to each owner
    int32_t* owner_done;   // [P]  rows of them stored so far (remote send)
    int32_t* group_rows;   // [E_l][P + 1] first row of each arrival group inside my expert
};

__host__ __device__ inline State state_view(int32_t* base, int ranks, int experts) {
    const int local = experts / ranks;
    State s;
    s.epoch = base;
    s.counters = base + 1;
    s.send_dst = base + 4;
    s.offsets = s.send_dst + experts;
    s.seg_start = s.offsets + local + 1;
    s.seg_count = s.seg_start + ranks * local;
    s.ret_dst = s.seg_count + ranks * local;
    s.recv_prefix = s.ret_dst + ranks * local;
    s.owner_total = s.recv_prefix + ranks * local + 1;
    s.owner_done = s.owner_total + ranks;
    s.group_rows = s.owner_done + ranks;
    return s;
}

// Inside an expert's grouped span on owner o the sources' rows follow the
// order in which they arrive: o's own rows first, then those of o-1, o-2, ...
// (mod P) -- the shifted send schedule reaches owner o from o-1 first.  GEMM
// rows are independent, so the order does not change any result bit.
__host__ __device__ inline int arrival_pos(int owner, int source, int ranks) {
    return (owner - source + ranks) % ranks;
}
__host__ __device__ inline int arrival_source(int owner, int pos, int ranks) {
    return (owner - pos + ranks) % ranks;
}

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void store_release_sys(uint32_t* addr, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* addr) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
    return v;
}

// Bounded wait until flags[s] >= epoch for s < ranks (one thread per source).
// Returns false (and records the status) when the limit runs out.
__device__ bool wait_flags(const uint32_t* flags, int ranks, uint32_t epoch, uint64_t limit_ns) {
    __shared__ int failed;
    if (threadIdx.x == 0) failed = 0;
    __syncthreads();
    if (threadIdx.x < ranks) {
        const uint64_t start = now_ns();
        while (load_acquire_sys(flags + threadIdx.x) < epoch) {
            if (now_ns() - start > limit_ns) {
                atomicCAS(&g_ep_status, 0, 2);
                failed = 1;
                break;
            }
            __nanosleep(64);
        }
    }
    __syncthreads();
    return failed == 0;
}

// One warp copies one row: batches of 8 16-byte loads per lane are issued
// before their stores, so each lane keeps 128 bytes in flight (peer stores over
// NVLink need many outstanding requests to reach link bandwidth).
__device__ __forceinline__ void warp_copy_row(uint4* __restrict__ target, const uint4* __restrict__ source,
                                              int64_t row_vecs, int lane) {
    constexpr int kBatch = 8;
    for (int64_t c0 = lane; c0 < row_vecs; c0 += 32 * kBatch) {
        uint4 v[kBatch];
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
            const int64_t c = c0 + 32 * b;
            if (c < row_vecs) v[b] = __ldg(source + c);
        }
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
            const int64_t c = c0 + 32 * b;
            if (c < row_vecs) target[c] = v[b];
        }
    }
}

constexpr int kCopyThreads = 256;

__global__ void __launch_bounds__(1024)
ep_exchange_counts_kernel(const int32_t* __restrict__ counts, Regions regions, int32_t* state_base,
                          int ranks, int me, int experts, int alignment, int64_t hidden,
                          int64_t grouped_rows, int64_t back_rows, uint64_t limit_ns) {
    const Layout l = region_layout(ranks, experts, hidden, grouped_rows, back_rows);
    State st = state_view(state_base, ranks, experts);
    const int local = experts / ranks;
    const uint32_t epoch = static_cast<uint32_t>(*st.epoch) + 1u;
    const int tid = threadIdx.x;
    // 1. my counts into every rank's inbox row `me`
    for (int i = tid; i < ranks * experts; i += blockDim.x) {
        const int d = i / experts, e = i % experts;
        int32_t* inbox = reinterpret_cast<int32_t*>(regions.base[d] + l.inbox);
        inbox[me * experts + e] = counts[e];
    }
    __threadfence_system();
    __syncthreads();
    if (tid < ranks) {
        uint32_t* flags = reinterpret_cast<uint32_t*>(regions.base[tid] + l.flags);
        store_release_sys(flags + me, epoch);  // count flag of source `me` on rank tid
    }
    const uint32_t* my_flags = reinterpret_cast<const uint32_t*>(regions.base[me] + l.flags);
    if (!wait_flags(my_flags, ranks, epoch, limit_ns)) return;
    const int32_t* inbox = reinterpret_cast<const int32_t*>(regions.base[me] + l.inbox);

    // 2. tables.  Expert e's grouped span on its owner d = e / local:
    //    offsets_d[e_l] = sum_{e' < e, same owner} align(sum_s counts[s][e']).
    extern __shared__ int32_t sm[];
    int32_t* span = sm;  // [E] aligned total rows per expert
    for (int e = tid; e < experts; e += blockDim.x) {
        int total = 0;
        for (int s = 0; s < ranks; ++s) total += inbox[s * experts + e];
        span[e] = alignment > 1 ? (total + alignment - 1) / alignment * alignment : total;
    }
    __syncthreads();
    for (int e = tid; e < experts; e += blockDim.x) {
        const int owner = e / local, owner_first = owner * local;
        int start = 0;
        for (int e2 = owner_first; e2 < e; ++e2) start += span[e2];
        int before = 0;  // rows of sources that come before me on this owner
        for (int g = 0; g < arrival_pos(owner, me, ranks); ++g)
            before += inbox[arrival_source(owner, g, ranks) * experts + e];
        st.send_dst[e] = start + before;
    }
    for (int o = tid; o < ranks; o += blockDim.x) {
        int total = 0;
        for (int e_l = 0; e_l < local; ++e_l) total += inbox[me * experts + o * local + e_l];
        st.owner_total[o] = total;
        st.owner_done[o] = 0;
    }
    if (tid == 0) {
        int run = 0;
        for (int e_l = 0; e_l < local; ++e_l) {
            st.offsets[e_l] = run;
            run += span[me * local + e_l];
        }
        st.offsets[local] = run;
        run = 0;
        for (int s = 0; s < ranks; ++s)
            for (int e_l = 0; e_l < local; ++e_l) {
                st.recv_prefix[s * local + e_l] = run;
                run += inbox[s * experts + me * local + e_l];
            }
        st.recv_prefix[ranks * local] = run;
    }
    __syncthreads();
    for (int e_l = tid; e_l < local; e_l += blockDim.x) {
        const int e = me * local + e_l;
        int run = 0;
        for (int g = 0; g < ranks; ++g) {
            st.group_rows[e_l * (ranks + 1) + g] = run;
            run += inbox[arrival_source(me, g, ranks) * experts + e];
        }
        st.group_rows[e_l * (ranks + 1) + ranks] = run;
    }
    for (int i = tid; i < ranks * local; i += blockDim.x) {
        const int s = i / local, e_l = i % local, e = me * local + e_l;
        int before = 0;
        for (int g = 0; g < arrival_pos(me, s, ranks); ++g)
            before += inbox[arrival_source(me, g, ranks) * experts + e];
        st.seg_start[i] = st.offsets[e_l] + before;
        st.seg_count[i] = inbox[s * experts + e];
        int packed = 0;  // source s packs compactly, expert-major
        for (int e2 = 0; e2 < e; ++e2) packed += inbox[s * experts + e2];
        st.ret_dst[i] = packed;
    }
    __syncthreads();
    if (tid == 0) *st.epoch = static_cast<int32_t>(epoch);
}

// Which rows a send launch moves.
enum SendMode { kSendAll = 0, kSendLocal = 1, kSendRemote = 2 };

// Rows of my compact packed buffer -> their owners' grouped buffers (a warp per row).
//   kSendAll     every row; the last CTA raises the rows flag of source `me`
//                on every rank.
//   kSendLocal   only the rows of my own experts (an HBM copy); no flag -- the
//                launches after it on the stream see them.
//   kSendRemote  only the rows of other ranks' experts.  Each warp counts its
//                stored row for the row's owner; the warp that completes an
//                owner's rows raises the rows flag of source `me` on that owner,
//                so an owner can start on my rows while I still send to others.
//                CTA 0 raises it at once on owners I send nothing, and on
//                myself (my own rows are kSendLocal's, ordered by the stream).
template <int kMode>
__global__ void __launch_bounds__(kCopyThreads)
ep_send_rows_kernel(const uint4* __restrict__ packed, const int32_t* __restrict__ dispatch_offsets,
                    Regions regions, int32_t* state_base, int ranks, int me, int experts,
                    int64_t row_vecs, int64_t hidden, int64_t grouped_rows, int64_t back_rows) {
    const Layout l = region_layout(ranks, experts, hidden, grouped_rows, back_rows);
    State st = state_view(state_base, ranks, experts);
    const int local = experts / ranks;
    const int lane = threadIdx.x & 31;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (kCopyThreads / 32);
    const uint32_t epoch = static_cast<uint32_t>(*st.epoch);
    const int64_t total = dispatch_offsets[experts];
    // Rows to walk: `rows` of them from packed row `first + rotate` on, wrapping.
    int64_t first = 0, rows = total, rotate = 0;
    if (kMode == kSendLocal) {
        first = dispatch_offsets[me * local];
        rows = dispatch_offsets[(me + 1) * local] - first;
    } else {
        // Start at the rows for rank me+1 and wrap around: at any moment the
        // ranks write to different owners (a shifted all-to-all), instead of
        // every rank writing to owner 0 first.
        rotate = dispatch_offsets[((me + 1) % ranks) * local];
        if (kMode == kSendRemote) {
            // my own rows are the range [a, b): walk b .. a (mod total)
            const int64_t a = dispatch_offsets[me * local], b = dispatch_offsets[(me + 1) * local];
            rows -= b - a;
            rotate = b;
        }
    }
    if (kMode == kSendRemote && blockIdx.x == 0 && static_cast<int>(threadIdx.x) < ranks) {
        const int o = threadIdx.x;
        if (o == me || st.owner_total[o] == 0) {
            uint32_t* flags = reinterpret_cast<uint32_t*>(regions.base[o] + l.flags);
            store_release_sys(flags + kMaxRanks + me, epoch);
        }
    }
    for (int64_t v = (static_cast<int64_t>(blockIdx.x) * kCopyThreads + threadIdx.x) >> 5; v < rows;
         v += warps) {
        int64_t r = first + v + rotate;
        if (r >= total) r -= total;
        int lo = 0, hi = experts - 1;  // expert of packed row r
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (dispatch_offsets[mid] <= r) lo = mid;
            else hi = mid - 1;
        }
        const int owner = lo / local;
        const int64_t dst = st.send_dst[lo] + (r - dispatch_offsets[lo]);
        if (dst >= grouped_rows) {
            if (lane == 0) atomicCAS(&g_ep_status, 0, 3);
            continue;
        }
        uint4* target = reinterpret_cast<uint4*>(regions.base[owner] + l.grouped) + dst * row_vecs;
        warp_copy_row(target, packed + r * row_vecs, row_vecs, lane);
        if (kMode == kSendRemote) {
            __threadfence_system();  // this lane's part of the row is visible on the owner
            __syncwarp();
            if (lane == 0 && atomicAdd(&st.owner_done[owner], 1) + 1 == st.owner_total[owner]) {
                st.owner_done[owner] = 0;  // every row counted: ready for the next step
                uint32_t* flags = reinterpret_cast<uint32_t*>(regions.base[owner] + l.flags);
                store_release_sys(flags + kMaxRanks + me, epoch);
            }
        }
    }
    if (kMode != kSendAll) return;
    // the last CTA to finish raises the rows flag of source `me` on every rank
    __threadfence_system();
    __syncthreads();
    __shared__ int last;
    if (threadIdx.x == 0) last = atomicAdd(&st.counters[0], 1) == static_cast<int>(gridDim.x) - 1;
    __syncthreads();
    if (!last) return;
    __threadfence_system();
    if (threadIdx.x < ranks) {
        uint32_t* flags = reinterpret_cast<uint32_t*>(regions.base[threadIdx.x] + l.flags);
        store_release_sys(flags + kMaxRanks + me, epoch);
    }
    if (threadIdx.x == 0) st.counters[0] = 0;
}

// Result rows of my grouped buffer -> the `back` buffers of their sources (a warp per row).
__global__ void __launch_bounds__(kCopyThreads)
ep_return_rows_kernel(const uint4* __restrict__ results, Regions regions, int32_t* state_base,
                      int ranks, int me, int experts, int64_t row_vecs, int64_t hidden,
                      int64_t grouped_rows, int64_t back_rows) {
    const Layout l = region_layout(ranks, experts, hidden, grouped_rows, back_rows);
    State st = state_view(state_base, ranks, experts);
    const int local = experts / ranks;
    const int segments = ranks * local;
    const int64_t rows = st.recv_prefix[segments];
    const int lane = threadIdx.x & 31;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (kCopyThreads / 32);
    // rows are source-major: start at source me+1's rows (shifted all-to-all)
    const int64_t rotate = st.recv_prefix[((me + 1) % ranks) * local];
    for (int64_t v = (static_cast<int64_t>(blockIdx.x) * kCopyThreads + threadIdx.x) >> 5; v < rows;
         v += warps) {
        const int64_t r = v + rotate < rows ? v + rotate : v + rotate - rows;
        int lo = 0, hi = segments - 1;  // last segment starting at or before r
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (st.recv_prefix[mid] <= r) lo = mid;
            else hi = mid - 1;
        }
        const int64_t i = r - st.recv_prefix[lo];
        if (i >= st.seg_count[lo]) continue;
        const int source = lo / local;
        const int64_t dst = st.ret_dst[lo] + i;
        if (dst >= back_rows) {
            if (lane == 0) atomicCAS(&g_ep_status, 0, 3);
            continue;
        }
        uint4* target = reinterpret_cast<uint4*>(regions.base[source] + l.back) + dst * row_vecs;
        warp_copy_row(target, results + (st.seg_start[lo] + i) * row_vecs, row_vecs, lane);
    }
    __threadfence_system();
    __syncthreads();
    __shared__ int last;
    if (threadIdx.x == 0) last = atomicAdd(&st.counters[1], 1) == static_cast<int>(gridDim.x) - 1;
    __syncthreads();
    if (!last) return;
    __threadfence_system();
    if (threadIdx.x < ranks) {
        uint32_t* flags = reinterpret_cast<uint32_t*>(regions.base[threadIdx.x] + l.flags);
        store_release_sys(flags + 2 * kMaxRanks + me, static_cast<uint32_t>(*st.epoch));
    }
    if (threadIdx.x == 0) st.counters[1] = 0;
}

__global__ void ep_wait_kernel(Regions regions, const int32_t* state_base, int ranks, int me,
                               int experts, int which, int64_t hidden, int64_t grouped_rows,
                               int64_t back_rows, uint64_t limit_ns) {
    const Layout l = region_layout(ranks, experts, hidden, grouped_rows, back_rows);
    const uint32_t epoch = static_cast<uint32_t>(state_base[0]);
    const uint32_t* flags = reinterpret_cast<const uint32_t*>(regions.base[me] + l.flags) +
                            which * kMaxRanks;
    wait_flags(flags, ranks, epoch, limit_ns);
}

// Grid of the send and return kernels: 4 CTAs per SM of a B200 by default;
// MOE_B200_EP_COPY_CTAS=n runs them on n CTAs, to leave SMs to a concurrent GEMM.
unsigned copy_grid() {
    static const unsigned grid = [] {
        const char* env = getenv("MOE_B200_EP_COPY_CTAS");
        const int n = env ? atoi(env) : 0;
        return static_cast<unsigned>(n > 0 && n <= 148 * 8 ? n : 148 * 4);
    }();
    return grid;
}

// Grid of the remote send, which runs beside the gate/up GEMM: one CTA per
// SM of a B200 (each fits beside a GEMM CTA); MOE_B200_EP_SEND_CTAS=n overrides.
unsigned remote_send_grid() {
    static const unsigned grid = [] {
        const char* env = getenv("MOE_B200_EP_SEND_CTAS");
        const int n = env ? atoi(env) : 0;
        return static_cast<unsigned>(n > 0 && n <= 148 * 8 ? n : 148);
    }();
    return grid;
}

Regions to_regions(void* const* regions, int ranks) {
    Regions r = {};
    for (int i = 0; i < ranks; ++i) r.base[i] = static_cast<char*>(regions[i]);
    return r;
}

}  // namespace

int64_t ep_p2p_region_bytes(int ranks, int experts, int64_t hidden, int64_t grouped_rows,
                            int64_t back_rows) {
    return region_layout(ranks, experts, hidden, grouped_rows, back_rows).total;
}

int64_t ep_p2p_region_offset(int ranks, int experts, int64_t hidden, int64_t grouped_rows,
                             int64_t back_rows, int section) {
    const Layout l = region_layout(ranks, experts, hidden, grouped_rows, back_rows);
    return section == 0 ? l.grouped : l.back;
}

int64_t ep_p2p_state_words(int ranks, int experts) {
    const int local = experts / ranks;
    return 4 + experts + (local + 1) + 3 * ranks * local + ranks * local + 1 + 2 * ranks +
           local * (ranks + 1);
}

cudaError_t launch_ep_p2p(int op, const void* rows, const int32_t* aux, void* const* regions,
                          int32_t* state, int ranks, int me, int experts, int alignment,
                          int64_t hidden, int64_t grouped_rows, int64_t back_rows,
                          int64_t timeout_ms, cudaStream_t stream) {
    const Regions r = to_regions(regions, ranks);
    const uint64_t limit_ns = static_cast<uint64_t>(timeout_ms) * 1000000ull;
    const int64_t row_vecs = hidden * 2 / 16;
    switch (op) {
        case kEpP2pCounts: {
            const size_t smem = static_cast<size_t>(experts) * sizeof(int32_t);
            ep_exchange_counts_kernel<<<1, 1024, smem, stream>>>(aux, r, state, ranks, me, experts,
                                                                alignment, hidden, grouped_rows,
                                                                back_rows, limit_ns);
            break;
        }
        case kEpP2pSend:
            ep_send_rows_kernel<kSendAll><<<copy_grid(), kCopyThreads, 0, stream>>>(
                static_cast<const uint4*>(rows), aux, r, state, ranks, me, experts, row_vecs, hidden,
                grouped_rows, back_rows);
            break;
        case kEpP2pSendLocal:
            ep_send_rows_kernel<kSendLocal><<<copy_grid(), kCopyThreads, 0, stream>>>(
                static_cast<const uint4*>(rows), aux, r, state, ranks, me, experts, row_vecs, hidden,
                grouped_rows, back_rows);
            break;
        case kEpP2pSendRemote:
            ep_send_rows_kernel<kSendRemote><<<remote_send_grid(), kCopyThreads, 0, stream>>>(
                static_cast<const uint4*>(rows), aux, r, state, ranks, me, experts, row_vecs, hidden,
                grouped_rows, back_rows);
            break;
        case kEpP2pReturn:
            ep_return_rows_kernel<<<copy_grid(), kCopyThreads, 0, stream>>>(static_cast<const uint4*>(rows), r,
                                                               state, ranks, me, experts, row_vecs,
                                                               hidden, grouped_rows, back_rows);
            break;
        case kEpP2pWaitRows:
        case kEpP2pWaitReturn:
            ep_wait_kernel<<<1, 32, 0, stream>>>(r, state, ranks, me, experts,
                                                 op == kEpP2pWaitRows ? 1 : 2, hidden, grouped_rows,
                                                 back_rows, limit_ns);
            break;
        default:
            return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_ep_p2p_gate_up(const void* gate_up, void* activated, void* const* regions,
                                  int32_t* state, int ranks, int me, int experts, int64_t hidden,
                                  int64_t intermediate, int64_t grouped_rows, int64_t back_rows,
                                  int64_t timeout_ms, cudaStream_t stream, const char** error) {
    const Layout l = region_layout(ranks, experts, hidden, grouped_rows, back_rows);
    const State st = state_view(state, ranks, experts);
    GemmArrival arrival;
    arrival.groups = ranks;
    arrival.group_rows = st.group_rows;
    arrival.flags = reinterpret_cast<const uint32_t*>(static_cast<char*>(regions[me]) + l.flags) + kMaxRanks;
    arrival.epoch = st.epoch;
    arrival.ranks = ranks;
    arrival.me = me;
    arrival.limit_ns = static_cast<uint64_t>(timeout_ms) * 1000000ull;
    const void* grouped = static_cast<char*>(regions[me]) + l.grouped;
    return launch_grouped_gemm(grouped, gate_up, st.offsets, activated, grouped_rows, intermediate,
                               hidden, experts / ranks, true, stream, error, nullptr, nullptr,
                               ranks > 1 ? &arrival : nullptr);
}

cudaError_t launch_ep_p2p_down_return(const void* activated, const void* down, void* const* regions,
                                      int32_t* state, int ranks, int me, int experts,
                                      int64_t hidden, int64_t intermediate, int64_t grouped_rows,
                                      int64_t back_rows, cudaStream_t stream, const char** error) {
    const Layout l = region_layout(ranks, experts, hidden, grouped_rows, back_rows);
    const State st = state_view(state, ranks, experts);
    GemmScatter sc = {};
    for (int i = 0; i < ranks; ++i) sc.base[i] = static_cast<char*>(regions[i]);
    sc.back_offset = l.back;
    sc.flags_offset = l.flags;
    sc.back_rows = back_rows;
    sc.seg_start = st.seg_start;
    sc.seg_count = st.seg_count;
    sc.ret_dst = st.ret_dst;
    sc.epoch = st.epoch;
    sc.ticket = st.counters + 1;
    sc.ranks = ranks;
    sc.me = me;
    sc.local_experts = experts / ranks;
    return launch_grouped_gemm_scatter(activated, down, st.offsets, grouped_rows, hidden,
                                       intermediate, experts / ranks, sc, stream, error);
}

cudaError_t read_ep_status(int32_t* code, bool clear) {
    MOE_CUDA_TRY(cudaMemcpyFromSymbol(code, g_ep_status, sizeof(int32_t)));
    if (clear) {
        const int32_t zero = 0;
        MOE_CUDA_TRY(cudaMemcpyToSymbol(g_ep_status, &zero, sizeof(int32_t)));
    }
    return cudaSuccess;
}

}  // namespace moe
