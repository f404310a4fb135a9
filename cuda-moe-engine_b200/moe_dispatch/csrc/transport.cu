// Token transport: dispatch (index + pack), combine and the standalone SwiGLU.
//
// Dispatch replaces the reference's count_slots / offsets / pack / zero_padding
// kernels (src/moe_dispatch/csrc/dispatch.cu:13-74, 194-275).  The reference
// assigns slots with atomicAdd, so its order inside an expert changes from run
// to run; here the order is the stable token-major order of p = t*K + k:
//
//   dispatch_index_kernel  one CTA per kDispatchChunk (1024) assignments.  match_any groups a
//                          warp's assignments by expert, per-warp histograms
//                          are scanned in warp order, so each assignment gets
//                          its rank inside the chunk without atomics.  The last
//                          CTA to finish (ticket in scratch) scans the per-chunk
//                          counts into chunk bases, writes counts[E] and the
//                          padded offsets[E+1].  Up to 8 chunks the CTAs form
//                          one cluster and hand their counts to CTA 0 through
//                          distributed shared memory instead.
//   pack_kernel            one CTA per token: reads the x row once, writes it to
//                          its K packed rows (16-byte vectors), writes slots and
//                          inverse; E extra CTAs zero the padding rows.
#include "common.cuh"
#include "launch.h"

#include <cstdlib>

namespace moe {
namespace {

constexpr int kIndexThreads = 1024;
// int32 words before the chunk table: [0] completion ticket, [1] running count
// of out-of-range expert ids, [2] that count for the last finished call; pad.
constexpr int kScratchHeader = 16;

template <int BYTES> struct VecOf;
template <> struct VecOf<16> { using T = uint4; };
template <> struct VecOf<8> { using T = uint2; };
template <> struct VecOf<4> { using T = uint32_t; };
template <> struct VecOf<2> { using T = uint16_t; };

// Up to this many chunks the index CTAs run as one thread-block cluster: the
// chunk totals travel to the leader CTA through distributed shared memory and
// a cluster barrier, instead of through the global chunk table, a fence, the
// completion ticket and the last CTA's reads (Mixtral shape: 8 chunks).
constexpr int kClusterChunks = 8;

__device__ __forceinline__ uint32_t shared_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

template <bool kCluster>
__global__ void __launch_bounds__(kIndexThreads)
dispatch_index_kernel(const int32_t* __restrict__ ids, int64_t n, int experts, int alignment,
                      int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                      int32_t* __restrict__ slots, int32_t* __restrict__ scratch, int chunks) {
    extern __shared__ int32_t smem[];
    // rows of E + 1 words: lane w of a warp scanning expert x reads word
    // w * (E + 1) + x, on 32 different banks whatever E is
    const int stride = experts + 1;
    int32_t* hist = smem;                     // [32][E+1] per-warp counts of this round
    int32_t* base = smem + 32 * stride;       // [32][E+1] per-warp bases of this round
    int32_t* running = smem + 64 * stride;    // [E] chunk-local running totals
    // cluster form: [kClusterChunks][E] chunk totals and [kClusterChunks]
    // out-of-range counts, filled in the leader CTA by every CTA of the cluster
    int32_t* table = running + experts;
    int32_t* bad_slots = table + kClusterChunks * experts;
    __shared__ int is_last;
    __shared__ int bad_here;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // The pack kernel may start now: it reads its token rows, then waits for
    // this grid (griddepcontrol.wait) before it needs anything computed here.
    pdl_trigger();
    for (int i = tid; i < 32 * stride; i += kIndexThreads) hist[i] = 0;
    for (int i = tid; i < experts; i += kIndexThreads) running[i] = 0;
    if (tid == 0) bad_here = 0;
    // cluster form: announce this CTA has started; its peers wait for that
    // before they store into the leader's shared memory
    if constexpr (kCluster) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    pdl_wait();  // the ids come from the kernel before (the router)
    __syncthreads();

    const int64_t chunk0 = static_cast<int64_t>(blockIdx.x) * kDispatchChunk;
    const unsigned lanes_below = (1u << lane) - 1u;
    for (int r = 0; r < kDispatchChunk / kIndexThreads; ++r) {
        const int64_t p = chunk0 + r * kIndexThreads + tid;
        const int e = p < n ? ids[p] : -1;
        const bool valid = e >= 0 && e < experts;
        const unsigned key = valid ? static_cast<unsigned>(e) : static_cast<unsigned>(experts + lane);
        const unsigned peers = __match_any_sync(0xffffffffu, key);
        const int rank = __popc(peers & lanes_below);
        if (valid && rank == 0) hist[warp * stride + e] = __popc(peers);
        __syncthreads();
        // each expert's 32 per-warp counts, scanned in warp order by one warp
        // (lane = warp index): exclusive prefix + running total = its base
        for (int x = warp; x < experts; x += kIndexThreads / 32) {
            const int c = hist[lane * stride + x];
            int inclusive = c;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, inclusive, off);
                if (lane >= off) inclusive += y;
            }
            const int run = running[x];
            base[lane * stride + x] = run + inclusive - c;
            hist[lane * stride + x] = 0;
            __syncwarp();
            if (lane == 31) running[x] = run + inclusive;
        }
        __syncthreads();
        if (p < n) slots[p] = valid ? base[warp * stride + e] + rank : -1;
        const unsigned bad = __ballot_sync(0xffffffffu, p < n && !valid);
        if (bad && lane == 0) {
            if constexpr (kCluster) atomicAdd(&bad_here, __popc(bad));
            else atomicAdd(scratch + 1, __popc(bad));
        }
    }

    int32_t* ticket = scratch;
    int32_t* chunk_table = scratch + kScratchHeader;  // [chunks][E]
    if constexpr (kCluster) {
        // this CTA's chunk totals (and bad-id count) into the leader's table
        __syncthreads();
        asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // every CTA has started
        const uint32_t me = blockIdx.x;  // the grid is one cluster
        for (int x = tid; x < experts; x += kIndexThreads) {
            uint32_t remote;
            asm volatile("mapa.shared::cluster.u32 %0, %1, 0;"
                         : "=r"(remote) : "r"(shared_u32(table + me * experts + x)));
            asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(remote), "r"(running[x]) : "memory");
        }
        if (tid == 0) {
            uint32_t remote;
            asm volatile("mapa.shared::cluster.u32 %0, %1, 0;"
                         : "=r"(remote) : "r"(shared_u32(bad_slots + me)));
            asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(remote), "r"(bad_here) : "memory");
        }
        asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
                     ::: "memory");
        if (me != 0) return;
        // leader: chunk bases (exclusive over the chunks, in chunk order),
        // counts and the aligned totals the offsets scan below uses
        for (int x = tid; x < experts; x += kIndexThreads) {
            int carry = 0;
            for (int c = 0; c < static_cast<int>(gridDim.x); ++c) {
                const int v = table[c * experts + x];
                if (c < chunks) chunk_table[static_cast<int64_t>(c) * experts + x] = carry;
                carry += v;
            }
            counts[x] = carry;
            running[x] = alignment > 1 ? (carry + alignment - 1) / alignment * alignment : carry;
        }
    } else {
    for (int x = tid; x < experts; x += kIndexThreads)
        chunk_table[static_cast<int64_t>(blockIdx.x) * experts + x] = running[x];
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = atomicAdd(ticket, 1) == static_cast<int>(gridDim.x) - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();

    // Chunk bases: each warp scans the chunk column of 4 experts at a time,
    // 32 chunks per step (lane = chunk), all loads of a step issued first.
    constexpr int kScanExperts = 4;
    for (int xb = warp * kScanExperts; xb < experts; xb += (kIndexThreads / 32) * kScanExperts) {
        int carry[kScanExperts] = {};
        for (unsigned c0 = 0; c0 < gridDim.x; c0 += 32) {
            const unsigned c = c0 + lane;
            int v[kScanExperts];
#pragma unroll
            for (int j = 0; j < kScanExperts; ++j)
                v[j] = (c < gridDim.x && xb + j < experts)
                           ? __ldcg(chunk_table + static_cast<int64_t>(c) * experts + xb + j)
                           : 0;
#pragma unroll
            for (int j = 0; j < kScanExperts; ++j) {
                int inclusive = v[j];
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const int y = __shfl_up_sync(0xffffffffu, inclusive, off);
                    if (lane >= off) inclusive += y;
                }
                if (c < gridDim.x && xb + j < experts)  // becomes the chunk's base for this expert
                    chunk_table[static_cast<int64_t>(c) * experts + xb + j] = carry[j] + inclusive - v[j];
                carry[j] += __shfl_sync(0xffffffffu, inclusive, 31);
            }
        }
        if (lane == 0) {
#pragma unroll
            for (int j = 0; j < kScanExperts; ++j) {
                const int x = xb + j;
                if (x >= experts) break;
                counts[x] = carry[j];
                running[x] = alignment > 1 ? (carry[j] + alignment - 1) / alignment * alignment
                                           : carry[j];
            }
        }
    }
    }  // kCluster
    __syncthreads();
    if (warp == 0) {
        const int per = (experts + 31) / 32;
        const int start = min(experts, lane * per), end = min(experts, start + per);
        int local = 0;
        for (int x = start; x < end; ++x) local += running[x];
        int inclusive = local;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, inclusive, off);
            if (lane >= off) inclusive += y;
        }
        int run = inclusive - local;
        for (int x = start; x < end; ++x) {
            offsets[x] = run;
            run += running[x];
        }
        if (lane == 31) offsets[experts] = inclusive;
        if (lane == 0) {
            if constexpr (kCluster) {
                int bad_total = 0;
                for (int c = 0; c < static_cast<int>(gridDim.x); ++c) bad_total += bad_slots[c];
                scratch[2] = bad_total;  // out-of-range ids of this call
            } else {
                scratch[2] = atomicExch(scratch + 1, 0);  // out-of-range ids of this call
                *ticket = 0;  // ready for the next call
            }
        }
    }
}

template <typename V>
__global__ void __launch_bounds__(256)
pack_kernel(const V* __restrict__ x, const int32_t* __restrict__ ids,
            const int32_t* __restrict__ counts, const int32_t* __restrict__ offsets,
            const int32_t* __restrict__ chunk_table, int32_t* __restrict__ slots,
            int32_t* __restrict__ inverse, V* __restrict__ packed, int64_t tokens, int topk,
            int experts, int64_t row_vecs, int64_t packed_rows) {
    __shared__ int64_t dest[kMaxTopk];
    const int64_t t = blockIdx.x;
    constexpr int kUnroll = 4;
    pdl_trigger();  // the grouped GEMM may launch and run its prologue
    // Launched as a programmatic dependent of the index kernel: the first
    // slice of this token's row does not depend on it, so load it first.
    V first[kUnroll];
    if (t < tokens) {
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t c = threadIdx.x + u * blockDim.x;
            if (c < row_vecs) first[u] = __ldg(x + t * row_vecs + c);
        }
    }
    pdl_wait();
    if (t < tokens) {
        if (threadIdx.x < topk) {
            const int64_t p = t * topk + threadIdx.x;
            const int e = ids[p];
            int64_t d = -1;
            if (e >= 0 && e < experts) {
                const int slot = chunk_table[(p / kDispatchChunk) * experts + e] + slots[p];
                slots[p] = slot;
                d = static_cast<int64_t>(offsets[e]) + slot;
                if (d >= packed_rows) d = -1;
            } else {
                slots[p] = -1;
            }
            inverse[p] = static_cast<int32_t>(d);
            dest[threadIdx.x] = d;
        }
        __syncthreads();
        const V* src = x + t * row_vecs;
        for (int64_t c0 = threadIdx.x; c0 < row_vecs; c0 += kUnroll * blockDim.x) {
            V v[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int64_t c = c0 + u * blockDim.x;
                if (c0 == threadIdx.x) v[u] = first[u];
                else if (c < row_vecs) v[u] = __ldg(src + c);
            }
            for (int k = 0; k < topk; ++k) {
                const int64_t d = dest[k];
                if (d < 0) continue;
                V* row = packed + d * row_vecs;
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    const int64_t c = c0 + u * blockDim.x;
                    if (c < row_vecs) row[c] = v[u];
                }
            }
        }
    } else {
        const int e = static_cast<int>(t - tokens);
        const int64_t start = static_cast<int64_t>(offsets[e]) + counts[e];
        int64_t end = offsets[e + 1];
        if (end > packed_rows) end = packed_rows;
        const V zero = {};
        const int64_t total = (end - start) * row_vecs;
        for (int64_t i = threadIdx.x; i < total; i += blockDim.x) packed[start * row_vecs + i] = zero;
    }
}

// combine: out[t] = cast(sum_k (w[t,k] * f32(eo[row_k]))) with every product and
// partial sum rounded to fp32 (__fmul_rn/__fadd_rn are never contracted to FMA).
template <int DT, int VB, int KB>
__global__ void __launch_bounds__(256)
combine_kernel(const typename VecOf<VB>::T* __restrict__ eo, const int32_t* __restrict__ inverse,
               const float* __restrict__ weights, typename VecOf<VB>::T* __restrict__ out,
               int64_t tokens, int topk, int64_t row_vecs, int64_t packed_rows) {
    using V = typename VecOf<VB>::T;
    using E = Elem<DT>;
    using T = typename E::T;
    constexpr int N = VB / sizeof(T);
    union Pun {
        V v;
        T e[N];
    };
    __shared__ int64_t rows[kMaxTopk];
    __shared__ float ws[kMaxTopk];
    const int64_t t = blockIdx.x;
    pdl_wait();  // a dependent launch of the down GEMM
    if (threadIdx.x < topk) {
        const int64_t p = t * topk + threadIdx.x;
        const int32_t r = inverse[p];
        rows[threadIdx.x] = (r >= 0 && r < packed_rows) ? r : -1;
        ws[threadIdx.x] = weights[p];
    }
    __syncthreads();
    // KB loads in flight per thread before the adds that use them: 8 for
    // top-k > 2; 2 for top-k <= 2, where wider batches only cost registers
    // (and occupancy) without more loads to overlap.
    constexpr int kBatch = KB;
    for (int64_t c = threadIdx.x; c < row_vecs; c += blockDim.x) {
        float acc[N];
#pragma unroll
        for (int i = 0; i < N; ++i) acc[i] = 0.0f;
        for (int k0 = 0; k0 < topk; k0 += kBatch) {
            Pun in[kBatch];
#pragma unroll
            for (int j = 0; j < kBatch; ++j) {
                const int64_t r = k0 + j < topk ? rows[k0 + j] : -1;
                if (r >= 0) in[j].v = __ldg(eo + r * row_vecs + c);
            }
            // the adds stay in k order, so batching does not change any bit
#pragma unroll
            for (int j = 0; j < kBatch; ++j) {
                if (k0 + j >= topk) break;
                if (rows[k0 + j] < 0) continue;
                const float wk = ws[k0 + j];
#pragma unroll
                for (int i = 0; i < N; ++i)
                    acc[i] = __fadd_rn(acc[i], __fmul_rn(wk, E::load(in[j].e[i])));
            }
        }
        Pun o;
#pragma unroll
        for (int i = 0; i < N; ++i) o.e[i] = E::store(acc[i]);
        out[t * row_vecs + c] = o.v;
    }
}

// combine for top-k <= 2: each thread takes CU columns of the token and issues
// the loads of all of them (2 * CU vectors) before the first add, instead of
// two per column; same products and the same k-ordered adds as combine_kernel.
template <int DT, int VB, int CU>
__global__ void __launch_bounds__(256)
combine_top2_kernel(const typename VecOf<VB>::T* __restrict__ eo, const int32_t* __restrict__ inverse,
                    const float* __restrict__ weights, typename VecOf<VB>::T* __restrict__ out,
                    int64_t tokens, int topk, int64_t row_vecs, int64_t packed_rows) {
    using V = typename VecOf<VB>::T;
    using E = Elem<DT>;
    using T = typename E::T;
    constexpr int N = VB / sizeof(T);
    union Pun {
        V v;
        T e[N];
    };
    const int64_t t = blockIdx.x;
    pdl_wait();  // a dependent launch of the down GEMM
    int64_t row[2];
    float w[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int64_t p = t * topk + j;
        const int32_t r = j < topk ? __ldg(inverse + p) : -1;
        row[j] = (r >= 0 && r < packed_rows) ? r : -1;
        w[j] = j < topk ? __ldg(weights + p) : 0.0f;
    }
    for (int64_t c0 = threadIdx.x; c0 < row_vecs; c0 += static_cast<int64_t>(blockDim.x) * CU) {
        Pun in[CU][2];
#pragma unroll
        for (int u = 0; u < CU; ++u) {
            const int64_t c = c0 + u * blockDim.x;
#pragma unroll
            for (int j = 0; j < 2; ++j)
                if (row[j] >= 0 && c < row_vecs) in[u][j].v = __ldg(eo + row[j] * row_vecs + c);
        }
#pragma unroll
        for (int u = 0; u < CU; ++u) {
            const int64_t c = c0 + u * blockDim.x;
            if (c >= row_vecs) break;
            float acc[N];
#pragma unroll
            for (int i = 0; i < N; ++i) acc[i] = 0.0f;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                if (row[j] < 0) continue;
#pragma unroll
                for (int i = 0; i < N; ++i)
                    acc[i] = __fadd_rn(acc[i], __fmul_rn(w[j], E::load(in[u][j].e[i])));
            }
            Pun o;
#pragma unroll
            for (int i = 0; i < N; ++i) o.e[i] = E::store(acc[i]);
            out[t * row_vecs + c] = o.v;
        }
    }
}

// swiglu: out[r,c] = cast(silu(g) * u), g = f32(proj[r,c]), u = f32(proj[r,c+W]);
// rows at or past *valid_rows are zero (dispatch.cu:277-292).
template <int DT, int VB>
__global__ void __launch_bounds__(256)
swiglu_kernel(const typename VecOf<VB>::T* __restrict__ proj, const int32_t* __restrict__ valid_rows,
              typename VecOf<VB>::T* __restrict__ out, int64_t rows, int64_t width_vecs) {
    using V = typename VecOf<VB>::T;
    using E = Elem<DT>;
    using T = typename E::T;
    constexpr int N = VB / sizeof(T);
    union Pun {
        V v;
        T e[N];
    };
    const int64_t valid = *valid_rows;
    const int64_t total = rows * width_vecs;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / width_vecs, c = i % width_vecs;
        Pun o;
        if (r >= valid) {
#pragma unroll
            for (int j = 0; j < N; ++j) o.e[j] = E::store(0.0f);
        } else {
            Pun g, u;
            g.v = __ldg(proj + r * 2 * width_vecs + c);
            u.v = __ldg(proj + r * 2 * width_vecs + width_vecs + c);
#pragma unroll
            for (int j = 0; j < N; ++j) {
                const float gv = E::load(g.e[j]);
                o.e[j] = E::store((gv / (1.0f + expf(-gv))) * E::load(u.e[j]));
            }
        }
        out[i] = o.v;
    }
}

// Threads per token CTA of the pack and combine kernels.  Each CTA first
// resolves its token's K destinations (or sources) through a chain of
// dependent loads; 128-thread CTAs let twice as many tokens per SM wait on
// those chains at once.  Measured against 256 on one B200 (eager stage
// events, same box): Mixtral block dispatch 31.7 -> 27.6 us, combine 21.0 ->
// 19.9 us; fine-grained block 0.132 -> 0.097 ms and 0.096 -> 0.084 ms; E = 256
// combine 0.717 -> 0.672 ms.  The top-8 packs (E = 256, the transport
// configuration) write 8 copies per row and were 2-3 % faster with 256.
// MOE_B200_TRANSPORT_THREADS=128|256 overrides both (a tuning knob, same bits).
int forced_transport_threads() {
    static const int forced = [] {
        const char* env = getenv("MOE_B200_TRANSPORT_THREADS");
        const int n = env ? atoi(env) : 0;
        return n == 128 || n == 256 ? n : 0;
    }();
    return forced;
}

int pack_threads(int topk) {
    if (const int forced = forced_transport_threads()) return forced;
    return topk <= 6 ? 128 : 256;
}

int combine_threads() {
    if (const int forced = forced_transport_threads()) return forced;
    return 128;
}

template <int VB>
cudaError_t launch_pack(const void* x, const int32_t* ids, const int32_t* counts,
                        const int32_t* offsets, const int32_t* table, int32_t* slots,
                        int32_t* inverse, void* packed, int64_t tokens, int topk, int experts,
                        int64_t row_bytes, int64_t packed_rows, int alignment, cudaStream_t stream) {
    using V = typename VecOf<VB>::T;
    const int64_t row_vecs = row_bytes / VB;
    const int64_t blocks = tokens + (alignment > 1 ? experts : 0);
    if (blocks == 0) return cudaSuccess;
    const int threads = pack_threads(topk);
    // programmatic dependent launch: may begin before the index kernel ends
    cudaLaunchConfig_t config = {};
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    config.gridDim = dim3(static_cast<unsigned>(blocks));
    config.blockDim = dim3(threads);
    config.stream = stream;
    config.attrs = attribute;
    config.numAttrs = 1;
    return cudaLaunchKernelEx(&config, pack_kernel<V>, static_cast<const V*>(x), ids, counts,
                              offsets, table, slots, inverse, static_cast<V*>(packed), tokens,
                              topk, experts, row_vecs, packed_rows);
}

template <int DT, int VB>
cudaError_t launch_combine_t(const void* eo, const int32_t* inverse, const float* weights,
                             void* output, int64_t tokens, int64_t row_bytes, int topk,
                             int64_t packed_rows, cudaStream_t stream) {
    using V = typename VecOf<VB>::T;
    const int64_t row_vecs = row_bytes / VB;
    // 256-thread CTAs: 512 (one vector per thread) measured slower, 29.7 vs 26.6 us
    // at top-2 and 62.4 vs 60 us at top-8 for 4096 rows of 8 KB.
    const int threads = combine_threads();
    const dim3 grid(static_cast<unsigned>(tokens));
    if (topk <= 2)
        return launch_dependent(combine_top2_kernel<DT, VB, 2>, grid, dim3(threads), 0, stream,
                                static_cast<const V*>(eo), inverse, weights, static_cast<V*>(output),
                                tokens, topk, row_vecs, packed_rows);
    return launch_dependent(combine_kernel<DT, VB, 8>, grid, dim3(threads), 0, stream,
                            static_cast<const V*>(eo), inverse, weights, static_cast<V*>(output),
                            tokens, topk, row_vecs, packed_rows);
}

template <int DT>
cudaError_t launch_combine_dt(const void* eo, const int32_t* inverse, const float* weights,
                              void* output, int64_t tokens, int64_t row_bytes, int topk,
                              int64_t packed_rows, int vb, cudaStream_t stream) {
    switch (vb) {
        case 16: return launch_combine_t<DT, 16>(eo, inverse, weights, output, tokens, row_bytes, topk, packed_rows, stream);
        case 8: return launch_combine_t<DT, 8>(eo, inverse, weights, output, tokens, row_bytes, topk, packed_rows, stream);
        case 4: return launch_combine_t<DT, 4>(eo, inverse, weights, output, tokens, row_bytes, topk, packed_rows, stream);
        default:
            if constexpr (DT == kF32) return cudaErrorInvalidValue;
            else return launch_combine_t<DT, 2>(eo, inverse, weights, output, tokens, row_bytes, topk, packed_rows, stream);
    }
}

template <int DT, int VB>
cudaError_t launch_swiglu_t(const void* proj, const int32_t* valid_rows, void* out, int64_t rows,
                            int64_t width_bytes, cudaStream_t stream) {
    using V = typename VecOf<VB>::T;
    const int64_t width_vecs = width_bytes / VB;
    const int64_t total = rows * width_vecs;
    const int64_t blocks = (total + 255) / 256;
    const unsigned grid = static_cast<unsigned>(blocks < 148 * 16 ? blocks : 148 * 16);
    swiglu_kernel<DT, VB><<<grid, 256, 0, stream>>>(static_cast<const V*>(proj), valid_rows,
                                                    static_cast<V*>(out), rows, width_vecs);
    return cudaGetLastError();
}

template <int DT>
cudaError_t launch_swiglu_dt(const void* proj, const int32_t* valid_rows, void* out, int64_t rows,
                             int64_t width_bytes, int vb, cudaStream_t stream) {
    switch (vb) {
        case 16: return launch_swiglu_t<DT, 16>(proj, valid_rows, out, rows, width_bytes, stream);
        case 8: return launch_swiglu_t<DT, 8>(proj, valid_rows, out, rows, width_bytes, stream);
        case 4: return launch_swiglu_t<DT, 4>(proj, valid_rows, out, rows, width_bytes, stream);
        default:
            if constexpr (DT == kF32) return cudaErrorInvalidValue;
            else return launch_swiglu_t<DT, 2>(proj, valid_rows, out, rows, width_bytes, stream);
    }
}

}  // namespace

int64_t dispatch_scratch_bytes(int64_t assignments, int experts) {
    const int64_t chunks = assignments > 0 ? (assignments + kDispatchChunk - 1) / kDispatchChunk : 1;
    return (kScratchHeader + chunks * experts) * static_cast<int64_t>(sizeof(int32_t));
}

cudaError_t launch_dispatch(const void* x, int dtype, const int32_t* ids, int32_t* counts,
                            int32_t* offsets, int32_t* slots, void* packed, int32_t* inverse,
                            int64_t tokens, int64_t hidden, int topk, int experts,
                            int64_t packed_rows, int alignment, int vector_bytes, int32_t* scratch,
                            cudaStream_t stream) {
    const int64_t n = tokens * topk;
    const int64_t chunks = n > 0 ? (n + kDispatchChunk - 1) / kDispatchChunk : 1;
    // [32][E+1] x 2 + [E], and for the cluster form [8][E] + [8]
    const size_t smem = static_cast<size_t>(65 * experts + 64) * sizeof(int32_t);
    const size_t cluster_smem = smem + static_cast<size_t>(kClusterChunks * (experts + 1)) * sizeof(int32_t);
    static bool configured[64] = {};
    int device = 0;
    MOE_CUDA_TRY(cudaGetDevice(&device));
    if (!configured[device & 63]) {  // once per device, for the largest expert count
        MOE_CUDA_TRY(cudaFuncSetAttribute(dispatch_index_kernel<false>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (65 * kMaxDispatchExperts + 64) * static_cast<int>(sizeof(int32_t))));
        MOE_CUDA_TRY(cudaFuncSetAttribute(
            dispatch_index_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
            (65 * kMaxDispatchExperts + 64 + kClusterChunks * (kMaxDispatchExperts + 1)) *
                static_cast<int>(sizeof(int32_t))));
        configured[device & 63] = true;
    }
    const char* cluster_env = getenv("MOE_B200_INDEX_CLUSTER");  // tuning knob: 0 = never
    if (chunks <= kClusterChunks && !(cluster_env && cluster_env[0] == '0')) {
        // one cluster of the next power of two CTAs; those past `chunks` see no ids
        unsigned size = 1;
        while (size < chunks) size <<= 1;
        cudaLaunchConfig_t config = {};
        cudaLaunchAttribute attribute[2];
        attribute[0].id = cudaLaunchAttributeClusterDimension;
        attribute[0].val.clusterDim.x = size;
        attribute[0].val.clusterDim.y = 1;
        attribute[0].val.clusterDim.z = 1;
        attribute[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attribute[1].val.programmaticStreamSerializationAllowed = 1;
        config.gridDim = dim3(size);
        config.blockDim = dim3(kIndexThreads);
        config.dynamicSmemBytes = cluster_smem;
        config.stream = stream;
        config.attrs = attribute;
        config.numAttrs = 2;
        MOE_CUDA_TRY(cudaLaunchKernelEx(&config, dispatch_index_kernel<true>, ids, n, experts,
                                        alignment, counts, offsets, slots, scratch,
                                        static_cast<int>(chunks)));
    } else {
        MOE_CUDA_TRY(launch_dependent(dispatch_index_kernel<false>, dim3(static_cast<unsigned>(chunks)),
                                      dim3(kIndexThreads), smem, stream, ids, n, experts, alignment,
                                      counts, offsets, slots, scratch, static_cast<int>(chunks)));
    }
    const int32_t* table = scratch + kScratchHeader;
    const int64_t row_bytes = hidden * dtype_bytes(dtype);
    switch (vector_bytes) {
        case 16: return launch_pack<16>(x, ids, counts, offsets, table, slots, inverse, packed, tokens, topk, experts, row_bytes, packed_rows, alignment, stream);
        case 8: return launch_pack<8>(x, ids, counts, offsets, table, slots, inverse, packed, tokens, topk, experts, row_bytes, packed_rows, alignment, stream);
        case 4: return launch_pack<4>(x, ids, counts, offsets, table, slots, inverse, packed, tokens, topk, experts, row_bytes, packed_rows, alignment, stream);
        default: return launch_pack<2>(x, ids, counts, offsets, table, slots, inverse, packed, tokens, topk, experts, row_bytes, packed_rows, alignment, stream);
    }
}

cudaError_t launch_combine(const void* expert_output, int dtype, const int32_t* inverse,
                           const float* weights, void* output, int64_t tokens, int64_t hidden,
                           int topk, int64_t packed_rows, int vector_bytes, cudaStream_t stream) {
    if (tokens == 0) return cudaSuccess;
    const int64_t row_bytes = hidden * dtype_bytes(dtype);
    switch (dtype) {
        case kF32: return launch_combine_dt<kF32>(expert_output, inverse, weights, output, tokens, row_bytes, topk, packed_rows, vector_bytes, stream);
        case kF16: return launch_combine_dt<kF16>(expert_output, inverse, weights, output, tokens, row_bytes, topk, packed_rows, vector_bytes, stream);
        default: return launch_combine_dt<kBF16>(expert_output, inverse, weights, output, tokens, row_bytes, topk, packed_rows, vector_bytes, stream);
    }
}

cudaError_t launch_swiglu(const void* projection, int dtype, const int32_t* valid_rows,
                          void* output, int64_t rows, int64_t width, int vector_bytes,
                          cudaStream_t stream) {
    if (rows == 0 || width == 0) return cudaSuccess;
    const int64_t width_bytes = width * dtype_bytes(dtype);
    switch (dtype) {
        case kF32: return launch_swiglu_dt<kF32>(projection, valid_rows, output, rows, width_bytes, vector_bytes, stream);
        case kF16: return launch_swiglu_dt<kF16>(projection, valid_rows, output, rows, width_bytes, vector_bytes, stream);
        default: return launch_swiglu_dt<kBF16>(projection, valid_rows, output, rows, width_bytes, vector_bytes, stream);
    }
}

}  // namespace moe
