// Expert-parallel receive layout: regroup rows that arrived from P source ranks
// into expert-major spans (and back), so the grouped GEMMs run on local experts.
//
// Each source rank p sends its assignments for this rank's E_l experts in its
// own packed order: expert-major, token order inside an expert.  counts[p][e]
// rows from rank p for local expert e arrive source-major:
//   src_start[p][e] = sum_{p' < p} rows(p') + sum_{e' < e} counts[p][e'].
// The grouped layout is expert-major with each expert's span rounded up to
// `alignment`, and inside an expert source-major:
//   offsets[e]      = sum_{e' < e} align(sum_p counts[p][e'])
//   dst_start[p][e] = offsets[e] + sum_{p' < p} counts[p'][e].
// Ranks hold consecutive token ranges, so source-major order inside an expert
// is the global token order: the grouped rows are exactly the rows a single
// GPU would pack for these experts.
#include "common.cuh"
#include "launch.h"

namespace moe {
namespace {

__global__ void __launch_bounds__(1024)
ep_layout_kernel(const int32_t* __restrict__ counts, int ranks, int experts, int alignment,
                 int32_t* __restrict__ src_start, int32_t* __restrict__ dst_start,
                 int32_t* __restrict__ offsets) {
    extern __shared__ int32_t sm[];
    int32_t* span = sm;                 // [E] padded span per expert
    int32_t* rank_rows = sm + experts;  // [P] rows from each source rank
    const int tid = threadIdx.x;
    for (int e = tid; e < experts; e += blockDim.x) {
        int total = 0;
        for (int p = 0; p < ranks; ++p) {
            dst_start[p * experts + e] = total;  // relative to offsets[e] for now
            total += counts[p * experts + e];
        }
        span[e] = alignment > 1 ? (total + alignment - 1) / alignment * alignment : total;
    }
    for (int p = tid; p < ranks; p += blockDim.x) {
        int run = 0;
        for (int e = 0; e < experts; ++e) {
            src_start[p * experts + e] = run;  // relative to the rank's first row for now
            run += counts[p * experts + e];
        }
        rank_rows[p] = run;
    }
    __syncthreads();
    if (tid == 0) {
        int run = 0;
        for (int e = 0; e < experts; ++e) {
            offsets[e] = run;
            run += span[e];
        }
        offsets[experts] = run;
        run = 0;
        for (int p = 0; p < ranks; ++p) {
            const int rows = rank_rows[p];
            rank_rows[p] = run;
            run += rows;
        }
    }
    __syncthreads();
    for (int i = tid; i < ranks * experts; i += blockDim.x) {
        src_start[i] += rank_rows[i / experts];
        dst_start[i] += offsets[i % experts];
    }
}

// One CTA per received row (grid-stride): find its segment by binary search on
// src_start (segments are in increasing source-major order), copy the row.
// Extra CTAs zero the padding rows of each expert when grouping.
template <typename V>
__global__ void __launch_bounds__(128)
ep_regroup_kernel(const V* __restrict__ from, V* __restrict__ to,
                  const int32_t* __restrict__ counts, const int32_t* __restrict__ src_start,
                  const int32_t* __restrict__ dst_start, const int32_t* __restrict__ offsets,
                  int segments, int experts, int64_t row_vecs, int64_t recv_rows,
                  int64_t grouped_rows, bool grouping) {
    for (int64_t block = blockIdx.x; block < recv_rows + experts; block += gridDim.x) {
        if (block < recv_rows) {
            int lo = 0, hi = segments - 1;
            while (lo < hi) {  // last segment starting at or before this row with rows in it
                const int mid = (lo + hi + 1) >> 1;
                if (src_start[mid] <= block) lo = mid;
                else hi = mid - 1;
            }
            while (lo > 0 && counts[lo] == 0) --lo;  // empty segments share a start
            const int64_t offset = block - src_start[lo];
            if (offset >= counts[lo]) continue;  // rows beyond the received total
            const int64_t src_row = grouping ? block : dst_start[lo] + offset;
            const int64_t dst_row = grouping ? dst_start[lo] + offset : block;
            if ((grouping ? dst_row : src_row) >= grouped_rows) continue;
            const V* s = from + src_row * row_vecs;
            V* d = to + dst_row * row_vecs;
            for (int64_t c = threadIdx.x; c < row_vecs; c += blockDim.x) d[c] = s[c];
        } else if (grouping) {
            const int e = static_cast<int>(block - recv_rows);
            int64_t filled = offsets[e];
            for (int p = 0; p < segments / experts; ++p) filled += counts[p * experts + e];
            int64_t end = offsets[e + 1];
            if (end > grouped_rows) end = grouped_rows;
            const V zero = {};
            for (int64_t i = filled * row_vecs + threadIdx.x; i < end * row_vecs; i += blockDim.x)
                to[i] = zero;
        }
    }
}

template <typename V>
cudaError_t launch_regroup_t(const void* from, void* to, const int32_t* counts,
                             const int32_t* src_start, const int32_t* dst_start,
                             const int32_t* offsets, int ranks, int experts, int64_t row_bytes,
                             int64_t recv_rows, int64_t grouped_rows, bool grouping,
                             cudaStream_t stream) {
    const int64_t row_vecs = row_bytes / static_cast<int64_t>(sizeof(V));
    const int64_t work = recv_rows + experts;
    const unsigned grid = static_cast<unsigned>(work < 148 * 64 ? work : 148 * 64);
    if (grid == 0) return cudaSuccess;
    ep_regroup_kernel<V><<<grid, 128, 0, stream>>>(
        static_cast<const V*>(from), static_cast<V*>(to), counts, src_start, dst_start, offsets,
        ranks * experts, experts, row_vecs, recv_rows, grouped_rows, grouping);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_ep_layout(const int32_t* counts, int ranks, int experts, int alignment,
                             int32_t* src_start, int32_t* dst_start, int32_t* offsets,
                             cudaStream_t stream) {
    const size_t smem = static_cast<size_t>(experts + ranks) * sizeof(int32_t);
    ep_layout_kernel<<<1, 1024, smem, stream>>>(counts, ranks, experts, alignment, src_start,
                                               dst_start, offsets);
    return cudaGetLastError();
}

cudaError_t launch_ep_regroup(const void* from, void* to, const int32_t* counts,
                              const int32_t* src_start, const int32_t* dst_start,
                              const int32_t* offsets, int ranks, int experts, int64_t row_bytes,
                              int64_t recv_rows, int64_t grouped_rows, bool grouping,
                              int vector_bytes, cudaStream_t stream) {
    switch (vector_bytes) {
        case 16: return launch_regroup_t<uint4>(from, to, counts, src_start, dst_start, offsets, ranks, experts, row_bytes, recv_rows, grouped_rows, grouping, stream);
        case 8: return launch_regroup_t<uint2>(from, to, counts, src_start, dst_start, offsets, ranks, experts, row_bytes, recv_rows, grouped_rows, grouping, stream);
        case 4: return launch_regroup_t<uint32_t>(from, to, counts, src_start, dst_start, offsets, ranks, experts, row_bytes, recv_rows, grouped_rows, grouping, stream);
        default: return launch_regroup_t<uint16_t>(from, to, counts, src_start, dst_start, offsets, ranks, experts, row_bytes, recv_rows, grouped_rows, grouping, stream);
    }
}

}  // namespace moe
