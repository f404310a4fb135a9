// Host-side launchers shared between the kernel files and the C ABI layer.
// Arguments are validated by the caller (capi.cu); these only enqueue work.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace moe {

constexpr int kMaxTopk = 32;
constexpr int kMaxRouteExperts = 256;
constexpr int kMaxDispatchExperts = 512;
constexpr int kDispatchChunk = 1024;  // assignments per dispatch-index CTA (one per thread)
constexpr int kRouterSlicedMaxExperts = 32;  // sliced-butterfly logit order up to here

cudaError_t launch_router_logits(const void* x, const float* w, float* logits, int64_t tokens,
                                 int64_t hidden, int experts, cudaStream_t stream);
// Logits + top-k + softmax; logits may be null for E <= 32 (then not written).
cudaError_t launch_route(const void* x, const float* w, const float* bias, float* logits,
                         int32_t* ids32, int64_t* ids64, float* weights, int64_t tokens,
                         int64_t hidden, int experts, int topk, cudaStream_t stream);
cudaError_t launch_topk(const float* logits, const float* bias, int32_t* ids32, int64_t* ids64,
                        float* weights, int64_t tokens, int experts, int topk, cudaStream_t stream);

int64_t dispatch_scratch_bytes(int64_t assignments, int experts);
cudaError_t launch_dispatch(const void* x, int dtype, const int32_t* ids, int32_t* counts,
                            int32_t* offsets, int32_t* slots, void* packed, int32_t* inverse,
                            int64_t tokens, int64_t hidden, int topk, int experts,
                            int64_t packed_rows, int alignment, int vector_bytes, int32_t* scratch,
                            cudaStream_t stream);
cudaError_t launch_combine(const void* expert_output, int dtype, const int32_t* inverse,
                           const float* weights, void* output, int64_t tokens, int64_t hidden,
                           int topk, int64_t packed_rows, int vector_bytes, cudaStream_t stream);
cudaError_t launch_swiglu(const void* projection, int dtype, const int32_t* valid_rows,
                          void* output, int64_t rows, int64_t width, int vector_bytes,
                          cudaStream_t stream);

// Rows that arrive from peer ranks while a grouped GEMM runs (P2P expert
// parallelism): each expert's rows are `groups` consecutive arrival groups,
// group g from rank (me - g) mod ranks (group 0 = this rank's own rows, in
// place before the launch).  group_rows[e * (groups + 1) + g] is the first row
// of group g relative to the expert's span, [.. + groups] its real rows.  The
// GEMM takes tiles group by group and loads a tile of group g once flags[s]
// >= *epoch for the sources s of groups 1..g (bounded by limit_ns; status 6).
struct GemmArrival {
    int groups;
    const int32_t* group_rows;
    const uint32_t* flags;
    const int32_t* epoch;
    int ranks, me;
    uint64_t limit_ns;
};

// Grouped GEMMs on tcgen05 (gemm_sm100.cu).  `error` receives a message when
// the returned status is not cudaSuccess because of a host-side check.
// With a_scale (and b_scale) non-null, a and b are e4m3 bytes and every
// accumulator is dequantised as (acc * a_scale[row]) * b_scale[weight row].
cudaError_t launch_grouped_gemm(const void* a, const void* b, const int32_t* offsets, void* out,
                                int64_t rows, int64_t n_out, int64_t k_dim, int experts,
                                bool swiglu, cudaStream_t stream, const char** error,
                                const float* a_scale = nullptr, const float* b_scale = nullptr,
                                const GemmArrival* arrival = nullptr);
// e4m3 quantisation of bf16 rows: scale[r] = amax_r / 448, q[r,c] = e4m3(x[r,c] * (448 / amax_r))
// (round to nearest even, saturating); an all-zero row gets scale 1 and zeros.
cudaError_t launch_quantize_rows_e4m3(const void* x, void* q, float* scale, int64_t rows,
                                      int64_t cols, cudaStream_t stream);
cudaError_t read_gemm_status(int32_t* code, bool clear);
cudaError_t read_route_status(int32_t* code, bool clear);
bool grouped_gemm_uses_pair(int64_t rows, int experts);

// Down GEMM whose epilogue returns each result row to its source rank (P2P
// expert parallelism): grouped row r of local expert e belongs to the segment
// s with seg_start[s*E_l+e] <= r < seg_start + seg_count; it is stored at row
// ret_dst[s*E_l+e] + (r - seg_start) of rank s's `back` section.  After the
// last CTA finishes, return flag `me` is raised on every rank with *epoch.
constexpr int kGemmScatterMaxRanks = 8;
struct GemmScatter {
    char* base[kGemmScatterMaxRanks];
    int64_t back_offset, flags_offset, back_rows;
    const int32_t* seg_start;
    const int32_t* seg_count;
    const int32_t* ret_dst;
    const int32_t* epoch;
    int32_t* ticket;
    int ranks, me, local_experts;
};
cudaError_t launch_grouped_gemm_scatter(const void* a, const void* b, const int32_t* offsets,
                                        int64_t rows, int64_t n_out, int64_t k_dim, int experts,
                                        const GemmScatter& scatter, cudaStream_t stream,
                                        const char** error);

// Expert-parallel receive layout (ep.cu).
cudaError_t launch_ep_layout(const int32_t* counts, int ranks, int experts, int alignment,
                             int32_t* src_start, int32_t* dst_start, int32_t* offsets,
                             cudaStream_t stream);
cudaError_t launch_ep_regroup(const void* from, void* to, const int32_t* counts,
                              const int32_t* src_start, const int32_t* dst_start,
                              const int32_t* offsets, int ranks, int experts, int64_t row_bytes,
                              int64_t recv_rows, int64_t grouped_rows, bool grouping,
                              int vector_bytes, cudaStream_t stream);

// Expert-parallel exchange over peer memory (ep_p2p.cu).
constexpr int kEpP2pMaxRanks = 8;
enum EpP2pOp { kEpP2pCounts = 0, kEpP2pSend = 1, kEpP2pWaitRows = 2, kEpP2pReturn = 3,
               kEpP2pWaitReturn = 4, kEpP2pSendLocal = 5, kEpP2pSendRemote = 6 };
int64_t ep_p2p_region_bytes(int ranks, int experts, int64_t hidden, int64_t grouped_rows,
                            int64_t back_rows);
int64_t ep_p2p_region_offset(int ranks, int experts, int64_t hidden, int64_t grouped_rows,
                             int64_t back_rows, int section);
int64_t ep_p2p_state_words(int ranks, int experts);
cudaError_t launch_ep_p2p(int op, const void* rows, const int32_t* aux, void* const* regions,
                          int32_t* state, int ranks, int me, int experts, int alignment,
                          int64_t hidden, int64_t grouped_rows, int64_t back_rows,
                          int64_t timeout_ms, cudaStream_t stream);
cudaError_t read_ep_status(int32_t* code, bool clear);
// The gate/up GEMM (+ SwiGLU) of the P2P step on this rank's grouped rows,
// taking each tile once the rows it needs have arrived (GemmArrival).
cudaError_t launch_ep_p2p_gate_up(const void* gate_up, void* activated, void* const* regions,
                                  int32_t* state, int ranks, int me, int experts, int64_t hidden,
                                  int64_t intermediate, int64_t grouped_rows, int64_t back_rows,
                                  int64_t timeout_ms, cudaStream_t stream, const char** error);
cudaError_t launch_ep_p2p_down_return(const void* activated, const void* down, void* const* regions,
                                      int32_t* state, int ranks, int me, int experts,
                                      int64_t hidden, int64_t intermediate, int64_t grouped_rows,
                                      int64_t back_rows, cudaStream_t stream, const char** error);

// Sets the calling thread's message returned by moe_last_error().
void set_last_error(const char* message);

// moe_dispatch's argument checks, except those on the scratch buffer (capi.cu).
// Returns MOE_OK, or a status with the calling thread's message set.
int check_dispatch_args(const void* x, int32_t dtype, const int32_t* ids, const int32_t* counts,
                        const int32_t* offsets, const int32_t* slots, const void* packed,
                        const int32_t* inverse, int64_t tokens, int64_t hidden, int32_t topk,
                        int32_t experts, int64_t packed_rows, int32_t alignment);

}  // namespace moe
