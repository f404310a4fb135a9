// extern "C" entry points declared in include/moe_b200.h.
//
// Each entry point checks what the reference's TORCH_CHECKs check
// (src/moe_dispatch/csrc/dispatch.cu:95-129, 160-180, 218-243, 294-310,
// 378-394) that can be checked from plain pointers and sizes -- sizes, limits,
// int32 index capacity, vector alignment -- and reports failures as a status
// code plus a per-thread message instead of a C++ exception.  Tensor
// properties (device, contiguity, dtype) are checked by the Python layer.
#include "../../../include/moe_b200.h"
#include "common.cuh"
#include "launch.h"

#include <climits>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

namespace {

thread_local std::string g_last_error;

int fail(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int status, const char* fmt, ...) {
    char buffer[512];
    va_list args;
    va_start(args, fmt);
    vsnprintf(buffer, sizeof(buffer), fmt, args);
    va_end(args);
    g_last_error = buffer;
    return status;
}

int cuda_status(cudaError_t err, const char* what) {
    if (err == cudaSuccess) return MOE_OK;
    return fail(MOE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

bool aligned(const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

// Widest vector (16/8/4/2 bytes) that divides the row and every row pointer.
int vector_bytes(int64_t row_bytes, int min_bytes, std::initializer_list<const void*> ptrs) {
    for (int vb = 16; vb > min_bytes; vb >>= 1) {
        if (row_bytes % vb) continue;
        bool ok = true;
        for (const void* p : ptrs) ok = ok && aligned(p, vb);
        if (ok) return vb;
    }
    return min_bytes;
}

bool valid_dtype(int32_t dtype) { return dtype == MOE_F32 || dtype == MOE_F16 || dtype == MOE_BF16; }

}  // namespace

namespace moe {
void set_last_error(const char* message) { g_last_error = message; }
}  // namespace moe

extern "C" {

int moe_abi_version(void) { return 1; }

const char* moe_last_error(void) { return g_last_error.c_str(); }

int moe_topk_route(const float* logits, const float* bias, int32_t* ids32, int64_t* ids64,
                   float* weights, int64_t tokens, int32_t experts, int32_t topk, void* stream) {
    if (tokens < 0) return fail(MOE_ERR_INVALID, "tokens must be >= 0");
    if (experts < 1 || experts > moe::kMaxRouteExperts)
        return fail(MOE_ERR_INVALID, "routing supports 1..%d experts", moe::kMaxRouteExperts);
    if (topk < 1 || topk > moe::kMaxTopk || topk > experts)
        return fail(MOE_ERR_INVALID, "topk must be in 1..min(experts, %d)", moe::kMaxTopk);
    if (tokens > INT_MAX / experts || tokens * topk > INT_MAX)
        return fail(MOE_ERR_INVALID, "shape exceeds int32 indexing capacity");
    if (tokens > 0 && (!logits || !ids32 || !weights))
        return fail(MOE_ERR_INVALID, "logits, ids32 and weights must be non-null");
    return cuda_status(moe::launch_topk(logits, bias, ids32, ids64, weights, tokens, experts, topk,
                                        static_cast<cudaStream_t>(stream)),
                       "moe_topk_route");
}

int moe_route(const void* x_bf16, const float* router_weight, const float* bias, float* logits,
              int32_t* ids32, int64_t* ids64, float* weights, int64_t tokens, int64_t hidden,
              int32_t experts, int32_t topk, void* stream) {
    if (hidden < 8 || hidden % 8 || hidden > INT_MAX)
        return fail(MOE_ERR_INVALID, "hidden must be a positive multiple of 8");
    if (tokens > 0 && (!x_bf16 || !router_weight))
        return fail(MOE_ERR_INVALID, "x and router_weight must be non-null");
    if (tokens > 0 && experts > moe::kRouterSlicedMaxExperts && !logits)
        return fail(MOE_ERR_INVALID, "logits must be non-null for more than %d experts",
                    moe::kRouterSlicedMaxExperts);
    if (tokens > 0 && (!aligned(x_bf16, 16) || !aligned(router_weight, 16)))
        return fail(MOE_ERR_INVALID, "x and router_weight must be 16-byte aligned");
    if (experts < 1 || experts > moe::kMaxRouteExperts)
        return fail(MOE_ERR_INVALID, "routing supports 1..%d experts", moe::kMaxRouteExperts);
    if (tokens < 0) return fail(MOE_ERR_INVALID, "tokens must be >= 0");
    if (topk < 1 || topk > moe::kMaxTopk || topk > experts)
        return fail(MOE_ERR_INVALID, "topk must be in 1..min(experts, %d)", moe::kMaxTopk);
    if (tokens > INT_MAX / experts || tokens * topk > INT_MAX)
        return fail(MOE_ERR_INVALID, "shape exceeds int32 indexing capacity");
    if (tokens > 0 && (!ids32 || !weights)) return fail(MOE_ERR_INVALID, "ids32 and weights must be non-null");
    return cuda_status(moe::launch_route(x_bf16, router_weight, bias, logits, ids32, ids64, weights,
                                         tokens, hidden, experts, topk,
                                         static_cast<cudaStream_t>(stream)),
                       "moe_route");
}

int64_t moe_dispatch_scratch_bytes(int64_t tokens, int32_t topk, int32_t experts) {
    if (tokens < 0 || topk < 1 || experts < 1) return -1;
    return moe::dispatch_scratch_bytes(tokens * topk, experts);
}

}  // extern "C"

namespace moe {

// Every check moe_dispatch makes on its arguments except the scratch buffer's,
// so callers that supply the scratch themselves can validate first.
int check_dispatch_args(const void* x, int32_t dtype, const int32_t* ids, const int32_t* counts,
                        const int32_t* offsets, const int32_t* slots, const void* packed,
                        const int32_t* inverse, int64_t tokens, int64_t hidden, int32_t topk,
                        int32_t experts, int64_t packed_rows, int32_t alignment) {
    if (!valid_dtype(dtype)) return fail(MOE_ERR_INVALID, "only FP32, FP16, and BF16 are supported");
    if (tokens < 0 || hidden < 1) return fail(MOE_ERR_INVALID, "incompatible token dimensions");
    if (topk < 1 || topk > moe::kMaxTopk)
        return fail(MOE_ERR_INVALID, "topk must be in 1..%d", moe::kMaxTopk);
    if (experts < 1 || experts > moe::kMaxDispatchExperts)
        return fail(MOE_ERR_INVALID, "dispatch supports 1..%d experts", moe::kMaxDispatchExperts);
    if (alignment < 1 || alignment > 128) return fail(MOE_ERR_INVALID, "alignment must be 1..128");
    const int64_t n = tokens * topk;
    const int64_t required =
        alignment == 1 ? n
                       : (n + static_cast<int64_t>(experts) * (alignment - 1) + 1 + alignment - 1) /
                             alignment * alignment;
    if (n > INT_MAX || hidden > INT_MAX || required > INT_MAX)
        return fail(MOE_ERR_INVALID, "shape exceeds int32 indexing capacity");
    if (alignment == 1 ? packed_rows != n : packed_rows < required)
        return fail(MOE_ERR_INVALID, "incorrect packed workspace: %lld rows, need %s%lld",
                    static_cast<long long>(packed_rows), alignment == 1 ? "" : ">= ",
                    static_cast<long long>(required));
    if (!counts || !offsets || (n > 0 && (!x || !ids || !slots || !packed || !inverse)))
        return fail(MOE_ERR_INVALID, "null workspace pointer");
    const int elem = moe::dtype_bytes(dtype);
    if (!aligned(x, elem) || !aligned(packed, elem))
        return fail(MOE_ERR_INVALID, "x and packed must be aligned to their element size");
    return MOE_OK;
}

}  // namespace moe

extern "C" {

int moe_dispatch(const void* x, int32_t dtype, const int32_t* ids, int32_t* counts,
                 int32_t* offsets, int32_t* slots, void* packed, int32_t* inverse, int64_t tokens,
                 int64_t hidden, int32_t topk, int32_t experts, int64_t packed_rows,
                 int32_t alignment, int32_t vectorized, void* scratch, int64_t scratch_bytes,
                 void* stream) {
    const int checked = moe::check_dispatch_args(x, dtype, ids, counts, offsets, slots, packed,
                                                 inverse, tokens, hidden, topk, experts,
                                                 packed_rows, alignment);
    if (checked != MOE_OK) return checked;
    const int64_t n = tokens * topk;
    if (!scratch) return fail(MOE_ERR_INVALID, "null workspace pointer");
    if (scratch_bytes < moe::dispatch_scratch_bytes(n, experts) || !aligned(scratch, 16))
        return fail(MOE_ERR_INVALID, "dispatch scratch too small or unaligned (%lld bytes needed)",
                    static_cast<long long>(moe::dispatch_scratch_bytes(n, experts)));
    const int elem = moe::dtype_bytes(dtype);
    const int64_t row_bytes = hidden * elem;
    // vectorized: the widest copy the rows allow; otherwise one element per copy
    // (the reference's pack_scalar_kernel, dispatch.cu:36-50).
    const int vb = vectorized ? vector_bytes(row_bytes, elem, {x, packed}) : elem;
    return cuda_status(moe::launch_dispatch(x, dtype, ids, counts, offsets, slots, packed, inverse,
                                            tokens, hidden, topk, experts, packed_rows, alignment,
                                            vb, static_cast<int32_t*>(scratch),
                                            static_cast<cudaStream_t>(stream)),
                       "moe_dispatch");
}

int moe_combine(const void* expert_output, int32_t dtype, const int32_t* inverse,
                const float* weights, void* output, int64_t tokens, int64_t hidden, int32_t topk,
                int64_t packed_rows, void* stream) {
    if (!valid_dtype(dtype)) return fail(MOE_ERR_INVALID, "unsupported output dtype");
    if (topk < 1 || topk > moe::kMaxTopk)
        return fail(MOE_ERR_INVALID, "topk must be in 1..%d", moe::kMaxTopk);
    if (tokens < 0 || hidden < 1 || tokens * topk > INT_MAX || hidden > INT_MAX)
        return fail(MOE_ERR_INVALID, "invalid output shape");
    if (packed_rows < tokens * topk) return fail(MOE_ERR_INVALID, "shape/dtype mismatch");
    if (tokens > 0 && (!expert_output || !inverse || !weights || !output))
        return fail(MOE_ERR_INVALID, "null pointer");
    const int elem = moe::dtype_bytes(dtype);
    const int vb = vector_bytes(hidden * elem, elem, {expert_output, output});
    return cuda_status(moe::launch_combine(expert_output, dtype, inverse, weights, output, tokens,
                                           hidden, topk, packed_rows, vb,
                                           static_cast<cudaStream_t>(stream)),
                       "moe_combine");
}

int moe_swiglu(const void* projection, int32_t dtype, const int32_t* valid_rows, void* output,
               int64_t rows, int64_t width, void* stream) {
    if (!valid_dtype(dtype)) return fail(MOE_ERR_INVALID, "unsupported dtype");
    if (rows < 0 || width < 0 || rows > INT_MAX || width > INT_MAX)
        return fail(MOE_ERR_INVALID, "shape exceeds index capacity");
    if (rows * width > 0 && (!projection || !valid_rows || !output))
        return fail(MOE_ERR_INVALID, "null pointer");
    const int elem = moe::dtype_bytes(dtype);
    const int vb = vector_bytes(width * elem, elem, {projection, output});
    // the up half starts width elements into each row: it must keep the vector alignment
    const int vb_ok = ((width * elem) % vb == 0) ? vb : elem;
    return cuda_status(moe::launch_swiglu(projection, dtype, valid_rows, output, rows, width, vb_ok,
                                          static_cast<cudaStream_t>(stream)),
                       "moe_swiglu");
}

static int grouped_gemm_common(const void* a, const void* w, const int32_t* offsets, void* out,
                               int64_t rows, int64_t n_out, int64_t k_dim, int32_t experts,
                               bool swiglu, void* stream) {
    if (rows < 0 || rows > INT_MAX) return fail(MOE_ERR_INVALID, "rows must be in 0..INT_MAX");
    if (n_out < 8 || n_out % 8 || k_dim < 8 || k_dim % 8)
        return fail(MOE_ERR_INVALID, "grouped GEMM dimensions must be positive multiples of 8");
    if (experts < 1) return fail(MOE_ERR_INVALID, "experts must be >= 1");
    const int64_t b_rows = (swiglu ? 2 : 1) * n_out * static_cast<int64_t>(experts);
    if (b_rows > INT_MAX || n_out > INT_MAX / 2)
        return fail(MOE_ERR_INVALID, "weight shape exceeds int32 coordinates");
    if (rows > 0 && (!a || !w || !offsets || !out)) return fail(MOE_ERR_INVALID, "null pointer");
    if (rows > 0 && (!aligned(a, 16) || !aligned(w, 16) || !aligned(out, 16)))
        return fail(MOE_ERR_INVALID, "GEMM operands must be 16-byte aligned");
    const char* message = nullptr;
    cudaError_t err = moe::launch_grouped_gemm(a, w, offsets, out, rows, n_out, k_dim, experts,
                                               swiglu, static_cast<cudaStream_t>(stream), &message);
    if (message) return fail(MOE_ERR_INVALID, "%s", message);
    return cuda_status(err, swiglu ? "moe_grouped_gemm_swiglu" : "moe_grouped_gemm");
}

int moe_grouped_gemm_swiglu(const void* packed, const void* gate_up, const int32_t* offsets,
                            void* activated, int64_t rows, int64_t hidden, int64_t intermediate,
                            int32_t experts, void* stream) {
    return grouped_gemm_common(packed, gate_up, offsets, activated, rows, intermediate, hidden,
                               experts, true, stream);
}

int moe_grouped_gemm(const void* a, const void* weight, const int32_t* offsets, void* out,
                     int64_t rows, int64_t n_cols, int64_t k_dim, int32_t experts, void* stream) {
    return grouped_gemm_common(a, weight, offsets, out, rows, n_cols, k_dim, experts, false, stream);
}

int moe_quantize_rows_e4m3(const void* x, int32_t dtype, void* q, float* scale, int64_t rows,
                           int64_t cols, void* stream) {
    if (dtype != moe::kBF16) return fail(MOE_ERR_INVALID, "e4m3 quantisation takes bf16 rows");
    if (rows < 0 || cols < 8 || cols % 16 || rows > INT_MAX)
        return fail(MOE_ERR_INVALID, "e4m3 rows need cols a positive multiple of 16");
    if (rows > 0 && (!x || !q || !scale)) return fail(MOE_ERR_INVALID, "null pointer");
    if (rows > 0 && (!aligned(x, 16) || !aligned(q, 16) || !aligned(scale, 4)))
        return fail(MOE_ERR_INVALID, "x and q must be 16-byte aligned");
    return cuda_status(moe::launch_quantize_rows_e4m3(x, q, scale, rows, cols,
                                                      static_cast<cudaStream_t>(stream)),
                       "moe_quantize_rows_e4m3");
}

static int grouped_gemm_e4m3_common(const void* a, const float* a_scale, const void* w,
                                    const float* w_scale, const int32_t* offsets, void* out,
                                    int64_t rows, int64_t n_out, int64_t k_dim, int32_t experts,
                                    bool swiglu, void* stream) {
    if (rows < 0 || rows > INT_MAX) return fail(MOE_ERR_INVALID, "rows must be in 0..INT_MAX");
    if (n_out < 8 || n_out % 8 || k_dim < 16 || k_dim % 16)
        return fail(MOE_ERR_INVALID,
                    "e4m3 grouped GEMM needs n a positive multiple of 8 and k of 16");
    if (experts < 1) return fail(MOE_ERR_INVALID, "experts must be >= 1");
    const int64_t b_rows = (swiglu ? 2 : 1) * n_out * static_cast<int64_t>(experts);
    if (b_rows > INT_MAX || n_out > INT_MAX / 2)
        return fail(MOE_ERR_INVALID, "weight shape exceeds int32 coordinates");
    if (rows > 0 && (!a || !a_scale || !w || !w_scale || !offsets || !out))
        return fail(MOE_ERR_INVALID, "null pointer");
    if (rows > 0 && (!aligned(a, 16) || !aligned(w, 16) || !aligned(out, 16)))
        return fail(MOE_ERR_INVALID, "GEMM operands must be 16-byte aligned");
    const char* message = nullptr;
    cudaError_t err = moe::launch_grouped_gemm(a, w, offsets, out, rows, n_out, k_dim, experts,
                                               swiglu, static_cast<cudaStream_t>(stream), &message,
                                               a_scale, w_scale);
    if (message) return fail(MOE_ERR_INVALID, "%s", message);
    return cuda_status(err, swiglu ? "moe_grouped_gemm_swiglu_e4m3" : "moe_grouped_gemm_e4m3");
}

int moe_grouped_gemm_swiglu_e4m3(const void* packed_q, const float* packed_scale,
                                 const void* gate_up_q, const float* gate_up_scale,
                                 const int32_t* offsets, void* activated, int64_t rows,
                                 int64_t hidden, int64_t intermediate, int32_t experts,
                                 void* stream) {
    return grouped_gemm_e4m3_common(packed_q, packed_scale, gate_up_q, gate_up_scale, offsets,
                                    activated, rows, intermediate, hidden, experts, true, stream);
}

int moe_grouped_gemm_e4m3(const void* a_q, const float* a_scale, const void* weight_q,
                          const float* weight_scale, const int32_t* offsets, void* out,
                          int64_t rows, int64_t n_cols, int64_t k_dim, int32_t experts,
                          void* stream) {
    return grouped_gemm_e4m3_common(a_q, a_scale, weight_q, weight_scale, offsets, out, rows,
                                    n_cols, k_dim, experts, false, stream);
}

int32_t moe_grouped_gemm_tile(int64_t rows, int32_t experts) {
    return moe::grouped_gemm_uses_pair(rows, experts) ? 1 : 0;
}

int moe_ep_layout(const int32_t* counts, int32_t ranks, int32_t experts, int32_t alignment,
                  int32_t* src_start, int32_t* dst_start, int32_t* offsets, void* stream) {
    if (ranks < 1 || experts < 1 || static_cast<int64_t>(ranks) * experts > (1 << 20))
        return fail(MOE_ERR_INVALID, "expert-parallel layout needs 1 <= ranks*experts <= 2^20");
    if (alignment < 1 || alignment > 128) return fail(MOE_ERR_INVALID, "alignment must be 1..128");
    if (!counts || !src_start || !dst_start || !offsets) return fail(MOE_ERR_INVALID, "null pointer");
    return cuda_status(moe::launch_ep_layout(counts, ranks, experts, alignment, src_start, dst_start,
                                             offsets, static_cast<cudaStream_t>(stream)),
                       "moe_ep_layout");
}

int moe_ep_regroup(const void* from, int32_t dtype, void* to, const int32_t* counts,
                   const int32_t* src_start, const int32_t* dst_start, const int32_t* offsets,
                   int32_t ranks, int32_t experts, int64_t hidden, int64_t recv_rows,
                   int64_t grouped_rows, int32_t grouping, void* stream) {
    if (!valid_dtype(dtype)) return fail(MOE_ERR_INVALID, "unsupported dtype");
    if (ranks < 1 || experts < 1 || hidden < 1 || recv_rows < 0 || grouped_rows < 0)
        return fail(MOE_ERR_INVALID, "invalid expert-parallel regroup shape");
    if (recv_rows > INT_MAX || grouped_rows > INT_MAX)
        return fail(MOE_ERR_INVALID, "shape exceeds int32 indexing capacity");
    if ((recv_rows > 0 || grouped_rows > 0) &&
        (!from || !to || !counts || !src_start || !dst_start || !offsets))
        return fail(MOE_ERR_INVALID, "null pointer");
    const int elem = moe::dtype_bytes(dtype);
    if (!aligned(from, elem) || !aligned(to, elem))
        return fail(MOE_ERR_INVALID, "rows must be aligned to their element size");
    const int vb = vector_bytes(hidden * elem, elem, {from, to});
    return cuda_status(moe::launch_ep_regroup(from, to, counts, src_start, dst_start, offsets, ranks,
                                              experts, hidden * elem, recv_rows, grouped_rows,
                                              grouping != 0, vb, static_cast<cudaStream_t>(stream)),
                       "moe_ep_regroup");
}

int moe_peer_alloc(int64_t bytes, void** ptr, void* ipc_handle) {
    if (bytes < 1 || !ptr || !ipc_handle) return fail(MOE_ERR_INVALID, "invalid peer allocation");
    void* p = nullptr;
    cudaError_t err = cudaMalloc(&p, static_cast<size_t>(bytes));
    if (err != cudaSuccess) return cuda_status(err, "moe_peer_alloc (cudaMalloc)");
    err = cudaMemset(p, 0, static_cast<size_t>(bytes));
    if (err == cudaSuccess)
        err = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
    if (err != cudaSuccess) {
        cudaFree(p);
        return cuda_status(err, "moe_peer_alloc");
    }
    *ptr = p;
    return MOE_OK;
}

int moe_peer_open(const void* ipc_handle, void** ptr) {
    if (!ipc_handle || !ptr) return fail(MOE_ERR_INVALID, "null pointer");
    cudaIpcMemHandle_t handle;
    memcpy(&handle, ipc_handle, sizeof(handle));
    return cuda_status(cudaIpcOpenMemHandle(ptr, handle, cudaIpcMemLazyEnablePeerAccess),
                       "moe_peer_open");
}

int moe_peer_close(void* ptr) {
    if (!ptr) return fail(MOE_ERR_INVALID, "null pointer");
    return cuda_status(cudaIpcCloseMemHandle(ptr), "moe_peer_close");
}

int moe_peer_free(void* ptr) {
    if (!ptr) return fail(MOE_ERR_INVALID, "null pointer");
    return cuda_status(cudaFree(ptr), "moe_peer_free");
}

int64_t moe_ep_p2p_region_bytes(int32_t ranks, int32_t experts, int64_t hidden,
                                int64_t grouped_rows, int64_t back_rows) {
    if (ranks < 1 || ranks > moe::kEpP2pMaxRanks || experts < ranks || experts % ranks ||
        hidden < 8 || hidden % 8 || grouped_rows < 0 || back_rows < 0)
        return -1;
    return moe::ep_p2p_region_bytes(ranks, experts, hidden, grouped_rows, back_rows);
}

int64_t moe_ep_p2p_region_offset(int32_t ranks, int32_t experts, int64_t hidden,
                                 int64_t grouped_rows, int64_t back_rows, int32_t section) {
    if (moe_ep_p2p_region_bytes(ranks, experts, hidden, grouped_rows, back_rows) < 0 ||
        section < 0 || section > 1)
        return -1;
    return moe::ep_p2p_region_offset(ranks, experts, hidden, grouped_rows, back_rows, section);
}

int64_t moe_ep_p2p_state_words(int32_t ranks, int32_t experts) {
    if (ranks < 1 || experts < ranks || experts % ranks) return -1;
    return moe::ep_p2p_state_words(ranks, experts);
}

int moe_ep_p2p(int32_t op, const void* rows, const int32_t* aux, void* const* regions,
               int32_t* state, int32_t ranks, int32_t rank, int32_t experts, int32_t alignment,
               int64_t hidden, int64_t grouped_rows, int64_t back_rows, int64_t timeout_ms,
               void* stream) {
    if (moe_ep_p2p_region_bytes(ranks, experts, hidden, grouped_rows, back_rows) < 0)
        return fail(MOE_ERR_INVALID, "expert-parallel P2P: 1 <= ranks <= %d, experts a multiple "
                                     "of ranks, hidden a multiple of 8", moe::kEpP2pMaxRanks);
    if (rank < 0 || rank >= ranks) return fail(MOE_ERR_INVALID, "rank out of range");
    if (experts > moe::kMaxRouteExperts)
        return fail(MOE_ERR_INVALID, "expert-parallel P2P supports up to %d experts",
                    moe::kMaxRouteExperts);
    if (alignment < 1 || alignment > 128) return fail(MOE_ERR_INVALID, "alignment must be 1..128");
    if (op < moe::kEpP2pCounts || op > moe::kEpP2pSendRemote) return fail(MOE_ERR_INVALID, "bad op");
    if (!regions || !state) return fail(MOE_ERR_INVALID, "null pointer");
    for (int i = 0; i < ranks; ++i)
        if (!regions[i] || !aligned(regions[i], 1024))
            return fail(MOE_ERR_INVALID, "peer regions must be non-null and 1024-byte aligned");
    const bool sends = op == moe::kEpP2pSend || op == moe::kEpP2pSendLocal ||
                       op == moe::kEpP2pSendRemote;
    if ((op == moe::kEpP2pCounts || sends) && !aux)
        return fail(MOE_ERR_INVALID, "counts / dispatch offsets required");
    if ((sends || op == moe::kEpP2pReturn) && (!rows || !aligned(rows, 16)))
        return fail(MOE_ERR_INVALID, "rows must be non-null and 16-byte aligned");
    if (timeout_ms < 1) return fail(MOE_ERR_INVALID, "timeout_ms must be >= 1");
    return cuda_status(moe::launch_ep_p2p(op, rows, aux, regions, state, ranks, rank, experts,
                                          alignment, hidden, grouped_rows, back_rows, timeout_ms,
                                          static_cast<cudaStream_t>(stream)),
                       "moe_ep_p2p");
}

int moe_ep_p2p_gate_up(const void* gate_up, void* activated, void* const* regions, int32_t* state,
                       int32_t ranks, int32_t rank, int32_t experts, int64_t hidden,
                       int64_t intermediate, int64_t grouped_rows, int64_t back_rows,
                       int64_t timeout_ms, void* stream) {
    if (moe_ep_p2p_region_bytes(ranks, experts, hidden, grouped_rows, back_rows) < 0)
        return fail(MOE_ERR_INVALID, "expert-parallel P2P: 1 <= ranks <= %d, experts a multiple "
                                     "of ranks, hidden a multiple of 8", moe::kEpP2pMaxRanks);
    if (rank < 0 || rank >= ranks) return fail(MOE_ERR_INVALID, "rank out of range");
    if (intermediate < 8 || intermediate % 8 || grouped_rows < 1 || grouped_rows > INT_MAX)
        return fail(MOE_ERR_INVALID, "invalid gate/up GEMM shape");
    if (!gate_up || !activated || !regions || !state || !aligned(gate_up, 16) ||
        !aligned(activated, 16))
        return fail(MOE_ERR_INVALID, "null or unaligned pointer");
    for (int i = 0; i < ranks; ++i)
        if (!regions[i] || !aligned(regions[i], 1024))
            return fail(MOE_ERR_INVALID, "peer regions must be non-null and 1024-byte aligned");
    if (timeout_ms < 1) return fail(MOE_ERR_INVALID, "timeout_ms must be >= 1");
    const char* message = nullptr;
    cudaError_t err = moe::launch_ep_p2p_gate_up(gate_up, activated, regions, state, ranks, rank,
                                                 experts, hidden, intermediate, grouped_rows,
                                                 back_rows, timeout_ms,
                                                 static_cast<cudaStream_t>(stream), &message);
    if (message) return fail(MOE_ERR_INVALID, "%s", message);
    return cuda_status(err, "moe_ep_p2p_gate_up");
}

int moe_ep_p2p_down_return(const void* activated, const void* down, void* const* regions,
                           int32_t* state, int32_t ranks, int32_t rank, int32_t experts,
                           int64_t hidden, int64_t intermediate, int64_t grouped_rows,
                           int64_t back_rows, void* stream) {
    if (moe_ep_p2p_region_bytes(ranks, experts, hidden, grouped_rows, back_rows) < 0)
        return fail(MOE_ERR_INVALID, "expert-parallel P2P: 1 <= ranks <= %d, experts a multiple "
                                     "of ranks, hidden a multiple of 8", moe::kEpP2pMaxRanks);
    if (rank < 0 || rank >= ranks) return fail(MOE_ERR_INVALID, "rank out of range");
    if (intermediate < 8 || intermediate % 8 || grouped_rows < 1 || grouped_rows > INT_MAX)
        return fail(MOE_ERR_INVALID, "invalid down GEMM shape");
    if (!activated || !down || !regions || !state || !aligned(activated, 16) || !aligned(down, 16))
        return fail(MOE_ERR_INVALID, "null or unaligned pointer");
    for (int i = 0; i < ranks; ++i)
        if (!regions[i] || !aligned(regions[i], 1024))
            return fail(MOE_ERR_INVALID, "peer regions must be non-null and 1024-byte aligned");
    const char* message = nullptr;
    cudaError_t err = moe::launch_ep_p2p_down_return(activated, down, regions, state, ranks, rank,
                                                     experts, hidden, intermediate, grouped_rows,
                                                     back_rows, static_cast<cudaStream_t>(stream),
                                                     &message);
    if (message) return fail(MOE_ERR_INVALID, "%s", message);
    return cuda_status(err, "moe_ep_p2p_down_return");
}

int moe_device_status(int32_t* code, int32_t clear) {
    if (!code) return fail(MOE_ERR_INVALID, "code must be non-null");
    int32_t gemm = 0, ep = 0, route = 0;
    int status = cuda_status(moe::read_gemm_status(&gemm, clear != 0), "moe_device_status");
    if (status != MOE_OK) return status;
    status = cuda_status(moe::read_ep_status(&ep, clear != 0), "moe_device_status");
    if (status != MOE_OK) return status;
    status = cuda_status(moe::read_route_status(&route, clear != 0), "moe_device_status");
    *code = gemm ? gemm : (ep ? ep : route);
    return status;
}

}  // extern "C"
