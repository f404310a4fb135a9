/*
 * moe_b200.h -- C ABI of the B200 (sm_100a) MoE feed-forward library.
 *
 * Plain pointers and sizes; no torch types.  Every entry point:
 *   - works on the calling thread's current CUDA device;
 *   - takes caller-allocated inputs and outputs (it never allocates);
 *   - enqueues asynchronously on `stream` (a cudaStream_t; NULL = legacy
 *     default stream) and performs no host synchronisation, so it can be
 *     captured in a CUDA graph;
 *   - returns MOE_OK or an error code; moe_last_error() gives the message
 *     of the calling thread's last failure.
 *
 * The reference (AarushRathore1729/cuda-moe-engine) binds five torch
 * functions through pybind (src/moe_dispatch/csrc/bindings.cpp:3-13).  Each
 * of them maps to one entry point here, cited beside it; the others are the
 * fused stages the reference runs through torch/cuBLAS/Triton.
 *
 * Element types: MOE_F32, MOE_F16, MOE_BF16.  Index tensors are int32,
 * routing weights fp32, ids64 int64 -- the reference's dtypes.
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum moe_dtype { MOE_F32 = 0, MOE_F16 = 1, MOE_BF16 = 2 };

enum moe_status {
    MOE_OK = 0,
    MOE_ERR_INVALID = 1,     /* bad shape, size, dtype or pointer alignment */
    MOE_ERR_CUDA = 2,        /* a CUDA runtime call or kernel launch failed */
    MOE_ERR_UNSUPPORTED = 3, /* valid request this build does not implement */
    MOE_ERR_DEVICE = 4       /* a kernel reported an error through its device status word */
};

/* ABI revision of this header. */
int moe_abi_version(void);

/* Message for the calling thread's last failing call ("" if none). */
const char* moe_last_error(void);

/* ---------------------------------------------------------------- routing */

/* Replaces topk_route_out (src/moe_dispatch/csrc/dispatch.cu:378-402,
 * bindings.cpp:13-14): top-k over logits + bias with ties to the lower expert
 * index, softmax over the selected scores.  Lifts the reference's limits
 * (topk 1..2, experts <= 64) to topk 1..32, experts 1..256. */
int moe_topk_route(const float* logits, const float* bias, int32_t* ids32, int64_t* ids64,
                   float* weights, int64_t tokens, int32_t experts, int32_t topk, void* stream);

/* Replaces MoEBlock.route for implementation="cuda_fused"
 * (src/moe_dispatch/layer.py:122-135): fp32 router logits from bf16 x
 * (F.linear(x.float(), W), layer.py:123), then the selection of
 * moe_topk_route.  The fp32 summation order of a logit is fixed: for
 * experts <= 32, 32 slices (slice l = the h with (h/8) mod 32 == l), each a
 * sequential FMA chain in increasing h, combined by a xor butterfly
 * (off = 16, 8, 4, 2, 1); for more experts, one sequential FMA chain over h.  `logits` [T,E] receives
 * the logits; it may be NULL when experts <= 32.  hidden % 8 == 0. */
int moe_route(const void* x_bf16, const float* router_weight, const float* bias, float* logits,
              int32_t* ids32, int64_t* ids64, float* weights, int64_t tokens, int64_t hidden,
              int32_t experts, int32_t topk, void* stream);

/* --------------------------------------------------------------- transport */

/* Device scratch (bytes) that moe_dispatch needs for `tokens*topk`
 * assignments over `experts` experts. */
int64_t moe_dispatch_scratch_bytes(int64_t tokens, int32_t topk, int32_t experts);

/* Replaces dispatch_out (dispatch.cu:102-158, bindings.cpp:3-5) when
 * alignment == 1 and dispatch_aligned_out (dispatch.cu:218-275,
 * bindings.cpp:8-10) when alignment > 1.  Writes counts[E], offsets[E+1]
 * (each expert's span rounded up to `alignment`), slots[T*K] (rank of each
 * assignment inside its expert), inverse[T*K] (its packed row) and copies
 * each x row to its packed rows; padding rows are zeroed.  The order inside
 * an expert is the stable token-major order of p = t*K + k, deterministic
 * from run to run.  Out-of-range ids get slot and inverse -1, and int32
 * word 2 of `scratch` receives how many there were (a device-side range
 * check: the reference's ops.dispatch checks on the host, ops.py:38).
 * `vectorized` != 0 selects the widest vector copies the row allows.
 * `scratch` must hold moe_dispatch_scratch_bytes() bytes, zeroed once
 * before its first use; the call leaves it ready for the next call. */
int moe_dispatch(const void* x, int32_t dtype, const int32_t* ids, int32_t* counts,
                 int32_t* offsets, int32_t* slots, void* packed, int32_t* inverse, int64_t tokens,
                 int64_t hidden, int32_t topk, int32_t experts, int64_t packed_rows,
                 int32_t alignment, int32_t vectorized, void* scratch, int64_t scratch_bytes,
                 void* stream);

/* moe_dispatch for callers that cannot allocate device memory -- serving hosts
 * that fix their device memory at start-up and forbid allocation afterwards,
 * bindings that hold only raw device pointers.  No counterpart in the reference: its
 * dispatch needs no scratch because its order is whatever atomics give.
 * Same arguments and results as moe_dispatch, minus the scratch: that lives in
 * a fixed array compiled into the library (256 KiB + 64 B on every GPU that
 * loads it, until exit), which limits the size to
 *   ceil(tokens * topk / 1024) * experts <= 65536
 * (e.g. 262144 assignments over 256 experts); larger requests fail with
 * MOE_ERR_INVALID.  Arguments are checked before the array is touched, so a
 * rejected call has no device effect.  Allocates nothing (no cudaMalloc/cudaFree).  The first
 * call on a device looks up the array's device address; make it before any
 * stream capture.  All calls share the array: calls that overlap on the GPU
 * race and must be serialised by the caller. */
int moe_dispatch_no_alloc(const void* x, int32_t dtype, const int32_t* ids, int32_t* counts,
                          int32_t* offsets, int32_t* slots, void* packed, int32_t* inverse,
                          int64_t tokens, int64_t hidden, int32_t topk, int32_t experts,
                          int64_t packed_rows, int32_t alignment, int32_t vectorized,
                          void* stream);

/* Replaces combine_out (dispatch.cu:160-192, bindings.cpp:6-7):
 * out[t] = cast(sum_k fp32(w[t,k] * fp32(eo[inverse[t,k]]))), the products
 * rounded to fp32 and summed in k order (the PyTorch path's rounding,
 * reference.py:67-76).  Rows outside [0, packed_rows) are skipped. */
int moe_combine(const void* expert_output, int32_t dtype, const int32_t* inverse,
                const float* weights, void* output, int64_t tokens, int64_t hidden, int32_t topk,
                int64_t packed_rows, void* stream);

/* ----------------------------------------------------------------- experts */

/* Replaces swiglu_out (dispatch.cu:294-323, bindings.cpp:11):
 * out[r,c] = cast(silu(fp32 proj[r,c]) * fp32 proj[r,c+width]) for
 * r < *valid_rows (a device int32), zero for the other rows. */
int moe_swiglu(const void* projection, int32_t dtype, const int32_t* valid_rows, void* output,
               int64_t rows, int64_t width, void* stream);

/* Replaces the gate/up grouped_linear plus swiglu_out of
 * MoEBlock.experts_forward (layer.py:162-172; experts.py:21-35;
 * _triton_gemm.py:16-104).  bf16 only.  For each expert e and packed row r in
 * [offsets[e], offsets[e+1]):
 *   g = bf16(packed[r] . gate_up[e, c]),  u = bf16(packed[r] . gate_up[e, I+c])
 *   activated[r, c] = bf16(silu(g) * u)                      (c < intermediate)
 * packed [rows, hidden], gate_up [experts, 2*intermediate, hidden],
 * activated [rows, intermediate]; fp32 accumulation on tcgen05 tensor cores.
 * hidden and intermediate must be multiples of 8.  Rows at or beyond
 * offsets[experts] are not written. */
int moe_grouped_gemm_swiglu(const void* packed, const void* gate_up, const int32_t* offsets,
                            void* activated, int64_t rows, int64_t hidden, int64_t intermediate,
                            int32_t experts, void* stream);

/* Replaces the down grouped_linear of MoEBlock.experts_forward
 * (layer.py:175-181): out[r] = bf16(a[r] . weight[e]^T) for r in expert e's
 * rows.  a [rows, k_dim], weight [experts, n_cols, k_dim], out [rows, n_cols];
 * bf16, n_cols and k_dim multiples of 8. */
int moe_grouped_gemm(const void* a, const void* weight, const int32_t* offsets, void* out,
                     int64_t rows, int64_t n_cols, int64_t k_dim, int32_t experts, void* stream);

/* ------------------------------------------------------ FP8 (e4m3) experts
 * No counterpart in the reference, whose experts are bf16 only
 * (layer.py:97-98): an extension on tcgen05.mma.kind::f8f6f4. */

/* e4m3 quantisation of bf16 rows x[rows, cols] (dtype must be BF16, cols a
 * multiple of 16): scale[r] = amax_r / 448 and q[r, c] = e4m3(x[r, c] *
 * (448 / amax_r)) rounded to nearest even and saturated at +-448, so
 * x ~ q * scale; an all-zero row gets scale 1 and zeros.  Used for the packed
 * activation rows before the e4m3 gate/up GEMM, and once for the weights
 * (one scale per output channel = weight row). */
int moe_quantize_rows_e4m3(const void* x, int32_t dtype, void* q, float* scale, int64_t rows,
                           int64_t cols, void* stream);

/* moe_grouped_gemm_swiglu with e4m3 operands: packed_q [rows, hidden] with
 * packed_scale [rows], gate_up_q [experts, 2*intermediate, hidden] with
 * gate_up_scale [experts * 2 * intermediate].  The e4m3 products are exact
 * and accumulate in fp32; then g = bf16((acc_g * packed_scale[r]) *
 * gate_up_scale[gate row]), u likewise, activated = bf16(silu(g) * u).
 * hidden must be a multiple of 16. */
int moe_grouped_gemm_swiglu_e4m3(const void* packed_q, const float* packed_scale,
                                 const void* gate_up_q, const float* gate_up_scale,
                                 const int32_t* offsets, void* activated, int64_t rows,
                                 int64_t hidden, int64_t intermediate, int32_t experts,
                                 void* stream);

/* moe_grouped_gemm with e4m3 operands: out[r, c] = bf16((acc * a_scale[r]) *
 * weight_scale[e * n_cols + c]). */
int moe_grouped_gemm_e4m3(const void* a_q, const float* a_scale, const void* weight_q,
                          const float* weight_scale, const int32_t* offsets, void* out,
                          int64_t rows, int64_t n_cols, int64_t k_dim, int32_t experts,
                          void* stream);

/* Which tile the two grouped GEMMs above use for `rows` packed rows over
 * `experts` experts (no counterpart in the reference): 1 = the 256-row
 * CTA-pair tile (cta_group::2), 0 = the 128-row one-CTA tile.  Every tile
 * kind gives the same bits; the choice only changes speed.  The environment
 * variable MOE_B200_GEMM_TILE=pair|single overrides it.  A bf16 pair launch
 * runs the operand-swapped pair tile (weights as the 256-row side, each
 * expert's rows spread over tiles of up to 256); MOE_B200_GEMM_SWAP=0 keeps
 * the pair tile over 256-row blocks of packed rows. */
int32_t moe_grouped_gemm_tile(int64_t rows, int32_t experts);

/* ------------------------------------------------------- expert parallel */

/* Receive layout for expert parallelism (no counterpart in the reference,
 * which is single-GPU, README.md:161-163).  counts[P][E_l] (device int32)
 * holds how many rows each of P source ranks sent for each of this rank's
 * E_l experts; they arrive source-major, each source's rows expert-major.
 * Writes src_start[P][E_l] (first received row of each segment),
 * dst_start[P][E_l] (its first row in the grouped layout) and
 * offsets[E_l+1]: expert-major spans rounded up to `alignment`, source-major
 * inside an expert -- which is the global token order, so grouped rows equal
 * what a single GPU would pack for these experts. */
int moe_ep_layout(const int32_t* counts, int32_t ranks, int32_t experts, int32_t alignment,
                  int32_t* src_start, int32_t* dst_start, int32_t* offsets, void* stream);

/* Moves rows between the received (source-major) and grouped (expert-major)
 * layouts of moe_ep_layout: grouping != 0 copies received -> grouped and
 * zeroes each expert's padding rows; grouping == 0 copies grouped rows back
 * to received order (for the return exchange).  `from`/`to` are [rows, hidden]
 * of `dtype`; recv_rows = sum(counts); grouped_rows = capacity of the grouped
 * buffer (rows at or past it are skipped). */
int moe_ep_regroup(const void* from, int32_t dtype, void* to, const int32_t* counts,
                   const int32_t* src_start, const int32_t* dst_start, const int32_t* offsets,
                   int32_t ranks, int32_t experts, int64_t hidden, int64_t recv_rows,
                   int64_t grouped_rows, int32_t grouping, void* stream);

/* Peer memory for the NVLink exchange (new; the reference is single-GPU).
 * moe_peer_alloc allocates `bytes` of zeroed device memory on the current
 * device and writes its 64-byte CUDA IPC handle to `ipc_handle`; another
 * process on the node maps it with moe_peer_open (and unmaps it with
 * moe_peer_close).  moe_peer_free releases the allocation.  Set-up calls:
 * they allocate and synchronise, so make them outside any timed or captured
 * region. */
int moe_peer_alloc(int64_t bytes, void** ptr, void* ipc_handle);
int moe_peer_open(const void* ipc_handle, void** ptr);
int moe_peer_close(void* ptr);
int moe_peer_free(void* ptr);

/* Layout of one rank's exchange region and local state for the P2P
 * expert-parallel step (ranks <= 8, experts a multiple of ranks, bf16 rows of
 * `hidden`): total bytes; byte offset of the grouped rows (section 0, capacity
 * grouped_rows) or of the returned rows (section 1, capacity back_rows); and
 * the int32 words of per-rank local state (zeroed once before the first step).
 * -1 on invalid arguments. */
int64_t moe_ep_p2p_region_bytes(int32_t ranks, int32_t experts, int64_t hidden,
                                int64_t grouped_rows, int64_t back_rows);
int64_t moe_ep_p2p_region_offset(int32_t ranks, int32_t experts, int64_t hidden,
                                 int64_t grouped_rows, int64_t back_rows, int32_t section);
int64_t moe_ep_p2p_state_words(int32_t ranks, int32_t experts);

/* One stage of the P2P expert-parallel step, enqueued on `stream` (no host
 * sync).  regions[P] are the ranks' exchange regions as mapped in this process
 * (this rank's own at regions[rank]).  op:
 *   0 exchange counts: aux = counts[E] from moe_dispatch; writes them to every
 *     rank, waits for all ranks', computes the send/receive tables and this
 *     rank's grouped expert offsets (state words 4+E .. 4+E+E_l);
 *   1 send rows: rows = the compact packed rows, aux = moe_dispatch's offsets;
 *     each row lands in its expert owner's grouped rows, source-major inside
 *     an expert (the global token order); the last CTA raises the rows flags;
 *   2 wait until every rank's rows arrived;
 *   3 return rows: rows = this rank's expert outputs in grouped order; each
 *     row goes back to its source's returned rows at its packed position;
 *   4 wait until every rank's results came back;
 *   5 send local rows: op 1 for the rows of this rank's own experts only (an
 *     HBM copy, no flag: the launches after it on the stream see them);
 *   6 send remote rows: op 1 for the other ranks' rows; the rows flag of this
 *     source is raised on each owner as soon as that owner's rows are stored
 *     (at once on owners it sends nothing, and on this rank), so owners can
 *     start on them while it still sends to others.  Runs beside the gate/up
 *     GEMM of moe_ep_p2p_gate_up, on another stream.
 * Inside an expert's grouped span the sources' rows follow their arrival
 * order on the owner o: o's own rows, then those of o-1, o-2, ... (mod P).
 * Waits give up after timeout_ms, record status 2 (read by
 * moe_device_status) and return; capacity overflows record status 3. */
int moe_ep_p2p(int32_t op, const void* rows, const int32_t* aux, void* const* regions,
               int32_t* state, int32_t ranks, int32_t rank, int32_t experts, int32_t alignment,
               int64_t hidden, int64_t grouped_rows, int64_t back_rows, int64_t timeout_ms,
               void* stream);

/* The gate/up GEMM (+ SwiGLU) of the P2P expert-parallel step, overlapped
 * with the row exchange (no counterpart in the reference, which is
 * single-GPU; replaces op 2 + moe_grouped_gemm_swiglu on the grouped rows):
 * activated [grouped_rows, intermediate] = swiglu(grouped rows x this rank's
 * gate_up [E_l, 2*intermediate, hidden]).  It takes the tiles of each expert
 * in arrival order -- first those of this rank's own rows (op 5, before it on
 * the stream), then, source by source, those whose rows have arrived (ops 6
 * of the other ranks): before a tile's first load the producer waits on the
 * rows flags it needs (bounded by timeout_ms; status 6).  The same bits as
 * moe_grouped_gemm_swiglu on the same rows. */
int moe_ep_p2p_gate_up(const void* gate_up, void* activated, void* const* regions, int32_t* state,
                       int32_t ranks, int32_t rank, int32_t experts, int64_t hidden,
                       int64_t intermediate, int64_t grouped_rows, int64_t back_rows,
                       int64_t timeout_ms, void* stream);

/* The down GEMM of the P2P expert-parallel step fused with the return
 * exchange (replaces moe_grouped_gemm + op 3 of moe_ep_p2p): tcgen05 grouped
 * GEMM of activated [grouped_rows, intermediate] with this rank's down
 * weights [E_l, hidden, intermediate]; its epilogue stores every result row
 * straight into its source rank's returned rows at the packed position, and
 * the last CTA raises the return flags.  Follow it with op 4 (wait). */
int moe_ep_p2p_down_return(const void* activated, const void* down, void* const* regions,
                           int32_t* state, int32_t ranks, int32_t rank, int32_t experts,
                           int64_t hidden, int64_t intermediate, int64_t grouped_rows,
                           int64_t back_rows, void* stream);

/* ------------------------------------------------------------ diagnostics */

/* Reads (and with clear != 0 resets) the current device's status words, which
 * kernels with bounded waits set when a wait runs out.  0 means no error;
 * 1 a grouped-GEMM pipeline wait, 2 an expert-parallel peer wait, 3 an
 * expert-parallel capacity overflow, 4 a router copy wait, 5 two grouped-GEMM
 * launches that shared one tile-claim slot at the same time (one captured
 * graph replayed on two streams at once, or more than 512 captured GEMM
 * launches in flight together); their results are void; 6 a gate/up GEMM of
 * moe_ep_p2p_gate_up that gave up waiting for a peer's rows. */
int moe_device_status(int32_t* code, int32_t clear);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H */
