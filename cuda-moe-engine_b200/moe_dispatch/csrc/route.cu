// Router: fp32 logits from bf16 tokens, then top-k + softmax (sm_100a).
//
// Reference behaviour (src/moe_dispatch/layer.py:122-139, csrc/dispatch.cu:325-376):
//   logits = F.linear(x.float(), W)             (fp32)
//   values = logits + bias                      (fp32 add)
//   top-k of values, ties -> lower expert index
//   weights = softmax(selected values)
//
// Logit order (the CPU oracle restates it, so logits -- and hence the selected
// experts -- are bit-identical between the two):
//   E <= 32: slice l (l = 0..31) holds the elements h with (h / 8) mod 32 == l;
//            each slice is a sequential fp32 FMA chain in increasing h from
//            +0.0f, and the 32 partial sums are combined by a xor butterfly
//            (off = 16..1).  Lane l owns slice l, so each warp load is 512
//            contiguous bytes.
//   E >  32: one sequential fp32 FMA chain over h = 0..H-1 from +0.0f.
#include "common.cuh"
#include "launch.h"

#include <climits>
#include <cstdlib>
#include <cstring>

namespace moe {

// Router status word: 4 when a staged-copy wait ran out (moe_device_status).
__device__ int32_t g_route_status;

cudaError_t read_route_status(int32_t* code, bool clear) {
    MOE_CUDA_TRY(cudaMemcpyFromSymbol(code, g_route_status, sizeof(int32_t)));
    if (clear) {
        const int32_t zero = 0;
        MOE_CUDA_TRY(cudaMemcpyToSymbol(g_route_status, &zero, sizeof(int32_t)));
    }
    return cudaSuccess;
}

namespace {

// Many experts (E > 32): TT-token x TE-expert tiles, (TT/MT)*(TE/ME) threads,
// an MT x ME register micro-tile per thread, hidden consumed in chunks of KC
// staged in two shared-memory buffers (the next chunk's global loads are in
// flight while the current one is used).  Every logit is still one sequential
// FMA chain in increasing h: the packed __ffma2_rn does two independent fp32
// FMAs (round to nearest, like fmaf), pairing neighbouring experts, so the
// tiling and pairing change no value.  The transposing stores into shared
// memory give consecutive lanes consecutive tokens (experts), so they are
// free of bank conflicts.
template <int TT, int TE, int MT, int ME>
struct TiledRouter {
    static constexpr int KC = 32;
    static constexpr int kThreads = (TT / MT) * (TE / ME);
    static constexpr int kTx = TE / ME;                    // threads along experts
    static constexpr int kXPieces = TT * (KC / 8) / kThreads;   // 16-byte x pieces per thread
    static constexpr int kWPieces = TE * (KC / 4) / kThreads;   // 16-byte w pieces per thread
    static constexpr int kSmemBytes = 2 * KC * (TT + TE) * 4;
    static_assert(kXPieces * kThreads == TT * (KC / 8), "x pieces split evenly");
    static_assert(kWPieces * kThreads == TE * (KC / 4), "w pieces split evenly");
    static_assert(MT % 4 == 0 && ME % 4 == 0, "float4 micro-tile loads");
};

// Inside a full chunk the next k-step's shared-memory operands are loaded
// before the current step's FMAs (two register sets), so the loads' latency
// hides behind the packed FMAs: 2-4 % faster than the plain loop at E = 64 and
// E = 256 (the kernel is latency-bound), same values.
template <int TT, int TE, int MT, int ME>
__global__ void __launch_bounds__(TiledRouter<TT, TE, MT, ME>::kThreads, 2)
router_logits_tiled_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
                           float* __restrict__ logits, int64_t tokens, int hidden, int experts) {
    using R = TiledRouter<TT, TE, MT, ME>;
    constexpr int KC = R::KC, NT = R::kThreads;
    extern __shared__ __align__(16) float router_smem[];
    float* xs = router_smem;                 // [2][KC][TT]
    float* ws = router_smem + 2 * KC * TT;   // [2][KC][TE]
    const int tid = threadIdx.x;
    const int tx = tid % R::kTx, ty = tid / R::kTx;
    const int64_t t0 = static_cast<int64_t>(blockIdx.x) * TT;
    const int e0 = blockIdx.y * TE;
    pdl_trigger();  // the top-k kernel may launch; it waits for these logits

    uint4 xr[R::kXPieces];
    float4 wr[R::kWPieces];
    auto load = [&](int h0) {
#pragma unroll
        for (int q = 0; q < R::kXPieces; ++q) {
            const int piece = tid + q * NT;
            const int row = piece % TT, part = piece / TT;
            const int64_t t = t0 + row;
            const int h = h0 + part * 8;
            xr[q] = make_uint4(0, 0, 0, 0);
            if (t < tokens && h < hidden) xr[q] = __ldg(reinterpret_cast<const uint4*>(x + t * hidden + h));
        }
#pragma unroll
        for (int q = 0; q < R::kWPieces; ++q) {
            const int piece = tid + q * NT;
            const int er = piece % TE, part = piece / TE;
            const int e = e0 + er;
            const int h = h0 + part * 4;
            wr[q] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (e < experts && h < hidden)
                wr[q] = __ldg(reinterpret_cast<const float4*>(w + static_cast<int64_t>(e) * hidden + h));
        }
    };
    auto store = [&](int buf) {
        float* xb = xs + buf * KC * TT;
        float* wb = ws + buf * KC * TE;
#pragma unroll
        for (int q = 0; q < R::kXPieces; ++q) {
            const int piece = tid + q * NT;
            const int row = piece % TT, part = piece / TT;
            const uint32_t words[4] = {xr[q].x, xr[q].y, xr[q].z, xr[q].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                xb[(part * 8 + 2 * j) * TT + row] = bf16_bits_to_f32(words[j] & 0xffffu);
                xb[(part * 8 + 2 * j + 1) * TT + row] = bf16_bits_to_f32(words[j] >> 16);
            }
        }
#pragma unroll
        for (int q = 0; q < R::kWPieces; ++q) {
            const int piece = tid + q * NT;
            const int er = piece % TE, part = piece / TE;
            wb[(part * 4 + 0) * TE + er] = wr[q].x;
            wb[(part * 4 + 1) * TE + er] = wr[q].y;
            wb[(part * 4 + 2) * TE + er] = wr[q].z;
            wb[(part * 4 + 3) * TE + er] = wr[q].w;
        }
    };

    // Thread (tx, ty) owns tokens ty*MH + i and TT/2 + ty*MH + i (i < MH), and
    // experts tx*NH + j and TE/2 + tx*NH + j (j < NH): each quarter-warp's
    // shared-memory reads of one half are contiguous, so they are free of bank
    // conflicts (a contiguous MT x ME block per thread strides them 2-way).
    constexpr int MH = MT / 2, NH = ME / 2;
    static_assert(MH == 4 && (NH == 4 || NH == 2), "micro-tile halves of 4 tokens, 2 or 4 experts");
    float2 acc[MT][NH];
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int j = 0; j < NH; ++j) acc[i][j] = make_float2(0.0f, 0.0f);

    auto operands = [&](const float* xk, const float* wk, float (&xv)[MT], float2 (&wv)[NH]) {
        const float4 x0 = *reinterpret_cast<const float4*>(xk + ty * MH);
        const float4 x1 = *reinterpret_cast<const float4*>(xk + TT / 2 + ty * MH);
        xv[0] = x0.x; xv[1] = x0.y; xv[2] = x0.z; xv[3] = x0.w;
        xv[4] = x1.x; xv[5] = x1.y; xv[6] = x1.z; xv[7] = x1.w;
        if constexpr (NH == 4) {
            const float4 w0 = *reinterpret_cast<const float4*>(wk + tx * NH);
            const float4 w1 = *reinterpret_cast<const float4*>(wk + TE / 2 + tx * NH);
            wv[0] = make_float2(w0.x, w0.y); wv[1] = make_float2(w0.z, w0.w);
            wv[2] = make_float2(w1.x, w1.y); wv[3] = make_float2(w1.z, w1.w);
        } else {
            wv[0] = *reinterpret_cast<const float2*>(wk + tx * NH);
            wv[1] = *reinterpret_cast<const float2*>(wk + TE / 2 + tx * NH);
        }
    };
    auto fmas = [&](const float (&xv)[MT], const float2 (&wv)[NH]) {
#pragma unroll
        for (int i = 0; i < MT; ++i) {
            const float2 xx = make_float2(xv[i], xv[i]);
#pragma unroll
            for (int j = 0; j < NH; ++j) acc[i][j] = __ffma2_rn(xx, wv[j], acc[i][j]);
        }
    };
    auto step = [&](const float* xk, const float* wk) {
        float xv[MT];
        float2 wv[NH];
        operands(xk, wk, xv, wv);
        fmas(xv, wv);
    };

    load(0);
    int buf = 0;
    for (int h0 = 0; h0 < hidden; h0 += KC) {
        store(buf);
        __syncthreads();
        if (h0 + KC < hidden) load(h0 + KC);
        const float* xb = xs + buf * KC * TT;
        const float* wb = ws + buf * KC * TE;
        const int steps = min(KC, hidden - h0);
        if (steps == KC) {
            float xa[MT], xn[MT];
            float2 wa[NH], wn[NH];
            operands(xb, wb, xa, wa);
#pragma unroll
            for (int k = 0; k < KC; k += 2) {
                operands(xb + (k + 1) * TT, wb + (k + 1) * TE, xn, wn);
                fmas(xa, wa);
                if (k + 2 < KC) operands(xb + (k + 2) * TT, wb + (k + 2) * TE, xa, wa);
                fmas(xn, wn);
            }
        } else {
            for (int k = 0; k < steps; ++k) step(xb + k * TT, wb + k * TE);
        }
        buf ^= 1;
    }
    const bool vector_ok = (experts % 2) == 0;
#pragma unroll
    for (int i = 0; i < MT; ++i) {
        const int64_t t = t0 + (i < MH ? ty * MH + i : TT / 2 + ty * MH + (i - MH));
        if (t >= tokens) continue;
        float* row = logits + t * experts;
#pragma unroll
        for (int j = 0; j < NH; ++j) {
            // pair j holds experts e, e + 1 of one half
            const int half = j / (NH / 2), jj = j % (NH / 2);
            const int e = e0 + half * (TE / 2) + tx * NH + 2 * jj;
            if (vector_ok && e + 2 <= experts) {
                *reinterpret_cast<float2*>(row + e) = acc[i][j];
            } else {
                if (e < experts) row[e] = acc[i][j].x;
                if (e + 1 < experts) row[e + 1] = acc[i][j].y;
            }
        }
    }
}

template <int TT, int TE, int MT, int ME>
cudaError_t launch_tiled(const __nv_bfloat16* x, const float* w, float* logits, int64_t tokens,
                         int hidden, int experts, cudaStream_t stream) {
    using R = TiledRouter<TT, TE, MT, ME>;
    static bool configured[64] = {};
    int device = 0;
    MOE_CUDA_TRY(cudaGetDevice(&device));
    if (!configured[device & 63]) {
        MOE_CUDA_TRY(cudaFuncSetAttribute(router_logits_tiled_kernel<TT, TE, MT, ME>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, R::kSmemBytes));
        configured[device & 63] = true;
    }
    dim3 grid(static_cast<unsigned>((tokens + TT - 1) / TT), static_cast<unsigned>((experts + TE - 1) / TE));
    router_logits_tiled_kernel<TT, TE, MT, ME><<<grid, R::kThreads, R::kSmemBytes, stream>>>(
        x, w, logits, tokens, hidden, experts);
    return cudaGetLastError();
}

// K rounds of warp argmax over one value per lane (lane = expert, E <= 32),
// ties to the lower index, then softmax over the selected values; lanes < K
// write (ids, weight) of the k-th choice.
__device__ __forceinline__ void warp_topk_one_per_lane(float v, bool avail, int lane, int topk,
                                                       int64_t out, int32_t* __restrict__ ids32,
                                                       int64_t* __restrict__ ids64,
                                                       float* __restrict__ weights) {
    float mine = 0.0f, first = 0.0f;
    int mine_id = 0;
    for (int k = 0; k < topk; ++k) {
        float bv = avail ? v : -INFINITY;
        int bi = avail ? lane : INT_MAX;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (bi == lane) avail = false;
        if (k == 0) first = bv;
        if (lane == k) {
            mine = bv;
            mine_id = bi;
        }
    }
    const float ex = lane < topk ? expf(mine - first) : 0.0f;
    float total = 0.0f;
    for (int k = 0; k < topk; ++k) total += __shfl_sync(0xffffffffu, ex, k);
    const float inv = 1.0f / total;
    if (lane < topk) {
        ids32[out + lane] = mine_id;
        if (ids64) ids64[out + lane] = mine_id;
        weights[out + lane] = ex * inv;
    }
}

// ---------------------------------------------------------- staged copies
// Bulk (non-tensor) async copies global -> shared completing on an mbarrier,
// and bounded mbarrier waits: a wait that takes kRouteWaitNs records status
// 4 in g_route_status and makes the CTA stop.
constexpr uint64_t kRouteWaitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void bar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void bar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void bar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool bar_try_wait(uint64_t* bar, uint32_t parity) {
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

__device__ __noinline__ bool bar_wait_slow(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    const uint64_t start = now_ns();
    for (uint32_t i = 1;; ++i) {
        if (bar_try_wait(bar, parity)) return true;
        if ((i & 31) == 0) {
            if (*abort_flag) return false;
            if (now_ns() - start > kRouteWaitNs) {
                atomicCAS(&g_route_status, 0, 4);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    return bar_try_wait(bar, parity) || bar_wait_slow(bar, parity, abort_flag);
}

__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Router for E <= 32, logits and top-k in one kernel.  A persistent CTA takes
// blocks of kWarps * TW tokens.  Warp kWarps issues bulk copies of each block's
// token rows and the router weights, 256 * JC hidden elements at a time, into
// a two-stage shared-memory ring; compute warp w owns TW tokens of the block.
// Lane l owns hidden slice l (8-element runs 256 apart) and keeps TW x EMAX
// partial sums (sequential FMA chains in increasing h); the xor butterfly
// leaves every logit in every lane, and lane e then holds expert e's biased
// score for the warp top-k.  The copies stream every token row from HBM once
// and put each weight chunk in shared memory once per block of tokens.
template <int EMAX, int TW, int JC, int STAGES>
struct StagedRouter {
    static constexpr int kWarps = 8;  // compute warps; one more issues the copies
    static constexpr int kThreads = 32 * (kWarps + 1);
    static constexpr int kBlockTokens = kWarps * TW;
    static constexpr int kChunk = 256 * JC;  // hidden elements per stage
    static constexpr int kXBytes = kBlockTokens * kChunk * 2;
    static constexpr int kWBytes = EMAX * kChunk * 4;
    static constexpr int kStageBytes = kXBytes + kWBytes;
    static constexpr int kStages = STAGES;
    static constexpr int kSmemBytes = kStages * kStageBytes + 2 * kStages * 8 + 16;
};

template <int EMAX, int TW, int JC, int STAGES>
__global__ void __launch_bounds__(StagedRouter<EMAX, TW, JC, STAGES>::kThreads, 1)
router_staged_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
                     const float* __restrict__ bias, float* __restrict__ logits,
                     int32_t* __restrict__ ids32, int64_t* __restrict__ ids64,
                     float* __restrict__ weights, int64_t tokens, int hidden, int experts,
                     int topk, int block_tokens) {
    // block_tokens (a multiple of TW, at most kBlockTokens): tokens per block,
    // so that small batches spread over every SM; warps past it idle through
    // the block (their results are not written).
    using R = StagedRouter<EMAX, TW, JC, STAGES>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + R::kStages * R::kStageBytes);
    uint64_t* empty = full + R::kStages;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + R::kStages);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int chunks = (hidden + R::kChunk - 1) / R::kChunk;
    const int64_t blocks = (tokens + block_tokens - 1) / block_tokens;
    pdl_trigger();  // the dispatch index kernel may launch; it waits for these ids
    if (threadIdx.x == 0) {
        for (int s = 0; s < R::kStages; ++s) {
            bar_init(&full[s], 1);
            bar_init(&empty[s], R::kWarps);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == R::kWarps) {
        if (lane != 0) return;
        // ---------------------------------------------------- copy issuer
        int stage = 0;
        uint32_t phase = 0, armed = 0, last_parity = 0;
        for (int64_t b = blockIdx.x; b < blocks && !*abort_flag; b += gridDim.x) {
            const int64_t t0 = b * block_tokens;
            const int nt = static_cast<int>(tokens - t0 < block_tokens ? tokens - t0 : block_tokens);
            for (int c = 0; c < chunks; ++c) {
                if (!bar_wait(&empty[stage], phase ^ 1u, abort_flag)) break;
                const int h0 = c * R::kChunk;
                const int len = hidden - h0 < R::kChunk ? hidden - h0 : R::kChunk;
                uint8_t* xs = smem + stage * R::kStageBytes;
                uint8_t* ws = xs + R::kXBytes;
                bar_expect_tx(&full[stage], static_cast<uint32_t>((nt * 2 + experts * 4) * len));
                for (int i = 0; i < nt; ++i)
                    bulk_copy(xs + i * R::kChunk * 2, x + (t0 + i) * hidden + h0, len * 2, &full[stage]);
                for (int e = 0; e < experts; ++e)
                    bulk_copy(ws + e * R::kChunk * 4, w + static_cast<int64_t>(e) * hidden + h0, len * 4,
                              &full[stage]);
                armed |= 1u << stage;
                last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
                if (++stage == R::kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
        if (*abort_flag) {
            // let the copies already issued land before the CTA's memory goes away
            volatile int never = 0;
            for (int s = 0; s < R::kStages; ++s)
                if (armed & (1u << s)) bar_wait(&full[s], (last_parity >> s) & 1u, &never);
        }
        return;
    }

    // -------------------------------------------------------- compute warps
    int stage = 0;
    uint32_t phase = 0;
    for (int64_t b = blockIdx.x; b < blocks; b += gridDim.x) {
        const int64_t t0 = b * block_tokens + warp * TW;
        // this block's tokens, and how many of them belong to this warp
        const int64_t block_end = (b + 1) * block_tokens < tokens ? (b + 1) * block_tokens : tokens;
        float acc[TW][EMAX];
#pragma unroll
        for (int i = 0; i < TW; ++i)
#pragma unroll
            for (int e = 0; e < EMAX; ++e) acc[i][e] = 0.0f;
        for (int c = 0; c < chunks; ++c) {
            if (!bar_wait(&full[stage], phase, abort_flag)) return;
            const uint8_t* xs = smem + stage * R::kStageBytes;
            const uint8_t* ws = xs + R::kXBytes;
            const int h0 = c * R::kChunk;
#pragma unroll
            for (int jj = 0; jj < JC; ++jj) {
                const int hl = 256 * jj + 8 * lane;
                if (h0 + hl >= hidden) break;
                float xv[TW][8];
#pragma unroll
                for (int i = 0; i < TW; ++i) {
                    uint4 raw = make_uint4(0, 0, 0, 0);
                    if (t0 + i < block_end)
                        raw = *reinterpret_cast<const uint4*>(xs + ((warp * TW + i) * R::kChunk + hl) * 2);
                    const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        xv[i][2 * q] = bf16_bits_to_f32(words[q] & 0xffffu);
                        xv[i][2 * q + 1] = bf16_bits_to_f32(words[q] >> 16);
                    }
                }
#pragma unroll
                for (int e = 0; e < EMAX; ++e) {
                    if (e >= experts) break;
                    const float4* wr = reinterpret_cast<const float4*>(ws + (e * R::kChunk + hl) * 4);
                    const float4 w0 = wr[0], w1 = wr[1];
                    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                    for (int i = 0; i < TW; ++i)
#pragma unroll
                        for (int j = 0; j < 8; ++j) acc[i][e] = fmaf(xv[i][j], wv[j], acc[i][e]);
                }
            }
            __syncwarp();
            if (lane == 0) bar_arrive(&empty[stage]);
            if (++stage == R::kStages) {
                stage = 0;
                phase ^= 1u;
            }
        }
#pragma unroll
        for (int i = 0; i < TW; ++i)
#pragma unroll
            for (int e = 0; e < EMAX; ++e)
#pragma unroll
                for (int off = 16; off > 0; off >>= 1)
                    acc[i][e] = acc[i][e] + __shfl_xor_sync(0xffffffffu, acc[i][e], off);
#pragma unroll
        for (int i = 0; i < TW; ++i) {
            const int64_t t = t0 + i;
            if (t >= block_end) break;  // uniform per warp
            float mine = 0.0f;
#pragma unroll
            for (int e = 0; e < EMAX; ++e)
                if (e == lane) mine = acc[i][e];
            const bool avail = lane < experts;
            if (avail && logits) logits[t * experts + lane] = mine;
            const float v = avail ? mine + (bias ? bias[lane] : 0.0f) : -INFINITY;
            warp_topk_one_per_lane(v, avail, lane, topk, t * topk, ids32, ids64, weights);
        }
    }
}

// One warp per token.  Lane l holds experts l, l+32, ... (VPL of them).  K
// rounds of warp argmax under the order (value desc, index asc); the winner is
// struck from its lane.  Softmax over the selected values: e_k = exp(v_k - v_0),
// summed in k order, multiplied by 1/sum (for K = 2 this is the reference's
// 1/(1+r), r/(1+r), dispatch.cu:366-374).
template <int VPL>
__global__ void __launch_bounds__(256)
topk_softmax_kernel(const float* __restrict__ logits, const float* __restrict__ bias,
                    int32_t* __restrict__ ids32, int64_t* __restrict__ ids64,
                    float* __restrict__ weights, int64_t tokens, int experts, int topk) {
    const int lane = threadIdx.x & 31;
    const int64_t token = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    pdl_trigger();
    pdl_wait();  // a dependent launch of the logits kernel
    if (token >= tokens) return;  // uniform per warp

    float v[VPL];
    bool avail[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int e = lane + 32 * i;
        avail[i] = e < experts;
        v[i] = avail[i] ? logits[token * experts + e] + (bias ? bias[e] : 0.0f) : -INFINITY;
    }
    float mine = 0.0f, first = 0.0f;
    int mine_id = 0;
    for (int k = 0; k < topk; ++k) {
        float bv = -INFINITY;
        int bi = INT_MAX;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            if (avail[i] && (bi == INT_MAX || v[i] > bv)) {
                bv = v[i];
                bi = lane + 32 * i;
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if ((bi & 31) == lane) {
#pragma unroll
            for (int i = 0; i < VPL; ++i)
                if (lane + 32 * i == bi) avail[i] = false;
        }
        if (k == 0) first = bv;
        if (lane == k) {
            mine = bv;
            mine_id = bi;
        }
    }
    const float ex = lane < topk ? expf(mine - first) : 0.0f;
    float total = 0.0f;
    for (int k = 0; k < topk; ++k) total += __shfl_sync(0xffffffffu, ex, k);
    const float inv = 1.0f / total;
    if (lane < topk) {
        const int64_t p = token * topk + lane;
        ids32[p] = mine_id;
        if (ids64) ids64[p] = mine_id;
        weights[p] = ex * inv;
    }
}

}  // namespace

cudaError_t launch_router_logits(const void* x, const float* w, float* logits, int64_t tokens,
                                 int64_t hidden, int experts, cudaStream_t stream) {
    if (tokens == 0) return cudaSuccess;
    const auto* xb = static_cast<const __nv_bfloat16*>(x);
    const int h = static_cast<int>(hidden);
    // Tile (tokens x experts) per CTA; MOE_B200_ROUTER_TILE overrides the
    // choice (a tuning knob: every tile gives the same bits).  Measured on B200
    // (L2 flushed before each launch), E=256, H=7168: 64x128 is the fastest at
    // 4096, 8192 and 32768 tokens (0.46, 0.83, 2.84 ms; 128x128 0.92, 0.93,
    // 3.13; 128x64 0.51, 0.98, 3.30; 64x64 0.55, 1.05, 3.56; 32x64 0.66, 1.28,
    // 4.33); E=64, H=2048, T=16384: 128x64 0.159 ms, 64x64 0.175, 32x64 0.204.
    const char* env = getenv("MOE_B200_ROUTER_TILE");
    const char* pick = env ? env : (experts <= 64 ? "128x64" : "64x128");
    if (strcmp(pick, "128x128") == 0) return launch_tiled<128, 128, 8, 8>(xb, w, logits, tokens, h, experts, stream);
    if (strcmp(pick, "64x128") == 0) return launch_tiled<64, 128, 8, 8>(xb, w, logits, tokens, h, experts, stream);
    if (strcmp(pick, "128x64") == 0) return launch_tiled<128, 64, 8, 4>(xb, w, logits, tokens, h, experts, stream);
    if (strcmp(pick, "32x64") == 0) return launch_tiled<32, 64, 8, 4>(xb, w, logits, tokens, h, experts, stream);
    return launch_tiled<64, 64, 8, 4>(xb, w, logits, tokens, h, experts, stream);
}

template <int EMAX, int TW, int JC, int STAGES>
static cudaError_t launch_staged(const void* x, const float* w, const float* bias, float* logits,
                                 int32_t* ids32, int64_t* ids64, float* weights, int64_t tokens,
                                 int64_t hidden, int experts, int topk, cudaStream_t stream) {
    using R = StagedRouter<EMAX, TW, JC, STAGES>;
    static int sms[64] = {};
    static bool configured[64] = {};
    int device = 0;
    MOE_CUDA_TRY(cudaGetDevice(&device));
    if (!configured[device & 63]) {
        MOE_CUDA_TRY(cudaFuncSetAttribute(router_staged_kernel<EMAX, TW, JC, STAGES>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, R::kSmemBytes));
        MOE_CUDA_TRY(cudaDeviceGetAttribute(&sms[device & 63], cudaDevAttrMultiProcessorCount, device));
        configured[device & 63] = true;
    }
    const int64_t sm = sms[device & 63];
    // Full blocks once there are at least as many as SMs; below that, fewer
    // tokens per block (a multiple of TW) so that every SM gets one.  At the
    // Mixtral shape (4096 tokens) that is 147 blocks of 28 instead of 128 of
    // 32: 20.9 against 22.8 us under ncu, equal (25.6 us) in an event loop.
    // Eight experts' weights loaded together with j-outer packed FMAs, and 16
    // warps of 2 tokens, were measured as well: no faster (26.6 and 31.7 us).
    int64_t block_tokens = R::kBlockTokens;
    if (tokens < sm * R::kBlockTokens) {
        block_tokens = ((tokens + sm - 1) / sm + TW - 1) / TW * TW;
        if (block_tokens < TW) block_tokens = TW;
    }
    const int64_t blocks = (tokens + block_tokens - 1) / block_tokens;
    const unsigned grid = static_cast<unsigned>(blocks < sm ? blocks : sm);
    router_staged_kernel<EMAX, TW, JC, STAGES><<<grid, R::kThreads, R::kSmemBytes, stream>>>(
        static_cast<const __nv_bfloat16*>(x), w, bias, logits, ids32, ids64, weights, tokens,
        static_cast<int>(hidden), experts, topk, static_cast<int>(block_tokens));
    return cudaGetLastError();
}

cudaError_t launch_route(const void* x, const float* w, const float* bias, float* logits,
                         int32_t* ids32, int64_t* ids64, float* weights, int64_t tokens,
                         int64_t hidden, int experts, int topk, cudaStream_t stream) {
    if (tokens == 0) return cudaSuccess;
    // Measured on B200 (Mixtral router, T=4096, H=4096, E=8): 1024-element
    // chunks in two stages 25.6 us; 512 in four 31.7 us; 256 in six 48.0 us.
    if (experts <= 8)
        return launch_staged<8, 4, 4, 2>(x, w, bias, logits, ids32, ids64, weights, tokens, hidden, experts, topk, stream);
    if (experts <= 16)
        return launch_staged<16, 2, 4, 2>(x, w, bias, logits, ids32, ids64, weights, tokens, hidden, experts, topk, stream);
    if (experts <= kRouterSlicedMaxExperts)
        return launch_staged<32, 2, 2, 2>(x, w, bias, logits, ids32, ids64, weights, tokens, hidden, experts, topk, stream);
    cudaError_t err = launch_router_logits(x, w, logits, tokens, hidden, experts, stream);
    if (err != cudaSuccess) return err;
    return launch_topk(logits, bias, ids32, ids64, weights, tokens, experts, topk, stream);
}

cudaError_t launch_topk(const float* logits, const float* bias, int32_t* ids32, int64_t* ids64,
                        float* weights, int64_t tokens, int experts, int topk, cudaStream_t stream) {
    if (tokens == 0) return cudaSuccess;
    const unsigned blocks = static_cast<unsigned>((tokens + 7) / 8);
    if (experts <= 32)
        return launch_dependent(topk_softmax_kernel<1>, dim3(blocks), dim3(256), 0, stream, logits, bias, ids32, ids64, weights, tokens, experts, topk);
    else if (experts <= 64)
        return launch_dependent(topk_softmax_kernel<2>, dim3(blocks), dim3(256), 0, stream, logits, bias, ids32, ids64, weights, tokens, experts, topk);
    else if (experts <= 128)
        return launch_dependent(topk_softmax_kernel<4>, dim3(blocks), dim3(256), 0, stream, logits, bias, ids32, ids64, weights, tokens, experts, topk);
    else
        return launch_dependent(topk_softmax_kernel<8>, dim3(blocks), dim3(256), 0, stream, logits, bias, ids32, ids64, weights, tokens, experts, topk);
}

}  // namespace moe
