// e4m3 quantisation of bf16 rows, for the FP8 expert path (no counterpart in
// the reference, whose experts are bf16 only: src/moe_dispatch/layer.py:97-98).
//
// Every row gets its own scale (a token's row of activations, or one output
// channel of an expert's weights):
//   amax = max_c |x[r,c]|,  scale[r] = amax / 448,
//   q[r,c] = e4m3(x[r,c] * (448 / amax))   round to nearest even, saturating at 448,
// so x[r,c] ~ q[r,c] * scale[r].  An all-zero row gets scale 1 and zeros.
// The grouped GEMM multiplies e4m3 by e4m3 exactly and accumulates in fp32,
// then dequantises with the two scales (gemm_sm100.cu).
#include "common.cuh"
#include "launch.h"

#include <cuda_fp8.h>

namespace moe {
namespace {

constexpr int kQuantThreads = 256;
constexpr int kQuantHeld = 4;  // 16-byte vectors a thread keeps between the two passes

__device__ __forceinline__ float block_max(float v, float* shared) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    if (lane == 0) shared[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < kQuantThreads / 32 ? shared[lane] : 0.0f;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
        if (lane == 0) shared[0] = v;
    }
    __syncthreads();
    return shared[0];
}

// Eight bf16 values (one 16-byte vector) -> eight e4m3 bytes.
__device__ __forceinline__ uint2 quantize8(uint4 v, float inv) {
    const uint32_t words[4] = {v.x, v.y, v.z, v.w};
    uint32_t out[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        uint32_t packed = 0;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint32_t w = words[2 * h + j];
            const float2 f = make_float2(bf16_bits_to_f32(w & 0xffffu) * inv, bf16_bits_to_f32(w >> 16) * inv);
            const __nv_fp8x2_storage_t q = __nv_cvt_float2_to_fp8x2(f, __NV_SATFINITE, __NV_E4M3);
            packed |= static_cast<uint32_t>(q) << (16 * j);
        }
        out[h] = packed;
    }
    return make_uint2(out[0], out[1]);
}

// One CTA per row (grid-stride over rows); cols is a multiple of 8.
__global__ void __launch_bounds__(kQuantThreads)
quantize_rows_e4m3_kernel(const uint4* __restrict__ x, uint2* __restrict__ q, float* __restrict__ scale,
                          int64_t rows, int64_t vecs) {
    __shared__ float reduce[kQuantThreads / 32];
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const uint4* row = x + r * vecs;
        uint4 held[kQuantHeld];
        float amax = 0.0f;
#pragma unroll
        for (int u = 0; u < kQuantHeld; ++u) {
            const int64_t c = threadIdx.x + static_cast<int64_t>(u) * kQuantThreads;
            held[u] = c < vecs ? __ldg(row + c) : make_uint4(0, 0, 0, 0);
        }
        auto absmax8 = [&](uint4 v) {
            const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; ++j)
                amax = fmaxf(amax, fmaxf(fabsf(bf16_bits_to_f32(words[j] & 0xffffu)),
                                         fabsf(bf16_bits_to_f32(words[j] >> 16))));
        };
#pragma unroll
        for (int u = 0; u < kQuantHeld; ++u) absmax8(held[u]);  // zeros past the row's end
        for (int64_t c = threadIdx.x + kQuantHeld * kQuantThreads; c < vecs; c += kQuantThreads)
            absmax8(__ldg(row + c));
        amax = block_max(amax, reduce);
        const float inv = amax > 0.0f ? 448.0f / amax : 0.0f;
        if (threadIdx.x == 0) scale[r] = amax > 0.0f ? amax / 448.0f : 1.0f;
#pragma unroll
        for (int u = 0; u < kQuantHeld; ++u) {
            const int64_t c = threadIdx.x + static_cast<int64_t>(u) * kQuantThreads;
            if (c < vecs) q[r * vecs + c] = quantize8(held[u], inv);
        }
        for (int64_t c = threadIdx.x + kQuantHeld * kQuantThreads; c < vecs; c += kQuantThreads)
            q[r * vecs + c] = quantize8(__ldg(row + c), inv);
        __syncthreads();  // `reduce` is reused by the next row
    }
}

}  // namespace

cudaError_t launch_quantize_rows_e4m3(const void* x, void* q, float* scale, int64_t rows,
                                      int64_t cols, cudaStream_t stream) {
    if (rows == 0) return cudaSuccess;
    const int64_t grid = rows < 148 * 8 ? rows : 148 * 8;
    quantize_rows_e4m3_kernel<<<static_cast<unsigned>(grid), kQuantThreads, 0, stream>>>(
        static_cast<const uint4*>(x), static_cast<uint2*>(q), scale, rows, cols / 8);
    return cudaGetLastError();
}

}  // namespace moe
