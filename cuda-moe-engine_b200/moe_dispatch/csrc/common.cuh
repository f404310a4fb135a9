// Shared device helpers for the MoE kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace moe {

enum Dtype : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

inline int dtype_bytes(int dtype) { return dtype == kF32 ? 4 : 2; }

// Element conversions: fp32 math, one round-to-nearest-even cast on store.
template <int DT> struct Elem;
template <> struct Elem<kF32> {
    using T = float;
    static __device__ __forceinline__ float load(T v) { return v; }
    static __device__ __forceinline__ T store(float v) { return v; }
};
template <> struct Elem<kF16> {
    using T = __half;
    static __device__ __forceinline__ float load(T v) { return __half2float(v); }
    static __device__ __forceinline__ T store(float v) { return __float2half_rn(v); }
};
template <> struct Elem<kBF16> {
    using T = __nv_bfloat16;
    static __device__ __forceinline__ float load(T v) { return __bfloat162float(v); }
    static __device__ __forceinline__ T store(float v) { return __float2bfloat16_rn(v); }
};

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t bits16) {
    return __uint_as_float(bits16 << 16);
}

// Round-to-nearest-even fp32 -> bf16 bits (finite inputs; NaN stays NaN).
__device__ __forceinline__ uint32_t f32_to_bf16_bits(float f) {
    return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(f)));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    return f32_to_bf16_bits(lo) | (f32_to_bf16_bits(hi) << 16);
}

// Programmatic dependent launch.  A kernel launched with launch_dependent may
// start while the kernel before it on the stream is still running; before it
// reads or writes anything that kernel (or work before it) touches, it
// executes pdl_wait(), which returns once that kernel has completed and its
// memory is visible.  pdl_trigger() lets the next dependent launch start early
// (it then waits in its own pdl_wait).  Both are no-ops without a dependent
// launch.  The block's kernels form one chain (router -> index -> pack ->
// gate/up -> down -> combine), so each launch and prologue overlaps the
// previous kernel's last wave instead of following it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... Params, typename... Args>
inline cudaError_t launch_dependent(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                                    cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t config = {};
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    config.attrs = attribute;
    config.numAttrs = 1;
    return cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...);
}

// Plain CUDA error wrapper for host launchers.
#define MOE_CUDA_TRY(expr)                                  \
    do {                                                    \
        cudaError_t moe_err_ = (expr);                      \
        if (moe_err_ != cudaSuccess) return moe_err_;       \
    } while (0)

}  // namespace moe
