// moe_dispatch_no_alloc: dispatch for callers that cannot allocate device memory.
//
// moe_dispatch needs a few KiB of device scratch (per-chunk expert counts and
// a completion ticket) that its caller allocates.  Some callers cannot:
// serving hosts that hand the library a fixed memory budget at start-up and
// forbid any allocation afterwards (so that memory use is known in advance
// and no allocation can fail or stall mid-request), and foreign-language
// bindings that receive only raw device pointers from their host and have no
// device allocator of their own.  This entry point takes the same inputs and
// outputs as moe_dispatch but keeps its scratch in a fixed array compiled
// into the library, so it allocates nothing.
//
// The array g_no_alloc_scratch lives in every GPU that loads the library, for
// as long as the library stays loaded.  Its capacity bounds the problem size:
// (tokens*topk / 1024 rounded up) * experts <= kNoAllocTableWords.
//
// Host code may not use the array's name as a device address (on the host it
// names a stand-in object).  The first call on each device looks its device
// address up with cudaGetSymbolAddress while that device is current and caches
// it; make that first call before any stream capture begins.
//
// Arguments are checked before the array is touched, so a rejected call has
// no effect on the device.  All calls share the one array and it keeps the
// previous call's contents: the completion ticket is cleared on the stream
// before every launch.  Calls whose work overlaps on the GPU (different
// streams, or different threads without ordering) race on the array;
// serialise them.
#include "../../../include/moe_b200.h"
#include "launch.h"

#include <cstdio>
#include <mutex>

namespace {

// 16 header words (ticket + pad) + the per-chunk table, as dispatch_scratch_bytes lays out.
constexpr int64_t kNoAllocHeaderWords = 16;
constexpr int64_t kNoAllocTableWords = 65536;  // e.g. 262144 assignments x 256 experts
constexpr int64_t kNoAllocWords = kNoAllocHeaderWords + kNoAllocTableWords;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) int32_t g_no_alloc_scratch[kNoAllocWords];

std::mutex g_setup_mutex;
int32_t* g_scratch_address[kMaxDevices] = {};

int scratch_address(int device, int32_t** out, const char** error) {
    if (device < 0 || device >= kMaxDevices) {
        *error = "device ordinal out of range for the no-alloc scratch table";
        return MOE_ERR_UNSUPPORTED;
    }
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_address[device]) {
        void* address = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&address, g_no_alloc_scratch);
        if (err != cudaSuccess) {
            *error = cudaGetErrorString(err);
            return MOE_ERR_CUDA;
        }
        g_scratch_address[device] = static_cast<int32_t*>(address);
    }
    *out = g_scratch_address[device];
    return MOE_OK;
}

int refuse(int status, const char* text) {
    moe::set_last_error(text);
    return status;
}

}  // namespace

extern "C" {

int moe_dispatch_no_alloc(const void* x, int32_t dtype, const int32_t* ids, int32_t* counts,
                          int32_t* offsets, int32_t* slots, void* packed, int32_t* inverse,
                          int64_t tokens, int64_t hidden, int32_t topk, int32_t experts,
                          int64_t packed_rows, int32_t alignment, int32_t vectorized,
                          void* stream) {
    // the size limit first (it needs only the shape), then moe_dispatch's own checks
    const int64_t needed_bytes = moe_dispatch_scratch_bytes(tokens, topk, experts);
    if (needed_bytes > kNoAllocWords * static_cast<int64_t>(sizeof(int32_t))) {
        char message[256];
        snprintf(message, sizeof(message),
                 "moe_dispatch_no_alloc: %lld assignments over %d experts need %lld scratch bytes; "
                 "the built-in array holds %lld (use moe_dispatch with caller scratch)",
                 static_cast<long long>(tokens * topk), experts,
                 static_cast<long long>(needed_bytes),
                 static_cast<long long>(kNoAllocWords * sizeof(int32_t)));
        return refuse(MOE_ERR_INVALID, message);
    }
    const int checked = moe::check_dispatch_args(x, dtype, ids, counts, offsets, slots, packed,
                                                 inverse, tokens, hidden, topk, experts,
                                                 packed_rows, alignment);
    if (checked != MOE_OK) return checked;
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return refuse(MOE_ERR_CUDA, "cudaGetDevice failed");
    int32_t* scratch = nullptr;
    const char* error = nullptr;
    const int status = scratch_address(device, &scratch, &error);
    if (status != MOE_OK) return refuse(status, error);
    // The ticket must start at zero; clear it on the caller's stream.
    if (cudaMemsetAsync(scratch, 0, kNoAllocHeaderWords * sizeof(int32_t),
                        static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return refuse(MOE_ERR_CUDA, "cudaMemsetAsync of the no-alloc ticket failed");
    return moe_dispatch(x, dtype, ids, counts, offsets, slots, packed, inverse, tokens, hidden,
                        topk, experts, packed_rows, alignment, vectorized, scratch,
                        kNoAllocWords * static_cast<int64_t>(sizeof(int32_t)), stream);
}

}  // extern "C"
