// fry_heads_noalloc: the heads (fry_heads) for callers that cannot allocate device memory.
//
// Some callers of this library cannot call cudaMalloc at the moment they evaluate positions: a search thread in the
// middle of a stream capture (cudaMalloc is not allowed while a stream captures), a latency-bound loop that must not
// risk the device-wide synchronisation an allocation can trigger while other lanes run, or a host in another language
// (such as the Rust search loop) that has no device allocator of its own. This entry point takes only the inputs and the
// outputs: its scratch is the file-scope array below, which every GPU that loads the library holds from load to exit.
//
// Limits: at most FRY_HEADS_NOALLOC_MAX_BOARDS boards of d_model up to FRY_HEADS_NOALLOC_MAX_D_MODEL a call; larger
// calls are refused before anything is enqueued. Every call on a device shares the one array and it keeps the last
// call's contents: calls whose work overlaps on the GPU (two streams, or two threads on one device) race on it and must
// be ordered by the caller. Nothing in the array needs to start at zero: each region (the normed stream, the a matmul,
// the narrow outputs, the eval head's units and logits) is written in full by the call before the call reads it.
//
// Set-up: the first call on each device looks up the array's device address (cudaGetSymbolAddress, with that device
// current) and keeps it for the device's context; make that first call on a device before any stream capture on it.
#include <map>
#include <mutex>
#include <string>
#include <utility>

#include "../../include/fry_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace fry {

constexpr int kNoAllocMaxBoards = FRY_HEADS_NOALLOC_MAX_BOARDS;
constexpr int kNoAllocMaxWidth = FRY_HEADS_NOALLOC_MAX_D_MODEL;

// heads_workspace_bytes(kNoAllocMaxBoards, kNoAllocMaxWidth), as a constant
constexpr size_t kHeadsScratchBytes = heads_workspace_bytes_of(kNoAllocMaxBoards, kNoAllocMaxWidth);

static __device__ __align__(256) uint8_t g_heads_scratch[kHeadsScratchBytes];

namespace {

// The id of the calling thread's current context (cuCtxGetId, unique over the process's life), or 0 when none is current
// yet or the driver lacks the call. The driver's functions come through the runtime, as the library links no libcuda.
unsigned long long current_context_id() {
    using GetCurrent = CUresult (*)(CUcontext*);
    using GetId = CUresult (*)(CUcontext, unsigned long long*);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* symbol = nullptr;
        cudaDriverEntryPointQueryResult found;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &symbol, cudaEnableDefault, &found) == cudaSuccess && found == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(symbol);
        if (cudaGetDriverEntryPoint("cuCtxGetId", &symbol, cudaEnableDefault, &found) == cudaSuccess && found == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(symbol);
    });
    CUcontext context = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&context) != CUDA_SUCCESS || !context || get_id(context, &id) != CUDA_SUCCESS) return 0;
    return id;
}

// The array's device address in the current device's context. In host code g_heads_scratch is only a host-side
// stand-in for the symbol, never a device address, so the address is looked up with the device current, once per
// context: a device reset (cudaDeviceReset) ends the context and reloads the library's module, and the next call looks
// the address up anew in the new context.
cudaError_t heads_scratch(void** address) {
    static std::mutex mutex;
    static std::map<std::pair<int, unsigned long long>, void*> found;
    int device = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status != cudaSuccess) return status;
    std::lock_guard<std::mutex> lock(mutex);
    unsigned long long context = current_context_id();
    if (context != 0) {
        auto known = found.find({device, context});
        if (known != found.end()) {
            *address = known->second;
            return cudaSuccess;
        }
    }
    void* pointer = nullptr;
    status = cudaGetSymbolAddress(&pointer, g_heads_scratch);
    if (status != cudaSuccess) return status;
    context = current_context_id();  // the lookup made the device's context current if none was
    if (context != 0) found[{device, context}] = pointer;
    *address = pointer;
    return cudaSuccess;
}

}  // namespace
}  // namespace fry

// fail() and check() are abi.cu's: this file is compiled in the same translation unit (fry_b200.cu includes it after
// abi.cu), so the message lands where fry_last_error() reads it.

extern "C" int fry_heads_noalloc(const uint16_t* stream_x, const FryHeads* heads, float eps, float* rows, int B, int D, void* stream) {
    if (!heads || B < 0) return fail(FRY_ERROR_SHAPE, "fry_heads_noalloc needs its weights and B >= 0");
    if (D < 16 || D % 16 != 0) return fail(FRY_ERROR_SHAPE, "fry_heads_noalloc takes d_model a multiple of 16 from 16, got " + std::to_string(D));
    if (B > fry::kNoAllocMaxBoards || D > fry::kNoAllocMaxWidth)
        return fail(FRY_ERROR_SHAPE, "fry_heads_noalloc takes at most " + std::to_string(fry::kNoAllocMaxBoards) + " boards of d_model up to " +
                                         std::to_string(fry::kNoAllocMaxWidth) + " (its scratch is a fixed device array); got " +
                                         std::to_string(B) + " boards of " + std::to_string(D) + ": call fry_heads with a workspace instead");
    if (B == 0) return check(cudaSuccess, "");
    if ((reinterpret_cast<uintptr_t>(stream_x) & 15u) || (reinterpret_cast<uintptr_t>(heads->a_weight) & 15u) ||
        (reinterpret_cast<uintptr_t>(heads->ln_gain) & 15u))
        return fail(FRY_ERROR_SHAPE, "fry_heads_noalloc needs 16-byte aligned tensors");
    void* scratch = nullptr;
    cudaError_t status = fry::heads_scratch(&scratch);
    if (status != cudaSuccess) return check(status, "fry_heads_noalloc: cudaGetSymbolAddress");
    fry::HeadWeights w{heads->ln_gain,       heads->a_weight,    heads->a_bias,     heads->narrow_weight, heads->narrow_bias,
                       heads->hidden_weight, heads->hidden_bias, heads->out_weight, heads->out_bias,      heads->bins};
    std::string detail;
    return check(fry::heads(stream_x, w, eps, rows, scratch, fry::kHeadsScratchBytes, B, D, static_cast<cudaStream_t>(stream), &detail),
                 "fry_heads_noalloc", detail);
}
