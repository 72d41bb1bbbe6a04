// dsa_forward_noalloc: the whole forward with its workspace in a fixed,
// library-owned device array instead of caller-provided memory.
//
// Who needs it: callers that cannot call cudaMalloc (or any allocator) at the
// point where they run the forward, for example code running under a
// framework that owns all device memory through its own pool and forbids
// raw allocations, or plugin hosts that only hand out input and output
// buffers.  dsa_forward needs a workspace for the score matrix and the
// kept-index lists; this entry point takes it from kScratchBytes of static
// device memory that every GPU loading the library reserves until exit.
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace dsa {
namespace {

constexpr size_t kScratchBytes = size_t(32) << 20;  // 32 MiB per device

// The workspace.  Host code must not use this name as a device address: the
// address comes from cudaGetSymbolAddress, once per device.
static __device__ __align__(256) unsigned char g_forward_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};
CUcontext g_scratch_ctx[kMaxDevices] = {};

// The calling thread's current driver context (the device's primary context
// under the runtime API), looked up through the runtime so the library needs
// no link against libcuda.  nullptr if unavailable.
CUcontext current_context() {
    using Fn = CUresult (*)(CUcontext*);
    static Fn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<Fn>(f);
        return static_cast<Fn>(nullptr);
    }();
    CUcontext c = nullptr;
    if (!fn || fn(&c) != CUDA_SUCCESS) return nullptr;
    return c;
}

// Device address of the scratch array on the current device, looked up on the
// first call for that device and again whenever the device's context changed
// (after a cudaDeviceReset the array lives at a new address).  Returns nullptr
// and sets the error on failure.
void* scratch_for_current_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        fail(DSA_ERR_CUDA, "dsa_forward_noalloc: no usable current device");
        return nullptr;
    }
    const CUcontext ctx = current_context();   // nullptr before the runtime made one current
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_ptr[dev] || !ctx || ctx != g_scratch_ctx[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_forward_scratch);
        if (e != cudaSuccess || !p) {
            fail(DSA_ERR_CUDA, std::string("dsa_forward_noalloc: cudaGetSymbolAddress failed: ") +
                                   cudaGetErrorString(e));
            return nullptr;
        }
        g_scratch_ptr[dev] = p;
        g_scratch_ctx[dev] = current_context();
    }
    return g_scratch_ptr[dev];
}

}  // namespace
}  // namespace dsa

using namespace dsa;

extern "C" {

int dsa_forward_noalloc(const void* q_idx, const void* k_idx, const float* w_idx, const void* Q,
                        const void* K, const void* V, float* O, int64_t B, int64_t T_q,
                        int64_t T_k, int64_t q_row0, int64_t HI, int64_t DI, int64_t HQ,
                        int64_t DQ, int64_t DV, int64_t top_k, int idx_dtype, int qkv_dtype,
                        void* stream) {
    clear_error();
    if (top_k < 1 || B < 0 || T_q < 0 || T_k < 1)
        return fail(DSA_ERR_INVALID, "dsa_forward_noalloc: bad sizes");
    // an empty call computes nothing (as dsa_forward); the arguments are still checked there
    if (B * T_q == 0)
        return dsa_forward(q_idx, k_idx, w_idx, Q, K, V, O, B, T_q, T_k, q_row0, HI, DI, HQ, DQ, DV,
                           top_k, idx_dtype, qkv_dtype, nullptr, 0, stream);
    const size_t need = dsa_forward_workspace_bytes(B, T_q, T_k, top_k);
    if (need == 0) return fail(DSA_ERR_INVALID, "dsa_forward_noalloc: bad sizes");
    if (need > kScratchBytes)
        return fail(DSA_ERR_INVALID, "dsa_forward_noalloc: this shape needs " + std::to_string(need) +
                                         " bytes of workspace; the built-in scratch holds " +
                                         std::to_string(kScratchBytes) +
                                         " (use dsa_forward with your own workspace)");
    void* ws = scratch_for_current_device();
    if (!ws) return DSA_ERR_CUDA;
    // Every stage overwrites the parts of the workspace it later reads, so
    // nothing has to be cleared between calls.
    return dsa_forward(q_idx, k_idx, w_idx, Q, K, V, O, B, T_q, T_k, q_row0, HI, DI, HQ, DQ, DV,
                       top_k, idx_dtype, qkv_dtype, ws, kScratchBytes, stream);
}

}  // extern "C"
