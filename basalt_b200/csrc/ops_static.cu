// bst_matmul_static: bst_matmul without any device allocation.
//
// Some callers cannot call cudaMalloc while they run: a host runtime that has already carved the
// GPU's memory into its own pool (a JVM process whose device memory belongs to another framework's
// caching allocator, where a stray cudaMalloc can fail or fragment the pool), a process that must
// stay inside a fixed device-memory budget fixed at start-up, or a latency-critical thread for which
// cudaMalloc/cudaFree are off limits because they can synchronise the whole device. For them this
// entry point takes its temporaries from a fixed scratch array that is part of the library image:
// the caller passes A, B and C as for bst_matmul, and nothing is allocated per call.
//
// The scratch is a file-scope __device__ array of kStaticScratchBytes. Every GPU that loads the
// library holds one copy of it until the process exits. In host code the array's name is only a
// host-side stand-in for the device symbol, not a device address: handing it to a kernel would
// fault or, where the GPU can reach host memory, silently use the wrong memory. So the first call
// on each device (with that device current) looks up the array's device address with
// cudaGetSymbolAddress, checks the result, and caches it; later calls reuse that address. Make the
// first call on a device before any stream capture. A device reset (cudaDeviceReset, or a reset of
// the primary context) unloads the module and invalidates the cached address: after one, the
// process must not call this entry point again on that device.
//
// All calls share the one array and it keeps whatever the last call left in it; the part that must
// start at zero (the pipeline error word) is cleared by every call.
// Calls whose work overlaps on the GPU (different streams, or different host threads on the same
// device) race on the scratch and must be serialised by the caller.

#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "basalt_cuda.h"
#include "kernels.h"

namespace bst {
size_t matmul_fixed_scratch_bytes(int64_t m, int64_t k, int64_t n);
int32_t matmul_with_scratch(cudaStream_t s, const float* a, const float* b, float* c, int64_t m,
                            int64_t k, int64_t n, void* scratch, size_t scratch_bytes,
                            std::string* error);
int32_t check_matmul_args(const float* a, const float* b, float* c, int64_t m, int64_t k,
                          int64_t n, std::string* error);
}  // namespace bst

namespace {

constexpr size_t kStaticScratchBytes = 16u << 20;  // 16 MiB per device
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_matmul_scratch[kStaticScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_address[kMaxDevices] = {};

// Device address of g_matmul_scratch on `device` (current), looked up once per device.
cudaError_t scratch_address(int device, void** out) {
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_address[device]) {
        void* ptr = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&ptr, g_matmul_scratch);
        if (err != cudaSuccess) return err;
        g_scratch_address[device] = ptr;
    }
    *out = g_scratch_address[device];
    return cudaSuccess;
}

}  // namespace

extern "C" int32_t bst_matmul_static(int32_t device, void* stream, const float* a,
                                     const float* b, float* c, int64_t m, int64_t k, int64_t n) {
    using namespace bst;
    std::string error;
    int32_t st = check_matmul_args(a, b, c, m, k, n, &error);
    if (st) {
        set_thread_error(error);
        return st;
    }
    if (device < 0 || device >= kMaxDevices) {
        set_thread_error("matmul_static: device " + std::to_string(device) + " is out of range");
        return BST_INVALID;
    }
    // The operand planes must fit; the split-K partials take what room is left (fewer K splits,
    // or none, when it is short).
    const size_t need = matmul_fixed_scratch_bytes(m, k, n);
    if (k > 0 && need > kStaticScratchBytes) {
        set_thread_error("matmul_static: " + std::to_string(m) + "x" + std::to_string(k) + "x" +
                         std::to_string(n) + " needs " + std::to_string(need) +
                         " bytes of scratch; the static scratch holds " +
                         std::to_string(kStaticScratchBytes) + " bytes (use bst_matmul)");
        return BST_SHAPE;
    }
    cudaError_t e = cudaSetDevice(device);
    if (e) {
        cudaGetLastError();
        set_thread_error("matmul_static: device " + std::to_string(device) + ": " +
                         cudaGetErrorString(e));
        return BST_UNSUPPORTED;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (m == 0 || n == 0) return BST_OK;
    if (k == 0) {
        e = cudaMemsetAsync(c, 0, sizeof(float) * static_cast<size_t>(m) * n, s);
        if (!e) e = cudaStreamSynchronize(s);
        return e ? BST_PANIC : BST_OK;
    }
    void* scratch = nullptr;
    if ((e = scratch_address(device, &scratch)) != cudaSuccess) {
        cudaGetLastError();
        set_thread_error(std::string("matmul_static: cannot resolve the scratch array: ") +
                         cudaGetErrorString(e));
        return BST_PANIC;
    }
    if ((e = configure_device_kernels_once(device)) != cudaSuccess) {
        set_thread_error(std::string("matmul_static: ") + cudaGetErrorString(e));
        return BST_PANIC;
    }
    st = matmul_with_scratch(s, a, b, c, m, k, n, scratch, kStaticScratchBytes, &error);
    if (st) set_thread_error(error);
    return st;
}
