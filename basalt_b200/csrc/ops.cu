// Op-level entry points on caller-owned device buffers.
//
// bst_matmul is Tensor.matMul (torch/Tensor.java:214-227) -> gemm::matmul (native/src/gemm.rs:42-74)
// on the GPU: C[m, n] = A[m, k] * B[k, n], row-major, C overwritten. It runs the same kernels as the
// decode engine's projections: the small-M GEMV for m <= 8, otherwise operand split + the tcgen05
// GEMM (3xTF32). Its temporaries (B transposed to K-major and the tf32 split planes) come from the
// stream-ordered allocator and are released before the call returns.

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <string>

#include "basalt_cuda.h"
#include "kernels.h"

namespace bst {
namespace {

// B [k, n] row-major -> Bt [n, k] (K-major), optionally split into tf32 hi / fp32 remainder.
__global__ void k_transpose_split(const float* __restrict__ b, int k, int n,
                                  float* __restrict__ bt, float* __restrict__ hi,
                                  float* __restrict__ lo) {
    __shared__ float tile[32][33];
    const int k0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int kk = k0 + r, nn = n0 + threadIdx.x;
        tile[r][threadIdx.x] = (kk < k && nn < n) ? b[static_cast<size_t>(kk) * n + nn] : 0.0f;
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int nn = n0 + r, kk = k0 + threadIdx.x;
        if (nn < n && kk < k) {
            const float v = tile[threadIdx.x][r];
            const size_t at = static_cast<size_t>(nn) * k + kk;
            if (bt) bt[at] = v;
            if (hi) {
                const float h = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
                hi[at] = h;
                lo[at] = __fsub_rn(v, h);
            }
        }
    }
}

}  // namespace

namespace {
// Partial-product bytes the split-K plan of this shape needs (0 when it does not split).
size_t split_part_bytes(int64_t m, int64_t k, int64_t n) {
    return tc_part_bytes(static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), 0);
}
}  // namespace

// Scratch of a matmul without its split-K partials: the error word and the operand planes (or the
// transposed B of the GEMV path). The split-K partials come on top, as much room as is left.
size_t matmul_fixed_scratch_bytes(int64_t m, int64_t k, int64_t n) {
    auto up = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
    if (tc_usable(static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), 0)) {
        return up(sizeof(int)) + 2 * up(static_cast<size_t>(m) * k * 4) +
               2 * up(static_cast<size_t>(n) * k * 4);
    }
    return up(sizeof(int)) + up(static_cast<size_t>(n) * k * 4);
}

size_t matmul_scratch_bytes(int64_t m, int64_t k, int64_t n) {
    auto up = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
    const bool tc = tc_usable(static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), 0);
    return matmul_fixed_scratch_bytes(m, k, n) + (tc ? up(split_part_bytes(m, k, n)) : 0);
}

// Runs C = A * B with `scratch` (scratch_bytes of room, at least matmul_fixed_scratch_bytes,
// 256-byte aligned) as the only device memory beyond A, B and C. The K split is planned for the
// room left after the operand planes (fewer splits, or none, when it is short). Synchronises the
// stream to report pipeline errors.
int32_t matmul_with_scratch(cudaStream_t s, const float* a, const float* b, float* c, int64_t m,
                            int64_t k, int64_t n, void* scratch, size_t scratch_bytes,
                            std::string* error) {
    auto up = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
    char* p = static_cast<char*>(scratch);
    int* err = reinterpret_cast<int*>(p);
    p += up(sizeof(int));
    cudaError_t e = cudaMemsetAsync(err, 0, sizeof(int), s);
    const int M = static_cast<int>(m), K = static_cast<int>(k), N = static_cast<int>(n);
    EpiArgs ea;
    ea.out = c;
    ea.ldo = N;
    const dim3 tgrid((N + 31) / 32, (K + 31) / 32), tblock(32, 8);
    if (!e && tc_usable(M, N, K, 0)) {
        float* ah = reinterpret_cast<float*>(p);
        p += up(static_cast<size_t>(m) * k * 4);
        float* al = reinterpret_cast<float*>(p);
        p += up(static_cast<size_t>(m) * k * 4);
        float* bh = reinterpret_cast<float*>(p);
        p += up(static_cast<size_t>(n) * k * 4);
        float* bl = reinterpret_cast<float*>(p);
        p += up(static_cast<size_t>(n) * k * 4);
        float* part = reinterpret_cast<float*>(p);
        const size_t used = static_cast<size_t>(p - static_cast<char*>(scratch));
        const size_t part_bytes =
            std::min(split_part_bytes(m, k, n), scratch_bytes > used ? scratch_bytes - used : 0);
        if (!e) {
            k_transpose_split<<<tgrid, tblock, 0, s>>>(b, K, N, nullptr, bh, bl);
            e = cudaGetLastError();
        }
        if (!e) e = launch_split_operand(s, a, K, M, K, 0, ah, al);
        if (!e) {
            e = launch_gemm_tc(s, ah, al, bh, bl, 0, nullptr, M, N, K, Epi::kStore, ea, err,
                               part_bytes ? part : nullptr, part_bytes);
        }
    } else if (!e) {
        float* bt = reinterpret_cast<float*>(p);
        k_transpose_split<<<tgrid, tblock, 0, s>>>(b, K, N, bt, nullptr, nullptr);
        e = cudaGetLastError();
        if (!e) e = launch_linear(s, a, K, bt, 0, nullptr, M, N, K, Epi::kStore, ea);
    }
    int flag = 0;
    if (!e) e = cudaMemcpyAsync(&flag, err, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (!e) e = cudaStreamSynchronize(s);
    if (e) {
        *error = std::string("matmul: ") + cudaGetErrorName(e) + ": " + cudaGetErrorString(e);
        cudaGetLastError();
        return e == cudaErrorMemoryAllocation ? BST_OOM : BST_PANIC;
    }
    if (flag) {
        *error = "matmul: a tensor-core pipeline wait timed out (stage " + std::to_string(flag) + ")";
        return BST_PANIC;
    }
    return BST_OK;
}

int32_t check_matmul_args(const float* a, const float* b, float* c, int64_t m, int64_t k,
                          int64_t n, std::string* error) {
    if (!a || !b || !c) {
        *error = "matmul: a, b and c must be device pointers";
        return BST_INVALID;
    }
    if (m < 0 || k < 0 || n < 0 || m > (1 << 30) || k > (1 << 30) || n > (1 << 30)) {
        *error = "matmul: dimensions must be non-negative and below 2^30";
        return BST_SHAPE;
    }
    return BST_OK;
}

}  // namespace bst

extern "C" int32_t bst_matmul(int32_t device, void* stream, const float* a, const float* b,
                              float* c, int64_t m, int64_t k, int64_t n) {
    using namespace bst;
    std::string error;
    int32_t st = check_matmul_args(a, b, c, m, k, n, &error);
    if (st) {
        set_thread_error(error);
        return st;
    }
    cudaError_t e = cudaSetDevice(device);
    if (e) {
        cudaGetLastError();
        set_thread_error(std::string("matmul: device ") + std::to_string(device) + ": " +
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
    if ((e = configure_device_kernels_once(device)) != cudaSuccess) {
        set_thread_error(std::string("matmul: ") + cudaGetErrorString(e));
        return BST_PANIC;
    }
    void* scratch = nullptr;
    const size_t scratch_bytes = matmul_scratch_bytes(m, k, n);
    e = cudaMallocAsync(&scratch, scratch_bytes, s);
    if (e) {
        cudaGetLastError();
        set_thread_error(std::string("matmul: cannot allocate scratch: ") + cudaGetErrorString(e));
        return BST_OOM;
    }
    st = matmul_with_scratch(s, a, b, c, m, k, n, scratch, scratch_bytes, &error);
    cudaFreeAsync(scratch, s);
    cudaStreamSynchronize(s);
    if (st) set_thread_error(error);
    return st;
}

