// Tensor-core projections for M > 8 rows on sm_100a: tcgen05.mma with accumulators in TMEM,
// operands staged in shared memory by TMA (cp.async.bulk.tensor, one CTA per copy).
//
// Y[M, N] = X[M, K] * W[N, K]^T + bias, epilogue fused (see Epi).
//
// Precision. TextEngine's reference computes in fp32, so the operands are split so that the
// tensor cores reproduce fp32 products to ~2^-21 (tf32) or ~2^-16 (bf16 weights):
//   * fp32 weights: 3xTF32. W = Wh + Wl with Wh the tf32 truncation of W (split once on upload),
//     X = Xh + Xl likewise (split per call); Y = Xh*Wh + Xh*Wl + Xl*Wh, fp32 accumulation.
//   * bf16 weights: X = Xh + Xl as two bf16 planes; Y = Xh*W + Xl*W (kind::f16, bf16 inputs).
//
// Tile: 128 x BN output per CTA (BN = 64 or 128), K staged in 128-byte rows (32 fp32 / 64 bf16)
// with the 128-byte swizzle. Warp 0 issues TMA, warp 1 owns TMEM and issues the MMAs, warps 2-5
// drain TMEM (each warp reads its 32-lane quarter) and apply the epilogue. Every mbarrier wait is
// bounded in time; on expiry the kernel records an error code, drains its own copies and returns.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "device.cuh"
#include "epilogue.cuh"
#include "kernels.h"

namespace bst {
namespace {

constexpr int BM = 128;
constexpr int kRowBytes = 128;                 // one swizzle atom row
constexpr int kTileRowsA = BM;
constexpr uint64_t kWaitNs = 2000000000ull;    // 2 s bound on any single wait
constexpr int kThreads = 192;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase of `bar` with the given parity; false (and an error code) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - start > kWaitNs) {
            atomicCAS(err, 0, code);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// Shared-memory matrix descriptor for a K-major tile of 128-byte rows with the 128-byte swizzle:
// 8-row groups 1024 bytes apart (SBO), leading offset unused (1), descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    uint64_t d = static_cast<uint64_t>((addr >> 4) & 0x3FFF);
    d |= static_cast<uint64_t>(1) << 16;
    d |= static_cast<uint64_t>(1024 >> 4) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(2) << 61;
    return d;
}

// Instruction descriptor: fp32 accumulate, A/B format (2 = tf32, 1 = bf16), both K-major,
// N = BN, M = 128.
template <int FMT, int BN>
__device__ __forceinline__ constexpr uint32_t instr_desc() {
    return (1u << 4) | (static_cast<uint32_t>(FMT) << 7) | (static_cast<uint32_t>(FMT) << 10) |
           (static_cast<uint32_t>(BN >> 3) << 17) | (static_cast<uint32_t>(BM >> 4) << 24);
}

template <int FMT>
__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                    uint32_t accumulate) {
    const uint32_t z = 0;
    if constexpr (FMT == 2) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
            "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z));
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
            "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z));
    }
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <int FMT, int BN>
struct Config {
    static constexpr int kPlanesA = 2;
    static constexpr int kPlanesB = FMT == 2 ? 2 : 1;
    static constexpr int kPasses = FMT == 2 ? 3 : 2;
    static constexpr int kBytesA = kTileRowsA * kRowBytes;  // one plane
    static constexpr int kBytesB = BN * kRowBytes;
    static constexpr int kStageBytes = kPlanesA * kBytesA + kPlanesB * kBytesB;
    // Narrow tiles serve the short decode GEMMs: two stages (<= 96 KB) let two CTAs share an SM.
    static constexpr int kStages = BN == 64 ? 2 : (192 * 1024) / kStageBytes;
    static constexpr int kElemsPerRow = FMT == 2 ? 32 : 64;  // K per stage
    static constexpr int kSmem = kStages * kStageBytes + 1024 + 256;
    static constexpr int kTmemCols = BN < 32 ? 32 : BN;
};

template <int FMT, int BN, Epi E>
__global__ __launch_bounds__(kThreads, 1) void k_gemm_tc(
    const __grid_constant__ CUtensorMap a0, const __grid_constant__ CUtensorMap a1,
    const __grid_constant__ CUtensorMap b0, const __grid_constant__ CUtensorMap b1,
    const float* __restrict__ bias, int M, int N, int K, EpiArgs ea, int* err, int splits,
    float* __restrict__ part) {
    using C = Config<FMT, BN>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(base + C::kStages * C::kStageBytes);
    uint64_t* empty = full + C::kStages;
    uint64_t* acc_full = empty + C::kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    // Split-K: this CTA accumulates k-tiles [kt0, kt1) (the host makes every split non-empty).
    const int k_total = (K + C::kElemsPerRow - 1) / C::kElemsPerRow;
    const int per = (k_total + splits - 1) / splits;
    const int kt0 = blockIdx.z * per;
    const int k_tiles = min(k_total, kt0 + per) - kt0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(C::kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    // Set-up above touches no data of earlier kernels; operands and outputs only after the wait.
    pdl_trigger();
    pdl_wait();

    auto stage_a = [&](int s, int p) { return base + s * C::kStageBytes + p * C::kBytesA; };
    auto stage_b = [&](int s, int p) {
        return base + s * C::kStageBytes + C::kPlanesA * C::kBytesA + p * C::kBytesB;
    };

    if (warp == 0) {
        if (lane == 0) {
            int issued = 0;
            bool ok = true;
            for (int kt = 0; kt < k_tiles && ok; ++kt) {
                const int s = kt % C::kStages;
                const uint32_t phase = (kt / C::kStages) & 1;
                ok = mbar_wait(&empty[s], phase ^ 1, err, 1);
                if (!ok) break;
                mbar_expect_tx(&full[s], C::kStageBytes);
                const int kx = (kt0 + kt) * C::kElemsPerRow;
                tma_load_2d(&a0, &full[s], stage_a(s, 0), kx, m0);
                tma_load_2d(&a1, &full[s], stage_a(s, 1), kx, m0);
                tma_load_2d(&b0, &full[s], stage_b(s, 0), kx, n0);
                if constexpr (C::kPlanesB == 2) tma_load_2d(&b1, &full[s], stage_b(s, 1), kx, n0);
                ++issued;
            }
            if (!ok) {
                // Drain this CTA's copies still in flight before shared memory goes away.
                for (int kt = (issued > C::kStages ? issued - C::kStages : 0); kt < issued; ++kt) {
                    mbar_wait(&full[kt % C::kStages], (kt / C::kStages) & 1, err, 1);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = instr_desc<FMT, BN>();
            bool ok = true;
            for (int kt = 0; kt < k_tiles; ++kt) {
                const int s = kt % C::kStages;
                const uint32_t phase = (kt / C::kStages) & 1;
                ok = mbar_wait(&full[s], phase, err, 2);
                if (!ok) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
                    for (int pass = 0; pass < C::kPasses; ++pass) {
                        // tf32: (Xh,Wh), (Xh,Wl), (Xl,Wh); bf16: (Xh,W), (Xl,W).
                        const int pa = (FMT == 2) ? (pass == 2 ? 1 : 0) : pass;
                        const int pb = (FMT == 2) ? (pass == 1 ? 1 : 0) : 0;
                        const uint64_t ad = smem_desc(smem_u32(stage_a(s, pa)) + kk * 32);
                        const uint64_t bd = smem_desc(smem_u32(stage_b(s, pb)) + kk * 32);
                        mma<FMT>(tmem, ad, bd, idesc, (kt | kk | pass) != 0);
                    }
                }
                mma_commit(&empty[s]);
            }
            if (ok) mma_commit(acc_full);
            else atomicCAS(err, 0, 2);
        }
    } else {
        // Epilogue warps 2..5 own TMEM lane quarters (warp % 4).
        const int quarter = warp & 3;
        const bool ok = mbar_wait(acc_full, 0, err, 3);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        // Stage the 128 x BN tile through shared memory (the drained pipeline ring), so the
        // global traffic below is row-coalesced.
        float* tile = reinterpret_cast<float*>(base);
        constexpr int LD = BN + 1;
        if (__all_sync(0xffffffffu, ok)) {
            const int r = quarter * 32 + lane;
            const uint32_t row_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
            for (int c = 0; c < BN; c += 16) {
                float v[16];
                tmem_ld16(row_addr + c, v);
#pragma unroll
                for (int j = 0; j < 16; ++j) tile[r * LD + c + j] = v[j];
            }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const int t = threadIdx.x - 64;
        if (splits > 1) {
            float* out = part + static_cast<size_t>(blockIdx.z) * M * N;
            for (int e = t; e < BM * BN; e += 128) {
                const int r = e / BN, c = e - r * BN;
                const int m = m0 + r, n = n0 + c;
                if (m < M && n < N) out[static_cast<size_t>(m) * N + n] = tile[r * LD + c];
            }
        } else {
            for (int e = t; e < BM * BN; e += 128) {
                const int r = e / BN, c = e - r * BN;
                const int m = m0 + r, n = n0 + c;
                if (m < M && n < N) {
                    const float v = tile[r * LD + c];
                    epi_apply<E>(ea, m, n, bias ? __fadd_rn(v, bias[n]) : v);
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(C::kTmemCols));
    }
}

// Split-K fix-up: out = sum over splits z = 0..S-1 (in that order) of part[z], then bias and the
// epilogue. Deterministic; coalesced over n.
template <Epi E>
__global__ void k_splitk_reduce(const float* __restrict__ part, int splits, int M, int N,
                                const float* __restrict__ bias, EpiArgs ea) {
    pdl_trigger();
    pdl_wait();
    // Grid: x over column blocks of 256, y over rows (strided).
    const size_t total = static_cast<size_t>(M) * N;
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    const float b = bias ? bias[n] : 0.0f;
    for (int m = blockIdx.y; m < M; m += gridDim.y) {
        const size_t e = static_cast<size_t>(m) * N + n;
        float v = 0.0f;
        for (int z = 0; z < splits; ++z) v += part[static_cast<size_t>(z) * total + e];
        epi_apply<E>(ea, m, n, bias ? __fadd_rn(v, b) : v);
    }
}

// Operand split: hi/lo planes of X (see the file comment).
__global__ void k_split_tf32(const float* __restrict__ x, int ldx, int M, int K,
                             float* __restrict__ hi, float* __restrict__ lo) {
    pdl_trigger();
    pdl_wait();
    // Grid: x over column blocks of 256, y over rows (strided).
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= K) return;
    for (int m = blockIdx.y; m < M; m += gridDim.y) {
        const float v = x[static_cast<size_t>(m) * ldx + k];
        const float h = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
        const size_t i = static_cast<size_t>(m) * K + k;
        hi[i] = h;
        lo[i] = __fsub_rn(v, h);
    }
}

__global__ void k_split_bf16(const float* __restrict__ x, int ldx, int M, int K,
                             __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
    pdl_trigger();
    pdl_wait();
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= K) return;
    for (int m = blockIdx.y; m < M; m += gridDim.y) {
        const float v = x[static_cast<size_t>(m) * ldx + k];
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        const size_t i = static_cast<size_t>(m) * K + k;
        hi[i] = h;
        lo[i] = __float2bfloat16_rn(__fsub_rn(v, __bfloat162float(h)));
    }
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

cudaError_t encoder() {
    std::call_once(g_encode_once, [] {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
        }
    });
    return g_encode ? cudaSuccess : cudaErrorNotSupported;
}

// 2-D row-major [rows, K] map with a (128-byte-row x box_rows) box, 128-byte swizzle, zero fill.
cudaError_t make_map(CUtensorMap* map, const void* ptr, int rows, int K, bool bf16,
                     int box_rows) {
    const size_t elem = bf16 ? 2 : 4;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * elem};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(kRowBytes / elem),
                         static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = g_encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                                2, const_cast<void*>(ptr), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

struct SplitK {
    int splits = 1;
    float* part = nullptr;
    bool defer = false;  // leave the split sums to the caller (launch_reduce_residual_ln)
};

template <int FMT, int BN, Epi E>
cudaError_t launch_typed(cudaStream_t s, const CUtensorMap& a0, const CUtensorMap& a1,
                         const CUtensorMap& b0, const CUtensorMap& b1, const float* bias, int M,
                         int N, int K, const EpiArgs& ea, int* err, const SplitK& sk) {
    using C = Config<FMT, BN>;
    const dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM, sk.splits);
    cudaError_t e = launch_pdl(k_gemm_tc<FMT, BN, E>, grid, dim3(kThreads), C::kSmem, s, a0, a1, b0,
                               b1, bias, M, N, K, ea, err, sk.splits, sk.part);
    if (e != cudaSuccess || sk.splits == 1 || sk.defer) return e;
    const dim3 rgrid((N + 255) / 256, std::min(M, std::max(1, 148 * 8 / ((N + 255) / 256))));
    return launch_pdl(k_splitk_reduce<E>, rgrid, dim3(256), 0, s, sk.part, sk.splits, M, N,
                      bias, ea);
}

template <int FMT, int BN>
cudaError_t launch_epi(cudaStream_t s, const CUtensorMap& a0, const CUtensorMap& a1,
                       const CUtensorMap& b0, const CUtensorMap& b1, const float* bias, int M,
                       int N, int K, Epi epi, const EpiArgs& ea, int* err, const SplitK& sk) {
    switch (epi) {
        case Epi::kStore: return launch_typed<FMT, BN, Epi::kStore>(s, a0, a1, b0, b1, bias, M, N, K, ea, err, sk);
        case Epi::kGelu: return launch_typed<FMT, BN, Epi::kGelu>(s, a0, a1, b0, b1, bias, M, N, K, ea, err, sk);
        case Epi::kResidual: return launch_typed<FMT, BN, Epi::kResidual>(s, a0, a1, b0, b1, bias, M, N, K, ea, err, sk);
        case Epi::kResidualGelu: return launch_typed<FMT, BN, Epi::kResidualGelu>(s, a0, a1, b0, b1, bias, M, N, K, ea, err, sk);
        case Epi::kQkv: return launch_typed<FMT, BN, Epi::kQkv>(s, a0, a1, b0, b1, bias, M, N, K, ea, err, sk);
        case Epi::kLogits: return launch_typed<FMT, BN, Epi::kLogits>(s, a0, a1, b0, b1, bias, M, N, K, ea, err, sk);
    }
    return cudaErrorInvalidValue;
}

template <int FMT, int BN>
cudaError_t set_smem_attrs() {
    using C = Config<FMT, BN>;
    const Epi all[] = {Epi::kStore, Epi::kGelu, Epi::kResidual, Epi::kResidualGelu, Epi::kQkv,
                       Epi::kLogits};
    cudaError_t err = cudaSuccess;
    for (Epi e : all) {
        const void* fn = nullptr;
        switch (e) {
            case Epi::kStore: fn = reinterpret_cast<const void*>(k_gemm_tc<FMT, BN, Epi::kStore>); break;
            case Epi::kGelu: fn = reinterpret_cast<const void*>(k_gemm_tc<FMT, BN, Epi::kGelu>); break;
            case Epi::kResidual: fn = reinterpret_cast<const void*>(k_gemm_tc<FMT, BN, Epi::kResidual>); break;
            case Epi::kResidualGelu: fn = reinterpret_cast<const void*>(k_gemm_tc<FMT, BN, Epi::kResidualGelu>); break;
            case Epi::kQkv: fn = reinterpret_cast<const void*>(k_gemm_tc<FMT, BN, Epi::kQkv>); break;
            case Epi::kLogits: fn = reinterpret_cast<const void*>(k_gemm_tc<FMT, BN, Epi::kLogits>); break;
        }
        err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
        if (err != cudaSuccess) return err;
    }
    return err;
}

}  // namespace

cudaError_t configure_tc_kernels() {
    cudaError_t err = encoder();
    if (err != cudaSuccess) return err;
    if ((err = set_smem_attrs<2, 64>()) != cudaSuccess) return err;
    if ((err = set_smem_attrs<2, 128>()) != cudaSuccess) return err;
    if ((err = set_smem_attrs<1, 64>()) != cudaSuccess) return err;
    return set_smem_attrs<1, 128>();
}

bool tc_usable(int M, int N, int K, int w_bf16) {
    if (M <= 8 || N < 16) return false;
    return w_bf16 ? (K % 8) == 0 : (K % 4) == 0;
}

size_t tc_split_bytes(int M, int K, int w_bf16) {
    return static_cast<size_t>(M) * K * (w_bf16 ? 2 : 4);
}

cudaError_t launch_split_operand(cudaStream_t s, const float* x, int ldx, int M, int K, int w_bf16,
                                 void* hi, void* lo) {
    if (M <= 0) return cudaSuccess;
    const dim3 grid((K + 255) / 256, std::min(M, std::max(1, 148 * 16 / ((K + 255) / 256))));
    if (w_bf16) {
        return launch_pdl(k_split_bf16, grid, dim3(256), 0, s, x, ldx, M, K,
                          static_cast<__nv_bfloat16*>(hi), static_cast<__nv_bfloat16*>(lo));
    }
    return launch_pdl(k_split_tf32, grid, dim3(256), 0, s, x, ldx, M, K,
                      static_cast<float*>(hi), static_cast<float*>(lo));
}

int tc_plan(int M, int N, int K, int w_bf16, size_t part_bytes, int* bn_out) {
    // Narrow tiles when the grid would not cover the SMs, then split K until it does (one wave);
    // each split keeps at least two k-tiles.
    const int tiles_m = (M + BM - 1) / BM;
    const int bn = ((N + 127) / 128) * tiles_m >= 148 ? 128 : 64;
    const int tiles = ((N + bn - 1) / bn) * tiles_m;
    const int k_tiles = (K + (w_bf16 ? 63 : 31)) / (w_bf16 ? 64 : 32);
    int splits = 1;
    if (tiles < 148) {
        splits = std::min((148 + tiles - 1) / tiles, std::max(1, k_tiles / 2));
        const size_t per_split = static_cast<size_t>(M) * N * sizeof(float);
        while (splits > 1 && per_split * splits > part_bytes) --splits;
        if (splits > 1) {
            const int per = (k_tiles + splits - 1) / splits;
            splits = (k_tiles + per - 1) / per;  // no empty split
        }
    }
    if (bn_out) *bn_out = bn;
    return splits;
}

size_t tc_part_bytes_max() { return static_cast<size_t>(296) * BM * 64 * sizeof(float); }

size_t tc_part_bytes(int M, int N, int K, int w_bf16) {
    const int splits = tc_plan(M, N, K, w_bf16, tc_part_bytes_max(), nullptr);
    return splits > 1 ? static_cast<size_t>(splits) * M * N * sizeof(float) : 0;
}

cudaError_t launch_gemm_tc(cudaStream_t s, const void* x_hi, const void* x_lo, const void* w,
                           const void* w_lo, int w_bf16, const float* bias, int M, int N, int K,
                           Epi epi, const EpiArgs& ea, int* err, float* part, size_t part_bytes,
                           bool defer_fixup) {
    if (M <= 0 || N <= 0) return cudaSuccess;
    cudaError_t e = encoder();
    if (e != cudaSuccess) return e;
    int bn = 64;
    SplitK sk;
    sk.splits = tc_plan(M, N, K, w_bf16, part ? part_bytes : 0, &bn);
    sk.part = part;
    sk.defer = defer_fixup;
    CUtensorMap a0, a1, b0, b1;
    if ((e = make_map(&a0, x_hi, M, K, w_bf16, BM)) != cudaSuccess) return e;
    if ((e = make_map(&a1, x_lo, M, K, w_bf16, BM)) != cudaSuccess) return e;
    if ((e = make_map(&b0, w, N, K, w_bf16, bn)) != cudaSuccess) return e;
    if (w_bf16) {
        b1 = b0;
    } else if ((e = make_map(&b1, w_lo, N, K, false, bn)) != cudaSuccess) {
        return e;
    }
    if (w_bf16) {
        return bn == 128 ? launch_epi<1, 128>(s, a0, a1, b0, b1, bias, M, N, K, epi, ea, err, sk)
                         : launch_epi<1, 64>(s, a0, a1, b0, b1, bias, M, N, K, epi, ea, err, sk);
    }
    return bn == 128 ? launch_epi<2, 128>(s, a0, a1, b0, b1, bias, M, N, K, epi, ea, err, sk)
                     : launch_epi<2, 64>(s, a0, a1, b0, b1, bias, M, N, K, epi, ea, err, sk);
}

}  // namespace bst
