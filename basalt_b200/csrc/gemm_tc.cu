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
// Tile: 128 x BN outputs (BN = 64 or 128), K staged in 128-byte rows (32 fp32 / 64 bf16) with the
// 128-byte swizzle. Two kernels share the tile machinery: k_gemm_tc runs one work unit (tile,
// k split) per CTA when all units fit in one wave (the decode GEMMs); k_gemm_tc_persistent loops
// each resident CTA over the units of larger GEMMs (prefill), with two TMEM accumulators so that
// the epilogue of one tile overlaps the MMAs of the next. In both, warp 0 issues TMA, warp 1
// owns TMEM and issues the MMAs, and the remaining warps drain TMEM (each warp reads its 32-lane
// quarter). Every mbarrier wait is bounded in time; on expiry the kernel records an error code,
// stops its other roles, drains its own copies and MMAs, and returns.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "device.cuh"
#include "epilogue.cuh"
#include "kernels.h"
#include "select.cuh"

namespace bst {
namespace {

constexpr int BM = 128;
constexpr int kRowBytes = 128;                 // one swizzle atom row
constexpr int kTileRowsA = BM;
constexpr uint64_t kWaitNs = 2000000000ull;    // 2 s bound on any single wait

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

// Waits for the phase of `bar` with the given parity. False on timeout (the error code is
// recorded and `abort` raised for the other roles of the CTA) or once another role has raised
// `abort`.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code,
                                          volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort) return false;
        if (global_ns() - start > kWaitNs) {
            atomicCAS(err, 0, code);
            *abort = 1;
            return false;
        }
    }
    return true;
}

// Bounded wait that ignores `abort`: used on the way out, to let copies and MMAs already issued
// finish before their shared memory or TMEM is released.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity, int* err, int code) {
    const uint64_t start = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - start > kWaitNs) {
            atomicCAS(err, 0, code);
            return;
        }
    }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// Tiled bulk store of one box from shared memory into a 3-D tensor (the split-K partials), then
// the wait until the box has been read out of shared memory. Elements outside the tensor are not
// written.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int x, int y,
                                             int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ void tma_store_commit_and_drain() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
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

// CW (16 or 32) consecutive accumulator columns of this thread's TMEM lane (one row of the tile).
template <int CW>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float* v) {
    uint32_t r[CW];
    if constexpr (CW == 32) {
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
            "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
            "%28, %29, %30, %31}, [%32];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
              "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
              "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
              "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
              "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
              "=r"(r[31])
            : "r"(taddr));
    } else {
        static_assert(CW == 16, "chunk width");
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
            "%11, %12, %13, %14, %15}, [%16];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
              "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
              "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
            : "r"(taddr));
    }
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < CW; ++i) v[i] = __uint_as_float(r[i]);
}

template <int FMT, int BN, int ST = 0>
struct Config {
    static constexpr int kPlanesA = 2;
    static constexpr int kPlanesB = FMT == 2 ? 2 : 1;
    static constexpr int kPasses = FMT == 2 ? 3 : 2;
    static constexpr int kBytesA = kTileRowsA * kRowBytes;  // one plane
    static constexpr int kBytesB = BN * kRowBytes;
    static constexpr int kStageBytes = kPlanesA * kBytesA + kPlanesB * kBytesB;
    // Narrow tiles serve the short decode GEMMs: three stages (<= 144 KB, one CTA per SM) when
    // the units fit one wave of the SMs. Measured on the two-lane decode step of 128-row lanes:
    // 2 stages (two CTAs per SM) and 4 stages (192 KB, little room left for the other lane's
    // kernels on the SM) were both ~4-5 % slower. GEMMs with up to two units per SM (512-row
    // lanes) run the ST = 2 variant, two CTAs per SM, in one wave.
    static constexpr int kStages = ST ? ST : BN == 64 ? 3 : (192 * 1024) / kStageBytes;
    static constexpr int kElemsPerRow = FMT == 2 ? 32 : 64;  // K per stage
    static constexpr int kSmem = kStages * kStageBytes + 1024 + 256;
    // Two accumulators for the persistent variant: the epilogue drains one while the MMAs fill
    // the other.
    static constexpr int kTmemCols = 2 * BN;
    static constexpr int kCtasPerSm = kStages * kStageBytes <= 100 * 1024 ? 2 : 1;
    // Epilogue warps 2.. cover the four TMEM lane quarters kColGroups times over, each warp a
    // column range of BN / kColGroups drained CW columns at a time. The narrow decode tiles keep
    // a small footprint (192 threads, 16-column chunks) so that the other decode lane's kernels
    // share the SM.
    static constexpr int kColGroups = BN == 64 ? 1 : 2;
    static constexpr int kEpiWarps = 4 * kColGroups;
    static constexpr int kThreads = 64 + 32 * kEpiWarps;
    static constexpr int CW = BN == 64 ? 16 : 32;
};

__device__ __forceinline__ void st4(float* p, float a, float b, float c, float d) {
    *reinterpret_cast<float4*>(p) = make_float4(a, b, c, d);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Writes CW consecutive values v[0..CW) of one row as fp32 (f32 = true) or bf16 to p, which is
// 16-byte aligned.
template <int CW>
__device__ __forceinline__ void store_row(void* p, const float* v, bool f32) {
    if (f32) {
        float* q = static_cast<float*>(p);
#pragma unroll
        for (int j = 0; j < CW; j += 4) st4(q + j, v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
        uint4* q = static_cast<uint4*>(p);
#pragma unroll
        for (int j = 0; j < CW; j += 8) {
            q[j / 8] = make_uint4(pack_bf16(v[j], v[j + 1]), pack_bf16(v[j + 2], v[j + 3]),
                                  pack_bf16(v[j + 4], v[j + 5]), pack_bf16(v[j + 6], v[j + 7]));
        }
    }
}

// Operand planes of CW values (store_split, vectorised): planes = 1 tf32 hi + fp32 remainder,
// planes = 2 bf16 hi + bf16 remainder.
template <int CW>
__device__ __forceinline__ void store_split_row(const float* v, const PlaneOut& po, size_t idx) {
#pragma unroll
    for (int g = 0; g < CW; g += 8) {
        float h[8], l[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (po.planes == 1) {
                h[j] = __uint_as_float(__float_as_uint(v[g + j]) & 0xFFFFE000u);
            } else {
                h[j] = __bfloat162float(__float2bfloat16_rn(v[g + j]));
            }
            l[j] = __fsub_rn(v[g + j], h[j]);
        }
        if (po.planes == 1) {
            float* hi = static_cast<float*>(po.hi) + idx + g;
            float* lo = static_cast<float*>(po.lo) + idx + g;
            st4(hi, h[0], h[1], h[2], h[3]);
            st4(hi + 4, h[4], h[5], h[6], h[7]);
            st4(lo, l[0], l[1], l[2], l[3]);
            st4(lo + 4, l[4], l[5], l[6], l[7]);
        } else {
            *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(po.hi) + idx + g) =
                make_uint4(pack_bf16(h[0], h[1]), pack_bf16(h[2], h[3]), pack_bf16(h[4], h[5]),
                           pack_bf16(h[6], h[7]));
            *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(po.lo) + idx + g) =
                make_uint4(pack_bf16(l[0], l[1]), pack_bf16(l[2], l[3]), pack_bf16(l[4], l[5]),
                           pack_bf16(l[6], l[7]));
        }
    }
}

__device__ __forceinline__ bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

// True when the CW-column vector epilogue applies to every full chunk of this launch: the
// destinations are 16-byte aligned with row strides that keep them so, and (kQkv) no chunk
// straddles a head.
template <Epi E, int CW>
__device__ __forceinline__ bool vector_epilogue_ok(const EpiArgs& ea, const float* bias, int N,
                                                   int splits, const float* part) {
    bool ok = bias == nullptr || aligned16(bias);
    if (splits > 1) return aligned16(part) && (N % 4) == 0;
    const bool planes_ok = ea.split.planes == 0 ||
                           (aligned16(ea.split.hi) && aligned16(ea.split.lo) &&
                            (ea.split.ld % (ea.split.planes == 1 ? 4 : 8)) == 0);
    if constexpr (E == Epi::kStore || E == Epi::kGelu) {
        ok = ok && aligned16(ea.out) && (ea.ldo % 4) == 0 && planes_ok;
    } else if constexpr (E == Epi::kResidual || E == Epi::kLogits) {
        ok = ok && aligned16(ea.out) && (ea.ldo % 4) == 0;
    } else if constexpr (E == Epi::kResidualGelu) {
        ok = ok && aligned16(ea.out) && (ea.ldo % 4) == 0 && aligned16(ea.res) && (ea.ldr % 4) == 0;
    } else if constexpr (E == Epi::kQkv) {
        ok = ok && aligned16(ea.out) && (ea.ldo % 4) == 0 && (ea.d % CW) == 0 &&
             (ea.head_dim % CW) == 0 && aligned16(ea.k_cache) && aligned16(ea.v_cache);
    }
    return ok;
}

// Epilogue of one row's CW consecutive columns [n, n + CW), all inside the matrix, vector path.
template <Epi E, int CW>
__device__ __forceinline__ void epilogue_row(const EpiArgs& ea, int m, int n, float* v, int M, int N,
                                           int z, float* part, int row_map, int row_slot) {
    if (part) {
        store_row<CW>(part + static_cast<size_t>(z) * M * N + static_cast<size_t>(m) * N + n, v, true);
        return;
    }
    if constexpr (E == Epi::kStore || E == Epi::kGelu) {
        if constexpr (E == Epi::kGelu) {
#pragma unroll
            for (int j = 0; j < CW; ++j) v[j] = gelu_ref(v[j]);
        }
        if (ea.out) store_row<CW>(ea.out + static_cast<size_t>(m) * ea.ldo + n, v, true);
        if (ea.split.planes) store_split_row<CW>(v, ea.split, static_cast<size_t>(m) * ea.split.ld + n);
    } else if constexpr (E == Epi::kResidual || E == Epi::kResidualGelu) {
        const float* src = E == Epi::kResidual ? ea.out + static_cast<size_t>(m) * ea.ldo + n
                                               : ea.res + static_cast<size_t>(m) * ea.ldr + n;
        float r[CW];
#pragma unroll
        for (int j = 0; j < CW; j += 4) {
            const float4 t = *reinterpret_cast<const float4*>(src + j);
            r[j] = t.x;
            r[j + 1] = t.y;
            r[j + 2] = t.z;
            r[j + 3] = t.w;
        }
#pragma unroll
        for (int j = 0; j < CW; ++j) {
            v[j] = E == Epi::kResidual ? __fadd_rn(r[j], v[j]) : gelu_ref(__fadd_rn(v[j], r[j]));
        }
        store_row<CW>(ea.out + static_cast<size_t>(m) * ea.ldo + n, v, true);
    } else if constexpr (E == Epi::kQkv) {
        if (n < ea.d) {
            store_row<CW>(ea.out + static_cast<size_t>(m) * ea.ldo + n, v, true);
        } else {
            const int which = n / ea.d;
            const int j = n - which * ea.d;
            const int h = j / ea.head_dim;
            const int e = j - h * ea.head_dim;
            const size_t idx =
                ((static_cast<size_t>(row_map) * ea.heads + h) * ea.slots + row_slot) * ea.head_dim + e;
            void* base = which == 1 ? ea.k_cache : ea.v_cache;
            if (ea.kv_bf16) {
                store_row<CW>(static_cast<__nv_bfloat16*>(base) + idx, v, false);
            } else {
                store_row<CW>(static_cast<float*>(base) + idx, v, true);
            }
        }
    } else if constexpr (E == Epi::kLogits) {
        store_row<CW>(ea.out + static_cast<size_t>(row_map) * ea.ldo + n, v, true);
        if (ea.best) {
            // One atomic per row chunk: the chunk's first maximum, packed.
            unsigned long long b = 0ull;
#pragma unroll
            for (int j = 0; j < CW; ++j) {
                if (!isnan(v[j])) {
                    const unsigned long long p = pack_best(v[j], n + j);
                    b = p > b ? p : b;
                }
            }
            if (b) atomicMax(ea.best + row_map, b);
        }
    }
}

// One tile per CTA (grid n x m x k-split): the short decode GEMMs, where every unit fits in one
// wave. Warp 0 issues TMA (the weight tiles of the first stages before the PDL wait), warp 1 owns
// TMEM and issues the MMAs, warps 2-5 drain TMEM (each warp reads its 32-lane quarter) through
// the idle ring into row-coalesced stores. ST overrides the ring depth (0: Config's default, one
// CTA per SM for narrow tiles; 2: two CTAs per SM). Kept apart from the persistent kernel below:
// these launches are short, and the lean code and the single accumulator measured faster here.
constexpr int kSingleThreads = 192;

// Bounded wait for the single-tile kernel (no other role to stop early).
__device__ __forceinline__ bool mbar_wait_tile(uint64_t* bar, uint32_t parity, int* err, int code) {
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

template <int FMT, int BN, Epi E, int ST>
__global__ __launch_bounds__(kSingleThreads, 1) void k_gemm_tc(
    const __grid_constant__ CUtensorMap a0, const __grid_constant__ CUtensorMap a1,
    const __grid_constant__ CUtensorMap b0, const __grid_constant__ CUtensorMap b1,
    const __grid_constant__ CUtensorMap pmap, const float* __restrict__ bias, int M, int N, int K,
    EpiArgs ea, int* err, int splits, float* __restrict__ part, int part_tma) {
    using C = Config<FMT, BN, ST>;
    constexpr int kSingleTmemCols = BN < 32 ? 32 : BN;
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
                     "r"(kSingleTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    auto stage_a = [&](int s, int p) { return base + s * C::kStageBytes + p * C::kBytesA; };
    auto stage_b = [&](int s, int p) {
        return base + s * C::kStageBytes + C::kPlanesA * C::kBytesA + p * C::kBytesB;
    };
    // Weights are constant: the first stages' weight tiles load while the previous kernel still
    // runs. Activations (operand planes) and every output only after the wait.
    const int pre = min(k_tiles, C::kStages);
    if (warp == 0 && lane == 0) {
        for (int kt = 0; kt < pre; ++kt) {
            mbar_expect_tx(&full[kt], C::kStageBytes);
            const int kx = (kt0 + kt) * C::kElemsPerRow;
            tma_load_2d(&b0, &full[kt], stage_b(kt, 0), kx, n0);
            if constexpr (C::kPlanesB == 2) tma_load_2d(&b1, &full[kt], stage_b(kt, 1), kx, n0);
        }
    }
    pdl_trigger();
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            int issued = 0;
            bool ok = true;
            for (int kt = 0; kt < k_tiles && ok; ++kt) {
                const int s = kt % C::kStages;
                const uint32_t phase = (kt / C::kStages) & 1;
                ok = mbar_wait_tile(&empty[s], phase ^ 1, err, 1);
                if (!ok) break;
                if (kt >= pre) mbar_expect_tx(&full[s], C::kStageBytes);
                const int kx = (kt0 + kt) * C::kElemsPerRow;
                tma_load_2d(&a0, &full[s], stage_a(s, 0), kx, m0);
                tma_load_2d(&a1, &full[s], stage_a(s, 1), kx, m0);
                if (kt >= pre) {
                    tma_load_2d(&b0, &full[s], stage_b(s, 0), kx, n0);
                    if constexpr (C::kPlanesB == 2) tma_load_2d(&b1, &full[s], stage_b(s, 1), kx, n0);
                }
                ++issued;
            }
            if (!ok) {
                // Drain this CTA's copies still in flight before shared memory goes away.
                for (int kt = (issued > C::kStages ? issued - C::kStages : 0); kt < issued; ++kt) {
                    mbar_wait_tile(&full[kt % C::kStages], (kt / C::kStages) & 1, err, 1);
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
                ok = mbar_wait_tile(&full[s], phase, err, 2);
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
        const bool ok = mbar_wait_tile(acc_full, 0, err, 3);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (part_tma) {
            // Split-K partials leave through the TMA unit: the tile is staged in the drained
            // ring as BN / 32 boxes of 128 rows x 128 bytes in the 128-byte swizzle (the 16-byte
            // chunk q of row r at chunk q ^ (r % 8), so each quarter-warp's vector stores hit
            // distinct banks), then one thread stores the boxes into part[z] and waits until
            // they have been read out of shared memory.
            const bool all_ok = __all_sync(0xffffffffu, ok);
            if (all_ok) {
                const int r = quarter * 32 + lane;
                const uint32_t row_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
                unsigned char* rowp = base + r * kRowBytes;
#pragma unroll 1
                for (int c = 0; c < BN; c += 16) {
                    float v[16];
                    tmem_ld<16>(row_addr + c, v);
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        const int col = c + 4 * g;
                        const int q = (col & 31) >> 2;
                        float4* dst = reinterpret_cast<float4*>(
                            rowp + (col >> 5) * (BM * kRowBytes) + ((q ^ (r & 7)) << 4));
                        *dst = make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
                    }
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (threadIdx.x == 64 && all_ok) {
#pragma unroll
                for (int j = 0; j < BN / 32; ++j) {
                    if (n0 + 32 * j < N) {
                        tma_store_3d(&pmap, base + j * (BM * kRowBytes), n0 + 32 * j, m0,
                                     blockIdx.z);
                    }
                }
                tma_store_commit_and_drain();
            }
        } else {
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
                tmem_ld<16>(row_addr + c, v);
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
        } else if (vector_epilogue_ok<E, 16>(ea, bias, N, 1, nullptr)) {
            // 16-column chunks of a row per thread through the vector epilogue (16-byte loads
            // and stores); chunks that stick out of the matrix go element by element.
            constexpr int kChunks = BN / 16;
            for (int e = t; e < BM * kChunks; e += 128) {
                const int r = e / kChunks, c = (e - r * kChunks) * 16;
                const int m = m0 + r, n = n0 + c;
                if (m >= M || n >= N) continue;
                float v[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    v[j] = tile[r * LD + c + j];
                    if (bias && n + j < N) v[j] = __fadd_rn(v[j], bias[n + j]);
                }
                if (n + 16 <= N) {
                    int row_map = 0, row_slot = 0;
                    if constexpr (E == Epi::kQkv || E == Epi::kLogits) {
                        row_map = ea.rowmap[m];
                        if constexpr (E == Epi::kQkv) row_slot = ea.slot[m];
                    }
                    epilogue_row<E, 16>(ea, m, n, v, M, N, 0, nullptr, row_map, row_slot);
                } else {
                    for (int j = 0; j < 16 && n + j < N; ++j) epi_apply<E>(ea, m, n + j, v[j]);
                }
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
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kSingleTmemCols));
    }
}


// Persistent tcgen05 GEMM. Work units are (n tile, m tile, k split), n fastest so that the CTAs
// running at one time share A rows in L2; CTA b takes units b, b + gridDim.x, ... Warp 0 streams
// k-tiles of all its units through the shared-memory ring, warp 1 issues the MMAs of unit i into
// accumulator i % 2, and the eight epilogue warps drain the other accumulator meanwhile.
template <int FMT, int BN, Epi E>
__global__ __launch_bounds__(Config<FMT, BN>::kThreads, Config<FMT, BN>::kCtasPerSm) void k_gemm_tc_persistent(
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
    uint64_t* acc_full = empty + C::kStages;     // [2]
    uint64_t* acc_empty = acc_full + 2;          // [2]
    uint64_t* drained = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_n = (N + BN - 1) / BN, tiles_m = (M + BM - 1) / BM;
    const int units = tiles_n * tiles_m * splits;
    // Split-K: split z accumulates k-tiles [z * per, min(k_total, (z + 1) * per)); the host makes
    // every split non-empty.
    const int k_total = (K + C::kElemsPerRow - 1) / C::kElemsPerRow;
    const int per = (k_total + splits - 1) / splits;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], C::kEpiWarps);
        }
        mbar_init(drained, 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    constexpr int kTmemCols = C::kTmemCols;
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols));
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
    auto unit_coords = [&](int u, int* m0, int* n0, int* z) {
        *n0 = (u % tiles_n) * BN;
        const int rest = u / tiles_n;
        *m0 = (rest % tiles_m) * BM;
        *z = rest / tiles_m;
    };

    if (warp == 0) {
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
                int m0, n0, z;
                unit_coords(u, &m0, &n0, &z);
                const int kt0 = z * per, kt1 = min(k_total, kt0 + per);
                for (int kt = kt0; kt < kt1; ++kt, ++it) {
                    const int s = it % C::kStages;
                    const uint32_t phase = (it / C::kStages) & 1;
                    ok = mbar_wait(&empty[s], phase ^ 1, err, 1, abort);
                    if (!ok) break;
                    mbar_expect_tx(&full[s], C::kStageBytes);
                    const int kx = kt * C::kElemsPerRow;
                    tma_load_2d(&a0, &full[s], stage_a(s, 0), kx, m0);
                    tma_load_2d(&a1, &full[s], stage_a(s, 1), kx, m0);
                    tma_load_2d(&b0, &full[s], stage_b(s, 0), kx, n0);
                    if constexpr (C::kPlanesB == 2) tma_load_2d(&b1, &full[s], stage_b(s, 1), kx, n0);
                }
            }
            if (!ok) {
                // Drain this CTA's copies still in flight before shared memory goes away.
                for (int i = (it > C::kStages ? it - C::kStages : 0); i < it; ++i) {
                    mbar_drain(&full[i % C::kStages], (i / C::kStages) & 1, err, 1);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = instr_desc<FMT, BN>();
            int it = 0, local = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++local) {
                int m0, n0, z;
                unit_coords(u, &m0, &n0, &z);
                const int kt0 = z * per, kt1 = min(k_total, kt0 + per);
                const int buf = local & 1;
                ok = mbar_wait(&acc_empty[buf], ((local >> 1) & 1) ^ 1, err, 4, abort);
                if (!ok) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t acc = tmem + static_cast<uint32_t>(buf * BN);
                for (int kt = kt0; kt < kt1; ++kt, ++it) {
                    const int s = it % C::kStages;
                    const uint32_t phase = (it / C::kStages) & 1;
                    ok = mbar_wait(&full[s], phase, err, 2, abort);
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
                            mma<FMT>(acc, ad, bd, idesc, (kt != kt0) | kk | pass);
                        }
                    }
                    mma_commit(&empty[s]);
                }
                if (!ok) break;
                mma_commit(&acc_full[buf]);
            }
            // Every MMA issued above completes before the accumulators are released.
            mma_commit(drained);
            mbar_drain(drained, 0, err, 5);
        }
    } else {
        // Epilogue warps: TMEM lane quarter warp % 4 (rows), column group (warp - 2) / 4.
        constexpr int CW = C::CW;
        constexpr int kSpan = BN / C::kColGroups;
        const int quarter = warp & 3;
        const int group = (warp - 2) >> 2;
        const bool vec = vector_epilogue_ok<E, CW>(ea, bias, N, splits, part);
        int local = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, ++local) {
            int m0, n0, z;
            unit_coords(u, &m0, &n0, &z);
            const int buf = local & 1;
            const bool ok = mbar_wait(&acc_full[buf], (local >> 1) & 1, err, 3, abort);
            if (!__all_sync(0xffffffffu, ok)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int m = m0 + quarter * 32 + lane;
            int row_map = 0, row_slot = 0;
            if constexpr (E == Epi::kQkv || E == Epi::kLogits) {
                if (splits == 1 && m < M) {
                    row_map = ea.rowmap[m];
                    if constexpr (E == Epi::kQkv) row_slot = ea.slot[m];
                }
            }
            const uint32_t row_addr =
                tmem + static_cast<uint32_t>(buf * BN) + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
            for (int c = group * kSpan; c < (group + 1) * kSpan; c += CW) {
                float v[CW];
                tmem_ld<CW>(row_addr + c, v);
                const int n = n0 + c;
                if (m < M && n < N) {
                if (splits == 1 && bias) {
#pragma unroll
                    for (int j = 0; j < CW; ++j) {
                        if (n + j < N) v[j] = __fadd_rn(v[j], __ldg(bias + n + j));
                    }
                }
                if (vec && n + CW <= N) {
                    epilogue_row<E, CW>(ea, m, n, v, M, N, z, splits > 1 ? part : nullptr, row_map,
                                        row_slot);
                } else if (splits > 1) {
                    float* out = part + static_cast<size_t>(z) * M * N + static_cast<size_t>(m) * N;
#pragma unroll
                    for (int j = 0; j < CW; ++j) {
                        if (n + j < N) out[n + j] = v[j];
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < CW; ++j) {
                        if (n + j < N) epi_apply<E>(ea, m, n + j, v[j]);
                    }
                }
                }
                __syncwarp();
            }
            // This warp's reads of the accumulator are done: hand it back to the MMA warp.
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols));
    }
}

// Split-K fix-up: out = sum over splits z = 0..S-1 (in that order) of part[z], then bias and the
// epilogue. Deterministic; coalesced over n.
template <Epi E>
__global__ void k_splitk_reduce(const float* __restrict__ part, int splits, int M, int N,
                                const float* __restrict__ bias, EpiArgs ea) {
    // Grid: x over column blocks of 256, y over rows (strided).
    const size_t total = static_cast<size_t>(M) * N;
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    const float b = bias && n < N ? bias[n] : 0.0f;  // a weight: read before the wait
    pdl_trigger();
    pdl_wait();
    if (n >= N) return;
    for (int m = blockIdx.y; m < M; m += gridDim.y) {
        const size_t e = static_cast<size_t>(m) * N + n;
        // Up to 8 splits' loads in flight, then summed in split order.
        float t[8];
#pragma unroll
        for (int z = 0; z < 8; ++z) t[z] = z < splits ? part[static_cast<size_t>(z) * total + e] : 0.0f;
        float v = 0.0f;
#pragma unroll
        for (int z = 0; z < 8; ++z) {
            if (z < splits) v += t[z];
        }
        for (int z = 8; z < splits; ++z) v += part[static_cast<size_t>(z) * total + e];
        epi_apply<E>(ea, m, n, bias ? __fadd_rn(v, b) : v);
    }
}

// k_splitk_reduce with 8 consecutive columns per thread through the vector epilogue: the split
// sums in the same order (then the bias), 16-byte loads of the partials and 16-byte stores.
// Grid: x over column blocks of 8 * blockDim.x, y over rows (one row per block).
template <Epi E>
__global__ __launch_bounds__(256) void k_splitk_reduce_vec(const float* __restrict__ part,
                                                          int splits, int M, int N,
                                                          const float* __restrict__ bias,
                                                          EpiArgs ea) {
    constexpr int CW = 8;
    const size_t total = static_cast<size_t>(M) * N;
    const int n = (blockIdx.x * blockDim.x + threadIdx.x) * CW;
    const int m = blockIdx.y;
    float b[CW];
#pragma unroll
    for (int j = 0; j < CW; ++j) b[j] = bias && n + j < N ? bias[n + j] : 0.0f;  // a weight
    pdl_trigger();
    pdl_wait();
    if (n >= N) return;
    const float* src = part + static_cast<size_t>(m) * N + n;
    float v[CW];
#pragma unroll
    for (int j = 0; j < CW; ++j) v[j] = 0.0f;
    for (int z0 = 0; z0 < splits; z0 += 4) {
        float4 t[4][2];
#pragma unroll
        for (int z = 0; z < 4; ++z) {
            if (z0 + z < splits) {
                t[z][0] = __ldcg(reinterpret_cast<const float4*>(src + (z0 + z) * total));
                t[z][1] = __ldcg(reinterpret_cast<const float4*>(src + (z0 + z) * total + 4));
            }
        }
#pragma unroll
        for (int z = 0; z < 4; ++z) {
            if (z0 + z < splits) {
                v[0] += t[z][0].x; v[1] += t[z][0].y; v[2] += t[z][0].z; v[3] += t[z][0].w;
                v[4] += t[z][1].x; v[5] += t[z][1].y; v[6] += t[z][1].z; v[7] += t[z][1].w;
            }
        }
    }
    if (bias) {
#pragma unroll
        for (int j = 0; j < CW; ++j) v[j] = __fadd_rn(v[j], b[j]);
    }
    int row_map = 0, row_slot = 0;
    if constexpr (E == Epi::kQkv || E == Epi::kLogits) {
        row_map = ea.rowmap[m];
        if constexpr (E == Epi::kQkv) row_slot = ea.slot[m];
    }
    epilogue_row<E, CW>(ea, m, n, v, M, N, 0, nullptr, row_map, row_slot);
}

// The split-K fix-up of the head when it folds the argmax: one block per row, so the row's
// packed first maximum is reduced inside the block and stored with one plain write (no atomics).
// The sums and the logits it writes are those of k_splitk_reduce<kLogits>.
__global__ __launch_bounds__(256) void k_splitk_reduce_logits_best(const float* __restrict__ part,
                                                                   int splits, int M, int N,
                                                                   const float* __restrict__ bias,
                                                                   EpiArgs ea) {
    pdl_trigger();
    pdl_wait();
    __shared__ unsigned long long s_best[8];
    __shared__ float s_first;
    __shared__ int s_step, s_token;
    const int m = blockIdx.x;
    if (ea.step && threadIdx.x == 0) s_step = *reinterpret_cast<volatile int*>(ea.step);
    const size_t total = static_cast<size_t>(M) * N;
    unsigned long long best = 0ull;
    float* out = ea.out + static_cast<size_t>(ea.rowmap[m]) * ea.ldo;
    // Vector path: every thread loads all its columns' partials (16-byte loads, up to kCols
    // columns and kMaxZ splits) before summing any, so the row costs one round trip to L2.
    constexpr int kCols = 16, kMaxZ = 4;
    const bool vec = splits <= kMaxZ && N <= kCols * static_cast<int>(blockDim.x) && (N % 4) == 0 &&
                     (reinterpret_cast<uintptr_t>(part) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
                     (bias == nullptr || (reinterpret_cast<uintptr_t>(bias) & 15) == 0);
    if (vec) {
        float4 t[kCols / 4][kMaxZ];
#pragma unroll
        for (int c = 0; c < kCols / 4; ++c) {
            const int n = 4 * (threadIdx.x + c * blockDim.x);
#pragma unroll
            for (int z = 0; z < kMaxZ; ++z) {
                t[c][z] = n < N && z < splits
                              ? __ldcg(reinterpret_cast<const float4*>(part + z * total + m * static_cast<size_t>(N) + n))
                              : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
        }
#pragma unroll
        for (int c = 0; c < kCols / 4; ++c) {
            const int n = 4 * (threadIdx.x + c * blockDim.x);
            if (n >= N) continue;
            float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int z = 0; z < kMaxZ; ++z) {
                if (z < splits) {
                    v[0] += t[c][z].x;
                    v[1] += t[c][z].y;
                    v[2] += t[c][z].z;
                    v[3] += t[c][z].w;
                }
            }
            if (bias) {
                const float4 b = *reinterpret_cast<const float4*>(bias + n);
                v[0] = __fadd_rn(v[0], b.x);
                v[1] = __fadd_rn(v[1], b.y);
                v[2] = __fadd_rn(v[2], b.z);
                v[3] = __fadd_rn(v[3], b.w);
            }
            *reinterpret_cast<float4*>(out + n) = make_float4(v[0], v[1], v[2], v[3]);
            if (n == 0) s_first = v[0];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (!isnan(v[j])) {
                    const unsigned long long p = pack_best(v[j], n + j);
                    best = p > best ? p : best;
                }
            }
        }
    }
    for (int n = vec ? N : threadIdx.x; n < N; n += blockDim.x) {
        const size_t e = static_cast<size_t>(m) * N + n;
        float t[8];
#pragma unroll
        for (int z = 0; z < 8; ++z) t[z] = z < splits ? part[static_cast<size_t>(z) * total + e] : 0.0f;
        float v = 0.0f;
#pragma unroll
        for (int z = 0; z < 8; ++z) {
            if (z < splits) v += t[z];
        }
        for (int z = 8; z < splits; ++z) v += part[static_cast<size_t>(z) * total + e];
        if (bias) v = __fadd_rn(v, bias[n]);
        out[n] = v;
        if (n == 0) s_first = v;
        if (!isnan(v)) {
            const unsigned long long p = pack_best(v, n);
            best = p > best ? p : best;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long q = __shfl_xor_sync(0xffffffffu, best, o);
        best = q > best ? q : best;
    }
    if ((threadIdx.x & 31) == 0) s_best[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) best = s_best[w] > best ? s_best[w] : best;
        if (ea.step) {
            // TextEngine.argmax (TextEngine.java:392-400): the first maximum; a NaN first
            // score is never replaced, so it selects token 0.
            s_token = (isnan(s_first) || best == 0ull) ? 0 : unpack_best_index(best);
        } else {
            ea.best[ea.rowmap[m]] = best;
        }
    }
    if (ea.step) {
        __syncthreads();
        finish_row(ea.rowmap[m], s_token, s_step, ea.rows, ea.window_len, ea.steps, ea.step,
                   ea.done, ea.tokens, ea.next, ea.window);
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

// Streaming multiprocessors of the current device (the persistent grid's size).
int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) {
        cudaGetLastError();
        return 148;
    }
    return n;
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

// 3-D map over split-K partials part[splits][M][N] (fp32) with a 32-column x 128-row box in the
// 128-byte swizzle, for the tiled bulk stores of k_gemm_tc. Needs N % 4 == 0 (16-byte strides).
cudaError_t make_part_map(CUtensorMap* map, float* part, int splits, int M, int N) {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M),
                          static_cast<cuuint64_t>(splits)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(N) * 4, static_cast<cuuint64_t>(M) * N * 4};
    cuuint32_t box[3] = {32, static_cast<cuuint32_t>(BM), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, part, dims, strides, box,
                                estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

struct SplitK {
    int splits = 1;
    float* part = nullptr;
    bool defer = false;  // leave the split sums to the caller (launch_reduce_residual_ln)
    CUtensorMap pmap{};  // over part, when tma is set
    int tma = 0;         // the one-tile kernel stores the partials with the TMA unit
};

// Host-side counterpart of vector_epilogue_ok for the kStore / kGelu epilogues of an 8-column
// vector fix-up: 16-byte aligned destinations whose row strides keep them so.
bool host_vector_epilogue_ok(const EpiArgs& ea, int N) {
    auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (ea.out && (!a16(ea.out) || ea.ldo % 4 != 0)) return false;
    if (ea.split.planes) {
        if (!a16(ea.split.hi) || !a16(ea.split.lo) || ea.split.ld % 8 != 0) return false;
    }
    return N % 8 == 0;
}

template <int FMT, int BN, Epi E>
cudaError_t launch_typed(cudaStream_t s, const CUtensorMap& a0, const CUtensorMap& a1,
                         const CUtensorMap& b0, const CUtensorMap& b1, const float* bias, int M,
                         int N, int K, const EpiArgs& ea, int* err, const SplitK& sk) {
    using C = Config<FMT, BN>;
    const long units = static_cast<long>((N + BN - 1) / BN) * ((M + BM - 1) / BM) * sk.splits;
    const long sms = sm_count();
    const long resident = sms * C::kCtasPerSm;
    const dim3 tiles((N + BN - 1) / BN, (M + BM - 1) / BM, sk.splits);
    cudaError_t e = cudaSuccess;
    if (units <= resident) {
        e = launch_pdl(k_gemm_tc<FMT, BN, E, 0>, tiles, dim3(kSingleThreads), C::kSmem, s, a0, a1,
                       b0, b1, sk.pmap, bias, M, N, K, ea, err, sk.splits, sk.part, sk.tma);
    } else if (BN == 64 && units <= sms * Config<FMT, BN, 2>::kCtasPerSm) {
        if constexpr (BN == 64) {
            e = launch_pdl(k_gemm_tc<FMT, BN, E, 2>, tiles, dim3(kSingleThreads),
                           Config<FMT, BN, 2>::kSmem, s, a0, a1, b0, b1, sk.pmap, bias, M, N, K,
                           ea, err, sk.splits, sk.part, sk.tma);
        }
    } else {
        const dim3 grid(static_cast<unsigned>(std::min<long>(units, resident)));
        e = launch_pdl(k_gemm_tc_persistent<FMT, BN, E>, grid, dim3(C::kThreads), C::kSmem, s, a0,
                       a1, b0, b1, bias, M, N, K, ea, err, sk.splits, sk.part);
    }
    if (e != cudaSuccess || sk.splits == 1 || sk.defer) return e;
    if constexpr (E == Epi::kLogits) {
        if (ea.best) {
            return launch_pdl(k_splitk_reduce_logits_best, dim3(M), dim3(256), 0, s, sk.part,
                              sk.splits, M, N, bias, ea);
        }
    }
    if constexpr (E == Epi::kGelu || E == Epi::kStore) {
        // Whole 8-column chunks, 16-byte aligned partials, bias and destinations: the vector
        // fix-up (the split-K FFN1 of a decode lane).
        const bool aligned = (reinterpret_cast<uintptr_t>(sk.part) & 15) == 0 &&
                             (bias == nullptr || (reinterpret_cast<uintptr_t>(bias) & 15) == 0);
        if (N % 8 == 0 && aligned && M <= 65535 && host_vector_epilogue_ok(ea, N)) {
            const dim3 vgrid((N / 8 + 255) / 256, M);
            return launch_pdl(k_splitk_reduce_vec<E>, vgrid, dim3(256), 0, s, sk.part, sk.splits,
                              M, N, bias, ea);
        }
    }
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
        for (int variant = 0; variant < (BN == 64 ? 3 : 2); ++variant) {
            int smem = C::kSmem;
            switch (e) {
#define BST_GEMM_FN(EP)                                                                          \
    if (variant == 2) {                                                                          \
        fn = reinterpret_cast<const void*>(k_gemm_tc<FMT, BN, EP, BN == 64 ? 2 : 0>);            \
        smem = Config<FMT, BN, BN == 64 ? 2 : 0>::kSmem;                                         \
    } else {                                                                                     \
        fn = variant ? reinterpret_cast<const void*>(k_gemm_tc_persistent<FMT, BN, EP>)          \
                     : reinterpret_cast<const void*>(k_gemm_tc<FMT, BN, EP, 0>);                 \
    }                                                                                            \
    break
                case Epi::kStore: BST_GEMM_FN(Epi::kStore);
                case Epi::kGelu: BST_GEMM_FN(Epi::kGelu);
                case Epi::kResidual: BST_GEMM_FN(Epi::kResidual);
                case Epi::kResidualGelu: BST_GEMM_FN(Epi::kResidualGelu);
                case Epi::kQkv: BST_GEMM_FN(Epi::kQkv);
                case Epi::kLogits: BST_GEMM_FN(Epi::kLogits);
#undef BST_GEMM_FN
            }
            err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (err != cudaSuccess) return err;
        }
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
    // each split keeps at least four k-tiles (measured on the decode step against two, six and
    // eight: fewer partials to sum beats the shorter split GEMMs up to that point).
    const int tiles_m = (M + BM - 1) / BM;
    const int k_tiles = (K + (w_bf16 ? 63 : 31)) / (w_bf16 ? 64 : 32);
    auto plan = [&](int bn) {
        const int tiles = ((N + bn - 1) / bn) * tiles_m;
        int splits = 1;
        if (tiles < 148) {
            splits = std::min((148 + tiles - 1) / tiles, std::max(1, k_tiles / 4));
            const size_t per_split = static_cast<size_t>(M) * N * sizeof(float);
            while (splits > 1 && per_split * splits > part_bytes) --splits;
            if (splits > 1) {
                const int per = (k_tiles + splits - 1) / splits;
                splits = (k_tiles + per - 1) / per;  // no empty split
            }
        }
        return splits;
    };
    int bn = ((N + 127) / 128) * tiles_m >= 148 ? 128 : 64;
    int splits = plan(bn);
    // A decode lane's GEMM (one 128-row tile) whose 64-wide plan takes more than half the SMs:
    // 128-wide tiles halve its CTAs, so that the two decode lanes' GEMMs run in one wave (and
    // each activation tile is read by half as many CTAs).
    if (bn == 64 && tiles_m == 1 && N >= 128 && ((N + 63) / 64) * splits > 74) {
        bn = 128;
        splits = plan(bn);
        // ... and with fewer splits where even the 128-wide plan takes more than half the SMs
        // (the head of the V4096 model: 32 tiles x 4 splits -> x 2).
        const int tiles128 = (N + 127) / 128;
        while (splits > 1 && tiles128 * splits > 74) {
            const int per = (k_tiles + splits - 2) / (splits - 1);
            splits = (k_tiles + per - 1) / per;
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
    if (sk.splits > 1 && N % 4 == 0 && (reinterpret_cast<uintptr_t>(part) & 15) == 0) {
        if ((e = make_part_map(&sk.pmap, part, sk.splits, M, N)) != cudaSuccess) return e;
        sk.tma = 1;
    }
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
