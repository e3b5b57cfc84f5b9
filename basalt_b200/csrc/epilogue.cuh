// Epilogue stages shared by the projection kernels (kernels.cu, gemm_tc.cu).
#pragma once

#include <cuda_bf16.h>

#include "device.cuh"
#include "kernels.h"

namespace bst {

// gelu_forward (nn_ops.rs:130-137): 0.5x(1 + tanh(sqrt(2/pi)(x + 0.044715x^3))), evaluated in
// f32 in the reference's operation order without contraction.
__device__ __forceinline__ float gelu_ref(float v) {
    const float c = __fsqrt_rn(__fdiv_rn(2.0f, 3.14159274101257324f));
    const float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, v), v), v);
    const float inner = __fmul_rn(c, __fadd_rn(v, cube));
    return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(inner)));
}

// Stores v as the tensor-core operand split at element idx: planes = 1 writes the tf32 truncation
// and the fp32 remainder, planes = 2 two bf16 values (hi, and the rounded remainder).
__device__ __forceinline__ void store_split(float v, int planes, void* hi, void* lo, size_t idx) {
    if (planes == 1) {
        const float h = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
        static_cast<float*>(hi)[idx] = h;
        static_cast<float*>(lo)[idx] = __fsub_rn(v, h);
    } else {
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        static_cast<__nv_bfloat16*>(hi)[idx] = h;
        static_cast<__nv_bfloat16*>(lo)[idx] = __float2bfloat16_rn(__fsub_rn(v, __bfloat162float(h)));
    }
}

// Orders floats as unsigned integers (ascending), +0 and -0 equal; the low word prefers the
// smaller index, so the largest packed value over a row is TextEngine.argmax's first maximum
// (TextEngine.java:392-400). NaN scores are never packed: the reference never moves past index 0
// to a NaN, and a NaN at index 0 is handled by whoever reads the result.
__device__ __forceinline__ unsigned long long pack_best(float v, int idx) {
    if (v == 0.0f) v = 0.0f;
    const unsigned b = __float_as_uint(v);
    const unsigned ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (static_cast<unsigned long long>(ord) << 32) | (0xffffffffu - static_cast<unsigned>(idx));
}

__device__ __forceinline__ int unpack_best_index(unsigned long long b) {
    return static_cast<int>(0xffffffffu - static_cast<unsigned>(b));
}

template <Epi E>
__device__ __forceinline__ void epi_apply(const EpiArgs& ea, int m, int n, float v) {
    if constexpr (E == Epi::kStore) {
        ea.out[static_cast<size_t>(m) * ea.ldo + n] = v;
        if (ea.split.planes) {
            store_split(v, ea.split.planes, ea.split.hi, ea.split.lo, static_cast<size_t>(m) * ea.split.ld + n);
        }
    } else if constexpr (E == Epi::kGelu) {
        const float g = gelu_ref(v);
        if (ea.out) ea.out[static_cast<size_t>(m) * ea.ldo + n] = g;
        if (ea.split.planes) {
            store_split(g, ea.split.planes, ea.split.hi, ea.split.lo, static_cast<size_t>(m) * ea.split.ld + n);
        }
    } else if constexpr (E == Epi::kResidual) {
        float* p = ea.out + static_cast<size_t>(m) * ea.ldo + n;
        *p = __fadd_rn(*p, v);
    } else if constexpr (E == Epi::kResidualGelu) {
        ea.out[static_cast<size_t>(m) * ea.ldo + n] =
            gelu_ref(__fadd_rn(v, ea.res[static_cast<size_t>(m) * ea.ldr + n]));
    } else if constexpr (E == Epi::kQkv) {
        if (n < ea.d) {
            ea.out[static_cast<size_t>(m) * ea.ldo + n] = v;
        } else {
            const int which = n / ea.d;
            const int j = n - which * ea.d;
            const int h = j / ea.head_dim;
            const int e = j - h * ea.head_dim;
            const size_t idx =
                ((static_cast<size_t>(ea.rowmap[m]) * ea.heads + h) * ea.slots + ea.slot[m]) *
                    ea.head_dim + e;
            void* base = which == 1 ? ea.k_cache : ea.v_cache;
            if (ea.kv_bf16) {
                static_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v);
            } else {
                static_cast<float*>(base)[idx] = v;
            }
        }
    } else if constexpr (E == Epi::kLogits) {
        ea.out[static_cast<size_t>(ea.rowmap[m]) * ea.ldo + n] = v;
        if (ea.best && !isnan(v)) atomicMax(ea.best + ea.rowmap[m], pack_best(v, n));
    }
}

// Block-level LayerNorm of `rows` rows of x into out ([rows][d], shared memory), with the
// statistics of nn_ops.rs:168-199 (f64 mean and population variance, f32 affine). One row uses
// every warp of the block; several rows take one warp each.
__device__ __forceinline__ void layernorm_rows(const float* __restrict__ x, int ldx, int rows, int d,
                               const LnArgs& ln, float* __restrict__ out) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __shared__ double red[32];
    __shared__ double s_stat[2];
    if (rows == 1) {
        const int nwarps = static_cast<int>(blockDim.x >> 5);
        double s = 0.0;
        for (int k = threadIdx.x; k < d; k += blockDim.x) s = __dadd_rn(s, static_cast<double>(x[k]));
        s = warp_sum_d(s);
        if (lane == 0) red[warp] = s;
        __syncthreads();
        if (warp == 0) {
            const double t = warp_sum_d(lane < nwarps ? red[lane] : 0.0);
            if (lane == 0) s_stat[0] = __ddiv_rn(t, static_cast<double>(d));
        }
        __syncthreads();
        const double mean = s_stat[0];
        double v = 0.0;
        for (int k = threadIdx.x; k < d; k += blockDim.x) {
            const double delta = __dadd_rn(static_cast<double>(x[k]), -mean);
            v = __dadd_rn(v, __dmul_rn(delta, delta));
        }
        v = warp_sum_d(v);
        if (lane == 0) red[warp] = v;
        __syncthreads();
        if (warp == 0) {
            const double t = warp_sum_d(lane < nwarps ? red[lane] : 0.0);
            if (lane == 0) {
                const double variance = __ddiv_rn(t, static_cast<double>(d));
                s_stat[1] = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(variance, static_cast<double>(ln.eps))));
            }
        }
        __syncthreads();
        const double inverse = s_stat[1];
        for (int k = threadIdx.x; k < d; k += blockDim.x) {
            const float nrm = static_cast<float>(__dmul_rn(__dadd_rn(static_cast<double>(x[k]), -mean), inverse));
            out[k] = __fadd_rn(__fmul_rn(nrm, ln.gamma[k]), ln.beta[k]);
        }
        return;
    }
    if (warp >= rows) return;
    const float* xr = x + static_cast<size_t>(warp) * ldx;
    float* yr = out + static_cast<size_t>(warp) * d;
    double s = 0.0;
    for (int k = lane; k < d; k += 32) s = __dadd_rn(s, static_cast<double>(xr[k]));
    const double mean = __ddiv_rn(warp_sum_d(s), static_cast<double>(d));
    double v = 0.0;
    for (int k = lane; k < d; k += 32) {
        const double delta = __dadd_rn(static_cast<double>(xr[k]), -mean);
        v = __dadd_rn(v, __dmul_rn(delta, delta));
    }
    const double variance = __ddiv_rn(warp_sum_d(v), static_cast<double>(d));
    const double inverse = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(variance, static_cast<double>(ln.eps))));
    for (int k = lane; k < d; k += 32) {
        const float nrm = static_cast<float>(__dmul_rn(__dadd_rn(static_cast<double>(xr[k]), -mean), inverse));
        yr[k] = __fadd_rn(__fmul_rn(nrm, ln.gamma[k]), ln.beta[k]);
    }
}

}  // namespace bst
