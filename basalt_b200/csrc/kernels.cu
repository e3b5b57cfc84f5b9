// sm_100a kernels of the TextEngine decode path.
//
// Layouts (all row-major):
//   weights   projection matrices are stored K-major, [out, in] — the transpose of the
//             reference's Linear weight [in, out] (torch/Linear.java:20-27) — as float32 or bf16;
//   residual  float32 [tokens, d];
//   KV cache  per layer [rows][heads][slots][head_dim], float32 or bf16; a row's real tokens sit
//             in slots 0..len-1 with slot == position.
//
// Every kernel computes in float32 (LayerNorm statistics and the sampler in float64, as the
// reference does). Nothing here traps: invalid ids are rejected on the host before launch.

#include "kernels.h"
#include "device.cuh"
#include "epilogue.cuh"
#include "select.cuh"

#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

#include <mutex>

namespace bst {

const char* kernel_class_name(int cls) {
    static const char* names[kKernelClassCount] = {
        "embed",       "layernorm",     "gemv",          "gemm",
        "attn_decode", "attn_combine",  "attn_prefill",  "select_greedy",
        "select_sample", "gather",      "head_last_token", "misc",
        "split",       "decode_step",   "gemm_step"};
    return cls >= 0 && cls < kKernelClassCount ? names[cls] : "unknown";
}

namespace {

constexpr int kMaxChunk = 1024;
constexpr size_t kSampleSmemLimit = 200 * 1024;

// ---------------------------------------------------------------------------------------------
// GEMV for small M: each output column n is a dot product of W's row n (contiguous, K-major)
// with up to MT activation rows. KS warps split one column's K range; 8 / KS columns per CTA.
// Weights are constant, so each lane loads its first NV 16-byte weight vectors before waiting on
// the kernel that produces the activations: under programmatic dependent launch the weight
// stream of this projection overlaps the previous kernel. With ln.gamma set, the CTA first
// applies LayerNorm to its input rows (the pre-norm of TransformerBlock) in shared memory.
// ---------------------------------------------------------------------------------------------
template <typename WT, int MT, int KS, Epi E>
__global__ __launch_bounds__(256) void k_gemv(const float* __restrict__ x, int ldx,
                                              const WT* __restrict__ w,
                                              const float* __restrict__ bias, int M, int N,
                                              int K, LnArgs ln, EpiArgs ea) {
    constexpr int VEC = Vec16<WT>::N;
    constexpr int COLS = 8 / KS;
    constexpr int NV = 4;
    extern __shared__ float xs[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int col = warp / KS, part = warp % KS;
    const int n = blockIdx.x * COLS + col;
    const int m0 = blockIdx.y * MT;
    const int mcount = min(MT, M - m0);
    const bool vector_path = (K % VEC) == 0 && (ln.gamma != nullptr || (ldx % 4) == 0);
    const int nvec = K / VEC;
    const int per = (nvec + KS - 1) / KS;
    const int v0 = part * per, v1 = min(nvec, v0 + per);
    const WT* wr = w + static_cast<size_t>(min(n, N - 1)) * K;
    float wv[NV][VEC];
    if (vector_path && n < N) {
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int v = v0 + lane + 32 * j;
            if (v < v1) Vec16<WT>::load(wr + static_cast<size_t>(v) * VEC, wv[j]);
        }
    }
    pdl_trigger();
    pdl_wait();
    const float* xr = x + static_cast<size_t>(m0) * ldx;
    int ld = ldx;
    if (ln.gamma != nullptr) {
        layernorm_rows(xr, ldx, mcount, K, ln, xs);
        __syncthreads();
        xr = xs;
        ld = K;
    }
    float acc[MT];
#pragma unroll
    for (int i = 0; i < MT; ++i) acc[i] = 0.0f;
    auto fma_vec = [&](const float* wvec, int k) {
#pragma unroll
        for (int i = 0; i < MT; ++i) {
            if (i < mcount) {
                const float* xp = xr + static_cast<size_t>(i) * ld + k;
#pragma unroll
                for (int c = 0; c < VEC; c += 4) {
                    const float4 xv = *reinterpret_cast<const float4*>(xp + c);
                    acc[i] = fmaf(wvec[c], xv.x, acc[i]);
                    acc[i] = fmaf(wvec[c + 1], xv.y, acc[i]);
                    acc[i] = fmaf(wvec[c + 2], xv.z, acc[i]);
                    acc[i] = fmaf(wvec[c + 3], xv.w, acc[i]);
                }
            }
        }
    };
    if (n < N) {
        if (vector_path) {
#pragma unroll
            for (int j = 0; j < NV; ++j) {
                const int v = v0 + lane + 32 * j;
                if (v < v1) fma_vec(wv[j], v * VEC);
            }
#pragma unroll 4
            for (int v = v0 + lane + 32 * NV; v < v1; v += 32) {
                float wt[VEC];
                Vec16<WT>::load(wr + static_cast<size_t>(v) * VEC, wt);
                fma_vec(wt, v * VEC);
            }
        } else {
            const int kper = (K + KS - 1) / KS;
            const int k0 = part * kper, k1 = min(K, k0 + kper);
            for (int k = k0 + lane; k < k1; k += 32) {
                const float wk = to_f(wr[k]);
#pragma unroll
                for (int i = 0; i < MT; ++i) {
                    if (i < mcount) acc[i] = fmaf(wk, xr[static_cast<size_t>(i) * ld + k], acc[i]);
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < MT; ++i) acc[i] = warp_sum(acc[i]);
    __shared__ float red[8][MT];
    if (lane == 0) {
#pragma unroll
        for (int i = 0; i < MT; ++i) red[warp][i] = acc[i];
    }
    __syncthreads();
    if (part == 0 && lane < mcount && n < N) {
        float sum = 0.0f;
#pragma unroll
        for (int p = 0; p < KS; ++p) sum += red[col * KS + p][lane];
        const float v = bias ? __fadd_rn(sum, bias[n]) : sum;
        epi_apply<E>(ea, m0 + lane, n, v);
    }
}

// ---------------------------------------------------------------------------------------------
// Tiled FFMA GEMM for larger M: 128x128 tile, k-step 16, 8x8 outputs per thread, double-buffered
// shared tiles. A is float32 [M, K]; B is [N, K] (float32 or bf16, converted on load).
// Requires K % 16 == 0.
// ---------------------------------------------------------------------------------------------
template <typename WT, Epi E>
__global__ __launch_bounds__(256) void k_gemm(const float* __restrict__ a, int lda,
                                              const WT* __restrict__ b,
                                              const float* __restrict__ bias, int M, int N,
                                              int K, EpiArgs ea) {
    pdl_trigger();
    pdl_wait();
    constexpr int BM = 128, BN = 128, BK = 16, PAD = 4;
    __shared__ __align__(16) float As[2][BK][BM + PAD];
    __shared__ __align__(16) float Bs[2][BK][BN + PAD];
    const int tid = threadIdx.x;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int tx = tid & 15, ty = tid >> 4;

    float4 ra[2];
    float rb[8];
    auto load_tile = [&](int k0) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int idx = tid + 256 * i;
            const int row = idx >> 2, kq = idx & 3;
            const int m = m0 + row;
            ra[i] = m < M ? *reinterpret_cast<const float4*>(a + static_cast<size_t>(m) * lda +
                                                             k0 + kq * 4)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if constexpr (sizeof(WT) == 4) {
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int idx = tid + 256 * i;
                const int row = idx >> 2, kq = idx & 3;
                const int n = n0 + row;
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (n < N) {
                    v = __ldg(reinterpret_cast<const float4*>(
                        reinterpret_cast<const float*>(b) + static_cast<size_t>(n) * K + k0 +
                        kq * 4));
                }
                rb[4 * i] = v.x; rb[4 * i + 1] = v.y; rb[4 * i + 2] = v.z; rb[4 * i + 3] = v.w;
            }
        } else {
            const int row = tid >> 1, kh = tid & 1;
            const int n = n0 + row;
            if (n < N) {
                Vec16<WT>::load(b + static_cast<size_t>(n) * K + k0 + kh * 8, rb);
            } else {
#pragma unroll
                for (int c = 0; c < 8; ++c) rb[c] = 0.0f;
            }
        }
    };
    auto store_tile = [&](int buf) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int idx = tid + 256 * i;
            const int row = idx >> 2, kq = idx & 3;
            As[buf][kq * 4 + 0][row] = ra[i].x;
            As[buf][kq * 4 + 1][row] = ra[i].y;
            As[buf][kq * 4 + 2][row] = ra[i].z;
            As[buf][kq * 4 + 3][row] = ra[i].w;
        }
        if constexpr (sizeof(WT) == 4) {
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int idx = tid + 256 * i;
                const int row = idx >> 2, kq = idx & 3;
#pragma unroll
                for (int c = 0; c < 4; ++c) Bs[buf][kq * 4 + c][row] = rb[4 * i + c];
            }
        } else {
            const int row = tid >> 1, kh = tid & 1;
#pragma unroll
            for (int c = 0; c < 8; ++c) Bs[buf][kh * 8 + c][row] = rb[c];
        }
    };

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

    load_tile(0);
    store_tile(0);
    __syncthreads();
    for (int k0 = 0; k0 < K; k0 += BK) {
        const int buf = (k0 / BK) & 1;
        const bool more = k0 + BK < K;
        if (more) load_tile(k0 + BK);
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
            const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        if (more) store_tile(buf ^ 1);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
            if (n >= N) continue;
            const float v = bias ? __fadd_rn(acc[i][j], bias[n]) : acc[i][j];
            epi_apply<E>(ea, m, n, v);
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Embedding gathers.
// ---------------------------------------------------------------------------------------------
template <typename WT>
__global__ void k_embed_tokens(const WT* __restrict__ tok, const WT* __restrict__ pos,
                               const int* __restrict__ ids, const int* __restrict__ positions,
                               float* __restrict__ x, int d) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x;
    const size_t id = static_cast<size_t>(ids[t]);
    const size_t p = static_cast<size_t>(positions[t]);
    for (int e = threadIdx.x; e < d; e += blockDim.x) {
        x[static_cast<size_t>(t) * d + e] = __fadd_rn(to_f(tok[id * d + e]), to_f(pos[p * d + e]));
    }
}

template <typename WT>
__global__ void k_embed_decode(const WT* __restrict__ tok, const WT* __restrict__ pos,
                               const int* __restrict__ rowmap, const int* __restrict__ next,
                               int* __restrict__ len, int* __restrict__ slot,
                               float* __restrict__ x, int d) {
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x;
    const int row = rowmap[i];
    __shared__ int s_slot;
    if (threadIdx.x == 0) s_slot = len[row];
    __syncthreads();
    const int sl = s_slot;
    const size_t id = static_cast<size_t>(next[row]);
    for (int e = threadIdx.x; e < d; e += blockDim.x) {
        x[static_cast<size_t>(i) * d + e] =
            __fadd_rn(to_f(tok[id * d + e]), to_f(pos[static_cast<size_t>(sl) * d + e]));
    }
    if (threadIdx.x == 0) {
        slot[i] = sl;
        len[row] = sl + 1;
    }
}

template <typename WT>
__global__ void k_window_embed(const int* __restrict__ window, int W, const WT* __restrict__ emb,
                               int d, float* __restrict__ x) {
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x;
    for (int idx = threadIdx.x; idx < W * d; idx += blockDim.x) {
        const int t = idx / d, e = idx - t * d;
        const size_t id = static_cast<size_t>(window[static_cast<size_t>(r) * W + t]);
        x[static_cast<size_t>(r) * W * d + idx] = to_f(emb[id * d + e]);
    }
}

__global__ void k_last_token(const int* __restrict__ window, int W, const float* __restrict__ w,
                             const float* __restrict__ bias, int V, float* __restrict__ logits) {
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x;
    const int token = window[static_cast<size_t>(r) * W + W - 1];
    const int t = ((token % V) + V) % V;  // Math.floorMod
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
        logits[static_cast<size_t>(r) * V + v] =
            __fadd_rn(w[static_cast<size_t>(t) * V + v], bias[v]);
    }
}

__global__ void k_prefill_tokens(const int* __restrict__ window, int W,
                                 const int* __restrict__ seg_row, const int* __restrict__ seg_npad,
                                 const int* __restrict__ seg_start, const int* __restrict__ seg_len,
                                 int pad_id, int* __restrict__ ids, int* __restrict__ positions,
                                 int* __restrict__ tok_row, int* __restrict__ len) {
    pdl_trigger();
    pdl_wait();
    const int j = blockIdx.x;
    const int row = seg_row[j], npad = seg_npad[j], start = seg_start[j], n = seg_len[j];
    for (int t = threadIdx.x; t < n; t += blockDim.x) {
        ids[start + t] = npad >= W ? pad_id : window[static_cast<size_t>(row) * W + npad + t];
        positions[start + t] = t;
        tok_row[start + t] = row;
    }
    if (threadIdx.x == 0) len[row] = n;
}

__global__ void k_gather_last(const float* __restrict__ x, const int* __restrict__ seg_start,
                              const int* __restrict__ seg_len, int d, float* __restrict__ last) {
    pdl_trigger();
    pdl_wait();
    const int j = blockIdx.x;
    const size_t src = static_cast<size_t>(seg_start[j] + seg_len[j] - 1) * d;
    for (int e = threadIdx.x; e < d; e += blockDim.x) last[static_cast<size_t>(j) * d + e] = x[src + e];
}

// Decode step begin fused with the first layer's LayerNorm: one CTA of 128 threads per row
// embeds the row's next token at its slot (as k_embed_decode), then normalises the row with f64
// statistics (as k_reduce_residual_ln, nn_ops.rs:168-199) straight into the QKV projection's
// operand planes.
template <typename WT, int EPT>
__global__ __launch_bounds__(128) void k_embed_ln_decode(
    const WT* __restrict__ tok, const WT* __restrict__ pos, const int* __restrict__ rowmap,
    const int* __restrict__ next, int* __restrict__ len, int* __restrict__ slot,
    float* __restrict__ x, int d, const float* __restrict__ gamma, const float* __restrict__ beta,
    float eps, void* __restrict__ hi, void* __restrict__ lo, int planes) {
    __shared__ double red[4];
    __shared__ double stat;
    __shared__ int s_slot, s_id;
    const int i = blockIdx.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // LayerNorm parameters are weights: read before the wait.
    float gv[EPT], tv[EPT];
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
        const int n = tid + 128 * j;
        gv[j] = n < d ? gamma[n] : 0.0f;
        tv[j] = n < d ? beta[n] : 0.0f;
    }
    pdl_trigger();
    pdl_wait();
    if (tid == 0) {
        const int row = rowmap[i];
        s_slot = len[row];
        s_id = next[row];
    }
    __syncthreads();
    const int sl = s_slot;
    const size_t id = static_cast<size_t>(s_id);
    float v[EPT];
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
        const int n = tid + 128 * j;
        v[j] = n < d ? __fadd_rn(to_f(tok[id * d + n]), to_f(pos[static_cast<size_t>(sl) * d + n]))
                     : 0.0f;
        if (n < d) x[static_cast<size_t>(i) * d + n] = v[j];
    }
    if (tid == 0) {
        slot[i] = sl;
        len[rowmap[i]] = sl + 1;
    }
    double s = 0.0;
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
        if (tid + 128 * j < d) s = __dadd_rn(s, static_cast<double>(v[j]));
    }
    s = warp_sum_d(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (tid == 0) stat = __ddiv_rn(__dadd_rn(__dadd_rn(red[0], red[1]), __dadd_rn(red[2], red[3])),
                                   static_cast<double>(d));
    __syncthreads();
    const double mean = stat;
    double q = 0.0;
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
        if (tid + 128 * j < d) {
            const double delta = __dadd_rn(static_cast<double>(v[j]), -mean);
            q = __dadd_rn(q, __dmul_rn(delta, delta));
        }
    }
    q = warp_sum_d(q);
    __syncthreads();
    if (lane == 0) red[warp] = q;
    __syncthreads();
    if (tid == 0) {
        const double variance = __ddiv_rn(__dadd_rn(__dadd_rn(red[0], red[1]), __dadd_rn(red[2], red[3])),
                                          static_cast<double>(d));
        stat = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(variance, static_cast<double>(eps))));
    }
    __syncthreads();
    const double inverse = stat;
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
        const int n = tid + 128 * j;
        if (n < d) {
            const float normalized =
                static_cast<float>(__dmul_rn(__dadd_rn(static_cast<double>(v[j]), -mean), inverse));
            const float out = __fadd_rn(__fmul_rn(normalized, gv[j]), tv[j]);
            store_split(out, planes, hi, lo, static_cast<size_t>(i) * d + n);
        }
    }
}

// ---------------------------------------------------------------------------------------------
// LayerNorm (nn_ops.rs:168-199): one warp per row; mean and population variance in f64, the
// normalised value rounded to f32, then f32 n * gamma + beta.
// ---------------------------------------------------------------------------------------------
__global__ __launch_bounds__(256) void k_layernorm(const float* __restrict__ x, int ldx,
                                                   const float* __restrict__ gamma,
                                                   const float* __restrict__ beta,
                                                   float* __restrict__ y, int ldy, int rows, int d,
                                                   float eps, void* __restrict__ hi,
                                                   void* __restrict__ lo, int planes) {
    pdl_trigger();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + warp;
    if (row >= rows) return;
    const float* xr = x + static_cast<size_t>(row) * ldx;
    float* yr = y ? y + static_cast<size_t>(row) * ldy : nullptr;
    double s = 0.0;
    for (int i = lane; i < d; i += 32) s = __dadd_rn(s, static_cast<double>(xr[i]));
    const double mean = __ddiv_rn(warp_sum_d(s), static_cast<double>(d));
    double v = 0.0;
    for (int i = lane; i < d; i += 32) {
        const double delta = __dadd_rn(static_cast<double>(xr[i]), -mean);
        v = __dadd_rn(v, __dmul_rn(delta, delta));
    }
    const double variance = __ddiv_rn(warp_sum_d(v), static_cast<double>(d));
    const double inverse = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(variance, static_cast<double>(eps))));
    for (int i = lane; i < d; i += 32) {
        const float normalized =
            static_cast<float>(__dmul_rn(__dadd_rn(static_cast<double>(xr[i]), -mean), inverse));
        const float out = __fadd_rn(__fmul_rn(normalized, gamma[i]), beta[i]);
        if (y) yr[i] = out;
        if (planes) store_split(out, planes, hi, lo, static_cast<size_t>(row) * d + i);
    }
}

// Split-K fix-up of a residual projection, then the LayerNorm of the updated rows into operand
// planes (see launch_reduce_residual_ln). One CTA of 128 threads per row; a thread owns EPT
// columns (n = tid + 128 j) and loads their partials of up to ZB splits at once, together with
// the residual row (bias, gamma and beta are read before the PDL wait). The splits are summed in
// order as k_splitk_reduce does; the f64 statistics are k_layernorm's up to the order of the f64
// additions. ZB is the launch's split count rounded up (4, 8 or 16), so that the registers
// holding loads in flight stay few enough for several CTAs per SM.
template <int EPT, int ZB>
__global__ __launch_bounds__(128) void k_reduce_residual_ln(
    const float* __restrict__ part, int splits, int M, int N, const float* __restrict__ bias,
    float* __restrict__ x, int ldx, const float* __restrict__ gamma, const float* __restrict__ beta,
    float eps, void* __restrict__ hi, void* __restrict__ lo, int planes) {
    __shared__ double red[4];
    __shared__ double stat;
    const int m = blockIdx.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t total = static_cast<size_t>(M) * N;
    float* xr = x + static_cast<size_t>(m) * ldx;
    const float* pr = part + static_cast<size_t>(m) * N;
    // Bias and LayerNorm parameters are weights: read before the wait, while the GEMM drains.
    float bv[EPT], gv[EPT], tv[EPT];
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
        const int n = tid + 128 * j;
        bv[j] = bias && n < N ? bias[n] : 0.0f;
        gv[j] = n < N ? gamma[n] : 0.0f;
        tv[j] = n < N ? beta[n] : 0.0f;
    }
    pdl_trigger();
    pdl_wait();
    // The residual row loads with the first batch of partial sums.
    float xv[EPT];
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
        const int n = tid + 128 * j;
        xv[j] = n < N ? xr[n] : 0.0f;
    }
    float v[EPT];
#pragma unroll
    for (int j = 0; j < EPT; ++j) v[j] = 0.0f;
    for (int z0 = 0; z0 < splits; z0 += ZB) {
        float t[EPT][ZB];
#pragma unroll
        for (int j = 0; j < EPT; ++j) {
            const int n = min(tid + 128 * j, N - 1);
#pragma unroll
            for (int z = 0; z < ZB; ++z) {
                t[j][z] = z0 + z < splits ? pr[static_cast<size_t>(z0 + z) * total + n] : 0.0f;
            }
        }
#pragma unroll
        for (int j = 0; j < EPT; ++j) {
#pragma unroll
            for (int z = 0; z < ZB; ++z) {
                if (z0 + z < splits) v[j] += t[j][z];
            }
        }
    }
    // v = sum of splits; the residual add in the order of the kResidual epilogue
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
        const int n = tid + 128 * j;
        if (n < N) {
            const float value = bias ? __fadd_rn(v[j], bv[j]) : v[j];
            v[j] = __fadd_rn(xv[j], value);
            xr[n] = v[j];
        }
    }
    // f64 statistics over the row: per-thread partial sums, then the block
    double s = 0.0;
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
        if (tid + 128 * j < N) s = __dadd_rn(s, static_cast<double>(v[j]));
    }
    s = warp_sum_d(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (tid == 0) stat = __ddiv_rn(__dadd_rn(__dadd_rn(red[0], red[1]), __dadd_rn(red[2], red[3])),
                                   static_cast<double>(N));
    __syncthreads();
    const double mean = stat;
    double q = 0.0;
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
        if (tid + 128 * j < N) {
            const double delta = __dadd_rn(static_cast<double>(v[j]), -mean);
            q = __dadd_rn(q, __dmul_rn(delta, delta));
        }
    }
    q = warp_sum_d(q);
    __syncthreads();
    if (lane == 0) red[warp] = q;
    __syncthreads();
    if (tid == 0) {
        const double variance = __ddiv_rn(__dadd_rn(__dadd_rn(red[0], red[1]), __dadd_rn(red[2], red[3])),
                                          static_cast<double>(N));
        stat = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(variance, static_cast<double>(eps))));
    }
    __syncthreads();
    const double inverse = stat;
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
        const int n = tid + 128 * j;
        if (n < N) {
            const float normalized =
                static_cast<float>(__dmul_rn(__dadd_rn(static_cast<double>(v[j]), -mean), inverse));
            const float out = __fadd_rn(__fmul_rn(normalized, gv[j]), tv[j]);
            store_split(out, planes, hi, lo, static_cast<size_t>(m) * N + n);
        }
    }
}


// Streaming loads for the decode attention's K/V: read once per step, so they are marked
// evict-first in L2 (the projections' weights and split-K partials stay resident instead).
__device__ __forceinline__ unsigned long long evict_first_policy() {
    unsigned long long pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void load16_stream(const float* p, float* out, unsigned long long pol) {
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=f"(out[0]), "=f"(out[1]), "=f"(out[2]), "=f"(out[3])
                 : "l"(p), "l"(pol));
}
__device__ __forceinline__ void load16_stream(const __nv_bfloat16* p, float* out,
                                              unsigned long long pol) {
    uint32_t w[4];
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.b32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
                 : "l"(p), "l"(pol));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        out[2 * i] = bf16_bits_to_f(w[i] & 0xffffu);
        out[2 * i + 1] = bf16_bits_to_f(w[i] >> 16);
    }
}
// DPL consecutive values (DPL = 1, 2 or 4) of a V row, streaming.
template <int DPL>
__device__ __forceinline__ void load_row_stream(const float* p, float* out, unsigned long long pol) {
    if constexpr (DPL == 4) {
        load16_stream(p, out, pol);
    } else if constexpr (DPL == 2) {
        asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.f32 {%0, %1}, [%2], %3;"
                     : "=f"(out[0]), "=f"(out[1]) : "l"(p), "l"(pol));
    } else {
        asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.f32 %0, [%1], %2;"
                     : "=f"(out[0]) : "l"(p), "l"(pol));
    }
}
template <int DPL>
__device__ __forceinline__ void load_row_stream(const __nv_bfloat16* p, float* out,
                                                unsigned long long pol) {
    if constexpr (DPL == 4) {
        uint32_t w[2];
        asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.b32 {%0, %1}, [%2], %3;"
                     : "=r"(w[0]), "=r"(w[1]) : "l"(p), "l"(pol));
        out[0] = bf16_bits_to_f(w[0] & 0xffffu); out[1] = bf16_bits_to_f(w[0] >> 16);
        out[2] = bf16_bits_to_f(w[1] & 0xffffu); out[3] = bf16_bits_to_f(w[1] >> 16);
    } else if constexpr (DPL == 2) {
        uint32_t w;
        asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.b32 %0, [%1], %2;"
                     : "=r"(w) : "l"(p), "l"(pol));
        out[0] = bf16_bits_to_f(w & 0xffffu); out[1] = bf16_bits_to_f(w >> 16);
    } else {
        unsigned short h;
        asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.b16 %0, [%1], %2;"
                     : "=h"(h) : "l"(p), "l"(pol));
        out[0] = bf16_bits_to_f(h);
    }
}

// ---------------------------------------------------------------------------------------------
// Decode attention, split over the cached keys. One CTA per (row, head, split); writes the
// split's running max, sum of exponentials and unnormalised output. Scores follow
// MultiheadAttention.forward (MultiheadAttention.java:57-82): dot(q, k) then * scale (f32).
// ---------------------------------------------------------------------------------------------
template <typename KT, int HD>
__global__ __launch_bounds__(128) void k_attn_decode(
    const float* __restrict__ q, const KT* __restrict__ kc, const KT* __restrict__ vc,
    const int* __restrict__ rowmap, const int* __restrict__ len, int heads, int slots,
    float scale, int splits, int chunk, float* __restrict__ part, int* __restrict__ tickets,
    float* __restrict__ out, PlaneOut po, QkvParts qp) {
    constexpr int EPV = Vec16<KT>::N;
    constexpr int LPK = HD / EPV;  // lanes per key
    constexpr int KPW = 32 / LPK;  // keys per warp step
    constexpr int DPL = HD / 32;   // output dims per lane
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x / heads, h = blockIdx.x % heads, sp = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row = rowmap[i];
    const int T = len[row];
    const int start = sp * chunk, end = min(T, start + chunk);
    const int n = max(0, end - start);
    const int d = heads * HD;
    __shared__ float qs[HD];
    __shared__ float sc[kMaxChunk];
    __shared__ float red[4 * HD];
    __shared__ float stat[8];
    __shared__ int s_last;
    const size_t base = (static_cast<size_t>(row) * heads + h) * slots + start;
    const unsigned long long pol = evict_first_policy();
    // With the QKV partial sums, the split holding slot T - 1 (this step's own token) takes that
    // key and value from shared memory and appends them to the cache; it never reads the slot
    // back, so every cache read stays on the read-only path.
    __shared__ float knew[HD], vnew[HD];
    const bool owner = qp.part && n > 0 && end == T;
    const int n_glob = owner ? n - 1 : n;  // keys read from the cache
    if (qp.part) {
        // The QKV projection's split-K fix-up for this (row, head), in split order then the
        // bias (as k_splitk_reduce sums it).
        const int R = gridDim.x / heads;
        const size_t plane = static_cast<size_t>(R) * 3 * d;
        const float* src = qp.part + static_cast<size_t>(i) * 3 * d;
        for (int e = tid; e < (owner ? 3 : 1) * HD; e += 128) {
            const int which = e / HD, ee = e - which * HD;
            const int col = which * d + h * HD + ee;
            // Up to 8 splits' loads in flight, then summed in split order.
            float t[8];
#pragma unroll
            for (int z = 0; z < 8; ++z) t[z] = z < qp.splits ? __ldcg(src + z * plane + col) : 0.0f;
            float v = 0.0f;
#pragma unroll
            for (int z = 0; z < 8; ++z) {
                if (z < qp.splits) v += t[z];
            }
            for (int z = 8; z < qp.splits; ++z) v += __ldcg(src + z * plane + col);
            if (qp.bias) v = __fadd_rn(v, qp.bias[col]);
            if (which == 0) {
                qs[ee] = v;
            } else {
                // The cache holds KT; attention uses the stored (rounded) value, as a read
                // would return it.
                KT* dst = const_cast<KT*>(which == 1 ? kc : vc) + (base + (n - 1)) * HD + ee;
                float stored;
                if constexpr (sizeof(KT) == 2) {
                    *dst = __float2bfloat16_rn(v);
                    stored = __bfloat162float(*dst);
                } else {
                    *dst = v;
                    stored = v;
                }
                (which == 1 ? knew : vnew)[ee] = stored;
            }
        }
    } else {
        for (int e = tid; e < HD; e += 128) qs[e] = q[static_cast<size_t>(i) * d + h * HD + e];
    }
    __syncthreads();
    const int sub = lane % LPK, kk = lane / LPK;
    // Scores: U key groups per round, their 16-byte loads all in flight before any is used
    // (32 floats per lane).
    constexpr int U = 32 / EPV;
    for (int j0 = warp * KPW; j0 < n; j0 += 4 * KPW * U) {
        float kv[U][EPV];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = j0 + u * 4 * KPW + kk;
            if (j < n_glob) {
                load16_stream(kc + (base + j) * HD + sub * EPV, kv[u], pol);
            } else if (j < n) {
#pragma unroll
                for (int c = 0; c < EPV; ++c) kv[u][c] = knew[sub * EPV + c];
            } else {
#pragma unroll
                for (int c = 0; c < EPV; ++c) kv[u][c] = 0.0f;
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = j0 + u * 4 * KPW + kk;
            float dot = 0.0f;
#pragma unroll
            for (int c = 0; c < EPV; ++c) dot = fmaf(kv[u][c], qs[sub * EPV + c], dot);
#pragma unroll
            for (int o = LPK / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(kFull, dot, o);
            if (sub == 0 && j < n) sc[j] = __fmul_rn(dot, scale);
        }
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int j = tid; j < n; j += 128) mx = fmaxf(mx, sc[j]);
    mx = warp_max(mx);
    if (lane == 0) stat[warp] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(stat[0], stat[1]), fmaxf(stat[2], stat[3]));
    float sum = 0.0f;
    for (int j = tid; j < n; j += 128) {
        const float p = expf(sc[j] - mx);
        sc[j] = p;
        sum += p;
    }
    sum = warp_sum(sum);
    __syncthreads();
    if (lane == 0) stat[4 + warp] = sum;
    __syncthreads();
    sum = stat[4] + stat[5] + stat[6] + stat[7];
    // Weighted values: each warp takes every 4th key, UV keys per round with their loads issued
    // before the multiply-adds (up to 32 floats per lane).
    constexpr int UV = 32 / DPL < 16 ? 32 / DPL : 16;
    float o[DPL];
#pragma unroll
    for (int c = 0; c < DPL; ++c) o[c] = 0.0f;
    for (int j0 = warp; j0 < n; j0 += 4 * UV) {
        float vv[UV][DPL];
#pragma unroll
        for (int u = 0; u < UV; ++u) {
            const int j = j0 + 4 * u;
            const int jj = min(j, n - 1);
            if (jj < n_glob) {
                load_row_stream<DPL>(vc + (base + jj) * HD + lane * DPL, vv[u], pol);
            } else {
#pragma unroll
                for (int c = 0; c < DPL; ++c) vv[u][c] = vnew[lane * DPL + c];
            }
        }
#pragma unroll
        for (int u = 0; u < UV; ++u) {
            const int j = j0 + 4 * u;
            const float p = j < n ? sc[j] : 0.0f;
#pragma unroll
            for (int c = 0; c < DPL; ++c) o[c] = fmaf(p, vv[u][c], o[c]);
        }
    }
#pragma unroll
    for (int c = 0; c < DPL; ++c) red[warp * HD + lane * DPL + c] = o[c];
    __syncthreads();
    if (splits == 1) {
        for (int e = tid; e < HD; e += 128) {
            const float acc = red[e] + red[HD + e] + red[2 * HD + e] + red[3 * HD + e];
            const size_t at = static_cast<size_t>(i) * d + h * HD + e;
            if (out) out[at] = acc / sum;
            if (po.planes) store_split(acc / sum, po.planes, po.hi, po.lo, at);
        }
        return;
    }
    // Several splits: publish this split's (output, max, sum); the last split of the head to
    // finish merges all of them in split order and re-arms the ticket.
    float* mine = part + (static_cast<size_t>(i * heads + h) * splits + sp) * (HD + 2);
    for (int e = tid; e < HD; e += 128) mine[e] = red[e] + red[HD + e] + red[2 * HD + e] + red[3 * HD + e];
    if (tid == 0) {
        mine[HD] = n > 0 ? mx : -INFINITY;
        mine[HD + 1] = n > 0 ? sum : 0.0f;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&tickets[i * heads + h], 1) == splits - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float* all = part + static_cast<size_t>(i * heads + h) * splits * (HD + 2);
    float M = -INFINITY;
    for (int z = 0; z < splits; ++z) M = fmaxf(M, __ldcg(all + z * (HD + 2) + HD));
    for (int e = tid; e < HD; e += 128) {
        float L = 0.0f, O = 0.0f;
        for (int z = 0; z < splits; ++z) {
            const float mz = __ldcg(all + z * (HD + 2) + HD);
            if (mz == -INFINITY) continue;
            const float wgt = expf(mz - M);
            L = fmaf(__ldcg(all + z * (HD + 2) + HD + 1), wgt, L);
            O = fmaf(__ldcg(all + z * (HD + 2) + e), wgt, O);
        }
        const size_t at = static_cast<size_t>(i) * d + h * HD + e;
        if (out) out[at] = O / L;
        if (po.planes) store_split(O / L, po.planes, po.hi, po.lo, at);
    }
    if (tid == 0) tickets[i * heads + h] = 0;
}

// ---------------------------------------------------------------------------------------------
// Causal prefill attention over one row's freshly written cache slots. CTA = (segment, head,
// tile of 64 queries), 256 threads; keys stream through shared memory 64 at a time with an online
// softmax. Register tiling: thread (ty, tx) = (tid / 16, tid % 16) owns queries 4ty..4ty+3 of the
// tile, their scores against keys 4tx..4tx+3 of the chunk, and output columns 64c + 4tx..+3
// (HD >= 64) or 2tx, 2tx+1 (HD = 32). Shared memory holds Q and K transposed ([e][query|key]) so
// both score operands are float4 reads, V as [key][e], and the probabilities transposed
// ([key][query]) with the query group XOR-swizzled by key / 4, which makes the 16 float4 stores
// of a half warp hit distinct bank groups.
// ---------------------------------------------------------------------------------------------
constexpr int kPrefillTile = 64;

template <int HD>
constexpr int attn_prefill_smem() {
    return (3 * HD * kPrefillTile + kPrefillTile * kPrefillTile) * static_cast<int>(sizeof(float));
}

__device__ __forceinline__ float4 load4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 load4(const __nv_bfloat16* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    return make_float4(bf16_bits_to_f(u.x & 0xffffu), bf16_bits_to_f(u.x >> 16),
                       bf16_bits_to_f(u.y & 0xffffu), bf16_bits_to_f(u.y >> 16));
}

template <typename KT, int HD>
__global__ __launch_bounds__(256, HD > 64 ? 2 : 3) void k_attn_prefill(
    const float* __restrict__ q, const KT* __restrict__ kc, const KT* __restrict__ vc,
    const int* __restrict__ seg_row, const int* __restrict__ seg_start,
    const int* __restrict__ seg_len, int heads, int slots, float scale, float* __restrict__ out,
    PlaneOut po) {
    pdl_trigger();
    pdl_wait();
    constexpr int T = kPrefillTile;
    constexpr int OC = HD / 16;  // output columns per thread
    extern __shared__ __align__(16) float smem_f[];
    float* Qt = smem_f;         // [HD][T]
    float* Kt = Qt + HD * T;    // [HD][T]
    float* Vs = Kt + HD * T;    // [T][HD]
    float* Pt = Vs + T * HD;    // [T][T], swizzled
    const int j = blockIdx.x, h = blockIdx.y, t0 = blockIdx.z * T;
    const int n = seg_len[j];
    if (t0 >= n) return;
    const int row = seg_row[j], start = seg_start[j], d = heads * HD;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;

    // Q tile, transposed; lanes run along queries so the transposed stores are conflict-free.
    for (int idx = tid; idx < T * (HD / 4); idx += 256) {
        const int r = idx % T, e4 = idx / T;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (t0 + r < n) v = load4(q + static_cast<size_t>(start + t0 + r) * d + h * HD + 4 * e4);
        Qt[(4 * e4 + 0) * T + r] = v.x;
        Qt[(4 * e4 + 1) * T + r] = v.y;
        Qt[(4 * e4 + 2) * T + r] = v.z;
        Qt[(4 * e4 + 3) * T + r] = v.w;
    }
    float m[4], l[4], o[4][OC];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
#pragma unroll
        for (int c = 0; c < OC; ++c) o[i][c] = 0.0f;
    }
    const size_t base = (static_cast<size_t>(row) * heads + h) * slots;
    const int kend = min(n, t0 + T);
    for (int kb = 0; kb < kend; kb += T) {
        __syncthreads();  // the previous chunk's K, V and P are no longer read
        for (int idx = tid; idx < T * (HD / 4); idx += 256) {
            const int r = idx % T, e4 = idx / T;
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (kb + r < n) v = load4(kc + (base + kb + r) * HD + 4 * e4);
            Kt[(4 * e4 + 0) * T + r] = v.x;
            Kt[(4 * e4 + 1) * T + r] = v.y;
            Kt[(4 * e4 + 2) * T + r] = v.z;
            Kt[(4 * e4 + 3) * T + r] = v.w;
        }
        for (int idx = tid; idx < T * (HD / 4); idx += 256) {
            const int e4 = idx % (HD / 4), r = idx / (HD / 4);
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (kb + r < n) v = load4(vc + (base + kb + r) * HD + 4 * e4);
            *reinterpret_cast<float4*>(Vs + r * HD + 4 * e4) = v;
        }
        __syncthreads();

        float sc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) sc[i][jj] = 0.0f;
        }
#pragma unroll 8
        for (int e = 0; e < HD; ++e) {
            const float4 qa = *reinterpret_cast<const float4*>(Qt + e * T + 4 * ty);
            const float4 ka = *reinterpret_cast<const float4*>(Kt + e * T + 4 * tx);
            const float qv[4] = {qa.x, qa.y, qa.z, qa.w};
            const float kv[4] = {ka.x, ka.y, ka.z, ka.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) sc[i][jj] = fmaf(qv[i], kv[jj], sc[i][jj]);
            }
        }

        // Online softmax per query row; a row's 64 scores live in the 16 lanes sharing ty.
        float p[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int t = t0 + 4 * ty + i;
            float mx = -INFINITY;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const int key = kb + 4 * tx + jj;
                sc[i][jj] = (t < n && key <= t) ? __fmul_rn(sc[i][jj], scale) : -INFINITY;
                mx = fmaxf(mx, sc[i][jj]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, off));
            const float mnew = fmaxf(m[i], mx);
            float corr = 1.0f, ps = 0.0f;
            if (mnew == -INFINITY) {
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) p[i][jj] = 0.0f;
            } else {
                corr = m[i] == -INFINITY ? 0.0f : expf(m[i] - mnew);
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    p[i][jj] = sc[i][jj] == -INFINITY ? 0.0f : expf(sc[i][jj] - mnew);
                    ps += p[i][jj];
                }
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) ps += __shfl_xor_sync(kFull, ps, off);
            l[i] = l[i] * corr + ps;
#pragma unroll
            for (int c = 0; c < OC; ++c) o[i][c] *= corr;
            m[i] = mnew;
        }
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const int k = 4 * tx + jj;
            *reinterpret_cast<float4*>(Pt + k * T + ((ty ^ (k >> 2)) << 2)) =
                make_float4(p[0][jj], p[1][jj], p[2][jj], p[3][jj]);
        }
        __syncthreads();

        const int kn = min(T, kend - kb);
#pragma unroll 4
        for (int k = 0; k < kn; ++k) {
            const float4 pa = *reinterpret_cast<const float4*>(Pt + k * T + ((ty ^ (k >> 2)) << 2));
            const float pv[4] = {pa.x, pa.y, pa.z, pa.w};
            if constexpr (HD == 32) {
                const float2 vb = *reinterpret_cast<const float2*>(Vs + k * HD + 2 * tx);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    o[i][0] = fmaf(pv[i], vb.x, o[i][0]);
                    o[i][1] = fmaf(pv[i], vb.y, o[i][1]);
                }
            } else {
#pragma unroll
                for (int c4 = 0; c4 < HD / 64; ++c4) {
                    const float4 vb = *reinterpret_cast<const float4*>(Vs + k * HD + 64 * c4 + 4 * tx);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        o[i][4 * c4 + 0] = fmaf(pv[i], vb.x, o[i][4 * c4 + 0]);
                        o[i][4 * c4 + 1] = fmaf(pv[i], vb.y, o[i][4 * c4 + 1]);
                        o[i][4 * c4 + 2] = fmaf(pv[i], vb.z, o[i][4 * c4 + 2]);
                        o[i][4 * c4 + 3] = fmaf(pv[i], vb.w, o[i][4 * c4 + 3]);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + 4 * ty + i;
        if (t >= n) continue;
        float* dst = out + static_cast<size_t>(start + t) * d + h * HD;
        const size_t at0 = static_cast<size_t>(start + t) * d + h * HD;
#pragma unroll
        for (int c = 0; c < OC; ++c) {
            const int col = HD == 32 ? 2 * tx + c : 64 * (c / 4) + 4 * tx + (c % 4);
            const float v = o[i][c] / l[i];
            if (out) dst[col] = v;
            if (po.planes) store_split(v, po.planes, po.hi, po.lo, at0 + col);
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Token selection and step bookkeeping.
// ---------------------------------------------------------------------------------------------
// TextEngine.argmax (TextEngine.java:392-400): strict '>' so the first maximum wins.
__global__ __launch_bounds__(256) void k_select_greedy(const float* __restrict__ logits, int V,
                                                       int W, int steps, int rows, int* step,
                                                       int* done, int* tokens, int* next,
                                                       int* window) {
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x;
    __shared__ int s_step;
    if (threadIdx.x == 0) s_step = *reinterpret_cast<volatile int*>(step);
    const int token = block_argmax(logits + static_cast<size_t>(r) * V, V);
    finish_row(r, token, s_step, rows, W, steps, step, done, tokens, next, window);
}

// Greedy selection when the head's epilogue already folded each row's first maximum into best[r]
// (pack_best): the logits are not read again, except the row's score at index 0, which wins when
// it is NaN (TextEngine.argmax only moves on to a larger score). best[r] is cleared for the next
// step.
__global__ __launch_bounds__(256) void k_select_greedy_packed(
    const float* __restrict__ logits, unsigned long long* __restrict__ best, int V, int W,
    int steps, int rows, int* step, int* done, int* tokens, int* next, int* window) {
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x;
    __shared__ int s_step, s_token;
    if (threadIdx.x == 0) {
        s_step = *reinterpret_cast<volatile int*>(step);
        const unsigned long long b = best[r];
        best[r] = 0ull;
        const float first = __ldcg(logits + static_cast<size_t>(r) * V);
        s_token = (isnan(first) || b == 0ull) ? 0 : unpack_best_index(b);
    }
    __syncthreads();
    finish_row(r, s_token, s_step, rows, W, steps, step, done, tokens, next, window);
}

// java.util.Random step and nextDouble (JDK specification).
__device__ __forceinline__ int rng_next(uint64_t& s, int bits) {
    s = (s * 0x5DEECE66DULL + 0xBULL) & ((1ULL << 48) - 1);
    return static_cast<int>(static_cast<int64_t>(s) >> (48 - bits));
}
__device__ __forceinline__ double rng_next_double(uint64_t& s) {
    const int64_t hi = rng_next(s, 26);
    const int64_t lo = rng_next(s, 27);
    return static_cast<double>((hi << 27) + lo) * 0x1.0p-53;
}

// Sort key: ascending key order == descending Double.compare order, ties by ascending index
// (the stable List.sort of TextEngine.java:408). -0.0 sorts after +0.0 and NaN first, as
// Double.compare orders them.
__device__ __forceinline__ uint64_t sort_key(float value, int index) {
    uint32_t f = __float_as_uint(value);
    if (isnan(value)) f = 0x7fc00000u;
    const uint32_t ascending = (f & 0x80000000u) ? ~f : (f | 0x80000000u);
    return (static_cast<uint64_t>(~ascending) << 32) | static_cast<uint32_t>(index);
}

// Threads of a sampling CTA: two CTAs share an SM (registers), so that one row's sequential sums
// run beside another row's sort.
constexpr int kSampleThreads = 512;

// One compare-exchange pass (k, j) of an ascending bitonic sort of keys[0..P) in shared memory,
// pairs spread over the block's threads.
__device__ __forceinline__ void bitonic_pass_shared(uint64_t* keys, int P, int k, int j) {
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
            const uint64_t a = keys[i], b = keys[ixj];
            if ((a > b) == ((i & k) == 0)) {
                keys[i] = b;
                keys[ixj] = a;
            }
        }
    }
}

// The same ascending bitonic network over P = E * blockDim.x keys, with thread t holding keys
// [E t, E t + E) in registers: the passes with j < E exchange inside a thread, those with
// E <= j < 32 E between the lanes of a warp (shuffles), and only those with j >= 32 E go through
// shared memory. Every pass compares and exchanges the same pairs as bitonic_pass_shared, so the
// result is the same sorted array. keys holds the input on entry and the sorted keys on return.
template <int E>
__device__ __forceinline__ void bitonic_sort_blocked(uint64_t* keys, int P) {
    const int t = threadIdx.x;
    uint64_t v[E];
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = keys[E * t + e];
    for (int k = 2; k <= P; k <<= 1) {
        if ((k >> 1) >= 32 * E) {
            __syncthreads();  // every thread has read the previous round's keys
#pragma unroll
            for (int e = 0; e < E; ++e) keys[E * t + e] = v[e];
            __syncthreads();
            for (int j = k >> 1; j >= 32 * E; j >>= 1) {
                bitonic_pass_shared(keys, P, k, j);
                __syncthreads();
            }
#pragma unroll
            for (int e = 0; e < E; ++e) v[e] = keys[E * t + e];
        }
        for (int j = min(k >> 1, 16 * E); j >= E; j >>= 1) {
            const int tj = j / E;  // partner lane offset
            const bool lower = (t & tj) == 0;
#pragma unroll
            for (int e = 0; e < E; ++e) {
                const uint64_t o = __shfl_xor_sync(kFull, v[e], tj);
                const bool up = ((E * t + e) & k) == 0;
                v[e] = (lower == up) ? (v[e] < o ? v[e] : o) : (v[e] > o ? v[e] : o);
            }
        }
#pragma unroll
        for (int j = E / 2; j >= 1; j >>= 1) {
            if (j < k) {
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    if ((e & j) == 0) {
                        const uint64_t a = v[e], b = v[e | j];
                        if ((a > b) == (((E * t + e) & k) == 0)) {
                            v[e] = b;
                            v[e | j] = a;
                        }
                    }
                }
            }
        }
    }
    __syncthreads();
#pragma unroll
    for (int e = 0; e < E; ++e) keys[E * t + e] = v[e];
    __syncthreads();
}

// Stable LSD radix sort of P = E * blockDim.x 64-bit keys, ascending by their high 32 bits, in
// eight passes of 4-bit digits; keys with equal high words keep their input order. With the sort
// keys of sort_key (ordered score in the high word, index in the low word, entered in index
// order) this is the same order as sorting the whole 64-bit keys. Per pass each thread holds E
// consecutive keys, counts their digits in its own column of cnt ([16][blockDim.x] 16-bit
// counters), an exclusive scan over cnt in digit-major order gives each (digit, thread) the
// number of keys that precede its keys in the output, and every key goes straight to its place.
__device__ __forceinline__ void scan_counts(uint16_t* cnt) {
    // Exclusive prefix sum over cnt[0 .. 16 * blockDim.x): thread t owns entries [16 t, 16 t + 16).
    __shared__ unsigned s_warp[32];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    uint4* c4 = reinterpret_cast<uint4*>(cnt) + 2 * t;
    const uint4 a = c4[0], b = c4[1];
    const unsigned w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    unsigned total = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) total += (w[i] & 0xffffu) + (w[i] >> 16);
    unsigned incl = total;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        unsigned x = lane < nw ? s_warp[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned y = __shfl_up_sync(kFull, x, o);
            if (lane >= o) x += y;
        }
        if (lane < nw) s_warp[lane] = x;
    }
    __syncthreads();
    unsigned run = incl - total + (warp > 0 ? s_warp[warp - 1] : 0u);
    unsigned out[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const unsigned lo = run;
        run += w[i] & 0xffffu;
        const unsigned hi = run;
        run += w[i] >> 16;
        out[i] = (lo & 0xffffu) | (hi << 16);
    }
    c4[0] = make_uint4(out[0], out[1], out[2], out[3]);
    c4[1] = make_uint4(out[4], out[5], out[6], out[7]);
}

// keys holds key p at p + p / 16 (E must be 16).
template <int E>
__device__ __forceinline__ void radix_sort_hi32(uint64_t* keys, uint16_t* cnt) {
    static_assert(E == 16, "the gap layout assumes 16 keys per thread");
    const int t = threadIdx.x, B = blockDim.x;
#pragma unroll 1
    for (int pass = 0; pass < 8; ++pass) {
        const int shift = 32 + 4 * pass;
        uint64_t v[E];
#pragma unroll
        for (int e = 0; e < E; ++e) v[e] = keys[(E + 1) * t + e];  // key E t + e, with its gap
#pragma unroll
        for (int dg = 0; dg < 16; ++dg) cnt[dg * B + t] = 0;
        unsigned lr[E / 2];  // each key's rank among the thread's earlier keys of its digit, two per word
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const int dg = static_cast<int>(v[e] >> shift) & 15;
            const unsigned c = cnt[dg * B + t];
            cnt[dg * B + t] = static_cast<uint16_t>(c + 1);
            if (e & 1) {
                lr[e / 2] |= c << 16;
            } else {
                lr[e / 2] = c;
            }
        }
        __syncthreads();
        scan_counts(cnt);
        __syncthreads();
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const int dg = static_cast<int>(v[e] >> shift) & 15;
            const unsigned rank = (e & 1) ? lr[e / 2] >> 16 : lr[e / 2] & 0xffffu;
            const unsigned pos = cnt[dg * B + t] + rank;
            keys[pos + (pos >> 4)] = v[e];
        }
        __syncthreads();
    }
}

// TextEngine.draw (TextEngine.java:403-427): stable descending sort, w_i = exp((s_i - max) / T)
// in double over the first topK, total summed in sorted order, target = nextDouble() * total,
// first i with target <= running sum (else topK - 1). The sums run sequentially in one thread so
// they round exactly as the reference's loop does.
__global__ __launch_bounds__(kSampleThreads, 2) void k_select_sample(const float* __restrict__ logits, int V,
                                                        int P, int W, int steps, int rows,
                                                        double temperature, int top_k,
                                                        uint64_t* rng, int* step, int* done,
                                                        int* tokens, int* next, int* window,
                                                        double* __restrict__ wout,
                                                        int* __restrict__ oout) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) unsigned char smem[];
    uint64_t* keys = reinterpret_cast<uint64_t*>(smem);
    // The radix path keeps key p at p + p / 16 (one gap per 16 keys), so that the 16 consecutive
    // keys each thread loads fall in different banks across a warp; the array has room for the
    // gaps, the token-order array follows it.
    const bool radix = P == 16 * static_cast<int>(blockDim.x);
    int* order = reinterpret_cast<int*>(keys + P + P / 16);
    const int r = blockIdx.x;
    const float* lr = logits + static_cast<size_t>(r) * V;
    __shared__ int s_step, s_token;
    if (threadIdx.x == 0) s_step = *reinterpret_cast<volatile int*>(step);
    for (int v = threadIdx.x; v < P; v += blockDim.x) {
        keys[radix ? v + (v >> 4) : v] = v < V ? sort_key(lr[v], v) : ~0ULL;
    }
    __syncthreads();
    if (radix) {
        // 16 x blockDim.x 16-bit counters in the token-order array, written only after the sort
        radix_sort_hi32<16>(keys, reinterpret_cast<uint16_t*>(order));
    } else if (P == 8 * static_cast<int>(blockDim.x)) {
        bitonic_sort_blocked<8>(keys, P);
    } else if (P == 4 * static_cast<int>(blockDim.x)) {
        bitonic_sort_blocked<4>(keys, P);
    } else {
        for (int k = 2; k <= P; k <<= 1) {
            for (int j = k >> 1; j > 0; j >>= 1) {
                bitonic_pass_shared(keys, P, k, j);
                __syncthreads();
            }
        }
    }
    for (int i = threadIdx.x; i < top_k; i += blockDim.x) {
        order[i] = static_cast<int>(keys[radix ? i + (i >> 4) : i] & 0xffffffffu);
    }
    __syncthreads();
    double* weights = reinterpret_cast<double*>(keys);  // reuse: keys are no longer needed
    const double maximum = static_cast<double>(lr[order[0]]);
    for (int i = threadIdx.x; i < top_k; i += blockDim.x) {
        weights[i] = exp(__ddiv_rn(__dadd_rn(static_cast<double>(lr[order[i]]), -maximum), temperature));
    }
    __syncthreads();
    if (wout) {
        // The sums and the draw run in k_sample_draw, a warp per row: hand over the sorted
        // weights and token ids.
        for (int i = threadIdx.x; i < top_k; i += blockDim.x) {
            wout[static_cast<size_t>(r) * V + i] = weights[i];
            oout[static_cast<size_t>(r) * V + i] = order[i];
        }
        return;
    }
    // The total, summed in sorted order by one thread; each running sum overwrites its weight,
    // so weights[i] becomes the reference loop's running sum after adding weight i. The weights
    // are read eight at a time ahead of the additions (16-byte shared loads), so the loop runs
    // at the latency of the f64 additions.
    __shared__ double s_target;
    __shared__ int s_first;
    if (threadIdx.x == 0) {
        double total = 0.0;
        int i = 0;
        double2* w2 = reinterpret_cast<double2*>(weights);  // P is a power of two >= 8
        for (; i + 8 <= top_k; i += 8) {
            const double2 a = w2[i / 2], b = w2[i / 2 + 1], c = w2[i / 2 + 2], e = w2[i / 2 + 3];
            double2 pa, pb, pc, pe;
            total = __dadd_rn(total, a.x); pa.x = total;
            total = __dadd_rn(total, a.y); pa.y = total;
            total = __dadd_rn(total, b.x); pb.x = total;
            total = __dadd_rn(total, b.y); pb.y = total;
            total = __dadd_rn(total, c.x); pc.x = total;
            total = __dadd_rn(total, c.y); pc.y = total;
            total = __dadd_rn(total, e.x); pe.x = total;
            total = __dadd_rn(total, e.y); pe.y = total;
            w2[i / 2] = pa;
            w2[i / 2 + 1] = pb;
            w2[i / 2 + 2] = pc;
            w2[i / 2 + 3] = pe;
        }
        for (; i < top_k; ++i) {
            total = __dadd_rn(total, weights[i]);
            weights[i] = total;
        }
        uint64_t state = rng[r];
        s_target = __dmul_rn(rng_next_double(state), total);
        rng[r] = state;
        s_first = top_k - 1;  // no running sum reaches the target: the last kept token
    }
    __syncthreads();
    // The first i with target <= running sum i (TextEngine.java:420-425), found by every thread
    // over its share of the running sums.
    {
        const double target = s_target;
        int first = top_k;
        for (int i = threadIdx.x; i < top_k; i += blockDim.x) {
            if (target <= weights[i]) {
                first = i;
                break;
            }
        }
        if (first < top_k) atomicMin(&s_first, first);
    }
    __syncthreads();
    if (threadIdx.x == 0) s_token = order[s_first];
    __syncthreads();
    finish_row(r, s_token, s_step, rows, W, steps, step, done, tokens, next, window);
}

// The rest of TextEngine.draw (TextEngine.java:416-427) for rows whose sorted weights and token
// ids k_select_sample handed over (wts, ord: [rows][V], the first top_k of each row), one warp per
// row, so that every row's sequential sums run at once. The whole warp walks the weights in
// sorted order, lane j's weight broadcast to all lanes, each lane adding in the same order from
// 0.0 (the reference's rounding); the running sum after every 32nd weight is kept (shared). The
// target is nextDouble() * total; the drawn index is the first whose running sum reaches it: the
// first 32-weight chunk whose last running sum does (running sums of non-negative weights never
// decrease), then the same additions again inside that chunk from the previous chunk's sum.
// Without a hit (NaN sums) the index is top_k - 1, as in the reference. Then the row's window
// push and the step counter, as finish_row does.
__global__ __launch_bounds__(256) void k_sample_draw(const double* __restrict__ wts,
                                                     const int* __restrict__ ord, int V, int top_k,
                                                     int W, int steps, int rows, uint64_t* rng,
                                                     int* step, int* done, int* tokens, int* next,
                                                     int* window) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ double s_ck[];  // [8 warps][chunks]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * 8 + warp;
    if (r >= rows) return;  // the whole warp
    const int g = *reinterpret_cast<volatile int*>(step);
    const double* w = wts + static_cast<size_t>(r) * V;
    const int nch = (top_k + 31) / 32;
    double* ck = s_ck + warp * nch;
    double total = 0.0;
    double cur = lane < top_k ? __ldcg(w + lane) : 0.0;
    for (int c = 0; c < nch; ++c) {
        const int base = c * 32;
        const double nxt = base + 32 + lane < top_k ? __ldcg(w + base + 32 + lane) : 0.0;
        const int n = min(32, top_k - base);
        if (n == 32) {
#pragma unroll
            for (int j = 0; j < 32; ++j) total = __dadd_rn(total, __shfl_sync(kFull, cur, j));
        } else {
            for (int j = 0; j < n; ++j) total = __dadd_rn(total, __shfl_sync(kFull, cur, j));
        }
        if (lane == 0) ck[c] = total;
        cur = nxt;
    }
    double target = 0.0;
    if (lane == 0) {
        uint64_t state = rng[r];
        target = __dmul_rn(rng_next_double(state), total);
        rng[r] = state;
    }
    target = __shfl_sync(kFull, target, 0);
    __syncwarp();
    int first = nch;
    for (int c = lane; c < nch; c += 32) {
        if (target <= ck[c]) {
            first = c;
            break;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) first = min(first, __shfl_xor_sync(kFull, first, o));
    int chosen = top_k - 1;
    if (first < nch) {
        const int base = first * 32;
        const int n = min(32, top_k - base);
        double run = first > 0 ? ck[first - 1] : 0.0;
        const double v = lane < n ? __ldcg(w + base + lane) : 0.0;
        int hit = n;
        for (int j = 0; j < n; ++j) {
            run = __dadd_rn(run, __shfl_sync(kFull, v, j));
            if (hit == n && target <= run) hit = j;
        }
        chosen = base + min(hit, n - 1);
    }
    const int token = __ldcg(ord + static_cast<size_t>(r) * V + chosen);
    // TextEngine.push (TextEngine.java:387-390): shift the window left by one, in 32-wide
    // chunks from the front (each chunk reads the positions after it before writing its own).
    int* win = window + static_cast<size_t>(r) * W;
    for (int base = 0; base < W; base += 32) {
        const int t = base + lane;
        const int carry = t + 1 < W ? win[t + 1] : token;
        __syncwarp();
        if (t < W) win[t] = carry;
        __syncwarp();
    }
    if (lane == 0) {
        tokens[static_cast<size_t>(r) * steps + g] = token;
        next[r] = token;
        __threadfence();
        const int prev = atomicAdd(done, 1);
        if (prev == rows - 1) {
            *done = 0;
            *step = g + 1;
            __threadfence();
        }
    }
}

__global__ void k_stash_logits(const float* __restrict__ logits, int V, int steps,
                               const int* __restrict__ step, const int* __restrict__ rows_of,
                               float* __restrict__ history) {
    pdl_trigger();
    pdl_wait();
    const int h = blockIdx.y;
    const int r = rows_of ? rows_of[h] : h;
    const int g = *step;
    const int v = blockIdx.x * blockDim.x + threadIdx.x;
    if (v < V) {
        history[(static_cast<size_t>(h) * steps + g) * V + v] = logits[static_cast<size_t>(r) * V + v];
    }
}

__global__ void k_fill_int(int* p, int value, int count) {
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) p[i] = value;
}
__global__ void k_iota(int* p, int count) {
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) p[i] = i;
}

// ---------------------------------------------------------------------------------------------
// Dispatch helpers.
// ---------------------------------------------------------------------------------------------
int pick_ks(int columns, int row_groups, int nvec) {
    // Enough CTAs to cover 2 waves of 148 SMs, but every warp keeps at least one full pass.
    int ks = 1;
    while (ks < 8) {
        const long ctas = static_cast<long>((columns + (8 / ks) - 1) / (8 / ks)) * row_groups;
        if (ctas >= 296 || nvec < 64 * ks) break;
        ks *= 2;
    }
    return ks;
}

template <typename WT, int MT, Epi E>
cudaError_t gemv_ks(cudaStream_t s, const float* x, int ldx, const void* w, const float* bias,
                    int M, int N, int K, const LnArgs& ln, const EpiArgs& ea) {
    const int row_groups = (M + MT - 1) / MT;
    const int ks = pick_ks(N, row_groups, K / Vec16<WT>::N);
    const WT* wt = static_cast<const WT*>(w);
    const dim3 block(256);
    const size_t smem = ln.gamma ? static_cast<size_t>(MT) * K * sizeof(float) : 0;
    switch (ks) {
        case 1: return launch_pdl(k_gemv<WT, MT, 1, E>, dim3((N + 7) / 8, row_groups), block, smem, s, x, ldx, wt, bias, M, N, K, ln, ea);
        case 2: return launch_pdl(k_gemv<WT, MT, 2, E>, dim3((N + 3) / 4, row_groups), block, smem, s, x, ldx, wt, bias, M, N, K, ln, ea);
        case 4: return launch_pdl(k_gemv<WT, MT, 4, E>, dim3((N + 1) / 2, row_groups), block, smem, s, x, ldx, wt, bias, M, N, K, ln, ea);
        default: return launch_pdl(k_gemv<WT, MT, 8, E>, dim3(N, row_groups), block, smem, s, x, ldx, wt, bias, M, N, K, ln, ea);
    }
}

template <typename WT, Epi E>
cudaError_t linear_typed(cudaStream_t s, const float* x, int ldx, const void* w,
                         const float* bias, int M, int N, int K, const EpiArgs& ea,
                         const LnArgs& ln) {
    if (linear_uses_gemv(M, N, K)) {
        if (M == 1) return gemv_ks<WT, 1, E>(s, x, ldx, w, bias, M, N, K, ln, ea);
        return gemv_ks<WT, 8, E>(s, x, ldx, w, bias, M, N, K, ln, ea);
    }
    if (ln.gamma) return cudaErrorInvalidValue;  // the tiled GEMM takes normalised inputs
    const dim3 grid((N + 127) / 128, (M + 127) / 128);
    return launch_pdl(k_gemm<WT, E>, grid, 256, 0, s, x, ldx, static_cast<const WT*>(w), bias, M, N, K, ea);
}

template <typename WT>
cudaError_t linear_epi(cudaStream_t s, const float* x, int ldx, const void* w, const float* bias,
                       int M, int N, int K, Epi epi, const EpiArgs& ea, const LnArgs& ln) {
    switch (epi) {
        case Epi::kStore: return linear_typed<WT, Epi::kStore>(s, x, ldx, w, bias, M, N, K, ea, ln);
        case Epi::kGelu: return linear_typed<WT, Epi::kGelu>(s, x, ldx, w, bias, M, N, K, ea, ln);
        case Epi::kResidual: return linear_typed<WT, Epi::kResidual>(s, x, ldx, w, bias, M, N, K, ea, ln);
        case Epi::kResidualGelu: return linear_typed<WT, Epi::kResidualGelu>(s, x, ldx, w, bias, M, N, K, ea, ln);
        case Epi::kQkv: return linear_typed<WT, Epi::kQkv>(s, x, ldx, w, bias, M, N, K, ea, ln);
        case Epi::kLogits: return linear_typed<WT, Epi::kLogits>(s, x, ldx, w, bias, M, N, K, ea, ln);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

bool linear_uses_gemv(int M, int N, int K) {
    (void)N;
    return M <= 8 || (K % 16) != 0;
}

bool linear_fuses_layernorm(int M, int N, int K) {
    const int mt = M == 1 ? 1 : 8;
    return linear_uses_gemv(M, N, K) && static_cast<size_t>(mt) * K * sizeof(float) <= 48 * 1024;
}

cudaError_t launch_linear(cudaStream_t s, const float* x, int ldx, const void* w, int w_bf16,
                          const float* bias, int M, int N, int K, Epi epi, const EpiArgs& ea,
                          const LnArgs* ln) {
    if (M <= 0 || N <= 0 || K <= 0) return cudaSuccess;
    LnArgs none;
    const LnArgs& use = ln ? *ln : none;
    if (use.gamma && !linear_fuses_layernorm(M, N, K)) return cudaErrorInvalidValue;
    return w_bf16 ? linear_epi<__nv_bfloat16>(s, x, ldx, w, bias, M, N, K, epi, ea, use)
                  : linear_epi<float>(s, x, ldx, w, bias, M, N, K, epi, ea, use);
}

cudaError_t launch_embed_tokens(cudaStream_t s, const void* tok, const void* pos, int w_bf16,
                                const int* ids, const int* positions, float* x, int count,
                                int d) {
    if (count <= 0) return cudaSuccess;
    const int threads = d >= 256 ? 256 : 128;
    cudaError_t err;
    if (w_bf16) {
        err = launch_pdl(k_embed_tokens<__nv_bfloat16>, count, threads, 0, s, 
            static_cast<const __nv_bfloat16*>(tok), static_cast<const __nv_bfloat16*>(pos), ids,
            positions, x, d);
    } else {
        err = launch_pdl(k_embed_tokens<float>, count, threads, 0, s, static_cast<const float*>(tok),
                                                        static_cast<const float*>(pos), ids,
                                                        positions, x, d);
    }
    return err;
}

cudaError_t launch_embed_decode(cudaStream_t s, const void* tok, const void* pos, int w_bf16,
                                const int* rowmap, const int* next, int* len, int* slot, float* x,
                                int R, int d) {
    if (R <= 0) return cudaSuccess;
    const int threads = d >= 256 ? 256 : 128;
    cudaError_t err;
    if (w_bf16) {
        err = launch_pdl(k_embed_decode<__nv_bfloat16>, R, threads, 0, s, 
            static_cast<const __nv_bfloat16*>(tok), static_cast<const __nv_bfloat16*>(pos),
            rowmap, next, len, slot, x, d);
    } else {
        err = launch_pdl(k_embed_decode<float>, R, threads, 0, s, static_cast<const float*>(tok),
                                                    static_cast<const float*>(pos), rowmap, next,
                                                    len, slot, x, d);
    }
    return err;
}

cudaError_t launch_embed_ln_decode(cudaStream_t s, const void* tok, const void* pos, int w_bf16,
                                   const int* rowmap, const int* next, int* len, int* slot, float* x,
                                   int R, int d, const float* gamma, const float* beta, float eps,
                                   void* hi, void* lo, int planes) {
    if (R <= 0) return cudaSuccess;
    if (d > 8 * 128 || planes < 1) return cudaErrorInvalidValue;
#define BST_EMBED_LN(WT, EPT)                                                                      \
    return launch_pdl(k_embed_ln_decode<WT, EPT>, R, 128, 0, s, static_cast<const WT*>(tok),       \
                      static_cast<const WT*>(pos), rowmap, next, len, slot, x, d, gamma, beta, eps, \
                      hi, lo, planes)
    const int ept = (d + 127) / 128;
    if (w_bf16) {
        if (ept <= 2) BST_EMBED_LN(__nv_bfloat16, 2);
        if (ept <= 4) BST_EMBED_LN(__nv_bfloat16, 4);
        BST_EMBED_LN(__nv_bfloat16, 8);
    }
    if (ept <= 2) BST_EMBED_LN(float, 2);
    if (ept <= 4) BST_EMBED_LN(float, 4);
    BST_EMBED_LN(float, 8);
#undef BST_EMBED_LN
}

cudaError_t launch_layernorm(cudaStream_t s, const float* x, int ldx, const float* gamma,
                             const float* beta, float* y, int ldy, int rows, int d, float eps,
                             void* hi, void* lo, int planes) {
    if (rows <= 0) return cudaSuccess;
    return launch_pdl(k_layernorm, (rows + 7) / 8, 256, 0, s, x, ldx, gamma, beta, y, ldy, rows,
                      d, eps, hi, lo, planes);
}

namespace {
template <typename KT, int HD>
cudaError_t attn_decode_typed(cudaStream_t s, const float* q, void* kc, void* vc,
                              const int* rowmap, const int* len, int R, int heads, int slots,
                              float scale, int splits, int chunk, float* part, int* tickets,
                              float* out, const PlaneOut& po, const QkvParts& qp) {
    return launch_pdl(k_attn_decode<KT, HD>, dim3(R * heads, splits), 128, 0, s, q,
                      static_cast<const KT*>(kc), static_cast<const KT*>(vc), rowmap, len, heads,
                      slots, scale, splits, chunk, part, tickets, out, po, qp);
}

template <typename KT, int HD>
cudaError_t attn_prefill_typed(cudaStream_t s, const float* q, const void* kc, const void* vc,
                               const int* seg_row, const int* seg_start, const int* seg_len,
                               int segments, int max_len, int heads, int slots, float scale,
                               float* out, const PlaneOut& po) {
    const dim3 grid(segments, heads, (max_len + kPrefillTile - 1) / kPrefillTile);
    return launch_pdl(k_attn_prefill<KT, HD>, grid, 256, attn_prefill_smem<HD>(), s,
        q, static_cast<const KT*>(kc), static_cast<const KT*>(vc), seg_row, seg_start, seg_len,
        heads, slots, scale, out, po);
}
}  // namespace

cudaError_t launch_reduce_residual_ln(cudaStream_t s, const float* part, int splits, int M, int N,
                                      const float* bias, float* x, int ldx, const LnArgs& ln,
                                      void* hi, void* lo, int planes) {
    if (M <= 0) return cudaSuccess;
#define BST_RRL(EPT, ZB)                                                                         \
    return launch_pdl(k_reduce_residual_ln<EPT, ZB>, dim3(M), 128, 0, s, part, splits, M, N, bias, \
                      x, ldx, ln.gamma, ln.beta, ln.eps, hi, lo, planes)
#define BST_RRL_Z(EPT)                    \
    if (splits <= 4) BST_RRL(EPT, 4);     \
    if (splits <= 8) BST_RRL(EPT, 8);     \
    BST_RRL(EPT, 16)
    if (N <= 256) { BST_RRL_Z(2); }
    if (N <= 512) { BST_RRL_Z(4); }
    if (N <= 768) { BST_RRL_Z(6); }
    if (N <= 1024) { BST_RRL_Z(8); }
#undef BST_RRL_Z
#undef BST_RRL
    return cudaErrorInvalidValue;
}

cudaError_t launch_attn_decode(cudaStream_t s, const float* q, void* k_cache, void* v_cache,
                               int kv_bf16, const int* rowmap, const int* len, int R, int heads,
                               int head_dim, int slots, float scale, int splits, int chunk,
                               float* part, int* tickets, float* out, const PlaneOut& planes,
                               const QkvParts& qkv) {
    if (R <= 0) return cudaSuccess;
    if (chunk > kMaxChunk) return cudaErrorInvalidValue;
#define BST_ATTN_DEC(KT, HD)                                                                    \
    return attn_decode_typed<KT, HD>(s, q, k_cache, v_cache, rowmap, len, R, heads, slots,      \
                                     scale, splits, chunk, part, tickets, out, planes, qkv)
    if (kv_bf16) {
        switch (head_dim) {
            case 32: BST_ATTN_DEC(__nv_bfloat16, 32);
            case 64: BST_ATTN_DEC(__nv_bfloat16, 64);
            case 128: BST_ATTN_DEC(__nv_bfloat16, 128);
        }
    } else {
        switch (head_dim) {
            case 32: BST_ATTN_DEC(float, 32);
            case 64: BST_ATTN_DEC(float, 64);
            case 128: BST_ATTN_DEC(float, 128);
        }
    }
#undef BST_ATTN_DEC
    return cudaErrorInvalidValue;
}

cudaError_t launch_attn_prefill(cudaStream_t s, const float* q, const void* k_cache,
                                const void* v_cache, int kv_bf16, const int* seg_row,
                                const int* seg_start, const int* seg_len, int segments,
                                int max_len, int heads, int head_dim, int slots, float scale,
                                float* out, const PlaneOut& planes) {
    if (segments <= 0) return cudaSuccess;
#define BST_ATTN_PRE(KT, HD)                                                                    \
    return attn_prefill_typed<KT, HD>(s, q, k_cache, v_cache, seg_row, seg_start, seg_len,      \
                                      segments, max_len, heads, slots, scale, out, planes)
    if (kv_bf16) {
        switch (head_dim) {
            case 32: BST_ATTN_PRE(__nv_bfloat16, 32);
            case 64: BST_ATTN_PRE(__nv_bfloat16, 64);
            case 128: BST_ATTN_PRE(__nv_bfloat16, 128);
        }
    } else {
        switch (head_dim) {
            case 32: BST_ATTN_PRE(float, 32);
            case 64: BST_ATTN_PRE(float, 64);
            case 128: BST_ATTN_PRE(float, 128);
        }
    }
#undef BST_ATTN_PRE
    return cudaErrorInvalidValue;
}

cudaError_t launch_prefill_tokens(cudaStream_t s, const int* window, int W, const int* seg_row,
                                  const int* seg_npad, const int* seg_start, const int* seg_len,
                                  int segments, int pad_id, int* ids, int* positions, int* tok_row,
                                  int* len) {
    if (segments <= 0) return cudaSuccess;
    return launch_pdl(k_prefill_tokens, segments, 256, 0, s, window, W, seg_row, seg_npad, seg_start, seg_len,
                                              pad_id, ids, positions, tok_row, len);
}

cudaError_t launch_gather_last(cudaStream_t s, const float* x, const int* seg_start,
                               const int* seg_len, int segments, int d, float* last) {
    if (segments <= 0) return cudaSuccess;
    return launch_pdl(k_gather_last, segments, 128, 0, s, x, seg_start, seg_len, d, last);
}

cudaError_t launch_window_embed(cudaStream_t s, const int* window, int W, const void* emb,
                                int w_bf16, int rows, int d, float* x) {
    if (rows <= 0) return cudaSuccess;
    cudaError_t err;
    if (w_bf16) {
        err = launch_pdl(k_window_embed<__nv_bfloat16>, rows, 256, 0, s, 
            window, W, static_cast<const __nv_bfloat16*>(emb), d, x);
    } else {
        err = launch_pdl(k_window_embed<float>, rows, 256, 0, s, window, W, static_cast<const float*>(emb), d,
                                                   x);
    }
    return err;
}

cudaError_t launch_last_token(cudaStream_t s, const int* window, int W, const float* weight,
                              const float* bias, int rows, int V, float* logits) {
    if (rows <= 0) return cudaSuccess;
    return launch_pdl(k_last_token, rows, 128, 0, s, window, W, weight, bias, V, logits);
}

cudaError_t launch_select_greedy(cudaStream_t s, const float* logits, int rows, int V, int W,
                                 int steps, int* step, int* done, int* tokens, int* next,
                                 int* window, unsigned long long* best) {
    if (rows <= 0) return cudaSuccess;
    if (W > 8 * 256) return cudaErrorInvalidValue;
    if (best) {
        return launch_pdl(k_select_greedy_packed, rows, 256, 0, s, logits, best, V, W, steps, rows,
                          step, done, tokens, next, window);
    }
    return launch_pdl(k_select_greedy, rows, 256, 0, s, logits, V, W, steps, rows, step, done, tokens, next,
                                         window);
}

size_t sample_draw_smem(int top_k) {
    return static_cast<size_t>(8) * ((top_k + 31) / 32) * sizeof(double);
}

size_t select_sample_smem(int V) {
    int P = 1;
    while (P < V) P <<= 1;
    // keys (with one gap per 16 on the radix path), then the token order
    return static_cast<size_t>(P + P / 16) * sizeof(uint64_t) + static_cast<size_t>(P) * sizeof(int);
}

cudaError_t launch_select_sample(cudaStream_t s, const float* logits, int rows, int V, int W,
                                 int steps, float temperature, int top_k, uint64_t* rng,
                                 int* step, int* done, int* tokens, int* next, int* window,
                                 double* sorted_w, int* sorted_ids) {
    if (rows <= 0) return cudaSuccess;
    if (W > 8 * kSampleThreads) return cudaErrorInvalidValue;
    int P = 1;
    while (P < V) P <<= 1;
    const size_t smem = select_sample_smem(V);
    if (smem > kSampleSmemLimit) return cudaErrorInvalidValue;
    const size_t draw_smem = sample_draw_smem(top_k);
    const bool split = sorted_w && sorted_ids && draw_smem <= 48 * 1024;
    cudaError_t err = launch_pdl(k_select_sample, rows, kSampleThreads, smem, s, logits, V, P, W,
                                 steps, rows, static_cast<double>(temperature), top_k, rng, step,
                                 done, tokens, next, window, split ? sorted_w : nullptr,
                                 split ? sorted_ids : nullptr);
    if (err || !split) return err;
    return launch_pdl(k_sample_draw, (rows + 7) / 8, 256, draw_smem, s, sorted_w, sorted_ids, V,
                      top_k, W, steps, rows, rng, step, done, tokens, next, window);
}

namespace {
template <typename KT, int HD>
cudaError_t configure_attn_prefill() {
    return cudaFuncSetAttribute(k_attn_prefill<KT, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                attn_prefill_smem<HD>());
}
}  // namespace

cudaError_t configure_device_kernels() {
    cudaError_t err = cudaFuncSetAttribute(k_select_sample,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(kSampleSmemLimit));
    if (err != cudaSuccess) return err;
    if ((err = configure_attn_prefill<float, 32>()) != cudaSuccess) return err;
    if ((err = configure_attn_prefill<float, 64>()) != cudaSuccess) return err;
    if ((err = configure_attn_prefill<float, 128>()) != cudaSuccess) return err;
    if ((err = configure_attn_prefill<__nv_bfloat16, 32>()) != cudaSuccess) return err;
    if ((err = configure_attn_prefill<__nv_bfloat16, 64>()) != cudaSuccess) return err;
    if ((err = configure_attn_prefill<__nv_bfloat16, 128>()) != cudaSuccess) return err;
    return configure_tc_kernels();
}

cudaError_t launch_stash_logits(cudaStream_t s, const float* logits, int rows, int V, int steps,
                                const int* step, const int* rows_of, float* history) {
    if (rows <= 0) return cudaSuccess;
    return launch_pdl(k_stash_logits, dim3((V + 255) / 256, rows), 256, 0, s, logits, V, steps, step,
                      rows_of, history);
}

cudaError_t configure_device_kernels_once(int device) {
    static std::mutex mu;
    static uint64_t done = 0;
    std::lock_guard<std::mutex> lock(mu);
    if (device >= 0 && device < 64 && (done >> device) & 1ull) return cudaSuccess;
    const cudaError_t err = configure_device_kernels();
    if (err == cudaSuccess && device >= 0 && device < 64) done |= 1ull << device;
    return err;
}

cudaError_t launch_fill_int(cudaStream_t s, int* p, int value, int count) {
    if (count <= 0) return cudaSuccess;
    return launch_pdl(k_fill_int, (count + 255) / 256, 256, 0, s, p, value, count);
}

cudaError_t launch_iota(cudaStream_t s, int* p, int count) {
    if (count <= 0) return cudaSuccess;
    return launch_pdl(k_iota, (count + 255) / 256, 256, 0, s, p, count);
}

}  // namespace bst
