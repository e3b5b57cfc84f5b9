// Greedy token selection and per-step bookkeeping shared by the selection kernels.
#pragma once

#include "device.cuh"

namespace bst {

// First index of the maximum of lr[0..V) over the whole block (TextEngine.argmax,
// TextEngine.java:392-400: strict '>' keeps the first maximum; a NaN first score is never
// replaced). Every thread of the block must call it; the result is returned to all threads. The
// scores are read through L2 (ld.global.cg), so they may have been written earlier in the same
// kernel by other CTAs.
__device__ __forceinline__ int block_argmax(const float* lr, int V) {
    __shared__ float s_val[32];
    __shared__ int s_idx[32];
    __shared__ int s_token;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
        const float x = __ldcg(lr + v);
        if (isnan(x)) continue;
        if (x > best || (x == best && v < bi)) {
            best = x;
            bi = v;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(kFull, best, o);
        const int oi = __shfl_xor_sync(kFull, bi, o);
        if (ov > best || (ov == best && oi < bi)) {
            best = ov;
            bi = oi;
        }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        s_val[warp] = best;
        s_idx[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w2 = 1; w2 < static_cast<int>(blockDim.x >> 5); ++w2) {
            if (s_val[w2] > best || (s_val[w2] == best && s_idx[w2] < bi)) {
                best = s_val[w2];
                bi = s_idx[w2];
            }
        }
        s_token = (isnan(__ldcg(lr)) || bi == 0x7fffffff) ? 0 : bi;
    }
    __syncthreads();
    return s_token;
}

// Writes the chosen token, shifts the row's window (TextEngine.push, TextEngine.java:387-390) and
// advances the step counter once the last row of the step is done.
__device__ __forceinline__ void finish_row(int r, int token, int g, int rows, int W, int steps, int* step,
                           int* done, int* tokens, int* next, int* window) {
    int* win = window + static_cast<size_t>(r) * W;
    constexpr int kPerThread = 8;
    int carry[kPerThread];
#pragma unroll
    for (int c = 0; c < kPerThread; ++c) {
        const int t = threadIdx.x + c * blockDim.x;
        carry[c] = t + 1 < W ? win[t + 1] : token;
    }
    __syncthreads();
#pragma unroll
    for (int c = 0; c < kPerThread; ++c) {
        const int t = threadIdx.x + c * blockDim.x;
        if (t < W) win[t] = carry[c];
    }
    if (threadIdx.x == 0) {
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

}  // namespace bst
