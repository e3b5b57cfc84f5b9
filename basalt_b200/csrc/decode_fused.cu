// One greedy decode step of the (padded) decoder for small batches, as one persistent kernel.
//
// At batch 1 a decode step is ~60 small dependent operations (per layer: LayerNorm + QKV,
// attention, output projection, LayerNorm + FFN1, FFN2; then the head and the argmax). Launched as
// separate kernels each pays a launch, a ramp-up and a DRAM round trip with most SMs idle. Here a
// single cooperative launch runs the whole step: one CTA per SM, 16 warps each. Every exchange of
// a full activation vector between CTAs costs a grid barrier plus the global-memory round trips
// around it, so the step is organised around as few of them as the data dependencies allow:
// three grid barriers per layer.
//
//   A (attention block)  The CTAs are split into one group per head (cph = grid / heads CTAs
//        each; leftover CTAs only wait). A group computes its head's q, k and v columns of the
//        QKV projection (LN1 fused; k and v go straight into the cache at slot len), meets at a
//        per-head counter, runs the head's attention over the cache (one warp per 32-key chunk;
//        the last chunk of a (row, head) merges the chunk partials in chunk order and counts the
//        head's merges), meets again, and multiplies the head's attention output by the head's
//        block of the output projection: a partial output-projection vector per head.
//   B    Every CTA sums the heads' partial vectors in head order, adds the bias and the residual
//        (x' = x + O), layer-normalises x' itself (f64 statistics over the whole row, as
//        nn_ops.rs:168-199) and computes its block of FFN1 columns with GELU.
//   C    Every CTA computes its block of FFN2 columns, adds bias and residual to the residual
//        columns it owns (kept in shared memory) and publishes LayerNorm partial statistics.
//   head after the last layer: logits (final LN fused) and each CTA's first maximum, combined
//        with a 64-bit atomic max; the last CTA to finish (ticket) applies TextEngine.argmax's
//        rule, pushes the token into the window and advances the step counter and lengths.
// (TransformerBlock.forward, torch/TransformerBlock.java:37-43, inside the padded decoder whose
// last-position head follows TextEngine.scores, infer/TextEngine.java:96-112.)
//
// Weights are constant during the step, so each CTA has the TMA unit copy its share of the next
// projections' weight rows into shared memory ahead of use, into one stage buffer per phase
// (cp.async.bulk into this CTA only, mbarrier completion): the weight stream overlaps the
// barriers and the activation loads. Rows that do not fit are read from global memory.
//
// Memory coherence: activations, the cache, partial sums and counters are written inside the
// kernel by other CTAs, so they are read with ld.global.cg (L2) after an acquire, never through
// the non-coherent read-only path; only weights and embeddings use that path. Every wait (grid
// barrier, head-group counter, weight stage) is bounded by %globaltimer: on expiry it records an
// error code in *err (11: grid barrier, 12: weight stage, 13: head-group counter) and the CTAs
// return at the next grid barrier.

#include <cuda_bf16.h>

#include <algorithm>

#include "device.cuh"
#include "epilogue.cuh"
#include "kernels.h"

namespace bst {
namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxRows = 8;
constexpr int kChunk = 32;
constexpr int kMaxChunkGroups = 4;  // chunk merge handles up to 4 * 32 chunks (4096 keys)
constexpr int kMaxHeadDim = 128;
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s bound on any single wait
constexpr size_t kSmemLimit = 212 * 1024;    // dynamic shared memory of one CTA
constexpr int kOPrefetch = 1;                // output-projection weight vectors held per thread

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Waits (one thread) until *ctr has reached target; bounded. The caller syncs the block after.
__device__ __forceinline__ void spin_until(const unsigned* ctr, unsigned target, int* err, int code,
                                           int* abort_flag) {
    if (static_cast<int>(ld_acquire(ctr) - target) >= 0) return;
    const uint64_t start = global_ns();
    while (static_cast<int>(ld_acquire(ctr) - target) < 0) {
        if (*reinterpret_cast<volatile int*>(abort_flag)) return;
        if (global_ns() - start > kWaitNs) {
            atomicCAS(err, 0, code);
            *abort_flag = 1;
            return;
        }
    }
}

// Grid barrier over the co-resident CTAs of a cooperative launch: a counter that only grows.
// Barrier b of a launch completes when the counter reaches base + b * gridDim.x, where the host
// passes base (the count every earlier launch left behind). Returns false when this or an earlier
// wait of the CTA timed out.
struct GridSync {
    unsigned* count;
    unsigned target;
    int* err;
    int* abort_flag;  // shared
};

__device__ __forceinline__ bool grid_sync(GridSync& g) {
    __syncthreads();
    g.target += gridDim.x;
    if (threadIdx.x == 0) {
        atom_add_acq_rel(g.count, 1);
        spin_until(g.count, g.target, g.err, 11, g.abort_flag);
    }
    __syncthreads();
    return *reinterpret_cast<volatile int*>(g.abort_flag) == 0;
}

// Block `part` of `parts` equal blocks of [0, N).
__device__ __forceinline__ void block_of(int N, int parts, int part, int* c0, int* c1) {
    const int cpc = (N + parts - 1) / parts;
    *c0 = min(N, part * cpc);
    *c1 = min(N, *c0 + cpc);
}

// This CTA's share of an [N, K] weight matrix in a grid-wide projection: a block of whole rows.
__device__ __forceinline__ void column_block(int N, int* c0, int* c1) {
    block_of(N, gridDim.x, blockIdx.x, c0, c1);
}

// Virtual columns of a projection to matrix rows: the identity, or (h >= 0) the q, k and v blocks
// of head h inside the fused [3d] QKV projection (virtual column j -> block j / hd).
struct ColMap {
    int d = 0, hd = 1, h = -1;
    __device__ __forceinline__ int operator()(int v) const {
        if (h < 0) return v;
        const int blk = v / hd;
        return blk * d + h * hd + (v - blk * hd);
    }
};

// How a CTA's threads cover its columns [c0, c1) of a projection with nvec 16-byte weight vectors
// per column. Up to 16 columns: `ks` whole warps per column, each on a contiguous part of K. More
// columns: groups of `gs` lanes (a power of two) per column, repeated `reps` times when there are
// more columns than groups.
struct Plan {
    int c0, c1;
    int gs, ks, reps;
    int col;         // this thread's column in rep 0
    int col_stride;  // column step between reps
    int vbeg, vend, vstep;
    int part;        // warp's part of its column (gs == 32)
};

__device__ __forceinline__ Plan make_plan(int c0, int c1, int nvec) {
    Plan p;
    p.c0 = c0;
    p.c1 = c1;
    const int ncols = c1 - c0;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (ncols <= kWarps) {
        p.gs = 32;
        p.ks = ncols > 0 ? kWarps / ncols : 1;
        p.reps = 1;
        p.part = warp % p.ks;
        p.col = c0 + warp / p.ks;
        p.col_stride = 0;
        const int per = (nvec + p.ks - 1) / p.ks;
        p.vbeg = p.part * per + lane;
        p.vend = min(nvec, p.part * per + per);
        p.vstep = 32;
    } else {
        int gs = 32;
        while (gs > 1 && gs * ncols > kThreads) gs >>= 1;
        const int groups = kThreads / gs;
        p.gs = gs;
        p.ks = 1;
        p.part = 0;
        p.reps = (ncols + groups - 1) / groups;
        p.col = c0 + tid / gs;
        p.col_stride = groups;
        p.vbeg = tid % gs;
        p.vend = nvec;
        p.vstep = gs;
    }
    return p;
}

template <typename WT>
struct Unpack;
template <>
struct Unpack<float> {
    static constexpr int N = 4;
    __device__ __forceinline__ static void run(const uint4& u, float* o) {
        o[0] = __uint_as_float(u.x); o[1] = __uint_as_float(u.y);
        o[2] = __uint_as_float(u.z); o[3] = __uint_as_float(u.w);
    }
};
template <>
struct Unpack<__nv_bfloat16> {
    static constexpr int N = 8;
    __device__ __forceinline__ static void run(const uint4& u, float* o) {
        const unsigned w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            o[2 * i] = bf16_bits_to_f(w[i] & 0xffffu);
            o[2 * i + 1] = bf16_bits_to_f(w[i] >> 16);
        }
    }
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
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

// One contiguous global -> shared copy by the TMA unit into this CTA, completing on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// A weight stage: a shared-memory buffer the TMA unit fills with this CTA's rows of one
// projection (as many whole rows as fit; the rest is read from global memory) plus the
// LayerNorm parameters of the projection's input. The descriptor lives in shared memory and only
// thread 0 changes it; every thread reads it after a __syncthreads().
struct WStage {
    uint64_t bar;           // mbarrier, one phase per issued copy
    unsigned char* buf;     // weight rows (shared), in virtual column order
    float* lnp;             // gamma [K], beta [K] (shared), or nullptr
    unsigned cap;           // bytes
    unsigned parity;        // phase the next wait expects
    int cols;               // weight rows of the current projection held in buf
    int pending;            // a copy was issued and not yet waited for
};

// Issues the stage of virtual columns [c0, c1) of Y[R, N] = X W^T (W [N, K] of WT) for this CTA.
// Every thread of the CTA calls it; thread 0 records it and issues the copies.
template <typename WT>
__device__ __forceinline__ void stage_issue(const void* w, int K, int c0, int c1, ColMap cm,
                                            const float* ln_gamma, const float* ln_beta,
                                            WStage& st) {
    if (c1 <= c0) return;  // uniform over the CTA
    const size_t row_bytes = static_cast<size_t>(K) * sizeof(WT);
    // Every thread is done with this buffer's previous contents: hand it to the TMA unit.
    __syncthreads();
    if (threadIdx.x == 0) {
        const int cols = min(c1 - c0, static_cast<int>(st.cap / row_bytes));
        st.cols = cols;
        st.pending = 1;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        const uint32_t lbytes = ln_gamma && st.lnp ? static_cast<uint32_t>(K) * 4u : 0u;
        mbar_expect_tx(&st.bar, static_cast<uint32_t>(cols * row_bytes) + 2 * lbytes);
        // Runs of virtual columns that are contiguous matrix rows: one copy each.
        int v = c0;
        while (v < c0 + cols) {
            const int row0 = cm(v);
            int n = 1;
            while (v + n < c0 + cols && cm(v + n) == row0 + n) ++n;
            bulk_load(st.buf + static_cast<size_t>(v - c0) * row_bytes,
                      static_cast<const WT*>(w) + static_cast<size_t>(row0) * K,
                      static_cast<uint32_t>(n * row_bytes), &st.bar);
            v += n;
        }
        if (lbytes) {
            bulk_load(st.lnp, ln_gamma, lbytes, &st.bar);
            bulk_load(st.lnp + K, ln_beta, lbytes, &st.bar);
        }
    }
}

// Waits for the stage issued by stage_issue (bounded; on expiry records code 12, waits once more
// for the copy to land and lets the next grid barrier end the kernel). Every thread of the CTA
// calls it; idempotent.
__device__ __forceinline__ void stage_wait(WStage& st, int* err, int* abort_flag) {
    __syncthreads();
    if (!st.pending) return;  // uniform: read after the barrier, changed only below
    const unsigned parity = st.parity;
    if (!mbar_try_wait(&st.bar, parity)) {
        uint64_t start = global_ns();
        bool late = false;
        while (!mbar_try_wait(&st.bar, parity)) {
            if (global_ns() - start > kWaitNs) {
                if (late) break;
                if (threadIdx.x == 0) {
                    atomicCAS(err, 0, 12);
                    *abort_flag = 1;
                }
                late = true;
                start = global_ns();
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        st.parity = parity ^ 1u;
        st.pending = 0;
    }
    __syncthreads();
}

// Copies rows [R][K] (row stride ldx, K % 4 == 0) from global memory into shared memory.
__device__ __forceinline__ void stage_rows(const float* x, int ldx, int R, int K, float* dst) {
    const int kv = K / 4;
    for (int e = threadIdx.x; e < R * kv; e += kThreads) {
        const int i = e / kv, k = e - i * kv;
        const float4 v = __ldcg(reinterpret_cast<const float4*>(x + static_cast<size_t>(i) * ldx) + k);
        reinterpret_cast<float4*>(dst + static_cast<size_t>(i) * K)[k] = v;
    }
}

// Where a projection's outputs go, beyond the shared epilogues.
struct Sink {
    float* xown = nullptr;  // kResidual: this CTA's residual columns [R][xown_ld] (shared)
    int xown_ld = 0;
    float* history = nullptr;  // kLogits: optional [R][steps][V] copy of the scores
    int step = 0, steps = 0;
    unsigned long long* best = nullptr;  // kLogits: per-row packed maximum (shared)
};

// One output of a projection through its epilogue (chosen at run time). c0: the CTA's first
// residual column (kResidual).
__device__ __forceinline__ void store_out(Epi epi, const EpiArgs& ea, const Sink& sk, int c0, int m,
                                       int n, float v) {
    switch (epi) {
        case Epi::kResidual: {
            float* own = sk.xown + m * sk.xown_ld + (n - c0);
            const float x = __fadd_rn(*own, v);
            *own = x;
            ea.out[static_cast<size_t>(m) * ea.ldo + n] = x;
            break;
        }
        case Epi::kLogits:
            ea.out[static_cast<size_t>(m) * ea.ldo + n] = v;
            if (sk.history) sk.history[(static_cast<size_t>(m) * sk.steps + sk.step) * ea.ldo + n] = v;
            if (!isnan(v)) atomicMax(sk.best + m, pack_best(v, n));
            break;
        case Epi::kGelu:
            epi_apply<Epi::kGelu>(ea, m, n, v);
            break;
        case Epi::kQkv:
            epi_apply<Epi::kQkv>(ea, m, n, v);
            break;
        default:
            epi_apply<Epi::kStore>(ea, m, n, v);
            break;
    }
}

// LayerNorm statistics without a block-wide pass: each residual phase publishes, per row, the sum
// and the centred sum of squares (M2) of the columns its CTA owns (f64); the next LayerNorm phase
// combines the per-CTA pairs in CTA order with Chan's formula, M2 = sum_c [M2_c + n_c (mean_c -
// mean)^2], which equals the two-pass statistics of nn_ops.rs:168-199 up to f64 rounding.
// stats layout: [row][cta][2].
__device__ __forceinline__ void publish_stats(const float* xown, int own_ld, int ncols, int R,
                                              double* stats) {
    if (threadIdx.x < R && ncols > 0) {
        const int i = threadIdx.x;
        const float* xr = xown + i * own_ld;
        double s = 0.0;
        for (int j = 0; j < ncols; ++j) s = __dadd_rn(s, static_cast<double>(xr[j]));
        const double mc = __ddiv_rn(s, static_cast<double>(ncols));
        double m2 = 0.0;
        for (int j = 0; j < ncols; ++j) {
            const double delta = __dadd_rn(static_cast<double>(xr[j]), -mc);
            m2 = __dadd_rn(m2, __dmul_rn(delta, delta));
        }
        double* out = stats + (static_cast<size_t>(i) * gridDim.x + blockIdx.x) * 2;
        out[0] = s;
        out[1] = m2;
    }
}

// Mean and 1/sqrt(var + eps) of R rows of width d from the published per-CTA statistics; warp i
// handles row i. Results in mean[i], inv[i] (shared) after the caller's __syncthreads().
__device__ __forceinline__ void combine_stats(const double* stats, int R, int d, float eps,
                                              double* mean, double* inv) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp >= R) return;
    const int G = gridDim.x;
    const int cpc = (d + G - 1) / G;
    const double* rs = stats + static_cast<size_t>(warp) * G * 2;
    constexpr int kPer = 8;  // CTAs per lane (grids up to 256)
    double sc[kPer], m2c[kPer];
    int nc[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const int c = lane + 32 * k;
        const int c0 = min(d, c * cpc);
        nc[k] = c < G ? min(d, c0 + cpc) - c0 : 0;
        sc[k] = nc[k] > 0 ? __ldcg(rs + 2 * c) : 0.0;
        m2c[k] = nc[k] > 0 ? __ldcg(rs + 2 * c + 1) : 0.0;
    }
    double s = 0.0;
#pragma unroll
    for (int k = 0; k < kPer; ++k) s = __dadd_rn(s, sc[k]);
    const double mu = __ddiv_rn(warp_sum_d(s), static_cast<double>(d));
    double m2 = 0.0;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        if (nc[k] > 0) {
            const double delta = __dadd_rn(__ddiv_rn(sc[k], static_cast<double>(nc[k])), -mu);
            m2 = __dadd_rn(m2, __dadd_rn(m2c[k], __dmul_rn(static_cast<double>(nc[k]), __dmul_rn(delta, delta))));
        }
    }
    m2 = warp_sum_d(m2);
    if (lane == 0) {
        const double variance = __ddiv_rn(m2, static_cast<double>(d));
        mean[warp] = mu;
        inv[warp] = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(variance, static_cast<double>(eps))));
    }
}

// xs = LayerNorm(xraw) for R rows of width K, from the published statistics (stats != nullptr) or
// from the rows themselves, with gamma/beta in lnp [2][K] (shared). Ends with __syncthreads().
template <int RT>
__device__ __forceinline__ void normalise_rows(const float* xraw, int R, int K, const double* stats,
                                               float eps, const float* lnp, float* xs) {
    __shared__ double s_mean[RT], s_inv[RT];
    if (stats) {
        combine_stats(stats, R, K, eps, s_mean, s_inv);
        __syncthreads();
        for (int e = threadIdx.x; e < R * K; e += kThreads) {
            const int i = e / K, k = e - i * K;
            const float nrm = static_cast<float>(
                __dmul_rn(__dadd_rn(static_cast<double>(xraw[e]), -s_mean[i]), s_inv[i]));
            xs[e] = __fadd_rn(__fmul_rn(nrm, lnp[k]), lnp[K + k]);
        }
    } else {
        const LnArgs lns{lnp, lnp + K, eps};
        layernorm_rows(xraw, K, RT == 1 ? 1 : R, K, lns, xs);
    }
    __syncthreads();
}

// Y[R, columns c0..c1) = X[R, K] * W[cm(c), K]^T + bias[cm(c)] with the inputs already in xs
// (shared, [R][K]) and the weight rows staged by stage_issue. Partial sums are combined in a fixed
// order, so results repeat bit for bit.
template <typename WT, int RT>
__device__ __forceinline__ void gemv(const float* xs, int R, int K, int c0, int c1, ColMap cm,
                                     const void* wv, const float* bias, Epi epi, const EpiArgs& ea,
                                     const Sink& sk, int res_c0, WStage& st, int* err,
                                     int* abort_flag) {
    constexpr int VEC = Unpack<WT>::N;
    __shared__ float red[kWarps][RT];
    const int nvec = K / VEC;
    const Plan pl = make_plan(c0, c1, nvec);
    if (c1 <= c0) return;  // uniform over the CTA
    stage_wait(st, err, abort_flag);
    const WT* w = static_cast<const WT*>(wv);
    const uint4* staged_w = reinterpret_cast<const uint4*>(st.buf);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int rep = 0; rep < pl.reps; ++rep) {
        const int col = pl.col + rep * pl.col_stride;
        const bool act = col < pl.c1;
        const int mcol = act ? cm(col) : 0;
        const float b = act && bias ? __ldg(bias + mcol) : 0.0f;
        float acc[RT];
#pragma unroll
        for (int i = 0; i < RT; ++i) acc[i] = 0.0f;
        if (act) {
            const bool in_smem = col - pl.c0 < st.cols;
            const uint4* wc = in_smem ? staged_w + static_cast<size_t>(col - pl.c0) * nvec
                                      : reinterpret_cast<const uint4*>(w + static_cast<size_t>(mcol) * K);
#pragma unroll 2
            for (int v = pl.vbeg; v < pl.vend; v += pl.vstep) {
                float wf[VEC];
                Unpack<WT>::run(in_smem ? wc[v] : __ldg(wc + v), wf);
#pragma unroll
                for (int i = 0; i < RT; ++i) {
                    if (i < R) {
                        const float* xp = xs + i * K + v * VEC;
#pragma unroll
                        for (int c = 0; c < VEC; ++c) acc[i] = fmaf(wf[c], xp[c], acc[i]);
                    }
                }
            }
        }
        bool storer;
        if (pl.gs == 32) {
#pragma unroll
            for (int i = 0; i < RT; ++i) acc[i] = warp_sum(acc[i]);
            storer = act && lane == 0;
            if (pl.ks > 1) {
                if (lane == 0) {
#pragma unroll
                    for (int i = 0; i < RT; ++i) red[warp][i] = acc[i];
                }
                __syncthreads();
                storer = storer && pl.part == 0;
                if (storer) {
#pragma unroll
                    for (int i = 0; i < RT; ++i) {
                        float sum = 0.0f;
                        for (int p = 0; p < pl.ks; ++p) sum += red[warp + p][i];
                        acc[i] = sum;
                    }
                }
            }
        } else {
            for (int o = pl.gs >> 1; o > 0; o >>= 1) {
#pragma unroll
                for (int i = 0; i < RT; ++i) acc[i] += __shfl_xor_sync(kFull, acc[i], o);
            }
            storer = act && threadIdx.x % pl.gs == 0;
        }
        if (storer) {
#pragma unroll
            for (int i = 0; i < RT; ++i) {
                if (i < R) store_out(epi, ea, sk, res_c0, i, mcol, bias ? __fadd_rn(acc[i], b) : acc[i]);
            }
        }
    }
}

// 16 bytes of cache through L2, as floats.
template <typename KT>
__device__ __forceinline__ void load_cg16(const KT* p, float* o) {
    const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p));
    Unpack<KT>::run(u, o);
}

// Decode attention of head h over every (row, 32-key chunk) that holds keys, by `workers` warps
// (this one is number `worker`): one warp per chunk. Lanes own keys for the scores; for P.V lanes
// own (key group, 16-byte slice of the head) pairs so that every V load of the chunk is
// independent. The last chunk of a (row, head) to finish (ticket) merges the chunk partials in
// chunk order, writes the row's attention output for the head and counts one merge on `merged`.
template <typename KT, int HD>
__device__ __forceinline__ void attention_head(int h, int worker, int workers, const float* q,
                                               const KT* kc, const KT* vc, const int* s_len, int R,
                                               int heads, int slots, int nchunks, float scale,
                                               float* part, int* tickets, float* out,
                                               unsigned* merged, float* qslot) {
    constexpr int VE = 16 / sizeof(KT);  // elements per 16-byte vector
    constexpr int DV = HD / VE;          // vectors per key row
    constexpr int KG = 32 / DV;          // key groups for P.V (>= 1)
    constexpr int KPL = 32 / KG;         // keys per lane for P.V
    constexpr int LB = DV < 64 / VE ? DV : 64 / VE;    // loads in flight per lane: 64 floats
    constexpr int PB = KPL < 64 / VE ? KPL : 64 / VE;
    constexpr int DPL = HD / 32;
    constexpr int MB = 32 / DPL;  // merge loads in flight per lane: 32 floats
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int d = heads * HD;
    float* qw = qslot + warp * HD;
    const int tasks = R * nchunks;
    for (int task = worker; task < tasks; task += workers) {
        const int i = task / nchunks;
        const int c = task - i * nchunks;
        const int T = s_len[i] + 1;  // cached keys plus this step's
        const int nck = (T + kChunk - 1) / kChunk;
        if (c >= nck) continue;
        const int start = c * kChunk;
        const int n = min(kChunk, T - start);
        const size_t base = (static_cast<size_t>(i) * heads + h) * slots + start;
        // This lane's key (the last key again for lanes past the chunk) and the query, together;
        // the chunk's values are asked into L2 at the same time.
        const KT* kr = kc + (base + min(lane, n - 1)) * HD;
        float kv[LB][VE];
#pragma unroll
        for (int e = 0; e < LB; ++e) load_cg16(kr + e * VE, kv[e]);
        {
            const char* vbase = reinterpret_cast<const char*>(vc + base * HD);
            const int vlines = (n * HD * static_cast<int>(sizeof(KT)) + 127) / 128;
            for (int ln = lane; ln < vlines; ln += 32) {
                asm volatile("prefetch.global.L2 [%0];" ::"l"(vbase + ln * 128));
            }
        }
        for (int e = lane; e < HD; e += 32) qw[e] = __ldcg(q + static_cast<size_t>(i) * d + h * HD + e);
        __syncwarp();
        float dot = 0.0f;
#pragma unroll 1
        for (int e0 = 0; e0 < DV; e0 += LB) {
            if (e0 > 0) {
#pragma unroll
                for (int e = 0; e < LB; ++e) load_cg16(kr + (e0 + e) * VE, kv[e]);
            }
#pragma unroll
            for (int e = 0; e < LB; ++e) {
#pragma unroll
                for (int cc = 0; cc < VE; ++cc) dot = fmaf(kv[e][cc], qw[(e0 + e) * VE + cc], dot);
            }
        }
        const float s = lane < n ? __fmul_rn(dot, scale) : -INFINITY;
        const float m = warp_max(s);
        const float p = lane < n ? expf(s - m) : 0.0f;
        const float l = warp_sum(p);
        const int kg = lane / DV, dv = lane % DV;
        float o[VE];
#pragma unroll
        for (int e = 0; e < VE; ++e) o[e] = 0.0f;
#pragma unroll 1
        for (int t0 = 0; t0 < KPL; t0 += PB) {
            float vv[PB][VE];
#pragma unroll
            for (int t = 0; t < PB; ++t) {
                const int j = kg + KG * (t0 + t);
                load_cg16(vc + (base + min(j, n - 1)) * HD + dv * VE, vv[t]);
            }
#pragma unroll
            for (int t = 0; t < PB; ++t) {
                const int j = kg + KG * (t0 + t);
                const float pj = __shfl_sync(kFull, p, j);
                if (j < n) {
#pragma unroll
                    for (int e = 0; e < VE; ++e) o[e] = fmaf(pj, vv[t][e], o[e]);
                }
            }
        }
#pragma unroll
        for (int off = DV; off < 32; off <<= 1) {
#pragma unroll
            for (int e = 0; e < VE; ++e) o[e] += __shfl_xor_sync(kFull, o[e], off);
        }
        float* mine = part + (static_cast<size_t>(i * heads + h) * nchunks + c) * (HD + 2);
        if (lane < DV) {
#pragma unroll
            for (int e = 0; e < VE; ++e) mine[dv * VE + e] = o[e];
        }
        if (lane == 0) {
            mine[HD] = m;
            mine[HD + 1] = l;
        }
        // Publish the partial: the ticket is a release (it orders the warp's stores above, which
        // __syncwarp orders before it) and an acquire for the warp that merges.
        __syncwarp();
        int last = 0;
        if (lane == 0) {
            last = atom_add_acq_rel(reinterpret_cast<unsigned*>(&tickets[i * heads + h]), 1) ==
                   static_cast<unsigned>(nck - 1);
        }
        last = __shfl_sync(kFull, last, 0);
        if (last) {
            __syncwarp();  // orders every lane's loads below after lane 0's acquire
            const float* all = part + static_cast<size_t>(i * heads + h) * nchunks * (HD + 2);
            // Every load of the merge in one round for up to 32 chunks: lane z reads chunk z's
            // (max, sum), and each lane its DPL dimensions of every chunk; more chunks take further
            // rounds of 32.
            float M = -INFINITY, L = 0.0f;
            float O[DPL];
#pragma unroll
            for (int cc = 0; cc < DPL; ++cc) O[cc] = 0.0f;
            for (int zb = 0; zb < nck; zb += 32) {
                const int zn = min(32, nck - zb);
                const float mz = lane < zn ? __ldcg(all + (zb + lane) * (HD + 2) + HD) : -INFINITY;
                const float lz = lane < zn ? __ldcg(all + (zb + lane) * (HD + 2) + HD + 1) : 0.0f;
                float ov[MB][DPL];
#pragma unroll
                for (int t = 0; t < MB; ++t) {
                    const int z = zb + min(t, zn - 1);
#pragma unroll
                    for (int cc = 0; cc < DPL; ++cc) ov[t][cc] = __ldcg(all + z * (HD + 2) + lane * DPL + cc);
                }
                // rescale what earlier rounds accumulated to the new running maximum
                const float Mn = fmaxf(M, warp_max(mz));
                const float carry = M == -INFINITY ? 0.0f : expf(M - Mn);
                const float wz = lane < zn ? expf(mz - Mn) : 0.0f;
                L = fmaf(L, carry, warp_sum(lz * wz));
#pragma unroll
                for (int cc = 0; cc < DPL; ++cc) O[cc] *= carry;
#pragma unroll
                for (int t0 = 0; t0 < 32; t0 += MB) {
                    if (t0 > 0) {
#pragma unroll
                        for (int t = 0; t < MB; ++t) {
                            const int z = zb + min(t0 + t, zn - 1);
#pragma unroll
                            for (int cc = 0; cc < DPL; ++cc) ov[t][cc] = __ldcg(all + z * (HD + 2) + lane * DPL + cc);
                        }
                    }
#pragma unroll
                    for (int t = 0; t < MB; ++t) {
                        const float wt = __shfl_sync(kFull, wz, t0 + t);
#pragma unroll
                        for (int cc = 0; cc < DPL; ++cc) O[cc] = fmaf(ov[t][cc], wt, O[cc]);
                    }
                }
                M = Mn;
            }
#pragma unroll
            for (int cc = 0; cc < DPL; ++cc) {
                out[static_cast<size_t>(i) * d + h * HD + lane * DPL + cc] = __fdiv_rn(O[cc], L);
            }
            if (lane == 0) tickets[i * heads + h] = 0;
            // Count the merge: a release of the output written above (ordered by __syncwarp).
            __syncwarp();
            if (lane == 0) atom_add_acq_rel(merged, 1);
        }
        __syncwarp();
    }
}

template <typename KT>
__device__ __forceinline__ void attention(int hd, int h, int worker, int workers, const float* q,
                                          const void* kc, const void* vc, const int* s_len, int R,
                                          int heads, int slots, int nchunks, float scale,
                                          float* part, int* tickets, float* out, unsigned* merged,
                                          float* qslot) {
    const KT* k = static_cast<const KT*>(kc);
    const KT* v = static_cast<const KT*>(vc);
    if (hd == 32) {
        attention_head<KT, 32>(h, worker, workers, q, k, v, s_len, R, heads, slots, nchunks, scale,
                               part, tickets, out, merged, qslot);
    } else if (hd == 64) {
        attention_head<KT, 64>(h, worker, workers, q, k, v, s_len, R, heads, slots, nchunks, scale,
                               part, tickets, out, merged, qslot);
    } else {
        attention_head<KT, 128>(h, worker, workers, q, k, v, s_len, R, heads, slots, nchunks, scale,
                                part, tickets, out, merged, qslot);
    }
}

// The head's block of the output projection for this CTA's columns [c0, c1) of d:
// opart[i][n] = sum_e att[i][e] * Wo[n][h * hd + e], with the weight vectors (16 bytes each, vpc
// per column) of the first round preloaded in `pre`.
template <typename WT, int RT>
__device__ __forceinline__ void head_output_block(const float* att, int R, int hd, int h, int d,
                                                  int c0, int c1, const WT* wo, const uint4* pre,
                                                  float* opart) {
    constexpr int VEC = Unpack<WT>::N;
    const int vpc = hd / VEC;  // a power of two <= 32: whole lane groups of one warp
    const int total = (c1 - c0) * vpc;
    const int rounds = (total + kThreads - 1) / kThreads;
#pragma unroll 1
    for (int r = 0; r < rounds; ++r) {
        const int e = r * kThreads + static_cast<int>(threadIdx.x);
        const bool act = e < total;
        const int col = c0 + (act ? e / vpc : 0), v = act ? e % vpc : 0;
        uint4 u = make_uint4(0, 0, 0, 0);
        if (act) {
            u = r == 0 ? pre[0]
                       : __ldg(reinterpret_cast<const uint4*>(wo + static_cast<size_t>(col) * d + h * hd) + v);
        }
        float wf[VEC];
        Unpack<WT>::run(u, wf);
        float acc[RT];
#pragma unroll
        for (int i = 0; i < RT; ++i) {
            acc[i] = 0.0f;
            if (act && i < R) {
#pragma unroll
                for (int c = 0; c < VEC; ++c) acc[i] = fmaf(wf[c], att[i * hd + v * VEC + c], acc[i]);
            }
        }
        for (int o = vpc >> 1; o > 0; o >>= 1) {
#pragma unroll
            for (int i = 0; i < RT; ++i) acc[i] += __shfl_xor_sync(kFull, acc[i], o);
        }
        if (act && v == 0) {
#pragma unroll
            for (int i = 0; i < RT; ++i) {
                if (i < R) opart[static_cast<size_t>(i) * d + col] = acc[i];
            }
        }
    }
}

template <typename WT, typename KT, int RT>
__global__ __launch_bounds__(kThreads, 1) void k_decode_step(FusedStep p,
                                                             const FusedLayer* __restrict__ layers) {
    // After a timed-out wait in an earlier step of the run, the barrier and head counters no
    // longer match what this launch expects: return at once (the host reports the error recorded
    // in *err once the run's queued steps have drained).
    if (__ldcg(p.err) != 0) return;
    extern __shared__ __align__(16) float smem[];
    __shared__ __align__(16) float qslot[kWarps * kMaxHeadDim];
    __shared__ __align__(16) float s_att[kMaxRows * kMaxHeadDim];
    __shared__ int abort_flag, s_len[kMaxRows], s_next[kMaxRows], s_rows[kMaxRows], s_step, s_last;
    __shared__ unsigned long long s_best[kMaxRows];
    __shared__ __align__(16) WStage s_stage[3];  // A: QKV slice / head, B: FFN1, C: FFN2
    const int R = p.R, d = p.d, F = p.F, H = p.H, L = p.L;
    const int hd = d / H;
    const int G = gridDim.x;
    const int cph = G / H;  // CTAs per head group
    const int grp = static_cast<int>(blockIdx.x) < cph * H ? static_cast<int>(blockIdx.x) / cph : -1;
    const int mem = static_cast<int>(blockIdx.x) % cph;
    const int own_ld = (d + G - 1) / G;
    const int widest = max(d, F);
    float* xs = smem;                                   // [R][max(d, F)] projection input
    float* xraw = xs + static_cast<size_t>(R) * widest;  // [R][d] residual stream x
    float* xprime = xraw + static_cast<size_t>(R) * d;  // [R][d] x + attention output
    float* lnA = xprime + static_cast<size_t>(R) * d;   // LayerNorm gamma, beta [2][d] (stage A)
    float* lnB = lnA + 2 * static_cast<size_t>(d);      // (stage B)
    float* xown = lnB + 2 * static_cast<size_t>(d);     // [R][own_ld]
    FusedLayer* lt = reinterpret_cast<FusedLayer*>(reinterpret_cast<unsigned char*>(smem) + p.table_offset);
    if (threadIdx.x == 0) {
        abort_flag = 0;
        s_step = __ldcg(p.step);
        unsigned char* base = reinterpret_cast<unsigned char*>(smem) + p.wstage_offset;
        const unsigned caps[3] = {p.wstage_a, p.wstage_b, p.wstage_c};
        float* lnps[3] = {lnA, lnB, nullptr};
        for (int b = 0; b < 3; ++b) {
            WStage& st = s_stage[b];
            st.buf = base;
            base += caps[b];
            st.lnp = lnps[b];
            st.cap = caps[b];
            st.parity = 0;
            st.cols = 0;
            st.pending = 0;
            mbar_init(&st.bar, 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x < R) {
        s_len[threadIdx.x] = __ldcg(p.len + threadIdx.x);
        s_next[threadIdx.x] = __ldcg(p.next + threadIdx.x);
        s_rows[threadIdx.x] = threadIdx.x;
        s_best[threadIdx.x] = 0ull;
    }
    // The per-layer table, copied to shared memory: read every phase, it must not depend on L1.
    {
        const unsigned long long* src = reinterpret_cast<const unsigned long long*>(layers);
        unsigned long long* dst = reinterpret_cast<unsigned long long*>(lt);
        const int words = L * static_cast<int>(sizeof(FusedLayer) / 8);
        for (int i = threadIdx.x; i < words; i += kThreads) dst[i] = src[i];
    }
    GridSync gsync{p.bar, p.bar_base, p.err, &abort_flag};
    __syncthreads();

    // Column blocks (kept in shared memory, read at phase boundaries): this CTA's QKV slice of its
    // head (virtual columns of the head's 3 * hd), its output-projection columns within the head
    // group, and its blocks of the grid-wide projections.
    enum { kQ0, kQ1, kO0, kO1, kF0, kF1, kD0, kD1, kV0, kV1 };
    __shared__ int cb[10];
    if (threadIdx.x == 0) {
        cb[kQ0] = cb[kQ1] = cb[kO0] = cb[kO1] = 0;
        if (grp >= 0) {
            block_of(3 * hd, cph, mem, &cb[kQ0], &cb[kQ1]);
            block_of(d, cph, mem, &cb[kO0], &cb[kO1]);
        }
        column_block(F, &cb[kF0], &cb[kF1]);
        column_block(d, &cb[kD0], &cb[kD1]);
        column_block(p.V, &cb[kV0], &cb[kV1]);
    }
    __syncthreads();
    stage_issue<WT>(lt[0].wqkv, d, cb[kQ0], cb[kQ1], ColMap{d, hd, grp}, lt[0].ln1_g, lt[0].ln1_b,
                    s_stage[0]);

    // embed, in every CTA: the full rows into xraw
    const WT* tok = static_cast<const WT*>(p.tok_emb);
    const WT* pos = static_cast<const WT*>(p.pos_emb);
    for (int e = threadIdx.x; e < R * d; e += kThreads) {
        const int i = e / d, k = e - i * d;
        xraw[e] = __fadd_rn(to_f(tok[static_cast<size_t>(s_next[i]) * d + k]),
                            to_f(pos[static_cast<size_t>(s_len[i]) * d + k]));
    }

    Sink sk;
    sk.xown = xown;
    sk.xown_ld = own_ld;
    sk.history = p.history;
    sk.step = s_step;
    sk.steps = p.steps;
    sk.best = s_best;
    // Head-group counters: [0, H) QKV arrivals (cph per layer), [H, 2H) merges (R per layer).
    unsigned* head_arrive = p.head_ctr;
    unsigned* head_merged = p.head_ctr + H;
    const unsigned arrive_base = p.launch_index * static_cast<unsigned>(L * cph);
    const unsigned merged_base = p.launch_index * static_cast<unsigned>(L * R);

    // Phase ph of the step: kind ph % 3 of layer ph / 3 (0: A, 1: B, 2: C), then the head. Each
    // phase has one LayerNorm site and one projection site, shared by all kinds.
    const int last = 3 * L;
    for (int ph = 0; ph <= last; ++ph) {
        const int kind = ph < last ? ph % 3 : 3;
        const int l = min(ph / 3, L - 1);
        const FusedLayer& lw = lt[l];
        // ---- before the projection ----
        uint4 wpre[kOPrefetch];
        if (kind == 0) {
            stage_issue<WT>(lw.w1, d, cb[kF0], cb[kF1], ColMap{}, lw.ln2_g, lw.ln2_b, s_stage[1]);
            if (l > 0) stage_rows(p.x, d, R, d, xraw);
            // The output-projection weights of this CTA's block, loaded early (they are constant).
            constexpr int VEC = Unpack<WT>::N;
            const int vpc = hd / VEC;
            const int total = grp >= 0 ? (cb[kO1] - cb[kO0]) * vpc : 0;
#pragma unroll
            for (int r = 0; r < kOPrefetch; ++r) {
                const int e = r * kThreads + static_cast<int>(threadIdx.x);
                wpre[r] = e < total ? __ldg(reinterpret_cast<const uint4*>(
                                          static_cast<const WT*>(lw.wo) +
                                          static_cast<size_t>(cb[kO0] + e / vpc) * d + grp * hd) + e % vpc)
                                    : make_uint4(0, 0, 0, 0);
            }
        } else if (kind == 1) {
            stage_issue<WT>(lw.w2, F, cb[kD0], cb[kD1], ColMap{}, nullptr, nullptr, s_stage[2]);
            // x' = x + (sum over heads of the partial output projections, in head order) + bias
            for (int e = threadIdx.x; e < R * d; e += kThreads) {
                const int i = e / d, n = e - i * d;
                float t[8];
                float o = 0.0f;
                for (int h0 = 0; h0 < H; h0 += 8) {
#pragma unroll
                    for (int z = 0; z < 8; ++z) {
                        t[z] = h0 + z < H ? __ldcg(p.opart + (static_cast<size_t>(h0 + z) * R + i) * d + n)
                                          : 0.0f;
                    }
#pragma unroll
                    for (int z = 0; z < 8; ++z) {
                        if (h0 + z < H) o += t[z];
                    }
                }
                o = __fadd_rn(o, __ldg(lw.bo + n));
                xprime[e] = __fadd_rn(xraw[e], o);
            }
        } else if (kind == 2) {
            if (l + 1 < L) {
                stage_issue<WT>(lt[l + 1].wqkv, d, cb[kQ0], cb[kQ1], ColMap{d, hd, grp},
                                lt[l + 1].ln1_g, lt[l + 1].ln1_b, s_stage[0]);
            } else {
                stage_issue<WT>(p.head_w, d, cb[kV0], cb[kV1], ColMap{}, p.lnf_g, p.lnf_b, s_stage[0]);
            }
            stage_rows(p.ffn, F, R, F, xs);
            const int n_own = cb[kD1] - cb[kD0];
            for (int e = threadIdx.x; e < R * n_own; e += kThreads) {
                const int i = e / n_own, j = e - i * n_own;
                xown[i * own_ld + j] = xprime[i * d + cb[kD0] + j];
            }
        } else {
            stage_rows(p.x, d, R, d, xraw);
        }
        // ---- the projection of this phase ----
        int c0, c1, K = d;
        ColMap cm{};
        const void* w;
        const float* bias;
        Epi epi;
        EpiArgs ea;
        int sidx;
        switch (kind) {
            case 0:
                c0 = cb[kQ0]; c1 = cb[kQ1]; cm = ColMap{d, hd, grp}; w = lw.wqkv; bias = lw.bqkv;
                epi = Epi::kQkv; sidx = 0;
                ea.out = p.q; ea.ldo = d; ea.rowmap = s_rows; ea.slot = s_len;
                ea.k_cache = lw.k_cache; ea.v_cache = lw.v_cache; ea.d = d; ea.heads = H;
                ea.head_dim = hd; ea.slots = p.slots; ea.kv_bf16 = sizeof(KT) == 2;
                break;
            case 1:
                c0 = cb[kF0]; c1 = cb[kF1]; w = lw.w1; bias = lw.b1; epi = Epi::kGelu; sidx = 1;
                ea.out = p.ffn; ea.ldo = F;
                break;
            case 2:
                c0 = cb[kD0]; c1 = cb[kD1]; K = F; w = lw.w2; bias = lw.b2; epi = Epi::kResidual;
                sidx = 2;
                ea.out = p.x; ea.ldo = d;
                break;
            default:
                c0 = cb[kV0]; c1 = cb[kV1]; w = p.head_w; bias = p.head_b; epi = Epi::kLogits;
                sidx = 0;
                ea.out = p.logits; ea.ldo = p.V;
                break;
        }
        __syncthreads();
        if (c1 > c0) {
            if (kind != 2) {
                // The projection's input: LayerNorm of x (A, head: published statistics after the
                // first layer) or of x' (B: computed here over the whole row).
                stage_wait(s_stage[sidx], p.err, &abort_flag);
                const bool use_stats = kind == 3 || (kind == 0 && l > 0);
                normalise_rows<RT>(kind == 1 ? xprime : xraw, R, d, use_stats ? p.stats : nullptr,
                                   p.eps, s_stage[sidx].lnp, xs);
            }
            gemv<WT, RT>(xs, R, K, c0, c1, cm, w, bias, epi, ea, sk, cb[kD0], s_stage[sidx], p.err,
                         &abort_flag);
        }
        // ---- after the projection ----
        if (kind == 0 && grp >= 0) {
            __syncthreads();
            if (threadIdx.x == 0) {
                atom_add_acq_rel(head_arrive + grp, 1);
                spin_until(head_arrive + grp, arrive_base + static_cast<unsigned>((l + 1) * cph),
                           p.err, 13, &abort_flag);
            }
            __syncthreads();
            const int warp = threadIdx.x >> 5;
            attention<KT>(hd, grp, warp * cph + mem, cph * kWarps, p.q, lw.k_cache, lw.v_cache,
                          s_len, R, H, p.slots, p.nchunks, p.scale, p.part, p.tickets, p.att,
                          head_merged + grp, qslot);
            __syncthreads();
            if (threadIdx.x == 0) {
                spin_until(head_merged + grp, merged_base + static_cast<unsigned>((l + 1) * R),
                           p.err, 13, &abort_flag);
            }
            __syncthreads();
            for (int e = threadIdx.x; e < R * hd; e += kThreads) {
                const int i = e / hd, k = e - i * hd;
                s_att[e] = __ldcg(p.att + static_cast<size_t>(i) * d + grp * hd + k);
            }
            __syncthreads();
            head_output_block<WT, RT>(s_att, R, hd, grp, d, cb[kO0], cb[kO1],
                                      static_cast<const WT*>(lw.wo), wpre,
                                      p.opart + static_cast<size_t>(grp) * R * d);
        } else if (kind == 2) {
            __syncthreads();
            publish_stats(xown, own_ld, cb[kD1] - cb[kD0], R, p.stats);
        }
        if (kind == 3) break;
        if (!grid_sync(gsync)) return;
    }

    // the head's per-row maxima, then the last CTA to get here finishes the step
    __syncthreads();
    if (threadIdx.x < R && s_best[threadIdx.x] != 0ull) {
        atomicMax(p.best + threadIdx.x, s_best[threadIdx.x]);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        s_last = atom_add_acq_rel(p.bar + 1, 1) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;

    // the last CTA: TextEngine.argmax (TextEngine.java:392-400) from the packed maxima, then the
    // step bookkeeping of TextEngine.push (TextEngine.java:387-390)
    __threadfence();
    __shared__ int s_token[kMaxRows];
    if (threadIdx.x < R) {
        const int i = threadIdx.x;
        const unsigned long long b = atomicExch(p.best + i, 0ull);
        const float first = __ldcg(p.logits + static_cast<size_t>(i) * p.V);
        int token = 0;
        if (!isnan(first) && b != 0ull) token = unpack_best_index(b);
        s_token[i] = token;
    }
    __syncthreads();
    for (int i = 0; i < R; ++i) {
        int* win = p.window + static_cast<size_t>(i) * p.W;
        for (int t0 = 0; t0 < p.W; t0 += kThreads) {
            const int t = t0 + threadIdx.x;
            const int v = t < p.W ? (t + 1 < p.W ? __ldcg(win + t + 1) : s_token[i]) : 0;
            __syncthreads();
            if (t < p.W) win[t] = v;
            __syncthreads();
        }
    }
    if (threadIdx.x < R) {
        const int i = threadIdx.x;
        p.tokens[static_cast<size_t>(i) * p.steps + s_step] = s_token[i];
        p.next[i] = s_token[i];
        p.len[i] = s_len[i] + 1;
    }
    if (threadIdx.x == 0) {
        *p.step = s_step + 1;
        p.bar[1] = 0;
    }
}

// Shared-memory layout of one CTA: activations, LayerNorm parameters and residual columns
// (floats), the layer table, then the three weight stages (A: a head's QKV slice, later the head
// projection; B: FFN1; C: FFN2), each as large as its rows need within the remaining budget.
struct Layout {
    size_t table_offset = 0;
    size_t stage_offset = 0;
    unsigned stage_a = 0, stage_b = 0, stage_c = 0;
    size_t total = 0;
    bool ok = false;
};

Layout fused_layout(int R, int d, int F, int V, int L, int H, int ctas, int wbytes) {
    Layout lay;
    if (H < 1 || ctas < H) return lay;
    const size_t own_ld = (d + ctas - 1) / ctas;
    const size_t floats = static_cast<size_t>(R) * (std::max(d, F) + 2 * d) + 4 * d +
                          (R * own_ld + 3) / 4 * 4;
    lay.table_offset = (floats * sizeof(float) + 15) / 16 * 16;
    lay.stage_offset = (lay.table_offset + sizeof(FusedLayer) * L + 127) / 128 * 128;
    if (lay.stage_offset > kSmemLimit) return lay;
    const int cph = ctas / H, hd = d / H;
    auto up = [](size_t x) { return (x + 15) / 16 * 16; };
    const size_t need_a = up(std::max(static_cast<size_t>((3 * hd + cph - 1) / cph),
                                      static_cast<size_t>((V + ctas - 1) / ctas)) * d * wbytes);
    const size_t need_b = up(static_cast<size_t>((F + ctas - 1) / ctas) * d * wbytes);
    const size_t need_c = up(static_cast<size_t>((d + ctas - 1) / ctas) * F * wbytes);
    const size_t room = (kSmemLimit - lay.stage_offset) / 16 * 16;
    const size_t need = need_a + need_b + need_c;
    if (need <= room) {
        lay.stage_a = static_cast<unsigned>(need_a);
        lay.stage_b = static_cast<unsigned>(need_b);
        lay.stage_c = static_cast<unsigned>(need_c);
    } else {
        // Proportional shares, whole 16-byte units; the rows beyond come from global memory.
        lay.stage_a = static_cast<unsigned>(room * need_a / need / 16 * 16);
        lay.stage_b = static_cast<unsigned>(room * need_b / need / 16 * 16);
        lay.stage_c = static_cast<unsigned>(room * need_c / need / 16 * 16);
    }
    lay.total = lay.stage_offset + lay.stage_a + lay.stage_b + lay.stage_c;
    lay.ok = true;
    return lay;
}

template <typename WT, typename KT, int RT>
int prepare_typed(int R, int d, int F, int V, int L, int H) {
    auto kernel = k_decode_step<WT, KT, RT>;
    int device = 0, sms = 0, coop = 0;
    if (cudaGetDevice(&device) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    const Layout lay = fused_layout(R, d, F, V, L, H, sms, sizeof(WT));
    if (!coop || !lay.ok || sms > 256) return 0;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmemLimit)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, lay.total) !=
        cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return per_sm >= 1 ? sms : 0;
}

template <typename WT, typename KT, int RT>
cudaError_t launch_typed(cudaStream_t s, const FusedStep& p, const FusedLayer* layers, int ctas,
                         size_t smem) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_decode_step<WT, KT, RT>, p, layers);
}

struct Prepare {
    int R, d, F, V, L, H;
    template <typename WT, typename KT, int RT>
    int run() const { return prepare_typed<WT, KT, RT>(R, d, F, V, L, H); }
};

struct Launch {
    cudaStream_t s;
    const FusedStep& p;
    const FusedLayer* layers;
    int ctas;
    size_t smem;
    template <typename WT, typename KT, int RT>
    cudaError_t run() const { return launch_typed<WT, KT, RT>(s, p, layers, ctas, smem); }
};

// fn.run<WT, KT, RT>() for the runtime weight type, cache type and row count (RT = 1 for one row,
// 8 for two to eight).
template <typename Fn>
auto dispatch(int w_bf16, int kv_bf16, int R, const Fn& fn) {
    if (R == 1) {
        if (w_bf16) {
            return kv_bf16 ? fn.template run<__nv_bfloat16, __nv_bfloat16, 1>()
                           : fn.template run<__nv_bfloat16, float, 1>();
        }
        return kv_bf16 ? fn.template run<float, __nv_bfloat16, 1>() : fn.template run<float, float, 1>();
    }
    if (w_bf16) {
        return kv_bf16 ? fn.template run<__nv_bfloat16, __nv_bfloat16, kMaxRows>()
                       : fn.template run<__nv_bfloat16, float, kMaxRows>();
    }
    return kv_bf16 ? fn.template run<float, __nv_bfloat16, kMaxRows>()
                   : fn.template run<float, float, kMaxRows>();
}

}  // namespace

bool fused_decode_supported(int R, int d, int F, int W, int hd, int w_bf16) {
    if (R < 1 || R > kMaxRows || W < 1 || W > kMaxChunkGroups * 32 * kChunk) return false;
    if (hd != 32 && hd != 64 && hd != 128) return false;
    const int vec = w_bf16 ? 8 : 4;
    return d % vec == 0 && F % vec == 0;
}

int fused_decode_prepare(int R, int d, int F, int V, int L, int hd, int w_bf16, int kv_bf16) {
    return dispatch(w_bf16, kv_bf16, R, Prepare{R, d, F, V, L, d / hd});
}

int fused_decode_barriers(int layers) { return 3 * layers; }

cudaError_t launch_decode_fused(cudaStream_t s, const FusedStep& step, const FusedLayer* layers,
                                int w_bf16, int kv_bf16, int hd, int ctas) {
    (void)hd;
    const Layout lay = fused_layout(step.R, step.d, step.F, step.V, step.L, step.H, ctas,
                                    w_bf16 ? 2 : 4);
    if (!lay.ok) return cudaErrorInvalidValue;
    FusedStep p = step;
    p.table_offset = static_cast<unsigned>(lay.table_offset);
    p.wstage_offset = static_cast<unsigned>(lay.stage_offset);
    p.wstage_a = lay.stage_a;
    p.wstage_b = lay.stage_b;
    p.wstage_c = lay.stage_c;
    return dispatch(w_bf16, kv_bf16, p.R, Launch{s, p, layers, ctas, lay.total});
}

}  // namespace bst
