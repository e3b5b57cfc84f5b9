// One greedy decode step of the (padded) decoder for small batches, as one persistent kernel.
//
// At batch 1 a decode step is ~60 small dependent operations (per layer: LayerNorm + QKV,
// attention, output projection, LayerNorm + FFN1, FFN2; then the head and the argmax). Launched as
// separate kernels each pays a launch, a ramp-up and a DRAM round trip with most SMs idle. Here a
// single cooperative launch runs the whole step: one CTA per SM, 16 warps each, phases separated
// by a grid barrier. Every projection spreads its weight rows over all SMs, so each weight byte is
// read once per step with the whole chip's memory parallelism. Weights are constant during the
// step: before the grid barrier that precedes a projection, each CTA has the TMA unit copy its
// block of weight rows into shared memory (cp.async.bulk into this CTA only), so the weight stream
// overlaps the barrier and the input staging.
//
// Phases (R <= 8 rows, every row extending its cache; TransformerBlock.forward,
// torch/TransformerBlock.java:37-43, inside the padded decoder whose last-position head follows
// TextEngine.scores, infer/TextEngine.java:96-112):
//   embed      every CTA computes x[i] = tok[next[i]] + pos[len[i]] itself (no barrier)
//   per layer  QKV (LN1 fused; K/V stored at slot len[i]) | attention (one warp per 32-key
//              chunk; the last chunk of a (row, head) merges the chunk partials in chunk order) |
//              O + residual | FFN1 (LN2 fused) + GELU | FFN2 + residual
//   head       logits (final LN fused) and each CTA's first maximum, combined with a 64-bit
//              atomic max; the last CTA to finish (ticket) applies TextEngine.argmax's rule, pushes
//              the token into the window and advances the step counter and lengths.
// Each CTA owns the same block of residual columns of x in every phase and keeps it in shared
// memory, so residual updates need no load.
//
// Code size matters as much as memory here: a phase runs for a few microseconds, too short to
// amortise instruction fetches from L2. All projection phases therefore share one non-inlined
// routine (the epilogue is chosen at run time) and attention is one routine per head size, so the
// code a layer runs stays resident in the instruction cache. The row count is a template
// parameter (1, or up to 8) so that batch 1 carries no code for other rows.
//
// Memory coherence: activations, the cache, scores and counters are written inside the kernel by
// other CTAs, so they are read with ld.global.cg (L2) after the barrier's acquire, never through
// the non-coherent read-only path; only weights and embeddings use that path. Every wait (grid
// barrier, weight stage) is bounded by %globaltimer: on expiry it records an error code in *err
// (11: grid barrier, 12: weight stage) and the CTAs return at the next barrier.

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
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s bound on any single wait
constexpr size_t kSmemLimit = 212 * 1024;    // dynamic shared memory of one CTA
constexpr size_t kStageMax = 96 * 1024;      // weight stage

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
        const unsigned old = atom_add_acq_rel(g.count, 1);
        if (static_cast<int>(old + 1 - g.target) < 0) {
            const uint64_t start = global_ns();
            while (static_cast<int>(ld_acquire(g.count) - g.target) < 0) {
                if (global_ns() - start > kWaitNs) {
                    atomicCAS(g.err, 0, 11);
                    *g.abort_flag = 1;
                    break;
                }
            }
        }
    }
    __syncthreads();
    return *reinterpret_cast<volatile int*>(g.abort_flag) == 0;
}

// This CTA's share of an [N, K] weight matrix in a projection phase: a block of whole rows.
__device__ __forceinline__ void column_block(int N, int* c0, int* c1) {
    const int cpc = (N + gridDim.x - 1) / gridDim.x;
    *c0 = min(N, static_cast<int>(blockIdx.x) * cpc);
    *c1 = min(N, *c0 + cpc);
}

// How a CTA's threads cover its columns of a projection with nvec 16-byte weight vectors per
// column. Up to 16 columns: `ks` whole warps per column, each on a contiguous part of K. More
// columns: groups of `gs` lanes (a power of two) per column, repeated `reps` times when there are
// more columns than groups.
struct Plan {
    int c0, c1;
    int gs, ks, reps;
    int col;         // this thread's column in rep 0 (absolute)
    int col_stride;  // column step between reps
    int vbeg, vend, vstep;
    int part;        // warp's part of its column (gs == 32)
};

__device__ __forceinline__ Plan make_plan(int N, int nvec) {
    Plan p;
    column_block(N, &p.c0, &p.c1);
    const int ncols = p.c1 - p.c0;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (ncols <= kWarps) {
        p.gs = 32;
        p.ks = ncols > 0 ? kWarps / ncols : 1;
        p.reps = 1;
        p.part = warp % p.ks;
        p.col = p.c0 + warp / p.ks;
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
        p.col = p.c0 + tid / gs;
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

// The CTA's weight stage: a shared-memory buffer the TMA unit fills with the CTA's block of the
// next projection's weight rows (as many whole rows as fit; the rest is read from global memory),
// plus the bias of those rows and the LayerNorm parameters of the projection's input.
struct WStage {
    uint64_t* bar;          // mbarrier (shared), one phase per issued copy
    unsigned char* buf;     // weight rows (shared)
    unsigned cap;           // bytes
    float* bias;            // [columns + 4] (shared), column c0 + j at bias[j + bias_off]
    float* lnp;             // gamma [K], beta [K] (shared)
    int* abort_flag;        // shared
    int* err;
    unsigned parity;        // phase the next wait expects
    int cols;               // weight rows of the current projection held in buf
    int bias_off;           // bias block starts bias_off floats before column c0
    bool pending;           // a copy was issued and not yet waited for
};

// Issues the stage of the projection Y[R, N] = X W^T (W [N, K] of WT) for this CTA.
template <typename WT>
__device__ __forceinline__ void stage_issue(const void* w, const float* bias, int N, int K,
                                         const float* ln_gamma, const float* ln_beta, WStage& st) {
    int c0, c1;
    column_block(N, &c0, &c1);
    const size_t row_bytes = static_cast<size_t>(K) * sizeof(WT);
    st.cols = c1 > c0 ? min(c1 - c0, static_cast<int>(st.cap / row_bytes)) : 0;
    st.bias_off = c0 & 3;
    st.pending = c1 > c0;
    if (c1 <= c0) return;  // uniform over the CTA
    // Every thread is done with the previous projection's stage: hand it to the TMA unit. All of
    // it arrives by bulk copies on one mbarrier: the weight rows, the LayerNorm parameters and the
    // bias block (its start rounded down, its end up, to 16 bytes).
    __syncthreads();
    if (threadIdx.x == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        const uint32_t wbytes = static_cast<uint32_t>(st.cols * row_bytes);
        const uint32_t lbytes = ln_gamma ? static_cast<uint32_t>(K) * 4u : 0u;
        const uint32_t bbytes = bias ? static_cast<uint32_t>((c1 - c0 + st.bias_off + 3) / 4 * 16) : 0u;
        mbar_expect_tx(st.bar, wbytes + 2 * lbytes + bbytes);
        if (wbytes) {
            bulk_load(st.buf, static_cast<const WT*>(w) + static_cast<size_t>(c0) * K, wbytes, st.bar);
        }
        if (lbytes) {
            bulk_load(st.lnp, ln_gamma, lbytes, st.bar);
            bulk_load(st.lnp + K, ln_beta, lbytes, st.bar);
        }
        if (bbytes) bulk_load(st.bias, bias + (c0 - st.bias_off), bbytes, st.bar);
    }
}

// Waits for the stage issued by stage_issue (bounded; on expiry records code 12, waits once more
// for the copy to land and lets the next grid barrier end the kernel).
__device__ __forceinline__ void stage_wait(WStage& st) {
    if (st.pending) {
        if (!mbar_try_wait(st.bar, st.parity)) {
            uint64_t start = global_ns();
            bool late = false;
            while (!mbar_try_wait(st.bar, st.parity)) {
                if (global_ns() - start > kWaitNs) {
                    if (late) break;
                    atomicCAS(st.err, 0, 12);
                    *st.abort_flag = 1;
                    late = true;
                    start = global_ns();
                }
            }
        }
        st.parity ^= 1u;
        st.pending = false;
    }
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

// One output of a projection through its epilogue (chosen at run time).
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

// Mean and 1/sqrt(var + eps) of R rows of width d from the published per-CTA statistics; the
// last R warps handle a row each (warp kWarps - R + i row i), so that their loads overlap the
// row staging that the first threads of the CTA do. Results in mean[i], inv[i] (shared) after
// the caller's __syncthreads().
__device__ __forceinline__ void combine_stats(const double* stats, int R, int d, float eps,
                                              double* mean, double* inv) {
    const int warp = (threadIdx.x >> 5) - (kWarps - R), lane = threadIdx.x & 31;
    if (warp < 0) return;
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

// Per-CTA state shared by the projection phases.
struct Ctx {
    float* xs;    // [R][max(d, F)] projection input (shared)
    float* xraw;  // [R][d] rows before LayerNorm (shared)
    int R;
    float eps;
    const double* stats;  // published per-CTA statistics of the input rows (LayerNorm phases)
};

// Y[R, N] = X[R, K] * W[N, K]^T + bias over the whole grid with the weights staged by
// stage_issue. The input rows are staged in shared memory (already in xraw when `staged`),
// layer-normalised first when `ln`. Partial sums are combined in a fixed order, so results repeat
// bit for bit.
template <typename WT, int RT>
__device__ __forceinline__ void gemv(const float* x, int ldx, bool staged, bool ln, bool use_stats,
                                  const void* wv, bool has_bias, int N, int K, Epi epi,
                                  const EpiArgs& ea, const Sink& sk, const Ctx& cx, WStage& st) {
    constexpr int VEC = Unpack<WT>::N;
    __shared__ float red[kWarps][RT];
    const int R = cx.R;
    float* xs = cx.xs;
    const int nvec = K / VEC;
    const Plan pl = make_plan(N, nvec);
    if (pl.c1 <= pl.c0) return;  // uniform over the CTA
    if (ln && use_stats) {
        __shared__ double s_mean[RT], s_inv[RT];
        stage_rows(x, ldx, R, K, cx.xraw);
        combine_stats(cx.stats, R, K, cx.eps, s_mean, s_inv);
        stage_wait(st);
        __syncthreads();
        for (int e = threadIdx.x; e < R * K; e += kThreads) {
            const int i = e / K, k = e - i * K;
            const float nrm = static_cast<float>(
                __dmul_rn(__dadd_rn(static_cast<double>(cx.xraw[e]), -s_mean[i]), s_inv[i]));
            xs[e] = __fadd_rn(__fmul_rn(nrm, st.lnp[k]), st.lnp[K + k]);
        }
    } else if (ln) {
        if (!staged) stage_rows(x, ldx, R, K, cx.xraw);
        stage_wait(st);
        __syncthreads();
        const LnArgs lns{st.lnp, st.lnp + K, cx.eps};
        layernorm_rows(cx.xraw, K, RT == 1 ? 1 : R, K, lns, xs);
    } else {
        stage_rows(x, ldx, R, K, xs);
        stage_wait(st);
    }
    __syncthreads();
    const WT* w = static_cast<const WT*>(wv);
    const uint4* staged_w = reinterpret_cast<const uint4*>(st.buf);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int rep = 0; rep < pl.reps; ++rep) {
        const int col = pl.col + rep * pl.col_stride;
        const bool act = col < pl.c1;
        float acc[RT];
#pragma unroll
        for (int i = 0; i < RT; ++i) acc[i] = 0.0f;
        if (act) {
            const bool in_smem = col - pl.c0 < st.cols;
            const uint4* wc = in_smem ? staged_w + static_cast<size_t>(col - pl.c0) * nvec
                                      : reinterpret_cast<const uint4*>(w + static_cast<size_t>(col) * K);
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
            const float b = has_bias ? st.bias[col - pl.c0 + st.bias_off] : 0.0f;
#pragma unroll
            for (int i = 0; i < RT; ++i) {
                if (i < R) store_out(epi, ea, sk, pl.c0, i, col, has_bias ? __fadd_rn(acc[i], b) : acc[i]);
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

// Decode attention over every (row, head, 32-key chunk) that holds keys: one warp per chunk. Lanes
// own keys for the scores; for P.V lanes own (key group, 16-byte slice of the head) pairs so that
// every V load of the chunk is independent. The last chunk of a (row, head) to finish (ticket)
// merges the chunk partials in chunk order, lanes in parallel over chunks and dimensions.
template <typename KT, int HD>
__device__ __forceinline__ void attention_phase(const float* q, const KT* kc, const KT* vc, const int* s_len,
                                int R, int heads, int slots, int nchunks, float scale, float* part,
                                int* tickets, float* out, float* qslot) {
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
    const int tasks = R * heads * nchunks;
    // Task t runs on CTA t % grid: consecutive chunks land on different SMs.
    for (int task = warp * gridDim.x + blockIdx.x; task < tasks; task += gridDim.x * kWarps) {
        const int i = task / (heads * nchunks);
        const int rem = task - i * heads * nchunks;
        const int h = rem / nchunks, c = rem - h * nchunks;
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
        }
        __syncwarp();
    }
}

template <typename KT>
__device__ __forceinline__ void attention(int hd, const float* q, const void* kc, const void* vc,
                                          const int* s_len, int R, int heads, int slots,
                                          int nchunks, float scale, float* part, int* tickets,
                                          float* out, float* qslot) {
    const KT* k = static_cast<const KT*>(kc);
    const KT* v = static_cast<const KT*>(vc);
    if (hd == 32) {
        attention_phase<KT, 32>(q, k, v, s_len, R, heads, slots, nchunks, scale, part, tickets, out, qslot);
    } else if (hd == 64) {
        attention_phase<KT, 64>(q, k, v, s_len, R, heads, slots, nchunks, scale, part, tickets, out, qslot);
    } else {
        attention_phase<KT, 128>(q, k, v, s_len, R, heads, slots, nchunks, scale, part, tickets, out, qslot);
    }
}

// Operands of one projection phase. Phase p < 5L is kind p % 5 of layer p / 5 (0 QKV, 1 attention,
// 2 output projection, 3 FFN1, 4 FFN2); phase 5L is the head.
struct ProjDesc {
    const void* w;
    const float* bias;
    const float* ln_g;  // input LayerNorm (nullptr: none)
    const float* ln_b;
    const float* x;     // input rows
    int ldx, N, K;
    Epi epi;
};

__device__ __forceinline__ ProjDesc describe(const FusedStep& p, const FusedLayer* lt, int phase) {
    ProjDesc pd;
    const int d = p.d;
    if (phase >= 5 * p.L) {
        pd = ProjDesc{p.head_w, p.head_b, p.lnf_g, p.lnf_b, p.x, d, p.V, d, Epi::kLogits};
        return pd;
    }
    const FusedLayer& lw = lt[phase / 5];
    switch (phase % 5) {
        case 0: pd = ProjDesc{lw.wqkv, lw.bqkv, lw.ln1_g, lw.ln1_b, p.x, d, 3 * d, d, Epi::kQkv}; break;
        case 2: pd = ProjDesc{lw.wo, lw.bo, nullptr, nullptr, p.att, d, d, d, Epi::kResidual}; break;
        case 3: pd = ProjDesc{lw.w1, lw.b1, lw.ln2_g, lw.ln2_b, p.x, d, p.F, d, Epi::kGelu}; break;
        case 4: pd = ProjDesc{lw.w2, lw.b2, nullptr, nullptr, p.ffn, p.F, d, p.F, Epi::kResidual}; break;
        default: pd = ProjDesc{nullptr, nullptr, nullptr, nullptr, nullptr, 0, 0, 0, Epi::kStore}; break;
    }
    return pd;
}

template <typename WT, typename KT, int RT>
__global__ __launch_bounds__(kThreads, 1) void k_decode_step(FusedStep p,
                                                             const FusedLayer* __restrict__ layers) {
    extern __shared__ __align__(16) float smem[];
    __shared__ __align__(16) float qslot[kWarps * 128];
    __shared__ int abort_flag, s_len[kMaxRows], s_next[kMaxRows], s_rows[kMaxRows], s_step, s_last;
    __shared__ unsigned long long s_best[kMaxRows];
    __shared__ __align__(8) uint64_t s_wbar;
    // After a timed-out barrier or weight stage in an earlier step of the run, the barrier count
    // no longer matches what this launch expects: return at once (the host reports the error
    // recorded in *err once the run's queued steps have drained).
    if (__ldcg(p.err) != 0) return;
    const int R = p.R, d = p.d, F = p.F;
    int dc0, dc1;
    column_block(d, &dc0, &dc1);
    const int own_ld = (d + gridDim.x - 1) / gridDim.x;
    float* xs = smem;                                        // [R][max(d, F)]
    float* xraw = xs + static_cast<size_t>(R) * max(d, F);   // [R][d]
    float* lnp = xraw + static_cast<size_t>(R) * d;          // LayerNorm gamma, beta [2][d]
    float* xown = lnp + 2 * static_cast<size_t>(d);          // [R][own_ld]
    float* bsm = xown + ((R * own_ld + 3) & ~3);             // [bias_cap], 16-byte aligned
    FusedLayer* lt = reinterpret_cast<FusedLayer*>(reinterpret_cast<unsigned char*>(smem) + p.table_offset);
    unsigned char* wbuf = reinterpret_cast<unsigned char*>(smem) + p.wstage_offset;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        s_step = __ldcg(p.step);
        mbar_init(&s_wbar, 1);
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
        const int words = p.L * static_cast<int>(sizeof(FusedLayer) / 8);
        for (int i = threadIdx.x; i < words; i += kThreads) dst[i] = src[i];
    }
    GridSync gsync{p.bar, p.bar_base, p.err, &abort_flag};
    WStage st{&s_wbar, wbuf, p.wstage_bytes, bsm, lnp, &abort_flag, p.err, 0u, 0, 0, false};
    const Ctx cx{xs, xraw, R, p.eps, p.stats};
    __syncthreads();
    {
        const ProjDesc pd = describe(p, lt, 0);
        stage_issue<WT>(pd.w, pd.bias, pd.N, pd.K, pd.ln_g, pd.ln_b, st);
    }

    // embed, in every CTA: the full rows into xraw; the CTA's own columns into xown and x
    const WT* tok = static_cast<const WT*>(p.tok_emb);
    const WT* pos = static_cast<const WT*>(p.pos_emb);
    for (int e = threadIdx.x; e < R * d; e += kThreads) {
        const int i = e / d, k = e - i * d;
        const float v = __fadd_rn(to_f(tok[static_cast<size_t>(s_next[i]) * d + k]),
                                  to_f(pos[static_cast<size_t>(s_len[i]) * d + k]));
        xraw[e] = v;
        if (k >= dc0 && k < dc1) {
            xown[i * own_ld + (k - dc0)] = v;
            p.x[e] = v;
        }
    }

    Sink sk;
    sk.xown = xown;
    sk.xown_ld = own_ld;
    sk.history = p.history;
    sk.step = s_step;
    sk.steps = p.steps;
    sk.best = s_best;
    const int hd = d / p.H;
    const int last = 5 * p.L;
    for (int phase = 0; phase <= last; ++phase) {
        const int kind = phase < last ? phase % 5 : 5;
        const FusedLayer& lw = lt[min(phase / 5, p.L - 1)];
        if (kind == 1) {
            attention<KT>(hd, p.q, lw.k_cache, lw.v_cache, s_len, R, p.H, p.slots, p.nchunks,
                          p.scale, p.part, p.tickets, p.att, qslot);
        } else {
            const ProjDesc pd = describe(p, lt, phase);
            EpiArgs ea;
            ea.out = kind == 0 ? p.q : kind == 3 ? p.ffn : kind == 5 ? p.logits : p.x;
            ea.ldo = kind == 3 ? F : kind == 5 ? p.V : d;
            ea.rowmap = s_rows;
            ea.slot = s_len;
            ea.k_cache = lw.k_cache;
            ea.v_cache = lw.v_cache;
            ea.d = d;
            ea.heads = p.H;
            ea.head_dim = hd;
            ea.slots = p.slots;
            ea.kv_bf16 = sizeof(KT) == 2;
            // LayerNorm inputs after a residual phase use its published statistics; layer 0's
            // input comes from the embedding every CTA computed itself.
            gemv<WT, RT>(pd.x, pd.ldx, phase == 0, pd.ln_g != nullptr, phase > 0, pd.w,
                         pd.bias != nullptr, pd.N, pd.K, pd.epi, ea, sk, cx, st);
            if (kind == 2 || kind == 4) {
                __syncthreads();
                publish_stats(xown, own_ld, dc1 - dc0, R, p.stats);
            }
        }
        if (phase == last) break;
        if (kind != 0) {  // the next phase is a projection: stage its weights before the barrier
            const ProjDesc nd = describe(p, lt, phase + 1);
            stage_issue<WT>(nd.w, nd.bias, nd.N, nd.K, nd.ln_g, nd.ln_b, st);
        }
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
        if (!isnan(first) && b != 0ull) token = static_cast<int>(0xffffffffu - static_cast<unsigned>(b));
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

// Shared-memory layout of one CTA: activations, LayerNorm parameters, residual columns and bias
// (floats), the layer table, then the weight stage (the rest of the budget, at most kStageMax).
struct Layout {
    size_t table_offset = 0;
    size_t stage_offset = 0;
    unsigned stage_bytes = 0;
    size_t total = 0;
    bool ok = false;
};

Layout fused_layout(int R, int d, int F, int V, int L, int ctas) {
    Layout lay;
    const size_t own_ld = (d + ctas - 1) / ctas;
    const size_t widest = std::max({static_cast<size_t>(3) * d, static_cast<size_t>(F),
                                    static_cast<size_t>(V)});
    const size_t bias_cap = ((widest + ctas - 1) / ctas + 3) / 4 * 4 + 4;
    const size_t floats = static_cast<size_t>(R) * (std::max(d, F) + d) + 2 * d +
                          (R * own_ld + 3) / 4 * 4 + bias_cap;
    lay.table_offset = (floats * sizeof(float) + 15) / 16 * 16;
    lay.stage_offset = (lay.table_offset + sizeof(FusedLayer) * L + 127) / 128 * 128;
    if (lay.stage_offset > kSmemLimit) return lay;
    lay.stage_bytes = static_cast<unsigned>(std::min(kStageMax, kSmemLimit - lay.stage_offset) / 16 * 16);
    lay.total = lay.stage_offset + lay.stage_bytes;
    lay.ok = true;
    return lay;
}

template <typename WT, typename KT, int RT>
int prepare_typed(int R, int d, int F, int V, int L) {
    auto kernel = k_decode_step<WT, KT, RT>;
    int device = 0, sms = 0, coop = 0;
    if (cudaGetDevice(&device) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    const Layout lay = fused_layout(R, d, F, V, L, sms);
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
cudaError_t launch_typed(cudaStream_t s, const FusedStep& p, const FusedLayer* layers, int ctas) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = p.wstage_offset + p.wstage_bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_decode_step<WT, KT, RT>, p, layers);
}

struct Prepare {
    int R, d, F, V, L;
    template <typename WT, typename KT, int RT>
    int run() const { return prepare_typed<WT, KT, RT>(R, d, F, V, L); }
};

struct Launch {
    cudaStream_t s;
    const FusedStep& p;
    const FusedLayer* layers;
    int ctas;
    template <typename WT, typename KT, int RT>
    cudaError_t run() const { return launch_typed<WT, KT, RT>(s, p, layers, ctas); }
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
    (void)hd;
    return dispatch(w_bf16, kv_bf16, R, Prepare{R, d, F, V, L});
}

int fused_decode_barriers(int layers) { return 5 * layers; }

cudaError_t launch_decode_fused(cudaStream_t s, const FusedStep& step, const FusedLayer* layers,
                                int w_bf16, int kv_bf16, int hd, int ctas) {
    (void)hd;
    const Layout lay = fused_layout(step.R, step.d, step.F, step.V, step.L, ctas);
    if (!lay.ok) return cudaErrorInvalidValue;
    FusedStep p = step;
    p.table_offset = static_cast<unsigned>(lay.table_offset);
    p.wstage_offset = static_cast<unsigned>(lay.stage_offset);
    p.wstage_bytes = lay.stage_bytes;
    return dispatch(w_bf16, kv_bf16, p.R, Launch{s, p, layers, ctas});
}

}  // namespace bst
