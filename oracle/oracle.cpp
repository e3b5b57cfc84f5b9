// CPU oracle for the TextEngine decode path — TEST INFRASTRUCTURE ONLY (see oracle.h).
//
// Every function names the reference file:line it restates. Numerics follow the reference
// exactly where the reference fixes them (operation order, fused vs separate multiply-add,
// f64 LayerNorm statistics); libm's expf/tanhf/exp stand in for Rust's f32::exp/tanh and
// Java's Math.exp, which may differ from them by at most one ulp.
//
// Build with -ffp-contract=off: the reference's scalar code never contracts a*b+c.

#include "oracle.h"

#include <immintrin.h>
#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

namespace {

// ---------------------------------------------------------------------------------------------
// java.util.Random — JDK specification (java/util/Random.java: setSeed, next, nextInt,
// nextInt(bound), nextFloat, nextDouble, nextGaussian). Used at TextEngine.java:43,288-290,417.
// ---------------------------------------------------------------------------------------------
constexpr uint64_t kMultiplier = 0x5DEECE66DULL;
constexpr uint64_t kAddend = 0xBULL;
constexpr uint64_t kMask = (1ULL << 48) - 1;

}  // namespace

extern "C" void orc_random_set_seed(orc_random* r, int64_t seed) {
    r->seed = (static_cast<uint64_t>(seed) ^ kMultiplier) & kMask;
    r->have_next_gaussian = 0;
    r->next_gaussian = 0.0;
}

extern "C" int32_t orc_random_next(orc_random* r, int32_t bits) {
    r->seed = (r->seed * kMultiplier + kAddend) & kMask;
    return static_cast<int32_t>(static_cast<int64_t>(r->seed) >> (48 - bits));
}

extern "C" int32_t orc_random_next_int(orc_random* r) { return orc_random_next(r, 32); }

extern "C" int32_t orc_random_next_int_bound(orc_random* r, int32_t bound) {
    if (bound <= 0) return -1;
    int32_t value = orc_random_next(r, 31);
    const int32_t m = bound - 1;
    if ((bound & m) == 0) {
        return static_cast<int32_t>((static_cast<int64_t>(bound) * value) >> 31);
    }
    // Rejection loop of the JDK: retry while u - r + m overflows int.
    for (int32_t u = value;; u = orc_random_next(r, 31)) {
        value = u % bound;
        if (static_cast<int32_t>(static_cast<uint32_t>(u) - static_cast<uint32_t>(value) +
                                 static_cast<uint32_t>(m)) >= 0) {
            break;
        }
    }
    return value;
}

extern "C" float orc_random_next_float(orc_random* r) {
    return static_cast<float>(orc_random_next(r, 24)) / static_cast<float>(1 << 24);
}

extern "C" double orc_random_next_double(orc_random* r) {
    const int64_t high = static_cast<int64_t>(orc_random_next(r, 26));
    const int64_t low = static_cast<int64_t>(orc_random_next(r, 27));
    return static_cast<double>((high << 27) + low) * 0x1.0p-53;
}

extern "C" double orc_random_next_gaussian(orc_random* r) {
    if (r->have_next_gaussian) {
        r->have_next_gaussian = 0;
        return r->next_gaussian;
    }
    double v1, v2, s;
    do {
        v1 = 2 * orc_random_next_double(r) - 1;
        v2 = 2 * orc_random_next_double(r) - 1;
        s = v1 * v1 + v2 * v2;
    } while (s >= 1 || s == 0);
    // StrictMath.sqrt is correctly rounded like sqrt(); StrictMath.log (fdlibm) and glibc log
    // agree except for rare last-ulp cases.
    const double multiplier = std::sqrt(-2 * std::log(s) / s);
    r->next_gaussian = v2 * multiplier;
    r->have_next_gaussian = 1;
    return v1 * multiplier;
}

namespace {

// ---------------------------------------------------------------------------------------------
// gemm.rs restatement. Per output element the reference computes a k-ordered sum starting from
// +0.0: with FMA inside the 6x16-tiled region (gemm.rs:190-250 with the micro-kernel at
// :113-172, which keeps C in registers across KC panels — storing and reloading an f32 is exact),
// and with `sum += a * b` (rounded product, then rounded add) in dot_row (:252-285).
// The loop nest below is this oracle's own (4x16 register blocks, k blocked by 256); only the
// per-element operation sequence is the reference's.
// ---------------------------------------------------------------------------------------------
constexpr int64_t kRowBlock = 4;
constexpr int64_t kColBlock = 16;
constexpr int64_t kDepthBlock = 256;

template <bool Fused>
__attribute__((target("avx2,fma"))) inline void block_4x16(const float* a, int64_t lda,
                                                           const float* b, int64_t ldb, float* c,
                                                           int64_t ldc, int64_t depth,
                                                           int64_t rows) {
    const float* a0 = a;
    const float* a1 = a + (rows > 1 ? 1 : 0) * lda;
    const float* a2 = a + (rows > 2 ? 2 : 0) * lda;
    const float* a3 = a + (rows > 3 ? 3 : 0) * lda;
    __m256 c00 = _mm256_loadu_ps(c), c01 = _mm256_loadu_ps(c + 8);
    __m256 c10 = _mm256_setzero_ps(), c11 = _mm256_setzero_ps();
    __m256 c20 = _mm256_setzero_ps(), c21 = _mm256_setzero_ps();
    __m256 c30 = _mm256_setzero_ps(), c31 = _mm256_setzero_ps();
    if (rows > 1) { c10 = _mm256_loadu_ps(c + ldc); c11 = _mm256_loadu_ps(c + ldc + 8); }
    if (rows > 2) { c20 = _mm256_loadu_ps(c + 2 * ldc); c21 = _mm256_loadu_ps(c + 2 * ldc + 8); }
    if (rows > 3) { c30 = _mm256_loadu_ps(c + 3 * ldc); c31 = _mm256_loadu_ps(c + 3 * ldc + 8); }
    for (int64_t p = 0; p < depth; ++p) {
        const __m256 b0 = _mm256_loadu_ps(b + p * ldb);
        const __m256 b1 = _mm256_loadu_ps(b + p * ldb + 8);
        const __m256 x0 = _mm256_broadcast_ss(a0 + p);
        const __m256 x1 = _mm256_broadcast_ss(a1 + p);
        const __m256 x2 = _mm256_broadcast_ss(a2 + p);
        const __m256 x3 = _mm256_broadcast_ss(a3 + p);
        if constexpr (Fused) {
            c00 = _mm256_fmadd_ps(x0, b0, c00); c01 = _mm256_fmadd_ps(x0, b1, c01);
            c10 = _mm256_fmadd_ps(x1, b0, c10); c11 = _mm256_fmadd_ps(x1, b1, c11);
            c20 = _mm256_fmadd_ps(x2, b0, c20); c21 = _mm256_fmadd_ps(x2, b1, c21);
            c30 = _mm256_fmadd_ps(x3, b0, c30); c31 = _mm256_fmadd_ps(x3, b1, c31);
        } else {
            c00 = _mm256_add_ps(c00, _mm256_mul_ps(x0, b0));
            c01 = _mm256_add_ps(c01, _mm256_mul_ps(x0, b1));
            c10 = _mm256_add_ps(c10, _mm256_mul_ps(x1, b0));
            c11 = _mm256_add_ps(c11, _mm256_mul_ps(x1, b1));
            c20 = _mm256_add_ps(c20, _mm256_mul_ps(x2, b0));
            c21 = _mm256_add_ps(c21, _mm256_mul_ps(x2, b1));
            c30 = _mm256_add_ps(c30, _mm256_mul_ps(x3, b0));
            c31 = _mm256_add_ps(c31, _mm256_mul_ps(x3, b1));
        }
    }
    _mm256_storeu_ps(c, c00); _mm256_storeu_ps(c + 8, c01);
    if (rows > 1) { _mm256_storeu_ps(c + ldc, c10); _mm256_storeu_ps(c + ldc + 8, c11); }
    if (rows > 2) { _mm256_storeu_ps(c + 2 * ldc, c20); _mm256_storeu_ps(c + 2 * ldc + 8, c21); }
    if (rows > 3) { _mm256_storeu_ps(c + 3 * ldc, c30); _mm256_storeu_ps(c + 3 * ldc + 8, c31); }
}

// Accumulates C[row0:row1, col0:col1] += A[row0:row1, p0:p1] * B[p0:p1, col0:col1].
template <bool Fused>
void tile_range(const float* a, const float* b, float* c, int64_t k, int64_t n, int64_t row0,
                int64_t row1, int64_t col0, int64_t col1, int64_t p0, int64_t p1) {
    const int64_t vector_end = col0 + ((col1 - col0) / kColBlock) * kColBlock;
    for (int64_t j = col0; j < vector_end; j += kColBlock) {
        for (int64_t i = row0; i < row1; i += kRowBlock) {
            const int64_t rows = std::min(kRowBlock, row1 - i);
            block_4x16<Fused>(a + i * k + p0, k, b + p0 * n + j, n, c + i * n + j, n, p1 - p0,
                              rows);
        }
    }
    for (int64_t i = row0; i < row1; ++i) {
        for (int64_t j = vector_end; j < col1; ++j) {
            float sum = c[i * n + j];
            for (int64_t p = p0; p < p1; ++p) {
                if constexpr (Fused) {
                    sum = std::fma(a[i * k + p], b[p * n + j], sum);
                } else {
                    sum = sum + a[i * k + p] * b[p * n + j];
                }
            }
            c[i * n + j] = sum;
        }
    }
}

int g_threads = 0;

int thread_count() { return g_threads > 0 ? g_threads : omp_get_max_threads(); }

void matmul_impl(const float* a, const float* b, float* c, int64_t m, int64_t k, int64_t n,
                 bool fused_tiles, bool allow_parallel) {
    std::fill(c, c + m * n, 0.0f);
    if (m == 0 || n == 0 || k == 0) return;
    const int64_t m_main = fused_tiles ? m - m % 6 : 0;
    const int64_t n_main = fused_tiles ? n - n % 16 : 0;
    const int64_t chunk = 32;
    const int64_t chunks = (m + chunk - 1) / chunk;
    const bool parallel = allow_parallel && m * n * k >= (1 << 20) && chunks > 1 &&
                          !omp_in_parallel();
#pragma omp parallel for schedule(dynamic) num_threads(thread_count()) if (parallel)
    for (int64_t block = 0; block < chunks; ++block) {
        const int64_t r0 = block * chunk;
        const int64_t r1 = std::min(m, r0 + chunk);
        for (int64_t p0 = 0; p0 < k; p0 += kDepthBlock) {
            const int64_t p1 = std::min(k, p0 + kDepthBlock);
            // Rows inside the tiled region: FMA columns [0, n_main), dot_row columns after.
            const int64_t tiled_end = std::min(r1, m_main);
            if (r0 < tiled_end) {
                tile_range<true>(a, b, c, k, n, r0, tiled_end, 0, n_main, p0, p1);
                tile_range<false>(a, b, c, k, n, r0, tiled_end, n_main, n, p0, p1);
            }
            // Remainder rows: dot_row everywhere.
            const int64_t rest = std::max(r0, m_main);
            if (rest < r1) tile_range<false>(a, b, c, k, n, rest, r1, 0, n, p0, p1);
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Elementwise / NN ops (native/src/ops.rs, native/src/nn_ops.rs).
// ---------------------------------------------------------------------------------------------
using Shape = std::vector<int64_t>;

int64_t numel(const Shape& s) {
    int64_t n = 1;
    for (int64_t d : s) n *= d;
    return n;
}

// Tensor.broadcastShape (torch/Tensor.java:830-850): trailing alignment, 1 broadcasts.
bool broadcast_shape(const Shape& a, const Shape& b, Shape* out) {
    const size_t rank = std::max(a.size(), b.size());
    out->assign(rank, 1);
    for (size_t i = 0; i < rank; ++i) {
        const int64_t da = i < rank - a.size() ? 1 : a[i - (rank - a.size())];
        const int64_t db = i < rank - b.size() ? 1 : b[i - (rank - b.size())];
        if (da != db && da != 1 && db != 1) return false;
        (*out)[i] = std::max(da, db);
    }
    return true;
}

// ops.rs:166-176 aligned_strides.
std::vector<int64_t> aligned_strides(const Shape& shape, const Shape& out) {
    const size_t offset = out.size() - shape.size();
    std::vector<int64_t> strides(out.size(), 0);
    int64_t stride = 1;
    for (size_t d = shape.size(); d-- > 0;) {
        const bool broadcast = shape[d] == 1 && out[offset + d] != 1;
        strides[offset + d] = broadcast ? 0 : stride;
        stride *= shape[d];
    }
    return strides;
}

enum class BinOp { Add, Mul };

inline float apply(BinOp op, float x, float y) { return op == BinOp::Add ? x + y : x * y; }

// ops.rs:186-284 binary_forward: same-shape, scalar and general broadcast walks. All three
// branches compute the same single f32 operation per element, so one strided walk restates them.
int binary(BinOp op, const float* a, const Shape& as, const float* b, const Shape& bs, float* out,
           Shape* out_shape) {
    Shape os;
    if (!broadcast_shape(as, bs, &os)) return -2;
    if (out_shape) *out_shape = os;
    const int64_t total = numel(os);
    if (as == bs) {
        for (int64_t i = 0; i < total; ++i) out[i] = apply(op, a[i], b[i]);
        return 0;
    }
    const auto sa = aligned_strides(as, os);
    const auto sb = aligned_strides(bs, os);
    const size_t rank = os.size();
    // Iterate over the last dimension in an inner loop; outer coordinates by div/mod.
    const int64_t inner = os[rank - 1];
    const int64_t outer = total / std::max<int64_t>(inner, 1);
#pragma omp parallel for schedule(static) num_threads(thread_count()) if (total > (1 << 18) && !omp_in_parallel())
    for (int64_t o = 0; o < outer; ++o) {
        int64_t rem = o, ia = 0, ib = 0;
        for (size_t d = rank - 1; d-- > 0;) {
            const int64_t coord = rem % os[d];
            rem /= os[d];
            ia += coord * sa[d];
            ib += coord * sb[d];
        }
        float* dst = out + o * inner;
        for (int64_t j = 0; j < inner; ++j) {
            dst[j] = apply(op, a[ia + j * sa[rank - 1]], b[ib + j * sb[rank - 1]]);
        }
    }
    return 0;
}

// nn_ops.rs:130-137 gelu_forward (tanh form, f32).
void gelu(const float* in, float* out, int64_t n) {
    const float constant = std::sqrt(2.0f / static_cast<float>(M_PI));
#pragma omp parallel for schedule(static) num_threads(thread_count()) if (n > (1 << 18) && !omp_in_parallel())
    for (int64_t i = 0; i < n; ++i) {
        const float v = in[i];
        const float inner = constant * (v + 0.044715f * v * v * v);
        out[i] = 0.5f * v * (1.0f + std::tanh(inner));
    }
}

// nn_ops.rs:13-38 softmax_forward over the last dimension.
int softmax_rows(const float* in, float* out, int64_t rows, int64_t dim) {
    if (dim == 0 || rows == 0) return -2;
    int status = 0;
#pragma omp parallel for schedule(static) num_threads(thread_count()) if (rows * dim > (1 << 16) && !omp_in_parallel())
    for (int64_t r = 0; r < rows; ++r) {
        const float* x = in + r * dim;
        float* y = out + r * dim;
        float maximum = -INFINITY;
        for (int64_t i = 0; i < dim; ++i) maximum = std::fmax(maximum, x[i]);
        float sum = 0.0f;
        for (int64_t i = 0; i < dim; ++i) {
            const float value = std::exp(x[i] - maximum);
            y[i] = value;
            sum += value;
        }
        if (!(sum > 0.0f) || !std::isfinite(sum)) {
#pragma omp atomic write
            status = -1;
            continue;
        }
        const float inverse = 1.0f / sum;
        for (int64_t i = 0; i < dim; ++i) y[i] *= inverse;
    }
    return status;
}

// nn_ops.rs:168-199 layer_norm_forward: f64 mean and population variance, f32 affine.
void layer_norm(const float* in, const float* gamma, const float* beta, float* out, int64_t rows,
                int64_t dim, float eps) {
#pragma omp parallel for schedule(static) num_threads(thread_count()) if (rows * dim > (1 << 16) && !omp_in_parallel())
    for (int64_t r = 0; r < rows; ++r) {
        const float* x = in + r * dim;
        float* y = out + r * dim;
        double mean = 0.0;
        for (int64_t i = 0; i < dim; ++i) mean += static_cast<double>(x[i]);
        mean /= static_cast<double>(dim);
        double variance = 0.0;
        for (int64_t i = 0; i < dim; ++i) {
            const double delta = static_cast<double>(x[i]) - mean;
            variance += delta * delta;
        }
        variance /= static_cast<double>(dim);
        const double inverse = 1.0 / std::sqrt(variance + static_cast<double>(eps));
        for (int64_t i = 0; i < dim; ++i) {
            const float normalized = static_cast<float>((static_cast<double>(x[i]) - mean) * inverse);
            y[i] = normalized * gamma[i] + beta[i];
        }
    }
}

}  // namespace

extern "C" void orc_matmul(const float* a, const float* b, float* c, int64_t m, int64_t k,
                           int64_t n, int32_t fused_tiles) {
    matmul_impl(a, b, c, m, k, n, fused_tiles != 0, true);
}

extern "C" int32_t orc_add(const float* a, const int64_t* a_shape, int32_t a_rank, const float* b,
                           const int64_t* b_shape, int32_t b_rank, float* out) {
    return binary(BinOp::Add, a, Shape(a_shape, a_shape + a_rank), b,
                  Shape(b_shape, b_shape + b_rank), out, nullptr);
}

extern "C" int32_t orc_mul(const float* a, const int64_t* a_shape, int32_t a_rank, const float* b,
                           const int64_t* b_shape, int32_t b_rank, float* out) {
    return binary(BinOp::Mul, a, Shape(a_shape, a_shape + a_rank), b,
                  Shape(b_shape, b_shape + b_rank), out, nullptr);
}

// ops.rs unary relu (used by NativeTestSuite.testQueue).
extern "C" void orc_relu(const float* a, float* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = a[i] > 0.0f ? a[i] : 0.0f;
}

extern "C" void orc_gelu(const float* a, float* out, int64_t n) { gelu(a, out, n); }

extern "C" int32_t orc_softmax(const float* a, float* out, int64_t rows, int64_t dim) {
    return softmax_rows(a, out, rows, dim);
}

extern "C" int32_t orc_layer_norm(const float* a, const float* gamma, const float* beta, float* out,
                                  int64_t rows, int64_t dim, float eps) {
    if (dim <= 0) return -2;
    layer_norm(a, gamma, beta, out, rows, dim, eps);
    return 0;
}

extern "C" int32_t orc_threads(void) { return thread_count(); }
extern "C" void orc_set_threads(int32_t threads) { g_threads = threads; }

// =============================================================================================
// Models and the TextEngine loop.
// =============================================================================================
struct orc_engine {
    orc_spec spec{};
    std::vector<std::string> names;
    std::vector<std::vector<float>> values;
    std::map<std::string, size_t> index;
    orc_random random{};
    std::string error;

    int fail(int code, const std::string& message) {
        error = message;
        return code;
    }
    const std::vector<float>& p(const std::string& name) const { return values[index.at(name)]; }
    void declare(const std::string& name, int64_t count, float fill = 0.0f) {
        index[name] = names.size();
        names.push_back(name);
        values.emplace_back(static_cast<size_t>(count), fill);
    }
};

namespace {

constexpr float kLayerNormEps = 1e-5f;  // TransformerBlock.java:26,29
constexpr float kMaskValue = -1.0e9f;   // MultiheadAttention.java:71

bool decoder_family(int family) {
    return family == ORC_FAMILY_PADDED_DECODER || family == ORC_FAMILY_DECODER;
}

// Linear.forward (torch/Linear.java:30-49): flat [rows, in] x W[in, out], then + bias [1, out].
void linear(orc_engine* e, const float* x, int64_t rows, int64_t in, int64_t out,
            const std::string& prefix, float* y) {
    matmul_impl(x, e->p(prefix + ".weight").data(), y, rows, in, out, e->spec.fused_tiles != 0,
                true);
    const auto& bias = e->p(prefix + ".bias");
    binary(BinOp::Add, y, {rows, out}, bias.data(), {1, out}, y, nullptr);
}

// embedding_forward (nn_ops.rs:1040-1063): row gather with the id checks.
int embedding(orc_engine* e, const float* ids, int64_t rows, const std::vector<float>& table,
              int64_t dim, float* out) {
    const int64_t vocab = static_cast<int64_t>(table.size()) / dim;
    for (int64_t r = 0; r < rows; ++r) {
        const float id = ids[r];
        if (!std::isfinite(id) || id < 0.0f || id >= static_cast<float>(vocab)) {
            char buffer[128];
            std::snprintf(buffer, sizeof(buffer), "embedding index %g is outside [0, %lld)",
                          static_cast<double>(id), static_cast<long long>(vocab));
            return e->fail(-1, buffer);
        }
        const int64_t row = static_cast<int64_t>(id);
        std::memcpy(out + r * dim, table.data() + row * dim, sizeof(float) * dim);
    }
    return 0;
}

// Decoder forward. Blocks follow TransformerBlock.forward (TransformerBlock.java:37-43) and
// MultiheadAttention.forward (MultiheadAttention.java:40-82) op by op; the wrapper adds token and
// position embeddings, a final LayerNorm, the last-position slice (Tensor.slice,
// torch/Tensor.java:321-338) and a Linear head. For the padded family the position of a token
// counts from the first non-PAD id of its row, and the additive mask also hides PAD key columns.
// Logits are written for window positions first_out..W-1 of every row ([rows, W - first_out, V]);
// TextEngine reads the last position only (first_out = W - 1).
int decoder_forward(orc_engine* e, const float* ids, int64_t rows, float* logits,
                    int64_t first_out) {
    const orc_spec& s = e->spec;
    const int64_t W = s.window, d = s.dimension, H = s.heads, hd = d / H, F = s.hidden;
    const int64_t V = s.vocabulary, T = rows * W;
    const bool padded = s.family == ORC_FAMILY_PADDED_DECODER;
    const float pad = static_cast<float>(V);

    std::vector<int64_t> npad(rows, 0);
    std::vector<float> pos_ids(T);
    for (int64_t r = 0; r < rows; ++r) {
        if (padded) {
            while (npad[r] < W && ids[r * W + npad[r]] == pad) ++npad[r];
        }
        for (int64_t t = 0; t < W; ++t) {
            pos_ids[r * W + t] = static_cast<float>(t < npad[r] ? 0 : t - npad[r]);
        }
    }

    std::vector<float> x(T * d), pe(T * d), h(T * d), q(T * d), k(T * d), v(T * d);
    int status = embedding(e, ids, T, e->p("embedding.weight"), d, x.data());
    if (status) return status;
    status = embedding(e, pos_ids.data(), T, e->p("position.weight"), d, pe.data());
    if (status) return status;
    binary(BinOp::Add, x.data(), {rows, W, d}, pe.data(), {rows, W, d}, x.data(), nullptr);

    // Additive mask [rows, W, W]: -1e9 above the diagonal and, for the padded family, on PAD keys.
    std::vector<float> mask(rows * W * W, 0.0f);
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t i = 0; i < W; ++i) {
            for (int64_t j = 0; j < W; ++j) {
                if (j > i || j < npad[r]) mask[(r * W + i) * W + j] = kMaskValue;
            }
        }
    }

    const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(hd)));
    std::vector<float> qh(T * d), kh(T * d), vh(T * d), ctx(T * d), merged(T * d);
    std::vector<float> scores(rows * H * W * W);
    std::vector<float> ffn(T * F);
    for (int64_t layer = 0; layer < s.layers; ++layer) {
        const std::string pre = "layer" + std::to_string(layer) + ".";
        layer_norm(x.data(), e->p(pre + "norm1.gamma").data(), e->p(pre + "norm1.beta").data(),
                   h.data(), T, d, kLayerNormEps);
        linear(e, h.data(), T, d, d, pre + "attention.query", q.data());
        linear(e, h.data(), T, d, d, pre + "attention.key", k.data());
        linear(e, h.data(), T, d, d, pre + "attention.value", v.data());
        // reshape [rows, W, H, hd] + permute (nn_ops.rs:1156-1191): q,v -> [rows*H, W, hd];
        // k -> [rows*H, hd, W].
        for (int64_t r = 0; r < rows; ++r)
            for (int64_t t = 0; t < W; ++t)
                for (int64_t hh = 0; hh < H; ++hh)
                    for (int64_t e2 = 0; e2 < hd; ++e2) {
                        const int64_t src = (r * W + t) * d + hh * hd + e2;
                        qh[((r * H + hh) * W + t) * hd + e2] = q[src];
                        vh[((r * H + hh) * W + t) * hd + e2] = v[src];
                        kh[((r * H + hh) * hd + e2) * W + t] = k[src];
                    }
        // batched_matmul_forward (nn_ops.rs:1081-1106): one gemm per batch item.
#pragma omp parallel for schedule(dynamic) num_threads(thread_count())
        for (int64_t item = 0; item < rows * H; ++item) {
            float* sc = scores.data() + item * W * W;
            matmul_impl(qh.data() + item * W * hd, kh.data() + item * hd * W, sc, W, hd, W,
                        s.fused_tiles != 0, false);
            // .mul(scale): scalar broadcast multiply; .add(mask): mask[r] for this item's row.
            const float* m = mask.data() + (item / H) * W * W;
            for (int64_t i = 0; i < W * W; ++i) sc[i] = sc[i] * scale;
            for (int64_t i = 0; i < W * W; ++i) sc[i] = sc[i] + m[i];
        }
        status = softmax_rows(scores.data(), scores.data(), rows * H * W, W);
        if (status) return e->fail(-1, "softmax denominator is not finite");
#pragma omp parallel for schedule(dynamic) num_threads(thread_count())
        for (int64_t item = 0; item < rows * H; ++item) {
            matmul_impl(scores.data() + item * W * W, vh.data() + item * W * hd,
                        ctx.data() + item * W * hd, W, W, hd, s.fused_tiles != 0, false);
        }
        // reshape [rows, H, W, hd] + permute(0, 2, 1, 3) -> [rows, W, d].
        for (int64_t r = 0; r < rows; ++r)
            for (int64_t hh = 0; hh < H; ++hh)
                for (int64_t t = 0; t < W; ++t)
                    for (int64_t e2 = 0; e2 < hd; ++e2)
                        merged[(r * W + t) * d + hh * hd + e2] =
                            ctx[((r * H + hh) * W + t) * hd + e2];
        linear(e, merged.data(), T, d, d, pre + "attention.output", q.data());
        // Dropout(p = 0) is the identity (nn_ops.rs:993-1008): residual add.
        binary(BinOp::Add, x.data(), {T, d}, q.data(), {T, d}, x.data(), nullptr);
        layer_norm(x.data(), e->p(pre + "norm2.gamma").data(), e->p(pre + "norm2.beta").data(),
                   h.data(), T, d, kLayerNormEps);
        linear(e, h.data(), T, d, F, pre + "ffn1", ffn.data());
        gelu(ffn.data(), ffn.data(), T * F);
        linear(e, ffn.data(), T, F, d, pre + "ffn2", q.data());
        binary(BinOp::Add, x.data(), {T, d}, q.data(), {T, d}, x.data(), nullptr);
    }
    // Final LayerNorm, then slice(1, W-1, W) -> [rows, d], then the head.
    layer_norm(x.data(), e->p("norm.gamma").data(), e->p("norm.beta").data(), h.data(), T, d,
               kLayerNormEps);
    const int64_t outs = W - first_out;
    std::vector<float> last(rows * outs * d);
    for (int64_t r = 0; r < rows; ++r) {
        std::memcpy(last.data() + r * outs * d, h.data() + (r * W + first_out) * d,
                    sizeof(float) * outs * d);
    }
    linear(e, last.data(), rows * outs, d, V, "head", logits);
    return 0;
}

// Zoo.WindowedLanguageModel.forward (zoo/Zoo.java:155-168).
int char_lm_forward(orc_engine* e, const float* ids, int64_t rows, float* logits) {
    const orc_spec& s = e->spec;
    const int64_t W = s.window, d = s.dimension, hidden = s.hidden, V = s.vocabulary;
    const int64_t flat = W * d;
    std::vector<float> x(rows * flat), hid(rows * hidden), back(rows * flat);
    int status = embedding(e, ids, rows * W, e->p("param0"), d, x.data());
    if (status) return status;
    matmul_impl(x.data(), e->p("param1").data(), hid.data(), rows, flat, hidden,
                s.fused_tiles != 0, true);
    binary(BinOp::Add, hid.data(), {rows, hidden}, e->p("param2").data(), {1, hidden}, hid.data(),
           nullptr);
    gelu(hid.data(), hid.data(), rows * hidden);
    matmul_impl(hid.data(), e->p("param3").data(), back.data(), rows, hidden, flat,
                s.fused_tiles != 0, true);
    binary(BinOp::Add, back.data(), {rows, flat}, e->p("param4").data(), {1, flat}, back.data(),
           nullptr);
    binary(BinOp::Add, back.data(), {rows, flat}, x.data(), {rows, flat}, back.data(), nullptr);
    gelu(back.data(), back.data(), rows * flat);
    matmul_impl(back.data(), e->p("param5").data(), logits, rows, flat, V, s.fused_tiles != 0,
                true);
    binary(BinOp::Add, logits, {rows, V}, e->p("param6").data(), {1, V}, logits, nullptr);
    return 0;
}

// TextEngineTest.LastTokenModel.forward (TextEngineTest.java:226-237): one-hot of the last id
// (Math.floorMod) through Linear(V, V).
int last_token_forward(orc_engine* e, const float* ids, int64_t rows, float* logits) {
    const int64_t V = e->spec.vocabulary, W = e->spec.window;
    std::vector<float> one_hot(rows * V, 0.0f);
    for (int64_t r = 0; r < rows; ++r) {
        const int32_t token = static_cast<int32_t>(ids[r * W + W - 1]);
        const int32_t slot = ((token % V) + V) % V;
        one_hot[r * V + slot] = 1.0f;
    }
    matmul_impl(one_hot.data(), e->p("param0").data(), logits, rows, V, V,
                e->spec.fused_tiles != 0, true);
    binary(BinOp::Add, logits, {rows, V}, e->p("param1").data(), {1, V}, logits, nullptr);
    return 0;
}

int forward(orc_engine* e, const float* ids, int64_t rows, float* logits) {
    switch (e->spec.family) {
        case ORC_FAMILY_PADDED_DECODER:
        case ORC_FAMILY_DECODER: return decoder_forward(e, ids, rows, logits, e->spec.window - 1);
        case ORC_FAMILY_CHAR_LM: return char_lm_forward(e, ids, rows, logits);
        case ORC_FAMILY_LAST_TOKEN: return last_token_forward(e, ids, rows, logits);
        default: return e->fail(-8, "unknown model family");
    }
}

// ---- TextEngine helpers (TextEngine.java:359-427) ----
int require_context(orc_engine* e, int32_t length) {
    if (length < e->spec.window) {
        return e->fail(-1, "context needs at least " + std::to_string(e->spec.window) +
                               " tokens, got " + std::to_string(length));
    }
    return 0;
}

int require_steps(orc_engine* e, int32_t steps) {
    if (steps < 1) return e->fail(-1, "steps must be at least 1, got " + std::to_string(steps));
    return 0;
}

void push(std::vector<int32_t>& carried, int32_t next) {
    std::memmove(carried.data(), carried.data() + 1, sizeof(int32_t) * (carried.size() - 1));
    carried.back() = next;
}

int32_t argmax(const double* scores, int32_t count) {
    int32_t best = 0;
    for (int32_t c = 1; c < count; ++c) {
        if (scores[c] > scores[best]) best = c;
    }
    return best;
}

// Double.compare (java/lang/Double.java): numeric order, -0.0 < 0.0, NaN above everything.
int double_compare(double a, double b) {
    if (a < b) return -1;
    if (a > b) return 1;
    auto bits = [](double x) {
        if (std::isnan(x)) return static_cast<int64_t>(0x7ff8000000000000LL);
        int64_t v;
        std::memcpy(&v, &x, sizeof(v));
        return v;
    };
    const int64_t ba = bits(a), bb = bits(b);
    return ba == bb ? 0 : (ba < bb ? -1 : 1);
}

int32_t draw(orc_engine* e, const double* scores, int32_t count, float temperature,
             int32_t top_k) {
    std::vector<int32_t> order(count);
    for (int32_t t = 0; t < count; ++t) order[t] = t;
    std::stable_sort(order.begin(), order.end(), [&](int32_t left, int32_t right) {
        return double_compare(scores[right], scores[left]) < 0;
    });
    const double maximum = scores[order[0]];
    double total = 0.0;
    std::vector<double> weights(top_k);
    for (int32_t i = 0; i < top_k; ++i) {
        weights[i] = std::exp((scores[order[i]] - maximum) / static_cast<double>(temperature));
        total += weights[i];
    }
    const double target = orc_random_next_double(&e->random) * total;
    double running = 0.0;
    for (int32_t i = 0; i < top_k; ++i) {
        running += weights[i];
        if (target <= running) return order[i];
    }
    return order[top_k - 1];
}

int scores_rows(orc_engine* e, const std::vector<std::vector<int32_t>>& windows,
                std::vector<double>* out) {
    const int32_t rows = static_cast<int32_t>(windows.size());
    const int32_t W = e->spec.window, V = e->spec.vocabulary;
    std::vector<float> ids(static_cast<size_t>(rows) * W);
    for (int32_t r = 0; r < rows; ++r)
        for (int32_t t = 0; t < W; ++t) ids[static_cast<size_t>(r) * W + t] = static_cast<float>(windows[r][t]);
    std::vector<float> logits(static_cast<size_t>(rows) * V);
    const int status = forward(e, ids.data(), rows, logits.data());
    if (status) return status;
    out->assign(logits.begin(), logits.end());
    return 0;
}

std::vector<int32_t> tail(const orc_engine* e, const int32_t* context, int32_t length) {
    const int32_t W = e->spec.window;
    return std::vector<int32_t>(context + (length - W), context + length);
}

int check_sampling(orc_engine* e, float temperature, int32_t top_k) {
    if (!(temperature > 0.0f) || !std::isfinite(temperature)) {
        return e->fail(-1, "temperature must be positive and finite");
    }
    if (top_k < 1) return e->fail(-1, "topK must be at least 1, got " + std::to_string(top_k));
    return 0;
}

// Parameter tables in namedParameters order.
void declare_parameters(orc_engine* e) {
    const orc_spec& s = e->spec;
    const int64_t V = s.vocabulary, W = s.window, d = s.dimension, F = s.hidden;
    switch (s.family) {
        case ORC_FAMILY_PADDED_DECODER:
        case ORC_FAMILY_DECODER: {
            const int64_t rows = s.family == ORC_FAMILY_PADDED_DECODER ? V + 1 : V;
            e->declare("embedding.weight", rows * d);
            e->declare("position.weight", W * d);
            for (int32_t l = 0; l < s.layers; ++l) {
                const std::string pre = "layer" + std::to_string(l) + ".";
                e->declare(pre + "norm1.gamma", d, 1.0f);
                e->declare(pre + "norm1.beta", d);
                for (const char* part : {"query", "key", "value", "output"}) {
                    e->declare(pre + "attention." + part + ".weight", d * d);
                    e->declare(pre + "attention." + part + ".bias", d);
                }
                e->declare(pre + "norm2.gamma", d, 1.0f);
                e->declare(pre + "norm2.beta", d);
                e->declare(pre + "ffn1.weight", d * F);
                e->declare(pre + "ffn1.bias", F);
                e->declare(pre + "ffn2.weight", F * d);
                e->declare(pre + "ffn2.bias", d);
            }
            e->declare("norm.gamma", d, 1.0f);
            e->declare("norm.beta", d);
            e->declare("head.weight", d * V);
            e->declare("head.bias", V);
            break;
        }
        case ORC_FAMILY_CHAR_LM: {
            const int64_t flat = W * d;
            e->declare("param0", V * d);
            e->declare("param1", flat * F);
            e->declare("param2", F);
            e->declare("param3", F * flat);
            e->declare("param4", flat);
            e->declare("param5", flat * V);
            e->declare("param6", V);
            break;
        }
        case ORC_FAMILY_LAST_TOKEN: {
            e->declare("param0", V * V);
            e->declare("param1", V);
            std::vector<float>& w = e->values[0];
            for (int64_t t = 0; t < V; ++t) w[t * V + (t + 1) % V] = 6.0f;
            break;
        }
        default: break;
    }
}

// ---- DataOutputStream / DataInputStream big-endian helpers ----
void put_u32(std::string& out, uint32_t v) {
    const char bytes[4] = {static_cast<char>(v >> 24), static_cast<char>(v >> 16),
                           static_cast<char>(v >> 8), static_cast<char>(v)};
    out.append(bytes, 4);
}

bool get_u32(FILE* f, uint32_t* v) {
    unsigned char b[4];
    if (std::fread(b, 1, 4, f) != 4) return false;
    *v = (uint32_t(b[0]) << 24) | (uint32_t(b[1]) << 16) | (uint32_t(b[2]) << 8) | uint32_t(b[3]);
    return true;
}

}  // namespace

extern "C" orc_engine* orc_engine_create(const orc_spec* spec) {
    if (!spec) return nullptr;
    const orc_spec& s = *spec;
    if (s.vocabulary < 2 || s.window < 1) return nullptr;
    if (decoder_family(s.family)) {
        if (s.dimension < 1 || s.heads < 1 || s.dimension % s.heads != 0 || s.layers < 0 ||
            s.hidden < 1) {
            return nullptr;
        }
    } else if (s.family == ORC_FAMILY_CHAR_LM) {
        if (s.dimension < 1 || s.hidden < 1) return nullptr;
    } else if (s.family != ORC_FAMILY_LAST_TOKEN) {
        return nullptr;
    }
    auto* e = new orc_engine();
    e->spec = s;
    orc_random_set_seed(&e->random, 0);
    declare_parameters(e);
    return e;
}

extern "C" void orc_engine_destroy(orc_engine* e) { delete e; }
extern "C" const char* orc_engine_error(orc_engine* e) { return e->error.c_str(); }
extern "C" int32_t orc_param_count(orc_engine* e) { return static_cast<int32_t>(e->names.size()); }
extern "C" const char* orc_param_name(orc_engine* e, int32_t i) { return e->names[i].c_str(); }
extern "C" int64_t orc_param_size(orc_engine* e, int32_t i) {
    return static_cast<int64_t>(e->values[i].size());
}

extern "C" int32_t orc_set_param(orc_engine* e, const char* name, const float* values,
                                 int64_t count) {
    auto it = e->index.find(name);
    if (it == e->index.end()) return e->fail(-1, std::string("unknown parameter ") + name);
    auto& dst = e->values[it->second];
    if (static_cast<int64_t>(dst.size()) != count) {
        return e->fail(-2, std::string("parameter ") + name + " expects " +
                               std::to_string(dst.size()) + " values, got " +
                               std::to_string(count));
    }
    std::copy(values, values + count, dst.begin());
    return 0;
}

extern "C" int32_t orc_get_param(orc_engine* e, const char* name, float* values, int64_t count) {
    auto it = e->index.find(name);
    if (it == e->index.end()) return e->fail(-1, std::string("unknown parameter ") + name);
    const auto& src = e->values[it->second];
    if (static_cast<int64_t>(src.size()) != count) return e->fail(-2, "size mismatch");
    std::copy(src.begin(), src.end(), values);
    return 0;
}

// TextEngine.save (TextEngine.java:298-319).
extern "C" int32_t orc_save(orc_engine* e, const char* path) {
    std::string out;
    put_u32(out, static_cast<uint32_t>(e->spec.vocabulary));
    put_u32(out, static_cast<uint32_t>(e->spec.window));
    put_u32(out, static_cast<uint32_t>(e->names.size()));
    for (size_t i = 0; i < e->names.size(); ++i) {
        const std::string& name = e->names[i];  // ASCII: modified UTF-8 == the bytes
        out.push_back(static_cast<char>(name.size() >> 8));
        out.push_back(static_cast<char>(name.size() & 0xff));
        out += name;
        put_u32(out, static_cast<uint32_t>(e->values[i].size()));
        for (float v : e->values[i]) {
            uint32_t bits;
            std::memcpy(&bits, &v, 4);
            if (std::isnan(v)) bits = 0x7fc00000u;  // Float.floatToIntBits canonical NaN
            put_u32(out, bits);
        }
    }
    FILE* f = std::fopen(path, "wb");
    if (!f) return e->fail(-1, std::string("cannot write model to ") + path);
    const size_t written = std::fwrite(out.data(), 1, out.size(), f);
    std::fclose(f);
    return written == out.size() ? 0 : e->fail(-1, std::string("cannot write model to ") + path);
}

// TextEngine.load (TextEngine.java:327-350) then Module.loadStateDict (torch/Module.java:68-76).
extern "C" int32_t orc_load(orc_engine* e, const char* path) {
    FILE* f = std::fopen(path, "rb");
    if (!f) return e->fail(-1, std::string("cannot read model from ") + path);
    uint32_t vocab, window, count;
    if (!get_u32(f, &vocab) || !get_u32(f, &window)) {
        std::fclose(f);
        return e->fail(-1, std::string("cannot read model from ") + path);
    }
    if (static_cast<int32_t>(vocab) != e->spec.vocabulary ||
        static_cast<int32_t>(window) != e->spec.window) {
        std::fclose(f);
        return e->fail(-4, "model was saved with vocabulary=" + std::to_string(int32_t(vocab)) +
                               " window=" + std::to_string(int32_t(window)) +
                               ", this engine is vocabulary=" +
                               std::to_string(e->spec.vocabulary) +
                               " window=" + std::to_string(e->spec.window));
    }
    std::map<std::string, std::vector<float>> stored;
    bool ok = get_u32(f, &count);
    for (uint32_t i = 0; ok && i < count; ++i) {
        unsigned char len[2];
        ok = std::fread(len, 1, 2, f) == 2;
        if (!ok) break;
        std::string name((size_t(len[0]) << 8) | len[1], '\0');
        ok = std::fread(name.data(), 1, name.size(), f) == name.size();
        uint32_t n;
        ok = ok && get_u32(f, &n);
        if (!ok) break;
        std::vector<float> values(n);
        for (uint32_t j = 0; ok && j < n; ++j) {
            uint32_t bits = 0;
            ok = get_u32(f, &bits);
            std::memcpy(&values[j], &bits, 4);
        }
        stored[name] = std::move(values);
    }
    std::fclose(f);
    if (!ok) return e->fail(-1, std::string("cannot read model from ") + path);
    for (size_t i = 0; i < e->names.size(); ++i) {
        auto it = stored.find(e->names[i]);
        if (it == stored.end()) return e->fail(-1, "missing state entry " + e->names[i]);
        if (it->second.size() != e->values[i].size()) {
            return e->fail(-2, "state entry " + e->names[i] + " has " +
                                   std::to_string(it->second.size()) + " values, expected " +
                                   std::to_string(e->values[i].size()));
        }
        e->values[i] = it->second;
    }
    return 0;
}

extern "C" int32_t orc_forward(orc_engine* e, const float* ids, int32_t rows, float* logits) {
    if (rows < 1) return e->fail(-1, "rows must be positive");
    return forward(e, ids, rows, logits);
}

// TextEngine.scoresBatch (TextEngine.java:121-148).
extern "C" int32_t orc_scores_batch(orc_engine* e, const int32_t* contexts, int32_t rows,
                                    int32_t length, double* scores) {
    if (rows < 1) return e->fail(-1, "contexts must not be empty");
    int status = require_context(e, length);
    if (status) return status;
    std::vector<std::vector<int32_t>> windows;
    for (int32_t r = 0; r < rows; ++r) windows.push_back(tail(e, contexts + int64_t(r) * length, length));
    std::vector<double> out;
    status = scores_rows(e, windows, &out);
    if (status) return status;
    std::copy(out.begin(), out.end(), scores);
    return 0;
}

// TextEngine.generate / stream (TextEngine.java:158-193).
extern "C" int32_t orc_generate(orc_engine* e, const int32_t* context, int32_t length,
                                int32_t steps, int32_t* produced, orc_sink sink, void* user) {
    int status = require_steps(e, steps);
    if (status) return status;
    status = require_context(e, length);
    if (status) return status;
    std::vector<std::vector<int32_t>> carried{tail(e, context, length)};
    std::vector<double> scores;
    for (int32_t step = 0; step < steps; ++step) {
        status = scores_rows(e, carried, &scores);
        if (status) return status;
        const int32_t next = argmax(scores.data(), e->spec.vocabulary);
        produced[step] = next;
        push(carried[0], next);
        if (sink) sink(user, 0, step, next);
    }
    return 0;
}

// TextEngine.generateBatch (TextEngine.java:232-254): one batched forward per step.
extern "C" int32_t orc_generate_batch(orc_engine* e, const int32_t* contexts, int32_t rows,
                                      int32_t length, int32_t steps, int32_t* produced) {
    int status = require_steps(e, steps);
    if (status) return status;
    if (rows < 1) return e->fail(-1, "contexts must not be empty");
    status = require_context(e, length);
    if (status) return status;
    std::vector<std::vector<int32_t>> carried;
    for (int32_t r = 0; r < rows; ++r) carried.push_back(tail(e, contexts + int64_t(r) * length, length));
    const int32_t V = e->spec.vocabulary;
    std::vector<double> scores;
    for (int32_t step = 0; step < steps; ++step) {
        status = scores_rows(e, carried, &scores);
        if (status) return status;
        for (int32_t r = 0; r < rows; ++r) {
            const int32_t next = argmax(scores.data() + int64_t(r) * V, V);
            produced[int64_t(r) * steps + step] = next;
            push(carried[r], next);
        }
    }
    return 0;
}

// Greedy batch decode of the padded decoder with a per-row KV cache: the CPU engine a cached
// implementation would be, for timing beside the full-window recompute above (which is what
// TextEngine does). Each row appends one token per step (TransformerBlock.forward,
// TransformerBlock.java:37-43, restated for one query position over the cached keys) and
// re-encodes its window token by token once the window no longer starts with PAD, as the
// positions of every cached token shift then. Rows run in parallel. Matrix products are the same
// gemm.rs restatement at one row, so logits agree with the recompute up to rounding order.
namespace {
struct RowCache {
    std::vector<float> k, v;  // [layers][W][d]
    int64_t len = 0;
};

// Appends token `id` at position `pos` to the row's cache and writes the next-token logits.
void cached_step(orc_engine* e, RowCache& rc, float id, float pos, float* logits) {
    const orc_spec& s = e->spec;
    const int64_t W = s.window, d = s.dimension, H = s.heads, hd = d / H, F = s.hidden;
    std::vector<float> x(d), pe(d), h(d), q(d), kk(d), vv(d), ctx(d), o(d), f(F), sc(W);
    embedding(e, &id, 1, e->p("embedding.weight"), d, x.data());
    embedding(e, &pos, 1, e->p("position.weight"), d, pe.data());
    for (int64_t i = 0; i < d; ++i) x[i] = x[i] + pe[i];
    const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(hd)));
    const int64_t t = rc.len;
    for (int64_t layer = 0; layer < s.layers; ++layer) {
        const std::string pre = "layer" + std::to_string(layer) + ".";
        layer_norm(x.data(), e->p(pre + "norm1.gamma").data(), e->p(pre + "norm1.beta").data(),
                   h.data(), 1, d, kLayerNormEps);
        linear(e, h.data(), 1, d, d, pre + "attention.query", q.data());
        linear(e, h.data(), 1, d, d, pre + "attention.key", kk.data());
        linear(e, h.data(), 1, d, d, pre + "attention.value", vv.data());
        float* kc = rc.k.data() + layer * W * d;
        float* vc = rc.v.data() + layer * W * d;
        std::memcpy(kc + t * d, kk.data(), sizeof(float) * d);
        std::memcpy(vc + t * d, vv.data(), sizeof(float) * d);
        for (int64_t hh = 0; hh < H; ++hh) {
            for (int64_t j = 0; j <= t; ++j) {
                float dot = 0.0f;
                for (int64_t e2 = 0; e2 < hd; ++e2) dot += q[hh * hd + e2] * kc[j * d + hh * hd + e2];
                sc[j] = dot * scale;
            }
            softmax_rows(sc.data(), sc.data(), 1, t + 1);
            for (int64_t e2 = 0; e2 < hd; ++e2) {
                float acc = 0.0f;
                for (int64_t j = 0; j <= t; ++j) acc += sc[j] * vc[j * d + hh * hd + e2];
                ctx[hh * hd + e2] = acc;
            }
        }
        linear(e, ctx.data(), 1, d, d, pre + "attention.output", o.data());
        for (int64_t i = 0; i < d; ++i) x[i] = x[i] + o[i];
        layer_norm(x.data(), e->p(pre + "norm2.gamma").data(), e->p(pre + "norm2.beta").data(),
                   h.data(), 1, d, kLayerNormEps);
        linear(e, h.data(), 1, d, F, pre + "ffn1", f.data());
        gelu(f.data(), f.data(), F);
        linear(e, f.data(), 1, F, d, pre + "ffn2", o.data());
        for (int64_t i = 0; i < d; ++i) x[i] = x[i] + o[i];
    }
    rc.len = t + 1;
    layer_norm(x.data(), e->p("norm.gamma").data(), e->p("norm.beta").data(), h.data(), 1, d,
               kLayerNormEps);
    linear(e, h.data(), 1, d, s.vocabulary, "head", logits);
}

// Encodes a window from scratch: its real tokens (after the leading PADs) one by one; a window
// of PADs only is one PAD token at position 0.
void encode_window(orc_engine* e, RowCache& rc, const std::vector<int32_t>& window, float* logits) {
    const int64_t W = e->spec.window;
    const int32_t pad = e->spec.vocabulary;
    int64_t npad = 0;
    while (npad < W && window[npad] == pad) ++npad;
    rc.len = 0;
    if (npad == W) {
        cached_step(e, rc, static_cast<float>(pad), 0.0f, logits);
        return;
    }
    for (int64_t t = npad; t < W; ++t) {
        cached_step(e, rc, static_cast<float>(window[t]), static_cast<float>(t - npad), logits);
    }
}
}  // namespace

extern "C" int32_t orc_generate_batch_cached(orc_engine* e, const int32_t* contexts, int32_t rows,
                                             int32_t length, int32_t steps, int32_t* produced) {
    if (e->spec.family != ORC_FAMILY_PADDED_DECODER) {
        return e->fail(-8, "the cached decode restates the padded decoder only");
    }
    int status = require_steps(e, steps);
    if (status) return status;
    if (rows < 1) return e->fail(-1, "contexts must not be empty");
    status = require_context(e, length);
    if (status) return status;
    const int64_t W = e->spec.window, d = e->spec.dimension, L = e->spec.layers;
    const int32_t V = e->spec.vocabulary;
    for (int32_t r = 0; r < rows; ++r) {
        const std::vector<int32_t> w = tail(e, contexts + int64_t(r) * length, length);
        for (int32_t id : w) {
            if (id < 0 || id > V) return e->fail(-1, "token id outside the vocabulary");
        }
    }
#pragma omp parallel for schedule(dynamic) num_threads(thread_count())
    for (int32_t r = 0; r < rows; ++r) {
        std::vector<int32_t> window = tail(e, contexts + int64_t(r) * length, length);
        RowCache rc;
        rc.k.assign(static_cast<size_t>(L * W * d), 0.0f);
        rc.v.assign(static_cast<size_t>(L * W * d), 0.0f);
        std::vector<float> logits(V);
        std::vector<double> scores(V);
        encode_window(e, rc, window, logits.data());
        for (int32_t step = 0; step < steps; ++step) {
            for (int32_t v = 0; v < V; ++v) scores[v] = logits[v];
            const int32_t next = argmax(scores.data(), V);
            produced[int64_t(r) * steps + step] = next;
            const bool had_pad = window[0] == V;
            push(window, next);
            if (step + 1 == steps) break;
            if (had_pad && rc.len < W) {
                cached_step(e, rc, static_cast<float>(next), static_cast<float>(rc.len), logits.data());
            } else {
                encode_window(e, rc, window, logits.data());
            }
        }
    }
    return 0;
}

// TextEngine.sample / streamSampled (TextEngine.java:201-227, 267-285).
extern "C" int32_t orc_sample(orc_engine* e, const int32_t* context, int32_t length, int32_t steps,
                              float temperature, int32_t top_k, int32_t* produced, orc_sink sink,
                              void* user) {
    int status = require_steps(e, steps);
    if (status) return status;
    status = check_sampling(e, temperature, top_k);
    if (status) return status;
    status = require_context(e, length);
    if (status) return status;
    const int32_t V = e->spec.vocabulary;
    std::vector<std::vector<int32_t>> carried{tail(e, context, length)};
    std::vector<double> scores;
    for (int32_t step = 0; step < steps; ++step) {
        status = scores_rows(e, carried, &scores);
        if (status) return status;
        const int32_t next = draw(e, scores.data(), V, temperature, std::min(top_k, V));
        produced[step] = next;
        push(carried[0], next);
        if (sink) sink(user, 0, step, next);
    }
    return 0;
}

extern "C" void orc_seed(orc_engine* e, int64_t seed) { orc_random_set_seed(&e->random, seed); }
extern "C" uint64_t orc_rng_state(orc_engine* e) { return e->random.seed; }
extern "C" void orc_set_rng_state(orc_engine* e, uint64_t state) {
    e->random.seed = state & ((1ULL << 48) - 1);
    e->random.have_next_gaussian = 0;
}

extern "C" int32_t orc_forced_scores(orc_engine* e, const int32_t* context, int32_t length,
                                     int32_t steps, const int32_t* forced, float* logits) {
    int status = require_steps(e, steps);
    if (status) return status;
    status = require_context(e, length);
    if (status) return status;
    const int32_t V = e->spec.vocabulary;
    std::vector<std::vector<int32_t>> carried{tail(e, context, length)};
    std::vector<double> scores;
    for (int32_t step = 0; step < steps; ++step) {
        status = scores_rows(e, carried, &scores);
        if (status) return status;
        for (int32_t v = 0; v < V; ++v) logits[int64_t(step) * V + v] = static_cast<float>(scores[v]);
        push(carried[0], forced[step]);
    }
    return 0;
}

// Teacher-forced logits of the padded decoder from one causal pass per row. While a row's window
// still starts with PAD at every step (steps - 1 <= leading PADs < W), the window scored at step g
// holds exactly the row's real tokens followed by forced[0..g-1], at positions counted from the
// first real token, and every PAD key is masked out (exp(-1e9 - max) is 0 in f32). The logits of
// step g are then the logits at position (real prompt length - 1 + g) of one forward over the
// real prompt followed by forced[0..steps-2]: the same sums TextEngine's full-window recompute
// forms (TextEngine.java:96-112, MultiheadAttention.java:40-82), with the matrix products taken
// at a different row count, so only the gemm.rs FMA-region membership of a row can differ.
// Returns -8 when a row's window would drop a real token; orc_forced_scores covers that case.
extern "C" int32_t orc_forced_scores_single_pass(orc_engine* e, const int32_t* contexts,
                                                 int32_t rows, int32_t length, int32_t steps,
                                                 const int32_t* forced, float* logits) {
    if (e->spec.family != ORC_FAMILY_PADDED_DECODER) {
        return e->fail(-8, "the single-pass teacher-forced logits restate the padded decoder");
    }
    int status = require_steps(e, steps);
    if (status) return status;
    if (rows < 1) return e->fail(-1, "contexts must not be empty");
    status = require_context(e, length);
    if (status) return status;
    const int32_t W = e->spec.window, V = e->spec.vocabulary;
    const float pad = static_cast<float>(V);
    std::vector<float> ids(static_cast<size_t>(rows) * W);
    for (int32_t r = 0; r < rows; ++r) {
        const std::vector<int32_t> w = tail(e, contexts + int64_t(r) * length, length);
        int32_t npad = 0;
        while (npad < W && w[npad] == V) ++npad;
        if (npad == W || steps - 1 > npad) {
            return e->fail(-8, "row " + std::to_string(r) + ": the window drops a real token "
                               "within the forced steps");
        }
        // Left-pad (prompt real tokens, forced[0..steps-2]) to the window.
        float* row = ids.data() + int64_t(r) * W;
        const int32_t lead = npad - (steps - 1);
        for (int32_t t = 0; t < lead; ++t) row[t] = pad;
        for (int32_t t = npad; t < W; ++t) row[lead + t - npad] = static_cast<float>(w[t]);
        for (int32_t g = 0; g + 1 < steps; ++g) {
            const int32_t id = forced[int64_t(r) * steps + g];
            if (id < 0 || id >= V) return e->fail(-1, "forced token outside the vocabulary");
            row[W - (steps - 1) + g] = static_cast<float>(id);
        }
    }
    // Rows in groups of four bound the [rows, H, W, W] attention scores.
    for (int32_t r0 = 0; r0 < rows; r0 += 4) {
        const int32_t n = std::min<int32_t>(4, rows - r0);
        status = decoder_forward(e, ids.data() + int64_t(r0) * W, n,
                                 logits + int64_t(r0) * steps * V, W - steps);
        if (status) return status;
    }
    return 0;
}

// Synthetic weights: every parameter N(0, stddev) from java.util.Random(seed).nextGaussian in
// namedParameters order, LayerNorm gamma 1 and beta 0, matrices and embedding tables rounded to
// bf16 (round to nearest even) when round_bf16 != 0. The LastTokenModel keeps its fixture weights.
extern "C" int32_t orc_fill_synthetic(orc_engine* e, int64_t seed, double stddev,
                                      int32_t round_bf16) {
    if (e->spec.family == ORC_FAMILY_LAST_TOKEN) return 0;
    orc_random random;
    orc_random_set_seed(&random, seed);
    auto ends = [](const std::string& n, const char* suffix) {
        const size_t k = std::strlen(suffix);
        return n.size() >= k && n.compare(n.size() - k, k, suffix) == 0;
    };
    for (size_t i = 0; i < e->names.size(); ++i) {
        const std::string& n = e->names[i];
        std::vector<float>& v = e->values[i];
        if (n.find("norm") != std::string::npos && (ends(n, ".gamma") || ends(n, ".beta"))) {
            std::fill(v.begin(), v.end(), ends(n, ".gamma") ? 1.0f : 0.0f);
            continue;
        }
        const bool matrix = e->spec.family == ORC_FAMILY_CHAR_LM
                                ? (n == "param0" || n == "param1" || n == "param3" || n == "param5")
                                : ends(n, ".weight");
        for (float& x : v) {
            x = static_cast<float>(orc_random_next_gaussian(&random) * stddev);
            if (round_bf16 && matrix && !std::isnan(x)) {
                uint32_t u;
                std::memcpy(&u, &x, 4);
                u += 0x7fffu + ((u >> 16) & 1u);
                u &= 0xffff0000u;
                std::memcpy(&x, &u, 4);
            }
        }
    }
    return 0;
}

// Prompts of java.util.Random(seed).nextInt(bound) ids, row after row.
extern "C" void orc_synthetic_prompts(int64_t seed, int32_t rows, int32_t length, int32_t bound,
                                      int32_t* out) {
    orc_random random;
    orc_random_set_seed(&random, seed);
    for (int64_t i = 0; i < int64_t(rows) * length; ++i) out[i] = orc_random_next_int_bound(&random, bound);
}

extern "C" int32_t orc_draw(orc_engine* e, const double* scores, int32_t count, float temperature,
                            int32_t top_k) {
    if (check_sampling(e, temperature, top_k)) return -1;
    return draw(e, scores, count, temperature, std::min(top_k, count));
}
