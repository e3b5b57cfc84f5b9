/*
 * CPU oracle for the TextEngine decode path — TEST INFRASTRUCTURE ONLY.
 *
 * This library restates, on the CPU, what the reference (Basalt 3.14.0) computes on the path
 * behind basalt.infer.TextEngine: the Java decode loop (src/main/java/basalt/infer/TextEngine.java)
 * and the Rust forward kernels it drives (native/src/gemm.rs, native/src/ops.rs,
 * native/src/nn_ops.rs), plus java.util.Random from the JDK's published specification.
 *
 * Only tests/, __graft_entry__.smoke() and the CPU-baseline leg of bench.py may load it, and only
 * as the checker or as the timed CPU baseline. The CUDA product never links or calls it.
 *
 * Parity pins: java.util.Random known answers from the JDK; the reference's own TextEngineTest
 * (LastTokenModel) known answers; NativeTestSuite op values and matmul shapes; gemm.rs unit cases.
 * Transformer logits have no reference golden vectors (the reference publishes none and cannot run
 * here: no JDK, no cargo), so those are pinned only through this restatement.
 */
#ifndef BASALT_ORACLE_H
#define BASALT_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- java.util.Random (JDK spec: 48-bit LCG, multiplier 0x5DEECE66D, addend 0xB) ---- */
typedef struct orc_random {
    uint64_t seed;            /* 48-bit state */
    int32_t have_next_gaussian;
    double next_gaussian;
} orc_random;

void orc_random_set_seed(orc_random* r, int64_t seed);
int32_t orc_random_next(orc_random* r, int32_t bits);
int32_t orc_random_next_int(orc_random* r);
int32_t orc_random_next_int_bound(orc_random* r, int32_t bound);
float orc_random_next_float(orc_random* r);
double orc_random_next_double(orc_random* r);
double orc_random_next_gaussian(orc_random* r);

/* ---- gemm.rs restatement: C[m,n] = A[m,k] * B[k,n] (row-major, C overwritten).
 * fused_tiles != 0 mirrors the AVX2/FMA path (gemm.rs:64-70): elements in the tiled region
 * (rows < m - m%6, cols < n - n%16) accumulate with fused multiply-add in k order
 * (gemm.rs:137-158); all others use the scalar dot_row (gemm.rs:268-285), a separate multiply then
 * add. fused_tiles == 0 mirrors BASALT_GEMM_SCALAR / no-AVX2 (gemm.rs:287-325). */
void orc_matmul(const float* a, const float* b, float* c, int64_t m, int64_t k, int64_t n,
                int32_t fused_tiles);

/* Elementwise ops of ops.rs::binary_forward (ops.rs:186-284) with trailing broadcast of b. */
int32_t orc_add(const float* a, const int64_t* a_shape, int32_t a_rank, const float* b,
                const int64_t* b_shape, int32_t b_rank, float* out);
int32_t orc_mul(const float* a, const int64_t* a_shape, int32_t a_rank, const float* b,
                const int64_t* b_shape, int32_t b_rank, float* out);
void orc_relu(const float* a, float* out, int64_t n);
void orc_gelu(const float* a, float* out, int64_t n);
int32_t orc_softmax(const float* a, float* out, int64_t rows, int64_t dim);
int32_t orc_layer_norm(const float* a, const float* gamma, const float* beta, float* out,
                       int64_t rows, int64_t dim, float eps);

/* ---- models ---- */
enum {
    ORC_FAMILY_PADDED_DECODER = 1, /* causal decoder whose mask also hides leading PAD (= V) ids */
    ORC_FAMILY_DECODER = 2,        /* stock TransformerBlock stack, causal mask only */
    ORC_FAMILY_CHAR_LM = 3,        /* Zoo.charLm windowed MLP (Zoo.java:135-168) */
    ORC_FAMILY_LAST_TOKEN = 4      /* TextEngineTest.LastTokenModel (TextEngineTest.java:210-243) */
};

typedef struct orc_spec {
    int32_t family;
    int32_t vocabulary; /* V: logits per row */
    int32_t window;     /* W */
    int32_t dimension;  /* d */
    int32_t layers;     /* L */
    int32_t heads;      /* H */
    int32_t hidden;     /* FFN width (decoders) or bottleneck width (charLm) */
    int32_t fused_tiles;/* gemm.rs AVX2 path on (1) or scalar path (0) */
} orc_spec;

typedef struct orc_engine orc_engine;

orc_engine* orc_engine_create(const orc_spec* spec);
void orc_engine_destroy(orc_engine* e);
const char* orc_engine_error(orc_engine* e);
/* Parameter table in TextEngine file order: count, then name / element count per entry. */
int32_t orc_param_count(orc_engine* e);
const char* orc_param_name(orc_engine* e, int32_t index);
int64_t orc_param_size(orc_engine* e, int32_t index);
int32_t orc_set_param(orc_engine* e, const char* name, const float* values, int64_t count);
int32_t orc_get_param(orc_engine* e, const char* name, float* values, int64_t count);
/* TextEngine.save / load (TextEngine.java:298-350): big-endian V, W, count, (UTF name, n, floats). */
int32_t orc_save(orc_engine* e, const char* path);
int32_t orc_load(orc_engine* e, const char* path);

/* Module.forward on [rows, W] float ids -> [rows, V] logits. */
int32_t orc_forward(orc_engine* e, const float* ids, int32_t rows, float* logits);

/* TextEngine methods. Contexts are [rows, length] int32, length >= W; only the tail is used.
 * The sink pointer receives each produced token in order (may be NULL). */
typedef void (*orc_sink)(void* user, int32_t row, int32_t step, int32_t token);
int32_t orc_scores_batch(orc_engine* e, const int32_t* contexts, int32_t rows, int32_t length,
                         double* scores);
int32_t orc_generate(orc_engine* e, const int32_t* context, int32_t length, int32_t steps,
                     int32_t* produced, orc_sink sink, void* user);
// Greedy batch decode of the padded decoder with a per-row KV cache (CPU timing baseline).
int32_t orc_generate_batch_cached(orc_engine* e, const int32_t* contexts, int32_t rows,
                                  int32_t length, int32_t steps, int32_t* produced);
int32_t orc_generate_batch(orc_engine* e, const int32_t* contexts, int32_t rows, int32_t length,
                           int32_t steps, int32_t* produced);
int32_t orc_sample(orc_engine* e, const int32_t* context, int32_t length, int32_t steps,
                   float temperature, int32_t top_k, int32_t* produced, orc_sink sink,
                   void* user);
void orc_seed(orc_engine* e, int64_t seed);
uint64_t orc_rng_state(orc_engine* e);
/* Sets the raw 48-bit generator state (as if `setSeed` had produced it). */
void orc_set_rng_state(orc_engine* e, uint64_t state);
/* Teacher-forced logits: runs `steps` greedy-shaped steps but pushes forced[step] instead of the
 * argmax, writing [steps, V] logits. Used to compare a GPU run step by step after a divergence. */
int32_t orc_forced_scores(orc_engine* e, const int32_t* context, int32_t length, int32_t steps,
                          const int32_t* forced, float* logits);
/* Teacher-forced logits of the padded decoder for `rows` rows ([rows, steps, V]), each row from
 * one causal pass over its real prompt tokens and forced[r*steps .. r*steps+steps-2]. Valid while
 * every step's window still starts with PAD (steps - 1 <= leading PADs < W); returns -8
 * otherwise. Agrees with orc_forced_scores up to the rounding of the row count's FMA region. */
int32_t orc_forced_scores_single_pass(orc_engine* e, const int32_t* contexts, int32_t rows,
                                      int32_t length, int32_t steps, const int32_t* forced,
                                      float* logits);
/* Fills the parameters with N(0, stddev) from java.util.Random(seed).nextGaussian in parameter
 * order (LayerNorm gamma 1, beta 0; matrices rounded to bf16 when round_bf16). */
int32_t orc_fill_synthetic(orc_engine* e, int64_t seed, double stddev, int32_t round_bf16);
/* java.util.Random(seed).nextInt(bound), rows * length values row after row. */
void orc_synthetic_prompts(int64_t seed, int32_t rows, int32_t length, int32_t bound, int32_t* out);
/* The reference's draw() on a given score row (TextEngine.java:403-427) with the engine RNG. */
int32_t orc_draw(orc_engine* e, const double* scores, int32_t count, float temperature,
                 int32_t top_k);

int32_t orc_threads(void);
void orc_set_threads(int32_t threads);

#ifdef __cplusplus
}
#endif
#endif
