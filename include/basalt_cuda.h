/*
 * basalt_cuda.h — C ABI of libbasalt_cuda.so, the B200 (sm_100a) decode engine behind
 * basalt.infer.TextEngine.
 *
 * The reference runs TextEngine's loop in Java and reaches its Rust kernels one op at a time
 * through JNI (src/main/java/basalt/nativebridge/NativeBindings.java:13-89, implemented by
 * native/src/api.rs:118-709). This library replaces that per-op traffic with one call per
 * TextEngine method: the whole decode loop — embedding, LayerNorm, projections, attention over an
 * HBM KV cache, LM head, argmax or seeded sampling — runs on the GPU. A JNI shim maps each
 * TextEngine method onto the entry point named in its comment.
 *
 * Conventions (native/src/error.rs:9-17, src/main/java/basalt/BasaltExceptionCode.java:7-15):
 * every entry returns 0 on success or a negative status; the message of the last failure is
 * available from bst_last_error. No C++ exception crosses this boundary.
 *
 * Handles are opaque 64-bit ids, never reused (native/src/tensor.rs:150-176 keeps the same rule
 * for tensors); destroying an engine twice returns BST_UNKNOWN_HANDLE. Calls on one engine are
 * serialised by the engine; engines on different devices are independent.
 */
#ifndef BASALT_CUDA_H
#define BASALT_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BST_ABI_VERSION 1

/* Status codes: native/src/error.rs:9-17. */
#define BST_OK 0
#define BST_INVALID (-1)          /* BasaltParameterException */
#define BST_SHAPE (-2)            /* BasaltShapeException */
#define BST_UNKNOWN_HANDLE (-3)   /* stale or unknown handle */
#define BST_CONTEXT (-4)          /* closed engine / mismatched saved model */
#define BST_GRAPH (-5)
#define BST_PANIC (-6)            /* CUDA fault or internal error */
#define BST_OOM (-7)              /* device or host allocation failed */
#define BST_UNSUPPORTED (-8)

/* Model families the engine runs. */
#define BST_FAMILY_PADDED_DECODER 1 /* pre-norm causal decoder (TransformerBlock.java:37-43) whose
                                       mask also hides leading PAD ids (PAD = vocabulary);
                                       positions count from the first non-PAD id */
#define BST_FAMILY_DECODER 2        /* the same blocks with the stock causal mask only: every step
                                       recomputes the full window, as the reference does */
#define BST_FAMILY_CHAR_LM 3        /* Zoo.charLm windowed MLP (zoo/Zoo.java:135-168) */
#define BST_FAMILY_LAST_TOKEN 4     /* TextEngineTest.LastTokenModel (TextEngineTest.java:210-243) */

#define BST_DTYPE_F32 0
#define BST_DTYPE_BF16 1

typedef uint64_t bst_engine;

typedef struct bst_model_spec {
    int32_t family;
    int32_t vocabulary;   /* V: tokens the head scores (TextEngine.vocabulary()) */
    int32_t window;       /* W: context length (TextEngine.window()) */
    int32_t dimension;    /* d */
    int32_t layers;       /* L (decoders) */
    int32_t heads;        /* H (decoders); d % H == 0 */
    int32_t hidden;       /* FFN width (decoders) or bottleneck width (charLm) */
    int32_t weight_dtype; /* BST_DTYPE_*: storage of matrices and embedding tables */
    int32_t kv_dtype;     /* BST_DTYPE_*: storage of the attention cache */
    int32_t max_rows;     /* rows decoded together per wave; 0 = sized from free memory */
    int32_t reserved[6];  /* must be zero */
} bst_model_spec;

/* Per-token callback (java.util.function.IntConsumer of TextEngine.stream / streamSampled,
 * TextEngine.java:181-221). Called once per produced token, in step order within each row.
 * Returning non-zero stops the call, which then returns BST_INVALID. */
typedef int32_t (*bst_token_sink)(void* user, int32_t row, int32_t step, int32_t token);

int32_t bst_abi_version(void);
int32_t bst_device_count(int32_t* count);

/* Engine lifecycle. Replaces TextEngine.of (TextEngine.java:61-74) together with the module it
 * binds: the spec names the architecture, parameters are then set by name. */
int32_t bst_engine_create(const bst_model_spec* spec, int32_t device, bst_engine* out);
int32_t bst_engine_destroy(bst_engine engine);

/* Recognition of a module by its namedParameters (torch/Module.java:27-34), the test TextEngine's
 * dispatch makes before it hands a module to this engine. `count` parameters: names[i] with
 * ranks[i] dimensions, all dimensions concatenated in `dims`, in the reference's layout (Linear
 * weight [in, out], bias [1, out]; LayerNorm gamma/beta [d]; Embedding [rows, d]). vocabulary and
 * window are TextEngine.of's arguments (TextEngine.java:61-74); heads is the decoder's head count
 * (MultiheadAttention's parameter shapes do not carry it; ignored otherwise). Recognised: the
 * padded decoder (embedding rows V + 1) and the stock decoder (V rows), Zoo.charLm
 * (zoo/Zoo.java:135-168) and the one-hot last-token head (TextEngineTest.java:210-243). Fills
 * `spec` (f32 storage, max_rows 0) or returns BST_UNSUPPORTED / BST_SHAPE with the reason. */
int32_t bst_recognize_model(const char* const* names, const int32_t* ranks, const int64_t* dims,
                            int32_t count, int32_t vocabulary, int32_t window, int32_t heads,
                            bst_model_spec* spec);
/* TextEngine.of(module, vocabulary, window) for a recognised module: creates the engine on
 * `device` with the given storage dtypes and copies every parameter by name
 * (Module.loadStateDict, torch/Module.java:68-76). values[i] holds parameter i's floats. */
int32_t bst_engine_create_from_parameters(const char* const* names, const int32_t* ranks,
                                          const int64_t* dims, const float* const* values,
                                          int32_t count, int32_t vocabulary, int32_t window,
                                          int32_t heads, int32_t weight_dtype, int32_t kv_dtype,
                                          int32_t device, bst_engine* out);

/* Parameters by name, in Module.namedParameters order (torch/Module.java:27-34). */
int32_t bst_parameter_count(bst_engine engine, int32_t* count);
int32_t bst_parameter_info(bst_engine engine, int32_t index, char* name, int32_t capacity,
                           int64_t* size);
/* Module.loadStateDict entry (torch/Module.java:68-76) / Tensor.setData. */
int32_t bst_set_parameter(bst_engine engine, const char* name, const float* values,
                          int64_t count);
/* Tensor.data of a parameter (float32 values as last set). */
int32_t bst_get_parameter(bst_engine engine, const char* name, float* values, int64_t count);
/* TextEngine.save / load (TextEngine.java:298-350): big-endian vocabulary, window, count, then
 * per parameter a modified-UTF-8 name, an element count and float32 values. */
int32_t bst_save(bst_engine engine, const char* path);
int32_t bst_load(bst_engine engine, const char* path);

/* TextEngine.scoresBatch / scores (TextEngine.java:96-148). contexts: [rows, length] row-major,
 * length >= window; only each row's tail is used. scores: [rows, vocabulary]. */
int32_t bst_scores(bst_engine engine, const int32_t* contexts, int32_t rows, int32_t length,
                   double* scores);

/* TextEngine.generate / stream / generateBatch (TextEngine.java:158-193, 232-254): greedy
 * decoding, first maximum wins. tokens: [rows, steps]. sink may be NULL. */
int32_t bst_generate(bst_engine engine, const int32_t* contexts, int32_t rows, int32_t length,
                     int32_t steps, int32_t* tokens, bst_token_sink sink, void* user);

/* TextEngine.sample / streamSampled (TextEngine.java:201-227, 267-285) with the engine's
 * java.util.Random. Rows are decoded together but draw exactly what `rows` successive calls on
 * one engine would: row r starts from the generator advanced by 2*steps*r, and the engine's
 * generator ends advanced by 2*steps*rows. */
int32_t bst_sample(bst_engine engine, const int32_t* contexts, int32_t rows, int32_t length,
                   int32_t steps, float temperature, int32_t top_k, int32_t* tokens,
                   bst_token_sink sink, void* user);

/* bst_generate / bst_sample that also return the logits each step was decided on:
 * logits [rows, steps, vocabulary] float32 (the scores TextEngine.scores would have returned for
 * that step's window, as the decode path computed them). */
int32_t bst_generate_logits(bst_engine engine, const int32_t* contexts, int32_t rows,
                            int32_t length, int32_t steps, int32_t* tokens, float* logits);
int32_t bst_sample_logits(bst_engine engine, const int32_t* contexts, int32_t rows,
                          int32_t length, int32_t steps, float temperature, int32_t top_k,
                          int32_t* tokens, float* logits);

/* bst_generate_logits / bst_sample_logits that keep the logits of `watch_count` chosen rows only:
 * logits [watch_count, steps, vocabulary], entry i for row watch_rows[i]. Lets a caller follow a
 * few sequences of a batch too large for every row's logits (TextEngine.scores of those rows'
 * windows at each step). Rows must be distinct and inside [0, rows). */
int32_t bst_generate_logits_rows(bst_engine engine, const int32_t* contexts, int32_t rows,
                                 int32_t length, int32_t steps, int32_t* tokens,
                                 int32_t watch_count, const int32_t* watch_rows, float* logits);
int32_t bst_sample_logits_rows(bst_engine engine, const int32_t* contexts, int32_t rows,
                               int32_t length, int32_t steps, float temperature, int32_t top_k,
                               int32_t* tokens, int32_t watch_count, const int32_t* watch_rows,
                               float* logits);

/* The same two calls for callers whose contexts and token buffers already live on the engine's
 * device (device pointers; no sink). */
int32_t bst_generate_device(bst_engine engine, const int32_t* contexts, int32_t rows,
                            int32_t length, int32_t steps, int32_t* tokens);
int32_t bst_sample_device(bst_engine engine, const int32_t* contexts, int32_t rows,
                          int32_t length, int32_t steps, float temperature, int32_t top_k,
                          int32_t* tokens);

/* TextEngine.seed (TextEngine.java:288-290) and raw access to the 48-bit generator state. */
int32_t bst_seed(bst_engine engine, int64_t seed);
int32_t bst_get_rng_state(bst_engine engine, int64_t* state);
int32_t bst_set_rng_state(bst_engine engine, int64_t state);

/* NativeContext.beginScope / endScope / scopeDepth (nativebridge/NativeContext.java:229-247,
 * native/src/context.rs:186-221): device buffers the engine allocates while a scope is open are
 * released when it ends. Weights are never scope-owned. */
int32_t bst_begin_scope(bst_engine engine);
int32_t bst_end_scope(bst_engine engine, int32_t* released);
int32_t bst_scope_depth(bst_engine engine, int32_t* depth);

/* NativeContext.stats (nativebridge/NativeContext.java:256-262, context.rs:404-414):
 * out[0] live device buffers, out[1] live device bytes, out[2] graph nodes (always 0: the engine
 * records no autograd graph), out[3] kernels launched so far. */
int32_t bst_engine_stats(bst_engine engine, int64_t out[4]);

/* The CUDA stream (cudaStream_t) all of the engine's work is queued on. */
int32_t bst_engine_stream(bst_engine engine, void** stream);

/* Per-kernel timing, the device-side counterpart of BasaltMetrics.recordOperator
 * (BasaltMetrics.java:203-281). While enabled, each launch is bracketed by CUDA events and the
 * engine accumulates launches, device milliseconds and algorithmic bytes per kernel class. */
#define BST_KERNEL_CLASSES 15
int32_t bst_profile_enable(bst_engine engine, int32_t enabled);
int32_t bst_profile_reset(bst_engine engine);
int32_t bst_profile_read(bst_engine engine, int32_t kernel_class, char* name, int32_t capacity,
                         int64_t* launches, double* milliseconds, double* bytes, double* flops);

/* Tensor.matMul (torch/Tensor.java:214-227) -> gemm::matmul (native/src/gemm.rs:42-74) on device
 * buffers: C[m, n] = A[m, k] * B[k, n], row-major float32, C overwritten. Runs on `device`, queued
 * on `stream` (a cudaStream_t; NULL is the legacy default stream) and returns once C is complete.
 * m <= 8 uses the GEMV kernel, larger m the tcgen05 GEMM (3xTF32). Temporaries (B transposed and
 * the split operand planes) come from the stream-ordered allocator. Errors: bst_last_error(0). */
int32_t bst_matmul(int32_t device, void* stream, const float* a, const float* b, float* c,
                   int64_t m, int64_t k, int64_t n);

/* bst_matmul that allocates no device memory, for callers that may not call cudaMalloc while
 * they run. No counterpart in the reference. Temporaries come from a 16 MiB scratch array built
 * into the library (held on every GPU that loads it until exit); problems whose scratch does not
 * fit are rejected with BST_SHAPE. The first call on a device looks up that array's device address
 * and should come before any stream capture. Calls share the array: work from calls that overlaps
 * on the GPU races, so such calls must be serialised by the caller. */
int32_t bst_matmul_static(int32_t device, void* stream, const float* a, const float* b, float* c,
                          int64_t m, int64_t k, int64_t n);

/* ---- Device tensors and the op queue (NativeContext on Device.cuda(i)) ----
 * A context is bound to one CUDA device. Its tensors live on that device (device tag 1000 + i,
 * Device.java:22,46-59) or on the host (tag 0). Tensor handles are monotonic per context and never
 * reused (native/src/tensor.rs:150-176). Ops run from the reference's packed queue of 128-byte
 * commands (CommandQueueBuilder.java:12-73): u8 op code, u8 flags, 6 pad, u64 inputs A..E, u64
 * output, i32 attrs[16], 8 reserved. Codes run on the GPU: MatMul 1, Add 2, ReLU 3, Sub 4, Mul 5,
 * Sigmoid 6, Tanh 7, Gelu 11, Exp 23, Log 24, Sqrt 25, Abs 26, Neg 27, Div 28 (binary ops broadcast
 * trailing axes as ops.rs:136-164); other codes return BST_UNSUPPORTED. Each executed op is
 * recorded as one graph node, as the reference's Graph::push does; no backward is offered. */
typedef uint64_t bst_context;
typedef uint64_t bst_tensor;
#define BST_DEVICE_TAG_CPU 0
#define BST_DEVICE_TAG_CUDA 1000
#define BST_COMMAND_BYTES 128

/* NativeContext.create for Device.cuda(i): device_tag = 1000 + i. Tag 0 (cpu) returns
 * BST_UNSUPPORTED: host contexts stay on the CPU engine. */
int32_t bst_context_create(int32_t device_tag, bst_context* out);
int32_t bst_context_destroy(bst_context context);
/* NativeContext.of / zeros (values NULL: zeros) on the device named by device_tag (0 or this
 * context's 1000 + i). */
int32_t bst_tensor_create(bst_context context, int32_t device_tag, const int64_t* shape,
                          int32_t rank, const float* values, bst_tensor* out);
/* NativeContext.transferTensor (native/src/context.rs:125-133): a copy on the target device, as
 * a new handle; host <-> device transfers are cudaMemcpy on the context's stream. */
int32_t bst_tensor_transfer(bst_context context, bst_tensor source, int32_t device_tag,
                            bst_tensor* out);
/* NativeTensorHandle.data / setData: count must equal the tensor's element count. */
int32_t bst_tensor_read(bst_context context, bst_tensor tensor, float* values, int64_t count);
int32_t bst_tensor_write(bst_context context, bst_tensor tensor, const float* values,
                         int64_t count);
/* Device tag, rank and up to `capacity` dimensions of a tensor. */
int32_t bst_tensor_info(bst_context context, bst_tensor tensor, int32_t* device_tag,
                        int32_t* rank, int64_t* shape, int32_t capacity);
/* NativeTensorHandle.close: releasing twice is harmless (*released 0 the second time); a handle
 * the context never issued returns BST_UNKNOWN_HANDLE. */
int32_t bst_tensor_release(bst_context context, bst_tensor tensor, int32_t* released);
/* NativeBindings.executeQueue (native/src/engine.rs:118-154): runs `count` commands in order and
 * returns once they have finished; the first failing command stops the queue with its status. */
int32_t bst_execute_queue(bst_context context, const void* commands, int32_t count);
/* out[0] live tensors, out[1] live device bytes, out[2] graph nodes (NativeContext.graphSize),
 * out[3] kernels launched. */
int32_t bst_context_stats(bst_context context, int64_t out[4]);
int32_t bst_context_clear_graph(bst_context context);

/* Message of the last failure on this engine (engine 0: on this thread). */
int32_t bst_last_error(bst_engine engine, char* buffer, int32_t capacity);

/* Synthetic inputs for tests and benchmarks: a TextEngine weight file whose parameters are
 * N(0, stddev) from java.util.Random(seed).nextGaussian (LayerNorm gamma 1, beta 0), and prompts
 * of java.util.Random(seed).nextInt(bound) ids, row after row. */
int32_t bst_write_synthetic_weights(const bst_model_spec* spec, const char* path, int64_t seed,
                                    double stddev);
int32_t bst_synthetic_prompts(int64_t seed, int32_t rows, int32_t length, int32_t bound,
                              int32_t* out);

#ifdef __cplusplus
}
#endif
#endif
