// Host-side launchers for the sm_100a decode kernels (kernels.cu). Every launcher queues work on
// the given stream and returns cudaGetLastError() of its launch.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace bst {

// Kernel classes, reported per class by the engine's timing counters.
enum KernelClass : int {
    kEmbed = 0,
    kLayerNorm = 1,
    kGemv = 2,
    kGemm = 3,
    kAttnDecode = 4,
    kAttnCombine = 5,
    kAttnPrefill = 6,
    kSelectGreedy = 7,
    kSelectSample = 8,
    kGather = 9,
    kHeadLastToken = 10,
    kMisc = 11,
    kSplit = 12,
    kDecodeStep = 13,
    kGemmStep = 14,  // tensor-core GEMMs inside a batched decode step (short, weight-streaming)
    kKernelClassCount = 15,
};

const char* kernel_class_name(int cls);

// Output stage fused into a projection. `value` = dot(x, w) + bias[n], the order of
// Linear.forward (torch/Linear.java:30-49): matMul, then the broadcast bias add.
enum class Epi : int {
    kStore = 0,        // out[m, n] = value
    kGelu = 1,         // out[m, n] = gelu(value)                           (Activation GELU)
    kResidual = 2,     // out[m, n] = out[m, n] + value                     (input.add(attended))
    kResidualGelu = 3, // out[m, n] = gelu(value + res[m, n])               (charLm back.add(flat))
    kQkv = 4,          // n < d: q[m, n] = value; else K/V cache at (row[m], slot[m])
    kLogits = 5,       // out[rowmap[m], n] = value
};

// Optional second copy of an output as tensor-core operand planes ([rows][ld], see
// launch_split_operand): the producer of a projection's input writes them so that the projection
// needs no separate split pass.
struct PlaneOut {
    void* hi = nullptr;
    void* lo = nullptr;
    int planes = 0;  // 0 none, 1 tf32 hi + fp32 remainder, 2 two bf16 planes
    int ld = 0;
};

struct EpiArgs {
    float* out = nullptr;
    int ldo = 0;
    const float* res = nullptr;
    int ldr = 0;
    const int* rowmap = nullptr;   // kLogits: destination row; kQkv: cache row
    const int* slot = nullptr;     // kQkv: cache slot
    void* k_cache = nullptr;       // kQkv: this layer's K cache [rows][H][S][hd]
    void* v_cache = nullptr;
    int d = 0, heads = 0, head_dim = 0, slots = 0;
    int kv_bf16 = 0;
    PlaneOut split;                // kStore, kGelu: also write the result as operand planes
    // kLogits: per destination row, the packed first maximum of the row's logits (pack_best),
    // combined with 64-bit atomicMax; nullptr when the caller selects from the logits itself.
    unsigned long long* best = nullptr;
    // kLogits with best and a K split: when step is set, the split-K fix-up (one block per row)
    // also takes TextEngine.argmax's token from the row's maximum and pushes it, as
    // k_select_greedy_packed does (window [rows][window_len], tokens [rows][steps], next, and
    // the step counter advanced once all `rows` rows of the step are done).
    int* step = nullptr;
    int* done = nullptr;
    int* tokens = nullptr;
    int* next = nullptr;
    int* window = nullptr;
    int window_len = 0, steps = 0, rows = 0;
};

// Optional LayerNorm applied to a projection's input rows (the pre-norm of TransformerBlock).
struct LnArgs {
    const float* gamma = nullptr;
    const float* beta = nullptr;
    float eps = 0.0f;
};

// Y = X[M, K] * W[N, K]^T + bias with the chosen epilogue. W is float32 or bf16 (w_bf16), K-major.
// With ln (GEMV path only; see linear_fuses_layernorm) the rows of X are layer-normalised first.
cudaError_t launch_linear(cudaStream_t s, const float* x, int ldx, const void* w, int w_bf16,
                          const float* bias, int M, int N, int K, Epi epi, const EpiArgs& ea,
                          const LnArgs* ln = nullptr);
// True when launch_linear can fuse the LayerNorm of its input for this shape.
bool linear_fuses_layernorm(int M, int N, int K);
// True when launch_linear(M, N, K) uses the small-M GEMV kernel.
bool linear_uses_gemv(int M, int N, int K);

// x[i] = tok[ids[i]] + pos[positions[i]] for a list of tokens.
cudaError_t launch_embed_tokens(cudaStream_t s, const void* tok, const void* pos, int w_bf16,
                                const int* ids, const int* positions, float* x, int count, int d);
// Decode step begin: for i < R, row = rowmap[i]: slot[i] = len[row]; len[row] += 1;
// x[i] = tok[next[row]] + pos[slot[i]].
cudaError_t launch_embed_decode(cudaStream_t s, const void* tok, const void* pos, int w_bf16,
                                const int* rowmap, const int* next, int* len, int* slot, float* x,
                                int R, int d);

// launch_embed_decode followed by the LayerNorm (gamma, beta, eps) of the embedded rows into
// operand planes hi/lo ([R, d]; planes = 1 tf32, 2 bf16) for the first layer's QKV projection.
// d <= 1024.
cudaError_t launch_embed_ln_decode(cudaStream_t s, const void* tok, const void* pos, int w_bf16,
                                   const int* rowmap, const int* next, int* len, int* slot, float* x,
                                   int R, int d, const float* gamma, const float* beta, float eps,
                                   void* hi, void* lo, int planes);

// LayerNorm over the last dimension with f64 statistics (nn_ops.rs:168-199). Writes y (fp32,
// optional) and, with planes = 1 (tf32) or 2 (bf16), the split operand planes hi/lo ([rows, d])
// that the tensor-core GEMM consumes.
cudaError_t launch_layernorm(cudaStream_t s, const float* x, int ldx, const float* gamma,
                             const float* beta, float* y, int ldy, int rows, int d, float eps,
                             void* hi = nullptr, void* lo = nullptr, int planes = 0);

// Split-K decode attention over the cache: q [R, d] -> out [R, d]. With splits > 1 each split
// writes (unnormalised output, max, sum of exponentials) to part [R, heads, splits, head_dim + 2]
// and the last split of each (row, head) to finish, found through tickets [R * heads] (zero
// between launches; the kernel re-arms them), merges them in split order.
// Split-K partial sums of the QKV projection ([splits][R][3d], launch_gemm_tc with
// defer_fixup) handed to the decode attention in place of q: each CTA sums the q of its head
// itself (in split order, then the bias, as k_splitk_reduce does), and the CTA whose cache range
// holds the step's own key sums that key and value and appends them to the cache.
struct QkvParts {
    const float* part = nullptr;
    int splits = 0;
    const float* bias = nullptr;
};
cudaError_t launch_attn_decode(cudaStream_t s, const float* q, void* k_cache, void* v_cache,
                               int kv_bf16, const int* rowmap, const int* len, int R, int heads,
                               int head_dim, int slots, float scale, int splits, int chunk,
                               float* part, int* tickets, float* out,
                               const PlaneOut& planes = PlaneOut{},
                               const QkvParts& qkv = QkvParts{});
// Causal prefill attention for `segments` rows; token t of segment j is packed at
// seg_start[j] + t and sits in cache slot t of row seg_row[j]. In both attention kernels `out`
// may be null when `planes` receives the result (the O projection reads only the planes).
cudaError_t launch_attn_prefill(cudaStream_t s, const float* q, const void* k_cache,
                                const void* v_cache, int kv_bf16, const int* seg_row,
                                const int* seg_start, const int* seg_len, int segments,
                                int max_len, int heads, int head_dim, int slots, float scale,
                                float* out, const PlaneOut& planes = PlaneOut{});

// Prefill token list from the device windows: for segment j (row seg_row[j], npad leading PAD
// ids), tokens window[row][npad + t] at positions t; a segment with no real token gets one PAD id
// at position 0. Also sets len[row] and the per-token (row, slot) pairs.
cudaError_t launch_prefill_tokens(cudaStream_t s, const int* window, int W, const int* seg_row,
                                  const int* seg_npad, const int* seg_start, const int* seg_len,
                                  int segments, int pad_id, int* ids, int* positions, int* tok_row,
                                  int* len);
// Gathers x[seg_start[j] + seg_len[j] - 1] into last[j].
cudaError_t launch_gather_last(cudaStream_t s, const float* x, const int* seg_start,
                               const int* seg_len, int segments, int d, float* last);
// charLm input: x[r, t*d + e] = emb[window[r][t], e] for r < rows.
cudaError_t launch_window_embed(cudaStream_t s, const int* window, int W, const void* emb,
                                int w_bf16, int rows, int d, float* x);
// LastTokenModel head: logits[r, v] = weight[floorMod(window[r][W-1], V), v] + bias[v].
cudaError_t launch_last_token(cudaStream_t s, const int* window, int W, const float* weight,
                              const float* bias, int rows, int V, float* logits);

// Token selection plus the step bookkeeping shared by both modes: tokens[r*steps + step] = t,
// next[r] = t, window[r] shifted left and t appended, and the device step counter advanced once
// every row is done. With `best`, the head's epilogue folded each row's first maximum into
// best[r] (EpiArgs::best) and the logits are not scanned again.
cudaError_t launch_select_greedy(cudaStream_t s, const float* logits, int rows, int V, int W,
                                 int steps, int* step, int* done, int* tokens, int* next,
                                 int* window, unsigned long long* best = nullptr);
// TextEngine.draw (TextEngine.java:403-427) per row with java.util.Random state rng[r]. With
// sorted_w / sorted_ids ([rows][V] scratch) the sums and the draw run in a second kernel, one
// warp per row, so that all rows' sequential sums run at once; without, one CTA does a row.
cudaError_t launch_select_sample(cudaStream_t s, const float* logits, int rows, int V, int W,
                                 int steps, float temperature, int top_k, uint64_t* rng,
                                 int* step, int* done, int* tokens, int* next, int* window,
                                 double* sorted_w = nullptr, int* sorted_ids = nullptr);
size_t select_sample_smem(int V);
size_t sample_draw_smem(int top_k);

// Sets kernel attributes that must be in place before the first launch on the current device.
cudaError_t configure_device_kernels();
// configure_device_kernels once per device for the process (the device must be current).
cudaError_t configure_device_kernels_once(int device);
// Message returned by bst_last_error(0) on this thread.
void set_thread_error(const std::string& message);

// ---- tensor-core projections (gemm_tc.cu) ----
cudaError_t configure_tc_kernels();
// True when Y = X W^T of this shape runs on tcgen05 (M > 8; K aligned for TMA).
bool tc_usable(int M, int N, int K, int w_bf16);
// Bytes of one split plane for an [M, K] operand.
size_t tc_split_bytes(int M, int K, int w_bf16);
// X -> (hi, lo) planes: tf32 truncation and fp32 remainder, or two bf16 planes (w_bf16).
cudaError_t launch_split_operand(cudaStream_t s, const float* x, int ldx, int M, int K, int w_bf16,
                                 void* hi, void* lo);
// Y = Xh*Wh + Xh*Wl + Xl*Wh (fp32 weights: w = Wh, w_lo = Wl) or Xh*W + Xl*W (bf16 weights),
// plus bias, through the epilogue. *err receives a non-zero code if a pipeline wait timed out.
// When the output tiles do not fill the SMs, K is split across CTAs: each writes its fp32 partial
// product to part[z] ([splits][M][N], part_bytes of room) and a second kernel sums the splits in
// order and runs the epilogue (deterministic). With part == nullptr the GEMM never splits.
cudaError_t launch_gemm_tc(cudaStream_t s, const void* x_hi, const void* x_lo, const void* w,
                           const void* w_lo, int w_bf16, const float* bias, int M, int N, int K,
                           Epi epi, const EpiArgs& ea, int* err, float* part = nullptr,
                           size_t part_bytes = 0, bool defer_fixup = false);
// Fix-up of a split residual projection fused with the LayerNorm that follows it, one warp per
// row: x[m, :] += sum_z part[z][m, :] + bias (splits in order, as the separate fix-up does), then
// LayerNorm of the new row (f64 statistics) written as the next projection's operand planes.
// N <= 1024.
cudaError_t launch_reduce_residual_ln(cudaStream_t s, const float* part, int splits, int M, int N,
                                      const float* bias, float* x, int ldx, const LnArgs& ln,
                                      void* hi, void* lo, int planes);
// Split count and tile width launch_gemm_tc chooses for this shape and scratch.
int tc_plan(int M, int N, int K, int w_bf16, size_t part_bytes, int* bn_out);
// Partial scratch that lets every shape reach one full wave of CTAs, and what one shape needs.
size_t tc_part_bytes_max();
size_t tc_part_bytes(int M, int N, int K, int w_bf16);

// Copies this step's logits of `rows` rows to history[h][*step][v] (history: [rows, steps, V]);
// history row h holds logits row rows_of[h] (h itself when rows_of is null).
cudaError_t launch_stash_logits(cudaStream_t s, const float* logits, int rows, int V, int steps,
                                const int* step, const int* rows_of, float* history);

// ---- whole decode step in one persistent kernel (decode_fused.cu) ----
// One layer's weights and cache for the fused step; an array of these lives in device memory.
struct FusedLayer {
    const void* wqkv = nullptr;  // [3d, d]
    const float* bqkv = nullptr;
    const void* wo = nullptr;    // [d, d]
    const float* bo = nullptr;
    const float *ln1_g = nullptr, *ln1_b = nullptr, *ln2_g = nullptr, *ln2_b = nullptr;
    const void* w1 = nullptr;    // [F, d]
    const float* b1 = nullptr;
    const void* w2 = nullptr;    // [d, F]
    const float* b2 = nullptr;
    void *k_cache = nullptr, *v_cache = nullptr;  // [R][H][slots][hd]
};

// Everything one greedy decode step of R rows reads and writes. Rows are cache rows 0..R-1;
// len[i] is row i's cache length before the step (the new key goes to slot len[i], and the
// select phase adds one).
struct FusedStep {
    int R = 0, d = 0, H = 0, F = 0, V = 0, W = 0, L = 0, slots = 0, steps = 0, nchunks = 0;
    float scale = 0.0f, eps = 0.0f;
    int *len = nullptr, *next = nullptr, *tokens = nullptr, *window = nullptr;
    int *step = nullptr, *done = nullptr;
    const int* rowmap = nullptr;  // identity [R]
    const void *tok_emb = nullptr, *pos_emb = nullptr;
    const float *lnf_g = nullptr, *lnf_b = nullptr;
    const void* head_w = nullptr;  // [V, d]
    const float* head_b = nullptr;
    float *x = nullptr, *q = nullptr, *att = nullptr, *ffn = nullptr, *logits = nullptr;
    float* part = nullptr;         // [R, H, nchunks, hd + 2]
    int* tickets = nullptr;        // [R * H], zero between launches
    unsigned* bar = nullptr;       // [0] grid barrier arrivals (only grows), [1] head ticket
    unsigned bar_base = 0;         // bar[0] when this launch starts
    unsigned long long* best = nullptr;  // [R] packed per-row maximum, zero between launches
    int* err = nullptr;            // non-zero when a grid barrier timed out
    double* stats = nullptr;       // [R][grid][2] per-CTA LayerNorm statistics (grid <= 256)
    float* history = nullptr;      // optional [R, steps, V] logits
    unsigned table_offset = 0;                     // layer table in shared memory (set by launch)
    unsigned wstage_offset = 0, wstage_bytes = 0;  // weight stage in shared memory (set by launch)
};

// True when the fused step handles this shape (R <= 8, head_dim 32/64/128, window <= 4096).
bool fused_decode_supported(int R, int d, int F, int W, int head_dim, int w_bf16);
// Prepares the kernel for this shape on the current device and returns the grid size (one CTA per
// SM), or 0 when its shared memory does not fit or the device cannot co-schedule it. Call outside
// stream capture.
int fused_decode_prepare(int R, int d, int F, int V, int L, int head_dim, int w_bf16, int kv_bf16);
// Grid barriers one launch passes (bar[0] grows by this times the grid size).
int fused_decode_barriers(int layers);
cudaError_t launch_decode_fused(cudaStream_t s, const FusedStep& p, const FusedLayer* layers,
                                int w_bf16, int kv_bf16, int head_dim, int ctas);

cudaError_t launch_fill_int(cudaStream_t s, int* p, int value, int count);
cudaError_t launch_iota(cudaStream_t s, int* p, int count);

}  // namespace bst
