// libbasalt_cuda.so — the TextEngine decode loop on one B200, behind the C ABI of
// include/basalt_cuda.h.
//
// One Engine = one model on one device with one CUDA stream. A call (generate / sample / scores)
// runs the reference's loop (src/main/java/basalt/infer/TextEngine.java:96-427) as a sequence of
// device steps:
//   * the host plans, per row and step, whether the row's window can extend its KV cache by one
//     token (the window only dropped a leading PAD) or must be re-encoded from scratch (first
//     step, a saturated window, or the stock causal decoder whose positions move every step);
//   * prefill encodes packed windows with the batched kernels; decode runs one token per row;
//   * selection (first-max argmax, or draw() with per-row java.util.Random state) and the window
//     shift happen on the device, so steady decoding needs no host round trip and replays as one
//     CUDA graph per step.

#include "basalt_cuda.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "java_random.h"
#include "kernels.h"

namespace {

namespace jrand = bst::jrand;
using bst::Epi;
using bst::EpiArgs;

constexpr float kLayerNormEps = 1e-5f;   // TransformerBlock.java:26,29
constexpr int kLanes = 4;                // most row groups a batched decode step runs at once
constexpr int kMaxPrefillTokens = 1 << 17;  // tokens encoded per prefill launch group

thread_local std::string t_last_error;

struct Failure {
    int code;
    std::string message;
};

bool decoder_family(int f) { return f == BST_FAMILY_PADDED_DECODER || f == BST_FAMILY_DECODER; }

// Matrices and embedding tables are stored in the weight dtype; biases and LayerNorm parameters
// always in float32.
bool stored_as_matrix(int family, const std::string& name) {
    if (family == BST_FAMILY_LAST_TOKEN) return false;
    if (family == BST_FAMILY_CHAR_LM) {
        return name == "param0" || name == "param1" || name == "param3" || name == "param5";
    }
    const size_t dot = name.rfind('.');
    return dot != std::string::npos && name.compare(dot, std::string::npos, ".weight") == 0;
}

bool is_layernorm_gamma(const std::string& name) {
    auto ends = [&](const char* s) {
        const size_t n = std::strlen(s);
        return name.size() >= n && name.compare(name.size() - n, n, s) == 0;
    };
    return ends("norm1.gamma") || ends("norm2.gamma") || name == "norm.gamma";
}

// Parameter table of a family, in namedParameters order (torch/Module.java:27-34,
// TransformerBlock.java:56-65, MultiheadAttention.java:94-102, Sequential.java:48-57).
void declare_parameters(const bst_model_spec& s, std::vector<std::string>* names,
                        std::vector<int64_t>* sizes) {
    const int64_t V = s.vocabulary, W = s.window, d = s.dimension, F = s.hidden;
    auto add = [&](const std::string& n, int64_t c) {
        names->push_back(n);
        sizes->push_back(c);
    };
    if (decoder_family(s.family)) {
        add("embedding.weight", (s.family == BST_FAMILY_PADDED_DECODER ? V + 1 : V) * d);
        add("position.weight", W * d);
        for (int l = 0; l < s.layers; ++l) {
            const std::string p = "layer" + std::to_string(l) + ".";
            add(p + "norm1.gamma", d);
            add(p + "norm1.beta", d);
            for (const char* part : {"query", "key", "value", "output"}) {
                add(p + "attention." + part + ".weight", d * d);
                add(p + "attention." + part + ".bias", d);
            }
            add(p + "norm2.gamma", d);
            add(p + "norm2.beta", d);
            add(p + "ffn1.weight", d * F);
            add(p + "ffn1.bias", F);
            add(p + "ffn2.weight", F * d);
            add(p + "ffn2.bias", d);
        }
        add("norm.gamma", d);
        add("norm.beta", d);
        add("head.weight", d * V);
        add("head.bias", V);
    } else if (s.family == BST_FAMILY_CHAR_LM) {
        const int64_t flat = W * d;
        add("param0", V * d);
        add("param1", flat * F);
        add("param2", F);
        add("param3", F * flat);
        add("param4", flat);
        add("param5", flat * V);
        add("param6", V);
    } else if (s.family == BST_FAMILY_LAST_TOKEN) {
        add("param0", V * V);
        add("param1", V);
    }
}

uint16_t to_bf16_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if (std::isnan(f)) return 0x7fc0;
    u += 0x7fffu + ((u >> 16) & 1u);  // round to nearest even
    return static_cast<uint16_t>(u >> 16);
}

float round_to_bf16(float f) {
    const uint32_t u = static_cast<uint32_t>(to_bf16_bits(f)) << 16;
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}

Failure validate_spec(const bst_model_spec& s) {
    if (s.vocabulary < 2) return {BST_INVALID, "vocabulary must be at least 2, got " + std::to_string(s.vocabulary)};
    if (s.window < 1) return {BST_INVALID, "window must be at least 1, got " + std::to_string(s.window)};
    for (int r : s.reserved) {
        if (r != 0) return {BST_INVALID, "reserved spec fields must be zero"};
    }
    if (s.weight_dtype != BST_DTYPE_F32 && s.weight_dtype != BST_DTYPE_BF16) {
        return {BST_INVALID, "weight_dtype must be BST_DTYPE_F32 or BST_DTYPE_BF16"};
    }
    if (s.kv_dtype != BST_DTYPE_F32 && s.kv_dtype != BST_DTYPE_BF16) {
        return {BST_INVALID, "kv_dtype must be BST_DTYPE_F32 or BST_DTYPE_BF16"};
    }
    if (s.max_rows < 0) return {BST_INVALID, "max_rows must be non-negative"};
    if (decoder_family(s.family)) {
        if (s.dimension < 1 || s.heads < 1 || s.layers < 1 || s.hidden < 1) {
            return {BST_INVALID, "dimension, heads, layers and hidden must be positive"};
        }
        if (s.dimension % s.heads != 0) return {BST_INVALID, "dimension must be divisible by heads"};
        const int hd = s.dimension / s.heads;
        if (hd != 32 && hd != 64 && hd != 128) {
            return {BST_UNSUPPORTED, "head dimension " + std::to_string(hd) + " is not one of 32, 64, 128"};
        }
        if (s.dimension % 8 != 0 || s.hidden % 8 != 0) {
            return {BST_UNSUPPORTED, "dimension and hidden must be multiples of 8"};
        }
        if (s.window > 2048) return {BST_UNSUPPORTED, "window above 2048 is not supported"};
    } else if (s.family == BST_FAMILY_CHAR_LM) {
        if (s.dimension < 1 || s.hidden < 1) {
            return {BST_INVALID, "dimension and hidden must be at least 1"};
        }
        if (s.window > 2048) return {BST_UNSUPPORTED, "window above 2048 is not supported"};
    } else if (s.family == BST_FAMILY_LAST_TOKEN) {
        if (s.window > 2048) return {BST_UNSUPPORTED, "window above 2048 is not supported"};
    } else {
        return {BST_UNSUPPORTED, "unknown model family " + std::to_string(s.family)};
    }
    return {BST_OK, ""};
}

// ---------------------------------------------------------------------------------------------
// Recognising a module from its namedParameters (torch/Module.java:27-34): the names, in order,
// and the shapes in the reference's layout (Linear weights [in, out], biases [1, out], LayerNorm
// parameters [d], Embedding tables [rows, d]).
// ---------------------------------------------------------------------------------------------
struct ParamView {
    std::string name;
    std::vector<int64_t> dims;
    int64_t numel() const {
        int64_t n = 1;
        for (int64_t x : dims) n *= x;
        return n;
    }
    bool is(int64_t a, int64_t b) const { return dims.size() == 2 && dims[0] == a && dims[1] == b; }
};

Failure recognize(const std::vector<ParamView>& params, int vocabulary, int window, int heads,
                  bst_model_spec* out) {
    bst_model_spec s{};
    s.vocabulary = vocabulary;
    s.window = window;
    s.heads = 1;
    auto find = [&](const std::string& n) -> const ParamView* {
        for (const auto& p : params) {
            if (p.name == n) return &p;
        }
        return nullptr;
    };
    const Failure unsupported{BST_UNSUPPORTED,
                              "the module is not one of the served language models (a "
                              "TransformerBlock decoder with token and position embeddings, "
                              "Zoo.charLm, or a one-hot last-token head)"};
    const ParamView* emb = find("embedding.weight");
    const ParamView* pos = find("position.weight");
    const ParamView* head = find("head.weight");
    const ParamView* ffn1 = find("layer0.ffn1.weight");
    if (emb && pos && head && ffn1) {
        if (pos->dims.size() != 2 || head->dims.size() != 2 || emb->dims.size() != 2 ||
            ffn1->dims.size() != 2) {
            return {BST_SHAPE, "decoder matrices must be rank 2"};
        }
        const int64_t d = pos->dims[1];
        if (pos->dims[0] != window) {
            return {BST_SHAPE, "position.weight has " + std::to_string(pos->dims[0]) +
                                   " rows; the window is " + std::to_string(window)};
        }
        if (!head->is(d, vocabulary)) {
            return {BST_SHAPE, "head.weight must be [" + std::to_string(d) + ", " +
                                   std::to_string(vocabulary) + "]"};
        }
        if (emb->is(vocabulary + 1, d)) {
            s.family = BST_FAMILY_PADDED_DECODER;  // the extra row is PAD = vocabulary
        } else if (emb->is(vocabulary, d)) {
            s.family = BST_FAMILY_DECODER;
        } else {
            return {BST_SHAPE, "embedding.weight must be [" + std::to_string(vocabulary) + " or " +
                                   std::to_string(vocabulary + 1) + ", " + std::to_string(d) + "]"};
        }
        int layers = 0;
        while (find("layer" + std::to_string(layers) + ".norm1.gamma")) ++layers;
        if (heads < 1) {
            return {BST_INVALID, "the head count of a decoder must be given: MultiheadAttention's "
                                 "parameter shapes do not carry it"};
        }
        s.dimension = static_cast<int32_t>(d);
        s.layers = layers;
        s.heads = heads;
        s.hidden = static_cast<int32_t>(ffn1->dims[1]);
    } else if (params.size() == 7 && find("param0") && find("param6")) {
        // Zoo.charLm: embedding [V, d], expand [W d, h] + [1, h], contract [h, W d] + [1, W d],
        // head [W d, V] + [1, V] (zoo/Zoo.java:135-168).
        const ParamView& e0 = params[0];
        const ParamView& e1 = params[1];
        if (e0.dims.size() != 2 || e1.dims.size() != 2 || e0.dims[0] != vocabulary) return unsupported;
        s.family = BST_FAMILY_CHAR_LM;
        s.dimension = static_cast<int32_t>(e0.dims[1]);
        s.hidden = static_cast<int32_t>(e1.dims[1]);
        if (e1.dims[0] != static_cast<int64_t>(window) * s.dimension) {
            return {BST_SHAPE, "charLm expand weight must have window x dimension = " +
                                   std::to_string(static_cast<int64_t>(window) * s.dimension) +
                                   " rows"};
        }
    } else if (params.size() == 2 && params[0].name == "param0" && params[1].name == "param1" &&
               params[0].is(vocabulary, vocabulary) && params[1].numel() == vocabulary) {
        s.family = BST_FAMILY_LAST_TOKEN;  // TextEngineTest.LastTokenModel (Linear(V, V))
    } else {
        return unsupported;
    }
    const Failure f = validate_spec(s);
    if (f.code) return f;
    // Every parameter of the recognised architecture, by name, in order, with its element count.
    std::vector<std::string> names;
    std::vector<int64_t> sizes;
    declare_parameters(s, &names, &sizes);
    if (names.size() != params.size()) {
        return {BST_SHAPE, "the module has " + std::to_string(params.size()) +
                               " parameters; the recognised architecture has " +
                               std::to_string(names.size())};
    }
    for (size_t i = 0; i < names.size(); ++i) {
        if (params[i].name != names[i]) {
            return {BST_SHAPE, "parameter " + std::to_string(i) + " is " + params[i].name +
                                   ", expected " + names[i]};
        }
        if (params[i].numel() != sizes[i]) {
            return {BST_SHAPE, "parameter " + names[i] + " has " +
                                   std::to_string(params[i].numel()) + " values, expected " +
                                   std::to_string(sizes[i])};
        }
    }
    *out = s;
    return {BST_OK, ""};
}

Failure parameter_views(const char* const* names, const int32_t* ranks, const int64_t* dims,
                        int32_t count, std::vector<ParamView>* out) {
    if (count < 1 || !names || !ranks || !dims) {
        return {BST_INVALID, "names, ranks and dims must describe at least one parameter"};
    }
    size_t at = 0;
    for (int32_t i = 0; i < count; ++i) {
        if (!names[i]) return {BST_INVALID, "parameter name " + std::to_string(i) + " is null"};
        if (ranks[i] < 1 || ranks[i] > 8) {
            return {BST_SHAPE, std::string("parameter ") + names[i] + " has rank " +
                                   std::to_string(ranks[i])};
        }
        ParamView v{names[i], std::vector<int64_t>(dims + at, dims + at + ranks[i])};
        at += static_cast<size_t>(ranks[i]);
        for (int64_t x : v.dims) {
            if (x < 0) return {BST_SHAPE, std::string("parameter ") + names[i] + " has a negative dimension"};
        }
        out->push_back(std::move(v));
    }
    return {BST_OK, ""};
}

// ---------------------------------------------------------------------------------------------
// TextEngine weight file (TextEngine.java:298-350): big-endian int V, int W, int count, then per
// parameter DataOutputStream.writeUTF(name), int n, n floats.
// ---------------------------------------------------------------------------------------------
void put_u32(std::string& out, uint32_t v) {
    const char b[4] = {static_cast<char>(v >> 24), static_cast<char>(v >> 16),
                       static_cast<char>(v >> 8), static_cast<char>(v)};
    out.append(b, 4);
}

Failure write_weight_file(const char* path, int V, int W, const std::vector<std::string>& names,
                          const std::vector<std::vector<float>>& values) {
    std::string out;
    put_u32(out, static_cast<uint32_t>(V));
    put_u32(out, static_cast<uint32_t>(W));
    put_u32(out, static_cast<uint32_t>(names.size()));
    for (size_t i = 0; i < names.size(); ++i) {
        const std::string& n = names[i];  // ASCII names: modified UTF-8 is the bytes themselves
        out.push_back(static_cast<char>((n.size() >> 8) & 0xff));
        out.push_back(static_cast<char>(n.size() & 0xff));
        out += n;
        put_u32(out, static_cast<uint32_t>(values[i].size()));
        const size_t base = out.size();
        out.resize(base + 4 * values[i].size());
        char* dst = out.data() + base;
        for (float v : values[i]) {
            uint32_t bits;
            std::memcpy(&bits, &v, 4);
            if (std::isnan(v)) bits = 0x7fc00000u;  // Float.floatToIntBits
            dst[0] = static_cast<char>(bits >> 24);
            dst[1] = static_cast<char>(bits >> 16);
            dst[2] = static_cast<char>(bits >> 8);
            dst[3] = static_cast<char>(bits);
            dst += 4;
        }
    }
    FILE* f = std::fopen(path, "wb");
    if (!f) return {BST_INVALID, std::string("cannot write model to ") + path};
    const size_t n = std::fwrite(out.data(), 1, out.size(), f);
    const bool ok = std::fclose(f) == 0 && n == out.size();
    if (!ok) return {BST_INVALID, std::string("cannot write model to ") + path};
    return {BST_OK, ""};
}

struct StoredModel {
    int32_t vocabulary = 0, window = 0;
    std::map<std::string, std::vector<float>> params;
};

Failure read_weight_file(const char* path, StoredModel* out) {
    FILE* f = std::fopen(path, "rb");
    if (!f) return {BST_INVALID, std::string("cannot read model from ") + path};
    std::fseek(f, 0, SEEK_END);
    const long size = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    std::vector<unsigned char> buf(size > 0 ? static_cast<size_t>(size) : 0);
    const bool read_ok = size >= 0 && std::fread(buf.data(), 1, buf.size(), f) == buf.size();
    std::fclose(f);
    if (!read_ok) return {BST_INVALID, std::string("cannot read model from ") + path};
    size_t pos = 0;
    auto u32 = [&](uint32_t* v) {
        if (pos + 4 > buf.size()) return false;
        *v = (uint32_t(buf[pos]) << 24) | (uint32_t(buf[pos + 1]) << 16) |
             (uint32_t(buf[pos + 2]) << 8) | uint32_t(buf[pos + 3]);
        pos += 4;
        return true;
    };
    const Failure truncated{BST_INVALID, std::string("cannot read model from ") + path + ": truncated"};
    uint32_t v, w, count;
    if (!u32(&v) || !u32(&w) || !u32(&count)) return truncated;
    out->vocabulary = static_cast<int32_t>(v);
    out->window = static_cast<int32_t>(w);
    for (uint32_t i = 0; i < count; ++i) {
        if (pos + 2 > buf.size()) return truncated;
        const size_t len = (size_t(buf[pos]) << 8) | buf[pos + 1];
        pos += 2;
        if (pos + len > buf.size()) return truncated;
        std::string name(reinterpret_cast<const char*>(buf.data() + pos), len);
        pos += len;
        uint32_t n;
        if (!u32(&n) || pos + 4ull * n > buf.size()) return truncated;
        std::vector<float> values(n);
        for (uint32_t j = 0; j < n; ++j) {
            const uint32_t bits = (uint32_t(buf[pos]) << 24) | (uint32_t(buf[pos + 1]) << 16) |
                                  (uint32_t(buf[pos + 2]) << 8) | uint32_t(buf[pos + 3]);
            pos += 4;
            std::memcpy(&values[j], &bits, 4);
        }
        out->params[name] = std::move(values);
    }
    return {BST_OK, ""};
}

// ---------------------------------------------------------------------------------------------
// Engine
// ---------------------------------------------------------------------------------------------
struct Buffer {
    void* ptr = nullptr;
    size_t bytes = 0;
    int scope = 0;  // scope depth that owns it; -1 = engine lifetime (weights)
};

// A projection matrix on the device, K-major [out, in]: `w` in the weight dtype, plus (fp32
// weights only) its tf32 split w = hi + lo that the tensor-core path multiplies.
struct Matrix {
    const void* w = nullptr;
    const void* hi = nullptr;
    const void* lo = nullptr;
};

struct LayerWeights {
    Matrix wqkv;  // [3d, d]
    const float* bqkv = nullptr;
    Matrix wo;    // [d, d]
    const float* bo = nullptr;
    const float *ln1_g = nullptr, *ln1_b = nullptr, *ln2_g = nullptr, *ln2_b = nullptr;
    Matrix w1;    // [F, d]
    const float* b1 = nullptr;
    Matrix w2;    // [d, F]
    const float* b2 = nullptr;
};

// Per-row, per-step plan entry.
struct StepPlan {
    std::vector<int> prefill_rows, prefill_npad, prefill_len;  // len: tokens encoded (>= 1)
    std::vector<int> decode_rows, decode_len;                    // len: cache length after step
};

struct Workspace {
    // Capacities the buffers were sized for.
    int rows = 0, steps = 0, slots = 0, tokens = 0, splits = 0;
    Buffer arena;
    int *window = nullptr, *len = nullptr, *next = nullptr, *slot = nullptr;
    int *rowmap_all = nullptr, *rowmap_dec = nullptr, *tokens_out = nullptr;
    int *step = nullptr, *done = nullptr;
    uint64_t* rng = nullptr;
    int *seg_row = nullptr, *seg_npad = nullptr, *seg_start = nullptr, *seg_len = nullptr;
    int *tok_id = nullptr, *tok_pos = nullptr, *tok_row = nullptr;
    float *x = nullptr, *h = nullptr, *q = nullptr, *att = nullptr, *ffn = nullptr;
    float *last = nullptr, *last_h = nullptr, *logits = nullptr, *part = nullptr;
    int* attn_tickets = nullptr;  // decode-attention split merge tickets [rows * heads]
    float *flat = nullptr, *mixed = nullptr;  // charLm
    float* history = nullptr;                 // per-step logits, when requested
    int* hist_rows_of = nullptr;              // history row h holds the logits of this wave row
    size_t hist_capacity = 0;                 // floats the history buffer holds
    // Sampled runs over more rows than SMs: each row's sorted weights and token ids, handed from
    // the sorting kernel to the warp-per-row draw ([rows][V]).
    double* sorted_w = nullptr;
    int* sorted_ids = nullptr;
    size_t sorted_capacity = 0;               // rows x V entries
    void *xs_hi = nullptr, *xs_lo = nullptr;  // split operand planes of the tensor-core path
    void *ys_hi = nullptr, *ys_lo = nullptr;  // planes a producer writes for the next projection
    // The second decode lane's operand planes ([rows][max(d, F)]) and split-K partials.
    // Lanes 1.. of the batched decode step: operand planes ([rows][max(d, F)]) and split-K
    // partials of their own.
    void *lane_xs_hi[kLanes] = {}, *lane_xs_lo[kLanes] = {}, *lane_ys_hi[kLanes] = {},
         *lane_ys_lo[kLanes] = {};
    float* lane_part[kLanes] = {};
    int* err = nullptr;                       // tensor-core pipeline error code
    float* tc_part = nullptr;                 // split-K partial products
    unsigned* bar = nullptr;                  // fused decode step: barrier count, head ticket
    unsigned long long* best = nullptr;       // fused decode step: per-row packed maximum [8]
    double* fused_stats = nullptr;            // fused decode step: LayerNorm statistics [8][256][2]
    bst::FusedLayer* fused_layers = nullptr;  // fused decode step: per-layer table [L]
    void *k_cache = nullptr, *v_cache = nullptr;
    size_t kv_layer_elems = 0;
    uint64_t generation = 0;
};

struct KernelStats {
    int64_t launches = 0;
    double ms = 0.0, bytes = 0.0, flops = 0.0;
};

struct PendingTiming {
    cudaEvent_t start, stop;
    int cls;
    double bytes, flops;
};

enum class Mode { kGreedy, kSample, kScores };

class Engine {
   public:
    bst_model_spec spec{};
    int device = 0;
    cudaStream_t stream = nullptr;
    // Lanes of the batched decode step: the rows split into up to kLanes groups, lane i > 0 running
    // its layers on lane_stream[i] (forked from and joined back into `stream`), so the groups'
    // kernels fill each other's idle SM time.
    cudaStream_t lane_stream[kLanes] = {};
    cudaEvent_t lane_fork = nullptr, lane_join[kLanes] = {};
    int V = 0, W = 0, d = 0, L = 0, H = 0, hd = 0, F = 0;
    bool wbf16 = false, kvbf16 = false;
    std::vector<std::string> names;
    std::vector<std::vector<float>> values;
    std::unordered_map<std::string, size_t> index;
    bool dirty = true;
    uint64_t rng_state = jrand::scramble(0);
    std::mutex mu;
    std::string error;

    std::vector<Buffer> buffers;  // live device allocations other than the workspace arena
    int scope_depth = 0;
    Buffer weights;
    std::vector<LayerWeights> layers;
    const void *tok_emb = nullptr, *pos_emb = nullptr;
    Matrix head_w;
    const float *lnf_g = nullptr, *lnf_b = nullptr, *head_b = nullptr;
    Matrix cl_expand, cl_contract;  // charLm
    const float *cl_expand_b = nullptr, *cl_contract_b = nullptr;
    const float *lt_w = nullptr, *lt_b = nullptr;  // LastTokenModel

    Workspace ws;
    uint64_t next_generation = 1;
    cudaGraphExec_t graph = nullptr;
    std::string graph_key;
    int64_t graph_nodes = 0;
    int fused_rows = 0, fused_ctas = 0;  // shape the fused decode step was prepared for
    // Rows (global indices, in output order) whose logits a *_logits_rows call returns; empty:
    // every row. hist_count: rows of the current wave whose logits are stashed.
    std::vector<int32_t> watch;
    int hist_count = 0;
    // Greedy decoder runs: the head GEMM's epilogue folds each row's argmax into ws.best, and the
    // selection reads that instead of scanning the logits.
    bool head_argmax = false;
    unsigned fused_bar_base = 0;         // the fused step's barrier count on the device
    std::vector<bst::FusedLayer> fused_table;

    bool profiling = false;
    bool in_step = false;  // enqueuing a batched decode step (decode_layers)
    // Greedy steps whose head runs with a K split: the head's fix-up kernel pushes each row's
    // token itself (decode_head sets it up, enqueue_select then has nothing left to do).
    bool push_in_head = false;
    bool push_allowed = false;  // this step decodes every row of the run (no prefill rows)
    int push_steps = 0, push_rows = 0;
    // Whether every decode lane's head (rows per lane in `lanes`) runs the split-K fix-up that
    // can push the tokens.
    bool head_pushes(const int* lanes, int n) const {
        if (!push_allowed || !head_argmax || hist_count != 0 || W > 8 * 256) return false;
        for (int i = 0; i < n; ++i) {
            if (!linear_on_tc(head_w, lanes[i], V, d) ||
                bst::tc_plan(lanes[i], V, d, wbf16, bst::tc_part_bytes_max(), nullptr) <= 1) {
                return false;
            }
        }
        return true;
    }
    struct StepScope {
        bool& flag;
        explicit StepScope(bool& f) : flag(f) { flag = true; }
        ~StepScope() { flag = false; }
    };
    KernelStats stats[bst::kKernelClassCount];
    std::vector<PendingTiming> pending;
    std::vector<cudaEvent_t> event_pool;
    int64_t launches = 0;

    ~Engine() { release_all(); }

    int fail(int code, const std::string& message) {
        error = message;
        return code;
    }

    int cuda_fail(cudaError_t err, const char* what) {
        cudaGetLastError();  // clear the sticky-free error state where possible
        const int code = err == cudaErrorMemoryAllocation ? BST_OOM : BST_PANIC;
        return fail(code, std::string(what) + ": " + cudaGetErrorName(err) + ": " +
                              cudaGetErrorString(err));
    }

    void release_all() {
        if (device >= 0) cudaSetDevice(device);
        if (graph) cudaGraphExecDestroy(graph);
        graph = nullptr;
        if (ws.arena.ptr) cudaFree(ws.arena.ptr);
        ws = Workspace{};
        if (weights.ptr) cudaFree(weights.ptr);
        weights = Buffer{};
        for (auto& b : buffers) cudaFree(b.ptr);
        buffers.clear();
        for (auto& p : pending) {
            event_pool.push_back(p.start);
            event_pool.push_back(p.stop);
        }
        pending.clear();
        for (auto e : event_pool) cudaEventDestroy(e);
        event_pool.clear();
        if (stream) cudaStreamDestroy(stream);
        stream = nullptr;
        for (int i = 0; i < kLanes; ++i) {
            if (lane_stream[i]) cudaStreamDestroy(lane_stream[i]);
            if (lane_join[i]) cudaEventDestroy(lane_join[i]);
            lane_stream[i] = nullptr;
            lane_join[i] = nullptr;
        }
        if (lane_fork) cudaEventDestroy(lane_fork);
        lane_fork = nullptr;
    }

    // ---- launches with optional per-class timing ----
    cudaEvent_t take_event() {
        if (!event_pool.empty()) {
            cudaEvent_t e = event_pool.back();
            event_pool.pop_back();
            return e;
        }
        cudaEvent_t e = nullptr;
        cudaEventCreate(&e);
        return e;
    }

    template <typename Fn>
    cudaError_t launch(int cls, double bytes, double flops, int kernels, Fn&& fn) {
        if (cls == bst::kGemm && in_step) cls = bst::kGemmStep;
        if (!profiling) {
            launches += kernels;
            return fn();
        }
        PendingTiming t{take_event(), take_event(), cls, bytes, flops};
        cudaEventRecord(t.start, stream);
        const cudaError_t err = fn();
        cudaEventRecord(t.stop, stream);
        pending.push_back(t);
        launches += kernels;
        stats[cls].launches += kernels;
        return err;
    }

    void collect_timings() {
        if (pending.empty()) return;
        cudaStreamSynchronize(stream);
        for (auto& p : pending) {
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, p.start, p.stop);
            stats[p.cls].ms += ms;
            stats[p.cls].bytes += p.bytes;
            stats[p.cls].flops += p.flops;
            event_pool.push_back(p.start);
            event_pool.push_back(p.stop);
        }
        pending.clear();
    }

    // ---- parameters ----
    int upload_weights();
    // hist_rows: rows whose per-step logits this run keeps (0: none).
    int ensure_workspace(int rows, int steps, int slots, int tokens, int splits, int hist_rows,
                         bool sampling);
    void free_workspace();

    // ---- runs ----
    int run(Mode mode, const int32_t* contexts, int32_t rows, int32_t length, int32_t steps,
            float temperature, int32_t top_k, int32_t* tokens, bool tokens_on_device,
            bst_token_sink sink, void* user, double* scores, float* logits = nullptr);
    int run_wave(Mode mode, const std::vector<int32_t>& windows, int row0, int rows, int steps,
                 float temperature, int top_k, uint64_t rng_base, int32_t* tokens,
                 bool tokens_on_device, int total_rows, bst_token_sink sink, void* user,
                 double* scores, float* logits);
    void plan(const std::vector<int32_t>& windows, int rows, int steps,
              std::vector<StepPlan>* plans, int* max_slots, int* max_tokens) const;
    // presplit: the operand planes are already in ws.ys_* (planes_for) or, with presplit_xs, in
    // ws.xs_* (written by residual_ln).
    int linear(const float* x, int ldx, const Matrix& m, const float* bias, int M, int N, int K,
               Epi epi, const EpiArgs& ea, const char* what, const bst::LnArgs* ln = nullptr,
               bool presplit = false, bool presplit_xs = false);
    // x += X W^T + bias (a residual projection) followed by the LayerNorm `next` of the new x.
    // On the tensor-core path with a K split, one fused fix-up kernel does both and leaves the
    // normalised rows as operand planes in ws.xs_* (*normalised = true); otherwise it runs the
    // plain residual projection and the caller applies `next` itself.
    int residual_ln(const float* x, int ldx, const Matrix& m, const float* bias, int M, int N,
                    int K, bool presplit, const bst::LnArgs& next, const char* what,
                    bool* normalised);
    // Whether linear() takes the tensor-core path for this shape, and the operand planes a
    // producer should write for it (into ws.ys_*; none when the GEMV path consumes fp32).
    bool linear_on_tc(const Matrix& m, int M, int N, int K) const;
    bst::PlaneOut planes_for(const Matrix& m, int M, int N, int K) const;
    int enqueue_prefill(const StepPlan& p, size_t begin, size_t end);
    int enqueue_decode(int R, const int* rowmap, const std::vector<int>& lens);
    // The layers and head of a decode step for R rows whose embedded inputs are in ws.x, on
    // `stream` (enqueue_decode runs it once, or runs decode_layer and decode_head per lane with
    // the workspace views shifted).
    struct DecodePlan {
        int splits = 1, chunk = 32;  // decode attention: cache splits per (row, head), keys each
        double sum_len = 0;          // cached keys over the rows (for the byte counts)
    };
    int decode_plan(int R, const std::vector<int>& lens, DecodePlan* dp);
    int decode_layers(int R, const int* rowmap, const std::vector<int>& lens,
                      bool x_normalised);
    // Embeds the step's next token of R rows into ws.x (and with `normalise`, the first
    // layer's LayerNorm of them into the operand planes ws.xs_*).
    int embed_rows(int R, const int* rowmap, bool normalise);
    int decode_layer(int l, int R, const int* rowmap, const DecodePlan& dp, bool* x_normalised);
    // Layer l after its QKV projection: attention over the cache for R rows (q in ws.q, or summed
    // from the projection's split-K partials), output projection, LN2, FFN, and the next LN.
    // attn_class: the profiling class of its attention launch (the prefill's last layer counts
    // as prefill attention).
    int decode_after_qkv(int l, int R, const int* rowmap, const DecodePlan& dp,
                         const bst::QkvParts& qparts, bool* x_normalised,
                         int attn_class = bst::kAttnDecode);
    int decode_head(int R, const int* rowmap, bool x_normalised);
    int qkv_partials(const LayerWeights& lw, const bst::LnArgs* ln, int R, int splits);
    int enqueue_direct(int rows);
    int prepare_fused(int rows);
    int enqueue_fused(int rows, int steps, const std::vector<int>& lens, bool history);
    int enqueue_select(Mode mode, int rows, int steps, float temperature, int top_k,
                       bool history);
};

// Message for an error code a kernel recorded in the workspace's status word.
std::string pipeline_message(int code) {
    if (code == 11) return "a grid barrier of the fused decode step timed out";
    if (code == 12) return "the fused decode step's weight staging (TMA bulk copy) timed out";
    return "a tensor-core GEMM pipeline wait timed out (stage " + std::to_string(code) + ")";
}

std::mutex g_registry_mutex;
std::unordered_map<uint64_t, std::shared_ptr<Engine>> g_engines;
uint64_t g_next_handle = 1;

std::shared_ptr<Engine> find_engine(bst_engine h) {
    std::lock_guard<std::mutex> lock(g_registry_mutex);
    auto it = g_engines.find(h);
    return it == g_engines.end() ? nullptr : it->second;
}

int Engine::upload_weights() {
    if (!dirty && weights.ptr) return BST_OK;
    // Lay out every device tensor in one arena (256-byte aligned), converting on the host.
    struct Item {
        size_t offset;
        std::vector<unsigned char> bytes;
    };
    std::vector<Item> items;
    size_t total = 0;
    auto place = [&](std::vector<unsigned char>&& bytes) {
        total = (total + 255) & ~size_t(255);
        items.push_back({total, std::move(bytes)});
        total += items.back().bytes.size();
        return items.size() - 1;
    };
    auto f32 = [&](const std::vector<float>& v) {
        std::vector<unsigned char> b(v.size() * 4);
        std::memcpy(b.data(), v.data(), b.size());
        return place(std::move(b));
    };
    // Stores `rows_out` rows of length `cols_in` in the weight dtype: element (r, c) of the
    // device matrix is src(r, c). With `planes` (projection weights in fp32) the tf32 split
    // hi = truncate(v), lo = v - hi is stored as well.
    struct MatIdx {
        size_t w = 0, hi = 0, lo = 0;
        bool planes = false;
    };
    auto matrix_planes = [&](int64_t rows_out, int64_t cols_in, bool planes, auto&& src) {
        const size_t es = wbf16 ? 2 : 4;
        const size_t count = static_cast<size_t>(rows_out * cols_in);
        std::vector<unsigned char> b(count * es);
        std::vector<unsigned char> hb, lb;
        const bool split = planes && !wbf16;
        if (split) {
            hb.resize(count * 4);
            lb.resize(count * 4);
        }
        for (int64_t r = 0; r < rows_out; ++r) {
            for (int64_t c = 0; c < cols_in; ++c) {
                const float v = src(r, c);
                const size_t i = static_cast<size_t>(r * cols_in + c);
                if (wbf16) {
                    const uint16_t bits = to_bf16_bits(v);
                    std::memcpy(b.data() + i * 2, &bits, 2);
                } else {
                    std::memcpy(b.data() + i * 4, &v, 4);
                    if (split) {
                        uint32_t u;
                        std::memcpy(&u, &v, 4);
                        u &= 0xFFFFE000u;
                        float hi;
                        std::memcpy(&hi, &u, 4);
                        const float lo = v - hi;
                        std::memcpy(hb.data() + i * 4, &hi, 4);
                        std::memcpy(lb.data() + i * 4, &lo, 4);
                    }
                }
            }
        }
        MatIdx idx;
        idx.w = place(std::move(b));
        if (split) {
            idx.hi = place(std::move(hb));
            idx.lo = place(std::move(lb));
            idx.planes = true;
        }
        return idx;
    };
    auto matrix = [&](int64_t rows_out, int64_t cols_in, auto&& src) {
        return matrix_planes(rows_out, cols_in, false, src).w;
    };
    auto P = [&](const std::string& n) -> const std::vector<float>& { return values[index.at(n)]; };
    // Linear weight [in, out] -> device [out, in].
    auto transposed = [&](const std::vector<float>& w, int64_t in, int64_t out) {
        return matrix_planes(out, in, true, [&](int64_t r, int64_t c) { return w[c * out + r]; });
    };

    std::vector<size_t> slots_idx;
    struct LayerIdx {
        MatIdx wqkv, wo, w1, w2;
        size_t bqkv, bo, ln1g, ln1b, ln2g, ln2b, b1, b2;
    };
    std::vector<LayerIdx> li;
    size_t i_tok = 0, i_pos = 0, i_lnfg = 0, i_lnfb = 0, i_headb = 0;
    size_t i_e1b = 0, i_cb = 0, i_lt = 0;
    MatIdx i_head, i_e1, i_c;
    if (decoder_family(spec.family)) {
        const int64_t emb_rows = static_cast<int64_t>(P("embedding.weight").size()) / d;
        i_tok = matrix(emb_rows, d, [&](int64_t r, int64_t c) { return P("embedding.weight")[r * d + c]; });
        i_pos = matrix(W, d, [&](int64_t r, int64_t c) { return P("position.weight")[r * d + c]; });
        for (int l = 0; l < L; ++l) {
            const std::string p = "layer" + std::to_string(l) + ".";
            const auto& wq = P(p + "attention.query.weight");
            const auto& wk = P(p + "attention.key.weight");
            const auto& wv = P(p + "attention.value.weight");
            LayerIdx x{};
            x.wqkv = matrix_planes(3 * d, d, true, [&](int64_t r, int64_t c) {
                const auto& src = r < d ? wq : (r < 2 * d ? wk : wv);
                return src[c * d + (r % d)];
            });
            std::vector<float> bqkv;
            for (const char* part : {"query", "key", "value"}) {
                const auto& b = P(p + "attention." + part + ".bias");
                bqkv.insert(bqkv.end(), b.begin(), b.end());
            }
            x.bqkv = f32(bqkv);
            x.wo = transposed(P(p + "attention.output.weight"), d, d);
            x.bo = f32(P(p + "attention.output.bias"));
            x.ln1g = f32(P(p + "norm1.gamma"));
            x.ln1b = f32(P(p + "norm1.beta"));
            x.ln2g = f32(P(p + "norm2.gamma"));
            x.ln2b = f32(P(p + "norm2.beta"));
            x.w1 = transposed(P(p + "ffn1.weight"), d, F);
            x.b1 = f32(P(p + "ffn1.bias"));
            x.w2 = transposed(P(p + "ffn2.weight"), F, d);
            x.b2 = f32(P(p + "ffn2.bias"));
            li.push_back(x);
        }
        i_lnfg = f32(P("norm.gamma"));
        i_lnfb = f32(P("norm.beta"));
        i_head = transposed(P("head.weight"), d, V);
        i_headb = f32(P("head.bias"));
    } else if (spec.family == BST_FAMILY_CHAR_LM) {
        const int64_t flat = static_cast<int64_t>(W) * d;
        i_tok = matrix(V, d, [&](int64_t r, int64_t c) { return P("param0")[r * d + c]; });
        i_e1 = transposed(P("param1"), flat, F);
        i_e1b = f32(P("param2"));
        i_c = transposed(P("param3"), F, flat);
        i_cb = f32(P("param4"));
        i_head = transposed(P("param5"), flat, V);
        i_headb = f32(P("param6"));
    } else {
        i_lt = f32(P("param0"));
        i_headb = f32(P("param1"));
    }

    cudaError_t err = cudaSetDevice(device);
    if (err != cudaSuccess) return cuda_fail(err, "cudaSetDevice");
    // Slack after the last tensor: the fused decode step copies bias blocks with their ends
    // rounded up to 16 bytes.
    total += 256;
    if (weights.ptr && weights.bytes < total) {
        cudaFree(weights.ptr);
        weights = Buffer{};
    }
    if (!weights.ptr) {
        err = cudaMalloc(&weights.ptr, std::max<size_t>(total, 256));
        if (err != cudaSuccess) {
            weights.ptr = nullptr;
            return cuda_fail(err, "allocating the weight store");
        }
        weights.bytes = std::max<size_t>(total, 256);
        weights.scope = -1;
    }
    std::vector<unsigned char> staging(total);
    for (auto& it : items) std::memcpy(staging.data() + it.offset, it.bytes.data(), it.bytes.size());
    err = cudaMemcpy(weights.ptr, staging.data(), total, cudaMemcpyHostToDevice);
    if (err != cudaSuccess) return cuda_fail(err, "uploading weights");

    auto at = [&](size_t i) { return static_cast<const void*>(static_cast<char*>(weights.ptr) + items[i].offset); };
    auto atf = [&](size_t i) { return static_cast<const float*>(at(i)); };
    auto atm = [&](const MatIdx& i) {
        Matrix m;
        m.w = at(i.w);
        if (i.planes) {
            m.hi = at(i.hi);
            m.lo = at(i.lo);
        }
        return m;
    };
    layers.clear();
    if (decoder_family(spec.family)) {
        tok_emb = at(i_tok);
        pos_emb = at(i_pos);
        for (const auto& x : li) {
            LayerWeights w;
            w.wqkv = atm(x.wqkv); w.bqkv = atf(x.bqkv); w.wo = atm(x.wo); w.bo = atf(x.bo);
            w.ln1_g = atf(x.ln1g); w.ln1_b = atf(x.ln1b); w.ln2_g = atf(x.ln2g); w.ln2_b = atf(x.ln2b);
            w.w1 = atm(x.w1); w.b1 = atf(x.b1); w.w2 = atm(x.w2); w.b2 = atf(x.b2);
            layers.push_back(w);
        }
        lnf_g = atf(i_lnfg);
        lnf_b = atf(i_lnfb);
        head_w = atm(i_head);
        head_b = atf(i_headb);
    } else if (spec.family == BST_FAMILY_CHAR_LM) {
        tok_emb = at(i_tok);
        cl_expand = atm(i_e1);
        cl_expand_b = atf(i_e1b);
        cl_contract = atm(i_c);
        cl_contract_b = atf(i_cb);
        head_w = atm(i_head);
        head_b = atf(i_headb);
    } else {
        lt_w = atf(i_lt);
        lt_b = atf(i_headb);
    }
    dirty = false;
    return BST_OK;
}

void Engine::free_workspace() {
    if (graph) {
        cudaGraphExecDestroy(graph);
        graph = nullptr;
        graph_key.clear();
    }
    if (ws.arena.ptr) {
        cudaStreamSynchronize(stream);
        cudaFree(ws.arena.ptr);
    }
    ws = Workspace{};
}

int Engine::ensure_workspace(int rows, int steps, int slots, int tokens, int splits,
                             int hist_rows, bool sampling) {
    const size_t hist_floats = static_cast<size_t>(hist_rows) * steps * V;
    // The split draw pays off once the rows outnumber the SMs (one sorting CTA per row).
    const size_t sorted = sampling && rows > 148 ? static_cast<size_t>(rows) * V : 0;
    if (ws.arena.ptr && ws.rows >= rows && ws.steps >= steps && ws.slots == slots &&
        ws.tokens >= tokens && ws.splits >= splits && ws.hist_capacity >= hist_floats &&
        ws.sorted_capacity >= sorted) {
        return BST_OK;
    }
    free_workspace();
    const int act_rows = std::max(tokens, rows);
    const int64_t flat = static_cast<int64_t>(W) * d;
    size_t total = 0;
    std::vector<std::pair<void**, size_t>> plan;
    auto add = [&](void** p, size_t bytes) { plan.push_back({p, bytes}); };
    add(reinterpret_cast<void**>(&ws.window), sizeof(int) * rows * W);
    add(reinterpret_cast<void**>(&ws.len), sizeof(int) * rows);
    add(reinterpret_cast<void**>(&ws.next), sizeof(int) * rows);
    add(reinterpret_cast<void**>(&ws.slot), sizeof(int) * rows);
    add(reinterpret_cast<void**>(&ws.rowmap_all), sizeof(int) * rows);
    add(reinterpret_cast<void**>(&ws.rowmap_dec), sizeof(int) * rows);
    add(reinterpret_cast<void**>(&ws.tokens_out), sizeof(int) * static_cast<size_t>(rows) * steps);
    add(reinterpret_cast<void**>(&ws.step), sizeof(int));
    add(reinterpret_cast<void**>(&ws.done), sizeof(int));
    add(reinterpret_cast<void**>(&ws.err), sizeof(int));
    add(reinterpret_cast<void**>(&ws.bar), 2 * sizeof(unsigned));
    add(reinterpret_cast<void**>(&ws.best), std::max(8, rows) * sizeof(unsigned long long));
    add(reinterpret_cast<void**>(&ws.fused_stats), 8 * 256 * 2 * sizeof(double));
    {
        // Split planes for the widest tensor-core operand this run can see.
        const int kmax = decoder_family(spec.family) ? std::max(d, F)
                                                     : std::max(W * d, std::max(F, 1));
        const size_t plane = bst::tc_split_bytes(act_rows, kmax, wbf16);
        add(&ws.xs_hi, plane);
        add(&ws.xs_lo, plane);
        add(&ws.ys_hi, plane);
        add(&ws.ys_lo, plane);
        if (decoder_family(spec.family)) {
            const size_t lane_plane = bst::tc_split_bytes((rows + 1) / 2, std::max(d, F), wbf16);
            for (int i = 1; i < kLanes; ++i) {
                add(&ws.lane_xs_hi[i], lane_plane);
                add(&ws.lane_xs_lo[i], lane_plane);
                add(&ws.lane_ys_hi[i], lane_plane);
                add(&ws.lane_ys_lo[i], lane_plane);
                add(reinterpret_cast<void**>(&ws.lane_part[i]), bst::tc_part_bytes_max());
            }
        }
        add(reinterpret_cast<void**>(&ws.tc_part), bst::tc_part_bytes_max());
    }
    add(reinterpret_cast<void**>(&ws.rng), sizeof(uint64_t) * rows);
    add(reinterpret_cast<void**>(&ws.logits), sizeof(float) * static_cast<size_t>(rows) * V);
    if (sorted) {
        add(reinterpret_cast<void**>(&ws.sorted_w), sizeof(double) * sorted);
        add(reinterpret_cast<void**>(&ws.sorted_ids), sizeof(int) * sorted);
    }
    if (hist_floats) {
        add(reinterpret_cast<void**>(&ws.history), sizeof(float) * hist_floats);
        add(reinterpret_cast<void**>(&ws.hist_rows_of), sizeof(int) * rows);
    }
    if (decoder_family(spec.family)) {
        add(reinterpret_cast<void**>(&ws.seg_row), sizeof(int) * rows);
        add(reinterpret_cast<void**>(&ws.seg_npad), sizeof(int) * rows);
        add(reinterpret_cast<void**>(&ws.seg_start), sizeof(int) * rows);
        add(reinterpret_cast<void**>(&ws.seg_len), sizeof(int) * rows);
        add(reinterpret_cast<void**>(&ws.tok_id), sizeof(int) * act_rows);
        add(reinterpret_cast<void**>(&ws.tok_pos), sizeof(int) * act_rows);
        add(reinterpret_cast<void**>(&ws.tok_row), sizeof(int) * act_rows);
        add(reinterpret_cast<void**>(&ws.x), sizeof(float) * static_cast<size_t>(act_rows) * d);
        add(reinterpret_cast<void**>(&ws.h), sizeof(float) * static_cast<size_t>(act_rows) * d);
        add(reinterpret_cast<void**>(&ws.q), sizeof(float) * static_cast<size_t>(act_rows) * d);
        add(reinterpret_cast<void**>(&ws.att), sizeof(float) * static_cast<size_t>(act_rows) * d);
        add(reinterpret_cast<void**>(&ws.ffn), sizeof(float) * static_cast<size_t>(act_rows) * F);
        add(reinterpret_cast<void**>(&ws.last), sizeof(float) * static_cast<size_t>(rows) * d);
        add(reinterpret_cast<void**>(&ws.last_h), sizeof(float) * static_cast<size_t>(rows) * d);
        add(reinterpret_cast<void**>(&ws.part),
            sizeof(float) * static_cast<size_t>(rows) * H * splits * (hd + 2));
        add(reinterpret_cast<void**>(&ws.attn_tickets), sizeof(int) * static_cast<size_t>(rows) * H);
        add(reinterpret_cast<void**>(&ws.fused_layers), sizeof(bst::FusedLayer) * L);
        ws.kv_layer_elems = static_cast<size_t>(rows) * H * slots * hd;
        const size_t kvb = (kvbf16 ? 2 : 4) * ws.kv_layer_elems * L;
        add(&ws.k_cache, kvb);
        add(&ws.v_cache, kvb);
    } else if (spec.family == BST_FAMILY_CHAR_LM) {
        add(reinterpret_cast<void**>(&ws.flat), sizeof(float) * static_cast<size_t>(rows) * flat);
        add(reinterpret_cast<void**>(&ws.ffn), sizeof(float) * static_cast<size_t>(rows) * F);
        add(reinterpret_cast<void**>(&ws.mixed), sizeof(float) * static_cast<size_t>(rows) * flat);
    }
    std::vector<size_t> offsets;
    for (auto& p : plan) {
        total = (total + 255) & ~size_t(255);
        offsets.push_back(total);
        total += p.second;
    }
    void* base = nullptr;
    cudaError_t err = cudaMalloc(&base, std::max<size_t>(total, 256));
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(BST_OOM, "cannot allocate " + std::to_string(total) +
                                 " bytes of device workspace: " + cudaGetErrorString(err));
    }
    for (size_t i = 0; i < plan.size(); ++i) *plan[i].first = static_cast<char*>(base) + offsets[i];
    ws.arena = Buffer{base, std::max<size_t>(total, 256), scope_depth};
    ws.rows = rows;
    ws.steps = steps;
    ws.slots = slots;
    ws.tokens = tokens;
    ws.splits = splits;
    ws.hist_capacity = hist_floats;
    ws.sorted_capacity = sorted;
    ws.generation = next_generation++;
    err = bst::launch_iota(stream, ws.rowmap_all, rows);
    if (!err && ws.attn_tickets) {
        err = cudaMemsetAsync(ws.attn_tickets, 0, sizeof(int) * static_cast<size_t>(rows) * H,
                              stream);
    }
    if (err != cudaSuccess) return cuda_fail(err, "initialising the workspace");
    return BST_OK;
}

// Plans every step of every row (padded and stock decoders). A row extends its cache at step g
// when its previous window held a real token and dropped a PAD (npad >= 1); otherwise the
// window is re-encoded. Generated tokens are never PAD (the head scores ids 0..V-1), so leading
// PAD counts follow from the context alone.
void Engine::plan(const std::vector<int32_t>& windows, int rows, int steps,
                  std::vector<StepPlan>* plans, int* max_slots, int* max_tokens) const {
    plans->assign(steps, StepPlan{});
    *max_slots = 1;
    *max_tokens = rows;
    const bool padded = spec.family == BST_FAMILY_PADDED_DECODER;
    std::vector<int64_t> tokens_at(steps, 0);
    for (int r = 0; r < rows; ++r) {
        const int32_t* w0 = windows.data() + static_cast<size_t>(r) * W;
        int npad_prev = -1, n_prev = -1;
        for (int g = 0; g < steps; ++g) {
            int npad = 0;
            if (padded) {
                if (g == 0) {
                    while (npad < W && w0[npad] == V) ++npad;
                } else if (npad_prev >= 1) {
                    npad = npad_prev - 1;
                } else {
                    while (npad < W && g + npad < W && w0[g + npad] == V) ++npad;
                }
            }
            const int n = W - npad;
            StepPlan& p = (*plans)[g];
            if (g == 0 || !padded || npad_prev < 1 || n_prev < 1) {
                const int encoded = std::max(n, 1);
                p.prefill_rows.push_back(r);
                p.prefill_npad.push_back(npad);
                p.prefill_len.push_back(encoded);
                tokens_at[g] += encoded;
                *max_slots = std::max(*max_slots, encoded);
            } else {
                p.decode_rows.push_back(r);
                p.decode_len.push_back(n);
                *max_slots = std::max(*max_slots, n);
            }
            npad_prev = npad;
            n_prev = n;
        }
    }
    for (int g = 0; g < steps; ++g) {
        *max_tokens = static_cast<int>(std::max<int64_t>(
            *max_tokens, std::min<int64_t>(tokens_at[g], kMaxPrefillTokens)));
    }
    for (int g = 0; g < steps; ++g) {
        for (int len : (*plans)[g].prefill_len) *max_tokens = std::max(*max_tokens, len);
    }
}

// One projection: GEMV (M <= 8) or tiled FFMA for odd shapes, otherwise split the operand and
// run the tcgen05 GEMM.
bool Engine::linear_on_tc(const Matrix& m, int M, int N, int K) const {
    return bst::tc_usable(M, N, K, wbf16) && (wbf16 || m.hi);
}

bst::PlaneOut Engine::planes_for(const Matrix& m, int M, int N, int K) const {
    bst::PlaneOut po;
    if (linear_on_tc(m, M, N, K)) {
        po.hi = ws.ys_hi;
        po.lo = ws.ys_lo;
        po.planes = wbf16 ? 2 : 1;
        po.ld = K;
    }
    return po;
}

int Engine::residual_ln(const float* x, int ldx, const Matrix& m, const float* bias, int M, int N,
                        int K, bool presplit, const bst::LnArgs& next, const char* what,
                        bool* normalised) {
    *normalised = false;
    EpiArgs res;
    res.out = ws.x;
    res.ldo = d;
    const int splits = linear_on_tc(m, M, N, K)
                           ? bst::tc_plan(M, N, K, wbf16, bst::tc_part_bytes_max(), nullptr)
                           : 1;
    if (splits <= 1 || N > 1024 || N != d) {
        return linear(x, ldx, m, bias, M, N, K, Epi::kResidual, res, what, nullptr, presplit);
    }
    const double plane = static_cast<double>(bst::tc_split_bytes(M, K, wbf16));
    const double wbytes = static_cast<double>(N) * K * (wbf16 ? 2.0 : 8.0);
    cudaError_t err;
    if (!presplit) {
        err = launch(bst::kSplit, M * K * 4.0 + 2 * plane, 0, 1, [&] {
            return bst::launch_split_operand(stream, x, ldx, M, K, wbf16, ws.ys_hi, ws.ys_lo);
        });
        if (err) return cuda_fail(err, what);
    }
    err = launch(bst::kGemm, wbytes + 2 * plane + static_cast<double>(splits) * M * N * 4.0,
                 2.0 * M * N * K, 1, [&] {
                     return bst::launch_gemm_tc(stream, ws.ys_hi, ws.ys_lo, wbf16 ? m.w : m.hi,
                                                m.lo, wbf16, bias, M, N, K, Epi::kResidual, res,
                                                ws.err, ws.tc_part, bst::tc_part_bytes_max(),
                                                true);
                 });
    if (err) return cuda_fail(err, what);
    const double out_plane = static_cast<double>(bst::tc_split_bytes(M, N, wbf16));
    err = launch(bst::kLayerNorm, (splits + 2.0) * M * N * 4.0 + 2 * out_plane, 0, 1, [&] {
        return bst::launch_reduce_residual_ln(stream, ws.tc_part, splits, M, N, bias, ws.x, d, next,
                                              ws.xs_hi, ws.xs_lo, wbf16 ? 2 : 1);
    });
    if (err) return cuda_fail(err, what);
    *normalised = true;
    return BST_OK;
}

int Engine::linear(const float* x, int ldx, const Matrix& m, const float* bias, int M, int N,
                   int K, Epi epi, const EpiArgs& ea, const char* what, const bst::LnArgs* ln,
                   bool presplit, bool presplit_xs) {
    const double wb = wbf16 ? 2.0 : 4.0;
    cudaError_t err;
    if (linear_on_tc(m, M, N, K)) {
        // Tensor-core path: the operand is split into hi/lo planes, by its producer (presplit:
        // already in ws.ys_*), by the LayerNorm when one precedes the projection, or by a split
        // pass.
        const double plane = static_cast<double>(bst::tc_split_bytes(M, K, wbf16));
        const int planes = wbf16 ? 2 : 1;
        const void* a_hi = presplit && !presplit_xs ? ws.ys_hi : ws.xs_hi;
        const void* a_lo = presplit && !presplit_xs ? ws.ys_lo : ws.xs_lo;
        if (presplit || presplit_xs) {
            err = cudaSuccess;
        } else if (ln) {
            err = launch(bst::kLayerNorm, M * K * 4.0 + 2 * plane, 0, 1, [&] {
                return bst::launch_layernorm(stream, x, ldx, ln->gamma, ln->beta, nullptr, 0, M,
                                             K, ln->eps, ws.xs_hi, ws.xs_lo, planes);
            });
        } else {
            err = launch(bst::kSplit, M * K * 4.0 + 2 * plane, 0, 1, [&] {
                return bst::launch_split_operand(stream, x, ldx, M, K, wbf16, ws.xs_hi, ws.xs_lo);
            });
        }
        if (err) return cuda_fail(err, what);
        const double wbytes = static_cast<double>(N) * K * (wbf16 ? 2.0 : 8.0);
        // A split-K GEMM is two kernels (partial products, then the ordered fix-up).
        const int kernels =
            bst::tc_plan(M, N, K, wbf16, bst::tc_part_bytes_max(), nullptr) > 1 ? 2 : 1;
        err = launch(bst::kGemm, wbytes + 2 * plane + static_cast<double>(M) * N * 4.0,
                     2.0 * M * N * K, kernels, [&] {
                         return bst::launch_gemm_tc(stream, a_hi, a_lo,
                                                    wbf16 ? m.w : m.hi, m.lo, wbf16, bias, M, N,
                                                    K, epi, ea, ws.err, ws.tc_part,
                                                    bst::tc_part_bytes_max());
                     });
        return err ? cuda_fail(err, what) : BST_OK;
    }
    if (presplit_xs) return fail(BST_PANIC, std::string(what) + ": operand planes on the GEMV path");
    const bst::LnArgs* fused = nullptr;
    if (ln) {
        if (bst::linear_fuses_layernorm(M, N, K)) {
            fused = ln;  // the GEMV normalises its input rows itself
        } else {
            err = launch(bst::kLayerNorm, M * K * 8.0, 0, 1, [&] {
                return bst::launch_layernorm(stream, x, ldx, ln->gamma, ln->beta, ws.h, K, M, K,
                                             ln->eps);
            });
            if (err) return cuda_fail(err, what);
            x = ws.h;
            ldx = K;
        }
    }
    const int cls = bst::linear_uses_gemv(M, N, K) ? bst::kGemv : bst::kMisc;
    err = launch(cls, static_cast<double>(N) * K * wb + static_cast<double>(M) * K * 4 +
                          static_cast<double>(M) * N * 4,
                 2.0 * M * N * K, 1, [&] {
                     return bst::launch_linear(stream, x, ldx, m.w, wbf16, bias, M, N, K, epi, ea,
                                               fused);
                 });
    return err ? cuda_fail(err, what) : BST_OK;
}

int Engine::enqueue_prefill(const StepPlan& p, size_t begin, size_t end) {
    const int segs = static_cast<int>(end - begin);
    std::vector<int> start(segs);
    int total = 0, max_len = 0;
    for (int j = 0; j < segs; ++j) {
        start[j] = total;
        total += p.prefill_len[begin + j];
        max_len = std::max(max_len, p.prefill_len[begin + j]);
    }
    cudaError_t err;
    err = cudaMemcpyAsync(ws.seg_row, p.prefill_rows.data() + begin, sizeof(int) * segs,
                          cudaMemcpyHostToDevice, stream);
    if (!err) err = cudaMemcpyAsync(ws.seg_npad, p.prefill_npad.data() + begin, sizeof(int) * segs,
                                    cudaMemcpyHostToDevice, stream);
    if (!err) err = cudaMemcpyAsync(ws.seg_start, start.data(), sizeof(int) * segs,
                                    cudaMemcpyHostToDevice, stream);
    if (!err) err = cudaMemcpyAsync(ws.seg_len, p.prefill_len.data() + begin, sizeof(int) * segs,
                                    cudaMemcpyHostToDevice, stream);
    // Pageable sources: make sure the copies have read the host vectors before they go away.
    if (!err) err = cudaStreamSynchronize(stream);
    if (err) return cuda_fail(err, "uploading prefill descriptors");

    const int T = total;
    const double wb = wbf16 ? 2.0 : 4.0, kvb = kvbf16 ? 2.0 : 4.0;
    const int slots = ws.slots;
    const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(hd)));
    auto check = [&](cudaError_t e, const char* what) { return e ? cuda_fail(e, what) : BST_OK; };
    int st;
    st = check(launch(bst::kGather, T * 12.0, 0, 1, [&] {
                   return bst::launch_prefill_tokens(stream, ws.window, W, ws.seg_row, ws.seg_npad,
                                                     ws.seg_start, ws.seg_len, segs, V, ws.tok_id,
                                                     ws.tok_pos, ws.tok_row, ws.len);
               }), "prefill tokens");
    if (st) return st;
    st = check(launch(bst::kEmbed, T * d * (2 * wb + 4.0), 0, 1, [&] {
                   return bst::launch_embed_tokens(stream, tok_emb, pos_emb, wbf16, ws.tok_id,
                                                   ws.tok_pos, ws.x, T, d);
               }), "embedding");
    if (st) return st;
    double attn_flops = 0, attn_bytes = 0;
    for (int j = 0; j < segs; ++j) {
        const double n = p.prefill_len[begin + j];
        attn_flops += 4.0 * H * hd * n * (n + 1) / 2.0;
        attn_bytes += n * d * (2 * kvb + 8.0);
    }
    for (int l = 0; l < L; ++l) {
        const LayerWeights& lw = layers[l];
        const bst::LnArgs ln1{lw.ln1_g, lw.ln1_b, kLayerNormEps};
        EpiArgs qkv;
        qkv.out = ws.q;
        qkv.ldo = d;
        qkv.rowmap = ws.tok_row;
        qkv.slot = ws.tok_pos;
        qkv.k_cache = static_cast<char*>(ws.k_cache) + l * ws.kv_layer_elems * static_cast<size_t>(kvb);
        qkv.v_cache = static_cast<char*>(ws.v_cache) + l * ws.kv_layer_elems * static_cast<size_t>(kvb);
        qkv.d = d;
        qkv.heads = H;
        qkv.head_dim = hd;
        qkv.slots = slots;
        qkv.kv_bf16 = kvbf16;
        st = linear(ws.x, d, lw.wqkv, lw.bqkv, T, 3 * d, d, Epi::kQkv, qkv, "qkv projection", &ln1);
        if (st) return st;
        if (l == L - 1 && T > segs) {
            // Only each segment's last position feeds the head, and the cache now holds every
            // key and value of the segment: the rest of the last layer runs as a decode step
            // over the segments' last queries and residual rows (attention over the row's
            // cached keys [0, len) is the causal attention of its last position).
            err = bst::launch_gather_last(stream, ws.q, ws.seg_start, ws.seg_len, segs, d,
                                          ws.last_h);
            if (!err) {
                err = bst::launch_gather_last(stream, ws.x, ws.seg_start, ws.seg_len, segs, d,
                                              ws.last);
            }
            if (err) return cuda_fail(err, "gather last");
            const Workspace saved = ws;
            ws.x = ws.last;
            ws.q = ws.last_h;
            DecodePlan dp;
            bool normalised = false;
            st = decode_plan(segs, std::vector<int>(p.prefill_len.begin() + begin,
                                                    p.prefill_len.begin() + end), &dp);
            if (!st) {
                st = decode_after_qkv(l, segs, ws.seg_row, dp, bst::QkvParts{}, &normalised,
                                      bst::kAttnPrefill);
            }
            ws = saved;
            if (st) return st;
            EpiArgs lg;
            lg.out = ws.logits;
            lg.ldo = V;
            lg.rowmap = ws.seg_row;
            lg.best = head_argmax ? ws.best : nullptr;
            if (normalised) {
                return linear(ws.last, d, head_w, head_b, segs, V, d, Epi::kLogits, lg, "head",
                              nullptr, false, true);
            }
            const bst::LnArgs lnf{lnf_g, lnf_b, kLayerNormEps};
            return linear(ws.last, d, head_w, head_b, segs, V, d, Epi::kLogits, lg, "head", &lnf);
        }
        const bst::PlaneOut att_planes = planes_for(lw.wo, T, d, d);
        st = check(launch(bst::kAttnPrefill, attn_bytes, attn_flops, 1, [&] {
                       return bst::launch_attn_prefill(stream, ws.q, qkv.k_cache, qkv.v_cache,
                                                       kvbf16, ws.seg_row, ws.seg_start,
                                                       ws.seg_len, segs, max_len, H, hd, slots,
                                                       scale, att_planes.planes ? nullptr : ws.att,
                                                       att_planes);
                   }), "prefill attention");
        if (st) return st;
        EpiArgs res;
        res.out = ws.x;
        res.ldo = d;
        st = linear(ws.att, d, lw.wo, lw.bo, T, d, d, Epi::kResidual, res, "output projection",
                    nullptr, att_planes.planes != 0);
        if (st) return st;
        const bst::LnArgs ln2{lw.ln2_g, lw.ln2_b, kLayerNormEps};
        EpiArgs act;
        act.ldo = F;
        act.split = planes_for(lw.w2, T, d, F);
        act.out = act.split.planes ? nullptr : ws.ffn;  // FFN2 reads only the planes
        st = linear(ws.x, d, lw.w1, lw.b1, T, F, d, Epi::kGelu, act, "ffn1", &ln2);
        if (st) return st;
        st = linear(ws.ffn, F, lw.w2, lw.b2, T, d, F, Epi::kResidual, res, "ffn2", nullptr,
                    act.split.planes != 0);
        if (st) return st;
    }
    st = check(launch(bst::kGather, segs * d * 8.0, 0, 1, [&] {
                   return bst::launch_gather_last(stream, ws.x, ws.seg_start, ws.seg_len, segs, d,
                                                  ws.last);
               }), "gather last");
    if (st) return st;
    const bst::LnArgs lnf{lnf_g, lnf_b, kLayerNormEps};
    EpiArgs lg;
    lg.out = ws.logits;
    lg.ldo = V;
    lg.rowmap = ws.seg_row;
    lg.best = head_argmax ? ws.best : nullptr;
    return linear(ws.last, d, head_w, head_b, segs, V, d, Epi::kLogits, lg, "head", &lnf);
}

int Engine::embed_rows(int R, const int* rowmap, bool normalise) {
    const double wb = wbf16 ? 2.0 : 4.0;
    cudaError_t err;
    if (normalise) {
        const double plane = static_cast<double>(bst::tc_split_bytes(R, d, wbf16));
        err = launch(bst::kEmbed, R * d * (2 * wb + 4.0) + 2 * plane, 0, 1, [&] {
            return bst::launch_embed_ln_decode(stream, tok_emb, pos_emb, wbf16, rowmap, ws.next,
                                               ws.len, ws.slot, ws.x, R, d, layers[0].ln1_g,
                                               layers[0].ln1_b, kLayerNormEps, ws.xs_hi, ws.xs_lo,
                                               wbf16 ? 2 : 1);
        });
    } else {
        err = launch(bst::kEmbed, R * d * (2 * wb + 4.0), 0, 1, [&] {
            return bst::launch_embed_decode(stream, tok_emb, pos_emb, wbf16, rowmap, ws.next,
                                            ws.len, ws.slot, ws.x, R, d);
        });
    }
    return err ? cuda_fail(err, "embedding") : BST_OK;
}

int Engine::enqueue_decode(int R, const int* rowmap, const std::vector<int>& lens) {
    int st = BST_OK;
    // Lanes: BST_DECODE_LANES (1 to 4) in the environment, 2 by default; each lane needs more
    // than 8 rows (the tensor-core path).
    int nl = 2;
    if (const char* env = std::getenv("BST_DECODE_LANES")) nl = std::atoi(env);
    nl = std::max(1, std::min(nl, kLanes));
    while (nl > 1 && (R / nl <= 8 || !ws.lane_part[nl - 1] ||
                      !linear_on_tc(layers[0].wqkv, R / nl, 3 * d, d))) {
        nl /= 2;
    }
    {
        int lanes[kLanes];
        for (int i = 0; i < nl; ++i) lanes[i] = (i + 1) * R / nl - i * R / nl;
        push_in_head = head_pushes(lanes, nl);
        push_rows = R;
    }
    if (nl == 1) {
        // On the tensor-core path the embedding kernel also writes the first LayerNorm's
        // operand planes; the GEMV path normalises inside its own projection.
        const bool normalise = linear_on_tc(layers[0].wqkv, R, 3 * d, d) && d <= 1024;
        st = embed_rows(R, rowmap, normalise);
        return st ? st : decode_layers(R, rowmap, lens, normalise);
    }
    // Lane i takes rows [i R / nl, (i + 1) R / nl) with every per-row workspace view shifted to
    // them; lanes > 0 run on their own streams with private planes and partials. The lanes are
    // enqueued layer by layer and start together (chaining their attention kernels so that one
    // lane streams the cache while the other runs its projections measured slower).
    cudaError_t err = cudaEventRecord(lane_fork, stream);
    for (int i = 1; i < nl && !err; ++i) err = cudaStreamWaitEvent(lane_stream[i], lane_fork, 0);
    if (err) return cuda_fail(err, "forking the decode lanes");
    const Workspace saved = ws;
    const cudaStream_t main = stream;
    Workspace lane_ws[kLanes];
    DecodePlan plan[kLanes];
    bool normalised[kLanes] = {};
    int first[kLanes + 1];
    for (int i = 0; i <= nl; ++i) first[i] = i * R / nl;
    for (int i = 0; i < nl && !st; ++i) {
        const int r0 = first[i];
        lane_ws[i] = saved;
        Workspace& w = lane_ws[i];
        if (i > 0) {
            w.x += static_cast<size_t>(r0) * d;
            w.q += static_cast<size_t>(r0) * d;
            w.att += static_cast<size_t>(r0) * d;
            w.ffn += static_cast<size_t>(r0) * F;
            w.slot += r0;
            w.attn_tickets += static_cast<size_t>(r0) * H;
            w.part += static_cast<size_t>(r0) * H * saved.splits * (hd + 2);
            w.xs_hi = saved.lane_xs_hi[i];
            w.xs_lo = saved.lane_xs_lo[i];
            w.ys_hi = saved.lane_ys_hi[i];
            w.ys_lo = saved.lane_ys_lo[i];
            w.tc_part = saved.lane_part[i];
        }
        st = decode_plan(first[i + 1] - r0,
                         std::vector<int>(lens.begin() + r0, lens.begin() + first[i + 1]), &plan[i]);
    }
    // Each lane embeds its own rows and writes the first LayerNorm's operand planes.
    const bool normalise = d <= 1024;
    for (int i = 0; i < nl && !st; ++i) {
        ws = lane_ws[i];
        stream = i ? lane_stream[i] : main;
        st = embed_rows(first[i + 1] - first[i], rowmap + first[i], normalise);
        normalised[i] = normalise;
    }
    {
        StepScope scope(in_step);
        for (int l = 0; l < L && !st; ++l) {
            for (int i = 0; i < nl && !st; ++i) {
                ws = lane_ws[i];
                stream = i ? lane_stream[i] : main;
                st = decode_layer(l, first[i + 1] - first[i], rowmap + first[i], plan[i],
                                  &normalised[i]);
            }
        }
        for (int i = 0; i < nl && !st; ++i) {
            ws = lane_ws[i];
            stream = i ? lane_stream[i] : main;
            st = decode_head(first[i + 1] - first[i], rowmap + first[i], normalised[i]);
        }
    }
    ws = saved;
    stream = main;
    if (st) return st;
    for (int i = 1; i < nl && !err; ++i) {
        err = cudaEventRecord(lane_join[i], lane_stream[i]);
        if (!err) err = cudaStreamWaitEvent(stream, lane_join[i], 0);
    }
    return err ? cuda_fail(err, "joining the decode lanes") : BST_OK;
}

// The decode QKV projection as split-K partial sums only (no fix-up kernel): LayerNorm of ws.x
// into the operand planes unless they already hold it (ln == nullptr), then the GEMM with
// the fix-up deferred to the attention kernel.
int Engine::qkv_partials(const LayerWeights& lw, const bst::LnArgs* ln, int R, int splits) {
    const int N = 3 * d, K = d;
    const double plane = static_cast<double>(bst::tc_split_bytes(R, K, wbf16));
    cudaError_t err = cudaSuccess;
    if (ln) {
        err = launch(bst::kLayerNorm, R * K * 4.0 + 2 * plane, 0, 1, [&] {
            return bst::launch_layernorm(stream, ws.x, d, ln->gamma, ln->beta, nullptr, 0, R, K,
                                         ln->eps, ws.xs_hi, ws.xs_lo, wbf16 ? 2 : 1);
        });
        if (err) return cuda_fail(err, "qkv projection");
    }
    const double wbytes = static_cast<double>(N) * K * (wbf16 ? 2.0 : 8.0);
    err = launch(bst::kGemm, wbytes + 2 * plane + static_cast<double>(splits) * R * N * 4.0,
                 2.0 * R * N * K, 1, [&] {
                     return bst::launch_gemm_tc(stream, ws.xs_hi, ws.xs_lo,
                                                wbf16 ? lw.wqkv.w : lw.wqkv.hi, lw.wqkv.lo, wbf16,
                                                lw.bqkv, R, N, K, Epi::kQkv, EpiArgs{}, ws.err,
                                                ws.tc_part, bst::tc_part_bytes_max(), true);
                 });
    return err ? cuda_fail(err, "qkv projection") : BST_OK;
}

int Engine::decode_plan(int R, const std::vector<int>& lens, DecodePlan* dp) {
    // Splits over the cache: enough CTAs for two waves of the SMs, chunks of >= 32 keys. Sized
    // by the run's slot capacity, not this step's lengths, so a captured step graph stays valid
    // as the cache grows; splits past a row's length return at once.
    const int max_len = std::max(1, ws.slots);
    dp->sum_len = 0;
    for (int n : lens) dp->sum_len += n;
    int splits = std::max(1, (592 + R * H - 1) / (R * H));
    int chunk = (max_len + splits - 1) / splits;
    chunk = std::max(32, (chunk + 31) / 32 * 32);
    chunk = std::min(chunk, 1024);
    splits = (max_len + chunk - 1) / chunk;
    if (splits > ws.splits) return fail(BST_PANIC, "decode split count exceeds the workspace");
    dp->splits = splits;
    dp->chunk = chunk;
    return BST_OK;
}

int Engine::decode_layers(int R, const int* rowmap, const std::vector<int>& lens,
                          bool x_normalised) {
    // GEMMs enqueued below are profiled as the decode step's (kGemmStep).
    StepScope scope(in_step);
    DecodePlan dp;
    int st = decode_plan(R, lens, &dp);
    // x_normalised: ws.xs_* holds this layer's LN1 (or the final LN) of ws.x
    for (int l = 0; l < L && !st; ++l) st = decode_layer(l, R, rowmap, dp, &x_normalised);
    return st ? st : decode_head(R, rowmap, x_normalised);
}

int Engine::decode_layer(int l, int R, const int* rowmap, const DecodePlan& dp,
                         bool* x_normalised) {
    const double kvb = kvbf16 ? 2.0 : 4.0;
    const int slots = ws.slots;
    int st = BST_OK;
    const LayerWeights& lw = layers[l];
    const bst::LnArgs ln1{lw.ln1_g, lw.ln1_b, kLayerNormEps};
    EpiArgs qkv;
    qkv.out = ws.q;
    qkv.ldo = d;
    qkv.rowmap = rowmap;
    qkv.slot = ws.slot;
    qkv.k_cache = static_cast<char*>(ws.k_cache) + l * ws.kv_layer_elems * static_cast<size_t>(kvb);
    qkv.v_cache = static_cast<char*>(ws.v_cache) + l * ws.kv_layer_elems * static_cast<size_t>(kvb);
    qkv.d = d;
    qkv.heads = H;
    qkv.head_dim = hd;
    qkv.slots = slots;
    qkv.kv_bf16 = kvbf16;
    // A split-K QKV projection leaves its partial sums to the attention kernel, which sums
    // q per head and appends the step's key and value to the cache itself.
    bst::QkvParts qparts;
    if (linear_on_tc(lw.wqkv, R, 3 * d, d)) {
        const int qkv_splits = bst::tc_plan(R, 3 * d, d, wbf16, bst::tc_part_bytes_max(), nullptr);
        if (qkv_splits > 1) qparts = bst::QkvParts{ws.tc_part, qkv_splits, lw.bqkv};
    }
    if (qparts.part) {
        st = qkv_partials(lw, *x_normalised ? nullptr : &ln1, R, qparts.splits);
    } else {
        st = *x_normalised ? linear(ws.x, d, lw.wqkv, lw.bqkv, R, 3 * d, d, Epi::kQkv, qkv,
                                    "qkv projection", nullptr, false, true)
                           : linear(ws.x, d, lw.wqkv, lw.bqkv, R, 3 * d, d, Epi::kQkv, qkv,
                                    "qkv projection", &ln1);
    }
    if (st) return st;
    return decode_after_qkv(l, R, rowmap, dp, qparts, x_normalised);
}

int Engine::decode_after_qkv(int l, int R, const int* rowmap, const DecodePlan& dp,
                             const bst::QkvParts& qparts, bool* x_normalised, int attn_class) {
    const double kvb = kvbf16 ? 2.0 : 4.0;
    const int slots = ws.slots;
    const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(hd)));
    auto check = [&](cudaError_t e, const char* what) { return e ? cuda_fail(e, what) : BST_OK; };
    int st = BST_OK;
    const LayerWeights& lw = layers[l];
    void* const k_cache =
        static_cast<char*>(ws.k_cache) + l * ws.kv_layer_elems * static_cast<size_t>(kvb);
    void* const v_cache =
        static_cast<char*>(ws.v_cache) + l * ws.kv_layer_elems * static_cast<size_t>(kvb);
    const double kv_bytes = dp.sum_len * 2.0 * d * kvb + R * d * 4.0 +
                            (qparts.part ? qparts.splits * R * 3.0 * d * 4.0 : 0.0);
    const bst::PlaneOut att_planes = planes_for(lw.wo, R, d, d);
    st = check(launch(attn_class, kv_bytes, 4.0 * dp.sum_len * d, 1, [&] {
                   return bst::launch_attn_decode(stream, ws.q, k_cache, v_cache,
                                                  kvbf16, rowmap, ws.len, R, H, hd, slots,
                                                  scale, dp.splits, dp.chunk, ws.part,
                                                  ws.attn_tickets,
                                                  att_planes.planes ? nullptr : ws.att,
                                                  att_planes, qparts);
               }), "decode attention");
    if (st) return st;
    const bst::LnArgs ln2{lw.ln2_g, lw.ln2_b, kLayerNormEps};
    bool ffn_in_normalised = false;
    st = residual_ln(ws.att, d, lw.wo, lw.bo, R, d, d, att_planes.planes != 0, ln2,
                     "output projection", &ffn_in_normalised);
    if (st) return st;
    EpiArgs act;
    act.ldo = F;
    act.split = planes_for(lw.w2, R, d, F);
    act.out = act.split.planes ? nullptr : ws.ffn;  // FFN2 reads only the planes
    st = ffn_in_normalised ? linear(ws.x, d, lw.w1, lw.b1, R, F, d, Epi::kGelu, act, "ffn1",
                                    nullptr, false, true)
                           : linear(ws.x, d, lw.w1, lw.b1, R, F, d, Epi::kGelu, act, "ffn1",
                                    &ln2);
    if (st) return st;
    const bst::LnArgs next = l + 1 < L ? bst::LnArgs{layers[l + 1].ln1_g, layers[l + 1].ln1_b,
                                                     kLayerNormEps}
                                       : bst::LnArgs{lnf_g, lnf_b, kLayerNormEps};
    return residual_ln(ws.ffn, F, lw.w2, lw.b2, R, d, F, act.split.planes != 0, next, "ffn2",
                       x_normalised);
}

int Engine::decode_head(int R, const int* rowmap, bool x_normalised) {
    const bst::LnArgs lnf{lnf_g, lnf_b, kLayerNormEps};
    EpiArgs lg;
    lg.out = ws.logits;
    lg.ldo = V;
    lg.rowmap = rowmap;
    lg.best = head_argmax ? ws.best : nullptr;
    if (push_in_head) {
        lg.step = ws.step;
        lg.done = ws.done;
        lg.tokens = ws.tokens_out;
        lg.next = ws.next;
        lg.window = ws.window;
        lg.window_len = W;
        lg.steps = push_steps;
        lg.rows = push_rows;
    }
    return x_normalised ? linear(ws.x, d, head_w, head_b, R, V, d, Epi::kLogits, lg, "head",
                                 nullptr, false, true)
                        : linear(ws.x, d, head_w, head_b, R, V, d, Epi::kLogits, lg, "head", &lnf);
}

// Families without a cache: the whole window is the input every step.
int Engine::enqueue_direct(int rows) {
    auto check = [&](cudaError_t e, const char* what) { return e ? cuda_fail(e, what) : BST_OK; };
    if (spec.family == BST_FAMILY_LAST_TOKEN) {
        return check(launch(bst::kHeadLastToken, rows * V * 8.0, 0, 1, [&] {
                         return bst::launch_last_token(stream, ws.window, W, lt_w, lt_b, rows, V,
                                                       ws.logits);
                     }), "last-token head");
    }
    // Zoo.WindowedLanguageModel.forward (zoo/Zoo.java:155-168).
    const double wb = wbf16 ? 2.0 : 4.0;
    const int flat = W * d;
    int st = check(launch(bst::kEmbed, rows * flat * (wb + 4.0), 0, 1, [&] {
                       return bst::launch_window_embed(stream, ws.window, W, tok_emb, wbf16, rows,
                                                       d, ws.flat);
                   }), "window embedding");
    if (st) return st;
    EpiArgs g;
    g.out = ws.ffn;
    g.ldo = F;
    st = linear(ws.flat, flat, cl_expand, cl_expand_b, rows, F, flat, Epi::kGelu, g, "expand");
    if (st) return st;
    EpiArgs rg;
    rg.out = ws.mixed;
    rg.ldo = flat;
    rg.res = ws.flat;
    rg.ldr = flat;
    st = linear(ws.ffn, F, cl_contract, cl_contract_b, rows, flat, F, Epi::kResidualGelu, rg, "contract");
    if (st) return st;
    EpiArgs lg;
    lg.out = ws.logits;
    lg.ldo = V;
    lg.rowmap = ws.rowmap_all;
    return linear(ws.mixed, flat, head_w, head_b, rows, V, flat, Epi::kLogits, lg, "head");
}

// Whether greedy decode steps of `rows` rows run as one persistent kernel (decode_fused.cu), and
// the per-layer table it reads. Returns the grid size, or 0 for the kernel-per-operation path.
// BST_FUSED_DECODE=0 in the environment turns the fused step off.
int Engine::prepare_fused(int rows) {
    const char* env = std::getenv("BST_FUSED_DECODE");
    if (env && std::strcmp(env, "0") == 0) return 0;
    if (!decoder_family(spec.family) || !bst::fused_decode_supported(rows, d, F, W, hd, wbf16)) {
        return 0;
    }
    if (fused_rows != rows) {
        fused_ctas = bst::fused_decode_prepare(rows, d, F, V, L, hd, wbf16, kvbf16);
        fused_rows = rows;
    }
    if (fused_ctas <= 0) return 0;
    const size_t kvb = kvbf16 ? 2 : 4;
    fused_table.assign(L, bst::FusedLayer{});
    for (int l = 0; l < L; ++l) {
        const LayerWeights& lw = layers[l];
        bst::FusedLayer& f = fused_table[l];
        f.wqkv = lw.wqkv.w;
        f.bqkv = lw.bqkv;
        f.wo = lw.wo.w;
        f.bo = lw.bo;
        f.ln1_g = lw.ln1_g;
        f.ln1_b = lw.ln1_b;
        f.ln2_g = lw.ln2_g;
        f.ln2_b = lw.ln2_b;
        f.w1 = lw.w1.w;
        f.b1 = lw.b1;
        f.w2 = lw.w2.w;
        f.b2 = lw.b2;
        f.k_cache = static_cast<char*>(ws.k_cache) + l * ws.kv_layer_elems * kvb;
        f.v_cache = static_cast<char*>(ws.v_cache) + l * ws.kv_layer_elems * kvb;
    }
    cudaError_t err = cudaMemcpyAsync(ws.fused_layers, fused_table.data(),
                                      sizeof(bst::FusedLayer) * L, cudaMemcpyHostToDevice, stream);
    if (!err) err = cudaMemsetAsync(ws.bar, 0, 2 * sizeof(unsigned), stream);
    if (!err) err = cudaMemsetAsync(ws.best, 0, 8 * sizeof(unsigned long long), stream);
    fused_bar_base = 0;
    if (err) {
        cuda_fail(err, "preparing the fused decode step");
        return -1;
    }
    return fused_ctas;
}

int Engine::enqueue_fused(int rows, int steps, const std::vector<int>& lens, bool history) {
    const double wb = wbf16 ? 2.0 : 4.0, kvb = kvbf16 ? 2.0 : 4.0;
    bst::FusedStep p;
    p.R = rows;
    p.d = d;
    p.H = H;
    p.F = F;
    p.V = V;
    p.W = W;
    p.L = L;
    p.slots = ws.slots;
    p.steps = steps;
    p.nchunks = (ws.slots + 31) / 32;
    p.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(hd)));
    p.eps = kLayerNormEps;
    p.len = ws.len;
    p.next = ws.next;
    p.tokens = ws.tokens_out;
    p.window = ws.window;
    p.step = ws.step;
    p.done = ws.done;
    p.rowmap = ws.rowmap_all;
    p.tok_emb = tok_emb;
    p.pos_emb = pos_emb;
    p.lnf_g = lnf_g;
    p.lnf_b = lnf_b;
    p.head_w = head_w.w;
    p.head_b = head_b;
    p.x = ws.x;
    p.q = ws.q;
    p.att = ws.att;
    p.ffn = ws.ffn;
    p.logits = ws.logits;
    p.part = ws.part;
    p.tickets = ws.attn_tickets;
    p.bar = ws.bar;
    p.bar_base = fused_bar_base;
    p.best = ws.best;
    p.err = ws.err;
    p.stats = ws.fused_stats;
    p.history = history ? ws.history : nullptr;
    if (p.nchunks > ws.splits) return fail(BST_PANIC, "decode chunk count exceeds the workspace");
    // Algorithmic bytes: every weight once, the cache rows attended, activations are negligible.
    double sum_len = 0;
    for (int n : lens) sum_len += n;
    const double params = static_cast<double>(L) * (4.0 * d * d + 2.0 * d * F) + double(V) * d;
    const double bytes = params * wb + sum_len * 2.0 * d * kvb * L + rows * V * 4.0;
    const double flops = 2.0 * params * rows + 4.0 * sum_len * d * L;
    const cudaError_t err = launch(bst::kDecodeStep, bytes, flops, 1, [&] {
        return bst::launch_decode_fused(stream, p, ws.fused_layers, wbf16, kvbf16, hd, fused_ctas);
    });
    if (err) return cuda_fail(err, "fused decode step");
    fused_bar_base += static_cast<unsigned>(fused_ctas) * bst::fused_decode_barriers(L);
    return BST_OK;
}

int Engine::enqueue_select(Mode mode, int rows, int steps, float temperature, int top_k,
                           bool history) {
    cudaError_t err;
    if (history) {
        err = launch(bst::kMisc, rows * V * 8.0, 0, 1, [&] {
            return bst::launch_stash_logits(stream, ws.logits, hist_count, V, steps, ws.step,
                                            ws.hist_rows_of, ws.history);
        });
        if (err) return cuda_fail(err, "stashing logits");
    }
    if (mode == Mode::kGreedy && push_in_head) {
        push_in_head = false;  // the head's fix-up pushed the tokens
        return BST_OK;
    }
    push_in_head = false;
    if (mode == Mode::kGreedy) {
        err = launch(bst::kSelectGreedy, rows * V * 4.0, 0, 1, [&] {
            return bst::launch_select_greedy(stream, ws.logits, rows, V, W, steps, ws.step, ws.done,
                                             ws.tokens_out, ws.next, ws.window,
                                             head_argmax ? ws.best : nullptr);
        });
    } else {
        err = launch(bst::kSelectSample, rows * V * 4.0, 0, 1, [&] {
            const bool split = ws.sorted_w && ws.sorted_capacity >= static_cast<size_t>(rows) * V;
            return bst::launch_select_sample(stream, ws.logits, rows, V, W, steps, temperature,
                                             top_k, ws.rng, ws.step, ws.done, ws.tokens_out,
                                             ws.next, ws.window, split ? ws.sorted_w : nullptr,
                                             split ? ws.sorted_ids : nullptr);
        });
    }
    return err ? cuda_fail(err, "token selection") : BST_OK;
}

int Engine::run_wave(Mode mode, const std::vector<int32_t>& all_windows, int row0, int rows,
                     int steps, float temperature, int top_k, uint64_t rng_base, int32_t* tokens,
                     bool tokens_on_device, int total_rows, bst_token_sink sink, void* user,
                     double* scores, float* logits) {
    const int run_steps = mode == Mode::kScores ? 1 : steps;
    // Rows of this wave whose per-step logits are kept (hist_local) and the output slot of each
    // (-1: kept only because the fused step writes every row's logits).
    std::vector<int> hist_local, hist_out;
    if (logits != nullptr && mode != Mode::kScores) {
        for (int r = 0; r < rows; ++r) {
            if (watch.empty()) {
                hist_local.push_back(r);
                hist_out.push_back(row0 + r);
                continue;
            }
            for (size_t i = 0; i < watch.size(); ++i) {
                if (watch[i] == row0 + r) {
                    hist_local.push_back(r);
                    hist_out.push_back(static_cast<int>(i));
                    break;
                }
            }
        }
        if (!hist_local.empty() && mode == Mode::kGreedy && rows <= 8 &&
            static_cast<int>(hist_local.size()) != rows) {
            std::vector<int> out(rows, -1);
            for (size_t i = 0; i < hist_local.size(); ++i) out[hist_local[i]] = hist_out[i];
            hist_local.resize(rows);
            for (int r = 0; r < rows; ++r) hist_local[r] = r;
            hist_out = out;
        }
    }
    const bool history = !hist_local.empty();
    const int hist_rows = static_cast<int>(hist_local.size());
    std::vector<int32_t> windows(all_windows.begin() + static_cast<size_t>(row0) * W,
                                 all_windows.begin() + static_cast<size_t>(row0 + rows) * W);
    std::vector<StepPlan> plans;
    int max_slots = 1, max_tokens = rows;
    const bool transformer = decoder_family(spec.family);
    if (transformer) plan(windows, rows, run_steps, &plans, &max_slots, &max_tokens);
    const int splits_cap = std::max(1, (max_slots + 31) / 32);
    int st = ensure_workspace(rows, run_steps, max_slots, max_tokens, splits_cap, hist_rows,
                              mode == Mode::kSample);
    if (st) return st;
    hist_count = hist_rows;
    push_steps = run_steps;
    push_in_head = false;

    cudaError_t err = cudaMemcpyAsync(ws.window, windows.data(), sizeof(int32_t) * windows.size(),
                                      cudaMemcpyHostToDevice, stream);
    if (!err && history) {
        err = cudaMemcpyAsync(ws.hist_rows_of, hist_local.data(), sizeof(int) * hist_rows,
                              cudaMemcpyHostToDevice, stream);
    }
    if (!err) err = cudaMemsetAsync(ws.step, 0, sizeof(int), stream);
    if (!err) err = cudaMemsetAsync(ws.done, 0, sizeof(int), stream);
    if (!err) err = cudaMemsetAsync(ws.err, 0, sizeof(int), stream);
    if (!err) err = cudaMemsetAsync(ws.len, 0, sizeof(int) * rows, stream);
    // Host-side fault injection for tests of the failure path: the status word starts out set,
    // as a kernel that gave up on a bounded wait leaves it. No kernel is made to fail.
    int injected = 0;
    if (const char* inject = std::getenv("BST_INJECT_PIPELINE_ERROR")) injected = std::atoi(inject);
    if (!err && injected) {
        err = cudaMemcpyAsync(ws.err, &injected, sizeof(int), cudaMemcpyHostToDevice, stream);
    }
    int fused = 0;
    if (!err && transformer && mode == Mode::kGreedy) {
        fused = prepare_fused(rows);
        if (fused < 0) return BST_PANIC;
    }
    head_argmax = transformer && mode == Mode::kGreedy;
    if (!err && head_argmax) {
        err = cudaMemsetAsync(ws.best, 0, sizeof(unsigned long long) * std::max(8, rows), stream);
    }
    if (!err && mode == Mode::kSample) {
        std::vector<uint64_t> states(rows);
        for (int r = 0; r < rows; ++r) {
            states[r] = jrand::advance(rng_base, 2ull * static_cast<uint64_t>(steps) * (row0 + r));
        }
        err = cudaMemcpyAsync(ws.rng, states.data(), sizeof(uint64_t) * rows,
                              cudaMemcpyHostToDevice, stream);
        if (!err) err = cudaStreamSynchronize(stream);
    }
    if (!err) err = cudaStreamSynchronize(stream);
    if (err) return cuda_fail(err, "uploading contexts");

    std::vector<int32_t> step_tokens(rows);
    for (int g = 0; g < run_steps; ++g) {
        const bool all_decode = transformer && plans[g].prefill_rows.empty();
        push_allowed = all_decode && static_cast<int>(plans[g].decode_rows.size()) == rows;
        const bool graphable = !profiling && mode != Mode::kScores &&
                               (transformer ? all_decode : true);
        if (transformer && !plans[g].prefill_rows.empty()) {
            const StepPlan& p = plans[g];
            size_t begin = 0;
            while (begin < p.prefill_rows.size()) {
                size_t end = begin;
                int64_t sum = 0;
                while (end < p.prefill_rows.size() &&
                       (end == begin || sum + p.prefill_len[end] <= ws.tokens)) {
                    sum += p.prefill_len[end];
                    ++end;
                }
                st = enqueue_prefill(p, begin, end);
                if (st) return st;
                begin = end;
            }
        }
        if (fused > 0 && all_decode) {
            // Small batches: the whole step (selection included) is one persistent kernel.
            st = enqueue_fused(rows, run_steps, plans[g].decode_len, history);
            if (st) return st;
        } else if (graphable) {
            // One CUDA graph per (shape, mode): the step body plus selection reads every
            // step-dependent value (lengths, step counter, RNG state) from device memory.
            char key[160];
            std::snprintf(key, sizeof(key), "%d/%d/%d/%d/%08x/%d/%d/%llu", static_cast<int>(mode),
                          rows, run_steps, ws.slots,
                          [&] { uint32_t b; std::memcpy(&b, &temperature, 4); return b; }(),
                          top_k, hist_rows, static_cast<unsigned long long>(ws.generation));
            if (!graph || graph_key != key) {
                if (graph) {
                    cudaGraphExecDestroy(graph);
                    graph = nullptr;
                }
                cudaGraph_t g_raw = nullptr;
                err = cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal);
                if (err) return cuda_fail(err, "beginning graph capture");
                const int64_t before = launches;
                st = transformer ? enqueue_decode(rows, ws.rowmap_all, plans[g].decode_len)
                                 : enqueue_direct(rows);
                if (!st) st = enqueue_select(mode, rows, run_steps, temperature, top_k, history);
                const cudaError_t end_err = cudaStreamEndCapture(stream, &g_raw);
                if (st) {
                    if (g_raw) cudaGraphDestroy(g_raw);
                    return st;
                }
                if (end_err) return cuda_fail(end_err, "ending graph capture");
                graph_nodes = launches - before;
                launches = before;
                err = cudaGraphInstantiate(&graph, g_raw, 0);
                cudaGraphDestroy(g_raw);
                if (err) {
                    graph = nullptr;
                    return cuda_fail(err, "instantiating the decode graph");
                }
                graph_key = key;
            }
            err = cudaGraphLaunch(graph, stream);
            if (err) return cuda_fail(err, "launching the decode graph");
            launches += graph_nodes;
        } else {
            if (transformer) {
                const StepPlan& p = plans[g];
                if (!p.decode_rows.empty()) {
                    const int R = static_cast<int>(p.decode_rows.size());
                    const int* rowmap = ws.rowmap_all;
                    if (R != rows) {
                        err = cudaMemcpyAsync(ws.rowmap_dec, p.decode_rows.data(), sizeof(int) * R,
                                              cudaMemcpyHostToDevice, stream);
                        if (!err) err = cudaStreamSynchronize(stream);
                        if (err) return cuda_fail(err, "uploading decode rows");
                        rowmap = ws.rowmap_dec;
                    }
                    st = enqueue_decode(R, rowmap, p.decode_len);
                    if (st) return st;
                }
            } else {
                st = enqueue_direct(rows);
                if (st) return st;
            }
            if (mode != Mode::kScores) {
                st = enqueue_select(mode, rows, run_steps, temperature, top_k, history);
                if (st) return st;
            }
        }
        if (sink && mode != Mode::kScores) {
            // The step's tokens and the pipeline status together: a step whose kernels gave up
            // on a wait produced no tokens, and the sink must not see them.
            int step_error = 0;
            err = cudaMemcpy2DAsync(step_tokens.data(), sizeof(int32_t), ws.tokens_out + g,
                                    sizeof(int32_t) * run_steps, sizeof(int32_t), rows,
                                    cudaMemcpyDeviceToHost, stream);
            if (!err) {
                err = cudaMemcpyAsync(&step_error, ws.err, sizeof(int), cudaMemcpyDeviceToHost,
                                      stream);
            }
            if (!err) err = cudaStreamSynchronize(stream);
            if (err) return cuda_fail(err, "reading tokens");
            if (step_error) return fail(BST_PANIC, pipeline_message(step_error));
            for (int r = 0; r < rows; ++r) {
                if (sink(user, row0 + r, g, step_tokens[r]) != 0) {
                    return fail(BST_INVALID, "the token sink stopped the call at row " +
                                                 std::to_string(row0 + r) + ", step " +
                                                 std::to_string(g));
                }
            }
        }
    }
    (void)total_rows;
    int pipeline_error = 0;
    err = cudaMemcpyAsync(&pipeline_error, ws.err, sizeof(int), cudaMemcpyDeviceToHost, stream);
    if (!err) err = cudaStreamSynchronize(stream);
    if (err) return cuda_fail(err, "reading the pipeline status");
    if (pipeline_error) return fail(BST_PANIC, pipeline_message(pipeline_error));
    if (mode == Mode::kScores) {
        std::vector<float> logits(static_cast<size_t>(rows) * V);
        err = cudaMemcpyAsync(logits.data(), ws.logits, sizeof(float) * logits.size(),
                              cudaMemcpyDeviceToHost, stream);
        if (!err) err = cudaStreamSynchronize(stream);
        if (err) return cuda_fail(err, "reading logits");
        for (size_t i = 0; i < logits.size(); ++i) scores[static_cast<size_t>(row0) * V + i] = logits[i];
    } else {
        int32_t* dst = tokens + static_cast<size_t>(row0) * steps;
        err = cudaMemcpyAsync(dst, ws.tokens_out, sizeof(int32_t) * static_cast<size_t>(rows) * steps,
                              tokens_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost,
                              stream);
        if (!err && history && watch.empty()) {
            err = cudaMemcpyAsync(logits + static_cast<size_t>(row0) * steps * V, ws.history,
                                  sizeof(float) * static_cast<size_t>(rows) * steps * V,
                                  cudaMemcpyDeviceToHost, stream);
        }
        for (int h = 0; !err && history && !watch.empty() && h < hist_rows; ++h) {
            if (hist_out[h] < 0) continue;
            const size_t n = static_cast<size_t>(steps) * V;
            err = cudaMemcpyAsync(logits + static_cast<size_t>(hist_out[h]) * n,
                                  ws.history + static_cast<size_t>(h) * n, sizeof(float) * n,
                                  cudaMemcpyDeviceToHost, stream);
        }
        if (!err) err = cudaStreamSynchronize(stream);
        if (err) return cuda_fail(err, "reading tokens");
    }
    collect_timings();
    return BST_OK;
}

int Engine::run(Mode mode, const int32_t* contexts, int32_t rows, int32_t length, int32_t steps,
                float temperature, int32_t top_k, int32_t* tokens, bool tokens_on_device,
                bst_token_sink sink, void* user, double* scores, float* logits) {
    // Argument checks in TextEngine's order (TextEngine.java:121-126, 158-160, 201-212, 359-374).
    if (mode != Mode::kScores && steps < 1) {
        return fail(BST_INVALID, "steps must be at least 1, got " + std::to_string(steps));
    }
    if (mode == Mode::kSample) {
        if (!(temperature > 0.0f) || !std::isfinite(temperature)) {
            return fail(BST_INVALID, "temperature must be positive and finite, got " +
                                         std::to_string(temperature));
        }
        if (top_k < 1) return fail(BST_INVALID, "topK must be at least 1, got " + std::to_string(top_k));
        top_k = std::min(top_k, V);
        if (bst::select_sample_smem(V) > 200 * 1024) {
            return fail(BST_UNSUPPORTED, "sampling supports vocabularies up to 16384");
        }
    }
    if (!contexts) return fail(BST_INVALID, "contexts must not be null");
    if (rows < 1) return fail(BST_INVALID, "contexts must not be empty");
    if (length < W) {
        return fail(BST_INVALID, "context needs at least " + std::to_string(W) + " tokens, got " +
                                     std::to_string(length));
    }
    if (mode != Mode::kScores && !tokens) return fail(BST_INVALID, "tokens must not be null");
    if (mode == Mode::kScores && !scores) return fail(BST_INVALID, "scores must not be null");

    // Tails (TextEngine.tail, TextEngine.java:376-380) and the embedding id checks
    // (nn_ops.rs:1051-1056).
    std::vector<int32_t> windows(static_cast<size_t>(rows) * W);
    for (int r = 0; r < rows; ++r) {
        std::memcpy(windows.data() + static_cast<size_t>(r) * W,
                    contexts + static_cast<size_t>(r) * length + (length - W), sizeof(int32_t) * W);
    }
    if (spec.family != BST_FAMILY_LAST_TOKEN) {
        const int limit = spec.family == BST_FAMILY_PADDED_DECODER ? V + 1 : V;
        for (size_t i = 0; i < windows.size(); ++i) {
            if (windows[i] < 0 || windows[i] >= limit) {
                return fail(BST_INVALID, "embedding index " + std::to_string(windows[i]) +
                                             " is outside [0, " + std::to_string(limit) + ")");
            }
        }
    }
    cudaError_t err = cudaSetDevice(device);
    if (err) return cuda_fail(err, "cudaSetDevice");
    int st = upload_weights();
    if (st) return st;

    // Waves bound the workspace (KV cache + activations) by max_rows.
    const int wave = spec.max_rows > 0 ? std::min<int>(rows, spec.max_rows) : rows;
    const uint64_t rng_base = rng_state;
    for (int row0 = 0; row0 < rows; row0 += wave) {
        const int n = std::min(wave, rows - row0);
        st = run_wave(mode, windows, row0, n, steps, temperature, top_k, rng_base, tokens,
                      tokens_on_device, rows, sink, user, scores, logits);
        if (st) {
            if (profiling) pending.clear();
            return st;
        }
    }
    if (mode == Mode::kSample) {
        rng_state = jrand::advance(rng_base, 2ull * static_cast<uint64_t>(steps) * rows);
    }
    return BST_OK;
}

}  // namespace

void bst::set_thread_error(const std::string& message) { t_last_error = message; }

namespace {

int set_error(const std::shared_ptr<Engine>& e, int code) {
    if (code != BST_OK && e) t_last_error = e->error;
    return code;
}

int unknown(bst_engine h) {
    t_last_error = "engine handle " + std::to_string(h) + " is not live";
    return BST_UNKNOWN_HANDLE;
}

#define BST_GUARDED(...)                                                   \
    try {                                                                  \
        __VA_ARGS__                                                        \
    } catch (const std::bad_alloc&) {                                      \
        t_last_error = "host allocation failed";                           \
        return BST_OOM;                                                    \
    } catch (const std::exception& ex) {                                   \
        t_last_error = std::string("internal error: ") + ex.what();        \
        return BST_PANIC;                                                  \
    } catch (...) {                                                        \
        t_last_error = "internal error";                                   \
        return BST_PANIC;                                                  \
    }

}  // namespace

// =============================================================================================
// C ABI
// =============================================================================================
extern "C" {

int32_t bst_abi_version(void) { return BST_ABI_VERSION; }

int32_t bst_device_count(int32_t* count) {
    if (!count) return BST_INVALID;
    int n = 0;
    const cudaError_t err = cudaGetDeviceCount(&n);
    if (err != cudaSuccess) {
        cudaGetLastError();
        *count = 0;
        t_last_error = std::string("no CUDA device: ") + cudaGetErrorString(err);
        return BST_UNSUPPORTED;
    }
    *count = n;
    return BST_OK;
}

int32_t bst_engine_create(const bst_model_spec* spec, int32_t device, bst_engine* out) {
    BST_GUARDED({
        if (!spec || !out) {
            t_last_error = "spec and out must not be null";
            return BST_INVALID;
        }
        const Failure f = validate_spec(*spec);
        if (f.code) {
            t_last_error = f.message;
            return f.code;
        }
        int n = 0;
        cudaError_t err = cudaGetDeviceCount(&n);
        if (err != cudaSuccess || device < 0 || device >= n) {
            cudaGetLastError();
            t_last_error = "CUDA device " + std::to_string(device) + " is not available" +
                           (err != cudaSuccess ? std::string(": ") + cudaGetErrorString(err) : "");
            return BST_UNSUPPORTED;
        }
        auto e = std::make_shared<Engine>();
        e->spec = *spec;
        e->device = device;
        e->V = spec->vocabulary;
        e->W = spec->window;
        e->d = spec->dimension;
        e->L = spec->layers;
        e->H = spec->heads > 0 ? spec->heads : 1;
        e->hd = spec->dimension > 0 ? spec->dimension / e->H : 0;
        e->F = spec->hidden;
        e->wbf16 = spec->weight_dtype == BST_DTYPE_BF16;
        e->kvbf16 = spec->kv_dtype == BST_DTYPE_BF16;
        std::vector<int64_t> sizes;
        declare_parameters(*spec, &e->names, &sizes);
        for (size_t i = 0; i < e->names.size(); ++i) {
            e->index[e->names[i]] = i;
            e->values.emplace_back(static_cast<size_t>(sizes[i]),
                                   is_layernorm_gamma(e->names[i]) ? 1.0f : 0.0f);
        }
        if (spec->family == BST_FAMILY_LAST_TOKEN) {
            // TextEngineTest.LastTokenModel: weight 6 at (t, (t + 1) mod V), bias 0.
            auto& w = e->values[0];
            for (int t = 0; t < e->V; ++t) w[static_cast<size_t>(t) * e->V + (t + 1) % e->V] = 6.0f;
        }
        err = cudaSetDevice(device);
        if (!err) err = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
        for (int i = 1; i < kLanes && !err; ++i) {
            err = cudaStreamCreateWithFlags(&e->lane_stream[i], cudaStreamNonBlocking);
            if (!err) err = cudaEventCreateWithFlags(&e->lane_join[i], cudaEventDisableTiming);
        }
        if (!err) err = cudaEventCreateWithFlags(&e->lane_fork, cudaEventDisableTiming);
        if (!err) err = bst::configure_device_kernels_once(device);
        if (err) {
            cudaGetLastError();
            t_last_error = std::string("cannot initialise the device: ") + cudaGetErrorString(err);
            return BST_PANIC;
        }
        std::lock_guard<std::mutex> lock(g_registry_mutex);
        const uint64_t h = g_next_handle++;
        g_engines[h] = e;
        *out = h;
        return BST_OK;
    })
}

int32_t bst_recognize_model(const char* const* names, const int32_t* ranks, const int64_t* dims,
                            int32_t count, int32_t vocabulary, int32_t window, int32_t heads,
                            bst_model_spec* spec) {
    BST_GUARDED({
        if (!spec) {
            t_last_error = "spec must not be null";
            return BST_INVALID;
        }
        std::vector<ParamView> params;
        Failure f = parameter_views(names, ranks, dims, count, &params);
        if (!f.code) f = recognize(params, vocabulary, window, heads, spec);
        if (f.code) t_last_error = f.message;
        return f.code;
    })
}

int32_t bst_engine_create_from_parameters(const char* const* names, const int32_t* ranks,
                                          const int64_t* dims, const float* const* values,
                                          int32_t count, int32_t vocabulary, int32_t window,
                                          int32_t heads, int32_t weight_dtype, int32_t kv_dtype,
                                          int32_t device, bst_engine* out) {
    BST_GUARDED({
        if (!out || !values) {
            t_last_error = "values and out must not be null";
            return BST_INVALID;
        }
        bst_model_spec spec{};
        int32_t st = bst_recognize_model(names, ranks, dims, count, vocabulary, window, heads, &spec);
        if (st) return st;
        spec.weight_dtype = weight_dtype;
        spec.kv_dtype = kv_dtype;
        std::vector<ParamView> params;
        parameter_views(names, ranks, dims, count, &params);
        for (int32_t i = 0; i < count; ++i) {
            if (!values[i] && params[i].numel() > 0) {
                t_last_error = "values of parameter " + params[i].name + " are null";
                return BST_INVALID;
            }
        }
        bst_engine h = 0;
        st = bst_engine_create(&spec, device, &h);
        if (st) return st;
        for (int32_t i = 0; i < count; ++i) {
            st = bst_set_parameter(h, names[i], values[i], params[i].numel());
            if (st) {
                const std::string why = t_last_error;
                bst_engine_destroy(h);
                t_last_error = why;
                return st;
            }
        }
        *out = h;
        return BST_OK;
    })
}

int32_t bst_engine_destroy(bst_engine h) {
    std::shared_ptr<Engine> e;
    {
        std::lock_guard<std::mutex> lock(g_registry_mutex);
        auto it = g_engines.find(h);
        if (it == g_engines.end()) return unknown(h);
        e = it->second;
        g_engines.erase(it);
    }
    std::lock_guard<std::mutex> lock(e->mu);
    e->release_all();
    return BST_OK;
}

int32_t bst_parameter_count(bst_engine h, int32_t* count) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    if (!count) return BST_INVALID;
    *count = static_cast<int32_t>(e->names.size());
    return BST_OK;
}

int32_t bst_parameter_info(bst_engine h, int32_t index, char* name, int32_t capacity,
                           int64_t* size) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    if (index < 0 || index >= static_cast<int32_t>(e->names.size())) {
        t_last_error = "parameter index out of range";
        return BST_INVALID;
    }
    if (name && capacity > 0) {
        std::snprintf(name, static_cast<size_t>(capacity), "%s", e->names[index].c_str());
    }
    if (size) *size = static_cast<int64_t>(e->values[index].size());
    return BST_OK;
}

int32_t bst_set_parameter(bst_engine h, const char* name, const float* values, int64_t count) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    BST_GUARDED({
        std::lock_guard<std::mutex> lock(e->mu);
        if (!name || (!values && count > 0)) return set_error(e, e->fail(BST_INVALID, "name and values must not be null"));
        auto it = e->index.find(name);
        if (it == e->index.end()) return set_error(e, e->fail(BST_INVALID, std::string("unknown parameter ") + name));
        auto& dst = e->values[it->second];
        if (static_cast<int64_t>(dst.size()) != count) {
            return set_error(e, e->fail(BST_SHAPE, std::string("parameter ") + name + " expects " +
                                                       std::to_string(dst.size()) + " values, got " +
                                                       std::to_string(count)));
        }
        std::copy(values, values + count, dst.begin());
        e->dirty = true;
        return BST_OK;
    })
}

int32_t bst_get_parameter(bst_engine h, const char* name, float* values, int64_t count) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    std::lock_guard<std::mutex> lock(e->mu);
    if (!name || !values) return set_error(e, e->fail(BST_INVALID, "name and values must not be null"));
    auto it = e->index.find(name);
    if (it == e->index.end()) return set_error(e, e->fail(BST_INVALID, std::string("unknown parameter ") + name));
    const auto& src = e->values[it->second];
    if (static_cast<int64_t>(src.size()) != count) {
        return set_error(e, e->fail(BST_SHAPE, "parameter size mismatch"));
    }
    std::copy(src.begin(), src.end(), values);
    return BST_OK;
}

int32_t bst_save(bst_engine h, const char* path) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    BST_GUARDED({
        std::lock_guard<std::mutex> lock(e->mu);
        if (!path) return set_error(e, e->fail(BST_INVALID, "path must not be null"));
        const Failure f = write_weight_file(path, e->V, e->W, e->names, e->values);
        if (f.code) return set_error(e, e->fail(f.code, f.message));
        return BST_OK;
    })
}

int32_t bst_load(bst_engine h, const char* path) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    BST_GUARDED({
        std::lock_guard<std::mutex> lock(e->mu);
        if (!path) return set_error(e, e->fail(BST_INVALID, "path must not be null"));
        StoredModel stored;
        Failure f = read_weight_file(path, &stored);
        if (f.code) return set_error(e, e->fail(f.code, f.message));
        if (stored.vocabulary != e->V || stored.window != e->W) {
            return set_error(e, e->fail(BST_CONTEXT,
                                        "model was saved with vocabulary=" + std::to_string(stored.vocabulary) +
                                            " window=" + std::to_string(stored.window) +
                                            ", this engine is vocabulary=" + std::to_string(e->V) +
                                            " window=" + std::to_string(e->W)));
        }
        // Module.loadStateDict: every named parameter must be present with the right size.
        for (size_t i = 0; i < e->names.size(); ++i) {
            auto it = stored.params.find(e->names[i]);
            if (it == stored.params.end()) {
                return set_error(e, e->fail(BST_INVALID, "missing state entry " + e->names[i]));
            }
            if (it->second.size() != e->values[i].size()) {
                return set_error(e, e->fail(BST_SHAPE, "state entry " + e->names[i] + " has " +
                                                           std::to_string(it->second.size()) +
                                                           " values, expected " +
                                                           std::to_string(e->values[i].size())));
            }
        }
        for (size_t i = 0; i < e->names.size(); ++i) e->values[i] = std::move(stored.params[e->names[i]]);
        e->dirty = true;
        return BST_OK;
    })
}

int32_t bst_scores(bst_engine h, const int32_t* contexts, int32_t rows, int32_t length,
                   double* scores) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    BST_GUARDED({
        std::lock_guard<std::mutex> lock(e->mu);
        return set_error(e, e->run(Mode::kScores, contexts, rows, length, 1, 1.0f, 1, nullptr,
                                   false, nullptr, nullptr, scores));
    })
}

int32_t bst_generate(bst_engine h, const int32_t* contexts, int32_t rows, int32_t length,
                     int32_t steps, int32_t* tokens, bst_token_sink sink, void* user) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    BST_GUARDED({
        std::lock_guard<std::mutex> lock(e->mu);
        return set_error(e, e->run(Mode::kGreedy, contexts, rows, length, steps, 1.0f, 1, tokens,
                                   false, sink, user, nullptr));
    })
}

int32_t bst_sample(bst_engine h, const int32_t* contexts, int32_t rows, int32_t length,
                   int32_t steps, float temperature, int32_t top_k, int32_t* tokens,
                   bst_token_sink sink, void* user) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    BST_GUARDED({
        std::lock_guard<std::mutex> lock(e->mu);
        return set_error(e, e->run(Mode::kSample, contexts, rows, length, steps, temperature,
                                   top_k, tokens, false, sink, user, nullptr));
    })
}

int32_t bst_generate_logits(bst_engine h, const int32_t* contexts, int32_t rows, int32_t length,
                            int32_t steps, int32_t* tokens, float* logits) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    BST_GUARDED({
        std::lock_guard<std::mutex> lock(e->mu);
        if (!logits) return set_error(e, e->fail(BST_INVALID, "logits must not be null"));
        return set_error(e, e->run(Mode::kGreedy, contexts, rows, length, steps, 1.0f, 1, tokens,
                                   false, nullptr, nullptr, nullptr, logits));
    })
}

int32_t bst_sample_logits(bst_engine h, const int32_t* contexts, int32_t rows, int32_t length,
                          int32_t steps, float temperature, int32_t top_k, int32_t* tokens,
                          float* logits) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    BST_GUARDED({
        std::lock_guard<std::mutex> lock(e->mu);
        if (!logits) return set_error(e, e->fail(BST_INVALID, "logits must not be null"));
        return set_error(e, e->run(Mode::kSample, contexts, rows, length, steps, temperature,
                                   top_k, tokens, false, nullptr, nullptr, nullptr, logits));
    })
}

// bst_generate_logits / bst_sample_logits keeping the logits of `watch_count` chosen rows only.
static int32_t logits_rows_call(bst_engine h, Mode mode, const int32_t* contexts, int32_t rows,
                                int32_t length, int32_t steps, float temperature, int32_t top_k,
                                int32_t* tokens, int32_t watch_count, const int32_t* watch_rows,
                                float* logits) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    BST_GUARDED({
        std::lock_guard<std::mutex> lock(e->mu);
        if (!logits) return set_error(e, e->fail(BST_INVALID, "logits must not be null"));
        if (watch_count < 1 || !watch_rows) {
            return set_error(e, e->fail(BST_INVALID, "watch_rows must name at least one row"));
        }
        std::vector<int32_t> watch(watch_rows, watch_rows + watch_count);
        for (size_t i = 0; i < watch.size(); ++i) {
            if (watch[i] < 0 || watch[i] >= rows) {
                return set_error(e, e->fail(BST_INVALID, "watched row " + std::to_string(watch[i]) +
                                                             " is outside [0, " +
                                                             std::to_string(rows) + ")"));
            }
            for (size_t j = 0; j < i; ++j) {
                if (watch[j] == watch[i]) {
                    return set_error(e, e->fail(BST_INVALID, "watched row " +
                                                                 std::to_string(watch[i]) +
                                                                 " is named twice"));
                }
            }
        }
        // The watch list lives for this call only, however it ends.
        struct WatchScope {
            std::vector<int32_t>& w;
            ~WatchScope() { w.clear(); }
        } scope{e->watch};
        e->watch = std::move(watch);
        return set_error(e, e->run(mode, contexts, rows, length, steps, temperature, top_k, tokens,
                                   false, nullptr, nullptr, nullptr, logits));
    })
}

int32_t bst_generate_logits_rows(bst_engine h, const int32_t* contexts, int32_t rows,
                                 int32_t length, int32_t steps, int32_t* tokens,
                                 int32_t watch_count, const int32_t* watch_rows, float* logits) {
    return logits_rows_call(h, Mode::kGreedy, contexts, rows, length, steps, 1.0f, 1, tokens,
                            watch_count, watch_rows, logits);
}

int32_t bst_sample_logits_rows(bst_engine h, const int32_t* contexts, int32_t rows,
                               int32_t length, int32_t steps, float temperature, int32_t top_k,
                               int32_t* tokens, int32_t watch_count, const int32_t* watch_rows,
                               float* logits) {
    return logits_rows_call(h, Mode::kSample, contexts, rows, length, steps, temperature, top_k,
                            tokens, watch_count, watch_rows, logits);
}

static int32_t device_call(bst_engine h, Mode mode, const int32_t* contexts, int32_t rows,
                           int32_t length, int32_t steps, float temperature, int32_t top_k,
                           int32_t* tokens) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    BST_GUARDED({
        std::lock_guard<std::mutex> lock(e->mu);
        if (!contexts || rows < 1 || length < 1) {
            return set_error(e, e->fail(BST_INVALID, "contexts must be a non-empty device buffer"));
        }
        cudaError_t err = cudaSetDevice(e->device);
        std::vector<int32_t> host(static_cast<size_t>(rows) * length);
        if (!err) err = cudaMemcpyAsync(host.data(), contexts, sizeof(int32_t) * host.size(),
                                        cudaMemcpyDeviceToHost, e->stream);
        if (!err) err = cudaStreamSynchronize(e->stream);
        if (err) return set_error(e, e->cuda_fail(err, "reading device contexts"));
        return set_error(e, e->run(mode, host.data(), rows, length, steps, temperature, top_k,
                                   tokens, true, nullptr, nullptr, nullptr));
    })
}

int32_t bst_generate_device(bst_engine h, const int32_t* contexts, int32_t rows, int32_t length,
                            int32_t steps, int32_t* tokens) {
    return device_call(h, Mode::kGreedy, contexts, rows, length, steps, 1.0f, 1, tokens);
}

int32_t bst_sample_device(bst_engine h, const int32_t* contexts, int32_t rows, int32_t length,
                          int32_t steps, float temperature, int32_t top_k, int32_t* tokens) {
    return device_call(h, Mode::kSample, contexts, rows, length, steps, temperature, top_k, tokens);
}

int32_t bst_seed(bst_engine h, int64_t seed) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    std::lock_guard<std::mutex> lock(e->mu);
    e->rng_state = jrand::scramble(seed);
    return BST_OK;
}

int32_t bst_get_rng_state(bst_engine h, int64_t* state) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    if (!state) return BST_INVALID;
    std::lock_guard<std::mutex> lock(e->mu);
    *state = static_cast<int64_t>(e->rng_state);
    return BST_OK;
}

int32_t bst_set_rng_state(bst_engine h, int64_t state) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    std::lock_guard<std::mutex> lock(e->mu);
    e->rng_state = static_cast<uint64_t>(state) & jrand::kMask;
    return BST_OK;
}

int32_t bst_begin_scope(bst_engine h) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    std::lock_guard<std::mutex> lock(e->mu);
    ++e->scope_depth;
    return BST_OK;
}

int32_t bst_end_scope(bst_engine h, int32_t* released) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    std::lock_guard<std::mutex> lock(e->mu);
    if (e->scope_depth == 0) return set_error(e, e->fail(BST_CONTEXT, "no native scope is open"));
    int count = 0;
    cudaSetDevice(e->device);
    if (e->ws.arena.ptr && e->ws.arena.scope >= e->scope_depth) {
        e->free_workspace();
        ++count;
    }
    for (auto it = e->buffers.begin(); it != e->buffers.end();) {
        if (it->scope >= e->scope_depth) {
            cudaFree(it->ptr);
            it = e->buffers.erase(it);
            ++count;
        } else {
            ++it;
        }
    }
    --e->scope_depth;
    if (released) *released = count;
    return BST_OK;
}

int32_t bst_scope_depth(bst_engine h, int32_t* depth) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    if (!depth) return BST_INVALID;
    std::lock_guard<std::mutex> lock(e->mu);
    *depth = e->scope_depth;
    return BST_OK;
}

int32_t bst_engine_stats(bst_engine h, int64_t out[4]) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    if (!out) return BST_INVALID;
    std::lock_guard<std::mutex> lock(e->mu);
    int64_t count = 0, bytes = 0;
    if (e->weights.ptr) {
        ++count;
        bytes += static_cast<int64_t>(e->weights.bytes);
    }
    if (e->ws.arena.ptr) {
        ++count;
        bytes += static_cast<int64_t>(e->ws.arena.bytes);
    }
    for (auto& b : e->buffers) {
        ++count;
        bytes += static_cast<int64_t>(b.bytes);
    }
    out[0] = count;
    out[1] = bytes;
    out[2] = 0;
    out[3] = e->launches;
    return BST_OK;
}

int32_t bst_engine_stream(bst_engine h, void** stream) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    if (!stream) return BST_INVALID;
    *stream = e->stream;
    return BST_OK;
}

int32_t bst_profile_enable(bst_engine h, int32_t enabled) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    std::lock_guard<std::mutex> lock(e->mu);
    e->profiling = enabled != 0;
    return BST_OK;
}

int32_t bst_profile_reset(bst_engine h) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    std::lock_guard<std::mutex> lock(e->mu);
    for (auto& s : e->stats) s = KernelStats{};
    return BST_OK;
}

int32_t bst_profile_read(bst_engine h, int32_t cls, char* name, int32_t capacity,
                         int64_t* launches, double* milliseconds, double* bytes, double* flops) {
    auto e = find_engine(h);
    if (!e) return unknown(h);
    if (cls < 0 || cls >= bst::kKernelClassCount) return BST_INVALID;
    std::lock_guard<std::mutex> lock(e->mu);
    if (name && capacity > 0) std::snprintf(name, static_cast<size_t>(capacity), "%s", bst::kernel_class_name(cls));
    if (launches) *launches = e->stats[cls].launches;
    if (milliseconds) *milliseconds = e->stats[cls].ms;
    if (bytes) *bytes = e->stats[cls].bytes;
    if (flops) *flops = e->stats[cls].flops;
    return BST_OK;
}

int32_t bst_last_error(bst_engine h, char* buffer, int32_t capacity) {
    std::string message;
    if (h == 0) {
        message = t_last_error;
    } else {
        auto e = find_engine(h);
        if (!e) return unknown(h);
        std::lock_guard<std::mutex> lock(e->mu);
        message = e->error;
    }
    if (buffer && capacity > 0) std::snprintf(buffer, static_cast<size_t>(capacity), "%s", message.c_str());
    return static_cast<int32_t>(message.size());
}

int32_t bst_write_synthetic_weights(const bst_model_spec* spec, const char* path, int64_t seed,
                                    double stddev) {
    BST_GUARDED({
        if (!spec || !path) {
            t_last_error = "spec and path must not be null";
            return BST_INVALID;
        }
        const Failure f = validate_spec(*spec);
        if (f.code) {
            t_last_error = f.message;
            return f.code;
        }
        std::vector<std::string> names;
        std::vector<int64_t> sizes;
        declare_parameters(*spec, &names, &sizes);
        std::vector<std::vector<float>> values(names.size());
        jrand::Random random(seed);
        const bool round_matrices = spec->weight_dtype == BST_DTYPE_BF16;
        for (size_t i = 0; i < names.size(); ++i) {
            auto& v = values[i];
            v.resize(static_cast<size_t>(sizes[i]));
            const std::string& n = names[i];
            const bool ln = n.find("norm") != std::string::npos &&
                            (n.size() > 6 && (n.compare(n.size() - 6, 6, ".gamma") == 0 ||
                                              n.compare(n.size() - 5, 5, ".beta") == 0));
            if (spec->family == BST_FAMILY_LAST_TOKEN) {
                if (i == 0) {
                    for (int t = 0; t < spec->vocabulary; ++t) {
                        v[static_cast<size_t>(t) * spec->vocabulary + (t + 1) % spec->vocabulary] = 6.0f;
                    }
                }
                continue;
            }
            if (ln) {
                std::fill(v.begin(), v.end(), is_layernorm_gamma(n) ? 1.0f : 0.0f);
                continue;
            }
            const bool bf = round_matrices && stored_as_matrix(spec->family, n);
            for (auto& x : v) {
                x = static_cast<float>(random.next_gaussian() * stddev);
                if (bf) x = round_to_bf16(x);
            }
        }
        const Failure w = write_weight_file(path, spec->vocabulary, spec->window, names, values);
        if (w.code) {
            t_last_error = w.message;
            return w.code;
        }
        return BST_OK;
    })
}

int32_t bst_synthetic_prompts(int64_t seed, int32_t rows, int32_t length, int32_t bound,
                              int32_t* out) {
    if (!out || rows < 0 || length < 0 || bound < 1) {
        t_last_error = "invalid prompt request";
        return BST_INVALID;
    }
    jrand::Random random(seed);
    for (int64_t i = 0; i < static_cast<int64_t>(rows) * length; ++i) out[i] = random.next_int(bound);
    return BST_OK;
}

}  // extern "C"
