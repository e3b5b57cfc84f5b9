// Device tensors and the op queue for NativeContext on Device.cuda(i).
//
// The reference keeps tensors in a per-context store of monotonic handles (native/src/tensor.rs:
// 150-176), moves them between devices with Context::transfer (native/src/context.rs:125-133,
// today CPU only: a CUDA target returns "not implemented") and runs ops from a packed queue of
// 128-byte commands (CommandQueueBuilder.java:12-73 -> engine.rs:118-154). Here a context is bound
// to one CUDA device. Its tensors live either on that device (tag 1000 + i, Device.java:22,46-59)
// or on the host (tag 0); transfer between the two is a real cudaMemcpy on the context's stream.
// Queued ops run as CUDA kernels on device tensors, checked the way execute_command checks them
// (null handles, shapes, broadcast), and each executed op is recorded as a graph node as
// Graph::push does (graph.rs:342-388), so graph sizes match the reference's. Backward is not
// offered: TextEngine never calls it.
//
// Errors follow the library's status codes. Every call on a context is serialised by its mutex;
// contexts on different devices are independent.

#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "basalt_cuda.h"
#include "epilogue.cuh"
#include "kernels.h"

namespace bst {
size_t matmul_scratch_bytes(int64_t m, int64_t k, int64_t n);
int32_t matmul_with_scratch(cudaStream_t s, const float* a, const float* b, float* c, int64_t m,
                            int64_t k, int64_t n, void* scratch, size_t scratch_bytes,
                            std::string* error);
}  // namespace bst

namespace {

constexpr int kMaxRank = 8;

// Op codes of the wire format (graph.rs:52-95, CommandQueueBuilder.java:31-68).
enum Op : int {
    kMatMul = 1, kAdd = 2, kReLU = 3, kSub = 4, kMul = 5, kSigmoid = 6, kTanh = 7, kGelu = 11,
    kExp = 23, kLog = 24, kSqrt = 25, kAbs = 26, kNeg = 27, kDiv = 28
};

const char* op_name(int op) {
    switch (op) {
        case kMatMul: return "MatMul";
        case kAdd: return "Add";
        case kReLU: return "ReLU";
        case kSub: return "Sub";
        case kMul: return "Mul";
        case kSigmoid: return "Sigmoid";
        case kTanh: return "Tanh";
        case kGelu: return "Gelu";
        case kExp: return "Exp";
        case kLog: return "Log";
        case kSqrt: return "Sqrt";
        case kAbs: return "Abs";
        case kNeg: return "Neg";
        case kDiv: return "Div";
        default: return "?";
    }
}

bool is_binary(int op) { return op == kAdd || op == kSub || op == kMul || op == kDiv; }
bool is_unary(int op) {
    return op == kReLU || op == kSigmoid || op == kTanh || op == kGelu || op == kExp ||
           op == kLog || op == kSqrt || op == kAbs || op == kNeg;
}

// ---- kernels ----
struct Broadcast {
    int rank;
    int64_t out_shape[kMaxRank];
    int64_t a_stride[kMaxRank];  // 0 along broadcast axes (ops.rs:166-176 aligned_strides)
    int64_t b_stride[kMaxRank];
};

// One f32 operation per element, as ops.rs::binary_forward (ops.rs:186-284).
__global__ void k_binary(int op, const float* __restrict__ a, const float* __restrict__ b,
                         float* __restrict__ out, Broadcast bc, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t rest = i, ia = 0, ib = 0;
        for (int axis = bc.rank - 1; axis >= 0; --axis) {
            const int64_t c = rest % bc.out_shape[axis];
            rest /= bc.out_shape[axis];
            ia += c * bc.a_stride[axis];
            ib += c * bc.b_stride[axis];
        }
        const float x = a[ia], y = b[ib];
        float v;
        switch (op) {
            case kAdd: v = __fadd_rn(x, y); break;
            case kSub: v = __fsub_rn(x, y); break;
            case kMul: v = __fmul_rn(x, y); break;
            default: v = __fdiv_rn(x, y); break;
        }
        out[i] = v;
    }
}

// ops.rs::unary_forward (ops.rs:771-820) and gelu_forward (nn_ops.rs:130-137), f32.
__global__ void k_unary(int op, const float* __restrict__ in, float* __restrict__ out, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float x = in[i];
        float v;
        switch (op) {
            case kReLU: v = fmaxf(x, 0.0f); break;
            case kSigmoid:
                if (x >= 0.0f) {
                    v = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
                } else {
                    const float e = expf(x);
                    v = __fdiv_rn(e, __fadd_rn(1.0f, e));
                }
                break;
            case kTanh: v = tanhf(x); break;
            case kGelu: v = bst::gelu_ref(x); break;
            case kExp: v = expf(x); break;
            case kLog: v = logf(x); break;
            case kSqrt: v = __fsqrt_rn(x); break;
            case kAbs: v = fabsf(x); break;
            default: v = -x; break;
        }
        out[i] = v;
    }
}

int grid_for(int64_t n) {
    const int64_t blocks = (n + 255) / 256;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, 148 * 8)));
}

// ---- the store ----
struct Tensor {
    int tag = 0;  // 0: host, 1000 + i: CUDA device i
    std::vector<int64_t> shape;
    int64_t numel = 0;
    float* device = nullptr;
    std::vector<float> host;
};

struct Node {
    int op;
    uint64_t inputs[2];
    uint64_t output;
};

struct Context {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::mutex mu;
    std::unordered_map<uint64_t, Tensor> tensors;
    uint64_t next_tensor = 1;
    std::vector<Node> graph;
    int64_t launches = 0;
    int64_t device_bytes = 0;
    std::string error;

    int fail(int code, const std::string& message) {
        error = message;
        return code;
    }
    int cuda_fail(cudaError_t e, const char* what) {
        cudaGetLastError();
        return fail(e == cudaErrorMemoryAllocation ? BST_OOM : BST_PANIC,
                    std::string(what) + ": " + cudaGetErrorName(e) + ": " + cudaGetErrorString(e));
    }
    int tag() const { return BST_DEVICE_TAG_CUDA + device; }

    ~Context() {
        cudaSetDevice(device);
        for (auto& kv : tensors) {
            if (kv.second.device) cudaFree(kv.second.device);
        }
        if (stream) cudaStreamDestroy(stream);
    }

    Tensor* find(uint64_t h) {
        auto it = tensors.find(h);
        return it == tensors.end() ? nullptr : &it->second;
    }
    int unknown_tensor(uint64_t h) {
        return fail(BST_UNKNOWN_HANDLE, "tensor handle " + std::to_string(h) + " is not live");
    }

    int add(Tensor t, uint64_t* out) {
        if (t.tag != 0) {
            const size_t bytes = sizeof(float) * static_cast<size_t>(std::max<int64_t>(t.numel, 1));
            const cudaError_t e = cudaMalloc(&t.device, bytes);
            if (e) return cuda_fail(e, "allocating a device tensor");
            device_bytes += static_cast<int64_t>(bytes);
        }
        const uint64_t h = next_tensor++;
        tensors.emplace(h, std::move(t));
        *out = h;
        return BST_OK;
    }
};

std::mutex g_mutex;
std::unordered_map<uint64_t, std::shared_ptr<Context>> g_contexts;
uint64_t g_next_context = 1;
std::shared_ptr<Context> find_context(bst_context h) {
    std::lock_guard<std::mutex> lock(g_mutex);
    auto it = g_contexts.find(h);
    return it == g_contexts.end() ? nullptr : it->second;
}

int unknown_context(bst_context h) {
    bst::set_thread_error("context handle " + std::to_string(h) + " is not live");
    return BST_UNKNOWN_HANDLE;
}

int finish(const std::shared_ptr<Context>& c, int code) {
    if (code != BST_OK) bst::set_thread_error(c->error);
    return code;
}

int check_tag(Context& c, int tag) {
    if (tag == BST_DEVICE_TAG_CPU || tag == c.tag()) return BST_OK;
    if (tag >= BST_DEVICE_TAG_CUDA && tag < BST_DEVICE_TAG_CUDA + 1000) {
        return c.fail(BST_UNSUPPORTED, "device cuda:" + std::to_string(tag - BST_DEVICE_TAG_CUDA) +
                                           " is not this context's device (cuda:" +
                                           std::to_string(c.device) + ")");
    }
    return c.fail(BST_INVALID, "unknown device tag: " + std::to_string(tag));
}

int64_t numel_of(const std::vector<int64_t>& shape) {
    int64_t n = 1;
    for (int64_t s : shape) n *= s;
    return n;
}

// Tensor.broadcastShape / ops.rs:136-164: trailing alignment, size-1 axes broadcast.
bool broadcast_shape(const std::vector<int64_t>& a, const std::vector<int64_t>& b,
                     std::vector<int64_t>* out) {
    const size_t rank = std::max(a.size(), b.size());
    out->assign(rank, 1);
    for (size_t i = 0; i < rank; ++i) {
        const int64_t ad = i < rank - a.size() ? 1 : a[i - (rank - a.size())];
        const int64_t bd = i < rank - b.size() ? 1 : b[i - (rank - b.size())];
        if (ad == bd || bd == 1) {
            (*out)[i] = ad;
        } else if (ad == 1) {
            (*out)[i] = bd;
        } else {
            return false;
        }
    }
    return true;
}

std::string shape_str(const std::vector<int64_t>& s) {
    std::string r = "[";
    for (size_t i = 0; i < s.size(); ++i) r += (i ? ", " : "") + std::to_string(s[i]);
    return r + "]";
}

// Strides of `shape` aligned to the trailing axes of `out` (0 where shape broadcasts).
void aligned_strides(const std::vector<int64_t>& shape, const std::vector<int64_t>& out,
                     int64_t* strides) {
    const size_t rank = out.size(), lead = rank - shape.size();
    int64_t stride = 1;
    for (size_t i = rank; i-- > 0;) {
        if (i < lead) {
            strides[i] = 0;
            continue;
        }
        const int64_t dim = shape[i - lead];
        strides[i] = dim == 1 ? 0 : stride;
        stride *= dim;
    }
}

struct Command {
    int op;
    uint64_t in[5];
    uint64_t out;
    int32_t attrs[16];
};

Command decode(const unsigned char* p) {
    Command c;
    c.op = p[0];
    std::memcpy(c.in, p + 8, sizeof(c.in));
    std::memcpy(&c.out, p + 48, sizeof(c.out));
    std::memcpy(c.attrs, p + 56, sizeof(c.attrs));
    return c;
}

// engine.rs:137-330 execute_command for the ops this library runs on the GPU.
int execute(Context& c, const Command& cmd) {
    const int op = cmd.op;
    if (op != kMatMul && !is_binary(op) && !is_unary(op)) {
        if (op < 1 || op > 37) {
            return c.fail(BST_UNSUPPORTED, "unknown op code " + std::to_string(op));
        }
        return c.fail(BST_UNSUPPORTED, "op code " + std::to_string(op) +
                                           " has no CUDA kernel in this library");
    }
    if (cmd.out == 0) return c.fail(BST_INVALID, "op output handle must not be null");
    const int arity = is_unary(op) ? 1 : 2;
    for (int i = 0; i < arity; ++i) {
        if (cmd.in[i] == 0) {
            return c.fail(BST_INVALID, "input " + std::to_string(i) + " of the command is null");
        }
    }
    Tensor* out = c.find(cmd.out);
    if (!out) return c.unknown_tensor(cmd.out);
    Tensor* a = c.find(cmd.in[0]);
    if (!a) return c.unknown_tensor(cmd.in[0]);
    Tensor* b = nullptr;
    if (arity == 2) {
        b = c.find(cmd.in[1]);
        if (!b) return c.unknown_tensor(cmd.in[1]);
    }
    for (const Tensor* t : {out, a, b}) {
        if (!t) continue;
        if (t->tag == BST_DEVICE_TAG_CPU) {
            return c.fail(BST_UNSUPPORTED, std::string(op_name(op)) +
                                               ": host tensors run on the CPU engine; transfer them "
                                               "to cuda:" + std::to_string(c.device) + " first");
        }
    }
    cudaError_t e = cudaSuccess;
    if (op == kMatMul) {
        if (a->shape.size() != 2 || b->shape.size() != 2) {
            return c.fail(BST_SHAPE, "MatMul expects rank-2 operands");
        }
        const int64_t m = a->shape[0], k = a->shape[1], n = b->shape[1];
        if (k != b->shape[0] || out->shape != std::vector<int64_t>{m, n}) {
            return c.fail(BST_SHAPE, "MatMul shape mismatch: " + shape_str(a->shape) + " x " +
                                         shape_str(b->shape) + " -> " + shape_str(out->shape));
        }
        if (m > 0 && n > 0) {
            if (k == 0) {
                e = cudaMemsetAsync(out->device, 0, sizeof(float) * m * n, c.stream);
            } else {
                if ((e = bst::configure_device_kernels_once(c.device)) != cudaSuccess) {
                    return c.cuda_fail(e, "MatMul");
                }
                void* scratch = nullptr;
                const size_t bytes = bst::matmul_scratch_bytes(m, k, n);
                e = cudaMallocAsync(&scratch, bytes, c.stream);
                if (e) return c.cuda_fail(e, "MatMul scratch");
                std::string why;
                const int st = bst::matmul_with_scratch(c.stream, a->device, b->device,
                                                        out->device, m, k, n, scratch, bytes, &why);
                cudaFreeAsync(scratch, c.stream);
                if (st) return c.fail(st, why);
                c.launches += 3;
            }
        }
    } else if (is_binary(op)) {
        std::vector<int64_t> shape;
        if (!broadcast_shape(a->shape, b->shape, &shape)) {
            return c.fail(BST_SHAPE, "cannot broadcast shapes " + shape_str(a->shape) + " and " +
                                         shape_str(b->shape));
        }
        if (out->shape != shape) {
            return c.fail(BST_SHAPE, std::string(op_name(op)) + " output shape must be " +
                                         shape_str(shape));
        }
        if (shape.size() > kMaxRank) return c.fail(BST_UNSUPPORTED, "rank above 8");
        Broadcast bc{};
        bc.rank = static_cast<int>(shape.size());
        for (int i = 0; i < bc.rank; ++i) bc.out_shape[i] = shape[i];
        aligned_strides(a->shape, shape, bc.a_stride);
        aligned_strides(b->shape, shape, bc.b_stride);
        if (out->numel > 0) {
            k_binary<<<grid_for(out->numel), 256, 0, c.stream>>>(op, a->device, b->device,
                                                                  out->device, bc, out->numel);
            e = cudaGetLastError();
            c.launches += 1;
        }
    } else {
        if (out->shape != a->shape) {
            return c.fail(BST_SHAPE, std::string(op_name(op)) + " output shape must be " +
                                         shape_str(a->shape));
        }
        if (out->numel > 0) {
            k_unary<<<grid_for(out->numel), 256, 0, c.stream>>>(op, a->device, out->device,
                                                                 out->numel);
            e = cudaGetLastError();
            c.launches += 1;
        }
    }
    if (e) return c.cuda_fail(e, op_name(op));
    c.graph.push_back(Node{op, {cmd.in[0], arity == 2 ? cmd.in[1] : 0}, cmd.out});
    return BST_OK;
}

#define BST_TENSOR_GUARDED(...)                                             \
    try {                                                                   \
        __VA_ARGS__                                                         \
    } catch (const std::bad_alloc&) {                                       \
        bst::set_thread_error("host allocation failed");                    \
        return BST_OOM;                                                     \
    } catch (const std::exception& ex) {                                    \
        bst::set_thread_error(std::string("internal error: ") + ex.what()); \
        return BST_PANIC;                                                   \
    }

}  // namespace

extern "C" {

int32_t bst_context_create(int32_t device_tag, bst_context* out) {
    BST_TENSOR_GUARDED({
        if (!out) {
            bst::set_thread_error("out must not be null");
            return BST_INVALID;
        }
        if (device_tag == BST_DEVICE_TAG_CPU) {
            bst::set_thread_error("cpu contexts are served by the CPU engine (NativeContext)");
            return BST_UNSUPPORTED;
        }
        if (device_tag < BST_DEVICE_TAG_CUDA || device_tag >= BST_DEVICE_TAG_CUDA + 1000) {
            bst::set_thread_error("unknown device tag: " + std::to_string(device_tag));
            return BST_INVALID;
        }
        const int device = device_tag - BST_DEVICE_TAG_CUDA;
        int n = 0;
        cudaError_t e = cudaGetDeviceCount(&n);
        if (e || device >= n) {
            cudaGetLastError();
            bst::set_thread_error("CUDA device " + std::to_string(device) + " is not available");
            return BST_UNSUPPORTED;
        }
        auto c = std::make_shared<Context>();
        c->device = device;
        if ((e = cudaSetDevice(device)) == cudaSuccess) {
            e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
        }
        if (e) {
            cudaGetLastError();
            bst::set_thread_error(std::string("creating a context stream: ") + cudaGetErrorString(e));
            return BST_PANIC;
        }
        std::lock_guard<std::mutex> lock(g_mutex);
        const uint64_t h = g_next_context++;
        g_contexts[h] = c;
        *out = h;
        return BST_OK;
    })
}

int32_t bst_context_destroy(bst_context h) {
    std::shared_ptr<Context> c;
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        auto it = g_contexts.find(h);
        if (it == g_contexts.end()) return unknown_context(h);
        c = it->second;
        g_contexts.erase(it);
    }
    std::lock_guard<std::mutex> lock(c->mu);
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    return BST_OK;
}

int32_t bst_tensor_create(bst_context h, int32_t device_tag, const int64_t* shape, int32_t rank,
                          const float* values, bst_tensor* out) {
    auto c = find_context(h);
    if (!c) return unknown_context(h);
    BST_TENSOR_GUARDED({
        std::lock_guard<std::mutex> lock(c->mu);
        if (!out || (rank > 0 && !shape)) return finish(c, c->fail(BST_INVALID, "shape and out must not be null"));
        if (rank < 1 || rank > kMaxRank) {
            return finish(c, c->fail(BST_SHAPE, "rank must be 1..8, got " + std::to_string(rank)));
        }
        int st = check_tag(*c, device_tag);
        if (st) return finish(c, st);
        Tensor t;
        t.tag = device_tag;
        t.shape.assign(shape, shape + rank);
        for (int64_t s : t.shape) {
            if (s < 0) return finish(c, c->fail(BST_SHAPE, "negative dimension in " + shape_str(t.shape)));
        }
        t.numel = numel_of(t.shape);
        if (device_tag == BST_DEVICE_TAG_CPU) {
            t.host.assign(static_cast<size_t>(t.numel), 0.0f);
            if (values) std::memcpy(t.host.data(), values, sizeof(float) * t.numel);
            return finish(c, c->add(std::move(t), out));
        }
        cudaSetDevice(c->device);
        const int64_t n = t.numel;
        st = c->add(std::move(t), out);
        if (st) return finish(c, st);
        Tensor* made = c->find(*out);
        cudaError_t e = values ? cudaMemcpyAsync(made->device, values, sizeof(float) * n,
                                                 cudaMemcpyHostToDevice, c->stream)
                               : cudaMemsetAsync(made->device, 0, sizeof(float) * n, c->stream);
        if (!e) e = cudaStreamSynchronize(c->stream);
        return finish(c, e ? c->cuda_fail(e, "initialising a device tensor") : BST_OK);
    })
}

int32_t bst_tensor_transfer(bst_context h, bst_tensor src, int32_t device_tag, bst_tensor* out) {
    auto c = find_context(h);
    if (!c) return unknown_context(h);
    BST_TENSOR_GUARDED({
        std::lock_guard<std::mutex> lock(c->mu);
        if (!out) return finish(c, c->fail(BST_INVALID, "out must not be null"));
        int st = check_tag(*c, device_tag);
        if (st) return finish(c, st);
        Tensor* s = c->find(src);
        if (!s) return finish(c, c->unknown_tensor(src));
        Tensor t;
        t.tag = device_tag;
        t.shape = s->shape;
        t.numel = s->numel;
        const int from = s->tag;
        if (device_tag == BST_DEVICE_TAG_CPU) t.host.assign(static_cast<size_t>(t.numel), 0.0f);
        cudaSetDevice(c->device);
        st = c->add(std::move(t), out);
        if (st) return finish(c, st);
        Tensor* d = c->find(*out);
        s = c->find(src);  // the map may have rehashed
        const size_t bytes = sizeof(float) * static_cast<size_t>(d->numel);
        cudaError_t e = cudaSuccess;
        if (bytes == 0) {
        } else if (from == BST_DEVICE_TAG_CPU && device_tag == BST_DEVICE_TAG_CPU) {
            std::memcpy(d->host.data(), s->host.data(), bytes);
        } else if (from == BST_DEVICE_TAG_CPU) {
            e = cudaMemcpyAsync(d->device, s->host.data(), bytes, cudaMemcpyHostToDevice, c->stream);
        } else if (device_tag == BST_DEVICE_TAG_CPU) {
            e = cudaMemcpyAsync(d->host.data(), s->device, bytes, cudaMemcpyDeviceToHost, c->stream);
        } else {
            e = cudaMemcpyAsync(d->device, s->device, bytes, cudaMemcpyDeviceToDevice, c->stream);
        }
        if (!e) e = cudaStreamSynchronize(c->stream);
        return finish(c, e ? c->cuda_fail(e, "transferring a tensor") : BST_OK);
    })
}

int32_t bst_tensor_read(bst_context h, bst_tensor t, float* values, int64_t count) {
    auto c = find_context(h);
    if (!c) return unknown_context(h);
    BST_TENSOR_GUARDED({
        std::lock_guard<std::mutex> lock(c->mu);
        Tensor* x = c->find(t);
        if (!x) return finish(c, c->unknown_tensor(t));
        if (!values || count != x->numel) {
            return finish(c, c->fail(BST_SHAPE, "tensor has " + std::to_string(x->numel) +
                                                    " elements, buffer holds " +
                                                    std::to_string(count)));
        }
        if (x->tag == BST_DEVICE_TAG_CPU) {
            std::memcpy(values, x->host.data(), sizeof(float) * count);
            return BST_OK;
        }
        cudaSetDevice(c->device);
        cudaError_t e = cudaMemcpyAsync(values, x->device, sizeof(float) * count,
                                        cudaMemcpyDeviceToHost, c->stream);
        if (!e) e = cudaStreamSynchronize(c->stream);
        return finish(c, e ? c->cuda_fail(e, "reading a tensor") : BST_OK);
    })
}

int32_t bst_tensor_write(bst_context h, bst_tensor t, const float* values, int64_t count) {
    auto c = find_context(h);
    if (!c) return unknown_context(h);
    BST_TENSOR_GUARDED({
        std::lock_guard<std::mutex> lock(c->mu);
        Tensor* x = c->find(t);
        if (!x) return finish(c, c->unknown_tensor(t));
        if (!values || count != x->numel) {
            return finish(c, c->fail(BST_SHAPE, "tensor has " + std::to_string(x->numel) +
                                                    " elements, got " + std::to_string(count)));
        }
        if (x->tag == BST_DEVICE_TAG_CPU) {
            std::memcpy(x->host.data(), values, sizeof(float) * count);
            return BST_OK;
        }
        cudaSetDevice(c->device);
        cudaError_t e = cudaMemcpyAsync(x->device, values, sizeof(float) * count,
                                        cudaMemcpyHostToDevice, c->stream);
        if (!e) e = cudaStreamSynchronize(c->stream);
        return finish(c, e ? c->cuda_fail(e, "writing a tensor") : BST_OK);
    })
}

int32_t bst_tensor_info(bst_context h, bst_tensor t, int32_t* device_tag, int32_t* rank,
                        int64_t* shape, int32_t capacity) {
    auto c = find_context(h);
    if (!c) return unknown_context(h);
    std::lock_guard<std::mutex> lock(c->mu);
    Tensor* x = c->find(t);
    if (!x) return finish(c, c->unknown_tensor(t));
    if (device_tag) *device_tag = x->tag;
    if (rank) *rank = static_cast<int32_t>(x->shape.size());
    for (int32_t i = 0; shape && i < capacity && i < static_cast<int32_t>(x->shape.size()); ++i) {
        shape[i] = x->shape[i];
    }
    return BST_OK;
}

// Context::release_tensor (context.rs): releasing twice is harmless, as NativeTensorHandle.close
// is idempotent; *released tells whether this call freed it.
int32_t bst_tensor_release(bst_context h, bst_tensor t, int32_t* released) {
    auto c = find_context(h);
    if (!c) return unknown_context(h);
    std::lock_guard<std::mutex> lock(c->mu);
    if (released) *released = 0;
    if (t == 0 || t >= c->next_tensor) return finish(c, c->unknown_tensor(t));
    auto it = c->tensors.find(t);
    if (it == c->tensors.end()) return BST_OK;
    // A node that reads or writes the tensor invalidates the recorded graph (context.rs).
    for (const Node& n : c->graph) {
        if (n.output == t || n.inputs[0] == t || n.inputs[1] == t) {
            c->graph.clear();
            break;
        }
    }
    if (it->second.device) {
        cudaSetDevice(c->device);
        cudaStreamSynchronize(c->stream);
        cudaFree(it->second.device);
        c->device_bytes -= static_cast<int64_t>(sizeof(float) *
                                                std::max<int64_t>(it->second.numel, 1));
    }
    c->tensors.erase(it);
    if (released) *released = 1;
    return BST_OK;
}

// NativeBindings.executeQueue (engine.rs:118-135): `count` packed 128-byte commands, run in order;
// the first failing command stops the queue with its status. Returns once every op has finished.
int32_t bst_execute_queue(bst_context h, const void* commands, int32_t count) {
    auto c = find_context(h);
    if (!c) return unknown_context(h);
    BST_TENSOR_GUARDED({
        std::lock_guard<std::mutex> lock(c->mu);
        if (count < 0 || (count > 0 && !commands)) {
            return finish(c, c->fail(BST_INVALID, "commands must hold count 128-byte records"));
        }
        cudaSetDevice(c->device);
        const unsigned char* p = static_cast<const unsigned char*>(commands);
        for (int32_t i = 0; i < count; ++i) {
            const int st = execute(*c, decode(p + static_cast<size_t>(i) * BST_COMMAND_BYTES));
            if (st) {
                cudaStreamSynchronize(c->stream);
                return finish(c, st);
            }
        }
        const cudaError_t e = cudaStreamSynchronize(c->stream);
        return finish(c, e ? c->cuda_fail(e, "executing the queue") : BST_OK);
    })
}

// NativeContext.stats / graphSize: out[0] live tensors, out[1] live device bytes, out[2] graph
// nodes recorded, out[3] kernels launched.
int32_t bst_context_stats(bst_context h, int64_t out[4]) {
    auto c = find_context(h);
    if (!c) return unknown_context(h);
    std::lock_guard<std::mutex> lock(c->mu);
    if (!out) return finish(c, c->fail(BST_INVALID, "out must not be null"));
    out[0] = static_cast<int64_t>(c->tensors.size());
    out[1] = c->device_bytes;
    out[2] = static_cast<int64_t>(c->graph.size());
    out[3] = c->launches;
    return BST_OK;
}

int32_t bst_context_clear_graph(bst_context h) {
    auto c = find_context(h);
    if (!c) return unknown_context(h);
    std::lock_guard<std::mutex> lock(c->mu);
    c->graph.clear();
    return BST_OK;
}

}  // extern "C"
