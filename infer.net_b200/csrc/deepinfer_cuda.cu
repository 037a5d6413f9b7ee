// deepinfer_cuda: C ABI of the B200 MoE block backend (see include/deepinfer_cuda.h).
#include "../../include/deepinfer_cuda.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <initializer_list>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "checkpoint.h"
#include "common.cuh"
#include "decode.cuh"
#include "decode_stack.cuh"
#include "ep.cuh"
#include "gemv.cuh"
#include "generate.cuh"
#include "grouped_gemm.cuh"
#include "route.cuh"

#define API extern "C" __attribute__((visibility("default")))

namespace {

using namespace di;

void set_error(char *error, int capacity, const char *fmt, ...) {
    if (!error || capacity <= 0) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(error, (size_t)capacity, fmt, ap);
    va_end(ap);
}

struct CudaFail {
    std::string what;
};
#define CK(call)                                                                                        \
    do {                                                                                                \
        cudaError_t e_ = (call);                                                                        \
        if (e_ != cudaSuccess) {                                                                        \
            cudaGetLastError(); /* a later call's launch check must not report this failure */          \
            throw CudaFail{std::string(#call) + ": " + cudaGetErrorString(e_)};                         \
        }                                                                                               \
    } while (0)

struct Context;

struct Matrix {
    Context *ctx = nullptr;
    int experts = 0, rows = 0, cols = 0, bits = 0;
    void *d[3] = {nullptr, nullptr, nullptr};
    void *h[3] = {nullptr, nullptr, nullptr};
    size_t bytes[3] = {0, 0, 0};
    bool dirty[3] = {false, false, false};
    uint64_t version = 1;  // bumped whenever the library changes the device bytes
    bool exposed = false;  // the device buffers were handed out: writes to them are not seen
    int refs = 1;  // the caller's handle plus one per layer binding it
    bool destroyed = false;
    QView view() const {
        return QView{(const uint32_t *)d[0], (const uint16_t *)d[1], (const uint16_t *)d[2], experts, rows, cols, bits};
    }
};

struct Layer {
    Context *ctx = nullptr;
    Matrix *m[8] = {};  // router, gate, up, down, shared_gate, shared_up, shared_down, shared_route
    float *bias = nullptr;  // device [E] or null
    int E = 0, D = 0, I = 0, bits = 0;
    uint64_t gen = 0;       // unique per layer object, for graph cache keys
    int E_local = 0, E_off = 0;  // expert-parallel shard: experts [E_off, E_off + E_local) are local
    float *router_rn = nullptr;  // device: router row norms [2E] then f32 router rows [E, D]
    uint64_t router_rn_version = 0;  // the router matrix version they were computed from
};
uint64_t g_layer_gen = 0;

// Device scratch of one context; grows, never shrinks.
struct Workspace {
    void *base = nullptr;
    size_t cap = 0;
};

enum Stage { S_ROUTER, S_TOPK, S_SCAN, S_SCATTER, S_GATE_UP, S_DOWN, S_COMBINE, S_N };
constexpr int kProfileSlots = S_N + 1;  // + rmsnorm for stacks

struct Context {
    int device = 0, sms = 0;
    bool resident = false;
    int refresh_ms = 1000;
    cudaStream_t stream = nullptr;
    cudaEvent_t ev_start = nullptr, ev_stop = nullptr, ev_stage[S_N + 1] = {};
    std::set<Matrix *> matrices;
    Workspace ws;
    uint32_t *d_err = nullptr, *h_err = nullptr;
    double last_stage_ms[kProfileSlots] = {};
    bool have_profile = false;
    std::vector<cudaEvent_t> layer_events;  // [layer][S_N + 2] for profiled stacks
    // CUDA graph of the last decode-path stack, replayed while its key matches
    std::vector<uint64_t> graph_key;
    cudaGraphExec_t graph_exec = nullptr;
    // persistent one-token stack kernel: exchange words + generation counter (zeroed once), and
    // the per-layer descriptors of the last stack, re-uploaded when its key changes
    unsigned long long *ll = nullptr;
    size_t ll_words = 0;
    size_t ll_used = 0;  // words of the layout the last stack call used
    ds::StackLayer *d_stack = nullptr;
    CUtensorMap *d_stack_maps = nullptr;  // [stack_cap][2] down-column maps of the stack kernel
    size_t stack_cap = 0;
    std::vector<ds::StackLayer> h_stack;
    std::vector<uint64_t> stack_key;
    // the expert-grouped permutation of the last grouped-path block (of the last layer of a stack):
    // device pointers into the workspace, valid until the next call on this context
    const int32_t *last_perm = nullptr, *last_seg_off = nullptr, *last_seg_count = nullptr;
    int last_routes_T = 0, last_routes_E = 0;
};

std::mutex g_registry;
std::set<Context *> g_contexts;
std::set<Matrix *> g_matrices;
std::set<Layer *> g_layers;

bool live_context(void *p) {
    std::lock_guard<std::mutex> g(g_registry);
    return p && g_contexts.count(static_cast<Context *>(p));
}
bool live_matrix(void *p) {
    std::lock_guard<std::mutex> g(g_registry);
    return p && g_matrices.count(static_cast<Matrix *>(p)) && !static_cast<Matrix *>(p)->destroyed;
}
bool live_layer(void *p) {
    std::lock_guard<std::mutex> g(g_registry);
    return p && g_layers.count(static_cast<Layer *>(p));
}

void release_matrix(Matrix *m) {
    if (--m->refs > 0) return;
    {
        std::lock_guard<std::mutex> g(g_registry);
        g_matrices.erase(m);
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(m->ctx->device);
    for (int i = 0; i < 3; ++i) {
        if (m->d[i]) cudaFree(m->d[i]);
        if (m->h[i]) cudaFreeHost(m->h[i]);
    }
    m->ctx->matrices.erase(m);
    cudaSetDevice(prev);
    delete m;
}

struct DeviceGuard {
    int prev = 0;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() { cudaSetDevice(prev); }
};

// Upload every host-staged buffer of m that was handed out since its last upload.
void sync_matrix(Matrix *m) {
    for (int i = 0; i < 3; ++i)
        if (m->dirty[i]) {
            CK(cudaMemcpyAsync(m->d[i], m->h[i], m->bytes[i], cudaMemcpyHostToDevice, m->ctx->stream));
            m->dirty[i] = false;
            m->version++;
        }
}

// Bump allocator over the context workspace; sizes are computed before any launch.
struct Carve {
    size_t off = 0;
    template <class T>
    size_t take(size_t n) {
        off = (off + 255) & ~(size_t)255;
        size_t o = off;
        off += n * sizeof(T);
        return o;
    }
};

void ensure_workspace(Context *c, size_t bytes) {
    if (c->ws.cap >= bytes) return;
    if (c->ws.base) {
        CK(cudaStreamSynchronize(c->stream));
        CK(cudaFree(c->ws.base));
        c->ws.base = nullptr;
        c->ws.cap = 0;
    }
    size_t cap = std::max(bytes, (size_t)64 << 20);
    CK(cudaMalloc(&c->ws.base, cap));
    c->ws.cap = cap;
}

template <class T>
T *at(Context *c, size_t off) {
    return reinterpret_cast<T *>(static_cast<uint8_t *>(c->ws.base) + off);
}

// True when p is memory that the context's kernels may be handed as a device pointer: device
// memory of that GPU, or managed memory. Pageable or pinned host memory and other GPUs' memory
// are refused before any GPU work (the reference validates every argument before submission,
// native/DeepInfer.Metal/quantized.mm:323-331), instead of faulting inside a kernel.
bool device_pointer_ok(const void *p, int device) {
    if (!p) return false;
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (a.type == cudaMemoryTypeManaged) return true;
    return a.type == cudaMemoryTypeDevice && a.device == device;
}
// The optional pointers of a device-I/O call: each one given must pass device_pointer_ok.
bool device_pointers_ok(int device, std::initializer_list<const void *> ptrs) {
    for (const void *p : ptrs)
        if (p && !device_pointer_ok(p, device)) return false;
    return true;
}

int launch_check(char *error, int capacity) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error(error, capacity, "CUDA launch failed: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

// Kernel launch, optionally with programmatic dependent launch (the kernel may start while
// the previous one on the stream finishes; it orders itself with griddepcontrol.wait).
template <typename... KArgs, typename... Args>
void launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    CK(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
}

// Cooperative launch: every CTA of the grid is resident at once, or the launch fails. Kernels
// whose CTAs wait on one another (a grid barrier) need it; other work on the GPU may otherwise
// hold SMs that a waiting CTA's partner needs.
template <typename... KArgs, typename... Args>
void launch_cooperative(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CK(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
}

constexpr int kDecodeSmemMax = 96 * 1024;  // decode_route_kernel: T*D bf16 rows

uint64_t eps_bits(float eps) {
    uint32_t u;
    std::memcpy(&u, &eps, 4);
    return u;
}

// The fused one-token decode FFN needs 16-byte scale rows (D, I multiples of 512) and its
// per-CTA weight share to fit in shared memory.
bool ffn_fits(const Context *c, const Layer *L) {
    if (L->D % 512 || L->I % 512) return false;
    const int smem = ffn_layout(L->D, L->I, L->bits, c->sms).total;
    if (smem > 227 * 1024) return false;
    // the cooperative launch needs one resident CTA per SM
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, L->bits == 8 ? decode_ffn_kernel<8> : decode_ffn_kernel<5>,
                                                      kFfnThreads, smem) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return per_sm >= 1;
}

// The persistent one-token stack kernel of a geometry (null when none is built for it).
using StackKernel = void (*)(const ds::StackParams);
StackKernel stack_kernel(int bits, int D) {
    if (bits == 8) return D == 512 ? ds::decode_stack_kernel<8, 512> : D == 1024 ? ds::decode_stack_kernel<8, 1024>
                                       : D == 2048 ? ds::decode_stack_kernel<8, 2048> : nullptr;
    if (bits == 5) return D == 512 ? ds::decode_stack_kernel<5, 512> : D == 1024 ? ds::decode_stack_kernel<5, 1024>
                                       : D == 2048 ? ds::decode_stack_kernel<5, 2048> : nullptr;
    return nullptr;
}

// The persistent one-token stack kernel: layers sharing D, I, E and bits; D in {512, 1024, 2048}
// (a power-of-two number of 16-element chunks per warp), I = 512 (16 units of 32 columns per
// expert slot), E <= 256, at least one CTA per unit (144), its shared-memory share within the
// limit, and one CTA resident on every SM (a cooperative launch).
bool stack_fits(Context *c, void *const *layers, int n) {
    const Layer *L0 = static_cast<const Layer *>(layers[0]);
    for (int l = 0; l < n; ++l) {
        const Layer *L = static_cast<const Layer *>(layers[l]);
        if (L->D != L0->D || L->I != L0->I || L->E != L0->E || L->bits != L0->bits) return false;
    }
    const int D = L0->D, I = L0->I;
    if ((D != 512 && D != 1024 && D != 2048) || I != ds::kI || L0->E > 256 || c->sms < ds::kUnits) return false;
    const int smem = ds::layout(D, L0->bits).total;
    if (smem > 227 * 1024) return false;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, stack_kernel(L0->bits, D), ds::kThreads, smem) !=
        cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return per_sm >= 1;
}

void encode_2d(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t dim0, uint64_t dim1,
               uint64_t stride, uint32_t b0, uint32_t b1, CUtensorMapSwizzle sw);

// Enqueue the persistent stack kernel for one token: x (f32 [D]) is updated in place; h_trace /
// ids_trace (device, optional) receive every layer's normalised input row and expert ids.
void enqueue_stack(Context *c, void *const *layers, int n, const float *norms, float eps, float *x, uint16_t *h_trace,
                   int32_t *ids_trace) {
    const Layer *L0 = static_cast<const Layer *>(layers[0]);
    const int D = L0->D, I = L0->I, E = L0->E;
    // exchange words: [0] the generation counter and the y arrivals, [1] the logit arrivals, then
    // the accumulators y [2][kAccCopies][D], logits [E + 1]
    const size_t words = 2 + 2 * (size_t)ds::kAccCopies * D + E + 1;
    if (c->ll_words < words) {
        if (c->ll) CK(cudaFree(c->ll));
        c->ll = nullptr;
        c->ll_words = 0;
        CK(cudaMalloc(&c->ll, words * 8));
        CK(cudaMemsetAsync(c->ll, 0, words * 8, c->stream));  // generation 0 matches no exchange
        c->ll_words = words;
    } else if (c->ll_used != words) {
        // another geometry's words may sit where this one's logit words are: start over
        CK(cudaMemsetAsync(c->ll, 0, c->ll_words * 8, c->stream));
    }
    c->ll_used = words;
    std::vector<uint64_t> key = {(uint64_t)n, (uint64_t)(uintptr_t)norms};
    for (int l = 0; l < n; ++l) {
        const Layer *L = static_cast<const Layer *>(layers[l]);
        key.push_back(L->gen);
        key.push_back((uint64_t)(uintptr_t)L->bias);
    }
    if (key != c->stack_key) {
        c->h_stack.resize(n);
        for (int l = 0; l < n; ++l) {
            const Layer *L = static_cast<const Layer *>(layers[l]);
            ds::StackLayer &s = c->h_stack[l];
            s.R = L->m[0]->view();
            s.G = L->m[1]->view();
            s.U = L->m[2]->view();
            s.Dn = L->m[3]->view();
            s.SG = L->m[4]->view();
            s.SU = L->m[5]->view();
            s.SD = L->m[6]->view();
            s.SR = L->m[7]->view();
            s.bias = L->bias;
            s.norm = norms + (size_t)l * D;
        }
        if (c->stack_cap < (size_t)n) {
            if (c->d_stack) CK(cudaFree(c->d_stack));
            c->d_stack = nullptr;
            c->stack_cap = 0;
            if (c->d_stack_maps) CK(cudaFree(c->d_stack_maps));
            c->d_stack_maps = nullptr;
            CK(cudaMalloc(&c->d_stack, (size_t)n * sizeof(ds::StackLayer)));
            CK(cudaMalloc(&c->d_stack_maps, (size_t)n * 2 * sizeof(CUtensorMap)));
            c->stack_cap = n;
        }
        // the down codes as 2-D byte tensors [rows][I * bits / 8]: a unit copies 32-byte columns of
        // 256 rows at a time
        std::vector<CUtensorMap> maps((size_t)n * 2);
        for (int l = 0; l < n; ++l) {
            const ds::StackLayer &s = c->h_stack[l];
            const uint64_t rb = (uint64_t)I * L0->bits / 8;
            encode_2d(&maps[2 * l], CU_TENSOR_MAP_DATA_TYPE_UINT8, s.Dn.packed, rb, (uint64_t)E * D, rb, ds::kDnRowBytes,
                      ds::kDnBox, CU_TENSOR_MAP_SWIZZLE_NONE);
            encode_2d(&maps[2 * l + 1], CU_TENSOR_MAP_DATA_TYPE_UINT8, s.SD.packed, rb, (uint64_t)D, rb, ds::kDnRowBytes,
                      ds::kDnBox, CU_TENSOR_MAP_SWIZZLE_NONE);
        }
        CK(cudaMemcpyAsync(c->d_stack, c->h_stack.data(), (size_t)n * sizeof(ds::StackLayer), cudaMemcpyHostToDevice,
                           c->stream));
        CK(cudaMemcpyAsync(c->d_stack_maps, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice,
                           c->stream));
        CK(cudaStreamSynchronize(c->stream));  // `maps` is pageable host memory
        c->stack_key = key;
    }
    ds::StackParams sp;
    sp.layers = c->d_stack;
    sp.dn_maps = c->d_stack_maps;
    sp.n_layers = n;
    sp.E = E;
    sp.eps = eps;
    sp.x = x;
    sp.h_trace = h_trace;
    sp.ids_trace = ids_trace;
    sp.gen_base = reinterpret_cast<uint32_t *>(c->ll);
    sp.ctr_y = sp.gen_base + 1;
    sp.ctr_logit = sp.gen_base + 2;
    sp.acc = c->ll + 2;
    sp.ll_logit = sp.acc + 2 * (size_t)ds::kAccCopies * D;
    sp.err = c->d_err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c->sms);
    cfg.blockDim = dim3(ds::kThreads);
    cfg.dynamicSmemBytes = ds::layout(D, L0->bits).total;
    cfg.stream = c->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once: they exchange data
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CK(cudaLaunchKernelEx(&cfg, stack_kernel(L0->bits, D), sp));
}

bool kernels_configured = false;
void configure_kernels() {
    if (kernels_configured) return;
    cudaFuncSetAttribute(router_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(router::Smem));
    cudaFuncSetAttribute(gg::grouped_gemm_kernel<gg::MODE_GATE_UP, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         gg::smem_bytes<gg::MODE_GATE_UP>());
    cudaFuncSetAttribute(gg::grouped_gemm_kernel<gg::MODE_GATE_UP, 5>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         gg::smem_bytes<gg::MODE_GATE_UP>());
    cudaFuncSetAttribute(gg::grouped_gemm_kernel<gg::MODE_DOWN, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         gg::smem_bytes<gg::MODE_DOWN>());
    cudaFuncSetAttribute(gg::grouped_gemm_kernel<gg::MODE_DOWN, 5>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         gg::smem_bytes<gg::MODE_DOWN>());
    cudaFuncSetAttribute(gg::grouped_gemm_pair_kernel<gg::MODE_GATE_UP, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         gg::P_SMEM);
    cudaFuncSetAttribute(gg::grouped_gemm_pair_kernel<gg::MODE_GATE_UP, 5>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         gg::P_SMEM);
    cudaFuncSetAttribute(gg::grouped_gemm_pair_kernel<gg::MODE_DOWN, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         gg::P_SMEM);
    cudaFuncSetAttribute(gg::grouped_gemm_pair_kernel<gg::MODE_DOWN, 5>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         gg::P_SMEM);
    cudaFuncSetAttribute(decode_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDecodeSmemMax);
    cudaFuncSetAttribute(ep_reduce_send_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ep_send_smem(2048));
    cudaFuncSetAttribute(decode_ffn_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    cudaFuncSetAttribute(decode_ffn_kernel<5>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    for (int bits : {8, 5})
        for (int D : {512, 1024, 2048})
            cudaFuncSetAttribute(stack_kernel(bits, D), cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    kernels_configured = true;
}

// ------------------------------------------------------------------------ tensor maps

// The driver's tensor-map encoder, resolved once through the runtime (no libcuda link).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    if (!fn) throw CudaFail{"cuTensorMapEncodeTiled is not available from the driver"};
    return fn;
}

// Row-major 2-D map: dim0 contiguous elements, dim1 rows `stride` bytes apart, box b0 x b1.
void encode_2d(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t dim0, uint64_t dim1,
               uint64_t stride, uint32_t b0, uint32_t b1, CUtensorMapSwizzle sw) {
    const cuuint64_t dims[2] = {dim0, dim1};
    const cuuint64_t strides[1] = {stride};
    const cuuint32_t box[2] = {b0, b1};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = tensor_map_encoder()(m, dt, 2, const_cast<void *>(base), dims, strides, box, es,
                                            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw CudaFail{"cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")"};
}

// Grouped-GEMM geometry limits beyond the layer's own: at most 32 scale groups per row (the
// per-unit scale buffer) and 16-byte rows of 5-bit codes for the tensor copies.
const char *grouped_geometry_error(const Layer *L) {
    if (L->D > 2048 || L->I > 2048) return "The grouped path supports hidden and intermediate sizes up to 2048.";
    if (L->bits == 5 && L->I % 128 != 0) return "The 5-bit grouped path needs an intermediate size divisible by 128.";
    return nullptr;
}

// Launch parameters of one grouped GEMM. mode GATE_UP: w = {gate, up, shared gate, shared
// up}, src = the permuted routed rows xp [src_rows, K], shared_src = x [shared_rows, K];
// DOWN: w = {down, down, shared down, shared down}, src = act [src_rows, K].
gg::Params grouped_params(int mode, const QView &w0, const QView &w1, const QView &s0, const QView &s1,
                          const uint16_t *src, int src_rows, const uint16_t *shared_src, int shared_rows,
                          const int32_t *perm, const Tile *tiles,
                          const int32_t *n_tiles, int shared_pos0, int shared_src0, int K, int rows, int E,
                          uint16_t *out, int out_rows, uint32_t *err, bool pair = false) {
    gg::Params p;
    std::memset(&p, 0, sizeof(p));
    const QView ws[4] = {w0, w1, s0, s1};
    const uint32_t rpu = mode == gg::MODE_GATE_UP ? gg::rows_per_unit<gg::MODE_GATE_UP>()
                                                  : gg::rows_per_unit<gg::MODE_DOWN>();
    for (int i = 0; i < 4; ++i) {
        p.w[i] = ws[i];
        const uint64_t row_bytes = (uint64_t)ws[i].cols * ws[i].bits / 8;
        encode_2d(&p.code[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, ws[i].packed, row_bytes,
                  (uint64_t)ws[i].experts * ws[i].rows, row_bytes, 64, rpu, CU_TENSOR_MAP_SWIZZLE_64B);
    }
    // B boxes of 16 << i rows (the single-CTA kernel) or 8 << i (a CTA pair: each CTA loads half a tile)
    const uint32_t box0 = pair ? 8u : 16u;
    for (int i = 0; i < gg::kBoxes; ++i) {
        encode_2d(&p.bmap[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, src, (uint64_t)K, (uint64_t)std::max(src_rows, 1),
                  (uint64_t)K * 2, gg::BK, box0 << i, CU_TENSOR_MAP_SWIZZLE_128B);
        if (shared_src)
            encode_2d(&p.smap[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, shared_src, (uint64_t)K,
                      (uint64_t)std::max(shared_rows, 1), (uint64_t)K * 2, gg::BK, box0 << i, CU_TENSOR_MAP_SWIZZLE_128B);
    }
    p.perm_route = perm;
    p.tiles = tiles;
    p.n_tiles = n_tiles;
    p.shared_pos0 = shared_pos0;
    p.shared_src0 = shared_src0;
    p.K = K;
    p.rows = rows;
    p.E = E;
    if (mode == gg::MODE_DOWN)
        encode_2d(&p.ymap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, out, (uint64_t)rows, (uint64_t)std::max(out_rows, 1),
                  (uint64_t)rows * 2, 32, 16, CU_TENSOR_MAP_SWIZZLE_NONE);
    p.out = out;
    p.err = err;
    return p;
}

template <int MODE>
void launch_grouped(const gg::Params &p, int bits, int grid, cudaStream_t st) {
    // programmatic dependent launch: the CTAs set up barriers and TMEM while the previous kernel
    // drains, then wait for it (pdl_wait) before their first global read
    if (bits == 8) launch(gg::grouped_gemm_kernel<MODE, 8>, dim3(grid), dim3(gg::THREADS), gg::smem_bytes<MODE>(), st, true, p);
    else launch(gg::grouped_gemm_kernel<MODE, 5>, dim3(grid), dim3(gg::THREADS), gg::smem_bytes<MODE>(), st, true, p);
}

// The CTA-pair grouped GEMM: clusters of two CTAs, one per SM of a pair of SMs (grid = the even
// number of SMs at most `sms`); its B maps hold 8 << i-row boxes (grouped_params(..., pair)).
template <int MODE>
void launch_grouped_pair(const gg::Params &p, int bits, int sms, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(sms & ~1));
    cfg.blockDim = dim3(gg::THREADS);
    cfg.dynamicSmemBytes = gg::P_SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (bits == 8) CK(cudaLaunchKernelEx(&cfg, gg::grouped_gemm_pair_kernel<MODE, 8>, p));
    else CK(cudaLaunchKernelEx(&cfg, gg::grouped_gemm_pair_kernel<MODE, 5>, p));
}

// The expert GEMMs of the block run on CTA pairs when DEEPINFER_GROUPED_PAIR=1 (the single-CTA
// kernel otherwise; it also serves the router's and the dense projections' GEMMs).
bool use_pair_gemm() {
    static const bool pair = [] {
        const char *v = std::getenv("DEEPINFER_GROUPED_PAIR");
        return v && std::strcmp(v, "1") == 0;
    }();
    return pair;
}

// ------------------------------------------------------------------------ the block

// Tokens per work unit of the approximate-logit GEMM: 128 rather than 256 gives an 8K-token batch
// twice as many units (128 of them for 256 experts) over the 148 SMs.
constexpr int kRouterTileRows = 128;
struct BlockBuffers {
    uint16_t *x, *y;
    float *logits, *probs, *gate;
    int32_t *ids, *block_counts, *block_base, *seg_count, *seg_off, *n_tiles, *perm, *route_pos;
    Tile *tiles;
    uint16_t *act, *yr, *ys, *xp;
    float *act32;
    float *wn;             // router row norms (tensor-core router): ||r_e||, then ||W_e||
    float *wf;             // the router rows' f32 weights [E][D] (exact candidate logits)
    Tile *rtiles;          // work tiles of the approximate-logit GEMM
    int32_t *rnt;
    uint32_t *counter;  // [0] last-CTA ticket of decode_route_kernel (kept at zero between launches),
                        // [1] grid-barrier arrivals of decode_ffn_kernel (zeroed per call)
    int nblocks, max_tiles;
    bool router_exact;  // grouped path: every router logit in the canonical order (no tensor-core bound)
};

size_t plan_block(Context *c, const Layer *L, int T, Carve &cv, BlockBuffers &b, bool host_io, bool gemv) {
    const int E = L->E, D = L->D, I = L->I;
    b.nblocks = (T + topk::TOK_PER_CTA - 1) / topk::TOK_PER_CTA;
    b.max_tiles = (8 * T + gg::BN - 1) / gg::BN + E + (T + gg::BN - 1) / gg::BN + 1;
    size_t o_x = host_io ? cv.take<uint16_t>((size_t)T * D) : 0;
    size_t o_y = host_io ? cv.take<uint16_t>((size_t)T * D) : 0;
    size_t o_lg = cv.take<float>((size_t)T * E);
    size_t o_p = cv.take<float>((size_t)T * 8);
    size_t o_g = cv.take<float>((size_t)T);
    size_t o_ids = cv.take<int32_t>((size_t)T * 8);
    size_t o_bc = cv.take<int32_t>((size_t)b.nblocks * E);
    size_t o_bb = cv.take<int32_t>((size_t)b.nblocks * E);
    size_t o_sc = cv.take<int32_t>(E + 1);
    size_t o_so = cv.take<int32_t>(E + 1);
    size_t o_nt = cv.take<int32_t>(1);
    size_t o_pm = cv.take<int32_t>((size_t)T * 8);
    size_t o_rp = cv.take<int32_t>((size_t)T * 8);
    size_t o_t = cv.take<Tile>((size_t)b.max_tiles);
    size_t o_a = gemv ? 0 : cv.take<uint16_t>((size_t)T * 9 * I);
    size_t o_yp = gemv ? 0 : cv.take<uint16_t>((size_t)T * 9 * D);  // expert rows by position, shared rows last
    size_t o_xp = gemv ? 0 : cv.take<uint16_t>((size_t)T * 8 * D);
    size_t o_a32 = gemv ? cv.take<float>((size_t)T * 9 * I) : 0;
    size_t o_ctr = cv.take<uint32_t>(2);
    size_t o_wn = cv.take<float>(2 * (size_t)E), o_rt = cv.take<Tile>((size_t)(T + kRouterTileRows - 1) / kRouterTileRows + 1);
    size_t o_rnt = cv.take<int32_t>(1), o_wf = gemv ? 0 : cv.take<float>((size_t)E * D);
    size_t need = cv.off + 256;
    ensure_workspace(c, need);
    b.x = host_io ? at<uint16_t>(c, o_x) : nullptr;
    b.y = host_io ? at<uint16_t>(c, o_y) : nullptr;
    b.logits = at<float>(c, o_lg);
    b.probs = at<float>(c, o_p);
    b.gate = at<float>(c, o_g);
    b.ids = at<int32_t>(c, o_ids);
    b.block_counts = at<int32_t>(c, o_bc);
    b.block_base = at<int32_t>(c, o_bb);
    b.seg_count = at<int32_t>(c, o_sc);
    b.seg_off = at<int32_t>(c, o_so);
    b.n_tiles = at<int32_t>(c, o_nt);
    b.perm = at<int32_t>(c, o_pm);
    b.route_pos = at<int32_t>(c, o_rp);
    b.tiles = at<Tile>(c, o_t);
    b.act = gemv ? nullptr : at<uint16_t>(c, o_a);
    b.yr = gemv ? nullptr : at<uint16_t>(c, o_yp);
    b.ys = gemv ? nullptr : b.yr + (size_t)T * 8 * D;
    b.xp = gemv ? nullptr : at<uint16_t>(c, o_xp);
    b.act32 = gemv ? at<float>(c, o_a32) : nullptr;
    b.counter = at<uint32_t>(c, o_ctr);
    b.wn = at<float>(c, o_wn);
    b.wf = gemv ? nullptr : at<float>(c, o_wf);
    b.rtiles = at<Tile>(c, o_rt);
    b.rnt = at<int32_t>(c, o_rnt);
    return need;
}

// Routing of a prefill-sized batch (E a multiple of 128) in two steps (route.cuh): approximate
// logits on the tensor cores (approx: scratch of T*E bf16) with the router rows' norms, then the
// exact canonical logits of the candidates only -> ids, probs, gate logits, per-block route counts.
// The router rows' norms and f32 weights (router_row_norms_kernel) depend only on the router matrix:
// each layer keeps them and recomputes them when the matrix version changes. A matrix whose device
// buffer was handed out may change unseen, so its norms are computed into the call's scratch
// (ws_wn, ws_wf) every time.
void router_norms(Layer *L, cudaStream_t st, float *ws_wn, float *ws_wf, const float **wn, const float **wf) {
    const int E = L->E, D = L->D;
    Matrix *R = L->m[0];
    if (R->exposed) {
        router_row_norms_kernel<<<(E + 7) / 8, 256, 0, st>>>(R->view(), E, D, ws_wn, ws_wf);
        *wn = ws_wn;
        *wf = ws_wf;
        return;
    }
    if (!L->router_rn) {
        CK(cudaMalloc(&L->router_rn, sizeof(float) * (2 * (size_t)E + (size_t)E * D)));
        L->router_rn_version = 0;
    }
    if (L->router_rn_version != R->version) {
        router_row_norms_kernel<<<(E + 7) / 8, 256, 0, st>>>(R->view(), E, D, L->router_rn, L->router_rn + 2 * E);
        L->router_rn_version = R->version;
    }
    *wn = L->router_rn;
    *wf = L->router_rn + 2 * E;
}
void enqueue_router_approx(const Layer *L, const uint16_t *x, int T, Tile *rtiles, int32_t *rnt, uint16_t *approx,
                           int grid, uint32_t *err, cudaStream_t st) {
    const int E = L->E, D = L->D;
    const QView R = L->m[0]->view();
    launch(router_tiles_kernel, dim3(1), dim3(256), 0, st, true, T, kRouterTileRows, rtiles, rnt);
    launch_grouped<gg::MODE_DOWN>(grouped_params(gg::MODE_DOWN, R, R, R, R, x, T, nullptr, 0, nullptr, rtiles, rnt, T,
                                                 0, D, E, 1, approx, T, err),
                                  8, grid, st);
}
// dsp: the expert-parallel dispatch fused into the router (block_counts may then be null)
void enqueue_router_select(const Layer *L, const uint16_t *x, int T, const int32_t *forced, int32_t *ids,
                           float *probs, float *gate, int32_t *block_counts, int nblocks, const float *wn,
                           const float *wf, const uint16_t *approx, uint32_t *err, cudaStream_t st,
                           const RouterDispatch *dsp = nullptr) {
    const int E = L->E, D = L->D;
    const QView R = L->m[0]->view(), SR = L->m[7]->view();
    if (block_counts) CK(cudaMemsetAsync(block_counts, 0, sizeof(int32_t) * (size_t)nblocks * E, st));
    if (dsp)
        launch(router_select_kernel<true>, dim3((T + 7) / 8), dim3(256), 0, st, true, approx, wn, wf, x, T, E, D, R, SR, L->bias, forced,
                                                                ids, probs, gate, block_counts, err, *dsp);
    else
        launch(router_select_kernel<false>, dim3((T + 7) / 8), dim3(256), 0, st, true, approx, wn, wf, x, T, E, D, R, SR, L->bias, forced,
                                                                 ids, probs, gate, block_counts, err, RouterDispatch{});
}
bool router_tc_fits(const Layer *L) { return L->E % 128 == 0 && L->D <= 2048; }

cudaEvent_t *g_marks = nullptr;  // event array the current enqueue records into
void stage_mark(Context *c, int s) { CK(cudaEventRecord(g_marks ? g_marks[s] : c->ev_stage[s], c->stream)); }

// Enqueue the block on the context stream. x/y/ids/probs are device pointers; resid (f32)
// optional. forced: ids holds input routes. Returns nothing; errors surface via d_err.
// Stack mode (decode path only): `x` is the bf16 scratch row that decode_route_kernel fills from
// the f32 residual `resid` normalised by `norm_w`; otherwise `x` is the block input.
// Grouped stacks: next_norm (the next layer's RMSNorm weights) makes the combine also write the
// next layer's input row to next_h (and next_trace).
void enqueue_block(Context *c, const Layer *L, const uint16_t *x, int T, uint16_t *y, float *resid,
                   const int32_t *forced_ids, float *probs_out, bool gemv, BlockBuffers &b, bool profile,
                   const float *norm_w = nullptr, float eps = 0.f, uint16_t *h_trace = nullptr,
                   const float *next_norm = nullptr, uint16_t *next_h = nullptr, uint16_t *next_trace = nullptr,
                   uint32_t gen = 1) {
    const int E = L->E, D = L->D, I = L->I;
    cudaStream_t st = c->stream;
    const QView R = L->m[0]->view(), G = L->m[1]->view(), U = L->m[2]->view(), Dn = L->m[3]->view();
    const QView SG = L->m[4]->view(), SU = L->m[5]->view(), SD = L->m[6]->view(), SR = L->m[7]->view();
    int32_t *ids = b.ids;  // sanitised ids; every later kernel indexes with these
    float *probs = probs_out ? probs_out : b.probs;
    if (profile) stage_mark(c, S_ROUTER);
    if (gemv && !forced_ids) {
        // decode path: three kernels chained with programmatic dependent launch
        const bool stacked = norm_w != nullptr;
        launch(decode_route_kernel, dim3((E + 7) / 8), dim3(256), (size_t)T * D * 2, st, true,
               stacked ? (const float *)resid : nullptr, norm_w, eps, stacked ? nullptr : x, T, D, R, SR,
               (const float *)L->bias, stacked ? const_cast<uint16_t *>(x) : nullptr, h_trace, b.logits, ids, probs,
               b.gate, b.counter, c->d_err);
        if (profile) {
            stage_mark(c, S_TOPK);
            stage_mark(c, S_SCAN);
            stage_mark(c, S_SCATTER);
            stage_mark(c, S_GATE_UP);
        }
        if (T == 1 && ffn_fits(c, L)) {
            // one token: the fused gate/up + down kernel (one CTA per SM, weights staged in smem);
            // its CTAs meet at a grid barrier, so it is launched cooperatively
            const FfnLayout f = ffn_layout(D, I, L->bits, c->sms);
            if (L->bits == 8)
                launch_cooperative(decode_ffn_kernel<8>, dim3(c->sms), dim3(kFfnThreads), (size_t)f.total, st,
                                   (const uint16_t *)x, D, I, G, U, SG, SU, Dn, SD, (const int32_t *)ids,
                                   (const float *)probs, (const float *)b.gate, b.act32, y, stacked ? resid : nullptr,
                                   b.counter + 1, gen, c->d_err);
            else
                launch_cooperative(decode_ffn_kernel<5>, dim3(c->sms), dim3(kFfnThreads), (size_t)f.total, st,
                                   (const uint16_t *)x, D, I, G, U, SG, SU, Dn, SD, (const int32_t *)ids,
                                   (const float *)probs, (const float *)b.gate, b.act32, y, stacked ? resid : nullptr,
                                   b.counter + 1, gen, c->d_err);
            if (profile) {
                stage_mark(c, S_DOWN);
                stage_mark(c, S_COMBINE);
                stage_mark(c, S_N);
            }
            return;
        }
        const int gw = T * 9 * I;
        if (L->bits == 8)
            launch(decode_gate_up_kernel<8>, dim3(gw / 8), dim3(256), (size_t)D * 2, st, true, x, T, D, I, G, U, SG, SU,
                   (const int32_t *)ids, b.act32);
        else
            launch(decode_gate_up_kernel<5>, dim3(gw / 8), dim3(256), (size_t)D * 2, st, true, x, T, D, I, G, U, SG, SU,
                   (const int32_t *)ids, b.act32);
        if (profile) stage_mark(c, S_DOWN);
        const int dw = T * D;
        if (L->bits == 8)
            launch(decode_down_kernel<8>, dim3((dw + 7) / 8), dim3(256), 0, st, true, (const float *)b.act32, T, D, I,
                   Dn, SD, (const int32_t *)ids, (const float *)probs, (const float *)b.gate, y, stacked ? resid : nullptr,
                   (const uint32_t *)c->d_err);
        else
            launch(decode_down_kernel<5>, dim3((dw + 7) / 8), dim3(256), 0, st, true, (const float *)b.act32, T, D, I,
                   Dn, SD, (const int32_t *)ids, (const float *)probs, (const float *)b.gate, y, stacked ? resid : nullptr,
                   (const uint32_t *)c->d_err);
        if (profile) {
            stage_mark(c, S_COMBINE);
            stage_mark(c, S_N);
        }
        return;
    }
    // 1-2. router logits, top-8, probabilities, shared gate logit, per-block expert counts
    if (!gemv && router_tc_fits(L) && !b.router_exact) {
        // tensor-core approximate logits + exact canonical logits of the candidates
        uint16_t *approx = reinterpret_cast<uint16_t *>(b.logits);
        const float *wn = nullptr, *wf = nullptr;
        router_norms(const_cast<Layer *>(L), st, b.wn, b.wf, &wn, &wf);
        enqueue_router_approx(L, x, T, b.rtiles, b.rnt, approx, c->sms, c->d_err, st);
        if (profile) stage_mark(c, S_TOPK);
        enqueue_router_select(L, x, T, forced_ids, ids, probs, b.gate, b.block_counts, b.nblocks, wn, wf, approx,
                              c->d_err, st);
    } else {
        // every logit in the canonical f32 order
        if (gemv) {
            router_logits_gemv_kernel<<<(E * 32 + 255) / 256, 256, 0, st>>>(x, T, D, R, L->bias, b.logits);
        } else {
            dim3 grid((T + router::TT - 1) / router::TT, (E + router::TE - 1) / router::TE);
            router_logits_kernel<<<grid, router::THREADS, sizeof(router::Smem), st>>>(x, T, D, R, L->bias, b.logits);
        }
        if (profile) stage_mark(c, S_TOPK);
        topk_count_kernel<<<b.nblocks, topk::WARPS * 32, 0, st>>>(b.logits, T, E, x, D, SR, forced_ids, ids, probs,
                                                                   b.gate, b.block_counts, c->d_err);
    }
    if (gemv) {
        if (profile) {
            stage_mark(c, S_SCAN);
            stage_mark(c, S_SCATTER);
            stage_mark(c, S_GATE_UP);
        }
        const int warps = T * 9 * I;
        const size_t xs = (size_t)D * sizeof(uint16_t);
        if (L->bits == 8)
            decode_gate_up_kernel<8><<<warps / 8, 256, xs, st>>>(x, T, D, I, G, U, SG, SU, ids, b.act32);
        else
            decode_gate_up_kernel<5><<<warps / 8, 256, xs, st>>>(x, T, D, I, G, U, SG, SU, ids, b.act32);
        if (profile) stage_mark(c, S_DOWN);
        const int dw = T * D;
        if (L->bits == 8)
            decode_down_kernel<8><<<(dw + 7) / 8, 256, 0, st>>>(b.act32, T, D, I, Dn, SD, ids, probs, b.gate, y, resid,
                                                               c->d_err);
        else
            decode_down_kernel<5><<<(dw + 7) / 8, 256, 0, st>>>(b.act32, T, D, I, Dn, SD, ids, probs, b.gate, y, resid,
                                                               c->d_err);
        if (profile) stage_mark(c, S_COMBINE);
        if (profile) stage_mark(c, S_N);
        return;
    }
    if (profile) stage_mark(c, S_SCAN);
    // 3. scan counts, segment offsets, GEMM tile list
    launch(scan_tiles_kernel, dim3(1), dim3(1024), 0, st, true, b.block_counts, b.nblocks, E, E, T, T, gg::BN, b.block_base, b.seg_count,
                                          b.seg_off, b.tiles, b.n_tiles, b.max_tiles, c->d_err);
    if (profile) stage_mark(c, S_SCATTER);
    // 4. stable scatter of routes into expert-grouped order
    // ... and the token rows copied into that order for the gate/up B operand
    // four CTAs per 64-token block share its row copies (measured: 2.26 ms/step against 2.56 for one)
    launch(scatter_permute_kernel<4>, dim3(b.nblocks * 4), dim3(kScatterWarps * 32), 0, st, true, 
        ids, T, E, b.block_base, b.seg_off, b.perm, b.route_pos, x, D, b.xp, E);
    c->last_perm = b.perm;
    c->last_seg_off = b.seg_off;
    c->last_seg_count = b.seg_count;
    c->last_routes_T = T;
    c->last_routes_E = E;
    if (profile) stage_mark(c, S_GATE_UP);
    // 5. grouped gate/up + SwiGLU (routed experts and the shared expert)
    const int grid = c->sms;
    const bool pair = use_pair_gemm();
    const gg::Params pgu = grouped_params(gg::MODE_GATE_UP, G, U, SG, SU, b.xp, 8 * T, x, T, b.perm, b.tiles,
                                         b.n_tiles, 8 * T, 0, D, I, E, b.act, 9 * T, c->d_err, pair);
    if (pair) launch_grouped_pair<gg::MODE_GATE_UP>(pgu, L->bits, grid, st);
    else launch_grouped<gg::MODE_GATE_UP>(pgu, L->bits, grid, st);
    if (profile) stage_mark(c, S_DOWN);
    // 6. grouped down -> expert rows in route order, shared rows
    const gg::Params pdn = grouped_params(gg::MODE_DOWN, Dn, Dn, SD, SD, b.act, 9 * T, nullptr, 0, b.perm, b.tiles,
                                         b.n_tiles, 8 * T, 0, I, D, E, b.yr, 9 * T, c->d_err, pair);
    if (pair) launch_grouped_pair<gg::MODE_DOWN>(pdn, L->bits, grid, st);
    else launch_grouped<gg::MODE_DOWN>(pdn, L->bits, grid, st);
    if (profile) stage_mark(c, S_COMBINE);
    // 7. combine (stacks: fused with the residual update and the next layer's RMSNorm)
    if (resid && !y) {
        launch(combine_norm_kernel<128>, dim3(T), dim3(128), 0, st, true, b.yr, b.route_pos, b.ys, b.gate, probs, D, resid, next_norm, eps, next_h,
                                               next_trace, c->d_err);
    } else {
        const size_t n = (size_t)T * (D / 8);
        launch(combine_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, true, b.yr, b.route_pos, b.ys, b.gate, probs, T, D, y, resid,
                                                                     c->d_err);
    }
    if (profile) stage_mark(c, S_N);
}

const char *device_error_text(uint32_t e) {
    if (e & kErrNonFinite) return "Non-finite router logits.";
    if (e & kErrBadExpert) return "Expert ID out of bounds";
    if (e & kErrTimeout) return "Device wait timed out";
    if (e & kErrRange) return "Decode output outside the fixed-point accumulator's range";
    return "Internal work list overflow";
}

bool env_flag(const char *name) {
    const char *v = std::getenv(name);
    return v && std::strcmp(v, "1") == 0;
}

}  // namespace

// ============================================================================ Part 1

API int di_abi_version(void) { return DI_ABI_VERSION; }

API void *di_quant_create_configured(int resident, int refresh_ms, char *error, int capacity) {
    if ((resident != 0 && resident != 1) || refresh_ms < 0 || refresh_ms > 60000) {
        set_error(error, capacity, "Invalid residency configuration");
        return nullptr;
    }
    int dev = 0, count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count < 1) {
        cudaGetLastError();
        set_error(error, capacity, "No CUDA device");
        return nullptr;
    }
    cudaGetDevice(&dev);
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
        set_error(error, capacity, "Cannot query CUDA device");
        return nullptr;
    }
    if (prop.major != 10 || prop.minor != 0) {
        set_error(error, capacity, "deepinfer_cuda requires an sm_100 (B200) device, found sm_%d%d", prop.major,
                  prop.minor);
        return nullptr;
    }
    Context *c = new Context();
    c->device = dev;
    c->sms = prop.multiProcessorCount;
    c->resident = resident == 1;
    c->refresh_ms = refresh_ms;
    try {
        CK(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
        CK(cudaEventCreate(&c->ev_start));
        CK(cudaEventCreate(&c->ev_stop));
        for (int i = 0; i <= S_N; ++i) CK(cudaEventCreate(&c->ev_stage[i]));
        CK(cudaMalloc(&c->d_err, sizeof(uint32_t)));
        CK(cudaMallocHost(&c->h_err, sizeof(uint32_t)));
        configure_kernels();
    } catch (const CudaFail &f) {
        set_error(error, capacity, "%s", f.what.c_str());
        delete c;
        return nullptr;
    }
    std::lock_guard<std::mutex> g(g_registry);
    g_contexts.insert(c);
    return c;
}

API void *di_quant_create(char *error, int capacity) {
    const char *v = std::getenv("DEEPINFER_CUDA_RESIDENCY_REFRESH_MS");
    return di_quant_create_configured(env_flag("DEEPINFER_CUDA_RESIDENCY") ? 1 : 0, v ? std::atoi(v) : 1000, error,
                                      capacity);
}

API void di_quant_destroy(void *p) {
    if (!live_context(p)) return;
    Context *c = static_cast<Context *>(p);
    {
        std::lock_guard<std::mutex> g(g_registry);
        g_contexts.erase(c);
    }
    DeviceGuard dg(c->device);
    cudaStreamSynchronize(c->stream);
    // matrices still alive keep their memory until their own destroy; detach them
    if (c->ws.base) cudaFree(c->ws.base);
    if (c->d_err) cudaFree(c->d_err);
    if (c->h_err) cudaFreeHost(c->h_err);
    for (int i = 0; i <= S_N; ++i)
        if (c->ev_stage[i]) cudaEventDestroy(c->ev_stage[i]);
    for (cudaEvent_t e : c->layer_events) cudaEventDestroy(e);
    if (c->graph_exec) cudaGraphExecDestroy(c->graph_exec);
    if (c->ll) cudaFree(c->ll);
    if (c->d_stack) cudaFree(c->d_stack);
    if (c->d_stack_maps) cudaFree(c->d_stack_maps);
    if (c->ev_start) cudaEventDestroy(c->ev_start);
    if (c->ev_stop) cudaEventDestroy(c->ev_stop);
    if (c->stream) cudaStreamDestroy(c->stream);
    // Context memory is intentionally kept while matrices reference it.
    if (c->matrices.empty()) delete c;
}

API uint64_t di_quant_residency_bytes(void *p) {
    if (!live_context(p)) return 0;
    Context *c = static_cast<Context *>(p);
    if (!c->resident) return 0;
    uint64_t total = 0;
    for (Matrix *m : c->matrices)
        if (!m->destroyed) total += m->bytes[0] + m->bytes[1] + m->bytes[2];
    return total;
}

API void di_quant_residency_prepare(void *p) {
    if (!live_context(p)) return;
    Context *c = static_cast<Context *>(p);
    DeviceGuard dg(c->device);
    try {
        for (Matrix *m : c->matrices)
            if (!m->destroyed) sync_matrix(m);
        CK(cudaStreamSynchronize(c->stream));
    } catch (const CudaFail &) {
    }
}

API void *di_quant_matrix_create(void *ctx, int experts, int rows, int columns, int bits, int group, char *error,
                                 int capacity) {
    if (!live_context(ctx) || experts < 1 || experts > 256 || rows < 1 || columns < 64 || (bits != 5 && bits != 8) ||
        group != 64 || columns % 64) {
        set_error(error, capacity, "Unsupported quantized matrix shape");
        return nullptr;
    }
    Context *c = static_cast<Context *>(ctx);
    DeviceGuard dg(c->device);
    Matrix *m = new Matrix();
    m->ctx = c;
    m->experts = experts;
    m->rows = rows;
    m->cols = columns;
    m->bits = bits;
    const size_t nrow = (size_t)experts * rows;
    m->bytes[0] = nrow * columns * bits / 8;
    m->bytes[1] = m->bytes[2] = nrow * (columns / 64) * 2;
    for (int i = 0; i < 3; ++i) {
        // +16 bytes of slack so vector loads of the last row stay inside the allocation
        if (cudaMalloc(&m->d[i], m->bytes[i] + 16) != cudaSuccess) {
            cudaGetLastError();
            for (int j = 0; j < i; ++j) cudaFree(m->d[j]);
            delete m;
            set_error(error, capacity, "Quantized buffer allocation failed");
            return nullptr;
        }
        cudaMemsetAsync(m->d[i], 0, m->bytes[i] + 16, c->stream);
    }
    c->matrices.insert(m);
    std::lock_guard<std::mutex> g(g_registry);
    g_matrices.insert(m);
    return m;
}

API void *di_quant_matrix_buffer(void *matrix, int index) {
    if (!live_matrix(matrix) || index < 0 || index > 2) return nullptr;
    Matrix *m = static_cast<Matrix *>(matrix);
    DeviceGuard dg(m->ctx->device);
    if (!m->h[index]) {
        if (cudaMallocHost(&m->h[index], m->bytes[index]) != cudaSuccess) {
            cudaGetLastError();
            m->h[index] = nullptr;
            return nullptr;
        }
        // the staging copy starts as the current device contents
        if (cudaMemcpy(m->h[index], m->d[index], m->bytes[index], cudaMemcpyDeviceToHost) != cudaSuccess) {
            cudaGetLastError();
            cudaFreeHost(m->h[index]);
            m->h[index] = nullptr;
            return nullptr;
        }
    }
    m->dirty[index] = true;
    return m->h[index];
}

API void *di_quant_matrix_device_buffer(void *matrix, int index) {
    if (!live_matrix(matrix) || index < 0 || index > 2) return nullptr;
    static_cast<Matrix *>(matrix)->exposed = true;
    return static_cast<Matrix *>(matrix)->d[index];
}

API int di_quant_matrix_upload(void *matrix, int index, const void *src, uint64_t bytes, char *error, int capacity) {
    if (!live_matrix(matrix) || index < 0 || index > 2 || !src) {
        set_error(error, capacity, "Invalid quantized buffer upload");
        return -1;
    }
    Matrix *m = static_cast<Matrix *>(matrix);
    if (bytes != m->bytes[index]) {
        set_error(error, capacity, "Quantized buffer length mismatch.");
        return -1;
    }
    DeviceGuard dg(m->ctx->device);
    try {
        CK(cudaMemcpyAsync(m->d[index], src, bytes, cudaMemcpyHostToDevice, m->ctx->stream));
        CK(cudaStreamSynchronize(m->ctx->stream));
        if (m->h[index]) std::memcpy(m->h[index], src, bytes);
        m->dirty[index] = false;
        m->version++;
    } catch (const CudaFail &f) {
        set_error(error, capacity, "%s", f.what.c_str());
        return -1;
    }
    return 0;
}

API int di_quant_matrix_generate(void *matrix, uint64_t seed, uint64_t stream, float stddev, int first_expert,
                                 char *error, int capacity) {
    if (!live_matrix(matrix) || !(stddev > 0.0f) || first_expert < 0) {
        set_error(error, capacity, "Invalid synthetic weight request");
        return -1;
    }
    Matrix *m = static_cast<Matrix *>(matrix);
    DeviceGuard dg(m->ctx->device);
    try {
        const int64_t rows = (int64_t)m->experts * m->rows;
        const int64_t groups = rows * (m->cols / 64);
        const float scale = (1.7320508075688772f / 65536.0f) * stddev;
        gen_quant_kernel<<<(unsigned)((groups + 127) / 128), 128, 0, m->ctx->stream>>>(
            stream_base(seed, stream), scale, rows, (int64_t)first_expert * m->rows, m->cols, m->bits,
            (uint32_t *)m->d[0], (uint16_t *)m->d[1], (uint16_t *)m->d[2]);
        CK(cudaGetLastError());
        CK(cudaStreamSynchronize(m->ctx->stream));
        for (int i = 0; i < 3; ++i) {
            m->dirty[i] = false;
            if (m->h[i]) CK(cudaMemcpy(m->h[i], m->d[i], m->bytes[i], cudaMemcpyDeviceToHost));
        }
        m->version++;
    } catch (const CudaFail &f) {
        set_error(error, capacity, "%s", f.what.c_str());
        return -1;
    }
    return 0;
}

API void di_quant_matrix_destroy(void *matrix) {
    if (!live_matrix(matrix)) return;
    Matrix *m = static_cast<Matrix *>(matrix);
    m->destroyed = true;
    Context *c = m->ctx;
    DeviceGuard dg(c->device);
    cudaStreamSynchronize(c->stream);
    release_matrix(m);
}

API int di_quant_batch(void *ctx, const di_quant_job *jobs, int count, double *ms, char *error, int capacity) {
    if (!live_context(ctx) || !jobs || count < 1 || count > 8) {
        set_error(error, capacity, "Invalid GEMV batch");
        return -1;
    }
    Context *c = static_cast<Context *>(ctx);
    for (int j = 0; j < count; ++j) {
        const di_quant_job &job = jobs[j];
        if (!live_matrix(job.matrix) || !job.input || !job.output || !job.experts || job.count < 1 || job.count > 8) {
            set_error(error, capacity, "Invalid quantized GEMV arguments");
            return -1;
        }
        Matrix *m = static_cast<Matrix *>(job.matrix);
        if (m->ctx != c) {
            set_error(error, capacity, "Batch matrices must belong to this device.");
            return -1;
        }
        for (int i = 0; i < job.count; ++i)
            if (job.experts[i] >= (uint32_t)m->experts) {
                set_error(error, capacity, "Expert ID out of bounds");
                return -1;
            }
        for (int i = 0; i < j; ++i)
            if (jobs[i].matrix == job.matrix) {
                set_error(error, capacity, "Batch matrices must be distinct");
                return -1;
            }
    }
    DeviceGuard dg(c->device);
    try {
        Carve cv;
        std::vector<size_t> o_in(count), o_out(count), o_ex(count);
        for (int j = 0; j < count; ++j) {
            const Matrix *m = static_cast<Matrix *>(jobs[j].matrix);
            o_in[j] = cv.take<float>((size_t)m->cols * (jobs[j].batched ? jobs[j].count : 1));
            o_out[j] = cv.take<float>((size_t)m->rows * jobs[j].count);
            o_ex[j] = cv.take<uint32_t>(8);
        }
        size_t o_jobs = cv.take<GemvJob>(8);
        ensure_workspace(c, cv.off + 256);
        std::vector<GemvJob> hj(count);
        int max_warps = 0;
        for (int j = 0; j < count; ++j) {
            Matrix *m = static_cast<Matrix *>(jobs[j].matrix);
            sync_matrix(m);
            const size_t nin = (size_t)m->cols * (jobs[j].batched ? jobs[j].count : 1);
            CK(cudaMemcpyAsync(at<float>(c, o_in[j]), jobs[j].input, nin * 4, cudaMemcpyHostToDevice, c->stream));
            CK(cudaMemcpyAsync(at<uint32_t>(c, o_ex[j]), jobs[j].experts, jobs[j].count * 4, cudaMemcpyHostToDevice,
                               c->stream));
            hj[j] = GemvJob{m->view(), at<float>(c, o_in[j]), at<float>(c, o_out[j]), at<uint32_t>(c, o_ex[j]),
                            jobs[j].count, jobs[j].batched ? 1 : 0};
            max_warps = std::max(max_warps, m->rows * jobs[j].count);
        }
        CK(cudaMemcpyAsync(at<GemvJob>(c, o_jobs), hj.data(), sizeof(GemvJob) * count, cudaMemcpyHostToDevice,
                           c->stream));
        CK(cudaEventRecord(c->ev_start, c->stream));
        quant_gemv_kernel<<<dim3((max_warps + 7) / 8, count), 256, 0, c->stream>>>(at<GemvJob>(c, o_jobs));
        if (launch_check(error, capacity)) return -1;
        CK(cudaEventRecord(c->ev_stop, c->stream));
        for (int j = 0; j < count; ++j) {
            const Matrix *m = static_cast<Matrix *>(jobs[j].matrix);
            CK(cudaMemcpyAsync(jobs[j].output, at<float>(c, o_out[j]), (size_t)m->rows * jobs[j].count * 4,
                               cudaMemcpyDeviceToHost, c->stream));
        }
        CK(cudaStreamSynchronize(c->stream));
        float t = 0;
        CK(cudaEventElapsedTime(&t, c->ev_start, c->ev_stop));
        if (ms) *ms = t;
    } catch (const CudaFail &f) {
        set_error(error, capacity, "%s", f.what.c_str());
        return -1;
    }
    return 0;
}

API int di_quant_matvec(void *ctx, void *matrix, const float *x, float *y, const uint32_t *experts, int count,
                        int batched, double *ms, char *error, int capacity) {
    di_quant_job job{matrix, x, y, experts, count, batched};
    return di_quant_batch(ctx, &job, 1, ms, error, capacity);
}

API int di_quant_experts(void *ctx, void *gate, void *up, void *down, void *shared, const float *input,
                         const float *shared_input, const uint32_t *experts, int count, float *expert_output,
                         float *shared_output, double *ms, char *error, int capacity) {
    // quantized.mm:354-361 checks, plus context ownership
    Matrix *g = live_matrix(gate) ? static_cast<Matrix *>(gate) : nullptr;
    Matrix *u = live_matrix(up) ? static_cast<Matrix *>(up) : nullptr;
    Matrix *d = live_matrix(down) ? static_cast<Matrix *>(down) : nullptr;
    Matrix *s = live_matrix(shared) ? static_cast<Matrix *>(shared) : nullptr;
    if (!live_context(ctx) || !g || !u || !d || !s || !input || !shared_input || !experts || !expert_output ||
        !shared_output || count < 1 || count > 8 || g == u || g == d || g == s || u == d || u == s || d == s ||
        g->rows != u->rows || g->cols != u->cols || g->experts != u->experts || g->bits != u->bits ||
        d->experts != g->experts || d->cols != g->rows || d->rows != g->cols || s->experts != 1 ||
        s->rows != d->rows) {
        set_error(error, capacity, "Incompatible fused expert matrices/arguments");
        return -1;
    }
    Context *c = static_cast<Context *>(ctx);
    if (g->ctx != c || u->ctx != c || d->ctx != c || s->ctx != c) {
        set_error(error, capacity, "Expert matrices must belong to this device.");
        return -1;
    }
    for (int i = 0; i < count; ++i)
        if (experts[i] >= (uint32_t)g->experts) {
            set_error(error, capacity, "Expert ID out of bounds");
            return -1;
        }
    DeviceGuard dg(c->device);
    try {
        Carve cv;
        size_t o_x = cv.take<float>(g->cols), o_sx = cv.take<float>(s->cols), o_ex = cv.take<uint32_t>(8);
        size_t o_act = cv.take<float>((size_t)g->rows * count), o_y = cv.take<float>((size_t)d->rows * count);
        size_t o_sy = cv.take<float>(s->rows), o_jobs = cv.take<GemvJob>(2), o_zero = cv.take<uint32_t>(1);
        ensure_workspace(c, cv.off + 256);
        for (Matrix *m : {g, u, d, s}) sync_matrix(m);
        CK(cudaMemcpyAsync(at<float>(c, o_x), input, (size_t)g->cols * 4, cudaMemcpyHostToDevice, c->stream));
        CK(cudaMemcpyAsync(at<float>(c, o_sx), shared_input, (size_t)s->cols * 4, cudaMemcpyHostToDevice, c->stream));
        CK(cudaMemcpyAsync(at<uint32_t>(c, o_ex), experts, (size_t)count * 4, cudaMemcpyHostToDevice, c->stream));
        GemvJob hj[2] = {
            GemvJob{d->view(), at<float>(c, o_act), at<float>(c, o_y), at<uint32_t>(c, o_ex), count, 1},
            GemvJob{s->view(), at<float>(c, o_sx), at<float>(c, o_sy), at<uint32_t>(c, o_zero), 1, 0}};
        CK(cudaMemsetAsync(at<uint32_t>(c, o_zero), 0, 4, c->stream));
        CK(cudaMemcpyAsync(at<GemvJob>(c, o_jobs), hj, sizeof(hj), cudaMemcpyHostToDevice, c->stream));
        CK(cudaEventRecord(c->ev_start, c->stream));
        quant_gate_up_kernel<<<(g->rows * count + 7) / 8, 256, 0, c->stream>>>(g->view(), u->view(), at<float>(c, o_x),
                                                                              at<uint32_t>(c, o_ex), count,
                                                                              at<float>(c, o_act));
        const int warps = std::max(d->rows * count, s->rows);
        quant_gemv_kernel<<<dim3((warps + 7) / 8, 2), 256, 0, c->stream>>>(at<GemvJob>(c, o_jobs));
        if (launch_check(error, capacity)) return -1;
        CK(cudaEventRecord(c->ev_stop, c->stream));
        CK(cudaMemcpyAsync(expert_output, at<float>(c, o_y), (size_t)d->rows * count * 4, cudaMemcpyDeviceToHost,
                           c->stream));
        CK(cudaMemcpyAsync(shared_output, at<float>(c, o_sy), (size_t)s->rows * 4, cudaMemcpyDeviceToHost, c->stream));
        CK(cudaStreamSynchronize(c->stream));
        float t = 0;
        CK(cudaEventElapsedTime(&t, c->ev_start, c->ev_stop));
        if (ms) *ms = t;
    } catch (const CudaFail &f) {
        set_error(error, capacity, "%s", f.what.c_str());
        return -1;
    }
    return 0;
}

API int di_quant_embedding(void *matrix, int token, float *out) {
    if (!live_matrix(matrix) || !out) return -1;
    Matrix *m = static_cast<Matrix *>(matrix);
    if (token < 0 || token >= m->rows || m->experts != 1) return -1;
    Context *c = m->ctx;
    DeviceGuard dg(c->device);
    try {
        Carve cv;
        size_t o = cv.take<float>(m->cols);
        ensure_workspace(c, cv.off + 256);
        sync_matrix(m);
        embedding_kernel<<<(m->cols + 255) / 256, 256, 0, c->stream>>>(m->view(), token, at<float>(c, o));
        CK(cudaGetLastError());
        CK(cudaMemcpyAsync(out, at<float>(c, o), (size_t)m->cols * 4, cudaMemcpyDeviceToHost, c->stream));
        CK(cudaStreamSynchronize(c->stream));
    } catch (const CudaFail &) {
        return -1;
    }
    return 0;
}

API int di_quant_gemm(void *ctx, void *matrix, int expert, const uint16_t *x, int tokens, uint16_t *y, int flags,
                      double *ms, char *error, int capacity) {
    if (!live_context(ctx) || !live_matrix(matrix)) {
        set_error(error, capacity, "Invalid context or quantized matrix");
        return -1;
    }
    Context *c = static_cast<Context *>(ctx);
    Matrix *m = static_cast<Matrix *>(matrix);
    const bool dev_io = flags & DI_MOE_DEVICE_IO;
    if (m->ctx != c) {
        set_error(error, capacity, "Quantized matrix must belong to this device.");
        return -1;
    }
    if (!x || !y || tokens < 1 || tokens > 1048576 || (flags & ~DI_MOE_DEVICE_IO)) {
        set_error(error, capacity, "Invalid quantized GEMM arguments");
        return -1;
    }
    if (expert < 0 || expert >= m->experts) {
        set_error(error, capacity, "Expert ID out of bounds");
        return -1;
    }
    // the GEMM kernel's limits: at most 32 scale groups per row (its per-unit scale buffer),
    // 16-byte rows of codes and of output for the tensor copies
    if (m->cols > 2048 || m->rows % 8 || (m->bits == 5 && m->cols % 128)) {
        set_error(error, capacity,
                  "Unsupported quantized GEMM shape: columns <= 2048 (a multiple of 128 for 5-bit), rows a multiple of 8");
        return -1;
    }
    if (dev_io && !device_pointers_ok(c->device, {x, y})) {
        set_error(error, capacity, "With DI_MOE_DEVICE_IO, x and y must be device memory of the context's GPU");
        return -1;
    }
    const int T = tokens, K = m->cols, N = m->rows;
    DeviceGuard dg(c->device);
    try {
        sync_matrix(m);
        Carve cv;
        const size_t o_x = dev_io ? 0 : cv.take<uint16_t>((size_t)T * K);
        const size_t o_y = dev_io ? 0 : cv.take<uint16_t>((size_t)T * N);
        const size_t o_t = cv.take<Tile>((size_t)(T + 255) / 256 + 1), o_nt = cv.take<int32_t>(1);
        ensure_workspace(c, cv.off + 256);
        const uint16_t *dx = dev_io ? x : at<uint16_t>(c, o_x);
        uint16_t *dy = dev_io ? y : at<uint16_t>(c, o_y);
        QView w = m->view();  // the chosen expert as a one-expert matrix
        w.packed += (size_t)expert * N * w.words_per_row();
        w.scales += (size_t)expert * N * w.groups_per_row();
        w.biases += (size_t)expert * N * w.groups_per_row();
        w.experts = 1;
        CK(cudaMemsetAsync(c->d_err, 0, sizeof(uint32_t), c->stream));
        CK(cudaEventRecord(c->ev_start, c->stream));
        if (!dev_io) CK(cudaMemcpyAsync(const_cast<uint16_t *>(dx), x, (size_t)T * K * 2, cudaMemcpyHostToDevice, c->stream));
        launch(router_tiles_kernel, dim3(1), dim3(256), 0, c->stream, true, T, 256, at<Tile>(c, o_t), at<int32_t>(c, o_nt));
        launch_grouped<gg::MODE_DOWN>(grouped_params(gg::MODE_DOWN, w, w, w, w, dx, T, nullptr, 0, nullptr,
                                                     at<Tile>(c, o_t), at<int32_t>(c, o_nt), T, 0, K, N, 1, dy, T,
                                                     c->d_err),
                                      m->bits, c->sms, c->stream);
        if (launch_check(error, capacity)) return -1;
        CK(cudaMemcpyAsync(c->h_err, c->d_err, sizeof(uint32_t), cudaMemcpyDeviceToHost, c->stream));
        if (dev_io) CK(cudaEventRecord(c->ev_stop, c->stream));
        CK(cudaStreamSynchronize(c->stream));
        if (*c->h_err) {
            set_error(error, capacity, "%s", device_error_text(*c->h_err));
            return -1;
        }
        if (!dev_io) {
            CK(cudaMemcpyAsync(y, dy, (size_t)T * N * 2, cudaMemcpyDeviceToHost, c->stream));
            CK(cudaEventRecord(c->ev_stop, c->stream));
            CK(cudaStreamSynchronize(c->stream));
        }
        float t = 0;
        CK(cudaEventElapsedTime(&t, c->ev_start, c->ev_stop));
        if (ms) *ms = t;
    } catch (const CudaFail &f) {
        set_error(error, capacity, "%s", f.what.c_str());
        return -1;
    }
    return 0;
}

// ============================================================================ Part 2

API void *di_moe_layer_create(void *ctx, void *router, void *gate, void *up, void *down, void *shared_gate,
                              void *shared_up, void *shared_down, void *shared_route, char *error, int capacity) {
    void *ptrs[8] = {router, gate, up, down, shared_gate, shared_up, shared_down, shared_route};
    if (!live_context(ctx)) {
        set_error(error, capacity, "Invalid context");
        return nullptr;
    }
    Context *c = static_cast<Context *>(ctx);
    Matrix *m[8];
    for (int i = 0; i < 8; ++i) {
        if (!live_matrix(ptrs[i])) {
            set_error(error, capacity, "MoE layer matrix %d is missing or destroyed", i);
            return nullptr;
        }
        m[i] = static_cast<Matrix *>(ptrs[i]);
        if (m[i]->ctx != c) {
            set_error(error, capacity, "MoE layer matrices must belong to this device.");
            return nullptr;
        }
        for (int j = 0; j < i; ++j)
            if (m[j] == m[i]) {
                set_error(error, capacity, "MoE layer matrices must be distinct.");
                return nullptr;
            }
    }
    const int E = m[0]->rows, D = m[0]->cols, I = m[1]->rows, bits = m[1]->bits;
    auto shape = [](Matrix *x, int e, int r, int col) { return x->experts == e && x->rows == r && x->cols == col; };
    bool okg = m[0]->experts == 1 && m[0]->bits == 8 && E >= 8 && E <= 256 && D % 256 == 0 && I % 64 == 0 &&
               shape(m[1], E, I, D) && shape(m[2], E, I, D) && shape(m[3], E, D, I) && shape(m[4], 1, I, D) &&
               shape(m[5], 1, I, D) && shape(m[6], 1, D, I) && shape(m[7], 1, 1, D) && m[7]->bits == 8;
    for (int i = 1; i < 7; ++i) okg = okg && m[i]->bits == bits;
    if (!okg) {
        set_error(error, capacity,
                  "Unsupported MoE layer geometry: router [1,E,D] 8-bit, gate/up [E,I,D], down [E,D,I], shared "
                  "[1,I,D]/[1,D,I], shared_route [1,1,D] 8-bit; E in [8,256], D %% 256 == 0, I %% 64 == 0");
        return nullptr;
    }
    Layer *L = new Layer();
    L->ctx = c;
    for (int i = 0; i < 8; ++i) {
        L->m[i] = m[i];
        m[i]->refs++;
    }
    L->E = E;
    L->D = D;
    L->I = I;
    L->bits = bits;
    L->gen = ++g_layer_gen;
    L->E_local = E;
    L->E_off = 0;
    std::lock_guard<std::mutex> g(g_registry);
    g_layers.insert(L);
    return L;
}

API void di_moe_layer_destroy(void *layer) {
    if (!live_layer(layer)) return;
    Layer *L = static_cast<Layer *>(layer);
    {
        std::lock_guard<std::mutex> g(g_registry);
        g_layers.erase(L);
    }
    DeviceGuard dg(L->ctx->device);
    cudaStreamSynchronize(L->ctx->stream);
    if (L->bias) cudaFree(L->bias);
    if (L->router_rn) cudaFree(L->router_rn);
    for (int i = 0; i < 8; ++i) release_matrix(L->m[i]);
    delete L;
}

API int di_moe_layer_set_router_bias(void *layer, const float *bias, char *error, int capacity) {
    if (!live_layer(layer)) {
        set_error(error, capacity, "Invalid MoE layer");
        return -1;
    }
    Layer *L = static_cast<Layer *>(layer);
    DeviceGuard dg(L->ctx->device);
    try {
        if (!bias) {
            if (L->bias) CK(cudaFree(L->bias));
            L->bias = nullptr;
            return 0;
        }
        for (int e = 0; e < L->E; ++e)
            if (!std::isfinite(bias[e])) {
                set_error(error, capacity, "Router bias must be finite");
                return -1;
            }
        if (!L->bias) CK(cudaMalloc(&L->bias, sizeof(float) * L->E));
        CK(cudaMemcpyAsync(L->bias, bias, sizeof(float) * L->E, cudaMemcpyHostToDevice, L->ctx->stream));
        CK(cudaStreamSynchronize(L->ctx->stream));
    } catch (const CudaFail &f) {
        set_error(error, capacity, "%s", f.what.c_str());
        return -1;
    }
    return 0;
}

// ---------------------------------------------------------------------------- MLX checkpoints

API int di_moe_checkpoint_probe(const char *directory, int layer, int32_t *geometry, char *error, int capacity) {
    if (!directory || !geometry) {
        set_error(error, capacity, "Invalid checkpoint probe arguments");
        return -1;
    }
    try {
        ckpt::LayerPlan P;
        ckpt::plan_layer(directory, layer, P);
        ckpt::read_norm(P);
        geometry[0] = P.E;
        geometry[1] = P.D;
        geometry[2] = P.I;
        geometry[3] = P.bits;
    } catch (const std::exception &e) {
        set_error(error, capacity, "%s", e.what());
        return -1;
    }
    return 0;
}

API void *di_moe_layer_load(void *ctx, const char *directory, int layer, float *norm, char *error, int capacity) {
    if (!live_context(ctx) || !directory) {
        set_error(error, capacity, "Invalid context or checkpoint directory");
        return nullptr;
    }
    Context *c = static_cast<Context *>(ctx);
    ckpt::LayerPlan P;
    std::vector<float> nw;
    try {
        ckpt::plan_layer(directory, layer, P);  // every tensor validated before any allocation
        nw = ckpt::read_norm(P);
    } catch (const std::exception &e) {
        set_error(error, capacity, "%s", e.what());
        return nullptr;
    }
    void *mats[8] = {};
    auto drop = [&]() {
        for (void *m : mats)
            if (m) di_quant_matrix_destroy(m);
    };
    for (int i = 0; i < 8; ++i) {
        const ckpt::PlannedMatrix &M = P.m[i];
        mats[i] = di_quant_matrix_create(c, M.experts, M.rows, M.cols, M.bits, 64, error, capacity);
        if (!mats[i]) {
            drop();
            return nullptr;
        }
        Matrix *m = static_cast<Matrix *>(mats[i]);
        for (int j = 0; j < 3; ++j) {
            if (M.t[j].bytes != m->bytes[j]) {
                set_error(error, capacity, "Tensor %s has %llu bytes; the matrix buffer holds %zu", M.t[j].name.c_str(),
                          (unsigned long long)M.t[j].bytes, m->bytes[j]);
                drop();
                return nullptr;
            }
            std::vector<uint8_t> host(M.t[j].bytes);
            try {
                M.shard[j]->read(M.t[j], host.data());
            } catch (const std::exception &e) {
                set_error(error, capacity, "%s", e.what());
                drop();
                return nullptr;
            }
            if (di_quant_matrix_upload(mats[i], j, host.data(), host.size(), error, capacity)) {
                drop();
                return nullptr;
            }
        }
    }
    void *layer_h = di_moe_layer_create(c, mats[0], mats[1], mats[2], mats[3], mats[4], mats[5], mats[6], mats[7],
                                        error, capacity);
    if (!layer_h) {
        drop();
        return nullptr;
    }
    // the layer holds the only references: its matrices are freed with it
    for (void *m : mats) release_matrix(static_cast<Matrix *>(m));
    if (norm) std::memcpy(norm, nw.data(), sizeof(float) * nw.size());
    return layer_h;
}

namespace {
bool pick_gemv(int T, int flags) {
    if (flags & DI_MOE_PATH_GEMV) return true;
    if (flags & DI_MOE_PATH_GROUPED) return false;
    return T <= 4;
}
}  // namespace

API int di_moe_block(void *ctx, void *layer, const uint16_t *x, int tokens, uint16_t *y, int32_t *ids, float *probs,
                     int flags, double *ms, char *error, int capacity) {
    if (!live_context(ctx) || !live_layer(layer)) {
        set_error(error, capacity, "Invalid context or MoE layer");
        return -1;
    }
    Context *c = static_cast<Context *>(ctx);
    Layer *L = static_cast<Layer *>(layer);
    const bool dev_io = flags & DI_MOE_DEVICE_IO, forced = flags & DI_MOE_FORCE_ROUTES;
    if (L->ctx != c) {
        set_error(error, capacity, "MoE layer must belong to this device.");
        return -1;
    }
    if (!x || !y || tokens < 1 || tokens > 65536 ||
        (flags & ~(DI_MOE_DEVICE_IO | DI_MOE_FORCE_ROUTES | DI_MOE_PATH_GEMV | DI_MOE_PATH_GROUPED | DI_MOE_ROUTER_EXACT)) ||
        ((flags & DI_MOE_PATH_GEMV) && (flags & DI_MOE_PATH_GROUPED)) || (forced && !ids) ||
        ((flags & DI_MOE_PATH_GEMV) && tokens > kDecodeMaxTokens)) {
        set_error(error, capacity, "Invalid MoE block arguments");
        return -1;
    }
    for (int i = 0; i < 8; ++i)
        if (L->m[i]->destroyed) {
            set_error(error, capacity, "MoE layer matrix was destroyed");
            return -1;
        }
    if (forced && !dev_io)
        for (size_t i = 0; i < (size_t)tokens * 8; ++i)
            if (ids[i] < 0 || ids[i] >= L->E) {
                set_error(error, capacity, "Expert ID out of bounds");
                return -1;
            }
    if (dev_io && !device_pointers_ok(c->device, {x, y, ids, probs})) {
        set_error(error, capacity, "With DI_MOE_DEVICE_IO, x, y, ids and probs must be device memory of the context's GPU");
        return -1;
    }
    const int T = tokens, D = L->D;
    const bool gemv = pick_gemv(T, flags);
    if (gemv && !forced && (size_t)T * D * 2 > (size_t)kDecodeSmemMax) {
        set_error(error, capacity, "Decode path supports T*D <= %d; use the grouped path", kDecodeSmemMax / 2);
        return -1;
    }
    if (!gemv)
        if (const char *why = grouped_geometry_error(L)) {
            set_error(error, capacity, "%s", why);
            return -1;
        }
    DeviceGuard dg(c->device);
    try {
        for (int i = 0; i < 8; ++i) sync_matrix(L->m[i]);
        c->last_routes_T = 0;
        Carve cv;
        BlockBuffers b{};
        b.router_exact = (flags & DI_MOE_ROUTER_EXACT) != 0;
        size_t o_ids_io = 0, o_probs_io = 0;
        if (!dev_io) {
            o_ids_io = cv.take<int32_t>((size_t)T * 8);
            o_probs_io = cv.take<float>((size_t)T * 8);
        }
        plan_block(c, L, T, cv, b, !dev_io, gemv);
        const uint16_t *dx = dev_io ? x : b.x;
        uint16_t *dy = dev_io ? y : b.y;
        int32_t *dids = dev_io ? ids : at<int32_t>(c, o_ids_io);
        float *dprobs = dev_io ? probs : at<float>(c, o_probs_io);
        CK(cudaMemsetAsync(c->d_err, 0, sizeof(uint32_t), c->stream));
        CK(cudaMemsetAsync(b.counter, 0, 2 * sizeof(uint32_t), c->stream));
        CK(cudaEventRecord(c->ev_start, c->stream));
        if (!dev_io) {
            CK(cudaMemcpyAsync(b.x, x, (size_t)T * D * 2, cudaMemcpyHostToDevice, c->stream));
            if (forced) CK(cudaMemcpyAsync(dids, ids, (size_t)T * 8 * 4, cudaMemcpyHostToDevice, c->stream));
        }
        const bool profile = true;
        g_marks = nullptr;
        enqueue_block(c, L, dx, T, dy, nullptr, forced ? dids : nullptr, (dev_io && !probs) ? nullptr : dprobs, gemv,
                      b, profile);
        if (ids && !forced) {
            if (dev_io) CK(cudaMemcpyAsync(ids, b.ids, (size_t)T * 8 * 4, cudaMemcpyDeviceToDevice, c->stream));
            else CK(cudaMemcpyAsync(dids, b.ids, (size_t)T * 8 * 4, cudaMemcpyDeviceToDevice, c->stream));
        }
        if (launch_check(error, capacity)) return -1;
        CK(cudaMemcpyAsync(c->h_err, c->d_err, sizeof(uint32_t), cudaMemcpyDeviceToHost, c->stream));
        if (dev_io) CK(cudaEventRecord(c->ev_stop, c->stream));
        CK(cudaStreamSynchronize(c->stream));
        if (*c->h_err) {
            set_error(error, capacity, "%s", device_error_text(*c->h_err));
            return -1;
        }
        if (!dev_io) {
            // outputs reach the caller only after the device reported success; `ms` covers the
            // host->device copies, the block and these device->host copies
            CK(cudaMemcpyAsync(y, b.y, (size_t)T * D * 2, cudaMemcpyDeviceToHost, c->stream));
            if (ids && !forced) CK(cudaMemcpyAsync(ids, dids, (size_t)T * 8 * 4, cudaMemcpyDeviceToHost, c->stream));
            if (probs) CK(cudaMemcpyAsync(probs, dprobs, (size_t)T * 8 * 4, cudaMemcpyDeviceToHost, c->stream));
            CK(cudaEventRecord(c->ev_stop, c->stream));
            CK(cudaStreamSynchronize(c->stream));
        }
        float t = 0;
        CK(cudaEventElapsedTime(&t, c->ev_start, c->ev_stop));
        if (ms) *ms = t;
        for (int s = 0; s < S_N; ++s) {
            float st = 0;
            cudaEventElapsedTime(&st, c->ev_stage[s], c->ev_stage[s + 1]);
            c->last_stage_ms[s] = st;
        }
        c->last_stage_ms[S_N] = 0;
        c->have_profile = true;
    } catch (const CudaFail &f) {
        set_error(error, capacity, "%s", f.what.c_str());
        return -1;
    }
    return 0;
}

API int di_moe_stack(void *ctx, void *const *layers, const float *norms, int n_layers, float eps, float *x, int tokens,
                     uint16_t *h_trace, int32_t *ids_trace, int flags, double *ms, char *error, int capacity) {
    if (!live_context(ctx) || !layers || n_layers < 1 || n_layers > 1024 || !norms || !x || tokens < 1 ||
        tokens > 65536 || !(eps > 0.0f) ||
        (flags & ~(DI_MOE_DEVICE_IO | DI_MOE_PATH_GEMV | DI_MOE_PATH_GROUPED | DI_MOE_PROFILE | DI_MOE_ROUTER_EXACT)) ||
        ((flags & DI_MOE_PATH_GEMV) && (flags & DI_MOE_PATH_GROUPED)) ||
        ((flags & DI_MOE_PATH_GEMV) && tokens > kDecodeMaxTokens)) {
        set_error(error, capacity, "Invalid MoE stack arguments");
        return -1;
    }
    Context *c = static_cast<Context *>(ctx);
    int D = -1;
    for (int l = 0; l < n_layers; ++l) {
        if (!live_layer(layers[l]) || static_cast<Layer *>(layers[l])->ctx != c) {
            set_error(error, capacity, "Invalid MoE layer %d", l);
            return -1;
        }
        Layer *L = static_cast<Layer *>(layers[l]);
        if (D < 0) D = L->D;
        if (L->D != D) {
            set_error(error, capacity, "MoE stack layers must share the hidden size");
            return -1;
        }
        for (int i = 0; i < 8; ++i)
            if (L->m[i]->destroyed) {
                set_error(error, capacity, "MoE layer matrix was destroyed");
                return -1;
            }
    }
    const bool dev_io = flags & DI_MOE_DEVICE_IO, profile = flags & DI_MOE_PROFILE;
    if (dev_io && !device_pointers_ok(c->device, {x, norms, h_trace, ids_trace})) {
        set_error(error, capacity,
                  "With DI_MOE_DEVICE_IO, x, norms and the traces must be device memory of the context's GPU");
        return -1;
    }
    const int T = tokens;
    const bool gemv = pick_gemv(T, flags);
    if (gemv && (size_t)T * D * 2 > (size_t)kDecodeSmemMax) {
        set_error(error, capacity, "Decode path supports T*D <= %d; use the grouped path", kDecodeSmemMax / 2);
        return -1;
    }
    if (!gemv)
        for (int l = 0; l < n_layers; ++l)
            if (const char *why = grouped_geometry_error(static_cast<Layer *>(layers[l]))) {
                set_error(error, capacity, "%s", why);
                return -1;
            }
    DeviceGuard dg(c->device);
    try {
        const size_t need_events = profile ? (size_t)n_layers * (S_N + 2) : 0;
        while (c->layer_events.size() < need_events) {
            cudaEvent_t e;
            CK(cudaEventCreate(&e));
            c->layer_events.push_back(e);
        }
        for (int l = 0; l < n_layers; ++l)
            for (int i = 0; i < 8; ++i) sync_matrix(static_cast<Layer *>(layers[l])->m[i]);
        Carve cv;
        size_t o_x = dev_io ? 0 : cv.take<float>((size_t)T * D);
        size_t o_n = dev_io ? 0 : cv.take<float>((size_t)n_layers * D);
        size_t o_h = cv.take<uint16_t>((size_t)T * D);
        size_t o_ht = (!dev_io && h_trace) ? cv.take<uint16_t>((size_t)n_layers * T * D) : 0;
        size_t o_it = (!dev_io && ids_trace) ? cv.take<int32_t>((size_t)n_layers * T * 8) : 0;
        int Emax = 0, Imax = 0;
        for (int l = 0; l < n_layers; ++l) {
            Emax = std::max(Emax, static_cast<Layer *>(layers[l])->E);
            Imax = std::max(Imax, static_cast<Layer *>(layers[l])->I);
        }
        c->last_routes_T = 0;
        BlockBuffers b{};
        b.router_exact = (flags & DI_MOE_ROUTER_EXACT) != 0;
        // size the block buffers for the widest layer (layers of one stack share E and I in practice)
        Layer probe = *static_cast<Layer *>(layers[0]);
        probe.E = Emax;
        probe.I = Imax;
        plan_block(c, &probe, T, cv, b, false, gemv);
        float *dx = dev_io ? x : at<float>(c, o_x);
        const float *dn = dev_io ? norms : at<float>(c, o_n);
        uint16_t *dh = at<uint16_t>(c, o_h);
        uint16_t *dht = dev_io ? h_trace : (h_trace ? at<uint16_t>(c, o_ht) : nullptr);
        int32_t *dit = dev_io ? ids_trace : (ids_trace ? at<int32_t>(c, o_it) : nullptr);
        CK(cudaMemsetAsync(c->d_err, 0, sizeof(uint32_t), c->stream));
        CK(cudaEventRecord(c->ev_start, c->stream));
        if (!dev_io) {
            CK(cudaMemcpyAsync(dx, x, (size_t)T * D * 4, cudaMemcpyHostToDevice, c->stream));
            CK(cudaMemcpyAsync(const_cast<float *>(dn), norms, (size_t)n_layers * D * 4, cudaMemcpyHostToDevice,
                               c->stream));
        }
        auto enqueue_layers = [&]() {
            for (int l = 0; l < n_layers; ++l) {
                Layer *L = static_cast<Layer *>(layers[l]);
                cudaEvent_t *ev = profile ? &c->layer_events[(size_t)l * (S_N + 2)] : nullptr;
                if (profile) CK(cudaEventRecord(ev[S_N + 1], c->stream));
                uint16_t *trace_l = dht ? dht + (size_t)l * T * D : nullptr;
                g_marks = ev;
                if (gemv) {
                    // RMSNorm is fused into the decode route kernel
                    enqueue_block(c, L, dh, T, nullptr, dx, nullptr, nullptr, true, b, profile, dn + (size_t)l * D, eps,
                                  trace_l, nullptr, nullptr, nullptr, (uint32_t)l + 1);
                } else {
                    // layer l's RMSNorm runs in layer l-1's combine; the first one on its own
                    if (l == 0) launch(rmsnorm_kernel, dim3(T), dim3(256), 0, c->stream, true, dx, dn, D, eps, dh, trace_l);
                    const bool more = l + 1 < n_layers;
                    enqueue_block(c, L, dh, T, nullptr, dx, nullptr, nullptr, false, b, profile, nullptr, eps, nullptr,
                                  more ? dn + (size_t)(l + 1) * D : nullptr, more ? dh : nullptr,
                                  more && dht ? dht + (size_t)(l + 1) * T * D : nullptr);
                }
                g_marks = nullptr;
                if (dit)
                    CK(cudaMemcpyAsync(dit + (size_t)l * T * 8, b.ids, (size_t)T * 8 * 4, cudaMemcpyDeviceToDevice,
                                       c->stream));
            }
        };
        CK(cudaMemsetAsync(b.counter, 0, 2 * sizeof(uint32_t), c->stream));
        bool persistent = gemv && T == 1 && !profile && stack_fits(c, layers, n_layers);
        if (persistent) {
            // one token: every layer in one persistent cooperative kernel
            enqueue_stack(c, layers, n_layers, dn, eps, dx, dht, dit);
        } else if (gemv && !profile) {
            // decode: one CUDA graph for the whole stack, rebuilt only when its inputs change
            std::vector<uint64_t> key = {(uint64_t)n_layers, (uint64_t)T, (uint64_t)(uintptr_t)dx,
                                         (uint64_t)(uintptr_t)dn, (uint64_t)(uintptr_t)dht, (uint64_t)(uintptr_t)dit,
                                         (uint64_t)(uintptr_t)c->ws.base, (uint64_t)c->ws.cap,
                                         eps_bits(eps)};
            for (int l = 0; l < n_layers; ++l) {
                const Layer *L = static_cast<Layer *>(layers[l]);
                key.push_back(L->gen);
                key.push_back((uint64_t)(uintptr_t)L->bias);
            }
            if (!c->graph_exec || key != c->graph_key) {
                if (c->graph_exec) {
                    cudaGraphExecDestroy(c->graph_exec);
                    c->graph_exec = nullptr;
                }
                cudaGraph_t graph = nullptr;
                CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
                try {
                    enqueue_layers();
                } catch (...) {
                    cudaStreamEndCapture(c->stream, &graph);
                    if (graph) cudaGraphDestroy(graph);
                    throw;
                }
                CK(cudaStreamEndCapture(c->stream, &graph));
                cudaError_t ie = cudaGraphInstantiate(&c->graph_exec, graph, 0);
                cudaGraphDestroy(graph);
                CK(ie);
                c->graph_key = key;
            }
            CK(cudaGraphLaunch(c->graph_exec, c->stream));
        } else {
            enqueue_layers();
        }
        if (launch_check(error, capacity)) return -1;
        CK(cudaMemcpyAsync(c->h_err, c->d_err, sizeof(uint32_t), cudaMemcpyDeviceToHost, c->stream));
        if (dev_io) CK(cudaEventRecord(c->ev_stop, c->stream));
        CK(cudaStreamSynchronize(c->stream));
        if (persistent && *c->h_err == kErrRange) {
            // an output outside the one-token kernel's fixed-point range (it left x unwritten):
            // start its exchange state over and compute the token with the per-layer kernels
            CK(cudaMemsetAsync(c->ll, 0, c->ll_words * 8, c->stream));
            CK(cudaMemsetAsync(c->d_err, 0, sizeof(uint32_t), c->stream));
            persistent = false;
            enqueue_layers();
            if (launch_check(error, capacity)) return -1;
            CK(cudaMemcpyAsync(c->h_err, c->d_err, sizeof(uint32_t), cudaMemcpyDeviceToHost, c->stream));
            if (dev_io) CK(cudaEventRecord(c->ev_stop, c->stream));
            CK(cudaStreamSynchronize(c->stream));
        }
        if (*c->h_err) {
            if (persistent && (*c->h_err & kErrTimeout)) {
                // an abandoned call leaves arrival counts and generations out of step: start over
                CK(cudaMemsetAsync(c->ll, 0, c->ll_words * 8, c->stream));
                CK(cudaStreamSynchronize(c->stream));
            }
            set_error(error, capacity, "%s", device_error_text(*c->h_err));
            return -1;
        }
        if (!dev_io) {
            CK(cudaMemcpyAsync(x, dx, (size_t)T * D * 4, cudaMemcpyDeviceToHost, c->stream));
            if (h_trace)
                CK(cudaMemcpyAsync(h_trace, dht, (size_t)n_layers * T * D * 2, cudaMemcpyDeviceToHost, c->stream));
            if (ids_trace)
                CK(cudaMemcpyAsync(ids_trace, dit, (size_t)n_layers * T * 8 * 4, cudaMemcpyDeviceToHost, c->stream));
            CK(cudaEventRecord(c->ev_stop, c->stream));
            CK(cudaStreamSynchronize(c->stream));
        }
        float t = 0;
        CK(cudaEventElapsedTime(&t, c->ev_start, c->ev_stop));
        if (ms) *ms = t;
        if (profile) {
            for (int s = 0; s < kProfileSlots; ++s) c->last_stage_ms[s] = 0;
            for (int l = 0; l < n_layers; ++l) {
                cudaEvent_t *ev = &c->layer_events[(size_t)l * (S_N + 2)];
                for (int s = 0; s < S_N; ++s) {
                    float st = 0;
                    CK(cudaEventElapsedTime(&st, ev[s], ev[s + 1]));
                    c->last_stage_ms[s] += st;
                }
                float rn = 0;
                CK(cudaEventElapsedTime(&rn, ev[S_N + 1], ev[S_ROUTER]));
                c->last_stage_ms[S_N] += rn;
            }
            c->have_profile = true;
        }
    } catch (const CudaFail &f) {
        set_error(error, capacity, "%s", f.what.c_str());
        return -1;
    }
    return 0;
}

API int di_moe_last_profile(void *ctx, double *stage_ms, int n) {
    if (!live_context(ctx) || !stage_ms || n < 1) return 0;
    Context *c = static_cast<Context *>(ctx);
    if (!c->have_profile) return 0;
    const int k = std::min(n, kProfileSlots);
    for (int i = 0; i < k; ++i) stage_ms[i] = c->last_stage_ms[i];
    return k;
}


API int di_moe_last_routes(void *ctx, int32_t *perm_route, int32_t *seg_offsets, int32_t *seg_counts, int max_routes,
                           char *error, int capacity) {
    if (!live_context(ctx) || !perm_route || !seg_offsets || !seg_counts) {
        set_error(error, capacity, "Invalid route readback arguments");
        return -1;
    }
    Context *c = static_cast<Context *>(ctx);
    if (c->last_routes_T < 1) {
        set_error(error, capacity, "The last call on this context built no expert-grouped permutation");
        return -1;
    }
    const int n = 8 * c->last_routes_T;
    if (max_routes < n) {
        set_error(error, capacity, "The permutation holds %d routes; the buffer takes %d", n, max_routes);
        return -1;
    }
    DeviceGuard dg(c->device);
    try {
        CK(cudaMemcpyAsync(perm_route, c->last_perm, (size_t)n * 4, cudaMemcpyDeviceToHost, c->stream));
        CK(cudaMemcpyAsync(seg_offsets, c->last_seg_off, (size_t)(c->last_routes_E + 1) * 4, cudaMemcpyDeviceToHost,
                           c->stream));
        CK(cudaMemcpyAsync(seg_counts, c->last_seg_count, (size_t)(c->last_routes_E + 1) * 4, cudaMemcpyDeviceToHost,
                           c->stream));
        CK(cudaStreamSynchronize(c->stream));
    } catch (const CudaFail &f) {
        set_error(error, capacity, "%s", f.what.c_str());
        return -1;
    }
    return n;
}

// ============================================================================ Part 3: expert parallelism

namespace {
// NCCL is resolved at run time, only when an expert-parallel group is created: a process that
// already loaded libnccl.so.2 (e.g. through torch) keeps that copy; otherwise the library named
// by DEEPINFER_NCCL_LIBRARY or the default libnccl.so.2 is loaded. Single-GPU use never loads it.
struct NcclApi {
    ncclResult_t (*getUniqueId)(ncclUniqueId *);
    ncclResult_t (*commInitRank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*commDestroy)(ncclComm_t);
    ncclResult_t (*allReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*allGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*groupStart)();
    ncclResult_t (*groupEnd)();
    const char *(*getErrorString)(ncclResult_t);
};
const NcclApi *nccl_api(std::string *why) {
    static NcclApi api{};
    static bool tried = false, ok = false;
    static std::string reason;
    static std::mutex m;
    std::lock_guard<std::mutex> g(m);
    if (!tried) {
        tried = true;
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) {
            const char *path = std::getenv("DEEPINFER_NCCL_LIBRARY");
            h = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        }
        if (!h) {
            reason = std::string("cannot load NCCL: ") + dlerror();
        } else {
            auto sym = [&](const char *n) { return dlsym(h, n); };
            api.getUniqueId = (decltype(api.getUniqueId))sym("ncclGetUniqueId");
            api.commInitRank = (decltype(api.commInitRank))sym("ncclCommInitRank");
            api.commDestroy = (decltype(api.commDestroy))sym("ncclCommDestroy");
            api.allReduce = (decltype(api.allReduce))sym("ncclAllReduce");
            api.allGather = (decltype(api.allGather))sym("ncclAllGather");
            api.send = (decltype(api.send))sym("ncclSend");
            api.recv = (decltype(api.recv))sym("ncclRecv");
            api.groupStart = (decltype(api.groupStart))sym("ncclGroupStart");
            api.groupEnd = (decltype(api.groupEnd))sym("ncclGroupEnd");
            api.getErrorString = (decltype(api.getErrorString))sym("ncclGetErrorString");
            ok = api.getUniqueId && api.commInitRank && api.commDestroy && api.allReduce && api.allGather && api.send &&
                 api.recv && api.groupStart && api.groupEnd && api.getErrorString;
            if (!ok) reason = "NCCL library lacks a required entry point";
        }
    }
    if (!ok && why) *why = reason;
    return ok ? &api : nullptr;
}

struct Ep {
    Context *ctx = nullptr;
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    int32_t *h_counts = nullptr;  // pinned [world*world]
    // symmetric buffers (ep.cuh), mapped into every rank through CUDA IPC
    size_t cap = 0;                        // tokens per rank they hold
    int sym_D = 0;                         // hidden size they were laid out for
    uint8_t *sym = nullptr;                // this rank's
    uint8_t *peer_sym[kMaxRanks] = {};     // every rank's, in this process's address space
    uint64_t steps = 0;                    // layer steps completed: every arrival counter reads this
    bool broken = false;                   // a device wait failed: the counters are out of step
};
struct EpSymLayout {
    size_t rx, meta, back, sync, bytes;
};
EpSymLayout ep_sym_layout(int G, size_t cap, int D) {
    auto up = [](size_t v) { return (v + 255) & ~(size_t)255; };
    EpSymLayout o;
    o.rx = 0;
    o.meta = up(o.rx + (size_t)G * cap * D * 2);
    o.back = up(o.meta + (size_t)G * cap * sizeof(RowMeta));
    o.sync = up(o.back + (size_t)G * cap * D * 2);
    o.bytes = up(o.sync + 4 * kMaxRanks * sizeof(uint32_t));
    return o;
}
EpPeers ep_peers(const Ep *ep) {
    const EpSymLayout o = ep_sym_layout(ep->world, ep->cap, ep->sym_D);
    EpPeers p{};
    for (int q = 0; q < ep->world; ++q) {
        p.rx[q] = reinterpret_cast<uint16_t *>(ep->peer_sym[q] + o.rx);
        p.meta[q] = reinterpret_cast<RowMeta *>(ep->peer_sym[q] + o.meta);
        p.back[q] = reinterpret_cast<uint16_t *>(ep->peer_sym[q] + o.back);
        p.sync[q] = reinterpret_cast<uint32_t *>(ep->peer_sym[q] + o.sync);
    }
    return p;
}
void ep_release_sym(Ep *ep) {
    for (int q = 0; q < ep->world; ++q)
        if (q != ep->rank && ep->peer_sym[q]) cudaIpcCloseMemHandle(ep->peer_sym[q]);
    if (ep->sym) cudaFree(ep->sym);
    ep->sym = nullptr;
    for (int q = 0; q < kMaxRanks; ++q) ep->peer_sym[q] = nullptr;
    ep->cap = 0;
    ep->sym_D = 0;
}
std::set<Ep *> g_eps;
bool live_ep(void *p) {
    std::lock_guard<std::mutex> g(g_registry);
    return p && g_eps.count(static_cast<Ep *>(p));
}
struct NcclFail {
    std::string what;
};
#define NK(call)                                                                                      \
    do {                                                                                              \
        ncclResult_t r_ = (call);                                                                     \
        if (r_ != ncclSuccess) throw NcclFail{std::string(#call) + ": " + nc->getErrorString(r_)};    \
    } while (0)

// Collective (every rank of the group calls it with the same arguments): make the symmetric
// buffers hold `cap` tokens per rank of hidden size D, allocating, zeroing and mapping them
// across the ranks (CUDA IPC handles gathered through NCCL) when they do not yet.
void ep_prepare(Ep *ep, size_t cap, int D) {
    if (ep->sym && cap <= ep->cap && D == ep->sym_D) return;
    const NcclApi *nc = nccl_api(nullptr);
    Context *c = ep->ctx;
    CK(cudaStreamSynchronize(c->stream));
    ep_release_sym(ep);
    const EpSymLayout o = ep_sym_layout(ep->world, cap, D);
    CK(cudaMalloc(&ep->sym, o.bytes));
    CK(cudaMemsetAsync(ep->sym, 0, o.bytes, c->stream));
    cudaIpcMemHandle_t mine;
    CK(cudaIpcGetMemHandle(&mine, ep->sym));
    Carve cv;
    const size_t o_h = cv.take<uint8_t>(sizeof(cudaIpcMemHandle_t) * (ep->world + 1));
    ensure_workspace(c, cv.off + 256);
    uint8_t *dh = at<uint8_t>(c, o_h);
    CK(cudaMemcpyAsync(dh, &mine, sizeof(mine), cudaMemcpyHostToDevice, c->stream));
    // every rank's handle; a rank's zeroing precedes its handle in stream order, so no rank can
    // write into a buffer before it is cleared
    NK(nc->allGather(dh, dh + sizeof(mine), sizeof(mine), ncclUint8, ep->comm, c->stream));
    std::vector<cudaIpcMemHandle_t> all(ep->world);
    CK(cudaMemcpyAsync(all.data(), dh + sizeof(mine), sizeof(mine) * ep->world, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    for (int q = 0; q < ep->world; ++q) {
        if (q == ep->rank) {
            ep->peer_sym[q] = ep->sym;
            continue;
        }
        void *p = nullptr;
        CK(cudaIpcOpenMemHandle(&p, all[q], cudaIpcMemLazyEnablePeerAccess));
        ep->peer_sym[q] = static_cast<uint8_t *>(p);
    }
    ep->cap = cap;
    ep->sym_D = D;
    ep->steps = 0;  // fresh counters
}
}  // namespace

API int di_moe_ep_unique_id(uint8_t *id, char *error, int capacity) {
    if (!id) {
        set_error(error, capacity, "Invalid unique id buffer");
        return -1;
    }
    static_assert(sizeof(ncclUniqueId) == DI_EP_ID_BYTES, "NCCL unique id size");
    std::string why;
    const NcclApi *nc = nccl_api(&why);
    if (!nc) {
        set_error(error, capacity, "%s", why.c_str());
        return -1;
    }
    ncclUniqueId u;
    ncclResult_t r = nc->getUniqueId(&u);
    if (r != ncclSuccess) {
        set_error(error, capacity, "ncclGetUniqueId: %s", nc->getErrorString(r));
        return -1;
    }
    std::memcpy(id, &u, sizeof(u));
    return 0;
}

API void *di_moe_ep_create(void *ctx, const uint8_t *id, int rank, int world, char *error, int capacity) {
    if (!live_context(ctx) || !id || world < 1 || world > kMaxRanks || rank < 0 || rank >= world) {
        set_error(error, capacity, "Invalid expert-parallel arguments (world 1..%d)", kMaxRanks);
        return nullptr;
    }
    Context *c = static_cast<Context *>(ctx);
    std::string why;
    const NcclApi *nc = nccl_api(&why);
    if (!nc) {
        set_error(error, capacity, "%s", why.c_str());
        return nullptr;
    }
    DeviceGuard dg(c->device);
    Ep *ep = new Ep();
    ep->ctx = c;
    ep->rank = rank;
    ep->world = world;
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    ncclResult_t r = nc->commInitRank(&ep->comm, world, u, rank);
    if (r != ncclSuccess) {
        set_error(error, capacity, "ncclCommInitRank: %s", nc->getErrorString(r));
        delete ep;
        return nullptr;
    }
    if (cudaMallocHost(&ep->h_counts, sizeof(int32_t) * kMaxRanks * kMaxRanks) != cudaSuccess) {
        cudaGetLastError();
        nc->commDestroy(ep->comm);
        delete ep;
        set_error(error, capacity, "Pinned host allocation failed");
        return nullptr;
    }
    std::lock_guard<std::mutex> g(g_registry);
    g_eps.insert(ep);
    return ep;
}

API void di_moe_ep_destroy(void *p) {
    if (!live_ep(p)) return;
    Ep *ep = static_cast<Ep *>(p);
    {
        std::lock_guard<std::mutex> g(g_registry);
        g_eps.erase(ep);
    }
    DeviceGuard dg(ep->ctx->device);
    cudaStreamSynchronize(ep->ctx->stream);
    ep_release_sym(ep);
    nccl_api(nullptr)->commDestroy(ep->comm);
    cudaFreeHost(ep->h_counts);
    delete ep;
}

API void *di_moe_ep_layer_create(void *ep_, void *router, void *gate, void *up, void *down, void *shared_gate,
                                 void *shared_up, void *shared_down, void *shared_route, char *error, int capacity) {
    if (!live_ep(ep_)) {
        set_error(error, capacity, "Invalid expert-parallel handle");
        return nullptr;
    }
    Ep *ep = static_cast<Ep *>(ep_);
    void *ptrs[8] = {router, gate, up, down, shared_gate, shared_up, shared_down, shared_route};
    Matrix *m[8];
    for (int i = 0; i < 8; ++i) {
        if (!live_matrix(ptrs[i]) || static_cast<Matrix *>(ptrs[i])->ctx != ep->ctx) {
            set_error(error, capacity, "MoE layer matrix %d is missing, destroyed or on another device", i);
            return nullptr;
        }
        m[i] = static_cast<Matrix *>(ptrs[i]);
        for (int j = 0; j < i; ++j)
            if (m[j] == m[i]) {
                set_error(error, capacity, "MoE layer matrices must be distinct.");
                return nullptr;
            }
    }
    const int E = m[0]->rows, D = m[0]->cols, El = m[1]->experts, I = m[1]->rows, bits = m[1]->bits;
    auto shape = [](Matrix *x, int e, int r, int col) { return x->experts == e && x->rows == r && x->cols == col; };
    bool ok = m[0]->experts == 1 && m[0]->bits == 8 && E >= 8 && E <= 256 && El * ep->world == E && D % 256 == 0 &&
              I % 64 == 0 && shape(m[1], El, I, D) && shape(m[2], El, I, D) && shape(m[3], El, D, I) &&
              shape(m[4], 1, I, D) && shape(m[5], 1, I, D) && shape(m[6], 1, D, I) && shape(m[7], 1, 1, D) &&
              m[7]->bits == 8;
    for (int i = 1; i < 7; ++i) ok = ok && m[i]->bits == bits;
    if (!ok) {
        set_error(error, capacity,
                  "Unsupported expert-parallel layer: router [1,E,D] 8-bit with E = world * E_local, expert shards "
                  "[E_local,I,D]/[E_local,D,I], shared [1,I,D]/[1,D,I], shared_route [1,1,D] 8-bit");
        return nullptr;
    }
    Layer *L = new Layer();
    L->ctx = ep->ctx;
    for (int i = 0; i < 8; ++i) {
        L->m[i] = m[i];
        m[i]->refs++;
    }
    L->E = E;
    L->D = D;
    L->I = I;
    L->bits = bits;
    L->gen = ++g_layer_gen;
    L->E_local = El;
    L->E_off = ep->rank * El;
    std::lock_guard<std::mutex> g(g_registry);
    g_layers.insert(L);
    return L;
}

API int di_moe_ep_stack(void *ep_, void *const *layers, const float *norms, int n_layers, float eps, float *x,
                        int tokens, uint16_t *h_trace, int32_t *ids_trace, int flags, double *ms, char *error,
                        int capacity) {
    if (!live_ep(ep_) || !layers || n_layers < 1 || n_layers > 1024 || !norms || !x || tokens < 1 ||
        tokens > 65536 || !(eps > 0.0f) || (flags & ~(DI_MOE_DEVICE_IO | DI_MOE_PROFILE))) {
        set_error(error, capacity, "Invalid expert-parallel stack arguments");
        return -1;
    }
    Ep *ep = static_cast<Ep *>(ep_);
    Context *c = ep->ctx;
    const int G = ep->world, rank = ep->rank, T = tokens;
    int D = -1, E = -1, El = -1, I = -1;
    for (int l = 0; l < n_layers; ++l) {
        if (!live_layer(layers[l]) || static_cast<Layer *>(layers[l])->ctx != c) {
            set_error(error, capacity, "Invalid MoE layer %d", l);
            return -1;
        }
        Layer *L = static_cast<Layer *>(layers[l]);
        if (l == 0) {
            D = L->D;
            E = L->E;
            El = L->E_local;
            I = L->I;
        }
        if (L->D != D || L->E != E || L->E_local != El || L->I != I || El * G != E || L->E_off != rank * El) {
            set_error(error, capacity, "Layer %d is not an expert-parallel shard of this rank", l);
            return -1;
        }
        for (int i = 0; i < 8; ++i)
            if (L->m[i]->destroyed) {
                set_error(error, capacity, "MoE layer matrix was destroyed");
                return -1;
            }
        if (const char *why = grouped_geometry_error(L)) {
            set_error(error, capacity, "%s", why);
            return -1;
        }
    }
    const bool dev_io = flags & DI_MOE_DEVICE_IO;
    if (dev_io && !device_pointers_ok(c->device, {x, norms, h_trace, ids_trace})) {
        set_error(error, capacity,
                  "With DI_MOE_DEVICE_IO, x, norms and the traces must be device memory of the context's GPU");
        return -1;
    }
    if (ep->broken) {
        set_error(error, capacity, "Expert-parallel group failed in an earlier call; create it again");
        return -1;
    }
    const NcclApi *nc = nccl_api(nullptr);
    DeviceGuard dg(c->device);
    cudaStream_t st = c->stream;
    try {
        for (int l = 0; l < n_layers; ++l)
            for (int i = 0; i < 8; ++i) sync_matrix(static_cast<Layer *>(layers[l])->m[i]);
        // the largest token count of any rank sizes the symmetric buffers (one host round trip
        // per call; the layers below run without any)
        Carve cv0;
        const size_t o_tok = cv0.take<int32_t>(2);
        ensure_workspace(c, cv0.off + 256);
        int32_t *d_tok = at<int32_t>(c, o_tok);
        CK(cudaMemcpyAsync(d_tok, &T, 4, cudaMemcpyHostToDevice, st));
        NK(nc->allReduce(d_tok, d_tok + 1, 1, ncclInt32, ncclMax, ep->comm, st));
        CK(cudaMemcpyAsync(ep->h_counts, d_tok + 1, 4, cudaMemcpyDeviceToHost, st));
        CK(cudaStreamSynchronize(st));
        ep_prepare(ep, (size_t)ep->h_counts[0], D);
        const int cap = (int)ep->cap;
        const int RC = G * cap;  // received row slots: region s = rows from rank s
        const EpPeers peers = ep_peers(ep);
        const EpSymLayout so_ = ep_sym_layout(G, cap, D);
        uint16_t *my_rx = reinterpret_cast<uint16_t *>(ep->sym + so_.rx);
        RowMeta *my_meta = reinterpret_cast<RowMeta *>(ep->sym + so_.meta);
        uint16_t *my_back = reinterpret_cast<uint16_t *>(ep->sym + so_.back);
        uint32_t *my_sync = reinterpret_cast<uint32_t *>(ep->sym + so_.sync);
        const int nb_l = (T + topk::TOK_PER_CTA - 1) / topk::TOK_PER_CTA;
        const int nbr = (RC + topk::TOK_PER_CTA - 1) / topk::TOK_PER_CTA;
        const int max_tiles = (8 * RC + gg::BN - 1) / gg::BN + El + (T + gg::BN - 1) / gg::BN + 2;
        Carve cv;
        cv.take<int32_t>(2);  // keep the token-count words
        const size_t o_x = dev_io ? 0 : cv.take<float>((size_t)T * D), o_n = dev_io ? 0 : cv.take<float>((size_t)n_layers * D);
        const size_t o_h = cv.take<uint16_t>((size_t)T * D), o_lg = cv.take<float>((size_t)T * E);
        const size_t o_ids = cv.take<int32_t>((size_t)T * 8), o_p = cv.take<float>((size_t)T * 8), o_g = cv.take<float>(T);
        const size_t o_bc = cv.take<int32_t>((size_t)nb_l * E);
        const size_t o_il = cv.take<int32_t>((size_t)RC * 8 + 8), o_rbc = cv.take<int32_t>((size_t)(nbr + 1) * (El + 1));
        const size_t o_rbb = cv.take<int32_t>((size_t)(nbr + 1) * (El + 1)), o_sgc = cv.take<int32_t>(El + 2);
        const size_t o_sgo = cv.take<int32_t>(El + 2), o_t = cv.take<Tile>(max_tiles), o_nt = cv.take<int32_t>(1);
        const size_t o_pm = cv.take<int32_t>((size_t)RC * 8 + 8), o_act = cv.take<uint16_t>(((size_t)RC * 8 + T) * I);
        const size_t o_y = cv.take<uint16_t>(((size_t)RC * 8 + T) * D + 8), o_rp = cv.take<int32_t>((size_t)RC * 8 + 8);
        const size_t o_xp = cv.take<uint16_t>((size_t)RC * 8 * D + 8);
        const size_t o_wn = cv.take<float>(2 * (size_t)E), o_rt = cv.take<Tile>((size_t)(T + kRouterTileRows - 1) / kRouterTileRows + 1);
        const size_t o_rnt = cv.take<int32_t>(1), o_wf = cv.take<float>((size_t)E * D);
        const size_t o_ht = (!dev_io && h_trace) ? cv.take<uint16_t>((size_t)n_layers * T * D) : 0;
        const size_t o_it = (!dev_io && ids_trace) ? cv.take<int32_t>((size_t)n_layers * T * 8) : 0;
        ensure_workspace(c, cv.off + 256);
        uint16_t *dht = dev_io ? h_trace : (h_trace ? at<uint16_t>(c, o_ht) : nullptr);
        int32_t *dit = dev_io ? ids_trace : (ids_trace ? at<int32_t>(c, o_it) : nullptr);
        float *dx = dev_io ? x : at<float>(c, o_x);
        const float *dn = dev_io ? norms : at<float>(c, o_n);
        uint16_t *h = at<uint16_t>(c, o_h), *act = at<uint16_t>(c, o_act), *y = at<uint16_t>(c, o_y);
        uint16_t *xp = at<uint16_t>(c, o_xp);
        int32_t *rpos = at<int32_t>(c, o_rp);
        float *logits = at<float>(c, o_lg), *probs = at<float>(c, o_p), *gate = at<float>(c, o_g);
        int32_t *ids = at<int32_t>(c, o_ids), *bc = at<int32_t>(c, o_bc);
        int32_t *il = at<int32_t>(c, o_il), *rbc = at<int32_t>(c, o_rbc), *rbb = at<int32_t>(c, o_rbb);
        int32_t *sgc = at<int32_t>(c, o_sgc), *sgo = at<int32_t>(c, o_sgo), *nt = at<int32_t>(c, o_nt);
        int32_t *perm = at<int32_t>(c, o_pm);
        Tile *tiles = at<Tile>(c, o_t);
        float *wn = at<float>(c, o_wn);
        Tile *rtiles = at<Tile>(c, o_rt);
        int32_t *rnt = at<int32_t>(c, o_rnt);
        float *wf = at<float>(c, o_wf);
        // DI_MOE_PROFILE: per-layer events at the stage boundaries [router logits, top-8 + dispatch,
        // receive + scan, scatter, gate_up, down, partial-row send, combine], summed over the layers
        const bool profile = (flags & DI_MOE_PROFILE) != 0;
        constexpr int kEpStages = 8;
        const size_t need_events = profile ? (size_t)n_layers * (kEpStages + 1) : 0;
        while (c->layer_events.size() < need_events) {
            cudaEvent_t e;
            CK(cudaEventCreate(&e));
            c->layer_events.push_back(e);
        }
        auto mark = [&](int l, int stage) {
            if (profile) CK(cudaEventRecord(c->layer_events[(size_t)l * (kEpStages + 1) + stage], st));
        };
        CK(cudaMemsetAsync(c->d_err, 0, sizeof(uint32_t), st));
        CK(cudaEventRecord(c->ev_start, st));
        if (!dev_io) {
            CK(cudaMemcpyAsync(dx, x, (size_t)T * D * 4, cudaMemcpyHostToDevice, st));
            CK(cudaMemcpyAsync(const_cast<float *>(dn), norms, (size_t)n_layers * D * 4, cudaMemcpyHostToDevice, st));
        }
        const int grid = c->sms;
        for (int l = 0; l < n_layers; ++l) {
            mark(l, 0);
            Layer *L = static_cast<Layer *>(layers[l]);
            const QView R = L->m[0]->view(), Gm = L->m[1]->view(), U = L->m[2]->view(), Dm = L->m[3]->view();
            const QView SG = L->m[4]->view(), SU = L->m[5]->view(), SD = L->m[6]->view(), SR = L->m[7]->view();
            const uint32_t target = (uint32_t)(ep->steps + (uint64_t)l + 1);  // arrivals per rank so far
            // 1. route the local tokens (layer l's RMSNorm ran in layer l-1's combine)
            if (l == 0) launch(rmsnorm_kernel, dim3(T), dim3(256), 0, st, true, dx, dn, D, eps, h, nullptr);
            if (router_tc_fits(L)) {
                uint16_t *approx = reinterpret_cast<uint16_t *>(logits);
                const float *rwn = nullptr, *rwf = nullptr;
                router_norms(L, st, wn, wf, &rwn, &rwf);
                enqueue_router_approx(L, h, T, rtiles, rnt, approx, grid, c->d_err, st);
                mark(l, 1);
                // 2. (fused) one row per (token, destination rank), written into the destinations over NVLink
                const RouterDispatch dsp{peers, G, rank, cap, El, my_sync + 3 * G + 1};
                enqueue_router_select(L, h, T, nullptr, ids, probs, gate, nullptr, nb_l, rwn, rwf, approx, c->d_err,
                                      st, &dsp);
            } else {
                router_logits_kernel<<<dim3((T + router::TT - 1) / router::TT, (E + router::TE - 1) / router::TE),
                                       router::THREADS, sizeof(router::Smem), st>>>(h, T, D, R, L->bias, logits);
                mark(l, 1);
                topk_count_kernel<<<nb_l, topk::WARPS * 32, 0, st>>>(logits, T, E, h, D, SR, nullptr, ids, probs, gate,
                                                                      bc, c->d_err);
            }
            if (dht)
                CK(cudaMemcpyAsync(dht + (size_t)l * T * D, h, (size_t)T * D * 2, cudaMemcpyDeviceToDevice, st));
            if (dit)
                CK(cudaMemcpyAsync(dit + (size_t)l * T * 8, ids, (size_t)T * 8 * 4, cudaMemcpyDeviceToDevice, st));
            // 2. one row per (token, destination rank), written into the destinations over NVLink (the
            // tensor-core router writes them itself)
            if (!router_tc_fits(L))
                launch(ep_dispatch_kernel, dim3(std::min((T * G + 7) / 8, 8 * c->sms)), dim3(256), 0, st, true, h, ids, probs, T, D, G, rank,
                                                                                          cap, El, peers,
                                                                                          my_sync + 3 * G + 1);
            // 3. the rows every rank sent here -> local routes, expert segments, GEMM tiles
            mark(l, 2);
            launch(ep_recv_routes_kernel, dim3(nbr), dim3(256), 0, st, true, my_meta, my_sync, target, G, cap, L->E_off, El, peers, il, rbc,
                                                       c->d_err);
            launch(scan_tiles_kernel, dim3(1), dim3(1024), 0, st, true, rbc, nbr, El + 1, El, RC, T, gg::BN, rbb, sgc, sgo, tiles, nt,
                                                  max_tiles, c->d_err);
            // stable scatter of the local routes and their received rows copied into expert order
            mark(l, 3);
            launch(scatter_permute_kernel<4>, dim3(nbr * 4), dim3(kScatterWarps * 32), 0, st, true, il, RC, El + 1, rbb, sgo, perm, rpos,
                                                                              my_rx, D, xp, El);
            // 4. local experts over the received rows, shared expert over the local rows
            mark(l, 4);
            launch_grouped<gg::MODE_GATE_UP>(grouped_params(gg::MODE_GATE_UP, Gm, U, SG, SU, xp, 8 * RC, h, T, perm,
                                                            tiles, nt, 8 * RC, 0, D, I, El + 1, act, 8 * RC + T,
                                                            c->d_err),
                                             L->bits, grid, st);
            mark(l, 5);
            launch_grouped<gg::MODE_DOWN>(grouped_params(gg::MODE_DOWN, Dm, Dm, SD, SD, act, 8 * RC + T, nullptr, 0,
                                                         perm, tiles, nt, 8 * RC, 0, I, D, El + 1, y, 8 * RC + T,
                                                         c->d_err),
                                          L->bits, grid, st);
            // 5. partial row sums straight back into the token owners, then the owner's combine
            mark(l, 6);
            launch(ep_reduce_send_kernel, dim3(std::min((RC + kSendWarps - 1) / kSendWarps, c->sms)), dim3(kSendWarps * 32), ep_send_smem(D), st, true, 
                y, rpos, il, my_meta, my_sync, G, rank, cap, D, El, peers, my_sync + 3 * G + 2, c->d_err);
            mark(l, 7);
            launch(ep_combine_kernel, dim3(T), dim3(256), 0, st, true, my_back, ids, El, G, cap, my_sync, target, peers, y + (size_t)8 * RC * D,
                                                 gate, D, dx, l + 1 < n_layers ? dn + (size_t)(l + 1) * D : nullptr,
                                                 eps, h, c->d_err);
            mark(l, 8);
            if (launch_check(error, capacity)) {
                ep->broken = true;  // the ranks' arrival counts no longer agree
                return -1;
            }
        }
        CK(cudaMemcpyAsync(c->h_err, c->d_err, sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
        if (dev_io) CK(cudaEventRecord(c->ev_stop, st));
        CK(cudaStreamSynchronize(st));
        // every kernel signalled its peers whatever happened, so the counts advanced by n_layers
        // steps unless a wait ran out
        ep->steps += (uint64_t)n_layers;
        if (*c->h_err) {
            if (*c->h_err & kErrTimeout) ep->broken = true;
            set_error(error, capacity, "%s", device_error_text(*c->h_err));
            return -1;
        }
        if (!dev_io) {
            CK(cudaMemcpyAsync(x, dx, (size_t)T * D * 4, cudaMemcpyDeviceToHost, st));
            if (h_trace)
                CK(cudaMemcpyAsync(h_trace, dht, (size_t)n_layers * T * D * 2, cudaMemcpyDeviceToHost, st));
            if (ids_trace)
                CK(cudaMemcpyAsync(ids_trace, dit, (size_t)n_layers * T * 8 * 4, cudaMemcpyDeviceToHost, st));
            CK(cudaEventRecord(c->ev_stop, st));
            CK(cudaStreamSynchronize(st));
        }
        float t = 0;
        CK(cudaEventElapsedTime(&t, c->ev_start, c->ev_stop));
        if (ms) *ms = t;
        if (profile) {
            for (int k = 0; k < kProfileSlots; ++k) c->last_stage_ms[k] = 0;
            for (int l = 0; l < n_layers; ++l) {
                cudaEvent_t *ev = &c->layer_events[(size_t)l * (kEpStages + 1)];
                for (int k = 0; k < kEpStages; ++k) {
                    float st_ms = 0;
                    CK(cudaEventElapsedTime(&st_ms, ev[k], ev[k + 1]));
                    c->last_stage_ms[k] += st_ms;
                }
            }
            c->have_profile = true;
        }
    } catch (const CudaFail &f) {
        set_error(error, capacity, "%s", f.what.c_str());
        return -1;
    } catch (const NcclFail &f) {
        set_error(error, capacity, "%s", f.what.c_str());
        return -1;
    }
    return 0;
}

#ifdef DI_DECODE_TIMELINE
// Profiling build only (-DDI_DECODE_TIMELINE): the decode stack kernel's per-layer timeline of two
// CTAs, [2][ds::kTlLayers][ds::kTlEvents] %globaltimer values of the last call.
API int di_debug_decode_timeline(unsigned long long *out) {
    return cudaMemcpyFromSymbol(out, ds::g_ds_tl, sizeof(ds::g_ds_tl)) == cudaSuccess ? 0 : -1;
}
#endif
#ifdef DI_GG_TIMING
// Profiling build only (-DDI_GG_TIMING): the grouped GEMMs' per-role cycle counters
// [4 kinds][256 CTAs][gg::T_COUNT], copied to out and cleared when reset != 0.
API int di_debug_gg_timing(unsigned long long *out, int reset) {
    if (cudaMemcpyFromSymbol(out, gg::g_gg_timing, sizeof(gg::g_gg_timing)) != cudaSuccess) return -1;
    if (reset) {
        static unsigned long long zero[4 * 256 * gg::T_COUNT];
        if (cudaMemcpyToSymbol(gg::g_gg_timing, zero, sizeof(zero)) != cudaSuccess) return -1;
    }
    return 0;
}
#endif

// ============================================================================ allocation-free block

namespace {
// Scratch of di_moe_block_static: one fixed array on every GPU that loads this library,
// held until the process exits. Host code must not take its address directly (that is a
// host-side stand-in); the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_static_scratch[DI_MOE_STATIC_SCRATCH_BYTES];
constexpr int kMaxStaticDevices = 64;
void *g_static_addr[kMaxStaticDevices] = {};  // device address of g_static_scratch, per device
std::mutex g_static_mutex;
}  // namespace

API int di_moe_block_static(void *ctx, void *layer, const uint16_t *x, int tokens, uint16_t *y, int32_t *ids,
                            float *probs, double *ms, char *error, int capacity) {
    if (!live_context(ctx) || !live_layer(layer)) {
        set_error(error, capacity, "Invalid context or MoE layer");
        return -1;
    }
    Context *c = static_cast<Context *>(ctx);
    Layer *L = static_cast<Layer *>(layer);
    if (L->ctx != c) {
        set_error(error, capacity, "MoE layer must belong to this device.");
        return -1;
    }
    if (!x || !y || tokens < 1 || tokens > DI_MOE_STATIC_MAX_TOKENS) {
        set_error(error, capacity, "Invalid allocation-free MoE block arguments: device x and y, 1 <= tokens <= %d",
                  DI_MOE_STATIC_MAX_TOKENS);
        return -1;
    }
    for (int i = 0; i < 8; ++i)
        if (L->m[i]->destroyed) {
            set_error(error, capacity, "MoE layer matrix was destroyed");
            return -1;
        }
    if (c->device < 0 || c->device >= kMaxStaticDevices) {
        set_error(error, capacity, "Device ordinal %d is outside the allocation-free entry's table", c->device);
        return -1;
    }
    if (!device_pointers_ok(c->device, {x, y, ids, probs})) {
        set_error(error, capacity, "Allocation-free MoE block: x, y, ids and probs must be device memory of the context's GPU");
        return -1;
    }
    // the route kernel stages the T input rows in shared memory (the same limit di_moe_block applies)
    if ((size_t)tokens * L->D * 2 > (size_t)kDecodeSmemMax) {
        set_error(error, capacity, "Decode path supports T*D <= %d; use the grouped path", kDecodeSmemMax / 2);
        return -1;
    }
    const int T = tokens, E = L->E, I = L->I;
    // carve the fixed array: the same buffers the decode path of di_moe_block uses
    BlockBuffers b{};
    b.nblocks = (T + topk::TOK_PER_CTA - 1) / topk::TOK_PER_CTA;
    Carve cv;
    const size_t o_lg = cv.take<float>((size_t)T * E), o_p = cv.take<float>((size_t)T * 8);
    const size_t o_g = cv.take<float>((size_t)T), o_ids = cv.take<int32_t>((size_t)T * 8);
    const size_t o_bc = cv.take<int32_t>((size_t)b.nblocks * E), o_a = cv.take<float>((size_t)T * 9 * I);
    const size_t o_ctr = cv.take<uint32_t>(2);
    if (cv.off > DI_MOE_STATIC_SCRATCH_BYTES) {
        set_error(error, capacity,
                  "Allocation-free MoE block needs %zu bytes of scratch for T=%d, E=%d, I=%d; the fixed array holds %u",
                  cv.off, T, E, I, (unsigned)DI_MOE_STATIC_SCRATCH_BYTES);
        return -1;
    }
    DeviceGuard dg(c->device);
    try {
        uint8_t *base = nullptr;
        {
            // once per device, with that device current: resolve the array's device address
            std::lock_guard<std::mutex> g(g_static_mutex);
            if (!g_static_addr[c->device]) {
                void *p = nullptr;
                cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
                if (e != cudaSuccess || !p) {
                    set_error(error, capacity, "cudaGetSymbolAddress(scratch) failed: %s", cudaGetErrorString(e));
                    return -1;
                }
                g_static_addr[c->device] = p;
            }
            base = static_cast<uint8_t *>(g_static_addr[c->device]);
        }
        b.logits = reinterpret_cast<float *>(base + o_lg);
        b.probs = reinterpret_cast<float *>(base + o_p);
        b.gate = reinterpret_cast<float *>(base + o_g);
        b.ids = reinterpret_cast<int32_t *>(base + o_ids);
        b.block_counts = reinterpret_cast<int32_t *>(base + o_bc);
        b.act32 = reinterpret_cast<float *>(base + o_a);
        b.counter = reinterpret_cast<uint32_t *>(base + o_ctr);
        for (int i = 0; i < 8; ++i) sync_matrix(L->m[i]);
        // every buffer above is fully rewritten by the kernels; the error word and the route
        // kernel's completion ticket must start at zero
        CK(cudaMemsetAsync(c->d_err, 0, sizeof(uint32_t), c->stream));
        CK(cudaMemsetAsync(b.counter, 0, 2 * sizeof(uint32_t), c->stream));
        CK(cudaEventRecord(c->ev_start, c->stream));
        enqueue_block(c, L, x, T, y, nullptr, nullptr, probs, true, b, false);
        if (launch_check(error, capacity)) return -1;
        if (ids) CK(cudaMemcpyAsync(ids, b.ids, (size_t)T * 8 * 4, cudaMemcpyDeviceToDevice, c->stream));
        CK(cudaMemcpyAsync(c->h_err, c->d_err, sizeof(uint32_t), cudaMemcpyDeviceToHost, c->stream));
        CK(cudaEventRecord(c->ev_stop, c->stream));
        CK(cudaStreamSynchronize(c->stream));
        if (*c->h_err) {
            set_error(error, capacity, "%s", device_error_text(*c->h_err));
            return -1;
        }
        float t = 0;
        CK(cudaEventElapsedTime(&t, c->ev_start, c->ev_stop));
        if (ms) *ms = t;
    } catch (const CudaFail &f) {
        set_error(error, capacity, "%s", f.what.c_str());
        return -1;
    }
    return 0;
}
