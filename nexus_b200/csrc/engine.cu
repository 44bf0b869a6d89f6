// engine.cu -- the CUDA backend behind include/nexus_cuda.h.
//
// Host orchestration of the decode step that InferenceEngine runs on the CPU
// in the reference (src/engine/mod.rs:539-1238): model upload, per-sequence KV
// caches, the per-token layer loop as one CUDA graph of fused kernels, greedy
// generation chained on the device, batched decode, and the generic KernelOp
// surface of Backend::execute (src/backend/mod.rs:92).
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <math.h>
#include <nccl.h>
#include <string.h>

#include <algorithm>
#include <memory>
#include <mutex>
#include <string>
#include <chrono>
#include <thread>
#include <vector>

#include "../../include/nexus_cuda.h"
#include "gguf.h"
#include "kernels.h"
#include "quant_math.cuh"
#include "tiles.cuh"
#include "trace.h"

namespace nx {
int synth_model_write(const char *path, const nexus_synth_config *cfg, std::string &err);
}

using namespace nx;

static thread_local std::string g_tls_error;

struct nexus_cuda_backend {
    nexus_cuda_config cfg;
    int device = 0;
    cudaStream_t stream = nullptr;
    std::string last_error;
    std::string step_error;  // why a collective of the step being enqueued failed
    std::mutex mu;
    // Models and resident weights keep their backend alive: destroying a
    // backend that still has children only marks it, and the last child
    // to go frees it.
    int children = 0;
    bool destroy_pending = false;
    // set by a kernel whose bounded wait gave up (op-level calls)
    int *dev_err = nullptr;
    // tensor parallelism (nexus_cuda_tp_init)
    int tp_rank = 0, tp_world = 1;
    ncclComm_t comm = nullptr;
    // one-shot peer-memory all-reduce of the hidden state (kernels_peer.cu):
    // this rank's staging buffers and flags, the peers' mapped through CUDA IPC
    bool peer_ok = false;
    bool tp_failed = false;
    PeerReduce peer = {};
    float *peer_buf = nullptr;        // [2][max_floats]
    unsigned *peer_flags = nullptr;   // [kPeerCtas][2]
    unsigned *peer_epoch = nullptr;   // [kPeerCtas]
    std::vector<void *> peer_mapped;  // peers' buffers opened with cudaIpcOpenMemHandle
};

// NCCL is opened at nexus_cuda_tp_init (no link-time dependency).
struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
    // for a bounded wait on the ranks joining (optional: without them the
    // join waits as long as ncclCommInitRank does)
    ncclResult_t (*comm_init_rank_config)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
    ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
    bool ok = false;
};

static NcclApi *nccl_api(std::string *why) {
    static NcclApi api;
    static std::once_flag once;
    static std::string load_error;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            load_error = std::string("cannot load NCCL: ") + dlerror();
            return;
        }
        api.get_unique_id = (decltype(api.get_unique_id))dlsym(h, "ncclGetUniqueId");
        api.comm_init_rank = (decltype(api.comm_init_rank))dlsym(h, "ncclCommInitRank");
        api.all_reduce = (decltype(api.all_reduce))dlsym(h, "ncclAllReduce");
        api.all_gather = (decltype(api.all_gather))dlsym(h, "ncclAllGather");
        api.comm_destroy = (decltype(api.comm_destroy))dlsym(h, "ncclCommDestroy");
        api.error_string = (decltype(api.error_string))dlsym(h, "ncclGetErrorString");
        api.comm_init_rank_config = (decltype(api.comm_init_rank_config))dlsym(h, "ncclCommInitRankConfig");
        api.get_async_error = (decltype(api.get_async_error))dlsym(h, "ncclCommGetAsyncError");
        api.comm_abort = (decltype(api.comm_abort))dlsym(h, "ncclCommAbort");
        api.ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.all_gather && api.comm_destroy &&
                 api.error_string;
        if (!api.ok) load_error = "NCCL library lacks a required symbol";
    });
    if (!api.ok && why) *why = load_error;
    return api.ok ? &api : nullptr;
}

static std::mutex g_backend_mu;

static void peer_release(nexus_cuda_backend *b) {
    for (void *p : b->peer_mapped) cudaIpcCloseMemHandle(p);
    b->peer_mapped.clear();
    if (b->peer_buf) cudaFree(b->peer_buf);
    if (b->peer_flags) cudaFree(b->peer_flags);
    if (b->peer_epoch) cudaFree(b->peer_epoch);
    b->peer_buf = nullptr;
    b->peer_flags = nullptr;
    b->peer_epoch = nullptr;
    b->peer_ok = false;
}

static void backend_free_now(nexus_cuda_backend *b) {
    cudaSetDevice(b->device);
    if (b->stream) {
        cudaStreamSynchronize(b->stream);
        cudaStreamDestroy(b->stream);
    }
    if (b->dev_err) cudaFree(b->dev_err);
    peer_release(b);
    if (b->comm) {
        if (NcclApi *api = nccl_api(nullptr)) api->comm_destroy(b->comm);
    }
    delete b;
}

static void backend_retain(nexus_cuda_backend *b) {
    std::lock_guard<std::mutex> lk(g_backend_mu);
    b->children++;
}

static void backend_release(nexus_cuda_backend *b) {
    bool free_now = false;
    {
        std::lock_guard<std::mutex> lk(g_backend_mu);
        b->children--;
        free_now = b->children == 0 && b->destroy_pending;
    }
    if (free_now) backend_free_now(b);
}

static int set_err(nexus_cuda_backend *b, int code, const std::string &msg) {
    if (b) b->last_error = msg;
    g_tls_error = msg;
    return code;
}

// A failed allocation is reported as NEXUS_E_OOM (and cleared: it does not
// poison the context); any other CUDA error as NEXUS_E_CUDA.
#define NX_CUDA(b, call)                                                                        \
    do {                                                                                        \
        cudaError_t e_ = (call);                                                                \
        if (e_ == cudaErrorMemoryAllocation) {                                                  \
            cudaGetLastError();                                                                 \
            return set_err((b), NEXUS_E_OOM, std::string(#call) + ": " + cudaGetErrorString(e_)); \
        }                                                                                       \
        if (e_ != cudaSuccess)                                                                  \
            return set_err((b), NEXUS_E_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

// ---------------------------------------------------------------------------
// device allocation helper
// ---------------------------------------------------------------------------
template <typename T>
static cudaError_t dalloc(T **p, size_t count) {
    *p = nullptr;
    if (count == 0) count = 1;
    return cudaMalloc((void **)p, count * sizeof(T));
}

struct Mat {
    int fmt = -1;
    int n = 0, k = 0;
    uint4 *main = nullptr;
    uint32_t *aux = nullptr;
    size_t bytes = 0;  // main + aux bytes (streamed per use)
    void release() {
        if (main) cudaFree(main);
        if (aux) cudaFree(aux);
        main = nullptr;
        aux = nullptr;
    }
};

// Upload rows x k raw block bytes (already row-permuted) and repack to tiles.
static int make_mat(nexus_cuda_backend *b, int fmt, int n, int k, const uint8_t *raw_host, Mat &m) {
    if (!tile_supported(fmt)) return set_err(b, NEXUS_E_UNSUPPORTED_FORMAT, "matrix format not supported by the GEMV");
    if (k % 256 != 0) return set_err(b, NEXUS_E_INVALID, "matrix columns must be a multiple of 256");
    m.fmt = fmt;
    m.n = n;
    m.k = k;
    size_t mb = tile_main_bytes(fmt, n, k), ab = tile_aux_bytes(fmt, n, k);
    size_t rawb = format_bytes(fmt, (size_t)n * k);
    NX_CUDA(b, dalloc((uint8_t **)&m.main, mb));
    if (ab) NX_CUDA(b, dalloc((uint8_t **)&m.aux, ab));
    m.bytes = mb + ab;
    uint8_t *draw = nullptr;
    NX_CUDA(b, dalloc(&draw, rawb));
    cudaError_t e = cudaMemcpyAsync(draw, raw_host, rawb, cudaMemcpyHostToDevice, b->stream);
    if (e == cudaSuccess) e = launch_repack_tiles(fmt, draw, n, k, m.main, m.aux, b->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
    cudaFree(draw);
    if (e != cudaSuccess) return set_err(b, NEXUS_E_CUDA, std::string("repack: ") + cudaGetErrorString(e));
    return NEXUS_OK;
}

// K-split scratch for an N-row GEMV of up to 4 tokens: 8 slices of partials.
// Batches of at least this many tokens run on the tensor-core GEMM.
static constexpr int kGemmMinM = 8;

// Grow one scratch buffer to `need` elements.  A zeroed buffer is cleared
// on `st`, so the clear is ordered before the kernels that read it.
template <typename T>
static cudaError_t grow(T **p, size_t *cap, size_t need, bool zero, cudaStream_t st) {
    if (need <= *cap) return cudaSuccess;
    if (*p) {
        cudaStreamSynchronize(st);
        cudaFree(*p);
    }
    *p = nullptr;
    *cap = 0;
    cudaError_t e = dalloc(p, need);
    if (e != cudaSuccess) return e;
    if (zero) e = cudaMemsetAsync(*p, 0, need * sizeof(T), st);
    if (e == cudaSuccess) *cap = need;
    return e;
}

// Scratch of the tcgen05 GEMM: prepared activations, token scales, K-split
// partials and self-resetting tile counters (zero between launches).
struct LinScratch {
    uint8_t *bimg = nullptr;
    size_t bimg_cap = 0;
    float *scale = nullptr;
    size_t scale_cap = 0;
    float *part = nullptr;
    size_t part_cap = 0;
    unsigned *count = nullptr;
    size_t count_cap = 0;
    cudaError_t ensure(int m, int n, int k, cudaStream_t st) {
        const GemmScratchSize z = gemm_scratch_size(m, n, k);
        cudaError_t e = grow(&bimg, &bimg_cap, z.bimg_bytes, false, st);
        if (e == cudaSuccess) e = grow(&scale, &scale_cap, z.tok_scale_floats, false, st);
        if (e == cudaSuccess) e = grow(&part, &part_cap, z.part_floats, false, st);
        if (e == cudaSuccess) e = grow(&count, &count_cap, z.counter_slots, true, st);
        return e;
    }
    void attach(GemvParams &p, GemmScratch &sc) const {
        p.part = part;
        p.part_floats = part_cap;
        p.counters = count;
        p.counter_slots = (int)count_cap;
        sc = {bimg, bimg_cap, scale, scale_cap};
    }
    void release() {
        if (bimg) cudaFree(bimg);
        if (scale) cudaFree(scale);
        if (part) cudaFree(part);
        if (count) cudaFree(count);
        *this = LinScratch();
    }
};

// y[m][n] = x[m][k] * W^T on device buffers: the tensor-core GEMM for
// batches of kGemmMinM+ tokens in a format it covers, else the GEMV.
static cudaError_t run_qmatvec(const Mat &mat, const float *x, int m, float *y, LinScratch &ls, int *err,
                               cudaStream_t st) {
    GemvParams p = {};
    p.fmt = mat.fmt;
    p.w_main = mat.main;
    p.w_aux = mat.aux;
    p.n = mat.n;
    p.k = mat.k;
    p.m = m;
    p.x = x;
    p.x_stride = mat.k;
    p.epi = EPI_STORE;
    p.y = y;
    p.y_stride = mat.n;
    p.err = err;
    if (m >= kGemmMinM && gemm_supported(mat.fmt)) {
        cudaError_t e = ls.ensure(m, mat.n, mat.k, st);
        if (e != cudaSuccess) return e;
        GemmScratch sc;
        ls.attach(p, sc);
        return launch_gemm(p, sc, st);
    }
    return launch_gemv(p, st);
}

// ---------------------------------------------------------------------------
// backend
// ---------------------------------------------------------------------------
// Internal accessors for other translation units of the library.
int nexus_backend_stream_device(nexus_cuda_backend *b, cudaStream_t *stream, int *device) {
    if (!b) return NEXUS_E_INVALID;
    *stream = b->stream;
    *device = b->device;
    return NEXUS_OK;
}

int nexus_backend_fail(nexus_cuda_backend *b, int code, const char *msg) { return set_err(b, code, msg); }

extern "C" void nexus_cuda_config_default(nexus_cuda_config *cfg) {
    memset(cfg, 0, sizeof(*cfg));
    cfg->device = 0;
    cfg->tp = 1;
    cfg->max_batch = 1;
    cfg->page_tokens = 16;
}

extern "C" int nexus_cuda_is_available(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return 0;
    }
    for (int i = 0; i < n; i++) {
        cudaDeviceProp p;
        if (cudaGetDeviceProperties(&p, i) == cudaSuccess && p.major == 10) return 1;
    }
    return 0;
}

extern "C" int nexus_cuda_capabilities(nexus_cuda_caps *caps) {
    if (!caps) return NEXUS_E_INVALID;
    memset(caps, 0, sizeof(*caps));
    caps->backend = "cuda";
    caps->available = nexus_cuda_is_available();
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    caps->device_count = n;
    static const char *features[] = {"sm_100a", "tile-gemv-dp4a", "pdl", "cuda-graphs", "packed-kv", "gqa-split-k"};
    static const char *ops[] = {"matmul", "attention", "rms_norm", "layer_norm", "softmax", "quantize", "dequantize"};
    if (caps->available) {
        for (const char *f : features) caps->features[caps->n_features++] = f;
        for (const char *o : ops) caps->supported_ops[caps->n_supported_ops++] = o;
    }
    return NEXUS_OK;
}

extern "C" int nexus_cuda_backend_create(const nexus_cuda_config *cfg, nexus_cuda_backend **out) {
    if (!out) return set_err(nullptr, NEXUS_E_INVALID, "out is NULL");
    *out = nullptr;
    nexus_cuda_config c;
    if (cfg) c = *cfg;
    else nexus_cuda_config_default(&c);
    if (c.tp < 1) c.tp = 1;
    if (c.max_batch < 1) c.max_batch = 1;
    if (c.page_tokens == 0) c.page_tokens = 16;
    if (c.tp != 1)
        return set_err(nullptr, NEXUS_E_INVALID,
                       "tensor parallelism runs one process per GPU: create each backend with tp 1, then nexus_cuda_tp_init");
    if ((c.kv_bits_k == 0) != (c.kv_bits_v == 0)) return set_err(nullptr, NEXUS_E_INVALID, "kv_bits_k and kv_bits_v must both be 0 or both set");
    if (c.kv_bits_k > 8 || c.kv_bits_v > 8) return set_err(nullptr, NEXUS_E_INVALID, "packed KV supports 1..8 bits");
    if (!nexus_cuda_is_available()) return set_err(nullptr, NEXUS_E_UNAVAILABLE, "no sm_100 CUDA device");
    int ndev = 0;
    cudaGetDeviceCount(&ndev);
    if (c.device < 0 || c.device >= ndev) return set_err(nullptr, NEXUS_E_INVALID, "bad device ordinal");
    auto *b = new nexus_cuda_backend();
    b->cfg = c;
    b->device = c.device;
    cudaError_t e = cudaSetDevice(c.device);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc((void **)&b->dev_err, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(b->dev_err, 0, sizeof(int));
    if (e != cudaSuccess) {
        if (b->stream) cudaStreamDestroy(b->stream);
        delete b;
        return set_err(nullptr, NEXUS_E_CUDA, std::string("backend init: ") + cudaGetErrorString(e));
    }
    *out = b;
    return NEXUS_OK;
}

extern "C" int nexus_cuda_backend_destroy(nexus_cuda_backend *b) {
    if (!b) return NEXUS_OK;
    {
        std::lock_guard<std::mutex> lk(g_backend_mu);
        if (b->destroy_pending) return NEXUS_OK;
        b->destroy_pending = true;
        if (b->children > 0) return NEXUS_OK;
    }
    backend_free_now(b);
    return NEXUS_OK;
}

extern "C" const char *nexus_cuda_backend_name(const nexus_cuda_backend *) { return "cuda"; }

extern "C" int nexus_cuda_memory_info(nexus_cuda_backend *b, size_t *total, size_t *free_bytes, size_t *used) {
    if (!b) return set_err(nullptr, NEXUS_E_INVALID, "backend is NULL");
    cudaSetDevice(b->device);
    size_t f = 0, t = 0;
    NX_CUDA(b, cudaMemGetInfo(&f, &t));
    if (total) *total = t;
    if (free_bytes) *free_bytes = f;
    if (used) *used = t - f;
    return NEXUS_OK;
}

// After a synchronize: report (and clear) a bounded wait that gave up.
static int check_dev_err(nexus_cuda_backend *b) {
    int v = 0;
    NX_CUDA(b, cudaMemcpy(&v, b->dev_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (v) {
        cudaMemset(b->dev_err, 0, sizeof(int));
        return set_err(b, NEXUS_E_TIMEOUT, "a kernel's bounded wait gave up (asynchronous copy or MMA never completed)");
    }
    return NEXUS_OK;
}

extern "C" int nexus_cuda_synchronize(nexus_cuda_backend *b) {
    if (!b) return set_err(nullptr, NEXUS_E_INVALID, "backend is NULL");
    cudaSetDevice(b->device);
    NX_CUDA(b, cudaStreamSynchronize(b->stream));
    return check_dev_err(b);
}

extern "C" int nexus_tp_plan(uint32_t Hq, uint32_t Hkv, uint32_t D, uint32_t F, uint32_t V, int rank, int world,
                             nexus_tp_slice *out) {
    if (!out || world < 1 || rank < 0 || rank >= world || !Hq || !Hkv || !D || !F || !V)
        return set_err(nullptr, NEXUS_E_INVALID, "tp plan: bad argument");
    const uint32_t w = (uint32_t)world;
    if (Hq % w || Hkv % w || F % w || V % w)
        return set_err(nullptr, NEXUS_E_INVALID, "tp plan: heads, FFN rows and vocab rows must divide by the world size");
    const uint32_t hq = Hq / w, hkv = Hkv / w, f = F / w, v = V / w;
    if (w > 1 && ((hq * D) % 256 || f % 256 || v % 32))
        return set_err(nullptr, NEXUS_E_INVALID,
                       "tp plan: per-rank attention and FFN column slices must be whole 256-element super-blocks "
                       "and vocab slices whole 32-row groups");
    out->q_head_begin = (uint32_t)rank * hq;
    out->q_heads = hq;
    out->kv_head_begin = (uint32_t)rank * hkv;
    out->kv_heads = hkv;
    out->ffn_begin = (uint32_t)rank * f;
    out->ffn_rows = f;
    out->vocab_begin = (uint32_t)rank * v;
    out->vocab_rows = v;
    return NEXUS_OK;
}

extern "C" int nexus_cuda_tp_unique_id(void *id, size_t id_bytes) {
    if (!id || id_bytes < sizeof(ncclUniqueId)) return set_err(nullptr, NEXUS_E_INVALID, "tp id buffer too small");
    std::string why;
    NcclApi *api = nccl_api(&why);
    if (!api) return set_err(nullptr, NEXUS_E_COMM, why);
    ncclUniqueId u;
    ncclResult_t r = api->get_unique_id(&u);
    if (r != ncclSuccess) return set_err(nullptr, NEXUS_E_COMM, std::string("ncclGetUniqueId: ") + api->error_string(r));
    memcpy(id, &u, sizeof(u));
    return NEXUS_OK;
}

// Polls a nonblocking communicator's pending call (on the host) until it
// settles or `limit_ms` passes; ncclInProgress means the limit passed.
static ncclResult_t nccl_settle(NcclApi *api, ncclComm_t *comm, ncclResult_t r, uint32_t limit_ms) {
    const auto t0 = std::chrono::steady_clock::now();
    while (r == ncclInProgress) {
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
        if (ms.count() > (long long)limit_ms) return ncclInProgress;
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
        ncclResult_t st = ncclSuccess;
        const ncclResult_t q = *comm ? api->get_async_error(*comm, &st) : ncclInvalidArgument;
        r = q != ncclSuccess ? q : st;
    }
    return r;
}

// Staging buffers and flags for the one-shot all-reduce, mapped into every
// peer: each rank's CUDA IPC handles are all-gathered over NCCL and opened.
static constexpr size_t kPeerMaxFloats = 1u << 20;  // 4 MB: up to 256 tokens of H = 4096
static cudaError_t peer_setup(nexus_cuda_backend *b, NcclApi *api) {
    const int world = b->tp_world, rank = b->tp_rank;
    cudaError_t e = dalloc(&b->peer_buf, 2 * kPeerMaxFloats);
    if (e == cudaSuccess) e = dalloc(&b->peer_flags, (size_t)2 * kPeerCtas);
    if (e == cudaSuccess) e = dalloc(&b->peer_epoch, (size_t)kPeerCtas);
    if (e == cudaSuccess) e = cudaMemset(b->peer_flags, 0, (size_t)2 * kPeerCtas * 4);
    if (e == cudaSuccess) e = cudaMemset(b->peer_epoch, 0, (size_t)kPeerCtas * 4);
    if (e != cudaSuccess) return e;
    cudaIpcMemHandle_t h[2];
    if ((e = cudaIpcGetMemHandle(&h[0], b->peer_buf)) != cudaSuccess) return e;
    if ((e = cudaIpcGetMemHandle(&h[1], b->peer_flags)) != cudaSuccess) return e;
    uint8_t *dh = nullptr;
    const size_t hb = sizeof(h);
    if ((e = dalloc(&dh, (size_t)world * hb)) != cudaSuccess) return e;
    std::vector<uint8_t> all((size_t)world * hb);
    e = cudaMemcpy(dh + (size_t)rank * hb, h, hb, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        ncclResult_t r = api->all_gather(dh + (size_t)rank * hb, dh, hb, ncclUint8, b->comm, b->stream);
        e = r == ncclSuccess ? cudaStreamSynchronize(b->stream) : cudaErrorUnknown;
    }
    if (e == cudaSuccess) e = cudaMemcpy(all.data(), dh, all.size(), cudaMemcpyDeviceToHost);
    cudaFree(dh);
    if (e != cudaSuccess) return e;
    PeerReduce &pr = b->peer;
    pr = PeerReduce{};
    for (int r = 0; r < world; r++) {
        if (r == rank) {
            pr.bufs[r][0] = b->peer_buf;
            pr.bufs[r][1] = b->peer_buf + kPeerMaxFloats;
            pr.flags[r] = b->peer_flags;
            continue;
        }
        cudaIpcMemHandle_t ph[2];
        memcpy(ph, all.data() + (size_t)r * hb, hb);
        void *pb = nullptr, *pf = nullptr;
        if ((e = cudaIpcOpenMemHandle(&pb, ph[0], cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess) return e;
        b->peer_mapped.push_back(pb);
        if ((e = cudaIpcOpenMemHandle(&pf, ph[1], cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess) return e;
        b->peer_mapped.push_back(pf);
        pr.bufs[r][0] = static_cast<float *>(pb);
        pr.bufs[r][1] = static_cast<float *>(pb) + kPeerMaxFloats;
        pr.flags[r] = static_cast<unsigned *>(pf);
    }
    pr.epoch = b->peer_epoch;
    pr.rank = rank;
    pr.world = world;
    pr.max_floats = kPeerMaxFloats;
    // every rank has mapped every peer before the first all-reduce
    ncclResult_t r = api->all_reduce(b->peer_epoch, b->peer_epoch, 1, ncclUint32, ncclMax, b->comm, b->stream);
    e = r == ncclSuccess ? cudaStreamSynchronize(b->stream) : cudaErrorUnknown;
    if (e == cudaSuccess) b->peer_ok = true;
    return e;
}

extern "C" int nexus_cuda_tp_allreduce_kind(const nexus_cuda_backend *b) {
    if (!b || b->tp_world < 2) return NEXUS_TP_NONE;
    return b->peer_ok ? NEXUS_TP_PEER : NEXUS_TP_NCCL;
}

extern "C" int nexus_cuda_tp_init(nexus_cuda_backend *b, int rank, int world, const void *id, size_t id_bytes) {
    if (!b || !id || id_bytes < sizeof(ncclUniqueId) || world < 1 || rank < 0 || rank >= world)
        return set_err(b, NEXUS_E_INVALID, "tp init: bad argument");
    if (b->comm) return set_err(b, NEXUS_E_INVALID, "tp init: already initialised");
    if (world == 1) return NEXUS_OK;
    std::string why;
    NcclApi *api = nccl_api(&why);
    if (!api) return set_err(b, NEXUS_E_COMM, why);
    cudaSetDevice(b->device);
    ncclUniqueId u;
    memcpy(&u, id, sizeof(u));
    const uint32_t limit_ms = b->cfg.tp_timeout_ms ? b->cfg.tp_timeout_ms : 120000u;
    if (api->comm_init_rank_config && api->get_async_error && api->comm_abort) {
        // Join on a nonblocking communicator, polled against the limit, so a
        // rank that never arrives ends the join with NEXUS_E_COMM.
        ncclConfig_t nb = NCCL_CONFIG_INITIALIZER;
        nb.blocking = 0;
        ncclComm_t boot = nullptr;
        ncclResult_t r = nccl_settle(api, &boot, api->comm_init_rank_config(&boot, world, u, rank, &nb), limit_ms);
        if (r != ncclSuccess) {
            if (boot) api->comm_abort(boot);
            cudaGetLastError();
            if (r == ncclInProgress)
                return set_err(b, NEXUS_E_COMM, "tp init: not every rank joined within " + std::to_string(limit_ms) +
                                                     " ms (group torn down on this rank)");
            return set_err(b, NEXUS_E_COMM, std::string("ncclCommInitRankConfig: ") + api->error_string(r));
        }
        // Every rank has joined.  The decode steps need a blocking
        // communicator (their collectives are captured in CUDA graphs): rank 0
        // draws a second id, the joining communicator carries it to every rank
        // (a byte-wise sum in which the other ranks contribute zeros), and each
        // rank builds the step communicator from it with ncclCommInitRank.
        ncclUniqueId u2 = {};
        if (rank == 0 && (r = api->get_unique_id(&u2)) != ncclSuccess) {
            api->comm_abort(boot);
            return set_err(b, NEXUS_E_COMM, std::string("ncclGetUniqueId: ") + api->error_string(r));
        }
        uint8_t *dbuf = nullptr;
        cudaError_t ce = dalloc(&dbuf, sizeof(u2));
        if (ce == cudaSuccess) ce = cudaMemcpy(dbuf, &u2, sizeof(u2), cudaMemcpyHostToDevice);
        if (ce == cudaSuccess) {
            r = api->all_reduce(dbuf, dbuf, sizeof(u2), ncclUint8, ncclSum, boot, b->stream);
            if (r == ncclInProgress) r = nccl_settle(api, &boot, r, limit_ms);
            // the reduction itself, bounded like the join
            const auto t0 = std::chrono::steady_clock::now();
            while (r == ncclSuccess && (ce = cudaStreamQuery(b->stream)) == cudaErrorNotReady) {
                const auto ms =
                    std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
                if (ms.count() > (long long)limit_ms) {
                    r = ncclInProgress;
                    break;
                }
                std::this_thread::sleep_for(std::chrono::milliseconds(1));
            }
            if (r == ncclSuccess && ce == cudaSuccess) ce = cudaMemcpy(&u2, dbuf, sizeof(u2), cudaMemcpyDeviceToHost);
        }
        api->comm_abort(boot);
        if (dbuf) cudaFree(dbuf);
        if (r != ncclSuccess || ce != cudaSuccess) {
            cudaGetLastError();
            if (r == ncclInProgress)
                return set_err(b, NEXUS_E_COMM, "tp init: the second id did not reach every rank within " +
                                                     std::to_string(limit_ms) + " ms");
            return set_err(b, NEXUS_E_COMM, r != ncclSuccess ? std::string("tp init id exchange: ") + api->error_string(r)
                                                             : std::string("tp init id exchange: ") + cudaGetErrorString(ce));
        }
        ncclComm_t comm = nullptr;
        r = api->comm_init_rank(&comm, world, u2, rank);
        if (r != ncclSuccess || !comm) {
            if (comm) api->comm_abort(comm);
            cudaGetLastError();
            return set_err(b, NEXUS_E_COMM, std::string("ncclCommInitRank: ") + api->error_string(r));
        }
        b->comm = comm;
    } else {
        ncclResult_t r = api->comm_init_rank(&b->comm, world, u, rank);
        if (r != ncclSuccess) {
            b->comm = nullptr;
            return set_err(b, NEXUS_E_COMM, std::string("ncclCommInitRank: ") + api->error_string(r));
        }
    }
    b->tp_rank = rank;
    b->tp_world = world;
    if (!(b->cfg.flags & NEXUS_CFG_NCCL_ALLREDUCE) && world <= kPeerMaxRanks) {
        // the peer-memory all-reduce; on any failure the NCCL all-reduce stays in use
        if (peer_setup(b, api) != cudaSuccess) {
            peer_release(b);
            cudaGetLastError();
        }
    }
    return NEXUS_OK;
}

extern "C" const char *nexus_cuda_last_error(const nexus_cuda_backend *b) {
    return b ? b->last_error.c_str() : g_tls_error.c_str();
}

// ---------------------------------------------------------------------------
// Backend::execute
// ---------------------------------------------------------------------------
namespace {
// Device view of an op operand: copies host data in (and out) when needed.
struct DevArg {
    void *d = nullptr;
    bool owned = false;
    ~DevArg() {
        if (owned && d) cudaFree(d);
    }
};
cudaError_t stage_in(const void *p, size_t bytes, bool device, DevArg &a, cudaStream_t st) {
    if (device || !p) {
        a.d = const_cast<void *>(p);
        return cudaSuccess;
    }
    cudaError_t e = cudaMalloc(&a.d, bytes ? bytes : 1);
    if (e != cudaSuccess) return e;
    a.owned = true;
    return bytes ? cudaMemcpyAsync(a.d, p, bytes, cudaMemcpyHostToDevice, st) : cudaSuccess;
}
cudaError_t stage_out(void *p, size_t bytes, bool device, DevArg &a) {
    if (device) {
        a.d = p;
        return cudaSuccess;
    }
    cudaError_t e = cudaMalloc(&a.d, bytes ? bytes : 1);
    a.owned = e == cudaSuccess;
    return e;
}
}  // namespace

extern "C" int nexus_cuda_execute(nexus_cuda_backend *b, const nexus_op *op) {
    if (!b || !op) return set_err(b, NEXUS_E_INVALID, "NULL backend or op");
    std::lock_guard<std::mutex> lk(b->mu);
    cudaSetDevice(b->device);
    cudaStream_t st = b->stream;
    const bool dev = op->device_ptrs != 0;
    DevArg A, B, Cc, O;
    size_t out_bytes = 0;
    cudaError_t e = cudaSuccess;
    switch (op->kind) {
    case NEXUS_OP_MATMUL: {
        size_t m = op->m, n = op->n, k = op->k;
        out_bytes = m * n * 4;
        NX_CUDA(b, stage_in(op->a, m * k * 4, dev, A, st));
        NX_CUDA(b, stage_in(op->b, n * k * 4, dev, B, st));
        NX_CUDA(b, stage_out(op->out, out_bytes, dev, O));
        e = launch_matmul_f32((const float *)A.d, (const float *)B.d, (float *)O.d, (int)m, (int)n, (int)k,
                              op->transpose_b, st);
        break;
    }
    case NEXUS_OP_RMS_NORM:
    case NEXUS_OP_LAYER_NORM: {
        size_t rows = op->m ? op->m : 1, n = op->n;
        out_bytes = rows * n * 4;
        NX_CUDA(b, stage_in(op->a, out_bytes, dev, A, st));
        NX_CUDA(b, stage_in(op->b, n * 4, dev, B, st));
        if (op->kind == NEXUS_OP_LAYER_NORM) NX_CUDA(b, stage_in(op->c, op->c ? n * 4 : 0, dev, Cc, st));
        NX_CUDA(b, stage_out(op->out, out_bytes, dev, O));
        if (op->kind == NEXUS_OP_RMS_NORM)
            e = launch_rms_norm((const float *)A.d, (const float *)B.d, (float *)O.d, (int)rows, (int)n, op->eps, st);
        else
            e = launch_layer_norm((const float *)A.d, (const float *)B.d, (const float *)Cc.d, (float *)O.d,
                                  (int)rows, (int)n, op->eps, st);
        break;
    }
    case NEXUS_OP_SOFTMAX: {
        size_t rows = op->m ? op->m : 1, n = op->n;
        out_bytes = rows * n * 4;
        NX_CUDA(b, stage_in(op->a, out_bytes, dev, A, st));
        NX_CUDA(b, stage_out(op->out, out_bytes, dev, O));
        e = launch_softmax((const float *)A.d, (float *)O.d, (int)rows, (int)n, st);
        break;
    }
    case NEXUS_OP_ADD:
    case NEXUS_OP_MUL: {
        out_bytes = op->len * 4;
        NX_CUDA(b, stage_in(op->a, out_bytes, dev, A, st));
        NX_CUDA(b, stage_in(op->b, out_bytes, dev, B, st));
        NX_CUDA(b, stage_out(op->out, out_bytes, dev, O));
        e = launch_binary(op->kind == NEXUS_OP_ADD ? 0 : 1, (const float *)A.d, (const float *)B.d, (float *)O.d,
                          op->len, st);
        break;
    }
    case NEXUS_OP_QUANTIZE: {
        if (!format_supported(op->format) || op->format == F32 || op->format == F16 || op->format == BF16)
            return set_err(b, NEXUS_E_UNSUPPORTED_FORMAT, "quantize: format must be Q8_0/Q4_0/Q4_K/Q2_K");
        out_bytes = format_bytes(op->format, op->len);
        NX_CUDA(b, stage_in(op->a, op->len * 4, dev, A, st));
        NX_CUDA(b, stage_out(op->out, out_bytes, dev, O));
        e = launch_quantize(op->format, (const float *)A.d, op->len, (uint8_t *)O.d, st);
        break;
    }
    case NEXUS_OP_DEQUANTIZE: {
        if (!format_supported(op->format)) return set_err(b, NEXUS_E_UNSUPPORTED_FORMAT, "dequantize: unsupported format");
        size_t need = format_bytes(op->format, op->len);
        // tensor_bytes_to_f32 rejects payloads shorter than their block count
        if (op->m && op->m < need) return set_err(b, NEXUS_E_TRUNCATED, "payload is truncated");
        out_bytes = op->len * 4;
        NX_CUDA(b, stage_in(op->a, need, dev, A, st));
        NX_CUDA(b, stage_out(op->out, out_bytes, dev, O));
        e = launch_dequant_raw(op->format, (const uint8_t *)A.d, op->len, (float *)O.d, st);
        break;
    }
    case NEXUS_OP_QMATVEC: {
        size_t m = op->m, n = op->n, k = op->k;
        if (!tile_supported(op->format)) return set_err(b, NEXUS_E_UNSUPPORTED_FORMAT, "qmatvec: unsupported format");
        if (k % 256) return set_err(b, NEXUS_E_INVALID, "qmatvec: k must be a multiple of 256");
        size_t wbytes = format_bytes(op->format, n * k);
        std::vector<uint8_t> hostw;
        const uint8_t *wsrc = (const uint8_t *)op->b;
        if (dev) {
            hostw.resize(wbytes);
            NX_CUDA(b, cudaMemcpy(hostw.data(), op->b, wbytes, cudaMemcpyDeviceToHost));
            wsrc = hostw.data();
        }
        Mat mat;
        int rc = make_mat(b, op->format, (int)n, (int)k, wsrc, mat);
        if (rc) return rc;
        out_bytes = m * n * 4;
        NX_CUDA(b, stage_in(op->a, m * k * 4, dev, A, st));
        NX_CUDA(b, stage_out(op->out, out_bytes, dev, O));
        LinScratch ls;
        e = run_qmatvec(mat, (const float *)A.d, (int)m, (float *)O.d, ls, b->dev_err, st);
        cudaError_t e2 = cudaStreamSynchronize(st);
        ls.release();
        mat.release();
        if (e == cudaSuccess) e = e2;
        if (e == cudaSuccess) {
            int rc2 = check_dev_err(b);
            if (rc2) return rc2;
        }
        break;
    }
    case NEXUS_OP_ROPE: {
        size_t heads = op->m, hd = op->k;
        out_bytes = heads * hd * 4;
        if (hd % 2) return set_err(b, NEXUS_E_INVALID, "rope: head_dim must be even");
        NX_CUDA(b, stage_in(op->a, out_bytes, dev, A, st));
        O.d = A.d;
        e = launch_rope((float *)A.d, (int)heads, (int)hd, (int)op->position, op->scale, st);
        if (e == cudaSuccess && !dev) {
            NX_CUDA(b, cudaMemcpyAsync(op->out ? op->out : (void *)op->a, A.d, out_bytes, cudaMemcpyDeviceToHost, st));
            NX_CUDA(b, cudaStreamSynchronize(st));
            return NEXUS_OK;
        }
        if (e == cudaSuccess && op->out && op->out != op->a)
            e = cudaMemcpyAsync(op->out, A.d, out_bytes, cudaMemcpyDeviceToDevice, st);
        O.d = nullptr;
        out_bytes = 0;
        break;
    }
    case NEXUS_OP_ARGMAX: {
        NX_CUDA(b, stage_in(op->a, op->len * 4, dev, A, st));
        unsigned long long *best = nullptr;
        NX_CUDA(b, dalloc(&best, 1));
        e = launch_argmax((const float *)A.d, op->len, best, st);
        unsigned long long hb = 0;
        if (e == cudaSuccess) e = cudaMemcpyAsync(&hb, best, 8, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        cudaFree(best);
        if (e != cudaSuccess) return set_err(b, NEXUS_E_CUDA, cudaGetErrorString(e));
        uint32_t tok = (uint32_t)(hb & 0xffffffffull);
        if (dev) NX_CUDA(b, cudaMemcpy(op->out, &tok, 4, cudaMemcpyHostToDevice));
        else memcpy(op->out, &tok, 4);
        return NEXUS_OK;
    }
    case NEXUS_OP_KV_QUANTIZE: {
        const size_t n = op->len, bits = op->k;
        if (n == 0 || bits < 1 || bits > 8) return set_err(b, NEXUS_E_INVALID, "kv_quantize: 1..8 bits, len > 0");
        const size_t bpt = (n * bits + 7) / 8;
        out_bytes = bpt + 8;
        float *scratch = nullptr, *mins = nullptr;
        uint8_t *data = nullptr;
        DevSeq *ds = nullptr;
        uint32_t *sid = nullptr;
        NX_CUDA(b, dalloc(&scratch, 2 * n));
        NX_CUDA(b, dalloc(&mins, 4));
        NX_CUDA(b, dalloc(&data, 2 * bpt + 16));
        NX_CUDA(b, dalloc(&ds, 1));
        NX_CUDA(b, dalloc(&sid, 1));
        NX_CUDA(b, cudaMemsetAsync(ds, 0, sizeof(DevSeq), st));
        NX_CUDA(b, cudaMemsetAsync(sid, 0, 4, st));
        NX_CUDA(b, cudaMemcpyAsync(scratch, op->a, n * 4, dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st));
        NX_CUDA(b, cudaMemcpyAsync(scratch + n, op->a, n * 4, dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st));
        KvPackParams kp = {};
        kp.m = 1;
        kp.kv_dim = (int)n;
        kp.bits_k = kp.bits_v = (int)bits;
        kp.kv_scratch = scratch;
        kp.kp_data = data;
        kp.vp_data = data + bpt + 8;
        kp.kp_min = mins;
        kp.kp_scale = mins + 1;
        kp.vp_min = mins + 2;
        kp.vp_scale = mins + 3;
        kp.pk_bpt_k = kp.pk_bpt_v = bpt;
        kp.seqs = ds;
        kp.seq_ids = sid;
        e = launch_kv_pack(kp, st);
        cudaMemcpyKind kind = dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
        if (e == cudaSuccess) e = cudaMemcpyAsync(op->out, data, bpt, kind, st);
        if (e == cudaSuccess) e = cudaMemcpyAsync((uint8_t *)op->out + bpt, mins, 8, kind, st);
        cudaError_t e2 = cudaStreamSynchronize(st);
        cudaFree(scratch);
        cudaFree(mins);
        cudaFree(data);
        cudaFree(ds);
        cudaFree(sid);
        if (e == cudaSuccess) e = e2;
        if (e != cudaSuccess) return set_err(b, NEXUS_E_CUDA, std::string("kv_quantize: ") + cudaGetErrorString(e));
        return NEXUS_OK;
    }
    case NEXUS_OP_ATTENTION: {
        // GQA decode attention of one query token over n cached tokens:
        // q [m*k], keys/values [n][kv_heads*k]
        size_t hq = op->m, seq = op->n, hd = op->k, hkv = op->kv_heads ? op->kv_heads : op->m;
        if (seq == 0 || hkv == 0 || hq % hkv) return set_err(b, NEXUS_E_INVALID, "attention: bad shape");
        size_t kv_dim = hkv * hd;
        out_bytes = hq * hd * 4;
        NX_CUDA(b, stage_in(op->a, hq * hd * 4, dev, A, st));
        NX_CUDA(b, stage_in(op->b, seq * kv_dim * 4, dev, B, st));
        NX_CUDA(b, stage_in(op->c, seq * kv_dim * 4, dev, Cc, st));
        NX_CUDA(b, stage_out(op->out, out_bytes, dev, O));
        DevSeq hs = {};
        hs.seq_len = (uint32_t)seq;
        hs.slot = (uint32_t)(seq - 1);
        DevSeq *ds = nullptr;
        uint32_t *sid = nullptr;
        float *part = nullptr;
        unsigned *ctr = nullptr;
        int nsplit = (int)std::min<size_t>(64, std::max<size_t>(1, (seq + 63) / 64));
        size_t G = hq / hkv;
        NX_CUDA(b, dalloc(&ds, 1));
        NX_CUDA(b, dalloc(&sid, 1));
        NX_CUDA(b, dalloc(&part, hkv * nsplit * G * (hd + 2)));
        NX_CUDA(b, dalloc(&ctr, hkv));
        NX_CUDA(b, cudaMemsetAsync(sid, 0, 4, st));
        NX_CUDA(b, cudaMemsetAsync(ctr, 0, hkv * 4, st));
        NX_CUDA(b, cudaMemcpyAsync(ds, &hs, sizeof(hs), cudaMemcpyHostToDevice, st));
        AttnParams p = {};
        p.hq = (int)hq;
        p.hkv = (int)hkv;
        p.head_dim = (int)hd;
        p.m = 1;
        p.q = (const float *)A.d;
        p.out = (float *)O.d;
        p.scale = op->scale != 0.0f ? op->scale : 1.0f / sqrtf((float)hd);
        p.k_cache = (const float *)B.d;
        p.v_cache = (const float *)Cc.d;
        p.seqs = ds;
        p.seq_ids = sid;
        p.kv_dim = (int)kv_dim;
        p.nsplit = nsplit;
        p.part = part;
        p.counters = ctr;
        e = launch_attention(p, st);
        cudaError_t e2 = cudaStreamSynchronize(st);
        cudaFree(ds);
        cudaFree(sid);
        cudaFree(part);
        cudaFree(ctr);
        if (e == cudaSuccess) e = e2;
        break;
    }
    case NEXUS_OP_ATTENTION_PACKED: {
        // packed keys/values: [n][bpt] codes, n mins, n scales, per stream
        size_t hq = op->m, seq = op->n, hd = op->k, hkv = op->kv_heads ? op->kv_heads : op->m;
        const int bk = op->format & 0xff, bv = (op->format >> 8) & 0xff;
        if (seq == 0 || hkv == 0 || hq % hkv || bk < 1 || bk > 8 || bv < 1 || bv > 8 || (hd != 32 && hd != 64 && hd != 128))
            return set_err(b, NEXUS_E_INVALID, "attention_packed: bad shape or bits");
        const size_t kv_dim = hkv * hd, bpk = (kv_dim * bk + 7) / 8, bpv = (kv_dim * bv + 7) / 8;
        const size_t offk = (seq * bpk + 15) / 16 * 16, offv = (seq * bpv + 15) / 16 * 16;
        out_bytes = hq * hd * 4;
        NX_CUDA(b, stage_in(op->a, hq * hd * 4, dev, A, st));
        NX_CUDA(b, stage_out(op->out, out_bytes, dev, O));
        uint8_t *kb = nullptr, *vb = nullptr;
        DevSeq *ds = nullptr;
        uint32_t *sid = nullptr;
        float *part = nullptr;
        unsigned *ctr = nullptr;
        const int nsplit = (int)std::min<size_t>(64, std::max<size_t>(1, (seq + 63) / 64));
        const size_t G = hq / hkv;
        NX_CUDA(b, dalloc(&kb, offk + 8 * seq));
        NX_CUDA(b, dalloc(&vb, offv + 8 * seq));
        NX_CUDA(b, dalloc(&ds, 1));
        NX_CUDA(b, dalloc(&sid, 1));
        NX_CUDA(b, dalloc(&part, hkv * nsplit * G * (hd + 2)));
        NX_CUDA(b, dalloc(&ctr, hkv));
        const cudaMemcpyKind kind = dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
        const uint8_t *sk = static_cast<const uint8_t *>(op->b), *sv = static_cast<const uint8_t *>(op->c);
        NX_CUDA(b, cudaMemcpyAsync(kb, sk, seq * bpk, kind, st));
        NX_CUDA(b, cudaMemcpyAsync(kb + offk, sk + seq * bpk, 8 * seq, kind, st));
        NX_CUDA(b, cudaMemcpyAsync(vb, sv, seq * bpv, kind, st));
        NX_CUDA(b, cudaMemcpyAsync(vb + offv, sv + seq * bpv, 8 * seq, kind, st));
        DevSeq hs = {};
        hs.seq_len = (uint32_t)seq;
        hs.slot = (uint32_t)(seq - 1);
        NX_CUDA(b, cudaMemsetAsync(sid, 0, 4, st));
        NX_CUDA(b, cudaMemsetAsync(ctr, 0, hkv * 4, st));
        NX_CUDA(b, cudaMemcpyAsync(ds, &hs, sizeof(hs), cudaMemcpyHostToDevice, st));
        AttnParams p = {};
        p.hq = (int)hq;
        p.hkv = (int)hkv;
        p.head_dim = (int)hd;
        p.m = 1;
        p.q = (const float *)A.d;
        p.out = (float *)O.d;
        p.scale = op->scale != 0.0f ? op->scale : 1.0f / sqrtf((float)hd);
        p.bits_k = bk;
        p.bits_v = bv;
        p.kp_data = kb;
        p.vp_data = vb;
        p.kp_min = reinterpret_cast<const float *>(kb + offk);
        p.kp_scale = p.kp_min + seq;
        p.vp_min = reinterpret_cast<const float *>(vb + offv);
        p.vp_scale = p.vp_min + seq;
        p.pk_bpt_k = bpk;
        p.pk_bpt_v = bpv;
        p.seqs = ds;
        p.seq_ids = sid;
        p.kv_dim = (int)kv_dim;
        p.nsplit = nsplit;
        p.part = part;
        p.counters = ctr;
        e = launch_attention(p, st);
        cudaError_t e2 = cudaStreamSynchronize(st);
        cudaFree(kb);
        cudaFree(vb);
        cudaFree(ds);
        cudaFree(sid);
        cudaFree(part);
        cudaFree(ctr);
        if (e == cudaSuccess) e = e2;
        break;
    }
    default: return set_err(b, NEXUS_E_INVALID, "unknown op kind");
    }
    if (e != cudaSuccess) return set_err(b, NEXUS_E_CUDA, std::string("execute: ") + cudaGetErrorString(e));
    if (!dev && out_bytes) NX_CUDA(b, cudaMemcpyAsync(op->out, O.d, out_bytes, cudaMemcpyDeviceToHost, st));
    NX_CUDA(b, cudaStreamSynchronize(st));
    return NEXUS_OK;
}

// ---------------------------------------------------------------------------
// resident quantized weights
// ---------------------------------------------------------------------------
struct nexus_cuda_qweight {
    nexus_cuda_backend *b = nullptr;
    Mat mat;
    float *xbuf = nullptr, *ybuf = nullptr;
    size_t xcap = 0, ycap = 0;
    LinScratch ls;
};


extern "C" int nexus_cuda_qweight_create(nexus_cuda_backend *b, int format, size_t rows, size_t cols,
                                         const void *blocks, size_t nbytes, nexus_cuda_qweight **out) {
    if (!b || !out || !blocks) return set_err(b, NEXUS_E_INVALID, "NULL argument");
    *out = nullptr;
    if (!tile_supported(format)) return set_err(b, NEXUS_E_UNSUPPORTED_FORMAT, "qweight: unsupported format");
    if (rows == 0 || cols == 0 || cols % 256) return set_err(b, NEXUS_E_INVALID, "qweight: cols must be a multiple of 256");
    if (nbytes < format_bytes(format, rows * cols)) return set_err(b, NEXUS_E_TRUNCATED, "qweight: payload is truncated");
    cudaSetDevice(b->device);
    auto *w = new nexus_cuda_qweight();
    w->b = b;
    int rc = make_mat(b, format, (int)rows, (int)cols, (const uint8_t *)blocks, w->mat);
    if (rc) {
        w->mat.release();
        delete w;
        return rc;
    }
    backend_retain(b);
    *out = w;
    return NEXUS_OK;
}

extern "C" int nexus_cuda_qweight_destroy(nexus_cuda_qweight *w) {
    if (!w) return NEXUS_OK;
    cudaSetDevice(w->b->device);
    cudaStreamSynchronize(w->b->stream);
    w->mat.release();
    if (w->xbuf) cudaFree(w->xbuf);
    if (w->ybuf) cudaFree(w->ybuf);
    w->ls.release();
    nexus_cuda_backend *b = w->b;
    delete w;
    backend_release(b);
    return NEXUS_OK;
}

extern "C" size_t nexus_cuda_qweight_bytes(const nexus_cuda_qweight *w) { return w ? w->mat.bytes : 0; }

extern "C" int nexus_cuda_qmatvec_device(nexus_cuda_qweight *w, const float *x_dev, size_t m, float *y_dev) {
    if (!w || !x_dev || !y_dev) return set_err(w ? w->b : nullptr, NEXUS_E_INVALID, "NULL argument");
    if (m == 0 || m > (1u << 20)) return set_err(w->b, NEXUS_E_INVALID, "qmatvec: bad batch size");
    nexus_cuda_backend *b = w->b;
    cudaSetDevice(b->device);
    NX_CUDA(b, run_qmatvec(w->mat, x_dev, (int)m, y_dev, w->ls, b->dev_err, b->stream));
    return NEXUS_OK;
}

extern "C" int nexus_cuda_qmatvec_bench(nexus_cuda_qweight *w, const float *x_dev, size_t m, float *y_dev, int iters,
                                        size_t flush_bytes, float *avg_ms) {
    if (!w || !x_dev || !y_dev || !avg_ms || iters < 1) return set_err(w ? w->b : nullptr, NEXUS_E_INVALID, "bad argument");
    nexus_cuda_backend *b = w->b;
    cudaSetDevice(b->device);
    cudaStream_t st = b->stream;
    void *flush = nullptr;
    if (flush_bytes) NX_CUDA(b, cudaMalloc(&flush, flush_bytes));
    std::vector<cudaEvent_t> ev(2 * (size_t)iters);
    for (auto &e : ev) cudaEventCreate(&e);
    int rc = NEXUS_OK;
    for (int i = 0; i < iters && rc == NEXUS_OK; i++) {
        if (flush) cudaMemsetAsync(flush, i & 0xff, flush_bytes, st);
        cudaEventRecord(ev[2 * i], st);
        rc = nexus_cuda_qmatvec_device(w, x_dev, m, y_dev);
        cudaEventRecord(ev[2 * i + 1], st);
    }
    cudaError_t e = cudaStreamSynchronize(st);
    float total = 0.0f;
    for (int i = 0; rc == NEXUS_OK && e == cudaSuccess && i < iters; i++) {
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, ev[2 * i], ev[2 * i + 1]);
        total += ms;
    }
    for (auto &x : ev) cudaEventDestroy(x);
    if (flush) cudaFree(flush);
    if (rc) return rc;
    if (e != cudaSuccess) return set_err(b, NEXUS_E_CUDA, cudaGetErrorString(e));
    if ((rc = check_dev_err(b))) return rc;
    *avg_ms = total / iters;
    return NEXUS_OK;
}

extern "C" int nexus_cuda_qmatvec_host(nexus_cuda_qweight *w, const float *x, size_t m, float *y) {
    if (!w || !x || !y) return set_err(w ? w->b : nullptr, NEXUS_E_INVALID, "NULL argument");
    nexus_cuda_backend *b = w->b;
    cudaSetDevice(b->device);
    size_t xn = m * w->mat.k, yn = m * w->mat.n;
    if (xn > w->xcap) {
        if (w->xbuf) cudaFree(w->xbuf);
        NX_CUDA(b, dalloc(&w->xbuf, xn));
        w->xcap = xn;
    }
    if (yn > w->ycap) {
        if (w->ybuf) cudaFree(w->ybuf);
        NX_CUDA(b, dalloc(&w->ybuf, yn));
        w->ycap = yn;
    }
    NX_CUDA(b, cudaMemcpyAsync(w->xbuf, x, xn * 4, cudaMemcpyHostToDevice, b->stream));
    int rc = nexus_cuda_qmatvec_device(w, w->xbuf, m, w->ybuf);
    if (rc) return rc;
    NX_CUDA(b, cudaMemcpyAsync(y, w->ybuf, yn * 4, cudaMemcpyDeviceToHost, b->stream));
    NX_CUDA(b, cudaStreamSynchronize(b->stream));
    return check_dev_err(b);
}

extern "C" int nexus_cuda_qweight_dequantize(nexus_cuda_qweight *w, float *out) {
    if (!w || !out) return set_err(w ? w->b : nullptr, NEXUS_E_INVALID, "NULL argument");
    nexus_cuda_backend *b = w->b;
    cudaSetDevice(b->device);
    size_t n = (size_t)w->mat.n * w->mat.k;
    float *d = nullptr;
    NX_CUDA(b, dalloc(&d, n));
    cudaError_t e = launch_dequant_tiles(w->mat.fmt, w->mat.main, w->mat.aux, w->mat.n, w->mat.k, d, b->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, d, n * 4, cudaMemcpyDeviceToHost, b->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
    cudaFree(d);
    if (e != cudaSuccess) return set_err(b, NEXUS_E_CUDA, cudaGetErrorString(e));
    return NEXUS_OK;
}

// ---------------------------------------------------------------------------
// model
// ---------------------------------------------------------------------------
static constexpr int kMaxChunk = 256;  // tokens per fused step (prefill chunk, decode batch)

struct Layer {
    float *attn_norm = nullptr, *ffn_norm = nullptr;
    Mat qkv, o, gateup, down;
    // KV page pool of this layer, [pool_pages * page_tokens] physical token
    // slots: float rows of kv_dim, or packed rows of bpt bytes plus a min and
    // a scale per slot
    float *k_cache = nullptr, *v_cache = nullptr;
    uint8_t *kp = nullptr, *vp = nullptr;
    float *kmin = nullptr, *kscale = nullptr, *vmin = nullptr, *vscale = nullptr;
};

// Host view of the KV pages (Scheduler::allocate_kv_pages,
// src/scheduler.rs:333-361, hands each request ceil((prompt + max_tokens)/16)
// page ids; ScheduledDecode carries them, :108-115).  Every sequence row has
// a page list: the one its caller bound, or else the library's own pages
// [sid * per_seq, (sid + 1) * per_seq).  Each page belongs to at most one
// sequence.  The device table holds the same lists; rows are uploaded before
// the next step after they change.
struct PageMap {
    uint32_t page_tokens = 16, shift = 4, per_seq = 0, pool = 0;
    std::vector<uint32_t> table;     // [rows][per_seq]
    std::vector<uint32_t> valid;     // usable leading entries of each row
    std::vector<uint8_t> caller;     // 1: the row holds a caller's list
    std::vector<int32_t> owner;      // [pool] sequence holding the page, or -1
    std::vector<uint8_t> dirty;      // rows to upload
};

struct nexus_cuda_model {
    nexus_cuda_backend *b = nullptr;
    nexus_cuda_model_info info = {};
    int embd_fmt = 0;
    uint8_t *embd = nullptr;
    size_t embd_rows = 0;
    float *out_norm = nullptr;
    Mat head;
    bool has_head = false;
    std::vector<Layer> layers;
    float *rope_cos = nullptr, *rope_sin = nullptr;
    float *hidden = nullptr, *q = nullptr, *attn = nullptr, *gated = nullptr, *kv_scratch = nullptr;
    float *logits = nullptr, *part = nullptr;
    unsigned *counters = nullptr;
    LinScratch lin;                   // tensor-core GEMM scratch (steps of kGemmMinM+ tokens)
    // this rank's slice (the whole model without tensor parallelism) and local sizes
    nexus_tp_slice sl = {};
    uint32_t hq_l = 0, hkv_l = 0, qdim_l = 0, kvd_l = 0, f_l = 0, v_l = 0;
    float *logits_gather = nullptr;   // [world][kMaxChunk][v_l] all-gather target
    DevSeq *seqs = nullptr;
    uint32_t *seq_ids = nullptr, *out_tokens = nullptr;
    DevSeq *h_seqs = nullptr;
    uint32_t *h_seq_ids = nullptr, *h_out_tokens = nullptr;
    std::vector<uint32_t> seq_len;
    PageMap pm;
    uint32_t *page_table = nullptr;   // device copy of pm.table
    uint32_t max_seq = 0, max_batch = 1, bits_k = 0, bits_v = 0;
    int x_bits_norm = 24;  // GEMV input bits for matrices with normalized inputs
    uint64_t rope_positions = 0;  // positions the RoPE table covers
    size_t bpt_k = 0, bpt_v = 0;
    int nsplit[kMaxChunk + 1] = {};     // attention slices per (sequence, KV head), float cache
    int nsplit_pk[kMaxChunk + 1] = {};  // the same for the packed-cache tensor-core kernel
    cudaGraphExec_t graph[kMaxChunk + 1] = {};
    cudaGraphExec_t graph_chunk[kMaxChunk + 1] = {};  // steps of one sequence's consecutive tokens
    bool use_graph = true, use_pdl = true;
    // single-token steps as one persistent kernel (kernels_step.cu)
    bool use_step = false;
    StepParams step = {};
    StepLaunch step_launch = {};
    StepLayer *step_layers = nullptr;     // device array of the layers' matrices and caches
    size_t step_gcounter_slots = 0;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    float last_ms = 0.0f;
    std::vector<void *> allocs;
    bool retained = false;  // holds a reference on its backend
};

template <typename T>
static cudaError_t malloc_tracked(nexus_cuda_model *m, T **p, size_t count) {
    cudaError_t e = dalloc(p, count);
    if (e == cudaSuccess) m->allocs.push_back((void *)*p);
    return e;
}

static void model_release(nexus_cuda_model *m) {
    if (!m) return;
    nexus_cuda_backend *owner = m->retained ? m->b : nullptr;
    cudaSetDevice(m->b->device);
    cudaStreamSynchronize(m->b->stream);
    for (auto &g : m->graph)
        if (g) cudaGraphExecDestroy(g);
    for (auto &g : m->graph_chunk)
        if (g) cudaGraphExecDestroy(g);
    for (auto &L : m->layers) {
        L.qkv.release();
        L.o.release();
        L.gateup.release();
        L.down.release();
    }
    m->head.release();
    m->lin.release();
    for (void *p : m->allocs) cudaFree(p);
    if (m->h_seqs) cudaFreeHost(m->h_seqs);
    if (m->h_seq_ids) cudaFreeHost(m->h_seq_ids);
    if (m->h_out_tokens) cudaFreeHost(m->h_out_tokens);
    if (m->ev0) cudaEventDestroy(m->ev0);
    if (m->ev1) cudaEventDestroy(m->ev1);
    delete m;
    if (owner) backend_release(owner);
}

static const GgufTensor *find_any(const GgufFile &f, const std::vector<std::string> &names) {
    for (const auto &n : names) {
        const GgufTensor *t = f.find(n);
        if (t && format_supported(t->type) && t->elems() > 0) return t;
    }
    return nullptr;
}

// layer_tensor_names, src/engine/mod.rs:696-733
static const GgufTensor *layer_tensor(const GgufFile &f, uint32_t l, const char *role, const char *hf) {
    std::string s = std::to_string(l);
    return find_any(f, {"blk." + s + "." + role + ".weight", "model.layers." + s + "." + hf + ".weight",
                        "layers." + s + "." + hf + ".weight"});
}

// Dequantize a 1-D tensor (norm weights) to f32 on the device, bit-exact.
static int upload_vector(nexus_cuda_model *m, const GgufFile &f, const GgufTensor *t, size_t n, float **out) {
    nexus_cuda_backend *b = m->b;
    NX_CUDA(b, malloc_tracked(m, out, n));
    if (!t) {
        std::vector<float> ones(n, 1.0f);
        NX_CUDA(b, cudaMemcpy(*out, ones.data(), n * 4, cudaMemcpyHostToDevice));
        return NEXUS_OK;
    }
    size_t nb = 0;
    const uint8_t *src = f.data(*t, &nb);
    if (!src || t->elems() < n) return set_err(b, NEXUS_E_TRUNCATED, "norm tensor truncated: " + t->name);
    size_t need = format_bytes(t->type, n);
    uint8_t *d = nullptr;
    NX_CUDA(b, dalloc(&d, need));
    cudaError_t e = cudaMemcpy(d, src, need, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = launch_dequant_raw(t->type, d, n, *out, b->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
    cudaFree(d);
    if (e != cudaSuccess) return set_err(b, NEXUS_E_CUDA, cudaGetErrorString(e));
    return NEXUS_OK;
}

// Row bytes of a matrix whose columns are a multiple of the block size.
static size_t row_bytes(int fmt, size_t k) { return k / (size_t)block_elems(fmt) * (size_t)block_bytes(fmt); }

static int check_matrix(nexus_cuda_backend *b, const GgufTensor *t, size_t rows, size_t cols, const char *what) {
    if (!t) return set_err(b, NEXUS_E_MISSING_TENSOR, std::string("Missing tensor: ") + what);
    if (!tile_supported(t->type))
        return set_err(b, NEXUS_E_UNSUPPORTED_FORMAT, std::string("GEMV format not supported for ") + t->name);
    // Self::matvec requires weight.len() >= rows*cols (src/engine/mod.rs:784-790)
    if (t->elems() < rows * cols) return set_err(b, NEXUS_E_INVALID, "Matvec weight too small: " + t->name);
    if (cols % 256) return set_err(b, NEXUS_E_INVALID, "matrix columns must be a multiple of 256: " + t->name);
    return NEXUS_OK;
}

// Columns [c0, c0 + n) of a rows x k block-format matrix (c0 and n whole
// blocks): the full matrix when they cover it, else a copy in `buf`.
static const uint8_t *column_slice(int fmt, const uint8_t *src, uint32_t rows, uint32_t k, uint32_t c0, uint32_t n,
                                   std::vector<uint8_t> &buf) {
    if (c0 == 0 && n == k) return src;
    const size_t rb = row_bytes(fmt, k), off = row_bytes(fmt, c0), nb = row_bytes(fmt, n);
    buf.resize((size_t)rows * nb);
    for (uint32_t r = 0; r < rows; r++) memcpy(buf.data() + (size_t)r * nb, src + (size_t)r * rb + off, nb);
    return buf.data();
}

static KvPages dev_pages(const nexus_cuda_model *m);

static int model_load(nexus_cuda_backend *b, const char *path, nexus_cuda_model **out) {
    GgufFile f;
    std::string err;
    int rc = f.open(path, err);
    if (rc) return set_err(b, rc, err);
    auto *m = new nexus_cuda_model();
    m->b = b;
    std::unique_ptr<nexus_cuda_model, void (*)(nexus_cuda_model *)> guard(m, model_release);
    nexus_cuda_model_info &I = m->info;
    uint64_t v;
    // load_model metadata defaults, src/engine/mod.rs:551-562
    I.num_layers = f.get_usize("llama.block_count", &v) ? (uint32_t)v : 32;
    I.hidden_size = f.get_usize("llama.embedding_length", &v) ? (uint32_t)v : 4096;
    I.ff_dim = f.get_usize("llama.feed_forward_length", &v) ? (uint32_t)v : 11008;
    I.num_heads = f.get_usize("llama.attention.head_count", &v) ? (uint32_t)v : 32;
    I.num_kv_heads = f.get_usize("llama.attention.head_count_kv", &v) ? (uint32_t)v : I.num_heads;
    float fb;
    I.rope_freq_base = f.get_f32("llama.rope.freq_base", &fb) ? fb : 1000000.0f;
    I.rms_norm_eps = 1e-5f;  // InferenceConfig default; the GGUF key is ignored (src/engine/mod.rs:94)
    if (!I.num_heads || !I.num_kv_heads || I.hidden_size % I.num_heads)
        return set_err(b, NEXUS_E_INVALID, "bad head configuration");
    I.head_dim = I.hidden_size / I.num_heads;
    uint32_t ctx = f.get_usize("llama.context_length", &v) ? (uint32_t)v : 4096;
    I.max_seq_len = b->cfg.max_seq_len ? b->cfg.max_seq_len : ctx;
    const uint32_t H = I.hidden_size, D = I.head_dim, F = I.ff_dim, Hq = I.num_heads, Hkv = I.num_kv_heads;
    const uint32_t kv_dim = Hkv * D, qdim = Hq * D;
    if (D % 32 || D > 128 || Hq % Hkv || (Hq / Hkv) > 8 || ((Hq / Hkv) & (Hq / Hkv - 1)))
        return set_err(b, NEXUS_E_INVALID, "head_dim must be 32/64/128 and Hq/Hkv a power of two <= 8");
    if (H % 256 || F % 256) return set_err(b, NEXUS_E_INVALID, "hidden and ffn sizes must be multiples of 256");
    m->max_seq = I.max_seq_len;
    m->rope_positions = 4 * (uint64_t)m->max_seq;
    m->max_batch = b->cfg.max_batch;
    m->bits_k = b->cfg.kv_bits_k;
    m->bits_v = b->cfg.kv_bits_v;
    {
        // KV pages: page_tokens a power of two, every sequence row able to
        // list max_seq_len tokens, a pool of max_pages pages
        PageMap &pm = m->pm;
        pm.page_tokens = b->cfg.page_tokens ? b->cfg.page_tokens : 16;
        if (pm.page_tokens > 4096 || (pm.page_tokens & (pm.page_tokens - 1)))
            return set_err(b, NEXUS_E_INVALID, "page_tokens must be a power of two <= 4096");
        pm.shift = 0;
        while ((1u << pm.shift) < pm.page_tokens) pm.shift++;
        pm.per_seq = (m->max_seq + pm.page_tokens - 1) / pm.page_tokens;
        const uint64_t pool = b->cfg.max_pages ? (uint64_t)b->cfg.max_pages : (uint64_t)m->max_batch * pm.per_seq;
        if (pool == 0 || pool > 0x7fffffffull) return set_err(b, NEXUS_E_INVALID, "bad KV page pool size");
        pm.pool = (uint32_t)pool;
        pm.table.assign((size_t)m->max_batch * pm.per_seq, 0u);
        pm.valid.assign(m->max_batch, 0u);
        pm.caller.assign(m->max_batch, 0);
        pm.owner.assign(pm.pool, -1);
        pm.dirty.assign(m->max_batch, 0);
        I.max_batch = m->max_batch;
        I.page_tokens = pm.page_tokens;
        I.max_pages = pm.pool;
    }
    m->use_graph = !(b->cfg.flags & NEXUS_CFG_NO_GRAPH);
    // GEMV inputs of qkv, o_proj, gate/up and the head (normalized) as 16-bit
    // integers only on request; down always reads 24-bit ones
    m->x_bits_norm = (b->cfg.flags & NEXUS_CFG_GEMV_16BIT) ? 16 : 24;
    m->use_pdl = !(b->cfg.flags & NEXUS_CFG_NO_PDL);
    cudaSetDevice(b->device);

    // embedding (raw blocks; rows decoded per token on the device)
    const GgufTensor *te = find_any(f, {"token_embd.weight", "token_embd", "model.embed_tokens.weight", "transformer.wte.weight"});
    if (!te) return set_err(b, NEXUS_E_MISSING_TENSOR, "Missing tensor: token_embd.weight");
    {
        size_t nb = 0;
        const uint8_t *src = f.data(*te, &nb);
        if (!src) return set_err(b, NEXUS_E_TRUNCATED, "token_embd payload truncated");
        m->embd_fmt = te->type;
        m->embd_rows = std::max<size_t>(1, te->elems() / H);
        NX_CUDA(b, malloc_tracked(m, &m->embd, nb + 16));
        NX_CUDA(b, cudaMemcpy(m->embd, src, nb, cudaMemcpyHostToDevice));
    }
    rc = upload_vector(m, f, find_any(f, {"output_norm.weight", "norm.weight", "model.norm.weight", "transformer.ln_f.weight"}), H,
                       &m->out_norm);
    if (rc) return rc;
    const GgufTensor *th = find_any(f, {"output.weight", "lm_head.weight", "model.embed_tokens.weight", "token_embd.weight"});
    uint64_t weight_bytes = 0;
    const int tp = b->tp_world, rk = b->tp_rank;
    if (tp > 1 && !th) return set_err(b, NEXUS_E_INVALID, "tensor parallelism needs an LM head tensor");
    if (tp > 1 && m->bits_k) return set_err(b, NEXUS_E_UNSUPPORTED_FORMAT, "tensor parallelism runs with the float KV cache");
    I.vocab_rows = th ? (uint32_t)(th->elems() / H) : H;  // no head: logits are the normed hidden state (:1040-1043)
    if ((rc = nexus_tp_plan(Hq, Hkv, D, F, I.vocab_rows, rk, tp, &m->sl))) return set_err(b, rc, g_tls_error);
    m->hq_l = m->sl.q_heads;
    m->hkv_l = m->sl.kv_heads;
    m->qdim_l = m->hq_l * D;
    m->kvd_l = m->hkv_l * D;
    m->f_l = m->sl.ffn_rows;
    m->v_l = m->sl.vocab_rows;
    if (th) {
        size_t rows = th->elems() / H;
        rc = check_matrix(b, th, rows, H, "output.weight");
        if (rc) return rc;
        size_t nb = 0;
        const uint8_t *src = f.data(*th, &nb);
        if (!src) return set_err(b, NEXUS_E_TRUNCATED, "output payload truncated");
        // this rank's vocab rows
        src += (size_t)m->sl.vocab_begin * row_bytes(th->type, H);
        rc = make_mat(b, th->type, (int)m->v_l, (int)H, src, m->head);
        if (rc) return rc;
        m->has_head = true;
        weight_bytes += m->head.bytes;
    }

    m->layers.resize(I.num_layers);
    std::vector<uint8_t> buf;
    for (uint32_t l = 0; l < I.num_layers; l++) {
        Layer &L = m->layers[l];
        rc = upload_vector(m, f, layer_tensor(f, l, "attn_norm", "input_layernorm"), H, &L.attn_norm);
        if (rc) return rc;
        rc = upload_vector(m, f, layer_tensor(f, l, "ffn_norm", "post_attention_layernorm"), H, &L.ffn_norm);
        if (rc) return rc;
        const GgufTensor *tq = layer_tensor(f, l, "attn_q", "self_attn.q_proj");
        const GgufTensor *tk = layer_tensor(f, l, "attn_k", "self_attn.k_proj");
        const GgufTensor *tv = layer_tensor(f, l, "attn_v", "self_attn.v_proj");
        const GgufTensor *to = layer_tensor(f, l, "attn_output", "self_attn.o_proj");
        const GgufTensor *tg = layer_tensor(f, l, "ffn_gate", "mlp.gate_proj");
        const GgufTensor *tu = layer_tensor(f, l, "ffn_up", "mlp.up_proj");
        const GgufTensor *td = layer_tensor(f, l, "ffn_down", "mlp.down_proj");
        std::string ls = "blk." + std::to_string(l) + ".";
        if ((rc = check_matrix(b, tq, qdim, H, (ls + "attn_q.weight").c_str()))) return rc;
        if ((rc = check_matrix(b, tk, kv_dim, H, (ls + "attn_k.weight").c_str()))) return rc;
        if ((rc = check_matrix(b, tv, kv_dim, H, (ls + "attn_v.weight").c_str()))) return rc;
        if ((rc = check_matrix(b, to, H, qdim, (ls + "attn_output.weight").c_str()))) return rc;
        if ((rc = check_matrix(b, tg, F, H, (ls + "ffn_gate.weight").c_str()))) return rc;
        if ((rc = check_matrix(b, tu, F, H, (ls + "ffn_up.weight").c_str()))) return rc;
        if ((rc = check_matrix(b, td, H, F, (ls + "ffn_down.weight").c_str()))) return rc;
        if (tq->type != tk->type || tq->type != tv->type)
            return set_err(b, NEXUS_E_UNSUPPORTED_FORMAT, "attn_q/k/v must share one format for the fused QKV GEMV");
        if (tg->type != tu->type)
            return set_err(b, NEXUS_E_UNSUPPORTED_FORMAT, "ffn_gate/up must share one format for the fused SwiGLU GEMV");
        const uint8_t *pq = f.data(*tq, nullptr), *pk = f.data(*tk, nullptr), *pv = f.data(*tv, nullptr);
        const uint8_t *po = f.data(*to, nullptr), *pg = f.data(*tg, nullptr), *pu = f.data(*tu, nullptr);
        const uint8_t *pd = f.data(*td, nullptr);
        if (!pq || !pk || !pv || !po || !pg || !pu || !pd) return set_err(b, NEXUS_E_TRUNCATED, "layer payload truncated");
        // fused Q|K|V with RoPE pairs (d, d + D/2) in lanes (i, i + 16) of a row group
        {
            const int fmt = tq->type;
            const size_t rb = row_bytes(fmt, H);
            const uint32_t qd = m->qdim_l, kd = m->kvd_l;  // this rank's heads
            const uint32_t nrows = qd + 2 * kd;
            buf.resize((size_t)nrows * rb);
            const uint32_t gph = D / 32;
            for (uint32_t r = 0; r < nrows; r++) {
                const uint8_t *src;
                if (r < qd + kd) {
                    const bool isq = r < qd;
                    const uint32_t rr = isq ? r : r - qd;
                    const uint32_t g = rr / 32, lane = rr % 32, head = g / gph, i = g % gph;
                    const uint32_t d = lane < 16 ? 16 * i + lane : 16 * i + (lane - 16) + D / 2;
                    const uint32_t ghead = head + (isq ? m->sl.q_head_begin : m->sl.kv_head_begin);
                    src = (isq ? pq : pk) + (size_t)(ghead * D + d) * rb;
                } else {
                    src = pv + (size_t)(m->sl.kv_head_begin * D + (r - qd - kd)) * rb;
                }
                memcpy(buf.data() + (size_t)r * rb, src, rb);
            }
            if ((rc = make_mat(b, fmt, (int)nrows, (int)H, buf.data(), L.qkv))) return rc;
        }
        // o_proj: this rank's columns (its heads' outputs), whole super-blocks
        if ((rc = make_mat(b, to->type, (int)H, (int)m->qdim_l,
                           column_slice(to->type, po, H, qdim, m->sl.q_head_begin * D, m->qdim_l, buf), L.o)))
            return rc;
        // gate/up interleaved: lanes 0..15 gate rows, lanes 16..31 the same up rows
        {
            const int fmt = tg->type;
            const size_t rb = row_bytes(fmt, H);
            const uint32_t fl = m->f_l, f0 = m->sl.ffn_begin;
            buf.resize((size_t)2 * fl * rb);
            for (uint32_t r = 0; r < 2 * fl; r++) {
                const uint32_t g = r / 32, lane = r % 32;
                const uint8_t *src = lane < 16 ? pg + (size_t)(f0 + 16 * g + lane) * rb
                                               : pu + (size_t)(f0 + 16 * g + lane - 16) * rb;
                memcpy(buf.data() + (size_t)r * rb, src, rb);
            }
            if ((rc = make_mat(b, fmt, (int)(2 * fl), (int)H, buf.data(), L.gateup))) return rc;
        }
        if ((rc = make_mat(b, td->type, (int)H, (int)m->f_l,
                           column_slice(td->type, pd, H, F, m->sl.ffn_begin, m->f_l, buf), L.down)))
            return rc;
        weight_bytes += L.qkv.bytes + L.o.bytes + L.gateup.bytes + L.down.bytes;
        if (l == 0) I.body_format = tq->type;
        // KV cache (KvCache::new(num_kv_heads*head_dim, max_seq_len, kv_quant), :593-597)
        const size_t toks = (size_t)m->pm.pool * m->pm.page_tokens;  // physical slots of the page pool
        if (m->bits_k == 0) {
            NX_CUDA(b, malloc_tracked(m, &L.k_cache, toks * m->kvd_l));
            NX_CUDA(b, malloc_tracked(m, &L.v_cache, toks * m->kvd_l));
        } else {
            m->bpt_k = ((size_t)kv_dim * m->bits_k + 7) / 8;
            m->bpt_v = ((size_t)kv_dim * m->bits_v + 7) / 8;
            NX_CUDA(b, malloc_tracked(m, &L.kp, toks * m->bpt_k + 16));
            NX_CUDA(b, malloc_tracked(m, &L.vp, toks * m->bpt_v + 16));
            NX_CUDA(b, malloc_tracked(m, &L.kmin, toks));
            NX_CUDA(b, malloc_tracked(m, &L.kscale, toks));
            NX_CUDA(b, malloc_tracked(m, &L.vmin, toks));
            NX_CUDA(b, malloc_tracked(m, &L.vscale, toks));
        }
    }
    I.weight_bytes = weight_bytes;

    // RoPE table with the reference's f32 formula and the host libm
    // (rope_single, src/kernel/mod.rs:259-263)
    {
        // positions keep growing after the cache is full (it holds the last
        // max_seq_len tokens): the table covers 4 x max_seq_len of them
        const size_t half = D / 2, npos = m->rope_positions;
        std::vector<float> cs(npos * half), sn(npos * half);
        for (size_t pos = 0; pos < npos; pos++)
            for (size_t d = 0; d < half; d++) {
                volatile float e = 2.0f * (float)d;
                e = e / (float)D;
                volatile float denom = powf(I.rope_freq_base, e);
                float ang = (float)pos / denom;
                cs[pos * half + d] = cosf(ang);
                sn[pos * half + d] = sinf(ang);
            }
        NX_CUDA(b, malloc_tracked(m, &m->rope_cos, cs.size()));
        NX_CUDA(b, malloc_tracked(m, &m->rope_sin, sn.size()));
        NX_CUDA(b, cudaMemcpy(m->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
        NX_CUDA(b, cudaMemcpy(m->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
    }

    // activations for up to kMaxChunk tokens per step
    // (this rank's heads, FFN rows and vocab rows under tensor parallelism)
    const int MC = kMaxChunk;
    const uint32_t qd = m->qdim_l, kd = m->kvd_l, fl = m->f_l, hkv_l = m->hkv_l;
    NX_CUDA(b, malloc_tracked(m, &m->hidden, (size_t)MC * H));
    NX_CUDA(b, malloc_tracked(m, &m->q, (size_t)MC * qd));
    NX_CUDA(b, malloc_tracked(m, &m->attn, (size_t)MC * qd));
    NX_CUDA(b, malloc_tracked(m, &m->gated, (size_t)MC * fl));
    NX_CUDA(b, malloc_tracked(m, &m->kv_scratch, (size_t)MC * 2 * kd));
    NX_CUDA(b, malloc_tracked(m, &m->logits, (size_t)MC * (m->has_head ? m->v_l : I.vocab_rows)));
    if (tp > 1) NX_CUDA(b, malloc_tracked(m, &m->logits_gather, (size_t)tp * MC * m->v_l));
    const int G = (int)(Hq / Hkv);
    // context slices of >= NX_ATTN_TPS tokens, at most 64 per (sequence, KV
    // head); the kernel uses only as many as the current context needs
    int max_split = std::max(1, std::min(64, (int)((m->max_seq + NX_ATTN_TPS - 1) / NX_ATTN_TPS)));
    for (int mm = 1; mm <= MC; mm++) m->nsplit[mm] = max_split;
    // the packed-cache kernel: about 8 CTAs per SM over the whole step (its
    // CTAs stream whole 64-token tiles and need no more slices than that)
    for (int mm = 1; mm <= MC; mm++)
        m->nsplit_pk[mm] = std::max(1, std::min(max_split, (148 * 8 + mm * (int)hkv_l - 1) / (mm * (int)hkv_l)));
    NX_CUDA(b, malloc_tracked(m, &m->part, (size_t)MC * hkv_l * max_split * G * (D + 2)));
    NX_CUDA(b, malloc_tracked(m, &m->counters, (size_t)MC * hkv_l));
    NX_CUDA(b, cudaMemset(m->counters, 0, (size_t)MC * hkv_l * 4));
    {
        // GEMM scratch for every step size that runs on the tensor cores
        const int shapes[5][2] = {{(int)(qd + 2 * kd), (int)H}, {(int)H, (int)qd}, {(int)(2 * fl), (int)H},
                                  {(int)H, (int)fl}, {(int)m->v_l, (int)H}};
        for (int mm = kGemmMinM; mm <= MC; mm++)
            for (auto &sh : shapes) NX_CUDA(b, m->lin.ensure(mm, sh[0], sh[1], b->stream));
    }
    NX_CUDA(b, malloc_tracked(m, &m->seqs, MC));
    NX_CUDA(b, malloc_tracked(m, &m->seq_ids, MC));
    NX_CUDA(b, malloc_tracked(m, &m->out_tokens, MC + 1));  // [MC] tokens + error flag
    NX_CUDA(b, cudaMemset(m->seqs, 0, MC * sizeof(DevSeq)));
    NX_CUDA(b, cudaMemset(m->seq_ids, 0, MC * 4));
    NX_CUDA(b, cudaHostAlloc((void **)&m->h_seqs, MC * sizeof(DevSeq), cudaHostAllocDefault));
    NX_CUDA(b, cudaHostAlloc((void **)&m->h_seq_ids, MC * 4, cudaHostAllocDefault));
    NX_CUDA(b, cudaHostAlloc((void **)&m->h_out_tokens, (MC + 1) * 4, cudaHostAllocDefault));
    NX_CUDA(b, cudaMemset(m->out_tokens, 0, (MC + 1) * 4));
    NX_CUDA(b, cudaEventCreate(&m->ev0));
    NX_CUDA(b, cudaEventCreate(&m->ev1));
    m->seq_len.assign(m->max_batch, 0);
    NX_CUDA(b, malloc_tracked(m, &m->page_table, m->pm.table.size()));
    NX_CUDA(b, cudaMemset(m->page_table, 0, m->pm.table.size() * 4));
    NX_CUDA(b, cudaDeviceSynchronize());
    // the persistent single-token step (opt-in): one GPU, float KV cache, an LM
    // head, shapes the step kernel covers (otherwise the kernel-per-op graph runs)
    if (tp == 1 && m->bits_k == 0 && m->has_head && (b->cfg.flags & NEXUS_CFG_PERSISTENT)) {
        StepParams &sp = m->step;
        auto sm_of = [](const Mat &w) { return StepMat{w.fmt, w.main, w.aux, w.n, w.k}; };
        std::vector<StepLayer> hl(I.num_layers);
        size_t groups = (m->head.n + 31) / 32;
        for (uint32_t l = 0; l < I.num_layers; l++) {
            const Layer &L = m->layers[l];
            hl[l] = StepLayer{sm_of(L.qkv), sm_of(L.o), sm_of(L.gateup), sm_of(L.down), L.attn_norm, L.ffn_norm,
                              L.k_cache, L.v_cache};
            for (const Mat *w : {&L.qkv, &L.o, &L.gateup, &L.down}) groups = std::max<size_t>(groups, (w->n + 31) / 32);
        }
        sp.num_layers = (int)I.num_layers;
        sp.head = sm_of(m->head);
        sp.out_norm = m->out_norm;
        sp.hidden = (int)H;
        sp.hq = (int)Hq;
        sp.hkv = (int)Hkv;
        sp.head_dim = (int)D;
        sp.ffn = (int)F;
        sp.eps = I.rms_norm_eps;
        sp.rope_cos = m->rope_cos;
        sp.rope_sin = m->rope_sin;
        sp.x_hidden = m->hidden;
        sp.q = m->q;
        sp.attn = m->attn;
        sp.gated = m->gated;
        sp.logits = m->logits;
        sp.seqs = m->seqs;
        sp.seq_ids = m->seq_ids;
        sp.pages = dev_pages(m);
        sp.out_tokens = m->out_tokens;
        sp.err = reinterpret_cast<int *>(m->out_tokens + kMaxChunk);
        sp.bar_extra = (b->cfg.flags & NEXUS_CFG_FAULT_STALL_BARRIER) ? 1u : 0u;
        bool fmts_ok = true;
        for (const StepLayer &L : hl)
            for (const StepMat *w : {&L.qkv, &L.o, &L.gateup, &L.down}) fmts_ok = fmts_ok && gemm_supported(w->fmt);
        fmts_ok = fmts_ok && gemm_supported(sp.head.fmt);
        if (fmts_ok && step_plan(sp, b->device, &m->step_launch) == cudaSuccess) {
            StepLaunch &sl = m->step_launch;
            // attention: slices of >= 32 tokens, about one block per CTA
            sp.attn_nsplit = std::max(1, std::min(64, sl.grid / (int)Hkv));
            sp.max_seq = m->max_seq;
            NX_CUDA(b, malloc_tracked(m, &m->step_layers, hl.size()));
            NX_CUDA(b, cudaMemcpy(m->step_layers, hl.data(), hl.size() * sizeof(StepLayer), cudaMemcpyHostToDevice));
            sp.layers = m->step_layers;
            NX_CUDA(b, malloc_tracked(m, &sp.attn_part, (size_t)Hkv * sp.attn_nsplit * (Hq / Hkv) * (D + 2)));
            NX_CUDA(b, malloc_tracked(m, &sp.attn_counters, (size_t)Hkv));
            NX_CUDA(b, malloc_tracked(m, &sp.gpart, step_gpart_floats(sl)));
            m->step_gcounter_slots = groups;
            NX_CUDA(b, malloc_tracked(m, &sp.gcounters, groups));
            NX_CUDA(b, malloc_tracked(m, &sp.bar, (size_t)2));
            NX_CUDA(b, cudaMemset(sp.attn_counters, 0, (size_t)Hkv * 4));
            NX_CUDA(b, cudaMemset(sp.gcounters, 0, groups * 4));
            NX_CUDA(b, cudaMemset(sp.bar, 0, 8));
            m->use_step = true;
        }
    }
    guard.release();
    backend_retain(b);
    m->retained = true;
    *out = m;
    return NEXUS_OK;
}

// ---------------------------------------------------------------------------
// KV pages
// ---------------------------------------------------------------------------
static KvPages dev_pages(const nexus_cuda_model *m) { return KvPages{m->page_table, m->pm.per_seq, m->pm.shift}; }

static void pages_release(nexus_cuda_model *m, uint32_t sid) {
    PageMap &pm = m->pm;
    uint32_t *row = pm.table.data() + (size_t)sid * pm.per_seq;
    for (uint32_t i = 0; i < pm.valid[sid]; i++)
        if (pm.owner[row[i]] == (int32_t)sid) pm.owner[row[i]] = -1;
    pm.valid[sid] = 0;
    pm.caller[sid] = 0;
}

// Bind ids[0..n) as the page list of sequence sid.  Pages holding the
// sequence's cached tokens must stay where they are; every page must be in
// the pool, listed once and free or already this sequence's.
static int pages_bind(nexus_cuda_model *m, uint32_t sid, const uint32_t *ids, uint32_t n) {
    PageMap &pm = m->pm;
    uint32_t *row = pm.table.data() + (size_t)sid * pm.per_seq;
    if (pm.caller[sid] && pm.valid[sid] == n && std::equal(ids, ids + n, row)) return NEXUS_OK;  // unchanged
    if (n > pm.per_seq)
        return set_err(m->b, NEXUS_E_INVALID, "page list longer than max_seq_len / page_tokens entries");
    const uint32_t cached = (std::min(m->seq_len[sid], m->max_seq) + pm.page_tokens - 1) / pm.page_tokens;
    if (n < cached) return set_err(m->b, NEXUS_E_INVALID, "page list shorter than the sequence's cached tokens");
    for (uint32_t i = 0; i < cached; i++)
        if (ids[i] != row[i])
            return set_err(m->b, NEXUS_E_INVALID,
                           "page list moves cached tokens (its first pages must be the ones the sequence was written "
                           "to; reset the sequence to rebind)");
    std::vector<uint32_t> sorted(ids, ids + n);
    std::sort(sorted.begin(), sorted.end());
    for (uint32_t i = 0; i < n; i++) {
        if (sorted[i] >= pm.pool) return set_err(m->b, NEXUS_E_INVALID, "page id beyond the KV page pool (max_pages)");
        if (i && sorted[i] == sorted[i - 1]) return set_err(m->b, NEXUS_E_INVALID, "page id listed twice");
        const int32_t o = pm.owner[sorted[i]];
        if (o >= 0 && o != (int32_t)sid)
            return set_err(m->b, NEXUS_E_INVALID,
                           "page " + std::to_string(sorted[i]) + " belongs to sequence " + std::to_string(o));
    }
    for (uint32_t i = 0; i < pm.valid[sid]; i++)
        if (pm.owner[row[i]] == (int32_t)sid) pm.owner[row[i]] = -1;
    std::copy(ids, ids + n, row);
    for (uint32_t i = 0; i < n; i++) pm.owner[ids[i]] = (int32_t)sid;
    pm.valid[sid] = n;
    pm.caller[sid] = 1;
    pm.dirty[sid] = 1;
    return NEXUS_OK;
}

// A sequence without a caller's list uses the library's pages
// [sid * per_seq, (sid + 1) * per_seq) of the pool (bound on first use).
static int pages_default(nexus_cuda_model *m, uint32_t sid) {
    PageMap &pm = m->pm;
    if (pm.caller[sid] || pm.valid[sid]) return NEXUS_OK;
    const uint64_t first = (uint64_t)sid * pm.per_seq;
    const uint32_t n = first >= pm.pool ? 0u : (uint32_t)std::min<uint64_t>(pm.per_seq, pm.pool - first);
    uint32_t *row = pm.table.data() + (size_t)sid * pm.per_seq;
    for (uint32_t i = 0; i < n; i++) {
        const int32_t o = pm.owner[first + i];
        if (o >= 0 && o != (int32_t)sid)
            return set_err(m->b, NEXUS_E_INVALID,
                           "the library's pages of sequence " + std::to_string(sid) + " are bound to sequence " +
                               std::to_string(o) + "; give this sequence a page list");
    }
    for (uint32_t i = 0; i < n; i++) {
        row[i] = (uint32_t)(first + i);
        pm.owner[first + i] = (int32_t)sid;
    }
    pm.valid[sid] = n;
    pm.dirty[sid] = 1;
    return NEXUS_OK;
}

// The sequence's pages must cover `tokens` tokens.
static int pages_cover(nexus_cuda_model *m, uint32_t sid, uint64_t tokens) {
    const PageMap &pm = m->pm;
    if (tokens > (uint64_t)pm.valid[sid] * pm.page_tokens)
        return set_err(m->b, NEXUS_E_INVALID,
                       "the KV pages of sequence " + std::to_string(sid) + " hold " +
                           std::to_string((uint64_t)pm.valid[sid] * pm.page_tokens) + " tokens; the step needs " +
                           std::to_string(tokens));
    return NEXUS_OK;
}

static cudaError_t pages_upload(nexus_cuda_model *m) {
    PageMap &pm = m->pm;
    for (uint32_t r = 0; r < m->max_batch; r++) {
        if (!pm.dirty[r]) continue;
        const size_t off = (size_t)r * pm.per_seq;
        cudaError_t e = cudaMemcpyAsync(m->page_table + off, pm.table.data() + off, (size_t)pm.per_seq * 4,
                                        cudaMemcpyHostToDevice, m->b->stream);
        if (e != cudaSuccess) return e;
        pm.dirty[r] = 0;
    }
    return cudaSuccess;
}

// Optional per-kernel timing of enqueue_step (profile mode only, never in a graph).
struct StepProfiler {
    struct Rec {
        std::string name;
        double bytes = 0;
        uint32_t launches = 0;
        float ms = 0;
        std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev;
    };
    std::vector<Rec> recs;
    cudaStream_t st = nullptr;
    cudaEvent_t cur = nullptr;
    int idx(const char *name) {
        for (size_t i = 0; i < recs.size(); i++)
            if (recs[i].name == name) return (int)i;
        recs.push_back(Rec());
        recs.back().name = name;
        return (int)recs.size() - 1;
    }
    void begin() {
        cudaEventCreate(&cur);
        cudaEventRecord(cur, st);
    }
    void end(const char *name, double bytes) {
        cudaEvent_t e;
        cudaEventCreate(&e);
        cudaEventRecord(e, st);
        Rec &r = recs[idx(name)];
        r.ev.push_back({cur, e});
        r.bytes = bytes;
        r.launches++;
    }
    void collect() {
        for (auto &r : recs) {
            for (auto &pr : r.ev) {
                float ms = 0;
                cudaEventSynchronize(pr.second);
                cudaEventElapsedTime(&ms, pr.first, pr.second);
                r.ms += ms;
                cudaEventDestroy(pr.first);
                cudaEventDestroy(pr.second);
            }
            r.ev.clear();
        }
    }
};

static void set_split_scratch(const nexus_cuda_model *m, GemvParams &g);

static double gemv_bytes(const Mat &w, int mc, int k, int n_out) {
    return (double)w.bytes + 4.0 * mc * k + 4.0 * mc * n_out;
}

static void set_split_scratch(const nexus_cuda_model *m, GemvParams &g) {
    g.err = reinterpret_cast<int *>(m->out_tokens + kMaxChunk);
}

// One fused linear layer of the step: the tensor-core GEMM for steps of
// kGemmMinM+ tokens in a format it covers, else the GEMV.
static cudaError_t launch_linear(nexus_cuda_model *m, GemvParams g, cudaStream_t st) {
    if (g.m >= kGemmMinM && gemm_supported(g.fmt)) {
        GemmScratch sc;
        m->lin.attach(g, sc);
        return launch_gemm(g, sc, st);
    }
    return launch_gemv(g, st);
}

// Tokens of the next fused step out of `remaining`.
static int step_chunk(size_t remaining) {
    if (remaining >= (size_t)kGemmMinM) return (int)std::min<size_t>(remaining, kMaxChunk);
    return remaining >= 4 ? 4 : remaining >= 2 ? 2 : 1;
}

// KV cache as a ring (KvCache::add, src/engine/mod.rs:410-426: a full cache
// drops its oldest token, so attention spans the last max_seq_len tokens).
// Token number `total` of a sequence (0-based) is written to ring slot
// total % max_seq_len and attends over min(total + 1, max_seq_len) slots --
// the same tokens as the reference's shifted cache, in rotated order.
static inline uint32_t ring_slot(const nexus_cuda_model *m, uint32_t total) { return total % m->max_seq; }
static inline uint32_t ring_len(const nexus_cuda_model *m, uint32_t total) { return std::min(total + 1, m->max_seq); }

// Tokens of the next step of one sequence that holds `total` tokens: a chunk
// of consecutive tokens stays inside the ring's first pass (a chunk's tokens
// attend to each other's slots); once the cache is full, one token per step.
static int seq_chunk(const nexus_cuda_model *m, uint32_t total, size_t remaining) {
    if (total >= m->max_seq) return 1;
    return step_chunk(std::min<size_t>(remaining, m->max_seq - total));
}

// Enqueue one fused decode step for `mc` tokens whose DevSeq entries are on the device.
// chunk: the mc tokens are consecutive positions of one sequence (a prefill
// chunk or a draft window), so attention runs as one causal chunk kernel.
static cudaError_t enqueue_step(nexus_cuda_model *m, int mc, StepProfiler *prof = nullptr, bool chunk = false) {
    const nexus_cuda_model_info &I = m->info;
    cudaStream_t st = m->b->stream;
    // this rank's share of heads and FFN rows (all of them without tensor parallelism)
    const int H = (int)I.hidden_size, D = (int)I.head_dim, F = (int)m->f_l;
    const int Hq = (int)m->hq_l, Hkv = (int)m->hkv_l, kv_dim = Hkv * D, qdim = Hq * D;
    const bool tp = m->b->tp_world > 1, lead = m->b->tp_rank == 0;
    NcclApi *nccl = tp ? nccl_api(nullptr) : nullptr;
    if (tp && !nccl) return cudaErrorInvalidValue;
    // partial sums of the column-sliced o_proj/down meet here: rank 0 adds the
    // residual, the others store their part, and the all-reduce sums them
    auto reduce_hidden = [&]() -> cudaError_t {
        if (!tp) return cudaSuccess;
        if (m->b->peer_ok && (size_t)mc * H <= m->b->peer.max_floats) {
            PeerReduce pr = m->b->peer;
            pr.err = reinterpret_cast<int *>(m->out_tokens + kMaxChunk);
            const cudaError_t pe = launch_peer_allreduce(pr, m->hidden, (size_t)mc * H, st);
            if (pe != cudaSuccess) m->b->step_error = std::string("peer all-reduce launch: ") + cudaGetErrorString(pe);
            return pe;
        }
        ncclResult_t r = nccl->all_reduce(m->hidden, m->hidden, (size_t)mc * H, ncclFloat32, ncclSum, m->b->comm, st);
        if (r != ncclSuccess) m->b->step_error = std::string("ncclAllReduce(hidden): ") + nccl->error_string(r);
        return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
    };
    const int pdl = m->use_pdl ? 1 : 0;
    cudaError_t e;
    EmbedParams ep = {};
    ep.fmt = m->embd_fmt;
    ep.m = mc;
    ep.hidden = H;
    ep.vocab_rows = m->embd_rows;
    ep.table = m->embd;
    ep.out = m->hidden;
    ep.seqs = m->seqs;
    ep.pdl = 0;  // first kernel of the step: plain stream order after the host copies
    if (prof) prof->begin();
    if ((e = launch_embed(ep, st)) != cudaSuccess) return e;
    if (prof) prof->end("embed", (double)format_bytes(m->embd_fmt, (size_t)H) * mc + 4.0 * mc * H);
    const bool packed = m->bits_k > 0;
    for (uint32_t l = 0; l < I.num_layers; l++) {
        Layer &L = m->layers[l];
        GemvParams g = {};
        set_split_scratch(m, g);
        g.m = mc;
        g.pdl = pdl;
        g.eps = I.rms_norm_eps;
        // attn_norm -> fused Q|K|V -> RoPE -> KV write
        g.fmt = L.qkv.fmt;
        g.w_main = L.qkv.main;
        g.w_aux = L.qkv.aux;
        g.n = L.qkv.n;
        g.k = H;
        g.x = m->hidden;
        g.x_stride = H;
        g.norm_w = L.attn_norm;
        g.epi = EPI_QKV;
        g.x_bits = m->x_bits_norm;
        g.qkv.hq = Hq;
        g.qkv.hkv = Hkv;
        g.qkv.head_dim = D;
        g.qkv.q_out = m->q;
        g.qkv.rope_cos = m->rope_cos;
        g.qkv.rope_sin = m->rope_sin;
        g.qkv.k_cache = L.k_cache;
        g.qkv.v_cache = L.v_cache;
        g.qkv.pages = dev_pages(m);
        g.qkv.kv_scratch = packed ? m->kv_scratch : nullptr;
        g.qkv.seqs = m->seqs;
        g.qkv.seq_ids = m->seq_ids;
        if (prof) prof->begin();
        if ((e = launch_linear(m, g, st)) != cudaSuccess) return e;
        if (prof) prof->end("qkv", gemv_bytes(L.qkv, mc, H, qdim + 2 * kv_dim) + 4.0 * H);
        if (packed) {
            KvPackParams kp = {};
            kp.m = mc;
            kp.kv_dim = kv_dim;
            kp.bits_k = (int)m->bits_k;
            kp.bits_v = (int)m->bits_v;
            kp.kv_scratch = m->kv_scratch;
            kp.kp_data = L.kp;
            kp.vp_data = L.vp;
            kp.kp_min = L.kmin;
            kp.kp_scale = L.kscale;
            kp.vp_min = L.vmin;
            kp.vp_scale = L.vscale;
            kp.pk_bpt_k = m->bpt_k;
            kp.pk_bpt_v = m->bpt_v;
            kp.pages = dev_pages(m);
            kp.seqs = m->seqs;
            kp.seq_ids = m->seq_ids;
            kp.pdl = pdl;
            if (prof) prof->begin();
        if ((e = launch_kv_pack(kp, st)) != cudaSuccess) return e;
        if (prof) prof->end("kv_pack", (double)mc * (8.0 * kv_dim + m->bpt_k + m->bpt_v + 16));
        }
        double attn_bytes = 0;
        if (prof) {
            for (int t = 0; t < mc; t++) {
                const double ctx = (double)m->h_seqs[t].seq_len;
                attn_bytes += packed ? ctx * (m->bpt_k + m->bpt_v + 16.0) : ctx * 8.0 * kv_dim;
                attn_bytes += 8.0 * qdim;
            }
        }
        AttnParams a = {};
        a.hq = Hq;
        a.hkv = Hkv;
        a.head_dim = D;
        a.m = mc;
        a.q = m->q;
        a.out = m->attn;
        a.scale = 1.0f / sqrtf((float)D);
        a.k_cache = L.k_cache;
        a.v_cache = L.v_cache;

        a.bits_k = (int)m->bits_k;
        a.bits_v = (int)m->bits_v;
        a.kp_data = L.kp;
        a.vp_data = L.vp;
        a.kp_min = L.kmin;
        a.kp_scale = L.kscale;
        a.vp_min = L.vmin;
        a.vp_scale = L.vscale;
        a.pk_bpt_k = m->bpt_k;
        a.pk_bpt_v = m->bpt_v;
        a.pages = dev_pages(m);
        a.seqs = m->seqs;
        a.seq_ids = m->seq_ids;
        a.kv_dim = kv_dim;
        a.nsplit = m->nsplit[mc];
        if (a.bits_k > 0 && attention_pk_supported(a)) a.nsplit = m->nsplit_pk[mc];
        a.part = m->part;
        a.counters = m->counters;
        a.pdl = pdl;
        if (prof) prof->begin();
        if (chunk && mc > 1 && attention_prefill_supported(a)) e = launch_attention_prefill(a, st);
        else e = launch_attention(a, st);
        if (e != cudaSuccess) return e;
        if (prof) prof->end("attention", attn_bytes);
        // o_proj + residual
        GemvParams o = {};
        set_split_scratch(m, o);
        o.m = mc;
        o.pdl = pdl;
        o.fmt = L.o.fmt;
        o.w_main = L.o.main;
        o.w_aux = L.o.aux;
        o.n = H;
        o.k = qdim;
        o.x = m->attn;
        o.x_stride = qdim;
        o.epi = lead ? EPI_ADD : EPI_STORE;
        o.x_bits = m->x_bits_norm;
        o.y = m->hidden;
        o.y_stride = H;
        if (prof) prof->begin();
        if ((e = launch_linear(m, o, st)) != cudaSuccess) return e;
        if ((e = reduce_hidden()) != cudaSuccess) return e;
        if (prof) prof->end("o_proj", gemv_bytes(L.o, mc, qdim, H) + 4.0 * mc * H);
        // ffn_norm -> gate/up -> SwiGLU
        GemvParams gu = {};
        set_split_scratch(m, gu);
        gu.m = mc;
        gu.pdl = pdl;
        gu.eps = I.rms_norm_eps;
        gu.fmt = L.gateup.fmt;
        gu.w_main = L.gateup.main;
        gu.w_aux = L.gateup.aux;
        gu.n = 2 * F;
        gu.k = H;
        gu.x = m->hidden;
        gu.x_stride = H;
        gu.norm_w = L.ffn_norm;
        gu.epi = EPI_SWIGLU;
        gu.x_bits = m->x_bits_norm;
        gu.y = m->gated;
        gu.y_stride = F;
        if (prof) prof->begin();
        if ((e = launch_linear(m, gu, st)) != cudaSuccess) return e;
        if (prof) prof->end("gate_up", gemv_bytes(L.gateup, mc, H, F) + 4.0 * H);
        // down + residual
        GemvParams dn = {};
        set_split_scratch(m, dn);
        dn.m = mc;
        dn.pdl = pdl;
        dn.fmt = L.down.fmt;
        dn.w_main = L.down.main;
        dn.w_aux = L.down.aux;
        dn.n = H;
        dn.k = F;
        dn.x = m->gated;
        dn.x_stride = F;
        dn.epi = lead ? EPI_ADD : EPI_STORE;
        dn.y = m->hidden;
        dn.y_stride = H;
        if (prof) prof->begin();
        if ((e = launch_linear(m, dn, st)) != cudaSuccess) return e;
        if ((e = reduce_hidden()) != cudaSuccess) return e;
        if (prof) prof->end("down", gemv_bytes(L.down, mc, F, H) + 4.0 * mc * H);
    }
    // transformer_logits: output norm + head + greedy argmax
    if (m->has_head) {
        GemvParams hd = {};
        set_split_scratch(m, hd);
        hd.m = mc;
        hd.pdl = pdl;
        hd.eps = I.rms_norm_eps;
        hd.fmt = m->head.fmt;
        hd.w_main = m->head.main;
        hd.w_aux = m->head.aux;
        hd.n = m->head.n;
        hd.k = H;
        hd.x = m->hidden;
        hd.x_stride = H;
        hd.norm_w = m->out_norm;
        hd.epi = EPI_ARGMAX;
        hd.x_bits = m->x_bits_norm;
        hd.y = m->logits;
        hd.y_stride = (int)m->v_l;
        hd.row_offset = (int)m->sl.vocab_begin;
        hd.seqs = m->seqs;
        if (prof) prof->begin();
        if ((e = launch_linear(m, hd, st)) != cudaSuccess) return e;
        if (tp) {
            // greedy over all ranks' vocab slices: the packed (value, index)
            // keys reduce with max; the rest of DevSeq is equal on every rank
            static_assert(sizeof(DevSeq) == 24, "DevSeq is three 64-bit words");
            ncclResult_t r = nccl->all_reduce(m->seqs, m->seqs, (size_t)mc * 3, ncclUint64, ncclMax, m->b->comm, st);
            if (r != ncclSuccess) {
                m->b->step_error = std::string("ncclAllReduce(argmax): ") + nccl->error_string(r);
                return cudaErrorUnknown;
            }
        }
        if (prof) prof->end("head", gemv_bytes(m->head, mc, H, (int)I.vocab_rows) + 4.0 * H);
    } else {
        if ((e = launch_rms_norm(m->hidden, m->out_norm, m->logits, mc, H, I.rms_norm_eps, st)) != cudaSuccess) return e;
        for (int t = 0; t < mc; t++) {
            // k_argmax accumulates into best (cleared by the embedding kernel)
            if ((e = launch_argmax(m->logits + (size_t)t * H, H, &m->seqs[t].best, st)) != cudaSuccess) return e;
        }
    }
    if (prof) prof->begin();
    e = launch_advance(m->seqs, mc, m->out_tokens, m->max_seq, m->has_head ? pdl : 0, st);
    if (prof) prof->end("advance", 64.0 * mc);
    return e;
}

// One single-token step on the persistent kernel: k_embed decodes the
// token's embedding row (bit-exact) and clears the argmax, then the step
// kernel runs every layer, the head and the advance.
static cudaError_t enqueue_persistent_step(nexus_cuda_model *m, StepProfiler *prof = nullptr) {
    cudaStream_t st = m->b->stream;
    EmbedParams ep = {};
    ep.fmt = m->embd_fmt;
    ep.m = 1;
    ep.hidden = (int)m->info.hidden_size;
    ep.vocab_rows = m->embd_rows;
    ep.table = m->embd;
    ep.out = m->hidden;
    ep.seqs = m->seqs;
    if (prof) prof->begin();
    cudaError_t e = launch_embed(ep, st);
    if (e != cudaSuccess) return e;
    if (prof) prof->end("embed", (double)format_bytes(m->embd_fmt, (size_t)m->info.hidden_size) + 4.0 * m->info.hidden_size);
    if (prof) prof->begin();
    e = launch_decode_step(m->step, m->step_launch, st);
    if (prof) {
        // algorithmic bytes: every weight once, the K/V read by attention
        const double ctx = (double)m->h_seqs[0].seq_len;
        prof->end("decode_step", (double)m->info.weight_bytes + ctx * 8.0 * m->kvd_l * m->info.num_layers);
    }
    return e;
}

static int run_step(nexus_cuda_model *m, int mc, bool chunk = false) {
    nx::TraceRange tr(chunk ? "step chunk" : "step", mc);
    nexus_cuda_backend *b = m->b;
    cudaStream_t st = b->stream;
    if (b->tp_failed)
        return set_err(b, NEXUS_E_TIMEOUT, "an earlier all-reduce gave up on a peer: the tensor-parallel group is "
                                           "out of step; free the backend and build a new group");
    if (mc == 1 && m->use_step) {
        NX_CUDA(b, enqueue_persistent_step(m));
        return NEXUS_OK;
    }
    chunk = chunk && mc > 1;
    cudaGraphExec_t *graphs = chunk ? m->graph_chunk : m->graph;
    if (m->use_graph && m->has_head) {
        if (!graphs[mc]) {
            cudaGraph_t g = nullptr;
            NX_CUDA(b, cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
            b->step_error.clear();
            cudaError_t e = enqueue_step(m, mc, nullptr, chunk);
            cudaError_t e2 = cudaStreamEndCapture(st, &g);
            if (e != cudaSuccess || e2 != cudaSuccess) {
                if (g) cudaGraphDestroy(g);
                return set_err(b, NEXUS_E_CUDA, std::string("graph capture: ") +
                                                   cudaGetErrorString(e != cudaSuccess ? e : e2) +
                                                   (b->step_error.empty() ? "" : " (" + b->step_error + ")"));
            }
            e = cudaGraphInstantiate(&graphs[mc], g, 0);
            cudaGraphDestroy(g);
            if (e != cudaSuccess) {
                graphs[mc] = nullptr;
                return set_err(b, NEXUS_E_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
            }
        }
        NX_CUDA(b, cudaGraphLaunch(graphs[mc], st));
    } else {
        NX_CUDA(b, enqueue_step(m, mc, nullptr, chunk));
    }
    return NEXUS_OK;
}

// A kernel gave up on a bounded wait: report it and clear the flag.
static int device_timeout(nexus_cuda_model *m) {
    cudaMemsetAsync(m->out_tokens + kMaxChunk, 0, 4, m->b->stream);
    if (m->use_step) {
        // an abandoned step may leave its arrival counters part-way
        cudaMemsetAsync(m->step.bar, 0, 8, m->b->stream);
        cudaMemsetAsync(m->step.gcounters, 0, m->step_gcounter_slots * 4, m->b->stream);
        cudaMemsetAsync(m->step.attn_counters, 0, (size_t)m->step.hkv * 4, m->b->stream);
    }
    cudaStreamSynchronize(m->b->stream);
    // the ranks no longer agree on how many all-reduces have run
    if (m->b->tp_world > 1) m->b->tp_failed = true;
    return set_err(m->b, NEXUS_E_TIMEOUT, "a device wait timed out (weight stream or a peer did not arrive)");
}

// Host-driven step over `items` (at most kMaxChunk), results to host.
struct StepItem {
    uint32_t sid, token, position, slot;
};

static int host_step(nexus_cuda_model *m, const StepItem *items, int mc, float *logits_out, int logits_last_only,
                     uint32_t *tokens_out) {
    nexus_cuda_backend *b = m->b;
    cudaStream_t st = b->stream;
    for (int t = 0; t < mc; t++) {
        DevSeq s = {};
        s.token = items[t].token;
        s.position = items[t].position;
        s.slot = ring_slot(m, items[t].slot);
        s.seq_len = ring_len(m, items[t].slot);
        m->h_seqs[t] = s;
        m->h_seq_ids[t] = items[t].sid;
    }
    NX_CUDA(b, pages_upload(m));
    NX_CUDA(b, cudaMemcpyAsync(m->seqs, m->h_seqs, mc * sizeof(DevSeq), cudaMemcpyHostToDevice, st));
    NX_CUDA(b, cudaMemcpyAsync(m->seq_ids, m->h_seq_ids, mc * 4, cudaMemcpyHostToDevice, st));
    bool chunk = true;  // one sequence, consecutive slots
    for (int t = 1; t < mc; t++)
        chunk = chunk && items[t].sid == items[0].sid && items[t].slot == items[0].slot + (uint32_t)t;
    int rc = run_step(m, mc, chunk);
    if (rc) return rc;
    const size_t V = m->info.vocab_rows;
    std::vector<float> gathered;
    if (logits_out && b->tp_world > 1) {
        // every rank holds its vocab slice: gather [world][mc][v_l], reorder on the host
        NcclApi *nccl = nccl_api(nullptr);
        const size_t per = (size_t)mc * m->v_l;
        ncclResult_t r = nccl->all_gather(m->logits, m->logits_gather, per, ncclFloat32, b->comm, st);
        if (r != ncclSuccess) return set_err(b, NEXUS_E_COMM, std::string("logits all-gather: ") + nccl->error_string(r));
        gathered.resize(per * b->tp_world);
        NX_CUDA(b, cudaMemcpyAsync(gathered.data(), m->logits_gather, gathered.size() * 4, cudaMemcpyDeviceToHost, st));
    } else if (logits_out) {
        if (logits_last_only)
            NX_CUDA(b, cudaMemcpyAsync(logits_out, m->logits + (size_t)(mc - 1) * V, V * 4, cudaMemcpyDeviceToHost, st));
        else
            NX_CUDA(b, cudaMemcpyAsync(logits_out, m->logits, (size_t)mc * V * 4, cudaMemcpyDeviceToHost, st));
    }
    NX_CUDA(b, cudaMemcpyAsync(m->h_out_tokens, m->out_tokens, (kMaxChunk + 1) * 4, cudaMemcpyDeviceToHost, st));
    NX_CUDA(b, cudaStreamSynchronize(st));
    if (m->h_out_tokens[kMaxChunk]) return device_timeout(m);
    if (!gathered.empty()) {
        const size_t vl = m->v_l;
        for (int t = logits_last_only ? mc - 1 : 0; t < mc; t++) {
            float *dst = logits_out + (logits_last_only ? 0 : (size_t)t * V);
            for (int r = 0; r < b->tp_world; r++)
                memcpy(dst + (size_t)r * vl, gathered.data() + ((size_t)r * mc + t) * vl, vl * 4);
        }
    }
    if (tokens_out) memcpy(tokens_out, m->h_out_tokens, mc * 4);
    return NEXUS_OK;
}

extern "C" int nexus_cuda_model_load(nexus_cuda_backend *b, const char *gguf_path, nexus_cuda_model **out) {
    nx::TraceRange tr("nexus_cuda_model_load");
    if (!b || !gguf_path || !out) return set_err(b, NEXUS_E_INVALID, "NULL argument");
    *out = nullptr;
    std::lock_guard<std::mutex> lk(b->mu);
    cudaSetDevice(b->device);
    return model_load(b, gguf_path, out);
}

extern "C" int nexus_cuda_model_free(nexus_cuda_model *m) {
    model_release(m);
    return NEXUS_OK;
}

extern "C" int nexus_cuda_model_get_info(const nexus_cuda_model *m, nexus_cuda_model_info *info) {
    if (!m || !info) return NEXUS_E_INVALID;
    *info = m->info;
    return NEXUS_OK;
}

extern "C" int nexus_cuda_seq_reset(nexus_cuda_model *m, uint32_t seq_id) {
    if (!m || seq_id >= m->max_batch) return set_err(m ? m->b : nullptr, NEXUS_E_INVALID, "bad sequence id");
    m->seq_len[seq_id] = 0;
    return NEXUS_OK;
}

extern "C" int nexus_cuda_seq_len(nexus_cuda_model *m, uint32_t seq_id, uint32_t *len) {
    if (!m || !len || seq_id >= m->max_batch) return set_err(m ? m->b : nullptr, NEXUS_E_INVALID, "bad sequence id");
    *len = std::min(m->seq_len[seq_id], m->max_seq);  // KvCache::seq_len: the cached tokens
    return NEXUS_OK;
}

// The sequence can take `add` more tokens: within max_seq_len and inside its
// KV pages (the library's own pages are bound here when it has no list).
extern "C" int nexus_cuda_seq_set_pages(nexus_cuda_model *m, uint32_t seq_id, const uint32_t *page_ids,
                                        uint32_t n_pages) {
    if (!m || (n_pages && !page_ids)) return set_err(m ? m->b : nullptr, NEXUS_E_INVALID, "NULL argument");
    if (seq_id >= m->max_batch) return set_err(m->b, NEXUS_E_INVALID, "bad sequence id");
    std::lock_guard<std::mutex> lk(m->b->mu);
    if (n_pages == 0) {
        // the request is done: its cache is cleared and its pages go back to the pool
        m->seq_len[seq_id] = 0;
        pages_release(m, seq_id);
        return NEXUS_OK;
    }
    return pages_bind(m, seq_id, page_ids, n_pages);
}

static int check_slot(nexus_cuda_model *m, uint32_t sid, uint32_t add) {
    if (sid >= m->max_batch) return set_err(m->b, NEXUS_E_INVALID, "bad sequence id");
    int rc = pages_default(m, sid);
    if (!rc) rc = pages_cover(m, sid, std::min<uint64_t>((uint64_t)m->seq_len[sid] + add, m->max_seq));
    return rc;
}

static int check_position(nexus_cuda_model *m, uint64_t position) {
    if (position >= m->rope_positions)
        return set_err(m->b, NEXUS_E_INVALID, "position beyond the RoPE table (4 x max_seq_len positions)");
    return NEXUS_OK;
}

extern "C" int nexus_cuda_decode(nexus_cuda_model *m, uint32_t seq_id, uint32_t token, uint32_t position,
                                 float *logits, uint32_t *argmax) {
    nx::TraceRange tr("nexus_cuda_decode");
    if (!m) return set_err(nullptr, NEXUS_E_INVALID, "model is NULL");
    std::lock_guard<std::mutex> lk(m->b->mu);
    cudaSetDevice(m->b->device);
    int rc = check_slot(m, seq_id, 1);
    if (!rc) rc = check_position(m, position);
    if (rc) return rc;
    StepItem it = {seq_id, token, position, m->seq_len[seq_id]};
    NX_CUDA(m->b, cudaEventRecord(m->ev0, m->b->stream));
    uint32_t tok = 0;
    rc = host_step(m, &it, 1, logits, 1, &tok);
    if (rc) return rc;
    cudaEventRecord(m->ev1, m->b->stream);
    cudaEventSynchronize(m->ev1);
    cudaEventElapsedTime(&m->last_ms, m->ev0, m->ev1);
    m->seq_len[seq_id] += 1;
    if (argmax) *argmax = tok;
    return NEXUS_OK;
}

static int prefill_impl(nexus_cuda_model *m, uint32_t seq_id, const uint32_t *tokens, size_t n, float *logits,
                        uint32_t *argmax) {
    m->seq_len[seq_id] = 0;
    if (n == 0) return NEXUS_OK;
    int rc = check_slot(m, seq_id, (uint32_t)std::min<size_t>(n, 0xffffffffu));
    if (!rc) rc = check_position(m, n - 1);
    if (rc) return rc;
    NX_CUDA(m->b, cudaEventRecord(m->ev0, m->b->stream));
    size_t p = 0;
    uint32_t last = 0;
    while (p < n) {
        const int mc = seq_chunk(m, (uint32_t)p, n - p);
        StepItem it[kMaxChunk];
        for (int j = 0; j < mc; j++) it[j] = {seq_id, tokens[p + j], (uint32_t)(p + j), (uint32_t)(p + j)};
        const bool final = p + mc == n;
        uint32_t toks[kMaxChunk];
        rc = host_step(m, it, mc, final ? logits : nullptr, 1, toks);
        if (rc) return rc;
        last = toks[mc - 1];
        p += mc;
        m->seq_len[seq_id] = (uint32_t)p;
    }
    cudaEventRecord(m->ev1, m->b->stream);
    cudaEventSynchronize(m->ev1);
    cudaEventElapsedTime(&m->last_ms, m->ev0, m->ev1);
    if (argmax) *argmax = last;
    return NEXUS_OK;
}

extern "C" int nexus_cuda_prefill(nexus_cuda_model *m, uint32_t seq_id, const uint32_t *tokens, size_t n,
                                  float *logits, uint32_t *argmax) {
    nx::TraceRange tr("nexus_cuda_prefill", (long long)n);
    if (!m || (n && !tokens)) return set_err(m ? m->b : nullptr, NEXUS_E_INVALID, "NULL argument");
    if (seq_id >= m->max_batch) return set_err(m->b, NEXUS_E_INVALID, "bad sequence id");
    std::lock_guard<std::mutex> lk(m->b->mu);
    cudaSetDevice(m->b->device);
    return prefill_impl(m, seq_id, tokens, n, logits, argmax);
}

extern "C" int nexus_cuda_generate(nexus_cuda_model *m, uint32_t seq_id, const uint32_t *prompt, size_t n,
                                   size_t max_tokens, uint32_t *out) {
    nx::TraceRange tr("nexus_cuda_generate", (long long)max_tokens);
    if (!m || !out || (n && !prompt)) return set_err(m ? m->b : nullptr, NEXUS_E_INVALID, "NULL argument");
    if (seq_id >= m->max_batch) return set_err(m->b, NEXUS_E_INVALID, "bad sequence id");
    std::lock_guard<std::mutex> lk(m->b->mu);
    cudaSetDevice(m->b->device);
    nexus_cuda_backend *b = m->b;
    memcpy(out, prompt, n * 4);
    uint32_t next = 0;
    int rc = prefill_impl(m, seq_id, prompt, n, nullptr, &next);
    if (rc) return rc;
    if (max_tokens == 0) return NEXUS_OK;
    rc = check_slot(m, seq_id, (uint32_t)max_tokens);
    if (!rc) rc = check_position(m, n + max_tokens - 1);
    if (rc) return rc;
    // sample_token on empty logits returns 0 (src/engine/mod.rs:825-827)
    if (n == 0) next = 0;
    // Device-chained greedy loop: each graph replay decodes one token and the
    // closing kernel feeds its argmax into the next replay.
    DevSeq s = {};
    s.token = next;
    s.position = (uint32_t)n;
    s.slot = ring_slot(m, m->seq_len[seq_id]);
    s.seq_len = ring_len(m, m->seq_len[seq_id]);
    m->h_seqs[0] = s;
    m->h_seq_ids[0] = seq_id;
    cudaStream_t st = b->stream;
    NX_CUDA(b, pages_upload(m));
    NX_CUDA(b, cudaMemcpyAsync(m->seqs, m->h_seqs, sizeof(DevSeq), cudaMemcpyHostToDevice, st));
    NX_CUDA(b, cudaMemcpyAsync(m->seq_ids, m->h_seq_ids, 4, cudaMemcpyHostToDevice, st));
    uint32_t *ring = nullptr;
    NX_CUDA(b, dalloc(&ring, max_tokens));
    out[n] = next;
    NX_CUDA(b, cudaEventRecord(m->ev0, st));
    for (size_t i = 0; i < max_tokens; i++) {
        rc = run_step(m, 1);
        if (rc) break;
        // out_tokens[0] is the token the next step consumes
        if (cudaMemcpyAsync(ring + i, m->out_tokens, 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess) {
            rc = set_err(b, NEXUS_E_CUDA, "ring copy failed");
            break;
        }
    }
    cudaEventRecord(m->ev1, st);
    if (!rc) cudaMemcpyAsync(m->h_out_tokens, m->out_tokens, (kMaxChunk + 1) * 4, cudaMemcpyDeviceToHost, st);
    if (!rc && max_tokens > 1)
        rc = cudaMemcpyAsync(out + n + 1, ring, (max_tokens - 1) * 4, cudaMemcpyDeviceToHost, st) == cudaSuccess
                 ? NEXUS_OK
                 : set_err(b, NEXUS_E_CUDA, "token copy failed");
    cudaError_t e = cudaStreamSynchronize(st);
    cudaEventElapsedTime(&m->last_ms, m->ev0, m->ev1);
    cudaFree(ring);
    if (rc) return rc;
    if (e != cudaSuccess) return set_err(b, NEXUS_E_CUDA, cudaGetErrorString(e));
    if (m->h_out_tokens[kMaxChunk]) return device_timeout(m);
    m->seq_len[seq_id] += (uint32_t)max_tokens;
    return NEXUS_OK;
}

// generate_with_draft_tokens at temperature 0 (src/engine/mod.rs:1244-1291):
// the output is the greedy continuation; a draft token counts as accepted when
// it equals the greedy token of its position.  Instead of one decode per token
// the draft is verified in windows: the next verified token and the following
// draft tokens run as one multi-token step (causal attention inside the step),
// the greedy token after each of them comes back, the drafts that match are
// kept and the cache is cut back to the first mismatch.
extern "C" int nexus_cuda_generate_with_draft(nexus_cuda_model *m, uint32_t seq_id, const uint32_t *prompt,
                                              size_t n, const uint32_t *draft, size_t n_draft, size_t max_tokens,
                                              uint32_t window, uint32_t *out, uint32_t *accepted, uint32_t *rejected) {
    nx::TraceRange tr("nexus_cuda_generate_with_draft", (long long)max_tokens);
    if (!m || !out || (n && !prompt) || (n_draft && !draft))
        return set_err(m ? m->b : nullptr, NEXUS_E_INVALID, "NULL argument");
    if (seq_id >= m->max_batch) return set_err(m->b, NEXUS_E_INVALID, "bad sequence id");
    std::lock_guard<std::mutex> lk(m->b->mu);
    cudaSetDevice(m->b->device);
    const uint32_t win = std::max<uint32_t>(1, std::min<uint32_t>(window ? window : 8, kMaxChunk));
    memcpy(out, prompt, n * 4);
    uint32_t next = 0;
    int rc = prefill_impl(m, seq_id, prompt, n, nullptr, &next);
    if (rc) return rc;
    if (n == 0) next = 0;  // sample_token on empty logits returns 0 (src/engine/mod.rs:825-827)
    if (max_tokens) {
        rc = check_slot(m, seq_id, (uint32_t)std::min<size_t>(max_tokens, 0xffffffffu));
        if (!rc) rc = check_position(m, n + max_tokens - 1);
        if (rc) return rc;
    }
    NX_CUDA(m->b, cudaEventRecord(m->ev0, m->b->stream));
    size_t i = 0;  // generated tokens so far; out[n + i] is the next to verify
    StepItem it[kMaxChunk];
    uint32_t am[kMaxChunk];
    while (i < max_tokens) {
        // window: the verified token, then the drafts that follow it
        size_t w = std::min<size_t>(win, max_tokens - i);
        if (i + 1 >= n_draft) w = 1;
        else w = std::min(w, n_draft - i);
        const uint32_t base = m->seq_len[seq_id];
        // a window is cut back to its first rejection, which a wrapped ring
        // cannot undo: windows stay inside the ring's first pass
        if ((uint64_t)base + w > m->max_seq) w = 1;
        std::vector<uint32_t> toks(w);
        toks[0] = next;
        for (size_t j = 1; j < w; j++) toks[j] = draft[i + j];
        for (size_t p = 0; p < w;) {
            const int mc = seq_chunk(m, base + (uint32_t)p, w - p);
            for (int j = 0; j < mc; j++)
                it[j] = {seq_id, toks[p + j], (uint32_t)(n + i + p + j), base + (uint32_t)(p + j)};
            rc = host_step(m, it, mc, nullptr, 0, am + p);
            if (rc) return rc;
            p += mc;
        }
        // keep the verified token and every draft that matches the greedy token before it
        size_t J = 1;
        while (J < w && toks[J] == am[J - 1]) J++;
        for (size_t j = 0; j < J; j++) out[n + i + j] = toks[j];
        m->seq_len[seq_id] = base + (uint32_t)J;  // drop the K/V of a rejected draft
        next = am[J - 1];
        i += J;
    }
    cudaEventRecord(m->ev1, m->b->stream);
    cudaEventSynchronize(m->ev1);
    cudaEventElapsedTime(&m->last_ms, m->ev0, m->ev1);
    uint32_t acc = 0, rej = 0;
    for (size_t p = 0; p < std::min(n_draft, max_tokens); p++) (draft[p] == out[n + p] ? acc : rej)++;
    if (accepted) *accepted = acc;
    if (rejected) *rejected = rej;
    return NEXUS_OK;
}

extern "C" int nexus_cuda_decode_batch(nexus_cuda_model *m, const nexus_decode_item *items, size_t n,
                                       uint32_t *out_tokens, float *out_logits) {
    nx::TraceRange tr("nexus_cuda_decode_batch", (long long)n);
    if (!m || (n && !items)) return set_err(m ? m->b : nullptr, NEXUS_E_INVALID, "NULL argument");
    std::lock_guard<std::mutex> lk(m->b->mu);
    cudaSetDevice(m->b->device);
    std::vector<bool> seen(m->max_batch, false);
    for (size_t i = 0; i < n; i++) {
        const uint32_t sid = items[i].seq_id;
        if (sid >= m->max_batch) return set_err(m->b, NEXUS_E_INVALID, "bad sequence id");
        int rc = check_position(m, items[i].position);
        if (rc) return rc;
        if (seen[sid]) return set_err(m->b, NEXUS_E_INVALID, "a sequence appears twice in one decode batch");
        seen[sid] = true;
    }
    // the scheduler's page lists (ScheduledDecode.kv_pages) become the
    // sequences' device page tables; then every item must fit its pages
    for (size_t i = 0; i < n; i++) {
        const uint32_t sid = items[i].seq_id;
        if (items[i].n_pages && !items[i].page_ids) return set_err(m->b, NEXUS_E_INVALID, "n_pages without page_ids");
        if (items[i].page_ids) {
            int rc = pages_bind(m, sid, items[i].page_ids, items[i].n_pages);
            if (rc) return rc;
        }
        int rc = check_slot(m, sid, 1);
        if (rc) return rc;
    }
    NX_CUDA(m->b, cudaEventRecord(m->ev0, m->b->stream));
    const size_t V = m->info.vocab_rows;
    for (size_t p = 0; p < n;) {
        const int mc = step_chunk(n - p);
        StepItem it[kMaxChunk];
        for (int j = 0; j < mc; j++) {
            const nexus_decode_item &d = items[p + j];
            it[j] = {d.seq_id, d.token, d.position, m->seq_len[d.seq_id]};
        }
        int rc = host_step(m, it, mc, out_logits ? out_logits + p * V : nullptr, 0, out_tokens ? out_tokens + p : nullptr);
        if (rc) return rc;
        for (int j = 0; j < mc; j++) m->seq_len[items[p + j].seq_id] += 1;
        p += mc;
    }
    cudaEventRecord(m->ev1, m->b->stream);
    cudaEventSynchronize(m->ev1);
    cudaEventElapsedTime(&m->last_ms, m->ev0, m->ev1);
    return NEXUS_OK;
}

extern "C" int nexus_cuda_last_step_ms(const nexus_cuda_model *m, float *ms) {
    if (!m || !ms) return NEXUS_E_INVALID;
    *ms = m->last_ms;
    return NEXUS_OK;
}

extern "C" int nexus_cuda_profile_decode(nexus_cuda_model *m, uint32_t seq_id, uint32_t token, uint32_t steps,
                                         nexus_kernel_profile *out, int max_out, int *n_out) {
    if (!m || !out || !n_out) return set_err(m ? m->b : nullptr, NEXUS_E_INVALID, "NULL argument");
    std::lock_guard<std::mutex> lk(m->b->mu);
    cudaSetDevice(m->b->device);
    int rc = check_slot(m, seq_id, steps);
    if (!rc) rc = check_position(m, (uint64_t)m->seq_len[seq_id] + steps);
    if (rc) return rc;
    nexus_cuda_backend *b = m->b;
    cudaStream_t st = b->stream;
    StepProfiler prof;
    prof.st = st;
    uint32_t tok = token;
    for (uint32_t i = 0; i < steps; i++) {
        const uint32_t slot = m->seq_len[seq_id];
        DevSeq s = {};
        s.token = tok;
        s.position = slot;
        s.slot = ring_slot(m, slot);
        s.seq_len = ring_len(m, slot);
        m->h_seqs[0] = s;
        m->h_seq_ids[0] = seq_id;
        NX_CUDA(b, pages_upload(m));
        NX_CUDA(b, cudaMemcpyAsync(m->seqs, m->h_seqs, sizeof(DevSeq), cudaMemcpyHostToDevice, st));
        NX_CUDA(b, cudaMemcpyAsync(m->seq_ids, m->h_seq_ids, 4, cudaMemcpyHostToDevice, st));
        if (m->use_step) NX_CUDA(b, enqueue_persistent_step(m, &prof));
        else NX_CUDA(b, enqueue_step(m, 1, &prof));
        NX_CUDA(b, cudaMemcpyAsync(m->h_out_tokens, m->out_tokens, (kMaxChunk + 1) * 4, cudaMemcpyDeviceToHost, st));
        NX_CUDA(b, cudaStreamSynchronize(st));
        if (m->h_out_tokens[kMaxChunk]) return device_timeout(m);
        tok = m->h_out_tokens[0];
        m->seq_len[seq_id] += 1;
    }
    prof.collect();
    int n = 0;
    for (auto &r : prof.recs) {
        if (n >= max_out) break;
        memset(&out[n], 0, sizeof(out[n]));
        strncpy(out[n].name, r.name.c_str(), sizeof(out[n].name) - 1);
        out[n].launches = r.launches;
        out[n].total_ms = r.ms;
        out[n].bytes_per_launch = r.bytes;
        n++;
    }
    *n_out = n;
    return NEXUS_OK;
}

extern "C" int nexus_synth_model_write(const char *path, const nexus_synth_config *cfg) {
    if (!path || !cfg) return set_err(nullptr, NEXUS_E_INVALID, "NULL argument");
    std::string err;
    int rc = nx::synth_model_write(path, cfg, err);
    if (rc) set_err(nullptr, rc, err);
    return rc;
}
