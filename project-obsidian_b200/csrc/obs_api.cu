// obs_api.cu -- the C ABI (include/obs_moe.h): context, HBM-resident weight
// store, scratch, and the MoE layer schedule on one CUDA stream.
//
// The reference keeps experts on SSD and pages the routed ones in per token
// (src/disk_io.rs:79-102, src/forward.rs:424-434), with the CPU blocking on the
// router every layer (src/router.rs:47-48).  Here every layer's experts are
// resident in HBM (about 340 MB per Qwen3-30B-A3B layer, 16.3 GB for 48), all
// scratch is allocated once in obs_create, and a forward call is a fixed
// sequence of kernel launches with no host synchronisation.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstddef>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

#include "../../include/obs_moe.h"

#include "obs_internal.cuh"

using namespace obs;

namespace {
constexpr int kDecodeMaxT = 64;  // largest T the decode path's scratch covers
// GEMM token tile (rows of one expert per work item).  The grouped GEMM kernel
// also has a 128-row form, withdrawn: on workloads whose tiles were mostly 65-127
// rows it ended in a device fault whose cause is not found, so only the 64-row
// form runs.
constexpr int kBNTile = 64;

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
}  // namespace

struct obs_ctx {
    obs_config cfg{};
    Shape sh{};
    int device = 0, num_sms = 148;
    std::string err;
    std::vector<LayerDev> layers;
    uint8_t* wmem = nullptr;
    uint8_t* smem_pool = nullptr;
    size_t wbytes = 0, sbytes = 0;
    size_t layer_bytes = 0;
    // scratch
    float* logits = nullptr;
    int32_t* ids = nullptr;
    float* wts = nullptr;
    DispatchBufs disp{};
    uint16_t* hbuf = nullptr;
    uint16_t* ybuf = nullptr;
    float* yf32 = nullptr;
    DecodeBufs dec{};
    FusedDecodeBufs fused{};
    int* err_flag = nullptr;
    uint16_t* x_dev = nullptr;
    uint16_t* out_dev = nullptr;
    uint16_t* res_dev = nullptr;
    float* bias_dev = nullptr;
    // obs_moe_forward_host_async: two staging slots of its own, an input and an
    // output copy stream (created on first use), and per slot the events that order them
    struct HostSlot {
        uint16_t *x = nullptr, *out = nullptr, *res = nullptr;
        float* bias = nullptr;
        cudaEvent_t in_done = nullptr, computed = nullptr, out_done = nullptr;
        bool used = false;
    } hs[2];
    cudaStream_t hs_in = nullptr, hs_out = nullptr;
    int hs_next = 0;
    bool hs_ready = false;
    uint16_t* xnorm_dev = nullptr;  // the layer stack's normalised input
    uint16_t* rtmp_dev = nullptr;   // the layer stack's other residual buffer
    int R_cap = 0, max_tiles = 0, decode_max = kDecodeAutoT;
    uint64_t wait_ns = kDefaultWaitNs;  // limit of every bounded device wait (obs_set_wait_limit)
    uint32_t* probe_stamp = nullptr;    // a stamp nothing writes (obs_probe_wait)
    uint64_t* trace = nullptr;  // obs_trace_enable
    int trace_n = 0;
    // expert parallelism (ep_world > 1): this rank holds E_local experts of each layer,
    // placement[layer][ep_rank * E_local + l] for local expert l (default: [e0, e0 + E_local))
    int ep_world = 1, ep_rank = 0, E_local = 0, e0 = 0;
    std::vector<std::vector<int32_t>> placement;  // [n_layers][E] global expert of each slot
    int32_t* place_dev = nullptr;                 // [n_layers][E] slot of each global expert
    uint8_t* ep_buf = nullptr;  // this rank's buffer, opened by its peers through CUDA IPC
    uint16_t** ep_row_ptr = nullptr;  // [R_cap] destination of each down-GEMM output row
    // the model's ends (obs_load_head): embedding, final norm, lm_head, and their scratch
    struct Head {
        int vocab = 0;
        uint8_t* mem = nullptr;
        uint32_t *embed_w = nullptr, *lm_w = nullptr;
        uint16_t *embed_s = nullptr, *embed_b = nullptr, *lm_s = nullptr, *lm_b = nullptr, *norm_w = nullptr;
        uint16_t* xn = nullptr;  // [kHeadMaxT, H]
        float* logits = nullptr; // [kHeadMaxT, vocab]
    } head;
    // the attention block (obs_attn_init / obs_load_attn): per layer weights and KV caches
    struct AttnLayer {
        uint8_t* mem = nullptr;
        uint32_t *qkv_w = nullptr, *o_w = nullptr;  // q | k | v rows concatenated; o
        uint16_t *qkv_s = nullptr, *qkv_b = nullptr, *o_s = nullptr, *o_b = nullptr;
        uint16_t *in_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
        uint16_t *kc = nullptr, *vc = nullptr;      // [n_seqs][n_kv][max_seq][hd]
        bool loaded = false;
    };
    obs_attn_config acfg{};
    std::vector<AttnLayer> attn;
    uint8_t* attn_scratch = nullptr;
    float* rope_cs = nullptr;   // [max_seq][hd/2][2]
    float* a_qkv = nullptr;     // [max_tokens][(nq + 2 nkv) hd]
    uint16_t* a_xn = nullptr;   // [max_tokens][H]
    uint16_t* a_q = nullptr;    // [max_tokens][nq hd]
    uint16_t* a_out = nullptr;  // [max_tokens][nq hd]
    float* a_o = nullptr;       // [max_tokens][H]
    float* a_part = nullptr;    // the attention splits' partial sums (sdpa_part_floats)
    size_t ep_bytes = 0;
    bool ep_connected = false;
    EpArgs ep{};
    // optional per-stage event timing (obs_profile_enable)
    bool prof = false;
    std::vector<cudaEvent_t> ev_pool;
    std::vector<std::pair<int, int>> ev_marks;  // (stage, index of start event; stop = +1)
};

static void prof_begin(obs_ctx* c, int stage, cudaStream_t st) {
    if (!c->prof) return;
    size_t i = c->ev_marks.size() * 2;
    while (c->ev_pool.size() < i + 2) {
        cudaEvent_t e;
        cudaEventCreate(&e);
        c->ev_pool.push_back(e);
    }
    cudaEventRecord(c->ev_pool[i], st);
    c->ev_marks.push_back({stage, (int)i});
}
static void prof_end(obs_ctx* c, cudaStream_t st) {
    if (!c->prof || c->ev_marks.empty()) return;
    cudaEventRecord(c->ev_pool[c->ev_marks.back().second + 1], st);
}

#define OBS_CHECK_CTX(c)                  \
    do {                                  \
        if (!(c)) return OBS_ERR_INVALID; \
    } while (0)

static int fail(obs_ctx* c, int code, const std::string& msg) {
    if (c) c->err = msg;
    return code;
}
static int cuda_fail(obs_ctx* c, cudaError_t e, const char* what) {
    return fail(c, OBS_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}
#define CU(call, what)                                          \
    do {                                                        \
        cudaError_t e_ = (call);                                \
        if (e_ != cudaSuccess) return cuda_fail(ctx, e_, what); \
    } while (0)

static inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ------------------------------------------------------------------ context
extern "C" int obs_abi_version(void) { return OBS_ABI_VERSION; }

// obs_create has no context to hold its message yet: it lands here (per thread)
static thread_local std::string g_create_err;

extern "C" const char* obs_last_error(const obs_ctx* ctx) { return ctx ? ctx->err.c_str() : g_create_err.c_str(); }

namespace obs {
// message of a context-free entry point, read back with obs_last_error(NULL)
void set_thread_error(const char* msg) { g_create_err = msg ? msg : ""; }
}  // namespace obs

static int fail(obs_ctx* c, int code, const std::string& msg);
namespace obs {
void ctx_shape(const obs_ctx* ctx, int* E, int* H, int* I) { *E = ctx->sh.E, *H = ctx->sh.H, *I = ctx->sh.I; }
int ctx_fail(obs_ctx* ctx, int code, const char* msg) { return fail(ctx, code, msg ? msg : ""); }
}  // namespace obs

static size_t layer_weight_bytes(const Shape& s, int E_local) {
    size_t router = align_up((size_t)s.E * s.H, 256) + 2 * align_up((size_t)s.E * (s.H / 64) * 2, 256);
    size_t gu = (size_t)E_local * (s.I / kRowTile) * (s.H / kGroup) * 2 * kBlockBytes;
    size_t dn = (size_t)E_local * (s.H / kRowTile) * (s.I / kGroup) * kBlockBytes;
    return router + align_up(gu, 256) + align_up(dn, 256);
}

extern "C" int obs_create(const obs_config* cfg, int device, obs_ctx** out) {
    if (!cfg || !out) return OBS_ERR_INVALID;
    *out = nullptr;
    obs_ctx* ctx = new obs_ctx();
    ctx->cfg = *cfg;
    ctx->sh = Shape{cfg->hidden, cfg->inter, cfg->n_experts, cfg->top_k};
    const Shape& s = ctx->sh;
    auto bad = [&](const char* m) {
        g_create_err = m;
        delete ctx;
        return OBS_ERR_INVALID;
    };
    if (cfg->group_size != 64) return bad("group_size must be 64");
    if (s.H <= 0 || s.H % 2048) return bad("hidden must be a multiple of 2048");
    if (s.I <= 0 || s.I % 256) return bad("inter must be a multiple of 256");
    if (s.E <= 0 || s.E > 256) return bad("n_experts must be in 1..256");
    if (s.K <= 0 || s.K > 16 || s.K > s.E) return bad("top_k must be in 1..min(16, n_experts)");
    if (cfg->n_layers <= 0 || cfg->max_tokens <= 0) return bad("n_layers and max_tokens must be positive");
    ctx->ep_world = cfg->ep_world > 1 ? cfg->ep_world : 1;
    ctx->ep_rank = ctx->ep_world > 1 ? cfg->ep_rank : 0;
    if (ctx->ep_world > kMaxWorld) return bad("ep_world must be at most 8");
    if (s.E % ctx->ep_world) return bad("n_experts must be a multiple of ep_world");
    if (ctx->ep_rank < 0 || ctx->ep_rank >= ctx->ep_world) return bad("ep_rank must be in [0, ep_world)");
    ctx->E_local = s.E / ctx->ep_world;
    ctx->e0 = ctx->ep_rank * ctx->E_local;
    // measured on B200: the mat-vec (fused) layer wins up to 2 tokens, the grouped GEMM from 3
    ctx->decode_max = cfg->decode_max_tokens > 0 ? cfg->decode_max_tokens : kDecodeAutoT;
    if (ctx->decode_max > kDecodeMaxT) ctx->decode_max = kDecodeMaxT;
    ctx->device = device;
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) {
        g_create_err = std::string("device: ") + cudaGetErrorString(e);
        delete ctx;
        return OBS_ERR_CUDA;
    }

    // weights for all layers
    ctx->layer_bytes = layer_weight_bytes(s, ctx->E_local);
    ctx->wbytes = ctx->layer_bytes * cfg->n_layers;
    e = cudaMalloc(&ctx->wmem, ctx->wbytes);
    if (e != cudaSuccess) {
        ctx->wmem = nullptr;
        g_create_err = std::string("weights: ") + cudaGetErrorString(e);
        obs_destroy(ctx);
        return OBS_ERR_NOMEM;
    }
    ctx->layers.resize(cfg->n_layers);
    for (int l = 0; l < cfg->n_layers; ++l) {
        uint8_t* p = ctx->wmem + ctx->layer_bytes * l;
        LayerDev& L = ctx->layers[l];
        L.router_w = reinterpret_cast<uint32_t*>(p);
        p += align_up((size_t)s.E * s.H, 256);
        L.router_s = reinterpret_cast<uint16_t*>(p);
        p += align_up((size_t)s.E * (s.H / 64) * 2, 256);
        L.router_b = reinterpret_cast<uint16_t*>(p);
        p += align_up((size_t)s.E * (s.H / 64) * 2, 256);
        L.gateup = p;
        p += align_up((size_t)ctx->E_local * (s.I / kRowTile) * (s.H / kGroup) * 2 * kBlockBytes, 256);
        L.down = p;
        L.loaded = false;
    }

    // scratch, one pool
    const int T = cfg->max_tokens, K = s.K, E = s.E, W = ctx->ep_world, EL = ctx->E_local;
    // rows the grouped GEMMs may see: every rank's routed rows for this rank's experts, padded
    ctx->R_cap = (int)align_up((size_t)W * T * K + (size_t)EL * (kSegAlign - 1), 128);
    ctx->max_tiles = ctx->R_cap / kBNTile + EL + 1;
    const int DT = ctx->decode_max > 0 ? kDecodeMaxT : 0;
    struct Item { void** p; size_t bytes; };
    std::vector<Item> items = {
        {(void**)&ctx->logits, (size_t)8 * T * E * 4},  // router partial planes (router_parts)
        {(void**)&ctx->ids, (size_t)T * K * 4},
        {(void**)&ctx->wts, (size_t)T * K * 4},
        {(void**)&ctx->disp.counts, (size_t)E * 4},
        {(void**)&ctx->disp.hist, (size_t)((W * T + kDispChunk - 1) / kDispChunk) * E * 4},
        {(void**)&ctx->disp.seg, (size_t)(E + 1) * 4},
        {(void**)&ctx->disp.slot_of, (size_t)W * T * K * 4},
        {(void**)&ctx->disp.src, (size_t)ctx->R_cap * 4},
        {(void**)&ctx->disp.tiles, (size_t)ctx->max_tiles * 16},
        {(void**)&ctx->disp.n_tiles, 16},
        {(void**)&ctx->disp.xp, (size_t)ctx->R_cap * s.H * 2},
        {(void**)&ctx->hbuf, (size_t)ctx->R_cap * s.I * 2},
        {(void**)&ctx->ybuf, (size_t)ctx->R_cap * s.H * 2},
        {(void**)&ctx->dec.part, (size_t)DT * K * (s.I / kRowTile) * kDecodeSplit * 2 * kRowTile * 4},
        {(void**)&ctx->dec.cnt_gu, (size_t)DT * K * (s.I / kRowTile) * 4},
        {(void**)&ctx->dec.hq, (size_t)DT * K * s.I * 2},
        {(void**)&ctx->dec.hmeta, (size_t)DT * K * (s.I / kGroup) * 8},
        {(void**)&ctx->dec.xq, (size_t)DT * s.H * 2},
        {(void**)&ctx->dec.xmeta, (size_t)DT * (s.H / kGroup) * 8},
        {(void**)&ctx->dec.y, (size_t)DT * K * s.H * 2},
        {(void**)&ctx->dec.cnt_dn, (size_t)DT * (s.H / kRowTile) * 4},
        {(void**)&ctx->err_flag, 16},
        {(void**)&ctx->x_dev, (size_t)T * s.H * 2},
        {(void**)&ctx->out_dev, (size_t)T * s.H * 2},
        {(void**)&ctx->res_dev, (size_t)T * s.H * 2},
        {(void**)&ctx->bias_dev, (size_t)E * 4},
        {(void**)&ctx->hs[0].x, (size_t)T * s.H * 2},
        {(void**)&ctx->hs[0].out, (size_t)T * s.H * 2},
        {(void**)&ctx->hs[0].res, (size_t)T * s.H * 2},
        {(void**)&ctx->hs[0].bias, (size_t)E * 4},
        {(void**)&ctx->hs[1].x, (size_t)T * s.H * 2},
        {(void**)&ctx->hs[1].out, (size_t)T * s.H * 2},
        {(void**)&ctx->hs[1].res, (size_t)T * s.H * 2},
        {(void**)&ctx->hs[1].bias, (size_t)E * 4},
        {(void**)&ctx->xnorm_dev, (size_t)T * s.H * 2},
        {(void**)&ctx->rtmp_dev, (size_t)T * s.H * 2},
        {(void**)&ctx->fused.ypart, (size_t)kFusedMaxT * K * (s.I / kGroup) * s.H * 8},
        {(void**)&ctx->fused.bar, 16},
        {(void**)&ctx->fused.lst, (size_t)4 * kFusedMaxT * E * 8},
        {(void**)&ctx->probe_stamp, 16},
        {(void**)&ctx->place_dev, (size_t)cfg->n_layers * E * 4},
        {(void**)&ctx->ep.send_cnt, (size_t)kMaxWorld * 4},
        {(void**)&ctx->ep.done, 16},
        {(void**)&ctx->ep.epoch, 16},
        {(void**)&ctx->ep.ids_local, W > 1 ? (size_t)W * T * K * 4 : 0},  // [W * cap_rows * K]
        {(void**)&ctx->ep.src_item, W > 1 ? (size_t)W * T * K * 4 : 0},
        {(void**)&ctx->ep.local_slot, W > 1 ? (size_t)T * K * 4 : 0},
        {(void**)&ctx->ep_row_ptr, W > 1 ? (size_t)ctx->R_cap * 8 : 0},
        {(void**)&ctx->ep.row_src, W > 1 ? (size_t)W * T * 8 : 0},
    };
    size_t total = 0;
    for (auto& it : items) total += align_up(it.bytes ? it.bytes : 16, 1024);
    e = cudaMalloc(&ctx->smem_pool, total);
    if (e != cudaSuccess) {
        ctx->smem_pool = nullptr;
        g_create_err = std::string("scratch: ") + cudaGetErrorString(e);
        obs_destroy(ctx);
        return OBS_ERR_NOMEM;
    }
    ctx->sbytes = total;
    size_t off = 0;
    for (auto& it : items) {
        *it.p = ctx->smem_pool + off;
        off += align_up(it.bytes ? it.bytes : 16, 1024);
    }
    ctx->dec.err = ctx->err_flag;
    ctx->fused.ids = ctx->ids;
    ctx->fused.wts = ctx->wts;
    ctx->fused.err = ctx->err_flag;
    ctx->fused.wait_ns = ctx->wait_ns;
    ctx->ep.wait_ns = ctx->wait_ns;
    if (W > 1) {
        // this rank's shared buffer (layout in k_ep.cu), zeroed: stamps and counts start at 0
        EpArgs& a = ctx->ep;
        a.world = W, a.rank = ctx->ep_rank, a.H = s.H, a.K = K, a.E_local = EL;
        a.cap_rows = T, a.cap_items = T * K;
        a.rows_cap = ctx->R_cap;
        a.err = ctx->err_flag;
        size_t o = 0;
        a.off_rx = o, o += align_up((size_t)W * a.cap_rows * s.H * 2, 256);
        a.off_meta = o, o += align_up((size_t)W * a.cap_rows * 32, 256);
        a.off_mtok = o, o += align_up((size_t)W * a.cap_rows * 4, 256);
        a.off_cnt = o, o += 256;
        a.off_rflag = o, o += 256;
        a.off_ret = o, o += align_up((size_t)a.cap_items * s.H * 2, 256);
        a.off_retflag = o, o += 256;
        ctx->ep_bytes = o;
        e = cudaMalloc(&ctx->ep_buf, o);
        if (e == cudaSuccess) e = cudaMemset(ctx->ep_buf, 0, o);
        if (e != cudaSuccess) {
            ctx->ep_buf = nullptr;
            g_create_err = std::string("expert-parallel buffer: ") + cudaGetErrorString(e);
            obs_destroy(ctx);
            return OBS_ERR_NOMEM;
        }
    }
    ctx->disp.atoms = ctx->R_cap / 8;
    ctx->disp.rows_cap = ctx->R_cap;
    ctx->disp.max_tiles = ctx->max_tiles;
    ctx->disp.max_chunks = (W * T + kDispChunk - 1) / kDispChunk;
    ctx->disp.err = ctx->err_flag;
    ctx->disp.bn = kBNTile;
    // counters must start at zero; the tiled buffers are zeroed so padding rows are finite
    e = cudaMemset(ctx->smem_pool, 0, total);
    // the identity placement of every layer
    ctx->placement.assign(cfg->n_layers, std::vector<int32_t>(E));
    for (auto& pl : ctx->placement)
        for (int i = 0; i < E; ++i) pl[i] = i;
    for (int l = 0; l < cfg->n_layers && e == cudaSuccess; ++l)
        e = cudaMemcpy(ctx->place_dev + (size_t)l * E, ctx->placement[l].data(), (size_t)E * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        g_create_err = std::string("scratch init: ") + cudaGetErrorString(e);
        obs_destroy(ctx);
        return OBS_ERR_CUDA;
    }
    *out = ctx;
    return OBS_OK;
}

extern "C" int obs_destroy(obs_ctx* ctx) {
    if (!ctx) return OBS_OK;
    cudaSetDevice(ctx->device);
    for (auto e : ctx->ev_pool) cudaEventDestroy(e);
    if (ctx->hs_ready) {
        cudaStreamSynchronize(ctx->hs_out);
        for (auto& h : ctx->hs) cudaEventDestroy(h.in_done), cudaEventDestroy(h.computed), cudaEventDestroy(h.out_done);
        cudaStreamDestroy(ctx->hs_in);
        cudaStreamDestroy(ctx->hs_out);
    }
    if (ctx->ep_connected)
        for (int r = 0; r < ctx->ep_world; ++r)
            if (r != ctx->ep_rank && ctx->ep.peer[r]) cudaIpcCloseMemHandle(ctx->ep.peer[r]);
    if (ctx->ep_buf) cudaFree(ctx->ep_buf);
    if (ctx->head.mem) cudaFree(ctx->head.mem);
    for (auto& a : ctx->attn)
        if (a.mem) cudaFree(a.mem);
    if (ctx->attn_scratch) cudaFree(ctx->attn_scratch);
    if (ctx->wmem) cudaFree(ctx->wmem);
    if (ctx->smem_pool) cudaFree(ctx->smem_pool);
    delete ctx;
    return OBS_OK;
}

extern "C" int obs_memory_bytes(const obs_ctx* ctx, size_t* weights, size_t* scratch) {
    if (!ctx) return OBS_ERR_INVALID;
    if (weights) *weights = ctx->wbytes;
    if (scratch) *scratch = ctx->sbytes;
    return OBS_OK;
}

// ------------------------------------------------------------------ loading
static int check_layer(obs_ctx* ctx, int layer, bool need_loaded) {
    if (layer < 0 || layer >= (int)ctx->layers.size()) return fail(ctx, OBS_ERR_INVALID, "layer out of range");
    if (need_loaded && !ctx->layers[layer].loaded) return fail(ctx, OBS_ERR_STATE, "layer not loaded");
    return OBS_OK;
}

// Copies (host or device) reference-format weights of one layer, re-tiles the
// experts into 4608-byte blocks.  src == nullptr: generate them (synth).
static int load_impl(obs_ctx* ctx, int layer, const obs_layer_weights* w, int on_dev, uint64_t seed, bool synth) {
    int rc = check_layer(ctx, layer, false);
    if (rc) return rc;
    CU(cudaSetDevice(ctx->device), "cudaSetDevice");
    const Shape& s = ctx->sh;
    LayerDev& L = ctx->layers[layer];
    // this context's experts (all of them without EP): placement[layer][e0 + l] for local expert l
    const int EL = ctx->E_local;
    const int32_t* mine = ctx->placement[layer].data() + ctx->e0;
    bool contiguous = true;
    for (int l = 1; l < EL; ++l) contiguous = contiguous && mine[l] == mine[0] + l;
    const size_t maxw = (size_t)EL * s.I * s.H / 8 * 4;  // one projection's words (all same size)
    const size_t maxg = (size_t)EL * s.I * s.H / 64 * 2;
    uint8_t* stage = nullptr;
    CU(cudaMalloc(&stage, maxw + 2 * maxg), "staging alloc");
    uint32_t* sw = reinterpret_cast<uint32_t*>(stage);
    uint16_t* ss = reinterpret_cast<uint16_t*>(stage + maxw);
    uint16_t* sb = reinterpret_cast<uint16_t*>(stage + maxw + maxg);
    cudaMemcpyKind kind = on_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    cudaError_t e = cudaSuccess;
    auto step = [&](cudaError_t r) { if (e == cudaSuccess) e = r; };
    if (synth) {
        step(launch_synth_router(seed, (uint32_t)layer, s.E, s.H, L.router_w, L.router_s, L.router_b, 0));
    } else {
        step(cudaMemcpy(L.router_w, w->router_w, (size_t)s.E * s.H, kind));
        step(cudaMemcpy(L.router_s, w->router_s, (size_t)s.E * (s.H / 64) * 2, kind));
        step(cudaMemcpy(L.router_b, w->router_b, (size_t)s.E * (s.H / 64) * 2, kind));
    }
    for (int proj = 0; proj < 3 && e == cudaSuccess; ++proj) {
        const int out_f = proj == 2 ? s.H : s.I, in_f = proj == 2 ? s.I : s.H;
        const size_t wpe = (size_t)out_f * (in_f / 8), gpe = (size_t)out_f * (in_f / 64);  // per expert
        if (synth) {
            if (contiguous)
                step(launch_synth_proj(seed, (uint32_t)layer, proj, mine[0], EL, out_f, in_f, sw, ss, sb, 0));
            else
                for (int l = 0; l < EL; ++l)
                    step(launch_synth_proj(seed, (uint32_t)layer, proj, mine[l], 1, out_f, in_f, sw + l * wpe,
                                           ss + l * gpe, sb + l * gpe, 0));
        } else {
            const uint32_t* pw = proj == 0 ? w->gate_w : proj == 1 ? w->up_w : w->down_w;
            const uint16_t* ps = proj == 0 ? w->gate_s : proj == 1 ? w->up_s : w->down_s;
            const uint16_t* pb = proj == 0 ? w->gate_b : proj == 1 ? w->up_b : w->down_b;
            if (!pw || !ps || !pb) {
                cudaFree(stage);
                return fail(ctx, OBS_ERR_INVALID, "null weight pointer");
            }
            const int runs = contiguous ? 1 : EL, per = contiguous ? EL : 1;  // copies of `per` experts each
            for (int r = 0; r < runs; ++r) {
                const size_t ge = (size_t)mine[r];
                step(cudaMemcpy(sw + r * wpe, pw + ge * wpe, per * wpe * 4, kind));
                step(cudaMemcpy(ss + r * gpe, ps + ge * gpe, per * gpe * 2, kind));
                step(cudaMemcpy(sb + r * gpe, pb + ge * gpe, per * gpe * 2, kind));
            }
        }
        if (proj < 2) step(launch_retile(sw, ss, sb, EL, out_f, in_f, L.gateup, 1, proj, 0));
        else step(launch_retile(sw, ss, sb, EL, out_f, in_f, L.down, 0, 0, 0));
        step(cudaDeviceSynchronize());
    }
    cudaFree(stage);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "load layer");
    L.loaded = true;
    return OBS_OK;
}

extern "C" int obs_load_layer(obs_ctx* ctx, int layer, const obs_layer_weights* w, int src_on_device) {
    OBS_CHECK_CTX(ctx);
    if (!w || !w->router_w || !w->router_s || !w->router_b) return fail(ctx, OBS_ERR_INVALID, "null weights");
    return load_impl(ctx, layer, w, src_on_device, 0, false);
}

extern "C" int obs_load_head(obs_ctx* ctx, int vocab, const obs_head_weights* w, int src_on_device) {
    OBS_CHECK_CTX(ctx);
    if (!w || !w->embed_w || !w->embed_s || !w->embed_b || !w->lm_w || !w->lm_s || !w->lm_b || !w->norm_w)
        return fail(ctx, OBS_ERR_INVALID, "null head weight pointer");
    if (vocab <= 0 || vocab > (1 << 24)) return fail(ctx, OBS_ERR_INVALID, "vocab out of range");
    CU(cudaSetDevice(ctx->device), "cudaSetDevice");
    auto& h = ctx->head;
    if (h.mem) {
        cudaFree(h.mem);
        h = obs_ctx::Head{};
    }
    const int H = ctx->sh.H;
    const size_t nw = (size_t)vocab * (H / 8) * 4, ng = (size_t)vocab * (H / 64) * 2;
    const size_t sizes[] = {nw, ng, ng, nw, ng, ng, (size_t)H * 2, (size_t)kHeadMaxT * H * 2,
                            (size_t)kHeadMaxT * vocab * 4};
    size_t total = 0;
    for (size_t sz : sizes) total += align_up(sz, 256);
    CU(cudaMalloc(&h.mem, total), "head alloc");
    uint8_t* p = h.mem;
    void** ptrs[] = {(void**)&h.embed_w, (void**)&h.embed_s, (void**)&h.embed_b, (void**)&h.lm_w, (void**)&h.lm_s,
                     (void**)&h.lm_b, (void**)&h.norm_w, (void**)&h.xn, (void**)&h.logits};
    for (int i = 0; i < 9; ++i) *ptrs[i] = p, p += align_up(sizes[i], 256);
    const cudaMemcpyKind kind = src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    const void* srcs[] = {w->embed_w, w->embed_s, w->embed_b, w->lm_w, w->lm_s, w->lm_b, w->norm_w};
    for (int i = 0; i < 7; ++i) CU(cudaMemcpy(*ptrs[i], srcs[i], sizes[i], kind), "head copy");
    h.vocab = vocab;
    return OBS_OK;
}

extern "C" int obs_embed(obs_ctx* ctx, const int32_t* tokens, int T, uint16_t* x, void* stream) {
    OBS_CHECK_CTX(ctx);
    if (!ctx->head.mem) return fail(ctx, OBS_ERR_STATE, "head not loaded (obs_load_head)");
    if (T < 0) return fail(ctx, OBS_ERR_INVALID, "T < 0");
    if (T == 0) return OBS_OK;
    if (!tokens || !x) return fail(ctx, OBS_ERR_INVALID, "null pointer");
    const auto& h = ctx->head;
    CU(launch_embed(h.embed_w, h.embed_s, h.embed_b, tokens, T, h.vocab, ctx->sh.H, x, ctx->err_flag,
                    as_stream(stream)),
       "embed");
    return OBS_OK;
}

extern "C" int obs_lm_head(obs_ctx* ctx, const uint16_t* x, int T, int32_t* ids, float* logits, void* stream) {
    OBS_CHECK_CTX(ctx);
    if (!ctx->head.mem) return fail(ctx, OBS_ERR_STATE, "head not loaded (obs_load_head)");
    if (T < 0 || T > kHeadMaxT) return fail(ctx, OBS_ERR_INVALID, "T out of range (0..16)");
    if (T == 0) return OBS_OK;
    if (!x || !ids) return fail(ctx, OBS_ERR_INVALID, "null pointer");
    const auto& h = ctx->head;
    cudaStream_t st = as_stream(stream);
    CU(launch_rmsnorm(x, h.norm_w, T, ctx->sh.H, ctx->cfg.rms_eps, h.xn, st), "final norm");
    CU(launch_lm_head(h.lm_w, h.lm_s, h.lm_b, h.xn, T, h.vocab, ctx->sh.H, logits ? logits : h.logits, ids,
                      ctx->num_sms, st),
       "lm_head");
    return OBS_OK;
}

namespace obs {
void rope_table(double theta, int hd, int max_seq, float* out) {
    for (int p = 0; p < max_seq; ++p)
        for (int i = 0; i < hd / 2; ++i) {
            const double ang = (double)p * std::pow(theta, -2.0 * i / hd);
            out[((size_t)p * (hd / 2) + i) * 2] = (float)std::cos(ang);
            out[((size_t)p * (hd / 2) + i) * 2 + 1] = (float)std::sin(ang);
        }
}
}  // namespace obs

extern "C" int obs_attn_init(obs_ctx* ctx, const obs_attn_config* ac) {
    OBS_CHECK_CTX(ctx);
    if (!ac) return fail(ctx, OBS_ERR_INVALID, "null attention config");
    if (!ctx->attn.empty()) return fail(ctx, OBS_ERR_STATE, "attention already initialised");
    const int nq = ac->n_heads, nkv = ac->n_kv_heads, hd = ac->head_dim;
    if (nq <= 0 || nkv <= 0 || nq % nkv || nq / nkv > 8 || hd <= 0 || hd > 128 || hd % 8 || (nq * hd) % 2048 ||
        ac->max_seq <= 0 || ac->max_seq > kAttnMaxSeq || ac->n_seqs <= 0 || !(ac->rope_theta > 0.0f))
        return fail(ctx, OBS_ERR_INVALID,
                    "bad attention config (heads a multiple of kv heads, at most 8 per kv head, head_dim <= 128 "
                    "a multiple of 8, heads*head_dim a multiple of 2048, 0 < max_seq <= 40960, n_seqs > 0, "
                    "rope_theta > 0)");
    CU(cudaSetDevice(ctx->device), "cudaSetDevice");
    ctx->acfg = *ac;
    const int T = ctx->cfg.max_tokens, H = ctx->sh.H, W = (nq + 2 * nkv) * hd;
    const size_t sizes[] = {(size_t)ac->max_seq * hd * 4, (size_t)T * W * 4, (size_t)T * H * 2, (size_t)T * nq * hd * 2,
                            (size_t)T * nq * hd * 2, (size_t)T * H * 4,
                            sdpa_part_floats(T, nq, nkv, hd, ctx->num_sms) * 4};
    size_t total = 0;
    for (size_t sz : sizes) total += align_up(sz, 256);
    CU(cudaMalloc(&ctx->attn_scratch, total), "attention scratch");
    uint8_t* p = ctx->attn_scratch;
    void** ptrs[] = {(void**)&ctx->rope_cs, (void**)&ctx->a_qkv, (void**)&ctx->a_xn, (void**)&ctx->a_q,
                     (void**)&ctx->a_out, (void**)&ctx->a_o, (void**)&ctx->a_part};
    for (int i = 0; i < 7; ++i) *ptrs[i] = p, p += align_up(sizes[i], 256);
    std::vector<float> tab((size_t)ac->max_seq * hd);
    rope_table(ac->rope_theta, hd, ac->max_seq, tab.data());
    CU(cudaMemcpy(ctx->rope_cs, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice), "rope table");
    ctx->attn.resize(ctx->cfg.n_layers);
    return OBS_OK;
}

extern "C" int obs_load_attn(obs_ctx* ctx, int layer, const obs_attn_weights* w, int src_on_device) {
    OBS_CHECK_CTX(ctx);
    if (ctx->attn.empty()) return fail(ctx, OBS_ERR_STATE, "attention not initialised (obs_attn_init)");
    if (layer < 0 || layer >= (int)ctx->attn.size()) return fail(ctx, OBS_ERR_INVALID, "layer out of range");
    if (!w || !w->q_w || !w->q_s || !w->q_b || !w->k_w || !w->k_s || !w->k_b || !w->v_w || !w->v_s || !w->v_b ||
        !w->o_w || !w->o_s || !w->o_b || !w->in_norm || !w->q_norm || !w->k_norm)
        return fail(ctx, OBS_ERR_INVALID, "null attention weight pointer");
    CU(cudaSetDevice(ctx->device), "cudaSetDevice");
    const auto& ac = ctx->acfg;
    const int nq = ac.n_heads, nkv = ac.n_kv_heads, hd = ac.head_dim, H = ctx->sh.H;
    const size_t rq = (size_t)nq * hd, rk = (size_t)nkv * hd;
    auto& L = ctx->attn[layer];
    if (!L.mem) {
        const size_t cache = (size_t)ac.n_seqs * nkv * ac.max_seq * hd * 2;
        const size_t sizes[] = {(rq + 2 * rk) * (H / 8) * 4, (rq + 2 * rk) * (H / 64) * 2, (rq + 2 * rk) * (H / 64) * 2,
                                (size_t)H * (rq / 8) * 4,      (size_t)H * (rq / 64) * 2,    (size_t)H * (rq / 64) * 2,
                                (size_t)H * 2,                  (size_t)hd * 2,               (size_t)hd * 2,
                                cache,                          cache};
        size_t total = 0;
        for (size_t sz : sizes) total += align_up(sz, 256);
        CU(cudaMalloc(&L.mem, total), "attention layer alloc");
        uint8_t* p = L.mem;
        void** ptrs[] = {(void**)&L.qkv_w, (void**)&L.qkv_s, (void**)&L.qkv_b, (void**)&L.o_w,   (void**)&L.o_s,
                         (void**)&L.o_b,   (void**)&L.in_norm, (void**)&L.q_norm, (void**)&L.k_norm, (void**)&L.kc,
                         (void**)&L.vc};
        for (int i = 0; i < 11; ++i) *ptrs[i] = p, p += align_up(sizes[i], 256);
        CU(cudaMemset(L.kc, 0, cache), "cache init");
        CU(cudaMemset(L.vc, 0, cache), "cache init");
    }
    const cudaMemcpyKind kind = src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    const size_t wq = rq * (H / 8) * 4, wk = rk * (H / 8) * 4, gq = rq * (H / 64) * 2, gk = rk * (H / 64) * 2;
    uint8_t* qw = reinterpret_cast<uint8_t*>(L.qkv_w);
    uint8_t* qs = reinterpret_cast<uint8_t*>(L.qkv_s);
    uint8_t* qb = reinterpret_cast<uint8_t*>(L.qkv_b);
    CU(cudaMemcpy(qw, w->q_w, wq, kind), "copy");
    CU(cudaMemcpy(qw + wq, w->k_w, wk, kind), "copy");
    CU(cudaMemcpy(qw + wq + wk, w->v_w, wk, kind), "copy");
    CU(cudaMemcpy(qs, w->q_s, gq, kind), "copy");
    CU(cudaMemcpy(qs + gq, w->k_s, gk, kind), "copy");
    CU(cudaMemcpy(qs + gq + gk, w->v_s, gk, kind), "copy");
    CU(cudaMemcpy(qb, w->q_b, gq, kind), "copy");
    CU(cudaMemcpy(qb + gq, w->k_b, gk, kind), "copy");
    CU(cudaMemcpy(qb + gq + gk, w->v_b, gk, kind), "copy");
    CU(cudaMemcpy(L.o_w, w->o_w, (size_t)H * (rq / 8) * 4, kind), "copy");
    CU(cudaMemcpy(L.o_s, w->o_s, (size_t)H * (rq / 64) * 2, kind), "copy");
    CU(cudaMemcpy(L.o_b, w->o_b, (size_t)H * (rq / 64) * 2, kind), "copy");
    CU(cudaMemcpy(L.in_norm, w->in_norm, (size_t)H * 2, kind), "copy");
    CU(cudaMemcpy(L.q_norm, w->q_norm, (size_t)hd * 2, kind), "copy");
    CU(cudaMemcpy(L.k_norm, w->k_norm, (size_t)hd * 2, kind), "copy");
    L.loaded = true;
    return OBS_OK;
}

extern "C" int obs_attn_forward(obs_ctx* ctx, int layer, const uint16_t* x, uint16_t* out, int T, const int32_t* seq,
                                const int32_t* pos, void* stream) {
    OBS_CHECK_CTX(ctx);
    if (ctx->attn.empty()) return fail(ctx, OBS_ERR_STATE, "attention not initialised (obs_attn_init)");
    if (layer < 0 || layer >= (int)ctx->attn.size()) return fail(ctx, OBS_ERR_INVALID, "layer out of range");
    if (!ctx->attn[layer].loaded) return fail(ctx, OBS_ERR_STATE, "attention layer not loaded");
    if (T < 0 || T > ctx->cfg.max_tokens) return fail(ctx, OBS_ERR_INVALID, "T out of range (0..max_tokens)");
    if (T == 0) return OBS_OK;
    if (!x || !out || !seq || !pos) return fail(ctx, OBS_ERR_INVALID, "null pointer");
    if (out == x) return fail(ctx, OBS_ERR_INVALID, "out may not alias x");
    const auto& ac = ctx->acfg;
    const auto& L = ctx->attn[layer];
    const int nq = ac.n_heads, nkv = ac.n_kv_heads, hd = ac.head_dim, H = ctx->sh.H;
    cudaStream_t st = as_stream(stream);
    CU(launch_rmsnorm(x, L.in_norm, T, H, ctx->cfg.rms_eps, ctx->a_xn, st), "input norm");
    CU(launch_linear4(L.qkv_w, L.qkv_s, L.qkv_b, ctx->a_xn, T, (nq + 2 * nkv) * hd, H, ctx->a_qkv, ctx->num_sms, st),
       "qkv projection");
    CU(launch_qk_norm_rope(ctx->a_qkv, T, nq, nkv, hd, L.q_norm, L.k_norm, ctx->cfg.rms_eps, ctx->rope_cs, ac.max_seq,
                           seq, pos, ctx->a_q, L.kc, L.vc, ac.n_seqs, ctx->err_flag, st),
       "q/k norm, rope, cache append");
    CU(launch_sdpa(ctx->a_q, L.kc, L.vc, T, nq, nkv, hd, ac.max_seq, ac.n_seqs, seq, pos, ctx->a_out, ctx->a_part,
                   ctx->num_sms, st),
       "attention");
    CU(launch_linear4(L.o_w, L.o_s, L.o_b, ctx->a_out, T, H, nq * hd, ctx->a_o, ctx->num_sms, st), "o projection");
    CU(launch_residual_add(x, ctx->a_o, (size_t)T * H, out, st), "residual");
    return OBS_OK;
}

extern "C" int obs_kv_read(obs_ctx* ctx, int layer, int seq, int pos0, int n, uint16_t* k, uint16_t* v,
                           void* stream) {
    OBS_CHECK_CTX(ctx);
    if (ctx->attn.empty() || layer < 0 || layer >= (int)ctx->attn.size() || !ctx->attn[layer].mem)
        return fail(ctx, OBS_ERR_STATE, "no attention layer there");
    const auto& ac = ctx->acfg;
    if (seq < 0 || seq >= ac.n_seqs || pos0 < 0 || n < 0 || pos0 + n > ac.max_seq)
        return fail(ctx, OBS_ERR_INVALID, "cache range out of bounds");
    const auto& L = ctx->attn[layer];
    const int hd = ac.head_dim;
    cudaStream_t st = as_stream(stream);
    for (int h = 0; h < ac.n_kv_heads; ++h) {
        const size_t src = (((size_t)seq * ac.n_kv_heads + h) * ac.max_seq + pos0) * hd;
        if (k) CU(cudaMemcpyAsync(k + (size_t)h * n * hd, L.kc + src, (size_t)n * hd * 2, cudaMemcpyDeviceToDevice, st), "copy");
        if (v) CU(cudaMemcpyAsync(v + (size_t)h * n * hd, L.vc + src, (size_t)n * hd * 2, cudaMemcpyDeviceToDevice, st), "copy");
    }
    return OBS_OK;
}

extern "C" int obs_synth_layer(obs_ctx* ctx, int layer, uint64_t seed) {
    OBS_CHECK_CTX(ctx);
    return load_impl(ctx, layer, nullptr, 1, seed, true);
}

extern "C" int obs_synth_activations(uint64_t seed, uint32_t layer, int row0, int T, int H, float eps,
                                     uint16_t* x, void* stream) {
    if (!x || T < 0 || H <= 0 || row0 < 0) return OBS_ERR_INVALID;
    return launch_synth_x(seed, layer, row0, T, H, eps, x, as_stream(stream)) == cudaSuccess ? OBS_OK
                                                                                              : OBS_ERR_CUDA;
}

// ------------------------------------------------------------------- stages
static int check_T(obs_ctx* ctx, int T) {
    if (T < 0 || T > ctx->cfg.max_tokens) return fail(ctx, OBS_ERR_INVALID, "T out of range (0..max_tokens)");
    return OBS_OK;
}

extern "C" int obs_gate(obs_ctx* ctx, int layer, const uint16_t* x, float* logits, int T, void* stream) {
    OBS_CHECK_CTX(ctx);
    int rc = check_layer(ctx, layer, true);
    if (rc || (rc = check_T(ctx, T))) return rc;
    if (T == 0) return OBS_OK;
    if (!x || !logits) return fail(ctx, OBS_ERR_INVALID, "null pointer");
    cudaStream_t st = as_stream(stream);
    if (router_parts(T) == 1) {
        CU(launch_router_logits(ctx->layers[layer], ctx->sh, x, T, logits, st), "router");
    } else {
        CU(launch_router_logits(ctx->layers[layer], ctx->sh, x, T, ctx->logits, st), "router");
        CU(launch_router_finish(ctx->logits, T, ctx->sh.E, logits, st), "router finish");
    }
    return OBS_OK;
}

extern "C" int obs_route(obs_ctx* ctx, const float* logits, const float* bias, int T, int32_t* ids, float* w,
                         void* stream) {
    OBS_CHECK_CTX(ctx);
    int rc = check_T(ctx, T);
    if (rc) return rc;
    if (T == 0) return OBS_OK;
    if (!logits || !ids || !w) return fail(ctx, OBS_ERR_INVALID, "null pointer");
    CU(launch_topk(logits, 1, bias, T, ctx->sh.E, ctx->sh.K, ctx->cfg.norm_topk, ids, w, nullptr,
                   as_stream(stream)),
       "topk");
    return OBS_OK;
}

// histogram of given routes into ctx->disp.counts, then the dispatch kernel
static int dispatch_from_ids(obs_ctx* ctx, const int32_t* ids, const uint16_t* x, int T, int permute,
                             cudaStream_t st);

extern "C" int obs_dispatch(obs_ctx* ctx, const int32_t* ids, int T, int32_t* counts, int32_t* seg,
                            int32_t* slot_of, void* stream) {
    OBS_CHECK_CTX(ctx);
    if (ctx->ep_world > 1) return fail(ctx, OBS_ERR_UNSUPPORTED, "stage entry points are single-GPU only (ep_world > 1)");
    int rc = check_T(ctx, T);
    if (rc) return rc;
    if (!ids) return fail(ctx, OBS_ERR_INVALID, "null ids");
    cudaStream_t st = as_stream(stream);
    rc = dispatch_from_ids(ctx, ids, nullptr, T, 0, st);
    if (rc) return rc;
    const Shape& s = ctx->sh;
    if (counts) CU(cudaMemcpyAsync(counts, ctx->disp.counts, s.E * 4, cudaMemcpyDeviceToDevice, st), "copy");
    if (seg) CU(cudaMemcpyAsync(seg, ctx->disp.seg, (s.E + 1) * 4, cudaMemcpyDeviceToDevice, st), "copy");
    if (slot_of && T)
        CU(cudaMemcpyAsync(slot_of, ctx->disp.slot_of, (size_t)T * s.K * 4, cudaMemcpyDeviceToDevice, st), "copy");
    return OBS_OK;
}

static int dispatch_from_ids(obs_ctx* ctx, const int32_t* ids, const uint16_t* x, int T, int permute,
                             cudaStream_t st) {
    const Shape& s = ctx->sh;
    if (T) CU(cudaMemsetAsync(ctx->disp.slot_of, 0, (size_t)T * s.K * 4, st), "memset");
    CU(launch_dispatch(ids, x, T, s, ctx->disp, permute, st), "dispatch");
    return OBS_OK;
}

static GemmArgs gemm_gateup(obs_ctx* ctx, const LayerDev& L, const uint16_t* x) {
    const Shape& s = ctx->sh;
    GemmArgs g{};
    g.wblocks = L.gateup;
    g.paired = 1;
    g.act = ctx->disp.xp;  // the routed rows, permuted and tiled by the dispatch
    g.atoms = ctx->disp.atoms;
    g.tiles = ctx->disp.tiles;
    g.n_tiles = ctx->disp.n_tiles;
    g.max_tiles = ctx->max_tiles;
    g.n_rt = s.I / 64;
    g.n_kt = s.H / kGroup;
    g.bn = ctx->disp.bn;
    g.n_experts = ctx->E_local;
    g.out = ctx->hbuf;
    g.out_atoms = ctx->disp.atoms;
    g.row_limit = ctx->R_cap;
    g.err = ctx->err_flag;
    g.trace = ctx->trace;
    g.trace_n = ctx->trace_n;
    g.wait_ns = ctx->wait_ns;
    return g;
}

static GemmArgs gemm_down(obs_ctx* ctx, const LayerDev& L) {
    const Shape& s = ctx->sh;
    GemmArgs g{};
    g.wblocks = L.down;
    g.paired = 0;
    g.act = ctx->hbuf;
    g.atoms = ctx->disp.atoms;
    g.tiles = ctx->disp.tiles;
    g.n_tiles = ctx->disp.n_tiles;
    g.max_tiles = ctx->max_tiles;
    g.n_rt = s.H / kRowTile;
    g.n_kt = s.I / kGroup;
    g.bn = ctx->disp.bn;
    g.n_experts = ctx->E_local;
    g.out = ctx->ybuf;
    g.out_ld = s.H;
    g.row_limit = ctx->R_cap;
    g.err = ctx->err_flag;
    g.wait_ns = ctx->wait_ns;
    return g;
}

// prefill expert FFN over the current dispatch: xp -> hbuf -> ybuf (slot rows)
static int prefill_ffn(obs_ctx* ctx, const LayerDev& L, const uint16_t* x, cudaStream_t st) {
    CU(launch_gemm(gemm_gateup(ctx, L, x), kEpiSwiglu, ctx->num_sms, st), "gemm gate/up");
    CU(launch_gemm(gemm_down(ctx, L), kEpiBf16, ctx->num_sms, st), "gemm down");
    return OBS_OK;
}

extern "C" int obs_debug_gemm_tiles(obs_ctx* ctx, int layer, const int32_t* tiles, int n_tiles, void* stream) {
    OBS_CHECK_CTX(ctx);
    if (ctx->ep_world > 1) return fail(ctx, OBS_ERR_UNSUPPORTED, "single-GPU only (ep_world > 1)");
    int rc = check_layer(ctx, layer, true);
    if (rc) return rc;
    if (!tiles || n_tiles < 0) return fail(ctx, OBS_ERR_INVALID, "bad tile list");
    cudaStream_t st = as_stream(stream);
    const int n_copy = n_tiles < ctx->max_tiles ? n_tiles : ctx->max_tiles;  // the count itself is not clipped
    if (n_copy)
        CU(cudaMemcpyAsync(ctx->disp.tiles, tiles, (size_t)n_copy * 16, cudaMemcpyHostToDevice, st), "copy");
    CU(cudaMemcpyAsync(ctx->disp.n_tiles, &n_tiles, 4, cudaMemcpyHostToDevice, st), "copy");
    CU(cudaStreamSynchronize(st), "sync");  // the host arrays may go away after the call
    CU(launch_gemm(gemm_gateup(ctx, ctx->layers[layer], nullptr), kEpiSwiglu, ctx->num_sms, st), "gemm gate/up");
    return OBS_OK;
}

extern "C" int obs_expert_ffn(obs_ctx* ctx, int layer, const uint16_t* x, const int32_t* ids, int T, int path,
                              uint16_t* y, void* stream) {
    OBS_CHECK_CTX(ctx);
    if (ctx->ep_world > 1) return fail(ctx, OBS_ERR_UNSUPPORTED, "stage entry points are single-GPU only (ep_world > 1)");
    int rc = check_layer(ctx, layer, true);
    if (rc || (rc = check_T(ctx, T))) return rc;
    if (T == 0) return OBS_OK;
    if (!x || !ids || !y) return fail(ctx, OBS_ERR_INVALID, "null pointer");
    const Shape& s = ctx->sh;
    const LayerDev& L = ctx->layers[layer];
    cudaStream_t st = as_stream(stream);
    if (path == OBS_PATH_DECODE) {
        if (T > kDecodeMaxT) return fail(ctx, OBS_ERR_INVALID, "decode path: T above its scratch (64)");
        CU(launch_decode_gateup(L, s, x, ids, T, ctx->dec, st), "decode gate/up");
        CU(launch_decode_down(L, s, ids, nullptr, nullptr, T, ctx->dec, nullptr, 0, st), "decode down");
        CU(cudaMemcpyAsync(y, ctx->dec.y, (size_t)T * s.K * s.H * 2, cudaMemcpyDeviceToDevice, st), "copy");
        return OBS_OK;
    }
    if (path != OBS_PATH_PREFILL) return fail(ctx, OBS_ERR_INVALID, "path must be DECODE or PREFILL");
    rc = dispatch_from_ids(ctx, ids, x, T, 1, st);
    if (rc) return rc;
    rc = prefill_ffn(ctx, L, x, st);
    if (rc) return rc;
    CU(launch_gather_rows(ctx->ybuf, ctx->disp.slot_of, T * s.K, s.H, y, st), "gather");
    return OBS_OK;
}

extern "C" int obs_expert_gemm_f32(obs_ctx* ctx, int layer, int proj, int expert, const uint16_t* x, int n,
                                   float* y, void* stream) {
    OBS_CHECK_CTX(ctx);
    if (ctx->ep_world > 1) return fail(ctx, OBS_ERR_UNSUPPORTED, "stage entry points are single-GPU only (ep_world > 1)");
    int rc = check_layer(ctx, layer, true);
    if (rc) return rc;
    const Shape& s = ctx->sh;
    if (proj < 0 || proj > 2 || expert < 0 || expert >= s.E) return fail(ctx, OBS_ERR_INVALID, "bad proj/expert");
    if (n < 0 || n > ctx->R_cap - kSegAlign) return fail(ctx, OBS_ERR_INVALID, "n out of range");
    if (n == 0) return OBS_OK;
    if (!x || !y) return fail(ctx, OBS_ERR_INVALID, "null pointer");
    cudaStream_t st = as_stream(stream);
    const LayerDev& L = ctx->layers[layer];
    const int in_f = proj == 2 ? s.I : s.H, out_f = proj == 2 ? s.H : s.I;
    const int rows = (n + kSegAlign - 1) / kSegAlign * kSegAlign;
    std::vector<int4> tiles;
    for (int r = 0; r < rows; r += kBNTile) tiles.push_back(make_int4(expert, r, std::min(kBNTile, rows - r), 0));
    int nt = (int)tiles.size();
    CU(cudaMemcpyAsync(ctx->disp.tiles, tiles.data(), tiles.size() * sizeof(int4), cudaMemcpyHostToDevice, st),
       "tiles");
    CU(cudaMemcpyAsync(ctx->disp.n_tiles, &nt, 4, cudaMemcpyHostToDevice, st), "tiles");
    CU(launch_tile_rows(x, n, in_f, ctx->disp.atoms, ctx->disp.xp, st), "tile rows");
    GemmArgs g{};
    g.wblocks = proj == 2 ? L.down : L.gateup;
    g.paired = proj < 2;  // the paired array computes gate and up together; the epilogue keeps one
    g.proj_sel = proj;
    g.act = ctx->disp.xp;
    g.atoms = ctx->disp.atoms;
    g.tiles = ctx->disp.tiles;
    g.n_tiles = ctx->disp.n_tiles;
    g.max_tiles = ctx->max_tiles;
    g.n_rt = proj == 2 ? out_f / kRowTile : out_f / 64;
    g.n_kt = in_f / kGroup;
    g.bn = kBNTile;
    g.n_experts = s.E;
    g.out = y;
    g.out_ld = out_f;
    g.row_limit = n;
    g.err = ctx->err_flag;
    g.wait_ns = ctx->wait_ns;
    CU(launch_gemm(g, kEpiF32, ctx->num_sms, st), "gemm f32");
    CU(cudaStreamSynchronize(st), "sync");  // the host tile list must outlive its copy
    return OBS_OK;
}

// ------------------------------------------------------ expert parallelism
extern "C" int obs_ep_handle(obs_ctx* ctx, void* handle) {
    OBS_CHECK_CTX(ctx);
    if (!handle) return fail(ctx, OBS_ERR_INVALID, "null handle");
    if (ctx->ep_world <= 1) return fail(ctx, OBS_ERR_STATE, "context has no expert parallelism (ep_world <= 1)");
    static_assert(sizeof(cudaIpcMemHandle_t) == OBS_EP_HANDLE_BYTES, "handle size");
    CU(cudaSetDevice(ctx->device), "cudaSetDevice");
    cudaIpcMemHandle_t h;
    CU(cudaIpcGetMemHandle(&h, ctx->ep_buf), "cudaIpcGetMemHandle");
    memcpy(handle, &h, sizeof(h));
    return OBS_OK;
}

extern "C" int obs_ep_connect(obs_ctx* ctx, const void* handles) {
    OBS_CHECK_CTX(ctx);
    if (!handles) return fail(ctx, OBS_ERR_INVALID, "null handles");
    if (ctx->ep_world <= 1) return fail(ctx, OBS_ERR_STATE, "context has no expert parallelism (ep_world <= 1)");
    if (ctx->ep_connected) return fail(ctx, OBS_ERR_STATE, "already connected");
    CU(cudaSetDevice(ctx->device), "cudaSetDevice");
    const cudaIpcMemHandle_t* h = static_cast<const cudaIpcMemHandle_t*>(handles);
    for (int r = 0; r < ctx->ep_world; ++r) {
        if (r == ctx->ep_rank) {
            ctx->ep.peer[r] = ctx->ep_buf;
            continue;
        }
        void* p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h[r], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < r; ++q)
                if (q != ctx->ep_rank && ctx->ep.peer[q]) cudaIpcCloseMemHandle(ctx->ep.peer[q]), ctx->ep.peer[q] = nullptr;
            return cuda_fail(ctx, e, "cudaIpcOpenMemHandle (peer buffer)");
        }
        ctx->ep.peer[r] = static_cast<uint8_t*>(p);
    }
    ctx->ep_connected = true;
    return OBS_OK;
}

extern "C" int obs_ep_set_placement(obs_ctx* ctx, int layer, const int32_t* experts) {
    OBS_CHECK_CTX(ctx);
    if (ctx->ep_world <= 1) return fail(ctx, OBS_ERR_UNSUPPORTED, "placement needs expert parallelism (ep_world > 1)");
    if (!experts) return fail(ctx, OBS_ERR_INVALID, "null placement");
    const int E = ctx->sh.E, n = (int)ctx->layers.size();
    if (layer < -1 || layer >= n) return fail(ctx, OBS_ERR_INVALID, "layer out of range");
    std::vector<int32_t> slot(E, -1);
    for (int i = 0; i < E; ++i) {
        if (experts[i] < 0 || experts[i] >= E || slot[experts[i]] >= 0)
            return fail(ctx, OBS_ERR_INVALID, "placement is not a permutation of the experts");
        slot[experts[i]] = i;
    }
    CU(cudaSetDevice(ctx->device), "cudaSetDevice");
    for (int l = layer < 0 ? 0 : layer; l < (layer < 0 ? n : layer + 1); ++l) {
        if (std::equal(ctx->placement[l].begin(), ctx->placement[l].end(), experts)) continue;
        CU(cudaMemcpy(ctx->place_dev + (size_t)l * E, slot.data(), (size_t)E * 4, cudaMemcpyHostToDevice),
           "placement copy");
        ctx->placement[l].assign(experts, experts + E);
        ctx->layers[l].loaded = false;  // this rank's experts changed: load them again
    }
    return OBS_OK;
}

extern "C" int obs_ep_get_placement(obs_ctx* ctx, int layer, int32_t* experts) {
    OBS_CHECK_CTX(ctx);
    if (!experts) return fail(ctx, OBS_ERR_INVALID, "null placement");
    if (layer < 0 || layer >= (int)ctx->layers.size()) return fail(ctx, OBS_ERR_INVALID, "layer out of range");
    std::copy(ctx->placement[layer].begin(), ctx->placement[layer].end(), experts);
    return OBS_OK;
}

extern "C" int obs_ep_plan_placement(const int64_t* load, int n_experts, int world, int32_t* experts) {
    if (!load || !experts || n_experts <= 0 || world <= 0 || n_experts % world) return OBS_ERR_INVALID;
    for (int i = 0; i < n_experts; ++i)
        if (load[i] < 0) return OBS_ERR_INVALID;
    const int per = n_experts / world;
    std::vector<int> order(n_experts);
    for (int i = 0; i < n_experts; ++i) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return load[a] > load[b]; });
    std::vector<int64_t> total(world, 0);
    std::vector<std::vector<int32_t>> held(world);
    for (int e : order) {
        int best = -1;
        for (int g = 0; g < world; ++g)
            if ((int)held[g].size() < per && (best < 0 || total[g] < total[best])) best = g;
        held[best].push_back(e);
        total[best] += load[e];
    }
    for (int g = 0; g < world; ++g) {
        std::sort(held[g].begin(), held[g].end());
        std::copy(held[g].begin(), held[g].end(), experts + (size_t)g * per);
    }
    return OBS_OK;
}

// One layer with the experts spread over the ranks (layout and protocol in k_ep.cu).
static int forward_ep(obs_ctx* ctx, int layer, const uint16_t* x, uint16_t* out, const uint16_t* residual,
                      int T, const float* logit_bias, cudaStream_t st) {
    if (!ctx->ep_connected) return fail(ctx, OBS_ERR_STATE, "expert parallelism not connected (obs_ep_connect)");
    const Shape& s = ctx->sh;
    const LayerDev& L = ctx->layers[layer];
    EpArgs a = ctx->ep;
    a.place = ctx->place_dev + (size_t)layer * s.E;
    prof_begin(ctx, OBS_STAGE_ROUTER, st);
    if (T > 0) CU(launch_router_logits(L, s, x, T, ctx->logits, st), "router");
    prof_end(ctx, st);
    prof_begin(ctx, OBS_STAGE_TOPK, st);
    if (T > 0)
        CU(launch_topk(ctx->logits, router_parts(T), logit_bias, T, s.E, s.K, ctx->cfg.norm_topk, ctx->ids, ctx->wts,
                       nullptr, st),
           "topk");
    prof_end(ctx, st);
    prof_begin(ctx, OBS_STAGE_EP_SEND, st);
    CU(launch_ep_send(ctx->ids, x, T, s.E, a, st), "ep send");
    prof_end(ctx, st);
    prof_begin(ctx, OBS_STAGE_EP_RECV, st);
    CU(launch_ep_recv(x, a, st), "ep receive");
    prof_end(ctx, st);
    prof_begin(ctx, OBS_STAGE_DISPATCH, st);
    // the received rows as a local routing problem: row j of source s (j < its count) with up to K
    // local experts; the other entries are -1
    const Shape sl{s.H, s.I, ctx->E_local, s.K};
    CU(launch_dispatch(a.ids_local, nullptr, a.world * a.cap_rows, sl, ctx->disp, 1, st, a.row_src, 1), "dispatch");
    CU(launch_ep_rowptr(ctx->disp.slot_of, ctx->disp.src, ctx->disp.seg + ctx->E_local, ctx->ybuf, ctx->ep_row_ptr, a,
                        st),
       "ep row destinations");
    prof_end(ctx, st);
    prof_begin(ctx, OBS_STAGE_GEMM_GATEUP, st);
    CU(launch_gemm(gemm_gateup(ctx, L, x), kEpiSwiglu, ctx->num_sms, st), "gemm gate/up");
    prof_end(ctx, st);
    prof_begin(ctx, OBS_STAGE_GEMM_DOWN, st);
    // the down GEMM's epilogue stores each output row at its destination: the return
    // all-to-all runs inside the GEMM, tile by tile, over NVLink
    GemmArgs gd = gemm_down(ctx, L);
    gd.row_ptr = ctx->ep_row_ptr;
    CU(launch_gemm(gd, kEpiBf16, ctx->num_sms, st), "gemm down");
    prof_end(ctx, st);
    prof_begin(ctx, OBS_STAGE_EP_RETURN, st);
    CU(launch_ep_returned(a, st), "ep returned");
    CU(launch_ep_finish(a, st), "ep finish");
    prof_end(ctx, st);
    prof_begin(ctx, OBS_STAGE_COMBINE, st);
    if (T > 0)
        CU(launch_combine(reinterpret_cast<const uint16_t*>(ctx->ep_buf + a.off_ret), s.H, nullptr, ctx->wts, residual,
                          T, s.H, s.K, out, st, ctx->ybuf, a.local_slot),
           "combine");
    prof_end(ctx, st);
    return OBS_OK;
}

// ------------------------------------------------------------- the layer
extern "C" int obs_moe_forward(obs_ctx* ctx, int layer, const uint16_t* x, uint16_t* out, const uint16_t* residual,
                               int T, const float* logit_bias, int path, void* stream) {
    OBS_CHECK_CTX(ctx);
    int rc = check_layer(ctx, layer, true);
    if (rc || (rc = check_T(ctx, T))) return rc;
    if (ctx->ep_world > 1) {
        // every rank takes part in every forward's exchange, T = 0 included
        if (T > 0 && (!x || !out)) return fail(ctx, OBS_ERR_INVALID, "null pointer");
        if (path != OBS_PATH_AUTO && path != OBS_PATH_DECODE && path != OBS_PATH_PREFILL)
            return fail(ctx, OBS_ERR_INVALID, "bad path");
        return forward_ep(ctx, layer, x, out, residual, T, logit_bias, as_stream(stream));
    }
    if (T == 0) return OBS_OK;
    if (!x || !out) return fail(ctx, OBS_ERR_INVALID, "null pointer");
    if (path == OBS_PATH_AUTO) path = T <= ctx->decode_max ? OBS_PATH_DECODE : OBS_PATH_PREFILL;
    if (path == OBS_PATH_DECODE && T > kDecodeMaxT) return fail(ctx, OBS_ERR_INVALID, "decode path: T > 64");
    if (path != OBS_PATH_DECODE && path != OBS_PATH_PREFILL) return fail(ctx, OBS_ERR_INVALID, "bad path");
    const Shape& s = ctx->sh;
    const LayerDev& L = ctx->layers[layer];
    cudaStream_t st = as_stream(stream);
    if (path == OBS_PATH_DECODE && decode_fused_supported(s, T)) {
        // router, top-k, experts and combine in one cooperative launch
        prof_begin(ctx, OBS_STAGE_DECODE_FUSED, st);
        CU(launch_decode_fused(L, s, x, residual, logit_bias, T, ctx->cfg.norm_topk, 0, 0.0f, ctx->fused, out,
                               ctx->num_sms, st),
           "fused decode");
        prof_end(ctx, st);
        return OBS_OK;
    }
    prof_begin(ctx, OBS_STAGE_ROUTER, st);
    CU(launch_router_logits(L, s, x, T, ctx->logits, st), "router");
    prof_end(ctx, st);
    if (path == OBS_PATH_DECODE) {
        prof_begin(ctx, OBS_STAGE_TOPK, st);
        CU(launch_topk(ctx->logits, router_parts(T), logit_bias, T, s.E, s.K, ctx->cfg.norm_topk, ctx->ids,
                       ctx->wts, nullptr, st),
           "topk");
        prof_end(ctx, st);
        prof_begin(ctx, OBS_STAGE_DECODE_GATEUP, st);
        CU(launch_decode_gateup(L, s, x, ctx->ids, T, ctx->dec, st), "decode gate/up");
        prof_end(ctx, st);
        prof_begin(ctx, OBS_STAGE_DECODE_DOWN, st);
        CU(launch_decode_down(L, s, ctx->ids, ctx->wts, residual, T, ctx->dec, out, 1, st), "decode down");
        prof_end(ctx, st);
        return OBS_OK;
    }
    prof_begin(ctx, OBS_STAGE_TOPK, st);
    CU(launch_topk(ctx->logits, router_parts(T), logit_bias, T, s.E, s.K, ctx->cfg.norm_topk, ctx->ids,
                   ctx->wts, nullptr, st),
       "topk");
    prof_end(ctx, st);
    prof_begin(ctx, OBS_STAGE_DISPATCH, st);
    CU(launch_dispatch(ctx->ids, x, T, s, ctx->disp, 1, st), "dispatch");
    prof_end(ctx, st);
    prof_begin(ctx, OBS_STAGE_GEMM_GATEUP, st);
    CU(launch_gemm(gemm_gateup(ctx, L, x), kEpiSwiglu, ctx->num_sms, st), "gemm gate/up");
    prof_end(ctx, st);
    prof_begin(ctx, OBS_STAGE_GEMM_DOWN, st);
    CU(launch_gemm(gemm_down(ctx, L), kEpiBf16, ctx->num_sms, st), "gemm down");
    prof_end(ctx, st);
    prof_begin(ctx, OBS_STAGE_COMBINE, st);
    CU(launch_combine(ctx->ybuf, s.H, ctx->disp.slot_of, ctx->wts, residual, T, s.H, s.K, out, st), "combine");
    prof_end(ctx, st);
    return OBS_OK;
}

extern "C" int obs_rmsnorm(obs_ctx* ctx, const uint16_t* x, const uint16_t* weight, int T, uint16_t* out,
                           void* stream) {
    OBS_CHECK_CTX(ctx);
    int rc = check_T(ctx, T);
    if (rc) return rc;
    if (T == 0) return OBS_OK;
    if (!x || !out) return fail(ctx, OBS_ERR_INVALID, "null pointer");
    if (x == out) return fail(ctx, OBS_ERR_INVALID, "out may not alias x");
    CU(launch_rmsnorm(x, weight, T, ctx->sh.H, ctx->cfg.rms_eps, out, as_stream(stream)), "rmsnorm");
    return OBS_OK;
}

extern "C" int obs_moe_stack_forward(obs_ctx* ctx, int layer0, int n_layers, uint16_t* resid, int T,
                                     const float* logit_bias, int path, void* stream) {
    OBS_CHECK_CTX(ctx);
    if (n_layers < 0 || layer0 < 0 || layer0 + n_layers > (int)ctx->layers.size())
        return fail(ctx, OBS_ERR_INVALID, "layer range out of the context's layers");
    int rc = check_T(ctx, T);
    if (rc) return rc;
    if (T > 0 && !resid) return fail(ctx, OBS_ERR_INVALID, "null pointer");
    if (T == 0 && ctx->ep_world <= 1) return OBS_OK;
    cudaStream_t st = as_stream(stream);
    uint16_t* r = resid;
    uint16_t* other = ctx->rtmp_dev;
    const int eff = path == OBS_PATH_AUTO ? (T <= ctx->decode_max ? OBS_PATH_DECODE : OBS_PATH_PREFILL) : path;
    const bool fused = ctx->ep_world <= 1 && eff == OBS_PATH_DECODE && decode_fused_supported(ctx->sh, T);
    for (int l = layer0; l < layer0 + n_layers; ++l) {
        if (fused) {
            // RMSNorm, router, top-k, experts and the residual combine of the layer in one launch
            rc = check_layer(ctx, l, true);
            if (rc) return rc;
            prof_begin(ctx, OBS_STAGE_DECODE_FUSED, st);
            CU(launch_decode_fused(ctx->layers[l], ctx->sh, r, r, logit_bias, T, ctx->cfg.norm_topk, 1,
                                   ctx->cfg.rms_eps, ctx->fused, other, ctx->num_sms, st),
               "fused decode");
            prof_end(ctx, st);
        } else {
            if (T > 0) CU(launch_rmsnorm(r, nullptr, T, ctx->sh.H, ctx->cfg.rms_eps, ctx->xnorm_dev, st), "rmsnorm");
            rc = obs_moe_forward(ctx, l, ctx->xnorm_dev, other, r, T, logit_bias, path, stream);
            if (rc) return rc;
        }
        std::swap(r, other);
    }
    if (r != resid && T > 0)
        CU(cudaMemcpyAsync(resid, r, (size_t)T * ctx->sh.H * 2, cudaMemcpyDeviceToDevice, st), "copy");
    return OBS_OK;
}

extern "C" int obs_moe_forward_host(obs_ctx* ctx, int layer, const uint16_t* x_host, uint16_t* out_host,
                                    const uint16_t* residual_host, int T, const float* bias_host, int path,
                                    void* stream) {
    OBS_CHECK_CTX(ctx);
    int rc = check_T(ctx, T);
    if (rc) return rc;
    if (T == 0) return OBS_OK;
    if (!x_host || !out_host) return fail(ctx, OBS_ERR_INVALID, "null pointer");
    const Shape& s = ctx->sh;
    cudaStream_t st = as_stream(stream);
    const size_t bytes = (size_t)T * s.H * 2;
    CU(cudaMemcpyAsync(ctx->x_dev, x_host, bytes, cudaMemcpyHostToDevice, st), "h2d x");
    if (residual_host) CU(cudaMemcpyAsync(ctx->res_dev, residual_host, bytes, cudaMemcpyHostToDevice, st), "h2d");
    if (bias_host) CU(cudaMemcpyAsync(ctx->bias_dev, bias_host, s.E * 4, cudaMemcpyHostToDevice, st), "h2d");
    rc = obs_moe_forward(ctx, layer, ctx->x_dev, ctx->out_dev, residual_host ? ctx->res_dev : nullptr, T,
                         bias_host ? ctx->bias_dev : nullptr, path, stream);
    if (rc) return rc;
    CU(cudaMemcpyAsync(out_host, ctx->out_dev, bytes, cudaMemcpyDeviceToHost, st), "d2h out");
    CU(cudaStreamSynchronize(st), "sync");
    return OBS_OK;
}

extern "C" int obs_moe_forward_host_async(obs_ctx* ctx, int layer, const uint16_t* x_host, uint16_t* out_host,
                                          const uint16_t* residual_host, int T, const float* bias_host, int path,
                                          void* stream) {
    OBS_CHECK_CTX(ctx);
    int rc = check_T(ctx, T);
    if (rc) return rc;
    if (T == 0) return OBS_OK;
    if (!x_host || !out_host) return fail(ctx, OBS_ERR_INVALID, "null pointer");
    if (ctx->ep_world > 1) return fail(ctx, OBS_ERR_UNSUPPORTED, "the asynchronous host entry is single-GPU only");
    CU(cudaSetDevice(ctx->device), "cudaSetDevice");
    if (!ctx->hs_ready) {
        CU(cudaStreamCreateWithFlags(&ctx->hs_in, cudaStreamNonBlocking), "copy stream");
        CU(cudaStreamCreateWithFlags(&ctx->hs_out, cudaStreamNonBlocking), "copy stream");
        for (auto& h : ctx->hs) {
            CU(cudaEventCreateWithFlags(&h.in_done, cudaEventDisableTiming), "event");
            CU(cudaEventCreateWithFlags(&h.computed, cudaEventDisableTiming), "event");
            CU(cudaEventCreateWithFlags(&h.out_done, cudaEventDisableTiming), "event");
        }
        ctx->hs_ready = true;
    }
    const Shape& s = ctx->sh;
    cudaStream_t st = as_stream(stream);
    auto& h = ctx->hs[ctx->hs_next];
    const size_t bytes = (size_t)T * s.H * 2;
    // input: after this slot's previous forward has read its staging buffers
    if (h.used) CU(cudaStreamWaitEvent(ctx->hs_in, h.computed, 0), "wait");
    CU(cudaMemcpyAsync(h.x, x_host, bytes, cudaMemcpyHostToDevice, ctx->hs_in), "h2d x");
    if (residual_host) CU(cudaMemcpyAsync(h.res, residual_host, bytes, cudaMemcpyHostToDevice, ctx->hs_in), "h2d");
    if (bias_host) CU(cudaMemcpyAsync(h.bias, bias_host, s.E * 4, cudaMemcpyHostToDevice, ctx->hs_in), "h2d");
    CU(cudaEventRecord(h.in_done, ctx->hs_in), "record");
    // forward on the caller's stream: after the input landed and the slot's previous result left
    CU(cudaStreamWaitEvent(st, h.in_done, 0), "wait");
    if (h.used) CU(cudaStreamWaitEvent(st, h.out_done, 0), "wait");
    rc = obs_moe_forward(ctx, layer, h.x, h.out, residual_host ? h.res : nullptr, T, bias_host ? h.bias : nullptr,
                         path, stream);
    if (rc) return rc;
    CU(cudaEventRecord(h.computed, st), "record");
    // output: after the forward
    CU(cudaStreamWaitEvent(ctx->hs_out, h.computed, 0), "wait");
    CU(cudaMemcpyAsync(out_host, h.out, bytes, cudaMemcpyDeviceToHost, ctx->hs_out), "d2h out");
    CU(cudaEventRecord(h.out_done, ctx->hs_out), "record");
    h.used = true;
    ctx->hs_next ^= 1;
    return OBS_OK;
}

extern "C" int obs_moe_host_join(obs_ctx* ctx, void* stream) {
    OBS_CHECK_CTX(ctx);
    if (!ctx->hs_ready) return OBS_OK;
    CU(cudaSetDevice(ctx->device), "cudaSetDevice");
    cudaStream_t st = as_stream(stream);
    for (auto& h : ctx->hs)
        if (h.used) CU(cudaStreamWaitEvent(st, h.out_done, 0), "wait");
    return OBS_OK;
}

extern "C" int obs_check_device(obs_ctx* ctx, void* stream) {
    OBS_CHECK_CTX(ctx);
    CU(cudaStreamSynchronize(as_stream(stream)), "stream sync");
    CU(cudaGetLastError(), "pending error");
    int words[4] = {0, 0, 0, 0};
    CU(cudaMemcpy(words, ctx->err_flag, 16, cudaMemcpyDeviceToHost), "read flag");
    const int flag = words[0];
    if (flag) {
        CU(cudaMemset(ctx->err_flag, 0, 16), "clear flag");
        // a wait that gave up leaves the fused decode layer's barrier counts behind: start over
        CU(cudaMemset(ctx->fused.bar, 0, 8), "reset tickets");
        CU(cudaMemset(ctx->fused.ypart, 0, (size_t)kFusedMaxT * ctx->sh.K * (ctx->sh.I / kGroup) * ctx->sh.H * 8), "reset");
        CU(cudaMemset(ctx->fused.lst, 0, (size_t)4 * kFusedMaxT * ctx->sh.E * 8), "reset");
        if (flag == kDevTimeout) {
            char msg[96];
            snprintf(msg, sizeof msg, "a device-side wait gave up (timeout; GEMM wait code %d)", words[1]);
            return fail(ctx, OBS_ERR_TIMEOUT, msg);
        }
        if (flag == kDevBadTile) return fail(ctx, OBS_ERR_INVALID, "device refused a GEMM tile outside its buffers");
        if (flag == kDevBadSlot) {
            static const char* const site[] = {"?", "source region full", "received pair without a slot",
                                               "received pair with a bad item", "dispatch beyond the row buffers",
                                               "permute row without data", "down-GEMM row without a destination"};
            char msg[192];
            snprintf(msg, sizeof msg, "device refused an expert-parallel row slot outside its buffers (first: %s; %d)",
                     site[words[2] >= 0 && words[2] <= 6 ? words[2] : 0], words[3]);
            return fail(ctx, OBS_ERR_INVALID, msg);
        }
        if (flag == kDevBadPos)
            return fail(ctx, OBS_ERR_INVALID, "device refused a token's sequence or position outside the KV caches");
        return fail(ctx, OBS_ERR_INVALID, "device reported an invalid route (expert id out of range)");
    }
    return OBS_OK;
}

extern "C" int obs_set_wait_limit(obs_ctx* ctx, uint64_t limit_ns) {
    OBS_CHECK_CTX(ctx);
    if (limit_ns == 0) limit_ns = kDefaultWaitNs;
    if (limit_ns < 1000000ull || limit_ns > 60000000000ull)
        return fail(ctx, OBS_ERR_INVALID, "wait limit must lie in [1 ms, 60 s] (0: the default 2 s)");
    ctx->wait_ns = limit_ns;
    ctx->fused.wait_ns = limit_ns;
    ctx->ep.wait_ns = limit_ns;
    return OBS_OK;
}

extern "C" int obs_probe_wait(obs_ctx* ctx, void* stream) {
    OBS_CHECK_CTX(ctx);
    CU(cudaSetDevice(ctx->device), "cudaSetDevice");
    CU(launch_probe_wait(ctx->probe_stamp, ctx->wait_ns, ctx->err_flag, as_stream(stream)), "probe wait");
    return OBS_OK;
}

extern "C" int obs_struct_layout(int32_t* out, int n) {
    if (!out && n) return OBS_ERR_INVALID;
#define OBS_OFF(T, f) (int32_t) offsetof(T, f)
    const int32_t v[] = {
        (int32_t)sizeof(obs_config),
        OBS_OFF(obs_config, hidden), OBS_OFF(obs_config, inter), OBS_OFF(obs_config, n_experts),
        OBS_OFF(obs_config, top_k), OBS_OFF(obs_config, group_size), OBS_OFF(obs_config, n_layers),
        OBS_OFF(obs_config, max_tokens), OBS_OFF(obs_config, norm_topk), OBS_OFF(obs_config, decode_max_tokens),
        OBS_OFF(obs_config, rms_eps), OBS_OFF(obs_config, ep_world), OBS_OFF(obs_config, ep_rank),
        (int32_t)sizeof(obs_layer_weights),
        OBS_OFF(obs_layer_weights, router_w), OBS_OFF(obs_layer_weights, router_s), OBS_OFF(obs_layer_weights, router_b),
        OBS_OFF(obs_layer_weights, gate_w), OBS_OFF(obs_layer_weights, gate_s), OBS_OFF(obs_layer_weights, gate_b),
        OBS_OFF(obs_layer_weights, up_w), OBS_OFF(obs_layer_weights, up_s), OBS_OFF(obs_layer_weights, up_b),
        OBS_OFF(obs_layer_weights, down_w), OBS_OFF(obs_layer_weights, down_s), OBS_OFF(obs_layer_weights, down_b),
        (int32_t)sizeof(obs_head_weights),
        OBS_OFF(obs_head_weights, embed_w), OBS_OFF(obs_head_weights, embed_s), OBS_OFF(obs_head_weights, embed_b),
        OBS_OFF(obs_head_weights, lm_w), OBS_OFF(obs_head_weights, lm_s), OBS_OFF(obs_head_weights, lm_b),
        OBS_OFF(obs_head_weights, norm_w),
        (int32_t)sizeof(obs_attn_weights),
        OBS_OFF(obs_attn_weights, q_w), OBS_OFF(obs_attn_weights, q_s), OBS_OFF(obs_attn_weights, q_b),
        OBS_OFF(obs_attn_weights, k_w), OBS_OFF(obs_attn_weights, k_s), OBS_OFF(obs_attn_weights, k_b),
        OBS_OFF(obs_attn_weights, v_w), OBS_OFF(obs_attn_weights, v_s), OBS_OFF(obs_attn_weights, v_b),
        OBS_OFF(obs_attn_weights, o_w), OBS_OFF(obs_attn_weights, o_s), OBS_OFF(obs_attn_weights, o_b),
        OBS_OFF(obs_attn_weights, in_norm), OBS_OFF(obs_attn_weights, q_norm), OBS_OFF(obs_attn_weights, k_norm),
        (int32_t)sizeof(obs_attn_config),
        OBS_OFF(obs_attn_config, n_heads), OBS_OFF(obs_attn_config, n_kv_heads), OBS_OFF(obs_attn_config, head_dim),
        OBS_OFF(obs_attn_config, max_seq), OBS_OFF(obs_attn_config, n_seqs), OBS_OFF(obs_attn_config, rope_theta),
    };
#undef OBS_OFF
    const int total = (int)(sizeof(v) / sizeof(v[0]));
    for (int i = 0; i < n && i < total; ++i) out[i] = v[i];
    return total;
}

extern "C" int obs_profile_enable(obs_ctx* ctx, int enable) {
    OBS_CHECK_CTX(ctx);
    ctx->prof = enable != 0;
    ctx->ev_marks.clear();
    return OBS_OK;
}

extern "C" int obs_profile_read(obs_ctx* ctx, float* ms_total, int32_t* launches) {
    OBS_CHECK_CTX(ctx);
    if (!ms_total || !launches) return fail(ctx, OBS_ERR_INVALID, "null pointer");
    for (int i = 0; i < OBS_N_STAGES; ++i) ms_total[i] = 0.0f, launches[i] = 0;
    for (auto& m : ctx->ev_marks) {
        CU(cudaEventSynchronize(ctx->ev_pool[m.second + 1]), "event sync");
        float ms = 0.0f;
        CU(cudaEventElapsedTime(&ms, ctx->ev_pool[m.second], ctx->ev_pool[m.second + 1]), "event time");
        ms_total[m.first] += ms;
        launches[m.first] += 1;
    }
    ctx->ev_marks.clear();
    return OBS_OK;
}

namespace obs {
static std::atomic<uint64_t> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
bool pdl_enabled() {
    static const bool on = [] {
        const char* v = getenv("OBS_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}
}  // namespace obs

extern "C" int obs_kernel_launches(uint64_t* count) {
    if (!count) return OBS_ERR_INVALID;
    *count = obs::g_launches.load(std::memory_order_relaxed);
    return OBS_OK;
}

extern "C" int obs_trace_enable(obs_ctx* ctx, uint64_t* trace, int n_steps) {
    OBS_CHECK_CTX(ctx);
    if (trace && n_steps <= 0) return fail(ctx, OBS_ERR_INVALID, "n_steps must be positive");
    ctx->trace = trace;
    ctx->trace_n = trace ? n_steps : 0;
    // the fused decode layer records the phase timeline of every CTA when the buffer holds it
    ctx->fused.trace = trace && (size_t)n_steps * kTrRoles >= (size_t)24 * ctx->num_sms ? trace : nullptr;
    return OBS_OK;
}
