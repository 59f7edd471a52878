// ref_driver.cpp -- CPU launcher for the reference's own Metal kernels.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles the reference's
// shaders/*.metal files, where they lie, as C++ (through the metal_stdlib
// stand-in in this folder) and links them with this launcher into
// oracle/_ref/libobs_refshaders.so.  The launcher runs each kernel over its
// grid on host threads, and strings them together the way the reference's
// host code does (src/forward.rs, src/router.rs), so the repository's C oracle
// can be pinned against the reference's literal f16 arithmetic.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

typedef _Float16 half;

struct DqParams { unsigned in_features, out_features, group_size; };          // forward.rs:22
struct MmParams { unsigned in_features, out_features, group_size, n_tokens; }; // forward.rs:23
struct RtParams { unsigned n_experts, top_k, norm_topk; };                     // router.rs:8-14
struct NParams { unsigned n; };
struct ScaledNParams { unsigned n; float scale; };
struct RmsParams { unsigned dim; float eps; };                               // rmsnorm.metal:7
struct RopeParams { unsigned n_heads, head_dim, pos; float theta; };         // rope.metal:8
struct KvParams { unsigned n_kv, head_dim, max_len, pos; };                  // ops.metal:9
struct SdpaParams { unsigned n_heads, n_kv, head_dim, seq_len, kv_stride; float scale; };  // sdpa_decode.metal:12

extern "C" {
void dequant_matvec_8bit(const unsigned char*, const half*, const half*, const half*, half*,
                         const DqParams&, unsigned);
void fused_dequant_matvec_4bit(const unsigned char*, const half*, const half*, const half*, half*,
                               const DqParams&, unsigned);
void matmul_dequant_4bit(const unsigned char*, const half*, const half*, const half*, half*,
                         const MmParams&, unsigned);
void moe_routing_topk(const half*, int*, half*, const RtParams&, unsigned);
void ew_swiglu(const half*, const half*, half*, const NParams&, unsigned);
void ew_scaled_add(half*, const half*, const ScaledNParams&, unsigned);
void rmsnorm(const half*, const half*, half*, const RmsParams&, unsigned, unsigned);
void ew_add(const half*, const half*, half*, const NParams&, unsigned);
void kv_append(const half*, half*, const KvParams&, unsigned);
void rope_apply(half*, const RopeParams&, unsigned);
void sdpa_decode(const half*, const half*, const half*, half*, float*, const SdpaParams&, unsigned, unsigned);
}

template <class F>
static void parallel_for(long n, int nthreads, F f) {
    if (nthreads <= 1 || n < 2) {
        for (long i = 0; i < n; ++i) f(i);
        return;
    }
    nthreads = (int)std::min<long>(nthreads, n);
    std::vector<std::thread> th;
    long chunk = (n + nthreads - 1) / nthreads;
    for (int t = 0; t < nthreads; ++t) {
        long lo = t * chunk, hi = std::min(n, lo + chunk);
        if (lo >= hi) break;
        th.emplace_back([=] { for (long i = lo; i < hi; ++i) f(i); });
    }
    for (auto& x : th) x.join();
}

static inline float bf2f(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
// weight_loader.rs:49-58: bf16 -> f32 -> f16 (round to nearest even)
static std::vector<half> to_f16(const uint16_t* p, size_t n) {
    std::vector<half> v(n);
    for (size_t i = 0; i < n; ++i) v[i] = (half)bf2f(p[i]);
    return v;
}

extern "C" {

// ---- single kernels, f16 in/out, one "thread" per grid position ----
void ref_dequant_matvec_8bit(const uint32_t* w, const half* s, const half* b, const half* x,
                             half* out, int in_f, int out_f) {
    DqParams p{(unsigned)in_f, (unsigned)out_f, 64};
    for (int t = 0; t < out_f; ++t) dequant_matvec_8bit((const unsigned char*)w, s, b, x, out, p, t);
}

void ref_fused_dequant_matvec_4bit(const uint32_t* w, const half* s, const half* b, const half* x,
                                   half* out, int in_f, int out_f, int nthreads) {
    DqParams p{(unsigned)in_f, (unsigned)out_f, 64};
    parallel_for(out_f, nthreads, [&](long t) {
        fused_dequant_matvec_4bit((const unsigned char*)w, s, b, x, out, p, (unsigned)t);
    });
}

void ref_matmul_dequant_4bit(const uint32_t* w, const half* s, const half* b, const half* x,
                             half* out, int n_tokens, int in_f, int out_f, int nthreads) {
    MmParams p{(unsigned)in_f, (unsigned)out_f, 64, (unsigned)n_tokens};
    parallel_for((long)n_tokens * out_f, nthreads, [&](long t) {
        matmul_dequant_4bit((const unsigned char*)w, s, b, x, out, p, (unsigned)t);
    });
}

// rmsnorm.metal: one threadgroup of 256 per row.  Its phases (partial sums, a
// halving tree, the output loop) are separated by barriers, which the stand-in
// header makes no-ops.  Running the 256 "threads" from 255 down to 0 lets every
// tree step read a partner that has finished all of its own steps; a second
// such pass then gives every thread the final sq[0] (thread 0 rewrites it last,
// with the same value).
void ref_rmsnorm(const half* x, const half* w, half* out, int rows, int dim, float eps) {
    RmsParams p{(unsigned)dim, eps};
    for (int r = 0; r < rows; ++r)
        for (int pass = 0; pass < 2; ++pass)
            for (int t = 255; t >= 0; --t) rmsnorm(x, w, out, p, (unsigned)r, (unsigned)t);
}

// router.rs:25-56: one threadgroup of 256; the serial section runs on thread 0
// after every thread stored its logit, so thread 0 goes last here.
void ref_moe_routing_topk(const half* logits, int n_experts, int top_k, int norm,
                          int* ids, half* weights) {
    RtParams p{(unsigned)n_experts, (unsigned)top_k, (unsigned)norm};
    for (unsigned t = 1; t < 256; ++t) moe_routing_topk(logits, ids, weights, p, t);
    moe_routing_topk(logits, ids, weights, p, 0);
}

// rope.metal: one "thread" per (head, pair), in place on [n_heads, head_dim]
void ref_rope(half* x, int n_heads, int head_dim, int pos, float theta) {
    RopeParams p{(unsigned)n_heads, (unsigned)head_dim, (unsigned)pos, theta};
    for (unsigned t = 0; t < (unsigned)(n_heads * head_dim / 2); ++t) rope_apply(x, p, t);
}

// sdpa_decode.metal: one threadgroup of 256 per head; the scores of every
// "thread" are in the scratch before thread 0's serial softmax, so thread 0
// runs last.  scratch: n_heads * kv_stride floats.
void ref_sdpa(const half* q, const half* k, const half* v, half* out, float* scratch, int n_heads, int n_kv,
              int head_dim, int seq_len, int kv_stride, float scale) {
    SdpaParams p{(unsigned)n_heads, (unsigned)n_kv, (unsigned)head_dim, (unsigned)seq_len, (unsigned)kv_stride,
                 scale};
    for (unsigned h = 0; h < (unsigned)n_heads; ++h) {
        for (unsigned t = 1; t < 256; ++t) sdpa_decode(q, k, v, out, scratch, p, h, t);
        sdpa_decode(q, k, v, out, scratch, p, h, 0);
    }
}

void ref_ew_swiglu(const half* g, const half* u, half* out, int n) {
    NParams p{(unsigned)n};
    for (int t = 0; t < n; ++t) ew_swiglu(g, u, out, p, (unsigned)t);
}

void ref_ew_scaled_add(half* acc, const half* y, float scale, int n) {
    ScaledNParams p{(unsigned)n, scale};
    for (int t = 0; t < n; ++t) ew_scaled_add(acc, y, p, (unsigned)t);
}

// ---- the reference's batched-prefill MoE section (forward.rs:164-232) ----
// Inputs in the repository's bf16 host format; converted to f16 on entry the
// way the reference's loaders do.  out [T,H] f16 = x1 after the rank-order
// scaled adds, x1 starting from `residual` (or zeros).  ids/weights per token.
// logit_bias (fp32 [E], may be NULL) is added to the f16 logits the router
// mat-vec wrote before its top-k kernel runs: the skewed-load configuration of
// the benchmark, which the reference's router has no input for.
struct RefLayer {
    int E, H, I, K;
    const uint32_t *router_w, *gate_w, *up_w, *down_w;
    const uint16_t *router_s, *router_b, *gate_s, *gate_b, *up_s, *up_b, *down_s, *down_b;
};

int ref_moe_prefill(const RefLayer* L, const uint16_t* x_bf16, const uint16_t* residual_bf16,
                    const float* logit_bias, int T, int nthreads, half* out, int* ids_out, float* w_out) {
    const int E = L->E, H = L->H, I = L->I, K = L->K, G = H / 64, GI = I / 64;
    std::vector<half> x = to_f16(x_bf16, (size_t)T * H);
    std::vector<half> rs = to_f16(L->router_s, (size_t)E * G), rb = to_f16(L->router_b, (size_t)E * G);
    // per-token gate + route (forward.rs:165-172; router.rs:62-94)
    std::vector<int> ids((size_t)T * K);
    std::vector<float> wts((size_t)T * K);
    parallel_for(T, nthreads, [&](long t) {
        std::vector<half> logits(E), w(K);
        ref_dequant_matvec_8bit(L->router_w, rs.data(), rb.data(), x.data() + (size_t)t * H,
                                logits.data(), H, E);
        if (logit_bias)
            for (int e = 0; e < E; ++e) logits[e] = (half)((float)logits[e] + logit_bias[e]);
        ref_moe_routing_topk(logits.data(), E, K, 1, ids.data() + (size_t)t * K, w.data());
        for (int k = 0; k < K; ++k) wts[(size_t)t * K + k] = (float)w[k];  // router.rs:91-92
    });
    // grouping per expert in token order (forward.rs:203-216)
    std::vector<std::vector<int>> toks(E);
    for (int t = 0; t < T; ++t)
        for (int k = 0; k < K; ++k) toks[ids[(size_t)t * K + k]].push_back(t);
    std::vector<std::vector<half>> ye(E);
    // experts run one at a time, each kernel spread over the host threads
    for (int e = 0; e < E; ++e) {
        int n = (int)toks[e].size();
        if (!n) continue;
        std::vector<half> xe((size_t)n * H);
        for (int r = 0; r < n; ++r)
            std::memcpy(&xe[(size_t)r * H], &x[(size_t)toks[e][r] * H], sizeof(half) * H);
        size_t gw = (size_t)e * I * (H / 8), gs = (size_t)e * I * G;
        size_t dw = (size_t)e * H * (I / 8), ds = (size_t)e * H * GI;
        std::vector<half> gsv = to_f16(L->gate_s + gs, (size_t)I * G), gbv = to_f16(L->gate_b + gs, (size_t)I * G);
        std::vector<half> usv = to_f16(L->up_s + gs, (size_t)I * G), ubv = to_f16(L->up_b + gs, (size_t)I * G);
        std::vector<half> dsv = to_f16(L->down_s + ds, (size_t)H * GI), dbv = to_f16(L->down_b + ds, (size_t)H * GI);
        std::vector<half> g((size_t)n * I), u((size_t)n * I), h((size_t)n * I);
        ye[e].resize((size_t)n * H);
        ref_matmul_dequant_4bit(L->gate_w + gw, gsv.data(), gbv.data(), xe.data(), g.data(), n, H, I, nthreads);
        ref_matmul_dequant_4bit(L->up_w + gw, usv.data(), ubv.data(), xe.data(), u.data(), n, H, I, nthreads);
        ref_ew_swiglu(g.data(), u.data(), h.data(), n * I);
        ref_matmul_dequant_4bit(L->down_w + dw, dsv.data(), dbv.data(), h.data(), ye[e].data(), n, I, H, nthreads);
    }
    // scatter in per-token rank order (forward.rs:225-232)
    std::vector<int> fill(E, 0);
    std::vector<int> row_of((size_t)T * K);
    for (int t = 0; t < T; ++t)
        for (int k = 0; k < K; ++k) {
            int e = ids[(size_t)t * K + k];
            row_of[(size_t)t * K + k] = fill[e]++;
        }
    parallel_for(T, nthreads, [&](long t) {
        half* acc = out + (size_t)t * H;
        for (int i = 0; i < H; ++i) acc[i] = residual_bf16 ? (half)bf2f(residual_bf16[(size_t)t * H + i]) : (half)0.0f;
        for (int k = 0; k < K; ++k) {
            int e = ids[(size_t)t * K + k];
            ref_ew_scaled_add(acc, ye[e].data() + (size_t)row_of[(size_t)t * K + k] * H,
                              wts[(size_t)t * K + k], H);
        }
    });
    if (ids_out) std::memcpy(ids_out, ids.data(), sizeof(int) * ids.size());
    if (w_out) std::memcpy(w_out, wts.data(), sizeof(float) * wts.size());
    return 0;
}

// ---- the reference's attention block for one decode token (forward.rs:404-419) ----
// Model::forward_layer up to the residual: RMSNorm(input_layernorm) -> q/k/v
// fused 4-bit mat-vecs -> per-head RMSNorm (q_norm, k_norm) -> RoPE at pos ->
// kv_append of k and v -> sdpa_decode over seq_len = pos + 1 positions with
// scale = head_dim^-0.5 (attention.rs:27-29) -> o_proj -> ew_add(x, o).
// Weights in the repository's bf16 host format, converted to f16 as the
// loader does; kc/vc are the layer's f16 caches [n_kv][max_len][head_dim],
// updated in place; out f16 [H].
struct RefAttn {
    int H, nq, nkv, hd, max_len;
    float theta, eps;
    const uint32_t *q_w, *k_w, *v_w, *o_w;
    const uint16_t *q_s, *q_b, *k_s, *k_b, *v_s, *v_b, *o_s, *o_b;
    const uint16_t *in_norm, *q_norm, *k_norm;
};

int ref_attn_token(const RefAttn* A, half* kc, half* vc, int pos, const uint16_t* x_bf16, int nthreads, half* out) {
    const int H = A->H, nq = A->nq, nkv = A->nkv, hd = A->hd, rq = nq * hd, rk = nkv * hd;
    if (pos < 0 || pos >= A->max_len) return -1;
    std::vector<half> x = to_f16(x_bf16, H), in_norm = to_f16(A->in_norm, H), qn = to_f16(A->q_norm, hd),
                      kn = to_f16(A->k_norm, hd);
    std::vector<half> xn(H), q(rq), k(rk), v(rk), qh(rq), kh(rk), att(rq), o(H);
    ref_rmsnorm(x.data(), in_norm.data(), xn.data(), 1, H, A->eps);
    struct { const uint32_t* w; const uint16_t *s, *b; half* y; int n; } proj[3] = {
        {A->q_w, A->q_s, A->q_b, q.data(), rq}, {A->k_w, A->k_s, A->k_b, k.data(), rk},
        {A->v_w, A->v_s, A->v_b, v.data(), rk}};
    for (auto& pj : proj) {
        std::vector<half> sv = to_f16(pj.s, (size_t)pj.n * (H / 64)), bv = to_f16(pj.b, (size_t)pj.n * (H / 64));
        ref_fused_dequant_matvec_4bit(pj.w, sv.data(), bv.data(), xn.data(), pj.y, H, pj.n, nthreads);
    }
    ref_rmsnorm(q.data(), qn.data(), qh.data(), nq, hd, A->eps);
    ref_rmsnorm(k.data(), kn.data(), kh.data(), nkv, hd, A->eps);
    ref_rope(qh.data(), nq, hd, pos, A->theta);
    ref_rope(kh.data(), nkv, hd, pos, A->theta);
    KvParams kp{(unsigned)nkv, (unsigned)hd, (unsigned)A->max_len, (unsigned)pos};
    for (unsigned t = 0; t < (unsigned)rk; ++t) kv_append(kh.data(), kc, kp, t);
    for (unsigned t = 0; t < (unsigned)rk; ++t) kv_append(v.data(), vc, kp, t);
    std::vector<float> scratch((size_t)nq * A->max_len);
    ref_sdpa(qh.data(), kc, vc, att.data(), scratch.data(), nq, nkv, hd, pos + 1, A->max_len,
             std::pow((float)hd, -0.5f));
    std::vector<half> os = to_f16(A->o_s, (size_t)H * (rq / 64)), ob = to_f16(A->o_b, (size_t)H * (rq / 64));
    ref_fused_dequant_matvec_4bit(A->o_w, os.data(), ob.data(), att.data(), o.data(), rq, H, nthreads);
    NParams np{(unsigned)H};
    for (unsigned t = 0; t < (unsigned)H; ++t) ew_add(x.data(), o.data(), out, np, t);
    return 0;
}

}  // extern "C"
