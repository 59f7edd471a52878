/*
 * obs_oracle.c -- CPU restatement of project-obsidian's MoE hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product): loaded by tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg.  Built with
 * -ffp-contract=off so every fused multiply-add below is an explicit fmaf.
 */
#include "obs_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ bf16 */
float orc_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t orc_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* bf16 nearest-even rounding of a double, in one step (no intermediate fp32
 * rounding); normal bf16 range only, other values go through fp32. */
static uint16_t d2bf(double d) {
    uint64_t u;
    memcpy(&u, &d, 8);
    int e = (int)((u >> 52) & 0x7FF) - 1023 + 127;
    if (e < 1 || e > 254) return orc_f32_to_bf16((float)d);
    uint64_t sign = u >> 63, man = u & 0xFFFFFFFFFFFFFull;
    uint64_t keep = man >> 45, rest = man & ((1ull << 45) - 1), half = 1ull << 44;
    if (rest > half || (rest == half && (keep & 1))) keep++;
    uint32_t v = ((uint32_t)e << 7) + (uint32_t)keep; /* a carry out of the mantissa bumps the exponent */
    return (uint16_t)((sign << 15) | v);
}

void orc_dequant4_bf16(const uint32_t* w, const uint16_t* s, const uint16_t* b, int out_f, int in_f,
                       uint16_t* out) {
    int groups = in_f / 64, words = in_f / 8;
    for (int r = 0; r < out_f; ++r)
        for (int c = 0; c < in_f; ++c) {
            uint32_t q = (w[(size_t)r * words + c / 8] >> (4 * (c % 8))) & 0xFu;
            double sc = orc_bf16_to_f32(s[(size_t)r * groups + c / 64]);
            double bi = orc_bf16_to_f32(b[(size_t)r * groups + c / 64]);
            out[(size_t)r * in_f + c] = d2bf((double)q * sc + bi); /* q*s + b is exact in double */
        }
}

/* ---------------------------------------------------------- synthetic data */
#define GOLDEN_GAMMA 0x9E3779B97F4A7C15ull

static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t orc_stream_key(uint64_t seed, uint32_t layer, uint32_t tensor) {
    uint64_t h = mix64(seed + GOLDEN_GAMMA);
    h = mix64(h ^ ((uint64_t)layer + 1u) * GOLDEN_GAMMA);
    h = mix64(h ^ ((uint64_t)tensor + 1u) * 0xD1B54A32D192ED03ull);
    return h;
}

uint64_t orc_stream_u64(uint64_t key, uint64_t idx) { return mix64(key + (idx + 1u) * GOLDEN_GAMMA); }

/* 24-bit uniform in [0,1): exact in fp32 */
static inline float u24(uint64_t r) { return (float)(uint32_t)(r >> 40) * (1.0f / 16777216.0f); }

/* Irwin-Hall(12) - 6: six 64-bit draws give twelve 24-bit uniforms; the sum is
 * formed in integers and converted once (round to nearest even). */
static inline float normal_ih(uint64_t key, uint64_t idx) {
    int64_t acc = 0;
    for (int m = 0; m < 6; ++m) {
        uint64_t r = orc_stream_u64(key, idx * 6u + (uint64_t)m);
        acc += (int64_t)(r >> 40) + (int64_t)((r >> 16) & 0xFFFFFFu);
    }
    acc -= 6ll * 16777216ll;
    return (float)(int32_t)acc * (1.0f / 16777216.0f);
}

/* scale = bf16(fmaf(u, hi-lo, lo)) */
static inline uint16_t uniform_scale(uint64_t key, uint64_t idx, float lo, float span) {
    return orc_f32_to_bf16(fmaf(u24(orc_stream_u64(key, idx)), span, lo));
}

void orc_synth_router(uint64_t seed, uint32_t layer, int E, int H,
                      uint32_t* w, uint16_t* s, uint16_t* b) {
    uint64_t kw = orc_stream_key(seed, layer, ORC_T_ROUTER_W);
    uint64_t ks = orc_stream_key(seed, layer, ORC_T_ROUTER_S);
    size_t nw = (size_t)E * (size_t)(H / 4), ng = (size_t)E * (size_t)(H / 64);
    for (size_t i = 0; i < nw; ++i) w[i] = (uint32_t)orc_stream_u64(kw, i);
    const float lo = 0.0005f, span = 0.005f - 0.0005f;
    for (size_t i = 0; i < ng; ++i) {
        uint16_t sc = uniform_scale(ks, i, lo, span);
        s[i] = sc;
        b[i] = orc_f32_to_bf16(-128.0f * orc_bf16_to_f32(sc)); /* exact */
    }
}

void orc_synth_proj(uint64_t seed, uint32_t layer, int proj, int E, int out_f, int in_f,
                    uint32_t* w, uint16_t* s, uint16_t* b) {
    uint32_t tw = ORC_T_GATE_W + 3u * (uint32_t)proj;
    uint64_t kw = orc_stream_key(seed, layer, tw);
    uint64_t ks = orc_stream_key(seed, layer, tw + 1u);
    uint64_t kb = orc_stream_key(seed, layer, tw + 2u);
    size_t nw = (size_t)E * out_f * (size_t)(in_f / 8), ng = (size_t)E * out_f * (size_t)(in_f / 64);
    for (size_t i = 0; i < nw; ++i) w[i] = (uint32_t)orc_stream_u64(kw, i);
    const float lo = 0.002f, span = 0.02f - 0.002f;
    for (size_t i = 0; i < ng; ++i) {
        uint16_t sc = uniform_scale(ks, i, lo, span);
        float n = normal_ih(kb, i);
        s[i] = sc;
        b[i] = orc_f32_to_bf16(fmaf(n, 1e-3f, -8.0f * orc_bf16_to_f32(sc)));
    }
}

void orc_rmsnorm_row(const uint16_t* x, int H, float eps, uint16_t* out) {
    /* rmsnorm.metal:20-35: rms = sqrt(mean(x^2) + eps); out = x / rms * w (w = 1) */
    float ss = 0.0f;
    for (int i = 0; i < H; ++i) {
        float v = orc_bf16_to_f32(x[i]);
        ss = fmaf(v, v, ss);
    }
    float rms = sqrtf(ss / (float)H + eps);
    for (int i = 0; i < H; ++i) out[i] = orc_f32_to_bf16(orc_bf16_to_f32(x[i]) / rms);
}

/* The layer-input RMSNorm of the MoE stack, in rmsnorm.metal:9-37's own order:
 * 256 "threads", thread l sums v*v over elements l, l+256, ... (a rounded
 * product, then a rounded add: ps += v * v uncontracted); the 256 partials meet
 * in the halving tree
 * sq[l] += sq[l + s], s = 128, 64, ..., 1; rms = sqrt(sq[0] / dim + eps);
 * out = (x / rms) * w (w = NULL: 1).  x, w and out bf16. */
float orc_rms_tg(const uint16_t* x, int H, float eps) {
    float sq[256];
    for (int l = 0; l < 256; ++l) {
        float ps = 0.0f;
        for (int i = l; i < H; i += 256) {
            float v = orc_bf16_to_f32(x[i]);
            ps = ps + v * v;
        }
        sq[l] = ps;
    }
    for (int st = 128; st > 0; st >>= 1)
        for (int l = 0; l < st; ++l) sq[l] = sq[l] + sq[l + st];
    return sqrtf(sq[0] / (float)H + eps);
}

void orc_rmsnorm_tg_row(const uint16_t* x, const uint16_t* w, int H, float eps, uint16_t* out) {
    const float rms = orc_rms_tg(x, H, eps);
    for (int i = 0; i < H; ++i) {
        float v = orc_bf16_to_f32(x[i]) / rms;
        out[i] = orc_f32_to_bf16(w ? v * orc_bf16_to_f32(w[i]) : v);
    }
}

void orc_synth_x(uint64_t seed, uint32_t layer, int row0, int T, int H, float eps, uint16_t* x) {
    uint64_t kx = orc_stream_key(seed, layer, ORC_T_X);
    uint16_t* raw = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)H);
    for (int t = 0; t < T; ++t) {
        size_t base = (size_t)(row0 + t) * (size_t)H;
        for (int i = 0; i < H; ++i) raw[i] = orc_f32_to_bf16(normal_ih(kx, base + (size_t)i));
        orc_rmsnorm_row(raw, H, eps, x + (size_t)t * H);
    }
    free(raw);
}

/* ---------------------------------------------------------------- dequant */
void orc_dequant4(const uint32_t* w, const uint16_t* s, const uint16_t* b,
                  int out_f, int in_f, float* out) {
    int groups = in_f / 64, words = in_f / 8;
    for (int r = 0; r < out_f; ++r)
        for (int c = 0; c < in_f; ++c) {
            uint32_t q = (w[(size_t)r * words + c / 8] >> (4 * (c % 8))) & 0xFu;
            float sc = orc_bf16_to_f32(s[(size_t)r * groups + c / 64]);
            float bi = orc_bf16_to_f32(b[(size_t)r * groups + c / 64]);
            out[(size_t)r * in_f + c] = fmaf((float)q, sc, bi);
        }
}

void orc_dequant8(const uint32_t* w, const uint16_t* s, const uint16_t* b,
                  int out_f, int in_f, float* out) {
    int groups = in_f / 64, words = in_f / 4;
    for (int r = 0; r < out_f; ++r)
        for (int c = 0; c < in_f; ++c) {
            uint32_t q = (w[(size_t)r * words + c / 4] >> (8 * (c % 4))) & 0xFFu;
            float sc = orc_bf16_to_f32(s[(size_t)r * groups + c / 64]);
            float bi = orc_bf16_to_f32(b[(size_t)r * groups + c / 64]);
            out[(size_t)r * in_f + c] = fmaf((float)q, sc, bi);
        }
}

/* ----------------------------------------------------------------- router */
static float router_dot(const uint32_t* wrow, const uint16_t* srow, const uint16_t* brow,
                        const float* x, int H) {
    int G = H / 64, m = G / 32;
    float lane[32];
    for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int g = l * m; g < (l + 1) * m; ++g) {
            float sc = orc_bf16_to_f32(srow[g]), bi = orc_bf16_to_f32(brow[g]);
            for (int j = 0; j < 64; ++j) {
                int c = g * 64 + j;
                uint32_t q = (wrow[c / 4] >> (8 * (c % 4))) & 0xFFu;
                acc = fmaf(fmaf((float)q, sc, bi), x[c], acc);
            }
        }
        lane[l] = acc;
    }
    for (int o = 1; o < 32; o <<= 1) {
        float nv[32];
        for (int l = 0; l < 32; ++l) nv[l] = lane[l] + lane[l ^ o];
        memcpy(lane, nv, sizeof lane);
    }
    return lane[0];
}

int orc_router_logits(const uint32_t* w, const uint16_t* s, const uint16_t* b,
                      const uint16_t* x, int T, int H, int E, float* logits) {
    if (H % 2048 != 0) return -1; /* 32 lanes x m groups of 64 */
    float* xf = (float*)malloc(sizeof(float) * (size_t)H);
    int G = H / 64;
    for (int t = 0; t < T; ++t) {
        for (int i = 0; i < H; ++i) xf[i] = orc_bf16_to_f32(x[(size_t)t * H + i]);
        for (int e = 0; e < E; ++e)
            logits[(size_t)t * E + e] = router_dot(w + (size_t)e * (H / 4), s + (size_t)e * G,
                                                   b + (size_t)e * G, xf, H);
    }
    free(xf);
    return 0;
}

/* ------------------------------------------------------------------- topk */
void orc_topk(const float* logits, const float* bias, int T, int E, int K, int norm,
              int32_t* ids, float* weights) {
    float* l = (float*)malloc(sizeof(float) * (size_t)E);
    float* p = (float*)malloc(sizeof(float) * (size_t)E);
    for (int t = 0; t < T; ++t) {
        float mx = -INFINITY;
        for (int e = 0; e < E; ++e) {
            l[e] = logits[(size_t)t * E + e] + (bias ? bias[e] : 0.0f);
            if (l[e] > mx) mx = l[e];
        }
        float sum = 0.0f;
        for (int e = 0; e < E; ++e) { p[e] = expf(l[e] - mx); sum += p[e]; }
        float wsum = 0.0f;
        for (int k = 0; k < K; ++k) {
            float best = -INFINITY;
            int bi = -1;
            for (int e = 0; e < E; ++e)
                if (l[e] > best) { best = l[e]; bi = e; }
            ids[(size_t)t * K + k] = bi;
            float pk = p[bi] / sum;
            weights[(size_t)t * K + k] = pk;
            wsum += pk;
            l[bi] = -INFINITY;
        }
        if (norm && wsum > 0.0f)
            for (int k = 0; k < K; ++k) weights[(size_t)t * K + k] /= wsum;
    }
    free(l);
    free(p);
}

/* --------------------------------------------------------------- dispatch */
void orc_dispatch(const int32_t* ids, int T, int E, int K,
                  int32_t* counts, int32_t* offsets, int32_t* slot_of, int32_t* src_token) {
    for (int e = 0; e < E; ++e) counts[e] = 0;
    for (int i = 0; i < T * K; ++i) counts[ids[i]]++;
    offsets[0] = 0;
    for (int e = 0; e < E; ++e) offsets[e + 1] = offsets[e] + counts[e];
    int32_t* fill = (int32_t*)calloc((size_t)E, sizeof(int32_t));
    for (int t = 0; t < T; ++t)
        for (int k = 0; k < K; ++k) {
            int e = ids[t * K + k];
            int slot = offsets[e] + fill[e]++;
            slot_of[t * K + k] = slot;
            if (src_token) src_token[slot] = t;
        }
    free(fill);
}

/* -------------------------------------------------------------- FFN/combine */
/* 8 interleaved fp32 partial sums, then a pairwise tree: deterministic and
 * vectorisable; the reference's exact summation order is not reproduced by
 * any parallel kernel, so outputs are compared within a tolerance. */
static inline float dot8(const float* a, const float* x, int n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int i = 0; i < n; i += 8)
        for (int j = 0; j < 8; ++j) acc[j] = fmaf(a[i + j], x[i + j], acc[j]);
    return ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
}

static inline float silu_mul(float g, float u) { return (g / (1.0f + expf(-g))) * u; }

typedef struct {
    const orc_experts* ex;
    const uint16_t* x;
    int T, wmode;
    const int32_t *counts, *offsets, *src_token;
    uint16_t* y_slots; /* [T*K, H] bf16, slot order */
    uint16_t* h_slots; /* [T*K, I] bf16 or NULL */
    int next_e;
    pthread_mutex_t mu;
} ffn_job;

static void dequant_proj(const orc_experts* ex, int proj, int e, int wmode, float* out) {
    int H = ex->H, I = ex->I;
    int out_f = proj == 2 ? H : I, in_f = proj == 2 ? I : H;
    const uint32_t* w = proj == 0 ? ex->gate_w : proj == 1 ? ex->up_w : ex->down_w;
    const uint16_t* s = proj == 0 ? ex->gate_s : proj == 1 ? ex->up_s : ex->down_s;
    const uint16_t* b = proj == 0 ? ex->gate_b : proj == 1 ? ex->up_b : ex->down_b;
    size_t wo = (size_t)e * out_f * (in_f / 8), so = (size_t)e * out_f * (in_f / 64);
    if (wmode == 1) {
        size_t n = (size_t)out_f * in_f;
        uint16_t* tmp = (uint16_t*)malloc(sizeof(uint16_t) * n);
        orc_dequant4_bf16(w + wo, s + so, b + so, out_f, in_f, tmp);
        for (size_t i = 0; i < n; ++i) out[i] = orc_bf16_to_f32(tmp[i]);
        free(tmp);
    } else {
        orc_dequant4(w + wo, s + so, b + so, out_f, in_f, out);
    }
}

/* One expert's slots in blocks of ORC_NB tokens: each weight row is read once
 * per block (the per-(row, token) dot product is unchanged, so the results do
 * not depend on the block size). */
#define ORC_NB 8
static void* ffn_worker(void* arg) {
    ffn_job* J = (ffn_job*)arg;
    const orc_experts* ex = J->ex;
    int H = ex->H, I = ex->I;
    float* wg = (float*)malloc(sizeof(float) * (size_t)I * H);
    float* wu = (float*)malloc(sizeof(float) * (size_t)I * H);
    float* wd = (float*)malloc(sizeof(float) * (size_t)H * I);
    float* xf = (float*)malloc(sizeof(float) * (size_t)H * ORC_NB);
    float* hf = (float*)malloc(sizeof(float) * (size_t)I * ORC_NB);
    for (;;) {
        pthread_mutex_lock(&J->mu);
        int e = J->next_e++;
        pthread_mutex_unlock(&J->mu);
        if (e >= ex->E) break;
        if (J->counts[e] == 0) continue;
        dequant_proj(ex, 0, e, J->wmode, wg);
        dequant_proj(ex, 1, e, J->wmode, wu);
        dequant_proj(ex, 2, e, J->wmode, wd);
        for (int s0 = J->offsets[e]; s0 < J->offsets[e + 1]; s0 += ORC_NB) {
            int nb = J->offsets[e + 1] - s0 < ORC_NB ? J->offsets[e + 1] - s0 : ORC_NB;
            for (int bt = 0; bt < nb; ++bt) {
                int t = J->src_token[s0 + bt];
                for (int i = 0; i < H; ++i) xf[(size_t)bt * H + i] = orc_bf16_to_f32(J->x[(size_t)t * H + i]);
            }
            for (int i = 0; i < I; ++i)
                for (int bt = 0; bt < nb; ++bt) {
                    float g = dot8(wg + (size_t)i * H, xf + (size_t)bt * H, H);
                    float u = dot8(wu + (size_t)i * H, xf + (size_t)bt * H, H);
                    uint16_t hb = orc_f32_to_bf16(silu_mul(g, u));
                    hf[(size_t)bt * I + i] = orc_bf16_to_f32(hb);
                    if (J->h_slots) J->h_slots[(size_t)(s0 + bt) * I + i] = hb;
                }
            for (int o = 0; o < H; ++o)
                for (int bt = 0; bt < nb; ++bt)
                    J->y_slots[(size_t)(s0 + bt) * H + o] =
                        orc_f32_to_bf16(dot8(wd + (size_t)o * I, hf + (size_t)bt * I, I));
        }
    }
    free(wg); free(wu); free(wd); free(xf); free(hf);
    return NULL;
}

int orc_moe_ffn_combine(const orc_experts* ex, const uint16_t* x, int T,
                        const int32_t* ids, const float* weights, const uint16_t* residual,
                        int wmode, int nthreads, uint16_t* out, uint16_t* h_out, uint16_t* y_out) {
    int E = ex->E, H = ex->H, I = ex->I, K = ex->K;
    if (H % 8 || I % 8 || H % 64 || I % 64) return -1;
    size_t nslots = (size_t)T * K;
    int32_t* counts = (int32_t*)malloc(sizeof(int32_t) * (size_t)E);
    int32_t* offsets = (int32_t*)malloc(sizeof(int32_t) * (size_t)(E + 1));
    int32_t* slot_of = (int32_t*)malloc(sizeof(int32_t) * (nslots ? nslots : 1));
    int32_t* src = (int32_t*)malloc(sizeof(int32_t) * (nslots ? nslots : 1));
    uint16_t* y = (uint16_t*)malloc(sizeof(uint16_t) * (nslots ? nslots : 1) * H);
    uint16_t* hs = h_out ? (uint16_t*)malloc(sizeof(uint16_t) * (nslots ? nslots : 1) * I) : NULL;
    orc_dispatch(ids, T, E, K, counts, offsets, slot_of, src);

    ffn_job J;
    J.ex = ex; J.x = x; J.T = T; J.wmode = wmode;
    J.counts = counts; J.offsets = offsets; J.src_token = src;
    J.y_slots = y; J.h_slots = hs; J.next_e = 0;
    pthread_mutex_init(&J.mu, NULL);
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    for (int i = 1; i < nthreads; ++i) pthread_create(&th[i], NULL, ffn_worker, &J);
    ffn_worker(&J);
    for (int i = 1; i < nthreads; ++i) pthread_join(th[i], NULL);
    pthread_mutex_destroy(&J.mu);

    /* rank-order combine (forward.rs:225-232), fp32 accumulate, one rounding */
    for (int t = 0; t < T; ++t)
        for (int o = 0; o < H; ++o) {
            float acc = residual ? orc_bf16_to_f32(residual[(size_t)t * H + o]) : 0.0f;
            for (int k = 0; k < K; ++k) {
                int slot = slot_of[t * K + k];
                acc = fmaf(weights[t * K + k], orc_bf16_to_f32(y[(size_t)slot * H + o]), acc);
            }
            out[(size_t)t * H + o] = orc_f32_to_bf16(acc);
        }
    if (y_out)
        for (int t = 0; t < T; ++t)
            for (int k = 0; k < K; ++k)
                memcpy(y_out + ((size_t)t * K + k) * H, y + (size_t)slot_of[t * K + k] * H,
                       sizeof(uint16_t) * H);
    if (h_out)
        for (int t = 0; t < T; ++t)
            for (int k = 0; k < K; ++k)
                memcpy(h_out + ((size_t)t * K + k) * I, hs + (size_t)slot_of[t * K + k] * I,
                       sizeof(uint16_t) * I);
    free(counts); free(offsets); free(slot_of); free(src); free(y); free(hs);
    return 0;
}

int orc_moe_layer(const orc_layer* L, const uint16_t* x, int T, const float* logit_bias,
                  const uint16_t* residual, int norm_topk, int wmode, int nthreads,
                  uint16_t* out, int32_t* ids_out, float* w_out) {
    const orc_experts* ex = &L->ex;
    float* logits = (float*)malloc(sizeof(float) * (size_t)T * ex->E + 1);
    int32_t* ids = ids_out ? ids_out : (int32_t*)malloc(sizeof(int32_t) * (size_t)T * ex->K + 1);
    float* w = w_out ? w_out : (float*)malloc(sizeof(float) * (size_t)T * ex->K + 1);
    int rc = orc_router_logits(L->router_w, L->router_s, L->router_b, x, T, ex->H, ex->E, logits);
    if (rc == 0) {
        orc_topk(logits, logit_bias, T, ex->E, ex->K, norm_topk, ids, w);
        rc = orc_moe_ffn_combine(ex, x, T, ids, w, residual, wmode, nthreads, out, NULL, NULL);
    }
    free(logits);
    if (!ids_out) free(ids);
    if (!w_out) free(w);
    return rc;
}

/* ------------------------------------------------------------ model ends */
void orc_embed(const uint32_t* w, const uint16_t* s, const uint16_t* b, int vocab, int H,
               const int32_t* tokens, int T, uint16_t* out) {
    /* forward.rs:449-460: w = nib * scale + bias per column, in f32 */
    int groups = H / 64, words = H / 8;
    for (int t = 0; t < T; ++t) {
        int tok = tokens[t] >= 0 && tokens[t] < vocab ? tokens[t] : 0;
        for (int i = 0; i < H; ++i) {
            uint32_t q = (w[(size_t)tok * words + i / 8] >> (4 * (i % 8))) & 0xFu;
            float sc = orc_bf16_to_f32(s[(size_t)tok * groups + i / 64]);
            float bi = orc_bf16_to_f32(b[(size_t)tok * groups + i / 64]);
            out[(size_t)t * H + i] = orc_f32_to_bf16(fmaf((float)q, sc, bi));
        }
    }
}

typedef struct {
    const uint32_t* w;
    const uint16_t *s, *b, *x;
    int vocab, H, T, nthreads, id;
    float* logits;
} head_job;

static void* head_worker(void* arg) {
    head_job* J = (head_job*)arg;
    int H = J->H, G = H / 64, m = G / 32;
    float* xf = (float*)malloc(sizeof(float) * (size_t)J->T * H);
    for (size_t i = 0; i < (size_t)J->T * H; ++i) xf[i] = orc_bf16_to_f32(J->x[i]);
    for (int r = J->id; r < J->vocab; r += J->nthreads) {
        const uint32_t* wr = J->w + (size_t)r * (H / 8);
        for (int t = 0; t < J->T; ++t) {
            float lane[32];
            for (int l = 0; l < 32; ++l) {
                float acc = 0.0f;
                for (int g = l * m; g < (l + 1) * m; ++g) {
                    float sc = orc_bf16_to_f32(J->s[(size_t)r * G + g]), bi = orc_bf16_to_f32(J->b[(size_t)r * G + g]);
                    for (int j = 0; j < 64; ++j) {
                        int c = g * 64 + j;
                        uint32_t q = (wr[c / 8] >> (4 * (c % 8))) & 0xFu;
                        acc = fmaf(fmaf((float)q, sc, bi), xf[(size_t)t * H + c], acc);
                    }
                }
                lane[l] = acc;
            }
            for (int o = 1; o < 32; o <<= 1) {
                float nv[32];
                for (int l = 0; l < 32; ++l) nv[l] = lane[l] + lane[l ^ o];
                memcpy(lane, nv, sizeof lane);
            }
            J->logits[(size_t)t * J->vocab + r] = lane[0];
        }
    }
    free(xf);
    return NULL;
}

int orc_lm_head_logits(const uint32_t* w, const uint16_t* s, const uint16_t* b, int vocab, int H,
                       const uint16_t* x, int T, int nthreads, float* logits) {
    if (H % 2048 != 0) return -1;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    head_job jobs[256];
    pthread_t th[256];
    for (int i = 0; i < nthreads; ++i) {
        head_job j = {w, s, b, x, vocab, H, T, nthreads, i, logits};
        jobs[i] = j;
        if (i) pthread_create(&th[i], NULL, head_worker, &jobs[i]);
    }
    head_worker(&jobs[0]);
    for (int i = 1; i < nthreads; ++i) pthread_join(th[i], NULL);
    return 0;
}

void orc_argmax_rows(const float* logits, int T, int n, int32_t* ids) {
    for (int t = 0; t < T; ++t) {
        int best = 0;
        float bv = -INFINITY;
        for (int i = 0; i < n; ++i)
            if (logits[(size_t)t * n + i] > bv) bv = logits[(size_t)t * n + i], best = i;
        ids[t] = best;
    }
}

/* ------------------------------------------------------- attention block */
void orc_rope_table(double theta, int hd, int max_seq, float* out) {
    for (int p = 0; p < max_seq; ++p)
        for (int i = 0; i < hd / 2; ++i) {
            double ang = (double)p * pow(theta, -2.0 * i / hd);
            out[((size_t)p * (hd / 2) + i) * 2] = (float)cos(ang);
            out[((size_t)p * (hd / 2) + i) * 2 + 1] = (float)sin(ang);
        }
}

int orc_attn_forward(const orc_attn* A, const uint16_t* x, int T, const int32_t* seq, const int32_t* pos,
                     float eps, int nthreads, uint16_t* out) {
    int H = A->H, nq = A->nq, nkv = A->nkv, hd = A->hd, half = hd / 2;
    if (H % 2048 || (nq * hd) % 2048) return -1;
    size_t rq = (size_t)nq * hd, rk = (size_t)nkv * hd;
    uint16_t* xn = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * H);
    float* q = (float*)malloc(sizeof(float) * (size_t)T * rq);
    float* k = (float*)malloc(sizeof(float) * (size_t)T * rk);
    float* v = (float*)malloc(sizeof(float) * (size_t)T * rk);
    uint16_t* qr = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * rq);
    uint16_t* att = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * rq);
    float* o = (float*)malloc(sizeof(float) * (size_t)T * H);
    float* sc = (float*)malloc(sizeof(float) * (size_t)A->max_seq);
    for (int t = 0; t < T; ++t) orc_rmsnorm_tg_row(x + (size_t)t * H, A->in_norm, H, eps, xn + (size_t)t * H);
    orc_lm_head_logits(A->q_w, A->q_s, A->q_b, (int)rq, H, xn, T, nthreads, q);
    orc_lm_head_logits(A->k_w, A->k_s, A->k_b, (int)rk, H, xn, T, nthreads, k);
    orc_lm_head_logits(A->v_w, A->v_s, A->v_b, (int)rk, H, xn, T, nthreads, v);
    /* head norms, rope, cache append (every token before any attention) */
    uint16_t hb[128], hn[128];
    for (int t = 0; t < T; ++t) {
        int s = seq[t], p = pos[t];
        for (int h = 0; h < nq + nkv; ++h) {
            int isq = h < nq, hh = isq ? h : h - nq;
            const float* src = isq ? q + (size_t)t * rq + (size_t)h * hd : k + (size_t)t * rk + (size_t)hh * hd;
            for (int d = 0; d < hd; ++d) hb[d] = orc_f32_to_bf16(src[d]);
            orc_rmsnorm_tg_row(hb, isq ? A->q_norm : A->k_norm, hd, eps, hn);
            uint16_t* dst = isq ? qr + ((size_t)t * nq + h) * hd
                                : A->kc + (((size_t)s * nkv + hh) * A->max_seq + p) * hd;
            for (int i = 0; i < half; ++i) {
                float c = A->rope[((size_t)p * half + i) * 2], sn = A->rope[((size_t)p * half + i) * 2 + 1];
                float x0 = orc_bf16_to_f32(hn[i]), x1 = orc_bf16_to_f32(hn[i + half]);
                float a = x1 * sn, b = x0 * sn;
                dst[i] = orc_f32_to_bf16(fmaf(x0, c, -a));
                dst[i + half] = orc_f32_to_bf16(fmaf(x1, c, b));
            }
            if (!isq)
                for (int d = 0; d < hd; ++d)
                    A->vc[(((size_t)s * nkv + hh) * A->max_seq + p) * hd + d] =
                        orc_f32_to_bf16(v[(size_t)t * rk + (size_t)hh * hd + d]);
        }
    }
    /* attention */
    float scale = 1.0f / sqrtf((float)hd);
    for (int t = 0; t < T; ++t) {
        int s = seq[t], p = pos[t];
        for (int h = 0; h < nq; ++h) {
            int kvh = h / (nq / nkv);
            const uint16_t* qh = qr + ((size_t)t * nq + h) * hd;
            const uint16_t* kb = A->kc + ((size_t)s * nkv + kvh) * A->max_seq * hd;
            const uint16_t* vb = A->vc + ((size_t)s * nkv + kvh) * A->max_seq * hd;
            float m = -INFINITY;
            for (int j = 0; j <= p; ++j) {
                float lane[32];
                for (int l = 0; l < 32; ++l) {
                    float a = 0.0f;
                    for (int d = l; d < hd; d += 32)
                        a = fmaf(orc_bf16_to_f32(qh[d]), orc_bf16_to_f32(kb[(size_t)j * hd + d]), a);
                    lane[l] = a;
                }
                for (int off = 1; off < 32; off <<= 1) {
                    float nv[32];
                    for (int l = 0; l < 32; ++l) nv[l] = lane[l] + lane[l ^ off];
                    memcpy(lane, nv, sizeof lane);
                }
                sc[j] = lane[0] * scale;
                if (sc[j] > m) m = sc[j];
            }
            float sum = 0.0f;
            for (int j = 0; j <= p; ++j) {
                sc[j] = expf(sc[j] - m);
                sum += sc[j];
            }
            for (int d = 0; d < hd; ++d) {
                float acc = 0.0f;
                for (int j = 0; j <= p; ++j) acc = fmaf(sc[j], orc_bf16_to_f32(vb[(size_t)j * hd + d]), acc);
                att[((size_t)t * nq + h) * hd + d] = orc_f32_to_bf16(acc / sum);
            }
        }
    }
    orc_lm_head_logits(A->o_w, A->o_s, A->o_b, H, (int)rq, att, T, nthreads, o);
    for (size_t i = 0; i < (size_t)T * H; ++i)
        out[i] = orc_f32_to_bf16(orc_bf16_to_f32(x[i]) + orc_bf16_to_f32(orc_f32_to_bf16(o[i])));
    free(xn); free(q); free(k); free(v); free(qr); free(att); free(o); free(sc);
    return 0;
}
