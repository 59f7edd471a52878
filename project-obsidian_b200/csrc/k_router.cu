// k_router.cu -- the MoE router: 8-bit gate mat-vec/GEMM and top-k.
//
// Router logits follow dequant_matvec_8bit.metal:8-31 (byte i of a row is
// column i; w = q*scale + bias per 64-column group) in ONE canonical fp32
// order shared with oracle/obs_oracle.c so expert selection is bit-exact:
//   32 lanes; lane l chains acc = fma(w, x, acc) over groups [l*m,(l+1)*m)
//   (m = H/2048) in column order; the lane sums meet in the adjacent pairwise
//   tree (xor-butterfly offsets 1,2,4,8,16).
// Top-k follows moe_routing_topk.metal:31-56 (softmax in fp32, repeated
// argmax with the lowest index winning ties, renormalise), selecting on the
// fp32 logits so the choice depends only on bit-exact values.  For T > 16 the
// logits are produced as eight partial subtree sums [8][T][E] (more CTAs) and
// combined in the fixed tree by the top-k kernel.
#include "obs_internal.cuh"

namespace obs {
namespace {

// ---------------------------------------------------------------- decode form
// One warp per (expert, token chunk).  Lane l owns group(s) l*m..; its 64
// dequantised weights per group stay in registers across the chunk's tokens.
constexpr int kWarpTok = 8;

__global__ void __launch_bounds__(256) k_router_warp(const uint32_t* __restrict__ w, const uint16_t* __restrict__ s,
                                                     const uint16_t* __restrict__ b, const uint16_t* __restrict__ x,
                                                     int T, int H, int E, float* __restrict__ logits) {
    const int lane = threadIdx.x & 31;
    const int e = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int t0 = blockIdx.y * kWarpTok;
    if (e >= E) return;
    const int G = H / kGroup, m = G / 32;
    float acc[kWarpTok];
#pragma unroll
    for (int i = 0; i < kWarpTok; ++i) acc[i] = 0.0f;
    for (int gi = 0; gi < m; ++gi) {
        const int g = lane * m + gi;
        const float sc = bf2f(s[(size_t)e * G + g]), bi = bf2f(b[(size_t)e * G + g]);
        const uint4* wr = reinterpret_cast<const uint4*>(w + (size_t)e * (H / 4) + (size_t)g * 16);
        float wf[64];
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            uint4 q = __ldg(wr + v);
            uint32_t qs[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int c = 0; c < 4; ++c)
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    wf[v * 16 + c * 4 + j] = __fmaf_rn((float)((qs[c] >> (8 * j)) & 0xFFu), sc, bi);
        }
#pragma unroll
        for (int i = 0; i < kWarpTok; ++i) {
            if (t0 + i < T) {
                const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)(t0 + i) * H + (size_t)g * 64);
                float a = acc[i];
#pragma unroll
                for (int v = 0; v < 8; ++v) {
                    uint4 q = __ldg(xr + v);
                    uint32_t qs[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        a = __fmaf_rn(wf[v * 8 + c * 2], __uint_as_float(qs[c] << 16), a);
                        a = __fmaf_rn(wf[v * 8 + c * 2 + 1], __uint_as_float(qs[c] & 0xFFFF0000u), a);
                    }
                }
                acc[i] = a;
            }
        }
    }
#pragma unroll
    for (int i = 0; i < kWarpTok; ++i) {
        float v = acc[i];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0 && t0 + i < T) logits[(size_t)(t0 + i) * E + e] = v;
    }
}

// ---------------------------------------------------------------- prefill form
// CTA tile: 32 tokens x 64 experts x one eighth of the 32 lanes (a 4-leaf
// subtree of the reduction tree).  Per group the CTA stages the group's
// dequantised weights and activations (fp32) in shared memory, the next
// group's global loads already in flight; every (token, expert) accumulator
// chains its group in column order and folds the lane sums into a 2-deep
// binary-counter stack, which evaluates exactly the adjacent pairwise tree of
// the decode form on its 4 leaves.  The eight subtree sums meet as
// (((S0+S1)+(S2+S3))+((S4+S5)+(S6+S7))) in the top-k kernel (or k_router_finish).
constexpr int kTT = 32, kTE = 64, kPad = 68, kSplit = 8;

struct RouterStage {
    uint32_t q[4];
    float sc[4], bi[4];
    uint4 xv;
};

__device__ __forceinline__ void router_load(RouterStage& r, const uint32_t* __restrict__ w,
                                            const uint16_t* __restrict__ s, const uint16_t* __restrict__ b,
                                            const uint16_t* __restrict__ x, int T, int H, int E, int G, int t0,
                                            int e0, int g, int tid) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int i = tid + 256 * u, el = i >> 4, wd = i & 15, e = e0 + el;
        r.q[u] = 0, r.sc[u] = 0.0f, r.bi[u] = 0.0f;
        if (e < E) {
            r.q[u] = __ldg(w + (size_t)e * (H / 4) + (size_t)g * 16 + wd);
            r.sc[u] = bf2f(s[(size_t)e * G + g]);
            r.bi[u] = bf2f(b[(size_t)e * G + g]);
        }
    }
    const int tl = tid >> 3, v = tid & 7, t = t0 + tl;
    r.xv = make_uint4(0, 0, 0, 0);
    if (t < T) r.xv = __ldg(reinterpret_cast<const uint4*>(x + (size_t)t * H + (size_t)g * 64) + v);
}

__global__ void __launch_bounds__(256) k_router_tiled(const uint32_t* __restrict__ w, const uint16_t* __restrict__ s,
                                                      const uint16_t* __restrict__ b, const uint16_t* __restrict__ x,
                                                      int T, int H, int E, float* __restrict__ parts) {
    __shared__ __align__(16) float ws[kTE][kPad];
    __shared__ __align__(16) float xs[kTT][kPad];
    const int tid = threadIdx.x;
    const int tt = tid & 15, te = tid >> 4;  // 16 x 16 threads; micro-tile 2 tokens x 4 experts
    const int t0 = blockIdx.x * kTT, e0 = blockIdx.y * kTE, split = blockIdx.z;
    const int G = H / kGroup, m = G / 32;
    const int g0 = split * 4 * m, g1 = g0 + 4 * m;  // this eighth's groups (leaves split*4 .. +3)
    float lane_acc[2][4], st0[2][4], st1[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) lane_acc[i][j] = st0[i][j] = st1[i][j] = 0.0f;

    RouterStage nxt;
    router_load(nxt, w, s, b, x, T, H, E, G, t0, e0, g0, tid);
    for (int g = g0; g < g1; ++g) {
        __syncthreads();
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int i = tid + 256 * u, el = i >> 4, wd = i & 15;
            float f[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) f[j] = __fmaf_rn((float)((nxt.q[u] >> (8 * j)) & 0xFFu), nxt.sc[u], nxt.bi[u]);
            *reinterpret_cast<float4*>(&ws[el][wd * 4]) = make_float4(f[0], f[1], f[2], f[3]);
        }
        {
            const uint32_t qs[4] = {nxt.xv.x, nxt.xv.y, nxt.xv.z, nxt.xv.w};
            float* d = &xs[tid >> 3][(tid & 7) * 8];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                d[2 * c] = __uint_as_float(qs[c] << 16);
                d[2 * c + 1] = __uint_as_float(qs[c] & 0xFFFF0000u);
            }
        }
        __syncthreads();
        if (g + 1 < g1) router_load(nxt, w, s, b, x, T, H, E, G, t0, e0, g + 1, tid);
#pragma unroll 4
        for (int j = 0; j < 64; j += 4) {
            float4 xv[2], wv[4];
#pragma unroll
            for (int i = 0; i < 2; ++i) xv[i] = *reinterpret_cast<const float4*>(&xs[tt + 16 * i][j]);
#pragma unroll
            for (int i = 0; i < 4; ++i) wv[i] = *reinterpret_cast<const float4*>(&ws[te + 16 * i][j]);
#pragma unroll
            for (int a = 0; a < 2; ++a)
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float acc = lane_acc[a][c];
                    acc = __fmaf_rn(wv[c].x, xv[a].x, acc);
                    acc = __fmaf_rn(wv[c].y, xv[a].y, acc);
                    acc = __fmaf_rn(wv[c].z, xv[a].z, acc);
                    acc = __fmaf_rn(wv[c].w, xv[a].w, acc);
                    lane_acc[a][c] = acc;
                }
        }
        if (((g - g0) % m) == m - 1) {
            const int leaf = (g - g0) / m;  // 0..3 inside this subtree
#pragma unroll
            for (int a = 0; a < 2; ++a)
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float v = lane_acc[a][c];
                    lane_acc[a][c] = 0.0f;
                    if (leaf & 1) {
                        v = __fadd_rn(st0[a][c], v);
                        if (leaf & 2) v = __fadd_rn(st1[a][c], v);
                        st1[a][c] = v;
                    } else {
                        st0[a][c] = v;
                    }
                }
        }
    }
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            int t = t0 + tt + 16 * a, e = e0 + te + 16 * c;
            if (t < T && e < E) parts[((size_t)split * T + t) * E + e] = st1[a][c];
        }
}

// logits = (((S0+S1)+(S2+S3))+((S4+S5)+(S6+S7))) of the eight subtree sums
__device__ __forceinline__ float tree8(const float* __restrict__ p, size_t plane, size_t i) {
    const float a = __fadd_rn(__fadd_rn(p[i], p[plane + i]), __fadd_rn(p[2 * plane + i], p[3 * plane + i]));
    const float c = __fadd_rn(__fadd_rn(p[4 * plane + i], p[5 * plane + i]), __fadd_rn(p[6 * plane + i], p[7 * plane + i]));
    return __fadd_rn(a, c);
}

__global__ void k_router_finish(const float* __restrict__ parts, size_t n, float* __restrict__ logits) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        logits[i] = tree8(parts, n, i);
}

// ---------------------------------------------------------------------- top-k
// One warp per token; lane l holds experts l, l+32, ...  Selection uses an
// order-preserving integer key of the fp32 logit (-0 folded onto +0): the
// warp max of the keys, then the lowest expert index holding that key, which
// is the reference's strict '>' scan (moe_routing_topk.metal:43-52).
constexpr int kMaxE = 256, kMaxK = 16;

__device__ __forceinline__ uint32_t order_key(float f) {
    uint32_t u = __float_as_uint(f == 0.0f ? 0.0f : f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

__global__ void __launch_bounds__(256) k_topk(const float* __restrict__ logits, int nparts,
                                              const float* __restrict__ bias, int T, int E, int K, int norm,
                                              int32_t* __restrict__ ids, float* __restrict__ wout,
                                              int32_t* __restrict__ counts, float* __restrict__ logits_out) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= T) return;
    const size_t plane = (size_t)T * E;
    uint32_t key[kMaxE / 32];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kMaxE / 32; ++i) {
        const int e = lane + 32 * i;
        key[i] = 0;  // below every real key: never selected
        if (e < E) {
            const size_t idx = (size_t)t * E + e;
            float l = nparts == kSplit ? tree8(logits, plane, idx) : logits[idx];
            if (logits_out) logits_out[idx] = l;
            l = __fadd_rn(l, bias ? bias[e] : 0.0f);
            key[i] = order_key(l);
            mx = fmaxf(mx, l);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float se = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxE / 32; ++i)
        if (lane + 32 * i < E) se += expf(key_value(key[i]) - mx);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) se += __shfl_xor_sync(0xffffffffu, se, o);

    float wk = 0.0f, wsum = 0.0f;
    int ik = 0;
#pragma unroll
    for (int k = 0; k < kMaxK; ++k) {
        if (k >= K) break;
        uint32_t kb = 0;
        int ib = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < kMaxE / 32; ++i)
            if (key[i] > kb) kb = key[i], ib = lane + 32 * i;
        const uint32_t best = __reduce_max_sync(0xffffffffu, kb);
        const int bi = (int)__reduce_min_sync(0xffffffffu, kb == best ? (uint32_t)ib : 0x7fffffffu);
        if ((bi & 31) == lane) key[bi >> 5] = 0;
        const float p = expf(key_value(best) - mx) / se;
        wsum += p;
        if (lane == k) wk = p, ik = bi;
    }
    if (lane < K) {
        ids[(size_t)t * K + lane] = ik;
        wout[(size_t)t * K + lane] = (norm && wsum > 0.0f) ? wk / wsum : wk;
        if (counts) atomicAdd(counts + ik, 1);
    }
}

}  // namespace

int router_parts(int T) { return T <= 2 * kWarpTok ? 1 : kSplit; }

cudaError_t launch_router_logits(const LayerDev& L, const Shape& sh, const uint16_t* x, int T, float* parts,
                                 cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (router_parts(T) == 1) {
        dim3 grid((sh.E + 7) / 8, (T + kWarpTok - 1) / kWarpTok);
        note_launch();
        k_router_warp<<<grid, 256, 0, st>>>(L.router_w, L.router_s, L.router_b, x, T, sh.H, sh.E, parts);
    } else {
        dim3 grid((T + kTT - 1) / kTT, (sh.E + kTE - 1) / kTE, kSplit);
        note_launch();
        k_router_tiled<<<grid, 256, 0, st>>>(L.router_w, L.router_s, L.router_b, x, T, sh.H, sh.E, parts);
    }
    return cudaGetLastError();
}

cudaError_t launch_router_finish(const float* parts, int T, int E, float* logits, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    size_t n = (size_t)T * E;
    note_launch();
    k_router_finish<<<(int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096), 256, 0, st>>>(parts, n, logits);
    return cudaGetLastError();
}

cudaError_t launch_topk(const float* logits, int nparts, const float* bias, int T, int E, int K, int norm,
                        int32_t* ids, float* w, int32_t* counts, float* logits_out, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (E > kMaxE || K > kMaxK || K > 32) return cudaErrorInvalidValue;
    note_launch();
    k_topk<<<(T + 7) / 8, 256, 0, st>>>(logits, nparts, bias, T, E, K, norm, ids, w, counts, logits_out);
    return cudaGetLastError();
}

}  // namespace obs
