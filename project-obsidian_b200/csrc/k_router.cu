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
// fp32 logits so the choice depends only on bit-exact values.
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
// CTA tile: 64 tokens x 64 experts, thread micro-tile 4 x 4.  Per group the
// CTA stages the group's dequantised weights and activations (fp32) in shared
// memory; every (token, expert) accumulator chains its group in column order
// and folds the lane sums into a 5-deep binary-counter stack, which evaluates
// exactly the adjacent pairwise tree of the decode form.
constexpr int kTT = 64, kTE = 64, kPad = 68;

__global__ void __launch_bounds__(256) k_router_tiled(const uint32_t* __restrict__ w, const uint16_t* __restrict__ s,
                                                      const uint16_t* __restrict__ b, const uint16_t* __restrict__ x,
                                                      int T, int H, int E, float* __restrict__ logits) {
    __shared__ __align__(16) float ws[kTE][kPad];
    __shared__ __align__(16) float xs[kTT][kPad];
    const int tid = threadIdx.x;
    const int tt = tid & 15, te = tid >> 4;  // 16 x 16 threads
    const int t0 = blockIdx.x * kTT, e0 = blockIdx.y * kTE;
    const int G = H / kGroup, m = G / 32;
    float lane_acc[4][4], st0[4][4], st1[4][4], st2[4][4], st3[4][4], st4[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) lane_acc[i][j] = 0.0f, st0[i][j] = st1[i][j] = st2[i][j] = st3[i][j] = st4[i][j] = 0.0f;

    for (int g = 0; g < G; ++g) {
        __syncthreads();
        // weights: 64 experts x 64 codes = 1024 words; thread -> 4 words
        for (int i = tid; i < kTE * 16; i += 256) {
            int el = i >> 4, wd = i & 15, e = e0 + el;
            float f[4] = {0, 0, 0, 0};
            if (e < E) {
                uint32_t q = __ldg(w + (size_t)e * (H / 4) + (size_t)g * 16 + wd);
                float sc = bf2f(s[(size_t)e * G + g]), bi = bf2f(b[(size_t)e * G + g]);
#pragma unroll
                for (int j = 0; j < 4; ++j) f[j] = __fmaf_rn((float)((q >> (8 * j)) & 0xFFu), sc, bi);
            }
            *reinterpret_cast<float4*>(&ws[el][wd * 4]) = make_float4(f[0], f[1], f[2], f[3]);
        }
        // activations: 64 tokens x 64 bf16 = 512 uint4
        for (int i = tid; i < kTT * 8; i += 256) {
            int tl = i >> 3, v = i & 7, t = t0 + tl;
            uint4 q = make_uint4(0, 0, 0, 0);
            if (t < T) q = __ldg(reinterpret_cast<const uint4*>(x + (size_t)t * H + (size_t)g * 64) + v);
            uint32_t qs[4] = {q.x, q.y, q.z, q.w};
            float* d = &xs[tl][v * 8];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                d[2 * c] = __uint_as_float(qs[c] << 16);
                d[2 * c + 1] = __uint_as_float(qs[c] & 0xFFFF0000u);
            }
        }
        __syncthreads();
#pragma unroll 4
        for (int j = 0; j < 64; j += 4) {
            float4 xv[4], wv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) xv[i] = *reinterpret_cast<const float4*>(&xs[tt + 16 * i][j]);
#pragma unroll
            for (int i = 0; i < 4; ++i) wv[i] = *reinterpret_cast<const float4*>(&ws[te + 16 * i][j]);
#pragma unroll
            for (int a = 0; a < 4; ++a)
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
        if ((g % m) == m - 1) {
            const int leaf = g / m;  // lane index of the decode form
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float v = lane_acc[a][c];
                    lane_acc[a][c] = 0.0f;
                    if (leaf & 1) {
                        v = __fadd_rn(st0[a][c], v);
                        if (leaf & 2) {
                            v = __fadd_rn(st1[a][c], v);
                            if (leaf & 4) {
                                v = __fadd_rn(st2[a][c], v);
                                if (leaf & 8) {
                                    v = __fadd_rn(st3[a][c], v);
                                    if (leaf & 16) v = __fadd_rn(st4[a][c], v);
                                    st4[a][c] = v;
                                } else st3[a][c] = v;
                            } else st2[a][c] = v;
                        } else st1[a][c] = v;
                    } else st0[a][c] = v;
                }
        }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            int t = t0 + tt + 16 * a, e = e0 + te + 16 * c;
            if (t < T && e < E) logits[(size_t)t * E + e] = st4[a][c];
        }
}

// ---------------------------------------------------------------------- top-k
// One warp per token.  Lane l holds experts l, l+32, ...
constexpr int kMaxE = 256, kMaxK = 16;

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

__global__ void __launch_bounds__(256) k_topk(const float* __restrict__ logits, const float* __restrict__ bias,
                                              int T, int E, int K, int norm, int32_t* __restrict__ ids,
                                              float* __restrict__ wout, int32_t* __restrict__ counts,
                                              int* __restrict__ err) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= T) return;
    const int per = (E + 31) / 32;
    float l[kMaxE / 32];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kMaxE / 32; ++i) {
        int e = lane + 32 * i;
        l[i] = -INFINITY;
        if (i < per && e < E) {
            l[i] = __fadd_rn(logits[(size_t)t * E + e], bias ? bias[e] : 0.0f);
            mx = fmaxf(mx, l[i]);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float se = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxE / 32; ++i)
        if (i < per && lane + 32 * i < E) se += expf(l[i] - mx);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) se += __shfl_xor_sync(0xffffffffu, se, o);

    float wk[kMaxK];
    int ik[kMaxK];
    float wsum = 0.0f;
    for (int k = 0; k < K; ++k) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < kMaxE / 32; ++i) {
            int e = lane + 32 * i;
            if (i < per && e < E && better(l[i], e, bv, bi)) bv = l[i], bi = e;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(ov, oi, bv, bi)) bv = ov, bi = oi;
        }
        if ((bi & 31) == lane) l[bi >> 5] = -INFINITY;
        float p = expf(bv - mx) / se;
        wk[k] = p;
        ik[k] = bi;
        wsum += p;
    }
    if (lane == 0) {
        for (int k = 0; k < K; ++k) {
            int e = ik[k];
            if (e < 0 || e >= E) {  // unreachable for finite logits; reported, never indexed
                atomicExch(err, kDevBadRoute);
                e = 0;
            }
            ids[(size_t)t * K + k] = e;
            wout[(size_t)t * K + k] = (norm && wsum > 0.0f) ? wk[k] / wsum : wk[k];
            if (counts) atomicAdd(counts + e, 1);
        }
    }
}

}  // namespace

cudaError_t launch_router_logits(const LayerDev& L, const Shape& sh, const uint16_t* x, int T, float* logits,
                                 cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (T <= 2 * kWarpTok) {
        dim3 grid((sh.E + 7) / 8, (T + kWarpTok - 1) / kWarpTok);
        k_router_warp<<<grid, 256, 0, st>>>(L.router_w, L.router_s, L.router_b, x, T, sh.H, sh.E, logits);
    } else {
        dim3 grid((T + kTT - 1) / kTT, (sh.E + kTE - 1) / kTE);
        k_router_tiled<<<grid, 256, 0, st>>>(L.router_w, L.router_s, L.router_b, x, T, sh.H, sh.E, logits);
    }
    return cudaGetLastError();
}

cudaError_t launch_topk(const float* logits, const float* bias, int T, int E, int K, int norm, int32_t* ids,
                        float* w, int32_t* counts, int* err, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    k_topk<<<(T + 7) / 8, 256, 0, st>>>(logits, bias, T, E, K, norm, ids, w, counts, err);
    return cudaGetLastError();
}

}  // namespace obs
