// router_dev.cuh -- device bodies of the router's decode form and of top-k,
// shared by the standalone kernels (k_router.cu) and the fused decode layer
// (k_decode.cu) so both compute bit-identical routes.
#pragma once
#include "obs_internal.cuh"

namespace obs {

constexpr int kWarpTok = 8;   // tokens per warp item of the decode-form router
constexpr int kMaxE = 256, kMaxK = 16;

// One warp: logits of expert e for tokens t0 .. t0+7 in the canonical order
// (dequant_matvec_8bit.metal:8-31): lane l chains fma(w, x, acc) over its
// groups l*m .. (l+1)*m-1 in column order, the lanes meet in the adjacent
// pairwise tree (xor-butterfly offsets 1, 2, 4, 8, 16).  The weights come
// through the read-only path; x, written by an earlier kernel of the stream,
// with ordinary loads after the dependent-launch wait.
__device__ __forceinline__ void router_warp_item(const uint32_t* __restrict__ w, const uint16_t* __restrict__ s,
                                                 const uint16_t* __restrict__ b, const uint16_t* x,
                                                 int T, int H, int E, int e, int t0, int lane,
                                                 float* __restrict__ logits) {
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
                    uint4 q = xr[v];
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

// Top-k selection uses an order-preserving integer key of the fp32 logit (-0
// folded onto +0): the warp max of the keys, then the lowest expert index
// holding that key, which is the reference's strict '>' scan
// (moe_routing_topk.metal:43-52).
__device__ __forceinline__ uint32_t order_key(float f) {
    uint32_t u = __float_as_uint(f == 0.0f ? 0.0f : f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// One warp, one token (moe_routing_topk.metal:31-56): softmax in fp32, K
// rounds of argmax (lowest index on ties), renormalise.  logit(i, e) returns
// the token's logit of expert e = lane + 32 i; lane k < K ends with (*id,
// *wt) of rank k.  The rounds only select; the maximum is the first winner's
// logit, and lane k forms e_k = exp(l_k - max).  With renormalisation the
// weights are e_k / sum_{j<K} e_j (the softmax denominator cancels; the sum
// adds in rank order), otherwise e_k / sum_e exp(l_e - max) (lane-strided
// partial sums, then the xor tree).
struct NoMark {
    __device__ __forceinline__ void operator()(int) const {}
};
template <class LogitFn, class Mark = NoMark>
__device__ __forceinline__ void topk_token(LogitFn logit, const float* bias, int E, int K, int norm,
                                           int lane, int* id, float* wt, Mark mark = Mark()) {
    uint32_t key[kMaxE / 32];
#pragma unroll
    for (int i = 0; i < kMaxE / 32; ++i) {
        const int e = lane + 32 * i;
        key[i] = 0;  // below every real key: never selected
        if (e < E) key[i] = order_key(__fadd_rn(logit(i, e), bias ? bias[e] : 0.0f));
    }
    mark(0);
    const int ne = (E + 31) >> 5;
    uint32_t kk = 0, top = 0;
    int ik = 0;
#pragma unroll
    for (int k = 0; k < kMaxK; ++k) {
        if (k >= K) break;
        uint32_t kb = 0;
        int ib = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < kMaxE / 32; ++i)
            if (i < ne && key[i] > kb) kb = key[i], ib = lane + 32 * i;
        const uint32_t best = __reduce_max_sync(0xffffffffu, kb);
        const int bi = (int)__reduce_min_sync(0xffffffffu, kb == best ? (uint32_t)ib : 0x7fffffffu);
        // clear the winner's key (compile-time indices: key[] stays in registers)
#pragma unroll
        for (int i = 0; i < kMaxE / 32; ++i)
            if (bi == lane + 32 * i) key[i] = 0;
        if (lane == k) kk = best, ik = bi;
        if (k == 0) top = best;
    }
    mark(1);
    const float mx = key_value(top);
    const float ek = lane < K ? expf(key_value(kk) - mx) : 0.0f;
    float den = 0.0f;
    if (norm) {
#pragma unroll
        for (int k = 0; k < kMaxK; ++k)
            if (k < K) den += __shfl_sync(0xffffffffu, ek, k);
    } else {
#pragma unroll
        for (int i = 0; i < kMaxE / 32; ++i) {
            const int e = lane + 32 * i;
            if (e < E) den += expf(__fadd_rn(logit(i, e), bias ? bias[e] : 0.0f) - mx);
        }
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    }
    mark(2);
    *id = ik;
    *wt = den > 0.0f ? ek / den : ek;
}

}  // namespace obs
