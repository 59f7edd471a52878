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
// logits are produced as 8 partial sums [8][T][E] (each the first two tree
// levels over four leaves) and combined in the rest of the fixed tree by the
// top-k kernel.
#include "router_dev.cuh"

namespace obs {
namespace {

// ---------------------------------------------------------------- decode form
// One warp per (expert, token chunk).  Lane l owns group(s) l*m..; its 64
// dequantised weights per group stay in registers across the chunk's tokens.
constexpr int kLeaves = 32;  // lanes of the canonical order = leaf sums of the prefill form

__global__ void __launch_bounds__(256) k_router_warp(const uint32_t* __restrict__ w, const uint16_t* __restrict__ s,
                                                     const uint16_t* __restrict__ b, const uint16_t* x,
                                                     int T, int H, int E, float* __restrict__ logits) {
    pdl_begin();
    const int e = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (e >= E) return;
    router_warp_item(w, s, b, x, T, H, E, e, blockIdx.y * kWarpTok, threadIdx.x & 31, logits);
}

// ---------------------------------------------------------------- prefill form
// One CTA per (64 tokens, 128 experts, node): node q covers the canonical
// order's leaves 4q .. 4q+3 (lane l's share: groups [l*m, (l+1)*m)) and adds
// them as the first two levels of the adjacent pairwise tree,
// (leaf 4q + leaf 4q+1) + (leaf 4q+2 + leaf 4q+3).  For each group the CTA
// stages the dequantised weights and activations (fp32) in shared memory; each
// of its 256 threads keeps a 4 x 8 register tile of (token, expert)
// accumulators (tokens tt + 16i, experts te + 16j; a warp's activation reads
// cover 16 rows and its weight reads two, served by broadcast) and chains the
// group's 64 columns in order with fused multiply-adds.  The node sums land in
// parts[node][T][E]; top-k (or k_router_finish) adds the 8 nodes in the rest of
// the tree, which together is the decode form's xor-butterfly (offsets 1, 2,
// 4, 8, 16).
constexpr int kRT = 64, kRE = 128, kRPad = 68, kLeafThreads = 256;
constexpr int kNodes = kLeaves / 4;  // partial planes of the prefill form
constexpr size_t kLeafSmem = (size_t)(kRT + kRE) * kRPad * 4;  // 52,224 bytes

__global__ void __launch_bounds__(kLeafThreads, 1) k_router_leaf(const uint32_t* __restrict__ w,
                                                                 const uint16_t* __restrict__ s,
                                                                 const uint16_t* __restrict__ b,
                                                                 const uint16_t* x, int T, int H, int E,
                                                                 float* __restrict__ parts) {
    pdl_begin();
    extern __shared__ __align__(16) float rsm[];
    float(*xs)[kRPad] = reinterpret_cast<float(*)[kRPad]>(rsm);
    float(*ws)[kRPad] = reinterpret_cast<float(*)[kRPad]>(rsm + kRT * kRPad);
    const int tid = threadIdx.x, tt = tid & 15, te = tid >> 4;
    const int t0 = blockIdx.x * kRT, e0 = blockIdx.y * kRE, node = blockIdx.z;
    const int G = H / kGroup, m = G / 32;
    float acc[4][8], pair[4][8], first[4][8];
    for (int lf = 0; lf < 4; ++lf) {
        const int leaf = node * 4 + lf;
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
        for (int g = leaf * m; g < (leaf + 1) * m; ++g) {
            __syncthreads();  // the previous group's tiles are consumed
            // activations: 64 tokens x 64 columns bf16 -> fp32 (8 columns per uint4)
#pragma unroll
            for (int u = 0; u < kRT * 8 / kLeafThreads; ++u) {
                const int i = tid + kLeafThreads * u, r = i >> 3, c8 = i & 7, t = t0 + r;
                uint4 v = make_uint4(0, 0, 0, 0);
                if (t < T) v = reinterpret_cast<const uint4*>(x + (size_t)t * H + (size_t)g * 64)[c8];
                const uint32_t q[4] = {v.x, v.y, v.z, v.w};
                float* d = &xs[r][c8 * 8];
#pragma unroll
                for (int c = 0; c < 4; ++c) d[2 * c] = __uint_as_float(q[c] << 16), d[2 * c + 1] = __uint_as_float(q[c] & 0xFFFF0000u);
            }
            // weights: 128 experts x 64 codes (16 per uint4), w = q * s + b (dequant_matvec_8bit.metal:26)
#pragma unroll
            for (int u = 0; u < kRE * 4 / kLeafThreads; ++u) {
                const int i = tid + kLeafThreads * u, r = i >> 2, c16 = i & 3, e = e0 + r;
                uint4 v = make_uint4(0, 0, 0, 0);
                float sc = 0.0f, bi = 0.0f;
                if (e < E) {
                    v = __ldg(reinterpret_cast<const uint4*>(w + (size_t)e * (H / 4) + (size_t)g * 16) + c16);
                    sc = bf2f(s[(size_t)e * G + g]);
                    bi = bf2f(b[(size_t)e * G + g]);
                }
                const uint32_t q[4] = {v.x, v.y, v.z, v.w};
                float* d = &ws[r][c16 * 16];
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                    for (int j = 0; j < 4; ++j) d[4 * c + j] = __fmaf_rn((float)((q[c] >> (8 * j)) & 0xFFu), sc, bi);
            }
            __syncthreads();
#pragma unroll 2
            for (int j = 0; j < 64; j += 4) {
                float4 xv[4], wv[8];
#pragma unroll
                for (int i = 0; i < 4; ++i) xv[i] = *reinterpret_cast<const float4*>(&xs[tt + 16 * i][j]);
#pragma unroll
                for (int i = 0; i < 8; ++i) wv[i] = *reinterpret_cast<const float4*>(&ws[te + 16 * i][j]);
                // column by column: 32 independent FMAs per column, each chain in column order
#pragma unroll
                for (int a = 0; a < 4; ++a)
#pragma unroll
                    for (int c = 0; c < 8; ++c) acc[a][c] = __fmaf_rn(wv[c].x, xv[a].x, acc[a][c]);
#pragma unroll
                for (int a = 0; a < 4; ++a)
#pragma unroll
                    for (int c = 0; c < 8; ++c) acc[a][c] = __fmaf_rn(wv[c].y, xv[a].y, acc[a][c]);
#pragma unroll
                for (int a = 0; a < 4; ++a)
#pragma unroll
                    for (int c = 0; c < 8; ++c) acc[a][c] = __fmaf_rn(wv[c].z, xv[a].z, acc[a][c]);
#pragma unroll
                for (int a = 0; a < 4; ++a)
#pragma unroll
                    for (int c = 0; c < 8; ++c) acc[a][c] = __fmaf_rn(wv[c].w, xv[a].w, acc[a][c]);
            }
        }
        // the first two tree levels: (l0 + l1) + (l2 + l3)
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (lf == 0) first[i][j] = acc[i][j];
                else if (lf == 1) pair[i][j] = __fadd_rn(first[i][j], acc[i][j]);
                else if (lf == 2) first[i][j] = acc[i][j];
                else pair[i][j] = __fadd_rn(pair[i][j], __fadd_rn(first[i][j], acc[i][j]));
            }
    }
    // node sums out through shared memory ([token][expert]) for coalesced stores
    __syncthreads();
    float(*os)[kRE + 4] = reinterpret_cast<float(*)[kRE + 4]>(rsm);
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 8; ++c) os[tt + 16 * a][te + 16 * c] = pair[a][c];
    __syncthreads();
    float* pl = parts + (size_t)node * T * E;
    for (int i = tid; i < kRT * kRE; i += kLeafThreads) {
        const int r = i / kRE, c = i % kRE, t = t0 + r, e = e0 + c;
        if (t < T && e < E) pl[(size_t)t * E + e] = os[r][c];
    }
}

// logit = the rest of the adjacent pairwise tree over the 8 node sums
__device__ __forceinline__ float tree8(const float* __restrict__ p, size_t plane, size_t i) {
    const float n0 = p[i], n1 = p[plane + i], n2 = p[2 * plane + i], n3 = p[3 * plane + i];
    const float n4 = p[4 * plane + i], n5 = p[5 * plane + i], n6 = p[6 * plane + i], n7 = p[7 * plane + i];
    return __fadd_rn(__fadd_rn(__fadd_rn(n0, n1), __fadd_rn(n2, n3)), __fadd_rn(__fadd_rn(n4, n5), __fadd_rn(n6, n7)));
}

__global__ void k_router_finish(const float* parts, size_t n, float* __restrict__ logits) {
    pdl_begin();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        logits[i] = tree8(parts, n, i);
}

// ---------------------------------------------------------------------- top-k
// Two tokens per CTA: every thread forms logits (the leaf tree when the router
// left 32 partial planes; its 32 loads are independent and coalesced across
// the CTA) into shared memory, then one warp per token selects (body in
// router_dev.cuh).  Enough CTAs to fill the GPU at prefill sizes.
constexpr int kTopkTok = 2;

__global__ void __launch_bounds__(256) k_topk(const float* logits, int nparts,
                                              const float* bias, int T, int E, int K, int norm,
                                              int32_t* __restrict__ ids, float* __restrict__ wout,
                                              float* __restrict__ logits_out) {
    pdl_begin();
    __shared__ float s_l[kTopkTok][kMaxE];
    const int t0 = blockIdx.x * kTopkTok;
    const size_t plane = (size_t)T * E;
    for (int i = threadIdx.x; i < kTopkTok * E; i += blockDim.x) {
        const int tt = i / E, e = i - tt * E, t = t0 + tt;
        if (t < T) {
            const size_t idx = (size_t)t * E + e;
            const float l = nparts == kNodes ? tree8(logits, plane, idx) : logits[idx];
            s_l[tt][e] = l;
            if (logits_out) logits_out[idx] = l;
        }
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = t0 + warp;
    if (warp >= kTopkTok || t >= T) return;
    auto logit = [&](int, int e) { return s_l[warp][e]; };
    int ik;
    float wk;
    topk_token(logit, bias, E, K, norm, lane, &ik, &wk);
    if (lane < K) {
        ids[(size_t)t * K + lane] = ik;
        wout[(size_t)t * K + lane] = wk;
    }
}

}  // namespace

int router_parts(int T) { return T <= 2 * kWarpTok ? 1 : kNodes; }

cudaError_t launch_router_logits(const LayerDev& L, const Shape& sh, const uint16_t* x, int T, float* parts,
                                 cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (router_parts(T) == 1) {
        dim3 grid((sh.E + 7) / 8, (T + kWarpTok - 1) / kWarpTok);
        {
            const cudaError_t le_ = launch_pdl(k_router_warp, dim3(grid), dim3(256), 0, st, L.router_w, L.router_s, L.router_b, x, T, sh.H, sh.E, parts);
            if (le_ != cudaSuccess) return le_;
        }
    } else {
        cudaError_t e = cudaFuncSetAttribute(k_router_leaf, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kLeafSmem);  // 52 KB of dynamic shared memory
        if (e != cudaSuccess) return e;
        dim3 grid((T + kRT - 1) / kRT, (sh.E + kRE - 1) / kRE, kNodes);
        {
            const cudaError_t le_ = launch_pdl(k_router_leaf, dim3(grid), dim3(kLeafThreads), kLeafSmem, st, L.router_w, L.router_s, L.router_b, x, T, sh.H, sh.E,
                                                              parts);
            if (le_ != cudaSuccess) return le_;
        }
    }
    return cudaGetLastError();
}

cudaError_t launch_router_finish(const float* parts, int T, int E, float* logits, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    size_t n = (size_t)T * E;
    {
        const cudaError_t le_ = launch_pdl(k_router_finish, dim3((int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096)), dim3(256), 0, st, parts, n, logits);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

cudaError_t launch_topk(const float* logits, int nparts, const float* bias, int T, int E, int K, int norm,
                        int32_t* ids, float* w, float* logits_out, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (E > kMaxE || K > kMaxK || K > 32) return cudaErrorInvalidValue;
    {
        const cudaError_t le_ = launch_pdl(k_topk, dim3((T + kTopkTok - 1) / kTopkTok), dim3(256), 0, st, logits, nparts,
                                           bias, T, E, K, norm, ids, w, logits_out);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

}  // namespace obs
