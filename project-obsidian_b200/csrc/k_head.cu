// k_head.cu -- the two ends of the model around the MoE stack: the 4-bit token
// embedding, and the final RMSNorm + 4-bit lm_head mat-vec + greedy argmax.
//
// The reference dequantises the embedding row on the CPU (src/forward.rs:445-462:
// w = nib * scale + bias, nibble (word >> 4*(i % 8)) & 15), and ends a decode step
// with rmsnorm(model.norm) -> fused_dequant_matvec_4bit over the vocabulary ->
// a CPU argmax where the first maximum wins (src/forward.rs:553-566).  Here the
// whole head runs on the device.  The lm_head is the largest mat-vec of the
// model (151,936 rows: ~156 MB of 4-bit codes + ~19 MB of scales and biases),
// HBM-bound: every weight byte is read once, with each warp's rows in flight
// together, for all T tokens of the step.
//
// Logits use one canonical fp32 order, shared with oracle/obs_oracle.c so the
// chosen token is bit-exact: w = fma(q, scale, bias) in fp32 (exact product, one
// rounding); 32 lanes, lane l chains acc = fma(w, x, acc) over its 64-column
// groups l*m .. (l+1)*m - 1 (m = H / 2048) in column order; the lane sums meet in
// the adjacent pairwise tree (xor-butterfly offsets 1, 2, 4, 8, 16) -- the
// router's order with 4-bit codes.
#include "obs_internal.cuh"

namespace obs {
namespace {

constexpr int kHeadWarps = 8;                 // warps per lm_head CTA
constexpr int kHeadRowsPerWarp = 2;           // rows a warp has in flight together

// embedding rows: one CTA per token, one thread per packed word (8 columns)
__global__ void __launch_bounds__(256) k_embed(const uint32_t* __restrict__ w, const uint16_t* __restrict__ s,
                                               const uint16_t* __restrict__ b, const int32_t* tokens,
                                               int vocab, int H, uint16_t* __restrict__ x, int* __restrict__ err) {
    pdl_begin();
    const int t = blockIdx.x;
    int tok = tokens[t];
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0) atomicExch(err, kDevBadRoute);
        tok = 0;
    }
    const int G = H / kGroup;
    for (int wi = threadIdx.x; wi < H / 8; wi += blockDim.x) {
        const uint32_t word = __ldg(w + (size_t)tok * (H / 8) + wi);
        const int g = wi / 8;
        const float sc = bf2f(__ldg(s + (size_t)tok * G + g)), bi = bf2f(__ldg(b + (size_t)tok * G + g));
        uint32_t packed[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float lo = __fmaf_rn((float)((word >> (8 * j)) & 0xFu), sc, bi);
            const float hi = __fmaf_rn((float)((word >> (8 * j + 4)) & 0xFu), sc, bi);
            packed[j] = pack_bf2(lo, hi);
        }
        *reinterpret_cast<uint4*>(x + (size_t)t * H + wi * 8) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    }
}

// lm_head logits [T, vocab] for T tokens.  x: the normalised rows, bf16 [T, H],
// staged in shared memory as fp32.  Each warp has kHeadRowsPerWarp rows' loads in
// flight before it computes.
template <int MAXT>
__global__ void __launch_bounds__(32 * kHeadWarps) k_lm_head(const uint32_t* __restrict__ w,
                                                            const uint16_t* __restrict__ s,
                                                            const uint16_t* __restrict__ b,
                                                            const uint16_t* xin, int T, int vocab, int H,
                                                            float* __restrict__ logits) {
    pdl_begin();
    extern __shared__ __align__(16) float s_x[];  // [T][H]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // 8 bf16 per 16-byte load, several loads in flight per thread (H is a multiple of 2048)
#pragma unroll 4
    for (int i = threadIdx.x; i < T * H / 8; i += blockDim.x) {
        const uint4 v = reinterpret_cast<const uint4*>(xin)[i];
        float4* d = reinterpret_cast<float4*>(s_x + 8 * (size_t)i);
        d[0] = make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u),
                           __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xFFFF0000u));
        d[1] = make_float4(__uint_as_float(v.z << 16), __uint_as_float(v.z & 0xFFFF0000u),
                           __uint_as_float(v.w << 16), __uint_as_float(v.w & 0xFFFF0000u));
    }
    __syncthreads();
    const int G = H / kGroup, m = G / 32;
    const int nwarps = gridDim.x * kHeadWarps, gw = blockIdx.x * kHeadWarps + warp;
    for (int r0 = gw * kHeadRowsPerWarp; r0 < vocab; r0 += nwarps * kHeadRowsPerWarp) {
        float acc[kHeadRowsPerWarp][MAXT];
#pragma unroll
        for (int rr = 0; rr < kHeadRowsPerWarp; ++rr)
#pragma unroll
            for (int t = 0; t < MAXT; ++t) acc[rr][t] = 0.0f;
        for (int gi = 0; gi < m; ++gi) {
            const int g = lane * m + gi;
            uint4 q[kHeadRowsPerWarp][2];
            float sc[kHeadRowsPerWarp], bs[kHeadRowsPerWarp];
#pragma unroll
            for (int rr = 0; rr < kHeadRowsPerWarp; ++rr) {  // both rows' loads in flight before any math
                const int row = min(r0 + rr, vocab - 1);
                const uint4* wp = reinterpret_cast<const uint4*>(w + (size_t)row * (H / 8) + (size_t)g * 8);
                q[rr][0] = __ldg(wp), q[rr][1] = __ldg(wp + 1);
                sc[rr] = bf2f(__ldg(s + (size_t)row * G + g));
                bs[rr] = bf2f(__ldg(b + (size_t)row * G + g));
            }
#pragma unroll
            for (int rr = 0; rr < kHeadRowsPerWarp; ++rr) {
                const uint32_t ws[8] = {q[rr][0].x, q[rr][0].y, q[rr][0].z, q[rr][0].w,
                                        q[rr][1].x, q[rr][1].y, q[rr][1].z, q[rr][1].w};
                float wf[64];
#pragma unroll
                for (int c = 0; c < 64; ++c) wf[c] = __fmaf_rn((float)((ws[c >> 3] >> (4 * (c & 7))) & 0xFu), sc[rr], bs[rr]);
#pragma unroll
                for (int t = 0; t < MAXT; ++t) {
                    if (t >= T) break;
                    const float4* xp = reinterpret_cast<const float4*>(s_x + (size_t)t * H + (size_t)g * 64);
                    float a = acc[rr][t];
#pragma unroll
                    for (int v = 0; v < 16; ++v) {
                        const float4 x4 = xp[v];
                        a = __fmaf_rn(wf[4 * v], x4.x, a);
                        a = __fmaf_rn(wf[4 * v + 1], x4.y, a);
                        a = __fmaf_rn(wf[4 * v + 2], x4.z, a);
                        a = __fmaf_rn(wf[4 * v + 3], x4.w, a);
                    }
                    acc[rr][t] = a;
                }
            }
        }
#pragma unroll
        for (int rr = 0; rr < kHeadRowsPerWarp; ++rr) {
            const int row = r0 + rr;
#pragma unroll
            for (int t = 0; t < MAXT; ++t) {
                if (t >= T) break;
                float v = acc[rr][t];
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
                if (lane == 0 && row < vocab) logits[(size_t)t * vocab + row] = v;
            }
        }
    }
}

// order-preserving key of an fp32 logit (-0 folded onto +0)
__device__ __forceinline__ uint32_t logit_key(float f) {
    uint32_t u = __float_as_uint(f == 0.0f ? 0.0f : f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
// better = larger logit, then lower index (the reference's strict '>' scan)
__device__ __forceinline__ bool better(uint32_t ka, int ia, uint32_t kb, int ib) {
    return ka > kb || (ka == kb && ia < ib);
}

// greedy next token: the first maximum of each token's logits (forward.rs:562-565)
__global__ void __launch_bounds__(1024) k_head_argmax(const float* logits, int vocab,
                                                      int32_t* __restrict__ ids) {
    pdl_begin();
    const int t = blockIdx.x;
    __shared__ uint32_t s_k[1024];
    __shared__ int s_i[1024];
    uint32_t k = 0;
    int idx = 0x7fffffff;
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
        const uint32_t ki = logit_key(__ldcg(logits + (size_t)t * vocab + i));
        if (better(ki, i, k, idx)) k = ki, idx = i;
    }
    s_k[threadIdx.x] = k, s_i[threadIdx.x] = idx;
    __syncthreads();
    for (int st = blockDim.x / 2; st > 0; st >>= 1) {
        if (threadIdx.x < st && better(s_k[threadIdx.x + st], s_i[threadIdx.x + st], s_k[threadIdx.x], s_i[threadIdx.x]))
            s_k[threadIdx.x] = s_k[threadIdx.x + st], s_i[threadIdx.x] = s_i[threadIdx.x + st];
        __syncthreads();
    }
    if (threadIdx.x == 0) ids[t] = s_i[0];
}

}  // namespace

cudaError_t launch_embed(const uint32_t* w, const uint16_t* s, const uint16_t* b, const int32_t* tokens, int T,
                         int vocab, int H, uint16_t* x, int* err, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    {
        const cudaError_t le_ = launch_pdl(k_embed, dim3(T), dim3(256), 0, st, w, s, b, tokens, vocab, H, x, err);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

template <int MAXT>
static cudaError_t lm_head_t(const uint32_t* w, const uint16_t* s, const uint16_t* b, const uint16_t* xn, int T,
                             int vocab, int H, float* logits, int num_sms, cudaStream_t st) {
    const size_t smem = (size_t)T * H * 4;
    cudaError_t e = cudaFuncSetAttribute(k_lm_head<MAXT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    // one wave: as many CTAs as fit on the SMs at once (shared memory, 8 x 256 threads), and no
    // more than the rows need, so no CTA stages x without rows to use it on
    int per_sm = (int)((size_t)220 * 1024 / smem);
    per_sm = per_sm < 1 ? 1 : per_sm > 8 ? 8 : per_sm;
    const int rows_per_cta = kHeadWarps * kHeadRowsPerWarp;
    int grid = (vocab + rows_per_cta - 1) / rows_per_cta;
    if (grid > num_sms * per_sm) grid = num_sms * per_sm;
    return launch_pdl(k_lm_head<MAXT>, dim3(grid), dim3(32 * kHeadWarps), smem, st, w, s, b, xn, T, vocab, H,
                      logits);
}

cudaError_t launch_linear4(const uint32_t* w, const uint16_t* s, const uint16_t* b, const uint16_t* x, int T,
                           int rows, int in_f, float* y, int num_sms, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (in_f % 2048) return cudaErrorInvalidValue;
    const int chunk = in_f <= 2048 ? kHeadMaxT : kHeadMaxT / 2;  // x of a chunk fits shared memory as fp32
    for (int t0 = 0; t0 < T; t0 += chunk) {
        const int n = T - t0 < chunk ? T - t0 : chunk;
        const uint16_t* xc = x + (size_t)t0 * in_f;
        float* yc = y + (size_t)t0 * rows;
        cudaError_t e = n <= 1   ? lm_head_t<1>(w, s, b, xc, n, rows, in_f, yc, num_sms, st)
                        : n <= 4 ? lm_head_t<4>(w, s, b, xc, n, rows, in_f, yc, num_sms, st)
                                 : lm_head_t<kHeadMaxT>(w, s, b, xc, n, rows, in_f, yc, num_sms, st);
        if (e != cudaSuccess) return e;
    }
    return cudaGetLastError();
}

cudaError_t launch_lm_head(const uint32_t* w, const uint16_t* s, const uint16_t* b, const uint16_t* xn, int T,
                           int vocab, int H, float* logits, int32_t* ids, int num_sms, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (T > kHeadMaxT || H % 2048) return cudaErrorInvalidValue;
    cudaError_t e = T <= 1   ? lm_head_t<1>(w, s, b, xn, T, vocab, H, logits, num_sms, st)
                    : T <= 4 ? lm_head_t<4>(w, s, b, xn, T, vocab, H, logits, num_sms, st)
                             : lm_head_t<kHeadMaxT>(w, s, b, xn, T, vocab, H, logits, num_sms, st);
    if (e != cudaSuccess) return e;
    e = launch_pdl(k_head_argmax, dim3(T), dim3(1024), 0, st, (const float*)logits, vocab, ids);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace obs
