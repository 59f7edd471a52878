// k_attn.cu -- the attention block of a Qwen3-MoE layer (the part of
// Model::forward_layer before the MoE, src/forward.rs:404-419):
//   xn = RMSNorm(x, input_layernorm)              rmsnorm.metal:9-37
//   q, k, v = 4-bit mat-vecs of xn                fused_dequant_matvec_4bit.metal
//   q, k = per-head RMSNorm (q_norm, k_norm)      rmsnorm over head_dim rows
//   q, k = NeoX RoPE at the token's position      rope.metal:10-27
//   cache[seq][pos] = k, v                        ops.metal:32-37 kv_append, kv_cache.rs:15-24
//   a = softmax(q k^T / sqrt(hd)) v over the sequence's positions <= pos, GQA
//                                                 sdpa_decode.metal:14-48, attention.rs:23-41
//   x1 = x + o_proj(a)                            ops.metal:11-15
// for T tokens, each of a given sequence (its own KV cache) at a given position:
// a batch of decode steps (one token per sequence) or a prefill (consecutive
// positions of one sequence; each token attends to its own prefix, so the
// block is causal).
//
// The mat-vecs use the lm_head's canonical fp32 order (k_lm_head), rounded to
// bf16 like the reference's half outputs.  RoPE takes cos/sin from a table the
// host computes once in double precision (rope_table), so the arithmetic after
// it is plain fp32 and the cached K rows are bit-exact with the CPU oracle.
// Attention uses fp32 scores, the exponential and one division; its output is
// compared within a tolerance.
#include "obs_internal.cuh"

namespace obs {
namespace {

constexpr int kAttnThreads = 128;  // one CTA per (token, query head); head_dim <= 128

// NeoX half-split rotation of one head in place (rope.metal:19-26): for i < hd/2,
// (x_i, x_{i+hd/2}) -> (x_i c - x_{i+hd/2} s, x_{i+hd/2} c + x_i s), with
// c, s = cos, sin of pos * theta^(-2i/hd) from the table.  In: fp32 after the
// head norm (bf16-rounded); out: bf16.
__device__ __forceinline__ void rope_pair(float x0, float x1, float c, float s, uint16_t* o0, uint16_t* o1) {
    const float a = __fmul_rn(x1, s), b = __fmul_rn(x0, s);
    *o0 = f2bf(__fmaf_rn(x0, c, -a));
    *o1 = f2bf(__fmaf_rn(x1, c, b));
}

// q/k head norm + RoPE + cache append.  One CTA per (token, head) of q (nq heads)
// and k (nkv heads): grid (T, nq + nkv), 128 threads.  qkv: fp32 projections
// [T][nq*hd + 2*nkv*hd] (q | k | v).  The head's rms in rmsnorm.metal's order
// (256 "threads" strided over hd, halving tree) -- here 128 threads carry the
// first 128 partials and the upper 128 are zero, which is the same sum.
__global__ void __launch_bounds__(kAttnThreads) k_qk_norm_rope(const float* qkv, int T, int nq, int nkv,
                                                               int hd, const uint16_t* __restrict__ qn,
                                                               const uint16_t* __restrict__ kn, float eps,
                                                               const float* __restrict__ rope_cs, int max_seq,
                                                               const int32_t* seq,
                                                               const int32_t* pos,
                                                               uint16_t* __restrict__ qout, uint16_t* kcache,
                                                               uint16_t* vcache, int n_seqs, int* err) {
    pdl_begin();
    __shared__ float sq[256];
    __shared__ float sx[128];
    const int t = blockIdx.x, h = blockIdx.y, l = threadIdx.x;
    const int width = (nq + 2 * nkv) * hd;
    const bool isq = h < nq;
    const int hh = isq ? h : h - nq;
    const float* src = qkv + (size_t)t * width + (isq ? (size_t)h * hd : (size_t)nq * hd + (size_t)hh * hd);
    const int s_id = seq[t], p = pos[t];
    if (s_id < 0 || s_id >= n_seqs || p < 0 || p >= max_seq) {
        if (l == 0) atomicExch(err, kDevBadPos);
        return;
    }
    // the projection rounded to bf16 (the reference's half output), then the head norm
    const float v = l < hd ? bf2f(f2bf(src[l])) : 0.0f;
    sq[l] = __fmul_rn(v, v);
    sq[l + 128] = 0.0f;
    __syncthreads();
    for (int st = 128; st > 0; st >>= 1) {
        if (l < st) sq[l] = __fadd_rn(sq[l], sq[l + st]);
        __syncthreads();
    }
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(sq[0], (float)hd), eps));
    const uint16_t* wn = isq ? qn : kn;
    if (l < hd) sx[l] = bf2f(f2bf(__fmul_rn(__fdiv_rn(v, rms), bf2f(wn[l]))));
    __syncthreads();
    const int half = hd / 2;
    if (l < half) {
        const float c = rope_cs[((size_t)p * half + l) * 2], s = rope_cs[((size_t)p * half + l) * 2 + 1];
        uint16_t o0, o1;
        rope_pair(sx[l], sx[l + half], c, s, &o0, &o1);
        if (isq) {
            uint16_t* dst = qout + ((size_t)t * nq + h) * hd;
            dst[l] = o0, dst[l + half] = o1;
        } else {
            uint16_t* dst = kcache + (((size_t)s_id * nkv + hh) * max_seq + p) * hd;
            dst[l] = o0, dst[l + half] = o1;
        }
    }
    if (!isq && l < hd) {  // v: the projection rounded to bf16, no norm, no rotation
        const float* vs = qkv + (size_t)t * width + (size_t)(nq + nkv) * hd + (size_t)hh * hd;
        vcache[(((size_t)s_id * nkv + hh) * max_seq + p) * hd + l] = f2bf(vs[l]);
    }
}

// Single-query GQA attention (sdpa_decode.metal:14-48) of token t, head h over
// its sequence's cache positions 0 .. pos[t]: scores s_j = (q . k_j) / sqrt(hd)
// (one warp per key, lanes over head_dim, fixed tree), m = max s, p_j =
// exp(s_j - m), out = (sum_j p_j v_j) / (sum_j p_j).  grid (T, nq), 128 threads;
// scores in shared memory (max_seq floats).
__global__ void __launch_bounds__(kAttnThreads) k_sdpa(const uint16_t* q, const uint16_t* kc,
                                                       const uint16_t* vc, int nq, int nkv, int hd,
                                                       int max_seq, int n_seqs, float scale,
                                                       const int32_t* seq,
                                                       const int32_t* pos, uint16_t* __restrict__ out) {
    pdl_begin();
    extern __shared__ float s_sc[];  // [max_seq]
    __shared__ float s_q[128];
    __shared__ float s_red[kAttnThreads / 32];
    const int t = blockIdx.x, h = blockIdx.y, l = threadIdx.x, lane = l & 31, warp = l >> 5;
    const int s_id = seq[t], p = pos[t], kvh = h / (nq / nkv);
    if (s_id < 0 || s_id >= n_seqs || p < 0 || p >= max_seq) return;  // flagged by k_qk_norm_rope
    if (l < hd) s_q[l] = bf2f(q[((size_t)t * nq + h) * hd + l]);
    __syncthreads();
    const uint16_t* kbase = kc + ((size_t)s_id * nkv + kvh) * max_seq * hd;
    const uint16_t* vbase = vc + ((size_t)s_id * nkv + kvh) * max_seq * hd;
    const int n = p + 1;
    for (int j = warp; j < n; j += kAttnThreads / 32) {
        const uint16_t* kr = kbase + (size_t)j * hd;
        float a = 0.0f;
        for (int d = lane; d < hd; d += 32) a = __fmaf_rn(s_q[d], bf2f(kr[d]), a);
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
        if (lane == 0) s_sc[j] = __fmul_rn(a, scale);
    }
    __syncthreads();
    float m = -INFINITY;
    for (int j = l; j < n; j += kAttnThreads) m = fmaxf(m, s_sc[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) s_red[warp] = m;
    __syncthreads();
    m = s_red[0];
    for (int w = 1; w < kAttnThreads / 32; ++w) m = fmaxf(m, s_red[w]);
    __syncthreads();
    float sum = 0.0f;
    for (int j = l; j < n; j += kAttnThreads) {
        const float e = expf(s_sc[j] - m);
        s_sc[j] = e;
        sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) s_red[warp] = sum;
    __syncthreads();
    sum = 0.0f;
    for (int w = 0; w < kAttnThreads / 32; ++w) sum += s_red[w];
    if (l < hd) {
        float acc = 0.0f;
        for (int j = 0; j < n; ++j) acc = __fmaf_rn(s_sc[j], bf2f(vbase[(size_t)j * hd + l]), acc);
        out[((size_t)t * nq + h) * hd + l] = f2bf(__fdiv_rn(acc, sum));
    }
}

// x1 = x + bf16(o): the o projection rounded to bf16, the residual add in fp32, one rounding
__global__ void k_residual_add(const uint16_t* x, const float* o, size_t n,
                               uint16_t* __restrict__ out) {
    pdl_begin();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = f2bf(__fadd_rn(bf2f(x[i]), bf2f(f2bf(o[i]))));
}

}  // namespace

cudaError_t launch_qk_norm_rope(const float* qkv, int T, int nq, int nkv, int hd, const uint16_t* qn,
                                const uint16_t* kn, float eps, const float* rope_cs, int max_seq, const int32_t* seq,
                                const int32_t* pos, uint16_t* qout, uint16_t* kcache, uint16_t* vcache, int n_seqs,
                                int* err, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (hd > 128 || hd % 2) return cudaErrorInvalidValue;
    const cudaError_t e = launch_pdl(k_qk_norm_rope, dim3(T, nq + nkv), dim3(kAttnThreads), 0, st, qkv, T, nq, nkv,
                                     hd, qn, kn, eps, rope_cs, max_seq, seq, pos, qout, kcache, vcache, n_seqs, err);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

cudaError_t launch_sdpa(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, int T, int nq, int nkv, int hd,
                        int max_seq, int n_seqs, const int32_t* seq, const int32_t* pos, uint16_t* out,
                        cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    const size_t smem = (size_t)max_seq * 4;
    cudaError_t e = cudaFuncSetAttribute(k_sdpa, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const float scale = 1.0f / sqrtf((float)hd);
    e = launch_pdl(k_sdpa, dim3(T, nq), dim3(kAttnThreads), smem, st, q, kc, vc, nq, nkv, hd, max_seq, n_seqs, scale, seq,
                   pos, out);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

cudaError_t launch_residual_add(const uint16_t* x, const float* o, size_t n, uint16_t* out, cudaStream_t st) {
    if (!n) return cudaSuccess;
    const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    const cudaError_t e = launch_pdl(k_residual_add, dim3(grid), dim3(256), 0, st, x, o, n, out);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace obs
