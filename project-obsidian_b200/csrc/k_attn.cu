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

// Single-query GQA attention (sdpa_decode.metal:14-48) of token t over its
// sequence's cache positions 0 .. pos[t], split over the positions so a decode
// step fills the GPU: scores s_j = (q . k_j) / sqrt(hd), out = sum_j e^(s_j - m)
// v_j / sum_j e^(s_j - m).  k_sdpa_part: one CTA per (token, KV head, split)
// takes the split's positions for all query heads of the KV head (each K and V
// row is read once for the group), 128 positions at a time (one per thread: its
// K row against every head's q, fp32, dimensions in order), with a running
// maximum and sum per head (the online softmax) and each thread accumulating one
// dimension of every head's sum p_j v_j; it leaves (m, l, acc) per (token, head,
// split).  k_sdpa_merge: one CTA per (token, head) rescales the splits to the
// common maximum and divides.  Against the reference's single pass this changes
// only the order of the fp32 sums and the rescalings.
constexpr int kSdpaTile = 128;      // cache positions per pass of a CTA, one per thread
constexpr int kSdpaMaxGroup = 8;    // query heads per KV head (one CTA takes them all)
constexpr int kSdpaMaxSplits = 32;  // position splits per (token, KV head)

__global__ void __launch_bounds__(kSdpaTile) k_sdpa_part(const uint16_t* q, const uint16_t* kc, const uint16_t* vc,
                                                         int nq, int nkv, int hd, int max_seq, int n_seqs,
                                                         float scale, const int32_t* seq, const int32_t* pos,
                                                         float* __restrict__ part_acc, float* __restrict__ part_ml) {
    pdl_begin();
    __shared__ float s_q[kSdpaMaxGroup][128];
    __shared__ float s_p[kSdpaMaxGroup][kSdpaTile];
    __shared__ float s_m[kSdpaMaxGroup], s_l[kSdpaMaxGroup], s_corr[kSdpaMaxGroup];
    const int t = blockIdx.x, kvh = blockIdx.y, sp = blockIdx.z, S = gridDim.z;
    const int G = nq / nkv, l = threadIdx.x, lane = l & 31, warp = l >> 5;
    const int s_id = seq[t], p = pos[t];
    if (s_id < 0 || s_id >= n_seqs || p < 0 || p >= max_seq) return;  // refused and recorded by k_qk_norm_rope
    const int n = p + 1, chunk = (n + S - 1) / S, js = sp * chunk, je = min(n, js + chunk);
    if (js >= je) return;  // no positions in this split: the merge reads only the splits that have some
    for (int i = l; i < G * hd; i += kSdpaTile) s_q[i / hd][i % hd] = bf2f(q[((size_t)t * nq + kvh * G) * hd + i]);
    if (l < kSdpaMaxGroup) s_m[l] = -INFINITY, s_l[l] = 0.0f;
    const uint16_t* kbase = kc + ((size_t)s_id * nkv + kvh) * max_seq * hd;
    const uint16_t* vbase = vc + ((size_t)s_id * nkv + kvh) * max_seq * hd;
    float acc[kSdpaMaxGroup];
#pragma unroll
    for (int h = 0; h < kSdpaMaxGroup; ++h) acc[h] = 0.0f;
    __syncthreads();
    for (int j0 = js; j0 < je; j0 += kSdpaTile) {
        const int j = j0 + l, len = min(kSdpaTile, je - j0);
        // scores of position j against every head of the group
        float sc[kSdpaMaxGroup];
#pragma unroll
        for (int h = 0; h < kSdpaMaxGroup; ++h) sc[h] = 0.0f;
        if (l < len) {
            const uint4* kr = reinterpret_cast<const uint4*>(kbase + (size_t)j * hd);
            for (int c = 0; c < hd / 8; ++c) {
                const uint4 v = kr[c];
                const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float k0 = __uint_as_float(w4[e] << 16), k1 = __uint_as_float(w4[e] & 0xFFFF0000u);
#pragma unroll
                    for (int h = 0; h < kSdpaMaxGroup; ++h)
                        if (h < G) sc[h] = __fmaf_rn(s_q[h][8 * c + 2 * e + 1], k1, __fmaf_rn(s_q[h][8 * c + 2 * e], k0, sc[h]));
                }
            }
        }
#pragma unroll
        for (int h = 0; h < kSdpaMaxGroup; ++h)
            if (h < G) s_p[h][l] = l < len ? __fmul_rn(sc[h], scale) : -INFINITY;
        __syncthreads();
        // per head (warp w takes heads w, w + 4): the tile's maximum, the new running maximum,
        // the probabilities, the rescaling of what came before and the running sum
        for (int h = warp; h < G; h += kSdpaTile / 32) {
            float mt = -INFINITY;
            for (int x = lane; x < len; x += 32) mt = fmaxf(mt, s_p[h][x]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
            const float m_old = s_m[h], m_new = fmaxf(m_old, mt);
            float sum = 0.0f;
            for (int x = lane; x < len; x += 32) {
                const float e = expf(s_p[h][x] - m_new);
                s_p[h][x] = e;
                sum += e;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            __syncwarp();
            if (lane == 0) {
                const float corr = expf(m_old - m_new);  // 0 for the first tile (m_old = -inf)
                s_corr[h] = corr;
                s_m[h] = m_new;
                s_l[h] = __fmaf_rn(s_l[h], corr, sum);
            }
        }
        __syncthreads();
        // dimension l of every head: rescale, then add the tile's p_j v_j
        if (l < hd) {
#pragma unroll
            for (int h = 0; h < kSdpaMaxGroup; ++h)
                if (h < G) acc[h] = __fmul_rn(acc[h], s_corr[h]);
            for (int x = 0; x < len; ++x) {
                const float v = bf2f(vbase[(size_t)(j0 + x) * hd + l]);
#pragma unroll
                for (int h = 0; h < kSdpaMaxGroup; ++h)
                    if (h < G) acc[h] = __fmaf_rn(s_p[h][x], v, acc[h]);
            }
        }
        __syncthreads();  // s_p is rewritten by the next tile
    }
    const size_t row0 = ((size_t)t * nq + kvh * G) * S + sp;  // (token, first head of the group, split)
    if (l < hd) {
#pragma unroll
        for (int h = 0; h < kSdpaMaxGroup; ++h)
            if (h < G) part_acc[(row0 + (size_t)h * S) * hd + l] = acc[h];
    }
    if (l < G) {
        part_ml[(row0 + (size_t)l * S) * 2] = s_m[l];
        part_ml[(row0 + (size_t)l * S) * 2 + 1] = s_l[l];
    }
}

__global__ void __launch_bounds__(kAttnThreads) k_sdpa_merge(const float* part_acc, const float* part_ml, int S,
                                                             int nq, int hd, int max_seq, int n_seqs,
                                                             const int32_t* seq, const int32_t* pos,
                                                             uint16_t* __restrict__ out) {
    pdl_begin();
    const int t = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
    const int s_id = seq[t], p = pos[t];
    if (s_id < 0 || s_id >= n_seqs || p < 0 || p >= max_seq) return;
    const int n = p + 1, chunk = (n + S - 1) / S, used = (n + chunk - 1) / chunk;
    const size_t row0 = ((size_t)t * nq + h) * S;
    float M = -INFINITY;
    for (int s = 0; s < used; ++s) M = fmaxf(M, part_ml[(row0 + s) * 2]);
    float L = 0.0f, a = 0.0f;
    for (int s = 0; s < used; ++s) {
        const float w = expf(part_ml[(row0 + s) * 2] - M);
        L = __fmaf_rn(w, part_ml[(row0 + s) * 2 + 1], L);
        if (d < hd) a = __fmaf_rn(w, part_acc[(row0 + s) * hd + d], a);
    }
    if (d < hd) out[((size_t)t * nq + h) * hd + d] = f2bf(__fdiv_rn(a, L));
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

int sdpa_splits(int T, int nkv, int num_sms) {
    const int want = (4 * num_sms + T * nkv - 1) / (T * nkv);
    return want < 1 ? 1 : want > kSdpaMaxSplits ? kSdpaMaxSplits : want;
}

size_t sdpa_part_floats(int max_tokens, int nq, int nkv, int hd, int num_sms) {
    size_t rows = 0;  // the largest T * splits of any launch
    for (int T = 1; T <= max_tokens; ++T) {
        const size_t r = (size_t)T * sdpa_splits(T, nkv, num_sms);
        if (r > rows) rows = r;
    }
    return rows * nq * (hd + 2);
}

cudaError_t launch_sdpa(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, int T, int nq, int nkv, int hd,
                        int max_seq, int n_seqs, const int32_t* seq, const int32_t* pos, uint16_t* out, float* part,
                        int num_sms, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (hd > 128 || hd % 8 || nq % nkv || nq / nkv > kSdpaMaxGroup) return cudaErrorInvalidValue;
    const int S = sdpa_splits(T, nkv, num_sms);
    float* part_acc = part;
    float* part_ml = part + (size_t)T * nq * S * hd;
    const float scale = 1.0f / sqrtf((float)hd);
    cudaError_t e = launch_pdl(k_sdpa_part, dim3(T, nkv, S), dim3(kSdpaTile), 0, st, q, kc, vc, nq, nkv, hd, max_seq,
                               n_seqs, scale, seq, pos, part_acc, part_ml);
    if (e != cudaSuccess) return e;
    e = launch_pdl(k_sdpa_merge, dim3(T, nq), dim3(kAttnThreads), 0, st, (const float*)part_acc,
                   (const float*)part_ml, S, nq, hd, max_seq, n_seqs, seq, pos, out);
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
