// k_decode.cu -- decode expert FFN: fused 4-bit dequant mat-vec on CUDA cores.
//
// Replaces the reference's per-rank loop of fused_dequant_matvec_4bit x3 +
// ew_swiglu + ew_scaled_add (src/forward.rs:431-441; shaders/
// fused_dequant_matvec_4bit.metal:14-53, ops.metal:18-29).  Weights are read
// once, coalesced, 128 rows x 64 columns at a time, all of a warp's loads in
// flight together.  The group's affine dequantisation is factored out of the
// inner loop: over one 64-column group, sum_j (q_j s + b) x_j =
// 16 s (sum_j f_j x_j - sum_j x_j) + b sum_j x_j with f_j = 1 + q_j/16, a float
// built from the code with one shift and one logic op; per weight that is a
// shift, a logic op and one fp32 FMA.  Split-K partial sums meet in a fixed
// order in the last CTA to finish (a per-tile arrival counter that resets
// itself), so results do not depend on CTA scheduling.
//
// The kernels read either the context's tiled 4608-byte blocks or the
// reference's MLX row-major layout directly.
#include "router_dev.cuh"

namespace obs {
namespace {

constexpr int kSplitGU = kDecodeSplit;  // k-splits of the gate/up mat-vec (one 64-column block per warp)

// 1 + q/16 as a float, q the 4-bit code at nibble j: the code becomes mantissa bits 19-22
__device__ __forceinline__ float nib_f16th(uint32_t w, int j) {
    const uint32_t m = (4 * j <= 19) ? (w << (19 - 4 * j)) : (w >> (4 * j - 19));
    return __uint_as_float((m & 0x00780000u) | 0x3F800000u);
}

// Weight sources: 128 rows x 64 columns of one block of one expert.
// Lane l covers rows (l>>1) + 16 i (i < 8) and the 32 columns of half (l & 1).
// The context's gate/up array is paired: the 128 features of gate/up row tile rt
// are blocks 2rt and 2rt+1, and feature c of block h sits in row paired_row(c)
// (gate) and paired_row(c) + 16 (up).  Each row's dot product is the same
// arithmetic whichever block it sits in; only the final pairing re-indexes.
__device__ __forceinline__ int paired_row(int c) { return 32 * (c >> 4) + (c & 15); }
struct TiledSrc {  // the context's blocks; nibble order c0,c2,c4,c6,c1,c3,c5,c7
    const uint8_t* base;
    int n_rt, KT, stride, off;  // block (e, rt, kt) = base + (((e*n_rt + rt)*KT + kt)*stride + off) * 4608
    static constexpr bool kNatural = false;
    __device__ __forceinline__ void load(int e, int rt, int kt, int lane, uint4 (&q)[8], float (&sc)[8],
                                         float (&bi)[8]) const {
        const uint8_t* blk = base + ((((size_t)e * n_rt + rt) * KT + kt) * stride + off) * kBlockBytes;
        const uint4* wq = reinterpret_cast<const uint4*>(blk + (lane & 1) * 2048);
        const uint16_t* sb = reinterpret_cast<const uint16_t*>(blk + kBlockWords * 4);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int row = (lane >> 1) + 16 * i;
            q[i] = __ldg(wq + row);
            sc[i] = bf2f(__ldg(sb + row));
            bi[i] = bf2f(__ldg(sb + kRowTile + row));
        }
    }
};
struct MlxSrc {  // reference layout: w [E, out, in/8] (column c at nibble c), s/b [E, out, in/64]
    const uint32_t* w;
    const uint16_t* s;
    const uint16_t* b;
    int out_f, in_f;
    static constexpr bool kNatural = true;
    __device__ __forceinline__ void load(int e, int rt, int kt, int lane, uint4 (&q)[8], float (&sc)[8],
                                         float (&bi)[8]) const {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const size_t row = (size_t)e * out_f + rt * kRowTile + (lane >> 1) + 16 * i;
            q[i] = __ldg(reinterpret_cast<const uint4*>(w + row * (in_f / 8) + kt * 8 + (lane & 1) * 4));
            sc[i] = bf2f(__ldg(s + row * (in_f / kGroup) + kt));
            bi[i] = bf2f(__ldg(b + row * (in_f / kGroup) + kt));
        }
    }
};

template <class Src>
__device__ __forceinline__ void block_dot(const Src& src, int e, int rt, int kt, const float (&xr)[32], float xsum,
                                          int lane, float (&acc)[8]) {
    uint4 q[8];
    float sc[8], bi[8];
    src.load(e, rt, kt, lane, q, sc, bi);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t ws[4] = {q[i].x, q[i].y, q[i].z, q[i].w};
        float f = 0.0f;  // sum_j (1 + q_j/16) x_j over the lane's 32 columns
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                // columns in the order (0,2,4,6,1,3,5,7) of every word for both layouts, so
                // the two give bit-identical sums: the tiled word holds that column at nibble j,
                // the MLX word at nibble nib_col(j)
                const int col = nib_col(j);
                f = __fmaf_rn(nib_f16th(ws[c], Src::kNatural ? col : j), xr[c * 8 + col], f);
            }
        // s * sum q x + b * sum x, with sum q x = 16 (f - sum x)
        acc[i] = __fmaf_rn(16.0f * sc[i], f - xsum, __fmaf_rn(bi[i], xsum, acc[i]));
    }
}

__device__ __forceinline__ float load_x32(const uint16_t* __restrict__ x, float (&xr)[32]) {
    const uint4* p = reinterpret_cast<const uint4*>(x);
    float sum = 0.0f;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
        uint4 q = __ldg(p + v);
        uint32_t qs[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            xr[v * 8 + 2 * c] = __uint_as_float(qs[c] << 16);
            xr[v * 8 + 2 * c + 1] = __uint_as_float(qs[c] & 0xFFFF0000u);
            sum += xr[v * 8 + 2 * c] + xr[v * 8 + 2 * c + 1];
        }
    }
    return sum;
}

// An out-of-range expert id is reported and replaced by 0, so every CTA still
// takes part in its tile's arrival count and no weight outside the layer is read.
__device__ __forceinline__ int checked_expert(int e, int E, int* err) {
    if (e >= 0 && e < E) return e;
    if (threadIdx.x == 0) atomicExch(err, kDevBadRoute);
    return 0;
}

// grid (I/128, kSplitGU, T*K), 256 threads.  warp w: projection w & 1,
// k-tiles kt0 + (w >> 1) + 4 j (one block per warp for H = 2048).
template <class Src>
__global__ void __launch_bounds__(256) k_decode_gateup(Src gsrc, Src usrc, const uint16_t* __restrict__ x,
                                                       const int32_t* __restrict__ ids, int H, int I, int K, int E,
                                                       DecodeBufs d) {
    pdl_begin();
    __shared__ float s_part[8][kRowTile];
    __shared__ float s_gu[2][kRowTile];
    __shared__ int s_last;
    const int rt = blockIdx.x, ks = blockIdx.y, p = blockIdx.z;
    const int n_rt = gridDim.x, KT = H / kGroup, nkt = KT / kSplitGU;
    const int t = p / K, e = checked_expert(ids[p], E, d.err);
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, proj = w & 1;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j = (w >> 1); j < nkt; j += 4) {
        const int kt = ks * nkt + j;
        float xr[32];
        const float xs = load_x32(x + (size_t)t * H + kt * kGroup + (lane & 1) * 32, xr);
        block_dot(proj ? usrc : gsrc, e, Src::kNatural ? rt : 2 * rt + proj, kt, xr, xs, lane, acc);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float v = acc[i] + __shfl_xor_sync(0xffffffffu, acc[i], 1);
        if ((lane & 1) == 0) s_part[w][(lane >> 1) + 16 * i] = v;
    }
    __syncthreads();
    // fixed-order sum of the 4 warps of each projection (paired blocks: of each block)
    const int pr = tid >> 7, row = tid & 127;
    const float v = ((s_part[pr][row] + s_part[pr + 2][row]) + s_part[pr + 4][row]) + s_part[pr + 6][row];
    float* part = d.part + (((size_t)p * n_rt + rt) * kSplitGU) * 2 * kRowTile;
    part[(size_t)ks * 2 * kRowTile + pr * kRowTile + row] = v;
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        uint32_t* c = d.cnt_gu + (size_t)p * n_rt + rt;
        unsigned old = atomicAdd(c, 1u);
        s_last = (old == kSplitGU - 1);
        if (s_last) *c = 0;  // ready for the next call
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < kSplitGU; ++j) sum += __ldcg(part + (size_t)j * 2 * kRowTile + pr * kRowTile + row);
    s_gu[pr][row] = sum;
    __syncthreads();
    if (tid < kRowTile) {
        float g, u;
        if constexpr (Src::kNatural) {
            g = s_gu[0][tid], u = s_gu[1][tid];
        } else {
            const int rr = paired_row(tid & 63);  // block 2rt + tid/64 holds feature tid
            g = s_gu[tid >> 6][rr], u = s_gu[tid >> 6][rr + 16];
        }
        d.h[(size_t)p * I + rt * kRowTile + tid] = f2bf(silu_mul(g, u));
    }
}

// grid (H/128, K, T), 32 * min(I/64, 16) threads.  warp w: k-tiles w, w + nwarps, ...
template <class Src>
__global__ void __launch_bounds__(512) k_decode_down(Src dsrc, const int32_t* __restrict__ ids,
                                                     const float* __restrict__ wts,
                                                     const uint16_t* __restrict__ residual, int H, int I, int K,
                                                     int E, DecodeBufs d, uint16_t* __restrict__ out,
                                                     int do_combine) {
    pdl_begin();
    __shared__ float s_part[16][kRowTile];
    __shared__ int s_last;
    const int rt = blockIdx.x, k = blockIdx.y, t = blockIdx.z;
    const int n_rt = gridDim.x, KT = I / kGroup, nwarps = blockDim.x >> 5;
    const int p = t * K + k, e = checked_expert(ids[p], E, d.err);
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int kt = w; kt < KT; kt += nwarps) {
        float xr[32];
        const float xs = load_x32(d.h + (size_t)p * I + kt * kGroup + (lane & 1) * 32, xr);
        block_dot(dsrc, e, rt, kt, xr, xs, lane, acc);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float v = acc[i] + __shfl_xor_sync(0xffffffffu, acc[i], 1);
        if ((lane & 1) == 0) s_part[w][(lane >> 1) + 16 * i] = v;
    }
    __syncthreads();
    for (int r = tid; r < kRowTile; r += blockDim.x) {  // blockDim may be below 128 (inter = 128)
        float v = 0.0f;
        for (int j = 0; j < nwarps; ++j) v += s_part[j][r];
        d.y[(size_t)p * H + rt * kRowTile + r] = f2bf(v);
    }
    if (!do_combine) return;
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        uint32_t* c = d.cnt_dn + (size_t)t * n_rt + rt;
        unsigned old = atomicAdd(c, 1u);
        s_last = (old == (unsigned)K - 1);
        if (s_last) *c = 0;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int r = tid; r < kRowTile; r += blockDim.x) {
        // rank-order combine, same operation order as k_combine (forward.rs:225-232)
        const int f = rt * kRowTile + r;
        float a = residual ? bf2f(residual[(size_t)t * H + f]) : 0.0f;
        for (int j = 0; j < K; ++j) {
            const uint16_t yv = __ldcg(d.y + ((size_t)t * K + j) * H + f);
            a = __fmaf_rn(wts[(size_t)t * K + j], bf2f(yv), a);
        }
        out[(size_t)t * H + f] = f2bf(a);
    }
}

int down_threads(int I) { return 32 * (I / kGroup < 16 ? I / kGroup : 16); }

// ----------------------------------------------------------- fused decode layer
// One cooperative launch runs the whole decode layer for T <= 4 tokens, so the
// step pays one launch instead of four dependent ones.  One CTA of 16 warps per
// SM; work units go round-robin over the CTAs first, so every SM works.
//   A  router logits: one warp per (expert, 8-token chunk), canonical order;
//      grid barrier;
//   B  top-k: every CTA computes the routes of all T tokens itself (identical,
//      deterministic), so no barrier follows;
//   C  gate/up: each half-CTA (8 warps) runs one CTA of k_decode_gateup -- a
//      (pair, row tile, split) unit, its shared-memory reduction, and, in the
//      last split to arrive, the split sum and SwiGLU over 256 threads;
//      grid barrier;
//   D  down: each CTA runs one CTA of k_decode_down -- a (pair, row tile) unit,
//      y, and in the last pair of a (token, row tile) the rank-order combine.
// The arithmetic is that of the separate decode kernels, term for term, so the
// two forms give identical outputs.  Barriers wait at most 2 s.
constexpr int kFusedThreads = 512, kFusedWarps = kFusedThreads / 32;

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// every CTA of the grid; false (error flag set) after a timeout.  The arrival
// counter only grows (launch n's barriers wait for (2n+1)G and (2n+2)G arrivals,
// n the generation read at the start), so no launch needs it cleared; the
// comparison is wrap-safe.
__device__ bool grid_sync(uint32_t* bar, uint32_t target, int* err, uint64_t limit_ns) {
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(bar, 1u);
        int ok = 1;
        const uint64_t t0 = global_ns();
        while ((int)(ld_acquire_gpu(bar) - target) < 0) {
            if (global_ns() - t0 > limit_ns) {
                ok = 0;
                atomicExch(err, kDevTimeout);
                break;
            }
        }
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

// load_x32 from shared memory (or any generic address)
__device__ __forceinline__ float load_x32_gen(const uint16_t* x, float (&xr)[32]) {
    const uint4* p = reinterpret_cast<const uint4*>(x);
    float sum = 0.0f;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
        uint4 q = p[v];
        uint32_t qs[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            xr[v * 8 + 2 * c] = __uint_as_float(qs[c] << 16);
            xr[v * 8 + 2 * c + 1] = __uint_as_float(qs[c] & 0xFFFF0000u);
            sum += xr[v * 8 + 2 * c] + xr[v * 8 + 2 * c + 1];
        }
    }
    return sum;
}

// load_x32 for data written earlier in this kernel (read through L2)
__device__ __forceinline__ float load_x32_cg(const uint16_t* __restrict__ x, float (&xr)[32]) {
    const uint4* p = reinterpret_cast<const uint4*>(x);
    float sum = 0.0f;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
        uint4 q = __ldcg(p + v);
        uint32_t qs[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            xr[v * 8 + 2 * c] = __uint_as_float(qs[c] << 16);
            xr[v * 8 + 2 * c + 1] = __uint_as_float(qs[c] & 0xFFFF0000u);
            sum += xr[v * 8 + 2 * c] + xr[v * 8 + 2 * c + 1];
        }
    }
    return sum;
}

__global__ void __launch_bounds__(kFusedThreads, 1) k_decode_fused(
    const uint32_t* __restrict__ rw, const uint16_t* __restrict__ rs, const uint16_t* __restrict__ rb,
    TiledSrc gsrc, TiledSrc dsrc, const uint16_t* __restrict__ x_in, const uint16_t* __restrict__ residual,
    const float* __restrict__ bias, int T, int H, int I, int E, int K, int norm, int normalize, float eps,
    FusedDecodeBufs f, uint16_t* __restrict__ out) {
    extern __shared__ __align__(16) uint16_t s_x[];  // [T][H] the layer input, this CTA's copy
    __shared__ float s_sq[2][256];
    __shared__ int s_ids[kFusedMaxT * kMaxK];
    __shared__ float s_wts[kFusedMaxT * kMaxK];
    __shared__ float s_part[kFusedWarps][kRowTile];  // C: [half][8 warps]; D: [16 warps]
    __shared__ int s_last[1];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, b = blockIdx.x;
    // phase timeline (diagnostics): start, A done, barrier 1, B done, C done, barrier 2, D done
    auto mark = [&](int k) {
        if (f.trace && tid == 0) f.trace[8 * b + k] = global_ns();
    };
    mark(0);
    // barrier generation of this launch (advanced by CTA 0 after the last barrier)
    const uint32_t gen = *reinterpret_cast<volatile uint32_t*>(f.bar + 1);

    // 0: the layer input into shared memory; with `normalize`, the MoE input
    // RMSNorm of rmsnorm.metal:9-37 in k_rmsnorm's order (256 threads per row,
    // strided rounded squares, halving tree, IEEE divide and square root)
    for (int t0 = 0; t0 < T; t0 += 2) {
        const int t = t0 + (tid >> 8), l = tid & 255;
        const uint16_t* row = x_in + (size_t)t * H;
        if (normalize) {
            float ps = 0.0f;
            if (t < T)
                for (int i = l; i < H; i += 256) {
                    const float v = bf2f(row[i]);
                    ps = __fadd_rn(ps, __fmul_rn(v, v));
                }
            s_sq[tid >> 8][l] = ps;
            __syncthreads();
            for (int st = 128; st > 0; st >>= 1) {
                if (l < st) s_sq[tid >> 8][l] = __fadd_rn(s_sq[tid >> 8][l], s_sq[tid >> 8][l + st]);
                __syncthreads();
            }
            if (t < T) {
                const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(s_sq[tid >> 8][0], (float)H), eps));
                for (int i = l; i < H; i += 256) s_x[(size_t)t * H + i] = f2bf(__fdiv_rn(bf2f(row[i]), rms));
            }
            __syncthreads();
        } else if (t < T) {
            for (int i = l * 8; i < H; i += 256 * 8)
                *reinterpret_cast<uint4*>(s_x + (size_t)t * H + i) = __ldg(reinterpret_cast<const uint4*>(row + i));
        }
    }
    __syncthreads();
    const uint16_t* x = s_x;

    // A: router logits; item i on warp i / G of CTA i % G
    const int n_tc = (T + kWarpTok - 1) / kWarpTok;
    for (int item = warp * G + b; item < E * n_tc; item += kFusedWarps * G)
        router_warp_item<true>(rw, rs, rb, x, T, H, E, item % E, (item / E) * kWarpTok, lane, f.logits);
    mark(1);
    if (!grid_sync(f.bar, (2 * gen + 1) * G, f.err, f.wait_ns)) return;
    mark(2);

    // B: top-k of every token, in every CTA
    if (warp < T) {
        const int t = warp;
        auto logit = [&](int e) { return __ldcg(f.logits + (size_t)t * E + e); };
        int ik;
        float wk;
        topk_token(logit, bias, E, K, norm, lane, &ik, &wk);
        if (lane < K) {
            s_ids[t * K + lane] = ik;
            s_wts[t * K + lane] = wk;
            if (b == 0) f.ids[t * K + lane] = ik, f.wts[t * K + lane] = wk;
        }
    }
    __syncthreads();
    mark(3);

    // C: gate/up -- half-CTA h takes units (pair p, row tile rt, split ks) like one
    // CTA of k_decode_gateup: warp w8 = block half (w8 & 1) of paired blocks
    // 2rt, 2rt+1, k-tiles ks*nkt + (w8 >> 1) + 4j
    {
        const int h = warp >> 3, w8 = warp & 7, t256 = tid & 255, half = w8 & 1;
        const int n_rt = I / kRowTile, KT = H / kGroup, nkt = KT / kSplitGU, n_pairs = T * K;
        const int units = n_pairs * n_rt * kSplitGU;
        float* part = f.part_gu;  // [p][rt][ks][2][128]
        for (int u = h * G + b; u < units; u += 2 * G) {
            const int ks = u % kSplitGU, rt = (u / kSplitGU) % n_rt, p = u / (kSplitGU * n_rt);
            const int t = p / K, e = checked_expert(s_ids[p], E, f.err);
            float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int j = (w8 >> 1); j < nkt; j += 4) {
                const int kt = ks * nkt + j;
                float xr[32];
                const float xs = load_x32_gen(x + (size_t)t * H + kt * kGroup + (lane & 1) * 32, xr);
                block_dot(gsrc, e, 2 * rt + half, kt, xr, xs, lane, acc);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float v = acc[i] + __shfl_xor_sync(0xffffffffu, acc[i], 1);
                if ((lane & 1) == 0) s_part[h * 8 + w8][(lane >> 1) + 16 * i] = v;
            }
            named_bar_sync(1 + h, 256);
            // fixed-order sum of the 4 warps of each block; the split partials meet in
            // phase D, after the grid barrier has published them
            const int pr = t256 >> 7, row = t256 & 127;
            const float* sp = &s_part[h * 8][0];
            const float v = ((sp[pr * kRowTile + row] + sp[(pr + 2) * kRowTile + row]) + sp[(pr + 4) * kRowTile + row]) +
                            sp[(pr + 6) * kRowTile + row];
            float* tp = part + (((size_t)p * n_rt + rt) * kSplitGU) * 2 * kRowTile;
            tp[(size_t)ks * 2 * kRowTile + pr * kRowTile + row] = v;
            named_bar_sync(1 + h, 256);  // s_part free for the next unit
        }
    }
    mark(4);
    if (!grid_sync(f.bar, (2 * gen + 2) * G, f.err, f.wait_ns)) return;
    mark(5);
    // every CTA read `gen` before the first barrier: the next launch may use the next one
    if (b == 0 && tid == 0) *reinterpret_cast<volatile uint32_t*>(f.bar + 1) = gen + 1;

    // D: down -- CTA units (pair p, row tile rt) like one CTA of k_decode_down
    {
        const int n_rd = H / kRowTile, KTd = I / kGroup, nwd = KTd < 16 ? KTd : 16, n_pairs = T * K;
        const int n_rt = I / kRowTile;
        uint16_t* s_h = s_x + (size_t)T * H;  // [I] this unit's SwiGLU input row, bf16
        int p_h = -1;                          // the pair s_h holds
        for (int u = b; u < n_pairs * n_rd; u += G) {
            const int rt = u % n_rd, p = u / n_rd, t = p / K;
            const int e = checked_expert(s_ids[p], E, f.err);
            if (p != p_h) {
                // h of pair p: gate and up summed over the k-splits in split order, then
                // SwiGLU (the last-split step of k_decode_gateup, term for term)
                for (int i = tid; i < I; i += kFusedThreads) {
                    const int rg = i / kRowTile, tt = i % kRowTile, pr = tt >> 6, rr = paired_row(tt & 63);
                    const float* tp = f.part_gu + (((size_t)p * n_rt + rg) * kSplitGU) * 2 * kRowTile + pr * kRowTile;
                    float g = 0.0f, uu = 0.0f;
#pragma unroll
                    for (int jj = 0; jj < kSplitGU; ++jj) {
                        g += __ldcg(tp + (size_t)jj * 2 * kRowTile + rr);
                        uu += __ldcg(tp + (size_t)jj * 2 * kRowTile + rr + 16);
                    }
                    s_h[i] = f2bf(silu_mul(g, uu));
                }
                __syncthreads();
                p_h = p;
            }
            if (warp < nwd) {
                float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                for (int kt = warp; kt < KTd; kt += nwd) {
                    float xr[32];
                    const float xs = load_x32_gen(s_h + kt * kGroup + (lane & 1) * 32, xr);
                    block_dot(dsrc, e, rt, kt, xr, xs, lane, acc);
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float v = acc[i] + __shfl_xor_sync(0xffffffffu, acc[i], 1);
                    if ((lane & 1) == 0) s_part[warp][(lane >> 1) + 16 * i] = v;
                }
            }
            __syncthreads();
            if (tid < kRowTile) {
                float v = 0.0f;
                for (int j = 0; j < nwd; ++j) v += s_part[j][tid];
                f.y[(size_t)p * H + rt * kRowTile + tid] = f2bf(v);
            }
            __threadfence();
            __syncthreads();
            if (tid == 0) {
                uint32_t* c = f.cnt_dn + (size_t)t * n_rd + rt;
                const unsigned old = atomicAdd(c, 1u);
                s_last[0] = (old == (unsigned)K - 1);
                if (s_last[0]) *c = 0;
            }
            __syncthreads();
            if (s_last[0]) {
                __threadfence();
                if (tid < kRowTile) {
                    // rank-order combine, same operation order as k_combine (forward.rs:225-232)
                    const int fo = rt * kRowTile + tid;
                    float a = residual ? bf2f(residual[(size_t)t * H + fo]) : 0.0f;
                    for (int jk = 0; jk < K; ++jk) {
                        const uint16_t yv = __ldcg(f.y + ((size_t)t * K + jk) * H + fo);
                        a = __fmaf_rn(s_wts[t * K + jk], bf2f(yv), a);
                    }
                    out[(size_t)t * H + fo] = f2bf(a);
                }
            }
            __syncthreads();  // s_part / s_last free for the next unit
        }
    }
    mark(6);
}

}  // namespace

cudaError_t launch_decode_gateup(const LayerDev& L, const Shape& sh, const uint16_t* x, const int32_t* ids, int T,
                                 const DecodeBufs& d, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    const TiledSrc g{L.gateup, sh.I / 64, sh.H / kGroup, 1, 0}, u = g;  // paired blocks
    dim3 grid(sh.I / kRowTile, kSplitGU, T * sh.K);
    {
        const cudaError_t le_ = launch_pdl(k_decode_gateup<TiledSrc>, dim3(grid), dim3(256), 0, st, g, u, x, ids, sh.H, sh.I, sh.K, sh.E, d);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

cudaError_t launch_decode_down(const LayerDev& L, const Shape& sh, const int32_t* ids, const float* w,
                               const uint16_t* residual, int T, const DecodeBufs& d, uint16_t* out, int do_combine,
                               cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    const TiledSrc dn{L.down, sh.H / kRowTile, sh.I / kGroup, 1, 0};
    dim3 grid(sh.H / kRowTile, sh.K, T);
    {
        const cudaError_t le_ = launch_pdl(k_decode_down<TiledSrc>, dim3(grid), dim3(down_threads(sh.I)), 0, st, dn, ids, w, residual, sh.H, sh.I, sh.K, sh.E, d, out,
                                                                 do_combine);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

cudaError_t launch_decode_fused(const LayerDev& L, const Shape& sh, const uint16_t* x, const uint16_t* residual,
                                const float* bias, int T, int norm, int normalize, float eps,
                                const FusedDecodeBufs& f, uint16_t* out, int num_sms, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (T > kFusedMaxT || sh.K > kMaxK || sh.E > kMaxE || sh.H % 2048) return cudaErrorInvalidValue;
    const TiledSrc g{L.gateup, sh.I / 64, sh.H / kGroup, 1, 0};  // paired blocks
    const TiledSrc dn{L.down, sh.H / kRowTile, sh.I / kGroup, 1, 0};
    const size_t smem = (size_t)T * sh.H * 2 + (size_t)sh.I * 2;  // the layer input rows, one SwiGLU row
    cudaError_t e = cudaFuncSetAttribute(k_decode_fused, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms);  // one CTA per SM: every CTA is resident (cooperative)
    cfg.blockDim = dim3(kFusedThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    note_launch();
    return cudaLaunchKernelEx(&cfg, k_decode_fused, L.router_w, L.router_s, L.router_b, g, dn, x, residual, bias, T,
                              sh.H, sh.I, sh.E, sh.K, norm, normalize, eps, f, out);
}

cudaError_t launch_decode_ffn_mlx(const uint32_t* gw, const uint16_t* gs, const uint16_t* gb, const uint32_t* uw,
                                  const uint16_t* us, const uint16_t* ub, const uint32_t* dw, const uint16_t* ds,
                                  const uint16_t* db, const Shape& sh, const uint16_t* x, const int32_t* ids,
                                  const float* w, const uint16_t* residual, int T, const DecodeBufs& d, uint16_t* out,
                                  cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    const MlxSrc g{gw, gs, gb, sh.I, sh.H}, u{uw, us, ub, sh.I, sh.H}, dn{dw, ds, db, sh.H, sh.I};
    dim3 g1(sh.I / kRowTile, kSplitGU, T * sh.K);
    {
        const cudaError_t le_ = launch_pdl(k_decode_gateup<MlxSrc>, dim3(g1), dim3(256), 0, st, g, u, x, ids, sh.H, sh.I, sh.K, sh.E, d);
        if (le_ != cudaSuccess) return le_;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    dim3 g2(sh.H / kRowTile, sh.K, T);
    {
        const cudaError_t le_ = launch_pdl(k_decode_down<MlxSrc>, dim3(g2), dim3(down_threads(sh.I)), 0, st, dn, ids, w, residual, sh.H, sh.I, sh.K, sh.E, d, out, 1);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

}  // namespace obs
