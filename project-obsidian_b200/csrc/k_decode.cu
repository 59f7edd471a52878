// k_decode.cu -- decode expert FFN: 4-bit dequant mat-vec on the integer units.
//
// Replaces the reference's per-rank loop of fused_dequant_matvec_4bit x3 +
// ew_swiglu + ew_scaled_add (src/forward.rs:431-441; shaders/
// fused_dequant_matvec_4bit.metal:14-53, ops.metal:18-29).
//
// Arithmetic.  Over one 64-column group g of a weight row,
//   sum_j (q_j s + b) x_j = s * sum_j q_j x_j + b * sum_j x_j.
// The activations of the group are put in fixed point once per token: with
// e the exponent of max_j |x_j| and k = 13 - e, X_j = round(x_j 2^k) (half away
// from zero), |X_j| <= 2^14, split X_j = 256 hi_j + lo_j (hi signed 8-bit, lo
// unsigned 8-bit).  sum_j q_j X_j is then exact in int32: dp4a multiplies four
// 4-bit codes by four 8-bit limbs per instruction, and the codes need one
// logic op per four of them (w & 0x0F0F0F0F, and w & 0xF0F0F0F0 which gives
// 16 q).  Integer sums do not depend on their order, so any layout or lane
// split gives the same integer.  Per (row, group) the fp32 value is
//   P = fma(s, float(16 sum q X) * 2^-(k+4), b * (sum X) 2^-k),
// and the P of the groups are added in a fixed fp32 order (below).  The
// rounding of x to 15 significant bits (relative to the group maximum) is far
// below the bf16 rounding of the outputs.
//
// Reduction orders (the same in the separate and the fused kernels, so they
// give identical results): gate/up -- the 8 k-splits of 4 groups each: per
// split ((P0 + P1) + P2) + P3, then the splits in order from 0; down -- the
// groups in order from 0 (warp w sums its groups w, w + 16, ..., the warps in
// order).  SwiGLU rounds h to bf16; the last split of each 128-feature tile
// writes h already in fixed point for the down projection.
//
// The kernels read either the context's tiled 4608-byte blocks or the
// reference's MLX row-major layout directly (then the activations are packed
// in the MLX nibble order).
#include "router_dev.cuh"

namespace obs {
namespace {

constexpr int kSplitGU = kDecodeSplit;  // k-splits of the gate/up mat-vec

// ------------------------------------------------------------ fixed point
// exact 2^n as a float (0 below the smallest subnormal)
__device__ __forceinline__ float pow2f(int n) {
    if (n > 127) return __uint_as_float(0x7F800000u);
    if (n >= -126) return __uint_as_float((uint32_t)(n + 127) << 23);
    if (n >= -149) return __uint_as_float(1u << (n + 149));
    return 0.0f;
}
// k for a group whose largest magnitude has bf16 bits gm (sign cleared)
__device__ __forceinline__ int fx_k(uint32_t gm) {
    if (gm == 0) return 0;
    const int ef = (int)(gm >> 7) & 0xFF;
    return 13 - (ef == 0 ? -126 : ef - 127);
}
// round(x 2^k), half away from zero, for a bf16 x no larger in magnitude than
// the group maximum (so the shift is at least 10)
__device__ __forceinline__ int fx_round(uint32_t xb, int k) {
    const uint32_t u = xb << 16;
    const int ef = (int)(u >> 23) & 0xFF;
    uint32_t mant = u & 0x7FFFFFu;
    int e;
    if (ef == 0) {
        if (mant == 0) return 0;
        e = -126;
    } else {
        mant |= 0x800000u;
        e = ef - 127;
    }
    const int s = 23 - e - k;
    const int mag = s >= 32 ? 0 : (int)((mant + (1u << (s - 1))) >> s);
    return (u >> 31) ? -mag : mag;
}
// Byte of column j (0..63) of a packed group, limb 0 (hi) or 1 (lo).  A group
// is two 64-byte halves (columns 0-31, 32-63) of 16 words: hi_even[4],
// hi_odd[4], lo_even[4], lo_odd[4]; word c of "even" holds, byte by byte, the
// columns that the even nibbles of weight word c hold (columns 8c..8c+7 of the
// half), "odd" those of the odd nibbles.  Tiled blocks store the columns of a
// word in the nibble order (0,2,4,6,1,3,5,7): even nibbles = (0,4,1,5), odd =
// (2,6,3,7); the MLX layout in natural order: even = (0,2,4,6), odd = (1,3,5,7).
template <bool kNatural>
__device__ __forceinline__ int fx_byte(int j, int limb) {
    const int half = j >> 5, jj = j & 31, c = jj >> 3, c8 = jj & 7;
    const int odd = kNatural ? (c8 & 1) : ((c8 >> 1) & 1);
    const int kb = kNatural ? (c8 >> 1) : (((c8 & 1) << 1) | (c8 >> 2));
    return half * 64 + (limb * 8 + odd * 4 + c) * 4 + kb;
}
constexpr int kFxGroupBytes = 128;

// One warp packs one 64-column bf16 group (x64, generic address) into
// dst (128 bytes, generic address; may be x64 itself) and meta = (sum_j X_j
// 2^-k, 2^-(k+4)).
template <bool kNatural>
__device__ __forceinline__ void fx_pack_group_warp(const uint16_t* x64, uint8_t* dst, float2* meta, int lane) {
    const uint32_t v = reinterpret_cast<const uint32_t*>(x64)[lane];  // columns 2 lane, 2 lane + 1
    const uint32_t m = max(v & 0x7FFFu, (v >> 16) & 0x7FFFu);
    const int k = fx_k(__reduce_max_sync(0xffffffffu, m));
    const int X0 = fx_round(v & 0xFFFFu, k), X1 = fx_round(v >> 16, k);
    const int sx = __reduce_add_sync(0xffffffffu, X0 + X1);
    __syncwarp();  // every lane has read its columns before any byte is written
    dst[fx_byte<kNatural>(2 * lane, 0)] = (uint8_t)(X0 >> 8);
    dst[fx_byte<kNatural>(2 * lane, 1)] = (uint8_t)(X0 & 255);
    dst[fx_byte<kNatural>(2 * lane + 1, 0)] = (uint8_t)(X1 >> 8);
    dst[fx_byte<kNatural>(2 * lane + 1, 1)] = (uint8_t)(X1 & 255);
    if (lane == 0) *meta = make_float2(__fmul_rn(__int2float_rn(sx), pow2f(-k)), pow2f(-k - 4));
}

__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {  // unsigned a bytes, signed b bytes
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// One 128 x 64 block against one packed group: lane l covers rows
// (l >> 1) + 16 i (i < 8) and the 32 columns of half (l & 1); the lane pair's
// integer dots are added exactly; every lane ends with P of its 8 rows.
// xp: the lane's half of the packed group (16 words).
__device__ __forceinline__ void block_fx(const uint4 (&q)[8], const float (&sc)[8], const float (&bi)[8],
                                         const uint32_t* xp, float xs, float sc16, float (&P)[8]) {
    const uint4 a = reinterpret_cast<const uint4*>(xp)[0], bq = reinterpret_cast<const uint4*>(xp)[1];
    const uint4 c = reinterpret_cast<const uint4*>(xp)[2], d = reinterpret_cast<const uint4*>(xp)[3];
    const uint32_t he[4] = {a.x, a.y, a.z, a.w}, ho[4] = {bq.x, bq.y, bq.z, bq.w};
    const uint32_t le[4] = {c.x, c.y, c.z, c.w}, lo[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t w[4] = {q[i].x, q[i].y, q[i].z, q[i].w};
        int h0 = 0, h1 = 0;
        uint32_t l0 = 0, l1 = 0;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
            const uint32_t we = w[cc] & 0x0F0F0F0Fu, wo = w[cc] & 0xF0F0F0F0u;
            h0 = dp4a_us(we, he[cc], h0);
            h1 = dp4a_us(wo, ho[cc], h1);
            l0 = __dp4a(we, le[cc], l0);
            l1 = __dp4a(wo, lo[cc], l1);
        }
        int D = (h0 * 16 + h1) * 256 + (int)(l0 * 16u + l1);  // 16 sum q X over the lane's 32 columns
        D += __shfl_xor_sync(0xffffffffu, D, 1);
        P[i] = __fmaf_rn(sc[i], __fmul_rn(__int2float_rn(D), sc16), __fmul_rn(bi[i], xs));
    }
}

// The tiled gate/up array is paired: the 128 features of gate/up row tile rt
// are blocks 2rt and 2rt+1; feature c of block h sits in row paired_row(c)
// (gate) and paired_row(c) + 16 (up).
__device__ __forceinline__ int paired_row(int c) { return 32 * (c >> 4) + (c & 15); }

// Weight sources: 128 rows x 64 columns of one block of one expert; lane l
// loads rows (l >> 1) + 16 i and the 16 bytes of half (l & 1).
struct TiledSrc {  // the context's blocks; nibble order c0,c2,c4,c6,c1,c3,c5,c7
    const uint8_t* base;
    int n_rt, KT, stride, off;  // block (e, rt, kt) = base + (((e*n_rt + rt)*KT + kt)*stride + off) * 4608
    static constexpr bool kNatural = false;
    __device__ __forceinline__ const uint8_t* block(int e, int rt, int kt) const {
        return base + ((((size_t)e * n_rt + rt) * KT + kt) * stride + off) * kBlockBytes;
    }
    __device__ __forceinline__ void load(int e, int rt, int kt, int lane, uint4 (&q)[8], float (&sc)[8],
                                         float (&bi)[8]) const {
        const uint8_t* blk = block(e, rt, kt);
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
// a tiled block already in shared memory
__device__ __forceinline__ void load_block_smem(const uint8_t* blk, int lane, uint4 (&q)[8], float (&sc)[8],
                                                float (&bi)[8]) {
    const uint4* wq = reinterpret_cast<const uint4*>(blk + (lane & 1) * 2048);
    const uint16_t* sb = reinterpret_cast<const uint16_t*>(blk + kBlockWords * 4);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int row = (lane >> 1) + 16 * i;
        q[i] = wq[row];
        sc[i] = bf2f(sb[row]);
        bi[i] = bf2f(sb[kRowTile + row]);
    }
}

// An out-of-range expert id is reported and replaced by 0, so every CTA still
// takes part in its tile's arrival count and no weight outside the layer is read.
__device__ __forceinline__ int checked_expert(int e, int E, int* err) {
    if (e >= 0 && e < E) return e;
    if (threadIdx.x == 0) atomicExch(err, kDevBadRoute);
    return 0;
}

// The last split of gate/up tile (p, rt), 256 threads (t256) synchronising on
// named barrier bid: g and u summed over the splits in split order from the
// partials tp[split][2][128], h = bf16(silu(g) u), and h's two 64-feature
// groups packed into hq/hmeta (pair p's row of I/64 groups) for the down
// projection's layout.  s_gsum [2][128], s_red [8] shared.
template <bool kNatural>
__device__ __forceinline__ void finish_gu_tile(const float* tp, int I, int p, int rt, uint8_t* hq, float2* hmeta,
                                               float (*s_gsum)[kRowTile], int* s_red, int t256, int bid) {
    const int pr = t256 >> 7, row = t256 & 127, lane = t256 & 31, w = t256 >> 5;
    float sum = 0.0f;
#pragma unroll
    for (int jj = 0; jj < kSplitGU; ++jj) sum += __ldcg(tp + (size_t)jj * 2 * kRowTile + pr * kRowTile + row);
    s_gsum[pr][row] = sum;
    named_bar_sync(bid, 256);
    uint32_t hb = 0;
    if (t256 < kRowTile) {
        float g, u;
        if (kNatural) {  // the MLX source: projection 0 = gate, 1 = up, rows in feature order
            g = s_gsum[0][t256], u = s_gsum[1][t256];
        } else {         // paired blocks: block 2rt + t256/64 holds feature t256
            const int rr = paired_row(t256 & 63);
            g = s_gsum[t256 >> 6][rr], u = s_gsum[t256 >> 6][rr + 16];
        }
        hb = f2bf(silu_mul(g, u));
    }
    if (w < 4) {
        const uint32_t wm = __reduce_max_sync(0xffffffffu, hb & 0x7FFFu);
        if (lane == 0) s_red[w] = (int)wm;
    }
    named_bar_sync(bid, 256);
    const int gl = t256 >> 6, gi = p * (I / kGroup) + 2 * rt + gl;
    int k = 0;
    if (w < 4) {
        k = fx_k((uint32_t)max(s_red[2 * gl], s_red[2 * gl + 1]));
        const int X = fx_round(hb, k), c = t256 & 63;
        uint8_t* dst = hq + (size_t)gi * kFxGroupBytes;
        dst[fx_byte<kNatural>(c, 0)] = (uint8_t)(X >> 8);
        dst[fx_byte<kNatural>(c, 1)] = (uint8_t)(X & 255);
        const int ws = __reduce_add_sync(0xffffffffu, X);
        if (lane == 0) s_red[4 + w] = ws;
    }
    named_bar_sync(bid, 256);
    if (w < 4 && (t256 & 63) == 0)
        hmeta[gi] = make_float2(__fmul_rn(__int2float_rn(s_red[4 + 2 * gl] + s_red[5 + 2 * gl]), pow2f(-k)),
                                pow2f(-k - 4));
}

// Fixed-point packs of T activation rows: one warp per 64-column group.
template <bool kNatural>
__global__ void __launch_bounds__(256) k_fx_pack(const uint16_t* x, int T, int H, uint8_t* xq,
                                                 float2* xmeta) {
    pdl_begin();
    const int G = H / kGroup, item = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (item >= T * G) return;
    fx_pack_group_warp<kNatural>(x + (size_t)item * kGroup, xq + (size_t)item * kFxGroupBytes, xmeta + item,
                                 threadIdx.x & 31);
}

// grid (I/128, kSplitGU, T*K), 256 threads.  warp w: block half / projection
// w & 1, groups kt0 + (w >> 1) + 4 j of the split.
template <class Src>
__global__ void __launch_bounds__(256) k_decode_gateup(Src gsrc, Src usrc, const int32_t* ids, int H,
                                                       int I, int K, int E, DecodeBufs d) {
    pdl_begin();
    __shared__ float s_part[8][kRowTile];
    __shared__ float s_gsum[2][kRowTile];
    __shared__ int s_red[8];
    __shared__ int s_last;
    const int rt = blockIdx.x, ks = blockIdx.y, p = blockIdx.z;
    const int n_rt = gridDim.x, KT = H / kGroup, nkt = KT / kSplitGU;
    const int t = p / K, e = checked_expert(ids[p], E, d.err);
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, proj = w & 1;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j = (w >> 1); j < nkt; j += 4) {
        const int kt = ks * nkt + j;
        uint4 q[8];
        float sc[8], bi[8], P[8];
        (proj ? usrc : gsrc).load(e, Src::kNatural ? rt : 2 * rt + proj, kt, lane, q, sc, bi);
        const size_t gi = (size_t)t * KT + kt;
        const float2 m = d.xmeta[gi];
        block_fx(q, sc, bi, reinterpret_cast<const uint32_t*>(d.xq + gi * kFxGroupBytes + (lane & 1) * 64), m.x,
                 m.y, P);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], P[i]);
    }
    if ((lane & 1) == 0)
#pragma unroll
        for (int i = 0; i < 8; ++i) s_part[w][(lane >> 1) + 16 * i] = acc[i];
    __syncthreads();
    // fixed-order sum of the 4 warps of each projection
    const int pr = tid >> 7, row = tid & 127;
    const float v = ((s_part[pr][row] + s_part[pr + 2][row]) + s_part[pr + 4][row]) + s_part[pr + 6][row];
    float* part = d.part + (((size_t)p * n_rt + rt) * kSplitGU) * 2 * kRowTile;
    part[(size_t)ks * 2 * kRowTile + pr * kRowTile + row] = v;
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        uint32_t* c = d.cnt_gu + (size_t)p * n_rt + rt;
        const unsigned old = atomicAdd(c, 1u);
        s_last = (old == kSplitGU - 1);
        if (s_last) *c = 0;  // ready for the next call
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    finish_gu_tile<Src::kNatural>(part, I, p, rt, d.hq, d.hmeta, s_gsum, s_red, tid, 0);
}

// grid (H/128, K, T), 32 * min(I/64, 16) threads.  warp w: groups w, w + nwarps, ...
template <class Src>
__global__ void __launch_bounds__(512) k_decode_down(Src dsrc, const int32_t* ids,
                                                     const float* wts,
                                                     const uint16_t* residual, int H, int I, int K,
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
        uint4 q[8];
        float sc[8], bi[8], P[8];
        dsrc.load(e, rt, kt, lane, q, sc, bi);
        const size_t gi = (size_t)p * KT + kt;
        const float2 m = __ldcg(d.hmeta + gi);
        uint32_t xp[16];
#pragma unroll
        for (int v = 0; v < 4; ++v)
            reinterpret_cast<uint4*>(xp)[v] =
                __ldcg(reinterpret_cast<const uint4*>(d.hq + gi * kFxGroupBytes + (lane & 1) * 64) + v);
        block_fx(q, sc, bi, xp, m.x, m.y, P);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], P[i]);
    }
    if ((lane & 1) == 0)
#pragma unroll
        for (int i = 0; i < 8; ++i) s_part[w][(lane >> 1) + 16 * i] = acc[i];
    __syncthreads();
    for (int r = tid; r < kRowTile; r += blockDim.x) {  // blockDim may be below 128 (inter = 128)
        float v = 0.0f;
        for (int j = 0; j < nwarps; ++j) v = __fadd_rn(v, s_part[j][r]);
        d.y[(size_t)p * H + rt * kRowTile + r] = f2bf(v);
    }
    if (!do_combine) return;
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        uint32_t* c = d.cnt_dn + (size_t)t * n_rt + rt;
        const unsigned old = atomicAdd(c, 1u);
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
// One cooperative launch runs the whole decode layer for T <= 8 tokens, one
// CTA of 16 warps per SM, with no grid-wide barrier:
//   0  warp 0 takes the CTA's ticket (launch generation = ticket / grid size)
//      and, for an input given as is, computes its router row (expert b)
//      straight from global memory; the other warps stage the input
//      (RMSNormed with `normalize`, then the router reads it from shared
//      memory);
//   A  router logits are stored with the launch's stamp in four replicas;
//   B  warps t < T poll token t's stamped logits and run top-k (every CTA, the
//      same result); the other warps meanwhile pack the input groups in fixed
//      point; warp 0 then issues the bulk copies of the CTA's first tile;
//   C  tiles (pair p, 64-feature group r2): the 32 gate/up blocks of block row
//      r2 (8 splits, streamed through an 8-slot ring) reduced in the CTA,
//      SwiGLU and h in fixed point in shared memory, then the 16 blocks of the
//      down projection's column group r2 (loaded into the ring once the
//      gate/up blocks are consumed); the 2048 down partials go to global
//      memory, each stored together with the launch's stamp;
//   D  combine jobs (token, 32 rows), on the CTAs with fewer tiles: once the
//      K * I/64 stamped partials of each row are in, y of every pair (the
//      groups summed in order, rounded to bf16) and the rank-order combine.
// Every wait is bounded (wait_ns); copies still in flight are drained before a
// CTA exits after a wait gave up.
constexpr int kFusedThreads = 512, kFusedWarps = kFusedThreads / 32;
constexpr int kLogitReplicas = 4;    // copies of the stamped logits (spreads the polling)

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// (logit bits | stamp << 32) as one 64-bit access: single-copy atomic, and
// "relaxed" at gpu scope, so the polling sees other SMs' stores (a weak load
// may keep returning a stale copy)
__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Router row of expert e (H = 2048: one 64-column group per lane), loaded into
// registers before anything else so its latency overlaps the input's.
struct RouterRow {
    uint4 q[4];
    float sc, bi;
};
__device__ __forceinline__ void router_row_load(const uint32_t* __restrict__ w, const uint16_t* __restrict__ s,
                                                const uint16_t* __restrict__ b, int H, int e, int lane,
                                                RouterRow& r) {
    const int G = H / kGroup;
    const uint4* wr = reinterpret_cast<const uint4*>(w + (size_t)e * (H / 4) + (size_t)lane * 16);
#pragma unroll
    for (int v = 0; v < 4; ++v) r.q[v] = __ldg(wr + v);
    r.sc = bf2f(__ldg(s + (size_t)e * G + lane));
    r.bi = bf2f(__ldg(b + (size_t)e * G + lane));
}
// router_warp_item's arithmetic for one group per lane, x in global
// (kGlobalX) or shared memory; lanes r < 4 store (logit, stamp) of every token
// into replica r.  The read-only path for x is safe here: the fused layer is a
// cooperative launch, never a programmatic dependent, so everything earlier in
// the stream has completed when it starts.
template <bool kGlobalX>
__device__ __forceinline__ void router_row_logits(const RouterRow& r, const uint16_t* x, int T, int H, int E, int e,
                                                  int lane, uint32_t stamp, uint64_t* lst) {
    float wf[64];
#pragma unroll
    for (int v = 0; v < 4; ++v) {
        const uint32_t qs[4] = {r.q[v].x, r.q[v].y, r.q[v].z, r.q[v].w};
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int j = 0; j < 4; ++j) wf[v * 16 + c * 4 + j] = __fmaf_rn((float)((qs[c] >> (8 * j)) & 0xFFu), r.sc, r.bi);
    }
    for (int t = 0; t < T; ++t) {
        const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)t * H + (size_t)lane * 64);
        float a = 0.0f;
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            const uint4 q = kGlobalX ? __ldg(xr + v) : xr[v];
            const uint32_t qs[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                a = __fmaf_rn(wf[v * 8 + c * 2], __uint_as_float(qs[c] << 16), a);
                a = __fmaf_rn(wf[v * 8 + c * 2 + 1], __uint_as_float(qs[c] & 0xFFFF0000u), a);
            }
        }
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
        if (lane < kLogitReplicas)
            st_relaxed_u64(lst + ((size_t)lane * kFusedMaxT + t) * E + e,
                           (uint64_t)__float_as_uint(a) | ((uint64_t)stamp << 32));
    }
}

// bounded wait on an mbarrier phase that ignores the abort flag (draining
// copies in flight before the CTA exits)
__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity))
        if (global_ns() - t0 > limit_ns) return;
}

__global__ void __launch_bounds__(kFusedThreads, 1) k_decode_fused(
    const uint32_t* __restrict__ rw, const uint16_t* __restrict__ rs, const uint16_t* __restrict__ rb,
    TiledSrc gsrc, TiledSrc dsrc, const uint16_t* x_in, const uint16_t* residual,
    const float* bias, int T, int H, int I, int E, int K, int norm, int normalize, float eps,
    FusedDecodeBufs f, FusedPlan pl, uint16_t* __restrict__ out) {
    extern __shared__ __align__(128) uint8_t smem[];
    // [T][H] bf16 layer input; after phase A, in place, its fixed-point packs [T][H/64][128 B]
    uint16_t* s_x = reinterpret_cast<uint16_t*>(smem + pl.off_x);
    uint8_t* s_xq = smem + pl.off_x;
    uint8_t* s_hq = smem + pl.off_h;  // [128 B] the tile's h group in fixed point
    __shared__ float2 s_xm[kFusedMaxT * 32];
    __shared__ float2 s_hm[1];
    __shared__ float s_sq[2][256];
    __shared__ int s_ids[kFusedMaxT * kMaxK];
    __shared__ float s_wts[kFusedMaxT * kMaxK];
    __shared__ float s_blk[32][kRowTile];  // C: a tile's per-block row values; D: the pairs' y of a job
    __shared__ float s_gsum[1][1][kRowTile];
    __shared__ int s_red[2][8];
    __shared__ __align__(8) uint64_t s_bar[9];  // ring slots 0-7, the down column group
    __shared__ int s_issued[9];                 // copies issued per barrier
    __shared__ uint32_t s_gen;
    __shared__ volatile int s_abort;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, b = blockIdx.x;
    // phase timeline (diagnostics, thread 0 of each CTA, 24 entries per CTA): 0 start, 1 A done,
    // 2 logits seen, 3 copies issued, 4 C done, 5 first h ready, 6 D done, 7 top-k + packs done;
    // 8 first wave landed, 9 computed, 10 done; 13 first down unit landed, 14 y written;
    // 16-18 inside top-k (logits in, softmax sum, selection)
    auto mark = [&](int k) {
        if (f.trace && tid == 0) f.trace[24 * b + k] = global_ns();
    };
    mark(0);
    // 0a: this CTA's router rows (experts b, b + G, ...: one per warp) into registers
    RouterRow rrow;
    const int e_r = b + G * warp;
    if (e_r < E) router_row_load(rw, rs, rb, H, e_r, lane, rrow);
    if (warp == 0) {
        // every CTA of launch n draws a ticket in [nG, (n+1)G): generation n
        uint32_t tk = 0;
        if (lane == 0) {
            tk = atomicAdd(f.bar, 1u);
            for (int i = 0; i < 9; ++i) mbar_init(smem_u32(&s_bar[i]), 1), s_issued[i] = 0;
            s_abort = 0;
            fence_mbar_init();
            fence_proxy_async_smem();
        }
        const uint32_t gen = __shfl_sync(0xffffffffu, tk, 0) / (uint32_t)G;
        if (lane == 0) s_gen = gen;
        // A (input as given): warp 0's router row straight from global memory,
        // while the other warps stage the input
        if (!normalize && e_r < E) {
            router_row_logits<true>(rrow, x_in, T, H, E, e_r, lane, gen + 1, f.lst);
            mark(1);
        }
    }

    // 0b: the layer input into shared memory; with `normalize`, the MoE input
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
    const uint32_t stamp = s_gen + 1;

    // A (normalised input, and any further router rows): from shared memory
    if (e_r < E && (normalize || warp > 0)) {
        router_row_logits<false>(rrow, s_x, T, H, E, e_r, lane, stamp, f.lst);
        if (warp == 0) mark(1);
    }
    __syncthreads();  // the router has read s_x: it may be packed in place

    const int KT = H / kGroup, nkt = KT / kSplitGU, P = T * K;
    // Work: tiles (p, r2) -- pair p's 64-feature group r2: the gate/up block
    // row r2 (its gate and up rows, all 8 splits = 32 blocks, streamed through
    // an 8-slot ring as 8 units of 4 contiguous blocks) and the down
    // projection's column group r2 (16 blocks, one per 128-row tile) -- on CTAs
    // b, b + G, ...; then combine jobs (token t, row tile rt) on the CTAs with
    // fewer tiles first.
    const int n_r2 = I / kGroup, n_tiles = P * n_r2;
    const int Nt = b < n_tiles ? (n_tiles - 1 - b) / G + 1 : 0;
    const int n_rd = H / kRowTile, KTd = I / kGroup;
    const int n_jobs = T * H / 32, jfirst = (b - n_tiles % G + G) % G;
    uint8_t* region = smem + pl.off_ring;
    // unit v of this CTA's tiles: tile v / 8, split v % 8, ring slot v % 8
    auto issue_unit = [&](int v) {
        const int tau = b + (v >> 3) * G, ks = v & 7;
        const int p = tau / n_r2, r2 = tau % n_r2;
        const int e = checked_expert(s_ids[p], E, f.err);
        const uint32_t bar = smem_u32(&s_bar[v & 7]);
        mbar_arrive_expect_tx(bar, (uint32_t)pl.unit_bytes);
        bulk_g2s(smem_u32(region + (size_t)(v & 7) * pl.unit_bytes), gsrc.block(e, r2, ks * nkt),
                 (uint32_t)pl.unit_bytes, bar);
        ++s_issued[v & 7];
    };
    // the down column group of this CTA's tile i: lane rt < 16 copies block (e, rt, r2)
    // into the ring's first 16 x 4608 bytes (slots 0-3); warp 0, all lanes
    auto issue_down_group = [&](int i) {
        const int tau = b + i * G, p = tau / n_r2, r2 = tau % n_r2;
        const uint32_t bar = smem_u32(&s_bar[8]);
        if (lane == 0) {
            mbar_arrive_expect_tx(bar, (uint32_t)(n_rd * kBlockBytes));
            ++s_issued[8];
        }
        __syncwarp();
        if (lane < n_rd) {
            const int e = checked_expert(s_ids[p], E, f.err);
            bulk_g2s(smem_u32(region + (size_t)lane * kBlockBytes), dsrc.block(e, lane, r2), (uint32_t)kBlockBytes,
                     bar);
        }
    };
    // warp 0: the first tile's 8 units, one copy per lane
    auto issue_first = [&]() {
        if (Nt > 0 && lane < 8) issue_unit(lane);
    };
    if (warp < T) {
        // B: token `warp`'s logits from replica b % 4, once all carry this launch's stamp
        const int t = warp;
        const uint64_t* src = f.lst + ((size_t)(b % kLogitReplicas) * kFusedMaxT + t) * E;
        float lv[kMaxE / 32];
        const uint64_t t0 = global_ns();
        for (;;) {
            bool ok = true;
#pragma unroll
            for (int i = 0; i < kMaxE / 32; ++i) {
                const int e = lane + 32 * i;
                lv[i] = 0.0f;
                if (e < E) {
                    const uint64_t v = ld_relaxed_u64(src + e);
                    lv[i] = __uint_as_float((uint32_t)v);
                    ok = ok && (uint32_t)(v >> 32) == stamp;
                }
            }
            if (__all_sync(0xffffffffu, ok)) break;
            if (global_ns() - t0 > f.wait_ns) {
                if (lane == 0) atomicExch(f.err, kDevTimeout);
                s_abort = 1;
                break;
            }
        }
        if (t == 0) mark(2);
        int ik;
        float wk;
        topk_token([&](int i, int) { return lv[i]; }, bias, E, K, norm, lane, &ik, &wk,
                   [&](int k) { mark(16 + k); });
        if (lane < K) {
            s_ids[t * K + lane] = ik;
            s_wts[t * K + lane] = wk;
            if (b == 0) f.ids[t * K + lane] = ik, f.wts[t * K + lane] = wk;
        }
        if (T == 1 && !s_abort) {
            // one token: this warp holds every route, so the weight copies go out now
            __syncwarp();
            issue_first();
            mark(3);
        }
    } else {
        // the input groups in fixed point, in place (tiled order)
        for (int it = warp - T; it < T * KT; it += kFusedWarps - T)
            fx_pack_group_warp<false>(s_x + (size_t)it * kGroup, s_xq + (size_t)it * kFxGroupBytes, &s_xm[it],
                                      lane);
    }
    __syncthreads();
    mark(7);
    if (T > 1 && warp == 0 && !s_abort) issue_first();

    // C: tiles.  Gate/up: 32 blocks, warp w takes blocks w and w + 16 (split
    // bi / 4, group ks * 4 + bi % 4); each row is summed over the splits in
    // order, each split's 4 groups as ((P0 + P1) + P2) + P3 (the separate
    // kernel's order); SwiGLU over the 64 features and h in fixed point, kept in
    // shared memory.  Down: warp w computes row tile w of the column group; the
    // 2048 values go to ypart[p][r2], and each row tile's counter of (token,
    // row tile) gets one acq_rel arrival.
    for (int i = 0; i < Nt; ++i) {
        const int tau = b + i * G, p = tau / n_r2, r2 = tau % n_r2, t = p / K;
        // two rounds: splits 0-3 (slots 0-3), then -- with the down column
        // group already on its way into slots 0-3 -- splits 4-7
        for (int bi = warp; bi < 32; bi += kFusedWarps) {
            const int ks = bi >> 2, j = bi & 3, v = 8 * i + ks, kt = ks * nkt + j;
            if (bi == kFusedWarps + warp) {
                __syncthreads();  // slots 0-3 consumed
                if (warp == 0 && !s_abort) {
                    fence_proxy_async_smem();
                    issue_down_group(i);
                }
            }
            if (!s_abort && mbar_wait(smem_u32(&s_bar[v & 7]), (uint32_t)(v >> 3) & 1u, &s_abort, 1, f.wait_ns)) {
                if (i == 0 && bi == 0) mark(8);
                uint4 q[8];
                float sc[8], bv[8], Pv[8];
                load_block_smem(region + (size_t)(v & 7) * pl.unit_bytes + (size_t)j * kBlockBytes, lane, q, sc, bv);
                const int gi = t * KT + kt;
                block_fx(q, sc, bv, reinterpret_cast<const uint32_t*>(s_xq + (size_t)gi * kFxGroupBytes + (lane & 1) * 64),
                         s_xm[gi].x, s_xm[gi].y, Pv);
                if ((lane & 1) == 0)
#pragma unroll
                    for (int r = 0; r < 8; ++r) s_blk[bi][(lane >> 1) + 16 * r] = Pv[r];
            }
        }
        __syncthreads();
        if (i == 0) mark(9);
        // slots 4-7 are free: the next tile's units 4-7 go out now
        if (warp == 0 && !s_abort && i + 1 < Nt && lane >= 4 && lane < 8) {
            fence_proxy_async_smem();
            issue_unit(8 * (i + 1) + lane);
        }
        if (tid < kRowTile) {
            float sum = 0.0f;
#pragma unroll
            for (int ks = 0; ks < kSplitGU; ++ks)
                sum += ((s_blk[4 * ks][tid] + s_blk[4 * ks + 1][tid]) + s_blk[4 * ks + 2][tid]) + s_blk[4 * ks + 3][tid];
            s_gsum[0][0][tid] = sum;
        }
        __syncthreads();
        // SwiGLU of the 64 features (rows paired_row(c) and + 16), h in fixed point
        if (warp < 2) {
            const int rr = paired_row(tid);
            const uint32_t hb = f2bf(silu_mul(s_gsum[0][0][rr], s_gsum[0][0][rr + 16]));
            const uint32_t wm = __reduce_max_sync(0xffffffffu, hb & 0x7FFFu);
            if (lane == 0) s_red[0][warp] = (int)wm;
            named_bar_sync(1, 64);
            const int k = fx_k((uint32_t)max(s_red[0][0], s_red[0][1]));
            const int X = fx_round(hb, k);
            s_hq[fx_byte<false>(tid, 0)] = (uint8_t)(X >> 8);
            s_hq[fx_byte<false>(tid, 1)] = (uint8_t)(X & 255);
            const int ws = __reduce_add_sync(0xffffffffu, X);
            if (lane == 0) s_red[1][warp] = ws;
            named_bar_sync(1, 64);
            if (tid == 0)
                s_hm[0] = make_float2(__fmul_rn(__int2float_rn(s_red[1][0] + s_red[1][1]), pow2f(-k)), pow2f(-k - 4));
        }
        __syncthreads();
        // down: row tile `warp` of column group r2
        if (warp < n_rd && !s_abort &&
            mbar_wait(smem_u32(&s_bar[8]), (uint32_t)i & 1u, &s_abort, 3, f.wait_ns)) {
            if (i == 0 && warp == 0) mark(13);
            uint4 q[8];
            float sc[8], bv[8], Pv[8];
            load_block_smem(region + (size_t)warp * kBlockBytes, lane, q, sc, bv);
            block_fx(q, sc, bv, reinterpret_cast<const uint32_t*>(s_hq + (lane & 1) * 64), s_hm[0].x, s_hm[0].y, Pv);
            // each partial carries the launch's stamp (one 64-bit store: the
            // reader sees the value together with its stamp, no fence needed)
            uint64_t* yp = f.ypart + ((size_t)p * n_r2 + r2) * H + warp * kRowTile;
            if ((lane & 1) == 0)
#pragma unroll
                for (int r = 0; r < 8; ++r)
                    st_relaxed_u64(yp + (lane >> 1) + 16 * r, (uint64_t)__float_as_uint(Pv[r]) | ((uint64_t)stamp << 32));
        }
        __syncthreads();  // the ring is free again
        if (i == 0) mark(14);
        if (s_abort) break;
        if (warp == 0 && i + 1 < Nt && lane < 4) {
            fence_proxy_async_smem();
            issue_unit(8 * (i + 1) + lane);
        }
        if (i == 0) mark(10);
    }
    mark(4);

    // D: combine jobs (token t, 32 rows): thread (row, pair k) polls the I/64
    // stamped partials of its row until all carry this launch's stamp, sums them
    // in group order and rounds y to bf16; then the rank-order combine
    // (forward.rs:225-232) into out
    for (int jb = jfirst; jb < n_jobs && !s_abort; jb += G) {
        const int t = jb / (4 * n_rd), r0 = (jb % (4 * n_rd)) * 32;
        const int row = tid & 31, k = tid >> 5;
        if (k < K) {
            const uint64_t* yp = f.ypart + (size_t)(t * K + k) * n_r2 * H + r0 + row;
            float pv[16];
            const uint64_t t0 = global_ns();
            for (;;) {
                bool ok = true;
#pragma unroll
                for (int g = 0; g < 16; ++g) {
                    pv[g] = 0.0f;
                    if (g < n_r2) {
                        const uint64_t v = ld_relaxed_u64(yp + (size_t)g * H);
                        pv[g] = __uint_as_float((uint32_t)v);
                        ok = ok && (uint32_t)(v >> 32) == stamp;
                    }
                }
                if (ok) break;
                if (global_ns() - t0 > f.wait_ns) {
                    atomicExch(f.err, kDevTimeout);
                    s_abort = 2;
                    break;
                }
            }
            float v = 0.0f;
#pragma unroll
            for (int g = 0; g < 16; ++g)
                if (g < n_r2) v = __fadd_rn(v, pv[g]);
            s_blk[k][row] = bf2f(f2bf(v));  // y, rounded to bf16
        }
        __syncthreads();
        if (jb == jfirst) mark(5);
        if (s_abort) break;
        if (tid < 32) {
            const int fo = r0 + tid;
            float a = residual ? bf2f(residual[(size_t)t * H + fo]) : 0.0f;
            for (int kk = 0; kk < K; ++kk) a = __fmaf_rn(s_wts[t * K + kk], s_blk[kk][tid], a);
            out[(size_t)t * H + fo] = f2bf(a);
        }
        __syncthreads();
    }
    mark(6);
    // copies still in flight (only after a wait gave up) land before the CTA exits
    __syncthreads();
    if (tid == 0 && s_abort) {
        for (int si = 0; si < 9; ++si)
            if (s_issued[si]) mbar_drain(smem_u32(&s_bar[si]), (uint32_t)(s_issued[si] - 1) & 1u, f.wait_ns);
    }
}

}  // namespace

template <bool kNatural>
static cudaError_t launch_fx_pack(const uint16_t* x, int T, int H, uint8_t* xq, float2* xmeta, cudaStream_t st) {
    const int items = T * (H / kGroup);
    const cudaError_t e = launch_pdl(k_fx_pack<kNatural>, dim3((items + 7) / 8), dim3(256), 0, st, x, T, H, xq, xmeta);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

cudaError_t launch_decode_gateup(const LayerDev& L, const Shape& sh, const uint16_t* x, const int32_t* ids, int T,
                                 const DecodeBufs& d, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    cudaError_t e = launch_fx_pack<false>(x, T, sh.H, d.xq, d.xmeta, st);
    if (e != cudaSuccess) return e;
    const TiledSrc g{L.gateup, sh.I / 64, sh.H / kGroup, 1, 0}, u = g;  // paired blocks
    dim3 grid(sh.I / kRowTile, kSplitGU, T * sh.K);
    e = launch_pdl(k_decode_gateup<TiledSrc>, grid, dim3(256), 0, st, g, u, ids, sh.H, sh.I, sh.K, sh.E, d);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

cudaError_t launch_decode_down(const LayerDev& L, const Shape& sh, const int32_t* ids, const float* w,
                               const uint16_t* residual, int T, const DecodeBufs& d, uint16_t* out, int do_combine,
                               cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    const TiledSrc dn{L.down, sh.H / kRowTile, sh.I / kGroup, 1, 0};
    dim3 grid(sh.H / kRowTile, sh.K, T);
    const cudaError_t e = launch_pdl(k_decode_down<TiledSrc>, grid, dim3(down_threads(sh.I)), 0, st, dn, ids, w,
                                     residual, sh.H, sh.I, sh.K, sh.E, d, out, do_combine);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

FusedPlan fused_plan(int T, int H, int I) {
    FusedPlan pl{};
    const int nkt = (H / kGroup) / kSplitGU;
    pl.off_x = 0;
    pl.off_h = (T * H * 2 + 127) / 128 * 128;
    pl.off_ring = pl.off_h + kFxGroupBytes;
    pl.unit_bytes = nkt * kBlockBytes;  // one split of one block row
    pl.dn_bytes = (H / kRowTile) * kBlockBytes;  // a down column group (in slots 0-3)
    pl.region_bytes = 8 * pl.unit_bytes;
    pl.nslot = 8;
    pl.smem_bytes = pl.off_ring + pl.region_bytes;
    return pl;
}

// dynamic shared memory the fused layer may use on this device (opt-in limit
// minus the kernel's static shared memory)
static int fused_smem_limit() {
    static int limit = -1;
    if (limit < 0) {
        int dev = 0, optin = 0;
        cudaFuncAttributes fa{};
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
            cudaFuncGetAttributes(&fa, k_decode_fused) != cudaSuccess)
            return 0;
        limit = optin - (int)fa.sharedSizeBytes;
    }
    return limit;
}

bool decode_fused_supported(const Shape& sh, int T) {
    if (T <= 0 || T > kFusedMaxT || sh.K > kMaxK || sh.E > kMaxE || sh.H != 2048 || sh.I % 256 || sh.I > 1024 ||
        sh.K > 32)
        return false;
    return fused_plan(T, sh.H, sh.I).smem_bytes <= fused_smem_limit();
}

cudaError_t launch_decode_fused(const LayerDev& L, const Shape& sh, const uint16_t* x, const uint16_t* residual,
                                const float* bias, int T, int norm, int normalize, float eps,
                                const FusedDecodeBufs& f, uint16_t* out, int num_sms, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (!decode_fused_supported(sh, T)) return cudaErrorInvalidValue;
    if ((sh.E + num_sms - 1) / num_sms > kFusedWarps) return cudaErrorInvalidValue;  // router rows: one per warp
    const TiledSrc g{L.gateup, sh.I / 64, sh.H / kGroup, 1, 0};  // paired blocks
    const TiledSrc dn{L.down, sh.H / kRowTile, sh.I / kGroup, 1, 0};
    const FusedPlan pl = fused_plan(T, sh.H, sh.I);
    cudaError_t e = cudaFuncSetAttribute(k_decode_fused, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem_bytes);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms);  // one CTA per SM: every CTA is resident (cooperative)
    cfg.blockDim = dim3(kFusedThreads);
    cfg.dynamicSmemBytes = pl.smem_bytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    note_launch();
    return cudaLaunchKernelEx(&cfg, k_decode_fused, L.router_w, L.router_s, L.router_b, g, dn, x, residual, bias, T,
                              sh.H, sh.I, sh.E, sh.K, norm, normalize, eps, f, pl, out);
}

cudaError_t launch_decode_ffn_mlx(const uint32_t* gw, const uint16_t* gs, const uint16_t* gb, const uint32_t* uw,
                                  const uint16_t* us, const uint16_t* ub, const uint32_t* dw, const uint16_t* ds,
                                  const uint16_t* db, const Shape& sh, const uint16_t* x, const int32_t* ids,
                                  const float* w, const uint16_t* residual, int T, const DecodeBufs& d, uint16_t* out,
                                  cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    cudaError_t e = launch_fx_pack<true>(x, T, sh.H, d.xq, d.xmeta, st);
    if (e != cudaSuccess) return e;
    const MlxSrc g{gw, gs, gb, sh.I, sh.H}, u{uw, us, ub, sh.I, sh.H}, dn{dw, ds, db, sh.H, sh.I};
    dim3 g1(sh.I / kRowTile, kSplitGU, T * sh.K);
    e = launch_pdl(k_decode_gateup<MlxSrc>, g1, dim3(256), 0, st, g, u, ids, sh.H, sh.I, sh.K, sh.E, d);
    if (e != cudaSuccess) return e;
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    dim3 g2(sh.H / kRowTile, sh.K, T);
    e = launch_pdl(k_decode_down<MlxSrc>, g2, dim3(down_threads(sh.I)), 0, st, dn, ids, w, residual, sh.H, sh.I, sh.K,
                   sh.E, d, out, 1);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace obs
