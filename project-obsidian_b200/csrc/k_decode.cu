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
#include "obs_internal.cuh"

namespace obs {
namespace {

constexpr int kSplitGU = kDecodeSplit;  // k-splits of the gate/up mat-vec (one 64-column block per warp)

// 1 + q/16 as a float, q the 4-bit code at nibble j: the code becomes mantissa bits 19-22
__device__ __forceinline__ float nib_f16th(uint32_t w, int j) {
    const uint32_t m = (4 * j <= 19) ? (w << (19 - 4 * j)) : (w >> (4 * j - 19));
    return __uint_as_float((m & 0x00780000u) | 0x3F800000u);
}

// Weight sources: 128 rows x 64 columns of one projection of one expert.
// Lane l covers rows (l>>1) + 16 i (i < 8) and the 32 columns of half (l & 1).
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
            for (int j = 0; j < 8; ++j)  // nibble j holds column j (MLX) or nib_col(j) (tiled)
                f = __fmaf_rn(nib_f16th(ws[c], j), xr[c * 8 + (Src::kNatural ? j : nib_col(j))], f);
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
        block_dot(proj ? usrc : gsrc, e, rt, kt, xr, xs, lane, acc);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float v = acc[i] + __shfl_xor_sync(0xffffffffu, acc[i], 1);
        if ((lane & 1) == 0) s_part[w][(lane >> 1) + 16 * i] = v;
    }
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
        const float g = s_gu[0][tid], u = s_gu[1][tid];
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
    if (tid < kRowTile) {
        float v = 0.0f;
        for (int j = 0; j < nwarps; ++j) v += s_part[j][tid];
        d.y[(size_t)p * H + rt * kRowTile + tid] = f2bf(v);
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
    if (tid < kRowTile) {
        // rank-order combine, same operation order as k_combine (forward.rs:225-232)
        const int f = rt * kRowTile + tid;
        float a = residual ? bf2f(residual[(size_t)t * H + f]) : 0.0f;
        for (int j = 0; j < K; ++j) {
            const uint16_t yv = __ldcg(d.y + ((size_t)t * K + j) * H + f);
            a = __fmaf_rn(wts[(size_t)t * K + j], bf2f(yv), a);
        }
        out[(size_t)t * H + f] = f2bf(a);
    }
}

int down_threads(int I) { return 32 * (I / kGroup < 16 ? I / kGroup : 16); }

}  // namespace

cudaError_t launch_decode_gateup(const LayerDev& L, const Shape& sh, const uint16_t* x, const int32_t* ids, int T,
                                 const DecodeBufs& d, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    const TiledSrc g{L.gateup, sh.I / kRowTile, sh.H / kGroup, 2, 0}, u{L.gateup, sh.I / kRowTile, sh.H / kGroup, 2, 1};
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
