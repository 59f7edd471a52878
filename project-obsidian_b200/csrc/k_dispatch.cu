// k_dispatch.cu -- token -> expert dispatch and the weighted combine.
//
// Replaces the reference's CPU grouping and gather (src/forward.rs:176-216:
// union of routed experts, per-expert token lists, memcpy of rows) and the
// rank-order scatter of scaled adds (forward.rs:225-232, ops.metal:25-29).
// Slots are ordered by expert, then token (the order of the reference's
// per-expert lists); each expert's segment is padded to 16 rows so a GEMM tile
// never straddles two experts and its row count is a legal tcgen05 N.
#include "obs_internal.cuh"

namespace obs {
namespace {

constexpr int kDispThreads = 512;

__device__ __forceinline__ int pad_rows(int c) { return (c + kSegAlign - 1) / kSegAlign * kSegAlign; }

// grid = E; CTA e computes its segment, the stable slot order of its tokens,
// and its GEMM token tiles.
__global__ void __launch_bounds__(kDispThreads) k_dispatch(const int32_t* __restrict__ ids, int T, int E, int K,
                                                           DispatchBufs d) {
    pdl_begin();
    __shared__ int s_red[2][kDispThreads / 32];
    __shared__ int s_warp[kDispThreads / 32];
    __shared__ int s_base;
    const int e = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int bn = d.bn;

    // padded segment start and tile start of expert e
    int my_seg = 0, my_tiles = 0;
    for (int i = tid; i < e; i += kDispThreads) {
        int p = pad_rows(d.counts[i]);
        my_seg += p;
        my_tiles += (p + bn - 1) / bn;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        my_seg += __shfl_xor_sync(0xffffffffu, my_seg, o);
        my_tiles += __shfl_xor_sync(0xffffffffu, my_tiles, o);
    }
    if (lane == 0) s_red[0][wid] = my_seg, s_red[1][wid] = my_tiles;
    if (tid == 0) s_base = 0;
    __syncthreads();
    int seg = 0, tile0 = 0;
    for (int i = 0; i < kDispThreads / 32; ++i) seg += s_red[0][i], tile0 += s_red[1][i];
    const int cnt = d.counts[e];
    const int P = pad_rows(cnt);
    const int ntile = (P + bn - 1) / bn;

    // stable ordered compaction of the tokens routed to e
    for (int c0 = 0; c0 < T; c0 += kDispThreads) {
        int t = c0 + tid, kfound = -1;
        if (t < T)
            for (int k = 0; k < K; ++k)
                if (ids[(size_t)t * K + k] == e) kfound = k;
        unsigned bal = __ballot_sync(0xffffffffu, kfound >= 0);
        if (lane == 0) s_warp[wid] = __popc(bal);
        __syncthreads();
        int before = 0, total = 0;
        for (int i = 0; i < kDispThreads / 32; ++i) {
            int v = s_warp[i];
            if (i < wid) before += v;
            total += v;
        }
        if (kfound >= 0) {
            int slot = seg + s_base + before + __popc(bal & ((1u << lane) - 1u));
            d.slot_of[(size_t)t * K + kfound] = slot;
            d.src[slot] = t;
        }
        __syncthreads();
        if (tid == 0) s_base += total;
        __syncthreads();
    }
    for (int r = cnt + tid; r < P; r += kDispThreads) d.src[seg + r] = -1;
    for (int j = tid; j < ntile; j += kDispThreads)
        d.tiles[tile0 + j] = make_int4(e, seg + j * bn, min(bn, P - j * bn), 0);
    if (e == E - 1 && tid == 0) {
        *d.n_tiles = tile0 + ntile;
        d.seg[E] = seg + P;
    }
    if (tid == 0) d.seg[e] = seg;
}

// The routed rows (slot order) into the tiled activation layout the grouped
// GEMM reads with bulk copies: one warp per slot row, 16-byte chunks (coalesced
// 512-byte reads of the source row, 128-byte runs per k-group in the
// destination); padding rows (src = -1) are written as zeros.  Token t's row is
// x[t], or row_src[t] when given (expert parallelism: received rows live in
// the exchange buffer, the rank's own in x).
__global__ void __launch_bounds__(256) k_permute(const uint16_t* __restrict__ x, int H, const int32_t* __restrict__ src,
                                                 const int32_t* __restrict__ seg_end, int atoms,
                                                 uint16_t* __restrict__ xp, const uint16_t* const* __restrict__ row_src) {
    pdl_begin();
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= *seg_end) return;
    const int t = src[row];
    const uint16_t* xrow = t >= 0 ? (row_src ? row_src[t] : x + (size_t)t * H) : nullptr;
    const int chunks = H / 8;
    for (int c0 = lane; c0 < chunks; c0 += 32 * 8) {  // H = 2048: the whole row in flight at once
        uint4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int c = c0 + 32 * u;
            v[u] = make_uint4(0, 0, 0, 0);
            if (t >= 0 && c < chunks) v[u] = __ldg(reinterpret_cast<const uint4*>(xrow) + c);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int c = c0 + 32 * u;
            if (c < chunks) *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(xp) + tiled_off(row, c * 8, atoms)) = v[u];
        }
    }
}

// The MoE stack's layer-input RMSNorm (rmsnorm.metal:9-37), in the reference
// kernel's own order: 256 threads per row, thread l sums v*v (rounded product,
// rounded add) over elements l, l+256, ...; the partials meet in the halving
// tree sq[l] += sq[l + s], s = 128 .. 1; rms = sqrt(sq[0] / H + eps);
// out = (x / rms) * w.  IEEE divide and square root, as the oracle.
__global__ void __launch_bounds__(256) k_rmsnorm(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                                                 int H, float eps, uint16_t* __restrict__ out) {
    pdl_begin();
    __shared__ float sq[256];
    const int t = blockIdx.x, l = threadIdx.x;
    const uint16_t* row = x + (size_t)t * H;
    float ps = 0.0f;
    for (int i = l; i < H; i += 256) {
        const float v = bf2f(row[i]);
        ps = __fadd_rn(ps, __fmul_rn(v, v));
    }
    sq[l] = ps;
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if (l < s) sq[l] = __fadd_rn(sq[l], sq[l + s]);
        __syncthreads();
    }
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(sq[0], (float)H), eps));
    for (int i = l; i < H; i += 256) {
        const float v = __fdiv_rn(bf2f(row[i]), rms);
        out[(size_t)t * H + i] = f2bf(w ? __fmul_rn(v, bf2f(w[i])) : v);
    }
}

// out[t] = bf16(residual[t] + sum_k w[t,k] * y[slot_of[t,k]]), rank order, fp32.
// slot_of == nullptr: y is in item order (row t*K + k).  local != nullptr
// (expert parallelism): an item whose entry is s + 1 > 0 was computed on this
// rank and is read from row s of y_local instead; the entry is cleared for the
// next forward.
constexpr int kCombineMaxK = 16;  // the context accepts top_k <= 16

__global__ void __launch_bounds__(256) k_combine(const uint16_t* __restrict__ y, int y_ld,
                                                 const int32_t* __restrict__ slot_of, const float* __restrict__ w,
                                                 const uint16_t* __restrict__ residual, int H, int K,
                                                 uint16_t* __restrict__ out, const uint16_t* __restrict__ y_local,
                                                 int32_t* __restrict__ local) {
    pdl_begin();
    const int t = blockIdx.x;
    // the token's K rows and weights once per CTA, so every row load below is independent
    __shared__ const uint16_t* s_row[kCombineMaxK];
    __shared__ float s_w[kCombineMaxK];
    if (threadIdx.x < K) {
        const size_t item = (size_t)t * K + threadIdx.x;
        const int slot = slot_of ? slot_of[item] : (int)item;  // nullptr: item order
        const int ls = local ? local[item] : 0;
        s_row[threadIdx.x] = ls > 0 ? y_local + (size_t)(ls - 1) * y_ld : y + (size_t)slot * y_ld;
        if (ls > 0) local[item] = 0;
        s_w[threadIdx.x] = w[item];
    }
    __syncthreads();
    for (int f = threadIdx.x * 8; f < H; f += blockDim.x * 8) {
        float acc[8];
        if (residual) {
            uint4 r = __ldg(reinterpret_cast<const uint4*>(residual + (size_t)t * H + f));
            uint32_t rs[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[2 * c] = __uint_as_float(rs[c] << 16), acc[2 * c + 1] = __uint_as_float(rs[c] & 0xFFFF0000u);
        } else {
#pragma unroll
            for (int c = 0; c < 8; ++c) acc[c] = 0.0f;
        }
        // ranks in order, eight rows in flight at a time
        for (int k0 = 0; k0 < K; k0 += 8) {
            uint4 v[8];
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
                if (k0 + kk < K) v[kk] = __ldg(reinterpret_cast<const uint4*>(s_row[k0 + kk] + f));
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                if (k0 + kk >= K) break;
                const float wk = s_w[k0 + kk];
                const uint32_t vs[4] = {v[kk].x, v[kk].y, v[kk].z, v[kk].w};
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    acc[2 * c] = __fmaf_rn(wk, __uint_as_float(vs[c] << 16), acc[2 * c]);
                    acc[2 * c + 1] = __fmaf_rn(wk, __uint_as_float(vs[c] & 0xFFFF0000u), acc[2 * c + 1]);
                }
            }
        }
        uint4 o = make_uint4(pack_bf2(acc[0], acc[1]), pack_bf2(acc[2], acc[3]), pack_bf2(acc[4], acc[5]),
                             pack_bf2(acc[6], acc[7]));
        *reinterpret_cast<uint4*>(out + (size_t)t * H + f) = o;
    }
}

// counts[e] += 1 per route; ids outside [0, E) are skipped and flagged
__global__ void k_histogram(const int32_t* __restrict__ ids, int n, int E, int32_t* __restrict__ counts,
                            int* __restrict__ err) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        int e = ids[i];
        if (e >= 0 && e < E) atomicAdd(counts + e, 1);
        else atomicExch(err, kDevBadRoute);
    }
}

__global__ void k_gather_rows(const uint16_t* __restrict__ y, const int32_t* __restrict__ slot_of, int H,
                              uint16_t* __restrict__ out) {
    const int i = blockIdx.x;
    const int slot = slot_of[i];
    for (int f = threadIdx.x * 8; f < H; f += blockDim.x * 8)
        *reinterpret_cast<uint4*>(out + (size_t)i * H + f) =
            __ldg(reinterpret_cast<const uint4*>(y + (size_t)slot * H + f));
}

__global__ void k_tile_rows(const uint16_t* __restrict__ x, int n, int cols, int atoms, uint16_t* __restrict__ dst) {
    const int r = blockIdx.x;  // rows [n, pad16(n)) are zero-filled
    for (int c = threadIdx.x * 8; c < cols; c += blockDim.x * 8) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < n) v = __ldg(reinterpret_cast<const uint4*>(x + (size_t)r * cols + c));
        *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(dst) + tiled_off(r, c, atoms)) = v;
    }
}

}  // namespace

cudaError_t launch_dispatch(const int32_t* ids, const uint16_t* x, int T, const Shape& sh, const DispatchBufs& d,
                            int permute, cudaStream_t st, const uint16_t* const* row_src) {
    {
        const cudaError_t le_ = launch_pdl(k_dispatch, dim3(sh.E), dim3(kDispThreads), 0, st, ids, T, sh.E, sh.K, d);
        if (le_ != cudaSuccess) return le_;
    }
    if (!permute) return cudaGetLastError();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    {
        const cudaError_t le_ =
            launch_pdl(k_permute, dim3(d.atoms), dim3(256), 0, st, x, sh.H, d.src, d.seg + sh.E, d.atoms, d.xp, row_src);
        if (le_ != cudaSuccess) return le_;
    }  // 8 rows per CTA
    return cudaGetLastError();
}

cudaError_t launch_combine(const uint16_t* y, int y_ld, const int32_t* slot_of, const float* w,
                           const uint16_t* residual, int T, int H, int K, uint16_t* out, cudaStream_t st,
                           const uint16_t* y_local, int32_t* local) {
    if (T <= 0) return cudaSuccess;
    if (K > kCombineMaxK) return cudaErrorInvalidValue;
    {
        const cudaError_t le_ =
            launch_pdl(k_combine, dim3(T), dim3(256), 0, st, y, y_ld, slot_of, w, residual, H, K, out, y_local, local);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm(const uint16_t* x, const uint16_t* w, int T, int H, float eps, uint16_t* out,
                           cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    {
        const cudaError_t le_ = launch_pdl(k_rmsnorm, dim3(T), dim3(256), 0, st, x, w, H, eps, out);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

cudaError_t launch_histogram(const int32_t* ids, int n, int E, int32_t* counts, int* err, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    note_launch();
    k_histogram<<<(n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024, 256, 0, st>>>(ids, n, E, counts, err);
    return cudaGetLastError();
}

cudaError_t launch_gather_rows(const uint16_t* y, const int32_t* slot_of, int rows, int H, uint16_t* out,
                               cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    note_launch();
    k_gather_rows<<<rows, 256, 0, st>>>(y, slot_of, H, out);
    return cudaGetLastError();
}

cudaError_t launch_tile_rows(const uint16_t* x, int n, int cols, int atoms, uint16_t* dst, cudaStream_t st) {
    int rows = (n + kSegAlign - 1) / kSegAlign * kSegAlign;
    if (rows <= 0) return cudaSuccess;
    note_launch();
    k_tile_rows<<<rows, 256, 0, st>>>(x, n, cols, atoms, dst);
    return cudaGetLastError();
}

}  // namespace obs
