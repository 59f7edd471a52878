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

constexpr int kDispThreads = kDispChunk;  // one token per thread and chunk
constexpr int kDispMaxE = 256;           // the context accepts n_experts <= 256

__device__ __forceinline__ int pad_rows(int c) { return (c + kSegAlign - 1) / kSegAlign * kSegAlign; }

// grid = token chunks of kDispChunk; hist[c][e] = routes of chunk c's tokens to
// expert e (every entry written, so nothing needs zeroing).  An id of -1 is "no
// expert" when allow_none (expert parallelism: slots of received rows without a
// local expert); any other id outside [0, E) is recorded and skipped.
__global__ void __launch_bounds__(kDispThreads) k_chunk_hist(const int32_t* ids, int T, int E, int K,
                                                             int allow_none, int32_t* __restrict__ hist,
                                                             int* __restrict__ err) {
    pdl_begin();
    __shared__ int s_h[kDispMaxE];
    for (int i = threadIdx.x; i < E; i += kDispThreads) s_h[i] = 0;
    __syncthreads();
    const int t = blockIdx.x * kDispChunk + threadIdx.x;
    if (t < T)
        for (int k = 0; k < K; ++k) {
            const int e = ids[(size_t)t * K + k];
            if (e >= 0 && e < E) atomicAdd(&s_h[e], 1);
            else if (!(allow_none && e == -1)) atomicExch(err, kDevBadRoute);
        }
    __syncthreads();
    for (int i = threadIdx.x; i < E; i += kDispThreads) hist[(size_t)blockIdx.x * E + i] = s_h[i];
}

// grid = (E, chunks): CTA (e, c) places chunk c's tokens routed to expert e.
// Slots are ordered by expert, then token: the CTA's first slot is the padded
// segment start of e (from the totals of the experts before it) plus the routes
// to e of the chunks before c; inside the chunk a ballot compaction keeps token
// order.  The c = 0 CTAs also write e's padding rows, GEMM token tiles and
// segment start, and counts[e].
__global__ void __launch_bounds__(kDispThreads) k_dispatch(const int32_t* ids, int T, int E, int K,
                                                           const int32_t* hist, DispatchBufs d) {
    pdl_begin();
    __shared__ int s_cnt[kDispMaxE];
    __shared__ int s_red[3][kDispThreads / 32];
    __shared__ int s_warp[kDispThreads / 32];
    const int e = blockIdx.x, c = blockIdx.y, C = gridDim.y, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int bn = d.bn;

    // totals of experts 0..e, and the routes to e of the chunks before c
    for (int i = tid; i <= e; i += kDispThreads) s_cnt[i] = 0;
    __syncthreads();
    int before_c = 0;
    for (int j = tid; j < (e + 1) * C; j += kDispThreads) {
        const int ee = j / C, cc = j - ee * C;
        const int v = hist[(size_t)cc * E + ee];
        atomicAdd(&s_cnt[ee], v);
        if (ee == e && cc < c) before_c += v;
    }
    __syncthreads();
    int my_seg = 0, my_tiles = 0;
    for (int i = tid; i < e; i += kDispThreads) {
        const int p = pad_rows(s_cnt[i]);
        my_seg += p;
        my_tiles += (p + bn - 1) / bn;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        my_seg += __shfl_xor_sync(0xffffffffu, my_seg, o);
        my_tiles += __shfl_xor_sync(0xffffffffu, my_tiles, o);
        before_c += __shfl_xor_sync(0xffffffffu, before_c, o);
    }
    if (lane == 0) s_red[0][wid] = my_seg, s_red[1][wid] = my_tiles, s_red[2][wid] = before_c;
    __syncthreads();
    int seg = 0, tile0 = 0, base = 0;
    for (int i = 0; i < kDispThreads / 32; ++i) seg += s_red[0][i], tile0 += s_red[1][i], base += s_red[2][i];
    const int cnt = s_cnt[e];
    const int P = pad_rows(cnt);
    const int ntile = (P + bn - 1) / bn;

    // stable ordered compaction of the chunk's tokens routed to e
    const int t = c * kDispChunk + tid;
    int kfound = -1;
    if (t < T)
        for (int k = 0; k < K; ++k)
            if (ids[(size_t)t * K + k] == e) kfound = k;
    const unsigned bal = __ballot_sync(0xffffffffu, kfound >= 0);
    if (lane == 0) s_warp[wid] = __popc(bal);
    __syncthreads();
    int before = 0;
    for (int i = 0; i < wid; ++i) before += s_warp[i];
    if (kfound >= 0) {
        const int slot = seg + base + before + __popc(bal & ((1u << lane) - 1u));
        if (slot < d.rows_cap) {
            d.slot_of[(size_t)t * K + kfound] = slot;
            d.src[slot] = t;
        } else {
            refuse_slot(d.err, kSiteDispatch, slot);  // more routed rows than the row buffers hold: refused
        }
    }
    if (c != 0) return;
    for (int r = cnt + tid; r < P && seg + r < d.rows_cap; r += kDispThreads) d.src[seg + r] = -1;
    for (int j = tid; j < ntile && tile0 + j < d.max_tiles; j += kDispThreads)
        d.tiles[tile0 + j] = make_int4(e, seg + j * bn, min(bn, P - j * bn), 0);
    if (e == E - 1 && tid == 0) {
        *d.n_tiles = tile0 + ntile;
        d.seg[E] = seg + P;
    }
    if (tid == 0) d.seg[e] = seg, d.counts[e] = cnt;
}

// The routed rows (slot order) into the tiled activation layout the grouped
// GEMM reads with bulk copies: one warp per slot row, 16-byte chunks (coalesced
// 512-byte reads of the source row, 128-byte runs per k-group in the
// destination); padding rows (src = -1) are written as zeros.  Token t's row is
// x[t], or row_src[t] when given (expert parallelism: received rows live in
// the exchange buffer, the rank's own in x).
__device__ __forceinline__ void permute_row(const uint16_t* x, int H, int T, const int32_t* src,
                                            int atoms, uint16_t* __restrict__ xp,
                                            const uint16_t* const* row_src, int row, int lane,
                                            int* __restrict__ err) {
    int t = src[row];
    const uint16_t* xrow = t >= 0 && t < T ? (row_src ? row_src[t] : x + (size_t)t * H) : nullptr;
    if (t >= 0 && !xrow) {  // a token outside the batch or a row without data: zeros, recorded
        if (lane == 0) refuse_slot(err, kSitePermute, row);
        t = -1;
    }
    const int chunks = H / 8;
    for (int c0 = lane; c0 < chunks; c0 += 32 * 8) {  // H = 2048: the whole row in flight at once
        uint4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int c = c0 + 32 * u;
            v[u] = make_uint4(0, 0, 0, 0);
            if (t >= 0 && c < chunks) v[u] = reinterpret_cast<const uint4*>(xrow)[c];
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int c = c0 + 32 * u;
            if (c < chunks) *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(xp) + tiled_off(row, c * 8, atoms)) = v[u];
        }
    }
}

__global__ void __launch_bounds__(256) k_permute(const uint16_t* x, int H, int T,
                                                 const int32_t* src, const int32_t* seg_end,
                                                 int atoms, uint16_t* __restrict__ xp,
                                                 const uint16_t* const* row_src, int* __restrict__ err) {
    pdl_begin();
    const int lane = threadIdx.x & 31, end = min(*seg_end, atoms * 8);
    for (int row = blockIdx.x * 8 + (threadIdx.x >> 5); row < end; row += gridDim.x * 8)
        permute_row(x, H, T, src, atoms, xp, row_src, row, lane, err);
}

// The MoE stack's layer-input RMSNorm (rmsnorm.metal:9-37), in the reference
// kernel's own order: 256 threads per row, thread l sums v*v (rounded product,
// rounded add) over elements l, l+256, ...; the partials meet in the halving
// tree sq[l] += sq[l + s], s = 128 .. 1; rms = sqrt(sq[0] / H + eps);
// out = (x / rms) * w.  IEEE divide and square root, as the oracle.
__global__ void __launch_bounds__(256) k_rmsnorm(const uint16_t* x, const uint16_t* __restrict__ w,
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

__global__ void __launch_bounds__(256) k_combine(const uint16_t* y, int y_ld,
                                                 const int32_t* slot_of, const float* w,
                                                 const uint16_t* residual, int H, int K,
                                                 uint16_t* __restrict__ out, const uint16_t* y_local,
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
            uint4 r = *reinterpret_cast<const uint4*>(residual + (size_t)t * H + f);
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
                if (k0 + kk < K) v[kk] = *reinterpret_cast<const uint4*>(s_row[k0 + kk] + f);
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
                            int permute, cudaStream_t st, const uint16_t* const* row_src, int allow_none) {
    const int C = T > 0 ? (T + kDispChunk - 1) / kDispChunk : 1;
    if (C > d.max_chunks || sh.E > kDispMaxE) return cudaErrorInvalidValue;
    {
        const cudaError_t le_ = launch_pdl(k_chunk_hist, dim3(C), dim3(kDispThreads), 0, st, ids, T, sh.E, sh.K,
                                           allow_none, d.hist, d.err);
        if (le_ != cudaSuccess) return le_;
    }
    {
        const cudaError_t le_ =
            launch_pdl(k_dispatch, dim3(sh.E, C), dim3(kDispThreads), 0, st, ids, T, sh.E, sh.K, (const int32_t*)d.hist, d);
        if (le_ != cudaSuccess) return le_;
    }
    if (!permute) return cudaGetLastError();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    {
        // 8 rows per CTA and pass; 1184 CTAs = 148 SMs x 8 resident
        const int grid = d.atoms < 1184 ? d.atoms : 1184;
        const cudaError_t le_ =
            launch_pdl(k_permute, dim3(grid), dim3(256), 0, st, x, sh.H, T, d.src, d.seg + sh.E, d.atoms, d.xp, row_src,
                       d.err);
        if (le_ != cudaSuccess) return le_;
    }
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
