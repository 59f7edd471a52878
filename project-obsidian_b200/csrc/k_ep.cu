// k_ep.cu -- expert parallelism over NVLink peer memory.
//
// The reference runs every expert on one device (src/forward.rs:164-247); on a
// multi-GPU box the experts are split across G ranks (E/G each) and the routed
// token rows travel to the ranks that hold their experts and the expert
// outputs travel back.  A token row is sent to a
// rank once, however many of its K experts live there, with the list of those
// experts (local id and rank-order position k) as metadata; the outputs come
// back once per (token, expert) pair, since each pair's output is distinct --
// written by the down GEMM's epilogue straight into the source rank's memory,
// so the return all-to-all overlaps the GEMM tile by tile.  Rows and outputs
// that stay on their rank are not copied at all.
//
// Which rank holds which expert is a per-layer table (obs_ep_set_placement; by
// default rank g holds experts [g*E/G, (g+1)*E/G)): a balanced placement keeps
// the busiest rank's GEMMs, which every rank's combine waits for, short under a
// skewed expert load.
//
// Each rank owns one device buffer (opened by its peers through CUDA IPC) laid
// out identically on every rank:
//   recv_x  [G][cap_rows][H] bf16  rows sent to this rank, one region per source
//   meta    [G][cap_rows][16] int16  per row: (k << 8 | local expert) of each of
//                                  the token's experts here, -1 elsewhere
//   mtok    [G][cap_rows] int32    the row's token index at its source
//   cnt     [G] int32              rows in each source region
//   rflag   [G] uint32             epoch stamp: source s finished writing
//   ret_y   [cap_items][H] bf16    this rank's expert outputs, indexed by item t*K+k
//   retflag [G] uint32             epoch stamp: rank d finished returning
// cap_rows = max_tokens, cap_items = max_tokens * top_k.  A forward writes
// peers' memory directly with plain stores, then a system-scope fence and a
// release store of the epoch stamp; readers spin (bounded) on acquire loads of
// the stamps.  The epoch lives in device memory (incremented by the last kernel
// of each forward), so a captured CUDA graph replays correctly.  Buffer reuse
// needs no extra handshake: a source writes forward e+1's rows to a peer only
// after its own forward e finished, which waited for that peer's returns of e,
// which that peer issued after it had consumed the received rows of e.
#include "obs_internal.cuh"

namespace obs {
namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int ld_volatile(const int32_t* p) { return *reinterpret_cast<const volatile int32_t*>(p); }

// threads [0, world) wait until stamp[t] == e (bounded); false on timeout
__device__ bool wait_stamps(const uint32_t* stamps, int world, uint32_t e, int* err, uint64_t limit_ns) {
    __shared__ int s_bad;
    if (threadIdx.x == 0) s_bad = 0;
    __syncthreads();
    if (threadIdx.x < world) {
        const uint64_t t0 = global_ns();
        while (ld_acquire_sys(stamps + threadIdx.x) != e) {
            if (global_ns() - t0 > limit_ns) {
                s_bad = 1;
                atomicExch(err, kDevTimeout);
                break;
            }
        }
    }
    __syncthreads();
    return s_bad == 0;
}

template <typename T>
__device__ __forceinline__ T* at(uint8_t* base, size_t off) {
    return reinterpret_cast<T*>(base + off);
}

constexpr int kSendPiece = 2048, kSendChunks = kSendPiece / 8 / 32;  // 16-byte chunks per lane and piece

// One warp per token: for every rank that holds one or more of the token's K
// experts, one copy of row x[t] into that rank's region for this source, with
// the (k, local expert) list and the token index -- for this rank itself only
// the list and the index: the permute reads the row from x.  The last CTA to
// finish publishes the per-destination counts and stamps.
__global__ void __launch_bounds__(256) k_ep_send(const int32_t* ids, const uint16_t* x,
                                                 int T, int E, EpArgs a) {
    pdl_begin();
    __shared__ int s_last;
    __shared__ int s_slot[8][kMaxWorld];  // per warp: the row's slot at each rank, -1 = not sent there
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t e = *a.epoch + 1;
    const int t = blockIdx.x * 8 + warp;
    if (t < T) {
        int id = lane < a.K ? ids[(size_t)t * a.K + lane] : 0;
        int slot_e = lane < a.K && id >= 0 && id < E ? a.place[id] : 0;
        if (lane < a.K && (id < 0 || id >= E || slot_e < 0 || slot_e >= E)) {
            atomicExch(a.err, kDevBadRoute);
            slot_e = 0;
        }
        const int dest = lane < a.K ? slot_e / a.E_local : -1;
        const int le = lane < a.K ? slot_e - dest * a.E_local : 0;
        // the destinations of the row (a bit per rank); lane d takes the slot at rank d, all in parallel
        const unsigned need = __reduce_or_sync(0xffffffffu, dest >= 0 ? 1u << dest : 0u);
        int slot = -1;
        if (lane < a.world && (need >> lane & 1u)) {
            slot = atomicAdd(a.send_cnt + lane, 1);
            if (slot >= a.cap_rows) {
                refuse_slot(a.err, kSiteSendFull, slot);  // more rows than the source's region holds: refused
                slot = -1;
            }
        }
        if (lane < kMaxWorld) s_slot[warp][lane] = slot;
        __syncwarp();
        // the (k, local expert) list and the token index at every destination
        for (int d = 0; d < a.world; ++d) {
            const int sd = s_slot[warp][d];
            if (sd < 0) continue;
            uint8_t* pb = a.peer[d];
            const size_t row = (size_t)a.rank * a.cap_rows + sd;
            if (lane < 16) at<int16_t>(pb, a.off_meta + row * 32)[lane] = (int16_t)(dest == d ? (lane << 8) | le : -1);
            if (lane == 0) at<int32_t>(pb, a.off_mtok + row * 4)[0] = t;
        }
        // the row to every remote destination, in pieces of 2048 columns: each piece in registers
        // once, then independent 16-byte stores.  Each token starts at a different peer (offset
        // 1 + t mod (world - 1) from this rank), so the warps of all ranks spread their stores over
        // the peers instead of all writing to the same GPU at once.
        if (need & ~(1u << a.rank)) {
            const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * a.H);
            for (int c0 = 0; c0 < a.H / 8; c0 += 32 * kSendChunks) {
                uint4 v[kSendChunks];
#pragma unroll
                for (int u = 0; u < kSendChunks; ++u) v[u] = src[c0 + lane + 32 * u];
                for (int i = 0; i < a.world - 1; ++i) {
                    const int d = (a.rank + 1 + (i + t) % (a.world - 1)) % a.world;  // every peer once
                    const int sd = s_slot[warp][d];
                    if (sd < 0) continue;
                    const size_t row = (size_t)a.rank * a.cap_rows + sd;
                    uint4* dst = at<uint4>(a.peer[d], a.off_rx + row * a.H * 2) + c0 + lane;
#pragma unroll
                    for (int u = 0; u < kSendChunks; ++u) dst[32 * u] = v[u];
                }
            }
        }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(a.done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    // pairs with every CTA's system fence before its count: their row stores and
    // slot counts are ordered before the stamps below
    __threadfence_system();
    if (threadIdx.x < a.world) {
        const int d = threadIdx.x;
        const int n = min(ld_volatile(a.send_cnt + d), a.cap_rows);
        *at<int32_t>(a.peer[d], a.off_cnt + (size_t)a.rank * 4) = n;
        __threadfence_system();
        st_release_sys(at<uint32_t>(a.peer[d], a.off_rflag + (size_t)a.rank * 4), e);
        a.send_cnt[d] = 0;
    }
    if (threadIdx.x == 0) a.done[0] = 0;
}

// Wait for every source's stamp, then turn the received rows into a local
// routing problem of W*cap_rows "tokens" with K slots each:
// ids_local[row*K + k] = local expert of slot k of the row (-1: none, or beyond
// the source's count) and src_item = the source's item t*K + k.  The rows this rank sent itself are read from x: row_src[row] is
// the row to permute, x[t] for its own region, recv_x[row] otherwise.
__global__ void __launch_bounds__(256) k_ep_recv(const uint16_t* x, EpArgs a) {
    pdl_begin();
    const uint32_t e = *a.epoch + 1;
    uint8_t* mine = a.peer[a.rank];
    if (!wait_stamps(at<uint32_t>(mine, a.off_rflag), a.world, e, a.err, a.wait_ns)) return;
    const int n = a.world * a.cap_rows * a.K;
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x) {
        const int row = j / a.K, kk = j - row * a.K;
        const int s = row / a.cap_rows, i = row - s * a.cap_rows;
        const int cnt = min(ld_volatile(at<int32_t>(mine, a.off_cnt) + s), a.cap_rows);
        int le = -1, item = -1;
        if (i < cnt) {
            const int code = at<int16_t>(mine, a.off_meta + (size_t)row * 32)[kk];
            const int t = at<int32_t>(mine, a.off_mtok + (size_t)row * 4)[0];
            if (kk == 0 && t >= 0 && t < a.cap_rows)
                a.row_src[row] = s == a.rank ? x + (size_t)t * a.H
                                             : at<uint16_t>(mine, a.off_rx + (size_t)row * a.H * 2);
            if (code >= 0) {
                const int l = code & 0xFF, k = code >> 8;
                if (l >= a.E_local || k >= a.K || t < 0 || t >= a.cap_rows) {
                    atomicExch(a.err, kDevBadRoute);
                } else {
                    le = l, item = t * a.K + k;
                }
            }
        }
        a.ids_local[j] = le;
        a.src_item[j] = item;
    }
}

// Every output row (slot) of the down GEMM gets its destination before the
// GEMM runs.  The slots below the dispatch's padded end are of two disjoint
// kinds: padding rows (src < 0), which stay in this rank's y, and exactly one
// received (row, k) pair each, whose output goes to its source rank's ret_y row
// (item t*K + k) over NVLink -- or, for this rank's own items, stays in y and is
// noted in local_slot for the combine.
__global__ void __launch_bounds__(256) k_ep_rowptr(const int32_t* slot_of,
                                                   const int32_t* src, const int32_t* seg_end,
                                                   uint16_t* y, uint16_t** __restrict__ row_ptr, EpArgs a) {
    pdl_begin();
    const int total = min(*seg_end, a.rows_cap), n = a.world * a.cap_rows * a.K;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total + n; i += gridDim.x * blockDim.x) {
        if (i < total) {
            if (src[i] < 0) row_ptr[i] = y + (size_t)i * a.H;
            continue;
        }
        const int j = i - total;
        if (a.ids_local[j] < 0) continue;
        const int s = j / (a.K * a.cap_rows), item = a.src_item[j], slot = slot_of[j];
        if (slot < 0 || slot >= total) {  // refused, recorded
            refuse_slot(a.err, kSiteRowSlot, slot * 65536 + total);
            continue;
        }
        if (item < 0 || item >= a.cap_items) {
            refuse_slot(a.err, kSiteRowItem, item);
            continue;
        }
        if (s == a.rank) {
            row_ptr[slot] = y + (size_t)slot * a.H;
            a.local_slot[item] = slot + 1;
        } else {
            row_ptr[slot] = at<uint16_t>(a.peer[s], a.off_ret + (size_t)item * a.H * 2);
        }
    }
}

// The down GEMM wrote every output row to its destination and fenced its stores
// system-wide: stamp every source.
__global__ void k_ep_returned(EpArgs a) {
    pdl_begin();
    const uint32_t e = *a.epoch + 1;
    __threadfence_system();
    if (threadIdx.x < a.world) st_release_sys(at<uint32_t>(a.peer[threadIdx.x], a.off_retflag + (size_t)a.rank * 4), e);
}

// The failure path of the peer waits, without peers: one wait on a stamp that
// nothing writes runs out after limit_ns and records the timeout, exactly as a
// k_ep_recv whose peer never sends would (obs_probe_wait).
__global__ void k_probe_wait(const uint32_t* stamp, uint64_t limit_ns, int* err) {
    wait_stamps(stamp, 1, 1u, err, limit_ns);
}

// Wait until every rank has returned this rank's rows, then close the epoch.
__global__ void k_ep_finish(EpArgs a) {
    pdl_begin();
    const uint32_t e = *a.epoch + 1;
    wait_stamps(at<uint32_t>(a.peer[a.rank], a.off_retflag), a.world, e, a.err, a.wait_ns);
    if (threadIdx.x == 0) *a.epoch = e;
}

}  // namespace

cudaError_t launch_ep_send(const int32_t* ids, const uint16_t* x, int T, int E, const EpArgs& a, cudaStream_t st) {
    if (a.K > 16 || a.H % kSendPiece) return cudaErrorInvalidValue;  // 16 metadata slots per row; whole pieces
    const int grid = T > 0 ? (T + 7) / 8 : 1;   // one warp per token; one CTA at least: it publishes the counts
    {
        const cudaError_t le_ = launch_pdl(k_ep_send, dim3(grid), dim3(256), 0, st, ids, x, T, E, a);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

cudaError_t launch_ep_recv(const uint16_t* x, const EpArgs& a, cudaStream_t st) {
    const int n = a.world * a.cap_rows * a.K;
    const int grid = (n + 255) / 256 < 296 ? (n + 255) / 256 : 296;
    {
        const cudaError_t le_ = launch_pdl(k_ep_recv, dim3(grid), dim3(256), 0, st, x, a);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

cudaError_t launch_ep_rowptr(const int32_t* slot_of, const int32_t* src, const int32_t* seg_end, uint16_t* y,
                             uint16_t** row_ptr, const EpArgs& a, cudaStream_t st) {
    const int n = a.rows_cap + a.world * a.cap_rows * a.K;
    const int grid = (n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184;
    {
        const cudaError_t le_ =
            launch_pdl(k_ep_rowptr, dim3(grid), dim3(256), 0, st, slot_of, src, seg_end, y, row_ptr, a);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

cudaError_t launch_ep_returned(const EpArgs& a, cudaStream_t st) {
    {
        const cudaError_t le_ = launch_pdl(k_ep_returned, dim3(1), dim3(32), 0, st, a);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

cudaError_t launch_probe_wait(const uint32_t* stamp, uint64_t limit_ns, int* err, cudaStream_t st) {
    note_launch();
    k_probe_wait<<<1, 32, 0, st>>>(stamp, limit_ns, err);
    return cudaGetLastError();
}

cudaError_t launch_ep_finish(const EpArgs& a, cudaStream_t st) {
    {
        const cudaError_t le_ = launch_pdl(k_ep_finish, dim3(1), dim3(32), 0, st, a);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

}  // namespace obs
