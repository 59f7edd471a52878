// k_ep.cu -- expert parallelism over NVLink peer memory.
//
// The reference runs every expert on one device (src/forward.rs:164-247); on a
// multi-GPU box the experts are split across G ranks (rank g holds experts
// [g*E/G, (g+1)*E/G)) and the routed token rows travel to the rank that holds
// their expert and back.  Each rank owns one device buffer (opened by its peers
// through CUDA IPC) laid out identically on every rank:
//   recv_x  [G][cap][H] bf16   rows sent to this rank, one region per source
//   meta    [G][cap] int2      (local expert, source item t*K+k) of each row
//   cnt     [G] int32          rows in each source region
//   rflag   [G] uint32         epoch stamp: source s finished writing
//   ret_y   [cap][H] bf16      this rank's expert outputs, indexed by item t*K+k
//   retflag [G] uint32         epoch stamp: rank d finished returning
// cap = max_tokens * top_k.  A forward writes peers' memory directly with plain
// stores (k_ep_send, k_ep_return), then a system-scope fence and a release store
// of the epoch stamp; readers spin (bounded, 2 s) on acquire loads of the stamps.
// The epoch lives in device memory (incremented by the last kernel of each
// forward), so a captured CUDA graph replays correctly.  Buffer reuse needs no
// extra handshake: a source writes forward e+1's rows to a peer only after its
// own forward e finished, which waited for that peer's returns of e, which that
// peer issued after it had consumed the received rows of e.
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

// One warp per routed item (t, k): copy row x[t] into the owning rank's region
// for this source, with its metadata.  The last CTA to finish publishes the
// per-destination counts and stamps.
__global__ void __launch_bounds__(256) k_ep_send(const int32_t* __restrict__ ids, const uint16_t* __restrict__ x,
                                                 int T, int E, EpArgs a) {
    pdl_begin();
    __shared__ int s_last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t e = *a.epoch + 1;
    const int item = blockIdx.x * 8 + warp;
    if (item < T * a.K) {
        int id = ids[item];
        if (id < 0 || id >= E) {
            if (lane == 0) atomicExch(a.err, kDevBadRoute);
            id = 0;
        }
        const int dest = id / a.E_local, le = id - dest * a.E_local;
        int slot = 0;
        if (lane == 0) slot = atomicAdd(a.send_cnt + dest, 1);
        slot = __shfl_sync(0xffffffffu, slot, 0);
        if (slot < a.cap) {
            uint8_t* pb = a.peer[dest];
            const size_t row = (size_t)a.rank * a.cap + slot;
            const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(item / a.K) * a.H);
            uint4* dst = at<uint4>(pb, a.off_rx + row * a.H * 2);
            for (int c = lane; c < a.H / 8; c += 32) dst[c] = __ldg(src + c);
            if (lane == 0) *at<int2>(pb, a.off_meta + row * 8) = make_int2(le, item);
        } else if (lane == 0) {
            atomicExch(a.err, kDevBadSlot);  // more rows than the source's region holds: refused
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
        const int n = min(ld_volatile(a.send_cnt + d), a.cap);
        *at<int32_t>(a.peer[d], a.off_cnt + (size_t)a.rank * 4) = n;
        __threadfence_system();
        st_release_sys(at<uint32_t>(a.peer[d], a.off_rflag + (size_t)a.rank * 4), e);
        a.send_cnt[d] = 0;
    }
    if (threadIdx.x == 0) a.done[0] = 0;
}

// Wait for every source's stamp, then turn the received rows into a local
// routing problem: ids_local[s*cap + i] = local expert of row i of source s
// (-1 beyond the source's count) and a histogram per local expert.
__global__ void __launch_bounds__(256) k_ep_recv(EpArgs a) {
    pdl_begin();
    const uint32_t e = *a.epoch + 1;
    uint8_t* mine = a.peer[a.rank];
    if (!wait_stamps(at<uint32_t>(mine, a.off_rflag), a.world, e, a.err, a.wait_ns)) return;
    const int n = a.world * a.cap;
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x) {
        const int s = j / a.cap, i = j - s * a.cap;
        const int cnt = min(ld_volatile(at<int32_t>(mine, a.off_cnt) + s), a.cap);
        int le = -1, item = -1;
        if (i < cnt) {
            const int2 m = *at<int2>(mine, a.off_meta + (size_t)j * 8);
            le = m.x, item = m.y;
            if (le < 0 || le >= a.E_local || item < 0 || item >= a.cap) {
                atomicExch(a.err, kDevBadRoute);
                le = -1;
            } else {
                atomicAdd(a.counts + le, 1);
            }
        }
        a.ids_local[j] = le;
        a.src_item[j] = item;
    }
}

// One warp per received row: its expert output (local slot slot_of[j]) goes back
// to the source rank's ret_y at the row's item index.  The last CTA stamps every
// source.
__global__ void __launch_bounds__(256) k_ep_return(const int32_t* __restrict__ slot_of, const uint16_t* __restrict__ y,
                                                   EpArgs a) {
    pdl_begin();
    __shared__ int s_last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t e = *a.epoch + 1;
    const int n = a.world * a.cap;
    for (int j = blockIdx.x * 8 + warp; j < n; j += gridDim.x * 8) {
        if (a.ids_local[j] < 0) continue;
        const int s = j / a.cap, item = a.src_item[j], slot = slot_of[j];
        if (slot < 0 || slot >= a.rows_cap || item < 0 || item >= a.cap) {  // refused, recorded
            if (lane == 0) atomicExch(a.err, kDevBadSlot);
            continue;
        }
        const uint4* src = reinterpret_cast<const uint4*>(y + (size_t)slot * a.H);
        uint4* dst = at<uint4>(a.peer[s], a.off_ret + (size_t)item * a.H * 2);
        for (int c = lane; c < a.H / 8; c += 32) dst[c] = src[c];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(a.done + 1, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence_system();  // pairs with the other CTAs' fences: their row stores precede the stamps
    if (threadIdx.x < a.world) st_release_sys(at<uint32_t>(a.peer[threadIdx.x], a.off_retflag + (size_t)a.rank * 4), e);
    if (threadIdx.x == 0) a.done[1] = 0;
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
    const int items = T * a.K;
    const int grid = items > 0 ? (items + 7) / 8 : 1;  // one CTA at least: it publishes the counts
    {
        const cudaError_t le_ = launch_pdl(k_ep_send, dim3(grid), dim3(256), 0, st, ids, x, T, E, a);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

cudaError_t launch_ep_recv(const EpArgs& a, cudaStream_t st) {
    const int n = a.world * a.cap;
    const int grid = (n + 255) / 256 < 296 ? (n + 255) / 256 : 296;
    {
        const cudaError_t le_ = launch_pdl(k_ep_recv, dim3(grid), dim3(256), 0, st, a);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

cudaError_t launch_ep_return(const int32_t* slot_of, const uint16_t* y, const EpArgs& a, cudaStream_t st) {
    const int n = a.world * a.cap;
    const int grid = (n + 7) / 8 < 1184 ? (n + 7) / 8 : 1184;
    {
        const cudaError_t le_ = launch_pdl(k_ep_return, dim3(grid), dim3(256), 0, st, slot_of, y, a);
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
