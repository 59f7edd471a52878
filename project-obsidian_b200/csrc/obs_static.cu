// obs_static.cu -- obs_decode_ffn_static: the decode expert FFN + combine for
// callers that cannot allocate device memory.
//
// Some callers cannot call cudaMalloc: code running while a CUDA graph is being
// captured (allocation is not a stream operation and is refused there), hosts
// whose framework owns all device memory through its own arena and forbids
// side allocations, and latency-critical loops that cannot afford the implicit
// synchronisation an allocation may cause.  This entry point needs no context
// and no allocation: its scratch (split-K partial sums, the SwiGLU outputs h,
// the per-expert outputs y, the arrival counters and an error word) lives in
// one file-scope device array of fixed size, present on every GPU that loads
// the library until the process exits.  (The scratch also holds the fixed-point
// forms of x and h that the decode kernels compute with.)
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/obs_moe.h"
#include "obs_internal.cuh"

namespace obs {
cudaError_t launch_decode_ffn_mlx(const uint32_t* gw, const uint16_t* gs, const uint16_t* gb, const uint32_t* uw,
                                  const uint16_t* us, const uint16_t* ub, const uint32_t* dw, const uint16_t* ds,
                                  const uint16_t* db, const Shape& sh, const uint16_t* x, const int32_t* ids,
                                  const float* w, const uint16_t* residual, int T, const DecodeBufs& d, uint16_t* out,
                                  cudaStream_t st);
void set_thread_error(const char* msg);
}  // namespace obs

namespace {
// scratch layout for the largest allowed call (OBS_STATIC_MAX_*)
constexpr size_t kPartBytes = (size_t)OBS_STATIC_MAX_PAIRS * (OBS_STATIC_MAX_INTER / 128) * obs::kDecodeSplit * 2 * 128 * 4;
constexpr size_t kCntGuBytes = (size_t)OBS_STATIC_MAX_PAIRS * (OBS_STATIC_MAX_INTER / 128) * 4;
constexpr size_t kCntDnBytes = (size_t)OBS_STATIC_MAX_PAIRS * (OBS_STATIC_MAX_HIDDEN / 128) * 4;
constexpr size_t kErrBytes = 256;
constexpr size_t kHBytes = (size_t)OBS_STATIC_MAX_PAIRS * OBS_STATIC_MAX_INTER * 2;  // h in fixed point
constexpr size_t kHMetaBytes = (size_t)OBS_STATIC_MAX_PAIRS * (OBS_STATIC_MAX_INTER / 64) * 8;
constexpr size_t kXBytes = (size_t)OBS_STATIC_MAX_PAIRS * OBS_STATIC_MAX_HIDDEN * 2;  // x in fixed point (T <= pairs)
constexpr size_t kXMetaBytes = (size_t)OBS_STATIC_MAX_PAIRS * (OBS_STATIC_MAX_HIDDEN / 64) * 8;
constexpr size_t kYBytes = (size_t)OBS_STATIC_MAX_PAIRS * OBS_STATIC_MAX_HIDDEN * 2;
// counters and the error word first: one memset clears everything that must start at zero
constexpr size_t kOffCntGu = 0;
constexpr size_t kOffCntDn = kOffCntGu + kCntGuBytes;
constexpr size_t kOffErr = kOffCntDn + kCntDnBytes;
constexpr size_t kZeroBytes = kOffErr + kErrBytes;
constexpr size_t kOffPart = (kZeroBytes + 255) / 256 * 256;
constexpr size_t kOffH = kOffPart + kPartBytes;
constexpr size_t kOffHMeta = kOffH + kHBytes;
constexpr size_t kOffX = kOffHMeta + kHMetaBytes;
constexpr size_t kOffXMeta = kOffX + kXBytes;
constexpr size_t kOffY = kOffXMeta + kXMetaBytes;
constexpr size_t kScratchBytes = kOffY + kYBytes;  // about 8 MB
constexpr int kMaxDevices = 64;

std::mutex g_mu;
uint8_t* g_scratch_addr[kMaxDevices] = {};  // per device, from cudaGetSymbolAddress
}  // namespace

// The scratch.  Host code must not use this name as an address: it is a
// host-side stand-in; the device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t g_decode_scratch[kScratchBytes];

static int fail(int code, const char* msg) {
    obs::set_thread_error(msg);
    return code;
}

// Once per device, with that device current: the array's device address.
static int scratch_for_current_device(uint8_t** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return fail(OBS_ERR_CUDA, "cudaGetDevice failed");
    if (dev < 0 || dev >= kMaxDevices) return fail(OBS_ERR_UNSUPPORTED, "device index above 63");
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (e != cudaSuccess || !p) return fail(OBS_ERR_CUDA, cudaGetErrorString(e));
        g_scratch_addr[dev] = static_cast<uint8_t*>(p);
    }
    *out = g_scratch_addr[dev];
    return OBS_OK;
}

extern "C" int obs_decode_ffn_static(const obs_layer_weights* w, int n_experts, int hidden, int inter, int top_k,
                                     const uint16_t* x, const int32_t* ids, const float* weights,
                                     const uint16_t* residual, int T, uint16_t* out, void* stream) {
    if (!w || !w->gate_w || !w->gate_s || !w->gate_b || !w->up_w || !w->up_s || !w->up_b || !w->down_w ||
        !w->down_s || !w->down_b)
        return fail(OBS_ERR_INVALID, "obs_decode_ffn_static: null expert weight pointer");
    if (T < 0 || top_k <= 0 || top_k > 16 || n_experts <= 0)
        return fail(OBS_ERR_INVALID, "obs_decode_ffn_static: bad T, top_k or n_experts");
    if ((long)T * top_k > OBS_STATIC_MAX_PAIRS)
        return fail(OBS_ERR_INVALID, "obs_decode_ffn_static: T * top_k above OBS_STATIC_MAX_PAIRS (64)");
    if (hidden <= 0 || hidden > OBS_STATIC_MAX_HIDDEN || hidden % 512)
        return fail(OBS_ERR_INVALID, "obs_decode_ffn_static: hidden must be a multiple of 512, at most 4096");
    if (inter <= 0 || inter > OBS_STATIC_MAX_INTER || inter % 128)
        return fail(OBS_ERR_INVALID, "obs_decode_ffn_static: inter must be a multiple of 128, at most 1536");
    if (T == 0) return OBS_OK;
    if (!x || !ids || !weights || !out) return fail(OBS_ERR_INVALID, "obs_decode_ffn_static: null pointer");
    uint8_t* base = nullptr;
    int rc = scratch_for_current_device(&base);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    // counters start at zero (the kernels reset them after use; cleared again in
    // case an earlier call on this device did not finish)
    cudaError_t e = cudaMemsetAsync(base, 0, kZeroBytes, st);
    if (e != cudaSuccess) return fail(OBS_ERR_CUDA, cudaGetErrorString(e));
    obs::DecodeBufs d{};
    d.cnt_gu = reinterpret_cast<uint32_t*>(base + kOffCntGu);
    d.cnt_dn = reinterpret_cast<uint32_t*>(base + kOffCntDn);
    d.err = reinterpret_cast<int*>(base + kOffErr);
    d.part = reinterpret_cast<float*>(base + kOffPart);
    d.hq = base + kOffH;
    d.hmeta = reinterpret_cast<float2*>(base + kOffHMeta);
    d.xq = base + kOffX;
    d.xmeta = reinterpret_cast<float2*>(base + kOffXMeta);
    d.y = reinterpret_cast<uint16_t*>(base + kOffY);
    const obs::Shape sh{hidden, inter, n_experts, top_k};
    e = obs::launch_decode_ffn_mlx(w->gate_w, w->gate_s, w->gate_b, w->up_w, w->up_s, w->up_b, w->down_w, w->down_s,
                                   w->down_b, sh, x, ids, weights, residual, T, d, out, st);
    if (e != cudaSuccess) return fail(OBS_ERR_CUDA, cudaGetErrorString(e));
    return OBS_OK;
}
