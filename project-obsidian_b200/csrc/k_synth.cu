// k_synth.cu -- seeded synthetic weights/activations on the device, and the
// loader's re-tiling of reference-format weights into the kernels' blocks.
//
// The generator is the device twin of oracle/obs_oracle.c (orc_synth_*): the
// same counter-based splitmix64 streams, 24-bit uniforms, Irwin-Hall(12)
// normals and explicitly fused arithmetic, so both produce identical bytes.
#include "obs_internal.cuh"

namespace obs {
namespace {

constexpr uint64_t kGamma = 0x9E3779B97F4A7C15ull;
enum { T_ROUTER_W = 0, T_ROUTER_S = 1, T_GATE_W = 2, T_X = 11 };

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__host__ __device__ inline uint64_t mix64_h(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
// key derivation runs on the host (same function as orc_stream_key)
inline uint64_t stream_key(uint64_t seed, uint32_t layer, uint32_t tensor) {
    uint64_t h = mix64_h(seed + kGamma);
    h = mix64_h(h ^ ((uint64_t)layer + 1u) * kGamma);
    h = mix64_h(h ^ ((uint64_t)tensor + 1u) * 0xD1B54A32D192ED03ull);
    return h;
}
__device__ __forceinline__ uint64_t stream_u64(uint64_t key, uint64_t idx) { return mix64(key + (idx + 1u) * kGamma); }
__device__ __forceinline__ float u24(uint64_t r) {
    return __fmul_rn(__uint2float_rn((uint32_t)(r >> 40)), 1.0f / 16777216.0f);
}
__device__ __forceinline__ float normal_ih(uint64_t key, uint64_t idx) {
    long long acc = 0;
#pragma unroll
    for (int m = 0; m < 6; ++m) {
        uint64_t r = stream_u64(key, idx * 6u + (uint64_t)m);
        acc += (long long)(r >> 40) + (long long)((r >> 16) & 0xFFFFFFu);
    }
    acc -= 6ll * 16777216ll;
    return __fmul_rn(__int2float_rn((int)acc), 1.0f / 16777216.0f);
}

__global__ void k_synth_router(uint64_t kw, uint64_t ks, size_t nw, size_t ng, uint32_t* w, uint16_t* s,
                               uint16_t* b) {
    const float lo = 0.0005f, span = 0.005f - 0.0005f;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nw; i += (size_t)gridDim.x * blockDim.x)
        w[i] = (uint32_t)stream_u64(kw, i);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < ng; i += (size_t)gridDim.x * blockDim.x) {
        uint16_t sc = f2bf(__fmaf_rn(u24(stream_u64(ks, i)), span, lo));
        s[i] = sc;
        b[i] = f2bf(__fmul_rn(-128.0f, bf2f(sc)));
    }
}

// elements [w0, w0 + nw) / [g0, g0 + ng) of the projection's streams (a slice
// of experts starts at its first expert's element index)
__global__ void k_synth_proj(uint64_t kw, uint64_t ks, uint64_t kb, size_t w0, size_t nw, size_t g0, size_t ng,
                             uint32_t* w, uint16_t* s, uint16_t* b) {
    const float lo = 0.002f, span = 0.02f - 0.002f;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nw; i += (size_t)gridDim.x * blockDim.x)
        w[i] = (uint32_t)stream_u64(kw, w0 + i);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < ng; i += (size_t)gridDim.x * blockDim.x) {
        uint16_t sc = f2bf(__fmaf_rn(u24(stream_u64(ks, g0 + i)), span, lo));
        float n = normal_ih(kb, g0 + i);
        s[i] = sc;
        b[i] = f2bf(__fmaf_rn(n, 1e-3f, __fmul_rn(-8.0f, bf2f(sc))));
    }
}

// one thread per row: raw bf16 normals, then the sequential RMSNorm of
// rmsnorm.metal:20-35 with weight 1 (same operation order as orc_rmsnorm_row)
__global__ void k_synth_x(uint64_t kx, int row0, int T, int H, float eps, uint16_t* x) {
    int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    uint16_t* row = x + (size_t)t * H;
    size_t base = (size_t)(row0 + t) * H;
    float ss = 0.0f;
    for (int i = 0; i < H; ++i) {
        uint16_t v = f2bf(normal_ih(kx, base + i));
        row[i] = v;
        float f = bf2f(v);
        ss = __fmaf_rn(f, f, ss);
    }
    float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), eps));
    for (int i = 0; i < H; ++i) row[i] = f2bf(__fdiv_rn(bf2f(row[i]), rms));
}

// MLX word (column c at nibble c) -> block word (column nib_col(p) at nibble p)
__device__ __forceinline__ uint32_t nib_order(uint32_t w) {
    uint32_t o = 0;
#pragma unroll
    for (int p = 0; p < 8; ++p) o |= ((w >> (4 * nib_col(p))) & 0xFu) << (4 * p);
    return o;
}
__device__ __forceinline__ uint4 nib_order(uint4 v) {
    return make_uint4(nib_order(v.x), nib_order(v.y), nib_order(v.z), nib_order(v.w));
}

// Thread per (block, source row): 8 packed words + scale + bias.  Group size 64
// equals the block width, so block kt uses scale/bias column kt.  Rows' first
// and second 16-byte halves go to separate 2 KB planes of the block, so 16-byte
// reads by consecutive rows are contiguous.  Unpaired: 128-row tiles, block row
// = tile row.  Paired (the gate/up array): 64-row tiles of each projection,
// tile feature c -> block row 32*(c/16) + 16*proj + c%16, so TMEM lane quarter
// q holds gate and up of the same 16 features.
__global__ void k_retile(const uint32_t* __restrict__ w, const uint16_t* __restrict__ s,
                         const uint16_t* __restrict__ b, int E, int out_f, int in_f, uint8_t* __restrict__ dst,
                         int paired, int proj) {
    const int tile_rows = paired ? kRowTile / 2 : kRowTile;
    const int n_rt = out_f / tile_rows, n_kt = in_f / kGroup;
    const size_t nblk = (size_t)E * n_rt * n_kt;
    const size_t total = nblk * tile_rows;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % tile_rows);
        const size_t blk = i / tile_rows;
        const int kt = (int)(blk % n_kt);
        const int rt = (int)((blk / n_kt) % n_rt);
        const int e = (int)(blk / ((size_t)n_kt * n_rt));
        const size_t row = (size_t)e * out_f + (size_t)rt * tile_rows + c;
        const int r = paired ? 32 * (c >> 4) + 16 * proj + (c & 15) : c;
        const uint4* src = reinterpret_cast<const uint4*>(w + row * (in_f / 8) + (size_t)kt * 8);
        uint8_t* d = dst + blk * (size_t)kBlockBytes;
        *reinterpret_cast<uint4*>(d + r * 16) = nib_order(src[0]);         // words 0-3
        *reinterpret_cast<uint4*>(d + 2048 + r * 16) = nib_order(src[1]);  // words 4-7
        uint16_t* ds = reinterpret_cast<uint16_t*>(d + kBlockWords * 4);
        ds[r] = s[row * (in_f / kGroup) + kt];
        ds[kRowTile + r] = b[row * (in_f / kGroup) + kt];
    }
}

inline int grid_for(size_t n, int threads) {
    size_t g = (n + threads - 1) / threads;
    return (int)(g < 1 ? 1 : (g > 65535 * 4 ? 65535 * 4 : g));
}

}  // namespace

cudaError_t launch_synth_router(uint64_t seed, uint32_t layer, int E, int H, uint32_t* w, uint16_t* s,
                                uint16_t* b, cudaStream_t st) {
    size_t nw = (size_t)E * (H / 4), ng = (size_t)E * (H / kGroup);
    note_launch();
    k_synth_router<<<grid_for(nw, 256), 256, 0, st>>>(stream_key(seed, layer, T_ROUTER_W),
                                                      stream_key(seed, layer, T_ROUTER_S), nw, ng, w, s, b);
    return cudaGetLastError();
}

cudaError_t launch_synth_proj(uint64_t seed, uint32_t layer, int proj, int e0, int E, int out_f, int in_f,
                              uint32_t* w, uint16_t* s, uint16_t* b, cudaStream_t st) {
    uint32_t tw = T_GATE_W + 3u * (uint32_t)proj;
    const size_t wpe = (size_t)out_f * (in_f / 8), gpe = (size_t)out_f * (in_f / kGroup);  // per expert
    note_launch();
    k_synth_proj<<<grid_for(E * wpe, 256), 256, 0, st>>>(stream_key(seed, layer, tw), stream_key(seed, layer, tw + 1),
                                                         stream_key(seed, layer, tw + 2), e0 * wpe, E * wpe, e0 * gpe,
                                                         E * gpe, w, s, b);
    return cudaGetLastError();
}

cudaError_t launch_synth_x(uint64_t seed, uint32_t layer, int row0, int T, int H, float eps, uint16_t* x,
                           cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    note_launch();
    k_synth_x<<<(T + 127) / 128, 128, 0, st>>>(stream_key(seed, layer, T_X), row0, T, H, eps, x);
    return cudaGetLastError();
}

cudaError_t launch_retile(const uint32_t* w, const uint16_t* s, const uint16_t* b, int E, int out_f, int in_f,
                          uint8_t* dst, int paired, int proj, cudaStream_t st) {
    const size_t total = (size_t)E * out_f * (in_f / kGroup);  // one thread per (source row, k-tile)
    note_launch();
    k_retile<<<grid_for(total, 256), 256, 0, st>>>(w, s, b, E, out_f, in_f, dst, paired, proj);
    return cudaGetLastError();
}

}  // namespace obs
