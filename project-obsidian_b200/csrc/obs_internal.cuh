// obs_internal.cuh -- launchers shared between the translation units of
// libobsmoe.so.  Not part of the public ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "obs_common.cuh"

namespace obs {

// One 128-row x 64-column block of a tiled 4-bit projection: 128 rows of
// 8 uint32 words, then 128 bf16 scales, then 128 bf16 biases (4608 bytes).
// gate and up are interleaved per block (gate, up) so one copy brings both.
struct LayerDev {
    uint32_t* router_w;   // [E, H/4]   reference layout
    uint16_t* router_s;   // [E, H/64]
    uint16_t* router_b;
    uint8_t* gateup;      // [E][I/128][H/64][2] blocks
    uint8_t* down;        // [E][H/128][I/64] blocks
    bool loaded;
};

struct Shape {
    int H, I, E, K;
};

// ---------------------------------------------------------------- k_synth.cu
cudaError_t launch_synth_router(uint64_t seed, uint32_t layer, int E, int H, uint32_t* w, uint16_t* s,
                                uint16_t* b, cudaStream_t st);
cudaError_t launch_synth_proj(uint64_t seed, uint32_t layer, int proj, int E, int out_f, int in_f,
                              uint32_t* w, uint16_t* s, uint16_t* b, cudaStream_t st);
cudaError_t launch_synth_x(uint64_t seed, uint32_t layer, int row0, int T, int H, float eps, uint16_t* x,
                           cudaStream_t st);
// reference layout -> tiled blocks.  interleave = 2 writes block p of each pair.
cudaError_t launch_retile(const uint32_t* w, const uint16_t* s, const uint16_t* b, int E, int out_f, int in_f,
                          uint8_t* dst, int interleave, int p, cudaStream_t st);

// --------------------------------------------------------------- k_router.cu
cudaError_t launch_router_logits(const LayerDev& L, const Shape& sh, const uint16_t* x, int T, float* logits,
                                 cudaStream_t st);
cudaError_t launch_topk(const float* logits, const float* bias, int T, int E, int K, int norm, int32_t* ids,
                        float* w, int32_t* counts, int* err, cudaStream_t st);

// ------------------------------------------------------------- k_dispatch.cu
struct DispatchBufs {
    int32_t* counts;    // [E]
    int32_t* seg;       // [E+1] padded segment starts
    int32_t* slot_of;   // [T*K]
    int32_t* src;       // [R_cap] source token of each slot (-1 for pad rows)
    int4* tiles;        // [max_tiles] {expert, row0, nrows, 0}
    int32_t* n_tiles;   // [1]
    uint16_t* xp;       // tiled activations [R_cap x H]
    int atoms;          // R_cap / 8
    int bn;             // token rows per GEMM tile
};
cudaError_t launch_dispatch(const int32_t* ids, const uint16_t* x, int T, const Shape& sh, const DispatchBufs& d,
                            int permute, cudaStream_t st);
cudaError_t launch_combine(const uint16_t* y, int y_ld, const int32_t* slot_of, const float* w,
                           const uint16_t* residual, int T, int H, int K, uint16_t* out, cudaStream_t st);
cudaError_t launch_gather_rows(const uint16_t* y, const int32_t* slot_of, int rows, int H, uint16_t* out,
                               cudaStream_t st);
cudaError_t launch_histogram(const int32_t* ids, int n, int E, int32_t* counts, int* err, cudaStream_t st);
cudaError_t launch_tile_rows(const uint16_t* x, int n, int cols, int atoms, uint16_t* dst, cudaStream_t st);

// --------------------------------------------------------------- k_decode.cu
struct DecodeBufs {
    float* part;        // [T*K][n_rt_gu][KSPLIT][2][128] gate/up partials
    uint32_t* cnt_gu;   // [T*K][n_rt_gu]
    uint16_t* h;        // [T*K][I] bf16
    uint16_t* y;        // [T*K][H] bf16
    uint32_t* cnt_dn;   // [T][n_rt_dn]
    int* err;           // device error flag (expert id out of range)
};
cudaError_t launch_decode_gateup(const LayerDev& L, const Shape& sh, const uint16_t* x, const int32_t* ids,
                                 int T, const DecodeBufs& d, cudaStream_t st);
cudaError_t launch_decode_down(const LayerDev& L, const Shape& sh, const int32_t* ids, const float* w,
                               const uint16_t* residual, int T, const DecodeBufs& d, uint16_t* out,
                               int do_combine, cudaStream_t st);

// ----------------------------------------------------------------- k_gemm.cu
enum GemmEpi : int { kEpiSwiglu = 0, kEpiBf16 = 1, kEpiF32 = 2 };
struct GemmArgs {
    const uint8_t* wblocks;   // tiled weight blocks of the projection(s)
    int wstride;              // blocks per k-tile step (2 for the gate/up array, 1 for down)
    int woff;                 // block offset inside a step (0 gate, 1 up)
    const uint16_t* act;      // tiled activations (B operand)
    int atoms;                // row atoms of the activation layout
    const int4* tiles;        // token tiles {expert, row0, nrows, 0}
    const int32_t* n_tiles;   // device count of token tiles
    int n_rt;                 // weight row tiles per expert
    int n_kt;                 // k-tiles (in / 64)
    int bn;                   // max token rows per tile (<= 128)
    void* out;                // kEpiSwiglu: tiled bf16 H; kEpiBf16: bf16 [rows, out_ld]; kEpiF32: fp32
    int out_ld;               // row stride of row-major outputs (elements)
    int out_atoms;            // row atoms of the tiled output
    int row_limit;            // rows >= row_limit are not stored
    int* err;                 // device error flag
};
cudaError_t launch_gemm(const GemmArgs& a, int epi, int num_sms, cudaStream_t st);
size_t gemm_smem_bytes(int epi);

}  // namespace obs
