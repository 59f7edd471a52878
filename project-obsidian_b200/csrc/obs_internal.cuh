// obs_internal.cuh -- launchers shared between the translation units of
// libobsmoe.so.  Not part of the public ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "obs_common.cuh"

namespace obs {

// Counts every kernel launch the library issues (obs_kernel_launches).
void note_launch();

// Programmatic dependent launch on/off (environment OBS_PDL=0 turns it off for
// the process; read once).
bool pdl_enabled();

// Launch with programmatic stream serialization (the kernel calls pdl_begin()
// first): it may be scheduled while the previous kernel of the stream finishes.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    note_launch();
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// One 128-row x 64-column block of a tiled 4-bit projection (4608 bytes):
// words 0-3 of the 128 rows, words 4-7 of the 128 rows, 128 bf16 scales,
// 128 bf16 biases.  The gate/up array is "paired": each block holds 64 gate
// and the same 64 up features, so one MMA chain yields both halves of SwiGLU.
struct LayerDev {
    uint32_t* router_w;   // [E, H/4]   reference layout
    uint16_t* router_s;   // [E, H/64]
    uint16_t* router_b;
    uint8_t* gateup;      // [E][I/64][H/64] paired blocks: rows 32q+i = gate (i < 16) / up (i >= 16)
                          // of feature 64*rt + 16q + (i & 15)
    uint8_t* down;        // [E][H/128][I/64] blocks
    bool loaded;
};

struct Shape {
    int H, I, E, K;
};

// ---------------------------------------------------------------- k_synth.cu
cudaError_t launch_synth_router(uint64_t seed, uint32_t layer, int E, int H, uint32_t* w, uint16_t* s,
                                uint16_t* b, cudaStream_t st);
cudaError_t launch_synth_proj(uint64_t seed, uint32_t layer, int proj, int e0, int E, int out_f, int in_f,
                              uint32_t* w, uint16_t* s, uint16_t* b, cudaStream_t st);
cudaError_t launch_synth_x(uint64_t seed, uint32_t layer, int row0, int T, int H, float eps, uint16_t* x,
                           cudaStream_t st);
// Re-tile one projection [E][out_f][in_f] (reference layout) into 4608-byte
// blocks [E][tiles][in_f/64].  paired = 0: 128-row tiles, row r of the block =
// row r of the tile.  paired = 1 (gate proj 0 / up proj 1 into the gate/up
// array): 64-row tiles, feature c of the tile goes to block row
// 32*(c/16) + 16*proj + c%16.
cudaError_t launch_retile(const uint32_t* w, const uint16_t* s, const uint16_t* b, int E, int out_f, int in_f,
                          uint8_t* dst, int paired, int proj, cudaStream_t st);

// --------------------------------------------------------------- k_router.cu
// Router logits for T tokens: router_parts(T) partial planes [parts][T][E]
// (1: final logits; 8: node sums that launch_topk / launch_router_finish
// combine in the fixed tree).  `parts` must hold 8*T*E floats.
int router_parts(int T);
cudaError_t launch_router_logits(const LayerDev& L, const Shape& sh, const uint16_t* x, int T, float* parts,
                                 cudaStream_t st);
cudaError_t launch_router_finish(const float* parts, int T, int E, float* logits, cudaStream_t st);
// logits_out (optional) receives the combined logits.
cudaError_t launch_topk(const float* logits, int nparts, const float* bias, int T, int E, int K, int norm,
                        int32_t* ids, float* w, float* logits_out, cudaStream_t st);

// ------------------------------------------------------------- k_dispatch.cu
constexpr int kDispChunk = 512;  // tokens per dispatch chunk (one CTA of the histogram / placement)
struct DispatchBufs {
    int32_t* counts;    // [E] routes per expert (written by the dispatch)
    int32_t* hist;      // [max_chunks][E] routes per (token chunk, expert)
    int max_chunks;     // chunks of kDispChunk tokens the hist buffer holds
    int* err;           // the context's device error word (kDevBadRoute)
    int32_t* seg;       // [E+1] padded segment starts
    int32_t* slot_of;   // [T*K]
    int32_t* src;       // [R_cap] source token of each slot (-1 for pad rows)
    int4* tiles;        // [max_tiles] {expert, row0, nrows, 0}
    int32_t* n_tiles;   // [1]
    uint16_t* xp;       // tiled activations [R_cap x H]
    int atoms;          // R_cap / 8
    int rows_cap;       // R_cap: rows of src / xp
    int max_tiles;      // entries of tiles
    int bn;             // token rows per GEMM tile
};
// row_src (optional): the row of token t is row_src[t] instead of x + t*H.
// allow_none: an id of -1 means "no expert" (received rows without a local expert).
cudaError_t launch_dispatch(const int32_t* ids, const uint16_t* x, int T, const Shape& sh, const DispatchBufs& d,
                            int permute, cudaStream_t st, const uint16_t* const* row_src = nullptr,
                            int allow_none = 0);
// y_local / local (expert parallelism): items computed on this rank, read from y_local (see k_combine)
cudaError_t launch_combine(const uint16_t* y, int y_ld, const int32_t* slot_of, const float* w,
                           const uint16_t* residual, int T, int H, int K, uint16_t* out, cudaStream_t st,
                           const uint16_t* y_local = nullptr, int32_t* local = nullptr);
cudaError_t launch_gather_rows(const uint16_t* y, const int32_t* slot_of, int rows, int H, uint16_t* out,
                               cudaStream_t st);
cudaError_t launch_rmsnorm(const uint16_t* x, const uint16_t* w, int T, int H, float eps, uint16_t* out,
                           cudaStream_t st);
cudaError_t launch_tile_rows(const uint16_t* x, int n, int cols, int atoms, uint16_t* dst, cudaStream_t st);

// ------------------------------------------------------------------- k_ep.cu
constexpr int kMaxWorld = 8;
struct EpArgs {
    uint8_t* peer[kMaxWorld];  // every rank's EP buffer (this rank's included), same layout
    int world, rank, H, K, E_local;
    const int32_t* place; // [E] slot of each global expert (slot = rank * E_local + local expert), this layer
    int cap_rows;        // rows of one source region: a token goes to a rank at most once (max_tokens)
    int cap_items;       // (token, rank) items of one source (max_tokens * K)
    size_t off_rx, off_meta, off_mtok, off_cnt, off_rflag, off_ret, off_retflag;
    int32_t* send_cnt;   // [world] rows sent to each rank (reset by the sender's last CTA)
    uint32_t* done;      // [2] CTA completion counters of k_ep_send / k_ep_return
    uint32_t* epoch;     // [1] completed forwards
    int32_t* ids_local;  // [world * cap_rows * K] local expert of each received (row, k), -1 = none
    int32_t* src_item;   // [world * cap_rows * K] source item t*K+k of each received (row, k)
    int32_t* local_slot; // [cap_items] 1 + this rank's output slot of each of its own items computed here,
                         // 0 otherwise (set by k_ep_rowptr, cleared by the combine)
    const uint16_t** row_src;  // [world * cap_rows] where each received row's data is (k_ep_recv)
    int rows_cap;        // rows of the expert-output buffer k_ep_return reads (slot_of bound)
    int* err;
    uint64_t wait_ns;    // limit of the bounded waits for peers
};
cudaError_t launch_ep_send(const int32_t* ids, const uint16_t* x, int T, int E, const EpArgs& a, cudaStream_t st);
cudaError_t launch_ep_recv(const uint16_t* x, const EpArgs& a, cudaStream_t st);
// The destination of every output slot of the down GEMM: the source rank's return
// buffer (over NVLink) for rows received from another rank, this rank's y for its
// own rows (noted in local_slot) and for padding rows.
cudaError_t launch_ep_rowptr(const int32_t* slot_of, const int32_t* src, const int32_t* seg_end, uint16_t* y,
                             uint16_t** row_ptr, const EpArgs& a, cudaStream_t st);
// After a down GEMM that wrote its rows through row_ptr: stamps every source.
cudaError_t launch_ep_returned(const EpArgs& a, cudaStream_t st);
cudaError_t launch_ep_finish(const EpArgs& a, cudaStream_t st);
// One bounded wait on a stamp that nothing writes (obs_probe_wait): gives up
// after limit_ns and records kDevTimeout in *err.
cudaError_t launch_probe_wait(const uint32_t* stamp, uint64_t limit_ns, int* err, cudaStream_t st);

// --------------------------------------------------------------- k_decode.cu
constexpr int kDecodeSplit = 8;  // k-splits of the decode gate/up mat-vec
struct DecodeBufs {
    float* part;        // [T*K][n_rt_gu][kDecodeSplit][2][128] gate/up partials
    uint32_t* cnt_gu;   // [T*K][n_rt_gu]
    uint8_t* hq;        // [T*K][I/64][128 B] SwiGLU rows h in fixed point (k_decode.cu)
    float2* hmeta;      // [T*K][I/64] (sum X 2^-k, 2^-(k+4)) per h group
    uint8_t* xq;        // [T][H/64][128 B] the layer input in fixed point
    float2* xmeta;      // [T][H/64]
    uint16_t* y;        // [T*K][H] bf16
    uint32_t* cnt_dn;   // [T][n_rt_dn]
    int* err;           // device error flag (expert id out of range)
};
// The fused decode layer (router -> top-k -> gate/up -> SwiGLU -> down ->
// combine in one cooperative launch) for T <= kFusedMaxT tokens.
constexpr int kFusedMaxT = 8;
// OBS_PATH_AUTO's default decode threshold: measured on B200 at the model's
// shape, the fused layer beats the grouped GEMM to T = 4 (37 vs 59 us per
// layer) and loses at T = 8 (68 vs 63 us: it reads each (token, expert) pair's
// weights, the GEMM each routed expert's once)
constexpr int kDecodeAutoT = 4;
struct FusedDecodeBufs {
    uint64_t* lst;      // [4][kFusedMaxT][E] logit bits | launch stamp << 32: router logits, four replicas
    int32_t* ids;       // [T][K]
    float* wts;         // [T][K]
    uint32_t* bar;      // [0] launch tickets (only grows; generation = ticket / grid size)
    uint64_t* ypart;    // [T*K][I/64][H] down partials per h group: value bits | launch stamp << 32
    int* err;
    uint64_t* trace;    // optional diagnostics: 24 %globaltimer marks per CTA (obs_trace_enable)
    uint64_t wait_ns;   // limit of every device-side wait
};
// Dynamic shared-memory plan of the fused layer (byte offsets): the input
// rows (then their fixed-point packs), one packed h group, and an 8-unit ring
// of gate/up weight blocks (slots 0-3 also take a down column group).
struct FusedPlan {
    int off_x, off_h, off_ring;
    int unit_bytes, dn_bytes, region_bytes, nslot, smem_bytes;
};
FusedPlan fused_plan(int T, int H, int I);
// Whether the fused layer handles this shape and T (H = 2048, I a multiple of
// 256 up to 1024, T <= kFusedMaxT, and its shared-memory plan fits the device).
bool decode_fused_supported(const Shape& sh, int T);
// normalize = 1: x is the residual stream and the kernel applies the MoE input
// RMSNorm (eps) itself, bit-identical to launch_rmsnorm.
cudaError_t launch_decode_fused(const LayerDev& L, const Shape& sh, const uint16_t* x, const uint16_t* residual,
                                const float* bias, int T, int norm, int normalize, float eps,
                                const FusedDecodeBufs& f, uint16_t* out, int num_sms, cudaStream_t st);
cudaError_t launch_decode_gateup(const LayerDev& L, const Shape& sh, const uint16_t* x, const int32_t* ids,
                                 int T, const DecodeBufs& d, cudaStream_t st);
cudaError_t launch_decode_down(const LayerDev& L, const Shape& sh, const int32_t* ids, const float* w,
                               const uint16_t* residual, int T, const DecodeBufs& d, uint16_t* out,
                               int do_combine, cudaStream_t st);

// ----------------------------------------------------------------- k_head.cu
constexpr int kHeadMaxT = 16;  // tokens of one obs_lm_head call
// longest KV cache (the model's max_position_embeddings): the attention kernel
// keeps one fp32 score per cached position in shared memory (160 KB)
constexpr int kAttnMaxSeq = 40960;
cudaError_t launch_embed(const uint32_t* w, const uint16_t* s, const uint16_t* b, const int32_t* tokens, int T,
                         int vocab, int H, uint16_t* x, int* err, cudaStream_t st);
// logits [T, vocab] fp32 of the normalised rows xn, then ids [T] = the first maximum of each row
cudaError_t launch_lm_head(const uint32_t* w, const uint16_t* s, const uint16_t* b, const uint16_t* xn, int T,
                           int vocab, int H, float* logits, int32_t* ids, int num_sms, cudaStream_t st);

// y [T, rows] fp32 = x [T, in_f] (bf16) . dequant(W [rows, in_f/8])^T in the canonical order (k_lm_head)
cudaError_t launch_linear4(const uint32_t* w, const uint16_t* s, const uint16_t* b, const uint16_t* x, int T,
                           int rows, int in_f, float* y, int num_sms, cudaStream_t st);

// ----------------------------------------------------------------- k_attn.cu
cudaError_t launch_qk_norm_rope(const float* qkv, int T, int nq, int nkv, int hd, const uint16_t* qn,
                                const uint16_t* kn, float eps, const float* rope_cs, int max_seq, const int32_t* seq,
                                const int32_t* pos, uint16_t* qout, uint16_t* kcache, uint16_t* vcache, int n_seqs,
                                int* err, cudaStream_t st);
// part: sdpa_part_floats(max_tokens, ...) floats of scratch (the splits' partial sums)
cudaError_t launch_sdpa(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, int T, int nq, int nkv, int hd,
                        int max_seq, int n_seqs, const int32_t* seq, const int32_t* pos, uint16_t* out, float* part,
                        int num_sms, cudaStream_t st);
int sdpa_splits(int T, int nkv, int num_sms);
size_t sdpa_part_floats(int max_tokens, int nq, int nkv, int hd, int num_sms);
cudaError_t launch_residual_add(const uint16_t* x, const float* o, size_t n, uint16_t* out, cudaStream_t st);
// cos/sin of pos * theta^(-2i/hd) for pos < max_seq, i < hd/2, interleaved, computed in double, as fp32
void rope_table(double theta, int hd, int max_seq, float* out);

// ----------------------------------------------------------------- k_gemm.cu
enum GemmEpi : int { kEpiSwiglu = 0, kEpiBf16 = 1, kEpiF32 = 2 };
struct GemmArgs {
    const uint8_t* wblocks;   // tiled weight blocks [E][n_rt][n_kt] of 4608 bytes
    int paired;               // 1: the gate/up array (each 128-row block = 64 gate + 64 up rows)
    int proj_sel;             // kEpiF32 on the paired array: 0 stores the gate rows, 1 the up rows
    const uint16_t* act;      // tiled activations (B operand): 8-row atoms of 1024 B per k-group
    int atoms;                // row atoms of the activation layout
    const int4* tiles;        // token tiles {expert, row0, nrows, 0}
    const int32_t* n_tiles;   // device count of token tiles
    int max_tiles;            // entries of the tiles buffer (a larger count is refused)
    int n_rt;                 // weight row tiles per expert (I/64 for the paired array, H/128 for down)
    int n_kt;                 // k-tiles (in / 64), a multiple of 4
    int bn;                   // max token rows per tile (<= 128)
    int n_experts;            // experts in wblocks (tile expert ids are checked against it)
    void* out;                // kEpiSwiglu: tiled bf16 H; kEpiBf16: bf16 [rows, out_ld]; kEpiF32: fp32
    int out_ld;               // row stride of row-major outputs (elements)
    int out_atoms;            // row atoms of the tiled output
    int row_limit;            // rows >= row_limit are not stored
    int* err;                 // device error flag
    uint64_t* trace;          // optional: CTA 0 records %globaltimer per role and k-step
    int trace_n;              // k-steps recorded per role
    uint64_t wait_ns;         // limit of every mbarrier wait
    uint16_t* const* row_ptr; // kEpiBf16, optional: destination of each output row (slot), row-major H wide
};
// trace roles (rows of the trace buffer, trace_n entries each)
enum TraceRole : int {
    kTrWIssue = 0,     // weight producer issued the copy of W stage i (four k-groups)
    kTrBSignal = 1,    // token-tile producer of the first k-group issued its copy for k-step i
    kTrDqStart = 2,    // dequant warp 0 passed its waits for k-step i
    kTrDqDone = 3,     // dequant warp 0 arrived "pair ready" for k-step i
    kTrMmaStart = 4,   // MMA thread passed its wait for pair i (k-steps 2i, 2i+1)
    kTrMmaIssued = 5,  // MMA thread committed pair i
    kTrEpStart = 6,    // epilogue passed accfull of item i
    kTrEpDone = 7,     // epilogue released the accumulator of item i
    kTrDqStored = 8,   // dequant warp 0 finished its TMEM stores of k-step i
    kTrMmaFenced = 9,  // MMA thread passed its fence for pair i
    kTrDqDoneQ1 = 10,  // as kTrDqDone, for the dequant warps of TMEM lane quarters 1, 2, 3
    kTrDqAFree = 13,   // dequant warp 0 passed the wait for its A stage of k-step i
    kTrRoles = 14
};
cudaError_t launch_gemm(const GemmArgs& a, int epi, int num_sms, cudaStream_t st);
size_t gemm_smem_bytes(int epi);
int gemm_tile_rows();  // token rows per GEMM tile (the dispatch's tile size)

}  // namespace obs
