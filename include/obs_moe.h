/*
 * obs_moe.h -- C ABI of the B200 (sm_100a) MoE hot path for project-obsidian.
 *
 * The library replaces the MoE section of the reference's per-layer forward
 * (src/forward.rs:421-441 decode, :164-247 batched prefill) and the Metal
 * helpers it encodes through ObsidianExecutor (src/executor.rs:60-70).  Every
 * entry point is plain C: pointers, sizes, an opaque context, a CUDA stream
 * passed as void*.  All return an int status (OBS_OK = 0); obs_last_error()
 * gives the message, the way the reference's helpers return Result<_, String>.
 *
 * Data formats are the reference's (MLX affine quantisation, row-major):
 *   router   W uint32 [E, H/4]   8-bit codes, byte i of a row = column i
 *            s, b bf16 [E, H/64]                       (dequant_matvec_8bit.metal:8-31)
 *   experts  W uint32 [E, out, in/8]  4-bit codes, nibble j of a word = (w>>4j)&15
 *            s, b bf16 [E, out, in/64]                 (fused_dequant_matvec_4bit.metal:14-53,
 *                                                       tools/split_experts.py:63-75)
 *   gate/up: out = I, in = H;  down: out = H, in = I.
 *   activations bf16 [T, H] (the reference uses f16; bf16 here, fp32 accumulate).
 *
 * Threading: one context per GPU, driven from one host thread at a time; the
 * context owns its scratch, so calls on one context must not overlap on the
 * GPU.  Device pointers unless a name ends in _host.
 */
#ifndef OBS_MOE_H
#define OBS_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OBS_ABI_VERSION 1

enum obs_status {
    OBS_OK = 0,
    OBS_ERR_INVALID = 1,   /* bad argument or shape */
    OBS_ERR_CUDA = 2,      /* a CUDA runtime call failed */
    OBS_ERR_NOMEM = 3,     /* device or host allocation failed */
    OBS_ERR_STATE = 4,     /* e.g. layer not loaded, EP not initialised */
    OBS_ERR_TIMEOUT = 5,   /* a bounded device-side wait gave up */
    OBS_ERR_NCCL = 6,      /* an NCCL call failed or a peer went away */
    OBS_ERR_UNSUPPORTED = 7
};

/* Execution path of obs_moe_forward. */
enum obs_path {
    OBS_PATH_AUTO = 0,     /* decode mat-vec for T <= decode_max_tokens, else prefill */
    OBS_PATH_DECODE = 1,   /* per-token fused 4-bit mat-vec (fused_dequant_matvec_4bit) */
    OBS_PATH_PREFILL = 2   /* dispatch + tcgen05 grouped GEMM (matmul_dequant_4bit) */
};

typedef struct obs_ctx obs_ctx;

/* Model shape; mirrors the fields of Qwen3MoeConfig the MoE path reads
 * (src/model.rs:7-23). */
typedef struct obs_config {
    int32_t hidden;            /* H: multiple of 2048 */
    int32_t inter;             /* I: moe_intermediate_size, multiple of 256 */
    int32_t n_experts;         /* E: <= 256 */
    int32_t top_k;             /* K: <= 16 */
    int32_t group_size;        /* must be 64 */
    int32_t n_layers;          /* layers whose weights the context holds */
    int32_t max_tokens;        /* largest T of one call (sizes the scratch) */
    int32_t norm_topk;         /* renormalise the top-k weights (norm_topk_prob) */
    int32_t decode_max_tokens; /* OBS_PATH_AUTO threshold; <= 0 picks 4 */
    float rms_eps;             /* RMSNorm epsilon of the fused input norm */
    int32_t ep_world;          /* expert parallelism: ranks sharing the experts (<= 1: off, max 8) */
    int32_t ep_rank;           /* this context's rank: it holds experts [rank*E/world, (rank+1)*E/world) */
} obs_config;

/* One layer's weights in the reference format (host or device memory). */
typedef struct obs_layer_weights {
    const uint32_t* router_w; const uint16_t* router_s; const uint16_t* router_b;
    const uint32_t* gate_w;   const uint16_t* gate_s;   const uint16_t* gate_b;
    const uint32_t* up_w;     const uint16_t* up_s;     const uint16_t* up_b;
    const uint32_t* down_w;   const uint16_t* down_s;   const uint16_t* down_b;
} obs_layer_weights;

/* The model's ends (the embedding, the final norm and the lm_head), MLX 4-bit
 * group-64 like the layers: embed/lm W uint32 [vocab, H/8], s/b bf16
 * [vocab, H/64]; norm_w bf16 [H] (model.norm.weight).  Host or device memory. */
typedef struct obs_head_weights {
    const uint32_t* embed_w; const uint16_t* embed_s; const uint16_t* embed_b;
    const uint32_t* lm_w;    const uint16_t* lm_s;    const uint16_t* lm_b;
    const uint16_t* norm_w;
} obs_head_weights;

/* The attention block of a layer (Qwen3-MoE): q/k/v/o MLX 4-bit group-64,
 * q [n_heads*head_dim, H/8], k and v [n_kv_heads*head_dim, H/8],
 * o [H, n_heads*head_dim/8], scales/biases bf16 [rows, in/64]; in_norm bf16 [H]
 * (input_layernorm), q_norm / k_norm bf16 [head_dim].  Host or device memory. */
typedef struct obs_attn_weights {
    const uint32_t* q_w; const uint16_t* q_s; const uint16_t* q_b;
    const uint32_t* k_w; const uint16_t* k_s; const uint16_t* k_b;
    const uint32_t* v_w; const uint16_t* v_s; const uint16_t* v_b;
    const uint32_t* o_w; const uint16_t* o_s; const uint16_t* o_b;
    const uint16_t* in_norm; const uint16_t* q_norm; const uint16_t* k_norm;
} obs_attn_weights;

/* Shape of the attention block and its KV caches (Qwen3MoeConfig, src/model.rs:7-35;
 * KvCache, src/kv_cache.rs:15-24): n_seqs independent sequences, each with a
 * bf16 cache [n_kv_heads][max_seq][head_dim] per layer for K and for V. */
typedef struct obs_attn_config {
    int32_t n_heads;     /* query heads (32) */
    int32_t n_kv_heads;  /* key/value heads (4); n_heads a multiple of it, at most 8 times it */
    int32_t head_dim;    /* <= 128, a multiple of 8; n_heads * head_dim a multiple of 2048 */
    int32_t max_seq;     /* positions per cache (<= 40960) */
    int32_t n_seqs;      /* sequences (caches) per layer */
    float rope_theta;    /* 1e7 */
} obs_attn_config;

/* ---------------------------------------------------------------- context */
int obs_abi_version(void);
/* Replaces ObsidianExecutor::new (src/executor.rs:39-58) and the expert pools
 * of Model::new (src/forward.rs:79-89): selects `device`, allocates the
 * HBM-resident expert store for n_layers layers and all scratch up front. */
int obs_create(const obs_config* cfg, int device, obs_ctx** out);
int obs_destroy(obs_ctx* ctx);
const char* obs_last_error(const obs_ctx* ctx);
/* Bytes of device memory the context holds (weights + scratch). */
int obs_memory_bytes(const obs_ctx* ctx, size_t* weights, size_t* scratch);

/* Replaces ExpertIndex::open + read_experts_parallel (src/disk_io.rs:24-102)
 * and the router part of Weights::load_non_expert (src/weight_loader.rs:19-71):
 * copies one layer into the context's HBM store, re-tiled for the kernels.
 * src_on_device != 0 if the pointers are device memory.  Synchronous. */
int obs_load_layer(obs_ctx* ctx, int layer, const obs_layer_weights* w, int src_on_device);

/* Replaces ExpertIndex::open + read_experts_parallel (src/disk_io.rs:24-102)
 * for one layer file of the reference's expert splitter
 * (tools/split_experts.py:63-75): layer_{il}_experts.safetensors with tensors
 * e{N}.{gate_proj,up_proj,down_proj}.{weight (U32 [out, in/8]), scales, biases
 * (F16 or BF16 [out, in/64])}.  The whole file is read once, stacked and loaded
 * like obs_load_layer (F16 scales/biases are rounded to bf16, exactly for every
 * value the splitter wrote from a bf16 checkpoint).  The router gate is not in
 * these files (src/weight_loader.rs:19-71 loads it from the model's shards):
 * router_w/_s/_b are its host arrays in obs_layer_weights' layout.  The file's
 * shapes must equal the context's.  Synchronous. */
int obs_load_layer_safetensors(obs_ctx* ctx, int layer, const char* path, const uint32_t* router_w,
                               const uint16_t* router_s, const uint16_t* router_b);
/* Reads only the header of such a file (no GPU needed) and reports its expert
 * count, hidden and intermediate sizes after checking that every expert has
 * all nine tensors with consistent dtypes and shapes; errors through
 * obs_last_error(NULL). */
int obs_expert_file_info(const char* path, int32_t* n_experts, int32_t* hidden, int32_t* inter);

/* Seeded synthetic layer generated on the device (bench/test support): the
 * same values oracle/obs_oracle.c produces on the host for (seed, layer). */
int obs_synth_layer(obs_ctx* ctx, int layer, uint64_t seed);
/* Seeded synthetic activations rows [row0, row0+T) of (seed, layer),
 * RMSNormed with eps, written to x [T, H] bf16 on `stream`. */
int obs_synth_activations(uint64_t seed, uint32_t layer, int row0, int T, int H, float eps,
                          uint16_t* x, void* stream);

/* ------------------------------------------------------- the model's ends */
/* Copies the embedding, the final norm weight and the lm_head into the
 * context's HBM (they replace the embed_tokens / model.norm / lm_head tensors
 * Weights::load_non_expert keeps, src/weight_loader.rs:19-71).  Synchronous. */
int obs_load_head(obs_ctx* ctx, int vocab, const obs_head_weights* w, int src_on_device);
/* Model::embed (src/forward.rs:445-462) on the device: x[t] = the dequantised
 * embedding row of tokens[t] (w = fma(q, s, b) in fp32, rounded to bf16).
 * tokens int32 [T], x bf16 [T, H], device memory. */
int obs_embed(obs_ctx* ctx, const int32_t* tokens, int T, uint16_t* x, void* stream);
/* The end of run_one_token (src/forward.rs:553-566): RMSNorm with model.norm's
 * weight, the 4-bit lm_head mat-vec over the vocabulary, and the greedy next
 * token -- the first maximum, as the reference's strict '>' scan -- for T <= 16
 * rows of the residual stream x (bf16 [T, H]).  ids int32 [T]; logits fp32
 * [T, vocab] or NULL.  The logits follow one canonical fp32 order (lane l of 32
 * chains fma(fma(q, s, b), x, acc) over its 64-column groups, then the adjacent
 * pairwise tree), so the ids are bit-exact with the CPU oracle's. */
int obs_lm_head(obs_ctx* ctx, const uint16_t* x, int T, int32_t* ids, float* logits, void* stream);

/* ------------------------------------------------------ the attention block */
/* Allocates the attention scratch and the RoPE table (cos/sin of
 * pos * theta^(-2i/head_dim), computed once in double precision) for the
 * context's n_layers layers; caches are allocated by obs_load_attn. */
int obs_attn_init(obs_ctx* ctx, const obs_attn_config* ac);
/* Copies one layer's attention weights into HBM (q, k and v concatenated into
 * one projection) and allocates its KV caches (zeroed).  Synchronous. */
int obs_load_attn(obs_ctx* ctx, int layer, const obs_attn_weights* w, int src_on_device);
/* The attention block of Model::forward_layer (src/forward.rs:404-419) for T
 * tokens: token t belongs to sequence seq[t] at position pos[t] (device int32
 * arrays).  xn = RMSNorm(x, in_norm); q, k, v = 4-bit projections (canonical
 * fp32 order, rounded to bf16); per-head RMSNorm of q and k (q_norm, k_norm);
 * NeoX RoPE (rope.metal:10-27) at pos[t]; K and V appended to the sequence's
 * cache at pos[t] (ops.metal:32-37); single-query GQA attention over the cache
 * positions 0 .. pos[t] (sdpa_decode.metal:14-48); out = x + o_proj(attention).
 * Tokens of one sequence in one call must have distinct positions, and a token
 * sees the K/V of every position <= its own (written by this call or earlier
 * ones): a prefill passes consecutive positions of one sequence (causal), a
 * batched decode step one token per sequence.  x, out bf16 [T, H], no aliasing. */
int obs_attn_forward(obs_ctx* ctx, int layer, const uint16_t* x, uint16_t* out, int T, const int32_t* seq,
                     const int32_t* pos, void* stream);
/* Copies cache positions [pos0, pos0 + n) of one sequence and layer: k and v
 * (either may be NULL) bf16 [n_kv_heads][n][head_dim], device memory. */
int obs_kv_read(obs_ctx* ctx, int layer, int seq, int pos0, int n, uint16_t* k, uint16_t* v, void* stream);

/* ------------------------------------------------------ the MoE layer path */
/* out = [residual +] sum_k w_k * expert_k(x): router -> top-k -> dispatch ->
 * 4-bit SwiGLU experts -> rank-order combine, all on `stream`, no host sync.
 * Replaces forward.rs:421-441 (decode) and :164-232 (batched prefill).
 * residual and logit_bias (fp32 [E], added to the router logits) may be NULL.
 * x and out are bf16 [T, H] device arrays; T <= max_tokens. */
int obs_moe_forward(obs_ctx* ctx, int layer, const uint16_t* x, uint16_t* out,
                    const uint16_t* residual, int T, const float* logit_bias, int path,
                    void* stream);
/* Same, from and to host memory: copies x (and residual) in, out back, and
 * waits for the stream.  Pinned host memory gives the full copy bandwidth. */
int obs_moe_forward_host(obs_ctx* ctx, int layer, const uint16_t* x_host, uint16_t* out_host,
                         const uint16_t* residual_host, int T, const float* logit_bias_host,
                         int path, void* stream);
/* The host entry without the wait, for callers that pipeline successive layers
 * or batches (the reference's forward.rs:421-441 / :164-232 call, issued ahead):
 * the input copy runs on an internal stream into one of two staging slots
 * (alternating per call), the forward on `stream`, the output copy on a second
 * internal stream, so call i+1's input and call i-1's output overlap call i's
 * forward.  x_host (and residual, bias) must stay unchanged, and out_host
 * unread, until obs_moe_host_join's stream has passed; pinned host memory is
 * needed for the copies to be asynchronous.  Successive calls use the same
 * `stream`.  Single-GPU contexts only. */
int obs_moe_forward_host_async(obs_ctx* ctx, int layer, const uint16_t* x_host, uint16_t* out_host,
                               const uint16_t* residual_host, int T, const float* logit_bias_host,
                               int path, void* stream);
/* Make `stream` wait (on the device) for every output copy issued by
 * obs_moe_forward_host_async so far; synchronise `stream` to read the results. */
int obs_moe_host_join(obs_ctx* ctx, void* stream);

/* ----------------------------------- stage entry points (tests, debugging) */
/* gate_gpu / dequant_matvec_8bit (forward.rs:386-397): router logits fp32
 * [T, E] in the canonical reduction order: 32 lanes, lane l chains
 * acc = fma(w, x, acc) over its 64-column groups in column order, then the
 * lane sums meet in the adjacent pairwise tree (offsets 1, 2, 4, 8, 16). */
int obs_gate(obs_ctx* ctx, int layer, const uint16_t* x, float* logits, int T, void* stream);
/* moe_routing_topk (moe_routing_topk.metal:15-57; router.rs:25-94): softmax,
 * top-k with the lowest index winning ties, renormalised weights. */
int obs_route(obs_ctx* ctx, const float* logits, const float* logit_bias, int T,
              int32_t* ids, float* weights, void* stream);
/* Token -> expert grouping (forward.rs:176-216) on the device: counts [E],
 * padded segment starts seg [E+1] (each segment a multiple of 16 rows), and
 * slot_of [T*K] (slots ordered by expert, then token). */
int obs_dispatch(obs_ctx* ctx, const int32_t* ids, int T, int32_t* counts, int32_t* seg,
                 int32_t* slot_of, void* stream);
/* Expert outputs y [T*K, H] bf16 in (token, rank) order for given routes,
 * through the decode mat-vec or the prefill grouped GEMM path. */
int obs_expert_ffn(obs_ctx* ctx, int layer, const uint16_t* x, const int32_t* ids, int T,
                   int path, uint16_t* y, void* stream);
/* One expert projection on the tcgen05 grouped GEMM with a plain fp32
 * epilogue: y [n, out] = x [n, in] . dequant(W)^T (matmul_dequant_4bit.metal:21-66).
 * proj 0 gate, 1 up, 2 down.  n <= max_tokens * top_k. */
int obs_expert_gemm_f32(obs_ctx* ctx, int layer, int proj, int expert, const uint16_t* x, int n,
                        float* y, void* stream);
/* Per-stage device timing of obs_moe_forward for benchmarks: when enabled,
 * every kernel launch of the layer is bracketed by CUDA events on the
 * caller's stream.  obs_profile_read fills ms_total[OBS_N_STAGES] and
 * launches[OBS_N_STAGES] with the sums since the last read, then resets. */
#define OBS_N_STAGES 12
enum obs_stage {
    OBS_STAGE_ROUTER = 0, OBS_STAGE_TOPK = 1, OBS_STAGE_DISPATCH = 2, OBS_STAGE_GEMM_GATEUP = 3,
    OBS_STAGE_GEMM_DOWN = 4, OBS_STAGE_COMBINE = 5, OBS_STAGE_DECODE_GATEUP = 6, OBS_STAGE_DECODE_DOWN = 7,
    OBS_STAGE_DECODE_FUSED = 8, /* the whole decode layer in one launch (T <= 8) */
    /* expert parallelism (ep_world > 1): the rows' sends to the owning GPUs; the wait for
     * every source and the received rows' routing table; the wait for every GPU's returned
     * outputs.  DISPATCH then covers the local dispatch of the received rows and COMBINE
     * the combine alone. */
    OBS_STAGE_EP_SEND = 9, OBS_STAGE_EP_RECV = 10, OBS_STAGE_EP_RETURN = 11
};
int obs_profile_enable(obs_ctx* ctx, int enable);
int obs_profile_read(obs_ctx* ctx, float* ms_total, int32_t* launches);
/* Pipeline trace of the gate/up grouped GEMM (diagnostics): while set, the
 * GEMM's CTA 0 writes %globaltimer (ns) into trace[role * n_steps + i] for
 * entry i of each role: 0 weight copy issued (per four k-groups), 1 token-tile
 * copies issued (per k-step), 2 dequant start, 3 dequant done, 8 dequant TMEM
 * stores done (per k-step, steps 0 mod 4, lane quarter 0), 10-12 dequant done
 * for lane quarters 1-3, 4 MMA pair ready, 9 MMA fence passed, 5 MMA pair
 * committed (per pair of k-steps), 6 epilogue start, 7 epilogue done (per
 * item), 13 token tile landed (per k-step).
 * When 14 * n_steps >= 24 * (SM count), the fused decode layer (T <= 8) writes
 * instead, for every CTA b, trace[24b + k]: k = 0 start, 1 router row done,
 * 2 stamped logits seen, 3 weight copies issued, 4 tiles done, 5 first combine
 * job's partials seen, 6 end, 7 top-k and input packs done, 8/9/10 first
 * tile's data landed / gate-up computed / tile done, 13/14 its down column
 * group landed / partials stored, 16-18 inside top-k (0 where a CTA has no
 * such phase).
 * trace = NULL switches it off.  Device memory of 14 * n_steps uint64. */
int obs_trace_enable(obs_ctx* ctx, uint64_t* trace, int n_steps);
/* No counterpart in the reference.  *count = the number of kernel launches the
 * library has issued in this process so far (all contexts and devices); the
 * difference around a region is how many of the library's kernels it ran. */
int obs_kernel_launches(uint64_t* count);
/* Waits for the stream and reports any device-side error flag (bounded waits
 * that gave up) raised since the last check; clears the flags. */
int obs_check_device(obs_ctx* ctx, void* stream);
/* Test hook, no counterpart in the reference: runs the gate/up grouped GEMM of
 * `layer` over a caller-given token-tile list (host int32 [n_tiles][4]:
 * expert, first row, rows, 0) on the context's activation scratch.  The GEMM
 * validates every tile (expert id, row range, the count against the tile
 * buffer) before any work; a bad list makes every CTA skip its work and
 * obs_check_device report OBS_ERR_INVALID.  Synchronises on the stream. */
int obs_debug_gemm_tiles(obs_ctx* ctx, int layer, const int32_t* tiles, int n_tiles, void* stream);
/* No counterpart in the reference (its waits are host-side and unbounded,
 * src/router.rs:47-48).  Every device-side wait of the context's kernels (GEMM
 * pipeline barriers, the fused decode layer's grid barriers, expert-parallel
 * peer stamps) gives up after limit_ns, records a timeout and returns, so a
 * stalled peer or pipeline ends in OBS_ERR_TIMEOUT from obs_check_device with
 * the GPU still answering.  limit_ns in [1 ms, 60 s]; 0 restores the default
 * 2 s.  Applies to work issued after the call. */
int obs_set_wait_limit(obs_ctx* ctx, uint64_t limit_ns);
/* Failure-path check without a failure: launches one bounded device wait on a
 * stamp that nothing writes -- the wait an expert-parallel receive runs for a
 * peer that never sends (same device code) -- which gives up after the wait
 * limit; obs_check_device then returns OBS_ERR_TIMEOUT and the context stays
 * usable. */
int obs_probe_wait(obs_ctx* ctx, void* stream);
/* ABI self-description for bindings in other languages: writes
 *   sizeof(obs_config), the offsets of its 12 fields in declaration order,
 *   sizeof(obs_layer_weights), the offsets of its 12 fields in declaration order,
 *   sizeof(obs_head_weights), the offsets of its 7 fields in declaration order
 * (34 values) into out[0 .. n), and returns 34.  A binding compares these with
 * its own struct layout (the reference passes its parameter structs by value
 * as #[repr(C)], src/forward.rs:22-28, src/router.rs:8-14). */
int obs_struct_layout(int32_t* out, int n);

/* ----------------------------------------------------- the layer stack */
/* The MoE input norm, rmsnorm.metal:9-37 (Model::rmsnorm, forward.rs:421):
 * out[t] = x[t] / sqrt(mean(x[t]^2) + rms_eps) * weight (weight NULL: 1), in
 * the reference kernel's own reduction order (bit-exact with the oracle).
 * x, out [T, hidden] bf16 device memory (out may not alias x). */
int obs_rmsnorm(obs_ctx* ctx, const uint16_t* x, const uint16_t* weight, int T, uint16_t* out, void* stream);
/* n_layers consecutive MoE layers on a residual stream r ([T, hidden] bf16,
 * device, updated in place), forward.rs:419-441 without the attention block
 * (BASELINE configs 2 and 3):
 *   for l = layer0 .. layer0 + n_layers - 1:  x = RMSNorm(r);  r = r + MoE_l(x)
 * (combine and residual summed in fp32, rounded once).  logit_bias as in
 * obs_moe_forward, applied to every layer.  Only stream-ordered work (CUDA
 * graph capture is fine); with expert parallelism every rank runs the same
 * layers. */
int obs_moe_stack_forward(obs_ctx* ctx, int layer0, int n_layers, uint16_t* resid, int T, const float* logit_bias,
                          int path, void* stream);

/* ----------------------------------------------- expert parallelism (EP) */
/* A context created with ep_world > 1 holds E/ep_world experts of each layer
 * (obs_load_layer takes all E experts' host or device arrays and keeps its own
 * slice; the router is replicated) and runs obs_moe_forward as expert
 * parallelism: every rank routes its own T tokens, writes each routed row
 * directly into the memory of the rank holding its expert (NVLink peer stores
 * through CUDA IPC), runs the grouped GEMMs on the rows it received, writes the
 * outputs back into the source rank's memory, and combines in rank order -- the
 * result equals the single-GPU forward bit for bit.  Replaces the per-layer
 * expert loop of forward.rs:164-247 when the experts span several GPUs (the
 * reference has no multi-device path).  Setup, once per context:
 *   obs_ep_handle(ctx, h)          this rank's buffer handle (OBS_EP_HANDLE_BYTES)
 *   ... exchange the handles between the ranks (host side, any transport) ...
 *   obs_ep_connect(ctx, all)       all = ep_world handles in rank order
 * Every rank must then call obs_moe_forward for the same layers in the same
 * order (T may differ, T = 0 included); the forward always takes the prefill
 * (grouped GEMM) path.  Device-side waits for peers are bounded (2 s) and end
 * in OBS_ERR_TIMEOUT from obs_check_device.  The stage entry points
 * (obs_dispatch, obs_expert_ffn, obs_expert_gemm_f32) are single-GPU only. */
#define OBS_EP_HANDLE_BYTES 64
int obs_ep_handle(obs_ctx* ctx, void* handle);
int obs_ep_connect(obs_ctx* ctx, const void* handles);
/* Expert placement (ep_world > 1).  experts[E] lists the global experts by slot:
 * GPU g holds experts[g*E/G .. (g+1)*E/G) as its local experts 0 .. E/G-1; every
 * expert appears once.  layer = -1 sets every layer.  Every rank must set the
 * same table.  A layer whose table changes is marked not loaded: load (or
 * synthesise) its weights again; obs_load_layer then keeps the listed experts.
 * The default is the identity (GPU g holds experts [g*E/G, (g+1)*E/G)).  The
 * result of a forward does not depend on the placement (bit for bit). */
int obs_ep_set_placement(obs_ctx* ctx, int layer, const int32_t* experts);
int obs_ep_get_placement(obs_ctx* ctx, int layer, int32_t* experts);
/* A balanced placement from per-expert loads (routed rows, e.g. a calibration
 * batch's histogram summed over the ranks); host only, no context.  Experts in
 * decreasing load (ties: lower id first) each go to the GPU with the smallest
 * total load among those with fewer than E/G experts (ties: lower GPU); each
 * GPU's experts are then listed in increasing id.  Writes experts[E]. */
int obs_ep_plan_placement(const int64_t* load, int n_experts, int world, int32_t* experts);

/* ------------------------------------------- allocation-free decode FFN */
/* No counterpart in the reference.  For callers that cannot allocate device
 * memory -- code running while a CUDA graph is being captured, hosts whose
 * framework owns every device byte through its own arena, latency-critical
 * loops that cannot pay for an allocation's implicit synchronisation -- this
 * computes, without a context and without allocating:
 *   out[t] = bf16([residual[t] +] sum_k weights[t,k] * down_e(silu(gate_e x_t) * up_e x_t)),
 * e = ids[t,k], the decode path's arithmetic, from expert weights in the
 * reference (MLX) layout given as device pointers in w (router fields unused).
 * Its scratch is one fixed device array inside the library (about 8 MB,
 * held on every GPU that loads the library until the process exits).
 * Limits: T * top_k <= OBS_STATIC_MAX_PAIRS, hidden a multiple of 512 up to
 * OBS_STATIC_MAX_HIDDEN, inter a multiple of 128 up to OBS_STATIC_MAX_INTER;
 * larger calls return OBS_ERR_INVALID.  ids must lie in [0, n_experts): an
 * out-of-range id reads expert 0.  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress); make that first call before
 * any stream capture.  All calls on a device share the array, so calls that
 * overlap on the GPU (different streams, no ordering) race; the arrival
 * counters are cleared at the start of each call. */
#define OBS_STATIC_MAX_PAIRS 64
#define OBS_STATIC_MAX_HIDDEN 4096
#define OBS_STATIC_MAX_INTER 1536
int obs_decode_ffn_static(const obs_layer_weights* w, int n_experts, int hidden, int inter, int top_k,
                          const uint16_t* x, const int32_t* ids, const float* weights,
                          const uint16_t* residual, int T, uint16_t* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* OBS_MOE_H */
