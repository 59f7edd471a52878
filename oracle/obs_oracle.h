/*
 * obs_oracle.h -- CPU restatement of project-obsidian's MoE hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path in
 * project-obsidian_b200/: only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py load it.  The product library never links it.
 *
 * Every routine cites the reference file:line whose arithmetic it restates
 * (paths relative to the vladiclick/project-obsidian tree).  Conventions that
 * the reference leaves open are fixed here once and shared with the CUDA
 * kernels (router reduction order, top-k on fp32 logits, rank-order combine).
 *
 * Layouts (all row-major, little-endian, MLX affine quantisation):
 *   8-bit router  W  uint32 [E, H/4]   byte i of a row = column i   (dequant_matvec_8bit.metal:20,26)
 *   4-bit expert  W  uint32 [out, in/8] nibble j of word = (w>>4j)&15 (fused_dequant_matvec_4bit.metal:39-42,
 *                                                                     validate_dequant.py:24-29)
 *   scales/biases bf16 [rows, in/64], index row*groups + g           (fused_dequant_matvec_4bit.metal:33-35)
 *   activations   bf16 [T, features]
 */
#ifndef OBS_ORACLE_H
#define OBS_ORACLE_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* ---- bf16 helpers (round to nearest even, as __float2bfloat16_rn) ---- */
float    orc_bf16_to_f32(uint16_t h);
uint16_t orc_f32_to_bf16(float f);

/* ---- seeded synthetic data: bit-identical twin of the device generator ----
 * Counter-based splitmix64 streams keyed by (seed, layer, tensor, index).
 * Uniforms are 24-bit; normals are the Irwin-Hall sum of 12 uniforms minus 6
 * (exact integer arithmetic, so host and device agree bit for bit). */
enum {
    ORC_T_ROUTER_W = 0, ORC_T_ROUTER_S = 1,
    ORC_T_GATE_W = 2, ORC_T_GATE_S = 3, ORC_T_GATE_B = 4,
    ORC_T_UP_W = 5,   ORC_T_UP_S = 6,   ORC_T_UP_B = 7,
    ORC_T_DOWN_W = 8, ORC_T_DOWN_S = 9, ORC_T_DOWN_B = 10,
    ORC_T_X = 11
};
uint64_t orc_stream_key(uint64_t seed, uint32_t layer, uint32_t tensor);
uint64_t orc_stream_u64(uint64_t key, uint64_t idx);
/* router: codes U{0..255}, s ~ U(0.0005,0.005) as bf16, b = -128 s */
void orc_synth_router(uint64_t seed, uint32_t layer, int E, int H,
                      uint32_t* w, uint16_t* s, uint16_t* b);
/* one projection of all experts: codes U{0..15}, s ~ U(0.002,0.02), b = -8 s + N(0,1e-3)
 * proj: 0 gate, 1 up, 2 down.  w [E, out, in/8], s/b [E, out, in/64] */
void orc_synth_proj(uint64_t seed, uint32_t layer, int proj, int E, int out_f, int in_f,
                    uint32_t* w, uint16_t* s, uint16_t* b);
/* activations: x ~ N(0,1) rounded to bf16, then RMSNorm (eps, weight 1), bf16 out.
 * Rows [row0, row0+T) of the stream, so any slice matches the full tensor. */
void orc_synth_x(uint64_t seed, uint32_t layer, int row0, int T, int H, float eps, uint16_t* x);

/* ---- a8: RMSNorm (rmsnorm.metal:20-36), sequential sum of squares ---- */
void orc_rmsnorm_row(const uint16_t* x, int H, float eps, uint16_t* out);
void orc_rmsnorm_tg_row(const uint16_t* x, const uint16_t* w, int H, float eps, uint16_t* out);
float orc_rms_tg(const uint16_t* x, int H, float eps);

/* ---- a1/a4 dequant (dequant_matvec_8bit.metal:22-27, fused_dequant_matvec_4bit.metal:33-45) ----
 * value = fmaf(q, scale, bias) in fp32.  For these formats q*scale is exact in
 * fp32, so this equals the reference's mul-then-add. */
void orc_dequant4(const uint32_t* w, const uint16_t* s, const uint16_t* b,
                  int out_f, int in_f, float* out);
/* The tensor-core path's weights: bf16 nearest-even rounding of the exact
 * q*scale + bias (one rounding, as fma.rn.bf16x2).  bf16 [out, in]. */
void orc_dequant4_bf16(const uint32_t* w, const uint16_t* s, const uint16_t* b,
                       int out_f, int in_f, uint16_t* out);
void orc_dequant8(const uint32_t* w, const uint16_t* s, const uint16_t* b,
                  int out_f, int in_f, float* out);

/* ---- a1: router logits, canonical fp32 order ----
 * Groups of 64 columns; 32 lanes; lane l owns groups [l*m, (l+1)*m) with
 * m = (H/64)/32 and chains acc = fmaf(w, x, acc) over them in column order;
 * the 32 lane sums are then combined by the adjacent pairwise tree
 * (offsets 1,2,4,8,16 -- a warp xor-butterfly).  logits fp32 [T, E]. */
int orc_router_logits(const uint32_t* w, const uint16_t* s, const uint16_t* b,
                      const uint16_t* x, int T, int H, int E, float* logits);

/* ---- a2: softmax / top-k / renormalise (moe_routing_topk.metal:31-56) ----
 * Selection on fp32 logits (+ optional per-expert bias), strict '>' so the
 * lowest index wins ties; weights p_k / sum(p_topk) when norm != 0. */
void orc_topk(const float* logits, const float* bias, int T, int E, int K, int norm,
              int32_t* ids, float* weights);

/* ---- a3: dispatch (forward.rs:176-216 grouping, canonical order) ----
 * counts[e]; offsets[e] = exclusive scan (offsets[E] = T*K); slots ordered by
 * expert then token; slot_of[t*K+k] = slot; src_token[slot] = t. */
void orc_dispatch(const int32_t* ids, int T, int E, int K,
                  int32_t* counts, int32_t* offsets, int32_t* slot_of, int32_t* src_token);

/* ---- a4/a5/a6: expert FFN + combine for a whole layer ----
 * wmode 0: weights dequantised in fp32 (reference matvec);
 * wmode 1: weights rounded once to bf16 (orc_dequant4_bf16, tensor-core GEMM path).
 * g,u fp32; h = bf16(silu(g)*u) (ops.metal:21); y = bf16(W_d h);
 * out[t] = bf16(residual[t] + sum_k w_k y_k) in rank order (forward.rs:225-232),
 * residual may be NULL.  Optional y_out [T*K, H] bf16 (slot = t*K+k) for tests. */
typedef struct {
    int E, H, I, K;
    const uint32_t *gate_w, *up_w, *down_w;
    const uint16_t *gate_s, *gate_b, *up_s, *up_b, *down_s, *down_b;
} orc_experts;
int orc_moe_ffn_combine(const orc_experts* ex, const uint16_t* x, int T,
                        const int32_t* ids, const float* weights, const uint16_t* residual,
                        int wmode, int nthreads, uint16_t* out, uint16_t* h_out, uint16_t* y_out);

/* full layer: logits -> topk -> ffn -> combine.  Returns 0 on success. */
typedef struct {
    orc_experts ex;
    const uint32_t* router_w; const uint16_t* router_s; const uint16_t* router_b;
} orc_layer;
int orc_moe_layer(const orc_layer* L, const uint16_t* x, int T, const float* logit_bias,
                  const uint16_t* residual, int norm_topk, int wmode, int nthreads,
                  uint16_t* out, int32_t* ids_out, float* w_out);

/* ---- the model's ends (config 4; src/forward.rs:445-462, :553-566) ----
 * Embedding: out[t][i] = bf16(fmaf(q, s, b)) of row tokens[t] (4-bit MLX layout,
 * nibble i%8 of word i/8, low nibble first).
 * lm_head logits fp32 [T, vocab] of the normalised rows x (bf16 [T, H]) in the
 * canonical order: w = fmaf(q, s, b); 32 lanes, lane l chains acc = fmaf(w, x,
 * acc) over its groups l*m .. (l+1)*m-1 (m = H/2048) in column order; the lane
 * sums meet in the adjacent pairwise tree (offsets 1, 2, 4, 8, 16).  argmax: the
 * first maximum (forward.rs:562-565).  Returns -1 if H is not a multiple of 2048. */
void orc_embed(const uint32_t* w, const uint16_t* s, const uint16_t* b, int vocab, int H,
               const int32_t* tokens, int T, uint16_t* out);
int orc_lm_head_logits(const uint32_t* w, const uint16_t* s, const uint16_t* b, int vocab, int H,
                       const uint16_t* x, int T, int nthreads, float* logits);
void orc_argmax_rows(const float* logits, int T, int n, int32_t* ids);

/* ---- the attention block (config 4; src/forward.rs:404-419) ----
 * The CUDA block's arithmetic: RMSNorm in rmsnorm.metal's order; q/k/v/o in the
 * lm_head's canonical order (orc_lm_head_logits); projections rounded to bf16;
 * per-head RMSNorm of q and k; NeoX RoPE (rope.metal:10-27) with cos/sin from
 * orc_rope_table (double precision) and a = x1*s, o0 = fmaf(x0, c, -a),
 * b = x0*s, o1 = fmaf(x1, c, b); K/V appended to the caches; scores
 * q.k * (1/sqrtf(hd)) with the dot product in the kernel's lane order (32 lanes
 * over head_dim, then the xor tree); softmax with expf; out = x + bf16(o). */
typedef struct {
    int H, nq, nkv, hd, max_seq, n_seqs;
    const uint32_t *q_w, *k_w, *v_w, *o_w;
    const uint16_t *q_s, *q_b, *k_s, *k_b, *v_s, *v_b, *o_s, *o_b;
    const uint16_t *in_norm, *q_norm, *k_norm;
    const float* rope;   /* [max_seq][hd/2][2] */
    uint16_t *kc, *vc;   /* [n_seqs][nkv][max_seq][hd] */
} orc_attn;
void orc_rope_table(double theta, int hd, int max_seq, float* out);
int orc_attn_forward(const orc_attn* A, const uint16_t* x, int T, const int32_t* seq, const int32_t* pos,
                     float eps, int nthreads, uint16_t* out);

#ifdef __cplusplus
}
#endif
#endif
