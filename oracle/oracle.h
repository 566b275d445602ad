/*
 * CPU oracle for the quantized decode hot path of g023/cuda_inf.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a scalar C restatement of the reference
 * algorithm (src/engine.cu and tools/export_weights.py of g023/cuda_inf) used as
 * the checker for the CUDA library.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it.  The product (cuda_inf_b200) never
 * links, loads or falls back to it.
 *
 * Pinning: the oracle is checked against golden vectors produced by the
 * reference's own code (tools/export_weights.py quantizer and format writer,
 * tools/make_index.py, and the reference kernels of src/engine.cu rebuilt for
 * sm_100a and run on a B200); see tests/golden/.
 *
 * Conventions: fp16 values are passed as raw uint16_t bit patterns, FP8 E4M3 as
 * uint8_t.  Every function mirrors one reference kernel or host block; the
 * citation is given beside it.
 */
#ifndef CUINF_ORACLE_H
#define CUINF_ORACLE_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar conversions ---- */
float    orc_h2f(uint16_t h);
uint16_t orc_f2h(float f);
/* FP8 E4M3 (OCP spec; bias 7, max finite 448, no inf).  Decode follows
 * e4m3f (engine.cu:27-30); encode follows f2e4m3 (engine.cu:24-26):
 * round-to-nearest-even with saturation to +-448, NaN stays NaN. */
float    orc_e4m3_to_f32(uint8_t b);
uint8_t  orc_f32_to_e4m3_sat(float x);

/* ---- offline format (tools/export_weights.py:64-79) ---- */
void orc_quant_int4_group(const float* w, int64_t N, int64_t K,
                          uint8_t* packed, uint16_t* scales);
void orc_dequant_int4(const uint8_t* packed, const uint16_t* scales,
                      int64_t N, int64_t K, float* w);

/* ---- kernels (engine.cu) ---- */
void orc_gemv_int4(const uint16_t* x, const uint8_t* packed, const uint16_t* scales,
                   float* y, int M, int N, int K);                 /* engine.cu:83-109 */
void orc_gemv_fp16(const uint16_t* x, const uint16_t* W, float* y,
                   int M, int N, int K);                           /* engine.cu:112-128 */
void orc_rmsnorm(const uint16_t* in, const uint16_t* w, uint16_t* out,
                 int M, int D, float eps);                         /* engine.cu:131-158 */
void orc_rope(uint16_t* q, uint16_t* k, const int* pos, int S, int nq, int nk,
              int head_dim, float theta);                          /* engine.cu:161-182 */
void orc_kv_write_tail(const uint16_t* k, const uint16_t* v, uint16_t* ktail,
                       uint16_t* vtail, int slot, int cnt, int nkv, int hd); /* 190-198 */
void orc_kv_commit_group(const uint16_t* ktail, const uint16_t* vtail,
                         uint8_t* kc8, uint8_t* vc8, uint16_t* ksc, uint16_t* vsc,
                         int dst_tok_base, int grp, int nkv, int hd);   /* 202-228 */
void orc_attn_decode(const uint16_t* q, const uint8_t* kc8, const uint8_t* vc8,
                     const uint16_t* ksc, const uint16_t* vsc,
                     const uint16_t* ktail, const uint16_t* vtail,
                     int committed, int qpos, float scale, uint16_t* out,
                     int nh, int nkv, int hd);                     /* 396-480 */
void orc_conv_pre(const float* inproj, uint16_t* C, uint16_t* Bx, int S, int H); /* 483-494 */
void orc_conv_apply(const uint16_t* Bx, const uint16_t* C, const uint16_t* w,
                    const uint16_t* state, uint16_t* y, int S, int H);       /* 498-512 */
void orc_conv_update_state(const uint16_t* Bx, uint16_t* state, int S, int H); /* 514-525 */
void orc_swiglu(const float* g, const float* u, uint16_t* out, int n);     /* 542-547 */
void orc_acc_scaled(uint16_t* dst, const float* src, float w, int n);      /* 556-559 */
void orc_add_inplace(uint16_t* a, const uint16_t* b, int n);               /* 527-530 */
void orc_add_f32_inplace(uint16_t* a, const float* b, int n);              /* 532-535 */
void orc_f32_to_f16(const float* src, uint16_t* dst, int n);               /* 537-540 */
/* MoE selection, host code at engine.cu:883-892 (sigmoid, +bias, top-k with
 * strict '>', weights = unbiased sigmoid / (sum + 1e-6)). */
void orc_moe_select(const float* logits, const float* bias, int n_exp, int topk,
                    int* idx, float* w);
/* argmax_kernel (engine.cu:562-572) with its blockDim of 256: returns the index
 * the reference kernel returns, ties included. */
int  orc_argmax(const float* logits, int n);

/* ---- whole model (engine.cu:784-940, decode path S == 1) ---- */
typedef struct {
    int32_t hidden, n_layers, n_heads, n_kv_heads, head_dim, vocab;
    int32_t n_dense, n_experts, top_k, moe_inter, dense_inter, conv_k;
    float   rope_theta, norm_eps;
    uint8_t attn_layer[64];
} orc_config;

typedef struct orc_model orc_model;
typedef struct orc_state orc_state;

/* blob = weights.bin bytes, index = index.bin bytes (tools/make_index.py:3-11).
 * The model keeps pointers into blob; the caller keeps blob alive. */
orc_model* orc_model_new(const orc_config* cfg, const uint8_t* blob, size_t blob_len,
                         const uint8_t* index, size_t index_len);
void       orc_model_free(orc_model* m);
orc_state* orc_state_new(const orc_model* m, int max_ctx);
void       orc_state_free(orc_state* s);
int        orc_state_pos(const orc_state* s);
/* Resume from a sequence-state snapshot in the layout documented at
 * cuinf_session_save_state (KV cache, group scales, fp16 tails and conv state
 * at a position; the reference keeps this state only in its device Buffers,
 * engine.cu:590-623).  Returns 0, or -1 when the snapshot does not fit this
 * model or state. */
int        orc_state_load(const orc_model* m, orc_state* s, const uint8_t* buf, size_t n);
/* One token through all layers at position state->pos, then the final norm,
 * lm_head and argmax.  Writes fp32 logits when logits != NULL and the final
 * hidden state (pre-norm, fp16) when hidden != NULL.  Returns the argmax. */
int        orc_forward_token(const orc_model* m, orc_state* s, int token,
                             float* logits, uint16_t* hidden);
/* Same, with optional forced expert choices [n_moe][top_k] (the weights are
 * recomputed from the oracle's router for those experts) and the oracle's
 * own selection scores sigmoid(logit)+bias written to scores [n_moe][E]. */
int        orc_forward_token_ex(const orc_model* m, orc_state* s, int token,
                                const int* forced_idx, float* scores,
                                float* logits, uint16_t* hidden);
/* Prefill of S tokens at positions pos..pos+S-1 the way the reference's
 * batched layer_forward(S) does it (all of a layer's K/V placed and full
 * groups committed before any query attends), then the last row's logits.
 * Returns their argmax; state->pos advances by S. */
int        orc_prefill(const orc_model* m, orc_state* s, const int* tokens, int S, float* logits_out);
/* Same, with optional forced experts [S][n_moe][top_k] and the oracle's own
 * selection scores written to scores [S][n_moe][E]. */
int        orc_prefill_ex(const orc_model* m, orc_state* s, const int* tokens, int S,
                          const int* forced_idx, float* scores, float* logits_out);
/* H2O eviction mode (engine.cu:310-384, 803-828), set before the first
 * token: `budget` per-token FP8 slots per attention layer, local window W.
 * own/used slots: per layer, the slot this oracle chose / used in the last
 * step (-1 for other layers); force: the next decode step uses these slots
 * per layer (-1 or NULL: its own choice). */
int          orc_state_set_h2o(const orc_model* m, orc_state* s, int budget, int window);
const int*   orc_state_h2o_own_slots(const orc_state* s);
const int*   orc_state_h2o_used_slots(const orc_state* s);
const float* orc_state_h2o_attn_sum(const orc_state* s, int layer);
const int*   orc_state_h2o_slot_pos(const orc_state* s, int layer);
int          orc_state_h2o_n_live(const orc_state* s, int layer);
void         orc_state_force_h2o_slots(orc_state* s, const int* slots);
/* Router decisions of the last forward_token: [n_moe_layers][top_k]. */
const int*   orc_state_route_idx(const orc_state* s);
const float* orc_state_route_w(const orc_state* s);

void orc_set_threads(int n);
int  orc_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
