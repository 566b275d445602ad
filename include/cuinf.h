/*
 * cuinf — B200-native (sm_100a) quantized decode hot path of g023/cuda_inf.
 *
 * C ABI.  Plain pointers and sizes only.  Device pointers are CUDA device
 * addresses owned by the caller unless stated otherwise; `stream` is a
 * cudaStream_t passed as void* (NULL = legacy default stream).
 *
 * Every function returns 0 on success, CUINF_ERR_ARG for a rejected argument
 * or CUINF_ERR_CUDA for a CUDA error; cuinf_last_error() gives the message.
 * Nothing here exits the process (the reference's CK() macro calls exit(1),
 * src/engine.cu:52-53).  Launches are asynchronous on `stream`.
 *
 * Reference citations are src/engine.cu of g023/cuda_inf unless a tools/ file
 * is named.  Where the reference hard-codes a dimension with a #define
 * (H, NH, NKV, HEAD_DIM, ...; engine.cu:33-50) the entry point takes it as an
 * argument; HEAD_DIM is fixed at 64 and the KV group at 64 tokens.
 *
 * fp16 data is IEEE binary16; FP8 is OCP E4M3 (the __NV_E4M3 of the reference).
 */
#ifndef CUINF_H
#define CUINF_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CUINF_OK 0
#define CUINF_ERR_ARG 1
#define CUINF_ERR_CUDA 2
#define CUINF_ERR_IO 3

/* Message of the most recent error on the calling thread ("" if none). */
const char* cuinf_last_error(void);
/* Library version string. */
const char* cuinf_version(void);

/* ------------------------------------------------------------------------ */
/* Operators: the kernel-level signatures of src/engine.cu, plus a stream.     */
/* ------------------------------------------------------------------------ */

/* y[m,n] = sum_k x[m,k] * (nib(W[n,k]) - 8) * scale[n, k/128], fp32 out.
 * x fp16 [M,K]; packed u8 [N,K/2] (low nibble = even k); scales fp16 [N,K/128]
 * (tools/export_weights.py:64-79 layout); K % 128 == 0.
 * Replaces gemv_int4 (engine.cu:83-109) + run_gemv_int4 (engine.cu:626-630). */
int cuinf_gemv_int4(const void* x, const uint8_t* packed, const void* scales, float* y,
                    int M, int N, int K, void* stream);

/* y[m,n] = sum_k x[m,k] * W[n,k], fp16 weights, fp32 out; K % 32 == 0.
 * Replaces gemv_fp16 (engine.cu:112-128) + run_gemv_fp16 (engine.cu:631-635). */
int cuinf_gemv_fp16(const void* x, const void* W, float* y, int M, int N, int K, void* stream);

/* out[m,:] = half(in[m,:] * rsqrt(mean(in^2) + eps) * w), in/out fp16 [M,D]
 * (may alias).  Replaces rmsnorm (engine.cu:131-144) and, with D = 64,
 * rmsnorm_head (engine.cu:148-158). */
int cuinf_rmsnorm(const void* in, const void* w, void* out, int M, int D, float eps, void* stream);

/* In-place NEOX RoPE on q fp16 [S,nq,64] and k fp16 [S,nk,64] at absolute
 * positions pos (device int [S]); inv_freq = theta^(-2d/64).
 * Replaces rope (engine.cu:161-182; theta = ROPE_THETA 5e6). */
int cuinf_rope(void* q, void* k, const int* pos, int S, int nq, int nk, float theta, void* stream);

/* Copy cnt tokens of k,v fp16 [cnt,nkv,64] into the tail at slot..slot+cnt-1.
 * Replaces kv_write_tail (engine.cu:190-198). */
int cuinf_kv_write_tail(const void* k, const void* v, void* ktail, void* vtail, int slot, int cnt,
                        int nkv, void* stream);

/* Commit the full 64-token tail to FP8 E4M3 at tokens dst_tok_base..+63 with
 * one fp16 scale per kv head: scale = absmax/448 + 1e-12, stored at
 * ksc/vsc[grp*nkv + h]; values quantized with the fp32 scale, satfinite.
 * kc8/vc8 u8 [T,nkv,64]; ktail/vtail fp16 [64,nkv,64].
 * Replaces kv_commit_group (engine.cu:202-228). */
int cuinf_kv_commit_group(const void* ktail, const void* vtail, uint8_t* kc8, uint8_t* vc8,
                          void* ksc, void* vsc, int dst_tok_base, int grp, int nkv, void* stream);

/* Workspace bytes cuinf_attn_decode needs for nh query heads. */
size_t cuinf_attn_decode_workspace_size(int nh, int nkv, int max_ctx);

/* Single-token flash-decoding attention over the FP8 cache [0, committed)
 * and the fp16 tail [committed, qpos]: out[h,:] = softmax(q_h . K^T * scale) V.
 * q/out fp16 [nh,64]; GQA group nh/nkv.  workspace: device scratch of
 * cuinf_attn_decode_workspace_size(nh, nkv, qpos+1) bytes, or NULL to use a
 * library-owned buffer (allocated on first use).
 * Replaces attn_decode_split + attn_decode_combine (engine.cu:396-480). */
int cuinf_attn_decode(const void* q, const uint8_t* kc8, const uint8_t* vc8, const void* ksc,
                      const void* vsc, const void* ktail, const void* vtail, int committed,
                      int qpos, float scale, void* out, int nh, int nkv, void* workspace,
                      size_t workspace_bytes, void* stream);

/* Same attention as cuinf_attn_decode, for callers that must not allocate
 * device memory (an allocator callback that calls back into this library, a
 * memory pool that forbids cudaMalloc, a host that has reserved all HBM up
 * front).  It allocates nothing: its split-K scratch is a static device array
 * of cuinf_attn_decode_static_scratch_bytes() (512 KiB) bytes inside the
 * library.  The first call on a device sets up (looks up that array's
 * address); make that first call before any stream capture on the device.
 * Shapes
 * whose scratch would exceed 512 KiB are rejected with CUINF_ERR_ARG: on a
 * B200, 8 kv heads x 4 query heads each (the model's shape) need at most
 * 0.31 MiB; 8 kv heads x 8 query heads need more than 512 KiB past 1920
 * tokens and are rejected there.
 * The scratch is shared by every call on a device, so calls on one device
 * must not overlap: issue them on one stream or order them with events;
 * overlapping calls race on the scratch.  The scratch's 256-byte ticket area
 * must start at zero; each call clears it on the stream before its launch.
 * The looked-up address is kept per device for the life of the process: a
 * device that uses this entry point must not be reset (cudaDeviceReset)
 * while the library is loaded, since the array's address may then change.
 * No counterpart in the reference. */
size_t cuinf_attn_decode_static_scratch_bytes(void);
int cuinf_attn_decode_noalloc(const void* q, const uint8_t* kc8, const uint8_t* vc8,
                              const void* ksc, const void* vsc, const void* ktail,
                              const void* vtail, int committed, int qpos, float scale, void* out,
                              int nh, int nkv, void* stream);

/* Short-conv pieces (H channels): inproj fp32 [S,3H] = B | C | x.
 * conv_pre: C = half(C), Bx = half(B*x)            (engine.cu:483-494)
 * conv_apply: y = half(C * (Bx[s-2]w0 + Bx[s-1]w1 + Bx[s]w2)), history from
 *             state fp16 [2,H], w fp16 [H,3]     (engine.cu:498-512)
 * conv_update_state: state <- last two Bx      (engine.cu:514-525) */
int cuinf_conv_pre(const float* inproj, void* C, void* Bx, int S, int H, void* stream);
int cuinf_conv_apply(const void* Bx, const void* C, const void* w, const void* state, void* y,
                     int S, int H, void* stream);
int cuinf_conv_update_state(const void* Bx, void* state, int S, int H, void* stream);

/* Elementwise (engine.cu:527-559). */
int cuinf_swiglu(const float* g, const float* u, void* out, int n, void* stream);      /* 542 */
int cuinf_acc_scaled(void* dst, const float* src, float w, int n, void* stream);      /* 556 */
int cuinf_add_inplace(void* a, const void* b, int n, void* stream);                   /* 527 */
int cuinf_add_f32_inplace(void* a, const float* b, int n, void* stream);              /* 532 */
int cuinf_f32_to_f16(const float* src, void* dst, int n, void* stream);               /* 537 */
int cuinf_embed_gather(const void* embed, const int* ids, void* out, int S, int H,
                       void* stream);                                                 /* 549 */

/* Index of the maximum of logits[n] with argmax_kernel's tie rule
 * (engine.cu:562-572).  out: device int. */
int cuinf_argmax(const float* logits, int n, int* out, void* stream);

/* MoE selection on the device for S tokens: sig = sigmoid(logit);
 * score = sig + bias; top-k by score (strict '>', lowest index on ties);
 * w = sig[sel] / (sum + 1e-6).  logits fp32 [S,n_exp], bias fp16 [n_exp];
 * idx int [S,topk], w fp32 [S,topk].  Replaces the host loop at
 * engine.cu:883-892 (which needs a D2H copy and a sync per MoE layer). */
int cuinf_moe_route(const float* logits, const void* bias, int S, int n_exp, int topk, int* idx,
                    float* w, void* stream);

/* Fused MoE FFN for one token (engine.cu:877-905): xn = the ffn-normed hidden
 * state fp16 [H]; router gate fp16 [n_exp,H]; expert_bias fp16 [n_exp];
 * experts: device array of n_exp*6 pointers {w1.packed, w1.scales,
 * w3.packed, w3.scales, w2.packed, w2.scales} (w1,w3 [I,H], w2 [H,I]).
 * h fp16 [H] is updated in place: h = half(h + acc), acc accumulated in fp16
 * over the selected experts in rank order.  idx/w (device, may be NULL)
 * receive the routing decision.  workspace: cuinf_moe_ffn_workspace_size
 * bytes, 16-byte aligned, whose first 256 + topk*H*8 bytes are zero before
 * the first call (every call leaves them zero), or NULL for a library-owned
 * buffer per device.  Calls sharing a workspace must not overlap. */
size_t cuinf_moe_ffn_workspace_size(int H, int I, int topk);
int cuinf_moe_ffn(const void* xn, const void* gate, const void* expert_bias,
                  const void* const* experts, void* h, int H, int I, int n_exp, int topk,
                  int* idx, float* w, void* workspace, size_t workspace_bytes, void* stream);

/* INT4 G=128 quantizer of tools/export_weights.py:64-79, bit-exact:
 * scale = amax/7 (fp32), q = rint(w/scale) clipped to [-7,7], nibble q+8,
 * scale stored fp16.  Device version (w, packed, scales device pointers) and
 * host version (host pointers).  K % 128 == 0. */
int cuinf_quantize_int4(const float* w, int64_t N, int64_t K, uint8_t* packed, void* scales,
                        void* stream);
int cuinf_quantize_int4_host(const float* w, int64_t N, int64_t K, uint8_t* packed,
                             uint16_t* scales);

/* ------------------------------------------------------------------------ */
/* Decode engine (replaces main's layer_forward / decode loop,                 */
/* engine.cu:784-963): the model of tools/export_weights.py in one device      */
/* blob, per-session KV/conv state, one decode step = one CUDA graph launch.   */
/* ------------------------------------------------------------------------ */
typedef struct {
    int32_t hidden, n_layers, n_heads, n_kv_heads, head_dim, vocab;
    int32_t n_dense, n_experts, top_k, moe_inter, dense_inter, conv_k;
    float rope_theta, norm_eps;
    uint8_t attn_layer[64]; /* 1 = attention layer, 0 = short-conv layer */
} cuinf_config;

/* The LFM2.5-8B-A1B configuration of engine.cu:33-50. */
void cuinf_default_config(cuinf_config* cfg);

typedef struct cuinf_model cuinf_model;
typedef struct cuinf_session cuinf_session;

/* Load dir/index.bin + dir/weights.bin (tools/make_index.py format) into one
 * device blob (engine.cu:664-692).  cfg NULL = cuinf_default_config. */
int cuinf_model_load(const char* dir, const cuinf_config* cfg, cuinf_model** out);
/* Wrap an existing device blob laid out like weights.bin; index = index.bin
 * bytes (host).  The blob is not copied and must outlive the model. */
int cuinf_model_from_device_blob(const cuinf_config* cfg, void* d_blob, size_t blob_bytes,
                                 const uint8_t* index, size_t index_bytes, cuinf_model** out);
int cuinf_model_free(cuinf_model* m);

/* Session: KV cache (FP8 + fp16 tail) and conv state for max_ctx tokens, on
 * `stream` (NULL = a new stream owned by the session). */
int cuinf_session_create(cuinf_model* m, int max_ctx, void* stream, cuinf_session** out);
int cuinf_session_free(cuinf_session* s);
/* Clear the KV cache and conv state; position back to 0. */
int cuinf_session_reset(cuinf_session* s);
int cuinf_session_pos(const cuinf_session* s);

/* Snapshots of a sequence's recurrent state at its position p: the FP8 KV
 * cache of every attention layer (C = 64*floor(p/64) committed tokens, their
 * group scales, the fp16 tails) and the conv state of every short-conv layer.
 * The reference keeps this state only in device buffers for the life of the
 * process (Buffers, engine.cu:590-623); a snapshot lets a caller park a
 * sequence on the host and resume it later (or start a session at a long
 * context from a stored prompt state).  Layout (little-endian):
 *   u32 magic 0x54534943, u32 version 1, i32 pos, i32 n_layers, i32 hidden,
 *   i32 n_kv_heads, i32 reserved[2]; then per layer in order:
 *   attention: kc8 u8 [C][nkv][64], vc8 same, ksc fp16 [C/64][nkv], vsc same,
 *              ktail fp16 [64][nkv][64] (slots 0..p-C-1 hold tokens C..p-1),
 *              vtail same;
 *   short-conv: state fp16 [2][hidden].
 * cuinf_session_state_bytes gives the size at the session's position.  save
 * copies device -> host; load checks the header against the model, copies
 * host -> device and moves the session to the snapshot's position (the next
 * cuinf_decode_step must pass its token explicitly).  Both synchronize the
 * session's stream.  Not available in H2O eviction mode. */
size_t cuinf_session_state_bytes(const cuinf_session* s);
int cuinf_session_save_state(cuinf_session* s, void* host, size_t n);
int cuinf_session_load_state(cuinf_session* s, const void* host, size_t n);

/* One token through all layers + final norm + lm_head + argmax, at the
 * session's position (then position + 1).  token >= 0 is the input token
 * (copied host->device); token < 0 feeds back the previous step's argmax,
 * which never leaves the device.  out_token (host, nullable) receives the
 * argmax after a stream sync.  Asynchronous when out_token == NULL. */
int cuinf_decode_step(cuinf_session* s, int token, int* out_token);
/* Tensor-core GEMMs for batched decode and prefill (no counterpart in the
 * reference, which runs gemv_int4 / gemv_fp16 with grid.y = M,
 * engine.cu:83-128): tcgen05 MMA with the accumulator in TMEM, weights
 * streamed by 2-D TMA.  cuinf_gemm_int4_tc computes the same y[M,N] fp32 as
 * cuinf_gemv_int4: the MMA sums exact products (nib-8)*x per 128-K group and
 * each group's sum is scaled in fp32, so results differ from the reference
 * only by fp32 summation order.
 * cuinf_gemm_fp16_tc: y[M,N] = x[M,K] . W[N,K]^T (y nullable) and, when
 * argmax_keys (device u64 [M], zeroed by the caller) is given, a fused
 * per-row argmax with the reference's tie rule (argmax_kernel, 562-572);
 * decode a key with cuinf_argmax_key_index.  K a multiple of 128, all
 * pointers 16-byte aligned.  Split-K uses a library-owned workspace, so calls
 * on a device must not overlap. */
int cuinf_gemm_int4_tc(const void* x, const uint8_t* packed, const void* scales, float* y, int M, int N, int K,
                       void* stream);
int cuinf_gemm_fp16_tc(const void* x, const void* W, float* y, int M, int N, int K,
                       unsigned long long* argmax_keys, void* stream);
int cuinf_argmax_key_index(unsigned long long key);
/* Sequence-batched decode (single GPU): n_seqs (<= 128)
 * independent sequences, each with its own FP8 KV cache and conv state,
 * advance one token per cuinf_batch_step.  Per sequence the arithmetic is
 * the reference's decode step (layer_forward with S = 1, engine.cu:784-908;
 * compute_logits_last, 932-940); the projections run on the tensor-core
 * GEMMs and the MoE experts as grouped GEMMs over the tokens routed to them.
 * No counterpart in the reference, which decodes one sequence.
 * tokens (host [n_seqs], nullable: feed back each sequence's last argmax);
 * out_tokens (host [n_seqs], nullable; synchronizes).  All sequences start at
 * position 0; cuinf_batch_fill_synthetic sets every sequence to position
 * ctx over pseudo-random FP8 caches (benchmarking at a context length).
 * cuinf_batch_routes: host [n_moe_layers][n_seqs][top_k] experts of the last
 * step.  cuinf_batch_logits: device [n_seqs][vocab] while keep_logits is on. */
typedef struct cuinf_batch cuinf_batch;
int cuinf_batch_create(cuinf_model* m, int n_seqs, int max_ctx, void* stream, cuinf_batch** out);
/* Expert-parallel form (BASELINE config 5 on `world` <= 8 GPUs of one node,
 * one process per GPU): this rank decodes its own n_seqs sequences and hosts
 * experts [rank*E/world, (rank+1)*E/world); per MoE layer each (token, slot)
 * row goes to its expert's rank and the fp32 expert output comes back.
 * The exchange writes the rows straight into the receiving rank's memory
 * (every rank's exchange arena is mapped into every process with cudaIpc;
 * only the rows that exist cross NVLink, the sender's own rows stay local)
 * and raises a flag there that the receiver's next kernel waits for (at most
 * 4 s, then bit 4 (value 16) of cuinf_batch_error's first word is set).  When an arena cannot be
 * mapped on some rank, every rank uses NCCL send/recv of fixed capacity
 * (n_seqs*top_k rows per peer) instead.  nccl_id: cuinf_ep_unique_id on
 * rank 0, broadcast to all ranks.  Every rank steps together. */
int cuinf_batch_create_ep(cuinf_model* m, int n_seqs, int max_ctx, void* stream, const unsigned char* nccl_id,
                          int rank, int world, cuinf_batch** out);
/* The exchange an expert-parallel batch uses: 1 peer memory, 0 NCCL
 * send/recv, -1 not expert-parallel. */
int cuinf_batch_ep_exchange(const cuinf_batch* b);
/* Select the exchange (1 peer memory, 0 NCCL) and rebuild the step graph.
 * All ranks must make the same choice between the same two steps. */
int cuinf_batch_set_ep_exchange(cuinf_batch* b, int peer_memory);
int cuinf_ep_unique_id(unsigned char* id, int id_bytes);
int cuinf_ep_unique_id_bytes(void);
/* Failure handling of the expert-parallel form (the reference runs on one
 * GPU and has none).  The communicator is non-blocking: its setup, every
 * group of sends/receives and every host wait on a step (cuinf_batch_step
 * with out_tokens or tokens, cuinf_batch_sync) poll NCCL's asynchronous
 * error state and give up after the batch's time limit (default 120 s,
 * cuinf_batch_set_timeout).  On an NCCL error or a time-out, or on
 * cuinf_batch_abort (a host that learned a peer failed), the communicator is
 * aborted, which releases kernels still waiting for peers; the batch then
 * refuses further steps (cuinf_batch_failed returns 1) and must be freed. */
/* The dispatch plan of one MoE layer, on the host (the device computes the
 * same inside the step): entry j = token j/top_k, slot j%top_k, routed to
 * expert ridx[j], goes to rank d = ridx[j] / e_loc at position r = the count
 * of earlier entries for d; dest_pos[j] = d*cap + r and meta[d*cap + r] =
 * the expert's index on d, -1 where a position is unused.  The expert's
 * output row returns to back[dest_pos[j]], and token j/top_k combines its
 * slots in slot order (acc_scaled, engine.cu:900-902). */
int cuinf_ep_plan_host(const int* ridx, int n, int e_loc, int world, int cap, int* dest_pos, int* meta);
int cuinf_batch_sync(cuinf_batch* b);
int cuinf_batch_abort(cuinf_batch* b);
int cuinf_batch_set_timeout(cuinf_batch* b, int timeout_ms);
int cuinf_batch_failed(const cuinf_batch* b);
int cuinf_batch_free(cuinf_batch* b);
int cuinf_batch_reset(cuinf_batch* b);
int cuinf_batch_step(cuinf_batch* b, const int* tokens, int* out_tokens);
int cuinf_batch_keep_logits(cuinf_batch* b, int on);
const float* cuinf_batch_logits(const cuinf_batch* b);
int cuinf_batch_routes(cuinf_batch* b, int* idx);
int cuinf_batch_kernels_per_step(const cuinf_batch* b);
int cuinf_batch_fill_synthetic(cuinf_batch* b, int ctx, unsigned long long seed);
/* Per-sequence state snapshots of a batch, in the layout of
 * cuinf_session_save_state (a snapshot moves freely between sessions and
 * batches of the same model): the size at sequence seq's position, save
 * (device -> host) and load (host -> device, which also sets that sequence's
 * position; its next token must be passed explicitly).  Synchronous. */
size_t cuinf_batch_seq_state_bytes(cuinf_batch* b, int seq);
int cuinf_batch_save_seq(cuinf_batch* b, int seq, void* host, size_t n);
int cuinf_batch_load_seq(cuinf_batch* b, int seq, const void* host, size_t n);
/* Error words of the tensor-core kernels, flags[4]: [0] bit 1 a bounded
 * pipeline wait timed out, bit 2 a final drain did, bit 3 a group had more
 * rows than its launch allowed (skipped); [1] the wait's barrier
 * code, [2] its block, [3] its stage counter (first failure). */
int cuinf_batch_error(unsigned* flags);
/* One step launched eagerly with an event after each launch: ms[i] is the
 * duration of launch i, names[i * name_len] its name; advances the batch. */
int cuinf_batch_profile_step(cuinf_batch* b, int max_kernels, float* ms, char* names, int name_len,
                             int* n_kernels);
/* Tokenizer (the reference's src/tokenizer.h and its files from
 * tools/export_tokenizer.py: vocab.tsv, merges.tsv, special.tsv in `dir`):
 * GPT-2 byte-level BPE with the reference's pre-tokenizer rules and literal
 * special tokens.  encode: *n_out = the full count (ids holds the first cap);
 * decode: *len_out = the full byte length (out holds the first cap).
 * cuinf_chat_prompt: the reference's single-turn template (engine.cu:697-699). */
typedef struct cuinf_tokenizer cuinf_tokenizer;
int cuinf_tokenizer_load(const char* dir, cuinf_tokenizer** out);
int cuinf_tokenizer_free(cuinf_tokenizer* t);
int cuinf_tokenizer_vocab_size(const cuinf_tokenizer* t);
int cuinf_tokenizer_encode(const cuinf_tokenizer* t, const char* text, size_t len, int* ids, int cap, int* n_out);
int cuinf_tokenizer_decode(const cuinf_tokenizer* t, const int* ids, int n, int skip_special, char* out, size_t cap,
                           size_t* len_out);
int cuinf_chat_prompt(const char* user, char* out, size_t cap, size_t* len_out);
/* Batched prompt processing, replacing the reference's prefill
 * (src/engine.cu:910-917: layer_forward with S = n_ids, 784-908): every layer
 * runs on all S tokens at positions pos..pos+S-1; each attention layer first
 * places all S keys/values (FP8-committing every full 64-token group,
 * 831-845), then every query attends over them (attention_fused, 236-308);
 * then the last row's logits and argmax (compute_logits_last, 932-940).
 * Synchronous; the session continues with cuinf_decode_step(s, -1, ...) from
 * position pos + S.  out_token (host, nullable) receives the argmax;
 * routes_out (host, nullable) [S][n_layers - n_dense][top_k] the expert ids
 * each token chose in each MoE layer.  Results differ from feeding the same
 * ids through decode steps exactly as the reference's prefill does. */
int cuinf_prefill(cuinf_session* s, const int* ids, int n_ids, int* out_token, int* routes_out);
/* Greedy generation like the reference's main (engine.cu:910-965): the prompt
 * through cuinf_prefill (or, with CUINF_OPT_PREFILL off, one decode step per
 * prompt id), then n_new tokens (stop early on eos >= 0).  out_ids host
 * [n_new]; returns the number generated in *n_out. */
int cuinf_generate(cuinf_session* s, const int* prompt, int n_prompt, int n_new, int eos,
                   int* out_ids, int* n_out);
/* Device pointer to this session's last fp32 logits [vocab] (filled only while
 * cuinf_session_keep_logits(s, 1) is set) and its final hidden state fp16 [H]. */
int cuinf_session_keep_logits(cuinf_session* s, int on);
/* Session options (rebuild the step graph; both default to 1):
 * CUINF_OPT_PREFETCH: each kernel pulls the next kernels' weights into L2;
 * CUINF_OPT_PDL: kernels launch with programmatic stream serialization so a
 * kernel's weight staging overlaps its predecessor. */
#define CUINF_OPT_PREFETCH 1
#define CUINF_OPT_PDL 2
/* CUINF_OPT_MEGAKERNEL: run the step as one persistent cooperative kernel
 * (one CTA per SM, TMA weight ring, grid barriers between stages) instead of
 * the captured multi-kernel graph (default 0); falls back to the graph when
 * the device or model does not fit. */
#define CUINF_OPT_MEGAKERNEL 3
/* CUINF_OPT_TRACE: the megakernel records %globaltimer at every stage start
 * and end of every CTA (read with cuinf_session_trace; default 0). */
#define CUINF_OPT_TRACE 4
/* CUINF_OPT_PREFILL: cuinf_generate consumes its prompt with cuinf_prefill,
 * as the reference does (default 1); 0 feeds it through decode steps. */
#define CUINF_OPT_PREFILL 5
/* CUINF_OPT_ATTN_CLUSTER: decode attention merges the splits of a kv head
 * over distributed shared memory inside a thread-block cluster (default 1;
 * used when the device holds all kv heads' clusters at once); 0 merges them
 * through global memory with an atomic ticket.  Both use the same splits and
 * give the same results. */
#define CUINF_OPT_ATTN_CLUSTER 6
/* CUINF_OPT_PREFETCH_MB / CUINF_OPT_PREFETCH_AHEAD: the L2 prefetch plan of
 * CUINF_OPT_PREFETCH: each kernel asks L2 for at most `value` MB (default 12,
 * 1..1024) of the weights of the kernels at most `value` launches after it
 * (default 3, 1..64).  Scheduling only: results do not change. */
#define CUINF_OPT_PREFETCH_MB 7
#define CUINF_OPT_PREFETCH_AHEAD 8
/* 1 if this session's decode attention can merge over clusters. */
int cuinf_session_attn_cluster(const cuinf_session* s);
int cuinf_session_set_option(cuinf_session* s, int option, int value);
/* H2O eviction mode (the reference's --kv-budget / --kv-window,
 * engine.cu:310-384, 579-581, 753-756, 803-828): each attention layer keeps
 * `budget` per-token FP8 slots (own per-head fp16 scale, logical position,
 * cumulative attention mass); once full, a fresh token takes the slot with
 * the least mass outside the last `window` positions (first minimum), else
 * the least overall.  window <= 0: budget/2.  budget 0 turns it off.  Only
 * before the first token; budget <= 8192; prompts must fit the budget.  The
 * slot choice runs on the device, inside the step graph.  The decode step
 * then uses the multi-kernel graph (not the megakernel). */
int cuinf_session_set_kv_budget(cuinf_session* s, int budget, int window);
/* Host copies of one attention layer's H2O state: slot positions and
 * cumulative attention [budget], live slots, slot of the last step. */
int cuinf_session_h2o_state(cuinf_session* s, int layer, int* slot_pos, float* attn_sum, int* n_live,
                            int* last_slot);
/* Device error flags of the engine kernels (bit 0: a bounded wait on a
 * weight-staging barrier timed out and the kernel skipped its math). */
int cuinf_device_error(unsigned* flags);
/* Self test of the failure path of those bounded waits (no counterpart in
 * the reference, whose kernels have no waits): one CTA arms a barrier for
 * bytes that never arrive and waits at most limit_us microseconds; flags
 * receives bit 0 when the wait gave up (expected) and bit 1 if the barrier
 * completed; waited_ns the time the wait took.  The context stays usable. */
int cuinf_selftest_wait_timeout(unsigned limit_us, unsigned* flags, unsigned long long* waited_ns);
/* Per-stage timestamps of the last traced megakernel step: buf receives
 * [n_stages][n_ctas][16]: %globaltimer ns at the stage start, prologue end
 * and end (words 0, 1, 3); SM cycles spent waiting for weight slabs (2); SM cycles
 * since the stage start for: pre-slab ready (4), the first item's slab
 * ready, dot done, epilogue done (5-7), MoE-up norm, router dots and expert
 * selection done (8-10); %clock64 at the stage start (11); the producer's
 * %clock64 at its pre-slab issue (12), first item ready to place (13) and
 * first item issue (14); SM cycles from the stage start to the prologue end
 * (15).  0 where a stage has no such point.  kinds (nullable) [n_stages]. */
int cuinf_session_trace(cuinf_session* s, unsigned long long* buf, int cap, int* kinds, int* n_stages,
                        int* n_ctas);
/* 1 when this session's step runs as the persistent megakernel. */
int cuinf_session_uses_megakernel(const cuinf_session* s);
/* Megakernel error state of this session (synchronizes its stream), 4 words:
 * flags[0] bits: 0 abort, 1 grid-barrier time-out, 2 producer ring time-out,
 * 3 producer routing time-out, 4 consumer slab time-out (0 = none);
 * flags[1..3]: stage, CTA and slab number of the first failure. */
int cuinf_session_error(cuinf_session* s, unsigned* flags);
const float* cuinf_session_logits(const cuinf_session* s);
const void* cuinf_session_hidden(const cuinf_session* s);
/* Host copy of the last step's routing decisions [n_moe_layers*top_k]. */
int cuinf_session_routes(cuinf_session* s, int* idx, float* w);
/* Number of kernels one decode step launches (for the bench's accounting). */
int cuinf_session_kernels_per_step(const cuinf_session* s);
/* One decode step launched kernel by kernel (not as the graph) with a CUDA
 * event after each launch: ms[i] = duration of kernel i, bytes[i] = its
 * algorithmic bytes (weights + activations), names[i*name_len] its name.
 * Advances the session like cuinf_decode_step. */
int cuinf_session_profile_step(cuinf_session* s, int token, int max_kernels, float* ms,
                               double* bytes, char* names, int name_len, int* n_kernels);

#ifdef __cplusplus
}
#endif
#endif
