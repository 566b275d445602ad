// Model and KV-state layout shared by the decode engines: the tensors of
// weights.bin resolved through index.bin (tools/export_weights.py:96-129,
// read by engine.cu:665-675 of the reference).
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include <string>
#include <unordered_map>
#include <vector>

#include "cuinf.h"

struct TDesc {
    uint8_t kind;
    uint64_t offset, packed, scales;
    int64_t d0, d1;
};
struct Q4 {
    const uint8_t* p = nullptr;
    const __half* s = nullptr;
};
struct LayerW {
    const __half *op_norm = nullptr, *ffn_norm = nullptr;
    Q4 wq, wk, wv, wo, in_proj, out_proj, w1, w3, w2;
    const __half *q_ln = nullptr, *k_ln = nullptr, *conv_w = nullptr, *gate = nullptr,
                 *ebias = nullptr;
    int moe_index = -1;  // index into the expert table / route buffers
};

struct cuinf_model {
    cuinf_config cfg;
    uint8_t* d_blob = nullptr;
    size_t blob_bytes = 0;
    bool own_blob = false;
    std::unordered_map<std::string, TDesc> idx;
    std::vector<LayerW> L;
    const __half *embed = nullptr, *emb_norm = nullptr;
    void** d_experts = nullptr;  // [n_moe][E][6]
    int n_moe = 0;
    void* tc_cache = nullptr;    // tensor-core prefill state (expert tensor maps, scratch), built on first use
};

// Grouped MoE FFN of S tokens of one sequence (prefill): h[S][H] += the
// reference's per-token expert mix, with the experts' weights streamed once
// per chunk of tokens by the tensor-core GEMM.  ridx (device, nullable)
// receives the experts [S][top_k].  Calls on one model must not overlap.
int moe_grouped_prefill(cuinf_model* m, int layer, const __half* xn, __half* h, int S, int* ridx,
                        cudaStream_t st);
void tc_cache_free(cuinf_model* m);
int kv_commit_rows(const __half* k, const __half* v, uint8_t* kc8, uint8_t* vc8, __half* ksc, __half* vsc,
                   int n_groups, int tok_base, int grp0, int nkv, cudaStream_t st);

struct AttnState {
    uint8_t *kc8 = nullptr, *vc8 = nullptr;
    __half *ksc = nullptr, *vsc = nullptr, *ktail = nullptr, *vtail = nullptr;
};


// One sequence's recurrent state in the snapshot layout of
// cuinf_session_save_state (include/cuinf.h): copies between a host buffer
// and the device pieces (attn[l] / conv[l], per layer; null where the layer
// has no such piece) on `st`, synchronously.  save: device -> host.
size_t seq_state_bytes(const cuinf_config& c, int pos);
int seq_state_copy(const cuinf_config& c, int pos, const AttnState* attn, __half* const* conv, void* host,
                   size_t n, bool save, cudaStream_t st);
// Reads and checks a snapshot's header; returns its position through *pos.
int seq_state_header(const cuinf_config& c, const void* host, size_t n, int max_ctx, int* pos);

// Decode attention over B sequences (grid z), each at its own device
// position: q [B][nh*64], caches at the given per-sequence element strides,
// partials [B][part_floats], counters [B][nkv] (zero, left zero).
struct BatchAttnArgs {
    const __half* q;
    const uint8_t *kc8, *vc8;
    const __half *ksc, *vsc, *ktail, *vtail;
    const int* pos;
    __half* out;
    float* part;
    unsigned* counters;
    int nh, nkv, nsplit, n_seqs;
    size_t bq, bkv8, bsc, btail, bout, bpart;
    float scale;
};
int attn_decode_batched(const BatchAttnArgs& a, cudaStream_t st);
int attn_batched_nsplit(int nh, int nkv, int max_ctx, int n_seqs, int num_sms);
size_t attn_batched_part_floats(int nh, int nkv, int nsplit);
