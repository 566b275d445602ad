// Launchers for the reference's own kernels, for parity checks and golden
// fixtures.  TEST INFRASTRUCTURE ONLY.
//
// This file contains no reference code: it includes src/engine.cu of
// g023/cuda_inf from the reference tree at build time (-I<reference>/src, see
// oracle/Makefile) with main renamed, and exposes each __global__ kernel behind
// an extern "C" function that launches it with the grid/block/shared-memory
// configuration the reference's host code uses (line numbers are
// src/engine.cu).  Dimensions are the reference's compile-time constants
// (H=2048, NH=32, NKV=8, HEAD_DIM=64, NSPLIT=16, VOCAB=128000).
#define main ref_main
#include "engine.cu"
#undef main

static int ref_status() { return (int)cudaGetLastError(); }

extern "C" {

// run_gemv_int4, 626-630
int ref_gemv_int4(const void* x, const uint8_t* packed, const void* scales, float* y,
                  int M, int N, int K, cudaStream_t st) {
    dim3 grid((N + 7) / 8, M);
    gemv_int4<<<grid, 256, (size_t)K * 4, st>>>((const half*)x, packed, (const half*)scales, y,
                                               N, K, K / GROUP);
    return ref_status();
}

// run_gemv_fp16, 631-635
int ref_gemv_fp16(const void* x, const void* W, float* y, int M, int N, int K, cudaStream_t st) {
    dim3 grid((N + 7) / 8, M);
    gemv_fp16<<<grid, 256, (size_t)K * 4, st>>>((const half*)x, (const half*)W, y, N, K);
    return ref_status();
}

// rmsnorm launch at 789 (block 256)
int ref_rmsnorm(const void* in, const void* w, void* out, int M, int D, float eps, cudaStream_t st) {
    rmsnorm<<<M, 256, 0, st>>>((const half*)in, (const half*)w, (half*)out, M, D, eps);
    return ref_status();
}

// rmsnorm_head launch at 799 (block HEAD_DIM)
int ref_rmsnorm_head(const void* in, const void* w, void* out, int rows, float eps, cudaStream_t st) {
    rmsnorm_head<<<rows, HEAD_DIM, 0, st>>>((const half*)in, (const half*)w, (half*)out, rows,
                                            HEAD_DIM, eps);
    return ref_status();
}

// rope launch at 801 (grid S, block HEAD_DIM/2)
int ref_rope(void* q, void* k, const int* pos, int S, cudaStream_t st) {
    rope<<<S, HEAD_DIM / 2, 0, st>>>((half*)q, (half*)k, pos, S, NH, NKV);
    return ref_status();
}

// kv_write_tail launch at 838
int ref_kv_write_tail(const void* k, const void* v, void* ktail, void* vtail, int slot, int cnt,
                      cudaStream_t st) {
    int n = cnt * NKV * HEAD_DIM;
    kv_write_tail<<<(n + 255) / 256, 256, 0, st>>>((const half*)k, (const half*)v, (half*)ktail,
                                                   (half*)vtail, slot, cnt);
    return ref_status();
}

// kv_commit_group launch at 841
int ref_kv_commit_group(const void* ktail, const void* vtail, uint8_t* kc8, uint8_t* vc8,
                        void* ksc, void* vsc, int dst_tok_base, int grp, cudaStream_t st) {
    kv_commit_group<<<NKV, 256, 0, st>>>((const half*)ktail, (const half*)vtail, kc8, vc8,
                                         (half*)ksc, (half*)vsc, dst_tok_base, grp);
    return ref_status();
}

// attn_decode_split + attn_decode_combine, 846-852.  pm/pl hold NH*NSPLIT
// floats, po NH*NSPLIT*HEAD_DIM floats.
int ref_attn_decode(const void* q, const uint8_t* kc8, const uint8_t* vc8, const void* ksc,
                    const void* vsc, const void* ktail, const void* vtail, int committed,
                    int qpos, float scale, float* pm, float* pl, float* po, void* out,
                    cudaStream_t st) {
    dim3 g(NH, NSPLIT);
    size_t sm = (size_t)(2 * ADEC_THREADS + ADEC_THREADS * HEAD_DIM) * sizeof(float);
    attn_decode_split<<<g, ADEC_THREADS, sm, st>>>(
        (const half*)q, kc8, vc8, (const half*)ksc, (const half*)vsc, (const half*)ktail,
        (const half*)vtail, committed, qpos, scale, pm, pl, po);
    attn_decode_combine<<<NH, HEAD_DIM, 0, st>>>(pm, pl, po, (half*)out);
    return ref_status();
}

// conv launches at 862-865
int ref_conv_pre(const float* inproj, void* C, void* Bx, int S, cudaStream_t st) {
    conv_pre<<<(S * H + 255) / 256, 256, 0, st>>>(inproj, (half*)C, (half*)Bx, S);
    return ref_status();
}
int ref_conv_apply(const void* Bx, const void* C, const void* w, void* state, void* y, int S,
                   cudaStream_t st) {
    conv_apply<<<(S * H + 255) / 256, 256, 0, st>>>((const half*)Bx, (const half*)C,
                                                    (const half*)w, (half*)state, (half*)y, S);
    return ref_status();
}
int ref_conv_update_state(const void* Bx, void* state, int S, cudaStream_t st) {
    conv_update_state<<<(H + 255) / 256, 256, 0, st>>>((const half*)Bx, (half*)state, S);
    return ref_status();
}

// elementwise launches at 859, 874, 901, 904, 794
int ref_swiglu(const float* g, const float* u, void* out, int n, cudaStream_t st) {
    swiglu<<<(n + 255) / 256, 256, 0, st>>>(g, u, (half*)out, n);
    return ref_status();
}
int ref_acc_scaled(void* dst, const float* src, float w, int n, cudaStream_t st) {
    acc_scaled<<<(n + 255) / 256, 256, 0, st>>>((half*)dst, src, w, n);
    return ref_status();
}
int ref_add_inplace(void* a, const void* b, int n, cudaStream_t st) {
    add_inplace<<<(n + 255) / 256, 256, 0, st>>>((half*)a, (const half*)b, n);
    return ref_status();
}
int ref_add_f32_inplace(void* a, const float* b, int n, cudaStream_t st) {
    add_f32_inplace<<<(n + 255) / 256, 256, 0, st>>>((half*)a, b, n);
    return ref_status();
}
int ref_f32_to_f16(const float* src, void* dst, int n, cudaStream_t st) {
    f32_to_f16<<<(n + 255) / 256, 256, 0, st>>>(src, (half*)dst, n);
    return ref_status();
}
int ref_embed_gather(const void* embed, const int* ids, void* out, int S, cudaStream_t st) {
    embed_gather<<<(S * H + 255) / 256, 256, 0, st>>>((const half*)embed, ids, (half*)out, S);
    return ref_status();
}
// argmax launch at 937 (1 block of 256)
int ref_argmax(const float* logits, int n, int* out, cudaStream_t st) {
    argmax_kernel<<<1, 256, 0, st>>>(logits, n, out);
    return ref_status();
}

// FP8 round trip through the reference's own helpers (24-30), elementwise.
__global__ void ref_fp8_kernel(const float* x, uint8_t* enc, float* dec, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint8_t b = f2e4m3(x[i]);
    enc[i] = b;
    dec[i] = e4m3f(b);
}
int ref_fp8_roundtrip(const float* x, uint8_t* enc, float* dec, int n, cudaStream_t st) {
    ref_fp8_kernel<<<(n + 255) / 256, 256, 0, st>>>(x, enc, dec, n);
    return ref_status();
}

int ref_dims(int* out) {
    out[0] = H; out[1] = NL; out[2] = HEAD_DIM; out[3] = NH; out[4] = NKV; out[5] = VOCAB;
    out[6] = NEXP; out[7] = TOPK; out[8] = MOE_INTER; out[9] = DENSE_INTER; out[10] = NSPLIT;
    return 0;
}

}  // extern "C"
