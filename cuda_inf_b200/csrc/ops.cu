// Standalone operators of the C ABI (include/cuinf.h): the kernel-level
// signatures of the reference (src/engine.cu of g023/cuda_inf), rebuilt for
// sm_100a.  The fused decode-step kernels live in engine.cu.
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <string>

#include "common.cuh"
#include "route.cuh"

// Device-side error word of this translation unit (bit 0: a bounded wait on
// a weight-staging barrier timed out).
static __device__ unsigned g_ops_err;

// ---------------------------------------------------------------------------
// status
// ---------------------------------------------------------------------------
static thread_local std::string g_last_error;

int cuinf_set_cuda_error(cudaError_t e) {
    g_last_error = std::string("CUDA error: ") + cudaGetErrorString(e);
    return CUINF_ERR_CUDA;
}
int cuinf_set_arg_error(const char* what) {
    g_last_error = std::string("invalid argument: ") + what;
    return CUINF_ERR_ARG;
}
int cuinf_launch_status() {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuinf_set_cuda_error(e);
    return CUINF_OK;
}

extern "C" const char* cuinf_last_error(void) { return g_last_error.c_str(); }
extern "C" const char* cuinf_version(void) { return "cuinf-b200 0.1 (sm_100a)"; }

#define ST(s) ((cudaStream_t)(s))
#define REQUIRE(cond, msg) \
    do {                   \
        if (!(cond)) return cuinf_set_arg_error(msg); \
    } while (0)

// ---------------------------------------------------------------------------
// INT4 GEMV (gemv_int4, engine.cu:83-109)
// grid (ceil(N/16), M), 256 threads.  Each CTA owns one 16-row tile: thread 0
// stages the tile (packed rows + scales) into shared memory with TMA bulk
// copies while the CTA permutes x into B-fragment order; the 8 warps then
// take the K groups w, w+8, ... (ragged or unaligned tiles use direct loads).
// Launched with programmatic stream serialization: the weights (which no
// earlier kernel writes) are requested before the dependency wait, so a
// GEMV that follows another kernel streams its tile while that kernel
// finishes; x is read, and y written, only after the wait.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_gemv_int4(const __half* __restrict__ x,
                                                   const uint8_t* __restrict__ packed,
                                                   const __half* __restrict__ scales,
                                                   float* __restrict__ y, int N, int K, int use_tma, int xvec) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t bar;
    const int m = blockIdx.y, row0 = blockIdx.x * 16;
    const bool tma = use_tma && row0 + 16 <= N;
    uint8_t* tile = smem;
    __half* xB = reinterpret_cast<__half*>(smem + (use_tma ? int4_tile_bytes(K) : 0));
    float* red = reinterpret_cast<float*>(xB + K);  // [8][16]
    if (tma) {
        if (threadIdx.x == 0) mbar_init(&bar, 1);
        __syncthreads();
        if (threadIdx.x == 0) {
            mbar_arrive_expect_tx(&bar, int4_tile_bytes(K));
            tma_tile_int4(packed, scales, K, row0, tile, &bar);
        }
    }
    pdl_trigger();
    pdl_wait();
    const __half* xm = x + (size_t)m * K;
    if (xvec)  // x 16-byte aligned: one 16-byte load per 8 elements
        for (int i = threadIdx.x; i < K / 8; i += blockDim.x) build_xB_chunk(xm, xB, i);
    else
        for (int e = threadIdx.x; e < K / 4; e += blockDim.x) build_xB_entry(xm, xB, e);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float y0 = 0.f, y1 = 0.f;
    if (tma) {
        if (mbar_wait_bounded(&bar, 0, &g_ops_err))
            int4_tile_dot_smem<2>(tile, K, warp, K >> 7, 8, reinterpret_cast<const uint2*>(xB), y0, y1);
    } else {
        int4_tile_dot<2>(packed, scales, N, K, row0, warp, K >> 7, 8,
                         reinterpret_cast<const uint2*>(xB), y0, y1);
    }
    if ((lane & 3) == 0) {
        red[warp * 16 + (lane >> 2)] = y0;
        red[warp * 16 + (lane >> 2) + 8] = y1;
    }
    __syncthreads();
    if (threadIdx.x < 16) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++) s += red[w * 16 + threadIdx.x];
        int n = row0 + threadIdx.x;
        if (n < N) y[(size_t)m * N + n] = s;
    }
}

extern "C" int cuinf_gemv_int4(const void* x, const uint8_t* packed, const void* scales, float* y,
                               int M, int N, int K, void* stream) {
    REQUIRE(x && packed && scales && y, "null pointer");
    REQUIRE(M > 0 && N > 0 && K > 0, "M, N, K must be positive");
    REQUIRE(K % 128 == 0, "K must be a multiple of 128 (INT4 group size)");
    REQUIRE(((uintptr_t)packed & 15) == 0, "packed must be 16-byte aligned");
    REQUIRE(((uintptr_t)scales & 1) == 0 && ((uintptr_t)x & 1) == 0, "misaligned fp16 pointer");
    REQUIRE(M <= 65535, "M too large");
    const int use_tma = ((uintptr_t)scales & 15) == 0;
    const int xvec = ((uintptr_t)x & 15) == 0;  // K % 128 == 0 keeps every row aligned too
    size_t smem = (size_t)K * 2 + 8 * 16 * 4 + (use_tma ? int4_tile_bytes(K) : 0);
    REQUIRE(smem <= 227 * 1024, "K too large");
    if (smem > 48 * 1024)
        CUINF_TRY(cudaFuncSetAttribute(k_gemv_int4, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((N + 15) / 16, M);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ST(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CUINF_TRY(cudaLaunchKernelEx(&cfg, k_gemv_int4, (const __half*)x, packed, (const __half*)scales, y, N, K,
                                 use_tma, xvec));
    return cuinf_launch_status();
}

// ---------------------------------------------------------------------------
// fp16 GEMV (gemv_fp16, engine.cu:112-128): grid (ceil(N/16), M), 256 threads
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_gemv_fp16(const __half* __restrict__ x,
                                                   const __half* __restrict__ W,
                                                   float* __restrict__ y, int N, int K) {
    extern __shared__ __align__(128) unsigned char smem[];
    __half* xs = reinterpret_cast<__half*>(smem);
    float* red = reinterpret_cast<float*>(smem + (size_t)K * 2);
    const int m = blockIdx.y, row0 = blockIdx.x * 16;
    for (int i = threadIdx.x; i < K; i += blockDim.x) xs[i] = x[(size_t)m * K + i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float y0 = 0.f, y1 = 0.f;
    f16_tile_dot<2>(W, N, K, row0, warp, K >> 5, 8, xs, y0, y1);
    if ((lane & 3) == 0) {
        red[warp * 16 + (lane >> 2)] = y0;
        red[warp * 16 + (lane >> 2) + 8] = y1;
    }
    __syncthreads();
    if (threadIdx.x < 16) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++) s += red[w * 16 + threadIdx.x];
        int n = row0 + threadIdx.x;
        if (n < N) y[(size_t)m * N + n] = s;
    }
}

extern "C" int cuinf_gemv_fp16(const void* x, const void* W, float* y, int M, int N, int K,
                               void* stream) {
    REQUIRE(x && W && y, "null pointer");
    REQUIRE(M > 0 && N > 0 && K > 0 && K % 32 == 0, "K must be a positive multiple of 32");
    REQUIRE(((uintptr_t)W & 15) == 0 && ((uintptr_t)x & 1) == 0, "W must be 16-byte aligned");
    REQUIRE(M <= 65535, "M too large");
    size_t smem = (size_t)K * 2 + 8 * 16 * 4;
    REQUIRE(smem <= 200 * 1024, "K too large");
    if (smem > 48 * 1024)
        CUINF_TRY(cudaFuncSetAttribute(k_gemv_fp16, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
    dim3 grid((N + 15) / 16, M);
    k_gemv_fp16<<<grid, 256, smem, ST(stream)>>>((const __half*)x, (const __half*)W, y, N, K);
    return cuinf_launch_status();
}

// ---------------------------------------------------------------------------
// RMSNorm (engine.cu:131-158): one CTA per row
// ---------------------------------------------------------------------------
__global__ void k_rmsnorm(const __half* __restrict__ in, const __half* __restrict__ w,
                          __half* out, int D, float eps) {
    __shared__ float red[32];
    const __half* row = in + (size_t)blockIdx.x * D;
    float ss = 0.f;
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        float v = __half2float(row[i]);
        ss += v * v;
    }
    ss = block_sum(ss, red);
    float inv = rsqrtf(ss / (float)D + eps);
    __syncthreads();  // in may alias out: all reads of row finished above
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        float v = __half2float(row[i]);
        out[(size_t)blockIdx.x * D + i] = __float2half_rn(v * inv * __half2float(w[i]));
    }
}

extern "C" int cuinf_rmsnorm(const void* in, const void* w, void* out, int M, int D, float eps,
                             void* stream) {
    REQUIRE(in && w && out, "null pointer");
    REQUIRE(M > 0 && D > 0, "M, D must be positive");
    int threads = D >= 256 ? 256 : ((D + 31) / 32) * 32;
    k_rmsnorm<<<M, threads, 0, ST(stream)>>>((const __half*)in, (const __half*)w, (__half*)out, D,
                                              eps);
    return cuinf_launch_status();
}

// ---------------------------------------------------------------------------
// RoPE (engine.cu:161-182): grid S, 32 threads (one per rotation pair)
// ---------------------------------------------------------------------------

__global__ void k_rope(__half* q, __half* k, const int* __restrict__ pos, int nq, int nk,
                       float theta) {
    const int s = blockIdx.x, d = threadIdx.x;
    if (d >= CUINF_HD / 2) return;
    float cs, sn;
    rope_pair_angle(pos[s], d, theta, cs, sn);
    for (int pass = 0; pass < 2; pass++) {
        __half* base = pass ? k : q;
        int nh = pass ? nk : nq;
        for (int h = 0; h < nh; h++) {
            __half* b = base + ((size_t)s * nh + h) * CUINF_HD;
            float x0 = __half2float(b[d]), x1 = __half2float(b[d + 32]);
            b[d] = __float2half_rn(x0 * cs - x1 * sn);
            b[d + 32] = __float2half_rn(x1 * cs + x0 * sn);
        }
    }
}

extern "C" int cuinf_rope(void* q, void* k, const int* pos, int S, int nq, int nk, float theta,
                          void* stream) {
    REQUIRE(q && pos && (k || nk == 0), "null pointer");
    REQUIRE(S > 0 && nq >= 0 && nk >= 0, "bad sizes");
    k_rope<<<S, 32, 0, ST(stream)>>>((__half*)q, (__half*)k, pos, nq, nk, theta);
    return cuinf_launch_status();
}

// ---------------------------------------------------------------------------
// FP8 KV cache (engine.cu:190-228)
// ---------------------------------------------------------------------------
__global__ void k_kv_write_tail(const __half* __restrict__ k, const __half* __restrict__ v,
                                __half* ktail, __half* vtail, int slot, int n, int row) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    size_t dst = (size_t)slot * row + i;
    ktail[dst] = k[i];
    vtail[dst] = v[i];
}

extern "C" int cuinf_kv_write_tail(const void* k, const void* v, void* ktail, void* vtail, int slot,
                                   int cnt, int nkv, void* stream) {
    REQUIRE(k && v && ktail && vtail, "null pointer");
    REQUIRE(slot >= 0 && cnt > 0 && slot + cnt <= CUINF_KVGROUP && nkv > 0, "slot range");
    int n = cnt * nkv * CUINF_HD;
    k_kv_write_tail<<<(n + 255) / 256, 256, 0, ST(stream)>>>(
        (const __half*)k, (const __half*)v, (__half*)ktail, (__half*)vtail, slot, n, nkv * CUINF_HD);
    return cuinf_launch_status();
}

// FP8 E4M3 helpers (the reference's f2e4m3 / e4m3f, engine.cu:24-30).
__device__ __forceinline__ uint8_t f32_to_e4m3(float x) {
    return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}

// One CTA per kv head; 256 threads.  Quantizes the 64 x 64 fp16 tail block of
// head h with the fp32 scale absmax/448 + 1e-12 and stores the fp16 scale.
__device__ __forceinline__ void kv_commit_head(const __half* __restrict__ tail, uint8_t* c8,
                                               __half* sc, int h, int nkv, int dst_tok_base,
                                               int grp, float* red) {
    float mx = 0.f;
    for (int e = threadIdx.x; e < CUINF_KVGROUP * CUINF_HD; e += blockDim.x) {
        int t = e >> 6, d = e & 63;
        mx = fmaxf(mx, fabsf(__half2float(tail[((size_t)t * nkv + h) * CUINF_HD + d])));
    }
    mx = warp_max(mx);
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[w] = mx;
    __syncthreads();
    float amax = 0.f;
    for (int i = 0; i < nw; i++) amax = fmaxf(amax, red[i]);
    float s = amax / 448.0f + 1e-12f;
    if (threadIdx.x == 0) sc[grp * nkv + h] = __float2half_rn(s);
    for (int e = threadIdx.x; e < CUINF_KVGROUP * CUINF_HD; e += blockDim.x) {
        int t = e >> 6, d = e & 63;
        float v = __half2float(tail[((size_t)t * nkv + h) * CUINF_HD + d]);
        c8[((size_t)(dst_tok_base + t) * nkv + h) * CUINF_HD + d] = f32_to_e4m3(v / s);
    }
}

__global__ void k_kv_commit_group(const __half* __restrict__ ktail, const __half* __restrict__ vtail,
                                  uint8_t* kc8, uint8_t* vc8, __half* ksc, __half* vsc,
                                  int dst_tok_base, int grp, int nkv) {
    __shared__ float red[32];
    const int h = blockIdx.x;
    kv_commit_head(ktail, kc8, ksc, h, nkv, dst_tok_base, grp, red);
    __syncthreads();
    kv_commit_head(vtail, vc8, vsc, h, nkv, dst_tok_base, grp, red);
}

extern "C" int cuinf_kv_commit_group(const void* ktail, const void* vtail, uint8_t* kc8,
                                     uint8_t* vc8, void* ksc, void* vsc, int dst_tok_base, int grp,
                                     int nkv, void* stream) {
    REQUIRE(ktail && vtail && kc8 && vc8 && ksc && vsc, "null pointer");
    REQUIRE(dst_tok_base >= 0 && grp >= 0 && nkv > 0, "bad sizes");
    k_kv_commit_group<<<nkv, 256, 0, ST(stream)>>>((const __half*)ktail, (const __half*)vtail, kc8,
                                                    vc8, (__half*)ksc, (__half*)vsc, dst_tok_base,
                                                    grp, nkv);
    return cuinf_launch_status();
}

// Prefill: n whole groups committed straight from rows [64n][nkv][64] of new
// keys and values (each group's rows have the tail's layout, so the result
// is what writing them to the tail and committing would give).  grid (n, nkv).
__global__ void k_kv_commit_rows(const __half* __restrict__ k, const __half* __restrict__ v, uint8_t* kc8,
                                 uint8_t* vc8, __half* ksc, __half* vsc, int tok_base, int grp0, int nkv) {
    __shared__ float red[32];
    const int g = blockIdx.x, h = blockIdx.y;
    const size_t off = (size_t)g * CUINF_KVGROUP * nkv * CUINF_HD;
    kv_commit_head(k + off, kc8, ksc, h, nkv, tok_base + g * CUINF_KVGROUP, grp0 + g, red);
    __syncthreads();
    kv_commit_head(v + off, vc8, vsc, h, nkv, tok_base + g * CUINF_KVGROUP, grp0 + g, red);
}
int kv_commit_rows(const __half* k, const __half* v, uint8_t* kc8, uint8_t* vc8, __half* ksc, __half* vsc,
                   int n_groups, int tok_base, int grp0, int nkv, cudaStream_t st) {
    if (n_groups <= 0) return CUINF_OK;
    k_kv_commit_rows<<<dim3(n_groups, nkv), 256, 0, st>>>(k, v, kc8, vc8, ksc, vsc, tok_base, grp0, nkv);
    return cuinf_launch_status();
}

// ---------------------------------------------------------------------------
// short conv (engine.cu:483-525)
// ---------------------------------------------------------------------------
__global__ void k_conv_pre(const float* __restrict__ inproj, __half* C, __half* Bx, int S, int H) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= S * H) return;
    int s = i / H, c = i % H;
    const float* row = inproj + (size_t)s * 3 * H;
    C[i] = __float2half_rn(row[H + c]);
    Bx[i] = __float2half_rn(row[c] * row[2 * H + c]);
}

// y = half(C * ((bx[s-2]*w0 + bx[s-1]*w1) + bx[s]*w2)), fp32 math.
__device__ __forceinline__ float conv3(float b0, float b1, float b2, const __half* w, int c) {
    float w0 = __half2float(w[c * 3 + 0]), w1 = __half2float(w[c * 3 + 1]),
          w2 = __half2float(w[c * 3 + 2]);
    return b0 * w0 + b1 * w1 + b2 * w2;
}

__global__ void k_conv_apply(const __half* __restrict__ Bx, const __half* __restrict__ C,
                             const __half* __restrict__ w, const __half* __restrict__ state,
                             __half* y, int S, int H) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= S * H) return;
    int s = i / H, c = i % H;
    float b[3];
#pragma unroll
    for (int j = 0; j < 3; j++) {
        int ss = s - 2 + j;
        b[j] = ss >= 0 ? __half2float(Bx[(size_t)ss * H + c]) : __half2float(state[(ss + 2) * H + c]);
    }
    y[i] = __float2half_rn(__half2float(C[i]) * conv3(b[0], b[1], b[2], w, c));
}

__global__ void k_conv_update_state(const __half* __restrict__ Bx, __half* state, int S, int H) {
    int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= H) return;
    if (S == 1) {
        state[c] = state[H + c];
        state[H + c] = Bx[c];
    } else {
        state[c] = Bx[(size_t)(S - 2) * H + c];
        state[H + c] = Bx[(size_t)(S - 1) * H + c];
    }
}

extern "C" int cuinf_conv_pre(const float* inproj, void* C, void* Bx, int S, int H, void* stream) {
    REQUIRE(inproj && C && Bx && S > 0 && H > 0, "bad arguments");
    int n = S * H;
    k_conv_pre<<<(n + 255) / 256, 256, 0, ST(stream)>>>(inproj, (__half*)C, (__half*)Bx, S, H);
    return cuinf_launch_status();
}
extern "C" int cuinf_conv_apply(const void* Bx, const void* C, const void* w, const void* state,
                                void* y, int S, int H, void* stream) {
    REQUIRE(Bx && C && w && state && y && S > 0 && H > 0, "bad arguments");
    int n = S * H;
    k_conv_apply<<<(n + 255) / 256, 256, 0, ST(stream)>>>((const __half*)Bx, (const __half*)C,
                                                          (const __half*)w, (const __half*)state,
                                                          (__half*)y, S, H);
    return cuinf_launch_status();
}
extern "C" int cuinf_conv_update_state(const void* Bx, void* state, int S, int H, void* stream) {
    REQUIRE(Bx && state && S > 0 && H > 0, "bad arguments");
    k_conv_update_state<<<(H + 255) / 256, 256, 0, ST(stream)>>>((const __half*)Bx, (__half*)state,
                                                                 S, H);
    return cuinf_launch_status();
}

// ---------------------------------------------------------------------------
// elementwise (engine.cu:527-559)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float silu_f(float x) { return x / (1.f + __expf(-x)); }

__global__ void k_swiglu(const float* __restrict__ g, const float* __restrict__ u, __half* out,
                         int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __float2half_rn(silu_f(g[i]) * u[i]);
}
__global__ void k_acc_scaled(__half* dst, const float* __restrict__ src, float w, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = __float2half_rn(__half2float(dst[i]) + w * src[i]);
}
__global__ void k_add_inplace(__half* a, const __half* __restrict__ b, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) a[i] = __float2half_rn(__half2float(a[i]) + __half2float(b[i]));
}
__global__ void k_add_f32_inplace(__half* a, const float* __restrict__ b, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) a[i] = __float2half_rn(__half2float(a[i]) + b[i]);
}
__global__ void k_f32_to_f16(const float* __restrict__ s, __half* d, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) d[i] = __float2half_rn(s[i]);
}
__global__ void k_embed_gather(const __half* __restrict__ embed, const int* __restrict__ ids,
                               __half* out, int S, int H) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= S * H) return;
    int s = i / H, c = i % H;
    out[i] = embed[(size_t)ids[s] * H + c];
}

#define EW_LAUNCH(n) <<<((n) + 255) / 256, 256, 0, ST(stream)>>>
extern "C" int cuinf_swiglu(const float* g, const float* u, void* out, int n, void* stream) {
    REQUIRE(g && u && out && n > 0, "bad arguments");
    k_swiglu EW_LAUNCH(n)(g, u, (__half*)out, n);
    return cuinf_launch_status();
}
extern "C" int cuinf_acc_scaled(void* dst, const float* src, float w, int n, void* stream) {
    REQUIRE(dst && src && n > 0, "bad arguments");
    k_acc_scaled EW_LAUNCH(n)((__half*)dst, src, w, n);
    return cuinf_launch_status();
}
extern "C" int cuinf_add_inplace(void* a, const void* b, int n, void* stream) {
    REQUIRE(a && b && n > 0, "bad arguments");
    k_add_inplace EW_LAUNCH(n)((__half*)a, (const __half*)b, n);
    return cuinf_launch_status();
}
extern "C" int cuinf_add_f32_inplace(void* a, const float* b, int n, void* stream) {
    REQUIRE(a && b && n > 0, "bad arguments");
    k_add_f32_inplace EW_LAUNCH(n)((__half*)a, b, n);
    return cuinf_launch_status();
}
extern "C" int cuinf_f32_to_f16(const float* src, void* dst, int n, void* stream) {
    REQUIRE(src && dst && n > 0, "bad arguments");
    k_f32_to_f16 EW_LAUNCH(n)(src, (__half*)dst, n);
    return cuinf_launch_status();
}
extern "C" int cuinf_embed_gather(const void* embed, const int* ids, void* out, int S, int H,
                                  void* stream) {
    REQUIRE(embed && ids && out && S > 0 && H > 0, "bad arguments");
    k_embed_gather EW_LAUNCH(S * H)((const __half*)embed, ids, (__half*)out, S, H);
    return cuinf_launch_status();
}

// ---------------------------------------------------------------------------
// argmax (argmax_kernel, engine.cu:562-572): one CTA of 1024 threads, 64-bit
// keys that encode the reference's tie rule.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) k_argmax(const float* __restrict__ v, int n, int* out) {
    __shared__ unsigned long long red[32];
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float x = v[i];
        if (x > -1e30f) best = umax64_dev(best, argmax_key(x == 0.f ? 0.f : x, i));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = umax64_dev(best, __shfl_xor_sync(0xffffffffu, best, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long b = 0ull;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) b = umax64_dev(b, red[i]);
        *out = b ? argmax_key_index(b) : 0;
    }
}

extern "C" int cuinf_argmax(const float* logits, int n, int* out, void* stream) {
    REQUIRE(logits && out && n > 0, "bad arguments");
    k_argmax<<<1, 1024, 0, ST(stream)>>>(logits, n, out);
    return cuinf_launch_status();
}

// ---------------------------------------------------------------------------
// MoE routing on the device (host loop of engine.cu:883-892)
// ---------------------------------------------------------------------------
__global__ void k_moe_route(const float* __restrict__ logits, const __half* __restrict__ bias,
                            int n_exp, int topk, int* idx, float* w) {
    const int s = blockIdx.x;
    route_select_warp(logits + (size_t)s * n_exp, bias, n_exp, topk, idx + (size_t)s * topk,
                      w + (size_t)s * topk);
}

extern "C" int cuinf_moe_route(const float* logits, const void* bias, int S, int n_exp, int topk,
                               int* idx, float* w, void* stream) {
    REQUIRE(logits && bias && idx && w, "null pointer");
    REQUIRE(S > 0 && n_exp > 0 && n_exp <= 256 && topk > 0 && topk <= 16 && topk <= n_exp,
            "n_exp <= 256, 0 < topk <= min(16, n_exp)");
    k_moe_route<<<S, 32, 0, ST(stream)>>>(logits, (const __half*)bias, n_exp, topk, idx, w);
    return cuinf_launch_status();
}

// ---------------------------------------------------------------------------
// INT4 quantizer (tools/export_weights.py:64-79), bit-exact.
// One warp per (row, group): 128 values, 4 per lane.
// ---------------------------------------------------------------------------
__global__ void k_quantize_int4(const float* __restrict__ w, long long N, long long K,
                                uint8_t* packed, __half* scales) {
    const long long KG = K / 128;
    long long item = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= N * KG) return;
    const int lane = threadIdx.x & 31;
    long long n = item / KG, g = item % KG;
    const float* src = w + n * K + g * 128 + lane * 4;
    float4 v = *reinterpret_cast<const float4*>(src);
    float a = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    a = warp_max(a);
    float scale = __fdiv_rn(a, 7.0f);
    float safe = scale == 0.f ? 1.0f : scale;
    float q[4] = {v.x, v.y, v.z, v.w};
    uint32_t nib[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float t = rintf(__fdiv_rn(q[i], safe));
        t = fminf(fmaxf(t, -7.0f), 7.0f);
        nib[i] = (uint32_t)((int)t + 8);
    }
    uint8_t* dst = packed + n * (K / 2) + g * 64 + lane * 2;
    dst[0] = (uint8_t)(nib[0] | (nib[1] << 4));
    dst[1] = (uint8_t)(nib[2] | (nib[3] << 4));
    if (lane == 0) scales[n * KG + g] = __float2half_rn(scale);
}

extern "C" int cuinf_quantize_int4(const float* w, int64_t N, int64_t K, uint8_t* packed,
                                   void* scales, void* stream) {
    REQUIRE(w && packed && scales, "null pointer");
    REQUIRE(N > 0 && K > 0 && K % 128 == 0, "K must be a positive multiple of 128");
    REQUIRE(((uintptr_t)w & 15) == 0, "w must be 16-byte aligned");
    long long items = (long long)N * (K / 128);
    long long blocks = (items + 7) / 8;
    REQUIRE(blocks < (1ll << 31), "tensor too large");
    k_quantize_int4<<<(unsigned)blocks, 256, 0, ST(stream)>>>(w, N, K, packed, (__half*)scales);
    return cuinf_launch_status();
}

extern "C" int cuinf_quantize_int4_host(const float* w, int64_t N, int64_t K, uint8_t* packed,
                                        uint16_t* scales) {
    REQUIRE(w && packed && scales, "null pointer");
    REQUIRE(N > 0 && K > 0 && K % 128 == 0, "K must be a positive multiple of 128");
    for (int64_t n = 0; n < N; n++)
        for (int64_t g = 0; g < K / 128; g++) {
            const float* src = w + n * K + g * 128;
            float a = 0.f;
            for (int i = 0; i < 128; i++) a = fmaxf(a, fabsf(src[i]));
            volatile float scale = a / 7.0f;
            float safe = scale == 0.f ? 1.0f : scale;
            __half hs = __float2half_rn(scale);
            memcpy(&scales[n * (K / 128) + g], &hs, 2);
            for (int i = 0; i < 128; i += 2) {
                volatile float r0 = src[i] / safe, r1 = src[i + 1] / safe;
                float q0 = fminf(fmaxf(rintf(r0), -7.f), 7.f);
                float q1 = fminf(fmaxf(rintf(r1), -7.f), 7.f);
                packed[n * (K / 2) + (g * 128 + i) / 2] =
                    (uint8_t)(((int)q0 + 8) | (((int)q1 + 8) << 4));
            }
        }
    return CUINF_OK;
}
