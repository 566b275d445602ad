// Tensor-core GEMMs (tcgen05) for batched decode and prefill: the INT4
// dequant-GEMM and the fp16 lm_head GEMM with a fused argmax, their 2-D TMA
// tensor maps and split-K plans.
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "tc_gemm.cuh"

int cuinf_set_cuda_error(cudaError_t e);
int cuinf_set_arg_error(const char* what);
int cuinf_launch_status();
#define ST(s) ((cudaStream_t)(s))
#define REQUIRE(cond, msg) \
    do {                   \
        if (!(cond)) return cuinf_set_arg_error(msg); \
    } while (0)

// Device error word of the tensor-core kernels (bit 1: a bounded pipeline
// wait timed out).
static __device__ unsigned g_tc_err;

unsigned cuinf_tc_error_word() {
    unsigned v = 0;
    cudaMemcpyFromSymbol(&v, g_tc_err, sizeof(v));
    return v;
}

// ---------------------------------------------------------------------------
// tensor maps (driver entry point, so the library links only the runtime)
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    });
    return fn;
}

// 2-D map over a row-major matrix [outer][inner] of `esize`-byte elements.
static int tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, uint64_t inner,
                   uint64_t outer, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw,
                   CUtensorMapL2promotion l2) {
    EncodeTiledFn fn = encode_fn();
    REQUIRE(fn, "cuTensorMapEncodeTiled unavailable");
    REQUIRE(((uintptr_t)base & 15) == 0, "tensor base must be 16-byte aligned");
    REQUIRE((inner * esize) % 16 == 0, "row pitch must be a multiple of 16 bytes");
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {inner * esize};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, l2,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    REQUIRE(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed");
    return CUINF_OK;
}

// packed INT4 [N][K/2] bytes: box 64 bytes (128 K) x 128 rows, 64-byte swizzle
int tc_map_int4(CUtensorMap* m, const uint8_t* packed, int N, int K) {
    return tmap_2d(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, packed, (uint64_t)K / 2, N, TC_KS / 2, TC_ROWS,
                   CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
}
// fp16 weights [N][K]: box 64 x 128 rows, 128-byte swizzle (the A operand)
int tc_map_f16w(CUtensorMap* m, const __half* W, int N, int K) {
    return tmap_2d(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, W, K, N, 64, TC_ROWS, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
}
// fp16 activations [rows][K]: box 64 x 16 rows, 128-byte swizzle (the B operand)
int tc_map_act(CUtensorMap* m, const __half* x, int rows, int K) {
    return tmap_2d(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, x, K, rows, 64, 16, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
}

// Split-K plan: enough CTAs to cover the SMs once, each split holding at
// most TC_MAX_KG scale groups.
struct TcPlan {
    int splits, kgps;
};
TcPlan tc_plan(int ctas_without_split, int K, int num_sms) {
    const int KG = K / TC_KS;
    int want = std::max(1, num_sms / std::max(1, ctas_without_split));
    want = std::max(want, (KG + TC_MAX_KG - 1) / TC_MAX_KG);
    want = std::min(want, KG);
    int kgps = (KG + want - 1) / want;
    kgps = std::min(kgps, TC_MAX_KG);
    return {(KG + kgps - 1) / kgps, kgps};
}

static int tc_attr_once() {
    static cudaError_t e = cudaFuncSetAttribute(k_tc_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                (int)TC_SMEM_BYTES);
    if (e != cudaSuccess) return cuinf_set_cuda_error(e);
    return CUINF_OK;
}

int tc_launch(const CUtensorMap& xmap, const CUtensorMap& wmap, TcParams P, int tiles, cudaStream_t st,
              bool pdl) {
    int rc = tc_attr_once();
    if (rc) return rc;
    unsigned* err = nullptr;
    CUINF_TRY(cudaGetSymbolAddress((void**)&err, g_tc_err));
    P.err = err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles, P.splits, P.n_groups);
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = TC_SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    CUINF_TRY(cudaLaunchKernelEx(&cfg, k_tc_gemm, xmap, wmap, P));
    return CUINF_OK;
}

// Library-owned split-K workspace of the standalone operators (grown on
// demand, never inside a graph capture; calls on a device must not overlap).
static float* g_tc_ws = nullptr;
static unsigned* g_tc_cnt = nullptr;
static size_t g_tc_ws_slots = 0, g_tc_cnt_n = 0;
static std::mutex g_tc_mu;

static int tc_workspace(size_t slots, size_t counters, float** ws, unsigned** cnt) {
    std::lock_guard<std::mutex> lk(g_tc_mu);
    if (slots > g_tc_ws_slots) {
        if (g_tc_ws) cudaFree(g_tc_ws);
        g_tc_ws = nullptr;
        CUINF_TRY(cudaMalloc(&g_tc_ws, slots * TC_NMAX * TC_ROWS * sizeof(float)));
        g_tc_ws_slots = slots;
    }
    if (counters > g_tc_cnt_n) {
        if (g_tc_cnt) cudaFree(g_tc_cnt);
        g_tc_cnt = nullptr;
        CUINF_TRY(cudaMalloc(&g_tc_cnt, counters * sizeof(unsigned)));
        CUINF_TRY(cudaMemset(g_tc_cnt, 0, counters * sizeof(unsigned)));
        g_tc_cnt_n = counters;
    }
    *ws = g_tc_ws;
    *cnt = g_tc_cnt;
    return CUINF_OK;
}

static int num_sms_now() {
    int dev = 0, n = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

// One standalone launch per 128 activation rows.
static int tc_gemm_op(const void* x, const void* w, const void* scales, float* y, int M, int N, int K,
                      unsigned long long* amax, bool fp16_w, void* stream) {
    REQUIRE(x && w && (y || amax), "null pointer");
    REQUIRE(M > 0 && N > 0 && K > 0, "M, N, K must be positive");
    REQUIRE(K % TC_KS == 0, "K must be a multiple of 128");
    REQUIRE(fp16_w || scales, "null scales");
    CUtensorMap xm, wm;
    int rc = tc_map_act(&xm, (const __half*)x, M, K);
    if (rc) return rc;
    rc = fp16_w ? tc_map_f16w(&wm, (const __half*)w, N, K) : tc_map_int4(&wm, (const uint8_t*)w, N, K);
    if (rc) return rc;
    const int tiles = (N + TC_ROWS - 1) / TC_ROWS;
    TcPlan pl = amax ? TcPlan{1, K / TC_KS} : tc_plan(tiles, K, num_sms_now());
    REQUIRE(pl.kgps <= TC_MAX_KG || fp16_w, "K too large for one split");
    float* ws = nullptr;
    unsigned* cnt = nullptr;
    if (pl.splits > 1) {
        rc = tc_workspace((size_t)tiles * pl.splits, tiles, &ws, &cnt);
        if (rc) return rc;
    }
    for (int m0 = 0; m0 < M; m0 += TC_NMAX) {
        TcParams P = {};
        P.groups = nullptr;
        P.g0.wmap = nullptr;
        P.g0.scales = (const __half*)scales;
        P.g0.y = y ? y + (size_t)m0 * N : nullptr;
        P.g0.x_row = m0;
        P.g0.rows = std::min(TC_NMAX, M - m0);
        P.g0.N = N;
        P.g0.ldy = N;
        P.n_groups = 1;
        P.K = K;
        P.splits = pl.splits;
        P.kg_per_split = pl.kgps;
        P.fp16_w = fp16_w;
        P.ws = ws;
        P.counters = cnt;
        P.amax = amax;
        rc = tc_launch(xm, wm, P, tiles, ST(stream), false);
        if (rc) return rc;
    }
    return cuinf_launch_status();
}

extern "C" int cuinf_gemm_int4_tc(const void* x, const uint8_t* packed, const void* scales, float* y, int M, int N,
                                  int K, void* stream) {
    REQUIRE(((uintptr_t)packed & 15) == 0, "packed must be 16-byte aligned");
    return tc_gemm_op(x, packed, scales, y, M, N, K, nullptr, false, stream);
}

extern "C" int cuinf_gemm_fp16_tc(const void* x, const void* W, float* y, int M, int N, int K,
                                  unsigned long long* argmax_keys, void* stream) {
    return tc_gemm_op(x, W, nullptr, y, M, N, K, argmax_keys, true, stream);
}

extern "C" int cuinf_argmax_key_index(unsigned long long key) {
    const uint32_t tie = 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFu);
    uint32_t r = tie >> 23, b = 0;
    for (int i = 0; i < 8; i++) b |= ((r >> i) & 1u) << (7 - i);
    return (int)(((tie & 0x7FFFFFu) << 8) | b);
}
