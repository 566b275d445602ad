// Tensor-core GEMMs (tcgen05) for batched decode and prefill: the INT4
// dequant-GEMM and the fp16 lm_head GEMM with a fused argmax, their 2-D TMA
// tensor maps and split-K plans.
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
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
static __device__ unsigned g_tc_err[4];

#ifdef TC_TRACE
extern "C" int cuinf_tc_trace_read(unsigned long long* out) {
    return cudaMemcpyFromSymbol(out, g_tc_trace, sizeof(g_tc_trace)) == cudaSuccess ? 0 : 1;
}
#endif

unsigned cuinf_tc_error_word() {
    unsigned v[4] = {0, 0, 0, 0};
    cudaMemcpyFromSymbol(v, g_tc_err, sizeof(v));
    return v[0];
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
// fp16 activations [rows][K]: box 64 x box_rows (16..128, a multiple of 16),
// 128-byte swizzle (the B operand)
int tc_map_act(CUtensorMap* m, const __half* x, int rows, int K, int box_rows) {
    return tmap_2d(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, x, K, rows, 64, box_rows, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
}
// fp16 weights [N][K]: box 64 x 128 rows, 128-byte swizzle (the A operand)
int tc_map_f16w(CUtensorMap* m, const __half* W, int N, int K) {
    return tmap_2d(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, W, K, N, 64, TC_ROWS, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
}

// Split-K plan: up to TC_SPLITS_MAX splits towards covering the SMs once,
// each split holding at most TC_MAX_KG scale groups.  Every split adds a
// partial write and a share of the last CTA's ordered reduction: for the
// batched-decode projections (64 rows, 16-48 tiles) a cap of 4 measured
// 4.32 -> 4.21 ms per 64-sequence step against filling all SMs (a cap of 2:
// 4.23).
#define TC_SPLITS_MAX 4
struct TcPlan {
    int splits, kgps;
};
TcPlan tc_plan(int ctas_without_split, int K, int num_sms) {
    const int KG = K / TC_KS;
    int want = std::max(1, std::min(TC_SPLITS_MAX, num_sms / std::max(1, ctas_without_split)));
    want = std::max(want, (KG + TC_MAX_KG - 1) / TC_MAX_KG);
    want = std::min(want, KG);
    int kgps = (KG + want - 1) / want;
    kgps = std::min(kgps, TC_MAX_KG);
    return {(KG + kgps - 1) / kgps, kgps};
}

// Kernel attribute and error-word address, set up once per process outside
// any graph capture.
static unsigned* g_tc_err_ptr = nullptr;
static int tc_attr_once() {
    static cudaError_t e = [] {
        cudaError_t r = cudaFuncSetAttribute(k_tc_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)TC_SMEM_BYTES);
        if (r == cudaSuccess) r = cudaGetSymbolAddress((void**)&g_tc_err_ptr, g_tc_err);
        return r;
    }();
    if (e != cudaSuccess) return cuinf_set_cuda_error(e);
    return CUINF_OK;
}

int tc_launch(const CUtensorMap& xmap, const CUtensorMap& wmap, TcParams P, int tiles, cudaStream_t st,
              bool pdl) {
    int rc = tc_attr_once();
    if (rc) return rc;
    P.err = g_tc_err_ptr;
    P.tiles = tiles;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long items = (long long)P.n_groups * tiles * P.splits;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::min<long long>(items, sms));  // persistent: one CTA per SM at most
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

// One standalone launch: every 128 activation rows form a group of items.
static int tc_gemm_op(const void* x, const void* w, const void* scales, float* y, int M, int N, int K,
                      unsigned long long* amax, bool fp16_w, void* stream) {
    REQUIRE(x && w && (y || amax), "null pointer");
    REQUIRE(M > 0 && N > 0 && K > 0, "M, N, K must be positive");
    REQUIRE(K % TC_KS == 0, "K must be a multiple of 128");
    REQUIRE(fp16_w || scales, "null scales");
    CUtensorMap xm, wm;
    const int xmax = (std::min(M, TC_NMAX) + 15) & ~15;  // one box covers a launch's rows
    int rc = tc_map_act(&xm, (const __half*)x, M, K, xmax);
    if (rc) return rc;
    rc = fp16_w ? tc_map_f16w(&wm, (const __half*)w, N, K) : tc_map_int4(&wm, (const uint8_t*)w, N, K);
    if (rc) return rc;
    const int tiles = (N + TC_ROWS - 1) / TC_ROWS, ng = (M + TC_NMAX - 1) / TC_NMAX;
    TcPlan pl = amax ? TcPlan{1, K / TC_KS} : tc_plan(tiles * ng, K, num_sms_now());
    REQUIRE(pl.kgps <= TC_MAX_KG || fp16_w, "K too large for one split");
    float* ws = nullptr;
    unsigned* cnt = nullptr;
    if (pl.splits > 1) {
        rc = tc_workspace((size_t)ng * tiles * pl.splits, (size_t)ng * tiles, &ws, &cnt);
        if (rc) return rc;
    }
    TcParams P = {};
    P.groups = nullptr;
    P.g0.wmap = nullptr;
    P.g0.scales = (const __half*)scales;
    P.g0.y = y;
    P.g0.x_row = 0;
    P.g0.rows = std::min(TC_NMAX, M);
    P.g0.N = N;
    P.g0.ldy = N;
    P.n_groups = ng;
    P.m_rows = M;
    P.K = K;
    P.splits = pl.splits;
    P.kg_per_split = pl.kgps;
    P.fp16_w = fp16_w;
    P.xmax = xmax;
    P.xbox = xmax;
    P.ws = ws;
    P.counters = cnt;
    P.amax = amax;
    rc = tc_launch(xm, wm, P, tiles, ST(stream), false);
    if (rc) return rc;
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

// ===========================================================================
// Sequence-batched decode engine: B independent sequences advance one token
// per step.  Per layer the B tokens go through the same operators as the
// reference's layer_forward(1) for each sequence (engine.cu:784-908), with
// every projection on the tensor-core GEMM above, attention batched over the
// sequences' own FP8 caches, and the MoE experts grouped: a device-side
// counting sort assigns each (token, slot) a row of its expert's group, one
// grouped GEMM runs w1/w3 of all experts, one runs w2, and a combine kernel
// applies the reference's per-token slot order (acc_scaled then add_inplace,
// engine.cu:894-904).  The step is one CUDA graph.
// ===========================================================================
#include <nccl.h>

#include <chrono>
#include <string>
#include <thread>

#include "model.h"
#include "route.cuh"

// Peer-memory exchange of the expert-parallel batch (kernels below).
#define EP_MAX_WORLD 8
struct EpLinks {
    char* base[EP_MAX_WORLD];  // every rank's exchange arena as mapped in this process (own included)
    size_t off_x, off_meta, off_back, off_flag;
    int rank, world, cap, H;
};
struct EpWait {
    const unsigned long long* flags;  // this rank's flags row ([0] dispatch or [1] return); null: no wait
    const unsigned long long* step;   // the device step counter
    int world, tag;                   // tag: 2 * MoE layer + direction
    unsigned* err;                    // bit 4 (16): a peer's flag did not come within the wait limit
};
struct cuinf_batch {
    cuinf_model* m = nullptr;
    int B = 0, max_ctx = 0, num_sms = 148;
    cudaStream_t st = nullptr;
    bool own_stream = false;
    std::vector<void*> allocs;
    // per-sequence state
    int *tok = nullptr, *pos = nullptr, *pinned = nullptr;
    std::vector<AttnState> attn;
    std::vector<__half*> conv_state;
    size_t kv8_seq = 0, sc_seq = 0, tail_seq = 0;
    // activations
    __half *h = nullptr, *xn = nullptr, *qkv16 = nullptr, *attn_out = nullptr, *conv_y = nullptr,
           *dmid = nullptr, *xg = nullptr, *mmid = nullptr;
    float *fqkv = nullptr, *fa = nullptr, *fb = nullptr, *fg = nullptr, *fu = nullptr, *fo = nullptr,
          *rlog = nullptr, *logits = nullptr;
    int *ridx = nullptr, *inv = nullptr, *src = nullptr;
    float* rw = nullptr;
    unsigned long long* amax = nullptr;
    float* apart = nullptr;
    unsigned* acnt = nullptr;
    int nsplit = 1;
    // tensor-core GEMM state
    std::vector<CUtensorMap> hmaps;  // weights (host copies)
    CUtensorMap* dmaps = nullptr;    // same, device
    TcGroup* dstatic = nullptr;      // q/k/v and dense w1/w3 group tables
    std::vector<int> qkv_tab, d13_tab;
    CUtensorMap x_h, x_conv, x_attn, x_dmid, x_xg, x_mmid;  // activation maps
    TcGroup *g13 = nullptr, *g2 = nullptr;  // MoE group tables, rewritten per layer
    std::vector<int> mi_in, mi_out, mi_q, mi_k, mi_v, mi_o, mi_w1, mi_w3, mi_w2;
    std::vector<int> mi_experts;  // per MoE layer: index of expert 0's w1 map (then w3, w2, next expert)
    int mi_embed = -1;
    float* ws = nullptr;
    unsigned* cnt = nullptr;
    size_t ws_slots = 0, cnt_n = 0;
    bool keep_logits = false;
    int kernels = 0;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    // expert parallelism: this rank hosts experts [e_lo, e_lo + e_loc) and
    // exchanges (token, slot) rows with the other ranks through NCCL
    int ep_rank = 0, ep_world = 1, e_lo = 0, e_loc = 0, cap = 0;
    ncclComm_t comm = nullptr;
    int ep_timeout_ms = 120000;  // host-side limit on a step's (and the setup's) collectives
    bool ep_failed = false;      // the communicator was aborted: the batch takes no more steps
    __half *send_x = nullptr, *recv_x = nullptr;
    int *send_meta = nullptr, *recv_meta = nullptr, *dest_pos = nullptr;
    float *back_o = nullptr, *recv_back = nullptr;
    // peer-memory exchange (the default when every peer's arena maps here;
    // otherwise the rows travel by NCCL send/recv through the buffers above)
    bool p2p = false, p2p_ok = false;
    EpLinks links = {};
    std::vector<void*> peer_open;         // the peers' arenas opened in this process
    unsigned long long* ep_step = nullptr;  // device step counter of the flag values
    unsigned* ep_ticket = nullptr;          // [2] tickets of the sending kernels
    // vocabulary-sharded lm_head (expert-parallel form, logits not kept): this
    // rank multiplies every rank's final rows by vocabulary rows
    // [rank*V/world, (rank+1)*V/world); the argmax keys are max-reduced
    __half* xall = nullptr;            // [world*B][H] final normed rows of all ranks
    unsigned long long* kall = nullptr;  // [world*B] argmax keys
    CUtensorMap x_all;
    int mi_embed_shard = -1;
    bool vocab_shard = false;
};

template <class T>
static int balloc(cuinf_batch* b, T** p, size_t bytes) {
    void* d = nullptr;
    CUINF_TRY(cudaMalloc(&d, bytes < 256 ? 256 : bytes));
    CUINF_TRY(cudaMemset(d, 0, bytes < 256 ? 256 : bytes));
    b->allocs.push_back(d);
    *p = (T*)d;
    return CUINF_OK;
}

// ---------------------------------------------------------------------------
// batched kernels
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint8_t bf32_to_e4m3(float x) {
    return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}
// kv_commit_group for one head of one sequence (engine.cu:202-228): scale =
// absmax/448 + 1e-12 in fp32, stored as fp16; codes = e4m3(x / scale_f32).
__device__ void bkv_commit_head(const __half* tail, uint8_t* c8, __half* sc, int h, int nkv, int grp, float* red) {
    float mx = 0.f;
    for (int e = threadIdx.x; e < CUINF_KVGROUP * CUINF_HD; e += blockDim.x) {
        const int t = e >> 6, d = e & 63;
        mx = fmaxf(mx, fabsf(__half2float(tail[((size_t)t * nkv + h) * CUINF_HD + d])));
    }
    mx = warp_max(mx);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    float amax = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) amax = fmaxf(amax, red[i]);
    const float s = amax / 448.0f + 1e-12f;
    if (threadIdx.x == 0) sc[grp * nkv + h] = __float2half_rn(s);
    for (int e = threadIdx.x; e < CUINF_KVGROUP * CUINF_HD; e += blockDim.x) {
        const int t = e >> 6, d = e & 63;
        const float v = __half2float(tail[((size_t)t * nkv + h) * CUINF_HD + d]);
        c8[((size_t)(grp * CUINF_KVGROUP + t) * nkv + h) * CUINF_HD + d] = bf32_to_e4m3(v / s);
    }
}

// Placement of each sequence's new K/V row (engine.cu:831-845 with S = 1):
// tail slot pos % 64; a full tail is committed as FP8 group pos / 64.
// grid (B, nkv), 256 threads.
__global__ void __launch_bounds__(256) k_bkv_place(const __half* __restrict__ k16, const __half* __restrict__ v16,
                                                   const int* __restrict__ pos, __half* ktail, __half* vtail,
                                                   uint8_t* kc8, uint8_t* vc8, __half* ksc, __half* vsc, int nkv,
                                                   size_t tail_seq, size_t kv8_seq, size_t sc_seq) {
    __shared__ float red[8];
    const int b = blockIdx.x, h = blockIdx.y, p = pos[b], slot = p & (CUINF_KVGROUP - 1);
    __half* kt = ktail + b * tail_seq;
    __half* vt = vtail + b * tail_seq;
    if (threadIdx.x < CUINF_HD) {
        const size_t src = ((size_t)b * nkv + h) * CUINF_HD + threadIdx.x;
        const size_t dst = ((size_t)slot * nkv + h) * CUINF_HD + threadIdx.x;
        kt[dst] = k16[src];
        vt[dst] = v16[src];
    }
    if (slot != CUINF_KVGROUP - 1) return;
    __syncthreads();
    bkv_commit_head(kt, kc8 + b * kv8_seq, ksc + b * sc_seq, h, nkv, p / CUINF_KVGROUP, red);
    __syncthreads();
    bkv_commit_head(vt, vc8 + b * kv8_seq, vsc + b * sc_seq, h, nkv, p / CUINF_KVGROUP, red);
}

// Short conv of one token per sequence (conv_pre / conv_apply /
// conv_update_state with S = 1, engine.cu:483-525): z = in_proj output
// [B][3H] in the order B | C | x.
__global__ void k_bconv(const float* __restrict__ z, const __half* __restrict__ w, __half* state, __half* y, int B,
                        int H) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * H) return;
    const int b = i / H, c = i - b * H;
    const float* row = z + (size_t)b * 3 * H;
    const __half Cx = __float2half_rn(row[H + c]);
    const __half Bx = __float2half_rn(row[c] * row[2 * H + c]);
    __half* sb = state + (size_t)b * 2 * H;
    const float b0 = __half2float(sb[c]), b1 = __half2float(sb[H + c]), b2 = __half2float(Bx);
    const float w0 = __half2float(w[c * 3 + 0]), w1 = __half2float(w[c * 3 + 1]), w2 = __half2float(w[c * 3 + 2]);
    y[i] = __float2half_rn(__half2float(Cx) * (b0 * w0 + b1 * w1 + b2 * w2));
    sb[c] = sb[H + c];
    sb[H + c] = Bx;
}

// ---------------------------------------------------------------------------
// Expert-parallel exchange through peer memory.  Every rank exports one
// "exchange arena" (cudaIpc) that the others map:
//   rx_x    [world][cap][H] fp16   rows sent to this rank, segment p from rank p
//   rx_meta [world][cap]    int    their local expert index (-1: unused slot)
//   rx_back [world][cap][H] fp32   expert outputs returned to this rank, segment d from rank d
//   flags   [2][world]      u64    arrival flags: [0][p] rows from p, [1][d] outputs from d
// A sender writes its rows straight into the receivers' arenas over NVLink
// (plain stores, no bulk copies), fences, and the last of its CTAs (atomic
// ticket) raises its flag in every receiver with a system-scope release
// store.  The receiver's next kernel waits (bounded) for every peer's flag
// with acquire loads.  Flag values grow monotonically: (step << 8) + 2 *
// (MoE layer) + 1 (+1 for returns), the step counter advanced on the device
// at the start of every step.  One buffer per direction suffices: a rank can
// send layer L+1's rows only after it has every peer's outputs of layer L,
// which each peer returns only after it has consumed layer L's rows (and
// read its metadata); likewise for the returned outputs.
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned long long ep_flag_value(unsigned long long step, int tag) {
    return (step << 8) + (unsigned long long)tag + 1ull;
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}
// One thread: wait until every peer's flag reached this step's value, at
// most CUINF_WAIT_LIMIT_NS in total; on time-out set the error bit and return
// (the kernel then runs on stale rows; the host reports the error).
__device__ void ep_wait_flags(const EpWait& W) {
    if (*(volatile unsigned*)W.err & 16u) return;  // an earlier wait gave up: do not wait again
    const unsigned long long want = ep_flag_value(*W.step, W.tag);
    const unsigned long long t0 = globaltimer_ns();
    for (int p = 0; p < W.world; p++) {
        while (ld_acquire_sys_u64(W.flags + p) < want) {
            if (globaltimer_ns() - t0 > CUINF_WAIT_LIMIT_NS) {
                atomicOr(W.err, 16u);
                return;
            }
            __nanosleep(32);
        }
    }
}
// Every CTA of a sending kernel ends here: fence its stores, take a ticket;
// the last CTA raises this rank's flag (row `dir`) in every rank's arena.
__device__ void ep_send_done(const EpLinks& L, unsigned* ticket, const unsigned long long* step, int tag, int dir) {
    __shared__ bool last;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    if (threadIdx.x == 0) {
        __threadfence_system();
        const unsigned long long v = ep_flag_value(*step, tag);
        for (int d = 0; d < L.world; d++)
            st_release_sys_u64(reinterpret_cast<unsigned long long*>(L.base[d] + L.off_flag) + dir * L.world + L.rank,
                               v);
        *ticket = 0u;  // the next sending kernel starts after this one ends (stream order)
    }
}
// Dispatch of this rank's (token, slot) entries (n = B * topk): entry j goes
// to rank d = expert / e_loc at position rank-of-j among the entries for d
// (the plan of cuinf_ep_plan_host); its row xn[j / topk] and the expert's
// local index are written into d's arena at segment `rank`.  CTAs n..n+world-1
// mark the unused slots of each receiver's segment with -1.
// grid n + world, 256 threads.
__global__ void __launch_bounds__(256) k_ep_send(EpLinks L, const int* __restrict__ ridx, int n, int e_loc,
                                                 const __half* __restrict__ xn, int topk, int* dest_pos,
                                                 unsigned* ticket, const unsigned long long* step, int tag) {
    __shared__ int s_cnt;
    if (threadIdx.x == 0) s_cnt = 0;
    __syncthreads();
    const bool entry = (int)blockIdx.x < n;
    const int d = entry ? ridx[blockIdx.x] / e_loc : (int)blockIdx.x - n;
    const int lim = entry ? (int)blockIdx.x : n;  // count the entries for d before j (or all of them)
    int c = 0;
    for (int i = threadIdx.x; i < lim; i += blockDim.x) c += ridx[i] / e_loc == d;
    if (c) atomicAdd(&s_cnt, c);
    __syncthreads();
    const int pos = s_cnt;
    int* meta = reinterpret_cast<int*>(L.base[d] + L.off_meta) + (size_t)L.rank * L.cap;
    if (entry) {
        const int j = blockIdx.x;
        if (threadIdx.x == 0) {
            dest_pos[j] = d * L.cap + pos;
            meta[pos] = ridx[j] - d * e_loc;
        }
        const uint4* s = reinterpret_cast<const uint4*>(xn + (size_t)(j / topk) * L.H);
        uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(L.base[d] + L.off_x) +
                                            ((size_t)L.rank * L.cap + pos) * L.H);
        for (int i = threadIdx.x; i < L.H / 8; i += blockDim.x) o[i] = s[i];
    } else {
        for (int i = pos + threadIdx.x; i < L.cap; i += blockDim.x) meta[i] = -1;
    }
    ep_send_done(L, ticket, step, tag, 0);
}
// Return of the expert outputs: slot i of this rank's received rows (from
// rank p = i / cap, its position i % cap) goes back to p's arena at segment
// `rank`, same position.  grid world * cap, 256 threads.
__global__ void __launch_bounds__(256) k_ep_send_back(EpLinks L, const float* __restrict__ fo,
                                                      const int* __restrict__ inv, unsigned* ticket,
                                                      const unsigned long long* step, int tag) {
    const int i = blockIdx.x, p = i / L.cap, pos = i - p * L.cap;
    const int r = inv[i];
    if (r >= 0) {
        const float4* s = reinterpret_cast<const float4*>(fo + (size_t)r * L.H);
        float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(L.base[p] + L.off_back) +
                                              ((size_t)L.rank * L.cap + pos) * L.H);
        for (int k = threadIdx.x; k < L.H / 4; k += blockDim.x) o[k] = s[k];
    }
    ep_send_done(L, ticket, step, tag, 1);
}
__global__ void k_ep_tick(unsigned long long* step) { *step += 1ull; }

// MoE routing of B tokens (engine.cu:883-892, one warp per token) and the
// expert grouping: rows of the gathered activation buffer are ordered by
// expert, then by token; each expert's rows form up to maxch groups of 128.
// One CTA of 1024 threads; E <= 256, B * topk <= 1024.
struct BRouteParams {
    const float* logits;  // [B][E]
    const __half* bias;
    int B, E, topk, I, H, maxch;
    int* ridx;  // [B][topk] (this layer's slice)
    float* rw;  // [B][topk]
    // grouping of n entries by key (an expert of this rank, -1 = none): with
    // keys null the entries are this batch's (token, slot) choices (n = B*topk,
    // source row = token); otherwise received rows (source row = entry)
    const int* keys;
    int n, n_local;  // entries; experts in the group tables (E, or E/world)
    int rowcap;      // rows per group (TC_NMAX for the tensor-core GEMM; the small-row GEMV takes any)
    int group;       // 0: route only
    int* inv;   // [n] row of entry (-1: none)
    int* src;   // [rows] source row of each grouped row
    TcGroup* g13;  // [2][n_local][maxch]
    TcGroup* g2;   // [n_local][maxch]
    const CUtensorMap* maps;  // [n_local][3]: w1, w3, w2
    void* const* experts;     // [n_local][6]: w1 packed, w1 scales, w3 .., w2 ..
    float *gbuf, *ubuf, *obuf;
    EpWait wait;  // expert-parallel peer exchange: the rows' arrival (flags null: none)
    int routed;   // 1: ridx / rw already hold this batch's choices (k_broute_tokens)
};
// Routing alone, one warp per token (engine.cu:883-892): many tokens (a
// prefill chunk) are routed by many CTAs instead of k_broute's 32 warps.
// grid ceil(B/8), 256 threads.
__global__ void __launch_bounds__(256) k_broute_tokens(const float* __restrict__ logits, const __half* __restrict__ bias,
                                                       int B, int E, int topk, int* ridx, float* rw) {
    const int b = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (b < B) route_select_warp(logits + (size_t)b * E, bias, E, topk, ridx + b * topk, rw + b * topk);
}
// The grouped GEMMs' tables from the per-expert row counts and offsets:
// expert ex's rows [off, off + cnt) of the gathered buffer form up to maxch
// groups of TC_NMAX rows (w1, w3 into gbuf / ubuf; w2 into obuf).
__device__ void bgroup_tables(const BRouteParams& P, const int* cnt, const int* off, int NE) {
    for (int ex = threadIdx.x; ex < NE; ex += blockDim.x) {
        for (int c = 0; c < P.maxch; c++) {
            const int cap = P.rowcap > 0 ? P.rowcap : TC_NMAX;
            const int r0 = off[ex] + c * cap;
            const int rows = max(0, min(cap, cnt[ex] - c * cap));
            const int gi = ex * P.maxch + c;
            TcGroup a;
            a.wmap = P.maps + ex * 3 + 0;
            a.packed = (const uint8_t*)P.experts[ex * 6 + 0];
            a.scales = (const __half*)P.experts[ex * 6 + 1];
            a.y = P.gbuf + (size_t)r0 * P.I;
            a.x_row = r0;
            a.rows = rows;
            a.N = P.I;
            a.ldy = P.I;
            P.g13[gi] = a;
            a.wmap = P.maps + ex * 3 + 1;
            a.packed = (const uint8_t*)P.experts[ex * 6 + 2];
            a.scales = (const __half*)P.experts[ex * 6 + 3];
            a.y = P.ubuf + (size_t)r0 * P.I;
            P.g13[NE * P.maxch + gi] = a;
            a.wmap = P.maps + ex * 3 + 2;
            a.packed = (const uint8_t*)P.experts[ex * 6 + 4];
            a.scales = (const __half*)P.experts[ex * 6 + 5];
            a.y = P.obuf + (size_t)r0 * P.H;
            a.N = P.H;
            a.ldy = P.H;
            P.g2[gi] = a;
        }
    }
}
__global__ void __launch_bounds__(1024) k_broute(const BRouteParams P) {
    __shared__ int cnt[256], off[256];
    __shared__ int wcnt[32][256];  // per warp and expert: its entries, then their offset among the warps
    if (P.wait.flags) {
        if (threadIdx.x == 0) ep_wait_flags(P.wait);
        __syncthreads();
    }
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int n = P.keys ? P.n : P.B * P.topk, NE = P.keys ? P.n_local : P.E;
    for (int i = threadIdx.x; i < 32 * NE; i += blockDim.x) wcnt[i / NE][i % NE] = 0;
    if (!P.keys && !P.routed)
        for (int b = warp; b < P.B; b += nw)
            route_select_warp(P.logits + (size_t)b * P.E, P.bias, P.E, P.topk, P.ridx + b * P.topk,
                              P.rw + b * P.topk);
    if (!P.group) return;
    __syncthreads();
    // rank of entry j among the entries of its expert that come before it:
    // the earlier lanes of its warp with the same expert (match), plus the
    // entries of that expert in the earlier warps (prefix over the warps)
    const int lane = threadIdx.x & 31;
    int e = -1;
    if (threadIdx.x < n) e = P.keys ? __ldcg(P.keys + threadIdx.x) : P.ridx[threadIdx.x];  // keys: written by peers
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    int rank = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0 && rank == 0) wcnt[warp][e] = __popc(peers);
    __syncthreads();
    for (int x = threadIdx.x; x < NE; x += blockDim.x) {
        int acc = 0;
        for (int w = 0; w < nw; w++) {
            const int v = wcnt[w][x];
            wcnt[w][x] = acc;
            acc += v;
        }
        cnt[x] = acc;
    }
    __syncthreads();
    if (e >= 0) rank += wcnt[warp][e];
    if (threadIdx.x < 32) {  // exclusive prefix over experts, one warp
        int carry = 0;
        for (int base = 0; base < NE; base += 32) {
            const int i = base + threadIdx.x;
            const int v = i < NE ? cnt[i] : 0;
            int x = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, o);
                if ((int)threadIdx.x >= o) x += y;
            }
            if (i < NE) off[i] = carry + x - v;
            carry += __shfl_sync(0xffffffffu, x, 31);
        }
    }
    __syncthreads();
    if (threadIdx.x < n) P.inv[threadIdx.x] = e >= 0 ? off[e] + rank : -1;
    if (e >= 0) P.src[off[e] + rank] = P.keys ? (int)threadIdx.x : (int)threadIdx.x / P.topk;
    bgroup_tables(P, cnt, off, NE);
}

// Grouping of n entries (any n; the prefill's (token, slot) choices, already
// routed): per-expert counts, offsets, then each entry takes the next row of
// its expert.  Rows of one expert are ordered by arrival, not by token: each
// row's products are independent of its place in the group, so the results
// are the same in any order.  One CTA of 1024 threads; E <= 256.
__global__ void __launch_bounds__(1024) k_bgroup_many(const BRouteParams P) {
    __shared__ int cnt[256], off[256], fill[256];
    const int n = P.n, NE = P.E;
    for (int e = threadIdx.x; e < NE; e += blockDim.x) cnt[e] = fill[e] = 0;
    __syncthreads();
    for (int j = threadIdx.x; j < n; j += blockDim.x) atomicAdd(&cnt[P.ridx[j]], 1);
    __syncthreads();
    if (threadIdx.x < 32) {  // exclusive prefix over experts, one warp
        int carry = 0;
        for (int base = 0; base < NE; base += 32) {
            const int i = base + threadIdx.x;
            const int v = i < NE ? cnt[i] : 0;
            int x = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, o);
                if ((int)threadIdx.x >= o) x += y;
            }
            if (i < NE) off[i] = carry + x - v;
            carry += __shfl_sync(0xffffffffu, x, 31);
        }
    }
    __syncthreads();
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        const int e = P.ridx[j], pos = off[e] + atomicAdd(&fill[e], 1);
        P.inv[j] = pos;
        P.src[pos] = j / P.topk;
    }
    bgroup_tables(P, cnt, off, NE);
}

__global__ void k_bgather(const __half* __restrict__ xn, const int* __restrict__ src, __half* xg, int H) {
    const int r = blockIdx.x;
    const uint4* s = reinterpret_cast<const uint4*>(xn + (size_t)src[r] * H);
    uint4* d = reinterpret_cast<uint4*>(xg + (size_t)r * H);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x) d[i] = s[i];
}

// h[b] += sum over slots in order: acc = half(acc + w_t * o_t) (acc_scaled),
// then h = half(h + acc) (add_inplace), engine.cu:894-904.
__global__ void k_bcombine(const float* __restrict__ obuf, const int* __restrict__ inv, const float* __restrict__ rw,
                           __half* h, int B, int H, int topk, EpWait wait) {
    if (wait.flags) {  // expert-parallel: the peers' outputs have arrived
        if (threadIdx.x == 0) ep_wait_flags(wait);
        __syncthreads();
    }
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * H) return;
    const int b = i / H, c = i - b * H;
    __half acc = __float2half_rn(0.f);
    for (int t = 0; t < topk; t++)  // (L2 loads: rows another GPU wrote during this kernel's wait)
        acc = __float2half_rn(__half2float(acc) + rw[b * topk + t] * __ldcg(obuf + (size_t)inv[b * topk + t] * H + c));
    h[i] = __float2half_rn(__half2float(h[i]) + __half2float(acc));
}

// The attention prologue after the q/k/v GEMM, one CTA of 64 threads per
// (sequence, head): fp32 -> fp16 of q, k and v; QK-RMSNorm of q and k
// (engine.cu:146-158, as cuinf_rmsnorm over 64 dims: one element per thread,
// the same block sum); RoPE of q and k at the sequence's position
// (engine.cu:161-182, as cuinf_rope).  grid (B, nh + 2*nkv): y < nh query
// heads, then key heads, then value heads (conversion only).
__global__ void __launch_bounds__(64) k_bqkv_post(const float* __restrict__ qkv, __half* q16, __half* k16, __half* v16,
                                                  const __half* __restrict__ qw, const __half* __restrict__ kw,
                                                  const int* __restrict__ pos, int nh, int nkv, float eps,
                                                  float theta) {
    __shared__ float red[2];
    __shared__ float y[CUINF_HD];
    const int b = blockIdx.x, j = blockIdx.y, d = threadIdx.x, B = gridDim.x;
    const size_t NQ = (size_t)nh * CUINF_HD, NK = (size_t)nkv * CUINF_HD;
    const float* src;
    __half* dst;
    const __half* w;
    if (j < nh) {
        src = qkv + b * NQ + (size_t)j * CUINF_HD;
        dst = q16 + b * NQ + (size_t)j * CUINF_HD;
        w = qw;
    } else if (j < nh + nkv) {
        src = qkv + B * NQ + b * NK + (size_t)(j - nh) * CUINF_HD;
        dst = k16 + b * NK + (size_t)(j - nh) * CUINF_HD;
        w = kw;
    } else {
        const size_t o = b * NK + (size_t)(j - nh - nkv) * CUINF_HD;
        v16[o + d] = __float2half_rn(qkv[B * (NQ + NK) + o + d]);
        return;
    }
    const float x = __half2float(__float2half_rn(src[d]));
    const float ss = block_sum(x * x, red);
    const float inv = rsqrtf(ss / (float)CUINF_HD + eps);
    y[d] = __half2float(__float2half_rn(x * inv * __half2float(w[d])));
    __syncthreads();
    if (d < CUINF_HD / 2) {
        float cs, sn;
        rope_pair_angle(pos[b], d, theta, cs, sn);
        const float x0 = y[d], x1 = y[d + CUINF_HD / 2];
        dst[d] = __float2half_rn(x0 * cs - x1 * sn);
        dst[d + CUINF_HD / 2] = __float2half_rn(x1 * cs + x0 * sn);
    }
}

// Residual add then the next RMSNorm, one CTA (256 threads) per sequence:
// h = half(h + f) (add_inplace, engine.cu:532-535), then xn = half(h *
// rsqrt(mean(h^2) + eps) * w) (rmsnorm, engine.cu:131-144).  Thread t takes
// elements t, t+256, ... as the separate rmsnorm kernel does (same rounding
// points and summation order); each round's loads, the norm weights
// included, are all issued first, and with H <= BRN_PER * 256 (one round)
// the normalisation uses the values still in registers.
#define BRN_PER 8
__global__ void __launch_bounds__(256) k_bres_norm(__half* h, const float* __restrict__ f,
                                                   const __half* __restrict__ w, __half* xn, int H, float eps) {
    __shared__ float red[32];
    __half* row = h + (size_t)blockIdx.x * H;
    const float* fr = f + (size_t)blockIdx.x * H;
    float ss = 0.f;
    __half hn[BRN_PER], wv[BRN_PER];
    for (int base = 0; base < H; base += BRN_PER * 256) {
        float hv[BRN_PER], fv[BRN_PER];
#pragma unroll
        for (int e = 0; e < BRN_PER; e++) {
            const int i = base + e * 256 + (int)threadIdx.x;
            hv[e] = i < H ? __half2float(row[i]) : 0.f;
            fv[e] = i < H ? fr[i] : 0.f;
            wv[e] = i < H ? w[i] : __float2half_rn(0.f);
        }
#pragma unroll
        for (int e = 0; e < BRN_PER; e++) {
            const int i = base + e * 256 + (int)threadIdx.x;
            hn[e] = __float2half_rn(hv[e] + fv[e]);
            if (i < H) {
                row[i] = hn[e];
                const float x = __half2float(hn[e]);
                ss += x * x;
            }
        }
    }
    ss = block_sum(ss, red);
    const float inv = rsqrtf(ss / (float)H + eps);
    if (H <= BRN_PER * 256) {
#pragma unroll
        for (int e = 0; e < BRN_PER; e++) {
            const int i = e * 256 + (int)threadIdx.x;
            if (i < H) xn[(size_t)blockIdx.x * H + i] = __float2half_rn(__half2float(hn[e]) * inv * __half2float(wv[e]));
        }
    } else {
        for (int i = threadIdx.x; i < H; i += 256)
            xn[(size_t)blockIdx.x * H + i] = __float2half_rn(__half2float(row[i]) * inv * __half2float(w[i]));
    }
}
// The MoE combine (k_bcombine's arithmetic: acc = half(acc + w_t * o_t) in
// slot order, then h = half(h + acc)) then the next RMSNorm, one CTA (256
// threads) per sequence, the same element mapping as k_bres_norm.
__global__ void __launch_bounds__(256) k_bcombine_norm(const float* __restrict__ obuf, const int* __restrict__ inv,
                                                       const float* __restrict__ rw, __half* h, int H, int topk,
                                                       EpWait wait, const __half* __restrict__ w, __half* xn,
                                                       float eps) {
    __shared__ float red[32];
    if (wait.flags) {  // expert-parallel: the peers' outputs have arrived
        if (threadIdx.x == 0) ep_wait_flags(wait);
        __syncthreads();
    }
    const int b = blockIdx.x;
    __half* row = h + (size_t)b * H;
    const float* src[8];
    float wt[8];
#pragma unroll
    for (int t = 0; t < 8; t++) {
        src[t] = t < topk ? obuf + (size_t)inv[b * topk + t] * H : obuf;
        wt[t] = t < topk ? rw[b * topk + t] : 0.f;
    }
    float ss = 0.f;
    if (H <= 8 * 256) {
        // every element of the thread in one round: all its loads (the norm
        // weights included) issued together, the normalisation from registers
        float o[8][8], hv[8];
        __half wv[8], hn[8];
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const int c = e * 256 + (int)threadIdx.x;
            hv[e] = c < H ? __half2float(row[c]) : 0.f;
            wv[e] = c < H ? w[c] : __float2half_rn(0.f);
#pragma unroll
            for (int t = 0; t < 8; t++)  // (L2 loads: rows another GPU may have written during the wait)
                o[e][t] = (c < H && t < topk) ? __ldcg(src[t] + c) : 0.f;
        }
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const int c = e * 256 + (int)threadIdx.x;
            __half acc = __float2half_rn(0.f);
#pragma unroll
            for (int t = 0; t < 8; t++)
                if (t < topk) acc = __float2half_rn(__half2float(acc) + wt[t] * o[e][t]);
            hn[e] = __float2half_rn(hv[e] + __half2float(acc));
            if (c < H) {
                row[c] = hn[e];
                const float x = __half2float(hn[e]);
                ss += x * x;
            }
        }
        ss = block_sum(ss, red);
        const float r = rsqrtf(ss / (float)H + eps);
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const int c = e * 256 + (int)threadIdx.x;
            if (c < H) xn[(size_t)b * H + c] = __float2half_rn(__half2float(hn[e]) * r * __half2float(wv[e]));
        }
        return;
    }
    for (int base = 0; base < H; base += 4 * 256) {
        float o[4][8], hv[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int c = base + e * 256 + (int)threadIdx.x;
            hv[e] = c < H ? __half2float(row[c]) : 0.f;
#pragma unroll
            for (int t = 0; t < 8; t++)
                o[e][t] = (c < H && t < topk) ? __ldcg(src[t] + c) : 0.f;
        }
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int c = base + e * 256 + (int)threadIdx.x;
            if (c < H) {
                __half acc = __float2half_rn(0.f);
#pragma unroll
                for (int t = 0; t < 8; t++)
                    if (t < topk) acc = __float2half_rn(__half2float(acc) + wt[t] * o[e][t]);
                const __half v = __float2half_rn(hv[e] + __half2float(acc));
                row[c] = v;
                const float x = __half2float(v);
                ss += x * x;
            }
        }
    }
    ss = block_sum(ss, red);
    const float r = rsqrtf(ss / (float)H + eps);
    for (int c = threadIdx.x; c < H; c += 256)
        xn[(size_t)b * H + c] = __float2half_rn(__half2float(row[c]) * r * __half2float(w[c]));
}

__global__ void k_btok(const unsigned long long* __restrict__ keys, int* tok, int* pos, int B) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    tok[b] = argmax_key_index(keys[b]);
    pos[b] += 1;
}

// Synthetic caches for benchmarking at a given context: every sequence's
// committed groups hold pseudo-random FP8 codes (the lowest exponent bit
// cleared, so no NaN codes; magnitudes up to 240) with group scales 1/112,
// and its position is set to ctx.
__global__ void k_bfill(uint8_t* c8, size_t n, unsigned long long seed) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        unsigned long long z = seed + i * 0x9E3779B97F4A7C15ull;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        z ^= z >> 31;
        c8[i] = (uint8_t)(z & 0xF7u);  // exponent field <= 14: finite E4M3
    }
}
__global__ void k_bfill_scales(__half* s, size_t n, float v) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        s[i] = __float2half_rn(v);
}
__global__ void k_bset(int* p, int B, int v) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) p[b] = v;
}

// Expert-parallel dispatch plan (one CTA, n = B*topk <= 1024 entries): entry
// j = (token, slot) goes to rank d = expert / e_loc at position rank-of-j
// among the entries for d (in entry order); dest_pos[j] = d * cap + position,
// meta[d * cap + position] = the expert's index on d, unused positions -1.
__global__ void __launch_bounds__(1024) k_ep_plan(const int* __restrict__ ridx, int n, int e_loc, int world,
                                                  int cap, int* dest_pos, int* meta) {
    __shared__ int sd[1024];
    const int j = threadIdx.x;
    for (int i = j; i < world * cap; i += blockDim.x) meta[i] = -1;
    int d = -1, e = -1;
    if (j < n) {
        e = ridx[j];
        d = e / e_loc;
        sd[j] = d;
    }
    __syncthreads();
    if (j < n) {
        int r = 0;
        for (int i = 0; i < j; i++) r += sd[i] == d;
        dest_pos[j] = d * cap + r;
        meta[d * cap + r] = e - d * e_loc;
    }
}
// The same plan on the host (for checking the exchange protocol without a
// GPU): identical outputs to k_ep_plan for the same routes.
extern "C" int cuinf_ep_plan_host(const int* ridx, int n, int e_loc, int world, int cap, int* dest_pos, int* meta) {
    REQUIRE(ridx && dest_pos && meta, "null pointer");
    REQUIRE(n >= 0 && e_loc > 0 && world > 0 && cap >= 0, "bad plan sizes");
    for (int i = 0; i < world * cap; i++) meta[i] = -1;
    std::vector<int> fill(world, 0);
    for (int j = 0; j < n; j++) {
        const int e = ridx[j], d = e / e_loc;
        REQUIRE(e >= 0 && d < world, "expert id out of range");
        const int r = fill[d]++;
        REQUIRE(r < cap, "more rows for one rank than the capacity");
        dest_pos[j] = d * cap + r;
        meta[d * cap + r] = e - d * e_loc;
    }
    return CUINF_OK;
}

// send_x[dest_pos[j]] = xn[j / topk]
__global__ void k_ep_pack(const __half* __restrict__ xn, const int* __restrict__ dest_pos, __half* send_x, int H,
                          int topk) {
    const int j = blockIdx.x;
    const uint4* s = reinterpret_cast<const uint4*>(xn + (size_t)(j / topk) * H);
    uint4* d = reinterpret_cast<uint4*>(send_x + (size_t)dest_pos[j] * H);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x) d[i] = s[i];
}
// back_o[j] = fo[inv[j]] for received entries that hold a row
__global__ void k_ep_unpack(const float* __restrict__ fo, const int* __restrict__ inv, float* back_o, int H) {
    const int j = blockIdx.x, r = inv[j];
    if (r < 0) return;
    const float4* s = reinterpret_cast<const float4*>(fo + (size_t)r * H);
    float4* d = reinterpret_cast<float4*>(back_o + (size_t)j * H);
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) d[i] = s[i];
}

// ---------------------------------------------------------------------------
// Grouped INT4 GEMV for the batched MoE: every group (an expert's rows of the
// gathered activations, up to 128) times that expert's weight matrix, 8
// activation rows per pass.  About top_k*B/E rows reach an expert (8 for 64
// sequences), far too few to amortise the dequantized 128x128 operand tile of
// the tensor-core GEMM: here the INT4 tile is dequantized in registers and
// fed to mma.sync m16n8k16 whose 8 columns are 8 activation rows, so one
// dequantization serves 8 rows and the kernel streams the weights at the pace
// of the batch-1 decode kernels.  Per 128-K group the products (nib-8)*x are
// exact and summed in fp32, then scaled in fp32 (as the reference's gemv_int4
// sums dequantized products in fp32, engine.cu:83-109).
// grid (N / (16*G8_TILES), groups), 256 threads: warps 4t..4t+3 take tile t
// (16 weight rows), each a quarter of the K groups.
// ---------------------------------------------------------------------------
#define G8_TILES 2
// x rows in shared memory at a pitch of 32 mod 128 bytes: the 16-byte loads
// of one 8-lane phase (rows g, g+1; chunks c = 0..3) then hit at most two
// lanes per 16-byte bank slot.
__host__ __device__ inline unsigned g8_pitch(int K) {
    const unsigned b = 2u * (unsigned)K;
    return b + ((32u - (b & 127u)) & 127u);
}
__host__ __device__ inline size_t g8_smem(int K) {
    return (size_t)G8_TILES * int4_tile_bytes(K) + (size_t)8 * g8_pitch(K) + 8 * 16 * 8 * 4;
}
// SwiGLU of the expert's w1 and w3 outputs (swiglu, engine.cu:542-547), the
// arithmetic of the standalone k_swiglu.
__device__ __forceinline__ float g8_silu(float x) { return x / (1.f + __expf(-x)); }
// xsrc (nullable): activation row of each grouped row (x holds the
// ungrouped rows, so no gathered copy is needed); null: row = grouped row.
// PAIR (the w1/w3 pass): CTA (x, y) takes rows [16x, 16x+16) of group y
// (w1, tile 0) and of group y + npair (w3, tile 1), whose activation rows
// are the same, and writes mid = half(silu(w1 . x) * (w3 . x)) at a row
// pitch of ldm instead of the two fp32 outputs (each sum as without PAIR,
// so mid is the same bits as the separate SwiGLU kernel's).
template <bool PAIR>
__global__ void __launch_bounds__(256) k_grouped_gemv8(const TcGroup* __restrict__ groups, const __half* __restrict__ x,
                                                       int ldx, int K, unsigned* err,
                                                       const int* __restrict__ xsrc = nullptr, int npair = 0,
                                                       __half* mid = nullptr, int ldm = 0) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t bar_w, bar_x;
    const TcGroup G = groups[blockIdx.y];
    const int rbase = blockIdx.x * 16 * (PAIR ? 1 : G8_TILES);
    if (G.rows <= 0 || rbase >= G.N) return;
    const uint32_t TB = int4_tile_bytes(K), XP = g8_pitch(K), XB = 2u * (uint32_t)K;
    uint8_t* xs = smem + G8_TILES * TB;                                              // [8][XP] x rows
    float* red = reinterpret_cast<float*>(smem + G8_TILES * TB + (size_t)8 * XP);  // [8][16][8]
    const int ntile = PAIR ? 2 : min(G8_TILES, (G.N - rbase) / 16);
    if (threadIdx.x == 0) {
        mbar_init(&bar_w, 1);
        mbar_init(&bar_x, 1);
        mbar_arrive_expect_tx(&bar_w, ntile * TB);
        if (PAIR) {
            const TcGroup G3 = groups[blockIdx.y + npair];
            tma_tile_int4(G.packed, G.scales, K, rbase, smem, &bar_w);
            tma_tile_int4(G3.packed, G3.scales, K, rbase, smem + TB, &bar_w);
        } else {
            for (int t = 0; t < ntile; t++)
                tma_tile_int4(G.packed, G.scales, K, rbase + 16 * t, smem + t * TB, &bar_w);
        }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int tile = warp >> 2, q = warp & 3, KG = K >> 7, KH = K >> 1;
    bool ok = true;
    int pass = 0;
    for (int p0 = 0; p0 < G.rows; p0 += 8, pass++) {
        const int np = min(8, G.rows - p0);
        if (threadIdx.x == 0) {
            // this pass's activation rows (rows past np keep stale values: their
            // mma columns are independent of the others and are never stored)
            mbar_arrive_expect_tx(&bar_x, np * XB);
            int sr[8];
#pragma unroll
            for (int r = 0; r < 8; r++) {
                const int gr = G.x_row + p0 + r;
                sr[r] = r < np ? (xsrc ? xsrc[gr] : gr) : 0;
            }
            for (int r = 0; r < np; r++) tma_load_1d(xs + r * XP, x + (size_t)sr[r] * ldx, XB, &bar_x);
        }
        __syncthreads();  // barrier inits are visible before anyone waits
        if (pass == 0) ok = mbar_wait_bounded(&bar_w, 0, err);
        ok = mbar_wait_bounded(&bar_x, pass & 1, err) && ok;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        if (ok && tile < ntile) {
            const uint8_t* tb = smem + tile * TB;
            const uint8_t* pa = tb + g * KH + c * 16;
            const uint8_t* pb = tb + (g + 8) * KH + c * 16;
            const __half* sc = reinterpret_cast<const __half*>(tb + 16 * KH);
            // lane (g, c) feeds x row g, k = 128Gk + 32c + 8j .. +7 for mma pair j
            const uint8_t* xr = xs + g * XP + c * 64;
            for (int Gk = q; Gk < KG; Gk += 4) {
                const uint4 wa = *reinterpret_cast<const uint4*>(pa + Gk * 64);
                const uint4 wb = *reinterpret_cast<const uint4*>(pb + Gk * 64);
                const float fa = __half2float(sc[g * KG + Gk]), fb = __half2float(sc[(g + 8) * KG + Gk]);
                const uint32_t wav[4] = {wa.x, wa.y, wa.z, wa.w}, wbv[4] = {wb.x, wb.y, wb.z, wb.w};
                float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    uint32_t ha[4], hb[4];
                    dequant8(wav[j], ha);
                    dequant8(wbv[j], hb);
                    // x[k..k+7] as words (k,k+1) (k+2,k+3) (k+4,k+5) (k+6,k+7);
                    // the fragments want (k,k+4) (k+1,k+5) and (k+2,k+6) (k+3,k+7)
                    const uint4 xv = *reinterpret_cast<const uint4*>(xr + Gk * 256 + j * 16);
                    mma_16816(d, ha[0], hb[0], ha[1], hb[1], __byte_perm(xv.x, xv.z, 0x5410),
                              __byte_perm(xv.x, xv.z, 0x7632));
                    mma_16816(d, ha[2], hb[2], ha[3], hb[3], __byte_perm(xv.y, xv.w, 0x5410),
                              __byte_perm(xv.y, xv.w, 0x7632));
                }
                acc[0] = fmaf(fa, d[0], acc[0]);
                acc[1] = fmaf(fa, d[1], acc[1]);
                acc[2] = fmaf(fb, d[2], acc[2]);
                acc[3] = fmaf(fb, d[3], acc[3]);
            }
        }
        // red[warp][row][token]: row g / g+8 of the warp's tile, tokens 2c, 2c+1
        red[(warp * 16 + g) * 8 + 2 * c] = acc[0];
        red[(warp * 16 + g) * 8 + 2 * c + 1] = acc[1];
        red[(warp * 16 + g + 8) * 8 + 2 * c] = acc[2];
        red[(warp * 16 + g + 8) * 8 + 2 * c + 1] = acc[3];
        __syncthreads();
        if (PAIR) {
            if (threadIdx.x < 128) {
                const int r = (threadIdx.x >> 3) & 15, tok = threadIdx.x & 7;
                if (tok < np) {
                    float gv = 0.f, uv = 0.f;
#pragma unroll
                    for (int w = 0; w < 4; w++) gv += red[(w * 16 + r) * 8 + tok];
#pragma unroll
                    for (int w = 0; w < 4; w++) uv += red[((4 + w) * 16 + r) * 8 + tok];
                    mid[(size_t)(G.x_row + p0 + tok) * ldm + rbase + r] = __float2half_rn(g8_silu(gv) * uv);
                }
            }
        } else {
            for (int i = threadIdx.x; i < ntile * 128; i += blockDim.x) {
                const int t = i >> 7, r = (i >> 3) & 15, tok = i & 7;
                if (tok < np) {
                    float v = 0.f;
#pragma unroll
                    for (int w = 0; w < 4; w++) v += red[((4 * t + w) * 16 + r) * 8 + tok];
                    G.y[(size_t)(p0 + tok) * G.ldy + rbase + 16 * t + r] = v;
                }
            }
        }
        __syncthreads();  // xs and red are refilled by the next pass
    }
}

// Shapes the grouped small-row GEMV takes (whole 32-row CTA tiles, and its
// shared memory within one SM's limit).
#define G8_SMEM_MAX (200 * 1024)
static bool g8_fits(int H, int I) {
    return H % (16 * G8_TILES) == 0 && I % (16 * G8_TILES) == 0 && H % 128 == 0 && I % 128 == 0 &&
           g8_smem(std::max(H, I)) <= G8_SMEM_MAX;
}
static int g8_attr_once() {
    static cudaError_t e = cudaFuncSetAttribute(k_grouped_gemv8<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                G8_SMEM_MAX);
    if (e != cudaSuccess) return cuinf_set_cuda_error(e);
    static cudaError_t e1 = cudaFuncSetAttribute(k_grouped_gemv8<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 G8_SMEM_MAX);
    if (e1 != cudaSuccess) return cuinf_set_cuda_error(e1);
    return CUINF_OK;
}

// ---------------------------------------------------------------------------
// host: one step as a sequence of launches (recorded into a graph)
// ---------------------------------------------------------------------------
#define BTRY(x)                      \
    do {                             \
        int rc_ = (x);               \
        if (rc_ != CUINF_OK) return rc_; \
    } while (0)

struct BStep {
    cuinf_batch* b;
    bool dry;  // size the split-K workspace only
    size_t need_slots = 0, need_cnt = 0;
    int launches = 0;
    // eager profiling: an event after each launch, with the launch's name
    std::vector<std::pair<const char*, cudaEvent_t>>* prof = nullptr;
    bool trace = false;  // eager profiling only: synchronize and report each launch
    int mark(const char* name) {
        if (dry || !prof) return CUINF_OK;
        cudaEvent_t e;
        CUINF_TRY(cudaEventCreate(&e));
        CUINF_TRY(cudaEventRecord(e, b->st));
        prof->push_back({name, e});
        if (trace) {
            CUINF_TRY(cudaStreamSynchronize(b->st));
            fprintf(stderr, "[cuinf batch] %3zu %s done\n", prof->size(), name);
            fflush(stderr);
        }
        return CUINF_OK;
    }

    // xrows: most activation rows any group of the launch can have
    int gemm(const CUtensorMap& xm, int xbox, int xrows, int wmap_idx, const TcGroup* dg, TcGroup g0, int ngroups,
             int tiles, int K, int active_ctas, bool fp16w, unsigned long long* amax, int n_base = 0) {
        TcPlan pl = amax ? TcPlan{1, K / TC_KS} : tc_plan(active_ctas, K, b->num_sms);
        REQUIRE(fp16w || pl.kgps <= TC_MAX_KG, "K too large");
        launches++;
        if (pl.splits > 1) {
            need_slots = std::max(need_slots, (size_t)ngroups * tiles * pl.splits);
            need_cnt = std::max(need_cnt, (size_t)ngroups * tiles);
        }
        if (dry) return CUINF_OK;
        TcParams P = {};
        P.groups = dg;
        P.g0 = g0;
        P.n_groups = ngroups;
        P.K = K;
        P.splits = pl.splits;
        P.kg_per_split = pl.kgps;
        P.fp16_w = fp16w;
        P.xmax = (std::min(xrows, TC_NMAX) + 15) & ~15;
        P.xbox = xbox;
        P.ws = b->ws;
        P.counters = b->cnt;
        P.amax = amax;
        P.n_base = n_base;
        const CUtensorMap& wm = wmap_idx >= 0 ? b->hmaps[wmap_idx] : b->hmaps[0];
        return tc_launch(xm, wm, P, tiles, b->st, false);
    }
    // single weight matrix, all B rows
    int gemm1(const CUtensorMap& xm, int wi, const __half* scales, float* y, int N, int K, bool fp16w = false,
              unsigned long long* amax = nullptr) {
        TcGroup g = {};
        g.wmap = nullptr;
        g.scales = scales;
        g.y = y;
        g.x_row = 0;
        g.rows = b->B;
        g.N = N;
        g.ldy = N;
        const int tiles = (N + TC_ROWS - 1) / TC_ROWS;
        return gemm(xm, (b->B + 15) & ~15, b->B, wi, nullptr, g, 1, tiles, K, tiles, fp16w, amax);
    }
    int ew(int rc) {
        launches++;
        return rc;
    }
};

// ---------------------------------------------------------------------------
// expert-parallel failure handling: the communicator is non-blocking, every
// host wait on NCCL work polls its asynchronous error state under a time
// limit, and a failure aborts the communicator (NCCL then releases the
// kernels still waiting for peers) and marks the batch unusable.
// ---------------------------------------------------------------------------
static double now_ms() {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}
static int ep_fail(cuinf_batch* b, const char* what) {
    if (b->comm) ncclCommAbort(b->comm);
    b->comm = nullptr;
    b->ep_failed = true;
    return cuinf_set_arg_error(what);
}
// Wait until a non-blocking NCCL call (init, group end) has been accepted.
static int ep_settle(cuinf_batch* b, ncclResult_t r, const char* what) {
    if (r != ncclSuccess && r != ncclInProgress) return ep_fail(b, what);
    const double t0 = now_ms();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        if (ncclCommGetAsyncError(b->comm, &st) != ncclSuccess) return ep_fail(b, what);
        if (st == ncclSuccess) return CUINF_OK;
        if (st != ncclInProgress) return ep_fail(b, what);
        if (now_ms() - t0 > b->ep_timeout_ms) return ep_fail(b, "NCCL call timed out (a peer did not join)");
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}
// Synchronize the batch stream; for an expert-parallel batch, poll the
// communicator's error state meanwhile and give up after the time limit.
static int batch_sync(cuinf_batch* b) {
    if (!b->comm) {
        if (b->ep_failed) return cuinf_set_arg_error("expert-parallel batch was aborted");
        CUINF_TRY(cudaStreamSynchronize(b->st));
        return CUINF_OK;
    }
    const double t0 = now_ms();
    for (int k = 0;; k++) {
        const cudaError_t e = cudaStreamQuery(b->st);
        if (e == cudaSuccess) return CUINF_OK;
        if (e != cudaErrorNotReady) return cuinf_set_cuda_error(e);
        ncclResult_t st = ncclSuccess;
        if (ncclCommGetAsyncError(b->comm, &st) != ncclSuccess || (st != ncclSuccess && st != ncclInProgress))
            return ep_fail(b, "expert-parallel step failed: NCCL reported an asynchronous error");
        if (now_ms() - t0 > b->ep_timeout_ms)
            return ep_fail(b, "expert-parallel step timed out (a peer did not complete it); communicator aborted");
        if (k > 64) std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

static int batch_record(cuinf_batch* b, BStep& S) {
    const cuinf_model* m = b->m;
    const cuinf_config& c = m->cfg;
    const int B = b->B, H = c.hidden, nh = c.n_heads, nkv = c.n_kv_heads, E = c.n_experts, K = c.top_k;
    const int NQ = nh * 64, NK = nkv * 64;
    void* vs = (void*)b->st;
    const bool dry = S.dry;
    auto run = [&](int rc) { return dry ? CUINF_OK : rc; };
    if (b->p2p) {
        S.launches++;
        if (!dry) {
            k_ep_tick<<<1, 1, 0, b->st>>>(b->ep_step);
            BTRY(cuinf_launch_status());
        }
    }
    BTRY(S.ew(run(cuinf_embed_gather(m->embed, b->tok, b->h, B, H, vs))));
    BTRY(S.mark("embed"));
    int moe_i = 0;
    bool xn_ready = false;  // the previous layer's last kernel already normalised h
    for (int l = 0; l < c.n_layers; l++) {
        const LayerW& L = m->L[l];
        // the RMSNorm that follows this layer's FFN: the next layer's, or the final one
        const __half* next_norm = l + 1 < c.n_layers ? m->L[l + 1].op_norm : m->emb_norm;
        if (!xn_ready) {
            BTRY(S.ew(run(cuinf_rmsnorm(b->h, L.op_norm, b->xn, B, H, c.norm_eps, vs))));
            BTRY(S.mark("rmsnorm"));
        }
        xn_ready = false;
        if (c.attn_layer[l]) {
            const AttnState& A = b->attn[l];
            float* qf = b->fqkv;  // q | k | v rows, converted together below
            __half* q16 = b->qkv16;
            __half* k16 = q16 + (size_t)B * NQ;
            __half* v16 = k16 + (size_t)B * NK;
            const int tiles = (NQ + TC_ROWS - 1) / TC_ROWS;
            const int active = tiles + 2 * ((NK + TC_ROWS - 1) / TC_ROWS);
            BTRY(S.gemm(b->x_h, (B + 15) & ~15, B, -1, b->dstatic + b->qkv_tab[l], TcGroup{}, 3, tiles, H, active,
                        false, nullptr));
            BTRY(S.mark("gemm_qkv"));
            S.launches++;
            if (!dry) {
                k_bqkv_post<<<dim3(B, nh + 2 * nkv), CUINF_HD, 0, b->st>>>(qf, q16, k16, v16, L.q_ln, L.k_ln, b->pos, nh,
                                                                        nkv, c.norm_eps, c.rope_theta);
                BTRY(cuinf_launch_status());
                BTRY(S.mark("qkv_norm_rope"));
            }
            S.launches++;
            if (!dry) {
                k_bkv_place<<<dim3(B, nkv), 256, 0, b->st>>>(k16, v16, b->pos, A.ktail, A.vtail, A.kc8, A.vc8, A.ksc,
                                                             A.vsc, nkv, b->tail_seq, b->kv8_seq, b->sc_seq);
                BTRY(cuinf_launch_status());
                BTRY(S.mark("kv_place"));
            }
            BatchAttnArgs a;
            a.q = q16;
            a.kc8 = A.kc8;
            a.vc8 = A.vc8;
            a.ksc = A.ksc;
            a.vsc = A.vsc;
            a.ktail = A.ktail;
            a.vtail = A.vtail;
            a.pos = b->pos;
            a.out = b->attn_out;
            a.part = b->apart;
            a.counters = b->acnt;
            a.nh = nh;
            a.nkv = nkv;
            a.nsplit = b->nsplit;
            a.n_seqs = B;
            a.bq = NQ;
            a.bkv8 = b->kv8_seq;
            a.bsc = b->sc_seq;
            a.btail = b->tail_seq;
            a.bout = NQ;
            a.bpart = attn_batched_part_floats(nh, nkv, b->nsplit);
            a.scale = 0.125f;
            BTRY(S.ew(run(attn_decode_batched(a, b->st))));
            BTRY(S.mark("attention"));
            BTRY(S.gemm1(b->x_attn, b->mi_o[l], L.wo.s, b->fa, H, NQ));
            BTRY(S.mark("gemm_o"));
        } else {
            BTRY(S.gemm1(b->x_h, b->mi_in[l], L.in_proj.s, b->fa, 3 * H, H));
            BTRY(S.mark("gemm_conv_in"));
            S.launches++;
            if (!dry) {
                k_bconv<<<(B * H + 255) / 256, 256, 0, b->st>>>(b->fa, L.conv_w, b->conv_state[l], b->conv_y, B, H);
                BTRY(cuinf_launch_status());
                BTRY(S.mark("conv"));
            }
            BTRY(S.gemm1(b->x_conv, b->mi_out[l], L.out_proj.s, b->fa, H, H));
            BTRY(S.mark("gemm_conv_out"));
        }
        S.launches++;
        if (!dry) {
            k_bres_norm<<<B, 256, 0, b->st>>>(b->h, b->fa, L.ffn_norm, b->xn, H, c.norm_eps);
            BTRY(cuinf_launch_status());
            BTRY(S.mark("residual_norm"));
        }
        if (l < c.n_dense) {
            const int I = c.dense_inter, tiles = (I + TC_ROWS - 1) / TC_ROWS;
            BTRY(S.gemm(b->x_h, (B + 15) & ~15, B, -1, b->dstatic + b->d13_tab[l], TcGroup{}, 2, tiles, H,
                        2 * tiles, false, nullptr));
            BTRY(S.mark("gemm_dense_w13"));
            BTRY(S.ew(run(cuinf_swiglu(b->fg, b->fu, b->dmid, B * I, vs))));
            BTRY(S.mark("swiglu"));
            BTRY(S.gemm1(b->x_dmid, b->mi_w2[l], L.w2.s, b->fa, H, I));
            BTRY(S.mark("gemm_dense_w2"));
            S.launches++;
            if (!dry) {
                k_bres_norm<<<B, 256, 0, b->st>>>(b->h, b->fa, next_norm, b->xn, H, c.norm_eps);
                BTRY(cuinf_launch_status());
                BTRY(S.mark("residual_norm"));
            }
            xn_ready = true;
        } else {
            const int I = c.moe_inter;
            const bool ep = b->ep_world > 1;
            const int EL = ep ? b->e_loc : E;           // experts in this rank's group tables
            const int NR = ep ? b->ep_world * b->cap : B * K;  // rows grouped here
            // the small-row GEMV takes each expert's rows as one group (any count,
            // in passes of 8); the tensor-core GEMM takes groups of TC_NMAX
            const bool g8 = g8_fits(H, I);
            const int mch = g8 ? 1 : (NR + TC_NMAX - 1) / TC_NMAX;
            BTRY(S.ew(run(cuinf_gemv_fp16(b->xn, L.gate, b->rlog, B, E, H, vs))));
            BTRY(S.mark("router_gemv"));
            BRouteParams R = {};
            R.logits = b->rlog;
            R.bias = L.ebias;
            R.B = B;
            R.E = E;
            R.topk = K;
            R.I = I;
            R.H = H;
            R.maxch = mch;
            R.rowcap = g8 ? NR : TC_NMAX;
            R.ridx = b->ridx + (size_t)moe_i * B * K;
            R.rw = b->rw;
            R.keys = nullptr;
            R.n = B * K;
            R.n_local = EL;
            R.group = 1;
            R.inv = b->inv;
            R.src = b->src;
            R.g13 = b->g13;
            R.g2 = b->g2;
            R.maps = b->dmaps + b->mi_experts[moe_i] + 3 * b->e_lo;
            R.experts = (void* const*)(m->d_experts + ((size_t)L.moe_index * E + b->e_lo) * 6);
            R.gbuf = b->fg;
            R.ubuf = b->fu;
            R.obuf = b->fo;
            if (!ep) {
                // (the small-row GEMV reads each grouped row straight from xn
                // through src; the tensor-core GEMM's map wants a gathered copy)
                S.launches += g8 ? 1 : 2;
                if (!dry) {
                    k_broute<<<1, 1024, 0, b->st>>>(R);
                    BTRY(cuinf_launch_status());
                    BTRY(S.mark("route_group"));
                    if (!g8) {
                        k_bgather<<<B * K, 256, 0, b->st>>>(b->xn, b->src, b->xg, H);
                        BTRY(cuinf_launch_status());
                        BTRY(S.mark("gather"));
                    }
                }
            } else if (b->p2p) {
                // route this rank's tokens, write each (token, slot) row into its
                // expert's rank, wait for every peer's rows, group them by local expert
                S.launches += 4;
                if (!dry) {
                    R.group = 0;
                    k_broute<<<1, 1024, 0, b->st>>>(R);
                    BTRY(cuinf_launch_status());
                    BTRY(S.mark("route"));
                    k_ep_send<<<B * K + b->ep_world, 256, 0, b->st>>>(b->links, R.ridx, B * K, b->e_loc, b->xn, K,
                                                                      b->dest_pos, b->ep_ticket, b->ep_step,
                                                                      2 * moe_i);
                    BTRY(cuinf_launch_status());
                    BTRY(S.mark("ep_dispatch"));
                    R.keys = reinterpret_cast<const int*>(b->links.base[b->ep_rank] + b->links.off_meta);
                    R.n = NR;
                    R.group = 1;
                    R.wait.flags = reinterpret_cast<const unsigned long long*>(b->links.base[b->ep_rank] +
                                                                               b->links.off_flag);
                    R.wait.step = b->ep_step;
                    R.wait.world = b->ep_world;
                    R.wait.tag = 2 * moe_i;
                    R.wait.err = g_tc_err_ptr;
                    k_broute<<<1, 1024, 0, b->st>>>(R);
                    BTRY(cuinf_launch_status());
                    k_bgather<<<NR, 256, 0, b->st>>>(
                        reinterpret_cast<const __half*>(b->links.base[b->ep_rank] + b->links.off_x), b->src, b->xg,
                        H);
                    BTRY(cuinf_launch_status());
                    BTRY(S.mark("ep_group"));
                }
            } else {
                // route this rank's tokens, pack each (token, slot) row for its
                // expert's rank, exchange, group the received rows by local expert
                S.launches += 5;
                if (!dry) {
                    R.group = 0;
                    k_broute<<<1, 1024, 0, b->st>>>(R);
                    BTRY(cuinf_launch_status());
                    BTRY(S.mark("route"));
                    k_ep_plan<<<1, 1024, 0, b->st>>>(R.ridx, B * K, b->e_loc, b->ep_world, b->cap, b->dest_pos,
                                                      b->send_meta);
                    BTRY(cuinf_launch_status());
                    k_ep_pack<<<B * K, 256, 0, b->st>>>(b->xn, b->dest_pos, b->send_x, H, K);
                    BTRY(cuinf_launch_status());
                    BTRY(S.mark("ep_pack"));
                    const size_t cx = (size_t)b->cap * H;
                    if (ncclGroupStart() != ncclSuccess) return cuinf_set_arg_error("ncclGroupStart failed");
                    for (int d = 0; d < b->ep_world; d++) {
                        ncclSend(b->send_x + d * cx, cx, ncclFloat16, d, b->comm, b->st);
                        ncclRecv(b->recv_x + d * cx, cx, ncclFloat16, d, b->comm, b->st);
                        ncclSend(b->send_meta + d * b->cap, b->cap, ncclInt32, d, b->comm, b->st);
                        ncclRecv(b->recv_meta + d * b->cap, b->cap, ncclInt32, d, b->comm, b->st);
                    }
                    BTRY(ep_settle(b, ncclGroupEnd(), "NCCL dispatch failed"));
                    BTRY(S.mark("ep_dispatch"));
                    R.keys = b->recv_meta;
                    R.n = NR;
                    R.group = 1;
                    k_broute<<<1, 1024, 0, b->st>>>(R);
                    BTRY(cuinf_launch_status());
                    k_bgather<<<NR, 256, 0, b->st>>>(b->recv_x, b->src, b->xg, H);
                    BTRY(cuinf_launch_status());
                    BTRY(S.mark("ep_group"));
                }
            }
            if (g8) {
                // few rows per expert: the grouped small-row GEMV (k_grouped_gemv8),
                // w1 and w3 of the same rows in one CTA with the SwiGLU applied there
                S.launches++;
                if (!dry) {
                    k_grouped_gemv8<true><<<dim3(I / 16, EL * mch), 256, g8_smem(H), b->st>>>(
                        b->g13, ep ? b->xg : b->xn, H, H, g_tc_err_ptr, ep ? nullptr : b->src, EL * mch, b->mmid, I);
                    BTRY(cuinf_launch_status());
                }
                BTRY(S.mark("gemv8_moe_w13_swiglu"));
                S.launches++;
                if (!dry) {
                    k_grouped_gemv8<false><<<dim3(H / (16 * G8_TILES), EL * mch), 256, g8_smem(I), b->st>>>(
                        b->g2, b->mmid, I, I, g_tc_err_ptr);
                    BTRY(cuinf_launch_status());
                }
                BTRY(S.mark("gemv8_moe_w2"));
            } else {
                const int t13 = (I + TC_ROWS - 1) / TC_ROWS, t2 = (H + TC_ROWS - 1) / TC_ROWS;
                // about min(experts, rows) experts are hit; each group is one tile row of CTAs
                const int hit = std::min(EL, NR);
                // an expert's group holds at most one row per token of every rank
                const int grows = B * b->ep_world;
                BTRY(S.gemm(b->x_xg, 16, grows, -1, b->g13, TcGroup{}, 2 * EL * mch, t13, H, 2 * hit * t13, false,
                            nullptr));
                BTRY(S.mark("gemm_moe_w13"));
                BTRY(S.ew(run(cuinf_swiglu(b->fg, b->fu, b->mmid, NR * I, vs))));
                BTRY(S.mark("swiglu_moe"));
                BTRY(S.gemm(b->x_mmid, 16, grows, -1, b->g2, TcGroup{}, EL * mch, t2, I, hit * t2, false, nullptr));
                BTRY(S.mark("gemm_moe_w2"));
            }
            const float* ob = b->fo;
            const int* oi = b->inv;
            EpWait cw = {};
            if (ep && b->p2p) {
                S.launches++;
                if (!dry) {
                    k_ep_send_back<<<NR, 256, 0, b->st>>>(b->links, b->fo, b->inv, b->ep_ticket + 1, b->ep_step,
                                                         2 * moe_i + 1);
                    BTRY(cuinf_launch_status());
                    BTRY(S.mark("ep_return"));
                }
                ob = reinterpret_cast<const float*>(b->links.base[b->ep_rank] + b->links.off_back);
                oi = b->dest_pos;
                cw.flags = reinterpret_cast<const unsigned long long*>(b->links.base[b->ep_rank] + b->links.off_flag) +
                           b->ep_world;
                cw.step = b->ep_step;
                cw.world = b->ep_world;
                cw.tag = 2 * moe_i + 1;
                cw.err = g_tc_err_ptr;
            } else if (ep) {
                S.launches++;
                if (!dry) {
                    k_ep_unpack<<<NR, 256, 0, b->st>>>(b->fo, b->inv, b->back_o, H);
                    BTRY(cuinf_launch_status());
                    const size_t co = (size_t)b->cap * H;
                    if (ncclGroupStart() != ncclSuccess) return cuinf_set_arg_error("ncclGroupStart failed");
                    for (int d = 0; d < b->ep_world; d++) {
                        ncclSend(b->back_o + d * co, co, ncclFloat32, d, b->comm, b->st);
                        ncclRecv(b->recv_back + d * co, co, ncclFloat32, d, b->comm, b->st);
                    }
                    BTRY(ep_settle(b, ncclGroupEnd(), "NCCL combine failed"));
                    BTRY(S.mark("ep_return"));
                }
                ob = b->recv_back;
                oi = b->dest_pos;
            }
            S.launches++;
            if (!dry) {
                k_bcombine_norm<<<B, 256, 0, b->st>>>(ob, oi, b->rw, b->h, H, K, cw, next_norm, b->xn, c.norm_eps);
                BTRY(cuinf_launch_status());
                BTRY(S.mark("combine_norm"));
            }
            xn_ready = true;
            moe_i++;
        }
    }
    // final norm (done by the last layer's closing kernel), lm_head with the
    // fused argmax (compute_logits_last, engine.cu:932-940)
    if (!xn_ready) {
        BTRY(S.ew(run(cuinf_rmsnorm(b->h, m->emb_norm, b->xn, B, H, c.norm_eps, vs))));
        BTRY(S.mark("rmsnorm_final"));
    }
    if (b->vocab_shard && !b->keep_logits) {
        // every rank's final rows, then this rank's vocabulary shard for all
        // of them, then the max over the ranks' argmax keys (the keys order
        // by value, then by the reference's tie rule on the global index)
        const int W = b->ep_world, GB = W * B, Vs = c.vocab / W;
        if (!dry) {
            BTRY(ep_settle(b, ncclAllGather(b->xn, b->xall, (size_t)B * H, ncclFloat16, b->comm, b->st),
                           "NCCL all-gather of the final rows failed"));
            CUINF_TRY(cudaMemsetAsync(b->kall, 0, (size_t)GB * 8, b->st));
        }
        BTRY(S.mark("ep_gather_rows"));
        TcGroup g = {};
        g.rows = GB;
        g.N = Vs;
        g.ldy = Vs;
        const int tiles = (Vs + TC_ROWS - 1) / TC_ROWS;
        BTRY(S.gemm(b->x_all, (GB + 15) & ~15, GB, b->mi_embed_shard, nullptr, g, 1, tiles, H, tiles, true, b->kall,
                    b->ep_rank * Vs));
        BTRY(S.mark("lm_head"));
        if (!dry)
            BTRY(ep_settle(b, ncclAllReduce(b->kall, b->kall, GB, ncclUint64, ncclMax, b->comm, b->st),
                           "NCCL all-reduce of the argmax keys failed"));
        BTRY(S.mark("ep_argmax_reduce"));
        S.launches++;
        if (!dry) {
            k_btok<<<(B + 127) / 128, 128, 0, b->st>>>(b->kall + (size_t)b->ep_rank * B, b->tok, b->pos, B);
            BTRY(cuinf_launch_status());
            BTRY(S.mark("next_token"));
        }
        return CUINF_OK;
    }
    if (!dry) CUINF_TRY(cudaMemsetAsync(b->amax, 0, (size_t)B * 8, b->st));
    BTRY(S.gemm1(b->x_h, b->mi_embed, nullptr, b->keep_logits ? b->logits : nullptr, c.vocab, H, true, b->amax));
    BTRY(S.mark("lm_head"));
    S.launches++;
    if (!dry) {
        k_btok<<<(B + 127) / 128, 128, 0, b->st>>>(b->amax, b->tok, b->pos, B);
        BTRY(cuinf_launch_status());
        BTRY(S.mark("next_token"));
    }
    return CUINF_OK;
}

static int batch_build_graph(cuinf_batch* b) {
    if (b->exec) cudaGraphExecDestroy(b->exec);
    if (b->graph) cudaGraphDestroy(b->graph);
    b->exec = nullptr;
    b->graph = nullptr;
    BStep D{b, true};
    BTRY(batch_record(b, D));
    if (D.need_slots > b->ws_slots) {
        if (b->ws) cudaFree(b->ws);
        b->ws = nullptr;
        CUINF_TRY(cudaMalloc(&b->ws, D.need_slots * TC_NMAX * TC_ROWS * sizeof(float)));
        b->ws_slots = D.need_slots;
    }
    if (D.need_cnt > b->cnt_n) {
        if (b->cnt) cudaFree(b->cnt);
        b->cnt = nullptr;
        CUINF_TRY(cudaMalloc(&b->cnt, D.need_cnt * sizeof(unsigned)));
        CUINF_TRY(cudaMemset(b->cnt, 0, D.need_cnt * sizeof(unsigned)));
        b->cnt_n = D.need_cnt;
    }
    BTRY(tc_attr_once());
    BTRY(g8_attr_once());
    CUINF_TRY(cudaStreamSynchronize(b->st));
    BStep R{b, false};
    CUINF_TRY(cudaStreamBeginCapture(b->st, cudaStreamCaptureModeThreadLocal));
    int rc = batch_record(b, R);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(b->st, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    CUINF_TRY(e);
    b->graph = g;
    CUINF_TRY(cudaGraphInstantiate(&b->exec, g, 0));
    b->kernels = R.launches;
    return CUINF_OK;
}

extern "C" int cuinf_batch_free(cuinf_batch* b) {
    if (!b) return CUINF_OK;
    if (b->st) cudaStreamSynchronize(b->st);
    if (b->exec) cudaGraphExecDestroy(b->exec);
    if (b->graph) cudaGraphDestroy(b->graph);
    for (void* p : b->peer_open) cudaIpcCloseMemHandle(p);
    for (void* p : b->allocs) cudaFree(p);
    if (b->ws) cudaFree(b->ws);
    if (b->cnt) cudaFree(b->cnt);
    if (b->pinned) cudaFreeHost(b->pinned);
    if (b->comm) ncclCommDestroy(b->comm);  // after the graph that holds its calls (an aborted one is gone)
    if (b->own_stream && b->st) cudaStreamDestroy(b->st);
    delete b;
    return CUINF_OK;
}

// Map every rank's exchange arena into this process (cudaIpc over the NCCL
// communicator).  All ranks take the same collective steps whatever happens
// locally; the peer-memory exchange is used only when every rank mapped
// every arena, otherwise the batch keeps the NCCL send/recv exchange.
static int ep_map_peers(cuinf_batch* b) {
    const int W = b->ep_world, H = b->m->cfg.hidden;
    const size_t rows = (size_t)W * b->cap;
    auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
    EpLinks& L = b->links;
    L.off_x = 0;
    L.off_meta = al(rows * H * 2);
    L.off_back = L.off_meta + al(rows * 4);
    L.off_flag = L.off_back + al(rows * H * 4);
    L.rank = b->ep_rank;
    L.world = W;
    L.cap = b->cap;
    L.H = H;
    char* arena = nullptr;
    BTRY(balloc(b, &arena, L.off_flag + al((size_t)2 * W * 8)));  // zeroed: every flag starts at 0
    BTRY(balloc(b, &b->ep_step, 8));
    BTRY(balloc(b, &b->ep_ticket, 8));
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    cudaIpcMemHandle_t mine;
    memset(&mine, 0, sizeof(mine));
    int ok = cudaIpcGetMemHandle(&mine, arena) == cudaSuccess;
    if (!ok) cudaGetLastError();
    unsigned char* dh = nullptr;
    int* dok = nullptr;
    BTRY(balloc(b, &dh, (size_t)W * hb));
    BTRY(balloc(b, &dok, 4));
    CUINF_TRY(cudaMemcpy(dh + (size_t)b->ep_rank * hb, &mine, hb, cudaMemcpyHostToDevice));
    BTRY(ep_settle(b, ncclAllGather(dh + (size_t)b->ep_rank * hb, dh, hb, ncclUint8, b->comm, b->st),
                   "NCCL all-gather of the exchange handles failed"));
    BTRY(batch_sync(b));
    std::vector<cudaIpcMemHandle_t> hs(W);
    CUINF_TRY(cudaMemcpy(hs.data(), dh, (size_t)W * hb, cudaMemcpyDeviceToHost));
    for (int p = 0; p < W; p++) {
        if (p == b->ep_rank) {
            L.base[p] = arena;
            continue;
        }
        void* ptr = nullptr;
        if (ok && cudaIpcOpenMemHandle(&ptr, hs[p], cudaIpcMemLazyEnablePeerAccess) == cudaSuccess) {
            b->peer_open.push_back(ptr);
            L.base[p] = (char*)ptr;
        } else {
            cudaGetLastError();
            ok = 0;
        }
    }
    CUINF_TRY(cudaMemcpy(dok, &ok, 4, cudaMemcpyHostToDevice));
    BTRY(ep_settle(b, ncclAllReduce(dok, dok, 1, ncclInt32, ncclMin, b->comm, b->st),
                   "NCCL all-reduce of the mapping status failed"));
    BTRY(batch_sync(b));
    int all = 0;
    CUINF_TRY(cudaMemcpy(&all, dok, 4, cudaMemcpyDeviceToHost));
    b->p2p_ok = all != 0;
    b->p2p = b->p2p_ok;
    return CUINF_OK;
}

static int batch_create(cuinf_model* m, int n_seqs, int max_ctx, void* stream, const unsigned char* nccl_id,
                        int rank, int world, cuinf_batch** out) {
    REQUIRE(m && out, "null pointer");
    const cuinf_config& c = m->cfg;
    REQUIRE(world >= 1 && rank >= 0 && rank < world, "bad rank / world");
    REQUIRE(world == 1 || (nccl_id && c.n_experts % world == 0),
            "expert parallelism needs an NCCL id and n_experts divisible by the world size");
    REQUIRE(world == 1 || (size_t)n_seqs * c.top_k * world <= 1024, "n_seqs * top_k * world must be <= 1024");
    REQUIRE(world <= EP_MAX_WORLD, "at most 8 ranks");
    REQUIRE(c.n_layers - c.n_dense <= 127, "at most 127 MoE layers");
    REQUIRE(n_seqs >= 1 && n_seqs <= TC_NMAX, "n_seqs must be in [1, 128]");
    REQUIRE(max_ctx >= 1, "max_ctx must be positive");
    REQUIRE(c.hidden % TC_KS == 0 && c.moe_inter % TC_KS == 0 && c.dense_inter % TC_KS == 0 &&
                (c.n_heads * 64) % TC_KS == 0,
            "batched decode needs hidden, intermediates and heads*64 multiples of 128");
    REQUIRE(c.n_experts <= 256 && c.top_k <= 8 && n_seqs * c.top_k <= 1024, "n_experts <= 256, top_k <= 8");
    REQUIRE(c.n_heads % c.n_kv_heads == 0 && c.n_heads / c.n_kv_heads <= 8, "GQA ratio <= 8");
    cuinf_batch* b = new cuinf_batch();
    b->m = m;
    b->B = n_seqs;
    b->ep_rank = rank;
    b->ep_world = world;
    b->e_loc = c.n_experts / world;
    b->e_lo = rank * b->e_loc;
    b->cap = n_seqs * c.top_k;
    b->max_ctx = max_ctx;
    int rc = CUINF_OK;
#define TRYB(x)                     \
    do {                            \
        if ((rc = (x)) != CUINF_OK) { \
            cuinf_batch_free(b);    \
            return rc;              \
        }                           \
    } while (0)
    if (stream) {
        b->st = (cudaStream_t)stream;
    } else {
        if (cudaStreamCreateWithFlags(&b->st, cudaStreamNonBlocking) != cudaSuccess) {
            delete b;
            return cuinf_set_arg_error("stream creation failed");
        }
        b->own_stream = true;
    }
    {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&b->num_sms, cudaDevAttrMultiProcessorCount, dev);
    }
    const int B = n_seqs, H = c.hidden, nkv = c.n_kv_heads, NQ = c.n_heads * 64, NK = nkv * 64, K = c.top_k;
    const int I = c.moe_inter, ID = c.dense_inter, E = c.n_experts;
    const int n_moe = c.n_layers - c.n_dense;
    const size_t groups = (size_t)max_ctx / CUINF_KVGROUP + 2;
    b->kv8_seq = (size_t)max_ctx * NK;
    b->sc_seq = groups * nkv;
    b->tail_seq = (size_t)CUINF_KVGROUP * NK;
    b->attn.assign(c.n_layers, AttnState());
    b->conv_state.assign(c.n_layers, nullptr);
    for (int l = 0; l < c.n_layers; l++) {
        if (c.attn_layer[l]) {
            AttnState& A = b->attn[l];
            TRYB(balloc(b, &A.kc8, B * b->kv8_seq));
            TRYB(balloc(b, &A.vc8, B * b->kv8_seq));
            TRYB(balloc(b, &A.ksc, B * b->sc_seq * 2));
            TRYB(balloc(b, &A.vsc, B * b->sc_seq * 2));
            TRYB(balloc(b, &A.ktail, B * b->tail_seq * 2));
            TRYB(balloc(b, &A.vtail, B * b->tail_seq * 2));
        } else {
            TRYB(balloc(b, &b->conv_state[l], (size_t)B * 2 * H * 2));
        }
    }
    const int maxN = std::max(std::max(3 * H, NQ + 2 * NK), ID);
    TRYB(balloc(b, &b->tok, (size_t)B * 4));
    TRYB(balloc(b, &b->pos, (size_t)B * 4));
    TRYB(balloc(b, &b->h, (size_t)B * H * 2));
    TRYB(balloc(b, &b->xn, (size_t)B * H * 2));
    TRYB(balloc(b, &b->qkv16, (size_t)B * (NQ + 2 * NK) * 2));
    TRYB(balloc(b, &b->attn_out, (size_t)B * NQ * 2));
    TRYB(balloc(b, &b->conv_y, (size_t)B * H * 2));
    TRYB(balloc(b, &b->dmid, (size_t)B * std::max(ID, 128) * 2));
    const int NR = world > 1 ? world * b->cap : B * K;  // rows the expert GEMMs group
    TRYB(balloc(b, &b->xg, (size_t)NR * H * 2));
    TRYB(balloc(b, &b->mmid, (size_t)NR * I * 2));
    TRYB(balloc(b, &b->fqkv, (size_t)B * (NQ + 2 * NK) * 4));
    TRYB(balloc(b, &b->fa, (size_t)B * maxN * 4));
    TRYB(balloc(b, &b->fb, (size_t)B * maxN * 4));
    TRYB(balloc(b, &b->fg, (size_t)std::max(NR * I, B * ID) * 4));
    TRYB(balloc(b, &b->fu, (size_t)std::max(NR * I, B * ID) * 4));
    TRYB(balloc(b, &b->fo, (size_t)NR * H * 4));
    TRYB(balloc(b, &b->rlog, (size_t)B * std::max(E, 1) * 4));
    TRYB(balloc(b, &b->logits, (size_t)B * c.vocab * 4));
    TRYB(balloc(b, &b->ridx, (size_t)std::max(n_moe, 1) * B * K * 4));
    TRYB(balloc(b, &b->rw, (size_t)B * K * 4));
    TRYB(balloc(b, &b->inv, (size_t)NR * 4));
    TRYB(balloc(b, &b->src, (size_t)NR * 4));
    if (world > 1) {
        const size_t rows = (size_t)world * b->cap;
        TRYB(balloc(b, &b->send_x, rows * H * 2));
        TRYB(balloc(b, &b->recv_x, rows * H * 2));
        TRYB(balloc(b, &b->send_meta, rows * 4));
        TRYB(balloc(b, &b->recv_meta, rows * 4));
        TRYB(balloc(b, &b->dest_pos, (size_t)B * K * 4));
        TRYB(balloc(b, &b->back_o, rows * H * 4));
        TRYB(balloc(b, &b->recv_back, rows * H * 4));
        ncclUniqueId id;
        memcpy(&id, nccl_id, sizeof(id));
        ncclConfig_t ncfg = NCCL_CONFIG_INITIALIZER;
        ncfg.blocking = 0;  // init and every group end are polled under b->ep_timeout_ms
        const ncclResult_t r = ncclCommInitRankConfig(&b->comm, world, id, rank, &ncfg);
        if (r != ncclSuccess && r != ncclInProgress) b->comm = nullptr;
        if (!b->comm || ep_settle(b, r, "ncclCommInitRankConfig failed")) {
            const std::string msg = cuinf_last_error();
            cuinf_batch_free(b);
            return cuinf_set_arg_error(msg.c_str());
        }
        TRYB(ep_map_peers(b));
    }
    TRYB(balloc(b, &b->amax, (size_t)B * 8));
    b->nsplit = attn_batched_nsplit(c.n_heads, nkv, max_ctx, B, b->num_sms);
    TRYB(balloc(b, &b->apart, (size_t)B * attn_batched_part_floats(c.n_heads, nkv, b->nsplit) * 4));
    TRYB(balloc(b, &b->acnt, (size_t)B * nkv * 4));
    const int maxch = (NR + TC_NMAX - 1) / TC_NMAX;
    TRYB(balloc(b, &b->g13, (size_t)2 * std::max(E, 1) * maxch * sizeof(TcGroup)));
    TRYB(balloc(b, &b->g2, (size_t)std::max(E, 1) * maxch * sizeof(TcGroup)));
    if (cudaHostAlloc(&b->pinned, (size_t)2 * B * 4, cudaHostAllocDefault) != cudaSuccess) {
        cuinf_batch_free(b);
        return cuinf_set_arg_error("pinned allocation failed");
    }
    // activation maps: shared layers one box over the batch, expert groups 16-row boxes
    const int xb = (B + 15) & ~15;
    TRYB(tc_map_act(&b->x_h, b->xn, B, H, xb));
    TRYB(tc_map_act(&b->x_conv, b->conv_y, B, H, xb));
    TRYB(tc_map_act(&b->x_attn, b->attn_out, B, NQ, xb));
    TRYB(tc_map_act(&b->x_dmid, b->dmid, B, ID, xb));
    TRYB(tc_map_act(&b->x_xg, b->xg, NR, H, 16));
    TRYB(tc_map_act(&b->x_mmid, b->mmid, NR, I, 16));
    // weight maps
    auto add4 = [&](const Q4& q, int N, int Kd, int* idx) -> int {
        CUtensorMap mm;
        int r = tc_map_int4(&mm, q.p, N, Kd);
        if (r) return r;
        *idx = (int)b->hmaps.size();
        b->hmaps.push_back(mm);
        return CUINF_OK;
    };
    const int nl = c.n_layers;
    b->mi_in.assign(nl, -1), b->mi_out.assign(nl, -1), b->mi_q.assign(nl, -1), b->mi_k.assign(nl, -1);
    b->mi_v.assign(nl, -1), b->mi_o.assign(nl, -1), b->mi_w1.assign(nl, -1), b->mi_w3.assign(nl, -1);
    b->mi_w2.assign(nl, -1);
    b->qkv_tab.assign(nl, -1), b->d13_tab.assign(nl, -1);
    std::vector<void*> ex((size_t)std::max(n_moe, 1) * E * 6);
    if (n_moe > 0)
        if (cudaMemcpy(ex.data(), m->d_experts, ex.size() * sizeof(void*), cudaMemcpyDeviceToHost) != cudaSuccess) {
            cuinf_batch_free(b);
            return cuinf_set_arg_error("expert table copy failed");
        }
    for (int l = 0; l < nl; l++) {
        const LayerW& L = m->L[l];
        if (c.attn_layer[l]) {
            TRYB(add4(L.wq, NQ, H, &b->mi_q[l]));
            TRYB(add4(L.wk, NK, H, &b->mi_k[l]));
            TRYB(add4(L.wv, NK, H, &b->mi_v[l]));
            TRYB(add4(L.wo, H, NQ, &b->mi_o[l]));
        } else {
            TRYB(add4(L.in_proj, 3 * H, H, &b->mi_in[l]));
            TRYB(add4(L.out_proj, H, H, &b->mi_out[l]));
        }
        if (l < c.n_dense) {
            TRYB(add4(L.w1, ID, H, &b->mi_w1[l]));
            TRYB(add4(L.w3, ID, H, &b->mi_w3[l]));
            TRYB(add4(L.w2, H, ID, &b->mi_w2[l]));
        } else {
            const int mi = L.moe_index;
            b->mi_experts.push_back((int)b->hmaps.size());
            for (int e = 0; e < E; e++) {
                void* const* t = &ex[((size_t)mi * E + e) * 6];
                int dummy;
                TRYB(add4(Q4{(const uint8_t*)t[0], (const __half*)t[1]}, I, H, &dummy));
                TRYB(add4(Q4{(const uint8_t*)t[2], (const __half*)t[3]}, I, H, &dummy));
                TRYB(add4(Q4{(const uint8_t*)t[4], (const __half*)t[5]}, H, I, &dummy));
            }
        }
    }
    {
        CUtensorMap mm;
        TRYB(tc_map_f16w(&mm, m->embed, c.vocab, H));
        b->mi_embed = (int)b->hmaps.size();
        b->hmaps.push_back(mm);
    }
    // the vocabulary shard of this rank (expert-parallel form), when the
    // shards are equal and every rank's rows fit one GEMM (<= 128 rows)
    if (world > 1 && c.vocab % world == 0 && (size_t)world * B <= TC_NMAX &&
        (((uintptr_t)(m->embed + (size_t)rank * (c.vocab / world) * H)) & 15) == 0) {
        const int Vs = c.vocab / world, GB = world * B;
        CUtensorMap mm;
        TRYB(tc_map_f16w(&mm, m->embed + (size_t)rank * Vs * H, Vs, H));
        b->mi_embed_shard = (int)b->hmaps.size();
        b->hmaps.push_back(mm);
        TRYB(balloc(b, &b->xall, (size_t)GB * H * 2));
        TRYB(balloc(b, &b->kall, (size_t)GB * 8));
        TRYB(tc_map_act(&b->x_all, b->xall, GB, H, (GB + 15) & ~15));
        b->vocab_shard = true;
    }
    TRYB(balloc(b, &b->dmaps, b->hmaps.size() * sizeof(CUtensorMap)));
    if (cudaMemcpy(b->dmaps, b->hmaps.data(), b->hmaps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice) !=
        cudaSuccess) {
        cuinf_batch_free(b);
        return cuinf_set_arg_error("tensor map upload failed");
    }
    // static group tables: q/k/v of attention layers, w1/w3 of dense layers
    std::vector<TcGroup> st;
    for (int l = 0; l < nl; l++) {
        const LayerW& L = m->L[l];
        if (c.attn_layer[l]) {
            b->qkv_tab[l] = (int)st.size();
            float* qf = b->fqkv;
            float* kf = qf + (size_t)B * NQ;
            float* vf = kf + (size_t)B * NK;
            st.push_back(TcGroup{b->dmaps + b->mi_q[l], L.wq.p, L.wq.s, qf, 0, B, NQ, NQ});
            st.push_back(TcGroup{b->dmaps + b->mi_k[l], L.wk.p, L.wk.s, kf, 0, B, NK, NK});
            st.push_back(TcGroup{b->dmaps + b->mi_v[l], L.wv.p, L.wv.s, vf, 0, B, NK, NK});
        }
        if (l < c.n_dense) {
            b->d13_tab[l] = (int)st.size();
            st.push_back(TcGroup{b->dmaps + b->mi_w1[l], L.w1.p, L.w1.s, b->fg, 0, B, ID, ID});
            st.push_back(TcGroup{b->dmaps + b->mi_w3[l], L.w3.p, L.w3.s, b->fu, 0, B, ID, ID});
        }
    }
    if (!st.empty()) {
        TRYB(balloc(b, &b->dstatic, st.size() * sizeof(TcGroup)));
        if (cudaMemcpy(b->dstatic, st.data(), st.size() * sizeof(TcGroup), cudaMemcpyHostToDevice) != cudaSuccess) {
            cuinf_batch_free(b);
            return cuinf_set_arg_error("group table upload failed");
        }
    }
    TRYB(batch_build_graph(b));
    *out = b;
    return CUINF_OK;
#undef TRYB
}

extern "C" int cuinf_batch_create(cuinf_model* m, int n_seqs, int max_ctx, void* stream, cuinf_batch** out) {
    return batch_create(m, n_seqs, max_ctx, stream, nullptr, 0, 1, out);
}
extern "C" int cuinf_batch_create_ep(cuinf_model* m, int n_seqs, int max_ctx, void* stream,
                                     const unsigned char* nccl_id, int rank, int world, cuinf_batch** out) {
    return batch_create(m, n_seqs, max_ctx, stream, nccl_id, rank, world, out);
}
extern "C" int cuinf_ep_unique_id(unsigned char* id, int id_bytes) {
    REQUIRE(id && id_bytes >= (int)sizeof(ncclUniqueId), "id buffer too small");
    ncclUniqueId u;
    if (ncclGetUniqueId(&u) != ncclSuccess) return cuinf_set_arg_error("ncclGetUniqueId failed");
    memcpy(id, &u, sizeof(u));
    return CUINF_OK;
}
extern "C" int cuinf_ep_unique_id_bytes(void) { return (int)sizeof(ncclUniqueId); }

extern "C" int cuinf_batch_reset(cuinf_batch* b) {
    REQUIRE(b, "null batch");
    const cuinf_config& c = b->m->cfg;
    for (int l = 0; l < c.n_layers; l++) {
        if (c.attn_layer[l]) {
            const AttnState& A = b->attn[l];
            CUINF_TRY(cudaMemsetAsync(A.kc8, 0, b->B * b->kv8_seq, b->st));
            CUINF_TRY(cudaMemsetAsync(A.vc8, 0, b->B * b->kv8_seq, b->st));
            CUINF_TRY(cudaMemsetAsync(A.ksc, 0, b->B * b->sc_seq * 2, b->st));
            CUINF_TRY(cudaMemsetAsync(A.vsc, 0, b->B * b->sc_seq * 2, b->st));
            CUINF_TRY(cudaMemsetAsync(A.ktail, 0, b->B * b->tail_seq * 2, b->st));
            CUINF_TRY(cudaMemsetAsync(A.vtail, 0, b->B * b->tail_seq * 2, b->st));
        } else {
            CUINF_TRY(cudaMemsetAsync(b->conv_state[l], 0, (size_t)b->B * 2 * c.hidden * 2, b->st));
        }
    }
    CUINF_TRY(cudaMemsetAsync(b->pos, 0, (size_t)b->B * 4, b->st));
    CUINF_TRY(cudaStreamSynchronize(b->st));
    return CUINF_OK;
}

extern "C" int cuinf_batch_step(cuinf_batch* b, const int* tokens, int* out_tokens) {
    REQUIRE(b && b->exec, "null batch");
    REQUIRE(!b->ep_failed, "expert-parallel batch was aborted");
    const int B = b->B;
    if (tokens) {
        for (int i = 0; i < B; i++) REQUIRE(tokens[i] >= 0 && tokens[i] < b->m->cfg.vocab, "token out of range");
        BTRY(batch_sync(b));  // the pinned slot is free
        memcpy(b->pinned, tokens, (size_t)B * 4);
        CUINF_TRY(cudaMemcpyAsync(b->tok, b->pinned, (size_t)B * 4, cudaMemcpyHostToDevice, b->st));
    }
    CUINF_TRY(cudaGraphLaunch(b->exec, b->st));
    if (out_tokens) {
        CUINF_TRY(cudaMemcpyAsync(b->pinned + B, b->tok, (size_t)B * 4, cudaMemcpyDeviceToHost, b->st));
        BTRY(batch_sync(b));
        memcpy(out_tokens, b->pinned + B, (size_t)B * 4);
    }
    return CUINF_OK;
}

extern "C" int cuinf_batch_sync(cuinf_batch* b) {
    REQUIRE(b, "null batch");
    return batch_sync(b);
}

extern "C" int cuinf_batch_abort(cuinf_batch* b) {
    REQUIRE(b, "null batch");
    if (b->ep_world <= 1) return CUINF_OK;
    if (b->comm) ncclCommAbort(b->comm);
    b->comm = nullptr;
    b->ep_failed = true;
    return CUINF_OK;
}

extern "C" int cuinf_batch_set_timeout(cuinf_batch* b, int timeout_ms) {
    REQUIRE(b && timeout_ms > 0, "null batch or non-positive timeout");
    b->ep_timeout_ms = timeout_ms;
    return CUINF_OK;
}

extern "C" int cuinf_batch_failed(const cuinf_batch* b) { return b && b->ep_failed ? 1 : 0; }

extern "C" int cuinf_batch_ep_exchange(const cuinf_batch* b) {
    if (!b || b->ep_world <= 1) return -1;
    return b->p2p ? 1 : 0;
}
extern "C" int cuinf_batch_set_ep_exchange(cuinf_batch* b, int peer_memory) {
    REQUIRE(b && b->ep_world > 1, "not an expert-parallel batch");
    REQUIRE(!b->ep_failed, "expert-parallel batch was aborted");
    REQUIRE(!peer_memory || b->p2p_ok, "the peers' exchange arenas could not be mapped");
    if ((bool)peer_memory == b->p2p) return CUINF_OK;
    BTRY(batch_sync(b));
    b->p2p = peer_memory != 0;
    return batch_build_graph(b);
}

extern "C" int cuinf_batch_keep_logits(cuinf_batch* b, int on) {
    REQUIRE(b, "null batch");
    if ((bool)on == b->keep_logits) return CUINF_OK;
    CUINF_TRY(cudaStreamSynchronize(b->st));
    b->keep_logits = on != 0;
    return batch_build_graph(b);
}
extern "C" const float* cuinf_batch_logits(const cuinf_batch* b) { return b ? b->logits : nullptr; }
extern "C" int cuinf_batch_routes(cuinf_batch* b, int* idx) {
    REQUIRE(b && idx, "null pointer");
    const cuinf_config& c = b->m->cfg;
    const size_t n = (size_t)std::max(1, c.n_layers - c.n_dense) * b->B * c.top_k;
    CUINF_TRY(cudaStreamSynchronize(b->st));
    CUINF_TRY(cudaMemcpy(idx, b->ridx, n * 4, cudaMemcpyDeviceToHost));
    return CUINF_OK;
}
extern "C" int cuinf_batch_kernels_per_step(const cuinf_batch* b) { return b ? b->kernels : -1; }
extern "C" int cuinf_batch_error(unsigned* flags) {
    REQUIRE(flags, "null pointer");
    CUINF_TRY(cudaMemcpyFromSymbol(flags, g_tc_err, 4 * sizeof(unsigned)));
    return CUINF_OK;
}

extern "C" int cuinf_batch_fill_synthetic(cuinf_batch* b, int ctx, unsigned long long seed) {
    REQUIRE(b, "null batch");
    REQUIRE(ctx >= 0 && ctx < b->max_ctx, "ctx must be below max_ctx");
    REQUIRE(ctx % CUINF_KVGROUP == 0, "ctx must be a multiple of 64 (whole FP8 groups)");
    const cuinf_config& c = b->m->cfg;
    const int grid = 4 * b->num_sms;
    for (int l = 0; l < c.n_layers; l++) {
        if (!c.attn_layer[l]) continue;
        const AttnState& A = b->attn[l];
        for (int s = 0; s < b->B; s++) {
            const size_t n = (size_t)ctx * c.n_kv_heads * 64;
            if (n) {
                k_bfill<<<grid, 256, 0, b->st>>>(A.kc8 + s * b->kv8_seq, n, seed + 977ull * l + 131ull * s);
                k_bfill<<<grid, 256, 0, b->st>>>(A.vc8 + s * b->kv8_seq, n, seed + 977ull * l + 131ull * s + 7);
                const size_t ns = (size_t)(ctx / CUINF_KVGROUP) * c.n_kv_heads;
                k_bfill_scales<<<grid, 256, 0, b->st>>>(A.ksc + s * b->sc_seq, ns, 1.0f / 112.0f);
                k_bfill_scales<<<grid, 256, 0, b->st>>>(A.vsc + s * b->sc_seq, ns, 1.0f / 112.0f);
            }
        }
    }
    k_bset<<<(b->B + 127) / 128, 128, 0, b->st>>>(b->pos, b->B, ctx);
    CUINF_TRY(cudaGetLastError());
    CUINF_TRY(cudaStreamSynchronize(b->st));
    return CUINF_OK;
}

// Sequence `seq`'s own slices of the batch's stacked caches and conv states.
static void batch_seq_views(const cuinf_batch* b, int seq, std::vector<AttnState>& A, std::vector<__half*>& C) {
    const cuinf_config& c = b->m->cfg;
    A.assign(c.n_layers, AttnState());
    C.assign(c.n_layers, nullptr);
    for (int l = 0; l < c.n_layers; l++) {
        if (c.attn_layer[l]) {
            const AttnState& S = b->attn[l];
            A[l].kc8 = S.kc8 + seq * b->kv8_seq;
            A[l].vc8 = S.vc8 + seq * b->kv8_seq;
            A[l].ksc = S.ksc + seq * b->sc_seq;
            A[l].vsc = S.vsc + seq * b->sc_seq;
            A[l].ktail = S.ktail + seq * b->tail_seq;
            A[l].vtail = S.vtail + seq * b->tail_seq;
        } else {
            C[l] = b->conv_state[l] + (size_t)seq * 2 * c.hidden;
        }
    }
}

extern "C" size_t cuinf_batch_seq_state_bytes(cuinf_batch* b, int seq) {
    if (!b || seq < 0 || seq >= b->B) return 0;
    int pos = 0;
    if (cudaStreamSynchronize(b->st) != cudaSuccess ||
        cudaMemcpy(&pos, b->pos + seq, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return 0;
    return seq_state_bytes(b->m->cfg, pos);
}

extern "C" int cuinf_batch_save_seq(cuinf_batch* b, int seq, void* host, size_t n) {
    REQUIRE(b && host, "null pointer");
    REQUIRE(seq >= 0 && seq < b->B, "sequence index out of range");
    int pos = 0;
    CUINF_TRY(cudaStreamSynchronize(b->st));
    CUINF_TRY(cudaMemcpy(&pos, b->pos + seq, 4, cudaMemcpyDeviceToHost));
    std::vector<AttnState> A;
    std::vector<__half*> C;
    batch_seq_views(b, seq, A, C);
    return seq_state_copy(b->m->cfg, pos, A.data(), C.data(), host, n, true, b->st);
}

extern "C" int cuinf_batch_load_seq(cuinf_batch* b, int seq, const void* host, size_t n) {
    REQUIRE(b && host, "null pointer");
    REQUIRE(seq >= 0 && seq < b->B, "sequence index out of range");
    int pos = 0;
    int rc = seq_state_header(b->m->cfg, host, n, b->max_ctx, &pos);
    if (rc) return rc;
    CUINF_TRY(cudaStreamSynchronize(b->st));
    std::vector<AttnState> A;
    std::vector<__half*> C;
    batch_seq_views(b, seq, A, C);
    rc = seq_state_copy(b->m->cfg, pos, A.data(), C.data(), const_cast<void*>(host), n, false, b->st);
    if (rc) return rc;
    CUINF_TRY(cudaMemcpy(b->pos + seq, &pos, 4, cudaMemcpyHostToDevice));
    return CUINF_OK;
}

// One step launched eagerly with an event after every launch: ms[i] is the
// duration of launch i (names[i * name_len] its name).  Advances the batch
// like cuinf_batch_step(b, NULL, NULL).
extern "C" int cuinf_batch_profile_step(cuinf_batch* b, int max_kernels, float* ms, char* names, int name_len,
                                        int* n_kernels) {
    REQUIRE(b && ms && names && n_kernels && name_len > 0, "null pointer");
    CUINF_TRY(cudaStreamSynchronize(b->st));
    std::vector<std::pair<const char*, cudaEvent_t>> ev;
    cudaEvent_t e0;
    CUINF_TRY(cudaEventCreate(&e0));
    CUINF_TRY(cudaEventRecord(e0, b->st));
    BStep S{b, false};
    S.prof = &ev;
    S.trace = getenv("CUINF_BATCH_TRACE") != nullptr;
    int rc = batch_record(b, S);
    cudaError_t se = cudaStreamSynchronize(b->st);
    int n = 0;
    if (rc == CUINF_OK && se == cudaSuccess) {
        cudaEvent_t prev = e0;
        for (auto& pe : ev) {
            if (n < max_kernels) {
                cudaEventElapsedTime(&ms[n], prev, pe.second);
                snprintf(names + (size_t)n * name_len, name_len, "%s", pe.first);
                n++;
            }
            prev = pe.second;
        }
    }
    for (auto& pe : ev) cudaEventDestroy(pe.second);
    cudaEventDestroy(e0);
    if (rc) return rc;
    CUINF_TRY(se);
    *n_kernels = n;
    return CUINF_OK;
}

// ===========================================================================
// Grouped MoE for prefill: the S tokens of one prompt go through the same
// routing / grouped-GEMM / combine kernels as a decode batch, in chunks of up
// to PF_MOE_ROWS/top_k tokens: routed one warp per token, grouped by
// k_bgroup_many.
// ===========================================================================
struct TcCache {
    std::mutex mu;
    std::vector<CUtensorMap> hmaps;
    CUtensorMap* dmaps = nullptr;  // [n_moe][E][3]
    int chunk = 0;
    float *rlog = nullptr, *rw = nullptr, *fg = nullptr, *fu = nullptr, *fo = nullptr;
    int *inv = nullptr, *src = nullptr, *ridx = nullptr;
    __half *xg = nullptr, *mmid = nullptr;
    TcGroup *g13 = nullptr, *g2 = nullptr;
    CUtensorMap x_xg, x_mmid;
    std::vector<void*> allocs;
};

void tc_cache_free(cuinf_model* m) {
    TcCache* c = (TcCache*)m->tc_cache;
    if (!c) return;
    for (void* p : c->allocs) cudaFree(p);
    delete c;
    m->tc_cache = nullptr;
}

// (token, slot) rows per prefill MoE chunk: every expert's weights are read
// once per chunk, so larger chunks read them fewer times (4096 rows = 1024
// tokens at top-4 hold about 120 MB of gathered rows and expert outputs)
#define PF_MOE_ROWS 4096
static int tc_cache_get(cuinf_model* m, TcCache** out) {
    if (m->tc_cache) {
        *out = (TcCache*)m->tc_cache;
        return CUINF_OK;
    }
    const cuinf_config& c = m->cfg;
    REQUIRE(c.hidden % TC_KS == 0 && c.moe_inter % TC_KS == 0, "grouped MoE needs H and I multiples of 128");
    const int E = c.n_experts, K = c.top_k, H = c.hidden, I = c.moe_inter;
    const int n_moe = c.n_layers - c.n_dense;
    TcCache* tc = new TcCache();
    auto fail = [&](int rc) {
        for (void* p : tc->allocs) cudaFree(p);
        delete tc;
        return rc;
    };
    auto al = [&](void** p, size_t bytes) -> int {
        if (cudaMalloc(p, bytes) != cudaSuccess) return cuinf_set_arg_error("prefill scratch allocation failed");
        tc->allocs.push_back(*p);
        return CUINF_OK;
    };
    std::vector<void*> ex((size_t)n_moe * E * 6);
    if (cudaMemcpy(ex.data(), m->d_experts, ex.size() * sizeof(void*), cudaMemcpyDeviceToHost) != cudaSuccess)
        return fail(cuinf_set_arg_error("expert table copy failed"));
    for (size_t e = 0; e < (size_t)n_moe * E; e++) {
        CUtensorMap a, b, d;
        int rc = tc_map_int4(&a, (const uint8_t*)ex[e * 6 + 0], I, H);
        if (!rc) rc = tc_map_int4(&b, (const uint8_t*)ex[e * 6 + 2], I, H);
        if (!rc) rc = tc_map_int4(&d, (const uint8_t*)ex[e * 6 + 4], H, I);
        if (rc) return fail(rc);
        tc->hmaps.push_back(a);
        tc->hmaps.push_back(b);
        tc->hmaps.push_back(d);
    }
    int rc = al((void**)&tc->dmaps, tc->hmaps.size() * sizeof(CUtensorMap));
    if (rc) return fail(rc);
    if (cudaMemcpy(tc->dmaps, tc->hmaps.data(), tc->hmaps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice) !=
        cudaSuccess)
        return fail(cuinf_set_arg_error("tensor map upload failed"));
    const int C = PF_MOE_ROWS / K, R = C * K, maxch = (C + TC_NMAX - 1) / TC_NMAX;
    tc->chunk = C;
    if ((rc = al((void**)&tc->rlog, (size_t)C * E * 4)) || (rc = al((void**)&tc->rw, (size_t)R * 4)) ||
        (rc = al((void**)&tc->fg, (size_t)R * I * 4)) || (rc = al((void**)&tc->fu, (size_t)R * I * 4)) ||
        (rc = al((void**)&tc->fo, (size_t)R * H * 4)) || (rc = al((void**)&tc->inv, (size_t)R * 4)) ||
        (rc = al((void**)&tc->src, (size_t)R * 4)) || (rc = al((void**)&tc->ridx, (size_t)R * 4)) ||
        (rc = al((void**)&tc->xg, (size_t)R * H * 2)) || (rc = al((void**)&tc->mmid, (size_t)R * I * 2)) ||
        (rc = al((void**)&tc->g13, (size_t)2 * E * maxch * sizeof(TcGroup))) ||
        (rc = al((void**)&tc->g2, (size_t)E * maxch * sizeof(TcGroup))))
        return fail(rc);
    if ((rc = tc_map_act(&tc->x_xg, tc->xg, R, H, 16)) || (rc = tc_map_act(&tc->x_mmid, tc->mmid, R, I, 16)))
        return fail(rc);
    m->tc_cache = tc;
    *out = tc;
    return CUINF_OK;
}

int moe_grouped_prefill(cuinf_model* m, int layer, const __half* xn, __half* h, int S, int* ridx_out,
                        cudaStream_t st) {
    TcCache* tc = nullptr;
    int rc = tc_cache_get(m, &tc);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(tc->mu);
    rc = tc_attr_once();
    if (rc) return rc;
    const cuinf_config& c = m->cfg;
    const LayerW& L = m->L[layer];
    const int E = c.n_experts, K = c.top_k, H = c.hidden, I = c.moe_inter;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    for (int c0 = 0; c0 < S; c0 += tc->chunk) {
        const int n = std::min(tc->chunk, S - c0), maxch = (n + TC_NMAX - 1) / TC_NMAX;
        rc = cuinf_gemv_fp16(xn + (size_t)c0 * H, L.gate, tc->rlog, n, E, H, st);
        if (rc) return rc;
        BRouteParams R = {};
        R.logits = tc->rlog;
        R.bias = L.ebias;
        R.B = n;
        R.E = E;
        R.topk = K;
        R.I = I;
        R.H = H;
        R.maxch = maxch;
        R.ridx = ridx_out ? ridx_out + (size_t)c0 * K : tc->ridx;
        R.rw = tc->rw;
        R.keys = nullptr;
        R.n = n * K;
        R.n_local = E;
        R.group = 1;
        R.inv = tc->inv;
        R.src = tc->src;
        R.g13 = tc->g13;
        R.g2 = tc->g2;
        R.maps = tc->dmaps + (size_t)L.moe_index * E * 3;
        R.experts = (void* const*)(m->d_experts + (size_t)L.moe_index * E * 6);
        R.gbuf = tc->fg;
        R.ubuf = tc->fu;
        R.obuf = tc->fo;
        R.routed = 1;
        k_broute_tokens<<<(n + 7) / 8, 256, 0, st>>>(tc->rlog, L.ebias, n, E, K, R.ridx, R.rw);
        k_bgroup_many<<<1, 1024, 0, st>>>(R);
        k_bgather<<<n * K, 256, 0, st>>>(xn + (size_t)c0 * H, tc->src, tc->xg, H);
        if ((rc = cuinf_launch_status())) return rc;
        const int t13 = (I + TC_ROWS - 1) / TC_ROWS, t2 = (H + TC_ROWS - 1) / TC_ROWS;
        const int hit = std::min(E, n * K);
        for (int pass = 0; pass < 2; pass++) {
            const int ng = pass ? E * maxch : 2 * E * maxch, tiles = pass ? t2 : t13, Kd = pass ? I : H;
            TcPlan pl = tc_plan((pass ? 1 : 2) * hit * tiles, Kd, sms);
            float* ws = nullptr;
            unsigned* cnt = nullptr;
            if (pl.splits > 1 && (rc = tc_workspace((size_t)ng * tiles * pl.splits, (size_t)ng * tiles, &ws, &cnt)))
                return rc;
            TcParams P = {};
            P.groups = pass ? tc->g2 : tc->g13;
            P.n_groups = ng;
            P.K = Kd;
            P.splits = pl.splits;
            P.kg_per_split = pl.kgps;
            P.fp16_w = 0;
            P.xmax = (std::min(n, TC_NMAX) + 15) & ~15;  // a group holds at most one row per token
            P.xbox = 16;
            P.ws = ws;
            P.counters = cnt;
            if ((rc = tc_launch(pass ? tc->x_mmid : tc->x_xg, tc->hmaps[0], P, tiles, st, false))) return rc;
            if (!pass && (rc = cuinf_swiglu(tc->fg, tc->fu, tc->mmid, n * K * I, st))) return rc;
        }
        k_bcombine<<<(n * H + 255) / 256, 256, 0, st>>>(tc->fo, tc->inv, tc->rw, h + (size_t)c0 * H, n, H, K,
                                                         EpWait{});
        if ((rc = cuinf_launch_status())) return rc;
    }
    return CUINF_OK;
}
