// Decode engine: model (one device blob in the tools/export_weights.py
// layout), session (KV cache, conv state, activations) and the per-token
// launch chain, captured once as a CUDA graph.  Host orchestration of the
// reference: main() in src/engine.cu:637-975 (load 664-692, buffers 711-770,
// layer_forward 784-908, logits 932-940, decode loop 954-963).
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <functional>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "attn.cuh"
#include "engine_kernels.cuh"
#include "megakernel.cuh"
#include "model.h"
#include "moe_fused.cuh"

#define REQUIRE(cond, msg) \
    do {                   \
        if (!(cond)) return cuinf_set_arg_error(msg); \
    } while (0)
#define ST(s) ((cudaStream_t)(s))

// ---------------------------------------------------------------------------
// standalone flash-decoding attention (attn_decode_split/combine, 396-480)
// ---------------------------------------------------------------------------
static int current_sms() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return 148;
    return sms;
}

extern "C" size_t cuinf_attn_decode_workspace_size(int nh, int nkv, int max_ctx) {
    if (nh <= 0 || nkv <= 0 || max_ctx <= 0) return 0;
    int units = (max_ctx + CUINF_KVGROUP - 1) / CUINF_KVGROUP + 1;
    int ns = attn_default_nsplit(nkv, nh / nkv, units, current_sms());
    return (size_t)nkv * ns * (nh / nkv) * ATTN_PART_STRIDE * 4 + 256;
}

// Library-owned scratch for calls that pass no workspace, one buffer per
// device ordinal and kind (grown on demand; zero-filled when allocated).  A
// kernel that needs zeroed words (tickets, accumulators) leaves them zero.
// Growing waits for the whole device, so no launch still uses the old buffer.
#define WS_MAX_DEVICES 64
enum { WS_ATTN = 0, WS_MOE = 1, WS_KINDS = 2 };
static std::mutex g_ws_mu;
static void* g_ws[WS_KINDS][WS_MAX_DEVICES];
static size_t g_ws_bytes[WS_KINDS][WS_MAX_DEVICES];

static int shared_workspace(int kind, size_t need, void** out) {
    int dev = 0;
    CUINF_TRY(cudaGetDevice(&dev));
    REQUIRE(dev >= 0 && dev < WS_MAX_DEVICES, "device ordinal beyond the library's table");
    std::lock_guard<std::mutex> lk(g_ws_mu);
    void*& p = g_ws[kind][dev];
    size_t& have = g_ws_bytes[kind][dev];
    if (have < need) {
        if (p) {
            CUINF_TRY(cudaDeviceSynchronize());
            CUINF_TRY(cudaFree(p));
            p = nullptr;
            have = 0;
        }
        CUINF_TRY(cudaMalloc(&p, need));
        CUINF_TRY(cudaMemset(p, 0, need));
        have = need;
    }
    *out = p;
    return CUINF_OK;
}

extern "C" int cuinf_attn_decode(const void* q, const uint8_t* kc8, const uint8_t* vc8,
                                 const void* ksc, const void* vsc, const void* ktail,
                                 const void* vtail, int committed, int qpos, float scale, void* out,
                                 int nh, int nkv, void* workspace, size_t workspace_bytes,
                                 void* stream) {
    REQUIRE(q && ktail && vtail && out, "null pointer");
    REQUIRE(nh > 0 && nkv > 0 && nkv <= 64 && nh % nkv == 0 && nh / nkv <= 8,
            "need nkv <= 64, nh % nkv == 0, nh/nkv <= 8");
    REQUIRE(qpos >= 0 && committed >= 0 && committed % CUINF_KVGROUP == 0, "committed % 64 == 0");
    REQUIRE(committed <= qpos + 1 && qpos + 1 - committed <= CUINF_KVGROUP,
            "tail length must be in [0, 64]");
    REQUIRE(committed == 0 || (kc8 && vc8 && ksc && vsc), "null FP8 cache");
    REQUIRE(((uintptr_t)ktail & 15) == 0 && ((uintptr_t)vtail & 15) == 0 &&
                ((uintptr_t)kc8 & 15) == 0 && ((uintptr_t)vc8 & 15) == 0 && ((uintptr_t)q & 3) == 0,
            "cache pointers must be 16-byte aligned");
    const int units = committed / CUINF_KVGROUP + (qpos + 1 > committed ? 1 : 0);
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int ns = attn_default_nsplit(nkv, nh / nkv, units, sms);
    const size_t need = (size_t)nkv * ns * (nh / nkv) * ATTN_PART_STRIDE * 4 + 256;
    void* ws = workspace;
    if (!ws) {
        int rc = shared_workspace(WS_ATTN, need, &ws);
        if (rc) return rc;
    } else {
        REQUIRE(workspace_bytes >= need, "workspace too small");
        REQUIRE(((uintptr_t)ws & 15) == 0, "workspace must be 16-byte aligned");
    }
    AttnParams P;
    P.q = (const __half*)q;
    P.kc8 = kc8;
    P.vc8 = vc8;
    P.ksc = (const __half*)ksc;
    P.vsc = (const __half*)vsc;
    P.ktail = (const __half*)ktail;
    P.vtail = (const __half*)vtail;
    P.pos_dev = nullptr;
    P.committed = committed;
    P.qpos = qpos;
    P.scale = scale;
    P.out = (__half*)out;
    P.counters = (unsigned*)ws;
    P.part = (float*)((char*)ws + 256);
    P.nh = nh;
    P.nkv = nkv;
    P.nsplit = ns;
    P.next.count = 0;
    if (workspace) CUINF_TRY(cudaMemsetAsync(ws, 0, 256, ST(stream)));
    k_attn_decode<2><<<dim3(nkv, ns), ATTN_THREADS, 0, ST(stream)>>>(P);
    return cuinf_launch_status();
}

// Batched form for the sequence-batched engine (batch.cu).
// Splits per (sequence, kv head): about two CTAs per SM over the whole batch,
// never more than the single-sequence engine uses at this context.
int attn_batched_nsplit(int nh, int nkv, int max_ctx, int n_seqs, int num_sms) {
    const int cap = attn_engine_nsplit(nh / nkv, (max_ctx + CUINF_KVGROUP - 1) / CUINF_KVGROUP);
    const int want = (2 * num_sms + n_seqs * nkv - 1) / (n_seqs * nkv);
    return std::max(1, std::min(cap, want));
}
size_t attn_batched_part_floats(int nh, int nkv, int nsplit) {
    return (size_t)nkv * nsplit * (nh / nkv) * ATTN_PART_STRIDE;
}
int attn_decode_batched(const BatchAttnArgs& a, cudaStream_t st) {
    AttnParams P;
    P.q = a.q;
    P.kc8 = a.kc8;
    P.vc8 = a.vc8;
    P.ksc = a.ksc;
    P.vsc = a.vsc;
    P.ktail = a.ktail;
    P.vtail = a.vtail;
    P.pos_dev = a.pos;
    P.committed = 0;
    P.qpos = 0;
    P.scale = a.scale;
    P.out = a.out;
    P.part = a.part;
    P.counters = a.counters;
    P.nh = a.nh;
    P.nkv = a.nkv;
    P.nsplit = a.nsplit;
    P.next.count = 0;
    P.bq = a.bq;
    P.bkv8 = a.bkv8;
    P.bsc = a.bsc;
    P.btail = a.btail;
    P.bout = a.bout;
    P.bpart = a.bpart;
    // two CTAs per SM: the batch's many (sequence, kv head) CTAs keep more
    // K/V requests in flight (64 sequences at 2048: 103 -> 73 us per layer)
    k_attn_decode<2><<<dim3(a.nkv, a.nsplit, a.n_seqs), ATTN_THREADS, 0, st>>>(P);
    return cuinf_launch_status();
}

// ---------------------------------------------------------------------------
// attention with library-static scratch: a variant for callers that may not
// allocate device memory at all (an allocator hook that re-enters this
// library, a pool that forbids cudaMalloc, or a caller that pre-reserves all
// HBM).  The split-K partials and tickets live in one file-scope __device__
// array; its address is taken once per device at set-up.
// ---------------------------------------------------------------------------
#define ATTN_STATIC_SCRATCH_BYTES (512u << 10)  // 256 B of tickets + partials
#define ATTN_STATIC_MAX_DEVICES 64

static __device__ __align__(256) unsigned char g_attn_static_scratch[ATTN_STATIC_SCRATCH_BYTES];

static std::mutex g_static_mu;
static void* g_static_ptr[ATTN_STATIC_MAX_DEVICES];
static int g_static_sms[ATTN_STATIC_MAX_DEVICES];

// Address of g_attn_static_scratch and the SM count on the current device.
// The first call on a device resolves the symbol (module load, no allocation);
// later calls only read the cached table.
static int static_scratch(void** ptr, int* sms) {
    int dev = 0;
    CUINF_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= ATTN_STATIC_MAX_DEVICES)
        return cuinf_set_arg_error("device ordinal beyond the static scratch table");
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (!g_static_ptr[dev]) {
        void* p = nullptr;
        int n = 0;
        CUINF_TRY(cudaGetSymbolAddress(&p, g_attn_static_scratch));
        CUINF_TRY(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
        if (!p || ((uintptr_t)p & 255)) return cuinf_set_arg_error("static scratch misaligned");
        g_static_sms[dev] = n;
        g_static_ptr[dev] = p;
    }
    *ptr = g_static_ptr[dev];
    *sms = g_static_sms[dev];
    return CUINF_OK;
}

extern "C" size_t cuinf_attn_decode_static_scratch_bytes(void) { return ATTN_STATIC_SCRATCH_BYTES; }

extern "C" int cuinf_attn_decode_noalloc(const void* q, const uint8_t* kc8, const uint8_t* vc8,
                                         const void* ksc, const void* vsc, const void* ktail,
                                         const void* vtail, int committed, int qpos, float scale,
                                         void* out, int nh, int nkv, void* stream) {
    REQUIRE(q && ktail && vtail && out, "null pointer");
    REQUIRE(nh > 0 && nkv > 0 && nkv <= 64 && nh % nkv == 0 && nh / nkv <= 8,
            "need nkv <= 64, nh % nkv == 0, nh/nkv <= 8");
    REQUIRE(qpos >= 0 && committed >= 0 && committed % CUINF_KVGROUP == 0, "committed % 64 == 0");
    REQUIRE(committed <= qpos + 1 && qpos + 1 - committed <= CUINF_KVGROUP,
            "tail length must be in [0, 64]");
    REQUIRE(committed == 0 || (kc8 && vc8 && ksc && vsc), "null FP8 cache");
    REQUIRE(((uintptr_t)ktail & 15) == 0 && ((uintptr_t)vtail & 15) == 0 &&
                ((uintptr_t)kc8 & 15) == 0 && ((uintptr_t)vc8 & 15) == 0 && ((uintptr_t)q & 3) == 0,
            "cache pointers must be 16-byte aligned");
    void* ws = nullptr;
    int sms = 0;
    int rc = static_scratch(&ws, &sms);
    if (rc) return rc;
    const int units = committed / CUINF_KVGROUP + (qpos + 1 > committed ? 1 : 0);
    const int ns = attn_default_nsplit(nkv, nh / nkv, units, sms);
    const size_t need = (size_t)nkv * ns * (nh / nkv) * ATTN_PART_STRIDE * 4 + 256;
    if (need > ATTN_STATIC_SCRATCH_BYTES)
        return cuinf_set_arg_error(
            "cuinf_attn_decode_noalloc: split-K partials exceed the 512 KiB static scratch; "
            "use cuinf_attn_decode with a workspace");
    AttnParams P;
    P.q = (const __half*)q;
    P.kc8 = kc8;
    P.vc8 = vc8;
    P.ksc = (const __half*)ksc;
    P.vsc = (const __half*)vsc;
    P.ktail = (const __half*)ktail;
    P.vtail = (const __half*)vtail;
    P.pos_dev = nullptr;
    P.committed = committed;
    P.qpos = qpos;
    P.scale = scale;
    P.out = (__half*)out;
    P.counters = (unsigned*)ws;
    P.part = (float*)((char*)ws + 256);
    P.nh = nh;
    P.nkv = nkv;
    P.nsplit = ns;
    P.next.count = 0;
    // The per-kv-head tickets must read zero when the kernel starts.  The array
    // is zero at module load and every completed launch returns its tickets to
    // zero; clearing them here on the stream (a memset, no allocation) also
    // covers a launch that an earlier error cut short.
    CUINF_TRY(cudaMemsetAsync(ws, 0, 256, ST(stream)));
    k_attn_decode<2><<<dim3(nkv, ns), ATTN_THREADS, 0, ST(stream)>>>(P);
    return cuinf_launch_status();
}

// ---------------------------------------------------------------------------
// standalone fused MoE FFN for one token (engine.cu:877-905)
// ---------------------------------------------------------------------------
// Launch with programmatic stream serialization (PDL) when pdl is set: the
// kernel may start while its predecessor runs and orders itself with
// griddepcontrol.wait before touching its predecessor's outputs.
template <typename Kern, typename Par>
static cudaError_t launch_k(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                            const Par& params) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, params);
}

// Same, with thread-block clusters of cluster_x CTAs along x.
template <typename Kern, typename Par>
static cudaError_t launch_kc(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                             int cluster_x, const Par& params) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster_x;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, params);
}

// Same, with thread-block clusters of cluster_y CTAs along y.
template <typename Kern, typename Par>
static cudaError_t launch_kcy(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                              int cluster_y, const Par& params) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = cluster_y;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, params);
}

// Largest cluster (<= 16 CTAs, one per split) with which the decode
// attention's nkv clusters all fit on the device at once; 0 if none.
static int attn_cluster_size(int nkv, int nsplit) {
    const int cl = std::min(nsplit, 16);
    if (cl < 2) return 0;
    if (cl > 8 && cudaFuncSetAttribute(k_attn_decode<1>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nkv, cl);
    cfg.blockDim = dim3(ATTN_THREADS);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = cl;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, k_attn_decode<1>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n >= nkv ? cl : 0;
}

static int set_kernel_attrs(const cuinf_config& c);

// Dynamic shared memory for a kernel whose grid fits on the SMs and whose
// CTAs should each hold an SM alone: more than half of the SM's 228 KB, so
// no second CTA of the kernel fits.  A launch that follows another kernel
// (programmatic dependent launch) otherwise gets its CTAs packed 2-3 to an
// SM on whichever SMs have room at that moment, and the per-CTA dot
// (dequantize + mma.sync, bound by the SM's issue rate) then runs 2-3 times
// in sequence there while other SMs idle.  Used for k_conv_in and
// k_gemv_residual (128 CTAs each at H = 2048).
#define ONE_PER_SM_SMEM ((size_t)116 * 1024)
static inline size_t one_per_sm(size_t bytes, int grid, int sms) {
    return grid <= sms ? std::max(bytes, ONE_PER_SM_SMEM) : bytes;
}

// k_moe_up + k_moe_down for one token: xn already normalized, h += the
// rank-ordered expert mix; mid [topk*I] fp16 and the routes are scratch.
static int moe_ffn_launch(const __half* xn, const __half* gate, const __half* bias, const void* const* experts,
                          __half* h, int H, int I, int n_exp, int topk, __half* mid, int* ridx, float* rw,
                          cudaStream_t st) {
    MoeUpParams U;
    U.h = nullptr;
    U.xn = xn;
    U.norm_w = nullptr;
    U.gate = gate;
    U.bias = bias;
    U.experts = experts;
    U.mid = mid;
    U.route_idx = ridx;
    U.route_w = rw;
    U.H = H;
    U.I = I;
    U.E = n_exp;
    U.topk = topk;
    U.eps = 0.f;
    U.next.count = 0;
    const size_t su = moe_up_smem(H, n_exp);
    REQUIRE(su <= 227 * 1024 && moe_down_smem(I, topk) <= 227 * 1024, "H/I too large for shared memory");
    if (su > 48 * 1024)
        CUINF_TRY(cudaFuncSetAttribute(k_moe_up, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)su));
    const int tiles = I / 16;
    const int grid_up = ((topk * tiles + 7) / 8) * 8;
    k_moe_up<<<grid_up, 256, su, st>>>(U);
    int rc = cuinf_launch_status();
    if (rc) return rc;
    MoeDownParams D;
    D.mid = mid;
    D.experts = experts;
    D.route_idx = ridx;
    D.route_w = rw;
    D.h = h;
    D.H = H;
    D.I = I;
    D.topk = topk;
    D.next.count = 0;
    const size_t sd = moe_down_smem(I, topk);
    if (sd > 48 * 1024)
        CUINF_TRY(cudaFuncSetAttribute(k_moe_down, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sd));
    CUINF_TRY(launch_kc(k_moe_down, dim3((H / 16) * topk), dim3(256), sd, st, false, topk, D));
    return cuinf_launch_status();
}

// Workspace of cuinf_moe_ffn: [0, 256) tickets, then the fused kernel's
// fixed-point accumulators [topk][H], then mid [topk][I] and the routes of
// the two-kernel form.  The first 256 + topk*H*8 bytes must be zero before the
// first call; every call leaves them zero.
extern "C" size_t cuinf_moe_ffn_workspace_size(int H, int I, int topk) {
    if (H <= 0 || I <= 0 || topk <= 0) return 0;
    return 256 + (size_t)topk * H * 8 + (size_t)topk * I * 2 + 256;
}

extern "C" int cuinf_moe_ffn(const void* xn, const void* gate, const void* expert_bias,
                             const void* const* experts, void* h, int H, int I, int n_exp, int topk,
                             int* idx, float* w, void* workspace, size_t workspace_bytes,
                             void* stream) {
    REQUIRE(xn && gate && expert_bias && experts && h, "null pointer");
    REQUIRE(H > 0 && H % 128 == 0 && I > 0 && I % 128 == 0, "H and I must be multiples of 128");
    REQUIRE(n_exp > 0 && n_exp <= 256 && topk > 0 && topk <= 8 && topk <= n_exp,
            "n_exp <= 256, topk <= 8");
    const size_t need = cuinf_moe_ffn_workspace_size(H, I, topk);
    void* ws = workspace;
    if (!ws) {
        int rc = shared_workspace(WS_MOE, need, &ws);
        if (rc) return rc;
    } else {
        REQUIRE(workspace_bytes >= need, "workspace too small (cuinf_moe_ffn_workspace_size)");
        REQUIRE(((uintptr_t)ws & 15) == 0, "workspace must be 16-byte aligned");
    }
    unsigned* tickets = (unsigned*)ws;
    unsigned long long* acc = (unsigned long long*)((char*)ws + 256);
    __half* mid = (__half*)((char*)ws + 256 + (size_t)topk * H * 8);
    char* rbuf = (char*)mid + (size_t)topk * I * 2;
    int* ridx = idx ? idx : (int*)rbuf;
    float* rw = w ? w : (float*)(rbuf + 128);
    {   // TMA / async-copy sources must be 16-byte aligned
        std::vector<uintptr_t> tab((size_t)n_exp * 6);
        CUINF_TRY(cudaMemcpy(tab.data(), experts, tab.size() * sizeof(uintptr_t), cudaMemcpyDeviceToHost));
        for (uintptr_t a : tab) REQUIRE(a && (a & 15) == 0, "expert tensors must be 16-byte aligned");
    }
    if (moef_supported(H, I, n_exp, topk) && ((uintptr_t)expert_bias & 15) == 0) {
        MoeFusedParams F;
        F.h = (const __half*)h;
        F.xn = (const __half*)xn;
        F.h_out = (__half*)h;
        F.norm_w = nullptr;
        F.gate = (const __half*)gate;
        F.bias = (const __half*)expert_bias;
        F.experts = experts;
        F.route_idx = ridx;
        F.route_w = rw;
        F.acc = acc;
        F.tickets = tickets;
        F.H = H;
        F.I = I;
        F.E = n_exp;
        F.topk = topk;
        F.eps = 0.f;
        F.next.count = 0;
        const size_t sm = moef_layout(H, n_exp).total;
        CUINF_TRY(cudaFuncSetAttribute(k_moe_fused, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
        k_moe_fused<<<topk * (I / 16), MOEF_THREADS, sm, ST(stream)>>>(F);
        return cuinf_launch_status();
    }
    return moe_ffn_launch((const __half*)xn, (const __half*)gate, (const __half*)expert_bias, experts,
                          (__half*)h, H, I, n_exp, topk, mid, ridx, rw, ST(stream));
}

// ---------------------------------------------------------------------------
// model
// ---------------------------------------------------------------------------
extern "C" void cuinf_default_config(cuinf_config* c) {
    memset(c, 0, sizeof(*c));
    c->hidden = 2048;
    c->n_layers = 24;
    c->n_heads = 32;
    c->n_kv_heads = 8;
    c->head_dim = 64;
    c->vocab = 128000;
    c->n_dense = 2;
    c->n_experts = 32;
    c->top_k = 4;
    c->moe_inter = 1792;
    c->dense_inter = 7168;
    c->conv_k = 3;
    c->rope_theta = 5000000.0f;
    c->norm_eps = 1e-5f;
    const int attn[] = {2, 6, 10, 14, 18, 21};  // ATTN_LAYER, engine.cu:50
    for (int i : attn) c->attn_layer[i] = 1;
}

static int parse_index(cuinf_model* m, const uint8_t* b, size_t len) {
    size_t p = 0;
    uint32_t n;
    if (len < 4) return cuinf_set_arg_error("index.bin truncated");
    memcpy(&n, b, 4);
    p = 4;
    for (uint32_t i = 0; i < n; i++) {
        if (p + 1 > len) return cuinf_set_arg_error("index.bin truncated");
        uint8_t nl = b[p++];
        if (p + nl + 1 + 40 > len) return cuinf_set_arg_error("index.bin truncated");
        std::string name((const char*)b + p, nl);
        p += nl;
        TDesc t;
        t.kind = b[p++];
        memcpy(&t.offset, b + p, 8); p += 8;
        memcpy(&t.packed, b + p, 8); p += 8;
        memcpy(&t.scales, b + p, 8); p += 8;
        memcpy(&t.d0, b + p, 8); p += 8;
        memcpy(&t.d1, b + p, 8); p += 8;
        m->idx[name] = t;
    }
    return CUINF_OK;
}

namespace {
struct Resolver {
    cuinf_model* m;
    std::string err;
    const TDesc* get(const std::string& n, int kind, int64_t d0, int64_t d1) {
        auto it = m->idx.find(n);
        if (it == m->idx.end()) { if (err.empty()) err = "missing tensor " + n; return nullptr; }
        const TDesc& t = it->second;
        if (t.kind != kind) { if (err.empty()) err = "wrong kind for " + n; return nullptr; }
        if (t.d0 != d0 || t.d1 != d1) {
            if (err.empty())
                err = "shape mismatch for " + n + ": got [" + std::to_string(t.d0) + "," +
                      std::to_string(t.d1) + "] want [" + std::to_string(d0) + "," + std::to_string(d1) + "]";
            return nullptr;
        }
        if (t.offset + t.packed + t.scales > m->blob_bytes) {
            if (err.empty()) err = "tensor " + n + " beyond weights.bin";
            return nullptr;
        }
        if (t.offset % 16 != 0 || (kind == 1 && (t.offset + t.packed) % 4 != 0)) {
            if (err.empty()) err = "tensor " + n + " not 16-byte aligned";
            return nullptr;
        }
        if (kind == 1 && (t.packed != (uint64_t)(d0 * d1 / 2) || t.scales != (uint64_t)(d0 * (d1 / 128) * 2))) {
            if (err.empty()) err = "bad INT4 sizes for " + n;
            return nullptr;
        }
        return &t;
    }
    const __half* f16(const std::string& n, int64_t d0, int64_t d1 = 0) {
        const TDesc* t = get(n, 0, d0, d1);
        return t ? (const __half*)(m->d_blob + t->offset) : nullptr;
    }
    Q4 q4(const std::string& n, int64_t N, int64_t K) {
        Q4 w;
        const TDesc* t = get(n, 1, N, K);
        if (t) {
            w.p = m->d_blob + t->offset;
            w.s = (const __half*)(m->d_blob + t->offset + t->packed);
        }
        return w;
    }
};
}  // namespace

static int check_config(const cuinf_config* c) {
    REQUIRE(c->head_dim == 64, "head_dim must be 64");
    REQUIRE(c->hidden > 0 && c->hidden % 128 == 0 && c->hidden <= 16384, "hidden % 128 == 0");
    REQUIRE(c->n_layers > 0 && c->n_layers <= 64, "1 <= n_layers <= 64");
    REQUIRE(c->n_heads > 0 && c->n_kv_heads > 0 && c->n_heads % c->n_kv_heads == 0 &&
                c->n_heads / c->n_kv_heads <= 8, "GQA group must divide and be <= 8");
    REQUIRE(c->vocab > 0, "vocab > 0");
    REQUIRE(c->n_dense >= 0 && c->n_dense <= c->n_layers, "n_dense");
    REQUIRE(c->n_dense == c->n_layers || (c->n_experts > 0 && c->n_experts <= 256 &&
                                          c->top_k > 0 && c->top_k <= 8 && c->top_k <= c->n_experts),
            "n_experts <= 256, top_k <= 8");
    REQUIRE(c->moe_inter % 128 == 0 && c->dense_inter % 128 == 0, "inter sizes % 128 == 0");
    REQUIRE(c->conv_k == 3, "conv kernel size must be 3");
    return CUINF_OK;
}

static int resolve_model(cuinf_model* m) {
    const cuinf_config& c = m->cfg;
    const int H = c.hidden, hd = c.head_dim;
    Resolver R{m, ""};
    m->embed = R.f16("model.embed_tokens.weight", c.vocab, H);
    m->emb_norm = R.f16("model.embedding_norm.weight", H);
    m->L.assign(c.n_layers, LayerW());
    std::vector<void*> table;
    for (int l = 0; l < c.n_layers; l++) {
        LayerW& L = m->L[l];
        const std::string p = "model.layers." + std::to_string(l) + ".";
        L.op_norm = R.f16(p + "operator_norm.weight", H);
        L.ffn_norm = R.f16(p + "ffn_norm.weight", H);
        if (c.attn_layer[l]) {
            L.wq = R.q4(p + "self_attn.q_proj.weight", c.n_heads * hd, H);
            L.wk = R.q4(p + "self_attn.k_proj.weight", c.n_kv_heads * hd, H);
            L.wv = R.q4(p + "self_attn.v_proj.weight", c.n_kv_heads * hd, H);
            L.wo = R.q4(p + "self_attn.out_proj.weight", H, c.n_heads * hd);
            L.q_ln = R.f16(p + "self_attn.q_layernorm.weight", hd);
            L.k_ln = R.f16(p + "self_attn.k_layernorm.weight", hd);
        } else {
            L.in_proj = R.q4(p + "conv.in_proj.weight", 3 * H, H);
            L.out_proj = R.q4(p + "conv.out_proj.weight", H, H);
            L.conv_w = R.f16(p + "conv.conv.weight", H, 3);
        }
        if (l < c.n_dense) {
            L.w1 = R.q4(p + "feed_forward.w1.weight", c.dense_inter, H);
            L.w3 = R.q4(p + "feed_forward.w3.weight", c.dense_inter, H);
            L.w2 = R.q4(p + "feed_forward.w2.weight", H, c.dense_inter);
        } else {
            L.gate = R.f16(p + "feed_forward.gate.weight", c.n_experts, H);
            L.ebias = R.f16(p + "feed_forward.expert_bias", c.n_experts);
            L.moe_index = m->n_moe++;
            for (int e = 0; e < c.n_experts; e++) {
                const std::string ep = p + "feed_forward.experts." + std::to_string(e) + ".";
                Q4 a = R.q4(ep + "w1.weight", c.moe_inter, H);
                Q4 b = R.q4(ep + "w3.weight", c.moe_inter, H);
                Q4 d = R.q4(ep + "w2.weight", H, c.moe_inter);
                table.push_back((void*)a.p); table.push_back((void*)a.s);
                table.push_back((void*)b.p); table.push_back((void*)b.s);
                table.push_back((void*)d.p); table.push_back((void*)d.s);
            }
        }
    }
    if (!R.err.empty()) return cuinf_set_arg_error(R.err.c_str());
    if (!table.empty()) {
        CUINF_TRY(cudaMalloc(&m->d_experts, table.size() * sizeof(void*)));
        CUINF_TRY(cudaMemcpy(m->d_experts, table.data(), table.size() * sizeof(void*),
                             cudaMemcpyHostToDevice));
    }
    return CUINF_OK;
}

extern "C" int cuinf_model_from_device_blob(const cuinf_config* cfg, void* d_blob, size_t blob_bytes,
                                            const uint8_t* index, size_t index_bytes,
                                            cuinf_model** out) {
    REQUIRE(d_blob && index && out, "null pointer");
    cuinf_config c;
    if (cfg) c = *cfg; else cuinf_default_config(&c);
    int rc = check_config(&c);
    if (rc) return rc;
    cuinf_model* m = new cuinf_model();
    m->cfg = c;
    m->d_blob = (uint8_t*)d_blob;
    m->blob_bytes = blob_bytes;
    rc = parse_index(m, index, index_bytes);
    if (!rc) rc = resolve_model(m);
    if (rc) { cuinf_model_free(m); return rc; }
    *out = m;
    return CUINF_OK;
}

static int read_file(const std::string& path, std::vector<uint8_t>& buf) {
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) { cuinf_set_arg_error(("cannot open " + path).c_str()); return CUINF_ERR_IO; }
    fseek(f, 0, SEEK_END);
    long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    buf.resize((size_t)sz);
    size_t r = fread(buf.data(), 1, (size_t)sz, f);
    fclose(f);
    if (r != (size_t)sz) { cuinf_set_arg_error(("short read " + path).c_str()); return CUINF_ERR_IO; }
    return CUINF_OK;
}

extern "C" int cuinf_model_load(const char* dir, const cuinf_config* cfg, cuinf_model** out) {
    REQUIRE(dir && out, "null pointer");
    std::vector<uint8_t> index;
    int rc = read_file(std::string(dir) + "/index.bin", index);
    if (rc) return rc;
    const std::string wp = std::string(dir) + "/weights.bin";
    FILE* f = fopen(wp.c_str(), "rb");
    if (!f) { cuinf_set_arg_error(("cannot open " + wp).c_str()); return CUINF_ERR_IO; }
    fseek(f, 0, SEEK_END);
    size_t sz = (size_t)ftell(f);
    fseek(f, 0, SEEK_SET);
    uint8_t* d = nullptr;
    cudaError_t e = cudaMalloc(&d, sz);
    if (e != cudaSuccess) { fclose(f); return cuinf_set_cuda_error(e); }
    const size_t chunk = 256ull << 20;  // the reference uploads in 256 MB chunks too
    uint8_t* host = nullptr;
    e = cudaMallocHost(&host, chunk);
    if (e != cudaSuccess) { fclose(f); cudaFree(d); return cuinf_set_cuda_error(e); }
    size_t done = 0;
    while (done < sz) {
        size_t n = fread(host, 1, std::min(chunk, sz - done), f);
        if (n == 0) break;
        e = cudaMemcpy(d + done, host, n, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) break;
        done += n;
    }
    fclose(f);
    cudaFreeHost(host);
    if (e != cudaSuccess) { cudaFree(d); return cuinf_set_cuda_error(e); }
    if (done != sz) { cudaFree(d); cuinf_set_arg_error("short read of weights.bin"); return CUINF_ERR_IO; }
    rc = cuinf_model_from_device_blob(cfg, d, sz, index.data(), index.size(), out);
    if (rc) { cudaFree(d); return rc; }
    (*out)->own_blob = true;
    return CUINF_OK;
}

extern "C" int cuinf_model_free(cuinf_model* m) {
    if (!m) return CUINF_OK;
    tc_cache_free(m);
    if (m->d_experts) cudaFree(m->d_experts);
    if (m->own_blob && m->d_blob) cudaFree(m->d_blob);
    delete m;
    return CUINF_OK;
}

// ---------------------------------------------------------------------------
// session
// ---------------------------------------------------------------------------

struct cuinf_session {
    cuinf_model* m = nullptr;
    int max_ctx = 0;
    cudaStream_t st = nullptr;
    bool own_stream = false;
    std::vector<void*> allocs;
    __half *h = nullptr, *q = nullptr, *attn_out = nullptr, *conv_y = nullptr, *mid = nullptr,
           *hidden = nullptr;
    int *pos = nullptr, *tok = nullptr, *route_idx = nullptr, *out_ring = nullptr;
    float *route_w = nullptr, *logits = nullptr, *attn_part = nullptr;
    unsigned* attn_cnt = nullptr;
    unsigned long long* am_key = nullptr;
    unsigned* am_ticket = nullptr;
    std::vector<AttnState> attn;
    std::vector<__half*> conv_state;
    int nsplit = 1;
    int kernels_per_step = 0;
    bool keep_logits = false;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    // Pinned staging for the per-step token copies: input tokens go through a
    // ring of slots, each reused only after the event of its last copy
    // (asynchronous steps may be queued far ahead of the device).
    static const int kTokRing = 64;
    int* pinned = nullptr;  // [0, kTokRing) token in, [kTokRing] token out
    cudaEvent_t tok_ev[kTokRing] = {};
    int tok_slot = 0;
    int host_pos = 0;
    int num_sms = 148;
    int attn_cluster = 0;        // cluster size of the DSMEM split merge (0: not available)
    bool attn_use_cluster = true;  // CUINF_OPT_ATTN_CLUSTER
    bool prefetch = true;  // L2 prefetch plans (cross-kernel weight streaming)
    int prefetch_mb = 12;     // CUINF_OPT_PREFETCH_MB: bytes a kernel prefetches for the next ones
    int prefetch_ahead = 3;   // CUINF_OPT_PREFETCH_AHEAD: how many launches ahead it looks
    bool pdl = true;       // programmatic dependent launch between the step's kernels
    bool prefill = true;   // cuinf_generate prefills its prompt
    // persistent megakernel (one cooperative launch per step)
    bool mk_ok = false, use_mk = false;  // the multi-kernel graph is the default
    MkParams mk;
    size_t mk_smem = 0;
    int mk_grid = 0;
    unsigned* mk_words = nullptr;  // [0] gbar [1] abort [2] err [3] lm_tick [4..6] failure info
    unsigned long long* mk_trace = nullptr;  // per-stage timestamps when tracing is on
    bool trace = false;
    std::vector<int> mk_kinds;  // stage kinds, for trace reports
    // prefill scratch, grown to the longest prompt seen (freed with the session)
    int pf_cap = 0;
    void* pf_buf = nullptr;
    // H2O eviction mode (0 slots = off): per attention layer C per-token FP8 slots
    int h2o_C = 0, h2o_W = 0;
    struct H2o {
        uint8_t *hk8 = nullptr, *hv8 = nullptr;
        __half *hks = nullptr, *hvs = nullptr;
        int* slot_pos = nullptr;
        float* attn_sum = nullptr;
        int* n_live = nullptr;
    };
    std::vector<H2o> h2o;
    __half* kv_new = nullptr;  // the decode token's K then V, [2][nkv][64]
    int* h2o_dst = nullptr;    // [n_layers] slot chosen in the last step
    // fused MoE layer (k_moe_fused): fixed-point down accumulators and
    // tickets, zero between launches (each launch leaves them zero)
    bool moe_fused = false;
    unsigned long long* moe_acc = nullptr;
    unsigned* moe_tick = nullptr;
};

template <class T>
static int dalloc(cuinf_session* s, T** p, size_t bytes) {
    void* d = nullptr;
    CUINF_TRY(cudaMalloc(&d, bytes < 16 ? 16 : bytes));
    CUINF_TRY(cudaMemset(d, 0, bytes < 16 ? 16 : bytes));
    s->allocs.push_back(d);
    *p = (T*)d;
    return CUINF_OK;
}

// Per-kernel timing of an eagerly launched step: an event after each launch
// plus the kernel's algorithmic bytes (weights + activations it must move).
struct Prof {
    std::vector<cudaEvent_t> ev;
    std::vector<const char*> name;
    std::vector<double> bytes;
};
static void prof_mark(Prof* p, cudaStream_t st, const char* name, double bytes) {
    if (!p) return;
    cudaEvent_t e;
    cudaEventCreate(&e);
    cudaEventRecord(e, st);
    p->ev.push_back(e);
    p->name.push_back(name);
    p->bytes.push_back(bytes);
}
static double q4_bytes(int64_t N, int64_t K) { return (double)(N * K / 2 + N * (K / 128) * 2); }

// One kernel of the step: how to launch it given its L2 prefetch plan, and
// the static weight ranges it reads (for the plans of the kernels before it).
struct Launch {
    const char* name;
    double bytes;
    std::vector<std::pair<const char*, unsigned long long>> weights;
    std::function<cudaError_t(const L2Ranges&, bool)> fire;
};

static std::pair<const char*, unsigned long long> q4_range(const Q4& w, int64_t N, int64_t K) {
    return {(const char*)w.p, (unsigned long long)(N * K / 2 + N * (K / 128) * 2)};
}

// Weight bytes a kernel prefetches for the kernels after it (at most `budget`
// bytes, from kernels at most `ahead` launches later): each static range is
// scheduled once, as early as the budget allows.
static void plan_prefetch(const std::vector<Launch>& L, std::vector<L2Ranges>& plans, unsigned long long budget,
                          int ahead) {
    const int n = (int)L.size();
    plans.assign(n, L2Ranges());
    // (kernel, range) in execution order, wrapping once into the next step
    std::vector<std::pair<int, std::pair<const char*, unsigned long long>>> q;
    for (int r = 0; r < 2; r++)
        for (int i = 0; i < n; i++)
            for (auto& w : L[i].weights) q.push_back({i + r * n, w});
    size_t next = 0;
    unsigned long long off = 0;  // bytes of q[next] already scheduled
    for (int i = 0; i < n; i++) {
        L2Ranges& R = plans[i];
        R.count = 0;
        while (next < q.size() && q[next].first <= i) { next++; off = 0; }  // too late
        unsigned long long acc = 0;
        while (next < q.size() && R.count < 8 && acc < budget && q[next].first <= i + ahead) {
            const unsigned long long left = q[next].second.second - off;
            unsigned long long len = std::min(left, budget - acc);
            len = (len + 15) & ~15ull;
            if (len > left) len = left;
            R.p[R.count] = q[next].second.first + off;
            R.n[R.count++] = len;
            acc += len;
            off += len;
            if (off >= q[next].second.second) { next++; off = 0; }
        }
    }
}

// Builds the megakernel's device tables (layer pointers, stage program) and
// buffers; leaves s->mk_ok false when the device or the model does not fit
// (the multi-kernel step is then used).
static int setup_megakernel(cuinf_session* s) {
    const cuinf_model* m = s->m;
    const cuinf_config& c = m->cfg;
    const int H = c.hidden, nh = c.n_heads, nkv = c.n_kv_heads, gqa = nh / nkv;
    int dev = 0, coop = 0;
    CUINF_TRY(cudaGetDevice(&dev));
    CUINF_TRY(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev));
    int max_smem = 0;
    CUINF_TRY(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    // stage program limits: at most 4 router tiles of 16 experts, norm of at
    // most 16 elements per consumer thread
    if (!coop || c.top_k > 5 || c.n_experts > 64 || c.n_experts % 8 || H % 64 || H > 16 * MK_CT)
        return CUINF_OK;
    const int xbn = std::max(std::max(H, nh * 64), std::max(c.dense_inter, c.top_k * c.moe_inter));
    const size_t fixed = mk_layout(H, xbn, 0, gqa).total;
    const size_t static_smem = sizeof(MkHeader) + 256;
    if ((size_t)max_smem < fixed + static_smem + 64 * 1024) return CUINF_OK;
    int ring = (int)(((size_t)max_smem - fixed - static_smem) / 1024 * 1024);
    // the largest slab must fit the ring
    const size_t slab_max = std::max(
        std::max((size_t)H * 2 + c.n_experts * 2, (size_t)16 * mk_f16_pitch(H)),
        std::max((size_t)3 * int4_tile_bytes(H) + 160,
                 std::max((size_t)c.top_k * int4_tile_bytes(c.moe_inter),
                          (size_t)int4_tile_bytes(std::max(c.dense_inter, nh * 64)))));
    if (slab_max > (size_t)ring) return CUINF_OK;
    const size_t smem = mk_layout(H, xbn, ring, gqa).total;
    CUINF_TRY(cudaFuncSetAttribute(k_decode_mk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int per_sm = 0;
    CUINF_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_mk, MK_THREADS, smem));
    if (per_sm < 1) return CUINF_OK;
    const int G = s->num_sms;

    // every TMA source of the stage program must be 16-byte aligned
    auto a16 = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
    bool aligned = a16(m->emb_norm) && a16(m->embed);
    for (int l = 0; l < c.n_layers; l++) {
        const LayerW& L = m->L[l];
        aligned = aligned && a16(L.op_norm) && a16(L.ffn_norm);
        if (c.attn_layer[l]) aligned = aligned && a16(L.q_ln) && a16(L.k_ln);
        else aligned = aligned && a16(L.conv_w) && a16(s->conv_state[l]);
        if (l >= c.n_dense) aligned = aligned && a16(L.gate) && a16(L.ebias);
    }
    if (!aligned) return CUINF_OK;

    std::vector<MkLayer> layers(c.n_layers);
    std::vector<MkStage> stages;
    for (int l = 0; l < c.n_layers; l++) {
        const LayerW& L = m->L[l];
        MkLayer& Y = layers[l];
        memset(&Y, 0, sizeof(Y));
        Y.op_norm = L.op_norm;
        Y.ffn_norm = L.ffn_norm;
        if (c.attn_layer[l]) {
            AttnState& A = s->attn[l];
            Y.wq = L.wq.p; Y.sq = L.wq.s; Y.wk = L.wk.p; Y.sk = L.wk.s; Y.wv = L.wv.p; Y.sv = L.wv.s;
            Y.q_ln = L.q_ln; Y.k_ln = L.k_ln;
            Y.kc8 = A.kc8; Y.vc8 = A.vc8; Y.ksc = A.ksc; Y.vsc = A.vsc; Y.ktail = A.ktail; Y.vtail = A.vtail;
            stages.push_back({MK_QKV, l, (nh + 2 * nkv) * 4, H, nullptr, nullptr, nullptr});
            stages.push_back({MK_ATTN, l, 0, 0, nullptr, nullptr, nullptr});
            stages.push_back({MK_RES, l, H / 16, nh * 64, L.wo.p, L.wo.s, s->attn_out});
        } else {
            Y.win = L.in_proj.p; Y.sin = L.in_proj.s; Y.conv_w = L.conv_w; Y.conv_state = s->conv_state[l];
            stages.push_back({MK_CONV_IN, l, H / 16, H, nullptr, nullptr, nullptr});
            stages.push_back({MK_RES, l, H / 16, H, L.out_proj.p, L.out_proj.s, s->conv_y});
        }
        if (l < c.n_dense) {
            Y.w1 = L.w1.p; Y.s1 = L.w1.s; Y.w3 = L.w3.p; Y.s3 = L.w3.s;
            stages.push_back({MK_DENSE_UP, l, c.dense_inter / 16, H, nullptr, nullptr, nullptr});
            stages.push_back({MK_RES, l, H / 16, c.dense_inter, L.w2.p, L.w2.s, s->mid});
        } else {
            Y.gate = L.gate; Y.ebias = L.ebias;
            Y.experts = (const void* const*)(m->d_experts + (size_t)L.moe_index * c.n_experts * 6);
            Y.route_idx = s->route_idx + L.moe_index * c.top_k;
            Y.route_w = s->route_w + L.moe_index * c.top_k;
            stages.push_back({MK_MOE_UP, l, c.top_k * c.moe_inter / 16, H, nullptr, nullptr, nullptr});
            stages.push_back({MK_MOE_DOWN, l, H / 16, c.moe_inter, nullptr, nullptr, nullptr});
        }
    }
    stages.push_back({MK_LMHEAD, -1, (c.vocab + 15) / 16, H, nullptr, nullptr, nullptr});
    s->mk_kinds.clear();
    for (auto& st : stages) s->mk_kinds.push_back(st.kind);
    MkLayer* dL = nullptr;
    MkStage* dS = nullptr;
    int rc = dalloc(s, &dL, layers.size() * sizeof(MkLayer));
    if (!rc) rc = dalloc(s, &dS, stages.size() * sizeof(MkStage));
    if (rc) return rc;
    CUINF_TRY(cudaMemcpy(dL, layers.data(), layers.size() * sizeof(MkLayer), cudaMemcpyHostToDevice));
    CUINF_TRY(cudaMemcpy(dS, stages.data(), stages.size() * sizeof(MkStage), cudaMemcpyHostToDevice));
    MkParams& P = s->mk;
    memset(&P, 0, sizeof(P));
    P.L = dL;
    P.S = dS;
    P.n_stages = (int)stages.size();
    P.H = H; P.nh = nh; P.nkv = nkv; P.I = c.moe_inter; P.E = c.n_experts; P.topk = c.top_k; P.V = c.vocab;
    P.ring_bytes = ring;
    P.xbn = xbn;
    P.attn_chunks = std::max(1, G / nkv);
    P.eps = c.norm_eps; P.theta = c.rope_theta; P.scale = 1.0f / sqrtf((float)c.head_dim);
    P.h = s->h; P.q = s->q; P.attn_out = s->attn_out; P.conv_y = s->conv_y; P.mid = s->mid;
    P.hidden_out = s->hidden;
    if ((rc = dalloc(s, &P.qkv_f32, (size_t)(nh + 2 * nkv) * 64 * 4))) return rc;
    if ((rc = dalloc(s, &P.qkv_tick, (size_t)(nh + 2 * nkv) * 4))) return rc;
    if ((rc = dalloc(s, &P.attn_part, (size_t)nkv * P.attn_chunks * gqa * ATTN_PART_STRIDE * 4))) return rc;
    if ((rc = dalloc(s, &P.attn_tick, (size_t)nkv * 4))) return rc;
    if ((rc = dalloc(s, &s->mk_words, 64))) return rc;
    P.gbar = s->mk_words + 0;
    P.abort_flag = s->mk_words + 1;
    P.err = s->mk_words + 2;
    P.lm_tick = s->mk_words + 3;
    P.am_key = s->am_key;
    P.embed = m->embed; P.emb_norm = m->emb_norm;
    P.tok = s->tok; P.pos = s->pos; P.out_ring = s->out_ring; P.ring = s->max_ctx;
    if ((rc = dalloc(s, &s->mk_trace, (size_t)P.n_stages * G * MK_TRACE_W * 8))) return rc;
    // the attention merge scratch also stages (m, l) of every chunk
    if ((size_t)(2 * P.attn_chunks * gqa + gqa) * 4 > mk_layout(H, xbn, ring, gqa).out - mk_layout(H, xbn, ring, gqa).xs)
        return CUINF_OK;
    s->mk_smem = smem;
    s->mk_grid = G;
    s->mk_ok = true;
    return CUINF_OK;
}

static int record_step_mk(cuinf_session* s) {
    MkParams P = s->mk;
    P.logits = s->keep_logits ? s->logits : nullptr;
    P.trace = s->trace ? s->mk_trace : nullptr;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(s->mk_grid);
    cfg.blockDim = dim3(MK_THREADS);
    cfg.dynamicSmemBytes = s->mk_smem;
    cfg.stream = s->st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CUINF_TRY(cudaLaunchKernelEx(&cfg, k_decode_mk, P));
    s->kernels_per_step = 1;
    return CUINF_OK;
}

// Records one decode step into the session stream (under capture, or eagerly
// with per-kernel events when prof is set).
static H2oParams h2o_params(cuinf_session* s, int l, const __half* k_new, const __half* v_new, const __half* q,
                            __half* out, const int* pos_dev, int past, int S, int* dst) {
    const cuinf_config& c = s->m->cfg;
    const cuinf_session::H2o& Z = s->h2o[l];
    H2oParams P;
    P.k_new = k_new;
    P.v_new = v_new;
    P.q = q;
    P.out = out;
    P.pos_dev = pos_dev;
    P.past = past;
    P.S = S;
    P.C = s->h2o_C;
    P.W = s->h2o_W;
    P.nh = c.n_heads;
    P.nkv = c.n_kv_heads;
    P.scale = 1.0f / sqrtf((float)c.head_dim);
    P.hk8 = Z.hk8;
    P.hv8 = Z.hv8;
    P.hks = Z.hks;
    P.hvs = Z.hvs;
    P.slot_pos = Z.slot_pos;
    P.attn_sum = Z.attn_sum;
    P.n_live = Z.n_live;
    P.dst = dst;
    return P;
}

static int record_step(cuinf_session* s, Prof* prof = nullptr) {
    if (s->use_mk && s->mk_ok && !prof && !s->h2o_C) return record_step_mk(s);
    const cuinf_model* m = s->m;
    const cuinf_config& c = m->cfg;
    const int H = c.hidden;
    cudaStream_t st = s->st;
    const int nh = c.n_heads, nkv = c.n_kv_heads;
    const int sms = s->num_sms;
    std::vector<Launch> Ls;
    for (int l = 0; l < c.n_layers; l++) {
        const LayerW& L = m->L[l];
        const bool first = l == 0;
        if (c.attn_layer[l]) {
            AttnState& A = s->attn[l];
            QkvParams Q;
            Q.h = s->h;
            Q.embed = first ? m->embed : nullptr;
            Q.tok = s->tok;
            Q.h_store = s->h;
            Q.norm_w = L.op_norm;
            Q.wq_p = L.wq.p; Q.wq_s = L.wq.s;
            Q.wk_p = L.wk.p; Q.wk_s = L.wk.s;
            Q.wv_p = L.wv.p; Q.wv_s = L.wv.s;
            Q.q_ln = L.q_ln;
            Q.k_ln = L.k_ln;
            Q.pos = s->pos;
            Q.q_out = s->q;
            Q.ktail = A.ktail; Q.vtail = A.vtail;
            Q.kc8 = A.kc8; Q.vc8 = A.vc8;
            Q.ksc = A.ksc; Q.vsc = A.vsc;
            Q.kv_new = s->h2o_C ? s->kv_new : nullptr;
            Q.H = H; Q.nh = nh; Q.nkv = nkv;
            Q.eps = c.norm_eps; Q.theta = c.rope_theta;
            const int heads = nh + 2 * nkv;
            const size_t sq = qkv_smem(H);
            Ls.push_back({"attn_qkv", q4_bytes((nh + 2 * nkv) * 64, H) + 2.0 * H + nh * 128 + 4 * nkv * 64,
                          {q4_range(L.wq, nh * 64, H), q4_range(L.wk, nkv * 64, H), q4_range(L.wv, nkv * 64, H)},
                          [=](const L2Ranges& nx, bool pdl) mutable {
                              Q.next = nx;
                              return launch_k(k_attn_qkv, dim3(heads * 4), dim3(256), sq, st, pdl, Q);
                          }});
            AttnParams P;
            P.q = s->q;
            P.kc8 = A.kc8; P.vc8 = A.vc8; P.ksc = A.ksc; P.vsc = A.vsc;
            P.ktail = A.ktail; P.vtail = A.vtail;
            P.pos_dev = s->pos;
            P.committed = 0; P.qpos = 0;
            P.scale = 1.0f / sqrtf((float)c.head_dim);
            P.out = s->attn_out;
            P.part = s->attn_part;
            P.counters = s->attn_cnt;
            P.nh = nh; P.nkv = nkv; P.nsplit = s->nsplit;
            const double ctx = s->host_pos + 1, cm = 64.0 * floor(ctx / 64.0);
            const int nsplit = s->nsplit;
            const int cluster = s->attn_use_cluster ? s->attn_cluster : 0;
            if (s->h2o_C) {  // H2O: slot choice + quantized write, then attention over the slots
                H2oParams Z = h2o_params(s, l, s->kv_new, s->kv_new + nkv * 64, s->q, s->attn_out, s->pos, 0, 1,
                                         s->h2o_dst + l);
                const double live = std::min<double>(ctx, s->h2o_C);
                Ls.push_back({"h2o_place", 12.0 * s->h2o_C + nkv * 256.0, {},
                              [=](const L2Ranges&, bool pdl) mutable {
                                  return launch_k(k_h2o_place, dim3(1), dim3(256), 0, st, pdl, Z);
                              }});
                const size_t smz = (size_t)s->h2o_C * 4;
                Ls.push_back({"h2o_attention", live * (nkv * 132.0 + 12.0) * 1.0 + nh * 256.0, {},
                              [=](const L2Ranges&, bool pdl) mutable {
                                  return launch_k(k_h2o_attn, dim3(1, nh), dim3(256), smz, st, pdl, Z);
                              }});
            } else {
                Ls.push_back({"attn_decode", cm * nkv * 128 + cm / 64 * nkv * 4 + (ctx - cm) * nkv * 256 + nh * 256.0,
                              {},
                              [=](const L2Ranges& nx, bool pdl) mutable {
                                  P.next = nx;
                                  if (cluster) {
                                      P.cluster = cluster;
                                      return launch_kcy(k_attn_decode<1>, dim3(nkv, nsplit), dim3(ATTN_THREADS), 0,
                                                        st, pdl, cluster, P);
                                  }
                                  return launch_k(k_attn_decode<1>, dim3(nkv, nsplit), dim3(ATTN_THREADS), 0, st, pdl, P);
                              }});
            }
            ResParams R;
            R.act = s->attn_out; R.wp = L.wo.p; R.ws = L.wo.s; R.h = s->h; R.N = H; R.K = nh * 64;
            Ls.push_back({"attn_out_proj", q4_bytes(H, nh * 64) + nh * 128 + 4.0 * H,
                          {q4_range(L.wo, H, nh * 64)},
                          [=](const L2Ranges& nx, bool pdl) mutable {
                              R.next = nx;
                              return launch_k(k_gemv_residual, dim3(H / 16), dim3(RES_WARPS * 32), one_per_sm(res_smem(nh * 64), H / 16, sms), st, pdl, R);
                          }});
        } else {
            ConvParams C;
            C.h = s->h;
            C.embed = first ? m->embed : nullptr;
            C.tok = s->tok;
            C.h_store = s->h;
            C.norm_w = L.op_norm;
            C.wp = L.in_proj.p; C.ws = L.in_proj.s;
            C.conv_w = L.conv_w;
            C.state = s->conv_state[l];
            C.y = s->conv_y;
            C.H = H; C.eps = c.norm_eps;
            Ls.push_back({"conv_in", q4_bytes(3 * H, H) + 18.0 * H, {q4_range(L.in_proj, 3 * H, H)},
                          [=](const L2Ranges& nx, bool pdl) mutable {
                              C.next = nx;
                              return launch_k(k_conv_in, dim3(H / 16), dim3(CONV_WARPS * 32), one_per_sm(conv_smem(H), H / 16, sms), st, pdl, C);
                          }});
            ResParams R;
            R.act = s->conv_y; R.wp = L.out_proj.p; R.ws = L.out_proj.s; R.h = s->h; R.N = H; R.K = H;
            Ls.push_back({"conv_out_proj", q4_bytes(H, H) + 6.0 * H, {q4_range(L.out_proj, H, H)},
                          [=](const L2Ranges& nx, bool pdl) mutable {
                              R.next = nx;
                              return launch_k(k_gemv_residual, dim3(H / 16), dim3(RES_WARPS * 32), one_per_sm(res_smem(H), H / 16, sms), st, pdl, R);
                          }});
        }
        if (l < c.n_dense) {
            FfnUpParams F;
            F.h = s->h; F.norm_w = L.ffn_norm;
            F.w1p = L.w1.p; F.w1s = L.w1.s; F.w3p = L.w3.p; F.w3s = L.w3.s;
            F.mid = s->mid; F.H = H; F.I = c.dense_inter; F.eps = c.norm_eps;
            const int I = c.dense_inter;
            Ls.push_back({"dense_up", 2 * q4_bytes(I, H) + 4.0 * H + 2.0 * I,
                          {q4_range(L.w1, I, H), q4_range(L.w3, I, H)},
                          [=](const L2Ranges& nx, bool pdl) mutable {
                              F.next = nx;
                              return launch_k(k_ffn_up, dim3((I + 15) / 16), dim3(256), ffn_up_smem(H), st, pdl, F);
                          }});
            ResParams R;
            R.act = s->mid; R.wp = L.w2.p; R.ws = L.w2.s; R.h = s->h; R.N = H; R.K = I;
            Ls.push_back({"dense_down", q4_bytes(H, I) + 2.0 * I + 4.0 * H, {q4_range(L.w2, H, I)},
                          [=](const L2Ranges& nx, bool pdl) mutable {
                              R.next = nx;
                              return launch_k(k_gemv_residual, dim3(H / 16), dim3(RES_WARPS * 32), one_per_sm(res_smem(I), H / 16, sms), st, pdl, R);
                          }});
        } else {
            const int mi = L.moe_index;
            const void* const* ex = (const void* const*)(m->d_experts + (size_t)mi * c.n_experts * 6);
            const double moe_bytes = 2.0 * c.top_k * q4_bytes(c.moe_inter, H) + c.top_k * q4_bytes(H, c.moe_inter) +
                                     (double)c.n_experts * H * 2 + c.n_experts * 2 + 4.0 * H;
            if (s->moe_fused) {
                MoeFusedParams F;
                F.h = s->h; F.xn = nullptr; F.h_out = s->h; F.norm_w = L.ffn_norm;
                F.gate = L.gate; F.bias = L.ebias; F.experts = ex;
                F.route_idx = s->route_idx + mi * c.top_k;
                F.route_w = s->route_w + mi * c.top_k;
                F.acc = s->moe_acc; F.tickets = s->moe_tick;
                F.H = H; F.I = c.moe_inter; F.E = c.n_experts; F.topk = c.top_k; F.eps = c.norm_eps;
                const int grid = c.top_k * (c.moe_inter / 16);
                const size_t sm = moef_layout(H, c.n_experts).total;
                Ls.push_back({"moe_ffn", moe_bytes,
                              {{(const char*)L.gate, (unsigned long long)c.n_experts * H * 2}},
                              [=](const L2Ranges& nx, bool pdl) mutable {
                                  F.next = nx;
                                  return launch_k(k_moe_fused, dim3(grid), dim3(MOEF_THREADS), sm, st, pdl, F);
                              }});
                continue;
            }
            MoeUpParams U;
            U.h = s->h; U.xn = nullptr; U.norm_w = L.ffn_norm;
            U.gate = L.gate; U.bias = L.ebias;
            U.experts = ex;
            U.mid = s->mid;
            U.route_idx = s->route_idx + mi * c.top_k;
            U.route_w = s->route_w + mi * c.top_k;
            U.H = H; U.I = c.moe_inter; U.E = c.n_experts; U.topk = c.top_k; U.eps = c.norm_eps;
            const int tiles = c.moe_inter / 16;
            const int grid_up = ((c.top_k * tiles + 7) / 8) * 8;
            Ls.push_back({"moe_up", 2.0 * c.top_k * q4_bytes(c.moe_inter, H) + (double)c.n_experts * H * 2 +
                                        c.n_experts * 2 + 4.0 * H + 2.0 * c.top_k * c.moe_inter,
                          {{(const char*)L.gate, (unsigned long long)c.n_experts * H * 2}},
                          [=](const L2Ranges& nx, bool pdl) mutable {
                              U.next = nx;
                              return launch_k(k_moe_up, dim3(grid_up), dim3(256), moe_up_smem(H, c.n_experts), st, pdl, U);
                          }});
            MoeDownParams D;
            D.mid = s->mid; D.experts = U.experts;
            D.route_idx = U.route_idx; D.route_w = U.route_w;
            D.h = s->h; D.H = H; D.I = c.moe_inter; D.topk = c.top_k;
            const size_t sd = moe_down_smem(c.moe_inter, c.top_k);
            Ls.push_back({"moe_down", c.top_k * q4_bytes(H, c.moe_inter) + 2.0 * c.top_k * c.moe_inter + 4.0 * H,
                          {},
                          [=](const L2Ranges& nx, bool pdl) mutable {
                              D.next = nx;
                              return launch_kc(k_moe_down, dim3((H / 16) * c.top_k), dim3(256), sd, st, pdl,
                                               c.top_k, D);
                          }});
        }
    }
    LmHeadParams LM;
    LM.h = s->h;
    LM.norm_w = m->emb_norm;
    LM.W = m->embed;
    LM.logits = s->keep_logits ? s->logits : nullptr;
    LM.hidden_out = s->hidden;
    LM.key = s->am_key;
    LM.ticket = s->am_ticket;
    LM.tok = s->tok;
    LM.pos = s->pos;
    LM.out_ring = s->out_ring;
    LM.ring = s->max_ctx;
    LM.H = H;
    LM.V = c.vocab;
    LM.eps = c.norm_eps;
    const int lm_stages = (c.vocab + lmhead_rows_per_stage(H) - 1) / lmhead_rows_per_stage(H);
    const int lm_grid = std::min(s->num_sms, lm_stages);
    Ls.push_back({"lm_head_argmax", (double)c.vocab * H * 2 + 6.0 * H,
                  {{(const char*)m->embed, (unsigned long long)c.vocab * H * 2}},
                  [=](const L2Ranges& nx, bool pdl) mutable {
                      LM.next = nx;
                      return launch_k(k_lmhead, dim3(lm_grid), dim3(LM_THREADS), lmhead_smem(H), st, pdl, LM);
                  }});

    std::vector<L2Ranges> plans;
    if (s->prefetch) plan_prefetch(Ls, plans, (unsigned long long)s->prefetch_mb << 20, s->prefetch_ahead);
    else plans.assign(Ls.size(), L2Ranges{{}, {}, 0});
    prof_mark(prof, st, "start", 0);
    for (size_t i = 0; i < Ls.size(); i++) {
        // the step's first kernel follows host copies / the previous graph: no PDL
        cudaError_t e = Ls[i].fire(plans[i], s->pdl && i > 0);
        if (e != cudaSuccess) return cuinf_set_cuda_error(e);
        prof_mark(prof, st, Ls[i].name, Ls[i].bytes);
    }
    s->kernels_per_step = (int)Ls.size();
    return cuinf_launch_status();
}

static int build_graph(cuinf_session* s) {
    if (s->exec) { cudaGraphExecDestroy(s->exec); s->exec = nullptr; }
    if (s->graph) { cudaGraphDestroy(s->graph); s->graph = nullptr; }
    CUINF_TRY(cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal));
    int rc = record_step(s);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(s->st, &g);
    if (rc) { if (g) cudaGraphDestroy(g); return rc; }
    if (e != cudaSuccess) return cuinf_set_cuda_error(e);
    s->graph = g;
    CUINF_TRY(cudaGraphInstantiate(&s->exec, g, 0));
    return CUINF_OK;
}

static int set_kernel_attrs(const cuinf_config& c) {
    const int H = c.hidden;

    struct { const void* k; size_t bytes; } need[] = {
        {(const void*)k_attn_qkv, qkv_smem(H)},
        {(const void*)k_conv_in, std::max(conv_smem(H), ONE_PER_SM_SMEM)},
        {(const void*)k_ffn_up, ffn_up_smem(H)},
        {(const void*)k_moe_up, moe_up_smem(H, std::max(1, c.n_experts))},
        {(const void*)k_moe_down, moe_down_smem(c.moe_inter, std::max(1, c.top_k))},
        {(const void*)k_lmhead, lmhead_smem(H)},
        {(const void*)k_moe_fused, moef_supported(H, c.moe_inter, c.n_experts, c.top_k)
                                       ? moef_layout(H, c.n_experts).total : (size_t)0},
        {(const void*)k_gemv_residual,
         std::max(ONE_PER_SM_SMEM, std::max(res_smem(H), std::max(res_smem(c.n_heads * 64), res_smem(c.dense_inter))))},
    };
    for (auto& n : need) {
        if (n.bytes > 227 * 1024) return cuinf_set_arg_error("model dims too large for shared memory");
        if (n.bytes > 48 * 1024)
            CUINF_TRY(cudaFuncSetAttribute(n.k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)n.bytes));
    }
    return CUINF_OK;
}

extern "C" int cuinf_session_free(cuinf_session* s) {
    if (!s) return CUINF_OK;
    if (s->st) cudaStreamSynchronize(s->st);
    if (s->pf_buf) cudaFree(s->pf_buf);
    for (auto& Z : s->h2o) {
        cudaFree(Z.hk8); cudaFree(Z.hv8); cudaFree(Z.hks); cudaFree(Z.hvs);
        cudaFree(Z.slot_pos); cudaFree(Z.attn_sum); cudaFree(Z.n_live);
    }
    if (s->kv_new) cudaFree(s->kv_new);
    if (s->h2o_dst) cudaFree(s->h2o_dst);
    if (s->exec) cudaGraphExecDestroy(s->exec);
    if (s->graph) cudaGraphDestroy(s->graph);
    for (void* p : s->allocs) cudaFree(p);
    for (int i = 0; i < cuinf_session::kTokRing; i++)
        if (s->tok_ev[i]) cudaEventDestroy(s->tok_ev[i]);
    if (s->pinned) cudaFreeHost(s->pinned);
    if (s->own_stream && s->st) cudaStreamDestroy(s->st);
    delete s;
    return CUINF_OK;
}

extern "C" int cuinf_session_create(cuinf_model* m, int max_ctx, void* stream, cuinf_session** out) {
    REQUIRE(m && out, "null pointer");
    REQUIRE(max_ctx > 0 && max_ctx <= (1 << 24), "max_ctx out of range");
    const cuinf_config& c = m->cfg;
    cuinf_session* s = new cuinf_session();
    s->m = m;
    s->max_ctx = max_ctx;
    int rc = CUINF_OK;
#define TRYS(x) do { rc = (x); if (rc) { cuinf_session_free(s); return rc; } } while (0)
#define TRYC(x) do { cudaError_t e_ = (x); if (e_ != cudaSuccess) { rc = cuinf_set_cuda_error(e_); cuinf_session_free(s); return rc; } } while (0)
    if (stream) s->st = ST(stream);
    else { TRYC(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking)); s->own_stream = true; }
    int dev = 0;
    TRYC(cudaGetDevice(&dev));
    TRYC(cudaDeviceGetAttribute(&s->num_sms, cudaDevAttrMultiProcessorCount, dev));
    TRYS(set_kernel_attrs(c));
    const int H = c.hidden, nkv = c.n_kv_heads, gqa = c.n_heads / c.n_kv_heads;
    const size_t maxI = std::max((size_t)c.dense_inter, (size_t)c.top_k * c.moe_inter);
    TRYS(dalloc(s, &s->h, (size_t)H * 2));
    TRYS(dalloc(s, &s->q, (size_t)c.n_heads * 64 * 2));
    TRYS(dalloc(s, &s->attn_out, (size_t)c.n_heads * 64 * 2));
    TRYS(dalloc(s, &s->conv_y, (size_t)H * 2));
    TRYS(dalloc(s, &s->mid, maxI * 2));
    TRYS(dalloc(s, &s->hidden, (size_t)H * 2));
    TRYS(dalloc(s, &s->pos, 16));
    TRYS(dalloc(s, &s->tok, 16));
    TRYS(dalloc(s, &s->out_ring, (size_t)max_ctx * 4));
    TRYS(dalloc(s, &s->route_idx, (size_t)std::max(1, m->n_moe * c.top_k) * 4));
    TRYS(dalloc(s, &s->route_w, (size_t)std::max(1, m->n_moe * c.top_k) * 4));
    TRYS(dalloc(s, &s->logits, (size_t)c.vocab * 4));
    TRYS(dalloc(s, &s->am_key, 16));
    TRYS(dalloc(s, &s->am_ticket, 16));
    const int units = max_ctx / CUINF_KVGROUP + 1;
    // k_attn_decode holds one CTA per SM (its registers): keep every split
    // of every kv head in one wave
    s->nsplit = std::min(attn_engine_nsplit(gqa, units), std::max(1, s->num_sms / nkv));
    // with clusters the splits of a kv head merge over DSMEM: at most 16
    // splits (both merge paths then use the same splits, so they agree bit
    // for bit)
    s->attn_cluster = attn_cluster_size(nkv, s->nsplit);
    if (s->attn_cluster) s->nsplit = s->attn_cluster;
    TRYS(dalloc(s, &s->attn_part, (size_t)nkv * s->nsplit * gqa * ATTN_PART_STRIDE * 4));
    TRYS(dalloc(s, &s->attn_cnt, (size_t)nkv * 4));
    bool bias16 = true;  // the fused MoE kernel copies each router bias with 16-byte async copies
    for (int l = c.n_dense; l < c.n_layers; l++) bias16 = bias16 && ((uintptr_t)m->L[l].ebias & 15) == 0;
    if (m->n_moe > 0 && bias16 && moef_supported(H, c.moe_inter, c.n_experts, c.top_k)) {
        TRYS(dalloc(s, &s->moe_acc, (size_t)c.top_k * H * 8));
        TRYS(dalloc(s, &s->moe_tick, 256));
        s->moe_fused = true;
    }
    s->attn.assign(c.n_layers, AttnState());
    s->conv_state.assign(c.n_layers, nullptr);
    const size_t row = (size_t)nkv * 64;
    const size_t groups = (size_t)max_ctx / CUINF_KVGROUP + 2;
    for (int l = 0; l < c.n_layers; l++) {
        if (c.attn_layer[l]) {
            AttnState& A = s->attn[l];
            TRYS(dalloc(s, &A.kc8, (size_t)max_ctx * row));
            TRYS(dalloc(s, &A.vc8, (size_t)max_ctx * row));
            TRYS(dalloc(s, &A.ksc, groups * nkv * 2));
            TRYS(dalloc(s, &A.vsc, groups * nkv * 2));
            TRYS(dalloc(s, &A.ktail, (size_t)CUINF_KVGROUP * row * 2));
            TRYS(dalloc(s, &A.vtail, (size_t)CUINF_KVGROUP * row * 2));
        } else {
            TRYS(dalloc(s, &s->conv_state[l], (size_t)2 * H * 2));
        }
    }
    TRYC(cudaMallocHost(&s->pinned, (cuinf_session::kTokRing + 1) * sizeof(int)));
    for (int i = 0; i < cuinf_session::kTokRing; i++)
        TRYC(cudaEventCreateWithFlags(&s->tok_ev[i], cudaEventDisableTiming));
    TRYS(setup_megakernel(s));
    TRYS(build_graph(s));
#undef TRYS
#undef TRYC
    *out = s;
    return CUINF_OK;
}

extern "C" int cuinf_session_reset(cuinf_session* s) {
    REQUIRE(s, "null session");
    const cuinf_config& c = s->m->cfg;
    const size_t row = (size_t)c.n_kv_heads * 64;
    const size_t groups = (size_t)s->max_ctx / CUINF_KVGROUP + 2;
    for (int l = 0; l < c.n_layers; l++) {
        if (c.attn_layer[l]) {
            AttnState& A = s->attn[l];
            CUINF_TRY(cudaMemsetAsync(A.kc8, 0, (size_t)s->max_ctx * row, s->st));
            CUINF_TRY(cudaMemsetAsync(A.vc8, 0, (size_t)s->max_ctx * row, s->st));
            CUINF_TRY(cudaMemsetAsync(A.ksc, 0, groups * c.n_kv_heads * 2, s->st));
            CUINF_TRY(cudaMemsetAsync(A.vsc, 0, groups * c.n_kv_heads * 2, s->st));
            CUINF_TRY(cudaMemsetAsync(A.ktail, 0, CUINF_KVGROUP * row * 2, s->st));
            CUINF_TRY(cudaMemsetAsync(A.vtail, 0, CUINF_KVGROUP * row * 2, s->st));
        } else {
            CUINF_TRY(cudaMemsetAsync(s->conv_state[l], 0, (size_t)2 * c.hidden * 2, s->st));
        }
    }
    for (auto& Z : s->h2o)
        if (Z.n_live) {
            CUINF_TRY(cudaMemsetAsync(Z.n_live, 0, 4, s->st));
            CUINF_TRY(cudaMemsetAsync(Z.attn_sum, 0, (size_t)s->h2o_C * 4, s->st));
            CUINF_TRY(cudaMemsetAsync(Z.slot_pos, 0, (size_t)s->h2o_C * 4, s->st));
        }
    CUINF_TRY(cudaMemsetAsync(s->pos, 0, 4, s->st));
    if (s->mk_words) CUINF_TRY(cudaMemsetAsync(s->mk_words, 0, 64, s->st));
    CUINF_TRY(cudaStreamSynchronize(s->st));
    s->host_pos = 0;
    return CUINF_OK;
}

extern "C" int cuinf_session_pos(const cuinf_session* s) { return s ? s->host_pos : -1; }

// ---------------------------------------------------------------------------
// sequence state snapshots (KV cache + conv state at a position)
// ---------------------------------------------------------------------------
static const uint32_t kStateMagic = 0x54534943u;  // "CIST"
static const uint32_t kStateVersion = 1;
struct StateHeader {
    uint32_t magic, version;
    int32_t pos, n_layers, hidden, n_kv_heads, reserved[2];
};

size_t seq_state_bytes(const cuinf_config& c, int pos) {
    const size_t row = (size_t)c.n_kv_heads * CUINF_HD;
    const size_t C = (size_t)(pos / CUINF_KVGROUP) * CUINF_KVGROUP;
    size_t n = sizeof(StateHeader);
    for (int l = 0; l < c.n_layers; l++) {
        if (c.attn_layer[l])
            n += 2 * C * row + 2 * (C / CUINF_KVGROUP) * c.n_kv_heads * 2 + 2 * (size_t)CUINF_KVGROUP * row * 2;
        else
            n += (size_t)2 * c.hidden * 2;
    }
    return n;
}

int seq_state_header(const cuinf_config& c, const void* host, size_t n, int max_ctx, int* pos) {
    REQUIRE(host && n >= sizeof(StateHeader), "state snapshot too short");
    StateHeader hd;
    memcpy(&hd, host, sizeof(hd));
    REQUIRE(hd.magic == kStateMagic && hd.version == kStateVersion, "not a cuinf state snapshot (v1)");
    REQUIRE(hd.n_layers == c.n_layers && hd.hidden == c.hidden && hd.n_kv_heads == c.n_kv_heads,
            "state snapshot of another model shape");
    REQUIRE(hd.pos >= 0 && hd.pos < max_ctx, "state snapshot position beyond max_ctx");
    REQUIRE(n == seq_state_bytes(c, hd.pos), "state snapshot size does not match its position");
    *pos = hd.pos;
    return CUINF_OK;
}

int seq_state_copy(const cuinf_config& c, int pos, const AttnState* attn, __half* const* conv, void* host,
                   size_t n, bool save, cudaStream_t st) {
    REQUIRE(n == seq_state_bytes(c, pos), "state buffer size does not match the position");
    const size_t row = (size_t)c.n_kv_heads * CUINF_HD;
    const size_t C = (size_t)(pos / CUINF_KVGROUP) * CUINF_KVGROUP;
    uint8_t* p = (uint8_t*)host;
    if (save) {
        StateHeader hd = {kStateMagic, kStateVersion, pos, c.n_layers, c.hidden, c.n_kv_heads, {0, 0}};
        memcpy(p, &hd, sizeof(hd));
    }
    p += sizeof(StateHeader);
    auto piece = [&](void* dev, size_t bytes) -> cudaError_t {
        cudaError_t e = bytes == 0 ? cudaSuccess
                        : save     ? cudaMemcpyAsync(p, dev, bytes, cudaMemcpyDeviceToHost, st)
                                   : cudaMemcpyAsync(dev, p, bytes, cudaMemcpyHostToDevice, st);
        p += bytes;
        return e;
    };
    for (int l = 0; l < c.n_layers; l++) {
        if (c.attn_layer[l]) {
            const AttnState& A = attn[l];
            const size_t sc = (C / CUINF_KVGROUP) * c.n_kv_heads * 2, tail = (size_t)CUINF_KVGROUP * row * 2;
            CUINF_TRY(piece(A.kc8, C * row));
            CUINF_TRY(piece(A.vc8, C * row));
            CUINF_TRY(piece(A.ksc, sc));
            CUINF_TRY(piece(A.vsc, sc));
            CUINF_TRY(piece(A.ktail, tail));
            CUINF_TRY(piece(A.vtail, tail));
        } else {
            CUINF_TRY(piece(conv[l], (size_t)2 * c.hidden * 2));
        }
    }
    CUINF_TRY(cudaStreamSynchronize(st));
    return CUINF_OK;
}

extern "C" size_t cuinf_session_state_bytes(const cuinf_session* s) {
    return s ? seq_state_bytes(s->m->cfg, s->host_pos) : 0;
}

extern "C" int cuinf_session_save_state(cuinf_session* s, void* host, size_t n) {
    REQUIRE(s && host, "null pointer");
    REQUIRE(!s->h2o_C, "state snapshots are not available in H2O eviction mode");
    CUINF_TRY(cudaStreamSynchronize(s->st));
    return seq_state_copy(s->m->cfg, s->host_pos, s->attn.data(), s->conv_state.data(), host, n, true, s->st);
}

extern "C" int cuinf_session_load_state(cuinf_session* s, const void* host, size_t n) {
    REQUIRE(s && host, "null pointer");
    REQUIRE(!s->h2o_C, "state snapshots are not available in H2O eviction mode");
    int pos = 0;
    int rc = seq_state_header(s->m->cfg, host, n, s->max_ctx, &pos);
    if (rc) return rc;
    CUINF_TRY(cudaStreamSynchronize(s->st));
    rc = seq_state_copy(s->m->cfg, pos, s->attn.data(), s->conv_state.data(), const_cast<void*>(host), n,
                        false, s->st);
    if (rc) return rc;
    CUINF_TRY(cudaMemcpy(s->pos, &pos, 4, cudaMemcpyHostToDevice));
    if (s->mk_words) CUINF_TRY(cudaMemset(s->mk_words, 0, 64));
    s->host_pos = pos;
    return CUINF_OK;
}

extern "C" int cuinf_decode_step(cuinf_session* s, int token, int* out_token) {
    REQUIRE(s && s->exec, "null session");
    REQUIRE(s->host_pos < s->max_ctx, "context full (max_ctx reached)");
    REQUIRE(token < s->m->cfg.vocab, "token out of range");
    if (token >= 0) {
        const int k = s->tok_slot;
        s->tok_slot = (k + 1) % cuinf_session::kTokRing;
        CUINF_TRY(cudaEventSynchronize(s->tok_ev[k]));  // its previous copy has run
        s->pinned[k] = token;
        CUINF_TRY(cudaMemcpyAsync(s->tok, &s->pinned[k], 4, cudaMemcpyHostToDevice, s->st));
        CUINF_TRY(cudaEventRecord(s->tok_ev[k], s->st));
    }
    CUINF_TRY(cudaGraphLaunch(s->exec, s->st));
    s->host_pos++;
    if (out_token) {
        int* o = &s->pinned[cuinf_session::kTokRing];
        CUINF_TRY(cudaMemcpyAsync(o, s->tok, 4, cudaMemcpyDeviceToHost, s->st));
        CUINF_TRY(cudaStreamSynchronize(s->st));
        *out_token = *o;
    }
    return CUINF_OK;
}

// ---------------------------------------------------------------------------
// prefill: the reference's batched layer_forward(S) (engine.cu:784-908, 910-917) for
// the S prompt tokens at positions pos..pos+S-1, then compute_logits_last
// (932-940).  Per attention layer all S tokens' K/V are placed first (tail up
// to each group boundary, full groups committed, 831-845) and then every
// query attends over what is committed (attention_fused, 236-308) -- which is
// why a prompt prefilled here differs from the same prompt decoded token by
// token.  Kernel by kernel on the session stream (not captured); afterwards
// the session continues with decode steps from position pos + S.
// ---------------------------------------------------------------------------
// From this many prompt rows on, prefill runs its projections on the
// tensor-core GEMM and its MoE as grouped expert GEMMs; shorter prompts use
// the batch-1 GEMV kernels.
#define PF_TC_MIN_ROWS 16
static int pf_gemm(const void* x, const uint8_t* packed, const void* scales, float* y, int M, int N, int K,
                   void* stream) {
    if (M >= PF_TC_MIN_ROWS) return cuinf_gemm_int4_tc(x, packed, scales, y, M, N, K, stream);
    return cuinf_gemv_int4(x, packed, scales, y, M, N, K, stream);
}

extern "C" int cuinf_prefill(cuinf_session* s, const int* ids, int S, int* out_token, int* routes_out) {
    REQUIRE(s && ids && S > 0, "bad arguments");
    const cuinf_model* m = s->m;
    const cuinf_config& c = m->cfg;
    REQUIRE(s->host_pos + S <= s->max_ctx, "context too long for max_ctx");
    REQUIRE(!s->h2o_C || S <= s->h2o_C, "with a KV budget the prompt must fit the budget (engine.cu:753)");
    for (int i = 0; i < S; i++) REQUIRE(ids[i] >= 0 && ids[i] < c.vocab, "token out of range");
    const int H = c.hidden, nh = c.n_heads, nkv = c.n_kv_heads, hd = 64, E = c.n_experts, K = c.top_k;
    const int NQ = nh * hd, NK = nkv * hd;
    const int maxN = std::max(std::max(3 * H, NQ), std::max(c.dense_inter, c.moe_inter));
    const int n_moe = c.n_layers - c.n_dense;
    cudaStream_t st = s->st;
    // scratch: ids, pos, hs, xn, q, k, v, ao, t16, t16b, acc (fp16), fa, fb (fp32), mid, routes
    auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t b_int = al((size_t)S * 4), b_h = al((size_t)S * H * 2), b_q = al((size_t)S * NQ * 2),
                 b_k = al((size_t)S * NK * 2), b_t = al((size_t)S * maxN * 2), b_f = al((size_t)S * maxN * 4),
                 b_mid = al((size_t)K * c.moe_inter * 2), b_r = al((size_t)S * std::max(1, n_moe) * K * 4);
    const size_t total = 2 * b_int + 3 * b_h + 2 * b_q + 2 * b_k + 2 * b_t + 2 * b_f + b_mid + 2 * b_r + al(4 * c.vocab);
    if (S > s->pf_cap) {
        if (s->pf_buf) {
            CUINF_TRY(cudaStreamSynchronize(st));
            CUINF_TRY(cudaFree(s->pf_buf));
            s->pf_buf = nullptr;
        }
        CUINF_TRY(cudaMalloc(&s->pf_buf, total));
        s->pf_cap = S;
    }
    char* b = (char*)s->pf_buf;
    auto take = [&](size_t n) { char* p = b; b += n; return p; };
    int* d_ids = (int*)take(b_int);
    int* d_pos = (int*)take(b_int);
    __half* hs = (__half*)take(b_h);
    __half* xn = (__half*)take(b_h);
    __half* acc = (__half*)take(b_h);
    __half* q16 = (__half*)take(b_q);
    __half* ao = (__half*)take(b_q);
    __half* k16 = (__half*)take(b_k);
    __half* v16 = (__half*)take(b_k);
    __half* t16 = (__half*)take(b_t);
    __half* t16b = (__half*)take(b_t);
    float* fa = (float*)take(b_f);
    float* fb = (float*)take(b_f);
    __half* mid = (__half*)take(b_mid);
    int* ridx = (int*)take(b_r);
    float* rw = (float*)take(b_r);
    float* logits = (float*)take(al(4 * c.vocab));
    const int past = s->host_pos;
    std::vector<int> hpos(S);
    for (int i = 0; i < S; i++) hpos[i] = past + i;
    CUINF_TRY(cudaMemcpyAsync(d_ids, ids, (size_t)S * 4, cudaMemcpyHostToDevice, st));
    CUINF_TRY(cudaMemcpyAsync(d_pos, hpos.data(), (size_t)S * 4, cudaMemcpyHostToDevice, st));
    int rc;
#define PF(call) do { if ((rc = (call)) != CUINF_OK) return rc; } while (0)
    void* vs = (void*)st;
    PF(cuinf_embed_gather(m->embed, d_ids, hs, S, H, vs));
    for (int l = 0; l < c.n_layers; l++) {
        const LayerW& L = m->L[l];
        PF(cuinf_rmsnorm(hs, L.op_norm, xn, S, H, c.norm_eps, vs));
        if (c.attn_layer[l]) {
            AttnState& A = s->attn[l];
            PF(pf_gemm(xn, L.wq.p, L.wq.s, fa, S, NQ, H, vs));
            PF(cuinf_f32_to_f16(fa, q16, S * NQ, vs));
            PF(pf_gemm(xn, L.wk.p, L.wk.s, fa, S, NK, H, vs));
            PF(cuinf_f32_to_f16(fa, k16, S * NK, vs));
            PF(pf_gemm(xn, L.wv.p, L.wv.s, fa, S, NK, H, vs));
            PF(cuinf_f32_to_f16(fa, v16, S * NK, vs));
            PF(cuinf_rmsnorm(q16, L.q_ln, q16, S * nh, hd, c.norm_eps, vs));
            PF(cuinf_rmsnorm(k16, L.k_ln, k16, S * nkv, hd, c.norm_eps, vs));
            PF(cuinf_rope(q16, k16, d_pos, S, nh, nkv, c.rope_theta, vs));
            if (s->h2o_C) {  // H2O: every fresh token's slot, then every query over the slots
                // d_ids (consumed by the embedding gather) holds the chosen slots
                H2oParams Z = h2o_params(s, l, k16, v16, q16, ao, nullptr, past, S, d_ids);
                k_h2o_place<<<1, 256, 0, st>>>(Z);
                PF(cuinf_launch_status());
                k_h2o_attn<<<dim3(S, nh), 256, (size_t)s->h2o_C * 4, st>>>(Z);
                PF(cuinf_launch_status());
                PF(pf_gemm(ao, L.wo.p, L.wo.s, fa, S, H, NQ, vs));
                PF(cuinf_add_f32_inplace(hs, fa, S * H, vs));
                goto ffn;
            }
            {
            // the group already begun in the tail is completed there; whole
            // groups of new rows are committed straight from the rows (one
            // launch); the remainder starts the new tail
            int committed = (past / CUINF_KVGROUP) * CUINF_KVGROUP, placed = 0;
            if (past > committed) {
                const int slot = past - committed, can = std::min(S, CUINF_KVGROUP - slot);
                PF(cuinf_kv_write_tail(k16, v16, A.ktail, A.vtail, slot, can, nkv, vs));
                placed = can;
                if (slot + can == CUINF_KVGROUP) {
                    PF(cuinf_kv_commit_group(A.ktail, A.vtail, A.kc8, A.vc8, A.ksc, A.vsc, committed,
                                             committed / CUINF_KVGROUP, nkv, vs));
                    committed += CUINF_KVGROUP;
                }
            }
            const int whole = (S - placed) / CUINF_KVGROUP;
            PF(kv_commit_rows(k16 + (size_t)placed * NK, v16 + (size_t)placed * NK, A.kc8, A.vc8, A.ksc, A.vsc,
                              whole, committed, committed / CUINF_KVGROUP, nkv, st));
            committed += whole * CUINF_KVGROUP;
            placed += whole * CUINF_KVGROUP;
            if (placed < S)
                PF(cuinf_kv_write_tail(k16 + (size_t)placed * NK, v16 + (size_t)placed * NK, A.ktail, A.vtail, 0,
                                       S - placed, nkv, vs));
            if (S >= PF_TC_MIN_ROWS && (nh / nkv == 1 || nh / nkv == 2 || nh / nkv == 4)) {
                const dim3 grid((S + APF_TOK - 1) / APF_TOK, nkv);
                const float sc = 1.0f / sqrtf((float)hd);
                if (nh / nkv == 4)
                    k_attn_prefill_mma<4><<<grid, 512, 0, st>>>(q16, A.kc8, A.vc8, A.ksc, A.vsc, A.ktail, A.vtail,
                                                                committed, past, S, sc, ao, nh, nkv);
                else if (nh / nkv == 2)
                    k_attn_prefill_mma<2><<<grid, 256, 0, st>>>(q16, A.kc8, A.vc8, A.ksc, A.vsc, A.ktail, A.vtail,
                                                                committed, past, S, sc, ao, nh, nkv);
                else
                    k_attn_prefill_mma<1><<<grid, 128, 0, st>>>(q16, A.kc8, A.vc8, A.ksc, A.vsc, A.ktail, A.vtail,
                                                                committed, past, S, sc, ao, nh, nkv);
            } else
                k_attn_prefill<<<dim3(S, nh), 32, 0, st>>>(q16, A.kc8, A.vc8, A.ksc, A.vsc, A.ktail, A.vtail,
                                                           committed, past, 1.0f / sqrtf((float)hd), ao, nh, nkv);
            PF(cuinf_launch_status());
            PF(pf_gemm(ao, L.wo.p, L.wo.s, fa, S, H, NQ, vs));
            PF(cuinf_add_f32_inplace(hs, fa, S * H, vs));
            }
        } else {
            PF(pf_gemm(xn, L.in_proj.p, L.in_proj.s, fa, S, 3 * H, H, vs));
            PF(cuinf_conv_pre(fa, t16, t16b, S, H, vs));
            PF(cuinf_conv_apply(t16b, t16, L.conv_w, s->conv_state[l], acc, S, H, vs));
            PF(cuinf_conv_update_state(t16b, s->conv_state[l], S, H, vs));
            PF(pf_gemm(acc, L.out_proj.p, L.out_proj.s, fa, S, H, H, vs));
            PF(cuinf_add_f32_inplace(hs, fa, S * H, vs));
        }
    ffn:
        PF(cuinf_rmsnorm(hs, L.ffn_norm, xn, S, H, c.norm_eps, vs));
        if (l < c.n_dense) {
            const int I = c.dense_inter;
            PF(pf_gemm(xn, L.w1.p, L.w1.s, fa, S, I, H, vs));
            PF(pf_gemm(xn, L.w3.p, L.w3.s, fb, S, I, H, vs));
            PF(cuinf_swiglu(fa, fb, t16, S * I, vs));
            PF(pf_gemm(t16, L.w2.p, L.w2.s, fa, S, H, I, vs));
            PF(cuinf_add_f32_inplace(hs, fa, S * H, vs));
        } else if (S >= PF_TC_MIN_ROWS) {
            // the prompt's tokens grouped by expert (each expert's weights streamed once per chunk);
            // experts of this layer into rw (free here), then into the [S][n_moe][K] layout
            int* rl = reinterpret_cast<int*>(rw);
            PF(moe_grouped_prefill(const_cast<cuinf_model*>(m), l, xn, hs, S, rl, st));
            CUINF_TRY(cudaMemcpy2DAsync(ridx + (size_t)L.moe_index * K, (size_t)n_moe * K * 4, rl, (size_t)K * 4,
                                        (size_t)K * 4, S, cudaMemcpyDeviceToDevice, st));
        } else {
            const void* const* ex = (const void* const*)(m->d_experts + (size_t)L.moe_index * E * 6);
            for (int i = 0; i < S; i++) {  // one token at a time, h_i += its expert mix (882-904)
                int* ri = ridx + ((size_t)i * n_moe + L.moe_index) * K;
                float* wi = rw + ((size_t)i * n_moe + L.moe_index) * K;
                PF(moe_ffn_launch(xn + (size_t)i * H, L.gate, L.ebias, ex, hs + (size_t)i * H, H, c.moe_inter,
                                  E, K, mid, ri, wi, st));
            }
        }
    }
    // compute_logits_last: final norm, lm_head and argmax of the last row
    const __half* last = hs + (size_t)(S - 1) * H;
    PF(cuinf_rmsnorm(last, m->emb_norm, xn, 1, H, c.norm_eps, vs));
    PF(cuinf_gemv_fp16(xn, m->embed, logits, 1, c.vocab, H, vs));
    PF(cuinf_argmax(logits, c.vocab, s->tok, vs));
    CUINF_TRY(cudaMemcpyAsync(s->out_ring + (past + S - 1) % s->max_ctx, s->tok, 4, cudaMemcpyDeviceToDevice, st));
    // session state for the decode steps that follow
    CUINF_TRY(cudaMemcpyAsync(s->h, last, (size_t)H * 2, cudaMemcpyDeviceToDevice, st));
    CUINF_TRY(cudaMemcpyAsync(s->hidden, last, (size_t)H * 2, cudaMemcpyDeviceToDevice, st));
    if (s->keep_logits)
        CUINF_TRY(cudaMemcpyAsync(s->logits, logits, (size_t)c.vocab * 4, cudaMemcpyDeviceToDevice, st));
    const int newpos = past + S;
    int* pin = &s->pinned[cuinf_session::kTokRing];
    *pin = newpos;
    CUINF_TRY(cudaMemcpyAsync(s->pos, pin, 4, cudaMemcpyHostToDevice, st));
    CUINF_TRY(cudaStreamSynchronize(st));
    s->host_pos = newpos;
    if (routes_out && n_moe > 0)
        CUINF_TRY(cudaMemcpy(routes_out, ridx, (size_t)S * n_moe * K * 4, cudaMemcpyDeviceToHost));
    if (out_token) CUINF_TRY(cudaMemcpy(out_token, s->tok, 4, cudaMemcpyDeviceToHost));
#undef PF
    return CUINF_OK;
}

extern "C" int cuinf_generate(cuinf_session* s, const int* prompt, int n_prompt, int n_new, int eos,
                              int* out_ids, int* n_out) {
    REQUIRE(s && prompt && out_ids && n_out && n_prompt > 0 && n_new > 0, "bad arguments");
    REQUIRE(s->host_pos + n_prompt + n_new - 1 <= s->max_ctx, "context too long for max_ctx");
    int next = -1, rc;
    if (s->prefill) {
        if ((rc = cuinf_prefill(s, prompt, n_prompt, &next, nullptr))) return rc;
    } else {
        for (int i = 0; i < n_prompt; i++) {
            rc = cuinf_decode_step(s, prompt[i], i == n_prompt - 1 ? &next : nullptr);
            if (rc) return rc;
        }
    }
    int n = 0;
    out_ids[n++] = next;
    // engine.cu:954-963: stop after n_new tokens or at EOS
    for (int step = 0; step < n_new - 1 && next != eos; step++) {
        rc = cuinf_decode_step(s, -1, &next);
        if (rc) return rc;
        out_ids[n++] = next;
        if (next == eos) break;
    }
    *n_out = n;
    return CUINF_OK;
}

// H2O eviction mode (engine.cu:579-581, 753-756): budget slots per attention
// layer, local window W (<= 0: budget/2).  Only before the first token.
extern "C" int cuinf_session_set_kv_budget(cuinf_session* s, int budget, int window) {
    REQUIRE(s, "null session");
    REQUIRE(s->host_pos == 0, "set the KV budget before the first token");
    REQUIRE(budget >= 0 && budget <= H2O_MAX_SLOTS, "budget must be in [0, 8192]");
    const cuinf_config& c = s->m->cfg;
    CUINF_TRY(cudaStreamSynchronize(s->st));
    for (auto& Z : s->h2o) {
        cudaFree(Z.hk8); cudaFree(Z.hv8); cudaFree(Z.hks); cudaFree(Z.hvs);
        cudaFree(Z.slot_pos); cudaFree(Z.attn_sum); cudaFree(Z.n_live);
    }
    s->h2o.clear();
    if (s->kv_new) cudaFree(s->kv_new);
    if (s->h2o_dst) cudaFree(s->h2o_dst);
    s->kv_new = nullptr;
    s->h2o_dst = nullptr;
    s->h2o_C = 0;
    if (budget > 0) {
        if (window <= 0) window = budget / 2;
        if (window >= budget) window = budget - 1;
        REQUIRE(window >= 1, "budget must be at least 2");
        const size_t row = (size_t)c.n_kv_heads * 64;
        s->h2o.assign(c.n_layers, cuinf_session::H2o());
        for (int l = 0; l < c.n_layers; l++) {
            if (!c.attn_layer[l]) continue;
            cuinf_session::H2o& Z = s->h2o[l];
            CUINF_TRY(cudaMalloc(&Z.hk8, budget * row));
            CUINF_TRY(cudaMalloc(&Z.hv8, budget * row));
            CUINF_TRY(cudaMalloc(&Z.hks, (size_t)budget * c.n_kv_heads * 2));
            CUINF_TRY(cudaMalloc(&Z.hvs, (size_t)budget * c.n_kv_heads * 2));
            CUINF_TRY(cudaMalloc(&Z.slot_pos, (size_t)budget * 4));
            CUINF_TRY(cudaMalloc(&Z.attn_sum, (size_t)budget * 4));
            CUINF_TRY(cudaMalloc(&Z.n_live, 4));
            CUINF_TRY(cudaMemset(Z.slot_pos, 0, (size_t)budget * 4));
            CUINF_TRY(cudaMemset(Z.attn_sum, 0, (size_t)budget * 4));
            CUINF_TRY(cudaMemset(Z.n_live, 0, 4));
        }
        CUINF_TRY(cudaMalloc(&s->kv_new, 2 * row * 2));
        CUINF_TRY(cudaMalloc(&s->h2o_dst, (size_t)c.n_layers * 4));
        CUINF_TRY(cudaMemset(s->h2o_dst, 0xff, (size_t)c.n_layers * 4));
        s->h2o_C = budget;
        s->h2o_W = window;
    }
    return build_graph(s);
}

// H2O state of one attention layer (host copies): slot positions and
// cumulative attention [budget], live slots, the slot of the last step.
extern "C" int cuinf_session_h2o_state(cuinf_session* s, int layer, int* slot_pos, float* attn_sum, int* n_live,
                                       int* last_slot) {
    REQUIRE(s && s->h2o_C, "no KV budget set");
    REQUIRE(layer >= 0 && layer < s->m->cfg.n_layers && s->m->cfg.attn_layer[layer], "not an attention layer");
    CUINF_TRY(cudaStreamSynchronize(s->st));
    const cuinf_session::H2o& Z = s->h2o[layer];
    if (slot_pos) CUINF_TRY(cudaMemcpy(slot_pos, Z.slot_pos, (size_t)s->h2o_C * 4, cudaMemcpyDeviceToHost));
    if (attn_sum) CUINF_TRY(cudaMemcpy(attn_sum, Z.attn_sum, (size_t)s->h2o_C * 4, cudaMemcpyDeviceToHost));
    if (n_live) CUINF_TRY(cudaMemcpy(n_live, Z.n_live, 4, cudaMemcpyDeviceToHost));
    if (last_slot) CUINF_TRY(cudaMemcpy(last_slot, s->h2o_dst + layer, 4, cudaMemcpyDeviceToHost));
    return CUINF_OK;
}

extern "C" int cuinf_session_keep_logits(cuinf_session* s, int on) {
    REQUIRE(s, "null session");
    if ((bool)on == s->keep_logits) return CUINF_OK;
    CUINF_TRY(cudaStreamSynchronize(s->st));
    s->keep_logits = on != 0;
    return build_graph(s);
}

extern "C" int cuinf_session_set_option(cuinf_session* s, int option, int value) {
    REQUIRE(s, "null session");
    if (option == CUINF_OPT_PREFILL) {  // host-side only, no graph rebuild
        s->prefill = value != 0;
        return CUINF_OK;
    }
    if (option == CUINF_OPT_PREFETCH_MB || option == CUINF_OPT_PREFETCH_AHEAD) {
        REQUIRE(option == CUINF_OPT_PREFETCH_MB ? (value >= 1 && value <= 1024) : (value >= 1 && value <= 64),
                "prefetch budget must be 1..1024 MB, look-ahead 1..64 launches");
        int& f = option == CUINF_OPT_PREFETCH_MB ? s->prefetch_mb : s->prefetch_ahead;
        if (f == value) return CUINF_OK;
        CUINF_TRY(cudaStreamSynchronize(s->st));
        f = value;
        return build_graph(s);
    }
    bool* f = option == CUINF_OPT_PREFETCH ? &s->prefetch
            : option == CUINF_OPT_PDL      ? &s->pdl
            : option == CUINF_OPT_MEGAKERNEL ? &s->use_mk
            : option == CUINF_OPT_TRACE      ? &s->trace
            : option == CUINF_OPT_ATTN_CLUSTER ? &s->attn_use_cluster
                                             : nullptr;
    REQUIRE(f, "unknown option");
    if ((bool)value == *f) return CUINF_OK;
    CUINF_TRY(cudaStreamSynchronize(s->st));
    *f = value != 0;
    return build_graph(s);
}

extern "C" int cuinf_session_attn_cluster(const cuinf_session* s) { return s && s->attn_cluster ? 1 : 0; }

extern "C" int cuinf_session_trace(cuinf_session* s, unsigned long long* buf, int cap, int* kinds,
                                   int* n_stages, int* n_ctas) {
    REQUIRE(s && buf && n_stages && n_ctas, "null pointer");
    REQUIRE(s->mk_ok && s->mk_trace, "no megakernel trace recorded (set CUINF_OPT_TRACE)");
    const int n = s->mk.n_stages, G = s->mk_grid;
    REQUIRE(cap >= n * G * MK_TRACE_W, "trace buffer too small");
    CUINF_TRY(cudaStreamSynchronize(s->st));
    CUINF_TRY(cudaMemcpy(buf, s->mk_trace, (size_t)n * G * MK_TRACE_W * 8, cudaMemcpyDeviceToHost));
    if (kinds)
        for (int i = 0; i < n; i++) kinds[i] = s->mk_kinds[i];
    *n_stages = n;
    *n_ctas = G;
    return CUINF_OK;
}

extern "C" int cuinf_session_uses_megakernel(const cuinf_session* s) {
    return s && !s->h2o_C && s->use_mk && s->mk_ok ? 1 : 0;
}

extern "C" int cuinf_session_error(cuinf_session* s, unsigned* flags) {
    REQUIRE(s && flags, "null pointer");
    unsigned w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (s->mk_words) {
        CUINF_TRY(cudaStreamSynchronize(s->st));
        CUINF_TRY(cudaMemcpy(w, s->mk_words, sizeof(w), cudaMemcpyDeviceToHost));
    }
    flags[0] = w[2] | (w[1] ? 1u : 0u);
    flags[1] = w[4];  // stage of the first failure
    flags[2] = w[5];  // CTA
    flags[3] = w[6];  // slab number
    return CUINF_OK;
}

extern "C" int cuinf_device_error(unsigned* flags) {
    REQUIRE(flags, "null pointer");
    unsigned v = 0;
    CUINF_TRY(cudaMemcpyFromSymbol(&v, g_engine_err, sizeof(v)));
    *flags = v;
    return CUINF_OK;
}

// Failure-path self test: one CTA arms an mbarrier for 16 bytes that no copy
// will ever deliver and waits on it with the given limit (the same bounded
// wait every staging kernel uses, there with a 4 s limit).  The wait gives
// up, records bit 0 in its own word and the kernel returns normally.
__global__ void k_wait_selftest(unsigned long long limit_ns, unsigned* word, unsigned long long* waited_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    mbar_arrive_expect_tx(&bar, 16);  // arrival done, 16 transaction bytes outstanding forever
    const uint64_t t0 = globaltimer_ns();
    const bool ok = mbar_wait_bounded_ns(&bar, 0, word, limit_ns);
    *waited_ns = globaltimer_ns() - t0;
    if (ok) atomicOr(word, 2u);  // the phase completed: must not happen
}

extern "C" int cuinf_selftest_wait_timeout(unsigned limit_us, unsigned* flags, unsigned long long* waited_ns) {
    REQUIRE(flags && waited_ns, "null pointer");
    REQUIRE(limit_us > 0 && limit_us <= 2000000u, "limit_us must be in (0, 2 s]");
    unsigned* d = nullptr;
    CUINF_TRY(cudaMalloc(&d, 16));
    cudaError_t e = cudaMemset(d, 0, 16);
    if (e == cudaSuccess) {
        k_wait_selftest<<<1, 32>>>((unsigned long long)limit_us * 1000ull, d, (unsigned long long*)(d + 2));
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    unsigned h[4] = {0, 0, 0, 0};
    if (e == cudaSuccess) e = cudaMemcpy(h, d, 16, cudaMemcpyDeviceToHost);
    cudaFree(d);
    CUINF_TRY(e);
    *flags = h[0];
    memcpy(waited_ns, &h[2], 8);
    return CUINF_OK;
}

extern "C" const float* cuinf_session_logits(const cuinf_session* s) { return s ? s->logits : nullptr; }
extern "C" const void* cuinf_session_hidden(const cuinf_session* s) { return s ? s->hidden : nullptr; }

extern "C" int cuinf_session_routes(cuinf_session* s, int* idx, float* w) {
    REQUIRE(s && idx && w, "null pointer");
    const size_t n = (size_t)std::max(1, s->m->n_moe * s->m->cfg.top_k);
    CUINF_TRY(cudaMemcpyAsync(idx, s->route_idx, n * 4, cudaMemcpyDeviceToHost, s->st));
    CUINF_TRY(cudaMemcpyAsync(w, s->route_w, n * 4, cudaMemcpyDeviceToHost, s->st));
    CUINF_TRY(cudaStreamSynchronize(s->st));
    return CUINF_OK;
}

extern "C" int cuinf_session_kernels_per_step(const cuinf_session* s) {
    return s ? s->kernels_per_step : -1;
}

extern "C" int cuinf_session_profile_step(cuinf_session* s, int token, int max_kernels, float* ms,
                                          double* bytes, char* names, int name_len, int* n_kernels) {
    REQUIRE(s && ms && bytes && n_kernels, "null pointer");
    REQUIRE(s->host_pos < s->max_ctx, "context full (max_ctx reached)");
    CUINF_TRY(cudaStreamSynchronize(s->st));
    if (token >= 0) {
        s->pinned[0] = token;  // the stream was synchronized above
        CUINF_TRY(cudaMemcpyAsync(s->tok, &s->pinned[0], 4, cudaMemcpyHostToDevice, s->st));
    }
    Prof prof;
    int rc = record_step(s, &prof);
    CUINF_TRY(cudaStreamSynchronize(s->st));
    s->host_pos++;
    const int n = (int)prof.ev.size() - 1;
    for (int i = 0; i < n && i < max_kernels; i++) {
        float t = 0.f;
        cudaEventElapsedTime(&t, prof.ev[i], prof.ev[i + 1]);
        ms[i] = t;
        bytes[i] = prof.bytes[i + 1];
        if (names && name_len > 0) {
            strncpy(names + (size_t)i * name_len, prof.name[i + 1], name_len - 1);
            names[(size_t)i * name_len + name_len - 1] = 0;
        }
    }
    for (cudaEvent_t e : prof.ev) cudaEventDestroy(e);
    *n_kernels = n;
    return rc;
}

#ifdef CUINF_PHASE_TRACE
// Diagnostic builds only: copies the phase timestamps of the latest launch of
// every decode-step kernel ([8 kernels][1024 CTAs][12] u64) to host memory.
extern "C" int cuinf_phase_trace_read(void* dst, size_t bytes) {
    REQUIRE(dst && bytes >= sizeof(g_phase), "buffer too small");
    CUINF_TRY(cudaMemcpyFromSymbol(dst, g_phase, sizeof(g_phase)));
    return CUINF_OK;
}
#endif
