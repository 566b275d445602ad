// Fused decode-step kernels.  One token (batch 1) per launch chain.
//
// Every weight-streaming kernel follows the same schedule:
//   1. thread 0 stages the CTA's weight tiles (16 rows x full K, packed
//      nibbles + fp16 scales, the tools/export_weights.py layout) into
//      shared memory with TMA bulk copies tracked by one mbarrier, and pulls
//      the weights of the kernels after it into L2;
//   2. griddepcontrol.launch_dependents, so the next kernel of the step
//      (launched with programmatic serialization) can start its own step 1
//      while this one runs;
//   3. griddepcontrol.wait: only now read what earlier kernels wrote;
//   4. prologue (RMSNorm of the residual, x permuted to B-fragment order),
//      wait for the tiles, dequantize in registers and run mma.m16n8k16
//      (fp32 accumulate) per 128-wide group, scale, reduce across warps;
//   5. fused epilogue replacing the reference's small kernels (f32_to_f16,
//      rmsnorm_head, rope, kv_write_tail, kv_commit_group, conv_pre/apply/
//      update_state, swiglu, acc_scaled, add_*, argmax).
// Per step: 3 kernels per attention layer, 2 per conv layer, 2 per FFN and
// one lm_head (src/engine.cu:784-940 launches ~760 plus 24 host syncs).
#pragma once
#include <cooperative_groups.h>

#include "common.cuh"
#include "route.cuh"

namespace cg = cooperative_groups;

// Device-side error word of this translation unit: bit 0 = an mbarrier wait
// timed out (its kernel then skipped its math).
static __device__ unsigned g_engine_err;

// Norm prologue: x = rmsnorm(src, w) (rmsnorm, engine.cu:131-144) into shared
// memory (fp16, natural order) and its B-fragment permutation xB.  src is the
// residual h, or the embedding row embed[*tok] for the first layer (then CTA 0
// also stores it into h).
// The norm weight is a static tensor, so each thread
// loads its 8-element chunks of it before the dependency wait (norm_w_load);
// after the wait, norm_prologue_fast reads its chunks of src once, reduces the
// sum of squares with one block barrier, and writes both xs and the two
// B-fragment entries its chunk forms (8 consecutive elements k0..k0+7 are
// entries m = 2j, 2j+1 of quad c of group G for k0 = 128G + 32c + 8j).
// H % 8 == 0 and H <= 16 * blockDim.x.
struct NormW {
    uint4 w[2];
};
__device__ __forceinline__ void norm_w_load(NormW& nw, const __half* __restrict__ w, int H) {
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const int i = threadIdx.x + r * blockDim.x;
        nw.w[r] = i < (H >> 3) ? ldg_stream(w + 8 * i) : make_uint4(0u, 0u, 0u, 0u);
    }
}
__device__ __forceinline__ void norm_prologue_fast(const NormW& nw, const __half* __restrict__ h,
                                                   const __half* __restrict__ embed,
                                                   const int* __restrict__ tok, __half* h_store, int H,
                                                   float eps, __half* xs, __half* xB, float* red) {
    const __half* src = h;
    if (embed) {
        src = embed + (size_t)(*tok) * H;
        if (h_store && blockIdx.x == 0 && blockIdx.y == 0)
            for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8)
                *reinterpret_cast<uint4*>(h_store + i) = *reinterpret_cast<const uint4*>(src + i);
    }
    const int n8 = H >> 3;
    uint4 v[2];
    float ss = 0.f;
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const int i = threadIdx.x + r * blockDim.x;
        if (i < n8) {
            v[r] = *reinterpret_cast<const uint4*>(src + 8 * i);
            const __half2* h2 = reinterpret_cast<const __half2*>(&v[r]);
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const float2 f = __half22float2(h2[q]);
                ss = fmaf(f.x, f.x, ss);
                ss = fmaf(f.y, f.y, ss);
            }
        }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) tot += red[i];
    const float inv = rsqrtf(tot / (float)H + eps);
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const int i = threadIdx.x + r * blockDim.x;
        if (i < n8) {
            const __half* xh = reinterpret_cast<const __half*>(&v[r]);
            const __half* wh = reinterpret_cast<const __half*>(&nw.w[r]);
            __align__(16) __half o[8];
#pragma unroll
            for (int q = 0; q < 8; q++) o[q] = __float2half_rn(__half2float(xh[q]) * inv * __half2float(wh[q]));
            *reinterpret_cast<uint4*>(xs + 8 * i) = *reinterpret_cast<const uint4*>(o);
            if (xB) {
                const int G = i >> 4, c = (i >> 2) & 3, j = i & 3;
                __half2* e0 = reinterpret_cast<__half2*>(xB + (size_t)((G * 8 + 2 * j) * 4 + c) * 4);
                __half2* e1 = reinterpret_cast<__half2*>(xB + (size_t)((G * 8 + 2 * j + 1) * 4 + c) * 4);
                e0[0] = __halves2half2(o[0], o[4]);
                e0[1] = __halves2half2(o[1], o[5]);
                e1[0] = __halves2half2(o[2], o[6]);
                e1[1] = __halves2half2(o[3], o[7]);
            }
        }
    }
    __syncthreads();
}

// A CTA may touch another cluster member's shared memory only once that member
// has started: every CTA arrives (relaxed) on the cluster barrier at its
// start, and waits on it right before its first remote access; by then the
// wait is normally already satisfied.
__device__ __forceinline__ void cluster_arrive_started() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_started() {
    asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");
}

// Stage begin: mbarrier init by thread 0, made visible to the CTA.
__device__ __forceinline__ void stage_begin(uint64_t* bar) {
    if (threadIdx.x == 0) mbar_init(bar, 1);
    __syncthreads();
}
// Wait for the staged tiles; false (and the error bit) on time-out.
__device__ __forceinline__ bool stage_wait(uint64_t* bar) {
    return mbar_wait_bounded(bar, 0, &g_engine_err);
}

__device__ __forceinline__ void warp_partials(float* red, int warp, float y0, float y1) {
    const int lane = threadIdx.x & 31;
    if ((lane & 3) == 0) {
        red[warp * 16 + (lane >> 2)] = y0;
        red[warp * 16 + (lane >> 2) + 8] = y1;
    }
}

// ---------------------------------------------------------------------------
// Attention q/k/v projection + QK-RMSNorm + RoPE + KV append (+ FP8 commit).
// grid: 4 CTAs (one cluster) per output head: nh q heads, nkv k heads, nkv v
// heads.  CTA rank r computes rows [16r, 16r+16) of its head; rank 0 gathers
// the head's 64 values over DSMEM and runs the epilogue
// (engine.cu:792-845: f32_to_f16, rmsnorm_head, rope, kv_write_tail,
// kv_commit_group when the 64-token tail fills).
// ---------------------------------------------------------------------------
struct QkvParams {
    const __half* h;
    const __half* embed;  // non-null on layer 0
    const int* tok;
    __half* h_store;
    const __half* norm_w;
    const uint8_t *wq_p, *wk_p, *wv_p;
    const __half *wq_s, *wk_s, *wv_s;
    const __half *q_ln, *k_ln;
    const int* pos;
    __half* q_out;
    __half *ktail, *vtail;
    uint8_t *kc8, *vc8;
    __half *ksc, *vsc;
    __half* kv_new;  // H2O mode: the token's K [nkv][64] then V [nkv][64] here, no tail/commit
    int H, nh, nkv;
    float eps, theta;
    L2Ranges next;
};

__host__ __device__ inline size_t qkv_smem(int H) {
    return int4_tile_bytes(H) + (size_t)H * 4 + (160 + 16 + 64) * 4 + 128;
}

__global__ void __cluster_dims__(4, 1, 1) __launch_bounds__(256) k_attn_qkv(QkvParams P) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t bar;
    uint8_t* tile = smem;
    __half* xs = reinterpret_cast<__half*>(smem + int4_tile_bytes(P.H));
    __half* xB = xs + P.H;
    float* red = reinterpret_cast<float*>(xB + P.H);  // [8][16] + 32
    float* res = red + 160;                           // [16] this CTA's rows
    float* head = res + 16;                           // [64] rank 0 only
    __half* hv = reinterpret_cast<__half*>(head + 64);  // [64]
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int hh = blockIdx.x >> 2;
    const int warp = threadIdx.x >> 5;
    PHASE(PH_QKV, 0);

    const uint8_t* wp;
    const __half* ws;
    int row0;
    if (hh < P.nh) { wp = P.wq_p; ws = P.wq_s; row0 = hh * CUINF_HD; }
    else if (hh < P.nh + P.nkv) { wp = P.wk_p; ws = P.wk_s; row0 = (hh - P.nh) * CUINF_HD; }
    else { wp = P.wv_p; ws = P.wv_s; row0 = (hh - P.nh - P.nkv) * CUINF_HD; }
    row0 += rank * 16;
    stage_begin(&bar);
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&bar, int4_tile_bytes(P.H));
        tma_tile_int4(wp, ws, P.H, row0, tile, &bar);
        l2_prefetch_share(P.next, blockIdx.x, gridDim.x);
    }
    NormW nw;
    norm_w_load(nw, P.norm_w, P.H);
    pdl_trigger();
    pdl_wait();
    PHASE(PH_QKV, 1);
    norm_prologue_fast(nw, P.h, P.embed, P.tok, P.h_store, P.H, P.eps, xs, xB, red + 128);
    PHASE(PH_QKV, 2);
    float y0 = 0.f, y1 = 0.f;
    if (stage_wait(&bar))
        int4_tile_dot_smem<2>(tile, P.H, warp, P.H >> 7, 8, reinterpret_cast<const uint2*>(xB), y0, y1);
    warp_partials(red, warp, y0, y1);
    __syncthreads();
    PHASE(PH_QKV, 4);
    if (threadIdx.x < 16) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++) s += red[w * 16 + threadIdx.x];
        res[threadIdx.x] = s;
    }
    cluster.sync();
    if (rank == 0 && threadIdx.x < 64) {
        const float* rr = cluster.map_shared_rank(res, threadIdx.x >> 4);
        head[threadIdx.x] = rr[threadIdx.x & 15];
    }
    cluster.sync();
    if (rank != 0) return;
    PHASE(PH_QKV, 5);

    const int pos = *P.pos;
    const int committed = (pos / CUINF_KVGROUP) * CUINF_KVGROUP;
    const int slot = pos - committed;
    const int d = threadIdx.x;
    const bool is_q = hh < P.nh, is_k = !is_q && hh < P.nh + P.nkv;
    if (d < 64) hv[d] = __float2half_rn(head[d]);  // f32_to_f16
    __syncthreads();
    if (is_q || is_k) {
        // rmsnorm_head (engine.cu:148-158)
        float v = d < 64 ? __half2float(hv[d]) : 0.f;
        float ss = block_sum(v * v, red + 128);
        float inv = rsqrtf(ss / 64.f + P.eps);
        const __half* lw = is_q ? P.q_ln : P.k_ln;
        __half nv = __float2half_rn(v * inv * __half2float(lw[d < 64 ? d : 0]));
        __syncthreads();
        if (d < 64) hv[d] = nv;
        __syncthreads();
        // rope (engine.cu:161-182)
        if (d < 32) {
            float invf = powf(P.theta, -(float)(2 * d) / (float)CUINF_HD);
            float ang = (float)pos * invf;
            float cs = cosf(ang), sn = sinf(ang);
            float x0 = __half2float(hv[d]), x1 = __half2float(hv[d + 32]);
            __half o0 = __float2half_rn(x0 * cs - x1 * sn);
            __half o1 = __float2half_rn(x1 * cs + x0 * sn);
            hv[d] = o0;
            hv[d + 32] = o1;
        }
        __syncthreads();
    }
    if (is_q) {
        if (d < 64) P.q_out[(size_t)hh * CUINF_HD + d] = hv[d];
        return;
    }
    const int kvh = is_k ? hh - P.nh : hh - P.nh - P.nkv;
    if (P.kv_new) {
        if (d < 64) P.kv_new[((is_k ? 0 : P.nkv) + kvh) * CUINF_HD + d] = hv[d];
        return;
    }
    __half* tail = is_k ? P.ktail : P.vtail;
    if (d < 64) tail[((size_t)slot * P.nkv + kvh) * CUINF_HD + d] = hv[d];  // kv_write_tail
    if (slot == CUINF_KVGROUP - 1) {  // kv_commit_group for this head
        __syncthreads();
        uint8_t* c8 = is_k ? P.kc8 : P.vc8;
        __half* sc = is_k ? P.ksc : P.vsc;
        const int grp = committed / CUINF_KVGROUP;
        float mx = 0.f;
        for (int e = threadIdx.x; e < CUINF_KVGROUP * CUINF_HD; e += blockDim.x) {
            int t = e >> 6, dd = e & 63;
            mx = fmaxf(mx, fabsf(__half2float(tail[((size_t)t * P.nkv + kvh) * CUINF_HD + dd])));
        }
        mx = warp_max(mx);
        __syncthreads();
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
        __syncthreads();
        float amax = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) amax = fmaxf(amax, red[i]);
        const float s = amax / 448.0f + 1e-12f;
        if (threadIdx.x == 0) sc[grp * P.nkv + kvh] = __float2half_rn(s);
        for (int e = threadIdx.x; e < CUINF_KVGROUP * CUINF_HD; e += blockDim.x) {
            int t = e >> 6, dd = e & 63;
            float v = __half2float(tail[((size_t)t * P.nkv + kvh) * CUINF_HD + dd]);
            c8[((size_t)(committed + t) * P.nkv + kvh) * CUINF_HD + dd] =
                (uint8_t)__nv_cvt_float_to_fp8(v / s, __NV_SATFINITE, __NV_E4M3);
        }
    }
    PHASE(PH_QKV, 9);
}

// ---------------------------------------------------------------------------
// Residual GEMV: h[n] = half(h[n] + (W . act)[n])  (out_proj of attention and
// conv layers, dense w2; engine.cu:858-859, 866-867, 875-876).  One 16-row
// tile per CTA, 8 warps interleaved over the K groups.
// ---------------------------------------------------------------------------
struct ResParams {
    const __half* act;
    const uint8_t* wp;
    const __half* ws;
    __half* h;
    int N, K;
    L2Ranges next;
};

#define RES_WARPS 16  // 16 warps per SM keep the mma.sync dot fed (8 warps reach ~3/4 of the pace)
__host__ __device__ inline size_t res_smem(int K) {
    return int4_tile_bytes(K) + (size_t)K * 2 + RES_WARPS * 16 * 4;
}

__global__ void __launch_bounds__(RES_WARPS * 32) k_gemv_residual(ResParams P) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t bar;
    uint8_t* tile = smem;
    __half* xB = reinterpret_cast<__half*>(smem + int4_tile_bytes(P.K));
    float* red = reinterpret_cast<float*>(xB + P.K);
    const int warp = threadIdx.x >> 5, row0 = blockIdx.x * 16;
    PHASE(PH_RES, 0);
    stage_begin(&bar);
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&bar, int4_tile_bytes(P.K));
        tma_tile_int4(P.wp, P.ws, P.K, row0, tile, &bar);
        l2_prefetch_share(P.next, blockIdx.x, gridDim.x);
    }
    pdl_trigger();
    pdl_wait();
    PHASE(PH_RES, 1);
    for (int i = threadIdx.x; i < P.K / 8; i += blockDim.x) build_xB_chunk(P.act, xB, i);
    __syncthreads();
    PHASE(PH_RES, 2);
    float y0 = 0.f, y1 = 0.f;
    if (stage_wait(&bar))
        int4_tile_dot_smem<2>(tile, P.K, warp, P.K >> 7, RES_WARPS, reinterpret_cast<const uint2*>(xB), y0, y1);
    warp_partials(red, warp, y0, y1);
    __syncthreads();
    PHASE(PH_RES, 4);
    if (threadIdx.x < 16) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < RES_WARPS; w++) s += red[w * 16 + threadIdx.x];
        const int n = row0 + threadIdx.x;
        if (n < P.N) P.h[n] = __float2half_rn(__half2float(P.h[n]) + s);
    }
    PHASE(PH_RES, 9);
}

// ---------------------------------------------------------------------------
// Short-conv layer input: in_proj rows {c, H+c, 2H+c} for 16 channels
// (B | C | x, engine.cu:861), then conv_pre/conv_apply/conv_update_state
// (engine.cu:483-525) in the epilogue.  24 warps: 8 per row tile.
// ---------------------------------------------------------------------------
struct ConvParams {
    const __half* h;
    const __half* embed;
    const int* tok;
    __half* h_store;
    const __half* norm_w;
    const uint8_t* wp;
    const __half* ws;
    const __half* conv_w;  // [H,3]
    __half* state;         // [2,H]
    __half* y;             // [H]
    int H;
    float eps;
    L2Ranges next;
};

#define CONV_WARPS 24
__host__ __device__ inline size_t conv_smem(int H) {
    return 3 * (size_t)int4_tile_bytes(H) + (size_t)H * 4 + (CONV_WARPS * 16 + 32) * 4;
}

__global__ void __launch_bounds__(CONV_WARPS * 32) k_conv_in(ConvParams P) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t bar;
    const uint32_t TB = int4_tile_bytes(P.H);
    uint8_t* tiles = smem;
    __half* xs = reinterpret_cast<__half*>(smem + 3 * TB);
    __half* xB = xs + P.H;
    float* red = reinterpret_cast<float*>(xB + P.H);  // [24][16] + 32
    const int warp = threadIdx.x >> 5;
    const int tile = warp >> 3, c0 = blockIdx.x * 16;
    PHASE(PH_CONV, 0);
    stage_begin(&bar);
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&bar, 3 * TB);
        for (int t = 0; t < 3; t++) tma_tile_int4(P.wp, P.ws, P.H, t * P.H + c0, tiles + t * TB, &bar);
        l2_prefetch_share(P.next, blockIdx.x, gridDim.x);
    }
    NormW nw;
    norm_w_load(nw, P.norm_w, P.H);
    // the conv taps and the two history rows of this CTA's 16 channels are
    // read before the dependency wait: the taps are static and the state was
    // last written by this layer's conv_in of the previous step
    float cw0 = 0.f, cw1 = 0.f, cw2 = 0.f, cs0 = 0.f;
    __half cs1 = __float2half_rn(0.f);
    if (threadIdx.x < 16) {
        const int c = c0 + threadIdx.x;
        cw0 = __half2float(P.conv_w[c * 3 + 0]);
        cw1 = __half2float(P.conv_w[c * 3 + 1]);
        cw2 = __half2float(P.conv_w[c * 3 + 2]);
        cs0 = __half2float(P.state[c]);
        cs1 = P.state[P.H + c];
    }
    pdl_trigger();
    pdl_wait();
    PHASE(PH_CONV, 1);
    norm_prologue_fast(nw, P.h, P.embed, P.tok, P.h_store, P.H, P.eps, xs, xB, red + CONV_WARPS * 16);
    PHASE(PH_CONV, 2);
    float y0 = 0.f, y1 = 0.f;
    if (stage_wait(&bar))
        int4_tile_dot_smem<2>(tiles + tile * TB, P.H, warp & 7, P.H >> 7, 8,
                              reinterpret_cast<const uint2*>(xB), y0, y1);
    warp_partials(red, warp, y0, y1);
    __syncthreads();
    PHASE(PH_CONV, 4);
    if (threadIdx.x < 16) {
        const int i = threadIdx.x, c = c0 + i;
        float v[3];
#pragma unroll
        for (int t = 0; t < 3; t++) {
            v[t] = 0.f;
#pragma unroll
            for (int w = 0; w < 8; w++) v[t] += red[(8 * t + w) * 16 + i];
        }
        const __half Cb = __float2half_rn(v[1]);
        const __half Bx = __float2half_rn(v[0] * v[2]);
        const float co = cs0 * cw0 + __half2float(cs1) * cw1 + __half2float(Bx) * cw2;
        P.y[c] = __float2half_rn(__half2float(Cb) * co);
        P.state[c] = cs1;
        P.state[P.H + c] = Bx;
    }
    PHASE(PH_CONV, 9);
}

// ---------------------------------------------------------------------------
// Dense FFN up: rows i of w1 and w3 -> mid[i] = half(silu(g) * u)
// (engine.cu:872-874 + swiglu 542-547).  8 warps: 4 per row tile.
// ---------------------------------------------------------------------------
struct FfnUpParams {
    const __half* h;
    const __half* norm_w;
    const uint8_t *w1p, *w3p;
    const __half *w1s, *w3s;
    __half* mid;
    int H, I;
    float eps;
    L2Ranges next;
};

__host__ __device__ inline size_t ffn_up_smem(int H) {
    return 2 * (size_t)int4_tile_bytes(H) + (size_t)H * 4 + (128 + 32) * 4;
}

__device__ __forceinline__ float silu_fast(float x) { return x / (1.f + __expf(-x)); }

__global__ void __launch_bounds__(256) k_ffn_up(FfnUpParams P) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t bar;
    const uint32_t TB = int4_tile_bytes(P.H);
    uint8_t* tiles = smem;
    __half* xs = reinterpret_cast<__half*>(smem + 2 * TB);
    __half* xB = xs + P.H;
    float* red = reinterpret_cast<float*>(xB + P.H);
    const int warp = threadIdx.x >> 5, row0 = blockIdx.x * 16;
    const int tile = warp & 1;
    PHASE(PH_FFN, 0);
    stage_begin(&bar);
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&bar, 2 * TB);
        tma_tile_int4(P.w1p, P.w1s, P.H, row0, tiles, &bar);
        tma_tile_int4(P.w3p, P.w3s, P.H, row0, tiles + TB, &bar);
        l2_prefetch_share(P.next, blockIdx.x, gridDim.x);
    }
    NormW nw;
    norm_w_load(nw, P.norm_w, P.H);
    pdl_trigger();
    pdl_wait();
    PHASE(PH_FFN, 1);
    norm_prologue_fast(nw, P.h, nullptr, nullptr, nullptr, P.H, P.eps, xs, xB, red + 128);
    PHASE(PH_FFN, 2);
    float y0 = 0.f, y1 = 0.f;
    if (stage_wait(&bar))
        int4_tile_dot_smem<2>(tiles + tile * TB, P.H, warp >> 1, P.H >> 7, 4,
                              reinterpret_cast<const uint2*>(xB), y0, y1);
    warp_partials(red, warp, y0, y1);
    __syncthreads();
    PHASE(PH_FFN, 4);
    if (threadIdx.x < 16) {
        const int i = threadIdx.x, r = row0 + i;
        float g = 0.f, u = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w += 2) {
            g += red[w * 16 + i];
            u += red[(w + 1) * 16 + i];
        }
        if (r < P.I) P.mid[r] = __float2half_rn(silu_fast(g) * u);
    }
    PHASE(PH_FFN, 9);
}

// ---------------------------------------------------------------------------
// MoE up: the router gate (fp16 [E,H]) is split over a cluster of 8 CTAs
// (each stages its rows with TMA before the dependency wait) and the logits
// are exchanged over DSMEM; device-side selection with the reference's rules
// (engine.cu:879-892); then this CTA's (rank slot t, 16-row tile) of the
// selected expert's w1 and w3 -> mid[t*I + i] = half(silu(g) * u).  The
// selected experts' w2 (for moe_down) is pulled into L2 across the grid.
// ---------------------------------------------------------------------------
struct MoeUpParams {
    const __half* h;       // residual (normalized here) or, if xn != null, ignored
    const __half* xn;      // already-normalized input (standalone cuinf_moe_ffn)
    const __half* norm_w;
    const __half* gate;    // [E,H]
    const __half* bias;    // [E]
    const void* const* experts;  // [E][6]
    __half* mid;           // [topk, I]
    int* route_idx;        // [topk]
    float* route_w;        // [topk]
    int H, I, E, topk;
    float eps;
    L2Ranges next;         // static weights of the kernels after moe_down
};

// The gate rows are consumed before the expert tiles arrive, so both share
// the first region (keeps 448 CTAs resident in one wave on 148 SMs).
__host__ __device__ inline size_t moe_up_stage_bytes(int H, int E) {
    const size_t gate = (size_t)((E + 7) / 8) * H * 2, tiles = 2 * (size_t)int4_tile_bytes(H);
    return gate > tiles ? gate : tiles;
}
// + the router bias (E <= 256 halves) and the expert pointer table [E][6],
// both static, copied to shared memory before the dependency wait so the
// selection and the route-dependent copies read no global memory.
__host__ __device__ inline size_t moe_up_smem(int H, int E) {
    return moe_up_stage_bytes(H, E) + (size_t)H * 4 + (160 + 32 + 256 + 32) * 4 + 512 + (size_t)E * 6 * 8;
}

__global__ void __cluster_dims__(8, 1, 1) __launch_bounds__(256) k_moe_up(MoeUpParams P) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t bar[2];
    const int rpc = (P.E + 7) / 8;
    const uint32_t TB = int4_tile_bytes(P.H);
    uint8_t* tiles = smem;
    __half* gs = reinterpret_cast<__half*>(smem);  // [rpc][H] gate rows, then the tiles
    __half* xs = reinterpret_cast<__half*>(smem + moe_up_stage_bytes(P.H, P.E));
    __half* xB = xs + P.H;
    float* red = reinterpret_cast<float*>(xB + P.H);  // [8][16] + 32
    float* lg_mine = red + 160;                       // [32]
    float* lg_all = lg_mine + 32;                     // [256]
    int* sidx = reinterpret_cast<int*>(lg_all + 256);  // [16]
    float* sw = reinterpret_cast<float*>(sidx + 16);   // [16]
    __half* sbias = reinterpret_cast<__half*>(sw + 16);  // [E]
    const void** stab = reinterpret_cast<const void**>(reinterpret_cast<unsigned char*>(sbias) + 512);  // [E][6]
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e0 = rank * rpc, ne = max(0, min(P.E - e0, rpc));
    cluster_arrive_started();
    PHASE(PH_MOE_UP, 0);

    if (threadIdx.x == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&bar[0], (uint32_t)ne * P.H * 2);
        if (ne > 0) tma_load_1d(gs, P.gate + (size_t)e0 * P.H, (uint32_t)ne * P.H * 2, &bar[0]);
        l2_prefetch_share(P.next, blockIdx.x, gridDim.x);
    }
    NormW nw;
    if (!P.xn) norm_w_load(nw, P.norm_w, P.H);
    for (int i = threadIdx.x; i < P.E; i += blockDim.x) sbias[i] = P.bias[i];
    for (int i = threadIdx.x; i < P.E * 6; i += blockDim.x) stab[i] = P.experts[i];
    pdl_trigger();
    pdl_wait();
    PHASE(PH_MOE_UP, 1);
    if (P.xn) {
        for (int i = threadIdx.x; i < P.H; i += blockDim.x) xs[i] = P.xn[i];
        __syncthreads();
        for (int e = threadIdx.x; e < P.H / 4; e += blockDim.x) build_xB_entry(xs, xB, e);
        __syncthreads();
    } else {
        norm_prologue_fast(nw, P.h, nullptr, nullptr, nullptr, P.H, P.eps, xs, xB, red + 128);
    }
    PHASE(PH_MOE_UP, 2);
    // router rows of this cluster member: one warp per half row, from smem
    const bool gate_ok = stage_wait(&bar[0]);
    PHASE(PH_MOE_UP, 3);
    float* lgp = red;  // [2*rpc] half-row partials
    for (int item = warp; item < 2 * rpc; item += 8) {
        const int j = item >> 1;
        float acc = 0.f;
        if (j < ne && gate_ok) {
            const int half = P.H >> 1, k0 = (item & 1) * half;
            const __half* gr = gs + (size_t)j * P.H + k0;
            for (int k = lane * 8; k < half; k += 256) {
                uint4 wv = *reinterpret_cast<const uint4*>(gr + k);
                uint4 xv = *reinterpret_cast<const uint4*>(xs + k0 + k);
                const __half2* w2 = reinterpret_cast<const __half2*>(&wv);
                const __half2* x2 = reinterpret_cast<const __half2*>(&xv);
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    float2 a = __half22float2(w2[q]), b = __half22float2(x2[q]);
                    acc = fmaf(a.x, b.x, acc);
                    acc = fmaf(a.y, b.y, acc);
                }
            }
            acc = warp_sum(acc);
        }
        if (lane == 0) lgp[item] = acc;
    }
    __syncthreads();
    // scatter this member's logits into every member's lg_all (DSMEM), then
    // one cluster barrier: every member then holds all E logits
    cluster_wait_started();
    for (int i = threadIdx.x; i < rpc * 8; i += blockDim.x) {
        const int j = i % rpc, r = i / rpc;
        if (j < ne) cluster.map_shared_rank(lg_all, r)[e0 + j] = lgp[2 * j] + lgp[2 * j + 1];
    }
    cluster.sync();
    PHASE(PH_MOE_UP, 4);
    // scratch for the selection: the gate rows' region, consumed by now (the
    // expert tiles are staged into it only after the selection)
    route_select_block(lg_all, sbias, P.E, P.topk, sidx, sw, reinterpret_cast<float*>(gs));
    if (blockIdx.x == 0 && threadIdx.x < P.topk) {
        P.route_idx[threadIdx.x] = sidx[threadIdx.x];
        P.route_w[threadIdx.x] = sw[threadIdx.x];
    }
    PHASE(PH_MOE_UP, 5);
    const int tiles_per = P.I / 16;
    const int item = blockIdx.x;
    const bool active = item < P.topk * tiles_per;
    const int t = active ? item / tiles_per : 0, row0 = active ? (item % tiles_per) * 16 : 0;
    const void* const* ex = stab + (size_t)sidx[t] * 6;
    if (threadIdx.x == 0 && active) {
        mbar_arrive_expect_tx(&bar[1], 2 * TB);
        tma_tile_int4((const uint8_t*)ex[0], (const __half*)ex[1], P.H, row0, tiles, &bar[1]);
        tma_tile_int4((const uint8_t*)ex[2], (const __half*)ex[3], P.H, row0, tiles + TB, &bar[1]);
    }
    PHASE(PH_MOE_UP, 6);
    // the selected experts' w2 (read by moe_down next) into L2, over the
    // grid, issued by another warp than the one that issued the tiles
    auto prefetch_w2 = [&]() {
        if (threadIdx.x != 32) return;
        L2Ranges R;
        R.count = 0;
        for (int k = 0; k < P.topk && R.count < 7; k++) {
            const void* const* e2 = stab + (size_t)sidx[k] * 6;
            R.p[R.count] = (const char*)e2[4];
            R.n[R.count++] = (unsigned long long)P.H * (P.I >> 1);
            R.p[R.count] = (const char*)e2[5];
            R.n[R.count++] = (unsigned long long)P.H * (P.I >> 6);
        }
        l2_prefetch_share(R, blockIdx.x, gridDim.x);
    };
    prefetch_w2();
    if (!active) return;
    const int tile = warp & 1;
    float y0 = 0.f, y1 = 0.f;
    const bool tiles_ok = stage_wait(&bar[1]);
    PHASE(PH_MOE_UP, 7);
    if (tiles_ok)
        int4_tile_dot_smem<2>(tiles + tile * TB, P.H, warp >> 1, P.H >> 7, 4,
                              reinterpret_cast<const uint2*>(xB), y0, y1);
    __syncthreads();
    warp_partials(red, warp, y0, y1);
    __syncthreads();
    PHASE(PH_MOE_UP, 8);
    if (threadIdx.x < 16) {
        const int i = threadIdx.x;
        float g = 0.f, u = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w += 2) {
            g += red[w * 16 + i];
            u += red[(w + 1) * 16 + i];
        }
        P.mid[(size_t)t * P.I + row0 + i] = __float2half_rn(silu_fast(g) * u);
    }
    PHASE(PH_MOE_UP, 9);
}

// ---------------------------------------------------------------------------
// MoE down: rows [16b, 16b+16) of every selected expert's w2 . mid[t], then
// acc = half(acc + w_t * o_t) in rank order and h = half(h + acc)
// (engine.cu:900-904, acc_scaled 556-559, add_inplace 527-530).  The expert
// ids come from moe_up, so the tiles are staged after the dependency wait.
// ---------------------------------------------------------------------------
struct MoeDownParams {
    const __half* mid;  // [topk, I]
    const void* const* experts;
    const int* route_idx;
    const float* route_w;
    __half* h;
    int H, I, topk;
    L2Ranges next;
};

// One cluster of topk CTAs per 16 output rows: CTA t (cluster rank t) stages
// and multiplies only expert t's w2 tile against mid[t], and sends its 16
// outputs to rank 0 over DSMEM; rank 0 adds them in rank order.  The four
// tiles are fetched and multiplied by four SMs at once instead of one after
// another.  Launch: grid (H/16)*topk, cluster (topk, 1, 1), topk <= 8.
__host__ __device__ inline size_t moe_down_smem(int I, int topk) {
    return (size_t)int4_tile_bytes(I) + (size_t)I * 2 + (8 * 16 + 8 * 16) * 4;
}

__global__ void __launch_bounds__(256) k_moe_down(MoeDownParams P) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t bar;
    const uint32_t TB = int4_tile_bytes(P.I);
    uint8_t* tile = smem;
    __half* xB = reinterpret_cast<__half*>(smem + TB);          // [I]
    float* red = reinterpret_cast<float*>(xB + P.I);            // [8][16]
    float* slots = red + 8 * 16;                                // [topk][16], used in rank 0
    cg::cluster_group cluster = cg::this_cluster();
    const int t = (int)cluster.block_rank();
    const int row0 = (blockIdx.x / P.topk) * 16;
    const int warp = threadIdx.x >> 5;
    cluster_arrive_started();
    PHASE(PH_MOE_DOWN, 0);
    stage_begin(&bar);
    if (threadIdx.x == 0) l2_prefetch_share(P.next, blockIdx.x, gridDim.x);
    pdl_trigger();
    pdl_wait();
    PHASE(PH_MOE_DOWN, 1);
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&bar, TB);
        const void* const* ex = P.experts + (size_t)P.route_idx[t] * 6;
        tma_tile_int4((const uint8_t*)ex[4], (const __half*)ex[5], P.I, row0, tile, &bar);
    }
    // mid[t] into B-fragment order, 8 consecutive elements per thread
    const __half* src = P.mid + (size_t)t * P.I;
    for (int i = threadIdx.x; i < (P.I >> 3); i += blockDim.x) {
        const uint4 v = *reinterpret_cast<const uint4*>(src + 8 * i);
        const __half* o = reinterpret_cast<const __half*>(&v);
        const int G = i >> 4, c = (i >> 2) & 3, j = i & 3;
        __half2* e0 = reinterpret_cast<__half2*>(xB + (size_t)((G * 8 + 2 * j) * 4 + c) * 4);
        __half2* e1 = reinterpret_cast<__half2*>(xB + (size_t)((G * 8 + 2 * j + 1) * 4 + c) * 4);
        e0[0] = __halves2half2(o[0], o[4]);
        e0[1] = __halves2half2(o[1], o[5]);
        e1[0] = __halves2half2(o[2], o[6]);
        e1[1] = __halves2half2(o[3], o[7]);
    }
    __syncthreads();
    PHASE(PH_MOE_DOWN, 2);
    float y0 = 0.f, y1 = 0.f;
    if (stage_wait(&bar))
        int4_tile_dot_smem<2>(tile, P.I, warp, P.I >> 7, 8, reinterpret_cast<const uint2*>(xB), y0, y1);
    warp_partials(red, warp, y0, y1);
    __syncthreads();
    cluster_wait_started();
    if (threadIdx.x < 16) {
        float o = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++) o += red[w * 16 + threadIdx.x];
        float* dst = cluster.map_shared_rank(slots, 0);
        dst[t * 16 + threadIdx.x] = o;
    }
    cluster.sync();
    PHASE(PH_MOE_DOWN, 4);
    if (t == 0 && threadIdx.x < 16) {
        const int n = row0 + threadIdx.x;
        __half acc = __float2half_rn(0.f);
        for (int k = 0; k < P.topk; k++)
            acc = __float2half_rn(__half2float(acc) + P.route_w[k] * slots[k * 16 + threadIdx.x]);
        P.h[n] = __float2half_rn(__half2float(P.h[n]) + __half2float(acc));
    }
    PHASE(PH_MOE_DOWN, 9);
}

// ---------------------------------------------------------------------------
// Final norm + tied lm_head (fp16 [V,H]) + argmax + next-token bookkeeping
// (engine.cu:932-940).  Persistent: one CTA per SM owns a contiguous run of
// vocabulary rows.  Warp 8 streams the rows into a ring of LM_NST 32 KB
// stages with bulk copies; it starts before the dependency wait (the
// weights are static), so the first stages are in flight while the
// previous kernel finishes.  Warps 0-7 normalise h and take the stage's
// rows round-robin: one row per warp at a time, 16-byte chunks per lane,
// fp32 products (exact for fp16 operands) summed in fp32.  Argmax: 64-bit
// keys (argmax_key) reduced per CTA, then atomicMax; the last CTA (atomic
// ticket) publishes the token, advances pos and resets.
// ---------------------------------------------------------------------------
struct LmHeadParams {
    const __half* h;
    const __half* norm_w;
    const __half* W;  // [V,H]
    float* logits;    // optional [V]
    __half* hidden_out;  // optional [H] (final pre-norm hidden)
    unsigned long long* key;  // zero between steps
    unsigned* ticket;         // zero between steps
    int* tok;                 // next input token
    int* pos;                 // advanced by one
    int* out_ring;            // optional [ring], out_ring[pos % ring] = token
    int ring;
    int H, V;
    float eps;
    L2Ranges next;  // the first kernels of the next step
};

#define LM_STAGE_BYTES 32768
#define LM_NST 4
#define LM_WARPS 8  // row warps; warp LM_WARPS streams the weights
#define LM_THREADS ((LM_WARPS + 1) * 32)
// Rows per stage (H <= 16384, H % 8 == 0: the host checks).
__host__ __device__ inline int lmhead_rows_per_stage(int H) { return LM_STAGE_BYTES / (2 * H); }
__host__ __device__ inline size_t lmhead_smem(int H) {
    return (size_t)LM_NST * LM_STAGE_BYTES + (size_t)H * 2 + 64 * 4;
}
// barrier of the row warps only (the streaming warp is not part of it)
__device__ __forceinline__ void lm_sync() { asm volatile("bar.sync 1, %0;\n" ::"n"(LM_WARPS * 32) : "memory"); }

__global__ void __launch_bounds__(LM_THREADS, 1) k_lmhead(LmHeadParams P) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t full[LM_NST], empty[LM_NST];
    __shared__ unsigned long long kred[LM_WARPS];
    __shared__ int s_last;
    unsigned char* ring = smem;
    __half* xs = reinterpret_cast<__half*>(smem + (size_t)LM_NST * LM_STAGE_BYTES);
    float* red = reinterpret_cast<float*>(xs + P.H);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rps = lmhead_rows_per_stage(P.H);
    const int nst = (P.V + rps - 1) / rps;
    const int s0 = (int)((long long)nst * blockIdx.x / gridDim.x);
    const int s1 = (int)((long long)nst * (blockIdx.x + 1) / gridDim.x);
    if (threadIdx.x == 0) {
        for (int i = 0; i < LM_NST; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], LM_WARPS);
        }
    }
    __syncthreads();
    pdl_trigger();
    PHASE(PH_LMHEAD, 0);
    if (warp == LM_WARPS) {
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_first();
            int last[LM_NST];
            for (int i = 0; i < LM_NST; i++) last[i] = -1;
            for (int j = 0; j < s1 - s0; j++) {
                const int slot = j % LM_NST;
                if (j >= LM_NST && !mbar_wait_bounded(&empty[slot], ((j / LM_NST) - 1) & 1, &g_engine_err)) break;
                const int r0 = (s0 + j) * rps, nr = min(rps, P.V - r0);
                mbar_arrive_expect_tx(&full[slot], (uint32_t)nr * P.H * 2);
                tma_load_1d_hint(ring + (size_t)slot * LM_STAGE_BYTES, P.W + (size_t)r0 * P.H,
                                 (uint32_t)nr * P.H * 2, &full[slot], pol);
                last[slot] = j;
                if (j == LM_NST - 1) l2_prefetch_share(P.next, blockIdx.x, gridDim.x);
            }
            if (s1 - s0 < LM_NST) l2_prefetch_share(P.next, blockIdx.x, gridDim.x);
            // copies still in flight land before the CTA can exit
            for (int i = 0; i < LM_NST; i++)
                if (last[i] >= 0) mbar_wait_bounded(&full[i], (last[i] / LM_NST) & 1, &g_engine_err);
        }
        return;
    }
    // the norm weight (static) is read before the dependency wait; h and the
    // weight move in 16-byte chunks, two per thread at H <= 4096
    const int n8 = P.H >> 3;
    uint4 nwv[2];
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const int i = threadIdx.x + r * LM_WARPS * 32;
        nwv[r] = i < n8 ? ldg_stream(P.norm_w + 8 * i) : make_uint4(0u, 0u, 0u, 0u);
    }
    pdl_wait();
    PHASE(PH_LMHEAD, 1);
    {  // rmsnorm (engine.cu:131-144) into xs; block 0 also keeps the raw h
        float ss = 0.f;
        for (int i = threadIdx.x; i < n8; i += LM_WARPS * 32) {
            const uint4 v = *reinterpret_cast<const uint4*>(P.h + 8 * i);
            *reinterpret_cast<uint4*>(xs + 8 * i) = v;
            if (blockIdx.x == 0 && P.hidden_out) *reinterpret_cast<uint4*>(P.hidden_out + 8 * i) = v;
            const __half* e = reinterpret_cast<const __half*>(&v);
#pragma unroll
            for (int q = 0; q < 8; q++) {
                const float f = __half2float(e[q]);
                ss = fmaf(f, f, ss);
            }
        }
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        lm_sync();
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < LM_WARPS; w++) t += red[w];
        const float inv = rsqrtf(t / (float)P.H + P.eps);
        for (int i = threadIdx.x, r = 0; i < n8; i += LM_WARPS * 32, r++) {
            const uint4 v = *reinterpret_cast<const uint4*>(xs + 8 * i);
            const uint4 wv = r == 0 ? nwv[0] : r == 1 ? nwv[1] : ldg_stream(P.norm_w + 8 * i);
            const __half* xe = reinterpret_cast<const __half*>(&v);
            const __half* we = reinterpret_cast<const __half*>(&wv);
            __align__(16) __half o[8];
#pragma unroll
            for (int q = 0; q < 8; q++) o[q] = __float2half_rn(__half2float(xe[q]) * inv * __half2float(we[q]));
            *reinterpret_cast<uint4*>(xs + 8 * i) = *reinterpret_cast<const uint4*>(o);
        }
        lm_sync();
    }
    PHASE(PH_LMHEAD, 2);
    unsigned long long best = 0ull;
    for (int j = 0; j < s1 - s0; j++) {
        const int slot = j % LM_NST;
        if (!mbar_wait_bounded(&full[slot], (j / LM_NST) & 1, &g_engine_err)) break;
        const int r0 = (s0 + j) * rps, nr = min(rps, P.V - r0);
        const __half* st = reinterpret_cast<const __half*>(ring + (size_t)slot * LM_STAGE_BYTES);
        for (int r = warp; r < nr; r += LM_WARPS) {
            const __half* wr = st + (size_t)r * P.H;
            float acc = 0.f;
            for (int k = lane * 8; k < P.H; k += 256) {
                const uint4 wv = *reinterpret_cast<const uint4*>(wr + k);
                const uint4 xv = *reinterpret_cast<const uint4*>(xs + k);
                const __half2* w2 = reinterpret_cast<const __half2*>(&wv);
                const __half2* x2 = reinterpret_cast<const __half2*>(&xv);
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const float2 a = __half22float2(w2[q]), b = __half22float2(x2[q]);
                    acc = fmaf(a.x, b.x, acc);
                    acc = fmaf(a.y, b.y, acc);
                }
            }
            acc = warp_sum(acc);
            const int row = r0 + r;
            if (lane == 0) {
                if (P.logits) P.logits[row] = acc;
                if (acc > -1e30f) best = umax64_dev(best, argmax_key(acc == 0.f ? 0.f : acc, row));
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }
    if (lane == 0) kred[warp] = best;
    PHASE(PH_LMHEAD, 3);
    lm_sync();
    if (threadIdx.x == 0) {
        unsigned long long b = 0ull;
#pragma unroll
        for (int w = 0; w < LM_WARPS; w++) b = umax64_dev(b, kred[w]);
        if (b) atomicMax(P.key, b);
        __threadfence();
        unsigned prev = atomicAdd(P.ticket, 1u);
        s_last = prev == gridDim.x - 1;
    }
    lm_sync();
    if (!s_last || threadIdx.x != 0) return;
    __threadfence();
    const unsigned long long k = atomicExch(P.key, 0ull);
    const int token = k ? argmax_key_index(k) : 0;
    const int pos = *P.pos;
    *P.tok = token;
    if (P.out_ring) P.out_ring[pos % P.ring] = token;
    *P.pos = pos + 1;
    *P.ticket = 0u;
    PHASE(PH_LMHEAD, 9);
}
