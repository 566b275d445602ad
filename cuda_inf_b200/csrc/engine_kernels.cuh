// Fused decode-step kernels.  One token (batch 1) per launch chain; every
// kernel streams its INT4 weights once with 16-byte loads and dequantizes in
// registers (int4_tile_dot), and fuses the reference's small kernels
// (rmsnorm, f32_to_f16, qk-norm, rope, kv_write_tail, kv_commit_group,
// conv_pre/apply/update, swiglu, acc_scaled, add_*, argmax) into its
// prologue or epilogue.  Per step: 3 kernels per attention layer, 2 per conv
// layer, 2 per FFN, 1 lm_head (src/engine.cu:784-940 launches ~760).
#pragma once
#include <cooperative_groups.h>

#include "common.cuh"
#include "route.cuh"

namespace cg = cooperative_groups;

// Norm prologue: x = rmsnorm(src, w) into shared memory (fp16, natural order)
// and its B-fragment permutation xB.  src is the residual h, or the embedding
// row embed[*tok] for the first layer (then CTA 0 also stores it into h).
__device__ __forceinline__ void norm_prologue(const __half* __restrict__ h,
                                              const __half* __restrict__ embed,
                                              const int* __restrict__ tok, __half* h_store,
                                              const __half* __restrict__ w, int H, float eps,
                                              __half* xs, __half* xB, float* red) {
    const __half* src = h;
    if (embed) {
        src = embed + (size_t)(*tok) * H;
        if (blockIdx.x == 0 && blockIdx.y == 0)
            for (int i = threadIdx.x; i < H; i += blockDim.x) h_store[i] = src[i];
    }
    for (int i = threadIdx.x; i < H; i += blockDim.x) xs[i] = src[i];
    __syncthreads();
    rmsnorm_smem(xs, w, xs, H, eps, red);
    __syncthreads();
    for (int e = threadIdx.x; e < H / 4; e += blockDim.x) build_xB_entry(xs, xB, e);
    __syncthreads();
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
    int H, nh, nkv;
    float eps, theta;
};

__global__ void __cluster_dims__(4, 1, 1) __launch_bounds__(256) k_attn_qkv(QkvParams P) {
    extern __shared__ __align__(16) unsigned char smem[];
    __half* xs = reinterpret_cast<__half*>(smem);
    __half* xB = xs + P.H;
    float* red = reinterpret_cast<float*>(xB + P.H);  // [8][16] + 32
    float* res = red + 8 * 16 + 32;                   // [16] this CTA's rows
    float* head = res + 16;                           // [64] rank 0 only
    __half* hv = reinterpret_cast<__half*>(head + 64);  // [64]
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int hh = blockIdx.x >> 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    norm_prologue(P.h, P.embed, P.tok, P.h_store, P.norm_w, P.H, P.eps, xs, xB, red + 128);

    const uint8_t* wp;
    const __half* ws;
    int N, row0;
    if (hh < P.nh) { wp = P.wq_p; ws = P.wq_s; N = P.nh * CUINF_HD; row0 = hh * CUINF_HD; }
    else if (hh < P.nh + P.nkv) { wp = P.wk_p; ws = P.wk_s; N = P.nkv * CUINF_HD; row0 = (hh - P.nh) * CUINF_HD; }
    else { wp = P.wv_p; ws = P.wv_s; N = P.nkv * CUINF_HD; row0 = (hh - P.nh - P.nkv) * CUINF_HD; }
    row0 += rank * 16;
    float y0 = 0.f, y1 = 0.f;
    int4_tile_dot<2>(wp, ws, N, P.H, row0, warp, P.H >> 7, 8, reinterpret_cast<const uint2*>(xB), y0, y1);
    if ((lane & 3) == 0) {
        red[warp * 16 + (lane >> 2)] = y0;
        red[warp * 16 + (lane >> 2) + 8] = y1;
    }
    __syncthreads();
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

    const int pos = *P.pos;
    const int committed = (pos / CUINF_KVGROUP) * CUINF_KVGROUP;
    const int slot = pos - committed;
    const int d = threadIdx.x;
    const bool is_q = hh < P.nh, is_k = !is_q && hh < P.nh + P.nkv;
    if (d < 64) hv[d] = __float2half_rn(head[d]);  // f32_to_f16
    __syncthreads();
    if (is_q || is_k) {
        // rmsnorm_head (engine.cu:148-158), 64 threads
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
}

// ---------------------------------------------------------------------------
// Residual GEMV: h[n] = half(h[n] + (W . act)[n])  (out_proj of attention and
// conv layers, dense w2; engine.cu:858-859, 866-867, 875-876).  One 16-row
// tile per CTA, 8 warps interleaved over K groups.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_gemv_residual(const __half* __restrict__ act,
                                                       const uint8_t* __restrict__ wp,
                                                       const __half* __restrict__ ws,
                                                       __half* h, int N, int K) {
    extern __shared__ __align__(16) unsigned char smem[];
    __half* xB = reinterpret_cast<__half*>(smem);
    float* red = reinterpret_cast<float*>(xB + K);
    for (int e = threadIdx.x; e < K / 4; e += blockDim.x) build_xB_entry(act, xB, e);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, row0 = blockIdx.x * 16;
    float y0 = 0.f, y1 = 0.f;
    int4_tile_dot<2>(wp, ws, N, K, row0, warp, K >> 7, 8, reinterpret_cast<const uint2*>(xB), y0, y1);
    if ((lane & 3) == 0) {
        red[warp * 16 + (lane >> 2)] = y0;
        red[warp * 16 + (lane >> 2) + 8] = y1;
    }
    __syncthreads();
    if (threadIdx.x < 16) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++) s += red[w * 16 + threadIdx.x];
        const int n = row0 + threadIdx.x;
        if (n < N) h[n] = __float2half_rn(__half2float(h[n]) + s);
    }
}

// ---------------------------------------------------------------------------
// Short-conv layer input: in_proj rows {c, H+c, 2H+c} for 16 channels
// (B | C | x, engine.cu:861), then conv_pre/conv_apply/conv_update_state
// (engine.cu:483-525) in the epilogue.  12 warps: 4 per row tile.
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
};

__global__ void __launch_bounds__(384) k_conv_in(ConvParams P) {
    extern __shared__ __align__(16) unsigned char smem[];
    __half* xs = reinterpret_cast<__half*>(smem);
    __half* xB = xs + P.H;
    float* red = reinterpret_cast<float*>(xB + P.H);  // [12][16] + 32
    norm_prologue(P.h, P.embed, P.tok, P.h_store, P.norm_w, P.H, P.eps, xs, xB, red + 192);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = warp >> 2, c0 = blockIdx.x * 16;
    float y0 = 0.f, y1 = 0.f;
    int4_tile_dot<2>(P.wp, P.ws, 3 * P.H, P.H, tile * P.H + c0, warp & 3, P.H >> 7, 4,
                     reinterpret_cast<const uint2*>(xB), y0, y1);
    if ((lane & 3) == 0) {
        red[warp * 16 + (lane >> 2)] = y0;
        red[warp * 16 + (lane >> 2) + 8] = y1;
    }
    __syncthreads();
    if (threadIdx.x < 16) {
        const int i = threadIdx.x, c = c0 + i;
        float v[3];
#pragma unroll
        for (int t = 0; t < 3; t++)
            v[t] = red[(4 * t + 0) * 16 + i] + red[(4 * t + 1) * 16 + i] + red[(4 * t + 2) * 16 + i] +
                   red[(4 * t + 3) * 16 + i];
        const __half Cb = __float2half_rn(v[1]);
        const __half Bx = __float2half_rn(v[0] * v[2]);
        const float s0 = __half2float(P.state[c]), s1 = __half2float(P.state[P.H + c]);
        const float w0 = __half2float(P.conv_w[c * 3 + 0]), w1 = __half2float(P.conv_w[c * 3 + 1]),
                    w2 = __half2float(P.conv_w[c * 3 + 2]);
        const float co = s0 * w0 + s1 * w1 + __half2float(Bx) * w2;
        P.y[c] = __float2half_rn(__half2float(Cb) * co);
        P.state[c] = P.state[P.H + c];
        P.state[P.H + c] = Bx;
    }
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
};

__device__ __forceinline__ float silu_fast(float x) { return x / (1.f + __expf(-x)); }

__global__ void __launch_bounds__(256) k_ffn_up(FfnUpParams P) {
    extern __shared__ __align__(16) unsigned char smem[];
    __half* xs = reinterpret_cast<__half*>(smem);
    __half* xB = xs + P.H;
    float* red = reinterpret_cast<float*>(xB + P.H);
    norm_prologue(P.h, nullptr, nullptr, nullptr, P.norm_w, P.H, P.eps, xs, xB, red + 128);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, row0 = blockIdx.x * 16;
    const int tile = warp & 1;
    float y0 = 0.f, y1 = 0.f;
    int4_tile_dot<2>(tile ? P.w3p : P.w1p, tile ? P.w3s : P.w1s, P.I, P.H, row0, warp >> 1,
                     P.H >> 7, 4, reinterpret_cast<const uint2*>(xB), y0, y1);
    if ((lane & 3) == 0) {
        red[warp * 16 + (lane >> 2)] = y0;
        red[warp * 16 + (lane >> 2) + 8] = y1;
    }
    __syncthreads();
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
}

// ---------------------------------------------------------------------------
// MoE up: router (gate fp16 [E,H] . x) computed cooperatively by a cluster
// of 8 CTAs (DSMEM exchange of logits), device-side selection with the
// reference's rules (engine.cu:879-892), then this CTA's (rank slot t,
// 16-row tile) of experts' w1 and w3 -> mid[t*I + i] = half(silu(g) * u).
// ---------------------------------------------------------------------------
struct MoeUpParams {
    const __half* h;       // residual (normalized here) or, if xn != null, ignored
    const __half* xn;      // already-normalized input (standalone cuinf_moe_ffn)
    const __half* norm_w;
    const __half* gate;    // [E,H]
    const __half* bias;    // [E]
    const void* const* experts;  // [E][6]
    __half* xn_store;      // if set, CTA 0 stores the normalized x here
    __half* mid;           // [topk, I]
    int* route_idx;        // [topk]
    float* route_w;        // [topk]
    int H, I, E, topk;
    float eps;
};


__global__ void __cluster_dims__(8, 1, 1) __launch_bounds__(256) k_moe_up(MoeUpParams P) {
    extern __shared__ __align__(16) unsigned char smem[];
    __half* xs = reinterpret_cast<__half*>(smem);
    __half* xB = xs + P.H;
    float* red = reinterpret_cast<float*>(xB + P.H);  // [8][16] + 32
    float* lg_mine = red + 160;                       // [32]
    float* lg_all = lg_mine + 32;                     // [256]
    int* sidx = reinterpret_cast<int*>(lg_all + 256);  // [16]
    float* sw = reinterpret_cast<float*>(sidx + 16);   // [16]
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (P.xn) {
        for (int i = threadIdx.x; i < P.H; i += blockDim.x) xs[i] = P.xn[i];
        __syncthreads();
        for (int e = threadIdx.x; e < P.H / 4; e += blockDim.x) build_xB_entry(xs, xB, e);
        __syncthreads();
    } else {
        norm_prologue(P.h, nullptr, nullptr, nullptr, P.norm_w, P.H, P.eps, xs, xB, red + 128);
    }
    // router rows [rank*rpc, rank*rpc + rpc): one warp per row, CUDA cores
    const int rpc = (P.E + 7) / 8;
    for (int j = warp; j < rpc; j += 8) {
        const int e = rank * rpc + j;
        float acc = 0.f;
        if (e < P.E) {
            const __half* gr = P.gate + (size_t)e * P.H;
            for (int k = lane * 8; k < P.H; k += 256) {
                uint4 wv = *reinterpret_cast<const uint4*>(gr + k);
                uint4 xv = *reinterpret_cast<const uint4*>(xs + k);
                const __half2* w2 = reinterpret_cast<const __half2*>(&wv);
                const __half2* x2 = reinterpret_cast<const __half2*>(&xv);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    float2 a = __half22float2(w2[i]), b = __half22float2(x2[i]);
                    acc = fmaf(a.x, b.x, acc);
                    acc = fmaf(a.y, b.y, acc);
                }
            }
            acc = warp_sum(acc);
        }
        if (lane == 0) lg_mine[j] = acc;
    }
    cluster.sync();
    for (int e = threadIdx.x; e < P.E; e += blockDim.x) {
        const float* src = cluster.map_shared_rank(lg_mine, e / rpc);
        lg_all[e] = src[e % rpc];
    }
    cluster.sync();
    if (warp == 0) route_select_warp(lg_all, P.bias, P.E, P.topk, sidx, sw);
    __syncthreads();
    if (blockIdx.x == 0 && threadIdx.x < P.topk) {
        P.route_idx[threadIdx.x] = sidx[threadIdx.x];
        P.route_w[threadIdx.x] = sw[threadIdx.x];
    }
    if (blockIdx.x == 0 && P.xn_store)
        for (int i = threadIdx.x; i < P.H; i += blockDim.x) P.xn_store[i] = xs[i];

    const int tiles = P.I / 16;
    const int item = blockIdx.x;
    if (item >= P.topk * tiles) return;
    const int t = item / tiles, row0 = (item % tiles) * 16;
    const int e = sidx[t];
    const void* const* ex = P.experts + (size_t)e * 6;
    const int tile = warp & 1;
    const uint8_t* wp = (const uint8_t*)ex[tile ? 2 : 0];
    const __half* ws = (const __half*)ex[tile ? 3 : 1];
    float y0 = 0.f, y1 = 0.f;
    int4_tile_dot<2>(wp, ws, P.I, P.H, row0, warp >> 1, P.H >> 7, 4,
                     reinterpret_cast<const uint2*>(xB), y0, y1);
    __syncthreads();
    if ((lane & 3) == 0) {
        red[warp * 16 + (lane >> 2)] = y0;
        red[warp * 16 + (lane >> 2) + 8] = y1;
    }
    __syncthreads();
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
}

// ---------------------------------------------------------------------------
// MoE down: rows [16b, 16b+16) of every selected expert's w2 . mid[t], then
// acc = half(acc + w_t * o_t) in rank order and h = half(h + acc)
// (engine.cu:900-904, acc_scaled 556-559, add_inplace 527-530).
// ---------------------------------------------------------------------------
struct MoeDownParams {
    const __half* mid;  // [topk, I]
    const void* const* experts;
    const int* route_idx;
    const float* route_w;
    __half* h;
    int H, I, topk;
};

__global__ void __launch_bounds__(256) k_moe_down(MoeDownParams P) {
    extern __shared__ __align__(16) unsigned char smem[];
    __half* xB = reinterpret_cast<__half*>(smem);          // [topk][I]
    float* red = reinterpret_cast<float*>(xB + (size_t)P.topk * P.I);  // [8][topk][16]
    for (int e = threadIdx.x; e < P.topk * (P.I / 4); e += blockDim.x) {
        const int t = e / (P.I / 4), r = e % (P.I / 4);
        build_xB_entry(P.mid + (size_t)t * P.I, xB + (size_t)t * P.I, r);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, row0 = blockIdx.x * 16;
    const int KG = P.I >> 7;
    for (int t = 0; t < P.topk; t++) {
        const void* const* ex = P.experts + (size_t)P.route_idx[t] * 6;
        float y0 = 0.f, y1 = 0.f;
        int4_tile_dot<2>((const uint8_t*)ex[4], (const __half*)ex[5], P.H, P.I, row0, warp, KG, 8,
                         reinterpret_cast<const uint2*>(xB + (size_t)t * P.I), y0, y1);
        if ((lane & 3) == 0) {
            red[(warp * P.topk + t) * 16 + (lane >> 2)] = y0;
            red[(warp * P.topk + t) * 16 + (lane >> 2) + 8] = y1;
        }
    }
    __syncthreads();
    if (threadIdx.x < 16) {
        const int i = threadIdx.x, n = row0 + i;
        __half acc = __float2half_rn(0.f);
        for (int t = 0; t < P.topk; t++) {
            float o = 0.f;
#pragma unroll
            for (int w = 0; w < 8; w++) o += red[(w * P.topk + t) * 16 + i];
            acc = __float2half_rn(__half2float(acc) + P.route_w[t] * o);
        }
        if (n < P.H) P.h[n] = __float2half_rn(__half2float(P.h[n]) + __half2float(acc));
    }
}

// ---------------------------------------------------------------------------
// Final norm + tied lm_head (fp16 [V,H]) + argmax + next-token bookkeeping
// (engine.cu:932-940).  One 16-row tile per warp, all tiles resident in one
// wave.  Argmax: 64-bit keys (argmax_key) reduced per CTA, then atomicMax;
// the last CTA (atomic ticket) publishes the token, advances pos and resets.
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
};

__global__ void __launch_bounds__(256) k_lmhead(LmHeadParams P) {
    extern __shared__ __align__(16) unsigned char smem[];
    __half* xs = reinterpret_cast<__half*>(smem);
    float* red = reinterpret_cast<float*>(xs + P.H);
    __shared__ unsigned long long kred[8];
    __shared__ int s_last;
    for (int i = threadIdx.x; i < P.H; i += blockDim.x) xs[i] = P.h[i];
    __syncthreads();
    if (blockIdx.x == 0 && P.hidden_out)
        for (int i = threadIdx.x; i < P.H; i += blockDim.x) P.hidden_out[i] = xs[i];
    rmsnorm_smem(xs, P.norm_w, xs, P.H, P.eps, red);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = (P.V + 15) / 16;
    unsigned long long best = 0ull;
    for (int tile = blockIdx.x * 8 + warp; tile < ntiles; tile += gridDim.x * 8) {
        float y0 = 0.f, y1 = 0.f;
        f16_tile_dot<4>(P.W, P.V, P.H, tile * 16, 0, P.H >> 5, 1, xs, y0, y1);
        const int r0 = tile * 16 + (lane >> 2), r1 = r0 + 8;
        if ((lane & 3) == 0) {
            if (r0 < P.V) {
                if (P.logits) P.logits[r0] = y0;
                if (y0 > -1e30f) best = umax64_dev(best, argmax_key(y0 == 0.f ? 0.f : y0, r0));
            }
            if (r1 < P.V) {
                if (P.logits) P.logits[r1] = y1;
                if (y1 > -1e30f) best = umax64_dev(best, argmax_key(y1 == 0.f ? 0.f : y1, r1));
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = umax64_dev(best, __shfl_xor_sync(0xffffffffu, best, o));
    if (lane == 0) kred[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long b = 0ull;
#pragma unroll
        for (int w = 0; w < 8; w++) b = umax64_dev(b, kred[w]);
        if (b) atomicMax(P.key, b);
        __threadfence();
        unsigned prev = atomicAdd(P.ticket, 1u);
        s_last = prev == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last || threadIdx.x != 0) return;
    __threadfence();
    const unsigned long long k = atomicExch(P.key, 0ull);
    const int token = k ? argmax_key_index(k) : 0;
    const int pos = *P.pos;
    *P.tok = token;
    if (P.out_ring) P.out_ring[pos % P.ring] = token;
    *P.pos = pos + 1;
    *P.ticket = 0u;
}
