// Fused MoE FFN decode layer, batch 1: router, selection, every selected
// expert's w1/w3 + SwiGLU and its w2 in ONE kernel (engine.cu:877-904:
// gemv_fp16 router, host top-k, per expert gemv w1/w3, swiglu, gemv w2,
// acc_scaled, add_inplace).
//
// Work split: CTA (t, r) computes intermediate rows [16r, 16r+16) of the
// expert in rank slot t (grid topk * I/16, 8 warps, small shared memory, so
// several CTAs share an SM and a launch can start beside its predecessor).
// A cluster of 8 CTAs covers 128 consecutive intermediate rows of one expert,
// i.e. one 128-wide scale group of w2's K dimension.  The cluster
//   * splits the router gate rows 8 ways and exchanges the logits (DSMEM),
//   * all-gathers its 128 SwiGLU values (DSMEM), and
//   * splits the H output rows of the down projection 8 ways: member m
//     multiplies rows [m*H/8, (m+1)*H/8) of w2, columns of this group (64
//     contiguous bytes per row, fetched right after the selection together
//     with the w1/w3 tiles), by the 128 values.
// The partial down sums are added into per-slot accumulators in global
// memory as 64-bit fixed-point integers (2^-32 units): integer addition does
// not depend on the order the clusters arrive in, so results are
// bit-identical from run to run.  The last cluster to finish an eighth of the
// outputs (atomic ticket) converts each slot's sum back to fp32 (o_t of the
// reference, up to fp32 summation order), applies acc = half(acc + w_t * o_t)
// in rank order and h = half(h + acc), and clears the accumulators and its
// ticket for the next layer.
#pragma once
#include "engine_kernels.cuh"

#define MOEF_THREADS 256
#define MOEF_CL 8      // cluster: 8 x 16 intermediate rows = one 128-wide w2 scale group
#define MOEF_EMAX 64   // experts the fused kernel handles (logits and bias arrays in smem)

struct MoeFusedParams {
    const __half* h;             // residual: normalized here (unless xn) and read by the finalizers
    const __half* xn;            // already-normalized input (standalone cuinf_moe_ffn), or null
    __half* h_out;               // updated residual (may alias h)
    const __half* norm_w;
    const __half* gate;          // [E,H]
    const __half* bias;          // [E]
    const void* const* experts;  // [E][6] {w1.p, w1.s, w3.p, w3.s, w2.p, w2.s}
    int* route_idx;              // [topk]
    float* route_w;              // [topk]
    unsigned long long* acc;     // [topk][H] fixed-point sums: zero on entry, left zero
    unsigned* tickets;           // [MOEF_CL]: zero on entry, left zero
    int H, I, E, topk;
    float eps;
    L2Ranges next;
};

struct MoefLayout {
    size_t stage, xs, misc, total;
};
// stage: the router rows of this member, then the w1/w3 tiles; xs: x and its
// B-fragment order; misc: reductions, logits, routes, the gathered SwiGLU
// values and their B-fragment order, the bias and the expert pointer table.
// The w2 slice is not staged: it is pulled into L2 at selection time and the
// down product reads it from there.
__host__ __device__ inline MoefLayout moef_layout(int H, int E) {
    MoefLayout L;
    const size_t tiles = 2 * (size_t)int4_tile_bytes(H);
    const size_t gate = (size_t)((E + MOEF_CL - 1) / MOEF_CL) * H * 2;
    L.stage = 0;
    L.xs = (((tiles > gate ? tiles : gate) + 127) / 128) * 128;
    L.misc = L.xs + (size_t)H * 4;
    // red 128 f, nred 16 f, lgp 32 f, lg_all 64 f, sidx 8 i, sw 8 f,
    // midall 128 h, xBm 128 h, sbias 64 h, stab E*6 pointers
    L.total = L.misc + (128 + 16 + 32 + 64 + 8 + 8) * 4 + (128 + 128 + 64) * 2 + (size_t)E * 6 * 8 + 64;
    return L;
}

// Whether the fused kernel can run this MoE shape (else: k_moe_up + k_moe_down).
__host__ inline bool moef_supported(int H, int I, int E, int topk) {
    return E <= MOEF_EMAX && E % 8 == 0 && topk <= 8 && I % 128 == 0 && H % (16 * MOEF_CL) == 0 && H % 128 == 0 &&
           H <= 16 * MOEF_THREADS && (E + MOEF_CL - 1) / MOEF_CL <= 8 && moef_layout(H, E).total <= 227 * 1024;
}

__device__ __forceinline__ void cp_async16_hint(void* smem_dst, const void* gsrc, uint64_t pol) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem_dst)),
                 "l"(gsrc), "l"(pol)
                 : "memory");
}
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }
__device__ __forceinline__ void red_add_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void prefetch_l2_line(const void* p) {
    asm volatile("prefetch.global.L2 [%0];\n" ::"l"(p));
}
__device__ __forceinline__ unsigned long long ld_cg_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.global.cg.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// (4 CTAs per SM, so that a whole grid of topk * I/16 = 448 CTAs is resident
// at once on 148 SMs: a second wave would hold up every ticket)
__global__ void __cluster_dims__(MOEF_CL, 1, 1) __launch_bounds__(MOEF_THREADS, 4) k_moe_fused(MoeFusedParams P) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t bar[2];  // [0] router rows, [1] w1/w3 tiles
    __shared__ int s_last;
    const MoefLayout Lo = moef_layout(P.H, P.E);
    const int H = P.H, I = P.I;
    const uint32_t TB = int4_tile_bytes(H);
    uint8_t* tiles = smem + Lo.stage;
    __half* gs = reinterpret_cast<__half*>(smem + Lo.stage);
    __half* xs = reinterpret_cast<__half*>(smem + Lo.xs);
    __half* xB = xs + H;
    float* red = reinterpret_cast<float*>(smem + Lo.misc);  // [8][16]
    float* nred = red + 128;                                // [16]
    float* lgp = nred + 16;                                 // [32]
    float* lg_all = lgp + 32;                               // [64]
    int* sidx = reinterpret_cast<int*>(lg_all + 64);        // [8]
    float* sw = reinterpret_cast<float*>(sidx + 8);         // [8]
    __half* midall = reinterpret_cast<__half*>(sw + 8);     // [128] the cluster's SwiGLU values
    __half* xBm = midall + 128;                             // [128] their B-fragment order
    __half* sbias = xBm + 128;                              // [64]
    const void** stab = reinterpret_cast<const void**>(sbias + 64);  // [E][6]
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_per = I / 16;
    const int t = blockIdx.x / tiles_per, row0 = (blockIdx.x % tiles_per) * 16;
    const int grp = row0 / 128;                             // this cluster's w2 scale group
    const int rpc = (P.E + MOEF_CL - 1) / MOEF_CL, e0 = rank * rpc, ne = max(0, min(P.E - e0, rpc));
    const int rows = H / MOEF_CL, n0 = rank * rows;         // this member's down-projection rows
    cluster_arrive_started();
    PHASE(PH_MOE_UP, 0);

    // ---- before the dependency wait: static data only ----
    if (threadIdx.x == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&bar[0], (uint32_t)ne * H * 2);
        if (ne > 0) tma_load_1d(gs, P.gate + (size_t)e0 * H, (uint32_t)ne * H * 2, &bar[0]);
        l2_prefetch_share(P.next, blockIdx.x, gridDim.x);
    }
    // the router bias and the expert pointer table by asynchronous copies
    // (the selection reads them from shared memory)
    if (threadIdx.x < (P.E * 2 + 15) / 16)
        cp_async16(reinterpret_cast<char*>(sbias) + 16 * threadIdx.x,
                   reinterpret_cast<const char*>(P.bias) + 16 * threadIdx.x);
    for (int i = threadIdx.x; i < P.E * 6 * 8 / 16; i += blockDim.x)
        cp_async16(reinterpret_cast<char*>(stab) + 16 * i, reinterpret_cast<const char*>(P.experts) + 16 * i);
    cp_async_commit();
    NormW nw;
    if (!P.xn) norm_w_load(nw, P.norm_w, H);
    pdl_trigger();
    pdl_wait();
    PHASE(PH_MOE_UP, 1);

    // ---- RMSNorm of the residual (rmsnorm, engine.cu:131-144) ----
    if (P.xn) {
        for (int i = threadIdx.x; i < H; i += blockDim.x) xs[i] = P.xn[i];
        __syncthreads();
        for (int e = threadIdx.x; e < H / 4; e += blockDim.x) build_xB_entry(xs, xB, e);
        __syncthreads();
    } else {
        norm_prologue_fast(nw, P.h, nullptr, nullptr, nullptr, H, P.eps, xs, xB, nred);
    }
    PHASE(PH_MOE_UP, 2);

    // ---- router logits (gemv_fp16, engine.cu:879): this member's rows, one
    // warp per half row ----
    const bool gate_ok = stage_wait(&bar[0]);
    for (int item = warp; item < 2 * rpc; item += MOEF_THREADS / 32) {
        const int j = item >> 1;
        float acc = 0.f;
        if (j < ne && gate_ok) {
            const int half = H >> 1, k0 = (item & 1) * half;
            const __half* gr = gs + (size_t)j * H + k0;
            for (int k = lane * 8; k < half; k += 256) {
                const uint4 wv = *reinterpret_cast<const uint4*>(gr + k);
                const uint4 xv = *reinterpret_cast<const uint4*>(xs + k0 + k);
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
        }
        if (lane == 0) lgp[item] = acc;
    }
    __syncthreads();
    cluster_wait_started();
    for (int i = threadIdx.x; i < rpc * MOEF_CL; i += blockDim.x) {
        const int j = i % rpc, r = i / rpc;
        if (j < ne) cluster.map_shared_rank(lg_all, r)[e0 + j] = lgp[2 * j] + lgp[2 * j + 1];
    }
    cp_async_wait_all();  // bias and pointer table (each thread its own copies; the barrier below publishes them)
    cluster.sync();
    PHASE(PH_MOE_UP, 3);

    // ---- selection (engine.cu:883-892) ----
    route_select_block(lg_all, sbias, P.E, P.topk, sidx, sw, lgp, PH_MOE_UP);
    if (blockIdx.x == 0 && threadIdx.x < P.topk) {
        P.route_idx[threadIdx.x] = sidx[threadIdx.x];
        P.route_w[threadIdx.x] = sw[threadIdx.x];
    }
    PHASE(PH_MOE_UP, 4);

    // ---- this CTA's weights: the w1/w3 tile (TMA); its rows of the w2
    // group slice (64 contiguous bytes per row) and their scale rows into L2 ----
    const void* const* ex = stab + (size_t)sidx[t] * 6;
    const uint8_t* w2p = (const uint8_t*)ex[4];
    const __half* w2s = (const __half*)ex[5];
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&bar[1], 2 * TB);
        tma_tile_int4((const uint8_t*)ex[0], (const __half*)ex[1], H, row0, tiles, &bar[1]);
        tma_tile_int4((const uint8_t*)ex[2], (const __half*)ex[3], H, row0, tiles + TB, &bar[1]);
    }
    // (per-thread prefetches through the load/store unit: hundreds of tiny
    // bulk prefetches would queue ahead of the tile copies in the TMA unit)
    for (int j = threadIdx.x; j < rows; j += blockDim.x) {
        prefetch_l2_line(w2p + (size_t)(n0 + j) * (I >> 1) + grp * 64);
        prefetch_l2_line(w2s + (size_t)(n0 + j) * (I >> 7) + grp);
    }
    PHASE(PH_MOE_UP, 5);

    // ---- w1/w3 dot + SwiGLU (swiglu, engine.cu:542-547) ----
    {
        const int tile = warp & 1;
        float y0 = 0.f, y1 = 0.f;
        if (stage_wait(&bar[1]))
            int4_tile_dot_smem<2>(tiles + tile * TB, H, warp >> 1, H >> 7, 4, reinterpret_cast<const uint2*>(xB),
                                  y0, y1);
        warp_partials(red, warp, y0, y1);
    }
    __syncthreads();
    PHASE(PH_MOE_UP, 6);
    if (threadIdx.x < 16) {
        const int i = threadIdx.x;
        float g = 0.f, u = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w += 2) {
            g += red[w * 16 + i];
            u += red[(w + 1) * 16 + i];
        }
        const __half m = __float2half_rn(silu_fast(g) * u);
        for (int r = 0; r < MOEF_CL; r++) cluster.map_shared_rank(midall, r)[rank * 16 + i] = m;
    }
    cluster.sync();  // the cluster's 128 SwiGLU values are in every member
    PHASE(PH_MOE_UP, 7);
    if (threadIdx.x < 32) build_xB_entry(midall, xBm, threadIdx.x);
    __syncthreads();

    // ---- down partial: rows n0 + [0, H/8) of w2 . the 128 values, one
    // 16-row tile per warp at a time; then the slot's fixed-point sums ----
    // (group grp of the K dimension: the B-fragment entries of group grp
    // start grp*32 entries into the array, so the pointer is offset back)
    const uint2* xg = reinterpret_cast<const uint2*>(xBm) - (size_t)grp * 32;
    for (int tt = warp; tt < rows / 16; tt += MOEF_THREADS / 32) {
        float y0 = 0.f, y1 = 0.f;
        int4_tile_dot<1>(w2p, w2s, H, I, n0 + tt * 16, grp, grp + 1, 1, xg, y0, y1);
        if ((lane & 3) == 0) {
            const int n = n0 + tt * 16 + (lane >> 2);
            red_add_u64(&P.acc[(size_t)t * H + n], (unsigned long long)llrint((double)y0 * 4294967296.0));
            red_add_u64(&P.acc[(size_t)t * H + n + 8], (unsigned long long)llrint((double)y1 * 4294967296.0));
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();  // the CTA's additions (ordered before it by the barrier) before the ticket
        s_last = atomicAdd(&P.tickets[rank], 1u) == gridDim.x / MOEF_CL - 1;
    }
    __syncthreads();
    PHASE(PH_MOE_UP, 8);
    if (!s_last) return;

    // ---- last cluster for this eighth: acc_scaled in rank order + residual
    // (engine.cu:900-904), then clear for the next layer ----
    __threadfence();
    for (int i = threadIdx.x; i < rows; i += blockDim.x) {
        const int n = n0 + i;
        long long q[8];  // topk <= 8; fully unrolled so the array stays in registers
#pragma unroll
        for (int k = 0; k < 8; k++) q[k] = k < P.topk ? (long long)ld_cg_u64(P.acc + (size_t)k * H + n) : 0ll;
        const float hn = __half2float(P.h[n]);
        __half acc = __float2half_rn(0.f);
#pragma unroll
        for (int k = 0; k < 8; k++) {
            if (k < P.topk) {
                const float o = (float)((double)q[k] * (1.0 / 4294967296.0));
                acc = __float2half_rn(__half2float(acc) + sw[k] * o);
                P.acc[(size_t)k * H + n] = 0ull;
            }
        }
        P.h_out[n] = __float2half_rn(hn + __half2float(acc));
    }
    if (threadIdx.x == 0) P.tickets[rank] = 0u;
    PHASE(PH_MOE_UP, 9);
}
