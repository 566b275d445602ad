// Fused MoE FFN decode layer, batch 1: router, selection, every selected
// expert's w1/w3 + SwiGLU and its w2 in ONE kernel (engine.cu:877-904:
// gemv_fp16 router, host top-k, per expert gemv w1/w3, swiglu, gemv w2,
// acc_scaled, add_inplace).
//
// Work split: CTA (t, c) owns intermediate rows [c, c+64) of the expert in
// rank slot t (grid topk * I/64, one CTA per SM, 16 warps).  It computes
// those 64 SwiGLU values and right away their share of the down projection:
// the w2 columns [c, c+64) of all H rows (32 bytes per row), so the down
// product is split over the intermediate dimension and no CTA waits for the
// whole SwiGLU vector.  The four CTAs of a cluster hold consecutive chunks of
// one expert; they reduce their partial down vectors over DSMEM (each rank
// owns H/4 outputs), then add them into per-slot accumulators in global
// memory as 64-bit fixed-point integers (2^-32 units), so the sum does not
// depend on the order the clusters arrive in: results are bit-identical from
// run to run.  The last cluster to finish a quarter of the outputs (atomic
// ticket) converts each slot's sum back to fp32 (o_t of the reference, up to
// fp32 summation order), applies acc = half(acc + w_t * o_t) in rank order
// and h = half(h + acc), and clears the accumulators and its ticket for the
// next layer.
#pragma once
#include "engine_kernels.cuh"

#define MOEF_THREADS 512
#define MOEF_CHUNK 64  // intermediate rows per CTA
#define MOEF_CL 4      // cluster: 4 consecutive chunks of one expert slot
#define MOEF_EMAX 64   // experts the fused kernel handles (router rows per CTA in smem)

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
    size_t up, dn, dsc, xs, part, misc, total;
};
// up: the 8 staged tiles (w1, w3 x 4 row tiles), which also hold this CTA's
// router rows before the selection; dn: the w2 column slice [H][32 B];
// dsc: its scales; xs: x and its B-fragment order; part: [4][H/4] partial
// down sums received over DSMEM; misc: reductions, logits, routes, tables.
__host__ __device__ inline MoefLayout moef_layout(int H, int E) {
    MoefLayout L;
    const size_t upb = 2 * (MOEF_CHUNK / 16) * (size_t)int4_tile_bytes(H);
    const size_t gate = (size_t)((E + MOEF_CL - 1) / MOEF_CL) * H * 2;
    L.up = 0;
    L.dn = (((upb > gate ? upb : gate) + 127) / 128) * 128;
    L.dsc = L.dn + (size_t)H * 32;
    L.xs = ((L.dsc + (size_t)H * 2 + 127) / 128) * 128;
    L.part = L.xs + (size_t)H * 4;
    L.misc = L.part + (size_t)H * 4;
    // red 256 f, nred 32 f, lgp 128 f, lg_all 64 f, sidx 8 i, sw 8 f, gu 128 f,
    // xB2 64 h, sbias 64 h, stab E*6 pointers
    L.total = L.misc + (256 + 32 + 128 + 64 + 8 + 8 + 128) * 4 + 64 * 2 * 2 + (size_t)MOEF_EMAX * 6 * 8 + 64;
    return L;
}

// Whether the fused kernel can run this MoE shape (else: k_moe_up + k_moe_down).
__host__ inline bool moef_supported(int H, int I, int E, int topk) {
    return E <= MOEF_EMAX && topk <= 8 && I % (MOEF_CHUNK * MOEF_CL) == 0 && H % (16 * MOEF_CL) == 0 &&
           H % 128 == 0 && H <= 16 * MOEF_THREADS && I % 128 == 0 && moef_layout(H, E).total <= 227 * 1024;
}

__device__ __forceinline__ void cp_async16_hint(void* smem_dst, const void* gsrc, uint64_t pol) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem_dst)),
                 "l"(gsrc), "l"(pol)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }
__device__ __forceinline__ unsigned long long ld_cg_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.global.cg.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __cluster_dims__(MOEF_CL, 1, 1) __launch_bounds__(MOEF_THREADS, 1) k_moe_fused(MoeFusedParams P) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t bar[1 + MOEF_CHUNK / 16];  // [0] router rows, [1 + j] w1/w3 tile pair j
    __shared__ int s_last;
    const MoefLayout Lo = moef_layout(P.H, P.E);
    const int H = P.H, I = P.I;
    const uint32_t TB = int4_tile_bytes(H);
    uint8_t* up = smem + Lo.up;
    __half* gs = reinterpret_cast<__half*>(smem + Lo.up);
    uint8_t* dn = smem + Lo.dn;
    __half* dsc = reinterpret_cast<__half*>(smem + Lo.dsc);
    __half* xs = reinterpret_cast<__half*>(smem + Lo.xs);
    __half* xB = xs + H;
    float* part = reinterpret_cast<float*>(smem + Lo.part);
    float* red = reinterpret_cast<float*>(smem + Lo.misc);  // [16][16]
    float* nred = red + 256;                                // [32]
    float* lgp = nred + 32;                                 // [128]
    float* lg_all = lgp + 128;                              // [64]
    int* sidx = reinterpret_cast<int*>(lg_all + 64);        // [8]
    float* sw = reinterpret_cast<float*>(sidx + 8);         // [8]
    float* gu = sw + 8;                                     // [2][64]
    __half* xB2 = reinterpret_cast<__half*>(gu + 128);      // [64]
    __half* sbias = xB2 + 64;                               // [64]
    const void** stab = reinterpret_cast<const void**>(sbias + 64);  // [E][6]
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int chunks = I / MOEF_CHUNK;
    const int t = blockIdx.x / chunks, c0 = (blockIdx.x % chunks) * MOEF_CHUNK;
    const int rpc = (P.E + MOEF_CL - 1) / MOEF_CL, e0 = rank * rpc, ne = max(0, min(P.E - e0, rpc));
    const int seg = H / MOEF_CL;
    cluster_arrive_started();

    // ---- before the dependency wait: static data only ----
    if (threadIdx.x == 0) {
        for (int i = 0; i < 1 + MOEF_CHUNK / 16; i++) mbar_init(&bar[i], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&bar[0], (uint32_t)ne * H * 2);
        if (ne > 0) tma_load_1d(gs, P.gate + (size_t)e0 * H, (uint32_t)ne * H * 2, &bar[0]);
        l2_prefetch_share(P.next, blockIdx.x, gridDim.x);
    }
    NormW nw;
    if (!P.xn) norm_w_load(nw, P.norm_w, H);
    for (int i = threadIdx.x; i < P.E; i += blockDim.x) sbias[i] = P.bias[i];
    for (int i = threadIdx.x; i < P.E * 6; i += blockDim.x) stab[i] = P.experts[i];
    pdl_trigger();
    pdl_wait();

    // ---- RMSNorm of the residual (rmsnorm, engine.cu:131-144) ----
    if (P.xn) {
        for (int i = threadIdx.x; i < H; i += blockDim.x) xs[i] = P.xn[i];
        __syncthreads();
        for (int e = threadIdx.x; e < H / 4; e += blockDim.x) build_xB_entry(xs, xB, e);
        __syncthreads();
    } else {
        norm_prologue_fast(nw, P.h, nullptr, nullptr, nullptr, H, P.eps, xs, xB, nred);
    }

    // ---- router logits (gemv_fp16, engine.cu:879): this member's rows ----
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
    cluster.sync();

    // ---- selection (engine.cu:883-892) ----
    route_select_block(lg_all, sbias, P.E, P.topk, sidx, sw, lgp);
    if (blockIdx.x == 0 && threadIdx.x < P.topk) {
        P.route_idx[threadIdx.x] = sidx[threadIdx.x];
        P.route_w[threadIdx.x] = sw[threadIdx.x];
    }

    // ---- this CTA's expert weights: w1/w3 rows [c0, c0+64) by TMA, the w2
    // column slice [H][c0/2 .. c0/2+32) bytes by 16-byte async copies ----
    const void* const* ex = stab + (size_t)sidx[t] * 6;
    if (threadIdx.x == 0) {
        for (int j = 0; j < MOEF_CHUNK / 16; j++) {
            mbar_arrive_expect_tx(&bar[1 + j], 2 * TB);
            tma_tile_int4((const uint8_t*)ex[0], (const __half*)ex[1], H, c0 + 16 * j, up + (2 * j) * TB, &bar[1 + j]);
            tma_tile_int4((const uint8_t*)ex[2], (const __half*)ex[3], H, c0 + 16 * j, up + (2 * j + 1) * TB,
                          &bar[1 + j]);
        }
    }
    {
        const uint8_t* w2p = (const uint8_t*)ex[4] + c0 / 2;
        const uint64_t pol = l2_policy_evict_first();
        for (int i = threadIdx.x; i < 2 * H; i += blockDim.x)
            cp_async16_hint(dn + (size_t)i * 16, w2p + (size_t)(i >> 1) * (I >> 1) + (i & 1) * 16, pol);
        cp_async_commit();
        const __half* w2s = (const __half*)ex[5] + c0 / 128;
        for (int n = threadIdx.x; n < H; n += blockDim.x) dsc[n] = w2s[(size_t)n * (I >> 7)];
    }

    // ---- w1/w3 dot + SwiGLU (swiglu, engine.cu:542-547): warp = 4 * pair
    // + 2 * matrix + half of the K groups ----
    {
        const int pair = warp >> 2, mat = (warp >> 1) & 1, hk = warp & 1;
        float y0 = 0.f, y1 = 0.f;
        if (stage_wait(&bar[1 + pair]))
            int4_tile_dot_smem<2>(up + (2 * pair + mat) * TB, H, hk, H >> 7, 2, reinterpret_cast<const uint2*>(xB),
                                  y0, y1);
        warp_partials(red, warp, y0, y1);
    }
    __syncthreads();
    if (threadIdx.x < MOEF_CHUNK) {
        const int r = threadIdx.x, wg = (r >> 4) * 4, i = r & 15;
        const float g = red[(wg + 0) * 16 + i] + red[(wg + 1) * 16 + i];
        const float u = red[(wg + 2) * 16 + i] + red[(wg + 3) * 16 + i];
        const __half m = __float2half_rn(silu_fast(g) * u);
        // B-fragment order of a 64-wide K chunk: lane quad c covers k in
        // [16c, 16c+16), word w = k/8 of it; entry (mma m, quad c) holds
        // x[k], x[k+4], x[k+1], x[k+5] for k = 16c + 8(m/2) + 2(m%2)
        const int c = r >> 4, q = r & 7, w = (r >> 3) & 1;
        const int mm = 2 * w + ((q >> 1) & 1), pos = ((q & 1) << 1) | (q >> 2);
        xB2[(mm * 4 + c) * 4 + pos] = m;
    }
    cp_async_wait_all();
    __syncthreads();

    // ---- down partial: rows n of w2 . mid[c0 .. c0+64), each sent to the
    // cluster member that owns output quarter n / (H/4) ----
    {
        const int g = lane >> 2, c = lane & 3;
        const uint2* xb2 = reinterpret_cast<const uint2*>(xB2);
        const uint2 b0 = xb2[0 * 4 + c], b1 = xb2[1 * 4 + c], b2 = xb2[2 * 4 + c], b3 = xb2[3 * 4 + c];
        for (int blk = warp; blk < H / 16; blk += MOEF_THREADS / 32) {
            const int r0 = blk * 16;
            const uint2 wa = *reinterpret_cast<const uint2*>(dn + (size_t)(r0 + g) * 32 + c * 8);
            const uint2 wb = *reinterpret_cast<const uint2*>(dn + (size_t)(r0 + g + 8) * 32 + c * 8);
            float d[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t ha[4], hb[4];
            dequant8(wa.x, ha);
            dequant8(wb.x, hb);
            mma_16816(d, ha[0], hb[0], ha[1], hb[1], b0.x, b0.y);
            mma_16816(d, ha[2], hb[2], ha[3], hb[3], b1.x, b1.y);
            dequant8(wa.y, ha);
            dequant8(wb.y, hb);
            mma_16816(d, ha[0], hb[0], ha[1], hb[1], b2.x, b2.y);
            mma_16816(d, ha[2], hb[2], ha[3], hb[3], b3.x, b3.y);
            if (c == 0) {
                const int n0 = r0 + g, n1 = r0 + g + 8;
                const float v0 = __half2float(dsc[n0]) * d[0], v1 = __half2float(dsc[n1]) * d[2];
                cluster.map_shared_rank(part, n0 / seg)[rank * seg + n0 % seg] = v0;
                cluster.map_shared_rank(part, n1 / seg)[rank * seg + n1 % seg] = v1;
            }
        }
    }
    cluster.sync();

    // ---- this member's output quarter: cluster sum (rank order), then the
    // slot's fixed-point accumulator ----
    for (int i = threadIdx.x; i < seg; i += blockDim.x) {
        float v = part[i];
        for (int r = 1; r < MOEF_CL; r++) v += part[r * seg + i];
        const long long q = llrint((double)v * 4294967296.0);
        atomicAdd(&P.acc[(size_t)t * H + rank * seg + i], (unsigned long long)q);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&P.tickets[rank], 1u) == gridDim.x / MOEF_CL - 1;
    __syncthreads();
    if (!s_last) return;

    // ---- last cluster for this quarter: acc_scaled in rank order + residual
    // (engine.cu:900-904), then clear for the next layer ----
    __threadfence();
    for (int i = threadIdx.x; i < seg; i += blockDim.x) {
        const int n = rank * seg + i;
        __half acc = __float2half_rn(0.f);
        for (int k = 0; k < P.topk; k++) {
            unsigned long long* a = P.acc + (size_t)k * H + n;
            const long long q = (long long)ld_cg_u64(a);
            const float o = (float)((double)q * (1.0 / 4294967296.0));
            acc = __float2half_rn(__half2float(acc) + sw[k] * o);
            *a = 0ull;
        }
        P.h_out[n] = __float2half_rn(__half2float(P.h[n]) + __half2float(acc));
    }
    if (threadIdx.x == 0) P.tickets[rank] = 0u;
}
