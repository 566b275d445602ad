// Single-token flash-decoding attention over the FP8 E4M3 group-64 KV cache and
// its fp16 tail (attn_decode_split + attn_decode_combine, src/engine.cu:396-480).
//
// Layout (the reference's, engine.cu:185-187, 599-603):
//   kc8/vc8  u8   [T, nkv, 64]    committed tokens [0, committed)
//   ksc/vsc  fp16 [T/64, nkv]     one scale per (64-token group, kv head)
//   ktail/vtail fp16 [64, nkv, 64] tokens [committed, qpos] at t - committed
//
// Work decomposition: grid (nkv, nsplit), 4 warps.  A "unit" is one 64-token
// group (the tail is the last unit).  CTA (h, sp) takes a contiguous run of
// units of kv head h; its warps take units round-robin.  Each warp handles
// all GQA query heads of h at once, so every K/V byte is read once.
//   S = Q K^T : mma m16n8k16, rows = query heads (<= 16), cols = 8 keys,
//               k = 64 dims; K converted FP8->f16 in registers (exact).
//   O += P V  : rows = query heads, k = 16 keys, cols = 8 dims; P in f16.
// Online softmax in base 2 with finite sentinels; per-unit V scale applied
// to a fresh accumulator.  Partials (m, l, O) per (h, sp, query head) go to
// the workspace; the last CTA of each kv head (atomic ticket) merges them.
// Cluster form (P.cluster = nsplit, launched with clusters of (1, nsplit)):
// the partials stay in each CTA's shared memory and the cluster's CTAs merge
// them over DSMEM, each a slice of the outputs, in the same split order and
// arithmetic (no workspace, no ticket).
#pragma once
#include <cooperative_groups.h>
#include "common.cuh"

struct AttnParams {
    const __half* q;
    const uint8_t* kc8;
    const uint8_t* vc8;
    const __half* ksc;
    const __half* vsc;
    const __half* ktail;
    const __half* vtail;
    const int* pos_dev;  // when set: qpos = *pos_dev, committed = 64*((qpos+1)/64)
    int committed, qpos;
    float scale;
    __half* out;
    float* part;          // [nkv][nsplit][gqa][68]
    unsigned* counters;   // [nkv], zero before the first launch; left zero
    int nh, nkv, nsplit;  // nsplit * (nh/nkv) <= ATTN_MAX_PARTS
    L2Ranges next;        // weights of the following kernels, prefetched to L2
    int cluster = 0;      // > 0: the nsplit (= cluster) CTAs of a kv head merge over DSMEM
    // batched decode: sequence blockIdx.z reads its q, cache, position and
    // writes its output at these element strides (counters at b * nkv)
    size_t bq = 0, bkv8 = 0, bsc = 0, btail = 0, bout = 0, bpart = 0;
};

#define ATTN_PART_STRIDE 68
#define ATTN_THREADS 256  // 8 warps
#define ATTN_PARTS 2      // each warp takes half a 64-token unit
#define ATTN_NEG (-1.0e30f)
#define ATTN_MAX_PARTS 1024

__device__ __forceinline__ uint32_t fp8x2_to_h2(uint32_t two_bytes) {
    __half2_raw r = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(two_bytes & 0xFFFFu), __NV_E4M3);
    return (uint32_t)r.x | ((uint32_t)r.y << 16);
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// One warp: online-softmax attention of its query heads (A-fragment rows,
// aq) over unit parts pi = p_begin, p_begin+p_step, ... < p_end of kv head h,
// where part pi is keys [64/PARTS * (pi % PARTS), +64/PARTS) of the 64-token
// unit pi / PARTS.  Keeps the running max m_run (base 2, per row), the
// per-lane partial sum l_run and the output accumulators O (n-tile j holds
// dims 16c+j and 16c+8+j of row g).  An FP8 part's K and V are all requested
// before any math, so a part costs one memory round trip.
// CG: read the cache with ld.global.cg (coherent at L2) because the caller's
// own launch may have written it (the persistent kernel); otherwise the
// cache is read through the non-coherent streaming path.
template <bool CG, int PARTS>
__device__ __forceinline__ void attn_warp_units(const uint8_t* __restrict__ kc8,
                                                const uint8_t* __restrict__ vc8,
                                                const __half* __restrict__ ksc,
                                                const __half* __restrict__ vsc,
                                                const __half* __restrict__ ktail,
                                                const __half* __restrict__ vtail, int nkv, int h,
                                                int n_fp8, int tail_len, float kfac,
                                                const uint32_t (&aq)[4][2], int p_begin, int p_end,
                                                int p_step, float& m_run, float& l_run,
                                                float (&O)[8][4]) {
    constexpr int NJ = 8 / PARTS;  // 8-key n-tiles per part (QK)
    constexpr int NS = 4 / PARTS;  // 16-key k-steps per part (PV)
    const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const size_t kstride = (size_t)nkv * CUINF_HD;
    for (int pi = p_begin; pi < p_end; pi += p_step) {
        const int u = pi / PARTS, k0 = (pi % PARTS) * (64 / PARTS);
        const bool tail = u >= n_fp8;
        const int valid = tail ? tail_len : CUINF_KVGROUP;
        const int kbase = u * CUINF_KVGROUP;
        uint4 kraw[NJ];
        uint2 vraw[NS][4];
        const int off[4] = {0, 1, 8, 9};
        if (!tail) {
#pragma unroll
            for (int jn = 0; jn < NJ; jn++) {
                const uint8_t* kp8 = kc8 + ((size_t)(kbase + k0 + 8 * jn + g) * nkv + h) * CUINF_HD + 16 * c;
                kraw[jn] = CG ? __ldcg(reinterpret_cast<const uint4*>(kp8)) : ldg_stream(kp8);
            }
#pragma unroll
            for (int s2 = 0; s2 < NS; s2++) {
                const uint8_t* vp = vc8 + ((size_t)(kbase + k0 + 16 * s2 + 2 * c) * nkv + h) * CUINF_HD + 8 * g;
#pragma unroll
                for (int i = 0; i < 4; i++)
                    vraw[s2][i] = CG ? __ldcg(reinterpret_cast<const uint2*>(vp + off[i] * kstride))
                                     : ldg_stream8(vp + off[i] * kstride);
            }
        }
        // ---- S = Q K^T for the part's keys (NJ n-tiles of 8 keys) ----
        float S[NJ][4];
#pragma unroll
        for (int jn = 0; jn < NJ; jn++) {
            S[jn][0] = S[jn][1] = S[jn][2] = S[jn][3] = 0.f;
            const int kk = k0 + 8 * jn + g;  // key within the unit
            uint32_t kb[8];
            if (!tail) {
                const uint4 raw = kraw[jn];
                const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    kb[2 * i] = fp8x2_to_h2(w4[i]);
                    kb[2 * i + 1] = fp8x2_to_h2(w4[i] >> 16);
                }
            } else {
                const __half* kp = ktail + ((size_t)kk * nkv + h) * CUINF_HD + 16 * c;
                uint4 r0 = CG ? __ldcg(reinterpret_cast<const uint4*>(kp)) : *reinterpret_cast<const uint4*>(kp);
                uint4 r1 = CG ? __ldcg(reinterpret_cast<const uint4*>(kp + 8)) : *reinterpret_cast<const uint4*>(kp + 8);
                kb[0] = r0.x; kb[1] = r0.y; kb[2] = r0.z; kb[3] = r0.w;
                kb[4] = r1.x; kb[5] = r1.y; kb[6] = r1.z; kb[7] = r1.w;
            }
#pragma unroll
            for (int s = 0; s < 4; s++)
                mma_16816(S[jn], aq[s][0], 0u, aq[s][1], 0u, kb[2 * s], kb[2 * s + 1]);
        }
        const float kscale = tail ? 1.0f : __half2float(CG ? __ldcg(ksc + (size_t)u * nkv + h) : ksc[(size_t)u * nkv + h]);
        const float f = kscale * kfac;
        float mx = ATTN_NEG;
#pragma unroll
        for (int jn = 0; jn < NJ; jn++) {
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const int key = k0 + 8 * jn + 2 * c + i;
                float sv = S[jn][i] * f;
                sv = key < valid ? sv : ATTN_NEG;
                S[jn][i] = sv;
                mx = fmaxf(mx, sv);
            }
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run, mx);
        const float alpha = exp2f(m_run - m_new);
        float lsum = 0.f;
#pragma unroll
        for (int jn = 0; jn < NJ; jn++) {
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const int key = k0 + 8 * jn + 2 * c + i;
                float pv = key < valid ? exp2f(S[jn][i] - m_new) : 0.f;
                S[jn][i] = pv;
                lsum += pv;
            }
        }
        l_run = l_run * alpha + lsum;
        m_run = m_new;
        // ---- tmp = P V (NS k-steps of 16 keys, 8 n-tiles of 8 dims) ----
        float T[8][4];
#pragma unroll
        for (int j = 0; j < 8; j++) T[j][0] = T[j][1] = T[j][2] = T[j][3] = 0.f;
#pragma unroll
        for (int s2 = 0; s2 < NS; s2++) {
            const uint32_t pa0 = pack_h2(S[2 * s2][0], S[2 * s2][1]);
            const uint32_t pa2 = pack_h2(S[2 * s2 + 1][0], S[2 * s2 + 1][1]);
            const int ka = k0 + 16 * s2 + 2 * c;  // keys ka, ka+1, ka+8, ka+9
            uint32_t b0[8], b1[8];
            if (!tail) {
                const uint2 va = vraw[s2][0], vb = vraw[s2][1], vc = vraw[s2][2], vd = vraw[s2][3];
                uint32_t r;
                r = prmt(va.x, vb.x, 0x5140u); b0[0] = fp8x2_to_h2(r); b0[1] = fp8x2_to_h2(r >> 16);
                r = prmt(va.x, vb.x, 0x7362u); b0[2] = fp8x2_to_h2(r); b0[3] = fp8x2_to_h2(r >> 16);
                r = prmt(va.y, vb.y, 0x5140u); b0[4] = fp8x2_to_h2(r); b0[5] = fp8x2_to_h2(r >> 16);
                r = prmt(va.y, vb.y, 0x7362u); b0[6] = fp8x2_to_h2(r); b0[7] = fp8x2_to_h2(r >> 16);
                r = prmt(vc.x, vd.x, 0x5140u); b1[0] = fp8x2_to_h2(r); b1[1] = fp8x2_to_h2(r >> 16);
                r = prmt(vc.x, vd.x, 0x7362u); b1[2] = fp8x2_to_h2(r); b1[3] = fp8x2_to_h2(r >> 16);
                r = prmt(vc.y, vd.y, 0x5140u); b1[4] = fp8x2_to_h2(r); b1[5] = fp8x2_to_h2(r >> 16);
                r = prmt(vc.y, vd.y, 0x7362u); b1[6] = fp8x2_to_h2(r); b1[7] = fp8x2_to_h2(r >> 16);
            } else {
                const __half* vp = vtail + ((size_t)ka * nkv + h) * CUINF_HD + 8 * g;
                const uint4 z = make_uint4(0u, 0u, 0u, 0u);
                // keys beyond the tail hold stale data: zero them
                auto ld16 = [](const __half* q) {
                    return CG ? __ldcg(reinterpret_cast<const uint4*>(q)) : *reinterpret_cast<const uint4*>(q);
                };
                uint4 va = ka < valid ? ld16(vp) : z;
                uint4 vb = ka + 1 < valid ? ld16(vp + kstride) : z;
                uint4 vc = ka + 8 < valid ? ld16(vp + 8 * kstride) : z;
                uint4 vd = ka + 9 < valid ? ld16(vp + 9 * kstride) : z;
                const uint32_t A4[4] = {va.x, va.y, va.z, va.w}, B4[4] = {vb.x, vb.y, vb.z, vb.w};
                const uint32_t C4[4] = {vc.x, vc.y, vc.z, vc.w}, D4[4] = {vd.x, vd.y, vd.z, vd.w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    b0[2 * i] = prmt(A4[i], B4[i], 0x5410u);
                    b0[2 * i + 1] = prmt(A4[i], B4[i], 0x7632u);
                    b1[2 * i] = prmt(C4[i], D4[i], 0x5410u);
                    b1[2 * i + 1] = prmt(C4[i], D4[i], 0x7632u);
                }
            }
#pragma unroll
            for (int j = 0; j < 8; j++) mma_16816(T[j], pa0, 0u, pa2, 0u, b0[j], b1[j]);
        }
        const float vscale = tail ? 1.0f : __half2float(CG ? __ldcg(vsc + (size_t)u * nkv + h) : vsc[(size_t)u * nkv + h]);
#pragma unroll
        for (int j = 0; j < 8; j++) {
            O[j][0] = O[j][0] * alpha + vscale * T[j][0];
            O[j][1] = O[j][1] * alpha + vscale * T[j][1];
        }
    }
}

// MINB: CTAs per SM the register budget is cut for (1: no spills, the
// batch-1 engine; 2: the standalone operator, whose default split count
// assumes two CTAs per SM, and the batched engine's many CTAs).
template <int MINB>
__global__ void __launch_bounds__(ATTN_THREADS, MINB) k_attn_decode(AttnParams P) {
    __shared__ __align__(16) float sm[ATTN_THREADS / 32][16][ATTN_PART_STRIDE];
    __shared__ int s_last;
    const int h = blockIdx.x, sp = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int nkv = P.nkv, gqa = P.nh / P.nkv;
    const size_t b = blockIdx.z;
    const uint8_t* kc8 = P.kc8 + b * P.bkv8;
    const uint8_t* vc8 = P.vc8 + b * P.bkv8;
    const __half* ksc = P.ksc + b * P.bsc;
    const __half* vsc = P.vsc + b * P.bsc;
    const __half* ktail = P.ktail + b * P.btail;
    const __half* vtail = P.vtail + b * P.btail;
    float* const part_b = P.part + b * P.bpart;
    unsigned* const cnt_b = P.counters + b * nkv;
    PHASE(PH_ATTN, 0);
    if (threadIdx.x == 0 && P.next.count)
        l2_prefetch_share(P.next, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);
    pdl_trigger();
    pdl_wait();  // q and the cache come from the previous kernel
    PHASE(PH_ATTN, 1);
    int qpos = P.qpos, committed = P.committed;
    if (P.pos_dev) {
        qpos = P.pos_dev[b];
        committed = ((qpos + 1) / CUINF_KVGROUP) * CUINF_KVGROUP;
    }
    const int total = qpos + 1;
    const int tail_len = total - committed;
    const int n_fp8 = committed / CUINF_KVGROUP;
    const int nunits = n_fp8 + (tail_len > 0 ? 1 : 0);
    const int ups = (nunits + P.nsplit - 1) / P.nsplit;
    const int u0 = sp * ups, u1 = min(u0 + ups, nunits);
    const float kfac = P.scale * 1.4426950408889634f;  // scores in base 2

    // Q as the A operand: row g = query head h*gqa+g (rows >= gqa are zero).
    uint32_t aq[4][2];
    {
        const bool real = g < gqa;
        const __half* qh = P.q + b * P.bq + (size_t)(h * gqa + (real ? g : 0)) * CUINF_HD + 16 * c;
#pragma unroll
        for (int s = 0; s < 4; s++) {
            uint32_t lo = *reinterpret_cast<const uint32_t*>(qh + 4 * s);
            uint32_t hi = *reinterpret_cast<const uint32_t*>(qh + 4 * s + 2);
            aq[s][0] = real ? lo : 0u;
            aq[s][1] = real ? hi : 0u;
        }
    }

    float m_run = ATTN_NEG, l_run = 0.f;
    float O[8][4];
#pragma unroll
    for (int j = 0; j < 8; j++) O[j][0] = O[j][1] = O[j][2] = O[j][3] = 0.f;

    attn_warp_units<false, ATTN_PARTS>(kc8, vc8, ksc, vsc, ktail, vtail, nkv, h, n_fp8, tail_len,
                                       kfac, aq, u0 * ATTN_PARTS + warp, u1 * ATTN_PARTS, ATTN_THREADS / 32,
                                       m_run, l_run, O);
    PHASE(PH_ATTN, 2);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);

    // ---- merge the 4 warps (rows g < gqa are real) ----
    if (g < gqa) {
        float* row = sm[warp][g];
        if (c == 0) { row[0] = m_run; row[1] = l_run; }
#pragma unroll
        for (int j = 0; j < 8; j++) {
            row[4 + 16 * c + j] = O[j][0];
            row[4 + 16 * c + 8 + j] = O[j][1];
        }
    }
    __syncthreads();
    if (P.cluster) {
        // ---- cluster form: this CTA's partial in shared memory, merged over DSMEM ----
        __shared__ __align__(16) float cpart[8][ATTN_PART_STRIDE];
        for (int it = threadIdx.x; it < gqa * 64; it += blockDim.x) {
            const int r = it >> 6, d = it & 63;
            float mm = ATTN_NEG;
#pragma unroll
            for (int w = 0; w < ATTN_THREADS / 32; w++) mm = fmaxf(mm, sm[w][r][0]);
            float l = 0.f, o = 0.f;
#pragma unroll
            for (int w = 0; w < ATTN_THREADS / 32; w++) {
                const float e = exp2f(sm[w][r][0] - mm);
                l += sm[w][r][1] * e;
                o += sm[w][r][4 + d] * e;
            }
            cpart[r][4 + d] = o;
            if (d == 0) { cpart[r][0] = mm; cpart[r][1] = l; }
        }
        cooperative_groups::cluster_group cl = cooperative_groups::this_cluster();
        cl.sync();  // every split's partial is in its CTA
        const int ncl = (int)cl.num_blocks(), rank = (int)cl.block_rank();
        const int per = (gqa * 64 + ncl - 1) / ncl, end = min(gqa * 64, (rank + 1) * per);
        for (int it = rank * per + (int)threadIdx.x; it < end; it += blockDim.x) {
            const int r = it >> 6, d = it & 63;
            float gm = ATTN_NEG, L = 0.f, o = 0.f;
            for (int s2 = 0; s2 < ncl; s2++) {
                const float* pr = cl.map_shared_rank(&cpart[r][0], s2);
                if (pr[1] > 0.f) gm = fmaxf(gm, pr[0]);
            }
            for (int s2 = 0; s2 < ncl; s2++) {
                const float* pr = cl.map_shared_rank(&cpart[r][0], s2);
                const float vl = pr[1];
                const float e = vl > 0.f ? exp2f(pr[0] - gm) : 0.f;
                L += vl * e;
                o += e * pr[4 + d];
            }
            P.out[b * P.bout + (size_t)(h * gqa + r) * CUINF_HD + d] = __float2half_rn(o / L);
        }
        PHASE(PH_ATTN, 3);
        cl.sync();  // no CTA leaves while another reads its partial
        PHASE(PH_ATTN, 4);
        return;
    }
    float* part = part_b + ((size_t)(h * P.nsplit + sp) * gqa) * ATTN_PART_STRIDE;
    for (int it = threadIdx.x; it < gqa * 64; it += blockDim.x) {
        const int r = it >> 6, d = it & 63;
        float mm = ATTN_NEG;
#pragma unroll
        for (int w = 0; w < ATTN_THREADS / 32; w++) mm = fmaxf(mm, sm[w][r][0]);
        float l = 0.f, o = 0.f;
#pragma unroll
        for (int w = 0; w < ATTN_THREADS / 32; w++) {
            const float e = exp2f(sm[w][r][0] - mm);
            l += sm[w][r][1] * e;
            o += sm[w][r][4 + d] * e;
        }
        float* pr = part + (size_t)r * ATTN_PART_STRIDE;
        pr[4 + d] = o;
        if (d == 0) { pr[0] = mm; pr[1] = l; }
    }
    // ---- last CTA of kv head h merges the splits ----
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned prev = atomicAdd(&cnt_b[h], 1u);
        s_last = prev == (unsigned)(P.nsplit - 1);
    }
    __syncthreads();
    if (!s_last) return;
    PHASE(PH_ATTN, 3);
    __threadfence();
    // Thread (r, d) merges output d of query row r over the splits, 32 splits
    // per round with all their (m, l, o) requested at once (one L2 round trip
    // per round), rescaled online; with nsplit <= 32 this is exactly
    // gm = max m, L = sum l*2^(m-gm), o = sum o*2^(m-gm) in split order.
    const float* hp = part_b + (size_t)h * P.nsplit * gqa * ATTN_PART_STRIDE;
    for (int it = threadIdx.x; it < gqa * 64; it += blockDim.x) {
        const int r = it >> 6, d = it & 63;
        float gm = ATTN_NEG, L = 0.f, o = 0.f;
        for (int sp0 = 0; sp0 < P.nsplit; sp0 += 32) {
            float vm[32], vl[32], vo[32];
#pragma unroll
            for (int k = 0; k < 32; k++) {
                vm[k] = ATTN_NEG;
                vl[k] = 0.f;
                vo[k] = 0.f;
                if (sp0 + k < P.nsplit) {
                    const float* pr = hp + (size_t)((sp0 + k) * gqa + r) * ATTN_PART_STRIDE;
                    vm[k] = __ldcg(pr);
                    vl[k] = __ldcg(pr + 1);
                    vo[k] = __ldcg(pr + 4 + d);
                }
            }
            float cm = gm;
#pragma unroll
            for (int k = 0; k < 32; k++)
                if (vl[k] > 0.f) cm = fmaxf(cm, vm[k]);
            if (cm > gm) {
                const float sc = exp2f(gm - cm);
                L *= sc;
                o *= sc;
                gm = cm;
            }
#pragma unroll
            for (int k = 0; k < 32; k++) {
                const float e = vl[k] > 0.f ? exp2f(vm[k] - gm) : 0.f;
                L += vl[k] * e;
                o += e * vo[k];
            }
        }
        P.out[b * P.bout + (size_t)(h * gqa + r) * CUINF_HD + d] = __float2half_rn(o / L);
    }
    if (threadIdx.x == 0) cnt_b[h] = 0u;
    PHASE(PH_ATTN, 4);
}

// Prefill attention (attention_fused, engine.cu:236-308): query token i of
// S (position past + i) attends to keys [0, past + i]; keys below
// `committed` (the count after all S tokens were placed) come from the FP8
// cache with their group scale, the rest from the fp16 tail at index
// t - committed.  One warp per (token, query head); lane d holds dims 2d and
// 2d+1; online softmax in fp32.  q/out fp16 [S][nh][64].
__global__ void __launch_bounds__(32) k_attn_prefill(const __half* __restrict__ q, const uint8_t* __restrict__ kc8,
                                                     const uint8_t* __restrict__ vc8,
                                                     const __half* __restrict__ ksc,
                                                     const __half* __restrict__ vsc,
                                                     const __half* __restrict__ ktail,
                                                     const __half* __restrict__ vtail, int committed,
                                                     int past, float scale, __half* __restrict__ out, int nh,
                                                     int nkv) {
    const int i = blockIdx.x, hq = blockIdx.y, d = threadIdx.x;
    const int kvh = hq / (nh / nkv), qpos = past + i;
    const __half2 qv = reinterpret_cast<const __half2*>(q + ((size_t)i * nh + hq) * CUINF_HD)[d];
    const float q0 = __low2float(qv), q1 = __high2float(qv);
    const int cend = committed < qpos + 1 ? committed : qpos + 1;
    float m = -1e30f, l = 0.f, o0 = 0.f, o1 = 0.f;
    for (int t = 0; t <= qpos; t++) {
        float k0, k1, v0, v1;
        if (t < cend) {
            const float ks = __half2float(ksc[(t / CUINF_KVGROUP) * nkv + kvh]);
            const float vs = __half2float(vsc[(t / CUINF_KVGROUP) * nkv + kvh]);
            const uint32_t kb = fp8x2_to_h2(reinterpret_cast<const uint16_t*>(kc8 + ((size_t)t * nkv + kvh) * CUINF_HD)[d]);
            const uint32_t vb = fp8x2_to_h2(reinterpret_cast<const uint16_t*>(vc8 + ((size_t)t * nkv + kvh) * CUINF_HD)[d]);
            const __half2 kh = *reinterpret_cast<const __half2*>(&kb), vh = *reinterpret_cast<const __half2*>(&vb);
            k0 = __low2float(kh) * ks; k1 = __high2float(kh) * ks;
            v0 = __low2float(vh) * vs; v1 = __high2float(vh) * vs;
        } else {
            const size_t row = ((size_t)(t - committed) * nkv + kvh) * CUINF_HD;
            const __half2 kh = reinterpret_cast<const __half2*>(ktail + row)[d];
            const __half2 vh = reinterpret_cast<const __half2*>(vtail + row)[d];
            k0 = __low2float(kh); k1 = __high2float(kh);
            v0 = __low2float(vh); v1 = __high2float(vh);
        }
        const float sc = warp_sum(q0 * k0 + q1 * k1) * scale;
        const float mn = fmaxf(m, sc), cf = __expf(m - mn), p = __expf(sc - mn);
        l = l * cf + p;
        o0 = o0 * cf + p * v0;
        o1 = o1 * cf + p * v1;
        m = mn;
    }
    reinterpret_cast<__half2*>(out + ((size_t)i * nh + hq) * CUINF_HD)[d] = __floats2half2_rn(o0 / l, o1 / l);
}

// Splits for the decode engine: one unit part per warp at the session's
// longest context (ATTN_THREADS/32/ATTN_PARTS units per CTA), so every warp of
// every CTA has work and the combine merges as few partials as that allows;
// at most ATTN_MAX_PARTS (split, query head) partials per kv head.
static inline int attn_engine_nsplit(int gqa, int max_units) {
    const int upc = ATTN_THREADS / 32 / ATTN_PARTS;
    int ns = (max_units + upc - 1) / upc;
    if (ns * gqa > ATTN_MAX_PARTS) ns = ATTN_MAX_PARTS / gqa;
    return ns < 1 ? 1 : ns;
}

// Splits that fill the GPU: about two CTAs per SM over all kv heads, at most
// ATTN_MAX_PARTS (split, query head) partials per kv head.
static inline int attn_default_nsplit(int nkv, int gqa, int max_units, int num_sms) {
    int ns = (2 * num_sms + nkv - 1) / nkv;
    if (ns > max_units) ns = max_units;
    if (ns * gqa > ATTN_MAX_PARTS) ns = ATTN_MAX_PARTS / gqa;
    if (ns < 1) ns = 1;
    return ns;
}

// ---------------------------------------------------------------------------
// H2O eviction mode (engine.cu:310-384, 803-828): a circular buffer of C
// per-token FP8 slots per attention layer, each with its own per-head fp16
// scale, its logical position and its cumulative attention mass.
// ---------------------------------------------------------------------------
#define H2O_MAX_SLOTS 8192
struct H2oParams {
    const __half *k_new, *v_new;  // [S][nkv][64] the fresh tokens' K/V
    const __half* q;              // [S][nh][64]
    __half* out;                  // [S][nh][64]
    const int* pos_dev;           // decode: the token's position (S = 1); null: past
    int past, S, C, W, nh, nkv;
    float scale;
    uint8_t *hk8, *hv8;  // [C][nkv][64]
    __half *hks, *hvs;   // [C][nkv]
    int* slot_pos;       // [C]
    float* attn_sum;     // [C]
    int* n_live;         // [1]
    int* dst;            // [S] slot of each fresh token
};

// Slot choice for the S fresh tokens in order (the reference's host loop,
// engine.cu:808-823): append while there is room; else the least cumulative
// attention among slots outside the local window (pos <= p - W), first such
// minimum; else the least overall; slots picked earlier in the same batch are
// excluded.  A reused slot's mass restarts at 0.  Then kv_quant_write
// (317-333): per token and head, scale = absmax/448 + 1e-12, codes
// e4m3(x / scale).  One CTA of 256 threads.
__global__ void __launch_bounds__(256) k_h2o_place(H2oParams P) {
    __shared__ unsigned char banned[H2O_MAX_SLOTS];
    __shared__ float rv[8];
    __shared__ int ri[8];
    __shared__ int s_live, s_slot;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int t = tid; t < P.C; t += blockDim.x) banned[t] = 0;
    pdl_wait();
    if (tid == 0) s_live = *P.n_live;
    __syncthreads();
    const int base = P.pos_dev ? *P.pos_dev : P.past;
    for (int j = 0; j < P.S; j++) {
        const int pos = base + j;
        if (s_live < P.C) {
            if (tid == 0) s_slot = s_live;
        } else {
            for (int pass = 0; pass < 2; pass++) {
                float v = 1e30f;
                int idx = 0x7fffffff;
                for (int t = tid; t < P.C; t += blockDim.x) {
                    const float a = banned[t] ? 1e30f : P.attn_sum[t];
                    if ((pass == 1 || P.slot_pos[t] <= pos - P.W) && a < v) {
                        v = a;
                        idx = t;
                    }
                }
#pragma unroll
                for (int o = 16; o; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
                    if (ov < v || (ov == v && oi < idx)) {
                        v = ov;
                        idx = oi;
                    }
                }
                if (lane == 0) {
                    rv[warp] = v;
                    ri[warp] = idx;
                }
                __syncthreads();
                if (tid == 0) {
                    float bv = rv[0];
                    int bi = ri[0];
                    for (int w = 1; w < 8; w++)
                        if (rv[w] < bv || (rv[w] == bv && ri[w] < bi)) {
                            bv = rv[w];
                            bi = ri[w];
                        }
                    s_slot = bi;
                }
                __syncthreads();
                if (s_slot != 0x7fffffff) break;
            }
        }
        __syncthreads();
        if (tid == 0) {
            const int slot = s_slot;
            if (s_live < P.C && slot == s_live) s_live++;
            banned[slot] = 1;
            P.attn_sum[slot] = 0.f;
            P.slot_pos[slot] = pos;
            P.dst[j] = slot;
        }
        __syncthreads();
    }
    if (tid == 0) *P.n_live = s_live;
    // quantize every (token, head, K|V) row of 64 into its slot: one warp per row
    for (int r = warp; r < P.S * P.nkv * 2; r += 8) {
        const int which = r & 1, jh = r >> 1, j = jh / P.nkv, h = jh - j * P.nkv;
        const __half* src = (which ? P.v_new : P.k_new) + ((size_t)j * P.nkv + h) * CUINF_HD;
        const float x0 = __half2float(src[2 * lane]), x1 = __half2float(src[2 * lane + 1]);
        const float mx = warp_max(fmaxf(fabsf(x0), fabsf(x1)));
        const float sc = mx / 448.0f + 1e-12f;
        const int slot = P.dst[j];
        uint8_t* d8 = (which ? P.hv8 : P.hk8) + ((size_t)slot * P.nkv + h) * CUINF_HD;
        d8[2 * lane] = (uint8_t)__nv_cvt_float_to_fp8(x0 / sc, __NV_SATFINITE, __NV_E4M3);
        d8[2 * lane + 1] = (uint8_t)__nv_cvt_float_to_fp8(x1 / sc, __NV_SATFINITE, __NV_E4M3);
        if (lane == 0) (which ? P.hvs : P.hks)[slot * P.nkv + h] = __float2half_rn(sc);
    }
}

// attention_h2o (engine.cu:337-384): query i of S (position base + i), head
// h, over the live slots with position <= the query's; exact two-pass
// softmax; each slot's normalized probability is added to its cumulative
// attention.  grid (S, nh), 256 threads, dynamic smem C floats.
__global__ void __launch_bounds__(256) k_h2o_attn(H2oParams P) {
    extern __shared__ float h2o_sm[];
    __shared__ float qs[CUINF_HD];
    __shared__ float red[32];
    __shared__ float part[4][CUINF_HD];
    const int i = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
    const int kvh = h / (P.nh / P.nkv);
    pdl_wait();
    const int qpos = (P.pos_dev ? *P.pos_dev : P.past) + i;
    const int n = *P.n_live;
    if (tid < CUINF_HD) qs[tid] = __half2float(P.q[((size_t)i * P.nh + h) * CUINF_HD + tid]);
    __syncthreads();
    float mx = -INFINITY;
    for (int t = tid; t < n; t += blockDim.x) {
        float s = -INFINITY;
        if (P.slot_pos[t] <= qpos) {
            const float ks = __half2float(P.hks[t * P.nkv + kvh]);
            const uint8_t* kp = P.hk8 + ((size_t)t * P.nkv + kvh) * CUINF_HD;
            float acc = 0.f;
#pragma unroll
            for (int d = 0; d < CUINF_HD; d += 2) {
                const uint32_t kb = fp8x2_to_h2(*reinterpret_cast<const uint16_t*>(kp + d));
                const __half2 k2 = *reinterpret_cast<const __half2*>(&kb);
                acc += qs[d] * (__low2float(k2) * ks) + qs[d + 1] * (__high2float(k2) * ks);
            }
            s = acc * P.scale;
        }
        h2o_sm[t] = s;
        mx = fmaxf(mx, s);
    }
    mx = warp_max(mx);
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    float m = -INFINITY;
    for (int w = 0; w < 8; w++) m = fmaxf(m, red[w]);
    __syncthreads();
    float l = 0.f;
    for (int t = tid; t < n; t += blockDim.x) {
        const float p = h2o_sm[t] == -INFINITY ? 0.f : __expf(h2o_sm[t] - m);
        h2o_sm[t] = p;
        l += p;
    }
    const float L = block_sum(l, red);
    __syncthreads();
    const float inv = 1.f / L;
    for (int t = tid; t < n; t += blockDim.x)
        if (h2o_sm[t] > 0.f) atomicAdd(&P.attn_sum[t], h2o_sm[t] * inv);
    // o[d] = sum_t p_t v_t[d]: four groups of 64 threads over t mod 4
    const int g = tid >> 6, d = tid & 63;
    float o = 0.f;
    for (int t = g; t < n; t += 4) {
        const float p = h2o_sm[t];
        if (p > 0.f) {
            const float vs = __half2float(P.hvs[t * P.nkv + kvh]);
            const uint8_t vb = P.hv8[((size_t)t * P.nkv + kvh) * CUINF_HD + d];
            const __half vh = __ushort_as_half((unsigned short)(fp8x2_to_h2(vb) & 0xFFFFu));
            o += p * (__half2float(vh) * vs);
        }
    }
    part[g][d] = o;
    __syncthreads();
    if (tid < CUINF_HD) {
        const float s = part[0][tid] + part[1][tid] + part[2][tid] + part[3][tid];
        P.out[((size_t)i * P.nh + h) * CUINF_HD + tid] = __float2half_rn(s * inv);
    }
}

// Prefill attention for long prompts (attention_fused, engine.cu:236-308) on
// the tensor cores: flash attention with mma.sync m16n8k16 (fp16 operands,
// fp32 accumulation).  One CTA = 64 query tokens x the GQA query heads of
// one kv head (16 rows per warp: one head, 16 tokens), so every K/V tile
// staged in shared memory serves all the heads that read it.  Keys come in
// tiles of 64 = one FP8 commit group, so a committed tile has one K and one
// V scale and both factor out of the products:
//   s = (q . k8) * (k_scale * scale)      k8: the E4M3 value, exact in fp16
//   o += (p * v_scale) . v8, l += p       p = exp(s - m), online over tiles
// which is the reference's fp32 arithmetic up to summation order (and p * v
// rounded to fp16 for the MMA).  The tail group (keys >= committed, fp16)
// has scale 1.  Keys beyond a query's position are masked, as the
// reference's loop bounds exclude them.  Tiles are double-buffered: the next
// tile's bytes are loaded into registers while the current one multiplies.
// grid (ceil(S/64), nkv) (longest key ranges first), 128 * GQA threads, GQA
// (query heads per kv head) in {1, 2, 4}.
#define APF_TOK 64
#define APF_KT 64
#define APF_PITCH 72  // halves per shared row: the 32-bit fragment loads of a warp hit 32 banks
template <int GQA>
__global__ void __launch_bounds__(128 * GQA, 1) k_attn_prefill_mma(const __half* __restrict__ q,
                                                                   const uint8_t* __restrict__ kc8,
                                                                   const uint8_t* __restrict__ vc8,
                                                                   const __half* __restrict__ ksc,
                                                                   const __half* __restrict__ vsc,
                                                                   const __half* __restrict__ ktail,
                                                                   const __half* __restrict__ vtail, int committed,
                                                                   int past, int S, float scale,
                                                                   __half* __restrict__ out, int nh, int nkv) {
    __shared__ __align__(16) __half Ks[2][APF_KT][APF_PITCH];
    __shared__ __align__(16) __half Vt[2][CUINF_HD][APF_PITCH];  // V transposed: [dim][key]
    __shared__ float kvs[2][2];                                  // per buffer: k_scale * scale, v_scale
    constexpr int nthr = 128 * GQA;
    const int nblk = (S + APF_TOK - 1) / APF_TOK;
    const int blk = nblk - 1 - (int)blockIdx.x, kvh = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
    const int hq = kvh * GQA + (warp >> 2), sub = warp & 3;
    const int i0 = blk * APF_TOK, tok0 = i0 + sub * 16;
    const int last_tok = min(i0 + APF_TOK, S) - 1;
    const int ntile = (past + last_tok + 1 + APF_KT - 1) / APF_KT;
    const int tailn = past + S - committed;  // keys in the fp16 tail (< 64)
    const int warp_last_key = tok0 < S ? past + min(tok0 + 15, S - 1) : -1;

    // query fragments (A operand, 16 tokens x 64 dims), zero past S
    uint32_t qa[4][4];
    {
        const int r0 = tok0 + g, r1 = tok0 + g + 8;
        const uint32_t* q0 = reinterpret_cast<const uint32_t*>(q + ((size_t)min(r0, S - 1) * nh + hq) * CUINF_HD);
        const uint32_t* q1 = reinterpret_cast<const uint32_t*>(q + ((size_t)min(r1, S - 1) * nh + hq) * CUINF_HD);
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            qa[kk][0] = r0 < S ? q0[8 * kk + c] : 0u;
            qa[kk][1] = r1 < S ? q1[8 * kk + c] : 0u;
            qa[kk][2] = r0 < S ? q0[8 * kk + 4 + c] : 0u;
            qa[kk][3] = r1 < S ? q1[8 * kk + 4 + c] : 0u;
        }
    }

    // tile loader: task = (key, 8-dim chunk); K by key-major tasks (16-byte
    // row stores), V by dim-chunk-major tasks (consecutive keys per warp, so
    // the transposed 2-byte stores are conflict-free)
    constexpr int ntask = (APF_KT * CUINF_HD / 8) / nthr;
    uint4 kr[ntask], vr[ntask];
    auto load = [&](int j) {
        const bool tail = j * APF_KT >= committed;
#pragma unroll
        for (int u = 0; u < ntask; u++) {
            const int task = tid + u * nthr;
            const int kk = task >> 3, ch = task & 7;    // K task
            const int vk = task & 63, vch = task >> 6;  // V task
            if (!tail) {
                const size_t kt = (size_t)(j * APF_KT + kk), vt = (size_t)(j * APF_KT + vk);
                const uint2 k2 = *reinterpret_cast<const uint2*>(kc8 + (kt * nkv + kvh) * CUINF_HD + 8 * ch);
                const uint2 v2 = *reinterpret_cast<const uint2*>(vc8 + (vt * nkv + kvh) * CUINF_HD + 8 * vch);
                kr[u] = make_uint4(k2.x, k2.y, 0u, 0u);
                vr[u] = make_uint4(v2.x, v2.y, 0u, 0u);
            } else {
                kr[u] = kk < tailn ? *reinterpret_cast<const uint4*>(ktail + ((size_t)kk * nkv + kvh) * CUINF_HD + 8 * ch)
                                   : make_uint4(0u, 0u, 0u, 0u);
                vr[u] = vk < tailn ? *reinterpret_cast<const uint4*>(vtail + ((size_t)vk * nkv + kvh) * CUINF_HD + 8 * vch)
                                   : make_uint4(0u, 0u, 0u, 0u);
            }
        }
    };
    auto store = [&](int j, int b) {
        const bool tail = j * APF_KT >= committed;
#pragma unroll
        for (int u = 0; u < ntask; u++) {
            const int task = tid + u * nthr;
            const int kk = task >> 3, ch = task & 7;
            const int vk = task & 63, vch = task >> 6;
            uint4 kh = kr[u], vh = vr[u];
            if (!tail) {
                kh = make_uint4(fp8x2_to_h2(kr[u].x), fp8x2_to_h2(kr[u].x >> 16), fp8x2_to_h2(kr[u].y),
                                fp8x2_to_h2(kr[u].y >> 16));
                vh = make_uint4(fp8x2_to_h2(vr[u].x), fp8x2_to_h2(vr[u].x >> 16), fp8x2_to_h2(vr[u].y),
                                fp8x2_to_h2(vr[u].y >> 16));
            }
            *reinterpret_cast<uint4*>(&Ks[b][kk][8 * ch]) = kh;
            const __half* v8 = reinterpret_cast<const __half*>(&vh);
#pragma unroll
            for (int e = 0; e < 8; e++) Vt[b][8 * vch + e][vk] = v8[e];
        }
        if (tid == 0) {
            kvs[b][0] = tail ? scale : __half2float(ksc[(size_t)j * nkv + kvh]) * scale;
            kvs[b][1] = tail ? 1.f : __half2float(vsc[(size_t)j * nkv + kvh]);
        }
    };

    float o[8][4], m0 = -1e30f, m1 = -1e30f, l0 = 0.f, l1 = 0.f;
#pragma unroll
    for (int nd = 0; nd < 8; nd++) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.f;
    load(0);
    store(0, 0);
    __syncthreads();
    for (int j = 0; j < ntile; j++) {
        const int b = j & 1;
        if (j + 1 < ntile) load(j + 1);
        if (j * APF_KT <= warp_last_key) {
            // S = Q K^T for 64 keys
            float sc[8][4];
#pragma unroll
            for (int nt = 0; nt < 8; nt++) {
                sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
                const __half* kr0 = &Ks[b][8 * nt + g][2 * c];
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    const uint32_t b0 = *reinterpret_cast<const uint32_t*>(kr0 + 16 * kk);
                    const uint32_t b1 = *reinterpret_cast<const uint32_t*>(kr0 + 16 * kk + 8);
                    mma_16816(sc[nt], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
                }
            }
            const float ks = kvs[b][0], vs = kvs[b][1];
            const int q0pos = past + tok0 + g, q1pos = q0pos + 8;
            float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
            for (int nt = 0; nt < 8; nt++) {
                const int key = j * APF_KT + 8 * nt + 2 * c;
                sc[nt][0] = key <= q0pos ? sc[nt][0] * ks : -INFINITY;
                sc[nt][1] = key + 1 <= q0pos ? sc[nt][1] * ks : -INFINITY;
                sc[nt][2] = key <= q1pos ? sc[nt][2] * ks : -INFINITY;
                sc[nt][3] = key + 1 <= q1pos ? sc[nt][3] * ks : -INFINITY;
                mx0 = fmaxf(mx0, fmaxf(sc[nt][0], sc[nt][1]));
                mx1 = fmaxf(mx1, fmaxf(sc[nt][2], sc[nt][3]));
            }
#pragma unroll
            for (int off = 1; off <= 2; off <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
            }
            const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
            const float cf0 = __expf(m0 - mn0), cf1 = __expf(m1 - mn1);
            m0 = mn0;
            m1 = mn1;
            l0 *= cf0;
            l1 *= cf1;
#pragma unroll
            for (int nd = 0; nd < 8; nd++) {
                o[nd][0] *= cf0;
                o[nd][1] *= cf0;
                o[nd][2] *= cf1;
                o[nd][3] *= cf1;
            }
            // P (scaled by the tile's V scale) as the A operand of O += P V
            uint32_t pa[4][4];
#pragma unroll
            for (int nt = 0; nt < 8; nt++) {
                const float p0 = __expf(sc[nt][0] - mn0), p1 = __expf(sc[nt][1] - mn0);
                const float p2 = __expf(sc[nt][2] - mn1), p3 = __expf(sc[nt][3] - mn1);
                l0 += p0 + p1;
                l1 += p2 + p3;
                const __half2 h01 = __floats2half2_rn(p0 * vs, p1 * vs), h23 = __floats2half2_rn(p2 * vs, p3 * vs);
                pa[nt >> 1][(nt & 1) * 2 + 0] = *reinterpret_cast<const uint32_t*>(&h01);
                pa[nt >> 1][(nt & 1) * 2 + 1] = *reinterpret_cast<const uint32_t*>(&h23);
            }
#pragma unroll
            for (int nd = 0; nd < 8; nd++) {
                const __half* vr0 = &Vt[b][8 * nd + g][2 * c];
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    const uint32_t b0 = *reinterpret_cast<const uint32_t*>(vr0 + 16 * kk);
                    const uint32_t b1 = *reinterpret_cast<const uint32_t*>(vr0 + 16 * kk + 8);
                    mma_16816(o[nd], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b0, b1);
                }
            }
        }
        if (j + 1 < ntile) store(j + 1, b ^ 1);
        __syncthreads();
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, off);
        l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    const float inv0 = 1.f / l0, inv1 = 1.f / l1;
    const int r0 = tok0 + g, r1 = tok0 + g + 8;
#pragma unroll
    for (int nd = 0; nd < 8; nd++) {
        if (r0 < S)
            *reinterpret_cast<__half2*>(out + ((size_t)r0 * nh + hq) * CUINF_HD + 8 * nd + 2 * c) =
                __floats2half2_rn(o[nd][0] * inv0, o[nd][1] * inv0);
        if (r1 < S)
            *reinterpret_cast<__half2*>(out + ((size_t)r1 * nh + hq) * CUINF_HD + 8 * nd + 2 * c) =
                __floats2half2_rn(o[nd][2] * inv1, o[nd][3] * inv1);
    }
}
