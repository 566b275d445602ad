// INT4 (or fp16) weights x fp16 activations on the 5th-generation tensor
// cores: the batched-decode / prefill form of gemv_int4 (engine.cu:83-109,
// y[M,N] = x[M,K] . deq(W[N,K])^T with deq = (nib-8) * scale[n, k/128]).
//
// One CTA owns a tile of 128 weight rows (the MMA's M) against up to 128
// activation rows (the MMA's N; tokens of a batch or of one expert's group)
// over a K range (split-K across CTAs, reduced in a fixed order).
//   warp 8   TMA producer of the packed INT4 rows (2-D tensor map, box
//            64 bytes x 128 rows, 64-byte swizzle) into a 4-deep ring; for
//            fp16 weights it loads the A operand directly into the three
//            A stages (128-byte swizzle);
//   warp 9   TMA producer of the activation rows (box 64 halves x xbox
//            rows, 128-byte swizzle, which is the K-major UMMA layout) into
//            their own ring of up to 8 stages, so they are requested several
//            stages ahead of the A stages they meet in the MMA;
//   warps 0-7 dequantize 128 K (one scale group) per stage to (nib-8),
//            exact in fp16 via the 1024-magic, written in the
//            128-byte-swizzled K-major layout;
//   warp 10  allocates TMEM and one thread issues tcgen05.mma.kind::f16
//            (M=128, N=rows rounded up to 16, K=16): each stage's 8 MMAs sum
//            exact products (nib-8)*x into one of three per-group
//            accumulators (128 lanes x 128 fp32 columns each);
//   warps 12-15 (lane = weight row, column = activation row) read each
//            group's sum with tcgen05.ld, multiply it by the row's fp32
//            scale and add it into a third TMEM region, so the result is the
//            reference's fp32 sum of (nib-8)*scale*x up to summation order;
//            they then run the epilogue.
// fp16 weights (lm_head) accumulate directly in the first region.
// Every wait is bounded; a time-out sets the error word and the CTA drains
// its copies and MMAs before it frees TMEM and exits.  No cluster multicast.
#pragma once
#include <cuda.h>
#include "common.cuh"

#define TC_ROWS 128
#define TC_KS 128
#define TC_NMAX 128
#define TC_PST 4     // packed-weight ring (INT4)
#define TC_NA 3      // A operand stages (dequantized INT4 or fp16 weights), 32 KB each
#define TC_XSTMAX 8  // activation stages: their own ring, so their copies run ahead of the A stages
#define TC_NACC 3   // INT4 per-group accumulators in TMEM (the sum follows them)
#define TC_DQ_WARPS 8
#define TC_ACC_WARP0 12
#define TC_THREADS ((TC_ACC_WARP0 + 4) * 32)
#define TC_A_BYTES (TC_ROWS * TC_KS * 2)  // 32 KB: two 64-K swizzle atoms
#define TC_P_BYTES (TC_ROWS * TC_KS / 2)  // 8 KB packed
#define TC_MAX_KG 64                      // scale groups per split (K range <= 8192)
#define TC_TMEM_COLS 512  // accumulators at columns 0, 128, 256; the INT4 sum at 384

struct TcGroup {
    const CUtensorMap* wmap;  // weights (global-memory tensor map); null = the launch's own map
    const uint8_t* packed;    // the same weights' packed rows (the grouped small-row GEMV reads them)
    const __half* scales;     // [N, K/128] for INT4 weights
    float* y;                 // y[j * ldy + n], j < rows
    int x_row;                // first activation row in the activation tensor map
    int rows;                 // activation rows, 0..TC_NMAX
    int N;                    // weight rows
    int ldy;
};

struct TcParams {
    const TcGroup* groups;  // device table, or null: g0, or (n_groups > 1) g0 cut into 128-row groups
    TcGroup g0;
    int n_groups;
    int m_rows;                    // without a table: g0's activation rows in all (group g = rows 128g..)
    int tiles;                     // 128-row tiles per group (of the largest N)
    int K;
    int splits, kg_per_split;
    int fp16_w;                    // weights are fp16 [N, K] (no dequantization)
    int xmax;                      // activation rows of the largest group, rounded up to 16
    int xbox;                      // rows per activation TMA box (the map's box height; divides xmax)
    float* ws;                     // split-K partials [slot][TC_NMAX][TC_ROWS]
    unsigned* counters;            // per (group, tile) arrival counters, self-resetting
    unsigned long long* amax;      // optional per activation row argmax key (lm_head)
    int n_base;                    // weight row n is vocabulary index n_base + n in the argmax keys
    unsigned* err;
};

struct TcSmem {
    uint64_t p_full[TC_PST], p_empty[TC_PST];
    uint64_t a_full[TC_NA], a_empty[TC_NA], x_full[TC_XSTMAX], x_empty[TC_XSTMAX];
    uint64_t acc_full[TC_NACC], acc_empty[TC_NACC];
    uint64_t epi;  // the four epilogue warps' own barrier (bounded, unlike bar.sync)
    uint64_t done;
    uint32_t tmem;
    int abort_;
    int last;
    unsigned long long amax[4][TC_NMAX];
};

// The A stages (TC_NA x 32 KB), then the activation stages (xmax*256 B each,
// as many as fit up to TC_XSTMAX), then the packed-weight ring (INT4).
static constexpr size_t TC_OPS_BYTES = 176 * 1024;
static constexpr size_t TC_RING_BYTES = TC_OPS_BYTES + TC_PST * (size_t)TC_P_BYTES;
static constexpr size_t TC_SMEM_BYTES = 1024 + TC_RING_BYTES + sizeof(TcSmem);
__host__ __device__ inline int tc_x_stages(int xmax) {
    const int n = (int)((TC_OPS_BYTES - (size_t)TC_NA * TC_A_BYTES) / ((size_t)xmax * TC_KS * 2));
    return n < TC_XSTMAX ? n : TC_XSTMAX;
}

__device__ __forceinline__ void tc_tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];\n" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tc_tma_2d_hint(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                               uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
        "[%1, {%2, %3}], [%4], %5;\n" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}
__device__ __forceinline__ void tc_prefetch_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(map) : "memory");
}
__device__ __forceinline__ void tc_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
// UMMA shared-memory descriptor, K-major, 128-byte swizzle: 8-row core
// groups 1024 bytes apart (SBO), leading offset unused (1), version 1.
__device__ __forceinline__ uint64_t tc_desc_sw128(const void* p) {
    const uint64_t a = smem_u32(p);
    return ((a >> 4) & 0x3FFFull) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor, kind::f16: fp32 accumulate, A = B = f16, both
// K-major, N = n, M = 128.
__device__ __forceinline__ uint32_t tc_idesc(int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(TC_ROWS >> 4) << 24);
}
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
            d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}
// tcgen05.ld of 16 columns without the wait (tc_wait_ld before use).
__device__ __forceinline__ void tc_ld16_issue(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void tc_st16(uint32_t taddr, const float (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
            taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
        "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
        "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
        : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

// A pipeline wait in these kernels takes microseconds; one that lasts this
// long has failed.
#define TC_WAIT_LIMIT_NS 200000000ull
// Bounded wait that also gives up as soon as another role of the CTA has.
// The first failure records err[1] = where (barrier code), err[2] = block,
// err[3] = the waiter's stage counter.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, TcSmem* S, unsigned* err, unsigned where = 0,
                                        unsigned ctr = 0) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (int k = 1;; k++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((k & 7) == 0) {
            if (*(volatile int*)&S->abort_) return false;
            if (globaltimer_ns() - t0 > TC_WAIT_LIMIT_NS) break;
        }
    }
    *(volatile int*)&S->abort_ = 1;
    if (err && (atomicOr(err, 2u) & 2u) == 0) {
        err[1] = where;
        err[2] = blockIdx.x;
        err[3] = ctr;
    }
    return false;
}
// Final drain: wait for a phase regardless of the abort flag (bounded).
__device__ __forceinline__ void tc_drain(uint64_t* bar, uint32_t parity, unsigned* err) {
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer_ns() - t0 > TC_WAIT_LIMIT_NS) {
            if (err) atomicOr(err, 4u);
            return;
        }
    }
}

// Diagnostic builds (-DTC_TRACE) record %globaltimer at each pipeline event
// of CTA 0; product builds compile the hooks away.
#ifdef TC_TRACE
static __device__ unsigned long long g_tc_trace[1024];
#define TC_T(slot)                                                          \
    do {                                                                    \
        if (blockIdx.x == 0 && (slot) < 1024) g_tc_trace[(slot)] = globaltimer_ns(); \
    } while (0)
#else
#define TC_T(slot) \
    do {           \
    } while (0)
#endif

// One work item = (group, 128-row tile, K split); CTA c takes items c,
// c + gridDim.x, ...  Items of empty groups (rows == 0) or beyond a group's N
// are skipped by every role alike.
struct TcItem {
    TcGroup G;
    int g, tile, split, n0, kg0, nk, npad, koff;
    // scale group of stage i: CTAs walk K from different offsets, so the SMs
    // do not all request the same activation lines from L2 at once
    __device__ __forceinline__ int kg(int i) const {
        const int j = i + koff;
        return kg0 + (j < nk ? j : j - nk);
    }
};
__device__ __forceinline__ bool tc_item(const TcParams& P, int it, int KG, TcItem& t) {
    t.split = it % P.splits;
    const int gt = it / P.splits;
    t.tile = gt % P.tiles;
    t.g = gt / P.tiles;
    if (P.groups) {
        t.G = P.groups[t.g];
    } else {
        t.G = P.g0;
        if (P.n_groups > 1) {
            t.G.x_row = P.g0.x_row + t.g * TC_NMAX;
            t.G.rows = min(TC_NMAX, P.m_rows - t.g * TC_NMAX);
            if (t.G.y) t.G.y += (size_t)t.g * TC_NMAX * t.G.ldy;
        }
    }
    t.n0 = t.tile * TC_ROWS;
    if (t.G.rows <= 0 || t.n0 >= t.G.N) return false;
    t.kg0 = t.split * P.kg_per_split;
    t.nk = min(KG, t.kg0 + P.kg_per_split) - t.kg0;
    t.npad = (t.G.rows + 15) & ~15;
    if (t.npad > P.xmax) {  // more rows than the activation stage holds: skip, report
        if (threadIdx.x == 0 && P.err) atomicOr(P.err, 8u);
        return false;
    }
    t.koff = t.nk > 0 ? (int)((blockIdx.x * 5u + (unsigned)t.tile) % (unsigned)t.nk) : 0;
    return t.nk > 0;
}

__global__ void __launch_bounds__(TC_THREADS, 1)
    k_tc_gemm(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap0, const TcParams P) {
    extern __shared__ __align__(1024) unsigned char tc_raw[];
    const int KG = P.K / TC_KS;
    const int n_items = P.n_groups * P.tiles * P.splits;
    const int nx = tc_x_stages(P.xmax);
    const int xatom = P.xmax * 128;  // bytes of one 64-K swizzle atom of activations

    unsigned char* sm = tc_raw + ((1024 - (smem_u32(tc_raw) & 1023)) & 1023);
    unsigned char* PK = sm + TC_OPS_BYTES;  // INT4 only
    TcSmem* S = reinterpret_cast<TcSmem*>(sm + TC_RING_BYTES);
    auto A_of = [&](int s) { return sm + (size_t)s * TC_A_BYTES; };
    auto X_of = [&](int s) { return sm + (size_t)TC_NA * TC_A_BYTES + (size_t)s * 2 * xatom; };
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0) {
        for (int i = 0; i < TC_PST; i++) {
            mbar_init(&S->p_full[i], 1);
            mbar_init(&S->p_empty[i], TC_DQ_WARPS);
        }
        for (int i = 0; i < TC_NA; i++) {
            mbar_init(&S->a_full[i], P.fp16_w ? 1 : TC_DQ_WARPS);
            mbar_init(&S->a_empty[i], 1);
        }
        for (int i = 0; i < TC_XSTMAX; i++) {
            mbar_init(&S->x_full[i], 1);
            mbar_init(&S->x_empty[i], 1);
        }
        for (int i = 0; i < TC_NACC; i++) {
            mbar_init(&S->acc_full[i], 1);
            mbar_init(&S->acc_empty[i], 4);
        }
        mbar_init(&S->epi, 4);
        mbar_init(&S->done, 1);
        S->abort_ = 0;
    }
    if (warp == TC_DQ_WARPS + 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(&S->tmem)),
                     "r"(TC_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    if (tid == 0) TC_T(0);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S->tmem;
    if (tid == 0) TC_T(1);

    // The producer and MMA warps iterate warp-uniformly (all lanes walk the
    // items and stages; lane 0 waits and issues, the result is broadcast), so
    // the issuing lane never runs diverged from a parked warp.
    if (warp == TC_DQ_WARPS) {
        // ---- weight producer ----
        const uint64_t pol = l2_policy_evict_first();
        // last copy issued per stage: the INT4 ring (TC_PST) or, for fp16
        // weights, the A stages (TC_NA)
        constexpr int NLAST = TC_PST > TC_NA ? TC_PST : TC_NA;
        int last[NLAST];
        for (int s = 0; s < NLAST; s++) last[s] = -1;
        uint32_t pc = 0;
        bool ok = true;
        if (lane == 0 && !P.groups) tc_prefetch_map(&wmap0);
        const CUtensorMap* prev = nullptr;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            TcItem t;
            if (!tc_item(P, it, KG, t)) continue;
            const CUtensorMap* wm = t.G.wmap ? t.G.wmap : &wmap0;
            if (wm != prev) {
                if (lane == 0) tc_prefetch_map(wm);
                prev = wm;
            }
            for (int i = 0; i < t.nk; i++, pc++) {
                const int kg = t.kg(i);
                const int s = P.fp16_w ? (int)(pc % TC_NA) : (int)(pc % TC_PST);
                bool w = true;
                if (lane == 0) {
                    if (P.fp16_w) {
                        w = tc_wait(&S->a_empty[s], ((pc / TC_NA) & 1) ^ 1, S, P.err, 10 + s, pc);
                        if (w) {
                            mbar_arrive_expect_tx(&S->a_full[s], TC_A_BYTES);
                            tc_tma_2d_hint(A_of(s), wm, kg * TC_KS, t.n0, &S->a_full[s], pol);
                            tc_tma_2d_hint(A_of(s) + TC_A_BYTES / 2, wm, kg * TC_KS + 64, t.n0, &S->a_full[s], pol);
                        }
                    } else {
                        w = tc_wait(&S->p_empty[s], ((pc / TC_PST) & 1) ^ 1, S, P.err, 20 + s, pc);
                        if (w) {
                            mbar_arrive_expect_tx(&S->p_full[s], TC_P_BYTES);
                            tc_tma_2d_hint(PK + s * TC_P_BYTES, wm, kg * (TC_KS / 2), t.n0, &S->p_full[s], pol);
                            if (pc < 64) TC_T(16 + pc);
                        }
                    }
                }
                if (!(ok = __shfl_sync(0xffffffffu, (int)w, 0) != 0)) break;
                last[s] = (int)pc;
            }
        }
        // copies still in flight land before the CTA can exit
        if (lane == 0) {
            const int depth = P.fp16_w ? TC_NA : TC_PST;
            for (int s = 0; s < depth; s++)
                if (last[s] >= 0) tc_drain(P.fp16_w ? &S->a_full[s] : &S->p_full[s], (last[s] / depth) & 1, P.err);
        }
        __syncwarp();
    } else if (warp == TC_DQ_WARPS + 1) {
        // ---- activation producer ----
        if (lane == 0) tc_prefetch_map(&xmap);
        pdl_wait();
        int last[TC_XSTMAX];
        for (int s = 0; s < TC_XSTMAX; s++) last[s] = -1;
        uint32_t oc = 0;
        bool ok = true;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            TcItem t;
            if (!tc_item(P, it, KG, t)) continue;
            for (int i = 0; i < t.nk; i++, oc++) {
                const int s = oc % nx;
                bool w = true;
                if (lane == 0) {
                    w = tc_wait(&S->x_empty[s], ((oc / nx) & 1) ^ 1, S, P.err, 30 + s, oc);
                    if (w) {
                        const int nb = (t.npad + P.xbox - 1) / P.xbox;
                        mbar_arrive_expect_tx(&S->x_full[s], (uint32_t)(nb * P.xbox) * TC_KS * 2);
                        if (oc < 64) TC_T(80 + oc);
                        const int kx = t.kg(i) * TC_KS;
                        for (int a = 0; a < 2; a++)
                            for (int b = 0; b < nb; b++)
                                tc_tma_2d(X_of(s) + a * xatom + b * P.xbox * 128, &xmap, kx + 64 * a,
                                          t.G.x_row + P.xbox * b, &S->x_full[s]);
                    }
                }
                if (!(ok = __shfl_sync(0xffffffffu, (int)w, 0) != 0)) break;
                last[s] = (int)oc;
            }
        }
        if (lane == 0)
            for (int s = 0; s < nx; s++)
                if (last[s] >= 0) tc_drain(&S->x_full[s], (last[s] / nx) & 1, P.err);
        __syncwarp();
    } else if (warp == TC_DQ_WARPS + 2) {
        // ---- MMA issuer ----
        uint32_t oc = 0, ac = 0, ic = 0;
        bool ok = true;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            TcItem t;
            if (!tc_item(P, it, KG, t)) continue;
            const uint32_t idesc = tc_idesc(t.npad);
            uint32_t d = 0;
            if (P.fp16_w) {  // the item accumulates in region ic%3, free once read back
                const uint32_t a3 = ic % TC_NACC;
                bool w = true;
                if (lane == 0) w = tc_wait(&S->acc_empty[a3], ((ic / TC_NACC) & 1) ^ 1, S, P.err, 40 + a3, ic);
                if (!(ok = __shfl_sync(0xffffffffu, (int)w, 0) != 0)) break;
                d = tmem + a3 * 128;
            }
            for (int i = 0; i < t.nk; i++, oc++) {
                const int s = oc % TC_NA, sx = oc % nx;
                const uint32_t ph = (oc / TC_NA) & 1, phx = (oc / nx) & 1;
                const uint32_t a3 = ac % TC_NACC;
                bool w = true;
                if (lane == 0) {
                    w = tc_wait(&S->a_full[s], ph, S, P.err, 50 + s, oc) && tc_wait(&S->x_full[sx], phx, S, P.err, 60 + sx, oc);
                    // INT4: one accumulator per scale group, read back by the scale warps
                    if (w && !P.fp16_w) w = tc_wait(&S->acc_empty[a3], ((ac / TC_NACC) & 1) ^ 1, S, P.err, 70 + a3, ac);
                    if (w) {
                        if (!P.fp16_w) d = tmem + a3 * 128;
                        tc_fence_after();
                        if (oc < 64) TC_T(272 + oc);
#pragma unroll
                        for (int kk = 0; kk < TC_KS / 16; kk++) {
                            const int off = (kk >> 2) * (TC_A_BYTES / 2) + (kk & 3) * 32;
                            const int xoff = (kk >> 2) * xatom + (kk & 3) * 32;
                            tc_mma(d, tc_desc_sw128(A_of(s) + off), tc_desc_sw128(X_of(sx) + xoff), idesc,
                                   P.fp16_w ? (i | kk) != 0 : kk != 0);
                        }
                        tc_commit(&S->a_empty[s]);
                        tc_commit(&S->x_empty[sx]);
                        if (!P.fp16_w) tc_commit(&S->acc_full[a3]);
                    }
                }
                if (!(ok = __shfl_sync(0xffffffffu, (int)w, 0) != 0)) break;
                if (!P.fp16_w) ac++;
            }
            if (ok && P.fp16_w) {
                if (lane == 0) tc_commit(&S->acc_full[ic % TC_NACC]);
                ic++;
            }
        }
        if (lane == 0) tc_commit(&S->done);  // tracks every MMA issued above
        __syncwarp();
    } else if (warp < TC_DQ_WARPS) {
        // ---- dequantization (INT4 weights) to exact (nib-8) ----
        const int r = tid & (TC_ROWS - 1), h = tid >> 7;
        if (!P.fp16_w) {
            uint32_t pc = 0, oc = 0;
            bool ok = true;
            for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
                TcItem t;
                if (!tc_item(P, it, KG, t)) continue;
                for (int i = 0; i < t.nk; i++, pc++, oc++) {
                    const int s = pc % TC_PST;
                    if (!(ok = tc_wait(&S->p_full[s], (pc / TC_PST) & 1, S, P.err, 80 + s, pc))) break;
                    if (tid == 0 && pc < 64) TC_T(144 + pc);
                    const unsigned char* row = PK + s * TC_P_BYTES + r * 64;
                    const int sw = (r >> 1) & 3;
                    const uint4 c0 = *reinterpret_cast<const uint4*>(row + (((2 * h) ^ sw) << 4));
                    const uint4 c1 = *reinterpret_cast<const uint4*>(row + (((2 * h + 1) ^ sw) << 4));
                    __syncwarp();
                    if (lane == 0) tc_arrive(&S->p_empty[s]);
                    const int so = oc % TC_NA;
                    if (!(ok = tc_wait(&S->a_empty[so], ((oc / TC_NA) & 1) ^ 1, S, P.err, 90 + so, oc))) break;
                    unsigned char* dst = A_of(so) + h * (TC_A_BYTES / 2) + r * 128;
                    const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        uint32_t q[4];
                        dequant8(w[j], q);  // (k0,k4) (k1,k5) (k2,k6) (k3,k7)
                        uint4 o;
                        o.x = __byte_perm(q[0], q[1], 0x5410);
                        o.y = __byte_perm(q[2], q[3], 0x5410);
                        o.z = __byte_perm(q[0], q[1], 0x7632);
                        o.w = __byte_perm(q[2], q[3], 0x7632);
                        *reinterpret_cast<uint4*>(dst + ((j ^ (r & 7)) << 4)) = o;
                    }
                    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                    __syncwarp();
                    if (lane == 0) tc_arrive(&S->a_full[so]);
                    if (tid == 0 && oc < 64) TC_T(208 + oc);
                }
            }
        }
    } else if (warp >= TC_ACC_WARP0) {
        // ---- per-group scale-accumulate, then the epilogue of each item ----
        // warp 12+q reads TMEM lanes 32q..32q+31 = weight rows
        const int q = warp - TC_ACC_WARP0, atid = tid - TC_ACC_WARP0 * 32;
        const int rr = q * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
        uint32_t ac = 0, ic = 0, ek = 0;
        bool ok = true, waited = false;
        // bounded barrier of the four epilogue warps (gives up on abort)
        auto sync4 = [&]() -> bool {
            __syncwarp();
            if (lane == 0) tc_arrive(&S->epi);
            const bool r = tc_wait(&S->epi, ek & 1, S, P.err, 120, ek);
            ek++;
            return r;
        };
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            TcItem t;
            if (!tc_item(P, it, KG, t)) continue;
            const TcGroup& G = t.G;
            const int n = t.n0 + rr;
            uint32_t res;
            if (!P.fp16_w) {
                const __half* srow = G.scales + (size_t)min(n, G.N - 1) * KG;
                float sc_next = n < G.N ? __half2float(__ldg(srow + t.kg(0))) : 0.f;
                for (int i = 0; i < t.nk; i++, ac++) {
                    const float sc = sc_next;
                    if (i + 1 < t.nk) sc_next = n < G.N ? __half2float(__ldg(srow + t.kg(i + 1))) : 0.f;
                    const uint32_t a3 = ac % TC_NACC;
                    if (!(ok = tc_wait(&S->acc_full[a3], (ac / TC_NACC) & 1, S, P.err, 100 + a3, ac))) break;
                    if (atid == 0 && ac < 64) TC_T(336 + ac);
                    tc_fence_after();
                    const uint32_t ab = lane_base + a3 * 128, yb = lane_base + 384;
                    // 32 columns per round: both loads issued, one wait
                    for (int c = 0; c < t.npad; c += 32) {
                        const bool two = c + 16 < t.npad;
                        uint32_t a[32], y[32];
                        tc_ld16_issue(ab + c, a);
                        if (two) tc_ld16_issue(ab + c + 16, a + 16);
                        if (i > 0) {
                            tc_ld16_issue(yb + c, y);
                            if (two) tc_ld16_issue(yb + c + 16, y + 16);
                        }
                        tc_wait_ld();
                        float o[32];
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            o[j] = i == 0 ? sc * __uint_as_float(a[j]) : fmaf(sc, __uint_as_float(a[j]), __uint_as_float(y[j]));
                        tc_st16(yb + c, *reinterpret_cast<const float(*)[16]>(o));
                        if (two) tc_st16(yb + c + 16, *reinterpret_cast<const float(*)[16]>(o + 16));
                    }
                    tc_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) tc_arrive(&S->acc_empty[a3]);
                    if (atid == 0 && ac < 64) TC_T(400 + ac);
                }
                if (!ok) break;
                res = lane_base + 384;
            } else {
                const uint32_t a3 = ic % TC_NACC;
                if (!(ok = tc_wait(&S->acc_full[a3], (ic / TC_NACC) & 1, S, P.err, 110 + a3, ic))) break;
                tc_fence_after();
                res = lane_base + a3 * 128;
            }
            if (!waited) {
                pdl_wait();
                waited = true;
            }
            const bool live = !*(volatile int*)&S->abort_;
            if (P.splits == 1) {
                for (int c = 0; c < t.npad; c += 16) {
                    float v[16];
                    tc_ld16(res + c, v);
                    if (!live) continue;
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        if (c + j >= G.rows) break;
                        if (n < G.N && G.y) G.y[(size_t)(c + j) * G.ldy + n] = v[j];
                        if (P.amax) {
                            unsigned long long key = n < G.N ? argmax_key(v[j], P.n_base + n) : 0ull;
#pragma unroll
                            for (int o = 16; o; o >>= 1) key = umax64_dev(key, __shfl_xor_sync(0xffffffffu, key, o));
                            if (lane == 0) S->amax[q][c + j] = key;
                        }
                    }
                }
                if (P.amax) {
                    if (!(ok = sync4())) break;
                    if (live && atid < G.rows) {
                        unsigned long long k = S->amax[0][atid];
                        for (int w = 1; w < 4; w++) k = umax64_dev(k, S->amax[w][atid]);
                        atomicMax(&P.amax[G.x_row + atid], k);
                    }
                    if (!(ok = sync4())) break;  // S->amax is reused by the next item
                }
            } else {
                const size_t tile = (size_t)t.g * P.tiles + t.tile;
                const size_t SLOT = (size_t)TC_NMAX * TC_ROWS;
                float* mine = P.ws + (tile * P.splits + t.split) * SLOT;
                for (int c = 0; c < t.npad; c += 16) {
                    float v[16];
                    tc_ld16(res + c, v);
#pragma unroll
                    for (int j = 0; j < 16; j++) __stcg(&mine[(c + j) * TC_ROWS + rr], v[j]);
                }
                __threadfence();
                if (!(ok = sync4())) break;
                if (atid == 0) {
                    const unsigned tk = atomicAdd(&P.counters[tile], 1u);
                    S->last = tk == (unsigned)P.splits - 1;
                    if (S->last) P.counters[tile] = 0;  // ready for the next launch
                }
                if (!(ok = sync4())) break;
                if (S->last && live && n < G.N) {
                    __threadfence();
                    const float* base = P.ws + tile * P.splits * SLOT;
                    for (int j0 = 0; j0 < G.rows; j0 += 8) {
                        float acc[8];
#pragma unroll
                        for (int u = 0; u < 8; u++) acc[u] = 0.f;
                        for (int sp = 0; sp < P.splits; sp++) {
                            float v[8];
#pragma unroll
                            for (int u = 0; u < 8; u++)
                                v[u] = j0 + u < G.rows ? __ldcg(&base[sp * SLOT + (size_t)(j0 + u) * TC_ROWS + rr]) : 0.f;
#pragma unroll
                            for (int u = 0; u < 8; u++) acc[u] += v[u];
                        }
#pragma unroll
                        for (int u = 0; u < 8; u++)
                            if (j0 + u < G.rows) G.y[(size_t)(j0 + u) * G.ldy + n] = acc[u];
                    }
                }
            }
            if (atid == 0) TC_T(464 + (it / gridDim.x < 32 ? it / gridDim.x : 31));
            if (P.fp16_w) {  // every lane advances ic; lane 0 arrives for the warp
                tc_fence_before();
                __syncwarp();
                if (lane == 0) tc_arrive(&S->acc_empty[ic % TC_NACC]);
                ic++;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (tid == 0) TC_T(500);
    if (warp == TC_DQ_WARPS + 2) {
        tc_fence_after();
        if (lane == 0) tc_drain(&S->done, 0, P.err);  // all MMAs retired before TMEM is freed
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(TC_TMEM_COLS)
                     : "memory");
    }
}
