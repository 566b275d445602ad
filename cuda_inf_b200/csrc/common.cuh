// Shared device helpers for the sm_100a decode hot path.
#pragma once
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/cuinf.h"

#define CUINF_HD 64       // head_dim (fixed by the reference: HEAD_DIM, engine.cu:35)
#define CUINF_KVGROUP 64  // FP8 KV commit group (KVGROUP, engine.cu:23)
#define CUINF_QGROUP 128  // INT4 scale group along K (GROUP, engine.cu:46)

// ---------------------------------------------------------------------------
// host-side status helpers
// ---------------------------------------------------------------------------
#define CUINF_TRY(expr)                                         \
    do {                                                        \
        cudaError_t e_ = (expr);                                \
        if (e_ != cudaSuccess) return cuinf_set_cuda_error(e_); \
    } while (0)

int cuinf_set_cuda_error(cudaError_t e);
int cuinf_set_arg_error(const char* what);
int cuinf_launch_status();

// ---------------------------------------------------------------------------
// loads
// ---------------------------------------------------------------------------
// Streaming 16-byte load of weights: read-only path, no L1 allocation.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint4 ldg_stream256(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint2 ldg_stream8(const void* p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];\n"
                 : "=r"(r.x), "=r"(r.y)
                 : "l"(p));
    return r;
}
// Bulk prefetch of [p, p+bytes) into L2 (TMA unit, no completion tracking).
// p must be 16-byte aligned and bytes a multiple of 16.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------------------
// TMA bulk copies (global -> this CTA's shared memory) tracked by an mbarrier,
// and programmatic dependent launch.  No multicast anywhere.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
// dst (shared) and src (global) 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void tma_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// L2 cache policy for data read once per step (weights streamed from HBM):
// evict those lines first so they do not push out activations, the KV cache
// or kernel code that is reused.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void tma_load_1d_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                 uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;\n" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}
// Non-blocking test of phase `parity` of bar.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Potentially blocking test of phase `parity`: the thread may be suspended in
// hardware until the phase completes or a short system time limit passes, and
// resumes as soon as the phase completes (no sleep granularity).
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;\n" : "=l"(t));
    return t;
}
// Phase timestamps of the decode-step kernels, for diagnostic builds only
// (-DCUINF_PHASE_TRACE, `python -m cuda_inf_b200.build --trace`): thread 0
// of every CTA stores %globaltimer at each marked phase of its kernel's
// latest launch (kernel id k, phase i < 11; slot 11 = the CTA's SM).
// Product builds compile the marks away.
#define PH_QKV 0
#define PH_RES 1
#define PH_CONV 2
#define PH_FFN 3
#define PH_MOE_UP 4
#define PH_MOE_DOWN 5
#define PH_LMHEAD 6
#define PH_ATTN 7
#ifdef CUINF_PHASE_TRACE
static __device__ unsigned long long g_phase[8][1024][12];
__device__ __forceinline__ void phase_mark(int k, int i) {
    if (threadIdx.x == 0) {
        const unsigned cta = blockIdx.x + blockIdx.y * gridDim.x;
        if (cta < 1024) {
            g_phase[k][cta][i] = globaltimer_ns();
            if (i == 0) {
                unsigned sm;
                asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
                g_phase[k][cta][11] = sm;
            }
        }
    }
}
#define PHASE(k, i) phase_mark(k, i)
#else
#define PHASE(k, i) \
    do {            \
    } while (0)
#endif

// Every wait in these kernels gives up after this long (wall time), sets an
// error flag and lets the kernel finish.
#define CUINF_WAIT_LIMIT_NS 4000000000ull
// Wait for phase `parity` of bar, at most CUINF_WAIT_LIMIT_NS.  On time-out
// the flag word (if given) is set and false returned; the caller then skips
// its math but still waits (bounded) before exiting so no copy targets freed
// shared memory.
__device__ __forceinline__ bool mbar_wait_bounded_ns(uint64_t* bar, uint32_t parity, unsigned* flag,
                                                     uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (int k = 1;; k++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((k & 7) == 0 && globaltimer_ns() - t0 > limit_ns) break;
    }
    if (flag) atomicOr(flag, 1u);
    return false;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned* flag) {
    return mbar_wait_bounded_ns(bar, parity, flag, CUINF_WAIT_LIMIT_NS);
}
// PDL: let the next kernel in the stream start launching, and wait until the
// previous kernel has completed and its writes are visible.  Both are no-ops
// when the launch carries no programmatic-serialization attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

// Bytes of one 16-row INT4 tile staged in shared memory: packed rows then
// their scales (K % 64 == 0 keeps every tile 16-byte aligned).
__host__ __device__ __forceinline__ uint32_t int4_tile_bytes(int K) {
    return 16u * (uint32_t)(K >> 1) + 16u * (uint32_t)(K >> 6);
}
// Thread-0 helper: TMA one full 16-row tile (rows row0..row0+15 of W[N,K])
// into dst; returns the bytes it will deliver to bar.  Weights are read once
// per step, so their L2 lines are marked evict-first.
__device__ __forceinline__ uint32_t tma_tile_int4(const uint8_t* packed, const __half* scales, int K,
                                                  int row0, uint8_t* dst, uint64_t* bar) {
    const uint32_t pb = 16u * (uint32_t)(K >> 1), sb = 16u * (uint32_t)(K >> 6);
    const uint64_t pol = l2_policy_evict_first();
    tma_load_1d_hint(dst, packed + (size_t)row0 * (K >> 1), pb, bar, pol);
    tma_load_1d_hint(dst + pb, (const uint8_t*)scales + (size_t)row0 * (K >> 6), sb, bar, pol);
    return pb + sb;
}

// Shared-memory pitch for rows of H fp16 values: 64 mod 128 bytes, so the
// 16-byte loads of two neighbouring rows by one 8-lane phase of a warp fall
// in different banks (rows H*2 = 4096 bytes apart would all hit the same).
__host__ __device__ __forceinline__ unsigned f16_row_pitch(int H) {
    const unsigned b = 2u * (unsigned)H;
    return b + ((64u - (b & 127u)) & 127u);
}

// Up to 8 byte ranges (16-byte aligned starts and sizes) to pull into L2.
struct L2Ranges {
    const char* p[8];
    unsigned long long n[8];
    int count;
};

// Part `part` of `nparts` of the concatenated ranges is prefetched into L2
// by the calling thread, in bulk pieces of at most 64 KB.
__device__ __forceinline__ void l2_prefetch_share(const L2Ranges& R, int part, int nparts) {
    unsigned long long total = 0;
    for (int i = 0; i < R.count; i++) total += R.n[i];
    if (total == 0) return;
    unsigned long long per = ((total + nparts - 1) / nparts + 15) & ~15ull;
    unsigned long long beg = (unsigned long long)part * per, end = beg + per;
    if (end > total) end = total;
    unsigned long long base = 0;
    for (int i = 0; i < R.count && beg < end; i++) {
        const unsigned long long rb = base, re = base + R.n[i];
        base = re;
        if (re <= beg || rb >= end) continue;
        unsigned long long a = beg > rb ? beg : rb, b = end < re ? end : re;
        const char* p = R.p[i] + (a - rb);
        unsigned long long len = b - a;
        if (((uintptr_t)p & 15) != 0) continue;
        while (len >= 16) {
            unsigned piece = len > 65536 ? 65536u : (unsigned)(len & ~15ull);
            prefetch_l2_bulk(p, piece);
            p += piece;
            len -= piece;
        }
    }
}

// L2 prefetch of one 16-row INT4 tile (rows are contiguous, scales follow
// the same row order).
__device__ __forceinline__ void l2_prefetch_tile_int4(const uint8_t* packed, const __half* scales,
                                                      int K, int row0, int rows) {
    const char* p = (const char*)packed + (size_t)row0 * (K >> 1);
    const char* s = (const char*)scales + (size_t)row0 * (K >> 6);
    const unsigned pb = (unsigned)rows * (K >> 1), sb = (unsigned)rows * (K >> 6);
    if ((((uintptr_t)p | pb) & 15) == 0) prefetch_l2_bulk(p, pb);
    if ((((uintptr_t)s | sb) & 15) == 0) prefetch_l2_bulk(s, sb);
}

// L2 prefetch of rows [row0, row0+rows) of an fp16 matrix [N,K] (clamped to N).
__device__ __forceinline__ void l2_prefetch_bulk_rows(const __half* W, int N, int K, int row0, int rows) {
    const int r1 = min(row0 + rows, N);
    if (r1 <= row0) return;
    const char* p = (const char*)(W + (size_t)row0 * K);
    unsigned long long len = (unsigned long long)(r1 - row0) * K * 2;
    if (((uintptr_t)p & 15) != 0) return;
    while (len >= 16) {
        unsigned piece = len > 65536 ? 65536u : (unsigned)(len & ~15ull);
        prefetch_l2_bulk(p, piece);
        p += piece;
        len -= piece;
    }
}

// ---------------------------------------------------------------------------
// tensor-core fragment math (mma.sync m16n8k16, f16 in, f32 accumulate)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(d) : "r"(a), "r"(b), "r"(c));  // (a & b) | c
    return d;
}
__device__ __forceinline__ uint32_t hadd2_u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.f16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hmul2_u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Dequantize one 32-bit word of packed INT4 (8 nibbles, k0..k7; byte j holds
// k=2j in its low nibble, tools/export_weights.py:74-77) into four f16x2
// registers holding (nibble - 8), exact in fp16:
//   h[0] = (k0,k4)  h[1] = (k1,k5)  h[2] = (k2,k6)  h[3] = (k3,k7)
// Low nibbles are OR-ed into the mantissa of 1024.0 and 1032 is subtracted;
// high nibbles land as 1024 + 16n and are mapped by n/16*... = t/16 - 72.
__device__ __forceinline__ void dequant8(uint32_t w, uint32_t (&h)[4]) {
    const uint32_t LO = 0x000F000Fu, HI = 0x00F000F0u, EX = 0x64006400u;
    const uint32_t NEG1032 = 0xE408E408u;  // -1032.0 in both halves
    const uint32_t SIXTEENTH = 0x2C002C00u; // 1/16
    const uint32_t NEG72 = 0xD480D480u;     // -72.0
    uint32_t w8 = w >> 8;
    h[0] = hadd2_u(lop3_and_or(w, LO, EX), NEG1032);
    h[1] = hfma2_u(lop3_and_or(w, HI, EX), SIXTEENTH, NEG72);
    h[2] = hadd2_u(lop3_and_or(w8, LO, EX), NEG1032);
    h[3] = hfma2_u(lop3_and_or(w8, HI, EX), SIXTEENTH, NEG72);
}

// x in "B-fragment order" for the INT4 tile core.  For group G (128 k values),
// mma m (0..7) and lane quad c (0..3) the 4 halves at index ((G*8+m)*4+c)*4 are
//   m even: x[k], x[k+4], x[k+1], x[k+5]     m odd: x[k+2], x[k+6], x[k+3], x[k+7]
// with k = 128G + 32c + 8(m/2).  This matches the A-fragment slots that
// dequant8 produces from the 16-byte chunk c of a row's group G.
__device__ __forceinline__ void build_xB_entry(const __half* x, __half* xB, int e) {
    int c = e & 3, m = (e >> 2) & 7, G = e >> 5;
    int k = 128 * G + 32 * c + 8 * (m >> 1) + ((m & 1) ? 2 : 0);
    __half* o = xB + (size_t)e * 4;
    o[0] = x[k];
    o[1] = x[k + 4];
    o[2] = x[k + 1];
    o[3] = x[k + 5];
}
// Chunk i of x (elements 8i..8i+7, one 16-byte load; x 16-byte aligned)
// into its two B-fragment entries: entry m = 2j and m = 2j+1 of quad c of
// group G for 8i = 128G + 32c + 8j, the same layout build_xB_entry writes.
__device__ __forceinline__ void build_xB_chunk(const __half* x, __half* xB, int i) {
    const uint4 v = *reinterpret_cast<const uint4*>(x + 8 * i);
    const __half* o = reinterpret_cast<const __half*>(&v);
    const int G = i >> 4, c = (i >> 2) & 3, j = i & 3;
    __half2* e0 = reinterpret_cast<__half2*>(xB + (size_t)((G * 8 + 2 * j) * 4 + c) * 4);
    __half2* e1 = reinterpret_cast<__half2*>(xB + (size_t)((G * 8 + 2 * j + 1) * 4 + c) * 4);
    e0[0] = __halves2half2(o[0], o[4]);
    e0[1] = __halves2half2(o[1], o[5]);
    e1[0] = __halves2half2(o[2], o[6]);
    e1[1] = __halves2half2(o[3], o[7]);
}
// Same, reading x from shared memory with a float source.
__device__ __forceinline__ void build_xB_entry_f(const float* x, __half* xB, int e) {
    int c = e & 3, m = (e >> 2) & 7, G = e >> 5;
    int k = 128 * G + 32 * c + 8 * (m >> 1) + ((m & 1) ? 2 : 0);
    __half* o = xB + (size_t)e * 4;
    o[0] = __float2half_rn(x[k]);
    o[1] = __float2half_rn(x[k + 4]);
    o[2] = __float2half_rn(x[k + 1]);
    o[3] = __float2half_rn(x[k + 5]);
}

// INT4 tile core.  One warp, 16 rows [row0, row0+16) of W[N,K] (INT4 G=128
// layout of tools/export_weights.py), groups gbeg, gbeg+gstep, ... < gend.
// Lane (g = lane/4, c = lane%4) returns partial dot products for rows row0+g
// (y0) and row0+g+8 (y1); all four lanes of a quad hold the same values.
// Rows >= N are clamped for loading (their results must be discarded).
// Per group: two 16-byte loads per lane, 8 mma.m16n8k16 with fp32
// accumulation of (nibble-8)*x, then one fp32 FMA with the group's scale.
template <int UNROLL>
__device__ __forceinline__ void int4_tile_dot(const uint8_t* __restrict__ packed,
                                              const __half* __restrict__ scales, int N, int K,
                                              int row0, int gbeg, int gend, int gstep,
                                              const uint2* __restrict__ xB, float& y0, float& y1) {
    const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int ra = min(row0 + g, N - 1), rb = min(row0 + g + 8, N - 1);
    const int KG = K >> 7;
    const uint8_t* pa = packed + (size_t)ra * (K >> 1) + c * 16;
    const uint8_t* pb = packed + (size_t)rb * (K >> 1) + c * 16;
    const __half* sa = scales + (size_t)ra * KG;
    const __half* sb = scales + (size_t)rb * KG;
    for (int G0 = gbeg; G0 < gend; G0 += gstep * UNROLL) {
        uint4 wa[UNROLL], wb[UNROLL];
        float fa[UNROLL], fb[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            int G = G0 + u * gstep;
            if (G < gend) {
                wa[u] = ldg_stream(pa + (size_t)G * 64);
                wb[u] = ldg_stream(pb + (size_t)G * 64);
                fa[u] = __half2float(sa[G]);
                fb[u] = __half2float(sb[G]);
            }
        }
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            int G = G0 + u * gstep;
            if (G < gend) {
                float d[4] = {0.f, 0.f, 0.f, 0.f};
                const uint2* xg = xB + (size_t)G * 32 + c;
                const uint32_t wav[4] = {wa[u].x, wa[u].y, wa[u].z, wa[u].w};
                const uint32_t wbv[4] = {wb[u].x, wb[u].y, wb[u].z, wb[u].w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    uint32_t ha[4], hb[4];
                    dequant8(wav[j], ha);
                    dequant8(wbv[j], hb);
                    uint2 b0 = xg[(2 * j) * 4];
                    uint2 b1 = xg[(2 * j + 1) * 4];
                    mma_16816(d, ha[0], hb[0], ha[1], hb[1], b0.x, b0.y);
                    mma_16816(d, ha[2], hb[2], ha[3], hb[3], b1.x, b1.y);
                }
                y0 = fmaf(fa[u], d[0], y0);
                y1 = fmaf(fb[u], d[2], y1);
            }
        }
    }
}

// INT4 tile core over a tile staged in shared memory by tma_tile_int4:
// packed [16][K/2] then scales [16][K/128].  Same lane mapping and math as
// int4_tile_dot.
template <int UNROLL>
__device__ __forceinline__ void int4_tile_dot_smem(const uint8_t* tile, int K, int gbeg, int gend,
                                                   int gstep, const uint2* __restrict__ xB, float& y0,
                                                   float& y1) {
    const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int KH = K >> 1, KG = K >> 7;
    const uint8_t* pa = tile + g * KH + c * 16;
    const uint8_t* pb = tile + (g + 8) * KH + c * 16;
    const __half* sc = reinterpret_cast<const __half*>(tile + 16 * KH);
    const __half* sa = sc + g * KG;
    const __half* sb = sc + (g + 8) * KG;
    for (int G0 = gbeg; G0 < gend; G0 += gstep * UNROLL) {
        uint4 wa[UNROLL], wb[UNROLL];
        float fa[UNROLL], fb[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            int G = G0 + u * gstep;
            if (G < gend) {
                wa[u] = *reinterpret_cast<const uint4*>(pa + G * 64);
                wb[u] = *reinterpret_cast<const uint4*>(pb + G * 64);
                fa[u] = __half2float(sa[G]);
                fb[u] = __half2float(sb[G]);
            }
        }
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            int G = G0 + u * gstep;
            if (G < gend) {
                float d[4] = {0.f, 0.f, 0.f, 0.f};
                const uint2* xg = xB + (size_t)G * 32 + c;
                const uint32_t wav[4] = {wa[u].x, wa[u].y, wa[u].z, wa[u].w};
                const uint32_t wbv[4] = {wb[u].x, wb[u].y, wb[u].z, wb[u].w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    uint32_t ha[4], hb[4];
                    dequant8(wav[j], ha);
                    dequant8(wbv[j], hb);
                    uint2 b0 = xg[(2 * j) * 4];
                    uint2 b1 = xg[(2 * j + 1) * 4];
                    mma_16816(d, ha[0], hb[0], ha[1], hb[1], b0.x, b0.y);
                    mma_16816(d, ha[2], hb[2], ha[3], hb[3], b1.x, b1.y);
                }
                y0 = fmaf(fa[u], d[0], y0);
                y1 = fmaf(fb[u], d[2], y1);
            }
        }
    }
}

// fp16-weight tile core (router gate, tied lm_head).  One warp, 16 rows,
// k-blocks of 32 (kb = 32*i for i in [ibeg, iend) step istep).  x is in natural
// order (fp16, shared memory).  Lane quad c loads 16 bytes = halves
// [kb+8c, kb+8c+8) of rows g and g+8; the mma slot order equals x's order.
template <int UNROLL>
__device__ __forceinline__ void f16_tile_dot(const __half* __restrict__ W, int N, int K, int row0,
                                             int ibeg, int iend, int istep,
                                             const __half* __restrict__ xs, float& y0, float& y1) {
    const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int ra = min(row0 + g, N - 1), rb = min(row0 + g + 8, N - 1);
    const __half* pa = W + (size_t)ra * K + c * 8;
    const __half* pb = W + (size_t)rb * K + c * 8;
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    for (int i0 = ibeg; i0 < iend; i0 += istep * UNROLL) {
        uint4 wa[UNROLL], wb[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            int i = i0 + u * istep;
            if (i < iend) {
                wa[u] = ldg_stream256(pa + (size_t)i * 32);
                wb[u] = ldg_stream256(pb + (size_t)i * 32);
            }
        }
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            int i = i0 + u * istep;
            if (i < iend) {
                const uint2* xv = reinterpret_cast<const uint2*>(xs + i * 32 + c * 8);
                uint2 b0 = xv[0], b1 = xv[1];
                mma_16816(d, wa[u].x, wb[u].x, wa[u].y, wb[u].y, b0.x, b0.y);
                mma_16816(d, wa[u].z, wb[u].z, wa[u].w, wb[u].w, b1.x, b1.y);
            }
        }
    }
    y0 += d[0];
    y1 += d[2];
}

// ---------------------------------------------------------------------------
// reductions
// ---------------------------------------------------------------------------
// RoPE angle of rotation pair d at position pos (rope, engine.cu:161-182):
// inv_freq = theta^(-2d/64), in float as the reference computes it.
__device__ __forceinline__ void rope_pair_angle(int pos, int d, float theta, float& cs, float& sn) {
    float invf = powf(theta, -(float)(2 * d) / (float)CUINF_HD);
    float ang = (float)pos * invf;
    cs = cosf(ang);
    sn = sinf(ang);
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum of one float per thread; red must hold blockDim.x/32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < nw; i++) t += red[i];
    return t;
}

// RMSNorm of an fp16 row held in shared memory (rmsnorm, engine.cu:131-144):
// out[i] = half(x[i] * rsqrt(mean(x^2) + eps) * w[i]).
__device__ __forceinline__ void rmsnorm_smem(const __half* x, const __half* __restrict__ w,
                                             __half* out, int D, float eps, float* red) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        float v = __half2float(x[i]);
        ss += v * v;
    }
    ss = block_sum(ss, red);
    float inv = rsqrtf(ss / (float)D + eps);
    for (int i = threadIdx.x; i < D; i += blockDim.x)
        out[i] = __float2half_rn(__half2float(x[i]) * inv * __half2float(w[i]));
}

__device__ __forceinline__ unsigned long long umax64_dev(unsigned long long a,
                                                        unsigned long long b) {
    return a > b ? a : b;
}

// Order-preserving key for (value, index) argmax that reproduces argmax_kernel
// (engine.cu:562-572, 256 threads, tree reduction keeping the lower slot on
// ties).  Each thread keeps its first maximum (lowest index of its residue
// i mod 256); two equal values from residues a and b meet at the lowest bit
// where a and b differ and the one with a 0 there survives, i.e. the winner
// has the smallest bit-reversed residue.  Larger key wins.
__device__ __forceinline__ uint32_t brev8(uint32_t r) { return __brev(r) >> 24; }
__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    uint32_t tie = (brev8((uint32_t)i & 255u) << 23) | ((uint32_t)i >> 8);
    return ((unsigned long long)b << 32) | (0xFFFFFFFFu - tie);
}
__device__ __forceinline__ int argmax_key_index(unsigned long long key) {
    uint32_t tie = 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFu);
    return (int)(((tie & 0x7FFFFFu) << 8) | brev8(tie >> 23));
}
