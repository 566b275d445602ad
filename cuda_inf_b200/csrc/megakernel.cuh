// Persistent decode megakernel: one cooperative launch runs a whole decode
// step (all 24 layers + lm_head + argmax) with one CTA per SM.
//
// Why: at batch 1 the step is ~100 dependent GEMV stages of 0.1-15 MB each.
// As separate kernels every stage pays launch, ramp-up and tail (ncu showed
// SMs active only ~40-50% of each kernel's duration).  Here the stages are
// separated by a grid barrier only, and the weights never wait for them:
//
//   warp 12 (producer, one lane) walks this CTA's work items of every stage
//     in order and streams each item's weight slab (INT4 tiles, the router
//     gate, lm_head rows) into a shared-memory ring with TMA bulk copies,
//     one mbarrier per slab.  It runs ahead across stage boundaries, limited
//     only by ring space; expert slabs wait for this CTA's routing result.
//   warps 0-11 (consumers) run the stage program: wait for the previous
//     stage on the grid barrier, build the stage's input vector (RMSNorm of
//     the residual, permuted to mma B-fragment order), then for each item
//     wait its slab, dequantize + mma.m16n8k16, and run the fused epilogue.
//
// Work item j of a stage belongs to CTA j mod gridDim.  Every wait is
// bounded; a time-out raises the abort word and all CTAs leave.
#pragma once
#include "attn.cuh"
#include "common.cuh"
#include "route.cuh"

#ifndef MK_CW
#define MK_CW 12                  // consumer warps
#endif
#define MK_CT (MK_CW * 32)        // consumer threads
#define MK_THREADS (MK_CT + 32)   // + producer warp (one lane issues TMA)
#define MK_QN 32                  // slabs in flight (one mbarrier each)
#define MK_MAXPC 10               // TMA pieces per slab
#define MK_TRACE_W 16             // trace words per (stage, CTA)

enum MkKind : int {
    MK_CONV_IN = 0,  // in_proj (B|C|x) + short conv epilogue
    MK_RES,          // residual GEMV: h += W . act (out_proj, dense w2)
    MK_QKV,          // q/k/v tiles; last tile of a head runs qk-norm/rope/KV append
    MK_ATTN,         // flash-decoding over the FP8 cache + fp16 tail
    MK_DENSE_UP,     // w1/w3 + SwiGLU
    MK_MOE_UP,       // router (gate slab) + selection, expert w1/w3 + SwiGLU
    MK_MOE_DOWN,     // expert w2, fp16 weighted accumulate, residual
    MK_LMHEAD        // final norm, tied lm_head, argmax, next-token bookkeeping
};

struct MkLayer {
    const __half *op_norm, *ffn_norm;
    const uint8_t *wq, *wk, *wv;
    const __half *sq, *sk, *sv, *q_ln, *k_ln;
    uint8_t *kc8, *vc8;
    __half *ksc, *vsc, *ktail, *vtail;
    const uint8_t* win;
    const __half *sin, *conv_w;
    __half* conv_state;
    const uint8_t *w1, *w3;
    const __half *s1, *s3, *gate, *ebias;
    const void* const* experts;  // [E][6]
    int* route_idx;
    float* route_w;
};

struct MkStage {
    int kind, layer, n_items, K;
    const uint8_t* wres;  // MK_RES weights [N=H, K]
    const __half* sres;
    const __half* act;    // MK_RES input vector [K]
};

struct MkParams {
    const MkLayer* L;
    const MkStage* S;
    int n_stages;
    int H, nh, nkv, I, E, topk, V;
    int ring_bytes, xbn, attn_chunks;
    float eps, theta, scale;
    __half *h, *q, *attn_out, *conv_y, *mid, *hidden_out;
    float *qkv_f32, *attn_part, *logits;
    unsigned *qkv_tick, *attn_tick, *lm_tick, *gbar, *abort_flag, *err;
    unsigned long long* am_key;
    const __half *embed, *emb_norm;
    int *tok, *pos, *out_ring;
    int ring;
    // optional [n_stages][G][MK_TRACE_W]: %globaltimer at start, prologue end
    // and end (words 0, 1, 3), SM cycles spent in slab waits (2), then SM cycles
    // since the stage start (%clock64): pre-slab ready (4), first item slab
    // ready (5), dot done (6), epilogue done (7), MoE-up norm done (8),
    // router dots done (9), selection done (10); word 11 = %clock64 at start;
    // producer %clock64 at: pre-slab issue (12), first item slab ready to
    // place (13, after any routing wait), first item slab issue (14); SM
    // cycles from the stage start to the prologue end (15)
    unsigned long long* trace;
};

// Shared-memory carve-up (identical on host and device).
struct MkSmemLayout {
    size_t ring, xs, xB, red, out, lg, total;
};
__host__ __device__ inline MkSmemLayout mk_layout(int H, int xbn, int ring_bytes, int gqa) {
    MkSmemLayout L;
    L.ring = 0;
    L.xs = (size_t)ring_bytes;
    L.xB = L.xs + (size_t)H * 2;
    L.red = L.xB + (size_t)xbn * 2;
    size_t red_bytes = (size_t)MK_CW * 4 * 16 * 4;
    // the attention merge ([MK_CW][gqa][68] floats) reuses xs..red
    size_t merge = (size_t)MK_CW * gqa * ATTN_PART_STRIDE * 4;
    size_t span = (L.red + red_bytes) - L.xs;
    if (merge > span) red_bytes += merge - span;
    L.out = L.red + red_bytes;
    L.lg = L.out + 64 * 4;
    L.total = L.lg + 256 * 4;
    return L;
}

struct MkHeader {
    uint64_t full[MK_QN];
    unsigned meta_off[MK_QN], meta_end[MK_QN];
    volatile unsigned tail;      // ring bytes freed by the consumers (monotonic)
    volatile unsigned consumed;  // slabs consumed
    volatile int route_stage;    // stage whose routing is in sidx/sw
    volatile int stop;           // producer must stop (abort)
    int sidx[16];
    float sw[16];
    int flag;                    // consumer-broadcast scratch
    unsigned long long kred[16];
    unsigned long long wait_cyc;  // trace: SM cycles thread 0 spent waiting for slabs
};

__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;\n" ::"n"(MK_CT) : "memory"); }

// Sum over the consumer threads; red needs MK_CW floats.  Ends with all
// consumers holding the total; the caller separates reuses of red by cbar().
__device__ __forceinline__ float cblock_sum(float v, float* red) {
    v = warp_sum(v);
    cbar();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    cbar();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < MK_CW; i++) t += red[i];
    return t;
}
__device__ __forceinline__ float cblock_max(float v, float* red) {
    v = warp_max(v);
    cbar();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    cbar();
    float t = red[0];
#pragma unroll
    for (int i = 1; i < MK_CW; i++) t = fmaxf(t, red[i]);
    return t;
}

// First failure of a launch: err[0] |= code, err[2..4] = stage, CTA, slab.
__device__ __forceinline__ void mk_fail(const MkParams& P, unsigned code, int stage, unsigned slab) {
    atomicOr(P.abort_flag, 1u);
    if (atomicOr(P.err, code) == 0u) {
        P.err[2] = (unsigned)stage;
        P.err[3] = blockIdx.x;
        P.err[4] = slab;
    }
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned ld_volatile_u32(const unsigned* p) {
    return *reinterpret_cast<const volatile unsigned*>(p);
}

// ---------------------------------------------------------------------------
// stage bookkeeping shared by producer and consumers
// ---------------------------------------------------------------------------
__device__ __forceinline__ int mk_attn_units(int pos) {
    const int total = pos + 1, committed = (total / CUINF_KVGROUP) * CUINF_KVGROUP;
    return committed / CUINF_KVGROUP + (total > committed ? 1 : 0);
}
__device__ __forceinline__ int mk_attn_nchunk(const MkParams& P, int pos) {
    return max(1, min(mk_attn_units(pos), P.attn_chunks));
}
__device__ __forceinline__ int mk_items(const MkParams& P, const MkStage& st, int pos) {
    if (st.kind == MK_ATTN) return P.nkv * mk_attn_nchunk(P, pos);
    return st.n_items;
}

// TMA pieces of item j of stage st, placed one after another in the slab.
// Piece k copies rows[k] rows of bytes[k] bytes, source rows sstride[k]
// apart, into slab rows dstride[k] apart (rows = 1 for a plain range), and
// occupies span[k] bytes of the slab.  total = ring bytes the slab occupies;
// tx = bytes actually copied.
struct MkPieces {
    const void* src[MK_MAXPC];
    unsigned bytes[MK_MAXPC], rows[MK_MAXPC], sstride[MK_MAXPC], dstride[MK_MAXPC], span[MK_MAXPC];
    int n;
    unsigned total, tx;
};
__device__ __forceinline__ void mk_add_piece(MkPieces& pc, const void* src, unsigned bytes) {
    pc.src[pc.n] = src;
    pc.bytes[pc.n] = bytes;
    pc.rows[pc.n] = 1;
    pc.sstride[pc.n] = pc.dstride[pc.n] = pc.span[pc.n] = bytes;
    pc.n++;
    pc.total += bytes;
    pc.tx += bytes;
}
// fp16 rows of H halves staged with a row pitch of mk_f16_pitch(H) bytes:
// 64 mod 128, so the 16-byte loads of two neighbouring rows by one 8-lane
// phase of a warp fall in different shared-memory banks.
__host__ __device__ __forceinline__ unsigned mk_f16_pitch(int H) { return f16_row_pitch(H); }
__device__ __forceinline__ void mk_add_f16_rows(MkPieces& pc, const __half* src, int rows, int H,
                                                int slab_rows) {
    const unsigned pitch = mk_f16_pitch(H);
    pc.src[pc.n] = src;
    pc.bytes[pc.n] = 2u * (unsigned)H;
    pc.rows[pc.n] = (unsigned)rows;
    pc.sstride[pc.n] = 2u * (unsigned)H;
    pc.dstride[pc.n] = pitch;
    pc.span[pc.n] = (unsigned)slab_rows * pitch;
    pc.n++;
    pc.total += (unsigned)slab_rows * pitch;
    pc.tx += (unsigned)rows * 2u * (unsigned)H;
}
__device__ __forceinline__ void mk_add_tile(MkPieces& pc, const uint8_t* packed, const __half* scales,
                                            int K, int row0) {
    mk_add_piece(pc, packed + (size_t)row0 * (K >> 1), 16u * (unsigned)(K >> 1));
    mk_add_piece(pc, (const uint8_t*)scales + (size_t)row0 * (K >> 6), 16u * (unsigned)(K >> 6));
}
__device__ __forceinline__ void mk_item_pieces(const MkParams& P, const MkStage& st, int j,
                                               const int* sidx, MkPieces& pc) {
    pc.n = 0;
    pc.total = pc.tx = 0;
    const MkLayer& L = P.L[st.layer < 0 ? 0 : st.layer];
    const int H = P.H;
    switch (st.kind) {
        case MK_CONV_IN:
            for (int t = 0; t < 3; t++) mk_add_tile(pc, L.win, L.sin, H, t * H + 16 * j);
            // conv taps [16][3] and the two history rows of the item's channels
            // (written only by this stage, in the previous step)
            mk_add_piece(pc, L.conv_w + (size_t)48 * j, 96u);
            mk_add_piece(pc, L.conv_state + (size_t)16 * j, 32u);
            mk_add_piece(pc, L.conv_state + (size_t)H + 16 * j, 32u);
            break;
        case MK_RES:
            mk_add_tile(pc, st.wres, st.sres, st.K, 16 * j);
            break;
        case MK_QKV: {
            const int hh = j >> 2, r = j & 3;
            if (hh < P.nh) mk_add_tile(pc, L.wq, L.sq, H, hh * 64 + r * 16);
            else if (hh < P.nh + P.nkv) mk_add_tile(pc, L.wk, L.sk, H, (hh - P.nh) * 64 + r * 16);
            else mk_add_tile(pc, L.wv, L.sv, H, (hh - P.nh - P.nkv) * 64 + r * 16);
            if (hh < P.nh + P.nkv)  // q/k-norm weight for whichever tile finishes the head
                mk_add_piece(pc, hh < P.nh ? L.q_ln : L.k_ln, 128u);
            break;
        }
        case MK_DENSE_UP:
            mk_add_tile(pc, L.w1, L.s1, H, 16 * j);
            mk_add_tile(pc, L.w3, L.s3, H, 16 * j);
            break;
        case MK_MOE_UP: {
            const int tiles = P.I / 16, t = j / tiles, row0 = (j % tiles) * 16;
            const void* const* ex = L.experts + (size_t)sidx[t] * 6;
            mk_add_tile(pc, (const uint8_t*)ex[0], (const __half*)ex[1], H, row0);
            mk_add_tile(pc, (const uint8_t*)ex[2], (const __half*)ex[3], H, row0);
            break;
        }
        case MK_MOE_DOWN:
            for (int t = 0; t < P.topk; t++) {
                const void* const* ex = L.experts + (size_t)sidx[t] * 6;
                mk_add_tile(pc, (const uint8_t*)ex[4], (const __half*)ex[5], P.I, 16 * j);
            }
            break;
        case MK_LMHEAD: {
            // the slab spans 16 pitched rows; rows past V are never read
            const int r0 = 16 * j;
            mk_add_f16_rows(pc, P.embed + (size_t)r0 * H, min(16, P.V - r0), H, 16);
            break;
        }
        default:
            break;
    }
}

// Stages whose prologue normalises the residual get a per-CTA "pre-slab" at
// their head: the RMSNorm weight, and for MoE-up also the router gate and the
// expert bias, so no prologue waits on a DRAM miss for a small static vector.
__device__ __forceinline__ bool mk_has_pre(int kind) {
    return kind == MK_CONV_IN || kind == MK_QKV || kind == MK_DENSE_UP || kind == MK_MOE_UP ||
           kind == MK_LMHEAD;
}
__device__ __forceinline__ void mk_pre_pieces(const MkParams& P, const MkStage& st, MkPieces& pc) {
    const MkLayer& L = P.L[st.layer < 0 ? 0 : st.layer];
    pc.n = 0;
    pc.total = pc.tx = 0;
    mk_add_piece(pc, st.kind == MK_LMHEAD ? P.emb_norm
                     : (st.kind == MK_CONV_IN || st.kind == MK_QKV) ? L.op_norm : L.ffn_norm,
                 2u * (unsigned)P.H);
    if (st.kind == MK_MOE_UP) mk_add_piece(pc, L.ebias, 2u * (unsigned)P.E);  // norm [H] | bias [E]
}

// ---------------------------------------------------------------------------
// producer
// ---------------------------------------------------------------------------
__device__ __noinline__ void mk_producer(const MkParams& P, MkHeader& S, uint8_t* ring, int pos) {
    const int G = gridDim.x, b = blockIdx.x;
    const unsigned RING = (unsigned)P.ring_bytes;
    const uint64_t pol_ef = l2_policy_evict_first();
    unsigned head = 0, nslab = 0;
    bool ok = true;
    for (int s = 0; s < P.n_stages && ok; s++) {
        const MkStage st = P.S[s];
        if (st.kind == MK_ATTN) continue;
        const int n = mk_items(P, st, pos);
        const bool moe = st.kind == MK_MOE_UP || st.kind == MK_MOE_DOWN;
        for (int j = (mk_has_pre(st.kind) ? -1 : b); j < n && ok; j = (j < 0 ? b : j + G)) {
            MkPieces pc;
            if (j < 0) {
                mk_pre_pieces(P, st, pc);
                const MkLayer& L = P.L[st.layer < 0 ? 0 : st.layer];
                if ((st.kind == MK_CONV_IN || st.kind == MK_QKV) && L.gate) {
                    // pull this layer's router gate into L2 ahead of its MoE
                    // stage, each CTA one slice
                    const unsigned gbytes = 2u * (unsigned)(P.E * P.H);
                    const unsigned chunk = ((gbytes + G - 1) / G + 15u) & ~15u;
                    const unsigned o = (unsigned)b * chunk;
                    if (o < gbytes) prefetch_l2_bulk(reinterpret_cast<const char*>(L.gate) + o, min(chunk, gbytes - o));
                }
            } else {
                if (moe) {  // expert slabs need this CTA's routing of this layer
                    const int want = st.kind == MK_MOE_UP ? s : s - 1;
                    const uint64_t t0 = globaltimer_ns();
                    for (unsigned it = 1; S.route_stage != want; it++) {
                        if ((it & 15) == 0) {  // the clock and the stop word every 16th poll
                            if (S.stop) { ok = false; break; }
                            if (globaltimer_ns() - t0 > CUINF_WAIT_LIMIT_NS) {
                                mk_fail(P, 8u, s, nslab);
                                ok = false;
                                break;
                            }
                        }
                    }
                    if (!ok) break;
                    __threadfence_block();
                }
                mk_item_pieces(P, st, j, S.sidx, pc);
            }
            unsigned long long* ptrace = (P.trace && j <= b) ? P.trace + ((size_t)s * G + b) * MK_TRACE_W : nullptr;
            if (ptrace && j >= 0) ptrace[13] = clock64();
            // Place the slab contiguously; if it does not fit before the end of
            // the ring it starts at offset 0 (the skipped bytes stay unused).
            // It may be written once the bytes it overwrites were consumed:
            // those are the previous lap's [head+total-RING, ...), but never
            // more than what was allocated before it (h0).
            const unsigned h0 = head;
            unsigned off = head % RING;
            if (off + pc.total > RING) { head += RING - off; off = 0; }
            const unsigned need = head + pc.total <= RING ? 0u : min(head + pc.total - RING, h0);
            // wait for ring space and a free mbarrier
            const uint64_t t0 = globaltimer_ns();
            for (unsigned it = 1; (int)(S.tail - need) < 0 || nslab - S.consumed >= MK_QN; it++) {
                if ((it & 15) == 0) {
                    if (S.stop) { ok = false; break; }
                    if (globaltimer_ns() - t0 > CUINF_WAIT_LIMIT_NS) {
                        mk_fail(P, 4u, s, nslab);
                        ok = false;
                        break;
                    }
                }
            }
            if (!ok) break;
            const unsigned q = nslab % MK_QN;
            S.meta_off[q] = off;
            S.meta_end[q] = head + pc.total;
            mbar_arrive_expect_tx(&S.full[q], pc.tx);
            unsigned doff = off;
            // bulk copies of at most 32 KB each; item slabs (weights read once
            // per step) are evict-first in L2, pre-slabs (norm weights and the
            // router gate, read by every CTA) keep the default policy
            for (int k = 0; k < pc.n; k++) {
                for (unsigned r = 0; r < pc.rows[k]; r++) {
                    const uint8_t* src = (const uint8_t*)pc.src[k] + (size_t)r * pc.sstride[k];
                    uint8_t* dst = ring + doff + r * pc.dstride[k];
                    for (unsigned done = 0; done < pc.bytes[k];) {
                        const unsigned len = min(pc.bytes[k] - done, 32768u);
                        if (j >= 0) tma_load_1d_hint(dst + done, src + done, len, &S.full[q], pol_ef);
                        else tma_load_1d(dst + done, src + done, len, &S.full[q]);
                        done += len;
                    }
                }
                doff += pc.span[k];
            }
            if (ptrace) ptrace[j < 0 ? 12 : 14] = clock64();
            head += pc.total;
            nslab++;
        }
    }
    if (!ok) atomicOr(P.abort_flag, 1u);
    // leave no copy in flight into this CTA's shared memory
    for (unsigned k = S.consumed; k < nslab; k++) {
        const unsigned q = k % MK_QN;
        mbar_wait_bounded(&S.full[q], (k / MK_QN) & 1, nullptr);
    }
}

// ---------------------------------------------------------------------------
// consumer helpers
// ---------------------------------------------------------------------------
// Wait for this CTA's next slab; returns its address (nullptr on time-out).
__device__ __forceinline__ const uint8_t* mk_slab_wait(const MkParams& P, MkHeader& S, uint8_t* ring,
                                                       unsigned slabno, int stage) {
    const unsigned q = slabno % MK_QN;
    const long long tw = (P.trace && threadIdx.x == 0) ? clock64() : 0ll;
    if (!mbar_wait_bounded(&S.full[q], (slabno / MK_QN) & 1, nullptr)) {
        mk_fail(P, 16u, stage, slabno);
        S.stop = 1;
    }
    if (P.trace && threadIdx.x == 0) S.wait_cyc += (unsigned long long)(clock64() - tw);
    cbar();  // a time-out in any consumer stops all of them (and the producer)
    return S.stop ? nullptr : ring + S.meta_off[q];
}
// All consumers are done with slab slabno: hand its space back.
__device__ __forceinline__ void mk_slab_free(MkHeader& S, unsigned slabno) {
    cbar();
    if (threadIdx.x == 0) {
        S.tail = S.meta_end[slabno % MK_QN];
        S.consumed = slabno + 1;
    }
}

// Grid barrier: stage s may start once all CTAs finished stage s-1.
__device__ __forceinline__ bool mk_grid_wait(const MkParams& P, MkHeader& S, unsigned target) {
    if (threadIdx.x == 0) {
        int ok = 1;
        uint64_t t0 = 0;
        // tight acquire polls of the counter; the abort word and the clock are
        // checked every 16th poll (each poll is an L2 round trip)
        for (unsigned it = 1; ld_acquire_u32(P.gbar) < target; it++) {
            if ((it & 15) == 0) {
                if (ld_volatile_u32(P.abort_flag)) { ok = 0; break; }
                const uint64_t now = globaltimer_ns();
                if (!t0) t0 = now;
                else if (now - t0 > CUINF_WAIT_LIMIT_NS) {
                    mk_fail(P, 2u, (int)(target / gridDim.x), 0u);
                    ok = 0;
                    break;
                }
            }
        }
        S.flag = ok;
    }
    cbar();
    return S.flag != 0;
}
// Arrival: the consumer barrier orders every consumer's writes before thread
// 0's release-add (bar.sync is cumulative), so a CTA that acquires the count
// sees them.
__device__ __forceinline__ void mk_grid_arrive(const MkParams& P) {
    cbar();
    if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;\n" ::"l"(P.gbar) : "memory");
}

// Data that other CTAs write during the launch (the residual, activation
// vectors, q, the KV tail, attention partials) is read with ld.global.cg: the
// SM's L1 is not coherent with other SMs' stores, and a line cached by an
// earlier stage of the same launch would be stale.

// x = rmsnorm(src) into xs (fp16) and, when xB != null, its B-fragment order
// (rmsnorm, engine.cu:131-144: half(x * rsqrt(mean(x^2) + eps) * w)).  Each
// thread owns 8 consecutive elements (H % 8 == 0, H <= 16 * MK_CT), which are
// exactly the two B-fragment entries m = 2j, 2j+1 of quad c of their group, so
// the whole norm takes one load of src and two consumer barriers.  red[0..11]
// must not be read by anyone after the caller's last barrier.
__device__ __noinline__ void mk_norm(const __half* src, const __half* w, int H, float eps,
                                     __half* xs, __half* xB, float* red) {
    const int tid = threadIdx.x;
    const int n8 = H >> 3;
    uint4 v[2];
    float ss = 0.f;
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const int i = tid + r * MK_CT;
        if (i < n8) {
            v[r] = __ldcg(reinterpret_cast<const uint4*>(src + 8 * i));
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
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    cbar();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < MK_CW; i++) tot += red[i];
    const float inv = rsqrtf(tot / (float)H + eps);
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const int i = tid + r * MK_CT;
        if (i < n8) {
            const uint4 wv = *reinterpret_cast<const uint4*>(w + 8 * i);
            const __half* xh = reinterpret_cast<const __half*>(&v[r]);
            const __half* wh = reinterpret_cast<const __half*>(&wv);
            __align__(16) __half o[8];
#pragma unroll
            for (int q = 0; q < 8; q++) o[q] = __float2half_rn(__half2float(xh[q]) * inv * __half2float(wh[q]));
            *reinterpret_cast<uint4*>(xs + 8 * i) = *reinterpret_cast<const uint4*>(o);
            if (xB) {
                // k0 = 8i = 128G + 32c + 8j: entries (G, 2j, c) and (G, 2j+1, c)
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
    cbar();
}

// xB = B-fragment order of the fp16 vector src[K] (K % 128 == 0), eight
// elements per thread; ends with a consumer barrier.
__device__ __noinline__ void mk_build_xB(const __half* src, int K, __half* xB) {
    for (int i = threadIdx.x; i < (K >> 3); i += MK_CT) {
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(src + 8 * i));
        const __half* o = reinterpret_cast<const __half*>(&v);
        const int G = i >> 4, c = (i >> 2) & 3, j = i & 3;
        __half2* e0 = reinterpret_cast<__half2*>(xB + (size_t)((G * 8 + 2 * j) * 4 + c) * 4);
        __half2* e1 = reinterpret_cast<__half2*>(xB + (size_t)((G * 8 + 2 * j + 1) * 4 + c) * 4);
        e0[0] = __halves2half2(o[0], o[4]);
        e0[1] = __halves2half2(o[1], o[5]);
        e1[0] = __halves2half2(o[2], o[6]);
        e1[1] = __halves2half2(o[3], o[7]);
    }
    cbar();
}

// T INT4 tiles (K wide, consecutive in the slab) times x (B-fragment order,
// tile t uses xB + t*xstride): out[t*16 + r] = row r of tile t.
__device__ __noinline__ void mk_dot_tiles(const uint8_t* slab, int T, int K, const __half* xB,
                                             int xstride, float* red, float* out) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KG = K >> 7;
    const uint32_t TB = int4_tile_bytes(K);
    float y0[4] = {0.f, 0.f, 0.f, 0.f}, y1[4] = {0.f, 0.f, 0.f, 0.f};
    for (int p = warp; p < T * KG; p += MK_CW) {
        const int t = p / KG, G = p - t * KG;
        float a = 0.f, c = 0.f;
        int4_tile_dot_smem<1>(slab + t * TB, K, G, G + 1, 1,
                              reinterpret_cast<const uint2*>(xB + (size_t)t * xstride), a, c);
#pragma unroll
        for (int i = 0; i < 4; i++)
            if (i == t) { y0[i] += a; y1[i] += c; }
    }
    if ((lane & 3) == 0) {
#pragma unroll
        for (int t = 0; t < 4; t++)
            if (t < T) {
                red[(warp * 4 + t) * 16 + (lane >> 2)] = y0[t];
                red[(warp * 4 + t) * 16 + (lane >> 2) + 8] = y1[t];
            }
    }
    cbar();
    for (int i = threadIdx.x; i < T * 16; i += MK_CT) {
        const int t = i >> 4, r = i & 15;
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < MK_CW; w++) s += red[(w * 4 + t) * 16 + r];
        out[i] = s;
    }
    cbar();
}

// T tiles of 16 fp16 rows (H halves each, rows mk_f16_pitch(H) bytes apart,
// tiles consecutive) times x (fp16, natural order): out[t*16 + r].  The
// 32-wide k blocks of each tile are spread over the consumer warps; a block is
// two mma.m16n8k16 whose A slots follow the 16-byte row chunk a lane loads,
// with x read in the same order.  T <= 4.
__device__ __noinline__ void mk_dot_f16_tiles(const uint8_t* slab, int T, int H, const __half* xs, float* red,
                                              float* out) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const unsigned pitch = mk_f16_pitch(H);
    const int KB = H >> 5;
    for (int t = 0; t < T; t++) {
        float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
        const uint8_t* tb = slab + (size_t)t * 16 * pitch + c * 16;
        for (int i = warp; i < KB; i += MK_CW) {
            const uint4 wa = *reinterpret_cast<const uint4*>(tb + g * pitch + i * 64);
            const uint4 wb = *reinterpret_cast<const uint4*>(tb + (g + 8) * pitch + i * 64);
            const uint2* xv = reinterpret_cast<const uint2*>(xs + i * 32 + c * 8);
            const uint2 b0 = xv[0], b1 = xv[1];
            mma_16816(d0, wa.x, wb.x, wa.y, wb.y, b0.x, b0.y);
            mma_16816(d1, wa.z, wb.z, wa.w, wb.w, b1.x, b1.y);
        }
        if (c == 0) {
            red[(warp * 4 + t) * 16 + g] = d0[0] + d1[0];
            red[(warp * 4 + t) * 16 + g + 8] = d0[2] + d1[2];
        }
    }
    cbar();
    for (int i = threadIdx.x; i < T * 16; i += MK_CT) {
        const int t = i >> 4, r = i & 15;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < MK_CW; w++) sum += red[(w * 4 + t) * 16 + r];
        out[i] = sum;
    }
    cbar();
}

// Router logits lg[e] = gate[e,:] . xs (gate fp16 [E][H] in global memory, E
// % 8 == 0).  The gate is read straight from L2: it is small, every CTA reads
// it, and it is fetched with the default L2 policy while the streamed weights
// are evict-first, so it stays resident across steps.  Units are (16-expert
// tile, 32-wide k block) pairs; rows past E are clamped and discarded.
__device__ __noinline__ void mk_router_l2(const __half* gate, int E, int H, const __half* xs, float* red,
                                          float* lg) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int KB = H >> 5, T = (E + 15) >> 4;
    for (int t = 0; t < T; t++) {
        const int ra = min(16 * t + g, E - 1), rb = min(16 * t + g + 8, E - 1);
        const __half* pa = gate + (size_t)ra * H + c * 8;
        const __half* pb = gate + (size_t)rb * H + c * 8;
        float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
        int i = warp;
        for (; i + 3 * MK_CW < KB; i += 4 * MK_CW) {  // four k blocks in flight
            uint4 wa[4], wb[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                wa[u] = __ldcg(reinterpret_cast<const uint4*>(pa + (i + u * MK_CW) * 32));
                wb[u] = __ldcg(reinterpret_cast<const uint4*>(pb + (i + u * MK_CW) * 32));
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const uint2* xv = reinterpret_cast<const uint2*>(xs + (i + u * MK_CW) * 32 + c * 8);
                const uint2 b0 = xv[0], b1 = xv[1];
                mma_16816(d0, wa[u].x, wb[u].x, wa[u].y, wb[u].y, b0.x, b0.y);
                mma_16816(d1, wa[u].z, wb[u].z, wa[u].w, wb[u].w, b1.x, b1.y);
            }
        }
        for (; i < KB; i += MK_CW) {
            const uint4 wa = __ldcg(reinterpret_cast<const uint4*>(pa + i * 32));
            const uint4 wb = __ldcg(reinterpret_cast<const uint4*>(pb + i * 32));
            const uint2* xv = reinterpret_cast<const uint2*>(xs + i * 32 + c * 8);
            const uint2 b0 = xv[0], b1 = xv[1];
            mma_16816(d0, wa.x, wb.x, wa.y, wb.y, b0.x, b0.y);
            mma_16816(d1, wa.z, wb.z, wa.w, wb.w, b1.x, b1.y);
        }
        if (c == 0) {
            red[(warp * 4 + t) * 16 + g] = d0[0] + d1[0];
            red[(warp * 4 + t) * 16 + g + 8] = d0[2] + d1[2];
        }
    }
    cbar();
    for (int i = threadIdx.x; i < T * 16; i += MK_CT) {
        const int t = i >> 4, r = i & 15;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < MK_CW; w++) sum += red[(w * 4 + t) * 16 + r];
        lg[i] = sum;
    }
    cbar();
}

// Expert selection of the reference's host loop (engine.cu:883-892) by rank:
// expert e is picked in slot rank(e) = #{e' : s' > s, or s' == s and e' < e}
// when that rank is below topk, which is the order of the reference's repeated
// strict-'>' scan.  Scores that are NaN or <= -1e30 rank last (by index), as
// the scan never picks them before the smallest unused index.  Weights are
// the unbiased sigmoids of the picks over (their sum in slot order + 1e-6).
// All consumer threads call it; E <= MK_CT; scratch: 2*E floats.
__device__ __noinline__ void mk_route_select(const float* lg, const __half* bias, int E, int topk, int* idx,
                                             float* w, float* scratch) {
    const int e = threadIdx.x;
    float* sc = scratch;
    float* sg = scratch + E;
    float sig = 0.f, key = -INFINITY;
    if (e < E) {
        sig = route_sigmoid_call(lg[e]);
        const float score = sig + __half2float(bias[e]);
        key = (score > -1e30f) ? score : -INFINITY;  // NaN compares false
        sc[e] = key;
    }
    cbar();
    if (e < E) {
        int rank = 0;
        for (int o = 0; o < E; o++) {
            const float ko = sc[o];
            rank += (ko > key || (ko == key && o < e)) ? 1 : 0;
        }
        if (rank < topk) {
            idx[rank] = e;
            sg[rank] = sig;
        }
    }
    cbar();
    if (e == 0) {
        float wsum = 0.f;
        for (int t = 0; t < topk; t++) wsum += sg[t];
        for (int t = 0; t < topk; t++) w[t] = sg[t] / (wsum + 1e-6f);
    }
    cbar();
}

// QK-RMSNorm + RoPE + KV append (+ FP8 commit) of one head's 64 values
// (engine.cu:792-845), run by the consumers of the CTA that finished the
// head's last tile.  lw: the head's q/k-norm weight (shared memory, unused
// for v heads); hv: 64 halves of scratch.
__device__ __noinline__ void mk_qkv_head(const MkParams& P, const MkLayer& L, int hh, const float* vals,
                                         const __half* lw, __half* hv, float* red, int pos) {
    const int d = threadIdx.x;
    const int committed = (pos / CUINF_KVGROUP) * CUINF_KVGROUP, slot = pos - committed;
    const bool is_q = hh < P.nh, is_k = !is_q && hh < P.nh + P.nkv;
    if (d < 64) hv[d] = __float2half_rn(vals[d]);
    cbar();
    if (is_q || is_k) {
        const float v = d < 64 ? __half2float(hv[d]) : 0.f;
        const float ss = cblock_sum(v * v, red);
        const float inv = rsqrtf(ss / 64.f + P.eps);
        const __half nv = __float2half_rn(v * inv * __half2float(lw[d < 64 ? d : 0]));
        cbar();
        if (d < 64) hv[d] = nv;
        cbar();
        if (d < 32) {
            const float invf = powf(P.theta, -(float)(2 * d) / (float)CUINF_HD);
            const float ang = (float)pos * invf;
            const float cs = cosf(ang), sn = sinf(ang);
            const float x0 = __half2float(hv[d]), x1 = __half2float(hv[d + 32]);
            const __half o0 = __float2half_rn(x0 * cs - x1 * sn);
            const __half o1 = __float2half_rn(x1 * cs + x0 * sn);
            hv[d] = o0;
            hv[d + 32] = o1;
        }
        cbar();
    }
    if (is_q) {
        if (d < 64) P.q[(size_t)hh * CUINF_HD + d] = hv[d];
        return;
    }
    const int kvh = is_k ? hh - P.nh : hh - P.nh - P.nkv;
    __half* tail = is_k ? L.ktail : L.vtail;
    if (d < 64) tail[((size_t)slot * P.nkv + kvh) * CUINF_HD + d] = hv[d];
    if (slot != CUINF_KVGROUP - 1) return;
    // kv_commit_group for this head (engine.cu:202-228)
    cbar();
    uint8_t* c8 = is_k ? L.kc8 : L.vc8;
    __half* sc = is_k ? L.ksc : L.vsc;
    float mx = 0.f;
    for (int e = d; e < CUINF_KVGROUP * CUINF_HD; e += MK_CT) {
        const int t = e >> 6, dd = e & 63;
        mx = fmaxf(mx, fabsf(__half2float(tail[((size_t)t * P.nkv + kvh) * CUINF_HD + dd])));
    }
    const float amax = cblock_max(mx, red);
    const float s = amax / 448.0f + 1e-12f;
    if (d == 0) sc[(committed / CUINF_KVGROUP) * P.nkv + kvh] = __float2half_rn(s);
    for (int e = d; e < CUINF_KVGROUP * CUINF_HD; e += MK_CT) {
        const int t = e >> 6, dd = e & 63;
        const float v = __half2float(tail[((size_t)t * P.nkv + kvh) * CUINF_HD + dd]);
        c8[((size_t)(committed + t) * P.nkv + kvh) * CUINF_HD + dd] =
            (uint8_t)__nv_cvt_float_to_fp8(v / s, __NV_SATFINITE, __NV_E4M3);
    }
}

// One attention item: kv head h, chunk ch of the units; partials to global,
// the last chunk of a head merges all chunks into attn_out.
__device__ __noinline__ void mk_attn_item(const MkParams& P, const MkLayer& L, int j, int pos,
                                          float* merge, int* flag) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int nkv = P.nkv, gqa = P.nh / P.nkv;
    const int h = j % nkv, ch = j / nkv;
    const int total = pos + 1, committed = (total / CUINF_KVGROUP) * CUINF_KVGROUP;
    const int tail_len = total - committed, n_fp8 = committed / CUINF_KVGROUP;
    const int nunits = mk_attn_units(pos), nchunk = mk_attn_nchunk(P, pos);
    const int upc = (nunits + nchunk - 1) / nchunk;
    const int u0 = ch * upc, u1 = min(u0 + upc, nunits);
    const float kfac = P.scale * 1.4426950408889634f;
    uint32_t aq[4][2];
    {
        const bool real = g < gqa;
        const __half* qh = P.q + (size_t)(h * gqa + (real ? g : 0)) * CUINF_HD + 16 * c;
#pragma unroll
        for (int s = 0; s < 4; s++) {
            const uint32_t lo = __ldcg(reinterpret_cast<const unsigned int*>(qh + 4 * s));
            const uint32_t hi = __ldcg(reinterpret_cast<const unsigned int*>(qh + 4 * s + 2));
            aq[s][0] = real ? lo : 0u;
            aq[s][1] = real ? hi : 0u;
        }
    }
    float m_run = ATTN_NEG, l_run = 0.f, O[8][4];
#pragma unroll
    for (int t = 0; t < 8; t++) O[t][0] = O[t][1] = O[t][2] = O[t][3] = 0.f;
    attn_warp_units<true, 1>(L.kc8, L.vc8, L.ksc, L.vsc, L.ktail, L.vtail, nkv, h, n_fp8, tail_len, kfac, aq,
                    u0 + warp, u1, MK_CW, m_run, l_run, O);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    if (g < gqa) {
        float* row = merge + ((size_t)warp * gqa + g) * ATTN_PART_STRIDE;
        if (c == 0) { row[0] = m_run; row[1] = l_run; }
#pragma unroll
        for (int t = 0; t < 8; t++) {
            row[4 + 16 * c + t] = O[t][0];
            row[4 + 16 * c + 8 + t] = O[t][1];
        }
    }
    cbar();
    float* part = P.attn_part + ((size_t)(h * P.attn_chunks + ch) * gqa) * ATTN_PART_STRIDE;
    for (int it = threadIdx.x; it < gqa * 64; it += MK_CT) {
        const int r = it >> 6, d = it & 63;
        float mm = ATTN_NEG;
        for (int w = 0; w < MK_CW; w++) mm = fmaxf(mm, merge[((size_t)w * gqa + r) * ATTN_PART_STRIDE]);
        float l = 0.f, o = 0.f;
        for (int w = 0; w < MK_CW; w++) {
            const float* row = merge + ((size_t)w * gqa + r) * ATTN_PART_STRIDE;
            const float e = exp2f(row[0] - mm);
            l += row[1] * e;
            o += row[4 + d] * e;
        }
        float* pr = part + (size_t)r * ATTN_PART_STRIDE;
        pr[4 + d] = o;
        if (d == 0) { pr[0] = mm; pr[1] = l; }
    }
    __threadfence();
    cbar();
    if (threadIdx.x == 0) *flag = atomicAdd(&P.attn_tick[h], 1u) == (unsigned)(nchunk - 1);
    cbar();
    if (!*flag) return;
    __threadfence();
    // merge the chunks: (m, l) of every chunk staged in shared memory first so
    // the output loop has only independent loads
    const float* hp = P.attn_part + (size_t)h * P.attn_chunks * gqa * ATTN_PART_STRIDE;
    float* s_m = merge;                      // [nchunk*gqa]
    float* s_l = merge + P.attn_chunks * gqa;  // [nchunk*gqa]
    float* s_L = s_l + P.attn_chunks * gqa;    // [gqa]
    for (int i = threadIdx.x; i < nchunk * gqa; i += MK_CT) {
        s_m[i] = __ldcg(hp + (size_t)i * ATTN_PART_STRIDE);
        s_l[i] = __ldcg(hp + (size_t)i * ATTN_PART_STRIDE + 1);
    }
    cbar();
    if (threadIdx.x < gqa) {
        const int r = threadIdx.x;
        float gm = ATTN_NEG;
        for (int k = 0; k < nchunk; k++)
            if (s_l[k * gqa + r] > 0.f) gm = fmaxf(gm, s_m[k * gqa + r]);
        float L = 0.f;
        for (int k = 0; k < nchunk; k++) {
            const int i = k * gqa + r;
            const float e = s_l[i] > 0.f ? exp2f(s_m[i] - gm) : 0.f;
            s_m[i] = e;
            L += s_l[i] * e;
        }
        s_L[r] = L;
    }
    cbar();
    for (int it = threadIdx.x; it < gqa * 64; it += MK_CT) {
        const int r = it >> 6, d = it & 63;
        float o = 0.f;
#pragma unroll 6
        for (int k = 0; k < nchunk; k++)
            o += s_m[k * gqa + r] * __ldcg(hp + ((size_t)k * gqa + r) * ATTN_PART_STRIDE + 4 + d);
        P.attn_out[(size_t)(h * gqa + r) * CUINF_HD + d] = __float2half_rn(o / s_L[r]);
    }
    if (threadIdx.x == 0) P.attn_tick[h] = 0u;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(MK_THREADS, 1) k_decode_mk(const __grid_constant__ MkParams P) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ MkHeader S;
    const int G = gridDim.x, b = blockIdx.x;
    const int gqa = P.nh / P.nkv;
    const MkSmemLayout lay = mk_layout(P.H, P.xbn, P.ring_bytes, gqa);
    uint8_t* ring = smem + lay.ring;
    __half* xs = reinterpret_cast<__half*>(smem + lay.xs);
    __half* xB = reinterpret_cast<__half*>(smem + lay.xB);
    float* red = reinterpret_cast<float*>(smem + lay.red);
    float* out = reinterpret_cast<float*>(smem + lay.out);
    float* lg = reinterpret_cast<float*>(smem + lay.lg);
    float* merge = reinterpret_cast<float*>(smem + lay.xs);  // attention only

    if (threadIdx.x == 0) {
        for (int q = 0; q < MK_QN; q++) mbar_init(&S.full[q], 1);
        S.tail = 0;
        S.consumed = 0;
        S.route_stage = -1;
        S.stop = 0;
    }
    __syncthreads();
    const int pos = *P.pos;
    if (threadIdx.x >= MK_CT) {  // producer warp
        if (threadIdx.x == MK_CT) mk_producer(P, S, ring, pos);
        return;
    }

    const int tid = threadIdx.x, H = P.H;
    unsigned slabno = 0;
    unsigned long long best = 0ull;  // lm_head: this thread's best key (tid < 16)
    bool alive = true;
    for (int s = 0; s < P.n_stages && alive; s++) {
        const MkStage st = P.S[s];
        const MkLayer& L = P.L[st.layer < 0 ? 0 : st.layer];
        if (s > 0 && !mk_grid_wait(P, S, (unsigned)s * G)) { alive = false; break; }
        long long clk0 = 0;
        if (P.trace && tid == 0) {
            unsigned long long* tr = P.trace + ((size_t)s * G + b) * MK_TRACE_W;
            tr[0] = globaltimer_ns();
            clk0 = clock64();
            for (int w = 4; w <= 10; w++) tr[w] = 0ull;
            tr[11] = (unsigned long long)clk0;
            S.wait_cyc = 0ull;
        }
        unsigned long long* trs = (P.trace && tid == 0) ? P.trace + ((size_t)s * G + b) * MK_TRACE_W : nullptr;
        // ---- stage prologue ----
        const uint8_t* pre = nullptr;
        if (mk_has_pre(st.kind)) {
            pre = mk_slab_wait(P, S, ring, slabno, s);
            if (!pre) { alive = false; break; }
            if (trs) trs[4] = clock64() - clk0;
        }
        const __half* nw = reinterpret_cast<const __half*>(pre);
        switch (st.kind) {
            case MK_CONV_IN:
            case MK_QKV: {
                const __half* src = P.h;
                if (s == 0) {
                    src = P.embed + (size_t)(*P.tok) * H;
                    if (b == 0)
                        for (int i = tid; i < H; i += MK_CT) P.h[i] = src[i];
                }
                mk_norm(src, nw, H, P.eps, xs, xB, red);
                break;
            }
            case MK_RES:
                mk_build_xB(st.act, st.K, xB);
                break;
            case MK_DENSE_UP:
                mk_norm(P.h, nw, H, P.eps, xs, xB, red);
                break;
            case MK_MOE_UP: {
                mk_norm(P.h, nw, H, P.eps, xs, xB, red);
                if (trs) trs[8] = clock64() - clk0;
                mk_router_l2(L.gate, P.E, H, xs, red, lg);
                if (trs) trs[9] = clock64() - clk0;
                mk_route_select(lg, reinterpret_cast<const __half*>(pre + 2 * H), P.E, P.topk, S.sidx, S.sw,
                                red + MK_CW * 4 * 16 - 2 * P.E);
                if (trs) trs[10] = clock64() - clk0;
                if (tid == 0) {
                    __threadfence_block();
                    S.route_stage = s;
                }
                if (b == 0 && tid < P.topk) {
                    L.route_idx[tid] = S.sidx[tid];
                    L.route_w[tid] = S.sw[tid];
                }
                break;
            }
            case MK_MOE_DOWN:
                mk_build_xB(P.mid, P.topk * P.I, xB);  // the expert slices are consecutive
                break;
            case MK_LMHEAD:
                if (b == 0 && P.hidden_out)
                    for (int i = tid; i < H; i += MK_CT) P.hidden_out[i] = __ldcg(P.h + i);
                mk_norm(P.h, nw, H, P.eps, xs, nullptr, red);
                break;
            default:
                break;
        }
        if (pre) mk_slab_free(S, slabno++);
        if (!alive) break;
        if (trs) {
            trs[1] = globaltimer_ns();
            trs[15] = clock64() - clk0;
        }
        // ---- items ----
        const int n = mk_items(P, st, pos);
        for (int j = b; j < n; j += G) {
            if (st.kind == MK_ATTN) {
                mk_attn_item(P, L, j, pos, merge, &S.flag);
                cbar();
                continue;
            }
            const uint8_t* slab = mk_slab_wait(P, S, ring, slabno, s);
            if (!slab) { alive = false; break; }
            const bool tr_item = trs && j == b;
            unsigned long long* tr = trs;
            if (tr_item) tr[5] = clock64() - clk0;
            // the residual rows this item updates, read before the dot so the
            // load latency hides behind it (only this CTA writes them)
            float hres = 0.f;
            if ((st.kind == MK_RES || st.kind == MK_MOE_DOWN) && tid < 16)
                hres = __half2float(__ldcg(P.h + 16 * j + tid));
            switch (st.kind) {
                case MK_CONV_IN: {
                    mk_dot_tiles(slab, 3, H, xB, 0, red, out);
                    if (tr_item) tr[6] = clock64() - clk0;
                    if (tid < 16) {
                        const int c = 16 * j + tid;
                        const __half* ex = reinterpret_cast<const __half*>(slab + 3 * int4_tile_bytes(H));
                        const __half Cb = __float2half_rn(out[16 + tid]);
                        const __half Bx = __float2half_rn(out[tid] * out[32 + tid]);
                        const __half s1h = ex[64 + tid];
                        const float s0 = __half2float(ex[48 + tid]), s1 = __half2float(s1h);
                        const float w0 = __half2float(ex[tid * 3 + 0]), w1 = __half2float(ex[tid * 3 + 1]),
                                    w2 = __half2float(ex[tid * 3 + 2]);
                        const float co = s0 * w0 + s1 * w1 + __half2float(Bx) * w2;
                        P.conv_y[c] = __float2half_rn(__half2float(Cb) * co);
                        L.conv_state[c] = s1h;
                        L.conv_state[H + c] = Bx;
                    }
                    break;
                }
                case MK_RES: {
                    mk_dot_tiles(slab, 1, st.K, xB, 0, red, out);
                    if (tr_item) tr[6] = clock64() - clk0;
                    if (tid < 16) P.h[16 * j + tid] = __float2half_rn(hres + out[tid]);
                    break;
                }
                case MK_QKV: {
                    mk_dot_tiles(slab, 1, H, xB, 0, red, out);
                    if (tr_item) tr[6] = clock64() - clk0;
                    const int hh = j >> 2;
                    if (tid < 16) P.qkv_f32[16 * j + tid] = out[tid];
                    __threadfence();
                    cbar();
                    if (tid == 0) S.flag = atomicAdd(&P.qkv_tick[hh], 1u) == 3u;
                    cbar();
                    if (S.flag) {
                        __threadfence();
                        if (tid < 64) out[tid] = __ldcg(P.qkv_f32 + 64 * hh + tid);
                        if (tid == 0) P.qkv_tick[hh] = 0u;
                        cbar();
                        mk_qkv_head(P, L, hh, out,
                                    reinterpret_cast<const __half*>(slab + int4_tile_bytes(H)),
                                    reinterpret_cast<__half*>(lg), red, pos);
                    }
                    break;
                }
                case MK_DENSE_UP:
                case MK_MOE_UP: {
                    mk_dot_tiles(slab, 2, H, xB, 0, red, out);
                    if (tr_item) tr[6] = clock64() - clk0;
                    if (tid < 16) {
                        const float gg = out[tid], u = out[16 + tid];
                        const float sv = gg / (1.f + __expf(-gg)) * u;
                        if (st.kind == MK_DENSE_UP) {
                            P.mid[16 * j + tid] = __float2half_rn(sv);
                        } else {
                            const int tiles = P.I / 16, t = j / tiles;
                            P.mid[(size_t)t * P.I + (j % tiles) * 16 + tid] = __float2half_rn(sv);
                        }
                    }
                    break;
                }
                case MK_MOE_DOWN: {
                    mk_dot_tiles(slab, P.topk, P.I, xB, P.I, red, out);
                    if (tr_item) tr[6] = clock64() - clk0;
                    if (tid < 16) {
                        __half acc = __float2half_rn(0.f);
                        for (int t = 0; t < P.topk; t++)
                            acc = __float2half_rn(__half2float(acc) + S.sw[t] * out[t * 16 + tid]);
                        P.h[16 * j + tid] = __float2half_rn(hres + __half2float(acc));
                    }
                    break;
                }
                case MK_LMHEAD: {
                    mk_dot_f16_tiles(slab, 1, H, xs, red, out);
                    if (tr_item) tr[6] = clock64() - clk0;
                    if (tid < 16) {
                        const int r = 16 * j + tid;
                        if (r < P.V) {
                            const float y = out[tid];
                            if (P.logits) P.logits[r] = y;
                            if (y > -1e30f) best = umax64_dev(best, argmax_key(y == 0.f ? 0.f : y, r));
                        }
                    }
                    break;
                }
                default:
                    break;
            }
            if (tr_item) tr[7] = clock64() - clk0;
            mk_slab_free(S, slabno++);
        }
        if (!alive) break;
        if (P.trace) {
            cbar();
            if (tid == 0) {
                P.trace[((size_t)s * G + b) * MK_TRACE_W + 2] = S.wait_cyc;
                P.trace[((size_t)s * G + b) * MK_TRACE_W + 3] = globaltimer_ns();
            }
        }
        if (st.kind != MK_LMHEAD) mk_grid_arrive(P);
    }
    if (!alive) {
        if (tid == 0) S.stop = 1;
        return;
    }
    // ---- argmax across the grid; the last CTA publishes the token ----
    if (tid < 16) S.kred[tid] = best;
    cbar();
    if (tid == 0) {
        unsigned long long bb = 0ull;
        for (int i = 0; i < 16; i++) bb = umax64_dev(bb, S.kred[i]);
        if (bb) atomicMax(P.am_key, bb);
        __threadfence();
        const unsigned prev = atomicAdd(P.lm_tick, 1u);
        if (prev == (unsigned)G - 1) {
            __threadfence();
            const unsigned long long k = atomicExch(P.am_key, 0ull);
            const int token = k ? argmax_key_index(k) : 0;
            *P.tok = token;
            if (P.out_ring) P.out_ring[pos % P.ring] = token;
            *P.pos = pos + 1;
            *P.lm_tick = 0u;
            *P.gbar = 0u;
        }
    }
}
