/*
 * CPU oracle for the quantized decode hot path of g023/cuda_inf.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA library, never part of
 * it.  See oracle.h for the contract.  Each function cites the reference code
 * (src/engine.cu, tools/export_weights.py, tools/make_index.py) it restates.
 *
 * Numerics: every point where the reference rounds to fp16 (__float2half) is
 * reproduced exactly (via float first, then RNE to half); fp32 products that
 * are exact in the reference stay exact here; long sums (GEMV dot products,
 * RMSNorm sum of squares, softmax) accumulate in double, which makes the
 * oracle at least as accurate as the reference's fp32 reductions.  Built with
 * -ffp-contract=off so that no FMA contraction changes a rounding.
 */
#include "oracle.h"

/* ORC_BASELINE builds the same restatement as the timed CPU baseline
 * (oracle/Makefile libcpubase.so: -O3, native ISA, FMA contraction allowed):
 * dot products and softmax sums accumulate in fp32 (eight partial sums per
 * dot product, which the compiler vectorizes), exp in float.  The checker
 * build (liboracle.so) keeps double accumulation and a fixed summation
 * order. */
#ifdef ORC_BASELINE
typedef float orc_acc;
#define ORC_EXP expf
#else
typedef double orc_acc;
#define ORC_EXP exp
#endif

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* scalar conversions                                                         */
/* ------------------------------------------------------------------------ */
float orc_h2f(uint16_t h) {
    _Float16 x;
    memcpy(&x, &h, 2);
    return (float)x;
}

uint16_t orc_f2h(float f) {
    _Float16 x = (_Float16)f; /* IEEE RNE, overflow -> inf, like __float2half */
    uint16_t h;
    memcpy(&h, &x, 2);
    return h;
}

/* E4M3: s eeee mmm, bias 7. exp 0 = subnormal (m * 2^-9); s1111111 = NaN. */
float orc_e4m3_to_f32(uint8_t b) {
    int s = b >> 7, e = (b >> 3) & 15, m = b & 7;
    float v;
    if (e == 15 && m == 7) return NAN;
    if (e == 0) v = ldexpf((float)m, -9);
    else        v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
    return s ? -v : v;
}

/* All 256 E4M3 codes decoded once (the same values as orc_e4m3_to_f32). */
static float g_e4m3[256];
__attribute__((constructor)) static void orc_init_e4m3(void) {
    for (int b = 0; b < 256; b++) g_e4m3[b] = orc_e4m3_to_f32((uint8_t)b);
}

/* Round-to-nearest-even at E4M3 precision with satfinite (|x| >= 448 -> 448). */
uint8_t orc_f32_to_e4m3_sat(float x) {
    if (isnan(x)) return 0x7F;
    uint8_t sign = signbit(x) ? 0x80 : 0x00;
    float a = fabsf(x);
    if (a >= 448.0f) return sign | 0x7E;
    if (a < 0.015625f) {                 /* below 2^-6: subnormal quantum 2^-9 */
        int q = (int)rintf(a * 512.0f);  /* exact scaling, RNE; q == 8 is 2^-6 */
        return sign | (uint8_t)q;
    }
    int e2;
    frexpf(a, &e2);                      /* a = f * 2^e2, f in [0.5, 1) */
    int E = e2 - 1;                      /* a in [2^E, 2^(E+1)), E in [-6, 8] */
    int q = (int)rintf(ldexpf(a, 3 - E));/* mantissa steps of 2^(E-3): q in [8,16] */
    if (q == 16) { q = 8; E += 1; }
    int code = ((E + 7) << 3) | (q - 8);
    if (code > 0x7E) code = 0x7E;
    return sign | (uint8_t)code;
}

/* ------------------------------------------------------------------------ */
/* offline INT4 format: tools/export_weights.py:64-79                         */
/* ------------------------------------------------------------------------ */
void orc_quant_int4_group(const float* w, int64_t N, int64_t K,
                          uint8_t* packed, uint16_t* scales) {
    const int G = 128;
    for (int64_t n = 0; n < N; n++) {
        for (int64_t g = 0; g < K / G; g++) {
            const float* wg = w + n * K + g * G;
            float amax = 0.0f;
            for (int i = 0; i < G; i++) { float a = fabsf(wg[i]); if (a > amax) amax = a; }
            float scale = amax / 7.0f;                 /* float32 divide */
            float safe = (scale == 0.0f) ? 1.0f : scale;
            scales[n * (K / G) + g] = orc_f2h(scale);
            for (int i = 0; i < G; i += 2) {
                float q0 = rintf(wg[i] / safe), q1 = rintf(wg[i + 1] / safe);
                if (q0 < -7.0f) q0 = -7.0f; if (q0 > 7.0f) q0 = 7.0f;
                if (q1 < -7.0f) q1 = -7.0f; if (q1 > 7.0f) q1 = 7.0f;
                uint8_t lo = (uint8_t)((int)q0 + 8), hi = (uint8_t)((int)q1 + 8);
                packed[n * (K / 2) + (g * G + i) / 2] = (uint8_t)(lo | (hi << 4));
            }
        }
    }
}

void orc_dequant_int4(const uint8_t* packed, const uint16_t* scales,
                      int64_t N, int64_t K, float* w) {
    for (int64_t n = 0; n < N; n++)
        for (int64_t k = 0; k < K; k++) {
            uint8_t b = packed[n * (K / 2) + k / 2];
            int nib = (k & 1) ? (b >> 4) : (b & 15);
            float sc = orc_h2f(scales[n * (K / 128) + k / 128]);
            w[n * K + k] = (float)(nib - 8) * sc;      /* exact in fp32 */
        }
}

/* ------------------------------------------------------------------------ */
/* kernels                                                                    */
/* ------------------------------------------------------------------------ */
/* gemv_int4, engine.cu:83-109: y[m,n] = sum_k x[m,k] * (nib-8)*scale[n,k/128] */
void orc_gemv_int4(const uint16_t* x, const uint8_t* packed, const uint16_t* scales,
                   float* y, int M, int N, int K) {
    /* Each weight row is dequantized once (exact fp32 (nib-8)*scale) and
     * dotted with every x row; per (m, n) the double sum runs over k in
     * order, the same arithmetic as one row at a time. */
    float* xs = (float*)malloc(sizeof(float) * (size_t)M * K);
    for (size_t i = 0; i < (size_t)M * K; i++) xs[i] = orc_h2f(x[i]);
#pragma omp parallel if ((size_t)N * K * M > (1u << 18))
    {
        float* wr = (float*)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(static)
        for (int n = 0; n < N; n++) {
            const uint8_t* prow = packed + (size_t)n * (K / 2);
            const uint16_t* srow = scales + (size_t)n * (K / 128);
            for (int g = 0; g < K / 128; g++) {
                float sc = orc_h2f(srow[g]);
                for (int j = g * 64; j < g * 64 + 64; j++) {
                    uint8_t b = prow[j];
                    wr[2 * j] = (float)((int)(b & 15) - 8) * sc;
                    wr[2 * j + 1] = (float)((int)(b >> 4) - 8) * sc;
                }
            }
            for (int m = 0; m < M; m++) {
                const float* xm = xs + (size_t)m * K;
#ifdef ORC_BASELINE
                float a8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                for (int k = 0; k < K; k += 8)
                    for (int u = 0; u < 8; u++) a8[u] += wr[k + u] * xm[k + u];
                y[(size_t)m * N + n] = ((a8[0] + a8[1]) + (a8[2] + a8[3])) + ((a8[4] + a8[5]) + (a8[6] + a8[7]));
#else
                double acc = 0.0;
                for (int j = 0; j < K / 2; j++)
                    acc += (double)wr[2 * j] * xm[2 * j] + (double)wr[2 * j + 1] * xm[2 * j + 1];
                y[(size_t)m * N + n] = (float)acc;
#endif
            }
        }
        free(wr);
    }
    free(xs);
}

/* gemv_fp16, engine.cu:112-128 */
void orc_gemv_fp16(const uint16_t* x, const uint16_t* W, float* y, int M, int N, int K) {
    for (int m = 0; m < M; m++) {
        float* xs = (float*)malloc(sizeof(float) * (size_t)K);
        for (int k = 0; k < K; k++) xs[k] = orc_h2f(x[(size_t)m * K + k]);
#pragma omp parallel for schedule(static) if ((size_t)N * K > (1u << 18))
        for (int n = 0; n < N; n++) {
            const uint16_t* wr = W + (size_t)n * K;
#ifdef ORC_BASELINE
            float a8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int k = 0; k + 8 <= K; k += 8)
                for (int u = 0; u < 8; u++) a8[u] += orc_h2f(wr[k + u]) * xs[k + u];
            float acc = ((a8[0] + a8[1]) + (a8[2] + a8[3])) + ((a8[4] + a8[5]) + (a8[6] + a8[7]));
            for (int k = K & ~7; k < K; k++) acc += orc_h2f(wr[k]) * xs[k];
            y[(size_t)m * N + n] = acc;
#else
            double acc = 0.0;
            for (int k = 0; k < K; k++) acc += (double)orc_h2f(wr[k]) * xs[k];
            y[(size_t)m * N + n] = (float)acc;
#endif
        }
        free(xs);
    }
}

/* rmsnorm / rmsnorm_head, engine.cu:131-158: half(x * rsqrt(mean(x^2)+eps) * w) */
void orc_rmsnorm(const uint16_t* in, const uint16_t* w, uint16_t* out, int M, int D, float eps) {
    for (int m = 0; m < M; m++) {
        const uint16_t* row = in + (size_t)m * D;
        double ss = 0.0;
        for (int i = 0; i < D; i++) { double v = orc_h2f(row[i]); ss += v * v; }
        float inv = 1.0f / sqrtf((float)ss / (float)D + eps);
        uint16_t* o = out + (size_t)m * D;
        for (int i = 0; i < D; i++) {
            float t = orc_h2f(row[i]) * inv;
            o[i] = orc_f2h(t * orc_h2f(w[i]));
        }
    }
}

/* rope, engine.cu:161-182 (NEOX rotate-half over pairs (d, d+hd/2)) */
void orc_rope(uint16_t* q, uint16_t* k, const int* pos, int S, int nq, int nk,
              int head_dim, float theta) {
    int half_d = head_dim / 2;
    for (int s = 0; s < S; s++) {
        for (int d = 0; d < half_d; d++) {
            float invf = powf(theta, -(float)(2 * d) / (float)head_dim);
            float ang = (float)pos[s] * invf;
            float cs = cosf(ang), sn = sinf(ang);
            for (int pass = 0; pass < 2; pass++) {
                uint16_t* base = pass == 0 ? q : k;
                int nh = pass == 0 ? nq : nk;
                for (int h = 0; h < nh; h++) {
                    uint16_t* b = base + ((size_t)s * nh + h) * head_dim;
                    float x0 = orc_h2f(b[d]), x1 = orc_h2f(b[d + half_d]);
                    float a = x0 * cs, bb = x1 * sn, c = x1 * cs, e = x0 * sn;
                    b[d] = orc_f2h(a - bb);
                    b[d + half_d] = orc_f2h(c + e);
                }
            }
        }
    }
}

/* kv_write_tail, engine.cu:190-198 */
void orc_kv_write_tail(const uint16_t* k, const uint16_t* v, uint16_t* ktail,
                       uint16_t* vtail, int slot, int cnt, int nkv, int hd) {
    size_t row = (size_t)nkv * hd;
    memcpy(ktail + (size_t)slot * row, k, (size_t)cnt * row * 2);
    memcpy(vtail + (size_t)slot * row, v, (size_t)cnt * row * 2);
}

/* kv_commit_group, engine.cu:202-228: one scale per kv head over 64 tokens;
 * quantized with the fp32 scale, stored fp16. */
void orc_kv_commit_group(const uint16_t* ktail, const uint16_t* vtail,
                         uint8_t* kc8, uint8_t* vc8, uint16_t* ksc, uint16_t* vsc,
                         int dst_tok_base, int grp, int nkv, int hd) {
    const int GROUP = 64;
    for (int h = 0; h < nkv; h++) {
        float mk = 0.0f, mv = 0.0f;
        for (int t = 0; t < GROUP; t++)
            for (int d = 0; d < hd; d++) {
                size_t off = ((size_t)t * nkv + h) * hd + d;
                float ak = fabsf(orc_h2f(ktail[off])), av = fabsf(orc_h2f(vtail[off]));
                if (ak > mk) mk = ak;
                if (av > mv) mv = av;
            }
        float sck = mk / 448.0f + 1e-12f;
        float scv = mv / 448.0f + 1e-12f;
        ksc[grp * nkv + h] = orc_f2h(sck);
        vsc[grp * nkv + h] = orc_f2h(scv);
        for (int t = 0; t < GROUP; t++)
            for (int d = 0; d < hd; d++) {
                size_t off = ((size_t)t * nkv + h) * hd + d;
                size_t dst = ((size_t)(dst_tok_base + t) * nkv + h) * hd + d;
                kc8[dst] = orc_f32_to_e4m3_sat(orc_h2f(ktail[off]) / sck);
                vc8[dst] = orc_f32_to_e4m3_sat(orc_h2f(vtail[off]) / scv);
            }
    }
}

/* attn_decode_split + attn_decode_combine, engine.cu:396-480: exact softmax
 * over keys [0, qpos]; keys < committed come from FP8 with their group scale,
 * the rest from the fp16 tail at index t - committed. */
void orc_attn_decode(const uint16_t* q, const uint8_t* kc8, const uint8_t* vc8,
                     const uint16_t* ksc, const uint16_t* vsc,
                     const uint16_t* ktail, const uint16_t* vtail,
                     int committed, int qpos, float scale, uint16_t* out,
                     int nh, int nkv, int hd) {
    int total = qpos + 1;
    int cend = committed < total ? committed : total;
    int gqa = nh / nkv;
#pragma omp parallel for schedule(static) if ((size_t)nh * total > 65536)
    for (int h = 0; h < nh; h++) {
        orc_acc* s = (orc_acc*)malloc(sizeof(orc_acc) * (size_t)total);
        orc_acc o[256];
        int kvh = h / gqa;
        const uint16_t* qh = q + (size_t)h * hd;
        float qf[256];
        for (int d = 0; d < hd; d++) qf[d] = orc_h2f(qh[d]);
        orc_acc mx = -INFINITY;
        for (int t = 0; t < total; t++) {
            orc_acc acc = 0.0;
            if (t < cend) {
                float kscl = orc_h2f(ksc[(t / 64) * nkv + kvh]);
                const uint8_t* kp = kc8 + ((size_t)t * nkv + kvh) * hd;
                for (int d = 0; d < hd; d++)
                    acc += (orc_acc)qf[d] * (orc_acc)(g_e4m3[kp[d]] * kscl);
            } else {
                const uint16_t* kp = ktail + ((size_t)(t - committed) * nkv + kvh) * hd;
                for (int d = 0; d < hd; d++) acc += (orc_acc)qf[d] * orc_h2f(kp[d]);
            }
            s[t] = acc * scale;
            if (s[t] > mx) mx = s[t];
        }
        orc_acc l = 0.0;
        for (int d = 0; d < hd; d++) o[d] = 0.0;
        for (int t = 0; t < total; t++) {
            orc_acc p = ORC_EXP(s[t] - mx);
            l += p;
            if (t < cend) {
                float vscl = orc_h2f(vsc[(t / 64) * nkv + kvh]);
                const uint8_t* vp = vc8 + ((size_t)t * nkv + kvh) * hd;
                for (int d = 0; d < hd; d++) o[d] += p * (orc_acc)(g_e4m3[vp[d]] * vscl);
            } else {
                const uint16_t* vp = vtail + ((size_t)(t - committed) * nkv + kvh) * hd;
                for (int d = 0; d < hd; d++) o[d] += p * orc_h2f(vp[d]);
            }
        }
        for (int d = 0; d < hd; d++) out[(size_t)h * hd + d] = orc_f2h((float)(o[d] / l));
        free(s);
    }
}

/* conv_pre, engine.cu:483-494: inproj rows are B | C | x */
void orc_conv_pre(const float* inproj, uint16_t* C, uint16_t* Bx, int S, int H) {
    for (int s = 0; s < S; s++)
        for (int c = 0; c < H; c++) {
            const float* row = inproj + (size_t)s * 3 * H;
            C[(size_t)s * H + c] = orc_f2h(row[H + c]);
            Bx[(size_t)s * H + c] = orc_f2h(row[c] * row[2 * H + c]);
        }
}

/* conv_apply, engine.cu:498-512: y = C * (Bx[s-2] w0 + Bx[s-1] w1 + Bx[s] w2) */
void orc_conv_apply(const uint16_t* Bx, const uint16_t* C, const uint16_t* w,
                    const uint16_t* state, uint16_t* y, int S, int H) {
    for (int s = 0; s < S; s++)
        for (int c = 0; c < H; c++) {
            float b[3];
            for (int j = 0; j < 3; j++) {
                int ss = s - 2 + j;
                b[j] = ss >= 0 ? orc_h2f(Bx[(size_t)ss * H + c]) : orc_h2f(state[(ss + 2) * H + c]);
            }
            float w0 = orc_h2f(w[c * 3 + 0]), w1 = orc_h2f(w[c * 3 + 1]), w2 = orc_h2f(w[c * 3 + 2]);
            float p0 = b[0] * w0, p1 = b[1] * w1, p2 = b[2] * w2;
            float co = (p0 + p1) + p2;
            y[(size_t)s * H + c] = orc_f2h(orc_h2f(C[(size_t)s * H + c]) * co);
        }
}

/* conv_update_state, engine.cu:514-525 */
void orc_conv_update_state(const uint16_t* Bx, uint16_t* state, int S, int H) {
    for (int c = 0; c < H; c++) {
        if (S == 1) {
            state[c] = state[H + c];
            state[H + c] = Bx[c];
        } else {
            state[c] = Bx[(size_t)(S - 2) * H + c];
            state[H + c] = Bx[(size_t)(S - 1) * H + c];
        }
    }
}

/* swiglu, engine.cu:542-547: half(g / (1 + exp(-g)) * u) */
void orc_swiglu(const float* g, const float* u, uint16_t* out, int n) {
    for (int i = 0; i < n; i++) {
        float x = g[i];
        float s = x / (1.0f + expf(-x));
        out[i] = orc_f2h(s * u[i]);
    }
}

/* acc_scaled, engine.cu:556-559 */
void orc_acc_scaled(uint16_t* dst, const float* src, float w, int n) {
    for (int i = 0; i < n; i++) {
        float t = w * src[i];
        dst[i] = orc_f2h(orc_h2f(dst[i]) + t);
    }
}

/* add_inplace / add_f32_inplace / f32_to_f16, engine.cu:527-540 */
void orc_add_inplace(uint16_t* a, const uint16_t* b, int n) {
    for (int i = 0; i < n; i++) a[i] = orc_f2h(orc_h2f(a[i]) + orc_h2f(b[i]));
}
void orc_add_f32_inplace(uint16_t* a, const float* b, int n) {
    for (int i = 0; i < n; i++) a[i] = orc_f2h(orc_h2f(a[i]) + b[i]);
}
void orc_f32_to_f16(const float* src, uint16_t* dst, int n) {
    for (int i = 0; i < n; i++) dst[i] = orc_f2h(src[i]);
}

/* MoE select, engine.cu:883-892 (host code, libm expf) */
void orc_moe_select(const float* logits, const float* bias, int n_exp, int topk,
                    int* idx, float* w) {
    float sig[256], score[256];
    int used[256];
    for (int e = 0; e < n_exp; e++) {
        sig[e] = 1.0f / (1.0f + expf(-logits[e]));
        score[e] = sig[e] + bias[e];
        used[e] = 0;
    }
    for (int t = 0; t < topk; t++) {
        int best = -1;
        float bv = -1e30f;
        for (int e = 0; e < n_exp; e++)
            if (!used[e] && score[e] > bv) { bv = score[e]; best = e; }
        used[best] = 1;
        idx[t] = best;
        w[t] = sig[best];
    }
    float wsum = 0.0f;
    for (int t = 0; t < topk; t++) wsum += w[t];
    for (int t = 0; t < topk; t++) w[t] /= (wsum + 1e-6f);
}

/* argmax_kernel, engine.cu:562-572, simulated with its 256 threads */
int orc_argmax(const float* v, int n) {
    float bv[256];
    int bi[256];
    for (int tid = 0; tid < 256; tid++) {
        float best = -1e30f;
        int bidx = 0;
        for (int i = tid; i < n; i += 256)
            if (v[i] > best) { best = v[i]; bidx = i; }
        bv[tid] = best;
        bi[tid] = bidx;
    }
    for (int s = 128; s > 0; s >>= 1)
        for (int tid = 0; tid < s; tid++)
            if (bv[tid + s] > bv[tid]) { bv[tid] = bv[tid + s]; bi[tid] = bi[tid + s]; }
    return bi[0];
}

/* ------------------------------------------------------------------------ */
/* whole model                                                                */
/* ------------------------------------------------------------------------ */
typedef struct { const uint8_t* p; const uint16_t* s; int N, K; } q4w;

typedef struct {
    const uint16_t *op_norm, *ffn_norm;
    q4w wq, wk, wv, wo;
    const uint16_t *q_ln, *k_ln;
    q4w in_proj, out_proj;
    const uint16_t* conv_w;
    q4w w1, w3, w2;
    const uint16_t *gate, *ebias;
    q4w *ew1, *ew3, *ew2;
} orc_layer;

typedef struct {
    char name[256];
    uint8_t kind;
    uint64_t offset, packed, scales;
    int64_t d0, d1;
} orc_tensor;

struct orc_model {
    orc_config cfg;
    const uint8_t* blob;
    size_t blob_len;
    orc_tensor* t;
    int nt;
    const uint16_t *embed, *emb_norm;
    orc_layer* L;
    int ok;
};

struct orc_state {
    int pos, max_ctx, nl;
    uint16_t* h;
    uint8_t **kc8, **vc8;
    uint16_t **ksc, **vsc, **ktail, **vtail, **conv_state;
    int* committed;
    int* route_idx;
    float* route_w;
    /* H2O eviction mode (engine.cu:310-384, 803-828): per attention layer a
     * circular buffer of `budget` per-token FP8 slots */
    int h2o_budget, h2o_window;
    uint8_t **hk8, **hv8;
    uint16_t **hks, **hvs;
    int** slot_pos;
    float** attn_sum;
    int* n_live;
    int* own_slot;     /* [nl] the slot this oracle chose in the last step */
    int* used_slot;    /* [nl] the slot it used (own, or forced) */
    int* forced_slot;  /* [nl] next step's forced slots, -1 = none */
};

static const orc_tensor* find_t(const orc_model* m, const char* name) {
    for (int i = 0; i < m->nt; i++)
        if (strcmp(m->t[i].name, name) == 0) return &m->t[i];
    return NULL;
}

static const uint16_t* f16_of(orc_model* m, const char* name) {
    const orc_tensor* t = find_t(m, name);
    if (!t || t->kind != 0 || t->offset + t->packed > m->blob_len) { m->ok = 0; return NULL; }
    return (const uint16_t*)(m->blob + t->offset);
}

static q4w q4_of(orc_model* m, const char* name) {
    q4w w = {0};
    const orc_tensor* t = find_t(m, name);
    if (!t || t->kind != 1 || t->offset + t->packed + t->scales > m->blob_len) { m->ok = 0; return w; }
    w.p = m->blob + t->offset;
    w.s = (const uint16_t*)(m->blob + t->offset + t->packed);
    w.N = (int)t->d0;
    w.K = (int)t->d1;
    return w;
}

/* index.bin, tools/make_index.py:3-11,21-36 */
static int parse_index(orc_model* m, const uint8_t* b, size_t len) {
    size_t p = 0;
    uint32_t n;
    if (len < 4) return -1;
    memcpy(&n, b, 4);
    p = 4;
    m->t = (orc_tensor*)calloc(n ? n : 1, sizeof(orc_tensor));
    m->nt = (int)n;
    for (uint32_t i = 0; i < n; i++) {
        if (p + 1 > len) return -1;
        uint8_t nl = b[p++];
        if (p + nl + 1 + 8 * 5 > len) return -1;
        memcpy(m->t[i].name, b + p, nl);
        m->t[i].name[nl] = 0;
        p += nl;
        m->t[i].kind = b[p++];
        memcpy(&m->t[i].offset, b + p, 8); p += 8;
        memcpy(&m->t[i].packed, b + p, 8); p += 8;
        memcpy(&m->t[i].scales, b + p, 8); p += 8;
        memcpy(&m->t[i].d0, b + p, 8); p += 8;
        memcpy(&m->t[i].d1, b + p, 8); p += 8;
    }
    return 0;
}

orc_model* orc_model_new(const orc_config* cfg, const uint8_t* blob, size_t blob_len,
                         const uint8_t* index, size_t index_len) {
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    m->cfg = *cfg;
    m->blob = blob;
    m->blob_len = blob_len;
    m->ok = 1;
    if (parse_index(m, index, index_len) != 0) { orc_model_free(m); return NULL; }
    m->embed = f16_of(m, "model.embed_tokens.weight");
    m->emb_norm = f16_of(m, "model.embedding_norm.weight");
    m->L = (orc_layer*)calloc((size_t)cfg->n_layers, sizeof(orc_layer));
    char nm[256];
    for (int l = 0; l < cfg->n_layers; l++) {
        orc_layer* L = &m->L[l];
#define P(s) (snprintf(nm, sizeof nm, "model.layers.%d.%s", l, s), nm)
        L->op_norm = f16_of(m, P("operator_norm.weight"));
        L->ffn_norm = f16_of(m, P("ffn_norm.weight"));
        if (cfg->attn_layer[l]) {
            L->wq = q4_of(m, P("self_attn.q_proj.weight"));
            L->wk = q4_of(m, P("self_attn.k_proj.weight"));
            L->wv = q4_of(m, P("self_attn.v_proj.weight"));
            L->wo = q4_of(m, P("self_attn.out_proj.weight"));
            L->q_ln = f16_of(m, P("self_attn.q_layernorm.weight"));
            L->k_ln = f16_of(m, P("self_attn.k_layernorm.weight"));
        } else {
            L->in_proj = q4_of(m, P("conv.in_proj.weight"));
            L->out_proj = q4_of(m, P("conv.out_proj.weight"));
            L->conv_w = f16_of(m, P("conv.conv.weight"));
        }
        if (l < cfg->n_dense) {
            L->w1 = q4_of(m, P("feed_forward.w1.weight"));
            L->w3 = q4_of(m, P("feed_forward.w3.weight"));
            L->w2 = q4_of(m, P("feed_forward.w2.weight"));
        } else {
            L->gate = f16_of(m, P("feed_forward.gate.weight"));
            L->ebias = f16_of(m, P("feed_forward.expert_bias"));
            L->ew1 = (q4w*)calloc((size_t)cfg->n_experts, sizeof(q4w));
            L->ew3 = (q4w*)calloc((size_t)cfg->n_experts, sizeof(q4w));
            L->ew2 = (q4w*)calloc((size_t)cfg->n_experts, sizeof(q4w));
            for (int e = 0; e < cfg->n_experts; e++) {
                char en[128];
                snprintf(en, sizeof en, "feed_forward.experts.%d.w1.weight", e);
                L->ew1[e] = q4_of(m, P(en));
                snprintf(en, sizeof en, "feed_forward.experts.%d.w3.weight", e);
                L->ew3[e] = q4_of(m, P(en));
                snprintf(en, sizeof en, "feed_forward.experts.%d.w2.weight", e);
                L->ew2[e] = q4_of(m, P(en));
            }
        }
#undef P
    }
    if (!m->ok) { orc_model_free(m); return NULL; }
    return m;
}

void orc_model_free(orc_model* m) {
    if (!m) return;
    if (m->L) {
        for (int l = 0; l < m->cfg.n_layers; l++) {
            free(m->L[l].ew1); free(m->L[l].ew3); free(m->L[l].ew2);
        }
        free(m->L);
    }
    free(m->t);
    free(m);
}

orc_state* orc_state_new(const orc_model* m, int max_ctx) {
    const orc_config* c = &m->cfg;
    orc_state* s = (orc_state*)calloc(1, sizeof(orc_state));
    int nl = c->n_layers, H = c->hidden, row = c->n_kv_heads * c->head_dim;
    int maxg = max_ctx / 64 + 2;
    s->max_ctx = max_ctx;
    s->nl = nl;
    s->h = (uint16_t*)calloc((size_t)H, 2);
    s->kc8 = (uint8_t**)calloc((size_t)nl, sizeof(void*));
    s->vc8 = (uint8_t**)calloc((size_t)nl, sizeof(void*));
    s->ksc = (uint16_t**)calloc((size_t)nl, sizeof(void*));
    s->vsc = (uint16_t**)calloc((size_t)nl, sizeof(void*));
    s->ktail = (uint16_t**)calloc((size_t)nl, sizeof(void*));
    s->vtail = (uint16_t**)calloc((size_t)nl, sizeof(void*));
    s->conv_state = (uint16_t**)calloc((size_t)nl, sizeof(void*));
    s->committed = (int*)calloc((size_t)nl, sizeof(int));
    s->route_idx = (int*)calloc((size_t)nl * (c->top_k > 0 ? c->top_k : 1), sizeof(int));
    s->route_w = (float*)calloc((size_t)nl * (c->top_k > 0 ? c->top_k : 1), sizeof(float));
    s->n_live = (int*)calloc((size_t)nl, sizeof(int));
    s->own_slot = (int*)calloc((size_t)nl, sizeof(int));
    s->used_slot = (int*)calloc((size_t)nl, sizeof(int));
    s->forced_slot = (int*)malloc((size_t)nl * sizeof(int));
    for (int l = 0; l < nl; l++) s->own_slot[l] = s->used_slot[l] = s->forced_slot[l] = -1;
    for (int l = 0; l < nl; l++) {
        if (c->attn_layer[l]) {
            s->kc8[l] = (uint8_t*)calloc((size_t)max_ctx * row, 1);
            s->vc8[l] = (uint8_t*)calloc((size_t)max_ctx * row, 1);
            s->ksc[l] = (uint16_t*)calloc((size_t)maxg * c->n_kv_heads, 2);
            s->vsc[l] = (uint16_t*)calloc((size_t)maxg * c->n_kv_heads, 2);
            s->ktail[l] = (uint16_t*)calloc((size_t)64 * row, 2);
            s->vtail[l] = (uint16_t*)calloc((size_t)64 * row, 2);
        } else {
            s->conv_state[l] = (uint16_t*)calloc((size_t)2 * H, 2);
        }
    }
    return s;
}

void orc_state_free(orc_state* s) {
    if (!s) return;
    for (int l = 0; l < s->nl; l++) {
        free(s->kc8[l]); free(s->vc8[l]); free(s->ksc[l]); free(s->vsc[l]);
        free(s->ktail[l]); free(s->vtail[l]); free(s->conv_state[l]);
    }
    if (s->h2o_budget > 0) {
        for (int l = 0; l < s->nl; l++) {
            free(s->hk8[l]); free(s->hv8[l]); free(s->hks[l]); free(s->hvs[l]);
            free(s->slot_pos[l]); free(s->attn_sum[l]);
        }
        free(s->hk8); free(s->hv8); free(s->hks); free(s->hvs); free(s->slot_pos); free(s->attn_sum);
    }
    free(s->n_live); free(s->own_slot); free(s->used_slot); free(s->forced_slot);
    free(s->h);
    free(s->committed);
    free(s->route_idx);
    free(s->route_w);
    free(s->kc8); free(s->vc8); free(s->ksc); free(s->vsc);
    free(s->ktail); free(s->vtail); free(s->conv_state);
    free(s);
}

int orc_state_pos(const orc_state* s) { return s->pos; }

int orc_state_load(const orc_model* m, orc_state* s, const uint8_t* buf, size_t n) {
    const orc_config* c = &m->cfg;
    int32_t hd[8];
    uint32_t magic, version;
    if (n < 32) return -1;
    memcpy(&magic, buf, 4);
    memcpy(&version, buf + 4, 4);
    memcpy(hd, buf + 8, 24);
    const int pos = hd[0];
    if (magic != 0x54534943u || version != 1 || hd[1] != c->n_layers || hd[2] != c->hidden ||
        hd[3] != c->n_kv_heads || pos < 0 || pos >= s->max_ctx || s->h2o_budget > 0)
        return -1;
    const size_t row = (size_t)c->n_kv_heads * c->head_dim;
    const size_t C = (size_t)(pos / 64) * 64;
    size_t need = 32;
    for (int l = 0; l < c->n_layers; l++)
        need += c->attn_layer[l] ? 2 * C * row + 2 * (C / 64) * c->n_kv_heads * 2 + 2 * 64 * row * 2
                                 : (size_t)2 * c->hidden * 2;
    if (n != need) return -1;
    const uint8_t* p = buf + 32;
    for (int l = 0; l < c->n_layers; l++) {
        if (c->attn_layer[l]) {
            const size_t sc = (C / 64) * c->n_kv_heads * 2, tail = 64 * row * 2;
            memcpy(s->kc8[l], p, C * row); p += C * row;
            memcpy(s->vc8[l], p, C * row); p += C * row;
            memcpy(s->ksc[l], p, sc); p += sc;
            memcpy(s->vsc[l], p, sc); p += sc;
            memcpy(s->ktail[l], p, tail); p += tail;
            memcpy(s->vtail[l], p, tail); p += tail;
            s->committed[l] = (int)C;
        } else {
            memcpy(s->conv_state[l], p, (size_t)2 * c->hidden * 2);
            p += (size_t)2 * c->hidden * 2;
        }
    }
    s->pos = pos;
    return 0;
}

/* H2O mode: budget slots per attention layer, local window W (the reference's
 * defaults: budget >= prompt, W = budget/2, W < budget; engine.cu:753-756). */
int orc_state_set_h2o(const orc_model* m, orc_state* s, int budget, int window) {
    const orc_config* c = &m->cfg;
    if (budget <= 0 || window <= 0 || window >= budget || s->pos != 0 || s->h2o_budget) return -1;
    const size_t row = (size_t)c->n_kv_heads * c->head_dim;
    s->h2o_budget = budget;
    s->h2o_window = window;
    s->hk8 = (uint8_t**)calloc((size_t)s->nl, sizeof(void*));
    s->hv8 = (uint8_t**)calloc((size_t)s->nl, sizeof(void*));
    s->hks = (uint16_t**)calloc((size_t)s->nl, sizeof(void*));
    s->hvs = (uint16_t**)calloc((size_t)s->nl, sizeof(void*));
    s->slot_pos = (int**)calloc((size_t)s->nl, sizeof(void*));
    s->attn_sum = (float**)calloc((size_t)s->nl, sizeof(void*));
    for (int l = 0; l < s->nl; l++) {
        if (!c->attn_layer[l]) continue;
        s->hk8[l] = (uint8_t*)calloc((size_t)budget * row, 1);
        s->hv8[l] = (uint8_t*)calloc((size_t)budget * row, 1);
        s->hks[l] = (uint16_t*)calloc((size_t)budget * c->n_kv_heads, 2);
        s->hvs[l] = (uint16_t*)calloc((size_t)budget * c->n_kv_heads, 2);
        s->slot_pos[l] = (int*)calloc((size_t)budget, sizeof(int));
        s->attn_sum[l] = (float*)calloc((size_t)budget, sizeof(float));
    }
    return 0;
}
const int* orc_state_h2o_own_slots(const orc_state* s) { return s->own_slot; }
const int* orc_state_h2o_used_slots(const orc_state* s) { return s->used_slot; }
const float* orc_state_h2o_attn_sum(const orc_state* s, int layer) {
    return s->h2o_budget && s->attn_sum[layer] ? s->attn_sum[layer] : NULL;
}
const int* orc_state_h2o_slot_pos(const orc_state* s, int layer) {
    return s->h2o_budget && s->slot_pos[layer] ? s->slot_pos[layer] : NULL;
}
int orc_state_h2o_n_live(const orc_state* s, int layer) { return s->n_live[layer]; }
void orc_state_force_h2o_slots(orc_state* s, const int* slots) {
    for (int l = 0; l < s->nl; l++) s->forced_slot[l] = slots ? slots[l] : -1;
}

/* The reference's slot choice for a fresh token at position pos (host loop,
 * engine.cu:808-823): append while there is room; else the slot with the
 * least cumulative attention among those outside the local window (first
 * such minimum), else the least overall.  `banned` slots (picked earlier in
 * the same batch) count as +inf. */
static int h2o_choose(const orc_state* s, int l, int pos, const unsigned char* banned) {
    const int C = s->h2o_budget, W = s->h2o_window;
    if (s->n_live[l] < C) return s->n_live[l];
    int best = -1;
    float bv = 1e30f;
    for (int t = 0; t < C; t++) {
        float a = banned && banned[t] ? 1e30f : s->attn_sum[l][t];
        if (s->slot_pos[l][t] <= pos - W && a < bv) { bv = a; best = t; }
    }
    if (best < 0)
        for (int t = 0; t < C; t++) {
            float a = banned && banned[t] ? 1e30f : s->attn_sum[l][t];
            if (a < bv) { bv = a; best = t; }
        }
    return best;
}

/* kv_quant_write, engine.cu:317-333: one token's K/V per head into a slot,
 * scale = absmax/448 + 1e-12 (fp32 for the quantization, stored fp16). */
static void h2o_write(orc_state* s, int l, int slot, const uint16_t* k, const uint16_t* v, int nkv, int hd) {
    for (int h = 0; h < nkv; h++) {
        for (int which = 0; which < 2; which++) {
            const uint16_t* src = (which ? v : k) + (size_t)h * hd;
            float mx = 0.f;
            for (int d = 0; d < hd; d++) {
                float a = fabsf(orc_h2f(src[d]));
                if (a > mx) mx = a;
            }
            float sc = mx / 448.0f + 1e-12f;
            uint8_t* dst = (which ? s->hv8[l] : s->hk8[l]) + ((size_t)slot * nkv + h) * hd;
            for (int d = 0; d < hd; d++) dst[d] = orc_f32_to_e4m3_sat(orc_h2f(src[d]) / sc);
            (which ? s->hvs[l] : s->hks[l])[slot * nkv + h] = orc_f2h(sc);
        }
    }
}

/* attention_h2o, engine.cu:337-384: exact softmax over the live slots with
 * slot position <= qpos; each slot's normalized probability is added to its
 * cumulative attention (summed over query heads). */
static void h2o_attend(orc_state* s, int l, const uint16_t* q, int qpos, float scale, uint16_t* out, int nh,
                       int nkv, int hd) {
    const int n = s->n_live[l], gqa = nh / nkv;
    double* sc = (double*)malloc(sizeof(double) * (size_t)(n > 0 ? n : 1));
    double* o = (double*)malloc(sizeof(double) * (size_t)hd);
    for (int h = 0; h < nh; h++) {
        const int kvh = h / gqa;
        const uint16_t* qh = q + (size_t)h * hd;
        double mx = -INFINITY;
        for (int t = 0; t < n; t++) {
            if (s->slot_pos[l][t] > qpos) continue;
            const float ks = orc_h2f(s->hks[l][t * nkv + kvh]);
            const uint8_t* kp = s->hk8[l] + ((size_t)t * nkv + kvh) * hd;
            double acc = 0.0;
            for (int d = 0; d < hd; d++) acc += (double)orc_h2f(qh[d]) * (double)(orc_e4m3_to_f32(kp[d]) * ks);
            sc[t] = acc * scale;
            if (sc[t] > mx) mx = sc[t];
        }
        double L = 0.0;
        for (int d = 0; d < hd; d++) o[d] = 0.0;
        for (int t = 0; t < n; t++) {
            if (s->slot_pos[l][t] > qpos) continue;
            const double p = exp(sc[t] - mx);
            L += p;
            const float vs = orc_h2f(s->hvs[l][t * nkv + kvh]);
            const uint8_t* vp = s->hv8[l] + ((size_t)t * nkv + kvh) * hd;
            for (int d = 0; d < hd; d++) o[d] += p * (double)(orc_e4m3_to_f32(vp[d]) * vs);
        }
        for (int d = 0; d < hd; d++) out[(size_t)h * hd + d] = orc_f2h((float)(o[d] / L));
        for (int t = 0; t < n; t++)
            if (s->slot_pos[l][t] <= qpos) s->attn_sum[l][t] += (float)(exp(sc[t] - mx) / L);
    }
    free(sc);
    free(o);
}

/* One token's H2O placement and attention in layer l (decode, S = 1). */
static void h2o_step(orc_state* s, int l, int pos, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                     float scale, uint16_t* out, int nh, int nkv, int hd) {
    int own = h2o_choose(s, l, pos, NULL);
    int slot = s->forced_slot[l] >= 0 ? s->forced_slot[l] : own;
    s->own_slot[l] = own;
    s->used_slot[l] = slot;
    if (s->n_live[l] < s->h2o_budget && slot == s->n_live[l]) s->n_live[l]++;
    s->attn_sum[l][slot] = 0.f;
    s->slot_pos[l][slot] = pos;
    h2o_write(s, l, slot, k, v, nkv, hd);
    h2o_attend(s, l, q, pos, scale, out, nh, nkv, hd);
}
const int* orc_state_route_idx(const orc_state* s) { return s->route_idx; }
const float* orc_state_route_w(const orc_state* s) { return s->route_w; }

int orc_forward_token(const orc_model* m, orc_state* s, int token, float* logits_out,
                      uint16_t* hidden_out) {
    return orc_forward_token_ex(m, s, token, NULL, NULL, logits_out, hidden_out);
}

/* layer_forward for S == 1 (engine.cu:784-908) + compute_logits_last (932-940).
 * forced_idx [n_moe][top_k] (nullable) replaces the selected experts (the
 * weights are still the oracle's sigmoid of those experts, normalized);
 * scores_out [n_moe][n_experts] (nullable) receives sigmoid+bias scores. */
int orc_forward_token_ex(const orc_model* m, orc_state* s, int token, const int* forced_idx,
                         float* scores_out, float* logits_out, uint16_t* hidden_out) {
    const orc_config* c = &m->cfg;
    const int H = c->hidden, hd = c->head_dim, nh = c->n_heads, nkv = c->n_kv_heads;
    const float eps = c->norm_eps;
    int pos = s->pos;
    int maxI = c->dense_inter > c->moe_inter ? c->dense_inter : c->moe_inter;
    int maxN = 3 * H;
    if (maxI > maxN) maxN = maxI;
    if (nh * hd > maxN) maxN = nh * hd;
    if (c->vocab > maxN) maxN = c->vocab;

    uint16_t* xn = (uint16_t*)malloc((size_t)H * 2);
    uint16_t* t16 = (uint16_t*)malloc((size_t)maxN * 2);
    uint16_t* t16b = (uint16_t*)malloc((size_t)maxN * 2);
    uint16_t* q16 = (uint16_t*)malloc((size_t)nh * hd * 2);
    uint16_t* k16 = (uint16_t*)malloc((size_t)nkv * hd * 2);
    uint16_t* v16 = (uint16_t*)malloc((size_t)nkv * hd * 2);
    uint16_t* ao = (uint16_t*)malloc((size_t)nh * hd * 2);
    uint16_t* acc = (uint16_t*)malloc((size_t)H * 2);
    float* fa = (float*)malloc((size_t)maxN * 4);
    float* fb = (float*)malloc((size_t)maxN * 4);

    memcpy(s->h, m->embed + (size_t)token * H, (size_t)H * 2); /* embed_gather 549-554 */
    int moe_i = 0;
    for (int l = 0; l < c->n_layers; l++) {
        const orc_layer* L = &m->L[l];
        orc_rmsnorm(s->h, L->op_norm, xn, 1, H, eps);
        if (c->attn_layer[l]) {
            orc_gemv_int4(xn, L->wq.p, L->wq.s, fa, 1, L->wq.N, H);
            orc_f32_to_f16(fa, q16, nh * hd);
            orc_gemv_int4(xn, L->wk.p, L->wk.s, fa, 1, L->wk.N, H);
            orc_f32_to_f16(fa, k16, nkv * hd);
            orc_gemv_int4(xn, L->wv.p, L->wv.s, fa, 1, L->wv.N, H);
            orc_f32_to_f16(fa, v16, nkv * hd);
            orc_rmsnorm(q16, L->q_ln, q16, nh, hd, eps);
            orc_rmsnorm(k16, L->k_ln, k16, nkv, hd, eps);
            orc_rope(q16, k16, &pos, 1, nh, nkv, hd, c->rope_theta);
            if (s->h2o_budget > 0) {
                h2o_step(s, l, pos, q16, k16, v16, 1.0f / sqrtf((float)hd), ao, nh, nkv, hd);
                orc_gemv_int4(ao, L->wo.p, L->wo.s, fa, 1, H, nh * hd);
                orc_add_f32_inplace(s->h, fa, H);
                goto ffn;
            }
            int slot = pos - s->committed[l];
            orc_kv_write_tail(k16, v16, s->ktail[l], s->vtail[l], slot, 1, nkv, hd);
            if (slot + 1 == 64) {
                orc_kv_commit_group(s->ktail[l], s->vtail[l], s->kc8[l], s->vc8[l],
                                    s->ksc[l], s->vsc[l], s->committed[l],
                                    s->committed[l] / 64, nkv, hd);
                s->committed[l] += 64;
            }
            float scale = 1.0f / sqrtf((float)hd);
            orc_attn_decode(q16, s->kc8[l], s->vc8[l], s->ksc[l], s->vsc[l], s->ktail[l],
                            s->vtail[l], s->committed[l], pos, scale, ao, nh, nkv, hd);
            orc_gemv_int4(ao, L->wo.p, L->wo.s, fa, 1, H, nh * hd);
            orc_add_f32_inplace(s->h, fa, H);
        } else {
            orc_gemv_int4(xn, L->in_proj.p, L->in_proj.s, fa, 1, 3 * H, H);
            uint16_t* Cb = t16;
            uint16_t* Bx = t16b;
            orc_conv_pre(fa, Cb, Bx, 1, H);
            orc_conv_apply(Bx, Cb, L->conv_w, s->conv_state[l], acc, 1, H);
            orc_conv_update_state(Bx, s->conv_state[l], 1, H);
            orc_gemv_int4(acc, L->out_proj.p, L->out_proj.s, fa, 1, H, H);
            orc_add_f32_inplace(s->h, fa, H);
        }
    ffn:
        orc_rmsnorm(s->h, L->ffn_norm, xn, 1, H, eps);
        if (l < c->n_dense) {
            int I = c->dense_inter;
            orc_gemv_int4(xn, L->w1.p, L->w1.s, fa, 1, I, H);
            orc_gemv_int4(xn, L->w3.p, L->w3.s, fb, 1, I, H);
            orc_swiglu(fa, fb, t16, I);
            orc_gemv_int4(t16, L->w2.p, L->w2.s, fa, 1, H, I);
            orc_add_f32_inplace(s->h, fa, H);
        } else {
            int E = c->n_experts, K = c->top_k, I = c->moe_inter;
            float rl[256], eb[256], w[16];
            int idx[16];
            orc_gemv_fp16(xn, L->gate, rl, 1, E, H);
            for (int e = 0; e < E; e++) eb[e] = orc_h2f(L->ebias[e]);
            orc_moe_select(rl, eb, E, K, idx, w);
            if (scores_out)
                for (int e = 0; e < E; e++)
                    scores_out[moe_i * E + e] = 1.0f / (1.0f + expf(-rl[e])) + eb[e];
            if (forced_idx) {  /* same weight rule (engine.cu:890-892) on the given experts */
                float wsum = 0.0f;
                for (int t = 0; t < K; t++) {
                    idx[t] = forced_idx[moe_i * K + t];
                    w[t] = 1.0f / (1.0f + expf(-rl[idx[t]]));
                }
                for (int t = 0; t < K; t++) wsum += w[t];
                for (int t = 0; t < K; t++) w[t] /= (wsum + 1e-6f);
            }
            for (int t = 0; t < K; t++) {
                s->route_idx[moe_i * K + t] = idx[t];
                s->route_w[moe_i * K + t] = w[t];
            }
            memset(acc, 0, (size_t)H * 2);
            for (int t = 0; t < K; t++) {
                int e = idx[t];
                orc_gemv_int4(xn, L->ew1[e].p, L->ew1[e].s, fa, 1, I, H);
                orc_gemv_int4(xn, L->ew3[e].p, L->ew3[e].s, fb, 1, I, H);
                orc_swiglu(fa, fb, t16, I);
                orc_gemv_int4(t16, L->ew2[e].p, L->ew2[e].s, fa, 1, H, I);
                orc_acc_scaled(acc, fa, w[t], H);
            }
            orc_add_inplace(s->h, acc, H);
            moe_i++;
        }
    }
    if (hidden_out) memcpy(hidden_out, s->h, (size_t)H * 2);
    orc_rmsnorm(s->h, m->emb_norm, xn, 1, H, eps);
    float* lg = (float*)malloc((size_t)c->vocab * 4);
    orc_gemv_fp16(xn, m->embed, lg, 1, c->vocab, H);
    int next = orc_argmax(lg, c->vocab);
    if (logits_out) memcpy(logits_out, lg, (size_t)c->vocab * 4);
    free(lg);
    s->pos++;
    free(xn); free(t16); free(t16b); free(q16); free(k16); free(v16);
    free(ao); free(acc); free(fa); free(fb);
    return next;
}

/* Prefill: layer_forward for S tokens at positions pos..pos+S-1
 * (engine.cu:784-908) followed by compute_logits_last (932-940).  Per layer,
 * all S tokens' K/V are placed first (the placement loop at 831-845 writes
 * the tail up to each group boundary and commits every full group), and only
 * then does each query attend (attention_fused, 236-308): query i sees keys
 * [0, pos+i], those below the post-placement committed count from FP8.
 * Routing is per token (883-892).  Returns the argmax of the last row's
 * logits; logits_out (nullable) receives them. */
int orc_prefill(const orc_model* m, orc_state* s, const int* tokens, int S, float* logits_out) {
    return orc_prefill_ex(m, s, tokens, S, NULL, NULL, logits_out);
}

/* Same, with optional forced expert choices forced_idx [S][n_moe][top_k]
 * (weights recomputed from the oracle's router for those experts) and the
 * oracle's own scores sigmoid+bias written to scores_out [S][n_moe][E]. */
int orc_prefill_ex(const orc_model* m, orc_state* s, const int* tokens, int S, const int* forced_idx,
                   float* scores_out, float* logits_out) {
    const orc_config* c = &m->cfg;
    const int H = c->hidden, hd = c->head_dim, nh = c->n_heads, nkv = c->n_kv_heads;
    const float eps = c->norm_eps;
    const int past = s->pos;
    int maxI = c->dense_inter > c->moe_inter ? c->dense_inter : c->moe_inter;
    int maxN = 3 * H;
    if (maxI > maxN) maxN = maxI;
    if (nh * hd > maxN) maxN = nh * hd;
    uint16_t* hs = (uint16_t*)malloc((size_t)S * H * 2);
    uint16_t* xn = (uint16_t*)malloc((size_t)S * H * 2);
    uint16_t* q16 = (uint16_t*)malloc((size_t)S * nh * hd * 2);
    uint16_t* k16 = (uint16_t*)malloc((size_t)S * nkv * hd * 2);
    uint16_t* v16 = (uint16_t*)malloc((size_t)S * nkv * hd * 2);
    uint16_t* ao = (uint16_t*)malloc((size_t)S * nh * hd * 2);
    uint16_t* t16 = (uint16_t*)malloc((size_t)S * maxN * 2);
    uint16_t* t16b = (uint16_t*)malloc((size_t)S * maxN * 2);
    uint16_t* acc = (uint16_t*)malloc((size_t)S * H * 2);
    float* fa = (float*)malloc((size_t)S * maxN * 4);
    float* fb = (float*)malloc((size_t)S * maxN * 4);
    int* pos = (int*)malloc((size_t)S * sizeof(int));
    for (int i = 0; i < S; i++) {
        memcpy(hs + (size_t)i * H, m->embed + (size_t)tokens[i] * H, (size_t)H * 2);  /* embed_gather */
        pos[i] = past + i;
    }
    int moe_i = 0;
    for (int l = 0; l < c->n_layers; l++) {
        const orc_layer* L = &m->L[l];
        orc_rmsnorm(hs, L->op_norm, xn, S, H, eps);
        if (c->attn_layer[l]) {
            orc_gemv_int4(xn, L->wq.p, L->wq.s, fa, S, L->wq.N, H);
            orc_f32_to_f16(fa, q16, S * nh * hd);
            orc_gemv_int4(xn, L->wk.p, L->wk.s, fa, S, L->wk.N, H);
            orc_f32_to_f16(fa, k16, S * nkv * hd);
            orc_gemv_int4(xn, L->wv.p, L->wv.s, fa, S, L->wv.N, H);
            orc_f32_to_f16(fa, v16, S * nkv * hd);
            orc_rmsnorm(q16, L->q_ln, q16, S * nh, hd, eps);
            orc_rmsnorm(k16, L->k_ln, k16, S * nkv, hd, eps);
            orc_rope(q16, k16, pos, S, nh, nkv, hd, c->rope_theta);
            if (s->h2o_budget > 0) {
                /* H2O (engine.cu:804-828): choose every fresh token's slot
                 * (earlier picks of this batch excluded), write them all,
                 * then every query attends over the live slots */
                unsigned char* banned = (unsigned char*)calloc((size_t)s->h2o_budget, 1);
                int* dst = (int*)malloc((size_t)S * sizeof(int));
                for (int j = 0; j < S; j++) {
                    int slot = h2o_choose(s, l, past + j, banned);
                    if (s->n_live[l] < s->h2o_budget && slot == s->n_live[l]) s->n_live[l]++;
                    banned[slot] = 1;
                    s->attn_sum[l][slot] = 0.f;
                    s->slot_pos[l][slot] = past + j;
                    dst[j] = slot;
                    s->own_slot[l] = s->used_slot[l] = slot;
                }
                for (int j = 0; j < S; j++)
                    h2o_write(s, l, dst[j], k16 + (size_t)j * nkv * hd, v16 + (size_t)j * nkv * hd, nkv, hd);
                for (int i = 0; i < S; i++)
                    h2o_attend(s, l, q16 + (size_t)i * nh * hd, past + i, 1.0f / sqrtf((float)hd),
                               ao + (size_t)i * nh * hd, nh, nkv, hd);
                free(banned);
                free(dst);
                orc_gemv_int4(ao, L->wo.p, L->wo.s, fa, S, H, nh * hd);
                orc_add_f32_inplace(hs, fa, S * H);
                goto ffn_pf;
            }
            int placed = 0;
            while (placed < S) {  /* engine.cu:831-845 */
                int slot = past + placed - s->committed[l];
                int can = S - placed < 64 - slot ? S - placed : 64 - slot;
                orc_kv_write_tail(k16 + (size_t)placed * nkv * hd, v16 + (size_t)placed * nkv * hd,
                                  s->ktail[l], s->vtail[l], slot, can, nkv, hd);
                placed += can;
                if (slot + can == 64) {
                    orc_kv_commit_group(s->ktail[l], s->vtail[l], s->kc8[l], s->vc8[l], s->ksc[l],
                                        s->vsc[l], s->committed[l], s->committed[l] / 64, nkv, hd);
                    s->committed[l] += 64;
                }
            }
            float scale = 1.0f / sqrtf((float)hd);
#pragma omp parallel for schedule(dynamic, 4) if (S > 8)
            for (int i = 0; i < S; i++)
                orc_attn_decode(q16 + (size_t)i * nh * hd, s->kc8[l], s->vc8[l], s->ksc[l], s->vsc[l],
                                s->ktail[l], s->vtail[l], s->committed[l], past + i, scale,
                                ao + (size_t)i * nh * hd, nh, nkv, hd);
            orc_gemv_int4(ao, L->wo.p, L->wo.s, fa, S, H, nh * hd);
            orc_add_f32_inplace(hs, fa, S * H);
        } else {
            orc_gemv_int4(xn, L->in_proj.p, L->in_proj.s, fa, S, 3 * H, H);
            orc_conv_pre(fa, t16, t16b, S, H);
            orc_conv_apply(t16b, t16, L->conv_w, s->conv_state[l], acc, S, H);
            orc_conv_update_state(t16b, s->conv_state[l], S, H);
            orc_gemv_int4(acc, L->out_proj.p, L->out_proj.s, fa, S, H, H);
            orc_add_f32_inplace(hs, fa, S * H);
        }
    ffn_pf:
        orc_rmsnorm(hs, L->ffn_norm, xn, S, H, eps);
        if (l < c->n_dense) {
            int I = c->dense_inter;
            orc_gemv_int4(xn, L->w1.p, L->w1.s, fa, S, I, H);
            orc_gemv_int4(xn, L->w3.p, L->w3.s, fb, S, I, H);
            orc_swiglu(fa, fb, t16, S * I);
            orc_gemv_int4(t16, L->w2.p, L->w2.s, fa, S, H, I);
            orc_add_f32_inplace(hs, fa, S * H);
        } else {
            int E = c->n_experts, K = c->top_k, I = c->moe_inter;
            float rl[256], eb[256], w[16];
            int idx[16];
            for (int e = 0; e < E; e++) eb[e] = orc_h2f(L->ebias[e]);
            memset(acc, 0, (size_t)S * H * 2);  /* expert_out_acc, engine.cu:882 */
            const int n_moe = c->n_layers - c->n_dense;
            int* idx_all = (int*)malloc((size_t)S * K * sizeof(int));
            float* w_all = (float*)malloc((size_t)S * K * sizeof(float));
            for (int i = 0; i < S; i++) {
                const uint16_t* xi = xn + (size_t)i * H;
                orc_gemv_fp16(xi, L->gate, rl, 1, E, H);
                orc_moe_select(rl, eb, E, K, idx, w);
                if (scores_out)
                    for (int e = 0; e < E; e++)
                        scores_out[((size_t)i * n_moe + moe_i) * E + e] = 1.0f / (1.0f + expf(-rl[e])) + eb[e];
                if (forced_idx) {
                    float wsum = 0.0f;
                    for (int t = 0; t < K; t++) {
                        idx[t] = forced_idx[((size_t)i * n_moe + moe_i) * K + t];
                        w[t] = 1.0f / (1.0f + expf(-rl[idx[t]]));
                    }
                    for (int t = 0; t < K; t++) wsum += w[t];
                    for (int t = 0; t < K; t++) w[t] /= (wsum + 1e-6f);
                }
                for (int t = 0; t < K; t++) {
                    s->route_idx[moe_i * K + t] = idx[t];
                    s->route_w[moe_i * K + t] = w[t];
                    idx_all[i * K + t] = idx[t];
                    w_all[i * K + t] = w[t];
                }
            }
            /* every (token, slot) row's expert output o = W2e . swiglu(W1e x, W3e x)
             * (engine.cu:894-902), the rows of one expert in one multi-row GEMV
             * (per row the same arithmetic as a single-row call) */
            float* o_all = (float*)malloc((size_t)S * K * H * sizeof(float));
            int* rows = (int*)malloc((size_t)S * K * sizeof(int));
            uint16_t* xg = (uint16_t*)malloc((size_t)S * K * H * 2);
            float* ga = (float*)malloc((size_t)S * K * I * 4);
            float* gb = (float*)malloc((size_t)S * K * I * 4);
            uint16_t* mid = (uint16_t*)malloc((size_t)S * K * I * 2);
            float* og = (float*)malloc((size_t)S * K * H * 4);
            for (int e = 0; e < E; e++) {
                int n_e = 0;
                for (int j = 0; j < S * K; j++)
                    if (idx_all[j] == e) rows[n_e++] = j;
                if (!n_e) continue;
                for (int r = 0; r < n_e; r++)
                    memcpy(xg + (size_t)r * H, xn + (size_t)(rows[r] / K) * H, (size_t)H * 2);
                orc_gemv_int4(xg, L->ew1[e].p, L->ew1[e].s, ga, n_e, I, H);
                orc_gemv_int4(xg, L->ew3[e].p, L->ew3[e].s, gb, n_e, I, H);
                orc_swiglu(ga, gb, mid, n_e * I);
                orc_gemv_int4(mid, L->ew2[e].p, L->ew2[e].s, og, n_e, H, I);
                for (int r = 0; r < n_e; r++)
                    memcpy(o_all + (size_t)rows[r] * H, og + (size_t)r * H, (size_t)H * 4);
            }
            for (int i = 0; i < S; i++)
                for (int t = 0; t < K; t++)  /* acc_scaled in rank order, engine.cu:901 */
                    orc_acc_scaled(acc + (size_t)i * H, o_all + ((size_t)i * K + t) * H, w_all[i * K + t], H);
            free(idx_all); free(w_all); free(o_all); free(rows); free(xg); free(ga); free(gb); free(mid); free(og);
            orc_add_inplace(hs, acc, S * H);
            moe_i++;
        }
    }
    memcpy(s->h, hs + (size_t)(S - 1) * H, (size_t)H * 2);
    orc_rmsnorm(s->h, m->emb_norm, xn, 1, H, eps);
    float* lg = (float*)malloc((size_t)c->vocab * 4);
    orc_gemv_fp16(xn, m->embed, lg, 1, c->vocab, H);
    int next = orc_argmax(lg, c->vocab);
    if (logits_out) memcpy(logits_out, lg, (size_t)c->vocab * 4);
    free(lg);
    s->pos += S;
    free(hs); free(xn); free(q16); free(k16); free(v16); free(ao); free(t16); free(t16b);
    free(acc); free(fa); free(fb); free(pos);
    return next;
}

void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int orc_get_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
