// MoE routing on the device, following the host loop of src/engine.cu:883-892.
#pragma once
#include "common.cuh"

// sigmoid as the reference's host computes it: 1.f / (1.f + expf(-z)) in
// float, with expf evaluated in double and rounded once to float.
__device__ __forceinline__ float route_sigmoid(float z) {
    float e = (float)exp(-(double)z);
    return 1.0f / (1.0f + e);
}
// One out-of-line copy: the double-precision exp is long code, and the
// selection below calls it from an unrolled loop.
static __device__ __noinline__ float route_sigmoid_call(float z) { return route_sigmoid(z); }

// One warp per token; n_exp <= 32*8.  idx/w receive the topk choices
// (written by lane 0; w is normalised in place at the end).
__device__ __forceinline__ void route_select_warp(const float* logits, const __half* bias, int n_exp, int topk,
                                                  int* idx, float* w) {
    const int lane = threadIdx.x & 31;
    float sig[8], score[8];
    bool used[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        int e = lane + 32 * j;
        used[j] = e >= n_exp;
        sig[j] = 0.f;
        score[j] = -INFINITY;
        if (e < n_exp) {
            sig[j] = route_sigmoid_call(logits[e]);
            score[j] = sig[j] + __half2float(bias[e]);
        }
    }
    float wsum = 0.f;  // summed in selection order, as the reference does
#pragma unroll 1
    for (int t = 0; t < topk; t++) {
        // max score, lowest index on ties (the reference scans e ascending with '>')
        float bv = -1e30f;
        int be = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            int e = lane + 32 * j;
            if (!used[j] && score[j] > bv) { bv = score[j]; be = e; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            int oe = __shfl_xor_sync(0xffffffffu, be, o);
            if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; }
        }
        if (be == 0x7fffffff) {
            // no candidate above -1e30 (NaN logits): take the smallest unused
            // index so the id is always a valid expert
            int cand = 0x7fffffff;
#pragma unroll
            for (int j = 0; j < 8; j++)
                if (!used[j]) cand = min(cand, lane + 32 * j);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) cand = min(cand, __shfl_xor_sync(0xffffffffu, cand, o));
            be = cand;
        }
        float sv = 0.f;
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (lane + 32 * j == be) { used[j] = true; sv = sig[j]; }
        sv = __shfl_sync(0xffffffffu, sv, be & 31);
        wsum += sv;
        if (lane == 0) {
            idx[t] = be;
            w[t] = sv;
        }
    }
    if (lane == 0)
        for (int t = 0; t < topk; t++) w[t] = w[t] / (wsum + 1e-6f);
    __syncwarp();
}
