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

// One warp per token; n_exp <= 32*8, topk <= 32.  idx/w receive the topk
// choices: lane t keeps slot t's expert and sigmoid in registers and writes
// both once the sum is known (no read-back of w from global memory).
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
    int my_idx = 0;
    float my_w = 0.f;
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
        if (lane == t) {
            my_idx = be;
            my_w = sv;
        }
    }
    if (lane < topk) {
        idx[lane] = my_idx;
        w[lane] = my_w / (wsum + 1e-6f);
    }
    __syncwarp();
}

// Block-wide selection by rank, for E <= blockDim.x (all threads call it):
// expert e is picked in slot rank(e) = #{e' : s' > s, or s' == s and e' < e}
// when that rank is below topk, which is the order of the reference's
// repeated strict-'>' scan.  Scores that are NaN or <= -1e30 rank last (by
// index), as the scan never picks them before the smallest unused index.
// Weights are the unbiased sigmoids over (their sum in slot order + 1e-6).
// scratch: 2*E floats of shared memory.  Ends with a block barrier.
// trace_kernel: phase-trace kernel id that receives mark 10 after the
// sigmoids (diagnostic builds only; -1 = none).
__device__ __forceinline__ void route_select_block(const float* logits, const __half* bias, int n_exp, int topk,
                                                   int* idx, float* w, float* scratch, int trace_kernel = -1) {
    const int e = threadIdx.x;
    if (n_exp <= 32) {  // one warp: the keys travel by shuffle, one block barrier
        if (e < 32) {
            float sig = 0.f, key = -INFINITY;
            if (e < n_exp) {
                sig = route_sigmoid_call(logits[e]);
                const float score = sig + __half2float(bias[e]);
                key = (score > -1e30f) ? score : -INFINITY;
            }
            if (trace_kernel >= 0) PHASE(trace_kernel, 10);
            int rank = 0;  // 32 independent shuffles, unrolled so they pipeline
#pragma unroll
            for (int o = 0; o < 32; o++) {
                const float ko = __shfl_sync(0xffffffffu, key, o);
                rank += (o < n_exp && (ko > key || (ko == key && o < e))) ? 1 : 0;
            }
            if (e < n_exp && rank < topk) {
                idx[rank] = e;
                scratch[rank] = sig;
            }
            __syncwarp();
            if (e == 0) {
                float wsum = 0.f;
                for (int t = 0; t < topk; t++) wsum += scratch[t];
                for (int t = 0; t < topk; t++) w[t] = scratch[t] / (wsum + 1e-6f);
            }
        }
        __syncthreads();
        return;
    }
    float* sc = scratch;
    float* sg = scratch + n_exp;
    float sig = 0.f, key = -INFINITY;
    if (e < n_exp) {
        sig = route_sigmoid_call(logits[e]);
        const float score = sig + __half2float(bias[e]);
        key = (score > -1e30f) ? score : -INFINITY;  // NaN compares false
        sc[e] = key;
    }
    __syncthreads();
    if (e < n_exp) {
        int rank = 0;
        for (int o = 0; o < n_exp; o++) {
            const float ko = sc[o];
            rank += (ko > key || (ko == key && o < e)) ? 1 : 0;
        }
        if (rank < topk) {
            idx[rank] = e;
            sg[rank] = sig;
        }
    }
    __syncthreads();
    if (e == 0) {
        float wsum = 0.f;
        for (int t = 0; t < topk; t++) wsum += sg[t];
        for (int t = 0; t < topk; t++) w[t] = sg[t] / (wsum + 1e-6f);
    }
    __syncthreads();
}
