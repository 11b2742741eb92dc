// k_router.cu — fused MoE router + token->expert permutation (sm_100a).
//
// One block per token runs the reference's stateful EDA router (build_moe,
// src/zonos2-graph.cpp:199-220): ffn_norm, down projection + bias, + previous MoE
// layer's state * eda_scale, RMSNorm, two erf-GELU layers, expert logits (+ mask),
// softmax, top-k over probs + balancing bias, route weight = probs[sel] (no
// renormalisation). The last block to finish (atomic ticket, no spinning) builds the
// expert segments: routes sorted by expert, then by token, then by rank within the
// token's top-k, so the permutation is a pure function of the selected ids.
#include "common.cuh"
#include "kernels.h"

namespace z2b {

namespace {

__device__ __forceinline__ float gelu_erf(float x) {
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f));
}

// y[i] = sum_j W[i][j] x[j] for i < rows (W row-major f32), one warp per row.
__device__ __forceinline__ void block_matvec(const float* __restrict__ W, const float* x, float* y,
                                             int rows, int cols) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int i = w; i < rows; i += nw) {
        const float* wr = W + (size_t)i * cols;
        float acc = 0.0f;
        for (int j = lane; j < cols; j += 32) acc += wr[j] * x[j];
        acc = warp_sum(acc);
        if (lane == 0) y[i] = acc;
    }
}

// Expert segments from the selected ids: routes sorted by expert, then token, then rank
// in the token's top-k. Called by one whole block; cnt is a [MAX_EXPERTS] shared array.
__device__ void build_segments(const int* sel, const float* selw, int T, int k, int kmax, int E, int* cnt,
                               int* seg_off, int* active, int* n_active, int* route_tok, float* route_w,
                               int* route_pos) {
    for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    const int R = T * k;
    for (int r = threadIdx.x; r < R; r += blockDim.x) {
        const int e = __ldcg(sel + (r / k) * kmax + r % k);
        if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int off = 0, na = 0;
        for (int e = 0; e < E; ++e) {
            seg_off[e] = off;
            if (cnt[e] > 0) active[na++] = e;
            off += cnt[e];
        }
        seg_off[E] = off;
        *n_active = na;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int e = w; e < E; e += nw) {
        if (cnt[e] == 0) continue;
        int p = seg_off[e];
        for (int base = 0; base < R; base += 32) {
            const int r = base + lane;
            const int se = r < R ? __ldcg(sel + (r / k) * kmax + r % k) : -1;
            const unsigned m = __ballot_sync(0xffffffffu, se == e);
            if (se == e) {
                const int pos = p + __popc(m & ((1u << lane) - 1u));
                const int tt = r / k, jj = r % k;
                route_tok[pos] = tt;
                route_w[pos] = __ldcg(selw + tt * kmax + jj);
                route_pos[tt * kmax + jj] = pos;
            }
            p += __popc(m);
        }
    }
    __syncthreads();
}

__global__ void __launch_bounds__(256) router_kernel(const StepBufs b, const LayerSmall ly, const Dims dm,
                                                     int first_moe, int T, int layer) {
    extern __shared__ float sh[];
    const int d = dm.n_embd, rd = dm.rd, t = blockIdx.x;
    const int E = ly.is_moe ? ly.n_expert : 1, k = ly.is_moe ? ly.top_k : 1;
    float* xs = sh;                 // [d]
    float* rh = xs + d;             // [rd]
    float* rn = rh + rd;            // [rd]
    float* h0 = rn + rd;            // [rd]
    float* pr = h0 + rd;            // [E]
    float* red = pr + MAX_EXPERTS;  // [32]
    __shared__ int s_last;
    __shared__ int cnt[MAX_EXPERTS];
    const bool active = b.tok_slot[t] >= 0;

    // ffn_norm -> cur (f16 for the experts) and xs (f32 for the router)
    const float* res = b.res + (size_t)t * d;
    float ss = 0.0f;
    for (int j = threadIdx.x; j < d; j += blockDim.x) ss += res[j] * res[j];
    ss = block_sum(ss, red);
    const float sc = 1.0f / sqrtf(ss / (float)d + dm.rms_eps);
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
        const float v = (res[j] * sc) * ly.ffn_norm[j];
        xs[j] = v;
        b.cur[(size_t)t * d + j] = __float2half_rn(v);
    }
    for (int j = threadIdx.x; j < b.kmax; j += blockDim.x) b.route_pos[t * b.kmax + j] = -1;
    __syncthreads();

    if (ly.is_moe) {
        block_matvec(ly.rdown_w, xs, rh, rd, d);
        __syncthreads();
        for (int i = threadIdx.x; i < rd; i += blockDim.x) {
            float v = rh[i] + ly.rdown_b[i];
            if (ly.eda && !first_moe) v = v + b.rstate[(size_t)t * rd + i] * ly.eda[i];
            rh[i] = v;
            b.rstate[(size_t)t * rd + i] = v;
        }
        __syncthreads();
        float s2 = 0.0f;
        for (int i = threadIdx.x; i < rd; i += blockDim.x) s2 += rh[i] * rh[i];
        s2 = block_sum(s2, red);
        const float sc2 = 1.0f / sqrtf(s2 / (float)rd + dm.rms_eps);
        for (int i = threadIdx.x; i < rd; i += blockDim.x) rn[i] = (rh[i] * sc2) * ly.rnorm[i];
        __syncthreads();
        block_matvec(ly.m0_w, rn, h0, rd, rd);
        __syncthreads();
        for (int i = threadIdx.x; i < rd; i += blockDim.x) h0[i] = gelu_erf(h0[i] + ly.m0_b[i]);
        __syncthreads();
        block_matvec(ly.m2_w, h0, rn, rd, rd);        // rn reused as h2
        __syncthreads();
        for (int i = threadIdx.x; i < rd; i += blockDim.x) rn[i] = gelu_erf(rn[i] + ly.m2_b[i]);
        __syncthreads();
        block_matvec(ly.m4_w, rn, pr, E, rd);
        __syncthreads();
        if (threadIdx.x == 0) {
            // softmax (ggml: sum in double, scale by the rounded reciprocal)
            if (ly.rmask) for (int e = 0; e < E; ++e) pr[e] = pr[e] + ly.rmask[e];
            float mx = -INFINITY;
            for (int e = 0; e < E; ++e) mx = fmaxf(mx, pr[e]);
            double sum = 0.0;
            for (int e = 0; e < E; ++e) { const float v = expf(pr[e] - mx); pr[e] = v; sum += (double)v; }
            const float inv = (float)(1.0 / sum);
            for (int e = 0; e < E; ++e) pr[e] = pr[e] * inv;
            // top-k over probs + bias (+ mask), ties to the lower expert id
            unsigned long long taken[MAX_EXPERTS / 64] = {0};
            for (int j = 0; j < k; ++j) {
                int best = -1; float bv = -INFINITY;
                for (int e = 0; e < E; ++e) {
                    if (taken[e >> 6] >> (e & 63) & 1ull) continue;
                    float sv = pr[e] + ly.rbias[e];
                    if (ly.rmask) sv = sv + ly.rmask[e];
                    if (best < 0 || sv > bv) { bv = sv; best = e; }
                }
                taken[best >> 6] |= 1ull << (best & 63);
                b.sel[t * b.kmax + j] = active ? best : -1;
                b.selw[t * b.kmax + j] = pr[best];
            }
        }
    } else if (threadIdx.x == 0) {
        b.sel[t * b.kmax] = active ? 0 : -1;
        b.selw[t * b.kmax] = 1.0f;
    }

    if (b.sel_log && threadIdx.x == 0)
        for (int j = 0; j < k; ++j) b.sel_log[((size_t)layer * b.sel_log_T + t) * b.kmax + j] = b.sel[t * b.kmax + j];

    // ---- last block: expert segments ----
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = (atomicAdd(b.ticket, 1) == T - 1) ? 1 : 0;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    build_segments(b.sel, b.selw, T, k, b.kmax, E, cnt, b.seg_off, b.active, b.n_active, b.route_tok, b.route_w,
                   b.route_pos);
    if (threadIdx.x == 0) {
        if (b.layer_active) b.layer_active[layer] = *b.n_active;
        *b.ticket = 0;
    }
}

__global__ void route_test_kernel(const int* sel, const float* selw, int T, int k, int E, int* seg_off, int* active,
                                  int* n_active, int* route_tok, float* route_w, int* route_pos) {
    __shared__ int cnt[MAX_EXPERTS];
    build_segments(sel, selw, T, k, k, E, cnt, seg_off, active, n_active, route_tok, route_w, route_pos);
}

}  // namespace

void launch_router(const StepBufs& b, const LayerSmall& ly, const Dims& d, int T, int first_moe, int layer,
                   cudaStream_t s) {
    const size_t smem = (size_t)(d.n_embd + 3 * d.rd + MAX_EXPERTS + 32) * sizeof(float);
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
        configured = true;
    }
    router_kernel<<<T, 256, smem, s>>>(b, ly, d, first_moe, T, layer);
}

}  // namespace z2b

extern "C" int z2b_test_route(const int32_t* sel, const float* selw, int T, int k, int E, int32_t* seg_off,
                              int32_t* route_tok, int32_t* route_pos) {
    using namespace z2b;
    if (T < 1 || k < 1 || E < 1 || E > MAX_EXPERTS) return 1;
    int *dsel = nullptr, *dseg = nullptr, *dact = nullptr, *dna = nullptr, *dtok = nullptr, *dpos = nullptr;
    float *dw = nullptr, *drw = nullptr;
    int rc = 0;
    const size_t R = (size_t)T * k;
    if (cudaMalloc(&dsel, R * 4) || cudaMalloc(&dw, R * 4) || cudaMalloc(&dseg, (E + 1) * 4) ||
        cudaMalloc(&dact, E * 4) || cudaMalloc(&dna, 4) || cudaMalloc(&dtok, R * 4) || cudaMalloc(&drw, R * 4) ||
        cudaMalloc(&dpos, R * 4)) rc = 4;
    if (!rc) {
        cudaMemcpy(dsel, sel, R * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(dw, selw, R * 4, cudaMemcpyHostToDevice);
        cudaMemset(dpos, 0xff, R * 4);
        route_test_kernel<<<1, 256>>>(dsel, dw, T, k, E, dseg, dact, dna, dtok, drw, dpos);
        if (cudaMemcpy(seg_off, dseg, (E + 1) * 4, cudaMemcpyDeviceToHost) ||
            cudaMemcpy(route_tok, dtok, R * 4, cudaMemcpyDeviceToHost) ||
            cudaMemcpy(route_pos, dpos, R * 4, cudaMemcpyDeviceToHost)) rc = 4;
    }
    cudaFree(dsel); cudaFree(dw); cudaFree(dseg); cudaFree(dact); cudaFree(dna); cudaFree(dtok); cudaFree(drw);
    cudaFree(dpos);
    return rc;
}
