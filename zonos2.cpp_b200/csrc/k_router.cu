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
#include "launch.cuh"
#include "../../include/z2b.h"
#include "../../include/z2b_tools.h"

#include <atomic>
#include <string>

namespace z2b {

namespace {

__device__ __forceinline__ float gelu_erf(float x) {
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f));
}

// y[i] = sum_j W[i][j] x[j] for i < rows (W row-major f32, x in shared memory): one warp
// per row group, every row's loads issued together (cols a multiple of 4).
__device__ __forceinline__ void block_matvec(const float* __restrict__ W, const float* x, float* y,
                                             int rows, int cols) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int c4 = cols / 4;
    for (int i0 = w; i0 < rows; i0 += 4 * nw) {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int j = lane; j < c4; j += 32) {
            const float4 xv = reinterpret_cast<const float4*>(x)[j];
            float4 wv[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int row = i0 + r * nw;
                wv[r] = row < rows ? reinterpret_cast<const float4*>(W + (size_t)row * cols)[j]
                                   : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[r] += wv[r].x * xv.x + wv[r].y * xv.y + wv[r].z * xv.z + wv[r].w * xv.w;
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const float a = warp_sum(acc[r]);
            const int row = i0 + r * nw;
            if (lane == 0 && row < rows) y[row] = a;
        }
    }
}

// Expert segments from the selected ids. Called by one whole block; cnt is a
// [MAX_EXPERTS] shared array. Routes are grouped by expert; within an expert, the routes
// for the tile GEMV come first (from seg_off[e]) and the routes for the tensor-core GEMM
// follow (from seg_mid[e]), each part ordered by token, then rank in the token's top-k.
// Which part a route joins depends on bulk_mode:
//   0: none take the GEMM;
//   1: all routes of an expert with >= gemm_min routes (the isolated expert op);
//   2: the routes of prompt rows (tokens whose descriptor feeds more than one row) of
//      experts with >= GEMM_MIN_PROMPT_ROUTES such routes (the decode step); an expert
//      with fewer takes them in its GEMV pass, which streams its weights anyway. Decode
//      rows always take the GEMV, and the choice for prompt rows depends on the step's
//      prompt routes only, so packing decode streams into a step never changes a result.
// active[0, n_small) lists the experts with GEMV routes, active[n_small, n_active) those
// with GEMM routes (an expert can be in both). tile_off (optional): prefix over the GEMV
// list of ceil(routes / 8).
// Up to st_cap routes (the caller's shared-memory staging area: st_se / st_sw, 8 bytes per
// route) are read from global memory once, in one pass, and placed from shared memory;
// larger steps read them again per expert, which costs a dependent global round trip per
// 32 routes and expert.
__device__ void build_segments(const int* sel, const float* selw, int T, int k, int kmax, int E, int* cnt,
                               int* seg_off, int* seg_mid, int* active, int* n_active, int* route_tok,
                               float* route_w, int* route_pos, int* tile_off, int* n_small, int bulk_mode,
                               const int* tok_desc, const SlotDesc* descs, int* s_se, float* s_sw, int st_cap,
                               int gemm_min = GEMM_MIN_TOKENS) {
    __shared__ int cntb[MAX_EXPERTS];
    __shared__ int s_off[MAX_EXPERTS];
    auto tok_bulk = [&](int t) -> bool {
        return bulk_mode == 2 && descs[tok_desc[t]].n_new > 1;
    };
    const int R = T * k;
    const bool staged = R <= st_cap;                 // s_se: expert | GEMM-part flag << 16, or -1
    for (int e = threadIdx.x; e < E; e += blockDim.x) { cnt[e] = 0; cntb[e] = 0; }
    __syncthreads();
    for (int r = threadIdx.x; r < R; r += blockDim.x) {
        const int t = r / k, j = r % k;
        int e = __ldcg(sel + t * kmax + j);
        const float w = staged ? __ldcg(selw + t * kmax + j) : 0.0f;
        const bool bk = tok_bulk(t);
        if (e >= 0 && e < E) {
            atomicAdd(&cnt[e], 1);
            if (bk) atomicAdd(&cntb[e], 1);
        } else {
            e = -1;
        }
        if (staged) { s_se[r] = e < 0 ? -1 : (e | (bk ? 1 << 16 : 0)); s_sw[r] = w; }
    }
    __syncthreads();
    if (bulk_mode == 1)
        for (int e = threadIdx.x; e < E; e += blockDim.x) cntb[e] = cnt[e] >= gemm_min ? cnt[e] : 0;
    if (bulk_mode == 2)
        for (int e = threadIdx.x; e < E; e += blockDim.x) if (cntb[e] < GEMM_MIN_PROMPT_ROUTES) cntb[e] = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (w == 0) {
        // lane owns experts [PER lane, PER lane + PER): exclusive scans over lanes of the
        // routes, GEMV experts, GEMV tiles and GEMM experts
        constexpr int PER = MAX_EXPERTS / 32;
        int c[PER], cb[PER];
        int off = 0, na = 0, tiles = 0, nb = 0;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            const int e = PER * lane + i;
            c[i] = e < E ? cnt[e] : 0;
            cb[i] = e < E ? cntb[e] : 0;
            off += c[i];
            na += c[i] - cb[i] > 0;
            tiles += (c[i] - cb[i] + 7) / 8;
            nb += cb[i] > 0;
        }
        int x_off = off, x_na = na, x_tiles = tiles, x_nb = nb;   // inclusive scans
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int a0 = __shfl_up_sync(0xffffffffu, x_off, o), a1 = __shfl_up_sync(0xffffffffu, x_na, o);
            const int a2 = __shfl_up_sync(0xffffffffu, x_tiles, o), a3 = __shfl_up_sync(0xffffffffu, x_nb, o);
            if (lane >= o) { x_off += a0; x_na += a1; x_tiles += a2; x_nb += a3; }
        }
        const int tot_off = __shfl_sync(0xffffffffu, x_off, 31), tot_na = __shfl_sync(0xffffffffu, x_na, 31);
        const int tot_tiles = __shfl_sync(0xffffffffu, x_tiles, 31);
        off = x_off - off; na = x_na - na; tiles = x_tiles - tiles; nb = tot_na + x_nb - nb;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            const int e = PER * lane + i;
            if (e >= E) break;
            seg_off[e] = off;
            s_off[e] = off;
            if (seg_mid) seg_mid[e] = off + c[i] - cb[i];
            off += c[i];
            if (c[i] - cb[i] > 0) {
                if (tile_off) tile_off[na] = tiles;
                tiles += (c[i] - cb[i] + 7) / 8;
                active[na++] = e;
            }
            if (cb[i] > 0) active[nb++] = e;
        }
        if (lane == 31) {
            seg_off[E] = tot_off;
            if (tile_off) tile_off[tot_na] = tot_tiles;
            if (n_small) *n_small = tot_na;
            *n_active = nb;
        }
    }
    __syncthreads();
    for (int e = w; e < E; e += nw) {
        if (cnt[e] == 0) continue;
        for (int part = 0; part < 2; ++part) {
            // part 0: GEMV routes from seg_off[e]; part 1: GEMM routes from the middle
            int p = part == 0 ? s_off[e] : s_off[e] + cnt[e] - cntb[e];
            if (part == 1 && cntb[e] == 0) break;
            for (int base = 0; base < R; base += 32) {
                const int r = base + lane;
                int se;
                bool bk;
                if (staged) {
                    const int v = r < R ? s_se[r] : -1;
                    se = v < 0 ? -1 : (v & 0xffff);
                    bk = v >= 0 && (v >> 16) != 0;
                } else {
                    se = r < R ? __ldcg(sel + (r / k) * kmax + r % k) : -1;
                    bk = se == e && bulk_mode == 2 && tok_bulk(r / k);
                }
                if (se == e && bulk_mode != 0) {
                    const bool b = cntb[e] > 0 && (bulk_mode == 1 || bk);
                    if (b != (part == 1)) se = -1;
                }
                const unsigned m = __ballot_sync(0xffffffffu, se == e);
                if (se == e) {
                    const int pos = p + __popc(m & ((1u << lane) - 1u));
                    const int tt = r / k, jj = r % k;
                    route_tok[pos] = tt;
                    route_w[pos] = staged ? s_sw[r] : __ldcg(selw + tt * kmax + jj);
                    route_pos[tt * kmax + jj] = pos;
                }
                p += __popc(m);
            }
        }
    }
    __syncthreads();
}

// Router down projection, split over (row block of 8, K slice of d/4, group of 16
// tokens). The weights are static, so each block dequantises its 8 x d/4 slice into
// shared memory (w = q * d exactly in f32 for Q8_0) before waiting on the step's
// predecessor. After the wait it stages u = res * ffn_norm for its tokens and writes
// the partial dot products sum_k w[r][k] * u[t][k]; the token's RMS scale is applied
// once to the summed partials in router_mlp_kernel (rh = Wd . (res * s * ffn_norm)).
constexpr int RP_ROWS = 8, RP_TOK = 16;
__host__ __device__ inline int router_kslices(int d) { return d % 128 == 0 ? 4 : 1; }

__global__ void __launch_bounds__(256) router_proj_kernel(const StepBufs b, const LayerSmall ly, const Dims dm, int T) {
    extern __shared__ __align__(16) float sh[];
    const int d = dm.n_embd, rd = dm.rd, L = d / router_kslices(d), S = L + 4, H = L / 2;
    const int rb = blockIdx.x, ks = blockIdx.y, t0 = blockIdx.z * RP_TOK, k0 = ks * L;
    float* xs = sh;                          // [RP_TOK][S]: k < H at k, k >= H at k + 4
    float* ws = xs + RP_TOK * S;             // [RP_ROWS][S], same split
    float* fn = ws + RP_ROWS * S;            // [L]
    auto at = [&](int k) { return k < H ? k : k + 4; };
    for (int i = threadIdx.x; i < RP_ROWS * L / 4; i += blockDim.x) {
        const int r = (4 * i) / L, kk = (4 * i) % L, row = rb * RP_ROWS + r;
        float4 v;
        if (ly.rdown_q) {
            const char4 q = *reinterpret_cast<const char4*>(ly.rdown_q + (size_t)row * d + k0 + kk);
            const float dv = ly.rdown_qd[(size_t)row * (d / 32) + (k0 + kk) / 32];
            v = make_float4((float)q.x * dv, (float)q.y * dv, (float)q.z * dv, (float)q.w * dv);
        } else {
            v = *reinterpret_cast<const float4*>(ly.rdown_w + (size_t)row * d + k0 + kk);
        }
        *reinterpret_cast<float4*>(ws + r * S + at(kk)) = v;
    }
    for (int i = threadIdx.x; i < L / 4; i += blockDim.x)
        reinterpret_cast<float4*>(fn)[i] = reinterpret_cast<const float4*>(ly.ffn_norm + k0)[i];
    pdl_wait();
    __syncthreads();                         // fn (and ws) written by other threads
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int tt = warp; tt < RP_TOK; tt += nw) {
        const int t = t0 + tt;
        for (int j = lane; j < L / 4; j += 32) {
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (t < T) v = *reinterpret_cast<const float4*>(b.res + (size_t)t * d + k0 + 4 * j);
            const float4 f = reinterpret_cast<const float4*>(fn)[j];
            *reinterpret_cast<float4*>(xs + tt * S + at(4 * j)) = make_float4(v.x * f.x, v.y * f.y, v.z * f.z, v.w * f.w);
        }
    }
    __syncthreads();
    // warp -> row, lane -> (token lane & 15, half lane >> 4)
    const int tt = lane & 15, h = lane >> 4;
    for (int r = warp; r < RP_ROWS; r += nw) {
        const float* xr = xs + tt * S + h * (H + 4);
        const float* wr = ws + r * S + h * (H + 4);
        float acc = 0.0f;
        for (int j = 0; j < H; j += 4) {
            const float4 xv = *reinterpret_cast<const float4*>(xr + j);
            const float4 wv = *reinterpret_cast<const float4*>(wr + j);
            acc += wv.x * xv.x + wv.y * xv.y + wv.z * xv.z + wv.w * xv.w;
        }
        acc += __shfl_xor_sync(0xffffffffu, acc, 16);
        if (h == 0 && t0 + tt < T) b.rpart[((size_t)ks * b.rpart_T + t0 + tt) * rd + rb * RP_ROWS + r] = acc;
    }
    pdl_release();
}

// One block per token (512 threads): ffn_norm (src/zonos2-graph.cpp:347) -> cur (f16
// for the experts); rh = s * sum of the router_proj partials + b (+ previous MoE layer's
// state * eda_scale), which becomes the next MoE layer's state (:199-203); RMSNorm(rh) *
// router_norm, two erf-GELU layers, expert logits (+ mask), softmax, top-k on probs +
// balancing bias (+ mask), route weight = probs[sel] with no renormalisation
// (:206-220). The MLP weights are static: when they fit, one bulk copy per matrix brings
// them into shared memory before the wait on router_proj. The last block to finish
// builds the expert segments.
__global__ void __launch_bounds__(512) router_mlp_kernel(const StepBufs b, const LayerSmall ly, const Dims dm,
                                                         int first_moe, int T, int layer, int stage, int seg_cap) {
    extern __shared__ __align__(128) float sh[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ float red[32];
    __shared__ int s_last;
    __shared__ int cnt[MAX_EXPERTS];
    const int d = dm.n_embd, rd = dm.rd, t = blockIdx.x;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int E = ly.is_moe ? ly.n_expert : 1, k = ly.is_moe ? ly.top_k : 1;
    const float* W0 = ly.m0_w;
    const float* W2 = ly.m2_w;
    const float* W4 = ly.m4_w;
    float* rh = sh;                  // [rd]
    float* rn = rh + rd;             // [rd]
    float* h0 = rn + rd;             // [rd]
    float* pr = h0 + rd;             // [MAX_EXPERTS]
    // static vectors, copied before the wait so no load of them sits on the critical path:
    // router_down bias | eda scale | router norm | mlp0 bias | mlp2 bias ([rd] each),
    // balancing bias | mask ([MAX_EXPERTS] each), ffn_norm [d]
    float* v_rdb = pr + MAX_EXPERTS;
    float* v_eda = v_rdb + rd;
    float* v_rnorm = v_eda + rd;
    float* v_m0b = v_rnorm + rd;
    float* v_m2b = v_m0b + rd;
    float* v_rbias = v_m2b + rd;
    float* v_rmask = v_rbias + MAX_EXPERTS;
    float* v_fn = v_rmask + MAX_EXPERTS;
    float* wst = v_fn + d;           // staged m0 [rd][rd], m2 [rd][rd], m4 [E][rd]
    const bool staged = ly.is_moe && stage;
    if (staged) {
        if (threadIdx.x == 0) {
            mbar_init(&bar, 1);
            fence_mbar_init();
            const uint32_t b0 = (uint32_t)(rd * rd * 4), b4 = (uint32_t)(E * rd * 4);
            mbar_expect_tx(&bar, 2 * b0 + b4);
            bulk_g2s(wst, ly.m0_w, b0, &bar);
            bulk_g2s(wst + rd * rd, ly.m2_w, b0, &bar);
            bulk_g2s(wst + 2 * rd * rd, ly.m4_w, b4, &bar);
        }
        W0 = wst;
        W2 = wst + rd * rd;
        W4 = wst + 2 * rd * rd;
    }
    for (int j = threadIdx.x; j < d / 4; j += blockDim.x)
        reinterpret_cast<float4*>(v_fn)[j] = reinterpret_cast<const float4*>(ly.ffn_norm)[j];
    if (ly.is_moe) {
        for (int i = threadIdx.x; i < rd; i += blockDim.x) {
            v_rdb[i] = ly.rdown_b[i];
            v_eda[i] = ly.eda ? ly.eda[i] : 0.0f;
            v_rnorm[i] = ly.rnorm[i];
            v_m0b[i] = ly.m0_b[i];
            v_m2b[i] = ly.m2_b[i];
        }
        for (int e = threadIdx.x; e < E; e += blockDim.x) {
            v_rbias[e] = ly.rbias[e];
            v_rmask[e] = ly.rmask ? ly.rmask[e] : 0.0f;
        }
    }
    const bool active = __ldcg(b.tok_slot + t) >= 0;        // packer output, complete before the predecessor
    pdl_wait();
    // the router projection's inputs load with the residual row: partial sums over the K
    // slices and the previous MoE layer's state
    float pa = 0.0f, pst = 0.0f;
    const bool eda_on = ly.is_moe && ly.eda && !first_moe;
    if (ly.is_moe && threadIdx.x < rd) {
        const int i = threadIdx.x;
        for (int ks = 0; ks < router_kslices(d); ++ks) pa += b.rpart[((size_t)ks * b.rpart_T + t) * rd + i];
        if (eda_on) pst = b.rstate[(size_t)t * rd + i];
    }

    // ffn_norm -> cur (f16)
    const float4* r4 = reinterpret_cast<const float4*>(b.res + (size_t)t * d);
    float ss = 0.0f;
    for (int j = threadIdx.x; j < d / 4; j += blockDim.x) { const float4 v = r4[j]; ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w; }
    ss = block_sum(ss, red);                                  // its barriers also publish the staged vectors
    const float sc = 1.0f / sqrtf(ss / (float)d + dm.rms_eps);
    for (int j = threadIdx.x; j < d / 4; j += blockDim.x) {
        const float4 r = r4[j];
        const float4 f = reinterpret_cast<const float4*>(v_fn)[j];
        __half2* o = reinterpret_cast<__half2*>(b.cur + (size_t)t * d) + 2 * j;
        o[0] = __floats2half2_rn((r.x * sc) * f.x, (r.y * sc) * f.y);
        o[1] = __floats2half2_rn((r.z * sc) * f.z, (r.w * sc) * f.w);
    }
    for (int j = threadIdx.x; j < b.kmax; j += blockDim.x) b.route_pos[t * b.kmax + j] = -1;

    bool ok = true;
    if (ly.is_moe) {
        if (threadIdx.x < rd) {
            const int i = threadIdx.x;
            float v = pa * sc + v_rdb[i];
            if (eda_on) v = v + pst * v_eda[i];
            rh[i] = v;
            b.rstate[(size_t)t * rd + i] = v;
        }
        __syncthreads();
        float s2 = 0.0f;
        for (int i = threadIdx.x; i < rd; i += blockDim.x) s2 += rh[i] * rh[i];
        s2 = block_sum(s2, red);
        const float sc2 = 1.0f / sqrtf(s2 / (float)rd + dm.rms_eps);
        for (int i = threadIdx.x; i < rd; i += blockDim.x) rn[i] = (rh[i] * sc2) * v_rnorm[i];
        if (staged) ok = mbar_wait(&bar, 0, b.err);
        __syncthreads();
        if (ok) {
            block_matvec(W0, rn, h0, rd, rd);
            __syncthreads();
            for (int i = threadIdx.x; i < rd; i += blockDim.x) h0[i] = gelu_erf(h0[i] + v_m0b[i]);
            __syncthreads();
            block_matvec(W2, h0, rn, rd, rd);        // rn reused as h2
            __syncthreads();
            for (int i = threadIdx.x; i < rd; i += blockDim.x) rn[i] = gelu_erf(rn[i] + v_m2b[i]);
            __syncthreads();
            block_matvec(W4, rn, pr, E, rd);
        }
        __syncthreads();
        if (w == 0 && ok) {
            // softmax (ggml: sum in double, scale by the rounded reciprocal), one warp: exp per
            // lane, the double sum over a fixed lane tree
            float mx = -INFINITY;
            for (int e = lane; e < E; e += 32) {
                if (ly.rmask) pr[e] = pr[e] + v_rmask[e];
                mx = fmaxf(mx, pr[e]);
            }
            mx = warp_max(mx);
            double sum = 0.0;
            for (int e = lane; e < E; e += 32) { const float v = expf(pr[e] - mx); pr[e] = v; sum += (double)v; }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            const float inv = (float)(1.0 / sum);
            for (int e = lane; e < E; e += 32) pr[e] = pr[e] * inv;
            __syncwarp();
            // top-k over probs + bias (+ mask), ties to the lower expert id: k rounds of
            // warp argmax; lane owns experts lane + 32 i
            float sv[MAX_EXPERTS / 32];
#pragma unroll
            for (int i = 0; i < MAX_EXPERTS / 32; ++i) {
                const int e = lane + 32 * i;
                float v = -INFINITY;
                if (e < E) {
                    v = pr[e] + v_rbias[e];
                    if (ly.rmask) v = v + v_rmask[e];
                }
                sv[i] = v;
            }
            unsigned taken = 0;
            for (int j = 0; j < k; ++j) {
                float bv = -INFINITY; int best = 0x7fffffff;
#pragma unroll
                for (int i = 0; i < MAX_EXPERTS / 32; ++i) {
                    const int e = lane + 32 * i;
                    if (e >= E || (taken >> i & 1u)) continue;
                    if (sv[i] > bv || (sv[i] == bv && e < best)) { bv = sv[i]; best = e; }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, best, o);
                    if (ov > bv || (ov == bv && oi < best)) { bv = ov; best = oi; }
                }
                if (best >= E) best = 0;              // all remaining scores -inf: keep a valid id
                if ((best & 31) == lane) taken |= 1u << (best >> 5);
                if (lane == 0) {
                    const int id = active ? best : -1;
                    b.sel[t * b.kmax + j] = id;
                    b.selw[t * b.kmax + j] = pr[best];
                    if (b.sel_log) b.sel_log[((size_t)layer * b.sel_log_T + t) * b.kmax + j] = id;
                }
            }
        }
        if (!ok && threadIdx.x < k) {                  // weights never arrived (error recorded)
            b.sel[t * b.kmax + threadIdx.x] = -1;
            b.selw[t * b.kmax + threadIdx.x] = 0.0f;
        }
    } else if (threadIdx.x == 0) {
        b.sel[t * b.kmax] = active ? 0 : -1;
        b.selw[t * b.kmax] = 1.0f;
    }
    __syncthreads();
    if (b.sel_log && !(ly.is_moe && ok) && threadIdx.x < k)   // dense layer, or the weights never arrived
        b.sel_log[((size_t)layer * b.sel_log_T + t) * b.kmax + threadIdx.x] = b.sel[t * b.kmax + threadIdx.x];

    pdl_release();
    // ---- last block: expert segments ----
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = (atomicAdd(b.ticket, 1) == T - 1) ? 1 : 0;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // the block's dynamic shared memory (MLP weights, vectors) is free now: it stages the routes
    build_segments(b.sel, b.selw, T, k, b.kmax, E, cnt, b.seg_off, b.seg_mid, b.active, b.n_active, b.route_tok,
                   b.route_w, b.route_pos, b.tile_off, b.n_small, ly.gemm_ok ? 2 : 0, b.tok_desc, b.descs,
                   reinterpret_cast<int*>(sh), sh + seg_cap, seg_cap);
    if (threadIdx.x == 0) {
        if (b.layer_active) b.layer_active[layer] = *b.n_active;
        *b.ticket = 0;
    }
}

__global__ void segments_kernel(const StepBufs b, int T, int k, int E, int bulk_mode, int seg_cap, int gemm_min) {
    extern __shared__ __align__(16) float seg_st[];  // [seg_cap] ids, then [seg_cap] weights
    __shared__ int cnt[MAX_EXPERTS];
    pdl_wait();
    pdl_release();
    for (int j = threadIdx.x; j < T * b.kmax; j += blockDim.x) b.route_pos[j] = -1;
    __syncthreads();
    build_segments(b.sel, b.selw, T, k, b.kmax, E, cnt, b.seg_off, b.seg_mid, b.active, b.n_active, b.route_tok,
                   b.route_w, b.route_pos, b.tile_off, b.n_small, bulk_mode, nullptr, nullptr,
                   reinterpret_cast<int*>(seg_st), seg_st + seg_cap, seg_cap, gemm_min);
}

__global__ void route_test_kernel(const int* sel, const float* selw, int T, int k, int E, int* seg_off, int* active,
                                  int* n_active, int* route_tok, float* route_w, int* route_pos) {
    constexpr int kStage = 2048;                     // routes staged in shared memory (static)
    __shared__ int cnt[MAX_EXPERTS];
    __shared__ int st_se[kStage];
    __shared__ float st_sw[kStage];
    build_segments(sel, selw, T, k, k, E, cnt, seg_off, nullptr, active, n_active, route_tok, route_w, route_pos,
                   nullptr, nullptr, 0, nullptr, nullptr, st_se, st_sw, kStage);
}

}  // namespace

constexpr int kMaxRouterDevices = 64;

size_t router_mlp_smem(const Dims& d, int E, bool* stage) {
    const size_t base = (size_t)(8 * d.rd + 3 * MAX_EXPERTS + d.n_embd) * sizeof(float);
    const size_t w = (size_t)(2 * d.rd * d.rd + E * d.rd) * sizeof(float);
    *stage = base + w <= 190 * 1024;
    return *stage ? base + w : base;
}

// The dynamic shared memory opt-in is a per-device function attribute: set it once on
// every device a context runs on (one process may drive several GPUs).
void router_attributes() {
    static std::atomic<bool> configured[kMaxRouterDevices];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxRouterDevices || !configured[dev].load(std::memory_order_acquire)) {
        cudaFuncSetAttribute(router_proj_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        cudaFuncSetAttribute(router_mlp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        cudaFuncSetAttribute(segments_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (dev >= 0 && dev < kMaxRouterDevices) configured[dev].store(true, std::memory_order_release);
    }
}

void launch_router(const StepBufs& b, const LayerSmall& ly, const Dims& d, int T, int first_moe, int layer,
                   cudaStream_t s) {
    router_attributes();
    if (ly.is_moe) {
        const int nks = router_kslices(d.n_embd), L = d.n_embd / nks, S = L + 4;
        const size_t smem = (size_t)((RP_TOK + RP_ROWS) * S + L) * sizeof(float);
        launch_pdl(router_proj_kernel, dim3(d.rd / RP_ROWS, nks, (T + RP_TOK - 1) / RP_TOK), dim3(256), smem, s,
                   b, ly, d, T);
    }
    bool stage = false;
    const size_t smem = router_mlp_smem(d, ly.is_moe ? ly.n_expert : 1, &stage);
    launch_pdl(router_mlp_kernel, dim3(T), dim3(512), smem, s, b, ly, d, first_moe, T, layer, stage ? 1 : 0,
               (int)(smem / 8));
}

int router_launches(const LayerSmall& ly) { return ly.is_moe ? 2 : 1; }

void launch_segments(const StepBufs& b, int T, int k, int E, int bulk_mode, cudaStream_t s, int gemm_min) {
    // every route staged in shared memory (8 bytes each, up to 24K routes)
    router_attributes();
    const int cap = std::min(T * k, 24 * 1024);
    launch_pdl(segments_kernel, dim3(1), dim3(1024), (size_t)cap * 8, s, b, T, k, E, bulk_mode, cap, gemm_min);
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

// ---------------------------------------------------------------- allocation-free variant
// z2b_route_segments_noalloc runs the same segment builder as z2b_test_route on a fixed
// device scratch area instead of buffers allocated per call. It is for callers that may
// not allocate device memory: a serving process that has handed all but a fixed budget of
// the GPU to its KV page pool, or a latency-critical thread, since cudaMalloc and cudaFree
// can synchronise the whole device and stall decode steps queued by other threads. The
// work runs on the calling thread's per-thread default stream, which does not join the
// streams of other threads or libraries. The scratch is one file-scope array, so calls
// that overlap on the GPU (from several host threads) race on it and must be serialised
// by the caller.
namespace z2b {
namespace {

constexpr int kNoAllocRoutes = Z2B_NOALLOC_MAX_ROUTES;
// [sel | selw | route_tok | route_w | route_pos] x kNoAllocRoutes, then seg_off
// [MAX_EXPERTS + 1], active [MAX_EXPERTS], n_active [1] (4-byte words)
constexpr size_t kNoAllocWords = 5 * (size_t)kNoAllocRoutes + 2 * MAX_EXPERTS + 2;
static __device__ __align__(256) uint32_t g_route_scratch[kNoAllocWords];

constexpr int kMaxDevices = 64;
uint32_t* g_route_scratch_ptr[kMaxDevices] = {};

}  // namespace
void set_error(const std::string& e);
}  // namespace z2b

extern "C" int z2b_route_segments_noalloc(const int32_t* sel, const float* selw, int T, int k, int E,
                                          int32_t* seg_off, int32_t* route_tok, int32_t* route_pos) {
    using namespace z2b;
    if (!sel || !selw || !seg_off || !route_tok || !route_pos) { set_error("null argument"); return Z2B_ERR_ARG; }
    if (T < 1 || k < 1 || E < 1 || E > MAX_EXPERTS) { set_error("route_segments_noalloc: bad T, k or E"); return Z2B_ERR_ARG; }
    if ((int64_t)T * k > kNoAllocRoutes) {
        set_error("route_segments_noalloc: T * k exceeds Z2B_NOALLOC_MAX_ROUTES (" +
                  std::to_string(kNoAllocRoutes) + ")");
        return Z2B_ERR_ARG;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        set_error("route_segments_noalloc: no usable current device");
        return Z2B_ERR_CUDA;
    }
    // set-up, once per device with that device current: the device address of the
    // scratch symbol (the host-side name of a __device__ array is not a device pointer)
    if (!g_route_scratch_ptr[dev]) {
        void* ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_route_scratch);
        if (e != cudaSuccess || !ptr) {
            set_error(std::string("route_segments_noalloc: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
            return Z2B_ERR_CUDA;
        }
        g_route_scratch_ptr[dev] = static_cast<uint32_t*>(ptr);
    }
    uint32_t* base = g_route_scratch_ptr[dev];
    int* dsel = reinterpret_cast<int*>(base);
    float* dw = reinterpret_cast<float*>(base + kNoAllocRoutes);
    int* dtok = reinterpret_cast<int*>(base + 2 * (size_t)kNoAllocRoutes);
    float* drw = reinterpret_cast<float*>(base + 3 * (size_t)kNoAllocRoutes);
    int* dpos = reinterpret_cast<int*>(base + 4 * (size_t)kNoAllocRoutes);
    int* dseg = reinterpret_cast<int*>(base + 5 * (size_t)kNoAllocRoutes);
    int* dact = dseg + MAX_EXPERTS + 1;
    int* dna = dact + MAX_EXPERTS;
    const size_t R = (size_t)T * k;
    cudaStream_t s = cudaStreamPerThread;
    bool ok = cudaMemcpyAsync(dsel, sel, R * 4, cudaMemcpyHostToDevice, s) == cudaSuccess &&
              cudaMemcpyAsync(dw, selw, R * 4, cudaMemcpyHostToDevice, s) == cudaSuccess &&
              // route_pos of routes with no expert stays -1; everything else is written
              cudaMemsetAsync(dpos, 0xff, R * 4, s) == cudaSuccess;
    if (ok) {
        route_test_kernel<<<1, 256, 0, s>>>(dsel, dw, T, k, E, dseg, dact, dna, dtok, drw, dpos);
        ok = cudaGetLastError() == cudaSuccess &&
             cudaMemcpyAsync(seg_off, dseg, (size_t)(E + 1) * 4, cudaMemcpyDeviceToHost, s) == cudaSuccess &&
             cudaMemcpyAsync(route_tok, dtok, R * 4, cudaMemcpyDeviceToHost, s) == cudaSuccess &&
             cudaMemcpyAsync(route_pos, dpos, R * 4, cudaMemcpyDeviceToHost, s) == cudaSuccess &&
             cudaStreamSynchronize(s) == cudaSuccess;
    }
    if (!ok) {
        set_error(std::string("route_segments_noalloc: ") + cudaGetErrorString(cudaGetLastError()));
        return Z2B_ERR_CUDA;
    }
    return Z2B_OK;
}
