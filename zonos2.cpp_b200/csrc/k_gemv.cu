// k_gemv.cu — tile GEMV for the decode step (sm_100a).
//
// Replaces ggml_mul_mat / ggml_mul_mat_id on quantised weights
// (src/zonos2-graph.cpp:107-111, 175, 181-184, 223-231, 357): the attention and head
// projections over all tokens of the step, and the grouped expert gate/up (+SwiGLU) and
// down (x route probability) passes over the tokens routed to each active expert.
//
// Work item = (matrix or expert, row-tile of 16 output rows). A CTA owns a contiguous
// run of items; its warps split each item's K range. Each warp streams its K-slice of
// every item through a private ring of shared-memory stages filled by one-lane
// cp.async.bulk copies (this CTA only), decodes the quantised weights in registers
// straight into mma.sync.m16n8k16 A fragments (tile_layout.h), multiplies them with the
// activation fragments (f16, 8 tokens per n-tile) and accumulates in f32. Partial sums
// are reduced across warps in shared memory in a fixed order, so results do not depend
// on timing, on the other tokens of the batch or on the grid size.
#include "common.cuh"
#include "gguf.h"
#include "kernels.h"
#include "launch.cuh"
#include "tile_layout.h"
#include "k_decode.cuh"

#include <algorithm>

namespace z2b {

namespace {

// unrolled k-step loop: decode one k-step of the tile, multiply with the first NTV token
// tiles (NTV is a compile-time count, so no branch guards the mma)
template <class D, int NTG, int s, int KS> struct KLoop {
    template <int NMAT, int NTV>
    __device__ __forceinline__ static void run(const D& dec, const uint8_t* T, int lane, int kbase,
                                               const uint32_t (&B)[NTG][MAXKS][2], float (&acc)[NMAT][NTG][4],
                                               int m) {
        uint32_t a[4];
        dec.template frag<s>(T, lane, a);
#pragma unroll
        for (int nt = 0; nt < NTV; ++nt)
            mma16816(acc[m][nt], a[0], a[1], a[2], a[3], B[nt][kbase + s][0], B[nt][kbase + s][1]);
        KLoop<D, NTG, s + 1, KS>::template run<NMAT, NTV>(dec, T, lane, kbase, B, acc, m);
    }
};
// gate/up variant of KLoop: both matrices' fragments per k-step, so the two accumulator
// chains interleave
template <class D, int NTG, int s, int KS> struct KLoop2 {
    template <int NTV>
    __device__ __forceinline__ static void run(const D& d0, const D& d1, const uint8_t* T0, const uint8_t* T1, int lane,
                                               int kbase, const uint32_t (&B)[NTG][MAXKS][2], float (&acc)[2][NTG][4]) {
        uint32_t a[4], c[4];
        d0.template frag<s>(T0, lane, a);
        d1.template frag<s>(T1, lane, c);
#pragma unroll
        for (int nt = 0; nt < NTV; ++nt) {
            mma16816(acc[0][nt], a[0], a[1], a[2], a[3], B[nt][kbase + s][0], B[nt][kbase + s][1]);
            mma16816(acc[1][nt], c[0], c[1], c[2], c[3], B[nt][kbase + s][0], B[nt][kbase + s][1]);
        }
        KLoop2<D, NTG, s + 1, KS>::template run<NTV>(d0, d1, T0, T1, lane, kbase, B, acc);
    }
};
template <class D, int NTG, int KS> struct KLoop2<D, NTG, KS, KS> {
    template <int NTV>
    __device__ __forceinline__ static void run(const D&, const D&, const uint8_t*, const uint8_t*, int, int,
                                               const uint32_t (&)[NTG][MAXKS][2], float (&)[2][NTG][4]) {}
};
template <class D, int NTG, int KS> struct KLoop<D, NTG, KS, KS> {
    template <int NMAT, int NTV>
    __device__ __forceinline__ static void run(const D&, const uint8_t*, int, int, const uint32_t (&)[NTG][MAXKS][2],
                                               float (&)[NMAT][NTG][4], int) {}
};

// Item = (segment or active expert s, row tile rt); a CTA walks a contiguous run of
// items, so positions advance by increment (no division per item).
struct ItemPos { int s, rt; };
struct ItemRef { int expert; int seg; int rt; const uint8_t* src[2]; int n_tok; int tok0; };

template <int MODE>
__device__ __forceinline__ ItemPos item_seek(const GemvParams& p, int item) {
    ItemPos q{0, 0};
    if constexpr (MODE == GM_PROJ) {
        int base = 0;
        while (q.s + 1 < p.n_seg && item >= base + p.seg[q.s].n_row_tiles) { base += p.seg[q.s].n_row_tiles; ++q.s; }
        q.rt = item - base;
    } else {
        q.s = item / p.n_row_tiles;
        q.rt = item - q.s * p.n_row_tiles;
    }
    return q;
}

template <int MODE>
__device__ __forceinline__ void item_next(const GemvParams& p, ItemPos& q) {
    const int nrt = (MODE == GM_PROJ) ? p.seg[q.s].n_row_tiles : p.n_row_tiles;
    if (++q.rt == nrt) { q.rt = 0; ++q.s; }
}

// The active expert of the last item resolved (expert id, first route, route count): a
// CTA's items change expert once per n_row_tiles items, so the dependent loads of
// active[] and the segment offsets are issued once per expert, not once per item.
struct ExpCache { int s = -1, expert = 0, tok0 = 0, n_tok = 0; };

template <int MODE>
__device__ __forceinline__ ItemRef item_ref(const GemvParams& p, ItemPos q, int c0, ExpCache& ec) {
    ItemRef r{};
    r.rt = q.rt;
    if constexpr (MODE == GM_PROJ) {
        r.seg = q.s; r.expert = -1;
        r.src[0] = p.seg[q.s].tiles + ((size_t)q.rt * p.chunks + c0) * p.tile_bytes;
        r.src[1] = nullptr;
        r.n_tok = p.T; r.tok0 = 0;
    } else {
        if (q.s != ec.s) {
            ec.s = q.s;
            ec.expert = p.active[q.s];
            ec.tok0 = p.seg_off[ec.expert];
            ec.n_tok = (p.seg_mid ? p.seg_mid[ec.expert] : p.seg_off[ec.expert + 1]) - ec.tok0;
        }
        r.expert = ec.expert;
        r.seg = 0;
        const size_t off = (size_t)r.expert * p.expert_stride + ((size_t)q.rt * p.chunks + c0) * p.tile_bytes;
        r.src[0] = p.w0 + off;
        r.src[1] = (MODE == GM_GATEUP) ? p.w1 + off : nullptr;
        r.tok0 = ec.tok0;
        r.n_tok = ec.n_tok;
    }
    return r;
}

template <int MODE>
__device__ __forceinline__ int x_row(const GemvParams& p, const ItemRef& it, int n) {
    if constexpr (MODE == GM_PROJ) return n;
    else if constexpr (MODE == GM_GATEUP) return p.route_tok[it.tok0 + n];
    else return it.tok0 + n;
}

// Token tiles per pass: 2 (up to 16 tokens) for the projections and gate/up, 1 for the
// down pass, whose lighter registers let three blocks share an SM (measured: gate/up
// keeps its two-stage ring at two blocks per SM; down gains from the third block).
template <int WT, int KSF, int MODE, int NTG, int MAXT, int MINB>
__global__ void __launch_bounds__(MAXT, MINB) gemv_kernel(const GemvParams p) {
    using D = typename DecSel<WT, KSF>::T;
    constexpr int KS = D::KS, KC = D::KC;
    constexpr int NMAT = (MODE == GM_GATEUP) ? 2 : 1;
    constexpr int MAXCPW = MAXKS / KS;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, NW = blockDim.x >> 5;
    const int q = lane & 3, r8 = lane >> 2;
    const int NS = p.n_stages;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);                         // [NW][NS]
    uint8_t* stages = smem + 128 * ((NW * NS * 8 + 127) / 128);                  // [NW][NS][stage_bytes]
    float* red = reinterpret_cast<float*>(stages + (size_t)NW * NS * p.stage_bytes);   // [2][NW][NMAT][NTG][32][4]
    // GM_PROJ: this warp's activation slice [8 NTG tokens][x_rs bytes]
    uint8_t* xw = reinterpret_cast<uint8_t*>(red + 2 * NW * NMAT * NTG * 128) + (size_t)warp * 8 * NTG * p.x_rs;
    uint64_t* mybar = bars + warp * NS;
    uint8_t* mystage = stages + (size_t)warp * NS * p.stage_bytes;

    const int c0 = warp * p.chunks / NW, c1 = (warp + 1) * p.chunks / NW, ncw = c1 - c0;
    const uint32_t wbytes = (uint32_t)(ncw * p.tile_bytes);

    if (lane == 0)
        for (int s = 0; s < NS; ++s) mbar_init(&mybar[s], 1);
    fence_mbar_init();
    __syncwarp();

    int it0 = 0, it1 = 0;
    ExpCache ec_issue, ec_use;                   // expert resolved by the copy issuer / the consumer
    int issued_upto = -1;                        // last item whose copy was issued
    ItemPos ipos{0, 0};                          // position of the next item to issue
    auto issue = [&](int item, int slot) {
        issued_upto = item;
        const ItemPos q = ipos;
        item_next<MODE>(p, ipos);
        if (lane == 0 && ncw > 0) {
            const ItemRef it = item_ref<MODE>(p, q, c0, ec_issue);
            mbar_expect_tx(&mybar[slot], wbytes * NMAT);
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
                bulk_g2s(mystage + slot * p.stage_bytes + m * wbytes, it.src[m], wbytes, &mybar[slot]);
        }
    };
    if constexpr (MODE == GM_PROJ) {
        // weights and the item list are static: start streaming before the predecessor ends
        it0 = (int)((int64_t)blockIdx.x * p.total_items / gridDim.x);
        it1 = (int)((int64_t)(blockIdx.x + 1) * p.total_items / gridDim.x);
        issued_upto = it0 - 1;
        ipos = item_seek<MODE>(p, it0);
        for (int i = 0; i < NS && it0 + i < it1; ++i) issue(it0 + i, i);
        pdl_wait();
    } else {
        pdl_wait();
        const int n_act = *p.n_active;
        const int n_items = n_act * p.n_row_tiles;
        it0 = (int)((int64_t)blockIdx.x * n_items / gridDim.x);
        it1 = (int)((int64_t)(blockIdx.x + 1) * n_items / gridDim.x);
        if (p.tile_off && n_act <= 32) {
            // Balanced split: an item of expert a costs W + (its 8-token tiles), fitted to
            // measured per-block times (an expert past 8 tokens takes a second 8-token pass in
            // the down GEMV, twice the n-tiles in gate/up); blocks take equal cost ranges, so
            // the blocks on heavily routed experts get fewer items. Warp 0 scans the experts'
            // tile prefix (tile_off, from the router) and finds this block's first and last
            // item; the result only moves items between blocks, never changes one.
            __shared__ int s_it[2];
            if (warp == 0) {
                constexpr int W = (MODE == GM_GATEUP) ? 2 : 1;
                const int nrt = p.n_row_tiles;
                const int t_lo = lane <= n_act ? p.tile_off[lane] : 0;
                int t_hi = __shfl_down_sync(0xffffffffu, t_lo, 1);
                if (lane == 31 && n_act == 32) t_hi = p.tile_off[32];
                const int unit = lane < n_act ? W + t_hi - t_lo : 0;   // < 2^16 (tiles of <= 2^19 routes)
                const int span = unit * nrt;
                int inc = span;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int v = __shfl_up_sync(0xffffffffu, inc, o);
                    if (lane >= o) inc += v;
                }
                const int total = __shfl_sync(0xffffffffu, inc, 31), base = inc - span;
#pragma unroll
                for (int which = 0; which < 2; ++which) {
                    const int c = (int)((long long)(blockIdx.x + which) * total / gridDim.x);
                    const bool mine = lane < n_act && c >= base && c < base + span;
                    const unsigned m = __ballot_sync(0xffffffffu, mine);
                    if (m == 0u) {
                        if (lane == 0) s_it[which] = n_items;
                    } else if (lane == __ffs(m) - 1) {
                        s_it[which] = lane * nrt + (int)((c - base) / unit);
                    }
                }
            }
            __syncthreads();
            it0 = s_it[0];
            it1 = s_it[1];
        }
        issued_upto = it0 - 1;
        ipos = item_seek<MODE>(p, it0);
        for (int i = 0; i < NS && it0 + i < it1; ++i) issue(it0 + i, i);
    }

    bool failed = false;
    uint32_t B[NTG][MAXKS][2];
    int b_key = -2;                              // token set the B fragments hold (expert, or 0)
    int red_par = 0;
    ItemPos cpos = item_seek<MODE>(p, it0);
    int slot = 0;
    uint32_t parity = 0;
    for (int item = it0; item < it1; ++item) {
        const ItemRef it = item_ref<MODE>(p, cpos, c0, ec_use);
        item_next<MODE>(p, cpos);
        // the item's weights are waited for after the first activation loads are issued
        const bool need_wait = !failed && ncw > 0 && item <= issued_upto;
        const uint8_t* st = mystage + slot * p.stage_bytes;
        const int n_groups = (it.n_tok + 8 * NTG - 1) / (8 * NTG);
        const int key = (MODE == GM_PROJ) ? 0 : it.expert;
        for (int g = 0; g < n_groups; ++g) {
            const int ntv = min(NTG, (it.n_tok - g * 8 * NTG + 7) / 8);
            float acc[NMAT][NTG][4];
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
#pragma unroll
                for (int nt = 0; nt < NTG; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[m][nt][e] = 0.0f;
            if (!failed && ncw > 0) {
                // activation fragments: token n = lane/4 of each n-tile, k = chunk*KC + q*KC/4 + 4s;
                // kept across items while the token set is the same. Two k-steps per 16-byte
                // load where a chunk has an even k-step count (every activation row stride is
                // a multiple of 16 halves, the K granularity of all weight types).
                const bool need_b = !(n_groups == 1 && key == b_key);
                bool b_done = false;
                if constexpr (MODE == GM_PROJ && KS % 2 == 0) {
                if (need_b && p.x_rs > 0) {
                    // coalesced 16-byte copies of the pass's token rows into the warp's slice
                    // (absent tokens zero-filled), then conflict-free 16-byte fragment reads
                    constexpr int QU = KC / 32;                  // 16-byte units per quarter-chunk
                    constexpr int QSB = (QU + 1) * 16;           // padded quarter-chunk bytes
                    const int upr = ncw * 4 * QU;                // units per token row
                    for (int i = lane; i < 8 * NTG * upr; i += 32) {
                        const int n = i / upr, u = i - n * upr;
                        const int cc = u / (4 * QU), w = u - cc * 4 * QU;
                        const int qq = w / QU, uu = w - qq * QU;
                        const int tok = g * 8 * NTG + n;
                        const bool ok = tok < it.n_tok;
                        const __half* src = p.X + (size_t)(ok ? x_row<MODE>(p, it, tok) : 0) * p.ldx + (c0 + cc) * KC + w * 8;
                        cp_async16(xw + (size_t)n * p.x_rs + cc * 4 * QSB + qq * QSB + uu * 16, src, ok);
                    }
                    cp_async_commit();
                    cp_async_wait_0();
                    __syncwarp();
#pragma unroll
                    for (int nt = 0; nt < NTG; ++nt) {
                        const uint8_t* xr = xw + (size_t)(nt * 8 + r8) * p.x_rs + q * QSB;
#pragma unroll
                        for (int cc = 0; cc < MAXCPW; ++cc) {
#pragma unroll
                            for (int s = 0; s < KS; s += 2) {
                                uint4 v = make_uint4(0u, 0u, 0u, 0u);
                                if (nt < ntv && cc < ncw) v = *(const uint4*)(xr + cc * 4 * QSB + (s / 2) * 16);
                                B[nt][cc * KS + s][0] = v.x;
                                B[nt][cc * KS + s][1] = v.y;
                                B[nt][cc * KS + s + 1][0] = v.z;
                                B[nt][cc * KS + s + 1][1] = v.w;
                            }
                        }
                    }
                    __syncwarp();                                // slice reads done before any refill
                    b_key = (n_groups == 1) ? key : -2;
                    b_done = true;
                }
                }
                if (need_b && !b_done) {
#pragma unroll
                    for (int nt = 0; nt < NTG; ++nt) {
                        const int n = g * 8 * NTG + nt * 8 + r8;
                        const bool ok = nt < ntv && n < it.n_tok;
                        const __half* xr = ok ? p.X + (size_t)x_row<MODE>(p, it, n) * p.ldx : nullptr;
#pragma unroll
                        for (int cc = 0; cc < MAXCPW; ++cc) {
                            if constexpr (KS % 2 == 0) {
#pragma unroll
                                for (int s = 0; s < KS; s += 2) {
                                    uint4 v = make_uint4(0u, 0u, 0u, 0u);
                                    if (ok && cc < ncw) v = *(const uint4*)(xr + (c0 + cc) * KC + q * (KC / 4) + 4 * s);
                                    B[nt][cc * KS + s][0] = v.x;
                                    B[nt][cc * KS + s][1] = v.y;
                                    B[nt][cc * KS + s + 1][0] = v.z;
                                    B[nt][cc * KS + s + 1][1] = v.w;
                                }
                            } else {
#pragma unroll
                                for (int s = 0; s < KS; ++s) {
                                    uint2 v = make_uint2(0u, 0u);
                                    if (ok && cc < ncw) v = *(const uint2*)(xr + (c0 + cc) * KC + q * (KC / 4) + 4 * s);
                                    B[nt][cc * KS + s][0] = v.x;
                                    B[nt][cc * KS + s][1] = v.y;
                                }
                            }
                        }
                    }
                    b_key = (n_groups == 1) ? key : -2;
                }
            }
            if (g == 0 && need_wait) failed = !mbar_wait(&mybar[slot], parity, p.err);
            if (!failed && ncw > 0) {
#pragma unroll
                for (int cc = 0; cc < MAXCPW; ++cc) {
                    if (cc < ncw) {
                        if constexpr (NMAT == 2 && WT != GT_F16) {
                            // gate and up decoded per k-step: two independent MMA chains
                            const uint8_t* T0 = st + cc * p.tile_bytes;
                            const uint8_t* T1 = st + wbytes + cc * p.tile_bytes;
                            D d0, d1;
                            d0.prep(T0, lane);
                            d1.prep(T1, lane);
                            if (ntv == NTG) KLoop2<D, NTG, 0, KS>::template run<NTG>(d0, d1, T0, T1, lane, cc * KS, B, acc);
                            else KLoop2<D, NTG, 0, KS>::template run<1>(d0, d1, T0, T1, lane, cc * KS, B, acc);
                        } else {
#pragma unroll
                        for (int m = 0; m < NMAT; ++m) {
                            const uint8_t* T = st + m * wbytes + cc * p.tile_bytes;
                            D dec;
                            dec.prep(T, lane);
                            if (ntv == NTG) KLoop<D, NTG, 0, KS>::template run<NMAT, NTG>(dec, T, lane, cc * KS, B, acc, m);
                            else KLoop<D, NTG, 0, KS>::template run<NMAT, 1>(dec, T, lane, cc * KS, B, acc, m);
                        }
                        }
                    }
                }
            }
            if (g == n_groups - 1) {                 // stage fully consumed: refill it
                __syncwarp();
                fence_proxy_async();
                if (!failed && item + NS < it1) issue(item + NS, slot);
            }
            // cross-warp reduction in a fixed order (double-buffered: one barrier per pass)
            float* rbuf = red + (size_t)red_par * NW * NMAT * NTG * 128;
            float* myred = rbuf + (size_t)warp * NMAT * NTG * 128;
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
#pragma unroll
                for (int nt = 0; nt < NTG; ++nt)
                    *(float4*)(myred + ((m * NTG + nt) * 32 + lane) * 4) =
                        make_float4(acc[m][nt][0], acc[m][nt][1], acc[m][nt][2], acc[m][nt][3]);
            __syncthreads();
            red_par ^= 1;
            for (int t = threadIdx.x; t < NTG * 128; t += blockDim.x) {
                const int nt = t >> 7, ln = (t & 127) >> 2, e = t & 3;
                const int rr = (ln >> 2) + 8 * (e >> 1);
                const int n = g * 8 * NTG + nt * 8 + 2 * (ln & 3) + (e & 1);
                if (n >= it.n_tok) continue;
                float v[NMAT];
#pragma unroll
                for (int m = 0; m < NMAT; ++m) {
                    float sum = 0.0f;
                    for (int w = 0; w < NW; ++w) sum += rbuf[(((size_t)w * NMAT + m) * NTG + nt) * 128 + ln * 4 + e];
                    v[m] = sum;
                }
                if constexpr (MODE == GM_PROJ) {
                    const ProjSeg& sg = p.seg[it.seg];
                    const int row = it.rt * 16 + rr;
                    if (row < sg.rows) {
                        float* o = p.out + (size_t)n * p.ldo + sg.out_off + row;
                        if (p.epi == EPI_ADD) *o = v[0] + *o;
                        else if (p.epi == EPI_SOFTCAP) *o = tanhf(v[0] * (1.0f / p.cap)) * p.cap;
                        else *o = v[0];
                    }
                } else if constexpr (MODE == GM_GATEUP) {
                    const int row = it.rt * 16 + rr;
                    if (row < p.out_rows) {
                        const float gt = v[0], up = v[1];
                        const float si = gt / (1.0f + expf(-gt));
                        p.yout[(size_t)(it.tok0 + n) * p.ldy + row] = __float2half_rn(up * si);
                    }
                } else {
                    const int row = it.rt * 16 + rr;
                    if (row < p.out_rows) {
                        const int pr = it.tok0 + n;
                        p.out[(size_t)pr * p.ldo + row] = v[0] * p.route_w[pr];
                    }
                }
            }
        }
        if (n_groups == 0 && need_wait) failed = !mbar_wait(&mybar[slot], parity, p.err);
        if (++slot == NS) { slot = 0; parity ^= 1u; }
    }
    pdl_release();
    // After a failed wait (error already recorded) later copies may still be in flight:
    // wait for each of them, bounded, before the shared memory goes away. Every warp
    // stayed in the item loop above, so the block-wide barriers always matched.
    if (failed && ncw > 0) {
        for (int item = issued_upto - NS + 1; item <= issued_upto; ++item) {
            if (item < it0) continue;
            const int j = item - it0;
            (void)mbar_wait(&mybar[j % NS], (uint32_t)((j / NS) & 1), nullptr);
        }
    }
}

template <int WT, int KSF>
void launch_typed(const GemvParams& p, int nwarps, int grid, int smem, cudaStream_t s) {
    void (*k)(const GemvParams);
    if (p.mode == GM_PROJ) k = gemv_kernel<WT, KSF, GM_PROJ, 2, 512, 1>;
    else if (p.mode == GM_GATEUP) k = gemv_kernel<WT, KSF, GM_GATEUP, 2, 256, 2>;
    else k = gemv_kernel<WT, KSF, GM_DOWN, 1, 256, 3>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    launch_pdl(k, dim3(grid), dim3(nwarps * 32), (size_t)smem, s, p);
}

}  // namespace

void gemv_geometry(const DevMat& m, int nmat, int ntg, int* nwarps, int* n_stages, int* stage_bytes, int* smem,
                   int* cps, int* x_rs) {
    *cps = 1;
    const int max_cpw = std::max(1, MAXKS / m.steps);       // chunks a warp can hold in registers
    const int min_nw = (m.chunks + max_cpw - 1) / max_cpw;
    int nw = 0;
    if (ntg == 1) {
        // expert passes: 8 warps (256 threads, three blocks per SM), K split as evenly as it goes
        nw = std::max(min_nw, std::min(8, m.chunks));
    } else {
        // smallest warp count >= min(8, chunks) that splits the chunks evenly, else the
        // register-bound minimum
        for (int cand = std::max(min_nw, std::min(8, m.chunks)); cand <= 16; ++cand)
            if (m.chunks % cand == 0) { nw = cand; break; }
        if (nw == 0) nw = std::max(min_nw, std::min(16, m.chunks));
    }
    const int cpw = (m.chunks + nw - 1) / nw;
    const int sb = cpw * m.tile_bytes * nmat;
    const int red = 2 * nw * nmat * ntg * 128 * 4;
    // projections: each warp stages its K-slice of the pass's tokens in shared memory, a
    // token row as 4 quarter-chunks of KC/4 halves each padded by 16 bytes, the row padded
    // so that the 8 lanes of a quarter-warp (2 tokens x 4 quarters) read 8 distinct 16-byte
    // bank groups
    int rs = 0;
    if (x_rs && nmat == 1 && ntg == 2 && m.steps % 2 == 0) {
        const int qsu = m.steps / 2 + 1;                     // 16-byte units per padded quarter
        const int base = cpw * 4 * qsu;
        for (int pad = 0; pad < 8 && rs == 0; ++pad) {
            const int r = (base + pad) % 8;
            bool ok = true;
            for (int a = 0; a < 4; ++a)
                for (int b2 = 0; b2 < 4; ++b2)
                    if ((a * qsu) % 8 == (b2 * qsu + r) % 8) ok = false;
            if (ok) rs = (base + pad) * 16;
        }
    }
    int xbytes = nw * 8 * ntg * rs;
    auto total = [&](int ns) { return 128 * ((nw * ns * 8 + 127) / 128) + nw * ns * sb + red + xbytes; };
    // deepest ring (up to 4 stages) at the target blocks per SM: three for the expert down
    // pass, two for gate/up (two matrices per stage) and the projections (one block's
    // barriers overlap the other's streaming)
    const int per_sm = 233472, per_block_reserved = 1024;
    const int want = (ntg == 1 && nmat == 1) ? 3 : 2;
    if (xbytes > 0 && want * (total(1) + per_block_reserved) > per_sm) { rs = 0; xbytes = 0; }   // keep the blocks per SM
    if (x_rs) *x_rs = rs;
    int ns = 0;
    for (int cand = 4; cand >= 1 && ns == 0; --cand)
        if (want * (total(cand) + per_block_reserved) <= per_sm) ns = cand;
    if (ns == 0) {
        ns = 1;
        for (int cand = 4; cand >= 1; --cand)
            if (total(cand) + per_block_reserved <= per_sm) { ns = cand; break; }
    }
    *nwarps = nw;
    *n_stages = ns;
    *stage_bytes = sb;
    *smem = total(ns);
}

void launch_gemv(const GemvParams& p, int nwarps, int grid, int smem, cudaStream_t s) {
    switch (p.type) {
        case GT_Q4_K: launch_typed<GT_Q4_K, 16>(p, nwarps, grid, smem, s); break;
        case GT_Q6_K: launch_typed<GT_Q6_K, 16>(p, nwarps, grid, smem, s); break;
        case GT_Q8_0: launch_typed<GT_Q8_0, 8>(p, nwarps, grid, smem, s); break;
        case GT_F16:
            if (p.steps == 4) launch_typed<GT_F16, 4>(p, nwarps, grid, smem, s);
            else if (p.steps == 2) launch_typed<GT_F16, 2>(p, nwarps, grid, smem, s);
            else launch_typed<GT_F16, 1>(p, nwarps, grid, smem, s);
            break;
        default: break;
    }
}

}  // namespace z2b
