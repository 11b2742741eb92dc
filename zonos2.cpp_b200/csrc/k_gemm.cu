// k_gemm.cu — grouped expert GEMM on the 5th-generation tensor cores (tcgen05), for the
// experts that receive many routed tokens in a step (prompt rows, large batches).
//
// Replaces ggml_mul_mat_id (src/zonos2-graph.cpp:223-231) for those experts; the tile
// GEMV in k_gemv.cu keeps the experts with few tokens. The same kernel runs the attention
// projections (ggml_mul_mat, :107-111, 175) over the prompt rows of a step (GM_PROJ: the
// segments' weights over a contiguous token range, store / add / softcap epilogue).
//
// Tile = (expert, 128 weight rows, up to 248 routes); the MMA is M 128 x N (the tile's
// activation rows, which start 8-aligned at or before its first route, rounded up to 16)
// x K 16, f16 x f16 -> f32 in tensor memory (TMEM: gate at columns [0, 256), up at [256,
// 512)). Before the GEMM a small kernel copies the activations in stage order (a stage's
// 64 k values contiguous; for gate/up one row per route, in expert order), so a tile's
// stage of activations is one TMA box. A persistent block walks its tiles with
// warp-specialised roles that hand over through mbarriers, never a block-wide barrier:
//   - 8 decode warps, one per 16-row weight tile. Lane 0 of each streams its tile's
//     quantised chunks (cp.async.bulk, one chunk of one matrix per ring slot, continuing
//     into the block's next tile); the warp decodes each 64-wide K stage with the same
//     in-register decoders as the GEMV (so the weight values are identical) into an A ring
//     slot in the UMMA K-major layout, with conflict-free 16-byte stores. The same warps
//     run the epilogue.
//   - 1 MMA warp: one lane waits for each stage's A and B, issues four tcgen05.mma and
//     releases the slots with tcgen05.commit; after a tile's last stage it commits to the
//     accumulator barrier the epilogue waits on.
//   - 1 activation producer: one TMA box per stage into a B ring slot (this CTA only).
// A stage covers, per lane quarter q of the decoders, k = chunk*KC + q*KC/4 + 16j + [0,16):
// four 16-wide runs of the chunk (the tile layout's fragment order); the stage-ordered
// activations hold the same k values in the same order, so the contraction is over the
// same 64 k values.
//
// Shared-memory operand layouts (K-major): A without swizzle, 8x8 core matrices of 16-byte
// rows, element (m, k) at (k / 8) * LBO + (m / 8) * 128 + (m % 8) * 16 + (k % 8) * 2 with
// LBO = 2048 + 16 (padded for the decoders' stores); B with the 128-byte swizzle, row n at
// n * 128 with its 16-byte chunk c at chunk c ^ (n % 8), 8-row atoms 1024 bytes apart.
#include "common.cuh"
#include "gguf.h"
#include "kernels.h"
#include "launch.cuh"
#include "tile_layout.h"
#include "k_decode.cuh"
#include "tc05.cuh"

#include <algorithm>

namespace z2b {

namespace {

constexpr int GT_M = 128;                        // weight rows per tile
constexpr int NT_MAX = 256;                      // MMA N / B rows per stage (a tile's rows start
                                                 // 8-aligned at or before its first route)
constexpr int NT_TILE_MAX = 248;                 // routes per tile, so that the aligned rows fit
constexpr int KG = 64;                           // K per stage
constexpr int DQW = 8;                           // decode warps (16 weight rows each)
constexpr int GM_THREADS = 32 * (DQW + 2);       // + the MMA warp + the activation (B) producer
constexpr int NA = 2;                            // A ring slots (one stage of one matrix)
constexpr int NB = 4;                            // B ring slots (one stage of activations)
constexpr int MAX_RR = 6;                        // raw chunk ring slots per decode warp
// A (decoded weights, no swizzle): K-direction stride between 8-wide core-matrix columns,
// padded by 16 bytes so that the 8 lanes of a quarter-warp storing one 16-byte row each
// (two rows x four k-columns) hit 8 distinct bank groups.
constexpr uint32_t A_LBO = GT_M / 8 * 128 + 16, CORE_SBO = 128;
constexpr int A_SLOT = (int)A_LBO * (KG / 8);    // 16.1 KB
// B (activations, 128-byte swizzle): stage row n (route or token row0 + n) is one 128-byte
// row at n * 128, its 16-byte chunk c at chunk c ^ (n % 8), as one TMA box writes it; 8-row
// atoms of 1024 B.
constexpr int B_SLOT = NT_MAX * KG * 2;          // 32 KB

// instruction descriptor: M 128 (weight rows) x N (activation rows)
__device__ __forceinline__ uint32_t idesc_n(int n) { return idesc_f16(GT_M, n); }

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(lbo >> 4) << 16) | ((uint64_t)(CORE_SBO >> 4) << 32) |
           (1ull << 46);
}

// Activation rows copied to Xp (row stride K) in stage order: within each KC-wide chunk,
// stage j's 64 values k = q*KC/4 + 16j + [0, 16) for q = 0..3 become the contiguous run
// [64j, 64j + 64), so a GEMM stage of a row is one 128-byte line and a tile's stage is one
// TMA box over consecutive rows. Row r of Xp is X row rowmap[r] (the gate/up pass: one row
// per route, in expert order) or X row r; rows [r0, r1), clipped to *n_rows when given.
// 16-byte pieces, one per thread.
template <int KC>
__global__ void gemm_x_stage_order_kernel(const __half* __restrict__ X, int ldx, const int* __restrict__ rowmap,
                                          const int* __restrict__ n_rows, int r0, int r1, int K,
                                          __half* __restrict__ Xp) {
    pdl_wait();
    if (n_rows) r1 = min(r1, *n_rows);
    const int ppr = K / 8;                           // pieces per row
    const long total = (long)max(r1 - r0, 0) * ppr;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int row = r0 + (int)(i / ppr), pc = (int)(i % ppr);
        const int src_row = rowmap ? rowmap[row] : row;
        const int kd = pc * 8, c = kd / KC, rem = kd % KC;
        const int j = rem / 64, q = (rem % 64) / 16, h = (rem % 16) / 8;
        const int ks = c * KC + q * (KC / 4) + 16 * j + 8 * h;
        *reinterpret_cast<uint4*>(Xp + (size_t)row * K + kd) =
            *reinterpret_cast<const uint4*>(X + (size_t)src_row * ldx + ks);
    }
    pdl_release();
}

__device__ __forceinline__ void st16(uint8_t* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    *reinterpret_cast<uint4*>(p) = make_uint4(a, b, c, d);
}

// Decode k-steps S0..S0+3 of this warp's 16-row tile chunk into an A slot. Lane (r, q)
// holds rows r and r + 8 at chunk k = q*KC/4 + 4s + [0, 4); in the slot they go to local
// k = 16q + 4(s - S0) + [0, 4), two k-steps per 16-byte core-matrix row. The 32 lanes of
// one store cover 32 distinct 16-byte rows (4 per bank group), the minimum 4 wavefronts.
template <class D, int S0>
__device__ __forceinline__ void dq_stage(const D& dec, const uint8_t* T, int lane, uint8_t* As, int warp) {
    uint32_t a0[4], a1[4], a2[4], a3[4];
    dec.template frag<S0 + 0>(T, lane, a0);
    dec.template frag<S0 + 1>(T, lane, a1);
    dec.template frag<S0 + 2>(T, lane, a2);
    dec.template frag<S0 + 3>(T, lane, a3);
    uint8_t* p0 = As + 2 * (lane & 3) * A_LBO + 2 * warp * 128 + (lane >> 2) * 16;
    st16(p0, a0[0], a0[2], a1[0], a1[2]);
    st16(p0 + 128, a0[1], a0[3], a1[1], a1[3]);
    st16(p0 + A_LBO, a2[0], a2[2], a3[0], a3[2]);
    st16(p0 + A_LBO + 128, a2[1], a2[3], a3[1], a3[3]);
}

template <class D>
__device__ __forceinline__ void dq_stage_j(int j, const D& dec, const uint8_t* T, int lane, uint8_t* As, int warp) {
    if constexpr (D::KS >= 16) {
        switch (j) {
            case 0: dq_stage<D, 0>(dec, T, lane, As, warp); break;
            case 1: dq_stage<D, 4>(dec, T, lane, As, warp); break;
            case 2: dq_stage<D, 8>(dec, T, lane, As, warp); break;
            default: dq_stage<D, 12>(dec, T, lane, As, warp); break;
        }
    } else if constexpr (D::KS >= 8) {
        if (j == 0) dq_stage<D, 0>(dec, T, lane, As, warp);
        else dq_stage<D, 4>(dec, T, lane, As, warp);
    } else {
        dq_stage<D, 0>(dec, T, lane, As, warp);
    }
}

// rows past the matrix: zeros
__device__ __forceinline__ void dq_zero(int lane, uint8_t* As, int warp) {
    uint8_t* p0 = As + 2 * (lane & 3) * A_LBO + 2 * warp * 128 + (lane >> 2) * 16;
    st16(p0, 0u, 0u, 0u, 0u);
    st16(p0 + 128, 0u, 0u, 0u, 0u);
    st16(p0 + A_LBO, 0u, 0u, 0u, 0u);
    st16(p0 + A_LBO + 128, 0u, 0u, 0u, 0u);
}

// Tile t of a launch: the full token tiles of every expert (or projection segment) first,
// then each one's remainder tile, largest remainder first (xord: experts by remainder,
// descending). Row blocks vary fastest. Blocks take tiles in serpentine order (round r:
// block b, or gridDim - 1 - b on odd rounds), so with tiles in decreasing size the load per
// block stays within about one small tile of the mean. The per-expert entries (id, first
// route, routes, row blocks) sit in a shared-memory table filled once per launch, so a
// lookup is a scan of shared memory, not a chain of dependent loads. e < 0: past the end.
struct GTile { int e, rb, tok0, nv; };
struct ExTab { int e[MAX_EXPERTS], tb0[MAX_EXPERTS], ne[MAX_EXPERTS], nrb[MAX_EXPERTS], ord[MAX_EXPERTS]; };

__device__ __forceinline__ int snake_tile(int r) {
    return r * (int)gridDim.x + ((r & 1) ? (int)gridDim.x - 1 - (int)blockIdx.x : (int)blockIdx.x);
}

template <int MODE>
__device__ __forceinline__ void gm_expert(const GemvParams& p, int a, int n_rb, int* e, int* tok_base, int* ne,
                                          int* nrb) {
    if constexpr (MODE == GM_PROJ) {
        *e = a; *tok_base = p.tok0; *ne = p.T; *nrb = (p.seg[a].rows + GT_M - 1) / GT_M;
    } else {
        *e = p.active[a]; *tok_base = p.seg_mid[*e]; *ne = p.seg_off[*e + 1] - *tok_base; *nrb = n_rb;
    }
}

__device__ GTile gm_tile(const ExTab& x, int n_ex, int t, int nt, int n_full) {
    const bool full = t < n_full;
    if (!full) t -= n_full;
    int base = 0;
    for (int i = 0; i < n_ex; ++i) {
        const int a = full ? i : x.ord[i];
        const int ne = x.ne[a], nrb = x.nrb[a];
        const int cnt = full ? (ne / nt) * nrb : ((ne % nt) ? nrb : 0);
        if (t < base + cnt) {
            const int j = t - base;
            if (full) return GTile{x.e[a], j % nrb, x.tb0[a] + (j / nrb) * nt, nt};
            return GTile{x.e[a], j, x.tb0[a] + (ne / nt) * nt, ne % nt};
        }
        base += cnt;
    }
    return GTile{-1, 0, 0, 0};
}

template <int WT, int KSF, int MODE>
__global__ void __launch_bounds__(GM_THREADS, 1) moe_gemm_kernel(const GemvParams p, const __grid_constant__ CUtensorMap tmx) {
    using D = typename DecSel<WT, KSF>::T;
    constexpr int KC = D::KC, KS = D::KS;
    static_assert(KS % 4 == 0, "a stage is four k-steps");
    constexpr int CPS = KS / 4;                      // stages per chunk
    constexpr int NMAT = (MODE == GM_GATEUP) ? 2 : 1;
    constexpr uint32_t NCOLS = NMAT * NT_MAX;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // the B atoms need 1024-byte alignment (the swizzle pattern follows address bits 7..9)
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* Bring = smem;                           // [NB][B_SLOT]
    uint8_t* Aring = smem + NB * B_SLOT;             // [NA][A_SLOT]
    uint8_t* raw = Aring + NA * A_SLOT;              // [DQW][RR][tile_bytes]
    __shared__ __align__(8) uint64_t a_full[NA], a_empty[NA], b_full[NB], b_empty[NB];
    __shared__ __align__(8) uint64_t acc_full, acc_empty, fin_bar;
    __shared__ __align__(8) uint64_t raw_bar[DQW][MAX_RR];
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag;
    __shared__ ExTab xt;
    volatile int* ab = &abort_flag;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int RR = p.n_stages, NT = p.gm_nt;

    if (warp == DQW) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(&tmem_base)), "r"(NCOLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int i = 0; i < NA; ++i) { mbar_init(&a_full[i], DQW); mbar_init(&a_empty[i], 1); }
        for (int i = 0; i < NB; ++i) { mbar_init(&b_full[i], 1); mbar_init(&b_empty[i], 1); }   // one producer per stage
        mbar_init(&acc_full, 1);
        mbar_init(&acc_empty, DQW);
        mbar_init(&fin_bar, 1);
        abort_flag = 0;
    }
    if (warp < DQW && lane == 0)
        for (int i = 0; i < RR; ++i) mbar_init(&raw_bar[warp][i], 1);
    fence_mbar_init();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = tmem_base;
    pdl_wait();
    pdl_release();

    // experts with GEMM routes: active[n_small .. n_active), routes [seg_mid[e], seg_off[e + 1]);
    // projections (GM_PROJ): the segments' rows over tokens [tok0, tok0 + T)
    int e_lo = 0, e_hi = 0, n_rb = 0;
    if constexpr (MODE == GM_PROJ) {
        e_hi = p.n_seg;
    } else {
        e_lo = *p.n_small;
        e_hi = *p.n_active;
        n_rb = (p.out_rows + GT_M - 1) / GT_M;
    }
    const int n_ex = min(e_hi - e_lo, MAX_EXPERTS);
    for (int i = tid; i < n_ex; i += blockDim.x) {
        int e, tb0, ne, nrb;
        gm_expert<MODE>(p, e_lo + i, n_rb, &e, &tb0, &ne, &nrb);
        xt.e[i] = e; xt.tb0[i] = tb0; xt.ne[i] = ne; xt.nrb[i] = nrb;
    }
    __syncthreads();
    for (int i = tid; i < n_ex; i += blockDim.x) {     // remainder tiles, largest first
        const int ri = xt.ne[i] % NT;
        int rank = 0;
        for (int j = 0; j < n_ex; ++j) {
            const int rj = xt.ne[j] % NT;
            rank += (rj > ri || (rj == ri && j < i)) ? 1 : 0;
        }
        xt.ord[rank] = i;
    }
    __syncthreads();
    int n_full = 0, n_tiles = 0;
    for (int a = 0; a < n_ex; ++a) {
        n_full += (xt.ne[a] / NT) * xt.nrb[a];
        n_tiles += (xt.ne[a] + NT - 1) / NT * xt.nrb[a];
    }
    const int n_groups = p.chunks * CPS;             // stages per matrix per tile

    bool ok = true;
    if (warp == DQW) {
        // ---- MMA warp: one lane issues ----
        if (lane == 0) {
            int aslot = 0, bslot = 0;
            uint32_t aph = 0, bph = 0, accph = 0;
            for (int r = 0, t = snake_tile(0); t < n_tiles && ok; t = snake_tile(++r)) {
                const GTile ti = gm_tile(xt, n_ex, t, NT, n_full);
                const uint32_t idesc = idesc_n((ti.tok0 % 8 + ti.nv + 15) & ~15);   // rows from tok0 & ~7
                ok = wait_ab(&acc_empty, accph ^ 1u, p.err, ab);   // previous tile's accumulators read
                accph ^= 1u;
                if (!ok) break;
                tc_fence_after();
                for (int g = 0; g < n_groups && ok; ++g) {
                    ok = wait_ab(&b_full[bslot], bph, p.err, ab);
                    if (!ok) break;
#pragma unroll
                    for (int m = 0; m < NMAT; ++m) {
                        if (!ok) break;
                        ok = wait_ab(&a_full[aslot], aph, p.err, ab);
                        if (!ok) break;
                        tc_fence_after();
                        const uint32_t sa = smem_u32(Aring + aslot * A_SLOT), sb = smem_u32(Bring + bslot * B_SLOT);
#pragma unroll
                        for (int kb = 0; kb < KG / 16; ++kb)
                            umma_f16(tm + m * NT_MAX, umma_desc(sa + 2 * kb * A_LBO, A_LBO),
                                     umma_desc_sw128(sb + 32 * kb), idesc, (g > 0 || kb > 0) ? 1u : 0u);
                        umma_commit(&a_empty[aslot]);            // A slot free once these MMAs complete
                        if (++aslot == NA) { aslot = 0; aph ^= 1u; }
                    }
                    if (!ok) break;
                    umma_commit(&b_empty[bslot]);
                    if (++bslot == NB) { bslot = 0; bph ^= 1u; }
                }
                if (!ok) break;
                umma_commit(&acc_full);
            }
            if (!ok) *ab = 1;
            // every MMA issued completes before the block releases its memory
            umma_commit(&fin_bar);
            (void)mbar_wait(&fin_bar, 0, nullptr, 1u << 16);
        }
        __syncwarp();
    } else if (warp < DQW) {
        // ---- decode warps ----
        const uint8_t* myraw = raw + (size_t)warp * RR * p.tile_bytes;
        // raw chunk stream (this warp's row tile of each of the block's tiles, chunk-major,
        // gate then up): issue cursor (tile, chunk index) and counts
        int is_r = 0, is_t = snake_tile(0), is_q = 0, n_issued = 0, n_waited = 0;
        GTile is_ti = is_t < n_tiles ? gm_tile(xt, n_ex, is_t, NT, n_full) : GTile{-1, 0, 0, 0};
        auto issue_chunk = [&]() {
            if (is_t >= n_tiles) return;
            const int slot = n_issued % RR, c = is_q / NMAT, m = is_q % NMAT;
            const int rt = is_ti.rb * DQW + warp;
            if (lane == 0) {
                uint64_t* bar = &raw_bar[warp][slot];
                const uint8_t* src;
                int nrt;
                if constexpr (MODE == GM_PROJ) {
                    src = p.seg[is_ti.e].tiles;
                    nrt = p.seg[is_ti.e].n_row_tiles;
                } else {
                    src = (m == 0 ? p.w0 : p.w1) + (size_t)is_ti.e * p.expert_stride;
                    nrt = p.n_row_tiles;
                }
                if (rt < nrt) {
                    mbar_expect_tx(bar, (uint32_t)p.tile_bytes);
                    bulk_g2s(const_cast<uint8_t*>(myraw) + (size_t)slot * p.tile_bytes,
                             src + ((size_t)rt * p.chunks + c) * p.tile_bytes, (uint32_t)p.tile_bytes, bar);
                } else {
                    mbar_expect_tx(bar, 0u);                 // no rows here: the phase completes empty
                }
            }
            ++n_issued;
            if (++is_q == p.chunks * NMAT) {
                is_q = 0;
                is_t = snake_tile(++is_r);
                if (is_t < n_tiles) is_ti = gm_tile(xt, n_ex, is_t, NT, n_full);
            }
        };
        for (int i = 0; i < RR; ++i) issue_chunk();
        int aslot = 0;
        uint32_t aph = 0, accph = 0;
        for (int r = 0, t = snake_tile(0); t < n_tiles && ok; t = snake_tile(++r)) {
            const GTile ti = gm_tile(xt, n_ex, t, NT, n_full);
            const int rt = ti.rb * DQW + warp;
            const bool rt_ok = rt < (MODE == GM_PROJ ? p.seg[ti.e].n_row_tiles : p.n_row_tiles);
            D dec[NMAT];
            int rslot[NMAT];
            for (int g = 0; g < n_groups && ok; ++g) {
                const int j = g % CPS;
#pragma unroll
                for (int m = 0; m < NMAT; ++m) {
                    if (!ok) break;
                    if (j == 0) {
                        // first stage of chunk (c, m): wait for its bytes, read its scales
                        rslot[m] = n_waited % RR;
                        bool w = wait_ab(&raw_bar[warp][rslot[m]], (uint32_t)((n_waited / RR) & 1), p.err, ab);
                        ok = __all_sync(0xffffffffu, w);
                        if (!ok) break;
                        ++n_waited;
                        if (rt_ok) dec[m].prep(myraw + (size_t)rslot[m] * p.tile_bytes, lane);
                    }
                    bool w = wait_ab(&a_empty[aslot], aph ^ 1u, p.err, ab);
                    ok = __all_sync(0xffffffffu, w);
                    if (!ok) break;
                    uint8_t* As = Aring + aslot * A_SLOT;
                    if (rt_ok) dq_stage_j<D>(j, dec[m], myraw + (size_t)rslot[m] * p.tile_bytes, lane, As, warp);
                    else dq_zero(lane, As, warp);
                    fence_proxy_async();                     // generic-proxy writes -> tensor core reads
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&a_full[aslot]);
                    if (++aslot == NA) { aslot = 0; aph ^= 1u; }
                    if (j == CPS - 1) issue_chunk();         // chunk (c, m) decoded: its slot refills
                }
            }
            if (!ok) break;
            // epilogue: warp w reads TMEM lanes 32 (w % 4).. (its rows), token columns in
            // 16-wide chunks alternating between the two warps of a lane quarter
            {
                bool w = wait_ab(&acc_full, accph, p.err, ab);
                accph ^= 1u;
                ok = __all_sync(0xffffffffu, w);
                if (!ok) break;
            }
            tc_fence_after();
            const int qd = warp & 3;
            const int row = ti.rb * GT_M + 32 * qd + lane;
            const int row_lim = MODE == GM_PROJ ? p.seg[ti.e].rows : p.out_rows;
            const uint32_t lane_addr = tm + ((uint32_t)(32 * qd) << 16);
            const int n_off = ti.tok0 % 8;             // column n holds row (tok0 & ~7) + n
            const int ncc = (n_off + ti.nv + 15) >> 4;
#pragma unroll 1
            for (int cc = warp >> 2; cc < ncc; cc += 2) {
                float v0[16], v1[16];
                tmem_ld16(lane_addr + cc * 16, v0);
                if constexpr (NMAT == 2) tmem_ld16(lane_addr + NT_MAX + cc * 16, v1);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int n = cc * 16 + i - n_off;
                    if (n < 0 || n >= ti.nv || row >= row_lim) continue;
                    if constexpr (MODE == GM_GATEUP) {
                        // SiLU with the fast exponential and division (about 1e-6 relative): a
                        // tile's 32K outputs would otherwise cost as much as its last stages
                        const float gt = v0[i], up = v1[i];
                        const float si = __fdividef(gt, 1.0f + __expf(-gt));
                        p.yout[(size_t)(ti.tok0 + n) * p.ldy + row] = __float2half_rn(up * si);
                    } else if constexpr (MODE == GM_PROJ) {
                        float* o = p.out + (size_t)(ti.tok0 + n) * p.ldo + p.seg[ti.e].out_off + row;
                        if (p.epi == EPI_ADD) *o = v0[i] + *o;
                        else if (p.epi == EPI_SOFTCAP) *o = tanhf(v0[i] * (1.0f / p.cap)) * p.cap;
                        else *o = v0[i];
                    } else {
                        p.out[(size_t)(ti.tok0 + n) * p.ldo + row] = v0[i] * p.route_w[ti.tok0 + n];
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty);
        }
        if (!ok) *ab = 1;
        cp_async_wait_0();
        // after a failure: chunk copies still in flight land (bounded) before release
        if (!ok && lane == 0)
            for (int J = n_waited; J < n_issued; ++J)
                (void)mbar_wait(&raw_bar[warp][J % RR], (uint32_t)((J / RR) & 1), nullptr, 1u << 16);
        __syncwarp();
    } else {
        // ---- activation (B) producer warp: stage g of a tile is the 64-wide stage-ordered
        // column block (chunk*KC + 64j) of the NT + 8 consecutive rows from tok0 & ~7 of Xp (the
        // tile's routes, then rows of the next routes or zero fill past the end, in columns
        // the epilogue never reads): one TMA box with the 128-byte swizzle. ----
        int slot = 0, issued = 0;
        uint32_t ph = 0;
        for (int r = 0, t = snake_tile(0); t < n_tiles && ok; t = snake_tile(++r)) {
            const GTile ti = gm_tile(xt, n_ex, t, NT, n_full);
            for (int g = 0; g < n_groups && ok; ++g) {
                bool w = wait_ab(&b_empty[slot], ph ^ 1u, p.err, ab);
                ok = __all_sync(0xffffffffu, w);
                if (!ok) break;
                if (lane == 0) {
                    mbar_expect_tx(&b_full[slot], (uint32_t)((NT + 8) * 128));
                    tma_load_2d(Bring + slot * B_SLOT, &tmx, (g / CPS) * KC + 64 * (g % CPS), ti.tok0 & ~7, &b_full[slot]);
                }
                __syncwarp();
                ++issued;
                if (++slot == NB) { slot = 0; ph ^= 1u; }
            }
        }
        if (!ok) {
            *ab = 1;
            // loads still in flight land (bounded) before the block releases its memory
            if (lane == 0)
                for (int G = max(0, issued - NB); G < issued; ++G)
                    (void)mbar_wait(&b_full[G % NB], (uint32_t)((G / NB) & 1), nullptr, 1u << 16);
        }
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == DQW) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tm), "r"(NCOLS) : "memory");
    }
}

// Raw ring depth (chunks per decode warp) that fits next to the A and B rings (static
// shared memory: barriers and the expert table; 1 KB of slack for the B alignment).
int gemm_raw_slots(int tile_bytes) {
    const int budget = 232448 - 6144 - 1024 - NA * A_SLOT - NB * B_SLOT;
    return std::min(MAX_RR, budget / (DQW * tile_bytes));
}

// The stage-ordered activations Xp[x_rows][K]: box {64, gm_nt + 8} at (chunk*KC + 64j, row)
// is one GEMM stage of a tile's rows (its routes start at most 7 rows in), written with the
// 128-byte swizzle (rows past x_rows read as zeros).
bool make_x_map(const GemvParams& p, CUtensorMap* map) {
    auto enc = tensor_map_encoder();
    if (!enc || p.x_rows <= 0 || ((uintptr_t)p.xperm & 15u) || p.K % 64) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)p.K, (cuuint64_t)p.x_rows};
    const cuuint64_t strides[1] = {(cuuint64_t)p.K * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)(p.gm_nt + 8)};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.xperm, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int WT, int KSF>
bool gemm_typed(const GemvParams& p, int grid, cudaStream_t s) {
    void (*k)(const GemvParams, const CUtensorMap) = p.mode == GM_GATEUP ? moe_gemm_kernel<WT, KSF, GM_GATEUP>
                                  : p.mode == GM_PROJ ? moe_gemm_kernel<WT, KSF, GM_PROJ>
                                                      : moe_gemm_kernel<WT, KSF, GM_DOWN>;
    GemvParams q = p;
    q.n_stages = gemm_raw_slots(p.tile_bytes);
    if (q.n_stages < (p.mode == GM_GATEUP ? 2 : 1)) return false;   // moe_gemm_supported excludes this
    if (q.gm_nt <= 0 || q.gm_nt > NT_TILE_MAX || q.gm_nt % 8) q.gm_nt = NT_TILE_MAX;
    constexpr int KC = DecSel<WT, KSF>::T::KC;
    alignas(64) CUtensorMap tmx;
    if (!q.xperm || q.K % KC || q.x_row0 < 0 || q.x_row0 >= q.x_rows || !make_x_map(q, &tmx)) return false;
    {
        // gate/up: one row per route (expert order, up to the step's route count); else X's rows
        const bool per_route = q.mode == GM_GATEUP;
        const long pieces = (long)(q.x_rows - q.x_row0) * (q.K / 8);
        const int blocks = (int)std::min<long>((pieces + 255) / 256, 4L * grid);
        launch_pdl(gemm_x_stage_order_kernel<KC>, dim3(blocks), dim3(256), 0, s, q.X, q.ldx,
                   per_route ? q.route_tok : (const int*)nullptr, per_route ? q.n_routes : (const int*)nullptr,
                   q.x_row0, q.x_rows, q.K, q.xperm);
    }
    const int smem = 1024 + NB * B_SLOT + NA * A_SLOT + q.n_stages * DQW * p.tile_bytes;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    launch_pdl(k, dim3(grid), dim3(GM_THREADS), (size_t)smem, s, q, tmx);
    return true;
}

}  // namespace

// cuTensorMapEncodeTiled from the driver, looked up once.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (PFN_cuTensorMapEncodeTiled_v12000) nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

bool moe_gemm_supported(const DevMat& m) {
    switch (m.type) {
        case GT_Q4_K: case GT_Q6_K: return true;              // 256-wide chunks, four stages each
        case GT_Q8_0: return true;                            // 128-wide chunks, two stages each
        case GT_F16: return m.steps == 4;                     // 64-wide chunks, one stage each
        default: return false;
    }
}

bool launch_moe_gemm(const GemvParams& p, int grid, cudaStream_t s) {
    switch (p.type) {
        case GT_Q4_K: return gemm_typed<GT_Q4_K, 16>(p, grid, s);
        case GT_Q6_K: return gemm_typed<GT_Q6_K, 16>(p, grid, s);
        case GT_Q8_0: return gemm_typed<GT_Q8_0, 8>(p, grid, s);
        case GT_F16: return gemm_typed<GT_F16, 4>(p, grid, s);
        default: return false;
    }
}

}  // namespace z2b
