// k_gemm.cu — grouped expert GEMM on the 5th-generation tensor cores (tcgen05), for the
// experts that receive many routed tokens in a step (prompt rows, large batches).
//
// Replaces ggml_mul_mat_id (src/zonos2-graph.cpp:223-231) for those experts; the tile
// GEMV in k_gemv.cu keeps the experts with few tokens. The same kernel runs the attention
// projections (ggml_mul_mat, :107-111, 175) over the prompt rows of a step (GM_PROJ: the
// segments' weights over a contiguous token range, store / add / softcap epilogue). Tile = (expert, 128 weight rows,
// 64 routed tokens). Per 256-wide K group the four warps dequantise the block's eight
// 16-row weight tiles (the same in-register decoders as the GEMV, so the weight values
// are identical) into shared memory in the UMMA K-major interleaved layout, gather the
// tokens' activation rows next to them, and one thread issues tcgen05.mma (M 128, N 64,
// K 16, f16 x f16 -> f32) into tensor-memory accumulators; a tcgen05.commit on an
// mbarrier tells the block when the operands may be overwritten. The epilogue reads the
// accumulators with tcgen05.ld: SwiGLU to f16 y (gate/up), or x route weight (down).
//
// Shared-memory operand layout (K-major, no swizzle): 8x8 core matrices of 16-byte rows;
// element (m, k) of a block at (k / 8) * LBO + (m / 8) * 128 + (m % 8) * 16 + (k % 8) * 2
// with LBO = 128 * rows / 8 (2048 B for 128 weight rows, 1024 B for 64 tokens).
#include "common.cuh"
#include "gguf.h"
#include "kernels.h"
#include "launch.cuh"
#include "tile_layout.h"
#include "k_decode.cuh"

#include <algorithm>

namespace z2b {

namespace {

constexpr int GT_M = 128;                        // weight rows per tile
constexpr int GT_N = 64;                         // routed tokens per tile
constexpr int GT_K = 256;                        // k per dequantised group
constexpr int GT_WARPS_ROWS = GT_M / 16;         // 16-row weight tiles per 128-row block
constexpr int A_BYTES = GT_M * GT_K * 2;         // 64 KB per matrix
constexpr int B_BYTES = GT_N * GT_K * 2;         // 32 KB
constexpr uint32_t A_LBO = GT_M / 8 * 128, B_LBO = GT_N / 8 * 128, CORE_SBO = 128;
// instruction descriptor, kind::f16: f32 accumulator, f16 A and B, both K-major, N, M
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(GT_N >> 3) << 17) | ((uint32_t)(GT_M >> 4) << 24);

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(lbo >> 4) << 16) | ((uint64_t)(CORE_SBO >> 4) << 32) |
           (1ull << 46);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
        :: "r"(tmem_d), "l"(da), "l"(db), "r"(kIdesc), "r"(accumulate) : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Decode k-steps s..KS-1 of one 16-row tile chunk into the A block: lane (r, q) holds
// rows r and r + 8 at k = kq + 4s with kq = kofs + q * KC / 4 a multiple of 8, so each
// store lands at a compile-time offset from the lane's two base pointers:
// (s / 2) * A_LBO + (s % 2) * 8 bytes.
template <class D, int s, int KS> struct DqLoop {
    __device__ __forceinline__ static void run(const D& dec, const uint8_t* T, int lane, uint8_t* b0, uint8_t* b1) {
        uint32_t a[4];
        dec.template frag<s>(T, lane, a);
        *reinterpret_cast<uint2*>(b0 + (s >> 1) * A_LBO + (s & 1) * 8) = make_uint2(a[0], a[2]);
        *reinterpret_cast<uint2*>(b1 + (s >> 1) * A_LBO + (s & 1) * 8) = make_uint2(a[1], a[3]);
        DqLoop<D, s + 1, KS>::run(dec, T, lane, b0, b1);
    }
};
template <class D, int KS> struct DqLoop<D, KS, KS> {
    __device__ __forceinline__ static void run(const D&, const uint8_t*, int, uint8_t*, uint8_t*) {}
};

// The lane's two base pointers into A for a chunk at k offset kofs (rows row0 + r, + 8).
template <int KC>
__device__ __forceinline__ void dq_bases(uint8_t* A, int lane, int row0, int kofs, uint8_t** b0, uint8_t** b1) {
    const int r = lane >> 2, q = lane & 3;
    const int kq8 = (kofs + q * (KC / 4)) >> 3;
    *b0 = A + kq8 * A_LBO + ((row0 + r) >> 3) * 128 + ((row0 + r) & 7) * 16;
    *b1 = A + kq8 * A_LBO + ((row0 + r + 8) >> 3) * 128 + ((row0 + r + 8) & 7) * 16;
}

constexpr int GM_WARPS = 8;                      // one 16-row weight tile per warp
constexpr int RAW_NS = 3;                        // raw weight stages per warp (K groups ahead)

// Per tile: the (K group g, matrix m) stages stream in order s = g * NMAT + m. Each warp
// bulk-copies its own 16-row tile's chunks of stage s into a ring up to RAW_NS stages
// ahead; the activation rows of group g are gathered with cp.async into one of two B
// buffers a group ahead; the single A buffer is rewritten once the MMAs of the previous
// stage have released it (tcgen05.commit -> mma_bar), then one thread issues the stage's
// MMAs.
template <int WT, int KSF, int MODE>
__global__ void __launch_bounds__(256, 1) moe_gemm_kernel(const GemvParams p) {
    using D = typename DecSel<WT, KSF>::T;
    constexpr int KC = D::KC, KS = D::KS;
    constexpr int CPG = GT_K / KC;                   // tile chunks per K group
    constexpr int NMAT = (MODE == GM_GATEUP) ? 2 : 1;
    constexpr uint32_t NCOLS = NMAT == 2 ? 128u : 64u;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* A = smem;                               // [A_BYTES]
    uint8_t* Bb = smem + A_BYTES;                    // [2][B_BYTES]
    uint8_t* raw = Bb + 2 * B_BYTES;                 // [GM_WARPS][RAW_NS][CPG * tile_bytes]
    __shared__ __align__(8) uint64_t mma_bar;
    __shared__ __align__(8) uint64_t raw_bar[GM_WARPS][RAW_NS];
    __shared__ uint32_t tmem_base;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t stage_bytes = (uint32_t)(CPG * p.tile_bytes);
    const int ns = p.n_stages;                       // raw ring depth per warp (1..RAW_NS)
    uint8_t* myraw = raw + (size_t)warp * ns * stage_bytes;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(&tmem_base)), "r"(NCOLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) mbar_init(&mma_bar, 1);
    if (lane == 0)
        for (int i = 0; i < RAW_NS; ++i) mbar_init(&raw_bar[warp][i], 1);
    fence_mbar_init();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = tmem_base;
    pdl_wait();
    pdl_release();

    // experts with GEMM routes: active[n_small .. n_active), routes [seg_mid[e], seg_off[e + 1]);
    // projections (GM_PROJ): the segments' rows over tokens [tok0, tok0 + T)
    const int n_groups = (p.chunks + CPG - 1) / CPG;
    const int n_st = n_groups * NMAT;
    int e_lo = 0, e_hi = 0, n_rb = 0, n_tiles = 0;
    if constexpr (MODE == GM_PROJ) {
        e_hi = p.n_seg;
        for (int a = 0; a < e_hi; ++a)
            n_tiles += (p.T + GT_N - 1) / GT_N * ((p.seg[a].rows + GT_M - 1) / GT_M);
    } else {
        e_lo = *p.n_small;
        e_hi = *p.n_active;
        n_rb = (p.out_rows + GT_M - 1) / GT_M;   // 128-row blocks per expert
        for (int a = e_lo; a < e_hi; ++a) {
            const int e = p.active[a];
            n_tiles += (p.seg_off[e + 1] - p.seg_mid[e] + GT_N - 1) / GT_N * n_rb;
        }
    }
    uint32_t mma_phase = 0;
    int mma_pending = 0;                             // commits not yet waited for
    uint32_t raw_phase[RAW_NS];
#pragma unroll
    for (int i = 0; i < RAW_NS; ++i) raw_phase[i] = 0;
    bool failed = false;
    auto wait_mma = [&]() {
        if (mma_pending) {
            failed = __syncthreads_or(mbar_wait(&mma_bar, mma_phase, p.err) ? 0 : 1) != 0 || failed;
            mma_phase ^= 1u;
            mma_pending = 0;
        }
    };

    for (int t = blockIdx.x; t < n_tiles && !failed; t += gridDim.x) {
        int a = e_lo, base = 0, e = 0, ne = 0, nrb = n_rb;
        for (; a < e_hi; ++a) {
            if constexpr (MODE == GM_PROJ) {
                e = a;
                ne = p.T;
                nrb = (p.seg[a].rows + GT_M - 1) / GT_M;
            } else {
                e = p.active[a];
                ne = p.seg_off[e + 1] - p.seg_mid[e];
            }
            const int nt = (ne + GT_N - 1) / GT_N * nrb;
            if (t < base + nt) break;
            base += nt;
        }
        const int tb = (t - base) / nrb, rb = (t - base) % nrb;
        int tok0;
        if constexpr (MODE == GM_PROJ) tok0 = p.tok0 + tb * GT_N;
        else tok0 = p.seg_mid[e] + tb * GT_N;
        const int nv = min(GT_N, ne - tb * GT_N);
        const int rt = rb * GT_WARPS_ROWS + warp;        // this warp's row tile
        int n_row_tiles = p.n_row_tiles;
        const uint8_t* wsrc0 = p.w0 + (size_t)e * p.expert_stride;
        const uint8_t* wsrc1 = p.w1 + (size_t)e * p.expert_stride;
        if constexpr (MODE == GM_PROJ) {
            n_row_tiles = p.seg[e].n_row_tiles;
            wsrc0 = p.seg[e].tiles;
        }
        const bool rt_ok = rt < n_row_tiles;

        // raw stage s -> this warp's ring slot s % RAW_NS
        auto issue_raw = [&](int s) {
            if (lane == 0 && rt_ok) {
                const int g = s / NMAT, m = s % NMAT, c0 = g * CPG, nc = min(CPG, p.chunks - c0);
                uint64_t* bar = &raw_bar[warp][s % ns];
                const uint8_t* src = (m == 0 ? wsrc0 : wsrc1) + ((size_t)rt * p.chunks + c0) * p.tile_bytes;
                mbar_expect_tx(bar, (uint32_t)(nc * p.tile_bytes));
                bulk_g2s(myraw + (size_t)(s % ns) * stage_bytes, src, (uint32_t)(nc * p.tile_bytes), bar);
            }
        };
        // B group g -> buffer g & 1 (token rows, 16 bytes per (token, 8-wide k chunk))
        // this thread's token column of B (fixed for the tile) and its first 8-wide k chunk
        constexpr int B_TPK = 32 * GM_WARPS / GT_N;     // threads per token (k chunks step by this)
        const int bn = tid % GT_N, bkc0 = tid / GT_N;
        const bool bn_ok = bn < nv;
        int brow = tok0 + (bn_ok ? bn : 0);
        if constexpr (MODE == GM_GATEUP) brow = p.route_tok[brow];
        const __half* bsrc = p.X + (size_t)brow * p.ldx;
        auto issue_b = [&](int g) {
            uint8_t* bdst = Bb + (g & 1) * B_BYTES + (bn >> 3) * 128 + (bn & 7) * 16;
            const int kg = g * CPG * KC, klim = min(GT_K, p.K - kg);
#pragma unroll
            for (int j = 0; j < GT_K / 8 / B_TPK; ++j) {
                const int kc = bkc0 + j * B_TPK;
                const bool ok = bn_ok && kc * 8 < klim;
                cp_async16(bdst + kc * B_LBO, bsrc + kg + (ok ? kc * 8 : 0), ok);
            }
            cp_async_commit();
        };

        for (int s = 0; s < ns && s < n_st; ++s) issue_raw(s);
        issue_b(0);
        for (int s = 0; s < n_st && !failed; ++s) {
            const int g = s / NMAT, m = s % NMAT, c0 = g * CPG, nc = min(CPG, p.chunks - c0);
            // raw weights of this stage have landed (warp-local); the A buffer (and at a new
            // group, the other B buffer) is free once the previous stage's MMAs completed.
            // One block-wide vote per stage keeps every thread on the same path.
            const int slot = s % ns;
            bool f = false;
            if (rt_ok) {
                f = !mbar_wait(&raw_bar[warp][slot], raw_phase[slot], p.err);
                raw_phase[slot] ^= 1u;
            }
            if (mma_pending) {
                f = !mbar_wait(&mma_bar, mma_phase, p.err) || f;
                mma_phase ^= 1u;
                mma_pending = 0;
            }
            failed = __syncthreads_or(f ? 1 : 0) != 0;
            if (failed) break;
            if (m == 0 && g + 1 < n_groups) issue_b(g + 1);
            // dequantise this warp's row tile into A
            const uint8_t* T0 = myraw + (size_t)slot * stage_bytes;
#pragma unroll
            for (int cc = 0; cc < CPG; ++cc) {
                uint8_t *b0, *b1;
                dq_bases<KC>(A, lane, 16 * warp, cc * KC, &b0, &b1);
                if (rt_ok && cc < nc) {
                    const uint8_t* T = T0 + cc * p.tile_bytes;
                    D dec;
                    dec.prep(T, lane);
                    DqLoop<D, 0, KS>::run(dec, T, lane, b0, b1);
                } else {
                    // rows past the matrix or k past K: zeros
#pragma unroll
                    for (int s2 = 0; s2 < KS; ++s2) {
                        *reinterpret_cast<uint2*>(b0 + (s2 >> 1) * A_LBO + (s2 & 1) * 8) = make_uint2(0u, 0u);
                        *reinterpret_cast<uint2*>(b1 + (s2 >> 1) * A_LBO + (s2 & 1) * 8) = make_uint2(0u, 0u);
                    }
                }
            }
            __syncwarp();
            if (s + ns < n_st) { fence_proxy_async(); issue_raw(s + ns); }
            // activation rows of group g complete (the newest group may still be in flight)
            if (m == 0) { if (g + 1 < n_groups) cp_async_wait_1(); else cp_async_wait_0(); }
            fence_proxy_async();                     // generic-proxy writes -> tensor core reads
            tc_fence_before();
            __syncthreads();
            if (tid == 0) {
                tc_fence_after();
                const uint8_t* Bs = Bb + (g & 1) * B_BYTES;
                const int kblocks = nc * KC / 16;
                for (int kb = 0; kb < kblocks; ++kb) {
                    const uint64_t da = umma_desc(smem_u32(A) + 2 * kb * A_LBO, A_LBO);
                    const uint64_t db = umma_desc(smem_u32(Bs) + 2 * kb * B_LBO, B_LBO);
                    umma_f16(tm + m * GT_N, da, db, (g > 0 || kb > 0) ? 1u : 0u);
                }
                umma_commit(&mma_bar);
            }
            mma_pending = 1;
        }
        wait_mma();
        cp_async_wait_0();
        tc_fence_after();
        if (!failed) {
            // epilogue: warp w reads TMEM lanes 32 (w % 4).., token columns 32 (w / 4) ..
            const int row = rb * GT_M + 32 * (warp & 3) + lane;
            const int row_lim = MODE == GM_PROJ ? p.seg[e].rows : p.out_rows;
            const uint32_t lane_addr = tm + ((uint32_t)(32 * (warp & 3)) << 16);
#pragma unroll 1
            for (int c = 32 * (warp >> 2); c < 32 * (warp >> 2) + 32; c += 16) {
                float v0[16], v1[16];
                tmem_ld16(lane_addr + c, v0);
                if constexpr (NMAT == 2) tmem_ld16(lane_addr + GT_N + c, v1);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int n = c + i;
                    if (n >= nv || row >= row_lim) continue;
                    if constexpr (MODE == GM_GATEUP) {
                        const float gt = v0[i], up = v1[i];
                        const float si = gt / (1.0f + expf(-gt));
                        p.yout[(size_t)(tok0 + n) * p.ldy + row] = __float2half_rn(up * si);
                    } else if constexpr (MODE == GM_PROJ) {
                        float* o = p.out + (size_t)(tok0 + n) * p.ldo + p.seg[e].out_off + row;
                        if (p.epi == EPI_ADD) *o = v0[i] + *o;
                        else if (p.epi == EPI_SOFTCAP) *o = tanhf(v0[i] * (1.0f / p.cap)) * p.cap;
                        else *o = v0[i];
                    } else {
                        p.out[(size_t)(tok0 + n) * p.ldo + row] = v0[i] * p.route_w[tok0 + n];
                    }
                }
            }
        }
        tc_fence_before();
        __syncthreads();                                 // accumulators read before the next tile
        tc_fence_after();
    }
    // after a failure: copies and MMAs still in flight finish (bounded) before release
    if (failed) {
        if (lane == 0)
            for (int i = 0; i < ns; ++i) (void)mbar_wait(&raw_bar[warp][i], raw_phase[i], nullptr, 1u << 12);
        (void)mbar_wait(&mma_bar, mma_phase, nullptr, 1u << 12);
        cp_async_wait_0();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tm), "r"(NCOLS) : "memory");
}

template <int WT, int KSF>
void gemm_typed(const GemvParams& p, int grid, cudaStream_t s) {
    void (*k)(const GemvParams) = p.mode == GM_GATEUP ? moe_gemm_kernel<WT, KSF, GM_GATEUP>
                                  : p.mode == GM_PROJ ? moe_gemm_kernel<WT, KSF, GM_PROJ>
                                                      : moe_gemm_kernel<WT, KSF, GM_DOWN>;
    constexpr int CPG = GT_K / DecSel<WT, KSF>::T::KC;
    // deepest raw ring (up to RAW_NS stages) that fits next to A and the two B buffers
    const int per_stage = GM_WARPS * CPG * p.tile_bytes;
    const int budget = 227 * 1024 - 1024 - A_BYTES - 2 * B_BYTES;
    GemvParams q = p;
    q.n_stages = std::max(1, std::min(RAW_NS, budget / per_stage));
    const int smem = A_BYTES + 2 * B_BYTES + q.n_stages * per_stage;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    launch_pdl(k, dim3(grid), dim3(32 * GM_WARPS), (size_t)smem, s, q);
}

}  // namespace

bool moe_gemm_supported(const DevMat& m) {
    switch (m.type) {
        case GT_Q4_K: case GT_Q6_K: return true;              // 256-wide chunks
        case GT_Q8_0: return true;                            // 128-wide chunks, two per group
        case GT_F16: return m.steps == 4;                     // 64-wide chunks, four per group
        default: return false;
    }
}

void launch_moe_gemm(const GemvParams& p, int grid, cudaStream_t s) {
    switch (p.type) {
        case GT_Q4_K: gemm_typed<GT_Q4_K, 16>(p, grid, s); break;
        case GT_Q6_K: gemm_typed<GT_Q6_K, 16>(p, grid, s); break;
        case GT_Q8_0: gemm_typed<GT_Q8_0, 8>(p, grid, s); break;
        case GT_F16: gemm_typed<GT_F16, 4>(p, grid, s); break;
        default: break;
    }
}

}  // namespace z2b
