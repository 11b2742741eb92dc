// k_dac.cu — DAC decoder kernels (sm_100a): folded-quantizer lookup, the decoder's
// convolutions as tcgen05 implicit GEMMs, and conv_out + tanh.
//
// Replaces the ggml graph of src/dac.cpp:199-245 (dac_run_decoder) and its helpers conv1d
// (:104-116), convt1d (:118-163), snake (:166-171), res_unit (:177-184), dec_block
// (:186-195) and dac_build_idx (:205-219).
//
// Convolution as a GEMM (dac_conv_kernel). Output channel o, output row t of a window:
//   y[t][o] = bias[o] + sum_{k < taps} sum_{i} x[m + k*dil - pad][i] * W[o][k][i]
// with t = m*ostride + phase - ooff. A Conv1d is one phase (ostride 1, ooff 0). A
// ConvTranspose1d with kernel 2s, stride s and padding s/2 (the decoder's upsampling) is s
// phases: output t = m*s + p - s/2 takes input rows m (tap p) and m - 1 (tap p + s), so
// phase p is a two-tap conv with dil -1 over W_p[o][j][i] = w[i][o][p + j*s], the same sum
// as the reference's GEMM + overlap-add fold (src/dac.cpp:135-162).
// Tile: 128 output channels (MMA M) x 128 rows m of one window (MMA N); the reduction runs
// over (tap, 64-channel chunk) stages. Each stage is two TMA boxes with the 128-byte swizzle:
// the weights' [128 x 64] box and the activations' [64 x 128] box at row offset k*dil - pad
// (rows before the window or past its allocation read as zeros, the convolution's zero
// padding). Roles, handing over through mbarriers: warp 0 lane 0 issues the TMA loads, warp
// 1 lane 0 the tcgen05.mma (accumulator in TMEM), warps 2-9 the epilogue: bias, residual
// add, the next snake, f32 residual stream and f16 conv input written time-major.
//
// Numerics follow the reference's CPU graph: conv inputs and weights in f16 (its im2col
// patches are f16 and ggml's f16 dot converts the f32 weights to f16), products summed in
// f32; bias, residual, snake and tanh in f32, the snake's sine from the hardware
// approximation (its error is far below the f16 rounding of the snake's output). The
// transposed convs, f32 x f32 in the reference, take f16 operands here too.
#include "common.cuh"
#include "dac.h"
#include "launch.cuh"
#include "tc05.cuh"

#include <algorithm>
#include <cstdlib>
#include <cstring>

namespace z2b {

namespace {

constexpr int BM = 128;                     // output channels per tile (MMA M)
constexpr int BN = 128;                     // rows per tile (MMA N)
constexpr int BK = 64;                      // input channels per stage
constexpr int NS = 3;                       // stages in flight (two blocks per SM)
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int EPI_WARPS = 8;                // two per TMEM lane quarter, alternating column chunks
constexpr int CONV_THREADS = 32 * (2 + EPI_WARPS);   // TMA warp, MMA warp, epilogue warps
constexpr int CONV_SMEM = 1024 + NS * (A_BYTES + B_BYTES);
constexpr uint32_t TMEM_COLS = 2 * BN;       // two accumulator buffers
constexpr int MAX_CB = 16;                  // codebooks
constexpr int OUT_TILE = 64;                // samples per conv_out block
constexpr int MAX_CFIN = 128;               // conv_out input channels (static shared-memory tile)

struct ConvK {
    const float* bias;
    const float* alpha;
    const float* inv;
    const float* xres;
    float* xout;
    __half* sout;
    const int* lw_out;
    uint32_t* err;
    int oc, oc_pad, cin_chunks, ic_pad, taps, dil, pad;
    int m_rows, n_tiles, ostride, ooff, lout, c_out_st;
    int n_win, n_tiles_total;
};

// Tile t of a launch: output-channel tile fastest (the CTAs working on one activation tile
// at the same time share it through L2), then (window, row tile), then phase.
struct ConvTile { int m0, win, n0, phase; };
__device__ __forceinline__ ConvTile conv_tile(const ConvK& p, int t) {
    const int mtc = p.oc_pad / BM, wt = p.n_win * p.n_tiles;
    const int mt = t % mtc, rest = t / mtc, y = rest % wt;
    return ConvTile{mt * BM, y / p.n_tiles, (y % p.n_tiles) * BN, rest / wt};
}

// Persistent: each CTA walks tiles blockIdx.x, + gridDim.x, ...; the accumulator is double
// buffered in TMEM (columns [0, 128) and [128, 256)), so the epilogue of one tile overlaps
// the main loop of the next.
__global__ void __launch_bounds__(CONV_THREADS, 2)
dac_conv_kernel(const ConvK p, const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // the swizzled boxes need 1024-byte alignment (the pattern follows address bits 7..9)
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* As = smem;
    uint8_t* Bs = smem + NS * A_BYTES;
    __shared__ __align__(8) uint64_t full[NS], empty[NS], acc_full[2], acc_empty[2], fin_bar;
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag;
    volatile int* ab = &abort_flag;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_total = p.n_tiles_total;

    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(&tmem_base)), "r"(TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], EPI_WARPS); }
        mbar_init(&fin_bar, 1);
        abort_flag = 0;
    }
    fence_mbar_init();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = tmem_base;
    pdl_wait();

    const int n_stages = p.taps * p.cin_chunks;
    bool ok = true;
    if (warp == 0) {
        // ---- TMA producer ----
        if (lane == 0) {
            int issued = 0;
            for (int t = blockIdx.x; t < n_total && ok; t += gridDim.x) {
                const ConvTile ti = conv_tile(p, t);
                for (int s = 0; s < n_stages && ok; ++s) {
                    const int slot = issued % NS;
                    ok = wait_ab(&empty[slot], (uint32_t)(((issued / NS) & 1) ^ 1), p.err, ab);
                    if (!ok) break;
                    const int k = s / p.cin_chunks, c = s % p.cin_chunks;
                    mbar_expect_tx(&full[slot], (uint32_t)(A_BYTES + B_BYTES));
                    tma_load_2d(As + slot * A_BYTES, &wmap, k * p.ic_pad + c * BK, ti.phase * p.oc_pad + ti.m0,
                                &full[slot]);
                    tma_load_3d(Bs + slot * B_BYTES, &xmap, c * BK, ti.n0 + k * p.dil - p.pad, ti.win, &full[slot]);
                    ++issued;
                }
            }
            if (!ok) {
                *ab = 1;
                // loads still in flight land (bounded) before the block releases its memory
                for (int G = max(0, issued - NS); G < issued; ++G)
                    (void)mbar_wait(&full[G % NS], (uint32_t)((G / NS) & 1), nullptr, 1u << 16);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- MMA issuer ----
        if (lane == 0) {
            const uint32_t idesc = idesc_f16(BM, BN);
            int consumed = 0, it = 0;
            for (int t = blockIdx.x; t < n_total && ok; t += gridDim.x, ++it) {
                const int buf = it & 1;
                // the epilogue has read this buffer's previous tile
                ok = wait_ab(&acc_empty[buf], (uint32_t)(((it >> 1) & 1) ^ 1), p.err, ab);
                if (!ok) break;
                tc_fence_after();
                const uint32_t acc = tm + (uint32_t)(buf * BN);
                for (int s = 0; s < n_stages && ok; ++s) {
                    const int slot = consumed % NS;
                    ok = wait_ab(&full[slot], (uint32_t)((consumed / NS) & 1), p.err, ab);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t sa = smem_u32(As + slot * A_BYTES), sb = smem_u32(Bs + slot * B_BYTES);
#pragma unroll
                    for (int kb = 0; kb < BK / 16; ++kb)
                        umma_f16(acc, umma_desc_sw128(sa + 32 * kb), umma_desc_sw128(sb + 32 * kb), idesc,
                                 (s > 0 || kb > 0) ? 1u : 0u);
                    umma_commit(&empty[slot]);           // the slot refills once these MMAs complete
                    ++consumed;
                }
                if (ok) umma_commit(&acc_full[buf]);
            }
            if (!ok) *ab = 1;
            // every MMA issued completes before the block releases its memory
            umma_commit(&fin_bar);
            (void)mbar_wait(&fin_bar, 0, nullptr, 1u << 16);
        }
        __syncwarp();
    } else {
        // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 = its 32 output channels, the
        // two warps of a lane quarter alternating 16-column chunks ----
        const int q = warp & 3, half = (warp - 2) >> 2;
        int it = 0;
        for (int t = blockIdx.x; t < n_total && ok; t += gridDim.x, ++it) {
            const int buf = it & 1;
            const bool w = wait_ab(&acc_full[buf], (uint32_t)((it >> 1) & 1), p.err, ab);
            ok = __all_sync(0xffffffffu, w);
            if (!ok) break;
            tc_fence_after();
            const ConvTile ti = conv_tile(p, t);
            const int oc = ti.m0 + 32 * q + lane, n0 = ti.n0, phase = ti.phase;
            const bool ch_ok = oc < p.oc;
            const float bias = ch_ok ? p.bias[oc] : 0.0f;
            const float al = (p.alpha && ch_ok) ? p.alpha[oc] : 0.0f;
            const float iv = (p.inv && ch_ok) ? p.inv[oc] : 0.0f;
            const int lw = p.lw_out[ti.win];
            const uint32_t taddr = tm + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * BN);
            const size_t wbase = (size_t)ti.win * p.lout;
#pragma unroll 1
            for (int cc = half; cc < BN / 16; cc += 2) {
                if (n0 + cc * 16 >= p.m_rows) break;     // warp-uniform
                float v[16], r[16];
                tmem_ld16(taddr + cc * 16, v);
                // column i of the chunk: GEMM row m0c + i, output row tt0 + i * ostride
                const int m0c = n0 + cc * 16, tt0 = m0c * p.ostride + phase - p.ooff;
                const long long base = ((long long)wbase + tt0) * p.c_out_st + oc;
                const long long step = (long long)p.ostride * p.c_out_st;
                // the residual may alias xout: read the chunk's 16 values before its stores, so
                // the loads issue together instead of each waiting behind the previous store
                if (p.xres) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int tt = tt0 + i * p.ostride;
                        const bool in = ch_ok && m0c + i < p.m_rows && tt >= 0 && tt < p.lout && tt < lw;
                        r[i] = in ? p.xres[base + i * step] : 0.0f;
                    }
                }
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int tt = tt0 + i * p.ostride;
                    if (m0c + i >= p.m_rows || tt < 0 || tt >= p.lout) continue;
                    const long long idx = base + i * step;
                    if (!ch_ok || tt >= lw) {
                        // the next conv reads these zeros (its zero padding); the residual
                        // stream there is never read, so xout is left as is
                        p.sout[idx] = __float2half_rn(0.0f);
                        continue;
                    }
                    float x = v[i] + bias;
                    if (p.xres) x = r[i] + x;
                    if (p.xout) p.xout[idx] = x;
                    float y = x;
                    if (p.alpha) {
                        // snake: x + sin(alpha x)^2 / alpha (inverse precomputed). The hardware
                        // sine's error (about 2^-21 absolute near zero, growing with |alpha x|)
                        // stays far below the f16 rounding of the result, the next conv's input.
                        const float sn = __sinf(__fmul_rn(x, al));
                        y = __fadd_rn(x, __fmul_rn(__fmul_rn(sn, sn), iv));
                    }
                    p.sout[idx] = __float2half_rn(y);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);   // the MMA warp may reuse this buffer
        }
        if (!ok) *ab = 1;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tm), "r"(TMEM_COLS) : "memory");
    }
    pdl_release();
}

// z[l][c] = sum_j table_j[idx_j(l)][c] + bias[c] in the reference's order (get_rows results
// added one codebook after another, then the bias: src/dac.cpp:207-215), rounded to f16
// for conv_in. idx_j(l) = codes[l + j][j] when that frame exists, else the pad id, clamped
// to [0, 1023] (the shear_up of dac_build_idx).
__global__ void dac_latent_kernel(const int32_t* __restrict__ codes, const int* __restrict__ win, int n_cb,
                                  int cb_size, int pad_id, const float* __restrict__ tables,
                                  const float* __restrict__ qbias, int latent, int lat_rows, int c_st,
                                  __half* __restrict__ out) {
    pdl_wait();
    const int w = blockIdx.y, l = blockIdx.x;
    const int coff = win[4 * w + 0], rows = win[4 * w + 1], nfr = win[4 * w + 3];
    __half* o = out + ((size_t)w * lat_rows + l) * c_st;
    if (l >= nfr) {
        for (int c = threadIdx.x; c < c_st; c += blockDim.x) o[c] = __float2half_rn(0.0f);
        pdl_release();
        return;
    }
    __shared__ int idx[MAX_CB];
    if (threadIdx.x < n_cb) {
        const int j = threadIdx.x, r = l + j;
        int v = r < rows ? codes[(size_t)(coff + r) * n_cb + j] : pad_id;
        v = max(min(v, 1023), 0);
        idx[j] = min(v, cb_size - 1);
    }
    __syncthreads();
    for (int c = threadIdx.x; c < c_st; c += blockDim.x) {
        float z = 0.0f;
        if (c < latent) {
            z = tables[(size_t)idx[0] * latent + c];
            for (int j = 1; j < n_cb; ++j) z = z + tables[((size_t)j * cb_size + idx[j]) * latent + c];
            z = z + qbias[c];
        }
        o[c] = __float2half_rn(z);
    }
    pdl_release();
}

// y[t] = tanh(b + sum_{k<7} sum_c x[t + k - 3][c] * w[k][c]) for the kept samples of each
// window (the input is already snake_out(x) in f16; the weights round to f16 as the
// reference's f16 dot product does).
__global__ void dac_out_kernel(const __half* __restrict__ in, int lin, int c_st, int c_fin,
                               const float* __restrict__ w, float b, const int64_t* __restrict__ spans,
                               float* __restrict__ audio) {
    pdl_wait();
    __shared__ float xs[(OUT_TILE + 6) * (MAX_CFIN + 1)];
    __shared__ float ws[7 * MAX_CFIN];
    const int wi = blockIdx.y;
    const int64_t s0 = spans[3 * wi], len = spans[3 * wi + 1], off = spans[3 * wi + 2];
    const int64_t j0 = (int64_t)blockIdx.x * OUT_TILE;
    if (j0 >= len) { pdl_release(); return; }
    const int ld = c_fin + 1;                         // odd stride: conflict-free column reads
    const int64_t t0 = s0 + j0 - 3;
    if (c_fin % 8 == 0 && c_st % 8 == 0) {
        // 16-byte loads of eight channels (rows start 16-byte aligned: c_st is a multiple of 8),
        // four in flight per thread before their shared-memory stores
        const int vpr = c_fin / 8, vtotal = (OUT_TILE + 6) * vpr;
        for (int i0 = threadIdx.x; i0 < vtotal; i0 += 4 * blockDim.x) {
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * blockDim.x, r = i / vpr, c8 = i % vpr;
                const int64_t t = t0 + r;
                v[u] = (i < vtotal && t >= 0 && t < lin)
                           ? *reinterpret_cast<const uint4*>(in + ((size_t)wi * lin + t) * c_st + 8 * c8)
                           : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * blockDim.x;
                if (i >= vtotal) continue;
                float* d = xs + (i / vpr) * ld + 8 * (i % vpr);
                const __half2* h = reinterpret_cast<const __half2*>(&v[u]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(h[e]);
                    d[2 * e] = f.x;
                    d[2 * e + 1] = f.y;
                }
            }
        }
    } else {
        // eight loads in flight per thread before their shared-memory stores
        const int total = (OUT_TILE + 6) * c_fin;
        for (int i0 = threadIdx.x; i0 < total; i0 += 8 * blockDim.x) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int i = i0 + u * blockDim.x, r = i / c_fin, c = i % c_fin;
                const int64_t t = t0 + r;
                v[u] = (i < total && t >= 0 && t < lin) ? __half2float(in[((size_t)wi * lin + t) * c_st + c]) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int i = i0 + u * blockDim.x;
                if (i < total) xs[(i / c_fin) * ld + i % c_fin] = v[u];
            }
        }
    }
    for (int i = threadIdx.x; i < 7 * c_fin; i += blockDim.x) ws[i] = __half2float(__float2half_rn(w[i]));
    __syncthreads();
    const int64_t j = j0 + threadIdx.x;
    if (j < len) {
        float acc = 0.0f;
        for (int k = 0; k < 7; ++k) {
            const float* xr = xs + (threadIdx.x + k) * ld;
            const float* wr = ws + k * c_fin;
            for (int c = 0; c < c_fin; ++c) acc += xr[c] * wr[c];
        }
        audio[off + j] = tanhf(acc + b);
    }
    pdl_release();
}

bool conv_attr_done[64] = {};
int conv_sms[64] = {};

}  // namespace

bool dac_make_wmap(DacConv& c) {
    auto enc = tensor_map_encoder();
    if (!enc || !c.w || c.ic_pad % BK || c.oc_pad % BM) return false;
    if (!c.wmap) c.wmap = aligned_alloc(64, 128);
    if (!c.wmap) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)c.taps * c.ic_pad, (cuuint64_t)c.phases * c.oc_pad};
    const cuuint64_t strides[1] = {(cuuint64_t)c.taps * c.ic_pad * 2};
    const cuuint32_t box[2] = {BK, BM};
    const cuuint32_t estr[2] = {1, 1};
    return enc(reinterpret_cast<CUtensorMap*>(c.wmap), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, c.w, dims, strides, box,
               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool launch_dac_conv(const DacConv& c, const DacConvIO& io, cudaStream_t s) {
    auto enc = tensor_map_encoder();
    if (!enc || !c.wmap || !io.in || !io.sout || !io.lw_out || io.n_win <= 0 || io.lin <= 0) return false;
    if (io.c_in_st < c.ic_pad || (io.c_in_st * 2) % 16 || ((uintptr_t)io.in & 15u) || io.c_out_st < c.oc_pad) return false;
    const bool convt = c.phases > 1 || c.stride > 1;
    ConvK p{};
    p.bias = c.b;
    p.alpha = io.snake ? io.snake->alpha : nullptr;
    p.inv = io.snake ? io.snake->inv : nullptr;
    p.xres = io.xres;
    p.xout = io.xout;
    p.sout = io.sout;
    p.lw_out = io.lw_out;
    p.err = io.err;
    p.oc = c.oc;
    p.oc_pad = c.oc_pad;
    p.ic_pad = c.ic_pad;
    p.cin_chunks = c.ic_pad / BK;
    p.taps = c.taps;
    p.dil = convt ? -1 : c.dil;
    p.pad = convt ? 0 : c.pad;
    p.m_rows = convt ? io.lin + 1 : io.lin;
    p.ostride = convt ? c.stride : 1;
    p.ooff = convt ? c.stride / 2 : 0;
    p.lout = io.lout;
    p.c_out_st = io.c_out_st;
    p.n_tiles = (p.m_rows + BN - 1) / BN;
    if (convt ? (io.lout != io.lin * c.stride || c.taps != 2) : io.lout != io.lin) return false;
    p.n_win = io.n_win;
    const long total = (long)(c.oc_pad / BM) * io.n_win * p.n_tiles * c.phases;
    if (total > 0x7fffffffL) return false;
    p.n_tiles_total = (int)total;
    alignas(64) CUtensorMap xmap;
    const cuuint64_t dims[3] = {(cuuint64_t)c.ic_pad, (cuuint64_t)io.lin, (cuuint64_t)io.n_win};
    const cuuint64_t strides[2] = {(cuuint64_t)io.c_in_st * 2, (cuuint64_t)io.lin * io.c_in_st * 2};
    const cuuint32_t box[3] = {BK, BN, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (enc(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(io.in), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return false;
    if (!conv_attr_done[dev]) {                       // the shared-memory opt-in is per device
        if (cudaFuncSetAttribute(dac_conv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, CONV_SMEM) != cudaSuccess ||
            cudaDeviceGetAttribute(&conv_sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return false;
        conv_attr_done[dev] = true;
    }
    // two persistent blocks per SM (TMEM: 2 x 256 columns; shared memory: 2 x 97 KB)
    const int grid = (int)std::min<long>(total, 2L * conv_sms[dev]);
    return launch_pdl(dac_conv_kernel, dim3(grid), dim3(CONV_THREADS), (size_t)CONV_SMEM, s, p,
                      *reinterpret_cast<const CUtensorMap*>(c.wmap), xmap) == cudaSuccess;
}

bool launch_dac_latent(const DacModel& m, const int32_t* codes, const int* win, int n_win, int lat_rows, int c_st,
                       __half* out, cudaStream_t s) {
    if (m.n_codebooks > MAX_CB || n_win <= 0 || lat_rows <= 0 || n_win > 65535) return false;
    return launch_pdl(dac_latent_kernel, dim3(lat_rows, n_win), dim3(256), 0, s, codes, win, m.n_codebooks,
                      m.codebook_size, m.pad_id, (const float*)m.tables, (const float*)m.qbias, m.latent, lat_rows,
                      c_st, out) == cudaSuccess;
}

bool launch_dac_out(const DacModel& m, const __half* in, int lin, int c_st, int n_win, const int64_t* spans,
                    int64_t max_span, float* audio, cudaStream_t s) {
    if (m.c_fin > MAX_CFIN || n_win <= 0 || n_win > 65535 || max_span <= 0) return false;
    const int64_t gx = (max_span + OUT_TILE - 1) / OUT_TILE;
    if (gx > 0x7fffffff) return false;
    return launch_pdl(dac_out_kernel, dim3((unsigned)gx, n_win), dim3(OUT_TILE), 0, s, in, lin, c_st, m.c_fin,
                      (const float*)m.w_out, m.b_out, spans, audio) == cudaSuccess;
}

}  // namespace z2b
