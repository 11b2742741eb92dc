// k_test.cu — device-side check entry points (declared in include/z2b_tools.h).
//
// z2b_test_dequant decodes weights on the device from the same tile image the GEMV
// reads (or from raw GGUF rows through the embedding-gather path) with gguf-py's
// rounding order, so layout and decode can be compared bit-exactly with
// gguf.quants.dequantize. z2b_test_gemv runs one projection-mode tile GEMV.
#include "common.cuh"
#include "gguf.h"
#include "kernels.h"
#include "repack.h"
#include "tile_layout.h"
#include "../../include/z2b_tools.h"

#include <cstring>
#include <vector>

namespace z2b {
namespace {

// one block per (row-tile, chunk), one warp: every lane decodes exactly the weights it
// feeds to the mma in the GEMV, using the tile_layout.h positions
__global__ void dequant_tiles_kernel(const uint8_t* tiles, uint32_t type, int rows, int K, int chunks, int tile_bytes,
                                     int steps, float* out) {
    const int t = blockIdx.x / chunks, c = blockIdx.x % chunks, lane = threadIdx.x;
    const uint8_t* T = tiles + (size_t)blockIdx.x * tile_bytes;
    const int r = lane >> 2, q = lane & 3;
    for (int half = 0; half < 2; ++half) {
        const int rr = r + 8 * half, R = t * 16 + rr;
        if (R >= rows) continue;
        float* orow = out + (size_t)R * K;
        if (type == GT_Q4_K) {
            const uint4 hd = *(const uint4*)(T + rr * 16);
            const float d = __half2float(__ushort_as_half((uint16_t)(hd.x & 0xffff)));
            const float dm = __half2float(__ushort_as_half((uint16_t)(hd.x >> 16)));
            uint32_t f;
            if (q == 0) f = hd.y;
            else if (q == 1) f = __funnelshift_r(hd.y, hd.z, 24);
            else if (q == 2) f = __funnelshift_r(hd.z, hd.w, 16);
            else f = hd.w >> 8;
            for (int s = 0; s < 16; ++s) {
                const uint4 w = *(const uint4*)(T + Q4K_HDR + ((s >> 2) * 32 + lane) * 16);
                uint32_t v = half ? ((s & 2) ? w.w : w.z) : ((s & 2) ? w.y : w.x);
                if (s & 1) v >>= 8;
                const int sb = s >> 3;
                const int sc = (f >> (6 * sb)) & 63, mm = (f >> (12 + 6 * sb)) & 63;
                const float ds = __fmul_rn(d, (float)sc), dmm = __fmul_rn(dm, (float)mm);
                const int e[4] = {(int)(v & 15), (int)((v >> 16) & 15), (int)((v >> 4) & 15), (int)((v >> 20) & 15)};
                for (int j = 0; j < 4; ++j)
                    orow[c * 256 + 64 * q + 4 * s + j] = __fsub_rn(__fmul_rn(ds, (float)e[j]), dmm);
            }
        } else if (type == GT_Q6_K) {
            const uint32_t sc4 = *(const uint32_t*)(T + rr * 16 + 4 * q);
            const float d = __half2float(*(const __half*)(T + 256 + 2 * rr));
            for (int s = 0; s < 16; ++s) {
                const uint4 w = *(const uint4*)(T + Q6K_HDR + ((s >> 2) * 32 + lane) * 16);
                const uint4 hv = *(const uint4*)(T + Q6K_HDR + Q6K_LO + ((s >> 3) * 32 + lane) * 16);
                uint32_t v = half ? ((s & 2) ? w.w : w.z) : ((s & 2) ? w.y : w.x);
                if (s & 1) v >>= 8;
                const uint32_t h = half ? (((s >> 2) & 1) ? hv.w : hv.z) : (((s >> 2) & 1) ? hv.y : hv.x);
                const int j4 = s & 3;
                const int lo[4] = {(int)(v & 15), (int)((v >> 16) & 15), (int)((v >> 4) & 15), (int)((v >> 20) & 15)};
                const int hpos[4] = {0, 16, 2, 18};
                const float ds = __fmul_rn(d, (float)(int8_t)(sc4 >> (8 * (s >> 2))));
                for (int j = 0; j < 4; ++j) {
                    const int hi = (h >> (hpos[j] + 4 * j4)) & 3;
                    orow[c * 256 + 64 * q + 4 * s + j] = __fmul_rn(ds, (float)((lo[j] | (hi << 4)) - 32));
                }
            }
        } else if (type == GT_Q8_0) {
            const float d = __half2float(*(const __half*)(T + (rr * 4 + q) * 2));
            for (int s = 0; s < 8; ++s) {
                const uint4 w = *(const uint4*)(T + Q80_HDR + ((s >> 1) * 32 + lane) * 16);
                const uint32_t v = half ? ((s & 1) ? w.w : w.z) : ((s & 1) ? w.y : w.x);
                for (int j = 0; j < 4; ++j)
                    orow[c * 128 + 32 * q + 4 * s + j] = __fmul_rn((float)((int)((v >> (8 * j)) & 255) - 128), d);
            }
        } else if (type == GT_F16) {
            for (int s = 0; s < steps; ++s) {
                const uint4 w = *(const uint4*)(T + (s * 32 + lane) * 16);
                const uint32_t a = half ? w.z : w.x, b = half ? w.w : w.y;
                const int base = c * 16 * steps + 4 * steps * q + 4 * s;
                orow[base + 0] = __half2float(__ushort_as_half((uint16_t)(a & 0xffff)));
                orow[base + 1] = __half2float(__ushort_as_half((uint16_t)(a >> 16)));
                orow[base + 2] = __half2float(__ushort_as_half((uint16_t)(b & 0xffff)));
                orow[base + 3] = __half2float(__ushort_as_half((uint16_t)(b >> 16)));
            }
        }
    }
}

}  // namespace

// embedding-path element decode (k_misc.cu)
void launch_dequant_rows(const uint8_t* rows_dev, uint32_t type, size_t row_bytes, int rows, int K, float* out,
                         cudaStream_t s);

}  // namespace z2b

using namespace z2b;

#define TCK(x) do { if ((x) != cudaSuccess) { rc = 4; goto done; } } while (0)

extern "C" int z2b_test_dequant(uint32_t type, int64_t rows, int64_t k, const void* gguf_rows, int from_tiles,
                                float* out) {
    int rc = 0;
    uint8_t *dsrc = nullptr, *dt = nullptr;
    float* dout = nullptr;
    const size_t rb = gtype_row_bytes(type, k);
    if (rb == 0) return 7;
    TCK(cudaMalloc(&dout, (size_t)rows * k * 4));
    if (from_tiles) {
        TileGeom g;
        if (!tile_geom(type, k, &g)) { rc = 7; goto done; }
        {
            const int64_t nb = tiles_bytes(type, rows, k);
            std::vector<uint8_t> img((size_t)nb);
            if (!repack_rows(type, rows, k, (const uint8_t*)gguf_rows, img.data())) { rc = 7; goto done; }
            TCK(cudaMalloc(&dt, (size_t)nb));
            TCK(cudaMemcpy(dt, img.data(), (size_t)nb, cudaMemcpyHostToDevice));
            const int ntiles = (int)((rows + 15) / 16);
            dequant_tiles_kernel<<<(unsigned)(ntiles * g.chunks), 32>>>(dt, type, (int)rows, (int)k, (int)g.chunks,
                                                                       g.tile_bytes, g.steps, dout);
        }
    } else {
        TCK(cudaMalloc(&dsrc, rb * (size_t)rows));
        TCK(cudaMemcpy(dsrc, gguf_rows, rb * (size_t)rows, cudaMemcpyHostToDevice));
        launch_dequant_rows(dsrc, type, rb, (int)rows, (int)k, dout, 0);
    }
    TCK(cudaGetLastError());
    TCK(cudaMemcpy(out, dout, (size_t)rows * k * 4, cudaMemcpyDeviceToHost));
done:
    if (dsrc) cudaFree(dsrc);
    if (dt) cudaFree(dt);
    if (dout) cudaFree(dout);
    return rc;
}

extern "C" int z2b_test_gemv_geometry(uint32_t type, int64_t k, int nmat, int ntg, int32_t* out) {
    using namespace z2b;
    TileGeom g{};
    if (!out || nmat < 1 || nmat > 2 || ntg < 1 || ntg > 2 || !tile_geom(type, k, &g)) return 7;
    DevMat m{};
    m.type = type; m.K = (int)k; m.chunks = (int)g.chunks; m.tile_bytes = g.tile_bytes; m.steps = g.steps;
    int nw = 0, ns = 0, sb = 0, smem = 0, cps = 0, xrs = 0;
    gemv_geometry(m, nmat, ntg, &nw, &ns, &sb, &smem, &cps, &xrs);
    out[0] = nw; out[1] = ns; out[2] = sb; out[3] = smem; out[4] = cps; out[5] = xrs;
    out[6] = (m.chunks + nw - 1) / nw;
    return 0;
}

extern "C" int z2b_test_gemv(uint32_t type, int64_t rows, int64_t k, const void* gguf_rows, const uint16_t* x_f16,
                             int n_tok, float* out) {
    int rc = 0;
    uint8_t* dt = nullptr;
    __half* dx = nullptr;
    float* dout = nullptr;
    uint32_t* derr = nullptr;
    uint32_t herr = 0;
    TileGeom g;
    if (!tile_geom(type, k, &g) || n_tok < 1) return 7;
    {
        const int64_t nb = tiles_bytes(type, rows, k);
        std::vector<uint8_t> img((size_t)nb);
        if (!repack_rows(type, rows, k, (const uint8_t*)gguf_rows, img.data())) return 7;
        TCK(cudaMalloc(&dt, (size_t)nb));
        TCK(cudaMemcpy(dt, img.data(), (size_t)nb, cudaMemcpyHostToDevice));
        TCK(cudaMalloc(&dx, (size_t)n_tok * k * 2));
        TCK(cudaMemcpy(dx, x_f16, (size_t)n_tok * k * 2, cudaMemcpyHostToDevice));
        TCK(cudaMalloc(&dout, (size_t)n_tok * rows * 4));
        TCK(cudaMalloc(&derr, 4));
        TCK(cudaMemset(derr, 0, 4));
        DevMat m{};
        m.tiles = dt; m.type = type; m.rows = (int)rows; m.K = (int)k;
        m.n_row_tiles = (int)((rows + 15) / 16); m.chunks = (int)g.chunks; m.tile_bytes = g.tile_bytes; m.steps = g.steps;
        GemvParams p{};
        p.mode = GM_PROJ; p.epi = EPI_STORE; p.type = type; p.K = (int)k; p.chunks = m.chunks;
        p.tile_bytes = m.tile_bytes; p.steps = m.steps;
        p.seg[0] = ProjSeg{dt, m.n_row_tiles, (int)rows, 0};
        p.n_seg = 1; p.total_items = m.n_row_tiles;
        p.X = dx; p.ldx = (int)k; p.T = n_tok; p.out = dout; p.ldo = (int)rows; p.err = derr;
        int nw, smem;
        gemv_geometry(m, 1, 2, &nw, &p.n_stages, &p.stage_bytes, &smem, &p.cps, &p.x_rs);
        int nsm = 148;
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, 0);
        launch_gemv(p, nw, m.n_row_tiles < nsm ? m.n_row_tiles : nsm, smem, 0);
        TCK(cudaGetLastError());
        TCK(cudaMemcpy(out, dout, (size_t)n_tok * rows * 4, cudaMemcpyDeviceToHost));
        TCK(cudaMemcpy(&herr, derr, 4, cudaMemcpyDeviceToHost));
        if (herr) rc = 6;
    }
done:
    if (dt) cudaFree(dt);
    if (dx) cudaFree(dx);
    if (dout) cudaFree(dout);
    if (derr) cudaFree(derr);
    return rc;
}

// The bounded wait the kernels use, on an mbarrier phase that nothing completes: the
// wait gives up after `polls` polls, records DERR_WAIT_TIMEOUT in the error word and the
// kernel returns normally, so the context stays usable.
namespace z2b {
namespace {
__global__ void wait_timeout_kernel(uint32_t polls, uint32_t* err, uint32_t* done, unsigned long long* ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        z2b::mbar_init(&bar, 1);                // one arrival expected, none will come
        z2b::fence_mbar_init();
    }
    __syncthreads();
    unsigned long long t0, t1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    const bool ok = z2b::mbar_wait(&bar, 0, err, polls);
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
    if (threadIdx.x == 0) { *done = ok ? 1u : 2u; *ns = t1 - t0; }
}
}  // namespace
}  // namespace z2b

extern "C" int z2b_test_wait_timeout(uint32_t polls, uint32_t* err_word, uint32_t* outcome, uint64_t* elapsed_ns) {
    if (!err_word || !outcome || !elapsed_ns || polls == 0 || polls > 4096) return 1;
    uint32_t* d = nullptr;
    if (cudaMalloc(&d, 16) != cudaSuccess) return 4;
    int rc = 0;
    uint32_t h[4] = {0, 0, 0, 0};
    if (cudaMemset(d, 0, 16) != cudaSuccess) rc = 4;
    if (!rc) {
        z2b::wait_timeout_kernel<<<1, 32>>>(polls, d, d + 1, reinterpret_cast<unsigned long long*>(d + 2));
        if (cudaGetLastError() != cudaSuccess || cudaMemcpy(h, d, 16, cudaMemcpyDeviceToHost) != cudaSuccess) rc = 4;
    }
    cudaFree(d);
    *err_word = h[0];
    *outcome = h[1];
    std::memcpy(elapsed_ns, h + 2, 8);
    return rc;
}
