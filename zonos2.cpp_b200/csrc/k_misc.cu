// k_misc.cu — step packing, embedding, MoE combine and the device sampler (sm_100a).
#include "common.cuh"
#include "gguf.h"
#include "kernels.h"
#include "launch.cuh"
#include "quant.h"

#include <algorithm>
#include <vector>

namespace z2b {

namespace {

// ---------------------------------------------------------------- packer
// Device-side ragged packing: prefix sums over the per-stream row counts give each
// stream's token range; every token gets (slot, logical position, input row) and
// streams that want logits get an output row. Replaces the host fill of ids / pos /
// mask in zonos2_batch_step (src/zonos2-graph.cpp:784-812); no dense mask is built,
// attention reads each token's slot and position directly. Single-row descriptors
// (decode) take tokens [0, T_dec) in descriptor order and the rows of prompt chunks
// follow, so the projections can run the decode rows on the tile GEMV and the prompt
// rows on the tensor-core GEMM. Input rows and output rows stay in descriptor order.
__global__ void pack_kernel(const StepBufs b, int T) {
    __shared__ int s_in[1024], s_out[1024], s_dec[1024], s_prm[1024];
    const int n = b.n_desc, tid = threadIdx.x;
    if (tid == 0) *b.err = 0;          // first kernel of a step: clear the error word
    auto n_out_of = [](const SlotDesc& d) {
        return (d.flags & SD_OUTPUT) ? ((d.flags & SD_ALL_ROWS) ? d.n_new : 1) : 0;
    };
    if (tid < n) {
        const SlotDesc d = b.descs[tid];
        s_in[tid] = d.n_new;
        s_out[tid] = n_out_of(d);
        s_dec[tid] = d.n_new == 1 ? 1 : 0;
        s_prm[tid] = d.n_new == 1 ? 0 : d.n_new;
    }
    __syncthreads();
    // Hillis-Steele inclusive scans (n <= 1024)
    for (int off = 1; off < n; off <<= 1) {
        int a = 0, c = 0, e = 0, f = 0;
        if (tid < n && tid >= off) { a = s_in[tid - off]; c = s_out[tid - off]; e = s_dec[tid - off]; f = s_prm[tid - off]; }
        __syncthreads();
        if (tid < n && tid >= off) { s_in[tid] += a; s_out[tid] += c; s_dec[tid] += e; s_prm[tid] += f; }
        __syncthreads();
    }
    const int t_dec = n > 0 ? s_dec[n - 1] : 0;
    for (int i = tid; i < n; i += blockDim.x) {
        const SlotDesc d = b.descs[i];
        const int in0 = s_in[i] - d.n_new;                                // first input row
        const int start = d.n_new == 1 ? s_dec[i] - 1 : t_dec + s_prm[i] - d.n_new;   // first token
        const bool all = (d.flags & SD_ALL_ROWS) != 0;
        const int orow = (d.flags & SD_OUTPUT) ? s_out[i] - 1 : -1;    // the desc's last row
        const int obase = orow >= 0 ? s_out[i] - n_out_of(d) : -1;
        b.desc_out[i] = orow;
        for (int r = 0; r < d.n_new; ++r) {
            const int t = start + r;
            if (t >= T || in0 + r >= T) { atomicOr(b.err, (uint32_t)DERR_BOUNDS); break; }
            b.tok_slot[t] = d.slot;
            b.tok_pos[t] = d.n_past + r;
            b.tok_desc[t] = i;
            b.tok_out[t] = orow < 0 ? -1 : (all ? obase + r : (r == d.n_new - 1 ? orow : -1));
            for (int c = 0; c < NCOL; ++c) b.ids[t * NCOL + c] = b.ids_in[(in0 + r) * NCOL + c];
        }
        if (orow >= 0)
            for (int o = obase; o <= orow; ++o) { b.out_tok[o] = start + d.n_new - 1 - (orow - o); b.out_desc[o] = i; }
    }
    // Attention work list: token t needs ceil((pos + 1) / split_keys) split blocks; the
    // (token, split) pairs are listed in token order, so the attention grid's blocks with
    // work come first and start in one wave.
    __syncthreads();                   // every token's position is written
    const int per = (T + blockDim.x - 1) / blockDim.x;
    const int t0 = min(T, tid * per), t1 = min(T, t0 + per);
    int cnt = 0;
    auto n_splits = [&](int t) { return min(max(b.tok_pos[t], 0) / b.split_keys + 1, b.max_split); };
    for (int t = t0; t < t1; ++t) cnt += n_splits(t);
    s_in[tid] = cnt;
    __syncthreads();
    for (int off = 1; off < (int)blockDim.x; off <<= 1) {
        const int a = tid >= off ? s_in[tid - off] : 0;
        __syncthreads();
        s_in[tid] += a;
        __syncthreads();
    }
    int item = s_in[tid] - cnt;
    for (int t = t0; t < t1; ++t) {
        const int ns = n_splits(t);
        for (int sp = 0; sp < ns; ++sp) b.attn_items[item++] = make_int2(t, sp);
    }
    if (tid == (int)blockDim.x - 1) *b.attn_n_items = s_in[tid];
}

// ---------------------------------------------------------------- embedding
// Element j of row `id` of a GGUF table, dequantised with gguf-py's rounding order.
__device__ __forceinline__ float emb_elem(const uint8_t* tbl, uint32_t type, size_t row_bytes, int id, int j) {
    const uint8_t* row = tbl + (size_t)id * row_bytes;
    switch (type) {
        case GT_F32: return ((const float*)row)[j];
        case GT_F16: return __half2float(((const __half*)row)[j]);
        case GT_Q8_0: {
            const uint8_t* blk = row + (j / 32) * 34;
            return __fmul_rn((float)(int8_t)blk[2 + (j % 32)], __half2float(*(const __half*)blk));
        }
        case GT_Q4_K: {
            const uint8_t* blk = row + (j / 256) * 144;
            const int n = j % 256, sb = n / 32, i = n % 32;
            const uint8_t* s = blk + 4;
            int sc, m;
            if (sb < 4) { sc = s[sb] & 63; m = s[sb + 4] & 63; }
            else { sc = (s[sb + 4] & 0x0f) | ((s[sb - 4] >> 6) << 4); m = (s[sb + 4] >> 4) | ((s[sb] >> 6) << 4); }
            const float d = __half2float(*(const __half*)blk), dmin = __half2float(*(const __half*)(blk + 2));
            const int q = (blk[16 + (sb / 2) * 32 + i] >> (4 * (sb & 1))) & 15;
            return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)m));
        }
        case GT_Q6_K: {
            const uint8_t* blk = row + (j / 256) * 210;
            const int n = j % 256, g = n / 32, i = n % 32;
            const int lo = (blk[(g / 4) * 64 + (g % 2) * 32 + i] >> (4 * ((g % 4) / 2))) & 15;
            const int hi = (blk[128 + (g / 4) * 32 + i] >> (2 * (g % 4))) & 3;
            const float d = __half2float(*(const __half*)(blk + 208));
            return __fmul_rn(__fmul_rn(d, (float)(int8_t)blk[192 + n / 16]), (float)((lo | (hi << 4)) - 32));
        }
        default: return 0.0f;
    }
}

// emb = sum of 10 table rows (src/zonos2-graph.cpp:249-259), or for token spk_t the
// speaker row, which replaces the sum (:262-292); x = rms_norm(emb) seeds the residual
// (:300), cur = rms_norm(x) * attn_norm[0] feeds layer 0 (:343).
__global__ void __launch_bounds__(1024) embed_kernel(const StepBufs b, const EmbedDev e, const float* __restrict__ w0,
                                                     const Dims dm, int spk_t, const float* __restrict__ spk_row) {
    extern __shared__ float sh[];
    pdl_wait();
    pdl_release();
    float* emb = sh;                      // [d]
    float* red = sh + dm.n_embd;          // [32]
    const int t = blockIdx.x, d = dm.n_embd;
    const int* id = b.ids + t * NCOL;
    int idc[NCOL];
    bool bad = false;
    for (int c = 0; c < NCOL; ++c) {
        int v = id[c];
        const int lim = c < dm.n_codebooks ? dm.audio_vocab : dm.text_vocab + 1;
        if (v < 0 || v >= lim) { bad = true; v = 0; }
        idc[c] = v;
    }
    if (bad && threadIdx.x == 0) atomicOr(b.err, (uint32_t)DERR_BOUNDS);
    float ss = 0.0f;
    const bool spk = t == spk_t;
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
        float acc = 0.0f;
        if (spk) {
            acc = spk_row[j];
        } else {
            for (int c = 0; c < NCOL; ++c) {
                const uint8_t* tbl = c < dm.n_codebooks ? e.audio[c] : e.text;
                const float v = emb_elem(tbl, e.type, e.row_bytes, idc[c], j);
                acc = (c == 0) ? v : __fadd_rn(acc, v);
            }
        }
        emb[j] = acc;
        ss += acc * acc;
    }
    ss = block_sum(ss, red);
    const float sc = 1.0f / sqrtf(ss / (float)d + dm.rms_eps);
    float ss2 = 0.0f;
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
        const float x = emb[j] * sc;
        emb[j] = x;
        b.res[(size_t)t * d + j] = x;
        ss2 += x * x;
    }
    ss2 = block_sum(ss2, red);
    const float sc2 = 1.0f / sqrtf(ss2 / (float)d + dm.rms_eps);
    for (int j = threadIdx.x; j < d; j += blockDim.x)
        b.cur[(size_t)t * d + j] = __float2half_rn((emb[j] * sc2) * w0[j]);
}

// ---------------------------------------------------------------- speaker injection
// s_lda = W_lda spk + b_lda (spk_dim -> lda_dim), s_proj = W_proj s_lda + b_proj
// (lda_dim -> n_embd), + the emotion delta when given (src/zonos2-graph.cpp:262-275). One
// block; a warp per output row, lane-strided f32 products summed in a fixed order.
__global__ void __launch_bounds__(1024) spk_proj_kernel(const float* __restrict__ lda_w, const float* __restrict__ lda_b,
                                                        const float* __restrict__ proj_w, const float* __restrict__ proj_b,
                                                        const float* __restrict__ spk, const float* __restrict__ delta,
                                                        int spk_dim, int lda_dim, int n_embd, float* __restrict__ row) {
    extern __shared__ float sl[];                 // [lda_dim]
    pdl_wait();
    pdl_release();
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int i = w; i < lda_dim; i += nw) {
        const float* wr = lda_w + (size_t)i * spk_dim;
        float acc = 0.0f;
        for (int k = lane; k < spk_dim; k += 32) acc += wr[k] * spk[k];
        acc = warp_sum(acc);
        if (lane == 0) sl[i] = acc + lda_b[i];
    }
    __syncthreads();
    for (int j = w; j < n_embd; j += nw) {
        const float* wr = proj_w + (size_t)j * lda_dim;
        float acc = 0.0f;
        for (int k = lane; k < lda_dim; k += 32) acc += wr[k] * sl[k];
        acc = warp_sum(acc);
        if (lane == 0) {
            float v = acc + proj_b[j];
            if (delta) v = v + delta[j];
            row[j] = v;
        }
    }
}

// ---------------------------------------------------------------- MoE combine
// x = sum_j out_route[pos(t, j)] in top-k order (src/zonos2-graph.cpp:232-238), then the
// residual fold res = x + res (:332/:353) and the next block's input norm
// (attn_norm of layer L+1, or output_norm after the last layer for output tokens).
__global__ void __launch_bounds__(512) moe_combine_kernel(const StepBufs b, int k, const float* __restrict__ next_norm,
                                                          const float* __restrict__ out_norm, const Dims dm, int last) {
    __shared__ float red[32];
    // the token's slot, output row and route positions come from the packer and the router,
    // both complete before the predecessor started: read through L2 before the wait
    const int t = blockIdx.x, d = dm.n_embd, d4 = d / 4;
    const bool active = __ldcg(b.tok_slot + t) >= 0;
    const int orow = __ldcg(b.tok_out + t);
    int pos[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) pos[j] = (active && j < k) ? __ldcg(b.route_pos + t * b.kmax + j) : -1;
    pdl_wait();
    pdl_release();
    float4* res = reinterpret_cast<float4*>(b.res + (size_t)t * d);
    float ss = 0.0f;
    for (int i = threadIdx.x; i < d4; i += blockDim.x) {
        float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (pos[j] < 0) continue;
            const float4 v = reinterpret_cast<const float4*>(b.out_route + (size_t)pos[j] * d)[i];
            if (j == 0) x = v;
            else { x.x = __fadd_rn(x.x, v.x); x.y = __fadd_rn(x.y, v.y); x.z = __fadd_rn(x.z, v.z); x.w = __fadd_rn(x.w, v.w); }
        }
        float4 r = res[i];
        r.x = __fadd_rn(x.x, r.x); r.y = __fadd_rn(x.y, r.y); r.z = __fadd_rn(x.z, r.z); r.w = __fadd_rn(x.w, r.w);
        res[i] = r;
        ss += r.x * r.x + r.y * r.y + r.z * r.z + r.w * r.w;
    }
    if (last && orow < 0) return;              // uniform per block
    ss = block_sum(ss, red);
    const float sc = 1.0f / sqrtf(ss / (float)d + dm.rms_eps);
    const float* w = last ? out_norm : next_norm;
    __half* dst = last ? b.hout + (size_t)orow * d : b.cur + (size_t)t * d;
    for (int i = threadIdx.x; i < d4; i += blockDim.x) {
        const float4 r = res[i];
        const float4 ww = reinterpret_cast<const float4*>(w)[i];
        __half2* o = reinterpret_cast<__half2*>(dst) + 2 * i;
        o[0] = __floats2half2_rn((r.x * sc) * ww.x, (r.y * sc) * ww.y);
        o[1] = __floats2half2_rn((r.z * sc) * ww.z, (r.w * sc) * ww.w);
    }
}

// ---------------------------------------------------------------- sampler
// One block per (output row, codebook); mirrors zonos2_sampler::sample
// (src/zonos2-sampler.cpp:16-77) and the history update of accept() (:9-14).
constexpr int SORT_N = 2048;

__device__ __forceinline__ bool before(float va, int ia, float vb, int ib) {   // descending value, ascending index
    return va > vb || (va == vb && ia < ib);
}

// Block-wide bitonic sort of (v, i)[SORT_N] into descending value, ascending index; entries
// from n on are padding (-inf, INT_MAX). Ends with a barrier.
__device__ void sort_desc(float* v, int* ix, int n) {
    for (int i = n + threadIdx.x; i < SORT_N; i += blockDim.x) { v[i] = -INFINITY; ix[i] = 0x7fffffff; }
    __syncthreads();
    for (int size = 2; size <= SORT_N; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < SORT_N; i += blockDim.x) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool asc = (i & size) == 0;     // segment direction
                    const bool sw = asc ? before(v[j], ix[j], v[i], ix[i]) : before(v[i], ix[i], v[j], ix[j]);
                    if (sw) { float tv = v[i]; v[i] = v[j]; v[j] = tv; int ti = ix[i]; ix[i] = ix[j]; ix[j] = ti; }
                }
            }
            __syncthreads();
        }
}

__global__ void __launch_bounds__(256) sampler_kernel(const StepBufs b, const SampDev* __restrict__ samp,
                                                      int* hist, int* hist_len, int hist_cap, const Dims dm) {
    __shared__ float lv[SORT_N];
    __shared__ int li[SORT_N];
    __shared__ float pv[SORT_N];
    __shared__ float sv[SORT_N];                // probability order when every token is a candidate
    __shared__ int si[SORT_N];
    __shared__ unsigned char keep[SORT_N];
    __shared__ int s_code;
    pdl_wait();
    pdl_release();
    const int o = blockIdx.x, cb = blockIdx.y, av = dm.audio_vocab;
    const int di = b.out_desc[o];
    const SlotDesc D = b.descs[di];
    if (!(D.flags & SD_SAMPLE)) return;
    const SampDev sp = samp[D.samp];
    const float* lg = b.logits + ((size_t)o * dm.n_codebooks + cb) * av;
    const float* lu = nullptr;
    if (D.twin >= 0) {
        const int to = b.desc_out[D.twin];
        if (to >= 0) lu = b.logits + ((size_t)to * dm.n_codebooks + cb) * av;
    }
    for (int i = threadIdx.x; i < av; i += blockDim.x) {
        float v = lg[i];
        if (lu) v = __fadd_rn(lu[i], __fmul_rn(D.cfg_scale, __fsub_rn(v, lu[i])));   // src/zonos2-graph.cpp:917-918
        lv[i] = v;
        li[i] = i;
    }
    __syncthreads();
    int* h = hist + ((size_t)D.slot * dm.n_codebooks + cb) * hist_cap;
    int* hl = hist_len + D.slot * dm.n_codebooks + cb;
    if (sp.greedy) {
        if (threadIdx.x == 0) {
            int best = 0; float bv = lv[0];
            for (int i = 1; i < av; ++i) if (lv[i] > bv) { bv = lv[i]; best = i; }
            s_code = best;
        }
    } else {
        if (threadIdx.x == 0) {
            if (sp.rep_penalty != 1.0f && cb < sp.rep_codebooks) {
                const int n = *hl, from = max(0, n - sp.rep_window);
                for (int i = from; i < n; ++i) {
                    const int tk = h[i % hist_cap];
                    if (tk >= 0 && tk < av) lv[tk] = lv[tk] > 0.0f ? lv[tk] / sp.rep_penalty : lv[tk] * sp.rep_penalty;
                }
            }
        }
        __syncthreads();
        if (sp.temperature > 0.0f)
            for (int i = threadIdx.x; i < av; i += blockDim.x) lv[i] = lv[i] / sp.temperature;
        const int k = (sp.top_k > 0 && sp.top_k < av) ? sp.top_k : av;
        const bool use_p = sp.top_p > 0.0f && sp.top_p < 1.0f;
        if (k < av) {
            // candidates: the top k logits in descending order, ties by position (the order
            // std::partial_sort gives when ties are broken by index)
            __syncthreads();
            sort_desc(lv, li, av);
        }
        __syncthreads();
        // Softmax over the candidates in candidate order with a double sum (:48-53); exp is
        // taken in double and rounded once to float, the correctly rounded expf of the host
        // libm the reference calls.
        if (threadIdx.x == 0) {
            float mx = -1e30f;
            for (int j = 0; j < k; ++j) mx = fmaxf(mx, lv[j]);
            double sum = 0.0;
            for (int j = 0; j < k; ++j) { pv[j] = (float)exp((double)(lv[j] - mx)); sum += (double)pv[j]; }
            for (int j = 0; j < k; ++j) pv[j] = (float)((double)pv[j] / sum);
        }
        __syncthreads();
        // top-p walks the candidates by descending probability (:55-63). After a top-k cut
        // that order is the candidate order itself (probabilities follow the logits); with
        // every token a candidate, the (probability, position) pairs are sorted first.
        const float* pord = pv;
        const int* iord = nullptr;
        if (use_p && k == av) {
            for (int i = threadIdx.x; i < SORT_N; i += blockDim.x) {
                sv[i] = i < av ? pv[i] : -INFINITY;
                si[i] = i < av ? i : 0x7fffffff;
            }
            __syncthreads();
            sort_desc(sv, si, av);
            __syncthreads();
            pord = sv;
            iord = si;
        }
        if (threadIdx.x == 0) {
            float pmax = 0.0f;
            for (int j = 0; j < k; ++j) pmax = fmaxf(pmax, pv[j]);
            for (int j = 0; j < k; ++j) keep[j] = 1;
            if (use_p) {
                double cc = 0.0;
                bool done = false;
                for (int r = 0; r < k; ++r) {
                    const int j = iord ? iord[r] : r;
                    if (done) keep[j] = 0;
                    cc += (double)pord[r];
                    if (cc >= (double)sp.top_p) done = true;
                }
            }
            const float thr = sp.min_p * pmax;                     // min-p (:64-67)
            double s2 = 0.0;
            int top = 0;                                           // first candidate of the largest probability
            for (int j = 0; j < k; ++j) {
                if (pv[j] > pv[top]) top = j;
                if (sp.min_p > 0.0f && pv[j] < thr) keep[j] = 0;
                if (!keep[j]) pv[j] = 0.0f;
                s2 += (double)pv[j];
            }
            int code = li[top];
            if (s2 > 0.0) {                                        // CDF walk with one draw (:70-75)
                const double r = b.canon[(size_t)o * dm.n_codebooks + cb] * s2;
                double acc = 0.0;
                for (int j = 0; j < k; ++j) { acc += (double)pv[j]; if (acc >= r) { code = li[j]; break; } }
            }
            s_code = code;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        b.codes[(size_t)o * dm.n_codebooks + cb] = s_code;
        const int n = *hl;
        h[n % hist_cap] = s_code;
        *hl = n + 1;
    }
}

__global__ void feed_kernel(SlotDesc* descs, int n, int* ids_in, const int* codes, const int* desc_out,
                            double* canon_dst, const double* canon_src, int ncb, int text_pad, int advance) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    if (advance) {
        const int o = desc_out[i];
        for (int c = 0; c < ncb; ++c) ids_in[i * NCOL + c] = o >= 0 ? codes[o * ncb + c] : 0;
        ids_in[i * NCOL + ncb] = text_pad;
        descs[i].n_past += 1;
    }
    for (int c = 0; c < ncb; ++c) canon_dst[i * ncb + c] = canon_src[i * ncb + c];
}

__global__ void dequant_rows_kernel(const uint8_t* rows, uint32_t type, size_t row_bytes, int n_rows, int K, float* out) {
    const int r = blockIdx.x;
    if (r >= n_rows) return;
    for (int j = threadIdx.x; j < K; j += blockDim.x) out[(size_t)r * K + j] = emb_elem(rows, type, row_bytes, r, j);
}

// Scheduled device loop: install step s's descriptors and input rows. Rows of streams
// with src >= 0 come from the uploaded prompt rows; a stream with src < 0 is fed its
// previous sampled frame (output row i of the previous step) plus the text pad.
__global__ void sched_feed_kernel(const SlotDesc* step_descs, const int* src, int n, SlotDesc* descs, int* ids_in,
                                  const int* codes, const int* rows, const double* canon_src, double* canon_dst,
                                  int ncb, int text_pad) {
    __shared__ int start[1024];
    const int tid = threadIdx.x;
    if (tid < n) start[tid] = step_descs[tid].n_new;
    __syncthreads();
    for (int off = 1; off < n; off <<= 1) {
        int a = 0;
        if (tid < n && tid >= off) a = start[tid - off];
        __syncthreads();
        if (tid < n && tid >= off) start[tid] += a;
        __syncthreads();
    }
    for (int i = tid; i < n; i += blockDim.x) {
        const SlotDesc d = step_descs[i];
        descs[i] = d;
        const int t0 = start[i] - d.n_new;
        if (src[i] >= 0) {
            for (int r = 0; r < d.n_new; ++r)
                for (int c = 0; c < NCOL; ++c) ids_in[(t0 + r) * NCOL + c] = rows[(src[i] + r) * NCOL + c];
        } else {
            for (int c = 0; c < ncb; ++c) ids_in[t0 * NCOL + c] = codes[i * ncb + c];
            ids_in[t0 * NCOL + ncb] = text_pad;
        }
        for (int c = 0; c < ncb; ++c) canon_dst[i * ncb + c] = canon_src[i * ncb + c];
    }
}

}  // namespace

void launch_sched_feed(const SlotDesc* step_descs, const int* src, int n, SlotDesc* descs, int* ids_in,
                       const int* codes, const int* rows, const double* canon_src, double* canon_dst, int ncb,
                       int text_pad, cudaStream_t s) {
    sched_feed_kernel<<<1, 1024, 0, s>>>(step_descs, src, n, descs, ids_in, codes, rows, canon_src, canon_dst, ncb,
                                         text_pad);
}

void launch_dequant_rows(const uint8_t* rows_dev, uint32_t type, size_t row_bytes, int rows, int K, float* out,
                         cudaStream_t s) {
    dequant_rows_kernel<<<rows, 256, 0, s>>>(rows_dev, type, row_bytes, rows, K, out);
}

void launch_feed(SlotDesc* descs, int n, int* ids_in, const int* codes, const int* desc_out, double* canon_dst,
                 const double* canon_src, int ncb, int text_pad, int advance, cudaStream_t s) {
    feed_kernel<<<(n + 127) / 128, 128, 0, s>>>(descs, n, ids_in, codes, desc_out, canon_dst, canon_src, ncb,
                                                text_pad, advance);
}

void launch_pack(const StepBufs& b, int T, int n_out, cudaStream_t s) {
    (void)n_out;
    pack_kernel<<<1, 1024, 0, s>>>(b, T);
}

__global__ void to_f16_kernel(const float* __restrict__ x, __half* __restrict__ y, size_t n) {
    pdl_wait();
    pdl_release();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = __float2half_rn(x[i]);
}

void launch_to_f16(const float* x, __half* y, size_t n, cudaStream_t s) {
    const int grid = (int)std::min<size_t>((n + 255) / 256, 4096);
    launch_pdl(to_f16_kernel, dim3(grid), dim3(256), 0, s, x, y, n);
}

void launch_embed(const StepBufs& b, const EmbedDev& e, const float* attn_norm0, const Dims& d, int T, int spk_t,
                  const float* spk_row, cudaStream_t s) {
    launch_pdl(embed_kernel, dim3(T), dim3(1024), (d.n_embd + 32) * sizeof(float), s, b, e, attn_norm0, d, spk_t,
               spk_row);
}

void launch_spk_proj(const float* lda_w, const float* lda_b, const float* proj_w, const float* proj_b, const float* spk,
                     const float* delta, int spk_dim, int lda_dim, int n_embd, float* row, cudaStream_t s) {
    launch_pdl(spk_proj_kernel, dim3(1), dim3(1024), (size_t)lda_dim * sizeof(float), s, lda_w, lda_b, proj_w, proj_b,
               spk, delta, spk_dim, lda_dim, n_embd, row);
}

void launch_moe_combine(const StepBufs& b, const LayerSmall& ly, const float* next_norm, const float* out_norm,
                        const Dims& d, int T, int last, cudaStream_t s) {
    launch_pdl(moe_combine_kernel, dim3(T), dim3(512), 0, s, b, ly.is_moe ? ly.top_k : 1, next_norm, out_norm, d, last);
}

void launch_sampler(const StepBufs& b, const SampDev* samp, int* hist, int* hist_len, int hist_cap,
                    const Dims& d, int n_out, cudaStream_t s) {
    if (n_out <= 0) return;
    dim3 grid(n_out, d.n_codebooks);
    launch_pdl(sampler_kernel, grid, dim3(256), 0, s, b, samp, hist, hist_len, hist_cap, d);
}

}  // namespace z2b

// Runs the device packer on host descriptors {slot, n_past, n_new, flags} (flags bit 0:
// wants an output row) and returns the per-token slot / position / output row and the
// token of each output row.
extern "C" int z2b_test_pack(const int32_t* desc4, int n, int T, int32_t* tok_slot, int32_t* tok_pos,
                             int32_t* tok_out, int32_t* out_tok) {
    using namespace z2b;
    if (n < 1 || n > 1024 || T < 1) return 1;
    std::vector<SlotDesc> d(n);
    int n_out = 0, tsum = 0;
    for (int i = 0; i < n; ++i) {
        d[i] = SlotDesc{desc4[4 * i], desc4[4 * i + 1], desc4[4 * i + 2], (desc4[4 * i + 3] & 1) ? (int)SD_OUTPUT : 0,
                        -1, 1.0f, desc4[4 * i], 0};
        n_out += (desc4[4 * i + 3] & 1) ? 1 : 0;
        tsum += desc4[4 * i + 2];
    }
    if (tsum != T) return 1;
    StepBufs b{};
    void* base = nullptr;
    constexpr int kTestSplits = 64;               // positions below 64 * 256 in the test descriptors
    const size_t bytes = (size_t)n * sizeof(SlotDesc) + (size_t)T * NCOL * 4 * 2 + (size_t)T * 16 + (size_t)n * 12 +
                         (size_t)T * kTestSplits * 8 + 8192;
    if (cudaMalloc(&base, bytes) != cudaSuccess) return 4;
    cudaMemset(base, 0, bytes);
    uint8_t* p = (uint8_t*)base;
    auto take = [&](size_t nb) { uint8_t* r = p; p += (nb + 255) / 256 * 256; return r; };
    b.descs = (const SlotDesc*)take(n * sizeof(SlotDesc));
    b.n_desc = n;
    b.ids_in = (const int*)take((size_t)T * NCOL * 4);
    b.ids = (int*)take((size_t)T * NCOL * 4);
    b.tok_slot = (int*)take(T * 4); b.tok_pos = (int*)take(T * 4); b.tok_desc = (int*)take(T * 4);
    b.tok_out = (int*)take(T * 4); b.out_tok = (int*)take(n * 4); b.out_desc = (int*)take(n * 4);
    b.desc_out = (int*)take(n * 4); b.err = (uint32_t*)take(4);
    b.attn_items = (int2*)take((size_t)T * kTestSplits * 8); b.attn_n_items = (int*)take(4);
    b.split_keys = PAGE; b.max_split = kTestSplits;
    cudaMemcpy((void*)b.descs, d.data(), n * sizeof(SlotDesc), cudaMemcpyHostToDevice);
    pack_kernel<<<1, 1024>>>(b, T);
    int rc = 0;
    if (cudaMemcpy(tok_slot, b.tok_slot, T * 4, cudaMemcpyDeviceToHost) ||
        cudaMemcpy(tok_pos, b.tok_pos, T * 4, cudaMemcpyDeviceToHost) ||
        cudaMemcpy(tok_out, b.tok_out, T * 4, cudaMemcpyDeviceToHost) ||
        cudaMemcpy(out_tok, b.out_tok, (size_t)(n_out > 0 ? n_out : 1) * 4, cudaMemcpyDeviceToHost)) rc = 4;
    cudaFree(base);
    return rc;
}
