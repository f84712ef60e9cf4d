// Decode-step kernels of the engine (sm_100a): shared structures, the
// attention, greedy bookkeeping and the encoder's embedding gather.
//
// Reference kernels they replace (crates/malaga-core/kernels/malaga.cu, launched
// by crates/malaga-core/src/kernels.rs) and candle ops (model.rs:552-612):
//   attend          attn_decode (malaga.cu:165-227), also the encoder's masked
//                   softmax attention (model.rs:101-109)
//   greedy_finalize greedy_finalize (malaga.cu:290-326)
//   embed_tokens    the encoder's embedding + position input (model.rs:270-273,
//                   455-458), gathered on the device
// The matmuls live in smallmm.cuh (at most 8 rows) and gemm_tc.cuh (more).
#pragma once
#include "engine.h"
#include "numerics.cuh"
#include "sync.cuh"

namespace mgb {

// ---------------------------------------------------------------------------
// Weight access (row layout, engine.h)

// Dequantized element i of row `row` (exact: every product below is exactly
// representable in f32, so the order of the factors does not matter).
__device__ __forceinline__ float deq_elem(const Matrix &W, int row, int i) {
    switch (W.type) {
        case T_F32: return reinterpret_cast<const float *>(W.ra)[(size_t)row * W.K + i];
        case T_Q8_0: {
            const size_t bi = (size_t)row * W.nb + (i >> 5);
            const float d = h2f(reinterpret_cast<const uint16_t *>(W.rb)[bi]);
            return __fmul_rn(d, (float)(int8_t)W.ra[bi * 32 + (i & 31)]);
        }
        case T_Q4_K: {
            const uint8_t *sb = W.ra + ((size_t)row * W.nsb + (i >> 8)) * 144;
            const int k = i & 255, j = k >> 5, l = k & 31;
            const uint8_t *s = sb + 4;
            int sc, m;
            if (j < 4) {
                sc = s[j] & 63;
                m = s[j + 4] & 63;
            } else {
                sc = (s[j + 4] & 0xf) | ((s[j - 4] >> 6) << 4);
                m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
            }
            const uint8_t byte = sb[16 + 32 * (j >> 1) + l];
            const int q = (j & 1) ? (byte >> 4) : (byte & 15);
            const float d = h2f(sb[0] | (sb[1] << 8)), dm = h2f(sb[2] | (sb[3] << 8));
            return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dm, (float)m));
        }
        case T_Q6_K: {
            const size_t u = (size_t)row * W.nsb + (i >> 8);
            const int k = i & 255, n = k >> 7, g = (k & 127) >> 5, l = k & 31;
            const uint8_t *ql = W.ra + u * 128 + 64 * n, *qh = W.rb + u * 64 + 32 * n;
            int q;
            switch (g) {
                case 0: q = (ql[l] & 0xf) | ((qh[l] & 3) << 4); break;
                case 1: q = (ql[l + 32] & 0xf) | (((qh[l] >> 2) & 3) << 4); break;
                case 2: q = (ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4); break;
                default: q = (ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4); break;
            }
            const int sc = (int8_t)W.rc[u * 16 + (k >> 4)];
            const float d = h2f(reinterpret_cast<const uint16_t *>(W.re)[u]);
            return __fmul_rn(__fmul_rn(d, (float)sc), (float)(q - 32));
        }
    }
    return 0.0f;
}

// ---------------------------------------------------------------------------
// Activation sources and matmul outputs

enum PrepMode { PREP_PLAIN = 0, PREP_LN = 1, PREP_EMBED_LN = 2 };

struct PrepArgs {
    const float *x;       // input rows [rows][K] (PLAIN, LN)
    float *x_out;         // EMBED_LN: residual stream written here
    const float *gamma, *beta;
    // EMBED_LN: x = E[id] * scale + pos_table[*step + pos_base]
    Matrix embed;
    const uint32_t *ids;
    const uint32_t *step;
    const float *pos_table;
    uint32_t pos_base;
    float scale;
    int rows, K;
};

enum Epi { EPI_STORE = 0, EPI_RELU = 1, EPI_RESID = 2, EPI_QKV = 3, EPI_CROSSKV = 4, EPI_ARGMAX = 5 };

// Where a matmul's outputs go (epilogue parameters).
struct GemvArgs {
    Matrix W;
    int rows;         // activation rows
    float *y;         // [rows][N] (STORE, RELU, RESID in place)
    // QKV: q out [rows][d]; caches [rows][H][m][hd] at slot *step, f16
    // (the fused greedy step, graph.rs:58-63) or f32 (kv_f32: the generic
    // decode's KvCache, model.rs:124-133)
    float *q;
    void *kc, *vc;
    int kv_f32;
    const uint32_t *step;
    int H, hd, m;
    // CROSSKV: f32 cross K/V [b][H][S][hd] (kc, vc), token row = bi * S + j
    int S;
    // ARGMAX: per (row, CTA) best (value, index); optional logits [rows][N]
    float *part_v;
    uint32_t *part_i;
    float *logits;
    // RELU on the tensor-core path: when qo.tq is set, the outputs go out as the
    // next matmul's q8_1 tensor-core activations (as qprep_row_kernel<PLAIN>
    // would make them from y) instead of f32 rows
    QAct qo;
};

// Epilogue of one output element (row of W, activation row n); v = the dot
// product. Bias, then the residual / ReLU / cache write of malaga.cu's fused
// kernels (bias_residual_ln: (y + bias) + resid, malaga.cu:100; bias_relu;
// qkv_decode's f16 K/V cache slot, malaga.cu:142-154).
template <int EPI>
__device__ __forceinline__ void epilogue_store(const GemvArgs &g, int row, int n, float v) {
    const Matrix &W = g.W;
    const float b = W.bias ? W.bias[row] : 0.0f;
    if constexpr (EPI == EPI_STORE) {
        g.y[(size_t)n * W.N + row] = W.bias ? __fadd_rn(v, b) : v;
    } else if constexpr (EPI == EPI_RELU) {
        const float y = __fadd_rn(v, b);
        g.y[(size_t)n * W.N + row] = y > 0.0f ? y : 0.0f;
    } else if constexpr (EPI == EPI_RESID) {
        float *xr = g.y + (size_t)n * W.N + row;
        *xr = __fadd_rn(__fadd_rn(v, b), __ldcg(xr));
    } else if constexpr (EPI == EPI_QKV) {
        const float y = __fadd_rn(v, b);
        const int dm = g.H * g.hd;
        if (row < dm) {
            g.q[(size_t)n * dm + row] = y;
        } else {
            const int c = row - dm, which = c / dm, h = (c % dm) / g.hd, t = c % g.hd;
            const size_t at = (((size_t)n * g.H + h) * g.m + *g.step) * g.hd + t;
            void *cache = which == 0 ? g.kc : g.vc;
            if (g.kv_f32) reinterpret_cast<float *>(cache)[at] = y;
            else reinterpret_cast<__half *>(cache)[at] = __float2half_rn(y);
        }
    } else if constexpr (EPI == EPI_CROSSKV) {
        const float y = __fadd_rn(v, b);
        const int dm = g.H * g.hd, which = row / dm, c = row % dm, h = c / g.hd, t = c % g.hd;
        const int bi = n / g.S, jj = n % g.S;
        float *cache = reinterpret_cast<float *>(which == 0 ? g.kc : g.vc);
        cache[(((size_t)bi * g.H + h) * g.S + jj) * g.hd + t] = y;
    }
}

// epilogue_store with its operands read beforehand: the row's bias b, the
// residual value resid (RESID) and the decode step (QKV).
template <int EPI>
__device__ __forceinline__ void epilogue_pre(const GemvArgs &g, int row, int n, float v, float b, float resid,
                                             int step) {
    const Matrix &W = g.W;
    if constexpr (EPI == EPI_STORE) {
        g.y[(size_t)n * W.N + row] = W.bias ? __fadd_rn(v, b) : v;
    } else if constexpr (EPI == EPI_RELU) {
        const float y = __fadd_rn(v, b);
        g.y[(size_t)n * W.N + row] = y > 0.0f ? y : 0.0f;
    } else if constexpr (EPI == EPI_RESID) {
        g.y[(size_t)n * W.N + row] = __fadd_rn(__fadd_rn(v, b), resid);
    } else if constexpr (EPI == EPI_QKV) {
        const float y = __fadd_rn(v, b);
        const int dm = g.H * g.hd;
        if (row < dm) {
            g.q[(size_t)n * dm + row] = y;
        } else {
            const int c = row - dm, which = c / dm, h = (c % dm) / g.hd, t = c % g.hd;
            const size_t at = (((size_t)n * g.H + h) * g.m + step) * g.hd + t;
            void *cache = which == 0 ? g.kc : g.vc;
            if (g.kv_f32) reinterpret_cast<float *>(cache)[at] = y;
            else reinterpret_cast<__half *>(cache)[at] = __float2half_rn(y);
        }
    }
}

// ---------------------------------------------------------------------------
// Tensor-core activation layout (QAct, written for the tensor-core matmul)

// Byte offset of (row r, 16-byte K chunk k16) of a K=32 int8 operand tile in
// the UMMA K-major no-swizzle layout: 8-row core groups of 256 bytes.
__host__ __device__ __forceinline__ int tile_off(int r, int k16) { return (r >> 3) * 256 + k16 * 128 + (r & 7) * 16; }

// Block j of activation row `tok` (value y at position lane) quantized to q8_1
// into the tensor-core layout: the byte into the tile, lane 0 the record.
__device__ __forceinline__ void store_block_tc(const QAct &o, int tok, int j, float y, int lane) {
    float d, s;
    const int q = q81_block(y, d, s);
    o.tq[((size_t)j * (o.rs / 8) + (tok >> 3)) * 256 + tile_off(tok & 7, lane >> 4) + (lane & 15)] =
        (uint8_t)(int8_t)q;
    if (lane == 0) o.trec[(size_t)j * o.rs + tok] = make_float2(d, s);
}

// ---------------------------------------------------------------------------
// Single-query attention: one warp per (row, head, query).

struct AttnArgs {
    const float *q;   // query base
    long q_row;       // stride between query rows (batch / token)
    const void *K, *V;
    long kv_row;      // stride between key rows (elements)
    long kv_head;     // stride between heads (elements)
    long kv_batch;    // stride between batch rows (elements)
    const uint32_t *lens;  // keys per batch row (cross / encoder)
    const uint32_t *step;  // self: keys = *step + 1
    float *out;       // [rows][H*hd]
    long out_row;
    int H, hd, rows, queries;  // queries per batch row (encoder: S)
    int max_keys;
    // Optional: the outputs also quantized to q8_1 in the next matmul's
    // tensor-core layout (qo.tq != null; single queries, hd a multiple of 32).
    QAct qo;
};

// Programmatic dependent launch: a kernel may start while its predecessor in
// the stream is still running; everything before pdl_wait() must not read the
// predecessor's outputs. Every CTA calls pdl_wait() before it exits, so a
// kernel completes only after its predecessor did (the chain stays ordered).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// HD values of a K/V row into registers (HD/8 16-byte loads for f16, HD/4 for f32).
template <int HD>
__device__ __forceinline__ void load_row(const __half *p, float (&v)[HD]) {
#pragma unroll
    for (int c = 0; c < HD / 8; ++c) {
        const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(p) + c);
        const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float2 f = __half22float2(h2[u]);
            v[8 * c + 2 * u] = f.x;
            v[8 * c + 2 * u + 1] = f.y;
        }
    }
}
template <int HD>
__device__ __forceinline__ void load_row(const float *p, float (&v)[HD]) {
#pragma unroll
    for (int c = 0; c < HD / 4; ++c) {
        const float4 f = *(reinterpret_cast<const float4 *>(p) + c);
        v[4 * c] = f.x;
        v[4 * c + 1] = f.y;
        v[4 * c + 2] = f.z;
        v[4 * c + 3] = f.w;
    }
}
__device__ __forceinline__ float load_kv(const __half *p) { return __half2float(*p); }
__device__ __forceinline__ float load_kv(const float *p) { return *p; }

// Element t of a K/V row held as raw 16-byte words.
template <typename KV, int RW>
__device__ __forceinline__ float kv_at(const uint4 (&r)[RW], int t) {
    if constexpr (sizeof(KV) == 2) return __half2float(reinterpret_cast<const __half *>(r)[t]);
    else return reinterpret_cast<const float *>(r)[t];
}

// 16 bytes global -> shared without registers (completion by cp_async_wait).
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// One (row n, head h, query qi) of single-query attention by one warp: lane
// `lane` gets the outputs of dims lane, lane+32, ... (res[c], valid when
// live). e: the warp's max_keys floats of scores; vs: its staging tile of 64 V
// rows (filled by cp.async while the scores run). Scores by an FMA chain over
// the head dimension (keys lane and lane+32 of each round of 64 side by side),
// e = exp(s - max), the sum in SUM32 order, outputs by an FMA chain over keys
// times 1/sum. Shared by the attention kernel and the fused matmul prologue.
template <typename KV, int HD>
__device__ __forceinline__ void attend_one(const AttnArgs &a, int n, int h, int qi, float *e, KV *vs, int lane,
                                           float (&res)[HD >= 32 ? HD / 32 : 1], bool &live) {
    const int keys = a.lens ? (int)a.lens[n] : (int)(*a.step) + 1;
    const float *qp = a.q + (size_t)(n * (long)a.queries + qi) * a.q_row + h * HD;
    const KV *K = reinterpret_cast<const KV *>(a.K) + n * a.kv_batch + h * a.kv_head;
    const KV *V = reinterpret_cast<const KV *>(a.V) + n * a.kv_batch + h * a.kv_head;
    constexpr int KC = 64, VEC = 16 / sizeof(KV), RW = HD / VEC;  // keys per chunk; 16-byte words per row
    // the first chunk of V rows is copied into shared memory while the scores run
    // (requested right after the first round of K rows)
    auto stage_v = [&](int j0, int nk) {
        for (int u = lane; u < nk * RW; u += 32)
            cp_async16(vs + (size_t)u * VEC, V + (size_t)(j0 + u / RW) * a.kv_row + (u % RW) * VEC);
        cp_async_commit();
    };
    float q[HD];
    if (HD % 4 == 0 && (a.q_row & 3) == 0) {
#pragma unroll
        for (int t = 0; t < HD / 4; ++t) {
            const float4 v = reinterpret_cast<const float4 *>(qp)[t];
            q[4 * t] = v.x;
            q[4 * t + 1] = v.y;
            q[4 * t + 2] = v.z;
            q[4 * t + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int t = 0; t < HD; ++t) q[t] = qp[t];
    }
    // scores: keys j0 + lane and j0 + 32 + lane per round, both rows loaded
    // before either FMA chain (each chain in head-dimension order); the first
    // round's rows are requested before the V rows
    float mx = kNegInf;
    for (int j0 = 0; j0 < keys; j0 += 64) {
        const int ja = j0 + lane, jb = j0 + 32 + lane;
        uint4 ra[RW], rb[RW];
#pragma unroll
        for (int c = 0; c < RW; ++c) {
            ra[c] = ja < keys ? __ldg(reinterpret_cast<const uint4 *>(K + (size_t)ja * a.kv_row) + c) : make_uint4(0, 0, 0, 0);
            rb[c] = jb < keys ? __ldg(reinterpret_cast<const uint4 *>(K + (size_t)jb * a.kv_row) + c) : make_uint4(0, 0, 0, 0);
        }
        if (j0 == 0) stage_v(0, min(KC, keys));
        float sa = 0.0f, sb = 0.0f;
#pragma unroll
        for (int t = 0; t < HD; ++t) {
            sa = __fmaf_rn(q[t], kv_at<KV, RW>(ra, t), sa);
            sb = __fmaf_rn(q[t], kv_at<KV, RW>(rb, t), sb);
        }
        if (ja < keys) {
            e[ja] = sa;
            mx = fmaxf(mx, sa);
        }
        if (jb < keys) {
            e[jb] = sb;
            mx = fmaxf(mx, sb);
        }
    }
    mx = warp_max(mx);
    __syncwarp();
    float s = 0.0f;
    for (int j = lane; j < keys; j += 32) {
        const float ex = mgb_exp(__fsub_rn(e[j], mx));
        e[j] = ex;
        s = j == lane ? ex : __fadd_rn(s, ex);
    }
    const float inv = __fdiv_rn(1.0f, warp_tree(s));
    constexpr int PER = HD >= 32 ? HD / 32 : 1;
    float acc[PER];
#pragma unroll
    for (int c = 0; c < PER; ++c) acc[c] = 0.0f;
    live = HD >= 32 || lane < HD;
    for (int j0 = 0; j0 < keys; j0 += KC) {
        const int nk = min(KC, keys - j0);
        if (j0 > 0) stage_v(j0, nk);
        cp_async_wait();
        __syncwarp();
        if (live)
            for (int jj = 0; jj < nk; ++jj)
#pragma unroll
                for (int c = 0; c < PER; ++c)
                    acc[c] = __fmaf_rn(e[j0 + jj], load_kv(vs + (size_t)jj * HD + lane + 32 * c), acc[c]);
        __syncwarp();
    }
#pragma unroll
    for (int c = 0; c < PER; ++c) res[c] = __fmul_rn(acc[c], inv);
}

// LATE: the next kernel is released after this one's attention rather than at
// its start (small decode batches: measured faster at batch 1, slower at 64).
template <typename KV, int HD, bool LATE>
__global__ void __launch_bounds__(128) attend_kernel(AttnArgs a) {
    extern __shared__ float e_sh[];
    if constexpr (!LATE) pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const long task = (long)blockIdx.x * 4 + warp;
    const long total = (long)a.rows * a.H * a.queries;
    if (task >= total) return;
    const int qi = (int)(task % a.queries), h = (int)((task / a.queries) % a.H), n = (int)(task / ((long)a.queries * a.H));
    constexpr int PER = HD >= 32 ? HD / 32 : 1;
    constexpr int KC = 64;
    KV *vs = reinterpret_cast<KV *>(e_sh + (size_t)4 * a.max_keys) + (size_t)warp * KC * HD;
    float res[PER];
    bool live;
    attend_one<KV, HD>(a, n, h, qi, e_sh + (size_t)warp * a.max_keys, vs, lane, res, live);
    if constexpr (LATE) pdl_launch_dependents();
    if (live) {
        float *o = a.out + (size_t)(n * (long)a.queries + qi) * a.out_row + h * HD;
#pragma unroll
        for (int c = 0; c < PER; ++c) o[lane + 32 * c] = res[c];
    }
    if (a.qo.tq && live) {
        // the head's outputs as q8_1 blocks of the next matmul's input: lane l
        // holds value 32c + l of the head, i.e. position l of block c
#pragma unroll
        for (int c = 0; c < PER; ++c) store_block_tc(a.qo, n, h * (HD / 32) + c, res[c], lane);
    }
}

// ---------------------------------------------------------------------------
// Greedy bookkeeping (malaga.cu:290-326): one warp per batch row, then ++step.

__global__ void greedy_finalize_kernel(const float *pv, const uint32_t *pi, int parts, int rows, uint8_t *finished,
                                       uint32_t *ids, uint32_t *out, int m, uint32_t *step, uint32_t eos, uint32_t pad,
                                       int force) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const uint32_t s = *step;
    for (int row = w; row < rows; row += nw) {
        float best = kNegInf;
        uint32_t bi = 0xffffffffu;
        for (int p = lane; p < parts; p += 32) argmax_merge(best, bi, pv[(size_t)row * parts + p], pi[(size_t)row * parts + p]);
        warp_argmax(best, bi);
        if (lane == 0) {
            uint32_t tok = bi;
            if (finished[row]) tok = pad;
            if (!force && tok == eos) finished[row] = 1;
            ids[row] = tok;
            out[(size_t)row * m + s] = tok;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) *step = s + 1;
}

// --fast-vocab: the source tokens' embedding rows E[src_ids] (dequantized, f32
// [n][d]), made once per batch as the reference's src_emb (graph.rs:98-105).
__global__ void src_embed_kernel(Matrix E, const uint32_t *src_ids, int n, int d, float *out) {
    const size_t total = (size_t)n * d;
    for (size_t k = blockIdx.x * (size_t)blockDim.x + threadIdx.x; k < total; k += (size_t)gridDim.x * blockDim.x)
        out[k] = deq_elem(E, (int)src_ids[k / d], (int)(k % d));
}

// --fast-vocab (model.rs:595-604): the logits of the row's source tokens next
// to the shortlist's. h = dec_norm(x[row]) (the LM head's LayerNorm: SUM32
// statistics, ((x - mean) * rstd) * g + b), then for each source position j of
// the state, dot(h, src_emb[row][j]) in the F32 order (lane l's FMA chain
// over elements l, l+32, ..., then the butterfly at 16, 8, 4, 2, 1; row_dots in
// malaga.cu:230-243 is fast-math and not restatable); the row's best (value,
// V1 + j), the lowest j on ties. CTA (row, p) takes positions 8p..8p+7 (a warp
// each; the LayerNorm is recomputed per CTA) and writes partial p of the row.
__global__ void __launch_bounds__(256) src_logits_kernel(const float *x, const float *gamma, const float *beta, int d,
                                                         const float *src_emb, int S, int V1, float *best_v,
                                                         uint32_t *best_i) {
    extern __shared__ __align__(16) float hs[];  // [d]
    __shared__ float stat[2];
    __shared__ float wv[8];
    __shared__ uint32_t wi[8];
    const int row = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, T = d >> 5;
    pdl_launch_dependents();
    pdl_wait();
    for (int i = threadIdx.x; i < d; i += blockDim.x) hs[i] = __ldcg(x + (size_t)row * d + i);
    __syncthreads();
    if (warp == 0) {
        float sum = 0.0f;
        for (int t = 0; t < T; ++t) sum = t == 0 ? hs[lane] : __fadd_rn(sum, hs[32 * t + lane]);
        const float mean = __fdiv_rn(warp_tree(sum), (float)d);
        float s2 = 0.0f;
        for (int t = 0; t < T; ++t) {
            const float c = __fsub_rn(hs[32 * t + lane], mean);
            const float c2 = __fmul_rn(c, c);
            s2 = t == 0 ? c2 : __fadd_rn(s2, c2);
        }
        const float var = __fdiv_rn(warp_tree(s2), (float)d);
        if (lane == 0) {
            stat[0] = mean;
            stat[1] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < d; i += blockDim.x)
        hs[i] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(hs[i], stat[0]), stat[1]), __ldg(gamma + i)), __ldg(beta + i));
    __syncthreads();
    float bv = kNegInf;
    uint32_t bi = 0xffffffffu;
    const int j = 8 * blockIdx.y + warp;
    if (j < S) {
        const float *e = src_emb + ((size_t)row * S + j) * d;
        float acc = 0.0f;
#pragma unroll 8
        for (int i = lane; i < d; i += 32) acc = __fmaf_rn(__ldg(e + i), hs[i], acc);
        argmax_merge(bv, bi, warp_sum_bf(acc), (uint32_t)(V1 + j));
    }
    if (lane == 0) {
        wv[warp] = bv;
        wi[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; ++w) argmax_merge(bv, bi, wv[w], wi[w]);
        best_v[(size_t)row * gridDim.y + blockIdx.y] = bv;
        best_i[(size_t)row * gridDim.y + blockIdx.y] = bi;
    }
}

// greedy_finalize_kernel over the virtual row concat(shortlist logits, source
// logits) (malaga.cu:280-326 with vocab_map and src_ids): the LM head's
// partials index the shortlist rows, the source partials index V1 + j; the
// winner (lowest index on ties) maps to sl_ids[i] or the row's source token j.
__global__ void greedy_finalize_sl_kernel(const float *pv, const uint32_t *pi, int parts, int rows, const float *sv,
                                          const uint32_t *si, int sparts, const uint32_t *sl_ids, int V1,
                                          const uint32_t *src_ids, int S, uint8_t *finished, uint32_t *ids,
                                          uint32_t *out, int m, uint32_t *step, uint32_t eos, uint32_t pad, int force) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const uint32_t s = *step;
    for (int row = w; row < rows; row += nw) {
        float best = kNegInf;
        uint32_t bi = 0xffffffffu;
        for (int p = lane; p < parts; p += 32) argmax_merge(best, bi, pv[(size_t)row * parts + p], pi[(size_t)row * parts + p]);
        for (int p = lane; p < sparts; p += 32)
            argmax_merge(best, bi, sv[(size_t)row * sparts + p], si[(size_t)row * sparts + p]);
        warp_argmax(best, bi);
        if (lane == 0) {
            uint32_t tok = bi < (uint32_t)V1           ? sl_ids[bi]
                           : bi < (uint32_t)(V1 + S) ? src_ids[(size_t)row * S + (bi - V1)]
                                                     : pad;  // (no finite candidate)
            if (finished[row]) tok = pad;
            if (!force && tok == eos) finished[row] = 1;
            ids[row] = tok;
            out[(size_t)row * m + s] = tok;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) *step = s + 1;
}

// Encoder input: x = E[id] * scale + pos[p]; padded tokens use id = pad, p = pad.
__global__ void __launch_bounds__(256) embed_tokens_kernel(Matrix E, const uint32_t *ids, const uint32_t *lens, int S,
                                                           int rows, const float *pos_table, uint32_t pad,
                                                           float scale, float *x) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int bi = row / S, j = row % S;
    const bool valid = j < (int)lens[bi];
    const uint32_t id = valid ? ids[row] : pad;
    const uint32_t p = valid ? (uint32_t)j + pad + 1 : pad;
    const int K = E.K;
    for (int i = lane; i < K; i += 32)
        x[(size_t)row * K + i] = __fadd_rn(__fmul_rn(deq_elem(E, (int)id, i), scale), pos_table[(size_t)p * K + i]);
}

// x += y (residual add where the matmul output is not fused in place).
__global__ void add_inplace_kernel(float *x, const float *y, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        x[i] = __fadd_rn(y[i], x[i]);
}

}  // namespace mgb
