// Decode-step kernels of the engine (sm_100a).
//
// Reference kernels they replace (crates/malaga-core/kernels/malaga.cu, launched
// by crates/malaga-core/src/kernels.rs) and candle ops (model.rs:552-612):
//   qprep_*         embed_pos_ln (malaga.cu:110-130) + bias_residual_ln's LayerNorm
//                   (malaga.cu:89-105) + candle's q8_1 activation quantization
//   gemv            candle QMatMul::forward (MMVQ) + the bias/residual/ReLU/K-V
//                   epilogues of bias_residual_ln, bias_relu (malaga.cu:133-138)
//                   and qkv_decode (malaga.cu:142-154)
//   attend          attn_decode (malaga.cu:165-227), also the encoder's masked
//                   softmax attention (model.rs:101-109)
//   lm head argmax  QMatMul::forward(token_embd) (model.rs:607) fused with
//                   argmax_partial (malaga.cu:247-280): logits never reach HBM
//   greedy_finalize greedy_finalize (malaga.cu:290-326)
#pragma once
#include "engine.h"
#include "numerics.cuh"

namespace mgb {

// ---------------------------------------------------------------------------
// Weight access

__device__ __forceinline__ size_t wslot(const Matrix &W, int row, int j) {
    return ((size_t)(row >> 5) * W.nb + j) * 32 + (row & 31);
}
__device__ __forceinline__ size_t wsslot(const Matrix &W, int row, int sb) {
    return ((size_t)(row >> 5) * W.nsb + sb) * 32 + (row & 31);
}

// Dequantized element i of row `row` (every product below is exact in f32).
__device__ __forceinline__ float deq_elem(const Matrix &W, int row, int i) {
    const int j = i >> 5, k = i & 31;
    const size_t bi = wslot(W, row, j);
    switch (W.type) {
        case T_F32: return reinterpret_cast<const float *>(W.a)[bi * 32 + k];
        case T_Q8_0: {
            const float d = h2f(reinterpret_cast<const uint16_t *>(W.b)[bi]);
            return __fmul_rn(d, (float)(int8_t)W.a[bi * 32 + k]);
        }
        case T_Q4_K: {
            const uint8_t byte = W.a[bi * 16 + (k & 15)];
            const int q = k < 16 ? (byte & 15) : (byte >> 4);
            const uint8_t *h = W.b + wsslot(W, row, j >> 3) * 16;
            const int sb = j & 7;
            const uint8_t *s = h + 4;
            int sc, m;
            if (sb < 4) {
                sc = s[sb] & 63;
                m = s[sb + 4] & 63;
            } else {
                sc = (s[sb + 4] & 0xf) | ((s[sb - 4] >> 6) << 4);
                m = (s[sb + 4] >> 4) | ((s[sb] >> 6) << 4);
            }
            const float d = h2f(h[0] | (h[1] << 8)), dm = h2f(h[2] | (h[3] << 8));
            return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dm, (float)m));
        }
        case T_Q6_K: {
            const uint8_t byte = W.a[bi * 16 + (k & 15)];
            const int lo = k < 16 ? (byte & 15) : (byte >> 4);
            const uint32_t word = reinterpret_cast<const uint32_t *>(W.b)[bi * 2 + (k >> 4)];
            const int kk = k & 15;
            const int hi = (word >> (8 * (kk & 3) + 2 * (kk >> 2))) & 3;
            const int q = lo | (hi << 4);
            const int sc = (int8_t)W.c[bi * 2 + (k >> 4)];
            const float d = h2f(reinterpret_cast<const uint16_t *>(W.e)[wsslot(W, row, j >> 3)]);
            return __fmul_rn(__fmul_rn(d, (float)sc), (float)(q - 32));
        }
    }
    return 0.0f;
}

// ---------------------------------------------------------------------------
// Activation preparation: one warp per row. Lane l owns elements l + 32 t, so
// block t of the q8_1 activation is exactly "element t of every lane".

enum PrepMode { PREP_PLAIN = 0, PREP_LN = 1, PREP_EMBED_LN = 2, PREP_ATTN = 3 };

struct PrepArgs {
    const float *x;       // input rows [rows][K] (PLAIN, LN)
    float *x_out;         // EMBED_LN: residual stream written here
    const float *gamma, *beta;
    // EMBED_LN
    Matrix embed;
    const uint32_t *ids;
    const uint32_t *step;
    const float *pos_table;
    uint32_t pos_base;
    float scale;
    int rows, K;
    QAct out;
    int keep_f32;  // also store the (normalised) f32 values (for F32 weights)
    float *xf;     // [rows][K]
    int group;     // blocks per activation scale: 1 (Q8_0 consumers) or 8 (Q4_K / Q6_K)
    int ctype;     // weight type of the consuming matrix (tensor-core layout)
};

// Activation scale group of a consumer weight type: k-quants take one f32 scale
// per 256-value super-block (Q8_K style), Q8_0 one f16-rounded scale per block.
__host__ __device__ constexpr int act_group(int type) { return type == T_Q4_K || type == T_Q6_K ? 8 : 1; }

// Quantizes G consecutive blocks (y[u] = element lane of block t0+u of `row`)
// with one scale: d = amax/127 over the G*32 values, q = round(y * (127/amax)).
// G = 1 stores the scale f16-rounded (q8_1 / Q8_0 style), G = 8 as f32 (Q8_K).
template <int G>
__device__ __forceinline__ void quantize_group(const float (&y)[G], int8_t *q, float *d, int *s32, int *s16, int t0,
                                               int lane) {
    float m = fabsf(y[0]);
#pragma unroll
    for (int u = 1; u < G; ++u) m = fmaxf(m, fabsf(y[u]));
    const float amax = warp_max_nonneg(m);
    const float dd = __fdiv_rn(amax, 127.0f), id = __fdiv_rn(127.0f, amax);
    // every block's values first, then the half sums as independent full-warp
    // reductions (no divergent branch between them), then one lane's stores
    int v[G], lo[G], hi[G];
#pragma unroll
    for (int u = 0; u < G; ++u) {
        v[u] = amax == 0.0f ? 0 : (int)roundf(__fmul_rn(y[u], id));
        q[32 * (t0 + u) + lane] = (int8_t)v[u];
    }
#pragma unroll
    for (int u = 0; u < G; ++u) {
        lo[u] = warp_isum_redux(lane < 16 ? v[u] : 0);
        hi[u] = warp_isum_redux(lane < 16 ? 0 : v[u]);
    }
    if (lane == 0) {
#pragma unroll
        for (int u = 0; u < G; ++u) {
            const int t = t0 + u;
            d[t] = G == 1 ? round_h(dd) : dd;
            s16[2 * t] = lo[u];
            s16[2 * t + 1] = hi[u];
            s32[t] = lo[u] + hi[u];
        }
    }
}

// Row `row` of a global QAct as quantize_group destinations.
#define QACT_ROW(o, row) (o).q + (size_t)(row) * (o).K, (o).d + (size_t)(row) * ((o).K >> 5), \
                         (o).s32 + (size_t)(row) * ((o).K >> 5), (o).s16 + (size_t)(row) * ((o).K >> 4)

template <int MODE>
__global__ void __launch_bounds__(256) qprep_kernel(PrepArgs p) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= p.rows) return;
    const int K = p.K, T = K >> 5, G = p.group == 8 ? 8 : 1;
    const float *x = p.x + (size_t)row * K;
    if constexpr (MODE == PREP_EMBED_LN) {
        const uint32_t id = p.ids[row];
        const float *pos = p.pos_table + (size_t)(*p.step + p.pos_base) * K;
        float *xo = p.x_out + (size_t)row * K;
        for (int t = 0; t < T; ++t) {
            const int i = 32 * t + lane;
            xo[i] = __fadd_rn(__fmul_rn(deq_elem(p.embed, (int)id, i), p.scale), pos[i]);
        }
        x = xo;
        __syncwarp();
    }
    if constexpr (MODE == PREP_PLAIN) {
        for (int t = 0; t < T; t += G) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                v[u] = u < G ? x[32 * (t + u) + lane] : 0.0f;
                if (u < G && p.keep_f32) p.xf[(size_t)row * K + 32 * (t + u) + lane] = v[u];
            }
            if (G == 8) quantize_group<8>(v, QACT_ROW(p.out, row), t, lane);
            else quantize_group<1>(reinterpret_cast<const float(&)[1]>(v[0]), QACT_ROW(p.out, row), t, lane);
        }
        return;
    }
    // LayerNorm (eps 1e-5): mean and variance with the lane-ordered pairwise sum.
    float s = 0.0f;
    for (int t = 0; t < T; ++t) s = t == 0 ? x[lane] : __fadd_rn(s, x[32 * t + lane]);
    const float mean = __fdiv_rn(warp_tree(s), (float)K);
    float s2 = 0.0f;
    for (int t = 0; t < T; ++t) {
        const float c = __fsub_rn(x[32 * t + lane], mean);
        const float c2 = __fmul_rn(c, c);
        s2 = t == 0 ? c2 : __fadd_rn(s2, c2);
    }
    const float var = __fdiv_rn(warp_tree(s2), (float)K);
    const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
    for (int t = 0; t < T; t += G) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = 32 * (t + u) + lane;
            v[u] = 0.0f;
            if (u < G) {
                v[u] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x[i], mean), rstd), p.gamma[i]), p.beta[i]);
                if (p.keep_f32) p.xf[(size_t)row * K + i] = v[u];
            }
        }
        if (G == 8) quantize_group<8>(v, QACT_ROW(p.out, row), t, lane);
        else quantize_group<1>(reinterpret_cast<const float(&)[1]>(v[0]), QACT_ROW(p.out, row), t, lane);
    }
}

// ---------------------------------------------------------------------------
// Matmul rows: one warp per weight row, lane l owns blocks [l*G, l*G+G).

enum Epi { EPI_STORE = 0, EPI_RELU = 1, EPI_RESID = 2, EPI_QKV = 3, EPI_CROSSKV = 4, EPI_ARGMAX = 5 };

struct GemvArgs {
    Matrix W;
    QAct x;           // quantized activations [rows][K]
    const float *xf;  // f32 activations (F32 weights)
    int rows;         // activation rows (batch)
    float *y;         // [rows][N] (STORE, RELU, RESID in place)
    // QKV: q out [rows][d]; caches [rows][H][m][hd]
    float *q;
    __half *kc, *vc;
    const uint32_t *step;
    int H, hd, m;
    // CROSSKV: caches [b][H][S][hd], token row = bi * S + j
    int S;
    // ARGMAX
    float *part_v;
    uint32_t *part_i;
    float *logits;  // optional [rows][N]
};

// Weight loads: read-only global loads, or plain loads when the weights were
// staged in shared memory (GLOBAL = false).
template <bool GLOBAL, typename T>
__device__ __forceinline__ T ldw(const T *p) {
    if constexpr (GLOBAL) return __ldg(p);
    else return *p;
}

// One 32-block of a weight row against one activation row. The integer part
// of the block is accumulated exactly into (S1, S2) by accum(); finish() turns
// the sums of a whole unit into its float partial. A unit is one block for
// Q8_0 and one 256-value super-block (8 blocks) for Q4_K / Q6_K:
//   Q8_0: S1 = I;                          p = (d*xd) * float(S1)
//   Q4_K: S1 += sc*I, S2 += m*sum(xq);     p = xd * (d*float(S1) - dmin*float(S2))
//   Q6_K: S1 += sc_a*I_a + sc_b*I_b;       p = (d*xd) * float(S1)
// (I = sum of weight x activation integers over the block, I_a / I_b over its
// 16-value halves with the 6-bit values offset by -32.)
template <int TYPE>
struct BlockW;

template <int TYPE>
__host__ __device__ constexpr int unit_blocks() { return TYPE == T_Q4_K || TYPE == T_Q6_K ? 8 : 1; }

template <>
struct BlockW<T_Q8_0> {
    int w[8];
    float d;
    template <bool GLOBAL = true>
    __device__ __forceinline__ void load(const Matrix &W, int row, int j) {
        const size_t bi = wslot(W, row, j);
        const int4 *src = reinterpret_cast<const int4 *>(W.a + bi * 32);
        const int4 a0 = ldw<GLOBAL>(src), a1 = ldw<GLOBAL>(src + 1);
        w[0] = a0.x; w[1] = a0.y; w[2] = a0.z; w[3] = a0.w;
        w[4] = a1.x; w[5] = a1.y; w[6] = a1.z; w[7] = a1.w;
        d = h2f(ldw<GLOBAL>(reinterpret_cast<const unsigned short *>(W.b) + bi));
    }
    __device__ __forceinline__ void accum(const int *x, int, int, int, int &S1, int &) const {
        int s = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) s = __dp4a(w[i], x[i], s);
        S1 += s;
    }
    __device__ __forceinline__ float finish(int S1, int, float xd) const {
        return __fmul_rn(__fmul_rn(d, xd), (float)S1);
    }
};

template <>
struct BlockW<T_Q4_K> {
    int q[4];
    float d, dm;
    int sc, m;
    template <bool GLOBAL = true>
    __device__ __forceinline__ void load(const Matrix &W, int row, int j) {
        const size_t bi = wslot(W, row, j);
        const int4 a = ldw<GLOBAL>(reinterpret_cast<const int4 *>(W.a + bi * 16));
        q[0] = a.x; q[1] = a.y; q[2] = a.z; q[3] = a.w;
        const uint4 h = ldw<GLOBAL>(reinterpret_cast<const uint4 *>(W.b + wsslot(W, row, j >> 3) * 16));
        d = h2f(h.x & 0xffff);
        dm = h2f(h.x >> 16);
        const uint32_t s0 = h.y, s1 = h.z, s2 = h.w;  // scales bytes 0-3, 4-7, 8-11
        const int sb = j & 7;
        auto byte = [&](int k) -> int {
            const uint32_t w = k < 4 ? s0 : (k < 8 ? s1 : s2);
            return (w >> (8 * (k & 3))) & 0xff;
        };
        if (sb < 4) {
            sc = byte(sb) & 63;
            m = byte(sb + 4) & 63;
        } else {
            sc = (byte(sb + 4) & 0xf) | ((byte(sb - 4) >> 6) << 4);
            m = (byte(sb + 4) >> 4) | ((byte(sb) >> 6) << 4);
        }
    }
    __device__ __forceinline__ void accum(const int *x, int s8, int, int, int &S1, int &S2) const {
        int s = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            s = __dp4a(q[i] & 0x0f0f0f0f, x[i], s);
            s = __dp4a((q[i] >> 4) & 0x0f0f0f0f, x[4 + i], s);
        }
        S1 += sc * s;
        S2 += m * s8;
    }
    __device__ __forceinline__ float finish(int S1, int S2, float xd) const {
        return __fmul_rn(xd, __fsub_rn(__fmul_rn(d, (float)S1), __fmul_rn(dm, (float)S2)));
    }
};

template <>
struct BlockW<T_Q6_K> {
    int w[8];
    int sa, sb;
    float d;
    template <bool GLOBAL = true>
    __device__ __forceinline__ void load(const Matrix &W, int row, int j) {
        const size_t bi = wslot(W, row, j);
        const int4 l = ldw<GLOBAL>(reinterpret_cast<const int4 *>(W.a + bi * 16));
        const uint2 h = ldw<GLOBAL>(reinterpret_cast<const uint2 *>(W.b + bi * 8));
        const int ql[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w[i] = (ql[i] & 0x0f0f0f0f) | (int)(((h.x >> (2 * i)) & 0x03030303u) << 4);
            w[4 + i] = ((ql[i] >> 4) & 0x0f0f0f0f) | (int)(((h.y >> (2 * i)) & 0x03030303u) << 4);
        }
        const unsigned short s = ldw<GLOBAL>(reinterpret_cast<const unsigned short *>(W.c) + bi);
        sa = (int8_t)(s & 0xff);
        sb = (int8_t)(s >> 8);
        d = h2f(ldw<GLOBAL>(reinterpret_cast<const unsigned short *>(W.e) + wsslot(W, row, j >> 3)));
    }
    __device__ __forceinline__ void accum(const int *x, int, int s16a, int s16b, int &S1, int &) const {
        int da = 0, db = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            da = __dp4a(w[i], x[i], da);
            db = __dp4a(w[4 + i], x[4 + i], db);
        }
        da -= 32 * s16a;
        db -= 32 * s16b;
        S1 += sa * da + sb * db;
    }
    __device__ __forceinline__ float finish(int S1, int, float xd) const {
        return __fmul_rn(__fmul_rn(d, xd), (float)S1);
    }
};

// Block partial p_j of row `row` against activation row n, for F32 weights:
// an FMA chain over the block's 32 values.
__device__ __forceinline__ float f32_block(const Matrix &W, int row, int j, const float *x) {
    const float4 *w = reinterpret_cast<const float4 *>(W.a + wslot(W, row, j) * 128);
    float p = 0.0f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const float4 v = __ldg(w + c);
        p = __fmaf_rn(v.x, x[4 * c], p);
        p = __fmaf_rn(v.y, x[4 * c + 1], p);
        p = __fmaf_rn(v.z, x[4 * c + 2], p);
        p = __fmaf_rn(v.w, x[4 * c + 3], p);
    }
    return p;
}

// Epilogue of one output element (row of W, activation row n); v = the
// row sum in block order.
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
        *xr = __fadd_rn(__fadd_rn(v, b), *xr);
    } else if constexpr (EPI == EPI_QKV) {
        const float y = __fadd_rn(v, b);
        const int dm = g.H * g.hd;
        if (row < dm) {
            g.q[(size_t)n * dm + row] = y;
        } else {
            const int c = row - dm, which = c / dm, h = (c % dm) / g.hd, t = c % g.hd;
            __half *cache = which == 0 ? g.kc : g.vc;
            cache[(((size_t)n * g.H + h) * g.m + *g.step) * g.hd + t] = __float2half_rn(y);
        }
    } else if constexpr (EPI == EPI_CROSSKV) {
        const float y = __fadd_rn(v, b);
        const int dm = g.H * g.hd, which = row / dm, c = row % dm, h = c / g.hd, t = c % g.hd;
        const int bi = n / g.S, jj = n % g.S;
        __half *cache = which == 0 ? g.kc : g.vc;
        cache[(((size_t)bi * g.H + h) * g.S + jj) * g.hd + t] = __float2half_rn(y);
    }
}

// Matmul over activations already quantized in global memory: one warp per
// group of 32 weight rows, lane = row, unit partials accumulated left to right;
// NB activation rows per pass.
template <int TYPE, int EPI>
__global__ void __launch_bounds__(256) gemv_kernel(GemvArgs g) {
    constexpr int NB = 8;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const Matrix &W = g.W;
    const int nb = W.nb, groups = W.Np >> 5;
    for (int grp = blockIdx.x * 8 + warp; grp < groups; grp += gridDim.x * 8) {
        const int row = grp * 32 + lane;
        for (int n0 = 0; n0 < g.rows; n0 += NB) {
            float acc[NB];
#pragma unroll
            for (int i = 0; i < NB; ++i) acc[i] = 0.0f;
            if constexpr (TYPE == T_F32) {
                for (int j = 0; j < nb; ++j)
#pragma unroll
                    for (int i = 0; i < NB; ++i) {
                        if (n0 + i >= g.rows) break;
                        const float p = f32_block(W, row, j, g.xf + (size_t)(n0 + i) * W.K + 32 * j);
                        acc[i] = j == 0 ? p : __fadd_rn(acc[i], p);
                    }
            } else {
                constexpr int UB = unit_blocks<TYPE>();
                for (int u = 0; u < nb; u += UB) {
                    int S1[NB], S2[NB];
#pragma unroll
                    for (int i = 0; i < NB; ++i) S1[i] = S2[i] = 0;
                    BlockW<TYPE> bw;
#pragma unroll 2
                    for (int j = u; j < u + UB; ++j) {
                        bw.load(W, row, j);
#pragma unroll
                        for (int i = 0; i < NB; ++i) {
                            const int n = n0 + i;
                            if (n >= g.rows) break;
                            const int4 *xs = reinterpret_cast<const int4 *>(g.x.q + (size_t)n * W.K + 32 * j);
                            const int4 x0 = xs[0], x1 = xs[1];
                            const int xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                            int s32 = 0, s16a = 0, s16b = 0;
                            if constexpr (TYPE == T_Q4_K) s32 = g.x.s32[(size_t)n * nb + j];
                            if constexpr (TYPE == T_Q6_K) {
                                s16a = g.x.s16[(size_t)n * 2 * nb + 2 * j];
                                s16b = g.x.s16[(size_t)n * 2 * nb + 2 * j + 1];
                            }
                            bw.accum(xv, s32, s16a, s16b, S1[i], S2[i]);
                        }
                    }
#pragma unroll
                    for (int i = 0; i < NB; ++i) {
                        const int n = n0 + i;
                        if (n >= g.rows) break;
                        const float p = bw.finish(S1[i], S2[i], g.x.d[(size_t)n * nb + u]);
                        acc[i] = u == 0 ? p : __fadd_rn(acc[i], p);
                    }
                }
            }
            if (row < W.N)
#pragma unroll
                for (int i = 0; i < NB; ++i) {
                    if (n0 + i >= g.rows) break;
                    epilogue_store<EPI>(g, row, n0 + i, acc[i]);
                }
        }
    }
}

// ---------------------------------------------------------------------------
// Tensor-core activation layout (QAct tq / trec, written for one consumer)

// Byte offset of (row r, 16-byte K chunk k16) of a K=32 int8 operand tile in
// the UMMA K-major no-swizzle layout: 8-row core groups of 256 bytes.
__host__ __device__ __forceinline__ int tile_off(int r, int k16) { return (r >> 3) * 256 + k16 * 128 + (r & 7) * 16; }

// One unit (G blocks of 32 values, y[g] = value lane of block j0+g of token
// `tok`) into a tensor-core activation buffer: one scale, the bytes in the UMMA
// layout, the unit record (same arithmetic as qprep_row_kernel).
template <int G>
__device__ __forceinline__ void store_unit(const QAct &o, int ctype, int tok, int j0, const float (&y)[G], int lane) {
    float m = fabsf(y[0]);
#pragma unroll
    for (int g = 1; g < G; ++g) m = fmaxf(m, fabsf(y[g]));
    const float amax = warp_max_nonneg(m);
    const float dd = __fdiv_rn(amax, 127.0f), id = __fdiv_rn(127.0f, amax);
    const int rs = o.rs;
    const bool sums = ctype == T_Q4_K && G == 8;  // only Q4_K records carry block sums
    int s32[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int q = amax == 0.0f ? 0 : (int)roundf(__fmul_rn(y[g], id));
        o.tq[((size_t)(j0 + g) * (rs / 8) + (tok >> 3)) * 256 + tile_off(tok & 7, lane >> 4) + (lane & 15)] =
            (uint8_t)(int8_t)q;
        s32[g] = sums ? warp_isum_redux(q) : 0;
    }
    if (lane == 0) {
        if (sums) {
            int4 *rec = reinterpret_cast<int4 *>(o.trec + ((size_t)(j0 / 8) * rs + tok) * 32);
            rec[0] = make_int4(__float_as_int(dd), (s32[0] & 0xffff) | (s32[1 % G] << 16),
                               (s32[2 % G] & 0xffff) | (s32[3 % G] << 16), (s32[4 % G] & 0xffff) | (s32[5 % G] << 16));
            rec[1] = make_int4((s32[6 % G] & 0xffff) | (s32[7 % G] << 16), 0, 0, 0);
        } else if (G == 8) {
            reinterpret_cast<float *>(o.trec)[(size_t)(j0 / 8) * rs + tok] = dd;
        } else {
            reinterpret_cast<float *>(o.trec)[(size_t)j0 * rs + tok] = round_h(dd);
        }
    }
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
    // Optional: the outputs also quantized into the next matmul's tensor-core
    // layout (qo.tq != null; single queries, 4 heads of one row per CTA whose
    // 4*hd values are whole units of the consumer qo_ctype).
    QAct qo;
    int qo_ctype;
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
    if (task >= total) return;  // (never with qo: the host launches whole CTAs then)
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
    if (a.qo.tq) {
        // the CTA's 4 heads (4*HD consecutive values of row n) as units of the consumer
        __shared__ float ov[4 * 128];
        if (live)
#pragma unroll
            for (int c = 0; c < PER; ++c) ov[warp * HD + lane + 32 * c] = res[c];
        __syncthreads();
        const int j0 = (h - warp) * HD / 32;  // first block of the CTA's values
        if (a.qo_ctype == T_Q4_K || a.qo_ctype == T_Q6_K) {
            for (int u = warp; u < 4 * HD / 256; u += 4) {
                float y[8];
#pragma unroll
                for (int g = 0; g < 8; ++g) y[g] = ov[256 * u + 32 * g + lane];
                store_unit<8>(a.qo, a.qo_ctype, n, j0 + 8 * u, y, lane);
            }
        } else {
            for (int t = warp; t < 4 * HD / 32; t += 4) {
                const float y[1] = {ov[32 * t + lane]};
                store_unit<1>(a.qo, a.qo_ctype, n, j0 + t, y, lane);
            }
        }
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
