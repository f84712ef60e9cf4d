// Small-batch quantized matmul (at most 8 activation rows) with the
// reference's MMVQ arithmetic, fused with its activation prologue and
// epilogue (sm_100a).
//
// One launch replaces the reference's chain "bias_residual_ln / embed_pos_ln
// (malaga.cu:89-130) -> candle quantize_q8_1 -> QMatMul MMVQ (candle-core
// 0.11.0 src/quantized/cuda.rs, candle-kernels 0.11.0 src/quantized.cu) ->
// bias / ReLU / residual / qkv_decode epilogue (malaga.cu:133-154)".
//
// Data flow of one CTA (a contiguous range of weight rows):
//   1. thread 0 starts 1-D bulk copies (TMA) of the first chunks of its rows
//      (row layout, engine.h) into a ring of shared-memory stages; weights do
//      not depend on the previous kernel, so this overlaps its tail (PDL);
//   2. after griddepcontrol.wait the warps build the q8_1 activations of the
//      NC batch rows in shared memory (LayerNorm / embedding + position +
//      LayerNorm / plain input, the engine's fixed LayerNorm order);
//   3. per chunk, warp w takes rows w, w+8, ...: the 32 lanes play MMVQ's
//      NW x 32 threads for that row -- lane l computes, for virtual warp v,
//      thread 32v + l's vec_dot sum over its blocks, adds the virtual warps in
//      order, and a butterfly sum over the lanes gives the output (identical in
//      every lane); lane n stores column n;
//   4. the freed stage is refilled with the chunk RS ahead.
// Every mbarrier wait is bounded; on a timeout the CTA records an error flag,
// waits (bounded) for its own copies in flight and returns.
#pragma once
#include "kernels.cuh"

namespace mgb {

// q8_1 activations of NC batch rows in shared memory (F32 weights: the f32
// values instead).
struct SmAct {
    int8_t *q;   // [NC][K]
    float *d;    // [NC][K/32] block scales (f16 values)
    float *xf;   // [NC][K] (F32 weights only)
};

// Bytes of one weight row in the row layout (= its GGUF bytes; F32: 4K).
__host__ __device__ inline int row_bytes_of(int type, int K) {
    switch (type) {
        case T_Q8_0: return K / 32 * 34;
        case T_Q4_K: return K / 256 * 144;
        case T_Q6_K: return K / 256 * 210;
        default: return 4 * K;
    }
}

// Per-row bytes of the row layout's regions ra, rb, rc, re.
__host__ __device__ inline void row_regions(int type, int K, int (&rb)[4]) {
    rb[1] = rb[2] = rb[3] = 0;
    switch (type) {
        case T_Q8_0: rb[0] = K; rb[1] = K / 16; break;
        case T_Q4_K: rb[0] = K / 256 * 144; break;
        case T_Q6_K: rb[0] = K / 2; rb[1] = K / 4; rb[2] = K / 16; rb[3] = K / 128; break;
        default: rb[0] = 4 * K; break;
    }
}

struct SmallArgs {
    GemvArgs g;        // matrix and outputs (g.rows: activation rows of the whole matmul)
    PrepArgs p;        // activation source
    int n0;            // first activation row of this launch (launches cover at most 8 rows)
    int rows_per_cta;  // weight rows per CTA (a multiple of 8)
    int stages;        // ring depth (1..4); 0 for F32 weights (read from global memory)
    uint32_t *err;
    // Failure-path test hooks (mgb_ctx, set from MGB_TEST_* at mgb_open; off by
    // default): the limit of every mbarrier wait, and one chunk of CTA 0 whose
    // copy is withheld (-1: none), so that a bounded wait runs out.
    uint64_t wait_ns;
    int withhold_chunk;
    // CTAs per thread-block cluster (1: none): the CTAs of a cluster share the
    // q8_1 quantization of the input rows (each takes 1/cluster of the blocks and
    // writes them into every CTA's shared memory)
    int cluster;
};

__host__ __device__ inline size_t small_act_bytes(int NC, int K, int type, int mode) {
    size_t n = (size_t)NC * K + (size_t)NC * (K / 32) * 4;        // q, d
    if (type == T_F32) n += (size_t)NC * K * 4;                   // xf
    if (mode != PREP_PLAIN) n += (size_t)NC * K * 4 + (size_t)8 * K + (size_t)NC * 8;  // rows, gamma/beta, stats
    return (n + 15) / 16 * 16;
}

__device__ __forceinline__ int lds32(const void *p) { return *reinterpret_cast<const int *>(p); }

// ---------------------------------------------------------------------------
// MMVQ per type. A warp computes R weight rows at once (local rows lr0,
// lr0 + 8, ... of the stage; region k of local row r at st + CR*off_k + r*rb[k]),
// the activation operands of each unit loaded once for all R rows.
// out[r][n] = the output of row r, column n, in every lane.

// Exact int -> float for |x| < 2^22: two full-rate instructions instead of one
// conversion on the quarter-rate pipe (1.5 * 2^23 + x has x in its mantissa).
__device__ __forceinline__ float i2f_exact(int x) { return __fsub_rn(__int_as_float(x + 0x4B400000), 12582912.0f); }

struct StageRows {
    const uint8_t *base[4];  // region k of local row 0
    int rb[4];               // bytes per row of region k
    __device__ __forceinline__ const uint8_t *row(int k, int lr) const { return base[k] + (size_t)lr * rb[k]; }
};

// Q6_K (candle vec_dot_q6_K_q8_1, qi 32, vdr 1): thread t handles super-blocks
// t/32 + i*NW; lane l reads ql int l, 4 values of blocks A and A+2 of the
// super-block (A = 4(l/16) + (l%16)/8) at positions 4(l%8)..+3:
//   sf = fma(dx_{A+2}, float(I_1*sc_1), fma(dx_A, float(I_0*sc_0), 0)), P = fma(d, sf, P)
// with I = sum (q - 32) * u, formed as dp4a(q, u, dp4a(-32 x 4, u, 0)).
template <int NC, int NW, int R>
__device__ __forceinline__ void mmvq_q6k(const StageRows &S, int lr0, int nsb, const SmAct &s, int K, int lane,
                                         float (&out)[R][NC]) {
    const int nb = K >> 5;
    const int A = 4 * (lane >> 4) + ((lane & 15) >> 3), p0 = 4 * (lane & 7);
    const int hoff = 4 * (8 * (lane >> 4) + (lane & 7)), hsh = 2 * ((lane & 15) >> 3);
    const int so = 8 * (lane >> 4) + ((lane & 15) >> 2);
    float leaf[R][NC];
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        float P[R][NC];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int n = 0; n < NC; ++n) P[r][n] = 0.0f;
        for (int kb = w; kb < nsb; kb += NW) {
            const int j0 = 8 * kb + A;
            int u0[NC], u1[NC], c0[NC], c1[NC];
            float d0[NC], d1[NC];
#pragma unroll
            for (int n = 0; n < NC; ++n) {
                const int8_t *xq = s.q + (size_t)n * K;
                u0[n] = lds32(xq + 32 * j0 + p0);
                u1[n] = lds32(xq + 32 * (j0 + 2) + p0);
                c0[n] = __dp4a((int)0xE0E0E0E0, u0[n], 0);
                c1[n] = __dp4a((int)0xE0E0E0E0, u1[n], 0);
                d0[n] = s.d[n * nb + j0];
                d1[n] = s.d[n * nb + j0 + 2];
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int lr = lr0 + 8 * r;
                const int vl = lds32(S.row(0, lr) + kb * 128 + 4 * lane);
                const int vh = lds32(S.row(1, lr) + kb * 64 + hoff) >> hsh;
                const int8_t *sc = reinterpret_cast<const int8_t *>(S.row(2, lr)) + kb * 16 + so;
                const int sc0 = sc[0], sc1 = sc[4];
                const float d6 = __half2float(reinterpret_cast<const __half *>(S.row(3, lr))[kb]);
                const int q0 = (vl & 0x0F0F0F0F) | ((vh << 4) & 0x30303030);
                const int q1 = ((vl >> 4) & 0x0F0F0F0F) | (vh & 0x30303030);
#pragma unroll
                for (int n = 0; n < NC; ++n) {
                    const float sf = __fmaf_rn(d1[n], i2f_exact(__dp4a(q1, u1[n], c1[n]) * sc1),
                                               __fmaf_rn(d0[n], i2f_exact(__dp4a(q0, u0[n], c0[n]) * sc0), 0.0f));
                    P[r][n] = __fmaf_rn(d6, sf, P[r][n]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int n = 0; n < NC; ++n) leaf[r][n] = w == 0 ? P[r][n] : __fadd_rn(leaf[r][n], P[r][n]);
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int n = 0; n < NC; ++n) out[r][n] = warp_sum_bf(leaf[r][n]);
}

// Q4_K (candle vec_dot_q4_K_q8_1, qi 32, vdr 2): 16 threads per super-block;
// thread t handles super-blocks t/16 + i*2NW, sub-blocks 2c (low nibbles) and
// 2c+1 (high) with c = (t%16)/4, positions 4o..4o+3 and 16+4o..+3 (o = t%4):
//   sumf_d = sum_i dx_i*float(I_i*sc_i), sumf_m = sum_i dx_i*float(Q_i*m_i)
//   P += fma(d, sumf_d, -(dmin*sumf_m))   (Q_i = sum of the 8 activation bytes)
template <int NC, int NW, int R>
__device__ __forceinline__ void mmvq_q4k(const StageRows &S, int lr0, int nsb, const SmAct &s, int K, int lane,
                                         float (&out)[R][NC]) {
    const int nb = K >> 5;
    const int c = (lane & 15) >> 2, o = lane & 3;
    float leaf[R][NC];
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        float P[R][NC];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int n = 0; n < NC; ++n) P[r][n] = 0.0f;
        for (int kb = 2 * w + (lane >> 4); kb < nsb; kb += 2 * NW) {
            const int ja = 8 * kb + 2 * c;
            int ua0[NC], ua1[NC], ub0[NC], ub1[NC], qa[NC], qb[NC];
            float d8a[NC], d8b[NC];
#pragma unroll
            for (int n = 0; n < NC; ++n) {
                const int8_t *xq = s.q + (size_t)n * K + 32 * ja + 4 * o;
                ua0[n] = lds32(xq);
                ua1[n] = lds32(xq + 16);
                ub0[n] = lds32(xq + 32);
                ub1[n] = lds32(xq + 48);
                qa[n] = __dp4a(0x01010101, ua1[n], __dp4a(0x01010101, ua0[n], 0));
                qb[n] = __dp4a(0x01010101, ub1[n], __dp4a(0x01010101, ub0[n], 0));
                d8a[n] = s.d[n * nb + ja];
                d8b[n] = s.d[n * nb + ja + 1];
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const uint8_t *sb = S.row(0, lr0 + 8 * r) + kb * 144;
                const uint32_t dmw = (uint32_t)lds32(sb);
                const float dall = h2f((uint16_t)(dmw & 0xffff)), dmin = h2f((uint16_t)(dmw >> 16));
                // 6-bit scale / min of sub-blocks 2c, 2c+1 (GGUF packing)
                const uint32_t s0 = (uint32_t)lds32(sb + 4), s1 = (uint32_t)lds32(sb + 8), s2 = (uint32_t)lds32(sb + 12);
                uint32_t scw, mw;  // bytes: scale of 2c, 2c+1 / min of 2c, 2c+1 in the low 16 bits
                if (c < 2) {
                    scw = (s0 >> (16 * c)) & 0x3f3f;
                    mw = (s1 >> (16 * c)) & 0x3f3f;
                } else {
                    const int h = 16 * (c - 2);
                    scw = ((s2 >> h) & 0x0f0f) | (((s0 >> h) & 0xc0c0) >> 2);
                    mw = (((s2 >> h) >> 4) & 0x0f0f) | (((s1 >> h) & 0xc0c0) >> 2);
                }
                const int sca = scw & 0xff, scb = scw >> 8, ma = mw & 0xff, mb = mw >> 8;
                const int v0 = lds32(sb + 16 + 32 * c + 4 * o), v1 = lds32(sb + 32 + 32 * c + 4 * o);
                const int la0 = v0 & 0x0F0F0F0F, la1 = v1 & 0x0F0F0F0F;
                const int hb0 = (v0 >> 4) & 0x0F0F0F0F, hb1 = (v1 >> 4) & 0x0F0F0F0F;
#pragma unroll
                for (int n = 0; n < NC; ++n) {
                    const int dot1a = __dp4a(la1, ua1[n], __dp4a(la0, ua0[n], 0));
                    const int dot1b = __dp4a(hb1, ub1[n], __dp4a(hb0, ub0[n], 0));
                    const float sd = __fmaf_rn(d8b[n], i2f_exact(dot1b * scb), __fmaf_rn(d8a[n], i2f_exact(dot1a * sca), 0.0f));
                    const float sm = __fmaf_rn(d8b[n], i2f_exact(qb[n] * mb), __fmaf_rn(d8a[n], i2f_exact(qa[n] * ma), 0.0f));
                    P[r][n] = __fadd_rn(P[r][n], __fmaf_rn(dall, sd, -__fmul_rn(dmin, sm)));
                }
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int n = 0; n < NC; ++n) leaf[r][n] = w == 0 ? P[r][n] : __fadd_rn(leaf[r][n], P[r][n]);
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int n = 0; n < NC; ++n) out[r][n] = warp_sum_bf(leaf[r][n]);
}

// Q8_0 (candle vec_dot_q8_0_q8_1, qi 8, vdr 2): 4 threads per block; thread t
// handles blocks t/4 + i*8NW, values 8o..8o+7 (o = t%4): P = fma(dw*dx, float(I), P).
template <int NC, int NW, int R>
__device__ __forceinline__ void mmvq_q80(const StageRows &S, int lr0, int nb, const SmAct &s, int K, int lane,
                                         float (&out)[R][NC]) {
    const int o = lane & 3;
    float leaf[R][NC];
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        float P[R][NC];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int n = 0; n < NC; ++n) P[r][n] = 0.0f;
        for (int kb = 8 * w + (lane >> 2); kb < nb; kb += 8 * NW) {
            int x0[NC], x1[NC];
            float dx[NC];
#pragma unroll
            for (int n = 0; n < NC; ++n) {
                const int8_t *xq = s.q + (size_t)n * K + 32 * kb + 8 * o;
                x0[n] = lds32(xq);
                x1[n] = lds32(xq + 4);
                dx[n] = s.d[n * nb + kb];
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int lr = lr0 + 8 * r;
                const uint8_t *qs = S.row(0, lr) + kb * 32 + 8 * o;
                const int v0 = lds32(qs), v1 = lds32(qs + 4);
                const float dw = __half2float(reinterpret_cast<const __half *>(S.row(1, lr))[kb]);
#pragma unroll
                for (int n = 0; n < NC; ++n)
                    P[r][n] = __fmaf_rn(__fmul_rn(dw, dx[n]), i2f_exact(__dp4a(v1, x1[n], __dp4a(v0, x0[n], 0))), P[r][n]);
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int n = 0; n < NC; ++n) leaf[r][n] = w == 0 ? P[r][n] : __fadd_rn(leaf[r][n], P[r][n]);
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int n = 0; n < NC; ++n) out[r][n] = warp_sum_bf(leaf[r][n]);
}

// F32 weights (candle: a cuBLAS matmul; this project's order): lane l's FMA
// chain over elements l, l+32, ..., then the butterfly sum. Rows from global memory.
template <int NC, int R>
__device__ __forceinline__ void mm_f32(const StageRows &S, int lr0, const SmAct &s, int K, int lane,
                                       float (&out)[R][NC]) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const float *w = reinterpret_cast<const float *>(S.row(0, lr0 + 8 * r));
#pragma unroll
        for (int n = 0; n < NC; ++n) {
            const float *x = s.xf + (size_t)n * K;
            float acc = 0.0f;
            for (int i = lane; i < K; i += 32) acc = __fmaf_rn(w[i], x[i], acc);
            out[r][n] = warp_sum_bf(acc);
        }
    }
}

// ---------------------------------------------------------------------------
// Activation prologue: the NC rows' inputs (rows >= p.rows are zero), the
// LayerNorm statistics (warp per row: lane-ordered sums, SUM32 tree), then
// (row, block) tasks over the warps: normalise and quantize to q8_1.

// (activation rows are read through L2 only: inside the persistent step kernel
// other CTAs wrote them earlier in the same launch)
template <int MODE>
__device__ __forceinline__ float small_input(const PrepArgs &p, const float *pos, int n, int i) {  // n: global row
    if constexpr (MODE == PREP_EMBED_LN)
        return __fadd_rn(__fmul_rn(deq_elem(p.embed, (int)__ldcg(p.ids + n), i), p.scale), pos[i]);
    else
        return __ldcg(p.x + (size_t)n * p.K + i);
}

// A barrier over the prologue's threads: __syncthreads when id is 0, else
// named barrier `id` over the first `n` threads (a caller whose other warps do
// not take part in the prologue).
struct CtaSync {
    int id, n;
    __device__ __forceinline__ void operator()() const {
        if (id == 0) __syncthreads();
        else asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
    }
};

struct NoMark {
    __device__ void operator()(int) const {}
};

// `mark(k)` is called after each of its three stages (timing probes). With
// csize > 1 (a cluster of csize CTAs, this one of rank crank, all started) the
// CTA quantizes blocks [crank * per, (crank + 1) * per) of the NC * K/32 and
// stores each into the activations of every CTA of the cluster, then waits at a
// cluster barrier: the same values as quantizing all of them, written once.
template <int MODE, bool F32W, typename Mark = NoMark>
__device__ void small_prologue(const PrepArgs &p, int n0, const SmAct &s, int NC, uint8_t *lnbuf, bool write_x,
                               int nthr, CtaSync sync, Mark &&mark = Mark{}, int crank = 0, int csize = 1) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = nthr >> 5;
    const int K = p.K, T = K >> 5, rows = min(NC, p.rows - n0);
    const float *pos = nullptr;
    float *xs = nullptr, *gb = nullptr, *st = nullptr;
    if constexpr (MODE != PREP_PLAIN) {
        xs = reinterpret_cast<float *>(lnbuf);     // [NC][K] input rows
        gb = xs + (size_t)NC * K;                  // gamma[K], beta[K]
        st = gb + 2 * K;                           // [NC] mean, rstd
        if constexpr (MODE == PREP_EMBED_LN) pos = p.pos_table + (size_t)(*p.step + p.pos_base) * K;
        // the rows' inputs, then gamma and beta, into shared memory (xs and gb
        // are one array): 16 loads in flight per thread before their stores
        const int nin = rows * K, nall = nin + 2 * K;
        for (int base = threadIdx.x; base < nall; base += 16 * nthr) {
            float v[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                const int idx = base + u * nthr;
                v[u] = idx < nin    ? small_input<MODE>(p, pos, n0 + idx / K, idx % K)
                       : idx < nin + K ? __ldg(p.gamma + (idx - nin))
                       : idx < nall    ? __ldg(p.beta + (idx - nin - K))
                                       : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                const int idx = base + u * nthr;
                if (idx >= nall) break;
                if (idx < nin) {
                    xs[idx] = v[u];
                    if constexpr (MODE == PREP_EMBED_LN)
                        if (write_x) p.x_out[(size_t)n0 * K + idx] = v[u];
                } else {
                    gb[idx - nin] = v[u];
                }
            }
        }
        sync();
        mark(1);
        for (int n = warp; n < rows; n += nw) {
            const float *xr = xs + (size_t)n * K;
            float sum = 0.0f;
#pragma unroll 8
            for (int t = 0; t < T; ++t) sum = t == 0 ? xr[lane] : __fadd_rn(sum, xr[32 * t + lane]);
            const float mean = __fdiv_rn(warp_tree(sum), (float)K);
            float s2 = 0.0f;
#pragma unroll 8
            for (int t = 0; t < T; ++t) {
                const float c = __fsub_rn(xr[32 * t + lane], mean);
                const float c2 = __fmul_rn(c, c);
                s2 = t == 0 ? c2 : __fadd_rn(s2, c2);
            }
            const float var = __fdiv_rn(warp_tree(s2), (float)K);
            if (lane == 0) {
                st[2 * n] = mean;
                st[2 * n + 1] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
            }
        }
        sync();
        mark(2);
    }
    // (row, block) tasks [lo, hi); loads of 8 tasks in flight per warp
    constexpr int PIPE = 8;
    const int tasks = NC * T, per = (tasks + csize - 1) / csize;
    const int lo = min(tasks, crank * per), hi = min(tasks, lo + per);
    for (int base = lo + warp; base < hi; base += nw * PIPE) {
        float y[PIPE];
#pragma unroll
        for (int u = 0; u < PIPE; ++u) {
            const int task = base + u * nw, n = task / T, i = 32 * (task % T) + lane;
            y[u] = 0.0f;
            if (task < hi && n < rows) {
                if constexpr (MODE == PREP_PLAIN) y[u] = __ldcg(p.x + (size_t)(n0 + n) * K + i);
                else y[u] = xs[(size_t)n * K + i];
            }
        }
#pragma unroll
        for (int u = 0; u < PIPE; ++u) {
            const int task = base + u * nw;
            if (task >= hi) break;  // uniform across the warp
            const int n = task / T, t = task % T, i = 32 * t + lane;
            float v = y[u];
            if constexpr (MODE != PREP_PLAIN)
                if (n < rows)
                    v = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v, st[2 * n]), st[2 * n + 1]), gb[i]), gb[K + i]);
            if constexpr (F32W) {
                s.xf[(size_t)n * K + i] = v;
            } else {
                float d, sm;
                const int q = q81_block(v, d, sm);
                if (csize == 1) {
                    s.q[(size_t)n * K + i] = (int8_t)q;
                    if (lane == 0) s.d[n * T + t] = d;
                } else {
                    const uint32_t aq = smem_u32(s.q + (size_t)n * K + i), ad = smem_u32(s.d + n * T + t);
                    for (int c = 0; c < csize; ++c) {
                        st_cluster_u8(aq, (uint32_t)c, (uint32_t)(q & 0xff));
                        if (lane == 0) st_cluster_f32(ad, (uint32_t)c, d);
                    }
                }
            }
        }
    }
    if (csize > 1) cluster_sync();
    else sync();
    mark(3);
}

// ---------------------------------------------------------------------------

// R: weight rows per warp per stage (a stage holds 8R rows).
template <int TYPE, int EPI, int MODE, int NC, int NW, int R>
__global__ void __launch_bounds__(256) small_mm_kernel(const __grid_constant__ SmallArgs A) {
    extern __shared__ __align__(16) uint8_t sm_raw[];
    __shared__ __align__(8) uint64_t full[4];
    __shared__ float best_v[8][NC];
    __shared__ uint32_t best_i[8][NC];
    const GemvArgs &g = A.g;
    const Matrix &W = g.W;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr bool STAGED = TYPE != T_F32;  // F32 rows are read from global memory
    constexpr int CR = 8 * R;               // weight rows per stage
    const int K = W.K, RS = STAGED ? A.stages : 1, n0 = A.n0;
    const int r0 = blockIdx.x * A.rows_per_cta, r1 = min(W.Np, r0 + A.rows_per_cta);
    const int nchunks = r0 < r1 ? (r1 - r0 + CR - 1) / CR : 0;
    int rb[4];
    row_regions(TYPE, K, rb);
    const int RB = rb[0] + rb[1] + rb[2] + rb[3];
    const size_t stage_bytes = (size_t)CR * RB;
    const uint8_t *src[4] = {W.ra, W.rb, W.rc, W.re};
    // shared layout: [RS stages][activations]
    uint8_t *stages = sm_raw;
    uint8_t *act = sm_raw + (STAGED ? (size_t)RS * stage_bytes : 0);
    auto issue = [&](int ci) {  // thread 0: chunk ci into stage ci % RS
        const int c0 = r0 + ci * CR, cr = min(CR, r1 - c0);
        uint64_t *bar = &full[ci % RS];
        uint8_t *dst = stages + (size_t)(ci % RS) * stage_bytes;
        mbar_expect_tx(bar, (uint32_t)(cr * RB));
        for (int k = 0; k < 4; ++k) {
            if (!rb[k]) continue;
            bulk_g2s(dst, src[k] + (size_t)c0 * rb[k], (uint32_t)(cr * rb[k]), bar);
            dst += (size_t)CR * rb[k];
        }
    };
    if (STAGED && tid == 0) {
        for (int i = 0; i < RS; ++i) mbar_init(&full[i], 1);
        for (int i = 0; i < min(RS, nchunks); ++i)
            if (!(blockIdx.x == 0 && i == A.withhold_chunk)) issue(i);
    }
    if constexpr (EPI == EPI_ARGMAX)
        if (lane < NC) {
            best_v[warp][lane] = kNegInf;
            best_i[warp][lane] = 0xffffffffu;
        }
    // CTAs with one chunk (the decode step's matrices): the epilogue's bias
    // values (weights) now, its residual values and the decode step right after
    // the dependency wait, so the stores after the dot products wait on no load
    constexpr bool PRE_EPI = EPI == EPI_STORE || EPI == EPI_RELU || EPI == EPI_RESID || EPI == EPI_QKV;
    const bool pre = PRE_EPI && nchunks == 1;
    float pb[R], px[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        pb[r] = 0.0f;
        px[r] = 0.0f;
        const int row = r0 + warp + 8 * r;
        if (pre && W.bias && warp + 8 * r < r1 - r0 && row < W.N) pb[r] = __ldg(W.bias + row);
    }
    // a cluster's CTAs write into each other's shared memory: all must have started
    const int csize = STAGED ? A.cluster : 1;
    const uint32_t crank = csize > 1 ? cluster_rank() : 0u;
    if (csize > 1) cluster_sync();
    pdl_launch_dependents();
    pdl_wait();
    int step = 0;
    if constexpr (EPI == EPI_QKV)
        if (pre) step = (int)*g.step;
    if constexpr (EPI == EPI_RESID)
        if (pre)
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int row = r0 + warp + 8 * r;
                if (warp + 8 * r < r1 - r0 && row < W.N && lane < NC && n0 + lane < g.rows)
                    px[r] = __ldcg(g.y + (size_t)(n0 + lane) * W.N + row);
            }
    SmAct s;
    s.q = reinterpret_cast<int8_t *>(act);
    s.d = reinterpret_cast<float *>(act + (size_t)NC * K);
    s.xf = reinterpret_cast<float *>(act + (size_t)NC * K + (size_t)NC * (K / 32) * 4);
    uint8_t *lnbuf = reinterpret_cast<uint8_t *>(s.xf) + (TYPE == T_F32 ? (size_t)NC * K * 4 : 0);
    small_prologue<MODE, TYPE == T_F32>(A.p, n0, s, NC, lnbuf, blockIdx.x == 0, blockDim.x, CtaSync{0, 0}, NoMark{},
                                        (int)crank, csize);

    float bv = kNegInf;
    uint32_t bi = 0xffffffffu;
    int ci = 0;
    bool ok = true;
    for (; ci < nchunks; ++ci) {
        if constexpr (STAGED) {
            ok = mbar_wait(&full[ci % RS], (uint32_t)((ci / RS) & 1), A.wait_ns);
            ok = __syncthreads_and(ok);
            if (!ok) break;
        }
        const int c0 = r0 + ci * CR, cr = min(CR, r1 - c0);
        StageRows S;
        {
            const uint8_t *st = STAGED ? stages + (size_t)(ci % RS) * stage_bytes : W.ra + (size_t)c0 * RB;
            size_t off = 0;
            for (int k = 0; k < 4; ++k) {
                S.base[k] = st + off;
                S.rb[k] = rb[k];
                off += (size_t)CR * rb[k];
            }
        }
        // warp w: local rows w, w+8, ..., w+8(R-1); rows past the chunk compute on
        // stale stage bytes and are not stored
        float out[R][NC];
        if constexpr (TYPE == T_Q6_K) mmvq_q6k<NC, NW, R>(S, warp, W.nsb, s, K, lane, out);
        else if constexpr (TYPE == T_Q4_K) mmvq_q4k<NC, NW, R>(S, warp, W.nsb, s, K, lane, out);
        else if constexpr (TYPE == T_Q8_0) mmvq_q80<NC, NW, R>(S, warp, W.nb, s, K, lane, out);
        else mm_f32<NC, R>(S, warp, s, K, lane, out);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int lr = warp + 8 * r, row = c0 + lr;
            if (lr >= cr || row >= W.N) continue;
            // lane n handles column n (every lane holds every output)
#pragma unroll
            for (int n = 0; n < NC; ++n) {
                if (n != lane || n0 + n >= g.rows) continue;
                if constexpr (EPI == EPI_ARGMAX) {
                    if (g.logits) g.logits[(size_t)(n0 + n) * W.N + row] = out[r][n];
                    argmax_merge(bv, bi, out[r][n], (uint32_t)row);
                } else if (pre) {
                    epilogue_pre<EPI>(g, row, n0 + n, out[r][n], pb[r], px[r], step);
                } else {
                    epilogue_store<EPI>(g, row, n0 + n, out[r][n]);
                }
            }
        }
        if constexpr (STAGED) {
            __syncthreads();  // the stage is free
            if (tid == 0 && ci + RS < nchunks && !(blockIdx.x == 0 && ci + RS == A.withhold_chunk)) issue(ci + RS);
        }
    }
    if (!ok) {
        // a copy never completed: report, wait (bounded) for this CTA's copies
        // still in flight, produce nothing more
        if (tid == 0) {
            atomicOr(A.err, 2u);
            for (int k = ci; k < min(nchunks, ci + RS); ++k)
                if (!(blockIdx.x == 0 && k == A.withhold_chunk))
                    mbar_wait(&full[k % RS], (uint32_t)((k / RS) & 1), A.wait_ns);
        }
        return;
    }
    if constexpr (EPI == EPI_ARGMAX) {
        if (lane < NC) {
            best_v[warp][lane] = bv;
            best_i[warp][lane] = bi;
        }
        __syncthreads();
        if (tid < NC && n0 + tid < g.rows) {
            float v = best_v[0][tid];
            uint32_t i = best_i[0][tid];
            for (int w = 1; w < 8; ++w) argmax_merge(v, i, best_v[w][tid], best_i[w][tid]);
            g.part_v[(size_t)(n0 + tid) * gridDim.x + blockIdx.x] = v;
            g.part_i[(size_t)(n0 + tid) * gridDim.x + blockIdx.x] = i;
        }
    }
}

}  // namespace mgb
