// Batched quantized matmul on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Replaces candle's MMQ path (QMatMul::forward for more than 8 activation rows,
// model.rs:571-607, and the encoder's projections model.rs:137-154 / 463-477).
// The arithmetic is the engine's (kernels.cuh, BlockW): per 32-block the
// integer dot of weight and activation values is exact, so the tensor core
// computes it (tcgen05.mma kind::i8, M = 128 weight rows x N = NT activation
// rows x K = 32), each block into its own TMEM columns; the epilogue adds the
// blocks of a unit (a 256-value super-block for Q4_K / Q6_K, one block for
// Q8_0) in int32, applies the unit's float scales and sums the units left to
// right, so the results are bit-identical to the small-batch kernels.
//
// One persistent CTA per SM walks its (128-row x NT-token) tiles in stages of
// 8 blocks (256 values) with warp-specialized roles linked by mbarriers:
//   warp 10     producer: one TMA tensor copy per weight region (and, when the
//               activations come from global memory, one for their tiles and
//               one for their scale records) into a ring of RS stages;
//   warps EW-9  converters (EW = 4 for tiles of at most 16 tokens, else 8):
//               they unpack each block's 128 weight rows (Q4_K nibbles, Q6_K
//               6-bit values minus 32, Q8_0 bytes), loads batched ahead of stores,
//               into int8 128x32 tiles in the canonical no-swizzle layout (ring
//               of AG groups); Q6_K gets two tiles per block, each with the
//               other 16-value half zeroed, since the halves carry different
//               scales;
//   warp 11     MMA: each block's tcgen05.mma (two for Q6_K) into its TMEM
//               columns (ring of TG groups), one commit per group to the
//               barriers that free the tiles and wake the epilogue, one per
//               stage to free the stage;
//   warps 0..EW-1 epilogue: warp w reads TMEM lanes 32(w%4).. (its weight
//               rows) for all (EW = 4) or half (EW = 8) of the tile's tokens,
//               accumulates, and stores.
// (12 warps: three per scheduler leave 168 registers per thread.)
// Activations either arrive by TMA in the layout qprep_row_kernel writes (XM <
// 0: the encoder's long inputs), or (XM = a PrepMode: the decode step) the
// epilogue warps build the CTA's whole token tile in shared memory first
// (LayerNorm / embedding / plain input, quantized in the engine's order), so
// no separate activation kernel runs. A CTA then serves one token tile.
// Roles hand over groups of BG blocks (2-8), one mbarrier operation per group.
// Every mbarrier wait is bounded in time; when one runs out the CTA records an
// error flag, every role stops, and the CTA waits for its own MMAs before it
// releases TMEM and returns.
#pragma once
#include <cuda.h>

#include "fused.cuh"

namespace mgb {

namespace tc {

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, no swizzle, version 1 (sm_100).
__device__ __forceinline__ uint64_t sdesc(const void *p, uint32_t lbo, uint32_t sbo) {
    const uint64_t a = smem_u32(p);
    return ((a >> 4) & 0x3fffull) | ((uint64_t)((lbo >> 4) & 0x3fff) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3fff) << 32) | (1ull << 46);
}

// Instruction descriptor: kind::i8, D s32, A and B signed int8, both K-major.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        :
        : "r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}

__device__ __forceinline__ void commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t t, int (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(t));
}
__device__ __forceinline__ void tmem_ld8(uint32_t t, int (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(t));
}
__device__ __forceinline__ void tmem_ld4(uint32_t t, int (&r)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(t));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// TMA tensor copies (tile mode, no multicast) of one box into shared memory.
__device__ __forceinline__ void tma3(void *dst, const CUtensorMap *m, int c0, int c1, int c2, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(m), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma2(void *dst, const CUtensorMap *m, int c0, int c1, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(m), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

// Tensor maps of one launch: weight regions a, b, c, e (3-D: 8-byte words of
// one (32-row group, block) slice, blocks or super-blocks, groups), activation
// tiles (3-D: 8-byte words of an 8-row core group, row groups, blocks) and
// activation scale records (2-D: 8-byte words of a unit's rows, units).
struct Maps {
    CUtensorMap w[4];
    CUtensorMap xq, xr;
};

// The next matmul's activations, written by the CTA that completes them
// (RESID / RELU launches of the decode step): mode PREP_LN = LayerNorm of the
// finished output rows, once every row tile of a token tile is done (the last
// CTA of the token tile, found with an atomic counter); mode PREP_PLAIN = the
// output quantized per 256-row super-block, once both row tiles of it are done.
// mode < 0: none. Compiled only with MGB_TC_POST_STEPS=1: the decode step
// measured slower with them, and their registers make the RESID / RELU
// epilogues spill.
#ifndef MGB_TC_POST_STEPS
#define MGB_TC_POST_STEPS 0
#endif
struct Post {
    int mode = -1;
    const float *gamma = nullptr, *beta = nullptr;
    int group = 1, ctype = 0;   // the consumer's activation format
    QAct out;                   // the consumer's tensor-core layout (tq, trec, rs)
    uint32_t *counters = nullptr;  // one per token tile (LN) or (token tile, super-block); zero between launches
};

struct Args {
    Maps m;
    Post post;
    Matrix W;
    int rows;        // activation rows
    int row_tiles;   // Np / 128
    int tok_tiles;   // ceil(rows / NT)
    int tok0;        // first activation row (a multiple of 64) of this launch (TMA activations)
    GemvArgs g;      // epilogue outputs
    PrepArgs p;      // activation source (activations built in the kernel)
    // split-K (TMA activations): `splits` CTAs share a tile's stages; split 0
    // keeps the running row sum, the others store their unit partials in kpart,
    // and the last of them (kcount) continues the sum in unit order
    int splits;
    float *kpart;
    uint32_t *kcount;
    uint32_t *err;
};

// N of the MMA instruction: at least MGB_MMA_MIN_N (16, the smallest N of an
// M = 128 tcgen05.mma); a narrower token tile (NT = 8) is read twice (the
// descriptor's 8-row stride is 0), and the duplicate columns are not read.
#ifndef MGB_MMA_MIN_N
#define MGB_MMA_MIN_N 16
#endif
template <int NT>
struct MmaN {
    static constexpr int N = NT < MGB_MMA_MIN_N ? MGB_MMA_MIN_N : NT;
    static constexpr uint32_t SBO = NT < N ? 0u : 256u;  // B: bytes between 8-row core groups
    static_assert(N == NT || NT == 8, "narrow tile");
};

// Stage geometry per weight type, tile width and activation source.
template <int TYPE, int NT, bool FX>
struct Geo {
    static constexpr bool Q6 = TYPE == T_Q6_K, Q4 = TYPE == T_Q4_K, Q8 = TYPE == T_Q8_0;
    static constexpr int MN = MmaN<NT>::N;            // MMA columns per block (half)
    static constexpr int COLS = Q6 ? 2 * MN : MN;   // TMEM columns per block
    static constexpr int ABYTES = Q6 ? 8192 : 4096;  // converted tile(s) of one block
    static constexpr int KB = 8;                     // blocks per stage
    static constexpr int WA = Q8 ? 4 * KB * 1024 : 4 * KB * 512;                   // q / qs / ql
    static constexpr int WB = Q8 ? 4 * KB * 64 : (Q4 ? 4 * 512 : 4 * KB * 256);    // d / header / qh
    static constexpr int WC = Q6 ? 4 * KB * 64 : 0;                                // Q6_K scales
    static constexpr int WE = Q6 ? 4 * 64 : 0;                                     // Q6_K d
    static constexpr int RB = Q4 ? 32 : 4;                                         // record bytes
    static constexpr int UPS = Q8 ? KB : 1;                                        // units per stage
    static constexpr int oB = WA, oC = oB + WB, oE = oC + WC;
    static constexpr int oXQ = (oE + WE + 1023) / 1024 * 1024;
    static constexpr int oXR = oXQ + (FX ? 0 : KB * NT * 32);
    static constexpr int STAGE = (oXR + (FX ? 0 : UPS * NT * RB) + 1023) / 1024 * 1024;
    static constexpr uint32_t TX = WA + WB + WC + WE + (FX ? 0 : KB * NT * 32 + UPS * NT * RB);
    // Handoffs between roles move groups of BG blocks (one mbarrier operation
    // per group, not per block). TMEM holds TG groups of BG * COLS columns; the
    // converted tiles AG groups of BG tiles.
    static constexpr int BG = Q6 ? (NT >= 64 ? 2 : 4) : (NT >= 64 ? 4 : 8);
    static constexpr int GCOLS = BG * COLS;
    static constexpr int TG = 512 / GCOLS >= 4 ? 4 : 512 / GCOLS;
    static constexpr int AGB = BG * ABYTES;   // bytes of one converted group
    // resident activations (fused: room for 4096-value rows, at most 66 KB)
    static constexpr int RES = NT * 32 * 128 + 2048 < 66 * 1024 ? NT * 32 * 128 + 2048 : 66 * 1024;
    // converted groups: 3 when two stages still fit beside them, else 2
    static constexpr int AG = 220 * 1024 - (FX ? RES : 0) - 2 * STAGE >= 3 * AGB ? 3 : 2;
    // raw stages: as many as fit (2 to 4) beside the rest
    static constexpr int BUDGET = 220 * 1024 - AG * AGB - (FX ? RES : 0);
    static constexpr int RS = BUDGET / STAGE >= 4 ? 4 : (BUDGET / STAGE >= 3 ? 3 : 2);
    static_assert(2 * STAGE <= BUDGET, "stage ring does not fit");
    static_assert(8 % BG == 0 && TG >= 2, "group geometry");
    static constexpr int TCOLS_RAW = TG * GCOLS;
    static constexpr int TCOLS = TCOLS_RAW <= 32 ? 32 : (TCOLS_RAW <= 64 ? 64 : (TCOLS_RAW <= 128 ? 128 :
                                 (TCOLS_RAW <= 256 ? 256 : 512)));
    static constexpr int oRES = RS * STAGE + AG * AGB;   // resident activations (fused)
};

constexpr int kThreads = 384;  // 12 warps
constexpr int kProducerWarp = 10, kMmaWarp = 11;
// Epilogue warps 0..EW-1 and converter warps EW..9: narrow tiles (NT <= 16)
// leave the epilogue little to do per block, so four warps take all the tile's
// tokens and six convert; wider tiles split their tokens over eight epilogue
// warps and convert with two.
template <int NT>
struct Roles {
    static constexpr int EW = NT <= 16 ? 4 : 8;
    static constexpr int CW = kProducerWarp - EW;
};

// Resident activation bytes of a fused launch: tiles of every block, then the
// scale records of every unit.
__host__ __device__ inline size_t fused_act_bytes(int type, int nt, int nb) {
    const int units = type == T_Q8_0 ? nb : nb / 8, rb = type == T_Q4_K ? 32 : 4;
    return (size_t)nb * nt * 32 + (size_t)units * nt * rb;
}

}  // namespace tc

template <int TYPE, int NT, bool FX>
__host__ __device__ constexpr size_t gemm_tc_smem_base() {
    return 1024 + (size_t)tc::Geo<TYPE, NT, FX>::oRES;
}

// Argmax over the 32 lanes of NH tokens at once: halving steps hand half of the
// remaining tokens to the partner lane, so after log2(NH) steps every lane
// holds one token (lane >> (5 - log2 NH)) and plain butterfly steps finish it.
// The merge keeps the larger value and the lower index on ties, so the result
// is the same as any other order of comparisons.
template <int NH>
__device__ __forceinline__ void argmax_scatter(float (&v)[NH], uint32_t (&ix)[NH], int lane) {
    int c = NH, o = 16;
#pragma unroll
    for (int step = 0; step < 6; ++step) {
        if (c <= 1) break;
        const bool up = (lane & o) != 0;
        const int h = c / 2;
#pragma unroll
        for (int t = 0; t < NH / 2; ++t) {
            if (t >= h) break;
            const float mv = up ? v[t + h] : v[t], tv = up ? v[t] : v[t + h];
            const uint32_t mi = up ? ix[t + h] : ix[t], ti = up ? ix[t] : ix[t + h];
            const float rv = __shfl_xor_sync(0xffffffffu, tv, o);
            const uint32_t ri = __shfl_xor_sync(0xffffffffu, ti, o);
            float bv = mv;
            uint32_t bi = mi;
            argmax_merge(bv, bi, rv, ri);
            v[t] = bv;
            ix[t] = bi;
        }
        c = h;
        o >>= 1;
    }
#pragma unroll
    for (int step = 0; step < 5; ++step) {
        if (o == 0) break;
        const float rv = __shfl_xor_sync(0xffffffffu, v[0], o);
        const uint32_t ri = __shfl_xor_sync(0xffffffffu, ix[0], o);
        argmax_merge(v[0], ix[0], rv, ri);
        o >>= 1;
    }
}

// Builds the q8 activations of token tile `tt` in shared memory (fused mode):
// tiles [block][NT rows][32] in the UMMA K-major layout and the unit records.
// One warp per token (warps w, w+nw, ...); same arithmetic as the activation
// kernels: SUM32 LayerNorm statistics, then one scale per unit (the consumer's
// groups). Units are handled UC at a time so that their loads and their amax
// reductions overlap; Q4_K's per-block sums are added afterwards from the bytes.
template <int TYPE, int NT, int MODE>
__device__ void fused_prologue(const PrepArgs &p, int rows, int tt, bool write_x, uint8_t *xt, uint8_t *xr, int w,
                               int nw, int lane) {
    constexpr int G = act_group(TYPE), MAXV = 64;  // LayerNorm rows up to 2048 values
    constexpr int UC = G == 8 ? 4 : 16;            // units per batch (32 or 16 values per lane)
    const int K = p.K, T = K >> 5, nb = T, nu = nb / G;
    for (int n = w; n < NT; n += nw) {
        const int tok = tt * NT + n;
        if (tok >= rows) break;  // uniform across the warp
        uint32_t id = 0;
        const float *pos = nullptr;
        if constexpr (MODE == PREP_EMBED_LN) {
            id = p.ids[tok];
            pos = p.pos_table + (size_t)(*p.step + p.pos_base) * K;
        }
        auto input = [&](int i) -> float {
            if constexpr (MODE == PREP_EMBED_LN) {
                const float v = __fadd_rn(__fmul_rn(deq_elem(p.embed, (int)id, i), p.scale), pos[i]);
                if (write_x) p.x_out[(size_t)tok * K + i] = v;
                return v;
            } else {
                return p.x[(size_t)tok * K + i];
            }
        };
        float vals[MAXV];
        float mean = 0.f, rstd = 0.f;
        if constexpr (MODE != PREP_PLAIN) {
            // the whole row in registers: element 32t + lane in vals[t]
#pragma unroll
            for (int t = 0; t < MAXV; ++t)
                if (t < T) vals[t] = input(32 * t + lane);
            float sum = 0.0f;
#pragma unroll
            for (int t = 0; t < MAXV; ++t)
                if (t < T) sum = t == 0 ? vals[t] : __fadd_rn(sum, vals[t]);
            mean = __fdiv_rn(warp_tree(sum), (float)K);
            float s2 = 0.0f;
#pragma unroll
            for (int t = 0; t < MAXV; ++t)
                if (t < T) {
                    const float c = __fsub_rn(vals[t], mean);
                    const float c2 = __fmul_rn(c, c);
                    s2 = t == 0 ? c2 : __fadd_rn(s2, c2);
                }
            const float var = __fdiv_rn(warp_tree(s2), (float)K);
            rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
            // normalized values in place
#pragma unroll
            for (int t = 0; t < MAXV; ++t)
                if (t < T) {
                    const int i = 32 * t + lane;
                    vals[t] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(vals[t], mean), rstd), p.gamma[i]), p.beta[i]);
                }
        }
        // a batch of UC units: amax of each (interleaved reductions), then the bytes
        auto batch = [&](int u0, float (&y)[UC][G]) {
            float m[UC];
#pragma unroll
            for (int c = 0; c < UC; ++c) {
                m[c] = fabsf(y[c][0]);
#pragma unroll
                for (int g = 1; g < G; ++g) m[c] = fmaxf(m[c], fabsf(y[c][g]));
            }
#pragma unroll
            for (int c = 0; c < UC; ++c) m[c] = warp_max_nonneg(m[c]);
#pragma unroll
            for (int c = 0; c < UC; ++c) {
                const int u = u0 + c;
                if (u >= nu) break;
                const float dd = __fdiv_rn(m[c], 127.0f), id = __fdiv_rn(127.0f, m[c]);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const int t = u * G + g;
                    const int q = m[c] == 0.0f ? 0 : (int)roundf(__fmul_rn(y[c][g], id));
                    xt[(size_t)t * NT * 32 + tile_off(n, lane >> 4) + (lane & 15)] = (uint8_t)(int8_t)q;
                }
                if (lane == 0) {
                    if constexpr (TYPE == T_Q4_K) reinterpret_cast<float *>(xr)[((size_t)u * NT + n) * 8] = dd;
                    else reinterpret_cast<float *>(xr)[(size_t)u * NT + n] = G == 1 ? round_h(dd) : dd;
                }
            }
        };
        if constexpr (MODE != PREP_PLAIN) {
#pragma unroll
            for (int u0 = 0; u0 < MAXV / G; u0 += UC) {
                if (u0 >= nu) break;
                float y[UC][G];
#pragma unroll
                for (int c = 0; c < UC; ++c)
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const int t = (u0 + c) * G + g;
                        y[c][g] = t < MAXV ? vals[t < MAXV ? t : 0] : 0.0f;
                    }
                batch(u0, y);
            }
        } else {
            // next batch's loads are issued before this batch is quantized
            float y[2][UC][G];
            auto load = [&](int u0, float (&yy)[UC][G]) {
#pragma unroll
                for (int c = 0; c < UC; ++c)
#pragma unroll
                    for (int g = 0; g < G; ++g)
                        yy[c][g] = u0 + c < nu ? input(32 * ((u0 + c) * G + g) + lane) : 0.0f;
            };
            load(0, y[0]);
            for (int u0 = 0, k = 0; u0 < nu; u0 += UC, k ^= 1) {
                if (u0 + UC < nu) {
                    if (k == 0) load(u0 + UC, y[1]);
                    else load(u0 + UC, y[0]);
                }
                if (k == 0) batch(u0, y[0]);
                else batch(u0, y[1]);
            }
        }
    }
}

// Per-block sums of the quantized activations into the Q4_K records (after the
// tiles are complete): thread i handles (token, block) pairs i, i+nthreads, ...
template <int NT>
__device__ void fused_block_sums(int nb, int rows_here, const uint8_t *xt, uint8_t *xr, int i0, int nthreads) {
    for (int i = i0; i < rows_here * nb; i += nthreads) {
        const int n = i % rows_here, t = i / rows_here;
        const uint8_t *row = xt + (size_t)t * NT * 32;
        const int4 a = *reinterpret_cast<const int4 *>(row + tile_off(n, 0));
        const int4 b = *reinterpret_cast<const int4 *>(row + tile_off(n, 1));
        int s = 0;
        s = __dp4a(a.x, 0x01010101, s);
        s = __dp4a(a.y, 0x01010101, s);
        s = __dp4a(a.z, 0x01010101, s);
        s = __dp4a(a.w, 0x01010101, s);
        s = __dp4a(b.x, 0x01010101, s);
        s = __dp4a(b.y, 0x01010101, s);
        s = __dp4a(b.z, 0x01010101, s);
        s = __dp4a(b.w, 0x01010101, s);
        // record of unit t/8: {f32 scale, int16 sums of its 8 blocks}
        reinterpret_cast<int16_t *>(xr + ((size_t)(t >> 3) * NT + n) * 32 + 4)[t & 7] = (int16_t)s;
    }
}

// LayerNorm of finished rows y[tok][0..K) (K <= 2048) into the consumer's
// layout: one warp per token, SUM32 statistics in the engine's order.
template <int G>
__device__ void post_ln(const tc::Post &P, const float *y, int K, int t0, int t1, int w, int nw, int lane) {
    constexpr int MAXV = 64;
    const int T = K >> 5;
    for (int tok = t0 + w; tok < t1; tok += nw) {
        float vals[MAXV];
#pragma unroll
        for (int t = 0; t < MAXV; ++t)
            if (t < T) vals[t] = __ldcg(y + (size_t)tok * K + 32 * t + lane);
        float sum = 0.0f;
#pragma unroll
        for (int t = 0; t < MAXV; ++t)
            if (t < T) sum = t == 0 ? vals[t] : __fadd_rn(sum, vals[t]);
        const float mean = __fdiv_rn(warp_tree(sum), (float)K);
        float s2 = 0.0f;
#pragma unroll
        for (int t = 0; t < MAXV; ++t)
            if (t < T) {
                const float c = __fsub_rn(vals[t], mean);
                const float c2 = __fmul_rn(c, c);
                s2 = t == 0 ? c2 : __fadd_rn(s2, c2);
            }
        const float var = __fdiv_rn(warp_tree(s2), (float)K);
        const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
#pragma unroll
        for (int u = 0; u < MAXV / G; ++u) {
            if (u * G >= T) break;
            float v[G];
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const int t = u * G + g;
                v[g] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(vals[t], mean), rstd), __ldg(P.gamma + 32 * t + lane)),
                                 __ldg(P.beta + 32 * t + lane));
            }
            store_unit<G>(P.out, P.ctype, tok, u * G, v, lane);
        }
    }
}

// Super-block `sb` (256 values) of finished rows y[tok][0..K) into the
// consumer's layout: one warp per token.
template <int G>
__device__ void post_plain(const tc::Post &P, const float *y, int K, int sb, int t0, int t1, int w, int nw, int lane) {
    for (int tok = t0 + w; tok < t1; tok += nw) {
        float v[8];
#pragma unroll
        for (int g = 0; g < 8; ++g) v[g] = __ldcg(y + (size_t)tok * K + 256 * sb + 32 * g + lane);
        if constexpr (G == 8) {
            store_unit<8>(P.out, P.ctype, tok, 8 * sb, v, lane);
        } else {
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                const float one[1] = {v[g]};
                store_unit<1>(P.out, P.ctype, tok, 8 * sb + g, one, lane);
            }
        }
    }
}

// XM < 0: activations by TMA from the qprep_row_kernel layout; otherwise the
// PrepMode of the activations the CTA builds itself.
template <int TYPE, int EPI, int NT, int XM>
__global__ void __launch_bounds__(tc::kThreads, 1) gemm_tc_kernel(const __grid_constant__ tc::Args A) {
    using namespace tc;
    constexpr bool FX = XM >= 0;
    using G = Geo<TYPE, NT, FX>;
    constexpr int RS = G::RS, AG = G::AG, TG = G::TG, BG = G::BG, COLS = G::COLS;
    constexpr int EW = Roles<NT>::EW, CW = Roles<NT>::CW;
    constexpr int NH = NT * 4 / EW;  // tokens per epilogue warp
    constexpr uint32_t IDESC = idesc_i8(128, G::MN);
    extern __shared__ __align__(16) uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full[RS], empty[RS], afull[AG], aempty[AG], tfull[TG], tempty[TG], fin, xready,
        ebar;
    __shared__ uint32_t tmem_base_sh;
    __shared__ volatile int abort_sh;
    __shared__ float best_v[4][64];
    __shared__ uint32_t best_i[4][64];
    __shared__ int post_last;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const Matrix &W = A.W;
    const int NS = (W.nb + 7) / 8;  // stages per tile (Q8_0: the last may hold fewer blocks)
    // tiles of this CTA: TMA activations walk all tiles; fused activations keep
    // one token tile per CTA (gridDim.x is then a multiple of tok_tiles)
    const int splits = FX ? 1 : max(1, A.splits), NSS = NS / splits;  // stages per split
    const int NU = G::Q8 ? W.nb : W.nsb;                                 // units of a row
    const int tiles = A.row_tiles * A.tok_tiles * splits;
    const int my_tt = FX ? (int)blockIdx.x % A.tok_tiles : 0;
    const int first = FX ? (int)blockIdx.x / A.tok_tiles : (int)blockIdx.x;
    const int stride = FX ? (int)gridDim.x / A.tok_tiles : (int)gridDim.x;
    const int count = FX ? A.row_tiles : tiles;
    const int my_tiles = first < count ? (count - first + stride - 1) / stride : 0;
    uint8_t *base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint8_t *ring = base;                                 // RS x STAGE
    uint8_t *atile = base + (size_t)RS * G::STAGE;        // AG x BG x ABYTES
    uint8_t *xt = base + G::oRES;                         // fused: [nb][NT x 32]
    uint8_t *xr = xt + (size_t)W.nb * NT * 32;            // fused: [units][NT x RB]

    if (tid == 0) {
        for (int i = 0; i < RS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], CW + 1 + EW);
        }
        for (int i = 0; i < AG; ++i) {
            mbar_init(&afull[i], CW);
            mbar_init(&aempty[i], 1);
        }
        for (int i = 0; i < TG; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], EW);
        }
        mbar_init(&fin, 1);
        mbar_init(&xready, EW);
        mbar_init(&ebar, EW);
        abort_sh = 0;
    }
    if (EPI == EPI_ARGMAX)
        for (int n = tid; n < 256; n += blockDim.x) {
            best_v[n >> 6][n & 63] = kNegInf;
            best_i[n >> 6][n & 63] = 0xffffffffu;
        }
    if constexpr (G::Q6) {
        // the zero halves of the masked Q6_K tiles never change
        for (int i = tid; i < AG * BG * 2 * 128; i += blockDim.x) {
            const int slot = i >> 8, h = (i >> 7) & 1, r = i & 127;
            *reinterpret_cast<int4 *>(atile + slot * 8192 + h * 4096 + tile_off(r, h ^ 1)) = make_int4(0, 0, 0, 0);
        }
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                     "r"(G::TCOLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_async_smem();
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = tmem_base_sh;
    pdl_launch_dependents();

    // A failed wait: record it and make every role stop.
    auto fail = [&](uint32_t code) {
        atomicOr(A.err, code);
        abort_sh = 1;
    };
    // Warp-uniform bounded wait (every lane polls; all agree on the outcome).
    auto wwait = [&](uint64_t *bar, uint32_t parity, uint32_t code) -> bool {
        bool ok = mbar_wait(bar, parity);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok && lane == 0) fail(code);
        return ok && !abort_sh;
    };
    auto tile_rt = [&](int k) { return FX ? first + k * stride : (first + k * stride) % A.row_tiles; };
    auto tile_tt = [&](int k) { return FX ? my_tt : ((first + k * stride) / A.row_tiles) % A.tok_tiles; };
    auto tile_s0 = [&](int k) { return FX ? 0 : (first + k * stride) / (A.row_tiles * A.tok_tiles) * NSS; };

    // Ring position: slot and phase parity, advanced by next().
    struct Pos {
        int slot = 0;
        uint32_t phase = 0, n = 0;
        __device__ void next(int size) {
            ++n;
            if (++slot == size) {
                slot = 0;
                phase ^= 1;
            }
        }
    };
    // blocks [g * BG, ...) of a stage holding nbs blocks
    auto group_blocks = [&](int g, int nbs) { return min(BG, nbs - g * BG); };

    if (warp == kProducerWarp) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const int first_stages = my_tiles > 0 ? min(RS, NSS) : 0;
            auto weights = [&](int rt, int s, uint8_t *dst, uint64_t *bar) {
                const int g0 = 4 * rt;
                tma3(dst, &A.m.w[0], 0, 8 * s, g0, bar);
                if constexpr (G::Q4) tma3(dst + G::oB, &A.m.w[1], 0, s, g0, bar);
                else tma3(dst + G::oB, &A.m.w[1], 0, 8 * s, g0, bar);
                if constexpr (G::Q6) {
                    tma3(dst + G::oC, &A.m.w[2], 0, 8 * s, g0, bar);
                    tma3(dst + G::oE, &A.m.w[3], 0, s, g0, bar);
                }
            };
            auto acts = [&](int tt, int s, uint8_t *dst, uint64_t *bar) {
                if constexpr (!FX) {
                    const int t0 = A.tok0 + tt * NT;
                    tma3(dst + G::oXQ, &A.m.xq, 0, t0 / 8, 8 * s, bar);
                    if constexpr (G::Q4) tma2(dst + G::oXR, &A.m.xr, t0 * 4, s, bar);
                    else if constexpr (G::Q6) tma2(dst + G::oXR, &A.m.xr, t0 / 2, s, bar);
                    else tma2(dst + G::oXR, &A.m.xr, t0 / 2, 8 * s, bar);
                }
            };
            // weights of the first stages do not depend on the previous kernel
            for (int s = 0; s < first_stages; ++s) {
                mbar_expect_tx(&full[s], G::TX);
                weights(tile_rt(0), tile_s0(0) + s, ring + (size_t)s * G::STAGE, &full[s]);
            }
            pdl_wait();
            Pos st;
            for (int k = 0; k < my_tiles && !abort_sh; ++k) {
                const int rt = tile_rt(k), tt = tile_tt(k), s0 = tile_s0(k);
                for (int s = s0; s < s0 + NSS; ++s, st.next(RS)) {
                    uint8_t *dst = ring + (size_t)st.slot * G::STAGE;
                    if (st.n >= (uint32_t)first_stages) {
                        if (st.n >= (uint32_t)RS && !mbar_wait(&empty[st.slot], st.phase ^ 1)) {
                            fail(8u);
                            break;
                        }
                        if (abort_sh) break;
                        mbar_expect_tx(&full[st.slot], G::TX);
                        weights(rt, s, dst, &full[st.slot]);
                    }
                    acts(tt, s, dst, &full[st.slot]);
                }
            }
        }
    } else if (warp == kMmaWarp) {
        // ----------------------------------------------------------------- MMA
        // (nothing to do before the predecessor's outputs exist: waiting here
        // keeps this warp off the issue slots of the predecessor's warps)
        if constexpr (!FX) pdl_wait();
        if (lane == 0) {
            Pos st, ag, tg;
            // Descriptors are formed once and advanced by constant 16-byte
            // steps (shared-memory offsets stay below 256 KB, so the 14-bit
            // address field never carries): the issue loop is the MMAs alone.
            const uint64_t a_base = sdesc(atile, 128, 256);
            const uint64_t x_base = sdesc(FX ? xt : ring + G::oXQ, 128, MmaN<NT>::SBO);
            if (FX && my_tiles > 0 && !mbar_wait(&xready, 0)) fail(16u);
            for (int k = 0; k < my_tiles && !abort_sh; ++k) {
                const int s0 = tile_s0(k);
                for (int s = s0; s < s0 + NSS && !abort_sh; ++s, st.next(RS)) {
                    if (!mbar_wait(&full[st.slot], st.phase)) {
                        fail(16u);
                        break;
                    }
                    const uint64_t xs =
                        x_base + (uint64_t)(FX ? (8 * s * NT * 32) >> 4 : (st.slot * G::STAGE) >> 4);
                    const int nbs = min(8, W.nb - 8 * s);
                    for (int g = 0; g * BG < nbs; ++g, ag.next(AG), tg.next(TG)) {
                        if (!mbar_wait(&afull[ag.slot], ag.phase) ||
                            (tg.n >= (uint32_t)TG && !mbar_wait(&tempty[tg.slot], tg.phase ^ 1))) {
                            fail(16u);
                            break;
                        }
                        if (abort_sh) break;
                        fence_after();
                        const uint64_t ag0 = a_base + (uint64_t)((ag.slot * G::AGB) >> 4);
                        const uint64_t xg0 = xs + (uint64_t)((g * BG * NT * 32) >> 4);
                        const uint32_t td = tmem + tg.slot * G::GCOLS;
                        const int gb = group_blocks(g, nbs);
#pragma unroll
                        for (int b = 0; b < BG; ++b) {
                            if (b >= gb) break;
                            const uint64_t db = xg0 + (uint64_t)((b * NT * 32) >> 4);
                            mma_i8(td + b * COLS, ag0 + (uint64_t)((b * G::ABYTES) >> 4), db, IDESC);
                            if constexpr (G::Q6)
                                mma_i8(td + b * COLS + G::MN, ag0 + (uint64_t)((b * G::ABYTES + 4096) >> 4), db, IDESC);
                        }
                        commit(&aempty[ag.slot]);
                        commit(&tfull[tg.slot]);
                    }
                    commit(&empty[st.slot]);
                }
            }
            // every MMA issued by this thread has completed before TMEM is released
            commit(&fin);
            if (!mbar_wait(&fin, 0)) fail(16u);
        }
    } else if (warp >= EW) {
        // ---------------------------------------------------------- converters
        if constexpr (!FX) pdl_wait();  // (as the MMA warp)
        // items of a group: (weight row r, block bb) = (i % 128, i / 128) for
        // i = ct, ct + CT, ...; a warp's 32 items are 32 consecutive rows of one
        // block. Each batch of LB items is loaded before any of it is stored.
        constexpr int CT = 32 * CW, IPT = (128 * BG + CT - 1) / CT, LB = IPT < 8 ? IPT : 8;
        const int ct = tid - 32 * EW;
        struct Raw {
            int4 a;
            int4 b;  // Q8_0: bytes 16-31; Q6_K: high bits in b.x, b.y
        };
        Pos st, ag;
        bool ok = true;
        for (int k = 0; k < my_tiles && ok && !abort_sh; ++k) {
            const int s0 = tile_s0(k);
            for (int s = s0; s < s0 + NSS && ok; ++s, st.next(RS)) {
                if (!(ok = wwait(&full[st.slot], st.phase, 32u))) break;
                const uint8_t *stg = ring + (size_t)st.slot * G::STAGE;
                const int nbs = min(8, W.nb - 8 * s);
                for (int g = 0; g * BG < nbs; ++g, ag.next(AG)) {
                    if (ag.n >= (uint32_t)AG && !(ok = wwait(&aempty[ag.slot], ag.phase ^ 1, 32u))) break;
                    const int items = 128 * group_blocks(g, nbs);
                    uint8_t *tg0 = atile + (size_t)ag.slot * G::AGB;
#pragma unroll
                    for (int k0 = 0; k0 < IPT; k0 += LB) {
                        Raw raw[LB];
#pragma unroll
                        for (int u = 0; u < LB; ++u) {
                            const int i = ct + (k0 + u) * CT;
                            if (k0 + u >= IPT || i >= items) break;
                            const int r = i & 127, b = g * BG + (i >> 7), gi = r >> 5, l = r & 31;
                            if constexpr (G::Q8) {
                                const int4 *src = reinterpret_cast<const int4 *>(stg + (gi * 8 + b) * 1024 + l * 32);
                                raw[u].a = src[0];
                                raw[u].b = src[1];
                            } else if constexpr (G::Q4) {
                                raw[u].a = *reinterpret_cast<const int4 *>(stg + (gi * 8 + b) * 512 + l * 16);
                            } else {
                                raw[u].a = *reinterpret_cast<const int4 *>(stg + (gi * 8 + b) * 512 + l * 16);
                                const uint2 hq = *reinterpret_cast<const uint2 *>(stg + G::oB + (gi * 8 + b) * 256 + l * 8);
                                raw[u].b.x = (int)hq.x;
                                raw[u].b.y = (int)hq.y;
                            }
                        }
#pragma unroll
                        for (int u = 0; u < LB; ++u) {
                            const int i = ct + (k0 + u) * CT;
                            if (k0 + u >= IPT || i >= items) break;
                            const int r = i & 127;
                            uint8_t *ta = tg0 + (i >> 7) * G::ABYTES;
                            const int4 v = raw[u].a;
                            if constexpr (G::Q8) {
                                *reinterpret_cast<int4 *>(ta + tile_off(r, 0)) = v;
                                *reinterpret_cast<int4 *>(ta + tile_off(r, 1)) = raw[u].b;
                            } else if constexpr (G::Q4) {
                                *reinterpret_cast<int4 *>(ta + tile_off(r, 0)) =
                                    make_int4(v.x & 0x0f0f0f0f, v.y & 0x0f0f0f0f, v.z & 0x0f0f0f0f, v.w & 0x0f0f0f0f);
                                *reinterpret_cast<int4 *>(ta + tile_off(r, 1)) =
                                    make_int4((v.x >> 4) & 0x0f0f0f0f, (v.y >> 4) & 0x0f0f0f0f,
                                              (v.z >> 4) & 0x0f0f0f0f, (v.w >> 4) & 0x0f0f0f0f);
                            } else {
                                const uint32_t hx = (uint32_t)raw[u].b.x, hy = (uint32_t)raw[u].b.y;
                                const int ql[4] = {v.x, v.y, v.z, v.w};
                                int a4[4], b4[4];
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    a4[e] = (int)__vsub4(
                                        (uint32_t)((ql[e] & 0x0f0f0f0f) | (int)(((hx >> (2 * e)) & 0x03030303u) << 4)),
                                        0x20202020u);
                                    b4[e] = (int)__vsub4((uint32_t)(((ql[e] >> 4) & 0x0f0f0f0f) |
                                                                    (int)(((hy >> (2 * e)) & 0x03030303u) << 4)),
                                                         0x20202020u);
                                }
                                // tile 0: values 0-15 (k16 = 0), tile 1: values 16-31 (k16 = 1)
                                *reinterpret_cast<int4 *>(ta + tile_off(r, 0)) = make_int4(a4[0], a4[1], a4[2], a4[3]);
                                *reinterpret_cast<int4 *>(ta + 4096 + tile_off(r, 1)) =
                                    make_int4(b4[0], b4[1], b4[2], b4[3]);
                            }
                        }
                    }
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&afull[ag.slot]);
                }
                if (!ok) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[st.slot]);
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3, e = warp >> 2;
        const int r = 32 * q + lane, gi = q, l = lane;
        const int n0 = e * NH;  // first token (within the tile) of this warp
        pdl_wait();
        // the decode step (QKV cache position), written by the previous step's kernels
        const int qkv_step = EPI == EPI_QKV ? (int)*A.g.step : 0;
        if constexpr (FX) {
            // this CTA's token tile, built once; the first row tile writes x (embedding)
            if (my_tiles > 0) {
                fused_prologue<TYPE, NT, (FX ? XM : 0)>(A.p, A.rows, my_tt, first == 0, xt, xr, warp, EW, lane);
                if constexpr (G::Q4) {
                    asm volatile("bar.sync 1, %0;" ::"r"(32 * EW) : "memory");  // the epilogue warps
                    fused_block_sums<NT>(W.nb, min(NT, A.rows - my_tt * NT), xt, xr, tid, 32 * EW);
                }
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&xready);
        }
        Pos st, tg;
        uint32_t ephase = 0;
        bool ok = true;
        for (int k = 0; k < my_tiles && ok && !abort_sh; ++k) {
            const int rt = tile_rt(k), tt = tile_tt(k), s0 = tile_s0(k);
            const int row = rt * 128 + r;
            const bool live = row < W.N;
            // split-K partials of this tile: [unit][NT tokens][128 rows]
            float *kp = splits > 1 ? A.kpart + (size_t)(tt * A.row_tiles + rt) * NU * NT * 128 : nullptr;
            float acc[NH];
#pragma unroll
            for (int n = 0; n < NH; ++n) acc[n] = 0.0f;
            // This row's bias (and for RESID the tile's residual values) read
            // while the tile's stages are still in flight, so the stores below
            // wait on no load (no other CTA writes these residual values)
            const float bias = live && W.bias ? __ldg(W.bias + row) : 0.0f;
            float res[EPI == EPI_RESID ? NH : 1];
            if constexpr (EPI == EPI_RESID) {
#pragma unroll
                for (int n = 0; n < NH; ++n) {
                    const int tok = tt * NT + n0 + n;
                    res[n] = live && tok < A.rows ? __ldcg(A.g.y + (size_t)tok * W.N + row) : 0.0f;
                }
            }
            // QKV: q row, or this row's place in the step's K or V cache entry
            float *qkv_q = nullptr;
            __half *qkv_c = nullptr;
            size_t qkv_tok = 0;
            if constexpr (EPI == EPI_QKV) {
                const int dm = A.g.H * A.g.hd;
                if (row < dm) {
                    qkv_q = A.g.q + row;
                    qkv_tok = dm;
                } else if (live) {
                    const int c = row - dm, which = c / dm, h = (c % dm) / A.g.hd, t = c % A.g.hd;
                    qkv_c = (which == 0 ? A.g.kc : A.g.vc) + ((size_t)h * A.g.m + qkv_step) * A.g.hd + t;
                    qkv_tok = (size_t)A.g.H * A.g.m * A.g.hd;
                }
            }
            for (int s = s0; s < s0 + NSS && ok; ++s, st.next(RS)) {
                if (!(ok = wwait(&full[st.slot], st.phase, 64u))) break;
                const uint8_t *stg = ring + (size_t)st.slot * G::STAGE;
                // records of this stage's units: [unit][NT x RB]
                const uint8_t *rec = FX ? xr + (size_t)(G::Q8 ? 8 * s : s) * NT * G::RB : stg + G::oXR;
                // this row's scales for the stage
                float d = 0.f, dm = 0.f;
                uint32_t mpk0 = 0, mpk1 = 0, scpk0 = 0, scpk1 = 0;
                if constexpr (G::Q4) {
                    const uint4 h = *reinterpret_cast<const uint4 *>(stg + G::oB + gi * 512 + l * 16);
                    d = h2f(h.x & 0xffff);
                    dm = h2f(h.x >> 16);
                    auto byte = [&](int kk) -> uint32_t {
                        const uint32_t w = kk < 4 ? h.y : (kk < 8 ? h.z : h.w);
                        return (w >> (8 * (kk & 3))) & 0xff;
                    };
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        uint32_t sc, mm;
                        if (kk < 4) {
                            sc = byte(kk) & 63;
                            mm = byte(kk + 4) & 63;
                        } else {
                            sc = (byte(kk + 4) & 0xf) | ((byte(kk - 4) >> 6) << 4);
                            mm = (byte(kk + 4) >> 4) | ((byte(kk) >> 6) << 4);
                        }
                        if (kk < 4) {
                            scpk0 |= sc << (8 * kk);
                            mpk0 |= mm << (8 * kk);
                        } else {
                            scpk1 |= sc << (8 * (kk - 4));
                            mpk1 |= mm << (8 * (kk - 4));
                        }
                    }
                } else if constexpr (G::Q6) {
                    d = h2f(*reinterpret_cast<const unsigned short *>(stg + G::oE + gi * 64 + l * 2));
                }
                int S[NH];
#pragma unroll
                for (int n = 0; n < NH; ++n) S[n] = 0;
                const int nbs = min(8, W.nb - 8 * s);
                for (int g = 0; g * BG < nbs && ok; ++g, tg.next(TG)) {
                    if (!(ok = wwait(&tfull[tg.slot], tg.phase, 64u))) break;
                    fence_after();
                    for (int bb = 0; bb < group_blocks(g, nbs); ++bb) {
                    const int b = g * BG + bb;
                    const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + tg.slot * G::GCOLS + bb * COLS + n0;
                    int sa = 0, sb = 0;
                    float db = 0.f;
                    if constexpr (G::Q4) {
                        sa = (int)(((b < 4 ? scpk0 : scpk1) >> (8 * (b & 3))) & 0xff);
                    } else if constexpr (G::Q6) {
                        const unsigned short sc2 =
                            *reinterpret_cast<const unsigned short *>(stg + G::oC + (gi * 8 + b) * 64 + l * 2);
                        sa = (int8_t)(sc2 & 0xff);
                        sb = (int8_t)(sc2 >> 8);
                    } else {
                        db = h2f(*reinterpret_cast<const unsigned short *>(stg + G::oB + (gi * 8 + b) * 64 + l * 2));
                    }
                    // TMEM -> registers in chunks of up to 16 tokens; the next chunk's
                    // load is in flight while the current one is accumulated
                    constexpr int CH = NH < 16 ? NH : 16, NC = NH / CH;
                    int va[2][CH], vb[2][CH];
                    auto ld = [&](int c, int (&a)[CH], int (&bv)[CH]) {
                        if constexpr (CH == 16) {
                            tmem_ld16(ta + c * CH, a);
                            if constexpr (G::Q6) tmem_ld16(ta + G::MN + c * CH, bv);
                        } else if constexpr (CH == 8) {
                            tmem_ld8(ta + c * CH, a);
                            if constexpr (G::Q6) tmem_ld8(ta + G::MN + c * CH, bv);
                        } else {
                            static_assert(CH == 4, "token chunk");
                            tmem_ld4(ta + c * CH, a);
                            if constexpr (G::Q6) tmem_ld4(ta + G::MN + c * CH, bv);
                        }
                    };
                    ld(0, va[0], vb[0]);
#pragma unroll
                    for (int c = 0; c < NC; ++c) {
                        tmem_wait_ld();
                        if (c + 1 < NC) ld(c + 1, va[(c + 1) & 1], vb[(c + 1) & 1]);
#pragma unroll
                        for (int i = 0; i < CH; ++i) {
                            const int n = c * CH + i;
                            const int I = va[c & 1][i];
                            if constexpr (G::Q4) {
                                S[n] += sa * I;
                            } else if constexpr (G::Q6) {
                                S[n] += sa * I + sb * vb[c & 1][i];
                            } else {
                                const float xd = reinterpret_cast<const float *>(rec)[b * NT + n0 + n];
                                const float p = __fmul_rn(__fmul_rn(db, xd), (float)I);
                                if (s0 == 0) acc[n] = (s == 0 && b == 0) ? p : __fadd_rn(acc[n], p);
                                else kp[((size_t)(8 * s + b) * NT + n0 + n) * 128 + r] = p;
                            }
                        }
                    }
                    }
                    fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[tg.slot]);
                }
                if (!ok) break;
                if constexpr (!G::Q8) {
                    // finish the super-block: float scales once, then the row sum
#pragma unroll
                    for (int n = 0; n < NH; ++n) {
                        float p;
                        if constexpr (G::Q4) {
                            const int4 rv = *reinterpret_cast<const int4 *>(rec + (n0 + n) * 32);
                            const float xd = __int_as_float(rv.x);
                            // S2 = sum_j m_j * s32_j (s32 pairs as int16x2, m_j as bytes)
                            int S2 = __dp2a_lo(rv.y, (int)mpk0, 0);
                            S2 = __dp2a_hi(rv.z, (int)mpk0, S2);
                            S2 = __dp2a_lo(rv.w, (int)mpk1, S2);
                            S2 = __dp2a_hi(*reinterpret_cast<const int *>(rec + (n0 + n) * 32 + 16), (int)mpk1, S2);
                            p = __fmul_rn(xd, __fsub_rn(__fmul_rn(d, (float)S[n]), __fmul_rn(dm, (float)S2)));
                        } else {
                            const float xd = reinterpret_cast<const float *>(rec)[n0 + n];
                            p = __fmul_rn(__fmul_rn(d, xd), (float)S[n]);
                        }
                        if (s0 == 0) acc[n] = s == 0 ? p : __fadd_rn(acc[n], p);
                        else kp[((size_t)s * NT + n0 + n) * 128 + r] = p;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[st.slot]);
            }
            if (!ok || abort_sh) break;
            if (splits > 1) {
                // split 0 leaves its running sum in unit slot 0 (a unit it summed itself)
                if (s0 == 0)
#pragma unroll
                    for (int n = 0; n < NH; ++n) kp[(size_t)(n0 + n) * 128 + r] = acc[n];
                __syncwarp();
                if (lane == 0) mbar_arrive(&ebar);
                if (!(ok = wwait(&ebar, ephase, 128u))) break;
                ephase ^= 1;
                if (tid == 0) {
                    __threadfence();
                    const uint32_t old = atomicAdd(&A.kcount[tt * A.row_tiles + rt], 1u);
                    post_last = old + 1 == (uint32_t)splits;
                    if (post_last) {
                        A.kcount[tt * A.row_tiles + rt] = 0;  // every split of this launch has counted
                        __threadfence();
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&ebar);
                if (!(ok = wwait(&ebar, ephase, 128u))) break;
                ephase ^= 1;
                if (!post_last) continue;  // another split finishes this tile
                // the row sum continued in unit order from the stored partials,
                // UB units x NH tokens of loads in flight per batch
                const int u1 = G::Q8 ? 8 * NSS : NSS;  // first unit of split 1
                constexpr int UB = NH <= 8 ? 8 : (NH <= 16 ? 4 : 2);
#pragma unroll
                for (int n = 0; n < NH; ++n) acc[n] = __ldcg(kp + (size_t)(n0 + n) * 128 + r);
                for (int u0 = u1; u0 < NU; u0 += UB) {
                    float v[UB][NH];
#pragma unroll
                    for (int j = 0; j < UB; ++j)
#pragma unroll
                        for (int n = 0; n < NH; ++n)
                            v[j][n] = u0 + j < NU ? __ldcg(kp + ((size_t)(u0 + j) * NT + n0 + n) * 128 + r) : 0.0f;
#pragma unroll
                    for (int j = 0; j < UB; ++j) {
                        if (u0 + j >= NU) break;
#pragma unroll
                        for (int n = 0; n < NH; ++n) acc[n] = __fadd_rn(acc[n], v[j][n]);
                    }
                }
            }
            // tile epilogue
            if constexpr (EPI == EPI_ARGMAX) {
                uint32_t bi[NH];
#pragma unroll
                for (int n = 0; n < NH; ++n) {
                    const int tok = tt * NT + n0 + n;
                    if (A.g.logits && live && tok < A.rows) A.g.logits[(size_t)tok * W.N + row] = acc[n];
                    if (!live) acc[n] = kNegInf;
                    bi[n] = live ? (uint32_t)row : 0xffffffffu;
                }
                argmax_scatter<NH>(acc, bi, lane);
                constexpr int LPT = 32 / NH;  // lanes per token after the scatter
                if (lane % LPT == 0) {
                    const int tok = tt * NT + n0 + lane / LPT;  // < 64 in an ARGMAX launch
                    if (tok < A.rows) argmax_merge(best_v[q][tok], best_i[q][tok], acc[0], bi[0]);
                }
            } else {
#pragma unroll
                for (int n = 0; n < NH; ++n) {
                    const int tok = tt * NT + n0 + n;
                    if (tok >= A.rows) break;  // uniform across the warp
                    if (!live) continue;
                    if constexpr (EPI == EPI_RESID) {
                        A.g.y[(size_t)tok * W.N + row] = __fadd_rn(__fadd_rn(acc[n], bias), res[n]);
                    } else if constexpr (EPI == EPI_STORE) {
                        A.g.y[(size_t)tok * W.N + row] = W.bias ? __fadd_rn(acc[n], bias) : acc[n];
                    } else if constexpr (EPI == EPI_RELU) {
                        const float y = __fadd_rn(acc[n], bias);
                        A.g.y[(size_t)tok * W.N + row] = y > 0.0f ? y : 0.0f;
                    } else if constexpr (EPI == EPI_QKV) {
                        const float y = __fadd_rn(acc[n], bias);
                        if (qkv_q) qkv_q[tok * qkv_tok] = y;
                        else qkv_c[tok * qkv_tok] = __float2half_rn(y);
                    } else {
                        epilogue_store<EPI>(A.g, row, tok, acc[n]);
                    }
                }
                if constexpr (MGB_TC_POST_STEPS && (EPI == EPI_RESID || EPI == EPI_RELU)) {
                    if (A.post.mode >= 0) {
                        // the tile's outputs are stored; count it, and the CTA that
                        // completes a token tile (LN) / super-block (PLAIN) prepares it
                        const bool ln = A.post.mode == PREP_LN;
                        // the 8 epilogue warps meet on a bounded mbarrier (a warp that
                        // stopped on an error makes the others time out, not hang)
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&ebar);
                        if (!(ok = wwait(&ebar, ephase, 128u))) break;
                        ephase ^= 1;
                        if (tid == 0) {
                            __threadfence();
                            const int idx = ln ? tt : tt * (A.row_tiles / 2) + rt / 2;
                            const uint32_t old = atomicAdd(&A.post.counters[idx], 1u);
                            post_last = old + 1 == (ln ? (uint32_t)A.row_tiles : 2u);
                            if (post_last) {
                                A.post.counters[idx] = 0;  // every CTA of this launch has counted
                                __threadfence();
                            }
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&ebar);
                        if (!(ok = wwait(&ebar, ephase, 128u))) break;
                        ephase ^= 1;
                        if (post_last) {
                            const int t0 = tt * NT, t1 = min(A.rows, t0 + NT);
                            if (ln) {
                                if (A.post.group == 8) post_ln<8>(A.post, A.g.y, W.N, t0, t1, warp, EW, lane);
                                else post_ln<1>(A.post, A.g.y, W.N, t0, t1, warp, EW, lane);
                            } else {
                                if (A.post.group == 8) post_plain<8>(A.post, A.g.y, W.N, rt / 2, t0, t1, warp, EW, lane);
                                else post_plain<1>(A.post, A.g.y, W.N, rt / 2, t0, t1, warp, EW, lane);
                            }
                        }
                    }
                }
            }
        }
    }
    // (the producer's lane 0 and the epilogue warps waited on the previous
    // kernel, so this CTA cannot finish before it)
    fence_before();
    __syncthreads();
    if constexpr (EPI == EPI_ARGMAX) {
        // one partial per (activation row, CTA); ARGMAX launches cover at most 64 rows
        for (int n = tid; n < A.rows && n < 64; n += blockDim.x) {
            float v = best_v[0][n];
            uint32_t i = best_i[0][n];
            for (int w = 1; w < 4; ++w) argmax_merge(v, i, best_v[w][n], best_i[w][n]);
            A.g.part_v[(size_t)n * gridDim.x + blockIdx.x] = v;
            A.g.part_i[(size_t)n * gridDim.x + blockIdx.x] = i;
        }
    }
    if (warp == kMmaWarp) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(G::TCOLS) : "memory");
    }
}

// Tensor-core layout of one activation row (one CTA per row): the row is staged
// in shared memory (embedding rows dequantized once), LayerNorm statistics by
// one warp in the fixed order, quantized with the consumer's scale groups, then
// written as
//   tq : per block j, 8-row core groups of 256 bytes [j][row/8][k16][row%8][16 B]
//        (the UMMA K-major no-swizzle layout);
//   trec: per unit u (super-block, or block for Q8_0 consumers) and row:
//        Q4_K: {f32 scale, int16 block sums x 8, 12 zero bytes} (32 B);
//        Q6_K: f32 scale; Q8_0: f32 (f16-rounded) scale.
template <int MODE>
__global__ void __launch_bounds__(256) qprep_row_kernel(PrepArgs p, QAct out) {
    extern __shared__ __align__(16) uint8_t qsm[];
    __shared__ float st[2];
    __shared__ uint32_t id_sh[1];
    const int r = blockIdx.x, K = p.K, nb = K >> 5;
    // LayerNorm parameters into shared memory before the dependency wait (they
    // are weights, not the predecessor's output)
    float *gb = reinterpret_cast<float *>(qsm + (size_t)K * 5 + (size_t)nb * 16);  // gamma[K], beta[K]
    if constexpr (MODE != PREP_PLAIN) {
        for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
            reinterpret_cast<float4 *>(gb)[i] = __ldg(reinterpret_cast<const float4 *>(p.gamma) + i);
            reinterpret_cast<float4 *>(gb + K)[i] = __ldg(reinterpret_cast<const float4 *>(p.beta) + i);
        }
    }
    pdl_wait();
    float *xs = reinterpret_cast<float *>(qsm);                 // K floats
    SmAct s;
    s.q = reinterpret_cast<int8_t *>(qsm + (size_t)K * 4);      // K bytes
    s.d = reinterpret_cast<float *>(qsm + (size_t)K * 5);       // nb
    s.s32 = reinterpret_cast<int *>(s.d + nb);                  // nb
    s.s16 = s.s32 + nb;                                         // 2 nb
    s.st = st;
    s.xf = nullptr;
    PrepArgs pa = p;
    if constexpr (MODE == PREP_EMBED_LN) {
        if (threadIdx.x == 0) id_sh[0] = p.ids[r];
        pa.pos_table += (size_t)(*p.step + p.pos_base) * K;
        pa.ids = id_sh;
        __syncthreads();
    }
    // 8 loads in flight per thread before their stores (one memory round trip)
    for (int base = threadIdx.x; base < K; base += 8 * blockDim.x) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = base + u * blockDim.x;
            v[u] = i < K ? act_input<MODE>(pa, MODE == PREP_EMBED_LN ? 0 : r, i) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = base + u * blockDim.x;
            if (i >= K) break;
            xs[i] = v[u];
            if constexpr (MODE == PREP_EMBED_LN) p.x_out[(size_t)r * K + i] = v[u];
        }
    }
    __syncthreads();
    PrepArgs q = p;
    q.x = xs;
    q.rows = 1;
    if constexpr (MODE != PREP_PLAIN) {
        q.gamma = gb;
        q.beta = gb + K;
    }
    constexpr int M2 = MODE == PREP_PLAIN ? PREP_PLAIN : PREP_LN;
    if (p.group == 8) build_activations_impl<M2, 8>(q, s, 1, false);
    else build_activations_impl<M2, 1>(q, s, 1, false);
    // build_activations_impl ends with __syncthreads
    // the next matmul is released once the activations are built (measured
    // slightly faster than releasing it at the start)
    pdl_launch_dependents();
    const int rs = out.rs;
    for (int c = threadIdx.x; c < nb * 2; c += blockDim.x) {
        const int j = c >> 1, k16 = c & 1;
        *reinterpret_cast<int4 *>(out.tq + ((size_t)j * (rs / 8) + (r >> 3)) * 256 + tile_off(r & 7, k16)) =
            *reinterpret_cast<const int4 *>(s.q + 32 * j + 16 * k16);
    }
    if (p.ctype == T_Q4_K) {
        for (int u = threadIdx.x; u < nb / 8; u += blockDim.x) {
            int w[8];
            w[0] = __float_as_int(s.d[8 * u]);
#pragma unroll
            for (int k = 0; k < 4; ++k)
                w[1 + k] = (s.s32[8 * u + 2 * k] & 0xffff) | (s.s32[8 * u + 2 * k + 1] << 16);
            w[5] = w[6] = w[7] = 0;
            int4 *dst = reinterpret_cast<int4 *>(out.trec + ((size_t)u * rs + r) * 32);
            dst[0] = make_int4(w[0], w[1], w[2], w[3]);
            dst[1] = make_int4(w[4], w[5], w[6], w[7]);
        }
    } else {
        const int units = p.ctype == T_Q6_K ? nb / 8 : nb, step = p.ctype == T_Q6_K ? 8 : 1;
        for (int u = threadIdx.x; u < units; u += blockDim.x)
            reinterpret_cast<float *>(out.trec)[(size_t)u * rs + r] = s.d[u * step];
    }
}

}  // namespace mgb
