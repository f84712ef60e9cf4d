// Batched quantized matmul on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Replaces candle's MMQ path (QMatMul::forward for more than 8 activation rows,
// model.rs:571-607, and the encoder's projections model.rs:137-154 / 463-477;
// candle-kernels 0.11.0 src/quantized.cu mul_mat_q). The arithmetic is MMQ's:
// activations are q8_1 blocks (qprep_row_kernel, or the attention kernel), the
// integer dot of weight and activation values per 32-block is exact, so the
// tensor core computes it (tcgen05.mma kind::i8, M = 128 weight rows x N = NT
// activation rows x K = 32, each block into its own TMEM columns; Q6_K twice,
// once per 16-value half), and the epilogue forms MMQ's units -- Q8_0: one
// block, fma(dw*dx, float(I), acc); Q4_K: a pair of sub-blocks,
// acc + fma(d, sum dx*float(sc*I), -(dmin * sum sx*float(m))); Q6_K: a pair of
// blocks, fma(d, sum dx*float(sa*Ia + sb*Ib), acc) -- summed from 0 in row
// order, as each MMQ thread sums its outputs.
//
// One persistent CTA per SM walks its (128-row x NT-token) tiles in stages of
// 8 blocks (256 values) with warp-specialized roles linked by mbarriers:
//   warp 10     producer: one TMA tensor copy per weight region, one for the
//               activation tiles and one for their {d, s} records, into a ring
//               of RS stages;
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
//               forms the units, accumulates, and stores.
// (12 warps: three per scheduler leave 168 registers per thread.)
// Roles hand over groups of BG blocks (2-8), one mbarrier operation per group.
// Every mbarrier wait is bounded in time; when one runs out the CTA records an
// error flag, every role stops, and the CTA waits for its own MMAs before it
// releases TMEM and returns.
#pragma once
#include <cuda.h>

#include "kernels.cuh"

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

struct Args {
    Maps m;
    Matrix W;
    int rows;        // activation rows
    int row_tiles;   // Np / 128
    int tok_tiles;   // ceil(rows / NT)
    int tok0;        // first activation row (a multiple of 64) of this launch (TMA activations)
    GemvArgs g;      // epilogue outputs
    // split-K: `splits` CTAs share a tile's stages; split 0 keeps the running
    // row sum, the others store their units in kpart (Q8_0 / Q6_K: the two
    // factors of the unit's fused multiply-add; Q4_K: its value), and the last
    // of them (kcount) continues the sum in unit order
    int splits;
    float2 *kpart;
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

// Stage geometry per weight type and tile width.
template <int TYPE, int NT>
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
    static constexpr int oB = WA, oC = oB + WB, oE = oC + WC;
    static constexpr int oXQ = (oE + WE + 1023) / 1024 * 1024;
    static constexpr int oXR = oXQ + KB * NT * 32;                                 // float2 records [KB][NT]
    static constexpr int STAGE = (oXR + KB * NT * 8 + 1023) / 1024 * 1024;
    static constexpr uint32_t TX = WA + WB + WC + WE + KB * NT * 32 + KB * NT * 8;
    // Handoffs between roles move groups of BG blocks (one mbarrier operation
    // per group, not per block). TMEM holds TG groups of BG * COLS columns; the
    // converted tiles AG groups of BG tiles.
    static constexpr int BG = Q6 ? (NT >= 64 ? 2 : 4) : (NT >= 64 ? 4 : 8);
    static constexpr int GCOLS = BG * COLS;
    static constexpr int TG = 512 / GCOLS >= 4 ? 4 : 512 / GCOLS;
    static constexpr int AGB = BG * ABYTES;   // bytes of one converted group
    // converted groups: 3 when two stages still fit beside them, else 2
    static constexpr int AG = 220 * 1024 - 2 * STAGE >= 3 * AGB ? 3 : 2;
    // raw stages: as many as fit (2 to 4) beside the rest
    static constexpr int BUDGET = 220 * 1024 - AG * AGB;
    static constexpr int RS = BUDGET / STAGE >= 4 ? 4 : (BUDGET / STAGE >= 3 ? 3 : 2);
    static_assert(2 * STAGE <= BUDGET, "stage ring does not fit");
    static_assert(8 % BG == 0 && TG >= 2 && BG % 2 == 0, "group geometry");
    static constexpr int TCOLS_RAW = TG * GCOLS;
    static constexpr int TCOLS = TCOLS_RAW <= 32 ? 32 : (TCOLS_RAW <= 64 ? 64 : (TCOLS_RAW <= 128 ? 128 :
                                 (TCOLS_RAW <= 256 ? 256 : 512)));
    static constexpr int oEND = RS * STAGE + AG * AGB;
};

// Tokens per TMEM read batch of the Q6_K epilogue (four values per token and
// unit): 8 leaves the 168-register epilogue room to interleave token pairs
// (batch-64 LM head 253.5 -> 250.6 us, A/B on one B200; 16 for the other types).
#ifndef MGB_TC_Q6_CH
#define MGB_TC_Q6_CH 8
#endif

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

}  // namespace tc

template <int TYPE, int NT>
__host__ __device__ constexpr size_t gemm_tc_smem() {
    return 1024 + (size_t)tc::Geo<TYPE, NT>::oEND;
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

template <int TYPE, int EPI, int NT>
__global__ void __launch_bounds__(tc::kThreads, 1) gemm_tc_kernel(const __grid_constant__ tc::Args A) {
    using namespace tc;
    using G = Geo<TYPE, NT>;
    constexpr int RS = G::RS, AG = G::AG, TG = G::TG, BG = G::BG, COLS = G::COLS;
    constexpr int EW = Roles<NT>::EW, CW = Roles<NT>::CW;
    constexpr int NH = NT * 4 / EW;  // tokens per epilogue warp
    constexpr uint32_t IDESC = idesc_i8(128, G::MN);
    extern __shared__ __align__(16) uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full[RS], empty[RS], afull[AG], aempty[AG], tfull[TG], tempty[TG], fin, ebar;
    __shared__ uint32_t tmem_base_sh;
    __shared__ volatile int abort_sh;
    __shared__ float best_v[4][64];
    __shared__ uint32_t best_i[4][64];
    __shared__ int split_last;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const Matrix &W = A.W;
    const int NS = (W.nb + 7) / 8;  // stages per tile (Q8_0: the last may hold fewer blocks)
    // tiles of this CTA: (row tile, token tile, split) in turn
    const int splits = max(1, A.splits), NSS = NS / splits;  // stages per split
    const int NU = G::Q8 ? W.nb : W.nb / 2;                  // MMQ units of a row
    const int tiles = A.row_tiles * A.tok_tiles * splits;
    const int first = (int)blockIdx.x, stride = (int)gridDim.x;
    const int my_tiles = first < tiles ? (tiles - first + stride - 1) / stride : 0;
    uint8_t *base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint8_t *ring = base;                                 // RS x STAGE
    uint8_t *atile = base + (size_t)RS * G::STAGE;        // AG x BG x ABYTES

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
    auto tile_rt = [&](int k) { return (first + k * stride) % A.row_tiles; };
    auto tile_tt = [&](int k) { return ((first + k * stride) / A.row_tiles) % A.tok_tiles; };
    auto tile_s0 = [&](int k) { return (first + k * stride) / (A.row_tiles * A.tok_tiles) * NSS; };

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
                const int t0 = A.tok0 + tt * NT;
                tma3(dst + G::oXQ, &A.m.xq, 0, t0 / 8, 8 * s, bar);
                tma2(dst + G::oXR, &A.m.xr, t0, 8 * s, bar);
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
        pdl_wait();
        if (lane == 0) {
            Pos st, ag, tg;
            // Descriptors are formed once and advanced by constant 16-byte
            // steps (shared-memory offsets stay below 256 KB, so the 14-bit
            // address field never carries): the issue loop is the MMAs alone.
            const uint64_t a_base = sdesc(atile, 128, 256);
            const uint64_t x_base = sdesc(ring + G::oXQ, 128, MmaN<NT>::SBO);
            for (int k = 0; k < my_tiles && !abort_sh; ++k) {
                const int s0 = tile_s0(k);
                for (int s = s0; s < s0 + NSS && !abort_sh; ++s, st.next(RS)) {
                    if (!mbar_wait(&full[st.slot], st.phase)) {
                        fail(16u);
                        break;
                    }
                    const uint64_t xs = x_base + (uint64_t)((st.slot * G::STAGE) >> 4);
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
        pdl_wait();  // (as the MMA warp)
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
        Pos st, tg;
        uint32_t ephase = 0;
        bool ok = true;
        for (int k = 0; k < my_tiles && ok && !abort_sh; ++k) {
            const int rt = tile_rt(k), tt = tile_tt(k), s0 = tile_s0(k);
            const int row = rt * 128 + r;
            const bool live = row < W.N;
            // split-K units of this tile: [unit][NT tokens][128 rows]
            float2 *kp = splits > 1 ? A.kpart + (size_t)(tt * A.row_tiles + rt) * NU * NT * 128 : nullptr;
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
            uint8_t *qkv_c = nullptr;  // cache element of token 0 (f16 or f32: A.g.kv_f32)
            size_t qkv_tok = 0;
            if constexpr (EPI == EPI_QKV) {
                const int dm = A.g.H * A.g.hd;
                if (row < dm) {
                    qkv_q = A.g.q + row;
                    qkv_tok = dm;
                } else if (live) {
                    const int c = row - dm, which = c / dm, h = (c % dm) / A.g.hd, t = c % A.g.hd;
                    qkv_c = reinterpret_cast<uint8_t *>(which == 0 ? A.g.kc : A.g.vc) +
                            (((size_t)h * A.g.m + qkv_step) * A.g.hd + t) * (A.g.kv_f32 ? 4 : 2);
                    qkv_tok = (size_t)A.g.H * A.g.m * A.g.hd;
                }
            }
            // add one unit to the running sum (split 0) or store it (later splits):
            // Q8_0 / Q6_K units are fused multiply-adds fma(x, y, acc), Q4_K values
            // (two tokens n, n + 1 at a time, as packed f32 pairs; ARGMAX launches never split)
            auto unit2 = [&](int n, int u, float2 x, float2 y) {
                if (EPI == EPI_ARGMAX || s0 == 0) {
                    float2 a = make_float2(acc[n], acc[n + 1]);
                    a = G::Q4 ? add2(a, x) : fma2(x, y, a);
                    acc[n] = a.x;
                    acc[n + 1] = a.y;
                } else {
                    kp[((size_t)u * NT + n0 + n) * 128 + r] = make_float2(x.x, y.x);
                    kp[((size_t)u * NT + n0 + n + 1) * 128 + r] = make_float2(x.y, y.y);
                }
            };
            for (int s = s0; s < s0 + NSS && ok; ++s, st.next(RS)) {
                if (!(ok = wwait(&full[st.slot], st.phase, 64u))) break;
                const uint8_t *stg = ring + (size_t)st.slot * G::STAGE;
                // the stage's activation records: {d, s} per [block][token]
                const float2 *rec = reinterpret_cast<const float2 *>(stg + G::oXR);
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
                const int nbs = min(8, W.nb - 8 * s);
                for (int g = 0; g * BG < nbs && ok; ++g, tg.next(TG)) {
                    if (!(ok = wwait(&tfull[tg.slot], tg.phase, 64u))) break;
                    fence_after();
                    const int gb = group_blocks(g, nbs);
                    // units of the group: Q8_0 one block each, Q4_K / Q6_K pairs of blocks
                    constexpr int UB = G::Q8 ? 1 : 2;
                    for (int bb = 0; bb < gb; bb += UB) {
                        const int b = g * BG + bb;
                        const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + tg.slot * G::GCOLS + bb * COLS + n0;
                        int sa0 = 0, sb0 = 0, sa1 = 0, sb1 = 0;
                        float mf0 = 0.f, mf1 = 0.f, db = 0.f;
                        if constexpr (G::Q4) {
                            sa0 = (int)(((b < 4 ? scpk0 : scpk1) >> (8 * (b & 3))) & 0xff);
                            sa1 = (int)(((b + 1 < 4 ? scpk0 : scpk1) >> (8 * ((b + 1) & 3))) & 0xff);
                            mf0 = (float)(((b < 4 ? mpk0 : mpk1) >> (8 * (b & 3))) & 0xff);
                            mf1 = (float)(((b + 1 < 4 ? mpk0 : mpk1) >> (8 * ((b + 1) & 3))) & 0xff);
                        } else if constexpr (G::Q6) {
                            const unsigned short c0 =
                                *reinterpret_cast<const unsigned short *>(stg + G::oC + (gi * 8 + b) * 64 + l * 2);
                            const unsigned short c1 =
                                *reinterpret_cast<const unsigned short *>(stg + G::oC + (gi * 8 + b + 1) * 64 + l * 2);
                            sa0 = (int8_t)(c0 & 0xff);
                            sb0 = (int8_t)(c0 >> 8);
                            sa1 = (int8_t)(c1 & 0xff);
                            sb1 = (int8_t)(c1 >> 8);
                        } else {
                            db = h2f(*reinterpret_cast<const unsigned short *>(stg + G::oB + (gi * 8 + b) * 64 + l * 2));
                        }
                        const int u = G::Q8 ? 8 * s + b : 4 * s + b / 2;  // unit index in the row
                        // TMEM -> registers in chunks of up to 16 tokens: the unit's
                        // blocks (and Q6_K halves) loaded together, then one wait
                        constexpr int CHM = G::Q6 ? MGB_TC_Q6_CH : 16;
                        constexpr int CH = NH < CHM ? NH : CHM, NC = NH / CH;
#pragma unroll
                        for (int c = 0; c < NC; ++c) {
                            int va0[CH], vb0[CH], va1[CH], vb1[CH];
                            auto ld = [&](uint32_t t, int (&v)[CH]) {
                                if constexpr (CH == 16) tmem_ld16(t, v);
                                else if constexpr (CH == 8) tmem_ld8(t, v);
                                else {
                                    static_assert(CH == 4, "token chunk");
                                    tmem_ld4(t, v);
                                }
                            };
                            ld(ta + c * CH, va0);
                            if constexpr (G::Q6) ld(ta + G::MN + c * CH, vb0);
                            if constexpr (!G::Q8) ld(ta + COLS + c * CH, va1);
                            if constexpr (G::Q6) ld(ta + COLS + G::MN + c * CH, vb1);
                            tmem_wait_ld();
                            const float2 z2 = make_float2(0.0f, 0.0f);
#pragma unroll
                            for (int i = 0; i < CH; i += 2) {
                                const int n = c * CH + i;
                                // both tokens' {d, s} records of a block in one 16-byte load
                                const float4 x0 = *reinterpret_cast<const float4 *>(rec + b * NT + n0 + n);
                                if constexpr (G::Q8) {
                                    unit2(n, u, mul2(make_float2(db, db), make_float2(x0.x, x0.z)),
                                          make_float2((float)va0[i], (float)va0[i + 1]));
                                } else {
                                    const float4 x1 = *reinterpret_cast<const float4 *>(rec + (b + 1) * NT + n0 + n);
                                    if constexpr (G::Q4) {
                                        const float2 sd =
                                            fma2(make_float2(x1.x, x1.z),
                                                 make_float2((float)(sa1 * va1[i]), (float)(sa1 * va1[i + 1])),
                                                 fma2(make_float2(x0.x, x0.z),
                                                      make_float2((float)(sa0 * va0[i]), (float)(sa0 * va0[i + 1])), z2));
                                        const float2 sm = fma2(make_float2(x1.y, x1.w), make_float2(mf1, mf1),
                                                               fma2(make_float2(x0.y, x0.w), make_float2(mf0, mf0), z2));
                                        const float2 t = mul2(make_float2(dm, dm), sm);  // fma(d, sd, -(dmin * sm))
                                        unit2(n, u, fma2(make_float2(d, d), sd, make_float2(-t.x, -t.y)), z2);
                                    } else {
                                        const float2 sf = fma2(
                                            make_float2(x1.x, x1.z),
                                            make_float2((float)(sa1 * va1[i] + sb1 * vb1[i]),
                                                        (float)(sa1 * va1[i + 1] + sb1 * vb1[i + 1])),
                                            fma2(make_float2(x0.x, x0.z),
                                                 make_float2((float)(sa0 * va0[i] + sb0 * vb0[i]),
                                                             (float)(sa0 * va0[i + 1] + sb0 * vb0[i + 1])),
                                                 z2));
                                        unit2(n, u, make_float2(d, d), sf);
                                    }
                                }
                            }
                        }
                    }
                    fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[tg.slot]);
                }
                if (!ok) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[st.slot]);
            }
            if (!ok || abort_sh) break;
            if (splits > 1) {
                // split 0 leaves its running sum in unit slot 0 (a unit it summed itself)
                if (s0 == 0)
#pragma unroll
                    for (int n = 0; n < NH; ++n) kp[(size_t)(n0 + n) * 128 + r] = make_float2(acc[n], 0.0f);
                __syncwarp();
                if (lane == 0) mbar_arrive(&ebar);
                if (!(ok = wwait(&ebar, ephase, 128u))) break;
                ephase ^= 1;
                if (tid == 0) {
                    __threadfence();
                    const uint32_t old = atomicAdd(&A.kcount[tt * A.row_tiles + rt], 1u);
                    split_last = old + 1 == (uint32_t)splits;
                    if (split_last) {
                        A.kcount[tt * A.row_tiles + rt] = 0;  // every split of this launch has counted
                        __threadfence();
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&ebar);
                if (!(ok = wwait(&ebar, ephase, 128u))) break;
                ephase ^= 1;
                if (!split_last) continue;  // another split finishes this tile
                // the row sum continued in unit order from the stored units,
                // UL units x NH tokens of loads in flight per batch
                const int u1 = G::Q8 ? 8 * NSS : 4 * NSS;  // first unit of split 1
                constexpr int UL = NH <= 8 ? 8 : (NH <= 16 ? 4 : 2);
#pragma unroll
                for (int n = 0; n < NH; ++n) acc[n] = __ldcg(&kp[(size_t)(n0 + n) * 128 + r].x);
                for (int u0 = u1; u0 < NU; u0 += UL) {
                    float2 v[UL][NH];
#pragma unroll
                    for (int j = 0; j < UL; ++j)
#pragma unroll
                        for (int n = 0; n < NH; ++n)
                            v[j][n] = u0 + j < NU ? __ldcg(kp + ((size_t)(u0 + j) * NT + n0 + n) * 128 + r)
                                                  : make_float2(0.0f, 0.0f);
#pragma unroll
                    for (int j = 0; j < UL; ++j) {
                        if (u0 + j >= NU) break;
#pragma unroll
                        for (int n = 0; n < NH; ++n)
                            acc[n] = G::Q4 ? __fadd_rn(acc[n], v[j][n].x) : __fmaf_rn(v[j][n].x, v[j][n].y, acc[n]);
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
            } else if (EPI == EPI_RELU && A.g.qo.tq) {
                // the warp's 32 rows are one q8_1 block of the next matmul's
                // activation row (every row live: the host requires N % 128 == 0)
#pragma unroll
                for (int n = 0; n < NH; ++n) {
                    const int tok = tt * NT + n0 + n;
                    if (tok >= A.rows) break;  // uniform across the warp
                    const float y = __fadd_rn(acc[n], bias);
                    store_block_tc(A.g.qo, tok, row >> 5, y > 0.0f ? y : 0.0f, lane);
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
                        else if (A.g.kv_f32) reinterpret_cast<float *>(qkv_c)[tok * qkv_tok] = y;
                        else reinterpret_cast<__half *>(qkv_c)[tok * qkv_tok] = __float2half_rn(y);
                    } else {
                        epilogue_store<EPI>(A.g, row, tok, acc[n]);
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

// Tensor-core layout of one activation row (one CTA per row): the row is
// staged in shared memory (embedding rows dequantized once), LayerNorm
// statistics by one warp in the engine's fixed order, then every 32-value
// block is quantized to q8_1 (store_block_tc) as
//   tq  : per block j, 8-row core groups of 256 bytes [j][row/8][k16][row%8][16 B]
//         (the UMMA K-major no-swizzle layout);
//   trec: per block j and row, float2 {d, s}.
template <int MODE>
__global__ void __launch_bounds__(1024) qprep_row_kernel(PrepArgs p, QAct out) {
    extern __shared__ __align__(16) float qsm[];
    __shared__ float st[2];
    const int r = blockIdx.x, K = p.K, T = K >> 5;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float *xs = qsm, *gb = qsm + K;  // row [K]; gamma [K], beta [K]
    // LayerNorm parameters into shared memory before the dependency wait (they
    // are weights, not the predecessor's output)
    if constexpr (MODE != PREP_PLAIN) {
        for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
            reinterpret_cast<float4 *>(gb)[i] = __ldg(reinterpret_cast<const float4 *>(p.gamma) + i);
            reinterpret_cast<float4 *>(gb + K)[i] = __ldg(reinterpret_cast<const float4 *>(p.beta) + i);
        }
    }
    pdl_wait();
    const float *pos = nullptr;
    uint32_t id = 0;
    if constexpr (MODE == PREP_EMBED_LN) {
        pos = p.pos_table + (size_t)(*p.step + p.pos_base) * K;
        id = p.ids[r];
    }
    // 8 loads in flight per thread before their stores (one memory round trip)
    for (int base = threadIdx.x; base < K; base += 8 * blockDim.x) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = base + u * blockDim.x;
            if (i < K) {
                if constexpr (MODE == PREP_EMBED_LN)
                    v[u] = __fadd_rn(__fmul_rn(deq_elem(p.embed, (int)id, i), p.scale), pos[i]);
                else
                    v[u] = p.x[(size_t)r * K + i];
            }
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
    if constexpr (MODE != PREP_PLAIN) {
        if (warp == 0) {
            float sum = 0.0f;
#pragma unroll 8
            for (int t = 0; t < T; ++t) sum = t == 0 ? xs[lane] : __fadd_rn(sum, xs[32 * t + lane]);
            const float mean = __fdiv_rn(warp_tree(sum), (float)K);
            float s2 = 0.0f;
#pragma unroll 8
            for (int t = 0; t < T; ++t) {
                const float c = __fsub_rn(xs[32 * t + lane], mean);
                const float c2 = __fmul_rn(c, c);
                s2 = t == 0 ? c2 : __fadd_rn(s2, c2);
            }
            const float var = __fdiv_rn(warp_tree(s2), (float)K);
            if (lane == 0) {
                st[0] = mean;
                st[1] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
            }
        }
        __syncthreads();
    }
    // the next matmul is released once the activations are about to be written
    pdl_launch_dependents();
    for (int j = warp; j < T; j += blockDim.x >> 5) {
        const int i = 32 * j + lane;
        float v = xs[i];
        if constexpr (MODE != PREP_PLAIN) v = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v, st[0]), st[1]), gb[i]), gb[K + i]);
        store_block_tc(out, r, j, v, lane);
    }
}

}  // namespace mgb
