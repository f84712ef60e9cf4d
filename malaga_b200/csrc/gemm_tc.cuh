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
//   warp 12     producer: one TMA tensor copy per weight region, one for the
//               activation tiles (already in the UMMA K-major layout), one for
//               the activation scale records, into a ring of RS stages;
//   warps 0-3   converters: thread t unpacks weight row t of each block (Q4_K
//               nibbles, Q6_K 6-bit values minus 32, Q8_0 bytes) into an int8
//               128x32 tile in the canonical no-swizzle layout (ring of AS);
//   warp 13     MMA: one tcgen05.mma per block into a ring of TS TMEM slots,
//               committed to the barriers that free the tile, the slot's
//               readers and the stage;
//   warps 4-11  epilogue: warp w reads TMEM lanes 32(w%4).. (its weight rows)
//               for half of the tile's tokens, accumulates, and stores.
// Q6_K needs the two 16-value halves of a block separately (their scales
// differ): its activation tiles hold every token twice, once with each half
// zeroed, so one MMA with N = 2 NT yields both sums.
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

// TMA tensor copy (tile mode, no multicast) of box `coords` into shared memory.
__device__ __forceinline__ void tma3(void *dst, const CUtensorMap *m, int c0, int c1, int c2, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(m), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma4(void *dst, const CUtensorMap *m, int c0, int c1, int c2, int c3, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(smem_u32(dst)),
        "l"(m), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma2(void *dst, const CUtensorMap *m, int c0, int c1, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(m), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

// Byte offset of (row r, 16-byte K chunk k16) of a K=32 int8 operand tile.
__host__ __device__ __forceinline__ int tile_off(int r, int k16) { return (r >> 3) * 256 + k16 * 128 + (r & 7) * 16; }

// Tensor maps of one launch: weight regions a, b, c, e (3-D: 8-byte words of
// one (32-row group, block) slice, blocks or super-blocks, groups), activation
// tiles (4-D: 8-byte words of an 8-row core group, row groups, halves, blocks)
// and activation scale records (2-D: 8-byte words of a unit's rows, units).
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
    int tok0;        // first activation row (a multiple of 64) of this launch
    GemvArgs g;      // epilogue outputs
    uint32_t *err;
};

// Stage geometry per weight type and tile width.
template <int TYPE, int NT>
struct Geo {
    static constexpr bool Q6 = TYPE == T_Q6_K, Q4 = TYPE == T_Q4_K, Q8 = TYPE == T_Q8_0;
    static constexpr int H = Q6 ? 2 : 1;   // activation copies per block
    static constexpr int COLS = H * NT;    // TMEM columns per block
    static constexpr int KB = 8;           // blocks per stage
    static constexpr int WA = Q8 ? 4 * KB * 1024 : 4 * KB * 512;                   // q / qs / ql
    static constexpr int WB = Q8 ? 4 * KB * 64 : (Q4 ? 4 * 512 : 4 * KB * 256);    // d / header / qh
    static constexpr int WC = Q6 ? 4 * KB * 64 : 0;                                // Q6_K scales
    static constexpr int WE = Q6 ? 4 * 64 : 0;                                     // Q6_K d
    static constexpr int RB = Q4 ? 32 : 4;                                         // record bytes
    static constexpr int UPS = Q8 ? KB : 1;                                        // units per stage
    static constexpr int oB = WA, oC = oB + WB, oE = oC + WC;
    static constexpr int oXQ = (oE + WE + 1023) / 1024 * 1024;
    static constexpr int oXR = oXQ + KB * H * NT * 32;
    static constexpr int STAGE = (oXR + UPS * NT * RB + 1023) / 1024 * 1024;
    static constexpr uint32_t TX = WA + WB + WC + WE + KB * H * NT * 32 + UPS * NT * RB;
    static constexpr int AS = 8;                                                   // A tile slots
    static constexpr int RS = (220 * 1024 - AS * 4096) / STAGE >= 4 ? 4 : 3;       // raw stages
    static constexpr int TS = 512 / COLS < 16 ? 512 / COLS : 16;                   // TMEM slots
    static constexpr int TCOLS_RAW = TS * COLS;
    static constexpr int TCOLS = TCOLS_RAW <= 32 ? 32 : (TCOLS_RAW <= 64 ? 64 : (TCOLS_RAW <= 128 ? 128 :
                                 (TCOLS_RAW <= 256 ? 256 : 512)));
    static constexpr int SMEM = 1024 + RS * STAGE + AS * 4096;
    static_assert(SMEM <= 227 * 1024, "stage ring too large");
};

constexpr int kThreads = 448;  // 14 warps
constexpr int kProducerWarp = 12, kMmaWarp = 13;

}  // namespace tc

template <int TYPE, int NT>
__host__ __device__ constexpr size_t gemm_tc_smem() {
    return (size_t)tc::Geo<TYPE, NT>::SMEM;
}

template <int TYPE, int EPI, int NT>
__global__ void __launch_bounds__(tc::kThreads, 1) gemm_tc_kernel(const __grid_constant__ tc::Args A) {
    using namespace tc;
    using G = Geo<TYPE, NT>;
    constexpr int RS = G::RS, AS = G::AS, TS = G::TS, COLS = G::COLS, H = G::H;
    constexpr int NH = NT / 2;  // tokens per epilogue warp
    constexpr uint32_t IDESC = idesc_i8(128, H * NT);
    extern __shared__ __align__(16) uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full[RS], empty[RS], afull[AS], aempty[AS], tfull[TS], tempty[TS], fin;
    __shared__ uint32_t tmem_base_sh;
    __shared__ volatile int abort_sh;
    __shared__ float best_v[4][64];
    __shared__ uint32_t best_i[4][64];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const Matrix &W = A.W;
    const int NS = (W.nb + 7) / 8;  // stages per tile (Q8_0: the last may hold fewer blocks)
    const int tiles = A.row_tiles * A.tok_tiles;
    uint8_t *base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint8_t *ring = base;                            // RS x STAGE
    uint8_t *atile = base + (size_t)RS * G::STAGE;   // AS x 4 KB

    if (tid == 0) {
        for (int i = 0; i < RS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 4 + 1 + 8);
        }
        for (int i = 0; i < AS; ++i) {
            mbar_init(&afull[i], 4);
            mbar_init(&aempty[i], 1);
        }
        for (int i = 0; i < TS; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], 8);
        }
        mbar_init(&fin, 1);
        abort_sh = 0;
    }
    if (EPI == EPI_ARGMAX)
        for (int n = tid; n < 256; n += blockDim.x) {
            best_v[n >> 6][n & 63] = kNegInf;
            best_i[n >> 6][n & 63] = 0xffffffffu;
        }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                     "r"(G::TCOLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
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

    if (warp == kProducerWarp) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const int first_stages = blockIdx.x < tiles ? min(RS, NS) : 0;
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
                tma4(dst + G::oXQ, &A.m.xq, 0, t0 / 8, 0, 8 * s, bar);
                if constexpr (G::Q4) tma2(dst + G::oXR, &A.m.xr, t0 * 4, s, bar);
                else if constexpr (G::Q6) tma2(dst + G::oXR, &A.m.xr, t0 / 2, s, bar);
                else tma2(dst + G::oXR, &A.m.xr, t0 / 2, 8 * s, bar);
            };
            // weights of the first stages do not depend on the previous kernel
            for (int s = 0; s < first_stages; ++s) {
                mbar_expect_tx(&full[s], G::TX);
                weights(blockIdx.x % A.row_tiles, s, ring + (size_t)s * G::STAGE, &full[s]);
            }
            pdl_wait();
            uint32_t gs = 0;
            for (int tile = blockIdx.x; tile < tiles && !abort_sh; tile += gridDim.x) {
                const int rt = tile % A.row_tiles, tt = tile / A.row_tiles;
                for (int s = 0; s < NS; ++s, ++gs) {
                    const int slot = gs % RS;
                    const uint32_t use = gs / RS;
                    uint8_t *dst = ring + (size_t)slot * G::STAGE;
                    if (gs >= (uint32_t)first_stages) {
                        if (use > 0 && !mbar_wait(&empty[slot], (use - 1) & 1)) {
                            fail(8u);
                            break;
                        }
                        if (abort_sh) break;
                        mbar_expect_tx(&full[slot], G::TX);
                        weights(rt, s, dst, &full[slot]);
                    }
                    acts(tt, s, dst, &full[slot]);
                }
            }
        }
    } else if (warp == kMmaWarp) {
        // ----------------------------------------------------------------- MMA
        if (lane == 0) {
            uint32_t gs = 0, gb = 0;
            for (int tile = blockIdx.x; tile < tiles && !abort_sh; tile += gridDim.x) {
                for (int s = 0; s < NS && !abort_sh; ++s, ++gs) {
                    const int slot = gs % RS;
                    if (!mbar_wait(&full[slot], (gs / RS) & 1)) {
                        fail(16u);
                        break;
                    }
                    const uint8_t *xq = ring + (size_t)slot * G::STAGE + G::oXQ;
                    const int nbs = min(8, W.nb - 8 * s);
                    for (int b = 0; b < nbs; ++b, ++gb) {
                        const int as = gb % AS, ts = gb % TS;
                        const uint32_t au = gb / AS, tu = gb / TS;
                        if (!mbar_wait(&afull[as], au & 1) || (tu > 0 && !mbar_wait(&tempty[ts], (tu - 1) & 1))) {
                            fail(16u);
                            break;
                        }
                        if (abort_sh) break;
                        fence_after();
                        mma_i8(tmem + ts * COLS, sdesc(atile + as * 4096, 128, 256),
                               sdesc(xq + b * H * NT * 32, 128, 256), IDESC);
                        commit(&aempty[as]);
                        commit(&tfull[ts]);
                    }
                    commit(&empty[slot]);
                }
            }
            // every MMA issued by this thread has completed before TMEM is released
            commit(&fin);
            if (!mbar_wait(&fin, 0)) fail(16u);
        }
    } else if (warp < 4) {
        // ---------------------------------------------------------- converters
        const int r = tid;  // weight row of the tile = TMEM lane
        uint32_t gs = 0, gb = 0;
        for (int tile = blockIdx.x; tile < tiles && !abort_sh; tile += gridDim.x) {
            bool ok = true;
            for (int s = 0; s < NS && ok; ++s, ++gs) {
                const int slot = gs % RS;
                if (!(ok = wwait(&full[slot], (gs / RS) & 1, 32u))) break;
                const uint8_t *st = ring + (size_t)slot * G::STAGE;
                const int nbs = min(8, W.nb - 8 * s);
                for (int b = 0; b < nbs; ++b, ++gb) {
                    const int as = gb % AS;
                    const uint32_t au = gb / AS;
                    if (au > 0 && !(ok = wwait(&aempty[as], (au - 1) & 1, 32u))) break;
                    uint8_t *ta = atile + as * 4096;
                    const int gi = r >> 5, l = r & 31;
                    int4 lo, hi;
                    if constexpr (G::Q8) {
                        const int4 *src = reinterpret_cast<const int4 *>(st + (gi * 8 + b) * 1024 + l * 32);
                        lo = src[0];
                        hi = src[1];
                    } else if constexpr (G::Q4) {
                        const int4 v = *reinterpret_cast<const int4 *>(st + (gi * 8 + b) * 512 + l * 16);
                        lo = make_int4(v.x & 0x0f0f0f0f, v.y & 0x0f0f0f0f, v.z & 0x0f0f0f0f, v.w & 0x0f0f0f0f);
                        hi = make_int4((v.x >> 4) & 0x0f0f0f0f, (v.y >> 4) & 0x0f0f0f0f, (v.z >> 4) & 0x0f0f0f0f,
                                       (v.w >> 4) & 0x0f0f0f0f);
                    } else {
                        const int4 lq = *reinterpret_cast<const int4 *>(st + (gi * 8 + b) * 512 + l * 16);
                        const uint2 hq = *reinterpret_cast<const uint2 *>(st + G::oB + (gi * 8 + b) * 256 + l * 8);
                        const int ql[4] = {lq.x, lq.y, lq.z, lq.w};
                        int a4[4], b4[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            a4[i] = (int)__vsub4((uint32_t)((ql[i] & 0x0f0f0f0f) | (int)(((hq.x >> (2 * i)) & 0x03030303u) << 4)),
                                                 0x20202020u);
                            b4[i] = (int)__vsub4(
                                (uint32_t)(((ql[i] >> 4) & 0x0f0f0f0f) | (int)(((hq.y >> (2 * i)) & 0x03030303u) << 4)),
                                0x20202020u);
                        }
                        lo = make_int4(a4[0], a4[1], a4[2], a4[3]);
                        hi = make_int4(b4[0], b4[1], b4[2], b4[3]);
                    }
                    *reinterpret_cast<int4 *>(ta + tile_off(r, 0)) = lo;
                    *reinterpret_cast<int4 *>(ta + tile_off(r, 1)) = hi;
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&afull[as]);
                }
                if (!ok) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
            }
            if (!ok) break;
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3, e = (warp - 4) >> 2;
        const int r = 32 * q + lane, gi = q, l = lane;
        const int n0 = e * NH;  // first token (within the tile) of this warp
        pdl_wait();
        uint32_t gs = 0, gb = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok && !abort_sh; tile += gridDim.x) {
            const int rt = tile % A.row_tiles, tt = tile / A.row_tiles;
            const int row = rt * 128 + r;
            const bool live = row < W.N;
            float acc[NH];
#pragma unroll
            for (int n = 0; n < NH; ++n) acc[n] = 0.0f;
            for (int s = 0; s < NS && ok; ++s, ++gs) {
                const int slot = gs % RS;
                if (!(ok = wwait(&full[slot], (gs / RS) & 1, 64u))) break;
                const uint8_t *st = ring + (size_t)slot * G::STAGE;
                // this row's scales for the stage
                float d = 0.f, dm = 0.f;
                uint32_t mpk0 = 0, mpk1 = 0, scpk0 = 0, scpk1 = 0;
                if constexpr (G::Q4) {
                    const uint4 h = *reinterpret_cast<const uint4 *>(st + G::oB + gi * 512 + l * 16);
                    d = h2f(h.x & 0xffff);
                    dm = h2f(h.x >> 16);
                    auto byte = [&](int k) -> uint32_t {
                        const uint32_t w = k < 4 ? h.y : (k < 8 ? h.z : h.w);
                        return (w >> (8 * (k & 3))) & 0xff;
                    };
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        uint32_t sc, mm;
                        if (k < 4) {
                            sc = byte(k) & 63;
                            mm = byte(k + 4) & 63;
                        } else {
                            sc = (byte(k + 4) & 0xf) | ((byte(k - 4) >> 6) << 4);
                            mm = (byte(k + 4) >> 4) | ((byte(k) >> 6) << 4);
                        }
                        if (k < 4) {
                            scpk0 |= sc << (8 * k);
                            mpk0 |= mm << (8 * k);
                        } else {
                            scpk1 |= sc << (8 * (k - 4));
                            mpk1 |= mm << (8 * (k - 4));
                        }
                    }
                } else if constexpr (G::Q6) {
                    d = h2f(*reinterpret_cast<const unsigned short *>(st + G::oE + gi * 64 + l * 2));
                }
                int S[NH];
#pragma unroll
                for (int n = 0; n < NH; ++n) S[n] = 0;
                const int nbs = min(8, W.nb - 8 * s);
                for (int b = 0; b < nbs; ++b, ++gb) {
                    const int ts = gb % TS;
                    if (!(ok = wwait(&tfull[ts], (gb / TS) & 1, 64u))) break;
                    fence_after();
                    const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + ts * COLS + n0;
                    int sa = 0, sb = 0;
                    float db = 0.f;
                    if constexpr (G::Q4) {
                        sa = (int)(((b < 4 ? scpk0 : scpk1) >> (8 * (b & 3))) & 0xff);
                    } else if constexpr (G::Q6) {
                        const unsigned short sc2 =
                            *reinterpret_cast<const unsigned short *>(st + G::oC + (gi * 8 + b) * 64 + l * 2);
                        sa = (int8_t)(sc2 & 0xff);
                        sb = (int8_t)(sc2 >> 8);
                    } else {
                        db = h2f(*reinterpret_cast<const unsigned short *>(st + G::oB + (gi * 8 + b) * 64 + l * 2));
                    }
                    constexpr int CH = NH < 16 ? NH : 16;
#pragma unroll
                    for (int c0 = 0; c0 < NH; c0 += CH) {
                        int va[16], vb[16];
                        if constexpr (CH == 16) {
                            tmem_ld16(ta + c0, va);
                            if constexpr (G::Q6) tmem_ld16(ta + NT + c0, vb);
                        } else if constexpr (CH == 8) {
                            int t8[8], u8[8];
                            tmem_ld8(ta + c0, t8);
                            if constexpr (G::Q6) tmem_ld8(ta + NT + c0, u8);
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                va[i] = t8[i];
                                vb[i] = G::Q6 ? u8[i] : 0;
                            }
                        } else {
                            static_assert(CH == 4, "token chunk");
                            int t4[4], u4[4];
                            tmem_ld4(ta + c0, t4);
                            if constexpr (G::Q6) tmem_ld4(ta + NT + c0, u4);
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                va[i] = t4[i];
                                vb[i] = G::Q6 ? u4[i] : 0;
                            }
                        }
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < CH; ++i) {
                            const int n = c0 + i;
                            if constexpr (G::Q4) {
                                S[n] += sa * va[i];
                            } else if constexpr (G::Q6) {
                                S[n] += sa * va[i] + sb * vb[i];
                            } else {
                                const float xd = reinterpret_cast<const float *>(st + G::oXR)[b * NT + n0 + n];
                                const float p = __fmul_rn(__fmul_rn(db, xd), (float)va[i]);
                                acc[n] = (s == 0 && b == 0) ? p : __fadd_rn(acc[n], p);
                            }
                        }
                    }
                    fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[ts]);
                }
                if (!ok) break;
                if constexpr (!G::Q8) {
                    // finish the super-block: float scales once, then the row sum
#pragma unroll
                    for (int n = 0; n < NH; ++n) {
                        float p;
                        if constexpr (G::Q4) {
                            const int4 rec = *reinterpret_cast<const int4 *>(st + G::oXR + (n0 + n) * 32);
                            const float xd = __int_as_float(rec.x);
                            // S2 = sum_j m_j * s32_j (s32 pairs as int16x2, m_j as bytes)
                            int S2 = __dp2a_lo(rec.y, (int)mpk0, 0);
                            S2 = __dp2a_hi(rec.z, (int)mpk0, S2);
                            S2 = __dp2a_lo(rec.w, (int)mpk1, S2);
                            S2 = __dp2a_hi(*reinterpret_cast<const int *>(st + G::oXR + (n0 + n) * 32 + 16), (int)mpk1,
                                           S2);
                            p = __fmul_rn(xd, __fsub_rn(__fmul_rn(d, (float)S[n]), __fmul_rn(dm, (float)S2)));
                        } else {
                            const float xd = reinterpret_cast<const float *>(st + G::oXR)[n0 + n];
                            p = __fmul_rn(__fmul_rn(d, xd), (float)S[n]);
                        }
                        acc[n] = s == 0 ? p : __fadd_rn(acc[n], p);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
            }
            if (!ok || abort_sh) break;
            // tile epilogue
#pragma unroll
            for (int n = 0; n < NH; ++n) {
                const int tok = tt * NT + n0 + n;
                if (tok >= A.rows) break;  // uniform across the warp
                if constexpr (EPI == EPI_ARGMAX) {
                    float bv = live ? acc[n] : kNegInf;
                    uint32_t bi = live ? (uint32_t)row : 0xffffffffu;
                    if (A.g.logits && live) A.g.logits[(size_t)tok * W.N + row] = acc[n];
                    warp_argmax(bv, bi);
                    if (lane == 0) argmax_merge(best_v[q][tok], best_i[q][tok], bv, bi);  // tok < 64
                } else if (live) {
                    epilogue_store<EPI>(A.g, row, tok, acc[n]);
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
//   tq : per block j and copy h, 8-row core groups of 256 bytes
//        [j][h][row/8][k16][row%8][16 B] (the UMMA K-major no-swizzle layout;
//        for Q6_K consumers copy 0 keeps values 0-15 and copy 1 values 16-31,
//        the other half zeroed);
//   trec: per unit u (super-block, or block for Q8_0 consumers) and row:
//        Q4_K: {f32 scale, int16 block sums x 8, 12 zero bytes} (32 B);
//        Q6_K: f32 scale; Q8_0: f32 (f16-rounded) scale.
template <int MODE>
__global__ void __launch_bounds__(256) qprep_row_kernel(PrepArgs p, QAct out) {
    extern __shared__ __align__(16) uint8_t qsm[];
    __shared__ float st[2];
    __shared__ uint32_t id_sh[1];
    pdl_launch_dependents();
    pdl_wait();
    const int r = blockIdx.x, K = p.K, nb = K >> 5;
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
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        const float v = act_input<MODE>(pa, MODE == PREP_EMBED_LN ? 0 : r, i);
        xs[i] = v;
        if constexpr (MODE == PREP_EMBED_LN) p.x_out[(size_t)r * K + i] = v;
    }
    __syncthreads();
    PrepArgs q = p;
    q.x = xs;
    q.rows = 1;
    constexpr int M2 = MODE == PREP_PLAIN ? PREP_PLAIN : PREP_LN;
    if (p.group == 8) build_activations_impl<M2, 8>(q, s, 1, false);
    else build_activations_impl<M2, 1>(q, s, 1, false);
    // build_activations_impl ends with __syncthreads
    const int H = p.ctype == T_Q6_K ? 2 : 1, rs = out.rs;
    for (int c = threadIdx.x; c < nb * H * 2; c += blockDim.x) {
        const int j = c / (2 * H), h = (c >> 1) % H, k16 = c & 1;
        int4 v = *reinterpret_cast<const int4 *>(s.q + 32 * j + 16 * k16);
        if (H == 2 && h != k16) v = make_int4(0, 0, 0, 0);
        *reinterpret_cast<int4 *>(out.tq + (((size_t)j * H + h) * (rs / 8) + (r >> 3)) * 256 + tc::tile_off(r & 7, k16)) = v;
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
