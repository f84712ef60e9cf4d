// Batched quantized matmul on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Replaces candle's MMQ path (QMatMul::forward for more than 8 activation rows,
// model.rs:571-607, and the encoder's projections model.rs:137-154 / 463-477).
// The arithmetic is the engine's (numerics.cuh): per 32-block j the integer
// dot I_j = sum q_w * q_x is exact, so the tensor core computes it
// (tcgen05.mma kind::i8, M = 128 weight rows x N = NT activation rows x K = 32),
// each block into its own TMEM columns; the epilogue applies the block's float
// scales exactly as the small-batch kernels do and sums the partials left to
// right in block order, so results are bit-identical to them.
//
// A CTA (4 warps; thread t owns weight row t of its 128-row tile, which is also
// TMEM lane t) walks the K blocks in chunks of CB blocks:
//   * thread 0 bulk-copies (cp.async.bulk, 1-D TMA) the raw weight bytes of
//     chunk c+2 into a 3-deep ring while chunk c is being processed;
//   * all threads unpack chunk c (Q4_K nibbles, Q6_K 6-bit values, Q8_0 bytes)
//     into int8 tiles in the canonical K-major no-swizzle UMMA layout (8-row x
//     16-byte core matrices, SBO 256 B between row groups, LBO 128 B between the
//     two 16-byte K chunks), copy the activation blocks the same way, and keep
//     the block's scales in shared memory;
//   * thread 0 issues the CB MMAs of chunk c into one half of the TMEM columns
//     and commits them to an mbarrier;
//   * meanwhile the epilogue reads chunk c-1 from the other half (tcgen05.ld).
// Tiles, buffers and TMEM halves are double-buffered; every mbarrier wait is
// bounded by time and, when it runs out, the CTA records an error flag, stops,
// releases TMEM and returns.
#pragma once
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

template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[N]);

template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t t, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(t));
}
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t t, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(t));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Byte offset of (row r, 16-byte K chunk k16) of a K=32 int8 operand tile.
__device__ __forceinline__ int tile_off(int r, int k16) { return (r >> 3) * 256 + k16 * 128 + (r & 7) * 16; }

struct Args {
    Matrix W;
    QAct x;          // activations [rows][K], q8_1
    int rows;        // activation rows
    int row_tiles;   // Np / 128 (rounded up)
    int tok_tiles;   // ceil(rows / NT)
    GemvArgs g;      // epilogue outputs
    uint32_t *err;
};

// Chunk geometry per weight type and tile width.
template <int TYPE, int NT>
struct Geo {
    static constexpr bool Q6 = TYPE == T_Q6_K;
    static constexpr int COLS = Q6 ? 2 * NT : NT;                    // TMEM columns per block
    static constexpr int A_BYTES = Q6 ? 8192 : 4096;                 // int8 tile(s) of one block
    // blocks per chunk: 2 TMEM halves <= 256 columns, 2 tile buffers <= 64 KB,
    // and a divisor of 8 (a chunk never straddles a 256-value super-block)
    static constexpr int CB1 = 128 / COLS < 32768 / A_BYTES ? 128 / COLS : 32768 / A_BYTES;
    static constexpr int CB = CB1 >= 8 ? 8 : (CB1 >= 4 ? 4 : (CB1 >= 2 ? 2 : 1));
    static constexpr int B_BYTES = NT * 32 < 256 ? 256 : NT * 32;    // one 8-row core group minimum
    // raw bytes of one block for 32 rows, per region
    static constexpr int RA = TYPE == T_Q8_0 ? 1024 : 512;           // q / qs / ql
    static constexpr int RB = TYPE == T_Q8_0 ? 64 : (TYPE == T_Q6_K ? 256 : 0);  // d / qh
    static constexpr int RC = Q6 ? 64 : 0;                           // Q6_K scales
    static constexpr int WRAW = 4 * CB * (RA + RB + RC) + (TYPE == T_Q8_0 ? 0 : 4 * (Q6 ? 64 : 512));
    // activation bytes of a chunk: NT rows x CB blocks x 32 B, then block-major scales
    static constexpr int XQ = WRAW, XD = XQ + NT * CB * 32, XS = XD + CB * NT * 4;
    static constexpr int RAW = XS + CB * NT * 4;
};

}  // namespace tc

// Dynamic shared memory of gemm_tc_kernel<TYPE, *, NT>.
template <int TYPE, int NT>
__host__ __device__ constexpr size_t gemm_tc_smem() {
    using G = tc::Geo<TYPE, NT>;
    return 1024 + 3 * (size_t)((G::RAW + 1023) / 1024 * 1024) + 2 * (size_t)G::CB * (G::A_BYTES + G::B_BYTES) +
           2 * (size_t)G::CB * (NT * 8 + 128 * 8);
}

template <int TYPE, int EPI, int NT>
__global__ void __launch_bounds__(128, 2) gemm_tc_kernel(tc::Args A) {
    using namespace tc;
    using G = Geo<TYPE, NT>;
    constexpr bool Q6 = G::Q6;
    constexpr int CB = G::CB, COLS = G::COLS;
    constexpr int RAWSZ = (G::RAW + 1023) / 1024 * 1024;
    constexpr uint32_t IDESC = idesc_i8(128, NT);
    extern __shared__ __align__(16) uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t tma_bar[3], mma_bar[2];
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;
    __shared__ float best_v[4][64];
    __shared__ uint32_t best_i[4][64];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const Matrix &W = A.W;
    const int nb = W.nb, nsb = W.nsb;
    const int nchunks = (nb + CB - 1) / CB;
    uint8_t *base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint8_t *raw = base;                                          // 3 x RAWSZ
    uint8_t *tA = raw + 3 * RAWSZ;                                // 2 x CB x A_BYTES
    uint8_t *tB = tA + 2 * CB * G::A_BYTES;                       // 2 x CB x B_BYTES
    float *tok_sc = reinterpret_cast<float *>(tB + 2 * CB * G::B_BYTES);   // [2][CB][NT][2]
    float *row_sc = tok_sc + 2 * CB * NT * 2;                    // [2][CB][128][2]

    if (tid == 0) {
        for (int i = 0; i < 3; ++i) mbar_init(&tma_bar[i], 1);
        for (int i = 0; i < 2; ++i) mbar_init(&mma_bar[i], 1);
        abort_sh = 0;
    }
    if (EPI == EPI_ARGMAX)
        for (int n = tid; n < 256; n += 128) {
            best_v[n >> 6][n & 63] = kNegInf;
            best_i[n >> 6][n & 63] = 0xffffffffu;
        }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(smem_u32(&tmem_base_sh))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = tmem_base_sh;
    const int tiles = A.row_tiles * A.tok_tiles;
    pdl_launch_dependents();

    // Raw bytes of chunk `c` of row tile `rt` into ring slot `slot` (thread 0).
    auto issue = [&](int rt, int tt, int c, int slot) {
        const int j0 = c * CB, nj = min(CB, nb - j0);
        uint8_t *dst = raw + (size_t)slot * RAWSZ;
        uint32_t bytes = 4 * nj * (G::RA + G::RB + G::RC) + (TYPE == T_Q4_K ? 4 * 512 : 0) + (Q6 ? 4 * 64 : 0);
        bytes += NT * nj * 32 + nj * NT * 4 * (TYPE == T_Q4_K ? 2 : 1);
        mbar_expect_tx(&tma_bar[slot], bytes);
        // activations of the token tile (rows padded to 64: always in bounds)
        for (int n = 0; n < NT; ++n)
            bulk_g2s(dst + G::XQ + n * CB * 32, A.x.q + (size_t)(tt * NT + n) * W.K + 32 * j0, nj * 32, &tma_bar[slot]);
        for (int b = 0; b < nj; ++b) {
            bulk_g2s(dst + G::XD + b * NT * 4, A.x.dT + (size_t)(j0 + b) * A.x.rs + tt * NT, NT * 4, &tma_bar[slot]);
            if (TYPE == T_Q4_K)
                bulk_g2s(dst + G::XS + b * NT * 4, A.x.sT + (size_t)(j0 + b) * A.x.rs + tt * NT, NT * 4, &tma_bar[slot]);
        }
        // per group: blocks j0..j0+nj of each region are contiguous
        for (int gi = 0; gi < 4; ++gi) {
            const size_t gg = (size_t)rt * 4 + gi;
            bulk_g2s(dst + gi * CB * G::RA, W.a + (gg * nb + j0) * 32 * (G::RA / 32), nj * G::RA, &tma_bar[slot]);
            if (G::RB)
                bulk_g2s(dst + 4 * CB * G::RA + gi * CB * G::RB, W.b + (gg * nb + j0) * 32 * (G::RB / 32), nj * G::RB,
                         &tma_bar[slot]);
            if (G::RC)
                bulk_g2s(dst + 4 * CB * (G::RA + G::RB) + gi * CB * G::RC, W.c + (gg * nb + j0) * 32 * 2, nj * G::RC,
                         &tma_bar[slot]);
            if (TYPE == T_Q4_K)  // the super-block header of this chunk (CB <= 8 blocks stay in one)
                bulk_g2s(dst + 4 * CB * G::RA + gi * 512, W.b + (gg * nsb + j0 / 8) * 32 * 16, 512, &tma_bar[slot]);
            if (Q6)
                bulk_g2s(dst + 4 * CB * (G::RA + G::RB + G::RC) + gi * 64, W.e + (gg * nsb + j0 / 8) * 32 * 2, 64,
                         &tma_bar[slot]);
        }
    };

    uint32_t tma_uses[3] = {0, 0, 0}, mma_uses[2] = {0, 0};
    bool waited = false;
    for (int tile = blockIdx.x; tile < tiles && !abort_sh; tile += gridDim.x) {
        const int rt = tile % A.row_tiles, tt = tile / A.row_tiles;
        const int row = rt * 128 + tid;
        const bool live = row < W.N;
        float acc[NT];
#pragma unroll
        for (int n = 0; n < NT; ++n) acc[n] = 0.0f;
        // chunks 0 and 1 in flight; the first tile waits for the previous kernel
        // before copying activations
        if (!waited) {
            pdl_wait();
            waited = true;
        }
        if (tid == 0) {
            issue(rt, tt, 0, 0);
            if (nchunks > 1) issue(rt, tt, 1, 1);
        }
        for (int c = 0; c <= nchunks; ++c) {
            const int half = c & 1;
            // every thread has finished the epilogue of chunk c-2, whose token
            // scales and tiles the unpacking of chunk c overwrites
            __syncthreads();
            if (abort_sh) break;
            if (c < nchunks) {
                const int slot = c % 3, j0 = c * CB, nj = min(CB, nb - j0);
                if (tid == 0 && c + 2 < nchunks) issue(rt, tt, c + 2, (c + 2) % 3);
                if (!mbar_wait(&tma_bar[slot], tma_uses[slot] & 1)) {
                    atomicOr(A.err, 2u);
                    abort_sh = 1;
                }
                ++tma_uses[slot];
                const uint8_t *rs = raw + (size_t)slot * RAWSZ;
                const int gi = tid >> 5, l = tid & 31;  // this thread unpacks its own row
                for (int b = 0; b < nj; ++b) {
                    uint8_t *ta = tA + (size_t)(half * CB + b) * G::A_BYTES;
                    float s0 = 0.f, s1 = 0.f;
                    if constexpr (TYPE == T_Q8_0) {
                        const int4 *src = reinterpret_cast<const int4 *>(rs + gi * CB * 1024 + b * 1024 + l * 32);
                        *reinterpret_cast<int4 *>(ta + tile_off(tid, 0)) = src[0];
                        *reinterpret_cast<int4 *>(ta + tile_off(tid, 1)) = src[1];
                        s0 = h2f(*reinterpret_cast<const unsigned short *>(rs + 4 * CB * 1024 + gi * CB * 64 + b * 64 + l * 2));
                    } else if constexpr (TYPE == T_Q4_K) {
                        const int4 v = *reinterpret_cast<const int4 *>(rs + gi * CB * 512 + b * 512 + l * 16);
                        *reinterpret_cast<int4 *>(ta + tile_off(tid, 0)) =
                            make_int4(v.x & 0x0f0f0f0f, v.y & 0x0f0f0f0f, v.z & 0x0f0f0f0f, v.w & 0x0f0f0f0f);
                        *reinterpret_cast<int4 *>(ta + tile_off(tid, 1)) =
                            make_int4((v.x >> 4) & 0x0f0f0f0f, (v.y >> 4) & 0x0f0f0f0f, (v.z >> 4) & 0x0f0f0f0f,
                                      (v.w >> 4) & 0x0f0f0f0f);
                        const uint4 h = *reinterpret_cast<const uint4 *>(rs + 4 * CB * 512 + gi * 512 + l * 16);
                        const int sbk = (j0 + b) & 7;
                        auto byte = [&](int kk) -> int {
                            const uint32_t w = kk < 4 ? h.y : (kk < 8 ? h.z : h.w);
                            return (w >> (8 * (kk & 3))) & 0xff;
                        };
                        int sc, mm;
                        if (sbk < 4) {
                            sc = byte(sbk) & 63;
                            mm = byte(sbk + 4) & 63;
                        } else {
                            sc = (byte(sbk + 4) & 0xf) | ((byte(sbk - 4) >> 6) << 4);
                            mm = (byte(sbk + 4) >> 4) | ((byte(sbk) >> 6) << 4);
                        }
                        // d*sc and dmin*m are exact products (11-bit f16 x 6-bit integer)
                        s0 = __fmul_rn(h2f(h.x & 0xffff), (float)sc);
                        s1 = __fmul_rn(h2f(h.x >> 16), (float)mm);
                    } else {
                        const int4 lq = *reinterpret_cast<const int4 *>(rs + gi * CB * 512 + b * 512 + l * 16);
                        const uint2 hq = *reinterpret_cast<const uint2 *>(rs + 4 * CB * 512 + gi * CB * 256 + b * 256 + l * 8);
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
                        const int4 z = make_int4(0, 0, 0, 0);
                        *reinterpret_cast<int4 *>(ta + tile_off(tid, 0)) = make_int4(a4[0], a4[1], a4[2], a4[3]);
                        *reinterpret_cast<int4 *>(ta + tile_off(tid, 1)) = z;
                        *reinterpret_cast<int4 *>(ta + 4096 + tile_off(tid, 0)) = z;
                        *reinterpret_cast<int4 *>(ta + 4096 + tile_off(tid, 1)) = make_int4(b4[0], b4[1], b4[2], b4[3]);
                        s0 = h2f(*reinterpret_cast<const unsigned short *>(rs + 4 * CB * (512 + 256 + 64) + gi * 64 + l * 2));
                        s1 = __int_as_float(
                            (int)*reinterpret_cast<const unsigned short *>(rs + 4 * CB * (512 + 256) + gi * CB * 64 + b * 64 + l * 2));
                    }
                    row_sc[((half * CB + b) * 128 + tid) * 2] = s0;
                    row_sc[((half * CB + b) * 128 + tid) * 2 + 1] = s1;
                }
                // activation blocks (staged raw by the bulk copies) into the UMMA layout
                for (int e = tid; e < NT * nj * 2; e += 128) {
                    const int n = e / (nj * 2), b = (e >> 1) % nj, k16 = e & 1;
                    *reinterpret_cast<int4 *>(tB + (size_t)(half * CB + b) * G::B_BYTES + tile_off(n, k16)) =
                        *reinterpret_cast<const int4 *>(rs + G::XQ + n * CB * 32 + b * 32 + 16 * k16);
                }
                for (int e = tid; e < NT * nj; e += 128) {
                    const int b = e / NT, n = e % NT;
                    tok_sc[((half * CB + b) * NT + n) * 2] = reinterpret_cast<const float *>(rs + G::XD)[b * NT + n];
                    tok_sc[((half * CB + b) * NT + n) * 2 + 1] =
                        TYPE == T_Q4_K ? reinterpret_cast<const float *>(rs + G::XS)[b * NT + n] : 0.0f;
                }
                fence_async_smem();
                fence_before();
                __syncthreads();
                fence_after();
                if (tid == 0 && !abort_sh) {
                    for (int b = 0; b < nj; ++b) {
                        const uint64_t da = sdesc(tA + (size_t)(half * CB + b) * G::A_BYTES, 128, 256);
                        const uint64_t db = sdesc(tB + (size_t)(half * CB + b) * G::B_BYTES, 128, 256);
                        const uint32_t col = tmem + (half * CB + b) * COLS;
                        mma_i8(col, da, db, IDESC);
                        if constexpr (Q6)
                            mma_i8(col + NT, sdesc(tA + (size_t)(half * CB + b) * G::A_BYTES + 4096, 128, 256), db, IDESC);
                    }
                    commit(&mma_bar[half]);
                }
            }
            // epilogue of chunk c-1 (its MMAs overlap the unpacking of chunk c)
            if (c > 0) {
                const int pc = c - 1, ph = pc & 1, pj0 = pc * CB, pnj = min(CB, nb - pj0);
                if (!mbar_wait(&mma_bar[ph], mma_uses[ph] & 1)) {
                    atomicOr(A.err, 4u);
                    abort_sh = 1;  // every thread stops at the next barrier
                }
                ++mma_uses[ph];
                fence_after();
                for (int b = 0; b < pnj && !abort_sh; ++b) {
                    const int j = pj0 + b;
                    const float r0 = row_sc[((ph * CB + b) * 128 + tid) * 2];
                    const float r1 = row_sc[((ph * CB + b) * 128 + tid) * 2 + 1];
                    int sa = 0, sb = 0;
                    if constexpr (Q6) {
                        const int packed = __float_as_int(r1);
                        sa = (int8_t)(packed & 0xff);
                        sb = (int8_t)((packed >> 8) & 0xff);
                    }
                    const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (ph * CB + b) * COLS;
                    constexpr int CH = NT < 16 ? NT : 16;
#pragma unroll
                    for (int c0 = 0; c0 < NT; c0 += CH) {
                        uint32_t v[CH], v2[CH];
                        tmem_ld<CH>(taddr + c0, v);
                        if constexpr (Q6) tmem_ld<CH>(taddr + NT + c0, v2);
                        tmem_wait_ld();
                        const float *ts = tok_sc + ((ph * CB + b) * NT + c0) * 2;
#pragma unroll
                        for (int u = 0; u < CH; u += 2) {
                            const float4 t4 = *reinterpret_cast<const float4 *>(ts + 2 * u);
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const int n = c0 + u + h;
                                const float xd = h ? t4.z : t4.x, s8f = h ? t4.w : t4.y;
                                const int I = (int)v[u + h];
                                float p;
                                if constexpr (TYPE == T_Q8_0) {
                                    p = __fmul_rn(__fmul_rn(r0, xd), (float)I);
                                } else if constexpr (TYPE == T_Q4_K) {
                                    // = xd * (d*float(I*sc) - dmin*float(s8*m)): the products are exact
                                    p = __fmul_rn(xd, __fsub_rn(__fmul_rn(r0, (float)I), __fmul_rn(r1, s8f)));
                                } else {
                                    p = __fmul_rn(__fmul_rn(r0, xd), (float)(sa * I + sb * (int)v2[u + h]));
                                }
                                acc[n] = j == 0 ? p : __fadd_rn(acc[n], p);
                            }
                        }
                    }
                }
                fence_before();
            }
        }
        __syncthreads();
        if (abort_sh) break;
        // tile epilogue
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const int tok = tt * NT + n;
            if (tok >= A.rows) break;  // uniform across the CTA
            if constexpr (EPI == EPI_ARGMAX) {
                float bv = live ? acc[n] : kNegInf;
                uint32_t bi = live ? (uint32_t)row : 0xffffffffu;
                if (A.g.logits && live) A.g.logits[(size_t)tok * W.N + row] = acc[n];
                warp_argmax(bv, bi);
                if (lane == 0) argmax_merge(best_v[warp][tok & 63], best_i[warp][tok & 63], bv, bi);
            } else if (live) {
                epilogue_store<EPI>(A.g, row, tok, acc[n]);
            }
        }
        __syncthreads();  // the tile's buffers are reused by the next tile
    }
    if (!waited) pdl_wait();  // a CTA without a tile still keeps the launch chain ordered
    fence_before();
    __syncthreads();
    if constexpr (EPI == EPI_ARGMAX) {
        for (int n = tid; n < A.rows && n < 64; n += 128) {
            float v = best_v[0][n];
            uint32_t i = best_i[0][n];
            for (int w = 1; w < 4; ++w) argmax_merge(v, i, best_v[w][n], best_i[w][n]);
            A.g.part_v[(size_t)n * gridDim.x + blockIdx.x] = v;
            A.g.part_i[(size_t)n * gridDim.x + blockIdx.x] = i;
        }
    }
    if (warp == 0) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem) : "memory");
    }
}

// q8_1 activations of one row per CTA into global memory (the tensor-core
// matmul's input): the row is staged in shared memory (embedding rows are
// dequantized once), LayerNorm statistics by one warp in the fixed order, and
// the 8 warps quantize the blocks.
template <int MODE>
__global__ void __launch_bounds__(256) qprep_row_kernel(PrepArgs p, QAct out) {
    extern __shared__ __align__(16) float xs[];
    __shared__ float st[2];
    __shared__ uint32_t id_sh[1];
    pdl_launch_dependents();
    pdl_wait();
    const int r = blockIdx.x, K = p.K, nb = K >> 5;
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
    SmAct s;
    s.q = out.q + (size_t)r * K;
    s.d = out.d + (size_t)r * nb;
    s.s32 = out.s32 + (size_t)r * nb;
    s.s16 = out.s16 + (size_t)r * 2 * nb;
    s.st = st;
    s.xf = nullptr;
    PrepArgs q = p;
    q.x = xs;
    q.rows = 1;
    build_activations_impl<MODE == PREP_PLAIN ? PREP_PLAIN : PREP_LN>(q, s, 1, false);
    if (out.rs) {  // block-major copies of the scales for the tensor-core matmul
        __syncthreads();
        for (int j = threadIdx.x; j < nb; j += blockDim.x) {
            out.dT[(size_t)j * out.rs + r] = s.d[j];
            out.sT[(size_t)j * out.rs + r] = (float)s.s32[j];
        }
    }
}

}  // namespace mgb
