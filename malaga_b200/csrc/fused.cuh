// Fused decode-step matmul for small batches: activation prologue + weight rows
// + epilogue in one kernel (sm_100a).
//
// One launch replaces the reference's chain "bias_residual_ln / embed_pos_ln
// (malaga.cu:89-130) -> candle q8_1 quantize -> QMatMul MMVQ -> bias / ReLU /
// residual / qkv_decode epilogue (malaga.cu:133-154)":
//   1. the CTA asks L2 to prefetch its slice of the weight matrix (bulk
//      prefetch; weights do not depend on the previous kernel),
//   2. programmatic dependent launch: it lets the next kernel start and waits for
//      the previous one,
//   3. it builds the q8_1 activations of every batch row in shared memory
//      (LayerNorm / embedding+position+LayerNorm / plain), in the engine's fixed
//      reduction order,
//   4. each warp computes a group of 32 weight rows (lane = row), summing the
//      block partials left to right, and the epilogue writes the result.
#pragma once
#include "kernels.cuh"

namespace mgb {

struct FusedArgs {
    GemvArgs g;     // matrix, outputs and epilogue parameters
    PrepArgs p;     // activation source (x or a/u, LayerNorm, embedding)
    int rows_per_cta;  // row groups (of 32) per CTA
    AttnArgs at;    // PREP_ATTN: the attention whose outputs are the input
};

// Shared memory of the attention prologue (PREP_ATTN): per warp the scores of
// max_keys keys and a 64-key f16 V staging tile.
__host__ __device__ inline size_t attn_prologue_bytes(int max_keys, int hd) {
    return 16 + (size_t)8 * max_keys * 4 + (size_t)8 * 64 * hd * 2;  // (16: alignment of the scratch)
}

// Bytes per 32-row group of each region of the engine layout (see engine.h).
__device__ __forceinline__ void region_group_bytes(const Matrix &W, size_t (&rb)[4]) {
    const size_t nb = W.nb, nsb = W.nsb;
    switch (W.type) {
        case T_F32: rb[0] = nb * 32 * 128; rb[1] = rb[2] = rb[3] = 0; break;
        case T_Q8_0: rb[0] = nb * 32 * 32; rb[1] = nb * 32 * 2; rb[2] = rb[3] = 0; break;
        case T_Q4_K: rb[0] = nb * 32 * 16; rb[1] = nsb * 32 * 16; rb[2] = rb[3] = 0; break;
        default: rb[0] = nb * 32 * 16; rb[1] = nb * 32 * 8; rb[2] = nb * 32 * 2; rb[3] = nsb * 32 * 2; break;
    }
}

// Bulk L2 prefetch of row groups [g0, g1) of every region (rounded out to 16
// bytes; regions are 256-byte aligned inside the weight arena).
__device__ __forceinline__ void prefetch_groups(const Matrix &W, int g0, int g1) {
    if (threadIdx.x >= 4 || g0 >= g1) return;
    size_t rb[4];
    region_group_bytes(W, rb);
    const uint8_t *base[4] = {W.a, W.b, W.c, W.e};
    const int k = threadIdx.x;
    if (!rb[k] || !base[k]) return;
    uint64_t lo = (uint64_t)(base[k] + (size_t)g0 * rb[k]);
    uint64_t hi = (uint64_t)(base[k] + (size_t)g1 * rb[k]);
    lo &= ~15ull;
    hi = (hi + 15) & ~15ull;
    while (lo < hi) {
        const uint64_t n = (hi - lo) > (1ull << 30) ? (1ull << 30) : (hi - lo);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(lo), "r"((uint32_t)n) : "memory");
        lo += n;
    }
}

// Shared-memory q8_1 activations of B rows.
struct SmAct {
    int8_t *q;   // [B][K]
    float *d;    // [B][nb]
    int *s32;    // [B][nb]
    int *s16;    // [B][2nb]
    float *st;   // [B][2] mean, rstd
    float *xf;   // [B][K] (F32 weights only)
};

__host__ __device__ inline size_t smact_bytes(int B, int K, bool f32) {
    const int nb = K / 32;
    size_t n = (size_t)B * K;
    n = (n + 15) / 16 * 16;
    n += (size_t)B * nb * 4 * 4 + (size_t)B * 2 * 4;
    if (f32) n += (size_t)B * K * 4;
    return n + 64;
}

__device__ __forceinline__ SmAct smact_carve(uint8_t *sm, int B, int K, bool f32) {
    const int nb = K / 32;
    SmAct s;
    size_t o = 0;
    s.q = reinterpret_cast<int8_t *>(sm);
    o += ((size_t)B * K + 15) / 16 * 16;
    s.d = reinterpret_cast<float *>(sm + o);
    o += (size_t)B * nb * 4;
    s.s32 = reinterpret_cast<int *>(sm + o);
    o += (size_t)B * nb * 4;
    s.s16 = reinterpret_cast<int *>(sm + o);
    o += (size_t)B * nb * 8;
    s.st = reinterpret_cast<float *>(sm + o);
    o += (size_t)B * 8;
    s.xf = f32 ? reinterpret_cast<float *>(sm + o) : nullptr;
    return s;
}

// Element i of batch row r of the activation input, before normalisation.
// When the rows were staged in shared memory (p.x points there, MODE is then
// treated as PLAIN/LN over those rows), the reads hit shared memory.
template <int MODE>
__device__ __forceinline__ float act_input(const PrepArgs &p, int r, int i) {
    if constexpr (MODE == PREP_EMBED_LN) {
        // p.ids / p.pos_table were rebased by the kernel: ids from shared memory,
        // pos_table pointing at this step's position row.
        return __fadd_rn(__fmul_rn(deq_elem(p.embed, (int)p.ids[r], i), p.scale), p.pos_table[i]);
    } else {
        return p.x[(size_t)r * p.K + i];
    }
}

// Builds the activations of all B rows in shared memory. Phase A (LN modes):
// one warp per row loads the whole row into registers (independent loads, one
// memory latency), then computes mean and 1/std with the lane-ordered pairwise
// sum. Phase B: warps quantize (row, block) pairs in parallel, loading the
// inputs of 8 pairs before processing them.
template <int MODE, int G>
__device__ void build_activations_impl(const PrepArgs &p, const SmAct &s, int B, bool write_x);

// Entry point: for LN / embedding inputs of at most 64 KB, all threads first
// bring the B input rows into shared memory (one memory round trip; the
// embedding rows are dequantized once), then the LayerNorm statistics and the
// quantization read them from there.
template <int MODE, int G>
__device__ void build_activations(const PrepArgs &p, const SmAct &s, int B, bool write_x, float *xs) {
    if constexpr (MODE != PREP_PLAIN) {
        if (xs) {
            const int K = p.K;
            // 8 loads in flight per thread before their stores (one memory round trip)
            for (int base = threadIdx.x; base < B * K; base += 8 * blockDim.x) {
                float v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int idx = base + u * blockDim.x;
                    v[u] = idx < B * K ? act_input<MODE>(p, idx / K, idx % K) : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int idx = base + u * blockDim.x;
                    if (idx >= B * K) break;
                    xs[idx] = v[u];
                    if constexpr (MODE == PREP_EMBED_LN)
                        if (write_x) p.x_out[idx] = v[u];
                }
            }
            __syncthreads();
            PrepArgs q = p;
            q.x = xs;
            build_activations_impl<PREP_LN, G>(q, s, B, false);
            return;
        }
    }
    build_activations_impl<MODE, G>(p, s, B, write_x);
}

template <int MODE, int G>
__device__ void build_activations_impl(const PrepArgs &p, const SmAct &s, int B, bool write_x) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int K = p.K, T = K >> 5, nb = T;
    if constexpr (MODE != PREP_PLAIN) {
        constexpr int CH = 16;  // loads in flight per lane; the sums stay strictly in order
        for (int r = warp; r < B; r += nw) {
            float sum = 0.0f;
            for (int t0 = 0; t0 < T; t0 += CH) {
                float v[CH];
#pragma unroll
                for (int u = 0; u < CH; ++u)
                    if (t0 + u < T) v[u] = act_input<MODE>(p, r, 32 * (t0 + u) + lane);
#pragma unroll
                for (int u = 0; u < CH; ++u) {
                    if (t0 + u >= T) break;
                    if constexpr (MODE == PREP_EMBED_LN)
                        if (write_x) p.x_out[(size_t)r * K + 32 * (t0 + u) + lane] = v[u];
                    sum = t0 + u == 0 ? v[u] : __fadd_rn(sum, v[u]);
                }
            }
            const float mean = __fdiv_rn(warp_tree(sum), (float)K);
            float s2 = 0.0f;
            for (int t0 = 0; t0 < T; t0 += CH) {
                float v[CH];
#pragma unroll
                for (int u = 0; u < CH; ++u)
                    if (t0 + u < T) v[u] = act_input<MODE>(p, r, 32 * (t0 + u) + lane);
#pragma unroll
                for (int u = 0; u < CH; ++u) {
                    if (t0 + u >= T) break;
                    const float c = __fsub_rn(v[u], mean);
                    const float c2 = __fmul_rn(c, c);
                    s2 = t0 + u == 0 ? c2 : __fadd_rn(s2, c2);
                }
            }
            const float var = __fdiv_rn(warp_tree(s2), (float)K);
            if (lane == 0) {
                s.st[2 * r] = mean;
                s.st[2 * r + 1] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
            }
        }
        __syncthreads();
    }
    auto norm = [&](float v, int r, int i) -> float {
        if constexpr (MODE != PREP_PLAIN)
            v = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v, s.st[2 * r]), s.st[2 * r + 1]), p.gamma[i]), p.beta[i]);
        if (s.xf) s.xf[(size_t)r * K + i] = v;
        return v;
    };
    if constexpr (G == 1) {
        // (row, block) tasks, 8 in flight per warp
        constexpr int PIPE = 8;
        const int tasks = B * T;
        for (int base = warp; base < tasks; base += nw * PIPE) {
            float y[PIPE];
#pragma unroll
            for (int u = 0; u < PIPE; ++u) {
                const int task = base + u * nw;
                y[u] = task < tasks ? act_input<MODE>(p, task / T, 32 * (task % T) + lane) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < PIPE; ++u) {
                const int task = base + u * nw;
                if (task >= tasks) break;  // uniform across the warp
                const int r = task / T, t = task % T;
                const float yy[1] = {norm(y[u], r, 32 * t + lane)};
                quantize_group<1>(yy, s.q + (size_t)r * K, s.d + (size_t)r * nb, s.s32 + (size_t)r * nb,
                                  s.s16 + (size_t)r * 2 * nb, t, lane);
            }
        }
    } else {
        // (row, super-block) tasks: the 8 blocks share one scale
        const int tasks = B * (T / 8);
        for (int task = warp; task < tasks; task += nw) {
            const int r = task / (T / 8), t0 = 8 * (task % (T / 8));
            float y[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) y[u] = act_input<MODE>(p, r, 32 * (t0 + u) + lane);
#pragma unroll
            for (int u = 0; u < 8; ++u) y[u] = norm(y[u], r, 32 * (t0 + u) + lane);
            quantize_group<8>(y, s.q + (size_t)r * K, s.d + (size_t)r * nb, s.s32 + (size_t)r * nb,
                              s.s16 + (size_t)r * 2 * nb, t0, lane);
        }
    }
    __syncthreads();
}

template <int TYPE, int EPI, int MODE, int NB>
__global__ void __launch_bounds__(256) gemv_fused_kernel(FusedArgs fa) {
    extern __shared__ __align__(16) uint8_t sm_raw[];
    const GemvArgs &g = fa.g;
    const Matrix &W = g.W;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int groups = W.Np >> 5;
    const int g0 = blockIdx.x * fa.rows_per_cta, g1 = min(groups, g0 + fa.rows_per_cta);
    prefetch_groups(W, g0, g1);
    pdl_launch_dependents();
    pdl_wait();
    const int B = g.rows;
    const SmAct s = smact_carve(sm_raw, B, W.K, TYPE == T_F32);
    PrepArgs pa = fa.p;
    if constexpr (MODE == PREP_EMBED_LN) {
        __shared__ uint32_t ids_sh[64];
        for (int r = threadIdx.x; r < B; r += blockDim.x) ids_sh[r] = pa.ids[r];
        pa.pos_table += (size_t)(*pa.step + pa.pos_base) * pa.K;
        pa.ids = ids_sh;
        __syncthreads();
    }
    float *xs = nullptr;
    if constexpr (MODE != PREP_PLAIN) xs = reinterpret_cast<float *>(sm_raw + smact_bytes(B, W.K, TYPE == T_F32));
    build_activations<MODE, act_group(TYPE)>(pa, s, B, blockIdx.x == 0,
                                             (size_t)B * W.K * 4 <= 64 * 1024 ? xs : nullptr);

    __shared__ float best_v[8][NB];
    __shared__ uint32_t best_i[8][NB];
    if constexpr (EPI == EPI_ARGMAX) {
        if (lane < NB) {
            best_v[warp][lane] = kNegInf;
            best_i[warp][lane] = 0xffffffffu;
        }
    }
    const int nb = W.nb;
    for (int grp = g0 + warp; grp < g1; grp += 8) {
        const int row = grp * 32 + lane;
        for (int n0 = 0; n0 < B; n0 += NB) {
            float acc[NB];
#pragma unroll
            for (int i = 0; i < NB; ++i) acc[i] = 0.0f;
            if constexpr (TYPE == T_F32) {
#pragma unroll 8
                for (int j = 0; j < nb; ++j)
#pragma unroll
                    for (int i = 0; i < NB; ++i) {
                        if (n0 + i >= B) break;
                        const float p = f32_block(W, row, j, s.xf + (size_t)(n0 + i) * W.K + 32 * j);
                        acc[i] = j == 0 ? p : __fadd_rn(acc[i], p);
                    }
            } else {
                constexpr int UB = unit_blocks<TYPE>();
                for (int u = 0; u < nb; u += UB) {
                    int S1[NB], S2[NB];
#pragma unroll
                    for (int i = 0; i < NB; ++i) S1[i] = S2[i] = 0;
                    BlockW<TYPE> bw;
#pragma unroll 8
                    for (int j = u; j < u + UB; ++j) {
                        bw.load(W, row, j);
#pragma unroll
                        for (int i = 0; i < NB; ++i) {
                            const int n = n0 + i;
                            if (n >= B) break;
                            const int4 *xs = reinterpret_cast<const int4 *>(s.q + (size_t)n * W.K + 32 * j);
                            const int4 x0 = xs[0], x1 = xs[1];
                            const int xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                            int s32 = 0, s16a = 0, s16b = 0;
                            if constexpr (TYPE == T_Q4_K) s32 = s.s32[(size_t)n * nb + j];
                            if constexpr (TYPE == T_Q6_K) {
                                s16a = s.s16[(size_t)n * 2 * nb + 2 * j];
                                s16b = s.s16[(size_t)n * 2 * nb + 2 * j + 1];
                            }
                            bw.accum(xv, s32, s16a, s16b, S1[i], S2[i]);
                        }
                    }
#pragma unroll
                    for (int i = 0; i < NB; ++i) {
                        const int n = n0 + i;
                        if (n >= B) break;
                        const float p = bw.finish(S1[i], S2[i], s.d[(size_t)n * nb + u]);
                        acc[i] = u == 0 ? p : __fadd_rn(acc[i], p);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                const int n = n0 + i;
                if (n >= B) break;  // uniform across the warp
                if constexpr (EPI == EPI_ARGMAX) {
                    if (g.logits && row < W.N) g.logits[(size_t)n * W.N + row] = acc[i];
                    float v = row < W.N ? acc[i] : kNegInf;
                    uint32_t idx = row < W.N ? (uint32_t)row : 0xffffffffu;
                    warp_argmax(v, idx);
                    if (lane == 0) argmax_merge(best_v[warp][i], best_i[warp][i], v, idx);
                } else {
                    if (row < W.N) epilogue_store<EPI>(g, row, n, acc[i]);
                }
            }
        }
    }
    if constexpr (EPI == EPI_ARGMAX) {
        __syncthreads();
        for (int n = threadIdx.x; n < B; n += blockDim.x) {
            float v = best_v[0][n];
            uint32_t i = best_i[0][n];
            for (int w = 1; w < 8; ++w) argmax_merge(v, i, best_v[w][n], best_i[w][n]);
            g.part_v[(size_t)n * gridDim.x + blockIdx.x] = v;
            g.part_i[(size_t)n * gridDim.x + blockIdx.x] = i;
        }
    }
}

}  // namespace mgb

namespace mgb {

// ---------------------------------------------------------------------------
// Small-batch matmul with TMA-staged weights: one CTA per group of 32 weight
// rows. Before waiting on the previous kernel, thread 0 starts 1-D bulk copies
// (cp.async.bulk, completion counted on an mbarrier) of the group's weight
// slices into shared memory. After the activation prologue, the 8 warps split
// the K blocks (lane = row) and write each block's integer sums (k-quants) or
// float partial (Q8_0) to shared memory; then each row's units are finished and
// summed left to right.

constexpr uint64_t kWaitNs = 500000000ull;  // give up a wait after 0.5 s of device time

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// One try_wait: a thread whose phase is not complete may sleep until it
// completes (or a time limit runs out: MGB_WAIT_HINT_NS when nonzero, else the
// hardware's own) instead of spinning, so waiting warps do not take issue
// slots from working ones.
#ifndef MGB_WAIT_HINT_NS
#define MGB_WAIT_HINT_NS 0
#endif
__device__ __forceinline__ bool mbar_try(uint32_t a, uint32_t parity) {
    uint32_t done;
#if MGB_WAIT_HINT_NS > 0
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(a), "r"(parity), "r"((uint32_t)MGB_WAIT_HINT_NS)
        : "memory");
#else
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
#endif
    return done != 0;
}

// Bounded wait for phase `parity` of the mbarrier; false once kWaitNs passed.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    if (mbar_try(a, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (;;) {
        if (mbar_try(a, parity)) return true;
        if (globaltimer() - t0 > kWaitNs) return false;
    }
}

// Shared-memory bytes of the staged kernel's per-block partials: two ints per
// (row, block, weight row) for Q4_K, one int or float otherwise.
__host__ __device__ constexpr size_t staged_partial_bytes(int type, int B, int nb) {
    return (size_t)B * nb * 32 * (type == T_Q4_K ? 8 : 4);
}

// Shared-memory bytes of one group's staged weights (each region 16-B aligned).
__host__ __device__ inline size_t staged_bytes(int type, int nb, int nsb) {
    switch (type) {
        case T_Q8_0: return (size_t)nb * 32 * 32 + (size_t)nb * 64;
        case T_Q4_K: return (size_t)nb * 32 * 16 + (size_t)nsb * 32 * 16;
        case T_Q6_K: return (size_t)nb * 32 * 16 + (size_t)nb * 32 * 8 + (size_t)nb * 64 + (size_t)nsb * 64;
    }
    return 0;
}

template <int TYPE, int EPI, int MODE>
__global__ void __launch_bounds__(256) gemv_staged_kernel(FusedArgs fa, uint32_t *err) {
    extern __shared__ __align__(16) uint8_t sm_raw[];
    __shared__ __align__(8) uint64_t bar;
    const GemvArgs &g = fa.g;
    const Matrix &W = g.W;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int grp = blockIdx.x, nb = W.nb, nsb = W.nsb;
    const size_t wbytes = staged_bytes(TYPE, nb, nsb);
    // shared layout: [staged weights][activations][partials]
    Matrix Ws = W;  // a view of this group as "group 0" in shared memory
    Ws.Np = 32;
    {
        uint8_t *p = sm_raw;
        size_t rb[4];
        region_group_bytes(W, rb);
        const uint8_t *src[4] = {W.a, W.b, W.c, W.e};
        const uint8_t **dst[4] = {&Ws.a, &Ws.b, &Ws.c, &Ws.e};
        if (threadIdx.x == 0) {
            mbar_init(&bar, 1);
            mbar_expect_tx(&bar, (uint32_t)wbytes);
        }
        __syncthreads();
        for (int k = 0; k < 4; ++k) {
            if (!rb[k] || !src[k]) continue;
            if (threadIdx.x == 0) bulk_g2s(p, src[k] + (size_t)grp * rb[k], (uint32_t)rb[k], &bar);
            *dst[k] = p;
            p += rb[k];
        }
    }
    const int B = g.rows;
    // LayerNorm parameters (constant weights) into shared memory while the
    // previous kernel finishes: after the partials (and any attention scratch)
    float *gb = nullptr;
    if constexpr (MODE == PREP_LN || MODE == PREP_EMBED_LN) {
        gb = reinterpret_cast<float *>(sm_raw + wbytes + smact_bytes(B, W.K, false) + staged_partial_bytes(TYPE, B, W.nb));
        for (int i = threadIdx.x; i < W.K; i += blockDim.x) {
            gb[i] = __ldg(fa.p.gamma + i);
            gb[W.K + i] = __ldg(fa.p.beta + i);
        }
    }
    pdl_launch_dependents();
    pdl_wait();
    const SmAct s = smact_carve(sm_raw + wbytes, B, W.K, false);
    float *P = reinterpret_cast<float *>(sm_raw + wbytes + smact_bytes(B, W.K, false));
    float *xs = MODE != PREP_PLAIN ? P : nullptr;  // input rows share the partials' space (used before them)
    PrepArgs pa = fa.p;
    if (gb) {
        pa.gamma = gb;
        pa.beta = gb + W.K;
    }
    if constexpr (MODE == PREP_EMBED_LN) {
        __shared__ uint32_t ids_sh[64];
        for (int r = threadIdx.x; r < B; r += blockDim.x) ids_sh[r] = pa.ids[r];
        pa.pos_table += (size_t)(*pa.step + pa.pos_base) * pa.K;
        pa.ids = ids_sh;
        __syncthreads();
    }
    if constexpr (MODE == PREP_ATTN) {
        // the attention outputs of the B rows (every head; one warp per (row, head),
        // the attention kernel's arithmetic) into shared memory, then quantized
        const AttnArgs &at = fa.at;
        float *xa = reinterpret_cast<float *>(sm_raw + wbytes + smact_bytes(B, W.K, false));  // B x K (partials' space)
        // scratch after the partials, 16-byte aligned (V rows are staged with 16-byte stores)
        uint8_t *eb = reinterpret_cast<uint8_t *>(xa) + staged_partial_bytes(TYPE, B, nb);
        float *esc = reinterpret_cast<float *>(eb + ((16 - (smem_u32(eb) & 15)) & 15));
        float *e = esc + (size_t)warp * at.max_keys;
        __half *vs = reinterpret_cast<__half *>(esc + (size_t)8 * at.max_keys) + (size_t)warp * 64 * at.hd;
        for (int t = warp; t < B * at.H; t += 8) {
            const int n = t / at.H, h = t % at.H;
            bool live;
            if (at.hd == 64) {
                float res[2];
                attend_one<__half, 64>(at, n, h, 0, e, vs, lane, res, live);
                xa[(size_t)n * W.K + h * 64 + lane] = res[0];
                xa[(size_t)n * W.K + h * 64 + 32 + lane] = res[1];
            } else {
                float res[4];
                attend_one<__half, 128>(at, n, h, 0, e, vs, lane, res, live);
#pragma unroll
                for (int c = 0; c < 4; ++c) xa[(size_t)n * W.K + h * 128 + 32 * c + lane] = res[c];
            }
        }
        __syncthreads();
        PrepArgs q = pa;
        q.x = xa;
        build_activations_impl<PREP_PLAIN, act_group(TYPE)>(q, s, B, false);
    } else {
        build_activations<MODE, act_group(TYPE)>(pa, s, B, blockIdx.x == 0,
                                                 (size_t)B * W.K * 4 <= staged_partial_bytes(TYPE, B, nb) ? xs : nullptr);
    }
    if (!mbar_wait(&bar, 0)) {
        if (lane == 0) atomicOr(err, 1u);  // copy never completed: report, produce nothing
        return;
    }
    // per-block integer sums (k-quants) or float partials (Q8_0) of every
    // (activation row, block, weight row); units are then finished in order
    constexpr int UB = unit_blocks<TYPE>();
    int *P1 = reinterpret_cast<int *>(P), *P2 = P1 + (size_t)B * nb * 32;
    const int cb = (nb + 7) / 8, j0 = warp * cb, j1 = min(nb, j0 + cb);
    for (int n = 0; n < B; ++n) {
        const int4 *xq = reinterpret_cast<const int4 *>(s.q + (size_t)n * W.K);
#pragma unroll 4
        for (int j = j0; j < j1; ++j) {
            BlockW<TYPE> bw;
            bw.template load<false>(Ws, lane, j);
            const int4 x0 = xq[2 * j], x1 = xq[2 * j + 1];
            const int xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            int s32 = 0, s16a = 0, s16b = 0;
            if constexpr (TYPE == T_Q4_K) s32 = s.s32[(size_t)n * nb + j];
            if constexpr (TYPE == T_Q6_K) {
                s16a = s.s16[(size_t)n * 2 * nb + 2 * j];
                s16b = s.s16[(size_t)n * 2 * nb + 2 * j + 1];
            }
            int S1 = 0, S2 = 0;
            bw.accum(xv, s32, s16a, s16b, S1, S2);
            const size_t o = ((size_t)n * nb + j) * 32 + lane;
            if constexpr (UB == 1) {
                P[o] = bw.finish(S1, S2, s.d[(size_t)n * nb + j]);
            } else {
                P1[o] = S1;
                if constexpr (TYPE == T_Q4_K) P2[o] = S2;
            }
        }
    }
    __syncthreads();
    const int row = grp * 32 + lane;
    for (int n = warp; n < B; n += 8) {
        float acc = 0.0f;
        if constexpr (UB == 1) {
            const float *pn = P + (size_t)n * nb * 32 + lane;
            acc = pn[0];
#pragma unroll 8
            for (int j = 1; j < nb; ++j) acc = __fadd_rn(acc, pn[(size_t)j * 32]);
        } else {
            for (int u = 0; u < nb; u += UB) {
                int S1 = 0, S2 = 0;
#pragma unroll
                for (int j = u; j < u + UB; ++j) {
                    const size_t o = ((size_t)n * nb + j) * 32 + lane;
                    S1 += P1[o];
                    if constexpr (TYPE == T_Q4_K) S2 += P2[o];
                }
                BlockW<TYPE> bw;
                bw.template load<false>(Ws, lane, u);
                const float p = bw.finish(S1, S2, s.d[(size_t)n * nb + u]);
                acc = u == 0 ? p : __fadd_rn(acc, p);
            }
        }
        if (row < W.N) epilogue_store<EPI>(g, row, n, acc);
    }
}

}  // namespace mgb
