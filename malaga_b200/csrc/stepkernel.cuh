// Persistent decoder layers for batches of at most 8 rows (sm_100a): the
// decoder-layer part of the greedy step (model.rs:552-612) in one cooperative
// launch; the LM head and the greedy bookkeeping follow as their own launches.
//
// Up to 8 rows the layers are a chain of ~100 small dependent operations (6
// projections and 2 attentions per layer); launched one kernel each, every
// link pays a grid launch and drain. Here one CTA per SM (8 warps) runs every
// link as a phase of one kernel:
//   * thread 0 feeds the CTA's weight rows of every matmul phase, in phase
//     order, into a ring of shared-memory slots with 1-D bulk copies (TMA): the
//     weights never depend on activations, so the copies run ahead of the
//     computation, across phase boundaries (thread 0 refills the ring while it
//     polls a grid barrier), limited only by free slots;
//   * a matmul phase builds the q8_1 activations of the batch rows in shared
//     memory (LayerNorm / plain input, the same code as the small-batch
//     kernel), then each warp waits for each chunk, computes its rows with the
//     reference's MMVQ arithmetic (smallmm.cuh) and frees the slot on its own;
//     the epilogue's bias and residual values are loaded at the phase start and
//     land while the activations are built;
//   * an attention phase gives one (row, head) to each warp of the grid, with
//     the arithmetic of attend_kernel;
//   * phases are separated by a grid barrier (an arrival counter in global
//     memory, zeroed before each launch; the kernel is launched cooperatively,
//     so all CTAs are resident); while thread 0 polls it, the next phase's
//     descriptor is copied into shared memory. Activations are read through L2
//     (ld.cg): other CTAs wrote them earlier in the launch.
// Every wait (mbarrier or grid barrier) is bounded; a CTA whose wait runs out
// raises an abort flag that every other wait also watches, records the error
// word, waits (bounded) for its own copies in flight and returns, so a failure
// ends the launch instead of hanging it.
#pragma once
#include <type_traits>

#include "smallmm.cuh"

namespace mgb {

enum PhaseKind { PH_MM = 0, PH_ATTN = 1 };

// Most output rows of one matmul phase in one CTA (bias / residual staging).
constexpr int kStepRows = 64;

// One phase of the step. Matmul phases: the matrix, epilogue, activation
// source and outputs; attention phases: queries, K/V caches and the output.
// (16-byte aligned and sized: copied into shared memory 16 bytes at a time.)
struct alignas(16) StepPhase {
    int kind;
    Matrix W;
    int epi, mode;      // Epi (QKV, STORE, RELU, RESID), PrepMode
    int rsel;           // rows per warp per slot: 1 or 4
    const float *x;     // input rows [b][K] (PLAIN / LN)
    const float *gamma, *beta;
    float *y;           // STORE / RELU / RESID output [b][N]
    void *kc, *vc;      // QKV: this layer's K/V caches
    // attention
    const float *aq;    // queries [b][H*hd]
    const void *K, *V;  // [b][H][keys][hd]
    long kv_head, kv_batch;
    int self;           // keys = step + 1 (self) or lens[row] (cross)
    float *aout;        // [b][H*hd]
};

struct StepArgs {
    const StepPhase *ph;   // device array of nph phases
    int nph;
    int rows;              // batch rows
    int H, hd, m, max_keys;
    int kv_f32;
    const uint32_t *lens;
    // layer-0 input (EMBED_LN) and the residual stream
    Matrix embed;
    const uint32_t *ids;
    uint32_t *step;
    const float *pos_table;
    uint32_t pos_base;
    float scale;
    float *x;
    float *q;
    // grid barrier, failure words
    uint32_t *bar;         // arrival counter, zero at launch
    uint32_t *abort_flag;  // zero at launch
    uint32_t *err;
    uint64_t wait_ns;
    int withhold;          // failure-path test hook: CTA 0 never copies this chunk (-1: off)
    // optional phase timing (null: off): 8 words per phase, summed over launches:
    // CTA 0's nanoseconds from the phase start to its inputs staged, statistics,
    // activations, first weight chunk, work done and barrier passed, and the sum
    // over CTAs of their time before the barrier; the last word counts launches
    unsigned long long *trace;
    // shared-memory geometry
    int slots, slot_bytes, act_bytes;
};

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Rows [r0, r1) of an Np-row matrix that CTA `cta` of `grid` computes (groups of 8).
__host__ __device__ __forceinline__ void cta_rows(int Np, int grid, int cta, int &r0, int &r1) {
    const int groups = Np / 8, per = (groups + grid - 1) / grid;
    r0 = min(Np, cta * per * 8);
    r1 = min(Np, r0 + per * 8);
}

// The grid barrier (arrival number `target`): a CTA barrier orders every
// thread's stores before thread 0's release reduction on the counter; thread 0
// then starts `prefetch` (the next phase's descriptor) and polls the counter
// with acquire loads, refilling the weight ring meanwhile (`spin`); a second
// CTA barrier publishes what it acquired to the other threads. A CTA one of
// whose warps failed (`fail_sh`, the abort flag already raised) does not arrive.
template <typename Pre, typename Spin>
__device__ bool grid_barrier(const StepArgs &A, uint32_t target, volatile int *ok_sh, volatile int *fail_sh,
                             Pre &&prefetch, Spin &&spin) {
    __syncthreads();
    if (threadIdx.x == 0) {
        bool ok = !*fail_sh;
        if (ok) asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(A.bar), "r"(1u) : "memory");
        prefetch();
        uint64_t t0 = 0;
        for (int it = 0; ok && ld_acquire_u32(A.bar) < target; ++it) {
            spin();
            if (*(volatile uint32_t *)A.abort_flag) {
                ok = false;
                break;
            }
            if (it == 0) t0 = globaltimer();
            else if (globaltimer() - t0 > A.wait_ns) {
                atomicExch(A.abort_flag, 1u);
                atomicOr(A.err, 4u);
                ok = false;
                break;
            }
        }
        cp_async_wait();
        *ok_sh = ok;
    }
    __syncthreads();
    return *ok_sh;
}

// Single-query attention of (row n, head h) by one warp over `keys` keys, from
// global K/V written earlier in the launch: the arithmetic of attend_one
// (scores by an FMA chain over the head dimension, exp(s - max), lane-ordered
// sums and the pairwise tree, outputs by an FMA chain over keys times 1/sum).
// The query goes through shared memory (broadcast reads); the first round of K
// rows and the first batch of V values are requested together, so that a head
// of at most KR*32 keys and VB values per lane costs one memory round trip.
template <typename KV, int HD>
__device__ void attend_warp(const StepPhase &P, int H, int n, int h, int keys, float *e, float *qs, int lane) {
    constexpr int VEC = 16 / sizeof(KV), RW = HD / VEC;  // 16-byte words per K/V row
    constexpr int KR = 1;  // K rows per lane per round (two spill beside the V batch)
    constexpr int PER = HD / 32, VB = HD == 64 ? 32 : 8;  // V values per lane per key; keys per V batch
    const float *qp = P.aq + (size_t)n * H * HD + h * HD;
    const KV *K = reinterpret_cast<const KV *>(P.K) + n * P.kv_batch + h * P.kv_head;
    const KV *V = reinterpret_cast<const KV *>(P.V) + n * P.kv_batch + h * P.kv_head;
    auto ldv = [&](int j, int c) -> float {
        const KV *vp = V + (size_t)j * HD + lane + 32 * c;
        if constexpr (sizeof(KV) == 2)
            return __half2float(__ushort_as_half(__ldcg(reinterpret_cast<const unsigned short *>(vp))));
        else
            return __ldcg(reinterpret_cast<const float *>(vp));
    };
    float qv[PER];
#pragma unroll
    for (int c = 0; c < PER; ++c) qv[c] = __ldcg(qp + lane + 32 * c);
    uint4 r[KR][RW];
#pragma unroll
    for (int k = 0; k < KR; ++k)
#pragma unroll
        for (int c = 0; c < RW; ++c)
            r[k][c] = lane + 32 * k < keys ? __ldcg(reinterpret_cast<const uint4 *>(K + (size_t)(lane + 32 * k) * HD) + c)
                                           : make_uint4(0, 0, 0, 0);
    float vv[VB][PER];
#pragma unroll
    for (int u = 0; u < VB; ++u)
#pragma unroll
        for (int c = 0; c < PER; ++c) vv[u][c] = u < keys ? ldv(u, c) : 0.0f;
#pragma unroll
    for (int c = 0; c < PER; ++c) qs[lane + 32 * c] = qv[c];
    __syncwarp();
    // scores
    float mx = kNegInf;
    for (int j0 = 0; j0 < keys; j0 += 32 * KR) {
        if (j0 > 0)
#pragma unroll
            for (int k = 0; k < KR; ++k)
#pragma unroll
                for (int c = 0; c < RW; ++c) {
                    const int j = j0 + lane + 32 * k;
                    r[k][c] = j < keys ? __ldcg(reinterpret_cast<const uint4 *>(K + (size_t)j * HD) + c)
                                       : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
        for (int k = 0; k < KR; ++k) {
            float sc = 0.0f;
#pragma unroll
            for (int t = 0; t < HD; ++t) sc = __fmaf_rn(qs[t], kv_at<KV, RW>(r[k], t), sc);
            const int j = j0 + lane + 32 * k;
            if (j < keys) {
                e[j] = sc;
                mx = fmaxf(mx, sc);
            }
        }
    }
    mx = warp_max(mx);
    __syncwarp();
    float sum = 0.0f;
    for (int j = lane; j < keys; j += 32) {
        const float ex = mgb_exp(__fsub_rn(e[j], mx));
        e[j] = ex;
        sum = j == lane ? ex : __fadd_rn(sum, ex);
    }
    const float inv = __fdiv_rn(1.0f, warp_tree(sum));
    __syncwarp();
    // outputs: lane owns dims lane + 32c, an FMA chain over the keys in order
    float acc[PER];
#pragma unroll
    for (int c = 0; c < PER; ++c) acc[c] = 0.0f;
    for (int j0 = 0; j0 < keys; j0 += VB) {
        if (j0 > 0)
#pragma unroll
            for (int u = 0; u < VB; ++u)
#pragma unroll
                for (int c = 0; c < PER; ++c) vv[u][c] = j0 + u < keys ? ldv(j0 + u, c) : 0.0f;
#pragma unroll
        for (int u = 0; u < VB; ++u) {  // predicated, not a loop exit: the batch stays unrolled
            const bool in = j0 + u < keys;
            const float ej = in ? e[j0 + u] : 0.0f;
#pragma unroll
            for (int c = 0; c < PER; ++c) acc[c] = in ? __fmaf_rn(ej, vv[u][c], acc[c]) : acc[c];
        }
    }
    float *o = P.aout + (size_t)n * H * HD + h * HD;
#pragma unroll
    for (int c = 0; c < PER; ++c) o[lane + 32 * c] = __fmul_rn(acc[c], inv);
    __syncwarp();
}

// Thread 0's weight feed: this CTA's chunks of every matmul phase, in phase
// order, into the ring of shared-memory slots (chunk k in slot k % slots).
// fill() issues while the next chunk's slot is free and never waits: thread 0
// calls it while it polls a grid barrier (not inside a phase, where it would
// hold up its warp); ensure(k) issues up to chunk k and may wait (bounded) for
// a slot, which only needs warps to finish chunks that were issued already.
struct Feed {
    int pi, c0, r1, n;  // next chunk: rows [c0, ...) of phase pi; chunks issued

    __device__ void advance(const StepArgs &A) {  // to the next matmul phase with rows in this CTA
        while (++pi < A.nph) {
            const StepPhase &P = A.ph[pi];
            if (P.kind != PH_MM) continue;
            int r0;
            cta_rows(P.W.Np, gridDim.x, blockIdx.x, r0, r1);
            if (r0 < r1) {
                c0 = r0;
                return;
            }
        }
    }
    __device__ void start(const StepArgs &A) {
        pi = -1;
        n = c0 = r1 = 0;
        advance(A);
    }
    __device__ void issue(const StepArgs &A, uint8_t *ring, uint64_t *full) {
        const Matrix &W = A.ph[pi].W;
        int rb[4];
        row_regions(W.type, W.K, rb);
        const int RB = rb[0] + rb[1] + rb[2] + rb[3], CR = 8 * A.ph[pi].rsel, cr = min(CR, r1 - c0);
        const int slot = n % A.slots;
        const uint8_t *src[4] = {W.ra, W.rb, W.rc, W.re};
        const bool withheld = blockIdx.x == 0 && n == A.withhold;
        if (!withheld) mbar_expect_tx(&full[slot], (uint32_t)(cr * RB));
        uint8_t *dst = ring + (size_t)slot * A.slot_bytes;
        for (int k = 0; k < 4 && !withheld; ++k) {
            if (!rb[k]) continue;
            bulk_g2s(dst, src[k] + (size_t)c0 * rb[k], (uint32_t)(cr * rb[k]), &full[slot]);
            dst += (size_t)CR * rb[k];
        }
        ++n;
        c0 += CR;
        if (c0 >= r1) advance(A);
    }
    __device__ void fill(const StepArgs &A, uint8_t *ring, uint64_t *full, uint64_t *empty) {
        while (pi < A.nph) {
            if (n >= A.slots && !mbar_try(smem_u32(&empty[n % A.slots]), (uint32_t)(((n / A.slots) - 1) & 1))) return;
            issue(A, ring, full);
        }
    }
    __device__ bool ensure(const StepArgs &A, int k, uint8_t *ring, uint64_t *full, uint64_t *empty) {
        while (n <= k && pi < A.nph) {
            if (n >= A.slots && !mbar_wait(&empty[n % A.slots], (uint32_t)(((n / A.slots) - 1) & 1), A.wait_ns))
                return false;
            issue(A, ring, full);
        }
        return true;
    }
    // after a failure: wait (bounded) for the copies that may still be in flight
    // (chunk k was issued only once chunk k - slots was consumed, so at most the
    // last `slots` chunks are outstanding)
    __device__ void drain(const StepArgs &A, uint64_t *full) {
        for (int k = max(0, n - A.slots); k < n; ++k)
            mbar_wait(&full[k % A.slots], (uint32_t)((k / A.slots) & 1), A.wait_ns);
    }
};

template <int HD>
__device__ void attend_phase(const StepArgs &A, const StepPhase &P, int step, const int *lens, float *e, float *qs,
                             int lane, int gwarp, int nwarps) {
    for (int t = gwarp; t < A.rows * A.H; t += nwarps) {
        const int n = t / A.H, h = t % A.H;
        const int keys = P.self ? step + 1 : lens[n];
        if (A.kv_f32) attend_warp<float, HD>(P, A.H, n, h, keys, e, qs, lane);
        else attend_warp<__half, HD>(P, A.H, n, h, keys, e, qs, lane);
    }
}

// Thread 0: the 16-byte words of descriptor `src` into shared `dst` (cp.async).
__device__ __forceinline__ void copy_phase(void *dst, const StepPhase *src) {
    for (int k = 0; k < (int)(sizeof(StepPhase) / 16); ++k)
        cp_async16(reinterpret_cast<uint8_t *>(dst) + 16 * k, reinterpret_cast<const uint8_t *>(src) + 16 * k);
    cp_async_commit();
}

template <int NC, int NW>
__global__ void __launch_bounds__(256, 1) step_kernel(const __grid_constant__ StepArgs A) {
    extern __shared__ __align__(16) uint8_t sm_raw[];
    __shared__ __align__(8) uint64_t full[8], empty[8];
    __shared__ __align__(16) uint8_t ph_raw[sizeof(StepPhase)];  // the current phase's descriptor
    __shared__ volatile int ok_sh, fail_sh;
    __shared__ int lens_sh[8];
    __shared__ float qsh[8][128];             // attention: each warp's query
    __shared__ float epi_b[kStepRows];        // this CTA's bias values of the phase
    __shared__ float epi_x[NC][kStepRows];    // and residual values
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int S = A.slots;
    uint8_t *ring = sm_raw;
    uint8_t *act = sm_raw + (size_t)S * A.slot_bytes;
    float *escr = reinterpret_cast<float *>(act + A.act_bytes);  // attention scores, per warp max_keys
    const StepPhase &P = *reinterpret_cast<const StepPhase *>(ph_raw);
    Feed feed;
    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 8);  // one arrival per warp
        }
        fail_sh = 0;
        feed.start(A);
        feed.fill(A, ring, full, empty);
        copy_phase(ph_raw, A.ph);
        cp_async_wait();
    }
    if (tid < A.rows) lens_sh[tid] = (int)__ldg(A.lens + tid);
    __syncthreads();
    auto refill = [&] { feed.fill(A, ring, full, empty); };

    const int gwarp = blockIdx.x * 8 + warp, nwarps = gridDim.x * 8;
    float *e = escr + (size_t)warp * A.max_keys;
    const int step = (int)__ldcg(A.step);  // advanced only after this launch
    int n = 0;  // chunks consumed
    uint32_t target = 0;
    bool ok = true;
    // phase timing (CTA 0, thread 0): m[0] phase start, m[1..3] prologue marks
    // (inputs staged, statistics, activations), m[4] first chunk arrived,
    // m[5] work done, m[6] barrier passed
    const bool tr = A.trace && tid == 0;
    uint64_t m[7];
    auto mark = [&](int k) {
        if (tr) m[k] = globaltimer();
    };
    for (int pi = 0; pi < A.nph && ok; ++pi) {
        if (tr) {
            m[0] = globaltimer();
            for (int k = 1; k < 5; ++k) m[k] = m[0];
        }
        if (P.kind == PH_ATTN) {
            if (A.hd == 64) attend_phase<64>(A, P, step, lens_sh, e, qsh[warp], lane, gwarp, nwarps);
            else attend_phase<128>(A, P, step, lens_sh, e, qsh[warp], lane, gwarp, nwarps);
        } else {
            const Matrix &W = P.W;
            const int K = W.K, epi = P.epi;
            int r0, r1;
            cta_rows(W.Np, gridDim.x, blockIdx.x, r0, r1);
            const int nr = max(0, min(r1, W.N) - r0);  // this CTA's output rows (at most kStepRows)
            // the epilogue's bias and residual values: requested now, stored after
            // the activations are built
            float pre_b = 0.0f, pre_x[2] = {0.0f, 0.0f};
            if (W.bias && tid < nr) pre_b = __ldg(W.bias + r0 + tid);
            if (epi == EPI_RESID)
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int i = tid + 256 * u;
                    if (i < A.rows * nr) pre_x[u] = __ldcg(P.y + (size_t)(i / nr) * W.N + r0 + i % nr);
                }
            PrepArgs p{};
            p.x = P.x;
            p.x_out = A.x;
            p.gamma = P.gamma;
            p.beta = P.beta;
            p.embed = A.embed;
            p.ids = A.ids;
            p.step = A.step;
            p.pos_table = A.pos_table;
            p.pos_base = A.pos_base;
            p.scale = A.scale;
            p.rows = A.rows;
            p.K = K;
            SmAct s;
            s.q = reinterpret_cast<int8_t *>(act);
            s.d = reinterpret_cast<float *>(act + (size_t)NC * K);
            s.xf = nullptr;
            uint8_t *lnbuf = act + (size_t)NC * K + (size_t)NC * (K / 32) * 4;
            const CtaSync sync{0, 0};
            if (P.mode == PREP_EMBED_LN)
                small_prologue<PREP_EMBED_LN, false>(p, 0, s, NC, lnbuf, blockIdx.x == 0, 256, sync, mark);
            else if (P.mode == PREP_LN) small_prologue<PREP_LN, false>(p, 0, s, NC, lnbuf, false, 256, sync, mark);
            else small_prologue<PREP_PLAIN, false>(p, 0, s, NC, lnbuf, false, 256, sync, mark);
            if (tid < nr) epi_b[tid] = pre_b;
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int i = tid + 256 * u;
                if (i < A.rows * nr) epi_x[i / nr][i % nr] = pre_x[u];
            }
            __syncthreads();
            const int dm = A.H * A.hd;
            auto store = [&](int row, int c, float v) {  // epilogue_store's arithmetic, staged operands
                const int j = row - r0;
                const float b = W.bias ? epi_b[j] : 0.0f;
                if (epi == EPI_STORE) {
                    P.y[(size_t)c * W.N + row] = W.bias ? __fadd_rn(v, b) : v;
                } else if (epi == EPI_RELU) {
                    const float y = __fadd_rn(v, b);
                    P.y[(size_t)c * W.N + row] = y > 0.0f ? y : 0.0f;
                } else if (epi == EPI_RESID) {
                    P.y[(size_t)c * W.N + row] = __fadd_rn(__fadd_rn(v, b), epi_x[c][j]);
                } else {  // EPI_QKV
                    const float y = __fadd_rn(v, b);
                    if (row < dm) {
                        A.q[(size_t)c * dm + row] = y;
                    } else {
                        const int cc = row - dm, which = cc / dm, h = (cc % dm) / A.hd, t = cc % A.hd;
                        const size_t at = (((size_t)c * A.H + h) * A.m + step) * A.hd + t;
                        void *cache = which == 0 ? P.kc : P.vc;
                        if (A.kv_f32) reinterpret_cast<float *>(cache)[at] = y;
                        else reinterpret_cast<__half *>(cache)[at] = __float2half_rn(y);
                    }
                }
            };
            int rb[4];
            row_regions(W.type, K, rb);
            const int CR = 8 * P.rsel;
            for (int c0 = r0; c0 < r1; c0 += CR, ++n) {
                // each warp waits for the chunk and frees it on its own (no CTA barrier)
                const int slot = n % S, cr = min(CR, r1 - c0);
                const bool fed = tid != 0 || feed.ensure(A, n, ring, full, empty);
                const bool got = fed && mbar_wait(&full[slot], (uint32_t)((n / S) & 1), A.wait_ns);
                if (c0 == r0) mark(4);
                if (!got) {
                    if (lane == 0) {
                        atomicExch(A.abort_flag, 1u);
                        atomicOr(A.err, 2u);
                        fail_sh = 1;
                    }
                    ok = false;
                    break;
                }
                StageRows St;
                {
                    const uint8_t *st = ring + (size_t)slot * A.slot_bytes;
                    size_t off = 0;
                    for (int k = 0; k < 4; ++k) {
                        St.base[k] = st + off;
                        St.rb[k] = rb[k];
                        off += (size_t)CR * rb[k];
                    }
                }
                auto rows_out = [&](auto rc) {
                    constexpr int R = decltype(rc)::value;
                    float out[R][NC];
                    if (W.type == T_Q6_K) mmvq_q6k<NC, NW, R>(St, warp, W.nsb, s, K, lane, out);
                    else if (W.type == T_Q4_K) mmvq_q4k<NC, NW, R>(St, warp, W.nsb, s, K, lane, out);
                    else mmvq_q80<NC, NW, R>(St, warp, W.nb, s, K, lane, out);
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const int lr = warp + 8 * r, row = c0 + lr;
                        if (lr >= cr || row >= W.N) continue;
#pragma unroll
                        for (int c = 0; c < NC; ++c)
                            if (c == lane && c < A.rows) store(row, c, out[r][c]);  // lane c: column c
                    }
                };
                if (P.rsel == 4) rows_out(std::integral_constant<int, 4>{});
                else rows_out(std::integral_constant<int, 1>{});
                __syncwarp();
                if (lane == 0) mbar_arrive_cta(&empty[slot]);  // this warp is done with the slot
            }
        }
        target += gridDim.x;
        mark(5);
        if (tr) atomicAdd(A.trace + 8 * pi + 6, (unsigned long long)(m[5] - m[0]));
        // (no barrier after the last phase: the launch's end is one)
        if (pi + 1 < A.nph &&
            !grid_barrier(A, target, &ok_sh, &fail_sh, [&] { copy_phase(ph_raw, A.ph + pi + 1); }, refill))
            ok = false;
        mark(6);
        if (tr && blockIdx.x == 0)
            for (int k = 0; k < 6; ++k) A.trace[8 * pi + k] += m[k + 1] - m[k];
    }
    if (tr && blockIdx.x == 0) A.trace[8 * A.nph] += 1;
    if (!ok && tid == 0) feed.drain(A, full);
}

}  // namespace mgb
