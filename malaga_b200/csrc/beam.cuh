// Beam search on the device (translator.rs:250-358): the per-row log_softmax
// statistics and top-k of the step's logits, the reorder of the self-attention
// caches between steps, and the replication of a sentence's cross K/V to its k
// beam rows. The k*k candidate merge runs on the host, as in the reference.
#pragma once
#include "kernels.cuh"

namespace mgb {

// (value, index) order of the top-k: larger value first, lower index on ties
// (the result of k argmax passes with the lowest-index tie-break).
__device__ __forceinline__ bool topk_before(float v, uint32_t i, float w, uint32_t j) {
    return v > w || (v == w && i < j);
}

// Row streaming of the top-k kernel: a row of logits passes through shared
// memory in chunks of kTopkCh floats, fetched by 1-D bulk copies into a ring of
// kTopkNs stages. A row that does not start on a 16-byte boundary is fetched
// from the boundary below it (the few floats before it belong to the previous
// row), so every slot holds its chunk at offset sh = (row address & 15) / 4.
constexpr int kTopkCh = 4096;                // floats per chunk
constexpr int kTopkNs = 6;                   // ring stages
constexpr int kTopkSlot = kTopkCh + 4;       // a chunk plus the alignment slack
constexpr int kTopkMaxCh = 128;              // rows of up to 128 chunks keep their chunk maxima
constexpr int kTopkThreads = 512;
constexpr int kTopkWarps = kTopkThreads / 32;
constexpr size_t kTopkSmem = ((size_t)kTopkNs * kTopkSlot + 2 * kTopkCh + (size_t)kTopkMaxCh * kTopkWarps) * 4;

// One CTA of 512 threads per row of logits [rows][V]:
//   mx = max_i x_i;  ls = log(SUM32_i exp(x_i - mx));  lp_i = (x_i - mx) - ls
// (model.rs:615-617, candle-nn log_softmax, in the engine's SUM32 order: lane l
// of one warp sums i = l, l+32, ... left to right, then the pairwise tree), and
// the K largest lp_i with their indices in topk order (translator.rs:343-358).
// The row is streamed three times:
//  1. the maximum, and each chunk's maximum;
//  2. exp(x - mx) of chunk c by warps 1-15 into a double buffer while warp 0
//     adds chunk c-1 in its lanes' order (the chains stay strictly sequential);
//  3. the top-K over the chunks that can hold one of them: lp is monotone in x,
//     so with T0 = lp(the K-th largest chunk maximum) every element of the
//     top-K has lp >= T0 and lies in a chunk whose maximum has lp >= T0 (the K
//     largest chunk maxima are K elements >= that maximum). Rows of more than
//     kTopkMaxCh chunks scan every chunk.
// NaN logits are never selected; a row with fewer than K selectable values
// pads with (-inf, 0). A bulk copy that does not land within wait_ns sets
// flag 8 in *err and ends the CTA without output (`withhold`: a test hook, the
// ring position whose copy row 0 never issues; -1 in use).
template <int K>
__global__ void __launch_bounds__(kTopkThreads, 1)
    beam_topk_kernel(const float *logits, int V, float *vals, uint32_t *idx, uint32_t *err, uint64_t wait_ns,
                     int withhold) {
    extern __shared__ __align__(16) float tk_sm[];
    float *ring = tk_sm;                           // [kTopkNs][kTopkSlot]
    float *ebuf = ring + kTopkNs * kTopkSlot;      // [2][kTopkCh] exponentials
    float *wmax = ebuf + 2 * kTopkCh;              // [kTopkMaxCh][warps] chunk maxima per warp
    __shared__ __align__(8) uint64_t full[kTopkNs];
    __shared__ float red[kTopkWarps], cmx[kTopkMaxCh];
    __shared__ float wv[kTopkWarps];
    __shared__ uint32_t wi[kTopkWarps];
    __shared__ int list[kTopkMaxCh];
    __shared__ int nlist;
    __shared__ float stat[2];
    const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float *x = logits + (size_t)r * V;
    const int sh = (int)(((uintptr_t)x & 15) >> 2);
    const float *xa = x - sh;
    const int nch = (V + kTopkCh - 1) / kTopkCh;
    const bool keep = nch <= kTopkMaxCh;
    // ring sequence q: [0, nch) the max pass, [nch, 2 nch) the exp pass, then
    // the top-k pass over its chunk list (issued once the list is known)
    int issued = 0;  // thread 0: copies issued so far
    auto issue = [&](int q, int c) {
        if (r == 0 && q == withhold) return;  // never issued: its wait runs out
        const int n = min(kTopkCh, V - c * kTopkCh) + sh;
        const uint32_t bytes = (uint32_t)((n * 4 + 15) & ~15);
        uint64_t *b = &full[q % kTopkNs];
        mbar_expect_tx(b, bytes);
        bulk_g2s(ring + (q % kTopkNs) * kTopkSlot, xa + (size_t)c * kTopkCh, bytes, b);
        issued = q + 1;
    };
    if (tid == 0) {
        for (int s = 0; s < kTopkNs; ++s) mbar_init(&full[s], 1);
        nlist = 0;
    }
    __syncthreads();
    if (tid == 0)
        for (int q = 0; q < min(kTopkNs, 2 * nch); ++q) issue(q, q < nch ? q : q - nch);
    bool ok = true;
    int q = 0;
    auto fail = [&]() {
        // a copy never landed: report, wait (bounded) for this CTA's copies
        // still in flight, write nothing
        if (tid == 0) {
            atomicOr(err, 8u);
            for (int k = q; k < issued; ++k)
                if (!(r == 0 && k == withhold)) mbar_wait(&full[k % kTopkNs], (uint32_t)((k / kTopkNs) & 1), wait_ns);
        }
    };

    // 1. maxima (order-free)
    float m = kNegInf;
    for (int c = 0; c < nch; ++c, ++q) {
        const bool got = mbar_wait(&full[q % kTopkNs], (uint32_t)((q / kTopkNs) & 1), wait_ns);
        float cm = kNegInf;
        if (got) {
            const float *s = ring + (q % kTopkNs) * kTopkSlot + sh;
            const int n = min(kTopkCh, V - c * kTopkCh);
#pragma unroll 8
            for (int j = tid; j < n; j += kTopkThreads) cm = fmaxf(cm, s[j]);
        }
        cm = warp_max(cm);
        if (keep && lane == 0) wmax[c * kTopkWarps + warp] = cm;
        m = fmaxf(m, cm);
        ok = __syncthreads_and(got);
        if (!ok) return fail();
        if (tid == 0 && q + kTopkNs < 2 * nch) issue(q + kTopkNs, q + kTopkNs < nch ? q + kTopkNs : q + kTopkNs - nch);
    }
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    float mx = red[0];
#pragma unroll
    for (int w = 1; w < kTopkWarps; ++w) mx = fmaxf(mx, red[w]);
    if (keep && tid < nch) {
        float v = wmax[tid * kTopkWarps];
        for (int w = 1; w < kTopkWarps; ++w) v = fmaxf(v, wmax[tid * kTopkWarps + w]);
        cmx[tid] = v;
    }

    // 2. SUM32 of exp(x - mx): warps 1-15 form chunk c's exponentials (zero past
    // the row's end, up to the next multiple of 32) while warp 0 adds chunk c-1
    float acc = 0.0f;  // warp 0: lane's chain (an empty lane sums to +0)
    for (int c = 0; c <= nch; ++c) {
        bool got = true;
        if (warp != 0 && c < nch) {
            got = mbar_wait(&full[q % kTopkNs], (uint32_t)((q / kTopkNs) & 1), wait_ns);
            if (got) {
                const float *s = ring + (q % kTopkNs) * kTopkSlot + sh;
                const int n = min(kTopkCh, V - c * kTopkCh), n32 = (n + 31) & ~31;
                float *e = ebuf + (c & 1) * kTopkCh;
                for (int j = tid - 32; j < n32; j += kTopkThreads - 32)
                    e[j] = j < n ? mgb_exp(__fsub_rn(s[j], mx)) : 0.0f;
            }
        }
        if (warp == 0 && c > 0) {
            const int n = min(kTopkCh, V - (c - 1) * kTopkCh), ng = (n + 31) >> 5;
            const float *e = ebuf + ((c - 1) & 1) * kTopkCh + lane;
            int g = 0;
            for (; g + 16 <= ng; g += 16) {
                float t[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) t[u] = e[(g + u) * 32];
#pragma unroll
                for (int u = 0; u < 16; ++u) acc = __fadd_rn(acc, t[u]);
            }
            for (; g < ng; ++g) acc = __fadd_rn(acc, e[g * 32]);
        }
        ok = __syncthreads_and(got);
        if (!ok) return fail();
        if (c < nch) {
            if (tid == 0 && q + kTopkNs < 2 * nch) issue(q + kTopkNs, q + kTopkNs - nch);
            ++q;
        }
    }
    if (warp == 0) {
        const float total = warp_tree(acc);
        if (lane == 0) stat[1] = mgb_log(total);
    }
    __syncthreads();
    const float ls = stat[1];

    // 3. the chunks that can hold a top-K element
    int nl = nch;
    if (keep) {
        if (tid == 0) stat[0] = kNegInf;
        __syncthreads();
        if (tid < nch) {
            // rank of this chunk's maximum by (value desc, chunk asc); NaN
            // maxima (chunks of NaN only) are not ranked
            const float v = cmx[tid];
            if (v == v) {
                int rank = 0;
                for (int c = 0; c < nch; ++c) {
                    const float w = cmx[c];
                    rank += (w > v || (w == v && c < tid)) ? 1 : 0;
                }
                if (rank == K - 1) stat[0] = __fsub_rn(__fsub_rn(v, mx), ls);
            }
        }
        __syncthreads();
        const float t0 = stat[0];
        if (tid < nch) {
            const float lpm = __fsub_rn(__fsub_rn(cmx[tid], mx), ls);
            if (lpm >= t0) list[atomicAdd(&nlist, 1)] = tid;
        }
        __syncthreads();
        nl = nlist;
    }
    auto chunk_of = [&](int i) { return keep ? list[i] : i; };
    if (tid == 0)
        for (int i = 0; i < min(kTopkNs, nl); ++i) issue(q + i, chunk_of(i));
    float bv[K];
    uint32_t bi[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
        bv[j] = kNegInf;
        bi[j] = 0xffffffffu;
    }
    for (int i = 0; i < nl; ++i, ++q) {
        const bool got = mbar_wait(&full[q % kTopkNs], (uint32_t)((q / kTopkNs) & 1), wait_ns);
        if (got) {
            const int c = chunk_of(i), n = min(kTopkCh, V - c * kTopkCh);
            const float *s = ring + (q % kTopkNs) * kTopkSlot + sh;
            for (int j = tid; j < n; j += kTopkThreads) {
                const float lp = __fsub_rn(__fsub_rn(s[j], mx), ls);
                const uint32_t ix = (uint32_t)(c * kTopkCh + j);
                if (!topk_before(lp, ix, bv[K - 1], bi[K - 1])) continue;
                // insert, keeping the list in topk order
                float v = lp;
                uint32_t iv = ix;
#pragma unroll
                for (int k = 0; k < K; ++k) {
                    if (topk_before(v, iv, bv[k], bi[k])) {
                        const float tv = bv[k];
                        const uint32_t ti = bi[k];
                        bv[k] = v;
                        bi[k] = iv;
                        v = tv;
                        iv = ti;
                    }
                }
            }
        }
        ok = __syncthreads_and(got);
        if (!ok) return fail();
        if (tid == 0 && i + kTopkNs < nl) issue(q + kTopkNs, chunk_of(i + kTopkNs));
    }
    // block top-K: K rounds of the best list head (value desc, index asc); the
    // owner of the winner pops it (indices are unique)
    for (int j = 0; j < K; ++j) {
        float v = bv[0];
        uint32_t iv = bi[0];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, iv, o);
            if (topk_before(ov, oi, v, iv)) {
                v = ov;
                iv = oi;
            }
        }
        if (lane == 0) {
            wv[warp] = v;
            wi[warp] = iv;
        }
        __syncthreads();
        v = wv[0];
        iv = wi[0];
        for (int w = 1; w < kTopkWarps; ++w)
            if (topk_before(wv[w], wi[w], v, iv)) {
                v = wv[w];
                iv = wi[w];
            }
        if (tid == 0) {
            const bool any = iv != 0xffffffffu;
            vals[(size_t)r * K + j] = any ? v : kNegInf;
            idx[(size_t)r * K + j] = any ? iv : 0u;
        }
        if (iv != 0xffffffffu && bi[0] == iv) {
#pragma unroll
            for (int k = 0; k + 1 < K; ++k) {
                bv[k] = bv[k + 1];
                bi[k] = bi[k + 1];
            }
            bv[K - 1] = kNegInf;
            bi[K - 1] = 0xffffffffu;
        }
        __syncthreads();
    }
}

// Self-attention caches [rows][H][m][hd] of every layer gathered by source row
// (DecoderState::reorder, model.rs:209-226): dst[r] = src[from[r]] for the first
// `npos` positions. Caches of up to 64 layers x {K, V}.
struct KvGather {
    const void *src[128];
    void *dst[128];
    int n;  // caches (2 per layer)
};

// Beam reorder (DecoderState::reorder, model.rs:209-226): row r of every cache
// takes the first npos positions of row from[r]; esz = element bytes (2: f16,
// 4: f32), moved as 16-byte words.
__global__ void __launch_bounds__(256) kv_gather_kernel(KvGather g, const int *from, int rows, int H, int m, int hd,
                                                        int npos, int esz) {
    const int wpp = hd * esz / 16;  // words per position
    const int per = npos * wpp;     // words per (row, head)
    const long total = (long)g.n * rows * H * per;
    for (long w = blockIdx.x * (long)blockDim.x + threadIdx.x; w < total; w += (long)gridDim.x * blockDim.x) {
        const int c = (int)(w / ((long)rows * H * per));
        long rem = w % ((long)rows * H * per);
        const int r = (int)(rem / ((long)H * per));
        rem %= (long)H * per;
        const int h = (int)(rem / per), o = (int)(rem % per);
        const size_t src = (((size_t)from[r] * H + h) * m) * wpp + o;
        const size_t dst = (((size_t)r * H + h) * m) * wpp + o;
        reinterpret_cast<uint4 *>(g.dst[c])[dst] = reinterpret_cast<const uint4 *>(g.src[c])[src];
    }
}

// A batch's f32 cross K/V [b][H][S][hd] into a decode state's buffers
// [b*rep][H][s][hd]: every sentence to its rep consecutive rows, as f16 (the
// fused greedy step's copy, graph.rs:95-96) or f32 (beam search's generic
// decode, model.rs:209-226).
__global__ void __launch_bounds__(256) cross_load_kernel(const float *src, void *dst, int to_f16, int rows, int rep,
                                                         int H, int S, int s, int hd) {
    const long total = (long)rows * H * S * hd;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int t = (int)(i % hd);
        long rem = i / hd;
        const int j = (int)(rem % S);
        rem /= S;
        const int h = (int)(rem % H), r = (int)(rem / H);
        const float v = src[(((size_t)(r / rep) * H + h) * S + j) * hd + t];
        const size_t at = (((size_t)r * H + h) * s + j) * hd + t;
        if (to_f16) reinterpret_cast<__half *>(dst)[at] = __float2half_rn(v);
        else reinterpret_cast<float *>(dst)[at] = v;
    }
}

}  // namespace mgb
