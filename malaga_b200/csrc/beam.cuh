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

// One CTA (256 threads) per row of logits [rows][V]:
//   mx = max_i x_i;  ls = log(SUM32_i exp(x_i - mx));  lp_i = (x_i - mx) - ls
// (model.rs:615-617, candle-nn log_softmax, in the engine's SUM32 order: lane l
// of one warp sums i = l, l+32, ... left to right, then the pairwise tree), and
// the K largest lp_i with their indices in topk order.
template <int K>
__global__ void __launch_bounds__(256) beam_topk_kernel(const float *logits, int V, float *vals, uint32_t *idx) {
    __shared__ float red[8];
    __shared__ float stat[2];
    __shared__ float cv[256 * K];
    __shared__ uint32_t ci[256 * K];
    const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float *x = logits + (size_t)r * V;
    // max (order-free)
    float m = kNegInf;
    for (int i = tid; i < V; i += blockDim.x) m = fmaxf(m, x[i]);
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (tid == 0) {
        float mm = red[0];
        for (int w = 1; w < 8; ++w) mm = fmaxf(mm, red[w]);
        stat[0] = mm;
    }
    __syncthreads();
    const float mx = stat[0];
    // SUM32 of exp(x - mx) by warp 0: each lane's chain strictly in order;
    // the exponentials of 8 elements are formed ahead of their adds
    if (warp == 0) {
        float acc = mgb_exp(__fsub_rn(x[lane], mx));
        int i = lane + 32;
        for (; i + 7 * 32 < V; i += 8 * 32) {
            float e[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) e[u] = mgb_exp(__fsub_rn(x[i + 32 * u], mx));
#pragma unroll
            for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, e[u]);
        }
        for (; i < V; i += 32) acc = __fadd_rn(acc, mgb_exp(__fsub_rn(x[i], mx)));
        const float total = warp_tree(acc);
        if (lane == 0) stat[1] = mgb_log(total);
    }
    __syncthreads();
    const float ls = stat[1];
    // per-thread top-K of lp, then the block's top-K from the 256*K candidates
    float bv[K];
    uint32_t bi[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
        bv[j] = kNegInf;
        bi[j] = 0xffffffffu;
    }
    for (int i = tid; i < V; i += blockDim.x) {
        const float lp = __fsub_rn(__fsub_rn(x[i], mx), ls);
        if (!topk_before(lp, (uint32_t)i, bv[K - 1], bi[K - 1])) continue;
        // insert, keeping the list in topk order
        float v = lp;
        uint32_t ix = (uint32_t)i;
#pragma unroll
        for (int j = 0; j < K; ++j) {
            if (topk_before(v, ix, bv[j], bi[j])) {
                const float tv = bv[j];
                const uint32_t ti = bi[j];
                bv[j] = v;
                bi[j] = ix;
                v = tv;
                ix = ti;
            }
        }
    }
#pragma unroll
    for (int j = 0; j < K; ++j) {
        cv[tid * K + j] = bv[j];
        ci[tid * K + j] = bi[j];
    }
    __syncthreads();
    if (tid == 0) {
        // K selection passes over the candidates (each index appears once)
        for (int j = 0; j < K; ++j) {
            int best = -1;
            for (int c = 0; c < 256 * K; ++c) {
                if (ci[c] == 0xffffffffu) continue;
                if (best < 0 || topk_before(cv[c], ci[c], cv[best], ci[best])) best = c;
            }
            vals[(size_t)r * K + j] = best >= 0 ? cv[best] : kNegInf;
            idx[(size_t)r * K + j] = best >= 0 ? ci[best] : 0u;
            if (best >= 0) ci[best] = 0xffffffffu;
        }
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
