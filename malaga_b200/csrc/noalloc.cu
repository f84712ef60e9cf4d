// Allocation-free greedy token choice over logits already in device memory.
//
// This is a variant of the two-pass argmax of the engine's LM head (the fused
// matmul kernels, small_mm_kernel / gemm_tc_kernel with EPI_ARGMAX, write
// per-CTA (value, index) partials to buffers the context allocated, and
// greedy_finalize_kernel merges them). Here the partials live in a file-scope
// __device__ array instead, so the entry point never calls cudaMalloc /
// cudaFree.
//
// Who needs it: callers that must not allocate device memory at this point --
// code running while another framework's stream capture is active (an
// allocation there either fails or is baked into the graph), hosts whose
// caching allocator has already reserved the GPU's memory (candle, PyTorch),
// and latency-critical serving loops that forbid allocation after start-up.
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <mutex>

#include "../../include/malaga_b200.h"
#include "numerics.cuh"

namespace {

constexpr int kMaxRows = 64;    // rows per call
constexpr int kParts = 256;     // first-pass CTAs per row
constexpr int kMaxDevices = 64;

// Scratch: one (value, index) partial per (row, first-pass CTA). 64 x 256 x 8 B
// = 128 KiB on every GPU that loads the library, held until the process exits.
// Every slot a call reads is written by the same call first; nothing needs
// zeroing. All calls share it, so calls that overlap on the GPU race.
struct Partial {
    float v;
    uint32_t i;
};
static __device__ __align__(256) Partial g_argmax_scratch[kMaxRows * kParts];

std::mutex g_mu;
Partial *g_scratch_ptr[kMaxDevices] = {};

__global__ void __launch_bounds__(256) argmax_partial_noalloc(const float *logits, uint32_t vocab, Partial *part) {
    const int row = blockIdx.y, p = blockIdx.x;
    const uint32_t chunk = (vocab + kParts - 1) / kParts;
    const uint32_t begin = p * chunk, end = min(begin + chunk, vocab);
    const float *x = logits + (size_t)row * vocab;
    float best = kNegInf;
    uint32_t bi = 0xffffffffu;
    for (uint32_t i = begin + threadIdx.x; i < end; i += blockDim.x) mgb::argmax_merge(best, bi, x[i], i);
    mgb::warp_argmax(best, bi);
    __shared__ float sv[8];
    __shared__ uint32_t si[8];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) {
        sv[w] = best;
        si[w] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < 8; ++k) mgb::argmax_merge(best, bi, sv[k], si[k]);
        part[row * kParts + p] = Partial{best, bi};
    }
}

__global__ void argmax_final_noalloc(const Partial *part, uint32_t rows, uint32_t *ids, float *vals) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    for (uint32_t row = w; row < rows; row += blockDim.x >> 5) {
        float best = kNegInf;
        uint32_t bi = 0xffffffffu;
        for (int p = lane; p < kParts; p += 32) mgb::argmax_merge(best, bi, part[row * kParts + p].v, part[row * kParts + p].i);
        mgb::warp_argmax(best, bi);
        if (lane == 0) {
            // NaN logits never win a comparison: a row of only NaNs keeps no
            // index and gets id 0 (value -inf), so the id is always < vocab
            ids[row] = bi == 0xffffffffu ? 0u : bi;
            if (vals) vals[row] = best;
        }
    }
}

}  // namespace

// Sets the text mgb_last_error() returns (defined in engine.cu).
void mgb_internal_set_error(const char *msg);

static mgb_status fail(mgb_status s, const char *msg) {
    mgb_internal_set_error(msg);
    return s;
}

extern "C" MGB_API mgb_status mgb_argmax_noalloc(const float *logits, uint32_t rows, uint32_t vocab, uint32_t *ids,
                                                float *vals, void *stream) {
    if (!logits || !ids) return fail(MGB_ERR_INVALID, "mgb_argmax_noalloc: null pointer");
    if (rows == 0 || vocab == 0) return fail(MGB_ERR_INVALID, "mgb_argmax_noalloc: empty input");
    if (rows > (uint32_t)kMaxRows) {
        char buf[160];
        snprintf(buf, sizeof buf, "mgb_argmax_noalloc: %u rows exceeds the static scratch limit of %d rows", rows,
                 kMaxRows);
        return fail(MGB_ERR_INVALID, buf);
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return fail(MGB_ERR_CUDA, "mgb_argmax_noalloc: no current CUDA device");
    Partial *scratch;
    {
        // Set-up, once per device with that device current: the device address
        // of the scratch array (its host-side name is not a device address).
        std::lock_guard<std::mutex> lock(g_mu);
        if (!g_scratch_ptr[dev]) {
            void *p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_argmax_scratch);
            if (e != cudaSuccess) {
                cudaGetLastError();
                return fail(MGB_ERR_CUDA, "mgb_argmax_noalloc: cudaGetSymbolAddress failed");
            }
            g_scratch_ptr[dev] = static_cast<Partial *>(p);
        }
        scratch = g_scratch_ptr[dev];
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    argmax_partial_noalloc<<<dim3(kParts, rows), 256, 0, s>>>(logits, vocab, scratch);
    argmax_final_noalloc<<<1, 32 * (rows < 32 ? rows : 32), 0, s>>>(scratch, rows, ids, vals);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(MGB_ERR_CUDA, cudaGetErrorString(e));
    return MGB_OK;
}
