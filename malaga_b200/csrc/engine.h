// Internal types of the decode engine (host + device).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

namespace mgb {

enum GgmlType : int { T_F32 = 0, T_F16 = 1, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14 };

// A matmul weight [N rows, K], held in two HBM layouts.
//
// Tensor-core layout (a, b, c, e; gemm_tc.cuh): rows stored in groups of 32
// ("row-interleaved"): for row group g and 32-block j, the 32 rows' data for
// that block are consecutive slots, slot s = (g*nb + j)*32 + (row % 32), so a
// 128-row tile is four consecutive groups that TMA boxes fetch per region. N is
// padded to Np (a multiple of 128) with zero rows. Per slot:
//   Q8_0: a = 32 B int8 q                      b = f16 d
//   Q4_K: a = 16 B, byte k = q[k] | q[k+16]<<4  b = per (g, super-block, row) the
//         GGUF 16 B header {f16 d, f16 dmin, 12 packed 6-bit sc/m}
//   Q6_K: a = 16 B, byte k = lo4(q[k]) | lo4(q[k+16])<<4 (q in 0..63)
//         b = 8 B: u32 A byte b bits 2i..2i+1 = hi2(q[4i+b]); u32 B the same for q[16..31]
//         c = 2 B int8 scales of the two 16-value halves; e = per (g, super-block, row) f16 d
//
// Row layout (ra, rb, rc, re; smallmm.cuh): every row's GGUF bytes
// contiguous, split into 4-byte-aligned regions (rows 0..Np-1, zero padded):
//   Q8_0: ra = [Np][nb][32] int8 q        rb = [Np][nb] f16 d
//   Q4_K: ra = [Np][nsb] GGUF super-blocks (144 B) as written
//   Q6_K: ra = [Np][nsb][128] ql   rb = [Np][nsb][64] qh   rc = [Np][nsb][16] scales   re = [Np][nsb] f16 d
//   F32 : ra = [Np][K] floats (the tensor-core pointers are unused)
// Byte counts of either layout equal the GGUF sizes (Q4_K 144 B, Q6_K 210 B
// per 256 values), so one pass over a matrix reads its GGUF bytes.
struct Matrix {
    int type = -1;
    int N = 0, Np = 0, K = 0, nb = 0, nsb = 0;
    const uint8_t *a = nullptr;
    const uint8_t *b = nullptr;
    const uint8_t *c = nullptr;
    const uint8_t *e = nullptr;
    const uint8_t *ra = nullptr;
    const uint8_t *rb = nullptr;
    const uint8_t *rc = nullptr;
    const uint8_t *re = nullptr;
    const float *bias = nullptr;
    size_t bytes = 0;  // GGUF bytes of the weight (algorithmic bytes of one pass)
};

struct Norm {
    const float *g = nullptr, *b = nullptr;
};

struct DecLayer {
    Norm attn_norm, cross_norm, ffn_norm;
    Matrix qkv, out, cq, ckv, co, up, down;
};

struct EncLayer {
    Norm attn_norm, ffn_norm;
    Matrix qkv, out, up, down;
};

struct Config {
    int V = 0, d = 0, enc_layers = 0, dec_layers = 0, enc_heads = 0, dec_heads = 0, enc_ffn = 0, dec_ffn = 0;
    int max_pos = 0, scale_embedding = 1, pad = 1, eos = 2, start = 2, bos = 0, max_length = 200;
};

// q8_1 activations of a tensor-core matmul (gemm_tc.cuh): tq = int8 tiles in
// the UMMA K-major layout, trec = per (block, row) float2 {d, s} (the block's
// f16 scale and f16 input sum, as floats); rows padded to rs (a multiple of 64).
struct QAct {
    uint8_t *tq = nullptr;
    float2 *trec = nullptr;
    int rs = 0;
};

}  // namespace mgb
