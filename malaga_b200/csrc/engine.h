// Internal types of the decode engine (host + device).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

namespace mgb {

enum GgmlType : int { T_F32 = 0, T_F16 = 1, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14 };

// A matmul weight [N rows, K] in the engine's HBM layout.
//
// Rows are stored in groups of 32 ("row-interleaved"): for row group g and
// 32-block j, the 32 rows' data for that block are consecutive slots, slot
// s = (g*nb + j)*32 + (row % 32). A warp whose lane l owns row 32g+l therefore
// reads one contiguous run per block (16 B x 32 lanes for Q4_K quants), and a
// 128-row tensor-core tile is four consecutive groups. N is padded to Np (a
// multiple of 32) with zero rows. Per slot:
//   Q8_0: a = 32 B int8 q                      b = f16 d
//   Q4_K: a = 16 B, byte k = q[k] | q[k+16]<<4  b = per (g, super-block, row) the
//         GGUF 16 B header {f16 d, f16 dmin, 12 packed 6-bit sc/m}
//   Q6_K: a = 16 B, byte k = lo4(q[k]) | lo4(q[k+16])<<4 (q in 0..63)
//         b = 8 B: u32 A byte b bits 2i..2i+1 = hi2(q[4i+b]); u32 B the same for q[16..31]
//         c = 2 B int8 scales of the two 16-value halves; e = per (g, super-block, row) f16 d
//   F32 : a = 32 floats
// Byte counts equal the GGUF block sizes (Q4_K 144 B, Q6_K 210 B per 256 values).
struct Matrix {
    int type = -1;
    int N = 0, Np = 0, K = 0, nb = 0, nsb = 0;
    const uint8_t *a = nullptr;
    const uint8_t *b = nullptr;
    const uint8_t *c = nullptr;
    const uint8_t *e = nullptr;
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

// Quantized activations (q8_1 blocks of 32): produced once per matmul input.
struct QAct {
    int8_t *q = nullptr;   // [rows][K]
    float *d = nullptr;    // [rows][K/32] f16-rounded block scales
    int *s32 = nullptr;    // [rows][K/32] sum of q per block
    int *s16 = nullptr;    // [rows][K/16] sum of q per 16-value half
    int rows = 0, K = 0;
    // Tensor-core layout (rs > 0: rows padded to a multiple of 64), written by
    // qprep_row_kernel for one consuming matrix: tq = int8 tiles in the UMMA
    // K-major layout, trec = per-unit scale records (gemm_tc.cuh).
    uint8_t *tq = nullptr, *trec = nullptr;
    int rs = 0;
};

}  // namespace mgb
