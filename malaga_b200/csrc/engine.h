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
// Blocks of 32 values are stored in "lane order": with nb = K/32 blocks and
// G = max(1, nb/32) blocks per lane, block j = l*G + t of a row sits at
// position t*32 + l (nb <= 32: position j). A warp reading iteration t of a
// row therefore touches 32 consecutive block slots: fully coalesced.
//   Q8_0: qs  [N][nb][32] int8           d   [N][nb] f16
//   Q4_K: qs  [N][nb][16]  byte k = q[k] | q[k+16] << 4 (q in 0..15)
//         hdr [N][K/256][16] = {f16 d, f16 dmin, 12 packed 6-bit sc/m} (GGUF)
//   Q6_K: ql  [N][nb][16]  byte k = lo4(q[k]) | lo4(q[k+16]) << 4 (q in 0..63)
//         qh  [N][nb][8]   u32 A: byte b bits 2i..2i+1 = hi2(q[4i+b]); u32 B: same for q[16..31]
//         sc  [N][nb][2]   int8 scales of the two 16-value halves
//         d   [N][K/256] f16
//   F32 : w   [N][K] f32 (natural order)
// Byte counts equal the GGUF block sizes (Q4_K 144 B, Q6_K 210 B per 256).
struct Matrix {
    int type = -1;
    int N = 0, K = 0, nb = 0, G = 1;
    const uint8_t *a = nullptr;  // qs / ql / w
    const uint8_t *b = nullptr;  // d / hdr / qh
    const uint8_t *c = nullptr;  // Q6_K sc
    const uint8_t *e = nullptr;  // Q6_K d
    const float *bias = nullptr;
    size_t bytes = 0;  // HBM bytes of the weight (algorithmic bytes of one pass)
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
};

}  // namespace mgb
