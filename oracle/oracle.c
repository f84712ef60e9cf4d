/*
 * CPU ORACLE for the NLLB decoder token loop — TEST INFRASTRUCTURE ONLY.
 *
 * This file is the checker the CUDA path is compared against. Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it; the
 * product (malaga_b200/) never links, imports or calls it.
 *
 * It restates the reference's decoding algorithm in plain C:
 *   - model math: crates/malaga-core/src/model.rs:87-189 (pre-LN layers, ReLU
 *     FFN, fused QKV with the 1/sqrt(hd) factor folded in at conversion),
 *     model.rs:325-340 (fairseq sinusoidal table, f64 then f32, pad row 0),
 *     model.rs:455-458/517-519 (positions = index + pad + 1, scaled
 *     embedding), model.rs:480-500 (right padding + key mask),
 *     model.rs:463-477 (encoder + per-layer cross K/V).
 *   - the fused greedy step: model.rs:552-612 and kernels/malaga.cu:89-326
 *     (f16 self/cross K/V, bias+residual+LayerNorm, lowest-index argmax,
 *     pad-after-finish bookkeeping), driven as graph.rs:262-297 does (step 0
 *     consumes </s> and is discarded, the target-language token is forced).
 *   - beam search: translator.rs:250-335 and topk 343-358.
 *   - quantized matmuls: candle-core 0.11.0's CUDA QMatMul (not in the
 *     reference tree; kernels in candle-kernels 0.11.0 src/quantized.cu):
 *     q8_1 activations, MMVQ for at most 8 rows, MMQ above, restated
 *     operation by operation in the section "Activation quantization and the
 *     quantized matmul" below.
 *
 * Outside the matmuls the reference's kernels are built with --use_fast_math
 * (rsqrtf, __expf, approximate division), whose hardware results cannot be
 * restated on a CPU; there this oracle FIXES one IEEE order for every float
 * reduction, and the CUDA kernels follow the same order, so the two agree bit
 * for bit:
 *   SUM32(v[0..n))  lane l (0..31) sums v[l], v[l+32], ... left to right
 *                   (empty lane = 0), then pairs are added at distances
 *                   1,2,4,8,16 (acc[l] + acc[l^o]); the result is acc[0].
 *   exp             own implementation (Cody-Waite reduction with a 2-term
 *                   ln2 split, degree-7 Taylor polynomial in fmaf, exact 2^k
 *                   scaling); see mgb_exp.
 *   FMA             only where written as fmaf(); compiled with
 *                   -ffp-contract=off so nothing else is fused.
 * Parity is pinned by tests/ against gguf-py's dequantizer (block layouts)
 * and Hugging Face transformers' M2M100 (f32 model semantics, tiny model);
 * the quantized matmul arithmetic itself is unpinned (candle cannot be built
 * here).
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* f16 <-> f32 (IEEE binary16, round to nearest even)                        */

static float h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu, x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {
            int sh = 0;
            while (!(m & 0x400u)) { m <<= 1; ++sh; }
            x = sign | ((uint32_t)(113 - sh) << 23) | ((m & 0x3ffu) << 13);
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

static uint16_t f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u, a = x & 0x7fffffffu;
    if (a >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (a > 0x7f800000u ? 0x200u : 0));
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
    if (a < 0x38800000u) {
        if (a < 0x33000000u) return (uint16_t)sign;
        uint32_t e = a >> 23, m = (a & 0x7fffffu) | 0x800000u, sh = 126 - e;
        uint32_t r = m >> sh, rem = m & ((1u << sh) - 1), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (r & 1))) ++r;
        return (uint16_t)(sign | r);
    }
    uint32_t h = (a - 0x38000000u) >> 13, rem = a & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) ++h;
    return (uint16_t)(sign | h);
}

static inline float rnd_h(float f) { return h2f(f2h(f)); }

/* ------------------------------------------------------------------------ */
/* exp: x = k*ln2 + r, |r| <= ln2/2, e^r by Taylor series to degree 7.        */

static float mgb_exp(float x) {
    if (!(x > -104.0f)) return 0.0f; /* also -inf */
    if (x > 88.7f) return INFINITY;
    const float k = rintf(x * 1.44269502162933350f);
    float r = fmaf(-k, 0.693145751953125f, x);
    r = fmaf(-k, 1.428606765330187e-06f, r);
    float p = 1.98412701138295233e-04f;
    p = fmaf(p, r, 1.38888892251998186e-03f);
    p = fmaf(p, r, 8.33333376795053482e-03f);
    p = fmaf(p, r, 4.16666679084300995e-02f);
    p = fmaf(p, r, 1.66666671633720398e-01f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ki = (int)k;
    if (ki >= -126) {
        uint32_t b = (uint32_t)(ki + 127) << 23;
        float s;
        memcpy(&s, &b, 4);
        return p * s;
    }
    uint32_t b1 = (uint32_t)(ki + 100 + 127) << 23, b2 = (uint32_t)(-100 + 127) << 23;
    float s1, s2;
    memcpy(&s1, &b1, 4);
    memcpy(&s2, &b2, 4);
    return (p * s1) * s2;
}

ORC_EXPORT float orc_exp(float x) { return mgb_exp(x); }

/* SUM32 over v[0..n) with stride `st` between elements. */
static float sum32(const float *v, int n, int st) {
    float a[32];
    for (int l = 0; l < 32; ++l) {
        if (l < n) {
            float acc = v[(size_t)l * st];
            for (int j = l + 32; j < n; j += 32) acc = acc + v[(size_t)j * st];
            a[l] = acc;
        } else {
            a[l] = 0.0f;
        }
    }
    for (int o = 1; o < 32; o <<= 1) {
        float b[32];
        for (int l = 0; l < 32; ++l) b[l] = a[l] + a[l ^ o];
        memcpy(a, b, sizeof a);
    }
    return a[0];
}


/* ------------------------------------------------------------------------ */
/* GGUF reading                                                              */

enum { GT_F32 = 0, GT_F16 = 1, GT_Q8_0 = 8, GT_Q4_K = 12, GT_Q6_K = 14 };

typedef struct {
    char name[96];
    int type;
    long rows, cols; /* cols = innermost (row length) */
    const uint8_t *data;
} tensor_t;

typedef struct {
    int V, d, enc_layers, dec_layers, enc_heads, dec_heads, enc_ffn, dec_ffn, max_pos;
    int scale_embedding, pad, eos, start, max_length;
} cfg_t;

typedef struct {
    const tensor_t *w;
    const float *b;
} linear_t;

typedef struct {
    const float *g, *b;
} norm_t;

typedef struct {
    norm_t attn_norm, cross_norm, ffn_norm;
    linear_t qkv, out, cq, ckv, co, up, down;
} layer_t;

typedef struct orc_model {
    cfg_t c;
    uint8_t *file;
    size_t file_size;
    int nt;
    tensor_t *t;
    const tensor_t *embed;
    layer_t *enc, *dec;
    norm_t enc_norm, dec_norm;
    float *pos; /* [max_pos + pad + 1, d] */
    float embed_scale;
    char err[256];
} orc_model;

static uint64_t rd64(const uint8_t **p) { uint64_t v; memcpy(&v, *p, 8); *p += 8; return v; }
static uint32_t rd32(const uint8_t **p) { uint32_t v; memcpy(&v, *p, 4); *p += 4; return v; }

static void skip_value(const uint8_t **p, uint32_t t) {
    static const int sz[] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (t == 8) { uint64_t n = rd64(p); *p += n; return; }
    if (t == 9) {
        uint32_t et = rd32(p);
        uint64_t n = rd64(p);
        for (uint64_t i = 0; i < n; ++i) skip_value(p, et);
        return;
    }
    *p += sz[t];
}

static long type_row_bytes(int t, long n) {
    switch (t) {
        case GT_F32: return 4 * n;
        case GT_F16: return 2 * n;
        case GT_Q8_0: return n / 32 * 34;
        case GT_Q4_K: return n / 256 * 144;
        case GT_Q6_K: return n / 256 * 210;
    }
    return -1;
}

static const tensor_t *find(orc_model *m, const char *name) {
    for (int i = 0; i < m->nt; ++i)
        if (!strcmp(m->t[i].name, name)) return &m->t[i];
    return NULL;
}

static const float *dense(orc_model *m, const char *name) {
    const tensor_t *t = find(m, name);
    if (!t || t->type != GT_F32) return NULL;
    return (const float *)t->data;
}

ORC_EXPORT void orc_free(orc_model *m);

/* Dequantized value j of row r (exact: every product below is exactly representable). */
static float deq(const tensor_t *t, long r, long j) {
    const uint8_t *row = t->data + (size_t)r * type_row_bytes(t->type, t->cols);
    switch (t->type) {
        case GT_F32: return ((const float *)row)[j];
        case GT_F16: { uint16_t h; memcpy(&h, row + 2 * j, 2); return h2f(h); }
        case GT_Q8_0: {
            const uint8_t *b = row + (j / 32) * 34;
            uint16_t h; memcpy(&h, b, 2);
            return h2f(h) * (float)(int8_t)b[2 + j % 32];
        }
        case GT_Q4_K: {
            const uint8_t *b = row + (j / 256) * 144;
            uint16_t hd, hm; memcpy(&hd, b, 2); memcpy(&hm, b + 2, 2);
            int i = (int)(j % 256), sb = i / 32, sc, mn;
            const uint8_t *s = b + 4;
            if (sb < 4) { sc = s[sb] & 63; mn = s[sb + 4] & 63; }
            else { sc = (s[sb + 4] & 0xf) | ((s[sb - 4] >> 6) << 4); mn = (s[sb + 4] >> 4) | ((s[sb] >> 6) << 4); }
            int c = i / 64, l = i % 32, hi = (i % 64) >= 32;
            int q = hi ? (b[16 + 32 * c + l] >> 4) : (b[16 + 32 * c + l] & 0xf);
            return (h2f(hd) * (float)sc) * (float)q - h2f(hm) * (float)mn;
        }
        case GT_Q6_K: {
            const uint8_t *b = row + (j / 256) * 210;
            int i = (int)(j % 256), n = i / 128, g = (i % 128) / 32, l = i % 32;
            const uint8_t *ql = b + 64 * n, *qh = b + 128 + 32 * n;
            int q;
            switch (g) {
                case 0: q = (ql[l] & 0xf) | (((qh[l] >> 0) & 3) << 4); break;
                case 1: q = (ql[l + 32] & 0xf) | (((qh[l] >> 2) & 3) << 4); break;
                case 2: q = (ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4); break;
                default: q = (ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4); break;
            }
            uint16_t hd; memcpy(&hd, b + 208, 2);
            return (h2f(hd) * (float)(int8_t)b[192 + i / 16]) * (float)(q - 32);
        }
    }
    return NAN;
}

ORC_EXPORT float orc_dequant(orc_model *m, const char *name, long r, long j) {
    const tensor_t *t = find(m, name);
    return t ? deq(t, r, j) : NAN;
}

ORC_EXPORT orc_model *orc_load(const char *path) {
    orc_model *m = calloc(1, sizeof *m);
    FILE *f = fopen(path, "rb");
    if (!f) { free(m); return NULL; }
    fseek(f, 0, SEEK_END);
    m->file_size = (size_t)ftell(f);
    fseek(f, 0, SEEK_SET);
    m->file = malloc(m->file_size);
    if (fread(m->file, 1, m->file_size, f) != m->file_size) { fclose(f); orc_free(m); return NULL; }
    fclose(f);
    const uint8_t *p = m->file;
    if (rd32(&p) != 0x46554747u) { orc_free(m); return NULL; }
    rd32(&p);
    uint64_t nt = rd64(&p), nkv = rd64(&p);
    uint32_t align = 32;
    cfg_t *c = &m->c;
    for (uint64_t i = 0; i < nkv; ++i) {
        uint64_t kl = rd64(&p);
        char key[128] = {0};
        memcpy(key, p, kl < 127 ? kl : 127);
        p += kl;
        uint32_t t = rd32(&p);
        if (t == 4 || t == 7) {
            uint32_t v = t == 4 ? rd32(&p) : *p++;
            struct { const char *k; int *dst; } map[] = {
                {"nllb.vocab_size", &c->V}, {"nllb.embedding_length", &c->d},
                {"nllb.encoder.block_count", &c->enc_layers}, {"nllb.decoder.block_count", &c->dec_layers},
                {"nllb.encoder.attention.head_count", &c->enc_heads},
                {"nllb.decoder.attention.head_count", &c->dec_heads},
                {"nllb.encoder.feed_forward_length", &c->enc_ffn}, {"nllb.decoder.feed_forward_length", &c->dec_ffn},
                {"nllb.context_length", &c->max_pos}, {"nllb.scale_embedding", &c->scale_embedding},
                {"nllb.max_length", &c->max_length}, {"tokenizer.ggml.padding_token_id", &c->pad},
                {"tokenizer.ggml.eos_token_id", &c->eos}, {"tokenizer.ggml.decoder_start_token_id", &c->start},
                {"general.alignment", (int *)&align}};
            for (size_t k = 0; k < sizeof map / sizeof map[0]; ++k)
                if (!strcmp(key, map[k].k)) *map[k].dst = (int)v;
        } else {
            skip_value(&p, t);
        }
    }
    m->nt = (int)nt;
    m->t = calloc(nt, sizeof(tensor_t));
    uint64_t *offs = calloc(nt, 8);
    for (uint64_t i = 0; i < nt; ++i) {
        uint64_t nl = rd64(&p);
        memcpy(m->t[i].name, p, nl < 95 ? nl : 95);
        p += nl;
        uint32_t nd = rd32(&p);
        uint64_t dims[4] = {1, 1, 1, 1};
        for (uint32_t k = 0; k < nd; ++k) dims[k] = rd64(&p);
        m->t[i].type = (int)rd32(&p);
        offs[i] = rd64(&p);
        m->t[i].cols = (long)dims[0];
        m->t[i].rows = (long)(dims[1] * dims[2] * dims[3]);
    }
    size_t data0 = ((size_t)(p - m->file) + align - 1) / align * align;
    for (uint64_t i = 0; i < nt; ++i) m->t[i].data = m->file + data0 + offs[i];
    free(offs);

    char nm[96];
    m->embed = find(m, "token_embd.weight");
    m->enc = calloc((size_t)c->enc_layers, sizeof(layer_t));
    m->dec = calloc((size_t)c->dec_layers, sizeof(layer_t));
#define LIN(dst, fmt, i)                                              \
    do {                                                              \
        snprintf(nm, sizeof nm, fmt ".weight", i); (dst).w = find(m, nm); \
        snprintf(nm, sizeof nm, fmt ".bias", i); (dst).b = dense(m, nm);  \
    } while (0)
#define NORM(dst, fmt, i)                                               \
    do {                                                                \
        snprintf(nm, sizeof nm, fmt ".weight", i); (dst).g = dense(m, nm); \
        snprintf(nm, sizeof nm, fmt ".bias", i); (dst).b = dense(m, nm);   \
    } while (0)
    for (int i = 0; i < c->enc_layers; ++i) {
        layer_t *l = &m->enc[i];
        NORM(l->attn_norm, "enc.blk.%d.attn_norm", i);
        NORM(l->ffn_norm, "enc.blk.%d.ffn_norm", i);
        LIN(l->qkv, "enc.blk.%d.attn_qkv", i);
        LIN(l->out, "enc.blk.%d.attn_out", i);
        LIN(l->up, "enc.blk.%d.ffn_up", i);
        LIN(l->down, "enc.blk.%d.ffn_down", i);
    }
    for (int i = 0; i < c->dec_layers; ++i) {
        layer_t *l = &m->dec[i];
        NORM(l->attn_norm, "dec.blk.%d.attn_norm", i);
        NORM(l->cross_norm, "dec.blk.%d.cross_attn_norm", i);
        NORM(l->ffn_norm, "dec.blk.%d.ffn_norm", i);
        LIN(l->qkv, "dec.blk.%d.attn_qkv", i);
        LIN(l->out, "dec.blk.%d.attn_out", i);
        LIN(l->cq, "dec.blk.%d.cross_attn_q", i);
        LIN(l->ckv, "dec.blk.%d.cross_attn_kv", i);
        LIN(l->co, "dec.blk.%d.cross_attn_out", i);
        LIN(l->up, "dec.blk.%d.ffn_up", i);
        LIN(l->down, "dec.blk.%d.ffn_down", i);
    }
    NORM(m->enc_norm, "enc.output_norm%s", "");
    NORM(m->dec_norm, "dec.output_norm%s", "");
#undef LIN
#undef NORM
    /* model.rs:325-340 and 361-366 */
    int n_pos = c->max_pos + c->pad + 1, d = c->d, half = d / 2;
    m->pos = calloc((size_t)n_pos * d, sizeof(float));
    double step = log(10000.0) / ((double)half - 1.0);
    for (int pp = 0; pp < n_pos; ++pp) {
        if (pp == c->pad) continue;
        for (int i = 0; i < half; ++i) {
            double a = (double)pp * exp(-(double)i * step);
            m->pos[(size_t)pp * d + i] = (float)sin(a);
            m->pos[(size_t)pp * d + half + i] = (float)cos(a);
        }
    }
    m->embed_scale = c->scale_embedding ? (float)sqrt((double)d) : 1.0f;
    return m;
}

ORC_EXPORT void orc_free(orc_model *m) {
    if (!m) return;
    free(m->file);
    free(m->t);
    free(m->enc);
    free(m->dec);
    free(m->pos);
    free(m);
}

ORC_EXPORT int orc_config(orc_model *m, int *out) {
    const cfg_t *c = &m->c;
    int v[] = {c->V, c->d, c->enc_layers, c->dec_layers, c->enc_heads, c->dec_heads, c->enc_ffn, c->dec_ffn,
               c->max_pos, c->pad, c->eos, c->start, c->max_length, c->scale_embedding};
    memcpy(out, v, sizeof v);
    return (int)(sizeof v / sizeof v[0]);
}

/* ------------------------------------------------------------------------ */
/* Activation quantization and the quantized matmul                          */
/*
 * The reference's GPU decode runs every quantized projection through candle's
 * QMatMul::forward (model.rs:79-81, 571-607), i.e. candle-core 0.11.0
 * src/quantized/cuda.rs with the kernels of candle-kernels 0.11.0
 * src/quantized.cu (vendored from llama.cpp's ggml-cuda). The reference
 * documents the consequence: activations are quantized to q8_1, MMVQ runs up
 * to 8 rows and MMQ above, and outputs depend on the batch size
 * (docs/performance.md:51-54). This section restates that published
 * arithmetic for the three weight types the presets use:
 *
 *   q8_1 (quantize_q8_1): per 32-value block, amax = max|x|, s = warp sum of x
 *     (xor butterfly 16,8,4,2,1), d = amax/127, q = amax == 0 ? 0 : roundf(x/d);
 *     d and s are stored as f16.
 *   MMVQ (mul_mat_vec_q, b_size <= 8 rows): nw = 4 warps for 1-4 rows, 2 for
 *     5-8 (candle's launch table). Thread t of nw*32 owns slices of blocks
 *     kbx = t/(qi/vdr) + i*blocks_per_iter and sums its vec_dot results in
 *     that order; warps 1.. add theirs to warp 0's in warp order; a butterfly
 *     sum over the 32 lanes gives the output. vec_dot per type:
 *       Q8_0 (8 values): (dw*dx) * float(I)
 *       Q4_K (8 values of 2 sub-blocks): dall*sumf_d - dmin*sumf_m with
 *             sumf_d = sum_i dx_i*float(I_i*sc_i), sumf_m = sum_i dx_i*float(Q_i*m_i)
 *             (Q_i = sum of the 8 activation integers)
 *       Q6_K (4 values of 2 blocks 64 apart): d * sum_i dx_i*float(I_i*sc_i)
 *   MMQ (mul_mat_q, more rows): every output is one thread's running sum over
 *     units in row order, starting at 0:
 *       Q8_0 unit = one block: (dw*dx) * float(I)
 *       Q4_K unit = 2 sub-blocks: dall*sumf_d - dmin*sumf_m, sumf_d = sum dx*float(sc*I),
 *             sumf_m = sum sx*float(m) (sx = the f16 block sum of the f32 inputs)
 *       Q6_K unit = 2 blocks: d * sum dx*float(sc_a*I_a + sc_b*I_b) (16-value halves)
 * Integer sums are exact. Every float "a += b*c" / "a*b - c*d" of those
 * kernels is written below as nvcc's default contraction computes it
 * (fmaf(b, c, a); fmaf(a, b, -(c*d))); all other operations round on their own.
 * F32 weights (candle: a cuBLAS matmul, not restated) use this project's order:
 * lane l's FMA chain over elements l, l+32, ..., then the butterfly sum.
 */

typedef struct {
    int8_t *q;  /* [rows, K] */
    float *d;   /* [rows, K/32]: block scale (f16 value) */
    float *s;   /* [rows, K/32]: block sum of the inputs (f16 value) */
} q81_t;

/* The reference's warp_reduce_sum over 32 lane values: x += shfl_xor(x, m), m = 16..1. */
static float bfly32(const float *v) {
    float a[32], b[32];
    memcpy(a, v, sizeof a);
    for (int m = 16; m > 0; m >>= 1) {
        for (int l = 0; l < 32; ++l) b[l] = a[l] + a[l ^ m];
        memcpy(a, b, sizeof a);
    }
    return a[0];
}

/* quantize_q8_1 of `rows` rows of K values (candle-kernels src/quantized.cu). */
static void quantize_q81(const float *x, int rows, int K, q81_t *o) {
    const int nb = K / 32;
    for (int r = 0; r < rows; ++r)
        for (int j = 0; j < nb; ++j) {
            const float *v = x + (size_t)r * K + 32 * j;
            float amax = 0.0f;
            for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
            const float sum = bfly32(v), d = amax / 127.0f;
            int8_t *q = o->q + (size_t)r * K + 32 * j;
            for (int i = 0; i < 32; ++i) q[i] = amax == 0.0f ? 0 : (int8_t)roundf(v[i] / d);
            o->d[(size_t)r * nb + j] = rnd_h(d);
            o->s[(size_t)r * nb + j] = rnd_h(sum);
        }
}

/* Unpacked weight row: integer values and scale data. */
typedef struct {
    int8_t *q;    /* [K]: Q8_0 int8; Q4_K 0..15; Q6_K q-32 */
    float *dw;    /* Q8_0: per block d; Q4_K: per super-block d; Q6_K: per super-block d */
    float *dm;    /* Q4_K: per super-block dmin */
    int *sc;      /* Q4_K: per block 6-bit scale; Q6_K: per 16 values int8 scale */
    int *mn;      /* Q4_K: per block 6-bit min */
} wrow_t;

static void unpack_row(const tensor_t *t, long r, wrow_t *w) {
    long K = t->cols;
    const uint8_t *row = t->data + (size_t)r * type_row_bytes(t->type, K);
    if (t->type == GT_Q8_0) {
        for (long j = 0; j < K / 32; ++j) {
            uint16_t h; memcpy(&h, row + 34 * j, 2);
            w->dw[j] = h2f(h);
            for (int i = 0; i < 32; ++i) w->q[32 * j + i] = (int8_t)row[34 * j + 2 + i];
        }
    } else if (t->type == GT_Q4_K) {
        for (long sbk = 0; sbk < K / 256; ++sbk) {
            const uint8_t *b = row + 144 * sbk, *s = b + 4;
            uint16_t hd, hm; memcpy(&hd, b, 2); memcpy(&hm, b + 2, 2);
            w->dw[sbk] = h2f(hd);
            w->dm[sbk] = h2f(hm);
            for (int sb = 0; sb < 8; ++sb) {
                int sc, mn;
                if (sb < 4) { sc = s[sb] & 63; mn = s[sb + 4] & 63; }
                else { sc = (s[sb + 4] & 0xf) | ((s[sb - 4] >> 6) << 4); mn = (s[sb + 4] >> 4) | ((s[sb] >> 6) << 4); }
                long j = sbk * 8 + sb;
                w->sc[j] = sc;
                w->mn[j] = mn;
                for (int i = 0; i < 32; ++i) {
                    uint8_t byte = b[16 + 32 * (sb / 2) + i];
                    w->q[256 * sbk + 32 * sb + i] = (int8_t)((sb & 1) ? byte >> 4 : byte & 0xf);
                }
            }
        }
    } else if (t->type == GT_Q6_K) {
        for (long sbk = 0; sbk < K / 256; ++sbk) {
            const uint8_t *b = row + 210 * sbk;
            uint16_t hd; memcpy(&hd, b + 208, 2);
            w->dw[sbk] = h2f(hd);
            for (int i = 0; i < 256; ++i) {
                int n = i / 128, g = (i % 128) / 32, l = i % 32, q;
                const uint8_t *ql = b + 64 * n, *qh = b + 128 + 32 * n;
                switch (g) {
                    case 0: q = (ql[l] & 0xf) | (((qh[l] >> 0) & 3) << 4); break;
                    case 1: q = (ql[l + 32] & 0xf) | (((qh[l] >> 2) & 3) << 4); break;
                    case 2: q = (ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4); break;
                    default: q = (ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4); break;
                }
                w->q[256 * sbk + i] = (int8_t)(q - 32);
            }
            for (int g = 0; g < 16; ++g) w->sc[sbk * 16 + g] = (int8_t)b[192 + g];
        }
    }
}

/* MMVQ: thread t's sum of its vec_dot results (mul_mat_vec_q's tmp). */
static float mmvq_thread(int type, const wrow_t *w, const int8_t *xq, const float *xd, int K, int nw, int t) {
    float P = 0.0f;
    if (type == GT_Q8_0) { /* qi 8, vdr 2: 4 threads per block, values 8o..8o+7 */
        const int nb = K / 32, bpi = nw * 8, o = t % 4;
        for (int kb = t / 4; kb < nb; kb += bpi) {
            int s = 0;
            for (int i = 8 * o; i < 8 * o + 8; ++i) s += w->q[32 * kb + i] * xq[32 * kb + i];
            P = fmaf(w->dw[kb] * xd[kb], (float)s, P);
        }
    } else if (type == GT_Q4_K) { /* qi 32, vdr 2: 16 threads per super-block */
        const int nsb = K / 256, bpi = nw * 2, c = (t % 16) / 4, o = t % 4;
        for (int kb = t / 16; kb < nsb; kb += bpi) {
            float sd = 0.0f, sm = 0.0f;
            for (int i = 0; i < 2; ++i) { /* sub-blocks 2c (low nibbles) and 2c+1 (high) */
                const int j = 8 * kb + 2 * c + i;
                int dot1 = 0, dot2 = 0;
                for (int h = 0; h < 2; ++h)
                    for (int p = 16 * h + 4 * o; p < 16 * h + 4 * o + 4; ++p) {
                        dot1 += w->q[32 * j + p] * xq[32 * j + p];
                        dot2 += xq[32 * j + p];
                    }
                sd = fmaf(xd[j], (float)(dot1 * w->sc[j]), sd);
                sm = fmaf(xd[j], (float)(dot2 * w->mn[j]), sm);
            }
            P = P + fmaf(w->dw[kb], sd, -(w->dm[kb] * sm));
        }
    } else { /* Q6_K: qi 32, vdr 1: 32 threads per super-block */
        const int nsb = K / 256, bpi = nw, l = t % 32;
        const int A = 4 * (l / 16) + (l % 16) / 8, p0 = 4 * (l % 8);
        for (int kb = t / 32; kb < nsb; kb += bpi) {
            float sf = 0.0f;
            for (int i = 0; i < 2; ++i) { /* blocks A and A+2 of the super-block */
                const int j = 8 * kb + A + 2 * i;
                int dot = 0;
                for (int p = p0; p < p0 + 4; ++p) dot += w->q[32 * j + p] * xq[32 * j + p];
                sf = fmaf(xd[j], (float)(dot * w->sc[(32 * j + p0) / 16]), sf);
            }
            P = fmaf(w->dw[kb], sf, P);
        }
    }
    return P;
}

/* One MMVQ output with nw warps. */
static float mmvq_out(int type, const wrow_t *w, const int8_t *xq, const float *xd, int K, int nw) {
    float leaf[32];
    for (int l = 0; l < 32; ++l) {
        float v = 0.0f;
        for (int wv = 0; wv < nw; ++wv) {
            const float P = mmvq_thread(type, w, xq, xd, K, nw, 32 * wv + l);
            v = wv == 0 ? P : v + P;
        }
        leaf[l] = v;
    }
    return bfly32(leaf);
}

/* One MMQ output: the running sum over units in row order. */
static float mmq_out(int type, const wrow_t *w, const int8_t *xq, const float *xd, const float *xs, int K) {
    const int nb = K / 32;
    float acc = 0.0f;
    if (type == GT_Q8_0) {
        for (int j = 0; j < nb; ++j) {
            int s = 0;
            for (int i = 0; i < 32; ++i) s += w->q[32 * j + i] * xq[32 * j + i];
            acc = fmaf(w->dw[j] * xd[j], (float)s, acc);
        }
    } else if (type == GT_Q4_K) {
        for (int j = 0; j < nb; j += 2) {
            int I[2];
            for (int i = 0; i < 2; ++i) {
                int s = 0;
                for (int p = 0; p < 32; ++p) s += w->q[32 * (j + i) + p] * xq[32 * (j + i) + p];
                I[i] = s;
            }
            const float sd = fmaf(xd[j + 1], (float)(w->sc[j + 1] * I[1]), fmaf(xd[j], (float)(w->sc[j] * I[0]), 0.0f));
            const float sm = fmaf(xs[j + 1], (float)w->mn[j + 1], fmaf(xs[j], (float)w->mn[j], 0.0f));
            acc = acc + fmaf(w->dw[j / 8], sd, -(w->dm[j / 8] * sm));
        }
    } else {
        for (int j = 0; j < nb; j += 2) {
            int X[2];
            for (int i = 0; i < 2; ++i) {
                int a = 0, b = 0;
                for (int p = 0; p < 16; ++p) {
                    a += w->q[32 * (j + i) + p] * xq[32 * (j + i) + p];
                    b += w->q[32 * (j + i) + 16 + p] * xq[32 * (j + i) + 16 + p];
                }
                X[i] = w->sc[2 * (j + i)] * a + w->sc[2 * (j + i) + 1] * b;
            }
            const float sf = fmaf(xd[j + 1], (float)X[1], fmaf(xd[j], (float)X[0], 0.0f));
            acc = fmaf(w->dw[j / 8], sf, acc);
        }
    }
    return acc;
}

/* F32 weights: lane l's FMA chain over elements l, l+32, ..., then the butterfly. */
static float f32_out(const float *wr, const float *x, int K) {
    float leaf[32];
    for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int i = l; i < K; i += 32) acc = fmaf(wr[i], x[i], acc);
        leaf[l] = acc;
    }
    return bfly32(leaf);
}

/*
 * y[n, r] = dot(row r, x[n]) + bias[r] (then ReLU) for the `rows` activation
 * rows. `cls` is the row count candle's QMatMul sees (the b_size of its kernel
 * choice): the decode step's padded batch, beam rows, or batch x tokens.
 */
static void linear_k(const linear_t *L, const float *x, int rows, int vec, int nw, float *y, int relu);

static void linear(const linear_t *L, const float *x, int rows, int cls, float *y, int relu) {
    linear_k(L, x, rows, cls <= 8, cls <= 4 ? 4 : 2, y, relu);
}

/* The same with the kernel choice explicit: vec = MMVQ with nw warps, else MMQ. */
static void linear_k(const linear_t *L, const float *x, int rows, int vec, int nw, float *y, int relu) {
    const tensor_t *t = L->w;
    const int K = (int)t->cols, N = (int)t->rows, nb = K / 32;
    q81_t xa = {0};
    if (t->type != GT_F32) {
        xa.q = malloc((size_t)rows * K);
        xa.d = malloc((size_t)rows * nb * sizeof(float));
        xa.s = malloc((size_t)rows * nb * sizeof(float));
        quantize_q81(x, rows, K, &xa);
    }
#pragma omp parallel
    {
        wrow_t w;
        w.q = malloc((size_t)K);
        w.dw = malloc(nb * sizeof(float));
        w.dm = malloc(nb * sizeof(float));
        w.sc = malloc(2 * nb * sizeof(int));
        w.mn = malloc(nb * sizeof(int));
#pragma omp for schedule(dynamic, 16)
        for (int r = 0; r < N; ++r) {
            const float *wr32 = NULL;
            if (t->type == GT_F32) wr32 = (const float *)(t->data + (size_t)r * 4 * K);
            else unpack_row(t, r, &w);
            for (int n = 0; n < rows; ++n) {
                float v;
                if (t->type == GT_F32) {
                    v = f32_out(wr32, x + (size_t)n * K, K);
                } else {
                    const int8_t *xq = xa.q + (size_t)n * K;
                    const float *xd = xa.d + (size_t)n * nb, *xs = xa.s + (size_t)n * nb;
                    v = vec ? mmvq_out(t->type, &w, xq, xd, K, nw) : mmq_out(t->type, &w, xq, xd, xs, K);
                }
                if (L->b) v = v + L->b[r];
                if (relu) v = v > 0.0f ? v : 0.0f;
                y[(size_t)n * N + r] = v;
            }
        }
        free(w.q); free(w.dw); free(w.dm); free(w.sc); free(w.mn);
    }
    free(xa.q);
    free(xa.d);
    free(xa.s);
}

/* y[rows, N] = x[rows, K] . W^T for a raw GGUF matrix (type, N rows of K values):
 * mode 0 = MMVQ with nw warps, 1 = MMQ. Test entry point (pins against other
 * builds of the same published kernels). */
ORC_EXPORT int orc_matmul(int type, const uint8_t *w, long N, long K, const float *x, int rows, int mode, int nw,
                          float *y) {
    if (K % 256 && type != GT_Q8_0 && type != GT_F32) return -1;
    tensor_t t;
    memset(&t, 0, sizeof t);
    t.type = type;
    t.rows = N;
    t.cols = K;
    t.data = w;
    linear_t L = {&t, NULL};
    linear_k(&L, x, rows, mode == 0, nw, y, 0);
    return 0;
}

/* q8_1 quantization of rows x K values: q [rows, K], d and s [rows, K/32]. */
ORC_EXPORT void orc_quantize_q81(const float *x, int rows, int K, int8_t *q, float *d, float *s) {
    q81_t o = {q, d, s};
    quantize_q81(x, rows, K, &o);
}

/* LayerNorm (eps 1e-5, config.rs:58): mean and variance by SUM32. */
static void layer_norm(const float *x, const norm_t *nrm, int rows, int d, float *y) {
    float *c = malloc((size_t)d * sizeof(float));
    for (int r = 0; r < rows; ++r) {
        const float *v = x + (size_t)r * d;
        float mean = sum32(v, d, 1) / (float)d;
        for (int i = 0; i < d; ++i) { float t = v[i] - mean; c[i] = t * t; }
        float var = sum32(c, d, 1) / (float)d;
        float rstd = 1.0f / sqrtf(var + 1e-5f);
        for (int i = 0; i < d; ++i) y[(size_t)r * d + i] = ((v[i] - mean) * rstd) * nrm->g[i] + nrm->b[i];
    }
    free(c);
}

/*
 * Single-query attention over n keys: s_j = fmaf chain q.k_j; e_j = exp(s_j - max);
 * out_t = (fmaf chain over j of e_j*v_jt) * (1 / SUM32(e)). K/V rows have stride `ks`.
 */
static void attend(const float *q, const float *K, const float *Vv, int n, int hd, long ks, float *out, float *e) {
    float mx = -INFINITY;
    for (int j = 0; j < n; ++j) {
        float acc = 0.0f;
        for (int t = 0; t < hd; ++t) acc = fmaf(q[t], K[(size_t)j * ks + t], acc);
        e[j] = acc;
        mx = fmaxf(mx, acc);
    }
    for (int j = 0; j < n; ++j) e[j] = mgb_exp(e[j] - mx);
    float inv = 1.0f / sum32(e, n, 1);
    for (int t = 0; t < hd; ++t) {
        float acc = 0.0f;
        for (int j = 0; j < n; ++j) acc = fmaf(e[j], Vv[(size_t)j * ks + t], acc);
        out[t] = acc * inv;
    }
}

/* ------------------------------------------------------------------------ */
/* Encoder (model.rs:463-500)                                                */

typedef struct orc_enc {
    int b, s;
    uint32_t *lens;
    float *ck, *cv;     /* per decoder layer [b, H, s, hd], values rounded to f16 (the fused step's copy) */
    float *ck32, *cv32; /* the same in f32, as encode_cross returns them (the generic decode's) */
} orc_enc;

ORC_EXPORT orc_enc *orc_encode(orc_model *m, const uint32_t *ids, const uint32_t *lens, int b, int s) {
    const cfg_t *c = &m->c;
    int d = c->d, H = c->enc_heads, hd = d / H, rows = b * s;
    float *x = malloc((size_t)rows * d * sizeof(float)), *h = malloc((size_t)rows * d * sizeof(float));
    float *qkv = malloc((size_t)rows * 3 * d * sizeof(float)), *a = malloc((size_t)rows * d * sizeof(float));
    float *y = malloc((size_t)rows * d * sizeof(float));
    float *u = malloc((size_t)rows * c->enc_ffn * sizeof(float));
    for (int bi = 0; bi < b; ++bi)
        for (int j = 0; j < s; ++j) {
            int valid = j < (int)lens[bi];
            uint32_t id = valid ? ids[bi * s + j] : (uint32_t)c->pad;
            int pp = valid ? j + c->pad + 1 : c->pad;
            for (int i = 0; i < d; ++i)
                x[((size_t)bi * s + j) * d + i] = deq(m->embed, id, i) * m->embed_scale + m->pos[(size_t)pp * d + i];
        }
    for (int l = 0; l < c->enc_layers; ++l) {
        const layer_t *L = &m->enc[l];
        layer_norm(x, &L->attn_norm, rows, d, h);
        linear(&L->qkv, h, rows, rows, qkv, 0);
#pragma omp parallel
        {
            float *e = malloc((size_t)s * sizeof(float));
#pragma omp for collapse(2)
            for (int bi = 0; bi < b; ++bi)
                for (int hh = 0; hh < H; ++hh)
                    for (int i = 0; i < s; ++i) {
                        const float *base = qkv + (size_t)bi * s * 3 * d;
                        attend(base + (size_t)i * 3 * d + hh * hd, base + d + hh * hd, base + 2 * d + hh * hd,
                               (int)lens[bi], hd, 3 * d, a + ((size_t)bi * s + i) * d + hh * hd, e);
                    }
            free(e);
        }
        linear(&L->out, a, rows, rows, y, 0);
        for (size_t i = 0; i < (size_t)rows * d; ++i) x[i] = y[i] + x[i];
        layer_norm(x, &L->ffn_norm, rows, d, h);
        linear(&L->up, h, rows, rows, u, 1);
        linear(&L->down, u, rows, rows, y, 0);
        for (size_t i = 0; i < (size_t)rows * d; ++i) x[i] = y[i] + x[i];
    }
    layer_norm(x, &m->enc_norm, rows, d, h);
    orc_enc *E = calloc(1, sizeof *E);
    E->b = b;
    E->s = s;
    E->lens = malloc(b * sizeof(uint32_t));
    memcpy(E->lens, lens, b * sizeof(uint32_t));
    int Hd = c->dec_heads, hdd = d / Hd;
    size_t per = (size_t)b * Hd * s * hdd;
    E->ck = malloc(per * c->dec_layers * sizeof(float));
    E->cv = malloc(per * c->dec_layers * sizeof(float));
    E->ck32 = malloc(per * c->dec_layers * sizeof(float));
    E->cv32 = malloc(per * c->dec_layers * sizeof(float));
    float *kv = malloc((size_t)rows * 2 * d * sizeof(float));
    for (int l = 0; l < c->dec_layers; ++l) {
        linear(&m->dec[l].ckv, h, rows, rows, kv, 0);
        for (int bi = 0; bi < b; ++bi)
            for (int hh = 0; hh < Hd; ++hh)
                for (int j = 0; j < s; ++j)
                    for (int t = 0; t < hdd; ++t) {
                        size_t src = ((size_t)bi * s + j) * 2 * d + hh * hdd + t;
                        size_t dst = per * l + (((size_t)bi * Hd + hh) * s + j) * hdd + t;
                        E->ck32[dst] = kv[src];
                        E->cv32[dst] = kv[src + d];
                        E->ck[dst] = rnd_h(kv[src]);
                        E->cv[dst] = rnd_h(kv[src + d]);
                    }
    }
    free(kv); free(x); free(h); free(qkv); free(a); free(y); free(u);
    return E;
}

/* An encoded-batch stand-in with pseudo-random f16-exact cross K/V and no
 * encoder pass: decode cost does not depend on these values. Timing only. */
ORC_EXPORT orc_enc *orc_enc_synthetic(orc_model *m, const uint32_t *lens, int b, int s, uint64_t seed) {
    const cfg_t *c = &m->c;
    orc_enc *E = calloc(1, sizeof *E);
    E->b = b;
    E->s = s;
    E->lens = malloc(b * sizeof(uint32_t));
    memcpy(E->lens, lens, b * sizeof(uint32_t));
    size_t n = (size_t)b * c->d * s * c->dec_layers;
    E->ck = malloc(n * sizeof(float));
    E->cv = malloc(n * sizeof(float));
    E->ck32 = E->ck;
    E->cv32 = E->cv;
    uint64_t x = seed * 0x9e3779b97f4a7c15ull + 1;
    for (size_t i = 0; i < n; ++i) {
        x ^= x << 13; x ^= x >> 7; x ^= x << 17;
        E->ck[i] = rnd_h((float)((int)(x & 0xffff) - 32768) / 32768.0f);
        E->cv[i] = rnd_h((float)((int)((x >> 16) & 0xffff) - 32768) / 32768.0f);
    }
    return E;
}

ORC_EXPORT void orc_enc_free(orc_enc *E) {
    if (!E) return;
    if (E->ck32 != E->ck) { free(E->ck32); free(E->cv32); }
    free(E->lens); free(E->ck); free(E->cv); free(E);
}

/* Cross K (which=0) or V (which=1) of decoder layer `l`, [b, H, s, hd] f32 (f16-exact values). */
ORC_EXPORT void orc_enc_cross(orc_model *m, orc_enc *E, int l, int which, float *out) {
    int d = m->c.d;
    size_t per = (size_t)E->b * E->s * d;
    memcpy(out, (which ? E->cv : E->ck) + per * l, per * sizeof(float));
}

/* ------------------------------------------------------------------------ */
/* Decoder state and the fused greedy step (model.rs:552-612)                */

typedef struct {
    int b, m;  /* rows, self-KV capacity */
    int cls;   /* rows of the reference's decoder-layer matmul calls (greedy: graph.rs:242, the batch
                  padded to a power of two; beam prefill: 2 tokens per row) */
    int lm_cls; /* rows of its LM head call */
    int kv32;  /* 1: the generic decode's f32 self / cross K/V (beam search); 0: the fused step's f16 */
    float *kc, *vc; /* per layer [b, H, m, hd] (f16-exact values) */
    float *x, *h, *qkv, *a, *y, *u, *logits;
} dstate_t;

static void dstate_init(orc_model *M, dstate_t *S, int b, int m, int cls) {
    const cfg_t *c = &M->c;
    int d = c->d;
    S->b = b;
    S->cls = cls;
    S->lm_cls = cls;
    S->kv32 = 0;
    S->m = m;
    size_t kv = (size_t)c->dec_layers * b * d * m;
    S->kc = calloc(kv, sizeof(float));
    S->vc = calloc(kv, sizeof(float));
    S->x = malloc((size_t)b * d * 4); S->h = malloc((size_t)b * d * 4); S->qkv = malloc((size_t)b * 3 * d * 4);
    S->a = malloc((size_t)b * d * 4); S->y = malloc((size_t)b * d * 4);
    S->u = malloc((size_t)b * c->dec_ffn * 4);
    S->logits = malloc((size_t)b * c->V * 4);
}

static void dstate_free(dstate_t *S) {
    free(S->kc); free(S->vc); free(S->x); free(S->h); free(S->qkv); free(S->a); free(S->y); free(S->u);
    free(S->logits);
}

/* One decoder step at position `step` for input tokens ids[b]; leaves logits [b, V] in S->logits
 * (lm = 0: no LM head). `src_row[r]` maps decoder row r to its encoder row (beam search
 * repeats sentences). */
static void dec_step(orc_model *M, orc_enc *E, dstate_t *S, const uint32_t *ids, int step, const int *src_row,
                     int lm) {
    const cfg_t *c = &M->c;
    int b = S->b, d = c->d, H = c->dec_heads, hd = d / H;
    for (int r = 0; r < b; ++r)
        for (int i = 0; i < d; ++i)
            S->x[(size_t)r * d + i] = deq(M->embed, ids[r], i) * M->embed_scale +
                                      M->pos[(size_t)(step + c->pad + 1) * d + i];
    size_t cper = (size_t)E->b * H * E->s * hd;
    for (int l = 0; l < c->dec_layers; ++l) {
        const layer_t *L = &M->dec[l];
        float *kc = S->kc + (size_t)l * b * d * S->m, *vc = S->vc + (size_t)l * b * d * S->m;
        layer_norm(S->x, &L->attn_norm, b, d, S->h);
        linear(&L->qkv, S->h, b, S->cls, S->qkv, 0);
        for (int r = 0; r < b; ++r)
            for (int hh = 0; hh < H; ++hh)
                for (int t = 0; t < hd; ++t) {
                    size_t slot = (((size_t)r * H + hh) * S->m + step) * hd + t;
                    const float kv_k = S->qkv[(size_t)r * 3 * d + d + hh * hd + t];
                    const float kv_v = S->qkv[(size_t)r * 3 * d + 2 * d + hh * hd + t];
                    kc[slot] = S->kv32 ? kv_k : rnd_h(kv_k);
                    vc[slot] = S->kv32 ? kv_v : rnd_h(kv_v);
                }
#pragma omp parallel
        {
            float *e = malloc((size_t)(S->m > E->s ? S->m : E->s) * sizeof(float));
#pragma omp for collapse(2)
            for (int r = 0; r < b; ++r)
                for (int hh = 0; hh < H; ++hh) {
                    size_t base = ((size_t)r * H + hh) * S->m * hd;
                    attend(S->qkv + (size_t)r * 3 * d + hh * hd, kc + base, vc + base, step + 1, hd, hd,
                           S->a + (size_t)r * d + hh * hd, e);
                }
            free(e);
        }
        linear(&L->out, S->a, b, S->cls, S->y, 0);
        for (size_t i = 0; i < (size_t)b * d; ++i) S->x[i] = S->y[i] + S->x[i];
        layer_norm(S->x, &L->cross_norm, b, d, S->h);
        linear(&L->cq, S->h, b, S->cls, S->y, 0);
#pragma omp parallel
        {
            float *e = malloc((size_t)E->s * sizeof(float));
#pragma omp for collapse(2)
            for (int r = 0; r < b; ++r)
                for (int hh = 0; hh < H; ++hh) {
                    int sr = src_row ? src_row[r] : r;
                    size_t base = cper * l + ((size_t)sr * H + hh) * E->s * hd;
                    attend(S->y + (size_t)r * d + hh * hd, (S->kv32 ? E->ck32 : E->ck) + base,
                           (S->kv32 ? E->cv32 : E->cv) + base, (int)E->lens[sr], hd, hd,
                           S->a + (size_t)r * d + hh * hd, e);
                }
            free(e);
        }
        linear(&L->co, S->a, b, S->cls, S->y, 0);
        for (size_t i = 0; i < (size_t)b * d; ++i) S->x[i] = S->y[i] + S->x[i];
        layer_norm(S->x, &L->ffn_norm, b, d, S->h);
        linear(&L->up, S->h, b, S->cls, S->u, 1);
        linear(&L->down, S->u, b, S->cls, S->y, 0);
        for (size_t i = 0; i < (size_t)b * d; ++i) S->x[i] = S->y[i] + S->x[i];
    }
    if (!lm) return;
    layer_norm(S->x, &M->dec_norm, b, d, S->h);
    linear_t head = {M->embed, NULL};
    linear(&head, S->h, b, S->lm_cls, S->logits, 0);
}

static uint32_t argmax_row(const float *v, int n) {
    float best = -INFINITY;
    uint32_t bi = 0;
    for (int i = 0; i < n; ++i)
        if (v[i] > best) { best = v[i]; bi = (uint32_t)i; }
    return bi;
}

/*
 * Greedy decoding of an encoded batch, as GraphCache::run (graph.rs:262-297):
 * step 0 feeds decoder_start (output discarded), then tgt_lang is forced and
 * steps 1..max_new produce out[:, 0..max_new). A finished row emits pad; a row
 * finishes when it emits eos (never with force_steps). Returns the number of
 * generated columns. logits (optional) receives [max_new, b, V] of steps 1..
 */
ORC_EXPORT int orc_greedy(orc_model *M, orc_enc *E, uint32_t tgt, int max_new, int force_steps, uint32_t *out,
                          float *logits) {
    const cfg_t *c = &M->c;
    int b = E->b, m = max_new + 2;
    dstate_t S;
    int cls = 1;
    while (cls < b) cls <<= 1; /* graph.rs:242 */
    dstate_init(M, &S, b, m, cls);
    uint32_t *ids = malloc(b * sizeof(uint32_t));
    uint8_t *fin = calloc(b, 1);
    for (int r = 0; r < b; ++r) ids[r] = (uint32_t)c->start;
    dec_step(M, E, &S, ids, 0, NULL, 1);
    for (int r = 0; r < b; ++r) ids[r] = tgt;
    for (int st = 1; st <= max_new; ++st) {
        dec_step(M, E, &S, ids, st, NULL, 1);
        if (logits) memcpy(logits + (size_t)(st - 1) * b * c->V, S.logits, (size_t)b * c->V * 4);
        for (int r = 0; r < b; ++r) {
            uint32_t tok = argmax_row(S.logits + (size_t)r * c->V, c->V);
            if (fin[r]) tok = (uint32_t)c->pad;
            if (!force_steps && tok == (uint32_t)c->eos) fin[r] = 1;
            ids[r] = tok;
            out[(size_t)r * max_new + st - 1] = tok;
        }
    }
    free(ids); free(fin);
    dstate_free(&S);
    return max_new;
}

/*
 * Greedy decoding over a vocabulary shortlist (--fast-vocab, not exact;
 * model.rs:556-612, graph.rs:98-105, malaga.cu:280-326). Each step scores, per
 * row, the LM head rows of the shortlist ids (rows of the tied embedding, so
 * their logits are those of the full head) followed by the row's S source
 * positions (its source ids, pad past its length), scored as
 * dot(dec_norm(x), E[id]) in the F32 order (f32_out); the first maximum of that
 * list wins and maps back to its token. The next input embedding is E[token],
 * as the reference's shortlist or source-embedding row of the token.
 * src: [b][src_stride] ids, lens: [b]; S: the state's source bucket.
 */
ORC_EXPORT int orc_greedy_sl(orc_model *M, orc_enc *E, const uint32_t *src, const uint32_t *lens, int src_stride,
                             uint32_t tgt, int max_new, int force_steps, const uint32_t *sl_ids, int V1, int S,
                             uint32_t *out) {
    const cfg_t *c = &M->c;
    const int b = E->b, m = max_new + 2, d = c->d;
    dstate_t St;
    int cls = 1;
    while (cls < b) cls <<= 1; /* graph.rs:242 */
    dstate_init(M, &St, b, m, cls);
    uint32_t *ids = malloc(b * sizeof(uint32_t));
    uint8_t *fin = calloc(b, 1);
    float *erow = malloc((size_t)d * sizeof(float));
    for (int r = 0; r < b; ++r) ids[r] = (uint32_t)c->start;
    dec_step(M, E, &St, ids, 0, NULL, 1);
    for (int r = 0; r < b; ++r) ids[r] = tgt;
    for (int st = 1; st <= max_new; ++st) {
        dec_step(M, E, &St, ids, st, NULL, 1);
        for (int r = 0; r < b; ++r) {
            float best = -INFINITY;
            uint32_t bi = 0, tok;
            const float *lg = St.logits + (size_t)r * c->V;
            for (int i = 0; i < V1; ++i)
                if (lg[sl_ids[i]] > best) { best = lg[sl_ids[i]]; bi = (uint32_t)i; }
            for (int j = 0; j < S; ++j) {
                const uint32_t id = j < (int)lens[r] ? src[(size_t)r * src_stride + j] : (uint32_t)c->pad;
                for (int i = 0; i < d; ++i) erow[i] = deq(M->embed, id, i);
                const float v = f32_out(erow, St.h + (size_t)r * d, d);
                if (v > best) { best = v; bi = (uint32_t)(V1 + j); }
            }
            if (bi < (uint32_t)V1) tok = sl_ids[bi];
            else {
                const int j = (int)bi - V1;
                tok = j < (int)lens[r] ? src[(size_t)r * src_stride + j] : (uint32_t)c->pad;
            }
            if (fin[r]) tok = (uint32_t)c->pad;
            if (!force_steps && tok == (uint32_t)c->eos) fin[r] = 1;
            ids[r] = tok;
            out[(size_t)r * max_new + st - 1] = tok;
        }
    }
    free(ids); free(fin); free(erow);
    dstate_free(&St);
    return max_new;
}

/* ------------------------------------------------------------------------ */
/* Beam search (translator.rs:250-358)                                       */

/* log_softmax (model.rs:615-617, candle-nn): y = (x - max) - log(sum exp(x - max)), sum by SUM32. */
static float mgb_log(float x);

typedef struct {
    float score;
    int beam;
    uint32_t tok;
} cand_t;

/* Rust's f32::total_cmp key: IEEE total order as a signed integer. */
static int32_t total_key(float f) {
    int32_t v;
    memcpy(&v, &f, 4);
    return v ^ (int32_t)(((uint32_t)(v >> 31)) >> 1);
}

/* > 0 when a sorts after b in descending score order (sort_by(|a, c| c.total_cmp(a))). */
static int cand_cmp(const void *a, const void *b) {
    int32_t x = total_key(((const cand_t *)a)->score), y = total_key(((const cand_t *)b)->score);
    return (y > x) - (y < x);
}

/* natural log: own implementation, x = 2^e * f, f in [sqrt(1/2), sqrt(2)),
 * log f = 2 atanh(z), z = (f-1)/(f+1), odd series to z^13, plus e*ln2 (2-term). */
static float mgb_log(float x) {
    if (!(x > 0.0f)) return x == 0.0f ? -INFINITY : NAN;
    if (isinf(x)) return x;
    uint32_t b;
    memcpy(&b, &x, 4);
    int e = 0;
    if (b < 0x00800000u) { /* subnormal: scale up by 2^32 */
        float y = x * 4294967296.0f;
        memcpy(&b, &y, 4);
        e = -32;
    }
    e += (int)(b >> 23) - 127;
    uint32_t mb = (b & 0x007fffffu) | 0x3f800000u;
    float f;
    memcpy(&f, &mb, 4);
    if (f > 1.41421353816986084f) { f = f * 0.5f; e += 1; }
    float z = (f - 1.0f) / (f + 1.0f), z2 = z * z;
    float p = 0.153846159577369690f; /* 1/13 */
    p = fmaf(p, z2, 0.181818187236785889f);
    p = fmaf(p, z2, 0.222222223877906799f);
    p = fmaf(p, z2, 0.285714298486709595f);
    p = fmaf(p, z2, 0.400000005960464478f);
    p = fmaf(p, z2, 0.666666686534881592f);
    p = fmaf(p, z2, 2.0f);
    float lf = p * z;
    float fe = (float)e;
    return fmaf(fe, 0.693145751953125f, fmaf(fe, 1.428606765330187e-06f, lf));
}

ORC_EXPORT float orc_log(float x) { return mgb_log(x); }

static void log_softmax_row(const float *x, int n, float *y, float *tmp) {
    float mx = -INFINITY;
    for (int i = 0; i < n; ++i) mx = fmaxf(mx, x[i]);
    for (int i = 0; i < n; ++i) tmp[i] = mgb_exp(x[i] - mx);
    float ls = mgb_log(sum32(tmp, n, 1));
    for (int i = 0; i < n; ++i) y[i] = (x[i] - mx) - ls;
}

/* top-k of one row by k argmax passes (translator.rs:343-358): highest value,
 * lowest index on ties, each index taken once. */
static void topk_row(const float *lp, int n, int k, float *vals, uint32_t *idx) {
    for (int j = 0; j < k; ++j) {
        float best = -INFINITY;
        uint32_t bi = 0;
        int found = 0;
        for (int i = 0; i < n; ++i) {
            int taken = 0;
            for (int q = 0; q < j; ++q) taken |= idx[q] == (uint32_t)i;
            if (taken) continue;
            if (!found || lp[i] > best) { best = lp[i]; bi = (uint32_t)i; found = 1; }
        }
        vals[j] = best;
        idx[j] = bi;
    }
}

/* log_softmax + top-k of rows x n logits (the device half of a beam step). */
ORC_EXPORT void orc_log_softmax_topk(const float *x, int rows, int n, int k, float *vals, uint32_t *idx) {
    float *y = malloc((size_t)n * sizeof(float)), *tmp = malloc((size_t)n * sizeof(float));
    for (int r = 0; r < rows; ++r) {
        log_softmax_row(x + (size_t)r * n, n, y, tmp);
        topk_row(y, n, k, vals + (size_t)r * k, idx + (size_t)r * k);
    }
    free(y);
    free(tmp);
}

/*
 * Batched beam search with beam k and length penalty lp; returns the best
 * hypothesis per sentence into out[b, max_new] (padded with pad) and its
 * length into out_len[b]. Candidate order: score descending, ties in
 * insertion order (beam-major, then top-k rank), as Rust's stable sort.
 */
ORC_EXPORT int orc_beam(orc_model *M, orc_enc *E, uint32_t tgt, int k, float lp, int max_new, uint32_t *out,
                        uint32_t *out_len) {
    const cfg_t *c = &M->c;
    int b = E->b, V = c->V, rows = b * k, m = max_new + 2;
    uint32_t eos = (uint32_t)c->eos;
    dstate_t S;
    dstate_init(M, &S, rows, m, rows);
    int *src_row = malloc(rows * sizeof(int));
    for (int r = 0; r < rows; ++r) src_row[r] = r / k;
    uint32_t *ids = malloc(rows * sizeof(uint32_t));
    /* alive[s][bi]: score + tokens; done[s]: list */
    float *alive_score = malloc(rows * sizeof(float));
    uint32_t *alive_tok = calloc((size_t)rows * (max_new + 1), sizeof(uint32_t));
    int *alive_len = calloc(rows, sizeof(int));
    int *n_alive = malloc(b * sizeof(int));
    int cap_done = 4 * k * (max_new + 1);
    float *done_score = malloc((size_t)b * cap_done * sizeof(float));
    uint32_t *done_tok = malloc((size_t)b * cap_done * (max_new + 1) * sizeof(uint32_t));
    int *done_len = malloc((size_t)b * cap_done * sizeof(int));
    int *n_done = calloc(b, sizeof(int));
    uint8_t *is_done = calloc(b, 1);
    for (int s = 0; s < b; ++s) { n_alive[s] = 1; alive_score[s * k] = 0.0f; alive_len[s * k] = 0; }
    float *lp_row = malloc((size_t)V * sizeof(float)), *tmp = malloc((size_t)V * sizeof(float));
    float *vals = malloc((size_t)rows * k * sizeof(float));
    uint32_t *idx = malloc((size_t)rows * k * sizeof(uint32_t));
    cand_t *cands = malloc((size_t)k * k * sizeof(cand_t));
    int *reorder = malloc(rows * sizeof(int));
    uint32_t *next = malloc(rows * sizeof(uint32_t));
    float *nscore = malloc(rows * sizeof(float));
    uint32_t *ntok = malloc((size_t)rows * (max_new + 1) * sizeof(uint32_t));
    int *nlen = malloc(rows * sizeof(int));
    float *kbuf = malloc((size_t)c->dec_layers * rows * c->d * m * sizeof(float));

    /* the generic decode (model.rs:515-540): f32 K/V; the prefill [</s>, tgt] is one call of 2
     * tokens per row (matmuls over 2*rows rows, the LM head over the last position's rows),
     * computed as two single-token steps with those row classes */
    S.kv32 = 1;
    S.cls = 2 * rows;
    S.lm_cls = rows;
    for (int r = 0; r < rows; ++r) ids[r] = (uint32_t)c->start;
    dec_step(M, E, &S, ids, 0, src_row, 0);
    for (int r = 0; r < rows; ++r) ids[r] = tgt;
    dec_step(M, E, &S, ids, 1, src_row, 1);
    S.cls = rows;
    for (int step = 1; step <= max_new; ++step) {
        for (int r = 0; r < rows; ++r) {
            log_softmax_row(S.logits + (size_t)r * V, V, lp_row, tmp);
            topk_row(lp_row, V, k, vals + (size_t)r * k, idx + (size_t)r * k);
        }
        int nr = 0;
        for (int s = 0; s < b; ++s) {
            int nc = 0;
            for (int bi = 0; bi < n_alive[s]; ++bi) {
                int row = s * k + bi;
                for (int j = 0; j < k; ++j) {
                    cands[nc].score = alive_score[row] + vals[(size_t)row * k + j];
                    cands[nc].beam = bi;
                    cands[nc].tok = idx[(size_t)row * k + j];
                    ++nc;
                }
            }
            /* stable sort, descending */
            for (int i = 1; i < nc; ++i) {
                cand_t t = cands[i];
                int q = i - 1;
                while (q >= 0 && cand_cmp(&cands[q], &t) > 0) { cands[q + 1] = cands[q]; --q; }
                cands[q + 1] = t;
            }
            int na = 0;
            for (int ci = 0; ci < nc && na < k; ++ci) {
                cand_t *cd = &cands[ci];
                int src = s * k + cd->beam;
                if (cd->tok == eos || step == max_new) {
                    if (!is_done[s] && n_done[s] < cap_done) {
                        int dl = alive_len[src];
                        uint32_t *dt = done_tok + ((size_t)s * cap_done + n_done[s]) * (max_new + 1);
                        memcpy(dt, alive_tok + (size_t)src * (max_new + 1), dl * sizeof(uint32_t));
                        if (cd->tok != eos) dt[dl++] = cd->tok;
                        float pen = powf((float)(dl + 1 > 1 ? dl + 1 : 1), lp);
                        done_score[(size_t)s * cap_done + n_done[s]] = cd->score / pen;
                        done_len[(size_t)s * cap_done + n_done[s]] = dl;
                        ++n_done[s];
                    }
                    continue;
                }
                int dst = s * k + na;
                memcpy(ntok + (size_t)dst * (max_new + 1), alive_tok + (size_t)src * (max_new + 1),
                       alive_len[src] * sizeof(uint32_t));
                ntok[(size_t)dst * (max_new + 1) + alive_len[src]] = cd->tok;
                nlen[dst] = alive_len[src] + 1;
                nscore[dst] = cd->score;
                reorder[nr] = src;
                next[nr] = cd->tok;
                ++nr;
                ++na;
            }
            float best_done = -INFINITY;
            for (int q = 0; q < n_done[s]; ++q) best_done = fmaxf(best_done, done_score[(size_t)s * cap_done + q]);
            float best_alive = na > 0 ? nscore[s * k] / powf((float)(step + 1), lp) : -INFINITY;
            if (n_done[s] >= k && best_done >= best_alive) is_done[s] = 1;
            while (na < k) {
                int dst = s * k + na;
                reorder[nr] = s * k;
                next[nr] = eos;
                ++nr;
                nscore[dst] = -INFINITY;
                nlen[dst] = 0;
                ++na;
            }
            n_alive[s] = k;
        }
        memcpy(alive_score, nscore, rows * sizeof(float));
        memcpy(alive_tok, ntok, (size_t)rows * (max_new + 1) * sizeof(uint32_t));
        memcpy(alive_len, nlen, rows * sizeof(int));
        int all = 1;
        for (int s = 0; s < b; ++s) all &= is_done[s];
        if (step == max_new || all) break;
        /* reorder the self-attention caches (DecoderState::reorder, model.rs:209-226) */
        size_t per_row = (size_t)c->d * m;
        for (int l = 0; l < c->dec_layers; ++l) {
            float *kc = S.kc + (size_t)l * rows * per_row, *vc = S.vc + (size_t)l * rows * per_row;
            float *kb = kbuf + (size_t)l * rows * per_row;
            for (int r = 0; r < rows; ++r) memcpy(kb + r * per_row, kc + (size_t)reorder[r] * per_row, per_row * 4);
            memcpy(kc, kb, rows * per_row * 4);
            for (int r = 0; r < rows; ++r) memcpy(kb + r * per_row, vc + (size_t)reorder[r] * per_row, per_row * 4);
            memcpy(vc, kb, rows * per_row * 4);
        }
        /* src_row is unchanged by reordering within a sentence */
        memcpy(ids, next, rows * sizeof(uint32_t));
        dec_step(M, E, &S, ids, step + 1, src_row, 1);
    }
    for (int s = 0; s < b; ++s) {
        int best = -1;
        float bs = -INFINITY;
        if (n_done[s] > 0) {
            for (int q = 0; q < n_done[s]; ++q) {
                float v = done_score[(size_t)s * cap_done + q];
                if (best < 0 || v >= bs) { bs = v; best = q; } /* max_by: last maximum wins */
            }
            out_len[s] = (uint32_t)done_len[(size_t)s * cap_done + best];
            for (int t = 0; t < max_new; ++t)
                out[(size_t)s * max_new + t] = t < (int)out_len[s]
                    ? done_tok[((size_t)s * cap_done + best) * (max_new + 1) + t] : (uint32_t)c->pad;
        } else {
            for (int bi = 0; bi < k; ++bi) {
                float v = alive_score[s * k + bi];
                if (best < 0 || v >= bs) { bs = v; best = bi; }
            }
            int row = s * k + best;
            out_len[s] = (uint32_t)alive_len[row];
            for (int t = 0; t < max_new; ++t)
                out[(size_t)s * max_new + t] = t < alive_len[row] ? alive_tok[(size_t)row * (max_new + 1) + t]
                                                                   : (uint32_t)c->pad;
        }
    }
    free(src_row); free(ids); free(alive_score); free(alive_tok); free(alive_len); free(n_alive);
    free(done_score); free(done_tok); free(done_len); free(n_done); free(is_done); free(lp_row); free(tmp);
    free(vals); free(idx); free(cands); free(reorder); free(next); free(nscore); free(ntok); free(nlen); free(kbuf);
    dstate_free(&S);
    return 0;
}

ORC_EXPORT int orc_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Threads of the following parallel regions (a launcher may have set
 * OMP_NUM_THREADS=1 for its processes). */
ORC_EXPORT void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
