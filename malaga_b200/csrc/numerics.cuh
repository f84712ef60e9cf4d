// Device-side arithmetic shared by every kernel of the decode engine.
//
// The engine computes in a fixed, reproducible order so that its tokens and
// logits are bit-identical to the CPU restatement it is tested against:
//   * warp_sum32: lane l first sums its own elements left to right, then lanes
//     are added pairwise at distances 1, 2, 4, 8, 16 (acc[l] + acc[l^o]).
//   * a matmul row is the same pairwise tree over per-32-block partials, lane l
//     owning blocks [l*G, (l+1)*G) (G = blocks/32), summed left to right.
//   * FMA only where written as __fmaf_rn: the library is compiled with
//     -fmad=false, every other multiply/add is rounded on its own.
//   * exp / log are this file's own (Cody-Waite argument reduction + Taylor /
//     atanh series), not the CUDA math library.
// The reference leaves these orders to candle's kernels (candle-core 0.11.0,
// CUDA QMatMul = llama.cpp MMVQ/MMQ with q8_1 activations; not in the
// reference tree), see crates/malaga-core/src/model.rs:571-607.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace mgb {

#define kNegInf (-__int_as_float(0x7f800000))

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }
__device__ __forceinline__ float round_h(float f) { return __half2float(__float2half_rn(f)); }

// e^x: x = k ln2 + r with a two-constant ln2 split (Cody & Waite), e^r by its
// Taylor series to degree 7 (|r| <= ln2/2, truncation < 1e-8 relative), and an
// exact 2^k scaling. Inputs here are <= 0 (softmax arguments).
__device__ __forceinline__ float mgb_exp(float x) {
    if (!(x > -104.0f)) return 0.0f;
    if (x > 88.7f) return __int_as_float(0x7f800000);
    const float k = rintf(__fmul_rn(x, 1.44269502162933350f));
    float r = __fmaf_rn(-k, 0.693145751953125f, x);
    r = __fmaf_rn(-k, 1.428606765330187e-06f, r);
    float p = 1.98412701138295233e-04f;
    p = __fmaf_rn(p, r, 1.38888892251998186e-03f);
    p = __fmaf_rn(p, r, 8.33333376795053482e-03f);
    p = __fmaf_rn(p, r, 4.16666679084300995e-02f);
    p = __fmaf_rn(p, r, 1.66666671633720398e-01f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ki = (int)k;
    if (ki >= -126) return __fmul_rn(p, __int_as_float((ki + 127) << 23));
    return __fmul_rn(__fmul_rn(p, __int_as_float((ki + 227) << 23)), __int_as_float(27 << 23));
}

// ln x: x = 2^e f, f in [sqrt(1/2), sqrt(2)); ln f = 2 atanh(z), z = (f-1)/(f+1),
// odd series to z^13; plus e ln2 with the same two-constant split.
__device__ __forceinline__ float mgb_log(float x) {
    if (!(x > 0.0f)) return x == 0.0f ? kNegInf : __int_as_float(0x7fc00000);
    if (isinf(x)) return x;
    uint32_t b = __float_as_uint(x);
    int e = 0;
    if (b < 0x00800000u) {
        b = __float_as_uint(__fmul_rn(x, 4294967296.0f));
        e = -32;
    }
    e += (int)(b >> 23) - 127;
    float f = __uint_as_float((b & 0x007fffffu) | 0x3f800000u);
    if (f > 1.41421353816986084f) {
        f = __fmul_rn(f, 0.5f);
        e += 1;
    }
    const float z = __fdiv_rn(__fsub_rn(f, 1.0f), __fadd_rn(f, 1.0f));
    const float z2 = __fmul_rn(z, z);
    float p = 0.153846159577369690f;
    p = __fmaf_rn(p, z2, 0.181818187236785889f);
    p = __fmaf_rn(p, z2, 0.222222223877906799f);
    p = __fmaf_rn(p, z2, 0.285714298486709595f);
    p = __fmaf_rn(p, z2, 0.400000005960464478f);
    p = __fmaf_rn(p, z2, 0.666666686534881592f);
    p = __fmaf_rn(p, z2, 2.0f);
    const float lf = __fmul_rn(p, z);
    const float fe = (float)e;
    return __fmaf_rn(fe, 0.693145751953125f, __fmaf_rn(fe, 1.428606765330187e-06f, lf));
}

// Pairwise butterfly at distances 1..16: every lane ends with the same value.
__device__ __forceinline__ float warp_tree(float v) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// The reference kernels' warp sum (llama.cpp / candle warp_reduce_sum):
// x += shfl_xor(x, m) for m = 16, 8, 4, 2, 1; every lane ends with the result.
__device__ __forceinline__ float warp_sum_bf(float v) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Max of non-negative floats across the warp in one reduction instruction
// (their bit patterns order like the values).
__device__ __forceinline__ float warp_max_nonneg(float v) {
    return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(v)));
}

// q8_1 quantization of one 32-value block held one value per lane (lane =
// position), as candle-kernels' quantize_q8_1: amax = max |x|, s = warp sum of
// x (warp_sum_bf), d = amax / 127, q = amax == 0 ? 0 : roundf(x / d) (IEEE
// division, halves away from zero). Returns q; d and s come back rounded to
// f16 (the values the matmuls read), identical in every lane.
__device__ __forceinline__ int q81_block(float x, float &d, float &s) {
    const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(x))));
    s = round_h(warp_sum_bf(x));
    const float dd = __fdiv_rn(amax, 127.0f);
    d = round_h(dd);
    return amax == 0.0f ? 0 : (int)roundf(__fdiv_rn(x, dd));
}

// Packed pairs of f32 operations (sm_100 f32x2): each element is rounded
// exactly as the scalar __fmaf_rn / __fmul_rn would round it.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 pa, pb, pc, pd;\n\t"
        "mov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\tmov.b64 pc, {%6, %7};\n\t"
        "fma.rn.f32x2 pd, pa, pb, pc;\n\tmov.b64 {%0, %1}, pd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 pa, pb, pd;\n\t"
        "mov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\t"
        "mul.rn.f32x2 pd, pa, pb;\n\tmov.b64 {%0, %1}, pd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

__device__ __forceinline__ float2 add2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 pa, pb, pd;\n\t"
        "mov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\t"
        "add.rn.f32x2 pd, pa, pb;\n\tmov.b64 {%0, %1}, pd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// Integer sum across the warp, one reduction instruction.
__device__ __forceinline__ int warp_isum_redux(int v) { return __reduce_add_sync(0xffffffffu, v); }

__device__ __forceinline__ int warp_isum(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// (value, index) argmax merge: larger value wins, lower index on ties.
__device__ __forceinline__ void argmax_merge(float &v, uint32_t &i, float ov, uint32_t oi) {
    if (ov > v || (ov == v && oi < i)) {
        v = ov;
        i = oi;
    }
}

__device__ __forceinline__ void warp_argmax(float &v, uint32_t &i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, i, o);
        argmax_merge(v, i, ov, oi);
    }
}

}  // namespace mgb
