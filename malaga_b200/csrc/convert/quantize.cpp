// Host-side GGUF block quantizers and the seeded weight generator used by the
// converter (malaga_b200/convert.py).
//
// Role in the reference: crates/malaga-core/src/convert.rs:128-136 calls
// candle's `QTensor::quantize` for every matmul weight, with the per-tensor
// types of convert.rs:67-91 and the fallback rule of convert.rs:150-162.
// candle-core 0.11.0 (absent from the reference tree) implements those
// quantizers after ggml. The block LAYOUTS written here are the published
// GGUF formats and are bit-compatible with any GGUF reader (the tests check
// them against gguf-py's dequantizer). The scale SEARCH is this project's own,
// simpler than ggml's iterative one: it produces valid blocks of the same
// type, but not byte-identical ones. Every parity check in this repository
// feeds the same GGUF file to both sides, so only the layout matters there.
//
// Formats (bytes per block):
//   Q8_0 : 32 values, {f16 d; int8 q[32]}                      = 34 B
//   Q4_K : 256 values, {f16 d; f16 dmin; u8 scales[12]; u8 qs[128]} = 144 B
//          value = d*sc_j*q - dmin*m_j, 8 sub-blocks of 32, 6-bit sc/m
//   Q6_K : 256 values, {u8 ql[128]; u8 qh[64]; i8 sc[16]; f16 d} = 210 B
//          value = d*sc_k*(q-32), 16 sub-blocks of 16, q 6-bit
#include <cmath>
#include <cstdint>
#include <cstring>

namespace {

// IEEE binary32 -> binary16, round to nearest even (with subnormals, inf/nan).
uint16_t f32_to_f16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) {  // inf or nan
        return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0u));
    }
    if (absx >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // rounds to >= 65520 -> inf
    if (absx < 0x38800000u) {                                      // below 2^-14: subnormal or zero
        if (absx < 0x33000000u) return (uint16_t)sign;            // < 2^-25 -> +-0
        // value = m * 2^(e-150); in units of the half subnormal step 2^-24 that is m * 2^(e-126).
        const uint32_t e = absx >> 23;
        const uint32_t m = (absx & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126 - e;
        uint32_t r = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1u))) ++r;
        return (uint16_t)(sign | r);
    }
    uint32_t h = ((absx - 0x38000000u) >> 13);  // rebias exponent 127 -> 15
    const uint32_t rem = absx & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu;
    const uint32_t m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {  // subnormal: normalise
            int sh = 0;
            uint32_t mm = m;
            while (!(mm & 0x400u)) { mm <<= 1; ++sh; }
            x = sign | ((uint32_t)(113 - sh) << 23) | ((mm & 0x3ffu) << 13);
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}

inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

void put_f16(uint8_t *p, float v) {
    const uint16_t h = f32_to_f16(v);
    p[0] = (uint8_t)(h & 0xff);
    p[1] = (uint8_t)(h >> 8);
}

void quantize_q8_0_block(const float *x, uint8_t *out) {
    float amax = 0.f;
    for (int i = 0; i < 32; ++i) amax = std::fmax(amax, std::fabs(x[i]));
    const float d = amax / 127.f;
    const float inv = d != 0.f ? 1.f / d : 0.f;
    put_f16(out, d);
    for (int i = 0; i < 32; ++i) out[2 + i] = (uint8_t)(int8_t)clampi((int)std::lround(x[i] * inv), -127, 127);
}

void quantize_q4_k_block(const float *x, uint8_t *out) {
    float scale[8], minv[8];
    for (int j = 0; j < 8; ++j) {
        float mn = 0.f, mx = 0.f;  // the min is clipped to <= 0 so that m_j >= 0
        for (int i = 0; i < 32; ++i) {
            mn = std::fmin(mn, x[32 * j + i]);
            mx = std::fmax(mx, x[32 * j + i]);
        }
        scale[j] = (mx - mn) / 15.f;
        minv[j] = -mn;
    }
    float smax = 0.f, mmax = 0.f;
    for (int j = 0; j < 8; ++j) {
        smax = std::fmax(smax, scale[j]);
        mmax = std::fmax(mmax, minv[j]);
    }
    const float d = smax / 63.f, dmin = mmax / 63.f;
    const float dh = f16_to_f32(f32_to_f16(d)), dminh = f16_to_f32(f32_to_f16(dmin));
    uint8_t sc[8], m[8];
    for (int j = 0; j < 8; ++j) {
        sc[j] = (uint8_t)(dh > 0.f ? clampi((int)std::lround(scale[j] / dh), 0, 63) : 0);
        m[j] = (uint8_t)(dminh > 0.f ? clampi((int)std::lround(minv[j] / dminh), 0, 63) : 0);
    }
    put_f16(out, d);
    put_f16(out + 2, dmin);
    uint8_t *s = out + 4;
    for (int j = 0; j < 4; ++j) {
        s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 0xf) | ((m[j + 4] & 0xf) << 4));
    }
    uint8_t q[256];
    for (int j = 0; j < 8; ++j) {
        const float ds = dh * (float)sc[j], dm = dminh * (float)m[j];
        for (int i = 0; i < 32; ++i) {
            const int v = ds > 0.f ? (int)std::lround((x[32 * j + i] + dm) / ds) : 0;
            q[32 * j + i] = (uint8_t)clampi(v, 0, 15);
        }
    }
    uint8_t *qs = out + 16;
    for (int c = 0; c < 4; ++c)
        for (int l = 0; l < 32; ++l) qs[32 * c + l] = (uint8_t)(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
}

void quantize_q6_k_block(const float *x, uint8_t *out) {
    float scale[16];
    float smax = 0.f;
    for (int k = 0; k < 16; ++k) {
        float amax = 0.f;
        for (int i = 0; i < 16; ++i) amax = std::fmax(amax, std::fabs(x[16 * k + i]));
        scale[k] = amax / 31.f;
        smax = std::fmax(smax, scale[k]);
    }
    const float d = smax / 127.f;
    const float dh = f16_to_f32(f32_to_f16(d));
    int8_t sc[16];
    for (int k = 0; k < 16; ++k) sc[k] = (int8_t)(dh > 0.f ? clampi((int)std::lround(scale[k] / dh), -128, 127) : 0);
    uint8_t q[256];
    for (int k = 0; k < 16; ++k) {
        const float ds = dh * (float)sc[k];
        for (int i = 0; i < 16; ++i) {
            const int v = ds != 0.f ? (int)std::lround(x[16 * k + i] / ds) : 0;
            q[16 * k + i] = (uint8_t)(clampi(v, -32, 31) + 32);
        }
    }
    uint8_t *ql = out, *qh = out + 128;
    for (int n = 0; n < 2; ++n) {
        for (int l = 0; l < 32; ++l) {
            const uint8_t q1 = q[128 * n + l], q2 = q[128 * n + 32 + l];
            const uint8_t q3 = q[128 * n + 64 + l], q4 = q[128 * n + 96 + l];
            ql[64 * n + l] = (uint8_t)((q1 & 0xf) | ((q3 & 0xf) << 4));
            ql[64 * n + 32 + l] = (uint8_t)((q2 & 0xf) | ((q4 & 0xf) << 4));
            qh[32 * n + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
        }
    }
    std::memcpy(out + 192, sc, 16);
    put_f16(out + 208, d);
}

// splitmix64: the standard 64-bit finaliser, used as a counter-based generator.
inline uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

}  // namespace

extern "C" {

// Bytes of one row of `n` values of GGML type `type` (0 F32, 1 F16, 8 Q8_0,
// 12 Q4_K, 14 Q6_K), or 0 when `n` is not a whole number of blocks.
long mgbc_row_bytes(int type, long n) {
    switch (type) {
        case 0: return 4 * n;
        case 1: return 2 * n;
        case 8: return n % 32 ? 0 : n / 32 * 34;
        case 12: return n % 256 ? 0 : n / 256 * 144;
        case 14: return n % 256 ? 0 : n / 256 * 210;
        default: return 0;
    }
}

// Quantizes `rows` rows of `n` f32 values into GGML blocks of `type`.
// Returns 0 on success, -1 for an unsupported type or row length.
int mgbc_quantize(int type, const float *x, long rows, long n, uint8_t *out) {
    const long rb = mgbc_row_bytes(type, n);
    if (rb == 0) return -1;
#pragma omp parallel for schedule(static)
    for (long r = 0; r < rows; ++r) {
        const float *xr = x + r * n;
        uint8_t *o = out + r * rb;
        switch (type) {
            case 0: std::memcpy(o, xr, 4 * n); break;
            case 1:
                for (long i = 0; i < n; ++i) put_f16(o + 2 * i, xr[i]);
                break;
            case 8:
                for (long b = 0; b < n / 32; ++b) quantize_q8_0_block(xr + 32 * b, o + 34 * b);
                break;
            case 12:
                for (long b = 0; b < n / 256; ++b) quantize_q4_k_block(xr + 256 * b, o + 144 * b);
                break;
            case 14:
                for (long b = 0; b < n / 256; ++b) quantize_q6_k_block(xr + 256 * b, o + 210 * b);
                break;
        }
    }
    return 0;
}

// Seeded N(0, std) values: element i of stream `stream` is a pure function of
// (seed, stream, i), so the output does not depend on the thread count.
// Box-Muller on two 53-bit uniforms drawn from splitmix64(counter).
void mgbc_normal(float *out, long n, uint64_t seed, uint64_t stream, float stdv) {
    const uint64_t key = mix64(seed * 0x100000001b3ull ^ mix64(stream + 0x51ed2701ull));
#pragma omp parallel for schedule(static)
    for (long p = 0; p < (n + 1) / 2; ++p) {
        const uint64_t a = mix64(key ^ (2 * (uint64_t)p));
        const uint64_t b = mix64(key ^ (2 * (uint64_t)p + 1));
        const double u1 = ((double)(a >> 11) + 1.0) * (1.0 / 9007199254740992.0);  // (0, 1]
        const double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);          // [0, 1)
        const double r = std::sqrt(-2.0 * std::log(u1));
        const double t = 6.283185307179586 * u2;
        out[2 * p] = (float)(stdv * r * std::cos(t));
        if (2 * p + 1 < n) out[2 * p + 1] = (float)(stdv * r * std::sin(t));
    }
}

// Seeded uniform integers in [lo, hi): same counter construction.
void mgbc_uniform_u32(uint32_t *out, long n, uint64_t seed, uint64_t stream, uint32_t lo, uint32_t hi) {
    const uint64_t key = mix64(seed * 0x100000001b3ull ^ mix64(stream + 0x2545f491ull));
    const uint64_t span = hi > lo ? (uint64_t)(hi - lo) : 1;
    for (long i = 0; i < n; ++i) out[i] = lo + (uint32_t)(mix64(key ^ (uint64_t)i) % span);
}

uint16_t mgbc_f32_to_f16(float f) { return f32_to_f16(f); }
float mgbc_f16_to_f32(uint16_t h) { return f16_to_f32(h); }

}  // extern "C"
