/*
 * Oracle (plain C): dequantisers and the RoPE table of the N730 hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg load the library built from this file.
 *
 * Per-tensor dequant restates src-code/cpp/n730core.cpp:57-142:
 *   dst[i] = ((float)q - zero_point) * scale       (fp32, no contraction)
 * INT4: low nibble first; INT2: four crumbs, least-significant first;
 * FP16: bit-level half -> float conversion (n730core.cpp:105-131 semantics,
 * written here from the IEEE-754 binary16 definition).
 *
 * Group-wise dequant (format extension): the same per-element formula with
 * the group's fp16 scale and fp16 zero converted to fp32.
 *
 * RoPE table restates src-code/cpp/n730_cuda.cu:650-661 on the host:
 *   freq = 1/powf(theta, (float)(2i)/hd); angle = pos*freq; cosf/sinf(angle).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

float oracle_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    int32_t e = (h >> 10) & 0x1F;
    uint32_t m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {               /* subnormal: normalise */
            int32_t shift = 0;
            while (!(m & 0x400u)) { m <<= 1; ++shift; }
            m &= 0x3FFu;
            bits = sign | ((uint32_t)(127 - 15 + 1 - shift) << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((uint32_t)(e - 15 + 127) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static inline uint32_t code_at(const uint8_t *raw, int bits, int64_t i) {
    if (bits == 8) return raw[i];
    int per = 8 / bits;
    uint8_t b = raw[i / per];
    return (b >> (bits * (int)(i % per))) & ((1u << bits) - 1u);
}

/* prec: 2, 4, 8 or 16 (per-tensor formats of the reference). */
int oracle_dequant_tensor(const uint8_t *raw, int prec, int64_t n,
                          float scale, float zp, float *out) {
    if (prec == 16) {
        const uint16_t *h = (const uint16_t *)raw;
        for (int64_t i = 0; i < n; ++i) out[i] = oracle_half_to_float(h[i]);
        return 0;
    }
    if (prec != 2 && prec != 4 && prec != 8) return -5;
    for (int64_t i = 0; i < n; ++i) {
        volatile float d = (float)code_at(raw, prec, i) - zp;  /* keep sub and mul separate */
        out[i] = d * scale;
    }
    return 0;
}

/* Grouped: codes are [rows, cols] packed row-major; scales/zeros [rows, cols/group] fp16. */
int oracle_dequant_grouped(const uint8_t *codes, const uint16_t *s16, const uint16_t *z16,
                           int bits, int64_t rows, int64_t cols, int64_t group, float *out) {
    if (bits != 2 && bits != 4 && bits != 8) return -5;
    if (group <= 0 || cols % group) return -4;
    int64_t G = cols / group;
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t c = 0; c < cols; ++c) {
            int64_t gi = r * G + c / group;
            float s = oracle_half_to_float(s16[gi]);
            float z = oracle_half_to_float(z16[gi]);
            volatile float d = (float)code_at(codes, bits, r * cols + c) - z;
            out[r * cols + c] = d * s;
        }
    }
    return 0;
}

void oracle_rope_table(int max_pos, int head_dim, float theta, float *cos_out, float *sin_out) {
    int h2 = head_dim / 2;
    for (int pos = 0; pos < max_pos; ++pos) {
        for (int i = 0; i < h2; ++i) {
            float freq = 1.0f / powf(theta, (float)(2 * i) / head_dim);
            float angle = pos * freq;
            cos_out[(int64_t)pos * h2 + i] = cosf(angle);
            sin_out[(int64_t)pos * h2 + i] = sinf(angle);
        }
    }
}
