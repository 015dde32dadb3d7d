/*
 * CPU oracle for the quantized-linear path: TEST INFRASTRUCTURE ONLY (see oracle.h).
 * Compiled with -ffp-contract=off so that every multiply and add rounds on its own, as the
 * reference's vDSP calls do (Widen.swift:94-97).
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* Forge/Numerics.swift:49-55: bias 7, no infinity, S.1111.111 is NaN, subnormals m/8 * 2^-6. */
float orc_e4m3_to_f32(uint8_t b) {
    const float sign = (b & 0x80) ? -1.0f : 1.0f;
    const int e = (b >> 3) & 0xF, m = b & 0x7;
    if (e == 0xF && m == 0x7) return bits_f32(0x7FC00000u);   /* Float.nan, either sign */
    if (e == 0) return sign * ldexpf((float)m / 8.0f, -6);
    return sign * ldexpf(1.0f + (float)m / 8.0f, e - 7);
}

void orc_e4m3_table(float out[256]) {
    for (int b = 0; b < 256; ++b) out[b] = orc_e4m3_to_f32((uint8_t)b);
}

/* IEEE binary16: 1 sign, 5 exponent (bias 15), 10 fraction bits; every value is an fp32. */
float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    const int e = (h >> 10) & 0x1F, f = h & 0x3FF;
    float v;
    if (e == 0x1F) return bits_f32(sign | 0x7F800000u | ((uint32_t)f << 13));
    if (e == 0) v = ldexpf((float)f, -24);
    else v = ldexpf(1.0f + (float)f / 1024.0f, e - 15);
    return bits_f32(f32_bits(v) | sign);
}

float orc_bf16_to_f32(uint16_t b) { return bits_f32((uint32_t)b << 16); }

/* TensorGEMMBF16.swift:43-47: NaN -> (u >> 16) | 0x40, otherwise round to nearest even. */
uint16_t orc_f32_to_bf16(float f) {
    const uint32_t u = f32_bits(f);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

void orc_f32_to_bf16_array(const float* in, uint16_t* out, int64_t count) {
    for (int64_t i = 0; i < count; ++i) out[i] = orc_f32_to_bf16(in[i]);
}

float orc_scale_at(const void* scales, int scale_dtype, int64_t i) {
    switch (scale_dtype) {
    case ORC_SCALE_F32: return ((const float*)scales)[i];
    case ORC_SCALE_BF16: return orc_bf16_to_f32(((const uint16_t*)scales)[i]);
    case ORC_SCALE_F16: return orc_f16_to_f32(((const uint16_t*)scales)[i]);
    default: return 1.0f;
    }
}

static float value_of(const uint8_t* values, int kind, int64_t i) {
    return kind == ORC_INT8 ? (float)(int8_t)values[i] : orc_e4m3_to_f32(values[i]);
}

void orc_dequantize(const uint8_t* values, int kind, int64_t count, const void* scales, int scale_dtype,
                    int layout, int64_t width, int64_t block, int64_t first_row, float* out) {
    if (count <= 0) return;
    if (scale_dtype == ORC_SCALE_NONE || scales == NULL) {
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < count; ++i) out[i] = value_of(values, kind, i);
        return;
    }
    switch (layout) {
    case ORC_LAYOUT_TENSOR: {
        const float s = orc_scale_at(scales, scale_dtype, 0);
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < count; ++i) out[i] = value_of(values, kind, i) * s;
        break;
    }
    case ORC_LAYOUT_COLUMNS: {
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < count; ++i) out[i] = value_of(values, kind, i) * orc_scale_at(scales, scale_dtype, i % width);
        break;
    }
    case ORC_LAYOUT_BLOCKS: {
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < count; ++i) {
            const int64_t row = first_row + i / width, col = i % width;
            out[i] = value_of(values, kind, i) * orc_scale_at(scales, scale_dtype, (row / block) * width + col);
        }
        break;
    }
    case ORC_LAYOUT_ROWS: {
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < count; ++i)
            out[i] = value_of(values, kind, i) * orc_scale_at(scales, scale_dtype, first_row + i / width);
        break;
    }
    default: break;
    }
}

/* c[r, :] = sum_k x[r, k] * w[k, :] in fp32, k ascending; four rows share each pass over w. */
static void gemm_rows_f32(const uint16_t* x, int64_t m, int64_t k, int64_t n, const float* w, float* c) {
    const int64_t groups = (m + 3) / 4;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t g = 0; g < groups; ++g) {
        const int64_t r0 = g * 4, rows = (m - r0) < 4 ? (m - r0) : 4;
        float* acc = c + r0 * n;
        memset(acc, 0, (size_t)(rows * n) * sizeof(float));
        for (int64_t kk = 0; kk < k; ++kk) {
            const float* wr = w + kk * n;
            for (int64_t r = 0; r < rows; ++r) {
                const float xv = orc_bf16_to_f32(x[(r0 + r) * k + kk]);
                float* a = acc + r * n;
                for (int64_t j = 0; j < n; ++j) a[j] = a[j] + xv * wr[j];
            }
        }
    }
}

static void finish(int64_t m, int64_t n, const float* s, const uint16_t* bias, float* c, uint16_t* y) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < m; ++r) {
        for (int64_t j = 0; j < n; ++j) {
            float v = c[r * n + j];
            if (s) v = v * s[j];
            if (bias) v = v + orc_bf16_to_f32(bias[j]);
            c[r * n + j] = v;
            if (y) y[r * n + j] = orc_f32_to_bf16(v);
        }
    }
}

void orc_linear_int8(const uint16_t* x, int64_t m, int64_t k, int64_t n, const int8_t* q, const float* s,
                     const uint16_t* bias, float* c, uint16_t* y) {
    float* qf = (float*)malloc((size_t)(k * n) * sizeof(float));
    if (!qf) return;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < k * n; ++i) qf[i] = (float)q[i];   /* exact */
    gemm_rows_f32(x, m, k, n, qf, c);
    free(qf);
    finish(m, n, s, bias, c, y);
}

void orc_linear_widened(const uint16_t* x, int64_t m, int64_t k, int64_t n, const float* w,
                        const uint16_t* bias, float* c, uint16_t* y) {
    gemm_rows_f32(x, m, k, n, w, c);
    finish(m, n, NULL, bias, c, y);
}

void orc_linear_fp64(const uint16_t* x, int64_t m, int64_t k, int64_t n, const float* w,
                     const uint16_t* bias, double* c) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t r = 0; r < m; ++r) {
        double* a = c + r * n;
        for (int64_t j = 0; j < n; ++j) a[j] = 0.0;
        for (int64_t kk = 0; kk < k; ++kk) {
            const double xv = (double)orc_bf16_to_f32(x[r * k + kk]);
            const float* wr = w + kk * n;
            for (int64_t j = 0; j < n; ++j) a[j] += xv * (double)wr[j];
        }
        if (bias)
            for (int64_t j = 0; j < n; ++j) a[j] += (double)orc_bf16_to_f32(bias[j]);
    }
}

void orc_gemv_int8_splits(const float* x, int64_t k, int64_t n, const int8_t* q, const float* s,
                          int64_t splits, float* parts, float* out) {
    /* DecodeKernels.swift:78-108: in split [k0, k1) eight simdgroups each accumulate, with a fused
     * multiply-add, the rows k0 + sg, k0 + sg + 8, ... in ascending order; the eight sums are then
     * added in the order sg = 0..7 starting from 0, and the column's scale multiplies the total. */
#pragma omp parallel for schedule(static)
    for (int64_t sp = 0; sp < splits; ++sp) {
        const int64_t k0 = sp * k / splits, k1 = (sp + 1) * k / splits;
        float* p = parts + sp * n;
        float* acc = (float*)calloc((size_t)(8 * n), sizeof(float));
        for (int sg = 0; sg < 8; ++sg)
            for (int64_t r = k0 + sg; r < k1; r += 8)
                for (int64_t j = 0; j < n; ++j)
                    acc[sg * n + j] = fmaf(x[r], (float)q[r * n + j], acc[sg * n + j]);
        for (int64_t j = 0; j < n; ++j) {
            float t = 0.0f;
            for (int sg = 0; sg < 8; ++sg) t = t + acc[sg * n + j];
            p[j] = t * s[j];
        }
        free(acc);
    }
    /* The consumer's sum of the partials: Qwen3VLDecoderTests.swift:215-217 adds them in fp64 in
     * split order and rounds once to fp32. */
    for (int64_t j = 0; j < n; ++j) {
        double t = 0.0;
        for (int64_t sp = 0; sp < splits; ++sp) t = t + (double)parts[sp * n + j];
        out[j] = (float)t;
    }
}

/* TensorGEMM.swift:183-201 (rotate_groups), operation for operation, on fp32 values. */
static void rotate_group_f32(float* v, int g) {
    for (int span = 1; span < g; span *= 4) {
        for (int t = 0; t < g / 4; ++t) {
            const int j = (t / span) * 4 * span + t % span;
            const float a = v[j], b = v[j + span], c = v[j + 2 * span], d = v[j + 3 * span];
            const float p = a + b, mm = a - b, u = c + d, w = c - d;
            v[j] = p + w;
            v[j + span] = p - w;
            v[j + 2 * span] = mm + u;
            v[j + 3 * span] = u - mm;
        }
    }
}

static float rotation_norm(int g) {
    int p = 0;
    while ((1 << (2 * p)) < g) ++p;          /* g = 4^p, sqrt(g) = 2^p */
    return ldexpf(1.0f, -p);
}

void orc_rotate_groups_bf16(const uint16_t* x, int64_t m, int64_t k, int group, uint16_t* out) {
    const float norm = rotation_norm(group);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < m; ++r) {
        float v[256];
        for (int64_t g0 = 0; g0 < k; g0 += group) {
            for (int i = 0; i < group; ++i) v[i] = orc_bf16_to_f32(x[r * k + g0 + i]);
            rotate_group_f32(v, group);
            for (int i = 0; i < group; ++i) out[r * k + g0 + i] = orc_f32_to_bf16(v[i] * norm);
        }
    }
}

/* Widen.hadamard (Widen.swift:550-566): m <- H . m, exact in int32. */
static void hadamard_i32(int32_t* v, int g) {
    for (int span = 1; span < g; span *= 4) {
        for (int base = 0; base < g; base += 4 * span) {
            for (int j = base; j < base + span; ++j) {
                const int32_t a = v[j], b = v[j + span], c = v[j + 2 * span], d = v[j + 3 * span];
                const int32_t p = a + b, mm = a - b, u = c + d, w = c - d;
                v[j] = p + w;
                v[j + span] = p - w;
                v[j + 2 * span] = mm + u;
                v[j + 3 * span] = u - mm;
            }
        }
    }
}

void orc_dequantize_rotated(const int8_t* q, int64_t k, int64_t n, int group, const float* s, float* out) {
    const float norm = rotation_norm(group);
#pragma omp parallel for schedule(static)
    for (int64_t j = 0; j < n; ++j) {
        int32_t v[256];
        const float factor = s[j] * norm;    /* exact: a power of two */
        for (int64_t g0 = 0; g0 < k; g0 += group) {
            for (int i = 0; i < group; ++i) v[i] = q[(g0 + i) * n + j];
            hadamard_i32(v, group);
            for (int i = 0; i < group; ++i) out[(g0 + i) * n + j] = (float)v[i] * factor;
        }
    }
}

void orc_w8a8_quantize(const float* x, int64_t m, int64_t k, int group, int8_t* codes, float* scales) {
    const float norm = group > 0 ? rotation_norm(group) : 1.0f;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < m; ++r) {
        float* y = (float*)malloc((size_t)k * sizeof(float));
        for (int64_t i = 0; i < k; ++i) y[i] = x[r * k + i];
        if (group > 0) {
            for (int64_t g0 = 0; g0 < k; g0 += group) {
                rotate_group_f32(y + g0, group);
                for (int i = 0; i < group; ++i) y[g0 + i] = y[g0 + i] * norm;
            }
        }
        float top = 0.0f;
        for (int64_t i = 0; i < k; ++i) top = fabsf(y[i]) > top ? fabsf(y[i]) : top;
        float scale = top / 127.0f;
        if (!(scale >= 1e-30f)) scale = 1e-30f;
        scales[r] = scale;
        for (int64_t i = 0; i < k; ++i) {
            float q = rintf(y[i] / scale);          /* default rounding mode: half to even */
            q = q < -128.0f ? -128.0f : (q > 127.0f ? 127.0f : q);
            codes[r * k + i] = (int8_t)q;
        }
        free(y);
    }
}

void orc_linear_w8a8(const int8_t* codes, const float* sx, int64_t m, int64_t k, int64_t n, const int8_t* q,
                     const float* sw, const uint16_t* bias, float* c, uint16_t* y) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < m; ++r) {
        int64_t* acc = (int64_t*)calloc((size_t)n, sizeof(int64_t));
        for (int64_t i = 0; i < k; ++i) {
            const int64_t a = codes[r * k + i];
            if (a == 0) continue;
            const int8_t* qr = q + i * n;
            for (int64_t j = 0; j < n; ++j) acc[j] += a * qr[j];
        }
        for (int64_t j = 0; j < n; ++j) {
            float v = (float)(int32_t)acc[j] * (sx[r] * sw[j]);
            if (bias) v = v + orc_bf16_to_f32(bias[j]);
            c[r * n + j] = v;
            if (y) y[r * n + j] = orc_f32_to_bf16(v);
        }
        free(acc);
    }
}

void orc_set_threads(int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
}

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
