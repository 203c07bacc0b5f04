/*
 * CPU oracle for nvcr.fx.v1: the profile's integer ops restated in plain C.
 * TEST INFRASTRUCTURE ONLY (see fx_oracle.h): the product never links or
 * calls this file.
 *
 * The loops visit outputs in the reference's order (fx.cpp), so that when an
 * op fails, the status names the rule the reference hits first.
 */
#include "fx_oracle.h"

/* floor(a / 2^s) for s >= 1, written without relying on the sign behaviour of >>. */
static int64_t floor_shift(int64_t a, int s) {
    if (a >= 0) return a >> s;
    const int64_t magnitude = -a;  /* |a| < 2^62 under the profile's bounds */
    return -((magnitude + ((INT64_C(1) << s) - 1)) >> s);
}

int64_t fx_rsr(int64_t a, int s) {
    if (s == 0) return a;
    return floor_shift(a + (INT64_C(1) << (s - 1)), s);
}

int64_t fx_delta_act(int64_t r, int64_t h, int shift, const int16_t *dc) {
    const int64_t base = r > 0 ? r : 0;
    if (r < -h || r > h) return base;
    return base + dc[(r + h) >> shift];  /* r + h >= 0 here */
}

static int stored(int64_t v, int32_t *out) {
    if (v > FX_STORED_MAX || v < -FX_STORED_MAX) return 0;
    *out = (int32_t)v;
    return 1;
}

static int64_t clamp64(int64_t v, int64_t lo, int64_t hi) {
    return v < lo ? lo : v > hi ? hi : v;
}

int fx_gemm(int32_t in_channels, int32_t out_channels, int group, int input_shift,
            const int32_t *weights, const int64_t *bias, const int32_t *shift,
            int64_t table_h, int table_shift, const int16_t *dc,
            const int32_t *x, size_t pixels, int residual_count, const int32_t *const *residuals,
            int32_t *y) {
    const int32_t groups = out_channels / group;
    for (size_t p = 0; p < pixels; ++p) {
        for (int32_t g = 0; g < groups; ++g) {
            int64_t sum = 0;
            for (int j = 0; j < group; ++j) {
                const size_t o = (size_t)g * (size_t)group + (size_t)j;
                int64_t acc = bias[o];
                const int32_t *row = weights + o * (size_t)in_channels;
                for (int32_t k = 0; k < in_channels; ++k) {
                    const int64_t digits = clamp64(fx_rsr(x[(size_t)k * pixels + p], input_shift),
                                                   -FX_DIGIT2_MAX, FX_DIGIT2_MAX);
                    acc += (int64_t)row[k] * digits;
                }
                const int64_t r = fx_rsr(acc, shift[o]);
                if (r >= FX_GEMM_LIMIT || r <= -FX_GEMM_LIMIT) return FX_GEMM_PRE_ACTIVATION;
                sum += dc != NULL ? fx_delta_act(r, table_h, table_shift, dc) : r;
            }
            const size_t at = (size_t)g * pixels + p;
            for (int i = 0; i < residual_count; ++i) sum += residuals[i][at];
            if (!stored(sum, &y[at])) return FX_STORED_BOUND;
        }
    }
    return FX_OK;
}

int fx_depthwise3x3(int32_t channels, int32_t height, int32_t width, const int32_t *weights,
                    const int64_t *bias, const int32_t *shift, const int32_t *x, int32_t *y) {
    const size_t plane = (size_t)height * (size_t)width;
    for (int32_t c = 0; c < channels; ++c) {
        const int32_t *taps = weights + (size_t)c * 9;
        const int32_t *src = x + (size_t)c * plane;
        for (int32_t row = 0; row < height; ++row) {
            for (int32_t col = 0; col < width; ++col) {
                int64_t acc = bias[c];
                for (int i = 0; i < 3; ++i) {
                    const int32_t yy = row + i - 1;
                    if (yy < 0 || yy >= height) continue;
                    for (int j = 0; j < 3; ++j) {
                        const int32_t xx = col + j - 1;
                        if (xx < 0 || xx >= width) continue;
                        acc += (int64_t)taps[i * 3 + j] * src[(size_t)yy * (size_t)width + (size_t)xx];
                    }
                }
                const size_t at = (size_t)c * plane + (size_t)row * (size_t)width + (size_t)col;
                if (!stored(fx_rsr(acc, shift[c]), &y[at])) return FX_STORED_BOUND;
            }
        }
    }
    return FX_OK;
}

int fx_mul(const int32_t *a, int32_t channels, size_t pixels, const int32_t *b, int32_t b_channels,
           size_t b_pixels, int shift, int32_t *y) {
    for (int32_t c = 0; c < channels; ++c) {
        const size_t bc = b_channels == 1 ? 0 : (size_t)c;
        for (size_t p = 0; p < pixels; ++p) {
            const size_t i = (size_t)c * pixels + p;
            const int64_t product = (int64_t)a[i] * b[bc * b_pixels + (b_pixels == 1 ? 0 : p)];
            if (!stored(fx_rsr(product, shift), &y[i])) return FX_STORED_BOUND;
        }
    }
    return FX_OK;
}

int fx_affine(const int32_t *x, size_t count, int64_t alpha, int64_t beta, int shift, int32_t *y) {
    for (size_t i = 0; i < count; ++i) {
        if (!stored(fx_rsr(alpha * x[i] + beta, shift), &y[i])) return FX_STORED_BOUND;
    }
    return FX_OK;
}

int fx_add(const int32_t *a, const int32_t *b, size_t count, int32_t *y) {
    for (size_t i = 0; i < count; ++i) {
        if (!stored((int64_t)a[i] + b[i], &y[i])) return FX_STORED_BOUND;
    }
    return FX_OK;
}

void fx_sat_table(const int32_t *x, size_t count, const int32_t *table, size_t table_size, int32_t top,
                  int32_t *y) {
    const int64_t n = (int64_t)(table_size / 2);
    for (size_t i = 0; i < count; ++i) {
        const int64_t v = x[i];
        y[i] = v >= n ? top : v < -n ? 0 : table[v + n];
    }
}

void fx_delta(const int32_t *x, size_t count, int64_t h, int shift, const int16_t *dc, int32_t *y) {
    for (size_t i = 0; i < count; ++i) y[i] = (int32_t)fx_delta_act(x[i], h, shift, dc);
}

void fx_clamp(const int32_t *x, size_t count, int32_t lo, int32_t hi, int32_t *y) {
    for (size_t i = 0; i < count; ++i) y[i] = x[i] < lo ? lo : x[i] > hi ? hi : x[i];
}
