/*
 * CPU oracle for the nvcr.fx.v1 fixed-point profile.
 *
 * TEST INFRASTRUCTURE ONLY. A plain-C restatement of the profile's integer
 * ops (reference: docs/spec/numerics-fx-v1.md sections 3-5, and the
 * reference's CPU arithmetic src/deterministic/fx.cpp). Only tests/ may load
 * it, and only as the checker; the product never links, loads or calls it.
 *
 * Tensors are batch-1 NCHW int32 arrays; every sum is taken in int64, which
 * the profile's load-time bounds make exact (spec section 5).
 *
 * Parity pin: tests/test_fx_oracle.py checks these functions against the
 * hand-computed vectors of the reference's own test (tests/fx_reference_tests.cpp)
 * and, value for value and failure for failure, against the reference's
 * fx.cpp and fx_program.cpp compiled from its sources into oracle/_ref.
 */
#ifndef NVCR_FX_ORACLE_H
#define NVCR_FX_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Largest magnitude of two balanced int8 digits, (256^2 - 1) * 127 / 255. */
#define FX_DIGIT2_MAX 32639
/* Bound on every stored value: |v| <= 2^30. */
#define FX_STORED_MAX (INT64_C(1) << 30)
/* A gemm pre-activation must satisfy |r| < 2^29 - 1. */
#define FX_GEMM_LIMIT ((INT64_C(1) << 29) - 1)

/* Status of an op: success, or which of the profile's failure rules fired
 * first in the reference's loop order (fx.cpp:38-61 and its store checks). */
enum fx_status {
    FX_OK = 0,
    FX_GEMM_PRE_ACTIVATION = 1, /* |r| >= 2^29 - 1 */
    FX_STORED_BOUND = 2         /* a written value outside [-2^30, 2^30] */
};

/* rsr(a, s): a for s = 0, floor((a + 2^(s-1)) / 2^s) for s >= 1 (spec section 3). */
int64_t fx_rsr(int64_t a, int s);

/* Bounded delta table act(r) (spec 4.5; fx.cpp:33-37): dc holds ((2h) >> shift) + 1 entries. */
int64_t fx_delta_act(int64_t r, int64_t h, int shift, const int16_t *dc);

/* 1x1 gemm (spec 4.1; fx.cpp:39-61). x is [in][pixels]; weights [out][in];
 * bias, shift [out]; residuals are [out / group][pixels] each; y is
 * [out / group][pixels]. dc is NULL when there is no table activation. */
int fx_gemm(int32_t in_channels, int32_t out_channels, int group, int input_shift,
            const int32_t *weights, const int64_t *bias, const int32_t *shift,
            int64_t table_h, int table_shift, const int16_t *dc,
            const int32_t *x, size_t pixels, int residual_count, const int32_t *const *residuals,
            int32_t *y);

/* depthwise 3x3, stride 1, zero padding 1 (spec 4.2; fx.cpp:63-86). */
int fx_depthwise3x3(int32_t channels, int32_t height, int32_t width, const int32_t *weights,
                    const int64_t *bias, const int32_t *shift, const int32_t *x, int32_t *y);

/* rsr(a * b, shift), b broadcast over channels (b_channels 1) and/or pixels
 * (b_pixels 1) (spec 4.3; fx.cpp:88-99). */
int fx_mul(const int32_t *a, int32_t channels, size_t pixels, const int32_t *b, int32_t b_channels,
           size_t b_pixels, int shift, int32_t *y);

/* rsr(alpha * x + beta, shift) (spec 4.6; fx.cpp:101-107). */
int fx_affine(const int32_t *x, size_t count, int64_t alpha, int64_t beta, int shift, int32_t *y);

/* a + b (spec 4.7; fx.cpp:109-115). */
int fx_add(const int32_t *a, const int32_t *b, size_t count, int32_t *y);

/* Saturating table: T[x + n] on [-n, n), top at or above n, 0 below -n; the
 * table holds 2n entries (spec 4.5; fx.cpp:117-125). Never fails. */
void fx_sat_table(const int32_t *x, size_t count, const int32_t *table, size_t table_size, int32_t top,
                  int32_t *y);

/* Standalone delta activation (fx.cpp:127-133). Never fails. */
void fx_delta(const int32_t *x, size_t count, int64_t h, int shift, const int16_t *dc, int32_t *y);

/* clamp(x, lo, hi) (fx.cpp:135-139). */
void fx_clamp(const int32_t *x, size_t count, int32_t lo, int32_t hi, int32_t *y);

#ifdef __cplusplus
}
#endif

#endif
