#pragma once

// The per-element work of the nvcr.fx.v1 kernels (k_fx.cu): one output value
// (or, for the gemm, one pixel's tile of four output groups) per call, with
// the index arithmetic and the integer arithmetic of the profile
// (docs/spec/numerics-fx-v1.md section 4; reference src/deterministic/fx.cpp).
// The kernels are grid-stride loops over these functions. They are also
// compiled for the host, so that a host build of the same code can be checked
// against the CPU oracle where no GPU is at hand.
//
// `record(key)` notes a stage failure; the kernels pass an atomicMin on the
// run's failure word (key layout in fx_kernels.hpp).

#include "fx_kernels.hpp"

#if defined(__CUDACC__)
#define FX_HD __host__ __device__ __forceinline__
#else
#define FX_HD inline
#endif

namespace nvcr_sm100::fx::elements {

inline constexpr std::int64_t digit2_max = 32639;
inline constexpr std::int64_t stored_max = std::int64_t{1} << 30;
inline constexpr std::int64_t gemm_limit = (std::int64_t{1} << 29) - 1;
inline constexpr int gemm_groups = 4;  // output groups per gemm tile

// rsr(a, s) = a for s = 0, floor((a + 2^(s-1)) / 2^s) otherwise (>> on a
// signed operand is an arithmetic shift).
FX_HD std::int64_t rsr(std::int64_t a, int s) { return s == 0 ? a : (a + (std::int64_t{1} << (s - 1))) >> s; }

FX_HD std::int64_t delta_act(std::int64_t r, const kernels::Table& table) {
    const std::int64_t base = r > 0 ? r : 0;
    if (r < -table.h || r > table.h) return base;
    return base + table.dc[(r + table.h) >> table.shift];
}

FX_HD bool outside_stored(std::int64_t v) { return v > stored_max || v < -stored_max; }

#if defined(__CUDACC__)
#pragma nv_exec_check_disable
#endif
template <class Record>
FX_HD void check_input(const std::int32_t* x, std::size_t i, unsigned long long base, const Record& record) {
    if (outside_stored(x[i])) record((base + i) << 1);
}

// One pixel p, output groups [g0, g0 + 4) clipped to the group count: the
// rounded, saturated input digit is formed once per input channel and reused
// for all 4 * G rows.
#if defined(__CUDACC__)
#pragma nv_exec_check_disable
#endif
template <int G, class Record>
FX_HD void gemm_tile(const kernels::GemmArgs& a, std::size_t p, int g0, unsigned long long node_key,
                     const Record& record) {
    constexpr int rows = gemm_groups * G;
    const int owned = a.groups - g0 < gemm_groups ? a.groups - g0 : gemm_groups;  // >= 1 for g0 < groups
    std::int64_t acc[rows];
#pragma unroll
    for (int r = 0; r < rows; ++r) acc[r] = 0;
    const std::int16_t* w = a.weights + static_cast<std::size_t>(g0) * G * a.in_channels;
    for (int k = 0; k < a.in_channels; ++k) {
        std::int64_t digit = rsr(a.x[static_cast<std::size_t>(k) * a.pixels + p], a.input_shift);
        digit = digit > digit2_max ? digit2_max : digit < -digit2_max ? -digit2_max : digit;
        const int xi = static_cast<int>(digit);
#pragma unroll
        for (int r = 0; r < rows; ++r) {
            if (r < owned * G) {
                const int wk = w[static_cast<std::size_t>(r) * a.in_channels + k];
                acc[r] += static_cast<std::int64_t>(wk) * xi;
            }
        }
    }
#pragma unroll
    for (int gi = 0; gi < gemm_groups; ++gi) {
        if (gi < owned) {
            const int g = g0 + gi;
            const unsigned long long position = static_cast<unsigned long long>(p) * a.groups + g;
            std::int64_t sum = 0;
#pragma unroll
            for (int j = 0; j < G; ++j) {
                const int o = g * G + j;
                const std::int64_t r = rsr(acc[gi * G + j] + a.bias[o], a.shifts[o]);
                if (r >= gemm_limit || r <= -gemm_limit) record(node_key | (position << 1));
                sum += a.table.dc != nullptr ? delta_act(r, a.table) : r;
            }
            const std::size_t at = static_cast<std::size_t>(g) * a.pixels + p;
            if (a.residual0 != nullptr) sum += a.residual0[at];
            if (a.residual1 != nullptr) sum += a.residual1[at];
            if (outside_stored(sum)) record(node_key | (position << 1) | 1u);
            a.y[at] = static_cast<std::int32_t>(sum);
        }
    }
}

#if defined(__CUDACC__)
#pragma nv_exec_check_disable
#endif
template <class Record>
FX_HD void depthwise3x3(const std::int32_t* x, int height, int width, const std::int32_t* weights,
                        const std::int64_t* bias, const std::int32_t* shifts, std::int32_t* y, std::size_t i,
                        unsigned long long node_key, const Record& record) {
    const std::size_t plane = static_cast<std::size_t>(height) * width;
    const int c = static_cast<int>(i / plane);
    const int row = static_cast<int>((i % plane) / width);
    const int col = static_cast<int>(i % width);
    const std::int32_t* src = x + static_cast<std::size_t>(c) * plane;
    const std::int32_t* taps = weights + static_cast<std::size_t>(c) * 9;
    std::int64_t acc = bias[c];
#pragma unroll
    for (int ti = 0; ti < 3; ++ti) {
        const int yy = row + ti - 1;
        if (yy < 0 || yy >= height) continue;
#pragma unroll
        for (int tj = 0; tj < 3; ++tj) {
            const int xx = col + tj - 1;
            if (xx < 0 || xx >= width) continue;
            acc += static_cast<std::int64_t>(taps[ti * 3 + tj]) * src[static_cast<std::size_t>(yy) * width + xx];
        }
    }
    const std::int64_t v = rsr(acc, shifts[c]);
    if (outside_stored(v)) record(node_key | (static_cast<unsigned long long>(i) << 1));
    y[i] = static_cast<std::int32_t>(v);
}

#if defined(__CUDACC__)
#pragma nv_exec_check_disable
#endif
template <class Record>
FX_HD void mul(const std::int32_t* a, std::size_t plane, const std::int32_t* b, int b_channels, std::size_t b_plane,
               int shift, std::int32_t* y, std::size_t i, unsigned long long node_key, const Record& record) {
    const std::size_t c = b_channels == 1 ? 0 : i / plane;
    const std::size_t p = b_plane == 1 ? 0 : i % plane;
    const std::int64_t v = rsr(static_cast<std::int64_t>(a[i]) * b[c * b_plane + p], shift);
    if (outside_stored(v)) record(node_key | (static_cast<unsigned long long>(i) << 1));
    y[i] = static_cast<std::int32_t>(v);
}

#if defined(__CUDACC__)
#pragma nv_exec_check_disable
#endif
template <class Record>
FX_HD void affine(const std::int32_t* x, std::int64_t alpha, std::int64_t beta, int shift, std::int32_t* y,
                  std::size_t i, unsigned long long node_key, const Record& record) {
    const std::int64_t v = rsr(alpha * x[i] + beta, shift);
    if (outside_stored(v)) record(node_key | (static_cast<unsigned long long>(i) << 1));
    y[i] = static_cast<std::int32_t>(v);
}

#if defined(__CUDACC__)
#pragma nv_exec_check_disable
#endif
template <class Record>
FX_HD void add(const std::int32_t* a, const std::int32_t* b, std::int32_t* y, std::size_t i,
               unsigned long long node_key, const Record& record) {
    const std::int64_t v = static_cast<std::int64_t>(a[i]) + b[i];
    if (outside_stored(v)) record(node_key | (static_cast<unsigned long long>(i) << 1));
    y[i] = static_cast<std::int32_t>(v);
}

FX_HD void sat_table(const std::int32_t* x, const std::int32_t* table, std::int64_t n, std::int32_t top,
                     std::int32_t* y, std::size_t i) {
    const std::int64_t v = x[i];
    y[i] = v >= n ? top : v < -n ? 0 : table[v + n];
}

FX_HD void delta(const std::int32_t* x, const kernels::Table& table, std::int32_t* y, std::size_t i) {
    y[i] = static_cast<std::int32_t>(delta_act(x[i], table));
}

FX_HD void clamp(const std::int32_t* x, std::int32_t lo, std::int32_t hi, std::int32_t* y, std::size_t i) {
    const std::int32_t v = x[i];
    y[i] = v < lo ? lo : v > hi ? hi : v;
}

// Element w of the wide tensor (deep_channels / r^2 channels at r x the deep
// size): wide[c][y r + i][x r + j] <-> deep[c r^2 + i r + j][y][x]; `up` reads
// deep and writes wide (pixel_shuffle), otherwise the reverse.
FX_HD void shuffle(const std::int32_t* x, int height, int width, int r, bool up, std::int32_t* y, std::size_t w) {
    const std::size_t wide_w = static_cast<std::size_t>(width) * r;
    const std::size_t wide_plane = static_cast<std::size_t>(height) * r * wide_w;
    const std::size_t c = w / wide_plane;
    const std::size_t wy = (w % wide_plane) / wide_w;
    const std::size_t wx = w % wide_w;
    const std::size_t deep_c = c * r * r + (wy % r) * r + (wx % r);
    const std::size_t d = (deep_c * height + wy / r) * width + wx / r;
    if (up) {
        y[w] = x[d];
    } else {
        y[d] = x[w];
    }
}

// Channels (c, ti, tj) of the k x k taps, zero outside; 3x3 pads 1, 2x2 pads 0.
FX_HD void im2col(const std::int32_t* x, int height, int width, int k, int stride, int out_h, int out_w,
                  std::int32_t* y, std::size_t i) {
    const int pad = k == 3 ? 1 : 0;
    const std::size_t out_plane = static_cast<std::size_t>(out_h) * out_w;
    const std::size_t oc = i / out_plane;
    const int oy = static_cast<int>((i % out_plane) / out_w);
    const int ox = static_cast<int>(i % out_w);
    const int c = static_cast<int>(oc / (k * k));
    const int ti = static_cast<int>((oc / k) % k);
    const int tj = static_cast<int>(oc % k);
    const int iy = oy * stride - pad + ti;
    const int ix = ox * stride - pad + tj;
    const bool inside = iy >= 0 && iy < height && ix >= 0 && ix < width;
    y[i] = inside ? x[(static_cast<std::size_t>(c) * height + iy) * width + ix] : 0;
}

FX_HD void crop(const std::int32_t* x, int height, int width, int out_h, int out_w, std::int32_t* y, std::size_t i) {
    const std::size_t out_plane = static_cast<std::size_t>(out_h) * out_w;
    const std::size_t c = i / out_plane;
    const std::size_t row = (i % out_plane) / out_w;
    const std::size_t col = i % out_w;
    y[i] = x[(c * height + row) * width + col];
}

// Channel c of the param_row output: rows[q * channels + c] for the one value
// q of x; q outside [0, row_count) is a failure (noted once, for c = 0).
#if defined(__CUDACC__)
#pragma nv_exec_check_disable
#endif
template <class Record>
FX_HD void param_row(const std::int32_t* x, const std::int64_t* rows, int row_count, int channels, std::int32_t* y,
                     int c, unsigned long long node_key, const Record& record) {
    const std::int32_t q = x[0];
    if (q < 0 || q >= row_count) {
        if (c == 0) record(node_key);
        return;
    }
    y[c] = static_cast<std::int32_t>(rows[static_cast<std::size_t>(q) * channels + c]);
}

}  // namespace nvcr_sm100::fx::elements
