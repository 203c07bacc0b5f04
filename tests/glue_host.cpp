// Host build of the DCVC-RT glue element functions (nvcr_b200/csrc/
// glue_elements.cuh), for CPU tests only. TEST INFRASTRUCTURE: built by
// tests/glue_host.py into tests/_build/libglue_host.so; the product never links
// or loads it. Each entry point visits every index the matching kernel in
// k_glue.cu visits, with the kernels' own argument checks.
#include "glue_elements.cuh"

namespace glue = nvcr_sm100::glue;

namespace {

const float thresholds[127] = {
#include "scale_thresholds.inc"
};

std::size_t volume(int batch, int channels, int height, int width) {
    return static_cast<std::size_t>(batch) * channels * height * width;
}

}  // namespace

extern "C" {

void gh_to_half(const float* in, std::uint16_t* out, std::size_t count) {
    for (std::size_t i = 0; i < count; ++i) out[i] = glue::to_half(in[i]);
}
void gh_to_float(const std::uint16_t* in, float* out, std::size_t count) {
    for (std::size_t i = 0; i < count; ++i) out[i] = glue::to_float(in[i]);
}
void gh_exact_scale_indexes(const float* in, std::uint8_t* out, std::size_t count) {
    for (std::size_t i = 0; i < count; ++i) out[i] = glue::exact_scale_index(in[i], thresholds);
}

int gh_decode_indexes(const std::uint16_t* scales, std::uint8_t* out, std::size_t count, float force_zero) {
    if (count == 0) return 0;
    for (std::size_t i = 0; i < count; ++i) glue::decode_index(scales, out, force_zero, thresholds, i);
    return 1;
}

int gh_encode_indexes(const std::uint16_t* symbols, const std::uint16_t* scales, std::int16_t* out, std::size_t count,
                      float force_zero) {
    if (count == 0) return 0;
    for (std::size_t i = 0; i < count; ++i) glue::encode_index(symbols, scales, out, force_zero, thresholds, i);
    return 1;
}

int gh_mask(std::uint16_t* mask, int batch, int channels, int height, int width, int ways, int stage) {
    if (!glue::valid_shape(batch, channels, height, width, ways) || stage < 0 || stage >= ways) return 0;
    const std::size_t count = volume(batch, channels, height, width);
    for (std::size_t i = 0; i < count; ++i) {
        if (ways == 4) {
            glue::four_way_mask(mask, channels, height, width, stage, i);
        } else {
            glue::two_way_mask(mask, channels, height, width, stage, i);
        }
    }
    return 1;
}

int gh_restore(const std::uint16_t* symbols, const std::uint16_t* means, const std::uint16_t* mask,
               std::uint16_t* out, int batch, int channels, int height, int width, int ways) {
    if (!glue::valid_shape(batch, channels, height, width, ways)) return 0;
    const std::size_t part = volume(batch, channels, height, width) / static_cast<std::size_t>(ways);
    for (std::size_t i = 0; i < part; ++i) glue::restore(symbols, means, mask, out, part, ways, i);
    return 1;
}

int gh_process(const std::uint16_t* values, const std::uint16_t* scales, const std::uint16_t* means,
               const std::uint16_t* mask, std::uint16_t* residual, std::uint16_t* symbols, std::uint16_t* reconstructed,
               std::uint16_t* masked_scales, std::size_t count, float force_zero) {
    if (count == 0) return 0;
    for (std::size_t i = 0; i < count; ++i) {
        glue::process_with_mask(values, scales, means, mask, residual, symbols, reconstructed, masked_scales,
                                force_zero, i);
    }
    return 1;
}

int gh_reduce(const std::uint16_t* input, const std::uint16_t* mask, std::uint16_t* output, int batch, int channels,
              int height, int width, int ways) {
    if (!glue::valid_shape(batch, channels, height, width, ways)) return 0;
    const std::size_t part = volume(batch, channels, height, width) / static_cast<std::size_t>(ways);
    for (std::size_t i = 0; i < part; ++i) glue::reduce_parts(input, mask, output, part, ways, i);
    return 1;
}

int gh_pointwise(int op, std::uint16_t* a, std::uint16_t* b, const std::uint16_t* c, std::int8_t* q, std::size_t count,
                 float scalar, std::size_t spatial_count) {
    if (count == 0) return 0;
    for (std::size_t i = 0; i < count; ++i) {
        switch (op) {
        case 0: glue::round_to_int8(a, q, i); break;
        case 1: glue::int8_to_half(q, a, i); break;
        case 2: glue::clamp_min(a, scalar, i); break;
        case 3: glue::clamp_reciprocal_with_quant(a, b, i); break;
        case 4: glue::add_in_place(a, b, i); break;
        case 5: glue::multiply_broadcast(a, b, spatial_count, i); break;
        case 6: glue::add_and_multiply(a, b, c, i); break;
        default: return -1;
        }
    }
    return 1;
}

int gh_pad_or_crop(const std::uint16_t* input, std::uint16_t* output, int batch, int channels, int height, int width,
                   int out_height, int out_width, int pad) {
    if (batch <= 0 || channels <= 0 || height <= 0 || width <= 0) return 0;
    if (pad ? (out_height < height || out_width < width)
            : (out_height <= 0 || out_width <= 0 || out_height > height || out_width > width)) {
        return 0;
    }
    const std::size_t count = static_cast<std::size_t>(batch) * channels * out_height * out_width;
    for (std::size_t i = 0; i < count; ++i) glue::replicate_or_crop(input, output, height, width, out_height, out_width, i);
    return 1;
}

int gh_to_ycbcr(const std::uint8_t* input, int width, int height, std::uint16_t* output, int padded_height,
                int padded_width, int yuv) {
    if (width <= 0 || height <= 0 || padded_height < height || padded_width < width ||
        (yuv && ((width & 1) != 0 || (height & 1) != 0))) {
        return 0;
    }
    const std::size_t count = static_cast<std::size_t>(padded_height) * padded_width;
    for (std::size_t i = 0; i < count; ++i) {
        if (yuv) {
            glue::yuv420p8_to_ycbcr(input, width, height, output, padded_height, padded_width, i);
        } else {
            glue::rgb24_to_ycbcr(input, width, height, output, padded_height, padded_width, i);
        }
    }
    return 1;
}

int gh_to_yuv(const std::uint16_t* input, int batch, int channels, int height, int width, int visible_width,
              int visible_height, std::uint8_t* output) {
    if (batch != 1 || channels != 3 || height <= 0 || width <= 0 || visible_width <= 0 || visible_height <= 0 ||
        (visible_width & 1) != 0 || (visible_height & 1) != 0 || visible_width > width || visible_height > height) {
        return 0;
    }
    const std::size_t y_size = static_cast<std::size_t>(visible_width) * visible_height;
    const std::size_t plane = static_cast<std::size_t>(height) * width;
    for (std::size_t i = 0; i < y_size + y_size / 4; ++i) {
        if (i < y_size) {
            glue::ycbcr_luma_to_y(input, static_cast<std::size_t>(width), visible_width, output, i);
        } else {
            glue::ycbcr_chroma_to_uv(input, plane, static_cast<std::size_t>(width), visible_width, visible_height, output,
                                     i - y_size);
        }
    }
    return 1;
}

}  // extern "C"
