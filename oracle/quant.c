/*
 * Symmetric grouped INT4/INT8 quantization: the CPU definition of the weight
 * format consumed by the CUDA quantized matmul.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * The reference's quantizer lives in the sl-precision crate (SeekStarAI/
 * sl-precision 0.1.0, .gitmodules:12, Cargo.lock "sl-precision"), which is an
 * empty submodule in the checkout; no call site or test in the checkout pins
 * its arithmetic, so parity of this format is UNPINNED. What is known from
 * the reference's own text: symmetric, grouped along K, INT4 or INT8, "U8
 * payload + F32 scale" with a 64-byte-aligned payload (README.md:164,
 * docs/ARCH-0008:85). The rest is this project's definition:
 *   - groups of `group` consecutive k per output row n; the final group of a
 *     row may be shorter (ragged) when group does not divide k;
 *   - scale[n, g] = max|w| over the group / qmax, one f32 division, with
 *     qmax = 7 (INT4) or 127 (INT8);
 *   - code = w / scale (f32 division) rounded half away from zero, clamped to
 *     [-qmax, qmax]; a zero scale gives code 0;
 *   - dequantized weight = (float)code * scale, one f32 multiply;
 *   - INT8 payload: one signed byte per k, rows of k bytes;
 *     INT4 payload: rows of ceil(k/2) bytes, two's-complement nibbles, the
 *     even k in the low nibble and the odd k in the high nibble.
 */
#include "oracle.h"

#include <math.h>
#include <string.h>

static int qmax_of(int format) { return format == ORC_INT4 ? 7 : 127; }

size_t orc_quant_row_bytes(int format, size_t k) {
    return format == ORC_INT4 ? (k + 1) / 2 : k;
}

size_t orc_quant_groups(size_t k, size_t group) {
    return group == 0 ? 0 : (k + group - 1) / group;
}

int32_t orc_code_at(int format, const uint8_t *codes, size_t k, size_t row, size_t col) {
    size_t rb = orc_quant_row_bytes(format, k);
    if (format == ORC_INT8) return (int32_t)(int8_t)codes[row * rb + col];
    uint8_t byte = codes[row * rb + col / 2];
    int32_t nib = (col & 1) ? (byte >> 4) : (byte & 0xF);
    return nib >= 8 ? nib - 16 : nib;
}

int orc_quantize(int format, const float *w, size_t n, size_t k, size_t group,
                 uint8_t *codes, float *scales, orc_err *err) {
    if (format != ORC_INT4 && format != ORC_INT8) {
        if (err) { err->code = ORC_UNSUPPORTED; err->reason = "unknown quantization format"; }
        return ORC_UNSUPPORTED;
    }
    if (group == 0) {
        if (err) { err->code = ORC_INVALID_SHAPE; err->reason = "group size must be nonzero"; }
        return ORC_INVALID_SHAPE;
    }
    const float qmax = (float)qmax_of(format);
    const size_t groups = orc_quant_groups(k, group);
    const size_t rb = orc_quant_row_bytes(format, k);
    memset(codes, 0, n * rb);
    for (size_t row = 0; row < n; row++) {
        const float *wr = w + row * k;
        for (size_t g = 0; g < groups; g++) {
            size_t begin = g * group;
            size_t end = begin + group < k ? begin + group : k;
            float max_abs = 0.0f;
            for (size_t c = begin; c < end; c++) {
                float a = fabsf(wr[c]);
                if (a > max_abs) max_abs = a;
            }
            float scale = max_abs / qmax;
            scales[row * groups + g] = scale;
            for (size_t c = begin; c < end; c++) {
                int32_t code = 0;
                if (scale != 0.0f) {
                    float q = roundf(wr[c] / scale);
                    if (q > qmax) q = qmax;
                    if (q < -qmax) q = -qmax;
                    code = (int32_t)q;
                }
                if (format == ORC_INT8) {
                    codes[row * rb + c] = (uint8_t)(int8_t)code;
                } else {
                    uint8_t nib = (uint8_t)(code & 0xF);
                    codes[row * rb + c / 2] |= (c & 1) ? (uint8_t)(nib << 4) : nib;
                }
            }
        }
    }
    if (err) err->code = ORC_OK;
    return ORC_OK;
}

int orc_dequantize(int format, const uint8_t *codes, const float *scales,
                   size_t n, size_t k, size_t group, float *w, orc_err *err) {
    if (group == 0) {
        if (err) { err->code = ORC_INVALID_SHAPE; err->reason = "group size must be nonzero"; }
        return ORC_INVALID_SHAPE;
    }
    const size_t groups = orc_quant_groups(k, group);
    for (size_t row = 0; row < n; row++)
        for (size_t c = 0; c < k; c++)
            w[row * k + c] = (float)orc_code_at(format, codes, k, row, c) *
                             scales[row * groups + c / group];
    if (err) err->code = ORC_OK;
    return ORC_OK;
}
