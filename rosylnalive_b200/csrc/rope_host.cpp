// rope_host.cpp -- T_spec, the RoPE table, built on the host (src/Lrm.Tensor.CpuReference/Rope.fs:163-251).
//
// For pos < max_pos and j < half: freq = f32(f32(pos) * inv_freq[j]); cos = f32(RN64(cos freq)) and
// sin = f32(RN64(sin freq)), RN64 being the correctly rounded float64. The reference computes RN64 in exact integer
// arithmetic. Here the value v = libm cos/sin in double is within one double ulp of the exact value, so RN64 is one
// of v - ulp, v, v + ulp; when all three round to the same float32, that float32 is certain. Otherwise the value is
// recomputed in x87 extended precision (64-bit significand) and accepted only when the three extended neighbours
// give one RN64 and that gives one float32. If neither certifies, the call fails rather than guess. The tests pin the
// result to the reference's table digests (tiny and Qwen3-0.6B) bit for bit.
#include <math.h>
#include <string.h>

#include "../../include/lrm_cuda.h"
#include "internal.h"

namespace {

bool certain_f32_from_double(double v, float *out) {
    float a = (float)v, b = (float)nextafter(v, INFINITY), c = (float)nextafter(v, -INFINITY);
    uint32_t ua, ub, uc;
    memcpy(&ua, &a, 4);
    memcpy(&ub, &b, 4);
    memcpy(&uc, &c, 4);
    if (ua != ub || ua != uc) return false;
    *out = a;
    return true;
}

bool certain_f32_from_long_double(long double v, float *out) {
    double a = (double)v, b = (double)nextafterl(v, INFINITY), c = (double)nextafterl(v, -INFINITY);
    if (a != b || a != c) return false;
    *out = (float)a;
    return true;
}

bool cos_sin_f32(float x, float *c, float *s) {
    if (fabsf(x) < 0x1p-27f) {  // RN64(cos x) = 1 and RN64(sin x) = x exactly (Rope.fs:150-152)
        *c = 1.0f;
        *s = x;
        return true;
    }
    double xd = (double)x;
    if (certain_f32_from_double(cos(xd), c) && certain_f32_from_double(sin(xd), s)) return true;
    long double xl = (long double)x;
    return certain_f32_from_long_double(cosl(xl), c) && certain_f32_from_long_double(sinl(xl), s);
}

}  // namespace

extern "C" lrm_status lrm_rope_table(const uint32_t *inv_freq_bits, int32_t half, int32_t max_pos, float *cos_out,
                                     float *sin_out) {
    if (!inv_freq_bits || !cos_out || !sin_out || half < 1 || max_pos < 1 || max_pos > (1 << 24)) {
        lrm::set_thread_error("lrm_rope_table: null pointer, half < 1 or max_pos outside 1..2^24");
        return LRM_ERR_ARGUMENT;
    }
    for (int32_t pos = 0; pos < max_pos; ++pos) {
        for (int32_t j = 0; j < half; ++j) {
            float inv;
            memcpy(&inv, &inv_freq_bits[j], 4);
            if (!isfinite(inv)) {
                lrm::set_thread_error("lrm_rope_table: an inv_freq entry is not finite");
                return LRM_ERR_ARGUMENT;
            }
            volatile float fpos = (float)pos;  // exact below 2^24
            float freq = fpos * inv;           // one float32 multiply
            size_t at = (size_t)pos * half + j;
            if (!cos_sin_f32(freq, &cos_out[at], &sin_out[at])) {
                lrm::set_thread_error("lrm_rope_table: a float64 rounding could not be certified");
                return LRM_ERR_ARGUMENT;
            }
        }
    }
    return LRM_OK;
}
