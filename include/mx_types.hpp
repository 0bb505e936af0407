// One-byte MX element and scale types of the drop-in API.
//
// The reference's include/kmeans.cuh:6-9 aliases MXFP8 / MXFP6 / MXFP4 / Scale
// to CUTLASS float_e4m3_t / float_e2m3_t / float_e2m1_t / float_ue8m0_t.  These
// are this library's own types with the same surface those uses need: a
// one-byte storage, bitcast(), raw(), construction from float and explicit
// conversion to float, following the same conversion rules (round to nearest
// even with saturation to the largest finite value; the UE8M0 scale rounds up to
// a power of two, saturating at 2^127).  No CUTLASS include is needed.
#pragma once

#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef __CUDACC__
#define MXK_TYPES_HD __host__ __device__
#else
#define MXK_TYPES_HD
#endif

namespace mxk_types {

MXK_TYPES_HD inline uint32_t float_bits(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    return u;
}

// Round-to-nearest-even encode of x into a sign/exponent/mantissa format with
// MB mantissa bits and bias BIAS, saturating at maxv (maxcode) -- NaN maps to
// nan_code (or to the signed maximum when nan_code < 0).
MXK_TYPES_HD inline uint8_t encode_minifloat(float x, int MB, int BIAS, int sign_shift, double maxv, uint32_t maxcode,
                                             int nan_code) {
    const uint32_t sign = float_bits(x) >> 31;
    if (x != x) return nan_code >= 0 ? (uint8_t)nan_code : (uint8_t)((sign << sign_shift) | maxcode);
    const double a = fabs((double)x);
    if (a > 2.0 * maxv) return (uint8_t)((sign << sign_shift) | maxcode);
    if (a == 0.0) return (uint8_t)(sign << sign_shift);
    const int emin = 1 - BIAS;
    int e = 0;
    frexp(a, &e);
    int ex = e - 1;
    if (ex < emin) ex = emin;
    const double quantum = ldexp(1.0, ex - MB);
    double q = nearbyint(a / quantum) * quantum;
    if (q > maxv) q = maxv;
    if (q == 0.0) return (uint8_t)(sign << sign_shift);
    int qe = 0;
    frexp(q, &qe);
    const int qx = qe - 1;
    uint32_t code;
    if (qx < emin)
        code = (uint32_t)(q / ldexp(1.0, emin - MB));
    else
        code = ((uint32_t)(qx + BIAS) << MB) | (uint32_t)((q / ldexp(1.0, qx) - 1.0) * (double)(1 << MB));
    return (uint8_t)((sign << sign_shift) | code);
}

MXK_TYPES_HD inline float decode_minifloat(uint8_t b, int MB, int BIAS, int sign_shift) {
    const uint32_t sign = (b >> sign_shift) & 1u;
    const uint32_t mag = b & ((1u << sign_shift) - 1u);
    const uint32_t e = mag >> MB, m = mag & ((1u << MB) - 1u);
    double v;
    if (e == 0)
        v = ldexp((double)m, 1 - BIAS - MB);
    else
        v = ldexp(1.0 + (double)m / (double)(1 << MB), (int)e - BIAS);
    return (float)(sign ? -v : v);
}

}  // namespace mxk_types

struct MXFP8 {  // E4M3 (no infinities; 0x7f/0xff are NaN)
    uint8_t storage = 0;
    MXFP8() = default;
    MXK_TYPES_HD explicit MXFP8(float x) : storage(mxk_types::encode_minifloat(x, 3, 7, 7, 448.0, 0x7e, 0x7f)) {}
    MXK_TYPES_HD static MXFP8 bitcast(uint8_t b) {
        MXFP8 v;
        v.storage = b;
        return v;
    }
    MXK_TYPES_HD uint8_t raw() const { return storage; }
    MXK_TYPES_HD explicit operator float() const {
        if ((storage & 0x7f) == 0x7f) return NAN;
        return mxk_types::decode_minifloat(storage, 3, 7, 7);
    }
};

struct MXFP6 {  // E2M3 in the low six bits
    uint8_t storage = 0;
    MXFP6() = default;
    MXK_TYPES_HD explicit MXFP6(float x) : storage(mxk_types::encode_minifloat(x, 3, 1, 5, 7.5, 0x1f, -1)) {}
    MXK_TYPES_HD static MXFP6 bitcast(uint8_t b) {
        MXFP6 v;
        v.storage = (uint8_t)(b & 0x3f);
        return v;
    }
    MXK_TYPES_HD uint8_t raw() const { return storage; }
    MXK_TYPES_HD explicit operator float() const { return mxk_types::decode_minifloat(storage, 3, 1, 5); }
};

struct MXFP4 {  // E2M1 in the low four bits
    uint8_t storage = 0;
    MXFP4() = default;
    MXK_TYPES_HD explicit MXFP4(float x) : storage(mxk_types::encode_minifloat(x, 1, 1, 3, 6.0, 0x7, -1)) {}
    MXK_TYPES_HD static MXFP4 bitcast(uint8_t b) {
        MXFP4 v;
        v.storage = (uint8_t)(b & 0xf);
        return v;
    }
    MXK_TYPES_HD uint8_t raw() const { return storage; }
    MXK_TYPES_HD explicit operator float() const { return mxk_types::decode_minifloat(storage, 1, 1, 3); }
};

struct Scale {  // UE8M0: 2^(storage - 127); 0xff is NaN
    uint8_t storage = 0;
    Scale() = default;
    MXK_TYPES_HD explicit Scale(float x) {
        if (x != x || x - x != 0.0f) {
            storage = 0xff;
            return;
        }
        uint32_t u = mxk_types::float_bits(x);
        uint32_t e = (u >> 23) & 0xff, m = u & 0x7fffff;
        if (m != 0 && e != 0xfe && !(e == 0 && m <= 0x400000)) e += 1;
        storage = (uint8_t)e;
    }
    MXK_TYPES_HD static Scale bitcast(uint8_t b) {
        Scale v;
        v.storage = b;
        return v;
    }
    MXK_TYPES_HD uint8_t raw() const { return storage; }
    MXK_TYPES_HD explicit operator float() const {
        if (storage == 0xff) return NAN;
        return (float)ldexp(1.0, (int)storage - 127);
    }
};

static_assert(sizeof(MXFP8) == 1 && sizeof(MXFP6) == 1 && sizeof(MXFP4) == 1 && sizeof(Scale) == 1,
              "MX element types must be one byte");

#undef MXK_TYPES_HD
