// MX element and scale codecs used by the device kernels.
//
// Rules (the ones ParCIS/MX-KMeans gets from CUTLASS, include/kmeans.cuh:6-9,
// and cuda_fp6.h, src/kernels/quantize.cu:89):
//   * UE8M0 scale: the power of two at or above the value (round toward +inf),
//     saturating to 2^127; hardware `cvt.rp.satfinite.ue8m0x2.f32`, the same
//     instruction the reference's Scale(float) issues on Blackwell.
//   * E4M3: round-to-nearest-even with saturation, `cvt.rn.satfinite.e4m3x2.f32`.
//   * E2M3 / E2M1 / E3M2: round-to-nearest-even with saturation to the largest
//     finite magnitude, computed in software below (the reference's CUTLASS
//     sub-byte types also convert in software).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace mxk::dev {

// UE8M0 byte for a non-negative value.
__device__ __forceinline__ uint32_t ue8m0_encode(float v) {
    uint16_t out;
    asm("cvt.rp.satfinite.ue8m0x2.f32 %0, %1, %2;" : "=h"(out) : "f"(0.0f), "f"(v));
    return out & 0xffu;
}

// MXFP8 block scale: the UE8M0 code of amax / 448 rounded up to a power of two,
// i.e. ue8m0_encode(amax > 0 ? amax / 448 : 1) with the IEEE division, without
// dividing and without a call.  With amax = (1 + f 2^-23) 2^(E-127) and the
// quotient normal (biased exponent E >= 10), the correctly rounded quotient
// fl(amax / 448) is at most 2^(E-135) exactly when f <= 6291456 (the rounding
// boundary lies at 1.75 (1 + 2^-24) 2^(E-127), strictly between two
// representable mantissas), else at most 2^(E-134); so the code is
// E - 8 + (f >= 6291457).  For E <= 9 the quotient is below 2^-125, where the
// float grid is 2^-149, so its bit pattern is the integer
// round-half-even(A 2^max(E-1,0) / 448) with A the integer significand of amax
// (below 2^32); the hardware conversion then rounds that quotient.  Infinity
// divided by 448 is infinity, converted directly.  Zero and NaN give code 127
// (the scale 1.0 the reference uses when amax is not > 0).  Checked against the
// division for every float32 bit pattern.
//
// ue8m0_mxfp8_scale_common is the branch-free common case: its code is exact
// unless it sets `rare` (amax tiny or infinite), where ue8m0_mxfp8_scale must be
// used instead.
__device__ __forceinline__ uint32_t ue8m0_mxfp8_scale_common(float amax, bool& rare) {
    const uint32_t bits = __float_as_uint(amax);
    const uint32_t e = bits >> 23;
    const bool pos = amax > 0.0f;
    rare = pos && (e < 10u || e == 255u);
    return pos ? e - 8u + ((bits & 0x7fffffu) >= 6291457u ? 1u : 0u) : 127u;
}
__device__ __forceinline__ uint32_t ue8m0_mxfp8_scale(float amax) {
    bool rare;
    const uint32_t common = ue8m0_mxfp8_scale_common(amax, rare);  // zero or NaN: 127 (scale 1.0)
    if (!rare) return common;
    const uint32_t bits = __float_as_uint(amax);
    const uint32_t e = bits >> 23;
    if (e == 255u) return ue8m0_encode(amax);  // +inf
    const uint32_t sig = e ? (bits & 0x7fffffu) | 0x800000u : bits;
    const uint32_t num = sig << (e ? e - 1u : 0u);
    const uint32_t quo = num / 448u, rem = num - quo * 448u;
    const uint32_t q = quo + ((rem > 224u || (rem == 224u && (quo & 1u))) ? 1u : 0u);
    return ue8m0_encode(__uint_as_float(q));
}

// 2^(e-127) as a float (e in 0..254); e == 255 is the NaN code.
__device__ __forceinline__ float ue8m0_value(uint32_t e) {
    if (e == 0) return __uint_as_float(0x00400000u);  // 2^-127 (subnormal)
    if (e == 255) return __uint_as_float(0x7fc00000u);
    return __uint_as_float(e << 23);
}

// Exact reciprocal of a UE8M0 scale: 2^(127-e).  Multiplying by it rounds
// exactly like dividing by the scale (both are the correctly rounded x/2^(e-127)).
__device__ __forceinline__ float ue8m0_reciprocal(uint32_t e) {
    if (e == 255) return __uint_as_float(0x7fc00000u);
    if (e == 254) return __uint_as_float(0x00400000u);  // 2^-127
    return __uint_as_float((254u - e) << 23);
}

// Two E4M3 codes: low byte from `lo`, high byte from `hi`.
__device__ __forceinline__ uint32_t e4m3x2_encode(float lo, float hi) {
    uint16_t out;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(out) : "f"(hi), "f"(lo));
    return out;
}

// Value of one E4M3 code.
__device__ __forceinline__ float e4m3_decode(uint32_t code) {
    uint32_t h2;
    uint16_t c = (uint16_t)(code & 0xffu);
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(c));
    return __half2float(__ushort_as_half((unsigned short)(h2 & 0xffffu)));
}

// Values of the two E4M3 codes of e4m3x2_encode's result (low byte -> .x).
__device__ __forceinline__ float2 e4m3x2_decode(uint32_t codes) {
    uint32_t h2;
    uint16_t c = (uint16_t)(codes & 0xffffu);
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(c));
    return __half22float2(*reinterpret_cast<const __half2*>(&h2));
}

// Software round-to-nearest-even encoder for a small IEEE-like format with
// MB mantissa bits, bias BIAS, sign at bit SIGN and largest magnitude MAXV.
template <int MB, int BIAS, int SIGN>
__device__ __forceinline__ uint32_t subbyte_encode(float x, float maxv, uint32_t maxcode, bool nan_signed) {
    const uint32_t sign = __float_as_uint(x) >> 31;
    const float a = fabsf(x);
    if (isnan(x)) return (nan_signed ? sign << SIGN : 0u) | maxcode;
    if (!(a <= 2.0f * maxv)) return (sign << SIGN) | maxcode;
    constexpr int emin = 1 - BIAS;
    int e = (int)((__float_as_uint(a) >> 23) & 0xffu) - 127;
    if (e < emin) e = emin;
    const float quantum = __uint_as_float((uint32_t)(e - MB + 127) << 23);
    float r = rintf(a / quantum) * quantum;  // exact scaling; rintf ties to even
    if (r > maxv) r = maxv;
    if (r == 0.0f) return sign << SIGN;
    const uint32_t rb = __float_as_uint(r);
    const int re = (int)(rb >> 23) - 127;
    uint32_t code;
    if (re < emin) {
        const float sub_quantum = __uint_as_float((uint32_t)(emin - MB + 127) << 23);
        code = (uint32_t)(r / sub_quantum);
    } else {
        code = ((uint32_t)(re + BIAS) << MB) | ((rb >> (23 - MB)) & ((1u << MB) - 1u));
    }
    return (sign << SIGN) | code;
}

__device__ __forceinline__ uint32_t e2m3_encode(float x) { return subbyte_encode<3, 1, 5>(x, 7.5f, 0x1fu, true); }
__device__ __forceinline__ uint32_t e2m1_encode(float x) { return subbyte_encode<1, 1, 3>(x, 6.0f, 0x7u, true); }
__device__ __forceinline__ uint32_t e3m2_encode(float x) { return subbyte_encode<2, 3, 5>(x, 28.0f, 0x1fu, false); }

template <int MB, int BIAS, int SIGN>
__device__ __forceinline__ float subbyte_decode(uint32_t code) {
    const uint32_t sign = (code >> SIGN) & 1u;
    const uint32_t mag = code & ((1u << SIGN) - 1u);
    const uint32_t e = mag >> MB, m = mag & ((1u << MB) - 1u);
    float v;
    if (e == 0)
        v = (float)m * __uint_as_float((uint32_t)(1 - BIAS - MB + 127) << 23);
    else
        v = __uint_as_float(((e - BIAS + 127) << 23) | (m << (23 - MB)));
    return sign ? -v : v;
}

__device__ __forceinline__ float e2m3_decode(uint32_t c) { return subbyte_decode<3, 1, 5>(c); }
__device__ __forceinline__ float e2m1_decode(uint32_t c) { return subbyte_decode<1, 1, 3>(c); }
__device__ __forceinline__ float e3m2_decode(uint32_t c) { return subbyte_decode<2, 3, 5>(c); }

// Hardware round trips through E2M1 and E3M2 (cvt.rn.satfinite encode, cvt to
// f16x2 decode).  For finite inputs inside the format's range they equal the
// software encoders above (round to nearest even); the point-bound kernel only
// feeds them values scaled into range by their block scale.
__device__ __forceinline__ float e2m1_round_trip(float x) {
    uint32_t h2;
    asm("{\n\t.reg .b8 q;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 q, %2, %1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, q;\n\t}"
        : "=r"(h2)
        : "f"(x), "f"(0.0f));
    return __half2float(__ushort_as_half((unsigned short)(h2 & 0xffffu)));
}

__device__ __forceinline__ float e3m2_round_trip(float x) {
    uint32_t h2;
    asm("{\n\t.reg .b16 q;\n\t"
        "cvt.rn.satfinite.e3m2x2.f32 q, %2, %1;\n\t"
        "cvt.rn.f16x2.e3m2x2 %0, q;\n\t}"
        : "=r"(h2)
        : "f"(x), "f"(0.0f));
    return __half2float(__ushort_as_half((unsigned short)(h2 & 0xffffu)));
}

// Re-encode an E2M3 / E2M1 code as the E4M3 code of the same value (every
// E2M3 and E2M1 value is exactly representable in E4M3).
__device__ __forceinline__ uint32_t e2m3_to_e4m3(uint32_t c) {
    const float v = e2m3_decode(c);
    return e4m3x2_encode(v, 0.0f) & 0xffu;
}
__device__ __forceinline__ uint32_t e2m1_to_e4m3(uint32_t c) {
    const float v = e2m1_decode(c);
    return e4m3x2_encode(v, 0.0f) & 0xffu;
}

// Byte offset of the scale of (row, 32-feature block) in the tcgen05 atom layout
// for tiles of tile_rows rows: ceil(tile_rows / 128) 512-byte atoms per (tile,
// 128-feature chunk), tile-major, slice row r's four block scales at
// (r % 32) * 16 + (r / 32) * 4 + block % 4.
__device__ __forceinline__ int64_t scale_atom_offset(int64_t row, int blk, int kchunks, int tile_rows) {
    const int64_t tile = row / tile_rows;
    const int rr = (int)(row - tile * tile_rows);
    const int per_tile = (tile_rows + 127) >> 7;
    const int r = rr & 127;
    return (((tile * kchunks + (blk >> 2)) * per_tile + (rr >> 7)) << 9) + ((r & 31) << 4) + ((r >> 5) << 2) +
           (blk & 3);
}

}  // namespace mxk::dev
