// Pins the oracle's MX element conversions to the library the reference uses.
//
// TEST INFRASTRUCTURE ONLY (built into oracle/_ref/, never linked by the product).
// ParCIS/MX-KMeans converts FP32 to its MX element and scale types through
// CUTLASS (include/kmeans.cuh:6-9: MXFP8/MXFP6/MXFP4/Scale are
// cutlass::float_e4m3_t / float_e2m3_t / float_e2m1_t / float_ue8m0_t) and the
// point-bound estimate through CUDA's __nv_fp6_e3m2 (src/kernels/quantize.cu:89).
// This file exposes those host conversions, compiled from the installed headers
// (CUTLASS 4.5.0 vendored with flashinfer; the reference pins 4.3.5 @ 6b3e607),
// so tests can compare oracle/oracle.c against them value by value.
#include <cstdint>
#include <cstddef>
#include "cutlass/numeric_types.h"
#include <cuda_fp6.h>

extern "C" void pin_encode(int format, int64_t n, const float* in, uint8_t* out) {
    for (int64_t i = 0; i < n; ++i) {
        const float x = in[i];
        switch (format) {
            case 0: out[i] = cutlass::float_e4m3_t(x).raw(); break;
            case 1: out[i] = cutlass::float_e2m3_t(x).raw(); break;
            case 2: out[i] = cutlass::float_e2m1_t(x).raw(); break;
            case 3: out[i] = (uint8_t)__nv_fp6_e3m2(x).__x; break;
            case 4: out[i] = cutlass::float_ue8m0_t(x).raw(); break;
            default: out[i] = 0;
        }
    }
}

extern "C" void pin_decode(int format, int64_t n, const uint8_t* in, float* out) {
    for (int64_t i = 0; i < n; ++i) {
        const uint8_t b = in[i];
        switch (format) {
            case 0: out[i] = float(cutlass::float_e4m3_t::bitcast(b)); break;
            case 1: out[i] = float(cutlass::float_e2m3_t::bitcast(b)); break;
            case 2: out[i] = float(cutlass::float_e2m1_t::bitcast(b)); break;
            case 3: { __nv_fp6_e3m2 v; v.__x = (__nv_fp6_storage_t)b; out[i] = float(v); break; }
            case 4: out[i] = float(cutlass::float_ue8m0_t::bitcast(b)); break;
            default: out[i] = 0;
        }
    }
}
