// Precision policy and distance trackers of MX-KMeans, usable from host and
// device code.  Drop-in for ParCIS/MX-KMeans include/precision.hpp:1-49 (same
// function names, arguments and results).
#pragma once

#ifdef __CUDACC__
#define MXK_HD __host__ __device__
#else
#define MXK_HD
#endif

// Candidate precision of a point group (include/precision.hpp:10-17): the
// FP4 / FP6 error bound plus the centroid-norm term, divided by 64, must fit in
// the point's distance gap.  lc is the largest centroid norm (not squared).
MXK_HD inline int precision_candidate(float p4, float p6, float lc, int dimensions, float gap) {
    const float bound4 = p4 + lc + dimensions * lc;
    const float bound6 = p6 + lc + dimensions * lc;
    if (bound4 / 64.0f <= gap) return 4;
    if (bound6 / 64.0f <= gap) return 6;
    return 8;
}

// Precision used by the point GEMM (include/precision.hpp:20-26).  The
// reference evaluates the candidate and then always selects MXFP8; the same
// policy is kept here so results match it.
MXK_HD inline int select_precision(float p4, float p6, float lc, float ec, int dimensions, float gap) {
    (void)precision_candidate(p4, p6, lc, dimensions, gap);
    (void)ec;
    return 8;
}

// select_precision above is MXFP8 whatever its inputs.  While this holds, the
// Lloyd driver puts every point in the MXFP8 group without computing the
// policy's inputs (point bounds, centroid errors, gaps) or compacting by
// precision -- the same groups, labels and centroids as evaluating it.
constexpr bool kSelectPrecisionIsForcedMxfp8 = true;

// Two largest distances seen so far (include/precision.hpp:29-36).
MXK_HD inline void insert_largest_distance(float value, float& first, float& second) {
    if (value > first) {
        second = first;
        first = value;
    } else if (value > second) {
        second = value;
    }
}

// Two smallest distances and the index of the smallest; equal distances keep
// the lowest centroid index (include/precision.hpp:39-48).
MXK_HD inline void insert_distance(float value, int index, float& first, float& second, int& nearest) {
    if (value < first || (value == first && index < nearest)) {
        second = first;
        first = value;
        nearest = index;
    } else if (value < second) {
        second = value;
    }
}

#undef MXK_HD
