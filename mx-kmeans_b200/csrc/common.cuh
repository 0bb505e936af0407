// Shared plumbing for the sm_100a kernels: status/error reporting, launch
// accounting, and thin wrappers over the PTX this library issues by hand
// (mbarrier, TMA bulk-tensor copies, tcgen05 TMEM/MMA).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "mxk.h"

namespace mxk {

// ---------------------------------------------------------------------------
// host-side status handling

int fail(int status, const std::string& message);
int fail_cuda(const char* what, cudaError_t err);
void clear_error();

#define MXK_CUDA(call)                                         \
    do {                                                       \
        cudaError_t e_ = (call);                               \
        if (e_ != cudaSuccess) return ::mxk::fail_cuda(#call, e_); \
    } while (0)

#define MXK_CHECK(expr)                 \
    do {                                \
        int s_ = (expr);                \
        if (s_ != MXK_OK) return s_;    \
    } while (0)

#define MXK_REQUIRE(cond, msg)                                      \
    do {                                                            \
        if (!(cond)) return ::mxk::fail(MXK_ERR_INVALID, (msg));    \
    } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Launch bookkeeping: counts every kernel this library launches and, when
// profiling is on, brackets the launch with CUDA events on its stream.
// Around each kernel launch: counts it, times it on its stream with CUDA
// events while profiling is on (mxk_profile_enable), and marks it with an NVTX
// range of the kernel's name for timeline tools (a no-op without one attached).
struct LaunchScope {
    LaunchScope(const char* name, cudaStream_t stream);
    ~LaunchScope();
    const char* name;
    cudaStream_t stream;
    int device = 0;
    cudaEvent_t start = nullptr, stop = nullptr;
};

// An NVTX range for a host-side phase (one Lloyd call, one iteration).
struct PhaseRange {
    explicit PhaseRange(const char* name);
    ~PhaseRange();
    PhaseRange(const PhaseRange&) = delete;
    PhaseRange& operator=(const PhaseRange&) = delete;
};

// Device-wide error word: kernels with bounded waits set it on timeout.
int check_device_error(cudaStream_t stream);
unsigned* device_error_word();
// Per-device count of 128 x 192 tiles the MX GEMM has multiplied (all K chunks),
// for reporting the tensor work actually executed when tiles are pruned.
unsigned long long* device_tile_counter();
// Per-device count of the point rows the MX GEMM has processed.
unsigned long long* device_row_counter();

// Driver entry point for cuTensorMapEncodeTiled (resolved through the runtime,
// so the library has no link-time dependency on libcuda).
int encode_tensor_map_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                         uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapDataType dtype, CUtensorMapSwizzle swizzle);

int sm_count();

// The library's stream-ordered memory pool on the current device (created on
// first use; freed blocks stay mapped until mxk_release_workspace).  Null if it
// cannot be created.
cudaMemPool_t workspace_pool();

}  // namespace mxk

// ---------------------------------------------------------------------------
// device-side helpers

namespace mxk::dev {

// A wait that has not completed after this many cycles is treated as a hang:
// the kernel records MXK_ERR_TIMEOUT in the error word and unwinds.  Normal
// waits here last micro- to milliseconds; the limit is several seconds.
constexpr long long kWaitLimitCycles = 1ll << 33;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

// One try_wait with a suspend-time hint: a waiting warp is parked by the
// hardware until the phase completes (or ~1 ms passes) instead of spinning and
// taking issue slots from the producer and MMA warps on its SM sub-partition.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    return done != 0;
}

// Non-blocking test of an mbarrier phase (never suspends).
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (after flagging the error
// word and the CTA-wide abort flag) if the phase does not complete in time or
// another thread of the CTA has already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned* err_word, long long limit_cycles = kWaitLimitCycles) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long start = clock64();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (clock64() - start > limit_cycles) {
            *abort_flag = 1;
            if (err_word) atomicOr(err_word, 1u << MXK_ERR_TIMEOUT);
            return false;
        }
    }
}

// mbar_wait for a phase that has usually completed already: a non-suspending
// test first (cheaper for a single issuing thread), then the bounded wait.
__device__ __forceinline__ bool mbar_wait_lean(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                               unsigned* err_word) {
    if (mbar_test(bar, parity)) return true;
    return mbar_wait(bar, parity, abort_flag, err_word);
}

// 2D tiled TMA load (global -> shared), completion signalled on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x, int32_t y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// TMA gather of four rows (y0..y3) of a 2-D tensor map whose box is one row
// high; the four box rows land consecutively at dst.
__device__ __forceinline__ void tma_gather4(void* dst, const CUtensorMap* map, int32_t x, int32_t y0, int32_t y1,
                                            int32_t y2, int32_t y3, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y0), "r"(y1), "r"(y2), "r"(y3), "r"(smem_addr(bar))
        : "memory");
}

// 1-D bulk copy global -> shared (16-byte aligned, size % 16 == 0),
// completion signalled on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void prefetch_tensor_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// --- tcgen05 -----------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Completion of all previously issued tcgen05 async ops of this thread arrives
// once on `bar`.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

// Copy a 32-row x 16-byte shared-memory block into TMEM lanes 0..31 starting
// at column taddr (4 columns), replicated into all four 32-lane quadrants.
__device__ __forceinline__ void tc_copy_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// D(tmem) (+)= A(smem) x B(smem)^T with per-32-element UE8M0 scales in TMEM.
__device__ __forceinline__ void tc_mma_mx(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale.scale_vec::1X [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
            d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i receives lane (base+i)'s
// columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]),
          "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
          "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// --- packed FP32 pairs and 3-input min (sm_100) ----------------------------

// (d0, d1) = fmaf(-2, (v0, v1), pn2 + (c0, c1)) with packed FP32 add and fma
// (add.f32x2 / fma.f32x2); every lane is rounded exactly as the scalar add and
// fmaf would round it.
__device__ __forceinline__ void dist2(uint32_t v0, uint32_t v1, float2 pn2, float c0, float c1, float& d0,
                                      float& d1) {
    const float2 s = __fadd2_rn(pn2, make_float2(c0, c1));
    const float2 d = __ffma2_rn(make_float2(-2.0f, -2.0f), make_float2(__uint_as_float(v0), __uint_as_float(v1)), s);
    d0 = d.x;
    d1 = d.y;
}

// 16-byte shared-memory load through an explicit shared-window address.
__device__ __forceinline__ float4 lds_f4(uint32_t saddr) {
    float4 r;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "r"(saddr));
    return r;
}
__device__ __forceinline__ void sts_u32(uint32_t saddr, uint32_t v) {
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(saddr), "r"(v) : "memory");
}
__device__ __forceinline__ void sts_u8(uint32_t saddr, uint32_t v) {
    asm volatile("st.shared.u8 [%0], %1;" ::"r"(saddr), "r"(v) : "memory");
}
__device__ __forceinline__ float lds_f1(uint32_t saddr) {
    float r;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(r) : "r"(saddr));
    return r;
}

// (k0, k1) = fmaf(-2, (v0, v1), (c0, c1)) with one packed FP32 fma.
__device__ __forceinline__ void key2(uint32_t v0, uint32_t v1, float c0, float c1, float& k0, float& k1) {
    const float2 k = __ffma2_rn(make_float2(-2.0f, -2.0f), make_float2(__uint_as_float(v0), __uint_as_float(v1)),
                                make_float2(c0, c1));
    k0 = k.x;
    k1 = k.y;
}

// (x0, x1) *= s with one packed FP32 multiply; each lane is rounded like the scalar multiply.
__device__ __forceinline__ void mul2(float& x0, float& x1, float s) {
    const float2 x = __fmul2_rn(make_float2(x0, x1), make_float2(s, s));
    x0 = x.x;
    x1 = x.y;
}

__device__ __forceinline__ float min3f(float a, float b, float c) {
    float r;
    asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// Shared-memory matrix descriptor (tcgen05 "version 1" format):
//   [0,14) start address >> 4, [16,30) leading byte offset >> 4,
//   [32,46) stride byte offset >> 4, [46,48) = 1, [61,64) layout type.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3fff);
    d |= (uint64_t)((lbo >> 4) & 0x3fff) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3fff) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)(layout & 7) << 61;
    return d;
}
constexpr uint32_t kLayoutNone = 0;
constexpr uint32_t kLayoutSwizzle128 = 2;

// Instruction descriptor of kind::mxf8f6f4 with UE8M0 scales, K-major A/B,
// M = 128, dense:  [4,6) B scale id, [7,10) A format, [10,13) B format,
// [17,23) N >> 3, [23] scale format (1 = UE8M0), [24,29) M >> 4, [29,31) A scale id.
__host__ __device__ constexpr uint32_t mx_idesc(uint32_t a_fmt, uint32_t b_fmt, uint32_t m, uint32_t n,
                                                uint32_t sf_id) {
    return (sf_id << 4) | (a_fmt << 7) | (b_fmt << 10) | ((n >> 3) << 17) | (1u << 23) | ((m >> 4) << 24) |
           (sf_id << 29);
}
// The scale-factor selector bits of an instruction descriptor (A and B byte sf_id).
__host__ __device__ constexpr uint32_t mx_idesc_sf(uint32_t sf_id) { return (sf_id << 4) | (sf_id << 29); }
constexpr uint32_t kFmtE4M3 = 0;

}  // namespace mxk::dev
