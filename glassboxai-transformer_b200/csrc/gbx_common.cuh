// gbx_common.cuh -- shared device helpers and launcher plumbing for the
// sm_100a hot-path kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "gbx.h"

namespace gbx {

// ---------------------------------------------------------------------------
// Status reporting (status.cu).  set_error records a one-line reason for the
// calling host thread and returns `code`, so launchers can `return set_error(...)`.
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);   // cudaGetLastError -> GBX_ECUDA + message
void clear_error();

// Per-device properties cached once per process (thread-safe).
struct DeviceInfo {
    int sm_count;
    int max_smem_optin;   // bytes of dynamic+static smem one CTA may opt into
};
int device_info(DeviceInfo* out);   // for the current device; returns GBX_OK / GBX_ECUDA

// Grid size for a grid-stride kernel: `waves` full waves of resident CTAs,
// never more CTAs than there are work blocks.
template <class K>
inline int persistent_grid(K kernel, int block, size_t smem, int64_t work_blocks, int waves = 1)
{
    DeviceInfo di;
    if (device_info(&di) != GBX_OK) return -1;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, block, smem) != cudaSuccess || occ < 1)
        occ = 1;
    int64_t g = (int64_t)di.sm_count * occ * waves;
    if (g > work_blocks) g = work_blocks;
    if (g < 1) g = 1;
    if (g > 0x7fffffff) g = 0x7fffffff;
    return (int)g;
}

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  With gbx_set_pdl(1) the row kernels are
// launched with programmatic stream serialization: the next grid may be
// scheduled while this one drains (its launch and CTA set-up overlap our
// tail), and each such kernel starts with grid_dependency_wait(), which
// returns once every earlier grid on the stream has completed and its
// memory is visible.  No global memory is touched before that wait, so a
// kernel never reads an input early or overwrites one an earlier kernel is
// still reading.  allow_dependents() lets the next grid be scheduled once
// every CTA of this one has started.  Both are no-ops for a kernel launched
// without the attribute.
bool pdl_enabled();

// Device waits (a CTA waiting on its own copies or its own pipeline) give up
// after kDeviceWaitNs of %globaltimer time and report a timeout status.  The
// first consumer wait of the staged embedding and of the tensor-core
// contractions takes its limit from first_wait_limit_ns() instead
// (gbx_set_first_wait_limit; kDeviceWaitNs unless a test shortens it; 0 =
// give up without waiting).  Every drain of copies or MMAs in flight keeps
// kDeviceWaitNs.
constexpr uint64_t kDeviceWaitNs = 1000000000ull;
uint64_t first_wait_limit_ns();

__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <class... KArgs, class... Args>
inline cudaError_t launch_row_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                     Args&&... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    if (pdl_enabled()) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// Memory access.  Activations are streamed exactly once per kernel, so loads
// do not allocate in L1 and stores are marked evict-first.  The coherent
// (not .nc) load is used because in-place calls write the buffer they read.
// In-place calls are safe: every value a thread stores depends on the values
// it loaded from the same addresses, so no store can be ordered before the
// load it overwrites, and no element is read after it is written.
__device__ __forceinline__ float4 ld_stream(const float* p)
{
    float4 v;
    asm("ld.global.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
        : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
        : "l"(p));
    return v;
}

__device__ __forceinline__ void st_stream(float* p, float4 v)
{
    asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};"
                 :: "l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w));
}

// Read-only parameters (gamma, beta, bias rows, small tables): cached path.
__device__ __forceinline__ float4 ld_param4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// ---------------------------------------------------------------------------
// Elementwise fp32 on float4s, two lanes per instruction (sm_100's packed
// FADD2 / FMUL2 / FFMA2 through __fadd2_rn / __fmul2_rn / __ffma2_rn).  Each
// component is rounded exactly as the scalar __fadd_rn / __fmul_rn /
// __fmaf_rn rounds it, so these are bit-identical to the scalar expressions
// they stand for, in half the arithmetic instructions.
__device__ __forceinline__ float2 lo2(float4 v) { return make_float2(v.x, v.y); }
__device__ __forceinline__ float2 hi2(float4 v) { return make_float2(v.z, v.w); }
__device__ __forceinline__ float4 cat2(float2 a, float2 b) { return make_float4(a.x, a.y, b.x, b.y); }
__device__ __forceinline__ float2 splat2(float s) { return make_float2(s, s); }

// a + b
__device__ __forceinline__ float4 add4(float4 a, float4 b)
{
    return cat2(__fadd2_rn(lo2(a), lo2(b)), __fadd2_rn(hi2(a), hi2(b)));
}

// a - s (IEEE a - s is a + (-s) exactly)
__device__ __forceinline__ float4 sub4s(float4 a, float s)
{
    return cat2(__fadd2_rn(lo2(a), splat2(-s)), __fadd2_rn(hi2(a), splat2(-s)));
}

// a * s
__device__ __forceinline__ float4 mul4s(float4 a, float s)
{
    return cat2(__fmul2_rn(lo2(a), splat2(s)), __fmul2_rn(hi2(a), splat2(s)));
}

// fmaf(a, b, c) per component
__device__ __forceinline__ float4 fma4(float4 a, float4 b, float4 c)
{
    return cat2(__ffma2_rn(lo2(a), lo2(b), lo2(c)), __ffma2_rn(hi2(a), hi2(b), hi2(c)));
}

// fmaf(a, s, c) per component
__device__ __forceinline__ float4 fma4s(float4 a, float s, float4 c)
{
    return cat2(__ffma2_rn(lo2(a), splat2(s), lo2(c)), __ffma2_rn(hi2(a), splat2(s), hi2(c)));
}

// The LayerNorm affine map fmaf((x - mean) * inv, g, b) per component.
__device__ __forceinline__ float4 ln_affine4(float4 x, float mean, float inv, float4 g, float4 b)
{
    return fma4(mul4s(sub4s(x, mean), inv), g, b);
}

// ---------------------------------------------------------------------------
// Division by a run-time constant without a hardware divide (Granlund-
// Montgomery round-up method): for 0 <= n < 2^32 and 1 <= d < 2^31,
// q = (umulhi(n, m) + n) >> s with s = ceil(log2 d), m = floor(2^32 (2^s - d) / d) + 1.
struct FastDiv {
    uint32_t d, m, s;
};

inline FastDiv make_fastdiv(uint32_t d)
{
    FastDiv f;
    f.d = d;
    uint32_t s = 0;
    while ((1ull << s) < d) ++s;
    f.s = s;
    f.m = (uint32_t)((((1ull << s) - d) << 32) / d + 1);
    return f;
}

__device__ __forceinline__ uint32_t fast_div(uint32_t n, FastDiv f)
{
    uint64_t t = (uint64_t)__umulhi(n, f.m) + n;
    return (uint32_t)(t >> f.s);
}

// ---------------------------------------------------------------------------
// Reductions across `TPR` consecutive lanes (TPR a power of two <= 32).
template <int TPR>
__device__ __forceinline__ float group_sum(float v)
{
#pragma unroll
    for (int o = TPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <int TPR>
__device__ __forceinline__ float group_max(float v)
{
#pragma unroll
    for (int o = TPR / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace gbx
