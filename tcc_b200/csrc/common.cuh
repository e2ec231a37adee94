// common.cuh -- shared helpers for the tcc_b200 CUDA library (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>

#include "../../include/tcc_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "tcc_b200 is built for sm_100a only"
#endif

namespace tcc {

constexpr uint32_t kWindow = 8;          // window height / tile width (8x8 tiles)
constexpr uint32_t kCacheRows = 32;      // repeat-cache rows per super-window
constexpr uint32_t kInvalid = 0xFFFFFFFFu;
constexpr int kWarp = 32;

// Host-side error carrying a tcc_status; converted to a status at the C-ABI.
struct Error : std::runtime_error {
    tcc_status status;
    Error(tcc_status s, const std::string& m) : std::runtime_error(m), status(s) {}
};

#define TCC_CUDA(call)                                                               \
    do {                                                                             \
        cudaError_t e_ = (call);                                                     \
        if (e_ != cudaSuccess) {                                                     \
            throw ::tcc::Error(e_ == cudaErrorMemoryAllocation ? TCC_ERR_OUT_OF_MEMORY \
                                                              : TCC_ERR_CUDA,       \
                               std::string(#call) + ": " + cudaGetErrorString(e_));  \
        }                                                                            \
    } while (0)

#define TCC_REQUIRE(cond, msg)                                                       \
    do {                                                                             \
        if (!(cond)) throw ::tcc::Error(TCC_ERR_INVALID_ARGUMENT, msg);              \
    } while (0)

inline unsigned ceil_div(uint64_t a, uint64_t b) { return (unsigned)((a + b - 1) / b); }

int sm_count();
// SMs the pull kernels size their grids for: all minus the reserve set by
// tcc_set_grid_reserve (room for kernels on other streams to become resident).
int grid_sms();
void set_grid_reserve(uint32_t sms);
uint32_t grid_reserve();
// Limit of the bounded mbarrier waits in the bulk-copy pull kernel
// (tcc_set_wait_limit_ns; process-wide, 2 s by default).
void set_wait_limit_ns(uint64_t ns);
uint64_t wait_limit_ns();

// ------------------------------------------------------------ device side --

__device__ __forceinline__ unsigned lanemask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// fp32 -> tf32 with round-to-nearest, ties away (the documented cvt.rna mode).
__device__ __forceinline__ uint32_t f32_to_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}

// Round-to-nearest (ties away from zero) to TF32 on the integer pipes: add
// half a TF32 ulp to the magnitude bits and clear the 13 dropped bits.  Same
// result as the documented cvt.rna mode for finite inputs, without the
// conversion-unit round trip.
// Round to TF32 (10 explicit mantissa bits), nearest with ties away from
// zero: two integer ops, measured faster than cvt.rna.tf32.f32 in the pull
// kernels.
__device__ __forceinline__ uint32_t tf32_rna_bits(float x) {
    return (__float_as_uint(x) + 0x1000u) & 0xFFFFE000u;
}

// D[16x8] += A[16x8] * B[8x8], TF32 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_tf32_16x8x8(float d[4], const uint32_t a[4],
                                                const uint32_t b[2]) {
    asm(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// 16-byte vector fp32 reduction into global memory (sm_90+ red.v4.f32).
__device__ __forceinline__ void red_add_v4(float* addr, float4 v) {
    asm volatile("red.global.add.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(addr), "f"(v.x), "f"(v.y),
                 "f"(v.z), "f"(v.w)
                 : "memory");
}

__device__ __forceinline__ float4 f4_add(float4 a, float4 b) {
    return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}
__device__ __forceinline__ float4 f4_scale(float4 a, float s) {
    return make_float4(a.x * s, a.y * s, a.z * s, a.w * s);
}

// Streaming (evict-first) loads for metadata that is read once per launch.
__device__ __forceinline__ uint32_t ld_stream_u32(const uint32_t* p) { return __ldcs(p); }
__device__ __forceinline__ unsigned long long ld_stream_u64(const uint64_t* p) {
    return __ldcs(reinterpret_cast<const unsigned long long*>(p));
}

// 8x8 bit-matrix transpose: bit (r*8+c) -> bit (c*8+r).
__device__ __forceinline__ uint64_t transpose8x8(uint64_t x) {
    uint64_t t;
    t = (x ^ (x >> 7)) & 0x00AA00AA00AA00AAull;
    x = x ^ t ^ (t << 7);
    t = (x ^ (x >> 14)) & 0x0000CCCC0000CCCCull;
    x = x ^ t ^ (t << 14);
    t = (x ^ (x >> 28)) & 0x00000000F0F0F0F0ull;
    x = x ^ t ^ (t << 28);
    return x;
}

}  // namespace tcc
