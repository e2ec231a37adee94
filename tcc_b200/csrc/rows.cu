// rows.cu -- row gather / scatter-add for the row-partitioned SpMM's halo
// exchange (scatter-add: the transposed pass returns partial rows to owners).
//
// out[i, :F] = X[idx[i], :F]: the rows a rank sends to its peers, packed
// contiguously for one all-to-all.  One warp per row per iteration, 16-byte
// lanes (F and the row strides are multiples of 4 floats), the grid sized to
// the SMs; streaming stores, since the packed rows are read once by NCCL.
#include "common.cuh"

#include <algorithm>

namespace tcc {

namespace {

__global__ void gather_rows_kernel(const float* __restrict__ X, uint64_t ldx,
                                   const int64_t* __restrict__ idx, uint64_t n,
                                   float* __restrict__ out, uint64_t ldo, uint32_t q4,
                                   uint64_t num_rows, uint32_t* __restrict__ bad) {
    const int lane = threadIdx.x & 31;
    const uint64_t warps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    for (uint64_t i = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < n; i += warps) {
        const int64_t r = idx[i];
        float4* dst = reinterpret_cast<float4*>(out + i * ldo);
        if (r < 0 || (uint64_t)r >= num_rows) {  // record and write zeros
            if (lane == 0 && bad) atomicExch(bad, 1u);
            for (uint32_t c = lane; c < q4; c += 32) __stcs(dst + c, make_float4(0.f, 0.f, 0.f, 0.f));
            continue;
        }
        const float4* src = reinterpret_cast<const float4*>(X + (uint64_t)r * ldx);
        for (uint32_t c = lane; c < q4; c += 32) __stcs(dst + c, __ldg(src + c));
    }
}

// out[idx[i]] += in[i] (rows may repeat in idx: vector fp32 reductions).
__global__ void scatter_add_rows_kernel(const float* __restrict__ in, uint64_t ldi,
                                        const int64_t* __restrict__ idx, uint64_t n,
                                        float* __restrict__ out, uint64_t ldo, uint32_t q4,
                                        uint64_t num_rows, uint32_t* __restrict__ bad) {
    const int lane = threadIdx.x & 31;
    const uint64_t warps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    for (uint64_t i = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < n; i += warps) {
        const int64_t r = idx[i];
        if (r < 0 || (uint64_t)r >= num_rows) {  // record and skip
            if (lane == 0 && bad) atomicExch(bad, 1u);
            continue;
        }
        const float4* src = reinterpret_cast<const float4*>(in + i * ldi);
        float* dst = out + (uint64_t)r * ldo;
        for (uint32_t c = lane; c < q4; c += 32) red_add_v4(dst + 4 * c, __ldcs(src + c));
    }
}

}  // namespace

void scatter_add_rows(const float* in, uint64_t ldi, const int64_t* idx, uint64_t n, float* out,
                      uint64_t ldo, uint64_t num_rows, uint32_t F, uint32_t* bad, cudaStream_t s) {
    TCC_REQUIRE(F > 0 && F % 4 == 0, "F must be a positive multiple of 4");
    TCC_REQUIRE(ldi % 4 == 0 && ldo % 4 == 0 && ldi >= F && ldo >= F,
                "row strides must be multiples of 4 and >= F");
    TCC_REQUIRE((uintptr_t)in % 16 == 0 && (uintptr_t)out % 16 == 0, "in and out must be 16-byte aligned");
    if (n == 0) return;
    const uint64_t want = (n + 7) / 8;
    const unsigned blocks = (unsigned)std::min<uint64_t>(want, (uint64_t)sm_count() * 8);
    scatter_add_rows_kernel<<<blocks, 256, 0, s>>>(in, ldi, idx, n, out, ldo, F / 4, num_rows, bad);
    TCC_CUDA(cudaGetLastError());
}

void gather_rows(const float* X, uint64_t ldx, uint64_t num_rows, const int64_t* idx, uint64_t n,
                 float* out, uint64_t ldo, uint32_t F, uint32_t* bad, cudaStream_t s) {
    TCC_REQUIRE(F > 0 && F % 4 == 0, "F must be a positive multiple of 4");
    TCC_REQUIRE(ldx % 4 == 0 && ldo % 4 == 0 && ldx >= F && ldo >= F,
                "row strides must be multiples of 4 and >= F");
    TCC_REQUIRE((uintptr_t)X % 16 == 0 && (uintptr_t)out % 16 == 0, "X and out must be 16-byte aligned");
    if (n == 0) return;
    const uint64_t want = (n + 7) / 8;
    const unsigned blocks = (unsigned)std::min<uint64_t>(want, (uint64_t)sm_count() * 8);
    gather_rows_kernel<<<blocks, 256, 0, s>>>(X, ldx, idx, n, out, ldo, F / 4, num_rows, bad);
    TCC_CUDA(cudaGetLastError());
}

}  // namespace tcc
