// gcn_ops.cu -- the elementwise epilogue of a GCN hidden layer, fused.
//
// The reference applies ReLU and then dropout to the transformed features as
// separate torch ops (train/tcgnn_conv_release.py:229-240: relu(conv1(...)),
// then F.dropout), each a full pass over the [N x hidden] activations, and
// dropout keeps a mask for its backward.  Here one pass does both:
//   out[i] = in[i] > 0 && keep(seed, i) ? in[i] * scale : 0,  scale = 1/(1-p)
// with keep(seed, i) a counter-based draw (no mask in memory), and the
// backward needs only the forward's output: out[i] > 0 exactly when in[i] > 0
// and element i was kept, so
//   grad_in[i] = out[i] > 0 ? grad_out[i] * scale : 0.
// keep(seed, i): the SplitMix64 finaliser (Steele, Lea and Flood, "Fast
// splittable pseudorandom number generators", OOPSLA 2014) applied to
// seed + (i + 1) * 0x9E3779B97F4A7C15; element i is kept when the top 32 bits
// of the result are >= p * 2^32.
#include "common.cuh"

#include <algorithm>
#include <cmath>

namespace tcc {

namespace {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ bool keep(uint64_t seed, uint64_t i, uint32_t thresh) {
    return (uint32_t)(mix64(seed + (i + 1) * 0x9E3779B97F4A7C15ull) >> 32) >= thresh;
}

__global__ void relu_dropout_fwd_kernel(const float4* __restrict__ in, float4* __restrict__ out,
                                        uint64_t n4, uint64_t seed, uint32_t thresh, float scale) {
    for (uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n4;
         q += (uint64_t)gridDim.x * blockDim.x) {
        const float4 v = in[q];
        const uint64_t i = 4 * q;
        float4 o;
        o.x = v.x > 0.f && keep(seed, i + 0, thresh) ? v.x * scale : 0.f;
        o.y = v.y > 0.f && keep(seed, i + 1, thresh) ? v.y * scale : 0.f;
        o.z = v.z > 0.f && keep(seed, i + 2, thresh) ? v.z * scale : 0.f;
        o.w = v.w > 0.f && keep(seed, i + 3, thresh) ? v.w * scale : 0.f;
        out[q] = o;
    }
}

__global__ void relu_dropout_bwd_kernel(const float4* __restrict__ grad_out,
                                        const float4* __restrict__ out,
                                        float4* __restrict__ grad_in, uint64_t n4, float scale) {
    for (uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n4;
         q += (uint64_t)gridDim.x * blockDim.x) {
        const float4 g = grad_out[q], o = out[q];
        grad_in[q] = make_float4(o.x > 0.f ? g.x * scale : 0.f, o.y > 0.f ? g.y * scale : 0.f,
                                 o.z > 0.f ? g.z * scale : 0.f, o.w > 0.f ? g.w * scale : 0.f);
    }
}

unsigned grid_for(uint64_t n4) {
    return (unsigned)std::max<uint64_t>(1, std::min<uint64_t>((n4 + 255) / 256, (uint64_t)sm_count() * 16));
}

}  // namespace

uint32_t dropout_threshold(float p) {
    // keep when the 32-bit draw is >= p * 2^32
    const double t = std::ceil((double)p * 4294967296.0);
    return t >= 4294967295.0 ? 0xFFFFFFFFu : (uint32_t)t;
}

void relu_dropout_forward(const float* in, float* out, uint64_t n, float p, uint64_t seed,
                          cudaStream_t s) {
    TCC_REQUIRE(p >= 0.f && p < 1.f, "dropout probability must be in [0, 1)");
    TCC_REQUIRE(n % 4 == 0, "element count must be a multiple of 4");
    TCC_REQUIRE((uintptr_t)in % 16 == 0 && (uintptr_t)out % 16 == 0, "buffers must be 16-byte aligned");
    if (n == 0) return;
    relu_dropout_fwd_kernel<<<grid_for(n / 4), 256, 0, s>>>(
        reinterpret_cast<const float4*>(in), reinterpret_cast<float4*>(out), n / 4, seed,
        dropout_threshold(p), 1.f / (1.f - p));
    TCC_CUDA(cudaGetLastError());
}

void relu_dropout_backward(const float* grad_out, const float* out, float* grad_in, uint64_t n,
                           float p, cudaStream_t s) {
    TCC_REQUIRE(p >= 0.f && p < 1.f, "dropout probability must be in [0, 1)");
    TCC_REQUIRE(n % 4 == 0, "element count must be a multiple of 4");
    TCC_REQUIRE((uintptr_t)grad_out % 16 == 0 && (uintptr_t)out % 16 == 0 &&
                    (uintptr_t)grad_in % 16 == 0,
                "buffers must be 16-byte aligned");
    if (n == 0) return;
    relu_dropout_bwd_kernel<<<grid_for(n / 4), 256, 0, s>>>(
        reinterpret_cast<const float4*>(grad_out), reinterpret_cast<const float4*>(out),
        reinterpret_cast<float4*>(grad_in), n / 4, 1.f / (1.f - p));
    TCC_CUDA(cudaGetLastError());
}

}  // namespace tcc
