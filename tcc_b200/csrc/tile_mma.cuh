// tile_mma.cuh -- one 8x8 window tile times a 64*NP-feature slice on the
// TF32 tensor cores (mma.sync m16n8k8), shared by the pull kernels.
#pragma once

#include "common.cuh"

namespace tcc {

constexpr uint32_t kOne = 0x3f800000u;  // 1.0f

__device__ __forceinline__ float comp(const float4& v, int c) {
    return c == 0 ? v.x : c == 1 ? v.y : c == 2 ? v.z : v.w;
}

// Tile MMAs of one 8x8 tile.  The warp's 64*NP features are permuted across
// MMA slots so that each lane's float4 gathers feed the A fragments directly:
// MMA j = 4p + c, slot m holds feature 4*(m + 16p) + c.  Lane (gid, tig) holds
// x[r][s] = X[gather row k = tig + 4r][4*(gid + 8s) .. +3]; B[k][n] = bit(n*8+k).
// pass2 == false: one TF32 pass with operands rounded like cvt.rna (the
// reference's dense-tile arithmetic).  pass2 == true: fp32-accurate split
// x = hi + lo (hi = x with the low 13 bits cleared, exact), all hi MMAs
// first, then all lo MMAs.  The hi MMAs take the raw fp32 bits and rely on
// the tensor core reading only the TF32 bits of an operand (the low 13 bits
// dropped, which leaves exactly hi).  That is behaviour measured on B200, not
// a documented guarantee: the fp32-accuracy tests (1e-5 relative against fp64
// CSR products, every tile on this path) check it, and masking hi explicitly
// would cost one AND per operand.
template <int NP>
__device__ __forceinline__ void tile_mma(float (&dacc)[4 * NP][4], const float4 (&x)[2][2 * NP],
                                         uint64_t bm, int gid, int tig, bool pass2) {
    uint32_t b[2];
    b[0] = ((bm >> (gid * 8 + tig)) & 1ull) ? kOne : 0u;
    b[1] = ((bm >> (gid * 8 + tig + 4)) & 1ull) ? kOne : 0u;
    if (!pass2) {
#pragma unroll
        for (int p = 0; p < NP; ++p)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint32_t a[4] = {tf32_rna_bits(comp(x[0][2 * p], c)), tf32_rna_bits(comp(x[0][2 * p + 1], c)),
                                       tf32_rna_bits(comp(x[1][2 * p], c)), tf32_rna_bits(comp(x[1][2 * p + 1], c))};
                mma_tf32_16x8x8(dacc[4 * p + c], a, b);
            }
        return;
    }
#pragma unroll
    for (int p = 0; p < NP; ++p)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint32_t hi[4] = {
                __float_as_uint(comp(x[0][2 * p], c)), __float_as_uint(comp(x[0][2 * p + 1], c)),
                __float_as_uint(comp(x[1][2 * p], c)), __float_as_uint(comp(x[1][2 * p + 1], c))};
            mma_tf32_16x8x8(dacc[4 * p + c], hi, b);
        }
    // lo = x - hi is exact in fp32
#pragma unroll
    for (int p = 0; p < NP; ++p)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float v[4] = {comp(x[0][2 * p], c), comp(x[0][2 * p + 1], c),
                                comp(x[1][2 * p], c), comp(x[1][2 * p + 1], c)};
            uint32_t lo[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
                lo[e] = __float_as_uint(v[e] - __uint_as_float(__float_as_uint(v[e]) & 0xFFFFE000u));
            mma_tf32_16x8x8(dacc[4 * p + c], lo, b);
        }
}

}  // namespace tcc
