// pull_tma.cu -- bulk-copy gather pull SpMM (BCSR forward, BCSC transposed) on sm_100a.
//
// Same arithmetic contract as the owner-computes pull pass (window w owns
// output rows 8w..8w+7; cnic BCSR kernel, cnic/src/core/spmm_kernel.cu:
// 1560-1843, and the transposed pass that replaces torch.sparse.mm(A_topo.T, .)
// at train/tcgnn_conv_release.py:152), with a different data path:
//
// * Work split: the tile range [0, T) is cut into G = kPieces x (CTAs x warps)
//   equal pieces; warp g takes pieces g, g + CTAs x warps, ..., so every warp
//   sees hub-heavy and many-small-window regions alike.  A warp walks the
//   windows that meet a piece in order and keeps the window's 8 x F-slice
//   partial sums in registers, so a window is written once with plain stores.  Windows cut by a piece boundary, and
//   windows longer than kFlushTiles tiles (whose warp flushes every
//   kFlushTiles tiles to keep fp32 sums short), are zeroed first and reduced
//   with red.global.add.v4.
// * Gathers: the 8 feature rows of a tile (up to 8 x 512 B) are fetched by the
//   TMA unit into a per-warp ring of kR shared-memory stages completed through
//   mbarriers.  Default: two cp.async.bulk.tensor tile::gather4 copies per tile
//   (rows 0-3 and 4-7, issued by two lanes in one instruction) through a 2D
//   tensor map over X whose box is one row high and 8 floats wider than the
//   row slice -- the extra floats (the next features, or zeros past the last
//   feature) give the 32-byte row pitch below, and a padding column's row
//   coordinate lies past the last row of X, so the TMA unit fills it with
//   zeros.  TCC_PULL_COPY=bulk instead issues one cp.async.bulk per real row
//   (8 lanes per tile) and copies a static zero row for padding.  Either way
//   the row gathers stay off the LSU/L1 fill path, where every missed 32-byte
//   sector costs a data-pipe wavefront (measured on B200: register gathers top
//   out near 32 B/clk/SM from L2, TMA copies above 48).  Rows sit 32 bytes
//   apart beyond their length, so the MMA fragment loads (4 rows x 2 float4
//   per quarter-warp) hit distinct banks.
// * Arithmetic: the register-gather kernel's (tile_mma): X rows scaled by the
//   column scale in fp32, then TF32 rounded like cvt.rna for tiles with
//   popcount >= tc_threshold (the reference's dense-tile arithmetic) and the
//   fp32-level hi/lo TF32 split for the others.
// * Metadata (gather indices, bitmaps, column scales) runs three 4-tile
//   batches ahead in registers, one lane per gathered row, so neither the
//   index stream nor the dependent scale loads stall the warp.
//
// Every mbarrier wait is bounded by %globaltimer (the limit set by
// tcc_set_wait_limit_ns, 2 s by default); on expiry the kernel records
// TCC_DEVERR_WAIT_TIMEOUT, waits for its own copies in flight (bounded by
// kDrainNs, whatever the limit) and returns.
#include "spmm.cuh"
#include "tile_mma.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

namespace tcc {

namespace {

constexpr int kTW = 16;                          // warps per CTA
constexpr int kR = 3;                            // ring stages per warp
constexpr uint32_t kMaxBox = 128;                // floats per gathered row segment
constexpr uint32_t kRowPad = 32;                 // bytes between rows beyond their length
constexpr uint32_t kStageBytes = 8 * (kMaxBox * 4 + kRowPad);
constexpr uint32_t kBatch = 4;                   // tiles per metadata batch (8 lanes each)
constexpr uint32_t kFlushTiles = 64;             // max tiles summed in one fp32 register chain
constexpr uint32_t kPieces = 12;                 // tile-range pieces per warp (default; 4-24 measured)
constexpr unsigned long long kDrainNs = 2000000000ull;  // bound of the drain after a failure

struct __align__(16) StageMeta {
    float cs[8];              // column scale of gathered row k (0 for padding) at
                              // [2 * (k % 4) + k / 4]: lane tig reads rows tig, tig + 4 at once
    unsigned long long bits;  // output-major bitmap: bit r*8 + k, padding columns cleared
    uint32_t pad[6];
};

// Source of the stage rows of padding columns: every stage row is written
// by one copy, so padding rows hold zeros, never stale data.
__device__ __align__(16) float g_zero_row[kMaxBox];
static_assert(((4 * (kMaxBox * 4 + kRowPad) + 127) & ~127u) + 4 * (kMaxBox * 4 + kRowPad) <=
                  kStageBytes && kStageBytes % 128 == 0,
              "two 128-byte aligned halves of 4 rows fit a stage");
static_assert(sizeof(StageMeta) == 64 && offsetof(StageMeta, cs) == 0,
              "stage metadata: 64 bytes, column scales 16-byte aligned");

constexpr size_t kSmemBytes =
    (size_t)kTW * kR * (kStageBytes + sizeof(StageMeta) + sizeof(uint64_t)) + 1024;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// One try_wait on phase `parity`; the warp may sleep up to kSuspendNs inside
// the instruction until the phase completes (no spinning on the issue slots).
constexpr uint32_t kSuspendNs = 200000;
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "n"(kSuspendNs)
        : "memory");
    return ok != 0;
}

// Non-blocking test of phase `parity`.
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of the mbarrier; false once limit_ns have passed.
// Limits shorter than one suspended try poll without suspending, so that the
// limit, not the suspend hint, decides when the wait gives up; limits below
// the timer's resolution (kTickNs) make the wait one test of the phase.
constexpr unsigned long long kTickNs = 1000;
__device__ __noinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned long long limit_ns) {
    if (limit_ns < kTickNs) return mbar_test(bar, parity);
    const bool poll = limit_ns < kSuspendNs;
    if (poll ? mbar_test(bar, parity) : mbar_try(bar, parity)) return true;
    const unsigned long long t0 = globaltimer();
    for (;;) {
        if (globaltimer() - t0 >= limit_ns) return false;
        if (poll ? mbar_test(bar, parity) : mbar_try(bar, parity)) return true;
    }
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

// Four rows (tensor-map row coordinates r) of the box at feature column c0 into
// consecutive box-sized pieces of shared memory at dst, completing on `bar`.
// Row coordinates outside the tensor read as zeros.
__device__ __forceinline__ void gather4(uint32_t dst, const CUtensorMap* tm, int32_t c0, uint4 r,
                                        uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(r.x), "r"(r.y), "r"(r.z),
        "r"(r.w), "r"(bar)
        : "memory");
}

// gather4 with an L2 eviction-priority policy (createpolicy) for the rows.
__device__ __forceinline__ void gather4_hint(uint32_t dst, const CUtensorMap* tm, int32_t c0,
                                             uint4 r, uint32_t bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(r.x), "r"(r.y), "r"(r.z),
        "r"(r.w), "r"(bar), "l"(pol)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// One contiguous global -> shared copy by the TMA unit, completing on `bar`
// (16-byte aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_copy(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

__device__ __forceinline__ uint32_t ld_nc_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ unsigned long long ld_nc_u64(const uint64_t* p) {
    unsigned long long v;
    asm volatile("ld.global.nc.L1::no_allocate.u64 %0, [%1];" : "=l"(v) : "l"(p));
    return v;
}

// First i in [lo, hi) with pred(i), hi if none (pred monotone false -> true);
// 32-way search over the warp, result uniform.
template <class P>
__device__ __forceinline__ uint32_t warp_lower_bound(uint32_t lo, uint32_t hi, P pred, int lane) {
    // invariant: the answer lies in [lo, hi]; hi is either the original
    // bound or an index already known to satisfy pred
    while (hi - lo > 32) {
        const uint32_t step = (hi - lo + 31) / 32;
        const uint32_t p = lo + lane * step;
        const bool tested = p < hi;
        const unsigned b = __ballot_sync(0xffffffffu, tested && pred(p));
        if (b == 0) {
            const unsigned tm = __ballot_sync(0xffffffffu, tested);
            lo += (31 - __clz(tm)) * step + 1;  // past the last tested probe
        } else {
            const int f = __ffs(b) - 1;
            hi = lo + f * step;
            if (f > 0) lo += (f - 1) * step + 1;
        }
    }
    const uint32_t p = lo + lane;
    const unsigned b = __ballot_sync(0xffffffffu, p < hi && pred(p));
    return b ? lo + __ffs(b) - 1 : hi;
}

// Metadata of one 4-tile batch as held by a lane: tile base + lane/8, gather
// row lane%8.  After finish(): bits in output-major form with padding
// columns cleared.
struct Batch {
    uint32_t idx;
    float cs;
    unsigned long long bits;
};

// Window w is "reduced" -- its rows are written with red.global.add into rows
// zeroed here -- when a warp-piece boundary T_g = floor(g*T/G) (0 < g < G)
// falls strictly inside its tiles, or when it has more than kFlushTiles tiles
// (its warp flushes every kFlushTiles tiles to keep fp32 sums short).  The
// kernel's own test is the same: o0 < T0 || o1 > T1 || o1 - o0 > kFlushTiles.
__device__ __forceinline__ bool window_reduced(uint32_t o0, uint32_t o1, uint32_t T, uint32_t G) {
    if (o1 - o0 > kFlushTiles) return true;
    if (T == 0 || o1 - o0 < 2) return false;
    // smallest g with floor(g*T/G) > o0
    const uint64_t g = ((uint64_t)(o0 + 1) * G + T - 1) / T;
    return g < G && (uint64_t)g * T / G < o1;
}

__global__ void zero_reduced_kernel(const uint32_t* __restrict__ off, uint32_t W, uint32_t T,
                                    uint32_t G, float* __restrict__ Y, uint64_t ldy, uint32_t F,
                                    uint32_t num_out) {
    const int lane = threadIdx.x & 31;
    const uint32_t q4 = F / 4;
    for (uint64_t w = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < W;
         w += ((uint64_t)gridDim.x * blockDim.x) >> 5) {
        if (!window_reduced(off[w], off[w + 1], T, G)) continue;
        for (uint32_t e = lane; e < 8 * q4; e += 32) {
            const uint64_t row = w * 8 + e / q4;
            if (row < num_out)
                *reinterpret_cast<float4*>(Y + row * ldy + 4 * (e % q4)) =
                    make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
}

// FULL: bw == 64 * NP (every float4 slot of the warp is a real feature).
// G4: rows by tile::gather4 through `tm` (else one bulk copy per row).
template <int NP, bool FULL, bool G4>
__global__ void __launch_bounds__(kTW * 32, 1)
    pull_tma_kernel(const __grid_constant__ CUtensorMap tm, PullTiles a, Dense d, uint32_t bw,
                    uint32_t thr, int accumulate, uint32_t* __restrict__ err,
                    unsigned long long wait_ns, int l2hint, uint32_t pieces) {
    extern __shared__ unsigned char smem_raw[];
    const int lane = threadIdx.x & 31;
    const int wib = threadIdx.x >> 5;
    // 1024-byte aligned base (TMA destinations need 128)
    const uint32_t raw = smem_u32(smem_raw);
    unsigned char* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    unsigned char* sdata = smem + (size_t)wib * kR * kStageBytes;
    StageMeta* smeta = reinterpret_cast<StageMeta*>(smem + (size_t)kTW * kR * kStageBytes) + wib * kR;
    uint64_t* sbar = reinterpret_cast<uint64_t*>(smem + (size_t)kTW * kR * (kStageBytes + sizeof(StageMeta))) +
                     wib * kR;

    if (lane < kR) mbar_init(smem_u32(&sbar[lane]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncwarp();

    const uint32_t rowbytes = FULL ? 256 * NP : bw * 4;
    const uint32_t pitch = rowbytes + kRowPad;
    // rows 0-3 of a stage at 0, pitch, 2 pitch, 3 pitch; rows 4-7 from the next
    // 128-byte boundary (a tensor copy's shared-memory destination is 128-byte
    // aligned); 8 x 544 bytes for a 128-float slice, which the stage size fits
    const uint32_t half = (4 * pitch + 127u) & ~127u;
    const int32_t fb = (int32_t)(blockIdx.y * kMaxBox);
    const int gid = lane >> 2, tig = lane & 3;
    // piece p = g + j * GW of the kPieces * GW equal tile pieces; a warp's
    // pieces are spread over the whole matrix, so hub-heavy and
    // many-small-window regions share out evenly across warps
    const uint64_t GW = (uint64_t)gridDim.x * kTW;
    const uint64_t G = GW * pieces;
    const uint64_t g0 = (uint64_t)blockIdx.x * kTW + wib;
    const uint32_t T = a.num_tiles, W = a.num_windows;
    const uint32_t* off = a.win_offset;
    uint32_t T0 = 0, T1 = 0;  // tile range of the current piece

    // ---- metadata pipeline: B0 current (complete), B1 (cs in flight), B2 (idx in flight)
    const int grp = lane >> 3, krow = lane & 7;
    // G4 with hints: bit 31 of a real gather index marks a hot row (real
    // indices are below 2^31; padding 0xFFFFFFFF stays past num_in either way)
    const bool hints = G4 && l2hint && a.hot != nullptr;
    auto load_idx = [&](uint32_t base, Batch& b) {
        const uint32_t t = base + grp;
        b.idx = kInvalid;
        b.bits = 0;
        if (t < T1) {
            b.idx = ld_nc_u32(a.idx + (uint64_t)t * 8 + krow);
            b.bits = ld_nc_u64(a.bits + t);
            if (hints && b.idx < a.num_in && ((__ldg(a.hot + t) >> krow) & 1u)) b.idx |= 0x80000000u;
        }
    };
    auto real = [&](uint32_t v) { return hints ? (v & 0x7FFFFFFFu) : v; };
    auto load_cs = [&](Batch& b) {
        const uint32_t r = real(b.idx);
        b.cs = r < a.num_in ? (d.cs ? __ldg(d.cs + r) : 1.f) : 0.f;
    };
    auto finish = [&](Batch& b) {
        unsigned long long bits = b.bits;
        if (a.bits_transposed) bits = transpose8x8(bits);
        const unsigned vm = __ballot_sync(0xffffffffu, real(b.idx) < a.num_in);
        const uint32_t valid = (vm >> (8 * grp)) & 0xFFu;
        b.bits = bits & (0x0101010101010101ull * (unsigned long long)valid);
    };

    Batch B0, B1, B2;
    // G4: row coordinates of rows (lane & ~3) .. +3 of B0 (a padding column:
    // past the last row of X, read as zeros)
    auto make_quad = [&]() {
        // the hot bit rides along in bit 31 (when hints are on)
        const uint32_t v = real(B0.idx) < a.num_in ? B0.idx : a.num_in;
        const int q0 = lane & ~3;
        return make_uint4(__shfl_sync(0xffffffffu, v, q0), __shfl_sync(0xffffffffu, v, q0 + 1),
                          __shfl_sync(0xffffffffu, v, q0 + 2), __shfl_sync(0xffffffffu, v, q0 + 3));
    };
    uint32_t mb = 0;
    uint32_t iq = 0;            // ring slot of the next issued tile
    uint32_t cq = 0, cpar = 0;  // ring slot and phase parity of the next consumed tile

    // tiles are issued in order, one ring slot after another, across pieces
    auto issue = [&](uint32_t t) {
        if (t >= mb + kBatch) {  // rotate (uniform: t is the same in every lane)
            B0 = B1;
            B1 = B2;
            mb += kBatch;
            load_cs(B1);
            load_idx(mb + 2 * kBatch, B2);
            finish(B0);
        }
        const uint32_t q = iq;
        if (++iq == (uint32_t)kR) iq = 0;
        uint4 quad;
        if (G4) quad = make_quad();
        if ((uint32_t)grp == t - mb) {
            const uint32_t bar = smem_u32(&sbar[q]);
            StageMeta& m = smeta[q];
            m.cs[2 * (krow & 3) + (krow >> 2)] = B0.cs;
            if (krow == 0) m.bits = B0.bits;
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            // the transaction count may run ahead of expect_tx (it goes
            // negative); the phase cannot complete before this arrival
            if (G4) {
                // rows krow .. krow + 3 of the tile, a padding column past the
                // last row of X (zero fill); lanes krow = 0, 4 issue
                if (krow == 0) mbar_arrive_tx(bar, 8 * pitch);
                if ((krow & 3) == 0) {
                    const uint32_t dst = smem_u32(sdata + q * kStageBytes) + (krow >> 2) * half;
                    if (hints) {
                        const bool hot = ((quad.x | quad.y | quad.z | quad.w) >> 31) != 0;
                        const uint4 rc = make_uint4(quad.x & 0x7FFFFFFFu, quad.y & 0x7FFFFFFFu,
                                                    quad.z & 0x7FFFFFFFu, quad.w & 0x7FFFFFFFu);
                        if (hot)
                            gather4_hint(dst, &tm, fb, rc, bar, policy_evict_last());
                        else if (l2hint == 1)
                            gather4_hint(dst, &tm, fb, rc, bar, policy_evict_first());
                        else
                            gather4(dst, &tm, fb, rc, bar);
                    } else {
                        gather4(dst, &tm, fb, quad, bar);
                    }
                }
            } else {
                if (krow == 0) mbar_arrive_tx(bar, 8 * rowbytes);
                const float* row =
                    B0.idx < a.num_in ? d.X + (uint64_t)B0.idx * d.ldx + fb : g_zero_row;
                bulk_copy(smem_u32(sdata + q * kStageBytes) + (krow >> 2) * half + (krow & 3) * pitch,
                          row, rowbytes, bar);
            }
        }
    };

    // window offsets, 32 at a time
    uint32_t ob = 0, offv = 0;
    auto off_at = [&](uint32_t i) -> uint32_t {  // uniform i, ob <= i < ob + 32
        return __shfl_sync(0xffffffffu, offv, (int)(i - ob));
    };
    // row scales of window w: lane r < 8 holds rs of row 8w + r
    auto load_rs = [&](uint32_t w) -> float {
        const uint32_t row = w * 8 + lane;
        return (d.rs && lane < 8 && row < a.num_out) ? __ldg(d.rs + row) : 1.f;
    };

    // Write (or reduce) a window's partial sums: lane holds output rows 2tig,
    // 2tig+1 at float4 slots gid + 8s.
    uint32_t row0 = 0;
    float rsv = 1.f;
    auto emit = [&](float (&acc)[4 * NP][4], bool red) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float rsc = __shfl_sync(0xffffffffu, rsv, 2 * tig + h);
            const uint32_t row = row0 + 2 * tig + h;
            if (row >= a.num_out) continue;
            float* yrow = d.Y + (uint64_t)row * d.ldy + fb;
#pragma unroll
            for (int sl = 0; sl < 2 * NP; ++sl) {
                const uint32_t f = 4 * (gid + 8 * sl);
                if (!FULL && f >= bw) continue;
                const int p = sl >> 1, e = (sl & 1) * 2 + h;
                float4 v = make_float4(acc[4 * p + 0][e], acc[4 * p + 1][e], acc[4 * p + 2][e],
                                       acc[4 * p + 3][e]);
                v = f4_scale(v, rsc);
                float* yp = yrow + f;
                // accumulate: a reduction, not load + add + store (the same fp32
                // add, without a DRAM round trip stalling the warp's copy ring)
                if (red || accumulate) {
                    red_add_v4(yp, v);
                } else {
                    __stcs(reinterpret_cast<float4*>(yp), v);
                }
            }
        }
    };

    bool failed = false;
    uint32_t t = 0, fq = 0, fpar = 0;  // on failure: tile t waited on slot fq, parity fpar
    for (uint32_t j = 0; j < pieces && !failed; ++j) {
        const uint64_t piece = g0 + j * GW;
        T0 = (uint32_t)(piece * T / G);
        T1 = (uint32_t)((piece + 1) * T / G);
        // windows meeting [T0, T1): first w with off[w+1] > T0 or off[w] >= T0,
        // up to the first window starting at or after T1 (all remaining for
        // the last piece, so trailing empty windows are written)
        const uint32_t wb = warp_lower_bound(
            0, W, [&](uint32_t w) { return off[w + 1] > T0 || off[w] >= T0; }, lane);
        const uint32_t we =
            piece + 1 == G ? W : warp_lower_bound(wb, W, [&](uint32_t w) { return off[w] >= T1; }, lane);

        mb = T0;
        if (T0 < T1) {
            load_idx(T0, B0);
            load_idx(T0 + kBatch, B1);
            load_idx(T0 + 2 * kBatch, B2);
            load_cs(B0);
            load_cs(B1);
            finish(B0);
        }
        ob = wb;
        offv = wb + lane <= W ? off[wb + lane] : 0;
        t = T0;
        for (uint32_t u = T0; u < T1 && u < T0 + kR; ++u) issue(u);
        __syncwarp();  // stage metadata written by the issuing lanes
        float rs_next = wb < we ? load_rs(wb) : 1.f;

        for (uint32_t w = wb; w < we; ++w) {
            if (w + 1 >= ob + 32) {
                ob = w;
                offv = ob + lane <= W ? off[ob + lane] : 0;
            }
            const uint32_t o0 = off_at(w), o1 = off_at(w + 1);
            const uint32_t te = min(o1, T1);
            const bool reduced = o0 < T0 || o1 > T1 || o1 - o0 > kFlushTiles;
            row0 = w * 8;
            rsv = rs_next;
            if (w + 1 < we) rs_next = load_rs(w + 1);  // one window ahead
            uint32_t chain = 0;

            float dacc[4 * NP][4];
#pragma unroll
            for (int k = 0; k < 4 * NP; ++k) dacc[k][0] = dacc[k][1] = dacc[k][2] = dacc[k][3] = 0.f;

            for (; t < te; ++t) {
                const uint32_t q = cq;
                const uint32_t par = cpar;
                if (++cq == (uint32_t)kR) {
                    cq = 0;
                    cpar ^= 1u;
                }
                bool ok = wait_ns >= kSuspendNs && mbar_try(smem_u32(&sbar[q]), par);
                if (!__all_sync(0xffffffffu, ok))
                    ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sbar[q]), par, wait_ns));
                if (!ok) {
                    failed = true;
                    fq = q;
                    fpar = par;
                    break;
                }
                const StageMeta& m = smeta[q];
                const unsigned long long bits = m.bits;
                const float2 cc = *reinterpret_cast<const float2*>(&m.cs[2 * tig]);
                const float c[2] = {cc.x, cc.y};
                const unsigned char* src = sdata + q * kStageBytes;
                // fragment-order rows k = tig + 4r, float4 slots 4*(gid + 8s) (tile_mma),
                // scaled by the column scale like the register-gather kernel
                float4 x[2][2 * NP];
#pragma unroll
                for (int r = 0; r < 2; ++r)
#pragma unroll
                    for (int sl = 0; sl < 2 * NP; ++sl) {
                        const uint32_t f = 4 * (gid + 8 * sl);
                        x[r][sl] = FULL || f < bw
                                       ? f4_scale(*reinterpret_cast<const float4*>(
                                                      src + r * half + tig * pitch + 4 * f),
                                                  c[r])
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                __syncwarp();
                if (t + kR < T1) issue(t + kR);
                tile_mma<NP>(dacc, x, bits, gid, tig, (uint32_t)__popcll(bits) < thr);
                if (++chain == kFlushTiles && t + 1 < te) {  // reduced windows only
                    emit(dacc, true);
#pragma unroll
                    for (int k = 0; k < 4 * NP; ++k) dacc[k][0] = dacc[k][1] = dacc[k][2] = dacc[k][3] = 0.f;
                    chain = 0;
                }
            }
            if (failed) break;

            emit(dacc, reduced);
        }
    }

    if (failed) {
        if (lane == 0) atomicExch(err, (uint32_t)TCC_DEVERR_WAIT_TIMEOUT);
        // copies still in flight: tiles t .. min(T1, t + kR) - 1 were issued and
        // not consumed, in ring order from slot fq
        uint32_t q = fq, par = fpar;
        for (uint32_t u = t; u < T1 && u < t + kR; ++u) {
            (void)mbar_wait(smem_u32(&sbar[q]), par, kDrainNs);
            if (++q == (uint32_t)kR) {
                q = 0;
                par ^= 1u;
            }
        }
    }
}

}  // namespace

bool pull_tma_eligible(const PullTiles& a, const Dense& d) {
    // The default pull kernel for F a multiple of 128: measured on B200 at
    // 1.04-1.24x the register-gather kernel for F = 128 and 256 on R-MAT and
    // SBM graphs, and at 0.5-0.74x for F < 128, where the fixed per-tile work
    // outweighs the smaller rows.  TCC_PULL_KERNEL=tma takes every F the
    // kernel accepts; any other value (ldg, umma) leaves it out.
    if (a.sw_rows || a.num_in == 0) return false;
    if ((uintptr_t)d.X % 16 != 0 || d.ldx % 4 != 0) return false;
    const char* e = std::getenv("TCC_PULL_KERNEL");
    if (!e || !*e) return d.F % kMaxBox == 0;
    if (std::strcmp(e, "tma") != 0) return false;
    return d.F % 4 == 0 && (d.F <= kMaxBox || d.F % kMaxBox == 0);
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                             &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    if (!fn) throw Error(TCC_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    return fn;
}

bool use_gather4() {
    const char* e = std::getenv("TCC_PULL_COPY");
    return !(e && std::strcmp(e, "bulk") == 0);
}

}  // namespace

void pull_tma(const PullTiles& a, const Dense& d, uint32_t thr, int accumulate, uint32_t* err,
              cudaStream_t s) {
    const uint32_t bw = d.F <= kMaxBox ? d.F : kMaxBox;
    const uint32_t slices = d.F <= kMaxBox ? 1 : d.F / kMaxBox;
    const uint32_t ctas = (uint32_t)grid_sms();
    // pieces per warp: TCC_PULL_PIECES (1-64) for measurements, else kPieces
    uint32_t pieces = kPieces;
    if (const char* e = std::getenv("TCC_PULL_PIECES")) {
        const long v = std::strtol(e, nullptr, 10);
        if (v >= 1 && v <= 64) pieces = (uint32_t)v;
    }
    const uint32_t G = ctas * kTW * pieces;
    const bool g4 = use_gather4();
    CUtensorMap tm;
    std::memset(&tm, 0, sizeof(tm));
    if (g4) {
        // rows of X as a 2D tensor [num_in][F]; box: one row, the slice plus
        // kRowPad bytes (the stage row pitch); x = slice start, a multiple of
        // kMaxBox floats (16-byte aligned)
        TCC_REQUIRE(a.num_in < 0x7FFFFFFFu, "gather4 row coordinates are 32-bit signed");
        cuuint64_t dims[2] = {d.F, a.num_in};
        cuuint64_t strides[1] = {d.ldx * sizeof(float)};
        cuuint32_t box[2] = {bw + kRowPad / 4, 1};
        cuuint32_t estr[2] = {1, 1};
        const CUresult r = tensor_map_encoder()(
            &tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(d.X), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) throw Error(TCC_ERR_CUDA, "cuTensorMapEncodeTiled failed for the X rows");
    }
    if (!accumulate && a.num_tiles > 0)
        zero_reduced_kernel<<<std::min<unsigned>(ceil_div(a.num_windows, 8), ctas * 8), 256, 0, s>>>(
            a.win_offset, a.num_windows, a.num_tiles, G, d.Y, d.ldy, d.F, a.num_out);
    auto pick = [&](auto full_tag, auto np_tag) {
        constexpr bool FULLv = decltype(full_tag)::value;
        constexpr int NPv = decltype(np_tag)::value;
        return g4 ? pull_tma_kernel<NPv, FULLv, true> : pull_tma_kernel<NPv, FULLv, false>;
    };
    using T = std::true_type;
    using Fa = std::false_type;
    using One = std::integral_constant<int, 1>;
    using Two = std::integral_constant<int, 2>;
    auto k = bw == 128  ? pick(T{}, Two{})
             : bw == 64 ? pick(T{}, One{})
             : bw < 64  ? pick(Fa{}, One{})
                        : pick(Fa{}, Two{});
    TCC_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    const int l2hint = l2_hint_mode();
    k<<<dim3(ctas, slices), kTW * 32, kSmemBytes, s>>>(tm, a, d, bw, thr, accumulate, err,
                                                       (unsigned long long)wait_limit_ns(), l2hint,
                                                       pieces);
    TCC_CUDA(cudaGetLastError());
}

}  // namespace tcc
