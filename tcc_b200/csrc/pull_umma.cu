// pull_umma.cu -- tcgen05 pull SpMM (BCSR forward, BCSC transposed) on sm_100a.
//
// Same contract as the other pull kernels (window w owns output rows
// 8w..8w+7; cnic BCSR kernel, cnic/src/core/spmm_kernel.cu:1560-1843, and the
// transposed pass replacing torch.sparse.mm(A_topo.T, .) at
// train/tcgnn_conv_release.py:152) for tc_threshold == 0: every tile on the
// TF32 tensor cores, the cnic reference's arithmetic.
//
// Per tile and 128-feature slice, one tcgen05.mma.kind::tf32 with
//   A  (M = 128 features x K = 8 gathered rows) -- the 8 feature rows, fetched
//      by eight TMA tile::gather4 copies (4 rows x 128 bytes each) straight into
//      the MN-major 128B_BASE32B shared-memory layout the tensor core reads;
//   B  (K = 8 x N = 16) -- [bits * cs_hi | bits * cs_lo]: the tile bitmap times
//      the column scales, split into a TF32-exact high part and the remainder,
//      so the column scale stays fp32-accurate (the tensor core drops the low
//      13 mantissa bits of every fp32 operand);
//   D  (128 x 16, fp32) in tensor memory: a window's accumulator, columns
//      0-7 + 8-15 summed by the epilogue.
// The feature rows themselves enter as TF32 (low 13 bits dropped).
//
// One persistent CTA per SM over a contiguous piece of the tile range (the
// merge-path split of pull_tma.cu, pieces = CTAs), warp-specialised:
//   warps 0..3   producers: steps of 16 tiles (two lanes per tile), the
//                warps taking turns; each keeps its tile metadata two steps
//                ahead in registers, waits for free stages, writes B and
//                issues the gathers;
//   warp 4       MMA issuer (one lane) and tensor-memory owner;
//   warps 5..8   epilogue: one tensor-memory lane quadrant each; load a
//                finished accumulator, scale rows by rs, store or reduce.
// Work items are window segments of at most kFlushTiles tiles; each gets one
// of kSlots accumulators.  Windows cut by a piece boundary or longer than
// kFlushTiles are "reduced": zeroed first (zero_reduced_kernel), then every
// segment adds with red.global.add.v4.
//
// Waits are bounded by %globaltimer and watch a CTA-wide abort word; the
// first role to give up sets it and TCC_DEVERR_WAIT_TIMEOUT, the others leave
// their loops, the CTA waits (bounded) for its copies and MMAs in flight and
// frees its tensor memory.
#include "spmm.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

namespace tcc {

namespace {

constexpr int kProducers = 4;         // warps 0..3
constexpr int kMmaWarp = kProducers;  // warp 4
constexpr int kWarps = kProducers + 5;  // + MMA warp + 4 epilogue warps
constexpr uint32_t kStages = 48;      // A/B ring
constexpr uint32_t kSlots = 32;       // accumulators (16 tensor-memory columns each)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kStep = 16;        // producer tiles per step
constexpr uint32_t kFlushTiles = 64;  // tiles summed in one accumulator at most
constexpr uint32_t kABytes = 4096;    // 8 rows x 128 features x 4 B
constexpr uint32_t kBBytes = 512;     // 16 x 8 TF32, K-major
constexpr unsigned long long kWaitNs = 2000000000ull;

struct Smem {
    unsigned char a[kStages][kABytes];  // 1024-aligned (base aligned by hand)
    unsigned char b[kStages][kBBytes];
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t accfull[kSlots];
    uint64_t accempty[kSlots];
    uint32_t tmem_base;
    uint32_t abort;
    uint32_t issued;  // producer steps issued so far (steps issue in order)
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;

__device__ __forceinline__ uint32_t su32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool bar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait; false on timeout or when another role aborted.
__device__ __noinline__ bool bar_wait_slow(uint32_t bar, uint32_t parity, volatile uint32_t* abort) {
    const unsigned long long t0 = gtimer();
    for (;;) {
        if (bar_try(bar, parity)) return true;
        if (*abort) return false;
        if (gtimer() - t0 > kWaitNs) {
            *abort = 1u;
            return false;
        }
    }
}
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity, volatile uint32_t* abort) {
    return bar_try(bar, parity) || bar_wait_slow(bar, parity, abort);
}

__device__ __forceinline__ void bar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void bar_arrive_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void gather4(uint32_t dst, const CUtensorMap* tm, int32_t c0, uint4 r,
                                        uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(r.x), "r"(r.y), "r"(r.z),
        "r"(r.w), "r"(bar)
        : "memory");
}

__device__ __forceinline__ uint4 ldnc4(const uint32_t* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ unsigned long long ldnc8(const uint64_t* p) {
    unsigned long long v;
    asm volatile("ld.global.nc.L1::no_allocate.u64 %0, [%1];" : "=l"(v) : "l"(p));
    return v;
}

// shared-memory matrix descriptors (tcgen05 "matrix descriptor" format:
// start >> 4 in bits 0-13, leading byte offset >> 4 in 16-29, stride byte
// offset >> 4 in 32-45, fixed 0b001 in 46-48, layout type in 61-63)
__device__ __forceinline__ uint64_t desc_a(uint32_t addr) {
    // MN-major, 128B swizzle with 32-byte atoms (layout type 1): 32 features x
    // 4 rows per 512-byte atom; next 32 features at +1024 (LBO), next 4 rows
    // at +512 (SBO)
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)(1024 >> 4) << 16) |
           ((uint64_t)(512 >> 4) << 32) | (1ull << 46) | (1ull << 61);
}
__device__ __forceinline__ uint64_t desc_b(uint32_t addr) {
    // K-major, no swizzle: 8 rows x 16 bytes per core matrix; k 4..7 at +128
    // (LBO), rows 8..15 at +256 (SBO)
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) |
           ((uint64_t)(256 >> 4) << 32) | (1ull << 46);
}
// kind::tf32, D fp32, A MN-major, B K-major, N = 16, M = 128
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | (1u << 15) | ((16u >> 3) << 17) |
                            ((128u >> 4) << 24);

__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(d), "l"(a), "l"(b), "r"(kIdesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// First i in [lo, hi) with pred(i), hi if none; 32-way warp search.
template <class P>
__device__ __forceinline__ uint32_t warp_lb(uint32_t lo, uint32_t hi, P pred, int lane) {
    while (hi - lo > 32) {
        const uint32_t step = (hi - lo + 31) / 32;
        const uint32_t p = lo + lane * step;
        const bool tested = p < hi;
        const unsigned b = __ballot_sync(0xffffffffu, tested && pred(p));
        if (b == 0) {
            const unsigned tm = __ballot_sync(0xffffffffu, tested);
            lo += (31 - __clz(tm)) * step + 1;
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

// Walks the windows of [T0, T1) as work items (window segments); every lane
// of the warp holds the same state.
struct ItemWalker {
    const uint32_t* off;
    uint32_t W, T0, T1, we;
    uint32_t w, ob, offv;  // current window, offset batch base, this lane's off[ob + lane]
    uint32_t o0, o1;       // current window's tile range
    uint32_t t, te;        // next tile of the current segment / end of this warp's part
    bool reduced;

    __device__ void load(uint32_t base, int lane) {
        ob = base;
        offv = ob + lane <= W ? off[ob + lane] : 0;
    }
    __device__ uint32_t off_at(uint32_t i) const {
        return __shfl_sync(0xffffffffu, offv, (int)(i - ob));
    }
    __device__ void enter(int lane) {  // current w valid
        if (w + 1 >= ob + 32) load(w, lane);
        o0 = off_at(w);
        o1 = off_at(w + 1);
        te = min(o1, T1);
        reduced = o0 < T0 || o1 > T1 || o1 - o0 > kFlushTiles;
    }
    // Next item: [t, t + n) of window w; false at the end.
    __device__ bool next(uint32_t& item_w, uint32_t& n, bool& red, bool first, int lane) {
        if (!first) {
            if (t >= te) {
                ++w;
                if (w >= we) return false;
                enter(lane);
            }
        } else {
            if (w >= we) return false;
            enter(lane);
        }
        item_w = w;
        n = min(te - t, kFlushTiles);
        red = reduced;
        return true;
    }
};

__global__ void __launch_bounds__(kWarps * 32, 1)
    pull_umma_kernel(const __grid_constant__ CUtensorMap tm, PullTiles a, Dense d, int accumulate,
                     uint32_t* __restrict__ err) {
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = su32(smem_raw);
    Smem& S = *reinterpret_cast<Smem*>(smem_raw + (((raw + 1023u) & ~1023u) - raw));
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    volatile uint32_t* abort = &S.abort;

    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < kStages; ++i) {
            bar_init(su32(&S.full[i]), 1);
            bar_init(su32(&S.empty[i]), 1);
        }
        for (uint32_t i = 0; i < kSlots; ++i) {
            bar_init(su32(&S.accfull[i]), 1);
            bar_init(su32(&S.accempty[i]), 4);
        }
        S.abort = 0;
        S.issued = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&S.tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

    const uint32_t T = a.num_tiles, W = a.num_windows;
    const uint64_t G = gridDim.x, g = blockIdx.x;
    const uint32_t T0 = (uint32_t)(g * T / G), T1 = (uint32_t)((g + 1) * T / G);
    const int32_t fb = (int32_t)(blockIdx.y * 128);
    const uint32_t* off = a.win_offset;
    const uint32_t n_in = a.num_in;

    if (warp < kProducers) {
        // ------------------------------------------------------- producer --
        const int h = lane & 1;
        struct Meta {
            uint4 idx;
            unsigned long long bits;
            float4 cs;
        };
        auto load_idx = [&](uint32_t step, Meta& m) {
            const uint32_t t = T0 + step * kStep + (lane >> 1);
            m.idx = make_uint4(kInvalid, kInvalid, kInvalid, kInvalid);
            m.bits = 0;
            if (step * kStep < T1 - T0 && t < T1) {
                m.idx = ldnc4(a.idx + (uint64_t)t * 8 + 4 * h);
                m.bits = ldnc8(a.bits + t);
            }
        };
        auto load_cs = [&](Meta& m) {
            auto one = [&](uint32_t k) { return k < n_in ? (d.cs ? __ldg(d.cs + k) : 1.f) : 0.f; };
            m.cs = make_float4(one(m.idx.x), one(m.idx.y), one(m.idx.z), one(m.idx.w));
        };
        const uint32_t nsteps = (T1 - T0 + kStep - 1) / kStep;
        // this warp's steps: warp, warp + kProducers, ...
        uint32_t k = (uint32_t)warp;
        Meta cur, nxt, nn;
        load_idx(k, cur);
        load_idx(k + kProducers, nxt);
        load_idx(k + 2 * kProducers, nn);
        load_cs(cur);
        load_cs(nxt);
        for (; k < nsteps && !*abort; k += kProducers) {
            const uint32_t t = T0 + k * kStep + (lane >> 1);
            const bool live = t < T1;
            unsigned long long bits = cur.bits;
            if (a.bits_transposed) bits = transpose8x8(bits);
            const uint4 idx = cur.idx;
            uint32_t vm = (idx.x < n_in ? 1u : 0u) | (idx.y < n_in ? 2u : 0u) | (idx.z < n_in ? 4u : 0u) |
                          (idx.w < n_in ? 8u : 0u);
            vm <<= 4 * h;
            vm |= __shfl_xor_sync(0xffffffffu, vm, 1);
            bits &= 0x0101010101010101ull * (unsigned long long)vm;
            // padding rows copy the tile's first real row (their B column is 0)
            const uint32_t other = __shfl_xor_sync(0xffffffffu, idx.x, 1);
            uint32_t first = h == 0 ? idx.x : other;
            if (first >= n_in) first = 0;
            uint4 rows = idx;
            if (rows.x >= n_in) rows.x = first;
            if (rows.y >= n_in) rows.y = first;
            if (rows.z >= n_in) rows.z = first;
            if (rows.w >= n_in) rows.w = first;
            const float c[4] = {cur.cs.x, cur.cs.y, cur.cs.z, cur.cs.w};

            // Steps issue in order.  A stage's uses then arm its barriers in
            // order, so the parity wait below is for the previous use of the
            // stage and cannot alias an older phase.
            bool turn = true;
            if (lane == 0) {
                volatile uint32_t* issued = &S.issued;
                if (*issued != k) {
                    const unsigned long long t0 = gtimer();
                    while (*issued != k) {
                        if (*abort) { turn = false; break; }
                        if (gtimer() - t0 > kWaitNs) { *abort = 1u; turn = false; break; }
                    }
                }
            }
            if (!__shfl_sync(0xffffffffu, turn, 0)) break;
            const uint32_t seq = k * kStep + (lane >> 1);
            const uint32_t st = seq % kStages, use = seq / kStages;
            bool ok = true;
            if (live) ok = bar_wait(su32(&S.empty[st]), (use & 1u) ^ 1u, abort);
            if (!__all_sync(0xffffffffu, ok)) break;
            if (live) {
                // B, K-major: row n (hi) / n + 8 (lo), k = 4h..4h+3 in core matrix h
                float* B = reinterpret_cast<float*>(S.b[st]);
#pragma unroll
                for (int n = 0; n < 8; ++n) {
                    float hi[4], lo[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float v = ((bits >> (n * 8 + 4 * h + e)) & 1ull) ? c[e] : 0.f;
                        hi[e] = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
                        lo[e] = v - hi[e];
                    }
                    *reinterpret_cast<float4*>(B + (h * 128 + n * 16) / 4) = make_float4(hi[0], hi[1], hi[2], hi[3]);
                    *reinterpret_cast<float4*>(B + (256 + h * 128 + n * 16) / 4) = make_float4(lo[0], lo[1], lo[2], lo[3]);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            }
            __syncwarp();
            if (live) {
                const uint32_t full = su32(&S.full[st]);
                if (h == 0) bar_arrive_tx(full, kABytes);
                const uint32_t dst = su32(S.a[st]) + h * 512;
#pragma unroll
                for (int j = 0; j < 4; ++j) gather4(dst + j * 1024, &tm, fb + 32 * j, rows, full);
            }
            __syncwarp();
            if (lane == 0) *reinterpret_cast<volatile uint32_t*>(&S.issued) = k + 1;
            cur = nxt;
            nxt = nn;
            load_cs(nxt);
            load_idx(k + 3 * kProducers, nn);
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------------------ MMA --
        const uint32_t tmem = S.tmem_base;
        ItemWalker it{off, W, T0, T1, 0, 0, 0, 0, 0, 0, T0, 0, false};
        it.we = (g + 1 == G) ? W : warp_lb(0, W, [&](uint32_t w) { return off[w] >= T1; }, lane);
        it.w = warp_lb(0, W, [&](uint32_t w) { return off[w + 1] > T0 || off[w] >= T0; }, lane);
        it.load(it.w, lane);
        uint32_t seq = 0, item = 0;
        bool first = true, failed = false;
        uint32_t iw, n;
        bool red;
        while (!failed && it.next(iw, n, red, first, lane)) {
            first = false;
            const uint32_t slot = item % kSlots, use = item / kSlots;
            if (!bar_wait(su32(&S.accempty[slot]), (use & 1u) ^ 1u, abort)) { failed = true; break; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            for (uint32_t i = 0; i < n; ++i, ++seq) {
                const uint32_t s = seq % kStages, su = seq / kStages;
                if (!bar_wait(su32(&S.full[s]), su & 1u, abort)) { failed = true; break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                if (lane == 0) {
                    mma(tmem + slot * 16, desc_a(su32(S.a[s])), desc_b(su32(S.b[s])), i > 0 ? 1u : 0u);
                    mma_commit(su32(&S.empty[s]));
                }
                __syncwarp();
            }
            if (failed) break;
            if (lane == 0) mma_commit(su32(&S.accfull[slot]));
            __syncwarp();
            it.t += n;
            ++item;
        }
    } else {
        // ------------------------------------------------------- epilogue --
        const int q = warp & 3;  // tensor-memory lane quadrant of this warp
        const uint32_t tmem = S.tmem_base + ((uint32_t)(32 * q) << 16);
        const uint32_t f = (uint32_t)fb + 32 * q + lane;
        ItemWalker it{off, W, T0, T1, 0, 0, 0, 0, 0, 0, T0, 0, false};
        it.we = (g + 1 == G) ? W : warp_lb(0, W, [&](uint32_t w) { return off[w] >= T1; }, lane);
        it.w = warp_lb(0, W, [&](uint32_t w) { return off[w + 1] > T0 || off[w] >= T0; }, lane);
        it.load(it.w, lane);
        uint32_t item = 0;
        bool first = true;
        uint32_t iw, n;
        bool red;
        // rs of the current window's rows, prefetched one window ahead
        uint32_t rs_w = kInvalid;
        float rsv[8], rsn[8];
        auto load_rs = [&](uint32_t w, float (&v)[8]) {
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                const uint32_t row = w * 8 + r;
                v[r] = (d.rs && w < W && row < a.num_out) ? __ldg(d.rs + row) : 1.f;
            }
        };
        while (it.next(iw, n, red, first, lane)) {
            first = false;
            if (iw != rs_w) {
                if (rs_w != kInvalid && iw == rs_w + 1) {
#pragma unroll
                    for (int r = 0; r < 8; ++r) rsv[r] = rsn[r];
                } else {
                    load_rs(iw, rsv);
                }
                rs_w = iw;
                load_rs(iw + 1, rsn);
            }
            const uint32_t slot = item % kSlots, use = item / kSlots;
            const bool ok = __all_sync(0xffffffffu, bar_wait(su32(&S.accfull[slot]), use & 1u, abort));
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            float y[8];
            if (n > 0) {
                uint32_t v[16];
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                      "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
                      "=r"(v[14]), "=r"(v[15])
                    : "r"(tmem + slot * 16));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int r = 0; r < 8; ++r) y[r] = __uint_as_float(v[r]) + __uint_as_float(v[r + 8]);
            } else {
#pragma unroll
                for (int r = 0; r < 8; ++r) y[r] = 0.f;
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) bar_arrive(su32(&S.accempty[slot]));
            if (f < d.F) {
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    const uint32_t row = iw * 8 + r;
                    if (row >= a.num_out) break;
                    float* yp = d.Y + (uint64_t)row * d.ldy + f;
                    const float v = y[r] * rsv[r];
                    if (red) atomicAdd(yp, v);
                    else if (accumulate) *yp += v;
                    else __stcs(yp, v);
                }
            }
            it.t += n;
            ++item;
        }
    }

    // ---------------------------------------------------------- teardown --
    __syncthreads();
    if (*abort) {
        if (threadIdx.x == 0) atomicExch(err, (uint32_t)TCC_DEVERR_WAIT_TIMEOUT);
        // bounded waits for gathers and MMAs still in flight
        if (threadIdx.x < kStages) {
            const unsigned long long t0 = gtimer();
            const uint32_t s = threadIdx.x;
            // a stage whose last phase has not completed still has copies or MMAs pending
            for (uint32_t par = 0; par < 2; ++par)
                while (!bar_try(su32(&S.full[s]), par) && gtimer() - t0 < kWaitNs) {
                }
        }
        __syncthreads();
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == kMmaWarp)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(S.tmem_base), "r"(kTmemCols)
                     : "memory");
}

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    if (!fn) throw Error(TCC_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    return fn;
}

// Same predicate as the main kernel's: see pull_tma.cu
__device__ __forceinline__ bool reduced_window(uint32_t o0, uint32_t o1, uint32_t T, uint32_t G) {
    if (o1 - o0 > kFlushTiles) return true;
    if (T == 0 || o1 - o0 < 2) return false;
    const uint64_t g = ((uint64_t)(o0 + 1) * G + T - 1) / T;
    return g < G && (uint64_t)g * T / G < o1;
}

__global__ void zero_reduced_umma(const uint32_t* __restrict__ off, uint32_t W, uint32_t T, uint32_t G,
                                  float* __restrict__ Y, uint64_t ldy, uint32_t F, uint32_t num_out) {
    const int lane = threadIdx.x & 31;
    const uint32_t q4 = F / 4;
    for (uint64_t w = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < W;
         w += ((uint64_t)gridDim.x * blockDim.x) >> 5) {
        if (!reduced_window(off[w], off[w + 1], T, G)) continue;
        for (uint32_t e = lane; e < 8 * q4; e += 32) {
            const uint64_t row = w * 8 + e / q4;
            if (row < num_out)
                *reinterpret_cast<float4*>(Y + row * ldy + 4 * (e % q4)) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
}

}  // namespace

bool pull_umma_eligible(const PullTiles& a, const Dense& d, uint32_t tc_threshold) {
    // opt-in (TCC_PULL_KERNEL=umma): one M=128 tcgen05.mma per 8x8 tile is
    // held to the tensor core's per-instruction floor (~105 cycles measured)
    const char* e = std::getenv("TCC_PULL_KERNEL");
    if (!e || std::strcmp(e, "umma") != 0) return false;
    if (a.sw_rows || tc_threshold != 0) return false;
    if (d.F == 0 || d.F % 128 != 0) return false;
    if (a.num_in == 0 || a.num_in > 0x7FFFFFFFu) return false;
    return (uintptr_t)d.X % 16 == 0 && d.ldx % 4 == 0;
}

void pull_umma(const PullTiles& a, const Dense& d, int accumulate, uint32_t* err, cudaStream_t s) {
    CUtensorMap tm;
    std::memset(&tm, 0, sizeof(tm));
    cuuint64_t dims[2] = {d.F, a.num_in};
    cuuint64_t strides[1] = {d.ldx * sizeof(float)};
    cuuint32_t box[2] = {32, 1};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = encoder()(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(d.X), dims, strides,
                                 box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw Error(TCC_ERR_CUDA, "cuTensorMapEncodeTiled failed for the X rows");
    const uint32_t ctas = (uint32_t)grid_sms();
    if (!accumulate && a.num_tiles > 0)
        zero_reduced_umma<<<std::min<unsigned>(ceil_div(a.num_windows, 8), ctas * 8), 256, 0, s>>>(
            a.win_offset, a.num_windows, a.num_tiles, ctas, d.Y, d.ldy, d.F, a.num_out);
    TCC_CUDA(cudaFuncSetAttribute(pull_umma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    pull_umma_kernel<<<dim3(ctas, d.F / 128), kWarps * 32, kSmemBytes, s>>>(tm, a, d, accumulate, err);
    TCC_CUDA(cudaGetLastError());
}

}  // namespace tcc
