// spmm.cu -- SpMM over 8x8 window tiles on sm_100a.
//
// Pull (owner-computes) pass: one warp per chunk of <= kChunkTiles tiles of a
// window; the window owns its 8 output rows, so rows are written once with
// plain 16-byte stores (windows split into several chunks reduce with
// red.global.add.v4.f32).  Per tile the 8 gather rows are loaded as coalesced
// 128-bit lanes; tiles whose popcount reaches tc_threshold go through TF32
// mma.sync m16n8k8 (the reference's arithmetic for dense tiles,
// src/swtcf_spmm.cu:186-214, cnic/src/core/spmm_kernel.cu:1783-1801), the
// others through fp32 FMA lanes.  Used for BCSR forward (cnic BCSR kernel,
// spmm_kernel.cu:1560-1843) and for the transposed passes over BCSC / SWTCF
// tiles, which replace torch.sparse.mm(A_topo.T, .) (train/tcgnn_conv_release.py:152).
//
// Push pass: one warp per column window; the window's 8 input rows are loaded
// once, each tile row is summed and reduced into Y with 16-byte vector
// reductions (the reference's fp32 atomicAdd, src/swtcf_spmm.cu:53-76 and
// spmm_kernel.cu:2060-2093).  The SWTCF variant keeps the super-window's 32
// repeat-cache rows in shared memory and flushes them once (src/swtcf_spmm.cu:
// 246-264).
#include "spmm.cuh"
#include "primitives.cuh"
#include "tile_mma.cuh"

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <cstddef>
#include <mutex>

namespace tcc {

int sm_count() {
    static std::mutex mu;
    static int cache[64] = {};
    int dev = 0;
    TCC_CUDA(cudaGetDevice(&dev));
    TCC_REQUIRE(dev >= 0 && dev < 64, "device ordinal out of range");
    std::lock_guard<std::mutex> lock(mu);
    if (!cache[dev]) TCC_CUDA(cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev));
    return cache[dev];
}

namespace {
std::atomic<uint32_t> g_grid_reserve{0};
std::atomic<uint64_t> g_wait_limit_ns{TCC_DEFAULT_WAIT_LIMIT_NS};
}  // namespace

void set_grid_reserve(uint32_t sms) { g_grid_reserve.store(sms); }
uint32_t grid_reserve() { return g_grid_reserve.load(); }
void set_wait_limit_ns(uint64_t ns) { g_wait_limit_ns.store(ns); }
uint64_t wait_limit_ns() { return g_wait_limit_ns.load(); }

int grid_sms() {
    const int n = sm_count();
    const int r = (int)std::min<uint32_t>(g_grid_reserve.load(), (uint32_t)std::max(0, n - 1));
    return n - r;
}

namespace {

constexpr uint32_t kChunkTiles = 16;  // max tiles per warp task
constexpr int kPushWarps = 8;         // warps per push block

struct PlanHeader {
    uint32_t num_chunks;
    uint32_t heavy_count;
    uint32_t pad[14];
};

// Hot-row selection: use counts of the gathered rows in a direct-mapped
// table of kSketch counters (row r counts at r mod kSketch: exact for up to
// kSketch rows, an overestimate beyond), then the most used rows up to
// kHotRows (one 128-float slice each: ~80 MB of L2) are "hot".
constexpr uint32_t kSketch = 1u << 18;
constexpr uint32_t kCountBins = 1u << 14;
constexpr uint32_t kHotRows = 160u << 10;

struct PlanLayout {
    size_t cstart, desc, heavy, tmp, hot, sketch, hist, total;
    uint64_t max_chunks;
    PlanLayout(uint32_t W, uint32_t T) {
        auto al = [](size_t b) { return (b + 255) / 256 * 256; };
        max_chunks = (uint64_t)W + (T + kChunkTiles - 1) / kChunkTiles + 1;
        cstart = 256;
        desc = cstart + al(((size_t)W + 1) * 4);
        heavy = desc + al(max_chunks * 16);
        tmp = heavy + al(((size_t)W + 1) * 4);
        hot = tmp + al(scan_tmp_bytes((uint64_t)W + 1));
        sketch = hot + al(std::max<size_t>(T, 1));
        hist = sketch + al((size_t)kSketch * 4);
        total = hist + al((size_t)kCountBins * 4 + 16);
    }
};

__global__ void hot_count_kernel(const uint32_t* __restrict__ idx, uint64_t n, uint32_t num_in,
                                 uint32_t* __restrict__ sketch) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t r = idx[i];
        if (r < num_in) atomicAdd(&sketch[r & (kSketch - 1)], 1u);
    }
}

__global__ void hot_hist_kernel(const uint32_t* __restrict__ sketch, uint32_t* __restrict__ hist) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < kSketch; i += gridDim.x * blockDim.x) {
        const uint32_t c = sketch[i];
        if (c > 1) atomicAdd(&hist[min(c, kCountBins - 1)], 1u);
    }
}

// One block: the smallest use count K (>= 2) whose rows with count >= K fit
// kHotRows; stored at hist[kCountBins] (kCountBins = none hot).
__global__ void hot_threshold_kernel(uint32_t* __restrict__ hist, uint32_t budget) {
    __shared__ uint32_t done;
    if (threadIdx.x == 0) {
        uint64_t rows = 0;
        uint32_t K = kCountBins;
        for (uint32_t c = kCountBins - 1; c >= 2; --c) {
            rows += hist[c];
            if (rows > budget) break;
            K = c;
        }
        hist[kCountBins] = K;
        done = 1;
    }
    __syncthreads();
    (void)done;
}

__global__ void hot_mask_kernel(const uint32_t* __restrict__ idx, uint32_t T, uint32_t num_in,
                                const uint32_t* __restrict__ sketch,
                                const uint32_t* __restrict__ hist, uint8_t* __restrict__ hot) {
    const uint32_t K = hist[kCountBins];
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += gridDim.x * blockDim.x) {
        uint32_t m = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint32_t r = idx[(uint64_t)t * 8 + k];
            if (r < num_in && sketch[r & (kSketch - 1)] >= K) m |= 1u << k;
        }
        hot[t] = (uint8_t)m;
    }
}

__global__ void plan_count_kernel(const uint32_t* __restrict__ off, uint32_t W,
                                  uint32_t* __restrict__ nch) {
    const uint32_t w = blockIdx.x * blockDim.x + threadIdx.x;
    if (w >= W) return;
    const uint32_t t = off[w + 1] - off[w];
    nch[w] = t <= kChunkTiles ? 1u : (t + kChunkTiles - 1) / kChunkTiles;
}

__global__ void plan_fill_kernel(const uint32_t* __restrict__ off, uint32_t W,
                                 const uint32_t* __restrict__ cstart, uint4* __restrict__ desc,
                                 uint32_t* __restrict__ heavy, PlanHeader* hdr) {
    const uint32_t w = blockIdx.x * blockDim.x + threadIdx.x;
    if (w == 0) hdr->num_chunks = cstart[W];
    if (w >= W) return;
    const uint32_t tb = off[w], te = off[w + 1];
    const uint32_t base = cstart[w], n = cstart[w + 1] - cstart[w];
    for (uint32_t j = 0; j < n; ++j) {
        const uint32_t b = tb + j * kChunkTiles;
        desc[base + j] = make_uint4(w, b, min(te, b + kChunkTiles), n > 1 ? 1u : 0u);
    }
    if (n > 1) heavy[atomicAdd(&hdr->heavy_count, 1u)] = w;
}

// Output rows of windows that several warps reduce into start from zero
// (16-byte stores; F and the row stride are multiples of 4).
__global__ void zero_heavy_kernel(const uint32_t* __restrict__ heavy,
                                  const PlanHeader* __restrict__ hdr, float* __restrict__ Y,
                                  uint64_t ldy, uint32_t F, uint32_t num_out) {
    const uint32_t n = hdr->heavy_count;
    const uint32_t q4 = F / 4;
    const uint32_t per_window = 8 * q4;
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < (uint64_t)n * per_window;
         e += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t h = (uint32_t)(e / per_window);
        const uint32_t r = (uint32_t)(e % per_window);
        const uint32_t row = heavy[h] * 8 + r / q4;
        if (row < num_out) *reinterpret_cast<float4*>(Y + (uint64_t)row * ldy + 4 * (r % q4)) = z;
    }
}

__device__ __forceinline__ float4 ld4(const float* p) {
    return __ldg(reinterpret_cast<const float4*>(p));
}

enum { kGatherDense = 0, kGatherSwtcf = 1, kGatherStore = 2 };

// Row pointer of condensed column c in the hot/cold feature store
// (cnic/src/core/spmm_kernel.cu:129-153 semantics).
__device__ __forceinline__ const float* store_row(const FeatureStore& fs, uint32_t c, uint32_t F) {
    const int32_t g = fs.cache_search_map[c];
    if (g >= 0) {
        const float* base = fs.gpu_features[g / fs.gpu_capacity];
        return base + (uint64_t)(g % fs.gpu_capacity) * F;
    }
    return fs.cpu_features + (uint64_t)fs.id_map[c] * F;
}

// ---------------------------------------------------------------- pull ----
// One warp per chunk; the 8 gather rows of a tile go straight to registers
// as 128-bit read-only loads in MMA fragment order (L1::no_allocate measured
// slower in gather probes), two tiles in flight
// per warp, 16 warps/SM.  Chunk metadata (bitmaps, gather indices) is
// double-buffered in shared memory with cp.async one chunk ahead.
constexpr int kPullWarps = 8;
struct WarpMeta {
    uint64_t bits[kChunkTiles];
    uint32_t idx[kChunkTiles * 8];
};
__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

template <int NP, int GATHER>
__device__ __forceinline__ void gather_tile(float4 (&x)[2][2 * NP], const PullTiles& a,
                                            const Dense& d, const WarpMeta& M,
                                            const float* const* ptrs, int t, int gid, int tig,
                                            uint32_t fb) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint32_t k = M.idx[t * 8 + tig + 4 * r];
        const bool ok = k < a.num_in;
        const float* row = nullptr;
        if constexpr (GATHER == kGatherStore) {
            row = ok ? ptrs[t * 8 + tig + 4 * r] : nullptr;
        } else {
            row = d.X + (uint64_t)(ok ? k : 0) * d.ldx;
        }
        const float sc = (ok && d.cs) ? __ldg(d.cs + k) : 1.f;
#pragma unroll
        for (int s = 0; s < 2 * NP; ++s) {
            const uint32_t f = fb + 4 * (gid + 8 * s);
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (ok && f < d.F) {
                if constexpr (GATHER == kGatherStore) v = *reinterpret_cast<const float4*>(row + f);
                else v = ld4(row + f);
            }
            x[r][s] = f4_scale(v, sc);
        }
    }
}

template <int NP, int GATHER>
__global__ void __launch_bounds__(kPullWarps * 32, 2) pull_kernel(PullTiles a, Dense d,
                                                                  const uint4* __restrict__ desc,
                                                                  PlanHeader* __restrict__ hdr,
                                                                  uint32_t thr, int accumulate,
                                                                  FeatureStore fs) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int lane = threadIdx.x & 31;
    const int wib = threadIdx.x >> 5;
    const int gid = lane >> 2, tig = lane & 3;
    WarpMeta* meta = reinterpret_cast<WarpMeta*>(smem_raw) + 2 * wib;
    const float** ptrs = nullptr;
    if constexpr (GATHER == kGatherStore)
        ptrs = reinterpret_cast<const float**>(smem_raw + sizeof(WarpMeta) * 2 * kPullWarps) +
               wib * kChunkTiles * 8;
    const uint32_t fb = blockIdx.y * (64 * NP);
    const uint32_t num_chunks = hdr->num_chunks;
    const uint32_t warps_total = gridDim.x * kPullWarps;

    auto prefetch = [&](const uint4& c, int b) {
        const uint32_t n = c.z - c.y;
        if ((uint32_t)lane < n) cp_async8(&meta[b].bits[lane], a.bits + c.y + lane);
        for (uint32_t p = lane; p < 2 * n; p += 32)
            cp_async16(&meta[b].idx[p * 4], a.idx + (uint64_t)c.y * 8 + p * 4);
    };

    uint32_t chunk = blockIdx.x * kPullWarps + wib;
    uint4 cur = make_uint4(0, 0, 0, 0), nxt = make_uint4(0, 0, 0, 0);
    if (chunk < num_chunks) {
        cur = desc[chunk];
        prefetch(cur, 0);
    }
    cp_async_commit();
    if (chunk + warps_total < num_chunks) nxt = desc[chunk + warps_total];
    int buf = 0;
    while (chunk < num_chunks) {
        const uint32_t next = chunk + warps_total;
        if (next < num_chunks) prefetch(nxt, buf ^ 1);
        cp_async_commit();
        uint4 nxt2 = make_uint4(0, 0, 0, 0);
        if (next + warps_total < num_chunks) nxt2 = desc[next + warps_total];
        cp_async_wait<1>();
        __syncwarp();
        WarpMeta& M = meta[buf];
        const uint32_t w = cur.x;
        const int n = (int)(cur.z - cur.y);
        if constexpr (GATHER == kGatherSwtcf) {
            const uint32_t swoff = a.sw_offset[w / a.S];
            for (int e = lane; e < n * 8; e += 32) {
                const uint32_t slot = M.idx[e];
                M.idx[e] = slot == kInvalid ? kInvalid : __ldg(a.sw_rows + swoff + slot);
            }
            __syncwarp();
        }
        if constexpr (GATHER == kGatherStore) {
            for (int e = lane; e < n * 8; e += 32) {
                const uint32_t c = M.idx[e];
                ptrs[e] = c < a.num_in ? store_row(fs, c, d.F) : nullptr;
            }
            __syncwarp();
        }
        float dacc[4 * NP][4];
#pragma unroll
        for (int j = 0; j < 4 * NP; ++j) dacc[j][0] = dacc[j][1] = dacc[j][2] = dacc[j][3] = 0.f;
        for (int t = 0; t < n; t += 2) {
            float4 xa[2][2 * NP], xb[2][2 * NP];
            gather_tile<NP, GATHER>(xa, a, d, M, ptrs, t, gid, tig, fb);
            const bool two = t + 1 < n;
            if (two) gather_tile<NP, GATHER>(xb, a, d, M, ptrs, t + 1, gid, tig, fb);
            uint64_t bma = M.bits[t];
            if (a.bits_transposed) bma = transpose8x8(bma);
            tile_mma<NP>(dacc, xa, bma, gid, tig, (uint32_t)__popcll(bma) < thr);
            if (two) {
                uint64_t bmb = M.bits[t + 1];
                if (a.bits_transposed) bmb = transpose8x8(bmb);
                tile_mma<NP>(dacc, xb, bmb, gid, tig, (uint32_t)__popcll(bmb) < thr);
            }
        }
        // epilogue: lane holds output rows 2tig, 2tig+1 at float4 slots q = gid + 8s
        const bool heavy = cur.w != 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t row = w * 8 + 2 * tig + h;
            if (row >= a.num_out) continue;
            const float rsc = d.rs ? __ldg(d.rs + row) : 1.f;
            float* yrow = d.Y + (uint64_t)row * d.ldy;
#pragma unroll
            for (int s = 0; s < 2 * NP; ++s) {
                const uint32_t f = fb + 4 * (gid + 8 * s);
                if (f >= d.F) continue;
                const int p = s >> 1, e = (s & 1) * 2 + h;  // d[.][e]: rows (2tig | 2tig+1), m (gid | gid+8)
                float4 v = make_float4(dacc[4 * p + 0][e], dacc[4 * p + 1][e], dacc[4 * p + 2][e],
                                       dacc[4 * p + 3][e]);
                v = f4_scale(v, rsc);
                float* yp = yrow + f;
                // accumulate: a reduction, not load + add + store (the same fp32
                // add, without a DRAM round trip in the epilogue)
                if (heavy || accumulate) {
                    red_add_v4(yp, v);
                } else {
                    __stcs(reinterpret_cast<float4*>(yp), v);
                }
            }
        }
        __syncwarp();
        buf ^= 1;
        chunk = next;
        cur = nxt;
        nxt = nxt2;
    }
    cp_async_wait<0>();
}

// ---------------------------------------------------------------- push ----
// A window scatters its 8 input rows into the output rows of its tiles.
// Work split: every warp takes an equal contiguous slice of the tile range
// and walks the windows that meet it (a window's 8 input rows are reloaded
// by each warp that meets it), so a hub window with thousands of tiles is
// shared by many warps instead of setting the kernel's length.  SWTCF: the
// slices stay inside one super-window (its repeat cache lives in the CTA's
// shared memory); a super-window with more than kPushPartTiles tiles is
// split over up to kPushParts CTAs (adjacent blocks), each of which flushes the
// cached rows it touched.  Tile arithmetic (push_tile_mma): TF32 with rna
// operands for tiles with popcount >= tc_threshold, the fp32-level hi/lo TF32
// split otherwise, on the window's rows held in registers in fragment order;
// the partial sums are reduced straight from the MMA accumulators.
constexpr uint32_t kPushParts = 8;       // most CTAs per SWTCF super-window
constexpr uint32_t kPushPartTiles = 2048;  // tiles per CTA before a super-window is split

// First w in [lo, hi) with off[w + 1] > t (hi if none); uniform result.
__device__ __forceinline__ uint32_t warp_first_window(const uint32_t* __restrict__ off, uint32_t lo,
                                                      uint32_t hi, uint32_t t, int lane) {
    while (hi - lo > 32) {
        const uint32_t step = (hi - lo + 31) / 32;
        const uint32_t q = lo + lane * step;
        const bool tested = q < hi;
        const unsigned m = __ballot_sync(0xffffffffu, tested && off[q + 1] > t);
        if (m == 0) {  // the answer lies past the last tested probe
            const unsigned tm = __ballot_sync(0xffffffffu, tested);
            lo += (31 - __clz(tm)) * step + 1;
        } else {
            const int k = __ffs(m) - 1;
            hi = lo + k * step;
            if (k > 0) lo += (k - 1) * step + 1;
        }
    }
    const uint32_t q = lo + lane;
    const unsigned m = __ballot_sync(0xffffffffu, q < hi && off[q + 1] > t);
    return m ? lo + __ffs(m) - 1 : hi;
}

// One tile of the push pass: D[128 features x 8 output slots] = X_window . B,
// B[k][n] = bit(n*8 + k), in the permuted fragment order of tile_mma (lane
// (gid, tig) ends up holding 4 consecutive features of output slots 2tig and
// 2tig+1).  The window's rows arrive scaled (xr) with their exact remainders
// below TF32 (xl), both built once per window.  dense: TF32 with cvt.rna
// operands (the reference's dense-tile arithmetic); otherwise the hi/lo
// split, whose hi MMAs take the raw fp32 bits.
__device__ __forceinline__ void push_tile_mma(float (&dacc)[8][4], const float4 (&xr)[2][4],
                                              const float4 (&xl)[2][4], uint64_t bm, int gid,
                                              int tig, bool dense) {
    uint32_t b[2];
    b[0] = ((bm >> (gid * 8 + tig)) & 1ull) ? kOne : 0u;
    b[1] = ((bm >> (gid * 8 + tig + 4)) & 1ull) ? kOne : 0u;
    if (dense) {
#pragma unroll
        for (int p = 0; p < 2; ++p)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint32_t av[4] = {tf32_rna_bits(comp(xr[0][2 * p], c)),
                                        tf32_rna_bits(comp(xr[0][2 * p + 1], c)),
                                        tf32_rna_bits(comp(xr[1][2 * p], c)),
                                        tf32_rna_bits(comp(xr[1][2 * p + 1], c))};
                mma_tf32_16x8x8(dacc[4 * p + c], av, b);
            }
        return;
    }
#pragma unroll
    for (int p = 0; p < 2; ++p)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint32_t hi[4] = {__float_as_uint(comp(xr[0][2 * p], c)),
                                    __float_as_uint(comp(xr[0][2 * p + 1], c)),
                                    __float_as_uint(comp(xr[1][2 * p], c)),
                                    __float_as_uint(comp(xr[1][2 * p + 1], c))};
            mma_tf32_16x8x8(dacc[4 * p + c], hi, b);
        }
#pragma unroll
    for (int p = 0; p < 2; ++p)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint32_t lo[4] = {__float_as_uint(comp(xl[0][2 * p], c)),
                                    __float_as_uint(comp(xl[0][2 * p + 1], c)),
                                    __float_as_uint(comp(xl[1][2 * p], c)),
                                    __float_as_uint(comp(xl[1][2 * p + 1], c))};
            mma_tf32_16x8x8(dacc[4 * p + c], lo, b);
        }
}

__device__ __forceinline__ float4 f4_lo(float4 v) {  // v minus its TF32 truncation, exact
    auto one = [](float x) { return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); };
    return make_float4(one(v.x), one(v.y), one(v.z), one(v.w));
}

template <bool SWTCF, bool STORE>
__global__ void __launch_bounds__(kPushWarps * 32, 2) push_kernel(PushTiles a, Dense d,
                                                                  uint32_t thr, FeatureStore fs) {
    extern __shared__ __align__(16) float cache[];  // SWTCF: 32 x 128 repeat-cache rows
    __shared__ uint32_t touched;  // bit c: repeat-cache row c received a partial sum
    const int lane = threadIdx.x & 31;
    const int wib = threadIdx.x >> 5;
    const int gid = lane >> 2, tig = lane & 3;
    const uint32_t fb = blockIdx.y * 128;
    const uint32_t* off = a.win_offset;

    uint32_t s = 0, swoff = 0, wlo = 0, whi = a.num_windows, t0, t1;
    if (SWTCF) {
        s = blockIdx.x / kPushParts;  // a super-window's parts are adjacent blocks
        const uint32_t part = blockIdx.x % kPushParts;
        wlo = s * a.S;
        whi = min(a.num_windows, wlo + a.S);
        const uint32_t ta = off[wlo], len = off[whi] - ta;
        const uint32_t parts = min(kPushParts, max(1u, (len + kPushPartTiles - 1) / kPushPartTiles));
        if (part >= parts) return;  // uniform over the block, before any barrier
        const uint64_t pieces = (uint64_t)parts * kPushWarps;
        const uint64_t piece = (uint64_t)part * kPushWarps + wib;
        t0 = ta + (uint32_t)(len * piece / pieces);
        t1 = ta + (uint32_t)(len * (piece + 1) / pieces);
        swoff = a.sw_offset[s];
        for (int e = threadIdx.x; e < 32 * 128; e += blockDim.x) cache[e] = 0.f;
        if (threadIdx.x == 0) touched = 0;
        __syncthreads();
    } else {
        const uint64_t G = (uint64_t)gridDim.x * kPushWarps;
        const uint64_t g = (uint64_t)blockIdx.x * kPushWarps + wib;
        const uint64_t T = off[a.num_windows];
        t0 = (uint32_t)(T * g / G);
        t1 = (uint32_t)(T * (g + 1) / G);
    }

    // ---- per-tile metadata, two tiles ahead: bitmap + raw index (t + 2);
    // output row, repeat-cache slot and row scale (t + 1; dependent loads).
    // Lane n < 8 holds output slot n.
    auto load_raw = [&](uint32_t t, unsigned long long& bm, uint32_t& raw) {
        bm = 0;
        raw = kInvalid;
        if (t < t1) {
            bm = ld_stream_u64(a.bits + t);
            if (lane < 8) raw = ld_stream_u32(a.idx + (uint64_t)t * 8 + lane);
        }
    };
    auto resolve = [&](uint32_t raw, uint32_t& orow, uint32_t& cslot, float& rsc) {
        orow = kInvalid;
        cslot = 0xFFu;
        if (SWTCF) {
            if (raw != kInvalid) {
                orow = __ldg(a.sw_rows + swoff + raw);
                cslot = __ldg(a.sw_cache_slot + swoff + raw);
            }
        } else {
            orow = raw < a.num_out ? raw : kInvalid;
        }
        rsc = (d.rs && orow < a.num_out) ? __ldg(d.rs + orow) : 1.f;
    };

    // the window's 8 input rows in fragment order: lane holds rows k = tig + 4r
    // at features fb + 4*(gid + 8*sl), scaled by the column scale
    float4 xr[2][4], xl[2][4];
    auto load_window = [&](uint32_t w) {
        const float* xp = nullptr;
        if (STORE && lane < 8 && w * 8 + lane < a.num_in) xp = store_row(fs, w * 8 + lane, d.F);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int k = tig + 4 * r;
            const uint32_t cidx = w * 8 + k;
            const bool ok = cidx < a.num_in;
            const float* rowp = nullptr;
            if (STORE)
                rowp = reinterpret_cast<const float*>(
                    __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(xp), k));
            uint32_t g = cidx;
            float qs = 1.f;
            if (!STORE && d.qX && ok) {
                g = d.qmap ? __ldg(d.qmap + cidx) : cidx;
                qs = __ldg(d.qscale + g);
            }
            const float sc = (ok && d.cs) ? __ldg(d.cs + cidx) : 1.f;
#pragma unroll
            for (int sl = 0; sl < 4; ++sl) {
                const uint32_t f = fb + 4 * (gid + 8 * sl);
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (ok && f < d.F) {
                    if (STORE) {
                        v = *reinterpret_cast<const float4*>(rowp + f);
                    } else if (d.qX) {
                        // dequantize like the reference: float(q) * scale[g] in fp32
                        const char4 q = __ldg(reinterpret_cast<const char4*>(d.qX + (uint64_t)g * d.ldq + f));
                        v = make_float4((float)q.x * qs, (float)q.y * qs, (float)q.z * qs, (float)q.w * qs);
                    } else {
                        v = ld4(d.X + (uint64_t)cidx * d.ldx + f);
                    }
                }
                if (d.cs) v = f4_scale(v, sc);
                xr[r][sl] = v;
                xl[r][sl] = f4_lo(v);
            }
        }
    };

    if (t0 < t1) {
        uint32_t w = warp_first_window(off, wlo, whi, t0, lane);
        uint32_t wend = off[w + 1];
        load_window(w);
        unsigned long long bm0, bm1;
        uint32_t raw0, raw1, orow0, cslot0;
        float rsc0;
        load_raw(t0, bm0, raw0);
        load_raw(t0 + 1, bm1, raw1);
        resolve(raw0, orow0, cslot0, rsc0);
        for (uint32_t t = t0; t < t1; ++t) {
            if (t >= wend) {  // uniform: next window that holds tile t
                do {
                    ++w;
                    wend = off[w + 1];
                } while (wend <= t);
                load_window(w);
            }
            uint32_t orow1, cslot1, raw2;
            float rsc1;
            unsigned long long bm2;
            resolve(raw1, orow1, cslot1, rsc1);
            load_raw(t + 2, bm2, raw2);

            unsigned long long bm = bm0;
            if (a.bits_transposed) bm = transpose8x8(bm);
            float dacc[8][4];
#pragma unroll
            for (int j = 0; j < 8; ++j) dacc[j][0] = dacc[j][1] = dacc[j][2] = dacc[j][3] = 0.f;
            push_tile_mma(dacc, xr, xl, bm, gid, tig, (uint32_t)__popcll(bm) >= thr);
            // lane (gid, tig) reduces output slots 2tig, 2tig+1 at features
            // fb + 4*(gid + 8*sl): 8 lanes x 4 float4 cover one 128-feature row
            uint32_t r[2], cs[2];
            float rsc[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                r[h] = __shfl_sync(0xffffffffu, orow0, 2 * tig + h);
                cs[h] = __shfl_sync(0xffffffffu, cslot0, 2 * tig + h);
                rsc[h] = __shfl_sync(0xffffffffu, rsc0, 2 * tig + h);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int slot = 2 * tig + h;
                if (((bm >> (8 * slot)) & 0xFFull) == 0 || r[h] >= a.num_out) continue;
                const bool cached = SWTCF && cs[h] != 0xFFu;
#pragma unroll
                for (int sl = 0; sl < 4; ++sl) {
                    const uint32_t f = fb + 4 * (gid + 8 * sl);
                    if (f >= d.F) continue;
                    const int p = sl >> 1, e = (sl & 1) * 2 + h;
                    float4 v = make_float4(dacc[4 * p + 0][e], dacc[4 * p + 1][e],
                                           dacc[4 * p + 2][e], dacc[4 * p + 3][e]);
                    if (cached) {
                        float* cp = cache + cs[h] * 128 + (f - fb);
                        atomicAdd(cp + 0, v.x);
                        atomicAdd(cp + 1, v.y);
                        atomicAdd(cp + 2, v.z);
                        atomicAdd(cp + 3, v.w);
                    } else {
                        red_add_v4(d.Y + (uint64_t)r[h] * d.ldy + f, f4_scale(v, rsc[h]));
                    }
                }
                if (cached && gid == 0) atomicOr(&touched, 1u << cs[h]);
            }
            bm0 = bm1;
            orow0 = orow1;
            cslot0 = cslot1;
            rsc0 = rsc1;
            bm1 = bm2;
            raw1 = raw2;
        }
    }
    if (SWTCF) {
        __syncthreads();
        const uint32_t cc = a.sw_cached_count[s];
        const uint32_t used = touched;
        const uint32_t f = fb + lane * 4;
        for (uint32_t c = wib; c < cc; c += kPushWarps) {
            if (!((used >> c) & 1u)) continue;
            const uint32_t slot = a.sw_cached_row_slot[(uint64_t)s * 32 + c];
            const uint32_t row = a.sw_rows[swoff + slot];
            if (f >= d.F || row >= a.num_out) continue;
            float4 o = *reinterpret_cast<const float4*>(cache + c * 128 + lane * 4);
            if (d.rs) o = f4_scale(o, __ldg(d.rs + row));
            red_add_v4(d.Y + (uint64_t)row * d.ldy + f, o);
        }
    }
}

template <typename K>
int resident_blocks(K kernel, int threads) {
    int per_sm = 0;
    TCC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0));
    return std::max(1, per_sm) * sm_count();
}

template <int NP, int GATHER>
void launch_pull(const PullTiles& a, const Dense& d, const uint4* desc, PlanHeader* hdr,
                     uint64_t max_chunks, uint32_t thr, int accumulate, const FeatureStore& fs,
                     cudaStream_t s) {
    auto k = pull_kernel<NP, GATHER>;
    size_t smem = sizeof(WarpMeta) * 2 * kPullWarps;
    if (GATHER == kGatherStore) smem += sizeof(void*) * kChunkTiles * 8 * kPullWarps;
    TCC_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int per_sm = 0;
    TCC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kPullWarps * 32, smem));
    const uint64_t want = (max_chunks + kPullWarps - 1) / kPullWarps;
    const uint64_t resident = (uint64_t)std::max(1, per_sm) * grid_sms();
    const unsigned gx = (unsigned)std::max<uint64_t>(1, std::min<uint64_t>(want, resident));
    const unsigned gy = ceil_div(d.F, 64 * NP);
    k<<<dim3(gx, gy), kPullWarps * 32, smem, s>>>(a, d, desc, hdr, thr, accumulate, fs);
}

}  // namespace

size_t pull_scratch_bytes(uint32_t num_windows, uint32_t num_tiles) {
    return PlanLayout(num_windows, num_tiles).total;
}

// TCC_PULL_L2=hot: the bulk-copy pull kernel gives hot rows an evict-last and
// the others an evict-first L2 priority; TCC_PULL_L2=hub: only the hottest
// rows (a quarter of the hot budget) get evict-last and the others keep the
// normal priority.  The plan then builds the hot mask.
int l2_hint_mode() {
    const char* e = std::getenv("TCC_PULL_L2");
    if (!e) return 0;
    if (std::strcmp(e, "hot") == 0) return 1;
    if (std::strcmp(e, "hub") == 0) return 2;
    return 0;
}
bool l2_hints_requested() { return l2_hint_mode() != 0; }

// Work plan of the register-gather kernel in the scratch: chunk descriptors,
// split windows and a zeroed header (which also clears the error word).
void pull_plan(const PullTiles& a, void* scratch, size_t scratch_bytes, cudaStream_t s) {
    if (a.num_windows == 0) return;
    const PlanLayout L(a.num_windows, a.num_tiles);
    TCC_REQUIRE(scratch && scratch_bytes >= L.total, "pull scratch smaller than tcc_pull_scratch_bytes()");
    char* base = reinterpret_cast<char*>(scratch);
    PlanHeader* hdr = reinterpret_cast<PlanHeader*>(base);
    uint32_t* cstart = reinterpret_cast<uint32_t*>(base + L.cstart);
    uint4* desc = reinterpret_cast<uint4*>(base + L.desc);
    uint32_t* heavy = reinterpret_cast<uint32_t*>(base + L.heavy);
    const uint32_t W = a.num_windows;
    TCC_CUDA(cudaMemsetAsync(hdr, 0, sizeof(PlanHeader), s));
    plan_count_kernel<<<ceil_div(W, 256), 256, 0, s>>>(a.win_offset, W, cstart);
    exclusive_scan<uint32_t>(cstart, cstart, W, cstart + W, base + L.tmp, s);
    plan_fill_kernel<<<ceil_div(W, 256), 256, 0, s>>>(a.win_offset, W, cstart, desc, heavy, hdr);
    // hot gathered rows of the tiling (the column-window passes gather
    // through super-window slots: no hot mask there)
    if (!a.sw_rows && a.num_tiles > 0 && !l2_hints_requested()) {
        TCC_CUDA(cudaMemsetAsync(base + L.hot, 0, a.num_tiles, s));  // defined: no hot rows
    } else if (!a.sw_rows && a.num_tiles > 0) {
        uint32_t* sketch = reinterpret_cast<uint32_t*>(base + L.sketch);
        uint32_t* hist = reinterpret_cast<uint32_t*>(base + L.hist);
        const unsigned g = (unsigned)std::max(1, sm_count() * 8);
        TCC_CUDA(cudaMemsetAsync(sketch, 0, (size_t)kSketch * 4, s));
        TCC_CUDA(cudaMemsetAsync(hist, 0, (size_t)kCountBins * 4 + 16, s));
        hot_count_kernel<<<g, 256, 0, s>>>(a.idx, (uint64_t)a.num_tiles * 8, a.num_in, sketch);
        hot_hist_kernel<<<g, 256, 0, s>>>(sketch, hist);
        hot_threshold_kernel<<<1, 32, 0, s>>>(hist, l2_hint_mode() == 2 ? kHotRows / 4 : kHotRows);
        hot_mask_kernel<<<g, 256, 0, s>>>(a.idx, a.num_tiles, a.num_in, sketch, hist,
                                          reinterpret_cast<uint8_t*>(base + L.hot));
    }
    TCC_CUDA(cudaGetLastError());
}

void pull_spmm(const PullTiles& a, const Dense& d, uint32_t tc_threshold, int accumulate,
               void* scratch, size_t scratch_bytes, bool plan_ready, const FeatureStore* fs,
               cudaStream_t s, bool keep_plan) {
    TCC_REQUIRE(d.F > 0 && d.F % 4 == 0, "F must be a positive multiple of 4");
    TCC_REQUIRE(d.ldx % 4 == 0 && d.ldy % 4 == 0 && d.ldx >= d.F && d.ldy >= d.F,
                "row strides must be multiples of 4 elements and >= F");
    TCC_REQUIRE(fs || ((uintptr_t)d.X % 16 == 0), "X must be 16-byte aligned");
    TCC_REQUIRE((uintptr_t)d.Y % 16 == 0, "Y must be 16-byte aligned");
    TCC_REQUIRE((uintptr_t)a.idx % 16 == 0 && (uintptr_t)a.bits % 8 == 0,
                "tile index / bitmap arrays must be 16 / 8-byte aligned");
    if (a.num_windows == 0) return;
    const PlanLayout L(a.num_windows, a.num_tiles);
    TCC_REQUIRE(scratch && scratch_bytes >= L.total, "pull scratch smaller than tcc_pull_scratch_bytes()");
    char* base = reinterpret_cast<char*>(scratch);
    PlanHeader* hdr = reinterpret_cast<PlanHeader*>(base);
    uint4* desc = reinterpret_cast<uint4*>(base + L.desc);
    uint32_t* heavy = reinterpret_cast<uint32_t*>(base + L.heavy);
    static_assert(offsetof(PlanHeader, pad) == kPullErrorOffset, "error word offset");
    // the bulk-copy and tcgen05 kernels split the tile range themselves and
    // read only the header's error word; the plan is built for them too unless
    // the caller will not reuse it (keep_plan false), so that a later call with
    // plan_ready = 1 that dispatches to the register-gather kernel finds it
    const bool umma = !fs && pull_umma_eligible(a, d, tc_threshold);
    const bool tma = !umma && !fs && pull_tma_eligible(a, d);
    if (!plan_ready) {
        if (keep_plan || !(umma || tma)) pull_plan(a, scratch, scratch_bytes, s);
        else TCC_CUDA(cudaMemsetAsync(hdr, 0, sizeof(PlanHeader), s));
    }
    if (umma) {
        pull_umma(a, d, accumulate, &hdr->pad[0], s);
        return;
    }
    if (tma) {
        PullTiles at = a;
        // the hot-row mask exists when the plan was built (plan_ready, or
        // built above); the no-allocation entry builds none for this kernel
        if (!a.sw_rows && a.num_tiles > 0 && (plan_ready || keep_plan))
            at.hot = reinterpret_cast<const uint8_t*>(base + L.hot);
        pull_tma(at, d, tc_threshold, accumulate, &hdr->pad[0], s);
        return;
    }
    if (!accumulate)
        zero_heavy_kernel<<<std::max(1, sm_count() * 2), 256, 0, s>>>(heavy, hdr, d.Y, d.ldy, d.F,
                                                                       a.num_out);
    FeatureStore none;
    const FeatureStore& f = fs ? *fs : none;
    // 64 features per MMA pass pair: F <= 64 uses one, wider F two per block
    const bool narrow = d.F <= 64;
    if (fs) {
        if (narrow) launch_pull<1, kGatherStore>(a, d, desc, hdr, L.max_chunks, tc_threshold, accumulate, f, s);
        else launch_pull<2, kGatherStore>(a, d, desc, hdr, L.max_chunks, tc_threshold, accumulate, f, s);
    } else if (a.sw_rows) {
        if (narrow) launch_pull<1, kGatherSwtcf>(a, d, desc, hdr, L.max_chunks, tc_threshold, accumulate, f, s);
        else launch_pull<2, kGatherSwtcf>(a, d, desc, hdr, L.max_chunks, tc_threshold, accumulate, f, s);
    } else {
        if (narrow) launch_pull<1, kGatherDense>(a, d, desc, hdr, L.max_chunks, tc_threshold, accumulate, f, s);
        else launch_pull<2, kGatherDense>(a, d, desc, hdr, L.max_chunks, tc_threshold, accumulate, f, s);
    }
    TCC_CUDA(cudaGetLastError());
}

void push_spmm(const PushTiles& a, const Dense& d, uint32_t tc_threshold, const FeatureStore* fs,
               cudaStream_t s) {
    TCC_REQUIRE(d.F > 0 && d.F % 4 == 0, "F must be a positive multiple of 4");
    TCC_REQUIRE(d.ldy % 4 == 0 && d.ldy >= d.F, "Y row stride must be a multiple of 4 and >= F");
    if (d.qX) {
        TCC_REQUIRE(!fs, "quantized rows and a feature store exclude each other");
        TCC_REQUIRE(d.qscale && d.ldq % 4 == 0 && d.ldq >= d.F && (uintptr_t)d.qX % 4 == 0,
                    "quantized X needs scales, a 4-byte aligned base and a row stride that is a "
                    "multiple of 4 and >= F");
    } else {
        TCC_REQUIRE(d.ldx % 4 == 0 && d.ldx >= d.F, "X row stride must be a multiple of 4 and >= F");
        TCC_REQUIRE(fs || ((uintptr_t)d.X % 16 == 0), "X must be 16-byte aligned");
    }
    TCC_REQUIRE((uintptr_t)d.Y % 16 == 0, "Y must be 16-byte aligned");
    if (a.num_windows == 0) return;
    const unsigned gy = ceil_div(d.F, 128);
    FeatureStore none;
    const FeatureStore& f = fs ? *fs : none;
    if (a.sw_rows) {
        TCC_REQUIRE(!fs, "the SWTCF pass reads a dense X");
        const uint32_t SW = (a.num_windows + a.S - 1) / a.S;
        auto k = push_kernel<true, false>;
        constexpr int kCacheBytes = 32 * 128 * sizeof(float);
        TCC_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kCacheBytes));
        k<<<dim3(SW * kPushParts, gy), kPushWarps * 32, kCacheBytes, s>>>(a, d, tc_threshold, f);
    } else {
        const unsigned want = ceil_div(a.num_windows, kPushWarps);
        if (fs) {
            auto k = push_kernel<false, true>;
            const unsigned gx = std::max(1u, std::min<unsigned>(want, resident_blocks(k, kPushWarps * 32)));
            k<<<dim3(gx, gy), kPushWarps * 32, 0, s>>>(a, d, tc_threshold, f);
        } else {
            auto k = push_kernel<false, false>;
            const unsigned gx = std::max(1u, std::min<unsigned>(want, resident_blocks(k, kPushWarps * 32)));
            k<<<dim3(gx, gy), kPushWarps * 32, 0, s>>>(a, d, tc_threshold, f);
        }
    }
    TCC_CUDA(cudaGetLastError());
}

}  // namespace tcc
