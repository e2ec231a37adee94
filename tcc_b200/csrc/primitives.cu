// primitives.cu -- exclusive scan and stable LSD radix sort (sm_100a).
//
// These replace the CUB DeviceScan / DeviceRadixSort / DeviceRunLengthEncode
// calls of the reference converter (src/swtcf_convert.cu:1951-2007).  The sort
// is a classic three-kernel LSD pass (tile histograms, scan of the digit-major
// histogram table, stable tile-local ranking + coalesced scatter).  Ranking:
// each warp owns a contiguous run of the tile and ranks it against a
// warp-private digit histogram (__match_any_sync groups equal digits; no
// block barrier per item); one block-wide prefix over the warps' histograms
// then places every warp's items after those of the warps before it, so each
// pass is stable and deterministic.
#include "primitives.cuh"

namespace tcc {
namespace {

constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;                       // per thread, striped
constexpr int kScanTile = kScanThreads * kScanItems;  // 2048 elements per block

template <typename T>
__device__ __forceinline__ T warp_inclusive(T v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        T n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

// Block-wide exclusive scan of one value per thread; returns the block total.
template <typename T>
__device__ __forceinline__ T block_exclusive(T v, T* warp_sums, T& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    T inc = warp_inclusive(v);
    if (lane == 31) warp_sums[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        T w = lane < (kScanThreads / 32) ? warp_sums[lane] : T(0);
        T wi = warp_inclusive(w);
        if (lane < (kScanThreads / 32)) warp_sums[lane] = wi - w;
        if (lane == (kScanThreads / 32) - 1) warp_sums[kScanThreads / 32] = wi;
    }
    __syncthreads();
    T excl = inc - v + warp_sums[warp];
    total = warp_sums[kScanThreads / 32];
    __syncthreads();
    return excl;
}

template <typename T>
__global__ void __launch_bounds__(kScanThreads) scan_reduce_kernel(const T* __restrict__ in,
                                                                   uint64_t n,
                                                                   T* __restrict__ partial) {
    __shared__ T ws[kScanThreads / 32 + 1];
    const uint64_t base = (uint64_t)blockIdx.x * kScanTile;
    T s = 0;
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        const uint64_t i = base + (uint64_t)j * kScanThreads + threadIdx.x;
        if (i < n) s += in[i];
    }
    T total;
    block_exclusive<T>(s, ws, total);
    if (threadIdx.x == 0) partial[blockIdx.x] = total;
}

template <typename T>
__global__ void __launch_bounds__(kScanThreads) scan_partials_kernel(T* __restrict__ partial,
                                                                     uint64_t nb,
                                                                     T* __restrict__ d_total) {
    __shared__ T ws[kScanThreads / 32 + 1];
    T carry = 0;
    for (uint64_t base = 0; base < nb; base += kScanThreads) {
        const uint64_t i = base + threadIdx.x;
        T v = i < nb ? partial[i] : T(0);
        T total;
        T e = block_exclusive<T>(v, ws, total);
        if (i < nb) partial[i] = e + carry;
        carry += total;
    }
    if (threadIdx.x == 0 && d_total) *d_total = carry;
}

template <typename T>
__global__ void __launch_bounds__(kScanThreads) scan_down_kernel(const T* in, uint64_t n,
                                                                 const T* __restrict__ partial,
                                                                 T* out) {
    __shared__ T ws[kScanThreads / 32 + 1];
    const uint64_t base = (uint64_t)blockIdx.x * kScanTile;
    T v[kScanItems];
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        const uint64_t i = base + (uint64_t)j * kScanThreads + threadIdx.x;
        v[j] = i < n ? in[i] : T(0);
    }
    __syncthreads();  // all reads of this tile precede writes (in == out allowed)
    T carry = partial[blockIdx.x];
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        T total;
        T e = block_exclusive<T>(v[j], ws, total);
        const uint64_t i = base + (uint64_t)j * kScanThreads + threadIdx.x;
        if (i < n) out[i] = e + carry;
        carry += total;
    }
}

// ------------------------------------------------------------ radix sort --
constexpr int kSortThreads = 256;
constexpr int kSortItems = 16;
constexpr int kSortTile = kSortThreads * kSortItems;  // 4096 keys per tile
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kRadix = 256;

__global__ void __launch_bounds__(kSortThreads) radix_upsweep_kernel(
    const uint64_t* __restrict__ keys, uint64_t n, int shift, uint32_t num_tiles,
    uint32_t* __restrict__ counts) {
    __shared__ uint32_t hist[kRadix];
    hist[threadIdx.x] = 0;
    __syncthreads();
    const uint64_t base = (uint64_t)blockIdx.x * kSortTile;
#pragma unroll 4
    for (int j = 0; j < kSortItems; ++j) {
        const uint64_t i = base + (uint64_t)j * kSortThreads + threadIdx.x;
        if (i < n) atomicAdd(&hist[(keys[i] >> shift) & 0xFFu], 1u);
    }
    __syncthreads();
    counts[(uint64_t)threadIdx.x * num_tiles + blockIdx.x] = hist[threadIdx.x];
}

struct SortSmem {
    uint64_t keys[kSortTile];
    uint32_t vals[kSortTile];
    uint32_t warp_cnt[kSortWarps][kRadix + 1];  // digit counts, then prefixes; [kRadix]: sentinel
    uint32_t digit_start[kRadix];
    uint32_t out_base[kRadix];  // global position of the tile's first key of each digit
    uint32_t scan_ws[kScanThreads / 32 + 1];
};

// Warp w ranks tile items [w * kWarpItems, (w + 1) * kWarpItems), item j of
// lane l at w * kWarpItems + j * 32 + l: the rank of an item among its warp's
// items with the same digit is the warp's running count for that digit plus
// the equal digits of lower lanes in the same step.
constexpr int kWarpItems = kSortTile / kSortWarps;  // 512
static_assert(kWarpItems == kSortItems * 32, "one warp-contiguous run per warp");

__global__ void __launch_bounds__(kSortThreads) radix_downsweep_kernel(
    const uint64_t* __restrict__ keys, const uint32_t* __restrict__ vals, uint64_t n, int shift,
    uint32_t num_tiles, const uint32_t* __restrict__ offsets, uint64_t* __restrict__ keys_out,
    uint32_t* __restrict__ vals_out) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    SortSmem& S = *reinterpret_cast<SortSmem*>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint64_t base = (uint64_t)blockIdx.x * kSortTile;
    const uint64_t rem_n = n - base;
    const uint32_t tile_n = rem_n < (uint64_t)kSortTile ? (uint32_t)rem_n : (uint32_t)kSortTile;
    for (int i = lane; i <= kRadix; i += 32) S.warp_cnt[warp][i] = 0;
    __syncwarp();
    uint64_t k[kSortItems];
    uint32_t v[kSortItems];
    uint32_t d[kSortItems];
    uint32_t rank[kSortItems];
#pragma unroll
    for (int j = 0; j < kSortItems; ++j) {
        const uint32_t p = (uint32_t)(warp * kWarpItems + j * 32 + lane);
        if (p < tile_n) {
            k[j] = keys[base + p];
            v[j] = vals[base + p];
            d[j] = (uint32_t)(k[j] >> shift) & 0xFFu;
        } else {
            k[j] = 0;
            v[j] = 0;
            d[j] = kRadix;  // sentinel bucket: never written out
        }
    }
    uint32_t* cnt = S.warp_cnt[warp];
#pragma unroll
    for (int j = 0; j < kSortItems; ++j) {
        const unsigned peers = __match_any_sync(0xffffffffu, d[j]);
        const uint32_t before = cnt[d[j]];
        __syncwarp();
        if ((peers & lanemask_lt()) == 0) cnt[d[j]] = before + __popc(peers);
        __syncwarp();
        rank[j] = before + __popc(peers & lanemask_lt());
    }
    __syncthreads();
    // digit t: exclusive prefix over the warps, then over the digits
    uint32_t run = 0;
#pragma unroll
    for (int w = 0; w < kSortWarps; ++w) {
        const uint32_t c = S.warp_cnt[w][tid];
        S.warp_cnt[w][tid] = run;
        run += c;
    }
    uint32_t total;
    const uint32_t start = block_exclusive<uint32_t>(run, S.scan_ws, total);
    S.digit_start[tid] = start;
    // one global offset per digit, read once here instead of once per key below
    S.out_base[tid] = offsets[(uint64_t)tid * num_tiles + blockIdx.x] - start;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kSortItems; ++j) {
        if (d[j] < kRadix) {
            const uint32_t p = S.digit_start[d[j]] + cnt[d[j]] + rank[j];
            S.keys[p] = k[j];
            S.vals[p] = v[j];
        }
    }
    __syncthreads();
#pragma unroll 4
    for (int j = 0; j < kSortItems; ++j) {
        const uint32_t p = (uint32_t)j * kSortThreads + tid;
        if (p < tile_n) {
            const uint64_t key = S.keys[p];
            const uint32_t dg = (uint32_t)(key >> shift) & 0xFFu;
            const uint64_t g = (uint64_t)S.out_base[dg] + p;
            keys_out[g] = key;
            vals_out[g] = S.vals[p];
        }
    }
}

}  // namespace

size_t scan_tmp_bytes(uint64_t n) {
    const uint64_t nb = (n + kScanTile - 1) / kScanTile;
    return (size_t)((nb + 1) * sizeof(uint64_t));
}

template <typename T>
void exclusive_scan(const T* in, T* out, uint64_t n, T* d_total, void* tmp, cudaStream_t s) {
    if (n == 0) {
        if (d_total) TCC_CUDA(cudaMemsetAsync(d_total, 0, sizeof(T), s));
        return;
    }
    const uint64_t nb = (n + kScanTile - 1) / kScanTile;
    T* partial = reinterpret_cast<T*>(tmp);
    scan_reduce_kernel<T><<<(unsigned)nb, kScanThreads, 0, s>>>(in, n, partial);
    scan_partials_kernel<T><<<1, kScanThreads, 0, s>>>(partial, nb, d_total);
    scan_down_kernel<T><<<(unsigned)nb, kScanThreads, 0, s>>>(in, n, partial, out);
    TCC_CUDA(cudaGetLastError());
}

template void exclusive_scan<uint32_t>(const uint32_t*, uint32_t*, uint64_t, uint32_t*, void*,
                                       cudaStream_t);
template void exclusive_scan<uint64_t>(const uint64_t*, uint64_t*, uint64_t, uint64_t*, void*,
                                       cudaStream_t);

size_t radix_tmp_bytes(uint64_t n) {
    const uint64_t tiles = (n + kSortTile - 1) / kSortTile;
    const uint64_t counts = tiles * kRadix;
    return (size_t)(counts * sizeof(uint32_t) + 256) + scan_tmp_bytes(counts);
}

bool radix_sort_pairs(uint64_t* keys, uint32_t* vals, uint64_t* keys_alt, uint32_t* vals_alt,
                      uint64_t n, int key_bits, void* tmp, cudaStream_t s, int first_bit) {
    TCC_REQUIRE(n < (1ull << 31), "radix sort supports fewer than 2^31 items per call");
    TCC_REQUIRE(first_bit >= 0, "negative first sort bit");
    if (n <= 1 || key_bits <= first_bit) return false;
    const uint32_t tiles = (uint32_t)((n + kSortTile - 1) / kSortTile);
    uint32_t* counts = reinterpret_cast<uint32_t*>(tmp);
    const uint64_t ncounts = (uint64_t)tiles * kRadix;
    void* scan_tmp = reinterpret_cast<char*>(tmp) + ((ncounts * sizeof(uint32_t) + 255) / 256) * 256;
    // per-device attribute: set on every call (cheap), the current device may change
    TCC_CUDA(cudaFuncSetAttribute(radix_downsweep_kernel,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)sizeof(SortSmem)));
    uint64_t* kin = keys;
    uint32_t* vin = vals;
    uint64_t* kout = keys_alt;
    uint32_t* vout = vals_alt;
    bool in_alt = false;
    for (int shift = first_bit; shift < key_bits; shift += 8) {
        radix_upsweep_kernel<<<tiles, kSortThreads, 0, s>>>(kin, n, shift, tiles, counts);
        exclusive_scan<uint32_t>(counts, counts, ncounts, nullptr, scan_tmp, s);
        radix_downsweep_kernel<<<tiles, kSortThreads, sizeof(SortSmem), s>>>(
            kin, vin, n, shift, tiles, counts, kout, vout);
        TCC_CUDA(cudaGetLastError());
        std::swap(kin, kout);
        std::swap(vin, vout);
        in_alt = !in_alt;
    }
    return in_alt;
}

}  // namespace tcc
