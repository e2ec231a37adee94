// convert.cu -- COO/CSR -> SWTCF and CSR -> BCSR / BCSC window tiling (sm_100a).
//
// One integer pipeline serves all three layouts.  Every nonzero (x, y) falls in
// window x>>3 with local bit x&7; a "group" is one distinct (window, y) with the
// OR of its local bits (SWTCF: x = src, y = dst; BCSR: x = row, y = col; BCSC:
// x = col, y = row).  Steps:
//   1. keys (window << ybits | y), payload = local bit      (src/swtcf_convert.cu:104-144)
//   2. stable radix sort of the keys                         (:1951-1966, CUB there)
//   3. run heads -> group ids -> group masks                 (:1977-2007, RLE there)
//   4. groups per window -> tiles per window -> offsets      (:147-289)
//   5. layout-specific fill:
//      BCSR/BCSC: group p of window w -> tile off[w]+p/8, slot p%8 (consumer
//                 layout of cnic/src/core/spmm_kernel.cu:1632-1660, :1922-1968)
//      SWTCF:     degree-descending order (stable radix sort on (window, 8-deg),
//                 replacing the atomic cursor of :292-376), super-window unique
//                 rows by sorting (replacing the hash table of :459-681 and
//                 :898-1000), repeat-cache ranks per super-window (:699-895).
// Nothing depends on atomic arrival order, so outputs are canonical.
#include "primitives.cuh"
#include "convert.cuh"

namespace tcc {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ void raise_error(uint32_t* err, uint32_t code) {
    atomicCAS(err, 0u, code);  // first error wins
}

// ---------------------------------------------------------------- step 1 --
__global__ void keys_from_coo_kernel(const uint32_t* __restrict__ dst,
                                     const uint32_t* __restrict__ src, uint64_t n, uint32_t rows,
                                     uint32_t cols, int ybits, uint64_t* __restrict__ keys,
                                     uint32_t* __restrict__ vals, uint32_t* err) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t x = src[i], y = dst[i];
    if (x >= cols || y >= rows) {  // keep every later index in bounds
        raise_error(err, TCC_DEVERR_INDEX_RANGE);
        x = 0;
        y = 0;
    }
    keys[i] = ((uint64_t)(x >> 3) << ybits) | y;
    vals[i] = x & 7u;
}

// CSR -> keys.  mode 0: window = row (BCSR); mode 1: window = col (BCSC, SWTCF).
// A block owns kKeyTile consecutive nonzeros; its first thread finds the rows
// of the first and last one (binary searches over rowptr), the block stages
// rowptr over that row range in shared memory when it fits, and every thread
// finds its nonzero's row by a binary search over that short range (the
// whole-array search per nonzero, and a warp per row, which serialises on
// the hub rows of power-law graphs, were both slower).
constexpr int kKeyTile = 2048;
constexpr int kKeyRows = 2048;
__device__ __forceinline__ uint32_t row_of(const uint64_t* rp, uint32_t lo, uint32_t hi, uint64_t i) {
    // largest r in [lo, hi] with rp[r] <= i
    while (lo < hi) {
        const uint32_t mid = lo + (hi - lo + 1) / 2;
        if (rp[mid] <= i) lo = mid; else hi = mid - 1;
    }
    return lo;
}

__global__ void __launch_bounds__(256) keys_from_csr_kernel(
    const uint64_t* __restrict__ rowptr, const uint32_t* __restrict__ col, uint32_t rows,
    uint32_t cols, uint64_t n, int mode, int ybits, uint64_t* __restrict__ keys,
    uint32_t* __restrict__ vals, uint32_t* err) {
    __shared__ uint64_t srp[kKeyRows + 1];
    __shared__ uint32_t range[2];
    const uint64_t b0 = (uint64_t)blockIdx.x * kKeyTile;
    if (b0 >= n || rows == 0) return;
    const uint64_t b1 = min(n, b0 + kKeyTile);
    if (threadIdx.x == 0) {
        const uint32_t last = rows - 1;
        range[0] = row_of(rowptr, 0, last, b0);
        range[1] = row_of(rowptr, range[0], last, b1 - 1);
    }
    __syncthreads();
    const uint32_t r0 = range[0], r1 = range[1];
    const bool staged = r1 - r0 < (uint32_t)kKeyRows;
    if (staged)
        for (uint32_t j = threadIdx.x; j <= r1 - r0; j += blockDim.x) srp[j] = rowptr[r0 + j];
    __syncthreads();
    for (uint64_t i = b0 + threadIdx.x; i < b1; i += blockDim.x) {
        const uint32_t r = staged ? r0 + row_of(srp, 0, r1 - r0, i) : row_of(rowptr, r0, r1, i);
        uint32_t c = col[i];
        if (c >= cols) {
            raise_error(err, TCC_DEVERR_INDEX_RANGE);
            c = 0;
        }
        const uint32_t x = mode == 0 ? r : c;
        const uint32_t y = mode == 0 ? c : r;
        keys[i] = ((uint64_t)(x >> 3) << ybits) | y;
        vals[i] = x & 7u;
    }
}

// SWTCF tile t of column window w (the largest w with col_off[w] <= t): each
// set bit (localRow r, localCol c) is the nonzero (sw_rows[sw_off[w/S] +
// slots[8t + r]], 8w + c), written as a row-window key at pos[t], pos[t] + 1, ...
// (pos = exclusive prefix of the tile popcounts).
__global__ void keys_from_swtcf_kernel(const uint32_t* __restrict__ col_off, uint32_t W, uint32_t S,
                                       const uint32_t* __restrict__ sw_off,
                                       const uint32_t* __restrict__ sw_rows,
                                       const uint32_t* __restrict__ slots,
                                       const uint64_t* __restrict__ bits,
                                       const uint32_t* __restrict__ pos, uint32_t T, uint32_t rows,
                                       uint32_t cols, int ybits, uint64_t* __restrict__ keys,
                                       uint32_t* __restrict__ vals, uint32_t* err) {
    const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    uint32_t lo = 0, hi = W - 1;
    while (lo < hi) {
        const uint32_t mid = lo + (hi - lo + 1) / 2;
        if (col_off[mid] <= t) lo = mid; else hi = mid - 1;
    }
    const uint32_t w = lo;
    const uint32_t swoff = sw_off[w / S];
    unsigned long long b = bits[t];
    uint32_t p = pos[t];
    while (b) {
        const int k = __ffsll((long long)b) - 1;
        b &= b - 1;
        const uint32_t slot = slots[(uint64_t)t * 8 + (k >> 3)];
        uint32_t row = slot == 0xFFFFFFFFu ? rows : sw_rows[swoff + slot];
        uint32_t col = w * 8 + (k & 7);
        if (row >= rows || col >= cols) {
            raise_error(err, TCC_DEVERR_INDEX_RANGE);
            row = 0;
            col = 0;
        }
        keys[p] = ((uint64_t)(row >> 3) << ybits) | col;
        vals[p] = row & 7u;
        ++p;
    }
}

// ---------------------------------------------------------------- step 3 --
__global__ void mark_heads_kernel(const uint64_t* __restrict__ keys, uint64_t n,
                                  uint32_t* __restrict__ head) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    head[i] = (i == 0 || keys[i] != keys[i - 1]) ? 1u : 0u;
}

__global__ void groups_kernel(const uint64_t* __restrict__ keys, const uint32_t* __restrict__ vals,
                              const uint32_t* __restrict__ head, const uint32_t* __restrict__ excl,
                              uint64_t n, uint64_t* __restrict__ gkey, uint32_t* __restrict__ gmask,
                              uint32_t* __restrict__ gstart) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t g = excl[i] + head[i] - 1;
    if (head[i]) {
        gkey[g] = keys[i];
        gstart[g] = (uint32_t)i;
    }
    atomicOr(&gmask[g], 1u << vals[i]);
}

// ---------------------------------------------------------------- step 4 --
// Duplicate check per group: a group's edge count must equal its popcount.
__global__ void group_check_kernel(const uint32_t* __restrict__ gmask,
                                   const uint32_t* __restrict__ gstart,
                                   const uint32_t* __restrict__ d_ng, uint64_t n,
                                   uint32_t* err) {
    const uint64_t g = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t ng = *d_ng;
    if (g >= ng) return;
    const uint32_t count = (g + 1 < ng ? gstart[g + 1] : (uint32_t)n) - gstart[g];
    if ((uint32_t)__popc(gmask[g]) != count) raise_error(err, TCC_DEVERR_GROUP_DEGREE);
}

// First group of each window (groups are sorted by window): lower bound of
// window w in the group keys; wgstart[W] = number of groups.
__global__ void window_start_kernel(const uint64_t* __restrict__ gkey,
                                    const uint32_t* __restrict__ d_ng, int ybits, uint32_t W,
                                    uint32_t* __restrict__ wgstart) {
    const uint32_t w = blockIdx.x * blockDim.x + threadIdx.x;
    if (w > W) return;
    uint32_t lo = 0, hi = *d_ng;
    while (lo < hi) {
        const uint32_t mid = lo + (hi - lo) / 2;
        if ((gkey[mid] >> ybits) < w) lo = mid + 1; else hi = mid;
    }
    wgstart[w] = lo;
}

__global__ void window_tiles_kernel(const uint32_t* __restrict__ wgstart, uint32_t W,
                                    uint32_t* __restrict__ wcnt, uint32_t* __restrict__ tiles) {
    const uint32_t w = blockIdx.x * blockDim.x + threadIdx.x;
    if (w >= W) return;
    const uint32_t c = wgstart[w + 1] - wgstart[w];
    wcnt[w] = c;
    tiles[w] = (c + 7u) / 8u;
}

// Padding of each window's last tile: slot / index 0xFFFFFFFF, bitmap byte 0.
// byte_bits: zero the padding bytes of tileLocalBit (SWTCF / BCSC byte rows).
__global__ void tile_padding_kernel(const uint32_t* __restrict__ wcnt,
                                    const uint32_t* __restrict__ off, uint32_t W,
                                    uint32_t* __restrict__ idx, uint64_t* __restrict__ bits,
                                    int byte_bits) {
    const uint32_t w = blockIdx.x * blockDim.x + threadIdx.x;
    if (w >= W) return;
    const uint32_t rem = wcnt[w] & 7u;
    if (rem == 0) return;
    const uint32_t last = off[w + 1] - 1;
    for (uint32_t k = rem; k < 8; ++k) {
        idx[(uint64_t)last * 8 + k] = kInvalid;
        if (byte_bits) reinterpret_cast<uint8_t*>(bits + last)[k] = 0;
    }
}

// ----------------------------------------------------------- BCSR / BCSC --
__global__ void fill_tiles_kernel(const uint64_t* __restrict__ gkey,
                                  const uint32_t* __restrict__ gmask, uint32_t ng, int ybits,
                                  const uint32_t* __restrict__ wgstart,
                                  const uint32_t* __restrict__ off, int row_major,
                                  uint32_t* __restrict__ idx, uint64_t* __restrict__ bits) {
    const uint32_t g = blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= ng) return;
    const uint64_t key = gkey[g];
    const uint32_t w = (uint32_t)(key >> ybits);
    const uint32_t y = (uint32_t)(key & ((1ull << ybits) - 1));
    const uint32_t p = g - wgstart[w];
    const uint64_t t = (uint64_t)off[w] + p / 8;
    const uint32_t k = p & 7u;
    idx[t * 8 + k] = y;
    const uint32_t m = gmask[g];
    if (row_major) {  // BCSR: mask bit r (local row) -> tile bit r*8 + k
        uint64_t b = 0;
#pragma unroll
        for (int r = 0; r < 8; ++r)
            if (m & (1u << r)) b |= 1ull << (r * 8 + k);
        atomicOr(reinterpret_cast<unsigned long long*>(bits + t), (unsigned long long)b);
    } else {          // BCSC: mask bit k (local col) -> tile byte k of row slot p
        reinterpret_cast<uint8_t*>(bits + t)[k] = (uint8_t)m;
    }
}

__global__ void popcount_kernel(const uint64_t* __restrict__ bits, uint64_t T,
                                uint32_t* __restrict__ out) {
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t < T) out[t] = (uint32_t)__popcll(bits[t]);
}

// ------------------------------------------------------------------ SWTCF --
// Sort keys for the degree-descending order: (window, 8 - degree); groups past
// the end sort last (pad key = all ones over the key bits).
__global__ void degree_keys_kernel(const uint64_t* __restrict__ gkey,
                                   const uint32_t* __restrict__ gmask,
                                   const uint32_t* __restrict__ d_ng, uint64_t n, int ybits,
                                   int key_bits, uint64_t* __restrict__ keys,
                                   uint32_t* __restrict__ vals) {
    const uint64_t g = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= n) return;
    const uint32_t ng = *d_ng;
    if (g < ng) {
        const uint64_t w = gkey[g] >> ybits;
        keys[g] = (w << 3) | (uint64_t)(8 - __popc(gmask[g]));
    } else {
        keys[g] = (1ull << key_bits) - 1;
    }
    vals[g] = (uint32_t)g;
}

__global__ void superwindow_keys_kernel(const uint64_t* __restrict__ gkey,
                                        const uint32_t* __restrict__ d_ng, uint64_t n, int ybits,
                                        uint32_t S, int key_bits, uint64_t* __restrict__ keys,
                                        uint32_t* __restrict__ vals) {
    const uint64_t g = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= n) return;
    const uint32_t ng = *d_ng;
    if (g < ng) {
        const uint64_t key = gkey[g];
        const uint64_t s = (key >> ybits) / S;
        keys[g] = (s << ybits) | (key & ((1ull << ybits) - 1));
    } else {
        keys[g] = (1ull << key_bits) - 1;
    }
    vals[g] = (uint32_t)g;
}

__global__ void row_heads_kernel(const uint64_t* __restrict__ keys,
                                 const uint32_t* __restrict__ d_ng, uint64_t n,
                                 uint32_t* __restrict__ head) {
    const uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= n) return;
    const uint32_t ng = *d_ng;
    head[q] = (q < ng && (q == 0 || keys[q] != keys[q - 1])) ? 1u : 0u;
}

__global__ void superwindow_rows_kernel(const uint64_t* __restrict__ keys,
                                        const uint32_t* __restrict__ head,
                                        const uint32_t* __restrict__ excl,
                                        const uint32_t* __restrict__ d_ng, int ybits,
                                        uint32_t* __restrict__ rows_out,
                                        uint32_t* __restrict__ rstart,
                                        uint32_t* __restrict__ rsw) {
    const uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= *d_ng || !head[q]) return;
    const uint32_t r = excl[q];
    const uint64_t key = keys[q];
    rows_out[r] = (uint32_t)(key & ((1ull << ybits) - 1));
    rstart[r] = (uint32_t)q;
    rsw[r] = (uint32_t)(key >> ybits);
}

// superWindowRowOffset[s] = number of unique rows of super-windows < s: the
// rows are sorted by super-window, so it is a lower bound in rsw[0, R).
__global__ void superwindow_offsets_kernel(const uint32_t* __restrict__ rsw,
                                           const uint32_t* __restrict__ d_R, uint32_t SW,
                                           uint32_t* __restrict__ swo) {
    const uint32_t s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s > SW) return;
    uint32_t lo = 0, hi = *d_R;
    while (lo < hi) {
        const uint32_t mid = lo + (hi - lo) / 2;
        if (rsw[mid] < s) lo = mid + 1; else hi = mid;
    }
    swo[s] = lo;
}

__global__ void superwindow_slots_kernel(const uint64_t* __restrict__ keys,
                                         const uint32_t* __restrict__ vals,
                                         const uint32_t* __restrict__ head,
                                         const uint32_t* __restrict__ excl,
                                         const uint32_t* __restrict__ d_ng,
                                         const uint32_t* __restrict__ d_R,
                                         const uint32_t* __restrict__ rstart,
                                         const uint32_t* __restrict__ swo, int ybits,
                                         uint32_t* __restrict__ gslot, uint32_t* __restrict__ occ) {
    const uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t ng = *d_ng;
    if (q >= ng) return;
    const uint32_t r = excl[q] + head[q] - 1;
    const uint32_t s = (uint32_t)(keys[q] >> ybits);
    gslot[vals[q]] = r - swo[s];
    if (head[q]) {
        const uint32_t R = *d_R;
        occ[r] = (r + 1 < R ? rstart[r + 1] : ng) - rstart[r];
    }
}

// Position q of the degree-sorted group list -> tile byte + row slot.
__global__ void swtcf_fill_kernel(const uint32_t* __restrict__ order,
                                  const uint32_t* __restrict__ d_ng,
                                  const uint64_t* __restrict__ gkey,
                                  const uint32_t* __restrict__ gmask,
                                  const uint32_t* __restrict__ gslot, int ybits,
                                  const uint32_t* __restrict__ wgstart,
                                  const uint32_t* __restrict__ cwo,
                                  uint64_t* __restrict__ tile_bits,
                                  uint32_t* __restrict__ tile_slot) {
    const uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= *d_ng) return;
    const uint32_t g = order[q];
    const uint32_t w = (uint32_t)(gkey[g] >> ybits);
    const uint32_t p = (uint32_t)q - wgstart[w];
    const uint64_t t = (uint64_t)cwo[w] + p / 8;
    const uint32_t lr = p & 7u;
    reinterpret_cast<uint8_t*>(tile_bits + t)[lr] = (uint8_t)gmask[g];
    tile_slot[t * 8 + lr] = gslot[g];
}

// Repeat cache of one super-window per block: rows seen in >= 2 windows,
// ranked by occurrence descending then slot ascending; ranks < 32 are cached.
__global__ void __launch_bounds__(kThreads) repeat_cache_kernel(
    const uint32_t* __restrict__ swo, const uint32_t* __restrict__ occ, uint32_t SW,
    uint8_t* __restrict__ row_cache_slot, uint32_t* __restrict__ cached_row_slot,
    uint8_t* __restrict__ cached_count, uint32_t* err) {
    constexpr int kB = TCC_SWTCF_MAX_SUPER_WINDOW + 1;
    __shared__ uint32_t hist[kB];
    __shared__ uint32_t base[kB];
    __shared__ uint32_t run[kB];
    __shared__ uint32_t wc[kThreads / 32][kB];
    const uint32_t s = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid < kB) { hist[tid] = 0; run[tid] = 0; }
    if (tid < 32) cached_row_slot[(uint64_t)s * 32 + tid] = kInvalid;
    __syncthreads();
    const uint32_t rb = swo[s], re = swo[s + 1];
    for (uint32_t r = rb + tid; r < re; r += kThreads) {
        const uint32_t o = occ[r];
        if (o > TCC_SWTCF_MAX_SUPER_WINDOW) raise_error(err, TCC_DEVERR_OCCURRENCE);
        else if (o >= 2) atomicAdd(&hist[o], 1u);
    }
    __syncthreads();
    if (tid == 0) {
        uint32_t acc = 0;
        for (int o = kB - 1; o >= 2; --o) { base[o] = acc; acc += hist[o]; }
        base[0] = base[1] = 0xFFFFFFFFu;
        cached_count[s] = (uint8_t)(acc < 32 ? acc : 32);
    }
    __syncthreads();
    for (uint32_t c = rb; c < re; c += kThreads) {
        const uint32_t r = c + tid;
        uint32_t o = r < re ? occ[r] : 0;
        if (o > TCC_SWTCF_MAX_SUPER_WINDOW) o = 0;
        // a row can still be cached while its occurrence bucket has ranks
        // below 32 left (run[] counts the bucket's rows in earlier chunks)
        const bool live = o >= 2 && base[o] + run[o] < 32;
        if (!__syncthreads_or(live)) {  // nothing left to rank in this chunk
            if (r < re) row_cache_slot[r] = 0xFF;
            continue;
        }
        const uint32_t key = live ? o : 0;
        const unsigned peers = __match_any_sync(0xffffffffu, key);
        const uint32_t lr = __popc(peers & lanemask_lt());
        if (tid < kB) {
#pragma unroll
            for (int w = 0; w < kThreads / 32; ++w) wc[w][tid] = 0;
        }
        __syncthreads();
        if (live && lr == 0) wc[warp][o] = __popc(peers);
        __syncthreads();
        if (r < re) {
            uint8_t slot = 0xFF;
            if (live) {
                uint32_t rank = base[o] + run[o] + lr;
                for (int w = 0; w < warp; ++w) rank += wc[w][o];
                if (rank < 32) {
                    slot = (uint8_t)rank;
                    cached_row_slot[(uint64_t)s * 32 + rank] = r - rb;
                }
            }
            row_cache_slot[r] = slot;
        }
        __syncthreads();
        if (tid < kB) {
            uint32_t add = 0;
#pragma unroll
            for (int w = 0; w < kThreads / 32; ++w) add += wc[w][tid];
            run[tid] += add;
        }
        __syncthreads();
    }
}

inline unsigned blocks(uint64_t n) { return (unsigned)((n + kThreads - 1) / kThreads); }
// keys_from_csr_kernel: one block per kKeyTile nonzeros
inline unsigned csr_blocks(uint64_t nnz) { return (unsigned)std::max<uint64_t>(1, (nnz + kKeyTile - 1) / kKeyTile); }

}  // namespace

// ------------------------------------------------------------- workspaces --

void Arena::reserve(size_t bytes) { total += (bytes + 255) / 256 * 256; }

void* Arena::take(size_t bytes) {
    void* p = base + used;
    used += (bytes + 255) / 256 * 256;
    if (used > total) throw Error(TCC_ERR_CAPACITY, "workspace arena overflow");
    return p;
}

static void plan_groups(Arena& a, uint64_t E) {
    for (int i = 0; i < 3; ++i) a.reserve(E * 8);
    for (int i = 0; i < 6; ++i) a.reserve(E * 4);
}

static GroupBuffers take_groups(Arena& a, uint64_t E) {
    GroupBuffers g;
    g.keys = (uint64_t*)a.take(E * 8);
    g.keys_alt = (uint64_t*)a.take(E * 8);
    g.gkey = (uint64_t*)a.take(E * 8);
    g.vals = (uint32_t*)a.take(E * 4);
    g.vals_alt = (uint32_t*)a.take(E * 4);
    g.head = (uint32_t*)a.take(E * 4);
    g.excl = (uint32_t*)a.take(E * 4);
    g.gmask = (uint32_t*)a.take(E * 4);
    g.gstart = (uint32_t*)a.take(E * 4);
    return g;
}

// Steps 2-4: sort the keys already in (keys, vals), build groups, count them
// per window and scan: wgstart[W+1] (groups before each window) and
// off[W+1] (tiles before each window; off[W] = T).  small[1] = groups.
// y_sorted: the keys arrive in nondecreasing y (keys built from a CSR with
// the window on the column side), so a stable sort of the window bits alone
// gives (window, y) order and the y digits are skipped.
static void build_windows(GroupBuffers& b, uint64_t n, int key_bits, int ybits, uint32_t W,
                          uint32_t* wcnt, uint32_t* wgstart, uint32_t* tiles, uint32_t* off,
                          uint32_t* small, void* tmp, cudaStream_t s, bool y_sorted = false) {
    if (radix_sort_pairs(b.keys, b.vals, b.keys_alt, b.vals_alt, n, key_bits, tmp, s,
                         y_sorted ? ybits : 0)) {
        std::swap(b.keys, b.keys_alt);
        std::swap(b.vals, b.vals_alt);
    }
    if (n) {
        mark_heads_kernel<<<blocks(n), kThreads, 0, s>>>(b.keys, n, b.head);
        exclusive_scan<uint32_t>(b.head, b.excl, n, small + 1, tmp, s);
        TCC_CUDA(cudaMemsetAsync(b.gmask, 0, n * 4, s));
        groups_kernel<<<blocks(n), kThreads, 0, s>>>(b.keys, b.vals, b.head, b.excl, n, b.gkey,
                                                     b.gmask, b.gstart);
    } else {
        TCC_CUDA(cudaMemsetAsync(small + 1, 0, 4, s));
    }
    if (n)
        group_check_kernel<<<blocks(n), kThreads, 0, s>>>(b.gmask, b.gstart, small + 1, n,
                                                          small + 0);
    window_start_kernel<<<blocks((uint64_t)W + 1), kThreads, 0, s>>>(b.gkey, small + 1, ybits, W,
                                                                      wgstart);
    window_tiles_kernel<<<blocks(W), kThreads, 0, s>>>(wgstart, W, wcnt, tiles);
    exclusive_scan<uint32_t>(tiles, off, W, off + W, tmp, s);
    TCC_CUDA(cudaGetLastError());
}

// ------------------------------------------------------------------ SWTCF --

SwtcfWorkspace::SwtcfWorkspace(uint64_t edge_capacity, uint32_t num_src, uint32_t S)
    : E(edge_capacity), S(S) {
    W = (num_src + 7) / 8;
    SW = (W + S - 1) / S;
    Arena a;
    plan_groups(a, E);
    for (int i = 0; i < 4; ++i) a.reserve(E * 4);  // gslot, rstart, occ, order
    for (int i = 0; i < 5; ++i) a.reserve(((uint64_t)W + 1) * 4);  // wcnt wgstart tiles + spare
    a.reserve(((uint64_t)SW + 1) * 4);
    a.reserve(64);
    tmp_bytes = std::max(radix_tmp_bytes(E), scan_tmp_bytes(std::max<uint64_t>(E, W + 1)));
    a.reserve(tmp_bytes);
    TCC_CUDA(cudaMalloc(&a.base, a.total));
    arena = a;
    g = take_groups(arena, E);
    gslot = (uint32_t*)arena.take(E * 4);
    rstart = (uint32_t*)arena.take(E * 4);
    occ = (uint32_t*)arena.take(E * 4);
    order = (uint32_t*)arena.take(E * 4);
    wcnt = (uint32_t*)arena.take(((uint64_t)W + 1) * 4);
    wgstart = (uint32_t*)arena.take(((uint64_t)W + 1) * 4);
    tiles = (uint32_t*)arena.take(((uint64_t)W + 1) * 4);
    swcnt = (uint32_t*)arena.take(((uint64_t)SW + 1) * 4);
    small = (uint32_t*)arena.take(64);
    tmp = arena.take(tmp_bytes);
    TCC_CUDA(cudaMemset(small, 0, 64));
}

SwtcfWorkspace::~SwtcfWorkspace() { cudaFree(arena.base); }

// small[0] = device error word, small[1] = groups, small[2] = R
void swtcf_convert(const uint32_t* d_dst, const uint32_t* d_src, const uint64_t* d_rowptr,
                   const uint32_t* d_col, uint64_t nnz, tcc_swtcf* m, SwtcfWorkspace& ws,
                   cudaStream_t s) {
    TCC_REQUIRE(m && m->tileLocalBit, "SWTCF matrix is not allocated");
    TCC_REQUIRE(nnz > 0 && nnz <= ws.E, "invalid COO -> SWTCF conversion arguments");
    TCC_REQUIRE(m->superWindowSize >= 1 && m->superWindowSize <= TCC_SWTCF_MAX_SUPER_WINDOW,
                "invalid super-window size");
    TCC_REQUIRE(m->numColWindows <= ws.W && m->superWindowSize == ws.S,
                "workspace was created for a different column count or super-window size");
    TCC_REQUIRE(nnz <= m->capacity_tiles && nnz <= m->capacity_rows,
                "SWTCF matrix capacity below nnz");
    const uint32_t W = m->numColWindows, SW = m->numSuperWindows, S = m->superWindowSize;
    const int ybits = std::max(1, bits_for(m->rows));
    const int wbits = std::max(1, bits_for(W));
    const int swbits = std::max(1, bits_for(SW));
    GroupBuffers b = ws.g;
    TCC_CUDA(cudaMemsetAsync(ws.small, 0, 64, s));
    TCC_REQUIRE(d_dst || m->rows > 0, "CSR conversion of a matrix without rows");
    if (d_dst) {
        keys_from_coo_kernel<<<blocks(nnz), kThreads, 0, s>>>(d_dst, d_src, nnz, m->rows, m->cols,
                                                             ybits, b.keys, b.vals, ws.small);
    } else {
        keys_from_csr_kernel<<<csr_blocks(nnz), kThreads, 0, s>>>(
            d_rowptr, d_col, m->rows, m->cols, nnz, 1, ybits, b.keys, b.vals, ws.small);
    }
    build_windows(b, nnz, wbits + ybits, ybits, W, ws.wcnt, ws.wgstart, ws.tiles,
                  m->colWindowOffset, ws.small, ws.tmp, s, /*y_sorted=*/d_dst == nullptr);

    // degree-descending, dst-ascending order inside each window
    GroupBuffers d = b;  // reuse the edge sort buffers for the group sorts
    const int dbits = wbits + 3;
    degree_keys_kernel<<<blocks(nnz), kThreads, 0, s>>>(b.gkey, b.gmask, ws.small + 1, nnz, ybits,
                                                        dbits, d.keys, d.vals);
    bool alt = radix_sort_pairs(d.keys, d.vals, d.keys_alt, d.vals_alt, nnz, dbits, ws.tmp, s);
    TCC_CUDA(cudaMemcpyAsync(ws.order, alt ? d.vals_alt : d.vals, nnz * 4,
                             cudaMemcpyDeviceToDevice, s));

    // super-window unique rows (dst ascending) and their window occurrence
    const int kbits = swbits + ybits;
    superwindow_keys_kernel<<<blocks(nnz), kThreads, 0, s>>>(b.gkey, ws.small + 1, nnz, ybits, S,
                                                             kbits, d.keys, d.vals);
    alt = radix_sort_pairs(d.keys, d.vals, d.keys_alt, d.vals_alt, nnz, kbits, ws.tmp, s);
    uint64_t* k3 = alt ? d.keys_alt : d.keys;
    uint32_t* v3 = alt ? d.vals_alt : d.vals;
    uint32_t* head3 = b.head;  // edge heads are no longer needed
    uint32_t* excl3 = b.excl;
    row_heads_kernel<<<blocks(nnz), kThreads, 0, s>>>(k3, ws.small + 1, nnz, head3);
    exclusive_scan<uint32_t>(head3, excl3, nnz, ws.small + 2, ws.tmp, s);
    // occ is free until the slots kernel: it holds each unique row's super-window
    superwindow_rows_kernel<<<blocks(nnz), kThreads, 0, s>>>(k3, head3, excl3, ws.small + 1, ybits,
                                                             m->superWindowRows, ws.rstart, ws.occ);
    superwindow_offsets_kernel<<<blocks((uint64_t)SW + 1), kThreads, 0, s>>>(
        ws.occ, ws.small + 2, SW, m->superWindowRowOffset);
    superwindow_slots_kernel<<<blocks(nnz), kThreads, 0, s>>>(
        k3, v3, head3, excl3, ws.small + 1, ws.small + 2, ws.rstart, m->superWindowRowOffset,
        ybits, ws.gslot, ws.occ);

    // tiles: bitmap bytes, row slots, padding of each window's last tile
    swtcf_fill_kernel<<<blocks(nnz), kThreads, 0, s>>>(ws.order, ws.small + 1, b.gkey, b.gmask,
                                                       ws.gslot, ybits, ws.wgstart,
                                                       m->colWindowOffset, m->tileLocalBit,
                                                       m->tileRowSlot);
    tile_padding_kernel<<<blocks(W), kThreads, 0, s>>>(ws.wcnt, m->colWindowOffset, W,
                                                       m->tileRowSlot, m->tileLocalBit, 1);
    repeat_cache_kernel<<<SW, kThreads, 0, s>>>(m->superWindowRowOffset, ws.occ, SW,
                                                m->superWindowRowCacheSlot,
                                                m->superWindowCachedRowSlot,
                                                m->superWindowCachedCount, ws.small);
    TCC_CUDA(cudaGetLastError());
}

// -------------------------------------------------------------- BCSR/BCSC --

TilesWorkspace::TilesWorkspace(uint64_t nnz_capacity, uint32_t rows, uint32_t cols)
    : E(nnz_capacity), rows(rows), cols(cols) {
    const uint64_t Wmax = (std::max(rows, cols) + 7ull) / 8;
    Arena a;
    plan_groups(a, std::max<uint64_t>(E, 1));
    for (int i = 0; i < 4; ++i) a.reserve((Wmax + 1) * 4);
    a.reserve(64);
    tmp_bytes = std::max(radix_tmp_bytes(E), scan_tmp_bytes(std::max<uint64_t>(E, Wmax)));
    a.reserve(tmp_bytes);
    TCC_CUDA(cudaMalloc(&a.base, a.total));
    arena = a;
    g = take_groups(arena, std::max<uint64_t>(E, 1));
    wcnt = (uint32_t*)arena.take((Wmax + 1) * 4);
    wgstart = (uint32_t*)arena.take((Wmax + 1) * 4);
    tiles = (uint32_t*)arena.take((Wmax + 1) * 4);
    off = (uint32_t*)arena.take((Wmax + 1) * 4);
    small = (uint32_t*)arena.take(64);
    tmp = arena.take(tmp_bytes);
    TCC_CUDA(cudaMemset(small, 0, 64));
}

TilesWorkspace::~TilesWorkspace() { cudaFree(arena.base); }

static uint64_t finish_prepare(TilesWorkspace& ws, cudaStream_t s);

uint64_t tiles_prepare(TilesWorkspace& ws, int kind, const uint64_t* d_rowptr,
                       const uint32_t* d_col, uint32_t rows, uint32_t cols, uint64_t nnz,
                       cudaStream_t s) {
    TCC_REQUIRE(kind == TCC_TILES_BCSR || kind == TCC_TILES_BCSC, "unknown tile layout");
    TCC_REQUIRE(rows > 0 && cols > 0, "empty matrix shape");
    TCC_REQUIRE(nnz <= ws.E && rows <= ws.rows && cols <= ws.cols,
                "tiles workspace smaller than the matrix");
    ws.kind = kind;
    ws.cur_rows = rows;
    ws.cur_cols = cols;
    ws.nnz = nnz;
    ws.W = kind == TCC_TILES_BCSR ? (rows + 7) / 8 : (cols + 7) / 8;
    ws.ybits = std::max(1, bits_for(kind == TCC_TILES_BCSR ? cols : rows));
    const int wbits = std::max(1, bits_for(ws.W));
    TCC_CUDA(cudaMemsetAsync(ws.small, 0, 64, s));
    if (nnz)
        keys_from_csr_kernel<<<csr_blocks(nnz), kThreads, 0, s>>>(
            d_rowptr, d_col, rows, cols, nnz, kind == TCC_TILES_BCSR ? 0 : 1, ws.ybits, ws.g.keys,
            ws.g.vals, ws.small);
    build_windows(ws.g, nnz, wbits + ws.ybits, ws.ybits, ws.W, ws.wcnt, ws.wgstart, ws.tiles,
                  ws.off, ws.small, ws.tmp, s, /*y_sorted=*/kind == TCC_TILES_BCSC);
    return finish_prepare(ws, s);
}

// Reads back the error word, group and tile counts after build_windows.
static uint64_t finish_prepare(TilesWorkspace& ws, cudaStream_t s) {
    uint32_t host[2] = {0, 0};
    TCC_CUDA(cudaMemcpyAsync(host, ws.small, 8, cudaMemcpyDeviceToHost, s));
    uint32_t T = 0;
    TCC_CUDA(cudaMemcpyAsync(&T, ws.off + ws.W, 4, cudaMemcpyDeviceToHost, s));
    TCC_CUDA(cudaStreamSynchronize(s));
    if (host[0] != 0)
        throw Error(TCC_ERR_DEVICE, "tile conversion raised device error " +
                                        std::to_string(host[0]) +
                                        (host[0] == TCC_DEVERR_GROUP_DEGREE ? " (duplicate edge)"
                                                                            : " (index range)"));
    ws.ng = host[1];
    ws.T = T;
    ws.prepared = true;
    return T;
}

uint64_t tiles_prepare_swtcf(TilesWorkspace& ws, const tcc_swtcf* m, cudaStream_t s) {
    TCC_REQUIRE(m->rows > 0 && m->cols > 0, "empty matrix shape");
    TCC_REQUIRE(m->rows <= ws.rows && m->cols <= ws.cols, "tiles workspace smaller than the matrix");
    uint32_t Tsw = 0;
    TCC_CUDA(cudaMemcpyAsync(&Tsw, m->colWindowOffset + m->numColWindows, 4, cudaMemcpyDeviceToHost, s));
    TCC_CUDA(cudaStreamSynchronize(s));
    TCC_REQUIRE(Tsw <= ws.E, "tiles workspace smaller than the matrix");
    ws.kind = TCC_TILES_BCSR;
    ws.cur_rows = m->rows;
    ws.cur_cols = m->cols;
    ws.W = (m->rows + 7) / 8;
    ws.ybits = std::max(1, bits_for(m->cols));
    const int wbits = std::max(1, bits_for(ws.W));
    TCC_CUDA(cudaMemsetAsync(ws.small, 0, 64, s));
    uint32_t nnz = 0;
    if (Tsw) {
        // tile popcounts -> write positions (the group buffers' head/excl are
        // free until build_windows); total at small[8]
        popcount_kernel<<<blocks(Tsw), kThreads, 0, s>>>(m->tileLocalBit, Tsw, ws.g.head);
        exclusive_scan<uint32_t>(ws.g.head, ws.g.excl, Tsw, ws.small + 8, ws.tmp, s);
        TCC_CUDA(cudaMemcpyAsync(&nnz, ws.small + 8, 4, cudaMemcpyDeviceToHost, s));
        TCC_CUDA(cudaStreamSynchronize(s));
        TCC_REQUIRE(nnz <= ws.E, "tiles workspace smaller than the matrix");
        keys_from_swtcf_kernel<<<blocks(Tsw), kThreads, 0, s>>>(
            m->colWindowOffset, m->numColWindows, m->superWindowSize, m->superWindowRowOffset,
            m->superWindowRows, m->tileRowSlot, m->tileLocalBit, ws.g.excl, Tsw, m->rows, m->cols,
            ws.ybits, ws.g.keys, ws.g.vals, ws.small);
    }
    ws.nnz = nnz;
    build_windows(ws.g, nnz, wbits + ws.ybits, ws.ybits, ws.W, ws.wcnt, ws.wgstart, ws.tiles,
                  ws.off, ws.small, ws.tmp, s);
    return finish_prepare(ws, s);
}

void tiles_fill(TilesWorkspace& ws, int kind, uint32_t* win_offset, uint32_t* tc_offset,
                uint32_t* idx, uint64_t* bits, cudaStream_t s) {
    TCC_REQUIRE(ws.prepared && ws.kind == kind, "tiles workspace was not prepared for this layout");
    const uint64_t T = ws.T;
    TCC_CUDA(cudaMemcpyAsync(win_offset, ws.off, ((uint64_t)ws.W + 1) * 4,
                             cudaMemcpyDeviceToDevice, s));
    if (T) {
        if (kind == TCC_TILES_BCSR) TCC_CUDA(cudaMemsetAsync(bits, 0, T * 8, s));
        fill_tiles_kernel<<<blocks(ws.ng), kThreads, 0, s>>>(ws.g.gkey, ws.g.gmask, ws.ng,
                                                             ws.ybits, ws.wgstart, ws.off,
                                                             kind == TCC_TILES_BCSR, idx, bits);
        tile_padding_kernel<<<blocks(ws.W), kThreads, 0, s>>>(ws.wcnt, ws.off, ws.W, idx, bits,
                                                              kind == TCC_TILES_BCSC);
        popcount_kernel<<<blocks(T), kThreads, 0, s>>>(bits, T, tc_offset);
    }
    exclusive_scan<uint32_t>(tc_offset, tc_offset, T, tc_offset + T, ws.tmp, s);
    TCC_CUDA(cudaGetLastError());
}

}  // namespace tcc
