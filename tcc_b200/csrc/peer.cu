// peer.cu -- the row-partitioned SpMM's halo exchange over NVLink peer memory.
//
// One process per GPU of one box.  Every rank owns, in its own HBM, one or
// more receive buffers per exchange tag (the halo rows it reads, grouped by owner)
// and one flag block; the peers map both through CUDA IPC.  One exchange of
// tag t, step number s (the same count on every rank):
//
//   sender g (halo_push_kernel, on a side stream):
//     1. waits until each receiver p it sends to has released step s-B of
//        tag t (flags_g.freed[t][p] >= s-B, B the receive buffers a receiver
//        rotates through, step s in buffer (s-1) % B), so the receive rows it
//        is about to overwrite are no longer read;
//     2. gathers its rows X[send_idx[i]] and stores them straight into the
//        receivers' buffers over NVLink (a warp moves 4 rows at a time in
//        16-byte lanes, loads before stores): the
//        pack and the transfer are one pass, no staging copy and no
//        collective kernel;
//     3. the last CTA to finish (a grid-wide counter) fences at system scope
//        and sets flags_p.arrived[t][g] = s at every receiver p (release).
//   receiver p (halo_wait_kernel, on the stream of the halo tiles):
//     waits until flags_p.arrived[t][g] >= s for every sender g (acquire); the
//     halo tiles launched after it read the rows.  After them,
//     halo_release_kernel sets flags_g.freed[t][p] = s at every sender g.
//
// Every wait is bounded (the caller's limit, via %globaltimer): on expiry the
// kernel records TCC_DEVERR_WAIT_TIMEOUT in the rank's flag block and returns
// without writing rows (push) or lets the stream continue (wait), so a missing
// peer turns into an error the host reads (tcc_peer_device_error), never into
// a hung GPU.  No multicast object and no multicast load is involved: plain
// peer stores and flag loads/stores only.
//
// Flag block (TCC_PEER_FLAGS_BYTES, zeroed at allocation), uint32 words:
//   [  0, 32)  arrived[tag][sender]   written by the senders
//   [ 64, 96)  freed[tag][receiver]   written by the receivers
//   [128,132)  done counter per tag    this rank's push kernel only
//   [136]      device error word       this rank only
#include "common.cuh"

#include <algorithm>

namespace tcc {

constexpr uint32_t kPeerMaxRanks = TCC_PEER_MAX_RANKS;
constexpr uint32_t kPeerMaxTags = TCC_PEER_MAX_TAGS;
constexpr uint32_t kArrivedWord = 0;
constexpr uint32_t kFreedWord = 64;
constexpr uint32_t kDoneWord = 128;
constexpr uint32_t kErrorWord = 136;

namespace {

__device__ __forceinline__ unsigned long long peer_clock() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// seq-space comparison (wraps after 2^31 steps)
__device__ __forceinline__ bool reached(uint32_t v, uint32_t want) { return (int32_t)(v - want) >= 0; }

// Wait until *p reaches `want`; false once limit_ns have passed.
__device__ bool wait_flag(const uint32_t* p, uint32_t want, unsigned long long limit_ns) {
    if (reached(ld_acquire_sys(p), want)) return true;
    const unsigned long long t0 = peer_clock();
    for (;;) {
        __nanosleep(200);
        if (reached(ld_acquire_sys(p), want)) return true;
        if (peer_clock() - t0 >= limit_ns) return false;
    }
}

__device__ __forceinline__ void record_timeout(uint32_t* flags) {
    atomicCAS(flags + kErrorWord, 0u, (uint32_t)TCC_DEVERR_WAIT_TIMEOUT);
}

struct PushParams {
    const float* x;
    uint64_t ldx, num_rows;
    const int64_t* send_idx;
    uint32_t q4, world, rank, tag, seq, reuse;  // reuse: the step that last used the buffer
    uint64_t seg[kPeerMaxRanks + 1];
    float* dst[kPeerMaxRanks];
    uint64_t ld_dst;
    uint32_t* peer_flags[kPeerMaxRanks];
    uint32_t* flags;
    unsigned long long wait_ns;
};

constexpr int kPushThreads = 512;
constexpr int kPushRows = 4;  // rows a warp has in flight (loads before stores)

// The segment (receiving rank) of send row i.
__device__ __forceinline__ uint32_t segment_of(const PushParams& a, uint64_t i) {
    uint32_t p = 0;
    while (i >= a.seg[p + 1]) ++p;
    return p;
}

__global__ void __launch_bounds__(kPushThreads) halo_push_kernel(const __grid_constant__ PushParams a) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
        int good = 1;
        if (a.reuse > 0) {
            for (uint32_t p = 0; p < a.world; ++p) {
                if (a.seg[p + 1] == a.seg[p]) continue;
                if (!wait_flag(a.flags + kFreedWord + a.tag * kPeerMaxRanks + p, a.reuse,
                               a.wait_ns)) {
                    record_timeout(a.flags);
                    good = 0;
                    break;
                }
            }
        }
        ok = good;
    }
    __syncthreads();
    if (ok) {
        // a warp moves kPushRows rows at a time: all their loads are issued
        // before the first store, so each warp keeps kPushRows x 512 B of
        // NVLink stores in flight (the stores are posted; nothing waits on them)
        const uint64_t n = a.seg[a.world];
        const int lane = threadIdx.x & 31;
        const uint64_t warps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
        const uint64_t gw = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
        for (uint64_t base = gw * kPushRows; base < n; base += warps * kPushRows) {
            const float4* src[kPushRows];
            float4* dst[kPushRows];
#pragma unroll
            for (int u = 0; u < kPushRows; ++u) {
                src[u] = nullptr;
                dst[u] = nullptr;
                const uint64_t i = base + u;
                if (i >= n) continue;
                const uint32_t p = segment_of(a, i);
                dst[u] = reinterpret_cast<float4*>(a.dst[p] + (i - a.seg[p]) * a.ld_dst);
                const int64_t r = a.send_idx[i];
                if (r >= 0 && (uint64_t)r < a.num_rows)
                    src[u] = reinterpret_cast<const float4*>(a.x + (uint64_t)r * a.ldx);
                else if (lane == 0)  // a bad index: zero row, error recorded
                    atomicCAS(a.flags + kErrorWord, 0u, (uint32_t)TCC_DEVERR_INDEX_RANGE);
            }
            for (uint32_t c = lane; c < a.q4; c += 32) {
                float4 v[kPushRows];
#pragma unroll
                for (int u = 0; u < kPushRows; ++u)
                    v[u] = src[u] ? __ldg(src[u] + c) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int u = 0; u < kPushRows; ++u)
                    if (dst[u]) dst[u][c] = v[u];
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();  // this CTA's peer stores before the counter
        const uint32_t prev = atomicInc(a.flags + kDoneWord + a.tag, gridDim.x - 1);
        if (prev == gridDim.x - 1) {  // the last CTA (the counter wrapped to 0)
            __threadfence_system();
            // a push that gave up signals nothing: its receivers time out too
            if (*(volatile uint32_t*)(a.flags + kErrorWord) == 0) {
                for (uint32_t p = 0; p < a.world; ++p)
                    if (a.seg[p + 1] > a.seg[p])
                        st_release_sys(a.peer_flags[p] + kArrivedWord + a.tag * kPeerMaxRanks + a.rank,
                                       a.seq);
            }
        }
    }
}

__global__ void halo_wait_kernel(uint32_t* flags, uint32_t tag, uint32_t seq, uint32_t mask,
                                 unsigned long long wait_ns) {
    const uint32_t p = threadIdx.x;
    if (p < kPeerMaxRanks && (mask >> p & 1u)) {
        if (!wait_flag(flags + kArrivedWord + tag * kPeerMaxRanks + p, seq, wait_ns))
            record_timeout(flags);
    }
}

struct ReleaseParams {
    uint32_t* peer_flags[kPeerMaxRanks];
};

__global__ void halo_release_kernel(const __grid_constant__ ReleaseParams a, uint32_t rank,
                                    uint32_t tag, uint32_t seq, uint32_t mask) {
    const uint32_t p = threadIdx.x;
    if (p < kPeerMaxRanks && (mask >> p & 1u)) {
        __threadfence_system();
        st_release_sys(a.peer_flags[p] + kFreedWord + tag * kPeerMaxRanks + rank, seq);
    }
}

}  // namespace

void peer_alloc(size_t bytes, void** ptr, void* handle) {
    TCC_REQUIRE(ptr && handle, "ptr and handle must not be NULL");
    TCC_REQUIRE(bytes > 0, "bytes must be positive");
    *ptr = nullptr;
    TCC_CUDA(cudaMalloc(ptr, bytes));
    cudaError_t e = cudaMemset(*ptr, 0, bytes);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), *ptr);
    if (e != cudaSuccess) {
        cudaFree(*ptr);
        *ptr = nullptr;
        TCC_CUDA(e);
    }
}

void peer_open(const void* handle, void** ptr) {
    TCC_REQUIRE(ptr && handle, "ptr and handle must not be NULL");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    *ptr = nullptr;
    TCC_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

void peer_close(void* mapped) {
    if (mapped) TCC_CUDA(cudaIpcCloseMemHandle(mapped));
}

void peer_free(void* ptr) {
    if (ptr) TCC_CUDA(cudaFree(ptr));
}

void halo_push(const tcc_halo_push_args* a, cudaStream_t s) {
    TCC_REQUIRE(a, "args must not be NULL");
    TCC_REQUIRE(a->world >= 1 && a->world <= kPeerMaxRanks && a->rank < a->world,
                "world must be in [1, TCC_PEER_MAX_RANKS] and rank < world");
    TCC_REQUIRE(a->tag < kPeerMaxTags, "tag must be < TCC_PEER_MAX_TAGS");
    TCC_REQUIRE(a->seq > 0, "step numbers start at 1");
    TCC_REQUIRE(a->width > 0 && a->width % 4 == 0, "width must be a positive multiple of 4");
    TCC_REQUIRE(a->ldx % 4 == 0 && a->ldx >= a->width && a->ld_dst % 4 == 0 && a->ld_dst >= a->width,
                "row strides must be multiples of 4 and >= width");
    TCC_REQUIRE(a->flags, "flags must not be NULL");
    TCC_REQUIRE(a->seg[0] == 0, "seg[0] must be 0");
    PushParams p{};
    for (uint32_t r = 0; r < a->world; ++r) {
        TCC_REQUIRE(a->seg[r + 1] >= a->seg[r], "seg must be non-decreasing");
        if (a->seg[r + 1] > a->seg[r]) {
            TCC_REQUIRE(r != a->rank, "a rank sends no rows to itself");
            TCC_REQUIRE(a->dst[r] && a->peer_flags[r], "a receiver's buffer and flags must be mapped");
            TCC_REQUIRE((uintptr_t)a->dst[r] % 16 == 0, "receive rows must be 16-byte aligned");
        }
        p.seg[r] = a->seg[r];
        p.dst[r] = a->dst[r];
        p.peer_flags[r] = static_cast<uint32_t*>(a->peer_flags[r]);
    }
    p.seg[a->world] = a->seg[a->world];
    const uint64_t n = a->seg[a->world];
    TCC_REQUIRE(n == 0 || (a->x && a->send_idx), "x and send_idx must not be NULL");
    TCC_REQUIRE(n == 0 || (uintptr_t)a->x % 16 == 0, "x must be 16-byte aligned");
    for (uint32_t r = a->world; r < kPeerMaxRanks; ++r) p.seg[r + 1] = p.seg[a->world];
    p.x = a->x;
    p.ldx = a->ldx;
    p.num_rows = a->num_rows;
    p.send_idx = a->send_idx;
    p.q4 = a->width / 4;
    p.world = a->world;
    p.rank = a->rank;
    p.tag = a->tag;
    p.seq = a->seq;
    const uint32_t buffers = a->buffers ? a->buffers : 1;
    p.reuse = a->seq > buffers ? a->seq - buffers : 0;
    p.ld_dst = a->ld_dst;
    p.flags = static_cast<uint32_t*>(a->flags);
    p.wait_ns = a->wait_ns;
    const uint64_t rows_per_block = (kPushThreads / 32) * kPushRows;
    const uint64_t want = std::max<uint64_t>(1, (n + rows_per_block - 1) / rows_per_block);
    const uint64_t cap = a->max_blocks ? a->max_blocks : (uint64_t)sm_count() * 4;
    const unsigned blocks = (unsigned)std::min<uint64_t>(want, cap);
    halo_push_kernel<<<blocks, kPushThreads, 0, s>>>(p);
    TCC_CUDA(cudaGetLastError());
}

void halo_wait(void* flags, uint32_t tag, uint32_t seq, uint32_t mask, unsigned long long wait_ns,
               cudaStream_t s) {
    TCC_REQUIRE(flags, "flags must not be NULL");
    TCC_REQUIRE(tag < kPeerMaxTags, "tag must be < TCC_PEER_MAX_TAGS");
    TCC_REQUIRE(mask < (1u << kPeerMaxRanks), "peer mask has bits above TCC_PEER_MAX_RANKS");
    if (!mask) return;
    halo_wait_kernel<<<1, 32, 0, s>>>(static_cast<uint32_t*>(flags), tag, seq, mask, wait_ns);
    TCC_CUDA(cudaGetLastError());
}

void halo_release(void* const* peer_flags, uint32_t world, uint32_t rank, uint32_t tag,
                  uint32_t seq, uint32_t mask, cudaStream_t s) {
    TCC_REQUIRE(peer_flags, "peer_flags must not be NULL");
    TCC_REQUIRE(world >= 1 && world <= kPeerMaxRanks && rank < world, "bad world/rank");
    TCC_REQUIRE(tag < kPeerMaxTags, "tag must be < TCC_PEER_MAX_TAGS");
    TCC_REQUIRE(mask < (1u << world), "peer mask has bits above world");
    if (!mask) return;
    ReleaseParams p{};
    for (uint32_t r = 0; r < world; ++r) {
        if (mask >> r & 1u) TCC_REQUIRE(peer_flags[r] && r != rank, "a released sender must be mapped");
        p.peer_flags[r] = static_cast<uint32_t*>(peer_flags[r]);
    }
    halo_release_kernel<<<1, 32, 0, s>>>(p, rank, tag, seq, mask);
    TCC_CUDA(cudaGetLastError());
}

void peer_device_error(void* flags, int* code, cudaStream_t s) {
    TCC_REQUIRE(flags && code, "flags and code must not be NULL");
    uint32_t v = 0;
    TCC_CUDA(cudaMemcpyAsync(&v, static_cast<uint32_t*>(flags) + kErrorWord, sizeof(v),
                             cudaMemcpyDeviceToHost, s));
    TCC_CUDA(cudaStreamSynchronize(s));
    *code = (int)v;
}

}  // namespace tcc
