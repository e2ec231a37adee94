// spmm.cuh -- SpMM over 8x8 window tiles (internal interface used by capi.cu).
#pragma once

#include "common.cuh"

namespace tcc {

// Tile source of a pull pass (owner-computes: window w owns outputs 8w..8w+7).
struct PullTiles {
    uint32_t num_windows;
    uint32_t num_tiles;
    const uint32_t* win_offset;  // [num_windows+1]
    const uint64_t* bits;        // [num_tiles]
    const uint32_t* idx;         // [8*num_tiles]: gather index, or SWTCF row slot
    bool bits_transposed;        // false: bit = out*8 + gather (BCSR); true: gather*8 + out
    // SWTCF transposed pass: gather row = sw_rows[sw_offset[w / S] + slot]
    const uint32_t* sw_offset = nullptr;
    const uint32_t* sw_rows = nullptr;
    uint32_t S = 0;
    uint32_t num_out;   // output rows (guards the last window)
    uint32_t num_in;    // gather rows (indices >= num_in are padding)
    // per tile, bit k: gathered row k is among the most used rows of the
    // tiling (built with the work plan; NULL = unknown).  The bulk-copy pull
    // kernel gives the copies of those rows an L2 evict-last priority and the
    // others evict-first, so that the rows most tiles share stay in L2.
    const uint8_t* hot = nullptr;
};

// Dense operands.  cs scales gathered rows, rs scales output rows (NULL = 1).
struct Dense {
    const float* X;
    uint64_t ldx;
    float* Y;
    uint64_t ldy;
    uint32_t F;
    const float* rs;
    const float* cs;
    // int8 input rows instead of X (push pass only; launchSWTCFSpMMQuantized):
    // input row c = float(qX[g * ldq + f]) * qscale[g], g = qmap[c] (qmap NULL:
    // g = c)
    const int8_t* qX = nullptr;
    uint64_t ldq = 0;
    const float* qscale = nullptr;
    const uint32_t* qmap = nullptr;
};

// Hot/cold feature store of the mixed first-layer pass.
struct FeatureStore {
    const int32_t* id_map = nullptr;
    const float* cpu_features = nullptr;
    const int32_t* cache_search_map = nullptr;
    const float* const* gpu_features = nullptr;
    int64_t gpu_capacity = 0;
};

size_t pull_scratch_bytes(uint32_t num_windows, uint32_t num_tiles);
// TCC_PULL_L2=hot is set: hot-row L2 hints in the bulk-copy pull kernel.
bool l2_hints_requested();
int l2_hint_mode();  // 0 none, 1 hot evict-last + cold evict-first, 2 hubs evict-last only
// Builds the pull work plan in `scratch` on stream s (what plan_ready = 1 reuses).
void pull_plan(const PullTiles& a, void* scratch, size_t scratch_bytes, cudaStream_t s);
// keep_plan = false: the caller never passes plan_ready = 1 for this scratch
// again, so the plan is built only when the dispatched kernel reads it.
void pull_spmm(const PullTiles& a, const Dense& d, uint32_t tc_threshold, int accumulate,
               void* scratch, size_t scratch_bytes, bool plan_ready, const FeatureStore* fs,
               cudaStream_t s, bool keep_plan = true);

// Bulk-copy gather pull kernel (pull_tma.cu): BCSR forward / BCSC transposed over
// a dense X; F a multiple of 4 and either <= 128 or a multiple of 128.
bool pull_tma_eligible(const PullTiles& a, const Dense& d);
void pull_tma(const PullTiles& a, const Dense& d, uint32_t thr, int accumulate, uint32_t* err,
              cudaStream_t s);
// tcgen05 pull kernel (pull_umma.cu): tc_threshold == 0 (every tile on the
// TF32 tensor cores), F a multiple of 128, dense X.
bool pull_umma_eligible(const PullTiles& a, const Dense& d, uint32_t tc_threshold);
void pull_umma(const PullTiles& a, const Dense& d, int accumulate, uint32_t* err, cudaStream_t s);
// rows.cu: out[idx[i]] += in[i] (the transposed pass's returned halo rows).
void scatter_add_rows(const float* in, uint64_t ldi, const int64_t* idx, uint64_t n, float* out,
                      uint64_t ldo, uint64_t num_rows, uint32_t F, uint32_t* bad, cudaStream_t s);
// rows.cu: out[i] = X[idx[i]] (halo pack of the row-partitioned SpMM).
// peer.cu: the halo exchange over NVLink peer memory
void peer_alloc(size_t bytes, void** ptr, void* handle);
void peer_open(const void* handle, void** ptr);
void peer_close(void* mapped);
void peer_free(void* ptr);
void halo_push(const tcc_halo_push_args* a, cudaStream_t s);
void halo_wait(void* flags, uint32_t tag, uint32_t seq, uint32_t mask, unsigned long long wait_ns,
               cudaStream_t s);
void halo_release(void* const* peer_flags, uint32_t world, uint32_t rank, uint32_t tag,
                  uint32_t seq, uint32_t mask, cudaStream_t s);
void peer_device_error(void* flags, int* code, cudaStream_t s);
void gather_rows(const float* X, uint64_t ldx, uint64_t num_rows, const int64_t* idx, uint64_t n,
                 float* out, uint64_t ldo, uint32_t F, uint32_t* bad, cudaStream_t s);
// gcn_ops.cu: fused ReLU + dropout of a GCN hidden layer and its backward.
uint32_t dropout_threshold(float p);
void relu_dropout_forward(const float* in, float* out, uint64_t n, float p, uint64_t seed,
                          cudaStream_t s);
void relu_dropout_backward(const float* grad_out, const float* out, float* grad_in, uint64_t n,
                           float p, cudaStream_t s);
// Offset of the device error word inside a pull scratch.
constexpr size_t kPullErrorOffset = 8;

// Tile source of a push pass (window w owns inputs 8w..8w+7 and scatters).
struct PushTiles {
    uint32_t num_windows;
    const uint32_t* win_offset;
    const uint64_t* bits;       // bit = outslot*8 + local input (transposed: input*8 + outslot)
    const uint32_t* idx;        // BCSC: output row; SWTCF: super-window row slot
    bool bits_transposed = false;
    // SWTCF: output row = sw_rows[sw_offset[s] + slot]; repeat cache per super-window
    const uint32_t* sw_offset = nullptr;
    const uint32_t* sw_rows = nullptr;
    const uint8_t* sw_cache_slot = nullptr;
    const uint32_t* sw_cached_row_slot = nullptr;
    const uint8_t* sw_cached_count = nullptr;
    uint32_t S = 0;
    uint32_t num_out;
    uint32_t num_in;
};

// Y += diag(rs) * A * diag(cs) * X over column windows (vector fp32 reductions).
void push_spmm(const PushTiles& a, const Dense& d, uint32_t tc_threshold, const FeatureStore* fs,
               cudaStream_t s);

}  // namespace tcc
