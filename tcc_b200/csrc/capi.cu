// capi.cu -- the extern "C" boundary (include/tcc_b200.h) over the sm_100a
// kernels.  Exceptions never cross it: every entry point returns a tcc_status
// and records a message for tcc_last_error().
#include "convert.cuh"
#include "spmm.cuh"

#include <nvtx3/nvToolsExt.h>

#include <mutex>
#include <string>

struct tcc_swtcf_workspace {
    tcc::SwtcfWorkspace impl;
    tcc_swtcf_workspace(uint64_t e, uint32_t n, uint32_t s) : impl(e, n, s) {}
};
struct tcc_tiles_workspace {
    tcc::TilesWorkspace impl;
    tcc_tiles_workspace(uint64_t e, uint32_t r, uint32_t c) : impl(e, r, c) {}
};

namespace {
thread_local std::string g_last_error;

// Every C-ABI call runs inside an NVTX range named after it (visible in
// Nsight timelines; a no-op when no tool is attached).
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
};

template <typename Fn>
tcc_status guarded(const char* where, Fn&& fn) {
    NvtxRange range(where);
    try {
        fn();
        return TCC_OK;
    } catch (const tcc::Error& e) {
        g_last_error = std::string(where) + ": " + e.what();
        return e.status;
    } catch (const std::bad_alloc&) {
        g_last_error = std::string(where) + ": host out of memory";
        return TCC_ERR_OUT_OF_MEMORY;
    } catch (const std::exception& e) {
        g_last_error = std::string(where) + ": " + e.what();
        return TCC_ERR_INVALID_ARGUMENT;
    }
}

template <typename T>
void dev_alloc(T** p, uint64_t n) {
    *p = nullptr;
    TCC_CUDA(cudaMalloc(reinterpret_cast<void**>(p), std::max<uint64_t>(n, 1) * sizeof(T)));
}

void zero_rows(float* Y, uint64_t ldy, uint32_t F, uint64_t rows, cudaStream_t s) {
    if (!rows) return;
    if (ldy == F) TCC_CUDA(cudaMemsetAsync(Y, 0, rows * F * sizeof(float), s));
    else TCC_CUDA(cudaMemset2DAsync(Y, ldy * sizeof(float), 0, F * sizeof(float), rows, s));
}

tcc::PullTiles bcsr_pull(const tcc_bcsr* a) {
    tcc::PullTiles t{};
    t.num_windows = a->num_rowWindows;
    t.num_tiles = a->num_TCBlocks;
    t.win_offset = a->rowWindowOffset;
    t.bits = a->tcLocalBit;
    t.idx = a->sparseA2B;
    t.bits_transposed = false;
    t.num_out = a->num_rows;
    t.num_in = a->num_cols;
    return t;
}

tcc::PullTiles bcsc_pull_t(const tcc_bcsc* a) {
    tcc::PullTiles t{};
    t.num_windows = a->num_colWindows;
    t.num_tiles = a->num_TCBlocks;
    t.win_offset = a->colWindowOffset;
    t.bits = a->tcLocalBit;
    t.idx = a->sparseA2C;
    t.bits_transposed = true;
    t.num_out = a->num_cols;
    t.num_in = a->num_rows;
    return t;
}

tcc::PushTiles bcsc_push(const tcc_bcsc* a) {
    tcc::PushTiles t{};
    t.num_windows = a->num_colWindows;
    t.win_offset = a->colWindowOffset;
    t.bits = a->tcLocalBit;
    t.idx = a->sparseA2C;
    t.num_out = a->num_rows;
    t.num_in = a->num_cols;
    return t;
}

// Scratch of tcc_bcsr_spmm_noalloc: a fixed device array in this library's
// image (every GPU that loads the library holds it until exit), so the entry
// point never allocates.  Host code reaches it only through the address that
// cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[TCC_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device, looked up once
// per device (the first call on a device does this set-up).
void* noalloc_scratch() {
    int dev = 0;
    TCC_CUDA(cudaGetDevice(&dev));
    TCC_REQUIRE(dev >= 0 && dev < kMaxDevices, "device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        TCC_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        g_noalloc_ptr[dev] = p;
    }
    return g_noalloc_ptr[dev];
}

// Transposed pass over BCSR tiles as a push: window w scatters rows 8w..8w+7
// of G into rows sparseA2B[.] of Z (bit = inrow*8 + k, transposed on load).
tcc::PushTiles bcsr_push_t(const tcc_bcsr* a) {
    tcc::PushTiles t{};
    t.num_windows = a->num_rowWindows;
    t.win_offset = a->rowWindowOffset;
    t.bits = a->tcLocalBit;
    t.idx = a->sparseA2B;
    t.bits_transposed = true;
    t.num_out = a->num_cols;
    t.num_in = a->num_rows;
    return t;
}

void check_bcsr(const tcc_bcsr* a) {
    TCC_REQUIRE(a && a->rowWindowOffset && a->tcLocalBit && a->sparseA2B, "BCSR arrays missing");
    TCC_REQUIRE(a->num_rowWindows == (a->num_rows + 7) / 8, "num_rowWindows != ceil(num_rows/8)");
}
// The SWTCF tiles as the operand of the transposed pull (column windows own
// their outputs; gather rows through the super-window row slots).
tcc::PullTiles swtcf_t_pull(const tcc_swtcf* m) {
    tcc::PullTiles t{};
    t.num_windows = m->numColWindows;
    t.num_tiles = (uint32_t)m->capacity_tiles;
    t.win_offset = m->colWindowOffset;
    t.bits = m->tileLocalBit;
    t.idx = m->tileRowSlot;
    t.bits_transposed = true;
    t.sw_offset = m->superWindowRowOffset;
    t.sw_rows = m->superWindowRows;
    t.S = m->superWindowSize;
    t.num_out = m->cols;
    t.num_in = m->rows;
    return t;
}

void check_bcsc(const tcc_bcsc* a) {
    TCC_REQUIRE(a && a->colWindowOffset && a->tcLocalBit && a->sparseA2C, "BCSC arrays missing");
    TCC_REQUIRE(a->num_colWindows == (a->num_cols + 7) / 8, "num_colWindows != ceil(num_cols/8)");
}
}  // namespace

extern "C" {

const char* tcc_last_error(void) { return g_last_error.c_str(); }
const char* tcc_version(void) { return "tcc_b200 0.1 (sm_100a)"; }

// ------------------------------------------------------------------- SWTCF --

tcc_status tcc_swtcf_alloc(tcc_swtcf* m, uint32_t rows, uint32_t cols, uint32_t nnz,
                           uint32_t S) {
    return guarded("tcc_swtcf_alloc", [&] {
        TCC_REQUIRE(m, "null matrix");
        TCC_REQUIRE(cols > 0 && nnz > 0 && S > 0 && S <= TCC_SWTCF_MAX_SUPER_WINDOW,
                    "invalid SWTCF allocation size");
        *m = tcc_swtcf{};
        m->rows = rows;
        m->cols = cols;
        m->nnz = nnz;
        m->colWindowWidth = 8;
        m->tileRows = 8;
        m->superWindowSize = S;
        m->numColWindows = (cols + 7) / 8;
        m->numSuperWindows = (m->numColWindows + S - 1) / S;
        m->capacity_tiles = nnz;
        m->capacity_rows = nnz;
        try {
            dev_alloc(&m->superWindowRowOffset, (uint64_t)m->numSuperWindows + 1);
            dev_alloc(&m->superWindowRows, nnz);
            dev_alloc(&m->superWindowRowCacheSlot, nnz);
            dev_alloc(&m->superWindowCachedRowSlot, (uint64_t)m->numSuperWindows * 32);
            dev_alloc(&m->superWindowCachedCount, m->numSuperWindows);
            dev_alloc(&m->colWindowOffset, (uint64_t)m->numColWindows + 1);
            dev_alloc(&m->tileRowSlot, (uint64_t)nnz * 8);
            dev_alloc(&m->tileLocalBit, nnz);
            m->pull_plan_bytes = tcc::pull_scratch_bytes(m->numColWindows, nnz);
            TCC_CUDA(cudaMalloc(&m->pull_plan, m->pull_plan_bytes));
        } catch (...) {
            tcc_swtcf_free(m);
            throw;
        }
    });
}

static void release_fwd(tcc_swtcf* m) {
    cudaFree(m->fwdRowWindowOffset);
    cudaFree(m->fwdTcOffset);
    cudaFree(m->fwdSparseA2B);
    cudaFree(m->fwdTcLocalBit);
    cudaFree(m->fwd_plan);
    m->fwdRowWindowOffset = m->fwdTcOffset = m->fwdSparseA2B = nullptr;
    m->fwdTcLocalBit = nullptr;
    m->fwd_plan = nullptr;
    m->fwd_tiles = m->fwd_plan_bytes = 0;
    m->fwd_ready = m->fwd_plan_ready = 0;
}

tcc_status tcc_swtcf_free(tcc_swtcf* m) {
    return guarded("tcc_swtcf_free", [&] {
        if (!m) return;
        release_fwd(m);
        cudaFree(m->superWindowRowOffset);
        cudaFree(m->superWindowRows);
        cudaFree(m->superWindowRowCacheSlot);
        cudaFree(m->superWindowCachedRowSlot);
        cudaFree(m->superWindowCachedCount);
        cudaFree(m->colWindowOffset);
        cudaFree(m->tileRowSlot);
        cudaFree(m->tileLocalBit);
        cudaFree(m->pull_plan);
        *m = tcc_swtcf{};
    });
}

tcc_status tcc_swtcf_workspace_create(tcc_swtcf_workspace** ws, uint64_t edge_capacity,
                                      uint32_t num_src, uint32_t S) {
    return guarded("tcc_swtcf_workspace_create", [&] {
        TCC_REQUIRE(ws, "null workspace pointer");
        *ws = nullptr;
        TCC_REQUIRE(edge_capacity > 0 && num_src > 0 && S > 0 && S <= TCC_SWTCF_MAX_SUPER_WINDOW,
                    "invalid converter workspace size");
        TCC_REQUIRE(edge_capacity < (1ull << 31), "edge capacity must stay below 2^31");
        *ws = new tcc_swtcf_workspace(edge_capacity, num_src, S);
    });
}

tcc_status tcc_swtcf_workspace_destroy(tcc_swtcf_workspace* ws) {
    return guarded("tcc_swtcf_workspace_destroy", [&] { delete ws; });
}

tcc_status tcc_swtcf_convert_coo(const uint32_t* d_dst, const uint32_t* d_src, uint64_t nnz,
                                 tcc_swtcf* out, tcc_swtcf_workspace* ws, cudaStream_t stream) {
    return guarded("tcc_swtcf_convert_coo", [&] {
        TCC_REQUIRE(ws && out && d_dst && d_src, "null argument");
        tcc::swtcf_convert(d_dst, d_src, nullptr, nullptr, nnz, out, ws->impl, stream);
        out->pull_plan_ready = 0;
        out->fwd_ready = 0;
        // the transposed pass's work plan, on the conversion's stream: ready
        // whenever the tiles are
        tcc::pull_plan(swtcf_t_pull(out), out->pull_plan, out->pull_plan_bytes, stream);
        out->pull_plan_ready = 1;
    });
}

tcc_status tcc_swtcf_convert_csr(const uint64_t* d_rowptr, const uint32_t* d_col, uint32_t rows,
                                 uint64_t nnz, tcc_swtcf* out, tcc_swtcf_workspace* ws,
                                 cudaStream_t stream) {
    return guarded("tcc_swtcf_convert_csr", [&] {
        TCC_REQUIRE(ws && out && d_rowptr && d_col, "null argument");
        TCC_REQUIRE(rows == out->rows, "CSR row count differs from the matrix's rows");
        tcc::swtcf_convert(nullptr, nullptr, d_rowptr, d_col, nnz, out, ws->impl, stream);
        out->pull_plan_ready = 0;
        out->fwd_ready = 0;
        // the transposed pass's work plan, on the conversion's stream: ready
        // whenever the tiles are
        tcc::pull_plan(swtcf_t_pull(out), out->pull_plan, out->pull_plan_bytes, stream);
        out->pull_plan_ready = 1;
    });
}

tcc_status tcc_swtcf_workspace_device_error(tcc_swtcf_workspace* ws, cudaStream_t stream,
                                            uint32_t* code) {
    return guarded("tcc_swtcf_workspace_device_error", [&] {
        TCC_REQUIRE(ws && code, "null argument");
        TCC_CUDA(cudaMemcpyAsync(code, ws->impl.small, 4, cudaMemcpyDeviceToHost, stream));
        TCC_CUDA(cudaStreamSynchronize(stream));
    });
}

tcc_status tcc_swtcf_sizes(const tcc_swtcf* m, cudaStream_t stream, uint64_t* num_tiles,
                           uint64_t* num_rows) {
    return guarded("tcc_swtcf_sizes", [&] {
        TCC_REQUIRE(m && num_tiles && num_rows, "null argument");
        uint32_t t = 0, r = 0;
        TCC_CUDA(cudaMemcpyAsync(&t, m->colWindowOffset + m->numColWindows, 4,
                                 cudaMemcpyDeviceToHost, stream));
        TCC_CUDA(cudaMemcpyAsync(&r, m->superWindowRowOffset + m->numSuperWindows, 4,
                                 cudaMemcpyDeviceToHost, stream));
        TCC_CUDA(cudaStreamSynchronize(stream));
        *num_tiles = t;
        *num_rows = r;
    });
}

static tcc::PushTiles swtcf_push(const tcc_swtcf* m) {
    tcc::PushTiles t{};
    t.num_windows = m->numColWindows;
    t.win_offset = m->colWindowOffset;
    t.bits = m->tileLocalBit;
    t.idx = m->tileRowSlot;
    t.sw_offset = m->superWindowRowOffset;
    t.sw_rows = m->superWindowRows;
    t.sw_cache_slot = m->superWindowRowCacheSlot;
    t.sw_cached_row_slot = m->superWindowCachedRowSlot;
    t.sw_cached_count = m->superWindowCachedCount;
    t.S = m->superWindowSize;
    t.num_out = m->rows;
    t.num_in = m->cols;
    return t;
}

// The prepared row-window tiling as a pull operand (tcc_swtcf_prepare_pull).
static tcc::PullTiles swtcf_fwd_pull(const tcc_swtcf* m) {
    tcc::PullTiles t{};
    t.num_windows = (m->rows + 7) / 8;
    t.num_tiles = (uint32_t)m->fwd_tiles;
    t.win_offset = m->fwdRowWindowOffset;
    t.bits = m->fwdTcLocalBit;
    t.idx = m->fwdSparseA2B;
    t.bits_transposed = false;
    t.num_out = m->rows;
    t.num_in = m->cols;
    return t;
}

static void swtcf_forward(const tcc_swtcf* m, const tcc::Dense& d, uint32_t tc_threshold,
                          int accumulate, cudaStream_t stream) {
    if (m->fwd_ready) {
        // plan built and synchronised by tcc_swtcf_prepare_pull
        tcc::pull_spmm(swtcf_fwd_pull(m), d, tc_threshold, accumulate, m->fwd_plan,
                       m->fwd_plan_bytes, m->fwd_plan_ready != 0, nullptr, stream);
        return;
    }
    if (!accumulate) zero_rows(d.Y, d.ldy, d.F, m->rows, stream);
    tcc::push_spmm(swtcf_push(m), d, tc_threshold, nullptr, stream);
}

tcc_status tcc_swtcf_prepare_pull(tcc_swtcf* m, cudaStream_t stream) {
    return guarded("tcc_swtcf_prepare_pull", [&] {
        TCC_REQUIRE(m && m->colWindowOffset, "null or unallocated matrix");
        release_fwd(m);
        tcc::TilesWorkspace ws(std::max<uint64_t>(m->nnz, 1), m->rows, m->cols);
        const uint64_t T = tcc::tiles_prepare_swtcf(ws, m, stream);
        const uint32_t W = (m->rows + 7) / 8;
        try {
            dev_alloc(&m->fwdRowWindowOffset, (uint64_t)W + 1);
            dev_alloc(&m->fwdTcOffset, T + 1);
            dev_alloc(&m->fwdSparseA2B, 8 * T);
            dev_alloc(&m->fwdTcLocalBit, T);
            tcc::tiles_fill(ws, TCC_TILES_BCSR, m->fwdRowWindowOffset, m->fwdTcOffset,
                            m->fwdSparseA2B, m->fwdTcLocalBit, stream);
            m->fwd_plan_bytes = tcc::pull_scratch_bytes(W, T);
            TCC_CUDA(cudaMalloc(&m->fwd_plan, m->fwd_plan_bytes));
            m->fwd_tiles = T;
            tcc::pull_plan(swtcf_fwd_pull(m), m->fwd_plan, m->fwd_plan_bytes, stream);
            // the workspace is freed on return, and forwards on any stream
            // reuse the plan: finish the fill and the plan first
            TCC_CUDA(cudaStreamSynchronize(stream));
            m->fwd_ready = 1;
            m->fwd_plan_ready = 1;
        } catch (...) {
            release_fwd(m);
            throw;
        }
    });
}

tcc_status tcc_swtcf_spmm(const tcc_swtcf* m, const float* X, float* Y, uint32_t tc_threshold,
                          cudaStream_t stream) {
    return guarded("tcc_swtcf_spmm", [&] {
        TCC_REQUIRE(m && X && Y, "null argument");
        TCC_REQUIRE(m->superWindowSize == 16, "SWTCF SpMM requires superWindowSize=16");
        tcc::Dense d{X, 128, Y, 128, 128, nullptr, nullptr};
        swtcf_forward(m, d, tc_threshold, 1, stream);
    });
}

tcc_status tcc_swtcf_spmm_quantized(const tcc_swtcf* m, const int8_t* q_x, const float* scales,
                                    const uint32_t* src_global, float* Y, uint32_t tc_threshold,
                                    cudaStream_t stream) {
    return guarded("tcc_swtcf_spmm_quantized", [&] {
        TCC_REQUIRE(m && q_x && scales && Y, "null argument");
        TCC_REQUIRE(m->superWindowSize == 16, "Quantized SWTCF SpMM requires superWindowSize=16");
        tcc::Dense d{nullptr, 128, Y, 128, 128, nullptr, nullptr};
        d.qX = q_x;
        d.ldq = 128;
        d.qscale = scales;
        d.qmap = src_global;
        tcc::push_spmm(swtcf_push(m), d, tc_threshold, nullptr, stream);
    });
}

tcc_status tcc_swtcf_spmm_ex(const tcc_swtcf* m, const float* X, uint64_t ldx, float* Y,
                             uint64_t ldy, uint32_t F, uint32_t tc_threshold,
                             const float* row_scale, const float* col_scale, int accumulate,
                             cudaStream_t stream) {
    return guarded("tcc_swtcf_spmm_ex", [&] {
        TCC_REQUIRE(m && X && Y, "null argument");
        tcc::Dense d{X, ldx, Y, ldy, F, row_scale, col_scale};
        swtcf_forward(m, d, tc_threshold, accumulate, stream);
    });
}

tcc_status tcc_swtcf_spmm_t(const tcc_swtcf* m, const float* G, uint64_t ldg, float* Z,
                            uint64_t ldz, uint32_t F, uint32_t tc_threshold,
                            const float* row_scale, const float* col_scale, int accumulate,
                            cudaStream_t stream) {
    return guarded("tcc_swtcf_spmm_t", [&] {
        TCC_REQUIRE(m && G && Z, "null argument");
        // Z = diag(cs) A^T diag(rs) G: G rows are scaled by rs, Z rows by cs
        tcc::Dense d{G, ldg, Z, ldz, F, col_scale, row_scale};
        // the plan was built on the conversion's stream, right after the tiles
        tcc::pull_spmm(swtcf_t_pull(m), d, tc_threshold, accumulate, m->pull_plan,
                       m->pull_plan_bytes, m->pull_plan_ready != 0, nullptr, stream);
    });
}

// -------------------------------------------------------------- BCSR/BCSC --

tcc_status tcc_tiles_workspace_create(tcc_tiles_workspace** ws, uint64_t nnz_capacity,
                                      uint32_t rows, uint32_t cols) {
    return guarded("tcc_tiles_workspace_create", [&] {
        TCC_REQUIRE(ws, "null workspace pointer");
        *ws = nullptr;
        TCC_REQUIRE(rows > 0 && cols > 0, "empty matrix shape");
        TCC_REQUIRE(nnz_capacity < (1ull << 31), "nnz capacity must stay below 2^31");
        *ws = new tcc_tiles_workspace(nnz_capacity, rows, cols);
    });
}

tcc_status tcc_tiles_workspace_destroy(tcc_tiles_workspace* ws) {
    return guarded("tcc_tiles_workspace_destroy", [&] { delete ws; });
}

tcc_status tcc_tiles_prepare_csr(tcc_tiles_workspace* ws, int kind, const uint64_t* d_rowptr,
                                 const uint32_t* d_col, uint32_t rows, uint32_t cols,
                                 uint64_t nnz, cudaStream_t stream, uint64_t* num_tiles) {
    return guarded("tcc_tiles_prepare_csr", [&] {
        TCC_REQUIRE(ws && d_rowptr && num_tiles && (d_col || nnz == 0), "null argument");
        *num_tiles = tcc::tiles_prepare(ws->impl, kind, d_rowptr, d_col, rows, cols, nnz, stream);
    });
}

tcc_status tcc_tiles_fill_bcsr(tcc_tiles_workspace* ws, tcc_bcsr* out, cudaStream_t stream) {
    return guarded("tcc_tiles_fill_bcsr", [&] {
        TCC_REQUIRE(ws && out, "null argument");
        auto& w = ws->impl;
        TCC_REQUIRE(out->rowWindowOffset && out->tcOffset && (w.T == 0 || (out->sparseA2B && out->tcLocalBit)),
                    "BCSR arrays missing");
        tcc::tiles_fill(w, TCC_TILES_BCSR, out->rowWindowOffset, out->tcOffset, out->sparseA2B,
                        out->tcLocalBit, stream);
        out->num_rows = w.cur_rows;
        out->num_cols = w.cur_cols;
        out->nnz = (uint32_t)w.nnz;
        out->num_TCBlocks = (uint32_t)w.T;
        out->num_rowWindows = w.W;
    });
}

tcc_status tcc_tiles_fill_bcsc(tcc_tiles_workspace* ws, tcc_bcsc* out, cudaStream_t stream) {
    return guarded("tcc_tiles_fill_bcsc", [&] {
        TCC_REQUIRE(ws && out, "null argument");
        auto& w = ws->impl;
        TCC_REQUIRE(out->colWindowOffset && out->tcOffset && (w.T == 0 || (out->sparseA2C && out->tcLocalBit)),
                    "BCSC arrays missing");
        tcc::tiles_fill(w, TCC_TILES_BCSC, out->colWindowOffset, out->tcOffset, out->sparseA2C,
                        out->tcLocalBit, stream);
        out->num_rows = w.cur_rows;
        out->num_cols = w.cur_cols;
        out->nnz = (uint32_t)w.nnz;
        out->num_TCBlocks = (uint32_t)w.T;
        out->num_colWindows = w.W;
    });
}

size_t tcc_pull_scratch_bytes(uint32_t num_windows, uint32_t num_tiles) {
    return tcc::pull_scratch_bytes(num_windows, num_tiles);
}

void tcc_set_grid_reserve(uint32_t sms) { tcc::set_grid_reserve(sms); }
uint32_t tcc_get_grid_reserve(void) { return tcc::grid_reserve(); }
void tcc_set_wait_limit_ns(uint64_t ns) {
    tcc::set_wait_limit_ns(ns ? ns : (uint64_t)TCC_DEFAULT_WAIT_LIMIT_NS);
}
uint64_t tcc_get_wait_limit_ns(void) { return tcc::wait_limit_ns(); }

tcc_status tcc_gather_rows(const float* X, uint64_t ldx, uint64_t num_rows, const int64_t* idx,
                           uint64_t n, float* out, uint64_t ldo, uint32_t F, uint32_t* bad_flag,
                           cudaStream_t stream) {
    return guarded("tcc_gather_rows", [&] {
        TCC_REQUIRE(n == 0 || (X && idx && out), "X, idx and out must not be NULL");
        tcc::gather_rows(X, ldx, num_rows, idx, n, out, ldo, F, bad_flag, stream);
    });
}

tcc_status tcc_scatter_add_rows(const float* in, uint64_t ldi, const int64_t* idx, uint64_t n,
                                float* out, uint64_t ldo, uint64_t num_rows, uint32_t F,
                                uint32_t* bad_flag, cudaStream_t stream) {
    return guarded("tcc_scatter_add_rows", [&] {
        TCC_REQUIRE(n == 0 || (in && idx && out), "in, idx and out must not be NULL");
        tcc::scatter_add_rows(in, ldi, idx, n, out, ldo, num_rows, F, bad_flag, stream);
    });
}

tcc_status tcc_peer_alloc(size_t bytes, void** ptr, tcc_ipc_handle* handle) {
    static_assert(sizeof(tcc_ipc_handle) == sizeof(cudaIpcMemHandle_t), "IPC handle size");
    return guarded("tcc_peer_alloc", [&] { tcc::peer_alloc(bytes, ptr, handle); });
}

tcc_status tcc_peer_open(const tcc_ipc_handle* handle, void** ptr) {
    return guarded("tcc_peer_open", [&] { tcc::peer_open(handle, ptr); });
}

tcc_status tcc_peer_close(void* mapped) {
    return guarded("tcc_peer_close", [&] { tcc::peer_close(mapped); });
}

tcc_status tcc_peer_free(void* ptr) {
    return guarded("tcc_peer_free", [&] { tcc::peer_free(ptr); });
}

tcc_status tcc_halo_push(const tcc_halo_push_args* args, cudaStream_t stream) {
    return guarded("tcc_halo_push", [&] { tcc::halo_push(args, stream); });
}

tcc_status tcc_halo_wait(void* flags, uint32_t tag, uint32_t seq, uint32_t peer_mask,
                         uint64_t wait_ns, cudaStream_t stream) {
    return guarded("tcc_halo_wait",
                   [&] { tcc::halo_wait(flags, tag, seq, peer_mask, wait_ns, stream); });
}

tcc_status tcc_halo_release(void* const* peer_flags, uint32_t world, uint32_t rank, uint32_t tag,
                            uint32_t seq, uint32_t peer_mask, cudaStream_t stream) {
    return guarded("tcc_halo_release", [&] {
        tcc::halo_release(peer_flags, world, rank, tag, seq, peer_mask, stream);
    });
}

tcc_status tcc_peer_device_error(void* flags, int* code, cudaStream_t stream) {
    return guarded("tcc_peer_device_error", [&] { tcc::peer_device_error(flags, code, stream); });
}

namespace {

// Fork/join events of tcc_dist_step, one pair per host thread and device.
struct StepEvents {
    int device = -1;
    cudaEvent_t fork = nullptr, join = nullptr;
};
thread_local StepEvents g_step_events;

StepEvents& step_events() {
    int dev = 0;
    TCC_CUDA(cudaGetDevice(&dev));
    StepEvents& e = g_step_events;
    if (e.device != dev) {
        TCC_CUDA(cudaEventCreateWithFlags(&e.fork, cudaEventDisableTiming));
        TCC_CUDA(cudaEventCreateWithFlags(&e.join, cudaEventDisableTiming));
        e.device = dev;
    }
    return e;
}

// The pull kernels' SM reserve for the scope of one pass.
struct ReserveScope {
    uint32_t prev;
    explicit ReserveScope(uint32_t sms) : prev(tcc::grid_reserve()) { tcc::set_grid_reserve(sms); }
    ~ReserveScope() { tcc::set_grid_reserve(prev); }
};

}  // namespace

tcc_status tcc_dist_step(const tcc_dist_step_args* a, cudaStream_t main, cudaStream_t side) {
    return guarded("tcc_dist_step", [&] {
        TCC_REQUIRE(a, "args must not be NULL");
        TCC_REQUIRE(a->n_ops == 1 || a->n_ops == 2, "n_ops must be 1 or 2");
        check_bcsr(a->local);
        if (a->halo) check_bcsr(a->halo);
        for (uint32_t i = 0; i < a->n_ops; ++i) {
            const tcc_dist_operand& op = a->ops[i];
            TCC_REQUIRE(op.push.x && op.y, "operand rows and outputs must not be NULL");
            TCC_REQUIRE(op.push.num_rows == a->local->num_rows && a->local->num_cols == a->local->num_rows,
                        "the local tiles cover this rank's rows and columns");
            TCC_REQUIRE(!a->halo || op.halo || a->halo->num_TCBlocks == 0,
                        "halo rows must not be NULL when there are halo tiles");
        }
        auto record = [&](int k, cudaStream_t s) {
            if (a->events[k]) TCC_CUDA(cudaEventRecord(a->events[k], s));
        };
        StepEvents& ev = step_events();
        TCC_CUDA(cudaEventRecord(ev.fork, main));
        TCC_CUDA(cudaStreamWaitEvent(side, ev.fork, 0));
        for (uint32_t i = 0; i < a->n_ops; ++i) {
            tcc::halo_push(&a->ops[i].push, side);
            record((int)i, side);
        }
        const tcc::PullTiles loc = bcsr_pull(a->local);
        bool loc_ready = a->local_plan_ready != 0;
        for (uint32_t i = 0; i < a->n_ops; ++i) {
            const tcc_dist_operand& op = a->ops[i];
            ReserveScope r((a->reserve_passes >> i & 1u) ? a->reserve_sms : 0);
            tcc::Dense d{op.push.x, op.push.ldx, op.y, op.ldy, op.push.width, a->rs, a->cs_local};
            tcc::pull_spmm(loc, d, a->tc_threshold, 0, a->local_scratch, a->local_scratch_bytes,
                           loc_ready, nullptr, main);
            loc_ready = true;
            record(2 + (int)i, main);
        }
        bool halo_ready = a->halo_plan_ready != 0;
        for (uint32_t i = 0; i < a->n_ops; ++i) {
            const tcc_dist_operand& op = a->ops[i];
            tcc::halo_wait(op.push.flags, op.push.tag, op.push.seq, a->recv_mask, op.push.wait_ns,
                           main);
            if (a->halo && a->halo->num_TCBlocks) {
                ReserveScope r((a->reserve_passes >> (2 + i) & 1u) ? a->reserve_sms : 0);
                tcc::Dense d{op.halo, op.ld_halo, op.y, op.ldy, op.push.width, a->rs, a->cs_halo};
                tcc::pull_spmm(bcsr_pull(a->halo), d, a->tc_threshold, 1, a->halo_scratch,
                               a->halo_scratch_bytes, halo_ready, nullptr, main);
                halo_ready = true;
            }
            tcc::halo_release(a->peer_flags, op.push.world, op.push.rank, op.push.tag, op.push.seq,
                              a->recv_mask, main);
            record(4 + (int)i, main);
        }
        TCC_CUDA(cudaEventRecord(ev.join, side));
        TCC_CUDA(cudaStreamWaitEvent(main, ev.join, 0));
    });
}

tcc_status tcc_relu_dropout_forward(const float* in, float* out, uint64_t n, float p,
                                    uint64_t seed, cudaStream_t stream) {
    return guarded("tcc_relu_dropout_forward", [&] {
        TCC_REQUIRE(n == 0 || (in && out), "null argument");
        tcc::relu_dropout_forward(in, out, n, p, seed, stream);
    });
}

tcc_status tcc_relu_dropout_backward(const float* grad_out, const float* out, float* grad_in,
                                     uint64_t n, float p, cudaStream_t stream) {
    return guarded("tcc_relu_dropout_backward", [&] {
        TCC_REQUIRE(n == 0 || (grad_out && out && grad_in), "null argument");
        tcc::relu_dropout_backward(grad_out, out, grad_in, n, p, stream);
    });
}

tcc_status tcc_pull_device_error(void* scratch, int* code, cudaStream_t stream) {
    return guarded("tcc_pull_device_error", [&] {
        TCC_REQUIRE(scratch && code, "scratch and code must not be NULL");
        uint32_t* word = reinterpret_cast<uint32_t*>(static_cast<char*>(scratch) + tcc::kPullErrorOffset);
        uint32_t v = 0;
        TCC_CUDA(cudaMemcpyAsync(&v, word, sizeof(v), cudaMemcpyDeviceToHost, stream));
        TCC_CUDA(cudaMemsetAsync(word, 0, sizeof(v), stream));
        TCC_CUDA(cudaStreamSynchronize(stream));
        *code = (int)v;
    });
}

tcc_status tcc_bcsr_spmm(const tcc_bcsr* a, const float* B, uint64_t ldb, float* C, uint64_t ldc,
                         uint32_t F, uint32_t tc_threshold, const float* rs, const float* cs,
                         int accumulate, void* scratch, size_t scratch_bytes, int plan_ready,
                         cudaStream_t stream) {
    return guarded("tcc_bcsr_spmm", [&] {
        check_bcsr(a);
        TCC_REQUIRE(B && C, "null argument");
        tcc::Dense d{B, ldb, C, ldc, F, rs, cs};
        tcc::pull_spmm(bcsr_pull(a), d, tc_threshold, accumulate, scratch, scratch_bytes,
                       plan_ready != 0, nullptr, stream);
    });
}

tcc_status tcc_bcsr_spmm_noalloc(const tcc_bcsr* a, const float* B, uint64_t ldb, float* C,
                                 uint64_t ldc, uint32_t F, uint32_t tc_threshold, const float* rs,
                                 const float* cs, int accumulate, cudaStream_t stream) {
    return guarded("tcc_bcsr_spmm_noalloc", [&] {
        check_bcsr(a);
        TCC_REQUIRE(B && C, "null argument");
        const size_t need = tcc::pull_scratch_bytes(a->num_rowWindows, a->num_TCBlocks);
        if (need > TCC_NOALLOC_SCRATCH_BYTES)
            throw tcc::Error(TCC_ERR_CAPACITY,
                             "tiling needs " + std::to_string(need) +
                                 " bytes of plan scratch; the built-in scratch holds " +
                                 std::to_string((size_t)TCC_NOALLOC_SCRATCH_BYTES) +
                                 " (use tcc_bcsr_spmm with caller scratch)");
        // the shared array keeps the last call's contents: the plan is rebuilt
        // (or, for the kernels that need none, only the header cleared) every
        // call, which also zeroes the error word; no later call reuses it
        tcc::Dense d{B, ldb, C, ldc, F, rs, cs};
        tcc::pull_spmm(bcsr_pull(a), d, tc_threshold, accumulate, noalloc_scratch(),
                       TCC_NOALLOC_SCRATCH_BYTES, false, nullptr, stream, /*keep_plan=*/false);
    });
}

tcc_status tcc_noalloc_device_error(int* code, cudaStream_t stream) {
    return guarded("tcc_noalloc_device_error", [&] {
        TCC_REQUIRE(code, "code must not be NULL");
        uint32_t* word = reinterpret_cast<uint32_t*>(static_cast<char*>(noalloc_scratch()) +
                                                     tcc::kPullErrorOffset);
        uint32_t v = 0;
        TCC_CUDA(cudaMemcpyAsync(&v, word, sizeof(v), cudaMemcpyDeviceToHost, stream));
        TCC_CUDA(cudaMemsetAsync(word, 0, sizeof(v), stream));
        TCC_CUDA(cudaStreamSynchronize(stream));
        *code = (int)v;
    });
}

tcc_status tcc_bcsr_spmm_t(const tcc_bcsr* a, const float* G, uint64_t ldg, float* Z, uint64_t ldz,
                           uint32_t F, uint32_t tc_threshold, const float* rs, const float* cs,
                           cudaStream_t stream) {
    return guarded("tcc_bcsr_spmm_t", [&] {
        check_bcsr(a);
        TCC_REQUIRE(G && Z, "null argument");
        // Z += diag(cs) A^T diag(rs) G: G rows (window inputs) scaled by rs, Z rows by cs
        tcc::Dense d{G, ldg, Z, ldz, F, cs, rs};
        tcc::push_spmm(bcsr_push_t(a), d, tc_threshold, nullptr, stream);
    });
}

tcc_status tcc_bcsc_spmm(const tcc_bcsc* a, const float* B, uint64_t ldb, float* C, uint64_t ldc,
                         uint32_t F, uint32_t tc_threshold, const float* rs, const float* cs,
                         cudaStream_t stream) {
    return guarded("tcc_bcsc_spmm", [&] {
        check_bcsc(a);
        TCC_REQUIRE(B && C, "null argument");
        tcc::Dense d{B, ldb, C, ldc, F, rs, cs};
        tcc::push_spmm(bcsc_push(a), d, tc_threshold, nullptr, stream);
    });
}

tcc_status tcc_bcsc_spmm_t(const tcc_bcsc* a, const float* G, uint64_t ldg, float* Z,
                           uint64_t ldz, uint32_t F, uint32_t tc_threshold, const float* rs,
                           const float* cs, int accumulate, void* scratch, size_t scratch_bytes,
                           int plan_ready, cudaStream_t stream) {
    return guarded("tcc_bcsc_spmm_t", [&] {
        check_bcsc(a);
        TCC_REQUIRE(G && Z, "null argument");
        tcc::Dense d{G, ldg, Z, ldz, F, cs, rs};
        tcc::pull_spmm(bcsc_pull_t(a), d, tc_threshold, accumulate, scratch, scratch_bytes,
                       plan_ready != 0, nullptr, stream);
    });
}

static void cnic_forward(const tcc_bcsr* bcsr, const tcc_bcsc* bcsc, const float* B, float* C,
                         uint32_t F, uint32_t thr, void* scratch, size_t scratch_bytes,
                         const tcc::FeatureStore* fs, cudaStream_t stream) {
    TCC_REQUIRE(bcsr || bcsc, "need a BCSR or a BCSC part");
    TCC_REQUIRE(C && (fs || B), "null argument");
    if (bcsr) check_bcsr(bcsr);
    if (bcsc) check_bcsc(bcsc);
    const uint32_t rows = bcsr ? bcsr->num_rows : bcsc->num_rows;
    const uint32_t cols = bcsr ? bcsr->num_cols : bcsc->num_cols;
    TCC_REQUIRE(!bcsr || !bcsc || (bcsr->num_rows == bcsc->num_rows && bcsr->num_cols == bcsc->num_cols),
                "BCSR and BCSC parts disagree on the matrix shape");
    const uint64_t padded = ((uint64_t)(rows + 7) / 8 + 1) * 8;  // spmm_launcher.cu:231
    if (bcsr) {
        tcc::Dense d{B, F, C, F, F, nullptr, nullptr};
        tcc::pull_spmm(bcsr_pull(bcsr), d, thr, 0, scratch, scratch_bytes, false, fs, stream);
        zero_rows(C + (uint64_t)rows * F, F, F, padded - rows, stream);
    } else {
        zero_rows(C, F, F, padded, stream);
    }
    (void)cols;
    if (bcsc) {
        tcc::Dense d{B, F, C, F, F, nullptr, nullptr};
        tcc::push_spmm(bcsc_push(bcsc), d, thr, fs, stream);
    }
}

tcc_status tcc_cnic_forward(const tcc_bcsr* bcsr, const tcc_bcsc* bcsc, const float* B, float* C,
                            uint32_t F, uint32_t tc_threshold, void* scratch, size_t scratch_bytes,
                            cudaStream_t stream) {
    return guarded("tcc_cnic_forward", [&] {
        cnic_forward(bcsr, bcsc, B, C, F, tc_threshold, scratch, scratch_bytes, nullptr, stream);
    });
}

tcc_status tcc_cnic_forward_mixed(const tcc_bcsr* bcsr, const tcc_bcsc* bcsc,
                                  const int32_t* id_map, const float* cpu_features,
                                  const int32_t* cache_search_map,
                                  const float* const* gpu_features, int64_t gpu_capacity,
                                  float* C, uint32_t F, uint32_t tc_threshold, void* scratch,
                                  size_t scratch_bytes, cudaStream_t stream) {
    return guarded("tcc_cnic_forward_mixed", [&] {
        TCC_REQUIRE(id_map && cache_search_map && cpu_features, "null feature-store argument");
        TCC_REQUIRE(gpu_capacity > 0 && gpu_features, "GPU feature cache missing");
        tcc::FeatureStore fs;
        fs.id_map = id_map;
        fs.cpu_features = cpu_features;
        fs.cache_search_map = cache_search_map;
        fs.gpu_features = gpu_features;
        fs.gpu_capacity = gpu_capacity;
        cnic_forward(bcsr, bcsc, nullptr, C, F, tc_threshold, scratch, scratch_bytes, &fs, stream);
    });
}

}  // extern "C"
