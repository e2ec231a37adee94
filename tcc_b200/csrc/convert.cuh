// convert.cuh -- converter workspaces (behind the opaque C-ABI workspace types)
// and the conversion entry points used by capi.cu.
#pragma once

#include "common.cuh"

namespace tcc {

// One cudaMalloc carved into 256-byte aligned pieces.
struct Arena {
    char* base = nullptr;
    size_t total = 0;
    size_t used = 0;
    void reserve(size_t bytes);
    void* take(size_t bytes);
};

// Sort / group buffers, each sized by the edge capacity.
struct GroupBuffers {
    uint64_t *keys, *keys_alt, *gkey;
    uint32_t *vals, *vals_alt, *head, *excl, *gmask, *gstart;
};

struct SwtcfWorkspace {
    uint64_t E;          // edge capacity
    uint32_t W, SW, S;   // windows / super-windows / super-window size it was sized for
    Arena arena;
    GroupBuffers g;
    uint32_t *gslot, *rstart, *occ, *order, *wcnt, *wgstart, *tiles, *swcnt;
    uint32_t* small;     // [0] device error word, [1] groups, [2] super-window rows R
    void* tmp;
    size_t tmp_bytes;
    SwtcfWorkspace(uint64_t edge_capacity, uint32_t num_src, uint32_t S);
    ~SwtcfWorkspace();
};

struct TilesWorkspace {
    uint64_t E;
    uint32_t rows, cols;  // capacity
    Arena arena;
    GroupBuffers g;
    uint32_t *wcnt, *wgstart, *tiles, *off, *small;
    void* tmp;
    size_t tmp_bytes;
    // state between prepare and fill
    bool prepared = false;
    int kind = -1;
    uint32_t cur_rows = 0, cur_cols = 0, W = 0, ng = 0;
    uint64_t nnz = 0, T = 0;
    int ybits = 1;
    TilesWorkspace(uint64_t nnz_capacity, uint32_t rows, uint32_t cols);
    ~TilesWorkspace();
};

// COO (d_dst/d_src) or CSR (d_rowptr/d_col) -> SWTCF; asynchronous.
void swtcf_convert(const uint32_t* d_dst, const uint32_t* d_src, const uint64_t* d_rowptr,
                   const uint32_t* d_col, uint64_t nnz, tcc_swtcf* m, SwtcfWorkspace& ws,
                   cudaStream_t s);

// CSR -> BCSR/BCSC: prepare (synchronises, returns T), then fill.
uint64_t tiles_prepare(TilesWorkspace& ws, int kind, const uint64_t* d_rowptr,
                       const uint32_t* d_col, uint32_t rows, uint32_t cols, uint64_t nnz,
                       cudaStream_t s);
// SWTCF tiles -> the same matrix as row-window (BCSR) tiles: prepare
// (synchronises, returns T), then tiles_fill with TCC_TILES_BCSR.
uint64_t tiles_prepare_swtcf(TilesWorkspace& ws, const tcc_swtcf* m, cudaStream_t s);
void tiles_fill(TilesWorkspace& ws, int kind, uint32_t* win_offset, uint32_t* tc_offset,
                uint32_t* idx, uint64_t* bits, cudaStream_t s);

}  // namespace tcc
