/*
 * tcc_b200.h -- C ABI of the B200-native (sm_100a) tcc graph-aggregation path.
 *
 * Plain pointers, sizes and cudaStream_t only.  Every entry point names the
 * reference interface it replaces (paths relative to the reference project
 * root; "cnic/" is TAC_training_backend/spmm_cnic/).  All device pointers are
 * global-memory pointers on the current device; calls are asynchronous on
 * `stream` unless marked "synchronises".  No C++ exception crosses this ABI:
 * each call returns a tcc_status and tcc_last_error() describes the last
 * failure of the calling thread.
 *
 * Layouts are the reference's, bit for bit:
 *   SWTCF  include/swtcf_convert.cuh:13-35 (8x8 tiles in 8-column windows,
 *          16-window super-windows, 32-row repeat cache)
 *   BCSR   cnic/include/class.h:20-37 (8-row windows, condensed columns)
 *   BCSC   cnic/include/class.h:39-57 (8-column windows, condensed rows)
 * with one canonical order where the reference's converter is order-free:
 * rows of an SWTCF window by degree descending then dst ascending, super-window
 * rows by dst ascending, cache ranks by occurrence descending then slot
 * ascending; BCSR/BCSC condensed indices ascending, padding 0xFFFFFFFF.
 */
#ifndef TCC_B200_H
#define TCC_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------- status ---- */
typedef int tcc_status;
#define TCC_OK 0
#define TCC_ERR_INVALID_ARGUMENT 1 /* reference: std::runtime_error("invalid ...") */
#define TCC_ERR_CUDA 2             /* a CUDA runtime call failed */
#define TCC_ERR_OUT_OF_MEMORY 3
#define TCC_ERR_UNSUPPORTED 4      /* configuration the path does not implement */
#define TCC_ERR_DEVICE 5           /* a kernel raised a device error code (below) */
#define TCC_ERR_CAPACITY 6         /* output/workspace capacity too small */

/* Device error codes written to a workspace error word (the reference's
 * SWTCFConvertWorkspace::deviceError, src/swtcf_convert.cu:190-194, :582-585,
 * :981-999, :765-775).  Codes 2 and 3 belong to the reference's hash table,
 * which this implementation replaces by sorting; they are never raised. */
#define TCC_DEVERR_NONE 0
#define TCC_DEVERR_GROUP_DEGREE 1  /* a (window,row) group holds a duplicate edge */
#define TCC_DEVERR_HASH_FULL 2
#define TCC_DEVERR_HASH_LOOKUP 3
#define TCC_DEVERR_OCCURRENCE 4    /* row occurrence above the super-window size */
#define TCC_DEVERR_INDEX_RANGE 5   /* an input index >= rows/cols */
#define TCC_DEVERR_WAIT_TIMEOUT 6  /* an in-kernel wait for a TMA copy expired (the
                                      limit of tcc_set_wait_limit_ns, 2 s by default); the
                                      kernel returned early and its output is incomplete */

const char* tcc_last_error(void);
const char* tcc_version(void);

/* ------------------------------------------------------------- SWTCF ----- */
#define TCC_SWTCF_WINDOW 8
#define TCC_SWTCF_CACHE_ROWS 32
#define TCC_SWTCF_MAX_SUPER_WINDOW 32
#define TCC_SWTCF_FEATURE_DIM 128      /* include/swtcf_spmm.cuh:7 */
#define TCC_SWTCF_DEFAULT_TC_THRESHOLD 12

/* Field-for-field DeviceSWTCFMatrix (include/swtcf_convert.cuh:13-35); the
 * trailing fields are this implementation's. */
typedef struct tcc_swtcf {
    uint32_t rows, cols, nnz;
    uint32_t colWindowWidth, tileRows, superWindowSize;
    uint32_t numColWindows, numSuperWindows;
    uint32_t* superWindowRowOffset;      /* [numSuperWindows+1] */
    uint32_t* superWindowRows;           /* [capacity_rows] */
    uint8_t* superWindowRowCacheSlot;    /* [capacity_rows], 0xFF = uncached */
    uint32_t* superWindowCachedRowSlot;  /* [32*numSuperWindows] */
    uint8_t* superWindowCachedCount;     /* [numSuperWindows] */
    uint32_t* colWindowOffset;           /* [numColWindows+1] */
    uint32_t* tileRowSlot;               /* [8*capacity_tiles], 0xFFFFFFFF = padding */
    uint64_t* tileLocalBit;              /* [capacity_tiles], bit = localRow*8+localCol */
    uint64_t capacity_tiles, capacity_rows;
    /* work plan of the transposed pass, owned by the matrix; rebuilt lazily
     * after each conversion */
    void* pull_plan;
    uint64_t pull_plan_bytes;
    int32_t pull_plan_ready;
    /* row-window (BCSR) tiling of the same matrix for the forward pull, built
     * only by tcc_swtcf_prepare_pull and owned by the matrix; a conversion
     * marks it stale (fwd_ready = 0) and tcc_swtcf_free releases it */
    int32_t fwd_ready;
    uint32_t* fwdRowWindowOffset;        /* [ceil(rows/8)+1] */
    uint32_t* fwdTcOffset;               /* [fwd_tiles+1] */
    uint32_t* fwdSparseA2B;              /* [8*fwd_tiles] */
    uint64_t* fwdTcLocalBit;             /* [fwd_tiles] */
    uint64_t fwd_tiles;
    void* fwd_plan;
    uint64_t fwd_plan_bytes;
    int32_t fwd_plan_ready;
} tcc_swtcf;

typedef struct tcc_swtcf_workspace tcc_swtcf_workspace; /* opaque */

/* allocateDeviceSWTCF (include/swtcf_convert.cuh:74; src/swtcf_convert.cu:1113-1263):
 * capacities = nnz tiles / rows, like the reference. */
tcc_status tcc_swtcf_alloc(tcc_swtcf* m, uint32_t rows, uint32_t cols, uint32_t nnz,
                           uint32_t super_window_size);
/* freeDeviceSWTCF (include/swtcf_convert.cuh:75) */
tcc_status tcc_swtcf_free(tcc_swtcf* m);
/* allocateSWTCFConvertWorkspace (include/swtcf_convert.cuh:76; src/swtcf_convert.cu:1306-1655) */
tcc_status tcc_swtcf_workspace_create(tcc_swtcf_workspace** ws, uint64_t edge_capacity,
                                      uint32_t num_src, uint32_t super_window_size);
/* freeSWTCFConvertWorkspace (include/swtcf_convert.cuh:77) */
tcc_status tcc_swtcf_workspace_destroy(tcc_swtcf_workspace* ws);
/* convertCOOToSWTCF (include/swtcf_convert.cuh:78; src/swtcf_convert.cu:1754-2342):
 * canonical, deterministic; device errors land in the workspace error word. */
tcc_status tcc_swtcf_convert_coo(const uint32_t* d_dst, const uint32_t* d_src, uint64_t nnz,
                                 tcc_swtcf* out, tcc_swtcf_workspace* ws, cudaStream_t stream);
/* The CSR entry of the same conversion (row = dst, column = src). */
tcc_status tcc_swtcf_convert_csr(const uint64_t* d_rowptr, const uint32_t* d_col,
                                 uint32_t rows, uint64_t nnz, tcc_swtcf* out,
                                 tcc_swtcf_workspace* ws, cudaStream_t stream);
/* Reads the workspace's device error word (synchronises the stream). */
tcc_status tcc_swtcf_workspace_device_error(tcc_swtcf_workspace* ws, cudaStream_t stream,
                                            uint32_t* code);
/* T = colWindowOffset[numColWindows], R = superWindowRowOffset[numSuperWindows]
 * (synchronises the stream). */
tcc_status tcc_swtcf_sizes(const tcc_swtcf* m, cudaStream_t stream, uint64_t* num_tiles,
                           uint64_t* num_rows);

/* launchSWTCFSpMM (include/swtcf_spmm.cuh:10-16; src/swtcf_spmm.cu:437-466):
 * Y[numDst x 128] += pattern(A) * X[numSrc x 128]; tiles with popcount >=
 * tc_threshold use TF32 tensor cores, the others fp32.  Requires
 * superWindowSize == 16, like the reference. */
tcc_status tcc_swtcf_spmm(const tcc_swtcf* m, const float* X, float* Y, uint32_t tc_threshold,
                          cudaStream_t stream);
/* No reference counterpart.  Builds, once per conversion, a row-window tiling
 * of the converted matrix owned by m (allocates device memory: about 40 B per
 * tile plus a transient workspace of the conversion's size; synchronises the
 * stream).  Until the next conversion, tcc_swtcf_spmm and tcc_swtcf_spmm_ex
 * then run the forward product as a pull over those row windows (each output
 * row written by its window, no reductions) instead of the push over column
 * windows; the TF32 / fp32 choice by tc_threshold then applies to the
 * row-window tiles, so results differ from the push's by TF32 rounding on
 * different tiles (within the reference's 1e-3 bound).  Without this call the
 * forward entry points allocate nothing, like the reference's. */
tcc_status tcc_swtcf_prepare_pull(tcc_swtcf* m, cudaStream_t stream);
/* launchSWTCFSpMMQuantized (include/swtcf_spmm.cuh:18-26; src/swtcf_spmm.cu:
 * 268-432, 469-502): Y[numDst x 128] += pattern(A) * Xq where source column c
 * reads global node g = src_global[c] (NULL: g = c) and uses the int8 row
 * q_x[g*128 .. g*128+127] times scales[g] in fp32; tiles with popcount >=
 * tc_threshold use TF32 tensor cores, the others fp32.  Requires
 * superWindowSize == 16, like the reference. */
tcc_status tcc_swtcf_spmm_quantized(const tcc_swtcf* m, const int8_t* q_x, const float* scales,
                                    const uint32_t* src_global, float* Y, uint32_t tc_threshold,
                                    cudaStream_t stream);
/* General form: any F (multiple of 4), row strides, diagonal scales fused
 * (Y = diag(row_scale) * A * diag(col_scale) * X, NULL = ones); accumulate = 0
 * overwrites Y (the reference always accumulates). */
tcc_status tcc_swtcf_spmm_ex(const tcc_swtcf* m, const float* X, uint64_t ldx, float* Y,
                             uint64_t ldy, uint32_t F, uint32_t tc_threshold,
                             const float* row_scale, const float* col_scale, int accumulate,
                             cudaStream_t stream);
/* Transposed pass over the same tiles: Z[numSrc x F] = diag(col_scale) * A^T *
 * diag(row_scale) * G[numDst x F].  Owner-computes per column window: each
 * output row is written once, except rows of windows with more than 32 tiles,
 * which several warps reduce into. */
tcc_status tcc_swtcf_spmm_t(const tcc_swtcf* m, const float* G, uint64_t ldg, float* Z,
                            uint64_t ldz, uint32_t F, uint32_t tc_threshold,
                            const float* row_scale, const float* col_scale, int accumulate,
                            cudaStream_t stream);

/* -------------------------------------------------------- BCSR / BCSC ---- */
/* Field-for-field BCSR<float> (cnic/include/class.h:20-37). */
typedef struct tcc_bcsr {
    uint32_t num_rows, num_cols, nnz, num_TCBlocks, num_rowWindows;
    uint32_t* rowWindowOffset; /* [num_rowWindows+1] */
    uint32_t* tcOffset;        /* [num_TCBlocks+1] prefix of tile popcounts */
    uint32_t* sparseA2B;       /* [8*num_TCBlocks] condensed columns, pad 0xFFFFFFFF */
    uint64_t* tcLocalBit;      /* [num_TCBlocks] bit = row*8 + k */
} tcc_bcsr;

/* Field-for-field BCSC<float> (cnic/include/class.h:39-57). */
typedef struct tcc_bcsc {
    uint32_t num_rows, num_cols, nnz, num_TCBlocks, num_colWindows;
    uint32_t* colWindowOffset; /* [num_colWindows+1] */
    uint32_t* tcOffset;        /* [num_TCBlocks+1] */
    uint32_t* sparseA2C;       /* [8*num_TCBlocks] condensed rows, pad 0xFFFFFFFF */
    uint64_t* tcLocalBit;      /* [num_TCBlocks] bit = n*8 + k */
} tcc_bcsc;

typedef struct tcc_tiles_workspace tcc_tiles_workspace; /* opaque */

#define TCC_TILES_BCSR 0
#define TCC_TILES_BCSC 1

/* CSR -> BCSR / BCSC window tiling on the GPU (the producer the reference
 * leaves to its absent sampler, train/tcgnn_conv_release.py:284-301), two steps:
 * prepare (sort + group; synchronises to return the tile count T) then fill
 * the caller's arrays (sized from T). */
tcc_status tcc_tiles_workspace_create(tcc_tiles_workspace** ws, uint64_t nnz_capacity,
                                      uint32_t rows, uint32_t cols);
tcc_status tcc_tiles_workspace_destroy(tcc_tiles_workspace* ws);
tcc_status tcc_tiles_prepare_csr(tcc_tiles_workspace* ws, int kind, const uint64_t* d_rowptr,
                                 const uint32_t* d_col, uint32_t rows, uint32_t cols,
                                 uint64_t nnz, cudaStream_t stream, uint64_t* num_tiles);
tcc_status tcc_tiles_fill_bcsr(tcc_tiles_workspace* ws, tcc_bcsr* out, cudaStream_t stream);
tcc_status tcc_tiles_fill_bcsc(tcc_tiles_workspace* ws, tcc_bcsc* out, cudaStream_t stream);

/* Pull-SpMM scratch (the window->chunk work plan): bytes needed for a tiling
 * with `num_windows` windows and `num_tiles` tiles.  The scratch belongs to the
 * caller; pass plan_ready = 1 to reuse a plan built by an earlier call on the
 * same tiling. */
size_t tcc_pull_scratch_bytes(uint32_t num_windows, uint32_t num_tiles);
/* No counterpart in the reference (its kernels have no bounded waits).  The
 * pull scratch also holds a device error word: TCC_DEVERR_WAIT_TIMEOUT when a
 * pull kernel gave up waiting for one of its TMA copies.  Synchronises
 * `stream`, stores the word in *code and clears it.  The word is also cleared
 * whenever a call builds the plan (plan_ready = 0). */
tcc_status tcc_pull_device_error(void* scratch, int* code, cudaStream_t stream);

/* No counterpart in the reference.  The pull SpMM kernels run one persistent
 * wave of blocks that fills every SM, so a kernel launched on another stream
 * while they run (the NCCL kernels of the halo exchange) cannot become
 * resident until they finish.  Pull kernels launched after
 * tcc_set_grid_reserve(n) size their grids for all SMs but n, leaving room
 * for such kernels; 0 restores full grids.  Process-wide setting. */
void tcc_set_grid_reserve(uint32_t sms);
uint32_t tcc_get_grid_reserve(void);

/* No counterpart in the reference (its kernels have no bounded waits).  Every
 * mbarrier wait of the bulk-copy pull kernel gives up after this many
 * nanoseconds, records TCC_DEVERR_WAIT_TIMEOUT in the pull scratch's error
 * word (tcc_pull_device_error), waits for its own copies still in flight and
 * returns, leaving the context usable.  Process-wide; applies to launches made
 * after the call; 0 restores the default.  Limits below 200 us poll the
 * barrier without suspending; limits below 1 us make every wait a single test
 * of the barrier (a wait whose copy has not landed gives up at once). */
#define TCC_DEFAULT_WAIT_LIMIT_NS 2000000000ull
void tcc_set_wait_limit_ns(uint64_t ns);
uint64_t tcc_get_wait_limit_ns(void);

/* No counterpart in the reference, whose multi-GPU path reads peer feature
 * caches inside the SpMM kernel (cnic/src/core/spmm_kernel.cu:145-147).  Packs
 * the rows a rank sends in the halo exchange of the row-partitioned SpMM:
 * out[i, :F] = X[idx[i], :F] for i < n (int64 indices, F and both row
 * strides multiples of 4, X and out 16-byte aligned).  An index outside
 * [0, num_rows) writes a zero row and sets the device word *bad_flag (may be
 * NULL). */
tcc_status tcc_gather_rows(const float* X, uint64_t ldx, uint64_t num_rows, const int64_t* idx,
                           uint64_t n, float* out, uint64_t ldo, uint32_t F, uint32_t* bad_flag,
                           cudaStream_t stream);

/* The hidden-layer epilogue of the GCN (train/tcgnn_conv_release.py:229-240:
 * relu, then F.dropout with probability p, as separate torch ops there), fused
 * into one pass: out[i] = in[i] > 0 && kept(seed, i) ? in[i] / (1 - p) : 0.
 * kept(seed, i) is a counter-based draw (SplitMix64 finaliser of
 * seed + (i + 1) * 0x9E3779B97F4A7C15; kept when its top 32 bits are >=
 * ceil(p * 2^32)), so no mask is stored: the backward reads the forward's
 * output, grad_in[i] = out[i] > 0 ? grad_out[i] / (1 - p) : 0.  n a multiple
 * of 4, buffers 16-byte aligned, 0 <= p < 1; in == out is allowed. */
tcc_status tcc_relu_dropout_forward(const float* in, float* out, uint64_t n, float p,
                                    uint64_t seed, cudaStream_t stream);
tcc_status tcc_relu_dropout_backward(const float* grad_out, const float* out, float* grad_in,
                                     uint64_t n, float p, cudaStream_t stream);

/* No counterpart in the reference.  The other half of the row-partitioned
 * transposed SpMM's exchange: a rank computes partial rows of A^T.G for the
 * remote columns its rows reference and returns them to their owners, who add
 * them in: out[idx[i], :F] += in[i, :F] for i < n (idx may repeat; vector fp32
 * reductions, so the order of additions is not fixed).  An index outside
 * [0, num_rows) is skipped and sets the device word *bad_flag (may be NULL).
 * F and the strides multiples of 4, in and out 16-byte aligned. */
tcc_status tcc_scatter_add_rows(const float* in, uint64_t ldi, const int64_t* idx, uint64_t n,
                                float* out, uint64_t ldo, uint64_t num_rows, uint32_t F,
                                uint32_t* bad_flag, cudaStream_t stream);

/* ------------------------------------------- halo exchange over NVLink ---- */
/* No counterpart in the reference, whose multi-GPU path reads peer feature
 * caches inside the SpMM kernel (cnic/src/core/spmm_kernel.cu:145-147).  The
 * row-partitioned SpMM's halo exchange through peer memory, one process per
 * GPU of one box: each rank allocates its receive buffers and one flag block
 * with tcc_peer_alloc, the ranks swap the IPC handles (any host channel) and
 * map each other's with tcc_peer_open.  Per exchange (tag t, step number s,
 * counted the same on every rank, starting at 1):
 *   sender:   tcc_halo_push -- once the receivers released the step that
 *             last used the buffer, gathers its rows and stores them into the
 *             receivers' buffers over NVLink, then marks them arrived;
 *   receiver: tcc_halo_wait -- the stream continues once every sender's rows
 *             of step s arrived; the kernels after it read the buffer;
 *             tcc_halo_release after the last of them -- the senders may
 *             overwrite the buffer with step s + 1.
 * Every wait is bounded by wait_ns (%globaltimer); on expiry the kernel
 * records TCC_DEVERR_WAIT_TIMEOUT in the flag block, writes no rows, and
 * returns.  Read the word with tcc_peer_device_error (synchronises).  No
 * multicast is involved. */
#define TCC_PEER_MAX_RANKS 8
#define TCC_PEER_MAX_TAGS 4
#define TCC_PEER_FLAGS_BYTES 4096
typedef struct tcc_ipc_handle {
    unsigned char bytes[64]; /* a cudaIpcMemHandle_t */
} tcc_ipc_handle;

/* cudaMalloc + zero fill + cudaIpcGetMemHandle (synchronises). */
tcc_status tcc_peer_alloc(size_t bytes, void** ptr, tcc_ipc_handle* handle);
/* Map another process's tcc_peer_alloc buffer into this one (peer access
 * enabled lazily); tcc_peer_close unmaps it, tcc_peer_free frees one's own
 * (after every peer closed its mapping). */
tcc_status tcc_peer_open(const tcc_ipc_handle* handle, void** ptr);
tcc_status tcc_peer_close(void* mapped);
tcc_status tcc_peer_free(void* ptr);

typedef struct tcc_halo_push_args {
    const float* x;          /* this rank's rows [num_rows x width], stride ldx */
    uint64_t ldx, num_rows;
    const int64_t* send_idx; /* rows to send, grouped by receiver */
    uint32_t width, world, rank, tag, seq;
    uint32_t max_blocks;     /* grid cap, CTAs of 512 threads (0: 4 per SM); one CTA per SM
                                the concurrent kernels leave free is the intended use */
    uint32_t buffers;        /* receive buffers each receiver rotates through for this tag
                                (step s in buffer (s-1) % buffers; 0 means 1): the push
                                waits for the receivers' release of step seq - buffers */
    uint64_t seg[TCC_PEER_MAX_RANKS + 1]; /* send_idx[seg[p]:seg[p+1]] go to rank p */
    float* dst[TCC_PEER_MAX_RANKS];       /* rank p's receive rows for this rank (mapped) */
    uint64_t ld_dst;                      /* their row stride (floats) */
    void* peer_flags[TCC_PEER_MAX_RANKS]; /* rank p's flag block (mapped) */
    void* flags;                          /* this rank's flag block */
    uint64_t wait_ns;                     /* bound of the wait for step seq-1's release */
} tcc_halo_push_args;

tcc_status tcc_halo_push(const tcc_halo_push_args* args, cudaStream_t stream);
/* peer_mask: bit p set when rank p sends rows to this rank. */
tcc_status tcc_halo_wait(void* flags, uint32_t tag, uint32_t seq, uint32_t peer_mask,
                         uint64_t wait_ns, cudaStream_t stream);
/* peer_flags[p]: rank p's mapped flag block; peer_mask: the senders. */
tcc_status tcc_halo_release(void* const* peer_flags, uint32_t world, uint32_t rank, uint32_t tag,
                            uint32_t seq, uint32_t peer_mask, cudaStream_t stream);
/* The flag block's device error word (TCC_DEVERR_*; synchronises `stream`). */
tcc_status tcc_peer_device_error(void* flags, int* code, cudaStream_t stream);

/* One step of the row-partitioned SpMM on this rank, enqueued by the library:
 * for each operand (one, or two pipelined -- a training step's forward and
 * backward), push the rows the peers need (on `side`), then on `main` the
 * local-column tiles of every operand, then per operand the arrival wait, the
 * halo-column tiles (accumulated) and the release.  Y = diag(rs) A_loc
 * diag(cs_local) X + diag(rs) A_halo diag(cs_halo) X_halo.  `side` first waits
 * for `main`, and `main` ends waiting for `side` (the pushes read X).  No
 * reference counterpart (the reference's kernels load peer caches in place,
 * cnic/src/core/spmm_kernel.cu:145-147); this is the C++ form of
 * tcc_b200.partition.DistGraph.spmm_pair with the peer transport. */
typedef struct tcc_dist_operand {
    tcc_halo_push_args push; /* push.x = this rank's rows of the operand; push.seq = the step */
    const float* halo;       /* this rank's receive rows of step push.seq (its own buffer) */
    uint64_t ld_halo;
    float* y;                /* output rows [local rows x push.width] */
    uint64_t ldy;
} tcc_dist_operand;

typedef struct tcc_dist_step_args {
    const tcc_bcsr* local;   /* local-column tiles (columns remapped to this rank's rows) */
    void* local_scratch;     /* their pull scratch (tcc_pull_scratch_bytes) */
    size_t local_scratch_bytes;
    int32_t local_plan_ready;
    const tcc_bcsr* halo;    /* halo-column tiles, NULL when the rank has no halo */
    void* halo_scratch;
    size_t halo_scratch_bytes;
    int32_t halo_plan_ready;
    const float* rs;         /* row scale of the local rows, or NULL */
    const float* cs_local;   /* column scale of the local columns, or NULL */
    const float* cs_halo;    /* column scale of the halo columns, or NULL */
    uint32_t tc_threshold;
    uint32_t recv_mask;      /* bit p: rank p sends rows to this rank */
    uint32_t reserve_sms;    /* SMs left to the pushes during the passes in reserve_passes */
    uint32_t reserve_passes; /* bit 0/1: local pass of operand 0/1; bit 2/3: halo pass */
    void* peer_flags[TCC_PEER_MAX_RANKS]; /* rank p's mapped flag block (for the release) */
    uint32_t n_ops;          /* 1 or 2 */
    tcc_dist_operand ops[2];
    cudaEvent_t events[6];   /* optional, NULL to skip: [0,1] pushes done (side), [2,3]
                                local passes done, [4,5] operands done (main) */
} tcc_dist_step_args;

tcc_status tcc_dist_step(const tcc_dist_step_args* args, cudaStream_t main, cudaStream_t side);

/* tf32_spmm_bcsr + tf32_computeX128TransposePipe2_BCSR
 * (cnic/src/core/spmm_dispatcher.cu:166-233, spmm_kernel.cu:1560-1843):
 * C[num_rows x F] = diag(rs) * A * diag(cs) * B[num_cols x F]; row windows own
 * their outputs (no atomics except for windows split across warps). */
tcc_status tcc_bcsr_spmm(const tcc_bcsr* a, const float* B, uint64_t ldb, float* C,
                         uint64_t ldc, uint32_t F, uint32_t tc_threshold, const float* rs,
                         const float* cs, int accumulate, void* scratch, size_t scratch_bytes,
                         int plan_ready, cudaStream_t stream);
/* No counterpart in the reference.  tcc_bcsr_spmm for callers that cannot
 * allocate device memory -- code that runs where cudaMalloc is not allowed
 * (inside a host-side memory pool's or allocator's own callbacks, plug-ins of
 * hosts that own all device memory, pre-planned real-time loops that forbid
 * allocation after start-up).  Same arguments and result as tcc_bcsr_spmm with
 * accumulate/scales, but the work plan lives in a scratch array built into
 * this library (TCC_NOALLOC_SCRATCH_BYTES per GPU, held by every GPU that loads
 * the library until exit) instead of caller scratch; nothing is allocated.
 *  - Tilings whose plan exceeds TCC_NOALLOC_SCRATCH_BYTES are rejected with
 *    TCC_ERR_CAPACITY (about 24 bytes per window plus 2 per tile plus 1.1 MB,
 *    tcc_pull_scratch_bytes: e.g. 300 K windows and 3.8 M tiles fit).
 *  - The first call on each device looks up the array's device address
 *    (cudaGetSymbolAddress); make that first call before any stream capture.
 *  - Every call rebuilds the plan in the same array: calls that overlap on the
 *    GPU (other streams, other host threads) race and must be serialised. */
#define TCC_NOALLOC_SCRATCH_BYTES (16u << 20)
tcc_status tcc_bcsr_spmm_noalloc(const tcc_bcsr* a, const float* B, uint64_t ldb, float* C,
                                 uint64_t ldc, uint32_t F, uint32_t tc_threshold, const float* rs,
                                 const float* cs, int accumulate, cudaStream_t stream);
/* No counterpart in the reference.  The device error word of the built-in
 * scratch that tcc_bcsr_spmm_noalloc uses on the current device (the caller
 * has no pointer to pass to tcc_pull_device_error): TCC_DEVERR_WAIT_TIMEOUT
 * when a pull kernel gave up waiting on one of its copies, so that result is
 * incomplete.  Synchronises `stream`, stores the word in *code and clears it.
 * The next tcc_bcsr_spmm_noalloc call also clears it: read it after each call
 * whose result matters.  Allocates nothing. */
tcc_status tcc_noalloc_device_error(int* code, cudaStream_t stream);
/* tf32_spmm_bcsc + tf32_computeX128TransposePipe2_BCSC
 * (cnic/src/core/spmm_dispatcher.cu:235-302, spmm_kernel.cu:1844-2167): the
 * column-window push pass, C += diag(rs) * A * diag(cs) * B, accumulated with
 * vector fp32 reductions (the reference accumulates with atomics too). */
tcc_status tcc_bcsc_spmm(const tcc_bcsc* a, const float* B, uint64_t ldb, float* C,
                         uint64_t ldc, uint32_t F, uint32_t tc_threshold, const float* rs,
                         const float* cs, cudaStream_t stream);
/* The transposed pass over BCSR tiles, as a push: Z[num_cols x F] +=
 * diag(cs) * A^T * diag(rs) * G[num_rows x F] with vector fp32 reductions.  The
 * backward of the BCSR part of a split (BCSR + BCSC) matrix; replaces
 * torch.sparse.mm(A_topo.T, d_output) of train/tcgnn_conv_release.py:150-154 for
 * that part. */
tcc_status tcc_bcsr_spmm_t(const tcc_bcsr* a, const float* G, uint64_t ldg, float* Z,
                           uint64_t ldz, uint32_t F, uint32_t tc_threshold, const float* rs,
                           const float* cs, cudaStream_t stream);
/* The transposed (backward) pass over BCSC tiles: Z[num_cols x F] =
 * diag(cs) * A^T * diag(rs) * G[num_rows x F], owner-computes per column
 * window.  Replaces torch.sparse.mm(A_topo.T, d_output) of
 * train/tcgnn_conv_release.py:150-154. */
tcc_status tcc_bcsc_spmm_t(const tcc_bcsc* a, const float* G, uint64_t ldg, float* Z,
                           uint64_t ldz, uint32_t F, uint32_t tc_threshold, const float* rs,
                           const float* cs, int accumulate, void* scratch,
                           size_t scratch_bytes, int plan_ready, cudaStream_t stream);
/* launch_spmm_kernel, non-mixed (cnic/src/core/spmm_launcher.cu:203-271):
 * C[(num_rowWindows+1)*8 x F] = BCSR*B + BCSC*B (either may be NULL).  The
 * reference memsets C and atomically adds both passes; here the BCSR pass
 * stores and the BCSC pass reduces after it, on one stream.  tc_threshold 0
 * reproduces the reference's TF32-on-every-tile arithmetic. */
tcc_status tcc_cnic_forward(const tcc_bcsr* bcsr, const tcc_bcsc* bcsc, const float* B,
                            float* C, uint32_t F, uint32_t tc_threshold, void* scratch,
                            size_t scratch_bytes, cudaStream_t stream);
/* launch_spmm_kernel, mixed (cnic/src/core/spmm_launcher.cu:115-200,
 * spmm_kernel.cu:129-153): the B row of condensed column c comes from the
 * feature store: g = cache_search_map[c] >= 0 -> gpu_features[g / gpu_capacity]
 * + (g % gpu_capacity) * F (device pointers, an array in device memory); else
 * cpu_features + id_map[c] * F (pinned host memory mapped into the device
 * address space).  Hot rows are read from HBM, cold rows over the host link. */
tcc_status tcc_cnic_forward_mixed(const tcc_bcsr* bcsr, const tcc_bcsc* bcsc,
                                  const int32_t* id_map, const float* cpu_features,
                                  const int32_t* cache_search_map,
                                  const float* const* gpu_features, int64_t gpu_capacity,
                                  float* C, uint32_t F, uint32_t tc_threshold, void* scratch,
                                  size_t scratch_bytes, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* TCC_B200_H */
