/*
 * tcc_oracle.h -- CPU restatement of the tcc graph-aggregation path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path in
 * tcc_b200/: it is linked by tests/, by __graft_entry__.smoke() and by the
 * cpu_baseline / reference legs of bench.py, and by nothing that ships.  The
 * product path never calls it and fails loudly when its CUDA library is absent.
 *
 * Every function restates one piece of the reference algorithm and names the
 * reference file:line it follows (paths relative to the reference project root;
 * "cnic/" abbreviates TAC_training_backend/spmm_cnic/).
 *
 * Parity pinning: the layout functions are checked against the reference's own
 * validators (restated below from src/swtcf_convert_main.cu:36-310) and the SpMM
 * against the reference's closed-form known-answer test
 * (src/swtcf_spmm_main.cu:33-112); the GPU test suite additionally runs the
 * reference converter/SpMM (built from source into oracle/_ref/) on the same
 * inputs and compares its canonicalised output with this oracle byte for byte.
 */
#ifndef TCC_ORACLE_H
#define TCC_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes shared with the product's C-ABI (include/tcc_b200.h) */
#define ORC_OK 0
#define ORC_ERR_ARG 1
#define ORC_ERR_DUPLICATE 7   /* duplicate (dst,src) edge: reference error 1 */
#define ORC_ERR_RANGE 8       /* index >= rows/cols */
#define ORC_ERR_CAPACITY 9    /* output buffer too small */
#define ORC_ERR_VALIDATE 10   /* a reference invariant failed */

#define ORC_WINDOW 8u
#define ORC_CACHE 32u
#define ORC_INVALID_SLOT 0xFFFFFFFFu
#define ORC_INVALID_CACHE 0xFFu

/* ---------------------------------------------------------------- SWTCF --- */
/* Canonical COO -> SWTCF conversion (the layout of src/swtcf_convert.cu:1754-2342
 * with the atomic tie-breaks replaced by: rows of a window ordered by degree
 * descending then dst ascending; super-window row slots by dst ascending; cache
 * ranks by occurrence descending then slot ascending).
 * Capacities: tile arrays hold cap_tiles entries (tileRowSlot 8*cap_tiles),
 * row arrays cap_rows entries; the reference sizes both by nnz.
 * On success *num_tiles / *num_rows receive T and R. */
int orc_swtcf_convert(uint32_t rows, uint32_t cols, uint32_t super_window, uint64_t nnz,
                      const uint32_t* dst, const uint32_t* src,
                      uint64_t cap_tiles, uint64_t cap_rows,
                      uint32_t* colWindowOffset,          /* W+1 */
                      uint64_t* tileLocalBit,             /* cap_tiles */
                      uint32_t* tileRowSlot,              /* 8*cap_tiles */
                      uint32_t* superWindowRowOffset,     /* SW+1 */
                      uint32_t* superWindowRows,          /* cap_rows */
                      uint8_t* superWindowRowCacheSlot,   /* cap_rows */
                      uint32_t* superWindowCachedRowSlot, /* 32*SW */
                      uint8_t* superWindowCachedCount,    /* SW */
                      uint64_t* num_tiles, uint64_t* num_rows);

/* The reference's layout validators, restated (src/swtcf_convert_main.cu:36-130
 * validateSWTCF and :132-310 validateRepeatCacheMetadata). Returns ORC_OK or
 * ORC_ERR_VALIDATE; `why` (may be NULL) receives a short reason. */
int orc_swtcf_validate(uint32_t cols, uint32_t super_window, uint64_t nnz,
                       const uint32_t* dst, const uint32_t* src, uint32_t num_col_windows,
                       const uint32_t* colWindowOffset, const uint64_t* tileLocalBit,
                       const uint32_t* tileRowSlot, uint32_t num_super_windows,
                       const uint32_t* superWindowRowOffset, const uint32_t* superWindowRows,
                       const uint8_t* superWindowRowCacheSlot,
                       const uint32_t* superWindowCachedRowSlot,
                       const uint8_t* superWindowCachedCount, char* why, size_t why_len);

/* Bring a reference-converter output (whose row order inside a degree bucket,
 * super-window slot order and cache-rank ties depend on atomic arrival order,
 * src/swtcf_convert.cu:345-349, :615-621, :851-857) into canonical form in place.
 * Arrays are T / R long as in the input. */
int orc_swtcf_canonicalize(uint32_t super_window, uint32_t num_col_windows,
                           const uint32_t* colWindowOffset, uint64_t* tileLocalBit,
                           uint32_t* tileRowSlot, uint32_t num_super_windows,
                           const uint32_t* superWindowRowOffset, uint32_t* superWindowRows,
                           uint8_t* superWindowRowCacheSlot, uint32_t* superWindowCachedRowSlot,
                           uint8_t* superWindowCachedCount);

/* The SWTCF SpMM arithmetic of src/swtcf_spmm.cu:105-265 on the CPU:
 * Y[dst,:] += sum over tiles; a tile whose popcount >= tc_threshold sums
 * tf32(X) (cvt.rna, include/mma_tf32.cuh:17-22) else fp32 X, per tile row in
 * column order.  Y is accumulated (caller zeroes), F columns, row stride ldx/ldy. */
void orc_swtcf_spmm(uint32_t num_col_windows, uint32_t super_window, uint32_t cols,
                    const uint32_t* colWindowOffset, const uint64_t* tileLocalBit,
                    const uint32_t* tileRowSlot, const uint32_t* superWindowRowOffset,
                    const uint32_t* superWindowRows, const float* X, uint32_t F, uint64_t ldx,
                    float* Y, uint64_t ldy, uint32_t tc_threshold);

/* ------------------------------------------------------------ BCSR/BCSC --- */
/* Canonical CSR -> BCSR (cnic/include/class.h:20-37 consumed by
 * cnic/src/core/spmm_kernel.cu:1560-1843): row window r = rows [8r,8r+8), its
 * distinct columns ascending, chunked by 8; sparseA2B padding 0xFFFFFFFF;
 * tcLocalBit bit = i*8+k; tcOffset = prefix of tile popcounts (T+1 entries).
 * Pass NULL outputs to only count: *num_tiles gets T either way. */
int orc_bcsr_from_csr(uint32_t rows, uint32_t cols, const uint64_t* rowptr, const uint32_t* col,
                      uint64_t cap_tiles, uint32_t* rowWindowOffset, uint32_t* tcOffset,
                      uint32_t* sparseA2B, uint64_t* tcLocalBit, uint64_t* num_tiles);

/* Canonical CSR -> BCSC (cnic/include/class.h:39-57 consumed by
 * cnic/src/core/spmm_kernel.cu:1844-2167): column window c = cols [8c,8c+8), its
 * distinct rows ascending chunked by 8; sparseA2C padding 0xFFFFFFFF; bit = n*8+k. */
int orc_bcsc_from_csr(uint32_t rows, uint32_t cols, const uint64_t* rowptr, const uint32_t* col,
                      uint64_t cap_tiles, uint32_t* colWindowOffset, uint32_t* tcOffset,
                      uint32_t* sparseA2C, uint64_t* tcLocalBit, uint64_t* num_tiles);

/* Tile arithmetic of the cnic kernels on the CPU.  bcsr: C[8w+i,:] += sum_k
 * bit(i,k) B[sparseA2B[8t+k],:]; bcsc: C[sparseA2C[8t+n],:] += sum_k bit(n,k)
 * B[8c+k,:].  Tiles with popcount >= tc_threshold use tf32(B) (the reference
 * runs every tile through TF32 mma, cnic/include/ptx_tf32.h:61-83: threshold 0). */
void orc_bcsr_spmm(uint32_t num_windows, uint32_t num_cols, const uint32_t* rowWindowOffset,
                   const uint32_t* sparseA2B, const uint64_t* tcLocalBit, const float* B,
                   uint32_t F, uint64_t ldb, float* C, uint64_t ldc, uint32_t num_rows,
                   uint32_t tc_threshold);
void orc_bcsc_spmm(uint32_t num_windows, uint32_t num_cols, const uint32_t* colWindowOffset,
                   const uint32_t* sparseA2C, const uint64_t* tcLocalBit, const float* B,
                   uint32_t F, uint64_t ldb, float* C, uint64_t ldc, uint32_t num_rows,
                   uint32_t tc_threshold);

/* ------------------------------------------------------------- CSR SpMM --- */
/* Y[r,:] = rs[r] * sum_{c in N(r)} cs[c] * X[c,:], fp64 accumulation, fp32 out.
 * rs / cs may be NULL (1).  accumulate != 0 adds into Y. */
void orc_csr_spmm(uint32_t rows, const uint64_t* rowptr, const uint32_t* col, const float* rs,
                  const float* cs, const float* X, uint32_t F, uint64_t ldx, float* Y,
                  uint64_t ldy, int accumulate);
/* Transposed: Y[c,:] (+)= cs[c] * sum_{r: c in N(r)} rs[r] * X[r,:] for Y with
 * `cols` rows; fp64 accumulation. */
void orc_csr_spmm_t(uint32_t rows, uint32_t cols, const uint64_t* rowptr, const uint32_t* col,
                    const float* rs, const float* cs, const float* X, uint32_t F, uint64_t ldx,
                    float* Y, uint64_t ldy, int accumulate);
/* CPU baseline: fp32 row-parallel CSR SpMM over `threads` OpenMP threads
 * (dynamic schedule, 64 rows per grab); the kernel bench.py times on the host. */
void orc_csr_spmm_f32_omp(uint32_t rows, const uint64_t* rowptr, const uint32_t* col,
                          const float* rs, const float* cs, const float* X, uint32_t F,
                          uint64_t ldx, float* Y, uint64_t ldy, int threads);

/* The reference's closed-form known-answer features (src/swtcf_spmm_main.cu:33-45). */
float orc_kat_feature(uint32_t source, uint32_t feature);

/* Round-to-nearest, ties away from zero, to TF32's 10 explicit mantissa bits:
 * the rounding cvt.rna.tf32.f32 is documented to perform. */
float orc_tf32_rna(float x);

#ifdef __cplusplus
}
#endif
#endif
