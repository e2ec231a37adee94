// ref_swtcf_harness.cu -- TEST INFRASTRUCTURE ONLY.
//
// A C-ABI shim around the UNMODIFIED reference SWTCF library
// (src/swtcf_convert.cu, src/swtcf_spmm.cu of the reference project), compiled
// from the reference sources by oracle/Makefile into oracle/_ref/libtcc_ref.so.
// Tests call it on the GPU box to pin the CPU oracle and to compare the CUDA
// path against the reference on identical inputs; bench.py's reference leg may
// time it.  Nothing in the product links it.
//
// Host buffers in, host buffers out: each call uploads, runs the reference entry
// point (allocateDeviceSWTCF / allocateSWTCFConvertWorkspace / convertCOOToSWTCF,
// include/swtcf_convert.cuh:74-78; launchSWTCFSpMM, include/swtcf_spmm.cuh:10-16)
// and downloads (also launchSWTCFSpMMQuantized, include/swtcf_spmm.cuh:18-26).
// Reference exceptions become return code -1 and a message.
#include "swtcf_convert.cuh"
#include "swtcf_spmm.cuh"

#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>
#include <cstdio>
#include <stdexcept>
#include <vector>

namespace {
thread_local char g_msg[512];

int fail(const char* what) {
    std::snprintf(g_msg, sizeof(g_msg), "%s", what);
    return -1;
}

#define H_CHECK(call)                                                            \
    do {                                                                         \
        cudaError_t e_ = (call);                                                 \
        if (e_ != cudaSuccess) { fail(cudaGetErrorString(e_)); throw std::runtime_error(g_msg); } \
    } while (0)

template <typename T>
void download(T* host, const T* dev, std::size_t n) {
    if (n) H_CHECK(cudaMemcpy(host, dev, n * sizeof(T), cudaMemcpyDeviceToHost));
}
}  // namespace

extern "C" {

const char* ref_last_error(void) { return g_msg; }

// Converts on the GPU with the reference converter and downloads T / R-sized
// outputs (caller sizes every array for T, R <= nnz as the reference does).
// *device_error receives the reference's deviceError word (codes 1-4).
int ref_swtcf_convert(uint32_t rows, uint32_t cols, uint32_t S, uint32_t nnz,
                      const uint32_t* dst, const uint32_t* src, uint32_t* colWindowOffset,
                      uint64_t* tileLocalBit, uint32_t* tileRowSlot,
                      uint32_t* superWindowRowOffset, uint32_t* superWindowRows,
                      uint8_t* superWindowRowCacheSlot, uint32_t* superWindowCachedRowSlot,
                      uint8_t* superWindowCachedCount, uint32_t* num_tiles, uint32_t* num_rows,
                      uint32_t* device_error) {
    g_msg[0] = 0;
    DeviceSWTCFMatrix m;
    SWTCFConvertWorkspace ws;
    uint32_t* d_dst = nullptr;
    uint32_t* d_src = nullptr;
    int rc = 0;
    try {
        H_CHECK(cudaMalloc(&d_dst, sizeof(uint32_t) * nnz));
        H_CHECK(cudaMalloc(&d_src, sizeof(uint32_t) * nnz));
        H_CHECK(cudaMemcpy(d_dst, dst, sizeof(uint32_t) * nnz, cudaMemcpyHostToDevice));
        H_CHECK(cudaMemcpy(d_src, src, sizeof(uint32_t) * nnz, cudaMemcpyHostToDevice));
        allocateDeviceSWTCF(m, rows, cols, nnz, S);
        allocateSWTCFConvertWorkspace(ws, nnz, cols, S);
        convertCOOToSWTCF(d_dst, d_src, nnz, m, ws, 0);
        H_CHECK(cudaDeviceSynchronize());
        download(device_error, ws.deviceError, 1);
        const uint32_t W = m.numColWindows, SW = m.numSuperWindows;
        download(colWindowOffset, m.colWindowOffset, W + 1);
        download(superWindowRowOffset, m.superWindowRowOffset, SW + 1);
        const uint32_t T = colWindowOffset[W];
        const uint32_t R = superWindowRowOffset[SW];
        *num_tiles = T;
        *num_rows = R;
        download(tileLocalBit, m.tileLocalBit, T);
        download(tileRowSlot, m.tileRowSlot, (std::size_t)T * 8);
        download(superWindowRows, m.superWindowRows, R);
        download(superWindowRowCacheSlot, m.superWindowRowCacheSlot, R);
        download(superWindowCachedRowSlot, m.superWindowCachedRowSlot, (std::size_t)SW * 32);
        download(superWindowCachedCount, m.superWindowCachedCount, SW);
    } catch (const std::exception& e) {
        if (!g_msg[0]) fail(e.what());
        rc = -1;
    }
    freeSWTCFConvertWorkspace(ws);
    freeDeviceSWTCF(m);
    cudaFree(d_dst);
    cudaFree(d_src);
    return rc;
}

// The reference converter's own throughput instrument
// (src/swtcf_convert_main.cu:376-417): COO uploaded and matrix + workspace
// allocated once, then `warmup` untimed and `reps` timed convertCOOToSWTCF calls
// on the default stream between CUDA events; *ms_per_call = mean.
int ref_swtcf_convert_timed(uint32_t rows, uint32_t cols, uint32_t S, uint32_t nnz,
                            const uint32_t* dst, const uint32_t* src, int warmup, int reps,
                            float* ms_per_call) {
    g_msg[0] = 0;
    DeviceSWTCFMatrix m;
    SWTCFConvertWorkspace ws;
    uint32_t* d_dst = nullptr;
    uint32_t* d_src = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    int rc = 0;
    try {
        H_CHECK(cudaMalloc(&d_dst, sizeof(uint32_t) * nnz));
        H_CHECK(cudaMalloc(&d_src, sizeof(uint32_t) * nnz));
        H_CHECK(cudaMemcpy(d_dst, dst, sizeof(uint32_t) * nnz, cudaMemcpyHostToDevice));
        H_CHECK(cudaMemcpy(d_src, src, sizeof(uint32_t) * nnz, cudaMemcpyHostToDevice));
        allocateDeviceSWTCF(m, rows, cols, nnz, S);
        allocateSWTCFConvertWorkspace(ws, nnz, cols, S);
        for (int i = 0; i < warmup; ++i) convertCOOToSWTCF(d_dst, d_src, nnz, m, ws, 0);
        H_CHECK(cudaDeviceSynchronize());
        H_CHECK(cudaEventCreate(&e0));
        H_CHECK(cudaEventCreate(&e1));
        H_CHECK(cudaEventRecord(e0));
        for (int i = 0; i < reps; ++i) convertCOOToSWTCF(d_dst, d_src, nnz, m, ws, 0);
        H_CHECK(cudaEventRecord(e1));
        H_CHECK(cudaEventSynchronize(e1));
        float ms = 0.f;
        H_CHECK(cudaEventElapsedTime(&ms, e0, e1));
        *ms_per_call = reps > 0 ? ms / reps : 0.f;
    } catch (const std::exception& e) {
        if (!g_msg[0]) fail(e.what());
        rc = -1;
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    freeSWTCFConvertWorkspace(ws);
    freeDeviceSWTCF(m);
    cudaFree(d_dst);
    cudaFree(d_src);
    return rc;
}

// The reference launchSWTCFSpMM on a GIVEN SWTCF tiling (e.g. the canonical
// form), so that its arithmetic can be compared with the oracle's on the same
// tiles: the arrays are uploaded into a reference-allocated DeviceSWTCFMatrix
// (capacity max(T, R)), Y (rows x 128) is zeroed, Y = pattern(A) * X.
int ref_swtcf_spmm_tiles(uint32_t rows, uint32_t cols, uint32_t S, uint32_t T, uint32_t R,
                         const uint32_t* colWindowOffset, const uint64_t* tileLocalBit,
                         const uint32_t* tileRowSlot, const uint32_t* superWindowRowOffset,
                         const uint32_t* superWindowRows, const uint8_t* superWindowRowCacheSlot,
                         const uint32_t* superWindowCachedRowSlot,
                         const uint8_t* superWindowCachedCount, const float* X, float* Y,
                         uint32_t tc_threshold) {
    g_msg[0] = 0;
    DeviceSWTCFMatrix m;
    float* d_x = nullptr;
    float* d_y = nullptr;
    int rc = 0;
    auto up = [](auto* dst, const auto* src, std::size_t n) {
        if (n) H_CHECK(cudaMemcpy(dst, src, n * sizeof(*src), cudaMemcpyHostToDevice));
    };
    try {
        allocateDeviceSWTCF(m, rows, cols, T > R ? (T ? T : 1) : (R ? R : 1), S);
        const uint32_t W = m.numColWindows, SW = m.numSuperWindows;
        up(m.colWindowOffset, colWindowOffset, W + 1);
        up(m.tileLocalBit, tileLocalBit, T);
        up(m.tileRowSlot, tileRowSlot, (std::size_t)T * 8);
        up(m.superWindowRowOffset, superWindowRowOffset, SW + 1);
        up(m.superWindowRows, superWindowRows, R);
        up(m.superWindowRowCacheSlot, superWindowRowCacheSlot, R);
        up(m.superWindowCachedRowSlot, superWindowCachedRowSlot, (std::size_t)SW * 32);
        up(m.superWindowCachedCount, superWindowCachedCount, SW);
        H_CHECK(cudaMalloc(&d_x, sizeof(float) * (std::size_t)cols * 128));
        H_CHECK(cudaMalloc(&d_y, sizeof(float) * (std::size_t)rows * 128));
        H_CHECK(cudaMemcpy(d_x, X, sizeof(float) * (std::size_t)cols * 128, cudaMemcpyHostToDevice));
        H_CHECK(cudaMemset(d_y, 0, sizeof(float) * (std::size_t)rows * 128));
        launchSWTCFSpMM(m, d_x, d_y, tc_threshold, 0);
        H_CHECK(cudaDeviceSynchronize());
        download(Y, d_y, (std::size_t)rows * 128);
    } catch (const std::exception& e) {
        if (!g_msg[0]) fail(e.what());
        rc = -1;
    }
    freeDeviceSWTCF(m);
    cudaFree(d_x);
    cudaFree(d_y);
    return rc;
}

// Reference converter + reference SpMM (F = 128 fixed, src/swtcf_spmm.cu) on
// one COO: Y (rows x 128, zeroed here) = pattern(A) * X (cols x 128).
// If ms_per_launch is non-NULL the SpMM is also timed: `warmup` untimed and
// `reps` timed launches with CUDA events (Y re-zeroed before the result run).
int ref_swtcf_spmm(uint32_t rows, uint32_t cols, uint32_t nnz, const uint32_t* dst,
                   const uint32_t* src, const float* X, float* Y, uint32_t tc_threshold,
                   int warmup, int reps, float* ms_per_launch) {
    g_msg[0] = 0;
    DeviceSWTCFMatrix m;
    SWTCFConvertWorkspace ws;
    uint32_t* d_dst = nullptr;
    uint32_t* d_src = nullptr;
    float* d_x = nullptr;
    float* d_y = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    int rc = 0;
    try {
        H_CHECK(cudaMalloc(&d_dst, sizeof(uint32_t) * nnz));
        H_CHECK(cudaMalloc(&d_src, sizeof(uint32_t) * nnz));
        H_CHECK(cudaMemcpy(d_dst, dst, sizeof(uint32_t) * nnz, cudaMemcpyHostToDevice));
        H_CHECK(cudaMemcpy(d_src, src, sizeof(uint32_t) * nnz, cudaMemcpyHostToDevice));
        allocateDeviceSWTCF(m, rows, cols, nnz, 16);
        allocateSWTCFConvertWorkspace(ws, nnz, cols, 16);
        convertCOOToSWTCF(d_dst, d_src, nnz, m, ws, 0);
        H_CHECK(cudaDeviceSynchronize());
        uint32_t derr = 0;
        download(&derr, ws.deviceError, 1);
        if (derr != 0) {
            std::snprintf(g_msg, sizeof(g_msg), "reference converter device error %u", derr);
            throw std::runtime_error(g_msg);
        }
        const std::size_t xe = (std::size_t)cols * 128, ye = (std::size_t)rows * 128;
        H_CHECK(cudaMalloc(&d_x, xe * sizeof(float)));
        H_CHECK(cudaMalloc(&d_y, ye * sizeof(float)));
        H_CHECK(cudaMemcpy(d_x, X, xe * sizeof(float), cudaMemcpyHostToDevice));
        if (ms_per_launch) {
            H_CHECK(cudaMemset(d_y, 0, ye * sizeof(float)));
            for (int i = 0; i < warmup; ++i) launchSWTCFSpMM(m, d_x, d_y, tc_threshold, 0);
            H_CHECK(cudaEventCreate(&e0));
            H_CHECK(cudaEventCreate(&e1));
            H_CHECK(cudaEventRecord(e0));
            for (int i = 0; i < reps; ++i) launchSWTCFSpMM(m, d_x, d_y, tc_threshold, 0);
            H_CHECK(cudaEventRecord(e1));
            H_CHECK(cudaEventSynchronize(e1));
            float ms = 0.f;
            H_CHECK(cudaEventElapsedTime(&ms, e0, e1));
            *ms_per_launch = reps > 0 ? ms / reps : 0.f;
        }
        H_CHECK(cudaMemset(d_y, 0, ye * sizeof(float)));
        launchSWTCFSpMM(m, d_x, d_y, tc_threshold, 0);
        H_CHECK(cudaGetLastError());
        H_CHECK(cudaDeviceSynchronize());
        download(Y, d_y, ye);
    } catch (const std::exception& e) {
        if (!g_msg[0]) fail(e.what());
        rc = -1;
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    freeSWTCFConvertWorkspace(ws);
    freeDeviceSWTCF(m);
    cudaFree(d_dst);
    cudaFree(d_src);
    cudaFree(d_x);
    cudaFree(d_y);
    return rc;
}

// Reference convert + launchSWTCFSpMMQuantized (include/swtcf_spmm.cuh:18-26):
// q_x [n_global x 128] int8, scales [n_global], src_global [cols]; Y zeroed first.
int ref_swtcf_spmm_quantized(uint32_t rows, uint32_t cols, uint32_t nnz, const uint32_t* dst,
                             const uint32_t* src, const int8_t* q_x, const float* scales,
                             uint32_t n_global, const uint32_t* src_global, float* Y,
                             uint32_t tc_threshold) {
    g_msg[0] = 0;
    DeviceSWTCFMatrix m;
    SWTCFConvertWorkspace ws;
    uint32_t* d_dst = nullptr;
    uint32_t* d_src = nullptr;
    int8_t* d_q = nullptr;
    float* d_s = nullptr;
    uint32_t* d_g = nullptr;
    float* d_y = nullptr;
    int rc = 0;
    try {
        H_CHECK(cudaMalloc(&d_dst, sizeof(uint32_t) * nnz));
        H_CHECK(cudaMalloc(&d_src, sizeof(uint32_t) * nnz));
        H_CHECK(cudaMemcpy(d_dst, dst, sizeof(uint32_t) * nnz, cudaMemcpyHostToDevice));
        H_CHECK(cudaMemcpy(d_src, src, sizeof(uint32_t) * nnz, cudaMemcpyHostToDevice));
        allocateDeviceSWTCF(m, rows, cols, nnz, 16);
        allocateSWTCFConvertWorkspace(ws, nnz, cols, 16);
        convertCOOToSWTCF(d_dst, d_src, nnz, m, ws, 0);
        H_CHECK(cudaDeviceSynchronize());
        uint32_t derr = 0;
        download(&derr, ws.deviceError, 1);
        if (derr != 0) {
            std::snprintf(g_msg, sizeof(g_msg), "reference converter device error %u", derr);
            throw std::runtime_error(g_msg);
        }
        const std::size_t qe = (std::size_t)n_global * 128, ye = (std::size_t)rows * 128;
        H_CHECK(cudaMalloc(&d_q, qe));
        H_CHECK(cudaMalloc(&d_s, sizeof(float) * n_global));
        H_CHECK(cudaMalloc(&d_g, sizeof(uint32_t) * cols));
        H_CHECK(cudaMalloc(&d_y, ye * sizeof(float)));
        H_CHECK(cudaMemcpy(d_q, q_x, qe, cudaMemcpyHostToDevice));
        H_CHECK(cudaMemcpy(d_s, scales, sizeof(float) * n_global, cudaMemcpyHostToDevice));
        H_CHECK(cudaMemcpy(d_g, src_global, sizeof(uint32_t) * cols, cudaMemcpyHostToDevice));
        H_CHECK(cudaMemset(d_y, 0, ye * sizeof(float)));
        launchSWTCFSpMMQuantized(m, d_q, d_s, d_g, d_y, tc_threshold, 0);
        H_CHECK(cudaGetLastError());
        H_CHECK(cudaDeviceSynchronize());
        download(Y, d_y, ye);
    } catch (const std::exception& e) {
        if (!g_msg[0]) fail(e.what());
        rc = -1;
    }
    freeSWTCFConvertWorkspace(ws);
    freeDeviceSWTCF(m);
    cudaFree(d_dst);
    cudaFree(d_src);
    cudaFree(d_q);
    cudaFree(d_s);
    cudaFree(d_g);
    cudaFree(d_y);
    return rc;
}

}  // extern "C"
