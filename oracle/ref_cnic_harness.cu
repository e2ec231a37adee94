// ref_cnic_harness.cu -- TEST INFRASTRUCTURE ONLY.
//
// A C-ABI shim around the UNMODIFIED reference spmm_cnic host dispatch and
// kernels (TAC_training_backend/spmm_cnic/src/core/spmm_dispatcher.cu,
// spmm_kernel.cu, class.cu), built from the reference sources by
// oracle/Makefile into oracle/_ref/libtcc_ref.so.  It reproduces the
// non-mixed launch sequence of launch_spmm_kernel (spmm_launcher.cu:203-271):
// memset C, tf32_spmm_bcsr on one stream, tf32_spmm_bcsc on another, both
// accumulating into the same C.
//
// Input hygiene (so the reference kernels stay in bounds): the kernels read
// tcLocalBit[start] and sparseA2X[8*start .. +7] of a window even when the
// window has no tile (spmm_kernel.cu:1629-1660, :1922-1930), so this shim
// uploads one extra padding tile; C is sized (numRowWindows+1)*8*F as the
// reference does (spmm_launcher.cu:231); F must be a multiple of 32, <= 512
// (spmm_dispatcher.cu:199-201) and every window count must be non-zero.
#include "class.h"
#include "spmm_dispatcher.h"

#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <vector>

namespace {
thread_local char g_msg[512];

#define C_CHECK(call)                                                            \
    do {                                                                         \
        cudaError_t e_ = (call);                                                 \
        if (e_ != cudaSuccess) {                                                 \
            std::snprintf(g_msg, sizeof(g_msg), "%s", cudaGetErrorString(e_));   \
            throw std::runtime_error(g_msg);                                     \
        }                                                                        \
    } while (0)

template <typename T>
T* upload_padded(const T* host, std::size_t n, std::size_t pad, T fill) {
    std::vector<T> tmp(n + pad, fill);
    if (n) std::memcpy(tmp.data(), host, n * sizeof(T));
    T* dev = nullptr;
    C_CHECK(cudaMalloc(&dev, tmp.size() * sizeof(T)));
    C_CHECK(cudaMemcpy(dev, tmp.data(), tmp.size() * sizeof(T), cudaMemcpyHostToDevice));
    return dev;
}
}  // namespace

extern "C" {

const char* ref_cnic_last_error(void) { return g_msg; }

// C (rows_c x F, host) = BCSR(A1) * B + BCSC(A2) * B with the reference kernels.
// Either part may be skipped by passing num windows = 0.  B is num_cols x F.
int ref_cnic_spmm(uint32_t num_rows, uint32_t num_cols, uint32_t F,
                  uint32_t bcsr_windows, uint32_t bcsr_tiles, const uint32_t* rowWindowOffset,
                  const uint32_t* bcsr_tcOffset, const uint32_t* sparseA2B,
                  const uint64_t* bcsr_bits, uint32_t bcsc_windows, uint32_t bcsc_tiles,
                  const uint32_t* colWindowOffset, const uint32_t* bcsc_tcOffset,
                  const uint32_t* sparseA2C, const uint64_t* bcsc_bits, const float* B,
                  float* C, uint32_t rows_c, int warmup, int reps, float* ms_per_call) {
    g_msg[0] = 0;
    if (F == 0 || F % 32 != 0 || F > 512) {
        std::snprintf(g_msg, sizeof(g_msg), "F must be a multiple of 32 in [32,512]");
        return -1;
    }
    const uint32_t numRowWindows = (num_rows + 7) / 8;
    std::vector<void*> owned;
    cudaStream_t s1 = nullptr, s2 = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    int rc = 0;
    try {
        C_CHECK(cudaStreamCreate(&s1));
        C_CHECK(cudaStreamCreate(&s2));
        const std::size_t c_elems = (std::size_t)(numRowWindows + 1) * 8 * F;
        float* dC = nullptr;
        C_CHECK(cudaMalloc(&dC, c_elems * sizeof(float)));
        owned.push_back(dC);
        float* dB = upload_padded(B, (std::size_t)num_cols * F, 0, 0.f);
        owned.push_back(dB);
        BCSR<float>* bcsr = nullptr;
        BCSC<float>* bcsc = nullptr;
        if (bcsr_windows) {
            uint32_t* rwo = upload_padded(rowWindowOffset, bcsr_windows + 1, 0, 0u);
            uint32_t* tco = upload_padded(bcsr_tcOffset, bcsr_tiles + 1, 1, 0u);
            uint32_t* a2b = upload_padded(sparseA2B, (std::size_t)bcsr_tiles * 8, 8, 0xFFFFFFFFu);
            uint64_t* bits = upload_padded(bcsr_bits, bcsr_tiles, 1, (uint64_t)0);
            owned.push_back(rwo); owned.push_back(tco); owned.push_back(a2b); owned.push_back(bits);
            bcsr = new BCSR<float>(num_rows, num_cols, 0, bcsr_tiles, bcsr_windows, rwo, tco, a2b, bits);
        }
        if (bcsc_windows) {
            uint32_t* cwo = upload_padded(colWindowOffset, bcsc_windows + 1, 0, 0u);
            uint32_t* tco = upload_padded(bcsc_tcOffset, bcsc_tiles + 1, 1, 0u);
            uint32_t* a2c = upload_padded(sparseA2C, (std::size_t)bcsc_tiles * 8, 8, 0xFFFFFFFFu);
            uint64_t* bits = upload_padded(bcsc_bits, bcsc_tiles, 1, (uint64_t)0);
            owned.push_back(cwo); owned.push_back(tco); owned.push_back(a2c); owned.push_back(bits);
            bcsc = new BCSC<float>(num_rows, num_cols, 0, bcsc_tiles, bcsc_windows, cwo, tco, a2c, bits);
        }
        auto run = [&]() {
            C_CHECK(cudaMemsetAsync(dC, 0, c_elems * sizeof(float), s1));
            C_CHECK(cudaStreamSynchronize(s1));
            if (bcsr) tf32_spmm_bcsr(*bcsr, (int32_t)F, dB, dC, s1);
            if (bcsc) tf32_spmm_bcsc(*bcsc, (int32_t)F, dB, dC, s2);
            C_CHECK(cudaGetLastError());
            C_CHECK(cudaStreamSynchronize(s1));
            C_CHECK(cudaStreamSynchronize(s2));
        };
        if (ms_per_call) {
            for (int i = 0; i < warmup; ++i) run();
            C_CHECK(cudaEventCreate(&e0));
            C_CHECK(cudaEventCreate(&e1));
            float total = 0.f;
            for (int i = 0; i < reps; ++i) {
                // both streams join s1's events: the kernels alone are timed
                C_CHECK(cudaMemsetAsync(dC, 0, c_elems * sizeof(float), s1));
                C_CHECK(cudaStreamSynchronize(s1));
                C_CHECK(cudaEventRecord(e0, s1));
                C_CHECK(cudaStreamWaitEvent(s2, e0, 0));
                if (bcsr) tf32_spmm_bcsr(*bcsr, (int32_t)F, dB, dC, s1);
                if (bcsc) tf32_spmm_bcsc(*bcsc, (int32_t)F, dB, dC, s2);
                cudaEvent_t j = nullptr;
                C_CHECK(cudaEventCreateWithFlags(&j, cudaEventDisableTiming));
                C_CHECK(cudaEventRecord(j, s2));
                C_CHECK(cudaStreamWaitEvent(s1, j, 0));
                C_CHECK(cudaEventRecord(e1, s1));
                C_CHECK(cudaEventSynchronize(e1));
                cudaEventDestroy(j);
                float ms = 0.f;
                C_CHECK(cudaEventElapsedTime(&ms, e0, e1));
                total += ms;
            }
            *ms_per_call = reps > 0 ? total / reps : 0.f;
        }
        run();
        std::vector<float> full(c_elems);
        C_CHECK(cudaMemcpy(full.data(), dC, c_elems * sizeof(float), cudaMemcpyDeviceToHost));
        const std::size_t keep = (std::size_t)rows_c * F;
        std::memcpy(C, full.data(), (keep < c_elems ? keep : c_elems) * sizeof(float));
        delete bcsr;
        delete bcsc;
    } catch (const std::exception& e) {
        if (!g_msg[0]) std::snprintf(g_msg, sizeof(g_msg), "%s", e.what());
        rc = -1;
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    for (void* p : owned) cudaFree(p);
    if (s1) cudaStreamDestroy(s1);
    if (s2) cudaStreamDestroy(s2);
    return rc;
}

}  // extern "C"
