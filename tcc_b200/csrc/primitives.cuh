// primitives.cuh -- device-wide integer building blocks of the converter:
// exclusive scan and a stable LSD radix sort of (u64 key, u32 value) pairs.
// Deterministic: results depend only on the input, never on scheduling.
#pragma once

#include "common.cuh"

namespace tcc {

// Exclusive prefix sum out[i] = sum(in[0..i)); optional device total.
// `tmp` must hold scan_tmp_bytes(n).  in == out is allowed.
size_t scan_tmp_bytes(uint64_t n);
template <typename T>
void exclusive_scan(const T* in, T* out, uint64_t n, T* d_total, void* tmp, cudaStream_t s);

// Stable LSD radix sort over key bits [first_bit, key_bits), 8 bits per pass
// (first_bit > 0 when the input is already ordered by the bits below it:
// the stable passes over the higher bits keep that order).  Ping-pongs between
// (keys, vals) and (keys_alt, vals_alt); returns true when the sorted result
// ends up in the *_alt buffers.  n < 2^31.
size_t radix_tmp_bytes(uint64_t n);
bool radix_sort_pairs(uint64_t* keys, uint32_t* vals, uint64_t* keys_alt, uint32_t* vals_alt,
                      uint64_t n, int key_bits, void* tmp, cudaStream_t s, int first_bit = 0);

inline int bits_for(uint64_t max_value_exclusive) {
    int b = 0;
    while (b < 64 && (1ull << b) < max_value_exclusive) ++b;
    return b;
}

}  // namespace tcc
