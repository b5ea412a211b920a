// Internal interface of the stable LSD radix sort (radix_sort.cu).
#pragma once

#include "hx_common.cuh"

namespace hx {

template <typename K>
size_t sort_workspace_bytes(int n);

template <typename K>
int sort_pairs(const K* keys_in, const int* vals_in, K* keys_out, int* vals_out, int n,
               int begin_bit, int end_bit, void* ws, size_t ws_bytes, cudaStream_t stream);

// Number of significant bits of a tile index in [0, num_tiles).
inline int tile_bits(int num_tiles) {
    int b = 0;
    while (b < 31 && (1 << b) < num_tiles) ++b;
    return b;
}

}  // namespace hx
