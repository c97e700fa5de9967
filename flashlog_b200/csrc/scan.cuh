// scan.cuh -- device-wide exclusive scan (out has n + 1 entries; out[n] = total).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

namespace fl {
size_t scan_workspace(int64_t n);
template <typename In>
int exclusive_scan(const In *in, int64_t n, int64_t *out, void *ws, size_t ws_bytes, cudaStream_t st);
}  // namespace fl
