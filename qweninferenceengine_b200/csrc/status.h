// status.h -- error reporting shared by the host-side translation units.
#pragma once
#include <cuda_runtime.h>

namespace qwen {
// Records a thread-local message (qwen_last_error) and returns `code`.
int set_error(int code, const char* fmt, ...);
// QWEN_OK for cudaSuccess, else records the CUDA error and maps it to a status.
int cuda_status(cudaError_t e, const char* what);
// cuda_status(cudaGetLastError(), what).
int launch_status(const char* what);
// Uploads the RoPE frequency table to the current device once.
int ensure_rope_table();
}  // namespace qwen

// Early return of a non-OK status (QWEN_OK is 0).
#define QWEN_TRY(expr)                \
  do {                                \
    int _rc = (expr);                 \
    if (_rc != 0) return _rc;         \
  } while (0)
#define QWEN_CUDA(expr, what) QWEN_TRY(::qwen::cuda_status((expr), (what)))
