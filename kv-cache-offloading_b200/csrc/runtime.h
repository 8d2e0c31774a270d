// Internal helpers shared by the libkvoff translation units: per-thread error
// text, host-side fault injection, CUDA status checks and cached device
// properties. Nothing here is part of the public C ABI (include/kvoff.h).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "kvoff.h"

namespace kvoff {

// Records a printf-style message for kvoff_last_error() and returns `code`.
int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));

// Clears the calling thread's error text; returns KVOFF_OK.
int ok();

// True (and error text set) when kvoff_debug_fail_next armed `op`.
bool injected(const char* op);

// Maps a CUDA error to KVOFF_ECUDA with context; KVOFF_OK for cudaSuccess.
int cuda_status(cudaError_t err, const char* what);

// Streaming-multiprocessor count of the current device (cached per device).
int sm_count();

// Resident CTAs per SM for `kernel` at `threads` threads and `smem` bytes of
// dynamic shared memory (cached by kernel pointer and device).
int ctas_per_sm(const void* kernel, int threads, size_t smem);

// Grid size for a persistent grid-stride kernel: min(units, full grid),
// further capped by max_ctas when it is positive.
int64_t grid_for(int64_t units, const void* kernel, int threads, size_t smem, int32_t max_ctas);

// Grid size for a streaming kernel that strides over `units`: one CTA per
// `per_cta` units, capped by max_ctas when it is positive and by the grid.x
// limit. On B200 such an oversubscribed grid of short-lived CTAs keeps HBM
// busier than a persistent grid of resident CTAs.
int64_t streaming_grid(int64_t units, int64_t per_cta, int32_t max_ctas);

}  // namespace kvoff

#define KVOFF_TRY(expr)              \
  do {                               \
    int kvoff_rc_ = (expr);          \
    if (kvoff_rc_ != KVOFF_OK) return kvoff_rc_; \
  } while (0)
