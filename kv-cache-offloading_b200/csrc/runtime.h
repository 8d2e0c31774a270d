// Internal helpers shared by the libkvoff translation units: per-thread error
// text, host-side fault injection, CUDA status checks and cached device
// properties. Nothing here is part of the public C ABI (include/kvoff.h).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

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

// Owning device of `p` when it is device memory, else -1, in *device. The
// answer comes from cudaPointerGetAttributes and is remembered per thread for
// the last few pointers asked about: callers pass the same pool and staging
// buffers on every call, so the driver query stays off the per-block path.
// A remembered answer outlives a free of that buffer; the checks it serves
// only catch a host pointer, or another device's buffer, passed by mistake.
int device_memory_of(const void* p, int* device);

// Copies dst[i] <- src[i] of `bytes` each, for i < n, merged into one
// cudaMemcpyAsync per run of entries that are adjacent on both sides (slots of
// a slab are consecutive, and so is a staging buffer), so a group of blocks
// moves with a handful of DMA operations instead of one per block.
int copy_runs(void* const* dst, void* const* src, int64_t n, int64_t bytes, cudaStream_t s,
              const char* what);

// Two-stage pipeline of the staged calls (FP8 and BF16). The caller's staging
// buffer is split into two halves. Kernels run on an auxiliary stream owned by
// the library (one per device and caller stream), and events hand each half
// back and forth between that stream and the caller's stream, so that the
// kernel of one group overlaps the DMA of the previous group. The ring
// position persists across calls on the same caller stream and staging buffer,
// so back-to-back one-block calls alternate halves and overlap too.
struct Pipe {
  cudaStream_t aux = nullptr;
  cudaEvent_t start = nullptr, done = nullptr;
  cudaEvent_t ready[2] = {nullptr, nullptr};
  cudaEvent_t freed[2] = {nullptr, nullptr};
  bool freed_recorded[2] = {false, false};
  int next = 0;
  const void* staging = nullptr;
};

// Guards every Pipe; hold it from pipe_for until the call has enqueued its work.
std::mutex& pipe_mutex();

// The pipeline of (current device, caller); a new staging buffer starts a
// fresh ring, after `caller` waits for the kernels already queued on the
// pipeline's stream. Creates the stream and events on first use.
int pipe_for(cudaStream_t caller, const void* staging, Pipe** out);

// Makes `caller` wait for everything its pipeline queued on the auxiliary
// stream (no-op without one). Takes pipe_mutex() itself.
int join_pipe(cudaStream_t caller);

// Before a group reuses staging half h, makes `waiter` wait for the last work
// that used half h.
int pipe_wait_half(Pipe* p, int h, cudaStream_t waiter);

// Starts a staged call on `caller`. Returns in *out the pipeline, with `lock`
// (on pipe_mutex()) held, or nullptr when the call runs serially on `caller`
// (a one-block staging buffer).
int pipe_begin(cudaStream_t caller, const void* staging, int64_t staging_blocks,
               std::unique_lock<std::mutex>& lock, Pipe** out);

}  // namespace kvoff

#define KVOFF_TRY(expr)              \
  do {                               \
    int kvoff_rc_ = (expr);          \
    if (kvoff_rc_ != KVOFF_OK) return kvoff_rc_; \
  } while (0)
