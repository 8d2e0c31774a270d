// Slot-mapping scatter of fresh K/V rows into the paged cache (the prefill /
// decode store that runs once per layer per step).
//
// Token i's K row (row_bytes, at key + i * key_stride_bytes) goes to
// k_cache + slot * row_bytes, and likewise for V; slot = slot_mapping[i],
// and -1 marks a padded token that is skipped. The copy is a pure byte move,
// so any cache dtype is moved bit-exactly. One warp moves one row: row r is
// token r / 2, its K row for even r and its V row for odd r. Each lane issues
// its row loads (the widest unit, 16, 8, 4, 2 or 1 bytes, that every address
// and stride allows) without waiting for the slot, and only the stores wait
// for it. The grid has one CTA per kWarps rows, so the rows of a prefill of a
// few thousand tokens are in flight in one or two waves. Offsets are 64-bit.
//
// The kernel is launched as a programmatic dependent of the previous kernel on
// its stream (cudaLaunchAttributeProgrammaticStreamSerialization). Its CTAs
// may then be scheduled while that kernel's last CTAs drain; each thread's
// first instruction, griddepcontrol.wait, holds it until the previous kernel
// has completed and its writes are visible, so every read of key, value and
// slot_mapping and every cache write still follows it. Each CTA signals
// griddepcontrol.launch_dependents once its rows are issued, so a following
// store launched the same way overlaps this one's tail. Back to back per-layer
// stores (36 in a Qwen3-8B forward) lose less time to launch ramp and drain.
// After a kernel that does not signal, the launch waits for its completion as
// usual.
#include <cuda_runtime.h>
#include <stdint.h>

#include "runtime.h"

namespace kvoff {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kPerLane = 4;  // loads per lane per pass: a warp moves 32 * kPerLane vectors

template <typename V>
__global__ void __launch_bounds__(kThreads)
    store_kvcache_kernel(const uint8_t* __restrict__ key, int64_t key_stride,
                         const uint8_t* __restrict__ value, int64_t value_stride,
                         uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
                         int64_t row_bytes, const int32_t* __restrict__ slot_mapping,
                         int64_t num_tokens, int64_t num_slots, int32_t* bad_slots) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t vecs = row_bytes / (int64_t)sizeof(V);
  const int lane = threadIdx.x & 31;
  const int64_t rows = 2 * num_tokens;
  for (int64_t r = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); r < rows;
       r += (int64_t)gridDim.x * kWarps) {
    const int64_t token = r >> 1;
    const bool is_v = (r & 1) != 0;
    const V* src = reinterpret_cast<const V*>(is_v ? value + token * value_stride
                                                   : key + token * key_stride);
    const int64_t slot = (int64_t)__ldg(slot_mapping + token);
    for (int64_t base = 0; base < vecs; base += 32 * kPerLane) {
      V v[kPerLane];
#pragma unroll
      for (int k = 0; k < kPerLane; ++k) {
        const int64_t j = base + k * 32 + lane;
        if (j < vecs) v[k] = __ldg(src + j);
      }
      if (slot >= 0 && slot < num_slots) {
        V* dst = reinterpret_cast<V*>((is_v ? v_cache : k_cache) + slot * row_bytes);
#pragma unroll
        for (int k = 0; k < kPerLane; ++k) {
          const int64_t j = base + k * 32 + lane;
          if (j < vecs) dst[j] = v[k];
        }
      }
    }
    if (!is_v && lane == 0 && slot >= num_slots && bad_slots != nullptr)
      atomicAdd(bad_slots, 1);  // out of range: skipped, counted once per token
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename V>
int launch(const void* key, int64_t ks, const void* value, int64_t vs, void* kc, void* vc,
           int64_t row_bytes, const int32_t* slots, int64_t n, int64_t num_slots, int32_t* bad,
           cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)streaming_grid(2 * n, kWarps, 0));
  cfg.blockDim = dim3(kThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(
      cudaLaunchKernelEx(&cfg, store_kvcache_kernel<V>, static_cast<const uint8_t*>(key), ks,
                         static_cast<const uint8_t*>(value), vs, static_cast<uint8_t*>(kc),
                         static_cast<uint8_t*>(vc), row_bytes, slots, n, num_slots, bad),
      "store_kvcache launch");
}

}  // namespace
}  // namespace kvoff

using namespace kvoff;

extern "C" int kvoff_store_kvcache(const void* key, int64_t key_stride_bytes, const void* value,
                                   int64_t value_stride_bytes, void* k_cache, void* v_cache,
                                   int64_t row_bytes, const int32_t* slot_mapping,
                                   int64_t num_tokens, int64_t num_slots, int32_t* bad_slots,
                                   void* stream) {
  if (injected("store_kvcache")) return KVOFF_EINJECTED;
  if (num_tokens < 0 || row_bytes <= 0 || num_slots < 0 || key_stride_bytes < 0 ||
      value_stride_bytes < 0)
    return fail(KVOFF_EINVAL, "kvoff_store_kvcache: bad sizes");
  if (num_tokens == 0) return ok();
  if (key == nullptr || value == nullptr || k_cache == nullptr || v_cache == nullptr ||
      slot_mapping == nullptr)
    return fail(KVOFF_EINVAL, "kvoff_store_kvcache: null pointer");
  // Widest unit dividing every base address, row stride and the row length.
  uintptr_t bits = reinterpret_cast<uintptr_t>(key) | reinterpret_cast<uintptr_t>(value) |
                   reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
                   (uintptr_t)key_stride_bytes | (uintptr_t)value_stride_bytes |
                   (uintptr_t)row_bytes;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc;
  if ((bits & 15u) == 0)
    rc = launch<uint4>(key, key_stride_bytes, value, value_stride_bytes, k_cache, v_cache,
                       row_bytes, slot_mapping, num_tokens, num_slots, bad_slots, s);
  else if ((bits & 7u) == 0)
    rc = launch<uint2>(key, key_stride_bytes, value, value_stride_bytes, k_cache, v_cache,
                       row_bytes, slot_mapping, num_tokens, num_slots, bad_slots, s);
  else if ((bits & 3u) == 0)
    rc = launch<uint32_t>(key, key_stride_bytes, value, value_stride_bytes, k_cache, v_cache,
                          row_bytes, slot_mapping, num_tokens, num_slots, bad_slots, s);
  else if ((bits & 1u) == 0)
    rc = launch<uint16_t>(key, key_stride_bytes, value, value_stride_bytes, k_cache, v_cache,
                          row_bytes, slot_mapping, num_tokens, num_slots, bad_slots, s);
  else
    rc = launch<uint8_t>(key, key_stride_bytes, value, value_stride_bytes, k_cache, v_cache,
                         row_bytes, slot_mapping, num_tokens, num_slots, bad_slots, s);
  if (rc != KVOFF_OK) return rc;
  return ok();
}
