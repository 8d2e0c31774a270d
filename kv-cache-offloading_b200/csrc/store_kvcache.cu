// Slot-mapping scatter of fresh K/V rows into the paged cache (the prefill /
// decode store that runs once per layer per step).
//
// Token i's K row (row_bytes, at key + i * key_stride_bytes) goes to
// k_cache + slot * row_bytes, and likewise for V; slot = slot_mapping[i],
// and -1 marks a padded token that is skipped. The copy is a pure byte move,
// so any cache dtype is moved bit-exactly. CTAs of 128 threads stride over the
// tokens; the K and V rows move with the widest unit (16, 8, 4, 2 or 1
// bytes) that every address and stride allows. Offsets are 64-bit. A CTA
// iteration covers kTokens tokens: their slots are loaded first, then every
// thread issues all of its K and V loads before the stores, so each thread
// keeps 2 * kTokens independent loads in flight.
#include <cuda_runtime.h>
#include <stdint.h>

#include "runtime.h"

namespace kvoff {
namespace {

constexpr int kThreads = 128;
constexpr int kTokens = 4;  // tokens per CTA iteration: 8 independent loads per thread

template <typename V>
__global__ void __launch_bounds__(kThreads)
    store_kvcache_kernel(const uint8_t* __restrict__ key, int64_t key_stride,
                         const uint8_t* __restrict__ value, int64_t value_stride,
                         uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
                         int64_t row_bytes, const int32_t* __restrict__ slot_mapping,
                         int64_t num_tokens, int64_t num_slots, int32_t* bad_slots) {
  const int64_t vecs = row_bytes / (int64_t)sizeof(V);
  for (int64_t first = (int64_t)blockIdx.x * kTokens; first < num_tokens;
       first += (int64_t)gridDim.x * kTokens) {
    int64_t slot[kTokens];
#pragma unroll
    for (int t = 0; t < kTokens; ++t) {
      const int64_t i = first + t;
      slot[t] = i < num_tokens ? (int64_t)__ldg(slot_mapping + i) : -1;
      if (slot[t] >= num_slots) {  // out of range: skipped, counted once per token
        if (threadIdx.x == 0 && bad_slots != nullptr) atomicAdd(bad_slots, 1);
        slot[t] = -1;
      }
    }
    for (int64_t j = threadIdx.x; j < vecs; j += kThreads) {
      V k[kTokens], v[kTokens];
#pragma unroll
      for (int t = 0; t < kTokens; ++t) {
        if (slot[t] >= 0) {
          k[t] = __ldg(reinterpret_cast<const V*>(key + (first + t) * key_stride) + j);
          v[t] = __ldg(reinterpret_cast<const V*>(value + (first + t) * value_stride) + j);
        }
      }
#pragma unroll
      for (int t = 0; t < kTokens; ++t) {
        if (slot[t] >= 0) {
          reinterpret_cast<V*>(k_cache + slot[t] * row_bytes)[j] = k[t];
          reinterpret_cast<V*>(v_cache + slot[t] * row_bytes)[j] = v[t];
        }
      }
    }
  }
}

template <typename V>
int launch(const void* key, int64_t ks, const void* value, int64_t vs, void* kc, void* vc,
           int64_t row_bytes, const int32_t* slots, int64_t n, int64_t num_slots, int32_t* bad,
           cudaStream_t stream) {
  const void* kernel = (const void*)store_kvcache_kernel<V>;
  const int64_t grid = grid_for((n + kTokens - 1) / kTokens, kernel, kThreads, 0, 0);
  store_kvcache_kernel<V><<<grid, kThreads, 0, stream>>>(
      static_cast<const uint8_t*>(key), ks, static_cast<const uint8_t*>(value), vs,
      static_cast<uint8_t*>(kc), static_cast<uint8_t*>(vc), row_bytes, slots, n, num_slots, bad);
  return cuda_status(cudaGetLastError(), "store_kvcache launch");
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
