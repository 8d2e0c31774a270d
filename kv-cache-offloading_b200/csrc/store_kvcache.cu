// Slot-mapping scatter of fresh K/V rows into the paged cache (the prefill /
// decode store that runs once per layer per step).
//
// Token i's K row (row_bytes, at key + i * key_stride_bytes) goes to
// k_cache + slot * row_bytes, and likewise for V; slot = slot_mapping[i],
// and -1 marks a padded token that is skipped. The copy is a pure byte move,
// so any cache dtype is moved bit-exactly.
//
// A group of T threads moves one token: thread i copies vectors i, i + T, ...
// of the token's K row and of its V row (the widest unit, 16, 8, 4, 2 or 1
// bytes, that every address and stride allows), issuing its loads before the
// slot is known; only the stores wait for it.
//
// * Row kernel (the usual case): rows of exactly 32, 64 or 128 16-byte
//   vectors (512 B to 2 KB: 2 to 8 KV heads of 128 bf16) and offsets that fit
//   in 32 bits. T is the row length, so each thread moves one vector of K and
//   one of V, with no loop and 32-bit address arithmetic; 128-thread CTAs.
// * General kernel: any row length and vector width, 64-bit offsets,
//   256-thread CTAs, T the row's vector count rounded up to a power of two
//   between 32 and 128.
//
// A launch of a few thousand tokens lasts a few microseconds, so its cost is
// mostly launch latency, instruction count and CTA ramp. The row kernel's
// short straight-line code is what brings it level with the reference's
// Triton kernel inside a forward pass (a kernel writing the qkv rows, the
// store, a kernel after it): one warp per row with 64-bit offsets and a
// loop added about 0.15 us per layer there.
//
// Both kernels are plain launches. A programmatic dependent launch
// (griddepcontrol.wait at entry, launch_dependents after the rows) was
// measured and dropped: 36 stores back to back gained 0.55 us per layer, but
// inside a forward pass, where the store follows a kernel that never signals
// early, it cost up to 1 us per layer at 4096 tokens.
#include <cuda_runtime.h>
#include <stdint.h>

#include "runtime.h"

namespace kvoff {
namespace {

constexpr int kThreads = 256;
constexpr int kRowThreads = 128;

// Rows of exactly T 16-byte vectors, offsets below 2^32 bytes.
template <int T>
__global__ void __launch_bounds__(kRowThreads)
    store_kvcache_row_kernel(const uint8_t* __restrict__ key, uint32_t key_stride,
                             const uint8_t* __restrict__ value, uint32_t value_stride,
                             uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
                             const int32_t* __restrict__ slot_mapping, uint32_t num_tokens,
                             int32_t num_slots, int32_t* bad_slots) {
  constexpr uint32_t kTokens = kRowThreads / T;
  const uint32_t token = blockIdx.x * kTokens + threadIdx.x / T;
  const uint32_t i = threadIdx.x % T;
  if (token < num_tokens) {
    const int32_t slot = slot_mapping[token];
    const uint4 k = reinterpret_cast<const uint4*>(key + token * key_stride)[i];
    const uint4 v = reinterpret_cast<const uint4*>(value + token * value_stride)[i];
    if (slot >= 0 && slot < num_slots) {
      const uint32_t row = (uint32_t)slot * (uint32_t)(T * sizeof(uint4));
      reinterpret_cast<uint4*>(k_cache + row)[i] = k;
      reinterpret_cast<uint4*>(v_cache + row)[i] = v;
    } else if (i == 0 && slot >= num_slots && bad_slots != nullptr) {
      atomicAdd(bad_slots, 1);  // out of range: skipped, counted once per token
    }
  }
}

// Any row length and vector width V; T threads per token.
template <typename V, int T>
__global__ void __launch_bounds__(kThreads)
    store_kvcache_kernel(const uint8_t* __restrict__ key, int64_t key_stride,
                         const uint8_t* __restrict__ value, int64_t value_stride,
                         uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
                         int64_t row_bytes, const int32_t* __restrict__ slot_mapping,
                         int64_t num_tokens, int64_t num_slots, int32_t* bad_slots) {
  constexpr int kTokens = kThreads / T;
  const int64_t token = (int64_t)blockIdx.x * kTokens + threadIdx.x / T;
  const int i = threadIdx.x % T;
  if (token < num_tokens) {
    const int64_t vecs = row_bytes / (int64_t)sizeof(V);
    const V* ksrc = reinterpret_cast<const V*>(key + token * key_stride);
    const V* vsrc = reinterpret_cast<const V*>(value + token * value_stride);
    const int64_t slot = (int64_t)__ldg(slot_mapping + token);
    for (int64_t base = 0; base < vecs; base += T) {
      const int64_t j = base + i;
      V k, v;
      if (j < vecs) {
        k = __ldg(ksrc + j);
        v = __ldg(vsrc + j);
      }
      if (j < vecs && slot >= 0 && slot < num_slots) {
        reinterpret_cast<V*>(k_cache + slot * row_bytes)[j] = k;
        reinterpret_cast<V*>(v_cache + slot * row_bytes)[j] = v;
      }
    }
    if (i == 0 && slot >= num_slots && bad_slots != nullptr)
      atomicAdd(bad_slots, 1);  // out of range: skipped, counted once per token
  }
}

template <int T>
int launch_rows(const void* key, int64_t ks, const void* value, int64_t vs, void* kc, void* vc,
                const int32_t* slots, int64_t n, int64_t num_slots, int32_t* bad,
                cudaStream_t stream) {
  constexpr int64_t kTokens = kRowThreads / T;
  store_kvcache_row_kernel<T><<<(n + kTokens - 1) / kTokens, kRowThreads, 0, stream>>>(
      static_cast<const uint8_t*>(key), (uint32_t)ks, static_cast<const uint8_t*>(value),
      (uint32_t)vs, static_cast<uint8_t*>(kc), static_cast<uint8_t*>(vc), slots, (uint32_t)n,
      (int32_t)num_slots, bad);
  return cuda_status(cudaGetLastError(), "store_kvcache launch");
}

template <typename V, int T>
int launch_general(const void* key, int64_t ks, const void* value, int64_t vs, void* kc, void* vc,
                   int64_t row_bytes, const int32_t* slots, int64_t n, int64_t num_slots,
                   int32_t* bad, cudaStream_t stream) {
  constexpr int64_t kTokens = kThreads / T;
  store_kvcache_kernel<V, T><<<(n + kTokens - 1) / kTokens, kThreads, 0, stream>>>(
      static_cast<const uint8_t*>(key), ks, static_cast<const uint8_t*>(value), vs,
      static_cast<uint8_t*>(kc), static_cast<uint8_t*>(vc), row_bytes, slots, n, num_slots, bad);
  return cuda_status(cudaGetLastError(), "store_kvcache launch");
}

template <typename V>
int launch(const void* key, int64_t ks, const void* value, int64_t vs, void* kc, void* vc,
           int64_t row_bytes, const int32_t* slots, int64_t n, int64_t num_slots, int32_t* bad,
           cudaStream_t stream) {
  const int64_t vecs = row_bytes / (int64_t)sizeof(V);
  if (sizeof(V) == 16 && (vecs == 32 || vecs == 64 || vecs == 128)) {
    // Every offset the row kernel forms must fit in 32 bits.
    constexpr int64_t kMax = 0xFFFFFFFFll;
    const int64_t stride = ks > vs ? ks : vs;
    const bool fits = stride <= (kMax - row_bytes) / n && num_slots <= kMax / row_bytes &&
                      num_slots <= 0x7FFFFFFFll;
    if (fits) {
      if (vecs == 128)
        return launch_rows<128>(key, ks, value, vs, kc, vc, slots, n, num_slots, bad, stream);
      if (vecs == 64)
        return launch_rows<64>(key, ks, value, vs, kc, vc, slots, n, num_slots, bad, stream);
      return launch_rows<32>(key, ks, value, vs, kc, vc, slots, n, num_slots, bad, stream);
    }
  }
  if (vecs > 64)
    return launch_general<V, 128>(key, ks, value, vs, kc, vc, row_bytes, slots, n, num_slots, bad,
                                  stream);
  if (vecs > 32)
    return launch_general<V, 64>(key, ks, value, vs, kc, vc, row_bytes, slots, n, num_slots, bad,
                                 stream);
  return launch_general<V, 32>(key, ks, value, vs, kc, vc, row_bytes, slots, n, num_slots, bad,
                               stream);
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
  if (num_tokens > 0x7FFFFFFFll)
    return fail(KVOFF_EINVAL, "kvoff_store_kvcache: %lld tokens exceed one launch",
                (long long)num_tokens);
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
