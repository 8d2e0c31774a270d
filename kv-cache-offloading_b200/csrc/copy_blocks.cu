// Byte-exact KV block passthrough between the paged pool and dense slots.
//
// A block is num_chunks chunks of chunk_bytes, chunk_stride_bytes apart in the
// pool and back to back in the slot. Three movers:
//  * copy engine: one cudaMemcpy2DAsync per block (rows = chunks), the DMA
//    engine walks the pool's stride itself; works for host or device slots;
//  * TMA: one elected thread per CTA streams 32 KiB pieces through a ring of
//    shared-memory stages with cp.async.bulk (global -> shared completing on
//    an mbarrier, shared -> global in bulk groups). Device memory only; no
//    cluster multicast anywhere. The grid has one CTA per kTmaStages + 1
//    pieces: on B200 that oversubscribed grid runs device copies at about
//    104 % of a STREAM-style copy, a persistent one at 94 %;
//  * SM: 16-byte vector loads/stores from all threads, one CTA per chunk; the
//    slots may be the device alias of mapped pinned host memory (zero-copy
//    over PCIe).
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "runtime.h"

namespace kvoff {

// Error flags of bounded device-side waits (read by kvoff_device_error).
__device__ int g_device_error = 0;
constexpr int kErrTmaWaitTimeout = 1;

namespace {

constexpr int kMaxBatch = 128;
constexpr int kTmaPiece = 32768;  // bytes per pipeline stage
constexpr int kTmaStages = 3;     // 96 KiB of shared memory: two CTAs per SM
constexpr int kSmThreads = 256;
constexpr int kSmUnroll = 4;
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s bound on any spin

struct CopyGeometry {
  int64_t num_chunks;
  int64_t chunk_stride;  // bytes
  int64_t block_stride;  // bytes
  int64_t chunk_bytes;
};

struct SlotTable {
  int64_t block[kMaxBatch];
  uint8_t* slot[kMaxBatch];
};

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for phase `parity` of the mbarrier for at most limit_ns of
// %globaltimer, and at most kMaxSpins polls whatever the timer does.
constexpr uint64_t kMaxSpins = 1ull << 24;

__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_ns();
  for (uint64_t spins = 0; !mbar_try_wait(bar, parity); ++spins)
    if (spins >= kMaxSpins || global_ns() - start > limit_ns) return false;
  return true;
}

// Test hook for the bounded-wait error path: one thread waits on an mbarrier
// that nothing arrives at, gives up after limit_ns, and reports it in
// g_device_error exactly as tma_copy_kernel does.
__global__ void __launch_bounds__(32) debug_bounded_wait_kernel(uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&bar)) : "memory");
  if (!mbar_wait_bounded(smem_addr(&bar), 0, limit_ns))
    atomicOr(&g_device_error, kErrTmaWaitTimeout);
  asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_addr(&bar)) : "memory");
}

__device__ __forceinline__ void tma_load(uint32_t dst_smem, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst_smem),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_store(void* dst, uint32_t src_smem, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(src_smem), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void tma_wait_reads_done() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

__device__ __forceinline__ void tma_wait_all_done() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Source and destination of piece `u` (pieces enumerate block, chunk, offset).
struct Piece {
  const uint8_t* src;
  uint8_t* dst;
  uint32_t bytes;
};

__device__ __forceinline__ Piece piece_of(int64_t u, int64_t pieces_per_chunk, uint8_t* pool,
                                          const CopyGeometry& g, const SlotTable& t,
                                          bool save) {
  const int64_t per_block = g.num_chunks * pieces_per_chunk;
  const int idx = (int)(u / per_block);
  const int64_t rem = u - idx * per_block;
  const int64_t c = rem / pieces_per_chunk;
  const int64_t off = (rem - c * pieces_per_chunk) * kTmaPiece;
  const int64_t left = g.chunk_bytes - off;
  uint8_t* p = pool + c * g.chunk_stride + t.block[idx] * g.block_stride + off;
  uint8_t* s = t.slot[idx] + c * g.chunk_bytes + off;
  Piece r;
  r.bytes = (uint32_t)(left < kTmaPiece ? left : kTmaPiece);
  r.src = save ? p : s;
  r.dst = save ? s : p;
  return r;
}

__global__ void __launch_bounds__(32)
    tma_copy_kernel(uint8_t* pool, const CopyGeometry g, const __grid_constant__ SlotTable t,
                    int64_t pieces_per_chunk, int64_t units, int save) {
  extern __shared__ __align__(128) uint8_t stage[];
  __shared__ __align__(8) uint64_t bar[kTmaStages];
  if (threadIdx.x != 0) return;
  for (int s = 0; s < kTmaStages; ++s)
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&bar[s])) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");

  const int64_t first = blockIdx.x;
  const int64_t stride = gridDim.x;
  const int64_t mine = first < units ? (units - first + stride - 1) / stride : 0;
  const int64_t prologue = mine < kTmaStages ? mine : kTmaStages;
  for (int64_t k = 0; k < prologue; ++k) {
    const Piece p = piece_of(first + k * stride, pieces_per_chunk, pool, g, t, save != 0);
    tma_load(smem_addr(stage + k * kTmaPiece), p.src, p.bytes, smem_addr(&bar[k]));
  }
  int64_t issued = prologue;
  int64_t k = 0;
  for (; k < mine; ++k) {
    const int s = (int)(k % kTmaStages);
    if (!mbar_wait_bounded(smem_addr(&bar[s]), (uint32_t)((k / kTmaStages) & 1))) {
      atomicOr(&g_device_error, kErrTmaWaitTimeout);
      break;
    }
    const Piece p = piece_of(first + k * stride, pieces_per_chunk, pool, g, t, save != 0);
    tma_store(p.dst, smem_addr(stage + s * kTmaPiece), p.bytes);
    if (issued < mine) {
      tma_wait_reads_done();  // stage s is free once the bulk store has read it
      const Piece q = piece_of(first + issued * stride, pieces_per_chunk, pool, g, t, save != 0);
      tma_load(smem_addr(stage + s * kTmaPiece), q.src, q.bytes, smem_addr(&bar[s]));
      ++issued;
    }
  }
  // After a timeout, let loads already in flight land (bounded) before the
  // CTA's shared memory can be handed to another CTA.
  for (int64_t j = k; j < issued; ++j) {
    const int s = (int)(j % kTmaStages);
    mbar_wait_bounded(smem_addr(&bar[s]), (uint32_t)((j / kTmaStages) & 1));
  }
  tma_wait_all_done();
}

template <typename V>
__global__ void __launch_bounds__(kSmThreads)
    sm_copy_kernel(uint8_t* pool, const CopyGeometry g, const __grid_constant__ SlotTable t,
                   int64_t units, int save) {
  const int64_t per_chunk = g.chunk_bytes / (int64_t)sizeof(V);
  for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
    const int idx = (int)(u / g.num_chunks);
    const int64_t c = u - idx * g.num_chunks;
    V* p = reinterpret_cast<V*>(pool + c * g.chunk_stride + t.block[idx] * g.block_stride);
    V* s = reinterpret_cast<V*>(t.slot[idx] + c * g.chunk_bytes);
    const V* src = save ? p : s;
    V* dst = save ? s : p;
    for (int64_t base = threadIdx.x; base < per_chunk; base += (int64_t)kSmThreads * kSmUnroll) {
      V v[kSmUnroll];
#pragma unroll
      for (int k = 0; k < kSmUnroll; ++k) {
        const int64_t j = base + (int64_t)k * kSmThreads;
        if (j < per_chunk) v[k] = src[j];
      }
#pragma unroll
      for (int k = 0; k < kSmUnroll; ++k) {
        const int64_t j = base + (int64_t)k * kSmThreads;
        if (j < per_chunk) dst[j] = v[k];
      }
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int copy_engine(uint8_t* pool, const CopyGeometry& g, const int64_t* ids, int64_t count,
                void* const* slots, bool save, cudaStream_t stream) {
  int dev = 0, max_pitch = 0;
  cudaGetDevice(&dev);
  if (cudaDeviceGetAttribute(&max_pitch, cudaDevAttrMaxPitch, dev) != cudaSuccess) max_pitch = 0;
  const bool two_d = g.num_chunks > 1 && max_pitch > 0 && g.chunk_stride <= max_pitch &&
                     g.chunk_bytes <= g.chunk_stride;
  for (int64_t i = 0; i < count; ++i) {
    uint8_t* block = pool + ids[i] * g.block_stride;
    uint8_t* slot = static_cast<uint8_t*>(slots[i]);
    if (two_d) {
      cudaError_t e = save ? cudaMemcpy2DAsync(slot, g.chunk_bytes, block, g.chunk_stride,
                                               g.chunk_bytes, g.num_chunks, cudaMemcpyDefault,
                                               stream)
                           : cudaMemcpy2DAsync(block, g.chunk_stride, slot, g.chunk_bytes,
                                               g.chunk_bytes, g.num_chunks, cudaMemcpyDefault,
                                               stream);
      KVOFF_TRY(cuda_status(e, "cudaMemcpy2DAsync (block copy)"));
    } else {
      for (int64_t c = 0; c < g.num_chunks; ++c) {
        uint8_t* p = block + c * g.chunk_stride;
        uint8_t* s = slot + c * g.chunk_bytes;
        KVOFF_TRY(cuda_status(cudaMemcpyAsync(save ? s : p, save ? p : s, g.chunk_bytes,
                                              cudaMemcpyDefault, stream),
                              "cudaMemcpyAsync (chunk copy)"));
      }
    }
  }
  return KVOFF_OK;
}

int copy_kernel(uint8_t* pool, const CopyGeometry& g, const int64_t* ids, int64_t count,
                void* const* slots, bool save, int method, int32_t max_ctas,
                cudaStream_t stream) {
  bool vec16 = aligned16(pool) && (g.chunk_stride % 16) == 0 && (g.block_stride % 16) == 0 &&
               (g.chunk_bytes % 16) == 0;
  for (int64_t i = 0; i < count && vec16; ++i) vec16 = aligned16(slots[i]);
  if (method == KVOFF_COPY_TMA && !vec16)
    return fail(KVOFF_EINVAL,
                "kvoff_copy_blocks: the TMA method needs 16-byte aligned addresses, strides "
                "and chunk_bytes");
  const size_t tma_smem = (size_t)kTmaStages * kTmaPiece;
  if (method == KVOFF_COPY_TMA) {
    static thread_local int configured_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
      KVOFF_TRY(cuda_status(cudaFuncSetAttribute((const void*)tma_copy_kernel,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)tma_smem),
                            "cudaFuncSetAttribute (tma smem)"));
      configured_dev = dev;
    }
  }
  for (int64_t first = 0; first < count; first += kMaxBatch) {
    const int n = (int)((count - first) < kMaxBatch ? (count - first) : kMaxBatch);
    SlotTable t;
    for (int i = 0; i < n; ++i) {
      t.block[i] = ids[first + i];
      t.slot[i] = static_cast<uint8_t*>(slots[first + i]);
    }
    if (method == KVOFF_COPY_TMA) {
      const int64_t ppc = (g.chunk_bytes + kTmaPiece - 1) / kTmaPiece;
      const int64_t units = (int64_t)n * g.num_chunks * ppc;
      // About one pipeline fill (kTmaStages + 1 pieces) per CTA.
      const int64_t grid = streaming_grid(units, kTmaStages + 1, max_ctas);
      tma_copy_kernel<<<grid, 32, tma_smem, stream>>>(pool, g, t, ppc, units, save ? 1 : 0);
    } else {
      const int64_t units = (int64_t)n * g.num_chunks;
      if (vec16) {
        const int64_t grid = streaming_grid(units, 1, max_ctas);  // one CTA per chunk
        sm_copy_kernel<uint4><<<grid, kSmThreads, 0, stream>>>(pool, g, t, units, save ? 1 : 0);
      } else {
        const int64_t grid = grid_for(units, (const void*)sm_copy_kernel<uint8_t>, kSmThreads, 0, max_ctas);
        sm_copy_kernel<uint8_t><<<grid, kSmThreads, 0, stream>>>(pool, g, t, units, save ? 1 : 0);
      }
    }
    KVOFF_TRY(cuda_status(cudaGetLastError(), "block copy kernel launch"));
  }
  return KVOFF_OK;
}

}  // namespace
}  // namespace kvoff

using namespace kvoff;

extern "C" {

int kvoff_copy_blocks(void* pool, int64_t num_chunks, int64_t chunk_stride_bytes,
                      int64_t block_stride_bytes, int64_t num_blocks, int64_t chunk_bytes,
                      const int64_t* block_ids, int64_t count, void* const* slots,
                      int32_t direction, int32_t method, int32_t max_ctas, void* stream) {
  if (injected("copy_blocks")) return KVOFF_EINJECTED;
  if (count < 0) return fail(KVOFF_EINVAL, "kvoff_copy_blocks: negative count");
  if (num_chunks <= 0 || chunk_bytes <= 0 || chunk_stride_bytes < 0 || block_stride_bytes < 0 ||
      num_blocks <= 0)
    return fail(KVOFF_EINVAL, "kvoff_copy_blocks: bad geometry");
  if (direction != KVOFF_SAVE && direction != KVOFF_RESTORE)
    return fail(KVOFF_EINVAL, "kvoff_copy_blocks: bad direction %d", direction);
  if (method != KVOFF_COPY_ENGINE && method != KVOFF_COPY_TMA && method != KVOFF_COPY_SM)
    return fail(KVOFF_EINVAL, "kvoff_copy_blocks: bad method %d", method);
  if (count == 0) return ok();
  if (pool == nullptr || block_ids == nullptr || slots == nullptr)
    return fail(KVOFF_EINVAL, "kvoff_copy_blocks: null pointer");
  for (int64_t i = 0; i < count; ++i) {
    if (block_ids[i] < 0 || block_ids[i] >= num_blocks)
      return fail(KVOFF_EINVAL, "kvoff_copy_blocks: block id %lld out of range [0, %lld)",
                  (long long)block_ids[i], (long long)num_blocks);
    if (slots[i] == nullptr)
      return fail(KVOFF_EINVAL, "kvoff_copy_blocks: null slot at %lld", (long long)i);
  }
  if (method == KVOFF_COPY_TMA) {
    for (int64_t i = 0; i < count; ++i) {
      cudaPointerAttributes attr;
      if (cudaPointerGetAttributes(&attr, slots[i]) != cudaSuccess ||
          attr.type != cudaMemoryTypeDevice) {
        cudaGetLastError();
        return fail(KVOFF_EINVAL, "kvoff_copy_blocks: the TMA method needs device-memory slots");
      }
    }
  }
  const CopyGeometry g{num_chunks, chunk_stride_bytes, block_stride_bytes, chunk_bytes};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool save = direction == KVOFF_SAVE;
  if (method == KVOFF_COPY_ENGINE)
    KVOFF_TRY(copy_engine(static_cast<uint8_t*>(pool), g, block_ids, count, slots, save, s));
  else
    KVOFF_TRY(copy_kernel(static_cast<uint8_t*>(pool), g, block_ids, count, slots, save, method,
                          max_ctas, s));
  return ok();
}

int kvoff_copy_blocks_staged(void* pool, int64_t num_chunks, int64_t chunk_stride_bytes,
                             int64_t block_stride_bytes, int64_t num_blocks, int64_t chunk_bytes,
                             const int64_t* block_ids, int64_t count, void* const* host_slots,
                             void* staging, int64_t staging_blocks, int32_t direction,
                             void* const* wait_events, int32_t num_wait_events, void* event,
                             void* stream) {
  if (injected("copy_blocks_staged")) return KVOFF_EINJECTED;
  if (count < 0) return fail(KVOFF_EINVAL, "kvoff_copy_blocks_staged: negative count");
  if (num_chunks <= 0 || chunk_bytes <= 0 || chunk_stride_bytes < 0 || block_stride_bytes < 0 ||
      num_blocks <= 0)
    return fail(KVOFF_EINVAL, "kvoff_copy_blocks_staged: bad geometry");
  if (direction != KVOFF_SAVE && direction != KVOFF_RESTORE)
    return fail(KVOFF_EINVAL, "kvoff_copy_blocks_staged: bad direction %d", direction);
  if (num_wait_events < 0 || (num_wait_events > 0 && wait_events == nullptr) ||
      (num_wait_events > 0 && direction != KVOFF_SAVE))
    return fail(KVOFF_EINVAL, "kvoff_copy_blocks_staged: bad wait event list");
  if (count == 0) return ok();
  if (pool == nullptr || block_ids == nullptr || host_slots == nullptr || staging == nullptr ||
      staging_blocks <= 0)
    return fail(KVOFF_EINVAL, "kvoff_copy_blocks_staged: null pointer or no staging");
  for (int64_t i = 0; i < count; ++i) {
    if (block_ids[i] < 0 || block_ids[i] >= num_blocks)
      return fail(KVOFF_EINVAL, "kvoff_copy_blocks_staged: block id %lld out of range [0, %lld)",
                  (long long)block_ids[i], (long long)num_blocks);
    if (host_slots[i] == nullptr)
      return fail(KVOFF_EINVAL, "kvoff_copy_blocks_staged: null slot at %lld", (long long)i);
  }
  // The staging buffer must be device memory (the query is remembered per
  // buffer, so it runs once for each staging buffer a caller reuses).
  int staging_device = -1;
  KVOFF_TRY(device_memory_of(staging, &staging_device));
  if (staging_device < 0)
    return fail(KVOFF_EINVAL, "kvoff_copy_blocks_staged: staging must be device memory");
  const CopyGeometry g{num_chunks, chunk_stride_bytes, block_stride_bytes, chunk_bytes};
  const int64_t bb = num_chunks * chunk_bytes;  // one dense block in staging and in a slot
  // TMA where every address and stride allows 16-byte bulk copies, else the SM kernel.
  const int method = aligned16(pool) && aligned16(staging) && chunk_stride_bytes % 16 == 0 &&
                             block_stride_bytes % 16 == 0 && chunk_bytes % 16 == 0
                         ? KVOFF_COPY_TMA
                         : KVOFF_COPY_SM;
  uint8_t* base = static_cast<uint8_t*>(pool);
  uint8_t* stage = static_cast<uint8_t*>(staging);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool save = direction == KVOFF_SAVE;
  std::unique_lock<std::mutex> lock(pipe_mutex(), std::defer_lock);
  Pipe* p = nullptr;
  KVOFF_TRY(pipe_begin(s, staging, staging_blocks, lock, &p));
  const bool pipelined = p != nullptr;
  const int64_t half = staging_blocks / 2;
  const int64_t cap = pipelined ? half : staging_blocks;
  const int64_t group = cap < kMaxBatch ? cap : kMaxBatch;
  cudaStream_t ks = s;  // stream that runs the gather / scatter kernels
  if (pipelined) {
    ks = p->aux;
  }
  if (num_wait_events > 0) {  // a save's kernels need only these, not earlier DMA on `s`
    for (int32_t i = 0; i < num_wait_events; ++i)
      KVOFF_TRY(cuda_status(cudaStreamWaitEvent(ks, static_cast<cudaEvent_t>(wait_events[i]), 0),
                            "cudaStreamWaitEvent (wait event)"));
  } else if (pipelined) {  // kernels follow the caller stream's earlier work
    KVOFF_TRY(cuda_status(cudaEventRecord(p->start, s), "cudaEventRecord"));
    KVOFF_TRY(cuda_status(cudaStreamWaitEvent(ks, p->start, 0), "cudaStreamWaitEvent"));
  }
  void* dense[kMaxBatch];
  for (int64_t first = 0; first < count; first += group) {
    const int64_t n = (count - first) < group ? (count - first) : group;
    const int h = pipelined ? p->next : 0;
    for (int64_t i = 0; i < n; ++i) dense[i] = stage + (h * half + i) * bb;
    if (save) {
      if (pipelined)  // earlier copies out of this half are done
        KVOFF_TRY(pipe_wait_half(p, h, ks));
      KVOFF_TRY(copy_kernel(base, g, block_ids + first, n, dense, true, method, 0, ks));
      if (event != nullptr && first + n >= count)  // every pool block has been read
        KVOFF_TRY(cuda_status(cudaEventRecord(static_cast<cudaEvent_t>(event), ks),
                              "cudaEventRecord (source done)"));
      if (pipelined) {
        KVOFF_TRY(cuda_status(cudaEventRecord(p->ready[h], ks), "cudaEventRecord"));
        KVOFF_TRY(cuda_status(cudaStreamWaitEvent(s, p->ready[h], 0), "cudaStreamWaitEvent"));
      }
      KVOFF_TRY(copy_runs(host_slots + first, dense, n, bb, s, "staged block save copy"));
      if (pipelined) {
        KVOFF_TRY(cuda_status(cudaEventRecord(p->freed[h], s), "cudaEventRecord"));
        p->freed_recorded[h] = true;
        p->next = 1 - h;
      }
    } else {
      if (pipelined)  // earlier kernels reading this half are done
        KVOFF_TRY(pipe_wait_half(p, h, s));
      KVOFF_TRY(copy_runs(dense, host_slots + first, n, bb, s, "staged block restore copy"));
      if (pipelined) {
        KVOFF_TRY(cuda_status(cudaEventRecord(p->ready[h], s), "cudaEventRecord"));
        KVOFF_TRY(cuda_status(cudaStreamWaitEvent(ks, p->ready[h], 0), "cudaStreamWaitEvent"));
      }
      KVOFF_TRY(copy_kernel(base, g, block_ids + first, n, dense, false, method, 0, ks));
      if (pipelined) {
        KVOFF_TRY(cuda_status(cudaEventRecord(p->freed[h], ks), "cudaEventRecord"));
        p->freed_recorded[h] = true;
        p->next = 1 - h;
      }
    }
  }
  if (!save) {
    if (event != nullptr) {  // the caller orders readers of the blocks on this event
      KVOFF_TRY(cuda_status(cudaEventRecord(static_cast<cudaEvent_t>(event), ks),
                            "cudaEventRecord (done)"));
    } else if (pipelined) {  // the caller's stream sees every pool write of this call
      KVOFF_TRY(cuda_status(cudaEventRecord(p->done, ks), "cudaEventRecord"));
      KVOFF_TRY(cuda_status(cudaStreamWaitEvent(s, p->done, 0), "cudaStreamWaitEvent"));
    }
  }
  return ok();
}

int kvoff_copy_tokens(void* pool, int64_t num_chunks, int64_t chunk_stride_bytes,
                      int64_t block_stride_bytes, int64_t num_blocks, int64_t block_size,
                      int64_t token_bytes, const int64_t* block_ids, int64_t num_tokens,
                      void* dense, int32_t direction, void* stream) {
  if (injected("copy_tokens")) return KVOFF_EINJECTED;
  if (num_tokens < 0 || num_chunks <= 0 || block_size <= 0 || token_bytes <= 0 ||
      num_blocks <= 0 || chunk_stride_bytes < block_size * token_bytes || block_stride_bytes < 0)
    return fail(KVOFF_EINVAL, "kvoff_copy_tokens: bad geometry");
  if (direction != KVOFF_SAVE && direction != KVOFF_RESTORE)
    return fail(KVOFF_EINVAL, "kvoff_copy_tokens: bad direction %d", direction);
  if (num_tokens == 0) return ok();
  if (pool == nullptr || dense == nullptr || block_ids == nullptr)
    return fail(KVOFF_EINVAL, "kvoff_copy_tokens: null pointer");
  const int64_t blocks = (num_tokens + block_size - 1) / block_size;
  for (int64_t i = 0; i < blocks; ++i)
    if (block_ids[i] < 0 || block_ids[i] >= num_blocks)
      return fail(KVOFF_EINVAL, "kvoff_copy_tokens: block id %lld out of range [0, %lld)",
                  (long long)block_ids[i], (long long)num_blocks);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t dense_pitch = num_tokens * token_bytes;  // one (K/V, layer) row of the dense copy
  for (int64_t i = 0; i < blocks; ++i) {
    const int64_t first = i * block_size;
    const int64_t n = (num_tokens - first) < block_size ? (num_tokens - first) : block_size;
    uint8_t* blk = static_cast<uint8_t*>(pool) + block_ids[i] * block_stride_bytes;
    uint8_t* dn = static_cast<uint8_t*>(dense) + first * token_bytes;
    const cudaError_t e =
        direction == KVOFF_SAVE
            ? cudaMemcpy2DAsync(dn, dense_pitch, blk, chunk_stride_bytes, n * token_bytes,
                                num_chunks, cudaMemcpyDefault, s)
            : cudaMemcpy2DAsync(blk, chunk_stride_bytes, dn, dense_pitch, n * token_bytes,
                                num_chunks, cudaMemcpyDefault, s);
    KVOFF_TRY(cuda_status(e, "cudaMemcpy2DAsync (token copy)"));
  }
  return ok();
}

int kvoff_debug_bounded_wait(int64_t limit_ns, void* stream) {
  if (limit_ns <= 0 || limit_ns > 2000000000ll)
    return fail(KVOFF_EINVAL, "kvoff_debug_bounded_wait: limit must be in (0, 2 s]");
  debug_bounded_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      (uint64_t)limit_ns);
  KVOFF_TRY(cuda_status(cudaGetLastError(), "debug_bounded_wait launch"));
  return ok();
}

int kvoff_device_error(int32_t device, int32_t* flags, int32_t clear) {
  if (flags == nullptr) return fail(KVOFF_EINVAL, "kvoff_device_error: null output");
  int prev = 0;
  KVOFF_TRY(cuda_status(cudaGetDevice(&prev), "cudaGetDevice"));
  KVOFF_TRY(cuda_status(cudaSetDevice(device), "cudaSetDevice"));
  int rc = cuda_status(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  int value = 0;
  if (rc == KVOFF_OK)
    rc = cuda_status(cudaMemcpyFromSymbol(&value, g_device_error, sizeof(int)),
                     "cudaMemcpyFromSymbol (error flags)");
  if (rc == KVOFF_OK && clear) {
    const int zero = 0;
    rc = cuda_status(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)),
                     "cudaMemcpyToSymbol (error flags)");
  }
  cudaSetDevice(prev);
  if (rc != KVOFF_OK) return rc;
  *flags = value;
  return ok();
}

}  // extern "C"
