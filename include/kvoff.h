/*
 * kvoff.h - C ABI of the B200 KV-cache offload copy path (libkvoff.so).
 *
 * Every entry point takes plain pointers, 64-bit sizes and an opaque CUDA
 * stream handle (a cudaStream_t cast to void*; NULL is the legacy default
 * stream). Nothing here synchronizes the host: all GPU work is enqueued on
 * the given stream. Every function returns a kvoff_status; on failure
 * kvoff_last_error() describes the problem for the calling thread.
 *
 * Paged pool geometry. The engine's KV pool is a tensor
 *     pool[2, L, NB, BS, H, D]     (K/V, layer, block, token, KV head, dim)
 * (nanovllm/engine/model_runner.py:120). One KV block is 2*L "chunks"; each
 * chunk holds BS*H rows of D contiguous elements and sits at
 *     pool + c * chunk_stride + block_id * block_stride      (c in [0, 2L))
 * counted in elements (bf16 here), so chunk_stride = NB*BS*H*D and
 * block_stride = BS*H*D for a contiguous pool. A "row" is one (token, KV
 * head) vector of D elements. A saved block ("slot") is laid out densely as
 * [2, L, BS, H, D] (cpu_prefix_cache.py:94), so row r of chunk c lands at
 * slot + (c * rows_per_chunk + r) * D.
 *
 * FP8 slots store the payload [2, L, BS, H, D] float8_e4m3fn and one bf16
 * scale per row, [2, L, BS, H, 1] (cpu_prefix_cache.py:96-100, 204-206).
 */
#ifndef KVOFF_H_
#define KVOFF_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define KVOFF_API __attribute__((visibility("default")))
#else
#define KVOFF_API
#endif

#define KVOFF_ABI_VERSION 1

/* Status codes returned by every entry point. */
enum kvoff_status {
  KVOFF_OK = 0,
  KVOFF_EINVAL = 1,    /* bad argument: null pointer, size, alignment, block id */
  KVOFF_ECUDA = 2,     /* a CUDA runtime call failed */
  KVOFF_EINJECTED = 3, /* failure injected by kvoff_debug_fail_next */
  KVOFF_ENOMEM = 4,    /* host allocation / pinning failed */
  KVOFF_EDEVICE = 5    /* a kernel reported a device-side error flag */
};

/* Directions and methods for kvoff_copy_blocks. */
enum kvoff_direction { KVOFF_SAVE = 0, KVOFF_RESTORE = 1 };
enum kvoff_copy_method {
  KVOFF_COPY_ENGINE = 0, /* cudaMemcpy2DAsync over the 2L strided chunks (DMA engine) */
  KVOFF_COPY_TMA = 1,    /* cp.async.bulk gather/scatter kernel; slots must be device memory */
  KVOFF_COPY_SM = 2      /* 16-byte vector copy kernel; slots may be mapped pinned host memory */
};

/* ABI version of the loaded library (KVOFF_ABI_VERSION at build time). */
KVOFF_API int32_t kvoff_abi_version(void);

/* Message of the last failure on this thread ("" when none). */
KVOFF_API const char* kvoff_last_error(void);

/*
 * Host-side fault injection for tests: the next `count` calls of entry point
 * `op` (its name without the "kvoff_" prefix, e.g. "fp8_save_blocks") fail
 * with KVOFF_EINJECTED before enqueuing any work. count = 0 clears it.
 * Replaces the reference tests' monkeypatching of torch.Tensor.copy_
 * (bench/test_cpu_prefix_cache.py:113-123, 133-143), which cannot reach
 * native copies.
 */
KVOFF_API int kvoff_debug_fail_next(const char* op, int32_t count);

/*
 * Device-side error flags of bounded waits in this library's kernels on
 * `device` (0 = none). clear != 0 resets them. Synchronizes `device`.
 */
KVOFF_API int kvoff_device_error(int32_t device, int32_t* flags, int32_t clear);

/*
 * Test hook for the bounded-wait error path (no counterpart in the
 * reference): enqueues one thread that waits on an mbarrier nothing arrives
 * at, gives up after limit_ns (at most 2 s), and sets the same flag as a
 * timed-out TMA copy wait. The context stays usable; kvoff_device_error
 * reads the flag.
 */
KVOFF_API int kvoff_debug_bounded_wait(int64_t limit_ns, void* stream);

/*
 * FP8 save: gather `count` KV blocks of a bf16 paged pool and quantize each
 * row to float8_e4m3fn with one bf16 scale per row:
 *     scale   = bf16_rne(max(f32(amax|x|) / 448, 1e-30))
 *     payload = e4m3_rne(clamp(f32(x) / f32(scale), -448, 448))
 * Replaces fp8_quantize (nanovllm/engine/cpu_prefix_cache.py:20-24) as used
 * by CPUBlockCache._quantize (:225-234) on the pool view cache[:, :, block_id]
 * (:305). payload_dst[i] / scale_dst[i] receive block_ids[i]'s slot; they
 * must be device-accessible: device memory (staging) or the device alias of
 * mapped pinned host memory (zero-copy save). max_ctas <= 0 picks a full grid.
 */
KVOFF_API int kvoff_fp8_save_blocks(const void* pool, int64_t num_chunks, int64_t chunk_stride,
                                    int64_t block_stride, int64_t num_blocks,
                                    int64_t rows_per_chunk, int64_t head_dim,
                                    const int64_t* block_ids, int64_t count,
                                    void* const* payload_dst, void* const* scale_dst,
                                    int32_t max_ctas, void* stream);

/*
 * FP8 restore: dequantize slots into pool blocks,
 *     x = bf16_rne(f32(payload) * f32(scale))
 * Replaces fp8_dequantize (cpu_prefix_cache.py:27-28) as used by
 * CPUBlockCache._dequantize (:236-243) into cache[:, :, block_id] (:373).
 * Sources must be device-accessible (staging or mapped pinned host).
 */
KVOFF_API int kvoff_fp8_restore_blocks(void* pool, int64_t num_chunks, int64_t chunk_stride,
                                       int64_t block_stride, int64_t num_blocks,
                                       int64_t rows_per_chunk, int64_t head_dim,
                                       const int64_t* block_ids, int64_t count,
                                       const void* const* payload_src,
                                       const void* const* scale_src, int32_t max_ctas,
                                       void* stream);

/*
 * Staged FP8 save: quantize up to `staging_blocks` blocks at a time into the
 * contiguous device staging buffers, then drain each block with two
 * cudaMemcpyAsync calls into host_payload[i] / host_scale[i] (pinned host).
 * Replaces CPUBlockCache._quantize's device-staging branch
 * (cpu_prefix_cache.py:227-234, staging from _stage :217-223).
 */
KVOFF_API int kvoff_fp8_save_blocks_staged(const void* pool, int64_t num_chunks,
                                           int64_t chunk_stride, int64_t block_stride,
                                           int64_t num_blocks, int64_t rows_per_chunk,
                                           int64_t head_dim, const int64_t* block_ids,
                                           int64_t count, void* const* host_payload,
                                           void* const* host_scale, void* staging_payload,
                                           void* staging_scale, int64_t staging_blocks,
                                           void* stream);

/*
 * kvoff_fp8_save_blocks_staged with explicit ordering. When num_wait_events > 0
 * the quantize kernels wait for those events (cudaEvent_t handles, e.g. the
 * point where the pool blocks were last written) instead of for all earlier
 * work on `stream`, so they can overlap the DMA of earlier calls; the caller
 * then orders the host-slot writes on `stream` itself. source_done, when not
 * NULL, is recorded once every pool block of the call has been read: a block
 * may be overwritten after it, before the slow drain to host finishes. Used by
 * CPUBlockCache.save_block (cpu_prefix_cache.py:306-322) and
 * before_block_reuse (:352-357).
 */
KVOFF_API int kvoff_fp8_save_blocks_staged_ev(const void* pool, int64_t num_chunks,
                                              int64_t chunk_stride, int64_t block_stride,
                                              int64_t num_blocks, int64_t rows_per_chunk,
                                              int64_t head_dim, const int64_t* block_ids,
                                              int64_t count, void* const* host_payload,
                                              void* const* host_scale, void* staging_payload,
                                              void* staging_scale, int64_t staging_blocks,
                                              void* const* wait_events, int32_t num_wait_events,
                                              void* source_done, void* stream);

/*
 * Staged FP8 save that allocates nothing, for callers that cannot allocate
 * device memory while saving: an engine that gives nearly all free HBM to its
 * KV pool at start-up has no room left for a staging buffer, and a host
 * runtime calling this library through its C ABI may have no device allocator
 * at all. Same result as kvoff_fp8_save_blocks_staged, but it stages through
 * a fixed 16 MiB scratch array inside the library (held on every GPU that
 * loads the library until the process exits) and calls no allocator. Blocks
 * larger than the scratch are processed in pieces of whole (K/V, layer)
 * chunks; a chunk whose payload (rounded up to 256 bytes) plus scales exceeds
 * 16 MiB is rejected with KVOFF_EINVAL. The pool's device must be the current
 * device (the scratch used is the current device's; another device's pool is
 * rejected with KVOFF_EINVAL). The first call on each device looks up the
 * scratch's device address, so make that first call before any stream
 * capture. All calls share the one scratch array and leave their data in it:
 * calls that may overlap on the GPU (different streams, or different host
 * threads) race and must be serialized by the caller. No counterpart in the
 * reference.
 */
KVOFF_API int kvoff_fp8_save_blocks_staged_noalloc(const void* pool, int64_t num_chunks,
                                                   int64_t chunk_stride, int64_t block_stride,
                                                   int64_t num_blocks, int64_t rows_per_chunk,
                                                   int64_t head_dim, const int64_t* block_ids,
                                                   int64_t count, void* const* host_payload,
                                                   void* const* host_scale, void* stream);

/*
 * Staged FP8 restore: copy each slot host->device into staging (two
 * cudaMemcpyAsync per block), then dequantize into the pool. Replaces
 * CPUBlockCache._dequantize's CUDA branch (cpu_prefix_cache.py:237-243).
 */
KVOFF_API int kvoff_fp8_restore_blocks_staged(void* pool, int64_t num_chunks,
                                              int64_t chunk_stride, int64_t block_stride,
                                              int64_t num_blocks, int64_t rows_per_chunk,
                                              int64_t head_dim, const int64_t* block_ids,
                                              int64_t count, const void* const* host_payload,
                                              const void* const* host_scale,
                                              void* staging_payload, void* staging_scale,
                                              int64_t staging_blocks, void* stream);

/*
 * kvoff_fp8_restore_blocks_staged that signals completion on `done_event`
 * (recorded after the last pool write) instead of making `stream` wait for
 * the dequantize kernels, so the next call's host-to-device copies can start
 * while this call's kernels run. The caller orders readers of the blocks on
 * done_event; kvoff_stream_join_pipeline(stream) makes `stream` itself wait.
 * Used by CPUBlockCache._copy_entry (cpu_prefix_cache.py:371-393).
 */
KVOFF_API int kvoff_fp8_restore_blocks_staged_ev(void* pool, int64_t num_chunks,
                                                 int64_t chunk_stride, int64_t block_stride,
                                                 int64_t num_blocks, int64_t rows_per_chunk,
                                                 int64_t head_dim, const int64_t* block_ids,
                                                 int64_t count, const void* const* host_payload,
                                                 const void* const* host_scale,
                                                 void* staging_payload, void* staging_scale,
                                                 int64_t staging_blocks, void* done_event,
                                                 void* stream);

/*
 * Make `stream` wait for all work the staged calls queued on their internal
 * kernel stream for `stream` (needed before synchronizing `stream` or freeing
 * its staging buffers after *_ev calls). No-op when there is none.
 *
 * The staged calls (FP8 and BF16) pipeline their kernels on that internal
 * stream when staging_blocks >= 2. With staging_blocks = 1 they run serially
 * on `stream` itself, one block at a time: the copy engine then goes idle
 * while each block's kernel runs, so small copies that other streams queue on
 * it meanwhile (a compute stream's per-step inputs and sampled tokens) run in
 * those gaps instead of waiting behind a whole run of block transfers, as
 * with the reference, whose copies and kernels share one stream
 * (cpu_prefix_cache.py:236-243, :311-322). Join before switching a stream
 * and staging buffer between the two forms.
 */
KVOFF_API int kvoff_stream_join_pipeline(void* stream);


/*
 * Byte-exact block passthrough (BF16 mode): move whole blocks between the
 * pool and dense slots. Strides and sizes are in BYTES here. direction
 * KVOFF_SAVE copies pool -> slots[i], KVOFF_RESTORE slots[i] -> pool.
 * Replaces payload.copy_(source) (cpu_prefix_cache.py:319) and
 * target.copy_(entry.kv) (:386). Method KVOFF_COPY_TMA needs device slots
 * and 16-byte alignment of every address and of chunk_bytes.
 */
KVOFF_API int kvoff_copy_blocks(void* pool, int64_t num_chunks, int64_t chunk_stride_bytes,
                                int64_t block_stride_bytes, int64_t num_blocks,
                                int64_t chunk_bytes, const int64_t* block_ids, int64_t count,
                                void* const* slots, int32_t direction, int32_t method,
                                int32_t max_ctas, void* stream);

/*
 * Staged byte-exact block passthrough between the pool and pinned host slots,
 * pipelined like the staged FP8 calls. TMA bulk-copy kernels (the SM copy
 * kernel where an address or stride is not 16-byte aligned) gather blocks
 * into, or scatter them out of, one half of the device staging buffer
 * (staging_blocks dense blocks of num_chunks * chunk_bytes) on a library-owned
 * kernel stream, while plain DMA moves the other half over PCIe on `stream`.
 * Every DMA is a contiguous copy: a strided DMA straight into the pool holds
 * up later small copies queued behind it, stalling the compute stream's
 * inputs while restores run. Same bytes as kvoff_copy_blocks.
 *   KVOFF_SAVE: the gather kernels wait for wait_events (none: for earlier work
 *     on `stream`); `event`, when non-null, is recorded once every pool block
 *     has been read, so a block's next writer need not wait for the drain.
 *   KVOFF_RESTORE: `event`, when non-null, is recorded after the last pool
 *     write and `stream` is not joined; without it `stream` waits for the
 *     kernels. wait_events must be empty.
 * kvoff_stream_join_pipeline(stream) makes `stream` wait for the kernels.
 * Replaces payload.copy_(source) (cpu_prefix_cache.py:319) and
 * target.copy_(entry.kv) (:386) in BF16 mode.
 */
KVOFF_API int kvoff_copy_blocks_staged(void* pool, int64_t num_chunks,
                                       int64_t chunk_stride_bytes, int64_t block_stride_bytes,
                                       int64_t num_blocks, int64_t chunk_bytes,
                                       const int64_t* block_ids, int64_t count,
                                       void* const* host_slots, void* staging,
                                       int64_t staging_blocks, int32_t direction,
                                       void* const* wait_events, int32_t num_wait_events,
                                       void* event, void* stream);

/*
 * Token-range copy for KV handoff: the first num_tokens tokens of a sequence,
 * stored in blocks block_ids[0 .. ceil(num_tokens / block_size)) of the pool,
 * to or from a dense [2L, num_tokens, H, D] buffer (direction KVOFF_SAVE:
 * pool -> dense, KVOFF_RESTORE: dense -> pool). token_bytes = H * D * elem;
 * strides in bytes. One strided DMA per block (the last one partial); dense may
 * be pinned host or device memory. Replaces the index_select + .contiguous() +
 * .cpu() gather of export_kv (nanovllm/engine/kv_handoff.py:46-55) and the
 * per-block scatter of import_kv (:112-118).
 */
KVOFF_API int kvoff_copy_tokens(void* pool, int64_t num_chunks, int64_t chunk_stride_bytes,
                                int64_t block_stride_bytes, int64_t num_blocks,
                                int64_t block_size, int64_t token_bytes,
                                const int64_t* block_ids, int64_t num_tokens, void* dense,
                                int32_t direction, void* stream);

/*
 * Slot-mapping scatter of fresh K/V rows into the paged cache:
 *     for i < num_tokens with slot = slot_mapping[i] != -1:
 *         k_cache[slot * row_bytes ...] = key[i * key_stride_bytes ...] (row_bytes)
 *         v_cache[slot * row_bytes ...] = value[i * value_stride_bytes ...]
 * Replaces store_kvcache / store_kvcache_kernel
 * (nanovllm/layers/attention.py:10-40). Negative slots are skipped; slots
 * >= num_slots are skipped and counted into *bad_slots when it is non-null
 * (device memory). No allocation and no host synchronization, so it can be
 * captured in a CUDA graph.
 */
KVOFF_API int kvoff_store_kvcache(const void* key, int64_t key_stride_bytes, const void* value,
                                  int64_t value_stride_bytes, void* k_cache, void* v_cache,
                                  int64_t row_bytes, const int32_t* slot_mapping,
                                  int64_t num_tokens, int64_t num_slots, int32_t* bad_slots,
                                  void* stream);

/*
 * Pinned host slab: mmap `bytes`, prefer NUMA node `numa_node` (-1: no
 * preference), page-lock it with cudaHostRegister(Portable | Mapped) and
 * return the host pointer and its device alias for zero-copy kernels.
 * Replaces the pin_memory=True slab chunks of CPUBlockCache._grow
 * (cpu_prefix_cache.py:199-208).
 */
KVOFF_API int kvoff_host_alloc(uint64_t bytes, int32_t numa_node, void** host_ptr,
                               void** device_ptr);

/* Unregister and unmap a slab from kvoff_host_alloc. */
KVOFF_API int kvoff_host_free(void* host_ptr);

/* NUMA node closest to CUDA device `device` (-1 when unknown). */
KVOFF_API int kvoff_device_numa_node(int32_t device, int32_t* numa_node);

/* cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, stream). */
KVOFF_API int kvoff_memcpy(void* dst, const void* src, uint64_t bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KVOFF_H_ */
