// Host runtime of libkvoff: error reporting, fault injection, pinned NUMA-local
// host slabs, plain async copies and the staged calls' two-half pipelines.
#include "runtime.h"

#include <errno.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <map>
#include <mutex>
#include <string>
#include <unordered_map>

namespace kvoff {
namespace {

thread_local std::string t_error;

std::mutex g_inject_mu;
std::map<std::string, int> g_inject;  // op name -> remaining injected failures

std::mutex g_prop_mu;
std::unordered_map<int, int> g_sm_count;                 // device -> SMs
std::map<std::pair<const void*, int>, int> g_occupancy;  // (kernel, device) -> CTAs/SM

struct Slab {
  size_t bytes;
};
std::mutex g_slab_mu;
std::unordered_map<void*, Slab> g_slabs;

}  // namespace

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_error = buf;
  return code;
}

int ok() {
  t_error.clear();
  return KVOFF_OK;
}

bool injected(const char* op) {
  std::lock_guard<std::mutex> lock(g_inject_mu);
  auto it = g_inject.find(op);
  if (it == g_inject.end() || it->second <= 0) return false;
  if (--it->second == 0) g_inject.erase(it);
  fail(KVOFF_EINJECTED, "kvoff_%s: injected failure (kvoff_debug_fail_next)", op);
  return true;
}

int cuda_status(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return KVOFF_OK;
  return fail(KVOFF_ECUDA, "%s: %s (%s)", what, cudaGetErrorString(err), cudaGetErrorName(err));
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 1;
  std::lock_guard<std::mutex> lock(g_prop_mu);
  auto it = g_sm_count.find(dev);
  if (it != g_sm_count.end()) return it->second;
  int sms = 1;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
    sms = 1;
  g_sm_count[dev] = sms;
  return sms;
}

int ctas_per_sm(const void* kernel, int threads, size_t smem) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 1;
  {
    std::lock_guard<std::mutex> lock(g_prop_mu);
    auto it = g_occupancy.find({kernel, dev});
    if (it != g_occupancy.end()) return it->second;
  }
  int n = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem) != cudaSuccess ||
      n < 1)
    n = 1;
  std::lock_guard<std::mutex> lock(g_prop_mu);
  g_occupancy[{kernel, dev}] = n;
  return n;
}

int64_t grid_for(int64_t units, const void* kernel, int threads, size_t smem, int32_t max_ctas) {
  int64_t full = (int64_t)sm_count() * ctas_per_sm(kernel, threads, smem);
  int64_t grid = units < full ? units : full;
  if (max_ctas > 0 && grid > max_ctas) grid = max_ctas;
  return grid < 1 ? 1 : grid;
}

int64_t streaming_grid(int64_t units, int64_t per_cta, int32_t max_ctas) {
  int64_t grid = (units + per_cta - 1) / per_cta;
  const int64_t cap = max_ctas > 0 ? max_ctas : 0x7FFFFFFF;
  if (grid > cap) grid = cap;
  return grid < 1 ? 1 : grid;
}

int device_memory_of(const void* p, int* device) {
  struct Seen {
    const void* p;
    int device;
  };
  constexpr int kSeen = 8;
  static thread_local Seen seen[kSeen] = {};
  static thread_local int next = 0;
  if (p != nullptr)
    for (const Seen& s : seen)
      if (s.p == p) {
        *device = s.device;
        return KVOFF_OK;
      }
  int dev = -1;
  cudaPointerAttributes attr;
  if (p != nullptr && cudaPointerGetAttributes(&attr, p) == cudaSuccess &&
      attr.type == cudaMemoryTypeDevice)
    dev = attr.device;
  else
    cudaGetLastError();  // clears the error a plain host pointer leaves behind
  if (p != nullptr) {
    seen[next] = Seen{p, dev};
    next = (next + 1) % kSeen;
  }
  *device = dev;
  return KVOFF_OK;
}

int copy_runs(void* const* dst, void* const* src, int64_t n, int64_t bytes, cudaStream_t s,
              const char* what) {
  for (int64_t i = 0; i < n;) {
    int64_t j = i + 1;
    while (j < n && static_cast<uint8_t*>(dst[j]) == static_cast<uint8_t*>(dst[j - 1]) + bytes &&
           static_cast<uint8_t*>(src[j]) == static_cast<uint8_t*>(src[j - 1]) + bytes)
      ++j;
    KVOFF_TRY(cuda_status(cudaMemcpyAsync(dst[i], src[i], (j - i) * bytes, cudaMemcpyDefault, s),
                          what));
    i = j;
  }
  return KVOFF_OK;
}

namespace {
std::mutex g_pipe_mu;
std::map<std::pair<int, cudaStream_t>, Pipe> g_pipes;  // (device, caller stream) -> pipeline
}  // namespace

std::mutex& pipe_mutex() { return g_pipe_mu; }

namespace {
int pipe_get(cudaStream_t caller, Pipe** out) {
  int dev = 0;
  KVOFF_TRY(cuda_status(cudaGetDevice(&dev), "cudaGetDevice"));
  Pipe& p = g_pipes[{dev, caller}];
  if (p.aux == nullptr) {
    KVOFF_TRY(cuda_status(cudaStreamCreateWithFlags(&p.aux, cudaStreamNonBlocking),
                          "cudaStreamCreateWithFlags (pipeline stream)"));
    cudaEvent_t* events[] = {&p.start, &p.done, &p.ready[0], &p.ready[1], &p.freed[0],
                             &p.freed[1]};
    for (cudaEvent_t* e : events)
      KVOFF_TRY(cuda_status(cudaEventCreateWithFlags(e, cudaEventDisableTiming),
                            "cudaEventCreateWithFlags (pipeline event)"));
  }
  *out = &p;
  return KVOFF_OK;
}
}  // namespace

int pipe_for(cudaStream_t caller, const void* staging, Pipe** out) {
  Pipe* p = nullptr;
  KVOFF_TRY(pipe_get(caller, &p));
  if (p->staging != staging) {  // a new staging buffer starts a fresh ring
    // The fresh ring drops the waits on the old ring's halves, so the caller
    // first waits for every kernel already queued on aux. Torch hands out
    // stream handles from a pool, so another user of the same handle may have
    // left kernels there that still read its own staging.
    if (p->staging != nullptr) {
      KVOFF_TRY(cuda_status(cudaEventRecord(p->done, p->aux), "cudaEventRecord"));
      KVOFF_TRY(cuda_status(cudaStreamWaitEvent(caller, p->done, 0), "cudaStreamWaitEvent"));
    }
    p->staging = staging;
    p->freed_recorded[0] = p->freed_recorded[1] = false;
    p->next = 0;
  }
  *out = p;
  return KVOFF_OK;
}

int pipe_wait_half(Pipe* p, int h, cudaStream_t waiter) {
  if (p->freed_recorded[h])
    KVOFF_TRY(cuda_status(cudaStreamWaitEvent(waiter, p->freed[h], 0), "cudaStreamWaitEvent"));
  return KVOFF_OK;
}

int pipe_begin(cudaStream_t caller, const void* staging, int64_t staging_blocks,
               std::unique_lock<std::mutex>& lock, Pipe** out) {
  *out = nullptr;
  if (staging_blocks < 2) return KVOFF_OK;
  lock.lock();
  KVOFF_TRY(pipe_for(caller, staging, out));
  return KVOFF_OK;
}

int join_pipe(cudaStream_t caller) {
  int dev = 0;
  KVOFF_TRY(cuda_status(cudaGetDevice(&dev), "cudaGetDevice"));
  std::lock_guard<std::mutex> lock(g_pipe_mu);
  auto it = g_pipes.find({dev, caller});
  if (it == g_pipes.end()) return KVOFF_OK;
  Pipe& p = it->second;
  KVOFF_TRY(cuda_status(cudaEventRecord(p.done, p.aux), "cudaEventRecord"));
  KVOFF_TRY(cuda_status(cudaStreamWaitEvent(caller, p.done, 0), "cudaStreamWaitEvent"));
  return KVOFF_OK;
}

}  // namespace kvoff

using namespace kvoff;

extern "C" {

int32_t kvoff_abi_version(void) { return KVOFF_ABI_VERSION; }

const char* kvoff_last_error(void) { return t_error.c_str(); }

int kvoff_debug_fail_next(const char* op, int32_t count) {
  if (op == nullptr || op[0] == '\0') return fail(KVOFF_EINVAL, "kvoff_debug_fail_next: empty op");
  if (count < 0) return fail(KVOFF_EINVAL, "kvoff_debug_fail_next: negative count");
  std::lock_guard<std::mutex> lock(g_inject_mu);
  if (count == 0)
    g_inject.erase(op);
  else
    g_inject[op] = count;
  return ok();
}

int kvoff_memcpy(void* dst, const void* src, uint64_t bytes, void* stream) {
  if (injected("memcpy")) return KVOFF_EINJECTED;
  if (bytes == 0) return ok();
  if (dst == nullptr || src == nullptr) return fail(KVOFF_EINVAL, "kvoff_memcpy: null pointer");
  KVOFF_TRY(cuda_status(
      cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)),
      "kvoff_memcpy"));
  return ok();
}

int kvoff_device_numa_node(int32_t device, int32_t* numa_node) {
  if (numa_node == nullptr) return fail(KVOFF_EINVAL, "kvoff_device_numa_node: null output");
  *numa_node = -1;
  char bus[32] = {0};
  KVOFF_TRY(cuda_status(cudaDeviceGetPCIBusId(bus, sizeof(bus), device), "cudaDeviceGetPCIBusId"));
  for (char* p = bus; *p; ++p)
    if (*p >= 'A' && *p <= 'F') *p = (char)(*p - 'A' + 'a');
  char path[128];
  snprintf(path, sizeof(path), "/sys/bus/pci/devices/%s/numa_node", bus);
  FILE* f = fopen(path, "r");
  if (f != nullptr) {
    int node = -1;
    if (fscanf(f, "%d", &node) == 1 && node >= 0) *numa_node = node;
    fclose(f);
  }
  return ok();
}

int kvoff_host_alloc(uint64_t bytes, int32_t numa_node, void** host_ptr, void** device_ptr) {
  if (injected("host_alloc")) return KVOFF_EINJECTED;
  if (host_ptr == nullptr) return fail(KVOFF_EINVAL, "kvoff_host_alloc: null output");
  *host_ptr = nullptr;
  if (device_ptr != nullptr) *device_ptr = nullptr;
  if (bytes == 0) return fail(KVOFF_EINVAL, "kvoff_host_alloc: zero bytes");
  const size_t page = (size_t)sysconf(_SC_PAGESIZE);
  const size_t len = (bytes + page - 1) / page * page;
  void* p = mmap(nullptr, len, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
  if (p == MAP_FAILED)
    return fail(KVOFF_ENOMEM, "kvoff_host_alloc: mmap(%zu) failed: %s", len, strerror(errno));
  // Large slabs benefit from transparent huge pages: fewer pages to pin and
  // fewer IOMMU entries for the DMA engines.
  madvise(p, len, MADV_HUGEPAGE);
  if (numa_node >= 0 && numa_node < 1024) {
    // MPOL_PREFERRED (1): allocate on the GPU's node when it has room, never
    // fail. Pages are placed at first touch, which cudaHostRegister does.
    unsigned long mask[1024 / (8 * sizeof(unsigned long))] = {0};
    mask[numa_node / (8 * sizeof(unsigned long))] |= 1UL << (numa_node % (8 * sizeof(unsigned long)));
    syscall(SYS_mbind, p, len, 1 /* MPOL_PREFERRED */, mask, (unsigned long)1024, 0U);
  }
  cudaError_t err = cudaHostRegister(p, len, cudaHostRegisterPortable | cudaHostRegisterMapped);
  if (err != cudaSuccess) {
    munmap(p, len);
    return fail(KVOFF_ENOMEM, "kvoff_host_alloc: cudaHostRegister(%zu) failed: %s", len,
                cudaGetErrorString(err));
  }
  void* dev = nullptr;
  err = cudaHostGetDevicePointer(&dev, p, 0);
  if (err != cudaSuccess) {
    cudaHostUnregister(p);
    munmap(p, len);
    return fail(KVOFF_ECUDA, "kvoff_host_alloc: cudaHostGetDevicePointer failed: %s",
                cudaGetErrorString(err));
  }
  {
    std::lock_guard<std::mutex> lock(g_slab_mu);
    g_slabs[p] = Slab{len};
  }
  *host_ptr = p;
  if (device_ptr != nullptr) *device_ptr = dev;
  return ok();
}

int kvoff_host_free(void* host_ptr) {
  if (host_ptr == nullptr) return ok();
  size_t len = 0;
  {
    std::lock_guard<std::mutex> lock(g_slab_mu);
    auto it = g_slabs.find(host_ptr);
    if (it == g_slabs.end())
      return fail(KVOFF_EINVAL, "kvoff_host_free: %p was not allocated by kvoff_host_alloc",
                  host_ptr);
    len = it->second.bytes;
    g_slabs.erase(it);
  }
  cudaError_t err = cudaHostUnregister(host_ptr);
  munmap(host_ptr, len);
  if (err != cudaSuccess)
    return fail(KVOFF_ECUDA, "kvoff_host_free: cudaHostUnregister failed: %s",
                cudaGetErrorString(err));
  return ok();
}

}  // extern "C"
