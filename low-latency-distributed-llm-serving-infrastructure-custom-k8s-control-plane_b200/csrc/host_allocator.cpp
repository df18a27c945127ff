// Host mirror of the reference allocator API (llm_allocator_cpp.PageAllocator), behind the C ABI.
//
// Same observable behaviour as csrc/include/page_allocator.hpp:45-374: a FIFO queue of free GPU
// block ids starting 0..N-1, per-block reference counts, a stack of host swap blocks with a
// gpu->cpu map, the same error classes and messages.  It exists so the reference's Python engine
// (Scheduler, PagedKVCacheManager) can run unchanged on top of this library; the engine's batched
// device path uses the device block pool (pool_api.cu) instead.
#include <cstdint>
#include <cstdlib>
#include <deque>
#include <limits>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "b200_paged.h"

namespace {
thread_local std::string g_msg;
int err(int code, const std::string& m) {
  g_msg = m;
  return code;
}
}  // namespace

struct B200HostAllocator {
  int64_t total = 0, tokens_per_block = 0, bytes_per_token = 0, total_cpu = 0;
  std::deque<int32_t> free_q;
  std::vector<int32_t> refcount;
  std::vector<uint8_t> cpu_used;
  std::vector<int32_t> cpu_free;  // used as a stack (back = next)
  std::unordered_map<int32_t, int32_t> gpu_to_cpu;
  uint8_t* host_pool = nullptr;
  int64_t block_bytes = 0;
  mutable std::mutex mu;

  bool valid_gpu(int32_t id) const { return id >= 0 && static_cast<int64_t>(id) < total; }

  void drop_stale_mapping(int32_t gpu) {
    auto it = gpu_to_cpu.find(gpu);
    if (it == gpu_to_cpu.end()) return;
    const int32_t cpu = it->second;
    if (cpu >= 0 && cpu < total_cpu && cpu_used[cpu]) {
      cpu_used[cpu] = 0;
      cpu_free.push_back(cpu);
    }
    gpu_to_cpu.erase(it);
  }

  void erase_mapping_to(int32_t cpu) {
    for (auto it = gpu_to_cpu.begin(); it != gpu_to_cpu.end(); ++it)
      if (it->second == cpu) {
        gpu_to_cpu.erase(it);
        return;
      }
  }
};

extern "C" {

const char* b200_host_last_message(void) { return g_msg.c_str(); }

int b200_host_allocator_create(int64_t total_blocks, int64_t tokens_per_block,
                               int64_t bytes_per_token, int64_t total_cpu_blocks,
                               B200HostAllocator** out) {
  if (out == nullptr) return err(B200_ERR_INVALID_ARGUMENT, "null out");
  *out = nullptr;
  if (total_blocks < 0 || total_cpu_blocks < 0 || total_blocks > std::numeric_limits<int32_t>::max())
    return err(B200_ERR_INVALID_ARGUMENT, "block counts must be non-negative");
  if (tokens_per_block <= 0) return err(B200_ERR_INVALID_ARGUMENT, "tokens_per_block must be greater than 0");
  if (bytes_per_token <= 0) return err(B200_ERR_INVALID_ARGUMENT, "bytes_per_token must be greater than 0");
  if (tokens_per_block > std::numeric_limits<int64_t>::max() / bytes_per_token)
    return err(B200_ERR_RUNTIME, "tokens_per_block * bytes_per_token overflows size_t");
  auto* a = new B200HostAllocator();
  a->total = total_blocks;
  a->tokens_per_block = tokens_per_block;
  a->bytes_per_token = bytes_per_token;
  a->total_cpu = total_cpu_blocks;
  a->block_bytes = tokens_per_block * bytes_per_token;
  if (total_cpu_blocks > 0) {
    if (total_cpu_blocks > std::numeric_limits<int64_t>::max() / a->block_bytes) {
      delete a;
      return err(B200_ERR_RUNTIME, "total_cpu_blocks * block_size_bytes overflows size_t");
    }
    void* p = nullptr;
    if (posix_memalign(&p, 4096, static_cast<size_t>(total_cpu_blocks * a->block_bytes)) != 0 ||
        p == nullptr) {
      delete a;
      return err(B200_ERR_OUT_OF_MEMORY, "std::bad_alloc");
    }
    a->host_pool = static_cast<uint8_t*>(p);
  }
  a->refcount.assign(static_cast<size_t>(total_blocks), 0);
  for (int64_t i = 0; i < total_blocks; ++i) a->free_q.push_back(static_cast<int32_t>(i));
  a->cpu_used.assign(static_cast<size_t>(total_cpu_blocks), 0);
  for (int64_t i = 0; i < total_cpu_blocks; ++i) a->cpu_free.push_back(static_cast<int32_t>(i));
  *out = a;
  return B200_OK;
}

void b200_host_allocator_destroy(B200HostAllocator* a) {
  if (a == nullptr) return;
  free(a->host_pool);
  delete a;
}

int b200_host_allocate_block(B200HostAllocator* a, int32_t* out_id) {
  std::lock_guard<std::mutex> g(a->mu);
  if (a->free_q.empty())
    return err(B200_ERR_OUT_OF_MEMORY, "Out of Memory: No free VRAM pages available in KV-Cache pool!");
  const int32_t id = a->free_q.front();
  a->free_q.pop_front();
  a->drop_stale_mapping(id);
  a->refcount[id] = 1;
  *out_id = id;
  return B200_OK;
}

int b200_host_allocate_blocks(B200HostAllocator* a, int64_t count, int32_t* out_ids) {
  std::lock_guard<std::mutex> g(a->mu);
  if (count < 0) return err(B200_ERR_INVALID_ARGUMENT, "count must be non-negative");
  if (static_cast<int64_t>(a->free_q.size()) < count)
    return err(B200_ERR_OUT_OF_MEMORY,
               "Out of Memory: Not enough free blocks available in KV-Cache pool!");
  for (int64_t i = 0; i < count; ++i) {
    const int32_t id = a->free_q.front();
    a->free_q.pop_front();
    a->drop_stale_mapping(id);
    a->refcount[id] = 1;
    out_ids[i] = id;
  }
  return B200_OK;
}

int b200_host_share_block(B200HostAllocator* a, int32_t id) {
  std::lock_guard<std::mutex> g(a->mu);
  if (!a->valid_gpu(id)) return err(B200_ERR_OUT_OF_RANGE, "Block ID out of range: " + std::to_string(id));
  if (a->refcount[id] <= 0)
    return err(B200_ERR_RUNTIME, "Cannot share unallocated block " + std::to_string(id));
  a->refcount[id] += 1;
  return B200_OK;
}

int b200_host_free_block(B200HostAllocator* a, int32_t id) {
  std::lock_guard<std::mutex> g(a->mu);
  if (!a->valid_gpu(id)) return err(B200_ERR_OUT_OF_RANGE, "Block ID out of range: " + std::to_string(id));
  auto it = a->gpu_to_cpu.find(id);
  if (it != a->gpu_to_cpu.end()) {
    const int32_t cpu = it->second;
    if (a->refcount[id] == 0 && cpu >= 0 && cpu < a->total_cpu && a->cpu_used[cpu]) {
      // a swapped-out block: freeing it returns its host copy
      a->cpu_used[cpu] = 0;
      a->cpu_free.push_back(cpu);
      a->gpu_to_cpu.erase(it);
      return B200_OK;
    }
  }
  if (a->refcount[id] <= 0)
    return err(B200_ERR_RUNTIME,
               "Double-free or free on unallocated block detected: ID " + std::to_string(id));
  a->refcount[id] -= 1;
  if (a->refcount[id] == 0) a->free_q.push_back(id);
  return B200_OK;
}

int b200_host_swap_out(B200HostAllocator* a, int32_t gpu, int32_t* out_cpu) {
  std::lock_guard<std::mutex> g(a->mu);
  if (!a->valid_gpu(gpu)) return err(B200_ERR_OUT_OF_RANGE, "Block ID out of range: " + std::to_string(gpu));
  if (a->refcount[gpu] != 1) return err(B200_ERR_RUNTIME, "Cannot swap out block with ref_count != 1");
  if (a->total_cpu == 0)
    return err(B200_ERR_RUNTIME, "Swap unsupported: no host pool configured (total_cpu_blocks == 0)");
  if (a->cpu_free.empty()) return err(B200_ERR_RUNTIME, "OOM: Host RAM Block Pool exhausted during swap out");
  const int32_t cpu = a->cpu_free.back();
  a->cpu_free.pop_back();
  a->cpu_used[cpu] = 1;
  a->refcount[gpu] = 0;
  a->free_q.push_back(gpu);
  a->gpu_to_cpu[gpu] = cpu;
  *out_cpu = cpu;
  return B200_OK;
}

int b200_host_swap_in(B200HostAllocator* a, int32_t cpu, int32_t* out_gpu) {
  std::lock_guard<std::mutex> g(a->mu);
  if (a->total_cpu == 0)
    return err(B200_ERR_RUNTIME, "Swap unsupported: no host pool configured (total_cpu_blocks == 0)");
  if (cpu < 0 || cpu >= a->total_cpu)
    return err(B200_ERR_OUT_OF_RANGE, "CPU block ID out of range: " + std::to_string(cpu));
  if (!a->cpu_used[cpu])
    return err(B200_ERR_RUNTIME, "CPU block " + std::to_string(cpu) + " is not currently swapped out");
  if (a->free_q.empty()) return err(B200_ERR_RUNTIME, "OOM: No free VRAM blocks available to swap in");
  const int32_t gpu = a->free_q.front();
  a->free_q.pop_front();
  a->refcount[gpu] = 1;
  a->cpu_used[cpu] = 0;
  a->cpu_free.push_back(cpu);
  a->erase_mapping_to(cpu);
  *out_gpu = gpu;
  return B200_OK;
}

int b200_host_get_cpu_block_id(B200HostAllocator* a, int32_t gpu, int32_t* out) {
  std::lock_guard<std::mutex> g(a->mu);
  if (!a->valid_gpu(gpu)) return err(B200_ERR_OUT_OF_RANGE, "Block ID out of range: " + std::to_string(gpu));
  auto it = a->gpu_to_cpu.find(gpu);
  if (it == a->gpu_to_cpu.end())
    return err(B200_ERR_RUNTIME, "Block " + std::to_string(gpu) + " is not swapped out");
  *out = it->second;
  return B200_OK;
}

int b200_host_release_swapped_block(B200HostAllocator* a, int32_t cpu) {
  std::lock_guard<std::mutex> g(a->mu);
  if (a->total_cpu == 0)
    return err(B200_ERR_RUNTIME, "Swap unsupported: no host pool configured (total_cpu_blocks == 0)");
  if (cpu < 0 || cpu >= a->total_cpu)
    return err(B200_ERR_OUT_OF_RANGE, "CPU block ID out of range: " + std::to_string(cpu));
  if (!a->cpu_used[cpu])
    return err(B200_ERR_RUNTIME, "CPU block " + std::to_string(cpu) + " is not currently swapped out");
  a->cpu_used[cpu] = 0;
  a->cpu_free.push_back(cpu);
  a->erase_mapping_to(cpu);
  return B200_OK;
}

int b200_host_get_host_ptr(B200HostAllocator* a, int32_t cpu, uint64_t* out) {
  std::lock_guard<std::mutex> g(a->mu);
  if (cpu < 0 || cpu >= a->total_cpu)
    return err(B200_ERR_OUT_OF_RANGE, "CPU block ID out of range: " + std::to_string(cpu));
  *out = a->cpu_used[cpu] ? reinterpret_cast<uint64_t>(a->host_pool + cpu * a->block_bytes) : 0;
  return B200_OK;
}

int b200_host_get_device_ptr(B200HostAllocator* a, int32_t gpu, uint64_t* out) {
  std::lock_guard<std::mutex> g(a->mu);
  if (!a->valid_gpu(gpu)) return err(B200_ERR_OUT_OF_RANGE, "Block ID out of range: " + std::to_string(gpu));
  *out = reinterpret_cast<uint64_t>(a->host_pool);  // host pool base (0 without a host pool)
  return B200_OK;
}

int64_t b200_host_num_free_blocks(const B200HostAllocator* a) {
  std::lock_guard<std::mutex> g(a->mu);
  return static_cast<int64_t>(a->free_q.size());
}
int64_t b200_host_num_free_cpu_blocks(const B200HostAllocator* a) {
  std::lock_guard<std::mutex> g(a->mu);
  return static_cast<int64_t>(a->cpu_free.size());
}
int64_t b200_host_total_blocks(const B200HostAllocator* a) { return a->total; }
int64_t b200_host_block_size(const B200HostAllocator* a) { return a->tokens_per_block; }
int64_t b200_host_bytes_per_token(const B200HostAllocator* a) { return a->bytes_per_token; }
int64_t b200_host_pool_bytes(const B200HostAllocator* a) {
  return a->total_cpu * a->tokens_per_block * a->bytes_per_token;
}
double b200_host_utilization(const B200HostAllocator* a) {
  std::lock_guard<std::mutex> g(a->mu);
  if (a->total == 0) return 0.0;
  return 100.0 * static_cast<double>(a->total - static_cast<int64_t>(a->free_q.size())) /
         static_cast<double>(a->total);
}

}  // extern "C"
