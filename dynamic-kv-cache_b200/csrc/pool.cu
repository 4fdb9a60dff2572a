// Growable device pools: virtual address space reserved once, physical memory
// mapped onto its front as the pool grows (CUDA virtual memory management).
//
// The reference grows a precision pool by allocating a larger tensor and copying
// every old row into it (GPUCache.reserve, src/gpu_cache.py:44-59). With the pools
// paged (pool_row in dkv_common.cuh: page p of every (layer, K|V, head) block side
// by side), a pool of more rows is the same pool with more pages at the end, so
// growth here maps the new pages behind the old ones: the base address never
// moves, no row is copied, and descriptors captured in a CUDA graph stay valid.
//
// The driver entry points are looked up through the runtime
// (cudaGetDriverEntryPointByVersion), so the library links no libcuda.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <vector>

#include "dkv.h"

namespace dkv {
int api_fail(int code, const char* fmt, ...);
int api_ok();
}  // namespace dkv

struct dkv_pool {
  int device;
  CUdeviceptr base;
  uint64_t reserved;  // bytes of address space
  uint64_t mapped;    // bytes mapped from base, a multiple of the granularity
  uint64_t granularity;
  struct Chunk {
    uint64_t offset, bytes;
    CUmemGenericAllocationHandle handle;
  };
  std::vector<Chunk> chunks;
};

namespace {

using FnGranularity = CUresult (*)(size_t*, const CUmemAllocationProp*, CUmemAllocationGranularity_flags);
using FnReserve = CUresult (*)(CUdeviceptr*, size_t, size_t, CUdeviceptr, unsigned long long);
using FnFree = CUresult (*)(CUdeviceptr, size_t);
using FnCreate = CUresult (*)(CUmemGenericAllocationHandle*, size_t, const CUmemAllocationProp*,
                              unsigned long long);
using FnRelease = CUresult (*)(CUmemGenericAllocationHandle);
using FnMap = CUresult (*)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long);
using FnUnmap = CUresult (*)(CUdeviceptr, size_t);
using FnSetAccess = CUresult (*)(CUdeviceptr, size_t, const CUmemAccessDesc*, size_t);

struct Driver {
  FnGranularity granularity = nullptr;
  FnReserve reserve = nullptr;
  FnFree free = nullptr;
  FnCreate create = nullptr;
  FnRelease release = nullptr;
  FnMap map = nullptr;
  FnUnmap unmap = nullptr;
  FnSetAccess set_access = nullptr;
  bool loaded = false;
};

std::mutex g_driver_mutex;
Driver g_driver;

template <class F>
bool lookup(const char* name, F& fn) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  if (cudaGetDriverEntryPointByVersion(name, &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || p == nullptr)
    return false;
  fn = reinterpret_cast<F>(p);
  return true;
}

const Driver* driver() {
  std::lock_guard<std::mutex> lock(g_driver_mutex);
  if (!g_driver.loaded) {
    Driver d;
    if (!(lookup("cuMemGetAllocationGranularity", d.granularity) && lookup("cuMemAddressReserve", d.reserve) &&
          lookup("cuMemAddressFree", d.free) && lookup("cuMemCreate", d.create) &&
          lookup("cuMemRelease", d.release) && lookup("cuMemMap", d.map) && lookup("cuMemUnmap", d.unmap) &&
          lookup("cuMemSetAccess", d.set_access)))
      return nullptr;
    d.loaded = true;
    g_driver = d;
  }
  return &g_driver;
}

CUmemAllocationProp device_prop(int device) {
  CUmemAllocationProp prop = {};
  prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  prop.location.id = device;
  return prop;
}

// Makes `device` current for the driver calls and restores the caller's device.
class DeviceScope {
 public:
  explicit DeviceScope(int device) {
    ok_ = cudaGetDevice(&previous_) == cudaSuccess && cudaSetDevice(device) == cudaSuccess &&
          cudaFree(nullptr) == cudaSuccess;  // the primary context exists and is current
  }
  ~DeviceScope() {
    if (previous_ >= 0) cudaSetDevice(previous_);
  }
  bool ok() const { return ok_; }

 private:
  int previous_ = -1;
  bool ok_ = false;
};

uint64_t round_up(uint64_t x, uint64_t g) { return (x + g - 1) / g * g; }

}  // namespace

extern "C" {

uint64_t dkv_pool_granularity(int32_t device) {
  const Driver* d = driver();
  if (d == nullptr) return 0;
  DeviceScope scope(device);
  if (!scope.ok()) return 0;
  const CUmemAllocationProp prop = device_prop(device);
  size_t g = 0;
  if (d->granularity(&g, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED) != CUDA_SUCCESS) return 0;
  return g;
}

int dkv_pool_create(int32_t device, uint64_t reserve_bytes, dkv_pool** pool) {
  if (pool == nullptr) return dkv::api_fail(DKV_EINVAL, "pool output pointer is NULL");
  *pool = nullptr;
  if (reserve_bytes == 0) return dkv::api_fail(DKV_EINVAL, "pool reservation must be positive");
  const Driver* d = driver();
  if (d == nullptr) return dkv::api_fail(DKV_ECUDA, "CUDA driver has no virtual memory management entry points");
  DeviceScope scope(device);
  if (!scope.ok()) return dkv::api_fail(DKV_ECUDA, "cannot make device %d current", device);
  const CUmemAllocationProp prop = device_prop(device);
  size_t g = 0;
  if (d->granularity(&g, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED) != CUDA_SUCCESS || g == 0)
    return dkv::api_fail(DKV_ECUDA, "no allocation granularity for device %d", device);
  const uint64_t bytes = round_up(reserve_bytes, g);
  CUdeviceptr base = 0;
  if (d->reserve(&base, bytes, g, 0, 0) != CUDA_SUCCESS)
    return dkv::api_fail(DKV_ECUDA, "cannot reserve %llu bytes of device address space",
                         static_cast<unsigned long long>(bytes));
  dkv_pool* p = new dkv_pool{device, base, bytes, 0, g, {}};
  *pool = p;
  return dkv::api_ok();
}

int dkv_pool_map(dkv_pool* pool, uint64_t bytes) {
  if (pool == nullptr) return dkv::api_fail(DKV_EINVAL, "pool is NULL");
  const uint64_t target = round_up(bytes, pool->granularity);
  if (target <= pool->mapped) return dkv::api_ok();
  if (target > pool->reserved)
    return dkv::api_fail(DKV_ECAPACITY, "pool needs %llu bytes but reserved %llu",
                         static_cast<unsigned long long>(target), static_cast<unsigned long long>(pool->reserved));
  const Driver* d = driver();
  if (d == nullptr) return dkv::api_fail(DKV_ECUDA, "CUDA driver has no virtual memory management entry points");
  DeviceScope scope(pool->device);
  if (!scope.ok()) return dkv::api_fail(DKV_ECUDA, "cannot make device %d current", pool->device);
  const uint64_t size = target - pool->mapped;
  const CUmemAllocationProp prop = device_prop(pool->device);
  CUmemGenericAllocationHandle h = 0;
  if (d->create(&h, size, &prop, 0) != CUDA_SUCCESS)
    return dkv::api_fail(DKV_ECUDA, "out of device memory growing a pool by %llu bytes",
                         static_cast<unsigned long long>(size));
  const CUdeviceptr at = pool->base + pool->mapped;
  if (d->map(at, size, 0, h, 0) != CUDA_SUCCESS) {
    d->release(h);
    return dkv::api_fail(DKV_ECUDA, "cannot map %llu bytes into a pool", static_cast<unsigned long long>(size));
  }
  CUmemAccessDesc access = {};
  access.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  access.location.id = pool->device;
  access.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  if (d->set_access(at, size, &access, 1) != CUDA_SUCCESS) {
    d->unmap(at, size);
    d->release(h);
    return dkv::api_fail(DKV_ECUDA, "cannot enable access to a pool's new pages");
  }
  pool->chunks.push_back({pool->mapped, size, h});
  pool->mapped = target;
  return dkv::api_ok();
}

void* dkv_pool_base(const dkv_pool* pool) {
  return pool == nullptr ? nullptr : reinterpret_cast<void*>(static_cast<uintptr_t>(pool->base));
}

uint64_t dkv_pool_mapped_bytes(const dkv_pool* pool) { return pool == nullptr ? 0 : pool->mapped; }

uint64_t dkv_pool_reserved_bytes(const dkv_pool* pool) { return pool == nullptr ? 0 : pool->reserved; }

int dkv_pool_destroy(dkv_pool* pool) {
  if (pool == nullptr) return dkv::api_ok();
  const Driver* d = driver();
  if (d == nullptr) return dkv::api_fail(DKV_ECUDA, "CUDA driver has no virtual memory management entry points");
  DeviceScope scope(pool->device);
  if (!scope.ok()) return dkv::api_fail(DKV_ECUDA, "cannot make device %d current", pool->device);
  // work still queued on any stream may read the pages: let it finish first
  if (cudaDeviceSynchronize() != cudaSuccess) return dkv::api_fail(DKV_ECUDA, "device synchronisation failed");
  bool clean = true;
  for (const auto& c : pool->chunks) {
    clean &= d->unmap(pool->base + c.offset, c.bytes) == CUDA_SUCCESS;
    clean &= d->release(c.handle) == CUDA_SUCCESS;
  }
  clean &= d->free(pool->base, pool->reserved) == CUDA_SUCCESS;
  delete pool;
  return clean ? dkv::api_ok() : dkv::api_fail(DKV_ECUDA, "pool release reported an error");
}

}  // extern "C"
