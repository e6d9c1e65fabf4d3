// Native row arena: a range of virtual addresses reserved once for max_rows fixed-size rows, of which a prefix is
// backed by physical memory in chunks. Growing maps chunks at the end of the backed prefix; shrinking unmaps the
// chunks that lie entirely beyond the rows kept and returns them to the driver. Row addresses never change, so
// kernels that address rows through slot tables or address tables -- and CUDA graphs that captured them -- stay
// valid across resizes (the behaviour of RowArena, gemv/row_arena.py:34-123, here as C++ behind the C ABI).
//
// The driver's virtual-memory calls are reached through a table of function pointers: the real one comes from the
// runtime's driver entry-point query (the library links no driver library); tests pass a fake table and check the
// chunk bookkeeping on a machine without a GPU.
#include <cudaTypedefs.h>
#include <new>

#include "../../include/w2a16_moe.h"
#include "w2a16_kernels.h"

struct w2a16_arena {
  w2a16_vmm_driver drv;
  int device;
  int64_t row_bytes, max_rows, chunk_bytes, va_bytes;
  uint64_t base;
  uint64_t* handles;      // handles[i] backs [base + i * chunk_bytes, + chunk_bytes)
  int64_t nchunks, cap_chunks;
};

namespace {

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

template <class F>
F entry(const char* name) {
  void* f = nullptr;
  cudaDriverEntryPointQueryResult q{};
  if (cudaGetDriverEntryPoint(name, &f, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<F>(f);
}

CUmemAllocationProp device_prop(int device) {
  CUmemAllocationProp p{};
  p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  p.location.id = device;
  return p;
}

// The real driver table: thin adapters from the function-pointer signatures of w2a16_vmm_driver to the CUDA
// driver API (each returns the driver's CUresult, 0 = success).
struct Real {
  static PFN_cuMemGetAllocationGranularity_v10020 gran;
  static PFN_cuMemAddressReserve_v10020 reserve;
  static PFN_cuMemAddressFree_v10020 addr_free;
  static PFN_cuMemCreate_v10020 create;
  static PFN_cuMemRelease_v10020 release;
  static PFN_cuMemMap_v10020 map;
  static PFN_cuMemUnmap_v10020 unmap;
  static PFN_cuMemSetAccess_v10020 set_access;
  static bool load() {
    static const bool ok = [] {
      gran = entry<PFN_cuMemGetAllocationGranularity_v10020>("cuMemGetAllocationGranularity");
      reserve = entry<PFN_cuMemAddressReserve_v10020>("cuMemAddressReserve");
      addr_free = entry<PFN_cuMemAddressFree_v10020>("cuMemAddressFree");
      create = entry<PFN_cuMemCreate_v10020>("cuMemCreate");
      release = entry<PFN_cuMemRelease_v10020>("cuMemRelease");
      map = entry<PFN_cuMemMap_v10020>("cuMemMap");
      unmap = entry<PFN_cuMemUnmap_v10020>("cuMemUnmap");
      set_access = entry<PFN_cuMemSetAccess_v10020>("cuMemSetAccess");
      return gran && reserve && addr_free && create && release && map && unmap && set_access;
    }();
    return ok;
  }
  static int granularity(void*, int device, uint64_t* out) {
    CUmemAllocationProp p = device_prop(device);
    size_t g = 0;
    const int r = (int)gran(&g, &p, CU_MEM_ALLOC_GRANULARITY_MINIMUM);
    *out = g;
    return r;
  }
  static int reserve_va(void*, uint64_t bytes, uint64_t* base) {
    CUdeviceptr p = 0;
    const int r = (int)reserve(&p, bytes, 0, 0, 0);
    *base = (uint64_t)p;
    return r;
  }
  static int free_va(void*, uint64_t base, uint64_t bytes) { return (int)addr_free((CUdeviceptr)base, bytes); }
  static int create_chunk(void*, int device, uint64_t bytes, uint64_t* handle) {
    CUmemAllocationProp p = device_prop(device);
    CUmemGenericAllocationHandle h = 0;
    const int r = (int)create(&h, bytes, &p, 0);
    *handle = (uint64_t)h;
    return r;
  }
  static int release_chunk(void*, uint64_t handle) { return (int)release((CUmemGenericAllocationHandle)handle); }
  static int map_chunk(void*, int device, uint64_t va, uint64_t bytes, uint64_t handle) {
    int r = (int)map((CUdeviceptr)va, bytes, 0, (CUmemGenericAllocationHandle)handle, 0);
    if (r != 0) return r;
    CUmemAccessDesc d{};
    d.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    d.location.id = device;
    d.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    r = (int)set_access((CUdeviceptr)va, bytes, &d, 1);
    if (r != 0) unmap((CUdeviceptr)va, bytes);
    return r;
  }
  static int unmap_chunk(void*, uint64_t va, uint64_t bytes) { return (int)unmap((CUdeviceptr)va, bytes); }
};
PFN_cuMemGetAllocationGranularity_v10020 Real::gran = nullptr;
PFN_cuMemAddressReserve_v10020 Real::reserve = nullptr;
PFN_cuMemAddressFree_v10020 Real::addr_free = nullptr;
PFN_cuMemCreate_v10020 Real::create = nullptr;
PFN_cuMemRelease_v10020 Real::release = nullptr;
PFN_cuMemMap_v10020 Real::map = nullptr;
PFN_cuMemUnmap_v10020 Real::unmap = nullptr;
PFN_cuMemSetAccess_v10020 Real::set_access = nullptr;

w2a16_vmm_driver real_driver() {
  w2a16_vmm_driver d{};
  d.ctx = nullptr;
  d.granularity = Real::granularity;
  d.reserve = Real::reserve_va;
  d.free_va = Real::free_va;
  d.create = Real::create_chunk;
  d.release = Real::release_chunk;
  d.map = Real::map_chunk;
  d.unmap = Real::unmap_chunk;
  return d;
}

bool complete(const w2a16_vmm_driver* d) {
  return d && d->granularity && d->reserve && d->free_va && d->create && d->release && d->map && d->unmap;
}

}  // namespace

extern "C" {

int w2a16_arena_create_with_driver(const w2a16_vmm_driver* drv, int device, int64_t row_bytes, int64_t max_rows,
                                   int64_t chunk_bytes, w2a16_arena** out) {
  if (!out) return W2A16_ERR_ARG;
  *out = nullptr;
  if (!complete(drv) || device < 0 || row_bytes <= 0 || max_rows <= 0 || chunk_bytes < 0) return W2A16_ERR_ARG;
  uint64_t gran = 0;
  if (drv->granularity(drv->ctx, device, &gran) != 0 || gran == 0) return W2A16_ERR_DEVICE;
  const int64_t chunk = round_up(chunk_bytes > 0 ? chunk_bytes : (int64_t)4 << 20, (int64_t)gran);
  const int64_t va = round_up(row_bytes * max_rows, chunk);
  w2a16_arena* a = new (std::nothrow) w2a16_arena{};
  if (!a) return W2A16_ERR_MEMORY;
  a->drv = *drv;
  a->device = device;
  a->row_bytes = row_bytes;
  a->max_rows = max_rows;
  a->chunk_bytes = chunk;
  a->va_bytes = va;
  a->cap_chunks = va / chunk;
  a->handles = new (std::nothrow) uint64_t[a->cap_chunks];
  if (!a->handles) {
    delete a;
    return W2A16_ERR_MEMORY;
  }
  if (drv->reserve(drv->ctx, (uint64_t)va, &a->base) != 0 || a->base == 0) {
    delete[] a->handles;
    delete a;
    return W2A16_ERR_MEMORY;
  }
  *out = a;
  return W2A16_OK;
}

int w2a16_arena_create(int device, int64_t row_bytes, int64_t max_rows, int64_t chunk_bytes, w2a16_arena** out) {
  if (!Real::load()) return W2A16_ERR_DEVICE;
  const w2a16_vmm_driver d = real_driver();
  return w2a16_arena_create_with_driver(&d, device, row_bytes, max_rows, chunk_bytes, out);
}

int w2a16_arena_ensure_rows(w2a16_arena* a, int64_t n, int64_t* mapped_bytes) {
  if (mapped_bytes) *mapped_bytes = 0;
  if (!a || n < 0) return W2A16_ERR_ARG;
  if (n > a->max_rows) n = a->max_rows;
  const int64_t want = n > 0 ? (n * a->row_bytes + a->chunk_bytes - 1) / a->chunk_bytes : 0;
  while (a->nchunks < want) {
    uint64_t h = 0;
    if (a->drv.create(a->drv.ctx, a->device, (uint64_t)a->chunk_bytes, &h) != 0) return W2A16_ERR_MEMORY;
    const uint64_t va = a->base + (uint64_t)(a->nchunks * a->chunk_bytes);
    if (a->drv.map(a->drv.ctx, a->device, va, (uint64_t)a->chunk_bytes, h) != 0) {
      a->drv.release(a->drv.ctx, h);
      return W2A16_ERR_MEMORY;
    }
    a->handles[a->nchunks++] = h;
    if (mapped_bytes) *mapped_bytes += a->chunk_bytes;
  }
  return W2A16_OK;
}

int w2a16_arena_shrink_rows(w2a16_arena* a, int64_t n, int64_t* freed_bytes) {
  if (freed_bytes) *freed_bytes = 0;
  if (!a || n < 0) return W2A16_ERR_ARG;
  if (n > a->max_rows) n = a->max_rows;
  const int64_t keep = n > 0 ? (n * a->row_bytes + a->chunk_bytes - 1) / a->chunk_bytes : 0;
  while (a->nchunks > keep) {
    const int64_t i = a->nchunks - 1;
    const uint64_t va = a->base + (uint64_t)(i * a->chunk_bytes);
    if (a->drv.unmap(a->drv.ctx, va, (uint64_t)a->chunk_bytes) != 0) return W2A16_ERR_DEVICE;
    a->drv.release(a->drv.ctx, a->handles[i]);
    a->nchunks = i;
    if (freed_bytes) *freed_bytes += a->chunk_bytes;
  }
  return W2A16_OK;
}

uint64_t w2a16_arena_base(const w2a16_arena* a) { return a ? a->base : 0; }

int64_t w2a16_arena_backed_rows(const w2a16_arena* a) {
  if (!a) return 0;
  const int64_t r = a->nchunks * a->chunk_bytes / a->row_bytes;
  return r < a->max_rows ? r : a->max_rows;
}

int64_t w2a16_arena_chunk_bytes(const w2a16_arena* a) { return a ? a->chunk_bytes : 0; }

int w2a16_arena_destroy(w2a16_arena* a) {
  if (!a) return W2A16_OK;
  int st = w2a16_arena_shrink_rows(a, 0, nullptr);
  if (a->drv.free_va(a->drv.ctx, a->base, (uint64_t)a->va_bytes) != 0 && st == W2A16_OK) st = W2A16_ERR_DEVICE;
  delete[] a->handles;
  delete a;
  return st;
}

}  // extern "C"
