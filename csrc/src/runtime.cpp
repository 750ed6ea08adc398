// runtime.cpp -- symmetric memory over CUDA VMM / IPC, NVLS multicast, device contexts.
#include "gicc/runtime.hpp"

#include "gicc/config.hpp"

#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <thread>

#include "gicc/driver.hpp"
#include "gicc/host_util.hpp"

namespace gicc {

namespace {
size_t round_up(size_t x, size_t g) { return (x + g - 1) / g * g; }

enum Kind : int32_t { K_VMM = 0, K_IPC = 1, K_HOST = 2 };

struct RegionMeta {
  int32_t kind;
  int32_t multicast;
  uint64_t size;
  uint64_t alloc_size;
  uint64_t ipc_offset;
  cudaIpcMemHandle_t ipc;
};

double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}
}  // namespace

struct Runtime::Region {
  void* ptr = nullptr;
  size_t size = 0;
  size_t alloc_size = 0;
  int kind = K_VMM;
  bool owned = false;  // allocated by alloc()
  bool multicast = false;
  CUmemGenericAllocationHandle handle = 0;
  int export_fd = -1;
  cudaIpcMemHandle_t ipc{};
  size_t ipc_offset = 0;
  Buffer buf{};
  // after exchange
  bool imported = false;
  std::vector<void*> peer_ptr;  // [rank] address usable in this process
  std::vector<CUmemGenericAllocationHandle> peer_handle;
  std::vector<void*> ipc_opened;  // IPC bases to close
  std::vector<size_t> peer_size;
  // multicast
  CUmemGenericAllocationHandle mc_handle = 0;
  void* mc_ptr = nullptr;
  size_t mc_size = 0;
};

Runtime::Runtime() : Runtime(std::make_shared<Bootstrap>()) {}

Runtime::Runtime(std::shared_ptr<Bootstrap> boot, RuntimeOptions opt) : boot_(std::move(boot)) { init(opt); }

Runtime::Runtime(Bootstrap& boot, RuntimeOptions opt) : boot_(&boot, [](Bootstrap*) {}) { init(opt); }

void Runtime::init(RuntimeOptions opt) {
  NvtxRange nvtx("gicc::Runtime::init");
  const Config cfg = config();  // validates every GICC_* variable (throws on a bad one)
  set_log_rank(boot_->rank());
  if (boot_->rank() == 0) log(LOG_INFO, "%s", cfg.summary().c_str());
  if (cfg.signal_heap_bytes) opt.signal_heap_bytes = cfg.signal_heap_bytes;
  int ndev = 0;
  GICC_CUDA(cudaGetDeviceCount(&ndev));
  if (ndev <= 0) throw std::runtime_error("gicc::Runtime: no CUDA device");
  device_ = opt.device >= 0 ? opt.device : boot_->local_rank() % ndev;
  GICC_CUDA(cudaSetDevice(device_));
  GICC_CUDA(cudaFree(nullptr));  // make the primary context current
  GICC_DRV(driver().DeviceGet(&cudev_, device_));
  cudaDeviceProp prop{};
  GICC_CUDA(cudaGetDeviceProperties(&prop, device_));
  gpu_name_ = prop.name;
  int khz = 0;
  cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, device_);
  clock_khz_ = khz;
  int mc = 0;
  driver().DeviceGetAttribute(&mc, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, cudev_);
  mc_supported_ = opt.enable_multicast && mc != 0 && size() > 1 && driver().MulticastCreate != nullptr &&
                  !cfg.disable_nvls;
  // every rank must agree on NVLS use
  auto all = boot_->allgather_fixed<int>(mc_supported_ ? 1 : 0);
  for (int v : all) mc_supported_ = mc_supported_ && v;
  timeout_ns_ = cfg.timeout_ms * 1000000ull;
  err_ = device_error_record();

  CUmemAllocationProp p{};
  p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  p.location.id = device_;
  p.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  size_t g = 0;
  GICC_DRV(driver().MemGetAllocationGranularity(&g, &p, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED));
  granularity_ = std::max<size_t>(g, 2u << 20);

  // host op queue (mapped pinned memory: the host fills it, flush() runs it)
  void* h = nullptr;
  GICC_CUDA(cudaHostAlloc(&h, sizeof(OpTable) + GICC_POOL_SIZE * sizeof(uint64_t), cudaHostAllocMapped));
  std::memset(h, 0, sizeof(OpTable) + GICC_POOL_SIZE * sizeof(uint64_t));
  ops_host_ = static_cast<OpTable*>(h);
  completion_host_ = reinterpret_cast<uint64_t*>(ops_host_ + 1);
  void* d = nullptr;
  GICC_CUDA(cudaHostGetDevicePointer(&d, h, 0));
  ops_dev_ = static_cast<OpTable*>(d);
  ops_host_->completion = reinterpret_cast<uint64_t*>(ops_dev_ + 1);
  ops_host_->epoch = op_epoch_;

  // signal heap: internal symmetric region (multicast-bound when NVLS is available)
  {
    auto r = std::make_unique<Region>();
    size_t sz = round_up(opt.signal_heap_bytes, granularity_);
    CUmemAllocationProp ap = p;
    GICC_DRV(driver().MemCreate(&r->handle, sz, &ap, 0));
    CUdeviceptr va = 0;
    GICC_DRV(driver().MemAddressReserve(&va, sz, granularity_, 0, 0));
    GICC_DRV(driver().MemMap(va, sz, 0, r->handle, 0));
    CUmemAccessDesc acc{};
    acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    acc.location.id = device_;
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    GICC_DRV(driver().MemSetAccess(va, sz, &acc, 1));
    GICC_CUDA(cudaMemset(reinterpret_cast<void*>(va), 0, sz));
    GICC_CUDA(cudaDeviceSynchronize());
    r->ptr = reinterpret_cast<void*>(va);
    r->size = r->alloc_size = sz;
    r->kind = K_VMM;
    r->owned = true;
    r->multicast = mc_supported_;
    internal_.push_back(std::move(r));
    sig_words_ = sz / sizeof(uint64_t);
    import_new_regions(internal_, 0, 1 << 20);
  }
  boot_->barrier();
}

Runtime::~Runtime() {
  try {
    finalize();
  } catch (const std::exception& e) {
    std::fprintf(stderr, "[gicc] rank %d: error while releasing the runtime: %s\n", rank(), e.what());
  }
}

void Runtime::finalize() {
  NvtxRange nvtx("gicc::Runtime::finalize");
  if (finalized_) return;
  finalized_ = true;
  cudaSetDevice(device_);
  cudaDeviceSynchronize();
  for (void* p : dev_allocs_) cudaFree(p);
  dev_allocs_.clear();
  auto release = [&](std::vector<std::unique_ptr<Region>>& list) {
    for (auto& rp : list) {
      Region& r = *rp;
      if (r.mc_ptr) {
        driver().MemUnmap(reinterpret_cast<CUdeviceptr>(r.mc_ptr), r.mc_size);
        driver().MemAddressFree(reinterpret_cast<CUdeviceptr>(r.mc_ptr), r.mc_size);
        if (driver().MulticastUnbind) driver().MulticastUnbind(r.mc_handle, cudev_, 0, r.mc_size);
        driver().MemRelease(r.mc_handle);
      }
      for (size_t p = 0; p < r.peer_ptr.size(); ++p) {
        if ((int)p == rank() || !r.peer_ptr[p]) continue;
        if (r.kind == K_VMM) {
          driver().MemUnmap(reinterpret_cast<CUdeviceptr>(r.peer_ptr[p]), r.peer_size[p]);
          driver().MemAddressFree(reinterpret_cast<CUdeviceptr>(r.peer_ptr[p]), r.peer_size[p]);
          if (r.peer_handle[p]) driver().MemRelease(r.peer_handle[p]);
        }
      }
      for (void* b : r.ipc_opened) cudaIpcCloseMemHandle(b);
      if (r.export_fd >= 0) ::close(r.export_fd);
      if (r.owned) {
        driver().MemUnmap(reinterpret_cast<CUdeviceptr>(r.ptr), r.alloc_size);
        driver().MemAddressFree(reinterpret_cast<CUdeviceptr>(r.ptr), r.alloc_size);
        driver().MemRelease(r.handle);
      } else if (r.kind == K_HOST) {
        cudaHostUnregister(r.ptr);
      }
    }
    list.clear();
  };
  // Peers may still read our memory until everybody is done: barrier first.
  try {
    boot_->barrier();
  } catch (...) {
  }
  release(regions_);
  release(internal_);
  if (ops_host_) cudaFreeHost(ops_host_);
  ops_host_ = nullptr;
}

Buffer Runtime::alloc(size_t bytes, bool multicast) {
  NvtxRange nvtx("gicc::Runtime::alloc");
  if (regions_.size() >= (size_t)GICC_MAX_BUFS) throw std::runtime_error("gicc::Runtime::alloc: GICC_MAX_BUFS reached");
  auto r = std::make_unique<Region>();
  size_t g = granularity_;
  if (multicast && mc_supported_) {
    CUmulticastObjectProp mp{};
    mp.numDevices = (unsigned)size();
    mp.size = round_up(bytes, g);
    mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    size_t mg = 0;
    GICC_DRV(driver().MulticastGetGranularity(&mg, &mp, CU_MULTICAST_GRANULARITY_RECOMMENDED));
    g = std::max(g, mg);
  }
  const size_t sz = round_up(std::max<size_t>(bytes, 1), g);
  CUmemAllocationProp p{};
  p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  p.location.id = device_;
  p.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  GICC_DRV(driver().MemCreate(&r->handle, sz, &p, 0));
  CUdeviceptr va = 0;
  GICC_DRV(driver().MemAddressReserve(&va, sz, g, 0, 0));
  GICC_DRV(driver().MemMap(va, sz, 0, r->handle, 0));
  CUmemAccessDesc acc{};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device_;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  GICC_DRV(driver().MemSetAccess(va, sz, &acc, 1));
  GICC_CUDA(cudaMemset(reinterpret_cast<void*>(va), 0, sz));
  r->ptr = reinterpret_cast<void*>(va);
  r->size = bytes;
  r->alloc_size = sz;
  r->kind = K_VMM;
  r->owned = true;
  r->multicast = multicast && mc_supported_;
  const int idx = (int)regions_.size();
  r->buf = Buffer{r->ptr, bytes, (uint64_t)va, (uint32_t)idx, (uint32_t)idx, idx};
  regions_.push_back(std::move(r));
  return regions_.back()->buf;
}

Buffer Runtime::register_buffer(void* ptr, size_t size, bool is_device) {
  NvtxRange nvtx("gicc::Runtime::register_buffer");
  if (regions_.size() >= (size_t)GICC_MAX_BUFS)
    throw std::runtime_error("gicc::Runtime::register_buffer: GICC_MAX_BUFS reached");
  if (!ptr || !size) throw std::runtime_error("gicc::Runtime::register_buffer: empty buffer");
  auto r = std::make_unique<Region>();
  r->ptr = ptr;
  r->size = size;
  r->alloc_size = size;
  if (!is_device) {
    r->kind = K_HOST;
    cudaError_t e = cudaHostRegister(ptr, size, cudaHostRegisterMapped | cudaHostRegisterPortable);
    if (e != cudaSuccess && e != cudaErrorHostMemoryAlreadyRegistered) GICC_CUDA(e);
    cudaGetLastError();
  } else {
    // Is this one of our VMM mappings (or inside one)?  Otherwise treat it as cudaMalloc.
    CUdeviceptr base = 0;
    size_t bsz = 0;
    GICC_DRV(driver().MemGetAddressRange(&base, &bsz, reinterpret_cast<CUdeviceptr>(ptr)));
    bool vmm_owned = false;
    for (auto& o : regions_)
      if (o->owned && o->ptr == reinterpret_cast<void*>(base)) vmm_owned = true;
    if (vmm_owned) throw std::runtime_error("gicc::Runtime::register_buffer: memory from alloc() is registered already");
    r->kind = K_IPC;
    GICC_CUDA(cudaIpcGetMemHandle(&r->ipc, reinterpret_cast<void*>(base)));
    r->ipc_offset = reinterpret_cast<uintptr_t>(ptr) - (uintptr_t)base;
  }
  const int idx = (int)regions_.size();
  r->buf = Buffer{ptr, size, (uint64_t)(uintptr_t)ptr, (uint32_t)idx, (uint32_t)idx, idx};
  regions_.push_back(std::move(r));
  return regions_.back()->buf;
}

void Runtime::exchange() {
  NvtxRange nvtx("gicc::Runtime::exchange");
  std::vector<int32_t> kinds, mc;
  for (size_t i = exchanged_; i < regions_.size(); ++i) {
    kinds.push_back(regions_[i]->kind);
    mc.push_back(regions_[i]->multicast ? 1 : 0);
  }
  check_exchange_consistency(*boot_, kinds, mc);
  ++exchange_epoch_;
  import_new_regions(regions_, exchanged_, exchange_epoch_ * 1024);
  exchanged_ = regions_.size();
  boot_->barrier();
}

void check_exchange_consistency(Bootstrap& boot, const std::vector<int32_t>& kinds,
                                const std::vector<int32_t>& multicast) {
  if (kinds.size() != multicast.size()) throw std::invalid_argument("check_exchange_consistency: table sizes differ");
  const int mine = (int)kinds.size();
  // Counts first: a rank with a different count must not enter an allgather of another size.
  const auto counts = boot.allgather_fixed<int>(mine);
  for (int r = 0; r < boot.size(); ++r)
    if (counts[r] != mine)
      throw BootstrapError(GICC_EMISMATCH, "gicc::Runtime::exchange: rank " + std::to_string(r) + " registered " +
                                               std::to_string(counts[r]) + " buffers, rank " +
                                               std::to_string(boot.rank()) + " registered " + std::to_string(mine));
  if (mine == 0) return;
  std::vector<int32_t> tab(2 * (size_t)mine);
  for (int i = 0; i < mine; ++i) {
    tab[2 * i] = kinds[i];
    tab[2 * i + 1] = multicast[i];
  }
  const auto all = boot.allgather(tab.data(), (int)(tab.size() * sizeof(int32_t)));
  for (int p = 0; p < boot.size(); ++p) {
    if (all[p].size() != tab.size() * sizeof(int32_t))
      throw BootstrapError(GICC_EMISMATCH, "gicc::Runtime::exchange: buffer table size differs on rank " + std::to_string(p));
    const int32_t* q = reinterpret_cast<const int32_t*>(all[p].data());
    for (int i = 0; i < mine; ++i) {
      if (q[2 * i] != kinds[i])
        throw BootstrapError(GICC_EMISMATCH, "gicc::Runtime::exchange: new buffer " + std::to_string(i) +
                                                 " has a different kind on rank " + std::to_string(p));
      if (q[2 * i + 1] != multicast[i])
        throw BootstrapError(GICC_EMISMATCH, "gicc::Runtime::exchange: multicast flag of new buffer " +
                                                 std::to_string(i) + " differs on rank " + std::to_string(p));
    }
  }
}

void Runtime::import_new_regions(std::vector<std::unique_ptr<Region>>& list, size_t first, int tag_base) {
  const int n = size(), me = rank();
  const size_t cnt = list.size() - first;
  if (cnt == 0) return;
  // 1. metadata
  std::vector<RegionMeta> meta(cnt);
  for (size_t i = 0; i < cnt; ++i) {
    Region& r = *list[first + i];
    RegionMeta& m = meta[i];
    std::memset(&m, 0, sizeof(m));
    m.kind = r.kind;
    m.multicast = r.multicast ? 1 : 0;
    m.size = r.size;
    m.alloc_size = r.alloc_size;
    m.ipc_offset = r.ipc_offset;
    m.ipc = r.ipc;
  }
  auto all = boot_->allgather(meta.data(), (int)(cnt * sizeof(RegionMeta)));
  std::vector<std::vector<RegionMeta>> pm(n);
  for (int p = 0; p < n; ++p) {
    if (all[p].size() != cnt * sizeof(RegionMeta))
      throw BootstrapError(GICC_EMISMATCH, "gicc::Runtime::exchange: buffer table size differs on rank " + std::to_string(p));
    pm[p].resize(cnt);
    std::memcpy(pm[p].data(), all[p].data(), all[p].size());
    for (size_t i = 0; i < cnt; ++i) {
      if (pm[p][i].kind != meta[i].kind)
        throw BootstrapError(GICC_EMISMATCH, "gicc::Runtime::exchange: buffer " + std::to_string(first + i) +
                                                 " has a different kind on rank " + std::to_string(p));
      if (pm[p][i].multicast != meta[i].multicast)
        throw BootstrapError(GICC_EMISMATCH, "gicc::Runtime::exchange: multicast flag differs for buffer " +
                                                 std::to_string(first + i));
    }
  }
  for (size_t i = 0; i < cnt; ++i) {
    Region& r = *list[first + i];
    r.peer_ptr.assign(n, nullptr);
    r.peer_handle.assign(n, 0);
    r.peer_size.assign(n, 0);
    r.peer_ptr[me] = r.ptr;
    r.peer_size[me] = r.alloc_size;
  }
  // 2. VMM: pass fds to every peer, then import theirs
  std::vector<int> my_fds;
  std::vector<size_t> vmm_idx;
  for (size_t i = 0; i < cnt; ++i) {
    Region& r = *list[first + i];
    if (r.kind != K_VMM) continue;
    if (r.export_fd < 0) {
      int fd = -1;
      GICC_DRV(driver().MemExportToShareableHandle(&fd, r.handle, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0));
      r.export_fd = fd;
    }
    my_fds.push_back(r.export_fd);
    vmm_idx.push_back(i);
  }
  if (!vmm_idx.empty() && n > 1) {
    for (int k = 1; k < n; ++k) boot_->send_fds((me + k) % n, tag_base, my_fds);
    for (int k = 1; k < n; ++k) {
      const int src = (me - k + n) % n;
      std::vector<int> fds = boot_->recv_fds(src, tag_base, vmm_idx.size());
      for (size_t j = 0; j < vmm_idx.size(); ++j) {
        const size_t i = vmm_idx[j];
        Region& r = *list[first + i];
        const size_t psz = pm[src][i].alloc_size;
        CUmemGenericAllocationHandle h = 0;
        GICC_DRV(driver().MemImportFromShareableHandle(&h, reinterpret_cast<void*>((uintptr_t)fds[j]),
                                                       CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR));
        ::close(fds[j]);
        CUdeviceptr va = 0;
        GICC_DRV(driver().MemAddressReserve(&va, psz, granularity_, 0, 0));
        GICC_DRV(driver().MemMap(va, psz, 0, h, 0));
        CUmemAccessDesc acc{};
        acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
        acc.location.id = device_;
        acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
        GICC_DRV(driver().MemSetAccess(va, psz, &acc, 1));
        r.peer_ptr[src] = reinterpret_cast<void*>(va);
        r.peer_handle[src] = h;
        r.peer_size[src] = psz;
      }
    }
  }
  // 3. IPC handles
  for (size_t i = 0; i < cnt; ++i) {
    Region& r = *list[first + i];
    if (r.kind != K_IPC) continue;
    for (int p = 0; p < n; ++p) {
      if (p == me) continue;
      void* base = nullptr;
      GICC_CUDA(cudaIpcOpenMemHandle(&base, pm[p][i].ipc, cudaIpcMemLazyEnablePeerAccess));
      r.ipc_opened.push_back(base);
      r.peer_ptr[p] = static_cast<char*>(base) + pm[p][i].ipc_offset;
      r.peer_size[p] = pm[p][i].size;
    }
  }
  // 4. multicast binding
  for (size_t i = 0; i < cnt; ++i) {
    Region& r = *list[first + i];
    if (r.multicast) bind_multicast(r, tag_base + 512 + (int)i);
    r.imported = true;
  }
}

void Runtime::bind_multicast(Region& r, int tag) {
  const int n = size(), me = rank();
  CUmulticastObjectProp mp{};
  mp.numDevices = (unsigned)n;
  mp.size = r.alloc_size;
  mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  // every rank must have the same size
  auto sizes = boot_->allgather_fixed<uint64_t>(r.alloc_size);
  for (auto s : sizes)
    if (s != r.alloc_size) throw BootstrapError(GICC_EMISMATCH, "gicc: multicast buffer size differs across ranks");
  if (me == 0) {
    GICC_DRV(driver().MulticastCreate(&r.mc_handle, &mp));
    int fd = -1;
    GICC_DRV(driver().MemExportToShareableHandle(&fd, r.mc_handle, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0));
    for (int p = 1; p < n; ++p) boot_->send_fds(p, tag, {fd});
    ::close(fd);
  } else {
    auto fds = boot_->recv_fds(0, tag, 1);
    GICC_DRV(driver().MemImportFromShareableHandle(&r.mc_handle, reinterpret_cast<void*>((uintptr_t)fds[0]),
                                                   CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR));
    ::close(fds[0]);
  }
  GICC_DRV(driver().MulticastAddDevice(r.mc_handle, cudev_));
  boot_->barrier();  // all devices added before any bind
  GICC_DRV(driver().MulticastBindMem(r.mc_handle, 0, r.handle, 0, r.alloc_size, 0));
  CUdeviceptr va = 0;
  size_t mg = 0;
  GICC_DRV(driver().MulticastGetGranularity(&mg, &mp, CU_MULTICAST_GRANULARITY_RECOMMENDED));
  GICC_DRV(driver().MemAddressReserve(&va, r.alloc_size, std::max(mg, granularity_), 0, 0));
  GICC_DRV(driver().MemMap(va, r.alloc_size, 0, r.mc_handle, 0));
  CUmemAccessDesc acc{};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device_;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  GICC_DRV(driver().MemSetAccess(va, r.alloc_size, &acc, 1));
  r.mc_ptr = reinterpret_cast<void*>(va);
  r.mc_size = r.alloc_size;
  boot_->barrier();
}

const Buffer& Runtime::buffer(int idx) const {
  if (idx < 0 || idx >= (int)regions_.size()) throw std::runtime_error("gicc::Runtime: bad buffer index");
  return regions_[idx]->buf;
}

RemoteBufferInfo Runtime::remote_buffer(int r, int idx) const {
  return RemoteBufferInfo{(uint64_t)(uintptr_t)remote_ptr(r, idx, 0), (uint32_t)idx};
}

void* Runtime::remote_ptr(int r, int idx, size_t offset) const {
  if (idx < 0 || idx >= (int)regions_.size()) throw std::runtime_error("gicc::Runtime::remote_ptr: bad buffer index");
  if (r < 0 || r >= size()) throw std::runtime_error("gicc::Runtime::remote_ptr: bad rank");
  const Region& reg = *regions_[idx];
  if (!reg.imported) throw std::runtime_error("gicc::Runtime::remote_ptr: call exchange() first");
  if (reg.kind == K_HOST && r != rank()) throw std::runtime_error("gicc::Runtime::remote_ptr: host buffers are local only");
  if (offset > reg.size) throw std::runtime_error("gicc::Runtime::remote_ptr: offset out of range");
  return static_cast<char*>(reg.peer_ptr[r]) + offset;
}

void* Runtime::multicast_ptr(int idx) const {
  if (idx < 0 || idx >= (int)regions_.size()) return nullptr;
  return regions_[idx]->mc_ptr;
}

Runtime::Region* Runtime::find_region(const void* p, int* idx) const {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  for (size_t i = 0; i < regions_.size(); ++i) {
    const uintptr_t b = reinterpret_cast<uintptr_t>(regions_[i]->ptr);
    if (a >= b && a < b + regions_[i]->size) {
      if (idx) *idx = (int)i;
      return regions_[i].get();
    }
  }
  return nullptr;
}

void* Runtime::translate(const void* local, int peer) const {
  int idx = -1;
  Region* r = find_region(local, &idx);
  if (!r) throw std::runtime_error("gicc::Runtime::translate: pointer is not inside a registered buffer");
  return remote_ptr(peer, idx, reinterpret_cast<uintptr_t>(local) - reinterpret_cast<uintptr_t>(r->ptr));
}

size_t Runtime::signal_alloc(size_t nwords) {
  const size_t aligned = (sig_used_ + 7) & ~size_t(7);  // 64-byte aligned groups
  if (aligned + nwords > sig_words_) throw std::runtime_error("gicc::Runtime::signal_alloc: signal heap exhausted");
  sig_used_ = aligned + nwords;
  return aligned;
}
uint64_t* Runtime::signal_local(size_t w) const { return static_cast<uint64_t*>(internal_[0]->ptr) + w; }
uint64_t* Runtime::signal_peer(int r, size_t w) const { return static_cast<uint64_t*>(internal_[0]->peer_ptr[r]) + w; }
uint64_t* Runtime::signal_multicast(size_t w) const {
  return internal_[0]->mc_ptr ? static_cast<uint64_t*>(internal_[0]->mc_ptr) + w : nullptr;
}

DeviceCtx* Runtime::prepare(int peer, int remote_buf_index) {
  NvtxRange nvtx("gicc::Runtime::prepare");
  if (peer < 0) peer = (rank() + 1) % size();
  if (peer >= size()) throw std::runtime_error("gicc::Runtime::prepare: bad peer");
  DeviceCtx c;
  std::memset(&c, 0, sizeof(c));
  c.my_rank = rank();
  c.n_ranks = size();
  c.peer = peer;
  c.n_bufs = (int)regions_.size();
  for (int i = 0; i < c.n_bufs; ++i) {
    const Region& r = *regions_[i];
    c.local_base[i] = (uint64_t)(uintptr_t)r.ptr;
    c.local_size[i] = r.size;
    if (r.imported && r.kind != K_HOST) {
      c.remote_base[i] = (uint64_t)(uintptr_t)r.peer_ptr[peer];
      c.remote_size[i] = r.size;
    }
  }
  if (remote_buf_index >= 0 && remote_buf_index < c.n_bufs) {
    c.remote_addr = c.remote_base[remote_buf_index];
    c.remote_rkey = (uint32_t)remote_buf_index;
  }
  c.sig_local = signal_local(0);
  c.sig_remote = signal_peer(peer, 0);
  c.ops = ops_dev_;
  c.err = err_;
  c.timeout_ns = timeout_ns_;
  c.checks = checks_enabled() ? 1u : 0u;
  void* d = nullptr;
  GICC_CUDA(cudaMalloc(&d, sizeof(c)));
  GICC_CUDA(cudaMemcpy(d, &c, sizeof(c), cudaMemcpyHostToDevice));
  dev_allocs_.push_back(d);
  return static_cast<DeviceCtx*>(d);
}

GiccContext* Runtime::build_context() {
  NvtxRange nvtx("gicc::Runtime::build_context");
  if (size() > GICC_MAX_PEERS) throw std::runtime_error("gicc::Runtime::build_context: more than GICC_MAX_PEERS ranks");
  auto c = std::make_unique<GiccContext>();
  std::memset(c.get(), 0, sizeof(GiccContext));
  c->my_rank = rank();
  c->n_ranks = size();
  c->n_bufs = (int)regions_.size();
  for (int i = 0; i < c->n_bufs; ++i) {
    const Region& r = *regions_[i];
    c->local_base[i] = (uint64_t)(uintptr_t)r.ptr;
    c->size[i] = r.size;
    c->mc_base[i] = (uint64_t)(uintptr_t)r.mc_ptr;
    for (int p = 0; p < size(); ++p)
      c->peer_base[p][i] = r.imported && (r.kind != K_HOST || p == rank()) ? (uint64_t)(uintptr_t)r.peer_ptr[p] : 0;
  }
  c->sig_local = signal_local(0);
  for (int p = 0; p < size(); ++p) {
    c->sig_peer[p] = signal_peer(p, 0);
    c->peer_ctxs[p] = p == rank() ? nullptr : prepare(p, 0);
  }
  c->sig_mc = signal_multicast(0);
  c->err = err_;
  c->timeout_ns = timeout_ns_;
  c->checks = checks_enabled() ? 1 : 0;
  void* d = nullptr;
  GICC_CUDA(cudaMalloc(&d, sizeof(GiccContext)));
  GICC_CUDA(cudaMemcpy(d, c.get(), sizeof(GiccContext), cudaMemcpyHostToDevice));
  dev_allocs_.push_back(d);
  return static_cast<GiccContext*>(d);
}

void Runtime::reset() {
  GICC_CUDA(cudaDeviceSynchronize());
  for (void* p : dev_allocs_) cudaFree(p);
  dev_allocs_.clear();
  // drain the host queue: start a new batch epoch
  ops_host_->n_ops = 0;
  ops_host_->n_done = 0;
  ops_host_->epoch = ++op_epoch_;
}

void Runtime::barrier() {
  NvtxRange nvtx("gicc::Runtime::barrier");
  boot_->barrier();
}

bool Runtime::checks_enabled() const { return config().checks; }

void Runtime::host_put(const void* src_local, int dest_rank, int dest_buf, size_t dst_off, size_t size,
                       cudaStream_t s) {
  NvtxRange nvtx("gicc::Runtime::host_put");
  if (config().debug_puts) log(LOG_ERROR, "host_put %zu bytes -> rank %d buf %d +%zu", size, dest_rank, dest_buf, dst_off);
  const Region& r = *regions_.at(dest_buf);
  if (dst_off + size > r.size) throw std::runtime_error("gicc::Runtime::host_put: range outside the buffer");
  GICC_CUDA(cudaMemcpyAsync(remote_ptr(dest_rank, dest_buf, dst_off), src_local, size, cudaMemcpyDeviceToDevice, s));
}

void Runtime::host_get(void* dst_local, int src_rank, int src_buf, size_t src_off, size_t size, cudaStream_t s) {
  NvtxRange nvtx("gicc::Runtime::host_get");
  if (config().debug_puts) log(LOG_ERROR, "host_get %zu bytes <- rank %d buf %d +%zu", size, src_rank, src_buf, src_off);
  const Region& r = *regions_.at(src_buf);
  if (src_off + size > r.size) throw std::runtime_error("gicc::Runtime::host_get: range outside the buffer");
  GICC_CUDA(cudaMemcpyAsync(dst_local, remote_ptr(src_rank, src_buf, src_off), size, cudaMemcpyDeviceToDevice, s));
}

Token Runtime::put_no_db(const Buffer& src, int dest_rank, int dest_buf_index, size_t size, size_t src_off,
                         size_t dst_off) {
  NvtxRange nvtx("gicc::Runtime::put_no_db");
  if (config().debug_puts) log(LOG_ERROR, "put_no_db %zu bytes -> rank %d buf %d +%zu", size, dest_rank, dest_buf_index, dst_off);
  if (ops_host_->n_ops >= (uint32_t)GICC_POOL_SIZE)
    throw std::runtime_error("gicc::Runtime::put_no_db: more than GICC_POOL_SIZE queued ops; call reset()");
  if (src.index < 0 || src.index >= (int)regions_.size()) throw std::runtime_error("put_no_db: bad source buffer");
  if (src_off + size > src.size) throw std::runtime_error("put_no_db: source range outside the buffer");
  const Region& dr = *regions_.at(dest_buf_index);
  if (dst_off + size > dr.size) throw std::runtime_error("put_no_db: destination range outside the buffer");
  const uint32_t slot = ops_host_->n_ops;
  QueuedOp& op = ops_host_->ops[slot];
  op.src = (uint64_t)(uintptr_t)src.ptr + src_off;
  op.dst = (uint64_t)(uintptr_t)remote_ptr(dest_rank, dest_buf_index, dst_off);
  op.size = size;
  op.peer = dest_rank;
  op.slot = slot;
  std::atomic_thread_fence(std::memory_order_release);
  ops_host_->n_ops = slot + 1;
  return Token{(int)slot, ops_host_->epoch};
}

DeviceCtx* Runtime::prepare_trigger(Token t) {
  (void)t;
  return prepare((rank() + 1) % size(), 0);
}

void Runtime::wait(Token t) {
  NvtxRange nvtx("gicc::Runtime::wait");
  if (t.slot < 0) return;
  const double deadline = now_s() + (double)timeout_ns_ * 1e-9;
  volatile uint64_t* c = completion_host_ + t.slot;
  while (*c < t.epoch) {
    if (now_s() > deadline)
      throw std::runtime_error("gicc::Runtime::wait: queued put " + std::to_string(t.slot) +
                               " did not complete (was flush() called on the device?)");
    std::this_thread::yield();
  }
}

void Runtime::check_device_errors(bool clear) {
  ErrorRecord r = read_error_record(clear);
  if (r.code != 0)
    throw std::runtime_error(std::string("gicc device error: ") + status_name(r.code) + " at " + where_name(r.where) +
                             " (rank " + std::to_string(r.rank) + ", peer " + std::to_string(r.peer) + ", value " +
                             std::to_string(r.value) + ", expected " + std::to_string(r.expected) + ", count " +
                             std::to_string(r.count) + ")");
}

}  // namespace gicc
