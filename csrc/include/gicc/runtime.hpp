// runtime.hpp -- gicc::Runtime for one 8xB200 NVLink 5 / NVSwitch node.
//
// Same contract as the reference Runtime (gicc.hpp:27-45; mlx5_runtime.hpp:52-243;
// ofi_runtime.hpp:59-332): construct (bootstrap + GPU selection), register_buffer,
// exchange (collective), remote_buffer, prepare, build_context, reset, barrier,
// rank/size/gpu_id, clock_rate_khz, gpu_name, boot, and the OFI-style host queue
// put_no_db -> Token, prepare_trigger, wait(Token).
//
// Transport: instead of InfiniBand queue pairs, every peer's buffer is mapped into this
// process.  `alloc` creates CUDA VMM memory with a POSIX-fd shareable handle; exchange()
// passes the fds over the bootstrap's Unix socket and each rank imports and maps every
// peer allocation (cuMemImportFromShareableHandle + cuMemMap + cuMemSetAccess).  Plain
// cudaMalloc memory registered with register_buffer goes through CUDA IPC handles.
// Buffers allocated with `multicast=true` are also bound to an NVLS multicast object
// (cuMulticastCreate/AddDevice/BindMem), giving one address whose multimem.* accesses
// reach every rank's copy through the NVSwitch.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <memory>
#include <string>
#include <vector>

#include "gicc/bootstrap.hpp"
#include "gicc/types.hpp"

namespace gicc {

struct Token {
  int slot = -1;
  uint64_t epoch = 0;
};

struct GICC_EXPORT RuntimeOptions {
  int device = -1;                  // -1: local_rank % device_count
  size_t signal_heap_bytes = 4u << 20;
  bool enable_multicast = true;     // NVLS when the device supports it (and size > 1)
};

class GICC_EXPORT Runtime {
 public:
  Runtime();  // bootstrap from the environment
  explicit Runtime(std::shared_ptr<Bootstrap> boot, RuntimeOptions opt = RuntimeOptions());
  // Over a Bootstrap the caller owns and keeps alive (the reference's OFI programs build
  // their transport this way: gicc::Fabric comm(boot)).
  explicit Runtime(Bootstrap& boot, RuntimeOptions opt = RuntimeOptions());
  Runtime& fabric() { return *this; }  // the reference's accessor of its transport object
  ~Runtime();
  Runtime(const Runtime&) = delete;
  Runtime& operator=(const Runtime&) = delete;

  // --- reference API -------------------------------------------------------------------
  // Registers local memory.  Device memory must come from alloc() (VMM) or cudaMalloc
  // (CUDA IPC).  Host memory (is_device=false) is pinned + mapped and stays local.
  Buffer register_buffer(void* ptr, size_t size, bool is_device = true);
  void exchange();  // collective; imports every buffer registered since the last call
  RemoteBufferInfo remote_buffer(int rank, int buf_index) const;
  DeviceCtx* prepare(int peer = -1, int remote_buf_index = 0);  // device memory, owned here
  GiccContext* build_context();                                    // device memory, owned here
  void reset();    // frees prepared contexts and clears the host op queue
  void barrier();  // host barrier through the bootstrap
  int rank() const { return boot_->rank(); }
  int size() const { return boot_->size(); }
  int gpu_id() const { return device_; }
  double clock_rate_khz() const { return clock_khz_; }
  const char* gpu_name() const { return gpu_name_.c_str(); }
  Bootstrap& boot() { return *boot_; }
  std::shared_ptr<Bootstrap> boot_ptr() { return boot_; }

  // --- OFI-style host queue (ofi_runtime.hpp:201-322) ------------------------------------
  Token put_no_db(const Buffer& src, int dest_rank, int dest_buf_index, size_t size, size_t src_off = 0,
                  size_t dst_off = 0);
  DeviceCtx* prepare_trigger(Token t);  // ctx whose flush() runs the queued ops
  void wait(Token t);                   // host wait (bounded) for the op's completion

  // --- host-driven transfers (copy engine; reference host verbs path, mlx5/comm.hpp:170-255)
  void host_put(const void* src_local, int dest_rank, int dest_buf, size_t dst_off, size_t size, cudaStream_t s);
  void host_get(void* dst_local, int src_rank, int src_buf, size_t src_off, size_t size, cudaStream_t s);
  bool checks_enabled() const;  // GICC_CHECKS=1: device contexts bounds-check every put

  // --- additions ------------------------------------------------------------------------
  // Symmetric allocation, registered under the next index (not collective by itself; all
  // ranks must allocate the same sequence and then call exchange()).
  Buffer alloc(size_t bytes, bool multicast = false);
  void* remote_ptr(int rank, int buf_index, size_t offset = 0) const;
  void* multicast_ptr(int buf_index) const;  // nullptr when not multicast-bound
  bool multicast_supported() const { return mc_supported_; }
  int num_buffers() const { return (int)regions_.size(); }
  const Buffer& buffer(int idx) const;
  // Translate a local pointer inside a registered buffer to the same offset on `peer`.
  void* translate(const void* local, int peer) const;
  // Signal heap: monotonic words in symmetric memory (bump allocated, deterministic).
  size_t signal_alloc(size_t nwords);
  uint64_t* signal_local(size_t word = 0) const;
  uint64_t* signal_peer(int rank, size_t word = 0) const;
  uint64_t* signal_multicast(size_t word = 0) const;  // nullptr without NVLS
  uint64_t timeout_ns() const { return timeout_ns_; }
  ErrorRecord* error_record() const { return err_; }
  // Raises gicc device errors recorded by kernels (after a synchronize).
  void check_device_errors(bool clear = true);
  // Releases every mapping and allocation (also done by the destructor).
  void finalize();

 private:
  struct Region;
  void init(RuntimeOptions opt);
  void import_new_regions(std::vector<std::unique_ptr<Region>>& list, size_t first, int tag_base);
  void bind_multicast(Region& r, int tag);
  Region* find_region(const void* p, int* idx) const;

  std::shared_ptr<Bootstrap> boot_;
  int device_ = 0;
  CUdevice cudev_ = 0;
  double clock_khz_ = 0;
  std::string gpu_name_;
  bool mc_supported_ = false;
  uint64_t timeout_ns_ = 0;
  ErrorRecord* err_ = nullptr;
  size_t granularity_ = 2u << 20;
  std::vector<std::unique_ptr<Region>> regions_;   // user-visible, index = position
  std::vector<std::unique_ptr<Region>> internal_;  // signal heap
  size_t exchanged_ = 0;
  int exchange_epoch_ = 0;
  size_t sig_words_ = 0, sig_used_ = 0;
  std::vector<void*> dev_allocs_;  // prepared ctxs
  // host op queue
  OpTable* ops_host_ = nullptr;
  OpTable* ops_dev_ = nullptr;
  uint64_t* completion_host_ = nullptr;
  uint64_t op_epoch_ = 1;
  bool finalized_ = false;
};

// One ordered pair of visible GPUs and what cudaDeviceGetP2PAttribute reports for it.
struct P2PLink {
  int src = 0, dst = 0;
  int access = 0;          // src can map dst's memory
  int native_atomics = 0;  // atomics on dst's memory are native over the link
  int array_access = 0;
  int perf_rank = 0;       // the driver's relative rank (lower is faster)
};
// Every ordered pair of the GPUs visible to this process (no runtime needed).
GICC_EXPORT std::vector<P2PLink> p2p_links();

// The reference's OFI programs name their transport object gicc::Fabric; here the Runtime
// is that object.
using Fabric = Runtime;

// The collective consistency check exchange() runs before any handle crosses a process
// boundary: every rank registered the same number of buffers since the last exchange, with
// the same kind and multicast flag, in the same order.  Throws BootstrapError
// (GICC_EMISMATCH) naming the first difference on every rank; uses only the bootstrap.
GICC_EXPORT void check_exchange_consistency(Bootstrap& boot, const std::vector<int32_t>& kinds,
                                            const std::vector<int32_t>& multicast);

}  // namespace gicc
