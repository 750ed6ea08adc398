// bootstrap.hpp -- the process plane: a TCP key-value store with collectives.
//
// Same method set as the reference's MPI/PMI2 bootstrap (bootstrap/detail/bootstrap_mpi.hpp:
// 70-159; bootstrap_pmi2.hpp:86-169): rank/size/local_rank/local_size, locality_map,
// barrier, allgather (variable length), allgather_fixed, broadcast, send/recv/sendrecv,
// wtime and a job-wide abort.  There is no MPI on a B200 box, so the transport is our
// own: rank 0 runs a small store server thread (poll() loop) that every rank, rank 0
// included, talks to over TCP.  Collectives are epoch-keyed store operations, the way the
// PMI2 variant builds them on Put/Fence/Get (keys `ag.<epoch>.<rank>`, raw bytes -- no hex
// encoding is needed over a socket).
//
// Failure detection: the server notices a rank whose socket closes without a goodbye
// and fails every pending and later request with "rank R left"; a rank that calls
// abort() makes the server fail the job for everybody.  Every blocking request is bounded
// by GICC_BOOTSTRAP_TIMEOUT_MS.  Errors are thrown as gicc::BootstrapError.
//
// Besides the store, every rank owns an abstract-namespace Unix socket used to pass file
// descriptors (CUDA VMM / multicast shareable handles) with SCM_RIGHTS.
#pragma once
#include <atomic>
#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>

#include "gicc/host_util.hpp"

namespace gicc {

struct GICC_EXPORT BootstrapError : std::runtime_error {
  int code;
  BootstrapError(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

class StoreServer;  // bootstrap.cpp

class GICC_EXPORT Bootstrap {
 public:
  // From the environment: GICC_RANK/GICC_SIZE (or torchrun's RANK/WORLD_SIZE),
  // GICC_LOCAL_RANK/GICC_LOCAL_SIZE (or LOCAL_RANK/LOCAL_WORLD_SIZE; otherwise derived
  // from host names), GICC_BOOTSTRAP_ADDR=host:port (or MASTER_ADDR with
  // GICC_BOOTSTRAP_PORT, default MASTER_PORT+1).  Blocks until every rank has joined.
  Bootstrap();
  Bootstrap(int* argc, char*** argv);  // argument-taking forms kept for API parity
  Bootstrap(int argc, char** argv);
  // Explicit form.  Rank 0 serves at `addr` ("host:port"; port 0 picks a free port, see
  // server_port()).  Does not wait for the other ranks; call setup() (collective) next.
  Bootstrap(int rank, int size, const std::string& addr, double timeout_s = -1.0);
  ~Bootstrap();
  Bootstrap(const Bootstrap&) = delete;
  Bootstrap& operator=(const Bootstrap&) = delete;

  // Collective: host names -> locality map, local rank/size; FD channel naming.
  void setup(int local_rank_hint = -1, int local_size_hint = -1);

  int rank() const { return rank_; }
  int size() const { return size_; }
  int local_rank() const { return local_rank_; }
  int local_size() const { return local_size_; }
  int server_port() const;
  const std::string& job_id() const { return job_id_; }
  std::vector<bool> locality_map() const { return locality_; }

  void barrier();
  std::vector<std::vector<uint8_t>> allgather(const void* data, int len);
  template <class T>
  std::vector<T> allgather_fixed(const T& v) {
    static_assert(std::is_trivially_copyable<T>::value, "allgather_fixed needs a trivially copyable type");
    auto all = allgather(&v, (int)sizeof(T));
    std::vector<T> out(all.size());
    for (size_t i = 0; i < all.size(); ++i) {
      if (all[i].size() != sizeof(T)) throw BootstrapError(7, "allgather_fixed: size mismatch across ranks");
      std::memcpy(&out[i], all[i].data(), sizeof(T));
    }
    return out;
  }
  template <class T>
  void broadcast(T& v, int root = 0) {
    static_assert(std::is_trivially_copyable<T>::value, "broadcast needs a trivially copyable type");
    broadcast_bytes(&v, sizeof(T), root);
  }
  void broadcast_bytes(void* data, size_t len, int root = 0);
  void send(const void* data, size_t len, int dst, int tag = 0);
  void recv(void* data, size_t len, int src, int tag = 0);
  void sendrecv(const void* sbuf, size_t slen, int dst, void* rbuf, size_t rlen, int src, int tag = 0);
  double wtime() const;

  // Store primitives (used by the collectives and by the Runtime).
  void kv_put(const std::string& key, const void* data, size_t len);
  // Blocks until `key` exists.  consume > 0: the key is deleted after that many gets.
  std::vector<uint8_t> kv_get(const std::string& key, int consume = 0);
  // Raises if the job has failed (a rank left or aborted).  Cheap round trip.
  void check();

  // Fails the job for every rank (peers' pending and next bootstrap calls raise), then
  // exits this process with `code`.  The reference's gicc::abort (bootstrap.hpp:29-33).
  [[noreturn]] void abort_job(int code, const std::string& msg);
  // Same, through the most recently constructed Bootstrap of this process.
  [[noreturn]] static void abort(int code, const char* msg);
  // Report a failure to the server without exiting (tests, graceful shutdown paths).
  void fail_job(int code, const std::string& msg);

  // File-descriptor passing between ranks of one host (SCM_RIGHTS over abstract Unix
  // sockets).  send_fds is asynchronous w.r.t. the receiver; recv_fds returns the fds of
  // the next message from `src` with this tag.
  void send_fds(int dst, int tag, const std::vector<int>& fds);
  std::vector<int> recv_fds(int src, int tag, size_t n);

  double timeout_s() const { return timeout_s_; }

 private:
  void init_client(const std::string& host, int port);
  std::vector<uint8_t> request(uint32_t op, const std::string& key, const void* data, size_t len, int consume);
  void open_fd_listener();

  int rank_ = 0, size_ = 1, local_rank_ = 0, local_size_ = 1;
  std::string job_id_;
  std::vector<bool> locality_;
  double timeout_s_ = 120.0;
  int sock_ = -1;
  int fd_listen_ = -1;
  uint64_t epoch_ = 0;
  std::vector<uint64_t> send_seq_, recv_seq_;
  std::unique_ptr<StoreServer> server_;
  std::vector<std::vector<int>> fd_stash_;  // early fd messages: {src, tag, fds...}
  double t0_ = 0.0;
  bool closed_ = false;
};

}  // namespace gicc
