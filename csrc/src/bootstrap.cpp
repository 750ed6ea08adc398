// bootstrap.cpp -- socket store server/client and the collectives built on it.
#include "gicc/bootstrap.hpp"

#include "gicc/config.hpp"

#include <arpa/inet.h>
#include <fcntl.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <signal.h>
#include <sys/socket.h>
#include <sys/types.h>
#include <sys/un.h>
#include <unistd.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <random>
#include <unordered_map>

#include "gicc/error.hpp"

namespace gicc {

namespace {

enum Op : uint32_t { OP_HELLO = 1, OP_PUT = 2, OP_GET = 3, OP_BARRIER = 4, OP_ABORT = 5, OP_BYE = 6, OP_PING = 7 };

#pragma pack(push, 1)
struct ReqHdr {
  uint32_t op;
  int32_t rank;
  uint32_t klen;
  uint64_t vlen;
  int32_t consume;
};
struct RepHdr {
  int32_t status;
  uint64_t vlen;
};
#pragma pack(pop)

double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

bool write_all(int fd, const void* p, size_t n) {
  const char* c = static_cast<const char*>(p);
  while (n) {
    ssize_t w = ::send(fd, c, n, MSG_NOSIGNAL);
    if (w < 0) {
      if (errno == EINTR) continue;
      return false;
    }
    c += w;
    n -= (size_t)w;
  }
  return true;
}

bool read_all(int fd, void* p, size_t n) {
  char* c = static_cast<char*>(p);
  while (n) {
    ssize_t r = ::recv(fd, c, n, 0);
    if (r == 0) return false;
    if (r < 0) {
      if (errno == EINTR) continue;
      return false;
    }
    c += r;
    n -= (size_t)r;
  }
  return true;
}

// Read exactly n bytes, giving up when `deadline` (steady seconds) passes.
bool read_all_deadline(int fd, void* p, size_t n, double deadline, bool* timed_out) {
  char* c = static_cast<char*>(p);
  *timed_out = false;
  while (n) {
    double left = deadline - now_s();
    if (left <= 0) {
      *timed_out = true;
      return false;
    }
    pollfd pf{fd, POLLIN, 0};
    int pr = ::poll(&pf, 1, (int)std::min(left * 1000.0 + 1, 1000.0));
    if (pr < 0 && errno != EINTR) return false;
    if (pr <= 0) continue;
    ssize_t r = ::recv(fd, c, n, 0);
    if (r == 0) return false;
    if (r < 0) {
      if (errno == EINTR || errno == EAGAIN) continue;
      return false;
    }
    c += r;
    n -= (size_t)r;
  }
  return true;
}

void parse_addr(const std::string& addr, std::string& host, int& port) {
  auto pos = addr.rfind(':');
  if (pos == std::string::npos) throw BootstrapError(GICC_EINVAL, "bootstrap address must be host:port, got '" + addr + "'");
  host = addr.substr(0, pos);
  port = std::atoi(addr.c_str() + pos + 1);
  if (host.empty()) host = "127.0.0.1";
}

int env_int(const char* a, const char* b, int dflt) {
  const char* s = std::getenv(a);
  if (!s && b) s = std::getenv(b);
  return s ? std::atoi(s) : dflt;
}

std::string abstract_name(const std::string& job, int rank) { return "gicc." + job + "." + std::to_string(rank); }

sockaddr_un make_abstract(const std::string& name, socklen_t* len) {
  sockaddr_un a{};
  a.sun_family = AF_UNIX;
  a.sun_path[0] = '\0';
  std::memcpy(a.sun_path + 1, name.data(), std::min(name.size(), sizeof(a.sun_path) - 2));
  *len = (socklen_t)(offsetof(sockaddr_un, sun_path) + 1 + std::min(name.size(), sizeof(a.sun_path) - 2));
  return a;
}

Bootstrap* g_last_bootstrap = nullptr;

}  // namespace

// ------------------------------------------------------------------------------------
// Server (rank 0)
// ------------------------------------------------------------------------------------
class StoreServer {
 public:
  StoreServer(const std::string& host, int port, int size) : size_(size) {
    lfd_ = ::socket(AF_INET, SOCK_STREAM, 0);
    if (lfd_ < 0) throw BootstrapError(GICC_EBOOT, "bootstrap: socket() failed");
    int one = 1;
    ::setsockopt(lfd_, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    sockaddr_in a{};
    a.sin_family = AF_INET;
    a.sin_port = htons((uint16_t)port);
    if (host == "0.0.0.0" || host == "*") {
      a.sin_addr.s_addr = htonl(INADDR_ANY);
    } else if (::inet_pton(AF_INET, host.c_str(), &a.sin_addr) != 1) {
      addrinfo hints{}, *res = nullptr;
      hints.ai_family = AF_INET;
      if (::getaddrinfo(host.c_str(), nullptr, &hints, &res) != 0 || !res)
        throw BootstrapError(GICC_EBOOT, "bootstrap: cannot resolve '" + host + "'");
      a.sin_addr = reinterpret_cast<sockaddr_in*>(res->ai_addr)->sin_addr;
      ::freeaddrinfo(res);
    }
    if (::bind(lfd_, reinterpret_cast<sockaddr*>(&a), sizeof(a)) != 0) {
      ::close(lfd_);
      throw BootstrapError(GICC_EBOOT, "bootstrap: bind(" + host + ":" + std::to_string(port) + ") failed: " +
                                           std::strerror(errno));
    }
    if (::listen(lfd_, 512) != 0) throw BootstrapError(GICC_EBOOT, "bootstrap: listen() failed");
    socklen_t al = sizeof(a);
    ::getsockname(lfd_, reinterpret_cast<sockaddr*>(&a), &al);
    port_ = ntohs(a.sin_port);
    if (::pipe(wake_) != 0) throw BootstrapError(GICC_EBOOT, "bootstrap: pipe() failed");
    th_ = std::thread([this] { loop(); });
  }
  // Wait (bounded) until every rank that joined has said goodbye or disconnected.
  void drain(double timeout_s) {
    const double deadline = now_s() + timeout_s;
    while (live_.load() > 0 && now_s() < deadline) ::usleep(2000);
  }
  ~StoreServer() {
    stop_ = true;
    char c = 1;
    (void)!::write(wake_[1], &c, 1);
    if (th_.joinable()) th_.join();
    for (auto& kv : clients_) ::close(kv.first);
    ::close(lfd_);
    ::close(wake_[0]);
    ::close(wake_[1]);
  }
  int port() const { return port_; }

 private:
  struct Client {
    int rank = -1;
    bool bye = false;
  };
  struct Pending {
    int fd;
    int consume;
  };
  struct Entry {
    std::vector<uint8_t> val;
    int left;  // <= 0: persistent
  };

  void reply(int fd, int status, const void* data, size_t len) {
    RepHdr h{status, len};
    if (!write_all(fd, &h, sizeof(h)) || (len && !write_all(fd, data, len))) {
      // the client is gone; the poll loop will notice
    }
  }
  void reply_err(int fd) { reply(fd, GICC_EPEER, fail_msg_.data(), fail_msg_.size()); }

  void fail(const std::string& msg) {
    if (failed_) return;
    failed_ = true;
    fail_msg_ = msg;
    for (auto& kv : pending_)
      for (auto& p : kv.second) reply_err(p.fd);
    pending_.clear();
    for (auto& kv : barriers_)
      for (int fd : kv.second) reply_err(fd);
    barriers_.clear();
  }

  void serve_get(int fd, const std::string& key, int consume) {
    auto it = store_.find(key);
    if (it == store_.end()) {
      pending_[key].push_back({fd, consume});
      return;
    }
    reply(fd, 0, it->second.val.data(), it->second.val.size());
    if (consume > 0) {
      if (it->second.left <= 0) it->second.left = consume;
      if (--it->second.left == 0) store_.erase(it);
    }
  }

  void handle(int fd, Client& cl) {
    ReqHdr h;
    if (!read_all(fd, &h, sizeof(h))) {
      drop(fd);
      return;
    }
    std::string key(h.klen, '\0');
    std::vector<uint8_t> val(h.vlen);
    if ((h.klen && !read_all(fd, &key[0], h.klen)) || (h.vlen && !read_all(fd, val.data(), h.vlen))) {
      drop(fd);
      return;
    }
    switch (h.op) {
      case OP_HELLO:
        cl.rank = h.rank;
        live_++;
        reply(fd, failed_ ? GICC_EPEER : 0, failed_ ? fail_msg_.data() : nullptr, failed_ ? fail_msg_.size() : 0);
        return;
      case OP_BYE:
        if (!cl.bye && cl.rank >= 0) live_--;
        cl.bye = true;
        reply(fd, 0, nullptr, 0);
        return;
      case OP_ABORT: {
        std::string m(val.begin(), val.end());
        fail("rank " + std::to_string(h.rank) + " aborted the job: " + m);
        reply(fd, 0, nullptr, 0);
        return;
      }
      default:
        break;
    }
    if (failed_) {
      reply_err(fd);
      return;
    }
    switch (h.op) {
      case OP_PING:
        reply(fd, 0, nullptr, 0);
        break;
      case OP_PUT: {
        Entry e{std::move(val), 0};
        auto pit = pending_.find(key);
        store_[key] = std::move(e);
        if (pit != pending_.end()) {
          auto waiters = std::move(pit->second);
          pending_.erase(pit);
          for (auto& p : waiters) {
            if (store_.find(key) == store_.end()) {
              pending_[key].push_back(p);
            } else {
              serve_get(p.fd, key, p.consume);
            }
          }
        }
        reply(fd, 0, nullptr, 0);
        break;
      }
      case OP_GET:
        serve_get(fd, key, h.consume);
        break;
      case OP_BARRIER: {
        auto& v = barriers_[key];
        v.push_back(fd);
        if ((int)v.size() == size_) {
          for (int f : v) reply(f, 0, nullptr, 0);
          barriers_.erase(key);
        }
        break;
      }
      default:
        reply(fd, GICC_EINVAL, "bad op", 6);
    }
  }

  void drop(int fd) {
    auto it = clients_.find(fd);
    if (it != clients_.end()) {
      if (!it->second.bye && it->second.rank >= 0) live_--;
      if (!it->second.bye && !stop_) {
        fail("rank " + std::to_string(it->second.rank) + " left the job (bootstrap connection closed)");
      }
      clients_.erase(it);
    }
    // forget any pending operation of this socket
    for (auto& kv : pending_) {
      auto& v = kv.second;
      for (size_t i = 0; i < v.size();)
        if (v[i].fd == fd) v.erase(v.begin() + i); else ++i;
    }
    for (auto& kv : barriers_) {
      auto& v = kv.second;
      for (size_t i = 0; i < v.size();)
        if (v[i] == fd) v.erase(v.begin() + i); else ++i;
    }
    ::close(fd);
  }

  void loop() {
    while (!stop_) {
      std::vector<pollfd> pf;
      pf.push_back({lfd_, POLLIN, 0});
      pf.push_back({wake_[0], POLLIN, 0});
      for (auto& kv : clients_) pf.push_back({kv.first, POLLIN, 0});
      int r = ::poll(pf.data(), pf.size(), 500);
      if (r < 0 && errno != EINTR) break;
      if (r <= 0) continue;
      if (pf[1].revents) break;
      if (pf[0].revents & POLLIN) {
        int c = ::accept(lfd_, nullptr, nullptr);
        if (c >= 0) {
          int one = 1;
          ::setsockopt(c, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
          clients_[c] = Client{};
        }
      }
      for (size_t i = 2; i < pf.size(); ++i) {
        if (!pf[i].revents) continue;
        int fd = pf[i].fd;
        auto it = clients_.find(fd);
        if (it == clients_.end()) continue;
        if (pf[i].revents & (POLLIN)) {
          handle(fd, it->second);
        } else if (pf[i].revents & (POLLHUP | POLLERR | POLLNVAL)) {
          drop(fd);
        }
      }
    }
  }

  int size_;
  int lfd_ = -1;
  int port_ = 0;
  int wake_[2] = {-1, -1};
  std::atomic<bool> stop_{false};
  std::atomic<int> live_{0};
  std::thread th_;
  std::map<int, Client> clients_;
  std::unordered_map<std::string, Entry> store_;
  std::unordered_map<std::string, std::vector<Pending>> pending_;
  std::unordered_map<std::string, std::vector<int>> barriers_;
  bool failed_ = false;
  std::string fail_msg_;
};

// ------------------------------------------------------------------------------------
// Client
// ------------------------------------------------------------------------------------
static std::mutex g_req_mu;

Bootstrap::Bootstrap() {
  rank_ = env_int("GICC_RANK", "RANK", 0);
  size_ = env_int("GICC_SIZE", "WORLD_SIZE", 1);
  if (const uint64_t ms = config().bootstrap_timeout_ms) timeout_s_ = ms / 1000.0;
  std::string addr;
  if (const char* a = std::getenv("GICC_BOOTSTRAP_ADDR")) {
    addr = a;
  } else {
    const char* ma = std::getenv("MASTER_ADDR");
    int port = env_int("GICC_BOOTSTRAP_PORT", nullptr, 0);
    if (port == 0) {
      int mp = env_int("MASTER_PORT", nullptr, 0);
      port = mp ? mp + 1 : 0;
    }
    if (size_ > 1 && (!ma || port == 0))
      throw BootstrapError(GICC_EINVAL, "bootstrap: set GICC_BOOTSTRAP_ADDR (host:port) or MASTER_ADDR/MASTER_PORT");
    addr = std::string(ma ? ma : "127.0.0.1") + ":" + std::to_string(port);
  }
  std::string host;
  int port = 0;
  parse_addr(addr, host, port);
  t0_ = now_s();
  if (rank_ == 0) server_.reset(new StoreServer(host == "localhost" ? "127.0.0.1" : host, port, size_));
  init_client(host, rank_ == 0 ? server_->port() : port);
  setup(env_int("GICC_LOCAL_RANK", "LOCAL_RANK", -1), env_int("GICC_LOCAL_SIZE", "LOCAL_WORLD_SIZE", -1));
}

Bootstrap::Bootstrap(int* /*argc*/, char*** /*argv*/) : Bootstrap() {}
Bootstrap::Bootstrap(int /*argc*/, char** /*argv*/) : Bootstrap() {}

Bootstrap::Bootstrap(int rank, int size, const std::string& addr, double timeout_s) {
  if (size < 1 || rank < 0 || rank >= size) throw BootstrapError(GICC_EINVAL, "bootstrap: bad rank/size");
  rank_ = rank;
  size_ = size;
  if (timeout_s > 0) {
    timeout_s_ = timeout_s;
  } else if (const uint64_t ms = config().bootstrap_timeout_ms) {
    timeout_s_ = ms / 1000.0;
  }
  std::string host;
  int port = 0;
  parse_addr(addr, host, port);
  t0_ = now_s();
  if (rank_ == 0) server_.reset(new StoreServer(host == "localhost" ? "127.0.0.1" : host, port, size_));
  init_client(host, rank_ == 0 ? server_->port() : port);
}

int Bootstrap::server_port() const { return server_ ? server_->port() : -1; }

void Bootstrap::init_client(const std::string& host_in, int port) {
  std::string host = (host_in == "0.0.0.0" || host_in == "*" || host_in == "localhost") ? "127.0.0.1" : host_in;
  sockaddr_in a{};
  a.sin_family = AF_INET;
  a.sin_port = htons((uint16_t)port);
  if (::inet_pton(AF_INET, host.c_str(), &a.sin_addr) != 1) {
    addrinfo hints{}, *res = nullptr;
    hints.ai_family = AF_INET;
    if (::getaddrinfo(host.c_str(), nullptr, &hints, &res) != 0 || !res)
      throw BootstrapError(GICC_EBOOT, "bootstrap: cannot resolve '" + host + "'");
    a.sin_addr = reinterpret_cast<sockaddr_in*>(res->ai_addr)->sin_addr;
    ::freeaddrinfo(res);
  }
  const double deadline = now_s() + timeout_s_;
  while (true) {
    sock_ = ::socket(AF_INET, SOCK_STREAM, 0);
    if (::connect(sock_, reinterpret_cast<sockaddr*>(&a), sizeof(a)) == 0) break;
    ::close(sock_);
    sock_ = -1;
    if (now_s() > deadline)
      throw BootstrapError(GICC_ETIMEDOUT, "bootstrap: rank " + std::to_string(rank_) + " could not reach the store at " +
                                               host + ":" + std::to_string(port));
    ::usleep(20000);
  }
  int one = 1;
  ::setsockopt(sock_, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
  request(OP_HELLO, "", nullptr, 0, 0);
  send_seq_.assign(size_, 0);
  recv_seq_.assign(size_, 0);
  fd_stash_.clear();
  g_last_bootstrap = this;
}

void Bootstrap::setup(int local_rank_hint, int local_size_hint) {
  // job id (for the fd channel names) from rank 0
  if (rank_ == 0) {
    std::random_device rd;
    char buf[64];
    std::snprintf(buf, sizeof(buf), "%08x%04x", (unsigned)rd(), (unsigned)(::getpid() & 0xffff));
    job_id_ = buf;
    kv_put("job_id", job_id_.data(), job_id_.size());
  } else {
    auto v = kv_get("job_id");
    job_id_.assign(v.begin(), v.end());
  }
  char hn[256] = {0};
  ::gethostname(hn, sizeof(hn) - 1);
  auto all = allgather(hn, (int)std::strlen(hn));
  locality_.assign(size_, false);
  int lr = 0, ls = 0;
  for (int r = 0; r < size_; ++r) {
    std::string h(all[r].begin(), all[r].end());
    if (h == hn) {
      locality_[r] = true;
      if (r < rank_) ++lr;
      ++ls;
    }
  }
  local_rank_ = lr;
  local_size_ = ls;
  if (local_rank_hint >= 0 && local_rank_hint != lr) {
    std::fprintf(stderr, "[gicc] rank %d: launcher local rank %d differs from host-name order %d; using launcher's\n",
                 rank_, local_rank_hint, lr);
    local_rank_ = local_rank_hint;
  }
  if (local_size_hint > 0) local_size_ = local_size_hint;
  open_fd_listener();
  barrier();
}

Bootstrap::~Bootstrap() {
  if (!closed_ && sock_ >= 0) {
    try {
      std::lock_guard<std::mutex> lk(g_req_mu);
      ReqHdr h{OP_BYE, rank_, 0, 0, 0};
      if (write_all(sock_, &h, sizeof(h))) {
        RepHdr r;
        bool to = false;
        read_all_deadline(sock_, &r, sizeof(r), now_s() + 2.0, &to);
      }
    } catch (...) {
    }
  }
  if (sock_ >= 0) ::close(sock_);
  if (fd_listen_ >= 0) ::close(fd_listen_);
  for (auto& v : fd_stash_)
    for (int fd : v) ::close(fd);
  // Rank 0 keeps serving until the other ranks said goodbye (bounded).
  if (server_) server_->drain(std::min(timeout_s_, 30.0));
  server_.reset();
  if (g_last_bootstrap == this) g_last_bootstrap = nullptr;
}

std::vector<uint8_t> Bootstrap::request(uint32_t op, const std::string& key, const void* data, size_t len,
                                        int consume) {
  std::lock_guard<std::mutex> lk(g_req_mu);
  if (sock_ < 0) throw BootstrapError(GICC_EBOOT, "bootstrap: not connected");
  ReqHdr h{op, rank_, (uint32_t)key.size(), (uint64_t)len, consume};
  if (!write_all(sock_, &h, sizeof(h)) || (!key.empty() && !write_all(sock_, key.data(), key.size())) ||
      (len && !write_all(sock_, data, len)))
    throw BootstrapError(GICC_EPEER, "bootstrap: lost the connection to the store (rank 0 gone?)");
  RepHdr r;
  bool to = false;
  const double deadline = now_s() + timeout_s_;
  if (!read_all_deadline(sock_, &r, sizeof(r), deadline, &to)) {
    if (to)
      throw BootstrapError(GICC_ETIMEDOUT, "bootstrap: rank " + std::to_string(rank_) + " timed out after " +
                                               std::to_string(timeout_s_) + " s (op " + std::to_string(op) +
                                               ", key '" + key + "')");
    throw BootstrapError(GICC_EPEER, "bootstrap: lost the connection to the store (rank 0 gone?)");
  }
  std::vector<uint8_t> out(r.vlen);
  if (r.vlen && !read_all_deadline(sock_, out.data(), r.vlen, now_s() + timeout_s_, &to))
    throw BootstrapError(GICC_EPEER, "bootstrap: truncated reply");
  if (r.status != 0) {
    std::string msg(out.begin(), out.end());
    throw BootstrapError(r.status, "bootstrap: job failed: " + msg);
  }
  return out;
}

void Bootstrap::kv_put(const std::string& key, const void* data, size_t len) { request(OP_PUT, key, data, len, 0); }
std::vector<uint8_t> Bootstrap::kv_get(const std::string& key, int consume) {
  return request(OP_GET, key, nullptr, 0, consume);
}
void Bootstrap::check() { request(OP_PING, "", nullptr, 0, 0); }

void Bootstrap::barrier() {
  if (size_ == 1) return;
  ++epoch_;
  request(OP_BARRIER, "bar." + std::to_string(epoch_), nullptr, 0, 0);
}

std::vector<std::vector<uint8_t>> Bootstrap::allgather(const void* data, int len) {
  ++epoch_;
  std::vector<std::vector<uint8_t>> out(size_);
  const std::string base = "ag." + std::to_string(epoch_) + ".";
  if (size_ == 1) {
    out[0].assign(static_cast<const uint8_t*>(data), static_cast<const uint8_t*>(data) + len);
    return out;
  }
  kv_put(base + std::to_string(rank_), data, (size_t)len);
  for (int r = 0; r < size_; ++r) out[r] = kv_get(base + std::to_string(r), size_);
  return out;
}

void Bootstrap::broadcast_bytes(void* data, size_t len, int root) {
  ++epoch_;
  if (size_ == 1) return;
  const std::string key = "bc." + std::to_string(epoch_);
  if (rank_ == root) {
    kv_put(key, data, len);
  } else {
    auto v = kv_get(key, size_ - 1);
    if (v.size() != len) throw BootstrapError(GICC_EMISMATCH, "broadcast: size mismatch across ranks");
    std::memcpy(data, v.data(), len);
  }
}

void Bootstrap::send(const void* data, size_t len, int dst, int tag) {
  if (dst < 0 || dst >= size_) throw BootstrapError(GICC_EINVAL, "send: bad destination rank");
  const std::string key = "p2p." + std::to_string(rank_) + "." + std::to_string(dst) + "." + std::to_string(tag) +
                          "." + std::to_string(send_seq_[dst]++);
  kv_put(key, data, len);
}

void Bootstrap::recv(void* data, size_t len, int src, int tag) {
  if (src < 0 || src >= size_) throw BootstrapError(GICC_EINVAL, "recv: bad source rank");
  const std::string key = "p2p." + std::to_string(src) + "." + std::to_string(rank_) + "." + std::to_string(tag) +
                          "." + std::to_string(recv_seq_[src]++);
  auto v = kv_get(key, 1);
  if (v.size() != len)
    throw BootstrapError(GICC_EMISMATCH, "recv: expected " + std::to_string(len) + " bytes, got " +
                                             std::to_string(v.size()));
  std::memcpy(data, v.data(), len);
}

void Bootstrap::sendrecv(const void* sbuf, size_t slen, int dst, void* rbuf, size_t rlen, int src, int tag) {
  send(sbuf, slen, dst, tag);  // the store buffers it, so this cannot deadlock
  recv(rbuf, rlen, src, tag);
}

double Bootstrap::wtime() const { return now_s() - t0_; }

void Bootstrap::fail_job(int code, const std::string& msg) {
  try {
    std::string m = "code " + std::to_string(code) + ": " + msg;
    std::lock_guard<std::mutex> lk(g_req_mu);
    ReqHdr h{OP_ABORT, rank_, 0, (uint64_t)m.size(), 0};
    if (sock_ >= 0 && write_all(sock_, &h, sizeof(h)) && write_all(sock_, m.data(), m.size())) {
      RepHdr r;
      bool to = false;
      read_all_deadline(sock_, &r, sizeof(r), now_s() + 2.0, &to);
      if (r.vlen) {
        std::vector<char> junk(r.vlen);
        read_all_deadline(sock_, junk.data(), r.vlen, now_s() + 2.0, &to);
      }
    }
  } catch (...) {
  }
}

void Bootstrap::abort_job(int code, const std::string& msg) {
  std::fprintf(stderr, "[gicc] rank %d aborting job (code %d): %s\n", rank_, code, msg.c_str());
  fail_job(code, msg);
  if (rank_ == 0) ::usleep(200000);  // let the server push the failure to the others
  std::fflush(nullptr);
  ::_exit(code == 0 ? 1 : code);
}

void Bootstrap::abort(int code, const char* msg) {
  if (g_last_bootstrap) g_last_bootstrap->abort_job(code, msg ? msg : "");
  std::fprintf(stderr, "[gicc] abort (code %d): %s\n", code, msg ? msg : "");
  std::fflush(nullptr);
  ::_exit(code == 0 ? 1 : code);
}

// ------------------------------------------------------------------------------------
// fd channel
// ------------------------------------------------------------------------------------
void Bootstrap::open_fd_listener() {
  if (fd_listen_ >= 0) return;
  fd_listen_ = ::socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
  socklen_t len;
  sockaddr_un a = make_abstract(abstract_name(job_id_, rank_), &len);
  if (::bind(fd_listen_, reinterpret_cast<sockaddr*>(&a), len) != 0)
    throw BootstrapError(GICC_EBOOT, std::string("bootstrap: fd channel bind failed: ") + std::strerror(errno));
  if (::listen(fd_listen_, 256) != 0) throw BootstrapError(GICC_EBOOT, "bootstrap: fd channel listen failed");
  fd_stash_.assign(0, {});
}

namespace {
struct FdMsgHdr {
  int32_t src;
  int32_t tag;
  int32_t n;
};
}  // namespace

void Bootstrap::send_fds(int dst, int tag, const std::vector<int>& fds) {
  if (fds.size() > 250) throw BootstrapError(GICC_EINVAL, "send_fds: too many descriptors in one message");
  int s = ::socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
  socklen_t len;
  sockaddr_un a = make_abstract(abstract_name(job_id_, dst), &len);
  const double deadline = now_s() + timeout_s_;
  while (::connect(s, reinterpret_cast<sockaddr*>(&a), len) != 0) {
    if (now_s() > deadline) {
      ::close(s);
      throw BootstrapError(GICC_ETIMEDOUT, "send_fds: cannot reach rank " + std::to_string(dst));
    }
    ::usleep(5000);
  }
  FdMsgHdr h{rank_, tag, (int32_t)fds.size()};
  iovec iov{&h, sizeof(h)};
  std::vector<char> cbuf(CMSG_SPACE(sizeof(int) * std::max<size_t>(fds.size(), 1)));
  msghdr m{};
  m.msg_iov = &iov;
  m.msg_iovlen = 1;
  if (!fds.empty()) {
    m.msg_control = cbuf.data();
    m.msg_controllen = CMSG_SPACE(sizeof(int) * fds.size());
    cmsghdr* c = CMSG_FIRSTHDR(&m);
    c->cmsg_level = SOL_SOCKET;
    c->cmsg_type = SCM_RIGHTS;
    c->cmsg_len = CMSG_LEN(sizeof(int) * fds.size());
    std::memcpy(CMSG_DATA(c), fds.data(), sizeof(int) * fds.size());
  }
  ssize_t w = ::sendmsg(s, &m, MSG_NOSIGNAL);
  ::close(s);
  if (w != (ssize_t)sizeof(h)) throw BootstrapError(GICC_EBOOT, "send_fds: sendmsg failed");
}

std::vector<int> Bootstrap::recv_fds(int src, int tag, size_t n) {
  // stash layout: fd_stash_[i] = {src, tag, fds...}
  for (size_t i = 0; i < fd_stash_.size(); ++i) {
    auto& e = fd_stash_[i];
    if (e.size() >= 2 && e[0] == src && e[1] == tag) {
      std::vector<int> out(e.begin() + 2, e.end());
      fd_stash_.erase(fd_stash_.begin() + i);
      if (out.size() != n) throw BootstrapError(GICC_EMISMATCH, "recv_fds: descriptor count mismatch");
      return out;
    }
  }
  const double deadline = now_s() + timeout_s_;
  while (true) {
    double left = deadline - now_s();
    if (left <= 0) throw BootstrapError(GICC_ETIMEDOUT, "recv_fds: timed out waiting for rank " + std::to_string(src));
    pollfd pf{fd_listen_, POLLIN, 0};
    int pr = ::poll(&pf, 1, (int)std::min(left * 1000.0 + 1, 500.0));
    if (pr <= 0) {
      check();  // surface a failed job instead of waiting out the timeout
      continue;
    }
    int c = ::accept4(fd_listen_, nullptr, nullptr, SOCK_CLOEXEC);
    if (c < 0) continue;
    FdMsgHdr h{};
    iovec iov{&h, sizeof(h)};
    std::vector<char> cbuf(CMSG_SPACE(sizeof(int) * 256));
    msghdr m{};
    m.msg_iov = &iov;
    m.msg_iovlen = 1;
    m.msg_control = cbuf.data();
    m.msg_controllen = cbuf.size();
    ssize_t r = ::recvmsg(c, &m, MSG_CMSG_CLOEXEC);
    ::close(c);
    if (r != (ssize_t)sizeof(h)) continue;
    std::vector<int> fds;
    for (cmsghdr* cm = CMSG_FIRSTHDR(&m); cm; cm = CMSG_NXTHDR(&m, cm)) {
      if (cm->cmsg_level == SOL_SOCKET && cm->cmsg_type == SCM_RIGHTS) {
        size_t k = (cm->cmsg_len - CMSG_LEN(0)) / sizeof(int);
        const int* p = reinterpret_cast<const int*>(CMSG_DATA(cm));
        fds.insert(fds.end(), p, p + k);
      }
    }
    if (h.src == src && h.tag == tag) {
      if (fds.size() != n) {
        for (int fd : fds) ::close(fd);
        throw BootstrapError(GICC_EMISMATCH, "recv_fds: descriptor count mismatch");
      }
      return fds;
    }
    std::vector<int> e{h.src, h.tag};
    e.insert(e.end(), fds.begin(), fds.end());
    fd_stash_.push_back(std::move(e));
  }
}

}  // namespace gicc
