// cxengine: the native transfer engine of connex-b200 (C++17, pybind11).
//
// It provides the data-plane surface the control plane expects from a
// one-sided transfer engine (the contract of connex-rs, whose source is not
// available: the reference's connex/pp/transports.py:181-238,
// connex/rl/transport.py:114-244, tests/test_connexrs_backend.py):
//
//   Engine(model, stage, shard, replica, listen_ip, port, advertise_ip,
//          heartbeat_ms, heartbeat_timeout_ms, spin_us)
//   local_url = "ip:port#model|stage|shard|replica", port
//   allocate/free_managed_buffer, write/read_bytes_to/from_buffer
//   register_memory / unregister_memory            (0 = ok)
//   transfer_sync_read / transfer_sync_write       (0 = ok, < 0 = error)
//   get_async / put_async / put_signal -> Handle.wait(ms)
//   send_msg(peer_or_url, bytes), recv_msg(ms) -> (peer, bytes)
//   connect(url), wait_event(ms) -> {"type": up|joined|failed, "peer", "reason"}
//   stats(), close()
//
// Transport: TCP between processes (host memory).  Each connection carries
// length-prefixed frames; one-sided reads/writes are served by the owner's
// connection thread after validating the range against its registered
// regions (an unknown region answers CX_INVALID, the link stays up).  Peer
// death is detected by socket EOF (immediate when a process dies) or by a
// missed heartbeat, and reported once as a "failed" event; every request in
// flight on that link completes with CX_PEER_FAILED.  All blocking calls
// release the GIL and every wait is bounded.  Inside one NVLink box, GPU
// memory moves through CUDA-IPC peer mappings and this package's copy
// kernels instead (connex_b200.parallel.peer); this engine is the
// identity / liveness / host-memory plane.
#include <arpa/inet.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <sys/socket.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <string>
#include <thread>
#include <tuple>
#include <vector>

namespace py = pybind11;

namespace cxe {

constexpr int CX_OK = 0;
constexpr int CX_ERR = -1;
constexpr int CX_PEER_FAILED = -2;
constexpr int CX_TIMEOUT = -3;
constexpr int CX_INVALID = -4;

enum FrameType : uint8_t {
  F_HELLO = 1,      // identity string
  F_HELLO_ACK = 2,  // identity string
  F_READ_REQ = 3,   // id, addr, len
  F_READ_RESP = 4,  // id, status, [data]
  F_WRITE_REQ = 5,  // id, addr, len, flags, [msg_len, msg], data
  F_WRITE_RESP = 6, // id, status
  F_MSG = 7,        // bytes
  F_HEARTBEAT = 8,
};

using Clock = std::chrono::steady_clock;
static int64_t now_ms() {
  return std::chrono::duration_cast<std::chrono::milliseconds>(Clock::now().time_since_epoch()).count();
}

struct Identity {
  std::string model;
  int64_t stage = 0, shard = 0, replica = 0;
  std::string str() const {
    return model + "|" + std::to_string(stage) + "|" + std::to_string(shard) + "|" + std::to_string(replica);
  }
  static Identity parse(const std::string& s) {
    Identity id;
    size_t a = s.find('|'), b = s.find('|', a + 1), c = s.find('|', b + 1);
    if (a == std::string::npos || b == std::string::npos || c == std::string::npos) return id;
    id.model = s.substr(0, a);
    id.stage = std::atoll(s.substr(a + 1, b - a - 1).c_str());
    id.shard = std::atoll(s.substr(b + 1, c - b - 1).c_str());
    id.replica = std::atoll(s.substr(c + 1).c_str());
    return id;
  }
  py::tuple py() const { return py::make_tuple(model, stage, shard, replica); }
};

static bool send_all(int fd, const void* p, size_t n) {
  const char* c = static_cast<const char*>(p);
  while (n > 0) {
    ssize_t k = ::send(fd, c, n, MSG_NOSIGNAL);
    if (k <= 0) {
      if (k < 0 && errno == EINTR) continue;
      return false;
    }
    c += k;
    n -= (size_t)k;
  }
  return true;
}
static bool recv_all(int fd, void* p, size_t n) {
  char* c = static_cast<char*>(p);
  while (n > 0) {
    ssize_t k = ::recv(fd, c, n, 0);
    if (k <= 0) {
      if (k < 0 && errno == EINTR) continue;
      return false;
    }
    c += k;
    n -= (size_t)k;
  }
  return true;
}

struct Pending {
  std::mutex m;
  std::condition_variable cv;
  bool done = false;
  int status = 0;
  uint8_t* dst = nullptr;  // read destination
  uint64_t len = 0;
  void complete(int st) {
    std::lock_guard<std::mutex> g(m);
    if (!done) {
      done = true;
      status = st;
    }
    cv.notify_all();
  }
  int wait(int64_t ms) {
    std::unique_lock<std::mutex> g(m);
    if (!cv.wait_for(g, std::chrono::milliseconds(ms), [&] { return done; })) return CX_TIMEOUT;
    return status;
  }
};

struct Conn {
  int fd = -1;
  std::string addr;  // host:port dialled (outgoing) or "" (incoming)
  Identity peer;
  bool outgoing = false;
  std::mutex wmu;
  std::atomic<bool> alive{true};
  std::atomic<int64_t> last_rx{0};
  std::thread reader;
  std::mutex pmu;
  std::map<uint64_t, std::shared_ptr<Pending>> pending;
  bool send_frame(uint8_t type, const std::vector<std::pair<const void*, size_t>>& parts) {
    uint64_t total = 1;
    for (auto& p : parts) total += p.second;
    std::lock_guard<std::mutex> g(wmu);
    if (!alive) return false;
    uint64_t len = total;
    if (!send_all(fd, &len, 8) || !send_all(fd, &type, 1)) return false;
    for (auto& p : parts)
      if (p.second && !send_all(fd, p.first, p.second)) return false;
    return true;
  }
};

struct Event {
  std::string type, reason;
  Identity peer;
};

class Engine;

class Handle {
 public:
  Handle(std::shared_ptr<Pending> p, int immediate) : p_(std::move(p)), immediate_(immediate) {}
  int wait(int64_t ms) {
    if (!p_) return immediate_;
    py::gil_scoped_release nogil;
    return p_->wait(ms);
  }
  bool done() {
    if (!p_) return true;
    std::lock_guard<std::mutex> g(p_->m);
    return p_->done;
  }

 private:
  std::shared_ptr<Pending> p_;
  int immediate_;
};

class Engine {
 public:
  Engine(const std::string& model, int64_t stage, int64_t shard, int64_t replica, const std::string& listen_ip,
         int port, const std::string& advertise_ip, int heartbeat_ms, int heartbeat_timeout_ms, int spin_us)
      : hb_ms_(heartbeat_ms), hb_timeout_ms_(heartbeat_timeout_ms), spin_us_(spin_us) {
    id_.model = model;
    id_.stage = stage;
    id_.shard = shard;
    id_.replica = replica;
    lfd_ = ::socket(AF_INET, SOCK_STREAM, 0);
    if (lfd_ < 0) throw std::runtime_error("cxengine: socket() failed");
    int one = 1;
    ::setsockopt(lfd_, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    sockaddr_in a{};
    a.sin_family = AF_INET;
    a.sin_port = htons((uint16_t)port);
    if (::inet_pton(AF_INET, listen_ip.c_str(), &a.sin_addr) != 1) throw std::runtime_error("cxengine: bad listen_ip");
    if (::bind(lfd_, (sockaddr*)&a, sizeof(a)) != 0) {
      ::close(lfd_);
      throw std::runtime_error("cxengine: bind failed on " + listen_ip + ":" + std::to_string(port));
    }
    ::listen(lfd_, 128);
    socklen_t sl = sizeof(a);
    ::getsockname(lfd_, (sockaddr*)&a, &sl);
    port_ = ntohs(a.sin_port);
    std::string ip = advertise_ip.empty() ? (listen_ip == "0.0.0.0" ? std::string("127.0.0.1") : listen_ip)
                                          : advertise_ip;
    url_ = ip + ":" + std::to_string(port_) + "#" + id_.str();
    accept_thread_ = std::thread([this] { accept_loop(); });
    hb_thread_ = std::thread([this] { heartbeat_loop(); });
  }
  ~Engine() { close(); }

  std::string local_url() const { return url_; }
  int port() const { return port_; }
  py::tuple identity() const { return id_.py(); }

  // ---- memory --------------------------------------------------------------
  uint64_t allocate_managed_buffer(uint64_t size) {
    void* p = nullptr;
    if (posix_memalign(&p, 4096, size ? size : 1) != 0) throw std::bad_alloc();
    std::memset(p, 0, size);
    std::lock_guard<std::mutex> g(mmu_);
    regions_[(uintptr_t)p] = size;
    managed_.insert((uintptr_t)p);
    return (uint64_t)(uintptr_t)p;
  }
  void free_managed_buffer(uint64_t ptr, uint64_t) {
    std::lock_guard<std::mutex> g(mmu_);
    if (managed_.erase((uintptr_t)ptr)) {
      regions_.erase((uintptr_t)ptr);
      std::free((void*)(uintptr_t)ptr);
    }
  }
  void write_bytes_to_buffer(uint64_t ptr, py::bytes data, uint64_t len) {
    std::string s = data;
    if (!inside((uintptr_t)ptr, len) || s.size() < len) throw std::runtime_error("cxengine: write outside a region");
    std::memcpy((void*)(uintptr_t)ptr, s.data(), len);
  }
  py::bytes read_bytes_from_buffer(uint64_t ptr, uint64_t len) {
    if (!inside((uintptr_t)ptr, len)) throw std::runtime_error("cxengine: read outside a region");
    return py::bytes((const char*)(uintptr_t)ptr, len);
  }
  int register_memory(uint64_t ptr, uint64_t len) {
    std::lock_guard<std::mutex> g(mmu_);
    regions_[(uintptr_t)ptr] = len;
    return CX_OK;
  }
  int unregister_memory(uint64_t ptr) {
    std::lock_guard<std::mutex> g(mmu_);
    if (managed_.count((uintptr_t)ptr)) return CX_OK;  // managed buffers stay until freed
    return regions_.erase((uintptr_t)ptr) ? CX_OK : CX_INVALID;
  }

  // ---- one-sided -------------------------------------------------------------
  int transfer_sync_read(const std::string& url, uint64_t dst, uint64_t src, uint64_t len, int64_t timeout_ms) {
    py::gil_scoped_release nogil;
    auto p = start_read(url, dst, src, len);
    if (!p.first) return p.second;
    int st = p.first->wait(timeout_ms);
    finish(st);
    return st;
  }
  // writes take (url, local source, remote destination, length)
  int transfer_sync_write(const std::string& url, uint64_t local, uint64_t remote, uint64_t len, int64_t timeout_ms) {
    py::gil_scoped_release nogil;
    auto p = start_write(url, remote, local, len, nullptr, 0);
    if (!p.first) return p.second;
    int st = p.first->wait(timeout_ms);
    finish(st);
    return st;
  }
  Handle get_async(const std::string& url, uint64_t dst, uint64_t src, uint64_t len, int64_t) {
    std::pair<std::shared_ptr<Pending>, int> p;
    {
      py::gil_scoped_release nogil;
      p = start_read(url, dst, src, len);
    }
    return Handle(p.first, p.second);
  }
  Handle put_async(const std::string& url, uint64_t local, uint64_t remote, uint64_t len, int64_t) {
    std::pair<std::shared_ptr<Pending>, int> p;
    {
      py::gil_scoped_release nogil;
      p = start_write(url, remote, local, len, nullptr, 0);
    }
    return Handle(p.first, p.second);
  }
  Handle put_signal(const std::string& url, uint64_t local, uint64_t remote, uint64_t len, py::bytes msg) {
    std::string m = msg;
    std::pair<std::shared_ptr<Pending>, int> p;
    {
      py::gil_scoped_release nogil;
      p = start_write(url, remote, local, len, m.data(), m.size());
    }
    return Handle(p.first, p.second);
  }

  // ---- messages / events -------------------------------------------------------
  bool send_msg(py::object peer_or_url, py::bytes data) {
    std::string d = data;
    std::shared_ptr<Conn> c;
    if (py::isinstance<py::str>(peer_or_url)) {
      std::string url = peer_or_url.cast<std::string>();
      py::gil_scoped_release nogil;
      c = get_conn(url);
    } else {
      py::tuple t = peer_or_url.cast<py::tuple>();
      Identity want;
      want.model = t[0].cast<std::string>();
      want.stage = t[1].cast<int64_t>();
      want.shard = t[2].cast<int64_t>();
      want.replica = t[3].cast<int64_t>();
      c = conn_by_identity(want);
    }
    if (!c) return false;
    py::gil_scoped_release nogil;
    return c->send_frame(F_MSG, {{d.data(), d.size()}});
  }
  py::object recv_msg(int64_t ms) {
    std::pair<Identity, std::string> m;
    bool got = false;
    {
      py::gil_scoped_release nogil;
      std::unique_lock<std::mutex> g(qmu_);
      qcv_.wait_for(g, std::chrono::milliseconds(ms), [&] { return !msgs_.empty() || closed_; });
      if (!msgs_.empty()) {
        m = std::move(msgs_.front());
        msgs_.pop_front();
        got = true;
      }
    }
    if (!got) return py::none();
    return py::make_tuple(m.first.py(), py::bytes(m.second));
  }
  bool connect(const std::string& url) {
    py::gil_scoped_release nogil;
    return (bool)get_conn(url);
  }
  py::object wait_event(int64_t ms) {
    Event e;
    bool got = false;
    {
      py::gil_scoped_release nogil;
      std::unique_lock<std::mutex> g(qmu_);
      ecv_.wait_for(g, std::chrono::milliseconds(ms), [&] { return !events_.empty() || closed_; });
      if (!events_.empty()) {
        e = events_.front();
        events_.pop_front();
        got = true;
      }
    }
    if (!got) return py::none();
    py::dict d;
    d["type"] = e.type;
    d["peer"] = e.peer.py();
    d["reason"] = e.reason;
    return d;
  }
  py::dict stats() {
    py::dict d;
    std::lock_guard<std::mutex> g(cmu_);
    int live = 0;
    for (auto& c : conns_)
      if (c->alive) ++live;
    d["eps_created"] = eps_created_.load();
    d["eps_closed"] = eps_closed_.load();
    d["live_peers"] = live;
    {
      std::lock_guard<std::mutex> g2(mmu_);
      uint64_t bytes = 0;
      for (auto& r : regions_) bytes += r.second;
      d["regions"] = (int64_t)(regions_.size() - managed_.size());
      d["region_bytes"] = bytes;
    }
    d["remote_rkeys"] = 0;
    d["inflight"] = inflight_.load();
    d["rma_ok"] = rma_ok_.load();
    d["rma_err"] = rma_err_.load();
    d["failures"] = failures_.load();
    return d;
  }
  void close() {
    {
      std::lock_guard<std::mutex> g(qmu_);
      if (closed_) return;
      closed_ = true;
    }
    qcv_.notify_all();
    ecv_.notify_all();
    ::shutdown(lfd_, SHUT_RDWR);
    ::close(lfd_);
    std::vector<std::shared_ptr<Conn>> all;
    {
      std::lock_guard<std::mutex> g(cmu_);
      all = conns_;
    }
    for (auto& c : all) drop(c, "closed", false);
    if (accept_thread_.joinable()) accept_thread_.join();
    if (hb_thread_.joinable()) hb_thread_.join();
    for (auto& c : all)
      if (c->reader.joinable()) c->reader.join();
    std::lock_guard<std::mutex> g(mmu_);
    for (auto p : managed_) std::free((void*)p);
    managed_.clear();
    regions_.clear();
  }

 private:
  bool inside(uintptr_t p, uint64_t n) {
    std::lock_guard<std::mutex> g(mmu_);
    auto it = regions_.upper_bound(p);
    if (it == regions_.begin()) return false;
    --it;
    return p >= it->first && p + n <= it->first + it->second;
  }
  void finish(int st) {
    if (st == CX_OK) rma_ok_++;
    else rma_err_++;
  }
  void push_event(const std::string& type, const Identity& peer, const std::string& reason) {
    {
      std::lock_guard<std::mutex> g(qmu_);
      events_.push_back({type, reason, peer});
    }
    ecv_.notify_all();
  }

  static std::string host_port(const std::string& url) {
    size_t h = url.find('#');
    return h == std::string::npos ? url : url.substr(0, h);
  }

  std::shared_ptr<Conn> conn_by_identity(const Identity& want) {
    std::lock_guard<std::mutex> g(cmu_);
    for (auto it = conns_.rbegin(); it != conns_.rend(); ++it) {
      auto& c = *it;
      if (c->alive && c->peer.model == want.model && c->peer.stage == want.stage && c->peer.shard == want.shard &&
          c->peer.replica == want.replica)
        return c;
    }
    return nullptr;
  }

  std::shared_ptr<Conn> get_conn(const std::string& url) {
    const std::string hp = host_port(url);
    {
      std::lock_guard<std::mutex> g(cmu_);
      auto it = out_.find(hp);
      if (it != out_.end() && it->second->alive) return it->second;
    }
    std::lock_guard<std::mutex> dial(dial_mu_);
    {
      std::lock_guard<std::mutex> g(cmu_);
      auto it = out_.find(hp);
      if (it != out_.end() && it->second->alive) return it->second;
    }
    size_t colon = hp.rfind(':');
    if (colon == std::string::npos) return nullptr;
    std::string host = hp.substr(0, colon);
    int port = std::atoi(hp.substr(colon + 1).c_str());
    int fd = ::socket(AF_INET, SOCK_STREAM, 0);
    if (fd < 0) return nullptr;
    sockaddr_in a{};
    a.sin_family = AF_INET;
    a.sin_port = htons((uint16_t)port);
    if (::inet_pton(AF_INET, host.c_str(), &a.sin_addr) != 1 || ::connect(fd, (sockaddr*)&a, sizeof(a)) != 0) {
      ::close(fd);
      return nullptr;
    }
    int one = 1;
    ::setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
    auto c = std::make_shared<Conn>();
    c->fd = fd;
    c->addr = hp;
    c->outgoing = true;
    c->last_rx = now_ms();
    // HELLO / HELLO_ACK handshake (bounded)
    std::string me = id_.str();
    if (!c->send_frame(F_HELLO, {{me.data(), me.size()}})) {
      ::close(fd);
      return nullptr;
    }
    pollfd pf{fd, POLLIN, 0};
    if (::poll(&pf, 1, 2000) <= 0) {
      ::close(fd);
      return nullptr;
    }
    uint64_t len;
    uint8_t type;
    if (!recv_all(fd, &len, 8) || !recv_all(fd, &type, 1) || type != F_HELLO_ACK || len > 4096) {
      ::close(fd);
      return nullptr;
    }
    std::string pid(len - 1, '\0');
    if (!recv_all(fd, &pid[0], len - 1)) {
      ::close(fd);
      return nullptr;
    }
    c->peer = Identity::parse(pid);
    eps_created_++;
    {
      std::lock_guard<std::mutex> g(cmu_);
      out_[hp] = c;
      conns_.push_back(c);
    }
    c->reader = std::thread([this, c] { reader_loop(c); });
    push_event("up", c->peer, "");
    return c;
  }

  std::pair<std::shared_ptr<Pending>, int> start_read(const std::string& url, uint64_t dst, uint64_t src,
                                                      uint64_t len) {
    if (!inside((uintptr_t)dst, len)) return {nullptr, CX_INVALID};
    auto c = get_conn(url);
    if (!c) return {nullptr, CX_PEER_FAILED};
    auto p = std::make_shared<Pending>();
    p->dst = (uint8_t*)(uintptr_t)dst;
    p->len = len;
    uint64_t id = next_id_++;
    {
      std::lock_guard<std::mutex> g(c->pmu);
      c->pending[id] = p;
    }
    inflight_++;
    uint64_t hdr[3] = {id, src, len};
    if (!c->send_frame(F_READ_REQ, {{hdr, sizeof(hdr)}})) {
      drop(c, "send failed", true);
    }
    return {p, CX_OK};
  }
  std::pair<std::shared_ptr<Pending>, int> start_write(const std::string& url, uint64_t dst, uint64_t src,
                                                       uint64_t len, const char* msg, size_t mlen) {
    if (!inside((uintptr_t)src, len)) return {nullptr, CX_INVALID};
    auto c = get_conn(url);
    if (!c) return {nullptr, CX_PEER_FAILED};
    auto p = std::make_shared<Pending>();
    uint64_t id = next_id_++;
    {
      std::lock_guard<std::mutex> g(c->pmu);
      c->pending[id] = p;
    }
    inflight_++;
    uint64_t hdr[5] = {id, dst, len, (uint64_t)(msg != nullptr), (uint64_t)mlen};
    if (!c->send_frame(F_WRITE_REQ, {{hdr, sizeof(hdr)}, {msg, mlen}, {(const void*)(uintptr_t)src, len}}))
      drop(c, "send failed", true);
    return {p, CX_OK};
  }

  void complete(const std::shared_ptr<Conn>& c, uint64_t id, int st) {
    std::shared_ptr<Pending> p;
    {
      std::lock_guard<std::mutex> g(c->pmu);
      auto it = c->pending.find(id);
      if (it == c->pending.end()) return;
      p = it->second;
      c->pending.erase(it);
    }
    inflight_--;
    p->complete(st);
  }

  void drop(const std::shared_ptr<Conn>& c, const std::string& reason, bool report) {
    bool was = c->alive.exchange(false);
    if (!was) return;
    ::shutdown(c->fd, SHUT_RDWR);
    std::map<uint64_t, std::shared_ptr<Pending>> pend;
    {
      std::lock_guard<std::mutex> g(c->pmu);
      pend.swap(c->pending);
    }
    for (auto& kv : pend) {
      inflight_--;
      kv.second->complete(CX_PEER_FAILED);
    }
    eps_closed_++;
    bool closed;
    {
      std::lock_guard<std::mutex> g(qmu_);
      closed = closed_;
    }
    if (report && !closed && !c->peer.model.empty()) {
      failures_++;
      push_event("failed", c->peer, reason);
    }
  }

  void accept_loop() {
    while (true) {
      int fd = ::accept(lfd_, nullptr, nullptr);
      if (fd < 0) {
        std::lock_guard<std::mutex> g(qmu_);
        if (closed_) return;
        if (errno == EINTR) continue;
        return;
      }
      int one = 1;
      ::setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
      auto c = std::make_shared<Conn>();
      c->fd = fd;
      c->last_rx = now_ms();
      {
        std::lock_guard<std::mutex> g(cmu_);
        conns_.push_back(c);
      }
      c->reader = std::thread([this, c] { reader_loop(c); });
    }
  }

  void reader_loop(std::shared_ptr<Conn> c) {
    std::vector<uint8_t> buf;
    while (c->alive) {
      pollfd pf{c->fd, POLLIN, 0};
      int r = ::poll(&pf, 1, 100);
      if (r == 0) continue;
      if (r < 0 && errno == EINTR) continue;
      uint64_t len;
      uint8_t type;
      if (r < 0 || !recv_all(c->fd, &len, 8) || len == 0 || !recv_all(c->fd, &type, 1)) break;
      c->last_rx = now_ms();
      uint64_t body = len - 1;
      if (type == F_READ_RESP) {
        uint64_t hdr[2];
        if (!recv_all(c->fd, hdr, sizeof(hdr))) break;
        uint64_t id = hdr[0];
        int st = (int)(int64_t)hdr[1];
        uint64_t data = body - sizeof(hdr);
        std::shared_ptr<Pending> p;
        {
          std::lock_guard<std::mutex> g(c->pmu);
          auto it = c->pending.find(id);
          if (it != c->pending.end()) p = it->second;
        }
        if (data > 0) {
          if (p && st == CX_OK && data == p->len) {
            if (!recv_all(c->fd, p->dst, data)) break;
          } else {
            buf.resize(data);
            if (!recv_all(c->fd, buf.data(), data)) break;
          }
        }
        complete(c, id, st);
        continue;
      }
      buf.resize(body);
      if (body && !recv_all(c->fd, buf.data(), body)) break;
      if (type == F_HELLO) {
        c->peer = Identity::parse(std::string((char*)buf.data(), body));
        std::string me = id_.str();
        c->send_frame(F_HELLO_ACK, {{me.data(), me.size()}});
        eps_created_++;
        push_event("joined", c->peer, "");
      } else if (type == F_READ_REQ && body >= 24) {
        uint64_t hdr[3];
        std::memcpy(hdr, buf.data(), sizeof(hdr));
        if (inside((uintptr_t)hdr[1], hdr[2])) {
          uint64_t rh[2] = {hdr[0], (uint64_t)(int64_t)CX_OK};
          c->send_frame(F_READ_RESP, {{rh, sizeof(rh)}, {(const void*)(uintptr_t)hdr[1], hdr[2]}});
        } else {
          uint64_t rh[2] = {hdr[0], (uint64_t)(int64_t)CX_INVALID};
          c->send_frame(F_READ_RESP, {{rh, sizeof(rh)}});
        }
      } else if (type == F_WRITE_REQ && body >= 40) {
        uint64_t hdr[5];
        std::memcpy(hdr, buf.data(), sizeof(hdr));
        const uint64_t id = hdr[0], dst = hdr[1], n = hdr[2], has_msg = hdr[3], mlen = hdr[4];
        int st = CX_INVALID;
        if (40 + mlen + n <= body && inside((uintptr_t)dst, n)) {
          std::memcpy((void*)(uintptr_t)dst, buf.data() + 40 + mlen, n);
          st = CX_OK;
          if (has_msg) {
            {
              std::lock_guard<std::mutex> g(qmu_);
              msgs_.emplace_back(c->peer, std::string((char*)buf.data() + 40, mlen));
            }
            qcv_.notify_all();
          }
        }
        uint64_t rh[2] = {id, (uint64_t)(int64_t)st};
        c->send_frame(F_WRITE_RESP, {{rh, sizeof(rh)}});
      } else if (type == F_WRITE_RESP && body >= 16) {
        uint64_t rh[2];
        std::memcpy(rh, buf.data(), sizeof(rh));
        complete(c, rh[0], (int)(int64_t)rh[1]);
      } else if (type == F_MSG) {
        {
          std::lock_guard<std::mutex> g(qmu_);
          msgs_.emplace_back(c->peer, std::string((char*)buf.data(), body));
        }
        qcv_.notify_all();
      }
      // F_HEARTBEAT: last_rx already refreshed
    }
    drop(c, "connection lost", true);
    ::close(c->fd);
  }

  void heartbeat_loop() {
    while (true) {
      {
        std::unique_lock<std::mutex> g(qmu_);
        if (ecv_.wait_for(g, std::chrono::milliseconds(hb_ms_ > 0 ? hb_ms_ : 1000), [&] { return closed_; })) return;
      }
      std::vector<std::shared_ptr<Conn>> all;
      {
        std::lock_guard<std::mutex> g(cmu_);
        all = conns_;
      }
      const int64_t t = now_ms();
      for (auto& c : all) {
        if (!c->alive) continue;
        if (hb_timeout_ms_ > 0 && t - c->last_rx > hb_timeout_ms_) {
          drop(c, "heartbeat timeout", true);
          continue;
        }
        c->send_frame(F_HEARTBEAT, {});
      }
    }
  }

  Identity id_;
  int lfd_ = -1;
  int port_ = 0;
  std::string url_;
  int hb_ms_, hb_timeout_ms_, spin_us_;
  std::thread accept_thread_, hb_thread_;
  std::mutex cmu_, dial_mu_;
  std::vector<std::shared_ptr<Conn>> conns_;
  std::map<std::string, std::shared_ptr<Conn>> out_;
  std::mutex mmu_;
  std::map<uintptr_t, uint64_t> regions_;
  std::set<uintptr_t> managed_;
  std::mutex qmu_;
  std::condition_variable qcv_, ecv_;
  std::deque<std::pair<Identity, std::string>> msgs_;
  std::deque<Event> events_;
  bool closed_ = false;
  std::atomic<uint64_t> next_id_{1};
  std::atomic<int64_t> inflight_{0}, rma_ok_{0}, rma_err_{0}, failures_{0}, eps_created_{0}, eps_closed_{0};
};

}  // namespace cxe

PYBIND11_MODULE(_cxengine, m) {
  using namespace cxe;
  m.doc() = "connex-b200 native transfer engine";
  m.attr("OK") = CX_OK;
  m.attr("PEER_FAILED") = CX_PEER_FAILED;
  m.attr("TIMEOUT") = CX_TIMEOUT;
  m.attr("INVALID") = CX_INVALID;
  py::class_<Handle>(m, "Handle").def("wait", &Handle::wait, py::arg("ms") = 5000).def("done", &Handle::done);
  py::class_<Engine>(m, "Engine")
      .def(py::init<const std::string&, int64_t, int64_t, int64_t, const std::string&, int, const std::string&, int,
                    int, int>(),
           py::arg("model"), py::arg("stage"), py::arg("shard") = 0, py::arg("replica") = 0,
           py::arg("listen_ip") = "0.0.0.0", py::arg("port") = 0, py::arg("advertise_ip") = "",
           py::arg("heartbeat_ms") = 1000, py::arg("heartbeat_timeout_ms") = 3000, py::arg("spin_us") = 500)
      .def_property_readonly("local_url", &Engine::local_url)
      .def_property_readonly("port", &Engine::port)
      .def_property_readonly("identity", &Engine::identity)
      .def("allocate_managed_buffer", &Engine::allocate_managed_buffer)
      .def("free_managed_buffer", &Engine::free_managed_buffer)
      .def("write_bytes_to_buffer", &Engine::write_bytes_to_buffer)
      .def("read_bytes_from_buffer", &Engine::read_bytes_from_buffer)
      .def("register_memory", &Engine::register_memory)
      .def("unregister_memory", &Engine::unregister_memory)
      .def("transfer_sync_read", &Engine::transfer_sync_read, py::arg("url"), py::arg("dst"), py::arg("src"),
           py::arg("length"), py::arg("timeout_ms") = 5000)
      .def("transfer_sync_write", &Engine::transfer_sync_write, py::arg("url"), py::arg("local"), py::arg("remote"),
           py::arg("length"), py::arg("timeout_ms") = 5000)
      .def("get_async", &Engine::get_async, py::arg("url"), py::arg("dst"), py::arg("src"), py::arg("length"),
           py::arg("timeout_ms") = 5000)
      .def("put_async", &Engine::put_async, py::arg("url"), py::arg("local"), py::arg("remote"), py::arg("length"),
           py::arg("timeout_ms") = 5000)
      .def("put_signal", &Engine::put_signal)
      .def("send_msg", &Engine::send_msg)
      .def("recv_msg", &Engine::recv_msg, py::arg("ms") = 1000)
      .def("connect", &Engine::connect)
      .def("wait_event", &Engine::wait_event, py::arg("ms") = 1000)
      .def("stats", &Engine::stats)
      .def("close", &Engine::close);
}
