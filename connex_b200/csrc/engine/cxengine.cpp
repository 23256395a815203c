// cxengine: the native transfer engine of connex-b200 (C++17, pybind11).
//
// It provides the data-plane surface the control plane expects from a
// one-sided transfer engine (the contract of connex-rs, whose source is not
// available: the reference's connex/pp/transports.py:181-238,
// connex/rl/transport.py:114-244, connex/adapters/vllm/pp/rdmachan.py:271-293,
// tests/test_connexrs_backend.py):
//
//   Engine(model, stage, shard, replica, listen_ip, port, advertise_ip,
//          heartbeat_ms, heartbeat_timeout_ms, spin_us)
//   local_url = "ip:port#model|stage|shard|replica", port
//   allocate/free_managed_buffer (host), allocate/free_device_buffer (GPU),
//   write/read_bytes_to/from_buffer
//   register_memory / unregister_memory            (0 = ok)
//   transfer_sync_read / transfer_sync_write       (0 = ok, < 0 = error)
//   get_async / put_async / put_signal / put_chain -> Handle.wait(ms)
//   send_msg(peer_or_url, bytes), recv_msg(ms) -> (peer, bytes)
//   connect(url), wait_event(ms) -> {"type": up|joined|failed, "peer", "reason"}
//   reap(ms), stats(), close()
//
// Two data planes behind one surface, chosen per region:
//
// * host memory -- length-prefixed frames over TCP; one-sided reads and
//   writes are served by the owner's connection thread after validating the
//   range against its registered HOST regions.  A device address is never
//   served on this path (it answers CX_INVALID): the owner would otherwise
//   memcpy a device pointer on the host.
// * device memory -- a registered GPU range is exported (engine-allocated
//   buffers as VMM allocations whose fd a same-user peer fetches over a Unix
//   socket; other device allocations through their legacy IPC handle).  A
//   peer on the same machine maps it once and moves bytes with the copy
//   engines (cuMemcpyAsync on a per-device stream, over NVLink between GPUs),
//   every wait bounded by an event polled against a deadline.
//
// A peer's region is resolved once per connection (kind, size, export
// handle) and cached; an owner that drops a region tells its peers, and a
// peer that dies takes its mappings to the graveyard: each is released once
// the last copy that touched it has passed, so the physical memory of a dead
// exporter is freed as soon as no copy can reach it any more.
//
// put_chain is the doorbell -> gate -> copy -> flag chain of a ring channel:
// it waits (bounded) until a local doorbell word reaches a value (written by
// a GPU stream), until the receiver's gate word says the slot is free, then
// copies the payload and writes the receiver's flag word after it; chains on
// one queue run in order, queues run in parallel, a cancel word aborts.
//
// Peer death is detected by socket EOF (immediate when a process dies) or by
// a missed heartbeat, and reported once as a "failed" event; every request
// in flight on that link completes with CX_PEER_FAILED.  All blocking calls
// release the GIL and every wait is bounded.
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

#include "devmem.h"

namespace py = pybind11;

namespace cxe {

constexpr int CX_OK = 0;
constexpr int CX_ERR = -1;
constexpr int CX_PEER_FAILED = -2;
constexpr int CX_TIMEOUT = -3;
constexpr int CX_INVALID = -4;
constexpr int CX_CANCELLED = -5;

enum FrameType : uint8_t {
  F_HELLO = 1,        // identity string
  F_HELLO_ACK = 2,    // identity string
  F_READ_REQ = 3,     // id, addr, len
  F_READ_RESP = 4,    // id, status, [data]
  F_WRITE_REQ = 5,    // id, addr, len, flags, [msg_len, msg], data
  F_WRITE_RESP = 6,   // id, status
  F_MSG = 7,          // bytes
  F_HEARTBEAT = 8,
  F_REGION_REQ = 9,   // id, addr, len
  F_REGION_RESP = 10, // id, RegionWire
  F_REGION_GONE = 11, // base of a region the owner dropped
};

using Clock = std::chrono::steady_clock;
static int64_t now_ms() {
  return std::chrono::duration_cast<std::chrono::milliseconds>(Clock::now().time_since_epoch()).count();
}
// wrap-around order of 32-bit sequence words: has `v` reached `want`?
static bool reached(uint32_t v, uint32_t want) { return (int32_t)(v - want) >= 0; }

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
  std::vector<uint8_t> payload;  // region answers, and reads into a buffer the request owns
  bool counted = true;           // a transfer (counted in flight), not a region question
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

// A local registered range.
struct Region {
  uint64_t len = 0;
  uint32_t kind = RK_HOST;
  int device = -1;
  uint64_t alloc_base = 0, alloc_size = 0, export_id = 0;
  uint8_t ipc[CU_IPC_HANDLE_SIZE] = {};
};

// A peer's region as this side knows it; device regions carry their mapping.
struct RemoteRegion {
  RegionWire w;
  std::mutex m;
  Import im;             // im.base != 0 once mapped
  uint64_t granted = 0;  // local devices the mapping is accessible from (bit mask)
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
  std::mutex rmu;
  std::map<uint64_t, std::shared_ptr<RemoteRegion>> remote;  // by the region's base in the peer
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

// One ordered job queue (a thread) of put_chain / device-path async jobs.
class Worker {
 public:
  Worker() : th_([this] { loop(); }) {}
  ~Worker() {
    {
      std::lock_guard<std::mutex> g(m_);
      stop_ = true;
    }
    cv_.notify_all();
    th_.join();
  }
  void post(std::function<int()> job, std::shared_ptr<Pending> p) {
    {
      std::lock_guard<std::mutex> g(m_);
      if (!stop_) {
        q_.emplace_back(std::move(job), std::move(p));
        cv_.notify_all();
        return;
      }
    }
    p->complete(CX_PEER_FAILED);
  }

 private:
  void loop() {
    while (true) {
      std::pair<std::function<int()>, std::shared_ptr<Pending>> j;
      {
        std::unique_lock<std::mutex> g(m_);
        cv_.wait(g, [&] { return stop_ || !q_.empty(); });
        if (q_.empty()) return;
        j = std::move(q_.front());
        q_.pop_front();
        if (stop_) {  // closing: do not start new work
          g.unlock();
          j.second->complete(CX_PEER_FAILED);
          continue;
        }
      }
      int st = CX_ERR;
      try {
        st = j.first();
      } catch (...) {
        st = CX_ERR;
      }
      j.second->complete(st);
    }
  }
  std::mutex m_;
  std::condition_variable cv_;
  std::deque<std::pair<std::function<int()>, std::shared_ptr<Pending>>> q_;
  bool stop_ = false;
  std::thread th_;
};

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
  void set_device(int device) { home_device_ = device; }
  int device() const { return home_device_; }

  // ---- memory --------------------------------------------------------------
  uint64_t allocate_managed_buffer(uint64_t size) {
    void* p = nullptr;
    if (posix_memalign(&p, 4096, size ? size : 1) != 0) throw std::bad_alloc();
    std::memset(p, 0, size);
    Region r;
    r.len = size;
    std::lock_guard<std::mutex> g(mmu_);
    regions_[(uintptr_t)p] = r;
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
  // GPU memory peers can map: a VMM allocation on `device`, registered.
  uint64_t allocate_device_buffer(uint64_t size, int device) {
    VmmAlloc a;
    {
      py::gil_scoped_release nogil;
      a = vmm_create(size, device, next_alloc_++);
    }
    Region r;
    r.len = size;
    r.kind = RK_VMM;
    r.device = device;
    r.alloc_base = a.ptr;
    r.alloc_size = a.size;
    r.export_id = a.id;
    std::lock_guard<std::mutex> g(mmu_);
    vmm_[a.id] = a;
    regions_[(uintptr_t)a.ptr] = r;
    return (uint64_t)a.ptr;
  }
  void free_device_buffer(uint64_t ptr) {
    VmmAlloc a;
    {
      std::lock_guard<std::mutex> g(mmu_);
      auto it = regions_.find((uintptr_t)ptr);
      if (it == regions_.end() || it->second.kind != RK_VMM) throw std::runtime_error("cxengine: not a device buffer");
      a = vmm_.at(it->second.export_id);
      vmm_.erase(it->second.export_id);
      regions_.erase(it);
    }
    announce_gone(ptr);
    py::gil_scoped_release nogil;
    vmm_destroy(a);  // importers keep the memory until their graveyards release it
  }
  void write_bytes_to_buffer(uint64_t ptr, py::bytes data, uint64_t len) {
    std::string s = data;
    Region r;
    if (!find_region((uintptr_t)ptr, len, &r) || s.size() < len) throw std::runtime_error("cxengine: write outside a region");
    if (r.kind == RK_HOST) {
      std::memcpy((void*)(uintptr_t)ptr, s.data(), len);
      return;
    }
    py::gil_scoped_release nogil;
    if (dev_copy(r.device, ptr, (uint64_t)(uintptr_t)s.data(), len, nullptr, 10000) != CX_OK)
      throw std::runtime_error("cxengine: device write failed");
  }
  py::bytes read_bytes_from_buffer(uint64_t ptr, uint64_t len) {
    Region r;
    if (!find_region((uintptr_t)ptr, len, &r)) throw std::runtime_error("cxengine: read outside a region");
    if (r.kind == RK_HOST) return py::bytes((const char*)(uintptr_t)ptr, len);
    std::string out(len, '\0');
    int st;
    {
      py::gil_scoped_release nogil;
      st = dev_copy(r.device, (uint64_t)(uintptr_t)&out[0], ptr, len, nullptr, 10000);
    }
    if (st != CX_OK) throw std::runtime_error("cxengine: device read failed");
    return py::bytes(out);
  }
  int register_memory(uint64_t ptr, uint64_t len) {
    Region r = classify((uintptr_t)ptr, len);
    std::lock_guard<std::mutex> g(mmu_);
    regions_[(uintptr_t)ptr] = r;
    return CX_OK;
  }
  int unregister_memory(uint64_t ptr) {
    uint32_t kind;
    {
      std::lock_guard<std::mutex> g(mmu_);
      if (managed_.count((uintptr_t)ptr)) return CX_OK;  // managed buffers stay until freed
      auto it = regions_.find((uintptr_t)ptr);
      if (it == regions_.end()) return CX_INVALID;
      if (it->second.kind == RK_VMM && it->second.alloc_base == ptr) return CX_OK;  // freed by free_device_buffer
      kind = it->second.kind;
      regions_.erase(it);
    }
    if (kind != RK_HOST) announce_gone(ptr);
    return CX_OK;
  }
  std::string region_kind(uint64_t ptr) {
    Region r;
    if (!find_region((uintptr_t)ptr, 1, &r)) return "none";
    return kind_name(r.kind);
  }

  // ---- one-sided -------------------------------------------------------------
  int transfer_sync_read(const std::string& url, uint64_t dst, uint64_t src, uint64_t len, int64_t timeout_ms) {
    py::gil_scoped_release nogil;
    int st = transfer(url, dst, src, len, false, timeout_ms, nullptr);
    finish(st);
    return st;
  }
  // writes take (url, local source, remote destination, length)
  int transfer_sync_write(const std::string& url, uint64_t local, uint64_t remote, uint64_t len, int64_t timeout_ms) {
    py::gil_scoped_release nogil;
    int st = transfer(url, local, remote, len, true, timeout_ms, nullptr);
    finish(st);
    return st;
  }
  Handle get_async(const std::string& url, uint64_t dst, uint64_t src, uint64_t len, int64_t timeout_ms) {
    py::gil_scoped_release nogil;
    return async_transfer(url, dst, src, len, false, timeout_ms, std::string(), false);
  }
  Handle put_async(const std::string& url, uint64_t local, uint64_t remote, uint64_t len, int64_t timeout_ms) {
    py::gil_scoped_release nogil;
    return async_transfer(url, local, remote, len, true, timeout_ms, std::string(), false);
  }
  Handle put_signal(const std::string& url, uint64_t local, uint64_t remote, uint64_t len, py::bytes msg) {
    std::string m = msg;
    py::gil_scoped_release nogil;
    return async_transfer(url, local, remote, len, true, 30000, m, true);
  }
  Handle put_chain(const std::string& url, uint64_t bell, uint32_t bell_value, uint64_t gate, uint32_t gate_value,
                   uint64_t src, uint64_t dst, uint64_t len, uint64_t flag, uint32_t flag_value, int64_t queue,
                   int64_t timeout_ms, uint64_t cancel, int64_t arm_timeout_ms) {
    auto p = std::make_shared<Pending>();
    inflight_++;
    auto job = [=]() -> int {
      int st = chain(url, bell, bell_value, gate, gate_value, src, dst, len, flag, flag_value, timeout_ms, cancel,
                     arm_timeout_ms);
      inflight_--;
      finish(st);
      (st == CX_OK ? chains_ok_ : chains_err_)++;
      return st;
    };
    py::gil_scoped_release nogil;
    worker(queue).post(job, p);
    return Handle(p, CX_OK);
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
  // Release the graveyard's mappings whose copies have passed, waiting up to
  // `ms` for the rest; returns how many are still held.
  int64_t reap(int64_t ms) {
    py::gil_scoped_release nogil;
    return (int64_t)(ms > 0 ? graveyard_.drain(ms) : graveyard_.reap());
  }
  py::dict stats() {
    py::dict d;
    std::lock_guard<std::mutex> g(cmu_);
    int live = 0;
    int64_t imports = 0, import_bytes = 0;
    for (auto& c : conns_) {
      if (c->alive) ++live;
      std::lock_guard<std::mutex> r(c->rmu);
      for (auto& kv : c->remote)
        if (kv.second->im.base) {
          imports++;
          import_bytes += (int64_t)kv.second->im.size;
        }
    }
    d["eps_created"] = eps_created_.load();
    d["eps_closed"] = eps_closed_.load();
    d["live_peers"] = live;
    {
      std::lock_guard<std::mutex> g2(mmu_);
      uint64_t bytes = 0;
      int64_t dev = 0;
      for (auto& r : regions_) {
        bytes += r.second.len;
        if (r.second.kind != RK_HOST) dev++;
      }
      d["regions"] = (int64_t)(regions_.size() - managed_.size());
      d["device_regions"] = dev;
      d["region_bytes"] = bytes;
    }
    d["remote_rkeys"] = imports;
    d["imports"] = imports;
    d["import_bytes"] = import_bytes;
    d["graveyard"] = (int64_t)graveyard_.pending();
    d["released"] = (int64_t)graveyard_.released();
    d["released_bytes"] = (int64_t)graveyard_.released_bytes();
    d["dev_copies"] = dev_copies_.load();
    d["chains_ok"] = chains_ok_.load();
    d["chains_err"] = chains_err_.load();
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
    py::gil_scoped_release nogil;
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
    {
      std::lock_guard<std::mutex> g(wmu_);
      workers_.clear();  // joins: jobs in flight finish (every wait in them is bounded)
    }
    graveyard_.drain(2000);  // a mapping a copy still uses is kept (a leak beats a fault)
    fds_.reset();
    std::map<uint64_t, VmmAlloc> vmm;
    {
      std::lock_guard<std::mutex> g(mmu_);
      for (auto p : managed_) std::free((void*)p);
      managed_.clear();
      regions_.clear();
      vmm.swap(vmm_);
    }
    for (auto& kv : vmm) vmm_destroy(kv.second);
  }

 private:
  // ---- regions ----------------------------------------------------------------
  bool find_region(uintptr_t p, uint64_t n, Region* out, uintptr_t* start = nullptr) {
    std::lock_guard<std::mutex> g(mmu_);
    auto it = regions_.upper_bound(p);
    if (it == regions_.begin()) return false;
    --it;
    if (!(p >= it->first && p + n <= it->first + it->second.len)) return false;
    if (out) *out = it->second;
    if (start) *start = it->first;
    return true;
  }
  bool inside_host(uintptr_t p, uint64_t n) {
    Region r;
    return find_region(p, n, &r) && r.kind == RK_HOST;
  }

  // What kind of memory [p, p+len) is, and how a peer can reach it.
  Region classify(uintptr_t p, uint64_t len) {
    Region r;
    r.len = len;
    const Driver& d = driver();
    if (!d.ok) return r;
    unsigned int mt = 0, managed = 0;
    if (d.PointerGetAttribute(&mt, CU_POINTER_ATTRIBUTE_MEMORY_TYPE, (CUdeviceptr)p) != CUDA_SUCCESS ||
        mt != CU_MEMORYTYPE_DEVICE)
      return r;  // host (pageable or pinned)
    if (d.PointerGetAttribute(&managed, CU_POINTER_ATTRIBUTE_IS_MANAGED, (CUdeviceptr)p) == CUDA_SUCCESS && managed)
      return r;  // managed memory is host-accessible
    int dev = 0;
    d.PointerGetAttribute(&dev, CU_POINTER_ATTRIBUTE_DEVICE_ORDINAL, (CUdeviceptr)p);
    r.device = dev;
    r.kind = RK_DEVICE_LOCAL;
    {
      std::lock_guard<std::mutex> g(mmu_);
      for (auto& kv : vmm_) {
        const VmmAlloc& a = kv.second;
        if (p >= a.ptr && p + len <= a.ptr + a.size) {
          r.kind = RK_VMM;
          r.alloc_base = a.ptr;
          r.alloc_size = a.size;
          r.export_id = a.id;
          return r;
        }
      }
    }
    d.use_device(dev);
    CUdeviceptr base = 0;
    size_t size = 0;
    CUipcMemHandle h;
    if (d.MemGetAddressRange(&base, &size, (CUdeviceptr)p) == CUDA_SUCCESS && d.IpcGetMemHandle(&h, base) == CUDA_SUCCESS) {
      r.kind = RK_IPC;
      r.alloc_base = base;
      r.alloc_size = size;
      std::memcpy(r.ipc, h.reserved, CU_IPC_HANDLE_SIZE);
    }
    return r;
  }

  RegionWire describe(uint64_t addr, uint64_t len) {
    RegionWire w;
    Region r;
    uintptr_t start = 0;
    if (!find_region((uintptr_t)addr, len, &r, &start)) {
      w.status = CX_INVALID;
      return w;
    }
    w.kind = r.kind;
    w.device = r.device;
    w.base = start;
    w.size = r.len;
    std::string host = boot_id();
    std::strncpy(w.host, host.c_str(), sizeof(w.host) - 1);
    if (r.kind == RK_DEVICE_LOCAL) {
      w.status = CX_INVALID;  // device memory that cannot be exported
    } else if (r.kind == RK_VMM || r.kind == RK_IPC) {
      w.alloc_offset = start - r.alloc_base;
      w.alloc_size = r.alloc_size;
      w.export_id = r.export_id;
      std::memcpy(w.ipc, r.ipc, sizeof(w.ipc));
      if (r.kind == RK_VMM) {
        std::string name = fd_server().name();
        std::strncpy(w.sock, name.c_str(), sizeof(w.sock) - 1);
      }
    }
    return w;
  }

  FdServer& fd_server() {
    std::lock_guard<std::mutex> g(fmu_);
    if (!fds_)
      fds_ = std::make_unique<FdServer>([this](uint64_t id) {
        std::lock_guard<std::mutex> l(mmu_);
        auto it = vmm_.find(id);
        return it == vmm_.end() ? -1 : vmm_export_fd(it->second);
      });
    return *fds_;
  }

  void announce_gone(uint64_t base) {
    std::vector<std::shared_ptr<Conn>> all;
    {
      std::lock_guard<std::mutex> g(cmu_);
      all = conns_;
    }
    for (auto& c : all)
      if (c->alive) c->send_frame(F_REGION_GONE, {{&base, 8}});
  }

  // ---- peer regions --------------------------------------------------------------
  std::shared_ptr<RemoteRegion> resolve(const std::shared_ptr<Conn>& c, uint64_t addr, uint64_t len, int64_t timeout_ms,
                                        int& st) {
    {
      std::lock_guard<std::mutex> g(c->rmu);
      auto it = c->remote.upper_bound(addr);
      if (it != c->remote.begin()) {
        --it;
        const RegionWire& w = it->second->w;
        if (addr >= w.base && addr + len <= w.base + w.size) return it->second;
      }
    }
    auto p = std::make_shared<Pending>();
    p->counted = false;
    uint64_t id = next_id_++;
    {
      std::lock_guard<std::mutex> g(c->pmu);
      c->pending[id] = p;
    }
    uint64_t hdr[3] = {id, addr, len};
    if (!c->send_frame(F_REGION_REQ, {{hdr, sizeof(hdr)}})) drop(c, "send failed", true);
    st = p->wait(timeout_ms);
    if (st != CX_OK) {
      std::lock_guard<std::mutex> g(c->pmu);
      c->pending.erase(id);
      return nullptr;
    }
    if (p->payload.size() != sizeof(RegionWire)) {
      st = CX_ERR;
      return nullptr;
    }
    auto rr = std::make_shared<RemoteRegion>();
    std::memcpy(&rr->w, p->payload.data(), sizeof(RegionWire));
    if (rr->w.status != CX_OK) {
      st = (int)rr->w.status;
      return nullptr;
    }
    if (rr->w.kind != RK_HOST && std::string(rr->w.host) != boot_id()) {
      st = CX_INVALID;  // device memory of another machine: no GPU RDMA on this transport
      return nullptr;
    }
    std::lock_guard<std::mutex> g(c->rmu);
    auto ins = c->remote.emplace(rr->w.base, rr);
    if (!ins.second) {
      if (ins.first->second->w.size >= rr->w.size) return ins.first->second;  // raced: keep the mapped one
      bury(ins.first->second);
      ins.first->second = rr;
    }
    return rr;
  }

  // The local address of the peer's byte `addr` in a mapping usable from `device`.
  bool map_remote(RemoteRegion& rr, int device, uint64_t addr, CUdeviceptr* out, std::string& why) {
    std::lock_guard<std::mutex> g(rr.m);
    const Driver& d = driver();
    if (!d.ok) {
      why = d.why;
      return false;
    }
    if (!rr.im.base) {
      bool ok;
      if (rr.w.kind == RK_VMM) {
        int fd = FdServer::fetch(rr.w.sock, rr.w.export_id, 2000);
        if (fd < 0) {
          why = "could not fetch the exported allocation";
          return false;
        }
        ok = import_vmm(fd, rr.w.alloc_size, device, rr.im, why);
      } else {
        ok = import_ipc(rr.w.ipc, rr.w.alloc_size, device, rr.im, why);
      }
      if (!ok) return false;
      rr.granted = 1ull << device;
    } else if (rr.im.kind == RK_VMM && !(rr.granted & (1ull << device))) {
      try {
        grant(rr.im.base, rr.im.size, device);
      } catch (const std::exception& e) {
        why = e.what();
        return false;
      }
      rr.granted |= 1ull << device;
    }
    *out = rr.im.base + rr.w.alloc_offset + (addr - rr.w.base);
    return true;
  }

  void bury(const std::shared_ptr<RemoteRegion>& rr) {
    if (!rr->im.base) return;
    graveyard_.bury({[rr] {
                       std::lock_guard<std::mutex> g(rr->m);
                       return rr->im.passed();
                     },
                     [rr] {
                       std::lock_guard<std::mutex> g(rr->m);
                       release_import(rr->im);
                     },
                     rr->im.size});
  }

  // ---- device copies --------------------------------------------------------------
  CUstream stream_for(int device) {
    std::lock_guard<std::mutex> g(smu_);
    auto it = streams_.find(device);
    if (it != streams_.end()) return it->second;
    CUstream s = nullptr;
    driver().check(driver().StreamCreate(&s, CU_STREAM_NON_BLOCKING), "cuStreamCreate");
    streams_[device] = s;
    return s;
  }

  // dst <- src (any two addresses the device can reach), bounded wait.
  int dev_copy(int device, uint64_t dst, uint64_t src, uint64_t len, RemoteRegion* touched, int64_t timeout_ms) {
    const Driver& d = driver();
    if (!d.ok || !d.use_device(device)) return CX_INVALID;
    CUstream s;
    try {
      s = stream_for(device);
    } catch (const std::exception&) {
      return CX_ERR;
    }
    CUevent ev = nullptr;
    if (d.EventCreate(&ev, CU_EVENT_DISABLE_TIMING) != CUDA_SUCCESS) return CX_ERR;
    int st = CX_OK;
    if (d.MemcpyAsync((CUdeviceptr)dst, (CUdeviceptr)src, len, s) != CUDA_SUCCESS) st = CX_ERR;
    if (touched) {
      std::lock_guard<std::mutex> g(touched->m);
      if (!touched->im.last) d.EventCreate(&touched->im.last, CU_EVENT_DISABLE_TIMING);
      if (touched->im.last) d.EventRecord(touched->im.last, s);  // the graveyard waits for this one
    }
    d.EventRecord(ev, s);
    if (st == CX_OK) {
      int w = wait_for_event(ev, timeout_ms);
      st = w == 0 ? CX_OK : (w == -3 ? CX_TIMEOUT : CX_ERR);
    }
    d.EventDestroy(ev);
    dev_copies_++;
    return st;
  }

  // ---- transfers ---------------------------------------------------------------------
  // One-sided transfer between local [local, +len) (described by `lr`) and the
  // peer's [remote, +len); `write` moves local -> remote.
  // `scratch`: `local` is a buffer of the caller's that may not outlive a
  // timed-out request (reads then land in a buffer the request owns).
  int transfer_with(const std::shared_ptr<Conn>& c, const Region& lr, uint64_t local, uint64_t remote, uint64_t len,
                    bool write, int64_t timeout_ms, const std::string* msg, bool scratch = false) {
    int st = CX_OK;
    auto rr = resolve(c, remote, len, timeout_ms, st);
    if (!rr) return st;
    if (rr->w.kind == RK_HOST) {
      if (lr.kind == RK_HOST) {
        if (write)
          return start_write(c, remote, local, len, msg ? msg->data() : nullptr, msg ? msg->size() : 0)->wait(timeout_ms);
        if (!scratch) return start_read(c, local, remote, len)->wait(timeout_ms);
        auto p = start_read(c, 0, remote, len);
        st = p->wait(timeout_ms);
        if (st == CX_OK) std::memcpy((void*)(uintptr_t)local, p->payload.data(), len);
        return st;
      }
      // local device memory, remote host memory: through a host bounce buffer
      if (write) {
        std::vector<uint8_t> tmp(len);
        uint64_t t = (uint64_t)(uintptr_t)tmp.data();
        st = dev_copy(lr.device, t, local, len, nullptr, timeout_ms);
        if (st != CX_OK) return st;
        return start_write(c, remote, t, len, msg ? msg->data() : nullptr, msg ? msg->size() : 0)->wait(timeout_ms);
      }
      auto p = start_read(c, 0, remote, len);
      st = p->wait(timeout_ms);
      return st == CX_OK ? dev_copy(lr.device, local, (uint64_t)(uintptr_t)p->payload.data(), len, nullptr, timeout_ms)
                         : st;
    }
    const int device = lr.kind == RK_HOST ? home_device_ : lr.device;
    CUdeviceptr peer = 0;
    std::string why;
    if (!map_remote(*rr, device, remote, &peer, why)) return CX_INVALID;
    st = write ? dev_copy(device, peer, local, len, rr.get(), timeout_ms)
               : dev_copy(device, local, peer, len, rr.get(), timeout_ms);
    if (st == CX_OK && msg) {  // put_signal: the message follows the landed bytes
      if (!c->send_frame(F_MSG, {{msg->data(), msg->size()}})) st = CX_PEER_FAILED;
    }
    return st;
  }

  int transfer(const std::string& url, uint64_t local, uint64_t remote, uint64_t len, bool write, int64_t timeout_ms,
               const std::string* msg) {
    Region lr;
    if (!find_region((uintptr_t)local, len, &lr)) return CX_INVALID;
    auto c = get_conn(url);
    if (!c) return CX_PEER_FAILED;
    return transfer_with(c, lr, local, remote, len, write, timeout_ms, msg);
  }

  Handle async_transfer(const std::string& url, uint64_t local, uint64_t remote, uint64_t len, bool write,
                        int64_t timeout_ms, const std::string& msg, bool with_msg) {
    Region lr;
    if (!find_region((uintptr_t)local, len, &lr)) return Handle(nullptr, CX_INVALID);
    auto c = get_conn(url);
    if (!c) return Handle(nullptr, CX_PEER_FAILED);
    // host <-> host with the peer's region known: a frame, answered by its reader
    if (lr.kind == RK_HOST) {
      std::shared_ptr<RemoteRegion> known;
      {
        std::lock_guard<std::mutex> g(c->rmu);
        auto it = c->remote.upper_bound(remote);
        if (it != c->remote.begin() && (--it)->second->w.kind == RK_HOST &&
            remote >= it->second->w.base && remote + len <= it->second->w.base + it->second->w.size)
          known = it->second;
      }
      if (known) {
        auto p = write ? start_write(c, remote, local, len, with_msg ? msg.data() : nullptr, msg.size())
                       : start_read(c, local, remote, len);
        return Handle(p, CX_OK);
      }
    }
    auto p = std::make_shared<Pending>();
    inflight_++;
    worker(0).post(
        [=]() -> int {
          int st = transfer_with(c, lr, local, remote, len, write, timeout_ms, with_msg ? &msg : nullptr);
          inflight_--;
          finish(st);
          return st;
        },
        p);
    return Handle(p, CX_OK);
  }

  // ---- put_chain ------------------------------------------------------------------------
  bool read_local_u32(uint64_t ptr, uint32_t* v) {
    Region r;
    if (!find_region((uintptr_t)ptr, 4, &r)) r = classify((uintptr_t)ptr, 4);
    if (r.kind == RK_HOST) {
      *v = __atomic_load_n((const uint32_t*)(uintptr_t)ptr, __ATOMIC_ACQUIRE);
      return true;
    }
    return dev_copy(r.device, (uint64_t)(uintptr_t)v, ptr, 4, nullptr, 1000) == CX_OK;
  }
  // busy-poll about spin_us, then sleep between polls
  void backoff(int& spins) {
    if (++spins > spin_us_) std::this_thread::sleep_for(std::chrono::microseconds(20));
    else std::this_thread::yield();
  }

  int chain(const std::string& url, uint64_t bell, uint32_t bell_value, uint64_t gate, uint32_t gate_value,
            uint64_t src, uint64_t dst, uint64_t len, uint64_t flag, uint32_t flag_value, int64_t timeout_ms,
            uint64_t cancel, int64_t arm_timeout_ms) {
    auto cancelled = [&] {
      uint32_t v = 0;
      return cancel && read_local_u32(cancel, &v) && v != 0;
    };
    // 1. doorbell: the producing stream has written the payload
    if (bell) {
      const int64_t end = now_ms() + (arm_timeout_ms >= 0 ? arm_timeout_ms : timeout_ms);
      int spins = 0;
      while (true) {
        uint32_t v = 0;
        if (!read_local_u32(bell, &v)) return CX_INVALID;
        if (reached(v, bell_value)) break;
        if (cancelled()) return CX_CANCELLED;
        if (now_ms() > end) return CX_TIMEOUT;
        backoff(spins);
      }
    }
    Region lr;
    if (!find_region((uintptr_t)src, len, &lr)) return CX_INVALID;
    auto c = get_conn(url);
    if (!c) return CX_PEER_FAILED;
    const int64_t end = now_ms() + timeout_ms;
    Region scratch;  // host words of this thread
    scratch.len = 4;
    // 2. gate: the receiver has freed the slot
    if (gate) {
      int spins = 0;
      while (true) {
        uint32_t g = 0;
        int st = transfer_with(c, scratch, (uint64_t)(uintptr_t)&g, gate, 4, false, timeout_ms, nullptr, true);
        if (st != CX_OK) return st;
        if (reached(g, gate_value)) break;
        if (cancelled()) return CX_CANCELLED;
        if (now_ms() > end) return CX_TIMEOUT;
        backoff(spins);
      }
    }
    if (cancelled()) return CX_CANCELLED;
    // 3. payload, then 4. the flag -- the flag lands only after the payload has
    int st = len ? transfer_with(c, lr, src, dst, len, true, std::max<int64_t>(1, end - now_ms()), nullptr) : CX_OK;
    if (st != CX_OK || !flag) return st;
    uint32_t f = flag_value;
    return transfer_with(c, scratch, (uint64_t)(uintptr_t)&f, flag, 4, true, std::max<int64_t>(1, end - now_ms()),
                         nullptr);
  }

  Worker& worker(int64_t queue) {
    std::lock_guard<std::mutex> g(wmu_);
    auto& w = workers_[queue];
    if (!w) w = std::make_unique<Worker>();
    return *w;
  }

  // ---- connections -------------------------------------------------------------------------
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

  // frame-path requests (host memory on both sides; ranges checked by the caller)
  // `dst` 0: the request owns its destination (p->payload), for buffers that
  // may be gone when a late answer arrives (bounce buffers, chain words)
  std::shared_ptr<Pending> start_read(const std::shared_ptr<Conn>& c, uint64_t dst, uint64_t src, uint64_t len) {
    auto p = std::make_shared<Pending>();
    if (!dst) p->payload.resize(len);
    p->dst = dst ? (uint8_t*)(uintptr_t)dst : p->payload.data();
    p->len = len;
    uint64_t id = next_id_++;
    {
      std::lock_guard<std::mutex> g(c->pmu);
      c->pending[id] = p;
    }
    inflight_++;
    uint64_t hdr[3] = {id, src, len};
    if (!c->send_frame(F_READ_REQ, {{hdr, sizeof(hdr)}})) drop(c, "send failed", true);
    return p;
  }
  std::shared_ptr<Pending> start_write(const std::shared_ptr<Conn>& c, uint64_t dst, uint64_t src, uint64_t len,
                                       const char* msg, size_t mlen) {
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
    return p;
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
    if (p->counted) inflight_--;
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
      if (kv.second->counted) inflight_--;
      kv.second->complete(CX_PEER_FAILED);
    }
    // the peer's memory: released once the copies that touched it have passed
    std::map<uint64_t, std::shared_ptr<RemoteRegion>> remote;
    {
      std::lock_guard<std::mutex> g(c->rmu);
      remote.swap(c->remote);
    }
    for (auto& kv : remote) bury(kv.second);
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
        if (inside_host((uintptr_t)hdr[1], hdr[2])) {
          uint64_t rh[2] = {hdr[0], (uint64_t)(int64_t)CX_OK};
          c->send_frame(F_READ_RESP, {{rh, sizeof(rh)}, {(const void*)(uintptr_t)hdr[1], hdr[2]}});
        } else {  // unknown, or device memory: never a host memcpy of a device address
          uint64_t rh[2] = {hdr[0], (uint64_t)(int64_t)CX_INVALID};
          c->send_frame(F_READ_RESP, {{rh, sizeof(rh)}});
        }
      } else if (type == F_WRITE_REQ && body >= 40) {
        uint64_t hdr[5];
        std::memcpy(hdr, buf.data(), sizeof(hdr));
        const uint64_t id = hdr[0], dst = hdr[1], n = hdr[2], has_msg = hdr[3], mlen = hdr[4];
        int st = CX_INVALID;
        if (40 + mlen + n <= body && inside_host((uintptr_t)dst, n)) {
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
      } else if (type == F_REGION_REQ && body >= 24) {
        uint64_t hdr[3];
        std::memcpy(hdr, buf.data(), sizeof(hdr));
        RegionWire w;
        try {
          w = describe(hdr[1], hdr[2]);
        } catch (const std::exception&) {
          w = RegionWire();
          w.status = CX_ERR;
        }
        c->send_frame(F_REGION_RESP, {{&hdr[0], 8}, {&w, sizeof(w)}});
      } else if (type == F_REGION_RESP && body >= 8) {
        uint64_t id;
        std::memcpy(&id, buf.data(), 8);
        std::shared_ptr<Pending> p;
        {
          std::lock_guard<std::mutex> g(c->pmu);
          auto it = c->pending.find(id);
          if (it != c->pending.end()) p = it->second;
        }
        if (p) p->payload.assign(buf.begin() + 8, buf.begin() + body);
        complete(c, id, CX_OK);
      } else if (type == F_REGION_GONE && body >= 8) {
        uint64_t base;
        std::memcpy(&base, buf.data(), 8);
        std::shared_ptr<RemoteRegion> rr;
        {
          std::lock_guard<std::mutex> g(c->rmu);
          auto it = c->remote.find(base);
          if (it != c->remote.end()) {
            rr = it->second;
            c->remote.erase(it);
          }
        }
        if (rr) bury(rr);
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
      graveyard_.reap();  // dead peers' mappings go as soon as their copies passed
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
  int home_device_ = 0;
  std::thread accept_thread_, hb_thread_;
  std::mutex cmu_, dial_mu_;
  std::vector<std::shared_ptr<Conn>> conns_;
  std::map<std::string, std::shared_ptr<Conn>> out_;
  std::mutex mmu_;
  std::map<uintptr_t, Region> regions_;
  std::set<uintptr_t> managed_;
  std::map<uint64_t, VmmAlloc> vmm_;  // by allocation id
  std::atomic<uint64_t> next_alloc_{1};
  std::mutex fmu_;
  std::unique_ptr<FdServer> fds_;
  std::mutex smu_;
  std::map<int, CUstream> streams_;
  std::mutex wmu_;
  std::map<int64_t, std::unique_ptr<Worker>> workers_;
  Graveyard graveyard_;
  std::mutex qmu_;
  std::condition_variable qcv_, ecv_;
  std::deque<std::pair<Identity, std::string>> msgs_;
  std::deque<Event> events_;
  bool closed_ = false;
  std::atomic<uint64_t> next_id_{1};
  std::atomic<int64_t> inflight_{0}, rma_ok_{0}, rma_err_{0}, failures_{0}, eps_created_{0}, eps_closed_{0};
  std::atomic<int64_t> dev_copies_{0}, chains_ok_{0}, chains_err_{0};
};

// ------------------------------------------------------ standalone device buffers
// A VMM allocation that other processes of this machine can map (for tensors
// that are shared without an engine, e.g. a KV cache or an expert buffer), and
// its import on the other side with the graveyard bookkeeping.
class DeviceBuffer {
 public:
  DeviceBuffer(uint64_t size, int device) {
    {
      py::gil_scoped_release nogil;
      a_ = vmm_create(size, device, next_id());
    }
    asked_ = size;
    std::lock_guard<std::mutex> g(reg_mu());
    registry()[a_.id] = this;
  }
  ~DeviceBuffer() { close(); }
  uint64_t ptr() const { return a_.ptr; }
  uint64_t size() const { return asked_; }
  uint64_t alloc_size() const { return a_.size; }
  int device() const { return a_.device; }
  py::dict describe() {
    py::dict d;
    d["kind"] = "vmm";
    d["sock"] = server().name();
    d["id"] = a_.id;
    d["size"] = asked_;
    d["alloc_size"] = (uint64_t)a_.size;
    d["device"] = a_.device;
    d["host"] = boot_id();
    d["pid"] = (int64_t)::getpid();
    return d;
  }
  void close() {
    {
      std::lock_guard<std::mutex> g(reg_mu());
      registry().erase(a_.id);
    }
    py::gil_scoped_release nogil;
    vmm_destroy(a_);
  }

 private:
  static uint64_t next_id() {
    static std::atomic<uint64_t> n{1};
    return n++;
  }
  static std::mutex& reg_mu() {
    static std::mutex m;
    return m;
  }
  static std::map<uint64_t, DeviceBuffer*>& registry() {
    static std::map<uint64_t, DeviceBuffer*> r;
    return r;
  }
  static FdServer& server() {
    static std::mutex m;
    static std::unique_ptr<FdServer> s;
    std::lock_guard<std::mutex> g(m);
    if (!s)
      s = std::make_unique<FdServer>([](uint64_t id) {
        std::lock_guard<std::mutex> l(reg_mu());
        auto it = registry().find(id);
        return it == registry().end() || !it->second->a_.ptr ? -1 : vmm_export_fd(it->second->a_);
      });
    return *s;
  }
  VmmAlloc a_;
  uint64_t asked_ = 0;
};

class Mapping {
 public:
  Mapping(py::dict desc, int device) {
    std::string host = desc["host"].cast<std::string>();
    if (host != boot_id()) throw std::runtime_error("cxengine: the buffer lives on another machine");
    std::string sock = desc["sock"].cast<std::string>();
    uint64_t id = desc["id"].cast<uint64_t>();
    uint64_t alloc = desc["alloc_size"].cast<uint64_t>();
    size_ = desc["size"].cast<uint64_t>();
    std::string why;
    bool ok;
    {
      py::gil_scoped_release nogil;
      int fd = FdServer::fetch(sock, id, 2000);
      ok = fd >= 0 && import_vmm(fd, alloc, device, im_, why);
      if (fd < 0) why = "the owner did not hand out the allocation (gone, or another user)";
    }
    if (!ok) throw std::runtime_error("cxengine: import failed: " + why);
  }
  ~Mapping() { release(); }
  uint64_t ptr() const { return im_.base; }
  uint64_t size() const { return size_; }
  int device() const { return im_.device; }
  // Note that work on `stream` (a CUstream handle) uses the mapping: `passed`
  // turns true only after everything queued there so far has finished.
  void record(uint64_t stream) {
    const Driver& d = driver();
    d.use_device(im_.device);
    if (!im_.last) d.check(d.EventCreate(&im_.last, CU_EVENT_DISABLE_TIMING), "cuEventCreate");
    d.check(d.EventRecord(im_.last, (CUstream)(uintptr_t)stream), "cuEventRecord");
  }
  bool passed() const { return im_.passed(); }
  void release() {
    py::gil_scoped_release nogil;
    release_import(im_);
  }
  bool released() const { return im_.base == 0; }

 private:
  Import im_;
  uint64_t size_ = 0;
};

}  // namespace cxe

PYBIND11_MODULE(_cxengine, m) {
  using namespace cxe;
  m.doc() = "connex-b200 native transfer engine";
  m.attr("OK") = CX_OK;
  m.attr("PEER_FAILED") = CX_PEER_FAILED;
  m.attr("TIMEOUT") = CX_TIMEOUT;
  m.attr("INVALID") = CX_INVALID;
  m.attr("CANCELLED") = CX_CANCELLED;
  m.def("device_plane", [] {
    const Driver& d = driver();
    return py::make_tuple(d.ok, d.ok ? std::string() : d.why);
  });
  m.def("device_memory_info", [](int device) {
    const Driver& d = driver();
    if (!d.ok || !d.use_device(device)) throw std::runtime_error("cxengine: no device plane");
    size_t f = 0, t = 0;
    d.check(d.MemGetInfo(&f, &t), "cuMemGetInfo");
    return py::make_tuple((uint64_t)f, (uint64_t)t);
  });
  m.def("boot_id", &boot_id);
  py::class_<Handle>(m, "Handle").def("wait", &Handle::wait, py::arg("ms") = 5000).def("done", &Handle::done);
  py::class_<DeviceBuffer>(m, "DeviceBuffer")
      .def(py::init<uint64_t, int>(), py::arg("size"), py::arg("device") = 0)
      .def_property_readonly("ptr", &DeviceBuffer::ptr)
      .def_property_readonly("size", &DeviceBuffer::size)
      .def_property_readonly("alloc_size", &DeviceBuffer::alloc_size)
      .def_property_readonly("device", &DeviceBuffer::device)
      .def("describe", &DeviceBuffer::describe)
      .def("close", &DeviceBuffer::close);
  py::class_<Mapping>(m, "Mapping")
      .def(py::init<py::dict, int>(), py::arg("desc"), py::arg("device") = 0)
      .def_property_readonly("ptr", &Mapping::ptr)
      .def_property_readonly("size", &Mapping::size)
      .def_property_readonly("device", &Mapping::device)
      .def_property_readonly("released", &Mapping::released)
      .def("record", &Mapping::record)
      .def("passed", &Mapping::passed)
      .def("release", &Mapping::release);
  py::class_<Engine>(m, "Engine")
      .def(py::init<const std::string&, int64_t, int64_t, int64_t, const std::string&, int, const std::string&, int,
                    int, int>(),
           py::arg("model"), py::arg("stage"), py::arg("shard") = 0, py::arg("replica") = 0,
           py::arg("listen_ip") = "0.0.0.0", py::arg("port") = 0, py::arg("advertise_ip") = "",
           py::arg("heartbeat_ms") = 1000, py::arg("heartbeat_timeout_ms") = 3000, py::arg("spin_us") = 500)
      .def_property_readonly("local_url", &Engine::local_url)
      .def_property_readonly("port", &Engine::port)
      .def_property_readonly("identity", &Engine::identity)
      .def_property_readonly("device", &Engine::device)
      .def("set_device", &Engine::set_device)
      .def("allocate_managed_buffer", &Engine::allocate_managed_buffer)
      .def("free_managed_buffer", &Engine::free_managed_buffer)
      .def("allocate_device_buffer", &Engine::allocate_device_buffer, py::arg("size"), py::arg("device") = 0)
      .def("free_device_buffer", &Engine::free_device_buffer)
      .def("write_bytes_to_buffer", &Engine::write_bytes_to_buffer)
      .def("read_bytes_from_buffer", &Engine::read_bytes_from_buffer)
      .def("register_memory", &Engine::register_memory)
      .def("unregister_memory", &Engine::unregister_memory)
      .def("region_kind", &Engine::region_kind)
      .def("transfer_sync_read", &Engine::transfer_sync_read, py::arg("url"), py::arg("dst"), py::arg("src"),
           py::arg("length"), py::arg("timeout_ms") = 5000)
      .def("transfer_sync_write", &Engine::transfer_sync_write, py::arg("url"), py::arg("local"), py::arg("remote"),
           py::arg("length"), py::arg("timeout_ms") = 5000)
      .def("get_async", &Engine::get_async, py::arg("url"), py::arg("dst"), py::arg("src"), py::arg("length"),
           py::arg("timeout_ms") = 5000)
      .def("put_async", &Engine::put_async, py::arg("url"), py::arg("local"), py::arg("remote"), py::arg("length"),
           py::arg("timeout_ms") = 5000)
      .def("put_signal", &Engine::put_signal)
      .def("put_chain", &Engine::put_chain, py::arg("url"), py::arg("doorbell"), py::arg("doorbell_value"),
           py::arg("gate"), py::arg("gate_value"), py::arg("src"), py::arg("dst"), py::arg("length"), py::arg("flag"),
           py::arg("flag_value"), py::arg("queue") = 0, py::arg("timeout_ms") = 5000, py::arg("cancel") = 0,
           py::arg("arm_timeout_ms") = -1)
      .def("send_msg", &Engine::send_msg)
      .def("recv_msg", &Engine::recv_msg, py::arg("ms") = 1000)
      .def("connect", &Engine::connect)
      .def("wait_event", &Engine::wait_event, py::arg("ms") = 1000)
      .def("reap", &Engine::reap, py::arg("ms") = 0)
      .def("stats", &Engine::stats)
      .def("close", &Engine::close);
}
