// Device memory of the transfer engine: exportable allocations, their import
// by another process of the same machine, the file-descriptor server that
// hands exported allocations out, and the graveyard that releases a peer's
// mappings only once the copies that touched them have finished.
//
// Export kinds
//   VMM  -- physical memory from cuMemCreate with a POSIX-fd handle type,
//           mapped by the owner; a peer receives a duplicate of the fd over a
//           Unix socket (SCM_RIGHTS, same user only), imports and maps it.
//           When the owner dies, the memory stays alive exactly as long as
//           some importer still maps it -- and the importer's graveyard
//           releases its mapping as soon as its last copy passed, so the
//           physical memory is freed deterministically.
//   IPC  -- any other device allocation (the caching allocator's cudaMalloc
//           blocks) through the allocation's legacy IPC handle.
//
// Peer copies run on the copy engines (cuMemcpyAsync between a local buffer
// and the mapped peer range) on one stream per local device; every wait is
// bounded by polling an event against a deadline.
#pragma once

#include <fcntl.h>
#include <poll.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <atomic>
#include <cstddef>
#include <cstdlib>
#include <type_traits>
#include <chrono>
#include <cstring>
#include <fstream>
#include <functional>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "cudrv.h"

namespace cxe {

enum RegionKind : uint32_t {
  RK_HOST = 1,          // host memory: served over the socket
  RK_VMM = 2,           // engine-allocated device memory, exported as an fd
  RK_IPC = 3,           // registered device memory, exported as a legacy IPC handle
  RK_DEVICE_LOCAL = 4,  // device memory that cannot be exported (local side of copies only)
};

inline const char* kind_name(uint32_t k) {
  switch (k) {
    case RK_HOST: return "host";
    case RK_VMM: return "vmm";
    case RK_IPC: return "ipc";
    default: return "device";
  }
}

// What a peer needs to reach a region (the body of a region answer).
struct RegionWire {
  int64_t status = 0;
  uint32_t kind = 0;
  int32_t device = -1;
  uint64_t base = 0;          // the region's first address in the owner's space
  uint64_t size = 0;
  uint64_t alloc_offset = 0;  // base minus the start of the exported allocation
  uint64_t alloc_size = 0;    // size of the exported allocation
  uint64_t export_id = 0;     // VMM: the allocation id to ask the fd server for
  uint8_t ipc[CU_IPC_HANDLE_SIZE] = {};
  char host[40] = {};         // boot id of the owner's machine
  char sock[64] = {};         // VMM: abstract socket name of the owner's fd server
};

// The machine's identity (its boot id).  CONNEX_ENGINE_HOST_ID overrides it:
// processes with different ids treat each other as separate machines.
inline std::string boot_id() {
  static std::string id = [] {
    if (const char* e = std::getenv("CONNEX_ENGINE_HOST_ID")) return std::string(e);
    std::ifstream f("/proc/sys/kernel/random/boot_id");
    std::string s;
    std::getline(f, s);
    return s.empty() ? std::string("unknown-host") : s;
  }();
  return id;
}

// Wait for `ev` with a deadline; 0 = passed, CX-style -3 on timeout, -1 on error.
inline int wait_for_event(CUevent ev, int64_t timeout_ms) {
  const Driver& d = driver();
  auto end = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
  int spins = 0;
  while (true) {
    CUresult r = d.EventQuery(ev);
    if (r == CUDA_SUCCESS) return 0;
    if (r != CUDA_ERROR_NOT_READY) return -1;
    if (std::chrono::steady_clock::now() >= end) return -3;
    if (++spins > 200) std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// ---------------------------------------------------------------- allocations
struct VmmAlloc {
  CUmemGenericAllocationHandle h = 0;
  CUdeviceptr ptr = 0;
  size_t size = 0;  // rounded up to the allocation granularity
  int device = 0;
  uint64_t id = 0;
};

inline CUmemAllocationProp vmm_prop(int device) {
  CUmemAllocationProp p{};
  p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  p.location.id = device;
  p.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return p;
}

inline void grant(CUdeviceptr ptr, size_t size, int device) {
  const Driver& d = driver();
  CUmemAccessDesc a{};
  a.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  a.location.id = device;
  a.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  d.check(d.MemSetAccess(ptr, size, &a, 1), "cuMemSetAccess");
}

inline VmmAlloc vmm_create(size_t bytes, int device, uint64_t id) {
  const Driver& d = driver();
  if (!d.ok) throw std::runtime_error("cxengine: no device memory: " + d.why);
  if (!d.use_device(device)) throw std::runtime_error("cxengine: cannot use device " + std::to_string(device));
  CUmemAllocationProp p = vmm_prop(device);
  size_t gran = 0;
  d.check(d.MemGetAllocationGranularity(&gran, &p, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED), "granularity");
  VmmAlloc a;
  a.size = ((bytes ? bytes : 1) + gran - 1) / gran * gran;
  a.device = device;
  a.id = id;
  d.check(d.MemCreate(&a.h, a.size, &p, 0), "cuMemCreate");
  CUresult r = d.MemAddressReserve(&a.ptr, a.size, gran, 0, 0);
  if (r == CUDA_SUCCESS) r = d.MemMap(a.ptr, a.size, 0, a.h, 0);
  if (r != CUDA_SUCCESS) {
    if (a.ptr) d.MemAddressFree(a.ptr, a.size);
    d.MemRelease(a.h);
    d.check(r, "map a new allocation");
  }
  grant(a.ptr, a.size, device);
  d.check(d.MemsetD8(a.ptr, 0, a.size), "zero a new allocation");
  return a;
}

inline void vmm_destroy(VmmAlloc& a) {
  const Driver& d = driver();
  if (!a.ptr) return;
  d.use_device(a.device);
  d.MemUnmap(a.ptr, a.size);
  d.MemAddressFree(a.ptr, a.size);
  d.MemRelease(a.h);  // the physical memory goes once no importer maps it either
  a.ptr = 0;
}

inline int vmm_export_fd(const VmmAlloc& a) {
  const Driver& d = driver();
  int fd = -1;
  if (d.MemExportToShareableHandle(&fd, a.h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0) != CUDA_SUCCESS) return -1;
  return fd;
}

// ------------------------------------------------------------------ fd server
// Hands out duplicates of exported allocations' fds to processes of the same
// user that connect to an abstract Unix socket and send the allocation id.
class FdServer {
 public:
  explicit FdServer(std::function<int(uint64_t)> export_fd) : export_fd_(std::move(export_fd)) {
    static std::atomic<int> seq{0};
    name_ = "cxe-fd-" + std::to_string(::getpid()) + "-" + std::to_string(seq++);
    lfd_ = ::socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (lfd_ < 0) throw std::runtime_error("cxengine: fd server socket");
    sockaddr_un a = addr(name_);
    if (::bind(lfd_, (sockaddr*)&a, addr_len(name_)) != 0 || ::listen(lfd_, 64) != 0) {
      ::close(lfd_);
      throw std::runtime_error("cxengine: fd server bind");
    }
    th_ = std::thread([this] { loop(); });
  }
  ~FdServer() {
    stop_ = true;
    ::shutdown(lfd_, SHUT_RDWR);
    if (th_.joinable()) th_.join();
    ::close(lfd_);
  }
  const std::string& name() const { return name_; }

  static sockaddr_un addr(const std::string& name) {
    sockaddr_un a{};
    a.sun_family = AF_UNIX;
    a.sun_path[0] = '\0';  // abstract namespace: no file, gone with the process
    std::memcpy(a.sun_path + 1, name.data(), std::min(name.size(), sizeof(a.sun_path) - 2));
    return a;
  }
  static socklen_t addr_len(const std::string& name) {
    return (socklen_t)(offsetof(sockaddr_un, sun_path) + 1 + std::min(name.size(), sizeof(sockaddr_un::sun_path) - 2));
  }

  // Client side: the fd of allocation `id` from the server `name` (-1 on failure).
  static int fetch(const std::string& name, uint64_t id, int timeout_ms) {
    int s = ::socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (s < 0) return -1;
    sockaddr_un a = addr(name);
    if (::connect(s, (sockaddr*)&a, addr_len(name)) != 0 || ::send(s, &id, 8, MSG_NOSIGNAL) != 8) {
      ::close(s);
      return -1;
    }
    pollfd pf{s, POLLIN, 0};
    if (::poll(&pf, 1, timeout_ms) <= 0) {
      ::close(s);
      return -1;
    }
    char ok = 0;
    char ctl[CMSG_SPACE(sizeof(int))] = {};
    iovec io{&ok, 1};
    msghdr m{};
    m.msg_iov = &io;
    m.msg_iovlen = 1;
    m.msg_control = ctl;
    m.msg_controllen = sizeof(ctl);
    int fd = -1;
    if (::recvmsg(s, &m, MSG_CMSG_CLOEXEC) == 1 && ok == 1) {
      cmsghdr* c = CMSG_FIRSTHDR(&m);
      if (c && c->cmsg_level == SOL_SOCKET && c->cmsg_type == SCM_RIGHTS) std::memcpy(&fd, CMSG_DATA(c), sizeof(int));
    }
    ::close(s);
    return fd;
  }

 private:
  void loop() {
    while (!stop_) {
      pollfd pf{lfd_, POLLIN, 0};
      int r = ::poll(&pf, 1, 100);
      if (r <= 0) continue;
      int c = ::accept4(lfd_, nullptr, nullptr, SOCK_CLOEXEC);
      if (c < 0) continue;
      serve(c);
      ::close(c);
    }
  }
  void serve(int c) {
    ucred cred{};
    socklen_t cl = sizeof(cred);
    if (::getsockopt(c, SOL_SOCKET, SO_PEERCRED, &cred, &cl) != 0 || cred.uid != ::getuid()) return;
    pollfd pf{c, POLLIN, 0};
    uint64_t id = 0;
    if (::poll(&pf, 1, 1000) <= 0 || ::recv(c, &id, 8, MSG_WAITALL) != 8) return;
    int fd = export_fd_(id);
    char ok = fd >= 0 ? 1 : 0;
    char ctl[CMSG_SPACE(sizeof(int))] = {};
    iovec io{&ok, 1};
    msghdr m{};
    m.msg_iov = &io;
    m.msg_iovlen = 1;
    if (fd >= 0) {
      m.msg_control = ctl;
      m.msg_controllen = sizeof(ctl);
      cmsghdr* h = CMSG_FIRSTHDR(&m);
      h->cmsg_level = SOL_SOCKET;
      h->cmsg_type = SCM_RIGHTS;
      h->cmsg_len = CMSG_LEN(sizeof(int));
      std::memcpy(CMSG_DATA(h), &fd, sizeof(int));
    }
    ::sendmsg(c, &m, MSG_NOSIGNAL);
    if (fd >= 0) ::close(fd);  // the receiver holds its own duplicate now
  }

  std::function<int(uint64_t)> export_fd_;
  std::string name_;
  int lfd_ = -1;
  std::atomic<bool> stop_{false};
  std::thread th_;
};

// -------------------------------------------------------------------- imports
// A peer allocation mapped into this process, accessible from `device`.
struct Import {
  uint32_t kind = 0;
  int device = 0;
  CUdeviceptr base = 0;  // local address of the allocation's first byte
  size_t size = 0;
  CUmemGenericAllocationHandle h = 0;  // VMM
  CUevent last = nullptr;              // recorded after every copy that touched the mapping
  std::string owner;                   // who exported it (for the stats / logs)

  bool passed() const {
    if (!last) return true;
    CUresult r = driver().EventQuery(last);
    return r != CUDA_ERROR_NOT_READY;  // an error means the context is gone: nothing is in flight either
  }
};

inline bool import_vmm(int fd, size_t size, int device, Import& out, std::string& why) {
  const Driver& d = driver();
  if (!d.use_device(device)) {
    why = "cannot use device " + std::to_string(device);
    return false;
  }
  CUmemGenericAllocationHandle h = 0;
  CUresult r = d.MemImportFromShareableHandle(&h, (void*)(uintptr_t)fd, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
  ::close(fd);  // the handle keeps the memory; the fd is no longer needed
  if (r != CUDA_SUCCESS) {
    why = "import: " + d.err(r);
    return false;
  }
  CUdeviceptr va = 0;
  r = d.MemAddressReserve(&va, size, 0, 0, 0);
  if (r == CUDA_SUCCESS) r = d.MemMap(va, size, 0, h, 0);
  if (r == CUDA_SUCCESS) {
    try {
      grant(va, size, device);
    } catch (const std::exception& e) {
      r = CUDA_ERROR_INVALID_VALUE;
      why = e.what();
    }
  }
  if (r != CUDA_SUCCESS) {
    if (va) {
      d.MemUnmap(va, size);
      d.MemAddressFree(va, size);
    }
    d.MemRelease(h);
    if (why.empty()) why = "map: " + d.err(r);
    return false;
  }
  out.kind = RK_VMM;
  out.device = device;
  out.base = va;
  out.size = size;
  out.h = h;
  return true;
}

inline bool import_ipc(const uint8_t* handle, size_t size, int device, Import& out, std::string& why) {
  const Driver& d = driver();
  if (!d.use_device(device)) {
    why = "cannot use device " + std::to_string(device);
    return false;
  }
  CUipcMemHandle h;
  std::memcpy(h.reserved, handle, CU_IPC_HANDLE_SIZE);
  CUdeviceptr p = 0;
  CUresult r = d.IpcOpenMemHandle(&p, h, CU_IPC_MEM_LAZY_ENABLE_PEER_ACCESS);
  if (r != CUDA_SUCCESS) {
    why = "open IPC handle: " + d.err(r);
    return false;
  }
  out.kind = RK_IPC;
  out.device = device;
  out.base = p;
  out.size = size;
  return true;
}

inline void release_import(Import& im) {
  const Driver& d = driver();
  if (!im.base) return;
  d.use_device(im.device);
  if (im.kind == RK_VMM) {
    d.MemUnmap(im.base, im.size);
    d.MemAddressFree(im.base, im.size);
    d.MemRelease(im.h);
  } else {
    d.IpcCloseMemHandle(im.base);
  }
  if (im.last) d.EventDestroy(im.last);
  im.last = nullptr;
  im.base = 0;
}

// ------------------------------------------------------------------ graveyard
// Mappings that must not be released yet.  `passed` says whether every copy
// that touched a mapping has finished; `reap` releases those and keeps the
// rest, so a stream still reading a dead peer's memory never sees it unmapped.
class Graveyard {
 public:
  struct Grave {
    std::function<bool()> passed;
    std::function<void()> release;
    uint64_t bytes = 0;
  };
  void bury(Grave g) {
    std::lock_guard<std::mutex> l(mu_);
    graves_.push_back(std::move(g));
    buried_++;
  }
  // Release what may be released now; returns how many are left.
  size_t reap() {
    std::vector<Grave> ready;
    {
      std::lock_guard<std::mutex> l(mu_);
      std::vector<Grave> keep;
      for (auto& g : graves_) (g.passed() ? ready : keep).push_back(std::move(g));
      graves_.swap(keep);
    }
    for (auto& g : ready) {
      g.release();
      released_++;
      released_bytes_ += g.bytes;
    }
    std::lock_guard<std::mutex> l(mu_);
    return graves_.size();
  }
  // Reap until nothing is left or `timeout_ms` passed; returns how many are left.
  size_t drain(int64_t timeout_ms) {
    auto end = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
    size_t left = reap();
    while (left && std::chrono::steady_clock::now() < end) {
      std::this_thread::sleep_for(std::chrono::microseconds(200));
      left = reap();
    }
    return left;
  }
  size_t pending() {
    std::lock_guard<std::mutex> l(mu_);
    return graves_.size();
  }
  uint64_t buried() const { return buried_; }
  uint64_t released() const { return released_; }
  uint64_t released_bytes() const { return released_bytes_; }

 private:
  std::mutex mu_;
  std::vector<Grave> graves_;
  std::atomic<uint64_t> buried_{0}, released_{0}, released_bytes_{0};
};

}  // namespace cxe
