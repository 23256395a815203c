// The CUDA driver API of the transfer engine, resolved at run time.
//
// The engine is a plain C++ module that must import on machines without a
// GPU driver (its host-memory plane and control surface run everywhere), so
// it does not link libcuda: the entry points it uses are looked up once in
// libcuda.so.1 by their exported (versioned) names.  Without a driver,
// `driver().ok` is false and every device path answers "no device memory".
#pragma once

#include <cuda.h>
#include <dlfcn.h>

#include <mutex>
#include <stdexcept>
#include <string>
#include <type_traits>

namespace cxe {

struct Driver {
  bool ok = false;
  std::string why;
  decltype(&::cuInit) Init = nullptr;
  decltype(&::cuDeviceGet) DeviceGet = nullptr;
  decltype(&::cuDevicePrimaryCtxRetain) PrimaryCtxRetain = nullptr;
  decltype(&::cuCtxSetCurrent) CtxSetCurrent = nullptr;
  decltype(&::cuPointerGetAttribute) PointerGetAttribute = nullptr;
  decltype(&::cuMemGetAddressRange) MemGetAddressRange = nullptr;
  decltype(&::cuMemGetAllocationGranularity) MemGetAllocationGranularity = nullptr;
  decltype(&::cuMemCreate) MemCreate = nullptr;
  decltype(&::cuMemRelease) MemRelease = nullptr;
  decltype(&::cuMemAddressReserve) MemAddressReserve = nullptr;
  decltype(&::cuMemAddressFree) MemAddressFree = nullptr;
  decltype(&::cuMemMap) MemMap = nullptr;
  decltype(&::cuMemUnmap) MemUnmap = nullptr;
  decltype(&::cuMemSetAccess) MemSetAccess = nullptr;
  decltype(&::cuMemExportToShareableHandle) MemExportToShareableHandle = nullptr;
  decltype(&::cuMemImportFromShareableHandle) MemImportFromShareableHandle = nullptr;
  decltype(&::cuIpcGetMemHandle) IpcGetMemHandle = nullptr;
  decltype(&::cuIpcOpenMemHandle) IpcOpenMemHandle = nullptr;
  decltype(&::cuIpcCloseMemHandle) IpcCloseMemHandle = nullptr;
  decltype(&::cuStreamCreate) StreamCreate = nullptr;
  decltype(&::cuEventCreate) EventCreate = nullptr;
  decltype(&::cuEventRecord) EventRecord = nullptr;
  decltype(&::cuEventQuery) EventQuery = nullptr;
  decltype(&::cuEventDestroy) EventDestroy = nullptr;
  decltype(&::cuMemcpyAsync) MemcpyAsync = nullptr;
  decltype(&::cuMemGetInfo) MemGetInfo = nullptr;
  decltype(&::cuMemsetD8) MemsetD8 = nullptr;
  decltype(&::cuGetErrorString) GetErrorString = nullptr;

  std::string err(CUresult r) const {
    const char* s = nullptr;
    if (GetErrorString) GetErrorString(r, &s);
    return s ? std::string(s) : ("CUDA driver error " + std::to_string((int)r));
  }
  void check(CUresult r, const char* what) const {
    if (r != CUDA_SUCCESS) throw std::runtime_error(std::string("cxengine: ") + what + ": " + err(r));
  }

  // Make the primary context of `device` current on this thread.
  bool use_device(int device) const {
    CUdevice d;
    CUcontext ctx;
    if (DeviceGet(&d, device) != CUDA_SUCCESS || PrimaryCtxRetain(&ctx, d) != CUDA_SUCCESS) return false;
    // one retain per (thread, call) is balanced by the process exit: primary
    // contexts live as long as the process that uses them
    return CtxSetCurrent(ctx) == CUDA_SUCCESS;
  }
};

inline const Driver& driver() {
  static Driver d;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libcuda.so.1", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      d.why = "libcuda.so.1 not found (no GPU driver)";
      return;
    }
    bool all = true;
    auto get = [&](auto& fn, const char* sym) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, sym));
      if (!fn) {
        all = false;
        d.why = std::string("driver entry point missing: ") + sym;
      }
    };
    get(d.Init, "cuInit");
    get(d.DeviceGet, "cuDeviceGet");
    get(d.PrimaryCtxRetain, "cuDevicePrimaryCtxRetain");
    get(d.CtxSetCurrent, "cuCtxSetCurrent");
    get(d.PointerGetAttribute, "cuPointerGetAttribute");
    get(d.MemGetAddressRange, "cuMemGetAddressRange_v2");
    get(d.MemGetAllocationGranularity, "cuMemGetAllocationGranularity");
    get(d.MemCreate, "cuMemCreate");
    get(d.MemRelease, "cuMemRelease");
    get(d.MemAddressReserve, "cuMemAddressReserve");
    get(d.MemAddressFree, "cuMemAddressFree");
    get(d.MemMap, "cuMemMap");
    get(d.MemUnmap, "cuMemUnmap");
    get(d.MemSetAccess, "cuMemSetAccess");
    get(d.MemExportToShareableHandle, "cuMemExportToShareableHandle");
    get(d.MemImportFromShareableHandle, "cuMemImportFromShareableHandle");
    get(d.IpcGetMemHandle, "cuIpcGetMemHandle");
    get(d.IpcOpenMemHandle, "cuIpcOpenMemHandle_v2");
    get(d.IpcCloseMemHandle, "cuIpcCloseMemHandle");
    get(d.StreamCreate, "cuStreamCreate");
    get(d.EventCreate, "cuEventCreate");
    get(d.EventRecord, "cuEventRecord");
    get(d.EventQuery, "cuEventQuery");
    get(d.EventDestroy, "cuEventDestroy_v2");
    get(d.MemcpyAsync, "cuMemcpyAsync");
    get(d.MemGetInfo, "cuMemGetInfo_v2");
    get(d.MemsetD8, "cuMemsetD8_v2");
    get(d.GetErrorString, "cuGetErrorString");
    if (!all) return;
    CUresult r = d.Init(0);
    if (r != CUDA_SUCCESS) {
      d.why = "cuInit failed: " + d.err(r);
      return;
    }
    d.ok = true;
  });
  return d;
}

}  // namespace cxe
