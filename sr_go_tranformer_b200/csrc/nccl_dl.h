// nccl_dl.h -- the handful of NCCL entry points the tensor-parallel step uses,
// bound at run time with dlopen("libnccl.so.2").  Binding at run time means the
// process keeps a single NCCL: the copy PyTorch (or any other host) already
// loaded, else the system library.  Declarations follow nccl.h's C API.
#pragma once

#include <cuda_runtime.h>
#include <dlfcn.h>

#include <mutex>
#include <string>

namespace sr {
namespace nccl {

typedef struct ncclComm* Comm;
typedef struct {
  char internal[128];
} UniqueId;
enum Result { kSuccess = 0 };
enum DataType { kFloat32 = 7 };
enum RedOp { kSum = 0 };

struct Api {
  int (*GetUniqueId)(UniqueId*) = nullptr;
  int (*CommInitRank)(Comm*, int, UniqueId, int) = nullptr;
  int (*AllReduce)(const void*, void*, size_t, int, int, Comm, cudaStream_t) = nullptr;
  int (*CommDestroy)(Comm) = nullptr;
  int (*CommAbort)(Comm) = nullptr;
  const char* (*GetErrorString)(int) = nullptr;
  bool ok = false;
  std::string error;
};

inline Api& api() {
  static Api a;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      a.error = std::string("cannot load libnccl.so.2: ") + dlerror();
      return;
    }
    a.GetUniqueId = (int (*)(UniqueId*))dlsym(h, "ncclGetUniqueId");
    a.CommInitRank = (int (*)(Comm*, int, UniqueId, int))dlsym(h, "ncclCommInitRank");
    a.AllReduce = (int (*)(const void*, void*, size_t, int, int, Comm, cudaStream_t))dlsym(h, "ncclAllReduce");
    a.CommDestroy = (int (*)(Comm))dlsym(h, "ncclCommDestroy");
    a.CommAbort = (int (*)(Comm))dlsym(h, "ncclCommAbort");
    a.GetErrorString = (const char* (*)(int))dlsym(h, "ncclGetErrorString");
    a.ok = a.GetUniqueId && a.CommInitRank && a.AllReduce && a.CommDestroy && a.CommAbort && a.GetErrorString;
    if (!a.ok) a.error = "libnccl.so.2 lacks an expected symbol";
  });
  return a;
}

}  // namespace nccl
}  // namespace sr
