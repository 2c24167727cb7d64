// NCCL entry points resolved at run time: dlopen of libnccl.so.2 (in a
// process that has already loaded NCCL, e.g. through torch, that copy), so
// the library links without NCCL and runs without it until an expert-
// parallel group is asked for. Only the calls the expert-parallel block
// makes: the communicator, and grouped point-to-point send/recv.
#pragma once
#include <dlfcn.h>
#include <nccl.h>

#include <cstdio>
#include <type_traits>

namespace ms {

struct NcclRt {
  bool ok = false;
  char why[256] = "";
  decltype(&ncclGetUniqueId) GetUniqueId = nullptr;
  decltype(&ncclCommInitRank) CommInitRank = nullptr;
  decltype(&ncclCommDestroy) CommDestroy = nullptr;
  decltype(&ncclCommAbort) CommAbort = nullptr;
  decltype(&ncclGroupStart) GroupStart = nullptr;
  decltype(&ncclGroupEnd) GroupEnd = nullptr;
  decltype(&ncclSend) Send = nullptr;
  decltype(&ncclRecv) Recv = nullptr;
  decltype(&ncclGetErrorString) GetErrorString = nullptr;
};

// Loaded once per process; ok is false (why says so) when no NCCL is found.
inline const NcclRt& nccl_rt() {
  static const NcclRt rt = [] {
    NcclRt r;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char* e = dlerror();
      snprintf(r.why, sizeof(r.why), "libnccl.so.2 not found: %s", e ? e : "?");
      return r;
    }
    bool all = true;
    auto get = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      if (!fn) {
        all = false;
        snprintf(r.why, sizeof(r.why), "libnccl.so.2 lacks %s", name);
      }
    };
    get(r.GetUniqueId, "ncclGetUniqueId");
    get(r.CommInitRank, "ncclCommInitRank");
    get(r.CommDestroy, "ncclCommDestroy");
    get(r.CommAbort, "ncclCommAbort");
    get(r.GroupStart, "ncclGroupStart");
    get(r.GroupEnd, "ncclGroupEnd");
    get(r.Send, "ncclSend");
    get(r.Recv, "ncclRecv");
    get(r.GetErrorString, "ncclGetErrorString");
    r.ok = all;
    return r;
  }();
  return rt;
}

}  // namespace ms
