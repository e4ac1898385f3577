// Run-time resolution of the NCCL functions of the multi-GPU build (see nccl_dl.h).
#include "nccl_dl.h"

#include <dlfcn.h>

#include <cstdlib>

#include <mutex>

namespace ungx
{

const NcclApi *nccl_api(std::string &err)
{
   static std::once_flag once;
   static NcclApi api;
   static bool ok = false;
   static std::string load_err;
   std::call_once(once, [] {
      // UNGX_NCCL_LIBRARY names the library to use; otherwise the copy already in the
      // process (a framework's), else libnccl.so.2 from the loader's search path
      const char *path = std::getenv("UNGX_NCCL_LIBRARY");
      void *h = nullptr;
      if (path && *path)
         h = dlopen(path, RTLD_NOW | RTLD_GLOBAL);
      else
      {
         h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
         if (!h)
            h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
         if (!h)
            h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
      }
      if (!h)
      {
         const char *e = dlerror();
         load_err = std::string("NCCL is not loadable (") + (path && *path ? path : "libnccl.so.2") +
                    "): " + (e ? e : "unknown error");
         return;
      }
      bool all = true;
      auto get = [&](auto &fn, const char *name) {
         fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
         if (!fn)
         {
            all = false;
            load_err = std::string("NCCL lacks ") + name;
         }
      };
      get(api.GetUniqueId, "ncclGetUniqueId");
      get(api.CommInitRank, "ncclCommInitRank");
      get(api.CommDestroy, "ncclCommDestroy");
      get(api.CommAbort, "ncclCommAbort");
      get(api.CommGetAsyncError, "ncclCommGetAsyncError");
      get(api.AllGather, "ncclAllGather");
      get(api.AllReduce, "ncclAllReduce");
      get(api.Send, "ncclSend");
      get(api.Recv, "ncclRecv");
      get(api.GroupStart, "ncclGroupStart");
      get(api.GroupEnd, "ncclGroupEnd");
      get(api.GetErrorString, "ncclGetErrorString");
      get(api.GetVersion, "ncclGetVersion");
      ok = all;
   });
   if (!ok)
   {
      err = load_err;
      return nullptr;
   }
   return &api;
}

} // namespace ungx
