// kimi_mla_decode_static_workspace: the decode entry point for callers that
// cannot allocate device memory.
//
// Some callers of this library have no way to obtain scratch memory: a
// foreign-language host (a cgo, JNI or ctypes binding) that holds only the
// raw device pointers an inference engine handed it and has no CUDA
// allocator of its own, or an engine that reserves all free HBM for its KV
// cache at start-up and treats any later cudaMalloc as out-of-memory.  This
// entry point runs the same split-K decode as kimi_mla_decode but takes its
// split-K partials from a fixed array compiled into the library, so the call
// needs nothing from the caller beyond its inputs and outputs.
//
// Cost and limits:
//  * every GPU that loads the library holds KIMI_MLA_STATIC_WORKSPACE_BYTES
//    (32 MiB) for this array until the process exits;
//  * a call whose split-K partials need more than that is rejected with
//    KIMI_ERR_STATIC_WORKSPACE_LIMIT before anything is launched;
//  * all calls on a device share the one array and it keeps the last call's
//    contents.  Calls that overlap on the GPU (different streams without
//    ordering, or different host threads) race on it; callers must order
//    them.  Nothing in it needs clearing between calls: each call writes
//    every log-sum-exp slot and every partial row that its merge reads.
//  * The device address of the array is looked up with cudaGetSymbolAddress
//    on the first call on each device (with that device current), and again
//    on the first call after that device's context changed (a
//    cudaDeviceReset); make those calls before any stream capture begins.
#include <cstddef>
#include <cstdint>
#include <mutex>

#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/kimi_mla.h"

namespace {

constexpr size_t kStaticWorkspaceBytes = KIMI_MLA_STATIC_WORKSPACE_BYTES;
constexpr int kMaxDevices = 64;

// The scratch array.  In host code `g_decode_scratch` names a host-side
// stand-in, not device memory: only the address from cudaGetSymbolAddress
// may be handed to a kernel.
static __device__ __align__(256) unsigned char g_decode_scratch[kStaticWorkspaceBytes];

std::mutex g_mutex;

// The address is valid for the device's primary context that was current
// when it was looked up; a later context on the same device (after
// cudaDeviceReset, say) gets its own lookup.  The current context comes from
// the driver through the runtime (no link against libcuda).
using CtxGetCurrentFn = CUresult (*)(CUcontext*);

CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  }
  return fn;
}

struct Entry {
  CUcontext ctx = nullptr;
  void* ptr = nullptr;
};
Entry g_entry[kMaxDevices];

// Device address of g_decode_scratch on the current device and context.
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return KIMI_ERR_CUDA_BASE + static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices) return KIMI_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_mutex);
  const CtxGetCurrentFn get = ctx_get_current();
  auto current = [get]() {
    CUcontext c = nullptr;
    if (get && get(&c) != CUDA_SUCCESS) c = nullptr;
    return c;
  };
  // (no context is current before the runtime first touches the device:
  // the lookup below creates it, and the context is read again after it)
  CUcontext ctx = current();
  Entry& en = g_entry[dev];
  if (!en.ptr || !ctx || en.ctx != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return KIMI_ERR_CUDA_BASE + static_cast<int>(e);
    en.ptr = p;
    en.ctx = current();
  }
  *out = en.ptr;
  return KIMI_OK;
}

}  // namespace

extern "C" {

int kimi_mla_decode_static_workspace(const KimiMlaDecodeParams* params, void* stream) {
  if (!params) return KIMI_ERR_NULL_POINTER;
  if (params->batch == 0) return kimi_mla_decode(params, nullptr, 0, stream);
  const size_t need = kimi_mla_decode_workspace_size(params->batch, params->num_heads, params->num_kv_splits);
  if (need > kStaticWorkspaceBytes) return KIMI_ERR_STATIC_WORKSPACE_LIMIT;
  void* scratch = nullptr;
  if (need > 0) {
    const int st = scratch_address(&scratch);
    if (st != KIMI_OK) return st;
  }
  return kimi_mla_decode(params, scratch, need > 0 ? kStaticWorkspaceBytes : 0, stream);
}

}  // extern "C"
