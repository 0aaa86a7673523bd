// Allocation-free entry point: the split (stream-K) attention schedule with its
// scratch memory in a fixed array compiled into this library.
//
// Some callers cannot allocate device memory, not even through a caching
// allocator: a plugin inside an inference runtime that owns all device memory
// and hands the plugin only tensors and a stream; an application that reserves
// a fixed memory budget at start-up and forbids allocation afterwards; code on
// a latency-critical path, where cudaMalloc/cudaFree take a driver-wide lock
// and cudaFree synchronises the device. gfx906_b200_attn_launch_noalloc lets
// them use the split schedule (which balances the key range of every query
// block across all SMs and combines partial results on the GPU) without
// providing a workspace. It calls no cudaMalloc, cudaFree or allocating
// library routine.
//
// The scratch is the file-scope array below. Every GPU on which this file's
// code is first used holds it (kNoallocWorkspaceBytes) until the process
// exits; with CUDA's default lazy module loading that happens on the first
// call of gfx906_b200_attn_launch_noalloc on that device, not when the library
// is loaded. Every call on a device shares the one array, which keeps the last
// call's contents: the kernel's arrival counters carry a per-launch tag, so no
// part of the array has to start at zero and nothing is cleared between calls.
// Calls that overlap on the GPU (different streams, or different host threads
// without ordering) race on the array and give wrong results: order them on
// one stream.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/gfx906_b200_attn.h"

namespace {

// Largest split plan on a B200 (148 SMs, head dim 128): ~40 MB.
constexpr size_t kNoallocWorkspaceBytes = 48ull << 20;

// In host code this name is a host-side stand-in for the device array, not a
// device address; the address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_workspace[kNoallocWorkspaceBytes];

constexpr int kMaxDevices = 64;
void* g_noalloc_ptr[kMaxDevices] = {};
std::mutex g_noalloc_mu;

// Device address of the array on the current device, looked up once per device
// (the first call on a device does this set-up; it should come before any
// stream capture on that device).
int noalloc_workspace(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GFX906_B200_ECUDA;
  if (dev < 0 || dev >= kMaxDevices) return GFX906_B200_ENODEV;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_workspace) != cudaSuccess || !p) {
      // Consume the runtime's pending error, so that the next, unrelated
      // launch's error check does not report it as its own.
      (void)cudaGetLastError();
      return GFX906_B200_ECUDA;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return GFX906_B200_OK;
}

}  // namespace

// Records the status for gfx906_b200_attn_last_error() (attn_fwd_sm100.cu).
extern "C" int gfx906_b200_internal_set_last_error(int status);

extern "C" {

size_t gfx906_b200_attn_noalloc_capacity(void) { return kNoallocWorkspaceBytes; }

int gfx906_b200_attn_launch_noalloc(const void* q, const void* k, const void* v, void* o, int B, int H, int Sq,
                                    int Skv, int D, float scale, cudaStream_t stream) {
  // 0 when this call does not split (or its arguments are invalid): the
  // workspace entry then runs without scratch and reports any error itself.
  const size_t need = gfx906_b200_attn_workspace_size(B, H, Sq, Skv, D);
  if (need == 0) return gfx906_b200_attn_launch_ws(q, k, v, o, B, H, Sq, Skv, D, scale, nullptr, 0, stream);
  // The scratch a split schedule needs grows with the SM count (about 40 MB
  // on a 148-SM B200); a device with more SMs can exceed the array.
  if (need > kNoallocWorkspaceBytes) return gfx906_b200_internal_set_last_error(GFX906_B200_ENOSPACE);
  void* ws = nullptr;
  const int rc = noalloc_workspace(&ws);
  if (rc != GFX906_B200_OK) return gfx906_b200_internal_set_last_error(rc);
  return gfx906_b200_attn_launch_ws(q, k, v, o, B, H, Sq, Skv, D, scale, ws, kNoallocWorkspaceBytes, stream);
}

}  // extern "C"
