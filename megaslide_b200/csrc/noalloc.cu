// msl_dsa_attn_bwd_noalloc: the backward of the deformable gather attention for callers that
// cannot allocate device memory.  Its scratch (float32 dK/dV accumulators and the extra-key
// coefficients) is one static device array; the entry point hands that array to
// msl_dsa_attn_bwd as the workspace, so the computation is exactly the workspace entry point's.

#include <cstdio>
#include <mutex>

#include <cuda_runtime.h>

#include "megaslide_b200.h"

namespace msl {
int record_error(int code, const char* msg);
}

// Host code may not use this name as an address: it is a host-side stand-in for the device
// array.  The device address comes from cudaGetSymbolAddress, once per device.
static __device__ __align__(256) unsigned char g_bwd_scratch[MSL_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};
}  // namespace

extern "C" int msl_dsa_attn_bwd_noalloc(const msl_dsa_geometry* geom, const msl_dsa_bwd_io* io, void* stream) {
  if (!geom || !io) return msl::record_error(MSL_ERR_INVALID, "geometry and io are required");
  const size_t need = msl_dsa_attn_bwd_workspace_bytes(geom, io->dk_acc != nullptr ? 1 : 0);
  if (need > MSL_NOALLOC_SCRATCH_BYTES) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "msl_dsa_attn_bwd_noalloc: this problem needs %zu bytes of scratch, the static array holds %u "
             "(use msl_dsa_attn_bwd with a workspace)", need, MSL_NOALLOC_SCRATCH_BYTES);
    return msl::record_error(MSL_ERR_WORKSPACE, msg);
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return msl::record_error(MSL_ERR_CUDA, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return msl::record_error(MSL_ERR_UNSUPPORTED, "device index beyond 63");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_scratch_addr[dev] == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_bwd_scratch);  // the current device is `dev`
      if (e != cudaSuccess || p == nullptr) {
        char msg[256];
        snprintf(msg, sizeof(msg), "cudaGetSymbolAddress of the no-alloc scratch failed: %s", cudaGetErrorString(e));
        return msl::record_error(MSL_ERR_CUDA, msg);
      }
      g_scratch_addr[dev] = p;
    }
    scratch = g_scratch_addr[dev];
  }
  return msl_dsa_attn_bwd(geom, io, scratch, MSL_NOALLOC_SCRATCH_BYTES, stream);
}
