// Chunked GLA forward for callers that cannot allocate device memory.
//
// Some hosts cannot hand this library a workspace: a framework that plans all
// device memory ahead of time and passes an operator only its inputs and outputs
// (a custom-call plugin with no scratch argument), or a serving loop that must
// never call cudaMalloc because the allocator can synchronize the device.  For
// them tops_gla_chunk_fwd_noalloc runs the same forward as tops_gla_chunk_fwd with
// its scratch (per-chunk states, chunk-local gate sums, intra-chunk matrix) placed
// in a fixed-size array that is part of this library's device image.
//
// Properties of the array:
//  * TOPS_GLA_NOALLOC_SCRATCH_BYTES (16 MiB) per GPU, placed when the library's
//    device image is loaded on that GPU and held until the process exits.  CUDA
//    loads device images lazily (the default since CUDA 12.2), so that happens at
//    the first use of any of the library's kernels there -- possibly this entry
//    point's first call, which then reserves the 16 MiB itself.  A host that must
//    not allocate after start-up makes one warm-up call per device at start-up,
//    before any stream capture;
//  * one array per device, shared by every call on that device: two calls whose
//    kernels overlap on the GPU (different streams, no ordering) race on it;
//  * it keeps the previous call's contents; the forward writes every scratch
//    element it reads (the only buffer that must start at zero, the gate sums when
//    g is NULL, is cleared in-stream by the forward itself).
#include "common.cuh"

namespace tops {
namespace noalloc {

static __device__ __align__(256) unsigned char g_scratch[TOPS_GLA_NOALLOC_SCRATCH_BYTES];

// Device address of the current device's scratch array, looked up on every call with
// that device current.  The first call on a device loads this library's device image
// there (CUDA loads modules lazily), which places the array; later calls are a host-side
// symbol lookup.  Not cached: a cudaDeviceReset or a different context current on the
// same device places the array at another address, and a cached address would then point
// at freed or foreign memory.  In host code `g_scratch` is only a host-side stand-in for
// the symbol, never a usable address.
static int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "chunk_fwd_noalloc: cudaGetDevice");
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_scratch);
  if (e != cudaSuccess) return cuda_status(e, "chunk_fwd_noalloc: cudaGetSymbolAddress");
  if (p == nullptr) return fail(TOPS_ERR_CUDA, "chunk_fwd_noalloc: scratch symbol has no device address");
  *out = p;
  return TOPS_OK;
}

}  // namespace noalloc
}  // namespace tops

extern "C" int tops_gla_chunk_fwd_noalloc(const tops_gla_chunk_fwd_args* a, void* stream) {
  using namespace tops;
  if (a == nullptr) return fail(TOPS_ERR_INVALID, "chunk_fwd_noalloc: args is NULL");
  const size_t need = tops_gla_chunk_fwd_workspace_size(a);
  if (need == 0 && check_shape(&a->s) != TOPS_OK) return TOPS_ERR_INVALID;
  if (need > (size_t)TOPS_GLA_NOALLOC_SCRATCH_BYTES)
    return fail(TOPS_ERR_WORKSPACE, "chunk_fwd_noalloc: the problem needs " + std::to_string(need) +
                                        " bytes of scratch, more than the fixed " +
                                        std::to_string((size_t)TOPS_GLA_NOALLOC_SCRATCH_BYTES) +
                                        "-byte array; use tops_gla_chunk_fwd with a caller workspace");
  void* scratch = nullptr;
  int rc = noalloc::scratch_address(&scratch);
  if (rc != TOPS_OK) return rc;
  tops_gla_chunk_fwd_args b = *a;
  b.workspace = scratch;
  b.workspace_bytes = (size_t)TOPS_GLA_NOALLOC_SCRATCH_BYTES;
  return tops_gla_chunk_fwd(&b, stream);
}
