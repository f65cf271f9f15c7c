// Sequence-parallel state exchange over NCCL.  Each rank holds one
// contiguous span of a long sequence.  The chunked scan is linear in its initial state
// (tops/ops/common/chunk_h.py:372-386): a span's final state is D * H_in + S, with S its
// final state from a zero state and D = exp(sum of its gates) (diagonal in K).
//  * forward: all ranks all-gather (S_r, D_r); rank r's incoming state is the prefix
//    H_0 = h0 (or 0), H_{r+1} = D_r H_r + S_r, and the whole sequence's final state is H_R;
//  * backward: all ranks all-gather (L_r, D_r), L_r = the gradient w.r.t. rank r's incoming
//    state from its own loss; rank r's final-state gradient is the suffix
//    G_{R-1} = dht (or 0), G_{r-1} = D_r G_r + L_r.
// One ncclAllGather of a packed (state | decay) buffer, then one elementwise kernel.  NCCL is
// loaded at run time (dlopen of libnccl.so.2; the torch process has it loaded already) so
// the library has no link-time NCCL dependency and loads on hosts without it.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

#include "common.cuh"
#include "p2p.cuh"
#include "ptx.cuh"

namespace tops {
namespace exchange {

struct Nccl {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  bool ok = false;
};

static const Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW);
    if (!h) return;
    n.get_unique_id = reinterpret_cast<decltype(n.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    n.comm_init_rank = reinterpret_cast<decltype(n.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    n.all_gather = reinterpret_cast<decltype(n.all_gather)>(dlsym(h, "ncclAllGather"));
    n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(h, "ncclGetErrorString"));
    n.comm_abort = reinterpret_cast<decltype(n.comm_abort)>(dlsym(h, "ncclCommAbort"));
    n.async_error = reinterpret_cast<decltype(n.async_error)>(dlsym(h, "ncclCommGetAsyncError"));
    n.ok = n.get_unique_id && n.comm_init_rank && n.comm_destroy && n.all_gather && n.error_string &&
           n.comm_abort && n.async_error;
  });
  return n;
}

static int nccl_status(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return TOPS_OK;
  return fail(TOPS_ERR_NCCL, std::string(what) + ": " + nccl().error_string(r));
}

// packed per rank: [state N*H*K*V | decay N*H*K], fp32
__global__ void k_pack(size_t ns, size_t nd, const float* __restrict__ s, const float* __restrict__ d,
                       float* __restrict__ out) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < ns + nd; i += (size_t)gridDim.x * blockDim.x)
    out[i] = i < ns ? s[i] : d[i - ns];
}

// forward: out = H_rank, total = H_R; backward: out = G_rank (suffix), total unused.
// `gathered` holds every rank's packed (state | decay), rank after rank.
__device__ __forceinline__ void combine_elems(int world, int rank, int backward, size_t ns, int V,
                                              const float* __restrict__ gathered, const float* __restrict__ boundary,
                                              float* __restrict__ out, float* __restrict__ total) {
  const size_t per = ns + ns / V;  // floats per rank
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < ns; i += (size_t)gridDim.x * blockDim.x) {
    const size_t row = i / V;  // (n*H + h)*K + k
    float x = boundary ? boundary[i] : 0.f;
    if (!backward) {
      for (int r = 0; r < world; ++r) {
        if (r == rank) out[i] = x;
        const float* g = gathered + (size_t)r * per;
        x = fmaf(g[ns + row], x, g[i]);
      }
      if (total) total[i] = x;
    } else {
      for (int r = world - 1; r > rank; --r) {
        const float* g = gathered + (size_t)r * per;
        x = fmaf(g[ns + row], x, g[i]);
      }
      out[i] = x;
    }
  }
}

__global__ void k_combine(int world, int rank, int backward, size_t ns, int V, const float* __restrict__ gathered,
                          const float* __restrict__ boundary, float* __restrict__ out, float* __restrict__ total) {
  combine_elems(world, rank, backward, ns, V, gathered, boundary, out, total);
}

// ---------------------------------------------------------------------------
// Peer-memory exchange (regions and flag protocol in p2p.cuh).  Exchange e writes slot
// parity e & 1: rank r's slot of e + 2 is written only after every rank has finished
// reading e (each rank's push of e + 1 follows its combine of e on its stream, and rank r
// pushes e + 2 only after its combine of e + 1 saw every rank's push of e + 1).
// ---------------------------------------------------------------------------

// This rank's packed (state | decay) into its slot of every rank's region (plain stores
// through the peer mappings, NVLink), then the epoch flags (p2p::signal).  `vec`: per, ns and
// the pointers allow 16-byte accesses.
__global__ void k_p2p_push(int rank, int world, size_t ns, size_t nd, const float* __restrict__ s,
                           const float* __restrict__ d, void* const* __restrict__ regions, void* own, int vec) {
  const uint32_t epoch = p2p::next_epoch(own);
  const size_t per = ns + nd;
  const size_t slot = p2p::slot_offset(epoch, world, rank, per);
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  if (vec) {
    const size_t per4 = per / 4, ns4 = ns / 4;
    const float4* s4 = reinterpret_cast<const float4*>(s);
    const float4* d4 = reinterpret_cast<const float4*>(d);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < per4; i += stride) {
      const float4 x = i < ns4 ? s4[i] : d4[i - ns4];
      for (int p = 0; p < world; ++p) reinterpret_cast<float4*>(p2p::slots(regions[p]) + slot)[i] = x;
    }
  } else {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < per; i += stride) {
      const float x = i < ns ? s[i] : d[i - ns];
      for (int p = 0; p < world; ++p) p2p::slots(regions[p])[slot + i] = x;
    }
  }
  p2p::signal(regions, own, world, rank, epoch);
}

// Wait (bounded: limit_ns, then DEVERR_PEER_TIMEOUT and no output) until every rank's slot of
// this rank's latest epoch has arrived, then the prefix / suffix of k_combine from this
// rank's own region.
__global__ void k_p2p_combine(int world, int rank, int backward, size_t ns, int V, void* own,
                              const float* __restrict__ boundary, float* __restrict__ out, float* __restrict__ total,
                              uint64_t limit_ns) {
  __shared__ int ok;
  const uint32_t epoch = p2p::ld_volatile(p2p::epoch_word(own));
  const uint32_t par = epoch & 1u;
  if (threadIdx.x == 0) {
    int good = 1;
    const uint32_t* fl = p2p::flags(own) + par * p2p::MAX_WORLD;
    const uint64_t t0 = ptx::globaltimer_ns();
    for (int j = 0; j < world && good; ++j) {
      while ((int32_t)(p2p::ld_acquire_sys(fl + j) - epoch) < 0) {
        if (ptx::globaltimer_ns() - t0 > limit_ns) {
          ptx::record_error(ptx::DEVERR_PEER_TIMEOUT);
          good = 0;
          break;
        }
      }
    }
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  combine_elems(world, rank, backward, ns, V, p2p::slots(own) + (size_t)par * world * (ns + ns / V), boundary, out,
                total);
}

TOPS_DEVICE_ERROR_READER(read_device_error)

}  // namespace exchange
}  // namespace tops

using namespace tops;
using namespace tops::exchange;

extern "C" {

TOPS_API int tops_gla_nccl_get_unique_id(void* id) {
  TOPS_CHECK_ARG(id, "nccl_get_unique_id: id buffer is required");
  if (!nccl().ok) return fail(TOPS_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) is not available");
  ncclUniqueId u;
  int rc = nccl_status(nccl().get_unique_id(&u), "ncclGetUniqueId");
  if (rc == TOPS_OK) std::memcpy(id, &u, sizeof(u));
  return rc;
}

TOPS_API int tops_gla_nccl_comm_init(void** comm, int32_t world, const void* id, int32_t rank) {
  TOPS_CHECK_ARG(comm && id && world > 0 && rank >= 0 && rank < world, "nccl_comm_init: bad arguments");
  if (!nccl().ok) return fail(TOPS_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) is not available");
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  ncclComm_t c = nullptr;
  const int rc = nccl_status(nccl().comm_init_rank(&c, world, u, rank), "ncclCommInitRank");
  *comm = c;
  return rc;
}

TOPS_API int tops_gla_nccl_comm_destroy(void* comm) {
  if (comm == nullptr) return TOPS_OK;
  if (!nccl().ok) return fail(TOPS_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) is not available");
  return nccl_status(nccl().comm_destroy(static_cast<ncclComm_t>(comm)), "ncclCommDestroy");
}

TOPS_API int tops_gla_nccl_comm_abort(void* comm) {
  if (comm == nullptr) return TOPS_OK;
  if (!nccl().ok) return fail(TOPS_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) is not available");
  return nccl_status(nccl().comm_abort(static_cast<ncclComm_t>(comm)), "ncclCommAbort");
}

TOPS_API int tops_gla_nccl_comm_check(void* comm) {
  TOPS_CHECK_ARG(comm != nullptr, "nccl_comm_check: comm is NULL");
  if (!nccl().ok) return fail(TOPS_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) is not available");
  ncclResult_t ar = ncclSuccess;
  int rc = nccl_status(nccl().async_error(static_cast<ncclComm_t>(comm), &ar), "ncclCommGetAsyncError");
  if (rc) return rc;
  if (ar != ncclSuccess && ar != ncclInProgress) return nccl_status(ar, "NCCL communicator error");
  return TOPS_OK;
}

TOPS_API int tops_gla_state_exchange_wait(void* comm, void* stream, int32_t timeout_ms) {
  TOPS_CHECK_ARG(comm != nullptr && timeout_ms > 0, "state_exchange_wait: comm and a positive timeout are required");
  if (!nccl().ok) return fail(TOPS_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) is not available");
  cudaEvent_t ev = nullptr;
  cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
  if (e != cudaSuccess) return cuda_status(e, "state_exchange_wait: event");
  if ((e = cudaEventRecord(ev, static_cast<cudaStream_t>(stream))) != cudaSuccess) {
    cudaEventDestroy(ev);
    return cuda_status(e, "state_exchange_wait: record");
  }
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
  int rc = TOPS_OK;
  for (;;) {
    e = cudaEventQuery(ev);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) {
      rc = cuda_status(e, "state_exchange_wait");
      break;
    }
    if ((rc = tops_gla_nccl_comm_check(comm)) != TOPS_OK) {
      nccl().comm_abort(static_cast<ncclComm_t>(comm));
      break;
    }
    if (std::chrono::steady_clock::now() > deadline) {
      nccl().comm_abort(static_cast<ncclComm_t>(comm));
      rc = fail(TOPS_ERR_TIMEOUT, "state_exchange_wait: the exchange did not complete within " +
                                      std::to_string(timeout_ms) + " ms; the communicator was aborted");
      break;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
  cudaEventDestroy(ev);
  return rc;
}

TOPS_API size_t tops_gla_state_exchange_workspace_size(const tops_gla_exchange_args* a) {
  if (!a || a->world <= 0 || a->N <= 0 || a->H <= 0 || a->K <= 0 || a->V <= 0) return 0;
  const size_t ns = (size_t)a->N * a->H * a->K * a->V, nd = (size_t)a->N * a->H * a->K;
  return (size_t)(a->world + 1) * (ns + nd) * sizeof(float);
}

TOPS_API int tops_gla_state_exchange(const tops_gla_exchange_args* a, void* stream) {
  TOPS_CHECK_ARG(a, "state_exchange: args are required");
  TOPS_CHECK_ARG(a->comm && a->world > 0 && a->rank >= 0 && a->rank < a->world, "state_exchange: bad communicator");
  TOPS_CHECK_ARG(a->N > 0 && a->H > 0 && a->K > 0 && a->V > 0, "state_exchange: bad shape");
  TOPS_CHECK_ARG(a->local_state && a->decay && a->out, "state_exchange: local_state, decay and out are required");
  if (!nccl().ok) return fail(TOPS_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) is not available");
  const size_t need = tops_gla_state_exchange_workspace_size(a);
  if (a->workspace == nullptr || a->workspace_bytes < need)
    return fail(TOPS_ERR_WORKSPACE, "state_exchange: workspace smaller than tops_gla_state_exchange_workspace_size()");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t ns = (size_t)a->N * a->H * a->K * a->V, nd = (size_t)a->N * a->H * a->K;
  float* send = static_cast<float*>(a->workspace);
  float* gathered = send + ns + nd;
  const int blocks = (int)((ns + nd + 255) / 256 < 4096 ? (ns + nd + 255) / 256 : 4096);
  {
    LaunchTimer lt(st, "exchange_pack");
    k_pack<<<blocks, 256, 0, st>>>(ns, nd, a->local_state, a->decay, send);
    TOPS_CUDA_LAUNCH_CHECK("state_exchange pack");
  }
  int rc = nccl_status(nccl().all_gather(send, gathered, ns + nd, ncclFloat32, static_cast<ncclComm_t>(a->comm), st),
                       "ncclAllGather");
  if (rc) return rc;
  {
    LaunchTimer lt(st, "exchange_combine");
    const int cb = (int)((ns + 255) / 256 < 4096 ? (ns + 255) / 256 : 4096);
    k_combine<<<cb, 256, 0, st>>>(a->world, a->rank, a->backward, ns, a->V, gathered, a->boundary, a->out,
                                  a->backward ? nullptr : a->total);
    TOPS_CUDA_LAUNCH_CHECK("state_exchange combine");
  }
  return TOPS_OK;
}


TOPS_API size_t tops_gla_p2p_region_size(const tops_gla_p2p_args* a) {
  if (!a || a->world <= 0 || a->world > p2p::MAX_WORLD || a->N <= 0 || a->H <= 0 || a->K <= 0 || a->V <= 0) return 0;
  const size_t ns = (size_t)a->N * a->H * a->K * a->V, nd = (size_t)a->N * a->H * a->K;
  return p2p::CTRL + 2 * (size_t)a->world * (ns + nd) * sizeof(float);
}

TOPS_API int tops_gla_p2p_alloc(size_t bytes, void** region) {
  TOPS_CHECK_ARG(region && bytes > p2p::CTRL, "p2p_alloc: a region of at least its control block is required");
  *region = nullptr;
  cudaError_t e = cudaMalloc(region, bytes);
  if (e == cudaSuccess) e = cudaMemset(*region, 0, bytes);
  if (e != cudaSuccess) {
    if (*region) cudaFree(*region);
    *region = nullptr;
    return cuda_status(e, "p2p_alloc");
  }
  return TOPS_OK;
}

TOPS_API int tops_gla_p2p_free(void* region) {
  if (!region) return TOPS_OK;
  const cudaError_t e = cudaFree(region);
  return e == cudaSuccess ? TOPS_OK : cuda_status(e, "p2p_free");
}

TOPS_API int tops_gla_ipc_handle(const void* region, void* handle) {
  TOPS_CHECK_ARG(region && handle, "ipc_handle: region and handle are required");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(region));
  if (e != cudaSuccess) return cuda_status(e, "cudaIpcGetMemHandle");
  static_assert(sizeof(h) == TOPS_GLA_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  return TOPS_OK;
}

TOPS_API int tops_gla_ipc_open(const void* handle, void** region) {
  TOPS_CHECK_ARG(handle && region, "ipc_open: handle and region are required");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *region = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(region, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? TOPS_OK : cuda_status(e, "cudaIpcOpenMemHandle");
}

TOPS_API int tops_gla_ipc_close(void* region) {
  if (!region) return TOPS_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(region);
  return e == cudaSuccess ? TOPS_OK : cuda_status(e, "cudaIpcCloseMemHandle");
}

TOPS_API int tops_gla_p2p_exchange(const tops_gla_p2p_args* a, void* stream) {
  TOPS_CHECK_ARG(a, "p2p_exchange: args are required");
  TOPS_CHECK_ARG(a->world > 0 && a->world <= p2p::MAX_WORLD && a->rank >= 0 && a->rank < a->world,
                 "p2p_exchange: bad rank / world (at most 64 ranks)");
  TOPS_CHECK_ARG(a->N > 0 && a->H > 0 && a->K > 0 && a->V > 0, "p2p_exchange: bad shape");
  TOPS_CHECK_ARG(a->local_state && a->decay && a->out, "p2p_exchange: local_state, decay and out are required");
  TOPS_CHECK_ARG(a->regions && a->own_region, "p2p_exchange: regions (device array) and own_region are required");
  TOPS_CHECK_ARG(a->timeout_ms > 0, "p2p_exchange: timeout_ms must be positive");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t ns = (size_t)a->N * a->H * a->K * a->V, nd = (size_t)a->N * a->H * a->K;
  const int vec = ns % 4 == 0 && nd % 4 == 0 && (reinterpret_cast<uintptr_t>(a->local_state) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(a->decay) & 15) == 0;
  {
    LaunchTimer lt(st, "exchange_p2p_push");
    const size_t units = vec ? (ns + nd) / 4 : ns + nd;
    const int blocks = (int)((units + 255) / 256 < 1184 ? (units + 255) / 256 : 1184);
    k_p2p_push<<<blocks, 256, 0, st>>>(a->rank, a->world, ns, nd, a->local_state, a->decay, a->regions,
                                        a->own_region, vec);
    TOPS_CUDA_LAUNCH_CHECK("p2p_exchange push");
  }
  return tops_gla_p2p_combine(a, stream);
}

TOPS_API int tops_gla_p2p_combine(const tops_gla_p2p_args* a, void* stream) {
  TOPS_CHECK_ARG(a, "p2p_combine: args are required");
  TOPS_CHECK_ARG(a->world > 0 && a->world <= p2p::MAX_WORLD && a->rank >= 0 && a->rank < a->world,
                 "p2p_combine: bad rank / world (at most 64 ranks)");
  TOPS_CHECK_ARG(a->N > 0 && a->H > 0 && a->K > 0 && a->V > 0, "p2p_combine: bad shape");
  TOPS_CHECK_ARG(a->out && a->own_region, "p2p_combine: out and own_region are required");
  TOPS_CHECK_ARG(a->timeout_ms > 0, "p2p_combine: timeout_ms must be positive");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t ns = (size_t)a->N * a->H * a->K * a->V;
  LaunchTimer lt(st, "exchange_p2p_combine");
  const int cb = (int)((ns + 255) / 256 < 4096 ? (ns + 255) / 256 : 4096);
  k_p2p_combine<<<cb, 256, 0, st>>>(a->world, a->rank, a->backward, ns, a->V, a->own_region, a->boundary, a->out,
                                    a->backward ? nullptr : a->total, (uint64_t)a->timeout_ms * 1000000ull);
  TOPS_CUDA_LAUNCH_CHECK("p2p_exchange combine");
  return TOPS_OK;
}

}  // extern "C"
