// Shared device/host helpers of libtops_gla.so.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/tops_gla.h"

namespace tops {

// ---------------------------------------------------------------------------
// status / error string (thread-local, read by tops_gla_last_error)
// ---------------------------------------------------------------------------
void set_error(const std::string& msg);
int fail(int status, const std::string& msg);
int cuda_status(cudaError_t e, const char* what);
// counts kernel launches issued by this library (tops_gla_launch_count)
void note_launch(int n);

// Optional per-launch timing (tops_gla_timing_enable): CUDA events recorded on the
// launch stream around one kernel launch.  A no-op unless timing is enabled.
struct LaunchTimer {
  cudaStream_t st;
  const char* name;
  cudaEvent_t a = nullptr, b = nullptr;
  LaunchTimer(cudaStream_t s, const char* n);
  ~LaunchTimer();
};

#define TOPS_CHECK_ARG(cond, msg)                                   \
  do {                                                              \
    if (!(cond)) return ::tops::fail(TOPS_ERR_INVALID, (msg));      \
  } while (0)

#define TOPS_CUDA_LAUNCH_CHECK(what)                                          \
  do {                                                                        \
    cudaError_t e__ = cudaGetLastError();                                     \
    if (e__ != cudaSuccess) return ::tops::cuda_status(e__, (what));          \
    ::tops::note_launch(1);                                                   \
  } while (0)

// ---------------------------------------------------------------------------
// element access
// ---------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

// ---------------------------------------------------------------------------
// chunk map: chunk index -> (sequence, row range) in the flattened [B*T] row space
// ---------------------------------------------------------------------------
struct ChunkRange {
  int n;      // sequence
  int s, e;   // rows [s, e) of this chunk (e - s <= C; ragged last chunk)
  int bos, eos;
};

__device__ __forceinline__ ChunkRange chunk_range(const tops_gla_shape& sh, int c) {
  ChunkRange r;
  const int C = sh.chunk_size;
  if (sh.cu_seqlens == nullptr) {
    const int nts = (sh.T + C - 1) / C;
    r.n = c / nts;
    const int i = c - r.n * nts;
    r.bos = r.n * sh.T;
    r.eos = r.bos + sh.T;
    r.s = r.bos + i * C;
  } else {
    // largest n with chunk_offsets[n] <= c
    int lo = 0, hi = sh.N - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (__ldg(sh.chunk_offsets + mid) <= c) lo = mid; else hi = mid - 1;
    }
    r.n = lo;
    r.bos = __ldg(sh.cu_seqlens + lo);
    r.eos = __ldg(sh.cu_seqlens + lo + 1);
    r.s = r.bos + (c - __ldg(sh.chunk_offsets + lo)) * C;
  }
  r.e = min(r.s + C, r.eos);
  return r;
}

// sequence n -> rows [bos, eos) and the index of its first chunk
__device__ __forceinline__ void seq_range(const tops_gla_shape& sh, int n, int& bos, int& eos, int& c0) {
  if (sh.cu_seqlens == nullptr) {
    bos = n * sh.T;
    eos = bos + sh.T;
    c0 = n * ((sh.T + sh.chunk_size - 1) / sh.chunk_size);
  } else {
    bos = __ldg(sh.cu_seqlens + n);
    eos = __ldg(sh.cu_seqlens + n + 1);
    c0 = __ldg(sh.chunk_offsets + n);
  }
}

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

// validates the fields every chunked entry point relies on
int check_shape(const tops_gla_shape* s);

}  // namespace tops
