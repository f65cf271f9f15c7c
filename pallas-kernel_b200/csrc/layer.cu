// Elementwise pieces of the GLA layer around the chunked op:
//  * fused RMSNorm x swish output gate, y = rmsnorm(o) * w * silu(g) per head row
//    (reference tops/modules/fused_norm_gate.py:28, the torch gold
//    tests/src/modules/fused_norm_gate.py:30-44), forward and backward;
//  * the gate activation gk = logsigmoid(x) / normalizer (optionally clamped from
//    below), tops/layers/gla.py:285-287, forward and backward.
// All arithmetic in fp32; tensors are fp32 or bf16 ([rows, V] row-major for the norm).
#include "common.cuh"

namespace tops {
namespace layer {

template <typename T>
struct Vec;  // 16-byte vector of T
template <>
struct Vec<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float (&r)[4]) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    r[0] = v.x; r[1] = v.y; r[2] = v.z; r[3] = v.w;
  }
  __device__ static void store(float* p, const float (&r)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(r[0], r[1], r[2], r[3]);
  }
};
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16* p, float (&r)[8]) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      r[2 * i] = f.x;
      r[2 * i + 1] = f.y;
    }
  }
  __device__ static void store(__nv_bfloat16* p, const float (&r)[8]) {
    uint4 v;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(r[2 * i], r[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = v;
  }
};

__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + __expf(-x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One warp per row; lane l owns vectors l, l+32, ... (MAXV vectors per lane, at most 4).
constexpr int MAXV_CAP = 4;

template <typename T, int MAXV>
__global__ void __launch_bounds__(256) k_norm_gate_fwd(int64_t rows, int V, float eps, const T* __restrict__ x,
                                                       const T* __restrict__ g, const T* __restrict__ w,
                                                       T* __restrict__ y, float* __restrict__ rstd) {
  constexpr int N = Vec<T>::N;
  const int lane = threadIdx.x & 31;
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int nvec = V / N;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += nw) {
    const T* xr = x + r * V;
    float xv[MAXV][N];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      const int c = lane + 32 * j;
      if (c < nvec) {
        Vec<T>::load(xr + c * N, xv[j]);
#pragma unroll
        for (int e = 0; e < N; ++e) ss = fmaf(xv[j][e], xv[j][e], ss);
      }
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / (float)V + eps);
    if (lane == 0 && rstd) rstd[r] = rs;
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      const int c = lane + 32 * j;
      if (c < nvec) {
        float gv[N], wv[N], out[N];
        Vec<T>::load(g + r * V + c * N, gv);
        if (w) Vec<T>::load(w + c * N, wv);
#pragma unroll
        for (int e = 0; e < N; ++e) {
          const float s = gv[e] * sigmoidf_(gv[e]);
          out[e] = xv[j][e] * rs * (w ? wv[e] : 1.f) * s;
        }
        Vec<T>::store(y + r * V + c * N, out);
      }
    }
  }
}

// dx, dg per row; each warp accumulates its rows' dw terms and writes them to its own
// workspace row, reduced over warps by k_colsum (fixed order: deterministic).
template <typename T, int MAXV>
__global__ void __launch_bounds__(256) k_norm_gate_bwd(int64_t rows, int V, const T* __restrict__ dy,
                                                       const T* __restrict__ x, const T* __restrict__ g,
                                                       const T* __restrict__ w, const float* __restrict__ rstd,
                                                       T* __restrict__ dx, T* __restrict__ dg,
                                                       float* __restrict__ dw_part) {
  constexpr int N = Vec<T>::N;
  const int lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int nvec = V / N;
  float dwacc[MAXV][N];
#pragma unroll
  for (int j = 0; j < MAXV; ++j)
#pragma unroll
    for (int e = 0; e < N; ++e) dwacc[j][e] = 0.f;
  for (int64_t r = gw; r < rows; r += nw) {
    const float rs = rstd[r];
    float xh[MAXV][N], gd[MAXV][N];  // xhat, then dxhat
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      const int c = lane + 32 * j;
      if (c < nvec) {
        float xv[N], gv[N], dv[N], wv[N], dgo[N];
        Vec<T>::load(x + r * V + c * N, xv);
        Vec<T>::load(g + r * V + c * N, gv);
        Vec<T>::load(dy + r * V + c * N, dv);
        if (w) Vec<T>::load(w + c * N, wv);
#pragma unroll
        for (int e = 0; e < N; ++e) {
          const float sg = sigmoidf_(gv[e]);
          const float s = gv[e] * sg;
          const float ds = sg * (1.f + gv[e] * (1.f - sg));
          const float wt = w ? wv[e] : 1.f;
          xh[j][e] = xv[e] * rs;
          dgo[e] = dv[e] * xh[j][e] * wt * ds;
          dwacc[j][e] = fmaf(dv[e] * s, xh[j][e], dwacc[j][e]);
          gd[j][e] = dv[e] * wt * s;
          dot = fmaf(gd[j][e], xh[j][e], dot);
        }
        Vec<T>::store(dg + r * V + c * N, dgo);
      }
    }
    dot = warp_sum(dot) / (float)V;
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      const int c = lane + 32 * j;
      if (c < nvec) {
        float o[N];
#pragma unroll
        for (int e = 0; e < N; ++e) o[e] = rs * (gd[j][e] - xh[j][e] * dot);
        Vec<T>::store(dx + r * V + c * N, o);
      }
    }
  }
  if (dw_part) {
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      const int c = lane + 32 * j;
      if (c < nvec) {
#pragma unroll
        for (int e = 0; e < N; ++e) dw_part[gw * V + c * N + e] = dwacc[j][e];
      }
    }
  }
}

// dw[v] = sum over parts of part[p][v] in a fixed order.  Block (32, 32): 32 columns,
// 32 interleaved slices of the parts, then a shared-memory sum over the slices.
template <typename T>
__global__ void __launch_bounds__(1024) k_colsum(int parts, int V, const float* __restrict__ part,
                                                 T* __restrict__ dw) {
  const int v = blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (v < V)
    for (int p = threadIdx.y; p < parts; p += 32) s += part[(size_t)p * V + v];
  __shared__ float red[32][33];
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && v < V) {
    float t = 0.f;
    for (int y = 0; y < 32; ++y) t += red[y][threadIdx.x];
    dw[v] = from_f<T>(t);
  }
}

template <typename T>
__global__ void k_gate_fwd(int64_t n, float inv_norm, float clamp_min, int has_clamp, const T* __restrict__ x,
                           float* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = to_f<T>(x[i]);
    float y = (fminf(v, 0.f) - log1pf(__expf(-fabsf(v)))) * inv_norm;  // logsigmoid(v) / normalizer
    if (has_clamp) y = fmaxf(y, clamp_min);
    out[i] = y;
  }
}

template <typename T>
__global__ void k_gate_bwd(int64_t n, float inv_norm, float clamp_min, int has_clamp, const T* __restrict__ x,
                           const float* __restrict__ dy, T* __restrict__ dx) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = to_f<T>(x[i]);
    float d = dy[i] * sigmoidf_(-v) * inv_norm;  // d logsigmoid(v) / dv = sigmoid(-v)
    if (has_clamp) {
      const float y = (fminf(v, 0.f) - log1pf(__expf(-fabsf(v)))) * inv_norm;
      if (y < clamp_min) d = 0.f;
    }
    dx[i] = from_f<T>(d);
  }
}

static int grid_for(int64_t rows, int warps_per_block, int per_sm = 8) {
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const int64_t need = (rows + warps_per_block - 1) / warps_per_block;
  const int64_t cap = (int64_t)nsm * per_sm;
  return (int)(need < cap ? (need > 0 ? need : 1) : cap);
}

static bool vec_ok(int V, int dtype) {
  const int N = dtype == TOPS_F32 ? 4 : 8;
  return V > 0 && V % N == 0 && V / N <= 32 * MAXV_CAP;
}

template <typename T>
static void launch_fwd(int grid, cudaStream_t st, int64_t rows, int V, float eps, const T* x, const T* g, const T* w,
                       T* y, float* rstd) {
  const int mv = (V / Vec<T>::N + 31) / 32;
  if (mv <= 1) k_norm_gate_fwd<T, 1><<<grid, 256, 0, st>>>(rows, V, eps, x, g, w, y, rstd);
  else if (mv == 2) k_norm_gate_fwd<T, 2><<<grid, 256, 0, st>>>(rows, V, eps, x, g, w, y, rstd);
  else k_norm_gate_fwd<T, 4><<<grid, 256, 0, st>>>(rows, V, eps, x, g, w, y, rstd);
}

template <typename T>
static void launch_bwd(int grid, cudaStream_t st, int64_t rows, int V, const T* dy, const T* x, const T* g, const T* w,
                       const float* rstd, T* dx, T* dg, float* part) {
  const int mv = (V / Vec<T>::N + 31) / 32;
  if (mv <= 1) k_norm_gate_bwd<T, 1><<<grid, 256, 0, st>>>(rows, V, dy, x, g, w, rstd, dx, dg, part);
  else if (mv == 2) k_norm_gate_bwd<T, 2><<<grid, 256, 0, st>>>(rows, V, dy, x, g, w, rstd, dx, dg, part);
  else k_norm_gate_bwd<T, 4><<<grid, 256, 0, st>>>(rows, V, dy, x, g, w, rstd, dx, dg, part);
}

}  // namespace layer
}  // namespace tops

using namespace tops;
using namespace tops::layer;

extern "C" {

TOPS_API int tops_gla_norm_gate_fwd(int64_t rows, int32_t V, int32_t dtype, float eps, const void* x, const void* g,
                                    const void* w, void* y, float* rstd, void* stream) {
  TOPS_CHECK_ARG(rows >= 0, "norm_gate: rows must be >= 0");
  TOPS_CHECK_ARG(dtype == TOPS_F32 || dtype == TOPS_BF16, "norm_gate: dtype must be fp32 or bf16");
  if (!vec_ok(V, dtype)) return fail(TOPS_ERR_UNSUPPORTED, "norm_gate: V must be a multiple of 16 bytes, <= 512 (fp32) / 1024 (bf16)");
  TOPS_CHECK_ARG(x && g && y, "norm_gate: x, g and y are required");
  if (rows == 0) return TOPS_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  LaunchTimer lt(st, "norm_gate_fwd");
  const int grid = grid_for(rows, 8);
  if (dtype == TOPS_F32)
    launch_fwd<float>(grid, st, rows, V, eps, static_cast<const float*>(x), static_cast<const float*>(g),
                      static_cast<const float*>(w), static_cast<float*>(y), rstd);
  else
    launch_fwd<__nv_bfloat16>(grid, st, rows, V, eps, static_cast<const __nv_bfloat16*>(x),
                              static_cast<const __nv_bfloat16*>(g), static_cast<const __nv_bfloat16*>(w),
                              static_cast<__nv_bfloat16*>(y), rstd);
  TOPS_CUDA_LAUNCH_CHECK("norm_gate_fwd");
  return TOPS_OK;
}

TOPS_API size_t tops_gla_norm_gate_bwd_workspace_size(int64_t rows, int32_t V) {
  if (rows <= 0 || V <= 0) return 0;
  return (size_t)grid_for(rows, 8, 2) * 8 * (size_t)V * sizeof(float);
}

TOPS_API int tops_gla_norm_gate_bwd(int64_t rows, int32_t V, int32_t dtype, const void* dy, const void* x,
                                    const void* g, const void* w, const float* rstd, void* dx, void* dg, void* dw,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  TOPS_CHECK_ARG(rows >= 0, "norm_gate: rows must be >= 0");
  TOPS_CHECK_ARG(dtype == TOPS_F32 || dtype == TOPS_BF16, "norm_gate: dtype must be fp32 or bf16");
  if (!vec_ok(V, dtype)) return fail(TOPS_ERR_UNSUPPORTED, "norm_gate: V must be a multiple of 16 bytes, <= 512 (fp32) / 1024 (bf16)");
  TOPS_CHECK_ARG(dy && x && g && rstd && dx && dg, "norm_gate_bwd: dy, x, g, rstd, dx and dg are required");
  TOPS_CHECK_ARG(!dw || w, "norm_gate_bwd: dw needs w");
  if (rows == 0) return TOPS_OK;
  const size_t need = tops_gla_norm_gate_bwd_workspace_size(rows, V);
  if (dw && (workspace == nullptr || workspace_bytes < need))
    return fail(TOPS_ERR_WORKSPACE, "norm_gate_bwd: workspace smaller than tops_gla_norm_gate_bwd_workspace_size()");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = grid_for(rows, 8, 2);  // few warps: each keeps its dw terms in registers
  float* part = dw ? static_cast<float*>(workspace) : nullptr;
  {
    LaunchTimer lt(st, "norm_gate_bwd");
    if (dtype == TOPS_F32)
      launch_bwd<float>(grid, st, rows, V, static_cast<const float*>(dy), static_cast<const float*>(x),
                        static_cast<const float*>(g), static_cast<const float*>(w), rstd, static_cast<float*>(dx),
                        static_cast<float*>(dg), part);
    else
      launch_bwd<__nv_bfloat16>(grid, st, rows, V, static_cast<const __nv_bfloat16*>(dy),
                                static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(g),
                                static_cast<const __nv_bfloat16*>(w), rstd, static_cast<__nv_bfloat16*>(dx),
                                static_cast<__nv_bfloat16*>(dg), part);
    TOPS_CUDA_LAUNCH_CHECK("norm_gate_bwd");
  }
  if (dw) {
    LaunchTimer lt(st, "norm_gate_dw");
    if (dtype == TOPS_F32)
      k_colsum<float><<<(V + 31) / 32, dim3(32, 32), 0, st>>>(grid * 8, V, part, static_cast<float*>(dw));
    else
      k_colsum<__nv_bfloat16><<<(V + 31) / 32, dim3(32, 32), 0, st>>>(grid * 8, V, part,
                                                                        static_cast<__nv_bfloat16*>(dw));
    TOPS_CUDA_LAUNCH_CHECK("norm_gate_dw");
  }
  return TOPS_OK;
}

TOPS_API int tops_gla_gate_logsigmoid_fwd(int64_t n, int32_t dtype, float normalizer, float clamp_min,
                                          int32_t has_clamp, const void* x, float* out, void* stream) {
  TOPS_CHECK_ARG(n >= 0 && normalizer != 0.f, "gate_logsigmoid: n >= 0 and a nonzero normalizer are required");
  TOPS_CHECK_ARG(dtype == TOPS_F32 || dtype == TOPS_BF16, "gate_logsigmoid: dtype must be fp32 or bf16");
  TOPS_CHECK_ARG(x && out, "gate_logsigmoid: x and out are required");
  if (n == 0) return TOPS_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  LaunchTimer lt(st, "gate_fwd");
  const int grid = grid_for((n + 255) / 256, 1);
  if (dtype == TOPS_F32)
    k_gate_fwd<float><<<grid, 256, 0, st>>>(n, 1.f / normalizer, clamp_min, has_clamp, static_cast<const float*>(x),
                                            out);
  else
    k_gate_fwd<__nv_bfloat16><<<grid, 256, 0, st>>>(n, 1.f / normalizer, clamp_min, has_clamp,
                                                    static_cast<const __nv_bfloat16*>(x), out);
  TOPS_CUDA_LAUNCH_CHECK("gate_fwd");
  return TOPS_OK;
}

TOPS_API int tops_gla_gate_logsigmoid_bwd(int64_t n, int32_t dtype, float normalizer, float clamp_min,
                                          int32_t has_clamp, const void* x, const float* dy, void* dx, void* stream) {
  TOPS_CHECK_ARG(n >= 0 && normalizer != 0.f, "gate_logsigmoid: n >= 0 and a nonzero normalizer are required");
  TOPS_CHECK_ARG(dtype == TOPS_F32 || dtype == TOPS_BF16, "gate_logsigmoid: dtype must be fp32 or bf16");
  TOPS_CHECK_ARG(x && dy && dx, "gate_logsigmoid_bwd: x, dy and dx are required");
  if (n == 0) return TOPS_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  LaunchTimer lt(st, "gate_bwd");
  const int grid = grid_for((n + 255) / 256, 1);
  if (dtype == TOPS_F32)
    k_gate_bwd<float><<<grid, 256, 0, st>>>(n, 1.f / normalizer, clamp_min, has_clamp, static_cast<const float*>(x),
                                            dy, static_cast<float*>(dx));
  else
    k_gate_bwd<__nv_bfloat16><<<grid, 256, 0, st>>>(n, 1.f / normalizer, clamp_min, has_clamp,
                                                    static_cast<const __nv_bfloat16*>(x), dy,
                                                    static_cast<__nv_bfloat16*>(dx));
  TOPS_CUDA_LAUNCH_CHECK("gate_bwd");
  return TOPS_OK;
}

}  // extern "C"
