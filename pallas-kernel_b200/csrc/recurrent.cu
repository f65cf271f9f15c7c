// Token-by-token GLA recurrence (decode path), fp32 state.
//
// Forward follows fused_recurrent_gla_fwd_ref / _fused_recurrent_gla_fwd_kernel
// (tops/ops/gla/fused_recurrent.py:17-132, 139-232):
//     h_t = h_{t-1} * e^{gk_t}[:,None] * e^{gv_t}[None,:] + k_t^T v_t,   o_t = (scale q_t)^T h_t
//
// B200 layout: one CTA of 8 warps owns a (sequence, head) state slab of
// (8*ROWS) K-rows x (32*VEC) V-columns kept in registers for the whole sequence.
// Lane l owns VEC consecutive columns, warp w owns ROWS consecutive rows, so every
// state row is one coalesced 128-bit-per-lane (512 B per warp) load/store.  The
// reduction over K for o is an in-register sum over ROWS plus an 8-way shared
// memory sum across warps.  At T = 1 (decode) the kernel is a single HBM pass:
// read h0, write ht, both streamed once.
#include "common.cuh"

namespace tops {
namespace rec {

constexpr int WARPS = 8;

struct Params {
  int B, T, H, K, V, N;
  float scale;
  int reverse;
  const int32_t* cu;
  const void* q; const void* k; const void* v;
  const float* gk; const float* gv; const float* h0;
  float* o;       // [B,T,H,V] (when gridDim.z == 1) or partial workspace [KS][B*T*H*V]
  float* ht;
};

template <int VEC> struct Vec;
template <> struct Vec<1> { using T = float; };
template <> struct Vec<4> { using T = float4; };

template <int VEC>
__device__ __forceinline__ void ld(const float* p, float (&x)[VEC]) {
  if constexpr (VEC == 4) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(p));
    x[0] = t.x; x[1] = t.y; x[2] = t.z; x[3] = t.w;
  } else {
    x[0] = __ldg(p);
  }
}
template <int VEC>
__device__ __forceinline__ void st_stream(float* p, const float (&x)[VEC]) {
  if constexpr (VEC == 4) {
    __stcs(reinterpret_cast<float4*>(p), make_float4(x[0], x[1], x[2], x[3]));
  } else {
    __stcs(p, x[0]);
  }
}

template <typename T, int ROWS, int VEC, bool GK, bool GV>
__global__ void __launch_bounds__(WARPS * 32)
k_fwd(Params p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = p.H, K = p.K, V = p.V;
  const int n = blockIdx.y / H, h = blockIdx.y - n * H;
  const int v0 = blockIdx.x * 32 * VEC + lane * VEC;
  const int kb = blockIdx.z * WARPS * ROWS + warp * ROWS;
  const bool vfull = (v0 + VEC <= V);
  __shared__ float red[WARPS][32 * VEC];

  float st[ROWS][VEC];
  const size_t sbase = ((size_t)n * H + h) * K;
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    const int kk = kb + r;
    if (p.h0 != nullptr && kk < K && vfull) {
      ld<VEC>(p.h0 + (sbase + kk) * V + v0, st[r]);
    } else {
#pragma unroll
      for (int c = 0; c < VEC; ++c)
        st[r][c] = (p.h0 != nullptr && kk < K && v0 + c < V) ? p.h0[(sbase + kk) * V + v0 + c] : 0.f;
    }
  }

  int bos, eos;
  if (p.cu != nullptr) { bos = p.cu[n]; eos = p.cu[n + 1]; }
  else { bos = n * p.T; eos = bos + p.T; }
  const T* q = static_cast<const T*>(p.q);
  const T* k = static_cast<const T*>(p.k);
  const T* vv = static_cast<const T*>(p.v);
  const int len = eos - bos;
  for (int step = 0; step < len; ++step) {
    const int t = p.reverse ? (eos - 1 - step) : (bos + step);
    const size_t kro = ((size_t)t * H + h) * K;
    const size_t vro = ((size_t)t * H + h) * V;
    float qr[ROWS], kr[ROWS], dr[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const int kk = kb + r;
      const bool ok = kk < K;
      qr[r] = ok ? to_f(q[kro + kk]) * p.scale : 0.f;
      kr[r] = ok ? to_f(k[kro + kk]) : 0.f;
      if constexpr (GK) dr[r] = ok ? expf(__ldg(p.gk + kro + kk)) : 1.f;
    }
    float vr[VEC], dv[VEC];
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
      const bool ok = v0 + c < V;
      vr[c] = ok ? to_f(vv[vro + v0 + c]) : 0.f;
      if constexpr (GV) dv[c] = ok ? expf(__ldg(p.gv + vro + v0 + c)) : 1.f;
    }
    float part[VEC];
#pragma unroll
    for (int c = 0; c < VEC; ++c) part[c] = 0.f;
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
#pragma unroll
      for (int c = 0; c < VEC; ++c) {
        float x = st[r][c];
        if constexpr (GK) x *= dr[r];
        if constexpr (GV) x *= dv[c];
        x = fmaf(kr[r], vr[c], x);
        st[r][c] = x;
        part[c] = fmaf(qr[r], x, part[c]);
      }
#pragma unroll
    for (int c = 0; c < VEC; ++c) red[warp][lane * VEC + c] = part[c];
    __syncthreads();
    if (threadIdx.x < 32 * VEC) {
      const int col = blockIdx.x * 32 * VEC + threadIdx.x;
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) s += red[w][threadIdx.x];
      if (col < V) {
        const size_t oo = vro + col;
        if (gridDim.z == 1) p.o[oo] = s;
        else p.o[(size_t)blockIdx.z * ((size_t)p.B * p.T * H * V) + oo] = s;
      }
    }
    __syncthreads();
  }

  if (p.ht != nullptr) {
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const int kk = kb + r;
      if (kk >= K) continue;
      if (vfull) {
        st_stream<VEC>(p.ht + (sbase + kk) * V + v0, st[r]);
      } else {
#pragma unroll
        for (int c = 0; c < VEC; ++c)
          if (v0 + c < V) p.ht[(sbase + kk) * V + v0 + c] = st[r][c];
      }
    }
  }
}

// sum of the K-split partial outputs (only when K > 8*32)
__global__ void k_sum_splits(const float* __restrict__ part, int splits, size_t n, float* __restrict__ o) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int z = 0; z < splits; ++z) s += part[(size_t)z * n + i];
    o[i] = s;
  }
}

template <typename T, int VEC, bool GK, bool GV>
static void launch_rows(const Params& p, int rows, dim3 grid, cudaStream_t st) {
  switch (rows) {
    case 1: k_fwd<T, 1, VEC, GK, GV><<<grid, WARPS * 32, 0, st>>>(p); break;
    case 2: k_fwd<T, 2, VEC, GK, GV><<<grid, WARPS * 32, 0, st>>>(p); break;
    case 4: k_fwd<T, 4, VEC, GK, GV><<<grid, WARPS * 32, 0, st>>>(p); break;
    case 8: k_fwd<T, 8, VEC, GK, GV><<<grid, WARPS * 32, 0, st>>>(p); break;
    case 16: k_fwd<T, 16, VEC, GK, GV><<<grid, WARPS * 32, 0, st>>>(p); break;
    default: k_fwd<T, 32, VEC, GK, GV><<<grid, WARPS * 32, 0, st>>>(p); break;
  }
}

template <typename T>
static void launch_typed(const Params& p, int rows, int vec, dim3 grid, cudaStream_t st) {
  const bool gk = p.gk != nullptr, gv = p.gv != nullptr;
  if (vec == 4) {
    if (gk && gv) launch_rows<T, 4, true, true>(p, rows, grid, st);
    else if (gk) launch_rows<T, 4, true, false>(p, rows, grid, st);
    else if (gv) launch_rows<T, 4, false, true>(p, rows, grid, st);
    else launch_rows<T, 4, false, false>(p, rows, grid, st);
  } else {
    if (gk && gv) launch_rows<T, 1, true, true>(p, rows, grid, st);
    else if (gk) launch_rows<T, 1, true, false>(p, rows, grid, st);
    else if (gv) launch_rows<T, 1, false, true>(p, rows, grid, st);
    else launch_rows<T, 1, false, false>(p, rows, grid, st);
  }
}

static void plan(int K, int& rows, int& splits) {
  rows = 1;
  while (rows < 32 && rows * WARPS < K) rows <<= 1;
  splits = ceil_div(K, rows * WARPS);
}

static bool aligned16(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace rec
namespace decode {
bool supported(const tops_gla_recurrent_args& a);
int fwd(const tops_gla_recurrent_args& a, cudaStream_t st);
}  // namespace decode
namespace rec {

// The forward over T > 1 steps splits K over more CTAs for the same reason as the backward
// (4 rows per warp; the partial outputs are summed by k_sum_splits): B64 T64 H16 K=V=128
// 1.59 -> 0.76 ms, B16 T256 1.79 -> 0.99 ms.  A decode step (T = 1) runs the decode kernel.
static void fwd_plan(const tops_gla_recurrent_args& a, int& rows, int& splits) {
  plan(a.K, rows, splits);
  if (a.T > 1 && rows > 4) {
    rows = 4;
    splits = ceil_div(a.K, rows * WARPS);
  }
}

size_t fwd_workspace(const tops_gla_recurrent_args& a) {
  if (decode::supported(a)) return 0;
  int rows, splits;
  fwd_plan(a, rows, splits);
  if (splits <= 1) return 0;
  return (size_t)splits * a.B * a.T * a.H * a.V * sizeof(float);
}

int fwd(const tops_gla_recurrent_args& a, cudaStream_t st) {
  if ((size_t)a.B * a.T * a.H == 0 && a.ht == nullptr) return TOPS_OK;
  if (decode::supported(a)) return decode::fwd(a, st);
  int rows, splits;
  fwd_plan(a, rows, splits);
  const size_t need = fwd_workspace(a);
  if (need > 0 && (a.workspace == nullptr || a.workspace_bytes < need))
    return fail(TOPS_ERR_WORKSPACE, "fused_recurrent: workspace smaller than tops_gla_recurrent_fwd_workspace_size()");
  const int vec = (a.V % 4 == 0 && aligned16(a.h0) && aligned16(a.ht)) ? 4 : 1;
  Params p{a.B, a.T, a.H, a.K, a.V, a.N, a.scale, a.reverse, a.cu_seqlens, a.q, a.k, a.v, a.gk, a.gv, a.h0,
           splits > 1 ? static_cast<float*>(a.workspace) : a.o, a.ht};
  dim3 grid(ceil_div(a.V, 32 * vec), a.N * a.H, splits);
  if (grid.y == 0) return TOPS_OK;
  LaunchTimer lt(st, "recurrent_fwd");
  switch (a.dtype) {
    case TOPS_F32: launch_typed<float>(p, rows, vec, grid, st); break;
    case TOPS_BF16: launch_typed<__nv_bfloat16>(p, rows, vec, grid, st); break;
    case TOPS_F16: launch_typed<__half>(p, rows, vec, grid, st); break;
    default: return fail(TOPS_ERR_INVALID, "fused_recurrent: unknown dtype");
  }
  TOPS_CUDA_LAUNCH_CHECK("fused_recurrent_fwd");
  if (splits > 1) {
    const size_t n = (size_t)a.B * a.T * a.H * a.V;
    const size_t blocks = (n + 255) / 256 > 4096 ? 4096 : (n + 255) / 256;
    k_sum_splits<<<(unsigned)blocks, 256, 0, st>>>(
        static_cast<const float*>(a.workspace), splits, n, a.o);
    TOPS_CUDA_LAUNCH_CHECK("fused_recurrent_fwd(sum)");
  }
  return TOPS_OK;
}

}  // namespace rec
}  // namespace tops

// ===========================================================================
// Backward of the recurrence (tops/ops/gla/fused_recurrent.py:879-956, kernel
// :495-790; CPU derivation tests/src/ops/common/fused_recurrent.py:118-305).
//
//   pass A (time order):    dq_t[k] = scale sum_v h_t[k,v] do_t[v]
//   pass B (reverse order): dh += scale q_t do_t^T;  dk_t = dh v_t;  dv_t = dh^T k_t;
//                           dh *= e^{gk_t} e^{gv_t};  dh0 = dh at the end
//   pass C (per sequence):  gate gradients by the reference's identity (:798-876)
//       dgk_t = sum_{s after-or-at t} (q_s dq_s - k_s dk_s) + sum_v dht*h_T
//       dgv_t = sum_{s after-or-at t} (o_s do_s - v_s dv_s) + sum_k dht*h_T
//   ("after" follows the processing order, i.e. a prefix sum when reverse=True).
// Partial sums over V-tiles (dq, dk) and K-splits (dv) go through the workspace
// and are added in a fixed order, so results are deterministic.
// ===========================================================================
namespace tops {
namespace rec {

struct BwdParams {
  Params f;
  const void* dO;
  const float* dht;
  float* dq_part;   // [VS][B*T*H*K]
  float* dk_part;   // [VS][B*T*H*K]
  float* dv_part;   // [KS][B*T*H*V]
  float* ck_part;   // [VS][N*H*K]  sum_v dht*h_T over the tile
  float* cv_part;   // [KS][N*H*V]
  float* dh0;
};

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// pass A: forward replay producing the per-tile partial dq and sum_v dht*h_T
template <typename T, int ROWS, int VEC, bool GK, bool GV>
__global__ void __launch_bounds__(WARPS * 32)
k_bwd_a(BwdParams bp) {
  const Params& p = bp.f;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = p.H, K = p.K, V = p.V;
  const int n = blockIdx.y / H, h = blockIdx.y - n * H;
  const int v0 = blockIdx.x * 32 * VEC + lane * VEC;
  const int kb = blockIdx.z * WARPS * ROWS + warp * ROWS;
  const size_t ntok = (size_t)p.B * p.T * H;
  float st[ROWS][VEC];
  const size_t sbase = ((size_t)n * H + h) * K;
#pragma unroll
  for (int r = 0; r < ROWS; ++r)
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
      const int kk = kb + r;
      st[r][c] = (p.h0 != nullptr && kk < K && v0 + c < V) ? p.h0[(sbase + kk) * V + v0 + c] : 0.f;
    }
  int bos, eos;
  if (p.cu != nullptr) { bos = p.cu[n]; eos = p.cu[n + 1]; }
  else { bos = n * p.T; eos = bos + p.T; }
  const T* k = static_cast<const T*>(p.k);
  const T* vv = static_cast<const T*>(p.v);
  const T* dO = static_cast<const T*>(bp.dO);
  for (int step = 0; step < eos - bos; ++step) {
    const int t = p.reverse ? (eos - 1 - step) : (bos + step);
    const size_t kro = ((size_t)t * H + h) * K, vro = ((size_t)t * H + h) * V;
    float vr[VEC], dv[VEC], dor[VEC];
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
      const bool ok = v0 + c < V;
      vr[c] = ok ? to_f(vv[vro + v0 + c]) : 0.f;
      dor[c] = ok ? to_f(dO[vro + v0 + c]) : 0.f;
      if constexpr (GV) dv[c] = ok ? expf(p.gv[vro + v0 + c]) : 1.f;
    }
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const int kk = kb + r;
      const bool ok = kk < K;
      const float kr = ok ? to_f(k[kro + kk]) : 0.f;
      float dr = 1.f;
      if constexpr (GK) dr = ok ? expf(p.gk[kro + kk]) : 1.f;
      float acc = 0.f;
#pragma unroll
      for (int c = 0; c < VEC; ++c) {
        float x = st[r][c] * dr;
        if constexpr (GV) x *= dv[c];
        x = fmaf(kr, vr[c], x);
        st[r][c] = x;
        acc = fmaf(x, dor[c], acc);
      }
      acc = warp_sum(acc);
      if (lane == 0 && ok) bp.dq_part[(size_t)blockIdx.x * ntok * K + kro + kk] = acc * p.scale;
    }
  }
  // corrections for the gate gradients: sum_v dht*h_T (per V-tile) and sum_k dht*h_T (per K-split)
  if (bp.dht != nullptr) {
    float cvs[VEC];
#pragma unroll
    for (int c = 0; c < VEC; ++c) cvs[c] = 0.f;
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const int kk = kb + r;
      float acc = 0.f;
#pragma unroll
      for (int c = 0; c < VEC; ++c) {
        const float d = (kk < K && v0 + c < V) ? bp.dht[(sbase + kk) * V + v0 + c] : 0.f;
        acc = fmaf(d, st[r][c], acc);
        cvs[c] = fmaf(d, st[r][c], cvs[c]);
      }
      acc = warp_sum(acc);
      if (lane == 0 && kk < K) bp.ck_part[(size_t)blockIdx.x * p.N * H * K + sbase + kk] = acc;
    }
    __shared__ float red[WARPS][32 * VEC];
#pragma unroll
    for (int c = 0; c < VEC; ++c) red[warp][lane * VEC + c] = cvs[c];
    __syncthreads();
    if (threadIdx.x < 32 * VEC) {
      const int col = blockIdx.x * 32 * VEC + threadIdx.x;
      float s = 0.f;
      for (int w = 0; w < WARPS; ++w) s += red[w][threadIdx.x];
      if (col < V) bp.cv_part[(size_t)blockIdx.z * p.N * H * V + ((size_t)n * H + h) * V + col] = s;
    }
  }
}

// pass B: reverse sweep for dk, dv and dh0
template <typename T, int ROWS, int VEC, bool GK, bool GV>
__global__ void __launch_bounds__(WARPS * 32)
k_bwd_b(BwdParams bp) {
  const Params& p = bp.f;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = p.H, K = p.K, V = p.V;
  const int n = blockIdx.y / H, h = blockIdx.y - n * H;
  const int v0 = blockIdx.x * 32 * VEC + lane * VEC;
  const int kb = blockIdx.z * WARPS * ROWS + warp * ROWS;
  const size_t ntok = (size_t)p.B * p.T * H;
  __shared__ float red[WARPS][32 * VEC];
  float dh[ROWS][VEC];
  const size_t sbase = ((size_t)n * H + h) * K;
#pragma unroll
  for (int r = 0; r < ROWS; ++r)
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
      const int kk = kb + r;
      dh[r][c] = (bp.dht != nullptr && kk < K && v0 + c < V) ? bp.dht[(sbase + kk) * V + v0 + c] : 0.f;
    }
  int bos, eos;
  if (p.cu != nullptr) { bos = p.cu[n]; eos = p.cu[n + 1]; }
  else { bos = n * p.T; eos = bos + p.T; }
  const T* q = static_cast<const T*>(p.q);
  const T* k = static_cast<const T*>(p.k);
  const T* vv = static_cast<const T*>(p.v);
  const T* dO = static_cast<const T*>(bp.dO);
  for (int step = eos - bos - 1; step >= 0; --step) {
    const int t = p.reverse ? (eos - 1 - step) : (bos + step);
    const size_t kro = ((size_t)t * H + h) * K, vro = ((size_t)t * H + h) * V;
    float vr[VEC], dv[VEC], dor[VEC], dvp[VEC];
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
      const bool ok = v0 + c < V;
      vr[c] = ok ? to_f(vv[vro + v0 + c]) : 0.f;
      dor[c] = ok ? to_f(dO[vro + v0 + c]) : 0.f;
      dv[c] = 1.f;
      if constexpr (GV) dv[c] = ok ? expf(p.gv[vro + v0 + c]) : 1.f;
      dvp[c] = 0.f;
    }
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const int kk = kb + r;
      const bool ok = kk < K;
      const float qr = ok ? to_f(q[kro + kk]) * p.scale : 0.f;
      const float kr = ok ? to_f(k[kro + kk]) : 0.f;
      float dr = 1.f;
      if constexpr (GK) dr = ok ? expf(p.gk[kro + kk]) : 1.f;
      float acc = 0.f;
#pragma unroll
      for (int c = 0; c < VEC; ++c) {
        const float x = fmaf(qr, dor[c], dh[r][c]);
        acc = fmaf(x, vr[c], acc);
        dvp[c] = fmaf(x, kr, dvp[c]);
        dh[r][c] = x * dr * dv[c];
      }
      acc = warp_sum(acc);
      if (lane == 0 && ok) bp.dk_part[(size_t)blockIdx.x * ntok * K + kro + kk] = acc;
    }
#pragma unroll
    for (int c = 0; c < VEC; ++c) red[warp][lane * VEC + c] = dvp[c];
    __syncthreads();
    if (threadIdx.x < 32 * VEC) {
      const int col = blockIdx.x * 32 * VEC + threadIdx.x;
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) s += red[w][threadIdx.x];
      if (col < V) bp.dv_part[(size_t)blockIdx.z * ntok * V + vro + col] = s;
    }
    __syncthreads();
  }
  if (bp.dh0 != nullptr) {
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
#pragma unroll
      for (int c = 0; c < VEC; ++c) {
        const int kk = kb + r;
        if (kk < K && v0 + c < V) bp.dh0[(sbase + kk) * V + v0 + c] = dh[r][c];
      }
  }
}

// pass C: add partials in a fixed order, then the gate-gradient scans; grid (N*H), block 256
template <typename T>
__global__ void k_bwd_c(BwdParams bp, int VS, int KS, float* dq, float* dk, float* dvo, float* dgk, float* dgv,
                        const float* o) {
  const Params& p = bp.f;
  const int H = p.H, K = p.K, V = p.V;
  const int n = blockIdx.x / H, h = blockIdx.x - n * H;
  const size_t ntok = (size_t)p.B * p.T * H;
  int bos, eos;
  if (p.cu != nullptr) { bos = p.cu[n]; eos = p.cu[n + 1]; }
  else { bos = n * p.T; eos = bos + p.T; }
  const T* q = static_cast<const T*>(p.q);
  const T* k = static_cast<const T*>(p.k);
  const T* vv = static_cast<const T*>(p.v);
  const T* dO = static_cast<const T*>(bp.dO);
  const int len = eos - bos;
  for (int kk = threadIdx.x; kk < K; kk += blockDim.x) {
    float run = 0.f;
    if (dgk != nullptr && bp.dht != nullptr)
      for (int z = 0; z < VS; ++z) run += bp.ck_part[(size_t)z * p.N * H * K + ((size_t)n * H + h) * K + kk];
    // walk in reverse processing order so `run` is the sum over steps processed at or after t
    for (int step = len - 1; step >= 0; --step) {
      const int t = p.reverse ? (eos - 1 - step) : (bos + step);
      const size_t i = ((size_t)t * H + h) * K + kk;
      float a = 0.f, b = 0.f;
      for (int z = 0; z < VS; ++z) {
        a += bp.dq_part[(size_t)z * ntok * K + i];
        b += bp.dk_part[(size_t)z * ntok * K + i];
      }
      dq[i] = a;
      dk[i] = b;
      if (dgk != nullptr) {
        run += to_f(q[i]) * a - to_f(k[i]) * b;
        dgk[i] = run;
      }
    }
  }
  for (int c = threadIdx.x; c < V; c += blockDim.x) {
    float run = 0.f;
    if (dgv != nullptr && bp.dht != nullptr)
      for (int z = 0; z < KS; ++z) run += bp.cv_part[(size_t)z * p.N * H * V + ((size_t)n * H + h) * V + c];
    for (int step = len - 1; step >= 0; --step) {
      const int t = p.reverse ? (eos - 1 - step) : (bos + step);
      const size_t i = ((size_t)t * H + h) * V + c;
      float a = 0.f;
      for (int z = 0; z < KS; ++z) a += bp.dv_part[(size_t)z * ntok * V + i];
      dvo[i] = a;
      if (dgv != nullptr) {
        run += o[i] * to_f(dO[i]) - to_f(vv[i]) * a;
        dgv[i] = run;
      }
    }
  }
}

// The backward's two passes walk T dependent steps per CTA; splitting K over more CTAs (4 rows
// per warp) gives the SMs 4x the CTAs to hide each step's latency and quarters the state held
// per thread.  The K-split partials of dv are summed in pass C.  Measured at H16 K=V=128:
// B16 T256 4.82 -> 2.43 ms, B64 T64 4.06 -> 1.99 ms (8 rows per warp: 3.55 / 2.65 ms; 2 rows:
// 2.78 / 2.34 ms).
static void bwd_plan(const tops_gla_recurrent_args& a, int& rows, int& splits, int& vec, int& vs) {
  plan(a.K, rows, splits);
  if (rows > 4) {
    rows = 4;
    splits = ceil_div(a.K, rows * WARPS);
  }
  vec = (a.V % 4 == 0) ? 4 : 1;
  vs = ceil_div(a.V, 32 * vec);
}

size_t bwd_workspace(const tops_gla_recurrent_bwd_args& a) {
  int rows, ks, vec, vs;
  bwd_plan(a.f, rows, ks, vec, vs);
  const size_t ntok = (size_t)a.f.B * a.f.T * a.f.H;
  const size_t ns = (size_t)a.f.N * a.f.H;
  size_t b = 0;
  auto take = [&](size_t elems) { b = (b + 255) & ~size_t(255); b += elems * sizeof(float); };
  take(vs * ntok * a.f.K);  // dq
  take(vs * ntok * a.f.K);  // dk
  take(ks * ntok * a.f.V);  // dv
  take(vs * ns * a.f.K);    // ck
  take(ks * ns * a.f.V);    // cv
  return b;
}

template <typename T, int VEC, bool GK, bool GV>
static void bwd_rows(const BwdParams& bp, int rows, dim3 grid, cudaStream_t st) {
#define TOPS_REC_BWD(R)                                              \
  k_bwd_a<T, R, VEC, GK, GV><<<grid, WARPS * 32, 0, st>>>(bp);        \
  k_bwd_b<T, R, VEC, GK, GV><<<grid, WARPS * 32, 0, st>>>(bp);
  switch (rows) {
    case 1: TOPS_REC_BWD(1) break;
    case 2: TOPS_REC_BWD(2) break;
    case 4: TOPS_REC_BWD(4) break;
    case 8: TOPS_REC_BWD(8) break;
    case 16: TOPS_REC_BWD(16) break;
    default: TOPS_REC_BWD(32) break;
  }
#undef TOPS_REC_BWD
}

template <typename T>
static void bwd_typed(const BwdParams& bp, int rows, int vec, dim3 grid, cudaStream_t st) {
  const bool gk = bp.f.gk != nullptr, gv = bp.f.gv != nullptr;
  if (vec == 4) {
    if (gk && gv) bwd_rows<T, 4, true, true>(bp, rows, grid, st);
    else if (gk) bwd_rows<T, 4, true, false>(bp, rows, grid, st);
    else if (gv) bwd_rows<T, 4, false, true>(bp, rows, grid, st);
    else bwd_rows<T, 4, false, false>(bp, rows, grid, st);
  } else {
    if (gk && gv) bwd_rows<T, 1, true, true>(bp, rows, grid, st);
    else if (gk) bwd_rows<T, 1, true, false>(bp, rows, grid, st);
    else if (gv) bwd_rows<T, 1, false, true>(bp, rows, grid, st);
    else bwd_rows<T, 1, false, false>(bp, rows, grid, st);
  }
}

int bwd(const tops_gla_recurrent_bwd_args& a, cudaStream_t st) {
  const tops_gla_recurrent_args& f = a.f;
  if (f.gv != nullptr && a.dgv != nullptr && a.o == nullptr)
    return fail(TOPS_ERR_INVALID, "fused_recurrent_bwd: o (forward output) is required when gv is used");
  int rows, ks, vec, vs;
  bwd_plan(f, rows, ks, vec, vs);
  const size_t need = bwd_workspace(a);
  if (f.workspace == nullptr || f.workspace_bytes < need)
    return fail(TOPS_ERR_WORKSPACE, "fused_recurrent_bwd: workspace smaller than the required size");
  const size_t ntok = (size_t)f.B * f.T * f.H;
  const size_t ns = (size_t)f.N * f.H;
  char* base = static_cast<char*>(f.workspace);
  size_t off = 0;
  auto take = [&](size_t elems) {
    off = (off + 255) & ~size_t(255);
    float* p = reinterpret_cast<float*>(base + off);
    off += elems * sizeof(float);
    return p;
  };
  BwdParams bp;
  bp.f = Params{f.B, f.T, f.H, f.K, f.V, f.N, f.scale, f.reverse, f.cu_seqlens, f.q, f.k, f.v, f.gk, f.gv, f.h0,
                nullptr, nullptr};
  bp.dO = a.do_;
  bp.dht = a.dht;
  bp.dq_part = take(vs * ntok * f.K);
  bp.dk_part = take(vs * ntok * f.K);
  bp.dv_part = take(ks * ntok * f.V);
  bp.ck_part = take(vs * ns * f.K);
  bp.cv_part = take(ks * ns * f.V);
  bp.dh0 = a.dh0;
  if (ns == 0) return TOPS_OK;
  dim3 grid(vs, f.N * f.H, ks);
  switch (f.dtype) {
    case TOPS_F32: bwd_typed<float>(bp, rows, vec, grid, st); break;
    case TOPS_BF16: bwd_typed<__nv_bfloat16>(bp, rows, vec, grid, st); break;
    case TOPS_F16: bwd_typed<__half>(bp, rows, vec, grid, st); break;
    default: return fail(TOPS_ERR_INVALID, "fused_recurrent_bwd: unknown dtype");
  }
  TOPS_CUDA_LAUNCH_CHECK("fused_recurrent_bwd(a,b)");
  note_launch(1);  // passes A and B are two launches
  switch (f.dtype) {
    case TOPS_F32:
      k_bwd_c<float><<<f.N * f.H, 256, 0, st>>>(bp, vs, ks, a.dq, a.dk, a.dv, a.dgk, a.dgv, a.o);
      break;
    case TOPS_BF16:
      k_bwd_c<__nv_bfloat16><<<f.N * f.H, 256, 0, st>>>(bp, vs, ks, a.dq, a.dk, a.dv, a.dgk, a.dgv, a.o);
      break;
    default:
      k_bwd_c<__half><<<f.N * f.H, 256, 0, st>>>(bp, vs, ks, a.dq, a.dk, a.dv, a.dgk, a.dgv, a.o);
      break;
  }
  TOPS_CUDA_LAUNCH_CHECK("fused_recurrent_bwd(c)");
  return TOPS_OK;
}

}  // namespace rec
}  // namespace tops
