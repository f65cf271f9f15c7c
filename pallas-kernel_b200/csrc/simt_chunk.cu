// Generic fp32 (CUDA-core) kernels for every chunked GLA sub-function.
//
// These follow the reference's decomposition one kernel per sub-function
// (tops/ops/gla/chunk.py, tops/ops/common/chunk_h.py) and compute in fp32 exactly
// as the reference does after its fp32 cast (chunk.py:1226-1231).  They serve
//   * fp32 inputs (parity 1e-4),
//   * the exported sub-function API (chunk_fwd_h, chunk_gla_fwd_intra_gk, ...),
//   * shapes the tcgen05 kernels do not cover.
// Ragged chunks (T or a segment not a multiple of C) are handled as zero padding,
// identical to the reference's padding (chunk.py:751-793, 1120-1126).
//
// Thread mapping used throughout: 256 threads own a 64x64 output tile,
// thread (ty, tx) = (tid/16, tid%16) holds rows ty+16a and columns tx+16b, a,b<4.

#include "common.cuh"

namespace tops {
namespace simt {

constexpr int TILE = 64;
constexpr int KT = 32;  // contraction tile
constexpr int NTHREADS = 256;

__device__ __forceinline__ size_t tok(int row, int h, int H, int D, int d) {
  return ((size_t)row * H + h) * D + d;
}
__device__ __forceinline__ size_t st_idx(int c, int h, int H, int K, int V, int k, int v) {
  return (((size_t)c * H + h) * K + k) * V + v;
}

// ---------------------------------------------------------------------------
// chunk-local cumsum: tops/ops/gla/chunk.py:55-107 (kernel), ref :20-52
// ---------------------------------------------------------------------------
__global__ void k_cumsum(tops_gla_shape sh, const float* __restrict__ g, float* __restrict__ out, int reverse,
                         float scale) {
  const ChunkRange r = chunk_range(sh, blockIdx.x);
  const int h = blockIdx.y;
  for (int kk = threadIdx.x; kk < sh.K; kk += blockDim.x) {
    float acc = 0.f;
    if (!reverse) {
      for (int t = r.s; t < r.e; ++t) {
        const size_t i = tok(t, h, sh.H, sh.K, kk);
        acc += g[i];
        out[i] = acc * scale;
      }
    } else {
      for (int t = r.e - 1; t >= r.s; --t) {
        const size_t i = tok(t, h, sh.H, sh.K, kk);
        acc += g[i];
        out[i] = acc * scale;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// forward state scan: tops/ops/common/chunk_h.py:277-396 (ref), kernel :18-119
// grid (K/64, V/64, N*H); the 64x64 state tile lives in registers.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NTHREADS)
k_fwd_h(tops_gla_shape sh, const T* __restrict__ k, const T* __restrict__ v, const float* __restrict__ gc,
        const float* __restrict__ h0, float* __restrict__ hout, float* __restrict__ ht) {
  const int H = sh.H, K = sh.K, V = sh.V, C = sh.chunk_size;
  const int k0 = blockIdx.x * TILE, v0 = blockIdx.y * TILE;
  const int n = blockIdx.z / H, h = blockIdx.z % H;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  __shared__ float kd[TILE][TILE + 1];
  __shared__ float vs[TILE][TILE + 1];
  __shared__ float gl[TILE];
  float st[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int kk = k0 + ty + 16 * a, vv = v0 + tx + 16 * b;
      st[a][b] = (h0 != nullptr && kk < K && vv < V) ? h0[st_idx(n, h, H, K, V, kk, vv)] : 0.f;
    }
  int bos, eos, ci;
  seq_range(sh, n, bos, eos, ci);
  for (int s = bos; s < eos; s += C, ++ci) {
    const int e = min(s + C, eos);
    if (hout != nullptr) {
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int kk = k0 + ty + 16 * a, vv = v0 + tx + 16 * b;
          if (kk < K && vv < V) hout[st_idx(ci, h, H, K, V, kk, vv)] = st[a][b];
        }
    }
    __syncthreads();
    if (tid < TILE) gl[tid] = (k0 + tid < K) ? gc[tok(e - 1, h, H, K, k0 + tid)] : 0.f;
    __syncthreads();
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const float d = expf(gl[ty + 16 * a]);
#pragma unroll
      for (int b = 0; b < 4; ++b) st[a][b] *= d;
    }
    for (int j0 = s; j0 < e; j0 += TILE) {
      const int L = min(TILE, e - j0);
      // every global load of the tile first, then the arithmetic: the loads of one thread's
      // 16 elements are in flight together instead of one dependent round trip each
      constexpr int PER = TILE * TILE / NTHREADS;
      float lk[PER], lg[PER], lv[PER];
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int i = tid + u * NTHREADS, j = i / TILE, c = i % TILE;
        lk[u] = 0.f;
        lg[u] = 0.f;
        lv[u] = 0.f;
        if (j < L && k0 + c < K) {
          const size_t o = tok(j0 + j, h, H, K, k0 + c);
          lk[u] = to_f(k[o]);
          lg[u] = gc[o];
        }
        if (j < L && v0 + c < V) lv[u] = to_f(v[tok(j0 + j, h, H, V, v0 + c)]);
      }
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int i = tid + u * NTHREADS, j = i / TILE, c = i % TILE;
        kd[j][c] = (j < L && k0 + c < K) ? lk[u] * expf(gl[c] - lg[u]) : 0.f;
        vs[j][c] = lv[u];
      }
      __syncthreads();
      for (int j = 0; j < L; ++j) {
        float kr[4], vr[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) kr[a] = kd[j][ty + 16 * a];
#pragma unroll
        for (int b = 0; b < 4; ++b) vr[b] = vs[j][tx + 16 * b];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int b = 0; b < 4; ++b) st[a][b] = fmaf(kr[a], vr[b], st[a][b]);
      }
      __syncthreads();
    }
  }
  if (ht != nullptr) {
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int kk = k0 + ty + 16 * a, vv = v0 + tx + 16 * b;
        if (kk < K && vv < V) ht[st_idx(n, h, H, K, V, kk, vv)] = st[a][b];
      }
  }
}

// ---------------------------------------------------------------------------
// reverse state-gradient scan: tops/ops/common/chunk_h.py:399-492 (ref), kernel :495-591
// dh[c] = gradient w.r.t. the state at the END of chunk c.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NTHREADS)
k_bwd_dh(tops_gla_shape sh, const T* __restrict__ q, const float* __restrict__ gc, const T* __restrict__ dO,
         const float* __restrict__ dht, float* __restrict__ dhout, float* __restrict__ dh0) {
  const int H = sh.H, K = sh.K, V = sh.V, C = sh.chunk_size;
  const int k0 = blockIdx.x * TILE, v0 = blockIdx.y * TILE;
  const int n = blockIdx.z / H, h = blockIdx.z % H;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const float scale = sh.scale;
  __shared__ float qh[TILE][TILE + 1];
  __shared__ float ds[TILE][TILE + 1];
  __shared__ float gl[TILE];
  float st[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int kk = k0 + ty + 16 * a, vv = v0 + tx + 16 * b;
      st[a][b] = (dht != nullptr && kk < K && vv < V) ? dht[st_idx(n, h, H, K, V, kk, vv)] : 0.f;
    }
  int bos, eos, c0;
  seq_range(sh, n, bos, eos, c0);
  const int nch = (eos - bos + C - 1) / C;
  for (int i = nch - 1; i >= 0; --i) {
    const int ci = c0 + i;
    const int s = bos + i * C, e = min(s + C, eos);
    if (dhout != nullptr) {
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int kk = k0 + ty + 16 * a, vv = v0 + tx + 16 * b;
          if (kk < K && vv < V) dhout[st_idx(ci, h, H, K, V, kk, vv)] = st[a][b];
        }
    }
    __syncthreads();
    if (tid < TILE) gl[tid] = (k0 + tid < K) ? gc[tok(e - 1, h, H, K, k0 + tid)] : 0.f;
    __syncthreads();
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const float d = expf(gl[ty + 16 * a]);
#pragma unroll
      for (int b = 0; b < 4; ++b) st[a][b] *= d;
    }
    for (int j0 = s; j0 < e; j0 += TILE) {
      const int L = min(TILE, e - j0);
      // every global load of the tile first, then the arithmetic (loads in flight together)
      constexpr int PER = TILE * TILE / NTHREADS;
      float lq[PER], lg[PER], ld[PER];
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int x = tid + u * NTHREADS, j = x / TILE, c = x % TILE;
        lq[u] = 0.f;
        lg[u] = 0.f;
        ld[u] = 0.f;
        if (j < L && k0 + c < K) {
          const size_t o = tok(j0 + j, h, H, K, k0 + c);
          lq[u] = to_f(q[o]);
          lg[u] = gc[o];
        }
        if (j < L && v0 + c < V) ld[u] = to_f(dO[tok(j0 + j, h, H, V, v0 + c)]);
      }
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int x = tid + u * NTHREADS, j = x / TILE, c = x % TILE;
        qh[j][c] = (j < L && k0 + c < K) ? lq[u] * expf(lg[u]) * scale : 0.f;
        ds[j][c] = ld[u];
      }
      __syncthreads();
      for (int j = 0; j < L; ++j) {
        float qr[4], dr[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) qr[a] = qh[j][ty + 16 * a];
#pragma unroll
        for (int b = 0; b < 4; ++b) dr[b] = ds[j][tx + 16 * b];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int b = 0; b < 4; ++b) st[a][b] = fmaf(qr[a], dr[b], st[a][b]);
      }
      __syncthreads();
    }
  }
  if (dh0 != nullptr) {
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int kk = k0 + ty + 16 * a, vv = v0 + tx + 16 * b;
        if (kk < K && vv < V) dh0[st_idx(n, h, H, K, V, kk, vv)] = st[a][b];
      }
  }
}

// ---------------------------------------------------------------------------
// per-chunk "row x row" products over a feature dimension:
//   MODE_INTRA: A_ij  = scale sum_k q_ik e^{G_ik-G_0k} k_jk e^{G_0k-G_jk}   (chunk.py:300-345)
//   MODE_DA   : dA_ij = scale sum_v do_iv v_jv                              (chunk.py:504-540)
// both causal (j <= i) and written as [rows, H, C].  grid (NT, H).
// ---------------------------------------------------------------------------
enum { MODE_INTRA = 0, MODE_DA = 1 };

template <typename T, int MODE>
__global__ void __launch_bounds__(NTHREADS)
k_rowrow(tops_gla_shape sh, const T* __restrict__ x, const T* __restrict__ y, const float* __restrict__ gc,
         float* __restrict__ out, int causal) {
  const ChunkRange r = chunk_range(sh, blockIdx.x);
  const int h = blockIdx.y;
  const int H = sh.H, C = sh.chunk_size;
  const int D = (MODE == MODE_INTRA) ? sh.K : sh.V;
  const int L = r.e - r.s;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  __shared__ float xs[TILE][KT + 1];
  __shared__ float ys[TILE][KT + 1];
  __shared__ float g0[KT];
  float acc[4][4] = {};
  for (int d0 = 0; d0 < D; d0 += KT) {
    if (MODE == MODE_INTRA) {
      if (tid < KT) g0[tid] = (d0 + tid < D) ? gc[tok(r.s, h, H, D, d0 + tid)] : 0.f;
      __syncthreads();
    }
    for (int z = tid; z < TILE * KT; z += NTHREADS) {
      const int i = z / KT, c = z % KT;
      float xv = 0.f, yv = 0.f;
      if (i < L && d0 + c < D) {
        const size_t o = tok(r.s + i, h, H, D, d0 + c);
        xv = to_f(x[o]);
        yv = to_f(y[o]);
        if (MODE == MODE_INTRA) {
          const float gg = gc[o] - g0[c];
          xv *= expf(gg);
          yv *= expf(-gg);
        }
      }
      xs[i][c] = xv;
      ys[i][c] = yv;
    }
    __syncthreads();
#pragma unroll 4
    for (int c = 0; c < KT; ++c) {
      float xr[4], yr[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) xr[a] = xs[ty + 16 * a][c];
#pragma unroll
      for (int b = 0; b < 4; ++b) yr[b] = ys[tx + 16 * b][c];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(xr[a], yr[b], acc[a][b]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int i = ty + 16 * a, j = tx + 16 * b;
      if (i < L && j < C) out[tok(r.s + i, h, H, C, j)] = ((!causal || j <= i) && j < L) ? acc[a][b] * sh.scale : 0.f;
    }
}

// ---------------------------------------------------------------------------
// Generic per-chunk 64x64 tile accumulation: acc[i][col] += sum_z X(i,z) Y(z,col).
// Loaders fill xs[i][z] and ys[z][col] for one KT-slice.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_tile(float (&acc)[4][4], const float (*xs)[KT + 1],
                                         const float (*ys)[TILE + 1], int ty, int tx) {
#pragma unroll 4
  for (int z = 0; z < KT; ++z) {
    float xr[4], yr[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) xr[a] = xs[ty + 16 * a][z];
#pragma unroll
    for (int b = 0; b < 4; ++b) yr[b] = ys[z][tx + 16 * b];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(xr[a], yr[b], acc[a][b]);
  }
}

// ---------------------------------------------------------------------------
// output: o = scale (q e^G) h_c + tril(A) v   (chunk.py:441-497, kernel :1259-1312)
// grid (NT, H, V/64)
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NTHREADS)
k_fwd_o(tops_gla_shape sh, const T* __restrict__ q, const T* __restrict__ v, const float* __restrict__ gc,
        const float* __restrict__ A, const float* __restrict__ hs, T* __restrict__ o) {
  const int c = blockIdx.x, h = blockIdx.y, v0 = blockIdx.z * TILE;
  const ChunkRange r = chunk_range(sh, c);
  const int H = sh.H, K = sh.K, V = sh.V, C = sh.chunk_size, L = r.e - r.s;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  __shared__ float xs[TILE][KT + 1];
  __shared__ float ys[KT][TILE + 1];
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += KT) {
    for (int z = tid; z < TILE * KT; z += NTHREADS) {
      const int i = z / KT, cc = z % KT;
      float xv = 0.f;
      if (i < L && k0 + cc < K) {
        const size_t off = tok(r.s + i, h, H, K, k0 + cc);
        xv = to_f(q[off]) * expf(gc[off]);
      }
      xs[i][cc] = xv;
    }
    for (int z = tid; z < KT * TILE; z += NTHREADS) {
      const int kk = z / TILE, cc = z % TILE;
      ys[kk][cc] = (k0 + kk < K && v0 + cc < V) ? hs[st_idx(c, h, H, K, V, k0 + kk, v0 + cc)] : 0.f;
    }
    __syncthreads();
    mma_tile(acc, xs, ys, ty, tx);
    __syncthreads();
  }
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] *= sh.scale;
  for (int j0 = 0; j0 < L; j0 += KT) {
    for (int z = tid; z < TILE * KT; z += NTHREADS) {
      const int i = z / KT, jj = z % KT, j = j0 + jj;
      xs[i][jj] = (i < L && j < L && j <= i) ? A[tok(r.s + i, h, H, C, j)] : 0.f;
    }
    for (int z = tid; z < KT * TILE; z += NTHREADS) {
      const int jj = z / TILE, cc = z % TILE, j = j0 + jj;
      ys[jj][cc] = (j < L && v0 + cc < V) ? to_f(v[tok(r.s + j, h, H, V, v0 + cc)]) : 0.f;
    }
    __syncthreads();
    mma_tile(acc, xs, ys, ty, tx);
    __syncthreads();
  }
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int i = ty + 16 * a, vv = v0 + tx + 16 * b;
      if (i < L && vv < V) o[tok(r.s + i, h, H, V, vv)] = from_f<T>(acc[a][b]);
    }
}

// ---------------------------------------------------------------------------
// dv = tril(A)^T do + (k e^{G_last - G}) dh_c    (chunk.py:547-596)
// grid (NT, H, V/64)
// ---------------------------------------------------------------------------
template <typename T, typename TO>
__global__ void __launch_bounds__(NTHREADS)
k_bwd_dv(tops_gla_shape sh, const T* __restrict__ k, const float* __restrict__ gc, const float* __restrict__ A,
         const T* __restrict__ dO, const float* __restrict__ dh, TO* __restrict__ dv) {
  const int c = blockIdx.x, h = blockIdx.y, v0 = blockIdx.z * TILE;
  const ChunkRange r = chunk_range(sh, c);
  const int H = sh.H, K = sh.K, V = sh.V, C = sh.chunk_size, L = r.e - r.s;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  __shared__ float xs[TILE][KT + 1];
  __shared__ float ys[KT][TILE + 1];
  __shared__ float gl[KT];
  float acc[4][4] = {};
  // intra: rows j, contraction over i >= j
  for (int i0 = 0; i0 < L; i0 += KT) {
    for (int z = tid; z < KT * TILE; z += NTHREADS) {
      const int ii = z / TILE, j = z % TILE, i = i0 + ii;
      xs[j][ii] = (i < L && j < L && j <= i) ? A[tok(r.s + i, h, H, C, j)] : 0.f;
    }
    for (int z = tid; z < KT * TILE; z += NTHREADS) {
      const int ii = z / TILE, cc = z % TILE, i = i0 + ii;
      ys[ii][cc] = (i < L && v0 + cc < V) ? to_f(dO[tok(r.s + i, h, H, V, v0 + cc)]) : 0.f;
    }
    __syncthreads();
    mma_tile(acc, xs, ys, ty, tx);
    __syncthreads();
  }
  // inter: rows j, contraction over k
  for (int k0 = 0; k0 < K; k0 += KT) {
    if (tid < KT) gl[tid] = (k0 + tid < K) ? gc[tok(r.e - 1, h, H, K, k0 + tid)] : 0.f;
    __syncthreads();
    for (int z = tid; z < TILE * KT; z += NTHREADS) {
      const int j = z / KT, kk = z % KT;
      float xv = 0.f;
      if (j < L && k0 + kk < K) {
        const size_t off = tok(r.s + j, h, H, K, k0 + kk);
        xv = to_f(k[off]) * expf(gl[kk] - gc[off]);
      }
      xs[j][kk] = xv;
    }
    for (int z = tid; z < KT * TILE; z += NTHREADS) {
      const int kk = z / TILE, cc = z % TILE;
      ys[kk][cc] = (k0 + kk < K && v0 + cc < V) ? dh[st_idx(c, h, H, K, V, k0 + kk, v0 + cc)] : 0.f;
    }
    __syncthreads();
    mma_tile(acc, xs, ys, ty, tx);
    __syncthreads();
  }
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int j = ty + 16 * a, vv = v0 + tx + 16 * b;
      if (j < L && vv < V) dv[tok(r.s + j, h, H, V, vv)] = from_f<TO>(acc[a][b]);
    }
}

// ---------------------------------------------------------------------------
// intra-chunk dq/dk from dA  (chunk.py:603-649), grid (NT, H, K/64)
//   dq_i = e^{G_i-G_0} sum_{j<=i} dA_ij (k_j e^{G_0-G_j})
//   dk_j = e^{G_0-G_j} sum_{i>=j} dA_ij (q_i e^{G_i-G_0})
// (the reference writes e^{G} and e^{-G}; the first-row reference point is the
//  same stabilisation its forward uses, chunk.py:330-332)
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NTHREADS)
k_bwd_dqk_intra(tops_gla_shape sh, const T* __restrict__ q, const T* __restrict__ k, const float* __restrict__ gc,
                const float* __restrict__ dA, float* __restrict__ dq, float* __restrict__ dk) {
  const int c = blockIdx.x, h = blockIdx.y, k0 = blockIdx.z * TILE;
  const ChunkRange r = chunk_range(sh, c);
  const int H = sh.H, K = sh.K, C = sh.chunk_size, L = r.e - r.s;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  __shared__ float xs[TILE][KT + 1];
  __shared__ float ys[KT][TILE + 1];
  __shared__ float g0[TILE];
  if (tid < TILE) g0[tid] = (k0 + tid < K) ? gc[tok(r.s, h, H, K, k0 + tid)] : 0.f;
  __syncthreads();
  float aq[4][4] = {}, ak[4][4] = {};
  for (int j0 = 0; j0 < L; j0 += KT) {
    // dq: X = dA[i][j], Y = kn[j][k]
    for (int z = tid; z < TILE * KT; z += NTHREADS) {
      const int i = z / KT, jj = z % KT, j = j0 + jj;
      xs[i][jj] = (i < L && j < L && j <= i) ? dA[tok(r.s + i, h, H, C, j)] : 0.f;
    }
    for (int z = tid; z < KT * TILE; z += NTHREADS) {
      const int jj = z / TILE, cc = z % TILE, j = j0 + jj;
      float yv = 0.f;
      if (j < L && k0 + cc < K) {
        const size_t off = tok(r.s + j, h, H, K, k0 + cc);
        yv = to_f(k[off]) * expf(g0[cc] - gc[off]);
      }
      ys[jj][cc] = yv;
    }
    __syncthreads();
    mma_tile(aq, xs, ys, ty, tx);
    __syncthreads();
  }
  for (int i0 = 0; i0 < L; i0 += KT) {
    // dk: X = dA^T[j][i], Y = qp[i][k]
    for (int z = tid; z < KT * TILE; z += NTHREADS) {
      const int ii = z / TILE, j = z % TILE, i = i0 + ii;
      xs[j][ii] = (i < L && j < L && j <= i) ? dA[tok(r.s + i, h, H, C, j)] : 0.f;
    }
    for (int z = tid; z < KT * TILE; z += NTHREADS) {
      const int ii = z / TILE, cc = z % TILE, i = i0 + ii;
      float yv = 0.f;
      if (i < L && k0 + cc < K) {
        const size_t off = tok(r.s + i, h, H, K, k0 + cc);
        yv = to_f(q[off]) * expf(gc[off] - g0[cc]);
      }
      ys[ii][cc] = yv;
    }
    __syncthreads();
    mma_tile(ak, xs, ys, ty, tx);
    __syncthreads();
  }
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int i = ty + 16 * a, kk = k0 + tx + 16 * b;
      if (i < L && kk < K) {
        const size_t off = tok(r.s + i, h, H, K, kk);
        const float gg = gc[off] - g0[tx + 16 * b];
        dq[off] = aq[a][b] * expf(gg);
        dk[off] = ak[a][b] * expf(-gg);
      }
    }
}

// ---------------------------------------------------------------------------
// inter-chunk dq/dk + gate gradient  (chunk.py:656-743), grid (NT, H, K/64)
// ---------------------------------------------------------------------------
template <typename T, typename TO>
__global__ void __launch_bounds__(NTHREADS)
k_bwd_dqkg(tops_gla_shape sh, const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
           const float* __restrict__ hs, const float* __restrict__ gc, const T* __restrict__ dO,
           const float* __restrict__ dh, const float* __restrict__ dq_in, const float* __restrict__ dk_in,
           TO* __restrict__ dq_out, TO* __restrict__ dk_out, float* __restrict__ dg) {
  const int c = blockIdx.x, h = blockIdx.y, k0 = blockIdx.z * TILE;
  const ChunkRange r = chunk_range(sh, c);
  const int H = sh.H, K = sh.K, V = sh.V, L = r.e - r.s;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  __shared__ float xab[2][TILE][KT + 1];  // reused as the dg_raw tile after the main loop
  float (*xa)[KT + 1] = xab[0];
  float (*xb)[KT + 1] = xab[1];
  __shared__ float ya[KT][TILE + 1];
  __shared__ float yb[KT][TILE + 1];
  __shared__ float hdh[TILE];
  __shared__ float red[16][TILE];
  float aq[4][4] = {}, ak[4][4] = {};
  float my_hdh = 0.f;
  for (int v0 = 0; v0 < V; v0 += KT) {
    for (int z = tid; z < TILE * KT; z += NTHREADS) {
      const int i = z / KT, vv = z % KT;
      float a = 0.f, b = 0.f;
      if (i < L && v0 + vv < V) {
        const size_t off = tok(r.s + i, h, H, V, v0 + vv);
        a = to_f(dO[off]);
        b = to_f(v[off]);
      }
      xa[i][vv] = a;
      xb[i][vv] = b;
    }
    for (int z = tid; z < TILE * KT; z += NTHREADS) {
      const int kk = z / KT, vv = z % KT;
      float a = 0.f, b = 0.f;
      if (k0 + kk < K && v0 + vv < V) {
        const size_t off = st_idx(c, h, H, K, V, k0 + kk, v0 + vv);
        a = hs[off];
        b = dh[off];
      }
      ya[vv][kk] = a;
      yb[vv][kk] = b;
    }
    __syncthreads();
    mma_tile(aq, xa, ya, ty, tx);
    mma_tile(ak, xb, yb, ty, tx);
    if (tid < TILE) {
      for (int vv = 0; vv < KT; ++vv) my_hdh = fmaf(ya[vv][tid], yb[vv][tid], my_hdh);
    }
    __syncthreads();
  }
  if (tid < TILE) hdh[tid] = my_hdh;
  // epilogue: combine, column sums; dg_raw goes to shared memory (aliases xa/xb, free after the loop)
  float (*dgr)[TILE + 1] = reinterpret_cast<float (*)[TILE + 1]>(&xab[0][0][0]);
  static_assert(2 * TILE * (KT + 1) >= TILE * (TILE + 1), "dg_raw tile must fit in the xa/xb buffer");
  float colsum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int i = ty + 16 * a, kc = tx + 16 * b, kk = k0 + kc;
      float dgraw = 0.f;
      if (i < L && kk < K) {
        const size_t off = tok(r.s + i, h, H, K, kk);
        const float G = gc[off];
        const float GL = gc[tok(r.e - 1, h, H, K, kk)];
        const float qv = to_f(q[off]), kv = to_f(k[off]);
        const float dqi = sh.scale * expf(G) * aq[a][b];
        const float dki = expf(GL - G) * ak[a][b];
        const float dqt = dq_in[off] + dqi;
        const float dkt = dk_in[off] + dki;
        dq_out[off] = from_f<TO>(dqt);
        dk_out[off] = from_f<TO>(dkt);
        dgraw = qv * dqt - kv * dkt;
        colsum[b] += dki * kv;
      }
      dgr[i][kc] = dgraw;
    }
#pragma unroll
  for (int b = 0; b < 4; ++b) red[ty][tx + 16 * b] = colsum[b];
  __syncthreads();
  if (tid < TILE) {
    const int kk = k0 + tid;
    if (kk < K) {
      float cs = 0.f;
      for (int y = 0; y < 16; ++y) cs += red[y][tid];
      const float GL = gc[tok(r.e - 1, h, H, K, kk)];
      const float inter = expf(GL) * hdh[tid] + cs;
      float run = 0.f;
      for (int i = L - 1; i >= 0; --i) {
        run += dgr[i][tid];
        dg[tok(r.s + i, h, H, K, kk)] = run + inter;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// launchers (validated by the C-ABI layer)
// ---------------------------------------------------------------------------
template <typename F>
static int dispatch_dtype(int dtype, F&& f) {
  switch (dtype) {
    case TOPS_F32: return f(float{});
    case TOPS_BF16: return f(__nv_bfloat16{});
    case TOPS_F16: return f(__half{});
  }
  return fail(TOPS_ERR_INVALID, "unknown dtype");
}

int cumsum(const tops_gla_shape& s, const float* g, float* out, int reverse, float scale, cudaStream_t st) {
  if (s.NT == 0 || s.H == 0) return TOPS_OK;
  const int threads = s.K >= 256 ? 256 : ((s.K + 31) / 32) * 32;
  LaunchTimer lt(st, "chunk_cumsum");
  k_cumsum<<<dim3(s.NT, s.H), threads, 0, st>>>(s, g, out, reverse, scale);
  TOPS_CUDA_LAUNCH_CHECK("chunk_local_cumsum");
  return TOPS_OK;
}

int fwd_h(const tops_gla_shape& s, const void* k, const void* v, const float* gc, const float* h0, float* h,
          float* ht, cudaStream_t st) {
  if (s.N == 0 || s.H == 0) return TOPS_OK;
  dim3 grid(ceil_div(s.K, TILE), ceil_div(s.V, TILE), s.N * s.H);
  return dispatch_dtype(s.dtype, [&](auto tag) {
    using T = decltype(tag);
    LaunchTimer lt(st, "chunk_fwd_h");
    k_fwd_h<T><<<grid, NTHREADS, 0, st>>>(s, (const T*)k, (const T*)v, gc, h0, h, ht);
    TOPS_CUDA_LAUNCH_CHECK("chunk_fwd_h");
    return (int)TOPS_OK;
  });
}

int bwd_dh(const tops_gla_shape& s, const void* q, const float* gc, const void* dO, const float* dht, float* dh,
           float* dh0, cudaStream_t st) {
  if (s.N == 0 || s.H == 0) return TOPS_OK;
  dim3 grid(ceil_div(s.K, TILE), ceil_div(s.V, TILE), s.N * s.H);
  return dispatch_dtype(s.dtype, [&](auto tag) {
    using T = decltype(tag);
    LaunchTimer lt(st, "chunk_bwd_dh");
    k_bwd_dh<T><<<grid, NTHREADS, 0, st>>>(s, (const T*)q, gc, (const T*)dO, dht, dh, dh0);
    TOPS_CUDA_LAUNCH_CHECK("chunk_bwd_dh");
    return (int)TOPS_OK;
  });
}

int fwd_intra(const tops_gla_shape& s, const void* q, const void* k, const float* gc, int causal, float* A,
              cudaStream_t st) {
  if (s.NT == 0 || s.H == 0) return TOPS_OK;
  return dispatch_dtype(s.dtype, [&](auto tag) {
    using T = decltype(tag);
    LaunchTimer lt(st, "chunk_fwd_intra");
    k_rowrow<T, MODE_INTRA><<<dim3(s.NT, s.H), NTHREADS, 0, st>>>(s, (const T*)q, (const T*)k, gc, A, causal);
    TOPS_CUDA_LAUNCH_CHECK("chunk_fwd_intra");
    return (int)TOPS_OK;
  });
}

int fwd_o(const tops_gla_shape& s, const void* q, const void* v, const float* gc, const float* A, const float* h,
          void* o, cudaStream_t st) {
  if (s.NT == 0 || s.H == 0) return TOPS_OK;
  return dispatch_dtype(s.dtype, [&](auto tag) {
    using T = decltype(tag);
    LaunchTimer lt(st, "chunk_fwd_o");
    k_fwd_o<T><<<dim3(s.NT, s.H, ceil_div(s.V, TILE)), NTHREADS, 0, st>>>(s, (const T*)q, (const T*)v, gc, A, h,
                                                                          (T*)o);
    TOPS_CUDA_LAUNCH_CHECK("chunk_fwd_o");
    return (int)TOPS_OK;
  });
}

int bwd_dA(const tops_gla_shape& s, const void* v, const void* dO, float* dA, cudaStream_t st) {
  if (s.NT == 0 || s.H == 0) return TOPS_OK;
  return dispatch_dtype(s.dtype, [&](auto tag) {
    using T = decltype(tag);
    LaunchTimer lt(st, "chunk_bwd_dA");
    k_rowrow<T, MODE_DA><<<dim3(s.NT, s.H), NTHREADS, 0, st>>>(s, (const T*)dO, (const T*)v, nullptr, dA, 1);
    TOPS_CUDA_LAUNCH_CHECK("chunk_bwd_dA");
    return (int)TOPS_OK;
  });
}

int bwd_dv(const tops_gla_shape& s, const void* k, const float* gc, const float* A, const void* dO, const float* dh,
           void* dv, int out_dtype, cudaStream_t st) {
  if (s.NT == 0 || s.H == 0) return TOPS_OK;
  return dispatch_dtype(s.dtype, [&](auto tag) {
    using T = decltype(tag);
    return dispatch_dtype(out_dtype, [&](auto otag) {
      using TO = decltype(otag);
      LaunchTimer lt(st, "chunk_bwd_dv");
      k_bwd_dv<T, TO><<<dim3(s.NT, s.H, ceil_div(s.V, TILE)), NTHREADS, 0, st>>>(s, (const T*)k, gc, A,
                                                                                 (const T*)dO, dh, (TO*)dv);
      TOPS_CUDA_LAUNCH_CHECK("chunk_bwd_dv");
      return (int)TOPS_OK;
    });
  });
}

int bwd_dqk_intra(const tops_gla_shape& s, const void* q, const void* k, const float* gc, const float* dA,
                  float* dq, float* dk, cudaStream_t st) {
  if (s.NT == 0 || s.H == 0) return TOPS_OK;
  return dispatch_dtype(s.dtype, [&](auto tag) {
    using T = decltype(tag);
    LaunchTimer lt(st, "chunk_bwd_dqk_intra");
    k_bwd_dqk_intra<T><<<dim3(s.NT, s.H, ceil_div(s.K, TILE)), NTHREADS, 0, st>>>(s, (const T*)q, (const T*)k, gc,
                                                                                  dA, dq, dk);
    TOPS_CUDA_LAUNCH_CHECK("chunk_bwd_dqk_intra");
    return (int)TOPS_OK;
  });
}

int bwd_dqkg(const tops_gla_shape& s, const void* q, const void* k, const void* v, const float* h, const float* gc,
             const void* dO, const float* dh, const float* dq_in, const float* dk_in, void* dq_out, void* dk_out,
             int out_dtype, float* dg, cudaStream_t st) {
  if (s.NT == 0 || s.H == 0) return TOPS_OK;
  dim3 grid(s.NT, s.H, ceil_div(s.K, TILE));
  return dispatch_dtype(s.dtype, [&](auto tag) {
    using T = decltype(tag);
    return dispatch_dtype(out_dtype, [&](auto otag) {
      using TO = decltype(otag);
      LaunchTimer lt(st, "chunk_bwd_dqkg");
      k_bwd_dqkg<T, TO><<<grid, NTHREADS, 0, st>>>(s, (const T*)q, (const T*)k, (const T*)v, h, gc, (const T*)dO,
                                                   dh, dq_in, dk_in, (TO*)dq_out, (TO*)dk_out, dg);
      TOPS_CUDA_LAUNCH_CHECK("chunk_bwd_dqkg");
      return (int)TOPS_OK;
    });
  });
}

}  // namespace simt
}  // namespace tops
