// Sequence-parallel state hand-off helpers (contiguous T/ngpu
// spans per rank).  The reference has no multi-device code; this is the exact
// linear decomposition of its chunked scan (tops/ops/common/chunk_h.py:372-386):
// a span's final state is  D * H_in + S  where S is the span's final state from a
// zero initial state and D = exp(sum of the span's gates) (diagonal in K).  The
// backward uses the same map transposed: dH_in = D * dH_out + dh0_local.
#include "common.cuh"

namespace tops {
namespace seqpar {

// grid (N*H, ceil(K/8)), 1024 threads: a warp reads 4 rows x 8 columns (one 32-byte sector
// per row), the 32 warps split the span and each thread keeps four independent
// accumulators (many loads in flight); partial sums are added in a fixed order, so the
// result is deterministic.
__global__ void __launch_bounds__(1024) k_span_decay(tops_gla_shape sh, const float* __restrict__ g,
                                                    float* __restrict__ decay) {
  const int H = sh.H, K = sh.K;
  const int n = blockIdx.x / H, h = blockIdx.x - n * H;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = lane & 7, r = (warp << 2) | (lane >> 3);  // column in tile, row slot 0..127
  const int kk = blockIdx.y * 8 + c;
  int bos, eos;
  if (sh.cu_seqlens != nullptr) { bos = sh.cu_seqlens[n]; eos = sh.cu_seqlens[n + 1]; }
  else { bos = n * sh.T; eos = bos + sh.T; }
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  if (kk < K) {
    const size_t stride = (size_t)H * K;
    const float* p = g + ((size_t)bos * H + h) * K + kk;
    const int len = eos - bos;
    int t = r;
    for (; t + 384 < len; t += 512) {
      a0 += __ldg(p + (size_t)t * stride);
      a1 += __ldg(p + (size_t)(t + 128) * stride);
      a2 += __ldg(p + (size_t)(t + 256) * stride);
      a3 += __ldg(p + (size_t)(t + 384) * stride);
    }
    for (; t < len; t += 128) a0 += __ldg(p + (size_t)t * stride);
  }
  __shared__ float red[128][9];
  red[r][c] = (a0 + a1) + (a2 + a3);
  __syncthreads();
  if (threadIdx.x < 8) {
    const int col = blockIdx.y * 8 + threadIdx.x;
    float s = 0.f;
    for (int y = 0; y < 128; ++y) s += red[y][threadIdx.x];
    if (col < K) decay[((size_t)n * H + h) * K + col] = expf(s);
  }
}

__global__ void k_state_combine(size_t total, int V, const float* __restrict__ decay, const float* __restrict__ hin,
                                const float* s_local, float* out) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    out[i] = fmaf(decay[i / V], hin[i], s_local[i]);
  }
}

int span_decay(const tops_gla_shape& s, const float* g, float* decay, cudaStream_t st) {
  if (s.N * s.H == 0) return TOPS_OK;
  k_span_decay<<<dim3(s.N * s.H, ceil_div(s.K, 8)), 1024, 0, st>>>(s, g, decay);
  TOPS_CUDA_LAUNCH_CHECK("span_decay");
  return TOPS_OK;
}

int state_combine(int N, int H, int K, int V, const float* decay, const float* h_in, const float* s_local,
                  float* out, cudaStream_t st) {
  const size_t total = (size_t)N * H * K * V;
  if (total == 0) return TOPS_OK;
  const size_t blocks = (total + 255) / 256 > 8192 ? 8192 : (total + 255) / 256;
  k_state_combine<<<(unsigned)blocks, 256, 0, st>>>(total, V, decay, h_in, s_local, out);
  TOPS_CUDA_LAUNCH_CHECK("state_combine");
  return TOPS_OK;
}

}  // namespace seqpar
}  // namespace tops
