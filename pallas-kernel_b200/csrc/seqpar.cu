// Sequence-parallel state hand-off helpers (contiguous T/ngpu
// spans per rank).  The reference has no multi-device code; this is the exact
// linear decomposition of its chunked scan (tops/ops/common/chunk_h.py:372-386):
// a span's final state is  D * H_in + S  where S is the span's final state from a
// zero initial state and D = exp(sum of the span's gates) (diagonal in K).  The
// backward uses the same map transposed: dH_in = D * dH_out + dh0_local.
#include "common.cuh"

namespace tops {
namespace seqpar {

// grid (N*H, ceil(K/32)), block (32, 8): lanes over K (coalesced), warps split the span
__global__ void k_span_decay(tops_gla_shape sh, const float* __restrict__ g, float* __restrict__ decay) {
  const int H = sh.H, K = sh.K;
  const int n = blockIdx.x / H, h = blockIdx.x - n * H;
  const int kk = blockIdx.y * 32 + threadIdx.x;
  int bos, eos;
  if (sh.cu_seqlens != nullptr) { bos = sh.cu_seqlens[n]; eos = sh.cu_seqlens[n + 1]; }
  else { bos = n * sh.T; eos = bos + sh.T; }
  float acc = 0.f;
  if (kk < K)
    for (int t = bos + threadIdx.y; t < eos; t += blockDim.y) acc += g[((size_t)t * H + h) * K + kk];
  __shared__ float red[8][32];
  red[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y == 0 && kk < K) {
    float s = 0.f;
    for (int y = 0; y < 8; ++y) s += red[y][threadIdx.x];
    decay[((size_t)n * H + h) * K + kk] = expf(s);
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
  k_span_decay<<<dim3(s.N * s.H, ceil_div(s.K, 32)), dim3(32, 8), 0, st>>>(s, g, decay);
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
