// Decode step (T == 1) of the GLA recurrence as a streaming HBM kernel.
//
// Semantics: fused_recurrent_gla with one token (tops/ops/gla/fused_recurrent.py:17-132):
//     h = h0 * e^{gk}[:,None] * e^{gv}[None,:] + k^T v,   o = (scale q)^T h,   ht = h.
// The work is dominated by reading h0 and writing ht (fp32 [N,H,K,V]).  Each
// (sequence, head) state is a contiguous K*V*4-byte tile, split into P row blocks
// ("parts") of 32 KB.  A persistent CTA per SM (512 threads) streams its parts through
// a 6-stage shared-memory ring: one thread issues 1D bulk copies (TMA) of the state part
// and of the part's q/k/gk rows and v/gv vectors onto the stage's mbarrier; every thread
// updates 16-byte column groups of the part's rows in registers, accumulates o, and
// writes the new state straight to ht with coalesced 16-byte streaming stores (a warp
// writes whole 512-byte rows; ht is not read again by the step, so its lines are marked
// evict-first).  A stage is free as soon as it has been read, so five parts' loads stay
// in flight while one is updated and HBM sees continuous read and write streams.  The
// store stream needs the warps: 16 per SM reach 0.96 of the measured copy bandwidth at
// config 2, 8 per SM (256 threads) 0.83.
#include "common.cuh"
#include "ptx.cuh"

namespace tops {
namespace decode {

constexpr int THREADS = 512;
constexpr int STAGES = 6;
constexpr int AHEAD = STAGES - 1;  // loads in flight while one stage is updated
constexpr int PART_BYTES = 32 * 1024;
constexpr int COEF_BYTES = 4 * 1024;  // q,k,gk rows + v,gv of one part (fits K_part,V <= 256)

struct Params {
  int NH, H, K, V, R, P;  // R rows per part, P = K / R parts per tile
  float scale;
  const void* q; const void* k; const void* v;   // [N, 1, H, K|V]
  const float* gk; const float* gv; const float* h0;
  float* o; float* ht;
};

template <typename T, bool GK, bool GV, bool HAS_H0, bool HAS_HT>
__global__ void __launch_bounds__(THREADS, 1) k_decode(Params p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const int K = p.K, V = p.V, R = p.R, P = p.P;
  const int part_elems = R * V;
  const uint32_t part_bytes = (uint32_t)part_elems * 4u;
  // coefficient block layout inside a stage: q[R] T, k[R] T, gk[R] f32, v[V] T, gv[V] f32 (16 B aligned pieces)
  const uint32_t qb = (uint32_t)(R * sizeof(T)), gkb = (uint32_t)(R * 4), vb = (uint32_t)(V * sizeof(T)),
                 gvb = (uint32_t)(V * 4);
  const uint32_t off_k = qb, off_gk = 2 * qb, off_v = off_gk + (GK ? gkb : 0), off_gv = off_v + vb;
  const uint32_t coef_bytes = off_gv + (GV ? gvb : 0);
  __shared__ __align__(8) uint64_t bars[STAGES];
  __shared__ __align__(16) float red[THREADS * 4];

  auto stage_state = [&](int s) { return reinterpret_cast<float*>(smem + (size_t)s * (PART_BYTES + COEF_BYTES)); };
  auto stage_coef = [&](int s) { return smem + (size_t)s * (PART_BYTES + COEF_BYTES) + PART_BYTES; };

  const int tid = threadIdx.x;
  const int VC = V / 4;        // 16-byte column groups per row
  const int G = THREADS / VC;  // row groups (VC divides THREADS, G divides R)
  const int c4 = tid % VC, grp = tid / VC;
  const int ntiles = (p.NH - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const int nitems = ntiles * P;
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) ptx::mbar_init(&bars[s], 1);
    ptx::fence_mbar_init();
  }
  __syncthreads();

  auto issue = [&](int j) {  // thread 0: loads of item j into stage j % STAGES
    const int s = j % STAGES;
    const int nh = (int)blockIdx.x + (j / P) * (int)gridDim.x, part = j % P;
    const size_t row0 = (size_t)nh * K + (size_t)part * R;
    unsigned char* cf = stage_coef(s);
    ptx::mbar_arrive_expect_tx(&bars[s], (HAS_H0 ? part_bytes : 0u) + coef_bytes);
    if (HAS_H0) ptx::bulk_load(stage_state(s), p.h0 + row0 * V, part_bytes, &bars[s]);
    ptx::bulk_load(cf, static_cast<const T*>(p.q) + row0, qb, &bars[s]);
    ptx::bulk_load(cf + off_k, static_cast<const T*>(p.k) + row0, qb, &bars[s]);
    if (GK) ptx::bulk_load(cf + off_gk, p.gk + row0, gkb, &bars[s]);
    ptx::bulk_load(cf + off_v, static_cast<const T*>(p.v) + (size_t)nh * V, vb, &bars[s]);
    if (GV) ptx::bulk_load(cf + off_gv, p.gv + (size_t)nh * V, gvb, &bars[s]);
  };

  int next_issue = 0;  // meaningful in thread 0 only
  if (tid == 0)
    for (; next_issue < AHEAD && next_issue < nitems; ++next_issue) issue(next_issue);

  bool ok = true;
  int failed_at = nitems;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j = 0; j < nitems; ++j) {
    const int s = j % STAGES;
    const int nh = (int)blockIdx.x + (j / P) * (int)gridDim.x, part = j % P;
    if (tid == 0 && j + AHEAD < nitems) {
      issue(j + AHEAD);  // its stage was read by item j-1 (barrier at the end of the last iteration)
      next_issue = j + AHEAD + 1;
    }
    ok = ptx::bar_and(1, THREADS, ptx::mbar_wait(&bars[s], (uint32_t)((j / STAGES) & 1)));  // uniform exit
    if (!ok) {
      failed_at = j;
      break;
    }
    const float* buf = stage_state(s);
    const unsigned char* cf = stage_coef(s);
    const T* qs = reinterpret_cast<const T*>(cf);
    const T* ks = reinterpret_cast<const T*>(cf + off_k);
    const float* gks = reinterpret_cast<const float*>(cf + off_gk);
    const T* vs = reinterpret_cast<const T*>(cf + off_v);
    const float* gvs = reinterpret_cast<const float*>(cf + off_gv);
    float vc[4], ec[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      vc[e] = to_f(vs[4 * c4 + e]);
      ec[e] = GV ? expf(gvs[4 * c4 + e]) : 1.f;
    }
    float* hrow = HAS_HT ? p.ht + ((size_t)nh * K + (size_t)part * R) * V + 4 * c4 : nullptr;
#pragma unroll 4
    for (int r = grp; r < R; r += G) {
      float4 x = HAS_H0 ? *reinterpret_cast<const float4*>(buf + r * V + 4 * c4) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float d = GK ? expf(gks[r]) : 1.f;
      const float kr = to_f(ks[r]), qr = to_f(qs[r]);
      x.x = fmaf(kr, vc[0], x.x * d * ec[0]);
      x.y = fmaf(kr, vc[1], x.y * d * ec[1]);
      x.z = fmaf(kr, vc[2], x.z * d * ec[2]);
      x.w = fmaf(kr, vc[3], x.w * d * ec[3]);
      if (HAS_HT) __stcs(reinterpret_cast<float4*>(hrow + (size_t)r * V), x);
      acc.x = fmaf(qr, x.x, acc.x);
      acc.y = fmaf(qr, x.y, acc.y);
      acc.z = fmaf(qr, x.z, acc.z);
      acc.w = fmaf(qr, x.w, acc.w);
    }
    __syncthreads();  // stage s has been read by every thread: it may be refilled
    if (part == P - 1) {
      reinterpret_cast<float4*>(red)[grp * VC + c4] = acc;
      __syncthreads();
      if (tid < V) {
        float o = 0.f;
        for (int gi = 0; gi < G; ++gi) o += red[gi * V + tid];
        p.o[(size_t)nh * V + tid] = o * p.scale;
      }
      acc = make_float4(0.f, 0.f, 0.f, 0.f);
      __syncthreads();
    }
  }
  if (!ok && tid == 0) {
    // give up: let the loads already issued land before the CTA exits (bounded waits)
    for (int jj = failed_at + 1; jj < next_issue; ++jj)
      ptx::mbar_wait(&bars[jj % STAGES], (uint32_t)((jj / STAGES) & 1));
  }
  __syncthreads();
}

TOPS_DEVICE_ERROR_READER(read_device_error)

static bool rows_per_part(const tops_gla_recurrent_args& a, int& R) {
  R = PART_BYTES / (a.V * 4);
  if (R > a.K) R = a.K;
  return R >= 8 && a.K % R == 0;
}

bool supported(const tops_gla_recurrent_args& a) {
  if (a.T != 1 || a.cu_seqlens != nullptr) return false;
  if (!(a.V == 32 || a.V == 64 || a.V == 128 || a.V == 256)) return false;
  int R;
  if (!rows_per_part(a, R)) return false;
  const size_t es = a.dtype == TOPS_F32 ? 4 : 2;
  if ((R * es) % 16 != 0 || (a.V * es) % 16 != 0) return false;
  if (R % (THREADS / (a.V / 4)) != 0) return false;  // row groups divide the part
  if (2 * R * es + 4 * R + a.V * es + 4 * a.V > (size_t)COEF_BYTES) return false;
  auto al = [](const void* x) { return x == nullptr || (reinterpret_cast<uintptr_t>(x) & 15u) == 0; };
  return al(a.h0) && al(a.ht) && al(a.q) && al(a.k) && al(a.v) && al(a.gk) && al(a.gv);
}

template <typename T, bool GK, bool GV>
static cudaError_t launch3(const Params& p, bool h0, bool ht, int grid, size_t smem, cudaStream_t st) {
  void (*fn)(Params) = nullptr;
  if (h0 && ht) fn = k_decode<T, GK, GV, true, true>;
  else if (h0) fn = k_decode<T, GK, GV, true, false>;
  else if (ht) fn = k_decode<T, GK, GV, false, true>;
  else fn = k_decode<T, GK, GV, false, false>;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  fn<<<grid, THREADS, smem, st>>>(p);
  return cudaGetLastError();
}

int fwd(const tops_gla_recurrent_args& a, cudaStream_t st) {
  int R = 0;
  rows_per_part(a, R);
  Params p{a.N * a.H, a.H, a.K, a.V, R, a.K / R, a.scale, a.q, a.k, a.v, a.gk, a.gv, a.h0, a.o, a.ht};
  if (p.NH == 0) return TOPS_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = p.NH < sms ? p.NH : sms;
  const size_t smem = (size_t)STAGES * (PART_BYTES + COEF_BYTES);
  const bool h0 = a.h0 != nullptr, ht = a.ht != nullptr;
  const bool gk = a.gk != nullptr, gv = a.gv != nullptr;
  LaunchTimer lt(st, "recurrent_decode");
  cudaError_t e = cudaSuccess;
  auto go = [&](auto tag) {
    using T = decltype(tag);
    if (gk && gv) e = launch3<T, true, true>(p, h0, ht, grid, smem, st);
    else if (gk) e = launch3<T, true, false>(p, h0, ht, grid, smem, st);
    else if (gv) e = launch3<T, false, true>(p, h0, ht, grid, smem, st);
    else e = launch3<T, false, false>(p, h0, ht, grid, smem, st);
  };
  switch (a.dtype) {
    case TOPS_F32: go(float{}); break;
    case TOPS_BF16: go(__nv_bfloat16{}); break;
    case TOPS_F16: go(__half{}); break;
    default: return fail(TOPS_ERR_INVALID, "decode: unknown dtype");
  }
  if (e != cudaSuccess) return cuda_status(e, "fused_recurrent decode");
  note_launch(1);
  return TOPS_OK;
}

}  // namespace decode
}  // namespace tops
