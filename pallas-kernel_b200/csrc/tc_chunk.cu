// tcgen05 (5th-gen tensor core) kernels of the bf16 chunked GLA path on sm_100a.
//
// Math (reference tops/ops/gla/chunk.py:1083-1179 forward, 815-977 backward;
// tops/ops/common/chunk_h.py:277-492 state scans), with chunks of BT = 128 tokens
// (the result is independent of the chunk length in exact arithmetic; 128 matches
// the M = 128 tcgen05 tile):
//   G      = chunk-local cumsum of g;  GL = G at the chunk's last row;  Gm = G at row 63
//   qhat   = scale q e^{G}           kdec = k e^{GL - G}           D = e^{GL}
//   A      = scale tril((q e^{G-Gm}) (k e^{Gm-G})^T)     (mid-chunk reference row)
//   h_{c+1}= D_c * h_c + kdec_c^T v_c          (state scan, fp32 state in TMEM)
//   o_c    = qhat_c h_c + A_c v_c              (one GEMM over [qhat | A] x [h ; v])
// Backward pieces reuse the same kernels: the reverse scan dh_{c-1} = D_c dh_c +
// qhat_c^T do_c and dv_c = A_c^T do_c + kdec_c dh_c.
//
// Kernels
//   k_prep : persistent over (batch, chunk, head).  TMA loads q/k/g tiles, computes the gates in
//            registers, writes qhat/kdec (TMA store) and D, and the intra-chunk matrix
//            A with tcgen05.mma (accumulator in TMEM).
//   k_scan_out : (default) per (batch, head, 128-wide V tile): the state scan fused with
//            the chunk-output GEMM (fwd o, bwd dv); the state stays in TMEM and its bf16
//            copy in shared memory feeds the output MMA, so the output never reads the
//            chunk states back from HBM.
//   k_scan : per (batch, head, 128-wide V tile).  Walks the chunks in order (or in
//            reverse), state [K x 128] fp32 resident in TMEM, operands double
//            buffered by TMA; optionally stores every chunk-start state in bf16.  Used
//            for the zero-state span pass, the state-only entry points and the unfused path.
//   k_out  : (unfused path) persistent, warp specialised GEMM: TMA producer warp, MMA warp,
//            four epilogue warps; 6-stage shared-memory ring, double-buffered TMEM
//            accumulator.  out[128 x 128] = X[128 x K] S[K x 128] + A'[128 x 128] Y[128 x 128].
//   k_dqk  : per (batch, chunk, head, 64-wide K tile): dq, dk, dg from the chunk states
//            h and dh, do, v, q, k and g (two CTAs per SM).
// All waits are bounded (ptx::mbar_wait).  Shared-memory tiles use the 128-byte
// swizzle that TMA writes and the UMMA descriptors describe.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "p2p.cuh"
#include "ptx.cuh"

namespace tops {
namespace tc {

constexpr int BT = 128;   // chunk length (tokens)
constexpr int BV = 128;   // V tile
constexpr int TILE_BYTES = 128 * 128;  // one [128 rows][64 bf16] swizzled tile = 16 KB

using bf16 = __nv_bfloat16;

// ---------------------------------------------------------------------------
// host: tensor maps
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// rank-4 map over a [B, T, H, D] tensor: dims {D, H, T, B}; box {bx, 1, by, 1}
static bool map_tok(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int es, int B, int T, int H, int D,
                    int bx, int by) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)D * es, (cuuint64_t)H * D * es, (cuuint64_t)T * H * D * es};
  cuuint32_t box[4] = {(cuuint32_t)bx, 1, (cuuint32_t)by, 1};
  cuuint32_t es1[4] = {1, 1, 1, 1};
  return fn(m, dt, 4, const_cast<void*>(base), dims, strides, box, es1, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// rank-3 map over per-chunk states [R, K, V] (R = chunks*heads): dims {V, K, R}; box {64, by, 1}
static bool map_state(CUtensorMap* m, const void* base, int R, int K, int V, int by) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)V, (cuuint64_t)K, (cuuint64_t)R};
  cuuint64_t strides[2] = {(cuuint64_t)V * 2, (cuuint64_t)K * V * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)by, 1};
  cuuint32_t es1[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es1,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// rank-3 store map over per-chunk states with a [32 rows][32 bf16] box and 64-byte swizzle
static bool map_state_store(CUtensorMap* m, const void* base, int R, int K, int V) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)V, (cuuint64_t)K, (cuuint64_t)R};
  cuuint64_t strides[2] = {(cuuint64_t)V * 2, (cuuint64_t)K * V * 2};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t es1[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es1,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t desc_kmajor(const void* tile, uint32_t byte_off) {
  return ptx::sdesc_sw128(ptx::smem_u32(tile) + byte_off, 16, 1024);
}
__device__ __forceinline__ uint64_t desc_mnmajor(const void* tile, uint32_t byte_off, uint32_t mn_block_stride) {
  return ptx::sdesc_sw128(ptx::smem_u32(tile) + byte_off, mn_block_stride, 1024);
}
__device__ __forceinline__ float bf(const unsigned char* tile, uint32_t row, uint32_t col) {
  return __bfloat162float(*reinterpret_cast<const bf16*>(tile + ptx::sw128(row, col * 2)));
}
__device__ __forceinline__ void st_bf(unsigned char* tile, uint32_t row, uint32_t col, float x) {
  *reinterpret_cast<bf16*>(tile + ptx::sw128(row, col * 2)) = __float2bfloat16_rn(x);
}
__device__ __forceinline__ uint32_t tmem_lane_addr(uint32_t base, uint32_t lane0, uint32_t col) {
  return base + (lane0 << 16) + col;
}

// ===========================================================================
// k_prep: gates, qhat/kdec, D and the intra-chunk matrix A.  Persistent: min(items, 2 x SMs)
// CTAs of 256 threads (two per SM) walk the items (chunk, head, batch), chunk fastest; TMEM and
// the barriers stay set up across items, and the next item's first gate tiles load while the
// current item's last K block is gated.
// ===========================================================================
struct PrepParams {
  int B, T, H, K, NTb;
  float scale;
  float* D;  // [B*NTb, H, K]
};

struct PrepMaps {
  CUtensorMap q, k, g, qh, kd, A;
};

template <bool F16>  // q, k stored as fp16 (bf16 otherwise); the gated copies are bf16 either way
__global__ void __launch_bounds__(256, 2) k_prep(const __grid_constant__ PrepMaps maps, PrepParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* qb = smem;                   // [128][64] bf16: q -> qhat (in place)
  unsigned char* kb = qb + TILE_BYTES;        // k -> kdec
  unsigned char* gb = kb + TILE_BYTES;        // 2 x [128][32] fp32
  unsigned char* qt = gb + 2 * TILE_BYTES;    // q e^{G-Gm}
  unsigned char* kt = qt + TILE_BYTES;        // k e^{Gm-G}
  __shared__ __align__(16) float wtot[8][64];  // per-warp column sums of g
  __shared__ __align__(8) uint64_t bar_g, bar_qk, bar_mma;
  __shared__ uint32_t tmem_base;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nkb = p.K / 64;
  // persistent: this CTA takes items blockIdx.x, + gridDim.x, ...; item = (chunk, head, batch), chunk fastest
  const int items = p.NTb * p.H * p.B;
  auto coords = [&](int it_, int& c_, int& h_, int& b_) {
    c_ = it_ % p.NTb;
    h_ = (it_ / p.NTb) % p.H;
    b_ = it_ / (p.NTb * p.H);
  };
  int c, h, b;
  coords((int)blockIdx.x, c, h, b);

  if (warp == 0) {
    ptx::tmem_alloc(&tmem_base, 128);
    ptx::tmem_relinquish();
  }
  if (tid == 0) {
    ptx::mbar_init(&bar_g, 1);
    ptx::mbar_init(&bar_qk, 1);
    ptx::mbar_init(&bar_mma, 1);
    ptx::fence_mbar_init();
    // the gates of K block 0; each later block's gates (and the next item's first) load as
    // soon as the previous block's gates are in registers (g tiles free), ahead of its q / k
    ptx::mbar_arrive_expect_tx(&bar_g, 2 * TILE_BYTES);
    ptx::tma_load_4d(gb, &maps.g, 0, h, c * BT, b, &bar_g);
    ptx::tma_load_4d(gb + TILE_BYTES, &maps.g, 32, h, c * BT, b, &bar_g);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tacc = tmem_base;
  constexpr uint32_t IDESC = ptx::idesc_bf16(128, 128, false, false);

  // gating thread mapping: warp w owns rows w*16 .. w*16+15; lane = (row quad sub, 8-column chunk c)
  const int c8 = lane & 7, sub = lane >> 3, r0 = warp * 16 + sub * 4;
  // fp32 g: chunk c8 lives in tile c8/4 at byte (c8%4)*32; chunks 4..7 read their two 16-byte
  // halves in the opposite order so each 8-lane access phase touches 8 different bank groups
  const uint32_t go0 = (uint32_t)(c8 & 3) * 32 + ((c8 >> 2) ? 16u : 0u);
  bool ok = true;
  uint32_t kc = 0;  // K blocks processed by this CTA (mbarrier phases)
  for (int it = (int)blockIdx.x; it < items && ok; it += (int)gridDim.x) {
  coords(it, c, h, b);
  const int row0 = c * BT;
  for (int kbi = 0; kbi < nkb && ok; ++kbi, ++kc) {
    if (tid == 0) {
      if (kc > 0) ptx::bulk_wait_read<0>();  // earlier stores (qhat/kdec, the last item's A) have read their tiles
      ptx::mbar_arrive_expect_tx(&bar_qk, 2 * TILE_BYTES);
      ptx::tma_load_4d(qb, &maps.q, kbi * 64, h, row0, b, &bar_qk);
      ptx::tma_load_4d(kb, &maps.k, kbi * 64, h, row0, b, &bar_qk);
      if (kbi + 1 < nkb) {  // the next K block's q, k into L2 while this one is gated
        ptx::tma_prefetch_4d(&maps.q, kbi * 64 + 64, h, row0, b);
        ptx::tma_prefetch_4d(&maps.k, kbi * 64 + 64, h, row0, b);
      }
    }
    ok = ptx::bar_and(1, 256, ptx::mbar_wait(&bar_g, kc & 1u));  // uniform exit on a timeout
    if (!ok) break;
    const unsigned char* gt = gb + (c8 >> 2) * TILE_BYTES;
    float gv[4][8], ps[8];
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) {
      float4 lo = *reinterpret_cast<const float4*>(gt + ptx::sw128(r0 + rr, go0));
      float4 hi = *reinterpret_cast<const float4*>(gt + ptx::sw128(r0 + rr, go0 ^ 16u));
      if (c8 >> 2) {
        const float4 t = lo;
        lo = hi;
        hi = t;
      }
      gv[rr][0] = lo.x; gv[rr][1] = lo.y; gv[rr][2] = lo.z; gv[rr][3] = lo.w;
      gv[rr][4] = hi.x; gv[rr][5] = hi.y; gv[rr][6] = hi.z; gv[rr][7] = hi.w;
    }
    // inclusive scan over the 4 row quads of this warp (lanes 8 apart), then warp totals
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float own = gv[0][j] + gv[1][j] + gv[2][j] + gv[3][j];
      float v = own, t = __shfl_up_sync(0xffffffffu, v, 8);
      if (sub >= 1) v += t;
      t = __shfl_up_sync(0xffffffffu, v, 16);
      if (sub >= 2) v += t;
      ps[j] = v - own;  // sum of this warp's rows above this quad
      if (sub == 3) wtot[warp][c8 * 8 + j] = v;
    }
    __syncthreads();  // every thread holds its gates: the g tiles are free
    if (tid == 0 && (kbi + 1 < nkb || it + (int)gridDim.x < items)) {
      int gc = c, gh = h, gbb = b, gk = kbi * 64 + 64;
      if (kbi + 1 == nkb) {  // the next item's first K block
        coords(it + (int)gridDim.x, gc, gh, gbb);
        gk = 0;
      }
      ptx::fence_async_smem();
      ptx::mbar_arrive_expect_tx(&bar_g, 2 * TILE_BYTES);
      ptx::tma_load_4d(gb, &maps.g, gk, gh, gc * BT, gbb, &bar_g);
      ptx::tma_load_4d(gb + TILE_BYTES, &maps.g, gk + 32, gh, gc * BT, gbb, &bar_g);
    }
    float off[8], gm[8], gl[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      off[j] = ps[j];
      gm[j] = 0.f;
      gl[j] = 0.f;
    }
#pragma unroll
    for (int w2 = 0; w2 < 8; ++w2) {
      const float4 a4 = *reinterpret_cast<const float4*>(&wtot[w2][c8 * 8]);
      const float4 b4 = *reinterpret_cast<const float4*>(&wtot[w2][c8 * 8 + 4]);
      const float t8[8] = {a4.x, a4.y, a4.z, a4.w, b4.x, b4.y, b4.z, b4.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (w2 < warp) off[j] += t8[j];
        if (w2 < 4) gm[j] += t8[j];  // rows 0..63: Gm is G at row 63
        gl[j] += t8[j];
      }
    }
    float sq[8], sk[8];  // scale e^{Gm}, e^{GL-Gm}
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sq[j] = p.scale * __expf(gm[j]);
      sk[j] = __expf(gl[j] - gm[j]);
    }
    if (warp == 0 && sub == 0) {
      float* dp = p.D + ((size_t)(b * p.NTb + c) * p.H + h) * p.K + kbi * 64 + c8 * 8;
      reinterpret_cast<float4*>(dp)[0] = make_float4(__expf(gl[0]), __expf(gl[1]), __expf(gl[2]), __expf(gl[3]));
      reinterpret_cast<float4*>(dp)[1] = make_float4(__expf(gl[4]), __expf(gl[5]), __expf(gl[6]), __expf(gl[7]));
    }
    ok = ptx::bar_and(1, 256, ptx::mbar_wait(&bar_qk, kc & 1u));
    if (!ok) break;
    // all loads of the four rows first, then the arithmetic, then the stores (the
    // compiler cannot move loads across stores to buffers it cannot disambiguate)
    uint4 xq[4], xk[4];
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) {
      const uint32_t o = ptx::sw128(r0 + rr, c8 * 16);
      xq[rr] = *reinterpret_cast<const uint4*>(qb + o);
      xk[rr] = *reinterpret_cast<const uint4*>(kb + o);
    }
    float run[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) run[j] = off[j] - gm[j];  // running G - Gm
    uint32_t wqt[4][4], wkt[4][4], wqh[4][4], wkd[4][4];
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) {
      const uint32_t* q2 = reinterpret_cast<const uint32_t*>(&xq[rr]);
      const uint32_t* k2 = reinterpret_cast<const uint32_t*>(&xk[rr]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 fq = ptx::unpack16(q2[e], F16), fk = ptx::unpack16(k2[e], F16);
        run[2 * e] += gv[rr][2 * e];
        run[2 * e + 1] += gv[rr][2 * e + 1];
        const float a0 = __expf(run[2 * e]), a1 = __expf(run[2 * e + 1]);
        const float b0 = __expf(-run[2 * e]), b1 = __expf(-run[2 * e + 1]);
        const float qt0 = fq.x * a0, qt1 = fq.y * a1, kt0 = fk.x * b0, kt1 = fk.y * b1;
        wqt[rr][e] = ptx::pack_bf16(qt0, qt1);
        wkt[rr][e] = ptx::pack_bf16(kt0, kt1);
        wqh[rr][e] = ptx::pack_bf16(qt0 * sq[2 * e], qt1 * sq[2 * e + 1]);
        wkd[rr][e] = ptx::pack_bf16(kt0 * sk[2 * e], kt1 * sk[2 * e + 1]);
      }
    }
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) {
      const uint32_t o = ptx::sw128(r0 + rr, c8 * 16);
      *reinterpret_cast<uint4*>(qt + o) = make_uint4(wqt[rr][0], wqt[rr][1], wqt[rr][2], wqt[rr][3]);
      *reinterpret_cast<uint4*>(kt + o) = make_uint4(wkt[rr][0], wkt[rr][1], wkt[rr][2], wkt[rr][3]);
      *reinterpret_cast<uint4*>(qb + o) = make_uint4(wqh[rr][0], wqh[rr][1], wqh[rr][2], wqh[rr][3]);
      *reinterpret_cast<uint4*>(kb + o) = make_uint4(wkd[rr][0], wkd[rr][1], wkd[rr][2], wkd[rr][3]);
    }
    ptx::fence_async_smem();
    ptx::tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      ptx::tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        ptx::mma_bf16_ss(tacc, desc_kmajor(qt, ks * 32), desc_kmajor(kt, ks * 32), IDESC, (kbi | ks) ? 1u : 0u);
      ptx::mma_commit(&bar_mma);
      ptx::tma_store_4d(&maps.qh, kbi * 64, h, row0, b, qb);
      ptx::tma_store_4d(&maps.kd, kbi * 64, h, row0, b, kb);
      ptx::bulk_commit();
    }
    ok = ptx::bar_and(1, 256, ptx::mbar_wait(&bar_mma, kc & 1u));
    ptx::tc_fence_after();
  }
  if (ok) {
    // epilogue: A (TMEM, 128 x 128 fp32) -> causal mask, scale -> bf16 -> qt | kt -> TMA store
    const int qd = warp & 3, ch = warp >> 2;  // lane quadrant, column half
    const int i = qd * 32 + lane;
    unsigned char* stg = ch ? kt : qt;
#pragma unroll
    for (int cb = 0; cb < 2; ++cb) {
      float r[32];
      ptx::tmem_ld32(tmem_lane_addr(tacc, qd * 32, ch * 64 + cb * 32), r);
      ptx::tmem_ld_wait();
#pragma unroll
      for (int j4 = 0; j4 < 4; ++j4) {
        uint32_t w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j0 = ch * 64 + cb * 32 + j4 * 8 + 2 * u;
          const float a0 = (j0 <= i) ? r[j4 * 8 + 2 * u] * p.scale : 0.f;
          const float a1 = (j0 + 1 <= i) ? r[j4 * 8 + 2 * u + 1] * p.scale : 0.f;
          w[u] = ptx::pack_bf16(a0, a1);
        }
        *reinterpret_cast<uint4*>(stg + ptx::sw128(i, (cb * 32 + j4 * 8) * 2)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    ptx::fence_async_smem();
    ptx::tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      ptx::tma_store_4d(&maps.A, 0, h, row0, b, qt);
      ptx::tma_store_4d(&maps.A, 64, h, row0, b, kt);
      ptx::bulk_commit();
    }
  }
  }
  if (!ok && tid == 0) {  // drain loads that may still be in flight (bounded)
    ptx::mbar_wait(&bar_g, 0);
    ptx::mbar_wait(&bar_qk, 0);
  }
  if (tid == 0) ptx::bulk_wait<0>();
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) ptx::tmem_dealloc(tacc, 128);
}

// ===========================================================================
// k_scan: state scan over chunks.  grid (V/128, H, B * nspan), 256 threads.
// Long sequences with few (batch, head, V-tile) units are split into nspan spans of
// span_len chunks that scan in parallel: a first launch runs every span from a zero
// state (no chunk states stored) and returns its final state and the product of its
// chunk decays; k_span_prefix chains those into each span's incoming state
// (H_{s+1} = P_s H_s + E_s, the scan is linear in its initial state); a second launch
// re-runs every span from its incoming state and stores the chunk states.
// ===========================================================================
struct ScanParams {
  int B, T, H, K, V, NTb, reverse;
  const float* D;     // [B*NTb, H, K]
  const float* init;  // [nspan][B, H, K, V] fp32 (span s starts from init[s]) or null (zero)
  float* fin;         // fin_mode 0: [nspan][B, H, K, V] every span's final state; 1: [B, H, K, V] last span only
  bf16* states;       // [B*NTb, H, K, V] bf16 (chunk-start states) or null
  int nspan, span_len, fin_mode;
  float* span_decay;  // [nspan][B, H, K] product of each span's chunk decays, or null
  // segments of a padded varlen problem (B == 1, one span): sequence n owns blocks
  // [blk_off[n], blk_off[n+1]); grid.z = sequences; init / fin indexed by sequence; or null
  const int* blk_off;
};

struct ScanMaps {
  CUtensorMap x, y;  // x: [B,T,H,K] bf16 box (64,1,128,1); y: [B,T,H,V] bf16 box (64,1,128,1)
  CUtensorMap st;    // chunk states [B*NTb*H, K, V] bf16, box (32,32,1), 64-byte swizzle (store only)
};

// byte offset of (row, byte) in a [rows][64 B] tile with 64-byte swizzle (TMA SWIZZLE_64B, 512 B-aligned base)
__device__ __forceinline__ uint32_t sw64(uint32_t row, uint32_t byte_in_row) {
  return row * 64u + ((((byte_in_row >> 4) ^ ((row >> 1) & 3u)) << 4) | (byte_in_row & 15u));
}

template <bool SEG>  // SEG: padded varlen problem, chunk ranges from p.blk_off
__global__ void __launch_bounds__(256, 1) k_scan(const __grid_constant__ ScanMaps maps, ScanParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nh = (p.K + 127) / 128;      // state halves (TMEM lane blocks); K = 64 uses half of one
  const int nkb = 2 * nh;                // X tiles per chunk (past K: zero-filled by the loads)
  const uint32_t buf_bytes = (uint32_t)(nkb + 2) * TILE_BYTES;
  unsigned char* stage_st = smem + 2 * buf_bytes;  // 8 warps x 2 slots x 2 KB
  __shared__ __align__(8) uint64_t bar_full[2], bar_mma;
  __shared__ uint32_t tmem_base;

  const int vt = blockIdx.x, h = blockIdx.y;
  constexpr bool seg = SEG;
  // b: batch index of the chunk data; sq: index of this CTA's initial / final state
  const int b = seg ? 0 : blockIdx.z / p.nspan, sp_ = seg ? 0 : blockIdx.z % p.nspan;
  const int sq = seg ? (int)blockIdx.z : b;
  const int v0 = vt * BV;
  const int i0 = seg ? p.blk_off[blockIdx.z] : sp_ * p.span_len;                        // first chunk
  const int n_it = seg ? p.blk_off[blockIdx.z + 1] - i0 : min(p.span_len, p.NTb - i0);  // chunks
  const size_t span_off = (size_t)sp_ * p.B * p.H * p.K * p.V;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = warp & 3, hf = warp >> 2;  // lane quadrant, state half handled by this warp
  const int krow = hf * 128 + qd * 32 + lane;
  const bool active = hf < nh;
  const bool krow_ok = krow < p.K;  // uniform per warp (K is a multiple of 64)

  if (warp == 0) {
    ptx::tmem_alloc(&tmem_base, 512);
    ptx::tmem_relinquish();
  }
  if (tid == 0) {
    ptx::mbar_init(&bar_full[0], 1);
    ptx::mbar_init(&bar_full[1], 1);
    ptx::mbar_init(&bar_mma, 1);
    ptx::fence_mbar_init();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  // two TMEM state buffers of 256 columns: the chunk-start state h_c (read) and the
  // next state D_c h_c + X^T Y (written by the MMA); they swap every chunk, so the
  // bf16 store of h_c overlaps the MMA that forms h_{c+1}.
  auto sbuf = [&](int i) { return tmem_base + (uint32_t)((i & 1) * 256); };
  constexpr uint32_t IDESC = ptx::idesc_bf16(128, 128, true, true);

  auto chunk_of = [&](int i) {
    if constexpr (SEG) return p.reverse ? i0 + n_it - 1 - i : i0 + i;
    else return p.reverse ? p.NTb - 1 - (i0 + i) : i0 + i;
  };
  auto issue = [&](int i) {
    const int c = chunk_of(i);
    unsigned char* buf = smem + (i & 1) * buf_bytes;
    ptx::mbar_arrive_expect_tx(&bar_full[i & 1], buf_bytes);
    for (int j = 0; j < nkb; ++j) ptx::tma_load_4d(buf + j * TILE_BYTES, &maps.x, j * 64, h, c * BT, b, &bar_full[i & 1]);
    ptx::tma_load_4d(buf + nkb * TILE_BYTES, &maps.y, v0, h, c * BT, b, &bar_full[i & 1]);
    ptx::tma_load_4d(buf + (nkb + 1) * TILE_BYTES, &maps.y, v0 + 64, h, c * BT, b, &bar_full[i & 1]);
  };
  if (tid == 0) {
    if (!SEG || n_it > 0) issue(0);  // a varlen segment may be empty
    if (n_it > 1) issue(1);
  }
  // initial state -> TMEM buffer 0
  if (active) {
    const size_t srow = ((size_t)(sq * p.H + h) * p.K + krow) * p.V + v0;
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) {
      float r[32];
#pragma unroll
      for (int j = 0; j < 32; ++j)
        r[j] = (p.init && krow_ok && v0 + cb * 32 + j < p.V) ? p.init[span_off + srow + cb * 32 + j] : 0.f;
      ptx::tmem_st32(tmem_lane_addr(sbuf(0), qd * 32, hf * 128 + cb * 32), r);
    }
    ptx::tmem_st_wait();
  }
  bool ok = true;
  // the decay of chunk i+1 is fetched one iteration ahead (its latency hides behind chunk i)
  auto decay_of = [&](int i) {
    return active && krow_ok && i < n_it ? __ldg(p.D + ((size_t)(b * p.NTb + chunk_of(i)) * p.H + h) * p.K + krow)
                                         : 1.f;
  };
  float d_next = decay_of(0), dprod = 1.f;
  for (int i = 0; i < n_it; ++i) {
    const int c = chunk_of(i);
    const float d = d_next;
    dprod *= d;
    d_next = decay_of(i + 1);
    if (i > 0) {
      ok = ptx::bar_and(1, 256, ptx::mbar_wait(&bar_mma, (uint32_t)((i - 1) & 1)));  // uniform exit on a timeout
      ptx::tc_fence_after();
      if (!ok) break;
      if (tid == 0 && i + 1 < n_it) issue(i + 1);  // buffer (i+1)&1 was read by chunk i-1, now complete
    }
    // pass A: next-state buffer <- D_c * h_c (h_c stays untouched in its buffer)
    if (active) {
#pragma unroll
      for (int cb = 0; cb < 4; cb += 2) {
        float r0[32], r1[32];
        const uint32_t src = tmem_lane_addr(sbuf(i), qd * 32, hf * 128 + cb * 32);
        const uint32_t dst = tmem_lane_addr(sbuf(i + 1), qd * 32, hf * 128 + cb * 32);
        ptx::tmem_ld32(src, r0);
        ptx::tmem_ld32(src + 32, r1);
        ptx::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          r0[j] *= d;
          r1[j] *= d;
        }
        ptx::tmem_st32(dst, r0);
        ptx::tmem_st32(dst + 32, r1);
      }
      ptx::tmem_st_wait();
    }
    ptx::tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      ok = ptx::mbar_wait(&bar_full[i & 1], (uint32_t)((i >> 1) & 1));
      if (ok) {
        ptx::tc_fence_after();
        const unsigned char* buf = smem + (i & 1) * buf_bytes;
        const unsigned char* ybuf = buf + nkb * TILE_BYTES;
        for (int half = 0; half < nh; ++half) {
          const unsigned char* xa = buf + (2 * half) * TILE_BYTES;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            ptx::mma_bf16_ss(sbuf(i + 1) + half * 128, desc_mnmajor(xa, ks * 2048, TILE_BYTES),
                             desc_mnmajor(ybuf, ks * 2048, TILE_BYTES), IDESC, 1u);
        }
        ptx::mma_commit(&bar_mma);
      }
    }
    // pass B (overlaps the MMA): store the chunk-start state h_c in bf16.  Each warp stages
    // 32 rows x 32 columns (2 KB, 64-byte swizzle, conflict-free) and lane 0 issues a TMA
    // store; two slots per warp alternate so staging overlaps the previous store.
    if (active && p.states) {
      const int rbase = (b * p.NTb + c) * p.H + h;
#pragma unroll 1
      for (int cb = 0; cb < 4; ++cb) {
        if (!krow_ok || v0 + cb * 32 >= p.V) continue;  // block past K or V (uniform per warp)
        float r[32];
        ptx::tmem_ld32(tmem_lane_addr(sbuf(i), qd * 32, hf * 128 + cb * 32), r);
        ptx::tmem_ld_wait();
        unsigned char* slot = stage_st + (warp * 2 + (cb & 1)) * 2048;
        if (lane == 0) ptx::bulk_wait_read<1>();  // the store that last used this slot has read it
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<uint4*>(slot + sw64(lane, j * 16)) =
              make_uint4(ptx::pack_bf16(r[j * 8 + 0], r[j * 8 + 1]), ptx::pack_bf16(r[j * 8 + 2], r[j * 8 + 3]),
                         ptx::pack_bf16(r[j * 8 + 4], r[j * 8 + 5]), ptx::pack_bf16(r[j * 8 + 6], r[j * 8 + 7]));
        ptx::fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          ptx::tma_store_3d(&maps.st, v0 + cb * 32, hf * 128 + qd * 32, rbase, slot);
          ptx::bulk_commit();
        }
      }
    }
    // a failed wait in thread 0 leaves bar_mma pending: the next wait times out for everyone
  }
  if (ok && (!SEG || n_it > 0)) ok = ptx::mbar_wait(&bar_mma, (uint32_t)((n_it - 1) & 1));
  ptx::tc_fence_after();
  if (ok && active && krow_ok && p.span_decay && vt == 0)
    p.span_decay[((size_t)(sp_ * p.B + b) * p.H + h) * p.K + krow] = dprod;
  if (ok && active && krow_ok && p.fin && (p.fin_mode == 0 || sp_ == p.nspan - 1)) {
    const size_t srow = ((size_t)(sq * p.H + h) * p.K + krow) * p.V + v0 + (p.fin_mode == 0 ? span_off : 0);
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) {
      if (v0 + cb * 32 >= p.V) break;
      float r[32];
      ptx::tmem_ld32(tmem_lane_addr(sbuf(n_it), qd * 32, hf * 128 + cb * 32), r);
      ptx::tmem_ld_wait();
      float4* dst = reinterpret_cast<float4*>(p.fin + srow + cb * 32);
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) dst[j4] = make_float4(r[4 * j4], r[4 * j4 + 1], r[4 * j4 + 2], r[4 * j4 + 3]);
    }
  }
  // drain loads that may still be in flight after an early exit
  if (!ok && tid == 0) {
    ptx::mbar_wait(&bar_full[0], 0);
    ptx::mbar_wait(&bar_full[1], 0);
  }
  if (lane == 0) ptx::bulk_wait<0>();  // this warp's state stores are complete
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) ptx::tmem_dealloc(tmem_base, 512);
}

// Incoming state of every span: H_0 = init (or 0), H_{s+1} = P_s * H_s + E_s (fp32, per
// element; P is per state row).  One thread per 4 consecutive state columns.
__global__ void k_span_prefix(int S, int B, int H, int K, int V, const float* __restrict__ init,
                              const float* __restrict__ P, const float* __restrict__ E, float* __restrict__ Hs) {
  const size_t n4 = (size_t)B * H * K * V / 4;
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n4) return;
  const size_t e = idx * 4, per = (size_t)B * H * K * V;
  const size_t row = e / V;  // (b*H + h)*K + k
  float4 cur = init ? reinterpret_cast<const float4*>(init)[idx] : make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s = 0; s < S; ++s) {
    reinterpret_cast<float4*>(Hs + s * per)[idx] = cur;
    const float d = P[s * (size_t)B * H * K + row];
    const float4 x = reinterpret_cast<const float4*>(E + s * per)[idx];
    cur = make_float4(fmaf(d, cur.x, x.x), fmaf(d, cur.y, x.y), fmaf(d, cur.z, x.z), fmaf(d, cur.w, x.w));
  }
}

// A rank's whole span from the per-span results of a zero-state pass (E, P): its final state
// from a zero state, out = fold over spans (out <- P_s out + E_s, from 0), and optionally its
// total decay dout = prod_s P_s (per state row).  One thread per 4 consecutive state columns.
// The span's own final state from a zero state S = fold over the in-GPU spans of (P, E), and
// (dout) the product of their decays.  PUSH: S, and the decay (push.decay_in if given, else
// the product), also go straight into this rank's slot of every rank's peer-memory region,
// followed by the exchange's epoch flags (p2p.cuh) -- the state computation and its transfer
// to the other GPUs in one kernel.  `out` may then be null.
template <bool PUSH>
__global__ void k_span_total(int S, int B, int H, int K, int V, const float* __restrict__ P,
                             const float* __restrict__ E, float* __restrict__ out, float* __restrict__ dout,
                             p2p::PeerPush push) {
  const size_t n4 = (size_t)B * H * K * V / 4;
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t per = (size_t)B * H * K * V, rows = (size_t)B * H * K;
  uint32_t epoch = 0;
  size_t slot = 0;
  if constexpr (PUSH) {
    epoch = p2p::next_epoch(push.own);
    slot = p2p::slot_offset(epoch, push.world, push.rank, per + rows);
  }
  if (idx < n4) {
    const size_t row = idx * 4 / V;  // (b*H + h)*K + k
    float4 cur = make_float4(0.f, 0.f, 0.f, 0.f);
    float dp = 1.f;
    for (int s = 0; s < S; ++s) {
      const float d = P[s * rows + row];
      const float4 x = reinterpret_cast<const float4*>(E + s * per)[idx];
      cur = make_float4(fmaf(d, cur.x, x.x), fmaf(d, cur.y, x.y), fmaf(d, cur.z, x.z), fmaf(d, cur.w, x.w));
      dp *= d;
    }
    if (out != nullptr) reinterpret_cast<float4*>(out)[idx] = cur;
    const bool row_start = (idx * 4) % V == 0;
    if (dout != nullptr && row_start) dout[row] = dp;
    if constexpr (PUSH) {
      for (int p = 0; p < push.world; ++p) reinterpret_cast<float4*>(p2p::slots(push.regions[p]) + slot)[idx] = cur;
      if (row_start) {
        const float dv = push.decay_in != nullptr ? push.decay_in[row] : dp;
        for (int p = 0; p < push.world; ++p) p2p::slots(push.regions[p])[slot + per + row] = dv;
      }
    }
  }
  if constexpr (PUSH) p2p::signal(push.regions, push.own, push.world, push.rank, epoch);
}

// ===========================================================================
// k_out: persistent GEMM  out[128 x 128] = X[128 x K] S[K x 128] + A'[128 x 128] Y[128 x 128]
// per item (batch, chunk, head, V tile).  grid = #SMs, 192 threads.
//   fwd: X = qhat, S = h_c, A' = A (K-major), Y = v, out = o
//   bwd: X = kdec, S = dh_c, A' = A^T (M-major), Y = do, out = dv
// ===========================================================================
constexpr int OUT_STAGES = 6;
constexpr int STAGE_BYTES = 2 * TILE_BYTES;  // A tile 16 KB + B tile 16 KB

struct OutParams {
  int B, T, H, K, V, NTb, trans_a;
  bf16* out;  // [B, T, H, V]
};

struct OutMaps {
  CUtensorMap x;   // [B,T,H,K] box (64,1,128,1)
  CUtensorMap s;   // [B*NTb*H, K, V] box (64,64,1)
  CUtensorMap a;   // A [B,T,H,128]: fwd box (64,1,128,1); bwd box (64,1,64,1)
  CUtensorMap y;   // [B,T,H,V] box (64,1,64,1)
  CUtensorMap o;   // output [B,T,H,V] box (64,1,128,1), store
};

__global__ void __launch_bounds__(192, 1) k_out(const __grid_constant__ OutMaps maps, OutParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[OUT_STAGES], empty[OUT_STAGES], accf[2], acce[2];
  __shared__ uint32_t tmem_base;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nvt = (p.V + BV - 1) / BV;
  const int items = p.B * p.NTb * p.H * nvt;
  const int nkb = p.K / 64 + 2;

  if (warp == 0) {
    ptx::tmem_alloc(&tmem_base, 256);
    ptx::tmem_relinquish();
  }
  if (tid == 32) {
    for (int s = 0; s < OUT_STAGES; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&accf[a], 1);
      ptx::mbar_init(&acce[a], 4);
    }
    ptx::fence_mbar_init();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tacc = tmem_base;

  auto decode = [&](int it, int& b, int& c, int& h, int& vt) {
    vt = it % nvt;
    int r = it / nvt;
    h = r % p.H;
    r /= p.H;
    c = r % p.NTb;
    b = r / p.NTb;
  };

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      uint32_t n = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
        int b, c, h, vt;
        decode(it, b, c, h, vt);
        const int row0 = c * BT, v0 = vt * BV;
        const int srow = (b * p.NTb + c) * p.H + h;
        for (int kb = 0; kb < nkb; ++kb, ++n) {
          const int s = n % OUT_STAGES;
          ok = ptx::mbar_wait(&empty[s], ((n / OUT_STAGES) & 1) ^ 1);
          if (!ok) break;
          unsigned char* at = smem + s * STAGE_BYTES;
          unsigned char* bt = at + TILE_BYTES;
          ptx::mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          if (kb < p.K / 64) {
            ptx::tma_load_4d(at, &maps.x, kb * 64, h, row0, b, &full[s]);
            ptx::tma_load_3d(bt, &maps.s, v0, kb * 64, srow, &full[s]);
            ptx::tma_load_3d(bt + TILE_BYTES / 2, &maps.s, v0 + 64, kb * 64, srow, &full[s]);
          } else {
            const int j = kb - p.K / 64;  // 64-token block of the intra part
            if (!p.trans_a) {
              ptx::tma_load_4d(at, &maps.a, j * 64, h, row0, b, &full[s]);
            } else {
              ptx::tma_load_4d(at, &maps.a, 0, h, row0 + j * 64, b, &full[s]);
              ptx::tma_load_4d(at + TILE_BYTES / 2, &maps.a, 64, h, row0 + j * 64, b, &full[s]);
            }
            ptx::tma_load_4d(bt, &maps.y, v0, h, row0 + j * 64, b, &full[s]);
            ptx::tma_load_4d(bt + TILE_BYTES / 2, &maps.y, v0 + 64, h, row0 + j * 64, b, &full[s]);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      uint32_t n = 0, t = 0;
      bool ok = true;
      const uint32_t ID_K = ptx::idesc_bf16(128, 128, false, true);
      const uint32_t ID_M = ptx::idesc_bf16(128, 128, true, true);
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x, ++t) {
        const int ab = t & 1;
        ok = ptx::mbar_wait(&acce[ab], ((t >> 1) & 1) ^ 1);
        if (!ok) break;
        ptx::tc_fence_after();
        const uint32_t d = tacc + ab * 128;
        for (int kb = 0; kb < nkb; ++kb, ++n) {
          const int s = n % OUT_STAGES;
          ok = ptx::mbar_wait(&full[s], (n / OUT_STAGES) & 1);
          if (!ok) break;
          ptx::tc_fence_after();
          const unsigned char* at = smem + s * STAGE_BYTES;
          const unsigned char* bt = at + TILE_BYTES;
          const bool mn = p.trans_a && kb >= p.K / 64;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint64_t ad = mn ? desc_mnmajor(at, ks * 2048, TILE_BYTES / 2) : desc_kmajor(at, ks * 32);
            ptx::mma_bf16_ss(d, ad, desc_mnmajor(bt, ks * 2048, TILE_BYTES / 2), mn ? ID_M : ID_K,
                             (kb | ks) ? 1u : 0u);
          }
          ptx::mma_commit(&empty[s]);
        }
        if (ok) ptx::mma_commit(&accf[ab]);
      }
    }
  } else {  // epilogue warps 2..5: lane quadrant (warp & 3)
    const int qd = warp & 3;
    const int i = qd * 32 + lane;
    unsigned char* stg = smem + OUT_STAGES * STAGE_BYTES;  // [128][128] bf16 as two swizzled [128][64] tiles
    const bool leader = (warp == 2 && lane == 0);
    uint32_t t = 0;
    for (int it = blockIdx.x; it < items; it += gridDim.x, ++t) {
      int b, c, h, vt;
      decode(it, b, c, h, vt);
      const int ab = t & 1;
      const bool got = ptx::mbar_wait(&accf[ab], (t >> 1) & 1);
      if (leader) ptx::bulk_wait_read<0>();  // the previous item's store has read the staging tiles
      if (!ptx::bar_and(1, 128, got)) break;  // all four warps stop together after a timeout
      ptx::tc_fence_after();
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {
        float r[32];
        ptx::tmem_ld32(tmem_lane_addr(tacc, qd * 32, ab * 128 + cb * 32), r);
        ptx::tmem_ld_wait();
        unsigned char* tile = stg + (cb >> 1) * TILE_BYTES;
#pragma unroll
        for (int j8 = 0; j8 < 4; ++j8)
          *reinterpret_cast<uint4*>(tile + ptx::sw128(i, (cb & 1) * 64 + j8 * 16)) =
              make_uint4(ptx::pack_bf16(r[j8 * 8 + 0], r[j8 * 8 + 1]), ptx::pack_bf16(r[j8 * 8 + 2], r[j8 * 8 + 3]),
                         ptx::pack_bf16(r[j8 * 8 + 4], r[j8 * 8 + 5]), ptx::pack_bf16(r[j8 * 8 + 6], r[j8 * 8 + 7]));
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&acce[ab]);  // TMEM accumulator free for the next item
      ptx::fence_async_smem();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (leader) {  // rows past T are clipped by the tensor map
        ptx::tma_store_4d(&maps.o, vt * BV, h, c * BT, b, stg);
        ptx::tma_store_4d(&maps.o, vt * BV + 64, h, c * BT, b, stg + TILE_BYTES);
        ptx::bulk_commit();
      }
    }
    if (leader) ptx::bulk_wait<0>();
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) ptx::tmem_dealloc(tacc, 256);
}

// ===========================================================================
// k_scan_out: the state scan fused with the chunk-output GEMM.  grid (V/128, H, B*nspan)
// (or (V/128, H, N) for a padded varlen problem), 384 threads, one CTA per SM.
//   fwd: h_{c+1} = D_c h_c + kdec_c^T v_c;   o_c  = qhat_c h_c + A_c v_c
//   bwd: dh_{c-1} = D_c dh_c + qhat_c^T do_c; dv_c = kdec_c dh_c + A_c^T do_c
// The chunk-start state is read from TMEM once per chunk: its bf16 copy is written into
// shared memory in the 128-byte-swizzled layout of the B operand of the output GEMM, so
// the output GEMM never reads the states back from HBM (the separate k_out does).  The
// copy and the output tiles go to HBM through ordinary coalesced stores (whole rows per
// warp instruction), not through TMA stores: the CTA's TMA stream is bounded by the bytes
// its ring keeps in flight (about 95 GB/s for 96 KB), which the operand loads (224 KB per
// chunk at K = 256) already need (TMA stores measured 164 us per launch at config 3
// against 152 us).
//   warp 0      TMA producer: per chunk the y tile (v or do; 2 slots) and a ring of
//               32 KB stages: the A tiles, output-side x tiles (qhat / kdec), scan-side x tiles
//   warp 1      MMA issuer: o = A' Y (8 MMAs; needs no state, so it overlaps the state pass),
//               then o += X h (K/64 x 4) and the scan (8 per state half)
//   warps 4-11  per chunk: wait for the chunk's MMAs, scale the state in TMEM by D and
//               write its bf16 copy (the next chunk's operand), store the copy's rows;
//               then drain the previous chunk's output accumulator into its (now free)
//               y slot and store it
// TMEM: state [K rows as 128-lane halves x 128 columns] fp32 in columns [0, 256), two
// output accumulators [128 tokens x 128] in [256, 384) and [384, 512).
// ===========================================================================
struct FusedMaps {
  CUtensorMap sx;  // scan-side x: fwd kdec, bwd qhat; [B,T,H,K] box (64,1,128,1)
  CUtensorMap y;   // fwd v, bwd do; [B,T,H,V] box (64,1,128,1)
  CUtensorMap ox;  // output-side x: fwd qhat, bwd kdec; box (64,1,128,1)
  CUtensorMap a;   // A [B,T,H,128]: fwd box (64,1,128,1), bwd box (64,1,64,1)
  bf16* out;       // output [B, T, H, V] (fwd o, bwd dv): bf16, or fp16 when out_f16
  int out_f16;     // selects the k_scan_out instantiation
};

constexpr int FO_THREADS = 384;
constexpr uint32_t FO_STAGE = 2 * TILE_BYTES;  // 32 KB
__host__ __device__ constexpr int fo_stages(int K) { return K == 256 ? 3 : 4; }
// shared memory of k_scan_out: the bf16 state copy (K padded to whole 128-row state halves),
// two y slots and the ring
static size_t fo_smem(int K) {
  const size_t Kp = (size_t)(K + 127) / 128 * 128;
  return Kp * 256 + 2 * (size_t)FO_STAGE + (size_t)fo_stages(K) * FO_STAGE + 1024;
}

template <bool SEG, bool F16>  // F16: the output (o / dv) is stored as fp16, bf16 otherwise
__global__ void __launch_bounds__(FO_THREADS, 1) k_scan_out(const __grid_constant__ FusedMaps maps, ScanParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nh = (p.K + 127) / 128;   // state halves; K = 64 uses half of one (loads past K read zeros)
  const int nxs = nh;                 // output-side x stages per chunk (two 64-column tiles each)
  const int S = fo_stages(p.K);  // ring stages
  const uint32_t half_bytes = (uint32_t)nh * 128 * 128;  // one 64-column half of the bf16 state copy (padded K rows)
  unsigned char* hs = smem;                         // bf16 state copy: 2 halves [K rows][64 cols]
  unsigned char* yslot0 = smem + 2 * half_bytes;    // 2 slots x [128 rows][128 cols] (two 16 KB tiles)
  unsigned char* ring = yslot0 + 2 * FO_STAGE;
  __shared__ __align__(8) uint64_t full[4], empty[4], y_full[2], y_empty[2], acc_empty[2], bar_pass, bar_chunk,
      bar_done;
  __shared__ uint32_t tmem_base;

  const int vt = blockIdx.x, h = blockIdx.y;
  const int b = SEG ? 0 : blockIdx.z / p.nspan, sp_ = SEG ? 0 : blockIdx.z % p.nspan;
  const int sq = SEG ? (int)blockIdx.z : b;
  const int v0 = vt * BV;
  const int i0 = SEG ? p.blk_off[blockIdx.z] : sp_ * p.span_len;
  const int n_it = SEG ? p.blk_off[blockIdx.z + 1] - i0 : min(p.span_len, p.NTb - i0);
  const size_t span_off = (size_t)sp_ * p.B * p.H * p.K * p.V;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (warp == 0) {
    ptx::tmem_alloc(&tmem_base, 512);
    ptx::tmem_relinquish();
  }
  if (tid == 32) {
    for (int s = 0; s < 4; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(&y_full[s], 1);
      ptx::mbar_init(&y_empty[s], 8);    // the eight epilogue warps, after they read their output rows
      ptx::mbar_init(&acc_empty[s], 8);  // the eight epilogue warps, after their TMEM reads
    }
    ptx::mbar_init(&bar_pass, 8);
    ptx::mbar_init(&bar_chunk, 1);
    ptx::mbar_init(&bar_done, 1);
    ptx::fence_mbar_init();
  }
  auto chunk_of = [&](int i) {
    if constexpr (SEG) return p.reverse ? i0 + n_it - 1 - i : i0 + i;
    else return p.reverse ? p.NTb - 1 - (i0 + i) : i0 + i;
  };
  auto yslot = [&](int i) { return yslot0 + (i & 1) * FO_STAGE; };
  auto oacc = [&](int i) { return tmem_base + 256u + (uint32_t)((i & 1) * 128); };

  // pass warps: state half hf, TMEM lane quadrant qd
  const int pw = warp - 4;
  const int hf = pw >> 2, qd = warp & 3;
  const int krow = hf * 128 + qd * 32 + lane;
  const bool pass_warp = warp >= 4;
  const bool active = pass_warp && hf < nh;
  const bool krow_ok = krow < p.K;  // uniform per warp
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (active) {  // initial state -> TMEM
    const size_t srow = ((size_t)(sq * p.H + h) * p.K + krow) * p.V + v0;
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) {
      float r[32];
#pragma unroll
      for (int j = 0; j < 32; ++j)
        r[j] = (p.init && krow_ok && v0 + cb * 32 + j < p.V) ? p.init[span_off + srow + cb * 32 + j] : 0.f;
      ptx::tmem_st32(tmem_lane_addr(tmem_base, qd * 32, hf * 128 + cb * 32), r);
    }
    ptx::tmem_st_wait();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      uint32_t n = 0;
      int ny = 0;  // y tiles armed
      bool ok = true;
      for (int i = 0; i < n_it && ok; ++i) {
        const int c = chunk_of(i), row0 = c * BT;
        const int nst = nxs + 1 + nh;
        for (int e = 0; e < nst && ok; ++e, ++n) {
          if (e == 0) {  // the y tile is first needed with the A stage
            ok = ptx::mbar_wait(&y_empty[i & 1], (uint32_t)(((i >> 1) & 1) ^ 1));
            if (!ok) break;
            ptx::mbar_arrive_expect_tx(&y_full[i & 1], FO_STAGE);
            ptx::tma_load_4d(yslot(i), &maps.y, v0, h, row0, b, &y_full[i & 1]);
            ptx::tma_load_4d(yslot(i) + TILE_BYTES, &maps.y, v0 + 64, h, row0, b, &y_full[i & 1]);
            ++ny;
          }
          const int s = (int)(n % (uint32_t)S);
          ok = ptx::mbar_wait(&empty[s], ((n / S) & 1) ^ 1);
          if (!ok) break;
          unsigned char* st = ring + s * FO_STAGE;
          ptx::mbar_arrive_expect_tx(&full[s], FO_STAGE);
          if (e >= 1 && e <= nxs) {  // output-side x: 64-column tiles 2x, 2x+1, x = e - 1
            ptx::tma_load_4d(st, &maps.ox, (2 * (e - 1)) * 64, h, row0, b, &full[s]);
            ptx::tma_load_4d(st + TILE_BYTES, &maps.ox, (2 * (e - 1) + 1) * 64, h, row0, b, &full[s]);
          } else if (e == 0) {  // A: two 64-token blocks
            for (int j = 0; j < 2; ++j) {
              if (!p.reverse) {
                ptx::tma_load_4d(st + j * TILE_BYTES, &maps.a, j * 64, h, row0, b, &full[s]);
              } else {
                ptx::tma_load_4d(st + j * TILE_BYTES, &maps.a, 0, h, row0 + j * 64, b, &full[s]);
                ptx::tma_load_4d(st + j * TILE_BYTES + TILE_BYTES / 2, &maps.a, 64, h, row0 + j * 64, b, &full[s]);
              }
            }
          } else {  // scan-side x: the two 64-column tiles of state half (e - nxs - 1)
            const int half = e - nxs - 1;
            ptx::tma_load_4d(st, &maps.sx, half * 128, h, row0, b, &full[s]);
            ptx::tma_load_4d(st + TILE_BYTES, &maps.sx, half * 128 + 64, h, row0, b, &full[s]);
          }
        }
      }
      // loads still in flight after an early exit land before the CTA leaves: wait for the
      // last armed phase of every stage and y slot
      const uint32_t armed = n;
      for (uint32_t m = armed > (uint32_t)S ? armed - S : 0; m < armed; ++m)
        ptx::mbar_wait(&full[m % S], (m / S) & 1);
      for (int m = ny > 2 ? ny - 2 : 0; m < ny; ++m) ptx::mbar_wait(&y_full[m & 1], (uint32_t)((m >> 1) & 1));
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      uint32_t n = 0;
      bool ok = true, any = false;
      const uint32_t ID_K = ptx::idesc_bf16(128, 128, false, true);
      const uint32_t ID_M = ptx::idesc_bf16(128, 128, true, true);
      for (int i = 0; i < n_it && ok; ++i) {
        // o = A' Y does not need the state: it runs while the pass warps prepare chunk i
        ok = ptx::mbar_wait(&acc_empty[i & 1], (uint32_t)(((i >> 1) & 1) ^ 1)) &&
             ptx::mbar_wait(&y_full[i & 1], (uint32_t)((i >> 1) & 1));
        if (!ok) break;
        ptx::tc_fence_after();
        any = true;
        const uint32_t dacc = oacc(i);
        const unsigned char* ys = yslot(i);
        {
          const int s = (int)(n % (uint32_t)S);
          ok = ptx::mbar_wait(&full[s], (n / S) & 1);
          if (!ok) break;
          ptx::tc_fence_after();
          const unsigned char* st = ring + s * FO_STAGE;
          for (int j = 0; j < 2; ++j) {
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              const uint64_t ad = p.reverse ? desc_mnmajor(st + j * TILE_BYTES, ks * 2048, TILE_BYTES / 2)
                                            : desc_kmajor(st + j * TILE_BYTES, ks * 32);
              ptx::mma_bf16_ss(dacc, ad, desc_mnmajor(ys, (uint32_t)(j * 64 + ks * 16) * 128, TILE_BYTES),
                               p.reverse ? ID_M : ID_K, (j | ks) ? 1u : 0u);
            }
          }
          ptx::mma_commit(&empty[s]);
          ++n;
        }
        ok = ptx::mbar_wait(&bar_pass, (uint32_t)(i & 1));  // scaled state and its bf16 copy are ready
        if (!ok) break;
        ptx::tc_fence_after();
        // o += X[128 x K] (K-major tiles) x h_c[K x 128] (bf16 copy, MN-major)
        for (int e = 0; e < nxs && ok; ++e, ++n) {
          const int s = (int)(n % (uint32_t)S);
          ok = ptx::mbar_wait(&full[s], (n / S) & 1);
          if (!ok) break;
          ptx::tc_fence_after();
          const unsigned char* st = ring + s * FO_STAGE;
          for (int t = 0; t < 2; ++t) {
            const int kb = 2 * e + t;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              ptx::mma_bf16_ss(dacc, desc_kmajor(st + t * TILE_BYTES, ks * 32),
                               desc_mnmajor(hs, (uint32_t)(kb * 64 + ks * 16) * 128, half_bytes), ID_K, 1u);
          }
          ptx::mma_commit(&empty[s]);
        }
        if (!ok) break;
        // state scan: state[half] += X_half^T Y (X M-major, Y N-major, contraction over tokens)
        for (int half = 0; half < nh && ok; ++half, ++n) {
          const int s = (int)(n % (uint32_t)S);
          ok = ptx::mbar_wait(&full[s], (n / S) & 1);
          if (!ok) break;
          ptx::tc_fence_after();
          const unsigned char* st = ring + s * FO_STAGE;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            ptx::mma_bf16_ss(tmem_base + half * 128, desc_mnmajor(st, ks * 2048, TILE_BYTES),
                             desc_mnmajor(ys, ks * 2048, TILE_BYTES), ID_M, 1u);
          ptx::mma_commit(&empty[s]);
        }
        if (ok) ptx::mma_commit(&bar_chunk);  // state, output accumulator, y slot and state copy are done
      }
      if (any) {  // every issued MMA has completed before TMEM is released
        ptx::mma_commit(&bar_done);
        ptx::mbar_wait(&bar_done, 0);
      }
    }
  } else if (pass_warp) {
    // epilogue of chunk j: output accumulator -> bf16 -> y slot of chunk j -> HBM.  Warp
    // (hf, qd) owns output rows qd*32 .. +31, columns hf*64 .. +63: it writes them into the
    // slot from TMEM (a row per lane) and reads them back four rows of 128 bytes per
    // instruction for coalesced stores.
    auto epilogue = [&](int j) {
      const int c = chunk_of(j);
      unsigned char* tile = yslot(j) + hf * TILE_BYTES;  // output columns hf*64 .. +63
      const int t = qd * 32 + lane;                      // token row of this thread
#pragma unroll
      for (int cb = 0; cb < 2; ++cb) {
        float r[32];
        ptx::tmem_ld32(tmem_lane_addr(oacc(j), qd * 32, hf * 64 + cb * 32), r);
        ptx::tmem_ld_wait();
        constexpr bool f16 = F16;
#pragma unroll
        for (int j8 = 0; j8 < 4; ++j8)
          *reinterpret_cast<uint4*>(tile + ptx::sw128(t, cb * 64 + j8 * 16)) =
              make_uint4(ptx::pack16(r[j8 * 8 + 0], r[j8 * 8 + 1], f16), ptx::pack16(r[j8 * 8 + 2], r[j8 * 8 + 3], f16),
                         ptx::pack16(r[j8 * 8 + 4], r[j8 * 8 + 5], f16), ptx::pack16(r[j8 * 8 + 6], r[j8 * 8 + 7], f16));
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&acc_empty[j & 1]);
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int rr = qd * 32 + 4 * it + (lane >> 3), row = c * BT + rr;
        const uint4 x = *reinterpret_cast<const uint4*>(tile + ptx::sw128(rr, (lane & 7) * 16));
        if (row < p.T && v0 + hf * 64 < p.V)
          *reinterpret_cast<uint4*>(maps.out + (((size_t)b * p.T + row) * p.H + h) * p.V + v0 + hf * 64 +
                                    (lane & 7) * 8) = x;
      }
      ptx::fence_async_smem();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&y_empty[j & 1]);
    };
    auto decay_of = [&](int i) {
      return active && krow_ok && i < n_it
                 ? __ldg(p.D + ((size_t)(b * p.NTb + chunk_of(i)) * p.H + h) * p.K + krow)
                 : 1.f;
    };
    bool ok = true;
    float d_next = decay_of(0);
    for (int i = 0; i < n_it; ++i) {
      const int c = chunk_of(i);
      const float d = d_next;
      d_next = decay_of(i + 1);
      if (i > 0) {
        ok = ptx::bar_and(1, 256, ptx::mbar_wait(&bar_chunk, (uint32_t)((i - 1) & 1)));
        ptx::tc_fence_after();
        if (!ok) break;
      }
      if (active) {
#pragma unroll
        for (int cb = 0; cb < 4; ++cb) {
          float r[32];
          const uint32_t ta = tmem_lane_addr(tmem_base, qd * 32, hf * 128 + cb * 32);
          ptx::tmem_ld32(ta, r);
          ptx::tmem_ld_wait();
          unsigned char* dst = hs + (cb >> 1) * half_bytes;
#pragma unroll
          for (int j8 = 0; j8 < 4; ++j8)
            *reinterpret_cast<uint4*>(dst + ptx::sw128(krow, (cb & 1) * 64 + j8 * 16)) =
                make_uint4(ptx::pack_bf16(r[j8 * 8 + 0], r[j8 * 8 + 1]), ptx::pack_bf16(r[j8 * 8 + 2], r[j8 * 8 + 3]),
                           ptx::pack_bf16(r[j8 * 8 + 4], r[j8 * 8 + 5]), ptx::pack_bf16(r[j8 * 8 + 6], r[j8 * 8 + 7]));
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] *= d;
          ptx::tmem_st32(ta, r);
        }
        ptx::tmem_st_wait();
      }
      ptx::fence_async_smem();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bar_pass);
      if (active && p.states) {  // this warp's 32 state rows, two rows (2 x 256 B) per instruction
        const size_t rbase = ((size_t)(b * p.NTb + c) * p.H + h) * p.K;
        const int hb = (lane >> 3) & 1, c16 = lane & 7;
#pragma unroll 4
        for (int it = 0; it < 16; ++it) {
          const int r = hf * 128 + qd * 32 + 2 * it + (lane >> 4);
          const uint4 x = *reinterpret_cast<const uint4*>(hs + hb * half_bytes + ptx::sw128(r, c16 * 16));
          if (r < p.K && v0 + hb * 64 < p.V)
            *reinterpret_cast<uint4*>(p.states + (rbase + r) * p.V + v0 + hb * 64 + c16 * 8) = x;
        }
      }
      if (i > 0) epilogue(i - 1);
    }
    if (ok && n_it > 0) {
      ok = ptx::bar_and(1, 256, ptx::mbar_wait(&bar_chunk, (uint32_t)((n_it - 1) & 1)));
      ptx::tc_fence_after();
      if (ok) epilogue(n_it - 1);
    }
    if (ok && active && krow_ok && p.fin && (p.fin_mode == 0 || sp_ == p.nspan - 1)) {
      const size_t srow = ((size_t)(sq * p.H + h) * p.K + krow) * p.V + v0 + (p.fin_mode == 0 ? span_off : 0);
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {
        if (v0 + cb * 32 >= p.V) break;
        float r[32];
        ptx::tmem_ld32(tmem_lane_addr(tmem_base, qd * 32, hf * 128 + cb * 32), r);
        ptx::tmem_ld_wait();
        float4* dst = reinterpret_cast<float4*>(p.fin + srow + cb * 32);
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4) dst[j4] = make_float4(r[4 * j4], r[4 * j4 + 1], r[4 * j4 + 2], r[4 * j4 + 3]);
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) ptx::tmem_dealloc(tmem_base, 512);
}

// ===========================================================================
// k_dqk: dq, dk, dg of one (batch, chunk, head, 64-wide K tile).  grid (K/64, NTb, B*H),
// 256 threads, two CTAs per SM (256 TMEM columns and ~100 KB shared memory each), so one
// CTA's epilogue runs while the other streams its operands.
//   dA      = scale tril(do v^T)                            (M1, contraction over V)
//   dqi     = do h_c^T            dki = v dh_c^T            (M2, M3, contraction over V)
//   dq      = e^{G-Gm} (dA ktil + scale e^{Gm} dqi)         (M4 = dA x ktil,  ktil = k e^{Gm-G})
//   dk      = e^{Gm-G} (dA^T qtil + e^{GL-Gm} dki)          (M5 = dA^T x qtil, qtil = q e^{G-Gm})
//   dg      = revcumsum_t(q dq - k dk) + e^{GL} sum_v(h_c dh_c) + sum_t(e^{GL-G} dki k)
//             with q dq = qtil (M4 + scale e^{Gm} dqi) and k dk = ktil (M5 + e^{GL-Gm} dki)
// (reference chunk_gla_bwd_fused_kernel tops/ops/gla/chunk.py:1423-1479 and the
//  _ref functions :504-743).
// During the V stream warp 0 is the TMA producer, warp 1 the MMA issuer and warps 4-7
// sum h*dh over V; the 2-stage ring is released by the MMA commit plus those four warps.
// After the stream stage 0 holds g -> G -> dg (fp32, in place) and q -> qtil -> dq,
// stage 1 holds k -> ktil -> dk and the bf16 dA; the outputs leave by TMA stores.
// dA is the same for every K tile of a chunk; the do/v re-reads of the K tiles of one
// chunk (adjacent CTAs) are served by L2.
// ===========================================================================
struct DqkParams {
  int B, T, H, K, V, NTb;
  float scale;
  bf16* dq; bf16* dk; float* dg;
};

struct DqkMaps {
  CUtensorMap dO, v;   // [B,T,H,V] bf16 box (64,1,128,1)
  CUtensorMap hs, dhs; // [B*NTb*H, K, V] bf16 box (64,64,1)
  CUtensorMap g, dg;   // [B,T,H,K] fp32 box (32,1,128,1); dg is a store map
  CUtensorMap q, k;    // [B,T,H,K] bf16 box (64,1,128,1)
  CUtensorMap dq, dk;  // [B,T,H,K] bf16 box (64,1,128,1), stores
};

constexpr uint32_t DQK_STG = 3 * TILE_BYTES;  // do 16K, v 16K, h 8K, dh 8K

// Sum of 16 per-lane values over the 32 lanes of a warp, for 16 columns at once: a
// transposing butterfly (each step keeps half the columns and adds the partner's
// other half).  Returns the full sum of column dqk_red_col(lane) (valid in every lane).
__device__ __forceinline__ int dqk_red_col(int lane) {
  return ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
}
__device__ __forceinline__ float dqk_reduce16(const float (&v)[16], int lane) {
  float r8[8], r4[4], r2[2];
  const bool u16 = lane & 16, u8 = lane & 8, u4 = lane & 4, u2 = lane & 2;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float keep = u16 ? v[j + 8] : v[j], send = u16 ? v[j] : v[j + 8];
    r8[j] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float keep = u8 ? r8[j + 4] : r8[j], send = u8 ? r8[j] : r8[j + 4];
    r4[j] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const float keep = u4 ? r4[j + 2] : r4[j], send = u4 ? r4[j] : r4[j + 2];
    r2[j] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  const float keep = u2 ? r2[1] : r2[0], send = u2 ? r2[0] : r2[1];
  const float r1 = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  return r1 + __shfl_xor_sync(0xffffffffu, r1, 1);
}

template <bool F16>  // q, k, dq, dk stored as fp16 (do, v and the states are bf16 either way)
__global__ void __launch_bounds__(256, 2) k_dqk(const __grid_constant__ DqkMaps maps, DqkParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* Gs = smem;                           // two fp32 [128][32] tiles: g -> G -> dg
  unsigned char* qtl = smem + 2 * TILE_BYTES;         // q -> qtil -> dq staging
  unsigned char* ktl = smem + DQK_STG;                // k -> ktil -> dk staging
  unsigned char* dAs = smem + DQK_STG + TILE_BYTES;   // dA bf16 [128][128] as two [128][64] tiles
  __shared__ __align__(16) float cS[64], cL[64], cGL[64];  // scale e^{Gm}, e^{GL-Gm}, e^{GL} per column
  __shared__ float hdh2[2][64], colsum[4][64], segs[4][64];
  __shared__ __align__(8) uint64_t full[2], empty[2], bar_g, bar_q, bar_k, bar_mma;
  __shared__ uint32_t tmem_base;

  const int kt = blockIdx.x, c = blockIdx.y, b = blockIdx.z / p.H, h = blockIdx.z % p.H;
  const int k0 = kt * 64, row0 = c * BT;
  const int srow = (b * p.NTb + c) * p.H + h;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nvb = p.V < 128 ? 2 : p.V / 64;  // even: V is 64 (second block read as zeros) or a multiple of 128

  if (warp == 0) {
    ptx::tmem_alloc(&tmem_base, 256);
    ptx::tmem_relinquish();
  }
  if (tid == 32) {
    for (int s_ = 0; s_ < 2; ++s_) {
      ptx::mbar_init(&full[s_], 1);
      ptx::mbar_init(&empty[s_], 1 + 4);  // MMA commit + 4 reducer warps
    }
    ptx::mbar_init(&bar_g, 1);
    ptx::mbar_init(&bar_q, 1);
    ptx::mbar_init(&bar_k, 1);
    ptx::mbar_init(&bar_mma, 1);
    ptx::fence_mbar_init();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tM1 = tmem_base, tM2 = tmem_base + 128, tM3 = tmem_base + 192;
  bool ok = true;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      for (int vb = 0; vb < nvb && ok; ++vb) {
        const int st = vb & 1;
        if (vb >= 2) ok = ptx::mbar_wait(&empty[st], (uint32_t)(((vb >> 1) - 1) & 1));
        if (!ok) break;
        unsigned char* sp = smem + st * DQK_STG;
        ptx::mbar_arrive_expect_tx(&full[st], DQK_STG);
        ptx::tma_load_4d(sp, &maps.dO, vb * 64, h, row0, b, &full[st]);
        ptx::tma_load_4d(sp + TILE_BYTES, &maps.v, vb * 64, h, row0, b, &full[st]);
        ptx::tma_load_3d(sp + 2 * TILE_BYTES, &maps.hs, vb * 64, k0, srow, &full[st]);
        ptx::tma_load_3d(sp + 2 * TILE_BYTES + TILE_BYTES / 2, &maps.dhs, vb * 64, k0, srow, &full[st]);
      }
      // stage 0 is last used by V block nvb-2, stage 1 by nvb-1
      if (ok) ok = ptx::mbar_wait(&empty[0], (uint32_t)(((nvb - 2) >> 1) & 1));
      if (ok) {
        ptx::mbar_arrive_expect_tx(&bar_g, 2 * TILE_BYTES);
        ptx::tma_load_4d(Gs, &maps.g, k0, h, row0, b, &bar_g);
        ptx::tma_load_4d(Gs + TILE_BYTES, &maps.g, k0 + 32, h, row0, b, &bar_g);
        ptx::mbar_arrive_expect_tx(&bar_q, TILE_BYTES);
        ptx::tma_load_4d(qtl, &maps.q, k0, h, row0, b, &bar_q);
      }
      if (ok) ok = ptx::mbar_wait(&empty[1], (uint32_t)(((nvb - 1) >> 1) & 1));
      if (ok) {
        ptx::mbar_arrive_expect_tx(&bar_k, TILE_BYTES);
        ptx::tma_load_4d(ktl, &maps.k, k0, h, row0, b, &bar_k);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer for the V stream ----------------
    if (lane == 0) {
      constexpr uint32_t ID_N128 = ptx::idesc_bf16(128, 128, false, false);
      constexpr uint32_t ID_N64 = ptx::idesc_bf16(128, 64, false, false);
      for (int vb = 0; vb < nvb && ok; ++vb) {
        const int st = vb & 1;
        ok = ptx::mbar_wait(&full[st], (uint32_t)((vb >> 1) & 1));
        if (!ok) break;
        ptx::tc_fence_after();
        const unsigned char* sp = smem + st * DQK_STG;
        const unsigned char* th = sp + 2 * TILE_BYTES;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint32_t acc = (vb | ks) ? 1u : 0u;
          ptx::mma_bf16_ss(tM1, desc_kmajor(sp, ks * 32), desc_kmajor(sp + TILE_BYTES, ks * 32), ID_N128, acc);
          ptx::mma_bf16_ss(tM2, desc_kmajor(sp, ks * 32), desc_kmajor(th, ks * 32), ID_N64, acc);
          ptx::mma_bf16_ss(tM3, desc_kmajor(sp + TILE_BYTES, ks * 32), desc_kmajor(th + TILE_BYTES / 2, ks * 32),
                           ID_N64, acc);
        }
        ptx::mma_commit(&empty[st]);
      }
      if (ok) ptx::mma_commit(&bar_mma);
    }
  } else if (warp >= 4) {
    // ---------------- sum_v h*dh of the 64 state rows: 2 threads per row ----------------
    const int hr = (tid - 128) & 63, hv = (tid - 128) >> 6;
    float acc = 0.f;
    for (int vb = 0; vb < nvb && ok; ++vb) {
      const int st = vb & 1;
      ok = ptx::mbar_wait(&full[st], (uint32_t)((vb >> 1) & 1));
      if (!ok) break;
      const unsigned char* th = smem + st * DQK_STG + 2 * TILE_BYTES;
      const unsigned char* tdh = th + TILE_BYTES / 2;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t off = ptx::sw128(hr, (hv * 4 + u) * 16);
        const uint4 a = *reinterpret_cast<const uint4*>(th + off);
        const uint4 d = *reinterpret_cast<const uint4*>(tdh + off);
        const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
        const __nv_bfloat162* d2 = reinterpret_cast<const __nv_bfloat162*>(&d);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 af = __bfloat1622float2(a2[e]), df = __bfloat1622float2(d2[e]);
          acc = fmaf(af.x, df.x, fmaf(af.y, df.y, acc));
        }
      }
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&empty[st]);
    }
    hdh2[hv][hr] = acc;
  }

  // ---------------- all threads: dA from M1 once the V-stream MMAs are done ----------------
  __syncthreads();
  if (ok) ok = ptx::mbar_wait(&bar_mma, 0);
  ptx::tc_fence_after();
  const int qd = warp & 3, ch = warp >> 2;
  const int i = qd * 32 + lane;  // TMEM lane = token row of this thread
  if (ok) {
    // dA = scale tril(M1) -> bf16 [i][j]; this warp writes columns ch*64.. (tile ch)
#pragma unroll
    for (int cb = 0; cb < 2; ++cb) {
      float r[32];
      ptx::tmem_ld32(tmem_lane_addr(tM1, qd * 32, ch * 64 + cb * 32), r);
      ptx::tmem_ld_wait();
      unsigned char* stg = dAs + ch * TILE_BYTES;
#pragma unroll
      for (int j4 = 0; j4 < 4; ++j4) {
        uint32_t w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j0 = ch * 64 + cb * 32 + j4 * 8 + 2 * u;
          w[u] = ptx::pack_bf16((j0 <= i) ? r[j4 * 8 + 2 * u] * p.scale : 0.f,
                                (j0 + 1 <= i) ? r[j4 * 8 + 2 * u + 1] * p.scale : 0.f);
        }
        *reinterpret_cast<uint4*>(stg + ptx::sw128(i, (cb * 32 + j4 * 8) * 2)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
  // ---------------- chunk-local cumsum of g: thread (column, 32-row segment) ----------------
  // The tile is overwritten with x = G - Gm (Gm = G at row 63, the mid-chunk reference).
  const int gcol = tid & 63, seg = tid >> 6;
  unsigned char* gt = Gs + (gcol >> 5) * TILE_BYTES;
  const uint32_t gby = (uint32_t)(gcol & 31) * 4;
  float gv[32];
  if (ok) ok = ptx::mbar_wait(&bar_g, 0);
  if (ok) {
    float sum = 0.f;
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      gv[r] = *reinterpret_cast<const float*>(gt + ptx::sw128(seg * 32 + r, gby));
      sum += gv[r];
    }
    segs[seg][gcol] = sum;
  }
  __syncthreads();
  if (ok) {
    const float gm = segs[0][gcol] + segs[1][gcol];
    float run = -gm;
    for (int s2 = 0; s2 < seg; ++s2) run += segs[s2][gcol];
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      run += gv[r];
      *reinterpret_cast<float*>(gt + ptx::sw128(seg * 32 + r, gby)) = run;
    }
    if (seg == 0) {
      const float glm = segs[2][gcol] + segs[3][gcol];  // GL - Gm
      cS[gcol] = p.scale * __expf(gm);
      cL[gcol] = __expf(glm);
      cGL[gcol] = __expf(gm + glm);
    }
  }
  __syncthreads();
  // ---------------- qtil = q e^{G-Gm}, ktil = k e^{Gm-G}, in place, 8 columns per item ----------------
  if (ok) ok = ptx::mbar_wait(&bar_q, 0);
  if (ok) ok = ptx::mbar_wait(&bar_k, 0);
  if (ok) {
    for (int it = tid; it < 128 * 8; it += 256) {
      const int chunk = it & 7, row = it >> 3, col0 = chunk * 8;
      // chunks 4..7 (second fp32 tile) read their two halves in the opposite order, so the
      // eight lanes of each 16-byte access phase hit eight different bank groups
      const unsigned char* gp = Gs + (col0 >> 5) * TILE_BYTES;
      const uint32_t o0 = (col0 & 31) * 4 + ((chunk >> 2) ? 16u : 0u);
      float4 ga = *reinterpret_cast<const float4*>(gp + ptx::sw128(row, o0));
      float4 gb = *reinterpret_cast<const float4*>(gp + ptx::sw128(row, o0 ^ 16u));
      if (chunk >> 2) {
        const float4 t = ga;
        ga = gb;
        gb = t;
      }
      const float x8[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
      uint4* pq = reinterpret_cast<uint4*>(qtl + ptx::sw128(row, chunk * 16));
      uint4* pk = reinterpret_cast<uint4*>(ktl + ptx::sw128(row, chunk * 16));
      uint4 xq = *pq, xk = *pk;
      uint32_t* q2 = reinterpret_cast<uint32_t*>(&xq);
      uint32_t* k2 = reinterpret_cast<uint32_t*>(&xk);
#pragma unroll
      for (int e = 0; e < 4; ++e) {  // raw q, k (bf16 or fp16) -> bf16 q~, k~
        const float2 fq = ptx::unpack16(q2[e], F16), fk = ptx::unpack16(k2[e], F16);
        q2[e] = ptx::pack_bf16(fq.x * __expf(x8[2 * e]), fq.y * __expf(x8[2 * e + 1]));
        k2[e] = ptx::pack_bf16(fk.x * __expf(-x8[2 * e]), fk.y * __expf(-x8[2 * e + 1]));
      }
      *pq = xq;
      *pk = xk;
    }
  }
  ptx::fence_async_smem();
  ptx::tc_fence_before();
  __syncthreads();
  if (tid == 32 && ok) {
    ptx::tc_fence_after();
    constexpr uint32_t ID_KM = ptx::idesc_bf16(128, 64, false, true);
    constexpr uint32_t ID_MM = ptx::idesc_bf16(128, 64, true, true);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      // M4 (M1 columns 0..63): dA[i][j] x ktil[j][k]
      ptx::mma_bf16_ss(tM1, desc_kmajor(dAs + (ks >> 2) * TILE_BYTES, (ks & 3) * 32),
                       desc_mnmajor(ktl, ks * 2048, TILE_BYTES), ID_KM, ks ? 1u : 0u);
      // M5 (M1 columns 64..127): dA^T[j][i] x qtil[i][k]
      ptx::mma_bf16_ss(tM1 + 64, desc_mnmajor(dAs, ks * 2048, TILE_BYTES), desc_mnmajor(qtl, ks * 2048, TILE_BYTES),
                       ID_MM, ks ? 1u : 0u);
    }
    ptx::mma_commit(&bar_mma);
  }
  if (ok) ok = ptx::mbar_wait(&bar_mma, 1);
  ptx::tc_fence_after();
  // ---------------- epilogue: dq, dk (in place of qtil, ktil), dg_raw (in place of x), column sums ----------------
  // Rows past T need no mask: their q, k, v, do were zero-filled by the loads, so every
  // term below is zero there, and the stores clip them.
  if (ok) {
#pragma unroll 1
    for (int g16 = 0; g16 < 2; ++g16) {
      const int cb = ch * 32 + g16 * 16;  // first column of this group
      float m4[16], m5[16], m2[16], m3[16];
      ptx::tmem_ld16(tmem_lane_addr(tM1, qd * 32, cb), m4);
      ptx::tmem_ld16(tmem_lane_addr(tM1 + 64, qd * 32, cb), m5);
      ptx::tmem_ld16(tmem_lane_addr(tM2, qd * 32, cb), m2);
      ptx::tmem_ld16(tmem_lane_addr(tM3, qd * 32, cb), m3);
      const uint32_t qb = ptx::sw128(i, cb * 2), qb2 = ptx::sw128(i, cb * 2 + 16);
      const uint4 qa = *reinterpret_cast<const uint4*>(qtl + qb), qa2 = *reinterpret_cast<const uint4*>(qtl + qb2);
      const uint4 ka = *reinterpret_cast<const uint4*>(ktl + qb), ka2 = *reinterpret_cast<const uint4*>(ktl + qb2);
      unsigned char* gp = Gs + (cb >> 5) * TILE_BYTES;
      float gv[16];  // x = G - Gm of this row
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4 t4 = *reinterpret_cast<const float4*>(gp + ptx::sw128(i, (cb & 31) * 4 + u * 16));
        gv[4 * u] = t4.x; gv[4 * u + 1] = t4.y; gv[4 * u + 2] = t4.z; gv[4 * u + 3] = t4.w;
      }
      float qv[16], kv[16];
      {
        const __nv_bfloat162* a = reinterpret_cast<const __nv_bfloat162*>(&qa);
        const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&qa2);
        const __nv_bfloat162* d = reinterpret_cast<const __nv_bfloat162*>(&ka);
        const __nv_bfloat162* d2 = reinterpret_cast<const __nv_bfloat162*>(&ka2);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 t0 = __bfloat1622float2(a[e]), t1 = __bfloat1622float2(a2[e]);
          const float2 u0 = __bfloat1622float2(d[e]), u1 = __bfloat1622float2(d2[e]);
          qv[2 * e] = t0.x; qv[2 * e + 1] = t0.y; qv[8 + 2 * e] = t1.x; qv[8 + 2 * e + 1] = t1.y;
          kv[2 * e] = u0.x; kv[2 * e + 1] = u0.y; kv[8 + 2 * e] = u1.x; kv[8 + 2 * e + 1] = u1.y;
        }
      }
      ptx::tmem_ld_wait();
      float cs[16];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4 f4s = *reinterpret_cast<const float4*>(&cS[cb + 4 * u]);
        const float4 f4l = *reinterpret_cast<const float4*>(&cL[cb + 4 * u]);
        const float fs[4] = {f4s.x, f4s.y, f4s.z, f4s.w}, fl[4] = {f4l.x, f4l.y, f4l.z, f4l.w};
#pragma unroll
        for (int e4 = 0; e4 < 4; ++e4) {
          const int e = 4 * u + e4;
          const float x = gv[e];
          const float pq = fmaf(fs[e4], m2[e], m4[e]);  // dq = e^{x} pq
          const float lm3 = fl[e4] * m3[e];
          const float pk = m5[e] + lm3;                 // dk = e^{-x} pk
          gv[e] = qv[e] * pq - kv[e] * pk;              // dg_raw = q dq - k dk
          cs[e] = kv[e] * lm3;                          // (e^{GL-G} dki) k
          m4[e] = __expf(x) * pq;
          m5[e] = __expf(-x) * pk;
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        *reinterpret_cast<float4*>(gp + ptx::sw128(i, (cb & 31) * 4 + u * 16)) =
            make_float4(gv[4 * u], gv[4 * u + 1], gv[4 * u + 2], gv[4 * u + 3]);
      uint32_t dqw[8], dkw[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        dqw[u] = ptx::pack16(m4[2 * u], m4[2 * u + 1], F16);
        dkw[u] = ptx::pack16(m5[2 * u], m5[2 * u + 1], F16);
      }
      *reinterpret_cast<uint4*>(qtl + qb) = make_uint4(dqw[0], dqw[1], dqw[2], dqw[3]);
      *reinterpret_cast<uint4*>(qtl + qb2) = make_uint4(dqw[4], dqw[5], dqw[6], dqw[7]);
      *reinterpret_cast<uint4*>(ktl + qb) = make_uint4(dkw[0], dkw[1], dkw[2], dkw[3]);
      *reinterpret_cast<uint4*>(ktl + qb2) = make_uint4(dkw[4], dkw[5], dkw[6], dkw[7]);
      const float tot = dqk_reduce16(cs, lane);
      if ((lane & 1) == 0) colsum[qd][cb + dqk_red_col(lane)] = tot;
    }
  }
  ptx::fence_async_smem();
  __syncthreads();
  if (tid == 0 && ok) {  // dq, dk tiles -> global (rows past T are clipped by the tensor map)
    ptx::tma_store_4d(&maps.dq, k0, h, row0, b, qtl);
    ptx::tma_store_4d(&maps.dk, k0, h, row0, b, ktl);
    ptx::bulk_commit();
  }
  // ---------------- dg = reverse cumsum over rows + inter term, in place, then one TMA store ----------------
  float dv[32];
  if (ok) {
    float sum = 0.f;
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      dv[r] = *reinterpret_cast<const float*>(gt + ptx::sw128(seg * 32 + r, gby));
      sum += dv[r];
    }
    segs[seg][gcol] = sum;
  }
  __syncthreads();
  if (ok) {
    float run = cGL[gcol] * (hdh2[0][gcol] + hdh2[1][gcol]) + colsum[0][gcol] + colsum[1][gcol] + colsum[2][gcol] +
                colsum[3][gcol];
    for (int s2 = seg + 1; s2 < 4; ++s2) run += segs[s2][gcol];
#pragma unroll
    for (int r = 31; r >= 0; --r) {
      run += dv[r];
      *reinterpret_cast<float*>(gt + ptx::sw128(seg * 32 + r, gby)) = run;
    }
  }
  ptx::fence_async_smem();
  __syncthreads();
  if (tid == 0 && ok) {
    ptx::tma_store_4d(&maps.dg, k0, h, row0, b, Gs);
    ptx::tma_store_4d(&maps.dg, k0 + 32, h, row0, b, Gs + TILE_BYTES);
    ptx::bulk_commit();
  }
  if (!ok && tid == 0) {  // drain loads that may still be in flight (bounded)
    ptx::mbar_wait(&full[0], 0);
    ptx::mbar_wait(&full[1], 0);
    ptx::mbar_wait(&bar_g, 0);
    ptx::mbar_wait(&bar_q, 0);
    ptx::mbar_wait(&bar_k, 0);
  }
  if (tid == 0) ptx::bulk_wait_read<0>();  // the stores have read the staging tiles
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) ptx::tmem_dealloc(tmem_base, 256);
}

TOPS_DEVICE_ERROR_READER(read_device_error)

// one thread waits on an mbarrier that nothing arrives on: the bounded wait gives up,
// records DEVERR_MBAR_TIMEOUT and the kernel returns (the failure path, exercised on purpose)
__global__ void k_wait_selftest() {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    ptx::mbar_init(&bar, 1);
    ptx::fence_mbar_init();
    ptx::mbar_wait(&bar, 0);
  }
}

int selftest_wait_timeout(cudaStream_t st) {
  k_wait_selftest<<<1, 32, 0, st>>>();
  TOPS_CUDA_LAUNCH_CHECK("wait_selftest");
  return TOPS_OK;
}

// ---------------------------------------------------------------------------
// host orchestration
// ---------------------------------------------------------------------------
// SM count of the current device, looked up once per device
static int sm_count() {
  static std::atomic<int> cache[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64) {
    const int c = cache[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev >= 0 && dev < 64) cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

// Span split of the state scans: enough spans that the scan grid fills the SMs (one CTA
// per SM: 512 TMEM columns), at least 4 chunks per span (config 3 at one sequence per GPU:
// 8 spans, 0.225 ms per fwd+bwd step against 0.260 with 4); one span when the (batch, head,
// V-tile) units alone fill half the GPU or the sequence is short.  A split runs every chunk
// twice (the zero-state pass, which has no output GEMM, then the re-scan), in exchange for a
// chain of NTb / spans chunks per CTA instead of NTb.
struct Spans {
  int n, len;
};
static Spans spans_for(const tops_gla_shape& s, int NTb) {
  const int units = ((s.V + BV - 1) / BV) * s.H * s.B;
  const int nsm = sm_count();
  Spans r{1, NTb};
  if (units * 2 > nsm || NTb < 8) return r;
  int S = nsm / units;
  if (S > NTb / 4) S = NTb / 4;
  if (S < 2) return r;
  r.len = (NTb + S - 1) / S;
  r.n = (NTb + r.len - 1) / r.len;
  return r;
}

// scratch of a span-split scan: final states E and incoming states Hs [nspan][B,H,K,V],
// span decays P [nspan][B,H,K] (fp32); bytes from `off` (1 KB aligned pieces)
struct SpanBufs {
  float *E = nullptr, *Hs = nullptr, *P = nullptr;
};
static size_t carve_spans(const tops_gla_shape& s, Spans spn, char* base, size_t off, SpanBufs* out,
                          bool force = false) {
  if (spn.n <= 1 && !force) return off;
  auto take = [&](size_t bytes) {
    off = (off + 1023) & ~size_t(1023);
    char* p = base ? base + off : nullptr;
    off += bytes;
    return reinterpret_cast<float*>(p);
  };
  const size_t st = (size_t)spn.n * s.B * s.H * s.K * s.V * 4;
  SpanBufs b;
  b.E = take(st);
  b.Hs = take(st);
  b.P = take((size_t)spn.n * s.B * s.H * s.K * 4);
  if (out) *out = b;
  return off;
}

// Varlen problems run on the fixed-length kernels after each segment is padded to a
// multiple of BT rows and packed (the reference pads segments to its chunk size the same
// way, tops/ops/gla/chunk.py:751-807): every BT-row block then lies inside one segment, and
// only the state scans need the segment boundaries (blk_off).  The padded length is bounded
// by (ceil(T/BT) + N) * BT rows, computed without reading cu_seqlens on the host.
static int varlen_rows(const tops_gla_shape& s) { return ((s.T + BT - 1) / BT + s.N) * BT; }

static tops_gla_shape padded_shape(const tops_gla_shape& s) {
  tops_gla_shape p = s;
  p.B = 1;
  p.T = varlen_rows(s);
  p.cu_seqlens = nullptr;
  p.chunk_offsets = nullptr;
  return p;
}

// K = 64 and V = 64 run as one 128-wide state tile whose upper half is padding: the loads past
// K or V read zeros (TMA fills out-of-bounds boxes), so the padded state rows / columns stay
// zero, and every store, decay read and initial / final state access is guarded to the real
// extent (as the reference pads K and V to 128, tops/ops/gla/chunk.py:1128-1132).
bool eligible(const tops_gla_shape& s) {
  const bool kok = s.K == 64 || s.K == 128 || s.K == 256;
  const bool vok = s.V == 64 || (s.V > 0 && s.V % BV == 0);
  if (!((s.dtype == TOPS_BF16 || s.dtype == TOPS_F16) && kok && vok && s.T > 0 && s.B > 0 && s.H > 0)) return false;
  // packed varlen: only while the block padding at most doubles the rows (long segments)
  if (s.cu_seqlens != nullptr && (s.B != 1 || s.N <= 0 || (size_t)varlen_rows(s) > 2 * (size_t)s.T + BT)) return false;
  return tops_gla_has_tcgen05() && encode_fn() != nullptr;
}

__global__ void k_blk_off(const int32_t* __restrict__ cu, int N, int32_t* __restrict__ blk_off) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    int acc = 0;
    blk_off[0] = 0;
    for (int n = 0; n < N; ++n) {
      acc += (cu[n + 1] - cu[n] + BT - 1) / BT;
      blk_off[n + 1] = acc;
    }
  }
}

// last n in [0, N) with a[n] <= x (a non-decreasing, a[0] <= x)
__device__ __forceinline__ int seg_of(const int32_t* __restrict__ a, int N, int x) {
  int lo = 0, hi = N - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a[mid] <= x) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// to_pad = 1: padded row r <- packed row (or zeros); to_pad = 0: packed row r <- padded row.
// One warp per row, 16-byte vectors.
__global__ void k_pad_rows(const uint4* __restrict__ src, uint4* __restrict__ dst, int row_vec, int rows,
                           const int32_t* __restrict__ cu, const int32_t* __restrict__ blk_off, int N, int to_pad) {
  const int lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
  for (int r = blockIdx.x * wpb + (threadIdx.x >> 5); r < rows; r += gridDim.x * wpb) {
    int other = -1;
    if (to_pad) {
      const int blk = r / BT;
      if (blk < blk_off[N]) {
        const int n = seg_of(blk_off, N, blk);
        const int off = r - blk_off[n] * BT;
        if (off < cu[n + 1] - cu[n]) other = cu[n] + off;
      }
    } else {
      const int n = seg_of(cu, N, r);
      other = blk_off[n] * BT + (r - cu[n]);
    }
    uint4* d = dst + (size_t)r * row_vec;
    if (other >= 0) {
      const uint4* sp = src + (size_t)other * row_vec;
      for (int c = lane; c < row_vec; c += 32) d[c] = sp[c];
    } else {
      for (int c = lane; c < row_vec; c += 32) d[c] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

static int pad_rows(const void* src, void* dst, size_t row_bytes, int rows, const tops_gla_shape& s,
                    const int32_t* blk_off, int to_pad, cudaStream_t st) {
  if (rows <= 0) return TOPS_OK;
  const int row_vec = (int)(row_bytes / 16);
  int grid = (rows + 7) / 8;
  if (grid > 148 * 16) grid = 148 * 16;
  k_pad_rows<<<grid, 256, 0, st>>>(static_cast<const uint4*>(src), static_cast<uint4*>(dst), row_vec, rows,
                                   s.cu_seqlens, blk_off, s.N, to_pad);
  TOPS_CUDA_LAUNCH_CHECK(to_pad ? "tc varlen pad" : "tc varlen unpad");
  return TOPS_OK;
}

// Intermediates of the forward that the backward reuses (one contiguous block).
struct Saved {
  bf16 *qh, *kd, *A, *h;
  bf16* vb = nullptr;  // fp16 problems: bf16 copy of v (an MMA operand of the scans and of k_dqk)
  float* D;
  SpanBufs sb;  // scratch of a span-split forward scan (empty when the scan runs in one span)
};

// force_spans: carve the span scratch even for one span (the two-phase sequence-parallel entry
// points keep the zero-state pass's results there between their two calls)
static size_t carve_saved(const tops_gla_shape& s, void* base, Saved* sv, bool spans = true, bool force_spans = false) {
  const int NTb = (s.T + BT - 1) / BT;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    off = (off + 1023) & ~size_t(1023);
    char* p = base ? static_cast<char*>(base) + off : nullptr;
    off += bytes;
    return p;
  };
  const size_t tok = (size_t)s.B * s.T * s.H;
  Saved v;
  v.qh = reinterpret_cast<bf16*>(take(tok * s.K * 2));
  v.kd = reinterpret_cast<bf16*>(take(tok * s.K * 2));
  v.A = reinterpret_cast<bf16*>(take(tok * BT * 2));
  v.D = reinterpret_cast<float*>(take((size_t)s.B * NTb * s.H * s.K * 4));
  v.h = reinterpret_cast<bf16*>(take((size_t)s.B * NTb * s.H * s.K * s.V * 2));
  if (s.dtype == TOPS_F16) v.vb = reinterpret_cast<bf16*>(take(tok * s.V * 2));
  if (spans) off = carve_spans(s, spans_for(s, NTb), static_cast<char*>(base), off, &v.sb, force_spans);
  if (sv) *sv = v;
  return off;
}

size_t saved_bytes(const tops_gla_shape& s) {
  return s.cu_seqlens ? carve_saved(padded_shape(s), nullptr, nullptr, false) : carve_saved(s, nullptr, nullptr);
}

static size_t prep_smem() { return 6 * TILE_BYTES + 1024; }
static size_t scan_smem(int K) { return 2 * (size_t)(K / 64 + 2) * TILE_BYTES + 8 * 2 * 2048 + 1024; }
static size_t out_smem() { return (size_t)OUT_STAGES * STAGE_BYTES + 2 * TILE_BYTES + 1024; }

// Dynamic shared memory limit of a kernel, set once per (device, kernel, size): the launches of
// a step then issue no attribute calls (host time that counts when a rank's step is short).
template <typename KernelT>
static cudaError_t set_smem(KernelT k, size_t bytes) {
  struct Entry {
    int dev;
    const void* fn;
    size_t bytes;
  };
  static std::mutex mu;
  static std::vector<Entry> done;
  int dev = 0;
  cudaGetDevice(&dev);
  const void* fn = reinterpret_cast<const void*>(k);
  std::lock_guard<std::mutex> lk(mu);
  for (const Entry& e : done)
    if (e.dev == dev && e.fn == fn && e.bytes >= bytes) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  // the largest shared-memory carveout: every kernel here keeps big tiles in shared memory
  // (k_prep and k_dqk need it for two CTAs per SM)
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e == cudaSuccess) done.push_back({dev, fn, bytes});
  return e;
}

// First launch of a span-split scan: every span from a zero state, its final state into
// sb.E and the product of its chunk decays into sb.P (also for a single span).
static int scan_spans_zero(const tops_gla_shape& s, const ScanMaps& sm, int reverse, const float* D,
                           const SpanBufs& sb, Spans spn, cudaStream_t st) {
  const int NTb = (s.T + BT - 1) / BT;
  cudaError_t e;
  if ((e = set_smem(k_scan<false>, scan_smem(s.K))) != cudaSuccess) return cuda_status(e, "tc scan attr");
  LaunchTimer lt(st, reverse ? "tc_scan_bwd_span" : "tc_scan_span");
  ScanParams sp{s.B, s.T, s.H, s.K, s.V, NTb, reverse, D, nullptr, sb.E, nullptr, spn.n, spn.len, 0, sb.P, nullptr};
  k_scan<false><<<dim3((s.V + BV - 1) / BV, s.H, s.B * spn.n), 256, scan_smem(s.K), st>>>(sm, sp);
  TOPS_CUDA_LAUNCH_CHECK("tc_scan_span");
  return TOPS_OK;
}

// Rest of a span-split scan after scan_spans_zero: every span's incoming state from `init`
// (k_span_prefix; a single span starts from `init` itself), then the re-scan from those
// states that stores the chunk states (and, with `fm`, writes the chunk outputs).
static int scan_spans_finish(const tops_gla_shape& s, const ScanMaps& sm, int reverse, const float* D,
                             const float* init, float* fin, bf16* states, const SpanBufs& sb, Spans spn,
                             cudaStream_t st, const char* name, const FusedMaps* fm) {
  const int NTb = (s.T + BT - 1) / BT;
  cudaError_t e;
  if ((e = set_smem(k_scan<false>, scan_smem(s.K))) != cudaSuccess) return cuda_status(e, "tc scan attr");
  const auto kso = fm && fm->out_f16 ? k_scan_out<false, true> : k_scan_out<false, false>;
  if (fm && (e = set_smem(kso, fo_smem(s.K))) != cudaSuccess) return cuda_status(e, "tc scan_out attr");
  const float* span_init = init;
  if (spn.n > 1) {
    LaunchTimer lt(st, "tc_span_prefix");
    const size_t n4 = (size_t)s.B * s.H * s.K * s.V / 4;
    k_span_prefix<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(spn.n, s.B, s.H, s.K, s.V, init, sb.P, sb.E, sb.Hs);
    TOPS_CUDA_LAUNCH_CHECK("tc_span_prefix");
    span_init = sb.Hs;
  }
  LaunchTimer lt(st, name);
  ScanParams sp{s.B, s.T, s.H, s.K, s.V, NTb, reverse, D, span_init, fin, states, spn.n, spn.len, 1, nullptr, nullptr};
  if (fm)
    kso<<<dim3((s.V + BV - 1) / BV, s.H, s.B * spn.n), FO_THREADS, fo_smem(s.K), st>>>(*fm, sp);
  else
    k_scan<false><<<dim3((s.V + BV - 1) / BV, s.H, s.B * spn.n), 256, scan_smem(s.K), st>>>(sm, sp);
  TOPS_CUDA_LAUNCH_CHECK(name);
  return TOPS_OK;
}

// One state scan (forward h or reverse dh), split into spans when that fills the GPU.
// With `fm`, the pass that stores the chunk states is k_scan_out, which also writes the
// chunk outputs (fwd o, bwd dv) through fm->o.
static int run_scan(const tops_gla_shape& s, const ScanMaps& sm, int reverse, const float* D, const float* init,
                    float* fin, bf16* states, const SpanBufs& sb, Spans spn, cudaStream_t st, const char* name,
                    const int* blk_off = nullptr, const FusedMaps* fm = nullptr) {
  const int NTb = (s.T + BT - 1) / BT;
  cudaError_t e;
  if ((e = set_smem(k_scan<false>, scan_smem(s.K))) != cudaSuccess) return cuda_status(e, "tc scan attr");
  const auto kso = fm && fm->out_f16 ? k_scan_out<false, true> : k_scan_out<false, false>;
  const auto kso_seg = fm && fm->out_f16 ? k_scan_out<true, true> : k_scan_out<true, false>;
  if (fm && (e = set_smem(kso, fo_smem(s.K))) != cudaSuccess) return cuda_status(e, "tc scan_out attr");
  if (blk_off != nullptr) {  // padded varlen problem: one CTA column per segment
    LaunchTimer lt(st, name);
    ScanParams sp{s.B, s.T, s.H, s.K, s.V, NTb, reverse, D, init, fin, states, 1, NTb, 0, nullptr, blk_off};
    if (fm) {
      if ((e = set_smem(kso_seg, fo_smem(s.K))) != cudaSuccess) return cuda_status(e, "tc scan_out attr");
      kso_seg<<<dim3((s.V + BV - 1) / BV, s.H, s.N), FO_THREADS, fo_smem(s.K), st>>>(*fm, sp);
    } else {
      if ((e = set_smem(k_scan<true>, scan_smem(s.K))) != cudaSuccess) return cuda_status(e, "tc scan attr");
      k_scan<true><<<dim3((s.V + BV - 1) / BV, s.H, s.N), 256, scan_smem(s.K), st>>>(sm, sp);
    }
    TOPS_CUDA_LAUNCH_CHECK(name);
    return TOPS_OK;
  }
  if (spn.n <= 1) {
    LaunchTimer lt(st, name);
    ScanParams sp{s.B, s.T, s.H, s.K, s.V, NTb, reverse, D, init, fin, states, 1, NTb, 0, nullptr, nullptr};
    if (fm)
      kso<<<dim3((s.V + BV - 1) / BV, s.H, s.B), FO_THREADS, fo_smem(s.K), st>>>(*fm, sp);
    else
      k_scan<false><<<dim3((s.V + BV - 1) / BV, s.H, s.B), 256, scan_smem(s.K), st>>>(sm, sp);
    TOPS_CUDA_LAUNCH_CHECK(name);
    return TOPS_OK;
  }
  int rc = scan_spans_zero(s, sm, reverse, D, sb, spn, st);
  return rc ? rc : scan_spans_finish(s, sm, reverse, D, init, fin, states, sb, spn, st, name, fm);
}

// The fused scan + output kernel is the default; TOPS_GLA_UNFUSED_OUT=1 selects the
// separate state scan and k_out GEMM (same results; kept for comparison).
static bool fused_out() {
  static const bool on = [] {
    const char* e = getenv("TOPS_GLA_UNFUSED_OUT");
    return !(e && e[0] == '1');
  }();
  return on;
}

// fp16 -> bf16 copy (8 elements per thread and step): the operands that feed tcgen05 MMAs next
// to bf16 intermediates (v, do) must be bf16 themselves, since one MMA takes one operand type.
__global__ void k_f16_to_bf16(const uint4* __restrict__ src, uint4* __restrict__ dst, size_t n8) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (size_t)gridDim.x * blockDim.x) {
    const uint4 x = src[i];
    const uint32_t w[4] = {x.x, x.y, x.z, x.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = ptx::unpack16(w[e], true);
      o[e] = ptx::pack_bf16(f.x, f.y);
    }
    dst[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

static int to_bf16(const void* src, bf16* dst, size_t n, cudaStream_t st) {
  const size_t n8 = n / 8;  // token tensors hold a multiple of 64 elements per row
  if (n8 == 0) return TOPS_OK;
  LaunchTimer lt(st, "tc_f16_to_bf16");
  const size_t blocks = (n8 + 255) / 256 < (size_t)sm_count() * 8 ? (n8 + 255) / 256 : (size_t)sm_count() * 8;
  k_f16_to_bf16<<<(unsigned)blocks, 256, 0, st>>>(static_cast<const uint4*>(src), reinterpret_cast<uint4*>(dst), n8);
  TOPS_CUDA_LAUNCH_CHECK("tc f16 to bf16");
  return TOPS_OK;
}

// storage type of q, k, o, dq, dk, dv for the tensor maps
static CUtensorMapDataType io_type(const tops_gla_shape& s) {
  return s.dtype == TOPS_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

// Tensor maps of k_prep (q, k, g in; qhat, kdec, A out) and of the forward state scan
// (kdec, v in; chunk states out) over the saved block `sv`.
static bool fwd_maps(const tops_gla_shape& s, const void* q, const void* k, const void* v, const float* g,
                     const Saved& sv, PrepMaps* pm, ScanMaps* sm) {
  const int NTb = (s.T + BT - 1) / BT;
  const CUtensorMapDataType BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, F32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const CUtensorMapDataType IO = io_type(s);
  if (sv.vb != nullptr) v = sv.vb;  // fp16 problem: the scans read the bf16 copy of v
  return map_tok(&pm->q, q, IO, 2, s.B, s.T, s.H, s.K, 64, BT) && map_tok(&pm->k, k, IO, 2, s.B, s.T, s.H, s.K, 64, BT) &&
         map_tok(&pm->g, g, F32, 4, s.B, s.T, s.H, s.K, 32, BT) &&
         map_tok(&pm->qh, sv.qh, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
         map_tok(&pm->kd, sv.kd, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
         map_tok(&pm->A, sv.A, BF, 2, s.B, s.T, s.H, BT, 64, BT) &&
         map_tok(&sm->x, sv.kd, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
         map_tok(&sm->y, v, BF, 2, s.B, s.T, s.H, s.V, 64, BT) &&
         map_state_store(&sm->st, sv.h, s.B * NTb * s.H, s.K, s.V);
}

static int launch_prep(const tops_gla_shape& s, const PrepMaps& pm, const Saved& sv, cudaStream_t st) {
  const int NTb = (s.T + BT - 1) / BT;
  cudaError_t e;
  LaunchTimer lt(st, "tc_prep");
  PrepParams pp{s.B, s.T, s.H, s.K, NTb, s.scale, sv.D};
  auto kern = s.dtype == TOPS_F16 ? k_prep<true> : k_prep<false>;
  if ((e = set_smem(kern, prep_smem())) != cudaSuccess) return cuda_status(e, "tc prep attr");
  const int items = NTb * s.H * s.B;
  kern<<<items < 2 * sm_count() ? items : 2 * sm_count(), 256, prep_smem(), st>>>(pm, pp);
  TOPS_CUDA_LAUNCH_CHECK("tc_prep");
  return TOPS_OK;
}

// Forward of a fixed-length (or padded varlen, blk_off != null) problem: o, ht and (in
// `saved`) qhat, kdec, A, D, chunk-start states h.
static int fwd_core(const tops_gla_shape& s, const void* q, const void* k, const void* v, const float* g,
                    const float* h0, void* o, float* ht, void* saved, cudaStream_t st, const int32_t* blk_off) {
  if (g == nullptr) return fail(TOPS_ERR_UNSUPPORTED, "tc fwd needs gates");
  Saved sv;
  carve_saved(s, saved, &sv, blk_off == nullptr);
  const int NTb = (s.T + BT - 1) / BT;
  const CUtensorMapDataType BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const void* fv = v;  // the caller's v (fp16 problems convert it into sv.vb first)
  PrepMaps pm;
  ScanMaps sm;
  bool okm = fwd_maps(s, q, k, v, g, sv, &pm, &sm);
  if (sv.vb != nullptr) v = sv.vb;
  OutMaps om;
  FusedMaps fm{};
  // fp16 and the padded head sizes run the fused kernel only (k_out stores bf16 through TMA, in
  // 64-column boxes that would lie wholly past V = 64)
  const bool fused = o != nullptr && (fused_out() || s.dtype == TOPS_F16 || s.K < 128 || s.V < BV);
  if (o != nullptr && !fused)
    okm = okm && map_tok(&om.x, sv.qh, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
          map_state(&om.s, sv.h, s.B * NTb * s.H, s.K, s.V, 64) &&
          map_tok(&om.a, sv.A, BF, 2, s.B, s.T, s.H, BT, 64, BT) &&
          map_tok(&om.y, v, BF, 2, s.B, s.T, s.H, s.V, 64, 64) && map_tok(&om.o, o, BF, 2, s.B, s.T, s.H, s.V, 64, BT);
  if (fused)
    okm = okm && map_tok(&fm.sx, sv.kd, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
          map_tok(&fm.y, v, BF, 2, s.B, s.T, s.H, s.V, 64, BT) &&
          map_tok(&fm.ox, sv.qh, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
          map_tok(&fm.a, sv.A, BF, 2, s.B, s.T, s.H, BT, 64, BT);
  fm.out = static_cast<bf16*>(o);
  fm.out_f16 = s.dtype == TOPS_F16;
  if (!okm) return fail(TOPS_ERR_CUDA, "tc fwd: cuTensorMapEncodeTiled failed (alignment?)");
  cudaError_t e;
  int rc;
  if (sv.vb != nullptr && (rc = to_bf16(fv, sv.vb, (size_t)s.B * s.T * s.H * s.V, st))) return rc;
  if ((rc = launch_prep(s, pm, sv, st))) return rc;
  rc = run_scan(s, sm, 0, sv.D, h0, ht, sv.h, sv.sb, spans_for(s, NTb), st, fused ? "tc_scan_out" : "tc_scan",
                    blk_off, fused ? &fm : nullptr);
  if (rc) return rc;
  if (o == nullptr || fused) return TOPS_OK;  // final state only, or o written by the fused scan
  {
    LaunchTimer lt(st, "tc_out");
    OutParams op{s.B, s.T, s.H, s.K, s.V, NTb, 0, static_cast<bf16*>(o)};
    if ((e = set_smem(k_out, out_smem())) != cudaSuccess) return cuda_status(e, "tc out attr");
    const int items = s.B * NTb * s.H * ((s.V + BV - 1) / BV);
    const int grid = items < sm_count() ? items : sm_count();
    k_out<<<grid, 192, out_smem(), st>>>(om, op);
    TOPS_CUDA_LAUNCH_CHECK("tc_out");
  }
  return TOPS_OK;
}

static size_t dqk_smem() { return 2 * (size_t)DQK_STG + 1024; }

// fp16 problems: bytes of the bf16 copy of do in the backward workspace (0 otherwise)
static size_t dob_bytes(const tops_gla_shape& s) {
  return s.dtype == TOPS_F16 ? (((size_t)s.B * s.T * s.H * s.V * 2 + 1023) & ~size_t(1023)) : 0;
}

// reverse scan: qhat (saved) and do in, chunk-end state gradients dh out
static bool bwd_scan_maps(const tops_gla_shape& s, const void* dO, const Saved& sv, bf16* dhs, ScanMaps* sm) {
  const int NTb = (s.T + BT - 1) / BT;
  const CUtensorMapDataType BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  return map_tok(&sm->x, sv.qh, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
         map_tok(&sm->y, dO, BF, 2, s.B, s.T, s.H, s.V, 64, BT) &&
         map_state_store(&sm->st, dhs, s.B * NTb * s.H, s.K, s.V);
}

// fused reverse scan + dv GEMM: qhat / kdec / A (saved) and do in, dv out
static bool bwd_fused_maps(const tops_gla_shape& s, const void* dO, void* dv, const Saved& sv, FusedMaps* fm) {
  const CUtensorMapDataType BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  fm->out = static_cast<bf16*>(dv);
  fm->out_f16 = s.dtype == TOPS_F16;
  return map_tok(&fm->sx, sv.qh, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
         map_tok(&fm->y, dO, BF, 2, s.B, s.T, s.H, s.V, 64, BT) &&
         map_tok(&fm->ox, sv.kd, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
         map_tok(&fm->a, sv.A, BF, 2, s.B, s.T, s.H, BT, 64, 64);
}

static bool dqk_maps(const tops_gla_shape& s, const void* q, const void* k, const void* v, const float* g,
                     const void* dO, const Saved& sv, bf16* dhs, void* dq, void* dk, float* dg, DqkMaps* dm) {
  const int NTb = (s.T + BT - 1) / BT;
  const CUtensorMapDataType BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, F32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const CUtensorMapDataType IO = io_type(s);
  if (sv.vb != nullptr) v = sv.vb;  // fp16: v and do are read as bf16 copies (dO is the copy already)
  return map_tok(&dm->dO, dO, BF, 2, s.B, s.T, s.H, s.V, 64, BT) && map_tok(&dm->v, v, BF, 2, s.B, s.T, s.H, s.V, 64, BT) &&
         map_state(&dm->hs, sv.h, s.B * NTb * s.H, s.K, s.V, 64) &&
         map_state(&dm->dhs, dhs, s.B * NTb * s.H, s.K, s.V, 64) &&
         map_tok(&dm->g, g, F32, 4, s.B, s.T, s.H, s.K, 32, BT) && map_tok(&dm->dg, dg, F32, 4, s.B, s.T, s.H, s.K, 32, BT) &&
         map_tok(&dm->q, q, IO, 2, s.B, s.T, s.H, s.K, 64, BT) && map_tok(&dm->k, k, IO, 2, s.B, s.T, s.H, s.K, 64, BT) &&
         map_tok(&dm->dq, dq, IO, 2, s.B, s.T, s.H, s.K, 64, BT) && map_tok(&dm->dk, dk, IO, 2, s.B, s.T, s.H, s.K, 64, BT);
}

static int launch_dqk(const tops_gla_shape& s, const DqkMaps& dm, void* dq, void* dk, float* dg, cudaStream_t st) {
  const int NTb = (s.T + BT - 1) / BT;
  cudaError_t e;
  LaunchTimer lt(st, "tc_dqk");
  DqkParams dp{s.B, s.T, s.H, s.K, s.V, NTb, s.scale, static_cast<bf16*>(dq), static_cast<bf16*>(dk), dg};
  auto kern = s.dtype == TOPS_F16 ? k_dqk<true> : k_dqk<false>;
  if ((e = set_smem(kern, dqk_smem())) != cudaSuccess) return cuda_status(e, "tc dqk attr");
  kern<<<dim3(s.K / 64, NTb, s.B * s.H), 256, dqk_smem(), st>>>(dm, dp);
  TOPS_CUDA_LAUNCH_CHECK("tc_dqk");
  return TOPS_OK;
}

// workspace of bwd_core: dh states, span scratch, and the saved block when it is recomputed
static size_t bwd_core_workspace(const tops_gla_shape& s, bool have_saved, bool spans) {
  const int NTb = (s.T + BT - 1) / BT;
  size_t n = ((size_t)s.B * NTb * s.H * s.K * s.V * 2 + 1023) & ~size_t(1023);  // dh states
  if (spans) n = (carve_spans(s, spans_for(s, NTb), nullptr, n, nullptr) + 1023) & ~size_t(1023);
  n += dob_bytes(s);
  if (!have_saved) n += carve_saved(s, nullptr, nullptr, spans);
  return n;
}

// Backward of a fixed-length (or padded varlen, blk_off != null) problem: dq, dk, dv (bf16),
// dg (fp32), dh0 (fp32, optional) from the forward's saved block.
static int bwd_core(const tops_gla_shape& s, const void* q, const void* k, const void* v, const float* g,
                    const float* h0, const void* dO, const float* dht, const void* saved_in, void* dq, void* dk,
                    void* dv, float* dg, float* dh0, void* workspace, cudaStream_t st, const int32_t* blk_off) {
  const int NTb = (s.T + BT - 1) / BT;
  char* ws = static_cast<char*>(workspace);
  bf16* dhs = reinterpret_cast<bf16*>(ws);
  const size_t dh_bytes = ((size_t)s.B * NTb * s.H * s.K * s.V * 2 + 1023) & ~size_t(1023);
  const Spans spn = blk_off ? Spans{1, NTb} : spans_for(s, NTb);
  SpanBufs sb;
  const size_t span_end = (carve_spans(s, spn, ws, dh_bytes, &sb) + 1023) & ~size_t(1023);
  bf16* dob = dob_bytes(s) ? reinterpret_cast<bf16*>(ws + span_end) : nullptr;
  void* saved = const_cast<void*>(saved_in);
  int rc;
  if (saved == nullptr) {  // recompute the forward intermediates (o is discarded into dv's buffer)
    saved = ws + span_end + dob_bytes(s);
    if ((rc = fwd_core(s, q, k, v, g, h0, dv, nullptr, saved, st, blk_off))) return rc;
  }
  if (dob != nullptr) {  // fp16: do feeds MMAs beside bf16 operands, so it is read as a bf16 copy
    if ((rc = to_bf16(dO, dob, (size_t)s.B * s.T * s.H * s.V, st))) return rc;
    dO = dob;
  }
  Saved sv;
  carve_saved(s, saved, &sv, blk_off == nullptr);
  const CUtensorMapDataType BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  ScanMaps sm;
  bool okm = bwd_scan_maps(s, dO, sv, dhs, &sm);
  const bool dh0_only = dq == nullptr;  // dq, dk, dv, dg all NULL: the reverse scan alone
  if (dh0_only) {
    if (!okm) return fail(TOPS_ERR_CUDA, "tc bwd: cuTensorMapEncodeTiled failed (alignment?)");
    return run_scan(s, sm, 1, sv.D, dht, dh0, nullptr, sb, spn, st, "tc_scan_bwd", blk_off);
  }
  OutMaps om;
  FusedMaps fm{};
  const bool fused = fused_out() || s.dtype == TOPS_F16 || s.K < 128 || s.V < BV;
  if (fused)
    okm = okm && bwd_fused_maps(s, dO, dv, sv, &fm);
  else
    okm = okm && map_tok(&om.x, sv.kd, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
          map_state(&om.s, dhs, s.B * NTb * s.H, s.K, s.V, 64) &&
          map_tok(&om.a, sv.A, BF, 2, s.B, s.T, s.H, BT, 64, 64) &&
          map_tok(&om.y, dO, BF, 2, s.B, s.T, s.H, s.V, 64, 64) && map_tok(&om.o, dv, BF, 2, s.B, s.T, s.H, s.V, 64, BT);
  DqkMaps dm;
  okm = okm && dqk_maps(s, q, k, v, g, dO, sv, dhs, dq, dk, dg, &dm);
  if (!okm) return fail(TOPS_ERR_CUDA, "tc bwd: cuTensorMapEncodeTiled failed (alignment?)");
  cudaError_t e;
  if ((rc = run_scan(s, sm, 1, sv.D, dht, dh0, dhs, sb, spn, st, fused ? "tc_scan_out_bwd" : "tc_scan_bwd", blk_off,
                     fused ? &fm : nullptr)))
    return rc;
  if (!fused) {
    LaunchTimer lt(st, "tc_out_dv");
    OutParams op{s.B, s.T, s.H, s.K, s.V, NTb, 1, static_cast<bf16*>(dv)};
    if ((e = set_smem(k_out, out_smem())) != cudaSuccess) return cuda_status(e, "tc out attr");
    const int items = s.B * NTb * s.H * ((s.V + BV - 1) / BV);
    const int grid = items < sm_count() ? items : sm_count();
    k_out<<<grid, 192, out_smem(), st>>>(om, op);
    TOPS_CUDA_LAUNCH_CHECK("tc_out_dv");
  }
  return launch_dqk(s, dm, dq, dk, dg, st);
}

// ---------------------------------------------------------------------------
// Two-phase forward / backward of one span of a sequence split over ranks (fixed length).
// The scan is linear in its incoming state, so everything that does not depend on it runs
// in the first phase: k_prep and the zero-state pass of the span-split scan, whose per-span
// results (E, P) stay in the saved block (forward) or the workspace (backward) and are also
// folded into the span's own final state S and decay D.  The host exchanges (S, D) between
// ranks; the second phase forms every in-GPU span's incoming state from the rank's incoming
// state (k_span_prefix) and runs the fused re-scan and, backward, k_dqk.  Per rank this is
// the single-GPU work plus one small combine kernel per direction.
// ---------------------------------------------------------------------------
static Spans spans_of(const tops_gla_shape& s) { return spans_for(s, (s.T + BT - 1) / BT); }

size_t span_saved_bytes(const tops_gla_shape& s) { return carve_saved(s, nullptr, nullptr, true, true); }

static int span_total(const tops_gla_shape& s, Spans spn, const SpanBufs& sb, float* out, float* dout,
                      cudaStream_t st, const p2p::PeerPush* push = nullptr) {
  const size_t n4 = (size_t)s.B * s.H * s.K * s.V / 4;
  const unsigned blocks = (unsigned)((n4 + 255) / 256);
  if (push == nullptr) {
    LaunchTimer lt(st, "tc_span_total");
    k_span_total<false><<<blocks, 256, 0, st>>>(spn.n, s.B, s.H, s.K, s.V, sb.P, sb.E, out, dout, p2p::PeerPush{});
    TOPS_CUDA_LAUNCH_CHECK("tc_span_total");
  } else {
    LaunchTimer lt(st, "tc_span_total_push");
    k_span_total<true><<<blocks, 256, 0, st>>>(spn.n, s.B, s.H, s.K, s.V, sb.P, sb.E, out, dout, *push);
    TOPS_CUDA_LAUNCH_CHECK("tc_span_total_push");
  }
  return TOPS_OK;
}

int fwd_span_begin(const tops_gla_shape& s, const void* q, const void* k, const void* v, const float* g, void* saved,
                   float* local_state, float* decay, cudaStream_t st, const p2p::PeerPush* push) {
  Saved sv;
  carve_saved(s, saved, &sv, true, true);
  PrepMaps pm;
  ScanMaps sm;
  if (!fwd_maps(s, q, k, v, g, sv, &pm, &sm)) return fail(TOPS_ERR_CUDA, "tc fwd span: cuTensorMapEncodeTiled failed");
  const Spans spn = spans_of(s);
  int rc;
  if (sv.vb != nullptr && (rc = to_bf16(v, sv.vb, (size_t)s.B * s.T * s.H * s.V, st))) return rc;
  if ((rc = launch_prep(s, pm, sv, st)) || (rc = scan_spans_zero(s, sm, 0, sv.D, sv.sb, spn, st))) return rc;
  return span_total(s, spn, sv.sb, local_state, decay, st, push);
}

int fwd_span_finish(const tops_gla_shape& s, const void* q, const void* k, const void* v, const float* g,
                    const float* h_in, void* o, float* ht, void* saved, cudaStream_t st) {
  Saved sv;
  carve_saved(s, saved, &sv, true, true);
  PrepMaps pm;
  ScanMaps sm;
  FusedMaps fm{};
  const CUtensorMapDataType BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const bool okm = fwd_maps(s, q, k, v, g, sv, &pm, &sm) && map_tok(&fm.sx, sv.kd, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
                   map_tok(&fm.y, sv.vb ? sv.vb : v, BF, 2, s.B, s.T, s.H, s.V, 64, BT) &&
                   map_tok(&fm.ox, sv.qh, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
                   map_tok(&fm.a, sv.A, BF, 2, s.B, s.T, s.H, BT, 64, BT);
  fm.out = static_cast<bf16*>(o);
  fm.out_f16 = s.dtype == TOPS_F16;
  if (!okm) return fail(TOPS_ERR_CUDA, "tc fwd span: cuTensorMapEncodeTiled failed");
  return scan_spans_finish(s, sm, 0, sv.D, h_in, ht, sv.h, sv.sb, spans_of(s), st, "tc_scan_out", &fm);
}

// backward workspace of the two-phase entry points: dh states and the span scratch
size_t bwd_span_workspace(const tops_gla_shape& s) {
  const int NTb = (s.T + BT - 1) / BT;
  const size_t n = ((size_t)s.B * NTb * s.H * s.K * s.V * 2 + 1023) & ~size_t(1023);
  return ((carve_spans(s, spans_of(s), nullptr, n, nullptr, true) + 1023) & ~size_t(1023)) + dob_bytes(s);
}

// dh states, span scratch and (fp16) the bf16 copy of do, which the first phase converts
static void carve_bwd_span(const tops_gla_shape& s, void* workspace, bf16** dhs, SpanBufs* sb, bf16** dob) {
  const int NTb = (s.T + BT - 1) / BT;
  char* ws = static_cast<char*>(workspace);
  *dhs = reinterpret_cast<bf16*>(ws);
  const size_t n = ((size_t)s.B * NTb * s.H * s.K * s.V * 2 + 1023) & ~size_t(1023);
  const size_t end = (carve_spans(s, spans_of(s), ws, n, sb, true) + 1023) & ~size_t(1023);
  *dob = dob_bytes(s) ? reinterpret_cast<bf16*>(ws + end) : nullptr;
}

int bwd_span_begin(const tops_gla_shape& s, const void* dO, const void* saved, void* workspace, float* local_dh0,
                   cudaStream_t st, const p2p::PeerPush* push) {
  Saved sv;
  carve_saved(s, const_cast<void*>(saved), &sv, true, true);
  bf16* dhs;
  bf16* dob;
  SpanBufs sb;
  carve_bwd_span(s, workspace, &dhs, &sb, &dob);
  int rc;
  if (dob != nullptr) {
    if ((rc = to_bf16(dO, dob, (size_t)s.B * s.T * s.H * s.V, st))) return rc;
    dO = dob;
  }
  ScanMaps sm;
  if (!bwd_scan_maps(s, dO, sv, dhs, &sm)) return fail(TOPS_ERR_CUDA, "tc bwd span: cuTensorMapEncodeTiled failed");
  const Spans spn = spans_of(s);
  rc = scan_spans_zero(s, sm, 1, sv.D, sb, spn, st);
  return rc ? rc : span_total(s, spn, sb, local_dh0, nullptr, st, push);
}

int bwd_span_finish(const tops_gla_shape& s, const void* q, const void* k, const void* v, const float* g,
                    const void* dO, const float* dht_in, const void* saved, void* dq, void* dk, void* dv, float* dg,
                    float* dh0, void* workspace, cudaStream_t st) {
  Saved sv;
  carve_saved(s, const_cast<void*>(saved), &sv, true, true);
  bf16* dhs;
  bf16* dob;
  SpanBufs sb;
  carve_bwd_span(s, workspace, &dhs, &sb, &dob);
  if (dob != nullptr) dO = dob;  // converted by the first phase
  ScanMaps sm;
  FusedMaps fm{};
  DqkMaps dm;
  const bool okm = bwd_scan_maps(s, dO, sv, dhs, &sm) && bwd_fused_maps(s, dO, dv, sv, &fm) &&
                   dqk_maps(s, q, k, v, g, dO, sv, dhs, dq, dk, dg, &dm);
  if (!okm) return fail(TOPS_ERR_CUDA, "tc bwd span: cuTensorMapEncodeTiled failed");
  int rc = scan_spans_finish(s, sm, 1, sv.D, dht_in, dh0, dhs, sb, spans_of(s), st, "tc_scan_out_bwd", &fm);
  return rc ? rc : launch_dqk(s, dm, dq, dk, dg, st);
}

// ---------------------------------------------------------------------------
// public entry points: fixed-length problems run directly; packed varlen problems
// (cu_seqlens, B == 1) are padded per segment to multiples of BT, run, and unpadded.
// ---------------------------------------------------------------------------
struct VarlenBufs {
  char* q = nullptr;
  char* k = nullptr;
  char* v = nullptr;
  char* g = nullptr;
  char* x = nullptr;  // o (forward) or do (backward)
  char* dq = nullptr;
  char* dk = nullptr;
  char* dv = nullptr;
  char* dg = nullptr;
  int32_t* blk = nullptr;
};

// padded copies of the token tensors (+ backward outputs) and the block offsets
static size_t carve_varlen(const tops_gla_shape& s, bool bwd, char* base, VarlenBufs* vb) {
  const size_t rows = (size_t)varlen_rows(s), H = (size_t)s.H;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    off = (off + 1023) & ~size_t(1023);
    char* p = base ? base + off : nullptr;
    off += bytes;
    return p;
  };
  VarlenBufs b;
  b.q = take(rows * H * s.K * 2);
  b.k = take(rows * H * s.K * 2);
  b.v = take(rows * H * s.V * 2);
  b.g = take(rows * H * s.K * 4);
  b.x = take(rows * H * s.V * 2);
  if (bwd) {
    b.dq = take(rows * H * s.K * 2);
    b.dk = take(rows * H * s.K * 2);
    b.dv = take(rows * H * s.V * 2);
    b.dg = take(rows * H * s.K * 4);
  }
  b.blk = reinterpret_cast<int32_t*>(take(((size_t)s.N + 1) * 4));
  if (vb) *vb = b;
  return (off + 1023) & ~size_t(1023);
}

size_t fwd_workspace(const tops_gla_shape& s, bool own_saved) {
  if (s.cu_seqlens == nullptr) return own_saved ? 0 : saved_bytes(s);
  return carve_varlen(s, false, nullptr, nullptr) + (own_saved ? 0 : saved_bytes(s));
}

int fwd(const tops_gla_shape& s, const void* q, const void* k, const void* v, const float* g, const float* h0,
        void* o, float* ht, void* saved, void* workspace, cudaStream_t st) {
  if (s.cu_seqlens == nullptr) return fwd_core(s, q, k, v, g, h0, o, ht, saved ? saved : workspace, st, nullptr);
  if (g == nullptr) return fail(TOPS_ERR_UNSUPPORTED, "tc fwd needs gates");
  char* ws = static_cast<char*>(workspace);
  VarlenBufs vb;
  const size_t used = carve_varlen(s, false, ws, &vb);
  void* block = saved ? saved : ws + used;
  const tops_gla_shape ps = padded_shape(s);
  k_blk_off<<<1, 32, 0, st>>>(s.cu_seqlens, s.N, vb.blk);
  TOPS_CUDA_LAUNCH_CHECK("tc varlen blocks");
  const size_t H = (size_t)s.H;
  int rc;
  if ((rc = pad_rows(q, vb.q, H * s.K * 2, ps.T, s, vb.blk, 1, st)) || (rc = pad_rows(k, vb.k, H * s.K * 2, ps.T, s, vb.blk, 1, st)) ||
      (rc = pad_rows(v, vb.v, H * s.V * 2, ps.T, s, vb.blk, 1, st)) || (rc = pad_rows(g, vb.g, H * s.K * 4, ps.T, s, vb.blk, 1, st)))
    return rc;
  if ((rc = fwd_core(ps, vb.q, vb.k, vb.v, reinterpret_cast<const float*>(vb.g), h0, o ? vb.x : nullptr, ht, block, st,
                     vb.blk)))
    return rc;
  if (o) return pad_rows(vb.x, o, H * s.V * 2, s.T, s, vb.blk, 0, st);
  return TOPS_OK;
}

size_t bwd_workspace(const tops_gla_shape& s, bool have_saved) {
  if (s.cu_seqlens == nullptr) return bwd_core_workspace(s, have_saved, true);
  return carve_varlen(s, true, nullptr, nullptr) + bwd_core_workspace(padded_shape(s), have_saved, false);
}

int bwd(const tops_gla_shape& s, const void* q, const void* k, const void* v, const float* g, const float* h0,
        const void* dO, const float* dht, const void* saved, void* dq, void* dk, void* dv, float* dg, float* dh0,
        void* workspace, cudaStream_t st) {
  if (s.cu_seqlens == nullptr)
    return bwd_core(s, q, k, v, g, h0, dO, dht, saved, dq, dk, dv, dg, dh0, workspace, st, nullptr);
  char* ws = static_cast<char*>(workspace);
  VarlenBufs vb;
  const size_t used = carve_varlen(s, true, ws, &vb);
  const tops_gla_shape ps = padded_shape(s);
  k_blk_off<<<1, 32, 0, st>>>(s.cu_seqlens, s.N, vb.blk);
  TOPS_CUDA_LAUNCH_CHECK("tc varlen blocks");
  const size_t H = (size_t)s.H;
  int rc;
  if ((rc = pad_rows(q, vb.q, H * s.K * 2, ps.T, s, vb.blk, 1, st)) || (rc = pad_rows(k, vb.k, H * s.K * 2, ps.T, s, vb.blk, 1, st)) ||
      (rc = pad_rows(v, vb.v, H * s.V * 2, ps.T, s, vb.blk, 1, st)) || (rc = pad_rows(g, vb.g, H * s.K * 4, ps.T, s, vb.blk, 1, st)) ||
      (rc = pad_rows(dO, vb.x, H * s.V * 2, ps.T, s, vb.blk, 1, st)))
    return rc;
  const bool grads = dq != nullptr;
  if ((rc = bwd_core(ps, vb.q, vb.k, vb.v, reinterpret_cast<const float*>(vb.g), h0, vb.x, dht, saved,
                     grads ? vb.dq : nullptr, grads ? vb.dk : nullptr, grads ? vb.dv : nullptr,
                     grads ? reinterpret_cast<float*>(vb.dg) : nullptr, dh0, ws + used, st, vb.blk)))
    return rc;
  if (!grads) return TOPS_OK;
  if ((rc = pad_rows(vb.dq, dq, H * s.K * 2, s.T, s, vb.blk, 0, st)) || (rc = pad_rows(vb.dk, dk, H * s.K * 2, s.T, s, vb.blk, 0, st)) ||
      (rc = pad_rows(vb.dv, dv, H * s.V * 2, s.T, s, vb.blk, 0, st)))
    return rc;
  return pad_rows(vb.dg, dg, H * s.K * 4, s.T, s, vb.blk, 0, st);
}

}  // namespace tc
}  // namespace tops
