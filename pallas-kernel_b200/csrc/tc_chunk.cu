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
//   k_prep : per (batch, chunk, head).  TMA loads q/k/g tiles, computes the gates in
//            registers, writes qhat/kdec (TMA store) and D, and the intra-chunk matrix
//            A with tcgen05.mma (accumulator in TMEM).
//   k_scan : per (batch, head, 128-wide V tile).  Walks the chunks in order (or in
//            reverse), state [K x 128] fp32 resident in TMEM, operands double
//            buffered by TMA; optionally stores every chunk-start state in bf16.
//   k_out  : persistent, warp specialised GEMM: TMA producer warp, MMA warp, four
//            epilogue warps; 6-stage shared-memory ring, double-buffered TMEM
//            accumulator.  out[128 x 128] = X[128 x K] S[K x 128] + A'[128 x 128] Y[128 x 128].
// All waits are bounded (ptx::mbar_wait).  Shared-memory tiles use the 128-byte
// swizzle that TMA writes and the UMMA descriptors describe.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
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
// k_prep: gates, qhat/kdec, D and the intra-chunk matrix A.  grid (NTb, H, B), 256 threads.
// ===========================================================================
struct PrepParams {
  int B, T, H, K, NTb;
  float scale;
  float* D;  // [B*NTb, H, K]
};

struct PrepMaps {
  CUtensorMap q, k, g, qh, kd, A;
};

__global__ void __launch_bounds__(256, 1) k_prep(const __grid_constant__ PrepMaps maps, PrepParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* qb = smem;                   // [128][64] bf16: q -> qhat (in place)
  unsigned char* kb = qb + TILE_BYTES;        // k -> kdec
  unsigned char* gb = kb + TILE_BYTES;        // 2 x [128][32] fp32
  unsigned char* qt = gb + 2 * TILE_BYTES;    // q e^{G-Gm}
  unsigned char* kt = qt + TILE_BYTES;        // k e^{Gm-G}
  __shared__ float psum[4][64];
  __shared__ __align__(8) uint64_t bar_load, bar_mma;
  __shared__ uint32_t tmem_base;

  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row0 = c * BT;
  const int nkb = p.K / 64;

  if (warp == 0) {
    ptx::tmem_alloc(&tmem_base, 128);
    ptx::tmem_relinquish();
  }
  if (tid == 0) {
    ptx::mbar_init(&bar_load, 1);
    ptx::mbar_init(&bar_mma, 1);
    ptx::fence_mbar_init();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tacc = tmem_base;
  constexpr uint32_t IDESC = ptx::idesc_bf16(128, 128, false, false);

  // gating thread mapping: part (32 rows) x column (64 per K block)
  const int part = warp >> 1, col = (warp & 1) * 32 + lane;
  bool ok = true;
  for (int kbi = 0; kbi < nkb && ok; ++kbi) {
    if (tid == 0) {
      if (kbi > 0) ptx::bulk_wait_read<0>();  // previous qhat/kdec stores have read qb/kb
      ptx::mbar_arrive_expect_tx(&bar_load, 4 * TILE_BYTES);
      ptx::tma_load_4d(qb, &maps.q, kbi * 64, h, row0, b, &bar_load);
      ptx::tma_load_4d(kb, &maps.k, kbi * 64, h, row0, b, &bar_load);
      ptx::tma_load_4d(gb, &maps.g, kbi * 64, h, row0, b, &bar_load);
      ptx::tma_load_4d(gb + TILE_BYTES, &maps.g, kbi * 64 + 32, h, row0, b, &bar_load);
    }
    ok = ptx::mbar_wait(&bar_load, (uint32_t)(kbi & 1));
    if (!ok) break;
    // g(row, col): fp32 tile (col / 32), byte (col % 32) * 4
    const unsigned char* gt = gb + (col >> 5) * TILE_BYTES;
    const uint32_t gbyte = (uint32_t)(col & 31) * 4;
    float s = 0.f;
    for (int r = part * 32; r < part * 32 + 32; ++r) s += *reinterpret_cast<const float*>(gt + ptx::sw128(r, gbyte));
    psum[part][col] = s;
    __syncthreads();
    float off = 0.f;
    for (int pp = 0; pp < part; ++pp) off += psum[pp][col];
    const float GL = psum[0][col] + psum[1][col] + psum[2][col] + psum[3][col];
    const float Gm = psum[0][col] + psum[1][col];
    const float eGm = __expf(Gm), eGLm = __expf(GL - Gm);
    if (part == 0) p.D[((size_t)(b * p.NTb + c) * p.H + h) * p.K + kbi * 64 + col] = __expf(GL);
    float run = off;
    for (int r = part * 32; r < part * 32 + 32; ++r) {
      run += *reinterpret_cast<const float*>(gt + ptx::sw128(r, gbyte));
      const float a = __expf(run - Gm), bb = __expf(Gm - run);
      const float qv = bf(qb, r, col), kv = bf(kb, r, col);
      st_bf(qt, r, col, qv * a);
      st_bf(kt, r, col, kv * bb);
      st_bf(qb, r, col, p.scale * qv * a * eGm);
      st_bf(kb, r, col, kv * bb * eGLm);
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
    ok = ptx::mbar_wait(&bar_mma, (uint32_t)(kbi & 1));
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
  if (tid == 0) ptx::bulk_wait<0>();
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) ptx::tmem_dealloc(tacc, 128);
}

// ===========================================================================
// k_scan: state scan over chunks.  grid (V/128, H, B), 256 threads.
// ===========================================================================
struct ScanParams {
  int B, T, H, K, V, NTb, reverse;
  const float* D;     // [B*NTb, H, K]
  const float* init;  // [B, H, K, V] fp32 or null
  float* fin;         // [B, H, K, V] fp32 or null
  bf16* states;       // [B*NTb, H, K, V] bf16 (chunk-start states) or null
};

struct ScanMaps {
  CUtensorMap x, y;  // x: [B,T,H,K] bf16 box (64,1,128,1); y: [B,T,H,V] bf16 box (64,1,128,1)
  CUtensorMap st;    // chunk states [B*NTb*H, K, V] bf16, box (32,32,1), 64-byte swizzle (store only)
};

// byte offset of (row, byte) in a [rows][64 B] tile with 64-byte swizzle (TMA SWIZZLE_64B, 512 B-aligned base)
__device__ __forceinline__ uint32_t sw64(uint32_t row, uint32_t byte_in_row) {
  return row * 64u + ((((byte_in_row >> 4) ^ ((row >> 1) & 3u)) << 4) | (byte_in_row & 15u));
}

__global__ void __launch_bounds__(256, 1) k_scan(const __grid_constant__ ScanMaps maps, ScanParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nkb = p.K / 64;              // X tiles per chunk
  const int nh = p.K / 128;              // state halves (TMEM lane blocks)
  const uint32_t buf_bytes = (uint32_t)(nkb + 2) * TILE_BYTES;
  unsigned char* stage_st = smem + 2 * buf_bytes;  // 8 warps x 2 slots x 2 KB
  __shared__ __align__(8) uint64_t bar_full[2], bar_mma;
  __shared__ uint32_t tmem_base;

  const int vt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int v0 = vt * BV;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = warp & 3, hf = warp >> 2;  // lane quadrant, state half handled by this warp
  const int krow = hf * 128 + qd * 32 + lane;
  const bool active = hf < nh;

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

  auto chunk_of = [&](int i) { return p.reverse ? p.NTb - 1 - i : i; };
  auto issue = [&](int i) {
    const int c = chunk_of(i);
    unsigned char* buf = smem + (i & 1) * buf_bytes;
    ptx::mbar_arrive_expect_tx(&bar_full[i & 1], buf_bytes);
    for (int j = 0; j < nkb; ++j) ptx::tma_load_4d(buf + j * TILE_BYTES, &maps.x, j * 64, h, c * BT, b, &bar_full[i & 1]);
    ptx::tma_load_4d(buf + nkb * TILE_BYTES, &maps.y, v0, h, c * BT, b, &bar_full[i & 1]);
    ptx::tma_load_4d(buf + (nkb + 1) * TILE_BYTES, &maps.y, v0 + 64, h, c * BT, b, &bar_full[i & 1]);
  };
  if (tid == 0) {
    issue(0);
    if (p.NTb > 1) issue(1);
  }
  // initial state -> TMEM buffer 0
  if (active) {
    const size_t srow = ((size_t)(b * p.H + h) * p.K + krow) * p.V + v0;
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) {
      float r[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) r[j] = p.init ? p.init[srow + cb * 32 + j] : 0.f;
      ptx::tmem_st32(tmem_lane_addr(sbuf(0), qd * 32, hf * 128 + cb * 32), r);
    }
    ptx::tmem_st_wait();
  }
  bool ok = true;
  // the decay of chunk i+1 is fetched one iteration ahead (its latency hides behind chunk i)
  auto decay_of = [&](int i) {
    return active && i < p.NTb ? __ldg(p.D + ((size_t)(b * p.NTb + chunk_of(i)) * p.H + h) * p.K + krow) : 1.f;
  };
  float d_next = decay_of(0);
  for (int i = 0; i < p.NTb; ++i) {
    const int c = chunk_of(i);
    const float d = d_next;
    d_next = decay_of(i + 1);
    if (i > 0) {
      ok = ptx::mbar_wait(&bar_mma, (uint32_t)((i - 1) & 1));
      ptx::tc_fence_after();
      if (!ok) break;
      if (tid == 0 && i + 1 < p.NTb) issue(i + 1);  // buffer (i+1)&1 was read by chunk i-1, now complete
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
  if (ok) ok = ptx::mbar_wait(&bar_mma, (uint32_t)((p.NTb - 1) & 1));
  ptx::tc_fence_after();
  if (ok && active && p.fin) {
    const size_t srow = ((size_t)(b * p.H + h) * p.K + krow) * p.V + v0;
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) {
      float r[32];
      ptx::tmem_ld32(tmem_lane_addr(sbuf(p.NTb), qd * 32, hf * 128 + cb * 32), r);
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
  const int nvt = p.V / BV;
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
// k_dqk: dq, dk, dg of one (batch, chunk, head, 128-wide K tile).  grid (K/128, NTb, B*H), 256 threads.
//   dA      = scale tril(do v^T)                            (M1, contraction over V)
//   dqi     = do h_c^T            dki = v dh_c^T            (M2, M3, contraction over V)
//   dq      = e^{G-Gm} (dA ktil + scale e^{Gm} dqi)         (M4 = dA x ktil,  ktil = k e^{Gm-G})
//   dk      = e^{Gm-G} (dA^T qtil + e^{GL-Gm} dki)          (M5 = dA^T x qtil, qtil = q e^{G-Gm})
//   dg      = revcumsum_t(q dq - k dk) + e^{GL} sum_v(h_c dh_c) + sum_t(e^{GL-G} dki k)
//             with q dq = qtil (M4 + scale e^{Gm} dqi) and k dk = ktil (M5 + e^{GL-Gm} dki)
// (reference chunk_gla_bwd_fused_kernel tops/ops/gla/chunk.py:1423-1479 and the
//  _ref functions :504-743).
// Roles during the V stream: warp 0 = TMA producer, warp 1 = MMA issuer, warps 2-3 =
// chunk-local cumsum of g (in place), warps 4-7 = sum_v h*dh.  The 2-stage operand
// ring is released by the MMA commit plus the four reducer warps.  After the stream
// the ring holds q -> qtil, k -> ktil (stage 0) and the bf16 dA (stage 1).
// ===========================================================================
struct DqkParams {
  int B, T, H, K, V, NTb;
  float scale;
  bf16* dq; bf16* dk; float* dg;
};

struct DqkMaps {
  CUtensorMap dO, v;   // [B,T,H,V] box (64,1,128,1)
  CUtensorMap hs, dhs; // [B*NTb*H, K, V] box (64,128,1)
  CUtensorMap g;       // [B,T,H,K] fp32 box (32,1,128,1)
  CUtensorMap q, k;    // [B,T,H,K] bf16 box (64,1,128,1)
  CUtensorMap dq, dk;  // [B,T,H,K] bf16 box (64,1,128,1), stores
};

__device__ __forceinline__ float gval(const unsigned char* Gs, int row, int col) {
  return *reinterpret_cast<const float*>(Gs + (col >> 5) * TILE_BYTES + ptx::sw128(row, (col & 31) * 4));
}

__global__ void __launch_bounds__(256, 1) k_dqk(const __grid_constant__ DqkMaps maps, DqkParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr uint32_t STG = 4 * TILE_BYTES;  // do, v, h, dh tiles of one V block
  unsigned char* ring = smem;               // 2 stages
  unsigned char* Gs = smem + 2 * STG;       // 4 x [128][32] fp32: G, then dg_raw
  unsigned char* qtl = ring;                // after the stream: qtil (2 tiles), ktil (2 tiles)
  unsigned char* ktl = ring + 2 * TILE_BYTES;
  unsigned char* dAs = ring + STG;          // dA bf16 (2 tiles), later the dk staging tiles
  unsigned char* dqs = ring + STG + 2 * TILE_BYTES;  // dq staging tiles (free after the V stream)
  __shared__ float GLs[128], Gms[128], eGm[128], eGLm[128], hdh2[2][128], colsum[4][128], dgtot[128];
  __shared__ __align__(8) uint64_t full[2], empty[2], bar_g, bar_qk, bar_mma;
  __shared__ uint32_t tmem_base;

  const int kt = blockIdx.x, c = blockIdx.y, b = blockIdx.z / p.H, h = blockIdx.z % p.H;
  const int k0 = kt * 128, row0 = c * BT;
  const int srow = (b * p.NTb + c) * p.H + h;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nvb = p.V / 64;

  if (warp == 0) {
    ptx::tmem_alloc(&tmem_base, 512);
    ptx::tmem_relinquish();
  }
  if (tid == 32) {
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1 + 4);  // MMA commit + 4 reducer warps
    }
    ptx::mbar_init(&bar_g, 1);
    ptx::mbar_init(&bar_qk, 1);
    ptx::mbar_init(&bar_mma, 1);
    ptx::fence_mbar_init();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tM1 = tmem_base, tM2 = tmem_base + 128, tM3 = tmem_base + 256, tM5 = tmem_base + 384;
  bool ok = true;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      ptx::mbar_arrive_expect_tx(&bar_g, 4 * TILE_BYTES);
      for (int j = 0; j < 4; ++j) ptx::tma_load_4d(Gs + j * TILE_BYTES, &maps.g, k0 + 32 * j, h, row0, b, &bar_g);
      for (int vb = 0; vb < nvb && ok; ++vb) {
        const int s = vb & 1;
        if (vb >= 2) ok = ptx::mbar_wait(&empty[s], (uint32_t)(((vb >> 1) - 1) & 1));
        if (!ok) break;
        unsigned char* st = ring + s * STG;
        ptx::mbar_arrive_expect_tx(&full[s], STG);
        ptx::tma_load_4d(st, &maps.dO, vb * 64, h, row0, b, &full[s]);
        ptx::tma_load_4d(st + TILE_BYTES, &maps.v, vb * 64, h, row0, b, &full[s]);
        ptx::tma_load_3d(st + 2 * TILE_BYTES, &maps.hs, vb * 64, k0, srow, &full[s]);
        ptx::tma_load_3d(st + 3 * TILE_BYTES, &maps.dhs, vb * 64, k0, srow, &full[s]);
      }
      // stage 0 gets q and k once its last V block is released
      if (ok) {
        const int last0 = (nvb - 1) & ~1;  // last V block that used stage 0
        ok = ptx::mbar_wait(&empty[0], (uint32_t)((last0 >> 1) & 1));
      }
      if (ok) {
        ptx::mbar_arrive_expect_tx(&bar_qk, 4 * TILE_BYTES);
        ptx::tma_load_4d(qtl, &maps.q, k0, h, row0, b, &bar_qk);
        ptx::tma_load_4d(qtl + TILE_BYTES, &maps.q, k0 + 64, h, row0, b, &bar_qk);
        ptx::tma_load_4d(ktl, &maps.k, k0, h, row0, b, &bar_qk);
        ptx::tma_load_4d(ktl + TILE_BYTES, &maps.k, k0 + 64, h, row0, b, &bar_qk);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer for the V stream ----------------
    if (lane == 0) {
      constexpr uint32_t ID_KK = ptx::idesc_bf16(128, 128, false, false);
      for (int vb = 0; vb < nvb && ok; ++vb) {
        const int s = vb & 1;
        ok = ptx::mbar_wait(&full[s], (uint32_t)((vb >> 1) & 1));
        if (!ok) break;
        ptx::tc_fence_after();
        const unsigned char* st = ring + s * STG;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint32_t acc = (vb | ks) ? 1u : 0u;
          ptx::mma_bf16_ss(tM1, desc_kmajor(st, ks * 32), desc_kmajor(st + TILE_BYTES, ks * 32), ID_KK, acc);
          ptx::mma_bf16_ss(tM2, desc_kmajor(st, ks * 32), desc_kmajor(st + 2 * TILE_BYTES, ks * 32), ID_KK, acc);
          ptx::mma_bf16_ss(tM3, desc_kmajor(st + TILE_BYTES, ks * 32), desc_kmajor(st + 3 * TILE_BYTES, ks * 32),
                           ID_KK, acc);
        }
        ptx::mma_commit(&empty[s]);
      }
      if (ok) ptx::mma_commit(&bar_mma);
    }
  } else if (warp < 4) {
    // ---------------- chunk-local cumsum of g, in place (2 columns per thread) ----------------
    ok = ptx::mbar_wait(&bar_g, 0);
    if (ok) {
      const int c0 = (tid - 64) * 2;
      float r0 = 0.f, r1 = 0.f;
      for (int r = 0; r < 128; ++r) {
        float* e0 = reinterpret_cast<float*>(Gs + (c0 >> 5) * TILE_BYTES + ptx::sw128(r, (c0 & 31) * 4));
        const float2 x = *reinterpret_cast<float2*>(e0);
        r0 += x.x;
        r1 += x.y;
        *reinterpret_cast<float2*>(e0) = make_float2(r0, r1);
        if (r == 63) {
          Gms[c0] = r0;
          Gms[c0 + 1] = r1;
        }
      }
      GLs[c0] = r0;
      GLs[c0 + 1] = r1;
      eGm[c0] = __expf(Gms[c0]);
      eGm[c0 + 1] = __expf(Gms[c0 + 1]);
      eGLm[c0] = __expf(r0 - Gms[c0]);
      eGLm[c0 + 1] = __expf(r1 - Gms[c0 + 1]);
    }
  } else {
    // ---------------- sum_v h*dh of the state rows, per V block ----------------
    const int hr = (tid - 128);  // state row 0..127
    float acc = 0.f;
    for (int vb = 0; vb < nvb && ok; ++vb) {
      const int s = vb & 1;
      ok = ptx::mbar_wait(&full[s], (uint32_t)((vb >> 1) & 1));
      if (!ok) break;
      const unsigned char* th = ring + s * STG + 2 * TILE_BYTES;
      const unsigned char* tdh = th + TILE_BYTES;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint4 a = *reinterpret_cast<const uint4*>(th + ptx::sw128(hr, u * 16));
        const uint4 d = *reinterpret_cast<const uint4*>(tdh + ptx::sw128(hr, u * 16));
        const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
        const __nv_bfloat162* d2 = reinterpret_cast<const __nv_bfloat162*>(&d);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 af = __bfloat1622float2(a2[e]), df = __bfloat1622float2(d2[e]);
          acc = fmaf(af.x, df.x, fmaf(af.y, df.y, acc));
        }
      }
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&empty[s]);
    }
    hdh2[0][hr] = acc;
  }
  // ---------------- all threads: V-stream MMAs done, G done ----------------
  __syncthreads();
  if (ok) ok = ptx::mbar_wait(&bar_mma, 0);
  ptx::tc_fence_after();
  const int qd = warp & 3, ch = warp >> 2;
  const int i = qd * 32 + lane;  // TMEM lane = token row of this thread
  if (ok) {
    // dA = scale tril(M1) -> bf16 [i][j] (2 tiles in stage 1)
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
    // qtil = q e^{G-Gm}, ktil = k e^{Gm-G}, in place, 8 columns (16 B) per step
    ok = ptx::mbar_wait(&bar_qk, 0);
    if (ok) {
      for (int it = tid; it < 2 * 2 * 128 * 8; it += 256) {
        const int chunk = it & 7, row = (it >> 3) & 127, tile = it >> 10;  // tile: q0 q1 k0 k1
        const bool isk = tile >= 2;
        const int col0 = (tile & 1) * 64 + chunk * 8;
        unsigned char* t = ring + tile * TILE_BYTES;
        uint4* pv = reinterpret_cast<uint4*>(t + ptx::sw128(row, chunk * 16));
        uint4 x = *pv;
        __nv_bfloat162* x2 = reinterpret_cast<__nv_bfloat162*>(&x);
        const float4 ga = *reinterpret_cast<const float4*>(Gs + (col0 >> 5) * TILE_BYTES + ptx::sw128(row, (col0 & 31) * 4));
        const float4 gb = *reinterpret_cast<const float4*>(Gs + (col0 >> 5) * TILE_BYTES +
                                                            ptx::sw128(row, ((col0 + 4) & 31) * 4));
        const float G8[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float2 f = __bfloat1622float2(x2[e]);
          const float d0 = G8[2 * e] - Gms[col0 + 2 * e], d1 = G8[2 * e + 1] - Gms[col0 + 2 * e + 1];
          f.x *= __expf(isk ? -d0 : d0);
          f.y *= __expf(isk ? -d1 : d1);
          x2[e] = __floats2bfloat162_rn(f.x, f.y);
        }
        *pv = x;
      }
    }
  }
  ptx::fence_async_smem();
  ptx::tc_fence_before();
  __syncthreads();
  if (tid == 32 && ok) {
    ptx::tc_fence_after();
    const uint32_t ID_KM = ptx::idesc_bf16(128, 128, false, true);
    const uint32_t ID_MM = ptx::idesc_bf16(128, 128, true, true);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      // M4 (into M1's columns): dA[i][j] x ktil[j][k]
      ptx::mma_bf16_ss(tM1, desc_kmajor(dAs + (ks >> 2) * TILE_BYTES, (ks & 3) * 32),
                       desc_mnmajor(ktl, ks * 2048, TILE_BYTES), ID_KM, ks ? 1u : 0u);
      // M5: dA^T[j][i] x qtil[i][k]
      ptx::mma_bf16_ss(tM5, desc_mnmajor(dAs, ks * 2048, TILE_BYTES), desc_mnmajor(qtl, ks * 2048, TILE_BYTES),
                       ID_MM, ks ? 1u : 0u);
    }
    ptx::mma_commit(&bar_mma);
  }
  if (ok) ok = ptx::mbar_wait(&bar_mma, 1);
  ptx::tc_fence_after();
  // ---------------- epilogue: dq, dk, dg_raw (in place of G), column sums ----------------
  const int row = row0 + i;
  const bool in = row < p.T;
  if (ok) {
    for (int g16 = 0; g16 < 4; ++g16) {
      const int cb = ch * 64 + g16 * 16;  // first column of this group
      float m4[16], m5[16], m2[16], m3[16];
      ptx::tmem_ld16(tmem_lane_addr(tM1, qd * 32, cb), m4);
      ptx::tmem_ld16(tmem_lane_addr(tM5, qd * 32, cb), m5);
      ptx::tmem_ld16(tmem_lane_addr(tM2, qd * 32, cb), m2);
      ptx::tmem_ld16(tmem_lane_addr(tM3, qd * 32, cb), m3);
      // qtil / ktil of this row, 16 columns: tile cb/64, bytes (cb%64)*2 .. +31
      const unsigned char* qt_ = qtl + (cb >> 6) * TILE_BYTES;
      const unsigned char* kt_ = ktl + (cb >> 6) * TILE_BYTES;
      uint4 qa = *reinterpret_cast<const uint4*>(qt_ + ptx::sw128(i, (cb & 63) * 2));
      uint4 qb2 = *reinterpret_cast<const uint4*>(qt_ + ptx::sw128(i, (cb & 63) * 2 + 16));
      uint4 ka = *reinterpret_cast<const uint4*>(kt_ + ptx::sw128(i, (cb & 63) * 2));
      uint4 kb2 = *reinterpret_cast<const uint4*>(kt_ + ptx::sw128(i, (cb & 63) * 2 + 16));
      ptx::tmem_ld_wait();
      float qv[16], kv[16];
      {
        const __nv_bfloat162* a = reinterpret_cast<const __nv_bfloat162*>(&qa);
        const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&qb2);
        const __nv_bfloat162* d = reinterpret_cast<const __nv_bfloat162*>(&ka);
        const __nv_bfloat162* d2 = reinterpret_cast<const __nv_bfloat162*>(&kb2);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float2 t0 = __bfloat1622float2(a[e]), t1 = __bfloat1622float2(a2[e]);
          float2 u0 = __bfloat1622float2(d[e]), u1 = __bfloat1622float2(d2[e]);
          qv[2 * e] = t0.x; qv[2 * e + 1] = t0.y; qv[8 + 2 * e] = t1.x; qv[8 + 2 * e + 1] = t1.y;
          kv[2 * e] = u0.x; kv[2 * e + 1] = u0.y; kv[8 + 2 * e] = u1.x; kv[8 + 2 * e + 1] = u1.y;
        }
      }
      uint32_t dqw[8], dkw[8];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int col = cb + e;
        float* gp = reinterpret_cast<float*>(Gs + (col >> 5) * TILE_BYTES + ptx::sw128(i, (col & 31) * 4));
        const float x = *gp - Gms[col];
        const float eglm = eGLm[col];
        const float pq = m4[e] + p.scale * eGm[col] * m2[e];          // dq = e^{x} pq
        const float pk = m5[e] + eglm * m3[e];                           // dk = e^{-x} pk
        *gp = in ? qv[e] * pq - kv[e] * pk : 0.f;                       // dg_raw = q dq - k dk
        float cs = in ? kv[e] * eglm * m3[e] : 0.f;                     // (e^{GL-G} dki) k
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) cs += __shfl_xor_sync(0xffffffffu, cs, o);
        if (lane == 0) colsum[qd][col] = cs;
        m4[e] = __expf(x) * pq;
        m5[e] = __expf(-x) * pk;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        dqw[u] = ptx::pack_bf16(m4[2 * u], m4[2 * u + 1]);
        dkw[u] = ptx::pack_bf16(m5[2 * u], m5[2 * u + 1]);
      }
      // stage [128 rows][128 cols] bf16 as two 128B-swizzled [128][64] tiles each
      unsigned char* tq = dqs + (cb >> 6) * TILE_BYTES;
      unsigned char* tk = dAs + (cb >> 6) * TILE_BYTES;
      const uint32_t by = (uint32_t)(cb & 63) * 2;
      *reinterpret_cast<uint4*>(tq + ptx::sw128(i, by)) = make_uint4(dqw[0], dqw[1], dqw[2], dqw[3]);
      *reinterpret_cast<uint4*>(tq + ptx::sw128(i, by + 16)) = make_uint4(dqw[4], dqw[5], dqw[6], dqw[7]);
      *reinterpret_cast<uint4*>(tk + ptx::sw128(i, by)) = make_uint4(dkw[0], dkw[1], dkw[2], dkw[3]);
      *reinterpret_cast<uint4*>(tk + ptx::sw128(i, by + 16)) = make_uint4(dkw[4], dkw[5], dkw[6], dkw[7]);
    }
  }
  ptx::fence_async_smem();
  ptx::tc_fence_before();
  __syncthreads();
  if (tid == 0 && ok) {  // dq, dk tiles -> global (rows past T are clipped by the tensor map)
    ptx::tma_store_4d(&maps.dq, k0, h, row0, b, dqs);
    ptx::tma_store_4d(&maps.dq, k0 + 64, h, row0, b, dqs + TILE_BYTES);
    ptx::tma_store_4d(&maps.dk, k0, h, row0, b, dAs);
    ptx::tma_store_4d(&maps.dk, k0 + 64, h, row0, b, dAs + TILE_BYTES);
    ptx::bulk_commit();
  }
  // ---------------- dg = reverse cumsum over rows + inter term: 2 threads per column ----------------
  const int col = tid & 127, half = tid >> 7;
  const unsigned char* gt = Gs + (col >> 5) * TILE_BYTES;
  const uint32_t by = (uint32_t)(col & 31) * 4;
  if (ok && half == 1) {
    float tsum = 0.f;
    for (int r = 64; r < 128; ++r) tsum += *reinterpret_cast<const float*>(gt + ptx::sw128(r, by));
    dgtot[col] = tsum;
  }
  __syncthreads();
  if (ok) {
    const float inter = __expf(GLs[col]) * hdh2[0][col] + colsum[0][col] + colsum[1][col] + colsum[2][col] +
                        colsum[3][col];
    float run = half ? 0.f : dgtot[col];
    for (int r = half * 64 + 63; r >= half * 64; --r) {
      run += *reinterpret_cast<const float*>(gt + ptx::sw128(r, by));
      if (row0 + r < p.T) p.dg[((size_t)(b * p.T + row0 + r) * p.H + h) * p.K + k0 + col] = run + inter;
    }
  }
  if (!ok && tid == 0) {  // drain loads that may still be in flight (bounded)
    ptx::mbar_wait(&full[0], 0);
    ptx::mbar_wait(&full[1], 0);
    ptx::mbar_wait(&bar_qk, 0);
  }
  if (tid == 0) ptx::bulk_wait<0>();
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) ptx::tmem_dealloc(tmem_base, 512);
}

TOPS_DEVICE_ERROR_READER(read_device_error)

// ---------------------------------------------------------------------------
// host orchestration
// ---------------------------------------------------------------------------
static int sm_count() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

bool eligible(const tops_gla_shape& s) {
  return s.dtype == TOPS_BF16 && s.cu_seqlens == nullptr && (s.K == 128 || s.K == 256) && s.V % BV == 0 &&
         s.T > 0 && s.B > 0 && s.H > 0 && tops_gla_has_tcgen05() && encode_fn() != nullptr;
}

// Intermediates of the forward that the backward reuses (one contiguous block).
struct Saved {
  bf16 *qh, *kd, *A, *h;
  float* D;
};

static size_t carve_saved(const tops_gla_shape& s, void* base, Saved* sv) {
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
  if (sv) *sv = v;
  return off;
}

size_t saved_bytes(const tops_gla_shape& s) { return carve_saved(s, nullptr, nullptr); }

static size_t prep_smem() { return 6 * TILE_BYTES + 1024; }
static size_t scan_smem(int K) { return 2 * (size_t)(K / 64 + 2) * TILE_BYTES + 8 * 2 * 2048 + 1024; }
static size_t out_smem() { return (size_t)OUT_STAGES * STAGE_BYTES + 2 * TILE_BYTES + 1024; }

template <typename KernelT>
static cudaError_t set_smem(KernelT k, size_t bytes) {
  return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

// Forward: o, ht and (in `saved`) qhat, kdec, A, D, chunk-start states h.
int fwd(const tops_gla_shape& s, const void* q, const void* k, const void* v, const float* g, const float* h0,
        void* o, float* ht, void* saved, cudaStream_t st) {
  if (g == nullptr) return fail(TOPS_ERR_UNSUPPORTED, "tc fwd needs gates");
  Saved sv;
  carve_saved(s, saved, &sv);
  const int NTb = (s.T + BT - 1) / BT;
  const CUtensorMapDataType BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, F32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  PrepMaps pm;
  bool okm = map_tok(&pm.q, q, BF, 2, s.B, s.T, s.H, s.K, 64, BT) && map_tok(&pm.k, k, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
             map_tok(&pm.g, g, F32, 4, s.B, s.T, s.H, s.K, 32, BT) &&
             map_tok(&pm.qh, sv.qh, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
             map_tok(&pm.kd, sv.kd, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
             map_tok(&pm.A, sv.A, BF, 2, s.B, s.T, s.H, BT, 64, BT);
  ScanMaps sm;
  okm = okm && map_tok(&sm.x, sv.kd, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
        map_tok(&sm.y, v, BF, 2, s.B, s.T, s.H, s.V, 64, BT) && map_state_store(&sm.st, sv.h, s.B * NTb * s.H, s.K, s.V);
  OutMaps om;
  okm = okm && map_tok(&om.x, sv.qh, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
        map_state(&om.s, sv.h, s.B * NTb * s.H, s.K, s.V, 64) &&
        map_tok(&om.a, sv.A, BF, 2, s.B, s.T, s.H, BT, 64, BT) && map_tok(&om.y, v, BF, 2, s.B, s.T, s.H, s.V, 64, 64) &&
        map_tok(&om.o, o, BF, 2, s.B, s.T, s.H, s.V, 64, BT);
  if (!okm) return fail(TOPS_ERR_CUDA, "tc fwd: cuTensorMapEncodeTiled failed (alignment?)");
  cudaError_t e;
  {
    LaunchTimer lt(st, "tc_prep");
    PrepParams pp{s.B, s.T, s.H, s.K, NTb, s.scale, sv.D};
    if ((e = set_smem(k_prep, prep_smem())) != cudaSuccess) return cuda_status(e, "tc prep attr");
    k_prep<<<dim3(NTb, s.H, s.B), 256, prep_smem(), st>>>(pm, pp);
    TOPS_CUDA_LAUNCH_CHECK("tc_prep");
  }
  {
    LaunchTimer lt(st, "tc_scan");
    ScanParams sp{s.B, s.T, s.H, s.K, s.V, NTb, 0, sv.D, h0, ht, sv.h};
    if ((e = set_smem(k_scan, scan_smem(s.K))) != cudaSuccess) return cuda_status(e, "tc scan attr");
    k_scan<<<dim3(s.V / BV, s.H, s.B), 256, scan_smem(s.K), st>>>(sm, sp);
    TOPS_CUDA_LAUNCH_CHECK("tc_scan");
  }
  {
    LaunchTimer lt(st, "tc_out");
    OutParams op{s.B, s.T, s.H, s.K, s.V, NTb, 0, static_cast<bf16*>(o)};
    if ((e = set_smem(k_out, out_smem())) != cudaSuccess) return cuda_status(e, "tc out attr");
    const int items = s.B * NTb * s.H * (s.V / BV);
    const int grid = items < sm_count() ? items : sm_count();
    k_out<<<grid, 192, out_smem(), st>>>(om, op);
    TOPS_CUDA_LAUNCH_CHECK("tc_out");
  }
  return TOPS_OK;
}

static size_t dqk_smem() { return 2 * 4 * (size_t)TILE_BYTES + 4 * (size_t)TILE_BYTES + 1024; }

size_t bwd_workspace(const tops_gla_shape& s, bool have_saved) {
  const int NTb = (s.T + BT - 1) / BT;
  size_t n = ((size_t)s.B * NTb * s.H * s.K * s.V * 2 + 1023) & ~size_t(1023);  // dh states
  if (!have_saved) n += saved_bytes(s);
  return n;
}

// Backward: dq, dk, dv (bf16), dg (fp32), dh0 (fp32, optional) from the forward's saved block.
int bwd(const tops_gla_shape& s, const void* q, const void* k, const void* v, const float* g, const float* h0,
        const void* dO, const float* dht, const void* saved_in, void* dq, void* dk, void* dv, float* dg, float* dh0,
        void* workspace, cudaStream_t st) {
  const int NTb = (s.T + BT - 1) / BT;
  char* ws = static_cast<char*>(workspace);
  bf16* dhs = reinterpret_cast<bf16*>(ws);
  const size_t dh_bytes = ((size_t)s.B * NTb * s.H * s.K * s.V * 2 + 1023) & ~size_t(1023);
  void* saved = const_cast<void*>(saved_in);
  int rc;
  if (saved == nullptr) {  // recompute the forward intermediates (o is discarded into dv's buffer)
    saved = ws + dh_bytes;
    if ((rc = fwd(s, q, k, v, g, h0, dv, nullptr, saved, st))) return rc;
  }
  Saved sv;
  carve_saved(s, saved, &sv);
  const CUtensorMapDataType BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, F32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  ScanMaps sm;
  bool okm = map_tok(&sm.x, sv.qh, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
             map_tok(&sm.y, dO, BF, 2, s.B, s.T, s.H, s.V, 64, BT) &&
             map_state_store(&sm.st, dhs, s.B * NTb * s.H, s.K, s.V);
  OutMaps om;
  okm = okm && map_tok(&om.x, sv.kd, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
        map_state(&om.s, dhs, s.B * NTb * s.H, s.K, s.V, 64) && map_tok(&om.a, sv.A, BF, 2, s.B, s.T, s.H, BT, 64, 64) &&
        map_tok(&om.y, dO, BF, 2, s.B, s.T, s.H, s.V, 64, 64) && map_tok(&om.o, dv, BF, 2, s.B, s.T, s.H, s.V, 64, BT);
  DqkMaps dm;
  okm = okm && map_tok(&dm.dO, dO, BF, 2, s.B, s.T, s.H, s.V, 64, BT) &&
        map_tok(&dm.v, v, BF, 2, s.B, s.T, s.H, s.V, 64, BT) &&
        map_state(&dm.hs, sv.h, s.B * NTb * s.H, s.K, s.V, 128) &&
        map_state(&dm.dhs, dhs, s.B * NTb * s.H, s.K, s.V, 128) &&
        map_tok(&dm.g, g, F32, 4, s.B, s.T, s.H, s.K, 32, BT) && map_tok(&dm.q, q, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
        map_tok(&dm.k, k, BF, 2, s.B, s.T, s.H, s.K, 64, BT) && map_tok(&dm.dq, dq, BF, 2, s.B, s.T, s.H, s.K, 64, BT) &&
        map_tok(&dm.dk, dk, BF, 2, s.B, s.T, s.H, s.K, 64, BT);
  if (!okm) return fail(TOPS_ERR_CUDA, "tc bwd: cuTensorMapEncodeTiled failed (alignment?)");
  cudaError_t e;
  {
    LaunchTimer lt(st, "tc_scan_bwd");
    ScanParams sp{s.B, s.T, s.H, s.K, s.V, NTb, 1, sv.D, dht, dh0, dhs};
    if ((e = set_smem(k_scan, scan_smem(s.K))) != cudaSuccess) return cuda_status(e, "tc scan attr");
    k_scan<<<dim3(s.V / BV, s.H, s.B), 256, scan_smem(s.K), st>>>(sm, sp);
    TOPS_CUDA_LAUNCH_CHECK("tc_scan_bwd");
  }
  {
    LaunchTimer lt(st, "tc_out_dv");
    OutParams op{s.B, s.T, s.H, s.K, s.V, NTb, 1, static_cast<bf16*>(dv)};
    if ((e = set_smem(k_out, out_smem())) != cudaSuccess) return cuda_status(e, "tc out attr");
    const int items = s.B * NTb * s.H * (s.V / BV);
    const int grid = items < sm_count() ? items : sm_count();
    k_out<<<grid, 192, out_smem(), st>>>(om, op);
    TOPS_CUDA_LAUNCH_CHECK("tc_out_dv");
  }
  {
    LaunchTimer lt(st, "tc_dqk");
    DqkParams dp{s.B, s.T, s.H, s.K, s.V, NTb, s.scale, static_cast<bf16*>(dq), static_cast<bf16*>(dk), dg};
    if ((e = set_smem(k_dqk, dqk_smem())) != cudaSuccess) return cuda_status(e, "tc dqk attr");
    k_dqk<<<dim3(s.K / 128, NTb, s.B * s.H), 256, dqk_smem(), st>>>(dm, dp);
    TOPS_CUDA_LAUNCH_CHECK("tc_dqk");
  }
  return TOPS_OK;
}

}  // namespace tc
}  // namespace tops
