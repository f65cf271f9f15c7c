// C ABI of libtops_gla.so: argument validation, workspace carving and the
// orchestration of the chunked forward/backward (tops/ops/gla/chunk.py:1083-1179,
// 815-977).  Every entry point returns a status; messages go to a thread-local
// string read by tops_gla_last_error().
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "p2p.cuh"

namespace tops {

static thread_local std::string g_last_error;
static std::atomic<unsigned long long> g_launches{0};

void note_launch(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }

// ---- per-launch timing --------------------------------------------------
struct TimedLaunch {
  const char* name;
  cudaEvent_t a, b;
};
static std::mutex g_timing_mu;
static bool g_timing = false;
static std::vector<TimedLaunch> g_timed;

LaunchTimer::LaunchTimer(cudaStream_t s, const char* n) : st(s), name(n) {
  if (!g_timing) return;
  if (cudaEventCreate(&a) != cudaSuccess || cudaEventCreate(&b) != cudaSuccess) {
    a = b = nullptr;
    return;
  }
  cudaEventRecord(a, st);
}

LaunchTimer::~LaunchTimer() {
  if (a == nullptr) return;
  cudaEventRecord(b, st);
  std::lock_guard<std::mutex> lk(g_timing_mu);
  g_timed.push_back({name, a, b});
}

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int status, const std::string& msg) {
  set_error(msg);
  return status;
}

int cuda_status(cudaError_t e, const char* what) {
  return fail(TOPS_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int check_shape(const tops_gla_shape* s) {
  TOPS_CHECK_ARG(s != nullptr, "shape is NULL");
  TOPS_CHECK_ARG(s->B >= 0 && s->T >= 0 && s->H >= 0 && s->K > 0 && s->V > 0, "negative or zero dimension");
  TOPS_CHECK_ARG(s->chunk_size > 0 && (s->chunk_size & (s->chunk_size - 1)) == 0,
                 "chunk_size must be a power of 2");
  TOPS_CHECK_ARG(s->dtype == TOPS_F32 || s->dtype == TOPS_BF16 || s->dtype == TOPS_F16, "unknown dtype");
  if (s->cu_seqlens != nullptr) {
    TOPS_CHECK_ARG(s->B == 1, "cu_seqlens requires B == 1");
    TOPS_CHECK_ARG(s->chunk_offsets != nullptr, "cu_seqlens requires chunk_offsets");
    TOPS_CHECK_ARG(s->N >= 1, "cu_seqlens requires N >= 1");
  } else {
    TOPS_CHECK_ARG(s->N == s->B, "N must equal B without cu_seqlens");
    TOPS_CHECK_ARG(s->NT == s->B * ((s->T + s->chunk_size - 1) / s->chunk_size), "NT != B*ceil(T/C)");
  }
  return TOPS_OK;
}

// bump allocator over the caller's workspace (dry run when base == nullptr)
struct Carve {
  char* base;
  size_t used = 0;
  explicit Carve(void* b) : base(static_cast<char*>(b)) {}
  template <typename T>
  T* take(size_t count) {
    used = (used + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + used) : nullptr;
    used += count * sizeof(T);
    return p;
  }
};

namespace simt {
int cumsum(const tops_gla_shape& s, const float* g, float* out, int reverse, float scale, cudaStream_t st);
int fwd_h(const tops_gla_shape& s, const void* k, const void* v, const float* gc, const float* h0, float* h,
          float* ht, cudaStream_t st);
int bwd_dh(const tops_gla_shape& s, const void* q, const float* gc, const void* dO, const float* dht, float* dh,
           float* dh0, cudaStream_t st);
int fwd_intra(const tops_gla_shape& s, const void* q, const void* k, const float* gc, int causal, float* A,
              cudaStream_t st);
int fwd_o(const tops_gla_shape& s, const void* q, const void* v, const float* gc, const float* A, const float* h,
          void* o, cudaStream_t st);
int bwd_dA(const tops_gla_shape& s, const void* v, const void* dO, float* dA, cudaStream_t st);
int bwd_dv(const tops_gla_shape& s, const void* k, const float* gc, const float* A, const void* dO, const float* dh,
           void* dv, int out_dtype, cudaStream_t st);
int bwd_dqk_intra(const tops_gla_shape& s, const void* q, const void* k, const float* gc, const float* dA,
                  float* dq, float* dk, cudaStream_t st);
int bwd_dqkg(const tops_gla_shape& s, const void* q, const void* k, const void* v, const float* h, const float* gc,
             const void* dO, const float* dh, const float* dq_in, const float* dk_in, void* dq_out, void* dk_out,
             int out_dtype, float* dg, cudaStream_t st);
}  // namespace simt

namespace rec {
size_t fwd_workspace(const tops_gla_recurrent_args& a);
int fwd(const tops_gla_recurrent_args& a, cudaStream_t st);
size_t bwd_workspace(const tops_gla_recurrent_bwd_args& a);
int bwd(const tops_gla_recurrent_bwd_args& a, cudaStream_t st);
}  // namespace rec

namespace decode {
int read_device_error();
}  // namespace decode

namespace exchange {
int read_device_error();
}  // namespace exchange

namespace tc {
bool eligible(const tops_gla_shape& s);
size_t saved_bytes(const tops_gla_shape& s);
size_t fwd_workspace(const tops_gla_shape& s, bool own_saved);
int fwd(const tops_gla_shape& s, const void* q, const void* k, const void* v, const float* g, const float* h0,
        void* o, float* ht, void* saved, void* workspace, cudaStream_t st);
int read_device_error();
int selftest_wait_timeout(cudaStream_t st);
size_t span_saved_bytes(const tops_gla_shape& s);
size_t bwd_span_workspace(const tops_gla_shape& s);
int fwd_span_begin(const tops_gla_shape& s, const void* q, const void* k, const void* v, const float* g, void* saved,
                   float* local_state, float* decay, cudaStream_t st, const p2p::PeerPush* push = nullptr);
int fwd_span_finish(const tops_gla_shape& s, const void* q, const void* k, const void* v, const float* g,
                    const float* h_in, void* o, float* ht, void* saved, cudaStream_t st);
int bwd_span_begin(const tops_gla_shape& s, const void* dO, const void* saved, void* workspace, float* local_dh0,
                   cudaStream_t st, const p2p::PeerPush* push = nullptr);
int bwd_span_finish(const tops_gla_shape& s, const void* q, const void* k, const void* v, const float* g,
                    const void* dO, const float* dht_in, const void* saved, void* dq, void* dk, void* dv, float* dg,
                    float* dh0, void* workspace, cudaStream_t st);
size_t bwd_workspace(const tops_gla_shape& s, bool have_saved);
int bwd(const tops_gla_shape& s, const void* q, const void* k, const void* v, const float* g, const float* h0,
        const void* dO, const float* dht, const void* saved, void* dq, void* dk, void* dv, float* dg, float* dh0,
        void* workspace, cudaStream_t st);
}  // namespace tc

namespace seqpar {
int span_decay(const tops_gla_shape& s, const float* g, float* decay, cudaStream_t st);
int state_combine(int N, int H, int K, int V, const float* decay, const float* h_in, const float* s_local,
                  float* out, cudaStream_t st);
}  // namespace seqpar

static inline cudaStream_t S(void* p) { return static_cast<cudaStream_t>(p); }
static inline size_t tok_elems(const tops_gla_shape& s, int D) { return (size_t)s.B * s.T * s.H * D; }
static inline size_t state_elems(const tops_gla_shape& s, int n) { return (size_t)n * s.H * s.K * s.V; }

// the per-chunk kernels of the fp32 path tile a chunk into one 64-row block
static int check_simt_chunk(const tops_gla_shape& s) {
  if (s.chunk_size > 64) return fail(TOPS_ERR_UNSUPPORTED, "chunk_size > 64 is not supported by this path");
  return TOPS_OK;
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
// the tensor-core path serves bf16 / fp16 problems that ask for no CUDA-core-format intermediates
static bool use_tc_fwd(const tops_gla_chunk_fwd_args* a) {
  return a->g_cumsum == nullptr && a->A == nullptr && a->h == nullptr && tc::eligible(a->s);
}

// Without gates (g == NULL) the tensor-core kernels read an all-zero gate tensor, as the
// reference substitutes zeros (tops/ops/gla/chunk.py:1114-1118); it sits at the end of the
// caller's workspace and is cleared in-stream before use.
static size_t zero_gate_bytes(const tops_gla_shape& s, const float* g) {
  return g != nullptr ? 0 : (((size_t)s.B * s.T * s.H * s.K * sizeof(float) + 1023) & ~size_t(1023));
}

static int zero_gates(const tops_gla_shape& s, void* workspace, size_t offset, const float** g, cudaStream_t st) {
  if (*g != nullptr) return TOPS_OK;
  float* z = reinterpret_cast<float*>(static_cast<char*>(workspace) + offset);
  cudaError_t e = cudaMemsetAsync(z, 0, (size_t)s.B * s.T * s.H * s.K * sizeof(float), st);
  if (e != cudaSuccess) return cuda_status(e, "chunk: clearing the zero gates");
  note_launch(1);
  *g = z;
  return TOPS_OK;
}

static int chunk_fwd_impl(const tops_gla_chunk_fwd_args* a, void* stream, size_t* ws_need) {
  int rc = check_shape(a ? &a->s : nullptr);
  if (rc) return rc;
  const tops_gla_shape& s = a->s;
  const bool dry = ws_need != nullptr;
  if (use_tc_fwd(a)) {
    const size_t need_saved = tc::saved_bytes(s);
    const bool own = a->saved != nullptr;
    if (own && a->saved_bytes < need_saved)
      return fail(TOPS_ERR_WORKSPACE, "chunk_fwd: saved block smaller than tops_gla_chunk_saved_size()");
    const size_t base = tc::fwd_workspace(s, own);  // the kernels' own scratch comes first
    const size_t zb = zero_gate_bytes(s, a->g), zoff = (base + 1023) & ~size_t(1023);
    const size_t need = zb ? zoff + zb : base;
    if (dry) {
      *ws_need = need;
      return TOPS_OK;
    }
    TOPS_CHECK_ARG(a->q && a->k && a->v && (a->o || a->ht), "chunk_fwd: q, k, v and o (or ht) are required");
    if (need > 0 && (a->workspace == nullptr || a->workspace_bytes < need))
      return fail(TOPS_ERR_WORKSPACE, "chunk_fwd: workspace smaller than tops_gla_chunk_fwd_workspace_size()");
    const float* g = a->g;
    if ((rc = zero_gates(s, a->workspace, zoff, &g, S(stream)))) return rc;
    return tc::fwd(s, a->q, a->k, a->v, g, a->h0, a->o, a->ht, own ? a->saved : nullptr, a->workspace, S(stream));
  }
  if ((rc = check_simt_chunk(s))) return rc;
  if (!dry) {
    TOPS_CHECK_ARG(a->q && a->k && a->v && (a->o || a->ht), "chunk_fwd: q, k, v and o (or ht) are required");
  }
  Carve cv(dry ? nullptr : a->workspace);
  float* gc = a->g_cumsum ? a->g_cumsum : cv.take<float>(tok_elems(s, s.K));
  float* h = a->h ? a->h : cv.take<float>(state_elems(s, s.NT));
  float* A = a->A ? a->A : cv.take<float>(tok_elems(s, s.chunk_size));
  if (dry) {
    *ws_need = cv.used;
    return TOPS_OK;
  }
  if (cv.used > a->workspace_bytes || (cv.used > 0 && a->workspace == nullptr))
    return fail(TOPS_ERR_WORKSPACE, "chunk_fwd: workspace smaller than tops_gla_chunk_fwd_workspace_size()");
  cudaStream_t st = S(stream);
  if (a->g != nullptr) {
    if ((rc = simt::cumsum(s, a->g, gc, 0, 1.f, st))) return rc;
  } else {
    cudaError_t e = cudaMemsetAsync(gc, 0, tok_elems(s, s.K) * sizeof(float), st);
    if (e != cudaSuccess) return cuda_status(e, "chunk_fwd: memset g_cumsum");
    note_launch(1);
  }
  if ((rc = simt::fwd_h(s, a->k, a->v, gc, a->h0, h, a->ht, st))) return rc;
  if (a->o == nullptr) return TOPS_OK;  // final state only
  if ((rc = simt::fwd_intra(s, a->q, a->k, gc, 1, A, st))) return rc;
  return simt::fwd_o(s, a->q, a->v, gc, A, h, a->o, st);
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------
static bool use_tc_bwd(const tops_gla_chunk_bwd_args* a) {
  return a->g_cumsum == nullptr && a->A == nullptr && a->h == nullptr && tc::eligible(a->s);
}

static int chunk_bwd_impl(const tops_gla_chunk_bwd_args* a, void* stream, size_t* ws_need) {
  int rc = check_shape(a ? &a->s : nullptr);
  if (rc) return rc;
  const tops_gla_shape& s = a->s;
  const bool dry = ws_need != nullptr;
  // dh0 only (no gradient outputs): the reverse state scan alone
  const bool dh0_only = !a->dq && !a->dk && !a->dv && !a->dg;
  if (use_tc_bwd(a)) {
    const bool have = a->saved != nullptr;
    if (have && a->saved_bytes < tc::saved_bytes(s))
      return fail(TOPS_ERR_WORKSPACE, "chunk_bwd: saved block smaller than tops_gla_chunk_saved_size()");
    const size_t base = tc::bwd_workspace(s, have);
    const size_t zb = zero_gate_bytes(s, a->g), zoff = (base + 1023) & ~size_t(1023);
    const size_t need = zb ? zoff + zb : base;
    if (dry) {
      *ws_need = need;
      return TOPS_OK;
    }
    TOPS_CHECK_ARG(a->q && a->k && a->v && a->do_ && ((a->dq && a->dk && a->dv && a->dg) || (dh0_only && a->dh0)),
                   "chunk_bwd: q, k, v, do and dq, dk, dv, dg (or dh0 alone) are required");
    if (a->workspace == nullptr || a->workspace_bytes < need)
      return fail(TOPS_ERR_WORKSPACE, "chunk_bwd: workspace smaller than tops_gla_chunk_bwd_workspace_size()");
    const float* g = a->g;
    if ((rc = zero_gates(s, a->workspace, zoff, &g, S(stream)))) return rc;
    return tc::bwd(s, a->q, a->k, a->v, g, a->h0, a->do_, a->dht, a->saved, a->dq, a->dk, a->dv, a->dg, a->dh0,
                   a->workspace, S(stream));
  }
  if ((rc = check_simt_chunk(s))) return rc;
  if (!dry) {
    TOPS_CHECK_ARG(a->q && a->k && a->v && a->do_ && ((a->dq && a->dk && a->dv && a->dg) || (dh0_only && a->dh0)),
                   "chunk_bwd: q, k, v, do and dq, dk, dv, dg (or dh0 alone) are required");
  }
  Carve cv(dry ? nullptr : a->workspace);
  const bool need_gc = a->g_cumsum == nullptr;
  const bool need_h = a->h == nullptr;
  const bool need_A = a->A == nullptr;
  float* gc = need_gc ? cv.take<float>(tok_elems(s, s.K)) : nullptr;
  float* h = need_h ? cv.take<float>(state_elems(s, s.NT)) : nullptr;
  float* A = need_A ? cv.take<float>(tok_elems(s, s.chunk_size)) : nullptr;
  float* dh = cv.take<float>(state_elems(s, s.NT));
  float* dA = cv.take<float>(tok_elems(s, s.chunk_size));
  float* dqi = cv.take<float>(tok_elems(s, s.K));
  float* dki = cv.take<float>(tok_elems(s, s.K));
  if (dry) {
    *ws_need = cv.used;
    return TOPS_OK;
  }
  if (cv.used > a->workspace_bytes || a->workspace == nullptr)
    return fail(TOPS_ERR_WORKSPACE, "chunk_bwd: workspace smaller than tops_gla_chunk_bwd_workspace_size()");
  cudaStream_t st = S(stream);
  const float* gcc = a->g_cumsum;
  if (need_gc) {
    if (a->g != nullptr) {
      if ((rc = simt::cumsum(s, a->g, gc, 0, 1.f, st))) return rc;
    } else {
      cudaError_t e = cudaMemsetAsync(gc, 0, tok_elems(s, s.K) * sizeof(float), st);
      if (e != cudaSuccess) return cuda_status(e, "chunk_bwd: memset g_cumsum");
      note_launch(1);
    }
    gcc = gc;
  }
  const float* hh = a->h;
  if (need_h) {
    if ((rc = simt::fwd_h(s, a->k, a->v, gcc, a->h0, h, nullptr, st))) return rc;
    hh = h;
  }
  if ((rc = simt::bwd_dh(s, a->q, gcc, a->do_, a->dht, dh, a->dh0, st))) return rc;
  if (dh0_only) return TOPS_OK;
  const float* AA = a->A;
  if (need_A) {
    if ((rc = simt::fwd_intra(s, a->q, a->k, gcc, 1, A, st))) return rc;
    AA = A;
  }
  if ((rc = simt::bwd_dv(s, a->k, gcc, AA, a->do_, dh, a->dv, s.dtype, st))) return rc;
  if ((rc = simt::bwd_dA(s, a->v, a->do_, dA, st))) return rc;
  if ((rc = simt::bwd_dqk_intra(s, a->q, a->k, gcc, dA, dqi, dki, st))) return rc;
  return simt::bwd_dqkg(s, a->q, a->k, a->v, hh, gcc, a->do_, dh, dqi, dki, a->dq, a->dk, s.dtype, a->dg, st);
}

// the two-phase span entry points serve fixed-length problems on the tensor-core path
static int check_span(const tops_gla_shape* s, const void* saved, size_t saved_bytes, const float* g) {
  int rc = check_shape(s);
  if (rc) return rc;
  TOPS_CHECK_ARG(s->cu_seqlens == nullptr, "span entry points: variable-length input is not supported");
  TOPS_CHECK_ARG(g != nullptr, "span entry points: g is required");
  if (!tc::eligible(*s))
    return fail(TOPS_ERR_UNSUPPORTED, "span entry points: the problem does not run on the tensor-core path");
  TOPS_CHECK_ARG(saved != nullptr, "span entry points: the saved block is required");
  if (saved_bytes < tc::span_saved_bytes(*s))
    return fail(TOPS_ERR_WORKSPACE, "span entry points: saved block smaller than tops_gla_chunk_span_saved_size()");
  return TOPS_OK;
}

static int check_rec(const tops_gla_recurrent_args* a) {
  TOPS_CHECK_ARG(a != nullptr, "args is NULL");
  TOPS_CHECK_ARG(a->B >= 0 && a->T >= 0 && a->H >= 0 && a->K > 0 && a->V > 0, "bad dimension");
  TOPS_CHECK_ARG(a->dtype == TOPS_F32 || a->dtype == TOPS_BF16 || a->dtype == TOPS_F16, "unknown dtype");
  if (a->cu_seqlens != nullptr) {
    TOPS_CHECK_ARG(a->B == 1, "cu_seqlens requires B == 1");
  } else {
    TOPS_CHECK_ARG(a->N == a->B, "N must equal B without cu_seqlens");
  }
  return TOPS_OK;
}

}  // namespace tops

using namespace tops;

extern "C" {

const char* tops_gla_last_error(void) { return g_last_error.c_str(); }
uint64_t tops_gla_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int32_t tops_gla_device_error(void) {
  const int32_t e = decode::read_device_error();
  const int32_t e2 = tc::read_device_error();
  const int32_t e3 = exchange::read_device_error();  // every word is read (and cleared)
  return e != 0 ? e : e2 != 0 ? e2 : e3;
}

int tops_gla_selftest_wait_timeout(void* stream) {
  return tc::selftest_wait_timeout(static_cast<cudaStream_t>(stream));
}

size_t tops_gla_chunk_saved_size(const tops_gla_shape* s) {
  if (check_shape(s) != TOPS_OK || !tc::eligible(*s)) return 0;
  return tc::saved_bytes(*s);
}

void tops_gla_timing_enable(int32_t on) {
  std::lock_guard<std::mutex> lk(g_timing_mu);
  g_timing = on != 0;
}

int32_t tops_gla_timing_collect(char* names, int32_t name_stride, float* ms, int32_t max_entries) {
  std::lock_guard<std::mutex> lk(g_timing_mu);
  int32_t n = 0;
  for (auto& t : g_timed) {
    if (n < max_entries) {
      float e = -1.f;
      if (cudaEventSynchronize(t.b) == cudaSuccess) cudaEventElapsedTime(&e, t.a, t.b);
      if (ms != nullptr) ms[n] = e;
      if (names != nullptr && name_stride > 0) {
        std::strncpy(names + (size_t)n * name_stride, t.name, (size_t)name_stride - 1);
        names[(size_t)n * name_stride + name_stride - 1] = 0;
      }
    }
    cudaEventDestroy(t.a);
    cudaEventDestroy(t.b);
    ++n;
  }
  g_timed.clear();
  return n;
}
int32_t tops_gla_abi_version(void) { return TOPS_GLA_ABI_VERSION; }

int32_t tops_gla_has_tcgen05(void) {
  static std::atomic<int> cache[64] = {};  // per device: 0 unknown, 1 no, 2 yes
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (dev >= 0 && dev < 64) {
    const int c = cache[dev].load(std::memory_order_relaxed);
    if (c != 0) return c == 2 ? 1 : 0;
  }
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) return 0;
  const int32_t yes = (major == 10 && minor == 0) ? 1 : 0;
  if (dev >= 0 && dev < 64) cache[dev].store(yes ? 2 : 1, std::memory_order_relaxed);
  return yes;
}

int32_t tops_gla_num_chunks(int32_t B, int32_t T, int32_t C, const int32_t* cu, int32_t N, int32_t* offs) {
  if (C <= 0 || B < 0 || T < 0) return -1;
  if (cu == nullptr) {
    const int32_t nts = (T + C - 1) / C;
    if (offs != nullptr)
      for (int32_t n = 0; n <= B; ++n) offs[n] = n * nts;
    return B * nts;
  }
  if (N < 1 || cu[0] != 0) return -1;
  int32_t acc = 0;
  for (int32_t n = 0; n < N; ++n) {
    if (offs != nullptr) offs[n] = acc;
    const int32_t L = cu[n + 1] - cu[n];
    if (L < 0) return -1;
    acc += (L + C - 1) / C;
  }
  if (offs != nullptr) offs[N] = acc;
  return acc;
}

int tops_gla_chunk_fwd(const tops_gla_chunk_fwd_args* a, void* stream) { return chunk_fwd_impl(a, stream, nullptr); }

size_t tops_gla_chunk_fwd_workspace_size(const tops_gla_chunk_fwd_args* a) {
  size_t need = 0;
  if (chunk_fwd_impl(a, nullptr, &need) != TOPS_OK) return 0;
  return need;
}

int tops_gla_chunk_bwd(const tops_gla_chunk_bwd_args* a, void* stream) { return chunk_bwd_impl(a, stream, nullptr); }

size_t tops_gla_chunk_bwd_workspace_size(const tops_gla_chunk_bwd_args* a) {
  size_t need = 0;
  if (chunk_bwd_impl(a, nullptr, &need) != TOPS_OK) return 0;
  return need;
}

size_t tops_gla_chunk_span_saved_size(const tops_gla_shape* s) {
  if (check_shape(s) != TOPS_OK || s->cu_seqlens != nullptr || !tc::eligible(*s)) return 0;
  return tc::span_saved_bytes(*s);
}

int tops_gla_chunk_fwd_span_begin(const tops_gla_chunk_fwd_args* a, float* local_state, float* decay, void* stream) {
  TOPS_CHECK_ARG(a != nullptr, "chunk_fwd_span_begin: args is NULL");
  int rc = check_span(&a->s, a->saved, a->saved_bytes, a->g);
  if (rc) return rc;
  TOPS_CHECK_ARG(a->q && a->k && a->v && local_state && decay,
                 "chunk_fwd_span_begin: q, k, v, local_state and decay are required");
  return tc::fwd_span_begin(a->s, a->q, a->k, a->v, a->g, a->saved, local_state, decay, S(stream));
}

// the peer-memory arguments of a fused span begin: a group this shape's state fits
static int check_push(const tops_gla_shape& s, const tops_gla_p2p_args* x) {
  TOPS_CHECK_ARG(x != nullptr, "span_begin_p2p: p2p args are required");
  TOPS_CHECK_ARG(x->world > 0 && x->world <= p2p::MAX_WORLD && x->rank >= 0 && x->rank < x->world,
                 "span_begin_p2p: bad rank / world (at most 64 ranks)");
  TOPS_CHECK_ARG(x->regions && x->own_region, "span_begin_p2p: regions (device array) and own_region are required");
  TOPS_CHECK_ARG(x->N == s.B && x->H == s.H && x->K == s.K && x->V == s.V,
                 "span_begin_p2p: the p2p shape (N, H, K, V) must be the problem's (B, H, K, V)");
  return TOPS_OK;
}

int tops_gla_chunk_fwd_span_begin_p2p(const tops_gla_chunk_fwd_args* a, float* decay, const tops_gla_p2p_args* x,
                                      void* stream) {
  TOPS_CHECK_ARG(a != nullptr, "chunk_fwd_span_begin_p2p: args is NULL");
  int rc = check_span(&a->s, a->saved, a->saved_bytes, a->g);
  if (rc || (rc = check_push(a->s, x))) return rc;
  TOPS_CHECK_ARG(a->q && a->k && a->v && decay, "chunk_fwd_span_begin_p2p: q, k, v and decay are required");
  const p2p::PeerPush push{x->regions, x->own_region, x->rank, x->world, nullptr};
  return tc::fwd_span_begin(a->s, a->q, a->k, a->v, a->g, a->saved, nullptr, decay, S(stream), &push);
}

int tops_gla_chunk_fwd_span_finish(const tops_gla_chunk_fwd_args* a, void* stream) {
  TOPS_CHECK_ARG(a != nullptr, "chunk_fwd_span_finish: args is NULL");
  int rc = check_span(&a->s, a->saved, a->saved_bytes, a->g);
  if (rc) return rc;
  TOPS_CHECK_ARG(a->q && a->k && a->v && a->o, "chunk_fwd_span_finish: q, k, v and o are required");
  return tc::fwd_span_finish(a->s, a->q, a->k, a->v, a->g, a->h0, a->o, a->ht, a->saved, S(stream));
}

size_t tops_gla_chunk_bwd_span_workspace_size(const tops_gla_chunk_bwd_args* a) {
  if (a == nullptr || check_shape(&a->s) != TOPS_OK || a->s.cu_seqlens != nullptr || !tc::eligible(a->s)) return 0;
  return tc::bwd_span_workspace(a->s);
}

static int check_bwd_span_ws(const tops_gla_chunk_bwd_args* a) {
  if (a->workspace == nullptr || a->workspace_bytes < tc::bwd_span_workspace(a->s))
    return fail(TOPS_ERR_WORKSPACE, "span entry points: workspace smaller than tops_gla_chunk_bwd_span_workspace_size()");
  return TOPS_OK;
}

int tops_gla_chunk_bwd_span_begin(const tops_gla_chunk_bwd_args* a, float* local_dh0, void* stream) {
  TOPS_CHECK_ARG(a != nullptr, "chunk_bwd_span_begin: args is NULL");
  int rc = check_span(&a->s, a->saved, a->saved_bytes, a->g);
  if (rc || (rc = check_bwd_span_ws(a))) return rc;
  TOPS_CHECK_ARG(a->do_ && local_dh0, "chunk_bwd_span_begin: do and local_dh0 are required");
  return tc::bwd_span_begin(a->s, a->do_, a->saved, a->workspace, local_dh0, S(stream));
}

int tops_gla_chunk_bwd_span_begin_p2p(const tops_gla_chunk_bwd_args* a, const float* decay, const tops_gla_p2p_args* x,
                                      void* stream) {
  TOPS_CHECK_ARG(a != nullptr, "chunk_bwd_span_begin_p2p: args is NULL");
  int rc = check_span(&a->s, a->saved, a->saved_bytes, a->g);
  if (rc || (rc = check_bwd_span_ws(a)) || (rc = check_push(a->s, x))) return rc;
  TOPS_CHECK_ARG(a->do_ && decay, "chunk_bwd_span_begin_p2p: do and decay are required");
  const p2p::PeerPush push{x->regions, x->own_region, x->rank, x->world, decay};
  return tc::bwd_span_begin(a->s, a->do_, a->saved, a->workspace, nullptr, S(stream), &push);
}

int tops_gla_chunk_bwd_span_finish(const tops_gla_chunk_bwd_args* a, void* stream) {
  TOPS_CHECK_ARG(a != nullptr, "chunk_bwd_span_finish: args is NULL");
  int rc = check_span(&a->s, a->saved, a->saved_bytes, a->g);
  if (rc || (rc = check_bwd_span_ws(a))) return rc;
  TOPS_CHECK_ARG(a->q && a->k && a->v && a->do_ && a->dq && a->dk && a->dv && a->dg,
                 "chunk_bwd_span_finish: q, k, v, do and dq, dk, dv, dg are required");
  return tc::bwd_span_finish(a->s, a->q, a->k, a->v, a->g, a->do_, a->dht, a->saved, a->dq, a->dk, a->dv, a->dg,
                             a->dh0, a->workspace, S(stream));
}

int tops_gla_recurrent_fwd(const tops_gla_recurrent_args* a, void* stream) {
  int rc = check_rec(a);
  if (rc) return rc;
  TOPS_CHECK_ARG(a->q && a->k && a->v && a->o, "fused_recurrent: q, k, v and o are required");
  return rec::fwd(*a, S(stream));
}

size_t tops_gla_recurrent_fwd_workspace_size(const tops_gla_recurrent_args* a) {
  if (check_rec(a) != TOPS_OK) return 0;
  return rec::fwd_workspace(*a);
}

int tops_gla_recurrent_bwd(const tops_gla_recurrent_bwd_args* a, void* stream) {
  int rc = check_rec(a ? &a->f : nullptr);
  if (rc) return rc;
  TOPS_CHECK_ARG(a->f.q && a->f.k && a->f.v && a->do_ && a->dq && a->dk && a->dv,
                 "fused_recurrent_bwd: q, k, v, do, dq, dk, dv are required");
  TOPS_CHECK_ARG(a->dgk == nullptr || a->f.gk != nullptr, "fused_recurrent_bwd: dgk needs gk");
  TOPS_CHECK_ARG(a->dgv == nullptr || a->f.gv != nullptr, "fused_recurrent_bwd: dgv needs gv");
  return rec::bwd(*a, S(stream));
}

size_t tops_gla_recurrent_bwd_workspace_size(const tops_gla_recurrent_bwd_args* a) {
  if (a == nullptr || check_rec(&a->f) != TOPS_OK) return 0;
  return rec::bwd_workspace(*a);
}

int tops_gla_chunk_local_cumsum(const tops_gla_shape* s, const float* g, float* out, int32_t reverse, float scale,
                                void* stream) {
  int rc = check_shape(s);
  if (rc) return rc;
  TOPS_CHECK_ARG(g && out, "chunk_local_cumsum: g and out are required");
  return simt::cumsum(*s, g, out, reverse, scale, S(stream));
}

int tops_gla_chunk_fwd_h(const tops_gla_shape* s, const void* k, const void* v, const float* gc, const float* h0,
                         float* h, float* ht, void* stream) {
  int rc = check_shape(s);
  if (rc) return rc;
  TOPS_CHECK_ARG(k && v && gc, "chunk_fwd_h: k, v and g_cumsum are required");
  return simt::fwd_h(*s, k, v, gc, h0, h, ht, S(stream));
}

int tops_gla_chunk_bwd_dh(const tops_gla_shape* s, const void* q, const float* gc, const void* dO, const float* dht,
                          float* dh, float* dh0, void* stream) {
  int rc = check_shape(s);
  if (rc) return rc;
  TOPS_CHECK_ARG(q && gc && dO, "chunk_bwd_dh: q, g_cumsum and do are required");
  return simt::bwd_dh(*s, q, gc, dO, dht, dh, dh0, S(stream));
}

int tops_gla_chunk_fwd_intra(const tops_gla_shape* s, const void* q, const void* k, const float* gc, int32_t causal,
                             float* A, void* stream) {
  int rc = check_shape(s);
  if (rc || (rc = check_simt_chunk(*s))) return rc;
  TOPS_CHECK_ARG(q && k && gc && A, "chunk_fwd_intra: q, k, g_cumsum and A are required");
  return simt::fwd_intra(*s, q, k, gc, causal, A, S(stream));
}

int tops_gla_chunk_fwd_o(const tops_gla_shape* s, const void* q, const void* v, const float* gc, const float* A,
                         const float* h, void* o, void* stream) {
  int rc = check_shape(s);
  if (rc || (rc = check_simt_chunk(*s))) return rc;
  TOPS_CHECK_ARG(q && v && gc && A && h && o, "chunk_fwd_o: all tensors are required");
  return simt::fwd_o(*s, q, v, gc, A, h, o, S(stream));
}

int tops_gla_chunk_bwd_dA(const tops_gla_shape* s, const void* v, const void* dO, float* dA, void* stream) {
  int rc = check_shape(s);
  if (rc || (rc = check_simt_chunk(*s))) return rc;
  TOPS_CHECK_ARG(v && dO && dA, "chunk_bwd_dA: v, do and dA are required");
  return simt::bwd_dA(*s, v, dO, dA, S(stream));
}

int tops_gla_chunk_bwd_dv(const tops_gla_shape* s, const void* k, const float* gc, const float* A, const void* dO,
                          const float* dh, float* dv, void* stream) {
  int rc = check_shape(s);
  if (rc || (rc = check_simt_chunk(*s))) return rc;
  TOPS_CHECK_ARG(k && gc && A && dO && dh && dv, "chunk_bwd_dv: all tensors are required");
  return simt::bwd_dv(*s, k, gc, A, dO, dh, dv, TOPS_F32, S(stream));
}

int tops_gla_chunk_bwd_dqk_intra(const tops_gla_shape* s, const void* q, const void* k, const float* gc,
                                 const float* dA, float* dq, float* dk, void* stream) {
  int rc = check_shape(s);
  if (rc || (rc = check_simt_chunk(*s))) return rc;
  TOPS_CHECK_ARG(q && k && gc && dA && dq && dk, "chunk_bwd_dqk_intra: all tensors are required");
  return simt::bwd_dqk_intra(*s, q, k, gc, dA, dq, dk, S(stream));
}

int tops_gla_chunk_bwd_dqkg(const tops_gla_shape* s, const void* q, const void* k, const void* v, const float* h,
                            const float* gc, const void* dO, const float* dh, const float* dq_in, const float* dk_in,
                            void* dq_out, void* dk_out, int32_t out_dtype, float* dg, void* stream) {
  int rc = check_shape(s);
  if (rc || (rc = check_simt_chunk(*s))) return rc;
  TOPS_CHECK_ARG(q && k && v && h && gc && dO && dh && dq_in && dk_in && dq_out && dk_out && dg,
                 "chunk_bwd_dqkg: all tensors are required");
  TOPS_CHECK_ARG(out_dtype == TOPS_F32 || out_dtype == TOPS_BF16 || out_dtype == TOPS_F16, "unknown out_dtype");
  return simt::bwd_dqkg(*s, q, k, v, h, gc, dO, dh, dq_in, dk_in, dq_out, dk_out, out_dtype, dg, S(stream));
}

int tops_gla_span_decay(const tops_gla_shape* s, const float* g, float* decay, void* stream) {
  int rc = check_shape(s);
  if (rc) return rc;
  TOPS_CHECK_ARG(g && decay, "span_decay: g and decay are required");
  return seqpar::span_decay(*s, g, decay, S(stream));
}

int tops_gla_state_combine(int32_t N, int32_t H, int32_t K, int32_t V, const float* decay, const float* h_in,
                           const float* s_local, float* out, void* stream) {
  TOPS_CHECK_ARG(N >= 0 && H >= 0 && K > 0 && V > 0, "state_combine: bad dimension");
  TOPS_CHECK_ARG(decay && h_in && s_local && out, "state_combine: all tensors are required");
  return seqpar::state_combine(N, H, K, V, decay, h_in, s_local, out, S(stream));
}

}  // extern "C"
