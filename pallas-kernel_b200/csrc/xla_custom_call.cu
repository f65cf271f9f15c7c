// XLA custom-call entry points (status-returning legacy API) over the C ABI, so the
// reference's JAX host code (tops.ops.gla with jax.custom_vjp) can call the B200
// kernels: `void f(cudaStream_t, void** buffers, const char* opaque, size_t, XlaCustomCallStatus*)`.
// The opaque bytes are a tops_gla_xla_desc; buffers are the operands followed by
// the results in the order documented per function.  Failures are reported through
// XlaCustomCallStatusSetFailure, resolved at run time from the hosting process
// (jaxlib), so this library has no link-time dependency on XLA.
#include <dlfcn.h>

#include <cstring>

#include "common.cuh"

namespace {

using SetFailureFn = void (*)(void*, const char*, size_t);

void report(void* status, int rc) {
  if (rc == TOPS_OK || status == nullptr) return;
  static SetFailureFn fn = reinterpret_cast<SetFailureFn>(dlsym(RTLD_DEFAULT, "XlaCustomCallStatusSetFailure"));
  if (fn != nullptr) {
    const char* m = tops_gla_last_error();
    fn(status, m, std::strlen(m));
  }
}

bool desc_of(const char* opaque, size_t len, tops_gla_xla_desc* d) {
  if (opaque == nullptr || len != sizeof(tops_gla_xla_desc)) return false;
  std::memcpy(d, opaque, sizeof(*d));
  return true;
}

tops_gla_shape shape_of(const tops_gla_xla_desc& d) {
  tops_gla_shape s{};
  s.B = d.B;
  s.T = d.T;
  s.H = d.H;
  s.K = d.K;
  s.V = d.V;
  s.N = d.B;
  s.chunk_size = d.chunk_size;
  s.NT = d.B * ((d.T + d.chunk_size - 1) / d.chunk_size);
  s.dtype = d.dtype;
  s.scale = d.scale;
  return s;
}

}  // namespace

extern "C" {

// buffers: q, k, v, g, [h0 if has_h0] | o, [ht if out_final], saved, workspace
TOPS_API void tops_gla_xla_chunk_fwd(void* stream, void** buffers, const char* opaque, size_t opaque_len,
                                     void* status) {
  tops_gla_xla_desc d;
  if (!desc_of(opaque, opaque_len, &d)) {
    report(status, tops::fail(TOPS_ERR_INVALID, "xla chunk_fwd: bad descriptor"));
    return;
  }
  int i = 0;
  tops_gla_chunk_fwd_args a{};
  a.s = shape_of(d);
  a.q = buffers[i++];
  a.k = buffers[i++];
  a.v = buffers[i++];
  a.g = static_cast<const float*>(buffers[i++]);
  a.h0 = d.has_h0 ? static_cast<const float*>(buffers[i++]) : nullptr;
  a.o = buffers[i++];
  a.ht = d.out_final ? static_cast<float*>(buffers[i++]) : nullptr;
  a.saved = buffers[i++];
  a.saved_bytes = d.saved_bytes;
  a.workspace = buffers[i++];
  a.workspace_bytes = d.workspace_bytes;
  report(status, tops_gla_chunk_fwd(&a, stream));
}

// buffers: q, k, v, g, [h0], do, [dht if has_dht], saved | dq, dk, dv, dg, [dh0 if want_dh0], workspace
TOPS_API void tops_gla_xla_chunk_bwd(void* stream, void** buffers, const char* opaque, size_t opaque_len,
                                     void* status) {
  tops_gla_xla_desc d;
  if (!desc_of(opaque, opaque_len, &d)) {
    report(status, tops::fail(TOPS_ERR_INVALID, "xla chunk_bwd: bad descriptor"));
    return;
  }
  int i = 0;
  tops_gla_chunk_bwd_args a{};
  a.s = shape_of(d);
  a.q = buffers[i++];
  a.k = buffers[i++];
  a.v = buffers[i++];
  a.g = static_cast<const float*>(buffers[i++]);
  a.h0 = d.has_h0 ? static_cast<const float*>(buffers[i++]) : nullptr;
  a.do_ = buffers[i++];
  a.dht = d.has_dht ? static_cast<const float*>(buffers[i++]) : nullptr;
  a.saved = buffers[i++];
  a.saved_bytes = d.saved_bytes;
  a.dq = buffers[i++];
  a.dk = buffers[i++];
  a.dv = buffers[i++];
  a.dg = static_cast<float*>(buffers[i++]);
  a.dh0 = d.want_dh0 ? static_cast<float*>(buffers[i++]) : nullptr;
  a.workspace = buffers[i++];
  a.workspace_bytes = d.workspace_bytes;
  report(status, tops_gla_chunk_bwd(&a, stream));
}

// buffers: q, k, v, [gk], [h0] | o, [ht], workspace  (has_g -> gk present)
TOPS_API void tops_gla_xla_recurrent_fwd(void* stream, void** buffers, const char* opaque, size_t opaque_len,
                                         void* status) {
  tops_gla_xla_desc d;
  if (!desc_of(opaque, opaque_len, &d)) {
    report(status, tops::fail(TOPS_ERR_INVALID, "xla recurrent_fwd: bad descriptor"));
    return;
  }
  int i = 0;
  tops_gla_recurrent_args a{};
  a.B = d.B;
  a.T = d.T;
  a.H = d.H;
  a.K = d.K;
  a.V = d.V;
  a.N = d.B;
  a.dtype = d.dtype;
  a.scale = d.scale;
  a.reverse = d.reverse;
  a.q = buffers[i++];
  a.k = buffers[i++];
  a.v = buffers[i++];
  a.gk = d.has_g ? static_cast<const float*>(buffers[i++]) : nullptr;
  a.h0 = d.has_h0 ? static_cast<const float*>(buffers[i++]) : nullptr;
  a.o = static_cast<float*>(buffers[i++]);
  a.ht = d.out_final ? static_cast<float*>(buffers[i++]) : nullptr;
  a.workspace = buffers[i++];
  a.workspace_bytes = d.workspace_bytes;
  report(status, tops_gla_recurrent_fwd(&a, stream));
}

}  // extern "C"
